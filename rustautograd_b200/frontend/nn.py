"""The compositions of rg's primitive ops that the GPT workload and its sampler use: softmax and
log-softmax over the last axis, cross-entropy, the tanh GELU, and the top-k / nucleus logit
filters. Each is written as the same sequence of primitive ops as rg's python/rg/nn.py
(softmax nn.py:40-42, log-softmax and logsumexp nn.py:29-37, cross-entropy nn.py:78-84, GELU
nn.py:25-27, filters nn.py:60-72), so the device receives the plan rg would build; the row
statistics go through `stop_gradient`, as in rg, so autodiff emits rg's backward chains.
"""
import math

from .tracing import argsort, cumsum, exp, stop_gradient, take_along_axis, tanh, top_k, where

_GELU_C = math.sqrt(2.0 / math.pi)


def gelu(x):
    return 0.5 * x * (1.0 + tanh(_GELU_C * (x + 0.044715 * x * x * x)))


def _row_max(x, axis):
    return stop_gradient(x.max(axis=axis, keepdims=True))


def softmax(x, axis=-1):
    e = exp(x - _row_max(x, axis))
    return e / e.sum(axis=axis, keepdims=True)


def logsumexp(x, axis=-1, keepdims=False):
    m = _row_max(x, axis)
    out = exp(x - m).sum(axis=axis, keepdims=True).log() + m
    return out if keepdims else out.squeeze(axis)


def log_softmax(x, axis=-1):
    return x - logsumexp(x, axis=axis, keepdims=True)


def cross_entropy(logits, labels, axis=-1):
    """Mean negative log-likelihood of int32 class labels."""
    picked = take_along_axis(log_softmax(logits, axis), labels.reshape(tuple(labels.shape) + (1,)))
    return -picked.mean()


def top_k_logits(logits, k):
    """Logits outside the k largest of the last axis drop to -1e9."""
    values, _ = top_k(logits, k)
    return where(logits >= values[..., -1:], logits, -1e9)


def top_p_logits(logits, p):
    """Nucleus filter: a token stays while the probability mass ranked above it is below p."""
    order = argsort(logits, descending=True)
    probs = softmax(take_along_axis(logits, order))
    kept = (cumsum(probs) - probs) < p
    return where(take_along_axis(kept, argsort(order.cast(logits.dtype))), logits, -1e9)
