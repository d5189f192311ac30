"""Model building blocks traced onto rg's primitive ops (the compositions of python/rg/nn.py).

Each function emits the same primitive ops in the same order as rg's version, so the CUDA
device sees the plan rg would build: softmax and layer norm as reductions plus elementwise
chains, cross-entropy as log-softmax then take-along then mean, attention with a materialised
masked score matrix.
"""
import math

from . import random
from .core import (argmax, argsort, concatenate, cumsum, equal, exp, eye, maximum, stop_gradient, swapaxes, take, take_along_axis, tanh,
                   top_k, where, zeros, ones)


def sigmoid(x): return 1.0 / (1.0 + exp(-x))
def softplus(x): return maximum(x, 0.0) + (1.0 + exp(-abs(x))).log()
def silu(x): return x * sigmoid(x)


def gelu(x):
    """Tanh approximation of the Gaussian error linear unit (nn.py:25-27)."""
    return 0.5 * x * (1.0 + tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x * x * x)))


def relu(x): return maximum(x, 0.0)


def logsumexp(x, axis=-1, keepdims=False):
    top = stop_gradient(x.max(axis=axis, keepdims=True))
    out = exp(x - top).sum(axis=axis, keepdims=True).log() + top
    return out if keepdims else out.squeeze(axis)


def log_softmax(x, axis=-1):
    return x - logsumexp(x, axis=axis, keepdims=True)


def softmax(x, axis=-1):
    e = exp(x - stop_gradient(x.max(axis=axis, keepdims=True)))
    return e / e.sum(axis=axis, keepdims=True)


def one_hot(idx, n, dtype="float32"):
    """Rows of the identity: one_hot(idx)[..., c] = 1 where idx == c (nn.py:45-46)."""
    return take(eye(n, dtype), idx, 0)


def dropout(key, x, rate, training=True):
    """Zeroes each element with probability `rate` and scales the kept ones by 1 / (1 - rate), so
    the expectation is unchanged (nn.py:49-55)."""
    if not training or rate == 0.0:
        return x
    keep = 1.0 - rate
    return x * random.bernoulli(key, keep, x.shape, x.dtype) / keep


def top_k_logits(logits, k):
    """Keeps the `k` largest logits of the last axis; the rest drop to -1e9 (nn.py:60-63)."""
    values, _ = top_k(logits, k)
    return where(logits >= values[..., -1:], logits, -1e9)


def top_p_logits(logits, p):
    """Nucleus filter (nn.py:66-72): keeps the smallest set of top tokens whose probability
    reaches `p`; a token stays while the probability mass ranked before it is below `p`."""
    order = argsort(logits, descending=True)
    probs = softmax(take_along_axis(logits, order))
    keep_sorted = (cumsum(probs) - probs) < p
    return where(take_along_axis(keep_sorted, argsort(order.cast(logits.dtype))), logits, -1e9)


def cross_entropy(logits, labels, axis=-1):
    """Mean negative log-likelihood of int32 labels (nn.py:78-84)."""
    lp = log_softmax(logits, axis)
    idx = labels.reshape(tuple(labels.shape) + (1,))
    return -take_along_axis(lp, idx).mean()


def binary_cross_entropy_with_logits(logits, targets):
    """Mean of max(z, 0) - z t + log(1 + exp(-|z|)), the stable form (nn.py:87-88)."""
    return (maximum(logits, 0.0) - logits * targets + (1.0 + exp(-abs(logits))).log()).mean()


def mse_loss(pred, target):
    d = pred - target
    return (d * d).mean()


def l1_loss(pred, target):
    return abs(pred - target).mean()


def accuracy(logits, labels):
    """Fraction of rows whose arg-max equals the int32 label (nn.py:100-101)."""
    return equal(argmax(logits), labels).cast(logits.dtype).mean()


def normal_init(std=0.02):
    return lambda key, shape, dtype="float32": random.normal(key, shape, dtype) * std


def xavier_uniform(key, shape, dtype="float32"):
    """Uniform in +-sqrt(6 / (fan_in + fan_out)) over the last two extents (nn.py:111-114)."""
    limit = math.sqrt(6.0 / (shape[-2] + shape[-1]))
    return random.uniform(key, shape, dtype, -limit, limit)


def kaiming_uniform(key, shape, dtype="float32"):
    """Uniform in +-sqrt(6 / fan_in) (nn.py:117-119)."""
    limit = math.sqrt(6.0 / shape[-2])
    return random.uniform(key, shape, dtype, -limit, limit)


class Linear:
    """`x @ w + b`, w of shape (in, out)."""

    def __init__(self, d_in, d_out, bias=True, init=None, dtype="float32"):
        self.d_in, self.d_out, self.bias, self.dtype = d_in, d_out, bias, dtype
        self.w_init = init or normal_init(0.02)

    def init(self, key):
        p = {"w": self.w_init(key, (self.d_in, self.d_out), self.dtype)}
        if self.bias:
            p["b"] = zeros(self.d_out, self.dtype)
        return p

    def __call__(self, p, x):
        y = x @ p["w"]
        return y + p["b"] if self.bias else y


class Embedding:
    def __init__(self, n, d, init=None, dtype="float32"):
        self.n, self.d, self.dtype = n, d, dtype
        self.w_init = init or normal_init(0.02)

    def init(self, key):
        return {"table": self.w_init(key, (self.n, self.d), self.dtype)}

    def __call__(self, p, idx):
        return take(p["table"], idx, 0)


class LayerNorm:
    def __init__(self, d, eps=1e-5, dtype="float32"):
        self.d, self.eps, self.dtype = d, eps, dtype

    def init(self, key=None):
        return {"scale": ones(self.d, self.dtype), "shift": zeros(self.d, self.dtype)}

    def __call__(self, p, x):
        d = x - x.mean(axis=-1, keepdims=True)
        v = (d * d).mean(axis=-1, keepdims=True)
        return d / (v + self.eps).sqrt() * p["scale"] + p["shift"]


class MultiHeadAttention:
    """Self-attention with a full (T, T) score matrix and an optional visibility mask; with a key
    and a dropout rate it drops attention weights and outputs while training (nn.py:170-199)."""

    def __init__(self, d, heads, bias=True, dropout_rate=0.0, init=None, dtype="float32"):
        if d % heads:
            raise ValueError(f"model dimension {d} is not divisible by {heads} heads")
        self.d, self.heads, self.rate = d, heads, dropout_rate
        self.qkv = Linear(d, 3 * d, bias, init, dtype)
        self.out = Linear(d, d, bias, init, dtype)

    def init(self, key):
        k1, k2 = random.split(key)
        return {"qkv": self.qkv.init(k1), "out": self.out.init(k2)}

    def __call__(self, p, x, mask=None, key=None):
        b, t, d = x.shape
        hd = d // self.heads
        qkv = self.qkv(p["qkv"], x).reshape(b, t, 3, self.heads, hd).transpose(2, 0, 3, 1, 4)
        q, k, v = qkv[0], qkv[1], qkv[2]
        scores = q @ swapaxes(k, -1, -2) / math.sqrt(hd)
        if mask is not None:
            scores = where(mask, scores, -1e9)
        weights = softmax(scores)
        training = key is not None and self.rate > 0.0
        if training:
            k1, key = random.split(key)
            weights = dropout(k1, weights, self.rate)
        h = (weights @ v).transpose(0, 2, 1, 3).reshape(b, t, d)
        out = self.out(p["out"], h)
        return dropout(key, out, self.rate) if training else out


class TransformerBlock:
    """Pre-norm block: attention, then a GELU MLP, each with a residual connection."""

    def __init__(self, d, heads, mlp_ratio=4, dropout_rate=0.0, init=None, dtype="float32"):
        self.rate = dropout_rate
        self.norm1, self.norm2 = LayerNorm(d, dtype=dtype), LayerNorm(d, dtype=dtype)
        self.attn = MultiHeadAttention(d, heads, True, dropout_rate, init, dtype)
        self.fc1 = Linear(d, mlp_ratio * d, True, init, dtype)
        self.fc2 = Linear(mlp_ratio * d, d, True, init, dtype)

    def init(self, key):
        k1, k2, k3 = random.split(key, 3)
        return {"norm1": self.norm1.init(), "attn": self.attn.init(k1), "norm2": self.norm2.init(), "fc1": self.fc1.init(k2), "fc2": self.fc2.init(k3)}

    def __call__(self, p, x, mask=None, key=None):
        # As in rg the block key is split even without dropout (the split is then dead code).
        k1, k2 = (None, None) if key is None else random.split(key)
        x = x + self.attn(p["attn"], self.norm1(p["norm1"], x), mask, k1)
        h = self.fc2(p["fc2"], gelu(self.fc1(p["fc1"], self.norm2(p["norm2"], x))))
        return x + (dropout(k2, h, self.rate) if key is not None else h)


class GRUCell:
    """One gated-recurrent-unit step: gates z, r from [x, h], candidate from [x, r h], then
    (1 - z) h + z c. Loop over time in Python; the trace unrolls it (nn.py:223-240)."""

    def __init__(self, d_in, d_hidden, init=None, dtype="float32"):
        self.d_hidden = d_hidden
        self.gates = Linear(d_in + d_hidden, 2 * d_hidden, True, init, dtype)
        self.cand = Linear(d_in + d_hidden, d_hidden, True, init, dtype)

    def init(self, key):
        k1, k2 = random.split(key)
        return {"gates": self.gates.init(k1), "cand": self.cand.init(k2)}

    def __call__(self, p, x, h):
        g = sigmoid(self.gates(p["gates"], concatenate([x, h], -1)))
        z, r = g[..., :self.d_hidden], g[..., self.d_hidden:]
        c = tanh(self.cand(p["cand"], concatenate([x, r * h], -1)))
        return (1.0 - z) * h + z * c


class Sequential:
    """Layers applied in order; plain functions such as `relu` are parameterless layers
    (nn.py:243-255)."""

    def __init__(self, *layers):
        self.layers = layers

    def init(self, key):
        keys = random.split(key, max(1, len(self.layers)))
        return {str(i): l.init(keys[i]) for i, l in enumerate(self.layers) if hasattr(l, "init")}

    def __call__(self, p, x):
        for i, l in enumerate(self.layers):
            x = l(p[str(i)], x) if hasattr(l, "init") else l(x)
        return x
