"""Optimisers as pure traced functions (the compositions of python/rg/optim.py)."""
from typing import Callable, NamedTuple

from .core import full, tree_leaves, tree_map, zeros_like


class Optimizer(NamedTuple):
    init: Callable
    update: Callable


def sgd(lr):
    def init(params):
        return {"count": full((), 0, tree_leaves(params)[0].dtype), "velocity": tree_map(zeros_like, params)}

    def update(grads, state, params):
        return tree_map(lambda p, d: p - lr * d, params, grads), {"count": state["count"] + 1.0, "velocity": state["velocity"]}

    return Optimizer(init, update)


def adamw(lr, b1=0.9, b2=0.999, eps=1e-8, weight_decay=0.01):
    """Adam with decoupled weight decay on parameters of rank >= 2 (optim.py:86-113)."""

    def init(params):
        return {"count": full((), 0, tree_leaves(params)[0].dtype), "mu": tree_map(zeros_like, params), "nu": tree_map(zeros_like, params)}

    def update(grads, state, params):
        t = state["count"] + 1.0
        rate = lr
        mu = tree_map(lambda m, g: b1 * m + (1.0 - b1) * g, state["mu"], grads)
        nu = tree_map(lambda n, g: b2 * n + (1.0 - b2) * (g * g), state["nu"], grads)
        c1, c2 = 1.0 - b1 ** t, 1.0 - b2 ** t

        def step(p, m, n):
            d = (m / c1) / ((n / c2).sqrt() + eps)
            if weight_decay and p.ndim >= 2:
                d = d + weight_decay * p
            return p - rate * d
        return tree_map(step, params, mu, nu), {"count": t, "mu": mu, "nu": nu}

    return Optimizer(init, update)
