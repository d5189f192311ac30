"""AdamW, the optimiser of BASELINE configs 2, 4 and 5, recorded as plain graph ops.

The update follows rg's python/rg/optim.py:86-113 op for op, since the plan the device runs and
its rounding depend on it: moments m = b1 m + (1 - b1) g and v = b2 v + (1 - b2) g^2, bias
corrections 1 - b^t with t = count + 1, step (m / c1) / (sqrt(v / c2) + eps) plus weight decay
times the parameter for parameters of rank >= 2, scaled by the learning rate. `max_grad_norm`
first scales all gradients by min(1, max_norm / global L2 norm).
"""
from .tracing import full, where, zeros_like
from .trees import tree_leaves, tree_map


class AdamW:
    """`init(params)` -> state {"count", "mu", "nu"}; `update(grads, state, params)` ->
    (new params, new state). `decays(param)` picks the parameters that take weight decay."""

    def __init__(self, lr, b1=0.9, b2=0.999, eps=1e-8, weight_decay=0.01, decays=None, max_grad_norm=None):
        self.lr, self.b1, self.b2, self.eps, self.wd = lr, b1, b2, eps, weight_decay
        self.decays = decays or (lambda p: p.ndim >= 2)
        self.max_grad_norm = max_grad_norm

    def init(self, params):
        dtype = tree_leaves(params)[0].dtype
        return {"count": full((), 0, dtype), "mu": tree_map(zeros_like, params), "nu": tree_map(zeros_like, params)}

    def _clipped(self, grads):
        if not self.max_grad_norm:
            return grads
        norm = sum((g * g).sum() for g in tree_leaves(grads)).sqrt()
        scale = self.max_grad_norm / where(norm >= self.max_grad_norm, norm, self.max_grad_norm)
        return tree_map(lambda g: g * scale, grads)

    def update(self, grads, state, params):
        b1, b2 = self.b1, self.b2
        grads = self._clipped(grads)
        t = state["count"] + 1.0
        lr = self.lr(state["count"]) if callable(self.lr) else self.lr
        mu = tree_map(lambda m, g: b1 * m + (1.0 - b1) * g, state["mu"], grads)
        nu = tree_map(lambda v, g: b2 * v + (1.0 - b2) * (g * g), state["nu"], grads)
        c1, c2 = 1.0 - b1 ** t, 1.0 - b2 ** t

        def new_param(p, m, v):
            d = (m / c1) / ((v / c2).sqrt() + self.eps)
            if self.wd and self.decays(p):
                d = d + self.wd * p
            return p - lr * d
        return tree_map(new_param, params, mu, nu), {"count": t, "mu": mu, "nu": nu}


def adamw(lr, b1=0.9, b2=0.999, eps=1e-8, weight_decay=0.01, max_grad_norm=None):
    return AdamW(lr, b1, b2, eps, weight_decay, max_grad_norm=max_grad_norm)
