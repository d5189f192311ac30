"""Helpers for trees: nested tuples, lists and dicts of tensors (python/rg/tree.py).

Leaves come in flatten order, with dict keys sorted, the order checkpoints and `run` use.
"""
from .checkpoint import paths
from .core import flatten
from .core import unflatten as _unflatten


def leaves(t):
    return flatten(t)[0]


def structure(t):
    """The tree's shape without its leaves; equal for trees that `map` can combine."""
    return flatten(t)[1]


def map(f, t, *rest):
    """`f` applied leaf by leaf across trees of one structure."""
    ls, d = flatten(t)
    others = [flatten(r) for r in rest]
    if any(o[1] != d for o in others):
        raise ValueError("tree.map needs trees of the same structure")
    return _unflatten(d, [f(*vals) for vals in zip(ls, *(o[0] for o in others))])


def unflatten(structure_, values):
    return _unflatten(structure_, values)


def size(t):
    """Total element count over all leaves."""
    return sum(l.size for l in leaves(t))


def global_norm(t):
    """The L2 norm of all leaves taken together."""
    return sum((l * l).sum() for l in leaves(t)).sqrt()


__all__ = ["leaves", "structure", "map", "unflatten", "paths", "size", "global_norm"]
