"""A small front end that records the workloads of BASELINE's configs as rg graphs and drives the
engine's compile / run over them: the linear regression (config 1), AdamW (config 2), matrix
chains (config 3), the character GPT training step and sampler (configs 4 and 5), and control
flow, gradient rules, observe statistics and checkpoints for the tests.

rg's own Python package (`python/rg/`) runs unchanged over this package's `_rg` module; this
front end exists for machines where rg's package is not installed (the GPU boxes), and records
the same graphs for the same programs (tests/golden holds graphs recorded by rg's front end).
"""
from . import checkpoint, gpt, nn, optim, random
from .checkpoint import Session
from .program import Compiled, Report, RunResult, compile, cond, custom_vjp, grad, run, scan, value_and_grad, while_loop
from .tracing import (DiagnosticError, Tensor, Traced, abs, all_reduce, arange, argmax, argsort, broadcast_to, concatenate, cumsum, exp, floor,
                      full, log, matmul, maximum, minimum, native, ones, ones_like, op, sort, sqrt, square, stop_gradient, swapaxes, take,
                      take_along_axis, tanh, tensor, top_k, tril, use, where, zeros, zeros_like)
from .trees import flatten, tree_leaves, tree_map, unflatten


def devices():
    """Device names the selected engine module compiles for."""
    return native().available_devices()
