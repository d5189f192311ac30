"""Python front end tracing rg programs onto an engine module with rg's `_rg` interface."""
from . import checkpoint, gpt, nn, optim, random
from .core import (Compiled, all_reduce, DiagnosticError, Tensor, Tracer, arange, argmax, argsort, compile, concatenate, cond, cumsum, exp,
                   flatten, floor, full, log, maximum, minimum, native, ones, op, run, scan, sort, sqrt, stop_gradient, swapaxes, take,
                   take_along_axis, tanh, tensor, top_k, tree_leaves, tree_map, tril, unflatten, use, value_and_grad, where, while_loop,
                   zeros, zeros_like)
from .checkpoint import Session
