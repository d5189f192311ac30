"""Python front end tracing rg programs onto an engine module with rg's `_rg` interface."""
from . import checkpoint, gpt, nn, optim, random, tree
from .core import (Compiled, DiagnosticError, Report, RunResult, Tensor, Tracer, abs, all_reduce, arange, argmax, argsort, broadcast_to, clip,
                   compile, concatenate, cond, cos, cumsum, custom_vjp, devices, equal, exp, expand_dims, eye, flatten, flip, floor, full,
                   grad, hessian, inspect, jvp, linspace, log, matmul, maximum, minimum, native, not_equal, ones, ones_like, op, reshape, run,
                   scan, sign, sin, sort, sqrt, square, squeeze, stack, stop_gradient, swapaxes, take, take_along_axis, tanh, tensor, top_k,
                   transpose, tree_leaves, tree_map, tril, unflatten, use, value_and_grad, where, while_loop, zeros, zeros_like)
from .checkpoint import Session


def sum(x, axis=None, keepdims=False): return x.sum(axis, keepdims)
def mean(x, axis=None, keepdims=False): return x.mean(axis, keepdims)
def max(x, axis=None, keepdims=False): return x.max(axis, keepdims)
def min(x, axis=None, keepdims=False): return x.min(axis, keepdims)
def var(x, axis=None, keepdims=False): return x.var(axis, keepdims)
def std(x, axis=None, keepdims=False): return x.std(axis, keepdims)
