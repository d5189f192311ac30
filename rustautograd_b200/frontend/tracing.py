"""Recording rg programs as graphs of rg's primitive ops.

An engine module with rg's `_rg` interface (this package's CUDA device module, or the CPU oracle
in tests) owns graphs, constants and evaluation. This module turns Python arithmetic on arrays
into nodes of such a graph:

* A `Tensor` is a concrete value held by the engine. Outside any recording, an operation on
  tensors runs at once as a one-node graph.
* While a function is being recorded (`compile`, `value_and_grad` and the control-flow bodies),
  its arguments are `Traced` nodes of a graph, and every operation appends a node.

Operands that are not nodes of the graph being recorded become nodes as they are met, left to
right: a Python number becomes a constant of the dtype of the operation's first array operand,
a concrete tensor (or nested list, or numpy array) becomes a constant, and a node of an
enclosing graph (read inside a control-flow body) becomes an extra input of the body. The order
in which nodes are created is part of the program's meaning for the engine (node ids, and so
the compiled plan, follow it), and rg's front end creates them in Python's evaluation order in
the same way, so equal programs give equal graphs.
"""
import array
import contextlib
import json
import os
import sys

_CODES = {"float32": "f", "float64": "d", "int32": "i"}
_HERE = os.path.dirname(os.path.abspath(__file__)) + os.sep


class _Engine:
    module = None
    device = None


def use(module, device=None):
    """Selects the engine module (rg's `_rg` interface) and the default device for `compile`."""
    _Engine.module, _Engine.device = module, device


def native():
    if _Engine.module is None:
        from .. import _rg
        _Engine.module = _rg
    return _Engine.module


def default_device():
    if _Engine.device is not None:
        return _Engine.device
    names = native().available_devices()
    return names[0] if names else "cuda"


def caller():
    """`file:line` of the innermost frame outside this package: where a user wrote the op."""
    f = sys._getframe(1)
    while f is not None and f.f_code.co_filename.startswith(_HERE):
        f = f.f_back
    return None if f is None else f"{f.f_code.co_filename}:{f.f_lineno}"


class DiagnosticError(Exception):
    """A front-end error, carrying a diagnostic of the engine's JSON shape in `.diagnostic`."""


def diagnostic(code, observation, cause):
    d = {"status": "validation_failed", "severity": "error", "code": code,
         "node": {"id": None, "operation": None, "source": caller(), "role": "forward"},
         "observation": observation, "diagnosis": {"cause": cause, "certainty": "verified"}}
    err = DiagnosticError(json.dumps(d))
    err.diagnostic = d
    return err


# ---------------------------------------------------------------------------------------------
# Recording frames
# ---------------------------------------------------------------------------------------------

class Frame:
    """A graph being recorded. A control-flow body's frame has the enclosing frame as `parent`;
    `captured` maps each enclosing node the body reads to the body input standing for it, in
    first-use order (that order is the order of the extra inputs of the control-flow node)."""

    def __init__(self, graph, parent=None):
        self.graph, self.parent, self.captured = graph, parent, {}

    def node(self, value, dtype):
        """Node id in this frame for an operand (see the module docstring for the rules)."""
        if isinstance(value, Traced):
            if value.frame is self:
                return value.id
            if self.parent is None:
                raise diagnostic("TRACER_LEAK", {"node": value.id}, "tracer_from_a_finished_trace")
            outer = self.parent.node(value, dtype)
            if outer not in self.captured:
                self.captured[outer] = self.graph.input(list(value.shape), value.dtype, caller())
            return self.captured[outer]
        if isinstance(value, float) and dtype == "int32" and not value.is_integer():
            raise diagnostic("DTYPE_MISMATCH", {"scalar": value, "tensor_dtype": dtype}, "fractional_scalar_with_int32_tensor_cast_first")
        if not isinstance(value, Tensor):
            value = tensor(value, dtype if isinstance(value, (int, float)) else None)
        return self.graph.constant(value._t, caller())

    def wrap(self, node_id):
        return Traced(self, node_id)


_active = []


def recording():
    """The innermost frame being recorded, or None."""
    return _active[-1] if _active else None


@contextlib.contextmanager
def record(frame):
    _active.append(frame)
    try:
        yield frame
    finally:
        _active.pop()


def dtype_of(values):
    """dtype of the first array among `values` (None if there is none)."""
    for v in values:
        if isinstance(v, Array):
            return v.dtype
    return None


def op(name, *operands, **attrs):
    """Appends primitive `name` to the graph being recorded, or evaluates it at once."""
    dtype = dtype_of(operands)
    frame = recording()
    if frame is not None:
        ids = [frame.node(o, dtype) for o in operands]
        return Traced(frame, frame.graph.op(name, ids, attrs or None, caller()))
    scratch = Frame(native().Graph())
    ids = [scratch.node(o, dtype) for o in operands]
    node = scratch.graph.op(name, ids, attrs or None, caller())
    return Tensor(scratch.graph.eval([node])[0])


# ---------------------------------------------------------------------------------------------
# Arrays
# ---------------------------------------------------------------------------------------------

class Array:
    """Operations shared by concrete tensors and recorded nodes."""

    @property
    def ndim(self):
        return len(self.shape)

    @property
    def size(self):
        n = 1
        for d in self.shape:
            n *= d
        return n

    def _axis(self, a):
        return a + self.ndim if a < 0 else a

    def _axes(self, axis):
        if axis is None:
            return list(range(self.ndim))
        return [self._axis(a) for a in (axis if isinstance(axis, (tuple, list)) else [axis])]

    # Reductions over axes: Sum/Max/Min with kept or dropped dimensions; the mean is the sum
    # divided by the element count of the reduced axes.
    def sum(self, axis=None, keepdims=False):
        return op("sum", self, axes=self._axes(axis), keepdims=keepdims)

    def max(self, axis=None, keepdims=False):
        return op("max", self, axes=self._axes(axis), keepdims=keepdims)

    def min(self, axis=None, keepdims=False):
        return op("min", self, axes=self._axes(axis), keepdims=keepdims)

    def mean(self, axis=None, keepdims=False):
        axes = self._axes(axis)
        count = 1
        for a in axes:
            if 0 <= a < self.ndim:
                count *= self.shape[a]
        return self.sum(axis=axes, keepdims=keepdims) / count

    def var(self, axis=None, keepdims=False):
        centred = self - self.mean(axis=axis, keepdims=True)
        return (centred * centred).mean(axis=axis, keepdims=keepdims)

    def reshape(self, *shape):
        dims = list(shape[0]) if len(shape) == 1 and isinstance(shape[0], (tuple, list)) else list(shape)
        if -1 in dims:
            known = 1
            for d in dims:
                if d != -1:
                    known *= d
            dims[dims.index(-1)] = self.size // known if known else 0
        return op("reshape", self, shape=dims)

    def transpose(self, *perm):
        p = list(perm[0]) if len(perm) == 1 and isinstance(perm[0], (tuple, list)) else list(perm)
        return op("transpose", self, perm=p if p else list(range(self.ndim))[::-1])

    @property
    def T(self):
        return self.transpose()

    def swapaxes(self, a, b):
        p = list(range(self.ndim))
        a, b = self._axis(a), self._axis(b)
        p[a], p[b] = p[b], p[a]
        return self.transpose(p)

    def squeeze(self, axis=None):
        drop = [i for i, d in enumerate(self.shape) if d == 1] if axis is None else self._axes(axis)
        return self.reshape([d for i, d in enumerate(self.shape) if i not in drop])

    def cast(self, dtype):
        return op("cast", self, dtype=dtype)

    def astype(self, dtype):
        return self if self.dtype == dtype else self.cast(dtype)

    def take(self, idx, axis=0):
        return take(self, idx, axis)

    def argmax(self, axis=-1):
        return argmax(self, axis)

    def __iter__(self):
        if self.ndim == 0:
            raise diagnostic("INVALID_SLICE", {"shape": self.shape}, "cannot_iterate_a_scalar")
        return (self[i] for i in range(self.shape[0]))

    def __getitem__(self, key):
        return _index(self, key)


# Operators. Reflected forms put the other operand first, as rg's ops are not commutative in
# general; x < y and x <= y are recorded as y > x and y >= x.
def _binary(name, reflected=False):
    if reflected:
        return lambda self, other: op(name, other, self)
    return lambda self, other: op(name, self, other)


for _name, _fwd, _rev in [("add", "__add__", "__radd__"), ("sub", "__sub__", "__rsub__"), ("mul", "__mul__", "__rmul__"),
                          ("div", "__truediv__", "__rtruediv__"), ("pow", "__pow__", "__rpow__"), ("matmul", "__matmul__", "__rmatmul__")]:
    setattr(Array, _fwd, _binary(_name))
    setattr(Array, _rev, _binary(_name, reflected=True))
Array.__gt__ = _binary("gt")
Array.__ge__ = _binary("ge")
Array.__lt__ = _binary("gt", reflected=True)
Array.__le__ = _binary("ge", reflected=True)
Array.__neg__ = lambda self: op("neg", self)
Array.__abs__ = lambda self: op("abs", self)
for _name in ("exp", "log", "sqrt", "sin", "cos", "tanh", "floor"):
    setattr(Array, _name, (lambda n: lambda self: op(n, self))(_name))
Array.std = lambda self, axis=None, keepdims=False: self.var(axis=axis, keepdims=keepdims).sqrt()


class Tensor(Array):
    """A concrete value: `_t` is the engine module's tensor handle."""

    def __init__(self, handle):
        self._t = handle

    @property
    def shape(self):
        return tuple(self._t.shape)

    @property
    def dtype(self):
        return self._t.dtype

    def numpy(self):
        import numpy as np
        return np.frombuffer(self._t.tobytes(), dtype=self.dtype).reshape(self.shape).copy()

    def __array__(self, dtype=None, copy=None):
        a = self.numpy()
        return a if dtype is None else a.astype(dtype)

    def tolist(self):
        return self.numpy().tolist()

    def __float__(self):
        first = array.array(_CODES[self.dtype])
        first.frombytes(self._t.tobytes()[:first.itemsize])
        return float(first[0])

    def __int__(self):
        return int(float(self))

    __index__ = __int__

    def item(self):
        return int(self) if self.dtype == "int32" else float(self)

    def __repr__(self):
        return f"Tensor({self.tolist()}, dtype={self.dtype})"


class Traced(Array):
    """Node `id` of the graph recorded by `frame`."""

    def __init__(self, frame, node_id):
        self.frame, self.id = frame, node_id

    @property
    def shape(self):
        return tuple(self.frame.graph.shape(self.id))

    @property
    def dtype(self):
        return self.frame.graph.dtype(self.id)

    def __bool__(self):
        raise diagnostic("CONTROL_FLOW_ON_TRACER", {"node": self.id}, "python_value_depends_on_traced_tensor_use_rg_where")

    def __repr__(self):
        return f"Traced(node={self.id}, shape={self.shape}, dtype={self.dtype})"


# ---------------------------------------------------------------------------------------------
# Indexing: `take` for index arrays and stepped slices, otherwise one `slice` over every axis
# followed by a `reshape` when integers drop axes or None adds them.
# ---------------------------------------------------------------------------------------------

def _index(x, key):
    if isinstance(key, (Array, list)) or (hasattr(key, "tobytes") and hasattr(key, "dtype")):
        return take(x, tensor(key, "int32") if isinstance(key, list) else key, 0)
    key = key if isinstance(key, tuple) else (key,)
    if any(k is Ellipsis for k in key):
        at = next(i for i, k in enumerate(key) if k is Ellipsis)
        named = sum(1 for k in key if k is not None and k is not Ellipsis)
        key = key[:at] + (slice(None),) * (x.ndim - named) + key[at + 1:]
    if sum(1 for k in key if k is not None) > x.ndim:
        raise diagnostic("INVALID_SLICE", {"shape": x.shape, "index_rank": len(key)}, "too_many_indices")
    if any(isinstance(k, slice) and k.step not in (None, 1) for k in key):
        picked, plain, axis = x, [], 0
        for k in key:
            if isinstance(k, slice) and k.step not in (None, 1):
                positions = list(range(*k.indices(x.shape[axis])))
                if not positions:
                    raise diagnostic("INVALID_SLICE", {"shape": x.shape, "axis": axis, "slice": repr(k)}, "stepped_slice_selects_nothing")
                picked = take(picked, tensor(positions, "int32"), axis)
                k = slice(None)
            plain.append(k)
            if k is not None:
                axis += 1
        return picked[tuple(plain)]
    key = key + (slice(None),) * (x.ndim - sum(1 for k in key if k is not None))
    starts, stops, result_shape, axis = [], [], [], 0
    for k in key:
        if k is None:
            result_shape.append(1)
            continue
        extent = x.shape[axis]
        if isinstance(k, slice):
            lo, hi, _ = k.indices(extent)
            starts.append(lo)
            stops.append(max(lo, hi))
            result_shape.append(max(0, hi - lo))
        elif isinstance(k, int):
            i = k + extent if k < 0 else k
            if not 0 <= i < extent:
                raise diagnostic("INVALID_SLICE", {"shape": x.shape, "axis": axis, "index": k}, "index_out_of_bounds")
            starts.append(i)
            stops.append(i + 1)
        else:
            raise diagnostic("INVALID_SLICE", {"shape": x.shape, "index_type": type(k).__name__}, "unsupported_index_type")
        axis += 1
    out = op("slice", x, starts=starts, stops=stops)
    return out if tuple(result_shape) == out.shape else out.reshape(result_shape)


# ---------------------------------------------------------------------------------------------
# Concrete values
# ---------------------------------------------------------------------------------------------

def _only_ints(x):
    if isinstance(x, (list, tuple)):
        return all(_only_ints(v) for v in x)
    return isinstance(x, int)


def tensor(data, dtype=None):
    """A Tensor from a Tensor, numpy array, number or nested list (ints give int32, floats
    float32 unless `dtype` says otherwise)."""
    if isinstance(data, Tensor):
        return data if dtype in (None, data.dtype) else data.cast(dtype)
    if hasattr(data, "tobytes") and hasattr(data, "dtype"):
        name = str(data.dtype)
        dt = dtype or (name if name in _CODES else ("int32" if data.dtype.kind in "iub" else "float32"))
        a = data if name == dt else data.astype(dt)
        return Tensor(native().Tensor(a.tobytes(order="C"), list(a.shape), dt))
    dt = dtype or ("int32" if _only_ints(data) else "float32")
    values, shape = array.array(_CODES[dt]), []
    convert = int if dt == "int32" else float

    def walk(v, depth):
        if isinstance(v, (list, tuple)):
            if depth == len(shape):
                shape.append(len(v))
            for item in v:
                walk(item, depth + 1)
        else:
            values.append(convert(v))
    walk(data, 0)
    return Tensor(native().Tensor(values.tobytes(), shape, dt))


def _of_values(shape, dtype, values):
    return Tensor(native().Tensor(array.array(_CODES[dtype], values).tobytes(), list(shape), dtype))


def full(shape, value, dtype="float32"):
    shape = [shape] if isinstance(shape, int) else list(shape)
    n = 1
    for d in shape:
        n *= d
    return _of_values(shape, dtype, [value] * n)


def zeros(shape, dtype="float32"):
    return full(shape, 0, dtype)


def ones(shape, dtype="float32"):
    return full(shape, 1, dtype)


def zeros_like(x):
    return full(x.shape, 0, x.dtype)


def ones_like(x):
    return full(x.shape, 1, x.dtype)


def arange(n, dtype="int32"):
    return _of_values([n], dtype, range(n))


def tril(n, dtype="float32"):
    """n x n lower-triangular ones (the causal mask)."""
    return _of_values([n, n], dtype, [1 if c <= r else 0 for r in range(n) for c in range(n)])


# ---------------------------------------------------------------------------------------------
# Functions over arrays
# ---------------------------------------------------------------------------------------------

def stop_gradient(x):
    return op("stop_gradient", x)


def where(c, a, b):
    """`a` where `c` is nonzero, else `b`; the condition takes the branches' dtype first."""
    dt = dtype_of((a, b))
    if dt is not None and isinstance(c, Array) and c.dtype != dt:
        c = c.cast(dt)
    return op("where", c, a, b)


def maximum(a, b):
    return op("maximum", a, b)


def minimum(a, b):
    return op("minimum", a, b)


def exp(x):
    return op("exp", x)


def log(x):
    return op("log", x)


def sqrt(x):
    return op("sqrt", x)


def tanh(x):
    return op("tanh", x)


def floor(x):
    return op("floor", x)


def abs(x):  # noqa: A001 - rg's name
    return op("abs", x)


def square(x):
    return x * x


def matmul(a, b):
    return op("matmul", a, b)


def broadcast_to(x, shape):
    return op("broadcast_to", x, shape=list(shape))


def all_reduce(x):
    """Sum over the data-parallel ranks (identity on one rank)."""
    return op("all_reduce", x)


def take(x, idx, axis=0):
    """Slices of `x` along `axis` at int32 positions `idx` (clamped to the extent)."""
    return op("take", x, idx if isinstance(idx, Array) else tensor(idx), axis=x._axis(axis))


def swapaxes(x, a, b):
    return x.swapaxes(a, b)


def _along_last(x, axis, f):
    """`f` applied with `axis` moved to the last position, and moved back."""
    axis = x._axis(axis)
    return f(x) if axis == x.ndim - 1 else f(x.swapaxes(axis, -1)).swapaxes(axis, -1)


def take_along_axis(x, idx, axis=-1):
    idx = idx if isinstance(idx, Array) else tensor(idx)
    axis = x._axis(axis)
    if axis == x.ndim - 1:
        return op("take_along", x, idx)
    return op("take_along", x.swapaxes(axis, -1), idx.swapaxes(axis, -1)).swapaxes(axis, -1)


def concatenate(xs, axis=0):
    xs = list(xs)
    return op("concat", *xs, axis=xs[0]._axis(axis))


def top_k(x, k, axis=-1):
    """The k largest values and their int32 positions, largest first (ties in position order,
    NaN last)."""
    idx = _along_last(x, axis, lambda v: op("arg_top_k", v, k=k))
    return take_along_axis(x, idx, axis), idx


def argsort(x, axis=-1, descending=False):
    """Stable sorting positions; NaN last either way."""
    n = x.shape[x._axis(axis)]
    return _along_last(x if descending else -x, axis, lambda v: op("arg_top_k", v, k=n))


def sort(x, axis=-1, descending=False):
    return take_along_axis(x, argsort(x, axis, descending), axis)


def cumsum(x, axis=-1):
    return _along_last(x, axis, lambda v: op("cumsum", v, reverse=False))


def argmax(x, axis=-1):
    """Position of the first largest value along `axis`, which is removed; None flattens."""
    if axis is None:
        return op("argmax", x.reshape(-1))
    axis = x._axis(axis)
    return op("argmax", x if axis == x.ndim - 1 else x.swapaxes(axis, -1))
