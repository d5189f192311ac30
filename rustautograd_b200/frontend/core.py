"""Tracing front end for the rg engine interface (`_rg` modules).

Python operations on `Tensor`s run eagerly (one-node graphs evaluated by the engine's device);
inside `compile`, `value_and_grad` and friends they record nodes on a `Tracer`. The op sequence
a program emits is the one rg's own front end emits (python/rg/_core.py), so the same program
yields the same graph and therefore the same compiled plan: scalars become constants of the
dtype of the first tensor operand, reductions over axes, `mean` as sum then divide, slicing as
`slice` plus `reshape`, and so on. This front end works over any module with rg's `_rg`
interface: the CUDA device module of this package (the default) or a CPU one.
"""
import array
import json
import os
import sys

_TYPECODES = {"float32": "f", "float64": "d", "int32": "i"}
_state = {"native": None, "device": None}
_trace_stack = []
_PKG = os.path.dirname(os.path.abspath(__file__)) + os.sep


def use(native, device=None):
    """Selects the engine module (rg's `_rg` interface) and the default compile device."""
    _state["native"] = native
    _state["device"] = device


def native():
    if _state["native"] is None:
        from .. import _rg
        _state["native"] = _rg
    return _state["native"]


def default_device():
    if _state["device"] is not None:
        return _state["device"]
    devs = native().available_devices()
    return devs[0] if devs else "cuda"


def _where_from():
    f = sys._getframe(1)
    while f is not None and f.f_code.co_filename.startswith(_PKG):
        f = f.f_back
    return f"{f.f_code.co_filename}:{f.f_lineno}" if f else None


class DiagnosticError(Exception):
    """A front-end diagnostic with the same JSON shape as the engine's."""


def _error(code, observation, cause):
    d = {"status": "validation_failed", "severity": "error", "code": code,
         "node": {"id": None, "operation": None, "source": _where_from(), "role": "forward"},
         "observation": observation, "diagnosis": {"cause": cause, "certainty": "verified"}}
    e = DiagnosticError(json.dumps(d))
    e.diagnostic = d
    return e


def _axis(x, axis):
    return axis + x.ndim if axis < 0 else axis


class _Math:
    """Operators shared by concrete tensors and tracers."""
    __array_ufunc__ = None

    def __add__(self, o): return op("add", self, o)
    def __radd__(self, o): return op("add", o, self)
    def __sub__(self, o): return op("sub", self, o)
    def __rsub__(self, o): return op("sub", o, self)
    def __mul__(self, o): return op("mul", self, o)
    def __rmul__(self, o): return op("mul", o, self)
    def __truediv__(self, o): return op("div", self, o)
    def __rtruediv__(self, o): return op("div", o, self)
    def __pow__(self, o): return op("pow", self, o)
    def __rpow__(self, o): return op("pow", o, self)
    def __matmul__(self, o): return op("matmul", self, o)
    def __rmatmul__(self, o): return op("matmul", o, self)
    def __neg__(self): return op("neg", self)
    def __abs__(self): return op("abs", self)
    def __gt__(self, o): return op("gt", self, o)
    def __ge__(self, o): return op("ge", self, o)
    def __lt__(self, o): return op("gt", o, self)
    def __le__(self, o): return op("ge", o, self)

    @property
    def ndim(self): return len(self.shape)

    @property
    def size(self):
        n = 1
        for d in self.shape:
            n *= d
        return n

    def _axes(self, axis):
        if axis is None:
            return list(range(self.ndim))
        axes = axis if isinstance(axis, (tuple, list)) else [axis]
        return [a + self.ndim if a < 0 else a for a in axes]

    def sum(self, axis=None, keepdims=False): return op("sum", self, axes=self._axes(axis), keepdims=keepdims)
    def max(self, axis=None, keepdims=False): return op("max", self, axes=self._axes(axis), keepdims=keepdims)
    def min(self, axis=None, keepdims=False): return op("min", self, axes=self._axes(axis), keepdims=keepdims)

    def mean(self, axis=None, keepdims=False):
        axes = self._axes(axis)
        count = 1
        for a in axes:
            count *= self.shape[a] if 0 <= a < self.ndim else 1
        return self.sum(axis=axes, keepdims=keepdims) / count

    def reshape(self, *shape):
        target = list(shape[0]) if len(shape) == 1 and isinstance(shape[0], (tuple, list)) else list(shape)
        if target.count(-1) == 1:
            known = 1
            for d in target:
                known *= d if d != -1 else 1
            target[target.index(-1)] = self.size // known if known else 0
        return op("reshape", self, shape=target)

    def transpose(self, *perm):
        p = list(perm[0]) if len(perm) == 1 and isinstance(perm[0], (tuple, list)) else list(perm)
        return op("transpose", self, perm=p or list(reversed(range(self.ndim))))

    @property
    def T(self): return self.transpose()

    def cast(self, dtype): return op("cast", self, dtype=dtype)
    def astype(self, dtype): return self if self.dtype == dtype else self.cast(dtype)
    def exp(self): return op("exp", self)
    def log(self): return op("log", self)
    def sqrt(self): return op("sqrt", self)
    def sin(self): return op("sin", self)
    def cos(self): return op("cos", self)
    def tanh(self): return op("tanh", self)
    def floor(self): return op("floor", self)
    def take(self, idx, axis=0): return take(self, idx, axis)
    def argmax(self, axis=-1): return argmax(self, axis)
    def swapaxes(self, a, b): return swapaxes(self, a, b)
    def squeeze(self, axis=None): return squeeze(self, axis)

    def var(self, axis=None, keepdims=False):
        """Mean squared deviation from the mean (population variance)."""
        d = self - self.mean(axis=axis, keepdims=True)
        return (d * d).mean(axis=axis, keepdims=keepdims)

    def std(self, axis=None, keepdims=False): return self.var(axis=axis, keepdims=keepdims).sqrt()

    def __iter__(self):
        if self.ndim == 0:
            raise _error("INVALID_SLICE", {"shape": self.shape}, "cannot_iterate_a_scalar")
        return (self[i] for i in range(self.shape[0]))

    def __getitem__(self, key):
        if isinstance(key, (Tensor, Tracer, list)) or (hasattr(key, "tobytes") and hasattr(key, "dtype")):
            return take(self, tensor(key, "int32") if isinstance(key, list) else key, 0)
        key = key if isinstance(key, tuple) else (key,)
        if any(k is Ellipsis for k in key):
            at = next(i for i, k in enumerate(key) if k is Ellipsis)
            used = sum(1 for k in key if k is not None and k is not Ellipsis)
            key = key[:at] + (slice(None),) * (self.ndim - used) + key[at + 1:]
        if sum(1 for k in key if k is not None) > self.ndim:
            raise _error("INVALID_SLICE", {"shape": self.shape, "index_rank": len(key)}, "too_many_indices")
        # A step other than 1 selects positions with `take`.
        stepped, plain, position = self, [], 0
        for k in key:
            if isinstance(k, slice) and k.step not in (None, 1):
                idx = list(range(*k.indices(self.shape[position])))
                if not idx:
                    raise _error("INVALID_SLICE", {"shape": self.shape, "axis": position, "slice": repr(k)}, "stepped_slice_selects_nothing")
                stepped = take(stepped, tensor(idx, "int32"), position)
                k = slice(None)
            plain.append(k)
            position += 0 if k is None else 1
        if stepped is not self:
            return stepped[tuple(plain)]
        starts, stops, keep, axis = [], [], [], 0
        for k in key + (slice(None),) * (self.ndim - sum(1 for k in key if k is not None)):
            if k is None:
                keep.append(1)
                continue
            dim = self.shape[axis]
            if isinstance(k, slice):
                start, stop, _ = k.indices(dim)
                starts.append(start)
                stops.append(max(start, stop))
                keep.append(max(0, stop - start))
            elif isinstance(k, int):
                i = k + dim if k < 0 else k
                if not 0 <= i < dim:
                    raise _error("INVALID_SLICE", {"shape": self.shape, "axis": axis, "index": k}, "index_out_of_bounds")
                starts.append(i)
                stops.append(i + 1)
            else:
                raise _error("INVALID_SLICE", {"shape": self.shape, "index_type": type(k).__name__}, "unsupported_index_type")
            axis += 1
        out = op("slice", self, starts=starts, stops=stops)
        return out.reshape(keep) if tuple(keep) != out.shape else out


class Tensor(_Math):
    """A concrete value held by the engine module."""

    def __init__(self, handle):
        self._t = handle

    @property
    def shape(self): return tuple(self._t.shape)

    @property
    def dtype(self): return self._t.dtype

    def numpy(self):
        import numpy as np
        return np.frombuffer(self._t.tobytes(), dtype=self.dtype).reshape(self.shape).copy()

    def __array__(self, dtype=None, copy=None):
        a = self.numpy()
        return a if dtype is None else a.astype(dtype)

    def tolist(self): return self.numpy().tolist()

    def __float__(self):
        flat = array.array(_TYPECODES[self.dtype])
        flat.frombytes(self._t.tobytes())
        return float(flat[0])

    def __int__(self): return int(float(self))

    def __index__(self): return int(float(self))

    def item(self): return int(self) if self.dtype == "int32" else float(self)

    def __repr__(self): return f"Tensor({self.tolist()}, dtype={self.dtype})"


class Tracer(_Math):
    """A node of the graph being traced."""

    def __init__(self, graph, node):
        self._g = graph
        self._id = node

    @property
    def shape(self): return tuple(self._g.shape(self._id))

    @property
    def dtype(self): return self._g.dtype(self._id)

    def __bool__(self):
        raise _error("CONTROL_FLOW_ON_TRACER", {"node": self._id}, "python_value_depends_on_traced_tensor_use_rg_where")

    def __repr__(self): return f"Tracer(node={self._id}, shape={self.shape}, dtype={self.dtype})"


def _ints_only(x):
    if isinstance(x, (list, tuple)):
        return all(_ints_only(i) for i in x)
    return isinstance(x, int)


def tensor(data, dtype=None):
    """A Tensor from a Tensor, numpy array, number or nested list (ints -> int32, floats -> float32)."""
    if isinstance(data, Tensor):
        return data if dtype in (None, data.dtype) else data.cast(dtype)
    if hasattr(data, "tobytes") and hasattr(data, "dtype"):
        name = str(data.dtype)
        dt = dtype or (name if name in _TYPECODES else ("int32" if data.dtype.kind in "iub" else "float32"))
        arr = data if name == dt else data.astype(dt)
        return Tensor(native().Tensor(arr.tobytes(order="C"), list(arr.shape), dt))
    dt = dtype or ("int32" if _ints_only(data) else "float32")
    flat = array.array(_TYPECODES[dt])
    conv = int if dt == "int32" else float
    shape = []

    def fill(x, depth):
        if isinstance(x, (list, tuple)):
            if depth == len(shape):
                shape.append(len(x))
            for v in x:
                fill(v, depth + 1)
        else:
            flat.append(conv(x))
    fill(data, 0)
    return Tensor(native().Tensor(flat.tobytes(), shape, dt))


def _filled(shape, value, dtype):
    shape = [shape] if isinstance(shape, int) else list(shape)
    n = 1
    for d in shape:
        n *= d
    return Tensor(native().Tensor((array.array(_TYPECODES[dtype], [value]) * n).tobytes(), shape, dtype))


def zeros(shape, dtype="float32"): return _filled(shape, 0, dtype)
def ones(shape, dtype="float32"): return _filled(shape, 1, dtype)
def full(shape, value, dtype="float32"): return _filled(shape, value, dtype)
def zeros_like(x): return _filled(x.shape, 0, x.dtype)
def ones_like(x): return _filled(x.shape, 1, x.dtype)


def arange(n, dtype="int32"):
    return Tensor(native().Tensor(array.array(_TYPECODES[dtype], range(n)).tobytes(), [n], dtype))


def linspace(start, stop, num, dtype="float32"):
    """`num` evenly spaced values from `start` to `stop`, both included (start + i * step)."""
    step = (stop - start) / (num - 1) if num > 1 else 0.0
    vals = array.array(_TYPECODES[dtype], [start + i * step for i in range(num)])
    return Tensor(native().Tensor(vals.tobytes(), [num], dtype))


def eye(n, dtype="float32"):
    """The n x n identity."""
    vals = array.array(_TYPECODES[dtype], [1 if j == i else 0 for i in range(n) for j in range(n)])
    return Tensor(native().Tensor(vals.tobytes(), [n, n], dtype))


def tril(n, dtype="float32"):
    """Lower-triangular ones: the causal mask."""
    vals = array.array(_TYPECODES[dtype], [1 if j <= i else 0 for i in range(n) for j in range(n)])
    return Tensor(native().Tensor(vals.tobytes(), [n, n], dtype))


def _first_dtype(args):
    for a in args:
        if isinstance(a, (Tensor, Tracer)):
            return a.dtype
    return None


class _BodyScope:
    """A control-flow body being traced: values of enclosing traces it reads become extra body
    inputs, in first-use order (`captures`: enclosing node -> body input)."""

    def __init__(self, parent, captures=None):
        self.parent = parent
        self.captures = dict(captures or {})


_body_scopes = {}  # id(body graph) -> _BodyScope


def _as_node(g, a, dtype):
    if isinstance(a, Tracer):
        if a._g is g:
            return a._id
        scope = _body_scopes.get(id(g))
        if scope is None:
            raise _error("TRACER_LEAK", {"node": a._id}, "tracer_from_a_finished_trace")
        outer = _as_node(scope.parent, a, dtype)
        if outer not in scope.captures:
            scope.captures[outer] = g.input(list(a.shape), a.dtype, _where_from())
        return scope.captures[outer]
    if isinstance(a, float) and dtype == "int32" and not a.is_integer():
        raise _error("DTYPE_MISMATCH", {"scalar": a, "tensor_dtype": dtype}, "fractional_scalar_with_int32_tensor_cast_first")
    t = a if isinstance(a, Tensor) else tensor(a, dtype if isinstance(a, (int, float)) else None)
    return g.constant(t._t, _where_from())


def op(name, *args, **attrs):
    """Records `name` on the current trace, or evaluates it at once outside one."""
    dtype = _first_dtype(args)
    src = _where_from()
    if _trace_stack:
        g = _trace_stack[-1]
        ids = [_as_node(g, a, dtype) for a in args]
        return Tracer(g, g.op(name, ids, attrs or None, src))
    g = native().Graph()
    ids = [_as_node(g, a, dtype) for a in args]
    return Tensor(g.eval([g.op(name, ids, attrs or None, src)])[0])


# ---- functions ----

def stop_gradient(x): return op("stop_gradient", x)


def where(c, a, b):
    dt = _first_dtype((a, b))
    if dt is not None and isinstance(c, (Tensor, Tracer)) and c.dtype != dt:
        c = c.cast(dt)
    return op("where", c, a, b)


def maximum(a, b): return op("maximum", a, b)
def equal(a, b): return op("ge", a, b) * op("ge", b, a)
def not_equal(a, b): return 1 - equal(a, b)
def minimum(a, b): return op("minimum", a, b)
def exp(x): return op("exp", x)
def log(x): return op("log", x)
def sqrt(x): return op("sqrt", x)
def sin(x): return op("sin", x)
def cos(x): return op("cos", x)
def tanh(x): return op("tanh", x)
def floor(x): return op("floor", x)
def abs(x): return op("abs", x)
def sign(x): return op("sign", x)
def square(x): return x * x
def clip(x, low, high): return minimum(maximum(x, low), high)
def broadcast_to(x, shape): return op("broadcast_to", x, shape=list(shape))
def matmul(a, b): return op("matmul", a, b)
def reshape(x, *shape): return x.reshape(*shape)
def transpose(x, *perm): return x.transpose(*perm)


def flip(x, axis=-1):
    """Reverses `x` along `axis` (a take of the positions in reverse order)."""
    axis = _axis(x, axis)
    return take(x, tensor(list(range(x.shape[axis] - 1, -1, -1)), "int32"), axis)


def expand_dims(x, axis):
    axis = axis + x.ndim + 1 if axis < 0 else axis
    return x.reshape(tuple(x.shape[:axis]) + (1,) + tuple(x.shape[axis:]))


def stack(xs, axis=0):
    """Joins equal-shaped tensors along a new axis: a concatenation of their expanded forms."""
    return concatenate([expand_dims(x, axis) for x in xs], axis)


def all_reduce(x):
    """Sum of `x` over every data-parallel rank (the identity on a single rank)."""
    return op("all_reduce", x)


def take(x, idx, axis=0):
    return op("take", x, tensor(idx) if not isinstance(idx, (Tensor, Tracer)) else idx, axis=_axis(x, axis))


def swapaxes(x, a, b):
    p = list(range(x.ndim))
    a, b = _axis(x, a), _axis(x, b)
    p[a], p[b] = p[b], p[a]
    return x.transpose(p)


def take_along_axis(x, idx, axis=-1):
    axis = _axis(x, axis)
    idx = tensor(idx) if not isinstance(idx, (Tensor, Tracer)) else idx
    if axis == x.ndim - 1:
        return op("take_along", x, idx)
    return swapaxes(op("take_along", swapaxes(x, axis, -1), swapaxes(idx, axis, -1)), axis, -1)


def concatenate(xs, axis=0):
    xs = list(xs)
    return op("concat", *xs, axis=_axis(xs[0], axis))


def _on_last(x, axis, fn):
    axis = _axis(x, axis)
    if axis == x.ndim - 1:
        return fn(x)
    return swapaxes(fn(swapaxes(x, axis, -1)), axis, -1)


def top_k(x, k, axis=-1):
    """The `k` largest values and their int32 indices, descending; ties keep index order, NaN last."""
    idx = _on_last(x, axis, lambda v: op("arg_top_k", v, k=k))
    return take_along_axis(x, idx, axis), idx


def argsort(x, axis=-1, descending=False):
    """Indices that sort `x`: stable, NaN last in both directions."""
    n = x.shape[_axis(x, axis)]
    return _on_last(x if descending else -x, axis, lambda v: op("arg_top_k", v, k=n))


def sort(x, axis=-1, descending=False):
    return take_along_axis(x, argsort(x, axis, descending), axis)


def cumsum(x, axis=-1):
    return _on_last(x, axis, lambda v: op("cumsum", v, reverse=False))


def argmax(x, axis=-1):
    """Index of the largest value on `axis` (int32, that axis removed); `axis=None` flattens first."""
    if axis is None:
        return op("argmax", x.reshape(-1))
    axis = _axis(x, axis)
    return op("argmax", x if axis == x.ndim - 1 else swapaxes(x, axis, -1))


# ---- control flow (one graph node each; bodies are traced into their own graphs) ----

def _lift(tree, g):
    leaves, tdef = flatten(tree)
    dtype = _first_dtype(leaves) or "float32"
    return [Tracer(g, _as_node(g, l, dtype)) for l in leaves], tdef


def _trace_body(fn, specs, make_args, seed=None):
    """Traces `fn` into a new graph whose first inputs follow `specs` ((shape, dtype) pairs).
    Returns (body graph, output ids, output tree, scope with the captured enclosing values)."""
    body = native().Graph()
    src = _where_from()
    args = [Tracer(body, body.input(list(sh), dt, src)) for sh, dt in specs]
    scope = _BodyScope(_trace_stack[-1])
    for outer, (sh, dt) in (seed or {}).items():
        scope.captures[outer] = body.input(list(sh), dt, src)
    _body_scopes[id(body)] = scope
    _trace_stack.append(body)
    try:
        out = fn(*make_args(args))
        leaves, tdef = flatten(out)
        ids = [_as_node(body, l, _first_dtype(leaves) or "float32") for l in leaves]
    finally:
        _trace_stack.pop()
        del _body_scopes[id(body)]
    return body, ids, tdef, scope


def _signature(g, ids):
    return [(tuple(g.shape(i)), g.dtype(i)) for i in ids]


def _shape_mismatch(part, want, got):
    return _error("CONTROL_FLOW_SHAPE_MISMATCH", {"part": part, "expected": repr(want), "got": repr(got)}, f"{part}_structure_or_shape_changed")


def _eagerly(fn, *args):
    """Control flow outside a trace: compile the call and run it once."""
    return compile(fn, args, validate="none")(*args)


def scan(f, init, xs=None, length=None):
    """`carry, y = f(carry, x)` over the first axis of `xs` in one graph node (python/rg/_core.py
    scan). Returns (final carry, stacked ys). `xs=None` needs `length`; `f` then gets None."""
    if not _trace_stack:
        if xs is None:
            return _eagerly(lambda i: scan(f, i, None, length), init)
        return _eagerly(lambda i, x: scan(f, i, x, length), init, xs)
    g = _trace_stack[-1]
    src = _where_from()
    carry, c_def = _lift(init, g)
    xl, x_def = _lift(xs, g) if xs is not None else ([], None)
    lengths = {t.shape[0] if t.ndim else None for t in xl}
    if length is not None:
        lengths.add(length)
    if len(lengths) != 1 or None in lengths:
        raise _error("CONTROL_FLOW_SHAPE_MISMATCH", {"part": "xs", "lengths": repr(sorted(map(str, lengths)))},
                     "xs_need_one_shared_first_axis_or_an_explicit_length")
    n = lengths.pop()

    def make_args(inputs):
        c = unflatten(c_def, inputs[:len(carry)])
        x = unflatten(x_def, inputs[len(carry):]) if xs is not None else None
        return c, x

    specs = [(t.shape, t.dtype) for t in carry] + [(t.shape[1:], t.dtype) for t in xl]

    def body_fn(c, x):
        out = f(c, x)
        if not (isinstance(out, tuple) and len(out) == 2):
            raise _error("CONTROL_FLOW_SHAPE_MISMATCH", {"part": "body", "returned": type(out).__name__}, "scan_body_must_return_carry_and_y")
        return out[0], (() if out[1] is None else out[1])

    body, ids, out_def, scope = _trace_body(body_fn, specs, make_args)
    if out_def[1][0] != c_def:
        raise _shape_mismatch("carry", c_def, out_def[1][0])
    want = [(t.shape, t.dtype) for t in carry]
    if _signature(body, ids[:len(carry)]) != want:
        raise _shape_mismatch("carry", want, _signature(body, ids[:len(carry)]))
    inputs = [t._id for t in carry] + [t._id for t in xl] + list(scope.captures)
    node = g.scan(body, ids, len(carry), len(xl), n, inputs, src)
    final = [Tracer(g, g.output(node, k, list(t.shape), t.dtype)) for k, t in enumerate(carry)]
    ys = [Tracer(g, g.output(node, len(carry) + k, [n] + list(sh), dt)) for k, (sh, dt) in enumerate(_signature(body, ids[len(carry):]))]
    return unflatten(c_def, final), (None if out_def[1][1] == ("tuple", ()) else unflatten(out_def[1][1], ys))


def while_loop(cond_fn, body_fn, init, max_iterations=100000):
    """`state = body_fn(state)` while `cond_fn(state)` is nonzero (python/rg/_core.py while_loop).
    Not differentiable; stops at `max_iterations`."""
    if not _trace_stack:
        return _eagerly(lambda i: while_loop(cond_fn, body_fn, i, max_iterations), init)
    g = _trace_stack[-1]
    src = _where_from()
    carry, c_def = _lift(init, g)
    specs = [(t.shape, t.dtype) for t in carry]
    make_args = lambda inputs: (unflatten(c_def, inputs[:len(carry)]),)
    cond_g, cond_ids, _, c_scope = _trace_body(cond_fn, specs, make_args)
    if len(cond_ids) != 1 or list(cond_g.shape(cond_ids[0])) not in ([], [1]):
        raise _error("CONTROL_FLOW_SHAPE_MISMATCH", {"part": "condition", "outputs": [cond_g.shape(i) for i in cond_ids]},
                     "condition_must_be_a_scalar")
    seen = {o: (tuple(g.shape(o)), g.dtype(o)) for o in c_scope.captures}
    body, ids, out_def, b_scope = _trace_body(body_fn, specs, make_args, seen)
    if out_def != c_def:
        raise _shape_mismatch("state", c_def, out_def)
    if _signature(body, ids) != [(tuple(s), d) for s, d in specs]:
        raise _shape_mismatch("state", specs, _signature(body, ids))
    # The condition takes the same inputs as the body (extra ones unused).
    for outer in b_scope.captures:
        if outer not in c_scope.captures:
            cond_g.input(list(g.shape(outer)), g.dtype(outer), src)
    inputs = [t._id for t in carry] + list(b_scope.captures)
    node = g.while_loop(cond_g, cond_ids[0], body, ids, len(carry), max_iterations, inputs, src)
    return unflatten(c_def, [Tracer(g, g.output(node, k, list(t.shape), t.dtype)) for k, t in enumerate(carry)])


def cond(pred, then_fn, else_fn, *args):
    """Runs only the chosen branch (python/rg/_core.py cond). Differentiable; both branches take
    `*args` and return the same structure, shapes and dtypes."""
    if not _trace_stack:
        return _eagerly(lambda p, *a: cond(p, then_fn, else_fn, *a), pred, *args)
    g = _trace_stack[-1]
    src = _where_from()
    leaves, tdef = _lift(args, g)
    pid = _as_node(g, pred, _first_dtype([pred]) or "float32")
    specs = [(t.shape, t.dtype) for t in leaves]
    make_args = lambda inputs: unflatten(tdef, inputs)
    then_g, then_ids, then_def, t_scope = _trace_body(then_fn, specs, make_args)
    seen = {o: (tuple(g.shape(o)), g.dtype(o)) for o in t_scope.captures}
    else_g, else_ids, else_def, e_scope = _trace_body(else_fn, specs, make_args, seen)
    if then_def != else_def:
        raise _shape_mismatch("branches", then_def, else_def)
    want, got = _signature(then_g, then_ids), _signature(else_g, else_ids)
    if want != got:
        raise _shape_mismatch("branches", want, got)
    for outer in e_scope.captures:
        if outer not in t_scope.captures:
            then_g.input(list(g.shape(outer)), g.dtype(outer), src)
    inputs = [pid] + [t._id for t in leaves] + list(e_scope.captures)
    node = g.cond(then_g, then_ids, else_g, else_ids, inputs, src)
    return unflatten(then_def, [Tracer(g, g.output(node, k, list(sh), dt)) for k, (sh, dt) in enumerate(want)])


def squeeze(x, axis=None):
    if axis is None:
        drop = [i for i, d in enumerate(x.shape) if d == 1]
    else:
        drop = [_axis(x, a) for a in (axis if isinstance(axis, (tuple, list)) else [axis])]
    return x.reshape([d for i, d in enumerate(x.shape) if i not in drop])


# ---- pytrees (dict keys sorted, as rg's _flatten) ----

def flatten(tree):
    if tree is None:
        return [], ("none",)
    if isinstance(tree, (tuple, list)):
        parts = [flatten(x) for x in tree]
        return [l for p in parts for l in p[0]], (type(tree).__name__, tuple(p[1] for p in parts))
    if isinstance(tree, dict):
        keys = sorted(tree)
        parts = [flatten(tree[k]) for k in keys]
        return [l for p in parts for l in p[0]], ("dict", tuple(keys), tuple(p[1] for p in parts))
    return [tree], None


def unflatten(tdef, leaves):
    it = iter(leaves)

    def build(d):
        if d is None:
            return next(it)
        if d[0] == "none":
            return None
        if d[0] == "dict":
            return {k: build(s) for k, s in zip(d[1], d[2])}
        items = [build(s) for s in d[1]]
        return tuple(items) if d[0] == "tuple" else items
    return build(tdef)


def _paths(tdef, prefix):
    if tdef is None:
        return [prefix]
    if tdef[0] == "none":
        return []
    if tdef[0] == "dict":
        return [p for k, s in zip(tdef[1], tdef[2]) for p in _paths(s, f"{prefix}.{k}")]
    return [p for i, s in enumerate(tdef[1]) for p in _paths(s, f"{prefix}.{i}")]


def tree_map(f, t, *rest):
    ls, d = flatten(t)
    others = [flatten(r)[0] for r in rest]
    return unflatten(d, [f(*vals) for vals in zip(ls, *others)])


def tree_leaves(t): return flatten(t)[0]


# ---- transformations ----

def value_and_grad(f, argnums=0, has_aux=False):
    """`(*args) -> (value, grads of args[argnums])`, recorded as gradient nodes on the trace.
    With `has_aux=True`, `f` returns `(scalar, aux)` and the result is `((value, aux), grads)`;
    a tuple `argnums` gives a tuple of gradients (python/rg/_core.py value_and_grad)."""
    many = isinstance(argnums, tuple)
    nums = argnums if many else (argnums,)

    def transformed(*args):
        if not _trace_stack:
            return compile(transformed, args, validate="none")(*args)
        g = _trace_stack[-1]
        src = _where_from()
        call_args = list(args)
        groups = []
        for n in nums:
            leaves, tdef = flatten(args[n])
            dtype = _first_dtype(leaves)
            lifted = [Tracer(g, _as_node(g, l, dtype or "float32")) for l in leaves]
            call_args[n] = unflatten(tdef, lifted)
            groups.append((lifted, tdef))
        out = f(*call_args)
        y, aux = out if has_aux else (out, None)
        if not isinstance(y, (Tensor, Tracer, int, float)):
            raise _error("GRAD_NON_SCALAR", {"returned_type": type(y).__name__}, "function_must_return_a_scalar_tensor")
        yid = _as_node(g, y, _first_dtype([t for lifted, _ in groups for t in lifted]) or "float32")
        grads = []
        for lifted, tdef in groups:
            ids = g.grad(yid, [t._id for t in lifted], src)
            grads.append(unflatten(tdef, [Tracer(g, i) for i in ids]))
        value = Tracer(g, yid)
        return ((value, aux) if has_aux else value), (tuple(grads) if many else grads[0])

    return transformed


def grad(f, argnums=0, has_aux=False):
    """The gradients of `value_and_grad` alone (then `aux`, with `has_aux=True`)."""
    vg = value_and_grad(f, argnums, has_aux)

    def transformed(*args):
        value, grads = vg(*args)
        return (grads, value[1]) if has_aux else grads
    return transformed


def _traced(fn):
    """`fn` on the current trace, or compiled and run once on concrete inputs outside one."""
    def wrapped(*args):
        return fn(*args) if _trace_stack else compile(fn, args, validate="none")(*args)
    return wrapped


def jvp(f, primals, tangents):
    """Forward-mode `(f(*primals), J @ tangents)` from two reverse passes: the gradient of
    <f(p), u> with respect to p is J^T u; its inner product with the tangents is linear in u,
    and differentiating that with respect to u gives J t."""

    def body(primals, tangents):
        g = _trace_stack[-1]
        ys = f(*primals)
        u = Tracer(g, _as_node(g, zeros_like(ys), ys.dtype))
        jt_u = grad(lambda ps: (f(*ps) * u).sum())(tuple(primals))
        dot = sum((a * b).sum() for a, b in zip(flatten(jt_u)[0], flatten(tuple(tangents))[0]))
        return ys, Tracer(g, g.grad(dot._id, [u._id], _where_from())[0])
    return _traced(body)(tuple(primals), tuple(tangents))


def hessian(f):
    """Dense Hessian of a scalar function of one tensor, one reverse pass per row of the
    flattened gradient; its size is the square of the input's."""

    def body(x):
        n = grad(f)(x).reshape(-1).shape[0]
        rows = [grad(lambda v, i=i: grad(f)(v).reshape(-1)[i])(x).reshape(-1) for i in range(n)]
        return stack(rows).reshape(tuple(x.shape) + tuple(x.shape))
    return _traced(body)


def custom_vjp(f, bwd):
    """`f` with a hand-written gradient: `bwd(args, y, cotangent)` returns one gradient per
    argument, each of its argument's shape and dtype. The graph records `f`'s output with the
    rule in place of differentiating through `f`."""

    def wrapped(*args):
        if not _trace_stack:
            return _traced(wrapped)(*args)
        g = _trace_stack[-1]
        src = _where_from()
        dtype = _first_dtype(args)
        lifted = [Tracer(g, _as_node(g, a, dtype or "float32")) for a in args]
        y = f(*lifted)
        ct = Tracer(g, g.placeholder(list(y.shape), y.dtype))
        grads = bwd(tuple(lifted), y, ct)
        if len(grads) != len(lifted):
            raise _error("CUSTOM_VJP_MISMATCH", {"inputs": len(lifted), "gradients": len(grads)}, "rule_must_return_one_gradient_per_input")
        rules = []
        for a, c in zip(lifted, grads):
            c = c if isinstance(c, Tracer) else Tracer(g, _as_node(g, c, a.dtype))
            if c.shape != a.shape or c.dtype != a.dtype:
                raise _error("CUSTOM_VJP_MISMATCH", {"input_shape": a.shape, "gradient_shape": c.shape, "input_dtype": a.dtype,
                                                     "gradient_dtype": c.dtype}, "gradient_must_match_its_input")
            rules.append((a._id, c._id))
        return Tracer(g, g.custom(y._id, ct._id, rules, src))
    return wrapped


def devices():
    """Device names `compile(device=...)` accepts on the selected engine module."""
    return native().available_devices()


class Report(dict):
    """A compile, check or run report: plain JSON data that prints as indented JSON."""

    def __str__(self): return json.dumps(self, indent=2, ensure_ascii=False)

    @property
    def ok(self): return self.get("status") != "validation_failed"


class Compiled:
    """An executable plan plus its compile report."""

    def __init__(self, handle, in_def, in_sig, out_def, n_out, extras=()):
        self._n = handle
        self._in_def = in_def
        self._in_sig = in_sig
        self._out_def = out_def
        self._n_out = n_out
        self._extras = list(extras)  # names of the observe=True instrument outputs after the outputs
        self.report = Report(json.loads(handle.report_json))

    def _inputs(self, args):
        leaves, tdef = flatten(args)
        ts = [tensor(l) for l in leaves]
        if tdef != self._in_def or [(t.shape, t.dtype) for t in ts] != self._in_sig:
            raise _error("INPUT_SIGNATURE_MISMATCH", {"expected": repr(self._in_sig), "recompile_required": True}, "input_signature_changed")
        return [t._t for t in ts]

    def __call__(self, *args):
        out = self._n.call(self._inputs(args))
        return unflatten(self._out_def, [Tensor(t) for t in out[:self._n_out]])

    def check(self, *args):
        """Runs the instrumented reference graph on these inputs and returns its diagnostics."""
        return Report(json.loads(self._n.check(self._inputs(args))))

    def profile(self, *args, repeats=5):
        """Per-operation timing of the optimized plan on these inputs, slowest first."""
        return Report(json.loads(self._n.profile(self._inputs(args), repeats)))

    def plan_blob(self):
        return self._n.plan_blob()


def _instruments(g, in_def, inputs, out_leaves, out_def):
    """observe=True statistics as (name, node) pairs (python/rg/_core.py _instruments): per
    differentiated input the gradient's norm, largest magnitude and zero fraction, the global
    gradient norm, and, when the step returns its new state, each parameter's relative update."""
    names = {t._id: n for t, n in zip(inputs, _paths(in_def, ""))}
    latest = {}
    for _, wrt, grad_id in g.grad_records():
        if wrt in names:
            latest[wrt] = grad_id
    extras, total = [], 0.0
    for wrt, grad_id in latest.items():
        name = names[wrt].lstrip(".")
        name = name[2:] if name.startswith("0.") else name
        gr = Tracer(g, grad_id)
        squared = (gr * gr).sum()
        total = total + squared
        extras.append((f"grad.{name}.norm", squared.sqrt()))
        extras.append((f"grad.{name}.max", abs(gr).max()))
        extras.append((f"grad.{name}.zero", (0.0 >= abs(gr)).sum() / max(1, gr.size)))
    if latest:
        extras.append(("grad.global_norm", total.sqrt()))
    state_def = in_def[1][0] if in_def and in_def[0] == "tuple" and in_def[1] else None
    n_state = len(_paths(state_def, "")) if state_def is not None else 0
    returns_state = state_def is not None and (out_def == state_def or (out_def is not None and out_def[0] == "tuple" and len(out_def[1]) == 2
                                                                          and out_def[1][0] == state_def))
    if returns_state:
        for old, new in zip(inputs[:n_state], out_leaves[:n_state]):
            if old._id in latest and isinstance(new, Tracer):
                name = names[old._id].lstrip(".")
                name = name[2:] if name.startswith("0.") else name
                d = new - old
                size_now = (old * old).sum().sqrt()
                # A parameter at exactly zero records 0, not a huge ratio (and not NaN, which
                # would stop `run`).
                extras.append((f"update.{name}", where(size_now > 0.0, (d * d).sum().sqrt() / where(size_now > 0.0, size_now, 1.0), 0.0)))
    return [(n, _as_node(g, v, "float32")) for n, v in extras]


def compile(fn, example_inputs, validate="standard", device=None, optimize="search-linear", observe=False):
    """Traces `fn(*example_inputs)` and compiles it for `device` (default: the module's first).
    `observe=True` adds per-parameter gradient and update statistics as extra outputs, computed
    in the plan on the device; `run` records them in its history."""
    if not isinstance(example_inputs, tuple):
        example_inputs = (example_inputs,)
    leaves, in_def = flatten(example_inputs)
    leaves = [tensor(l) for l in leaves]
    g = native().Graph()
    src = _where_from()
    tracers = [Tracer(g, g.input(list(t.shape), t.dtype, src)) for t in leaves]
    _trace_stack.append(g)
    try:
        out = fn(*unflatten(in_def, tracers))
        out_leaves, out_def = flatten(out)
        dtype = _first_dtype(leaves) or "float32"
        out_ids = [_as_node(g, l, dtype) for l in out_leaves]
        extras = _instruments(g, in_def, tracers, out_leaves, out_def) if observe else []
    finally:
        _trace_stack.pop()
    handle = native().compile(g, out_ids + [i for _, i in extras], [t._t for t in leaves], validate, device or default_device(), optimize)
    return Compiled(handle, in_def, [(t.shape, t.dtype) for t in leaves], out_def, len(out_ids), [n for n, _ in extras])


class RunResult:
    """Outcome of `run`: `state`, the last `aux`, `history` (each scalar aux per step), `status`,
    `steps` run of `requested_steps`, `nonfinite_step`, `elapsed` device seconds."""

    def __init__(self, **kw):
        self.__dict__.update(kw)

    def __repr__(self):
        return f"RunResult(status={self.status!r}, steps={self.steps}, elapsed={self.elapsed:.4f}s)"


def _mismatch(k, want, got):
    return _error("INPUT_SIGNATURE_MISMATCH", {"input_index": k, "expected": repr(want), "actual": repr(got), "recompile_required": True},
                  "input_signature_changed")


def _batch(compiled, batch, n_state):
    ts = [tensor(l) for l in flatten(batch)[0]]
    for k, t in enumerate(ts):
        want = compiled._in_sig[n_state + k]
        if (t.shape, t.dtype) != want:
            raise _mismatch(n_state + k, want, (t.shape, t.dtype))
    return [t._t for t in ts]


def _run_contract(compiled, state, data):
    """Checks `state` and `data` against the compiled step (python/rg/_core.py _setup): the step
    takes `state` or `(state, data)` and returns `state` or `(state, aux)`; `data` is one batch,
    a list of batches, or an iterator of batches."""
    arity = len(compiled._in_def[1])
    if arity not in (1, 2):
        raise _error("STATE_CONTRACT_VIOLATION", {"arity": arity}, "step_must_take_state_or_state_and_data")
    leaves, state_def = flatten(state)
    leaves = [tensor(l) for l in leaves]
    if state_def != compiled._in_def[1][0]:
        raise _error("INPUT_SIGNATURE_MISMATCH", {"expected_structure": repr(compiled._in_def[1][0]), "actual_structure": repr(state_def),
                                                  "recompile_required": True}, "state_structure_changed")
    for k, t in enumerate(leaves):
        if (t.shape, t.dtype) != compiled._in_sig[k]:
            raise _mismatch(k, compiled._in_sig[k], (t.shape, t.dtype))
    d = compiled._out_def
    if d == state_def:
        aux_def, has_aux = None, False
    elif d is not None and d[0] == "tuple" and len(d[1]) == 2 and d[1][0] == state_def:
        aux_def, has_aux = d[1][1], True
    else:
        raise _error("STATE_CONTRACT_VIOLATION", {"state_structure": repr(state_def), "output_structure": repr(d)},
                     "step_must_return_new_state_or_new_state_and_aux")
    iterator, batches = None, []
    if arity == 2:
        data_def = compiled._in_def[1][1]
        if hasattr(data, "__next__"):
            iterator = data
        elif flatten(data)[1] == data_def:
            batches = [_batch(compiled, data, len(leaves))]
        elif isinstance(data, (list, tuple)) and data and all(flatten(b)[1] == data_def for b in data):
            batches = [_batch(compiled, b, len(leaves)) for b in data]
        else:
            raise _error("INPUT_SIGNATURE_MISMATCH", {"expected_batch_structure": repr(data_def), "actual_structure": repr(flatten(data)[1]),
                                                      "recompile_required": True}, "data_structure_changed")
    return leaves, state_def, has_aux, aux_def, iterator, batches


def run(compiled, state, data=None, steps=1, callback=None, every=None):
    """Iterates `state = step(state[, data])` in the engine, with no Python between steps.

    Batches in a list are cycled. With `every`, or an iterator (pulled 256 batches at a time by
    default), the run goes in chunks of that many steps, and `callback(result)` after each chunk
    may return False to stop. A non-finite step ends the run (status "stopped_nonfinite")."""
    if not compiled.report.ok:
        d = next(x for x in compiled.report["diagnostics"] if x["severity"] == "error")
        e = DiagnosticError(json.dumps(d))
        e.diagnostic = d
        raise e
    leaves, state_def, has_aux, aux_def, iterator, batches = _run_contract(compiled, state, data)
    n_state = len(leaves)
    aux_names = _paths(aux_def, "aux") if has_aux else []
    shapes = compiled._n.output_shapes
    scalar = [k for k in range(n_state, n_state + len(aux_names)) if all(x == 1 for x in shapes[k])]
    names = {k: aux_names[k - n_state] for k in scalar}
    for j, name in enumerate(compiled._extras):
        scalar.append(compiled._n_out + j)
        names[compiled._n_out + j] = name
    state_map = [(k, k) for k in range(n_state)]
    data_inputs = list(range(n_state, len(compiled._in_sig)))
    chunk = every if every else (256 if iterator is not None else steps)
    chunk = max(1, min(chunk, steps)) if steps else 1

    current = [t._t for t in leaves]
    history = {names[k]: [] for k in scalar}
    done, elapsed, bad_step, aux, stopped = 0, 0.0, None, None, False
    last = (current, batches[:1], 0, 0)  # the latest chunk's start state, batches, steps and offset
    result = None
    while done < steps and bad_step is None and not stopped:
        n = min(chunk, steps - done)
        if iterator is not None:
            part = []
            for _ in range(n):
                try:
                    part.append(_batch(compiled, next(iterator), n_state))
                except StopIteration:
                    break
            if not part:
                break
            n = len(part)
        else:
            at = done % len(batches) if batches else 0
            part = batches[at:] + batches[:at]
        new_state, outputs, hist, ran, bad, seconds = compiled._n.run(state_map, data_inputs, scalar, current, part, n)
        last = (current, part, ran, done)
        for k, h in zip(scalar, hist):
            history[names[k]].extend(h)
        done += ran
        elapsed += seconds
        bad_step = None if bad is None else done - ran + bad
        if bad_step is None and not all(t.is_finite() for t in new_state):
            bad_step = done - 1
        current = new_state
        if has_aux and outputs:
            aux = unflatten(aux_def, [Tensor(t) for t in outputs[n_state:compiled._n_out]])
        result = RunResult(status="stopped_nonfinite" if bad_step is not None else "running", state=unflatten(state_def, [Tensor(t) for t in current]),
                           aux=aux, history=history, steps=done, requested_steps=steps, nonfinite_step=bad_step, elapsed=elapsed,
                           compiled=compiled, _replay=(state_map, data_inputs, scalar, state_def) + last)
        if callback is not None and bad_step is None and callback(result) is False:
            stopped = True
    if result is None:
        return RunResult(status="completed", state=unflatten(state_def, [Tensor(t) for t in current]), aux=None, history=history, steps=0,
                         requested_steps=steps, nonfinite_step=None, elapsed=0.0, compiled=compiled,
                         _replay=(state_map, data_inputs, scalar, state_def) + last)
    if bad_step is None:
        result.status = "stopped_by_callback" if stopped else "completed"
    return result


def _json_num(x):
    if x != x:
        return "nan"
    if x in (float("inf"), float("-inf")):
        return "inf" if x > 0 else "-inf"
    return x


def inspect(target):
    """Explains a Compiled (its report) or a RunResult. A run that stopped on a non-finite value
    is replayed from the start of its last chunk (every chunk ends with a finiteness check, so it
    holds the failure) to the first bad step, whose inputs are checked node by node."""
    if isinstance(target, Compiled):
        return target.report
    state_map, data_inputs, scalar, state_def, start, part, ran, offset = target._replay
    c = target.compiled
    out = Report(status=target.status, run={"steps": target.steps, "requested_steps": target.requested_steps, "elapsed_seconds": target.elapsed},
                 history={k: {"first": _json_num(h[0]), "last": _json_num(h[-1]), "min": _json_num(min(h)), "max": _json_num(max(h))}
                          for k, h in target.history.items() if h},
                 diagnostics=[])
    if target.status != "stopped_nonfinite":
        batch = part[(ran - 1) % len(part)] if part and ran else (part[0] if part else [])
        checked = json.loads(c._n.check([t._t for t in flatten(target.state)[0]] + batch))
        out["gradients"] = checked["gradients"]
        out["diagnostics"] = checked["diagnostics"]
        return out
    found = c._n.replay(state_map, data_inputs, scalar, start, part, ran)
    if found is None:
        out["status"] = "not_reproduced"
        out["diagnostics"] = [{"code": "REPLAY_DID_NOT_REPRODUCE", "severity": "warning", "diagnosis": {"cause": "unknown", "certainty": "unknown"}}]
        return out
    step, batch_index, before = found
    checked = json.loads(c._n.check(before + (part[batch_index] if part else [])))
    out["status"] = "nonfinite_detected"
    out["diagnostics"] = checked["diagnostics"]
    if not any(d.get("severity") == "error" for d in out["diagnostics"]):
        # The unoptimized reference graph can round differently from the plan near overflow.
        out["diagnostics"].append({"code": "NONFINITE_NOT_LOCALIZED", "severity": "warning",
                                   "diagnosis": {"cause": "reference_run_stayed_finite", "certainty": "unknown"}})
    out["repro"] = {"step": offset + step, "batch_index": batch_index if part else None, "validate": c.report["repro"]["level"],
                    "seed": c.report["repro"]["seed"]}
    return out
