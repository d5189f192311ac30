"""Transformations recorded into graphs (gradients, custom gradient rules, control flow) and the
compile / run cycle over the engine module.

* `value_and_grad` records one gradient node group per differentiated argument (the engine's
  autodiff runs on the graph at compile time).
* `scan`, `while_loop` and `cond` record their bodies as separate graphs. A body reads values of
  the enclosing program through extra inputs, created in first-use order; a loop's condition
  and body, and a branch pair, share those extra inputs.
* `compile` records a step function on example inputs and asks the engine for a plan on a
  device; `run` iterates `state = step(state[, data])` inside the engine, with no Python between
  steps, and collects each scalar output per step.
"""
import json

from .trees import flatten, leaf_names, unflatten
from .tracing import (Array, Frame, Tensor, Traced, caller, default_device, diagnostic, dtype_of, native, record, recording, tensor,
                      where, DiagnosticError)


def _lift(frame, tree):
    """The leaves of `tree` as nodes of `frame` (concrete leaves become constants)."""
    leaves, shape = flatten(tree)
    dt = dtype_of(leaves) or "float32"
    return [frame.wrap(frame.node(v, dt)) for v in leaves], shape


def _eager(fn, *args):
    """A transformation used outside any recording: compile the call and run it once."""
    return compile(fn, args, validate="none")(*args)


# ---------------------------------------------------------------------------------------------
# Gradients
# ---------------------------------------------------------------------------------------------

def value_and_grad(f, argnums=0, has_aux=False):
    """`(*args) -> (value, gradients of args[argnums])` for a scalar-valued `f`; a tuple
    `argnums` gives a tuple of gradient trees. With `has_aux`, `f` returns `(value, aux)` and the
    first result is `(value, aux)`."""
    many = isinstance(argnums, tuple)
    which = argnums if many else (argnums,)

    def transformed(*args):
        frame = recording()
        if frame is None:
            return _eager(transformed, *args)
        call, groups = list(args), []
        for n in which:
            lifted, shape = _lift(frame, args[n])
            call[n] = unflatten(shape, lifted)
            groups.append((lifted, shape))
        result = f(*call)
        value, aux = result if has_aux else (result, None)
        if not isinstance(value, (Array, int, float)):
            raise diagnostic("GRAD_NON_SCALAR", {"returned_type": type(value).__name__}, "function_must_return_a_scalar_tensor")
        vid = frame.node(value, dtype_of([t for lifted, _ in groups for t in lifted]) or "float32")
        src = caller()
        grads = [unflatten(shape, [frame.wrap(i) for i in frame.graph.grad(vid, [t.id for t in lifted], src)]) for lifted, shape in groups]
        v = frame.wrap(vid)
        return ((v, aux) if has_aux else v), (tuple(grads) if many else grads[0])
    return transformed


def grad(f, argnums=0, has_aux=False):
    vg = value_and_grad(f, argnums, has_aux)

    def transformed(*args):
        value, grads = vg(*args)
        return (grads, value[1]) if has_aux else grads
    return transformed


def custom_vjp(f, rule):
    """`f` whose gradient is `rule(args, y, cotangent)`, one gradient per argument of that
    argument's shape and dtype, instead of the derivative of `f`'s own ops."""

    def wrapped(*args):
        frame = recording()
        if frame is None:
            return _eager(wrapped, *args)
        dt = dtype_of(args) or "float32"
        xs = [frame.wrap(frame.node(a, dt)) for a in args]
        y = f(*xs)
        ct = frame.wrap(frame.graph.placeholder(list(y.shape), y.dtype))
        gs = rule(tuple(xs), y, ct)
        if len(gs) != len(xs):
            raise diagnostic("CUSTOM_VJP_MISMATCH", {"inputs": len(xs), "gradients": len(gs)}, "rule_must_return_one_gradient_per_input")
        pairs = []
        for x, g in zip(xs, gs):
            g = g if isinstance(g, Traced) else frame.wrap(frame.node(g, x.dtype))
            if g.shape != x.shape or g.dtype != x.dtype:
                raise diagnostic("CUSTOM_VJP_MISMATCH", {"input_shape": x.shape, "gradient_shape": g.shape, "input_dtype": x.dtype,
                                                         "gradient_dtype": g.dtype}, "gradient_must_match_its_input")
            pairs.append((x.id, g.id))
        return frame.wrap(frame.graph.custom(y.id, ct.id, pairs, caller()))
    return wrapped


# ---------------------------------------------------------------------------------------------
# Control flow
# ---------------------------------------------------------------------------------------------

class _Body:
    """A recorded body graph: `outputs` node ids, `shape` of the output tree, and the frame
    whose `captured` lists the enclosing nodes it reads."""

    def __init__(self, parent, fn, specs, to_args, shared=None):
        self.graph = native().Graph()
        src = caller()
        self.frame = Frame(self.graph, parent)
        inputs = [self.frame.wrap(self.graph.input(list(sh), dt, src)) for sh, dt in specs]
        # Enclosing values that an earlier body of the same construct captured come next, in
        # that body's order, so both bodies agree on their extra inputs.
        for outer, (sh, dt) in (shared or {}).items():
            self.frame.captured[outer] = self.graph.input(list(sh), dt, src)
        with record(self.frame):
            out = fn(*to_args(inputs))
            leaves, self.shape = flatten(out)
            dt = dtype_of(leaves) or "float32"
            self.outputs = [self.frame.node(v, dt) for v in leaves]

    def signature(self, ids=None):
        ids = self.outputs if ids is None else ids
        return [(tuple(self.graph.shape(i)), self.graph.dtype(i)) for i in ids]

    def shared_with(self, parent_graph):
        """This body's captures as (shape, dtype) specs, to seed a sibling body."""
        return {o: (tuple(parent_graph.shape(o)), parent_graph.dtype(o)) for o in self.frame.captured}


def _mismatch(part, want, got):
    return diagnostic("CONTROL_FLOW_SHAPE_MISMATCH", {"part": part, "expected": repr(want), "got": repr(got)}, f"{part}_structure_or_shape_changed")


def scan(f, init, xs=None, length=None):
    """`carry, y = f(carry, x)` over the leading axis of `xs` (or `length` times with x = None)
    as one graph node. Returns the final carry and the ys stacked along a new leading axis."""
    frame = recording()
    if frame is None:
        if xs is None:
            return _eager(lambda c: scan(f, c, None, length), init)
        return _eager(lambda c, x: scan(f, c, x, length), init, xs)
    carry, c_shape = _lift(frame, init)
    xl, x_shape = _lift(frame, xs) if xs is not None else ([], None)
    lengths = {t.shape[0] if t.ndim else None for t in xl} | ({length} if length is not None else set())
    if len(lengths) != 1 or None in lengths:
        raise diagnostic("CONTROL_FLOW_SHAPE_MISMATCH", {"part": "xs", "lengths": repr(sorted(map(str, lengths)))},
                         "xs_need_one_shared_first_axis_or_an_explicit_length")
    n = lengths.pop()
    nc = len(carry)

    def body_fn(c, x):
        out = f(c, x)
        if not (isinstance(out, tuple) and len(out) == 2):
            raise diagnostic("CONTROL_FLOW_SHAPE_MISMATCH", {"part": "body", "returned": type(out).__name__}, "scan_body_must_return_carry_and_y")
        return out[0], (() if out[1] is None else out[1])

    def to_args(inputs):
        return unflatten(c_shape, inputs[:nc]), (unflatten(x_shape, inputs[nc:]) if xs is not None else None)

    specs = [(t.shape, t.dtype) for t in carry] + [(t.shape[1:], t.dtype) for t in xl]
    body = _Body(frame, body_fn, specs, to_args)
    carry_out_shape, ys_shape = body.shape.children
    if carry_out_shape != c_shape:
        raise _mismatch("carry", c_shape, carry_out_shape)
    want = [(t.shape, t.dtype) for t in carry]
    if body.signature(body.outputs[:nc]) != want:
        raise _mismatch("carry", want, body.signature(body.outputs[:nc]))
    g = frame.graph
    node = g.scan(body.graph, body.outputs, nc, len(xl), n, [t.id for t in carry] + [t.id for t in xl] + list(body.frame.captured), caller())
    final = [frame.wrap(g.output(node, k, list(t.shape), t.dtype)) for k, t in enumerate(carry)]
    ys = [frame.wrap(g.output(node, nc + k, [n] + list(sh), dt)) for k, (sh, dt) in enumerate(body.signature(body.outputs[nc:]))]
    no_ys = ys_shape.kind == "tuple" and not ys_shape.children
    return unflatten(c_shape, final), (None if no_ys else unflatten(ys_shape, ys))


def while_loop(cond_fn, body_fn, init, max_iterations=100000):
    """`state = body_fn(state)` while `cond_fn(state)` is nonzero, at most `max_iterations`
    times, as one graph node (not differentiable)."""
    frame = recording()
    if frame is None:
        return _eager(lambda s: while_loop(cond_fn, body_fn, s, max_iterations), init)
    carry, c_shape = _lift(frame, init)
    specs = [(t.shape, t.dtype) for t in carry]
    to_args = lambda inputs: (unflatten(c_shape, inputs[:len(carry)]),)
    test = _Body(frame, cond_fn, specs, to_args)
    if len(test.outputs) != 1 or list(test.graph.shape(test.outputs[0])) not in ([], [1]):
        raise diagnostic("CONTROL_FLOW_SHAPE_MISMATCH", {"part": "condition", "outputs": [test.graph.shape(i) for i in test.outputs]},
                         "condition_must_be_a_scalar")
    body = _Body(frame, body_fn, specs, to_args, shared=test.shared_with(frame.graph))
    if body.shape != c_shape:
        raise _mismatch("state", c_shape, body.shape)
    if body.signature() != [(tuple(s), d) for s, d in specs]:
        raise _mismatch("state", specs, body.signature())
    g = frame.graph
    for outer in body.frame.captured:
        if outer not in test.frame.captured:
            test.graph.input(list(g.shape(outer)), g.dtype(outer), caller())
    node = g.while_loop(test.graph, test.outputs[0], body.graph, body.outputs, len(carry), max_iterations,
                        [t.id for t in carry] + list(body.frame.captured), caller())
    return unflatten(c_shape, [frame.wrap(g.output(node, k, list(t.shape), t.dtype)) for k, t in enumerate(carry)])


def cond(pred, then_fn, else_fn, *args):
    """`then_fn(*args)` if `pred` is nonzero else `else_fn(*args)`; only the chosen branch runs.
    Both branches return the same structure, shapes and dtypes. Differentiable."""
    frame = recording()
    if frame is None:
        return _eager(lambda p, *a: cond(p, then_fn, else_fn, *a), pred, *args)
    leaves, a_shape = _lift(frame, args)
    pid = frame.node(pred, dtype_of([pred]) or "float32")
    specs = [(t.shape, t.dtype) for t in leaves]
    to_args = lambda inputs: unflatten(a_shape, inputs)
    then_b = _Body(frame, then_fn, specs, to_args)
    else_b = _Body(frame, else_fn, specs, to_args, shared=then_b.shared_with(frame.graph))
    if then_b.shape != else_b.shape:
        raise _mismatch("branches", then_b.shape, else_b.shape)
    if then_b.signature() != else_b.signature():
        raise _mismatch("branches", then_b.signature(), else_b.signature())
    g = frame.graph
    for outer in else_b.frame.captured:
        if outer not in then_b.frame.captured:
            then_b.graph.input(list(g.shape(outer)), g.dtype(outer), caller())
    node = g.cond(then_b.graph, then_b.outputs, else_b.graph, else_b.outputs, [pid] + [t.id for t in leaves] + list(else_b.frame.captured), caller())
    return unflatten(then_b.shape, [frame.wrap(g.output(node, k, list(sh), dt)) for k, (sh, dt) in enumerate(then_b.signature())])


# ---------------------------------------------------------------------------------------------
# Compile
# ---------------------------------------------------------------------------------------------

class Report(dict):
    """A compile, check or profile report (the engine's JSON), printed indented."""

    def __str__(self):
        return json.dumps(self, indent=2, ensure_ascii=False)

    @property
    def ok(self):
        return self.get("status") != "validation_failed"


def _strip_arg(name):
    """'0.params.w' -> 'params.w': names of the step's first argument lose its position."""
    return name[2:] if name.startswith("0.") else name


def _observed(frame, in_shape, inputs, out_leaves, out_shape):
    """observe=True statistics as (name, node id) pairs: per differentiated input its gradient's
    L2 norm, largest magnitude and fraction of zeros, the norm of all gradients together, and,
    when the step returns its new state, each updated parameter's relative change."""
    g = frame.graph
    names = {t.id: _strip_arg(n) for t, n in zip(inputs, leaf_names(in_shape))}
    latest = {}
    for _, wrt, gid in g.grad_records():
        if wrt in names:
            latest[wrt] = gid
    stats, total = [], 0.0
    for wrt, gid in latest.items():
        gr = frame.wrap(gid)
        squared = (gr * gr).sum()
        total = total + squared
        stats.append((f"grad.{names[wrt]}.norm", squared.sqrt()))
        stats.append((f"grad.{names[wrt]}.max", abs(gr).max()))
        stats.append((f"grad.{names[wrt]}.zero", (0.0 >= abs(gr)).sum() / max(1, gr.size)))
    if latest:
        stats.append(("grad.global_norm", total.sqrt()))
    state_shape = in_shape.children[0] if in_shape.kind == "tuple" and in_shape.children else None
    returns_state = state_shape is not None and (out_shape == state_shape or (
        out_shape.kind == "tuple" and len(out_shape.children) == 2 and out_shape.children[0] == state_shape))
    if returns_state:
        for old, new in zip(inputs[:state_shape.n_leaves], out_leaves[:state_shape.n_leaves]):
            if old.id in latest and isinstance(new, Traced):
                step = new - old
                size = (old * old).sum().sqrt()
                # A parameter at zero records 0 rather than an unbounded (or NaN) ratio.
                stats.append((f"update.{names[old.id]}", where(size > 0.0, (step * step).sum().sqrt() / where(size > 0.0, size, 1.0), 0.0)))
    return [(n, frame.node(v, "float32")) for n, v in stats]


class Compiled:
    """A compiled step: the engine's handle `_n` and the step's input and output structure."""

    def __init__(self, handle, in_shape, in_sig, out_shape, n_out, observed=()):
        self._n = handle
        self._in_shape, self._in_sig = in_shape, in_sig
        self._out_shape, self._n_out = out_shape, n_out
        self._observed = list(observed)
        self.report = Report(json.loads(handle.report_json))

    def _handles(self, args):
        leaves, shape = flatten(args)
        ts = [tensor(v) for v in leaves]
        if shape != self._in_shape or [(t.shape, t.dtype) for t in ts] != self._in_sig:
            raise diagnostic("INPUT_SIGNATURE_MISMATCH", {"expected": repr(self._in_sig), "recompile_required": True}, "input_signature_changed")
        return [t._t for t in ts]

    def __call__(self, *args):
        outs = self._n.call(self._handles(args))
        return unflatten(self._out_shape, [Tensor(t) for t in outs[:self._n_out]])

    def check(self, *args):
        """The engine's instrumented check of the unoptimised graph on these inputs."""
        return Report(json.loads(self._n.check(self._handles(args))))

    def profile(self, *args, repeats=5):
        return Report(json.loads(self._n.profile(self._handles(args), repeats)))

    def plan_blob(self):
        return self._n.plan_blob()


def compile(fn, example_inputs, validate="standard", device=None, optimize="search-linear", observe=False):
    """Records `fn(*example_inputs)` and compiles it for `device` (default: the engine's first
    device). `observe=True` appends the gradient and update statistics as extra outputs,
    computed in the plan; `run` records them per step."""
    if not isinstance(example_inputs, tuple):
        example_inputs = (example_inputs,)
    leaves, in_shape = flatten(example_inputs)
    leaves = [tensor(v) for v in leaves]
    frame = Frame(native().Graph())
    src = caller()
    inputs = [frame.wrap(frame.graph.input(list(t.shape), t.dtype, src)) for t in leaves]
    with record(frame):
        out = fn(*unflatten(in_shape, inputs))
        out_leaves, out_shape = flatten(out)
        dt = dtype_of(leaves) or "float32"
        out_ids = [frame.node(v, dt) for v in out_leaves]
        observed = _observed(frame, in_shape, inputs, out_leaves, out_shape) if observe else []
    handle = native().compile(frame.graph, out_ids + [i for _, i in observed], [t._t for t in leaves], validate, device or default_device(), optimize)
    return Compiled(handle, in_shape, [(t.shape, t.dtype) for t in leaves], out_shape, len(out_ids), [n for n, _ in observed])


# ---------------------------------------------------------------------------------------------
# Run
# ---------------------------------------------------------------------------------------------

class RunResult:
    """What `run` returns: `state`, the last `aux`, `history` (scalar outputs per step, by
    name), `status` ("completed", "stopped_nonfinite", "stopped_by_callback"), `steps` done of
    `requested_steps`, `nonfinite_step`, and `elapsed` engine seconds."""

    def __init__(self, **fields):
        self.__dict__.update(fields)

    def __repr__(self):
        return f"RunResult(status={self.status!r}, steps={self.steps}, elapsed={self.elapsed:.4f}s)"


def _signature_error(k, want, got):
    return diagnostic("INPUT_SIGNATURE_MISMATCH", {"input_index": k, "expected": repr(want), "actual": repr(got), "recompile_required": True},
                      "input_signature_changed")


class _Loop:
    """The step's contract for `run`: it takes `state` or `(state, data)` and returns `state` or
    `(state, aux)`; `data` is one batch, a list of batches (cycled) or an iterator."""

    def __init__(self, compiled, state, data):
        self.c = compiled
        args = compiled._in_shape.children
        if len(args) not in (1, 2):
            raise diagnostic("STATE_CONTRACT_VIOLATION", {"arity": len(args)}, "step_must_take_state_or_state_and_data")
        leaves, self.state_shape = flatten(state)
        self.state = [tensor(v) for v in leaves]
        if self.state_shape != args[0]:
            raise diagnostic("INPUT_SIGNATURE_MISMATCH", {"expected_structure": repr(args[0]), "actual_structure": repr(self.state_shape),
                                                          "recompile_required": True}, "state_structure_changed")
        for k, t in enumerate(self.state):
            if (t.shape, t.dtype) != compiled._in_sig[k]:
                raise _signature_error(k, compiled._in_sig[k], (t.shape, t.dtype))
        out = compiled._out_shape
        if out == self.state_shape:
            self.aux_shape = None
        elif out.kind == "tuple" and len(out.children) == 2 and out.children[0] == self.state_shape:
            self.aux_shape = out.children[1]
        else:
            raise diagnostic("STATE_CONTRACT_VIOLATION", {"state_structure": repr(self.state_shape), "output_structure": repr(out)},
                             "step_must_return_new_state_or_new_state_and_aux")
        self.n_state = len(self.state)
        self.iterator, self.batches = None, []
        if len(args) == 2:
            data_shape = args[1]
            if hasattr(data, "__next__"):
                self.iterator = data
            elif flatten(data)[1] == data_shape:
                self.batches = [self.batch(data)]
            elif isinstance(data, (list, tuple)) and data and all(flatten(b)[1] == data_shape for b in data):
                self.batches = [self.batch(b) for b in data]
            else:
                raise diagnostic("INPUT_SIGNATURE_MISMATCH", {"expected_batch_structure": repr(data_shape), "actual_structure": repr(flatten(data)[1]),
                                                              "recompile_required": True}, "data_structure_changed")
        # History: every scalar aux output, then the observe=True statistics.
        aux_names = leaf_names(self.aux_shape, "aux") if self.aux_shape is not None else []
        shapes = compiled._n.output_shapes
        self.history = [(k, aux_names[k - self.n_state]) for k in range(self.n_state, self.n_state + len(aux_names))
                        if all(d == 1 for d in shapes[k])]
        self.history += [(compiled._n_out + j, name) for j, name in enumerate(compiled._observed)]

    def batch(self, b):
        ts = [tensor(v) for v in flatten(b)[0]]
        for k, t in enumerate(ts):
            want = self.c._in_sig[self.n_state + k]
            if (t.shape, t.dtype) != want:
                raise _signature_error(self.n_state + k, want, (t.shape, t.dtype))
        return [t._t for t in ts]

    def aux(self, outputs):
        if self.aux_shape is None or not outputs:
            return None
        return unflatten(self.aux_shape, [Tensor(t) for t in outputs[self.n_state:self.c._n_out]])


def run(compiled, state, data=None, steps=1, callback=None, every=None):
    """Iterates `state = step(state[, data])` in the engine for `steps` steps.

    A list of batches is cycled. With `every` (or an iterator, pulled 256 batches at a time), the
    run goes in chunks of that many steps and `callback(result)` after each chunk may return
    False to stop. A step that leaves a non-finite value ends the run."""
    if not compiled.report.ok:
        d = next(x for x in compiled.report["diagnostics"] if x["severity"] == "error")
        err = DiagnosticError(json.dumps(d))
        err.diagnostic = d
        raise err
    loop = _Loop(compiled, state, data)
    state_map = [(k, k) for k in range(loop.n_state)]
    data_inputs = list(range(loop.n_state, len(compiled._in_sig)))
    hist_ids = [k for k, _ in loop.history]
    history = {name: [] for _, name in loop.history}
    chunk = every or (256 if loop.iterator is not None else steps)
    chunk = max(1, min(chunk, steps)) if steps else 1
    current = [t._t for t in loop.state]
    done, elapsed, bad, aux, status = 0, 0.0, None, None, "completed"
    while done < steps:
        n = min(chunk, steps - done)
        if loop.iterator is not None:
            part = []
            for _ in range(n):
                try:
                    part.append(loop.batch(next(loop.iterator)))
                except StopIteration:
                    break
            if not part:
                break
            n = len(part)
        else:
            at = done % len(loop.batches) if loop.batches else 0
            part = loop.batches[at:] + loop.batches[:at]
        new_state, outputs, hist, ran, bad_k, seconds = compiled._n.run(state_map, data_inputs, hist_ids, current, part, n)
        for (_, name), h in zip(loop.history, hist):
            history[name].extend(h)
        done += ran
        elapsed += seconds
        if bad_k is not None:
            bad = done - ran + bad_k
        elif not all(t.is_finite() for t in new_state):
            bad = done - 1
        current = new_state
        if outputs and loop.aux_shape is not None:
            aux = loop.aux(outputs)
        if bad is not None:
            status = "stopped_nonfinite"
            break
        if callback is not None and callback(RunResult(status="running", state=unflatten(loop.state_shape, [Tensor(t) for t in current]), aux=aux,
                                                       history=history, steps=done, requested_steps=steps, nonfinite_step=None,
                                                       elapsed=elapsed)) is False:
            status = "stopped_by_callback"
            break
    return RunResult(status=status, state=unflatten(loop.state_shape, [Tensor(t) for t in current]), aux=aux, history=history, steps=done,
                     requested_steps=steps, nonfinite_step=bad, elapsed=elapsed, compiled=compiled)
