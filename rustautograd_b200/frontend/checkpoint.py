"""Checkpoints in the safetensors file format (the layout of python/rg/checkpoint.py, so files
move between rg and this package), and device-resident training sessions whose checkpoints
stream straight between the device frame and the file.

Layout: an 8-byte little-endian header length, a JSON header mapping each dotted tensor name to
{"dtype", "shape", "data_offsets"} plus "__metadata__" (the tree structure under "rg_tree" and
any user strings), then the tensors' bytes in name order.
"""
import json
import os
import struct

import numpy as np

from .core import Tensor, flatten, native, run as _run, tensor, unflatten, _paths

_CODES = {"float32": "F32", "float64": "F64", "int32": "I32"}
_DTYPES = {v: k for k, v in _CODES.items()}
_SIZES = {"F32": 4, "F64": 8, "I32": 4}
_MAX_HEADER = 100 * 1024 * 1024


def paths(t, prefix=""):
    """(dotted name, leaf) pairs in flatten order: the names checkpoints use."""
    if t is None:
        return []
    if isinstance(t, dict):
        return [p for k in sorted(t) for p in paths(t[k], f"{prefix}{k}.")]
    if isinstance(t, (tuple, list)):
        return [p for i, v in enumerate(t) for p in paths(v, f"{prefix}{i}.")]
    return [(prefix[:-1], t)]


def _encode(d):
    if d is None:
        return None
    if d[0] == "none":
        return ["none"]
    if d[0] == "dict":
        return ["dict", list(d[1]), [_encode(s) for s in d[2]]]
    return [d[0], [_encode(s) for s in d[1]]]


def _decode(d):
    if d is None:
        return None
    if d[0] == "none":
        return ("none",)
    if d[0] == "dict":
        return ("dict", tuple(d[1]), tuple(_decode(s) for s in d[2]))
    return (d[0], tuple(_decode(s) for s in d[1]))


def _header(names, specs, tdef, metadata):
    """Header bytes for tensors `names` with (shape, dtype) `specs`, stored in that order."""
    header, offset = {}, 0
    for name, (shape, dtype) in zip(names, specs):
        n = _SIZES[_CODES[dtype]] * int(np.prod(shape, dtype=np.int64))
        header[name] = {"dtype": _CODES[dtype], "shape": list(shape), "data_offsets": [offset, offset + n]}
        offset += n
    meta = {"rg_tree": json.dumps(_encode(tdef))}
    for k, v in (metadata or {}).items():
        if not isinstance(v, str):
            raise TypeError(f"checkpoint metadata {k!r} must be a string")
        meta[k] = v
    header["__metadata__"] = meta
    return json.dumps(header).encode()


def _read_header(path):
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: not a safetensors file (truncated header)")
        size = struct.unpack("<Q", head)[0]
        if size > _MAX_HEADER:
            raise ValueError(f"{path}: header of {size} bytes is implausibly large")
        header = json.loads(f.read(size))
    return header, 8 + size


def save(path, tree, metadata=None):
    """Writes a tree of tensors atomically: a crash leaves any previous file intact."""
    named = [(n or "value", tensor(t)) for n, t in paths(tree)]
    raw = _header([n for n, _ in named], [(t.shape, t.dtype) for _, t in named], flatten(tree)[1], metadata)
    tmp = f"{path}.tmp.{os.getpid()}"
    try:
        with open(tmp, "wb") as f:
            f.write(struct.pack("<Q", len(raw)))
            f.write(raw)
            for _, t in named:
                f.write(t._t.tobytes())
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, path)
    finally:
        if os.path.exists(tmp):
            os.remove(tmp)


def load(path, with_metadata=False):
    """Reads a checkpoint; files from other tools load as a flat dict of dotted names."""
    header, data_start = _read_header(path)
    with open(path, "rb") as f:
        f.seek(data_start)
        body = f.read()
    meta = header.pop("__metadata__", {})
    values = {}
    for name, info in header.items():
        code = info["dtype"]
        if code not in _DTYPES:
            raise ValueError(f"{path}: tensor {name!r} has unsupported dtype {code}")
        n = _SIZES[code] * int(np.prod(info["shape"], dtype=np.int64))
        start, end = info["data_offsets"]
        if not (0 <= start <= end <= len(body)) or end - start != n:
            raise ValueError(f"{path}: tensor {name!r} has inconsistent offsets or shape")
        values[name] = Tensor(native().Tensor(body[start:end], list(info["shape"]), _DTYPES[code]))
    if "rg_tree" in meta:
        tdef = _decode(json.loads(meta["rg_tree"]))
        names = [n or "value" for n, _ in paths(unflatten(tdef, [0] * len(values)))] if values else []
        if set(names) != set(values):
            raise ValueError(f"{path}: tree metadata does not match the stored tensors")
        result = unflatten(tdef, [values[n] for n in names])
    else:
        result = values
    user_meta = {k: v for k, v in meta.items() if k != "rg_tree"}
    return (result, user_meta) if with_metadata else result


class Session:
    """A training run whose state stays on the device between `run` calls.

    `run(steps)` continues from where the last call stopped without uploading or downloading
    the state; `state` reads it back; `save(path)` streams it from the device frame straight
    into a checkpoint file (the layout of `save`), and `restore(path)` streams a checkpoint of
    the same state structure back into the frame.
    """

    def __init__(self, compiled, state, data=None):
        self._c = compiled
        leaves, self._state_def = flatten(state)
        leaves = [tensor(l) for l in leaves]
        self._names = [n or "value" for n, _ in paths(unflatten(self._state_def, leaves))]
        self._specs = [(t.shape, t.dtype) for t in leaves]
        n_state = len(leaves)
        d = compiled._out_def
        self._has_aux = not (d == self._state_def)
        self._aux_def = d[1][1] if self._has_aux else None
        aux_names = _paths(self._aux_def, "aux") if self._has_aux else []
        shapes = compiled._n.output_shapes
        scalar = [k for k in range(n_state, n_state + len(aux_names)) if all(x == 1 for x in shapes[k])]
        self._hist_names = [aux_names[k - n_state] for k in scalar] + list(compiled._extras)
        history = scalar + [compiled._n_out + j for j in range(len(compiled._extras))]
        data_inputs = list(range(n_state, len(compiled._in_sig)))
        self._batches = [[tensor(l)._t for l in flatten(data)[0]]] if data is not None else []
        self._n_state = n_state
        self._h = compiled._n.session([(k, k) for k in range(n_state)], data_inputs, history, [t._t for t in leaves])

    def run(self, steps):
        outputs, hist, ran, bad, seconds = self._h.run(self._batches, steps)
        aux = None
        if self._has_aux and outputs:
            aux = unflatten(self._aux_def, [Tensor(t) for t in outputs[self._n_state:self._c._n_out]])
        from .core import RunResult
        return RunResult(status="stopped_nonfinite" if bad is not None else "completed", aux=aux,
                         history=dict(zip(self._hist_names, hist)), steps=ran, nonfinite_step=bad, elapsed=seconds)

    @property
    def state(self):
        return unflatten(self._state_def, [Tensor(t) for t in self._h.state()])

    def save(self, path, metadata=None):
        self._h.save(path, _header(self._names, self._specs, self._state_def, metadata))

    def restore(self, path):
        header, data_start = _read_header(path)
        meta = header.get("__metadata__", {})
        if "rg_tree" in meta and _decode(json.loads(meta["rg_tree"])) != self._state_def:
            raise ValueError(f"{path}: the checkpoint's tree does not match this session's state")
        offsets = []
        for name, (shape, dtype) in zip(self._names, self._specs):
            info = header.get(name)
            if info is None or info["dtype"] != _CODES[dtype] or list(info["shape"]) != list(shape):
                raise ValueError(f"{path}: tensor {name!r} is missing or has another dtype or shape")
            offsets.append(data_start + info["data_offsets"][0])
        self._h.restore(path, offsets)
