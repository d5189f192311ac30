"""Checkpoints in the safetensors file format, and device-resident training sessions whose state
streams between the device frame and a checkpoint file.

The file layout is rg's (python/rg/checkpoint.py:37-105), so checkpoints move between rg and
this package: an 8-byte little-endian header length; a JSON header mapping each leaf's dotted
name to {"dtype": F32|F64|I32, "shape", "data_offsets": [begin, end]} plus "__metadata__" with
the tree structure (JSON under "rg_tree") and any user strings; then the leaves' bytes in
flatten order.
"""
import json
import os
import struct
import tempfile

import numpy as np

from .program import RunResult
from .tracing import Tensor, native, tensor
from .trees import Shape, flatten, leaf_names, unflatten

_FILE_CODE = {"float32": "F32", "float64": "F64", "int32": "I32"}
_DTYPE_OF = {code: dt for dt, code in _FILE_CODE.items()}
_ITEM = {"F32": 4, "F64": 8, "I32": 4}
_HEADER_LIMIT = 100 << 20
_TREE_KEY = "rg_tree"


def _names(shape):
    """Tensor names of a structure's leaves; a lone tensor is stored as "value"."""
    return [n or "value" for n in leaf_names(shape)]


def _nbytes(code, shape):
    return _ITEM[code] * int(np.prod(shape, dtype=np.int64))


def _header_bytes(shape, specs, metadata):
    """The JSON header for leaves of `shape` with (dims, dtype) `specs`, stored in that order."""
    entries, at = {}, 0
    for name, (dims, dtype) in zip(_names(shape), specs):
        code = _FILE_CODE[dtype]
        size = _nbytes(code, dims)
        entries[name] = {"dtype": code, "shape": list(dims), "data_offsets": [at, at + size]}
        at += size
    meta = {_TREE_KEY: json.dumps(shape.encode())}
    for k, v in (metadata or {}).items():
        if not isinstance(v, str):
            raise TypeError(f"checkpoint metadata {k!r} must be a string, not {type(v).__name__}")
        meta[k] = v
    entries["__metadata__"] = meta
    return json.dumps(entries).encode()


def _parse_header(path):
    """(header dict, offset of the first data byte)."""
    with open(path, "rb") as f:
        prefix = f.read(8)
        if len(prefix) < 8:
            raise ValueError(f"{path}: too short for a safetensors header")
        (n,) = struct.unpack("<Q", prefix)
        if n > _HEADER_LIMIT:
            raise ValueError(f"{path}: header length {n} exceeds {_HEADER_LIMIT} bytes")
        return json.loads(f.read(n)), 8 + n


def _stored_shape(meta):
    return Shape.decode(json.loads(meta[_TREE_KEY])) if _TREE_KEY in meta else None


def save(path, tree, metadata=None):
    """Writes `tree` to `path`. The bytes go to a temporary file in the same directory, synced
    before it is renamed over `path`, so an interrupted save never leaves a partial file."""
    leaves, shape = flatten(tree)
    ts = [tensor(v) for v in leaves]
    head = _header_bytes(shape, [(t.shape, t.dtype) for t in ts], metadata)
    directory = os.path.dirname(os.path.abspath(path))
    fd, partial = tempfile.mkstemp(prefix=os.path.basename(path) + ".", suffix=".partial", dir=directory)
    done = False
    try:
        with os.fdopen(fd, "wb") as out:
            out.write(struct.pack("<Q", len(head)) + head)
            for t in ts:
                out.write(t._t.tobytes())
            out.flush()
            os.fsync(out.fileno())
        os.replace(partial, path)
        done = True
    finally:
        if not done and os.path.exists(partial):
            os.unlink(partial)


def load(path, with_metadata=False):
    """Reads a checkpoint as the tree it was saved from (files without tree metadata, from other
    tools, as a flat dict of tensor names)."""
    header, start = _parse_header(path)
    meta = header.pop("__metadata__", {})
    with open(path, "rb") as f:
        f.seek(start)
        data = f.read()
    tensors = {}
    for name, entry in header.items():
        code = entry["dtype"]
        if code not in _DTYPE_OF:
            raise ValueError(f"{path}: {name!r} has dtype {code}, which rg does not store")
        lo, hi = entry["data_offsets"]
        if not 0 <= lo <= hi <= len(data) or hi - lo != _nbytes(code, entry["shape"]):
            raise ValueError(f"{path}: {name!r} has offsets that do not fit its shape or the file")
        tensors[name] = Tensor(native().Tensor(data[lo:hi], list(entry["shape"]), _DTYPE_OF[code]))
    shape = _stored_shape(meta)
    if shape is None:
        tree = tensors
    else:
        names = _names(shape)
        if sorted(names) != sorted(tensors):
            raise ValueError(f"{path}: the stored tree does not name the stored tensors")
        tree = unflatten(shape, [tensors[n] for n in names])
    user = {k: v for k, v in meta.items() if k != _TREE_KEY}
    return (tree, user) if with_metadata else tree


class Session:
    """A training run whose state stays in one device frame between `run` calls.

    `run(steps)` continues where the previous call stopped, without moving the state; `state`
    reads it back; `save(path)` streams it from the frame into a checkpoint file (the layout of
    `save`) and `restore(path)` streams a checkpoint of the same state structure back."""

    def __init__(self, compiled, state, data=None):
        leaves, self._shape = flatten(state)
        ts = [tensor(v) for v in leaves]
        self._specs = [(t.shape, t.dtype) for t in ts]
        self._c = compiled
        n = len(ts)
        out = compiled._out_shape
        self._aux_shape = None if out == self._shape else out.children[1]
        aux_names = leaf_names(self._aux_shape, "aux") if self._aux_shape is not None else []
        dims = compiled._n.output_shapes
        scalars = [k for k in range(n, n + len(aux_names)) if all(d == 1 for d in dims[k])]
        history = scalars + [compiled._n_out + j for j in range(len(compiled._observed))]
        self._history_names = [aux_names[k - n] for k in scalars] + list(compiled._observed)
        self._n_state = n
        self._batches = [] if data is None else [[tensor(v)._t for v in flatten(data)[0]]]
        self._h = compiled._n.session([(k, k) for k in range(n)], list(range(n, len(compiled._in_sig))), history, [t._t for t in ts])

    def run(self, steps):
        outputs, hist, ran, bad, seconds = self._h.run(self._batches, steps)
        aux = None
        if self._aux_shape is not None and outputs:
            aux = unflatten(self._aux_shape, [Tensor(t) for t in outputs[self._n_state:self._c._n_out]])
        return RunResult(status="completed" if bad is None else "stopped_nonfinite", aux=aux, history=dict(zip(self._history_names, hist)),
                         steps=ran, nonfinite_step=bad, elapsed=seconds)

    @property
    def state(self):
        return unflatten(self._shape, [Tensor(t) for t in self._h.state()])

    def save(self, path, metadata=None):
        self._h.save(path, _header_bytes(self._shape, self._specs, metadata))

    def restore(self, path):
        header, start = _parse_header(path)
        stored = _stored_shape(header.get("__metadata__", {}))
        if stored is not None and stored != self._shape:
            raise ValueError(f"{path}: the checkpoint's tree is not this session's state structure")
        offsets = []
        for name, (dims, dtype) in zip(_names(self._shape), self._specs):
            entry = header.get(name)
            if entry is None or entry["dtype"] != _FILE_CODE[dtype] or list(entry["shape"]) != list(dims):
                raise ValueError(f"{path}: {name!r} is missing, or stored with another dtype or shape")
            offsets.append(start + entry["data_offsets"][0])
        self._h.restore(path, offsets)


__all__ = ["save", "load", "Session"]
