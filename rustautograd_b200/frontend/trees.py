"""Nested containers of tensors ("trees"): tuples, lists and dicts with tensors (or numbers) at
the leaves, and `None` as an empty subtree.

A tree flattens to its leaves plus a `Shape` describing everything else. Dict entries are
visited in sorted key order; that fixes the order of a compiled step's inputs and outputs and
of a checkpoint's tensors, and it is the order rg's engine interface expects.
"""


class Shape:
    """The structure of a tree without its leaves. `kind` is "leaf", "none", "tuple", "list" or
    "dict"; `keys` holds a dict's sorted keys; `children` the sub-structures."""

    __slots__ = ("kind", "keys", "children", "n_leaves")

    def __init__(self, kind, keys=(), children=()):
        self.kind, self.keys, self.children = kind, tuple(keys), tuple(children)
        self.n_leaves = 1 if kind == "leaf" else sum(c.n_leaves for c in self.children)

    def _id(self):
        return (self.kind, self.keys, tuple(c._id() for c in self.children))

    def __eq__(self, other):
        return isinstance(other, Shape) and self._id() == other._id()

    def __hash__(self):
        return hash(self._id())

    def __repr__(self):
        if self.kind == "leaf":
            return "*"
        if self.kind == "none":
            return "None"
        if self.kind == "dict":
            return "{" + ", ".join(f"{k!r}: {c!r}" for k, c in zip(self.keys, self.children)) + "}"
        inner = ", ".join(map(repr, self.children))
        return f"({inner},)" if self.kind == "tuple" and len(self.children) == 1 else ("(%s)" if self.kind == "tuple" else "[%s]") % inner

    # The checkpoint metadata's encoding of a structure (rg's checkpoint format): a leaf is
    # null, None is ["none"], a dict ["dict", keys, children], a tuple or list [kind, children].
    def encode(self):
        if self.kind == "leaf":
            return None
        if self.kind == "none":
            return ["none"]
        if self.kind == "dict":
            return ["dict", list(self.keys), [c.encode() for c in self.children]]
        return [self.kind, [c.encode() for c in self.children]]

    @staticmethod
    def decode(obj):
        if obj is None:
            return LEAF
        kind = obj[0]
        if kind == "none":
            return Shape("none")
        if kind == "dict":
            return Shape("dict", obj[1], [Shape.decode(c) for c in obj[2]])
        return Shape(kind, (), [Shape.decode(c) for c in obj[1]])


LEAF = Shape("leaf")


def flatten(tree):
    """(leaves, Shape) of a tree."""
    leaves = []

    def walk(t):
        if t is None:
            return Shape("none")
        if isinstance(t, dict):
            keys = sorted(t)
            return Shape("dict", keys, [walk(t[k]) for k in keys])
        if isinstance(t, (tuple, list)):
            return Shape(type(t).__name__ if type(t) in (tuple, list) else "tuple", (), [walk(v) for v in t])
        leaves.append(t)
        return LEAF
    return leaves, walk(tree)


def unflatten(shape, leaves):
    """The tree of `shape` with `leaves` in flatten order."""
    it = iter(leaves)

    def build(s):
        if s.kind == "leaf":
            return next(it)
        if s.kind == "none":
            return None
        if s.kind == "dict":
            return {k: build(c) for k, c in zip(s.keys, s.children)}
        items = [build(c) for c in s.children]
        return tuple(items) if s.kind == "tuple" else items
    return build(shape)


def leaf_names(shape, prefix=""):
    """Dotted names of the leaves in flatten order ("params.blocks.0.fc1.w"); a lone leaf at
    the root is named by `prefix`."""
    if shape.kind == "leaf":
        return [prefix]
    if shape.kind == "none":
        return []
    labels = shape.keys if shape.kind == "dict" else [str(i) for i in range(len(shape.children))]
    out = []
    for label, child in zip(labels, shape.children):
        out += leaf_names(child, f"{prefix}.{label}" if prefix else str(label))
    return out


def tree_map(f, tree, *others):
    """`f` applied leaf by leaf across trees of one structure."""
    leaves, shape = flatten(tree)
    rest = [flatten(o) for o in others]
    for _, s in rest:
        if s != shape:
            raise ValueError(f"tree_map needs trees of one structure: {shape!r} vs {s!r}")
    return unflatten(shape, [f(*vals) for vals in zip(leaves, *(r[0] for r in rest))])


def tree_leaves(tree):
    return flatten(tree)[0]
