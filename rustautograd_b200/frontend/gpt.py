"""The character-level GPT workload (the model and training step of rg's examples/gpt.py).

Batches are sampled inside the compiled step from a token array with the step's own key, so a
training run never returns to Python between steps. `make_train_step` can also build one
rank's share of a data-parallel step: every rank draws the same global window starts, takes its
own rows, and scales its loss by the global token count, so that the all-reduced gradients are
the full-batch gradients.
"""
from . import nn, random
from .core import all_reduce, arange, compile, concatenate, run, take, tensor, tree_map, tril, value_and_grad, zeros


class GPT:
    def __init__(self, vocab, block, d=128, heads=4, layers=4, dropout_rate=0.0):
        self.block = block
        self.tok = nn.Embedding(vocab, d)
        self.pos = nn.Embedding(block, d)
        self.blocks = [nn.TransformerBlock(d, heads, dropout_rate=dropout_rate) for _ in range(layers)]
        self.norm = nn.LayerNorm(d)
        self.head = nn.Linear(d, vocab, bias=False)
        self.mask = tril(block)

    def init(self, key):
        keys = random.split(key, len(self.blocks) + 3)
        return {
            "tok": self.tok.init(keys[0]),
            "pos": self.pos.init(keys[1]),
            "head": self.head.init(keys[2]),
            "norm": self.norm.init(),
            "blocks": [b.init(keys[3 + i]) for i, b in enumerate(self.blocks)],
        }

    def __call__(self, p, idx, key=None):
        t = idx.shape[1]
        x = self.tok(p["tok"], idx) + self.pos(p["pos"], arange(t))
        mask = self.mask[:t, :t]
        keys = random.split(key, len(self.blocks)) if key is not None else [None] * len(self.blocks)
        for i, b in enumerate(self.blocks):
            x = b(p["blocks"][i], x, mask, keys[i])
        return self.head(p["head"], self.norm(p["norm"], x))


def windows(tokens, key, batch, block):
    """Random contiguous windows of block + 1 tokens: inputs and next-token targets."""
    n = tokens.shape[0]
    start = random.randint(key, (batch,), 0, n - block - 1)
    w = take(tokens, start[:, None] + arange(block + 1))
    return w[:, :-1], w[:, 1:]


def make_train_step(model, opt, batch, world=1, rank=0):
    """The training step of examples/gpt.py:58-68. With world > 1 it is rank `rank`'s share of a
    data-parallel step over a global batch of `batch` windows: the windows are drawn for the whole
    batch (identically on every rank), the rank keeps rows [rank * batch / world, ...), its loss
    is the local mean over `world`, and gradients and loss are summed over ranks before the
    optimiser update, so every rank applies the full-batch update."""
    if batch % world:
        raise ValueError(f"global batch {batch} does not split over {world} ranks")
    local = batch // world

    def loss_fn(params, x, y, key):
        loss = nn.cross_entropy(model(params, x, key), y)
        return loss if world == 1 else loss / world

    def step(state, tokens):
        keys = random.split(state["key"], 3)
        x, y = windows(tokens, keys[1], batch, model.block)
        if world > 1:
            x, y = x[rank * local:(rank + 1) * local], y[rank * local:(rank + 1) * local]
        value, grads = value_and_grad(loss_fn)(state["params"], x, y, keys[2])
        if world > 1:
            grads = tree_map(all_reduce, grads)
            value = all_reduce(value)
        params, opt_state = opt.update(grads, state["opt"], state["params"])
        return {"params": params, "opt": opt_state, "key": keys[0]}, value
    return step


def compile_sampler(model, params, temperature=1.0, top_k=None, top_p=None, device=None):
    """A compiled step that appends one sampled token to a fixed-length context (examples/gpt.py
    compile_sampler): `run` then generates with no Python per token."""

    def step(state):
        k1, k2 = random.split(state["key"])
        logits = model(params, state["ctx"])[:, -1, :] / temperature
        if top_k:
            logits = nn.top_k_logits(logits, top_k)
        if top_p:
            logits = nn.top_p_logits(logits, top_p)
        token = random.categorical(k2, logits)
        ctx = concatenate([state["ctx"][:, 1:], token[:, None]], axis=1)
        return {"ctx": ctx, "key": k1}, token[0]

    start = {"ctx": zeros((1, model.block), "int32"), "key": random.key(0)}
    return compile(step, (start,), validate="basic", device=device)


def generate(sampler, block, prompt_ids, n, seed=0):
    """`n` tokens after `prompt_ids`, left-padded to the fixed context length."""
    ids = ([prompt_ids[0]] * block + list(prompt_ids))[-block:]
    state = {"ctx": tensor([ids], "int32"), "key": random.key(seed)}
    out = run(sampler, state, steps=n)
    return [int(t) for t in out.history["aux"]]
