"""The character-level GPT of BASELINE configs 4 and 5 (rg's examples/gpt.py:20-93): learned token
and position embeddings, pre-LayerNorm blocks of causal multi-head self-attention and a GELU MLP
(4x), a final LayerNorm and an unbiased output projection; next-token cross-entropy; AdamW.

Parameters are a plain dict tree of the layout rg's model produces (so checkpoints move between
the two):
  tok.table (V, d), pos.table (T, d), head.w (d, V), norm.{scale, shift},
  blocks[i].{norm1, norm2}.{scale, shift}, blocks[i].attn.qkv.{w (d, 3d), b}, attn.out.{w, b},
  blocks[i].fc1.{w (d, 4d), b}, blocks[i].fc2.{w (4d, d), b}.
Weights are N(0, 0.02) drawn from keys split in rg's order, biases zero, LayerNorm scales one.
The forward pass is written as functions over that tree; each emits rg's primitive ops in rg's
order, so a training step records the graph rg's front end records (pinned by the graph
fixtures under tests/golden).

Batches are sampled inside the compiled step from the token array with the step's own key, so a
run never returns to Python between steps. A data-parallel rank draws the same global window
starts as every other rank, keeps its rows, scales its loss by 1 / world, and all-reduces loss
and gradients before the update, so every rank applies the full-batch update.
"""
import math

from . import nn, random
from .optim import AdamW
from .program import compile, run, value_and_grad
from .tracing import all_reduce, arange, concatenate, full, ones, take, tensor, tril, where, zeros
from .trees import tree_map

STD = 0.02


def _dense(key, rows, cols):
    return random.normal(key, (rows, cols)) * STD


def _affine(key, d_in, d_out):
    return {"w": _dense(key, d_in, d_out), "b": zeros(d_out)}


def _norm_params(d):
    return {"scale": ones(d), "shift": zeros(d)}


def linear(p, x):
    y = x @ p["w"]
    return y + p["b"] if "b" in p else y


def layer_norm(p, x, eps=1e-5):
    centred = x - x.mean(axis=-1, keepdims=True)
    var = (centred * centred).mean(axis=-1, keepdims=True)
    return centred / (var + eps).sqrt() * p["scale"] + p["shift"]


def attention(p, x, heads, mask):
    """Causal self-attention with the full (T, T) score matrix (nn.py:170-199 without dropout)."""
    b, t, d = x.shape
    hd = d // heads
    qkv = linear(p["qkv"], x).reshape(b, t, 3, heads, hd).transpose(2, 0, 3, 1, 4)
    q, k, v = qkv[0], qkv[1], qkv[2]
    scores = where(mask, q @ k.swapaxes(-1, -2) / math.sqrt(hd), -1e9)
    mixed = (nn.softmax(scores) @ v).transpose(0, 2, 1, 3).reshape(b, t, d)
    return linear(p["out"], mixed)


def block(p, x, heads, mask, key):
    if key is not None:
        # rg's block splits its key even when dropout is off; the split is then unused, but it
        # is part of the recorded program.
        _k_attn, _k_mlp = random.split(key)
    x = x + attention(p["attn"], layer_norm(p["norm1"], x), heads, mask)
    return x + linear(p["fc2"], nn.gelu(linear(p["fc1"], layer_norm(p["norm2"], x))))


class GPT:
    """The model's sizes; `init(key)` draws parameters and `model(params, idx)` gives logits."""

    def __init__(self, vocab, block, d=128, heads=4, layers=4):
        if d % heads:
            raise ValueError(f"model dimension {d} is not divisible by {heads} heads")
        self.vocab, self.block, self.d, self.heads, self.layers = vocab, block, d, heads, layers
        self.mask = tril(block)

    def init(self, key):
        d = self.d
        keys = random.split(key, self.layers + 3)
        params = {"tok": {"table": _dense(keys[0], self.vocab, d)}, "pos": {"table": _dense(keys[1], self.block, d)},
                  "head": {"w": _dense(keys[2], d, self.vocab)}, "norm": _norm_params(d), "blocks": []}
        for i in range(self.layers):
            k_attn, k_fc1, k_fc2 = random.split(keys[3 + i], 3)
            k_qkv, k_out = random.split(k_attn)
            params["blocks"].append({
                "norm1": _norm_params(d), "norm2": _norm_params(d),
                "attn": {"qkv": _affine(k_qkv, d, 3 * d), "out": _affine(k_out, d, d)},
                "fc1": _affine(k_fc1, d, 4 * d), "fc2": _affine(k_fc2, 4 * d, d)})
        return params

    def __call__(self, params, idx, key=None):
        t = idx.shape[1]
        x = take(params["tok"]["table"], idx, 0) + take(params["pos"]["table"], arange(t), 0)
        mask = self.mask[:t, :t]
        keys = random.split(key, self.layers) if key is not None else None
        for i in range(self.layers):
            x = block(params["blocks"][i], x, self.heads, mask, keys[i] if keys is not None else None)
        return layer_norm(params["norm"], x) @ params["head"]["w"]


def windows(tokens, key, batch, block_len):
    """`batch` random windows of block_len + 1 consecutive tokens: inputs and next-token targets."""
    start = random.randint(key, (batch,), 0, tokens.shape[0] - block_len - 1)
    w = take(tokens, start[:, None] + arange(block_len + 1))
    return w[:, :-1], w[:, 1:]


def make_train_step(model, opt, batch, world=1, rank=0):
    """One training step `(state, tokens) -> (state, loss)` with state {"params", "opt", "key"}
    (examples/gpt.py:58-68). With world > 1 it is rank `rank`'s share of a data-parallel step
    over a global batch of `batch` windows."""
    if batch % world:
        raise ValueError(f"global batch {batch} does not split over {world} ranks")
    rows = slice(rank * (batch // world), (rank + 1) * (batch // world))

    def loss_of(params, x, y, key):
        loss = nn.cross_entropy(model(params, x, key), y)
        return loss if world == 1 else loss / world

    def step(state, tokens):
        keys = random.split(state["key"], 3)
        x, y = windows(tokens, keys[1], batch, model.block)
        if world > 1:
            x, y = x[rows], y[rows]
        loss, grads = value_and_grad(loss_of)(state["params"], x, y, keys[2])
        if world > 1:
            grads = tree_map(all_reduce, grads)
            loss = all_reduce(loss)
        params, opt_state = opt.update(grads, state["opt"], state["params"])
        return {"params": params, "opt": opt_state, "key": keys[0]}, loss
    return step


def compile_sampler(model, params, temperature=1.0, top_k=None, top_p=None, device=None):
    """A compiled step appending one sampled token to a fixed-length context (examples/gpt.py
    compile_sampler), so `run` generates with no Python per token."""

    def step(state):
        k_next, k_draw = random.split(state["key"])
        logits = model(params, state["ctx"])[:, -1, :] / temperature
        if top_k:
            logits = nn.top_k_logits(logits, top_k)
        if top_p:
            logits = nn.top_p_logits(logits, top_p)
        token = random.categorical(k_draw, logits)
        ctx = concatenate([state["ctx"][:, 1:], token[:, None]], axis=1)
        return {"ctx": ctx, "key": k_next}, token[0]

    start = {"ctx": zeros((1, model.block), "int32"), "key": random.key(0)}
    return compile(step, (start,), validate="basic", device=device)


def generate(sampler, block_len, prompt_ids, n, seed=0):
    """`n` tokens after `prompt_ids`, the context left-padded with the first prompt token."""
    ids = ([prompt_ids[0]] * block_len + list(prompt_ids))[-block_len:]
    out = run(sampler, {"ctx": tensor([ids], "int32"), "key": random.key(seed)}, steps=n)
    return [int(t) for t in out.history["aux"]]
