"""Keyed random numbers. A key is a pair of int32 words; every draw is a pure function of its key
(the engine's SplitMix64 streams), so a step that carries its key in its state replays exactly.

`key(seed)` derives the pair as rg does (the seed times the 64-bit golden-ratio constant, high
word first, each word as a signed int32), so seeds give the same streams in both front ends.
"""
from .tracing import argmax, floor, log, maximum, op, tensor

_GOLDEN = 0x9E3779B97F4A7C15


def _i32(word):
    return word - (1 << 32) if word >= (1 << 31) else word


def key(seed):
    mixed = (seed * _GOLDEN) & ((1 << 64) - 1)
    return tensor([_i32(mixed >> 32), _i32(mixed & 0xFFFFFFFF)], "int32")


def split(k, n=2):
    """`n` independent keys, shape (n, 2)."""
    return op("key_split", k, n=n)


def uniform(k, shape=(), dtype="float32", low=0.0, high=1.0):
    u = op("random_uniform", k, shape=list(shape), dtype=dtype)
    return u if (low, high) == (0.0, 1.0) else low + (high - low) * u


def normal(k, shape=(), dtype="float32"):
    return op("random_normal", k, shape=list(shape), dtype=dtype)


def randint(k, shape, low, high):
    """int32 uniform over [low, high): drawn in float64 so every integer of a large range is
    reachable, then floored."""
    u = op("random_uniform", k, shape=list(shape), dtype="float64")
    return floor(low + (high - low) * u).cast("int32")


def categorical(k, logits, axis=-1):
    """Indices drawn from unnormalised log-probabilities by the Gumbel-max trick."""
    u = op("random_uniform", k, shape=list(logits.shape), dtype=logits.dtype)
    tiny = 1e-7 if logits.dtype == "float32" else 1e-15
    return argmax(logits + -log(-log(maximum(u, tiny))), axis)
