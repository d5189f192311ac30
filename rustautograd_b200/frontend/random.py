"""Keyed random numbers (the op compositions of python/rg/random.py): every function is pure
in its key, so a compiled step that carries its key in its state replays exactly."""
from .core import argmax, floor, log, maximum, op, tensor


def key(seed):
    """A key from an integer seed: the seed times the 64-bit golden ratio, as two int32 halves."""
    mixed = seed * 0x9E3779B97F4A7C15 % (1 << 64)
    signed = lambda v: v - (1 << 32) if v >= (1 << 31) else v
    return tensor([signed(mixed >> 32), signed(mixed & 0xFFFFFFFF)], "int32")


def split(k, n=2):
    return op("key_split", k, n=n)


def uniform(k, shape=(), dtype="float32", low=0.0, high=1.0):
    u = op("random_uniform", k, shape=list(shape), dtype=dtype)
    return u if low == 0.0 and high == 1.0 else low + (high - low) * u


def normal(k, shape=(), dtype="float32"):
    return op("random_normal", k, shape=list(shape), dtype=dtype)


def randint(k, shape, low, high):
    """Uniform int32 in [low, high), drawn in float64 so every integer of the range is reachable."""
    u = op("random_uniform", k, shape=list(shape), dtype="float64")
    return floor(low + (high - low) * u).cast("int32")


def bernoulli(k, p=0.5, shape=(), dtype="float32"):
    """1 with probability `p`, else 0, as floats."""
    return op("gt", tensor(float(p), dtype), op("random_uniform", k, shape=list(shape), dtype=dtype))


def gumbel(k, shape=(), dtype="float32"):
    u = op("random_uniform", k, shape=list(shape), dtype=dtype)
    eps = 1e-7 if dtype == "float32" else 1e-15
    return -log(-log(maximum(u, eps)))


def categorical(k, logits, axis=-1):
    """Indices drawn from unnormalised log-probabilities with the Gumbel-max trick."""
    return argmax(logits + gumbel(k, logits.shape, logits.dtype), axis)
