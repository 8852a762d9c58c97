"""Seeded synthetic decode workloads (prompts and their lengths).

Uses the generator of csrc/synth_rng.h (splitmix64 counters): prompt i's token
t is bits(key(seed, stream_i), t) mod vocab; prompt lengths are uniform
integers in [lo, hi]. Vectorised numpy, bit-identical to the C definition.
"""
from __future__ import annotations

import numpy as np

_M = np.uint64(0xFFFFFFFFFFFFFFFF)
TOKENS_STREAM = 3
LENGTHS_STREAM = 4


def _mix64(z):
    with np.errstate(over="ignore"):
        z = (z + np.uint64(0x9E3779B97F4A7C15)) & _M
        z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & _M
        z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & _M
        return z ^ (z >> np.uint64(31))


def _key(seed: int, stream: int) -> np.uint64:
    return _mix64(np.array([seed], np.uint64) ^ _mix64(np.array([stream], np.uint64)))[0]


def _bits(key, n: int):
    idx = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix64(np.uint64(key) + idx * np.uint64(0xD1B54A32D192ED03))


def tokens(n: int, seed: int, stream: int = TOKENS_STREAM, vocab: int = 151936) -> np.ndarray:
    return (_bits(_key(seed, stream), n) % np.uint64(vocab)).astype(np.uint32)


def prompt_lengths(count: int, seed: int, lo: int = 512, hi: int = 4096) -> list[int]:
    b = _bits(_key(seed, LENGTHS_STREAM), count) % np.uint64(hi - lo + 1)
    return [int(lo + v) for v in b]


def prompt(i: int, length: int, seed: int, vocab: int = 151936) -> np.ndarray:
    """Prompt of sequence i: its own stream (1000 + i) so prompts are independent."""
    return tokens(length, seed, 1000 + i, vocab)
