"""Deterministic synthetic inputs (numpy), bit-identical to ``oracle/nsrand.h``.

Element ``i`` of stream ``seed`` depends only on ``(seed, i)``:

* ``raw(seed, i)``  = splitmix64 finaliser of ``seed + (i + 1) * 0x9E3779B97F4A7C15``
* ``unit``          = ``(raw >> 40) * 2**-24`` (an exact 24-bit fraction)
* ``uniform``       = ``float32(lo + unit * (hi - lo))`` in float64 arithmetic
* ``normal``        = ``float32(mu + sd * (sum of 12 units - 6))`` (Irwin-Hall,
  exact in float64, so the C and numpy versions agree bit for bit)
* ``tokens``        = ``float32(int(unit * vocab))`` (token ids carried as fp32,
  as the reference ABI carries them)

The benchmark configurations use these streams in place of the
``std::mt19937``/``normal_distribution`` draws of the reference's tests, so
fixtures can be regenerated from a seed instead of being stored.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_CHUNK = 1 << 22


def _raw(seed: int, start: int, count: int) -> np.ndarray:
    idx = np.arange(start + 1, start + count + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + idx * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def unit(seed: int, start: int, count: int) -> np.ndarray:
    """float64 array of exact 24-bit fractions in [0, 1)."""
    return (_raw(seed, start, count) >> np.uint64(40)).astype(np.float64) * (1.0 / 16777216.0)


def uniform(n: int, seed: int, lo: float, hi: float) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    w = float(hi) - float(lo)
    for s in range(0, n, _CHUNK):
        c = min(_CHUNK, n - s)
        out[s:s + c] = (float(lo) + unit(seed, s, c) * w).astype(np.float32)
    return out


def normal(n: int, seed: int, mu: float = 0.0, sd: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    step = _CHUNK // 12
    for s in range(0, n, step):
        c = min(step, n - s)
        u = unit(seed, 12 * s, 12 * c).reshape(c, 12)
        acc = u.sum(axis=1)  # every partial sum is exact in float64
        out[s:s + c] = (float(mu) + float(sd) * (acc - 6.0)).astype(np.float32)
    return out


def tokens(n: int, seed: int, vocab: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    for s in range(0, n, _CHUNK):
        c = min(_CHUNK, n - s)
        out[s:s + c] = np.floor(unit(seed, s, c) * float(vocab)).astype(np.int64).astype(np.float32)
    return out


def one_hot(targets: np.ndarray, classes: int) -> np.ndarray:
    """Dense fp32 one-hot labels [rows, classes], the reference ABI's label form."""
    t = targets.astype(np.int64)
    out = np.zeros((t.size, classes), dtype=np.float32)
    out[np.arange(t.size), t] = 1.0
    return out
