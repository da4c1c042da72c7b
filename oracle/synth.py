"""Deterministic, platform-independent synthetic inputs -- TEST INFRASTRUCTURE ONLY.

The golden fixtures under ``tests/golden`` store only seeds, index tables and
reference outputs; the (large) attention inputs are regenerated from the seed
on whichever machine runs the test.  To make that bit-exact across numpy
versions and CPU instruction sets, this module uses no library RNG and no
transcendental function:

* ``splitmix64`` over a counter gives 64-bit integers (integer arithmetic only);
* ``det_normal`` is the Irwin-Hall(12) approximation of N(0, 1): the sum of 12
  uniforms ``k / 2**32`` minus 6 (exact in float64, mean 0, variance 1).

Values are then rounded once to float32 (and, by the callers, to bf16), which is
deterministic.
"""

from __future__ import annotations

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    """SplitMix64 finaliser applied elementwise to uint64 counters."""
    with np.errstate(over="ignore"):
        z = x + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def _stream(seed: int, n: int) -> np.ndarray:
    base = np.uint64((int(seed) * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF)
    with np.errstate(over="ignore"):
        ctr = np.arange(n, dtype=np.uint64) + base
    return _splitmix64(ctr)


def det_normal(seed: int, shape) -> np.ndarray:
    """Approximately N(0,1) float32 array, bit-identical on every platform."""
    shape = tuple(int(s) for s in shape)
    n = int(np.prod(shape)) if shape else 1
    words = _stream(seed, 6 * n).reshape(n, 6)
    lo = (words & np.uint64(0xFFFFFFFF)).astype(np.float64)
    hi = (words >> np.uint64(32)).astype(np.float64)
    s = lo.sum(axis=1) + hi.sum(axis=1)          # exact: < 2**36
    x = s / 4294967296.0 - 6.0                   # exact scaling by 2**-32
    return x.astype(np.float32).reshape(shape)


def det_uniform_int(seed: int, lo: int, hi: int, n: int) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive), deterministic."""
    span = int(hi) - int(lo) + 1
    w = _stream(seed ^ 0x5DEECE66D, n)
    return (w % np.uint64(span)).astype(np.int64) + int(lo)


def det_permutation(seed: int, n: int) -> np.ndarray:
    """A deterministic permutation of range(n) (sort by hashed keys)."""
    keys = _stream(seed ^ 0xA5A5A5A5, n)
    return np.argsort(keys, kind="stable").astype(np.int64)
