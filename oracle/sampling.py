"""CPU restatement of the reference's fused token sampling -- TEST
INFRASTRUCTURE ONLY (used by tests/, __graft_entry__.smoke() and bench.py's
CPU legs; never by the product path).

Reference: qwen3/sampling.py -- ``sample_tokens`` (:234-270) takes the
Triton path ``_sample_tokens_triton`` (:181-231): one batched
``torch.topk(logits, max_k)`` (sorted, descending), then
``_sample_topk_kernel`` (:112-178) per row: temperature scaling, the per-row
top-k mask, softmax, the top-p mask (keep[0]; keep[j] = cumsum(p)[j-1] <=
top_p), and Gumbel-max sampling with ``tl.rand(seed, row * BLOCK_K + j)``;
greedy rows (temperature <= 0) take the first top-k index.

``tl.rand`` comes from Triton (a dependency not vendored by the reference;
PERFORMANCE.md:10 pins Triton 2.2.0): Philox4x32-10 (Salmon, Moraes, Dror,
Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011) with key =
(seed low 32 bits, seed high 32 bits) and counter = (offset, 0, 0, 0); the
first output word, read as int32 x, maps to (x if x >= 0 else -x - 1) *
4.6566127342e-10 in float32.  Pinned by tests/golden/sampling.npz (Triton's own
``tl.rand`` / ``tl.randint`` and the reference kernel run under Triton's CPU
interpreter).
"""

from __future__ import annotations

import numpy as np

_M0 = np.uint64(0xD2511F53)   # Philox4x32 multipliers
_M1 = np.uint64(0xCD9E8D57)
_W0 = np.uint64(0x9E3779B9)   # Weyl key increments
_W1 = np.uint64(0xBB67AE85)
_MASK = np.uint64(0xFFFFFFFF)


def philox4x32_10(seed: int, c0, c1=0, c2=0, c3=0):
    """Ten Philox4x32 rounds on counter (c0, c1, c2, c3) with the key from
    ``seed``; returns the four uint32 output words (numpy arrays)."""
    c0 = np.asarray(c0, dtype=np.uint64) & _MASK
    shape = c0.shape
    c1 = np.broadcast_to(np.asarray(c1, np.uint64), shape) & _MASK
    c2 = np.broadcast_to(np.asarray(c2, np.uint64), shape) & _MASK
    c3 = np.broadcast_to(np.asarray(c3, np.uint64), shape) & _MASK
    k0 = np.uint64(seed & 0xFFFFFFFF)
    k1 = np.uint64((seed >> 32) & 0xFFFFFFFF)
    for _ in range(10):
        p0 = _M0 * c0            # exact in uint64 (both factors < 2**32)
        p1 = _M1 * c2
        n0 = (p1 >> np.uint64(32)) ^ c1 ^ k0
        n2 = (p0 >> np.uint64(32)) ^ c3 ^ k1
        n1 = p1 & _MASK
        n3 = p0 & _MASK
        c0, c1, c2, c3 = n0 & _MASK, n1, n2 & _MASK, n3
        k0 = (k0 + _W0) & _MASK
        k1 = (k1 + _W1) & _MASK
    return (c0.astype(np.uint32), c1.astype(np.uint32), c2.astype(np.uint32),
            c3.astype(np.uint32))


def rand_uniform(seed: int, offsets) -> np.ndarray:
    """float32 uniforms in [0, 1) for 32-bit ``offsets`` (Triton ``tl.rand``)."""
    w = philox4x32_10(seed, np.asarray(offsets, dtype=np.int64) & 0xFFFFFFFF)[0]
    x = w.view(np.int32).astype(np.int64)
    x = np.where(x < 0, -x - 1, x)
    return (x.astype(np.float32) * np.float32(4.6566127342e-10)).astype(np.float32)


def topk_sorted(logits: np.ndarray, k: int):
    """Top-k values and indices per row, descending; ties by ascending index."""
    idx = np.argsort(-logits, axis=-1, kind="stable")[:, :k]
    return np.take_along_axis(logits, idx, axis=-1), idx


def sample_tokens(logits, temperature, top_k, top_p, seed: int, block_k: int | None = None):
    """Token ids (B,) exactly as the reference's Triton path computes them
    (qwen3/sampling.py:112-178, :181-231), all in float32.  ``top_k`` per row
    must be in [1, 1024] (the Triton path's range, :34,198-200)."""
    logits = np.asarray(logits, np.float32)
    B, V = logits.shape
    temperature = np.broadcast_to(np.asarray(temperature, np.float32), (B,))
    top_k = np.broadcast_to(np.asarray(top_k, np.int64), (B,))
    top_p = np.broadcast_to(np.asarray(top_p, np.float32), (B,))
    max_k = int(min(top_k.max(), V))
    if block_k is None:
        block_k = max(16, 1 << (max_k - 1).bit_length())
    vals, idx = topk_sorted(logits, max_k)
    out = np.empty(B, np.int64)
    j = np.arange(max_k)
    for r in range(B):
        t = np.float32(temperature[r])
        tsafe = t if t > 0 else np.float32(1.0)
        x = (vals[r] / tsafe).astype(np.float32)
        x = np.where(j < min(int(top_k[r]), V), x, np.float32(-np.inf)).astype(np.float32)
        m = x.max()
        e = np.exp((x - m).astype(np.float32)).astype(np.float32)
        p = (e / e.sum(dtype=np.float32)).astype(np.float32)
        c = np.cumsum(p, dtype=np.float32)
        keep = (j == 0) | ((c - p).astype(np.float32) <= top_p[r])
        x = np.where(keep, x, np.float32(-np.inf)).astype(np.float32)
        u = np.maximum(rand_uniform(seed, r * block_k + j), np.float32(1e-7))
        g = (-np.log(-np.log(u).astype(np.float32))).astype(np.float32)
        best = int(np.argmax((x + g).astype(np.float32)))
        out[r] = idx[r, 0] if t <= 0 else idx[r, best]
    return out
