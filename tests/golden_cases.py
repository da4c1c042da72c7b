"""Load the golden fixtures and rebuild their inputs from the stored seeds.

The fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py from the
reference's own functions) store seeds, index tables and outputs; this module
regenerates the bf16 inputs with oracle.synth and checks them against the
stored SHA-256 so a generator drift fails loudly instead of silently.
"""

from __future__ import annotations

import glob
import hashlib
import json
import os

import numpy as np

from oracle import synth
from oracle.attention import bf16_bits, bf16_round

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bf16_normal(seed, shape):
    return bf16_round(synth.det_normal(seed, shape))


def case_names(kind: str) -> list[str]:
    names = []
    for p in sorted(glob.glob(os.path.join(GOLDEN, "*.npz"))):
        with np.load(p) as z:
            meta = json.loads(str(z["meta"]))
        if meta.get("kind") == kind:
            names.append(os.path.basename(p)[:-4])
    return names


def load(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        d = {k: z[k] for k in z.files}
    d["meta"] = json.loads(str(d["meta"]))
    return d


def decode_inputs(case: dict) -> dict:
    """Regenerate a decode case's inputs: per-request context K/V (the prefix
    the reference wrote with PagedKVCache.update), q, k_new, v_new."""
    m = case["meta"]
    seed, H, Hkv, D = m["seed"], m["H"], m["Hkv"], m["D"]
    lens = case["lens"]
    ctx = []
    for b, L in enumerate(lens):
        n = int(L) - 1
        if n > 0:
            k = bf16_normal(seed * 1000 + 10 * b + 1, (1, Hkv, n, D))
            v = bf16_normal(seed * 1000 + 10 * b + 2, (1, Hkv, n, D))
        else:
            k = v = None
        ctx.append((k, v))
    B = len(lens)
    q = bf16_normal(m["q_seed"], (B, H, D))
    k_new = bf16_normal(m["k_new_seed"], (B, Hkv, D))
    v_new = bf16_normal(m["v_new_seed"], (B, Hkv, D))
    digest = sha(bf16_bits(q)) + sha(bf16_bits(k_new)) + sha(bf16_bits(v_new))
    assert digest == m["input_digest"], "regenerated decode inputs differ from the fixture's"
    return dict(ctx=ctx, q=q, k_new=k_new, v_new=v_new)


def prefill_inputs(case: dict) -> dict:
    m = case["meta"]
    H, Hkv, D, lens = m["H"], m["Hkv"], m["D"], m["lens"]
    B, S = len(lens), m["S"]
    q = bf16_normal(m["q_seed"], (B, H, S, D))
    k = bf16_normal(m["k_seed"], (B, Hkv, S, D))
    v = bf16_normal(m["v_seed"], (B, Hkv, S, D))
    digest = sha(bf16_bits(q)) + sha(bf16_bits(k)) + sha(bf16_bits(v))
    assert digest == m["input_digest"], "regenerated prefill inputs differ from the fixture's"
    return dict(q=q, k=k, v=v)


def pool_digest(k_pool: np.ndarray, v_pool: np.ndarray) -> str:
    """SHA-256 pair over the bf16 bit patterns of a (float32 or bf16-bits) pool."""
    kb = k_pool if k_pool.dtype == np.uint16 else bf16_bits(k_pool)
    vb = v_pool if v_pool.dtype == np.uint16 else bf16_bits(v_pool)
    return sha(kb) + sha(vb)


def pack_varlen(x: np.ndarray, lens) -> np.ndarray:
    """(B, h, S, D) right-padded -> (T, h, D) packed valid rows."""
    return np.concatenate([np.transpose(x[b, :, :int(L)], (1, 0, 2)) for b, L in enumerate(lens)],
                          axis=0)
