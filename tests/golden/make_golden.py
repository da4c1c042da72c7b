"""Generate the golden fixtures in this folder from the REFERENCE implementation.

Run in a container where the reference repository (uphome/Qwen3-engine-from-scratch)
is checked out; its path comes from ``--reference`` (default: the
``QWEN3_REFERENCE`` environment variable).  The reference's own PyTorch
functions run on CPU in float32:

* decode:   qwen3/paged_attention.py:paged_attention (per request, as
            qwen3/attention.py:181-186 calls it), with the pool, block tables and
            row slots managed by qwen3/PagedKVcache.py (KVCachePool/PagedKVCache);
* scatter:  PagedKVCache.update (qwen3/PagedKVcache.py:177-214) -- recorded as a
            SHA-256 of the pool's bf16 bytes after every write phase;
* prefill:  Qwen3Attention._standard_attention (qwen3/attention.py:193-207) on
            a right-padded batch with the mask of qwen3/model.py:150-161;
* inputs:   RMSNorm (qwen3/norm.py) and RotaryEmbedding/apply_rotary_pos_emb
            (qwen3/rope.py).

Large inputs are not stored: they are regenerated bit-exactly from the stored
seeds by ``oracle.synth.det_normal`` (integer-only generator) and rounded to
bf16, and a SHA-256 of those bf16 inputs is stored so a generator drift fails
loudly.  Outputs are stored as float32 (decode, norm/rope) or float16
(prefill, to keep the files small).

Usage:  python tests/golden/make_golden.py --reference <path-to-reference-checkout>
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import synth  # noqa: E402
from oracle.attention import bf16_bits, bf16_round  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def pool_digest(buf) -> str:
    """SHA-256 of the pool's bf16 bit patterns (values are bf16-representable)."""
    return sha(bf16_bits(buf.numpy()))


def bf16_normal(seed, shape):
    return bf16_round(synth.det_normal(seed, shape))


# ---------------------------------------------------------------------------
# Decode cases: prefix written by PagedKVCache.update, then one decode step
# through paged_attention (which writes the new token first).
# ---------------------------------------------------------------------------

DECODE_CASES = {
    # config 1 of the benchmark plan: 16/8/128, B=4, L~U[64,512], 256-block pool
    "decode_c1": dict(H=16, Hkv=8, D=128, num_blocks=256, num_layers=1, layer=0,
                      max_seq_len=512, max_requests=8, lens=("uniform", 64, 512, 4), seed=101),
    # GQA 4 (Qwen3-4B/8B shape), page-boundary lengths, second layer of a 2-layer pool
    "decode_g4_edges": dict(H=32, Hkv=8, D=128, num_blocks=64, num_layers=2, layer=1,
                            max_seq_len=128, max_requests=10,
                            lens=("list", [1, 16, 17, 31, 33, 128]), seed=202),
    # GQA 8 (Qwen3-30B-A3B shape: 32 q / 4 kv heads)
    "decode_g8": dict(H=32, Hkv=4, D=128, num_blocks=48, num_layers=1, layer=0,
                      max_seq_len=256, max_requests=4, lens=("list", [5, 64, 200]), seed=303),
    # GQA 5 (Qwen3-14B shape: 40 q / 8 kv heads) and MHA-like G=1
    "decode_g5": dict(H=40, Hkv=8, D=128, num_blocks=32, num_layers=1, layer=0,
                      max_seq_len=160, max_requests=3, lens=("list", [2, 150]), seed=404),
    "decode_g1": dict(H=8, Hkv=8, D=128, num_blocks=24, num_layers=1, layer=0,
                      max_seq_len=96, max_requests=3, lens=("list", [9, 96]), seed=505),
}


def make_decode_case(name, cfg, ref):
    torch = ref["torch"]
    KVCachePool, PagedKVCache = ref["KVCachePool"], ref["PagedKVCache"]
    paged_attention = ref["paged_attention"]

    H, Hkv, D = cfg["H"], cfg["Hkv"], cfg["D"]
    seed = cfg["seed"]
    kind = cfg["lens"][0]
    if kind == "uniform":
        _, lo, hi, n = cfg["lens"]
        lens = synth.det_uniform_int(seed, lo, hi, n)
    else:
        lens = np.asarray(cfg["lens"][1], dtype=np.int64)
    B = len(lens)
    nb = cfg["num_blocks"]
    pool = KVCachePool(num_blocks=nb, num_layers=cfg["num_layers"], block_size=16,
                       num_kv_heads=Hkv, head_dim=D, device=torch.device("cpu"),
                       dtype=torch.float32, max_seq_len=cfg["max_seq_len"],
                       max_requests=cfg["max_requests"])
    # random placement: alloc() pops from the END of free_block_ids
    # (qwen3/PagedKVcache.py:68-69), so install a seeded permutation there.
    perm = synth.det_permutation(seed + 1, nb)
    pool.free_block_ids = [int(x) for x in perm]
    layer = cfg["layer"]

    caches = []
    for b in range(B):
        c = PagedKVCache(pool)
        n_ctx = int(lens[b]) - 1
        if n_ctx > 0:
            k_ctx = torch.from_numpy(bf16_normal(seed * 1000 + 10 * b + 1, (1, Hkv, n_ctx, D)))
            v_ctx = torch.from_numpy(bf16_normal(seed * 1000 + 10 * b + 2, (1, Hkv, n_ctx, D)))
            c.update(layer, k_ctx, v_ctx)
            c.advance_seq_len(n_ctx)
        caches.append(c)
    digest_prefix = pool_digest(pool.k_buffer) + pool_digest(pool.v_buffer)

    q = bf16_normal(seed * 1000 + 7, (B, H, D))
    k_new = bf16_normal(seed * 1000 + 8, (B, Hkv, D))
    v_new = bf16_normal(seed * 1000 + 9, (B, Hkv, D))
    outs = []
    scaling = D ** -0.5
    with torch.no_grad():
        for b, c in enumerate(caches):
            L = int(lens[b])
            mask = torch.zeros(1, 1, 1, L, dtype=torch.float32)
            o = paged_attention(torch.from_numpy(q[b:b + 1, :, None, :].copy()),
                                torch.from_numpy(k_new[b:b + 1, :, None, :].copy()),
                                torch.from_numpy(v_new[b:b + 1, :, None, :].copy()),
                                c, layer, mask, scaling)
            outs.append(o.reshape(H, D).numpy())
    out = np.stack(outs).astype(np.float32)
    digest_final = pool_digest(pool.k_buffer) + pool_digest(pool.v_buffer)

    input_digest = sha(bf16_bits(q)) + sha(bf16_bits(k_new)) + sha(bf16_bits(v_new))
    meta = dict(case=name, kind="decode", H=H, Hkv=Hkv, D=D, block_size=16,
                num_blocks=nb, num_layers=cfg["num_layers"], layer=layer,
                max_seq_len=cfg["max_seq_len"], max_requests=cfg["max_requests"],
                seed=seed, scaling=scaling,
                ctx_seed=dict(k="seed*1000+10*b+1", v="seed*1000+10*b+2"),
                q_seed=seed * 1000 + 7, k_new_seed=seed * 1000 + 8, v_new_seed=seed * 1000 + 9,
                input_digest=input_digest, pool_digest_prefix=digest_prefix,
                pool_digest_final=digest_final,
                reference_fn="qwen3/paged_attention.py:paged_attention")
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"),
        meta=np.array(json.dumps(meta)),
        lens=lens.astype(np.int64),
        row_ids=np.array([c.row_id for c in caches], dtype=np.int32),
        block_table_2d=pool.block_table_2d.numpy().astype(np.int32),
        seq_lens=pool.seq_lens.numpy().astype(np.int32),
        out=out,
    )
    print(f"{name}: B={B} lens={lens.tolist()} |out|max={np.abs(out).max():.4f}")


# ---------------------------------------------------------------------------
# Prefill case: right-padded batch, per-request PagedKVCache.update of all S
# positions (qwen3/attention.py:160-161), then _standard_attention with the
# model's 4-D mask.
# ---------------------------------------------------------------------------

PREFILL_CASES = {
    "prefill_varlen": dict(H=4, Hkv=2, D=128, lens=[1, 5, 16, 33, 130, 257], seed=606,
                           num_blocks=128, max_seq_len=512, max_requests=8),
    "prefill_g4": dict(H=8, Hkv=2, D=128, lens=[64, 129, 3], seed=707,
                       num_blocks=32, max_seq_len=256, max_requests=4),
}


def model_prefill_mask(torch, lens, S):
    """The (B,1,S,S) additive mask Qwen3Model.forward builds for a padded
    prefill batch (restated from qwen3/model.py:150-161)."""
    B = len(lens)
    row = torch.arange(S).view(1, S, 1)
    col = torch.arange(S).view(1, 1, S)
    lens_t = torch.tensor(lens).view(B, 1, 1)
    valid = (row < lens_t) & (col < lens_t) & (col <= row)
    pad_keep = (row >= lens_t) & (col == 0)
    m = torch.full((B, S, S), float("-inf"), dtype=torch.float32)
    m[valid | pad_keep] = 0
    return m.unsqueeze(1)


def make_prefill_case(name, cfg, ref):
    torch = ref["torch"]
    Qwen3Attention, Qwen3Config = ref["Qwen3Attention"], ref["Qwen3Config"]
    KVCachePool, PagedKVCache = ref["KVCachePool"], ref["PagedKVCache"]
    H, Hkv, D, lens, seed = cfg["H"], cfg["Hkv"], cfg["D"], cfg["lens"], cfg["seed"]
    B, S = len(lens), max(lens)
    q = bf16_normal(seed * 1000 + 1, (B, H, S, D))
    k = bf16_normal(seed * 1000 + 2, (B, Hkv, S, D))
    v = bf16_normal(seed * 1000 + 3, (B, Hkv, S, D))
    conf = Qwen3Config(hidden_size=H * D, num_attention_heads=H, num_key_value_heads=Hkv,
                       head_dim=D, num_hidden_layers=1, vocab_size=16,
                       intermediate_size=16, rms_norm_eps=1e-6, rope_theta=1e6)
    attn = Qwen3Attention(conf, 0)
    mask = model_prefill_mask(torch, lens, S)
    with torch.no_grad():
        o = attn._standard_attention(torch.from_numpy(q), torch.from_numpy(k),
                                     torch.from_numpy(v), mask)        # (B,S,H*D)
    o = o.numpy().reshape(B, S, H, D)
    packed = np.concatenate([o[b, :lens[b]] for b in range(B)], axis=0)  # (T,H,D)

    # the per-request prefill page write of qwen3/attention.py:160-161
    pool = KVCachePool(num_blocks=cfg["num_blocks"], num_layers=1, block_size=16,
                       num_kv_heads=Hkv, head_dim=D, device=torch.device("cpu"),
                       dtype=torch.float32, max_seq_len=cfg["max_seq_len"],
                       max_requests=cfg["max_requests"])
    pool.free_block_ids = [int(x) for x in synth.det_permutation(seed + 1, cfg["num_blocks"])]
    caches = [PagedKVCache(pool) for _ in range(B)]
    for i, c in enumerate(caches):
        c.update(0, torch.from_numpy(k[i:i + 1]), torch.from_numpy(v[i:i + 1]))
    digest = pool_digest(pool.k_buffer) + pool_digest(pool.v_buffer)

    meta = dict(case=name, kind="prefill", H=H, Hkv=Hkv, D=D, lens=list(lens), S=S,
                seed=seed, scaling=D ** -0.5, q_seed=seed * 1000 + 1,
                k_seed=seed * 1000 + 2, v_seed=seed * 1000 + 3,
                input_digest=sha(bf16_bits(q)) + sha(bf16_bits(k)) + sha(bf16_bits(v)),
                num_blocks=cfg["num_blocks"], max_seq_len=cfg["max_seq_len"],
                max_requests=cfg["max_requests"], pool_digest=digest,
                reference_fn="qwen3/attention.py:Qwen3Attention._standard_attention")
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"),
        meta=np.array(json.dumps(meta)),
        out_packed_f16=packed.astype(np.float16),
        row_ids=np.array([c.row_id for c in caches], dtype=np.int32),
        block_table_2d=pool.block_table_2d.numpy().astype(np.int32),
    )
    print(f"{name}: lens={lens} T={packed.shape[0]} |out|max={np.abs(packed).max():.4f}")


def make_norm_rope(ref):
    torch = ref["torch"]
    RMSNorm, RotaryEmbedding, apply_rope = ref["RMSNorm"], ref["RotaryEmbedding"], ref["apply_rope"]
    B, H, Hkv, S, D = 2, 4, 2, 9, 128
    q = synth.det_normal(801, (B, H, S, D))
    k = synth.det_normal(802, (B, Hkv, S, D))
    norm = RMSNorm(D, 1e-6)
    rope = RotaryEmbedding(D, 1e6, max_seq_len=4096)
    pos = np.stack([np.arange(S) + 100, np.arange(S) + 3000]).astype(np.int64)
    with torch.no_grad():
        qn = norm(torch.from_numpy(q))
        kn = norm(torch.from_numpy(k))
        cos, sin = rope(torch.from_numpy(pos))
        qr, kr = apply_rope(qn, kn, cos, sin)
    meta = dict(case="norm_rope", seed_q=801, seed_k=802, D=D, theta=1e6, eps=1e-6,
                reference_fn="qwen3/norm.py:RMSNorm, qwen3/rope.py:RotaryEmbedding/apply_rotary_pos_emb")
    np.savez_compressed(os.path.join(HERE, "norm_rope.npz"), meta=np.array(json.dumps(meta)),
                        positions=pos, q_norm=qn.numpy(), k_norm=kn.numpy(),
                        q_rope=qr.numpy(), k_rope=kr.numpy(), cos=cos.numpy(), sin=sin.numpy())
    print("norm_rope: ok")


def make_norm_rope_bf16(ref):
    """The reference's QK-norm + RoPE modules on bf16 tensors (its serving dtype)."""
    torch = ref["torch"]
    RMSNorm, RotaryEmbedding, apply_rope = ref["RMSNorm"], ref["RotaryEmbedding"], ref["apply_rope"]
    B, H, Hkv, S, D = 3, 4, 2, 5, 128
    q = synth.det_normal(811, (B, H, S, D)).astype(np.float32) * 2.0
    k = synth.det_normal(812, (B, Hkv, S, D)).astype(np.float32)
    wq = 1.0 + 0.1 * synth.det_normal(813, (D,)).astype(np.float32)
    wk = 1.0 + 0.1 * synth.det_normal(814, (D,)).astype(np.float32)
    seq = np.array([0, 37, 250], dtype=np.int64)          # positions start per request
    pos = seq[:, None] + np.arange(S)[None]                 # (B, S)
    bf = torch.bfloat16
    qn_mod, kn_mod = RMSNorm(D, 1e-6), RMSNorm(D, 1e-6)
    with torch.no_grad():
        qn_mod.weight.copy_(torch.from_numpy(wq))
        kn_mod.weight.copy_(torch.from_numpy(wk))
        qn_mod, kn_mod = qn_mod.to(bf), kn_mod.to(bf)
        rope = RotaryEmbedding(D, 1e6, max_seq_len=512)
        qb = torch.from_numpy(q).to(bf)
        kb = torch.from_numpy(k).to(bf)
        cos, sin = rope(torch.from_numpy(pos))
        qr, kr = apply_rope(qn_mod(qb), kn_mod(kb), cos, sin)
    as_bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    meta = dict(case="norm_rope_bf16", seeds=[811, 812, 813, 814], D=D, theta=1e6, eps=1e-6,
                B=B, H=H, Hkv=Hkv, S=S, seq_lens=seq.tolist(),
                reference_fn="qwen3/norm.py:RMSNorm (bf16 weight), qwen3/rope.py:"
                             "RotaryEmbedding/apply_rotary_pos_emb on bf16 q/k")
    np.savez_compressed(os.path.join(HERE, "norm_rope_bf16.npz"), meta=np.array(json.dumps(meta)),
                        q_bits=as_bits(qb), k_bits=as_bits(kb),
                        wq_bits=as_bits(qn_mod.weight.data), wk_bits=as_bits(kn_mod.weight.data),
                        cos=cos.numpy(), sin=sin.numpy(),
                        q_rope_bits=as_bits(qr), k_rope_bits=as_bits(kr))
    print("norm_rope_bf16: ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("QWEN3_REFERENCE"),
                    help="path of the reference repository checkout")
    ap.add_argument("--only", default=None, help="generate only this fixture (e.g. norm_rope_bf16)")
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        sys.exit("make_golden.py: pass --reference <path> (the reference checkout)")
    sys.path.insert(0, args.reference)
    import torch
    from qwen3.PagedKVcache import KVCachePool, PagedKVCache
    from qwen3.paged_attention import paged_attention
    from qwen3.attention import Qwen3Attention
    from qwen3.config import Qwen3Config
    from qwen3.norm import RMSNorm
    from qwen3.rope import RotaryEmbedding, apply_rotary_pos_emb
    torch.set_num_threads(1)
    ref = dict(torch=torch, KVCachePool=KVCachePool, PagedKVCache=PagedKVCache,
               paged_attention=paged_attention, Qwen3Attention=Qwen3Attention,
               Qwen3Config=Qwen3Config, RMSNorm=RMSNorm, RotaryEmbedding=RotaryEmbedding,
               apply_rope=apply_rotary_pos_emb)
    want = (lambda name: args.only is None or args.only == name)
    for name, cfg in DECODE_CASES.items():
        if want(name):
            make_decode_case(name, cfg, ref)
    for name, cfg in PREFILL_CASES.items():
        if want(name):
            make_prefill_case(name, cfg, ref)
    if want("norm_rope"):
        make_norm_rope(ref)
    if want("norm_rope_bf16"):
        make_norm_rope_bf16(ref)


if __name__ == "__main__":
    main()
