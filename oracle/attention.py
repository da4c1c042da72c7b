"""numpy restatement of the reference attention hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may use
this module, and only as the checker / the timed CPU baseline.  The product
never routes through it.

All citations are ``path:line`` in the reference repository
(uphome/Qwen3-engine-from-scratch).  Arithmetic is float32 like the reference's
CPU fallback path, which is the parity oracle for the GPU kernels.
"""

from __future__ import annotations

import math

import numpy as np

# --------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, the rounding torch's .to(bfloat16) uses)
# --------------------------------------------------------------------------


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even; NaN kept quiet."""
    f = np.ascontiguousarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    rounding = ((u >> np.uint64(16)) & np.uint64(1)) + np.uint64(0x7FFF)
    r = ((u + rounding) >> np.uint64(16)).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        r = r.copy()
        r[nan] = np.uint16(0x7FC0)
    return r


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 values."""
    u = np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)
    return u.view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (result kept as float32)."""
    return from_bf16_bits(bf16_bits(x))


# --------------------------------------------------------------------------
# Input transforms: QK-RMSNorm and RoPE
# --------------------------------------------------------------------------


def rms_norm(x: np.ndarray, weight: np.ndarray | None = None, eps: float = 1e-6) -> np.ndarray:
    """RMSNorm over the last axis in float32 (qwen3/norm.py:22-26)."""
    xf = np.asarray(x, dtype=np.float32)
    rms = 1.0 / np.sqrt((xf * xf).mean(axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps))
    y = xf * rms.astype(np.float32)
    if weight is not None:
        y = y * np.asarray(weight, dtype=np.float32)
    return y.astype(np.float32)


def rope_cos_sin(positions: np.ndarray, head_dim: int, base: float = 1e6):
    """cos/sin rows for the given positions (qwen3/rope.py:42-58 table, :60-69 gather).

    inv_freq_i = 1 / base**(2i/d); angle = pos * inv_freq; the table is
    cat(freqs, freqs) so both halves share one frequency.
    """
    idx = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    inv_freq = (1.0 / (np.float32(base) ** idx)).astype(np.float32)
    pos = np.asarray(positions, dtype=np.float32)
    freqs = pos[..., None] * inv_freq                      # (..., d/2)
    emb = np.concatenate([freqs, freqs], axis=-1)          # (..., d)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x*cos + rotate_half(x)*sin with rotate_half = cat(-x2, x1) (qwen3/rope.py:71-110).

    ``x`` is (..., S, D) and cos/sin broadcast against it.
    """
    d = x.shape[-1]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    rot = np.concatenate([-x2, x1], axis=-1)
    return (x * cos + rot * sin).astype(np.float32)


def qk_norm_rope_bf16(x: np.ndarray, weight: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                      eps: float = 1e-6, return_terms: bool = False):
    """QK-RMSNorm then RoPE on bf16 tensors, with the reference's rounding steps.

    ``x``: (..., D) bf16 values held in float32; ``weight``: (D,) bf16 values;
    ``cos``/``sin``: fp32 rows broadcasting against ``x`` (the RotaryEmbedding
    gather).  Follows qwen3/norm.py:22-26 (fp32 norm, one cast to bf16) and
    qwen3/rope.py:104-110 (cos/sin cast to bf16, then ``x*cos + rotate_half(x)*sin``
    in bf16 arithmetic: every product and the sum rounded to bf16).  With
    ``return_terms`` also returns the two rounded products, whose magnitude
    bounds how far a one-ulp change of the normed input can move the output.
    """
    xf = np.asarray(x, dtype=np.float32)
    ms = (xf * xf).mean(axis=-1, keepdims=True, dtype=np.float32)
    rms = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    y = bf16_round(((xf * rms).astype(np.float32) * np.asarray(weight, np.float32)).astype(np.float32))
    c = bf16_round(np.asarray(cos, np.float32))
    s = bf16_round(np.asarray(sin, np.float32))
    d = y.shape[-1]
    rot = np.concatenate([-y[..., d // 2:], y[..., : d // 2]], axis=-1)
    a, b = bf16_round(y * c), bf16_round(rot * s)
    out = bf16_round(a + b)
    return (out, a, b) if return_terms else out


# --------------------------------------------------------------------------
# KV-cache slot scatter
# --------------------------------------------------------------------------


def kv_scatter_rows(k_new, v_new, k_pool, v_pool, seq_lens, block_table_2d, row_ids, layer_idx):
    """Write S new tokens per request into the paged pool, in place.

    Request b writes token s at logical position ``seq_lens[row_ids[b]] + s``:
    page = block_table_2d[row, pos // bs], slot = pos % bs.
      * S == 1 is the decode write ``update_kv_batch_kernel``
        (qwen3/kernels/paged_attention.py:324-350).
      * general S is ``PagedKVCache.update`` (qwen3/PagedKVcache.py:187-214),
        which writes all S positions (right-pad positions included).

    k_new/v_new: (B, Hkv, S, D); pools: (num_blocks, num_layers, Hkv, bs, D).
    """
    B, Hkv, S, D = k_new.shape
    bs = k_pool.shape[3]
    for b in range(B):
        row = int(row_ids[b])
        start = int(seq_lens[row])
        pos = np.arange(start, start + S)
        phys = block_table_2d[row, pos // bs].astype(np.int64)
        off = pos % bs
        k_pool[phys, layer_idx, :, off] = np.transpose(k_new[b], (1, 0, 2))
        v_pool[phys, layer_idx, :, off] = np.transpose(v_new[b], (1, 0, 2))


def kv_scatter_slots(k, v, k_pool, v_pool, slot_mapping, layer_idx):
    """vLLM-style packed scatter: token t -> slot ``slot_mapping[t] = phys*bs + off``.

    Same addressing as qwen3/PagedKVcache.py:198-214 with the (phys, off) pair
    flattened into one slot number; negative slots are skipped (padding).
    k, v: (T, Hkv, D).
    """
    bs = k_pool.shape[3]
    slots = np.asarray(slot_mapping, dtype=np.int64)
    keep = slots >= 0
    phys = slots[keep] // bs
    off = slots[keep] % bs
    k_pool[phys, layer_idx, :, off] = k[keep]
    v_pool[phys, layer_idx, :, off] = v[keep]


# --------------------------------------------------------------------------
# Paged decode attention
# --------------------------------------------------------------------------


def paged_decode(q, k_layer, v_layer, block_table_2d, seq_lens, row_ids, block_size, scaling):
    """Page-by-page online-softmax decode attention in float32.

    Follows qwen3/paged_attention.py:39-122 (the reference CPU path): for each
    physical page, zero the invalid slots (:92-96), expand KV heads for GQA
    (:98-99, repeat_kv :31-36), score = q.k * scaling with invalid slots at
    -inf (:103-104, padded mask :68-73), then the running-max update
    m' = max(m, page max), alpha = exp(m - m'), p = exp(s - m'),
    l = l*alpha + sum p, acc = acc*alpha + p@v (:108-118), out = acc / l (:121).
    The number of visible tokens is L = seq_lens[row] + 1 -- the current
    token was written by the scatter first -- as in
    qwen3/kernels/paged_attention.py:54-56.

    q: (B, H, D); k_layer/v_layer: (num_blocks, Hkv, bs, D).  Returns (B, H, D) f32.
    """
    q = np.asarray(q, dtype=np.float32)
    B, H, D = q.shape
    Hkv = k_layer.shape[1]
    G = H // Hkv
    out = np.empty((B, H, D), dtype=np.float32)
    slot_idx = np.arange(block_size)
    for b in range(B):
        row = int(row_ids[b])
        L = int(seq_lens[row]) + 1
        npages = (L + block_size - 1) // block_size
        m = np.full((H, 1), -np.inf, dtype=np.float32)
        l = np.zeros((H, 1), dtype=np.float32)
        acc = np.zeros((H, D), dtype=np.float32)
        qb = q[b]
        for j in range(npages):
            phys = int(block_table_2d[row, j])
            valid = min(block_size, L - j * block_size)
            keep = (slot_idx < valid).astype(np.float32)[None, :, None]
            kp = np.asarray(k_layer[phys], dtype=np.float32) * keep     # (Hkv, bs, D)
            vp = np.asarray(v_layer[phys], dtype=np.float32) * keep
            kp = np.repeat(kp, G, axis=0)                              # (H, bs, D)
            vp = np.repeat(vp, G, axis=0)
            s = np.einsum("hd,htd->ht", qb, kp).astype(np.float32) * np.float32(scaling)
            s[:, valid:] = -np.inf
            m_new = np.maximum(m, s.max(axis=-1, keepdims=True))
            alpha = np.exp(m - m_new)
            p = np.exp(s - m_new)
            l = l * alpha + p.sum(axis=-1, keepdims=True)
            acc = acc * alpha + np.einsum("ht,htd->hd", p, vp).astype(np.float32)
            m = m_new
        out[b] = acc / l
    return out


# --------------------------------------------------------------------------
# Varlen causal prefill attention
# --------------------------------------------------------------------------


def _causal_attention(qh, kh, vh, scale):
    """softmax(q k^T * scale + causal mask, fp32) @ v for one sequence.

    qh: (H, L, D), kh/vh: (H, L, D) (KV heads already expanded).  This is
    Qwen3Attention._standard_attention (qwen3/attention.py:193-207) with the
    causal mask of qwen3/model.py:150-161 restricted to the valid rows.
    """
    L = qh.shape[1]
    w = np.matmul(qh, np.transpose(kh, (0, 2, 1))).astype(np.float32) * np.float32(scale)
    mask = np.triu(np.ones((L, L), dtype=bool), k=1)
    w[:, mask] = -np.inf
    w = w - w.max(axis=-1, keepdims=True)
    e = np.exp(w)
    p = e / e.sum(axis=-1, keepdims=True)
    return np.matmul(p.astype(np.float32), vh).astype(np.float32)


def varlen_prefill(q, k, v, cu_seqlens, scale):
    """Causal attention inside each packed sequence (GQA), float32.

    Semantics of flash_attention_varlen_kernel
    (qwen3/kernels/flash_attention_varlen.py:25-123): sequence i owns rows
    cu[i]..cu[i+1]; q head h uses kv head h // (H/Hkv) (:46); query m sees keys
    n <= m of its own sequence (:95-96).  The arithmetic follows the reference's
    fp32 oracle _standard_attention (qwen3/attention.py:193-207).

    q: (T, H, D); k, v: (T, Hkv, D).  Returns (T, H, D) float32.
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    T, H, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    out = np.zeros((T, H, D), dtype=np.float32)
    for i in range(len(cu) - 1):
        s0, s1 = int(cu[i]), int(cu[i + 1])
        if s1 <= s0:
            continue
        qh = np.transpose(q[s0:s1], (1, 0, 2))
        kh = np.repeat(np.transpose(k[s0:s1], (1, 0, 2)), G, axis=0)
        vh = np.repeat(np.transpose(v[s0:s1], (1, 0, 2)), G, axis=0)
        out[s0:s1] = np.transpose(_causal_attention(qh, kh, vh, scale), (1, 0, 2))
    return out


def paged_prefill(q, k_pool, v_pool, block_table_2d, ctx_lens, row_ids, cu_seqlens, scale):
    """Chunked prefill over a paged cache (the prefix-continuation case the
    reference leaves open, qwen3/attention.py:109-120): the causal softmax of
    qwen3/attention.py:193-207 with the new tokens' positions offset by the
    cached context.  q (T, H, D); k_pool/v_pool one layer (num_blocks, Hkv, 16,
    D); sequence i = pool row row_ids[i] with ctx_lens[i] cached tokens and
    its new tokens at rows cu[i]..cu[i+1] of q, their K/V already in the pool.
    Returns (T, H, D) float32.
    """
    q = np.asarray(q, np.float32)
    T, H, D = q.shape
    Hkv = k_pool.shape[1]
    G = H // Hkv
    out = np.zeros((T, H, D), np.float32)
    for i in range(len(cu_seqlens) - 1):
        s0, s1 = int(cu_seqlens[i]), int(cu_seqlens[i + 1])
        n, c, row = s1 - s0, int(ctx_lens[i]), int(row_ids[i])
        if n == 0:
            continue
        total = c + n
        pages = block_table_2d[row, :(total + 15) // 16]
        k = np.asarray(k_pool[pages], np.float32).transpose(0, 2, 1, 3).reshape(-1, Hkv, D)[:total]
        v = np.asarray(v_pool[pages], np.float32).transpose(0, 2, 1, 3).reshape(-1, Hkv, D)[:total]
        kq = np.repeat(k, G, axis=1)                         # (total, H, D)
        vq = np.repeat(v, G, axis=1)
        sc = np.einsum("thd,jhd->htj", q[s0:s1], kq) * np.float32(scale)
        mask = np.arange(total)[None, :] <= (c + np.arange(n))[:, None]
        sc = np.where(mask[None], sc, -np.inf)
        sc = sc - sc.max(-1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(-1, keepdims=True)
        out[s0:s1] = np.einsum("htj,jhd->thd", p, vq)
    return out


def prefill_batched(q, k, v, lens, scaling):
    """Right-padded batch adapter (qwen3/kernels/flash_attention_varlen.py:197-258).

    q: (B, H, S, D); k, v: (B, Hkv, S, D); lens: valid length per request.
    Returns (B, S, H*D) float32 with zero rows at the padded positions (:255-257).
    """
    q = np.asarray(q, dtype=np.float32)
    B, H, S, D = q.shape
    G = H // k.shape[1]
    out = np.zeros((B, S, H, D), dtype=np.float32)
    for b in range(B):
        L = int(lens[b])
        kh = np.repeat(np.asarray(k[b, :, :L], dtype=np.float32), G, axis=0)
        vh = np.repeat(np.asarray(v[b, :, :L], dtype=np.float32), G, axis=0)
        o = _causal_attention(q[b, :, :L], kh, vh, scaling)       # (H, L, D)
        out[b, :L] = np.transpose(o, (1, 0, 2))
    return out.reshape(B, S, H * D)


# --------------------------------------------------------------------------
# Algorithmic work (roofline numerators)
# --------------------------------------------------------------------------


def decode_bytes(lens, num_heads, num_kv_heads, head_dim=128, block_size=16, elem=2):
    """Algorithmic HBM bytes of one batched decode call over visible lengths ``lens``.

    K and V of every visible token of every kv head, q read + out written,
    the block-table entry of every visible page (once per request), plus
    row_ids and seq_lens.
    """
    lens = np.asarray(lens, dtype=np.int64)
    B = len(lens)
    kv = int(lens.sum()) * num_kv_heads * head_dim * elem * 2
    qo = B * num_heads * head_dim * elem * 2
    tables = int(((lens + block_size - 1) // block_size).sum()) * 4
    return kv + qo + tables + B * 8


def prefill_flops(lens, num_heads, head_dim=128):
    """Causal attention FLOPs: 4*H*D per (query, visible key) pair, L(L+1)/2 pairs."""
    lens = np.asarray(lens, dtype=np.int64)
    return int((4 * num_heads * head_dim * (lens * (lens + 1) // 2)).sum())


def default_scale(head_dim: int) -> float:
    """head_dim ** -0.5 (qwen3/attention.py:46)."""
    return 1.0 / math.sqrt(head_dim)
