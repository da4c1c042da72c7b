"""Reference-facing host API of the B200 attention hot path.

Each function keeps the name, argument meaning and error behaviour of the
reference function it replaces, so the reference engine can bind it in place
of its Triton kernels (see ``shim.py``):

==========================================  ==================================================
this module                                 reference (uphome/Qwen3-engine-from-scratch)
==========================================  ==================================================
``paged_attention_decode_triton``           qwen3/kernels/paged_attention.py:132-178
``triton_paged_attention_decode``           qwen3/kernels/paged_attention.py:181-219
``triton_paged_attention_decode_batch``     qwen3/kernels/paged_attention.py:222-289
``update_kv_batch_triton``                  qwen3/kernels/paged_attention.py:353-377
``flash_attention_prefill``                 qwen3/kernels/flash_attention_varlen.py:126-194
``flash_attention_prefill_batched``         qwen3/kernels/flash_attention_varlen.py:197-258
``kv_scatter_rows``                         PagedKVCache.update (qwen3/PagedKVcache.py:177-214)
                                            for a whole batch, one launch
``kv_scatter_slots``                        vLLM-style slot_mapping write (new entry point)
``kv_scatter_span``                         the write of PagedKVCache.update
                                            (qwen3/PagedKVcache.py:187-214), host position
==========================================  ==================================================

The ``triton_*`` names are kept only so existing call sites bind unchanged; no
Triton is involved.  Every call goes to the C-ABI library (``_native``); all
work is enqueued on the current torch CUDA stream with no host sync, so the
decode path can be captured in a CUDA graph.  Inputs outside the kernels'
contract raise ``AssertionError`` (as the reference's ``assert``s do) or
``RuntimeError`` (non-zero C status); there is no fallback path.
"""

from __future__ import annotations

import math
import threading

import torch

from . import _native

__all__ = [
    "paged_attention_decode_triton",
    "triton_paged_attention_decode",
    "triton_paged_attention_decode_batch",
    "update_kv_batch_triton",
    "flash_attention_prefill",
    "flash_attention_prefill_batched",
    "paged_decode",
    "paged_decode_kv_write",
    "kv_scatter_rows",
    "kv_scatter_slots",
    "kv_scatter_span",
    "paged_cache_update",
    "qk_norm_rope_kv_write",
    "paged_prefill",
    "sample_tokens",
    "device_status",
    "clear_device_status",
    "check_device_status",
    "decode_workspace_bytes",
]

HEAD_DIM = 128
BLOCK_SIZE = 16

# ---------------------------------------------------------------------------
# device status word (one int32 per device, OR-ed by the kernels on bad input)
# ---------------------------------------------------------------------------

_status_lock = threading.Lock()
_status: dict[int, torch.Tensor] = {}


def _status_ptr(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        with _status_lock:
            t = _status.get(idx)
            if t is None:
                t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
                _status[idx] = t
    return t.data_ptr()


def device_status(device=None) -> int:
    """Read (with a sync) the error bits the kernels set on ``device``."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    _status_ptr(device)
    return int(_status[device.index if device.index is not None else torch.cuda.current_device()].item())


def clear_device_status(device=None) -> None:
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    _status_ptr(device)
    _status[device.index if device.index is not None else torch.cuda.current_device()].zero_()


def check_device_status(device=None) -> None:
    """Raise RuntimeError if a kernel met an out-of-range index since the last clear."""
    bits = device_status(device)
    if bits:
        raise RuntimeError(f"b200 attention kernels reported: {_native.describe_dev_status(bits)} "
                           f"(status bits {bits:#x})")


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _aligned(t: torch.Tensor, *dims: int) -> bool:
    """16-byte aligned base and every listed stride a multiple of 8 elements."""
    return t.data_ptr() % 16 == 0 and all(t.stride(d) % 8 == 0 for d in dims)


def _vec_ready(t: torch.Tensor, *dims: int) -> torch.Tensor:
    """Return ``t`` if the kernels can read it with 16-byte vectors, else a contiguous copy."""
    if t.stride(-1) == 1 and _aligned(t, *dims):
        return t
    return t.contiguous()


def _check_pool(k_buffer: torch.Tensor, v_buffer: torch.Tensor) -> None:
    assert k_buffer.is_cuda and v_buffer.is_cuda, "b200 kernels need CUDA tensors"
    assert k_buffer.dtype == torch.bfloat16 and v_buffer.dtype == torch.bfloat16, \
        "b200 kernels support bf16 KV pools only"
    assert k_buffer.shape == v_buffer.shape, "k_buffer / v_buffer shapes differ"
    assert k_buffer.stride(-1) == 1 and v_buffer.stride(-1) == 1, "pool head_dim must be contiguous"


def _check_table(block_table_2d: torch.Tensor, seq_lens: torch.Tensor, row_ids: torch.Tensor) -> None:
    for name, t in (("block_table_2d", block_table_2d), ("seq_lens", seq_lens), ("row_ids", row_ids)):
        assert t.dtype == torch.int32, f"{name} must be int32 (got {t.dtype})"
        assert t.is_cuda, f"{name} must be on the GPU"
    assert block_table_2d.dim() == 2 and block_table_2d.stride(1) == 1, \
        "block_table_2d must be (max_requests, max_pages) with contiguous rows"
    assert seq_lens.is_contiguous() and row_ids.is_contiguous(), "seq_lens/row_ids must be contiguous"


# ---------------------------------------------------------------------------
# KV scatter
# ---------------------------------------------------------------------------


def kv_scatter_rows(k_new, v_new, k_buffer, v_buffer, seq_lens, block_table_2d, row_ids, layer_idx):
    """Write S tokens per request into the paged pool in one launch.

    k_new, v_new: (B, Hkv, S, D) bf16, any strides with a contiguous head_dim
    (views of the fused qkv projection are fine).  Request b's token s lands at
    position ``seq_lens[row_ids[b]] + s`` -- exactly PagedKVCache.update
    (qwen3/PagedKVcache.py:187-214) for every request of the batch, and
    update_kv_batch_triton (qwen3/kernels/paged_attention.py:324-350) for S == 1.
    Pages must already be allocated in ``block_table_2d``.
    """
    assert k_new.dim() == 4 and k_new.shape == v_new.shape, "k_new/v_new must be (B, Hkv, S, D)"
    assert k_new.dtype == torch.bfloat16 and v_new.dtype == torch.bfloat16, "bf16 only"
    _check_pool(k_buffer, v_buffer)
    _check_table(block_table_2d, seq_lens, row_ids)
    B, Hkv, S, D = k_new.shape
    nb, nl, hkv_p, bs, d_p = k_buffer.shape
    assert Hkv == hkv_p and D == d_p, "k_new heads/head_dim do not match the pool"
    assert row_ids.numel() == B, "row_ids must have one entry per request"
    k_new = _vec_ready(k_new, 0, 1, 2)
    v_new = _vec_ready(v_new, 0, 1, 2)
    lib = _native.load()
    st = lib.b200_kv_scatter_rows(
        k_new.data_ptr(), v_new.data_ptr(),
        k_new.stride(0), k_new.stride(1), k_new.stride(2),
        v_new.stride(0), v_new.stride(1), v_new.stride(2),
        k_buffer.data_ptr(), v_buffer.data_ptr(),
        k_buffer.stride(0), k_buffer.stride(1), k_buffer.stride(2), k_buffer.stride(3),
        v_buffer.stride(0), v_buffer.stride(1), v_buffer.stride(2), v_buffer.stride(3),
        seq_lens.data_ptr(), block_table_2d.data_ptr(), block_table_2d.stride(0), row_ids.data_ptr(),
        B, S, Hkv, D, bs, nb, block_table_2d.shape[1], block_table_2d.shape[0], int(layer_idx),
        _status_ptr(k_buffer.device), _stream())
    _native.check(st, "b200_kv_scatter_rows")


def kv_scatter_span(k_new, v_new, k_buffer, v_buffer, block_table_row, num_pages, start_pos,
                    layer_idx):
    """Write one request's S tokens from the host position ``start_pos``.

    The byte movement of PagedKVCache.update (qwen3/PagedKVcache.py:198-214):
    token s lands at position ``start_pos + s`` through ``block_table_row``
    (the handle's row of the 2-D block table, ``num_pages`` entries allocated).
    k_new, v_new: (Hkv, S, D) bf16, any strides with a contiguous head_dim.
    A position past ``num_pages`` pages is flagged in the device status and
    skipped (the reference's indexing would raise).  One launch.
    """
    assert k_new.dim() == 3 and k_new.shape == v_new.shape, "k_new/v_new must be (Hkv, S, D)"
    assert k_new.dtype == torch.bfloat16 and v_new.dtype == torch.bfloat16, "bf16 only"
    _check_pool(k_buffer, v_buffer)
    assert block_table_row.dtype == torch.int32 and block_table_row.is_cuda, \
        "block_table_row must be an int32 GPU tensor"
    assert block_table_row.dim() == 1 and block_table_row.stride(0) == 1, \
        "block_table_row must be one contiguous row of the block table"
    Hkv, S, D = k_new.shape
    nb, nl, hkv_p, bs, d_p = k_buffer.shape
    assert Hkv == hkv_p and D == d_p, "k_new heads/head_dim do not match the pool"
    assert 0 <= int(num_pages) <= block_table_row.numel(), "num_pages outside the block-table row"
    k_new = _vec_ready(k_new, 0, 1)
    v_new = _vec_ready(v_new, 0, 1)
    st = _native.load().b200_kv_scatter_span(
        k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), k_new.stride(1),
        v_new.stride(0), v_new.stride(1), k_buffer.data_ptr(), v_buffer.data_ptr(),
        k_buffer.stride(0), k_buffer.stride(1), k_buffer.stride(2), k_buffer.stride(3),
        v_buffer.stride(0), v_buffer.stride(1), v_buffer.stride(2), v_buffer.stride(3),
        block_table_row.data_ptr(), int(num_pages), int(start_pos), S, Hkv, D, bs, nb,
        int(layer_idx), _status_ptr(k_buffer.device), _stream())
    _native.check(st, "b200_kv_scatter_span")


def paged_cache_update(cache, layer_idx, k_new, v_new):
    """``PagedKVCache.update`` (qwen3/PagedKVcache.py:177-214) on the scatter kernel.

    ``cache`` is a request handle with the reference's attributes (``_pool``,
    ``seq_len``, ``block_table``, ``num_pages``, ``block_table_tensor``,
    ``_allocate_block``): the reference's own class or this package's mirror.
    Same steps as the reference: pages for ``ceil((seq_len + S_new) / 16)``
    positions are allocated first (host bookkeeping, :193-195), then request
    0's S_new tokens are written from position ``seq_len`` (:198-214) -- in one
    launch instead of two torch ``index_put`` plus their index arithmetic.
    k_new, v_new: (B, Hkv, S_new, D) bf16 on the GPU; as in the reference only
    ``k_new[0]`` / ``v_new[0]`` are written.  ``seq_len`` is not advanced.
    """
    pool = cache._pool
    S_new = k_new.shape[2]
    write_pos = int(cache.seq_len)
    need_blocks = (write_pos + S_new + pool.block_size - 1) // pool.block_size
    while len(cache.block_table) < need_blocks:
        cache._allocate_block()
    kv_scatter_span(k_new[0], v_new[0], pool.k_buffer, pool.v_buffer, cache.block_table_tensor,
                    cache.num_pages, write_pos, layer_idx)


def update_kv_batch_triton(k_new, v_new, k_buffer, v_buffer, seq_lens, block_table_2d, row_ids,
                           layer_idx):
    """Decode KV write (qwen3/kernels/paged_attention.py:353-377).

    k_new, v_new: (B, num_kv_heads, head_dim) bf16, explicit strides allowed
    (the reference's non-contiguous qkv slices, :319-322).  Writes token
    ``seq_lens[row_ids[b]]`` of every request into the (5-D) pool in place.
    """
    kv_scatter_rows(k_new.unsqueeze(2), v_new.unsqueeze(2), k_buffer, v_buffer, seq_lens,
                    block_table_2d, row_ids, layer_idx)


def qk_norm_rope_kv_write(q, k, v, q_weight, k_weight, cos, sin, eps=1e-6, k_buffer=None,
                          v_buffer=None, seq_lens=None, block_table_2d=None, row_ids=None,
                          layer_idx=0, return_k=False):
    """Fused QK-RMSNorm + RoPE + KV-cache write (one launch).

    Replaces ``q_norm``/``k_norm`` and ``apply_rotary_pos_emb`` of
    qwen3/attention.py:90-95 and the KV write that follows it, with the
    reference's bf16 rounding steps (qwen3/norm.py:22-26, qwen3/rope.py:104-110).
    q: (B, H, S, D), k/v: (B, Hkv, S, D) bf16 views (e.g. of the fused qkv
    projection); q_weight/k_weight: (D,) bf16; cos/sin: the (B, S, D) fp32 rows of
    the reference's RotaryEmbedding for these tokens.  With the pool arguments
    given, token s of request b lands at position ``seq_lens[row_ids[b]] + s``
    (as ``kv_scatter_rows``).  Returns ``q_out`` (B, H, S, D), and the roped k
    as well when ``return_k``.
    """
    assert q.dim() == 4 and k.dim() == 4, "q/k must be (B, heads, S, D)"
    for name, t in (("q", q), ("k", k), ("q_weight", q_weight), ("k_weight", k_weight)):
        assert t.dtype == torch.bfloat16 and t.is_cuda, f"{name} must be bf16 on the GPU"
    assert cos.dtype == torch.float32 and sin.dtype == torch.float32, "cos/sin must be fp32"
    B, H, S, D = q.shape
    Hkv = k.shape[1]
    assert k.shape == (B, Hkv, S, D) and D == HEAD_DIM, "k shape / head_dim mismatch"
    assert cos.shape == (B, S, D) and sin.shape == cos.shape, "cos/sin must be (B, S, D)"
    assert cos.stride() == sin.stride(), "cos/sin must share strides"
    q = q if q.stride(-1) == 1 else q.contiguous()
    k = k if k.stride(-1) == 1 else k.contiguous()
    cos = cos if cos.stride(-1) == 1 else cos.contiguous()
    sin = sin if sin.stride() == cos.stride() else sin.contiguous()
    q_weight = q_weight.contiguous()
    k_weight = k_weight.contiguous()
    q_out = torch.empty((B, H, S, D), dtype=torch.bfloat16, device=q.device)
    k_out = torch.empty((B, Hkv, S, D), dtype=torch.bfloat16, device=q.device) if return_k else None
    pool = k_buffer is not None
    if pool:
        assert v is not None and v.shape == k.shape and v.dtype == torch.bfloat16
        _check_pool(k_buffer, v_buffer)
        _check_table(block_table_2d, seq_lens, row_ids)
        assert k_buffer.dim() == 5 and k_buffer.shape[2] == Hkv and k_buffer.shape[4] == D, \
            "pool must be (num_blocks, num_layers, Hkv, block_size, D)"
        assert row_ids.numel() == B, "row_ids must have one entry per request"
        v = v if v.stride(-1) == 1 else v.contiguous()
    lib = _native.load()
    nul = (None, 0, 0, 0)
    kb = k_buffer if pool else None
    vb = v_buffer if pool else None
    st = lib.b200_qk_norm_rope_kv_write(
        q.data_ptr(), q.stride(0), q.stride(1), q.stride(2),
        k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
        *((v.data_ptr(), v.stride(0), v.stride(1), v.stride(2)) if pool else nul),
        q_weight.data_ptr(), k_weight.data_ptr(), float(eps),
        cos.data_ptr(), sin.data_ptr(), cos.stride(0), cos.stride(1),
        q_out.data_ptr(), q_out.stride(0), q_out.stride(1), q_out.stride(2),
        *((k_out.data_ptr(), k_out.stride(0), k_out.stride(1), k_out.stride(2)) if return_k else nul),
        kb.data_ptr() if pool else None, vb.data_ptr() if pool else None,
        *((kb.stride(0), kb.stride(1), kb.stride(2), kb.stride(3)) if pool else (0, 0, 0, 0)),
        *((vb.stride(0), vb.stride(1), vb.stride(2), vb.stride(3)) if pool else (0, 0, 0, 0)),
        seq_lens.data_ptr() if pool else None, block_table_2d.data_ptr() if pool else None,
        block_table_2d.stride(0) if pool else 0, row_ids.data_ptr() if pool else None,
        B, S, H, Hkv, D, kb.shape[3] if pool else BLOCK_SIZE, kb.shape[0] if pool else 0,
        block_table_2d.shape[1] if pool else 0, block_table_2d.shape[0] if pool else 0,
        int(layer_idx), _status_ptr(q.device), _stream())
    _native.check(st, "b200_qk_norm_rope_kv_write")
    return (q_out, k_out) if return_k else q_out


def kv_scatter_slots(k, v, k_buffer, v_buffer, slot_mapping, layer_idx=0):
    """Packed (vLLM ``store_kvcache``-style) KV write.

    k, v: (T, Hkv, D) bf16; slot_mapping: (T,) int32/int64 with
    ``slot = phys_block * 16 + offset``; negative slots are skipped.
    """
    assert k.dim() == 3 and k.shape == v.shape, "k/v must be (T, Hkv, D)"
    assert k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16, "bf16 only"
    _check_pool(k_buffer, v_buffer)
    assert slot_mapping.dtype in (torch.int32, torch.int64) and slot_mapping.is_cuda
    T, Hkv, D = k.shape
    nb, nl, hkv_p, bs, d_p = k_buffer.shape
    assert Hkv == hkv_p and D == d_p, "k heads/head_dim do not match the pool"
    assert slot_mapping.numel() == T, "one slot per token"
    slot_mapping = slot_mapping.contiguous()
    k = _vec_ready(k, 0, 1)
    v = _vec_ready(v, 0, 1)
    st = _native.load().b200_kv_scatter_slots(
        k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
        k_buffer.data_ptr(), v_buffer.data_ptr(),
        k_buffer.stride(0), k_buffer.stride(1), k_buffer.stride(2), k_buffer.stride(3),
        v_buffer.stride(0), v_buffer.stride(1), v_buffer.stride(2), v_buffer.stride(3),
        slot_mapping.data_ptr(), int(slot_mapping.dtype == torch.int64),
        T, Hkv, D, bs, nb, int(layer_idx), _status_ptr(k_buffer.device), _stream())
    _native.check(st, "b200_kv_scatter_slots")


# ---------------------------------------------------------------------------
# paged decode
# ---------------------------------------------------------------------------


def decode_workspace_bytes(batch, num_heads, max_pages, pages_per_split=0) -> int:
    return int(_native.load().b200_paged_decode_workspace_size(batch, num_heads, max_pages,
                                                               pages_per_split))


_split_cache: dict[tuple[int, int, int, int], int] = {}
_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
_retired_workspaces: list[torch.Tensor] = []


def _decode_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """The decode workspace of (device, current stream), at least ``nbytes``.

    Zero-filled when allocated: its split-arrival counters must start at zero,
    and every decode launch leaves them zero, so launches on one stream (also
    inside captured graphs) reuse it.  A grown workspace replaces the old one,
    which is kept alive because a captured graph may still point at it.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(idx).cuda_stream)
    t = _workspaces.get(key)
    if t is None or t.numel() < nbytes:
        with _ws_lock:
            t = _workspaces.get(key)
            if t is None or t.numel() < nbytes:
                size = max(nbytes, 2 * t.numel() if t is not None else 0)
                if t is not None:
                    _retired_workspaces.append(t)
                t = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
                _workspaces[key] = t
    return t


def _default_split(lib, batch, num_kv_heads, max_pages) -> int:
    key = (torch.cuda.current_device(), batch, num_kv_heads, max_pages)
    v = _split_cache.get(key)
    if v is None:
        v = int(lib.b200_paged_decode_default_split(batch, num_kv_heads, max_pages))
        _split_cache[key] = v
    return v


def paged_decode(q, k_buffer, v_buffer, block_table_2d, seq_lens, row_ids, scale,
                 out=None, pages_per_split=0):
    """Split-K paged decode on one layer view of the pool.

    q: (B, H, D) bf16 (strided views allowed); k_buffer/v_buffer:
    (num_blocks, Hkv, 16, D) layer views (``pool.k_buffer[:, layer]``).
    Returns (B, H, D) bf16.  ``scale`` multiplies q.k before the softmax.
    """
    assert q.dim() == 3, "q must be (B, num_heads, head_dim)"
    assert q.dtype == torch.bfloat16, "b200 decode supports bf16 only"
    assert k_buffer.dim() == 4, "k_buffer must be a (num_blocks, Hkv, block_size, D) layer view"
    _check_pool(k_buffer, v_buffer)
    _check_table(block_table_2d, seq_lens, row_ids)
    B, H, D = q.shape
    nb, Hkv, bs, d_p = k_buffer.shape
    assert d_p == D, "head_dim mismatch between q and the pool"
    assert k_buffer.stride() == v_buffer.stride(), "k/v pool views must share strides"
    assert row_ids.numel() == B, "row_ids must have one entry per request"
    q = _vec_ready(q, 0, 1)
    if out is None:
        out = torch.empty((B, H, D), dtype=torch.bfloat16, device=q.device)
    max_pages = block_table_2d.shape[1]
    lib = _native.load()
    if pages_per_split <= 0:
        pages_per_split = _default_split(lib, B, Hkv, max_pages)
    ws_bytes = lib.b200_paged_decode_workspace_size(B, H, max_pages, pages_per_split)
    ws = _decode_workspace(q.device, ws_bytes) if ws_bytes else None
    st = lib.b200_paged_decode(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_buffer.data_ptr(), v_buffer.data_ptr(),
        k_buffer.stride(0), k_buffer.stride(1), k_buffer.stride(2),
        block_table_2d.data_ptr(), block_table_2d.stride(0),
        seq_lens.data_ptr(), row_ids.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        B, H, Hkv, D, bs, nb, max_pages, block_table_2d.shape[0],
        float(scale), int(pages_per_split),
        ws.data_ptr() if ws is not None else None, ws_bytes,
        _status_ptr(q.device), _stream())
    _native.check(st, "b200_paged_decode")
    return out


def paged_decode_kv_write(q, k_new, v_new, k_buffer, v_buffer, block_table_2d, seq_lens, row_ids,
                          scale, out=None, pages_per_split=0):
    """One layer's decode step in one launch: the KV write of the new token
    (``kv_scatter_rows`` with one token) fused into the split-K decode.

    q: (B, H, D) bf16; k_new/v_new: (B, Hkv, D) bf16 (strided views allowed);
    k_buffer/v_buffer: (num_blocks, Hkv, 16, D) layer views of the pool
    (``pool.k_buffer[:, layer]``), written at position ``seq_lens[row]``.
    Returns (B, H, D) bf16, attending over ``seq_lens[row] + 1`` tokens.
    """
    assert q.dim() == 3, "q must be (B, num_heads, head_dim)"
    assert q.dtype == torch.bfloat16, "b200 decode supports bf16 only"
    assert k_new.dtype == torch.bfloat16 and v_new.dtype == torch.bfloat16, \
        "b200 decode supports bf16 only"
    assert k_buffer.dim() == 4, "k_buffer must be a (num_blocks, Hkv, block_size, D) layer view"
    _check_pool(k_buffer, v_buffer)
    _check_table(block_table_2d, seq_lens, row_ids)
    B, H, D = q.shape
    nb, Hkv, bs, d_p = k_buffer.shape
    assert d_p == D, "head_dim mismatch between q and the pool"
    assert k_buffer.stride() == v_buffer.stride(), "k/v pool views must share strides"
    assert row_ids.numel() == B, "row_ids must have one entry per request"
    assert k_new.shape == (B, Hkv, D) and v_new.shape == (B, Hkv, D), \
        "k_new/v_new must be (B, num_kv_heads, head_dim)"
    q = _vec_ready(q, 0, 1)
    k_new = _vec_ready(k_new, 0, 1)
    v_new = _vec_ready(v_new, 0, 1)
    if out is None:
        out = torch.empty((B, H, D), dtype=torch.bfloat16, device=q.device)
    max_pages = block_table_2d.shape[1]
    lib = _native.load()
    if pages_per_split <= 0:
        pages_per_split = _default_split(lib, B, Hkv, max_pages)
    ws_bytes = lib.b200_paged_decode_workspace_size(B, H, max_pages, pages_per_split)
    ws = _decode_workspace(q.device, ws_bytes) if ws_bytes else None
    st = lib.b200_paged_decode_kv_write(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_new.data_ptr(), k_new.stride(0), k_new.stride(1),
        v_new.data_ptr(), v_new.stride(0), v_new.stride(1),
        k_buffer.data_ptr(), v_buffer.data_ptr(),
        k_buffer.stride(0), k_buffer.stride(1), k_buffer.stride(2),
        block_table_2d.data_ptr(), block_table_2d.stride(0),
        seq_lens.data_ptr(), row_ids.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        B, H, Hkv, D, bs, nb, max_pages, block_table_2d.shape[0],
        float(scale), int(pages_per_split),
        ws.data_ptr() if ws is not None else None, ws_bytes,
        _status_ptr(q.device), _stream())
    _native.check(st, "b200_paged_decode_kv_write")
    return out


def paged_attention_decode_triton(q, k_buffer, v_buffer, block_table_2d, seq_lens_full, row_ids,
                                  block_size):
    """Bare decode entry (qwen3/kernels/paged_attention.py:132-178).

    q: (B, num_heads, head_dim) bf16; k_buffer/v_buffer: (num_blocks, Hkv,
    block_size, head_dim) layer views; block_table_2d (max_requests, max_pages)
    int32; seq_lens_full (max_requests,) int32 EXCLUDING the token written this
    step; row_ids (B,) int32.  Like the reference it uses scale 1/sqrt(head_dim)
    (:161).  Returns a new (B, num_heads, head_dim) bf16 tensor.
    """
    B, num_heads, head_dim = q.shape
    num_blocks, num_kv_heads, block_size_check, head_dim_check = k_buffer.shape
    assert block_size_check == block_size
    assert head_dim_check == head_dim
    assert v_buffer.shape == k_buffer.shape
    return paged_decode(q, k_buffer, v_buffer, block_table_2d, seq_lens_full, row_ids,
                        1.0 / math.sqrt(head_dim))


def _pool_of(cache):
    return cache._pool


def _row_ids_of(cache, device) -> torch.Tensor:
    """Device tensor [cache.row_id], built once per cache handle (the reference
    rebuilds it with an H2D copy every layer, kernels/paged_attention.py:204)."""
    t = getattr(cache, "_b200_row_ids", None)
    if t is None or t.device != device or int(getattr(cache, "_b200_row_id_src", -1)) != cache.row_id:
        t = torch.tensor([cache.row_id], dtype=torch.int32, device=device)
        cache._b200_row_ids = t
        cache._b200_row_id_src = cache.row_id
    return t


def triton_paged_attention_decode_batch(q, k_new, v_new, kv_caches, layer_idx, scaling,
                                        row_ids=None):
    """Batched decode step of one layer (qwen3/kernels/paged_attention.py:222-289).

    q: (B, H, 1, D) bf16; k_new/v_new: (B, Hkv, 1, D) bf16 (strided views OK);
    kv_caches: list of B PagedKVCache handles sharing one pool; row_ids: (B,)
    int32 device tensor of block-table rows (None: reserve_next + build here,
    as the reference's test path does, :257-264).  Writes the new K/V at
    ``seq_lens[row]`` (the scatter) and then attends over ``seq_lens[row] + 1``
    tokens.  Returns (B, 1, H*D).  Like the reference, ``scaling`` is accepted
    and ignored: its Triton path always scales q.k by 1/sqrt(head_dim)
    (qwen3/kernels/paged_attention.py:161), which for Qwen3 equals the
    caller's ``head_dim ** -0.5``.
    """
    assert q.shape[2] == 1, "decode kernel supports S == 1 only"
    assert q.dtype == torch.bfloat16, "decode kernel supports bf16 only"
    B = q.shape[0]
    assert len(kv_caches) == B, "kv_caches must have one entry per request"
    if row_ids is None:
        for c in kv_caches:
            c.reserve_next()
        row_ids = torch.tensor([c.row_id for c in kv_caches], dtype=torch.int32, device=q.device)
    pool = _pool_of(kv_caches[0])
    out = paged_decode_kv_write(q.squeeze(2), k_new.squeeze(2), v_new.squeeze(2),
                                pool.k_buffer[:, layer_idx], pool.v_buffer[:, layer_idx],
                                pool.block_table_2d, pool.seq_lens, row_ids,
                                1.0 / math.sqrt(q.shape[3]))
    num_heads, head_dim = q.shape[1], q.shape[3]
    return out.reshape(B, 1, num_heads * head_dim)


def triton_paged_attention_decode(q, k_new, v_new, kv_cache, layer_idx, scaling):
    """Single-request decode (qwen3/kernels/paged_attention.py:181-219): B == 1.

    ``scaling`` is accepted and ignored, as in the reference (its kernel entry
    uses 1/sqrt(head_dim), qwen3/kernels/paged_attention.py:161).
    """
    assert q.shape[2] == 1, "decode kernel supports S == 1 only"
    assert q.dtype == torch.bfloat16, "decode kernel supports bf16 only"
    row_ids = _row_ids_of(kv_cache, q.device)
    pool = _pool_of(kv_cache)
    out = paged_decode_kv_write(q.squeeze(2), k_new.squeeze(2), v_new.squeeze(2),
                                pool.k_buffer[:, layer_idx], pool.v_buffer[:, layer_idx],
                                pool.block_table_2d, pool.seq_lens, row_ids,
                                1.0 / math.sqrt(q.shape[3]))
    B, num_heads, head_dim = q.shape[0], q.shape[1], q.shape[3]
    return out.reshape(B, 1, num_heads * head_dim)


# ---------------------------------------------------------------------------
# varlen prefill
# ---------------------------------------------------------------------------


_counter_lock = threading.Lock()
_counters: dict[tuple[int, int], torch.Tensor] = {}


def _work_counter(device: torch.device) -> torch.Tensor:
    """The prefill kernel's work counter for (device, current stream).

    Two int32 that are zero at launch; the kernel hands out work items through
    them and its last CTA zeroes them again, so launches on one stream (also
    inside a captured graph) reuse the same pair.  Each stream gets its own
    pair, because launches on different streams may overlap.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(idx).cuda_stream)
    t = _counters.get(key)
    if t is None:
        with _counter_lock:
            t = _counters.get(key)
            if t is None:
                t = torch.zeros(2, dtype=torch.int32, device=torch.device("cuda", idx))
                _counters[key] = t
    return t


def _prefill(q, k, v, out, cu_seqlens, seq_lens_opt, max_seqlen, scale, num_heads, num_kv_heads,
             head_dim, zero_pad_rows):
    lib = _native.load()
    counter = _work_counter(q.device)
    st = lib.b200_varlen_prefill(
        q.data_ptr(), q.stride(0), q.stride(1),
        k.data_ptr(), k.stride(0), k.stride(1),
        v.data_ptr(), v.stride(0), v.stride(1),
        out.data_ptr(), out.stride(0), out.stride(1),
        cu_seqlens.data_ptr(), seq_lens_opt.data_ptr() if seq_lens_opt is not None else None,
        cu_seqlens.numel() - 1 if seq_lens_opt is None else seq_lens_opt.numel(),
        q.shape[0], int(max_seqlen), num_heads, num_kv_heads, head_dim, float(scale),
        int(zero_pad_rows), counter.data_ptr(), _status_ptr(q.device), _stream())
    _native.check(st, "b200_varlen_prefill")


def flash_attention_prefill(q, k, v, cu_seqlens, scale, num_heads, num_kv_heads, head_dim,
                            max_seqlen=None):
    """Varlen causal prefill (qwen3/kernels/flash_attention_varlen.py:126-194).

    q: (T, H, D), k/v: (T, Hkv, D) bf16 (token/head strides allowed);
    cu_seqlens: (num_seqs+1,) int32 on the GPU.  ``max_seqlen`` (keyword, new)
    avoids the reference's host sync (``cu_seqlens.cpu()``, :177-178); without
    it the longest length is read back like the reference does.
    Returns (T, H, D) bf16.
    """
    assert q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16, \
        "b200 prefill supports bf16 only"
    assert cu_seqlens.dtype == torch.int32 and cu_seqlens.is_cuda, "cu_seqlens must be int32 on GPU"
    assert q.shape[1] == num_heads and k.shape[1] == num_kv_heads and q.shape[2] == head_dim
    if max_seqlen is None:
        cu = cu_seqlens.cpu()
        max_seqlen = int((cu[1:] - cu[:-1]).max().item()) if cu.numel() > 1 else 0
    q = _vec_ready(q, 0, 1)
    k = _vec_ready(k, 0, 1)
    v = _vec_ready(v, 0, 1)
    out = torch.empty((q.shape[0], num_heads, head_dim), dtype=q.dtype, device=q.device)
    _prefill(q, k, v, out, cu_seqlens.contiguous(), None, max_seqlen, scale, num_heads,
             num_kv_heads, head_dim, False)
    return out


_scratch_lock = threading.Lock()
_scratches: dict[tuple[str, int, int], torch.Tensor] = {}


def _scratch(device: torch.device, name: str, nbytes: int) -> torch.Tensor:
    """A reusable uninitialised buffer of (name, device, current stream), at
    least ``nbytes`` (kept alive once handed out: a captured graph may use it)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (name, idx, torch.cuda.current_stream(idx).cuda_stream)
    t = _scratches.get(key)
    if t is None or t.numel() < nbytes:
        with _scratch_lock:
            t = _scratches.get(key)
            if t is None or t.numel() < nbytes:
                if t is not None:
                    _retired_workspaces.append(t)
                t = torch.empty(max(nbytes, 16), dtype=torch.uint8,
                                device=torch.device("cuda", idx))
                _scratches[key] = t
    return t


_SEED_COUNTER = 0


def _next_seed() -> int:
    """Per-call seed when none is given (qwen3/sampling.py:42-48)."""
    global _SEED_COUNTER
    _SEED_COUNTER += 1
    return (torch.initial_seed() + _SEED_COUNTER * 0x9E3779B1) & 0x7FFFFFFF


def _row_param(value, B, device, dtype):
    if isinstance(value, torch.Tensor):
        t = value.to(device=device, dtype=dtype)
        return t.expand(B).contiguous() if t.ndim == 0 else t.contiguous()
    if isinstance(value, (list, tuple)):
        return torch.tensor(value, device=device, dtype=dtype)
    return torch.full((B,), value, device=device, dtype=dtype)


def _host_list(value, B):
    if isinstance(value, torch.Tensor):
        return None if value.is_cuda else value.reshape(-1).tolist() * (B if value.ndim == 0 else 1)
    if isinstance(value, (list, tuple)):
        return list(value)
    return [value] * B


def sample_tokens(logits, temperature=0.0, top_k=0, top_p=1.0, seed=None):
    """Fused sampling of (B, V) logits -> (B, 1) int64 token ids, one launch
    (qwen3/sampling.py:234-270: the torch.topk + _sample_topk_kernel path, and
    the greedy argmax).  Parameters: scalars or per-row lists / tensors.

    temperature <= 0: argmax.  1 <= top_k <= 1024: top-k, top-p and Gumbel-max
    with the reference kernel's random stream for the same ``seed``.
    top_k == 0 with top_p == 1: temperature sampling over the whole vocabulary
    (the reference uses torch.multinomial there: same distribution, another
    stream).  top_k == 0 with top_p < 1 (a nucleus over the whole sorted
    vocabulary) is not supported and raises ValueError.
    """
    if logits.ndim != 2:
        raise ValueError(f"logits must be (B, V), got shape={tuple(logits.shape)}")
    assert logits.is_cuda and logits.dtype in (torch.float32, torch.bfloat16), \
        "logits must be fp32 or bf16 on the GPU"
    B, V = logits.shape
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    dev = logits.device
    temps, ks, ps = _host_list(temperature, B), _host_list(top_k, B), _host_list(top_p, B)
    if ks is not None and ps is not None and temps is not None:
        for t, k, p in zip(temps, ks, ps):
            if float(t) > 0 and int(k) == 0 and float(p) < 1.0:
                raise ValueError("top_k == 0 with top_p < 1 is not supported by the fused sampler")
            if float(t) > 0 and not (0 <= int(k) <= 1024):
                raise ValueError("top_k must be in [0, 1024]")
        sampled_k = [min(int(k), V) for t, k in zip(temps, ks) if float(t) > 0 and int(k) > 0]
        max_k = max(sampled_k) if sampled_k else 1
        block_k = max(16, 1 << (max_k - 1).bit_length())
    else:
        block_k = 1024        # device parameters: the largest k the kernel takes
    # a parameter shared by every row goes to the kernel as a scalar (no device array)
    scalar = lambda v: not isinstance(v, (torch.Tensor, list, tuple))
    t_t = None if scalar(temperature) else _row_param(temperature, B, dev, torch.float32)
    k_t = None if scalar(top_k) else _row_param(top_k, B, dev, torch.int32)
    p_t = None if scalar(top_p) else _row_param(top_p, B, dev, torch.float32)
    out = torch.empty(B, dtype=torch.int64, device=dev)
    if seed is None:
        seed = _next_seed()
    lib = _native.load()
    ws_bytes = int(lib.b200_sample_workspace_size(B, V, int(block_k)))
    ws = _scratch(dev, "sample", ws_bytes)
    ptr = lambda t: t.data_ptr() if t is not None else None
    st = lib.b200_sample_tokens(logits.data_ptr(), int(logits.dtype == torch.bfloat16),
                                logits.stride(0), B, V, ptr(t_t), ptr(k_t), ptr(p_t),
                                float(temperature) if t_t is None else 0.0,
                                int(top_k) if k_t is None else 0,
                                float(top_p) if p_t is None else 1.0,
                                int(seed) & 0xFFFFFFFFFFFFFFFF, int(block_k),
                                ws.data_ptr(), ws_bytes, out.data_ptr(), _status_ptr(dev),
                                _stream())
    _native.check(st, "b200_sample_tokens")
    return out.unsqueeze(1)


def paged_prefill(q, k_buffer, v_buffer, block_table_2d, seq_lens, row_ids, cu_seqlens, scale,
                  max_new_tokens=None, out=None):
    """Chunked prefill over the paged KV cache (no reference counterpart: its
    prefill ignores cached context, qwen3/attention.py:109-120).

    q: (T, H, D) bf16, the packed new tokens of every sequence (cu_seqlens);
    k_buffer/v_buffer: (num_blocks, Hkv, 16, D) layer views of the pool, which
    already holds the new tokens' K/V at positions seq_lens[row] .. +len-1
    (e.g. written by ``qk_norm_rope_kv_write``).  Sequence i = pool row
    row_ids[i]; new token t attends to positions 0 .. seq_lens[row] + t.
    ``max_new_tokens`` (keyword) avoids reading the lengths back to the host.
    Returns (T, H, D) bf16.
    """
    assert q.dim() == 3 and q.dtype == torch.bfloat16, "q must be (T, H, D) bf16"
    assert k_buffer.dim() == 4, "k_buffer must be a (num_blocks, Hkv, block_size, D) layer view"
    _check_pool(k_buffer, v_buffer)
    _check_table(block_table_2d, seq_lens, row_ids)
    assert cu_seqlens.dtype == torch.int32 and cu_seqlens.is_cuda, "cu_seqlens must be int32 on GPU"
    T, H, D = q.shape
    nb, Hkv, bs, d_p = k_buffer.shape
    assert d_p == D and k_buffer.stride() == v_buffer.stride(), "pool views mismatch"
    n = cu_seqlens.numel() - 1
    assert row_ids.numel() == n, "row_ids must have one entry per sequence"
    if max_new_tokens is None:
        cu = cu_seqlens.cpu()
        max_new_tokens = int((cu[1:] - cu[:-1]).max().item()) if n > 0 else 0
    q = _vec_ready(q, 0, 1)
    if out is None:
        out = torch.empty((T, H, D), dtype=torch.bfloat16, device=q.device)
    lib = _native.load()
    st = lib.b200_paged_prefill(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_buffer.data_ptr(), v_buffer.data_ptr(),
        k_buffer.stride(0), k_buffer.stride(1), k_buffer.stride(2),
        block_table_2d.data_ptr(), block_table_2d.stride(0),
        seq_lens.data_ptr(), row_ids.data_ptr(), cu_seqlens.contiguous().data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        n, T, int(max_new_tokens), H, Hkv, D, bs, nb, block_table_2d.shape[1],
        block_table_2d.shape[0], float(scale), _work_counter(q.device).data_ptr(),
        _status_ptr(q.device), _stream())
    _native.check(st, "b200_paged_prefill")
    return out


def flash_attention_prefill_batched(q, k, v, lens, scaling, num_heads, num_kv_heads, head_dim):
    """Right-padded batch prefill (qwen3/kernels/flash_attention_varlen.py:197-258).

    q: (B, H, S, D), k/v: (B, Hkv, S, D) bf16; lens: list[int] of valid lengths.
    Returns (B, S, H*D) with zero rows at the padded positions.  Unlike the
    reference, the padded batch is read in place (token stride = the S stride)
    with per-sequence lengths: no permute, gather or scatter copies, no host
    sync.
    """
    B, H, S, D = q.shape
    assert len(lens) == B, "lens must have one entry per request"
    assert all(0 < l <= S for l in lens), "lens out of range (0 < lens_i <= S)"
    assert q.dtype == torch.bfloat16, "b200 prefill supports bf16 only"
    H_kv = k.shape[1]
    q2 = q.permute(0, 2, 1, 3)   # (B, S, H, D) views
    k2 = k.permute(0, 2, 1, 3)
    v2 = v.permute(0, 2, 1, 3)

    def flat(t):
        # (B, S, h, D) -> (B*S, h, D) without a copy when the batch stride is S * token stride
        if t.stride(0) == S * t.stride(1) and t.stride(-1) == 1:
            return t.as_strided((B * S, t.shape[2], D), (t.stride(1), t.stride(2), 1))
        return t.reshape(B * S, t.shape[2], D)

    qf, kf, vf = flat(q2), flat(k2), flat(v2)
    qf, kf, vf = _vec_ready(qf, 0, 1), _vec_ready(kf, 0, 1), _vec_ready(vf, 0, 1)
    out = torch.empty((B, S, H, D), dtype=q.dtype, device=q.device)
    cu = torch.arange(B + 1, dtype=torch.int32) * S
    lens_t = torch.tensor(list(lens), dtype=torch.int32)
    host = torch.cat([cu, lens_t]).pin_memory() if torch.cuda.is_available() else torch.cat([cu, lens_t])
    dev = host.to(q.device, non_blocking=True)
    _prefill(qf, kf, vf, out.view(B * S, H, D), dev[:B + 1], dev[B + 1:], S, scaling, num_heads,
             H_kv, head_dim, True)
    return out.reshape(B, S, H * D)
