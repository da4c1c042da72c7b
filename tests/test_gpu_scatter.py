"""KV-cache slot scatter on the GPU vs the oracle and the reference's pool bytes (bit-exact)."""

import numpy as np
import pytest
import torch

import golden_cases as gc
from oracle import attention as oa
from oracle import synth

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16(x: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device).to(torch.bfloat16)


@pytest.mark.parametrize("name", gc.case_names("decode"))
def test_reference_write_sequence_bitexact(name, cuda, native_lib):
    """Replay the fixture's PagedKVCache.update prefix + decode write through the
    B200 pool mirror: block tables and pool bytes equal the reference's."""
    import qwen3_engine_from_scratch_b200 as qb
    case = gc.load(name)
    m = case["meta"]
    inp = gc.decode_inputs(case)
    pool = qb.KVCachePool(m["num_blocks"], m["num_layers"], 16, m["Hkv"], m["D"], device=cuda,
                          dtype=torch.bfloat16, max_seq_len=m["max_seq_len"],
                          max_requests=m["max_requests"])
    pool.free_block_ids = [int(x) for x in synth.det_permutation(m["seed"] + 1, m["num_blocks"])]
    qb.clear_device_status()
    caches = []
    for b, (k, v) in enumerate(inp["ctx"]):
        c = qb.PagedKVCache(pool)
        if k is not None:
            c.update(m["layer"], _bf16(k, cuda), _bf16(v, cuda))
            c.advance_seq_len(k.shape[2])
        caches.append(c)
    assert [c.row_id for c in caches] == case["row_ids"].tolist()
    assert gc.pool_digest(_bits(pool.k_buffer), _bits(pool.v_buffer)) == m["pool_digest_prefix"]
    for c in caches:
        c.reserve_next()
    rows = torch.tensor([c.row_id for c in caches], dtype=torch.int32, device=cuda)
    pool.update_kv_batch(m["layer"], _bf16(inp["k_new"], cuda)[:, :, None],
                         _bf16(inp["v_new"], cuda)[:, :, None], rows)
    torch.cuda.synchronize()
    assert np.array_equal(pool.block_table_2d.cpu().numpy(), case["block_table_2d"])
    assert gc.pool_digest(_bits(pool.k_buffer), _bits(pool.v_buffer)) == m["pool_digest_final"]
    qb.check_device_status()


@pytest.mark.parametrize("name", gc.case_names("prefill"))
def test_batched_prefill_write_bitexact(name, cuda, native_lib):
    """update_batch (one launch) == the reference's per-request update loop."""
    import qwen3_engine_from_scratch_b200 as qb
    case = gc.load(name)
    m = case["meta"]
    inp = gc.prefill_inputs(case)
    pool = qb.KVCachePool(m["num_blocks"], 1, 16, m["Hkv"], m["D"], device=cuda,
                          dtype=torch.bfloat16, max_seq_len=m["max_seq_len"],
                          max_requests=m["max_requests"])
    pool.free_block_ids = [int(x) for x in synth.det_permutation(m["seed"] + 1, m["num_blocks"])]
    caches = [qb.PagedKVCache(pool) for _ in m["lens"]]
    pool.update_batch(caches, 0, _bf16(inp["k"], cuda), _bf16(inp["v"], cuda))
    torch.cuda.synchronize()
    assert np.array_equal(pool.block_table_2d.cpu().numpy(), case["block_table_2d"])
    assert gc.pool_digest(_bits(pool.k_buffer), _bits(pool.v_buffer)) == m["pool_digest"]


def _fused_qkv(B, S, H, Hkv, D, seed, device):
    """k/v as the strided slices of a fused qkv projection (qwen3/attention.py:82-88)."""
    W = (H + 2 * Hkv) * D
    qkv = _bf16(synth.det_normal(seed, (B, S, W)), device)
    k = qkv[..., H * D:(H + Hkv) * D].view(B, S, Hkv, D).transpose(1, 2)
    v = qkv[..., (H + Hkv) * D:].view(B, S, Hkv, D).transpose(1, 2)
    return k, v


@pytest.mark.parametrize("S", [1, 7, 40])
def test_rows_scatter_strided_inputs_bitexact(S, cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    B, H, Hkv, D, nb, nl, layer = 5, 16, 8, 128, 64, 3, 2
    k, v = _fused_qkv(B, S, H, Hkv, D, 31 + S, cuda)
    assert not k.is_contiguous()
    max_pages = 8
    perm = synth.det_permutation(5, nb)
    bt = np.full((9, max_pages), -1, np.int32)
    rows = np.array([8, 3, 0, 5, 1], np.int32)
    seq = np.zeros(9, np.int32)
    start = np.array([0, 15, 16, 33, 70], np.int32)
    seq[rows] = start
    used = 0
    for r, s0 in zip(rows, start):
        need = (int(s0) + S + 15) // 16
        bt[r, :need] = perm[used:used + need]
        used += need
    kp = torch.zeros(nb, nl, Hkv, 16, D, dtype=torch.bfloat16, device=cuda)
    vp = torch.zeros_like(kp)
    qb.clear_device_status()
    qb.kv_scatter_rows(k, v, kp, vp, torch.from_numpy(seq).to(cuda), torch.from_numpy(bt).to(cuda),
                       torch.from_numpy(rows).to(cuda), layer)
    torch.cuda.synchronize()
    qb.check_device_status()
    kr = np.zeros((nb, nl, Hkv, 16, D), np.float32)
    vr = np.zeros_like(kr)
    oa.kv_scatter_rows(k.float().cpu().numpy(), v.float().cpu().numpy(), kr, vr, seq, bt, rows, layer)
    assert np.array_equal(_bits(kp), oa.bf16_bits(kr))
    assert np.array_equal(_bits(vp), oa.bf16_bits(vr))


@pytest.mark.parametrize("slot_dtype", [torch.int32, torch.int64])
def test_slot_scatter_bitexact_with_padding(slot_dtype, cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    T, Hkv, D, nb = 1000, 8, 128, 128
    kv = _bf16(synth.det_normal(77, (T, 2 * Hkv + 3, D)), cuda)  # strided token rows
    k, v = kv[:, :Hkv], kv[:, Hkv + 3:]
    slots = synth.det_permutation(9, nb * 16)[:T].astype(np.int64)
    slots[::37] = -1                      # padding tokens are skipped
    kp = torch.zeros(nb, 2, Hkv, 16, D, dtype=torch.bfloat16, device=cuda)
    vp = torch.zeros_like(kp)
    qb.clear_device_status()
    qb.kv_scatter_slots(k, v, kp, vp, torch.from_numpy(slots).to(cuda, slot_dtype), layer_idx=1)
    torch.cuda.synchronize()
    qb.check_device_status()
    kr = np.zeros((nb, 2, Hkv, 16, D), np.float32)
    vr = np.zeros_like(kr)
    oa.kv_scatter_slots(k.float().cpu().numpy(), v.float().cpu().numpy(), kr, vr, slots, 1)
    assert np.array_equal(_bits(kp), oa.bf16_bits(kr))
    assert np.array_equal(_bits(vp), oa.bf16_bits(vr))


def test_scatter_bad_indices_are_flagged_not_written(cuda, native_lib):
    """-1 pages, rows past the table and slots past the pool raise a device
    status bit and write nothing (the reference would write out of bounds)."""
    import qwen3_engine_from_scratch_b200 as qb
    Hkv, D, nb = 2, 128, 8
    kp = torch.zeros(nb, 1, Hkv, 16, D, dtype=torch.bfloat16, device=cuda)
    vp = torch.zeros_like(kp)
    k = torch.ones(3, Hkv, 1, D, dtype=torch.bfloat16, device=cuda)
    bt = torch.full((4, 2), -1, dtype=torch.int32, device=cuda)
    bt[1, 0] = 3
    seq = torch.tensor([0, 0, 0, 40], dtype=torch.int32, device=cuda)
    rows = torch.tensor([0, 7, 3], dtype=torch.int32, device=cuda)  # -1 page, bad row, overflow
    qb.clear_device_status()
    qb.kv_scatter_rows(k, k, kp, vp, seq, bt, rows, 0)
    torch.cuda.synchronize()
    bits = qb.device_status()
    assert bits & 0x1 and bits & 0x2 and bits & 0x8
    assert not kp.any() and not vp.any()
    qb.clear_device_status()
    slots = torch.tensor([nb * 16 + 3, -5], dtype=torch.int64, device=cuda)
    qb.kv_scatter_slots(k[:2, :, 0], k[:2, :, 0], kp, vp, slots)
    torch.cuda.synchronize()
    assert qb.device_status() & 0x4
    assert not kp.any()
    with pytest.raises(RuntimeError):
        qb.check_device_status()
    qb.clear_device_status()
    assert qb.device_status() == 0
    qb.check_device_status()


def test_scatter_rejects_wrong_dtype(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    kp = torch.zeros(4, 1, 2, 16, 128, dtype=torch.float16, device=cuda)
    k = torch.zeros(1, 2, 1, 128, dtype=torch.float16, device=cuda)
    t = torch.zeros(1, 1, dtype=torch.int32, device=cuda)
    with pytest.raises(AssertionError):
        qb.kv_scatter_rows(k, k, kp, kp, t[0], t, t[0], 0)
