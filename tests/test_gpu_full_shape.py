"""Full-shape decode parity and the reference-named entries that carry reference quirks.

* Config 2 at its real size (B = 64, L ~ U[128, 4096], a 32,768-block pool)
  through the fused KV-write decode that the batch entry calls: every request
  against the oracle, and the written rows bit-exact.
* One length-balanced (LPT) shard of config 4 (Qwen3-8B heads 32/8, 512
  requests of log-uniform [256, 32768] tokens split over 8 ranks) through
  ``triton_paged_attention_decode_batch``: longest, shortest and 8 random
  requests against the oracle, every output finite.
* ``paged_attention_decode_triton`` by name, and the reference's decode
  entries ignoring the caller's ``scaling`` (their kernel always uses
  1/sqrt(head_dim), qwen3/kernels/paged_attention.py:161).
* ``paged_cache_update`` (the bound ``PagedKVCache.update``) writing at the
  handle's host ``seq_len``, bit-exact against the oracle's write.

Tolerance (north_star): max-abs 2e-2 and mean-abs 2e-3 against fp32.
"""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oa
from oracle import synth
from test_gpu_decode import _bf16, _c2_like, _close, _golden_setup, _oracle_subset

pytestmark = pytest.mark.gpu

D = 128


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_config2_full_pool_fused_write_all_requests(cuda, native_lib):
    """Config 2 at full size through paged_decode_kv_write: all 64 requests vs the oracle."""
    import qwen3_engine_from_scratch_b200 as qb
    w = _c2_like(cuda, num_blocks=32768, seed=2024)
    B, H, Hkv = len(w["lens"]), w["H"], w["Hkv"]
    g = torch.Generator(device=cuda).manual_seed(7)
    k_new = torch.randn(B, Hkv, D, generator=g, device=cuda).to(torch.bfloat16)
    v_new = torch.randn(B, Hkv, D, generator=g, device=cuda).to(torch.bfloat16)
    qb.clear_device_status()
    out = qb.paged_decode_kv_write(w["q"], k_new, v_new, w["kp"], w["vp"], w["bt"], w["seq"],
                                   w["rows"], 1 / math.sqrt(D))
    torch.cuda.synchronize()
    qb.check_device_status()
    # the new token's K/V rows landed at position seq_lens[row] of each request
    pos = w["seq_np"][w["rows_np"]]
    phys = torch.from_numpy(w["bt_np"][w["rows_np"], pos // 16].astype(np.int64)).to(cuda)
    off = torch.from_numpy((pos % 16).astype(np.int64)).to(cuda)
    assert torch.equal(w["kp"][phys, :, off], k_new)
    assert torch.equal(w["vp"][phys, :, off], v_new)
    # every request against the oracle, on the pool after the write
    idx = np.arange(B)
    ref = _oracle_subset(w, idx)
    _close(out, ref)


def _c4_shard(device, world=8, seed=4321):
    """The heaviest LPT shard of config 4 as a pool of request handles."""
    import qwen3_engine_from_scratch_b200 as qb
    from qwen3_engine_from_scratch_b200.dist import decode_cost, lpt_partition, shard_loads
    rng = np.random.default_rng(seed)
    all_lens = np.exp(rng.uniform(np.log(256), np.log(32768), size=512)).astype(np.int64)
    shards = lpt_partition(decode_cost(all_lens), world)
    loads = shard_loads(decode_cost(all_lens), shards)
    mine = shards[int(np.argmax(loads))]
    lens = all_lens[mine]
    H, Hkv = 32, 8
    pages = int(((lens + 15) // 16).sum())
    pool = qb.KVCachePool(num_blocks=pages + 16, num_layers=1, block_size=16, num_kv_heads=Hkv,
                          head_dim=D, device=device, dtype=torch.bfloat16, max_seq_len=32768,
                          max_requests=len(lens) + 1)
    g = torch.Generator(device=device).manual_seed(seed)
    pool.free_block_ids = torch.randperm(pages + 16, generator=g, device=device).cpu().tolist()
    caches = []
    for L in lens:
        c = qb.PagedKVCache(pool)
        c._ensure_pages(int(L))           # the context and this step's token
        c.seq_len = int(L) - 1
        caches.append(c)
    rows = torch.tensor([c.row_id for c in caches], dtype=torch.int32, device=device)
    pool.seq_lens[rows.long()] = torch.from_numpy((lens - 1).astype(np.int32)).to(device)
    # N(0,1) K/V (K RMS-normed) in every allocated block, in chunks
    kp, vp = pool.k_buffer[:, 0], pool.v_buffer[:, 0]
    for s0 in range(0, pages + 16, 4096):
        s1 = min(pages + 16, s0 + 4096)
        kx = torch.randn(s1 - s0, Hkv, 16, D, generator=g, device=device)
        kp[s0:s1] = (kx * torch.rsqrt(kx.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
        vp[s0:s1] = torch.randn(s1 - s0, Hkv, 16, D, generator=g, device=device).to(torch.bfloat16)
    return pool, caches, rows, lens, H, Hkv


def test_config4_lpt_shard_vs_oracle(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    pool, caches, rows, lens, H, Hkv = _c4_shard(cuda)
    B = len(lens)
    g = torch.Generator(device=cuda).manual_seed(44)
    q = torch.randn(B, H, 1, D, generator=g, device=cuda)
    q = (q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    k_new = torch.randn(B, Hkv, 1, D, generator=g, device=cuda).to(torch.bfloat16)
    v_new = torch.randn(B, Hkv, 1, D, generator=g, device=cuda).to(torch.bfloat16)
    qb.clear_device_status()
    out = qb.triton_paged_attention_decode_batch(q, k_new, v_new, caches, 0, D ** -0.5, rows)
    torch.cuda.synchronize()
    qb.check_device_status()
    o = out.view(B, H, D)
    assert torch.isfinite(o.float()).all()
    rng = np.random.default_rng(1)
    pick = {int(np.argmax(lens)), int(np.argmin(lens))}
    pick |= set(rng.choice([i for i in range(B) if i not in pick], size=8, replace=False).tolist())
    idx = np.array(sorted(pick))
    w = dict(q=q[:, :, 0], kp=pool.k_buffer[:, 0], vp=pool.v_buffer[:, 0],
             rows_np=rows.cpu().numpy(), bt_np=pool.block_table_2d.cpu().numpy(),
             seq_np=pool.seq_lens.cpu().numpy())
    ref = _oracle_subset(w, idx)
    _close(o[torch.from_numpy(idx).to(cuda)], ref)


def test_bare_decode_entry_by_name(cuda, native_lib):
    """paged_attention_decode_triton (qwen3/kernels/paged_attention.py:132-178) by
    its own name on the reference fixture, after the decode write."""
    import qwen3_engine_from_scratch_b200 as qb
    case, m, inp, pool, caches = _golden_setup("decode_c1", cuda)
    for c in caches:
        c.reserve_next()
    rows = torch.tensor([c.row_id for c in caches], dtype=torch.int32, device=cuda)
    qb.update_kv_batch_triton(_bf16(inp["k_new"], cuda), _bf16(inp["v_new"], cuda),
                              pool.k_buffer, pool.v_buffer, pool.seq_lens, pool.block_table_2d,
                              rows, m["layer"])
    out = qb.paged_attention_decode_triton(_bf16(inp["q"], cuda), pool.k_buffer[:, m["layer"]],
                                           pool.v_buffer[:, m["layer"]], pool.block_table_2d,
                                           pool.seq_lens, rows, 16)
    assert out.shape == (len(caches), m["H"], m["D"])
    _close(out, case["out"])


@pytest.mark.parametrize("entry", ["batch", "single"])
def test_decode_entries_ignore_caller_scaling(entry, cuda, native_lib):
    """The reference's decode entries accept ``scaling`` but their kernel uses
    1/sqrt(head_dim); a caller's 0.5 must give the fixture's 1/sqrt(128) output."""
    import qwen3_engine_from_scratch_b200 as qb
    case, m, inp, pool, caches = _golden_setup("decode_c1", cuda)
    assert abs(m["scaling"] - 1 / math.sqrt(m["D"])) < 1e-12
    q = _bf16(inp["q"], cuda)[:, :, None]
    kn = _bf16(inp["k_new"], cuda)[:, :, None]
    vn = _bf16(inp["v_new"], cuda)[:, :, None]
    if entry == "batch":
        out = qb.triton_paged_attention_decode_batch(q, kn, vn, caches, m["layer"], 0.5)
    else:
        outs = []
        for b, c in enumerate(caches):
            c.reserve_next()
            outs.append(qb.triton_paged_attention_decode(q[b:b + 1], kn[b:b + 1], vn[b:b + 1], c,
                                                         m["layer"], 0.5))
        out = torch.cat(outs)
    _close(out, case["out"])


def test_paged_cache_update_writes_at_host_seq_len(cuda, native_lib):
    """The bound PagedKVCache.update writes from the handle's host seq_len (as the
    reference's arange(seq_len, seq_len + S) does), whatever the device seq_lens
    holds, and allocates its pages first: bit-exact against the oracle."""
    import qwen3_engine_from_scratch_b200 as qb
    nb, nl, Hkv, layer = 64, 2, 8, 1
    pool = qb.KVCachePool(nb, nl, 16, Hkv, D, device=cuda, dtype=torch.bfloat16,
                          max_seq_len=512, max_requests=4)
    pool.free_block_ids = [int(x) for x in synth.det_permutation(3, nb)]
    c = qb.PagedKVCache(pool)
    chunks = [(0, 37), (37, 1), (38, 90)]          # (host seq_len before, tokens written)
    kr = np.zeros((nb, nl, Hkv, 16, D), np.float32)
    vr = np.zeros_like(kr)
    qb.clear_device_status()
    for i, (start, S) in enumerate(chunks):
        kx = _bf16(synth.det_normal(50 + i, (1, Hkv, S, D)), cuda)
        vx = _bf16(synth.det_normal(60 + i, (1, Hkv, S, D)), cuda)
        c.seq_len = start
        pool.seq_lens[c.row_id] = 999               # stale device copy: must not be used
        qb.paged_cache_update(c, layer, kx, vx)
        assert c.num_pages == (start + S + 15) // 16
        bt = pool.block_table_2d.cpu().numpy()
        oa.kv_scatter_rows(kx.float().cpu().numpy(), vx.float().cpu().numpy(), kr, vr,
                           np.array([start], np.int32), bt[c.row_id:c.row_id + 1],
                           np.array([0], np.int32), layer)
    torch.cuda.synchronize()
    qb.check_device_status()
    assert np.array_equal(_bits(pool.k_buffer), oa.bf16_bits(kr))
    assert np.array_equal(_bits(pool.v_buffer), oa.bf16_bits(vr))
