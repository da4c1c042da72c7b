"""GraphRunner on the GPU: captured decode steps replay exactly what the
model computes eagerly.

Each step snapshots the pool, replays the bucket's graph, restores the pool
and runs ``forward_decode`` eagerly on the same padded batch (the real rows,
then the dummy row in the unused slots).  Logits of the real rows and every
pool page but the dummy row's must be bit-identical (the graph records the
same kernels); the dummy page is written by every unused slot at once and is
excluded.  Batches come and go between steps and cross bucket sizes up to
256; host inputs (lists) and device tensors must give the same result.
"""

import numpy as np
import pytest
import torch

from _decode_model import TinyDecodeModel

pytestmark = pytest.mark.gpu


def _setup(cuda, n_req, max_ctx, seed):
    from qwen3_engine_from_scratch_b200 import KVCachePool, PagedKVCache, ops
    model = TinyDecodeModel(cuda, seed=seed)
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, max_ctx + 1, n_req)
    pages = int(sum((int(L) + 16) // 16 + 1 for L in lens))
    pool = KVCachePool(num_blocks=pages + 256 + 8, num_layers=model.layers, block_size=16,
                       num_kv_heads=model.Hkv, head_dim=model.D, device=cuda,
                       dtype=torch.bfloat16, max_seq_len=max_ctx + 64,
                       max_requests=n_req + 256 + 1)
    g = torch.Generator(device=cuda).manual_seed(seed)
    reqs = []
    for L in lens:
        c = PagedKVCache(pool)
        for layer in range(model.layers):
            k = torch.randn(1, model.Hkv, int(L), model.D, generator=g, device=cuda)
            v = torch.randn(1, model.Hkv, int(L), model.D, generator=g, device=cuda)
            c.update(layer, k.to(torch.bfloat16), v.to(torch.bfloat16))
        c.advance_seq_len(int(L))
        reqs.append(c)
    placeholders = [PagedKVCache(pool) for _ in range(256)]
    torch.cuda.synchronize()
    return model, pool, reqs, placeholders, ops


def _snapshot(pool):
    return pool.k_buffer.clone(), pool.v_buffer.clone(), pool.seq_lens.clone()


def _restore(pool, snap):
    pool.k_buffer.copy_(snap[0])
    pool.v_buffer.copy_(snap[1])
    pool.seq_lens.copy_(snap[2])


def _check_step(runner, model, pool, active, rng, cuda, host_inputs):
    from qwen3_engine_from_scratch_b200.graph_runner import bucket_for
    k = len(active)
    b = bucket_for(runner.buckets, k)
    for c in active:
        c.reserve_next()
    ids = rng.integers(0, 1024, k)
    pos = np.array([c.seq_len for c in active])
    rows = np.array([c.row_id for c in active])
    snap = _snapshot(pool)
    if host_inputs:
        logits = runner.replay(ids.tolist(), pos.tolist(), rows.tolist())
    else:
        logits = runner.replay(torch.tensor(ids, device=cuda).view(k, 1),
                               torch.tensor(pos, device=cuda).view(k, 1),
                               torch.tensor(rows, dtype=torch.int32, device=cuda))
    got = logits[:k].clone()
    torch.cuda.synchronize()
    after = _snapshot(pool)
    _restore(pool, snap)
    pad = b - k
    e_ids = torch.tensor(np.concatenate([ids, np.zeros(pad, np.int64)]), device=cuda).view(b, 1)
    e_pos = torch.tensor(np.concatenate([pos, np.zeros(pad, np.int64)]), device=cuda).view(b, 1)
    e_rows = torch.tensor(np.concatenate([rows, np.full(pad, runner.dummy_row)]),
                          dtype=torch.int32, device=cuda)
    with torch.no_grad():
        want = model.forward_decode(e_ids, e_pos, e_rows, list(active) + [active[0]] * pad)[:k]
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    keep = torch.ones(pool.k_buffer.shape[0], dtype=torch.bool, device=cuda)
    keep[runner._dummy_phys] = False
    assert torch.equal(after[0][keep].view(torch.int16), pool.k_buffer[keep].view(torch.int16))
    assert torch.equal(after[1][keep].view(torch.int16), pool.v_buffer[keep].view(torch.int16))
    assert torch.equal(after[2], pool.seq_lens)
    for c in active:
        c.advance_seq_len(1)


def test_replay_matches_eager_across_buckets(cuda, native_lib):
    from qwen3_engine_from_scratch_b200.graph_runner import GraphRunner, DEFAULT_BUCKETS
    import qwen3_engine_from_scratch_b200 as qb
    model, pool, reqs, placeholders, _ = _setup(cuda, n_req=150, max_ctx=300, seed=3)
    free_before = pool.free_count
    runner = GraphRunner(model, pool, placeholders, buckets=DEFAULT_BUCKETS, reserve_pages=1)
    assert sorted(runner.graphs) == list(DEFAULT_BUCKETS)
    # one page per placeholder (reserve_pages=1) and the dummy row's page
    assert pool.free_count == free_before - len(placeholders) - 1
    rng = np.random.default_rng(7)
    # batch compositions: shrink, grow, single request, largest bucket
    for step, (n, host) in enumerate([(12, False), (5, True), (1, False), (9, True),
                                       (150, False), (130, True), (64, False)]):
        idx = rng.choice(len(reqs), n, replace=False)
        _check_step(runner, model, pool, [reqs[i] for i in idx], rng, cuda, host)
    qb.check_device_status(cuda)
    free_now = pool.free_count          # the requests' reserve_next took pages meanwhile
    runner.free()
    assert pool.free_count == free_now + 1


def test_host_and_device_inputs_agree(cuda, native_lib):
    from qwen3_engine_from_scratch_b200.graph_runner import GraphRunner
    model, pool, reqs, placeholders, _ = _setup(cuda, n_req=6, max_ctx=200, seed=11)
    runner = GraphRunner(model, pool, placeholders[:8], buckets=(4, 8), reserve_pages=1)
    active = reqs[:6]
    for c in active:
        c.reserve_next()
    ids = [5, 17, 900, 3, 64, 1000]
    pos = [c.seq_len for c in active]
    rows = [c.row_id for c in active]
    snap = _snapshot(pool)
    a = runner.replay(ids, pos, rows)[:6].clone()
    _restore(pool, snap)
    b = runner.replay(torch.tensor(ids, device=cuda).view(6, 1),
                      torch.tensor(pos, device=cuda).view(6, 1),
                      torch.tensor(rows, dtype=torch.int32, device=cuda))[:6].clone()
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    with pytest.raises(ValueError):
        runner.replay(list(range(9)), list(range(9)), list(range(9)))
    runner.free()
