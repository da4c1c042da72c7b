"""Host-side logic that needs no GPU: request sharding, the KV-head TP exchange
(world size 2 over gloo), the shim's name binding, and the FMA-pipe exp2 method
the prefill kernel uses."""

import os
import socket
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# checkout of the reference engine (its `qwen3` package), for the tests that bind
# into its modules; they are skipped when QWEN3_REFERENCE is not set
REFERENCE = os.environ.get("QWEN3_REFERENCE")
needs_reference = pytest.mark.skipif(
    not REFERENCE or not os.path.isdir(os.path.join(REFERENCE, "qwen3")),
    reason="set QWEN3_REFERENCE to a checkout of the reference engine")


def test_lpt_partition_balances_and_covers():
    from qwen3_engine_from_scratch_b200.dist import lpt_partition, shard_loads, decode_cost
    rng = np.random.default_rng(0)
    lens = np.exp(rng.uniform(np.log(256), np.log(32768), size=512)).astype(int)
    for n in (1, 2, 4, 8):
        shards = lpt_partition(decode_cost(lens), n)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(512))
        loads = shard_loads(decode_cost(lens), shards)
        # LPT bound: max load <= mean + max item
        assert max(loads) <= sum(loads) / n + max(lens)
        assert max(loads) / (sum(loads) / n) < 1.02
    assert lpt_partition([5, 5, 5], 2) == [[0, 2], [1]]


def test_lpt_prefill_cost_is_quadratic():
    from qwen3_engine_from_scratch_b200.dist import prefill_cost
    assert prefill_cost([1, 2, 2048]) == [1, 3, 2048 * 2049 // 2]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, q):
    import torch.distributed as dist
    from qwen3_engine_from_scratch_b200.dist import kv_head_tp_all_gather, lpt_partition
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, H, D = 3, 16, 128
        full = torch.arange(B * H * D, dtype=torch.float32).reshape(B, H, D)
        hl = H // world
        local = full[:, rank * hl:(rank + 1) * hl]
        gathered = kv_head_tp_all_gather(local)
        ok_tp = torch.equal(gathered, full.reshape(B, H * D))
        # request sharding: every rank derives the same partition, no exchange needed
        lens = [300, 20, 4000, 128, 77, 1000]
        mine = lpt_partition(lens, world)[rank]
        t = torch.tensor([sum(lens[i] for i in mine)], dtype=torch.float64)
        dist.all_reduce(t)
        q.put((rank, ok_tp, float(t.item())))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_tp_gather_and_sharding():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [q.get(timeout=10) for _ in procs]
    assert all(ok for _, ok, _ in res)
    assert all(total == sum([300, 20, 4000, 128, 77, 1000]) for _, _, total in res)


def _leaving_rank_worker(rank, world, port, q):
    """Rank 1 takes one exchange, then leaves between steps (no collective in
    flight); rank 0's next exchange has to end with an error, not hang."""
    import time
    from datetime import timedelta

    import torch.distributed as dist
    from qwen3_engine_from_scratch_b200.dist import kv_head_tp_all_gather
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    local = torch.full((2, 8, 128), float(rank))
    kv_head_tp_all_gather(local)                 # step 1: both ranks take part
    if rank == 1:
        q.put((rank, "left", 0.0))
        q.close()
        q.join_thread()                          # the message is out before the exit
        os._exit(0)                              # leaves between steps
    t0 = time.monotonic()
    try:
        kv_head_tp_all_gather(local)             # step 2: the peer is gone
        q.put((rank, "no error", time.monotonic() - t0))
    except Exception:  # noqa: BLE001 -- gloo reports the lost peer as a RuntimeError subclass
        q.put((rank, "error", time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_gloo_peer_that_leaves_ends_the_next_exchange_with_an_error():
    """Failure detection without a GPU: a rank that exits between steps makes
    its peer's next KV-head all-gather raise within the process group's short
    timeout (5 s here) instead of waiting forever."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung on the lost peer"
    res = dict((r, (what, dt)) for r, what, dt in (q.get(timeout=10) for _ in procs))
    assert res[1][0] == "left"
    assert res[0][0] == "error", res
    assert res[0][1] < 60.0, res


@needs_reference
def test_shim_binds_into_reference_modules(monkeypatch):
    monkeypatch.syspath_prepend(REFERENCE)
    import importlib
    from qwen3_engine_from_scratch_b200 import ops, shim
    bound = shim.install()
    try:
        attn = importlib.import_module("qwen3.attention")
        kvc = importlib.import_module("qwen3.PagedKVcache")
        assert attn.triton_paged_attention_decode_batch is ops.triton_paged_attention_decode_batch
        assert attn.triton_paged_attention_decode is ops.triton_paged_attention_decode
        assert attn.flash_attention_prefill_batched is ops.flash_attention_prefill_batched
        assert kvc.update_kv_batch_triton is ops.update_kv_batch_triton
        assert kvc.PagedKVCache.update is shim._paged_cache_update
        assert "qwen3.PagedKVcache.PagedKVCache.update" in bound
        assert len(bound) == 14
        assert importlib.import_module("qwen3.sampling").sample_tokens is ops.sample_tokens
        from qwen3_engine_from_scratch_b200 import graph_runner
        assert importlib.import_module("qwen3.graph_runner").GraphRunner is graph_runner.GraphRunner
    finally:
        shim.uninstall()
    attn = importlib.import_module("qwen3.attention")
    assert attn.triton_paged_attention_decode_batch is not ops.triton_paged_attention_decode_batch
    assert importlib.import_module("qwen3.PagedKVcache").PagedKVCache.update is not \
        shim._paged_cache_update


@needs_reference
def test_shim_cache_update_keeps_reference_cpu_path(monkeypatch):
    """With the shim installed, the reference's PagedKVCache.update on CPU tensors
    (outside the kernel's contract) still runs the reference's own method: the
    block table and pool bytes equal an uninstalled run's."""
    monkeypatch.syspath_prepend(REFERENCE)
    import importlib
    from qwen3_engine_from_scratch_b200 import shim
    kvc = importlib.import_module("qwen3.PagedKVcache")

    def run():
        pool = kvc.KVCachePool(num_blocks=16, num_layers=2, block_size=16, num_kv_heads=2,
                               head_dim=128, dtype=torch.float32, max_seq_len=128, max_requests=4)
        c = kvc.PagedKVCache(pool)
        g = torch.Generator().manual_seed(5)
        c.update(1, torch.randn(1, 2, 21, 128, generator=g), torch.randn(1, 2, 21, 128, generator=g))
        c.advance_seq_len(21)
        c.update(1, torch.randn(1, 2, 15, 128, generator=g), torch.randn(1, 2, 15, 128, generator=g))
        return pool.block_table_2d.clone(), pool.k_buffer.clone(), pool.v_buffer.clone()

    want = run()
    shim.install()
    try:
        assert kvc.PagedKVCache.update is shim._paged_cache_update
        got = run()
    finally:
        shim.uninstall()
    assert all(torch.equal(a, b) for a, b in zip(got, want))


def test_reference_signatures_match():
    """The drop-in names take the reference's positional arguments."""
    import inspect
    from qwen3_engine_from_scratch_b200 import ops
    expect = {
        "paged_attention_decode_triton": ["q", "k_buffer", "v_buffer", "block_table_2d",
                                          "seq_lens_full", "row_ids", "block_size"],
        "triton_paged_attention_decode": ["q", "k_new", "v_new", "kv_cache", "layer_idx", "scaling"],
        "triton_paged_attention_decode_batch": ["q", "k_new", "v_new", "kv_caches", "layer_idx",
                                                "scaling", "row_ids"],
        "update_kv_batch_triton": ["k_new", "v_new", "k_buffer", "v_buffer", "seq_lens",
                                   "block_table_2d", "row_ids", "layer_idx"],
        "flash_attention_prefill": ["q", "k", "v", "cu_seqlens", "scale", "num_heads",
                                    "num_kv_heads", "head_dim"],
        "flash_attention_prefill_batched": ["q", "k", "v", "lens", "scaling", "num_heads",
                                            "num_kv_heads", "head_dim"],
    }
    for name, params in expect.items():
        got = list(inspect.signature(getattr(ops, name)).parameters)
        assert got[:len(params)] == params, (name, got)


@needs_reference
def test_graph_runner_signature_matches_reference(monkeypatch):
    """GraphRunner takes the reference's constructor and replay arguments."""
    import inspect
    monkeypatch.syspath_prepend(REFERENCE)
    import importlib
    ref = importlib.import_module("qwen3.graph_runner").GraphRunner
    from qwen3_engine_from_scratch_b200 import shim
    ours = shim._BINDINGS[("qwen3.graph_runner", "GraphRunner")]
    for meth in ("__init__", "replay", "free"):
        want = list(inspect.signature(getattr(ref, meth)).parameters)
        got = list(inspect.signature(getattr(ours, meth)).parameters)
        assert got[:len(want)] == want, (meth, got, want)


def test_fma_exp2_method():
    """The exponent-split + degree-3 polynomial 2^x of the prefill kernel
    (common.cuh ex2_fma), restated in float32 numpy: relative error below
    1e-4 on the range the softmax uses, finite and tiny below it."""
    x = np.concatenate([np.linspace(-200, 8, 400001), [-np.inf, -125.0, -126.0]]).astype(np.float32)
    xc = np.maximum(x, np.float32(-125))
    t = (xc + np.float32(12582912.0)).astype(np.float32)
    j = (t - np.float32(12582912.0)).astype(np.float32)
    f = (xc - j).astype(np.float32)
    c = [np.float32(v) for v in (0.0551716685, 0.2426111400, 0.6932609677, 0.9999280572)]
    p = (((c[0] * f + c[1]) * f + c[2]) * f + c[3]).astype(np.float32)
    res = (p.view(np.int32) + (t.view(np.int32) << 23)).view(np.float32)
    assert np.isfinite(res).all() and (res > 0).all()
    ok = x >= -125
    rel = np.abs(res[ok].astype(np.float64) / np.exp2(x[ok].astype(np.float64)) - 1)
    assert rel.max() < 1e-4
    assert res[~ok].max() < 1e-37


def test_graph_runner_bucket_choice():
    from qwen3_engine_from_scratch_b200.graph_runner import bucket_for, DEFAULT_BUCKETS
    assert DEFAULT_BUCKETS[-1] == 256
    assert bucket_for(DEFAULT_BUCKETS, 0) == 1
    assert bucket_for(DEFAULT_BUCKETS, 1) == 1
    assert bucket_for(DEFAULT_BUCKETS, 3) == 4
    assert bucket_for(DEFAULT_BUCKETS, 129) == 256
    assert bucket_for((1, 2, 4, 8), 8) == 8
    with pytest.raises(ValueError):
        bucket_for(DEFAULT_BUCKETS, 257)
    with pytest.raises(ValueError):
        bucket_for(DEFAULT_BUCKETS, -1)


def test_graph_runner_packs_host_inputs_with_dummy_rows():
    from qwen3_engine_from_scratch_b200.graph_runner import pack_host_inputs
    ids = np.full(8, -7, np.int64)
    pos = np.full(8, -7, np.int64)
    rows = np.full(8, -7, np.int32)
    k = pack_host_inputs(ids, pos, rows, torch.tensor([[3], [9], [4]]), [10, 20, 30],
                         np.array([5, 6, 7]), dummy_row=99)
    assert k == 3
    assert ids.tolist() == [3, 9, 4, 0, 0, 0, 0, 0]
    assert pos.tolist() == [10, 20, 30, 0, 0, 0, 0, 0]
    assert rows.tolist() == [5, 6, 7, 99, 99, 99, 99, 99]
    with pytest.raises(ValueError):
        pack_host_inputs(ids, pos, rows, [1, 2], [1], [1, 2], dummy_row=0)
    with pytest.raises(ValueError):
        pack_host_inputs(ids[:2], pos[:2], rows[:2], [1, 2, 3], [1, 2, 3], [1, 2, 3], 0)


def test_kv_pool_blocks_from_free_memory():
    from qwen3_engine_from_scratch_b200.graph_runner import kv_pool_blocks
    # Qwen3-0.6B: 28 layers x 8 kv heads x 16 x 128 bf16, K and V: 1,835,008 B per block
    per_block = 2 * 28 * 8 * 16 * 128 * 2
    free = 170 * (1 << 30)
    n = kv_pool_blocks(28, 8, 128, free_bytes=free, fraction=0.9, reserve_bytes=4 << 30)
    assert n == (int(free * 0.9) - (4 << 30)) // per_block
    assert kv_pool_blocks(28, 8, 128, free_bytes=1 << 30) == 0
    assert kv_pool_blocks(28, 8, 128, dtype=torch.float32, free_bytes=free, fraction=1.0,
                          reserve_bytes=0) == free // (2 * per_block)


def test_graph_runner_rejects_bad_setup():
    from qwen3_engine_from_scratch_b200.graph_runner import GraphRunner
    with pytest.raises(ValueError):
        GraphRunner(None, None, [], buckets=())
    with pytest.raises(AssertionError):
        GraphRunner(None, None, [object()] * 3, buckets=(1, 2, 4))
