"""KV-head tensor parallelism on two GPUs over NCCL (skipped on one GPU).

Rank r of 2 keeps kv heads [r*Hkv/2, (r+1)*Hkv/2) of a seeded pool and their
query heads, runs the paged decode on them, and dist.kv_head_tp_all_gather
rebuilds (B, H*D) before o_proj.  Rank 0 compares the gathered output with the
decode of all heads on one GPU: equal bit for bit (same pages, same split size,
so the same arithmetic per (request, kv head)).
"""

import os
import socket
import traceback

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _state(seed=11, B=8, H=16, Hkv=8, D=128, max_len=700):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, max_len, size=B)
    max_pages = (max_len + 15) // 16
    need = int(sum((L + 15) // 16 for L in lens))
    nb = need + 8
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.full((B + 2, max_pages), -1, np.int32)
    rows = np.arange(B, dtype=np.int32) + 1
    used = 0
    for b in range(B):
        n = (int(lens[b]) + 15) // 16
        bt[rows[b], :n] = perm[used:used + n]
        used += n
    seq = np.zeros(B + 2, np.int32)
    seq[rows] = lens - 1
    g = torch.Generator().manual_seed(seed)
    kp = torch.randn(nb, Hkv, 16, D, generator=g).to(torch.bfloat16)
    vp = torch.randn(nb, Hkv, 16, D, generator=g).to(torch.bfloat16)
    q = torch.randn(B, H, D, generator=g).to(torch.bfloat16)
    return q, kp, vp, torch.from_numpy(bt), torch.from_numpy(seq), torch.from_numpy(rows)


def _worker(rank, world, port, result_path):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    ok = False
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        import qwen3_engine_from_scratch_b200 as qb
        from qwen3_engine_from_scratch_b200.dist import kv_head_tp_all_gather
        q, kp, vp, bt, seq, rows = (t.to(dev) for t in _state())
        B, H, D = q.shape
        Hkv = kp.shape[1]
        hk, hq = Hkv // world, H // world
        pps = 8
        local = qb.paged_decode(q[:, rank * hq:(rank + 1) * hq].contiguous(),
                                kp[:, rank * hk:(rank + 1) * hk].contiguous(),
                                vp[:, rank * hk:(rank + 1) * hk].contiguous(),
                                bt, seq, rows, D ** -0.5, pages_per_split=pps)
        gathered = kv_head_tp_all_gather(local)
        torch.cuda.synchronize()
        qb.check_device_status(dev)
        if rank == 0:
            full = qb.paged_decode(q, kp, vp, bt, seq, rows, D ** -0.5, pages_per_split=pps)
            torch.cuda.synchronize()
            ok = gathered.shape == (B, H * D) and torch.equal(gathered, full.reshape(B, H * D))
        else:
            ok = True
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        traceback.print_exc()
        ok = False
    with open(f"{result_path}.{rank}", "w") as f:
        f.write("ok" if ok else "fail")


def test_kv_head_tp_two_gpus_matches_one_gpu(tmp_path, native_lib):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    path = str(tmp_path / "tp_result")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    for r in range(2):
        with open(f"{path}.{r}") as f:
            assert f.read() == "ok", f"rank {r} failed"
