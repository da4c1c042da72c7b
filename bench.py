"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config c2|c4]

Headline workload (config 2 of the benchmark plan, per GPU): batched paged
decode of Qwen3-0.6B attention -- B=64 requests, 16 q / 8 kv heads, head_dim
128, context lengths uniform in [128, 4096], 16-token pages placed by a random
permutation in a 32768-block pool, Q/K RMS-normed and RoPE'd at theta 1e6.
A step is one decode step of the whole 28-layer attention stack: for every
layer, the KV write of the new token (scatter) and the split-K decode.  The
step is captured once in a CUDA graph and replayed, as the reference engine
serves decode (qwen3/graph_runner.py); ``eager_ms_per_step`` is the same step
issued call by call from Python.

``value`` = algorithmic bytes of all ranks' steps / max-over-ranks device time
(GB/s); inputs resident in HBM; the KV read per step (~16 GB) is far larger
than L2 (126 MB), so no flush is needed between steps.  ``e2e`` repeats the
step through the reference-named public API ``triton_paged_attention_decode_batch``
with the step's q/k/v copied from pinned host memory and the outputs copied
back inside the timed (graph-replayed) region; its ``eager`` field is the same
without the graph.  ``roofline`` is for the decode kernel (splits merged
in-kernel by the last split of each request x kv head): its launch time is the
graph-replayed step time / 28 launches; the per-call eager figure sits beside it.

Multi-GPU: one process per GPU (torchrun), each rank owns its own requests,
pool and block table -- no collective on the data path ("scaling": "weak").
The default line also carries a ``c4`` object: config 4 (Qwen3-8B heads 32/8,
512 requests of log-uniform [256,32768] tokens) with the 512 requests sharded
over the ranks by LPT on length ("scaling": "strong"), max-over-ranks time; a
``c5`` object (config 5: Qwen3-0.6B end to end, 256 requests decoded from CUDA
graphs, data parallel over the ranks, tokens/s); and a ``prefill`` object (config 3 varlen prefill, with its own ``e2e``, ``clocks``
and ``cpu_baseline``).  ``--config c4`` / ``--config c3`` make those the headline.

``--impl reference``: the reference's own algorithm (the CPU oracle port of
qwen3/paged_attention.py:paged_attention) on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

HEAD_DIM = 128
BLOCK = 16
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


# ---------------------------------------------------------------------------
# workloads (shapes only; data generated on the device)
# ---------------------------------------------------------------------------

def workload(config: str, rank: int, world: int):
    if config == "c2":
        rng = np.random.default_rng(1234 + rank)
        lens = rng.integers(128, 4096, size=64, endpoint=True)
        return dict(name="c2_paged_decode_qwen3_0.6b", H=16, Hkv=8, lens=lens, layers=28,
                    num_blocks=32768, max_seq_len=4096, scaling="weak", batch_per_gpu=64)
    if config == "c4":
        rng = np.random.default_rng(4321)
        all_lens = np.exp(rng.uniform(np.log(256), np.log(32768), size=512)).astype(np.int64)
        from qwen3_engine_from_scratch_b200.dist import decode_cost, lpt_partition
        shards = lpt_partition(decode_cost(all_lens), world)
        lens = all_lens[shards[rank]]
        blocks = int(sum((int(L) + BLOCK - 1) // BLOCK for L in lens)) + 64
        return dict(name="c4_paged_decode_qwen3_8b_sharded", H=32, Hkv=8, lens=lens, layers=1,
                    num_blocks=blocks, max_seq_len=32768, scaling="strong", batch_total=512,
                    all_lens=all_lens)
    if config == "c3":
        rng = np.random.default_rng(3000 + rank)
        lens = rng.integers(64, 2048, size=32, endpoint=True)
        return dict(name="c3_varlen_prefill_qwen3_0.6b", H=16, Hkv=8, lens=lens, layers=1,
                    scaling="weak", batch_per_gpu=32)
    raise SystemExit(f"unknown config {config}")


def decode_bytes(lens, H, Hkv, D=HEAD_DIM, elem=2):
    lens = np.asarray(lens, dtype=np.int64)
    B = len(lens)
    kv = int(lens.sum()) * Hkv * D * elem * 2
    qo = B * H * D * elem * 2
    tables = int(((lens + BLOCK - 1) // BLOCK).sum()) * 4
    return kv + qo + tables + B * 8


def prefill_flops(lens, H, D=HEAD_DIM):
    lens = np.asarray(lens, dtype=np.int64)
    return int((4 * H * D * (lens * (lens + 1) // 2)).sum())


def scatter_bytes(B, Hkv, D=HEAD_DIM, elem=2):
    return B * Hkv * D * elem * 2 * 2 + B * 12   # read + write K and V, row/len/table reads


# ---------------------------------------------------------------------------
# clocks (NVML sampled in a thread during the timed region)
# ---------------------------------------------------------------------------

REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
           0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
           0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
           0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, torch_device_index: int, period_s: float = 0.01):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.error = None
        try:
            import pynvml
            pynvml.nvmlInit()
            import torch
            props = torch.cuda.get_device_properties(torch_device_index)
            handle = None
            bus = getattr(props, "pci_bus_id", None)
            if bus is not None:
                dom = getattr(props, "pci_domain_id", 0)
                devid = getattr(props, "pci_device_id", 0)
                try:
                    handle = pynvml.nvmlDeviceGetHandleByPciBusId(
                        f"{dom:08x}:{bus:02x}:{devid:02x}.0".encode())
                except Exception:
                    handle = None
            if handle is None:
                handle = pynvml.nvmlDeviceGetHandleByIndex(torch_device_index)
            self._nv = pynvml
            self._h = handle
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: report what we could not sample
            self.error = repr(e)
            self._nv = None
        self.period = period_s

    def _run(self):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                except Exception:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                self.samples.append(mhz)
                self.reasons |= int(r)
            except Exception as e:
                self.error = repr(e)
                return
            time.sleep(self.period)

    def start(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        reasons = [name for bit, name in REASONS.items() if self.reasons & bit and bit != 0x1]
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None,
               "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples),
               "source": "nvml"}
        if self.error:
            out["error"] = self.error
        return out


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------

def build_decode_state(w, device, seed):
    """Pool, block table, row slots and per-layer inputs on the device."""
    import torch
    import qwen3_engine_from_scratch_b200 as qb

    H, Hkv, D, layers = w["H"], w["Hkv"], HEAD_DIM, w["layers"]
    lens = np.asarray(w["lens"], dtype=np.int64)
    B = len(lens)
    g = torch.Generator(device=device).manual_seed(seed)
    pool = qb.KVCachePool(num_blocks=w["num_blocks"], num_layers=layers, block_size=BLOCK,
                          num_kv_heads=Hkv, head_dim=D, device=device, dtype=torch.bfloat16,
                          max_seq_len=w["max_seq_len"], max_requests=B + 1)
    perm = torch.randperm(w["num_blocks"], generator=g, device=device).cpu().tolist()
    pool.free_block_ids = perm
    caches = []
    for L in lens:
        c = qb.PagedKVCache(pool)
        c._ensure_pages(int(L))           # pages for the L-1 context tokens + this step's token
        c.seq_len = int(L) - 1
        caches.append(c)
    pool.seq_lens[[c.row_id for c in caches]] = torch.tensor([int(L) - 1 for L in lens],
                                                             dtype=torch.int32, device=device)
    rows = torch.tensor([c.row_id for c in caches], dtype=torch.int32, device=device)
    # K/V of the context: N(0,1), K RMS-normed + RoPE'd (theta 1e6); written per layer
    pos = np.concatenate([np.arange(int(L) - 1) for L in lens])
    slots = np.concatenate([np.asarray(c.block_table, np.int64)[np.arange(int(L) - 1) // BLOCK] * BLOCK
                            + np.arange(int(L) - 1) % BLOCK for c, L in zip(caches, lens)])
    pos_t = torch.from_numpy(pos).to(device).float()
    slots_t = torch.from_numpy(slots).to(device)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D))

    def rope(x, p):
        ang = p[:, None] * inv[None]
        cos = torch.cat([ang, ang], -1).cos()[:, None]
        sin = torch.cat([ang, ang], -1).sin()[:, None]
        return x * cos + torch.cat([-x[..., D // 2:], x[..., :D // 2]], -1) * sin

    def rms(x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)

    T = len(pos)
    chunk = 1 << 16
    for layer in range(layers):
        for s0 in range(0, T, chunk):
            s1 = min(T, s0 + chunk)
            k = rope(rms(torch.randn(s1 - s0, Hkv, D, generator=g, device=device)), pos_t[s0:s1])
            v = torch.randn(s1 - s0, Hkv, D, generator=g, device=device)
            qb.kv_scatter_slots(k.to(torch.bfloat16), v.to(torch.bfloat16), pool.k_buffer,
                                pool.v_buffer, slots_t[s0:s1], layer)
    qpos = torch.from_numpy(lens - 1).to(device).float()
    qs = rope(rms(torch.randn(layers * B, H, D, generator=g, device=device)), qpos.repeat(layers))
    q = qs.view(layers, B, H, 1, D).to(torch.bfloat16)
    knew = rope(rms(torch.randn(layers * B, Hkv, D, generator=g, device=device)), qpos.repeat(layers))
    k_new = knew.view(layers, B, Hkv, 1, D).to(torch.bfloat16)
    v_new = torch.randn(layers, B, Hkv, 1, D, generator=g, device=device).to(torch.bfloat16)
    torch.cuda.synchronize()
    return dict(pool=pool, caches=caches, rows=rows, q=q, k_new=k_new, v_new=v_new, B=B)


def run_b200(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import qwen3_engine_from_scratch_b200 as qb
    from qwen3_engine_from_scratch_b200 import ops

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    w = workload(args.config, rank, world)
    if args.layers > 0:
        w["layers"] = args.layers
    st = build_decode_state(w, device, seed=1000 + rank)
    pool, caches, rows = st["pool"], st["caches"], st["rows"]
    q, k_new, v_new, B = st["q"], st["k_new"], st["v_new"], st["B"]
    H, Hkv, layers = w["H"], w["Hkv"], w["layers"]
    scale = HEAD_DIM ** -0.5
    lens = np.asarray(w["lens"], dtype=np.int64)
    max_pages = pool.block_table_2d.shape[1]
    # one launch per layer: the KV write of the new token is fused into the
    # decode kernel, and the split merge runs inside it too
    launches_per_layer = 1

    def layer_call(l):
        return ops.paged_decode_kv_write(q[l, :, :, 0], k_new[l, :, :, 0], v_new[l, :, :, 0],
                                         pool.k_buffer[:, l], pool.v_buffer[:, l],
                                         pool.block_table_2d, pool.seq_lens, rows, scale)

    stream = torch.cuda.current_stream()
    # warm-up
    for _ in range(args.warmup):
        for l in range(layers):
            layer_call(l)
    torch.cuda.synchronize()
    qb.check_device_status(device)

    # ---- per-call timing, eager: CUDA events around every decode call (roofline)
    ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps * layers)]
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps * layers)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    i = 0
    for _ in range(args.steps):
        for l in range(layers):
            ev_a[i].record(stream)
            layer_call(l)
            ev_b[i].record(stream)
            i += 1
    stop.record(stream)
    torch.cuda.synchronize()
    eager_ms = start.elapsed_time(stop)
    decode_ms = sum(a.elapsed_time(b) for a, b in zip(ev_a, ev_b)) / len(ev_a)

    # ---- timed region: the 28-layer step captured once in a CUDA graph and
    # replayed, as the reference's GraphRunner serves decode (qwen3/graph_runner.py)
    def step():
        for l in range(layers):
            layer_call(l)

    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        step()                              # the capture stream's workspace, allocated eagerly
    stream.wait_stream(side)
    torch.cuda.synchronize()
    step_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(step_graph, stream=side):
        step()
    for _ in range(2):
        step_graph.replay()
    clocks = ClockSampler(local_rank)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    start.record(stream)
    for _ in range(args.steps):
        step_graph.replay()
    stop.record(stream)
    torch.cuda.synchronize()
    clocks.stop()
    if world > 1:
        dist.barrier()
    del step_graph
    ms = start.elapsed_time(stop)
    qb.check_device_status(device)

    # ---- e2e: host q/k/v (pinned) -> device, the public batch API, outputs -> host
    hq = q.cpu().pin_memory()
    hk = k_new.cpu().pin_memory()
    hv = v_new.cpu().pin_memory()
    hout = torch.empty((layers, B, 1, H * HEAD_DIM), dtype=torch.bfloat16).pin_memory()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k_new), torch.empty_like(v_new)
    e2e_steps = max(3, min(args.steps, 50))

    # layer-pipelined copies: the step's q/k/v go up on a copy stream in
    # groups of layers 1, 1, 2, 4, 8, ... (each group lands while the layers
    # before it compute, with far fewer copies and cross-stream waits than one
    # group per layer: 2.635 -> 2.588 ms per C2 step), each layer's output
    # goes down on a second copy stream, and the step ends only after the last
    # output reached the host.
    cs_in, cs_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    groups, lo, size = [], 0, 1
    while lo < layers:
        groups.append((lo, min(layers, lo + size)))
        lo, size = lo + size, (size * 2 if lo > 0 else 1)
    ev_in = {a: torch.cuda.Event() for a, _ in groups}
    ev_done = [torch.cuda.Event() for _ in range(layers)]

    def e2e_step():
        cur = torch.cuda.current_stream(device)
        cs_in.wait_stream(cur)          # after the previous step (and joins a capture)
        cs_out.wait_stream(cur)
        with torch.cuda.stream(cs_in):
            for a, b in groups:
                dq[a:b].copy_(hq[a:b], non_blocking=True)
                dk[a:b].copy_(hk[a:b], non_blocking=True)
                dv[a:b].copy_(hv[a:b], non_blocking=True)
                ev_in[a].record(cs_in)
        for l in range(layers):
            if l in ev_in:
                cur.wait_event(ev_in[l])
            o = qb.triton_paged_attention_decode_batch(dq[l], dk[l], dv[l], caches, l, scale, rows)
            ev_done[l].record(cur)
            cs_out.wait_event(ev_done[l])
            o.record_stream(cs_out)
            with torch.cuda.stream(cs_out):
                hout[l].copy_(o, non_blocking=True)
        cur.wait_stream(cs_out)

    def time_e2e(run):
        for _ in range(2):
            run()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for _ in range(e2e_steps):
            run()
        e_stop.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return e_start.elapsed_time(e_stop) / e2e_steps

    # eager: every public-API call issued from Python each step
    e2e_eager_ms = time_e2e(e2e_step)
    # the reference engine serves decode from a CUDA graph of the whole step
    # (qwen3/graph_runner.py): capture the same step, copies included, once
    graph = torch.cuda.CUDAGraph()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        e2e_step()                      # warm the per-stream workspaces of the capture stream
    stream.wait_stream(side)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph, stream=side):
        e2e_step()
    e2e_ms = time_e2e(graph.replay)
    del graph

    step_bytes = layers * (decode_bytes(lens, H, Hkv) + scatter_bytes(B, Hkv))
    # the roofline kernel reads every visible K/V token, q and the tables, and
    # reads + writes the new token's K/V rows
    dec_bytes = decode_bytes(lens, H, Hkv) + scatter_bytes(B, Hkv)
    t = torch.tensor([ms, e2e_ms, float(step_bytes), decode_ms, e2e_eager_ms, eager_ms],
                     dtype=torch.float64, device=device)
    if world > 1:
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tsum = t.clone()
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        ms, e2e_ms, e2e_eager_ms, eager_ms = (float(tmax[0]), float(tmax[1]), float(tmax[4]),
                                              float(tmax[5]))
        total_bytes_per_step = float(tsum[2])
    else:
        total_bytes_per_step = float(step_bytes)
    h2d_bytes = int(hq.numel() * 2 + hk.numel() * 2 + hv.numel() * 2)
    d2h_bytes = int(hout.numel() * 2)
    # the other legs run on their own device memory: the decode pool (tens of
    # GB) and its buffers are released first, on every rank
    del st, pool, caches, q, k_new, v_new, dq, dk, dv, hq, hk, hv, hout
    del layer_call, step, e2e_step, time_e2e
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    c4 = c5 = None
    if args.config == "c2" and not args.no_c4:
        # config 4 strong scaling, every rank (collectives inside)
        c4 = run_c4_leg(args, rank, world, local_rank, steps=max(5, min(args.steps, 20)),
                        warmup=3)
    if args.config == "c2" and not args.no_c5:
        # config 5 end to end, data parallel over the ranks (collectives inside)
        try:
            c5 = run_c5_leg(args, rank, world, local_rank)
        except RuntimeError as e:
            c5 = {"error": str(e)[:200]}
    if rank != 0:
        return None

    ms_per_step = ms / args.steps
    value = total_bytes_per_step * args.steps / (ms / 1e3) / 1e9
    peaks, peak_src = read_peaks()
    # the kernel's launch time inside the timed region: the graph replays the
    # step's `layers` launches back to back on one stream, so one launch takes
    # the step time / layers (inter-launch gaps included: a lower bound on the
    # kernel's own rate)
    launch_ms = ms_per_step / (layers * launches_per_layer)
    achieved = dec_bytes / (launch_ms / 1e3) / 1e9
    traffic = read_traffic("paged_decode_split_kernel")
    tokens = (w.get("batch_total") or B * world)
    line = {
        "metric": "paged_decode_attention_hbm_bandwidth",
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": w["scaling"],
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: N(0,1) q/k/v, q/k RMS-normed + RoPE theta 1e6, random page permutation",
        "config": {"workload": w["name"], "heads": f"{H}/{Hkv}", "head_dim": HEAD_DIM,
                   "batch_per_gpu": B, "layers_per_step": layers,
                   "context": "U[128,4096]" if args.config == "c2" else "logU[256,32768]",
                   "block_size": BLOCK, "pool_blocks": w["num_blocks"],
                   "l2": "inputs larger than L2 (KV read per step %.1f GB)" % (
                       layers * dec_bytes / 1e9),
                   "parallelism": f"request-sharded x{world}" if world > 1 else "single GPU"},
        "tok_per_s": round(tokens / (ms_per_step / 1e3), 1),
        "timing": "step captured in a CUDA graph and replayed (as the reference's GraphRunner); "
                  "eager_ms_per_step = the same step issued call by call from Python",
        "eager_ms_per_step": round(eager_ms / args.steps, 4),
        "e2e": {"value": round(total_bytes_per_step / (e2e_ms / 1e3) / 1e9, 1), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4),
                "tok_per_s": round(tokens / (e2e_ms / 1e3), 1),
                "h2d_bytes_per_step": h2d_bytes,
                "d2h_bytes_per_step": d2h_bytes,
                "api": "triton_paged_attention_decode_batch for every layer, the step captured in "
                       "a CUDA graph as the reference's GraphRunner serves decode; pinned host "
                       "q/k/v in and outputs out inside the graph on two copy streams "
                       "overlapping the compute (uploads in layer groups 1, 1, 2, 4, 8, 12, "
                       "downloads per layer)",
                "eager": {"value": round(total_bytes_per_step / (e2e_eager_ms / 1e3) / 1e9, 1),
                          "ms_per_step": round(e2e_eager_ms, 4),
                          "api": "the same calls issued from Python every step"}},
        "roofline": {"kernel": "paged_decode_split_kernel",
                     "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": peak_src, "avg_launch_us": round(launch_ms * 1e3, 2),
                     "launch_timing": "graph-replayed timed region: ms_per_step / %d launches "
                                      "per step (back to back on one stream)" % (
                                          layers * launches_per_layer),
                     "eager_avg_launch_us": round(decode_ms * 1e3, 2),
                     "eager_achieved": round(dec_bytes / (decode_ms / 1e3) / 1e9, 1),
                     "eager_timing": "CUDA events around every call of an eager pass (each "
                                     "launch timed alone, launch gaps included)",
                     "bytes_per_launch": dec_bytes,
                     "traffic": traffic},
        "gpu_launches": args.steps * layers * launches_per_layer,
        "clocks": clocks.summary(),
    }
    if c4 is not None:
        line["c4"] = c4
    if c5 is not None:
        line["c5"] = c5
    if not args.no_prefill:
        try:
            line["prefill"] = run_prefill(args, rank, world, local_rank, steps=30, warmup=5,
                                          headline=True)
            if world == 1 and not args.no_cpu_baseline:
                line["prefill"]["cpu_baseline"] = prefill_cpu_baseline(args.cpu_budget)
        except RuntimeError as e:   # the prefill kernel is optional for the decode headline
            line["prefill"] = {"error": str(e)[:200]}
    if not args.no_prefill:
        try:
            line["sampling"] = bench_sampling(device)
        except RuntimeError as e:
            line["sampling"] = {"error": str(e)[:200]}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w, budget_s=args.cpu_budget,
                                            procs=max(1, os.cpu_count() or 1))
    return line


def run_c4_leg(args, rank, world, local_rank, steps, warmup):
    """Config 4 (Qwen3-8B heads 32/8, 512 requests of log-uniform [256, 32768]
    tokens, one layer) as strong scaling: the 512 requests are split over the
    ranks by greedy LPT on length (``dist.lpt_partition``); each rank decodes its
    shard from its own pool with no collective on the data path.  Every rank
    times ``steps`` decode launches (the fused KV-write decode of the batch
    entry) with CUDA events; the job's time is the max over ranks."""
    import torch
    import torch.distributed as dist
    from qwen3_engine_from_scratch_b200 import ops
    from qwen3_engine_from_scratch_b200.dist import decode_cost, lpt_partition, shard_loads

    device = torch.device("cuda", local_rank)
    w = workload("c4", rank, world)
    st = build_decode_state(w, device, seed=2000 + rank)
    pool, rows, q, k_new, v_new, B = st["pool"], st["rows"], st["q"], st["k_new"], st["v_new"], st["B"]
    H, Hkv = w["H"], w["Hkv"]
    lens = np.asarray(w["lens"], dtype=np.int64)
    scale = HEAD_DIM ** -0.5

    def call():
        ops.paged_decode_kv_write(q[0, :, :, 0], k_new[0, :, :, 0], v_new[0, :, :, 0],
                                  pool.k_buffer[:, 0], pool.v_buffer[:, 0], pool.block_table_2d,
                                  pool.seq_lens, rows, scale)

    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a.record(stream)
    for _ in range(steps):
        call()
    b.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = a.elapsed_time(b) / steps
    nbytes = decode_bytes(lens, H, Hkv) + scatter_bytes(B, Hkv)
    t = torch.tensor([ms, float(nbytes), ms], dtype=torch.float64, device=device)
    if world > 1:
        tmax, tsum, tmin = t.clone(), t.clone(), t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        dist.all_reduce(tmin, op=dist.ReduceOp.MIN)
        ms_max, total_bytes, ms_min = float(tmax[0]), float(tsum[1]), float(tmin[2])
    else:
        ms_max, total_bytes, ms_min = ms, float(nbytes), ms
    del st, pool, rows, q, k_new, v_new, call
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    all_lens = w["all_lens"]
    costs = decode_cost(all_lens)
    loads = shard_loads(costs, lpt_partition(costs, world))
    peaks, src = read_peaks()
    gbs = total_bytes / (ms_max / 1e3) / 1e9
    return {"workload": w["name"], "heads": f"{H}/{Hkv}", "requests": int(len(all_lens)),
            "context": "logU[256,32768]", "layers_per_step": 1, "scaling": "strong",
            "partition": f"greedy LPT on length over {world} rank(s)",
            "requests_per_rank_max": int(max(len(s) for s in lpt_partition(costs, world))),
            "lpt_load_max_over_mean": round(max(loads) / (sum(loads) / world), 4),
            "steps": steps, "ms_per_step": round(ms_max, 4),
            "rank_ms_min": round(ms_min, 4), "rank_ms_max": round(ms_max, 4),
            "bytes_per_step": int(total_bytes), "value": round(gbs, 1), "unit": "GB/s",
            "tok_per_s": round(len(all_lens) / (ms_max / 1e3), 1),
            "frac": round(gbs / (peaks["hbm_gbs"] * world), 4),
            "peak": round(peaks["hbm_gbs"] * world, 1), "peak_source": src + " x n_gpus",
            "timing": "CUDA events around the decode launches on every rank, max over ranks; "
                      "inputs larger than L2 (%.2f GB read per rank per step)" % (nbytes / 1e9),
            "limiter": "the slowest rank (LPT length imbalance and per-rank wave quantisation); "
                       "no collective on the path"}


def run_c5_leg(args, rank, world, local_rank, new_tokens=256, requests=256):
    """Config 5: Qwen3-0.6B end to end (28 layers, random N(0, 0.02) weights),
    256 concurrent requests with prompts U[32, 1024] and 256 generated tokens
    each: one prefill of every prompt, then decode steps of the whole batch
    replayed from a CUDA graph (GraphRunner), greedy sampling with the fused
    sampler.  Requests are sharded over the ranks (data parallel, LPT on prompt
    length); tokens/s = all generated tokens / max-over-ranks device time."""
    import torch
    import torch.distributed as dist
    from qwen3_engine_from_scratch_b200 import e2e_model
    from qwen3_engine_from_scratch_b200.dist import lpt_partition

    device = torch.device("cuda", local_rank)
    cfg = e2e_model.QWEN3_0_6B
    prompts = e2e_model.synthetic_prompts(requests, 32, 1024, cfg["vocab"], seed=55)
    mine = lpt_partition([len(p) + new_tokens for p in prompts], world)[rank]
    local = [prompts[i] for i in mine]
    model = e2e_model.Qwen3DecodeModel(device, seed=5, **cfg)
    # warm-up: a small serve of the same shapes compiles nothing but loads every kernel
    e2e_model.serve(model, local[:4], 4, device, graph=True, buckets=(4,))
    if world > 1:
        dist.barrier()
    tokens, st = e2e_model.serve(model, local, new_tokens, device, graph=True,
                                 buckets=(len(local),))
    t = torch.tensor([st["prefill_ms"] + st["decode_ms"], st["decode_ms"], st["prefill_ms"],
                      float(len(local))], dtype=torch.float64, device=device)
    if world > 1:
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        total_ms, dec_ms, pre_ms = float(tmax[0]), float(tmax[1]), float(tmax[2])
    else:
        total_ms, dec_ms, pre_ms = float(t[0]), float(t[1]), float(t[2])
    del model
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    gen = requests * new_tokens
    ok = bool((tokens >= 0).all() and (tokens < cfg["vocab"]).all())
    return {"workload": "c5_qwen3_0.6b_end_to_end", "model": "Qwen3-0.6B shape, random N(0,0.02)",
            "layers": cfg["layers"], "requests": requests, "prompts": "U[32,1024]",
            "new_tokens_per_request": new_tokens, "parallelism": f"data parallel x{world}",
            "requests_per_rank_max": int(max(len(s) for s in lpt_partition(
                [len(p) + new_tokens for p in prompts], world))),
            "tok_per_s": round(gen / (total_ms / 1e3), 1),
            "tok_per_s_per_gpu": round(gen / (total_ms / 1e3) / world, 1),
            "decode_tok_per_s": round(requests * (new_tokens - 1) / (dec_ms / 1e3), 1),
            "ms_total": round(total_ms, 2), "ms_prefill": round(pre_ms, 2),
            "ms_decode": round(dec_ms, 2), "decode_steps": new_tokens - 1,
            "tokens_in_vocab": ok,
            "timing": "CUDA events around the prefill of all prompts and the decode loop "
                      "(graph replays + fused greedy sampler, host page reservation between "
                      "steps), max over ranks",
            "path": "prologue qk_norm_rope_kv_write, varlen prefill, kv_scatter_slots, fused "
                    "KV-write decode via triton_paged_attention_decode_batch, sample_tokens; "
                    "GEMMs / MLP / norms in torch"}


def bench_sampling(device, steps=20, warmup=3):
    """Fused sampler on a Qwen3 decode batch (64 x 151936 bf16 logits) against
    torch.topk alone, the first of the reference path's two launches
    (qwen3/sampling.py:215-216), and greedy against torch.argmax."""
    import torch
    from qwen3_engine_from_scratch_b200 import ops
    g = torch.Generator(device=device).manual_seed(17)
    B, V = 64, 151936
    logits = (torch.randn(B, V, generator=g, device=device) * 3).to(torch.bfloat16)

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps * 1e3   # us

    def graphed(fn):   # device time of one call: the call captured in a CUDA graph
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            fn()
        t = timed(graph.replay)
        del graph
        return t

    calls = {"fused": lambda: ops.sample_tokens(logits, 0.7, 50, 0.9, seed=1),
             "torch_topk_only": lambda: torch.topk(logits, 50, dim=-1, largest=True, sorted=True),
             "greedy": lambda: ops.sample_tokens(logits, 0.0),
             "torch_argmax": lambda: logits.argmax(dim=-1)}
    res = {"kernel": "sample_chunk_kernel + sample_row_fast_kernel", "batch": B, "vocab": V,
           "dtype": "bf16", "params": "temperature 0.7, top_k 50, top_p 0.9",
           "timing": "per call from Python (eager, host included) and device time of the "
                     "call replayed from a CUDA graph"}
    for name, fn in calls.items():
        res[name + "_us"] = round(timed(fn), 2)
        res[name + "_graph_us"] = round(graphed(fn), 2)
    return res


def run_prefill(args, rank, world, local_rank, steps, warmup, headline=False):
    """Config 3: varlen causal prefill of 32 packed sequences (+ the slot scatter of
    their K/V into a paged pool through a random slot_mapping), timed with CUDA events."""
    import torch
    import qwen3_engine_from_scratch_b200 as qb
    from qwen3_engine_from_scratch_b200 import ops

    device = torch.device("cuda", local_rank)
    w = workload("c3", rank, world)
    H, Hkv, D = w["H"], w["Hkv"], HEAD_DIM
    lens = np.asarray(w["lens"], dtype=np.int64)
    T = int(lens.sum())
    g = torch.Generator(device=device).manual_seed(77 + rank)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=device)
    pos = torch.from_numpy(np.concatenate([np.arange(L) for L in lens])).to(device).float()
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D))
    ang = pos[:, None] * inv[None]
    cos = torch.cat([ang, ang], -1).cos()[:, None]
    sin = torch.cat([ang, ang], -1).sin()[:, None]

    def rms_rope(x):
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)
        return x * cos + torch.cat([-x[..., D // 2:], x[..., :D // 2]], -1) * sin

    q = rms_rope(torch.randn(T, H, D, generator=g, device=device)).to(torch.bfloat16)
    k = rms_rope(torch.randn(T, Hkv, D, generator=g, device=device)).to(torch.bfloat16)
    v = torch.randn(T, Hkv, D, generator=g, device=device).to(torch.bfloat16)
    nb = (T + 15) // 16 + 64
    kp = torch.zeros(nb, 1, Hkv, 16, D, dtype=torch.bfloat16, device=device)
    vp = torch.zeros_like(kp)
    slots = torch.randperm(nb * 16, generator=g, device=device)[:T].to(torch.int64)
    max_len = int(lens.max())
    scale = D ** -0.5
    out = torch.empty(T, H, D, dtype=torch.bfloat16, device=device)

    def prefill():
        ops._prefill(q, k, v, out, cu, None, max_len, scale, H, Hkv, D, False)

    for _ in range(warmup):
        prefill()
        ops.kv_scatter_slots(k, v, kp, vp, slots)
    torch.cuda.synchronize()
    qb.check_device_status(device)
    stream = torch.cuda.current_stream()
    pa = [torch.cuda.Event(enable_timing=True)]
    pb = [torch.cuda.Event(enable_timing=True)]
    sb = [torch.cuda.Event(enable_timing=True)]
    clocks = ClockSampler(local_rank) if headline else None
    if clocks is not None:
        clocks.start()
    # the prefill launches back to back between one pair of events (each one's
    # q/k/v reads miss L2 anyway: 259.6 MB per launch), as the chunked and
    # prologue legs are timed; then the slot-mode KV write of the same tokens
    # in a loop of its own
    pa[0].record(stream)
    for i in range(steps):
        prefill()
    pb[0].record(stream)
    for i in range(steps):
        ops.kv_scatter_slots(k, v, kp, vp, slots)
    sb[0].record(stream)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.stop()
    qb.check_device_status(device)
    p_ms = pa[0].elapsed_time(pb[0]) / steps
    s_ms = pb[0].elapsed_time(sb[0]) / steps
    flops = prefill_flops(lens, H)
    sbytes = T * Hkv * D * 2 * 2 * 2 + T * 8
    peaks, src = read_peaks()
    tflops = flops / (p_ms / 1e3) / 1e12
    extra = {}
    if headline:
        # e2e through the public entry point: every step uploads its q/k/v from
        # pinned host memory, runs the prefill and downloads the output, all
        # inside the timed region.  Steps are pipelined over two buffer slots as
        # a serving loop would run them: step i's download (one copy engine)
        # overlaps step i + 1's upload (the other) and the prefill between them.
        hq, hk, hv = q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()
        hout = [torch.empty((T, H, D), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        dq = [torch.empty_like(q) for _ in range(2)]
        dk = [torch.empty_like(k) for _ in range(2)]
        dv = [torch.empty_like(v) for _ in range(2)]
        up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
        landed = [torch.cuda.Event() for _ in range(2)]
        computed = [torch.cuda.Event() for _ in range(2)]
        issued = [0]

        def e2e_step():
            i = issued[0]
            issued[0] += 1
            sl = i & 1
            with torch.cuda.stream(up):
                if i >= 2:
                    up.wait_event(computed[sl])   # the prefill of step i - 2 read this slot
                dq[sl].copy_(hq, non_blocking=True)
                dk[sl].copy_(hk, non_blocking=True)
                dv[sl].copy_(hv, non_blocking=True)
                landed[sl].record(up)
            stream.wait_event(landed[sl])
            o = ops.flash_attention_prefill(dq[sl], dk[sl], dv[sl], cu, scale, H, Hkv, D,
                                            max_seqlen=max_len)
            computed[sl].record(stream)
            with torch.cuda.stream(down):
                down.wait_event(computed[sl])
                hout[sl].copy_(o, non_blocking=True)
                o.record_stream(down)

        for _ in range(max(2, warmup)):
            e2e_step()
        torch.cuda.synchronize()
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ea.record(stream)
        up.wait_stream(stream)
        down.wait_stream(stream)
        for _ in range(steps):
            e2e_step()
        stream.wait_stream(up)
        stream.wait_stream(down)
        eb.record(stream)
        torch.cuda.synchronize()
        e_ms = ea.elapsed_time(eb) / steps
        extra["e2e"] = {"value": round(flops / (e_ms / 1e3) / 1e12, 1), "unit": "TFLOP/s",
                        "ms_per_step": round(e_ms, 4),
                        "h2d_bytes_per_step": int((hq.numel() + hk.numel() + hv.numel()) * 2),
                        "d2h_bytes_per_step": int(hout[0].numel() * 2),
                        "api": "flash_attention_prefill (qwen3/kernels/flash_attention_varlen.py:"
                               "126-194 signature, max_seqlen given: no host sync) with q/k/v "
                               "copied from pinned host memory and the output copied back, every "
                               "step; steps pipelined over two buffer slots (a step's download "
                               "overlaps the next step's upload on the other copy engine)"}
        extra["clocks"] = clocks.summary()
        extra["gpu_launches"] = steps * 2   # the prefill and the slot-mode KV write per step
    prologue = bench_prologue(torch, ops, device, g, T, H, Hkv, D, steps, warmup, peaks)
    chunked = bench_paged_prefill(torch, ops, device, rank, H, Hkv, D, steps, warmup, peaks)
    return {"workload": w["name"], "tokens": T, "sequences": len(lens),
            "lengths": "U[64,2048]", "heads": f"{H}/{Hkv}",
            "ms_per_prefill": round(p_ms, 4), "tflops": round(tflops, 1),
            "flops_per_launch": flops,
            "roofline": {"kernel": "varlen_prefill_kernel", "bound": "tensor",
                         "achieved": round(tflops, 1), "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": round(tflops / peaks["bf16_tflops"], 4),
                         "peak_source": src, "traffic": read_traffic("varlen_prefill_kernel")},
            "scatter": {"kernel": "kv_scatter_slots_kernel", "ms": round(s_ms, 4),
                        "bytes": sbytes, "gbs": round(sbytes / (s_ms / 1e3) / 1e9, 1),
                        "frac_hbm": round(sbytes / (s_ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
                        "traffic": read_traffic("kv_scatter_slots_kernel")},
            "prologue": prologue,
            "paged_prefill": chunked,
            "gpu_launches_per_step": 2, **extra}


def bench_paged_prefill(torch, ops, device, rank, H, Hkv, D, steps, warmup, peaks):
    """Chunked prefill over the paged cache: 32 sequences with U[0, 2048] tokens
    already cached and a new chunk of U[64, 512] tokens each (pages placed by a
    random permutation), attention of the new tokens over context + chunk."""
    rng = np.random.default_rng(5000 + rank)
    ctx = rng.integers(0, 2048, size=32, endpoint=True)
    new = rng.integers(64, 512, size=32, endpoint=True)
    g = torch.Generator(device=device).manual_seed(91 + rank)
    totals = ctx + new
    max_pages = int(((totals + 15) // 16).max())
    nb = int(((totals + 15) // 16).sum()) + 8
    kp = torch.randn(nb, Hkv, 16, D, generator=g, device=device).to(torch.bfloat16)
    vp = torch.randn(nb, Hkv, 16, D, generator=g, device=device).to(torch.bfloat16)
    perm = torch.randperm(nb, generator=g, device=device).to(torch.int32)
    bt = torch.full((32, max_pages), -1, dtype=torch.int32, device=device)
    used = 0
    for i in range(32):
        npg = int((totals[i] + 15) // 16)
        bt[i, :npg] = perm[used:used + npg]
        used += npg
    seq = torch.from_numpy(ctx.astype(np.int32)).to(device)
    rows = torch.arange(32, dtype=torch.int32, device=device)
    T = int(new.sum())
    q = torch.randn(T, H, D, generator=g, device=device).to(torch.bfloat16)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(new)]).astype(np.int32)).to(device)
    out = torch.empty(T, H, D, dtype=torch.bfloat16, device=device)
    mx = int(new.max())

    def call():
        ops.paged_prefill(q, kp, vp, bt, seq, rows, cu, D ** -0.5, max_new_tokens=mx, out=out)

    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        call()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    # causal pairs: new token t of sequence i sees ctx_i + t + 1 keys
    pairs = int(sum(int(n) * int(c) + int(n) * (int(n) + 1) // 2 for c, n in zip(ctx, new)))
    flops = 4 * H * D * pairs
    tf = flops / (ms / 1e3) / 1e12
    return {"kernel": "varlen_prefill_kernel (paged mode)", "sequences": 32,
            "cached": "U[0,2048]", "new_tokens": T, "chunk": "U[64,512]", "ms": round(ms, 4),
            "flops_per_launch": flops, "tflops": round(tf, 1),
            "frac_bf16": round(tf / peaks["bf16_tflops"], 4)}


def bench_prologue(torch, ops, device, g, T, H, Hkv, D, steps, warmup, peaks):
    """The fused QK-norm + RoPE + KV write over the config-3 tokens (as one request of T
    positions, q/k/v views of a fused projection output), against the reference's
    unfused op sequence (RMSNorm modules, apply_rotary_pos_emb, then the KV write)."""
    qkv = torch.randn(1, T, (H + 2 * Hkv) * D, generator=g, device=device).to(torch.bfloat16)
    q = qkv[..., :H * D].view(1, T, H, D).transpose(1, 2)
    k = qkv[..., H * D:(H + Hkv) * D].view(1, T, Hkv, D).transpose(1, 2)
    v = qkv[..., (H + Hkv) * D:].view(1, T, Hkv, D).transpose(1, 2)
    wq = (1 + 0.1 * torch.randn(D, generator=g, device=device)).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(D, generator=g, device=device)).to(torch.bfloat16)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D))
    ang = torch.arange(T, device=device, dtype=torch.float32)[:, None] * inv[None]
    emb = torch.cat([ang, ang], -1)[None]
    cos, sin = emb.cos(), emb.sin()                      # (1, T, D) fp32 rows
    pages = (T + 15) // 16
    kp = torch.zeros(pages + 1, 1, Hkv, 16, D, dtype=torch.bfloat16, device=device)
    vp = torch.zeros_like(kp)
    bt = torch.arange(pages, dtype=torch.int32, device=device)[None].contiguous()
    seq = torch.zeros(1, dtype=torch.int32, device=device)
    rows = torch.zeros(1, dtype=torch.int32, device=device)

    def fused():
        return ops.qk_norm_rope_kv_write(q, k, v, wq, wk, cos, sin, k_buffer=kp, v_buffer=vp,
                                         seq_lens=seq, block_table_2d=bt, row_ids=rows, layer_idx=0)

    def rms(x, w):   # qwen3/norm.py:22-26
        xf = x.float()
        return ((xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)) * w).to(x.dtype)

    def unfused():   # qwen3/attention.py:90-95 with qwen3/rope.py:104-110, then the KV write
        qn, kn = rms(q, wq), rms(k, wk)
        c, s_ = cos[:, None].to(torch.bfloat16), sin[:, None].to(torch.bfloat16)
        rq = qn * c + torch.cat([-qn[..., D // 2:], qn[..., :D // 2]], -1) * s_
        rk = kn * c + torch.cat([-kn[..., D // 2:], kn[..., :D // 2]], -1) * s_
        ops.kv_scatter_rows(rk, v, kp, vp, seq, bt, rows, 0)
        return rq

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps

    f_ms, u_ms = timed(fused), timed(unfused)
    nbytes = T * (H + 2 * Hkv) * D * 2 + 2 * T * D * 4 + T * H * D * 2 + 2 * T * Hkv * D * 2
    gbs = nbytes / (f_ms / 1e3) / 1e9
    return {"kernel": "qk_norm_rope_kv_write_kernel", "tokens": T, "ms": round(f_ms, 4),
            "bytes": nbytes, "gbs": round(gbs, 1), "frac_hbm": round(gbs / peaks["hbm_gbs"], 4),
            "traffic": read_traffic("qk_norm_rope_kv_write_kernel"),
            "unfused_ms": round(u_ms, 4), "speedup_vs_unfused": round(u_ms / f_ms, 2),
            "unfused": "the reference's RMSNorm x2 + apply_rotary_pos_emb in torch ops, then "
                       "kv_scatter_rows"}


def read_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"]))}, \
            "measured (MEASURED_PEAKS.json)"
    except Exception:
        return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
                "bf16_tflops_sustained": 1400.0}, "fallback"


def read_traffic(kernel):
    """dram bytes (read+write) per launch from the committed ncu summary, if any."""
    p = os.path.join(REPO, "profiles", "traffic.json")
    try:
        return json.load(open(p)).get(kernel)
    except Exception:
        return None


# ---------------------------------------------------------------------------
# CPU baseline / reference arm: the oracle port of the reference algorithm
# ---------------------------------------------------------------------------

def _cpu_work(w, seed=7):
    """A host copy of one layer of the workload (compact pool of the used pages)."""
    from oracle import synth
    lens = np.asarray(w["lens"], dtype=np.int64)
    H, Hkv, D = w["H"], w["Hkv"], HEAD_DIM
    pages = (lens + BLOCK - 1) // BLOCK
    n = int(pages.sum())
    perm = synth.det_permutation(seed, n)
    bt = np.full((len(lens), int(pages.max())), -1, np.int32)
    o = 0
    for b, p in enumerate(pages):
        bt[b, :p] = perm[o:o + p]
        o += p
    rng = np.random.default_rng(seed)
    kp = rng.standard_normal((n, Hkv, BLOCK, D), dtype=np.float32)
    vp = rng.standard_normal((n, Hkv, BLOCK, D), dtype=np.float32)
    q = rng.standard_normal((len(lens), H, D), dtype=np.float32)
    seq = (lens - 1).astype(np.int32)
    return q, kp, vp, bt, seq


def _cpu_worker(args):
    """Spawned worker: attach the shared pool and run the oracle on some requests."""
    from multiprocessing import shared_memory
    from oracle.attention import paged_decode
    (names, shapes, idx) = args
    shms = [shared_memory.SharedMemory(name=n) for n in names]
    arrs = [np.ndarray(s, dtype=np.float32 if i < 3 else np.int32, buffer=m.buf)
            for i, (m, s) in enumerate(zip(shms, shapes))]
    q, kp, vp, bt, seq = arrs
    t0 = time.perf_counter()
    paged_decode(q[idx], kp, vp, bt[idx], seq[idx], np.arange(len(idx)), BLOCK, HEAD_DIM ** -0.5)
    dt = time.perf_counter() - t0
    for m in shms:
        m.close()
    return dt


class CpuDecodePool:
    """The oracle decode of one layer of the workload on ``procs`` spawned processes."""

    def __init__(self, w, procs):
        import multiprocessing as mp
        from multiprocessing import shared_memory
        self.w = w
        arrays = _cpu_work(w)
        self.shm = []
        self.names, self.shapes = [], []
        for a in arrays:
            m = shared_memory.SharedMemory(create=True, size=max(1, a.nbytes))
            np.ndarray(a.shape, dtype=a.dtype, buffer=m.buf)[...] = a
            self.shm.append(m)
            self.names.append(m.name)
            self.shapes.append(a.shape)
        self.procs = procs
        self.pool = mp.get_context("spawn").Pool(procs) if procs > 1 else None

    def run(self, idx):
        parts = [idx[i::self.procs] for i in range(self.procs)] if self.pool else [idx]
        parts = [p for p in parts if len(p)]
        jobs = [(self.names, self.shapes, p) for p in parts]
        t0 = time.perf_counter()
        if self.pool is not None:
            self.pool.map(_cpu_worker, jobs)
        else:
            for j in jobs:
                _cpu_worker(j)
        return time.perf_counter() - t0

    def close(self):
        if self.pool is not None:
            self.pool.close()
            self.pool.join()
        for m in self.shm:
            m.close()
            m.unlink()


def cpu_baseline(w, budget_s=20.0, procs=1):
    """Oracle port timed on the host: one layer of the batch on ``procs``
    spawned processes (requests dealt round-robin), repeated until about
    ``budget_s`` seconds of CPU work."""
    lens = np.asarray(w["lens"], dtype=np.int64)
    H, Hkv = w["H"], w["Hkv"]
    cp = CpuDecodePool(w, procs)
    try:
        idx = np.arange(len(lens))
        cp.run(idx[:min(len(idx), procs)])         # warm-up: every worker imports the oracle
        reps, dt = 0, 0.0
        while reps == 0 or dt < budget_s:
            dt += cp.run(idx)
            reps += 1
    finally:
        cp.close()
    b = decode_bytes(lens, H, Hkv) * reps
    return {"value": round(b / dt / 1e9, 3), "unit": "GB/s", "cores": procs, "kind": "port",
            "sample": f"{reps} x 1 layer x {len(lens)} requests of the workload ({dt:.2f} s) on "
                      f"{procs} spawned processes, oracle.paged_decode (numpy fp32 restatement of "
                      f"the reference's CPU path qwen3/paged_attention.py; a restatement, so its "
                      f"speed stands in for, and is not, the reference's own torch code)"}


def prefill_cpu_baseline(budget_s):
    """cpu_baseline object of the prefill leg: the oracle's fp32 varlen prefill
    of config-3 sequences on the host cores."""
    fl, dt, used = prefill_cpu_sample(workload("c3", 0, 1), budget_s)
    threads = max(1, os.cpu_count() or 1)
    return {"value": round(fl / dt / 1e12, 6), "unit": "TFLOP/s", "cores": threads,
            "kind": "port",
            "sample": f"{len(used)}/32 sequences of the config-3 batch (shortest first, lengths "
                      f"{min(used)}-{max(used)}) in {dt:.1f} s, oracle.varlen_prefill (numpy fp32 "
                      f"restatement of the reference's causal _standard_attention; its matmuls on "
                      f"OpenBLAS threads over the {threads} host cores, the softmax on one)"}


def prefill_cpu_sample(w, budget_s):
    """Oracle varlen prefill (numpy fp32, the reference's _standard_attention
    semantics) on the shortest-first sequences of the config-3 batch until about
    ``budget_s`` seconds of CPU work; returns (flops, seconds, sequences)."""
    from oracle import attention as oa
    lens = np.asarray(w["lens"], dtype=np.int64)
    H, Hkv, D = w["H"], w["Hkv"], HEAD_DIM
    rng = np.random.default_rng(3)
    order = np.argsort(lens, kind="stable")
    flops = 0
    used = []
    t0 = time.perf_counter()
    for i in order:
        L = int(lens[i])
        q = rng.standard_normal((L, H, D), dtype=np.float32)
        k = rng.standard_normal((L, Hkv, D), dtype=np.float32)
        v = rng.standard_normal((L, Hkv, D), dtype=np.float32)
        oa.varlen_prefill(q, k, v, np.array([0, L]), D ** -0.5)
        flops += prefill_flops([L], H)
        used.append(L)
        if time.perf_counter() - t0 > budget_s:
            break
    return flops, time.perf_counter() - t0, used


def run_reference(args, rank, world):
    """--impl reference: the reference algorithm (oracle port) on the host cores."""
    if rank != 0:
        return None
    if args.config == "c3":
        w = workload("c3", 0, 1)
        threads = max(1, os.cpu_count() or 1)
        budget = 150.0 / max(1, args.steps + args.warmup)
        fl, dt, used = 0, 0.0, []
        for i in range(args.warmup + args.steps):
            f_, d_, u_ = prefill_cpu_sample(w, budget)
            if i >= args.warmup:
                fl, dt, used = fl + f_, dt + d_, u_
        value = fl / dt / 1e12
        sample = (f"{len(used)}/{len(w['lens'])} sequences of the config-3 batch per step "
                  f"(shortest first, lengths {min(used)}-{max(used)}), oracle.varlen_prefill (numpy "
                  f"fp32 restatement of the reference's causal _standard_attention), numpy BLAS "
                  f"threads on {threads} host cores")
        return {
            "metric": "varlen_prefill_tflops", "value": round(value, 6), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "config": {"workload": w["name"]},
            "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
    w = workload(args.config, 0, 1)
    lens = np.asarray(w["lens"], dtype=np.int64)
    H, Hkv = w["H"], w["Hkv"]
    procs = max(1, os.cpu_count() or 1)
    cp = CpuDecodePool(w, procs)
    try:
        idx = np.arange(len(lens))
        dt1 = cp.run(idx[: min(len(idx), procs)])
        # size each step's sample so the whole run stays within ~3 minutes
        per_req = dt1 / max(1, min(len(idx), procs)) * procs
        budget_step = 150.0 / max(1, args.steps + args.warmup)
        n = int(max(1, min(len(idx), budget_step / max(per_req / procs, 1e-4))))
        sample = idx[:n]
        for _ in range(args.warmup):
            cp.run(sample)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            cp.run(sample)
        dt = time.perf_counter() - t0
    finally:
        cp.close()
    b = decode_bytes(lens[:n], H, Hkv)
    value = b * args.steps / dt / 1e9
    line = {
        "metric": "paged_decode_attention_hbm_bandwidth", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": w["scaling"], "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": w["name"], "heads": f"{H}/{Hkv}", "head_dim": HEAD_DIM,
                   "batch_per_gpu": len(lens), "layers_per_step": 1},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": procs, "kind": "port",
                         "sample": f"1 layer x {n}/{len(lens)} requests per step, oracle.paged_decode "
                                   f"(numpy restatement of qwen3/paged_attention.py) on {procs} "
                                   f"spawned processes; the reference's own torch code is not on "
                                   f"the GPU box, so this restatement's speed stands in for it"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c2", choices=["c2", "c3", "c4", "sampling"],
                    help="sampling: only the fused sampler's leg (a small case for profiling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-c4", action="store_true",
                    help="skip the config-4 strong-scaling leg of the default run")
    ap.add_argument("--no-c5", action="store_true",
                    help="skip the config-5 end-to-end leg of the default run")
    ap.add_argument("--layers", type=int, default=0,
                    help="layers per step (default: 28 for c2); 1 gives a small case for profiling")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    from qwen3_engine_from_scratch_b200.dist import rank_env
    rank, world, local_rank = rank_env()
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.config == "sampling":
            torch.cuda.set_device(local_rank)
            line = bench_sampling(torch.device("cuda", local_rank)) if rank == 0 else None
        elif args.config == "c3":
            torch.cuda.set_device(local_rank)
            r = run_prefill(args, rank, world, local_rank, steps=args.steps, warmup=args.warmup,
                            headline=True)
            line = None
            if rank == 0:
                line = {"metric": "varlen_prefill_tflops", "value": r["tflops"], "unit": "TFLOP/s",
                        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                        "ms_per_step": r["ms_per_prefill"], "higher_is_better": True,
                        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                        "data": "synthetic: N(0,1) q/k/v, q/k RMS-normed + RoPE theta 1e6",
                        "config": {"workload": r["workload"], "sequences": r["sequences"],
                                   "tokens": r["tokens"], "lengths": r["lengths"],
                                   "heads": r["heads"], "head_dim": HEAD_DIM,
                                   "l2": "inputs larger than L2 (q/k/v 259.6 MB per step)",
                                   "parallelism": f"request-sharded x{world}" if world > 1
                                   else "single GPU"},
                        "roofline": r["roofline"], "e2e": r["e2e"], "clocks": r["clocks"],
                        "gpu_launches": r["gpu_launches"], "detail": r}
                if world == 1 and not args.no_cpu_baseline:
                    fl, dt, used = prefill_cpu_sample(workload("c3", 0, 1), args.cpu_budget)
                    line["cpu_baseline"] = {
                        "value": round(fl / dt / 1e12, 6), "unit": "TFLOP/s",
                        "cores": max(1, os.cpu_count() or 1), "kind": "port",
                        "sample": f"{len(used)}/32 sequences (shortest first, lengths "
                                  f"{min(used)}-{max(used)}) in {dt:.1f} s, oracle.varlen_prefill "
                                  f"(numpy fp32, BLAS threads on the host cores)"}
        else:
            line = run_b200(args, rank, world, local_rank)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
