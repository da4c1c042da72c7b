"""CUDA-graph pool for the decode step: one captured graph per batch bucket.

Keeps the constructor and ``replay`` contract of the reference's GraphRunner
(qwen3/graph_runner.py:26-200).  ``model.forward_decode(input_ids,
position_ids, row_ids, caches)`` (qwen3/model.py:186-251) is captured once per
bucket with fixed input tensors whose addresses the graph bakes in
(:105-162); ``replay`` copies a step's inputs into them, fills the unused
slots with a dummy row (:80-89, :188-191) and replays the smallest bucket
that holds the batch (:181-186).  The attention path inside
``forward_decode`` (the KV write and the split-K decode, both with
device-side state only) is capture-safe as it is: its workspaces are
allocated on the capture stream during warm-up and every launch leaves their
counters at zero.

Changes for serving one engine per GPU (data parallel over 8 GPUs, one
process per GPU):

* buckets default to the powers of two up to 256 (the reference's default
  stops at 8, :39);
* graphs are captured largest bucket first, on one capture stream, into one
  shared memory pool: the smaller graphs reuse the largest one's
  intermediates, and the kernels' per-stream workspaces reach their final
  size during the first warm-up, before any capture (the reference captures
  smallest first, :104);
* the placeholder handles need one page each (``reserve_pages=1``): the
  decode reads only the pages below ``seq_len + 1``, so the reference's
  default of 64 pages per placeholder (:39, :62-65) would hold
  ``64 * max_bucket`` pool blocks for nothing;
* ``replay`` also takes host inputs (Python lists, numpy arrays or CPU
  tensors): they are packed, dummy slots included, into a pinned staging
  buffer and reach the fixed tensors with one asynchronous copy each, where
  the reference's loop builds two device tensors per step
  (bench_batched.py:180-187) and ``replay`` adds a fill (:190-191);
* ``kv_pool_blocks`` sizes a rank's pool from the free HBM of its GPU.
"""

from __future__ import annotations

import numpy as np
import torch

DEFAULT_BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256)


def bucket_for(buckets, k: int) -> int:
    """The smallest bucket >= k (qwen3/graph_runner.py:181-186).

    ``buckets`` is sorted ascending.  Raises ValueError when k exceeds the
    largest bucket (the reference's ``min()`` of an empty sequence).
    """
    if k < 0:
        raise ValueError(f"batch size must be >= 0, got {k}")
    for b in buckets:
        if b >= k:
            return b
    raise ValueError(f"batch of {k} requests exceeds the largest captured bucket "
                     f"{buckets[-1]}")


def pack_host_inputs(ids_out: np.ndarray, pos_out: np.ndarray, rows_out: np.ndarray,
                     input_ids, positions, rows, dummy_row: int) -> int:
    """Write one step's host inputs into staging arrays of the bucket size.

    ``ids_out``/``pos_out`` (int64) and ``rows_out`` (int32) have the bucket's
    length b; slots ``[k, b)`` get token 0, position 0 and ``dummy_row``.
    Returns k.
    """
    ids = np.asarray(input_ids, dtype=np.int64).reshape(-1)
    pos = np.asarray(positions, dtype=np.int64).reshape(-1)
    rws = np.asarray(rows, dtype=np.int64).reshape(-1)
    k = ids.shape[0]
    if pos.shape[0] != k or rws.shape[0] != k:
        raise ValueError(f"input_ids, positions and rows must have one entry per request "
                         f"(got {k}, {pos.shape[0]}, {rws.shape[0]})")
    b = ids_out.shape[0]
    if k > b:
        raise ValueError(f"{k} requests do not fit a bucket of {b}")
    ids_out[:k] = ids
    pos_out[:k] = pos
    rows_out[:k] = rws
    ids_out[k:] = 0
    pos_out[k:] = 0
    rows_out[k:] = dummy_row
    return k


def kv_pool_blocks(num_layers: int, num_kv_heads: int, head_dim: int, block_size: int = 16,
                   dtype=torch.bfloat16, device=None, fraction: float = 0.9,
                   reserve_bytes: int = 4 << 30, free_bytes: int | None = None) -> int:
    """Blocks of a K+V pool ``(num_blocks, num_layers, Hkv, block_size, D)``
    (qwen3/PagedKVcache.py:44-53) that fit in this GPU's free memory.

    Takes ``fraction`` of the free bytes (``torch.cuda.mem_get_info`` unless
    ``free_bytes`` is given) minus ``reserve_bytes`` for weights and graph
    intermediates still to be allocated.  Each rank sizes its own pool.
    """
    elem = torch.empty((), dtype=dtype).element_size()
    per_block = 2 * num_layers * num_kv_heads * block_size * head_dim * elem
    if free_bytes is None:
        free_bytes, _ = torch.cuda.mem_get_info(device)
    avail = int(free_bytes * fraction) - int(reserve_bytes)
    return max(0, avail // per_block)


class GraphRunner:
    """CUDA-graph pool of the decode step, one graph per batch bucket.

    runner = GraphRunner(model, pool, caches, buckets=DEFAULT_BUCKETS, reserve_pages=1)
    logits = runner.replay(input_ids, positions, rows)   # (b, 1, vocab); rows [0, k) valid

    ``caches`` are placeholder handles (at least ``max(buckets)``) that give
    the capture stable rows and pool state; at run time the real requests'
    rows are copied in.  The caller reserves pages (``reserve_next``) before
    and advances lengths (``advance_seq_len``) after each replay
    (bench_batched.py:177-197).  Replays must be issued from one stream at a
    time: all graphs share the capture stream's workspaces.
    """

    def __init__(self, model, pool, caches, buckets=DEFAULT_BUCKETS, reserve_pages=1,
                 warmup_iters: int = 3):
        self.model = model
        self.pool = pool
        self.buckets = tuple(sorted(set(int(b) for b in buckets)))
        if not self.buckets or self.buckets[0] < 1:
            raise ValueError(f"buckets must be positive batch sizes, got {buckets!r}")
        self.max_batch = self.buckets[-1]
        assert len(caches) >= self.max_batch, \
            f"need >= max bucket ({self.max_batch}) placeholder caches, got {len(caches)}"
        reserve_pages = max(1, int(reserve_pages))

        # placeholders in the decode state with their pages reserved (:56-73):
        # no page allocation may happen during capture
        for c in caches[:self.max_batch]:
            while c.num_pages < reserve_pages:
                c._allocate_block()
            c.seq_len = 1
            pool.seq_lens[c.row_id] = 1

        # the dummy row for unused slots: seq_len 0 and one valid page (:80-89)
        self.dummy_row = pool.alloc_row()
        self._dummy_phys = pool.alloc(1)[0]
        pool.block_table_2d[self.dummy_row, 0] = self._dummy_phys
        pool.seq_lens[self.dummy_row] = 0

        self.device = pool.k_buffer.device
        self._pool_handle = torch.cuda.graph_pool_handle()
        self._stream = torch.cuda.Stream(self.device)
        self.graphs: dict[int, tuple[torch.cuda.CUDAGraph, dict]] = {}
        self._capture_all(caches, warmup_iters)

        # pinned host staging, two slots so a step can be packed while the
        # previous step's copies are still in flight
        self._stage_ids = torch.zeros((2, self.max_batch), dtype=torch.int64).pin_memory()
        self._stage_pos = torch.zeros((2, self.max_batch), dtype=torch.int64).pin_memory()
        self._stage_rows = torch.zeros((2, self.max_batch), dtype=torch.int32).pin_memory()
        self._stage_done = [None, None]
        self._slot = 0

    @torch.no_grad()
    def _capture_all(self, caches, warmup_iters):
        dev = self.device
        cur = torch.cuda.current_stream(dev)
        self._stream.wait_stream(cur)
        for b in sorted(self.buckets, reverse=True):
            s_input = torch.zeros((b, 1), dtype=torch.long, device=dev)
            s_pos = torch.zeros((b, 1), dtype=torch.long, device=dev)
            s_rows = torch.tensor([c.row_id for c in caches[:b]], dtype=torch.int32, device=dev)
            self._stream.wait_stream(cur)
            with torch.cuda.stream(self._stream):
                for _ in range(warmup_iters):
                    self.model.forward_decode(s_input, s_pos, s_rows, caches[:b])
            self._stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self._pool_handle, stream=self._stream):
                logits = self.model.forward_decode(s_input, s_pos, s_rows, caches[:b])
            self._stream.synchronize()
            self.graphs[b] = (g, {"input": s_input, "pos": s_pos, "rows": s_rows,
                                  "logits": logits})
        cur.wait_stream(self._stream)

    def replay(self, input_ids, positions, rows):
        """One decode step for k requests; returns the bucket's (b, 1, vocab)
        logits tensor (rows [0, k) valid, overwritten by the next replay).

        Device tensors are copied as the reference does (:188-191); host
        inputs go through the pinned staging buffer.
        """
        on_device = isinstance(input_ids, torch.Tensor) and input_ids.is_cuda
        k = int(input_ids.shape[0]) if hasattr(input_ids, "shape") else len(input_ids)
        b = bucket_for(self.buckets, k)
        g, t = self.graphs[b]
        if on_device:
            t["input"][:k].copy_(input_ids)
            t["pos"][:k].copy_(positions)
            t["rows"][:k].copy_(rows)
            if k < b:
                t["rows"][k:].fill_(self.dummy_row)
        else:
            slot = self._slot
            self._slot ^= 1
            done = self._stage_done[slot]
            if done is not None:
                done.synchronize()       # the copies that last read this slot
            ids = self._stage_ids[slot, :b]
            pos = self._stage_pos[slot, :b]
            rws = self._stage_rows[slot, :b]
            pack_host_inputs(ids.numpy(), pos.numpy(), rws.numpy(),
                             _host(input_ids), _host(positions), _host(rows), self.dummy_row)
            t["input"].view(-1).copy_(ids, non_blocking=True)
            t["pos"].view(-1).copy_(pos, non_blocking=True)
            t["rows"].copy_(rws, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self._stage_done[slot] = ev
        g.replay()
        return t["logits"]

    def free(self):
        """Release the graphs, the dummy row and its page (:194-200)."""
        self.graphs.clear()
        self.pool.free(self._dummy_phys)
        self.pool.free_row(self.dummy_row)


def _host(x):
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().numpy()
    return x
