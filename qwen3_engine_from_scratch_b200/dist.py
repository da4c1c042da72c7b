"""Multi-GPU request sharding (one process per GPU).

The reference engine is single-GPU (no torch.distributed anywhere).  Its hot
path shards naturally: every request's decode / prefill reads only its own
pages, so requests are partitioned across ranks with no collective on the data
path.  The partition balances work with greedy LPT (longest processing time
first): requests sorted by cost, each to the currently lightest rank.

Decode cost of a request is its visible length L (bytes read ~ L); prefill
cost is L*(L+1)/2 (causal pairs).

``kv_head_tp_all_gather`` is the optional KV-head tensor-parallel exchange:
rank r computes attention for its Hkv/n kv heads (and their query heads) and
one all-gather before o_proj rebuilds (B, H*D).
"""

from __future__ import annotations

import heapq
import os

import torch


def lpt_partition(costs, world_size: int) -> list[list[int]]:
    """Greedy LPT: indices of ``costs`` split into ``world_size`` balanced shards.

    Deterministic (ties broken by index / rank), every index appears once,
    each shard's indices are returned in ascending order.
    """
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(world_size)]
    heapq.heapify(heap)
    shards = [[] for _ in range(world_size)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return [sorted(s) for s in shards]


def shard_loads(costs, shards) -> list[int]:
    return [sum(costs[i] for i in s) for s in shards]


def decode_cost(lens) -> list[int]:
    return [int(x) for x in lens]


def prefill_cost(lens) -> list[int]:
    return [int(x) * (int(x) + 1) // 2 for x in lens]


def rank_env():
    """(rank, world_size, local_rank) from the torchrun environment (1 process if unset)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def kv_head_tp_all_gather(local_out: torch.Tensor, group=None) -> torch.Tensor:
    """KV-head tensor parallelism: gather per-rank attention outputs.

    local_out: (B, H/n, D) -- this rank's query heads, which are the contiguous
    head block [r*H/n, (r+1)*H/n) (rank r owns kv heads [r*Hkv/n, (r+1)*Hkv/n)).
    Returns (B, H*D) in the head order o_proj expects.  One all_gather_into_tensor.
    """
    import torch.distributed as dist
    n = dist.get_world_size(group)
    B, Hl, D = local_out.shape
    buf = torch.empty((n * B, Hl, D), dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(buf, local_out.contiguous(), group=group)
    return buf.view(n, B, Hl, D).permute(1, 0, 2, 3).reshape(B, n * Hl * D)
