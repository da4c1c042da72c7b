"""Host-side mirror of the reference's KV-cache pool and request handles.

``KVCachePool`` / ``PagedKVCache`` keep the attributes, layout and semantics of
qwen3/PagedKVcache.py (the B200 kernels read these tensors as-is):

* pool tensors ``k_buffer``/``v_buffer``: (num_blocks, num_layers, Hkv, 16, D),
  zero-initialised (:44-53); reused blocks are zeroed again on alloc (:58-73);
* ``block_table_2d``: (max_requests, max_pages) int32 filled with -1 (:37-39);
* ``seq_lens``: (max_requests,) int32, the committed length of each row (:40);
* row slots and the block free-list popping from the END (:41, :55, :68-69).

The only behavioural change is where bytes move: ``PagedKVCache.update`` and
``KVCachePool.update_kv_batch`` run the B200 scatter kernel, and
``update_batch`` writes a whole right-padded prefill batch in one launch
(replacing the per-request loop of qwen3/attention.py:160-161).  Allocation
bookkeeping stays on the host, as in the reference.
"""

from __future__ import annotations

import torch

from . import ops


class KVCachePool:
    """Shared physical block pool (qwen3/PagedKVcache.py:19-114)."""

    def __init__(self, num_blocks: int, num_layers: int, block_size: int, num_kv_heads: int,
                 head_dim: int, device=None, dtype=None, max_seq_len: int = 2048,
                 max_requests: int = 256):
        self.num_layers = num_layers
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        max_pages = (max_seq_len + block_size - 1) // block_size
        self.block_table_2d = torch.full((max_requests, max_pages), -1, dtype=torch.int32,
                                         device=device)
        self.seq_lens = torch.zeros(max_requests, dtype=torch.int32, device=device)
        self._free_rows = list(range(max_requests))
        self.max_requests = max_requests
        self.k_buffer = torch.zeros(num_blocks, num_layers, num_kv_heads, block_size, head_dim,
                                    device=device, dtype=dtype)
        self.v_buffer = torch.zeros(num_blocks, num_layers, num_kv_heads, block_size, head_dim,
                                    device=device, dtype=dtype)
        self.free_block_ids = list(range(num_blocks))
        self.total_blocks = num_blocks

    def alloc(self, n: int):
        """Take n blocks from the END of the free list; zero their K/V (:58-73)."""
        if len(self.free_block_ids) < n:
            raise RuntimeError(f"OOM: requested {n} blocks, {len(self.free_block_ids)} / "
                               f"{self.total_blocks} free")
        allocated = self.free_block_ids[-n:]
        del self.free_block_ids[-n:]
        for blk in allocated:
            self.k_buffer[blk].zero_()
            self.v_buffer[blk].zero_()
        return allocated

    def free(self, block_ids):
        if isinstance(block_ids, int):
            block_ids = [block_ids]
        self.free_block_ids.extend(block_ids)

    @property
    def free_count(self):
        return len(self.free_block_ids)

    def alloc_row(self) -> int:
        if not self._free_rows:
            raise RuntimeError(f"OOM: no free row slot (max_requests={self.max_requests})")
        row = self._free_rows.pop()
        self.seq_lens[row] = 0
        return row

    def free_row(self, row: int):
        self._free_rows.append(row)

    def update_kv_batch(self, layer_idx: int, k_new: torch.Tensor, v_new: torch.Tensor,
                        row_ids: torch.Tensor):
        """Decode write of one token per request (qwen3/PagedKVcache.py:99-114).

        k_new, v_new: (B, Hkv, 1, D); pages must be reserved (reserve_next).
        """
        ops.update_kv_batch_triton(k_new.squeeze(2), v_new.squeeze(2), self.k_buffer,
                                   self.v_buffer, self.seq_lens, self.block_table_2d, row_ids,
                                   layer_idx)

    def update_batch(self, caches, layer_idx: int, k_new: torch.Tensor, v_new: torch.Tensor,
                     row_ids: torch.Tensor | None = None):
        """Prefill write of a right-padded batch in one launch.

        Same effect as ``for i, c in enumerate(caches): c.update(layer_idx,
        k_new[i:i+1], v_new[i:i+1])`` (qwen3/attention.py:160-161): every
        request writes all S positions from its current seq_len.
        """
        S = k_new.shape[2]
        for c in caches:
            c._ensure_pages(c.seq_len + S)
        if row_ids is None:
            row_ids = torch.tensor([c.row_id for c in caches], dtype=torch.int32,
                                   device=k_new.device)
        ops.kv_scatter_rows(k_new, v_new, self.k_buffer, self.v_buffer, self.seq_lens,
                            self.block_table_2d, row_ids, layer_idx)


class PagedKVCache:
    """Per-request handle (qwen3/PagedKVcache.py:117-228)."""

    def __init__(self, pool: KVCachePool):
        self._pool = pool
        self.seq_len = 0
        self.block_table = []
        self.row_id = pool.alloc_row()
        self.block_table_tensor = pool.block_table_2d[self.row_id]
        self.num_pages = 0

    def _allocate_block(self):
        max_pages = self.block_table_tensor.shape[0]
        assert self.num_pages < max_pages, \
            f"request exceeds max_seq_len ({self._pool.max_seq_len} tokens / {max_pages} pages)"
        new = self._pool.alloc(1)
        self.block_table.append(new[0])
        self.block_table_tensor[self.num_pages] = new[0]
        self.num_pages += 1

    def _ensure_pages(self, end_pos: int):
        need = (end_pos + self._pool.block_size - 1) // self._pool.block_size
        while len(self.block_table) < need:
            self._allocate_block()

    def reserve_next(self):
        """Reserve the page of the token written this decode step (:152-162)."""
        need = (self.seq_len + 1 + self._pool.block_size - 1) // self._pool.block_size
        if need > self.num_pages:
            self._allocate_block()

    def get_kv(self, layer_idx: int):
        if self.seq_len == 0 or not self.block_table:
            return None, None
        k = torch.cat([self._pool.k_buffer[p, layer_idx] for p in self.block_table], dim=1)
        v = torch.cat([self._pool.v_buffer[p, layer_idx] for p in self.block_table], dim=1)
        return k[:, :self.seq_len].unsqueeze(0), v[:, :self.seq_len].unsqueeze(0)

    def update(self, layer_idx: int, k_new: torch.Tensor, v_new: torch.Tensor):
        """Write S_new tokens from position seq_len (:177-214) with the scatter kernel.

        k_new, v_new: (1, Hkv, S_new, D).  Allocates pages first, like the
        reference, then one launch writes request 0's tokens from the host
        ``seq_len`` through this handle's block-table row.
        """
        ops.paged_cache_update(self, layer_idx, k_new, v_new)

    def advance_seq_len(self, n: int = 1):
        self.seq_len += n
        self._pool.seq_lens[self.row_id] = self.seq_len

    def free(self):
        if self.block_table:
            self._pool.free(self.block_table)
            self.block_table = []
            self.num_pages = 0
        self.seq_len = 0
        self._pool.free_row(self.row_id)
