"""Qwen3-shaped model and serving loop for the end-to-end benchmark (config 5).

Config 5 measures whole-engine decode throughput with this package's kernels
swapped in: Qwen3-0.6B (28 layers, hidden 1024, 16 query / 8 kv heads of 128,
SwiGLU 3072, vocab 151,936, bf16) with seeded N(0, 0.02) weights, 256
concurrent requests with prompts of U[32, 1024] tokens and 256 generated
tokens each, decode replayed from CUDA graphs.  The reference serves this with
its Scheduler, model.forward (prefill) and GraphRunner (decode)
(bench_batched.py:150-200, qwen3/model.py:186-251, qwen3/graph_runner.py).

The GEMMs, embedding, RMSNorms and the MLP are plain torch (cuBLAS): they are
outside the attention hot path.  The attention path is this package's:

* prefill (packed tokens of all requests): ``qk_norm_rope_kv_write`` (QK norm
  + RoPE), ``kv_scatter_slots`` (the prompt's K/V into the paged pool) and
  ``flash_attention_prefill`` (varlen causal prefill);
* decode (``forward_decode``, the contract of qwen3/model.py:240-251 that
  ``GraphRunner`` captures): ``qk_norm_rope_kv_write`` and
  ``triton_paged_attention_decode_batch`` (KV write + split-K decode, one
  launch);
* sampling: ``sample_tokens`` (greedy here).

As in the reference's scheduler (qwen3/scheduler.py:59-89), with room for all
requests the first step prefills every prompt and every later step decodes
the whole running batch; no request finishes early (no EOS), so the batch
stays full until the last step.
"""

from __future__ import annotations

import time

import numpy as np
import torch

from . import ops
from .graph_runner import GraphRunner
from .paged_kv import KVCachePool, PagedKVCache

QWEN3_0_6B = dict(layers=28, hidden=1024, heads=16, kv_heads=8, head_dim=128,
                  intermediate=3072, vocab=151936, rope_theta=1e6, eps=1e-6)


class Qwen3DecodeModel:
    """Random-init Qwen3 decoder (seeded N(0, std) linear and embedding weights,
    unit RMSNorm weights, tied lm_head as in Qwen3-0.6B)."""

    def __init__(self, device, layers=28, hidden=1024, heads=16, kv_heads=8, head_dim=128,
                 intermediate=3072, vocab=151936, rope_theta=1e6, eps=1e-6, max_pos=4096,
                 seed=0, std=0.02):
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16

        def w(*shape):
            return (torch.randn(*shape, generator=g, device=device) * std).to(bf)

        self.layers, self.hidden, self.H, self.Hkv, self.D = layers, hidden, heads, kv_heads, head_dim
        self.inter, self.vocab, self.eps = intermediate, vocab, eps
        self.embed = w(vocab, hidden)                                  # tied with lm_head
        self.wqkv = [w(hidden, (heads + 2 * kv_heads) * head_dim) for _ in range(layers)]
        self.wo = [w(heads * head_dim, hidden) for _ in range(layers)]
        self.wgu = [w(hidden, 2 * intermediate) for _ in range(layers)]  # gate | up
        self.wd = [w(intermediate, hidden) for _ in range(layers)]
        ones = torch.ones(hidden, dtype=bf, device=device)
        self.ln1 = [ones] * layers
        self.ln2 = [ones] * layers
        self.ln_f = ones
        self.qn = [torch.ones(head_dim, dtype=bf, device=device)] * layers
        self.kn = [torch.ones(head_dim, dtype=bf, device=device)] * layers
        inv = 1.0 / (rope_theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32,
                                                 device=device) / head_dim))
        f = torch.outer(torch.arange(max_pos, dtype=torch.float32, device=device), inv)
        emb = torch.cat([f, f], dim=-1)
        self.cos_t, self.sin_t = emb.cos(), emb.sin()                 # fp32 rows, as the reference
        self.scale = head_dim ** -0.5

    def _rms(self, x, w):
        xf = x.float()
        return ((xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)) * w).to(x.dtype)

    def _mlp(self, i, h):
        gu = self._rms(h, self.ln2[i]) @ self.wgu[i]
        gate, up = gu[..., :self.inter], gu[..., self.inter:]
        return h + (torch.nn.functional.silu(gate) * up) @ self.wd[i]

    def logits(self, h):
        return self._rms(h, self.ln_f) @ self.embed.t()

    @torch.no_grad()
    def forward_prefill(self, tokens, cu_seqlens, max_len, positions, slots, pool):
        """All prompts as packed tokens: (T,) ids, int32 cu_seqlens, (T,) positions
        and (T,) int64 pool slots.  Writes every layer's K/V into ``pool`` and
        returns the final hidden state of each sequence's last token."""
        H, Hkv, D = self.H, self.Hkv, self.D
        T = tokens.shape[0]
        cos = self.cos_t[positions][None]          # (1, T, D)
        sin = self.sin_t[positions][None]
        h = self.embed[tokens][None]               # (1, T, hidden)
        for i in range(self.layers):
            qkv = self._rms(h, self.ln1[i]) @ self.wqkv[i]
            q = qkv[..., :H * D].view(1, T, H, D).transpose(1, 2)
            k = qkv[..., H * D:(H + Hkv) * D].view(1, T, Hkv, D).transpose(1, 2)
            v = qkv[..., (H + Hkv) * D:].view(1, T, Hkv, D).transpose(1, 2)
            q, k = ops.qk_norm_rope_kv_write(q, k, v, self.qn[i], self.kn[i], cos, sin,
                                             eps=self.eps, return_k=True)
            k_t, v_t = k[0].transpose(0, 1), v[0].transpose(0, 1)   # (T, Hkv, D) views
            ops.kv_scatter_slots(k_t, v_t, pool.k_buffer, pool.v_buffer, slots, i)
            o = ops.flash_attention_prefill(q[0].transpose(0, 1), k_t, v_t, cu_seqlens,
                                            self.scale, H, Hkv, D, max_seqlen=max_len)
            h = h + o.reshape(1, T, H * D) @ self.wo[i]
            h = self._mlp(i, h)
        return h[0, cu_seqlens[1:].long() - 1]     # (B, hidden)

    @torch.no_grad()
    def forward_decode(self, input_ids, position_ids, row_ids, caches):
        """One decode step (qwen3/model.py:240-251 contract): (B, 1) ids and
        positions, (B,) int32 rows -> (B, 1, vocab) logits.  Capture-safe."""
        B = input_ids.shape[0]
        H, Hkv, D = self.H, self.Hkv, self.D
        cos = self.cos_t[position_ids]             # (B, 1, D)
        sin = self.sin_t[position_ids]
        h = self.embed[input_ids]                  # (B, 1, hidden)
        for i in range(self.layers):
            qkv = self._rms(h, self.ln1[i]) @ self.wqkv[i]
            q = qkv[..., :H * D].view(B, 1, H, D).transpose(1, 2)
            k = qkv[..., H * D:(H + Hkv) * D].view(B, 1, Hkv, D).transpose(1, 2)
            v = qkv[..., (H + Hkv) * D:].view(B, 1, Hkv, D).transpose(1, 2)
            q, k = ops.qk_norm_rope_kv_write(q, k, v, self.qn[i], self.kn[i], cos, sin,
                                             eps=self.eps, return_k=True)
            o = ops.triton_paged_attention_decode_batch(q, k, v, caches, i, self.scale, row_ids)
            h = h + o @ self.wo[i]
            h = self._mlp(i, h)
        return self.logits(h)


def synthetic_prompts(n, lo, hi, vocab, seed):
    """``n`` prompt lengths U[lo, hi] and token ids U[0, vocab) (seeded)."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi, size=n, endpoint=True)
    return [rng.integers(0, vocab, size=int(L)) for L in lens]


def serve(model, prompts, new_tokens, device, graph=True, buckets=None, pool_blocks=None,
          timers=None):
    """Prefill every prompt, then decode ``new_tokens - 1`` steps of the whole
    batch (the prefill produces the first token).  Returns (tokens (B, new_tokens)
    int64 on the host, stats).  Greedy sampling."""
    B = len(prompts)
    lens = np.array([len(p) for p in prompts], dtype=np.int64)
    max_total = int(lens.max()) + new_tokens
    pages = int(((lens + new_tokens + 15) // 16).sum())
    buckets = tuple(buckets) if buckets is not None else (B,)
    nb = pool_blocks or pages + max(buckets) + 16
    pool = KVCachePool(nb, model.layers, 16, model.Hkv, model.D, device=device,
                       dtype=torch.bfloat16, max_seq_len=max_total,
                       max_requests=B + max(buckets) + 2)
    caches = [PagedKVCache(pool) for _ in range(B)]
    for c, L in zip(caches, lens):
        c._ensure_pages(int(L))
    slots = np.concatenate([np.asarray(c.block_table, np.int64)[np.arange(L) // 16] * 16
                            + np.arange(L) % 16 for c, L in zip(caches, lens)])
    positions = np.concatenate([np.arange(L) for L in lens])
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tok = torch.from_numpy(np.concatenate(prompts).astype(np.int64)).to(device)
    d_slots = torch.from_numpy(slots).to(device)
    d_pos = torch.from_numpy(positions).to(device)
    d_cu = torch.from_numpy(cu).to(device)
    rows = torch.tensor([c.row_id for c in caches], dtype=torch.int32, device=device)

    runner = None
    if graph:
        holders = [PagedKVCache(pool) for _ in range(max(buckets))]
        runner = GraphRunner(model, pool, holders, buckets=buckets)
    out = torch.empty((B, new_tokens), dtype=torch.int64, device=device)

    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    t0 = time.perf_counter()
    ev[0].record()
    last_h = model.forward_prefill(tok, d_cu, int(lens.max()), d_pos, d_slots, pool)
    for c, L in zip(caches, lens):
        c.advance_seq_len(int(L))
    nxt = ops.sample_tokens(model.logits(last_h), 0.0)             # (B, 1) greedy
    out[:, 0] = nxt[:, 0]
    ev[1].record()
    pos = torch.from_numpy(lens).to(device)[:, None]               # position of the next token
    for step in range(1, new_tokens):
        for c in caches:
            c.reserve_next()
        if runner is not None:
            logits = runner.replay(nxt, pos, rows)[:B]
        else:
            logits = model.forward_decode(nxt, pos, rows, caches)
        for c in caches:
            c.advance_seq_len(1)
        nxt = ops.sample_tokens(logits[:, 0], 0.0)
        out[:, step] = nxt[:, 0]
        pos = pos + 1
    ev[2].record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    prefill_ms = ev[0].elapsed_time(ev[1])
    decode_ms = ev[1].elapsed_time(ev[2])
    stats = {"requests": B, "prompt_tokens": int(lens.sum()), "new_tokens_per_request": new_tokens,
             "prefill_ms": prefill_ms, "decode_ms": decode_ms, "wall_s": wall,
             "decode_steps": new_tokens - 1, "pool_blocks": nb}
    if runner is not None:
        runner.free()
    del pool
    return out.cpu(), stats
