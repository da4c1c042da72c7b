"""A small Qwen3-shaped decode model for the graph-runner tests.

Random bf16 weights; per layer: RMSNorm, fused qkv projection, the fused
QK-RMSNorm + RoPE (``ops.qk_norm_rope_kv_write``), the reference's batched
decode entry (``triton_paged_attention_decode_batch``: KV write + paged
decode) and o_proj with a residual; a final RMSNorm and lm_head.  It has the
``forward_decode(input_ids, position_ids, row_ids, caches)`` contract of
qwen3/model.py:240-251, which is all ``GraphRunner`` needs.
"""

from __future__ import annotations

import torch

from qwen3_engine_from_scratch_b200 import ops


class TinyDecodeModel:
    def __init__(self, device, layers=2, vocab=1024, hidden=512, heads=16, kv_heads=8,
                 head_dim=128, max_pos=8192, seed=0):
        g = torch.Generator().manual_seed(seed)
        bf = torch.bfloat16

        def w(*shape, s=0.02):
            return (torch.randn(*shape, generator=g) * s).to(bf).to(device)

        self.layers, self.H, self.Hkv, self.D = layers, heads, kv_heads, head_dim
        self.embed = w(vocab, hidden, s=1.0)
        self.wqkv = [w(hidden, (heads + 2 * kv_heads) * head_dim) for _ in range(layers)]
        self.wo = [w(heads * head_dim, hidden) for _ in range(layers)]
        self.qn = [(1 + 0.1 * torch.randn(head_dim, generator=g)).to(bf).to(device)
                   for _ in range(layers)]
        self.kn = [(1 + 0.1 * torch.randn(head_dim, generator=g)).to(bf).to(device)
                   for _ in range(layers)]
        self.lm = w(hidden, vocab)
        inv = 1.0 / (1e6 ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        f = torch.outer(torch.arange(max_pos, dtype=torch.float32), inv)
        emb = torch.cat([f, f], dim=-1)
        self.cos_t = emb.cos().to(device)
        self.sin_t = emb.sin().to(device)
        self.scale = head_dim ** -0.5

    @staticmethod
    def _rms(x, eps=1e-6):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)

    def forward_decode(self, input_ids, position_ids, row_ids, caches):
        B = input_ids.shape[0]
        H, Hkv, D = self.H, self.Hkv, self.D
        cos = self.cos_t[position_ids]              # (B, 1, D)
        sin = self.sin_t[position_ids]
        h = self.embed[input_ids]                   # (B, 1, hidden)
        for i in range(self.layers):
            qkv = self._rms(h) @ self.wqkv[i]
            q = qkv[..., :H * D].view(B, 1, H, D).transpose(1, 2)
            k = qkv[..., H * D:(H + Hkv) * D].view(B, 1, Hkv, D).transpose(1, 2)
            v = qkv[..., (H + Hkv) * D:].view(B, 1, Hkv, D).transpose(1, 2)
            q, k = ops.qk_norm_rope_kv_write(q, k, v, self.qn[i], self.kn[i], cos, sin,
                                             return_k=True)
            o = ops.triton_paged_attention_decode_batch(q, k, v, caches, i, self.scale, row_ids)
            h = h + o @ self.wo[i]
        return self._rms(h) @ self.lm               # (B, 1, vocab)
