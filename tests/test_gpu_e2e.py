"""End-to-end decode of a small Qwen3-shaped model through this package's kernels.

The config-5 harness (``e2e_model``) serves its decode steps from CUDA graphs
(``GraphRunner``), as the reference's engine does.  Greedy decoding must give
the same tokens whether the steps are replayed from the graphs or issued
eagerly, and the model's prefill (packed varlen kernel + slot scatter) must
leave the pool in the state a decode step expects: the first decode step's
logits equal those of a torch attention over the same K/V (fp32 softmax,
tolerance of the attention tests: max-abs 2e-2 on the attention output feeds
the logits through o_proj, so the check is on tokens).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _small(device):
    from qwen3_engine_from_scratch_b200 import e2e_model
    return e2e_model.Qwen3DecodeModel(device, layers=2, hidden=512, heads=16, kv_heads=8,
                                      head_dim=128, intermediate=1024, vocab=4096, seed=3,
                                      max_pos=1024)


def test_graph_replay_tokens_equal_eager(cuda, native_lib):
    from qwen3_engine_from_scratch_b200 import e2e_model
    model = _small(cuda)
    prompts = e2e_model.synthetic_prompts(12, 5, 150, 4096, seed=9)
    eager, st_e = e2e_model.serve(model, prompts, 8, cuda, graph=False)
    graphed, st_g = e2e_model.serve(model, prompts, 8, cuda, graph=True, buckets=(4, 16))
    assert eager.shape == (12, 8)
    assert torch.equal(eager, graphed)
    assert st_g["decode_steps"] == 7


def test_prefill_then_decode_matches_torch_attention(cuda, native_lib):
    """The first generated token of each request from a torch re-computation of
    the prompt (fp32 causal attention on the model's own q/k/v) equals the
    harness's (bf16 kernels)."""
    from qwen3_engine_from_scratch_b200 import e2e_model, ops
    model = _small(cuda)
    prompts = e2e_model.synthetic_prompts(6, 20, 90, 4096, seed=4)
    toks, _ = e2e_model.serve(model, prompts, 1, cuda, graph=False)
    H, Hkv, D = model.H, model.Hkv, model.D
    for b, p in enumerate(prompts):
        T = len(p)
        ids = torch.from_numpy(np.asarray(p, np.int64)).to(cuda)
        pos = torch.arange(T, device=cuda)
        cos, sin = model.cos_t[pos][None], model.sin_t[pos][None]
        h = model.embed[ids][None]
        for i in range(model.layers):
            qkv = model._rms(h, model.ln1[i]) @ model.wqkv[i]
            q = qkv[..., :H * D].view(1, T, H, D).transpose(1, 2)
            k = qkv[..., H * D:(H + Hkv) * D].view(1, T, Hkv, D).transpose(1, 2)
            v = qkv[..., (H + Hkv) * D:].view(1, T, Hkv, D).transpose(1, 2)
            q, k = ops.qk_norm_rope_kv_write(q, k, v, model.qn[i], model.kn[i], cos, sin,
                                             return_k=True)
            kf = k.float().repeat_interleave(H // Hkv, dim=1)
            vf = v.float().repeat_interleave(H // Hkv, dim=1)
            s = (q.float() @ kf.transpose(-1, -2)) * model.scale
            s = s + torch.triu(torch.full((T, T), float("-inf"), device=cuda), 1)
            o = (torch.softmax(s, -1) @ vf).to(torch.bfloat16)          # (1, H, T, D)
            h = h + o.transpose(1, 2).reshape(1, T, H * D) @ model.wo[i]
            h = model._mlp(i, h)
        logits = model.logits(h[:, -1]).float()
        top2 = torch.topk(logits[0], 2).values
        if (top2[0] - top2[1]).item() > 0.05:     # a clear winner: the kernels must agree
            assert int(torch.argmax(logits[0])) == int(toks[b, 0])
