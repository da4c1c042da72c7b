"""Chunked prefill over the paged KV cache on the GPU vs the oracle, and
against the varlen prefill / paged decode kernels it generalises.

Tolerance (north_star): max-abs 2e-2 and mean-abs 2e-3 against fp32.
"""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oa

pytestmark = pytest.mark.gpu

D = 128
MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _close(out, ref):
    o = out.float().cpu().numpy().reshape(ref.shape)
    assert np.isfinite(o).all()
    err = np.abs(o - ref)
    assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())


def _setup(device, ctx, new, H, Hkv, seed):
    """A pool holding every sequence's cached context and its new tokens, pages
    placed by a random permutation; q for the new tokens (packed)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    n = len(ctx)
    totals = [c + m for c, m in zip(ctx, new)]
    max_pages = max((t + 15) // 16 for t in totals) + 2
    nb = sum((t + 15) // 16 for t in totals) + 8
    kp = torch.zeros(nb, 2, Hkv, 16, D, dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    perm = torch.randperm(nb, generator=g)
    rows = torch.randperm(n + 3, generator=g)[:n].to(torch.int32)
    bt = torch.full((n + 3, max_pages), -1, dtype=torch.int32)
    seq = torch.zeros(n + 3, dtype=torch.int32)
    used = 0
    layer = 1
    for i in range(n):
        npg = (totals[i] + 15) // 16
        bt[rows[i], :npg] = perm[used:used + npg].to(torch.int32)
        used += npg
        kk = torch.randn(totals[i], Hkv, D, generator=g).to(torch.bfloat16)
        vv = torch.randn(totals[i], Hkv, D, generator=g).to(torch.bfloat16)
        t = torch.arange(totals[i])
        pg = bt[rows[i]][t // 16].long()
        kp[pg, layer, :, t % 16] = kk
        vp[pg, layer, :, t % 16] = vv
        seq[rows[i]] = ctx[i]
    q = torch.randn(sum(new), H, D, generator=g).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(new)]), dtype=torch.int32)
    dev = lambda x: x.to(device)
    return dict(q=dev(q), kp=dev(kp), vp=dev(vp), bt=dev(bt), seq=dev(seq), rows=dev(rows),
                cu=dev(cu), layer=layer, ctx=ctx, new=new)


def _oracle(c, scale):
    L = c["layer"]
    return oa.paged_prefill(c["q"].float().cpu().numpy(), c["kp"][:, L].float().cpu().numpy(),
                            c["vp"][:, L].float().cpu().numpy(), c["bt"].cpu().numpy(), c["ctx"],
                            c["rows"].cpu().numpy(), c["cu"].cpu().numpy(), scale)


def _run(qb, c, scale, max_new=None):
    L = c["layer"]
    return qb.paged_prefill(c["q"], c["kp"][:, L], c["vp"][:, L], c["bt"], c["seq"], c["rows"],
                            c["cu"], scale, max_new_tokens=max_new or max(c["new"]))


@pytest.mark.parametrize("H,Hkv", [(16, 8), (8, 8), (32, 4), (40, 8)])
def test_context_and_chunk_boundaries_vs_oracle(H, Hkv, cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    ctx = [0, 1, 15, 16, 100, 300, 1000, 129]
    new = [7, 1, 128, 129, 300, 5, 130, 256]
    c = _setup(cuda, ctx, new, H, Hkv, seed=H + 7 * Hkv)
    scale = 1 / math.sqrt(D)
    qb.clear_device_status()
    out = _run(qb, c, scale)
    torch.cuda.synchronize()
    qb.check_device_status()
    _close(out, _oracle(c, scale))


def test_bench_chunk_shape_vs_oracle(cuda, native_lib):
    """The bench's chunk case: 32 sequences with U[0, 2048] cached tokens and a
    new chunk of U[64, 512] each (16/8 heads), every sequence against the oracle."""
    import qwen3_engine_from_scratch_b200 as qb
    rng = np.random.default_rng(5000)
    ctx = rng.integers(0, 2048, size=32, endpoint=True).tolist()
    new = rng.integers(64, 512, size=32, endpoint=True).tolist()
    c = _setup(cuda, ctx, new, 16, 8, seed=501)
    scale = 1 / math.sqrt(D)
    qb.clear_device_status()
    out = _run(qb, c, scale)
    torch.cuda.synchronize()
    qb.check_device_status()
    _close(out, _oracle(c, scale))


def test_no_context_equals_varlen_prefill_bitexact(cuda, native_lib):
    """With nothing cached, the paged kernel reads the same K/V values the packed
    kernel reads, in the same tiles: outputs are bit-identical."""
    import qwen3_engine_from_scratch_b200 as qb
    new = [1, 2, 127, 128, 129, 300, 17]
    c = _setup(cuda, [0] * len(new), new, 16, 8, seed=3)
    L = c["layer"]
    # the same K/V, packed
    k = torch.cat([c["kp"][c["bt"][r][torch.arange(m, device=cuda) // 16].long(), L, :,
                          torch.arange(m, device=cuda) % 16] for r, m in zip(c["rows"].tolist(), new)])
    v = torch.cat([c["vp"][c["bt"][r][torch.arange(m, device=cuda) // 16].long(), L, :,
                          torch.arange(m, device=cuda) % 16] for r, m in zip(c["rows"].tolist(), new)])
    scale = 1 / math.sqrt(D)
    paged = _run(qb, c, scale)
    packed = qb.flash_attention_prefill(c["q"], k, v, c["cu"], scale, 16, 8, D, max_seqlen=max(new))
    torch.cuda.synchronize()
    assert torch.equal(paged, packed)


def test_single_new_token_matches_paged_decode(cuda, native_lib):
    """len 1 per sequence is a decode step: same result as the split-K decode kernel
    within the tolerance (different reduction orders)."""
    import qwen3_engine_from_scratch_b200 as qb
    ctx = [0, 15, 16, 200, 777, 2047]
    c = _setup(cuda, ctx, [1] * len(ctx), 16, 8, seed=11)
    L = c["layer"]
    scale = 1 / math.sqrt(D)
    pre = _run(qb, c, scale)
    dec = qb.paged_decode(c["q"], c["kp"][:, L], c["vp"][:, L], c["bt"], c["seq"], c["rows"], scale)
    torch.cuda.synchronize()
    err = (pre.float() - dec.float()).abs()
    assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS
    _close(pre, _oracle(c, scale))


def test_two_chunks_equal_one_prefill(cuda, native_lib):
    """A prompt prefilled in two chunks (the second with the first cached) gives
    the same rows as one prefill of the whole prompt."""
    import qwen3_engine_from_scratch_b200 as qb
    total, first = 900, 333
    c = _setup(cuda, [0], [total], 16, 8, seed=21)
    scale = 1 / math.sqrt(D)
    whole = _run(qb, c, scale)
    seq = c["seq"].clone()
    seq[c["rows"][0]] = first
    L = c["layer"]
    cu2 = torch.tensor([0, total - first], dtype=torch.int32, device=cuda)
    second = qb.paged_prefill(c["q"][first:], c["kp"][:, L], c["vp"][:, L], c["bt"], seq, c["rows"],
                              cu2, scale, max_new_tokens=total - first)
    torch.cuda.synchronize()
    err = (second.float() - whole[first:].float()).abs()
    assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS


def test_bad_row_flagged(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    c = _setup(cuda, [5, 40], [10, 20], 16, 8, seed=4)
    rows = c["rows"].clone()
    rows[1] = 9999
    L = c["layer"]
    qb.clear_device_status()
    qb.paged_prefill(c["q"], c["kp"][:, L], c["vp"][:, L], c["bt"], c["seq"], rows, c["cu"],
                     0.1, max_new_tokens=20)
    torch.cuda.synchronize()
    assert qb.device_status() & qb._native.DEV_BAD_ROW
    qb.clear_device_status()
