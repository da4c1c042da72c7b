"""Varlen causal prefill on the GPU vs the reference's outputs and the oracle.

Tolerance (north_star): max-abs 2e-2 and mean-abs 2e-3 against fp32.
"""

import math

import numpy as np
import pytest
import torch

import golden_cases as gc
from oracle import attention as oa

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3
D = 128


def _bf16(x, device):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device).to(torch.bfloat16)


def _close(out, ref, max_abs=MAX_ABS, mean_abs=MEAN_ABS):
    o = out.float().cpu().numpy().reshape(ref.shape)
    assert np.isfinite(o).all()
    err = np.abs(o - ref)
    assert err.max() <= max_abs and err.mean() <= mean_abs, (err.max(), err.mean())


@pytest.mark.parametrize("name", gc.case_names("prefill"))
def test_packed_varlen_matches_reference_golden(name, cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    case = gc.load(name)
    m = case["meta"]
    inp = gc.prefill_inputs(case)
    lens = m["lens"]
    q = _bf16(gc.pack_varlen(inp["q"], lens), cuda)
    k = _bf16(gc.pack_varlen(inp["k"], lens), cuda)
    v = _bf16(gc.pack_varlen(inp["v"], lens), cuda)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=cuda)
    qb.clear_device_status()
    out = qb.flash_attention_prefill(q, k, v, cu, m["scaling"], m["H"], m["Hkv"], D)
    torch.cuda.synchronize()
    qb.check_device_status()
    # the fixture holds the reference output rounded to fp16
    _close(out, case["out_packed_f16"].astype(np.float32))
    # without max_seqlen the entry point reads it back like the reference does
    out2 = qb.flash_attention_prefill(q, k, v, cu, m["scaling"], m["H"], m["Hkv"], D,
                                      max_seqlen=max(lens))
    assert torch.equal(out, out2)


@pytest.mark.parametrize("name", gc.case_names("prefill"))
def test_padded_batch_adapter_matches_reference_golden(name, cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    case = gc.load(name)
    m = case["meta"]
    inp = gc.prefill_inputs(case)
    lens, B, S, H = m["lens"], len(m["lens"]), m["S"], m["H"]
    out = qb.flash_attention_prefill_batched(_bf16(inp["q"], cuda), _bf16(inp["k"], cuda),
                                             _bf16(inp["v"], cuda), lens, m["scaling"], H,
                                             m["Hkv"], D)
    torch.cuda.synchronize()
    assert out.shape == (B, S, H * D)
    o = out.view(B, S, H, D)
    packed = torch.cat([o[b, :lens[b]] for b in range(B)])
    _close(packed, case["out_packed_f16"].astype(np.float32))
    for b in range(B):
        assert not o[b, lens[b]:].any(), "padded rows must be zero"


def _rand_varlen(device, lens, H, Hkv, seed, fused=False):
    g = torch.Generator(device=device).manual_seed(seed)
    T = int(sum(lens))
    if fused:   # q/k/v as views of one fused projection output (qwen3/attention.py:82-88)
        qkv = torch.randn(T, H + 2 * Hkv, D, generator=g, device=device).to(torch.bfloat16)
        q, k, v = qkv[:, :H], qkv[:, H:H + Hkv], qkv[:, H + Hkv:]
    else:
        q = torch.randn(T, H, D, generator=g, device=device).to(torch.bfloat16)
        k = torch.randn(T, Hkv, D, generator=g, device=device).to(torch.bfloat16)
        v = torch.randn(T, Hkv, D, generator=g, device=device).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=device)
    return q, k, v, cu


def _oracle_seqs(q, k, v, lens, idx, scale):
    cu = np.concatenate([[0], np.cumsum(lens)])
    outs = []
    for i in idx:
        s0, s1 = cu[i], cu[i + 1]
        outs.append(oa.varlen_prefill(q[s0:s1].float().cpu().numpy(), k[s0:s1].float().cpu().numpy(),
                                      v[s0:s1].float().cpu().numpy(), np.array([0, s1 - s0]), scale))
    return outs


@pytest.mark.parametrize("H,Hkv", [(16, 8), (32, 8), (8, 8), (32, 4)])
def test_tile_boundaries_and_gqa(H, Hkv, cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    lens = [1, 2, 127, 128, 129, 255, 256, 300, 17]
    q, k, v, cu = _rand_varlen(cuda, lens, H, Hkv, seed=H * 10 + Hkv)
    scale = 1 / math.sqrt(D)
    qb.clear_device_status()
    out = qb.flash_attention_prefill(q, k, v, cu, scale, H, Hkv, D, max_seqlen=max(lens))
    torch.cuda.synchronize()
    qb.check_device_status()
    refs = _oracle_seqs(q, k, v, lens, range(len(lens)), scale)
    _close(out, np.concatenate(refs))


def test_config3_shape_vs_oracle(cuda, native_lib):
    """Config 3: 32 sequences, L~U[64,2048], 16/8/128; every sequence against
    the oracle, and per-sequence independence (order permutation)."""
    import qwen3_engine_from_scratch_b200 as qb
    rng = np.random.default_rng(3)
    lens = rng.integers(64, 2048, size=32, endpoint=True).tolist()
    H, Hkv = 16, 8
    q, k, v, cu = _rand_varlen(cuda, lens, H, Hkv, seed=33)
    scale = 1 / math.sqrt(D)
    out = qb.flash_attention_prefill(q, k, v, cu, scale, H, Hkv, D, max_seqlen=max(lens))
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    idx = list(range(len(lens)))
    refs = _oracle_seqs(q, k, v, lens, idx, scale)
    cun = np.concatenate([[0], np.cumsum(lens)])
    for i, ref in zip(idx, refs):
        _close(out[cun[i]:cun[i + 1]], ref)
    # reversing the sequence order permutes the output rows bit-exactly
    order = list(range(len(lens)))[::-1]
    q2 = torch.cat([q[cun[i]:cun[i + 1]] for i in order])
    k2 = torch.cat([k[cun[i]:cun[i + 1]] for i in order])
    v2 = torch.cat([v[cun[i]:cun[i + 1]] for i in order])
    lens2 = [lens[i] for i in order]
    cu2 = torch.tensor(np.concatenate([[0], np.cumsum(lens2)]), dtype=torch.int32, device=cuda)
    out2 = qb.flash_attention_prefill(q2, k2, v2, cu2, scale, H, Hkv, D, max_seqlen=max(lens))
    back = torch.cat([out2[int(np.sum(lens2[:j])):int(np.sum(lens2[:j + 1]))]
                      for j in range(len(order))][::-1])
    assert torch.equal(back, out)


def test_strided_fused_qkv_inputs(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    lens = [40, 200, 7]
    H, Hkv = 16, 8
    q, k, v, cu = _rand_varlen(cuda, lens, H, Hkv, seed=5, fused=True)
    assert not q.is_contiguous()
    scale = 1 / math.sqrt(D)
    out = qb.flash_attention_prefill(q, k, v, cu, scale, H, Hkv, D, max_seqlen=200)
    ref = qb.flash_attention_prefill(q.contiguous(), k.contiguous(), v.contiguous(), cu, scale, H,
                                     Hkv, D, max_seqlen=200)
    assert torch.equal(out, ref)
    _close(out, np.concatenate(_oracle_seqs(q, k, v, lens, range(3), scale)))


def test_batched_adapter_large_padded(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    B, H, Hkv, S = 4, 16, 8, 700
    lens = [700, 1, 333, 512]
    g = torch.Generator(device=cuda).manual_seed(8)
    qkv = torch.randn(B, S, H + 2 * Hkv, D, generator=g, device=cuda).to(torch.bfloat16)
    q = qkv[:, :, :H].transpose(1, 2)
    k = qkv[:, :, H:H + Hkv].transpose(1, 2)
    v = qkv[:, :, H + Hkv:].transpose(1, 2)
    out = qb.flash_attention_prefill_batched(q, k, v, lens, 1 / math.sqrt(D), H, Hkv, D)
    torch.cuda.synchronize()
    ref = oa.prefill_batched(q.float().cpu().numpy(), k.float().cpu().numpy(),
                             v.float().cpu().numpy(), lens, 1 / math.sqrt(D))
    _close(out, ref)
    o = out.view(B, S, H, D)
    for b in range(B):
        assert not o[b, lens[b]:].any()


def test_prefill_argument_errors(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    q = torch.zeros(8, 2, 64, dtype=torch.bfloat16, device=cuda)
    cu = torch.tensor([0, 8], dtype=torch.int32, device=cuda)
    with pytest.raises(AssertionError):          # head_dim 64 is not this kernel's shape
        qb.flash_attention_prefill(q, q, q, cu, 0.125, 2, 2, 128)
    with pytest.raises(RuntimeError):            # caught by the C ABI: head_dim != 128
        qb.flash_attention_prefill(q, q, q, cu, 0.125, 2, 2, 64)
    q16 = torch.zeros(8, 2, 128, dtype=torch.float16, device=cuda)
    with pytest.raises(AssertionError):
        qb.flash_attention_prefill(q16, q16, q16, cu, 0.1, 2, 2, 128)


def test_work_counter_reset_fixed_order_and_graph_replay(cuda, native_lib):
    """The dynamic schedule only decides which CTA computes an item, so the
    result is bit-exact against the fixed order (no counter); the counter is
    zero again after every launch, also across CUDA graph replays."""
    import qwen3_engine_from_scratch_b200 as qb
    from qwen3_engine_from_scratch_b200 import _native, ops
    lens = [2048, 1, 700, 129, 1500, 64, 300, 1000] * 3
    H, Hkv = 16, 8
    q, k, v, cu = _rand_varlen(cuda, lens, H, Hkv, seed=21)
    scale = 1 / math.sqrt(D)
    out = qb.flash_attention_prefill(q, k, v, cu, scale, H, Hkv, D, max_seqlen=max(lens))
    counter = ops._work_counter(q.device)
    torch.cuda.synchronize()
    assert counter.tolist() == [0, 0]
    fixed = torch.empty_like(out)
    lib = _native.load()
    st = lib.b200_varlen_prefill(q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0),
                                 k.stride(1), v.data_ptr(), v.stride(0), v.stride(1),
                                 fixed.data_ptr(), fixed.stride(0), fixed.stride(1), cu.data_ptr(),
                                 None, len(lens), q.shape[0], max(lens), H, Hkv, D, scale, 0, None,
                                 ops._status_ptr(q.device), ops._stream())
    _native.check(st, "b200_varlen_prefill")
    torch.cuda.synchronize()
    assert torch.equal(out, fixed)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        qb.flash_attention_prefill(q, k, v, cu, scale, H, Hkv, D, max_seqlen=max(lens))  # warm
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            o_g = qb.flash_attention_prefill(q, k, v, cu, scale, H, Hkv, D, max_seqlen=max(lens))
            o_g2 = qb.flash_attention_prefill(q, k, v, cu, scale, H, Hkv, D, max_seqlen=max(lens))
        for _ in range(3):
            o_g.zero_()
            g.replay()
        s.synchronize()
        assert ops._work_counter(q.device).tolist() == [0, 0]
    torch.cuda.current_stream().wait_stream(s)
    assert torch.equal(o_g, out) and torch.equal(o_g2, out)
