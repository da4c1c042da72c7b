"""Pin the numpy oracle against the reference's own outputs (CPU only).

The fixtures were produced by running the reference's PyTorch functions
(tests/golden/make_golden.py).  The oracle must reproduce:
  * the pool bytes written by PagedKVCache.update / the decode write, BIT-EXACT
    (row-addressed and slot_mapping-addressed scatter);
  * paged_attention's decode output (fp32, up to summation-order rounding);
  * _standard_attention's prefill output (stored as fp16);
  * RMSNorm and RoPE.
"""

import numpy as np
import pytest

import golden_cases as gc
from oracle import attention as oa
from oracle import synth

DECODE = gc.case_names("decode")
PREFILL = gc.case_names("prefill")


def test_fixtures_present():
    assert len(DECODE) >= 5 and len(PREFILL) >= 2


def test_det_normal_is_deterministic_and_normalish():
    a = synth.det_normal(7, (4096,))
    b = synth.det_normal(7, (4096,))
    assert np.array_equal(a, b)
    assert abs(float(a.mean())) < 0.05 and abs(float(a.std()) - 1.0) < 0.05
    assert not np.array_equal(a, synth.det_normal(8, (4096,)))
    p = synth.det_permutation(3, 100)
    assert sorted(p.tolist()) == list(range(100))


def test_bf16_rounding_matches_torch():
    import torch
    x = synth.det_normal(11, (10000,)) * 37.0
    x[:4] = [np.inf, -np.inf, 0.0, -0.0]
    ours = oa.bf16_bits(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, ref)


def _build_pool(case, inputs):
    """Replay the reference's write sequence with the oracle scatter."""
    m = case["meta"]
    nb, nl, Hkv, D = m["num_blocks"], m["num_layers"], m["Hkv"], m["D"]
    kp = np.zeros((nb, nl, Hkv, 16, D), np.float32)
    vp = np.zeros_like(kp)
    bt = case["block_table_2d"]
    zero_lens = np.zeros(bt.shape[0], np.int32)
    for b, (k, v) in enumerate(inputs["ctx"]):
        if k is None:
            continue
        oa.kv_scatter_rows(k, v, kp, vp, zero_lens, bt, case["row_ids"][b:b + 1], m["layer"])
    return kp, vp


@pytest.mark.parametrize("name", DECODE)
def test_oracle_decode_scatter_bitexact(name):
    case = gc.load(name)
    m = case["meta"]
    inp = gc.decode_inputs(case)
    kp, vp = _build_pool(case, inp)
    assert gc.pool_digest(kp, vp) == m["pool_digest_prefix"]
    # decode write: token at seq_lens[row] (update_kv_batch semantics)
    oa.kv_scatter_rows(inp["k_new"][:, :, None], inp["v_new"][:, :, None], kp, vp,
                       case["seq_lens"], case["block_table_2d"], case["row_ids"], m["layer"])
    assert gc.pool_digest(kp, vp) == m["pool_digest_final"]


@pytest.mark.parametrize("name", DECODE)
def test_oracle_slot_scatter_matches_reference_update(name):
    case = gc.load(name)
    m = case["meta"]
    inp = gc.decode_inputs(case)
    nb, nl, Hkv, D = m["num_blocks"], m["num_layers"], m["Hkv"], m["D"]
    kp = np.zeros((nb, nl, Hkv, 16, D), np.float32)
    vp = np.zeros_like(kp)
    bt = case["block_table_2d"]
    ks, vs, slots = [], [], []
    for b, (k, v) in enumerate(inp["ctx"]):
        if k is None:
            continue
        row = int(case["row_ids"][b])
        pos = np.arange(k.shape[2])
        slots.append(bt[row, pos // 16].astype(np.int64) * 16 + pos % 16)
        ks.append(np.transpose(k[0], (1, 0, 2)))
        vs.append(np.transpose(v[0], (1, 0, 2)))
    slots = np.concatenate(slots)
    ks, vs = np.concatenate(ks), np.concatenate(vs)
    # padding tokens (slot -1) must be skipped
    pad = np.full(3, -1, np.int64)
    oa.kv_scatter_slots(np.concatenate([ks, ks[:3] * 0 + 9.0]), np.concatenate([vs, vs[:3] * 0 + 9.0]),
                        kp, vp, np.concatenate([slots, pad]), m["layer"])
    assert gc.pool_digest(kp, vp) == m["pool_digest_prefix"]


@pytest.mark.parametrize("name", DECODE)
def test_oracle_decode_matches_reference(name):
    case = gc.load(name)
    m = case["meta"]
    inp = gc.decode_inputs(case)
    kp, vp = _build_pool(case, inp)
    oa.kv_scatter_rows(inp["k_new"][:, :, None], inp["v_new"][:, :, None], kp, vp,
                       case["seq_lens"], case["block_table_2d"], case["row_ids"], m["layer"])
    out = oa.paged_decode(inp["q"], kp[:, m["layer"]], vp[:, m["layer"]], case["block_table_2d"],
                          case["seq_lens"], case["row_ids"], 16, m["scaling"])
    err = np.abs(out - case["out"])
    assert err.max() < 2e-5, err.max()


@pytest.mark.parametrize("name", PREFILL)
def test_oracle_prefill_matches_reference(name):
    case = gc.load(name)
    m = case["meta"]
    inp = gc.prefill_inputs(case)
    lens = m["lens"]
    q = gc.pack_varlen(inp["q"], lens)
    k = gc.pack_varlen(inp["k"], lens)
    v = gc.pack_varlen(inp["v"], lens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    out = oa.varlen_prefill(q, k, v, cu, m["scaling"])
    ref = case["out_packed_f16"].astype(np.float32)
    # the fixture is stored as fp16: 2**-11 relative rounding
    assert np.abs(out - ref).max() <= 2e-3 * max(1.0, float(np.abs(ref).max()))
    # batched adapter: same rows, zeros at the padding
    ob = oa.prefill_batched(inp["q"], inp["k"], inp["v"], lens, m["scaling"])
    B, S = len(lens), m["S"]
    ob = ob.reshape(B, S, m["H"], m["D"])
    packed = np.concatenate([ob[b, :lens[b]] for b in range(B)])
    assert np.abs(packed - out).max() < 1e-5
    for b in range(B):
        assert not ob[b, lens[b]:].any()


@pytest.mark.parametrize("name", PREFILL)
def test_oracle_prefill_scatter_bitexact(name):
    """The per-request prefill page write (all S positions) of qwen3/attention.py:160-161."""
    case = gc.load(name)
    m = case["meta"]
    inp = gc.prefill_inputs(case)
    kp = np.zeros((m["num_blocks"], 1, m["Hkv"], 16, m["D"]), np.float32)
    vp = np.zeros_like(kp)
    zero = np.zeros(case["block_table_2d"].shape[0], np.int32)
    oa.kv_scatter_rows(inp["k"], inp["v"], kp, vp, zero, case["block_table_2d"], case["row_ids"], 0)
    assert gc.pool_digest(kp, vp) == m["pool_digest"]


def test_oracle_norm_rope_matches_reference():
    case = gc.load("norm_rope")
    m = case["meta"]
    q = synth.det_normal(m["seed_q"], case["q_norm"].shape)
    k = synth.det_normal(m["seed_k"], case["k_norm"].shape)
    qn, kn = oa.rms_norm(q, eps=m["eps"]), oa.rms_norm(k, eps=m["eps"])
    assert np.abs(qn - case["q_norm"]).max() < 1e-5
    assert np.abs(kn - case["k_norm"]).max() < 1e-5
    cos, sin = oa.rope_cos_sin(case["positions"], m["D"], m["theta"])
    # float32 pow differs by an ulp between numpy and torch; at angle pos*inv_freq
    # that is an absolute angle error of ~pos * 2**-22
    tol = float(case["positions"].max()) * 2.0 ** -21
    assert np.abs(cos - case["cos"]).max() < tol and np.abs(sin - case["sin"]).max() < tol
    near = case["positions"] < 200
    assert np.abs(cos - case["cos"])[near].max() < 2e-5
    qr = oa.apply_rope(case["q_norm"], case["cos"][:, None], case["sin"][:, None])
    kr = oa.apply_rope(case["k_norm"], case["cos"][:, None], case["sin"][:, None])
    assert np.abs(qr - case["q_rope"]).max() < 1e-5
    assert np.abs(kr - case["k_rope"]).max() < 1e-5


def test_oracle_norm_rope_bf16_bitexact_vs_reference():
    """bf16 QK-norm + RoPE (the serving dtype): the oracle's rounding sequence
    reproduces the reference modules bit for bit, and the stored bf16 inputs
    are the seeded values rounded once."""
    case = gc.load("norm_rope_bf16")
    m = case["meta"]
    f = oa.from_bf16_bits
    q, k = f(case["q_bits"]), f(case["k_bits"])
    assert np.array_equal(case["q_bits"],
                          oa.bf16_bits(synth.det_normal(m["seeds"][0], q.shape) * np.float32(2.0)))
    assert np.array_equal(case["k_bits"], oa.bf16_bits(synth.det_normal(m["seeds"][1], k.shape)))
    cos, sin = case["cos"][:, None], case["sin"][:, None]
    qo = oa.qk_norm_rope_bf16(q, f(case["wq_bits"]), cos, sin, m["eps"])
    ko = oa.qk_norm_rope_bf16(k, f(case["wk_bits"]), cos, sin, m["eps"])
    assert np.array_equal(oa.bf16_bits(qo), case["q_rope_bits"])
    assert np.array_equal(oa.bf16_bits(ko), case["k_rope_bits"])


def test_roofline_numerators():
    lens = np.array([128, 4096])
    b = oa.decode_bytes(lens, 16, 8)
    assert b == (128 + 4096) * 8 * 128 * 2 * 2 + 2 * 16 * 128 * 4 + (8 + 256) * 4 + 16
    assert oa.prefill_flops([1, 2], 16) == 4 * 16 * 128 * (1 + 3)


def test_oracle_paged_prefill_restates_the_reference_prefill():
    """Chunked prefill has no reference counterpart; its oracle is pinned through
    the reference-pinned varlen oracle: with no cached context it equals it, and
    a sequence prefilled in two chunks equals the rows of one full prefill."""
    case = gc.load(gc.case_names("prefill")[0])
    m = case["meta"]
    inp = gc.prefill_inputs(case)
    lens = m["lens"]
    q, k, v = (gc.pack_varlen(inp[n], lens) for n in ("q", "k", "v"))
    cu = np.concatenate([[0], np.cumsum(lens)])
    Hkv, D = m["Hkv"], 128
    nb = sum((L + 15) // 16 for L in lens) + 4
    kp = np.zeros((nb, Hkv, 16, D), np.float32)
    vp = np.zeros_like(kp)
    perm = np.random.default_rng(5).permutation(nb)
    bt = np.full((len(lens), 64), -1, np.int32)
    used = 0
    for i, L in enumerate(lens):
        npg = (L + 15) // 16
        bt[i, :npg] = perm[used:used + npg]
        used += npg
        t = np.arange(L)
        kp[bt[i, t // 16], :, t % 16] = k[cu[i] + t]
        vp[bt[i, t // 16], :, t % 16] = v[cu[i] + t]
    rows = np.arange(len(lens))
    full = oa.varlen_prefill(q, k, v, cu, m["scaling"])
    assert np.abs(oa.paged_prefill(q, kp, vp, bt, np.zeros(len(lens)), rows, cu, m["scaling"])
                  - full).max() < 1e-5
    # the longest sequence in two chunks: a third cached, the rest new
    i = int(np.argmax(lens))
    c = lens[i] // 3
    s0, s1 = cu[i] + c, cu[i + 1]
    part = oa.paged_prefill(q[s0:s1], kp, vp, bt, [c], [i], np.array([0, s1 - s0]), m["scaling"])
    assert np.abs(part - full[s0:s1]).max() < 1e-5


def test_oracle_sampling_bitexact_vs_reference_kernel():
    """Philox4x32-10 words and uniforms equal Triton's tl.randint / tl.rand, and
    the oracle's tokens equal the reference's _sample_topk_kernel on every row
    (fixture made under Triton's CPU interpreter)."""
    from oracle import sampling as osmp
    case = gc.load("sampling")
    m = case["meta"]
    for i, sd in enumerate(m["rand_seeds"]):
        n = case["rand_bits"].shape[1]
        assert np.array_equal(osmp.philox4x32_10(sd, np.arange(n))[0], case["rand_bits"][i])
        assert np.array_equal(osmp.rand_uniform(sd, np.arange(n)), case["rand_u"][i])
    logits = synth.det_normal(m["seed_logits"], (m["B"], m["V"])) * np.float32(m["scale"])
    tok = osmp.sample_tokens(logits, m["temperature"], m["top_k"], m["top_p"], m["seed"],
                             m["block_k"])
    assert np.array_equal(tok, case["tokens"])
