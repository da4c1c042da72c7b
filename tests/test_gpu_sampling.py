"""Fused sampling on the GPU vs tokens of the reference's own kernel
(tests/golden/sampling.npz), the oracle, and exact distributions.

Token ids are discrete: the fixture and oracle comparisons are exact per row;
the distribution tests bound the total-variation distance between empirical
frequencies and the exact truncated softmax (the bound is several standard
errors of the sample size).
"""

import json

import numpy as np
import pytest
import torch

import golden_cases as gc
from oracle import sampling as osmp
from oracle import synth

pytestmark = pytest.mark.gpu


def test_reference_tokens_from_fixture(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    case = gc.load("sampling")
    m = case["meta"]
    logits = synth.det_normal(m["seed_logits"], (m["B"], m["V"])) * np.float32(m["scale"])
    out = qb.sample_tokens(torch.from_numpy(logits).to(cuda), m["temperature"], m["top_k"],
                           m["top_p"], seed=m["seed"])
    torch.cuda.synchronize()
    assert out.shape == (m["B"], 1)
    assert np.array_equal(out[:, 0].cpu().numpy(), case["tokens"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_greedy_and_top1_are_argmax_full_vocab(dtype, cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    g = torch.Generator(device=cuda).manual_seed(5)
    logits = (torch.randn(64, 151936, generator=g, device=cuda) * 4).to(dtype)
    # bf16 logits hold many exact ties: the first index of the maximum wins
    want = logits.float().argmax(dim=-1)
    greedy = qb.sample_tokens(logits, 0.0)
    top1 = qb.sample_tokens(logits, 0.8, top_k=1, top_p=0.5)
    torch.cuda.synchronize()
    assert torch.equal(greedy[:, 0], want) and torch.equal(top1[:, 0], want)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_full_vocab_topk_topp_vs_oracle(dtype, cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    g = torch.Generator(device=cuda).manual_seed(6)
    B, V = 12, 151936
    logits = (torch.randn(B, V, generator=g, device=cuda) * 3).to(dtype)
    temps = [0.7, 1.0, 1.5, 0.3] * 3
    ks = [1, 20, 50, 1024, 200, 7, 999, 64, 3, 512, 1000, 16]
    ps = [0.9, 1.0, 0.8, 0.95, 0.5, 1.0, 0.99, 0.7, 1.0, 0.9, 0.6, 0.85]
    out = qb.sample_tokens(logits, temps, ks, ps, seed=4242)
    torch.cuda.synchronize()
    want = osmp.sample_tokens(logits.float().cpu().numpy(), temps, ks, ps, 4242)
    assert np.array_equal(out[:, 0].cpu().numpy(), want)


def test_ties_at_the_topk_threshold(cuda, native_lib):
    """Coarsely quantised logits: the k-th value is shared by many entries and
    the lowest indices are kept (as a stable sort keeps them)."""
    import qwen3_engine_from_scratch_b200 as qb
    g = torch.Generator(device=cuda).manual_seed(8)
    logits = torch.round(torch.randn(16, 5000, generator=g, device=cuda) * 2) / 2
    ks = [10, 33, 100, 250] * 4
    out = qb.sample_tokens(logits, 1.0, ks, 1.0, seed=77)
    torch.cuda.synchronize()
    want = osmp.sample_tokens(logits.cpu().numpy(), 1.0, ks, 1.0, 77)
    assert np.array_equal(out[:, 0].cpu().numpy(), want)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_small_k_batch_vs_oracle(dtype, cuda, native_lib):
    """Every k <= 64: the chunks take the bound-and-rank selection and the rows
    the one-warp kernel; tokens equal the oracle's (Qwen3 vocabulary)."""
    import qwen3_engine_from_scratch_b200 as qb
    g = torch.Generator(device=cuda).manual_seed(16)
    B, V = 64, 151936
    logits = (torch.randn(B, V, generator=g, device=cuda) * 3).to(dtype)
    temps = [0.7, 1.0, 1.5, 0.3, 0.0, 1.2, 0.9, 0.5] * 8
    ks = [50, 1, 20, 64, 7, 33, 2, 16] * 8
    ps = [0.9, 1.0, 0.8, 0.95, 0.5, 1.0, 0.99, 0.7] * 8
    out = qb.sample_tokens(logits, temps, ks, ps, seed=99)
    torch.cuda.synchronize()
    want = osmp.sample_tokens(logits.float().cpu().numpy(), temps, ks, ps, 99)
    assert np.array_equal(out[:, 0].cpu().numpy(), want)


def test_small_k_ties_vs_oracle(cuda, native_lib):
    """Coarsely quantised logits with k <= 64: the threads' maxima tie at the
    bound, so some chunks fall back to the bit-by-bit search; the lowest
    indices are kept at the threshold."""
    import qwen3_engine_from_scratch_b200 as qb
    g = torch.Generator(device=cuda).manual_seed(17)
    logits = torch.round(torch.randn(16, 40000, generator=g, device=cuda) * 2) / 2
    ks = [10, 33, 64, 5] * 4
    out = qb.sample_tokens(logits, 1.0, ks, 1.0, seed=78)
    torch.cuda.synchronize()
    want = osmp.sample_tokens(logits.cpu().numpy(), 1.0, ks, 1.0, 78)
    assert np.array_equal(out[:, 0].cpu().numpy(), want)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_ragged_last_chunk_ties_vs_oracle(dtype, cuda, native_lib):
    """Vocabularies whose last 8192-logit chunk is short, with heavily tied
    logits and k <= 64: the row kernel's samples then include empty slots of
    the short chunk (the bound must fall back to taking every candidate), and
    the full chunks' tied bounds take the block-wide search.  Several seeds
    and rows, every token equal to the oracle's."""
    import qwen3_engine_from_scratch_b200 as qb
    g = torch.Generator(device=cuda).manual_seed(21)
    for V in (2 * 8192 + 16, 8192 + 16, 3 * 8192 + 300):
        logits = torch.randint(0, 7, (64, V), generator=g, device=cuda).float().to(dtype)
        lf = logits.float().cpu().numpy()
        for k, t, p, seed in ((64, 0.7, 0.9, 1), (64, 1.0, 1.0, 3), (50, 0.7, 0.9, 2),
                              (33, 1.0, 1.0, 4)):
            out = qb.sample_tokens(logits, t, k, p, seed=seed)
            torch.cuda.synchronize()
            want = osmp.sample_tokens(lf, t, k, p, seed)
            got = out[:, 0].cpu().numpy()
            assert np.array_equal(got, want), (V, k, seed, np.nonzero(got != want)[0][:8])


def _tv(counts, probs):
    return 0.5 * np.abs(counts / counts.sum() - probs).sum()


def test_topk_topp_distribution(cuda, native_lib):
    """Many rows with the same logits (each row draws its own uniforms): the
    empirical distribution matches the truncated, renormalised softmax."""
    import qwen3_engine_from_scratch_b200 as qb
    rng = np.random.default_rng(9)
    V, N, T, K, P = 300, 20000, 0.8, 40, 0.9
    row = (rng.standard_normal(V) * 1.5).astype(np.float32)
    logits = torch.from_numpy(np.tile(row, (N, 1))).to(cuda)
    out = qb.sample_tokens(logits, T, K, P, seed=123)[:, 0].cpu().numpy()
    order = np.argsort(-row, kind="stable")[:K]
    x = row[order] / T
    p = np.exp(x - x.max())
    p /= p.sum()
    keep = np.concatenate([[True], np.cumsum(p)[:-1] <= P])
    q = np.where(keep, p, 0)
    q /= q.sum()
    probs = np.zeros(V)
    probs[order] = q
    assert set(np.unique(out)) <= set(order[keep])
    assert _tv(np.bincount(out, minlength=V).astype(float), probs) < 0.03


def test_temperature_only_distribution(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    rng = np.random.default_rng(10)
    V, N, T = 200, 20000, 1.3
    row = (rng.standard_normal(V) * 2).astype(np.float32)
    logits = torch.from_numpy(np.tile(row, (N, 1))).to(cuda).to(torch.bfloat16)
    out = qb.sample_tokens(logits, T, 0, 1.0, seed=321)[:, 0].cpu().numpy()
    x = logits[0].float().cpu().numpy() / T
    probs = np.exp(x - x.max())
    probs /= probs.sum()
    assert _tv(np.bincount(out, minlength=V).astype(float), probs) < 0.03


def test_unsupported_parameters_raise(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    logits = torch.zeros(2, 10, device=cuda)
    with pytest.raises(ValueError):
        qb.sample_tokens(logits, 1.0, 0, 0.9)
    with pytest.raises(ValueError):
        qb.sample_tokens(logits, 1.0, 2000, 1.0)
