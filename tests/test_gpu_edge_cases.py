"""Edge cases of the attention path on the GPU: empty batches, zero-length
sequences, more sequences than one prefill launch takes, the longest decode
context of config 4, and decode rows with nothing cached.

Tolerance (north_star): max-abs 2e-2 and mean-abs 2e-3 against fp32; the
cases with one visible key are exact (softmax of one score is 1, so the
output is that key's value).
"""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oa

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3
D = 128


def _close(out, ref):
    o = out.float().cpu().numpy().reshape(ref.shape)
    assert np.isfinite(o).all()
    err = np.abs(o - ref)
    assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())


def _varlen(device, lens, H, Hkv, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    T = int(sum(lens))
    q = torch.randn(T, H, D, generator=g, device=device).to(torch.bfloat16)
    k = torch.randn(T, Hkv, D, generator=g, device=device).to(torch.bfloat16)
    v = torch.randn(T, Hkv, D, generator=g, device=device).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=device)
    return q, k, v, cu


def _oracle(q, k, v, s0, s1, scale):
    return oa.varlen_prefill(q[s0:s1].float().cpu().numpy(), k[s0:s1].float().cpu().numpy(),
                             v[s0:s1].float().cpu().numpy(), np.array([0, s1 - s0]), scale)


def test_prefill_zero_length_sequences(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    lens = [0, 5, 0, 130, 0, 0, 1, 257, 0]
    H, Hkv = 16, 8
    q, k, v, cu = _varlen(cuda, lens, H, Hkv, seed=5)
    scale = 1 / math.sqrt(D)
    qb.clear_device_status()
    out = qb.flash_attention_prefill(q, k, v, cu, scale, H, Hkv, D, max_seqlen=max(lens))
    torch.cuda.synchronize()
    qb.check_device_status()
    cun = np.concatenate([[0], np.cumsum(lens)])
    for i, L in enumerate(lens):
        if L:
            _close(out[cun[i]:cun[i + 1]], _oracle(q, k, v, cun[i], cun[i + 1], scale))


def test_prefill_empty_batch(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    H, Hkv = 16, 8
    for lens in ([0, 0, 0], []):
        q, k, v, cu = _varlen(cuda, lens, H, Hkv, seed=1)
        out = qb.flash_attention_prefill(q, k, v, cu, D ** -0.5, H, Hkv, D, max_seqlen=0)
        torch.cuda.synchronize()
        assert out.shape == (0, H, D)
    qb.check_device_status()


def test_prefill_more_sequences_than_one_launch(cuda, native_lib):
    """300 sequences (one launch takes 256): every sequence's rows equal the
    same sequence computed alone, bit for bit, and the oracle on a sample."""
    import qwen3_engine_from_scratch_b200 as qb
    rng = np.random.default_rng(300)
    lens = rng.integers(1, 48, size=300).tolist()
    H, Hkv = 16, 8
    q, k, v, cu = _varlen(cuda, lens, H, Hkv, seed=300)
    scale = 1 / math.sqrt(D)
    out = qb.flash_attention_prefill(q, k, v, cu, scale, H, Hkv, D, max_seqlen=max(lens))
    torch.cuda.synchronize()
    cun = np.concatenate([[0], np.cumsum(lens)])
    for i in (0, 100, 255, 256, 257, 299):
        s0, s1 = int(cun[i]), int(cun[i + 1])
        one = torch.tensor([0, s1 - s0], dtype=torch.int32, device=cuda)
        alone = qb.flash_attention_prefill(q[s0:s1], k[s0:s1], v[s0:s1], one, scale, H, Hkv, D,
                                           max_seqlen=s1 - s0)
        assert torch.equal(alone, out[s0:s1])
        _close(out[s0:s1], _oracle(q, k, v, s0, s1, scale))
    qb.check_device_status()


def _pool_with(device, lens, Hkv, seed, extra_rows=2):
    """A one-layer pool holding random K/V for requests of the given cached lengths."""
    import qwen3_engine_from_scratch_b200 as qb
    pages = sum((L + 16) // 16 for L in lens) + 4
    pool = qb.KVCachePool(pages, 1, 16, Hkv, D, device=device, dtype=torch.bfloat16,
                          max_seq_len=max(lens) + 16, max_requests=len(lens) + extra_rows)
    g = torch.Generator(device=device).manual_seed(seed)
    caches = []
    for L in lens:
        c = qb.PagedKVCache(pool)
        if L:
            k = torch.randn(1, Hkv, L, D, generator=g, device=device).to(torch.bfloat16)
            v = torch.randn(1, Hkv, L, D, generator=g, device=device).to(torch.bfloat16)
            c.update(0, k, v)
            c.advance_seq_len(L)
        caches.append(c)
    return pool, caches


def test_decode_empty_batch(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    pool, _ = _pool_with(cuda, [16], 8, seed=0)
    q = torch.empty(0, 16, D, dtype=torch.bfloat16, device=cuda)
    rows = torch.empty(0, dtype=torch.int32, device=cuda)
    out = qb.paged_decode(q, pool.k_buffer[:, 0], pool.v_buffer[:, 0], pool.block_table_2d,
                          pool.seq_lens, rows, D ** -0.5)
    torch.cuda.synchronize()
    assert out.shape == (0, 16, D)
    qb.check_device_status()


def test_decode_rows_with_nothing_cached_return_the_new_value(cuda, native_lib):
    """seq_len 0: the only visible key is the token written this step, so every
    query head returns its kv head's new value exactly."""
    import qwen3_engine_from_scratch_b200 as qb
    H, Hkv = 16, 8
    lens = [0, 37, 0, 0, 5]
    pool, caches = _pool_with(cuda, lens, Hkv, seed=9)
    g = torch.Generator(device=cuda).manual_seed(10)
    B = len(lens)
    q = torch.randn(B, H, 1, D, generator=g, device=cuda).to(torch.bfloat16)
    kn = torch.randn(B, Hkv, 1, D, generator=g, device=cuda).to(torch.bfloat16)
    vn = torch.randn(B, Hkv, 1, D, generator=g, device=cuda).to(torch.bfloat16)
    for c in caches:
        c.reserve_next()
    rows = torch.tensor([c.row_id for c in caches], dtype=torch.int32, device=cuda)
    qb.clear_device_status()
    out = qb.triton_paged_attention_decode_batch(q, kn, vn, caches, 0, D ** -0.5, rows)
    torch.cuda.synchronize()
    qb.check_device_status()
    o = out.view(B, H, D)
    for b, L in enumerate(lens):
        if L == 0:
            want = vn[b, :, 0].repeat_interleave(H // Hkv, dim=0)
            assert torch.equal(o[b], want)


@pytest.mark.parametrize("pages_per_split", [0, 16, 128])
def test_decode_longest_config4_context(pages_per_split, cuda, native_lib):
    """Config 4's longest context (32,768 cached tokens, 2,048 pages) beside a
    one-token request, Qwen3-8B heads (32/8), default and explicit splits."""
    import qwen3_engine_from_scratch_b200 as qb
    H, Hkv = 32, 8
    lens = [32768, 1, 20000]
    pool, caches = _pool_with(cuda, lens, Hkv, seed=32)
    # the request's own row: seq_lens excludes the current token, which is the last cached one
    rows = torch.tensor([c.row_id for c in caches], dtype=torch.int32, device=cuda)
    for c in caches:
        pool.seq_lens[c.row_id] = c.seq_len - 1
    g = torch.Generator(device=cuda).manual_seed(33)
    q = torch.randn(len(lens), H, D, generator=g, device=cuda).to(torch.bfloat16)
    qb.clear_device_status()
    out = qb.paged_decode(q, pool.k_buffer[:, 0], pool.v_buffer[:, 0], pool.block_table_2d,
                          pool.seq_lens, rows, D ** -0.5, pages_per_split=pages_per_split)
    torch.cuda.synchronize()
    qb.check_device_status()
    ref = oa.paged_decode(q.float().cpu().numpy(), pool.k_buffer[:, 0].float().cpu().numpy(),
                          pool.v_buffer[:, 0].float().cpu().numpy(),
                          pool.block_table_2d.cpu().numpy(), pool.seq_lens.cpu().numpy(),
                          rows.cpu().numpy(), 16, D ** -0.5)
    _close(out, ref)
