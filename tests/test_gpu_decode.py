"""Paged decode attention on the GPU vs the reference's outputs and the oracle.

Tolerance (north_star): max-abs 2e-2 and mean-abs 2e-3 against fp32.
"""

import math

import numpy as np
import pytest
import torch

import golden_cases as gc
from oracle import attention as oa
from oracle import synth

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _bf16(x, device):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device).to(torch.bfloat16)


def _close(out: torch.Tensor, ref: np.ndarray):
    o = out.float().cpu().numpy().reshape(ref.shape)
    assert np.isfinite(o).all()
    err = np.abs(o - ref)
    assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())
    return err


def _golden_setup(name, device):
    import qwen3_engine_from_scratch_b200 as qb
    case = gc.load(name)
    m = case["meta"]
    inp = gc.decode_inputs(case)
    pool = qb.KVCachePool(m["num_blocks"], m["num_layers"], 16, m["Hkv"], m["D"], device=device,
                          dtype=torch.bfloat16, max_seq_len=m["max_seq_len"],
                          max_requests=m["max_requests"])
    pool.free_block_ids = [int(x) for x in synth.det_permutation(m["seed"] + 1, m["num_blocks"])]
    caches = []
    for k, v in inp["ctx"]:
        c = qb.PagedKVCache(pool)
        if k is not None:
            c.update(m["layer"], _bf16(k, device), _bf16(v, device))
            c.advance_seq_len(k.shape[2])
        caches.append(c)
    return case, m, inp, pool, caches


@pytest.mark.parametrize("name", gc.case_names("decode"))
def test_decode_batch_matches_reference_golden(name, cuda, native_lib):
    """triton_paged_attention_decode_batch (scatter + decode) vs the reference's
    paged_attention outputs stored in the fixture."""
    import qwen3_engine_from_scratch_b200 as qb
    case, m, inp, pool, caches = _golden_setup(name, cuda)
    qb.clear_device_status()
    q = _bf16(inp["q"], cuda)[:, :, None]
    out = qb.triton_paged_attention_decode_batch(
        q, _bf16(inp["k_new"], cuda)[:, :, None], _bf16(inp["v_new"], cuda)[:, :, None], caches,
        m["layer"], m["scaling"], row_ids=None)
    torch.cuda.synchronize()
    qb.check_device_status()
    assert out.shape == (len(caches), 1, m["H"] * m["D"])
    _close(out, case["out"])


@pytest.mark.parametrize("name", ["decode_c1", "decode_g4_edges"])
def test_single_request_entry_matches_golden(name, cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    case, m, inp, pool, caches = _golden_setup(name, cuda)
    for b, c in enumerate(caches):
        c.reserve_next()
        out = qb.triton_paged_attention_decode(
            _bf16(inp["q"][b:b + 1], cuda)[:, :, None], _bf16(inp["k_new"][b:b + 1], cuda)[:, :, None],
            _bf16(inp["v_new"][b:b + 1], cuda)[:, :, None], c, m["layer"], m["scaling"])
        _close(out, case["out"][b:b + 1])


@pytest.mark.parametrize("pps", [1, 2, 5, 16, 128])
def test_split_sizes_agree(pps, cuda, native_lib):
    """Every split size gives the oracle's answer (exercises 1..many splits per request)."""
    import qwen3_engine_from_scratch_b200 as qb
    case, m, inp, pool, caches = _golden_setup("decode_c1", cuda)
    for c in caches:
        c.reserve_next()
    rows = torch.tensor([c.row_id for c in caches], dtype=torch.int32, device=cuda)
    pool.update_kv_batch(m["layer"], _bf16(inp["k_new"], cuda)[:, :, None],
                         _bf16(inp["v_new"], cuda)[:, :, None], rows)
    out = qb.paged_decode(_bf16(inp["q"], cuda), pool.k_buffer[:, m["layer"]],
                          pool.v_buffer[:, m["layer"]], pool.block_table_2d, pool.seq_lens, rows,
                          m["scaling"], pages_per_split=pps)
    _close(out, case["out"])


def _c2_like(device, B=64, H=16, Hkv=8, lo=128, hi=4096, num_blocks=32768, seed=1234,
             max_seq_len=4096):
    """Config-2 shaped pool: random block placement, Q/K RMS-normed + RoPE'd
    (theta 1e6) on the GPU.  Returns the tensors plus host copies for the oracle."""
    g = torch.Generator(device=device).manual_seed(seed)
    lens = torch.randint(lo, hi + 1, (B,), generator=g, device=device).cpu().numpy()
    max_pages = (max_seq_len + 15) // 16
    perm = torch.randperm(num_blocks, generator=g, device=device).cpu().numpy()
    bt = np.full((B + 3, max_pages), -1, np.int32)
    rows = (np.arange(B) * 7 + 2) % (B + 3)                      # non-trivial row slots
    used = 0
    for b in range(B):
        n = (int(lens[b]) + 15) // 16
        bt[rows[b], :n] = perm[used:used + n]
        used += n
    seq = np.zeros(B + 3, np.int32)
    seq[rows] = lens - 1                                         # excludes the current token
    D = 128
    kp = torch.zeros(num_blocks, Hkv, 16, D, dtype=torch.bfloat16, device=device)
    vp = torch.zeros_like(kp)
    # fill only the used pages with N(0,1) data; K is RMS-normed and RoPE'd per position
    pos_all, pages_all, rows_k = [], [], []
    for b in range(B):
        L = int(lens[b])
        pos = np.arange(L)
        pos_all.append(pos)
        pages_all.append(bt[rows[b], pos // 16].astype(np.int64) * 16 + pos % 16)
    pos_all = torch.from_numpy(np.concatenate(pos_all)).to(device)
    slots = torch.from_numpy(np.concatenate(pages_all)).to(device)
    T = slots.numel()
    kx = torch.randn(T, Hkv, D, generator=g, device=device)
    vx = torch.randn(T, Hkv, D, generator=g, device=device)
    kx = kx * torch.rsqrt(kx.pow(2).mean(-1, keepdim=True) + 1e-6)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D))
    ang = pos_all.float()[:, None] * inv[None]
    cos = torch.cat([ang, ang], -1).cos()[:, None]
    sin = torch.cat([ang, ang], -1).sin()[:, None]
    kx = kx * cos + torch.cat([-kx[..., D // 2:], kx[..., :D // 2]], -1) * sin
    kp5 = kp.view(num_blocks, 1, Hkv, 16, D)
    vp5 = vp.view(num_blocks, 1, Hkv, 16, D)
    import qwen3_engine_from_scratch_b200 as qb
    qb.kv_scatter_slots(kx.to(torch.bfloat16), vx.to(torch.bfloat16), kp5, vp5, slots)
    q = torch.randn(B, H, D, generator=g, device=device)
    q = q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + 1e-6)
    qpos = torch.from_numpy(lens - 1).to(device).float()
    ang = qpos[:, None] * inv[None]
    cq = torch.cat([ang, ang], -1).cos()[:, None]
    sq = torch.cat([ang, ang], -1).sin()[:, None]
    q = (q * cq + torch.cat([-q[..., D // 2:], q[..., :D // 2]], -1) * sq).to(torch.bfloat16)
    return dict(q=q, kp=kp, vp=vp, bt=torch.from_numpy(bt).to(device),
                seq=torch.from_numpy(seq).to(device), rows=torch.from_numpy(rows.astype(np.int32)).to(device),
                lens=lens, bt_np=bt, seq_np=seq, rows_np=rows, H=H, Hkv=Hkv)


def _oracle_subset(w, idx):
    """Oracle on a subset of requests, on a compact copy of the pages they use."""
    q = w["q"][idx].float().cpu().numpy()
    rows = w["rows_np"][idx]
    bt = w["bt_np"]
    pages = np.unique(np.concatenate([bt[r][bt[r] >= 0] for r in rows]))
    remap = np.full(w["kp"].shape[0], -1, np.int64)
    remap[pages] = np.arange(len(pages))
    bt_sub = np.full((len(idx), bt.shape[1]), -1, np.int32)
    for j, r in enumerate(rows):
        ok = bt[r] >= 0
        bt_sub[j, ok] = remap[bt[r][ok]]
    pages_t = torch.from_numpy(pages).to(w["kp"].device)
    kp = w["kp"][pages_t].float().cpu().numpy()
    vp = w["vp"][pages_t].float().cpu().numpy()
    return oa.paged_decode(q, kp, vp, bt_sub, w["seq_np"][rows], np.arange(len(idx)), 16,
                           1 / math.sqrt(128))


@pytest.mark.parametrize("H,Hkv", [(16, 8), (32, 8)])
def test_config2_shape_vs_oracle(H, Hkv, cuda, native_lib):
    """Config 2 (B=64, L~U[128,4096], 32768-block pool), and the Qwen3-8B head shape."""
    import qwen3_engine_from_scratch_b200 as qb
    w = _c2_like(cuda, H=H, Hkv=Hkv, num_blocks=16384)
    qb.clear_device_status()
    out = qb.paged_decode(w["q"], w["kp"], w["vp"], w["bt"], w["seq"], w["rows"], 1 / math.sqrt(128))
    torch.cuda.synchronize()
    qb.check_device_status()
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    idx = np.array([0, 1, int(np.argmax(w["lens"])), int(np.argmin(w["lens"])), 17, 63])
    ref = _oracle_subset(w, idx)
    _close(out[idx], ref)


def test_batch_permutation_and_split_invariance(cuda, native_lib):
    """Size-independent properties at full config-2 size: permuting the batch
    permutes the output bit-exactly; two half batches equal one full batch at
    the same split size (the default split depends on the batch size)."""
    import qwen3_engine_from_scratch_b200 as qb
    w = _c2_like(cuda, num_blocks=16384, seed=99)
    scale = 1 / math.sqrt(128)
    full = qb.paged_decode(w["q"], w["kp"], w["vp"], w["bt"], w["seq"], w["rows"], scale)
    perm = torch.randperm(64, device=cuda)
    permuted = qb.paged_decode(w["q"][perm], w["kp"], w["vp"], w["bt"], w["seq"], w["rows"][perm], scale)
    assert torch.equal(permuted, full[perm])
    pps = int(qb._native.load().b200_paged_decode_default_split(64, 8, w["bt"].shape[1]))
    a = qb.paged_decode(w["q"][:32], w["kp"], w["vp"], w["bt"], w["seq"], w["rows"][:32], scale,
                        pages_per_split=pps)
    b = qb.paged_decode(w["q"][32:], w["kp"], w["vp"], w["bt"], w["seq"], w["rows"][32:], scale,
                        pages_per_split=pps)
    assert torch.equal(torch.cat([a, b]), full)


def test_strided_q_from_fused_qkv(cuda, native_lib):
    """q as a non-contiguous view of a fused qkv projection (qwen3/attention.py:83-84)."""
    import qwen3_engine_from_scratch_b200 as qb
    case, m, inp, pool, caches = _golden_setup("decode_c1", cuda)
    B, H, Hkv, D = len(caches), m["H"], m["Hkv"], m["D"]
    qkv = torch.zeros(B, 1, (H + 2 * Hkv) * D, dtype=torch.bfloat16, device=cuda)
    qkv[..., :H * D] = _bf16(inp["q"], cuda).reshape(B, 1, H * D)
    qkv[..., H * D:(H + Hkv) * D] = _bf16(inp["k_new"], cuda).reshape(B, 1, Hkv * D)
    qkv[..., (H + Hkv) * D:] = _bf16(inp["v_new"], cuda).reshape(B, 1, Hkv * D)
    q = qkv[..., :H * D].view(B, 1, H, D).transpose(1, 2)
    k = qkv[..., H * D:(H + Hkv) * D].view(B, 1, Hkv, D).transpose(1, 2)
    v = qkv[..., (H + Hkv) * D:].view(B, 1, Hkv, D).transpose(1, 2)
    assert not q.is_contiguous() and not k.is_contiguous()
    out = qb.triton_paged_attention_decode_batch(q, k, v, caches, m["layer"], m["scaling"])
    _close(out, case["out"])


def test_cuda_graph_capture_and_replay(cuda, native_lib):
    """The decode step captures into a CUDA graph; replays follow seq_lens changes."""
    import qwen3_engine_from_scratch_b200 as qb
    case, m, inp, pool, caches = _golden_setup("decode_c1", cuda)
    B = len(caches)
    for c in caches:
        c._ensure_pages(c.seq_len + 3)   # room for this token and the next two
    rows = torch.tensor([c.row_id for c in caches], dtype=torch.int32, device=cuda)
    sq = _bf16(inp["q"], cuda)[:, :, None].clone()
    sk = _bf16(inp["k_new"], cuda)[:, :, None].clone()
    sv = _bf16(inp["v_new"], cuda)[:, :, None].clone()
    layer, scale = m["layer"], m["scaling"]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            qb.triton_paged_attention_decode_batch(sq, sk, sv, caches, layer, scale, rows)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gout = qb.triton_paged_attention_decode_batch(sq, sk, sv, caches, layer, scale, rows)
    g.replay()
    torch.cuda.synchronize()
    _close(gout, case["out"])
    # advance every request by one token, feed a new step, compare with eager
    for c in caches:
        c.advance_seq_len(1)
    sq.copy_(torch.roll(sq, 1, dims=1))
    g.replay()
    torch.cuda.synchronize()
    graph_out = gout.clone()
    # the eager call rewrites the same token at the same slot, then attends
    eager = qb.triton_paged_attention_decode_batch(sq, sk, sv, caches, layer, scale, rows)
    assert torch.equal(graph_out, eager)


def test_bad_rows_and_pages_are_flagged(cuda, native_lib):
    """Invalid row ids give zeros + a status bit; -1 pages are flagged (the
    reference would read out of bounds)."""
    import qwen3_engine_from_scratch_b200 as qb
    case, m, inp, pool, caches = _golden_setup("decode_c1", cuda)
    rows = torch.tensor([caches[0].row_id, 999], dtype=torch.int32, device=cuda)
    qb.clear_device_status()
    out = qb.paged_decode(_bf16(inp["q"][:2], cuda), pool.k_buffer[:, 0], pool.v_buffer[:, 0],
                          pool.block_table_2d, pool.seq_lens, rows, m["scaling"])
    torch.cuda.synchronize()
    assert qb.device_status() & 0x1
    assert not out[1].any()
    # a row whose table says -1 for a visible page
    free_row = pool.alloc_row()
    pool.seq_lens[free_row] = 20
    qb.clear_device_status()
    qb.paged_decode(_bf16(inp["q"][:1], cuda), pool.k_buffer[:, 0], pool.v_buffer[:, 0],
                    pool.block_table_2d, pool.seq_lens,
                    torch.tensor([free_row], dtype=torch.int32, device=cuda), m["scaling"])
    torch.cuda.synchronize()
    assert qb.device_status() & 0x2
    qb.clear_device_status()


def test_decode_argument_errors(cuda, native_lib):
    import qwen3_engine_from_scratch_b200 as qb
    case, m, inp, pool, caches = _golden_setup("decode_g1", cuda)
    q = _bf16(inp["q"], cuda)
    with pytest.raises(AssertionError):
        qb.triton_paged_attention_decode_batch(q[:, :, None].half(), q[:, :, None], q[:, :, None],
                                               caches, 0, 1.0)
    with pytest.raises(AssertionError):   # S != 1
        qb.triton_paged_attention_decode_batch(torch.cat([q[:, :, None]] * 2, 2), q, q, caches, 0, 1.0)
    with pytest.raises(AssertionError):   # len(kv_caches) != B
        qb.triton_paged_attention_decode_batch(q[:, :, None], q, q, caches[:1], 0, 1.0)


def _fused_state(device, B=64, Hkv=8, H=16, layers=2, max_len=2000, seed=77):
    """A 2-layer pool filled with N(0,1) everywhere (so a stale read of the new
    token's slot changes the result), random page placement, row slots that
    are not 0..B-1, lengths including page-boundary cases."""
    g = torch.Generator(device=device).manual_seed(seed)
    lens = torch.randint(1, max_len, (B,), generator=g, device=device).cpu().numpy()
    lens[:4] = [1, 16, 17, 33]                          # seq_lens 0, 15, 16, 32: page starts
    spare = 4                                           # room for a few more steps
    max_pages = (max_len + spare + 15) // 16 + 1
    need = int(sum((L + spare + 15) // 16 for L in lens))
    num_blocks = need + 64
    perm = torch.randperm(num_blocks, generator=g, device=device).cpu().numpy()
    R = B + 5
    rows = (np.arange(B) * 11 + 3) % R
    bt = np.full((R, max_pages), -1, np.int32)
    used = 0
    for b in range(B):
        n = (int(lens[b]) + spare + 15) // 16
        bt[rows[b], :n] = perm[used:used + n]
        used += n
    seq = np.zeros(R, np.int32)
    seq[rows] = lens - 1
    D = 128
    kp = torch.randn(num_blocks, layers, Hkv, 16, D, generator=g, device=device).to(torch.bfloat16)
    vp = torch.randn(num_blocks, layers, Hkv, 16, D, generator=g, device=device).to(torch.bfloat16)
    q = torch.randn(B, H, D, generator=g, device=device).to(torch.bfloat16)
    # k/v new as strided views of one fused (B, H + 2 Hkv, D) projection
    qkv = torch.randn(B, H + 2 * Hkv, D, generator=g, device=device).to(torch.bfloat16)
    return dict(q=q, k_new=qkv[:, H:H + Hkv], v_new=qkv[:, H + Hkv:], kp=kp, vp=vp,
                bt=torch.from_numpy(bt).to(device), seq=torch.from_numpy(seq).to(device),
                rows=torch.from_numpy(rows.astype(np.int32)).to(device))


@pytest.mark.parametrize("pps", [0, 1, 4, 128])
def test_fused_kv_write_equals_write_then_decode(pps, cuda, native_lib):
    """b200_paged_decode_kv_write == b200_kv_scatter_rows + b200_paged_decode,
    bit for bit: the outputs and every byte of both layers of the pool."""
    import qwen3_engine_from_scratch_b200 as qb
    w = _fused_state(cuda)
    scale = 128 ** -0.5
    for layer in (1, 0):
        ka, va = w["kp"].clone(), w["vp"].clone()
        kb, vb = w["kp"].clone(), w["vp"].clone()
        qb.clear_device_status()
        qb.kv_scatter_rows(w["k_new"][:, :, None], w["v_new"][:, :, None], ka, va, w["seq"],
                           w["bt"], w["rows"], layer)
        ref = qb.paged_decode(w["q"], ka[:, layer], va[:, layer], w["bt"], w["seq"], w["rows"],
                              scale, pages_per_split=pps)
        out = qb.paged_decode_kv_write(w["q"], w["k_new"], w["v_new"], kb[:, layer], vb[:, layer],
                                       w["bt"], w["seq"], w["rows"], scale, pages_per_split=pps)
        torch.cuda.synchronize()
        qb.check_device_status()
        assert torch.equal(out, ref)
        assert torch.equal(ka, kb) and torch.equal(va, vb)
        # the new rows really landed (the pool held other values there before)
        assert not torch.equal(ka, w["kp"])


def test_fused_kv_write_repeated_and_in_graph(cuda, native_lib):
    """Several fused steps in a row (seq_lens advancing, as the engine does
    between steps) match the unfused pair, also when captured in a CUDA graph."""
    import qwen3_engine_from_scratch_b200 as qb
    w = _fused_state(cuda, B=32, max_len=600, seed=5)
    scale = 128 ** -0.5
    ka, va = w["kp"].clone(), w["vp"].clone()
    kb, vb = w["kp"].clone(), w["vp"].clone()
    seq_a, seq_b = w["seq"].clone(), w["seq"].clone()
    out_b = torch.empty_like(w["q"])

    def fused():
        qb.paged_decode_kv_write(w["q"], w["k_new"], w["v_new"], kb[:, 0], vb[:, 0], w["bt"],
                                 seq_b, w["rows"], scale, out=out_b)

    fused()                                   # warm-up (workspace) before capture
    torch.cuda.synchronize()
    kb.copy_(w["kp"])
    vb.copy_(w["vp"])
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fused()
    for step in range(3):
        qb.kv_scatter_rows(w["k_new"][:, :, None], w["v_new"][:, :, None], ka, va, seq_a, w["bt"],
                           w["rows"], 0)
        ref = qb.paged_decode(w["q"], ka[:, 0], va[:, 0], w["bt"], seq_a, w["rows"], scale)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out_b, ref), step
        assert torch.equal(ka, kb) and torch.equal(va, vb), step
        seq_a[w["rows"].long()] += 1
        seq_b[w["rows"].long()] += 1
    del graph


def test_fused_kv_write_bad_page_flagged(cuda, native_lib):
    """A -1 block-table entry at the new token's page: flagged, no store."""
    import qwen3_engine_from_scratch_b200 as qb
    w = _fused_state(cuda, B=8, max_len=300, seed=9)
    bt = w["bt"].clone()
    r0 = int(w["rows"][0])
    pos = int(w["seq"][r0])
    bt[r0, pos // 16] = -1
    kb, vb = w["kp"].clone(), w["vp"].clone()
    qb.clear_device_status()
    qb.paged_decode_kv_write(w["q"], w["k_new"], w["v_new"], kb[:, 0], vb[:, 0], bt, w["seq"],
                             w["rows"], 128 ** -0.5)
    torch.cuda.synchronize()
    assert qb.device_status() & 0x2
    qb.clear_device_status()
