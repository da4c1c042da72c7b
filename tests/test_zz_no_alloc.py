"""GPU test of ``b200_paged_decode_noalloc``, the decode entry point that allocates nothing.

Some callers cannot allocate device memory at the moment they launch decode:
an engine that has handed nearly all HBM to its KV-cache pool and runs a fixed
arena, a foreign-language binding that holds raw device pointers but no device
allocator, a loop that cannot pay cudaMalloc's latency or its implicit
synchronisation.  ``b200_paged_decode`` needs a caller workspace for its
split-K partials; ``b200_paged_decode_noalloc`` keeps them in a static
16 MiB per-GPU array instead.

This file calls the new entry point through the C ABI twice in a row, on
different inputs, and checks each result against ``b200_paged_decode`` (the
workspace-taking entry point) within the decode tolerance used everywhere in
these tests: max-abs 2e-2, mean-abs 2e-3.  It also checks that a request
needing more scratch than the static maximum is refused.  The file name makes
pytest collect it last.
"""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3
D = 128


def _workload(device, seed, B=16, H=16, Hkv=8, lo=100, hi=1500, max_seq_len=2048, num_blocks=4096):
    g = torch.Generator(device=device).manual_seed(seed)
    lens = torch.randint(lo, hi + 1, (B,), generator=g, device=device).cpu().numpy()
    max_pages = (max_seq_len + 15) // 16
    perm = torch.randperm(num_blocks, generator=g, device=device).cpu().numpy()
    bt = np.full((B + 2, max_pages), -1, np.int32)
    rows = np.arange(B, dtype=np.int32)[::-1].copy() + 1
    used = 0
    for b in range(B):
        n = (int(lens[b]) + 15) // 16
        bt[rows[b], :n] = perm[used:used + n]
        used += n
    seq = np.zeros(B + 2, np.int32)
    seq[rows] = lens - 1
    kp = torch.randn(num_blocks, Hkv, 16, D, generator=g, device=device).to(torch.bfloat16)
    vp = torch.randn(num_blocks, Hkv, 16, D, generator=g, device=device).to(torch.bfloat16)
    q = torch.randn(B, H, D, generator=g, device=device).to(torch.bfloat16)
    return dict(q=q, kp=kp, vp=vp, bt=torch.from_numpy(bt).to(device),
                seq=torch.from_numpy(seq).to(device), rows=torch.from_numpy(rows).to(device),
                B=B, H=H, Hkv=Hkv, num_blocks=num_blocks, max_pages=max_pages)


def _noalloc(lib, w, out, status_ptr):
    q, kp, bt = w["q"], w["kp"], w["bt"]
    return lib.b200_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), kp.data_ptr(), w["vp"].data_ptr(),
        kp.stride(0), kp.stride(1), kp.stride(2), bt.data_ptr(), bt.stride(0),
        w["seq"].data_ptr(), w["rows"].data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
        w["B"], w["H"], w["Hkv"], D, 16, w["num_blocks"], w["max_pages"], bt.shape[0],
        1.0 / math.sqrt(D), 0, status_ptr, torch.cuda.current_stream().cuda_stream)


def test_noalloc_decode_matches_workspace_entry_twice(cuda, native_lib):
    from qwen3_engine_from_scratch_b200 import ops
    lib = native_lib
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    for seed in (11, 12):          # two calls in a row, different inputs
        w = _workload(cuda, seed)
        # the shapes need split partials, i.e. the static scratch is really used
        need = lib.b200_paged_decode_workspace_size(w["B"], w["H"], w["max_pages"], 0)
        assert 0 < need <= (16 << 20)
        out = torch.empty(w["B"], w["H"], D, dtype=torch.bfloat16, device=cuda)
        st = _noalloc(lib, w, out, status.data_ptr())
        assert st == 0, f"b200_paged_decode_noalloc returned {st}"
        ref = ops.paged_decode(w["q"], w["kp"], w["vp"], w["bt"], w["seq"], w["rows"],
                               1.0 / math.sqrt(D))
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        err = (out.float() - ref.float()).abs()
        assert torch.isfinite(out.float()).all()
        assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS, \
            (err.max().item(), err.mean().item())


def test_noalloc_refuses_shapes_beyond_its_scratch(native_lib):
    lib = native_lib
    # 512 requests x 64 heads x 2048 pages at 16 pages per split needs ~2 GB of partials
    assert lib.b200_paged_decode_workspace_size(512, 64, 2048, 16) > (16 << 20)
    st = lib.b200_paged_decode_noalloc(None, 0, 0, None, None, 0, 0, 0, None, 1, None, None, None,
                                       0, 0, 512, 64, 8, D, 16, 1, 2048, 1, 1.0, 16, None, None)
    assert st == -4   # B200_ERR_WORKSPACE: beyond the static maximum, nothing launched
