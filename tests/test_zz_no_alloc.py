"""GPU test of ``b200_paged_decode_noalloc``, the decode entry point that allocates nothing.

Some callers cannot allocate device memory at the moment they launch decode:
an engine that has handed nearly all HBM to its KV-cache pool and runs a fixed
arena, a foreign-language binding that holds raw device pointers but no device
allocator, a loop that cannot pay cudaMalloc's latency or its implicit
synchronisation.  ``b200_paged_decode`` needs a caller workspace for its
split-K partials; ``b200_paged_decode_noalloc`` keeps them in a static
16 MiB per-GPU array instead.

It runs the same kernel at the same (default) split as ``ops.paged_decode``,
whose partials are merged in a fixed order, so the two outputs must be equal
bit for bit.  This file calls the new entry point through the C ABI three
times in a row -- the second call with another batch, head count, block-table
width and split count than the first, so stale contents of the shared array
sit at other offsets, the third back on the first shape with new data -- and
checks each result with ``torch.equal`` against ``b200_paged_decode`` (the
workspace-taking entry point), and the first also against the fp32 oracle
within the decode tolerance of these tests (max-abs 2e-2, mean-abs 2e-3).  It
also checks the size limit at its boundary: the largest batch whose workspace
at the resolved default split fits the array is accepted although the
worst-case sizing query reports more than the array holds, and one request
more is refused.  The file name makes pytest collect it last.
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
SCRATCH = 16 << 20      # B200_DECODE_NOALLOC_SCRATCH_BYTES


def _workload(device, seed, B=16, H=16, Hkv=8, lo=100, hi=1500, max_seq_len=2048,
              num_blocks=4096):
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
    assert used <= num_blocks
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


def _run_and_compare(lib, w, status, cuda):
    from qwen3_engine_from_scratch_b200 import ops
    pps = int(lib.b200_paged_decode_default_split(w["B"], w["Hkv"], w["max_pages"]))
    # the shapes need split partials, i.e. the static array is really used
    need = lib.b200_paged_decode_workspace_size(w["B"], w["H"], w["max_pages"], pps)
    assert 0 < need <= SCRATCH
    out = torch.full((w["B"], w["H"], D), float("nan"), dtype=torch.bfloat16, device=cuda)
    st = _noalloc(lib, w, out, status.data_ptr())
    assert st == 0, f"b200_paged_decode_noalloc returned {st}"
    ref = ops.paged_decode(w["q"], w["kp"], w["vp"], w["bt"], w["seq"], w["rows"],
                           1.0 / math.sqrt(D))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(out, ref), (out.float() - ref.float()).abs().max().item()
    return out, pps


def test_noalloc_decode_equals_workspace_entry_three_calls(cuda, native_lib):
    lib = native_lib
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    first = _workload(cuda, 11)
    out, pps1 = _run_and_compare(lib, first, status, cuda)
    # the first call against the fp32 oracle
    ref = oa.paged_decode(first["q"].float().cpu().numpy(), first["kp"].float().cpu().numpy(),
                          first["vp"].float().cpu().numpy(), first["bt"].cpu().numpy(),
                          first["seq"].cpu().numpy(), first["rows"].cpu().numpy(), 16,
                          1.0 / math.sqrt(D))
    err = np.abs(out.float().cpu().numpy() - ref)
    assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())
    # another batch, head count, table width and split count: the pairs and the
    # partials of this call sit at other offsets of the shared array
    second = _workload(cuda, 12, B=24, H=32, Hkv=8, lo=600, hi=4000, max_seq_len=4096,
                       num_blocks=8192)
    _, pps2 = _run_and_compare(lib, second, status, cuda)
    ms1 = (first["max_pages"] + pps1 - 1) // pps1
    ms2 = (second["max_pages"] + pps2 - 1) // pps2
    assert (second["B"] * second["Hkv"], ms2) != (first["B"] * first["Hkv"], ms1)
    # back to the first shape with new data, over what the second call left
    _run_and_compare(lib, _workload(cuda, 13), status, cuda)


def test_noalloc_limit_at_its_boundary(cuda, native_lib):
    """The limit is checked at the split the call resolves (the default split),
    not at the worst-case size that workspace_size(..., 0) reports."""
    lib = native_lib
    H, Hkv, max_pages = 32, 8, 512

    def need(B):
        return lib.b200_paged_decode_workspace_size(
            B, H, max_pages, lib.b200_paged_decode_default_split(B, Hkv, max_pages))

    b_max = max(B for B in range(1, 1024) if need(B) <= SCRATCH)
    assert need(b_max + 1) > SCRATCH
    # the worst-case query disagrees: it would refuse b_max
    assert lib.b200_paged_decode_workspace_size(b_max, H, max_pages, 0) > SCRATCH
    # b_max requests of 100-300 tokens in a 512-page-wide block table: accepted,
    # equal to the workspace entry
    w = _workload(cuda, 21, B=b_max, H=H, Hkv=Hkv, lo=100, hi=300, max_seq_len=max_pages * 16,
                  num_blocks=b_max * 20 + 16)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    _run_and_compare(lib, w, status, cuda)
    # one request more: refused before anything is launched
    st = lib.b200_paged_decode_noalloc(None, 0, 0, None, None, 0, 0, 0, None, 1, None, None,
                                       None, 0, 0, b_max + 1, H, Hkv, D, 16, 1, max_pages, 1,
                                       1.0, 0, None, None)
    assert st == -4   # B200_ERR_WORKSPACE


def test_noalloc_refuses_shapes_beyond_its_scratch(native_lib):
    lib = native_lib
    # 512 requests x 64 heads x 2048 pages at 16 pages per split needs ~2 GB of partials
    assert lib.b200_paged_decode_workspace_size(512, 64, 2048, 16) > SCRATCH
    st = lib.b200_paged_decode_noalloc(None, 0, 0, None, None, 0, 0, 0, None, 1, None, None, None,
                                       0, 0, 512, 64, 8, D, 16, 1, 2048, 1, 1.0, 16, None, None)
    assert st == -4   # B200_ERR_WORKSPACE: beyond the static maximum, nothing launched
