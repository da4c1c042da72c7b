"""Failure detection on the GPU, without a fault.

Every pipeline wait of the prefill kernel is bounded: after its limit it
records B200_DEV_TIMEOUT in the device status word and the kernel returns, so
the CUDA context stays usable; a status word that already holds a timeout ends
the waits of every other CTA of the grid and keeps later prefill launches from
starting work until the host clears it.  These tests make a wait run out on an
mbarrier that nothing completes (b200_selftest_bounded_wait, through the same
wait helper), check the status the host reads back, and check that the library
still computes correct results afterwards.

Tolerance of the prefill check (north_star): max-abs 2e-2 and mean-abs 2e-3
against the fp32 oracle.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from oracle import attention as oa

pytestmark = pytest.mark.gpu

DEV_TIMEOUT = 0x10
MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _probe(lib, status, result, limit_ns):
    t0 = time.perf_counter()
    rc = lib.b200_selftest_bounded_wait(status.data_ptr(), result.data_ptr(), int(limit_ns),
                                        _stream())
    torch.cuda.synchronize()
    return rc, time.perf_counter() - t0


def test_bounded_wait_gives_up_and_flags_timeout(cuda, native_lib):
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    result = torch.full((1,), -1, dtype=torch.int32, device=cuda)
    rc, dt = _probe(native_lib, status, result, 2_000_000)   # 2 ms of device time
    assert rc == 0
    assert int(result.item()) == 0, "the wait reported a completion nothing made"
    assert int(status.item()) & DEV_TIMEOUT
    assert dt < 5.0, dt


def test_recorded_timeout_ends_a_long_wait_at_once(cuda, native_lib):
    """A status word that already holds a timeout (another CTA gave up) ends a
    wait whose own limit is far away, as the prefill's CTAs end together."""
    status = torch.full((1,), DEV_TIMEOUT, dtype=torch.int32, device=cuda)
    result = torch.full((1,), -1, dtype=torch.int32, device=cuda)
    rc, dt = _probe(native_lib, status, result, 8_000_000_000)   # 8 s limit
    assert rc == 0
    assert int(result.item()) == 0
    assert dt < 2.0, dt


def test_probe_rejects_bad_arguments(cuda, native_lib):
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    result = torch.zeros(1, dtype=torch.int32, device=cuda)
    lib = native_lib
    assert lib.b200_selftest_bounded_wait(None, result.data_ptr(), 1000, _stream()) == -1
    assert lib.b200_selftest_bounded_wait(status.data_ptr(), result.data_ptr(), 0, _stream()) == -1
    assert lib.b200_selftest_bounded_wait(status.data_ptr(), result.data_ptr(), 20_000_000_000,
                                          _stream()) == -1


def test_prefill_waits_for_a_cleared_status_then_computes(cuda, native_lib):
    """After a timeout the prefill starts no work (its output stays as it was)
    until the host clears the status word; then it computes the right result:
    the context survived the timeout."""
    from qwen3_engine_from_scratch_b200 import ops
    lens = [200, 77, 129]
    H, Hkv, D = 16, 8, 128
    g = torch.Generator(device=cuda).manual_seed(31)
    T = sum(lens)
    q = torch.randn(T, H, D, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(T, Hkv, D, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(T, Hkv, D, generator=g, device=cuda).to(torch.bfloat16)
    cun = np.concatenate([[0], np.cumsum(lens)])
    cu = torch.tensor(cun, dtype=torch.int32, device=cuda)
    scale = D ** -0.5

    # a timeout recorded in the package's status word, as a timed-out wait leaves it
    ops.clear_device_status(cuda)
    ops._status_ptr(cuda)
    pkg_status = ops._status[cuda.index if cuda.index is not None else 0]
    result = torch.zeros(1, dtype=torch.int32, device=cuda)
    try:
        rc, _ = _probe(native_lib, pkg_status, result, 1_000_000)
        assert rc == 0 and ops.device_status(cuda) & DEV_TIMEOUT

        out = torch.full((T, H, D), 7.0, dtype=torch.bfloat16, device=cuda)
        ops._prefill(q, k, v, out, cu, None, max(lens), scale, H, Hkv, D, False)
        torch.cuda.synchronize()
        assert bool((out == 7.0).all()), "the prefill started work under a recorded timeout"

        ops.clear_device_status(cuda)
        ops._prefill(q, k, v, out, cu, None, max(lens), scale, H, Hkv, D, False)
        torch.cuda.synchronize()
        ops.check_device_status(cuda)
    finally:
        ops.clear_device_status(cuda)
    ref = oa.varlen_prefill(q.float().cpu().numpy(), k.float().cpu().numpy(),
                            v.float().cpu().numpy(), cun, scale)
    err = np.abs(out.float().cpu().numpy() - ref)
    assert np.isfinite(err).all()
    assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())
