"""The allocation-free entry point, apk_sgemm_f32_noalloc, through the C ABI.

It serves callers that cannot call cudaMalloc (their device memory belongs
to a pool they do not control, or they must not allocate while serving), so
its scratch lives in a static device array instead.  This file is collected
last on purpose: a failure here leaves every other test already run.

The check: two calls in a row on the same inputs must each match the
allocating entry point (apk_gemm, same kernel) within the fp32 tolerance the
other tests use (1e-5*sqrt(K) of float64, and against apk_gemm's output),
so the second call also shows that the shared scratch is reset between
calls.  Device buffers come from torch (plumbing only: the test is not the
caller that cannot allocate).
"""
import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def test_noalloc_matches_allocating_entry_point_twice(libapk):
    import torch

    import apk_b200

    M, N, K = 1024, 768, 512
    A, B = oracle.gen_uniform(M, N, K, 21)
    with apk_b200.Context(poll="off") as c:
        C_ref = c.gemm(A, B)  # the existing (allocating) entry point
    ref64 = oracle.gemm_f64(A, B)
    tol = oracle.fp32_tol(K)

    dA = torch.from_numpy(A).cuda()
    dB = torch.from_numpy(B).cuda()
    dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
    for call in range(2):
        dC.fill_(float("nan"))
        torch.cuda.synchronize()
        st = libapk.apk_sgemm_f32_noalloc(ctypes.c_void_p(dA.data_ptr()), ctypes.c_void_p(dB.data_ptr()),
                                          ctypes.c_void_p(dC.data_ptr()), M, N, K, 0, None)
        assert st == 0, f"call {call}: status {st}"
        torch.cuda.synchronize()
        C = dC.cpu().numpy()
        mr, bad, nans = oracle.check(C, ref64, tol)
        assert nans == 0 and bad == 0, f"call {call}: {bad} bad, {nans} NaN, max rel {mr:.3e}"
        mr2, bad2, _ = oracle.check(C, C_ref.astype(np.float64), tol)
        assert bad2 == 0, f"call {call}: differs from apk_gemm (max rel {mr2:.3e})"


def test_noalloc_rejects_beyond_limits(libapk):
    import torch

    dA = torch.zeros((128, 32), dtype=torch.float32, device="cuda")
    dB = torch.zeros((32, 128), dtype=torch.float32, device="cuda")
    dC = torch.zeros((128, 128), dtype=torch.float32, device="cuda")
    p = [ctypes.c_void_p(t.data_ptr()) for t in (dA, dB, dC)]
    # a grid beyond the kernel's residency (2 CTAs per SM) is refused before
    # the scratch-size check, whose 2016-CTA limit no B200 grid reaches
    assert libapk.apk_sgemm_f32_noalloc(*p, 128, 128, 32, 100000, None) == 1  # APK_EINVAL
    # a shape that is not tile-aligned
    assert libapk.apk_sgemm_f32_noalloc(*p, 100, 128, 32, 0, None) == 1
    # and a valid call still works afterwards
    assert libapk.apk_sgemm_f32_noalloc(*p, 128, 128, 32, 0, None) == 0
    torch.cuda.synchronize()
    assert float(dC.abs().sum()) == 0.0
    st = ctypes.c_int(-1)
    assert libapk.apk_sgemm_f32_noalloc_status(None, ctypes.byref(st)) == 0
    assert st.value == 0


def test_noalloc_status_reports_a_wait_that_ran_out(libapk):
    """A kernel whose bounded wait gives up leaves C incomplete while the
    asynchronous call has already returned APK_OK: the status query must show
    it.  The self-test queues the same kind of bounded spin on a scratch word
    nothing sets (no fault, no hang: it gives up after 50 ms), then a normal
    call clears the word again."""
    import torch

    st = ctypes.c_int(-1)
    assert libapk.apk_sgemm_f32_noalloc_selftest(50_000_000, None) == 0
    assert libapk.apk_sgemm_f32_noalloc_status(None, ctypes.byref(st)) == 0
    assert st.value == 3  # DEV_WAIT_TIMEOUT_SPIN

    A, B = oracle.gen_uniform(256, 256, 128, 5)
    dA = torch.from_numpy(A).cuda()
    dB = torch.from_numpy(B).cuda()
    dC = torch.full((256, 256), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    assert libapk.apk_sgemm_f32_noalloc(ctypes.c_void_p(dA.data_ptr()), ctypes.c_void_p(dB.data_ptr()),
                                        ctypes.c_void_p(dC.data_ptr()), 256, 256, 128, 0, None) == 0
    assert libapk.apk_sgemm_f32_noalloc_status(None, ctypes.byref(st)) == 0
    assert st.value == 0
    mr, bad, nans = oracle.check(dC.cpu().numpy(), oracle.gemm_f64(A, B), oracle.fp32_tol(128))
    assert bad == 0 and nans == 0, f"{bad} bad, {nans} NaN, max rel {mr:.3e}"
