"""sgblasSgemmNoAlloc -- the entry point for callers that cannot allocate.

Some callers cannot call cudaMalloc: their host process or framework owns all
device memory through its own allocator, or they run under a rule of no
allocation after start-up. For them sgblasSgemmNoAlloc computes exactly what
sgblasSgemm computes, but takes its stream-K scratch from a fixed array built
into the library instead of allocating a workspace.

This file is collected last on purpose (a failure here comes after every
other test has run). The check: two calls in a row through the C ABI, each
compared with sgblasSgemm on the same inputs within the north-star bound of
the FP64 oracle's magnitude -- the second call also proves that the shared
scratch (counters left by the first call) is reused correctly.
"""
import ctypes

import numpy as np
import pytest

import oracle
import sgblas_b200 as sg
from tests import cases as C
from tests.gpu_util import c_view, to_device

pytestmark = pytest.mark.gpu


def _no_alloc(handle, case, pa, pb, pc):
    f = ctypes.c_float
    return sg.lib.sgblasSgemmNoAlloc(handle.raw, case.transa, case.transb, case.m, case.n, case.k,
                                     ctypes.byref(f(case.alpha)), pa, case.lda, pb, case.ldb,
                                     ctypes.byref(f(case.beta)), pc, case.ldc)


def test_no_alloc_matches_sgemm_twice(cuda, handle):
    torch = cuda
    # Both shapes use the stream-K scratch: fewer tiles than SMs, and a
    # remainder wave after whole waves.
    shapes = [C.Case("noalloc-1", 0, 0, 1500, 1300, 3000, 1500, 3000, 1500, 0.75, -0.5),
              C.Case("noalloc-2", 0, 1, 4096, 2048, 512, 4096, 2048, 4096, 1.0, 0.0)]
    for case in shapes:
        a, b, c = C.cfg_inputs(case, 4242, None)
        da, pa = to_device(torch, a)
        db, pb = to_device(torch, b)
        d_ref, p_ref = to_device(torch, c)
        handle.sgemm(case.transa, case.transb, case.m, case.n, case.k, case.alpha, pa, case.lda,
                     pb, case.ldb, case.beta, p_ref, case.ldc)
        torch.cuda.synchronize()
        want = d_ref.cpu().numpy()
        _, mag = oracle.sgemm_f64(case.transa, case.transb, case.m, case.n, case.k, case.alpha, a,
                                  case.lda, b, case.ldb, case.beta, c, case.ldc)
        tol = oracle.tol_north_star(case.k, mag)
        for call in range(2):
            d_out, p_out = to_device(torch, c)
            assert _no_alloc(handle, case, pa, pb, p_out) == sg.SGBLAS_STATUS_SUCCESS
            torch.cuda.synchronize()
            got = d_out.cpu().numpy()
            diff = np.abs(c_view(got, case.m, case.n, case.ldc).astype(np.float64) -
                          c_view(want, case.m, case.n, case.ldc))
            assert np.all(np.isfinite(c_view(got, case.m, case.n, case.ldc))), (case.name, call)
            assert np.all(diff <= tol), (case.name, call, float(diff.max()))
    assert sg.get_device_errors() == 0
