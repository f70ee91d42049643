"""The TF32 lane (SGBLAS_MATH_TF32) on the GPU: tcgen05 tensor cores.

TF32 mode is outside the strict-FP32 contract (the reference returns
NOT_SUPPORTED for it, src/sgemm_cuda.cu:719-721; its design lists a TF32 lane
as future work). The bound used here follows from the format: each input
keeps 10 explicit mantissa bits (the tensor core reads the top 19 bits of the
FP32 word), so each product a*b carries a relative error below 2^-9, and the
FP32 accumulation adds at most (K + 2) roundings:

    |C - C_ref| <= (2^-9 + (K + 2) * 2^-22) * (|alpha| sum|a*b| + |beta*c|)

Beyond the bound, every test keeps sgblasSgemm's other guarantees: beta == 0
never reads C (NaN poison), padding rows stay untouched, and results are
reproducible run to run.
"""
import ctypes

import numpy as np
import pytest

import oracle
import sgblas_b200 as sg
from tests import cases as C
from tests.gpu_util import c_view, check_guards, run_sgemm, to_device

pytestmark = pytest.mark.gpu


def tol_tf32(k, mag):
    return (2.0 ** -9 + (k + 2) * 2.0 ** -22) * mag


def check_tf32(case, a, b, c0, out, what):
    ref, mag = oracle.sgemm_f64(case.transa, case.transb, case.m, case.n, case.k, case.alpha, a,
                                case.lda, b, case.ldb, case.beta, c0, case.ldc)
    got = c_view(out, case.m, case.n, case.ldc).astype(np.float64)
    assert np.all(np.isfinite(got)), what
    err = np.abs(got - ref)
    bound = tol_tf32(case.k, mag)
    assert np.all(err <= bound), (what, float((err / np.maximum(bound, 1e-30)).max()))
    pad_in = c0.reshape(case.n, case.ldc)[:, case.m:]
    pad_out = out.reshape(case.n, case.ldc)[:, case.m:]
    assert np.array_equal(pad_in, pad_out, equal_nan=True), (what, "padding rows written")
    return err, mag


@pytest.fixture
def tf32_handle(handle):
    handle.set_math_mode(sg.SGBLAS_MATH_TF32)
    yield handle
    handle.set_math_mode(sg.SGBLAS_MATH_FP32)


# 64-wide tiles for the first three and the last but one (128-wide tiles
# would leave over half the SMs idle), 128-wide for (1, 1, 1) and
# 1152 x 1200 (90 tiles of 128 x 128 for 148 SMs).
SHAPES = [(300, 200, 70), (257, 513, 100), (128, 256, 32), (1, 1, 1), (640, 768, 999),
          (1152, 1200, 200)]


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_tf32_modes_and_tails(cuda, tf32_handle, ta, tb, m, n, k):
    for alpha, beta in ((1.0, 0.0), (0.75, -1.25), (1.0, 1.0)):
        # leading dimensions rounded to 4 floats: the tensor-core kernel reads
        # the operands in place with TMA
        lda = -(-(k if ta else m) // 4) * 4 + 4
        ldb = -(-(n if tb else k) // 4) * 4
        case = C.Case("tf32", ta, tb, m, n, k, lda, ldb, m + 3, alpha, beta)
        a, b, c = C.cfg_inputs(case, 700 + m + n + k, None)
        C.pad_and_poison(c, m, n, case.ldc, beta, C.PRODUCT_PAD)
        status, out = run_sgemm(cuda, tf32_handle, case, a, b, c)
        assert status == 0
        check_tf32(case, a, b, c, out, (ta, tb, m, n, k, alpha, beta))
    assert sg.get_device_errors() == 0


def test_tf32_uses_tensor_cores_and_is_deterministic(cuda, handle):
    """The TF32 result differs from the strict-FP32 one by TF32-sized errors
    (so the tensor-core path ran), and repeats bit for bit."""
    case = C.Case("tf32-vs-fp32", 0, 0, 512, 512, 512, 512, 512, 512, 1.0, 0.0)
    a, b, c = C.cfg_inputs(case, 5, -1)
    _, fp32 = run_sgemm(cuda, handle, case, a, b, c)
    handle.set_math_mode(sg.SGBLAS_MATH_TF32)
    try:
        _, t1 = run_sgemm(cuda, handle, case, a, b, c)
        _, t2 = run_sgemm(cuda, handle, case, a, b, c)
    finally:
        handle.set_math_mode(sg.SGBLAS_MATH_FP32)
    assert np.array_equal(t1, t2)
    err, mag = check_tf32(case, a, b, c, t1, "tf32")
    diff = np.abs(t1.astype(np.float64) - fp32)
    assert diff.max() > 0.0
    # far above FP32 rounding, within the TF32 bound
    assert diff.max() > 64 * 2.0 ** -24 * mag.max()


@pytest.mark.parametrize("pad,offs", [(1, (0, 0, 0)), (0, (1, 2, 3))])
def test_tf32_operands_tma_cannot_read(cuda, tf32_handle, pad, offs):
    """Odd leading dimensions or misaligned bases: the operands are copied
    into the workspace first, then computed on the tensor cores."""
    for ta, tb in ((0, 0), (1, 1)):
        m, n, k = 333, 444, 123
        case = C.Case("tf32-copy", ta, tb, m, n, k, (k if ta else m) + pad,
                      (n if tb else k) + pad, m + 1, 1.5, 0.5)
        a, b, c = C.cfg_inputs(case, 31, None)
        status, out = run_sgemm(cuda, tf32_handle, case, a, b, c, offsets=offs)
        assert status == 0
        check_tf32(case, a, b, c, out, (ta, tb, pad, offs))


def test_tf32_large_sampled(cuda, tf32_handle):
    torch = cuda
    m = n = k = 4096
    case = C.Case("tf32-4096", 0, 0, m, n, k, m, k, m, 1.0, 0.0)
    a, b, c = C.cfg_inputs(case, 1, -1)
    status, out = run_sgemm(torch, tf32_handle, case, a, b, c)
    assert status == 0
    rng = np.random.default_rng(3)
    rows = np.concatenate([rng.integers(0, m, 2048), np.arange(0, m, 128), np.arange(127, m, 128)])
    cols = np.concatenate([rng.integers(0, n, 2048), rng.integers(0, n, 2 * (m // 128))])
    ref, mag = oracle.sgemm_f64_points(0, 0, k, 1.0, a, m, b, k, 0.0, c, m, rows, cols)
    got = out[rows + cols * m].astype(np.float64)
    assert np.all(np.abs(got - ref) <= tol_tf32(k, mag))
    assert np.all(np.isfinite(out))


def test_tf32_no_alloc_and_batched(cuda, tf32_handle):
    """sgblasSgemmNoAlloc runs the TF32 lane; a batch whose strides TMA
    cannot use (here 0: one A and one B for every product) computes in FP32
    (within the strict bound, which is tighter)."""
    torch = cuda
    case = C.Case("tf32-noalloc", 0, 1, 300, 260, 90, 300, 260, 300, 1.0, 0.0)
    a, b, c = C.cfg_inputs(case, 9, -1)
    da, pa = to_device(torch, a)
    db, pb = to_device(torch, b)
    dc, pc = to_device(torch, c)
    f = ctypes.c_float
    st = sg.lib.sgblasSgemmNoAlloc(tf32_handle.raw, 0, 1, case.m, case.n, case.k,
                                   ctypes.byref(f(1.0)), pa, case.lda, pb, case.ldb,
                                   ctypes.byref(f(0.0)), pc, case.ldc)
    torch.cuda.synchronize()
    assert st == 0
    check_guards(da, db, dc)
    check_tf32(case, a, b, c, dc.cpu().numpy(), "noalloc")
    dc2, pc2 = to_device(torch, np.concatenate([c, c]))
    tf32_handle.sgemm_strided_batched(0, 1, case.m, case.n, case.k, 1.0, pa, case.lda, 0, pb,
                                      case.ldb, 0, 0.0, pc2, case.ldc, case.c_size, 2)
    torch.cuda.synchronize()
    ref, mag = oracle.sgemm_f64(0, 1, case.m, case.n, case.k, 1.0, a, case.lda, b, case.ldb, 0.0,
                                c, case.ldc)
    both = dc2.cpu().numpy()
    for i in range(2):
        got = both[i * case.c_size:(i + 1) * case.c_size]
        res = oracle.check(c_view(got, case.m, case.n, case.ldc), ref, mag, case.k)
        assert res["ok_north_star"], (i, res)


def test_tf32_no_alloc_split_tiles(cuda, tf32_handle):
    """The TF32 lane through sgblasSgemmNoAlloc on shapes whose schedule
    splits tiles into k pieces, so the pieces and their arrival counters live
    in the fixed scratch: two calls in a row (the second reuses the counters
    the first left), each equal to sgblasSgemm on the same TF32 handle and
    within the TF32 bound."""
    torch = cuda
    f = ctypes.c_float
    for m, n, k in ((128, 128, 65536), (640, 520, 4100)):
        case = C.Case("tf32-noalloc-split", 0, 0, m, n, k, m, k, m, 1.0, 0.5)
        a, b, c = C.cfg_inputs(case, 19, None)
        status, want = run_sgemm(torch, tf32_handle, case, a, b, c)
        assert status == 0
        check_tf32(case, a, b, c, want, "sgemm")
        da, pa = to_device(torch, a)
        db, pb = to_device(torch, b)
        for call in range(2):
            dc, pc = to_device(torch, c)
            st = sg.lib.sgblasSgemmNoAlloc(tf32_handle.raw, 0, 0, m, n, k, ctypes.byref(f(1.0)),
                                           pa, m, pb, k, ctypes.byref(f(0.5)), pc, m)
            torch.cuda.synchronize()
            assert st == 0
            check_guards(da, db, dc)
            got = dc.cpu().numpy()
            check_tf32(case, a, b, c, got, f"noalloc call {call}")
            assert np.array_equal(got, want), (m, n, k, call)
    assert sg.get_device_errors() == 0


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_tf32_wide_tiles(cuda, tf32_handle, ta, tb):
    """2048 x 2048: 128 single-CTA 256-wide tiles for 148 SMs (fewer pair
    tiles than pairs, too many tiles for the 128-wide kernel); sampled."""
    m, n, k = 2048, 2048, 96
    lda, ldb = (k if ta else m), (n if tb else k)
    case = C.Case("tf32-wide", ta, tb, m, n, k, lda, ldb, m, 0.5, 2.0)
    a, b, c = C.cfg_inputs(case, 17, None)
    status, out = run_sgemm(cuda, tf32_handle, case, a, b, c)
    assert status == 0
    rng = np.random.default_rng(ta * 2 + tb)
    rows = np.concatenate([rng.integers(0, m, 4096), np.arange(0, m, 128), np.arange(127, m, 128)])
    cols = np.concatenate([rng.integers(0, n, 4096), rng.integers(0, n, 2 * (m // 128))])
    ref, mag = oracle.sgemm_f64_points(ta, tb, k, 0.5, a, lda, b, ldb, 2.0, c, m, rows, cols)
    got = out[rows + cols * m].astype(np.float64)
    assert np.all(np.abs(got - ref) <= tol_tf32(k, mag))
    assert np.all(np.isfinite(out))


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_tf32_pair_cta_tiles(cuda, tf32_handle, ta, tb):
    """9472 x 512: exactly one wave of 256 x 256 tiles over the 74 CTA pairs,
    so the cta_group::2 kernel runs; integer inputs make the TF32 products
    exact, so C must equal the FP64 reference exactly, then a random case is
    sampled against the TF32 bound."""
    torch = cuda
    m, n, k = 9472, 512, 96
    lda, ldb = (k if ta else m), (n if tb else k)
    rng = np.random.default_rng(40 + 2 * ta + tb)
    a = rng.integers(-3, 4, lda * (m if ta else k)).astype(np.float32)
    b = rng.integers(-3, 4, ldb * (k if tb else n)).astype(np.float32)
    case = C.Case("tf32-pair", ta, tb, m, n, k, lda, ldb, m, 1.0, 0.0)
    c = np.full(m * n, np.nan, np.float32)
    status, out = run_sgemm(torch, tf32_handle, case, a, b, c)
    assert status == 0
    ref, _ = oracle.sgemm_f64(ta, tb, m, n, k, 1.0, a, lda, b, ldb, 0.0, c, m)
    assert np.array_equal(c_view(out, m, n, m).astype(np.float64), ref)
    case = C.Case("tf32-pair-rand", ta, tb, m, n, k, lda, ldb, m + 4, -0.5, 1.5)
    a, b, c = C.cfg_inputs(case, 41, None)
    status, out = run_sgemm(torch, tf32_handle, case, a, b, c)
    assert status == 0
    rows = np.concatenate([rng.integers(0, m, 4096), np.arange(0, m, 256), np.arange(255, m, 256)])
    cols = np.concatenate([rng.integers(0, n, 4096), rng.integers(0, n, 2 * (m // 256))])
    ref, mag = oracle.sgemm_f64_points(ta, tb, k, -0.5, a, lda, b, ldb, 1.5, c, m + 4, rows, cols)
    got = out[rows + cols * (m + 4)].astype(np.float64)
    assert np.all(np.abs(got - ref) <= tol_tf32(k, mag))
    assert sg.get_device_errors() == 0


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_tf32_pair_cta_stream_k(cuda, tf32_handle, ta, tb):
    """4096 x 4096 x 3072: 256 pair tiles are 3.46 waves of 74 pairs and deep
    enough (96 slices of 32) for the last wave to be split by k over all
    pairs (each CTA publishes and sums its half); integer inputs: exact."""
    torch = cuda
    m, n, k = 4096, 4096, 3072
    lda, ldb = (k if ta else m), (n if tb else k)
    rng = np.random.default_rng(60 + 2 * ta + tb)
    a = rng.integers(-2, 3, lda * (m if ta else k)).astype(np.float32)
    b = rng.integers(-2, 3, ldb * (k if tb else n)).astype(np.float32)
    c = rng.integers(-2, 3, m * n).astype(np.float32)
    case = C.Case("tf32-pair-sk", ta, tb, m, n, k, lda, ldb, m, 1.0, 1.0)
    status, out = run_sgemm(torch, tf32_handle, case, a, b, c)
    assert status == 0
    rows = np.concatenate([rng.integers(0, m, 8192), np.arange(0, m, 64)])
    cols = np.concatenate([rng.integers(0, n, 8192), rng.integers(0, n, m // 64)])
    ref, _ = oracle.sgemm_f64_points(ta, tb, k, 1.0, a, lda, b, ldb, 1.0, c, m, rows, cols)
    assert np.array_equal(out[rows + cols * m].astype(np.float64), ref)
    assert sg.get_device_errors() == 0


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_tf32_small_deep_k_pieces(cuda, tf32_handle, ta, tb):
    """640 x 520 x 4100: 25 single-CTA tiles of 128 x 128 with 129 k slices,
    each tile split into pieces of at least 1024 k that meet in the
    workspace (ragged last tile row and column, k tail); integer inputs make
    the result exact, then a random case is checked against the TF32 bound."""
    torch = cuda
    m, n, k = 640, 520, 4100
    lda, ldb = (k if ta else m), (n if tb else k)
    rng = np.random.default_rng(80 + 2 * ta + tb)
    a = rng.integers(-2, 3, lda * (m if ta else k)).astype(np.float32)
    b = rng.integers(-2, 3, ldb * (k if tb else n)).astype(np.float32)
    case = C.Case("tf32-deep", ta, tb, m, n, k, lda, ldb, m, 1.0, 0.0)
    c = np.full(m * n, np.nan, np.float32)
    status, out = run_sgemm(torch, tf32_handle, case, a, b, c)
    assert status == 0
    ref, _ = oracle.sgemm_f64(ta, tb, m, n, k, 1.0, a, lda, b, ldb, 0.0, c, m)
    assert np.array_equal(c_view(out, m, n, m).astype(np.float64), ref)
    case = C.Case("tf32-deep-rand", ta, tb, m, n, k, lda, ldb, m + 2, 0.75, -0.5)
    a, b, c = C.cfg_inputs(case, 81, None)
    status, out = run_sgemm(torch, tf32_handle, case, a, b, c)
    assert status == 0
    check_tf32(case, a, b, c, out, (ta, tb))
    assert sg.get_device_errors() == 0


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k,count", [(300, 200, 70, 3), (1024, 1024, 96, 5)])
def test_tf32_strided_batched(cuda, tf32_handle, ta, tb, m, n, k, count):
    """Strided batches on the tensor cores (3-D tensor maps, batch-major
    tiles): single-CTA tiles for the small batch, pair-CTA tiles for the
    larger one. Integer inputs: every matrix exact."""
    torch = cuda
    lda, ldb, ldc = (k if ta else m) + 4, (n if tb else k) + 4, m + 2
    sa = lda * (m if ta else k) + 8
    sb = ldb * (k if tb else n) + 4
    sc = ldc * n + 12
    rng = np.random.default_rng(80 + m + 2 * ta + tb)
    a = rng.integers(-2, 3, sa * count).astype(np.float32)
    b = rng.integers(-2, 3, sb * count).astype(np.float32)
    c = np.full(sc * count, np.nan, np.float32)
    da = torch.from_numpy(a).cuda()
    db = torch.from_numpy(b).cuda()
    dc = torch.from_numpy(c).cuda()
    tf32_handle.sgemm_strided_batched(ta, tb, m, n, k, 1.0, da, lda, sa, db, ldb, sb, 0.0, dc,
                                      ldc, sc, count)
    torch.cuda.synchronize()
    out = dc.cpu().numpy()
    for i in range(count):
        ref, _ = oracle.sgemm_f64(ta, tb, m, n, k, 1.0, a[i * sa:(i + 1) * sa], lda,
                                  b[i * sb:(i + 1) * sb], ldb, 0.0, c[i * sc:(i + 1) * sc], ldc)
        got = c_view(out[i * sc:i * sc + ldc * n], m, n, ldc).astype(np.float64)
        assert np.array_equal(got, ref), (i, ta, tb, m)
    assert sg.get_device_errors() == 0
