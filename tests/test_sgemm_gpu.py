"""GPU parity of sgblasSgemm (through the C ABI) against the CPU oracle.

Covers the reference's whole device correctness suite with its exact inputs
(tests/cuda/correctness.cu:450-647 of AG0708/sgBLAS: 11 products, 3 scale
cases, 10 null-pointer no-ops), the BASELINE configurations, every loader path
(TMA and cp.async) in every transpose mode with tails, odd leading dimensions
and misaligned pointers, and run-to-run determinism.

Bounds: every checked entry must satisfy the north-star bound
|C - C_ref| <= 2*max(K,2)*2^-24*(|alpha| sum|a b| + |beta c|) (and therefore the
reference's looser 2e-6 + 8*eps*(K+1)*max(mag,1)); padding rows [m, ldc) must
be bit-identical; beta == 0 must overwrite NaN-poisoned C.
"""
import numpy as np
import pytest

import oracle
import sgblas_b200 as sg
from tests import cases as C
from tests.gpu_util import c_view, check_full, check_guards, check_sampled, run_sgemm, to_device

pytestmark = pytest.mark.gpu


def _assert(res, name):
    assert res["ok_north_star"] and res["ok_reference"], (name, res)
    if "padding_ok" in res:
        assert res["padding_ok"], (name, "padding overwritten")


# ---- the reference suite, with its exact inputs -------------------------------
def test_reference_suite(cuda, handle):
    torch = cuda
    stream = torch.cuda.Stream()   # the suite runs on a non-default stream
    for item in C.reference_suite():
        if item[0] == "scale":
            _, name, k, alpha, beta, c0 = item
            case = C.Case(name, 0, 0, 7, 5, k, 11, max(1, k + 3), 10, alpha, beta)
            status, out = run_sgemm(torch, handle, case, np.zeros(1, np.float32),
                                    np.zeros(1, np.float32), c0, stream=stream)
            assert status == 0, name
            want = np.zeros((7, 5)) if beta == 0 else beta * c0.reshape(5, 10).T[:7, :].astype(np.float64)
            got = out.reshape(5, 10).T[:7, :]
            assert np.all(np.isfinite(got))
            assert np.all(np.abs(got - want) <= 2 * 2.0 ** -23 * np.maximum(np.abs(want), 1.0)), name
            assert np.array_equal(out.reshape(5, 10).T[7:, :], c0.reshape(5, 10).T[7:, :]), name
        else:
            _, case, a, b, c0 = item
            status, out = run_sgemm(torch, handle, case, a, b, c0, stream=stream)
            assert status == 0, case.name
            _assert(check_full(case, a, b, c0, out), case.name)
    assert sg.get_device_errors() == 0


def test_null_pointer_noops_never_touch_memory(cuda, handle):
    torch = cuda
    for ta in (0, 1):
        for tb in (0, 1):
            for m, n in ((0, 7), (7, 0)):
                k = 5
                lda = max(1, m if ta == 0 else k)
                ldb = max(1, k if tb == 0 else n)
                assert handle.sgemm_status(ta, tb, m, n, k, None, None, lda, None, ldb, None, None,
                                           max(1, m)) == 0
    assert handle.sgemm_status(0, 0, 7, 5, 9, 0.0, None, 7, None, 9, 1.0, None, 7) == 0
    assert handle.sgemm_status(0, 0, 7, 5, 0, 2.0, None, 7, None, 1, 1.0, None, 7) == 0
    torch.cuda.synchronize()   # an accidental launch on NULL would fault here


# ---- BASELINE configurations --------------------------------------------------
def test_cfg1_256_full(cuda, handle):
    case = C.cfg1()
    a, b, c = C.cfg_inputs(case, 0, -1)
    status, out = run_sgemm(cuda, handle, case, a, b, c)
    assert status == 0
    _assert(check_full(case, a, b, c, out), case.name)


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_cfg3_transpose_tail_sweep(cuda, handle, ta, tb):
    torch = cuda
    case = C.cfg3(ta, tb)
    a, b, c = C.cfg_inputs(case, 3, None, normal=True)
    stream = torch.cuda.Stream()
    status, out = run_sgemm(torch, handle, case, a, b, c, stream=stream)
    assert status == 0
    _assert(check_full(case, a, b, c, out), case.name)


@pytest.mark.parametrize("size", [4096, 8192])
def test_cfg2_large_square(cuda, handle, size):
    case = C.cfg2(size)
    a, b, c = C.cfg_inputs(case, 1, 2)
    status, out = run_sgemm(cuda, handle, case, a, b, c)
    assert status == 0
    res = check_sampled(case, a, b, c, out)
    assert res["all_finite"]
    _assert(res, case.name)


@pytest.mark.parametrize("shape", C.CFG4_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_cfg4_medium_skinny(cuda, handle, shape):
    case = C.cfg4(*shape)
    a, b, c = C.cfg_inputs(case, 4, None)
    status, out = run_sgemm(cuda, handle, case, a, b, c)
    assert status == 0
    res = check_sampled(case, a, b, c, out)
    assert res["all_finite"]
    _assert(res, case.name)


# ---- loader paths, tails, leading dimensions, alignment -----------------------
# The first five shapes run on the small-problem cluster kernel, the last four
# (more than 37 tiles of 128 x 128) on the persistent tile kernel's loaders.
PATH_SHAPES = ((300, 200, 70), (257, 129, 33), (1, 1, 1), (5, 300, 17), (511, 3, 1),
               (1300, 1000, 70), (1029, 1157, 33), (1, 9000, 17), (9001, 3, 1))
PATH_CASES = []
for ta in (0, 1):
    for tb in (0, 1):
        for (m, n, k) in PATH_SHAPES:
            for pad, offs in ((0, (0, 0, 0)), (4, (0, 0, 0)), (1, (0, 0, 0)), (0, (1, 2, 3))):
                PATH_CASES.append((ta, tb, m, n, k, pad, offs))


@pytest.mark.parametrize("ta,tb,m,n,k,pad,offs", PATH_CASES)
def test_paths_tails_alignment(cuda, handle, ta, tb, m, n, k, pad, offs):
    lda = (k if ta else m) + pad
    ldb = (n if tb else k) + pad
    ldc = m + (pad or 1)
    for alpha, beta in ((1.0, 0.0), (-0.5, 1.0), (0.75, -1.25)):
        case = C.Case("path", ta, tb, m, n, k, lda, ldb, ldc, alpha, beta)
        a, b, c = C.cfg_inputs(case, 100 + m + n + k, None)
        C.pad_and_poison(c, m, n, ldc, beta, C.PRODUCT_PAD)
        status, out = run_sgemm(cuda, handle, case, a, b, c, offsets=offs)
        assert status == 0
        _assert(check_full(case, a, b, c, out), (ta, tb, m, n, k, pad, offs, alpha, beta))


# Without a workspace (sgblasSgemmNoAlloc) an operand TMA cannot read is
# staged by the tile kernel's cp.async producer in 4-, 8- or 16-byte copies
# instead of being copied into the workspace first: cover those paths too
# (shapes large enough for the tile kernel).
COPY_CASES = []
for ta in (0, 1):
    for tb in (0, 1):
        for (m, n, k) in ((1300, 1000, 70), (1029, 1157, 33), (5, 9000, 17)):
            for pad, offs in ((1, (0, 0, 0)), (2, (0, 0, 0)), (0, (1, 2, 3)), (4, (2, 0, 1))):
                COPY_CASES.append((ta, tb, m, n, k, pad, offs))


@pytest.mark.parametrize("ta,tb,m,n,k,pad,offs", COPY_CASES)
def test_copy_staging_without_workspace(cuda, handle, ta, tb, m, n, k, pad, offs):
    import ctypes
    torch = cuda
    lda = (k if ta else m) + pad
    ldb = (n if tb else k) + pad
    ldc = m + (pad or 1)
    f = ctypes.c_float
    for alpha, beta in ((1.0, 0.0), (0.75, -1.25)):
        case = C.Case("copy", ta, tb, m, n, k, lda, ldb, ldc, alpha, beta)
        a, b, c = C.cfg_inputs(case, 300 + m + n + k, None)
        C.pad_and_poison(c, m, n, ldc, beta, C.PRODUCT_PAD)
        da, pa = to_device(torch, a, offs[0])
        db, pb = to_device(torch, b, offs[1])
        dc, pc = to_device(torch, c, offs[2])
        status = sg.lib.sgblasSgemmNoAlloc(handle.raw, ta, tb, m, n, k, ctypes.byref(f(alpha)), pa,
                                           lda, pb, ldb, ctypes.byref(f(beta)), pc, ldc)
        torch.cuda.synchronize()
        assert status == 0
        check_guards(da, db, dc)
        out = dc[offs[2]:].cpu().numpy()
        _assert(check_full(case, a, b, c, out), (ta, tb, m, n, k, pad, offs, alpha, beta))
    assert sg.get_device_errors() == 0


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("pad", [1, 2, 3])
def test_packed_operands_large(cuda, handle, ta, tb, pad):
    # Odd or 8-byte leading dimensions on a multi-tile problem: both operands
    # go through the workspace copies (transposing the k-contiguous ones).
    m, n, k = 1023, 1537, 777
    case = C.Case("packed", ta, tb, m, n, k, (k if ta else m) + pad, (n if tb else k) + pad,
                  m + pad, 1.5, -0.5)
    a, b, c = C.cfg_inputs(case, 900 + pad, None)
    status, out = run_sgemm(cuda, handle, case, a, b, c)
    assert status == 0
    _assert(check_full(case, a, b, c, out), (ta, tb, pad))


def test_deterministic(cuda, handle):
    case = C.cfg3(0, 0)
    a, b, c = C.cfg_inputs(case, 3, None, normal=True)
    _, out1 = run_sgemm(cuda, handle, case, a, b, c)
    _, out2 = run_sgemm(cuda, handle, case, a, b, c)
    assert np.array_equal(out1, out2, equal_nan=True)


# ---- parity with the reference library itself ---------------------------------
def test_parity_with_reference_library(cuda, handle):
    """Both libraries on identical buffers: each within the bound of the FP64
    oracle, hence within twice the bound of each other."""
    import oracle
    try:
        ref = oracle.RefLib()
    except (FileNotFoundError, OSError) as e:
        pytest.skip(f"reference library unavailable: {e}")
    torch = cuda
    shapes = [C.cfg3(0, 0), C.cfg3(0, 1), C.cfg3(1, 0), C.cfg3(1, 1),
              C.Case("768x768x128", 0, 0, 768, 768, 128, 768, 128, 768, -0.375, 0.625),
              C.Case("1024x2048x64", 0, 0, 1024, 2048, 64, 1024, 64, 1024, 0.625, -0.375)]
    for case in shapes:
        a, b, c = C.cfg_inputs(case, 3, None, normal=True)
        da, pa = to_device(torch, a)
        db, pb = to_device(torch, b)
        dc_ref, pc_ref = to_device(torch, c)
        assert ref.sgemm(case.transa, case.transb, case.m, case.n, case.k, case.alpha, pa,
                         case.lda, pb, case.ldb, case.beta, pc_ref, case.ldc) == 0
        torch.cuda.synchronize()
        out_ref = dc_ref.cpu().numpy()
        status, out = run_sgemm(torch, handle, case, a, b, c)
        assert status == 0
        r_ref = check_full(case, a, b, c, out_ref)
        r_us = check_full(case, a, b, c, out)
        assert r_ref["ok_north_star"], ("reference outside the bound?", case.name, r_ref)
        _assert(r_us, case.name)
    ref.close()


# ---- the persistent stream-K schedule -----------------------------------------
# (m, n, k): one tile split over every SM; fewer tiles than SMs; a remainder
# wave after whole waves; odd tails with many pieces per tile; K below the
# split threshold.
SK_SHAPES = [(256, 128, 65536), (512, 512, 4096), (1500, 1300, 3000), (2560, 1920, 1024),
             (4096, 2048, 512), (300, 700, 100), (9472, 512, 384)]


@pytest.mark.parametrize("m,n,k", SK_SHAPES)
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 1)])
def test_stream_k_shapes(cuda, handle, m, n, k, ta, tb):
    lda = k if ta else m
    ldb = n if tb else k
    case = C.Case("sk", ta, tb, m, n, k, lda, ldb, m, 0.5, -1.5)
    a, b, c = C.cfg_inputs(case, m + n + k, None)
    status, out = run_sgemm(cuda, handle, case, a, b, c)
    assert status == 0
    if m * n * k <= (1 << 31):
        _assert(check_full(case, a, b, c, out), (m, n, k))
    else:
        _assert(check_sampled(case, a, b, c, out), (m, n, k))


# Thin edge tiles under stream-K: n % 128 of 1, 20, 64 and 65 leave a last
# tile column that is mostly outside C; m % 128 == 1 puts the thin edge on the
# other side of C. Operands are copied (ld % 4 != 0) or read in place.
THIN_SHAPES = [(896, 2049, 333), (1000, 1300, 2000), (1024, 1088, 640), (640, 1089, 1500),
               (1025, 1024, 900)]


@pytest.mark.parametrize("m,n,k", THIN_SHAPES)
@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 1)])
def test_thin_edge_tiles(cuda, handle, m, n, k, ta, tb):
    lda = (k if ta else m) + 3
    ldb = (n if tb else k) + 4
    case = C.Case("thin", ta, tb, m, n, k, lda, ldb, m + 1, 1.5, -0.5)
    a, b, c = C.cfg_inputs(case, m + 2 * n + k, None, normal=True)
    status, out = run_sgemm(cuda, handle, case, a, b, c)
    assert status == 0
    _assert(check_full(case, a, b, c, out), (m, n, k, ta, tb))


# ---- transpose-free copies of k-contiguous operands --------------------------
# Both sides of C at least 3072 long: in a large FP32 product a k-contiguous
# operand that TMA could read in place (A in TN/TT, B in NN/TN) is copied into
# the workspace first, so that the kernel needs no transposes. Every entry
# against the oracle, with padded leading dimensions and beta != 0.
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_transpose_free_copies(cuda, handle, ta, tb):
    m, n, k = 3100, 3072, 700
    lda = (k if ta else m) + 4
    ldb = (n if tb else k) + 8
    case = C.Case("copy-large", ta, tb, m, n, k, lda, ldb, m + 4, 0.75, -0.5)
    a, b, c = C.cfg_inputs(case, 17 + 2 * ta + tb, None, normal=True)
    status, out = run_sgemm(cuda, handle, case, a, b, c)
    assert status == 0
    _assert(check_full(case, a, b, c, out), (ta, tb))


# ---- stage refills behind a slow epilogue ---------------------------------------
@pytest.mark.parametrize("ta,tb", [(0, 1), (0, 0)])
@pytest.mark.parametrize("beta", [1.0, 0.5])
def test_stage_refill_after_slow_epilogue(cuda, handle, ta, tb, beta):
    """A TMA refill of a pipeline stage must not land while a compute warp still
    reads the stage's previous contents. 8192 x 8192 x 256 with beta != 0 has 16
    k-iterations per tile and a 256 MiB C (larger than L2): every tile's epilogue
    reads C from HBM, the compute warps fall behind the producer and drift apart.
    Before the cross-proxy fence between the empty-barrier hand-off and the TMA
    refill, about half of such calls returned one to three tiles with a few
    k-terms wrong. Three calls each, every entry against an FP64 product on the
    GPU (a sampled check would miss a single bad tile most of the time)."""
    torch = cuda
    m = n = 8192
    k = 256
    g = torch.Generator(device="cuda")
    g.manual_seed(11 + 2 * ta + tb)
    a = torch.rand(m * k, device="cuda", generator=g) * 2 - 1
    b = torch.rand(k * n, device="cuda", generator=g) * 2 - 1
    c = torch.rand(m * n, device="cuda", generator=g) * 2 - 1
    lda, ldb = (k if ta else m), (n if tb else k)
    op_a = (a.view(m, k) if ta else a.view(k, m).T).double()
    op_b = (b.view(k, n) if tb else b.view(n, k).T).double()
    c0 = c.view(n, m).T.double()
    ref = op_a @ op_b + beta * c0
    bound = 2 * k * 2.0 ** -24 * (op_a.abs() @ op_b.abs() + abs(beta) * c0.abs())
    del op_a, op_b
    for call in range(3):
        out = c.clone()
        handle.sgemm(ta, tb, m, n, k, 1.0, a, lda, b, ldb, beta, out, m)
        torch.cuda.synchronize()
        bad = int(((out.view(n, m).T.double() - ref).abs() > bound).sum())
        assert bad == 0, (ta, tb, beta, call, bad)
    assert sg.get_device_errors() == 0


def test_workspace_shared_across_streams(cuda, handle):
    """One handle alternating between two streams with no host sync between
    calls: the workspace is ordered by an event, results are bit-identical to
    a single-stream run."""
    torch = cuda
    case = C.Case("sk", 0, 0, 1500, 1300, 3000, 1500, 3000, 1500, 1.0, 0.0)
    a, b, c = C.cfg_inputs(case, 77, None)
    _, expect = run_sgemm(torch, handle, case, a, b, c)
    da, pa = to_device(torch, a)
    db, pb = to_device(torch, b)
    outs = [torch.zeros(case.c_size, device="cuda") for _ in range(6)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        handle.set_stream(streams[i % 2])
        handle.sgemm(0, 0, case.m, case.n, case.k, 1.0, pa, case.lda, pb, case.ldb, 0.0, o,
                     case.ldc)
    torch.cuda.synchronize()
    handle.set_stream(None)
    for o in outs:
        assert np.array_equal(o.cpu().numpy(), expect)
    assert sg.get_device_errors() == 0


def test_one_handle_many_stream_k_shapes(cuda, handle):
    """One handle, successive problems whose stream-K schedules split
    different numbers of tiles: the workspace layout must not move between
    calls (counters zeroed by one launch stay zero for the next)."""
    torch = cuda
    shapes = [(1500, 1300, 3000), (4096, 2048, 512), (512, 512, 4096), (4096, 2048, 512),
              (1500, 1300, 3000)]
    for i, (m, n, k) in enumerate(shapes):
        case = C.Case("reuse", 0, 1, m, n, k, m, n, m, 1.0, 0.0)
        a, b, c = C.cfg_inputs(case, 900 + i, None)
        status, out = run_sgemm(torch, handle, case, a, b, c)
        assert status == 0
        _assert(check_sampled(case, a, b, c, out, count=8192, seed=i), (i, m, n, k))


def test_split_products_exact_after_interrupted_launch(cuda, handle):
    """A split launch that stops early (a bounded wait that timed out) leaves
    its arrival counters part-counted. sgblasTestInterruptScratch puts the
    handle's counters in exactly that state; the next split product on the
    same handle -- FP32 tile kernel, cluster kernel with several clusters
    per tile, TF32 lane -- must still be exact and bit-identical to the
    product before it. Then a captured graph of a split product is replayed
    three times (each replay reuses one epoch; the last arrival of each tile
    resets its counter)."""
    import ctypes
    torch = cuda
    shapes = [("fp32", 1500, 1300, 3000), ("fp32", 128, 128, 8192), ("tf32", 1024, 1024, 4096)]
    try:
        for math, m, n, k in shapes:
            handle.set_math_mode(sg.SGBLAS_MATH_TF32 if math == "tf32" else sg.SGBLAS_MATH_FP32)
            case = C.Case("interrupt", 0, 0, m, n, k, m, k, m, 1.0, 0.5)
            a, b, c = C.cfg_inputs(case, 313, None)
            status, first = run_sgemm(torch, handle, case, a, b, c)
            assert status == 0
            assert sg.lib.sgblasTestInterruptScratch(handle.raw) == 0
            status, again = run_sgemm(torch, handle, case, a, b, c)
            assert status == 0
            assert np.array_equal(first, again), (math, m, n, k)
            if math == "fp32":
                _assert(check_sampled(case, a, b, c, again, count=8192), (m, n, k))
    finally:
        handle.set_math_mode(sg.SGBLAS_MATH_FP32)
    case = C.Case("graph-sk", 0, 0, 1500, 1300, 3000, 1500, 3000, 1500, 1.0, 0.0)
    a, b, c = C.cfg_inputs(case, 314, None)
    _, expect = run_sgemm(torch, handle, case, a, b, c)
    da, pa = to_device(torch, a)
    db, pb = to_device(torch, b)
    dc, pc = to_device(torch, c)
    stream = torch.cuda.Stream()
    handle.set_stream(stream)
    try:
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            handle.sgemm(0, 0, case.m, case.n, case.k, 1.0, pa, case.lda, pb, case.ldb, 0.0, pc,
                         case.ldc)
        for _ in range(3):
            dc.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            assert np.array_equal(dc.cpu().numpy(), expect)
        del graph
    finally:
        handle.set_stream(None)
    assert sg.get_device_errors() == 0


def test_handle_moves_between_devices(cuda, handle):
    """One handle used on device 0, 1, 0, 1 in turn with a product that needs
    the workspace: each move frees the old workspace on its own device,
    stream-ordered (no host synchronization), and allocates a new one; every
    result matches the oracle. Needs 2 GPUs."""
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    case = C.Case("move", 0, 0, 1500, 1300, 3000, 1500, 3000, 1500, 1.0, 0.0)
    a, b, c = C.cfg_inputs(case, 71, None)
    try:
        for dev in (0, 1, 0, 1):
            torch.cuda.set_device(dev)
            status, out = run_sgemm(torch, handle, case, a, b, c)
            assert status == 0, dev
            _assert(check_sampled(case, a, b, c, out, count=4096, seed=dev), ("device", dev))
            assert sg.get_device_errors() == 0
    finally:
        torch.cuda.set_device(0)


def test_matches_reference_golden_outputs(cuda, handle):
    """Our outputs at the entries the reference library produced on a B200
    (tests/golden/reference_suite.npz): both lie within the north-star bound
    of the FP64 oracle, so they agree to within twice that bound."""
    import pathlib

    import oracle
    from tests.golden.make_golden import golden_cases
    gold = np.load(pathlib.Path(__file__).resolve().parent / "golden" / "reference_suite.npz")
    for case, a, b, c in golden_cases():
        rows, cols = gold[f"{case.name}/rows"], gold[f"{case.name}/cols"]
        theirs = gold[f"{case.name}/vals"].astype(np.float64)
        status, out = run_sgemm(cuda, handle, case, a, b, c)
        assert status == 0
        ours = out[rows.astype(np.int64) + cols.astype(np.int64) * case.ldc].astype(np.float64)
        _, mag = oracle.sgemm_f64_points(case.transa, case.transb, case.k, case.alpha, a,
                                         case.lda, b, case.ldb, case.beta, c, case.ldc, rows, cols)
        assert np.all(np.abs(ours - theirs) <= 2 * oracle.tol_north_star(case.k, mag)), case.name


# ---- failure detection: bounded waits ------------------------------------------
def test_bounded_wait_times_out_and_reports(cuda):
    """A wait on a barrier nothing completes gives up, raises the device error
    flag and returns; the context stays usable (an SGEMM right after is exact)."""
    import ctypes
    assert sg.get_device_errors(clear=True) == 0
    timed_out = ctypes.c_int(-1)
    assert sg.lib.sgblasSelfTestWaitTimeout(2000, ctypes.byref(timed_out)) == 0
    assert timed_out.value == 1
    assert sg.get_device_errors(clear=True) & 1
    assert sg.get_device_errors(clear=True) == 0
    with sg.Handle() as h:
        case = C.cfg1()
        a, b, c = C.cfg_inputs(case, 0, -1)
        status, out = run_sgemm(cuda, h, case, a, b, c)
        assert status == 0
        _assert(check_full(case, a, b, c, out), "after timeout")


# ---- the reference's own benchmark, built against this library -----------------
def test_reference_benchmark_runs_against_product(cuda):
    """bench/benchmark.cu of the reference, compiled unchanged against this
    repository's header and libsgblas.so (oracle/Makefile), runs a shape and
    emits its JSONL evidence schema (metadata + result records)."""
    import json
    import pathlib
    import subprocess
    exe = pathlib.Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "sgblas_benchmark_b200"
    if not exe.exists():
        pytest.skip("reference benchmark not built (make -C oracle ref)")
    run = subprocess.run([str(exe), "512", "384", "256", "--order", "sgblas-first", "--output",
                          "jsonl", "--warmups", "2", "--repeats", "5"], capture_output=True,
                         text=True, timeout=300)
    assert run.returncode == 0, run.stderr
    records = [json.loads(line) for line in run.stdout.splitlines() if line.startswith("{")]
    assert [r["record_type"] for r in records] == ["metadata", "result"]
    meta, res = records
    assert meta["schema_version"] == 1
    assert meta["benchmark"]["sgblas_math_mode"] == "SGBLAS_MATH_FP32"
    assert meta["device"]["compute_capability_major"] == 10
    assert (res["m"], res["n"], res["k"]) == (512, 384, 256)
    assert res["sgblas_gflops"] > 0 and res["cublas_gflops"] > 0 and res["ratio"] > 0


# ---- 64-bit addressing and grid limits ---------------------------------------
@pytest.mark.parametrize("math", ["fp32", "tf32"])
def test_huge_outputs(cuda, handle, math):
    """C with more than 2^31 elements (64-bit offsets in the epilogue), and n
    of five million columns (far past the 65535 grid-Y limit a 2-D launch of
    the reference has to work around); sampled against the oracle, including
    the last row and column."""
    torch = cuda
    handle.set_math_mode(sg.SGBLAS_MATH_TF32 if math == "tf32" else sg.SGBLAS_MATH_FP32)
    try:
        for (m, n, k) in ((50000, 44000, 4), (8, 5_000_000, 8)):
            rng = np.random.default_rng(m + n)
            a = rng.uniform(-1, 1, m * k).astype(np.float32)
            b = rng.uniform(-1, 1, k * n).astype(np.float32)
            da = torch.from_numpy(a).cuda()
            db = torch.from_numpy(b).cuda()
            dc = torch.full((m * n,), float("nan"), dtype=torch.float32, device="cuda")
            handle.sgemm(0, 0, m, n, k, 1.0, da, m, db, k, 0.0, dc, m)
            torch.cuda.synchronize()
            rows = np.concatenate([rng.integers(0, m, 4000), [0, m - 1, m - 1, 0]])
            cols = np.concatenate([rng.integers(0, n, 4000), [0, n - 1, 0, n - 1]])
            flat = torch.from_numpy(rows.astype(np.int64) + cols.astype(np.int64) * m).cuda()
            got = dc[flat].cpu().numpy().astype(np.float64)
            c0 = np.zeros(1, np.float32)
            ref, mag = oracle.sgemm_f64_points(0, 0, k, 1.0, a, m, b, k, 0.0, c0, m, rows, cols)
            tol = (2.0 ** -9 + (k + 2) * 2.0 ** -22) * mag if math == "tf32" else \
                oracle.tol_north_star(k, mag)
            assert np.all(np.abs(got - ref) <= tol), (m, n, k, math)
            assert not torch.isnan(dc).any().item(), (m, n, k, math)
            del dc
            torch.cuda.empty_cache()
    finally:
        handle.set_math_mode(sg.SGBLAS_MATH_FP32)
    assert sg.get_device_errors() == 0


def test_cuda_graph_capture_and_replay(cuda, handle):
    """After a first call has set up the workspace, products (FP32 with a
    stream-K split and an operand copy, and TF32) can be captured in a CUDA
    graph and replayed with new inputs."""
    torch = cuda
    stream = torch.cuda.Stream()
    handle.set_stream(stream)
    try:
        for math, (m, n, k, ldb_pad) in (("fp32", (1000, 700, 900, 1)), ("tf32", (512, 512, 512, 0))):
            handle.set_math_mode(sg.SGBLAS_MATH_TF32 if math == "tf32" else sg.SGBLAS_MATH_FP32)
            case = C.Case("graph", 0, 0, m, n, k, m, k + ldb_pad, m, 1.0, 0.0)
            a, b, c = C.cfg_inputs(case, 55, -1)
            da, pa = to_device(torch, a)
            db, pb = to_device(torch, b)
            dc, pc = to_device(torch, c)
            with torch.cuda.stream(stream):
                handle.sgemm(0, 0, m, n, k, 1.0, pa, case.lda, pb, case.ldb, 0.0, pc, m)  # set-up
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                handle.sgemm(0, 0, m, n, k, 1.0, pa, case.lda, pb, case.ldb, 0.0, pc, m)
            a2, b2, _ = C.cfg_inputs(case, 56, -1)
            da.copy_(torch.from_numpy(a2))
            db.copy_(torch.from_numpy(b2))
            dc.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            ref, mag = oracle.sgemm_f64(0, 0, m, n, k, 1.0, a2, case.lda, b2, case.ldb, 0.0, c, m)
            got = dc.cpu().numpy().reshape(n, m).T.astype(np.float64)
            bound = (2.0 ** -9 + (k + 2) * 2.0 ** -22) * mag if math == "tf32" else \
                oracle.tol_north_star(k, mag)
            assert np.all(np.abs(got - ref) <= bound), math
            del graph
    finally:
        handle.set_math_mode(sg.SGBLAS_MATH_FP32)
        handle.set_stream(None)
    assert sg.get_device_errors() == 0


def test_concurrent_handles_from_host_threads(cuda):
    """Four host threads, each with its own handle and stream, issue products
    concurrently (ctypes releases the GIL): stream-K splits, operand copies,
    both math modes. The lazily initialised per-device state (kernel
    attributes, tensor-map encoder, error word) must tolerate the race."""
    import threading
    torch = cuda
    shapes = [(1000, 700, 900, 0, "fp32"), (333, 444, 123, 1, "fp32"), (512, 512, 512, 0, "tf32"),
              (2048, 512, 256, 0, "fp32")]
    results = {}

    def worker(idx):
        try:
            m, n, k, pad, math = shapes[idx]
            with sg.Handle() as h:
                stream = torch.cuda.Stream()
                h.set_stream(stream)
                if math == "tf32":
                    h.set_math_mode(sg.SGBLAS_MATH_TF32)
                case = C.Case("threads", 0, 0, m, n, k, m + pad, k + pad, m, 1.0, 0.0)
                a, b, c = C.cfg_inputs(case, 70 + idx, -1)
                da, pa = to_device(torch, a)
                db, pb = to_device(torch, b)
                outs = []
                for rep in range(10):
                    dc, pc = to_device(torch, c)
                    with torch.cuda.stream(stream):
                        h.sgemm(0, 0, m, n, k, 1.0, pa, case.lda, pb, case.ldb, 0.0, pc, m)
                    outs.append(dc)
                stream.synchronize()
                results[idx] = (case, a, b, c, [o.cpu().numpy() for o in outs], math)
        except Exception as e:  # reported by the main thread
            results[idx] = e

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(len(shapes))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    for idx in range(len(shapes)):
        res = results.get(idx)
        assert not isinstance(res, Exception) and res is not None, (idx, res)
        case, a, b, c, outs, math = res
        ref, mag = oracle.sgemm_f64(0, 0, case.m, case.n, case.k, 1.0, a, case.lda, b, case.ldb,
                                    0.0, c, case.ldc)
        bound = (2.0 ** -9 + (case.k + 2) * 2.0 ** -22) * mag if math == "tf32" else \
            oracle.tol_north_star(case.k, mag)
        for out in outs:
            assert np.array_equal(out, outs[0]), (idx, "repeat differs")
            got = c_view(out, case.m, case.n, case.ldc).astype(np.float64)
            assert np.all(np.abs(got - ref) <= bound), (idx, math)
    assert sg.get_device_errors() == 0
