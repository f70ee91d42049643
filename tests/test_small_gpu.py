"""The small-problem cluster kernel (sgemm_small.cu) against the CPU oracle.

Shapes are chosen for each cluster size the launcher picks (1, 2, 4 and 8
CTAs splitting a tile's k range, including CTAs left without a k slice),
ragged m/n/k tails, every transpose mode, padded and odd leading dimensions,
misaligned base pointers, the three epilogue forms (beta 0 with NaN-poisoned
C, 1, general), batches, sgblasSgemmNoAlloc and CUDA graph capture on a
handle that has never allocated. Every entry of C is checked within the
north-star bound and padding rows must stay bit-identical.
"""
import ctypes

import numpy as np
import pytest

import oracle
import sgblas_b200 as sg
from tests import cases as C
from tests.gpu_util import check_full, check_guards, run_sgemm, to_device

pytestmark = pytest.mark.gpu

SMS_B200 = 148


def _plan_for(m, n, k, batch, sms, bm):
    tiles = -(-m // bm) * -(-n // 64) * batch
    slices = -(-k // 32)
    split = 1
    while split * 2 <= 8 and split * 2 <= slices and tiles * split * 2 <= sms:
        split *= 2
    slots = sms * (2 if bm == 64 else 1)   # resident CTAs: two 64-row CTAs per SM
    groups = 1
    if tiles * split * 2 <= slots:
        groups = max(1, min(slots // (tiles * split), slices // (split * 4)))
    return split, groups, -(-slices // (split * groups)), bm, tiles * split * groups


def _plan(m, n, k, batch=1, sms=SMS_B200):
    """The launcher's (cluster size, clusters per tile, slices per CTA, tile
    rows) on a GPU with `sms` SMs (sgemm_small.cu planSmall)."""
    tall = _plan_for(m, n, k, batch, sms, 128)
    if m > 64 and tall[4] * 2 > sms and tall[2] >= 4 and tall[0] <= 4:
        return tall[:4]
    return _plan_for(m, n, k, batch, sms, 64)[:4]


def _split(m, n, k, batch=1):
    return _plan(m, n, k, batch)[0]


# (m, n, k): cluster size and clusters per tile in the comment (148 SMs);
# 512^3 and 450 x 300 x 640 run on 128-row tiles
SHAPES = [(256, 256, 256),    # 8
          (512, 512, 512),    # 2
          (384, 384, 384),    # 4
          (700, 600, 50),     # 1 (110 tiles): launched without clusters
          (700, 600, 256),    # 2, 128-row tiles
          (64, 64, 150),      # 4: five slices, the last CTA has none
          (100, 37, 1000),    # 8, ragged tiles
          (65, 129, 33),      # 2 (two slices)
          (1, 1, 1),          # 1
          (3, 250, 7),        # 1
          (128, 128, 8192),   # 8 x 8 clusters per tile (two CTAs per SM)
          (64, 200, 3000),    # 8 x 2, ragged k and n
          (37, 19, 4111),     # 8 x 4, the last cluster's k range is short
          (500, 200, 1000),   # 4
          (450, 300, 640)]    # 4, 128-row tiles with ragged m and n


def _idle_cta(m, n, k):
    """True if some CTA gets no k slice."""
    split, groups, per_cta, _ = _plan(m, n, k)
    return (split * groups - 1) * per_cta >= -(-k // 32)


def test_shape_list_covers_every_cluster_size():
    plans = [_plan(*s) for s in SHAPES]
    assert {p[0] for p in plans} == {1, 2, 4, 8}
    assert {p[1] for p in plans} >= {1, 2, 4}
    assert {p[3] for p in plans} == {64, 128}
    assert any(_idle_cta(*s) for s in SHAPES)


def _assert(res, name):
    assert res["ok_north_star"] and res["ok_reference"], (name, res)
    assert res["padding_ok"], (name, "padding overwritten")


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_small_modes_and_tails(cuda, handle, m, n, k, ta, tb):
    for pad, offs in ((0, (0, 0, 0)), (1, (0, 0, 0)), (3, (1, 2, 3))):
        lda = (k if ta else m) + pad
        ldb = (n if tb else k) + pad
        ldc = m + (pad or 1)
        for alpha, beta in ((1.0, 0.0), (-0.5, 1.0), (0.75, -1.25)):
            case = C.Case("small", ta, tb, m, n, k, lda, ldb, ldc, alpha, beta)
            a, b, c = C.cfg_inputs(case, 40 + m + n + k + pad, None)
            C.pad_and_poison(c, m, n, ldc, beta, C.PRODUCT_PAD)
            status, out = run_sgemm(cuda, handle, case, a, b, c, offsets=offs)
            assert status == 0
            _assert(check_full(case, a, b, c, out), (ta, tb, m, n, k, pad, offs, alpha, beta))
    assert sg.get_device_errors() == 0


@pytest.mark.parametrize("m,n,k", [(256, 256, 256), (128, 128, 8192)])
def test_small_deterministic(cuda, handle, m, n, k):
    """Partial tiles are summed in rank order and then in cluster order,
    whatever order the clusters finish in: bit-identical reruns."""
    case = C.Case("det", 0, 0, m, n, k, m, k, m, 1.0, 0.0)
    a, b, c = C.cfg_inputs(case, 5, None)
    _, out1 = run_sgemm(cuda, handle, case, a, b, c)
    for _ in range(5):
        _, out2 = run_sgemm(cuda, handle, case, a, b, c)
        assert np.array_equal(out1, out2)


def test_small_no_alloc(cuda, handle):
    torch = cuda
    f = ctypes.c_float
    # the last two use the fixed scratch (several clusters per tile)
    for (m, n, k, pad) in ((256, 256, 256, 0), (100, 37, 1000, 1), (65, 129, 33, 3),
                           (128, 128, 8192, 0), (64, 200, 3000, 1)):
        case = C.Case("noalloc-small", 1, 0, m, n, k, k + pad, k + pad, m + 1, 0.5, 2.0)
        a, b, c = C.cfg_inputs(case, 600 + m, None)
        C.pad_and_poison(c, m, n, case.ldc, case.beta, C.PRODUCT_PAD)
        da, pa = to_device(torch, a)
        db, pb = to_device(torch, b, 1)
        dc, pc = to_device(torch, c)
        status = sg.lib.sgblasSgemmNoAlloc(handle.raw, 1, 0, m, n, k, ctypes.byref(f(case.alpha)),
                                           pa, case.lda, pb, case.ldb, ctypes.byref(f(case.beta)),
                                           pc, case.ldc)
        torch.cuda.synchronize()
        assert status == 0
        check_guards(da, db, dc)
        _assert(check_full(case, a, b, c, dc.cpu().numpy()), (m, n, k))
    assert sg.get_device_errors() == 0


def test_small_batched(cuda, handle):
    """Strided (odd strides: 4-byte staging) and pointer-array batches of
    small matrices; 6 x 2 x 2 tiles of 64 x 64 give clusters of 4."""
    torch = cuda
    count, m, n, k = 6, 100, 90, 200
    assert _plan(m, n, k, count)[:2] == (4, 1)
    case = C.Case("batch-small", 0, 1, m, n, k, m + 1, n + 2, m + 3, 1.5, -0.5)
    mats = []
    for i in range(count):
        a, b, c = C.cfg_inputs(case, 70 + i, None)
        mats.append((a, b, c))
    sa, sb, sc = case.a_size + 3, case.b_size + 1, case.c_size + 5
    host = {key: np.zeros(size * count, np.float32) for key, size in (("a", sa), ("b", sb), ("c", sc))}
    for i, (a, b, c) in enumerate(mats):
        host["a"][i * sa:i * sa + a.size] = a
        host["b"][i * sb:i * sb + b.size] = b
        host["c"][i * sc:i * sc + c.size] = c
    dev = {key: torch.from_numpy(v).cuda() for key, v in host.items()}
    handle.sgemm_strided_batched(0, 1, m, n, k, case.alpha, dev["a"].data_ptr(), case.lda, sa,
                                 dev["b"].data_ptr(), case.ldb, sb, case.beta,
                                 dev["c"].data_ptr(), case.ldc, sc, count)
    torch.cuda.synchronize()
    out = dev["c"].cpu().numpy()
    for i, (a, b, c) in enumerate(mats):
        res = check_full(case, a, b, c, out[i * sc:i * sc + case.c_size])
        _assert(res, ("strided", i))
    # The same products through pointer arrays, in reverse order.
    dev_c2 = torch.from_numpy(host["c"]).cuda()
    arrays = [torch.tensor([base.data_ptr() + 4 * i * s for i in reversed(range(count))],
                           dtype=torch.int64, device="cuda")
              for base, s in ((dev["a"], sa), (dev["b"], sb), (dev_c2, sc))]
    handle.sgemm_batched(0, 1, m, n, k, case.alpha, arrays[0], case.lda, arrays[1], case.ldb,
                         case.beta, arrays[2], case.ldc, count)
    torch.cuda.synchronize()
    out2 = dev_c2.cpu().numpy()
    assert np.array_equal(out2, out)
    assert sg.get_device_errors() == 0


@pytest.mark.parametrize("m,n,k", [(256, 192, 320), (128, 128, 8192)])
def test_small_graph_capture_on_fresh_handle(cuda, m, n, k):
    """The cluster kernel needs no workspace (with several clusters per tile
    it falls back to one while capturing): the very first call of a new
    handle can be captured into a CUDA graph and replayed."""
    torch = cuda
    with sg.Handle() as h:
        stream = torch.cuda.Stream()
        h.set_stream(stream)
        case = C.Case("graph-small", 0, 0, m, n, k, m, k, m, 1.0, 0.0)
        a, b, c = C.cfg_inputs(case, 8, -1)
        da, pa = to_device(torch, a)
        db, pb = to_device(torch, b)
        dc, pc = to_device(torch, c)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            h.sgemm(0, 0, m, n, k, 1.0, pa, m, pb, k, 0.0, pc, m)
        dc.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        ref, mag = oracle.sgemm_f64(0, 0, m, n, k, 1.0, a, m, b, k, 0.0, c, m)
        got = dc.cpu().numpy().reshape(n, m).T.astype(np.float64)
        assert np.all(np.abs(got - ref) <= oracle.tol_north_star(k, mag))
        del graph
    assert sg.get_device_errors() == 0


def test_shared_workspace_counters_alternate(cuda, handle):
    """One handle alternating between deep-k cluster launches (arrival
    counters and partial tiles in the handle's workspace) and stream-K tile
    kernel launches (counters and slots at the same offsets), without a host
    sync in between: every launch must leave its counters at zero for the
    next, so each result equals the one a fresh handle computes."""
    torch = cuda
    cases = [C.Case("alt-small", 0, 0, 128, 128, 8192, 128, 8192, 128, 1.0, 0.0),
             C.Case("alt-tile", 0, 1, 1500, 1300, 3000, 1500, 1300, 1500, 0.5, 1.0),
             C.Case("alt-small2", 1, 0, 64, 200, 3000, 3000, 3000, 64, -1.0, 0.5)]
    inputs, expect = [], []
    for i, case in enumerate(cases):
        a, b, c = C.cfg_inputs(case, 950 + i, None)
        with sg.Handle() as fresh:
            _, out = run_sgemm(torch, fresh, case, a, b, c)
        inputs.append((to_device(torch, a), to_device(torch, b), c))
        expect.append(out)
    outs = []
    torch.cuda.synchronize()
    for rep in range(3):
        for case, ((_, pa), (_, pb), c) in zip(cases, inputs):
            dc, pc = to_device(torch, c)
            handle.sgemm(case.transa, case.transb, case.m, case.n, case.k, case.alpha, pa,
                         case.lda, pb, case.ldb, case.beta, pc, case.ldc)
            outs.append(dc)
    torch.cuda.synchronize()
    for i, dc in enumerate(outs):
        assert np.array_equal(dc.cpu().numpy(), expect[i % len(cases)]), (i, cases[i % 3].name)
    assert sg.get_device_errors() == 0


def test_kernel_selection(cuda, handle):
    """Small products launch the cluster kernel, larger ones the persistent
    tile kernel (kernel names from the profiler's CUDA activity)."""
    torch = cuda
    from torch.profiler import ProfilerActivity, profile

    def kernels(m, n, k):
        a = torch.rand(m * k, device="cuda")
        b = torch.rand(k * n, device="cuda")
        c = torch.zeros(m * n, device="cuda")
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            handle.sgemm(0, 0, m, n, k, 1.0, a.data_ptr(), m, b.data_ptr(), k, 0.0, c.data_ptr(), m)
            torch.cuda.synchronize()
        return [e.name for e in prof.events() if "Kernel" in e.name or "kernel" in e.name]

    small = kernels(256, 256, 256)
    large = kernels(1300, 1000, 70)
    if not small and not large:
        pytest.skip("the profiler recorded no CUDA kernels")
    assert any("smallKernel" in s for s in small), small
    assert any("sgemmKernel" in s for s in large) and not any("smallKernel" in s for s in large), \
        large
