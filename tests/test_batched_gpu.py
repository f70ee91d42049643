"""Batched SGEMM on the GPU: sgblasSgemmStridedBatched and sgblasSgemmBatched.

Every matrix of a batch is checked in full against the FP64 oracle within the
north-star bound, the same check the single-matrix tests apply, plus the
untouched padding rows of C and no read of C when beta == 0 (NaN poison).
Layouts cover both staging paths: strides that keep every matrix 16-byte
aligned (TMA, one 3-D tensor map per operand), strides or pointers that do
not (cp.async), reuse of one matrix (stride 0), negative strides and
shuffled pointer arrays.
"""
import numpy as np
import pytest

import oracle
import sgblas_b200 as sg
from tests import cases as C
from tests.gpu_util import c_view

pytestmark = pytest.mark.gpu


def _matrices(case, count, seed):
    out = []
    for i in range(count):
        a, b, c = C.cfg_inputs(case, seed + 7 * i, None)
        C.pad_and_poison(c, case.m, case.n, case.ldc, case.beta, C.PRODUCT_PAD)
        out.append((a, b, c))
    return out


def _check(case, a, b, c0, got, what):
    ref, mag = oracle.sgemm_f64(case.transa, case.transb, case.m, case.n, case.k, case.alpha, a,
                                case.lda, b, case.ldb, case.beta, c0, case.ldc)
    res = oracle.check(c_view(got, case.m, case.n, case.ldc), ref, mag, case.k)
    assert res["ok_north_star"], (what, res)
    pad_in = c0.reshape(case.n, case.ldc)[:, case.m:]
    pad_out = got.reshape(case.n, case.ldc)[:, case.m:]
    assert np.array_equal(pad_in, pad_out, equal_nan=True), (what, "padding rows written")


def _place(torch, mats, stride, size, offset=0):
    """One device buffer holding matrix i at offset + i*stride floats (stride
    may be 0 or negative: then the base is the first matrix's position)."""
    count = len(mats)
    first = offset + (0 if stride >= 0 else -stride * (count - 1))
    span = first + max(stride * (count - 1), 0) + size
    host = np.full(span, np.nan, dtype=np.float32)
    for i, m in enumerate(mats):
        host[first + i * stride:first + i * stride + size] = m
    buf = torch.from_numpy(host).cuda()
    return buf, buf.data_ptr() + 4 * first, first


STRIDED = []
for ta in (0, 1):
    for tb in (0, 1):
        # (m, n, k, pad, extra stride floats): extra % 4 == 0 keeps TMA
        # small-problem cluster kernel (at most 37 tiles of 128 x 128) ...
        STRIDED.append((ta, tb, 300, 200, 70, 0, 8))
        STRIDED.append((ta, tb, 257, 129, 33, 4, 3))
        # ... and the persistent tile kernel
        STRIDED.append((ta, tb, 700, 600, 70, 0, 8))
        STRIDED.append((ta, tb, 650, 520, 33, 4, 3))
STRIDED += [(0, 0, 1000, 700, 900, 0, 0), (1, 0, 129, 1031, 400, 4, 4)]


@pytest.mark.parametrize("ta,tb,m,n,k,pad,extra", STRIDED)
def test_strided_batched(cuda, handle, ta, tb, m, n, k, pad, extra):
    torch = cuda
    count = 3
    for alpha, beta in ((1.0, 0.0), (0.75, -1.25)):
        case = C.Case("strided", ta, tb, m, n, k, (k if ta else m) + pad, (n if tb else k) + pad,
                      m + (pad or 1), alpha, beta)
        mats = _matrices(case, count, 500 + m + k)
        sa, sb, sc = (case.a_size + extra, case.b_size + extra, case.c_size + extra)
        da, pa, _ = _place(torch, [x[0] for x in mats], sa, case.a_size)
        db, pb, _ = _place(torch, [x[1] for x in mats], sb, case.b_size)
        dc, pc, first = _place(torch, [x[2] for x in mats], sc, case.c_size)
        handle.sgemm_strided_batched(ta, tb, m, n, k, alpha, pa, case.lda, sa, pb, case.ldb, sb,
                                     beta, pc, case.ldc, sc, count)
        torch.cuda.synchronize()
        out = dc.cpu().numpy()
        for i, (a, b, c) in enumerate(mats):
            got = out[first + i * sc:first + i * sc + case.c_size]
            _check(case, a, b, c, got, (ta, tb, m, n, k, pad, extra, alpha, beta, i))
    assert sg.get_device_errors() == 0


@pytest.mark.parametrize("m,n", [(260, 190), (1000, 700)])
@pytest.mark.parametrize("stride_sign", [0, -1])
def test_strided_batched_reuse_and_negative_strides(cuda, handle, stride_sign, m, n):
    """stride_a == 0 reuses one A for every product; negative strides walk
    the batch backwards from the base pointer (small and tile kernels)."""
    torch = cuda
    count, k = 4, 150
    case = C.Case("reuse", 0, 1, m, n, k, m, n, m, 1.5, 0.5)
    mats = _matrices(case, count, 77)
    a_shared = mats[0][0]
    sa = 0
    sb = stride_sign * (case.b_size + 4) if stride_sign else case.b_size + 4
    sc = -(case.c_size + 8) if stride_sign else case.c_size + 8
    da, pa, _ = _place(torch, [a_shared], 0, case.a_size)
    db, pb, _ = _place(torch, [x[1] for x in mats], sb, case.b_size)
    dc, pc, first = _place(torch, [x[2] for x in mats], sc, case.c_size)
    handle.sgemm_strided_batched(0, 1, m, n, k, case.alpha, pa, m, sa, pb, n, sb, case.beta, pc, m,
                                 sc, count)
    torch.cuda.synchronize()
    out = dc.cpu().numpy()
    for i, (_, b, c) in enumerate(mats):
        got = out[first + i * sc:first + i * sc + case.c_size]
        _check(case, a_shared, b, c, got, (stride_sign, i))


@pytest.mark.parametrize("m,n", [(231, 300), (700, 600)])
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_pointer_array_batched(cuda, handle, ta, tb, m, n):
    """Device arrays of pointers, in shuffled order, one matrix misaligned
    (small and tile kernels)."""
    torch = cuda
    count, k = 5, 97
    case = C.Case("arrays", ta, tb, m, n, k, (k if ta else m) + 1, (n if tb else k) + 2, m + 3,
                  -0.5, 2.0)
    mats = _matrices(case, count, 901)
    order = [3, 0, 4, 1, 2]
    bufs, ptrs = [], {"a": [], "b": [], "c": []}
    for i in range(count):
        for key, host, off in (("a", mats[i][0], 1 if i == 2 else 0), ("b", mats[i][1], 0),
                               ("c", mats[i][2], 0)):
            buf = torch.empty(host.size + off, dtype=torch.float32, device="cuda")
            buf[off:].copy_(torch.from_numpy(host))
            bufs.append((key, i, buf, off))
            ptrs[key].append(buf.data_ptr() + 4 * off)
    arrays = {key: torch.tensor([ptrs[key][j] for j in order], dtype=torch.int64, device="cuda")
              for key in ptrs}
    handle.sgemm_batched(ta, tb, m, n, k, case.alpha, arrays["a"], case.lda, arrays["b"],
                         case.ldb, case.beta, arrays["c"], case.ldc, count)
    torch.cuda.synchronize()
    for key, i, buf, off in bufs:
        if key != "c":
            continue
        a, b, c = mats[i]
        _check(case, a, b, c, buf[off:].cpu().numpy(), (ta, tb, i))
    assert sg.get_device_errors() == 0


@pytest.mark.parametrize("beta", [0.0, 0.5])
def test_batched_scale_only(cuda, handle, beta):
    """alpha == 0: C_i = beta*C_i for every matrix, C never read when beta == 0."""
    torch = cuda
    count, m, n = 3, 70, 40
    case = C.Case("scale", 0, 0, m, n, 5, m, 5, m + 2, 0.0, beta)
    mats = _matrices(case, count, 3)
    dc, pc, first = _place(torch, [x[2] for x in mats], case.c_size, case.c_size)
    handle.sgemm_strided_batched(0, 0, m, n, 5, 0.0, None, m, 0, None, 5, 0, beta, pc, case.ldc,
                                 case.c_size, count)
    torch.cuda.synchronize()
    out = dc.cpu().numpy()
    for i, (_, _, c) in enumerate(mats):
        got = c_view(out[first + i * case.c_size:first + (i + 1) * case.c_size], m, n, case.ldc)
        want = np.zeros((m, n), np.float32) if beta == 0.0 else \
            (np.float32(beta) * c_view(c, m, n, case.ldc)).astype(np.float32)
        assert np.array_equal(got, want), i


def test_large_batch_uses_every_sm(cuda, handle):
    """Many small products in one launch (tiles across the batch feed the
    persistent schedule), sampled against the oracle."""
    torch = cuda
    count, m, n, k = 64, 128, 96, 256
    case = C.Case("many", 0, 0, m, n, k, m, k, m, 1.0, 1.0)
    mats = _matrices(case, count, 11)
    da, pa, _ = _place(torch, [x[0] for x in mats], case.a_size, case.a_size)
    db, pb, _ = _place(torch, [x[1] for x in mats], case.b_size, case.b_size)
    dc, pc, first = _place(torch, [x[2] for x in mats], case.c_size, case.c_size)
    handle.sgemm_strided_batched(0, 0, m, n, k, 1.0, pa, m, case.a_size, pb, k, case.b_size, 1.0,
                                 pc, m, case.c_size, count)
    torch.cuda.synchronize()
    out = dc.cpu().numpy()
    for i in (0, 1, 31, 63):
        a, b, c = mats[i]
        _check(case, a, b, c, out[i * case.c_size:(i + 1) * case.c_size], i)
