"""Two copies of libsgblas.so in one process.

A process can hold two copies of the library: two packages that each ship it,
or an A/B timing harness that loads two builds. Each copy statically links its
own CUDA runtime and registers its own kernels; none may depend on the other's
state. Before the library exported only its C API, the per-kernel "shared
memory attribute set" flags were STB_GNU_UNIQUE symbols that the dynamic
linker merged across the copies, so the second copy skipped
cudaFuncSetAttribute for its own tile kernels and their launches failed.

Here both copies run the persistent tile kernel (and the small-problem
kernel), interleaved, each checked against the FP64 oracle.
"""
import ctypes
import shutil

import numpy as np
import pytest

import oracle
import sgblas_b200 as sg

pytestmark = pytest.mark.gpu


def _load_copy(path):
    dll = ctypes.CDLL(str(path))
    for name, (res, args) in sg._SIGNATURES.items():
        fn = getattr(dll, name)
        fn.restype = res
        fn.argtypes = args
    return dll


def _run(torch, dll, m, n, k, seed):
    rng = oracle.Rng(seed)
    a, b, c = rng.uniform(m * k), rng.uniform(k * n), rng.uniform(m * n)
    da, db, dc = (torch.from_numpy(x).cuda() for x in (a, b, c))
    h = ctypes.c_void_p()
    assert dll.sgblasCreate(ctypes.byref(h)) == 0
    f = ctypes.c_float
    st = dll.sgblasSgemm(h, 0, 0, m, n, k, ctypes.byref(f(0.5)), da.data_ptr(), m, db.data_ptr(),
                         k, ctypes.byref(f(-1.5)), dc.data_ptr(), m)
    torch.cuda.synchronize()
    assert dll.sgblasDestroy(h) == 0
    assert st == 0, st
    ref, mag = oracle.sgemm_f64(0, 0, m, n, k, 0.5, a, m, b, k, -1.5, c, m)
    return oracle.check(dc.cpu().numpy().reshape(n, m).T, ref, mag, k)


def test_two_copies_in_one_process(cuda, tmp_path):
    torch = cuda
    copies = []
    for i in range(2):
        path = tmp_path / f"copy{i}" / "libsgblas.so"
        path.parent.mkdir()
        shutil.copy(sg.LIB_PATH, path)
        copies.append(_load_copy(path))
    # The package's own copy first (as in a harness that imported it), then
    # both extra copies, interleaved; tile kernel (1300 x 1000 x 700: 88
    # tiles of 128 x 128) and cluster kernel (256^3).
    order = [sg.lib, copies[0], copies[1], copies[0], sg.lib, copies[1]]
    for i, dll in enumerate(order):
        for shape in ((1300, 1000, 700), (256, 256, 256)):
            res = _run(torch, dll, *shape, seed=11 + i)
            assert res["ok_north_star"], (i, shape, res)
    assert sg.get_device_errors() == 0
