"""Host-side API contract, no GPU needed.

Restates the reference's host test (tests/host/host_tests.cpp:29-150 of
AG0708/sgBLAS): status codes of create/destroy, stream and math-mode
accessors, argument validation and quick returns with fake device pointers
that are never dereferenced. Where the reference host build was compiled
(oracle/_ref/libsgblas_ref_host.so), the same calls are also run against it
and the statuses must agree.
"""
import ctypes
import itertools
import pathlib
import re
import subprocess

import pytest

import sgblas_b200 as sg

ROOT = pathlib.Path(__file__).resolve().parent.parent
FAKE_A = 0x1000
FAKE_C = 0x2000


def declared_symbols():
    names = set()
    for header in (ROOT / "include" / "sgblas").glob("*.h"):
        text = header.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(sgblas[A-Z]\w*)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    names = declared_symbols()
    assert "sgblasSgemm" in names and "sgblasCreate" in names
    out = subprocess.run(["nm", "-D", "--defined-only", str(sg.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in names if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for n in names:
        assert hasattr(sg.lib, n)
    assert set(sg.EXPORTED_SYMBOLS) >= set(names) - set(), "ctypes table incomplete"


def test_library_exports_only_the_c_api():
    """Nothing but the declared C API leaves the library: no C++ template
    instances, kernel stubs or CUDA-runtime symbols, and in particular no
    STB_GNU_UNIQUE objects, which the dynamic linker merges across every
    library of the process even under RTLD_LOCAL (two copies of the library
    would then share their per-kernel set-up flags)."""
    out = subprocess.run(["readelf", "--dyn-syms", "-W", str(sg.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    defined = []
    for line in out.splitlines():
        f = line.split()
        if len(f) >= 8 and f[6] != "UND" and f[4] in ("GLOBAL", "WEAK", "UNIQUE"):
            defined.append((f[4], f[7].split("@")[0]))
    assert not [n for b, n in defined if b == "UNIQUE"], "GNU_UNIQUE symbols exported"
    assert sorted(n for _, n in defined) == declared_symbols()


def test_create_destroy_contract():
    assert sg.lib.sgblasCreate(None) == sg.SGBLAS_STATUS_INVALID_VALUE
    assert sg.lib.sgblasDestroy(None) == sg.SGBLAS_STATUS_NOT_INITIALIZED
    h = ctypes.c_void_p()
    assert sg.lib.sgblasCreate(ctypes.byref(h)) == sg.SGBLAS_STATUS_SUCCESS
    assert h.value is not None
    assert sg.lib.sgblasDestroy(h) == sg.SGBLAS_STATUS_SUCCESS


def test_stream_and_math_mode(handle):
    h = handle.raw
    fake_stream = ctypes.c_void_p(0x1234)
    assert sg.lib.sgblasSetStream(h, fake_stream) == 0
    out = ctypes.c_void_p()
    assert sg.lib.sgblasGetStream(h, ctypes.byref(out)) == 0
    assert out.value == 0x1234
    assert sg.lib.sgblasGetStream(h, None) == sg.SGBLAS_STATUS_INVALID_VALUE
    assert sg.lib.sgblasSetStream(None, fake_stream) == sg.SGBLAS_STATUS_NOT_INITIALIZED
    mode = ctypes.c_int(sg.SGBLAS_MATH_TF32)
    assert sg.lib.sgblasGetMathMode(h, ctypes.byref(mode)) == 0
    assert mode.value == sg.SGBLAS_MATH_FP32
    assert sg.lib.sgblasSetMathMode(h, sg.SGBLAS_MATH_TF32) == 0
    assert handle.get_math_mode() == sg.SGBLAS_MATH_TF32
    assert sg.lib.sgblasSetMathMode(h, 99) == sg.SGBLAS_STATUS_INVALID_VALUE
    assert sg.lib.sgblasGetMathMode(h, None) == sg.SGBLAS_STATUS_INVALID_VALUE
    assert sg.lib.sgblasSetMathMode(h, sg.SGBLAS_MATH_FP32) == 0


def test_status_strings():
    expected = ["success", "not initialized", "allocation failed", "invalid value",
                "architecture mismatch", "execution failed", "internal error", "not supported"]
    for code, text in enumerate(expected):
        assert sg.status_string(code) == text
    assert sg.status_string(42) == "unknown status"
    assert sg.status_string(0x7FFFFFFF) == "unknown status"


# (name, args, expected): args = transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc
ONE, ZERO, TWO = 1.0, 0.0, 2.0
VALIDATION_CASES = [
    ("invalid operation", (9, 0, 2, 3, 4, ONE, FAKE_A, 2, FAKE_A, 4, ZERO, FAKE_C, 2), 3),
    ("negative m", (0, 0, -1, 3, 4, ONE, FAKE_A, 2, FAKE_A, 4, ZERO, FAKE_C, 2), 3),
    ("negative n", (0, 0, 2, -3, 4, ONE, FAKE_A, 2, FAKE_A, 4, ZERO, FAKE_C, 2), 3),
    ("negative k", (0, 0, 2, 3, -4, ONE, FAKE_A, 2, FAKE_A, 4, ZERO, FAKE_C, 2), 3),
    ("NN lda", (0, 0, 2, 3, 4, ONE, FAKE_A, 1, FAKE_A, 4, ZERO, FAKE_C, 2), 3),
    ("TN lda against k", (1, 0, 2, 3, 4, ONE, FAKE_A, 3, FAKE_A, 4, ZERO, FAKE_C, 2), 3),
    ("NT ldb against n", (0, 1, 2, 3, 4, ONE, FAKE_A, 2, FAKE_A, 2, ZERO, FAKE_C, 2), 3),
    ("ldc", (0, 0, 2, 3, 4, ONE, FAKE_A, 2, FAKE_A, 4, ZERO, FAKE_C, 1), 3),
    ("missing alpha", (0, 0, 2, 3, 4, None, FAKE_A, 2, FAKE_A, 4, ZERO, FAKE_C, 2), 3),
    ("missing beta", (0, 0, 2, 3, 4, ONE, FAKE_A, 2, FAKE_A, 4, None, FAKE_C, 2), 3),
    ("missing A", (0, 0, 2, 3, 4, ONE, None, 2, FAKE_A, 4, ZERO, FAKE_C, 2), 3),
    ("missing B", (0, 0, 2, 3, 4, ONE, FAKE_A, 2, None, 4, ZERO, FAKE_C, 2), 3),
    ("missing C", (0, 0, 2, 3, 4, ONE, FAKE_A, 2, FAKE_A, 4, ZERO, None, 2), 3),
    ("empty output quick return", (0, 0, 0, 3, 4, None, None, 1, None, 4, None, None, 1), 0),
    ("n == 0 quick return", (1, 1, 5, 0, 4, None, None, 4, None, 1, None, None, 5), 0),
    ("alpha zero beta one", (0, 0, 2, 3, 4, ZERO, None, 2, None, 4, ONE, None, 2), 0),
    ("k zero beta one", (0, 0, 2, 3, 0, TWO, None, 2, None, 1, ONE, None, 2), 0),
    ("scale requires C", (0, 0, 2, 3, 4, ZERO, None, 2, None, 4, ZERO, None, 2), 3),
    ("lda minimum is 1 when m == 0", (0, 0, 0, 3, 4, ONE, None, 0, None, 4, ONE, None, 1), 3),
]


@pytest.mark.parametrize("name,args,expected", VALIDATION_CASES, ids=[c[0] for c in VALIDATION_CASES])
def test_validation_statuses(handle, name, args, expected):
    assert handle.sgemm_status(*args) == expected


def test_null_handle():
    h = sg.Handle()
    status = sg.lib.sgblasSgemm(None, 0, 0, 2, 3, 4, ctypes.byref(ctypes.c_float(1.0)), FAKE_A, 2,
                                FAKE_A, 4, ctypes.byref(ctypes.c_float(0.0)), FAKE_C, 2)
    assert status == sg.SGBLAS_STATUS_NOT_INITIALIZED
    h.close()


def test_tf32_mode_quick_returns(handle):
    """The TF32 lane computes work on the tensor cores (GPU tests); the quick
    returns that need no device keep sgblasSgemm's statuses in TF32 mode.
    (Work is not called here: fake pointers must never reach a kernel.)"""
    handle.set_math_mode(sg.SGBLAS_MATH_TF32)
    assert handle.sgemm_status(0, 0, 2, 3, 4, ZERO, None, 2, None, 4, ONE, None, 2) == 0
    assert handle.sgemm_status(0, 0, 0, 3, 4, None, None, 1, None, 4, None, None, 1) == 0
    assert handle.sgemm_status(0, 0, 2, 3, 4, ONE, FAKE_A, 1, FAKE_A, 4, ZERO, FAKE_C, 2) == 3
    handle.set_math_mode(sg.SGBLAS_MATH_FP32)


def _ref_host():
    import oracle
    try:
        return oracle.RefLib(host=True)
    except FileNotFoundError:
        pytest.skip("reference host build not present (make -C oracle ref)")


def test_validation_matches_reference_host_build(handle):
    """Differential check over a grid of argument combinations whose outcome
    needs no device: every status must equal the reference's."""
    ref = _ref_host()
    dims = [0, 1, 3]
    lds = [0, 1, 2, 3, 4]
    scalars = [None, 0.0, 1.0, 2.0]
    ptrs = [None, FAKE_A]
    checked = 0
    for ta, tb, m, n, k in itertools.product([0, 1, 2], [0, 1], dims, dims, dims):
        for lda, ldb, ldc in itertools.product(lds, lds, lds[1:4]):
            for alpha, beta in itertools.product(scalars, scalars):
                for a, c in itertools.product(ptrs, [None, FAKE_C]):
                    args = (ta, tb, m, n, k, alpha, a, lda, a, ldb, beta, c, ldc)
                    expect = ref.sgemm(*args)
                    if expect == sg.SGBLAS_STATUS_NOT_SUPPORTED:
                        continue  # the host stub refuses real work; we would launch
                    assert handle.sgemm_status(*args) == expect, args
                    checked += 1
    ref.close()
    assert checked > 10000


def test_status_strings_match_reference():
    ref = _ref_host()
    for code in list(range(0, 9)) + [0x7FFFFFFF]:
        assert sg.status_string(code) == ref.dll.refSgblasGetStatusString(code).decode()
    ref.close()


# ---- batched entry points: same validation, then the batch count --------------
@pytest.mark.parametrize("name,args,expected", VALIDATION_CASES, ids=[c[0] for c in VALIDATION_CASES])
def test_batched_validation_matches_single(handle, name, args, expected):
    """Every single-matrix validation outcome carries over to both batched
    forms (strided: base pointers; pointer arrays: the arrays)."""
    ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc = args
    for count in (1, 3):
        assert handle.sgemm_strided_batched_status(ta, tb, m, n, k, alpha, a, lda, 64, b, ldb, 64,
                                                   beta, c, ldc, 64, count) == expected
        assert handle.sgemm_batched_status(ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc,
                                           count) == expected


def test_batched_count_rules(handle):
    work = (0, 0, 2, 3, 4, ONE, FAKE_A, 2, FAKE_A, 4, ZERO, FAKE_C, 2)
    ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc = work
    strided = lambda count, **kw: handle.sgemm_strided_batched_status(
        ta, tb, kw.get("m", m), n, k, alpha, a, kw.get("lda", lda), 8, b, ldb, 12, beta, c, ldc,
        6, count)
    arrays = lambda count, **kw: handle.sgemm_batched_status(
        ta, tb, kw.get("m", m), n, k, alpha, a, kw.get("lda", lda), b, ldb, beta, c, ldc, count)
    for call in (strided, arrays):
        assert call(-1) == sg.SGBLAS_STATUS_INVALID_VALUE
        assert call(0) == sg.SGBLAS_STATUS_SUCCESS              # no work, no device access
        assert call(-1, m=0) == sg.SGBLAS_STATUS_INVALID_VALUE  # the count is checked after
        assert call(0, m=0) == sg.SGBLAS_STATUS_SUCCESS         # validation, before quick returns
        assert call(-1, lda=1) == sg.SGBLAS_STATUS_INVALID_VALUE
    assert sg.lib.sgblasSgemmStridedBatched(None, 0, 0, 2, 3, 4, None, None, 2, 0, None, 4, 0,
                                            None, None, 2, 0, 1) == sg.SGBLAS_STATUS_NOT_INITIALIZED
    assert sg.lib.sgblasSgemmBatched(None, 0, 0, 2, 3, 4, None, None, 2, None, 4, None, None, 2,
                                     1) == sg.SGBLAS_STATUS_NOT_INITIALIZED
    handle.set_math_mode(sg.SGBLAS_MATH_TF32)
    assert strided(0) == sg.SGBLAS_STATUS_SUCCESS
    assert arrays(-1) == sg.SGBLAS_STATUS_INVALID_VALUE
    handle.set_math_mode(sg.SGBLAS_MATH_FP32)


def test_reference_install_consumer_runs_against_product():
    """The reference's own C consumer (cmake/install-consumer/main.c),
    compiled unchanged against include/sgblas/sgblas.h and linked to this
    library by oracle/Makefile, runs to exit status 0 (create, status string,
    destroy)."""
    exe = ROOT / "oracle" / "_ref" / "install_consumer_b200"
    if not exe.exists():
        pytest.skip("install consumer not built (make -C oracle ref)")
    libs = subprocess.run(["ldd", str(exe)], capture_output=True, text=True).stdout
    assert str((ROOT / "sgblas_b200" / "lib" / "libsgblas.so").resolve()) in libs or \
        "sgblas_b200/lib/libsgblas.so" in libs, libs
    assert subprocess.run([str(exe)], timeout=60).returncode == 0
