"""CPU oracle for strict-FP32 SGEMM -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package; the product never does.

It wraps ``oracle/_build/liboracle.so`` (built from ``oracle/oracle.cpp`` by
``make -C oracle oracle``), a restatement of the reference's FP64 triple-loop
oracle (tests/cuda/correctness.cu:373-392 of AG0708/sgBLAS) and of its seeded
input generator (tests/cuda/correctness.cu:170-174), and -- when it was built
from the reference sources by ``make -C oracle ref`` -- the reference library
itself (``oracle/_ref/libsgblas_ref.so``, symbols renamed ``refSgblas*``).

Tolerances:
  * north star: |C - C_ref| <= 2 * K * 2^-24 * mag elementwise,
    mag = |alpha| * sum|a*b| + |beta * c|. K + 2 roundings can occur (K fused
    multiply-adds, alpha*acc, and the beta update); for K >= 2 they are within
    2*K*u*mag. For K = 1 the bound is applied as 2 * max(K, 2) * u * mag.
  * the reference's own test bound (tests/cuda/correctness.cu:404-406):
    2e-6 + 8 * eps * (K + 1) * max(mag, 1), eps = 2^-23.
"""
from __future__ import annotations

import ctypes
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_SO = HERE / "_ref" / "libsgblas_ref.so"
REF_HOST_SO = HERE / "_ref" / "libsgblas_ref_host.so"

U = 2.0 ** -24           # unit roundoff of FP32
EPS = 2.0 ** -23         # FLT_EPSILON


def _build_oracle() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)


def _load_oracle() -> ctypes.CDLL:
    if not ORACLE_SO.exists():
        _build_oracle()
    dll = ctypes.CDLL(str(ORACLE_SO))
    vp, fp, dp, ip = ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p, ctypes.c_int
    dll.oracle_rng_new.restype = vp
    dll.oracle_rng_new.argtypes = [ctypes.c_uint32]
    dll.oracle_rng_free.argtypes = [vp]
    dll.oracle_rng_uniform.argtypes = [vp, vp, ctypes.c_size_t]
    dll.oracle_rng_normal.argtypes = [vp, vp, ctypes.c_size_t]
    dll.oracle_sgemm_f64.argtypes = [ip, ip, ip, ip, ip, fp, vp, ip, vp, ip, fp, vp, ip, ip, ip,
                                     dp, dp, ip]
    dll.oracle_sgemm_f64_points.argtypes = [ip, ip, ip, fp, vp, ip, vp, ip, fp, vp, ip, vp, vp, ip,
                                            dp, dp, ip]
    dll.oracle_sgemm_cpu.argtypes = [ip, ip, ip, ip, fp, vp, ip, vp, ip, fp, vp, ip, ip, ip, ip]
    dll.oracle_hardware_threads.restype = ip
    return dll


_lib = _load_oracle()


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


class Rng:
    """std::mt19937(seed); successive draws continue one stream."""

    def __init__(self, seed: int):
        self._h = _lib.oracle_rng_new(seed)

    def __del__(self):
        if getattr(self, "_h", None):
            _lib.oracle_rng_free(self._h)
            self._h = None

    def uniform(self, count: int) -> np.ndarray:
        out = np.empty(count, dtype=np.float32)
        _lib.oracle_rng_uniform(self._h, _p(out), count)
        return out

    def normal(self, count: int) -> np.ndarray:
        out = np.empty(count, dtype=np.float32)
        _lib.oracle_rng_normal(self._h, _p(out), count)
        return out


def stored_shape(trans: int, rows: int, cols: int, ld: int) -> tuple[int, int]:
    """(ld, stored columns) of op(X) = rows x cols in column-major storage."""
    return (ld, rows) if trans else (ld, cols)


def hardware_threads() -> int:
    return _lib.oracle_hardware_threads()


def _f32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    assert x.flags["F_CONTIGUOUS"] or x.ndim == 1
    return x


def sgemm_f64(transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c0, ldc,
              cols: tuple[int, int] | None = None, threads: int = 0):
    """FP64 reference and error magnitude for columns [j0, j1) of C.

    a, b, c0: float32 arrays holding the column-major storage (flattened, or
    Fortran-ordered 2-D); c0 may be None when beta == 0. Returns (ref, mag),
    float64 arrays of shape (m, j1 - j0), Fortran order.
    """
    j0, j1 = cols if cols is not None else (0, n)
    ref = np.empty((m, j1 - j0), dtype=np.float64, order="F")
    mag = np.empty_like(ref)
    a = np.ascontiguousarray(np.asarray(a, np.float32).ravel(order="F"))
    b = np.ascontiguousarray(np.asarray(b, np.float32).ravel(order="F"))
    c = None if c0 is None else np.ascontiguousarray(np.asarray(c0, np.float32).ravel(order="F"))
    _lib.oracle_sgemm_f64(int(transa), int(transb), m, n, k, float(alpha), _p(a), lda, _p(b), ldb,
                          float(beta), _p(c), ldc, j0, j1, _p(ref), _p(mag), threads)
    return ref, mag


def sgemm_f64_points(transa, transb, k, alpha, a, lda, b, ldb, beta, c0, ldc, rows, cols,
                     threads: int = 0):
    """FP64 reference and magnitude at the entries (rows[i], cols[i])."""
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    cols = np.ascontiguousarray(cols, dtype=np.int32)
    ref = np.empty(rows.size, dtype=np.float64)
    mag = np.empty_like(ref)
    a = np.ascontiguousarray(np.asarray(a, np.float32).ravel(order="F"))
    b = np.ascontiguousarray(np.asarray(b, np.float32).ravel(order="F"))
    c = None if c0 is None else np.ascontiguousarray(np.asarray(c0, np.float32).ravel(order="F"))
    _lib.oracle_sgemm_f64_points(int(transa), int(transb), k, float(alpha), _p(a), lda, _p(b), ldb,
                                 float(beta), _p(c), ldc, _p(rows), _p(cols), rows.size, _p(ref),
                                 _p(mag), threads)
    return ref, mag


def sgemm_cpu(transa, transb, m, k, alpha, a, lda, b, ldb, beta, c, ldc, j0, j1, threads=0):
    """The timed CPU baseline: the oracle loop writing FP32 results into c."""
    _lib.oracle_sgemm_cpu(int(transa), int(transb), m, k, float(alpha), _p(a), lda, _p(b), ldb,
                          float(beta), _p(c), ldc, j0, j1, threads)


def tol_north_star(k: int, mag: np.ndarray) -> np.ndarray:
    return 2.0 * max(k, 2) * U * mag


def tol_reference(k: int, mag: np.ndarray) -> np.ndarray:
    return 2.0e-6 + 8.0 * EPS * (k + 1) * np.maximum(mag, 1.0)


def check(observed: np.ndarray, ref: np.ndarray, mag: np.ndarray, k: int) -> dict:
    """Elementwise comparison against both bounds; non-finite output fails."""
    obs = np.asarray(observed, dtype=np.float64)
    err = np.abs(obs - ref)
    finite = np.isfinite(obs)
    ns = tol_north_star(k, mag)
    rf = tol_reference(k, mag)
    with np.errstate(divide="ignore", invalid="ignore"):
        ratio_ns = np.where(ns > 0, err / ns, np.where(err > 0, np.inf, 0.0))
    return {
        "ok_north_star": bool(np.all(finite) and np.all(err <= ns)),
        "ok_reference": bool(np.all(finite) and np.all(err <= rf)),
        "max_ratio_north_star": float(np.max(ratio_ns)) if ratio_ns.size else 0.0,
        "max_ratio_reference": float(np.max(err / rf)) if err.size else 0.0,
        "max_abs": float(np.max(err)) if err.size else 0.0,
        "n_bad": int(np.sum(~finite | (err > ns))),
    }


# ---- the reference library (built from the reference sources) --------------
class RefLib:
    """ctypes binding of oracle/_ref/libsgblas_ref.so (CUDA build) or of the
    host-only build (``host=True``), whose entry points are renamed
    ``refSgblas*``."""

    def __init__(self, host: bool = False):
        path = REF_HOST_SO if host else REF_SO
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (make -C oracle ref)")
        self.dll = ctypes.CDLL(str(path))
        vp, ip, fpp = ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float)
        d = self.dll
        d.refSgblasCreate.argtypes = [ctypes.POINTER(vp)]
        d.refSgblasDestroy.argtypes = [vp]
        d.refSgblasSetStream.argtypes = [vp, vp]
        d.refSgblasGetStream.argtypes = [vp, ctypes.POINTER(vp)]
        d.refSgblasSetMathMode.argtypes = [vp, ip]
        d.refSgblasGetMathMode.argtypes = [vp, ctypes.POINTER(ip)]
        d.refSgblasSgemm.argtypes = [vp, ip, ip, ip, ip, ip, fpp, vp, ip, vp, ip, fpp, vp, ip]
        d.refSgblasGetStatusString.restype = ctypes.c_char_p
        d.refSgblasGetStatusString.argtypes = [ip]
        h = vp()
        assert d.refSgblasCreate(ctypes.byref(h)) == 0
        self.h = h

    def set_stream(self, stream) -> None:
        self.dll.refSgblasSetStream(self.h, getattr(stream, "cuda_stream", stream))

    def sgemm(self, transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc) -> int:
        def fp(v):
            return None if v is None else ctypes.byref(ctypes.c_float(v))

        def ptr(x):
            return None if x is None else (x if isinstance(x, int) else x.data_ptr())

        return self.dll.refSgblasSgemm(self.h, transa, transb, m, n, k, fp(alpha), ptr(a), lda,
                                       ptr(b), ldb, fp(beta), ptr(c), ldc)

    def close(self) -> None:
        if self.h is not None:
            self.dll.refSgblasDestroy(self.h)
            self.h = None
