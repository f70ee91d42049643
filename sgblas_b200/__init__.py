"""sgblas_b200 -- strict-FP32 column-major SGEMM for NVIDIA B200 (sm_100a).

The product is the C library ``sgblas_b200/lib/libsgblas.so`` whose ABI is the
reference sgBLAS API (``include/sgblas/sgblas.h``). This module is a thin
ctypes mirror of that API for Python callers and for the test-suite: the same
entry-point names, the same argument meaning and the same status codes
(``sgblasCreate`` ... ``sgblasSgemm``; reference ``include/sgblas/sgblas.h:38-62``
of AG0708/sgBLAS), plus a small object wrapper (:class:`Handle`).

There is no CPU fallback: importing this module fails loudly when the library
has not been built (``python sgblas_b200/build.py``).
"""
from __future__ import annotations

import ctypes
import pathlib

__all__ = [
    "LIB_PATH", "lib", "SgblasError", "Handle", "status_string",
    "SGBLAS_STATUS_SUCCESS", "SGBLAS_STATUS_NOT_INITIALIZED", "SGBLAS_STATUS_ALLOC_FAILED",
    "SGBLAS_STATUS_INVALID_VALUE", "SGBLAS_STATUS_ARCH_MISMATCH",
    "SGBLAS_STATUS_EXECUTION_FAILED", "SGBLAS_STATUS_INTERNAL_ERROR",
    "SGBLAS_STATUS_NOT_SUPPORTED", "SGBLAS_OP_N", "SGBLAS_OP_T", "SGBLAS_MATH_FP32",
    "SGBLAS_MATH_TF32", "EXPORTED_SYMBOLS", "MgHandle", "mg_unique_id", "get_device_errors",
]

LIB_PATH = pathlib.Path(__file__).resolve().parent / "lib" / "libsgblas.so"

# Status / operation / math-mode values (fixed by the ABI).
SGBLAS_STATUS_SUCCESS = 0
SGBLAS_STATUS_NOT_INITIALIZED = 1
SGBLAS_STATUS_ALLOC_FAILED = 2
SGBLAS_STATUS_INVALID_VALUE = 3
SGBLAS_STATUS_ARCH_MISMATCH = 4
SGBLAS_STATUS_EXECUTION_FAILED = 5
SGBLAS_STATUS_INTERNAL_ERROR = 6
SGBLAS_STATUS_NOT_SUPPORTED = 7
SGBLAS_OP_N = 0
SGBLAS_OP_T = 1
SGBLAS_MATH_FP32 = 0
SGBLAS_MATH_TF32 = 1

_c_int_p = ctypes.POINTER(ctypes.c_int)
_c_float_p = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes); every symbol declared in include/sgblas/*.h.
_SIGNATURES = {
    "sgblasCreate": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p)]),
    "sgblasDestroy": (ctypes.c_int, [ctypes.c_void_p]),
    "sgblasSetStream": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "sgblasGetStream": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "sgblasSetMathMode": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "sgblasGetMathMode": (ctypes.c_int, [ctypes.c_void_p, _c_int_p]),
    "sgblasSgemm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, _c_float_p, ctypes.c_void_p,
                                    ctypes.c_int, ctypes.c_void_p, ctypes.c_int, _c_float_p,
                                    ctypes.c_void_p, ctypes.c_int]),
    "sgblasGetStatusString": (ctypes.c_char_p, [ctypes.c_int]),
    "sgblasGetDeviceErrors": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint), ctypes.c_int]),
    "sgblasSelfTestWaitTimeout": (ctypes.c_int, [ctypes.c_uint, ctypes.POINTER(ctypes.c_int)]),
    "sgblasTestInterruptScratch": (ctypes.c_int, [ctypes.c_void_p]),
    "sgblasSgemmStridedBatched": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                 _c_float_p, ctypes.c_void_p, ctypes.c_int,
                                                 ctypes.c_longlong, ctypes.c_void_p, ctypes.c_int,
                                                 ctypes.c_longlong, _c_float_p, ctypes.c_void_p,
                                                 ctypes.c_int, ctypes.c_longlong, ctypes.c_int]),
    "sgblasSgemmBatched": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, _c_float_p, ctypes.c_void_p,
                                          ctypes.c_int, ctypes.c_void_p, ctypes.c_int, _c_float_p,
                                          ctypes.c_void_p, ctypes.c_int, ctypes.c_int]),
    "sgblasSgemmNoAlloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_int, ctypes.c_int, _c_float_p,
                                           ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                           ctypes.c_int, _c_float_p, ctypes.c_void_p,
                                           ctypes.c_int]),
    # multi-GPU extension (include/sgblas/sgblas_mg.h)
    "sgblasMgGetUniqueId": (ctypes.c_int, [ctypes.c_void_p]),
    "sgblasMgCreate": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_int]),
    "sgblasMgDestroy": (ctypes.c_int, [ctypes.c_void_p]),
    "sgblasMgAbort": (ctypes.c_int, [ctypes.c_void_p]),
    "sgblasMgSetStream": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "sgblasMgSetMathMode": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "sgblasMgGetRank": (ctypes.c_int, [ctypes.c_void_p, _c_int_p, _c_int_p]),
    "sgblasMgSgemm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, _c_float_p, ctypes.c_void_p,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                      _c_float_p, ctypes.c_void_p, ctypes.c_int]),
    "sgblasMgAllGather": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_size_t]),
}
EXPORTED_SYMBOLS = tuple(_SIGNATURES)


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python sgblas_b200/build.py` "
            "(there is no CPU fallback)")
    dll = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(dll, name)
        fn.restype = res
        fn.argtypes = args
    return dll


lib = _load()


def status_string(status: int) -> str:
    return lib.sgblasGetStatusString(status).decode()


class SgblasError(RuntimeError):
    def __init__(self, where: str, status: int):
        super().__init__(f"{where}: {status_string(status)} ({status})")
        self.status = status


def _check(where: str, status: int) -> None:
    if status != SGBLAS_STATUS_SUCCESS:
        raise SgblasError(where, status)


def _ptr(x) -> int | None:
    """Device pointer of a torch tensor, or an integer address, or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _fp(v):
    return None if v is None else ctypes.byref(ctypes.c_float(v))


class Handle:
    """Owns one sgblasHandle_t (``with Handle() as h: h.sgemm(...)``)."""

    def __init__(self):
        raw = ctypes.c_void_p()
        _check("sgblasCreate", lib.sgblasCreate(ctypes.byref(raw)))
        self._h = raw

    @property
    def raw(self) -> ctypes.c_void_p:
        return self._h

    def close(self) -> None:
        if self._h is not None and self._h.value is not None:
            _check("sgblasDestroy", lib.sgblasDestroy(self._h))
        self._h = None

    def __enter__(self) -> "Handle":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream) -> None:
        """stream: a torch.cuda.Stream, an integer cudaStream_t, or None."""
        handle = getattr(stream, "cuda_stream", stream)
        _check("sgblasSetStream", lib.sgblasSetStream(self._h, handle))

    def get_stream(self) -> int | None:
        out = ctypes.c_void_p()
        _check("sgblasGetStream", lib.sgblasGetStream(self._h, ctypes.byref(out)))
        return out.value

    def set_math_mode(self, mode: int) -> None:
        _check("sgblasSetMathMode", lib.sgblasSetMathMode(self._h, mode))

    def get_math_mode(self) -> int:
        out = ctypes.c_int()
        _check("sgblasGetMathMode", lib.sgblasGetMathMode(self._h, ctypes.byref(out)))
        return out.value

    def sgemm_status(self, transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc) -> int:
        """Raw sgblasSgemm: returns the status code. alpha/beta are Python
        floats (or None for a NULL pointer); a/b/c are torch tensors, integer
        device addresses or None."""
        return lib.sgblasSgemm(self._h, transa, transb, m, n, k, _fp(alpha), _ptr(a), lda,
                               _ptr(b), ldb, _fp(beta), _ptr(c), ldc)

    def sgemm(self, transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc) -> None:
        _check("sgblasSgemm",
               self.sgemm_status(transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc))

    def sgemm_strided_batched_status(self, transa, transb, m, n, k, alpha, a, lda, stride_a, b,
                                     ldb, stride_b, beta, c, ldc, stride_c, batch_count) -> int:
        """Raw sgblasSgemmStridedBatched (strides in elements)."""
        return lib.sgblasSgemmStridedBatched(self._h, transa, transb, m, n, k, _fp(alpha), _ptr(a),
                                             lda, stride_a, _ptr(b), ldb, stride_b, _fp(beta),
                                             _ptr(c), ldc, stride_c, batch_count)

    def sgemm_strided_batched(self, *args) -> None:
        _check("sgblasSgemmStridedBatched", self.sgemm_strided_batched_status(*args))

    def sgemm_batched_status(self, transa, transb, m, n, k, alpha, a_array, lda, b_array, ldb,
                             beta, c_array, ldc, batch_count) -> int:
        """Raw sgblasSgemmBatched: a_array/b_array/c_array are device arrays
        of device pointers (e.g. int64 torch tensors on the GPU)."""
        return lib.sgblasSgemmBatched(self._h, transa, transb, m, n, k, _fp(alpha), _ptr(a_array),
                                      lda, _ptr(b_array), ldb, _fp(beta), _ptr(c_array), ldc,
                                      batch_count)

    def sgemm_batched(self, *args) -> None:
        _check("sgblasSgemmBatched", self.sgemm_batched_status(*args))


MG_UNIQUE_ID_BYTES = 128


def mg_unique_id() -> bytes:
    """A fresh NCCL unique id (call on one rank, share the bytes)."""
    buf = (ctypes.c_ubyte * MG_UNIQUE_ID_BYTES)()
    _check("sgblasMgGetUniqueId", lib.sgblasMgGetUniqueId(buf))
    return bytes(buf)


class MgHandle:
    """One rank of a column-sharded multi-GPU SGEMM (sgblas_mg.h)."""

    def __init__(self, nranks: int, rank: int, unique_id: bytes, device: int):
        raw = ctypes.c_void_p()
        uid = (ctypes.c_ubyte * MG_UNIQUE_ID_BYTES).from_buffer_copy(unique_id)
        _check("sgblasMgCreate", lib.sgblasMgCreate(ctypes.byref(raw), nranks, rank, uid, device))
        self._h = raw

    def close(self) -> int:
        """sgblasMgDestroy; returns its status (EXECUTION_FAILED after an
        abort, or when work was still waiting for a peer at the deadline)."""
        status = SGBLAS_STATUS_SUCCESS
        if self._h is not None and self._h.value is not None:
            status = lib.sgblasMgDestroy(self._h)
        self._h = None
        return status

    def set_math_mode(self, mode: int) -> None:
        _check("sgblasMgSetMathMode", lib.sgblasMgSetMathMode(self._h, mode))

    def set_stream(self, stream) -> None:
        _check("sgblasMgSetStream",
               lib.sgblasMgSetStream(self._h, getattr(stream, "cuda_stream", stream)))

    def sgemm_status(self, transa, transb, m, n_local, k, alpha, a, lda, root, b, ldb, beta, c,
                     ldc) -> int:
        return lib.sgblasMgSgemm(self._h, transa, transb, m, n_local, k, _fp(alpha), _ptr(a), lda,
                                 root, _ptr(b), ldb, _fp(beta), _ptr(c), ldc)

    def sgemm(self, *args) -> None:
        _check("sgblasMgSgemm", self.sgemm_status(*args))

    def abort(self) -> None:
        _check("sgblasMgAbort", lib.sgblasMgAbort(self._h))

    def all_gather(self, send, recv, count: int) -> None:
        _check("sgblasMgAllGather", lib.sgblasMgAllGather(self._h, _ptr(send), _ptr(recv), count))


def get_device_errors(clear: bool = True) -> int:
    """Device error flags of the current device (synchronizes it)."""
    out = ctypes.c_uint()
    _check("sgblasGetDeviceErrors", lib.sgblasGetDeviceErrors(ctypes.byref(out), int(clear)))
    return out.value
