"""Case tables and input generation shared by the tests.

REFERENCE_PRODUCT_CASES and REFERENCE_SCALE_CASES restate, value for value,
the device correctness suite of the reference (tests/cuda/correctness.cu:
466-492 product cases, :530-539 scale cases, :513-528 null no-ops of
AG0708/sgBLAS). reference_suite() replays its input generation exactly: one
std::mt19937(20260711) stream, consumed by the three scale cases and then by
every product case (A, then B, then C), NaN in C when beta == 0 and sentinel
padding rows below m (correctness.cu:314-331, :226-240).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

import oracle

N, T = 0, 1


@dataclass(frozen=True)
class Case:
    name: str
    transa: int
    transb: int
    m: int
    n: int
    k: int
    lda: int
    ldb: int
    ldc: int
    alpha: float
    beta: float

    @property
    def a_cols(self) -> int:
        return self.m if self.transa else self.k

    @property
    def b_cols(self) -> int:
        return self.k if self.transb else self.n

    @property
    def a_size(self) -> int:
        return self.lda * self.a_cols

    @property
    def b_size(self) -> int:
        return self.ldb * self.b_cols

    @property
    def c_size(self) -> int:
        return self.ldc * self.n


REFERENCE_PRODUCT_CASES = [
    Case("NN odd beta=0", N, N, 37, 29, 43, 42, 50, 41, 1.0, 0.0),
    Case("NT padded alpha/beta", N, T, 31, 27, 35, 36, 33, 38, 0.75, -0.25),
    Case("TN padded alpha/beta", T, N, 25, 33, 39, 46, 44, 31, -1.25, 0.5),
    Case("TT odd alpha/beta", T, T, 17, 23, 19, 24, 29, 22, 0.375, 1.25),
    Case("NN alpha=0 beta!=0", N, N, 7, 5, 9, 11, 12, 10, 0.0, -0.75),
    Case("NN register tile tails", N, N, 769, 771, 37, 774, 42, 775, 0.875, -0.125),
    Case("NN exact 512 small pocket", N, N, 512, 512, 512, 512, 512, 512, 0.5, -0.25),
    Case("NN aligned full tiles", N, N, 768, 768, 64, 768, 64, 768, -0.625, 0.375),
    Case("NN medium async tile", N, N, 1024, 2048, 64, 1024, 64, 1024, 0.625, -0.375),
    Case("NN small async tile", N, N, 768, 768, 128, 768, 128, 768, -0.375, 0.625),
    Case("NT skinny tall grid limit", N, T, 1048561, 1, 1, 1048564, 3, 1048566, 1.0, 0.0),
]

# (name, k, alpha, beta) with m=7, n=5, lda=11, ldb=max(1,k+3), ldc=10.
REFERENCE_SCALE_CASES = [
    ("alpha=0 beta=0 null A/B", 9, 0.0, 0.0),
    ("alpha=0 beta=general null A/B", 9, 0.0, -0.75),
    ("k=0 beta=general null A/B", 0, 2.0, -0.5),
]

PRODUCT_PAD = 123.0
SCALE_PAD = 211.0


def pad_and_poison(c: np.ndarray, m: int, n: int, ldc: int, beta: float, pad: float) -> None:
    """NaN in C when beta == 0 (C must not be read); sentinel rows [m, ldc)."""
    cm = c.reshape(n, ldc)  # column-major: row index is the fast one
    if beta == 0.0:
        cm[:, :m] = np.nan
    rows = np.arange(m, ldc, dtype=np.float32)
    for col in range(n):
        cm[col, m:] = np.float32(pad) + rows * np.float32(0.25) + np.float32(col) * np.float32(0.03125)


def reference_suite():
    """Yields ("scale", name, k, alpha, beta, C0) then ("product", case, A, B, C0)
    with the reference suite's exact inputs."""
    rng = oracle.Rng(20260711)
    for name, k, alpha, beta in REFERENCE_SCALE_CASES:
        c = rng.uniform(10 * 5)
        pad_and_poison(c, 7, 5, 10, beta, SCALE_PAD)
        yield ("scale", name, k, alpha, beta, c)
    for case in REFERENCE_PRODUCT_CASES:
        a = rng.uniform(case.a_size)
        b = rng.uniform(case.b_size)
        c = rng.uniform(case.c_size)
        pad_and_poison(c, case.m, case.n, case.ldc, case.beta, PRODUCT_PAD)
        yield ("product", case, a, b, c)


# ---- BASELINE.json configurations --------------------------------------------
def config_case(name, transa, transb, m, n, k, lda, ldb, ldc, alpha, beta) -> Case:
    return Case(name, transa, transb, m, n, k, lda, ldb, ldc, alpha, beta)


def cfg1() -> Case:   # 256^3 NN, seed 0, C zero
    return config_case("cfg1 256^3", N, N, 256, 256, 256, 256, 256, 256, 1.0, 0.0)


def cfg2(size: int) -> Case:   # large square NN, seeds 1 (A, B) and 2 (C)
    return config_case(f"cfg2 {size}^3", N, N, size, size, size, size, size, size, 1.0, 0.0)


def cfg3(transa: int, transb: int) -> Case:   # transpose/tail sweep, ld = rows + 13
    m, n, k = 1023, 1537, 777
    lda = (k if transa else m) + 13
    ldb = (n if transb else k) + 13
    tag = ("T" if transa else "N") + ("T" if transb else "N")
    return config_case(f"cfg3 {tag}", transa, transb, m, n, k, lda, ldb, m + 13, 1.5, -0.5)


CFG4_SHAPES = [(8192, 8192, 256), (16384, 128, 16384), (128, 16384, 8192), (2048, 2048, 2048)]


def cfg4(m: int, n: int, k: int) -> Case:
    # lda = ldb = ldc = M as BASELINE.json states, except where NN needs
    # ldb >= K: (128, 16384, 8192) runs with ldb = 8192 (ldb = 128 is invalid).
    return config_case(f"cfg4 {m}x{n}x{k}", N, N, m, n, k, m, max(m, k), m, 1.0, 1.0)


def cfg_inputs(case: Case, seed_ab: int, seed_c: int | None, normal: bool = False):
    """A, B (and C) drawn in storage order; C from its own seed when seed_c is
    given, else continuing the A/B stream; zeros when seed_c == -1."""
    rng = oracle.Rng(seed_ab)
    draw = rng.normal if normal else rng.uniform
    a = draw(case.a_size)
    b = draw(case.b_size)
    if seed_c is None:
        c = draw(case.c_size)
    elif seed_c < 0:
        c = np.zeros(case.c_size, dtype=np.float32)
    else:
        rc = oracle.Rng(seed_c)
        c = rc.normal(case.c_size) if normal else rc.uniform(case.c_size)
    return a, b, c
