"""Generates tests/golden/reference_suite.npz from the reference library itself.

Run on a machine with a GPU, after `make -C oracle ref` built the reference
sgBLAS (AG0708/sgBLAS, compiled from its own sources for sm_100a into
oracle/_ref/libsgblas_ref.so):

    python tests/golden/make_golden.py [OUT.npz]

For every product case of the reference's device correctness suite (with the
suite's exact inputs: tests/cases.py replays its mt19937 stream) and for the
BASELINE transpose/tail sweep (config 3, all four modes), it runs the
reference's sgblasSgemm and stores, per case, a fixed sample of output
entries: "<name>/rows", "<name>/cols" (int32) and "<name>/vals" (float32, what
the reference computed). Small outputs are stored whole.
"""
import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

SAMPLES = 2048


def sample(m: int, n: int, seed: int):
    if m * n <= SAMPLES:
        rows, cols = np.meshgrid(np.arange(m), np.arange(n), indexing="ij")
        return rows.ravel().astype(np.int32), cols.ravel().astype(np.int32)
    rng = np.random.default_rng(seed)
    return (rng.integers(0, m, SAMPLES).astype(np.int32),
            rng.integers(0, n, SAMPLES).astype(np.int32))


def golden_cases():
    from tests import cases as C
    for item in C.reference_suite():
        if item[0] == "product":
            _, case, a, b, c = item
            yield case, a, b, c
    for ta in (0, 1):
        for tb in (0, 1):
            case = C.cfg3(ta, tb)
            a, b, c = C.cfg_inputs(case, 3, None, normal=True)
            yield case, a, b, c


def main(out_path: str) -> None:
    import torch

    import oracle

    ref = oracle.RefLib()
    torch.cuda.set_device(0)
    data = {}
    for i, (case, a, b, c) in enumerate(golden_cases()):
        da = torch.from_numpy(a).cuda()
        db = torch.from_numpy(b).cuda()
        dc = torch.from_numpy(c).cuda()
        status = ref.sgemm(case.transa, case.transb, case.m, case.n, case.k, case.alpha, da,
                           case.lda, db, case.ldb, case.beta, dc, case.ldc)
        torch.cuda.synchronize()
        assert status == 0, (case.name, status)
        out = dc.cpu().numpy()
        rows, cols = sample(case.m, case.n, 1000 + i)
        data[f"{case.name}/rows"] = rows
        data[f"{case.name}/cols"] = cols
        data[f"{case.name}/vals"] = out[rows.astype(np.int64) + cols.astype(np.int64) * case.ldc]
        print(f"{case.name}: {rows.size} entries")
    ref.close()
    np.savez_compressed(out_path, **data)
    print("wrote", out_path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(ROOT / "tests" / "golden" / "reference_suite.npz"))
