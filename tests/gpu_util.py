"""GPU helpers for the parity tests: upload, run through the C ABI, compare."""
from __future__ import annotations

import numpy as np

import oracle


# Guard bands: every operand sits between two 64 KiB bands of a sentinel bit
# pattern (a NaN), in place of compute-sanitizer's bounds checking: a read
# outside an operand picks up NaN (which the oracle comparison rejects), and a
# write outside it changes a band (check_guards).
GUARD_FLOATS = 16384
GUARD_BITS = 0x7F8C0DE5


def to_device(torch, host: np.ndarray, offset: int = 0):
    """Copy a float32 array to the GPU; offset > 0 places it `offset` floats
    into the buffer (for misaligned-pointer cases). Returns (buffer, device
    address of element 0): buffer[offset:] is the array. The buffer sits
    between guard bands (the offset gap belongs to the band before it)."""
    g = GUARD_FLOATS
    full = torch.empty(g + offset + host.size + g, dtype=torch.float32, device="cuda")
    full.view(torch.int32).fill_(GUARD_BITS - (1 << 32) if GUARD_BITS >= 1 << 31 else GUARD_BITS)
    buf = full[g:g + offset + host.size]
    buf[offset:].copy_(torch.from_numpy(np.ascontiguousarray(host)))
    buf._sg_guard = (full, g + offset, g + offset + host.size)
    return buf, buf.data_ptr() + 4 * offset


def check_guards(*bufs) -> None:
    """Asserts that the guard bands around each to_device buffer still hold
    the sentinel bits: nothing was written before or after the operand."""
    for i, buf in enumerate(bufs):
        full, lo, hi = buf._sg_guard
        bits = full.view(full.dtype).cpu().numpy().view(np.uint32)
        bad_lo = np.flatnonzero(bits[:lo] != GUARD_BITS)
        bad_hi = np.flatnonzero(bits[hi:] != GUARD_BITS)
        assert bad_lo.size == 0 and bad_hi.size == 0, (
            f"operand {i}: {bad_lo.size} floats written before it (nearest {lo - bad_lo.max() if bad_lo.size else 0} "
            f"floats before), {bad_hi.size} after it (first at +{bad_hi.min() if bad_hi.size else 0})")


def run_sgemm(torch, handle, case, a, b, c, offsets=(0, 0, 0), stream=None):
    """Runs sgblasSgemm on copies of a, b, c; returns (status, C after)."""
    da, pa = to_device(torch, a, offsets[0])
    db, pb = to_device(torch, b, offsets[1])
    dc, pc = to_device(torch, c, offsets[2])
    if stream is not None:
        torch.cuda.synchronize()
        handle.set_stream(stream)
    status = handle.sgemm_status(case.transa, case.transb, case.m, case.n, case.k, case.alpha, pa,
                                 case.lda, pb, case.ldb, case.beta, pc, case.ldc)
    torch.cuda.synchronize()
    check_guards(da, db, dc)
    out = dc[offsets[2]:].cpu().numpy()
    if stream is not None:
        handle.set_stream(None)
    return status, out


def c_view(flat: np.ndarray, m: int, n: int, ldc: int) -> np.ndarray:
    return flat.reshape(n, ldc).T[:m, :]


def check_full(case, a, b, c0, out) -> dict:
    """Every entry of C against the oracle, plus untouched padding rows."""
    ref, mag = oracle.sgemm_f64(case.transa, case.transb, case.m, case.n, case.k, case.alpha, a,
                                case.lda, b, case.ldb, case.beta, c0, case.ldc)
    res = oracle.check(c_view(out, case.m, case.n, case.ldc), ref, mag, case.k)
    pad_in = c0.reshape(case.n, case.ldc)[:, case.m:]
    pad_out = out.reshape(case.n, case.ldc)[:, case.m:]
    res["padding_ok"] = bool(np.array_equal(pad_in, pad_out, equal_nan=True))
    return res


def sample_points(m: int, n: int, count: int, seed: int, tile_m: int = 128, tile_n: int = 128):
    """Random entries plus every row/column on tile boundaries and the edges."""
    rng = np.random.default_rng(seed)
    rows = [rng.integers(0, m, count)]
    cols = [rng.integers(0, n, count)]
    edge_r = np.unique(np.clip(np.concatenate([np.arange(0, m, tile_m), np.arange(tile_m - 1, m, tile_m),
                                               [m - 1]]), 0, m - 1))
    edge_c = np.unique(np.clip(np.concatenate([np.arange(0, n, tile_n), np.arange(tile_n - 1, n, tile_n),
                                               [n - 1]]), 0, n - 1))
    rows.append(edge_r); cols.append(rng.integers(0, n, edge_r.size))
    rows.append(rng.integers(0, m, edge_c.size)); cols.append(edge_c)
    return np.concatenate(rows).astype(np.int32), np.concatenate(cols).astype(np.int32)


def check_sampled(case, a, b, c0, out, count=4096, seed=0) -> dict:
    rows, cols = sample_points(case.m, case.n, count, seed)
    ref, mag = oracle.sgemm_f64_points(case.transa, case.transb, case.k, case.alpha, a, case.lda, b,
                                       case.ldb, case.beta, c0, case.ldc, rows, cols)
    got = out[rows.astype(np.int64) + cols.astype(np.int64) * case.ldc]
    res = oracle.check(got, ref, mag, case.k)
    res["all_finite"] = bool(np.isfinite(c_view(out, case.m, case.n, case.ldc)).all())
    return res
