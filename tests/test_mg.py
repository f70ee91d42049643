"""Multi-GPU column-sharded SGEMM (sgblas_mg.h).

CPU part (gloo, world size 2, spawned processes): the host logic around the
collective -- the column split, the NCCL id exchange and the pre-flight
argument check that turns a mismatch into an error on every rank instead of a
hang.

GPU part, one GPU: communicator initialisation that fails, or never finishes,
injected on the host through a stand-in NCCL library (tests/fake_nccl.c); the
call must return an error within its deadline and abort the communicator.

GPU part, two GPUs (skipped with fewer): sgblasMgSgemm with A passed along the
copy-engine chain, each rank's shard checked against the FP64 oracle --
single and multi-panel A, both transposes of A, a transposed B, a root other
than rank 0, the TF32 lane, a rank with an invalid argument (it returns the
error, the other rank is unaffected and the next call still lines up), A
delivered to non-root ranks, and sgblasMgAllGather assembling C. Then a rank
that leaves between calls: the other rank's enqueued call waits for it,
sgblasMgAbort on the host releases the wait.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, fn, q):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        q.put((rank, fn(rank, world)))
    except Exception as e:  # report, do not hang the parent
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def _run_gloo(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


def test_shard_columns_cover_exactly():
    from sgblas_b200.mg import shard_columns, shard_sizes
    for n in (0, 1, 7, 32768, 32769):
        for world in (1, 2, 3, 4, 8):
            cols = []
            for r in range(world):
                first, count = shard_columns(n, world, r)
                cols.extend(range(first, first + count))
            assert cols == list(range(n))
            assert max(shard_sizes(n, world)) - min(shard_sizes(n, world)) <= 1
    with pytest.raises(ValueError):
        shard_columns(10, 2, 2)


def test_panel_plan():
    from sgblas_b200.mg import panel_plan
    for m, k, world in ((32768, 8192, 8), (4096, 2048, 2), (1500, 700, 2), (100000, 4096, 4),
                        (1024, 8192, 2), (5000, 8192, 1)):
        plan = panel_plan(m, k, world)
        assert plan[0][0] == 0 and sum(r for _, r in plan) == m
        assert all(a + r == b for (a, r), (b, _) in zip(plan, plan[1:]))
        assert len(plan) <= 16 and all(f % 128 == 0 for f, _ in plan)
    assert panel_plan(4096, 2048, 2) == [(0, 512), (512, 1024), (1536, 2560)]
    assert [r for _, r in panel_plan(32768, 8192, 8)][:3] == [512, 1024, 2048]
    assert panel_plan(1500, 700, 2) == [(0, 1500)]


def _uid_fn(rank, world):
    from sgblas_b200.mg import exchange_unique_id
    return exchange_unique_id(lambda: bytes(range(128)))


def test_unique_id_exchange_gloo():
    out = _run_gloo(_uid_fn)
    assert out[0] == out[1] == bytes(range(128))


def _consistent_fn(rank, world):
    from sgblas_b200.mg import check_consistent
    args = dict(transa=0, transb=0, m=64, k=32, alpha=1.0, beta=0.0, lda=64, root=0)
    check_consistent(args)                      # identical: passes
    bad = dict(args, k=32 + rank)               # rank 1 disagrees on k
    try:
        check_consistent(bad)
    except ValueError as e:
        return "raised: " + str(e)[:40]
    return "no error"


def test_mismatched_arguments_raise_on_every_rank():
    out = _run_gloo(_consistent_fn)
    assert all(v.startswith("raised") for v in out.values()), out


# ---- one GPU: injected NCCL initialisation failures ----------------------------
_CREATE_SCRIPT = r"""
import ctypes, json, os, sys, time
sys.path.insert(0, os.environ["SGBLAS_ROOT"])
import torch
import sgblas_b200 as sg
torch.cuda.set_device(0)
raw = ctypes.c_void_p()
uid = (ctypes.c_ubyte * 128)(*([7] * 128))
t0 = time.monotonic()
st = sg.lib.sgblasMgCreate(ctypes.byref(raw), 1, 0, uid, 0)
dt = time.monotonic() - t0
extra = None
if st == 0:
    h = sg.MgHandle.__new__(sg.MgHandle)
    h._h = raw
    m, n, k = 300, 200, 100
    a = torch.rand(m * k, device="cuda"); b = torch.rand(k * n, device="cuda")
    c = torch.zeros(m * n, device="cuda")
    h.sgemm(0, 0, m, n, k, 1.0, a, m, 0, b, k, 0.0, c, m)
    torch.cuda.synchronize()
    ref = (a.view(k, m).T.double() @ b.view(n, k).T.double())
    extra = float((c.view(n, m).T.double() - ref).abs().max())
    extra = [extra, h.close()]
print(json.dumps({"status": st, "seconds": dt, "extra": extra}))
"""


def _fake_nccl(tmp_path):
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    so = tmp_path / "libfakenccl.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", str(so),
                    os.path.join(ROOT, "tests", "fake_nccl.c")], check=True)
    return so


@pytest.mark.gpu
@pytest.mark.parametrize("mode,status", [("fail", 6), ("hang", 5), ("ok", 0)])
def test_communicator_init_failures_end_in_errors(cuda, tmp_path, mode, status):
    """sgblasMgCreate with a stand-in NCCL: an initialisation error gives
    INTERNAL_ERROR; one that never finishes gives EXECUTION_FAILED at the
    deadline (0.5 s here) and the communicator is aborted; a working one gives
    a handle whose products are right and whose destroy releases the
    communicator."""
    import json
    import subprocess
    so = _fake_nccl(tmp_path)
    log = tmp_path / "nccl.log"
    env = dict(os.environ, SGBLAS_NCCL_LIBRARY=str(so), FAKE_NCCL_MODE=mode,
               FAKE_NCCL_LOG=str(log), SGBLAS_MG_TIMEOUT_MS="500", SGBLAS_ROOT=ROOT)
    out = subprocess.run([sys.executable, "-c", _CREATE_SCRIPT], env=env, capture_output=True,
                         text=True, timeout=240)
    assert out.returncode == 0, out.stderr[-2000:]
    res = json.loads(out.stdout.strip().splitlines()[-1])
    assert res["status"] == status, res
    calls = log.read_text().split() if log.exists() else []
    assert calls[0] == "init"
    if mode == "hang":
        assert 0.4 <= res["seconds"] < 30, res
        assert calls[-1] == "abort", calls
    if mode == "fail":
        assert "abort" not in calls and "destroy" not in calls   # nothing was created
    if mode == "ok":
        err, close_status = res["extra"]
        assert err < 1e-3 and close_status == 0, res
        assert calls[-1] == "destroy", calls


# ---- two GPUs ---------------------------------------------------------------------
def _mg_spawn(scenario, world=2, timeout=600):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mg_worker, args=(r, world, port, q, scenario))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = dict(q.get(timeout=timeout) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return out


def _mg_worker(rank, world, port, q, scenario):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                          SGBLAS_MG_TIMEOUT_MS="60000")
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=120))
        import sgblas_b200 as sg
        from sgblas_b200.mg import exchange_unique_id
        h = sg.MgHandle(world, rank, exchange_unique_id(sg.mg_unique_id), rank)
        stream = torch.cuda.Stream()
        h.set_stream(stream)
        result = globals()[scenario](rank, world, h, stream)
        status = h.close()
        q.put((rank, (result, status)))
        dist.destroy_process_group()
    except Exception as e:  # report, do not hang the parent
        import traceback
        q.put((rank, f"error: {type(e).__name__}: {e}\n{traceback.format_exc()[-1500:]}"))


# (name, transa, transb, m, n, k, lda pad, ldb pad, ldc pad, alpha, beta, root, math, deliver A)
MG_CASES = [
    ("small-nn", 0, 0, 1500, 1000, 700, 3, 1, 5, 0.75, -0.5, 0, "fp32", True),
    ("panels-nn-root1", 0, 0, 4096, 600, 2048, 0, 0, 4, 1.0, 0.0, 1, "fp32", False),
    ("panels-tn", 1, 0, 4096, 512, 2048, 4, 0, 0, 1.0, 0.5, 0, "fp32", True),
    ("panels-nt", 0, 1, 4096, 520, 2048, 0, 3, 0, -1.25, 1.0, 1, "fp32", False),
    ("panels-tf32", 0, 0, 4096, 512, 2048, 0, 0, 0, 1.0, 0.0, 1, "tf32", True),
    ("bad-ldb-rank1", 0, 0, 4096, 512, 2048, 0, 0, 0, 1.0, 0.0, 0, "fp32", False),
    ("after-error", 0, 0, 4096, 512, 2048, 0, 0, 0, 0.5, 2.0, 0, "fp32", True),
    # every column on rank 0: rank 1 only passes A on (n_local = 0)
    ("all-on-0", 0, 0, 4096, 300, 2048, 0, 0, 0, 1.0, 0.0, 1, "fp32", True),
    # alpha = 0: nothing is sent, each rank scales its block of C
    ("scale-only", 0, 0, 1000, 600, 500, 0, 0, 2, 0.0, 0.5, 0, "fp32", False),
]


def _scenario_products(rank, world, h, stream):
    import oracle
    import sgblas_b200 as sg
    from sgblas_b200.mg import shard_columns
    out = []
    for idx, (name, ta, tb, m, n, k, pa, pb, pc, alpha, beta, root, math, deliver) in \
            enumerate(MG_CASES):
        h.set_math_mode(sg.SGBLAS_MATH_TF32 if math == "tf32" else sg.SGBLAS_MATH_FP32)
        lda = (k if ta else m) + pa
        ldb = (n if tb else k) + pb
        ldc = m + pc
        rng = oracle.Rng(100 + idx)           # the same full problem on every rank
        a = rng.uniform(lda * (m if ta else k))
        b = rng.uniform(ldb * (k if tb else n))
        c = rng.uniform(ldc * n)
        first, cols = shard_columns(n, world, rank)
        if name == "all-on-0":
            first, cols = (0, n) if rank == 0 else (n, 0)
        if tb:   # op(B) columns are rows of the stored n x k matrix
            b_loc = np.ascontiguousarray(b.reshape(k, ldb)[:, first:first + cols]).ravel()
            ldb_loc = max(cols, 1)
        else:
            b_loc = np.ascontiguousarray(b.reshape(n, ldb)[first:first + cols]).ravel()
            ldb_loc = ldb
        c_loc = np.ascontiguousarray(c.reshape(n, ldc)[first:first + cols]).ravel()
        if rank == root:
            da = torch.from_numpy(a).cuda()
        elif deliver:
            da = torch.full((a.size,), float("nan"), device="cuda")
        else:
            da = None
        if cols == 0:   # no block of its own: any valid pointers (never read)
            b_loc = c_loc = np.zeros(1, np.float32)
        db, dc = torch.from_numpy(b_loc).cuda(), torch.from_numpy(c_loc).cuda()
        if name == "bad-ldb-rank1" and rank == 1:
            ldb_loc = 0   # invalid on this rank only
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            status = h.sgemm_status(ta, tb, m, cols, k, alpha, da, lda, root, db, ldb_loc, beta,
                                    dc, ldc)
        torch.cuda.synchronize()
        res = {"case": name, "status": status}
        if status == 0 and cols == 0:
            res.update(ok=True, padding_ok=True)
            if da is not None and rank != root:
                rows_used = k if ta else m
                got_a = da.cpu().numpy().reshape(-1, lda)[:, :rows_used]
                res["a_delivered"] = bool(np.array_equal(got_a, a.reshape(-1, lda)[:, :rows_used]))
        elif status == 0:
            got = dc.cpu().numpy().reshape(cols, ldc).T[:m, :].astype(np.float64)
            ref, mag = oracle.sgemm_f64(ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc,
                                        cols=(first, first + cols))
            bound = (2.0 ** -9 + (k + 2) * 2.0 ** -22) * mag if math == "tf32" else \
                oracle.tol_north_star(k, mag)
            err = np.abs(got - ref)
            res["ok"] = bool(np.all(np.isfinite(got)) and np.all(err <= bound))
            res["max_ratio"] = float(np.max(err / np.maximum(bound, 1e-30)))
            res["padding_ok"] = bool(np.array_equal(
                dc.cpu().numpy().reshape(cols, ldc)[:, m:], c_loc.reshape(cols, ldc)[:, m:]))
            if da is not None and rank != root:
                rows_used = k if ta else m
                got_a = da.cpu().numpy().reshape(-1, lda)[:, :rows_used]
                res["a_delivered"] = bool(np.array_equal(got_a, a.reshape(-1, lda)[:, :rows_used]))
        out.append(res)
    h.set_math_mode(sg.SGBLAS_MATH_FP32)
    # sgblasMgAllGather assembles C from equal shards (ldc == m).
    m, n, k = 1024, 2 * 300, 512
    rng = oracle.Rng(999)
    a, b = rng.uniform(m * k), rng.uniform(k * n)
    first, cols = shard_columns(n, world, rank)
    da = torch.from_numpy(a).cuda() if rank == 0 else None
    db = torch.from_numpy(np.ascontiguousarray(b.reshape(n, k)[first:first + cols]).ravel()).cuda()
    dc = torch.empty(m * cols, device="cuda")
    full = torch.full((m * n,), float("nan"), device="cuda")
    with torch.cuda.stream(stream):
        h.sgemm(0, 0, m, cols, k, 1.0, da, m, 0, db, k, 0.0, dc, m)
        h.all_gather(dc, full, m * cols)
    torch.cuda.synchronize()
    ref, mag = oracle.sgemm_f64(0, 0, m, n, k, 1.0, a, m, b, k, 0.0, None, m)
    got = full.cpu().numpy().reshape(n, m).T
    out.append({"case": "all-gather", "status": 0,
                "ok": bool(oracle.check(got, ref, mag, k)["ok_north_star"]),
                "padding_ok": True})
    return out


@pytest.mark.gpu
def test_mg_sgemm_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = _mg_spawn("_scenario_products", timeout=300)
    for rank, v in out.items():
        assert isinstance(v, tuple), (rank, v)
        results, close_status = v
        assert close_status == 0, (rank, close_status)
        for res in results:
            if res["case"] == "bad-ldb-rank1" and rank == 1:
                assert res["status"] == 3, res          # INVALID_VALUE, no hang
                continue
            assert res["status"] == 0, (rank, res)
            assert res["ok"] and res["padding_ok"], (rank, res)
            if "a_delivered" in res:
                assert res["a_delivered"], (rank, res)


def _scenario_leaver(rank, world, h, stream):
    """Rank 1 leaves between calls; rank 0's second call waits for it until
    its host learns of the departure (a gloo barrier) and aborts."""
    import time
    m, n, k = 4096, 256, 2048
    a = torch.rand(m * k, device="cuda") if rank == 0 else None
    b = torch.rand(k * n, device="cuda")
    c = torch.zeros(m * n, device="cuda")
    with torch.cuda.stream(stream):
        h.sgemm(0, 0, m, n, k, 1.0, a, m, 0, b, k, 0.0, c, m)   # both ranks: staging set up
    torch.cuda.synchronize()
    dist.barrier()
    result = {}
    if rank == 0:
        with torch.cuda.stream(stream):
            h.sgemm(0, 0, m, n, k, 1.0, a, m, 0, b, k, 0.0, c, m)
        time.sleep(2.0)
        result["blocked"] = not stream.query()   # waiting for rank 1's staging
        dist.barrier()                            # rank 1 has left the computation
        h.abort()
        t0 = time.monotonic()
        while not stream.query() and time.monotonic() - t0 < 30:
            time.sleep(0.01)
        result["released"] = stream.query()
        result["later_call"] = h.sgemm_status(0, 0, m, n, k, 1.0, a, m, 0, b, k, 0.0, c, m)
    else:
        dist.barrier()                            # announces its departure
    dist.barrier()
    return result


@pytest.mark.gpu
def test_mg_abort_releases_a_waiting_call():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = _mg_spawn("_scenario_leaver", timeout=300)
    assert isinstance(out[0], tuple) and isinstance(out[1], tuple), out
    res0, _ = out[0]
    assert res0["blocked"] and res0["released"], res0
    assert res0["later_call"] == 5, res0   # EXECUTION_FAILED after the abort
