"""Multi-GPU column-sharded SGEMM.

CPU part (gloo, world size 2, spawned processes): the host logic around the
collective -- the column split, the NCCL id exchange and the pre-flight
argument check that turns a mismatch into an error on every rank instead of a
hang. GPU part (needs 2 GPUs; skipped otherwise): sgblasMgSgemm over NCCL, each
rank's shard checked against the FP64 oracle.
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


# ---- 2 GPUs ---------------------------------------------------------------------
def _mg_worker(rank, world, port, q):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=120))
        import oracle
        import sgblas_b200 as sg
        from sgblas_b200.mg import check_consistent, exchange_unique_id, shard_columns
        from tests.gpu_util import sample_points
        m, n, k = 1500, 1000, 700
        lda, ldb, ldc = m + 3, k + 1, m + 5
        alpha, beta = 0.75, -0.5
        rng = oracle.Rng(31)                 # identical full problem on every rank
        a = rng.uniform(lda * k)
        b = rng.uniform(ldb * n)
        c = rng.uniform(ldc * n)
        first, cols = shard_columns(n, world, rank)
        b_loc = np.ascontiguousarray(b.reshape(n, ldb)[first:first + cols]).ravel()
        c_loc = np.ascontiguousarray(c.reshape(n, ldc)[first:first + cols]).ravel()
        da = torch.from_numpy(a).cuda() if rank == 0 else torch.full((lda * k,), float("nan"),
                                                                        device="cuda")
        db, dc = torch.from_numpy(b_loc).cuda(), torch.from_numpy(c_loc).cuda()
        check_consistent(dict(transa=0, transb=0, m=m, k=k, alpha=alpha, beta=beta, lda=lda,
                              root=0))
        h = sg.MgHandle(world, rank, exchange_unique_id(sg.mg_unique_id), rank)
        h.sgemm(0, 0, m, cols, k, alpha, da, lda, 0, db, ldb, beta, dc, ldc)
        torch.cuda.synchronize()
        h.close()
        out = dc.cpu().numpy()
        a_ok = bool(np.array_equal(da.cpu().numpy(), a))    # the broadcast delivered A
        ref, mag = oracle.sgemm_f64(0, 0, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc,
                                    cols=(first, first + cols))
        res = oracle.check(out.reshape(cols, ldc).T[:m, :], ref, mag, k)
        q.put((rank, (a_ok, res["ok_north_star"], res["max_ratio_north_star"])))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, f"error: {type(e).__name__}: {e}"))


@pytest.mark.gpu
def test_mg_sgemm_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mg_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, v in out.items():
        assert isinstance(v, tuple), (rank, v)
        a_ok, ok, ratio = v
        assert a_ok and ok, (rank, v)
