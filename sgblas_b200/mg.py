"""Host-side helpers for the column-sharded multi-GPU SGEMM (sgblas_mg.h).

One process per GPU. These helpers hold the host logic around the collective
C entry point ``sgblasMgSgemm``, and need no GPU (they are tested with
``gloo`` ranks on CPU):

* :func:`shard_columns` -- the column block of C and op(B) a rank owns (the
  split the bench and the tests use; the C API accepts any per-rank n_local).
* :func:`exchange_unique_id` -- rank 0 creates the NCCL id, every rank gets it.
* :func:`check_consistent` -- before entering the collective, every rank's
  problem-wide arguments are compared on the host; a mismatch raises on every
  rank instead of leaving ranks waiting for panels of A that never come.
* :func:`panel_plan` -- the row panels in which sgblasMgSgemm sends A (one
  product launch per panel per rank), the rule of planPanels in
  csrc/mg.cu.
"""
from __future__ import annotations

from typing import Callable, Sequence


def shard_columns(n: int, world: int, rank: int) -> tuple[int, int]:
    """(first column, column count) of rank's block of n columns: equal blocks,
    the first n % world ranks one column larger."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard request n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def exchange_unique_id(make_id: Callable[[], bytes], group=None) -> bytes:
    """Rank 0 calls make_id(); the bytes reach every rank of the group."""
    import torch.distributed as dist

    box = [make_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group else 0,
                               group=group)
    return box[0]


# The arguments of sgblasMgSgemm that must be identical on every rank.
UNIFORM_ARGS = ("transa", "transb", "m", "k", "alpha", "beta", "lda", "root")


def check_consistent(args: dict, group=None) -> None:
    """Raises ValueError on every rank if the problem-wide arguments differ."""
    import torch.distributed as dist

    mine = tuple(args[name] for name in UNIFORM_ARGS)
    everyone: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(everyone, mine, group=group)
    bad = [r for r, theirs in enumerate(everyone) if theirs != everyone[0]]
    if bad:
        raise ValueError(f"sgblasMgSgemm arguments differ on ranks {bad}: "
                         f"{dict(zip(UNIFORM_ARGS, everyone[bad[0]]))} vs "
                         f"{dict(zip(UNIFORM_ARGS, everyone[0]))}")


def shard_sizes(n: int, world: int) -> Sequence[int]:
    return [shard_columns(n, world, r)[1] for r in range(world)]


PANEL_SPLIT_BYTES = 32 << 20
MAX_PANELS = 16


def panel_plan(m: int, k: int, nranks: int) -> list[tuple[int, int]]:
    """(first row, rows) of each panel of op(A) (m x k floats) that
    sgblasMgSgemm sends along the chain: one panel for one rank, a small A
    (< 32 MiB) or m < 1024; else 512, 1024 and 2048 rows while at least twice
    that many rows remain, then the rest in at most 16 - (ramp panels)
    near-equal panels of about 4096 rows, rounded up to multiples of 128."""
    if nranks == 1 or m * k * 4 < PANEL_SPLIT_BYTES or m < 1024:
        return [(0, m)]
    out, at, rows = [], 0, 512
    while rows <= 2048 and m - at >= 2 * rows:
        out.append((at, rows))
        at += rows
        rows *= 2
    rest = m - at
    count = max(1, min(MAX_PANELS - len(out), (rest + 4095) // 4096))
    step = (rest // count + 127) // 128 * 128
    for i in range(count):
        if at >= m:
            break
        take = m - at if i == count - 1 else min(step, m - at)
        out.append((at, take))
        at += take
    return out
