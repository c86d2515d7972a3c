"""Partition of the sage_attn (batch x head) grid across ranks, one process per GPU.

Every (batch, head) slab is independent (the reference's grid, triton_impl.py:186, is over
query blocks x heads x batches; nothing crosses heads), so ranks take contiguous ranges of the
flattened (b*H + h) index and compute them with no collective. The only data movement, when a
caller wants the whole output on one rank, is the final gather: each rank sends its finished
head ranges to the destination point-to-point, wave by wave, so that the transfer of wave w
overlaps the computation of wave w+1.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .inputs import make_inputs


def head_range(rank: int, world: int, total: int) -> tuple[int, int]:
    """Contiguous flattened-head range [lo, hi) of `rank` (sizes differ by at most one)."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of world {world}")
    return rank * total // world, (rank + 1) * total // world


def wave_ranges(lo: int, hi: int, waves: int) -> list[tuple[int, int]]:
    n = hi - lo
    waves = max(1, min(waves, n)) if n > 0 else 1
    return [(lo + w * n // waves, lo + (w + 1) * n // waves) for w in range(waves)]


@dataclass
class Shard:
    rank: int
    world: int
    lo: int
    hi: int
    total: int

    @property
    def heads(self) -> int:
        return self.hi - self.lo


def make_shard(case: dict, rank: int, world: int) -> Shard:
    total = case.get("batch_size", 8) * case.get("num_heads", 16)
    lo, hi = head_range(rank, world, total)
    return Shard(rank, world, lo, hi, total)


def shard_inputs(case: dict, shard: Shard, device, seed: int, dtype):
    """This rank's q/k/v as [1, heads, S, D] (the same values a 1-GPU run sees for these heads)."""
    return make_inputs(case, device, seed, dtype, heads=(shard.lo, shard.hi))


def gather_to(dst: int, out_local: torch.Tensor, shard: Shard, full: torch.Tensor | None, group=None,
              waves: int = 1, compute=None, timeout_s: float = 60.0):
    """Assemble every rank's [1, heads, S, D] output into `full` ([total, S, D] view) on rank `dst`.

    `compute(wave_lo, wave_hi)` (optional) fills out_local for one wave of this rank's heads
    before it is sent, so sends of finished waves overlap the computation of the next. The
    destination posts all its receives first, one group per wave (the peers' transfers of a
    wave run concurrently), so they land while it computes its own heads; `out_local` may be
    the destination's own slice of `full`, which is then not copied.
    Returns `full` on `dst`, None elsewhere. Uses point-to-point send/recv of contiguous head
    slices (works with NCCL on GPUs and gloo on CPUs). Every wait is bounded by `timeout_s`, so a
    rank that never sends (it failed) makes the destination raise instead of hang.
    """
    import datetime

    import torch.distributed as dist

    limit = datetime.timedelta(seconds=timeout_s)

    rank, world = shard.rank, shard.world
    local = out_local.reshape(shard.heads, *out_local.shape[2:])
    reqs = []
    flat = None
    if rank == dst:
        if full is None:
            raise ValueError("the destination rank needs the `full` output buffer")
        flat = full.reshape(shard.total, *full.shape[-2:])
        per_rank = [wave_ranges(*head_range(r, world, shard.total), waves) for r in range(world)]
        for w in range(waves):
            ops = [dist.P2POp(dist.irecv, flat[a:b], r, group=group)
                   for r in range(world) if r != dst and w < len(per_rank[r])
                   for (a, b) in [per_rank[r][w]] if b > a]
            if ops:
                reqs.extend(dist.batch_isend_irecv(ops))
    for (a, b) in wave_ranges(shard.lo, shard.hi, waves):
        if compute is not None:
            compute(a, b)
        if rank != dst and b > a:
            # a one-op batch: NCCL runs it as plain point to point, not as a serialised collective
            reqs.extend(dist.batch_isend_irecv(
                [dist.P2POp(dist.isend, local[a - shard.lo:b - shard.lo].contiguous(), dst, group=group)]))
    if rank == dst and shard.heads > 0 and local.data_ptr() != flat[shard.lo].data_ptr():
        flat[shard.lo:shard.hi].copy_(local)
    for q in reqs:
        q.wait(limit)
    return full if rank == dst else None
