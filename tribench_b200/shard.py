"""Partition of the sage_attn (batch x head) grid across ranks, one process per GPU.

Every (batch, head) slab is independent (the reference's grid, triton_impl.py:186, is over
query blocks x heads x batches; nothing crosses heads), so ranks take contiguous ranges of the
flattened (b*H + h) index and compute them with no collective. The only data movement, when a
caller wants the whole output on one rank, is the final gather, in one of three forms:
  * CopyGather (over a PeerOutput): the destination's output buffer is mapped into every rank
    (CUDA IPC with peer access over NVLink); each rank computes its heads in waves into its own
    memory, on two compute streams so that consecutive waves overlap (no SM idles at a wave's
    end), and a copy stream sends every finished wave into the mapping with the copy engine
    (cudaMemcpyAsync, no SM involved) while the next waves compute;
  * PeerOutput alone: each rank's attention kernel stores its heads' rows straight into the
    mapping from its epilogue — no extra pass, but SM stores into another GPU's memory reach
    only ~170 GB/s at the destination on B200, a quarter of what the copy engine moves;
  * gather_to: each rank sends its finished head ranges to the destination point to point
    (NCCL on GPUs, gloo on CPUs), wave by wave, so that the transfer of wave w overlaps the
    computation of wave w+1.
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


class _CudaArray:
    """A bare device pointer presented through the CUDA array interface (bytes, no ownership)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerOutput:
    """The whole job's output `[*shape]` of `dtype`, resident on rank `dst`'s GPU and mapped into
    every rank of `group`: ``.tensor`` views it on every rank (on rank `dst` it is local memory;
    elsewhere a peer mapping of it, opened with CUDA IPC and NVLink peer access), so a rank that
    computes into its slice of ``.tensor`` stores its rows directly into rank `dst`'s memory.

    Collective: every rank of the group constructs it (one broadcast of the 64-byte IPC handle).
    ``close()`` is collective too: the mappings are closed before the owner frees the buffer.
    Rank `dst` allocates the buffer with cudaMalloc (outside torch's caching allocator, so the
    IPC handle describes exactly this buffer). Stores from other ranks become visible on `dst`
    once their kernels complete; a barrier after those kernels (e.g. the one that ends a timed
    region) orders them before `dst` reads the output."""

    def __init__(self, shape, dtype: torch.dtype, dst: int, device, group=None):
        import math

        import torch.distributed as dist
        from cuda.bindings import runtime as rt

        self._rt, self._group, self._dst = rt, group, dst
        self.dst = dst
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.nbytes = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
        self._ptr = None

        def ok(res, what):
            err = res[0] if isinstance(res, tuple) else res
            if err != rt.cudaError_t.cudaSuccess:
                raise RuntimeError(f"{what} failed: {err}")
            return res[1] if isinstance(res, tuple) and len(res) > 1 else None

        self._ok = ok
        with torch.cuda.device(self.device):
            if self.rank == dst:
                self._ptr = int(ok(rt.cudaMalloc(self.nbytes), "cudaMalloc"))
                handle = ok(rt.cudaIpcGetMemHandle(self._ptr), "cudaIpcGetMemHandle")
                payload = [bytes(handle.reserved)]
            else:
                payload = [None]
            dist.broadcast_object_list(payload, src=dst, group=group, device=self.device)
            if self.rank != dst:
                handle = rt.cudaIpcMemHandle_t()
                handle.reserved = payload[0]
                self._ptr = int(ok(rt.cudaIpcOpenMemHandle(handle, rt.cudaIpcMemLazyEnablePeerAccess),
                                   "cudaIpcOpenMemHandle"))
        self.tensor = torch.as_tensor(_CudaArray(self._ptr, self.nbytes)).view(dtype).view(*shape)

    def close(self):
        import torch.distributed as dist

        if self._ptr is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self._group)
        with torch.cuda.device(self.device):
            if self.rank != self._dst:
                self._ok(self._rt.cudaIpcCloseMemHandle(self._ptr), "cudaIpcCloseMemHandle")
        dist.barrier(group=self._group)
        if self.rank == self._dst:
            with torch.cuda.device(self.device):
                self._ok(self._rt.cudaFree(self._ptr), "cudaFree")
        self.tensor = None
        self._ptr = None


class CopyGather:
    """Per-step driver of the copy-engine gather into a PeerOutput (see the module docstring).

    ``step(waves, compute)`` runs ``compute(a, b, slot)`` for every head range [a, b) of this
    rank, alternating between the caller's current stream (slot 0) and a second stream (slot 1);
    ``compute`` launches on the current stream and uses per-slot buffers, so two waves never
    share scratch. On ranks other than the destination each finished wave's rows,
    ``out_local[:, a - lo : b - lo]``, are then copied into ``peer.tensor[:, a:b]`` on a copy
    stream; the destination computes into its slice of the buffer directly (``out_local`` is
    that slice there). Everything is joined back into the current stream before ``step``
    returns, so an event recorded after it covers the whole step, copies included.

    Returns the step's CUDA events (start, compute end per slot, copy end), for timing."""

    def __init__(self, peer: "PeerOutput", lo: int, out_local: torch.Tensor):
        self.peer, self.lo, self.out_local = peer, lo, out_local
        self.send = peer.rank != peer.dst
        self.alt = torch.cuda.Stream(peer.device)
        self.copy = torch.cuda.Stream(peer.device)

    def step(self, waves, compute):
        main = torch.cuda.current_stream(self.peer.device)
        ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
        start, end_main, end_alt, end_copy = ev(), ev(), ev(), ev()
        start.record(main)
        self.alt.wait_stream(main)
        self.copy.wait_stream(main)
        streams = (main, self.alt)
        for w, (a, b) in enumerate(waves):
            s = streams[w % 2]
            with torch.cuda.stream(s):
                compute(a, b, w % 2)
            if self.send:
                done = torch.cuda.Event()
                done.record(s)
                self.copy.wait_event(done)
                with torch.cuda.stream(self.copy):
                    self.peer.tensor[:, a:b].copy_(self.out_local[:, a - self.lo:b - self.lo], non_blocking=True)
        end_main.record(main)
        end_alt.record(self.alt)
        end_copy.record(self.copy)
        main.wait_stream(self.alt)
        main.wait_stream(self.copy)
        return start, end_main, end_alt, end_copy
