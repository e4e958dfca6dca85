"""Data-parallel serving over one process per GPU.

The batched decode has no cross-GPU data dependency: every rank holds a full
weight replica and its own sequences.  This module holds the host-side logic
that does cross ranks — the partition of the job's sequences, the waves a
rank decodes them in, and the max-over-ranks reduction of a device-timed
interval — so it can be tested with CPU (``gloo``) process groups.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    """Rank ``rank``'s slice ``[begin, end)`` of the job's sequences, decoded
    in ``n_waves`` waves of ``wave`` sequences."""
    rank: int
    world: int
    begin: int
    end: int
    n_waves: int
    wave: int

    @property
    def n(self) -> int:
        return self.end - self.begin

    def wave_slice(self, i: int) -> tuple[int, int]:
        """Global sequence indices of wave ``i``."""
        b = self.begin + i * self.wave
        return b, b + self.wave


def shard(total: int, world: int, rank: int, max_wave: int = 256) -> Shard:
    """Even partition of ``total`` sequences over ``world`` ranks (contiguous
    slices, rank order), each rank's slice cut into equal waves of at most
    ``max_wave``.  ``world`` must divide ``total`` and the per-rank count must
    split into equal waves."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    if total % world:
        raise ValueError(f"world size {world} must divide {total}")
    n = total // world
    n_waves = (n + max_wave - 1) // max_wave
    if n % n_waves:
        raise ValueError(f"{n} sequences do not split into {n_waves} equal waves")
    return Shard(rank, world, rank * n, (rank + 1) * n, n_waves, n // n_waves)


def max_over_ranks(value: float, device=None) -> float:
    """Max of ``value`` over the default process group (identity without
    one).  Every rank must call it, in the same order."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_ranks(value: float, device=None) -> list:
    """``value`` of every rank of the default process group, in rank order
    (``[value]`` without one).  Every rank must call it, in the same order."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [float(value)]
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    out = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]
