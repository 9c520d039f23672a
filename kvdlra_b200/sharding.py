"""Data-parallel sequences across the GPUs of one box.

Independent sequences shard with no collective on the data path: each rank
(one process per GPU) owns the sequences ``s`` with ``s % world == rank`` and
runs its own cache over them.  The only collectives are the timing and the
metric reductions around a measured region: the wall time of a step is the
maximum over ranks, throughput the sum of every rank's tokens over that time.
The helpers work on any ``torch.distributed`` backend (NCCL on the GPUs,
gloo on the host for tests).
"""

from __future__ import annotations

from datetime import timedelta

import torch
import torch.distributed as dist

__all__ = ["shard_sequences", "max_over_ranks", "sum_over_ranks", "init_ranks"]


def shard_sequences(n_sequences: int, world: int, rank: int) -> list[int]:
    """The sequences rank ``rank`` of ``world`` owns (round-robin, so every
    rank's share differs by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return list(range(rank, n_sequences, world))


def _reduce(values: list[float], op: dist.ReduceOp, device: torch.device | None) -> list[float]:
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return [float(v) for v in values]
    t = torch.tensor(values, dtype=torch.float64, device=device or torch.device("cpu"))
    dist.all_reduce(t, op=op)
    return [float(v) for v in t.tolist()]


def max_over_ranks(values: list[float], device: torch.device | None = None) -> list[float]:
    """Element-wise maximum of per-rank values (step times)."""
    return _reduce(values, dist.ReduceOp.MAX, device)


def sum_over_ranks(values: list[float], device: torch.device | None = None) -> list[float]:
    """Element-wise sum of per-rank values (tokens processed)."""
    return _reduce(values, dist.ReduceOp.SUM, device)


def init_ranks(backend: str, device: torch.device | None, timeout_s: float = 600.0) -> tuple[int, int]:
    """Join the process group torchrun describes (RANK / WORLD_SIZE /
    MASTER_*), with a bounded timeout so a rank that never arrives ends the
    others' collective with an error; returns ``(rank, world)``."""
    kw = {"timeout": timedelta(seconds=timeout_s)}
    if backend == "nccl" and device is not None:
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
    return dist.get_rank(), dist.get_world_size()
