"""Sequences and KV heads across the GPUs of one box.

Data-parallel sequences.  Independent sequences shard with no collective on
the data path: each rank (one process per GPU) owns the sequences ``s`` with
``s % world == rank`` and runs its own cache over them.  The only collectives
are the timing and the metric reductions around a measured region: the wall
time of a step is the maximum over ranks, throughput the sum of every rank's
tokens over that time.

KV heads of one sequence.  Rank ``i`` of ``world`` answers the attention of
KV heads ``[i H / world, (i + 1) H / world)`` and their query heads.  The
reference's basis is joint over the heads (bug_cache.py:605-607): an absorb
projects, scores and updates every head's keys together, so no rank can
maintain a head's share of the cache alone.  Every rank therefore computes
all KV heads' keys and values (``k_proj``/``v_proj`` whole) and keeps the
whole cache, stepping it identically (the same kernels on the same inputs);
the query projection is split by head, the factored kernels answer the
rank's head range, and one all-gather of the per-head attention outputs runs
before ``o_proj`` -- the only collective on the data path.

The helpers work on any ``torch.distributed`` backend (NCCL on the GPUs,
gloo on the host for tests; gloo gathers CUDA tensors through host memory).
"""

from __future__ import annotations

from datetime import timedelta

import torch
import torch.distributed as dist

__all__ = ["shard_sequences", "shard_heads", "GatherHeads", "shard_attention_heads", "max_over_ranks",
           "sum_over_ranks", "init_ranks"]


def shard_sequences(n_sequences: int, world: int, rank: int) -> list[int]:
    """The sequences rank ``rank`` of ``world`` owns (round-robin, so every
    rank's share differs by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return list(range(rank, n_sequences, world))


def shard_heads(num_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """``(first KV head, KV heads)`` rank ``rank`` of ``world`` answers:
    contiguous equal blocks, in rank order."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split over {world} ranks")
    hc = num_kv_heads // world
    return rank * hc, hc


def _all_gather_last(x: torch.Tensor, group: dist.ProcessGroup | None) -> torch.Tensor:
    """Concatenate every rank's ``x`` along the last dimension, in rank order."""
    world = dist.get_world_size(group)
    src = x.contiguous()
    if dist.get_backend(group) == "gloo":  # host-side exchange (CUDA tensors through host memory)
        parts = [torch.empty_like(src, device="cpu") for _ in range(world)]
        dist.all_gather(parts, src.cpu(), group=group)
        return torch.cat(parts, dim=-1).to(x.device)
    flat = torch.empty((world, *src.shape), dtype=src.dtype, device=src.device)
    dist.all_gather_into_tensor(flat, src, group=group)
    return flat.movedim(0, -2).reshape(*src.shape[:-1], world * src.shape[-1])


class GatherHeads(torch.nn.Module):
    """``o_proj`` preceded by the all-gather of every rank's attention output
    (its heads' features, ``(..., Hq_local * D)``) into the full
    ``(..., Hq * D)``; every rank then applies the whole projection."""

    def __init__(self, o_proj: torch.nn.Module, group: dist.ProcessGroup | None = None) -> None:
        super().__init__()
        self.o_proj = o_proj
        self.group = group

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1:
            x = _all_gather_last(x, self.group)
        return self.o_proj(x)


def shard_attention_heads(model: torch.nn.Module, rank: int, world: int,
                          group: dist.ProcessGroup | None = None) -> torch.nn.Module:
    """Split ``model``'s attention by KV head for rank ``rank`` of ``world``:
    each attention module keeps the ``q_proj`` rows (and bias) of its query
    heads and records its head range as ``kvd_heads``; ``k_proj``/``v_proj``
    and the cache stay whole; ``o_proj`` gets the all-gather in front
    (:class:`GatherHeads`).  Works on transformers models whose attention
    modules have ``q_proj``/``o_proj`` and a ``head_dim`` (Llama and its
    relatives).  Returns the model."""
    cfg = model.config
    H, Hq = int(cfg.num_key_value_heads), int(cfg.num_attention_heads)
    h0, hc = shard_heads(H, world, rank)
    G = Hq // H
    for mod in model.modules():
        if not (hasattr(mod, "q_proj") and hasattr(mod, "o_proj") and hasattr(mod, "head_dim")):
            continue
        if getattr(mod, "kvd_heads", None) is not None:
            raise RuntimeError("attention heads are already sharded")
        D = int(mod.head_dim)
        rows = slice(h0 * G * D, (h0 + hc) * G * D)
        old = mod.q_proj
        new = torch.nn.Linear(old.in_features, hc * G * D, bias=old.bias is not None,
                              device=old.weight.device, dtype=old.weight.dtype)
        with torch.no_grad():
            new.weight.copy_(old.weight[rows])
            if old.bias is not None:
                new.bias.copy_(old.bias[rows])
        mod.q_proj = new
        mod.o_proj = GatherHeads(mod.o_proj, group)
        mod.kvd_heads = (h0, hc)
    return model


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
