"""Float-equivalent memory accounting of the streaming-BUG cache.

Mirrors the BUG part of kvdlra's ``accounting.py`` (src/kvdlra/accounting.py:
53-191, 363-450): the same unit (one fp32 word per stored element, bf16
verbatim elements counted as one element each), the same component rules, so
``bug_footprint(...).float_equiv()`` equals
:meth:`kvdlra_b200.BugStreamingCache.stored_state_numel` for the same state.

Conventions:
* verbatim K/V and basis/coordinate elements: 1 float-equivalent each;
* the diagonal BUG core: ``r`` per stream (not ``r**2``);
* positions (int32) and surprise scores (fp32): 1 each;
* quantised codes: ``bits/32`` each, ``ceil`` over all codes;
* the full fp16 cache: ``2*T*n`` elements per layer (``2*T*n*16`` bits).
"""

from __future__ import annotations

import math
from collections.abc import Callable, Iterator
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Any

FP16_BITS = 16
FP32_BITS = 32
N_SINK = 4

_TRACK_SCORE = ("attn", "blend")
_TRACK_SURPRISE = ("lowrank_surprise", "blend")

__all__ = [
    "Footprint", "MemoryReport", "bug_footprint", "bug_footprint_saturated",
    "bug_prefill_footprint", "full_cache_footprint", "measure_peak_gpu", "report",
    "audit_matched", "assert_all_within",
]


@dataclass(frozen=True)
class Footprint:
    """Per-layer stored footprint: verbatim elements, packed code bits and fp32
    bookkeeping words (accounting.py:53-103)."""

    verbatim_elems: float
    quant_code_bits: float = 0.0
    aux_words: float = 0.0
    gpu_verbatim_elems: float | None = None
    cpu_verbatim_elems: float = 0.0

    def float_equiv(self) -> float:
        codes = math.ceil(self.quant_code_bits / 32) if self.quant_code_bits else 0
        return self.verbatim_elems + codes + self.aux_words

    def bits(self, store_bits: int = FP16_BITS) -> float:
        return self.verbatim_elems * store_bits + self.quant_code_bits + self.aux_words * FP32_BITS

    def ratio_fp16(self, t: int, n: int) -> float:
        return self.bits(FP16_BITS) / (2 * t * n * FP16_BITS)

    def tok_equiv(self, n: int) -> float:
        return self.float_equiv() / (2 * n)

    def gpu_ratio_fp16(self, t: int, n: int) -> float:
        gpu = self.verbatim_elems if self.gpu_verbatim_elems is None else self.gpu_verbatim_elems
        return (gpu * FP16_BITS + self.quant_code_bits + self.aux_words * FP32_BITS) / (2 * t * n * FP16_BITS)

    def cpu_ratio_fp16(self, t: int, n: int) -> float:
        return self.cpu_verbatim_elems * FP16_BITS / (2 * t * n * FP16_BITS)


def bug_footprint(
    n: int,
    rank: int,
    coord_count: int,
    recent_len: int,
    *,
    n_sink: int = N_SINK,
    retention: str = "fifo",
    hh_count: int = 0,
    hh_select: str = "attn",
    merge: bool = False,
    u_present: bool = True,
    quant_count: int = 0,
    quant_bits: int | None = None,
    w_key: bool = False,
) -> Footprint:
    """One streaming layer's footprint (accounting.py:109-164): sinks and ring
    verbatim (``2n`` per token), ``2*rank`` per coordinate column, ``2n`` per
    exact-tier token, basis ``2*n*rank`` + diagonal cores ``2*rank`` when a basis
    exists, and the bookkeeping words of the retention rule."""
    track_pos = retention != "fifo" or merge
    track_score = retention in _TRACK_SCORE
    track_surprise = retention in _TRACK_SURPRISE
    n_cols = coord_count + quant_count
    verbatim = 2 * n * n_sink + 2 * n * recent_len + 2 * rank * coord_count + 2 * n * hh_count
    aux = 0.0
    if u_present:
        verbatim += 2 * n * rank
        aux += 2 * rank
    aux += n_cols * (int(track_pos) + int(track_score) + int(merge) + int(track_surprise))
    if track_score:
        aux += recent_len
    aux += hh_count * (2 if hh_select == "attn" else 1)
    code_bits = 0.0
    if quant_count and quant_bits is not None:
        code_bits = 2 * rank * quant_count * quant_bits
        aux += 2 * quant_count
    if w_key:
        aux += n
    return Footprint(verbatim_elems=verbatim, quant_code_bits=code_bits, aux_words=aux)


def bug_footprint_saturated(
    n: int,
    rank: int,
    coord_budget: int,
    recent_window: int,
    absorb_block: int,
    *,
    n_sink: int = N_SINK,
    retention: str = "fifo",
    hh_budget: int = 0,
) -> Footprint:
    """High-water footprint: ``coord_budget`` columns and the ring at
    ``recent_window + absorb_block - 1`` (accounting.py:167-191)."""
    return bug_footprint(n, rank, coord_budget, recent_window + absorb_block - 1,
                         n_sink=n_sink, retention=retention, hh_count=hh_budget)


def bug_prefill_footprint(t: int, n: int, rank: int, *, n_sink: int = N_SINK,
                          quant_bits: int | None = None) -> Footprint:
    """The prefill-press model: every non-sink token as a coordinate, the basis
    and exact sinks, no ring or core (accounting.py:194-213)."""
    t_pay = t - n_sink
    verbatim = 2 * n * n_sink + 2 * n * rank
    if quant_bits is None:
        return Footprint(verbatim_elems=verbatim + 2 * rank * t_pay)
    return Footprint(verbatim_elems=verbatim + t_pay, quant_code_bits=2 * rank * t_pay * quant_bits)


def full_cache_footprint(t: int, n: int) -> Footprint:
    """The uncompressed reference: ``2*t*n`` verbatim elements per layer."""
    return Footprint(verbatim_elems=2 * t * n)


@contextmanager
def measure_peak_gpu(device: str) -> Iterator[Callable[[], int | None]]:
    """Getter for ``torch.cuda.max_memory_allocated`` over the block (``None``
    off-GPU), reported beside -- never instead of -- the analytic footprint."""
    import torch

    if str(device).startswith("cuda"):
        torch.cuda.reset_peak_memory_stats()
        torch.cuda.synchronize()
        yield lambda: int(torch.cuda.max_memory_allocated())
    else:
        yield lambda: None


@dataclass(frozen=True)
class MemoryReport:
    arm: str
    t: int
    n: int
    float_equiv_per_layer: float
    tok_equiv_per_layer: float
    ratio_fp16: float
    gpu_ratio_fp16: float
    cpu_ratio_fp16: float
    bytes_native: int
    peak_gpu_bytes: int | None
    detail: dict[str, Any] = field(default_factory=dict)


def report(arm: str, footprint: Footprint, t: int, n: int, *, store_bits: int = FP16_BITS,
           peak_gpu_bytes: int | None = None, detail: dict[str, Any] | None = None) -> MemoryReport:
    """Render a footprint into the report fields (accounting.py:399-424)."""
    return MemoryReport(
        arm=arm, t=t, n=n,
        float_equiv_per_layer=footprint.float_equiv(),
        tok_equiv_per_layer=footprint.tok_equiv(n),
        ratio_fp16=footprint.ratio_fp16(t, n),
        gpu_ratio_fp16=footprint.gpu_ratio_fp16(t, n),
        cpu_ratio_fp16=footprint.cpu_ratio_fp16(t, n),
        bytes_native=int(footprint.bits(store_bits) / 8),
        peak_gpu_bytes=peak_gpu_bytes,
        detail=detail or {},
    )


def audit_matched(mem_max_per_layer: float, budget_per_layer: float, arm: str, *,
                  tol: float = 0.0) -> dict[str, Any]:
    within = mem_max_per_layer <= budget_per_layer + tol
    over = mem_max_per_layer / budget_per_layer if budget_per_layer else math.inf
    return {"arm": arm, "mem_max": mem_max_per_layer, "over_budget": over, "within": within}


def assert_all_within(mem_by_arm: dict[str, float], budget_per_layer: float, *,
                      tol: float = 0.0) -> None:
    """Raise if any arm's per-layer footprint exceeds the matched budget."""
    over = {a: m for a, m in mem_by_arm.items() if m > budget_per_layer + tol}
    if over:
        raise ValueError(
            f"matched-memory audit FAILED: {over} exceed budget {budget_per_layer}/layer"
        )
