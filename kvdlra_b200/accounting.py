"""Float-equivalent charge of the streaming-BUG cache.

Every stored element costs one float-equivalent, whatever its storage type:
a bf16 verbatim key is one, an fp32 coordinate is one, an int32 position is
one.  The charge of a layer is built here as a table of components -- what is
stored, how many items, how many elements per item, and whether the elements
are model-dtype payload ("verbatim", priced at the storage width in bit
ratios) or fp32/int bookkeeping (priced at 32 bits).  The total of that table
is, by construction, the number :meth:`BugStreamingCache.stored_state_numel`
measures for the same state (the reference pins the same equality for its
formula, src/kvdlra/accounting.py:109-191 against bug_cache.py:1609-1675).

Scope is the surprise-selected streaming path: retention ``"fifo"`` or
``"lowrank_surprise"``, an exact tier selected by surprise, and the BUGPress
prefill model.  The research tiers (PolarQuant codes, merge, Q-BUG whitening,
attention-scored retention) are refused with ``NotImplementedError`` rather
than priced by a formula nothing here can measure.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

__all__ = ["Component", "Footprint", "bug_footprint", "bug_footprint_saturated",
           "bug_prefill_footprint", "full_cache_footprint", "assert_all_within"]

FP16_BITS = 16
WORD_BITS = 32


@dataclass(frozen=True)
class Component:
    """``items`` stored things of ``size`` elements each."""

    name: str
    items: int
    size: int
    verbatim: bool  # model-dtype payload (else fp32 / integer bookkeeping)

    @property
    def elems(self) -> int:
        return self.items * self.size


@dataclass(frozen=True)
class Footprint:
    """A layer's stored state as a component table."""

    parts: tuple[Component, ...]

    def float_equiv(self) -> int:
        """Total stored elements (the unit of ``stored_state_numel``)."""
        return sum(p.elems for p in self.parts)

    def breakdown(self) -> dict[str, int]:
        out: dict[str, int] = {}
        for p in self.parts:
            out[p.name] = out.get(p.name, 0) + p.elems
        return out

    def bits(self, store_bits: int = FP16_BITS) -> int:
        """Bits with payload at ``store_bits`` and bookkeeping at 32."""
        return sum(p.elems * (store_bits if p.verbatim else WORD_BITS) for p in self.parts)

    def ratio_fp16(self, t: int, n: int) -> float:
        """Bits against the uncompressed fp16 K+V cache of ``t`` tokens."""
        return self.bits(FP16_BITS) / (2 * t * n * FP16_BITS)

    def tok_equiv(self, n: int) -> float:
        """Float-equivalents expressed as full-cache tokens (``2n`` each)."""
        return self.float_equiv() / (2 * n)


def _table(rows: list[tuple[str, int, int, bool]]) -> Footprint:
    return Footprint(tuple(Component(*r) for r in rows if r[1] > 0 and r[2] > 0))


def bug_footprint(
    n: int,
    rank: int,
    coord_count: int,
    recent_len: int,
    *,
    n_sink: int = 4,
    retention: str = "fifo",
    hh_count: int = 0,
    hh_select: str = "attn",
    merge: bool = False,
    u_present: bool = True,
    quant_count: int = 0,
    quant_bits: int | None = None,
    w_key: bool = False,
) -> Footprint:
    """One streaming layer holding ``coord_count`` coordinate columns,
    ``recent_len`` ring tokens, ``n_sink`` sinks and ``hh_count`` exact-tier
    tokens (the reference's ``bug_footprint`` signature,
    src/kvdlra/accounting.py:109-164).

    K and V each keep: verbatim sinks, ring and exact tier (``n`` per token),
    the basis (``n`` x ``rank``) and its diagonal core (``rank``) once a basis
    exists, and ``rank`` coordinates per column.  Bookkeeping: one position per
    column unless retention is FIFO (positions are implicit there), one
    graduation surprise per column under ``"lowrank_surprise"``, one position
    per exact-tier token, plus its selection score when the tier is
    attention-selected (a surprise-selected tier re-scores from the basis and
    stores none)."""
    if retention not in ("fifo", "lowrank_surprise"):
        raise NotImplementedError(f"retention {retention!r} is outside the surprise-selected path")
    if merge or quant_count or quant_bits is not None or w_key:
        raise NotImplementedError("merge, quantised tiers and key whitening are not in scope")
    if hh_select not in ("attn", "surprise"):
        raise ValueError(f"hh_select must be 'attn' or 'surprise', got {hh_select!r}")
    streams = 2  # K and V
    basis = rank if u_present else 0
    return _table([
        ("sinks", streams * n_sink, n, True),
        ("ring", streams * recent_len, n, True),
        ("exact tier", streams * hh_count, n, True),
        ("coordinates", streams * coord_count, rank, True),
        ("basis", streams * basis, n, True),
        ("core", streams * basis, 1, False),
        ("positions", coord_count if retention != "fifo" else 0, 1, False),
        ("surprise", coord_count if retention == "lowrank_surprise" else 0, 1, False),
        ("exact positions", hh_count, 1, False),
        ("exact scores", hh_count if hh_select == "attn" else 0, 1, False),
    ])


def bug_footprint_saturated(
    n: int,
    rank: int,
    coord_budget: int,
    recent_window: int,
    absorb_block: int,
    *,
    n_sink: int = 4,
    retention: str = "fifo",
    hh_budget: int = 0,
    hh_select: str = "attn",
) -> Footprint:
    """The layer at its high-water mark: a full coordinate budget and the ring
    one token short of the next absorb (``recent_window + absorb_block - 1``),
    src/kvdlra/accounting.py:167-191.  The reference's helper prices the exact
    tier as attention-selected (position + score per token); ``hh_select``
    defaults to that so the numbers agree, ``"surprise"`` prices the tier
    this cache keeps."""
    return bug_footprint(n, rank, coord_budget, recent_window + absorb_block - 1, n_sink=n_sink,
                         retention=retention, hh_count=hh_budget, hh_select=hh_select)


def bug_prefill_footprint(t: int, n: int, rank: int, *, n_sink: int = 4) -> Footprint:
    """The BUGPress prefill model (src/kvdlra/accounting.py:194-213): sinks
    verbatim, one basis per stream, and every other token as ``rank``
    coordinates per stream (no ring, no core)."""
    payload = max(0, t - n_sink)
    return _table([
        ("sinks", 2 * n_sink, n, True),
        ("basis", 2 * rank, n, True),
        ("coordinates", 2 * payload, rank, True),
    ])


def full_cache_footprint(t: int, n: int) -> Footprint:
    """The uncompressed K+V cache of ``t`` tokens."""
    return _table([("keys and values", 2 * t, n, True)])


def assert_all_within(mem_by_arm: dict[str, float], budget_per_layer: float, *,
                      tol: float = 0.0) -> None:
    """Matched-memory gate: raise ``ValueError`` naming every arm whose
    per-layer charge exceeds ``budget_per_layer`` (+ ``tol``)."""
    limit = budget_per_layer + tol
    over = sorted(a for a, m in mem_by_arm.items() if not m <= limit or math.isnan(m))
    if over:
        detail = ", ".join(f"{a}={mem_by_arm[a]:g}" for a in over)
        raise ValueError(f"matched-memory audit FAILED: {detail} over the budget of "
                         f"{budget_per_layer:g} float-equivalents per layer")
