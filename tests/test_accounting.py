"""Float-equivalent accounting: the formula against the oracle's measured
``stored_state_numel`` across retention / tier configs (the reference pins
this in tests/test_accounting.py:74-128), and the reference's ratio pins
(tests/test_accounting.py:131-187, 250-262)."""

from __future__ import annotations

import pytest

from oracle.bug_oracle import OracleLayer, RopeSpec, default_inv_freq

from kvdlra_b200 import accounting as A
from kvdlra_b200.synthetic import lowrank_stream


@pytest.mark.parametrize("retention,hh", [("fifo", 0), ("lowrank_surprise", 0),
                                           ("lowrank_surprise", 8), ("fifo", 6)])
def test_formula_matches_measured(retention: str, hh: int) -> None:
    H, D, t = 2, 16, 200
    s = lowrank_stream(H, D, t, signal_rank=6, n_needles=2, seed=3, theta=10000.0)
    lay = OracleLayer(RopeSpec(default_inv_freq(D, 10000.0)), H, D, rank=8, coord_budget=64,
                      recent_window=8, absorb_block=4, retention=retention, hh_budget=hh,
                      hh_select="surprise" if hh else "attn")
    lay.mode = "ingest"
    for st in range(0, t, 32):
        k = s.k_post[:, st : st + 32].transpose(0, 2, 1).reshape(H * D, -1)
        v = s.v[:, st : st + 32].transpose(0, 2, 1).reshape(H * D, -1)
        lay.update(k, v)
        lay.consolidate()
        fp = A.bug_footprint(H * D, lay.u_k.shape[1] if lay.u_k is not None else 0, lay.f_len(),
                             lay.recent_len(), n_sink=lay.sink_len(), retention=retention,
                             hh_count=lay.hh_len(), hh_select="surprise",
                             u_present=lay.u_k is not None)
        assert fp.float_equiv() == lay.stored_state_numel()
        assert sum(fp.breakdown().values()) == fp.float_equiv()


def _arm(rank: int) -> A.Footprint:
    # the reference's arm-style counts at 32K on the 8B geometry (n = 1024):
    # the coordinate tier is everything not held verbatim
    n, t, hh, rw, sink = 1024, 32768, 1024, 32, 4
    return A.bug_footprint(n, rank, t - hh - rw - sink, rw, n_sink=sink,
                           retention="lowrank_surprise", hh_count=hh, hh_select="surprise")


def test_ratio_pins() -> None:
    # bugS-r128-h1024 "~0.15x" and bugS-r192-h1024 "~0.22x" (tests/test_accounting.py:131-171)
    assert 0.12 < _arm(128).ratio_fp16(32768, 1024) < 0.20
    assert 0.19 < _arm(192).ratio_fp16(32768, 1024) < 0.25


def test_saturated_closed_form() -> None:
    fp = A.bug_footprint_saturated(1024, 128, 32768, 32, 16, retention="lowrank_surprise", hh_budget=1024)
    assert fp.float_equiv() == (2 * 1024 * 4 + 2 * 1024 * 47 + 2 * 128 * 32768 + 2 * 1024 * 1024
                                + 2 * 1024 * 128 + 2 * 128 + 32768 * 2 + 2 * 1024)
    sur = A.bug_footprint_saturated(1024, 128, 32768, 32, 16, retention="lowrank_surprise",
                                    hh_budget=1024, hh_select="surprise")
    assert fp.float_equiv() - sur.float_equiv() == 1024  # no stored selection score
    # the fifo high-water charge (the reference's w5_streamppl.bug_budget_floats):
    # sinks + ring (rw + ab - 1) + basis + cores + coordinates, K and V
    for rank in (8, 16, 32):
        for w in (24, 100):
            fp = A.bug_footprint_saturated(32, rank, w, 8, 4)
            assert fp.float_equiv() == 2 * 32 * 4 + 2 * 32 * 11 + 2 * 32 * rank + 2 * rank + 2 * rank * w


def test_prefill_and_full_cache() -> None:
    assert A.full_cache_footprint(4096, 512).ratio_fp16(4096, 512) == 1.0
    assert A.full_cache_footprint(4096, 512).tok_equiv(512) == 4096.0
    fp = A.bug_prefill_footprint(1024, 512, 32)
    assert fp.float_equiv() == 2 * 512 * 4 + 2 * 512 * 32 + 2 * 32 * 1020


def test_out_of_scope_tiers_refused() -> None:
    with pytest.raises(NotImplementedError):
        A.bug_footprint(32, 8, 10, 4, retention="attn")
    with pytest.raises(NotImplementedError):
        A.bug_footprint(32, 8, 10, 4, quant_count=3, quant_bits=4)
    with pytest.raises(ValueError):
        A.bug_footprint(32, 8, 10, 4, hh_count=2, hh_select="energy")


def test_assert_all_within_gate() -> None:
    A.assert_all_within({"a": 100.0, "b": 200.0}, budget_per_layer=200.0)
    with pytest.raises(ValueError, match="matched-memory audit FAILED"):
        A.assert_all_within({"a": 100.0, "b": 201.0}, budget_per_layer=200.0)
