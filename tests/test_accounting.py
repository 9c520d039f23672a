"""Float-equivalent accounting: the formula against the oracle's measured
``stored_state_numel`` across retention / tier configs (the reference pins
this in tests/test_accounting.py:74-128), and the ratio pins."""

from __future__ import annotations

import numpy as np
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
                             hh_count=lay.hh_len(), hh_select="surprise" if hh else "attn",
                             u_present=lay.u_k is not None)
        assert fp.float_equiv() == lay.stored_state_numel()


def test_balanced_config_ratio_pin() -> None:
    # bugS-r128-h1024 at 32K, Llama-3.1-8B geometry (n = 1024)
    fp = A.bug_footprint_saturated(1024, 128, 32768, 32, 16, retention="lowrank_surprise", hh_budget=1024)
    ratio = fp.ratio_fp16(32768, 1024)
    assert 0.15 < ratio < 0.35
    assert fp.float_equiv() == (2 * 1024 * 4 + 2 * 1024 * 47 + 2 * 128 * 32768 + 2 * 1024 * 1024
                                + 2 * 1024 * 128 + 2 * 128 + 32768 * 2 + 2 * 1024)


def test_full_cache_ratio_is_one_and_gate() -> None:
    assert A.full_cache_footprint(100, 64).ratio_fp16(100, 64) == 1.0
    A.assert_all_within({"a": 1.0, "b": 2.0}, 2.0)
    with pytest.raises(ValueError, match="matched-memory audit FAILED"):
        A.assert_all_within({"a": 3.0}, 2.0)
    rep = A.report("x", A.full_cache_footprint(10, 8), 10, 8)
    assert rep.ratio_fp16 == 1.0 and rep.bytes_native == 2 * 10 * 8 * 2
