"""Factored decode against dense attention over the same cache state.

The factored kernel never materialises the middle tier: it rebuilds each
middle key from its coordinates (RoPE applied at the token's true position)
and accumulates values in coordinate space.  Its output must equal softmax
attention over the cache's own dense reconstruction (``_decode_peek``, the
reference's peek of bug_cache.py:1496-1575) -- this pins the tiled decode
path (head_dim 64 and 128) on every tier boundary, partial tiles, several
query-group sizes, fp32 and bf16.  Tolerances: 1e-4 relative (fp32), 2e-2
relative (bf16), the attention-output bounds of the parity rules.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.bug_oracle import default_inv_freq, gqa_attention

from kvdlra_b200 import BugStreamingLayer, RopeAngles
from kvdlra_b200.synthetic import lowrank_stream

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _rel(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.abs(a.astype(np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("H,D,G,T,rank", [
    (8, 128, 4, 1300, 128),  # tcgen05 middle tier, 128 rank columns, one group per CTA
    (4, 128, 8, 900, 64),    # 64 rank columns
    (4, 64, 4, 1100, 96),    # two groups of 64 per CTA, rank 96 in 128 columns
    (2, 64, 8, 700, 128),    # 16 query heads per CTA
    (8, 64, 2, 1000, 40),
    (8, 128, 4, 1300, 192),  # 192 rank columns: keys and values share one buffer
    (4, 64, 2, 900, 160),
])
def test_factored_decode_wide_rank_bf16(H: int, D: int, G: int, T: int, rank: int) -> None:
    """Ranks 33..192 in bf16 (the whole-box and decode-sweep ranks): the
    middle tier on the tensor cores with the basis staged in 64, 128 or 192
    rank columns, against dense attention over the peek within the bf16
    rule."""
    s = lowrank_stream(H, D, T, n_needles=5, seed=H * 7 + D + rank, signal_rank=min(D, max(16, rank // H + 8)))
    inv = default_inv_freq(D, 500000.0)
    layer = BugStreamingLayer(RopeAngles(inv_freq=torch.from_numpy(inv), attention_scaling=1.0),
                              rank=rank, coord_budget=T + 200, recent_window=96, absorb_block=16,
                              n_sink=4, retention="lowrank_surprise", hh_budget=70,
                              hh_select="surprise")
    layer._mode = "ingest"
    k = torch.from_numpy(s.k_post)[None].to(DEV, torch.bfloat16)
    v = torch.from_numpy(s.v)[None].to(DEV, torch.bfloat16)
    for st in range(0, T, 128):
        layer.update(k[:, :, st : st + 128], v[:, :, st : st + 128])
        layer.consolidate()
    kr, vr = layer._decode_peek()
    kd = kr[0].float().cpu().numpy()
    vd = vr[0].float().cpu().numpy()
    assert layer._ranks()[0] > 32  # the basis grew past 32 columns
    rng = np.random.default_rng(T + rank)
    for _ in range(3):
        q = torch.from_numpy(rng.standard_normal((H * G, D)).astype(np.float32)).to(DEV, torch.bfloat16)
        out = layer.factored_attention(q[None])[0].float().cpu().numpy()
        ref = gqa_attention(q.float().cpu().numpy(), kd, vd)
        assert _rel(out, ref) < 2e-2, _rel(out, ref)
    layer._group.check_status()


@pytest.mark.parametrize("H,D,G,T,dtype", [
    (2, 128, 8, 1000, torch.float32),
    (4, 64, 4, 777, torch.float32),
    (2, 64, 1, 450, torch.float32),
    (3, 128, 2, 600, torch.bfloat16),
    (8, 64, 4, 1300, torch.bfloat16),
    (8, 128, 4, 1300, torch.bfloat16),  # tcgen05 middle tier, two group ranges per tile
    (2, 128, 4, 700, torch.bfloat16),   # tcgen05 middle tier, n = 256
])
def test_factored_decode_equals_dense_over_peek(H: int, D: int, G: int, T: int, dtype) -> None:
    s = lowrank_stream(H, D, T, n_needles=5, seed=H * 100 + D + G)
    inv = default_inv_freq(D, 500000.0)
    layer = BugStreamingLayer(RopeAngles(inv_freq=torch.from_numpy(inv), attention_scaling=1.0),
                              rank=32, coord_budget=T + 200, recent_window=96, absorb_block=16,
                              n_sink=4, retention="lowrank_surprise", hh_budget=70,
                              hh_select="surprise")
    layer._mode = "ingest"
    k = torch.from_numpy(s.k_post)[None].to(DEV, dtype)
    v = torch.from_numpy(s.v)[None].to(DEV, dtype)
    for st in range(0, T, 128):  # tier lengths end mid-tile
        layer.update(k[:, :, st : st + 128], v[:, :, st : st + 128])
        layer.consolidate()
    kr, vr = layer._decode_peek()
    kd = kr[0].float().cpu().numpy()
    vd = vr[0].float().cpu().numpy()
    assert kd.shape[1] > 2 * 64  # several tiles, with a middle tier
    rng = np.random.default_rng(T)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    for _ in range(3):
        q = torch.from_numpy(rng.standard_normal((H * G, D)).astype(np.float32)).to(DEV, dtype)
        out = layer.factored_attention(q[None])[0].float().cpu().numpy()
        ref = gqa_attention(q.float().cpu().numpy(), kd, vd)
        assert _rel(out, ref) < tol, _rel(out, ref)
    layer._group.check_status()
