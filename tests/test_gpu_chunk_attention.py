"""Factored chunk attention against dense attention over the same cache state.

``kvd_factored_chunk_attention`` answers every query of an ingest chunk (the
chunk already appended to the ring, bug_cache.py:1404-1423) or of a frozen
scoring window (the window as a tail, 1390-1402) without materialising the
middle tier: middle keys are rebuilt per tile on the tensor cores with RoPE
at each token's true position, values accumulate in coordinate space.  Its
output must equal softmax attention over the cache's own dense return value
(``_decode_peek``, with the window as tail when scoring) under the
bottom-right causal mask transformers builds from ``get_mask_sizes``.  The
cases put tier and tile boundaries mid-tile, use query counts that are not a
multiple of the 128-row tile and several query-group sizes.  Tolerance: the
bf16 attention rule, 2e-2 relative to the largest output.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.bug_oracle import default_inv_freq

from kvdlra_b200 import BugStreamingLayer, RopeAngles
from kvdlra_b200.synthetic import lowrank_stream

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _dense_causal(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> np.ndarray:
    """fp64 softmax attention of q (Hq, Q, D) over k, v (H, L, D), query i
    seeing keys up to L - Q + i; returns (Q, Hq, D)."""
    hq, nq, _ = q.shape
    h, L, _ = k.shape
    g = hq // h
    qd, kd, vd = q.double(), k.double(), v.double()
    kd = kd.repeat_interleave(g, dim=0)
    vd = vd.repeat_interleave(g, dim=0)
    s = torch.einsum("hqd,hkd->hqk", qd, kd) * scale
    lim = (L - nq + torch.arange(nq))[:, None]
    mask = torch.arange(L)[None, :] > lim
    s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,hkd->qhd", p, vd).numpy()


def _layer(H: int, D: int, T: int, rank: int, hh: int, retention: str):
    inv = default_inv_freq(D, 500000.0)
    kw = dict(hh_budget=hh, hh_select="surprise") if hh else {}
    layer = BugStreamingLayer(RopeAngles(inv_freq=torch.from_numpy(inv), attention_scaling=1.0),
                              rank=rank, coord_budget=T + 400, recent_window=96, absorb_block=16,
                              n_sink=4, retention=retention, **kw)
    layer._mode = "ingest"
    return layer


@pytest.mark.parametrize("H,G,T,q_len,rank,hh,retention", [
    (8, 4, 1300, 200, 32, 70, "lowrank_surprise"),
    (2, 4, 900, 128, 16, 32, "lowrank_surprise"),
    (4, 1, 700, 77, 32, 0, "fifo"),
    (8, 2, 1100, 300, 24, 256, "lowrank_surprise"),
])
@pytest.mark.parametrize("mode", ["ingest", "score"])
def test_chunk_attention_equals_dense_causal(H: int, G: int, T: int, q_len: int, rank: int, hh: int,
                                             retention: str, mode: str) -> None:
    D = 64
    s = lowrank_stream(H, D, T + q_len, n_needles=5, seed=H * 1000 + T + rank)
    layer = _layer(H, D, T, rank, hh, retention)
    k = torch.from_numpy(s.k_post)[None].to(DEV, torch.bfloat16)
    v = torch.from_numpy(s.v)[None].to(DEV, torch.bfloat16)
    for st in range(0, T, 128):  # tier lengths end mid-tile
        layer.update(k[:, :, st : min(T, st + 128)], v[:, :, st : min(T, st + 128)])
        layer.consolidate()
    kc, vc = k[:, :, T : T + q_len], v[:, :, T : T + q_len]
    rng = np.random.default_rng(T + q_len)
    q = torch.from_numpy(rng.standard_normal((1, H * G, q_len, D)).astype(np.float32)).to(DEV, torch.bfloat16)
    scale = D ** -0.5
    if mode == "ingest":
        layer._append(kc, vc)
        kr, vr = layer._decode_peek()
        out = layer.factored_chunk_attention(q, scaling=scale)
    else:
        layer._mode = "score"
        kr, vr = layer._decode_peek(tail=(kc, vc))
        out = layer.factored_chunk_attention(q, scaling=scale, tail=(kc, vc))
    assert kr.shape[2] > 4 + hh + 256  # a middle tier of several tiles
    ref = _dense_causal(q[0].float().cpu(), kr[0].float().cpu(), vr[0].float().cpu(), scale)
    got = out[0].float().cpu().numpy()
    err = float(np.abs(got - ref).max() / np.abs(ref).max())
    assert err < 2e-2, err
    layer._group.check_status()


def test_chunk_attention_two_sequences() -> None:
    """Two sequences of one layer (different streams, so different ranks,
    tiers and coordinates) answered by one call: each equals its own dense
    causal attention."""
    H, G, T, q_len, D = 4, 4, 900, 150, 64
    streams = [lowrank_stream(H, D, T + q_len, n_needles=4, seed=77 + i) for i in range(2)]
    layer = _layer(H, D, T, 32, 64, "lowrank_surprise")
    k = torch.stack([torch.from_numpy(st.k_post) for st in streams]).to(DEV, torch.bfloat16)
    v = torch.stack([torch.from_numpy(st.v) for st in streams]).to(DEV, torch.bfloat16)
    for st in range(0, T, 128):
        layer.update(k[:, :, st : min(T, st + 128)], v[:, :, st : min(T, st + 128)])
        layer.consolidate()
    layer._append(k[:, :, T:], v[:, :, T:])
    rng = np.random.default_rng(5)
    q = torch.from_numpy(rng.standard_normal((2, H * G, q_len, D)).astype(np.float32)).to(DEV, torch.bfloat16)
    kr, vr = layer._decode_peek()
    out = layer.factored_chunk_attention(q, scaling=D ** -0.5)
    for b in range(2):
        ref = _dense_causal(q[b].float().cpu(), kr[b].float().cpu(), vr[b].float().cpu(), D ** -0.5)
        got = out[b].float().cpu().numpy()
        err = float(np.abs(got - ref).max() / np.abs(ref).max())
        assert err < 2e-2, (b, err)
    layer._group.check_status()


def test_chunk_attention_refuses_unsupported_shape() -> None:
    """fp32 caches (or head_dim != 64, rank > 32) have no chunk kernel: the
    call fails loudly instead of computing something else."""
    H, D, T = 2, 64, 400
    s = lowrank_stream(H, D, T, n_needles=0, seed=3)
    inv = default_inv_freq(D, 500000.0)
    layer = BugStreamingLayer(RopeAngles(inv_freq=torch.from_numpy(inv), attention_scaling=1.0),
                              rank=16, coord_budget=T + 200, recent_window=96, absorb_block=16,
                              n_sink=4, retention="fifo")
    layer._mode = "ingest"
    k = torch.from_numpy(s.k_post)[None].to(DEV)
    v = torch.from_numpy(s.v)[None].to(DEV)
    layer.update(k, v)
    layer.consolidate()
    q = torch.zeros(1, 2 * H, 8, D, device=DEV)
    with pytest.raises(Exception, match="unsupported shape"):
        layer.factored_chunk_attention(q)
