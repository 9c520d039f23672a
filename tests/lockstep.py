"""Lock-step comparison of the CUDA cache against the CPU oracle.

Both sides receive the same chunks; the absorb loop is stepped one block at a
time on both.  After every exact-tier selection the kept positions must be
identical, except where the oracle's scores of the swapped candidates are
within ``tol`` relative of each other (a near-tie: fp32 rounding decides it);
on such an event the GPU state is re-synchronised from the oracle and the
event is counted.  Any other mismatch fails immediately.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from oracle.bug_oracle import OracleLayer, principal_angle


@dataclass
class Stats:
    events: int = 0
    near_ties: int = 0
    max_angle_k: float = 0.0
    max_angle_v: float = 0.0
    notes: list = field(default_factory=list)


def to_mat(x_htd: np.ndarray) -> np.ndarray:
    h, t, d = x_htd.shape
    return np.ascontiguousarray(x_htd.transpose(0, 2, 1).reshape(h * d, t))


def oracle_state(o: OracleLayer) -> dict:
    st = {
        "hh_k": o.hh_k if o.hh_k is not None else np.zeros((o.n, 0), np.float32),
        "hh_v": o.hh_v if o.hh_v is not None else np.zeros((o.n, 0), np.float32),
        "hh_pos": o.hh_pos if o.hh_pos is not None else np.zeros(0, np.int64),
        "u_k": o.u_k, "u_v": o.u_v,
        "sigma_k": None if o.b_k is None else np.diag(o.b_k).copy(),
        "sigma_v": None if o.b_v is None else np.diag(o.b_v).copy(),
        "c_k": o.c_k if o.c_k is not None else np.zeros((0 if o.u_k is None else o.u_k.shape[1], 0), np.float32),
        "c_v": o.c_v if o.c_v is not None else np.zeros((0 if o.u_v is None else o.u_v.shape[1], 0), np.float32),
        "mid_pos": o.mid_pos if o.track_positions else None,
        "mid_surprise": o.mid_surprise if o.track_surprise else None,
    }
    if st["mid_pos"] is None:
        st["mid_pos"] = np.zeros(o.f_len(), np.int64)
        st["_no_pos"] = True
    return st


def _gpu_hh(layer) -> np.ndarray:
    x = layer.hh_pos
    return np.zeros(0, np.int64) if x is None else x.cpu().numpy()


def check_event(layer, oracle: OracleLayer, stats: Stats, tol: float) -> None:
    stats.events += 1
    g = _gpu_hh(layer)
    o = oracle.hh_pos if oracle.hh_pos is not None else np.zeros(0, np.int64)
    if not np.array_equal(g, o):
        ev = oracle.trace[-1] if oracle.trace else None
        assert ev is not None, "exact tiers differ outside a selection event"
        score = {int(p): float(s) for p, s in zip(ev["cand_pos"], ev["sel"])}
        only_g = sorted(set(g.tolist()) - set(o.tolist()))
        only_o = sorted(set(o.tolist()) - set(g.tolist()))
        assert len(only_g) == len(only_o), (only_g, only_o)
        worst = 0.0
        for a in only_g:
            for b in only_o:
                sa, sb = score[a], score[b]
                worst = max(worst, abs(sa - sb) / max(abs(sa), abs(sb), 1e-30))
        assert worst <= tol, (
            f"exact tier differs beyond a near-tie at event {stats.events}: gpu-only {only_g} "
            f"oracle-only {only_o}, relative score gap {worst:.3e} > {tol}"
        )
        stats.near_ties += 1
        stats.notes.append((stats.events, only_g, only_o, worst))
        st = oracle_state(oracle)
        if st.pop("_no_pos", False):
            st["mid_pos"] = None
        layer.load_state(st)
    else:
        mp_g = layer.mid_pos
        if oracle.mid_pos is not None and mp_g is not None:
            assert np.array_equal(mp_g.cpu().numpy(), oracle.mid_pos)
    if oracle.u_k is not None and layer.u_k is not None:
        stats.max_angle_k = max(stats.max_angle_k, principal_angle(layer.u_k.cpu().numpy(), oracle.u_k))
        stats.max_angle_v = max(stats.max_angle_v, principal_angle(layer.u_v.cpu().numpy(), oracle.u_v))


def run_ingest(layer, oracle: OracleLayer, k_htd: np.ndarray, v_htd: np.ndarray, chunk: int,
               *, dtype: torch.dtype, tol: float = 1e-5, check_angles_every: int = 1) -> Stats:
    """Chunked ingest through both; returns the comparison statistics."""
    stats = Stats()
    t = k_htd.shape[1]
    dev = torch.device("cuda")
    layer._mode = "ingest"
    oracle.mode = "ingest"
    rw, b = oracle.recent_window, oracle.absorb_block
    for start in range(0, t, chunk):
        stop = min(t, start + chunk)
        kt = torch.from_numpy(np.ascontiguousarray(k_htd[:, start:stop]))[None].to(dev, dtype)
        vt = torch.from_numpy(np.ascontiguousarray(v_htd[:, start:stop]))[None].to(dev, dtype)
        if oracle.cumulative_length:
            assert layer.get_mask_sizes(stop - start) == oracle.get_mask_sizes(stop - start)
        n_before = len(oracle.trace)
        oracle.update(to_mat(k_htd[:, start:stop]), to_mat(v_htd[:, start:stop]))
        layer.update(kt, vt)
        if len(oracle.trace) > n_before or start == 0:
            check_event(layer, oracle, stats, tol)
        while oracle.recent_len() >= rw + b:
            oracle.absorb_block_into_stream(b)
            layer._absorb_block_into_stream()
            check_event(layer, oracle, stats, tol)
        assert layer.attended_length() == oracle.attended_length()
        assert layer._f_len() == oracle.f_len() and layer._hh_len() == oracle.hh_len()
    layer._mode = "normal"
    oracle.mode = "normal"
    return stats
