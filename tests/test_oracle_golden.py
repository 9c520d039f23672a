"""The CPU oracle against golden fixtures produced by the reference itself
(tests/golden/make_golden.py runs kvdlra's BugStreamingLayer on the same
seeded inputs).  Pins the oracle before it is trusted as the GPU checker."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from golden.make_golden import CASES
from oracle.bug_oracle import (OracleLayer, RopeSpec, augmented_bug_step, default_inv_freq,
                               gqa_attention, principal_angle)

from kvdlra_b200.synthetic import lowrank_stream

GOLDEN = Path(__file__).resolve().parent / "golden"


def _to_mat(x: np.ndarray) -> np.ndarray:
    h, t, d = x.shape
    return x.transpose(0, 2, 1).reshape(h * d, t)


def test_integrator_steps_match_reference() -> None:
    g = np.load(GOLDEN / "steps.npz")
    data = g["data"]
    u = b = None
    start = 0
    for i, bs in enumerate(g["blocks"].tolist()):
        u, b, rot, _ = augmented_bug_step(u, b, data[:, start : start + bs], 12)
        assert np.allclose(np.diag(b), g[f"sigma_{i}"], rtol=1e-4, atol=1e-5)
        assert principal_angle(u, g[f"u_{i}"]) < 1e-4
        assert rot.shape == g[f"rot_{i}"].shape
        start += bs


@pytest.mark.parametrize("case", list(CASES))
def test_oracle_layer_matches_reference(case: str) -> None:
    kw = CASES[case]
    g = np.load(GOLDEN / f"{case}.npz")
    H, D, t, chunk = kw["heads"], kw["head_dim"], kw["t"], kw["chunk"]
    dec = kw.get("decode_tokens", 0)
    s = lowrank_stream(H, D, t + dec, theta=kw["theta"], seed=kw["seed"], **kw["stream_kw"])
    import hashlib

    h = hashlib.sha256()
    h.update(np.ascontiguousarray(s.k_post).tobytes())
    h.update(np.ascontiguousarray(s.v).tobytes())
    assert h.digest() == g["input_sha"].tobytes(), "synthetic inputs drifted from the fixtures"
    lay = OracleLayer(RopeSpec(default_inv_freq(D, kw["theta"])), H, D, dtype=kw.get("dtype", "float32"),
                      **kw["layer_kw"])
    lay.mode = "ingest"
    ntr = len(g["tr_keep_off"]) - 1
    ref_keep = [g["tr_keep_pos"][g["tr_keep_off"][i] : g["tr_keep_off"][i + 1]] for i in range(ntr)]
    ref_sel = [g["tr_sel"][g["tr_cand_off"][i] : g["tr_cand_off"][i + 1]] for i in range(ntr)]
    near_ties: list[tuple[int, float]] = []

    def arbiter(cand_pos: np.ndarray, sel: np.ndarray, keep_pos: np.ndarray) -> np.ndarray:
        # Every selection must equal the reference's.  Where it does not, the
        # swap must be a near-tie: the swapped candidates' reference scores lie
        # within max(1e-5, twice the two implementations' own disagreement on
        # those scores) of each other -- fp32 rounding decided the order (scores
        # of in-span keys are formed by cancellation, |k|^2 - |U^T k|^2, so two
        # fp32 implementations drift apart by more than 1e-5 over a long stream).
        # The oracle then continues from the reference's choice.
        i = len(lay.trace)
        if i >= ntr or np.array_equal(keep_pos, ref_keep[i]):
            return keep_pos
        ref = {int(p): float(x) for p, x in zip(cand_pos, ref_sel[i])}
        own = {int(p): float(x) for p, x in zip(cand_pos, sel)}
        mine = set(keep_pos.tolist()) - set(ref_keep[i].tolist())
        theirs = set(ref_keep[i].tolist()) - set(keep_pos.tolist())
        for a in mine:
            for b in theirs:
                scale = max(abs(ref[a]), abs(ref[b]), 1e-30)
                gap = abs(ref[a] - ref[b]) / scale
                drift = max(abs(own[a] - ref[a]), abs(own[b] - ref[b])) / scale
                assert gap <= max(1e-5, 2.0 * drift), (
                    f"selection {i} differs beyond a near-tie: gap {gap:.3e}, score drift {drift:.3e}")
        near_ties.append((i, len(mine)))
        return ref_keep[i]

    lay.arbiter = arbiter
    masks = []
    for st in range(0, t, chunk):
        sp = min(t, st + chunk)
        if lay.cumulative_length:
            masks.append(lay.get_mask_sizes(sp - st))
        lay.update(_to_mat(s.k_post[:, st:sp]), _to_mat(s.v[:, st:sp]))
        lay.consolidate()
    lay.mode = "normal"
    assert np.array_equal(np.array(masks, np.int64).reshape(-1, 2), g["mask_sizes"])
    assert len(lay.trace) >= ntr
    assert len(near_ties) <= max(1, ntr // 20), near_ties  # near-ties are rare events
    for i in range(ntr):  # the scores of every selection agree with the reference's
        assert np.array_equal(lay.trace[i]["cand_pos"], g["tr_cand_pos"][g["tr_cand_off"][i] : g["tr_cand_off"][i + 1]])
        assert np.allclose(lay.trace[i]["sel"], ref_sel[i], rtol=1e-3, atol=1e-4)
    assert lay.stored_state_numel() == int(g["final_stored_numel"])
    assert lay.attended_length() == int(g["final_attended"])
    if "final_hh_pos" in g:
        assert np.array_equal(lay.hh_pos, g["final_hh_pos"])
    if "final_mid_pos" in g:
        assert np.array_equal(lay.mid_pos, g["final_mid_pos"])
    if "final_sigma_k" in g:
        assert np.allclose(np.diag(lay.b_k), g["final_sigma_k"], rtol=1e-4, atol=1e-4 * g["final_sigma_k"].max())
        assert principal_angle(lay.u_k, g["final_u_k"]) < 1e-2
        assert principal_angle(lay.u_v, g["final_u_v"]) < 1e-2
    if "final_mid_surprise" in g:
        assert np.allclose(lay.mid_surprise, g["final_mid_surprise"], atol=1e-4)
    kr, vr = lay.decode_peek()
    assert kr.shape[1] == int(g["peek_len"])
    assert abs(kr.astype(np.float64).sum() - float(g["peek_k_sum"])) <= 1e-3 * max(1.0, abs(float(g["peek_k_sum"])))
    if "gist_err_k" in g:
        pos = lay.mid_pos
        kp = np.concatenate([s.k_pre[hh][pos].T for hh in range(H)], axis=0)
        err = np.linalg.norm(kp - lay.u_k.astype(np.float64) @ lay.c_k) / np.linalg.norm(kp)
        assert abs(err - float(g["gist_err_k"])) <= 1e-3 * float(g["gist_err_k"]) + 1e-7
    if "attn_out" in g:
        # fp32: 1e-4 relative.  bf16: the reconstructed middle is rounded to bf16
        # after an fp32 product whose last bits differ between implementations, so
        # an element can land one bf16 ulp (2^-8 relative) away; 2e-3 relative on
        # the output bounds that (the bf16 attention rule itself is 2e-2).
        tol = 1e-4 if kw.get("dtype", "float32") == "float32" else 2e-3
        for qi in range(g["queries"].shape[0]):
            o = gqa_attention(g["queries"][qi], lay.to_hf(kr), lay.to_hf(vr))
            ref = g["attn_out"][qi]
            assert np.abs(o - ref).max() <= tol * np.abs(ref).max()
    if dec:
        dm, dn = [], []
        for j in range(dec):
            p = t + j
            dm.append(lay.get_mask_sizes(1))
            lay.update(_to_mat(s.k_post[:, p : p + 1]), _to_mat(s.v[:, p : p + 1]))
            dn.append(lay.stored_state_numel())
        assert np.array_equal(np.array(dm), g["dec_masks"])
        assert np.array_equal(np.array(dn), g["dec_numel"])
        if "dec_hh_pos" in g:
            assert np.array_equal(lay.hh_pos, g["dec_hh_pos"])


def test_stable_descending_order_ties_to_lower_index() -> None:
    sel = np.array([0.5, 1.0, 0.5, 1.0, 0.2], np.float32)
    assert OracleLayer.stable_desc_order(sel).tolist() == [1, 3, 0, 2, 4]


def test_span_boost_windowed_max() -> None:
    sel = np.array([0.1, 0.9, 0.2, 0.0, 0.8, 0.05], np.float32)
    pos = np.array([10, 11, 12, 50, 51, 52])
    out = OracleLayer.span_boost(sel, pos, 1)
    assert np.allclose(out, [0.9, 0.9, 0.9, 0.8, 0.8, 0.8])
    assert np.allclose(OracleLayer.span_boost(np.array([1.0, 0.0], np.float32), np.array([0, 100]), 1), [1.0, 0.0])
