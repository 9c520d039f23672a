"""GPU augmented BUG step (kvd_bug_step) against the oracle and the
reference's integrator properties (tests/test_bug_cache.py:83-123 and
tests/test_streaming_torch.py of the reference, restated)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.bug_oracle import augmented_bug_step as oracle_step, blocked_bug_subspace as oracle_blocked
from oracle.bug_oracle import principal_angle

from kvdlra_b200 import augmented_bug_step, blocked_bug_subspace
from kvdlra_b200.integrator import bug_step_batched

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
GOLDEN = Path(__file__).resolve().parent / "golden"


def test_step_sequence_matches_golden_and_oracle() -> None:
    g = np.load(GOLDEN / "steps.npz")
    data = g["data"]
    u = b = None
    uo = bo = None
    start = 0
    for i, bs in enumerate(g["blocks"].tolist()):
        blk = data[:, start : start + bs]
        u, b, rot = augmented_bug_step(u, b, torch.from_numpy(blk).to(DEV), 12)
        uo, bo, roto, _ = oracle_step(uo, bo, blk, 12)
        sig = torch.diagonal(b).cpu().numpy()
        # singular values: fp32-level agreement with the reference (golden)
        assert np.allclose(sig, g[f"sigma_{i}"], rtol=1e-4, atol=1e-6 * sig.max())
        assert principal_angle(u.cpu().numpy(), g[f"u_{i}"]) < 1e-3
        # orthonormal basis
        un = u.cpu().double().numpy()
        assert np.abs(un.T @ un - np.eye(un.shape[1])).max() < 1e-5
        # rot = u_new^T u_old (the carry map), checked on the GPU's own bases
        if i > 0:
            assert np.abs(rot.cpu().numpy() - u.cpu().numpy().T @ u_prev).max() < 1e-5
        u_prev = u.cpu().numpy()
        start += bs


def test_clamp_overfull_augmentation_and_full_rank_identity() -> None:
    rng = np.random.default_rng(2)
    n = 16
    m = rng.standard_normal((n, 64)).astype(np.float32)
    mt = torch.from_numpy(m).to(DEV)
    u, b, _ = augmented_bug_step(None, None, mt[:, :12], 12)
    u2, _, _ = augmented_bug_step(u, b, mt[:, 12:40], 16)  # 12 + 28 > 16
    assert u2.shape[1] <= n
    un = u2.cpu().double().numpy()
    assert np.abs(un.T @ un - np.eye(un.shape[1])).max() < 1e-5
    u3, b3, _ = augmented_bug_step(None, None, mt[:, :12], 16)
    u3, b3, _ = augmented_bug_step(u3, b3, mt[:, 12:40], 16)
    proj = (u3 @ (u3.mT @ mt)).cpu().numpy()
    assert np.abs(proj - m).max() < 1e-4


def test_rank_deficient_seed_gets_orthonormal_completion() -> None:
    """A rank-1 first block with rank cap 4: the basis still has 4 orthonormal
    columns (the reference's QR completes it the same way), one of them the
    data direction."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal(32).astype(np.float32)
    blk = np.stack([x] * 6, axis=1)
    u, b, _ = augmented_bug_step(None, None, torch.from_numpy(blk).to(DEV), 4)
    assert u.shape[1] == 4
    un = u.cpu().double().numpy()
    assert np.abs(un.T @ un - np.eye(4)).max() < 1e-5
    assert np.linalg.norm(un.T @ (x / np.linalg.norm(x))) > 1 - 1e-5


def test_blocked_sweep_matches_oracle_and_theta() -> None:
    rng = np.random.default_rng(5)
    basis = np.linalg.qr(rng.standard_normal((64, 10)))[0]
    data = (basis @ rng.standard_normal((10, 300)) + 1e-3 * rng.standard_normal((64, 300))).astype(np.float32)
    u = blocked_bug_subspace(torch.from_numpy(data).to(DEV), 8, 32).cpu().numpy()
    uo = oracle_blocked(data, 8, 32)
    assert principal_angle(u, uo) < 1e-3
    # theta truncation gives the oracle's rank
    nb = torch.zeros(1, 64, 16, device=DEV)
    sig = torch.zeros(1, 16, device=DEV)
    r = torch.zeros(1, dtype=torch.int32, device=DEV)
    blk = torch.from_numpy(data[:, :40].T.copy())[None].to(DEV)
    _, sig, r, _, _ = bug_step_batched(nb, sig, r, blk, 16, theta=0.5)
    _, bo, _, _ = oracle_step(None, None, data[:, :40], 16, theta=0.5)
    assert int(r[0]) == bo.shape[0]


def test_batched_problems_independent() -> None:
    rng = np.random.default_rng(6)
    nb, n, ld, bsz = 5, 48, 12, 16
    blocks = rng.standard_normal((nb, bsz, n)).astype(np.float32)
    u = torch.zeros(nb, n, ld, device=DEV)
    sig = torch.zeros(nb, ld, device=DEV)
    r = torch.zeros(nb, dtype=torch.int32, device=DEV)
    u, sig, r, _, _ = bug_step_batched(u, sig, r, torch.from_numpy(blocks).to(DEV), 10)
    blocks2 = rng.standard_normal((nb, bsz, n)).astype(np.float32)
    u, sig, r, _, _ = bug_step_batched(u, sig, r, torch.from_numpy(blocks2).to(DEV), 10)
    for i in range(nb):
        uo, bo, _, _ = oracle_step(None, None, blocks[i].T.copy(), 10)
        uo, bo, _, _ = oracle_step(uo, bo, blocks2[i].T.copy(), 10)
        assert int(r[i]) == uo.shape[1]
        assert principal_angle(u[i, :, : int(r[i])].cpu().numpy(), uo) < 1e-3
        assert np.allclose(sig[i, : int(r[i])].cpu().numpy(), np.diag(bo), rtol=1e-4)


@pytest.mark.parametrize("rank", [32, 48])
def test_long_stream_stays_orthonormal(rank: int) -> None:
    """300 BUG steps of 16 tokens: the basis stays orthonormal to fp32 level
    (each step ends with a Newton-Schulz correction, so rounding and the
    Jacobi stopping tolerance do not accumulate) and tracks the oracle's
    subspace.  rank 48 exercises the correction for more than 32 columns."""
    rng = np.random.default_rng(11)
    n, t = 256, 300 * 16
    basis = np.linalg.qr(rng.standard_normal((n, rank + 8)))[0]
    scale = np.concatenate([2.0 ** (-np.arange(rank) / 16), np.full(8, 1e-2)])  # clear gap at rank
    coef = rng.standard_normal((rank + 8, t)) * scale[:, None]
    data = (basis @ coef + 1e-3 * rng.standard_normal((n, t))).astype(np.float32)
    u = blocked_bug_subspace(torch.from_numpy(data).to(DEV), rank, 16).cpu().double().numpy()
    assert u.shape[1] == rank
    assert np.abs(u.T @ u - np.eye(rank)).max() < 1e-5
    uo = oracle_blocked(data[:, :1600], rank, 16)
    u_short = blocked_bug_subspace(torch.from_numpy(data[:, :1600]).to(DEV), rank, 16).cpu().numpy()
    assert principal_angle(u_short, uo) < 1e-3


@pytest.mark.parametrize("blocks,cap", [([1, 2, 1, 3, 2, 5, 1], 4), ([2, 2, 2, 2], 3), ([3, 1, 2, 7, 16, 2], 9)])
def test_tiny_and_odd_blocks_match_oracle(blocks: list[int], cap: int) -> None:
    """Blocks of 1, 2 and odd sizes drive the one-sided Jacobi with one pair,
    a dummy column and odd column counts (residual factor and core): every
    step's singular values and subspace match the oracle's."""
    rng = np.random.default_rng(sum(blocks) + cap)
    n = 40
    basis = np.linalg.qr(rng.standard_normal((n, 6)))[0]
    total = sum(blocks)
    data = (basis @ (rng.standard_normal((6, total)) * (2.0 ** -np.arange(6))[:, None])
            + 1e-2 * rng.standard_normal((n, total))).astype(np.float32)
    u = b = None
    uo = bo = None
    start = 0
    for bs in blocks:
        blk = data[:, start:start + bs]
        u, b, _ = augmented_bug_step(u, b, torch.from_numpy(blk).to(DEV), cap)
        uo, bo, _, _ = oracle_step(uo, bo, blk, cap)
        sig = torch.diagonal(b).cpu().numpy()
        assert sig.shape[0] == bo.shape[0]
        assert np.allclose(sig, np.diag(bo), rtol=1e-4, atol=1e-6 * np.diag(bo).max())
        assert principal_angle(u.cpu().numpy(), uo) < 1e-3
        un = u.cpu().double().numpy()
        assert np.abs(un.T @ un - np.eye(un.shape[1])).max() < 1e-5
        start += bs
