"""The stand-alone selection primitives of the C ABI, called through it.

``kvd_surprise`` (bug_cache.py:906-921) against the surprise formula in
float64, and ``kvd_select_topk`` (bug_cache.py:810-812) against the stable
descending order the reference takes with ``torch.argsort(..., stable=True,
descending=True)`` -- ties to the lower index, NaN above every number, -0
tied with +0 -- including inputs made of ties.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.bug_oracle import OracleLayer, surprise_against

from kvdlra_b200 import _native as N

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("n,m,ld,ranks", [(512, 272, 32, (32, 0, 17)), (1024, 1040, 128, (128, 96)),
                                          (64, 5, 48, (48,))])
def test_surprise_through_the_abi(n: int, m: int, ld: int, ranks: tuple) -> None:
    rng = np.random.default_rng(n + m)
    nb = len(ranks)
    u = np.zeros((nb, n, ld), np.float32)
    x = np.empty((nb, m, n), np.float32)
    for b, r in enumerate(ranks):
        q = np.linalg.qr(rng.standard_normal((n, max(r, 1))))[0][:, :r].astype(np.float32)
        u[b, :, :r] = q
        u[b, :, r:] = rng.standard_normal((n, ld - r))  # columns past the rank are ignored
        # half the columns in span (plus 1e-2 noise: scores formed by cancellation), half generic
        inspan = (q @ rng.standard_normal((r, m // 2)) if r else np.zeros((n, m // 2))) \
            + 1e-2 * rng.standard_normal((n, m // 2))
        x[b] = np.concatenate([inspan, rng.standard_normal((n, m - m // 2))], axis=1).T
    ud = torch.from_numpy(u).to(DEV)
    xd = torch.from_numpy(x).to(DEV)
    rd = torch.tensor(ranks, dtype=torch.int32, device=DEV)
    out = torch.full((nb, m), -1.0, device=DEV)
    N.check(N.lib().kvd_surprise(nb, n, m, ld, ud.data_ptr(), rd.data_ptr(), xd.data_ptr(),
                                 out.data_ptr(), _stream()), "kvd_surprise")
    got = out.cpu().numpy()
    for b, r in enumerate(ranks):
        want = surprise_against(u[b, :, :r] if r else None, x[b].T)
        # fp32 sums: the in-span scores (~1e-2) lose ~eps |k|^2 / score to cancellation
        assert np.abs(got[b] - want).max() < 2e-5, (b, r, np.abs(got[b] - want).max())
        if r == 0:
            assert np.all(got[b] == 1.0)


def _order(sel: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    o = OracleLayer.stable_desc_order(sel)
    return np.sort(o[:k]), np.sort(o[k:])


@pytest.mark.parametrize("m,k", [(272, 256), (1040, 1024), (300, 100), (17, 0), (9, 9)])
def test_select_topk_ties_and_specials(m: int, k: int) -> None:
    rng = np.random.default_rng(m * 7 + k)
    rows = [
        np.round(rng.random(m), 1).astype(np.float32),  # mostly ties
        np.full(m, 0.25, np.float32),  # all tied: the lowest indices are kept
        rng.random(m).astype(np.float32),
    ]
    special = rng.random(m).astype(np.float32)
    special[rng.choice(m, size=max(1, m // 8), replace=False)] = np.nan
    special[rng.choice(m, size=max(1, m // 8), replace=False)] = -0.0
    special[rng.choice(m, size=max(1, m // 8), replace=False)] = 0.0
    special[rng.choice(m, size=max(1, m // 16), replace=False)] = np.inf
    rows.append(special)
    sc = np.stack(rows)
    nb = sc.shape[0]
    sd = torch.from_numpy(sc).to(DEV)
    keep = torch.full((nb, max(k, 1)), -7, dtype=torch.int32, device=DEV)
    dem = torch.full((nb, max(m - k, 1)), -7, dtype=torch.int32, device=DEV)
    N.check(N.lib().kvd_select_topk(nb, m, k, sd.data_ptr(), keep.data_ptr(), dem.data_ptr(),
                                    _stream()), "kvd_select_topk")
    kg, dg = keep.cpu().numpy(), dem.cpu().numpy()
    for b in range(nb):
        wk, wd = _order(sc[b], k)
        assert np.array_equal(kg[b, :k], wk), b
        assert np.array_equal(dg[b, : m - k], wd), b
        # torch's own stable descending argsort agrees (the reference's call)
        o = torch.argsort(torch.from_numpy(sc[b]), stable=True, descending=True).numpy()
        assert np.array_equal(np.sort(o[:k]), wk)
    # nothing written past the k kept / m - k demoted entries
    if k == 0:
        assert np.all(kg == -7)
    if k == m:
        assert np.all(dg == -7)


def test_select_topk_rejects_bad_sizes() -> None:
    dummy = torch.zeros(4, device=DEV)
    with pytest.raises(N.KvdError):
        N.check(N.lib().kvd_select_topk(1, 4, 5, dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
                                        _stream()), "kvd_select_topk")
