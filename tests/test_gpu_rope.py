"""RoPE angle tables on the GPU against fp64 cos/sin of the same fp32 angle.

The cache forms every rotary angle as the model's rotary module does: one
fp32 product pos * inv_freq, then cos/sin scaled by attention_scaling.  The
full-precision path (sincosf) must sit within 1e-6 of the exact cos/sin of
that fp32 angle; the factored decode's reduced path (Cody-Waite reduction by
2*pi in three fp32 parts, hardware sin/cos on the reduced angle) within 2e-6,
for positions up to 2^17 and the frequencies of head_dim 64 and 128 (theta
500000 and 10000) plus inv_freq = 1, the fastest-turning case.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from oracle.bug_oracle import default_inv_freq

from kvdlra_b200 import _native as N

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _table(pos: np.ndarray, inv: np.ndarray, scale: float, fast: int) -> tuple[np.ndarray, np.ndarray]:
    p = torch.from_numpy(pos.astype(np.int32)).to(DEV)
    f = torch.from_numpy(inv.astype(np.float32)).to(DEV)
    co = torch.empty(len(pos), len(inv), device=DEV)
    so = torch.empty_like(co)
    N.check(N.lib().kvd_rope_table(len(pos), p.data_ptr(), len(inv), f.data_ptr(), C.c_float(scale),
                                   fast, co.data_ptr(), so.data_ptr(), N.stream_ptr(DEV)),
            "kvd_rope_table")
    return co.cpu().numpy(), so.cpu().numpy()


@pytest.mark.parametrize("head_dim,theta", [(64, 500000.0), (128, 10000.0), (2, 1.0)])
@pytest.mark.parametrize("scale", [1.0, 1.25])
def test_rope_angles_full_and_fast(head_dim: int, theta: float, scale: float) -> None:
    rng = np.random.default_rng(head_dim)
    pos = np.concatenate([np.arange(0, 64), [8191, 8192, 65535, 131071],
                          rng.integers(0, 1 << 17, 2000)]).astype(np.int64)
    inv = default_inv_freq(head_dim, theta).astype(np.float32)
    if head_dim == 2:
        inv = np.array([1.0], dtype=np.float32)
    ang = (pos.astype(np.float32)[:, None] * inv[None, :]).astype(np.float64)  # the fp32 product
    c_ref = np.cos(ang) * np.float64(np.float32(scale))
    s_ref = np.sin(ang) * np.float64(np.float32(scale))
    for fast, tol in ((0, 1e-6), (1, 2e-6)):
        co, so = _table(pos, inv, scale, fast)
        assert np.abs(co - c_ref).max() <= tol * scale, (fast, np.abs(co - c_ref).max())
        assert np.abs(so - s_ref).max() <= tol * scale, (fast, np.abs(so - s_ref).max())
