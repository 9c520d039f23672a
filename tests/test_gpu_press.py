"""BUGPress on the GPU: the reference's math tests (tests/test_bug_press.py
of the reference, restated for CUDA tensors), parity of the blocked BUG
projection with the oracle, and the press hook on a small random-init Llama.

Tolerances: exact columns byte-identical; full-rank / exact-rank recovery to
1e-4 absolute (the reference's torch-backend bound, fp32 compute); oracle
parity on reconstruction within 1e-4 relative and principal angle <= 1e-3.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.bug_oracle import blocked_bug_project as oracle_project
from oracle.bug_oracle import blocked_bug_subspace as oracle_subspace
from oracle.bug_oracle import principal_angle

from kvdlra_b200 import BUGPress, blocked_bug_project

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
H, D = 8, 64
N_FEATURES = H * D


def _random_kv(bsz: int, t: int, seed: int = 0, dtype=torch.float64) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(bsz, H, t, D, generator=g, dtype=torch.float64).to(DEV, dtype)


def test_shape_and_dtype_preserved() -> None:
    x = _random_kv(bsz=2, t=40)
    out = BUGPress(rank=8)._compress_tensor(x)
    assert out.shape == x.shape and out.dtype == x.dtype and out.device == x.device


def test_full_rank_recovers_input() -> None:
    t = 40
    x = _random_kv(bsz=1, t=t, seed=1)
    out = BUGPress(rank=t, n_sink=4)._compress_tensor(x)
    assert torch.allclose(out, x, atol=1e-4)


def test_sinks_preserved_exactly_at_low_rank() -> None:
    x = _random_kv(bsz=1, t=60, seed=2)
    out = BUGPress(rank=2, n_sink=4)._compress_tensor(x)
    assert torch.equal(out[:, :, :4, :], x[:, :, :4, :])
    assert not torch.allclose(out[:, :, 4:, :], x[:, :, 4:, :])


def test_n_exact_zero_is_pure_lowrank() -> None:
    mat = torch.randn(N_FEATURES, 200, generator=torch.Generator().manual_seed(3)).to(DEV)
    a = BUGPress(rank=16, n_exact=0)._lowrank_reconstruct(mat)
    b = BUGPress(rank=16)._lowrank_reconstruct(mat)
    assert torch.equal(a, b)


def test_hybrid_keeps_high_norm_tokens_exact_and_helps() -> None:
    g = torch.Generator().manual_seed(4)
    mat = torch.randn(N_FEATURES, 300, generator=g) * 0.3
    outliers = torch.tensor([20, 77, 140, 210, 260])
    mat[:, outliers] *= 10.0
    mat = mat.to(DEV)
    press = BUGPress(rank=32, n_exact=len(outliers))
    mask = press._exact_mask(mat)
    kept = set(torch.nonzero(mask).flatten().cpu().tolist())
    assert kept == set(range(4)) | set(outliers.tolist())
    out = press._lowrank_reconstruct(mat)
    assert torch.equal(out[:, mask], mat[:, mask])
    nonx = ~mask
    pure = BUGPress(rank=32)._lowrank_reconstruct(mat)
    hyb_err = torch.linalg.norm(mat[:, nonx] - out[:, nonx])
    pure_err = torch.linalg.norm(mat[:, nonx] - pure[:, nonx])
    assert hyb_err <= pure_err + 1e-6


def test_exact_set_ties_and_saturation() -> None:
    """Top-n_exact by norm with equal norms resolved to the lower index, and
    n_exact past the column count keeping every column."""
    mat = torch.ones(16, 12, device=DEV)
    mat[:, 9] = 3.0
    press = BUGPress(rank=4, n_sink=2, n_exact=3)
    kept = torch.nonzero(press._exact_mask(mat)).flatten().cpu().tolist()
    assert kept == [0, 1, 2, 3, 9]
    everything = BUGPress(rank=4, n_sink=2, n_exact=50)._exact_mask(mat)
    assert bool(everything.all())


def test_exact_rank_r_input_reconstructed_exactly() -> None:
    r, t = 5, 50
    rng = np.random.default_rng(3)
    mat = rng.standard_normal((N_FEATURES, r)) @ rng.standard_normal((r, t))
    x = torch.from_numpy(mat).reshape(H, D, t).permute(0, 2, 1).unsqueeze(0).to(DEV)
    out = BUGPress(rank=r, n_sink=0)._compress_tensor(x)
    assert torch.allclose(out, x, atol=1e-4)


def test_low_rank_is_lossy_on_full_rank_input() -> None:
    x = _random_kv(bsz=1, t=80, seed=4)
    out = BUGPress(rank=4, n_sink=0)._compress_tensor(x)
    rel = float((out - x).norm() / x.norm())
    assert 0.0 < rel < 1.0


@pytest.mark.parametrize("t,rank,block", [(300, 16, 128), (1000, 32, 64), (257, 24, 16)])
def test_blocked_projection_matches_oracle(t: int, rank: int, block: int) -> None:
    """Blocked BUG projection against the oracle (streaming_torch.py:192-258):
    low-rank-plus-noise columns, several block sizes and a ragged last block."""
    rng = np.random.default_rng(t)
    basis = np.linalg.qr(rng.standard_normal((N_FEATURES, rank + 4)))[0]
    coef = rng.standard_normal((rank + 4, t)) * (2.0 ** (-np.arange(rank + 4) / 3))[:, None]
    mat = (basis @ coef + 1e-3 * rng.standard_normal((N_FEATURES, t))).astype(np.float32)
    got = blocked_bug_project(torch.from_numpy(mat).to(DEV), rank, block).cpu().numpy()
    ref = oracle_project(mat, rank, block)
    assert np.linalg.norm(got - ref) <= 1e-4 * np.linalg.norm(ref)
    # the subspace the projection used is the oracle's
    u_ref = oracle_subspace(mat, rank, block)
    q = np.linalg.qr(got)[0][:, :rank]
    assert principal_angle(q, u_ref) < 1e-3


def test_press_hook_on_small_llama() -> None:
    """The press inside a model forward: keys are replaced by the rank-r
    reconstruction of the pre-RoPE keys re-rotated, values by theirs; the
    cache keeps its shape and the hook is removed afterwards."""
    transformers = pytest.importorskip("transformers")
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=4, head_dim=32, vocab_size=128,
                      max_position_embeddings=512, rope_theta=10000.0)
    model = LlamaForCausalLM(cfg).to(DEV).eval()
    ids = torch.randint(0, 128, (1, 96), generator=torch.Generator().manual_seed(1)).to(DEV)
    with torch.no_grad():
        plain = model(ids, use_cache=True).past_key_values
        press = BUGPress(rank=8, n_sink=4)
        press.post_init_from_model(model)
        assert press.n_features == 4 * 32
        with press(model):
            pressed = model(ids, use_cache=True).past_key_values
        again = model(ids, use_cache=True).past_key_values  # hooks are gone
    for li in range(2):
        k0, v0 = plain.layers[li].keys, plain.layers[li].values
        k1, v1 = pressed.layers[li].keys, pressed.layers[li].values
        assert k1.shape == k0.shape and v1.shape == v0.shape
        assert torch.equal(v1[:, :, :4], v0[:, :, :4])          # sinks exact
        assert not torch.allclose(v1[:, :, 4:], v0[:, :, 4:])  # the rest low-rank
        expect_v = BUGPress(rank=8, n_sink=4)._compress_tensor(v0)
        assert torch.allclose(v1, expect_v, atol=1e-5)
        assert torch.equal(again.layers[li].keys, k0)
