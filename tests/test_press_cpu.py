"""BUGPress host logic without a GPU: the reference's constructor guards,
the nominal compression ratio, the config-driven feature count and the
single-shot guard (tests/test_bug_press.py:145-216 of the reference,
restated), plus the loud refusal of CPU tensors."""

from __future__ import annotations

from types import SimpleNamespace
from typing import Any, cast

import pytest
import torch

from kvdlra_b200 import BUGPress


def test_compression_ratio_value_and_readonly() -> None:
    press = BUGPress(rank=32, n_sink=4)
    press.n_features = 512
    assert press.compression_ratio == pytest.approx(1.0 - 32 / 512)
    with pytest.raises(AttributeError):
        press.compression_ratio = 0.5


def test_post_init_from_model_sets_n_features() -> None:
    cfg = SimpleNamespace(num_attention_heads=32, num_key_value_heads=8, head_dim=64, hidden_size=2048)
    press = BUGPress(rank=16)
    press.post_init_from_model(cast(Any, SimpleNamespace(config=cfg)))
    assert press.n_features == 512
    cfg2 = SimpleNamespace(num_attention_heads=32, num_key_value_heads=8, hidden_size=4096)
    press.post_init_from_model(cast(Any, SimpleNamespace(config=cfg2)))
    assert press.n_features == 8 * 128


def test_constructor_guards() -> None:
    with pytest.raises(ValueError, match="rank"):
        BUGPress(rank=0)
    with pytest.raises(ValueError, match="n_sink"):
        BUGPress(rank=8, n_sink=-1)
    with pytest.raises(ValueError, match="n_exact"):
        BUGPress(rank=8, n_exact=-1)
    with pytest.raises(ValueError, match="backend"):
        BUGPress(rank=8, backend="jax")
    with pytest.raises(ValueError, match="block_size"):
        BUGPress(rank=8, block_size=0)
    with pytest.raises(ValueError, match="quant_bits requires backend='torch'"):
        BUGPress(rank=16, quant_bits=4, backend="numpy")
    with pytest.raises(ValueError, match="quant_bits must be"):
        BUGPress(rank=16, quant_bits=0)


def test_compress_rejects_partial_cache_forward() -> None:
    press = BUGPress(rank=8)
    hidden = torch.zeros(1, 8, 16)
    keys = torch.zeros(1, 8, 16, 64)
    values = torch.zeros(1, 8, 16, 64)
    with pytest.raises(NotImplementedError, match="single-shot"):
        press.compress(cast(Any, None), hidden, keys, values, cast(Any, None), {})


def test_cpu_tensors_and_out_of_scope_options_fail_loudly() -> None:
    x = torch.zeros(1, 8, 40, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        BUGPress(rank=8)._compress_tensor(x)
    with pytest.raises(NotImplementedError, match="numpy"):
        BUGPress(rank=8, backend="numpy")._compress_tensor(x)
    with pytest.raises(NotImplementedError, match="quant_bits"):
        BUGPress(rank=8, quant_bits=4)._compress_tensor(x)


def test_short_context_is_returned_unchanged_without_compute() -> None:
    x = torch.randn(1, 8, 3, 64)
    assert torch.equal(BUGPress(rank=8, n_sink=4)._compress_tensor(x), x)
