"""Host-side API checks that need no GPU: constructor validation (same
messages as the reference, bug_cache.py:342-494), scope errors, and the
no-CPU-fallback guarantee."""

from __future__ import annotations

import pytest
import torch

from kvdlra_b200 import BugStreamingCache, BugStreamingLayer, RopeAngles

ROPE = RopeAngles(inv_freq=torch.ones(8))


def _cache(**kw):
    return BugStreamingCache(None, num_layers=2, rope=ROPE, **kw)


def test_constructor_validation_messages() -> None:
    with pytest.raises(ValueError, match="recent_window"):
        _cache(rank=8, coord_budget=16, recent_window=0)
    with pytest.raises(ValueError, match=">= 0"):
        _cache(rank=-1, coord_budget=16)
    with pytest.raises(ValueError, match="absorb_block"):
        _cache(rank=8, coord_budget=16, absorb_block=0)
    with pytest.raises(ValueError, match="hh_select must be"):
        _cache(rank=4, coord_budget=32, hh_budget=4, hh_select="bogus")
    with pytest.raises(ValueError, match="requires retention='attn'"):
        _cache(rank=4, coord_budget=32, retention="lowrank_surprise", hh_budget=4, hh_select="attn")
    with pytest.raises(ValueError, match=r"hh_neighbor.*requires hh_select='surprise'"):
        _cache(rank=4, coord_budget=32, retention="attn", hh_budget=4, hh_select="attn", hh_neighbor=1)
    for kw in ({"merge": True}, {"quant_bits": 4, "quant_budget": 16}):
        with pytest.raises(ValueError, match="fp32 low-rank tail only"):
            _cache(rank=4, coord_budget=64, recent_window=8, absorb_block=4,
                   retention="lowrank_surprise", hh_budget=2, hh_select="surprise",
                   seed_hh_warmup=True, **kw)
    with pytest.raises(ValueError, match="hh_budget >= 1"):
        _cache(rank=4, coord_budget=32, hh_retain=False)


def test_in_scope_configs_construct() -> None:
    _cache(rank=4, coord_budget=32, retention="lowrank_surprise", hh_budget=4, hh_select="surprise")
    _cache(rank=4, coord_budget=32, retention="fifo", hh_budget=4, hh_select="surprise")
    _cache(rank=0, coord_budget=0)  # sinks + recent window only


@pytest.mark.parametrize("kw", [
    {"retention": "attn"}, {"retention": "energy"}, {"retention": "blend"},
    {"quant_bits": 4, "quant_budget": 8},
])
def test_out_of_scope_variants_raise_not_implemented(kw) -> None:
    with pytest.raises(NotImplementedError):
        _cache(rank=4, coord_budget=32, **kw)


def test_cpu_tensors_are_rejected_loudly() -> None:
    layer = BugStreamingLayer(ROPE, rank=4, coord_budget=32)
    k = torch.zeros(1, 2, 8, 16)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        layer.update(k, k)


def test_fresh_layer_lengths_and_masks() -> None:
    layer = BugStreamingLayer(ROPE, rank=4, coord_budget=32, recent_window=8, absorb_block=4)
    assert layer.get_seq_length() == 0
    assert layer.get_mask_sizes(10) == (10, 0)  # prefill returns the full input
    assert layer.get_max_cache_shape() == -1
    assert layer.stored_state_numel() == 0


def test_mode_context_managers_restore_normal() -> None:
    cache = _cache(rank=4, coord_budget=32)
    with cache.ingesting():
        assert all(ly._mode == "ingest" for ly in cache.layers)
    assert all(ly._mode == "normal" for ly in cache.layers)
    with pytest.raises(KeyError):
        with cache.frozen_scoring():
            assert all(ly._mode == "score" for ly in cache.layers)
            raise KeyError("x")
    assert all(ly._mode == "normal" for ly in cache.layers)


def test_factored_attention_routing_without_gpu() -> None:
    """transformers' attention call (attention.py): an untagged key goes to
    SDPA; a tagged key goes to the chunk kernel in ingest (no tail) and score
    (the step's own K/V as tail) modes and to the factored decode otherwise,
    with the output in transformers' (B, q, Hq, D) layout.  A module with a
    KV-head range passes it to the kernels and gives SDPA only those heads.
    The layer is a stand-in that records the calls (nothing runs on a GPU)."""
    from kvdlra_b200 import attention as A

    calls, heads_seen = [], []

    class FakeLayer:
        def __init__(self, mode):
            self._mode = mode

        def factored_chunk_attention(self, query, scaling=None, tail=None, heads=None):
            calls.append(("chunk", self._mode, tail is not None, tuple(query.shape)))
            heads_seen.append(heads)
            b, hq, q, d = query.shape
            return torch.zeros(b, q, hq, d)

        def factored_attention(self, query, scaling=None, heads=None):
            calls.append(("decode", self._mode, False, tuple(query.shape)))
            heads_seen.append(heads)
            return torch.zeros(query.shape)

    module = torch.nn.Module()
    module.num_key_value_groups, module.is_causal = 2, True
    q = torch.zeros(1, 4, 5, 8)
    k = torch.zeros(1, 2, 5, 8)
    v = torch.zeros(1, 2, 5, 8)
    out, _ = A.factored_attention_forward(module, q, k, v, None)  # untagged: SDPA
    assert tuple(out.shape) == (1, 5, 4, 8) and not calls
    for mode, expect_tail in (("ingest", False), ("score", True)):
        kk = A.tag_step(k.clone(), FakeLayer(mode))
        out, w = A.factored_attention_forward(module, q, kk, v, None, scaling=0.5)
        assert w is None and tuple(out.shape) == (1, 5, 4, 8)
        assert calls[-1] == ("chunk", mode, expect_tail, (1, 4, 5, 8))
    q1 = torch.zeros(1, 4, 1, 8)
    kd = A.tag_step(torch.zeros(1, 2, 1, 8), FakeLayer("normal"))
    out, _ = A.factored_attention_forward(module, q1, kd, torch.zeros(1, 2, 1, 8), None)
    assert tuple(out.shape) == (1, 1, 4, 8) and calls[-1][0] == "decode"
    with pytest.raises(RuntimeError, match="one query token"):
        A.factored_attention_forward(module, q, A.tag_step(k.clone(), FakeLayer("normal")), v, None)
    with pytest.raises(NotImplementedError, match="dropout"):
        A.factored_attention_forward(module, q, A.tag_step(k.clone(), FakeLayer("ingest")), v, None,
                                     dropout=0.1)
    assert all(h is None for h in heads_seen)
    # KV head 1 of 2 (query heads 2, 3): the kernels get the range, SDPA the head
    module.kvd_heads = (1, 1)
    q2 = torch.randn(1, 2, 5, 8)
    k2, v2 = torch.randn(1, 2, 5, 8), torch.randn(1, 2, 5, 8)
    out, _ = A.factored_attention_forward(module, q2, k2, v2, None)
    ref, _ = A.sdpa_attention_forward(module, q2, k2[:, 1:], v2[:, 1:], None)
    assert torch.equal(out, ref)
    A.factored_attention_forward(module, q2, A.tag_step(k2.clone(), FakeLayer("ingest")), v2, None)
    A.factored_attention_forward(module, q2[:, :, :1], A.tag_step(k2[:, :, :1].clone(), FakeLayer("normal")),
                                 v2[:, :, :1], None)
    assert heads_seen[-2:] == [(1, 1), (1, 1)]
