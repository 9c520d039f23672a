"""Model-level parity: a random-init Llama on the CUDA cache, driven as the
reference's harness drives it (chunked prefill with consolidate, one-token
greedy decode at true positions), against logits the reference's own
``BugStreamingCache`` produced for the same model and prompt
(``tests/golden/model_llama_tiny.npz``, made by ``make_golden.py``).

The decode steps run both ways: through SDPA over the cache's dense peek
(the reference's path) and through the factored decode kernel selected with
``enable_factored_decode`` -- transformers' ``LlamaAttention`` then calls the
kernel itself.  Tolerances are relative to the step's largest logit: fp32
2e-3 (the cache states differ by fp32 rounding of the BUG math and of the
attention), bf16 2e-2 (the attention rule for bf16).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from golden.make_golden import MODEL_CASE, tiny_llama

from kvdlra_b200 import BugStreamingCache, BugStreamingLayer, enable_factored_decode
from kvdlra_b200.harness import decode_greedy, prefill_chunked

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
GOLDEN = Path(__file__).resolve().parent / "golden"


def _rel(a: torch.Tensor, b: np.ndarray) -> float:
    a64 = a.double().cpu().numpy()
    return float(np.abs(a64 - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("factored", [False, True])
def test_tiny_llama_matches_reference_logits(factored: bool) -> None:
    g = np.load(GOLDEN / "model_llama_tiny.npz")
    c = MODEL_CASE
    model = tiny_llama(c).to(DEV)
    if factored:
        enable_factored_decode(model)
    cache = BugStreamingCache(model, **c["cache_kw"])
    ids = torch.from_numpy(g["ids"]).to(DEV)
    worst = 0.0
    with torch.no_grad():
        with cache.ingesting():
            for i, start in enumerate(range(0, c["tokens"], c["chunk"])):
                stop = min(c["tokens"], start + c["chunk"])
                pos = torch.arange(start, stop, device=DEV).unsqueeze(0)
                out = model(ids[:, start:stop], past_key_values=cache, use_cache=True, position_ids=pos,
                            logits_to_keep=1)
                cache.consolidate()
                worst = max(worst, _rel(out.logits[0, -1], g["chunk_logits"][i]))
        first = torch.from_numpy(g["chunk_logits"][-1])[None].to(DEV)
        forced = torch.from_numpy(g["dec_tokens"])[None]
        toks, logits = decode_greedy(model, cache, first, c["tokens"], c["decode"], forced=forced)
    for j in range(c["decode"]):
        worst = max(worst, _rel(logits[0, j], g["dec_logits"][j]))
    assert worst < 2e-3, worst
    assert cache.stored_state_numel() == int(g["stored_numel"])
    cache.check_status()


def test_factored_decode_behind_llama_attention_bf16(monkeypatch) -> None:
    """bf16: the same prompt and teacher-forced tokens through the factored
    kernels (chunk attention for the ingest chunks, factored decode for the
    steps) and through SDPA over the dense peek agree within the bf16 rule,
    and greedy ``model.generate`` runs on the factored path."""
    g = np.load(GOLDEN / "model_llama_tiny.npz")
    c = MODEL_CASE
    model = tiny_llama(c).to(DEV, torch.bfloat16)
    ids = torch.from_numpy(g["ids"]).to(DEV)
    forced = torch.from_numpy(g["dec_tokens"])[None]
    calls = {"chunk": 0, "decode": 0}
    chunk_fn, dec_fn = BugStreamingLayer.factored_chunk_attention, BugStreamingLayer.factored_attention

    def chunk_spy(self, *a, **k):
        calls["chunk"] += 1
        return chunk_fn(self, *a, **k)

    def dec_spy(self, *a, **k):
        calls["decode"] += 1
        return dec_fn(self, *a, **k)

    monkeypatch.setattr(BugStreamingLayer, "factored_chunk_attention", chunk_spy)
    monkeypatch.setattr(BugStreamingLayer, "factored_attention", dec_spy)
    runs = {}
    for mode in ("sdpa", "factored"):
        if mode == "factored":
            enable_factored_decode(model)
        else:
            model.set_attn_implementation("sdpa")
        cache = BugStreamingCache(model, **c["cache_kw"])
        first = prefill_chunked(model, cache, ids, c["chunk"], keep_logits=True)
        _, logits = decode_greedy(model, cache, first, c["tokens"], c["decode"], forced=forced)
        runs[mode] = torch.cat([first[:, None].float(), logits.float()], dim=1)
    ref = runs["sdpa"]
    err = float((runs["factored"] - ref).abs().max() / ref.abs().max())
    assert err < 2e-2, err
    # every chunk after the first (the single-shot prefill) and every step, per layer
    n_chunks = -(-c["tokens"] // c["chunk"])
    assert calls["chunk"] == c["layers"] * (n_chunks - 1), calls
    assert calls["decode"] == c["layers"] * c["decode"], calls
    # model.generate: single-shot prefill of the prompt, then factored decode steps
    cache = BugStreamingCache(model, **c["cache_kw"])
    out = model.generate(ids[:, :256], past_key_values=cache, max_new_tokens=12, do_sample=False)
    assert out.shape[1] == 256 + 12
    assert cache.get_seq_length() == 256 + 11
    cache.check_status()


def test_frozen_scoring_through_chunk_attention_bf16() -> None:
    """``frozen_scoring()`` (bug_cache.py:1871-1882, 1390-1402) under the
    factored attention: a window scored against the retained cache (the
    window as the chunk kernel's tail, nothing mutated) gives the logits SDPA
    over the dense ``[retained | window]`` gives, within the bf16 rule."""
    g = np.load(GOLDEN / "model_llama_tiny.npz")
    c = MODEL_CASE
    model = tiny_llama(c).to(DEV, torch.bfloat16)
    ids = torch.from_numpy(g["ids"]).to(DEV)
    ctx, win = ids[:, :512], ids[:, 512:640]
    pos = torch.arange(512, 640, device=DEV)[None]
    out = {}
    for mode in ("sdpa", "factored"):
        if mode == "factored":
            enable_factored_decode(model)
        else:
            model.set_attn_implementation("sdpa")
        cache = BugStreamingCache(model, **c["cache_kw"])
        prefill_chunked(model, cache, ctx, c["chunk"])
        n0 = cache.stored_state_numel()
        with torch.no_grad(), cache.frozen_scoring():
            out[mode] = model(win, past_key_values=cache, use_cache=True, position_ids=pos).logits.float()
        assert cache.stored_state_numel() == n0  # scoring does not mutate
        assert cache.get_seq_length() == 512
        cache.check_status()
    err = float((out["factored"] - out["sdpa"]).abs().max() / out["sdpa"].abs().max())
    assert err < 2e-2, err
