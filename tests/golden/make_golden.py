"""Generate the golden fixtures by running the reference kvdlra implementation.

Run where the reference source tree is available (read-only is enough)::

    python tests/golden/make_golden.py <reference>/src [case ...]

or with ``KVDLRA_REFERENCE_SRC=<reference>/src`` set; naming cases regenerates
only those fixtures.
It imports the reference's own ``BugStreamingLayer`` / ``augmented_bug_step``
(src/kvdlra/cache/bug_cache.py, src/kvdlra/integrators/streaming_torch.py),
drives it on seeded synthetic inputs from ``kvdlra_b200.synthetic`` and stores
the outputs as small ``.npz`` files beside this script.  The fixtures pin the
CPU oracle (``oracle/bug_oracle.py``); the GPU parity tests then compare the
CUDA path against that oracle.  Nothing at test time reads the reference.
"""

from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from kvdlra_b200.synthetic import gaussian_kv, lowrank_stream  # noqa: E402


def _sha(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _rotary(head_dim: int, theta: float):
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    cfg = LlamaConfig(
        hidden_size=head_dim * 4, num_attention_heads=4, num_key_value_heads=2,
        head_dim=head_dim, rope_theta=theta, max_position_embeddings=1 << 17,
    )
    return LlamaRotaryEmbedding(cfg)


def _layer(rotary, **kw):
    from kvdlra.cache.bug_cache import BugStreamingLayer, _RopeAngles

    return BugStreamingLayer(rope=_RopeAngles(rotary), **kw)


def _instrument(layer) -> list[dict]:
    """Record every SLASH selection event: candidate positions, selection
    scores and kept positions."""
    trace: list[dict] = []
    orig_slash = layer._absorb_block_slash
    orig_surprise = layer._surprise_scores
    state = {"want": False, "sel": None}

    def surprise(block_k):
        out = orig_surprise(block_k)
        if state["want"]:
            state["sel"] = out.clone()
            state["want"] = False
        return out

    def slash(grad_k, grad_v, grad_pos, grad_score):
        prev = layer.hh_pos.clone() if layer.hh_pos is not None else grad_pos[:0]
        cand_pos = np.concatenate([prev.numpy(), grad_pos.numpy()])
        state["want"] = True
        orig_slash(grad_k, grad_v, grad_pos, grad_score)
        sel = state["sel"].numpy()
        if layer.hh_neighbor > 0:
            import torch

            sel = layer._span_boost(torch.from_numpy(sel), torch.from_numpy(cand_pos), layer.hh_neighbor).numpy()
        trace.append({"cand_pos": cand_pos, "sel": sel, "keep_pos": layer.hh_pos.numpy().copy()})

    layer._absorb_block_slash = slash
    layer._surprise_scores = surprise
    return trace


def _boundary_gap(trace: list[dict], keep_counts: list[int]) -> float:
    """Smallest relative gap between the last kept and first demoted score
    (exactly equal scores -- e.g. all 1.0 before a basis exists -- are decided
    by the stable index rule on every implementation and are skipped)."""
    best = np.inf
    for ev, keep_n in zip(trace, keep_counts):
        s = np.sort(ev["sel"].astype(np.float64))[::-1]
        if keep_n < len(s):
            a, b = s[keep_n - 1], s[keep_n]
            if a != b:
                best = min(best, (a - b) / max(abs(a), 1e-30))
    return float(best)


def _pack_trace(trace: list[dict]) -> dict[str, np.ndarray]:
    off = np.cumsum([0] + [len(e["cand_pos"]) for e in trace])
    koff = np.cumsum([0] + [len(e["keep_pos"]) for e in trace])
    return {
        "tr_cand_off": off.astype(np.int64),
        "tr_cand_pos": np.concatenate([e["cand_pos"] for e in trace]).astype(np.int32) if trace else np.zeros(0, np.int32),
        "tr_sel": np.concatenate([e["sel"] for e in trace]).astype(np.float32) if trace else np.zeros(0, np.float32),
        "tr_keep_off": koff.astype(np.int64),
        "tr_keep_pos": np.concatenate([e["keep_pos"] for e in trace]).astype(np.int32) if trace else np.zeros(0, np.int32),
    }


def _tdtype(name: str):
    import torch

    return {"float32": torch.float32, "bfloat16": torch.bfloat16}[name]


def _ingest(layer, k_htd: np.ndarray, v_htd: np.ndarray, chunk: int,
            dtype: str = "float32") -> list[tuple[int, int]]:
    """Chunked ingest through the reference layer; returns the mask sizes seen."""
    import torch

    t = k_htd.shape[1]
    masks = []
    layer._mode = "ingest"
    dt = _tdtype(dtype)
    for start in range(0, t, chunk):
        stop = min(t, start + chunk)
        k = torch.from_numpy(np.ascontiguousarray(k_htd[:, start:stop]))[None].to(dt)
        v = torch.from_numpy(np.ascontiguousarray(v_htd[:, start:stop]))[None].to(dt)
        if layer.is_initialized:
            masks.append(layer.get_mask_sizes(stop - start))
        layer.update(k, v)
        layer.consolidate()
    layer._mode = "normal"
    return masks


def _state(layer) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    # (coordinates are not stored: the tests recompute the gist from the oracle's own)
    for name in ("u_k", "u_v", "hh_pos", "mid_pos", "mid_surprise"):
        t = getattr(layer, name)
        if t is not None:
            out[name] = t.numpy().copy()
    for name in ("b_k", "b_v"):
        t = getattr(layer, name)
        if t is not None:
            out["sigma_" + name[-1]] = np.diag(t.numpy()).copy()
    out["stored_numel"] = np.array(layer.stored_state_numel(), np.int64)
    out["attended"] = np.array(layer.attended_length(), np.int64)
    out["cumulative"] = np.array(layer.cumulative_length, np.int64)
    return out


def case_steps() -> dict[str, np.ndarray]:
    """A sequence of augmented BUG steps on float32 data."""
    import torch
    from kvdlra.integrators.streaming_torch import augmented_bug_step

    rng = np.random.default_rng(11)
    n, rank = 48, 12
    # Low-rank-plus-noise columns so the spectrum has structure.
    basis = np.linalg.qr(rng.standard_normal((n, 20)))[0]
    coef = rng.standard_normal((20, 112)) * (2.0 ** (-np.arange(20) / 3.0))[:, None]
    data = (basis @ coef + 0.01 * rng.standard_normal((n, 112))).astype(np.float32)
    blocks = [16, 16, 8, 32, 24, 16]
    u = b = None
    out: dict[str, np.ndarray] = {"data": data, "blocks": np.array(blocks, np.int64)}
    start = 0
    for i, bs in enumerate(blocks):
        blk = torch.from_numpy(data[:, start : start + bs].copy())
        u, b, rot = augmented_bug_step(u, b, blk, rank)
        out[f"u_{i}"] = u.numpy().copy()
        out[f"sigma_{i}"] = torch.diag(b).numpy().copy()
        out[f"rot_{i}"] = rot.numpy().copy()
        start += bs
    return out


MODEL_CASE = dict(vocab=256, hidden=256, ffn=512, layers=2, heads=8, kv_heads=2, head_dim=64,
                  theta=500000.0, tokens=704, chunk=128, decode=24, seed=0,
                  cache_kw=dict(rank=16, coord_budget=4096, recent_window=32, absorb_block=16,
                                n_sink=4, retention="lowrank_surprise", hh_budget=32,
                                hh_select="surprise"))


def tiny_llama(case: dict):
    """The random-init Llama of the model-level fixture (fp32, CPU init:
    ``torch.manual_seed`` then ``LlamaForCausalLM`` -- the same weights on
    every machine with this torch)."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=case["vocab"], hidden_size=case["hidden"],
                      intermediate_size=case["ffn"], num_hidden_layers=case["layers"],
                      num_attention_heads=case["heads"], num_key_value_heads=case["kv_heads"],
                      head_dim=case["head_dim"], rope_theta=case["theta"],
                      max_position_embeddings=1 << 16, initializer_range=0.02)
    torch.manual_seed(case["seed"])
    return LlamaForCausalLM(cfg).eval()


def case_model() -> dict[str, np.ndarray]:
    """The reference's BugStreamingCache under a random-init Llama, driven as
    its harness does (scripts/w10_frontier.py:72-91 chunked prefill with
    consolidate, scripts/w10_ruler.py:176-189 greedy decode): the last
    position's logits after every chunk, the greedy tokens and their logits."""
    import torch
    from kvdlra.cache import BugStreamingCache

    c = MODEL_CASE
    model = tiny_llama(c)
    ids = torch.randint(0, c["vocab"], (1, c["tokens"]), generator=torch.Generator().manual_seed(c["seed"] + 1))
    cache = BugStreamingCache(model, **c["cache_kw"])
    chunk_logits = []
    with torch.no_grad():
        with cache.ingesting():
            for start in range(0, c["tokens"], c["chunk"]):
                stop = min(c["tokens"], start + c["chunk"])
                pos = torch.arange(start, stop).unsqueeze(0)
                out = model(ids[:, start:stop], past_key_values=cache, use_cache=True, position_ids=pos,
                            logits_to_keep=1)
                cache.consolidate()
                chunk_logits.append(out.logits[0, -1].numpy().copy())
        nxt = int(out.logits[0, -1].argmax())
        toks, dec_logits = [], []
        for j in range(c["decode"]):
            toks.append(nxt)
            pos = torch.tensor([[c["tokens"] + j]])
            out = model(torch.tensor([[nxt]]), past_key_values=cache, use_cache=True, position_ids=pos)
            dec_logits.append(out.logits[0, -1].numpy().copy())
            nxt = int(out.logits[0, -1].argmax())
    lay = cache.layers[0]
    print(f"model: numel={cache.stored_state_numel()} hh={lay._hh_len()} W={lay._f_len()}")
    return {"ids": ids.numpy(), "chunk_logits": np.stack(chunk_logits), "dec_tokens": np.array(toks, np.int64),
            "dec_logits": np.stack(dec_logits), "stored_numel": np.array(cache.stored_state_numel(), np.int64),
            "hh_pos0": lay.hh_pos.numpy().copy()}


def _run_case(name: str, *, heads: int, head_dim: int, t: int, chunk: int, theta: float,
              layer_kw: dict, stream_kw: dict, n_queries: int = 0, q_heads: int = 0,
              decode_tokens: int = 0, seed: int = 0, dtype: str = "float32") -> dict[str, np.ndarray]:
    import torch

    s = lowrank_stream(heads, head_dim, t + decode_tokens, theta=theta, seed=seed, **stream_kw)
    rotary = _rotary(head_dim, theta)
    layer = _layer(rotary, **layer_kw)
    trace = _instrument(layer)
    masks = _ingest(layer, s.k_post[:, :t], s.v[:, :t], chunk, dtype)
    out = {"input_sha": np.frombuffer(bytes.fromhex(_sha(s.k_post, s.v)), np.uint8)}
    out.update(_pack_trace(trace))
    out["mask_sizes"] = np.array(masks, np.int64).reshape(-1, 2)
    out.update({"final_" + k: v for k, v in _state(layer).items()})
    hh = layer_kw.get("hh_budget", 0)
    out["boundary_gap"] = np.array(_boundary_gap(trace, [min(hh, len(e["cand_pos"])) for e in trace]))
    k_ret, v_ret = layer._decode_peek()
    k_ret, v_ret = k_ret.float(), v_ret.float()  # attention over the peek's values in fp32
    out["peek_k_sum"] = np.array(float(k_ret.double().sum()))
    out["peek_v_sum"] = np.array(float(v_ret.double().sum()))
    out["peek_len"] = np.array(k_ret.shape[2], np.int64)
    # gist error over the middle, in the reference's own state
    if layer.c_k is not None and layer.mid_pos is not None:
        pos = layer.mid_pos.numpy()
        kp = np.concatenate([s.k_pre[h][pos].T for h in range(heads)], axis=0)  # (n, W)
        rec = (layer.u_k @ layer.c_k).double().numpy()
        out["gist_err_k"] = np.array(np.linalg.norm(kp - rec) / np.linalg.norm(kp))
        vp = np.concatenate([s.v[h][pos].T for h in range(heads)], axis=0)
        recv = (layer.u_v @ layer.c_v).double().numpy()
        out["gist_err_v"] = np.array(np.linalg.norm(vp - recv) / np.linalg.norm(vp))
    if n_queries:
        rng = np.random.default_rng(seed + 1000)
        qs = rng.standard_normal((n_queries, q_heads, head_dim)).astype(np.float32)
        outs = []
        for qi in range(n_queries):
            q = torch.from_numpy(qs[qi])[None, :, None, :]  # (1, Hq, 1, D)
            o = torch.nn.functional.scaled_dot_product_attention(
                q, k_ret, v_ret, enable_gqa=True
            )
            outs.append(o[0, :, 0, :].numpy().copy())
        out["queries"] = qs
        out["attn_out"] = np.stack(outs)
    if decode_tokens:
        dec_masks, dec_numel = [], []
        for j in range(decode_tokens):
            p = t + j
            k = torch.from_numpy(np.ascontiguousarray(s.k_post[:, p : p + 1]))[None].to(_tdtype(dtype))
            v = torch.from_numpy(np.ascontiguousarray(s.v[:, p : p + 1]))[None].to(_tdtype(dtype))
            dec_masks.append(layer.get_mask_sizes(1))
            kr, _ = layer.update(k, v)
            assert kr.shape[2] == dec_masks[-1][0]
            dec_numel.append(layer.stored_state_numel())
        out["dec_masks"] = np.array(dec_masks, np.int64)
        out["dec_numel"] = np.array(dec_numel, np.int64)
        if layer.hh_pos is not None:
            out["dec_hh_pos"] = layer.hh_pos.numpy().copy()
        out["dec_trace_len"] = np.array(len(trace), np.int64)
    out["trace_len"] = np.array(len(trace), np.int64)
    print(f"{name}: absorbs={len(trace)} boundary_gap={float(out['boundary_gap']):.3e} "
          f"numel={int(out['final_stored_numel'])}")
    return out


CASES = {
    "slash_tiny": dict(heads=2, head_dim=16, t=96, chunk=16, theta=10000.0,
                       layer_kw=dict(rank=4, coord_budget=4096, recent_window=8, absorb_block=4,
                                     n_sink=4, retention="lowrank_surprise", hh_budget=8,
                                     hh_select="surprise"),
                       stream_kw=dict(signal_rank=3, n_needles=3), n_queries=2, q_heads=4,
                       decode_tokens=9, seed=3),
    "cfg1_reduced": dict(heads=8, head_dim=64, t=1536, chunk=256, theta=500000.0,
                         layer_kw=dict(rank=32, coord_budget=1536 + 128 + 16, recent_window=128,
                                       absorb_block=16, n_sink=4, retention="lowrank_surprise",
                                       hh_budget=128, hh_select="surprise"),
                         stream_kw=dict(n_needles=6), n_queries=3, q_heads=32, seed=0),
    "seed_warmup": dict(heads=4, head_dim=32, t=768, chunk=256, theta=500000.0,
                        layer_kw=dict(rank=16, coord_budget=768 + 64 + 16, recent_window=64,
                                      absorb_block=16, n_sink=4, prefill_block_size=32,
                                      retention="lowrank_surprise", hh_budget=32,
                                      hh_select="surprise", seed_hh_warmup=True),
                        stream_kw=dict(signal_rank=8, n_needles=5), n_queries=1, q_heads=8,
                        decode_tokens=20, seed=5),
    "fifo_evict": dict(heads=2, head_dim=16, t=160, chunk=32, theta=10000.0,
                       layer_kw=dict(rank=8, coord_budget=48, recent_window=8, absorb_block=4,
                                     n_sink=4, retention="fifo"),
                       stream_kw=dict(signal_rank=6, n_needles=0), n_queries=1, q_heads=4,
                       decode_tokens=7, seed=7),
    "surprise_evict": dict(heads=2, head_dim=16, t=160, chunk=32, theta=10000.0,
                           layer_kw=dict(rank=6, coord_budget=40, recent_window=8, absorb_block=4,
                                         n_sink=4, retention="lowrank_surprise", hh_budget=4,
                                         hh_select="surprise", hh_neighbor=1),
                           stream_kw=dict(signal_rank=6, n_needles=4), n_queries=1, q_heads=4,
                           decode_tokens=7, seed=9),
    # bf16 verbatim tiers (the model workloads' dtype), at the bench geometry:
    # 8 KV heads x 64, chunk 512, r=32, h=256, ring 128, absorb 16
    "cfg2_bf16": dict(heads=8, head_dim=64, t=2048, chunk=512, theta=500000.0, dtype="bfloat16",
                      layer_kw=dict(rank=32, coord_budget=2048 + 128 + 16, recent_window=128,
                                    absorb_block=16, n_sink=4, retention="lowrank_surprise",
                                    hh_budget=256, hh_select="surprise"),
                      stream_kw=dict(n_needles=8), n_queries=3, q_heads=32, decode_tokens=24, seed=21),
    # head_dim 128 (n = 1024), warm-up seed on, ring 256, chunk 1024 (the 8B geometry)
    "cfg3_bf16": dict(heads=8, head_dim=128, t=3072, chunk=1024, theta=500000.0, dtype="bfloat16",
                      layer_kw=dict(rank=32, coord_budget=3072 + 256 + 16, recent_window=256,
                                    absorb_block=16, n_sink=4, retention="lowrank_surprise",
                                    hh_budget=256, hh_select="surprise", seed_hh_warmup=True),
                      stream_kw=dict(n_needles=8), n_queries=2, q_heads=32, decode_tokens=8, seed=31),
    # rank 128, exact tier 1024, ring 256, chunk 2048 (the whole-box configuration's cache)
    "cfg5_bf16": dict(heads=8, head_dim=128, t=4096, chunk=2048, theta=500000.0, dtype="bfloat16",
                      layer_kw=dict(rank=128, coord_budget=4096 + 256 + 16, recent_window=256,
                                    absorb_block=16, n_sink=4, retention="lowrank_surprise",
                                    hh_budget=1024, hh_select="surprise"),
                      stream_kw=dict(signal_rank=24, n_needles=8), n_queries=2, q_heads=32,
                      decode_tokens=4, seed=41),
}


def main() -> None:
    import os

    args = sys.argv[1:]
    src = (args.pop(0) if args and args[0] not in CASES and args[0] not in ("steps", "model")
           else os.environ.get("KVDLRA_REFERENCE_SRC"))
    if not src or not (Path(src) / "kvdlra").is_dir():
        sys.exit("usage: make_golden.py <reference>/src [case ...]  (or set KVDLRA_REFERENCE_SRC)")
    sys.path.insert(0, src)
    import torch

    torch.set_num_threads(1)
    names = args or ["steps", *CASES]
    if "steps" in names:
        np.savez_compressed(HERE / "steps.npz", **case_steps())
    if "model" in names or not args:
        np.savez_compressed(HERE / "model_llama_tiny.npz", **case_model())
    for name in names:
        if name in CASES:
            np.savez_compressed(HERE / f"{name}.npz", **_run_case(name, **CASES[name]))


if __name__ == "__main__":
    main()
