"""Benchmark: BUG ingest tokens/s + factored-decode tokens/s on B200.

Workload (default, the Llama-3.2-1B configuration): the KV stream of a
16-layer model with 8 KV heads x head_dim 64 (n = 512), bf16, one sequence of
8192 tokens ingested in chunks of 512 through ``BugStreamingCache`` (rank 32,
exact tier 256, 4 sinks, ring 128, absorb block 16, prefill sub-blocks 128,
``retention="lowrank_surprise"``, surprise-selected tier, coordinate budget
T + ring + absorb so nothing is evicted), then 256 decode tokens with 32
query heads answered by the factored decode kernel.  Keys/values are seeded
synthetic low-rank-plus-noise streams with planted needles (one per layer);
inputs (268 MB of K/V) exceed L2, so no flush is needed between steps.

One step = reset + the whole ingest + the whole decode.  ``value`` is ingest
tokens/s over all ranks (each rank streams its own sequence: weak scaling, no
collective on the data path); decode tokens/s is reported beside it.

``--impl reference`` times the reference's own CPU implementation (kvdlra's
``BugStreamingLayer`` on CPU PyTorch, installed unmodified in
``baseline/_ref`` by ``baseline/install_ref.py``) on the host cores, each step
one full-length layer of the same workload scaled by the layer count; without
that install it times the oracle port (numpy restatement) instead.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

WORKLOADS = {
    # the Llama-3.2-1B configuration's cache (the default line)
    "llama-3.2-1b-kv": dict(
        name="llama-3.2-1b-kv", layers=16, kv_heads=8, head_dim=64, q_heads=32, tokens=8192,
        chunk=512, rank=32, hh=256, sinks=4, ring=128, absorb=16, prefill_block=128, decode=256,
        theta=500000.0, batch=1, seed_warmup=False, needles=dict(n_needles=16)),
    # the Llama-3.1-8B configuration's cache: head_dim 128, the warm-up seed,
    # a 32-token span copied verbatim to 4 places (exact-tier capture reported)
    "llama-3.1-8b-kv": dict(
        name="llama-3.1-8b-kv", layers=32, kv_heads=8, head_dim=128, q_heads=32, tokens=32768,
        chunk=1024, rank=32, hh=256, sinks=4, ring=256, absorb=16, prefill_block=128, decode=128,
        theta=500000.0, batch=1, seed_warmup=True, needles=dict(span_copies=(4, 32))),
    # the whole-box configuration's cache: rank 128, exact tier 1024, several
    # independent sequences per GPU; run at a reduced length (``tokens``),
    # the configuration's own length is ``config_tokens``
    "whole-box-kv": dict(
        name="whole-box-kv", layers=32, kv_heads=8, head_dim=128, q_heads=32, tokens=4096,
        config_tokens=131072, chunk=2048, rank=128, hh=1024, sinks=4, ring=256, absorb=16,
        prefill_block=128, decode=64, theta=500000.0, batch=8, seed_warmup=False,
        needles=dict(n_needles=16)),
    # the whole-box configuration's single sequence with its 8 KV heads split
    # over the GPUs, run at a reduced length
    "head-sharded-kv": dict(
        name="head-sharded-kv", layers=32, kv_heads=8, head_dim=128, q_heads=32, tokens=8192,
        config_tokens=131072, chunk=2048, rank=128, hh=1024, sinks=4, ring=256, absorb=16,
        prefill_block=128, decode=64, theta=500000.0, batch=1, seed_warmup=False,
        needles=dict(n_needles=16)),
}
WORKLOAD = WORKLOADS["llama-3.2-1b-kv"]
METRIC = "BUG ingest tokens/s + factored-decode tokens/s at 1/2/4/8 B200; % HBM roofline"


def _peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle sampling while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc: subprocess.Popen | None = None
        self.lines: list[str] = []

    def __enter__(self) -> "ClockSampler":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc: object) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[3:7]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_inputs(w: dict, seed: int, device, torch):
    """Per-(layer, sequence) synthetic streams -- post-RoPE keys and values of
    ``tokens + decode`` positions -- as bf16 device tensors ``(L, B, H, T', D)``,
    the decode queries ``(decode, L, B, Hq, D)`` and the planted needle
    positions ``[layer][sequence]``.  Each stream is built on the host
    (numpy, seeded) and moved to the device at once, so host memory holds one
    stream at a time."""
    from kvdlra_b200.synthetic import lowrank_stream

    L, B, H, D = w["layers"], w["batch"], w["kv_heads"], w["head_dim"]
    T, dec = w["tokens"], w["decode"]
    bf = torch.bfloat16
    K = torch.empty((L, B, H, T + dec, D), dtype=bf, device=device)
    V = torch.empty_like(K)
    needles = []
    for layer in range(L):
        row = []
        for b in range(B):
            s = lowrank_stream(H, D, T + dec, theta=w["theta"], seed=1000 * (seed * B + b) + layer,
                               **w["needles"])
            K[layer, b] = torch.from_numpy(s.k_post).to(device, bf)
            V[layer, b] = torch.from_numpy(s.v).to(device, bf)
            row.append(s.needles)
        needles.append(row)
    g = torch.Generator(device="cpu").manual_seed(7 + seed)
    Q = (torch.randn((dec, L, B, w["q_heads"], D), generator=g) / math.sqrt(D)).to(device, bf)
    return K, V, Q, needles


def new_cache(w: dict, torch):
    from kvdlra_b200 import BugStreamingCache, RopeAngles
    from kvdlra_b200.synthetic import default_inv_freq

    rope = RopeAngles(inv_freq=torch.from_numpy(default_inv_freq(w["head_dim"], w["theta"])))
    return BugStreamingCache(
        None, num_layers=w["layers"], rope=rope, rank=w["rank"],
        coord_budget=w["tokens"] + w["ring"] + w["absorb"], recent_window=w["ring"],
        absorb_block=w["absorb"], n_sink=w["sinks"], prefill_block_size=w["prefill_block"],
        retention="lowrank_surprise", hh_budget=w["hh"], hh_select="surprise",
        seed_hh_warmup=w["seed_warmup"])


# DRAM bytes (read + write) of one launch, from an ncu capture of the same
# launch shape (the steady-state absorb step: n = 512, r = 32, 16 columns);
# kernels not captured at the workload's shape are left out.
DRAM_BYTES_PER_LAUNCH = {"llama-3.2-1b-kv": {"bug_step_kernel": 3.39e6}}


def kernel_bytes(w: dict) -> dict[str, float]:
    """Algorithmic HBM bytes of one bench step, per kernel, from a replay of
    the cache's absorb schedule (every length decision is count-driven).

    Per launch, with P = layers x sequences problems, n = H*D, bf16 tiers
    (2 B), fp32 state:
      bug_step      2 streams x P x (read U n*r*4 + block b*n*4 + write U' n*r*4
                    + coords b*r*4)
      slash_score   P x (read candidates m*n*2 + basis n*r*4 + scores m*4)
      slash_keep    P x (read kept K,V rows 2*h*n*2 + write tier 2*h*n*2)
      carry         2 x P x W*r*4*2 (read + write the coordinates)
      mid_hat       P x (read C_k, C_v 2*W*r*4 + write K, V 2*W*n*2)
      decode_mid    P x (C_k, C_v 2*W*r*4 + positions W*4 + U_k, U_v 2*n*r*4 + q/out)
      decode_mma    P x (verbatim tiers 2*n*(hh+ring+sinks)*2 + q/out)   (with the merge)
    """
    P = w["layers"] * w["batch"]
    H, D, r = w["kv_heads"], w["head_dim"], w["rank"]
    n, T, C = H * D, w["tokens"], w["chunk"]
    sinks, ring, b, h, pbs = w["sinks"], w["ring"], w["absorb"], w["hh"], w["prefill_block"]
    out = {k: 0.0 for k in ("bug_step_kernel", "slash_score_kernel", "slash_keep_kernel",
                            "carry_kernel", "mid_hat_kernel", "decode_mid_kernel",
                            "decode_mma_kernel")}
    rk, W, hh, rl = 0, 0, 0, 0

    def bug(bb: int) -> None:
        nonlocal rk, W
        out["bug_step_kernel"] += 2 * P * (2 * n * r * 4 + bb * n * 4 + bb * r * 4)
        if W > 0:
            out["carry_kernel"] += 2 * P * W * r * 4 * 2
        rk = min(r, rk + bb)
        W += bb

    def slash(gb: int) -> None:
        nonlocal hh
        m = hh + gb
        keep = min(h, m)
        out["slash_score_kernel"] += P * (m * n * 2 + n * r * 4 + m * 4)
        out["slash_keep_kernel"] += P * (2 * keep * n * 2 + 2 * keep * n * 2)
        hh = keep
        if m - keep:
            bug(m - keep)

    # first chunk: sinks, ring, the middle in prefill sub-blocks (through the
    # exact-tier selection with the warm-up seed)
    mid = C - sinks - ring
    for s0 in range(0, mid, pbs):
        (slash if w["seed_warmup"] else bug)(min(pbs, mid - s0))
    rl = ring
    for _ in range(C, T, C):
        rl += C
        out["mid_hat_kernel"] += P * (2 * W * r * 4 + 2 * W * n * 2)
        while rl >= ring + b:
            rl -= b
            slash(b)
    for _ in range(w["decode"]):
        rl += 1
        while rl >= ring + b:
            rl -= b
            slash(b)
        exact = hh + rl + sinks
        out["decode_mid_kernel"] += P * (2 * W * r * 4 + W * 4 + 2 * n * r * 4 + 2 * w["q_heads"] * D)
        out["decode_mma_kernel"] += P * (2 * n * exact * 2 + 2 * w["q_heads"] * D)
    return out


def run_ours(args, w: dict) -> None:
    import torch
    import torch.distributed as dist

    from kvdlra_b200.sharding import init_ranks, max_over_ranks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        init_ranks("nccl", dev, timeout_s=600)
    from kvdlra_b200 import _native as N

    # each rank streams its own sequences (seeded by rank): data-parallel, no
    # collective on the data path
    K, V, Q, needles = make_inputs(w, rank, dev, torch)
    T, C, dec, B = w["tokens"], w["chunk"], w["decode"], w["batch"]
    cache = new_cache(w, torch)

    def step(Kd, Vd, Qd, ev=None, host=None):
        cache.reset()
        if ev:
            ev[0].record()
        if host is not None:
            # each chunk sits contiguous in pinned host memory and is copied on a
            # copy stream into one of two device buffers while the previous
            # chunk is ingested; the ingest waits for its copy, the copy into a
            # buffer waits for the ingest that last read it
            cur = torch.cuda.current_stream(dev)
            cs, bufs = host["stream"], host["bufs"]
            ready, done = [None, None], [None, None]

            def issue(ci):
                slot = ci % 2
                with torch.cuda.stream(cs):
                    if ci == 0 and ev:
                        cs.wait_event(ev[0])  # the copies belong to the timed region
                    if done[slot] is not None:
                        cs.wait_event(done[slot])
                    q = host["kc"][ci].shape[3]  # (the last chunk may be shorter)
                    bufs[slot][0][:, :, :, :q].copy_(host["kc"][ci], non_blocking=True)
                    bufs[slot][1][:, :, :, :q].copy_(host["vc"][ci], non_blocking=True)
                    e = torch.cuda.Event()
                    e.record(cs)
                    ready[slot] = e

            nch = (T + C - 1) // C
            issue(0)
            for ci in range(nch):
                if ci + 1 < nch:
                    issue(ci + 1)
                slot = ci % 2
                cur.wait_event(ready[slot])
                q = host["kc"][ci].shape[3]
                cache.ingest_all(bufs[slot][0][:, :, :, :q], bufs[slot][1][:, :, :, :q], peek=True)
                e = torch.cuda.Event()
                e.record(cur)
                done[slot] = e
            # the ingest's result read back inside the window: every layer's
            # exact-tier (heavy-hitter) positions, into pinned host memory
            res = torch.stack([ly.hh_pos for ly in cache.layers])
            if "res" not in host:
                host["res"] = torch.empty(res.shape, dtype=res.dtype, pin_memory=True)
            host["res"].copy_(res, non_blocking=True)
        else:
            for c0 in range(0, T, C):
                cache.ingest_all(Kd[:, :, :, c0 : c0 + C], Vd[:, :, :, c0 : c0 + C], peek=True)
        if ev:
            ev[1].record()
        outs = []
        for j in range(dec):
            p = T + j
            if host is not None:  # (the host copies hold the decode positions only)
                kk = host["k"][:, :, :, j : j + 1].to(dev, non_blocking=True)
                vv = host["v"][:, :, :, j : j + 1].to(dev, non_blocking=True)
                qq = host["q"][j].to(dev, non_blocking=True)
            else:
                kk, vv, qq = Kd[:, :, :, p : p + 1], Vd[:, :, :, p : p + 1], Qd[j]
            o = cache.decode_all(kk, vv, qq)
            if host is not None:
                outs.append(o.to("cpu", non_blocking=True))
        if ev:
            ev[2].record()
        return outs

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step(K, V, Q)
    barrier()
    # exact-tier capture of the planted needles that left the ring (the
    # Llama-3.1-8B configuration's retrieval measure)
    graduated = cache.layers[0].cumulative_length - cache.layers[0]._recent_len()
    cap_num = cap_den = 0
    for li, ly in enumerate(cache.layers):
        g = cache._group
        sel = ly._ctr.hh_sel
        for b in range(B):
            kept = set(g.t["hh_pos"][sel, li * B + b, : ly._hh_len()].tolist())
            want = [int(x) for x in needles[li][b] if x < graduated]
            cap_num += sum(x in kept for x in want)
            cap_den += len(want)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with ClockSampler(dev.index) as clk:
        barrier()
        t_wall = time.perf_counter()
        for i in range(args.steps):
            torch.cuda.nvtx.range_push("timed_step")  # lets a profiler select the timed launches
            step(K, V, Q, ev[i])
            torch.cuda.nvtx.range_pop()
        barrier()
        t_wall = time.perf_counter() - t_wall
    ingest_ms = sum(e[0].elapsed_time(e[1]) for e in ev)
    decode_ms = sum(e[1].elapsed_time(e[2]) for e in ev)
    ingest_ms, decode_ms = max_over_ranks([ingest_ms, decode_ms], dev)

    # ---- end to end through the public API from pinned host buffers
    e2e = None
    if not args.no_e2e:
        kc = K[:, :, :, :T].cpu()
        vc = V[:, :, :, :T].cpu()
        host = {"k": K[:, :, :, T:].cpu().pin_memory(), "v": V[:, :, :, T:].cpu().pin_memory(),
                "q": Q.cpu().pin_memory()}
        host["kc"] = [kc[:, :, :, c0 : c0 + C].contiguous().pin_memory() for c0 in range(0, T, C)]
        host["vc"] = [vc[:, :, :, c0 : c0 + C].contiguous().pin_memory() for c0 in range(0, T, C)]
        del kc, vc
        host["stream"] = torch.cuda.Stream(dev)
        host["bufs"] = [(torch.empty_like(host["kc"][0], device=dev), torch.empty_like(host["vc"][0], device=dev))
                        for _ in range(2)]
        step(None, None, None, host=host)
        barrier()
        ev2 = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
        for i in range(args.steps):
            step(None, None, None, ev2[i], host=host)
        barrier()
        (e_ing,) = max_over_ranks([sum(e[0].elapsed_time(e[1]) for e in ev2)], dev)
        h2d = sum(t.numel() * t.element_size() for t in host["kc"] + host["vc"])  # the window's copies
        d2h = host["res"].numel() * host["res"].element_size()
        e2e = {"value": world * B * T * args.steps / (e_ing / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)}
        del host

    # ---- per-kernel event timing over one more step (profiling pass)
    N.profile(True)
    step(K, V, Q)
    torch.cuda.synchronize(dev)
    prof = N.profile_read()
    N.profile(False)
    launches_total = sum(v[1] for v in prof.values())

    if rank == 0:
        peaks, peak_kind = _peaks()
        dom = max(prof.items(), key=lambda kv: kv[1][0])[0] if prof else None
        kb = kernel_bytes(w)
        peak = peaks["hbm_gbs"]
        traffic = DRAM_BYTES_PER_LAUNCH.get(w["name"], {})

        def roof(name: str) -> dict:
            ms, launches = prof.get(name, (0.0, 0))
            if name == "decode_mma_kernel":  # verbatim tiles + the merge of all partials: one op
                ms += prof.get("decode_merge_kernel", (0.0, 0))[0]
            nbytes = kb.get(name)
            ach = nbytes / (ms / 1e3) / 1e9 if (nbytes and ms) else None
            return {"kernel": name, "bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                    "frac": (ach / peak) if ach else None, "peak_source": peak_kind,
                    "traffic": traffic.get(name),
                    "bytes_per_launch": (nbytes / launches) if (nbytes and launches) else None,
                    "avg_launch_ms": (ms / launches) if launches else None}

        roof_all = {k: roof(k) for k in kb if k in prof}
        roof_dom = roof_all.get(dom) or roof("decode_mid_kernel")
        total_ms = sum(x[0] for x in prof.values()) or 1e-9
        kernels = {k: {"total_ms": round(v[0], 4), "launches": v[1], "share": round(v[0] / total_ms, 4)}
                   for k, v in sorted(prof.items(), key=lambda kv: -kv[1][0])}
        cpu = None if args.no_cpu_baseline else cpu_baseline(w)
        result = {
            "metric": METRIC,
            "value": world * B * T * args.steps / (ingest_ms / 1e3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": (ingest_ms + decode_ms) / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded low-rank+noise KV streams with needles; inputs > L2)",
            "config": bench_config(w, world),
            "decode": {"value": world * B * dec * args.steps / (decode_ms / 1e3), "unit": "tokens/s"},
            "ingest_ms_per_step": ingest_ms / args.steps,
            "decode_ms_per_step": decode_ms / args.steps,
            "needle_capture": (cap_num / cap_den) if cap_den else None,
            "e2e": e2e,
            "gpu_launches": int(launches_total * args.steps),
            "roofline": roof_dom,
            "roofline_all": roof_all,
            "dominant_kernel": dom,
            "kernels": kernels,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            "wall_s": t_wall,
        }
        print(json.dumps(result))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


REF_DIR = REPO / "baseline" / "_ref"


def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def _reference_layer(w: dict):
    """The reference's own ``BugStreamingLayer`` (kvdlra, installed unmodified
    in ``baseline/_ref``), configured as the workload's layers, with the
    model's rotary module (transformers' Llama rotary at the workload's
    head_dim and RoPE theta)."""
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    from kvdlra.cache.bug_cache import BugStreamingLayer, _RopeAngles
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    H, D = w["kv_heads"], w["head_dim"]
    rot = LlamaRotaryEmbedding(LlamaConfig(
        hidden_size=w["q_heads"] * D, num_attention_heads=w["q_heads"], num_key_value_heads=H,
        head_dim=D, rope_theta=w["theta"], max_position_embeddings=1 << 18))
    return BugStreamingLayer(
        rope=_RopeAngles(rot), rank=w["rank"], coord_budget=w["tokens"] + w["ring"] + w["absorb"],
        recent_window=w["ring"], absorb_block=w["absorb"], n_sink=w["sinks"],
        prefill_block_size=w["prefill_block"], retention="lowrank_surprise", hh_budget=w["hh"],
        hh_select="surprise", seed_hh_warmup=w.get("seed_warmup", False))


def cpu_reference(w: dict, sample_tokens: int, sample_decode: int) -> dict:
    """Time the reference's own CPU implementation of the path (PyTorch on the
    host cores, every thread): one layer of the workload ingests
    ``sample_tokens`` tokens in the workload's chunks (update in ingest mode +
    consolidate, bug_cache.py:1404-1429), then ``sample_decode`` decode steps
    (update + peek, bug_cache.py:1483-1519) each followed by the GQA attention
    HF runs over the returned peek (SDPA).  Every layer of the model does the
    same work per token, so model tokens/s = layer tokens/s / layers."""
    import torch

    from kvdlra_b200.synthetic import lowrank_stream

    threads = _host_threads()
    torch.set_num_threads(threads)
    H, D = w["kv_heads"], w["head_dim"]
    s = lowrank_stream(H, D, sample_tokens + sample_decode, n_needles=16, theta=w["theta"], seed=0)
    bf = torch.bfloat16
    k = torch.from_numpy(s.k_post)[None].to(bf)
    v = torch.from_numpy(s.v)[None].to(bf)
    q = (torch.randn(sample_decode, 1, w["q_heads"], 1, D, generator=torch.Generator().manual_seed(0))
         / math.sqrt(D)).to(bf)
    layer = _reference_layer(w)
    with torch.no_grad():
        layer._mode = "ingest"  # what BugStreamingCache.ingesting() sets (bug_cache.py:1884-1895)
        t0 = time.perf_counter()
        for c0 in range(0, sample_tokens, w["chunk"]):
            c1 = min(sample_tokens, c0 + w["chunk"])
            layer.update(k[:, :, c0:c1], v[:, :, c0:c1])
            layer.consolidate()
        t_ing = time.perf_counter() - t0
        layer._mode = "normal"
        t0 = time.perf_counter()
        for j in range(sample_decode):
            p = sample_tokens + j
            kr, vr = layer.update(k[:, :, p : p + 1], v[:, :, p : p + 1])
            torch.nn.functional.scaled_dot_product_attention(q[j], kr, vr, enable_gqa=True)
        t_dec = time.perf_counter() - t0
    L = w["layers"]
    return {"value": sample_tokens / t_ing / L, "unit": "tokens/s", "cores": threads,
            "kind": "reference", "decode_tokens_per_s": sample_decode / t_dec / L,
            "sample": (f"kvdlra BugStreamingLayer (the reference, CPU PyTorch, {threads} threads): "
                       f"1 of {L} layers, {sample_tokens} ingested tokens in chunks of {w['chunk']} "
                       f"+ {sample_decode} decode steps with SDPA over the peek, scaled by the layer count")}


def cpu_port(w: dict, sample_tokens: int = 2048, sample_decode: int = 16) -> dict:
    """The oracle port (numpy restatement of the reference path) on one layer,
    scaled by the layer count: the fallback when the reference itself is not
    installed, and a labelled second line beside it."""
    from oracle.bug_oracle import OracleLayer, RopeSpec, default_inv_freq, gqa_attention
    from kvdlra_b200.synthetic import lowrank_stream

    H, D = w["kv_heads"], w["head_dim"]
    s = lowrank_stream(H, D, sample_tokens + sample_decode, n_needles=4, theta=w["theta"], seed=0)
    lay = OracleLayer(RopeSpec(default_inv_freq(D, w["theta"])), H, D, rank=w["rank"],
                      coord_budget=w["tokens"] + w["ring"] + w["absorb"], recent_window=w["ring"],
                      absorb_block=w["absorb"], n_sink=w["sinks"],
                      prefill_block_size=w["prefill_block"], retention="lowrank_surprise",
                      hh_budget=w["hh"], hh_select="surprise", dtype="bfloat16",
                      seed_hh_warmup=w.get("seed_warmup", False))

    def mat(x):
        return x.transpose(0, 2, 1).reshape(H * D, -1)

    lay.mode = "ingest"
    t0 = time.perf_counter()
    for c0 in range(0, sample_tokens, w["chunk"]):
        lay.update(mat(s.k_post[:, c0 : c0 + w["chunk"]]), mat(s.v[:, c0 : c0 + w["chunk"]]))
        lay.consolidate()
    t_ing = time.perf_counter() - t0
    lay.mode = "normal"
    rng = np.random.default_rng(0)
    t0 = time.perf_counter()
    for j in range(sample_decode):
        p = sample_tokens + j
        kr, vr = lay.update(mat(s.k_post[:, p : p + 1]), mat(s.v[:, p : p + 1]))
        gqa_attention(rng.standard_normal((w["q_heads"], D)).astype(np.float32), lay.to_hf(kr), lay.to_hf(vr))
    t_dec = time.perf_counter() - t0
    try:
        from threadpoolctl import threadpool_info

        cores = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:  # noqa: BLE001
        cores = os.cpu_count() or 1
    return {"value": sample_tokens / t_ing / w["layers"], "unit": "tokens/s", "cores": int(cores),
            "kind": "port", "decode_tokens_per_s": sample_decode / t_dec / w["layers"],
            "sample": (f"oracle port (numpy): 1 of {w['layers']} layers, {sample_tokens} ingested tokens "
                       f"(chunk {w['chunk']}) + {sample_decode} decode steps, scaled by the layer count")}


def cpu_baseline(w: dict) -> dict:
    """The CPU baseline beside our arm's line: the reference itself when it is
    installed (one full-length layer of the workload), else the oracle port."""
    if (REF_DIR / "kvdlra").is_dir():
        return cpu_reference(w, w["tokens"], 32)
    return cpu_port(w)


def bench_config(w: dict, world: int) -> dict:
    """The ``config`` object both arms print (identical for the same workload)."""
    return {"workload": w["name"], "layers": w["layers"], "kv_heads": w["kv_heads"],
            "head_dim": w["head_dim"], "q_heads": w["q_heads"], "tokens": w["tokens"],
            "chunk": w["chunk"], "rank": w["rank"], "hh_budget": w["hh"], "sinks": w["sinks"],
            "ring": w["ring"], "absorb_block": w["absorb"], "decode_tokens": w["decode"],
            "seed_warmup": bool(w.get("seed_warmup", False)),
            "config_tokens": w.get("config_tokens", w["tokens"]),
            "sequences_per_gpu": w.get("batch", 1),
            "parallelism": f"dp{world} (independent sequences)", "l2": "inputs larger than L2"}


def run_reference(args, w: dict) -> None:
    """The reference arm: the reference's own CPU implementation on the host
    cores (rank 0 only), each step one full-length layer of the workload."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    have_ref = (REF_DIR / "kvdlra").is_dir()
    for _ in range(args.warmup):
        if have_ref:
            cpu_reference(w, min(1024, w["tokens"]), 4)
        else:
            cpu_port(w, 512, 4)
    vals, decs, t_tot = [], [], time.perf_counter()
    for _ in range(args.steps):
        cb = cpu_reference(w, w["tokens"], 32) if have_ref else cpu_port(w)
        vals.append(cb["value"])
        decs.append(cb["decode_tokens_per_s"])
    t_tot = time.perf_counter() - t_tot
    v = float(np.mean(vals))
    port = cpu_port(w) if have_ref else None
    out = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * t_tot / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (tiers), f32 (BUG math)", "data": "synthetic",
        "config": bench_config(w, world),
        "decode": {"value": float(np.mean(decs)), "unit": "tokens/s"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cb["cores"], "kind": cb["kind"],
                         "sample": cb["sample"]},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if port is not None:
        out["oracle_port"] = {"value": port["value"], "decode_tokens_per_s": port["decode_tokens_per_s"],
                              "cores": port["cores"], "sample": port["sample"]}
    print(json.dumps(out))


# ------------------------------------------------------------ decode sweep

SWEEP = dict(batch=(1, 8, 32, 64), rank=(32, 128, 192), hh=(256, 1024), context=(16384, 65536, 131072))


def decode_state(cache, B: int, W: int, H: int, D: int, r: int, h: int, ring: int, sinks: int,
                 torch, seed: int = 0) -> None:
    """Fill a one-layer cache of ``B`` sequences with the factored-decode
    microbenchmark's state: bases U_k, U_v orthonormal (QR of N(0,1)),
    coordinates C = diag(2^(-i/8)) V^T with V orthonormal (QR of a W x r
    N(0,1) draw), exact tier / ring / sinks N(0,1) bf16, middle positions the
    sorted values of [4, W + h + 4) the tier's random positions leave."""
    ly = cache.layers[0]
    dev = torch.device("cuda")
    n = H * D
    kd = torch.zeros((B, H, 1, D), dtype=torch.bfloat16, device=dev)
    ly.lazy_initialization(kd, kd)
    g = cache._group
    g.ensure([ly], ring, W + g.max_block + 1)
    gen = torch.Generator(device=dev).manual_seed(seed)
    t = g.t
    bf = torch.bfloat16
    for name in ("sink_k", "sink_v"):
        t[name][:, :sinks] = torch.randn((B, sinks, n), generator=gen, device=dev).to(bf)
    for name in ("ring_k", "ring_v"):
        t[name][:, :ring] = torch.randn((B, ring, n), generator=gen, device=dev).to(bf)
    for name in ("hh_k", "hh_v"):
        t[name][0, :, :h] = torch.randn((B, h, n), generator=gen, device=dev).to(bf)
    scale = torch.pow(2.0, -torch.arange(r, device=dev, dtype=torch.float32) / 8)
    for b in range(B):
        for name in ("u_k", "u_v"):
            t[name][0, b, :, :r] = torch.linalg.qr(torch.randn((n, r), generator=gen, device=dev))[0]
        for name in ("c_k", "c_v"):
            vq = torch.linalg.qr(torch.randn((W, r), generator=gen, device=dev))[0]
            t[name][b, :W, :r] = vq * scale
        perm = torch.randperm(W + h, generator=gen, device=dev) + sinks
        t["hh_pos"][0, b, :h] = torch.sort(perm[:h])[0].to(torch.int32)
        t["mid_pos"][b, :W] = torch.sort(perm[h:])[0].to(torch.int32)
    t["sig_k"][:, :r] = 1.0
    t["sig_v"][:, :r] = 1.0
    t["r_k"][:] = r
    t["r_v"][:] = r
    c = ly._ctr
    c.cumulative_length, c.sink_len, c.ring_head, c.ring_len = sinks + h + W + ring, sinks, 0, ring
    c.hh_len, c.hh_sel, c.u_sel, c.w_len, c.seeded, c.n_absorbs = h, 0, 0, W, 1, 1
    ly._started = True
    ly._r_cache = None
    torch.cuda.synchronize()


def run_decode_sweep(args) -> None:
    """The factored-decode microbenchmark (32 query heads over 8 KV heads,
    head_dim 128, ring 128, 4 sinks): every (batch, rank, exact tier,
    compressed context) point, one decode step per call, CUDA-event time of
    ``steps`` calls after ``warmup``; algorithmic bytes and FLOPs per step
    give GB/s against the HBM roofline and the binding roofline
    ``max(bytes / BW, flops / peak)``."""
    import torch

    from kvdlra_b200 import BugStreamingCache, RopeAngles
    from kvdlra_b200.synthetic import default_inv_freq

    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    H, D, Hq, ring, sinks = 8, 128, 32, 128, 4
    n = H * D
    peaks, peak_kind = _peaks()
    bw, fl = peaks["hbm_gbs"] * 1e9, peaks["bf16_tflops"] * 1e12
    inv = torch.from_numpy(default_inv_freq(D, 500000.0))
    pts = []
    grid = [(B, r, h, W) for B in SWEEP["batch"] for r in SWEEP["rank"] for h in SWEEP["hh"]
            for W in SWEEP["context"]]
    if args.sweep_points:
        grid = grid[: args.sweep_points]
    with ClockSampler(dev.index) as clk:
        for B, r, h, W in grid:
            if B * W * r * 8 > 40e9:  # fp32 C_k + C_v beyond 40 GB: skipped, reported
                pts.append({"batch": B, "rank": r, "hh": h, "context": W, "skipped": "memory"})
                continue
            cache = BugStreamingCache(None, num_layers=1, rope=RopeAngles(inv_freq=inv), rank=r,
                                      coord_budget=W + 64, recent_window=ring, absorb_block=16,
                                      n_sink=sinks, retention="lowrank_surprise", hh_budget=h,
                                      hh_select="surprise")
            decode_state(cache, B, W, H, D, r, h, ring, sinks, torch, seed=B * 7 + r + h + W)
            q = (torch.randn((B, Hq, D), device=dev) / math.sqrt(D)).to(torch.bfloat16)
            ly = cache.layers[0]
            for _ in range(args.warmup):
                ly.factored_attention(q)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                ly.factored_attention(q)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            nbytes = B * (8 * r * W + 4 * W + 8 * n * r + 4 * n * (h + ring + sinks) + 4 * Hq * D)
            flops = B * (2 * r * W * (n + Hq) + 4 * Hq * D * (W + h + ring + sinks))
            t_bound = max(nbytes / bw, flops / fl)
            pts.append({"batch": B, "rank": r, "hh": h, "context": W, "ms": ms,
                        "tokens_per_s": B / (ms / 1e3), "gb_s": nbytes / (ms / 1e3) / 1e9,
                        "hbm_frac": nbytes / (ms / 1e3) / bw,
                        "bound": "hbm" if nbytes / bw >= flops / fl else "tensor",
                        "roofline_frac": t_bound / (ms / 1e3)})
            del cache
            torch.cuda.empty_cache()
    head = next((p for p in pts if p.get("batch") == 64 and p.get("rank") == 32 and p.get("hh") == 256
                 and p.get("context") == 131072 and "ms" in p), next((p for p in pts if "ms" in p), {}))
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": head.get("tokens_per_s"), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head.get("ms"),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (orthonormal factors, N(0,1) tiers; inputs > L2 at every point)",
            "config": {"workload": "decode-sweep", "q_heads": Hq, "kv_heads": H, "head_dim": D,
                       "ring": ring, "sinks": sinks, "headline_point": {k: head.get(k) for k in ("batch", "rank", "hh", "context")},
                       "coordinates": "fp32", "l2": "inputs larger than L2"},
            "roofline": {"bound": head.get("bound"), "achieved": head.get("gb_s"), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": head.get("hbm_frac"), "binding_frac": head.get("roofline_frac"),
                         "peak_source": peak_kind, "traffic": None},
            "sweep": pts, "gpu_launches": None, "clocks": clk.summary()}))


def run_reference_decode(args) -> None:
    """The reference's decode step at the sweep's smallest point (one
    sequence, rank 32, exact tier 256, 16K compressed tokens) on the host
    cores: the dense peek ``[sinks | tier | middle | ring]`` concatenated as
    ``_decode_peek`` does (bug_cache.py:1496-1519, the middle already
    materialised) and SDPA over it with GQA, as HF runs it.  The middle's
    re-materialisation after each absorb (every 16 steps) is not counted."""
    import torch

    if int(os.environ.get("RANK", "0")) != 0:
        return
    threads = _host_threads()
    torch.set_num_threads(threads)
    H, D, Hq, ring, sinks, h, W = 8, 128, 32, 128, 4, 256, 16384
    bf = torch.bfloat16
    g = torch.Generator().manual_seed(0)
    parts_k = [torch.randn((1, H, x, D), generator=g).to(bf) for x in (sinks, h, W, ring)]
    parts_v = [torch.randn((1, H, x, D), generator=g).to(bf) for x in (sinks, h, W, ring)]
    q = (torch.randn((1, Hq, 1, D), generator=g) / math.sqrt(D)).to(bf)

    def one():
        k = torch.cat(parts_k, dim=2)
        v = torch.cat(parts_v, dim=2)
        return torch.nn.functional.scaled_dot_product_attention(q, k, v, enable_gqa=True)

    for _ in range(args.warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    ms = 1e3 * (time.perf_counter() - t0) / args.steps
    v = 1e3 / ms
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "decode-sweep", "batch": 1, "rank": 32, "hh": h, "context": W},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "sample": "dense peek concatenation + SDPA (CPU torch), batch 1, rank 32, tier 256, 16K middle"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def run_head_sharded(args, w: dict) -> None:
    """One sequence with its KV heads split over the ranks (the whole-box
    configuration's single-sequence mode).  The basis is joint over heads, so
    every rank ingests the whole sequence into the whole cache (the same
    kernels on the same inputs: identical caches); each rank answers the
    decode attention of its own KV heads' query heads
    (``kvd_factored_decode_heads``) and the per-head outputs of every layer
    are all-gathered over NCCL, as before each layer's ``o_proj``.  ``value``
    is the sequence's decode tokens/s (strong scaling: the work is fixed as
    N grows); ingest tokens/s (replicated work) beside it."""
    import torch
    import torch.distributed as dist

    from kvdlra_b200 import _native as N
    from kvdlra_b200.sharding import init_ranks, max_over_ranks, shard_heads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if world > 1:
        init_ranks("nccl", dev, timeout_s=600)
    K, V, Q, _ = make_inputs(w, 0, dev, torch)  # one sequence, the same on every rank
    T, C, dec, L, B, D = w["tokens"], w["chunk"], w["decode"], w["layers"], w["batch"], w["head_dim"]
    H, G = w["kv_heads"], w["q_heads"] // w["kv_heads"]
    h0, hc = shard_heads(H, world, rank)
    Ql = Q[:, :, :, h0 * G : (h0 + hc) * G].contiguous()  # this rank's query heads
    del Q
    cache = new_cache(w, torch)
    gbuf = torch.empty((L, world, B, hc * G, D), dtype=torch.bfloat16, device=dev)

    def step(ev=None):
        cache.reset()
        if ev:
            ev[0].record()
        for c0 in range(0, T, C):
            cache.ingest_all(K[:, :, :, c0 : c0 + C], V[:, :, :, c0 : c0 + C], peek=True)
        if ev:
            ev[1].record()
        for j in range(dec):
            p = T + j
            o = cache.decode_all(K[:, :, :, p : p + 1], V[:, :, :, p : p + 1], Ql[j], heads=(h0, hc))
            if world > 1:
                for li in range(L):  # each layer's heads gathered before its o_proj
                    dist.all_gather_into_tensor(gbuf[li], o[li])
        if ev:
            ev[2].record()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with ClockSampler(dev.index) as clk:
        barrier()
        for i in range(args.steps):
            step(ev[i])
        barrier()
    ingest_ms = sum(e[0].elapsed_time(e[1]) for e in ev)
    decode_ms = sum(e[1].elapsed_time(e[2]) for e in ev)
    ingest_ms, decode_ms = max_over_ranks([ingest_ms, decode_ms], dev)
    N.profile(True)
    step()
    torch.cuda.synchronize(dev)
    prof = N.profile_read()
    N.profile(False)
    if rank == 0:
        total_ms = sum(x[0] for x in prof.values()) or 1e-9
        cfg = bench_config(w, world)
        cfg["parallelism"] = f"KV heads {hc} per GPU over {world} GPU(s); whole cache on every GPU"
        cfg["sequences_per_gpu"] = None
        print(json.dumps({
            "metric": "factored-decode tokens/s of one sequence, KV heads sharded over N B200",
            "value": B * dec * args.steps / (decode_ms / 1e3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": (ingest_ms + decode_ms) / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded low-rank+noise KV stream with needles; inputs > L2)",
            "config": cfg,
            "ingest": {"value": B * T * args.steps / (ingest_ms / 1e3), "unit": "tokens/s",
                       "note": "replicated on every GPU"},
            "decode_ms_per_step": decode_ms / args.steps,
            "ingest_ms_per_step": ingest_ms / args.steps,
            "gpu_launches": int(sum(v[1] for v in prof.values()) * args.steps),
            "kernels": {k: {"total_ms": round(v[0], 4), "launches": v[1], "share": round(v[0] / total_ms, 4)}
                        for k, v in sorted(prof.items(), key=lambda kv: -kv[1][0])},
            "clocks": clk.summary(),
        }))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_chunk_attention(args) -> None:
    """Chunk attention at the Llama-3.2-1B cache shape (16 layers, 8 KV heads x
    64, 32 query heads, bf16, r=32, h=256): the cache ingests ``tokens - 512``
    tokens, then every layer takes a 512-token chunk (appended to its ring)
    and answers its 512 x 32 queries (a) with the factored chunk kernel and (b)
    with the reference's dataflow: the dense retained cache re-materialised
    (``_decode_peek``) and SDPA under the bottom-right causal mask.  CUDA-event
    time of ``steps`` repetitions after ``warmup``; chunk tokens/s (all 16
    layers per chunk) and the largest relative difference of the outputs."""
    import torch
    import torch.nn.functional as F

    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = dict(WORKLOADS["llama-3.2-1b-kv"])
    if args.tokens:
        w["tokens"] = args.tokens
    T, C, D, Hq = w["tokens"], w["chunk"], w["head_dim"], w["q_heads"]
    w["decode"] = 0
    K, V, _, _ = make_inputs(w, 0, dev, torch)
    cache = new_cache(w, torch)
    with cache.ingesting():
        for c0 in range(0, T - C, C):
            cache.ingest_all(K[:, :, :, c0:c0 + C], V[:, :, :, c0:c0 + C], peek=False)
    layers = cache.layers
    for li, ly in enumerate(layers):
        ly._mode = "ingest"
        ly._append(K[li, :, :, T - C:T], V[li, :, :, T - C:T])
    g = torch.Generator(device="cpu").manual_seed(11)
    q = (torch.randn((len(layers), w["batch"], Hq, C, D), generator=g) / math.sqrt(D)).to(dev, torch.bfloat16)
    sc = D ** -0.5

    def factored():
        return [ly.factored_chunk_attention(q[li], scaling=sc) for li, ly in enumerate(layers)]

    def dense():
        outs = []
        for li, ly in enumerate(layers):
            kr, vr = ly._decode_peek()
            L = kr.shape[2]
            mask = torch.arange(L, device=dev)[None, :] <= (L - C + torch.arange(C, device=dev))[:, None]
            o = F.scaled_dot_product_attention(q[li], kr, vr, attn_mask=mask, enable_gqa=True, scale=sc)
            outs.append(o.transpose(1, 2))
        return outs

    res = {}
    with ClockSampler(dev.index) as clk:
        for name, fn in (("factored", factored), ("dense_peek_sdpa", dense)):
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            res[name] = {"ms_per_chunk": ms, "tokens_per_s": C * w["batch"] / (ms / 1e3)}
    a, b = factored(), dense()
    err = max(float((x.float() - y.float()).abs().max() / y.float().abs().max()) for x, y in zip(a, b))
    print(json.dumps({
        "metric": "chunk attention tokens/s (16 layers, 512 queries x 32 heads per chunk)",
        "value": res["factored"]["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": res["factored"]["ms_per_chunk"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded low-rank+noise KV streams; random queries)",
        "config": {"workload": "chunk-attention", "layers": w["layers"], "kv_heads": w["kv_heads"],
                   "head_dim": D, "q_heads": Hq, "rank": w["rank"], "hh_budget": w["hh"],
                   "retained_tokens": T - C, "chunk": C, "sequences_per_gpu": w["batch"]},
        "dense_peek_sdpa": res["dense_peek_sdpa"], "max_rel_diff": err, "clocks": clk.summary()}))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--tokens", type=int, default=None, help="override the ingest length (testing)")
    ap.add_argument("--workload", default="llama-3.2-1b-kv",
                    choices=[*WORKLOADS, "decode-sweep", "chunk-attention"],
                    help="the configuration to run (default: the Llama-3.2-1B cache)")
    ap.add_argument("--sweep-points", type=int, default=0, help="decode-sweep: first N points only")
    ap.add_argument("--batch", type=int, default=None, help="override the sequences per GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the CPU oracle timing (profiling runs)")
    args = ap.parse_args()
    if args.workload == "chunk-attention":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "chunk-attention is a kernel comparison "
                              "line; the reference's dataflow is its dense_peek_sdpa field"}))
        else:
            run_chunk_attention(args)
        return
    if args.workload == "decode-sweep":
        if args.impl == "reference":
            run_reference_decode(args)
        else:
            run_decode_sweep(args)
        return
    w = dict(WORKLOADS[args.workload])
    if args.tokens:
        w["tokens"] = args.tokens
    if args.batch:
        w["batch"] = args.batch
    if w["name"] == "head-sharded-kv":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference runs one device; its "
                              "single-sequence CPU path is the whole-box-kv reference line"}))
        else:
            run_head_sharded(args, w)
        return
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
