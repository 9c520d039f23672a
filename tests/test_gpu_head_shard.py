"""KV-head sharding of one sequence: the factored kernels over a range of KV
heads, and a head-sharded model.

A rank of a head-sharded sequence keeps the whole cache (the basis is joint
over heads, bug_cache.py:605-607) and answers only its KV heads' query heads.
``kvd_factored_decode_heads`` / ``kvd_factored_chunk_attention_heads`` over
the ranges of a partition of the heads must concatenate to the full call's
output, and each range must equal dense attention over the cache's own peek
restricted to its heads (1e-4 fp32, 2e-2 bf16).  The partitions cover the
launch paths a narrower range takes: the tcgen05 middle tier while a range
holds a multiple of 256 features, the CUDA-core middle-tier kernel below.

At model level, two ranks (processes on one GPU exchanging over gloo through
host memory, or one GPU each over NCCL when two are present) run a bf16
random-init Llama through ``BugStreamingCache`` with the factored attention
and ``shard_attention_heads``; their logits must equal the unsharded model's
within the bf16 rule and their caches must be bit-identical.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle.bug_oracle import default_inv_freq, gqa_attention

from kvdlra_b200 import BugStreamingLayer, RopeAngles
from kvdlra_b200.synthetic import lowrank_stream

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _rel(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.abs(a.astype(np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


def _layer(H: int, D: int, T: int, rank: int, dtype, hh: int = 70):
    s = lowrank_stream(H, D, T + 300, n_needles=5, seed=H * 100 + D + rank)
    inv = default_inv_freq(D, 500000.0)
    layer = BugStreamingLayer(RopeAngles(inv_freq=torch.from_numpy(inv), attention_scaling=1.0),
                              rank=rank, coord_budget=T + 400, recent_window=96, absorb_block=16,
                              n_sink=4, retention="lowrank_surprise", hh_budget=hh, hh_select="surprise")
    layer._mode = "ingest"
    k = torch.from_numpy(s.k_post)[None].to(DEV, dtype)
    v = torch.from_numpy(s.v)[None].to(DEV, dtype)
    for st in range(0, T, 128):
        layer.update(k[:, :, st : min(T, st + 128)], v[:, :, st : min(T, st + 128)])
        layer.consolidate()
    return layer, k, v


@pytest.mark.parametrize("H,D,G,T,rank,dtype,widths", [
    (8, 64, 4, 1300, 32, torch.bfloat16, (4, 2, 1)),   # tcgen05 at 4 heads, CUDA cores at 2 and 1
    (8, 128, 4, 1300, 32, torch.bfloat16, (2, 1)),     # tcgen05 at 2 heads of 128
    (4, 64, 4, 777, 32, torch.float32, (2, 1)),
    (2, 128, 8, 1000, 32, torch.float32, (1,)),
    (4, 128, 4, 900, 64, torch.bfloat16, (2, 1)),      # rank 64: the warp-MMA middle tier
])
def test_decode_head_ranges_concatenate_to_full(H, D, G, T, rank, dtype, widths) -> None:
    layer, _, _ = _layer(H, D, T, rank, dtype)
    kr, vr = layer._decode_peek()
    kd, vd = kr[0].float().cpu().numpy(), vr[0].float().cpu().numpy()
    rng = np.random.default_rng(T + rank)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    q = torch.from_numpy(rng.standard_normal((1, H * G, D)).astype(np.float32)).to(DEV, dtype)
    full = layer.factored_attention(q)[0].float().cpu().numpy()
    for hc in widths:
        parts = []
        for h0 in range(0, H, hc):
            qs = q[:, h0 * G : (h0 + hc) * G]
            out = layer.factored_attention(qs, heads=(h0, hc))[0].float().cpu().numpy()
            ref = gqa_attention(qs[0].float().cpu().numpy(), kd[h0 : h0 + hc], vd[h0 : h0 + hc])
            assert _rel(out, ref) < tol, (hc, h0, _rel(out, ref))
            parts.append(out)
        cat = np.concatenate(parts, axis=0)
        assert _rel(cat, full) < (1e-5 if dtype == torch.float32 else 1e-2), (hc, _rel(cat, full))
    with pytest.raises(Exception, match="KV heads"):
        layer.factored_attention(q[:, : 3 * G], heads=(H - 1, 2))
    layer._group.check_status()


def _dense_causal(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> np.ndarray:
    hq, nq, _ = q.shape
    h, L, _ = k.shape
    g = hq // h
    kd, vd = k.double().repeat_interleave(g, dim=0), v.double().repeat_interleave(g, dim=0)
    s = torch.einsum("hqd,hkd->hqk", q.double(), kd) * scale
    lim = (L - nq + torch.arange(nq))[:, None]
    s = s.masked_fill((torch.arange(L)[None, :] > lim)[None], float("-inf"))
    return torch.einsum("hqk,hkd->qhd", torch.softmax(s, dim=-1), vd).numpy()


@pytest.mark.parametrize("mode", ["ingest", "score"])
def test_chunk_attention_head_ranges(mode: str) -> None:
    H, G, D, T, q_len = 8, 4, 64, 1300, 200
    layer, k, v = _layer(H, D, T, 32, torch.bfloat16)
    kc, vc = k[:, :, T : T + q_len], v[:, :, T : T + q_len]
    rng = np.random.default_rng(11)
    q = torch.from_numpy(rng.standard_normal((1, H * G, q_len, D)).astype(np.float32)).to(DEV, torch.bfloat16)
    scale = D ** -0.5
    tail = None
    if mode == "ingest":
        layer._append(kc, vc)
        kr, vr = layer._decode_peek()
    else:
        layer._mode = "score"
        tail = (kc, vc)
        kr, vr = layer._decode_peek(tail=tail)
    full = layer.factored_chunk_attention(q, scaling=scale, tail=tail)[0].float().cpu().numpy()
    for hc in (2, 1):
        parts = []
        for h0 in range(0, H, hc):
            qs = q[:, h0 * G : (h0 + hc) * G]
            out = layer.factored_chunk_attention(qs, scaling=scale, tail=tail, heads=(h0, hc))
            got = out[0].float().cpu().numpy()
            ref = _dense_causal(qs[0].float().cpu(), kr[0, h0 : h0 + hc].float().cpu(),
                                vr[0, h0 : h0 + hc].float().cpu(), scale)
            assert _rel(got, ref) < 2e-2, (hc, h0, _rel(got, ref))
            parts.append(got)
        assert _rel(np.concatenate(parts, axis=1), full) < 1e-2
    layer._group.check_status()


# ------------------------------------------------------------- model level

def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model_worker(rank: int, world: int, port: int, backend: str, q) -> None:
    import copy

    import torch.distributed as dist

    from golden.make_golden import MODEL_CASE, tiny_llama

    from kvdlra_b200 import BugStreamingCache, enable_factored_decode
    from kvdlra_b200.harness import decode_greedy, prefill_chunked
    from kvdlra_b200.sharding import init_ranks, shard_attention_heads

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dev = torch.device("cuda", rank if backend == "nccl" else 0)
    torch.cuda.set_device(dev)
    r, w = init_ranks(backend, dev if backend == "nccl" else None, timeout_s=120)
    try:
        c = MODEL_CASE
        model = enable_factored_decode(tiny_llama(c).to(dev, torch.bfloat16))
        ids = torch.randint(0, c["vocab"], (1, 640), generator=torch.Generator().manual_seed(3)).to(dev)
        forced = torch.randint(0, c["vocab"], (1, 12), generator=torch.Generator().manual_seed(4))

        def run(m):
            cache = BugStreamingCache(m, **c["cache_kw"])
            first = prefill_chunked(m, cache, ids, c["chunk"], keep_logits=True)
            _, logits = decode_greedy(m, cache, first, ids.shape[1], 12, forced=forced)
            cache.check_status()
            return torch.cat([first[:, None].float(), logits.float()], dim=1), cache

        full, _ = run(model)
        sharded = shard_attention_heads(copy.deepcopy(model), r, w)
        got, cache = run(sharded)
        err = float((got - full).abs().max() / full.abs().max())
        # the whole cache on every rank, stepped identically: a digest of its state
        vals = []
        for ly in cache.layers:
            pk, pv = ly._decode_peek()
            vals += [pk.double().sum(), pv.double().sum(), pk.double().square().sum(),
                     ly.hh_pos.double().sum()]
        digest = torch.stack(vals).to(dev if backend == "nccl" else "cpu")
        digests = [torch.empty_like(digest) for _ in range(w)]
        dist.all_gather(digests, digest)
        same = all(torch.equal(d.cpu(), digests[0].cpu()) for d in digests)
        q.put((r, err, same))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _two_ranks(backend: str) -> list[tuple[int, float, bool]]:
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_model_worker, args=(r, 2, port, backend, qu)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(qu.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return out


def test_head_sharded_llama_two_ranks_one_gpu() -> None:
    for r, err, same in _two_ranks("gloo"):
        assert err < 2e-2, (r, err)
        assert same, r


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_head_sharded_llama_two_gpus_nccl() -> None:
    for r, err, same in _two_ranks("nccl"):
        assert err < 2e-2, (r, err)
        assert same, r
