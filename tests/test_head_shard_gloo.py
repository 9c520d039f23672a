"""KV-head sharding of one sequence on world_size 2, as gloo ranks on the host.

Each rank keeps the whole cache and the whole k/v projections, splits the
query projection by head, answers its own heads' attention and all-gathers
the per-head outputs before ``o_proj`` (``shard_attention_heads``).  On the
host the cache is transformers' ``DynamicCache`` and the attention SDPA over
the rank's heads (the factored kernels take the same head ranges on the GPU:
tests/test_gpu_head_shard.py).  The sharded model's logits must equal the
unsharded model's on every rank, through a chunked prefill and decode steps.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from kvdlra_b200.sharding import GatherHeads, shard_heads


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(model, ids: torch.Tensor, chunk: int, steps: int) -> torch.Tensor:
    """Logits of the last position of every chunk and of every greedy step."""
    from transformers import DynamicCache

    cache = DynamicCache()
    rows = []
    with torch.no_grad():
        for s0 in range(0, ids.shape[1], chunk):
            pos = torch.arange(s0, min(ids.shape[1], s0 + chunk))[None]
            out = model(ids[:, s0 : s0 + chunk], past_key_values=cache, use_cache=True, position_ids=pos)
            rows.append(out.logits[0, -1])
        nxt = int(rows[-1].argmax())
        for j in range(steps):
            pos = torch.tensor([[ids.shape[1] + j]])
            out = model(torch.tensor([[nxt]]), past_key_values=cache, use_cache=True, position_ids=pos)
            rows.append(out.logits[0, -1])
            nxt = int(rows[-1].argmax())
    return torch.stack(rows)


def _worker(rank: int, world: int, port: int, q) -> None:
    import copy

    import torch.distributed as dist

    from golden.make_golden import MODEL_CASE, tiny_llama

    from kvdlra_b200 import enable_factored_decode
    from kvdlra_b200.sharding import init_ranks, shard_attention_heads

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    r, w = init_ranks("gloo", None, timeout_s=60)
    try:
        torch.set_num_threads(2)
        model = tiny_llama(MODEL_CASE)
        ids = torch.randint(0, MODEL_CASE["vocab"], (1, 96), generator=torch.Generator().manual_seed(7))
        model.set_attn_implementation("sdpa")
        full = _run(model, ids, chunk=32, steps=4)
        sharded = enable_factored_decode(shard_attention_heads(copy.deepcopy(model), r, w))
        att = sharded.model.layers[0].self_attn
        got = _run(sharded, ids, chunk=32, steps=4)
        err = float((got - full).abs().max() / full.abs().max())
        q.put((r, att.kvd_heads, tuple(att.q_proj.weight.shape), err))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_ranks_head_sharded_logits_equal_unsharded() -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, world = _port(), 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # MODEL_CASE: 8 query heads over 2 KV heads of 64, hidden 256
    assert [o[1] for o in out] == [(0, 1), (1, 1)]
    assert all(o[2] == (4 * 64, 256) for o in out)
    for r, _, _, err in out:
        assert err < 1e-5, (r, err)


def test_head_ranges() -> None:
    assert shard_heads(8, 8, 3) == (3, 1)
    assert shard_heads(8, 2, 1) == (4, 4)
    assert shard_heads(8, 1, 0) == (0, 8)
    with pytest.raises(ValueError):
        shard_heads(8, 3, 0)
    with pytest.raises(ValueError):
        shard_heads(8, 2, 2)


def test_gather_heads_is_o_proj_on_one_rank() -> None:
    """Without a process group (or on one rank) the wrapper is ``o_proj``."""
    lin = torch.nn.Linear(16, 8)
    x = torch.randn(2, 3, 16)
    assert torch.equal(GatherHeads(lin)(x), lin(x))
