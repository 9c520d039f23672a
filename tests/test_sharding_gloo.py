"""Data-parallel sequences on world_size 2, as gloo ranks on the host: the
sequence assignment covers every sequence exactly once, the step time is the
maximum over ranks and throughput sums the ranks' tokens; a rank that never
joins makes the others' first collective fail within its timeout instead of
hanging (the failure is made on the host, nothing runs on a GPU)."""

from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp

from kvdlra_b200.sharding import shard_sequences


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, n_seq: int, q) -> None:
    import torch.distributed as dist

    from kvdlra_b200.sharding import init_ranks, max_over_ranks, shard_sequences, sum_over_ranks

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    r, w = init_ranks("gloo", None, timeout_s=60)
    mine = shard_sequences(n_seq, w, r)
    step_ms = 10.0 + 5.0 * r  # rank 1 is the slower one
    tokens = 128 * len(mine)
    (t_max,) = max_over_ranks([step_ms])
    (tok_sum,) = sum_over_ranks([float(tokens)])
    dist.barrier()
    dist.destroy_process_group()
    q.put((r, mine, t_max, tok_sum))


def test_two_ranks_cover_every_sequence_once() -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, n_seq, world = _port(), 13, 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_seq, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    seqs = sorted(s for _, mine, _, _ in out for s in mine)
    assert seqs == list(range(n_seq))
    assert all(t == 15.0 for _, _, t, _ in out)  # the slower rank's time
    assert all(tok == 128.0 * n_seq for *_, tok in out)


def _lonely(port: int, q) -> None:
    import torch.distributed as dist

    from kvdlra_b200.sharding import init_ranks

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK="0", WORLD_SIZE="2")
    try:
        init_ranks("gloo", None, timeout_s=3)
        dist.barrier()
        q.put("joined")
    except Exception as e:  # noqa: BLE001 -- the expected outcome
        q.put(type(e).__name__)


def test_missing_rank_times_out_instead_of_hanging() -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_port(), q))
    p.start()
    res = q.get(timeout=120)
    p.join(timeout=60)
    assert res != "joined"


def test_shard_rules() -> None:
    assert shard_sequences(64, 8, 3) == [3, 11, 19, 27, 35, 43, 51, 59]
    assert shard_sequences(3, 4, 3) == []
    with pytest.raises(ValueError):
        shard_sequences(4, 2, 2)
