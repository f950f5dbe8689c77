"""Data-parallel host logic (rich_triplet_b200.dp) on two gloo ranks on the
CPU: the sequence shards cover every sequence exactly once, and the job time
is the maximum over ranks.  No GPU."""

import os
import socket

import pytest
import torch.multiprocessing as mp

from rich_triplet_b200 import dp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_seqs, out):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        start, end = dp.shard(n_seqs, world, rank)
        mine = torch.tensor([start, end], dtype=torch.int64)
        spans = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(spans, mine)
        local_ms = 10.0 + 5.0 * rank  # rank 1 is the slower one
        ms_max = dp.max_over_ranks(local_ms, dist)
        out.put((rank, [tuple(t.tolist()) for t in spans], ms_max,
                 dp.job_rate(n_seqs * 4, ms_max), dp.prompt_stream(start)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_seqs", [2, 7, 64])
def test_two_gloo_ranks_shard_and_time(n_seqs):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_seqs, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    spans = results[0][1]
    assert spans == results[1][1]
    covered = sorted(i for s, e in spans for i in range(s, e))
    assert covered == list(range(n_seqs))
    assert max(e - s for s, e in spans) - min(e - s for s, e in spans) <= 1
    for rank, _, ms_max, rate, stream in results:
        assert ms_max == 15.0
        assert rate == pytest.approx(n_seqs * 4 / 0.015)
        assert stream == 100 + spans[rank][0]


def test_shard_rejects_bad_arguments():
    with pytest.raises(ValueError):
        dp.shard(4, 0, 0)
    with pytest.raises(ValueError):
        dp.shard(4, 2, 2)
    assert dp.shard(1, 2, 0) == (0, 0) and dp.shard(1, 2, 1) == (0, 1)
