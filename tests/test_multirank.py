"""Request-parallel multi-GPU host logic on CPU: two gloo ranks each take
their share of a request list from the partitioner, decode it (a host
stand-in for the per-GPU engine) and gather the results; the merged map equals
the serial one, and a request claimed twice is reported."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from rapidocrvl_b200 import config, partition, synth


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _fake_decode(i, n):
    return [(i * 7919 + k * 104729) % 103424 for k in range(n)]


def _worker(rank, world, port, costs, duplicate, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        mine = partition.shard(costs, rank, world)
        if duplicate and rank == 1:
            mine = mine + [partition.shard(costs, 0, world)[0]]
        local = {i: _fake_decode(i, 4) for i in mine}
        try:
            merged = partition.gather_results(local)
            q.put((rank, "ok", sorted(merged.items()), mine))
        except RuntimeError as e:
            q.put((rank, "dup", str(e), mine))
    finally:
        dist.destroy_process_group()


def _run(world, costs, duplicate=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, costs, duplicate, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(out)


@pytest.mark.timeout(300)
def test_two_rank_partition_and_gather():
    cfg = config.Config(**synth.BENCH_CONFIG)
    prompts = [1024 + 397 * i % 7000 for i in range(17)]
    costs = [partition.request_cost(cfg, p, 256) for p in prompts]
    res = _run(2, costs)
    serial = sorted((i, _fake_decode(i, 4)) for i in range(len(costs)))
    shards = []
    for rank, status, merged, mine in res:
        assert status == "ok"
        assert [(k, list(v)) for k, v in merged] == serial
        shards.append(set(mine))
    assert not (shards[0] & shards[1]) and (shards[0] | shards[1]) == set(range(len(costs)))


@pytest.mark.timeout(300)
def test_two_rank_gather_reports_duplicate_request():
    res = _run(2, [10, 9, 8, 7], duplicate=True)
    assert all(status == "dup" for _, status, _, _ in res)
