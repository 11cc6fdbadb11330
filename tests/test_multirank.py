"""Request sharding across ranks, exercised with world-size-2 gloo process groups on the CPU: the
assignment is a partition, balanced, identical on every rank, and a rank that fails is noticed by
the other through the host-side store (no GPU involved)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from instantllm_b200 import shard


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    prefixes = shard.config5_requests()
    mine = shard.assign(prefixes, world)[rank]
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    store = dist.distributed_c10d._get_default_store()
    status = "ok"
    if rank == fail_rank:
        store.set(f"failed/{rank}", "1")  # the host-side failure report of a crashed worker
        status = "failed"
    elif fail_rank >= 0:
        # before its next collective a healthy rank checks the store for failure reports
        try:
            store.wait([f"failed/{fail_rank}"], datetime.timedelta(seconds=10))
            status = "saw-failure"
        except Exception:
            status = "missed"
    q.put((rank, gathered, status))
    if fail_rank < 0:
        dist.barrier()
    dist.destroy_process_group()


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=60) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    return sorted(res)


def test_assignment_is_a_balanced_partition():
    prefixes = shard.config5_requests()
    assert len(prefixes) == 256 and min(prefixes) >= 128 and max(prefixes) <= 2048
    for world in (1, 2, 4, 8):
        parts = shard.assign(prefixes, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(256))
        loads = [sum(shard.request_cost(prefixes[i]) for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(shard.request_cost(p) for p in prefixes)


def test_pairs_cover_a_rank_and_match_neighbouring_lengths():
    prefixes = shard.config5_requests(n=64)
    for world in (1, 2, 8):
        for mine in shard.assign(prefixes, world):
            ps = shard.pairs(mine, prefixes)
            assert sorted(i for p in ps for i in p) == sorted(mine)
            assert all(len(p) == 2 for p in ps[:-1]) and len(ps[-1]) == (2 if len(mine) % 2 == 0 else 1)
            lens = [prefixes[i] for p in ps for i in p]
            assert lens == sorted(lens, reverse=True)  # longest first, neighbours together
    assert shard.pairs([3, 1, 2], [10, 30, 30, 20]) == [(1, 2), (3,)]
    assert shard.groups([0, 1, 2, 3, 4], [5, 9, 7, 8, 6], 4) == [(1, 3, 2, 4), (0,)]


def test_two_gloo_ranks_agree_on_the_partition():
    res = _run(2)
    (r0, g0, s0), (r1, g1, s1) = res
    assert s0 == s1 == "ok"
    assert g0 == g1
    assert sorted(g0[0] + g0[1]) == list(range(256))
    assert not set(g0[0]) & set(g0[1])


def test_failed_rank_is_detected_on_the_host():
    res = _run(2, fail_rank=1)
    status = {r: s for r, _, s in res}
    assert status[1] == "failed" and status[0] == "saw-failure"
