"""Window sharding over ranks (host logic), with a world-size-2 gloo group on CPU."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from redukt_b200.shard import check_partition, gather_results, max_over_ranks, windows_for_rank


def test_windows_partition_exactly_once():
    for n in (0, 1, 7, 4096):
        for world in (1, 2, 3, 8):
            parts = [windows_for_rank(n, r, world) for r in range(world)]
            check_partition(n, world, parts)
            assert all(i % world == r for r in range(world) for i in parts[r])
    with pytest.raises(ValueError):
        windows_for_rank(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = windows_for_rank(10, rank, world)
        # stand-in for per-window work: a result keyed by window index
        res = {i: i * i for i in mine}
        merged = gather_results(res, dist)
        t = max_over_ranks(1.0 + rank, dist)
        q.put((rank, sorted(merged.items()), t))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_gather_and_max():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, merged, t in out:
        assert merged == [(i, i * i) for i in range(10)]
        assert t == 2.0
