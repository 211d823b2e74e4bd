"""Multi-rank host logic on CPU with gloo (world_size 2): layer sharding and
the statistics all-gather the benchmark uses over NCCL."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from kvforge_b200.dist import STAT_KEYS, gather_stats, layer_shard, reduce_stats


def test_layer_shard_covers_all_layers():
    for L_ in (1, 4, 31, 32, 80):
        for W in (1, 2, 3, 4, 8):
            got = [l for r in range(W) for l in layer_shard(L_, W, r)]
            assert got == list(range(L_))
            sizes = [len(layer_shard(L_, W, r)) for r in range(W)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        layer_shard(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    layers = layer_shard(32, world, rank)
    stats = {"layers": len(layers), "input_bytes": 1000.0 * len(layers), "compressed_bytes": 10.0 * (rank + 1),
             "ms": 5.0 + rank}
    per = gather_stats(stats)
    dist.destroy_process_group()
    q.put((rank, per))


def test_gather_stats_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1]
    tot = reduce_stats(res[0])
    assert tot["layers"] == 32 and tot["input_bytes"] == 32000.0
    assert tot["compressed_bytes"] == 30.0 and tot["ms"] == 6.0
    assert set(res[0][0]) == set(STAT_KEYS)
