"""Data-parallel host logic on CPU ranks (gloo, world size 2)."""
import os

import numpy as np
import pytest

from crispembed_b200.dist import shard_sequences


def test_shard_sequences_cover_batch():
    lens = np.arange(1, 12, dtype=np.int32)
    for world in (1, 2, 3, 4, 8):
        got = [shard_sequences(lens, r, world) for r in range(world)]
        assert sum(g[1] for g in got) == len(lens)
        assert sum(g[3] for g in got) == int(lens.sum())
        starts = [g[0] for g in got]
        assert starts == sorted(starts)
        assert max(g[1] for g in got) - min(g[1] for g in got) <= 1


def _worker(rank, world, port, out):
    import torch.distributed as dist

    from crispembed_b200.dist import max_over_ranks
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    t = max_over_ranks(1.5 + rank)
    dist.barrier()
    dist.destroy_process_group()
    out.put((rank, t))


def test_max_over_ranks_gloo():
    import socket

    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == {0: 2.5, 1: 2.5}
