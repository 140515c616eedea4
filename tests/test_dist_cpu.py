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


def _gather_worker(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    from crispembed_b200.dist import all_gather_bytes
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    blob = bytes([rank]) * 64  # stands in for a 64-byte IPC handle
    got = all_gather_bytes(blob)
    dist.barrier()
    dist.destroy_process_group()
    out.put((rank, got))


def test_handle_exchange_gloo_rank_order():
    """connect_expert_parallel's host step: every rank sees every handle, in rank order."""
    import socket

    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [bytes([0]) * 64, bytes([1]) * 64]
    assert res == {0: want, 1: want}


@pytest.mark.parametrize("world,E", [(1, 8), (2, 8), (4, 8), (8, 8), (2, 4), (4, 32)])
def test_ep_recv_plan_partitions_every_row(world, E):
    """The receive layout the exchange kernels implement: on every rank, the
    segments (local expert, source) tile [0, rows of its experts) in
    expert-major, source-minor order, and each segment maps onto the source's own
    expert-major rows of that expert, so every (source, expert) row lands once."""
    from crispembed_b200.dist import ep_recv_plan
    rng = np.random.default_rng(world * 100 + E)
    counts = rng.integers(0, 50, size=(world, E))
    counts[0, 0] = 0  # an empty segment
    seen = {p: np.zeros(int(counts[p].sum()), dtype=np.int32) for p in range(world)}
    for r in range(world):
        off, segs = ep_recv_plan(counts, r)
        E_loc = E // world
        assert off[0] == 0 and off[-1] == counts[:, r * E_loc:(r + 1) * E_loc].sum()
        pos = 0
        for el in range(E_loc):
            assert off[el] == pos
            for p in range(world):
                start, n, src0 = segs[(el, p)]
                assert start == pos and n == counts[p, r * E_loc + el]
                seen[p][src0:src0 + n] += 1
                pos += n
    for p in range(world):
        assert (seen[p] == 1).all()
