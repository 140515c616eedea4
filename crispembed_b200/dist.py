"""Multi-process helpers (one process per GPU).

Data-parallel replicas shard by sequence: every rank embeds its own sequences
with a full model replica and no collective touches the data path.  Expert
parallelism adds one exchange per MoE block, done by the library's own kernels
over peer memory; the host side only all-gathers the ranks' IPC handles once
(connect_expert_parallel).  Besides that, the collectives are the timing barrier
and the max-over-ranks reduction of the measured time.
"""
from __future__ import annotations

import numpy as np


def shard_sequences(lens: np.ndarray, rank: int, world: int):
    """Contiguous block of sequences for `rank` (sizes differ by at most one).
    Returns (first_sequence, n_sequences, first_token, n_tokens)."""
    n = len(lens)
    base, extra = divmod(n, world)
    s0 = rank * base + min(rank, extra)
    cnt = base + (1 if rank < extra else 0)
    cu = np.concatenate([[0], np.cumsum(lens)])
    return s0, cnt, int(cu[s0]), int(cu[s0 + cnt] - cu[s0])


def max_over_ranks(value: float, device=None) -> float:
    """All-reduce MAX of a per-rank time (identity when not distributed)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_gather_bytes(blob: bytes, group=None) -> list:
    """Every rank's `blob` in rank order (torch.distributed.all_gather_object)."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return [blob]
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, blob, group=group)
    return out


def connect_expert_parallel(ep, group=None):
    """Exchange the ranks' IPC handles and map the peers' regions (collective)."""
    ep.connect(all_gather_bytes(ep.handle(), group))


def ep_recv_plan(counts: np.ndarray, rank: int):
    """Host restatement of the receive layout of `rank` (for tests): counts is the
    [world, E] matrix of per-source expert totals.  Returns (offsets_recv of the
    local experts [E_loc+1], {(local expert, source): (first row, rows, first row
    in the source's own expert-major order)})."""
    world, E = counts.shape
    E_loc = E // world
    g0 = rank * E_loc
    off = [0]
    for el in range(E_loc):
        off.append(off[-1] + int(counts[:, g0 + el].sum()))
    segs = {}
    for el in range(E_loc):
        g = g0 + el
        start = off[el]
        for p in range(world):
            segs[(el, p)] = (start, int(counts[p, g]), int(counts[p, :g].sum()))
            start += int(counts[p, g])
    return np.array(off, dtype=np.int64), segs
