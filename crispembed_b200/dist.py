"""Multi-process helpers for data-parallel runs (one process per GPU).

The encoder shards by sequence: every rank embeds its own sequences with a full
model replica and no collective touches the data path.  The only collectives are
the timing barrier and the max-over-ranks reduction of the measured time.
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
