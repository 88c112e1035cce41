"""Host-side plumbing of the sequence-sharded batched decode across GPUs.

Sequences are independent, so the multi-GPU path has no collective on its data
path: rank ``r`` of ``world`` owns the contiguous block of sequences
``[r * per_rank, (r + 1) * per_rank)`` with its own weights, caches and graph.
The only cross-rank traffic is the timing: every rank's device time is reduced
with MAX (the job is as fast as its slowest rank) and the aggregate tokens/s
is the total tokens of all ranks over that time.  Works with any
``torch.distributed`` backend (``nccl`` on GPUs, ``gloo`` on CPU).
"""

from __future__ import annotations

import torch


def sequence_shard(global_sequences: int, world: int, rank: int) -> range:
    """The contiguous block of global sequence indices owned by ``rank``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if global_sequences % world:
        raise ValueError("the global batch must split evenly over the ranks")
    per = global_sequences // world
    return range(rank * per, (rank + 1) * per)


def shard_contexts(seed: int, shard: range, low: int, high: int) -> tuple[list[int], list[int]]:
    """Seeded (context length, first token) of each sequence of a shard; a
    sequence's values depend only on its global index, not on the world size."""
    lengths, tokens = [], []
    for index in shard:
        gen = torch.Generator().manual_seed(seed * 1_000_003 + index)
        lengths.append(int(torch.randint(low, high + 1, (1,), generator=gen)))
        tokens.append(int(torch.randint(0, 49152, (1,), generator=gen)))
    return lengths, tokens


def max_over_ranks(values: list[float], device: torch.device | str = "cpu") -> list[float]:
    """Element-wise MAX of ``values`` over all ranks (identity without a process group)."""
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def aggregate_tokens_per_s(tokens_per_rank: int, world: int, max_ms: float) -> float:
    """Whole-job throughput: every rank's tokens over the slowest rank's time."""
    if max_ms <= 0:
        raise ValueError("time must be positive")
    return world * tokens_per_rank / (max_ms * 1e-3)
