"""Row sharding across the GPUs of one node.

Every fused layer op is row-independent, so multi-GPU work is split by whole
sequences (all rows of one sample stay on one GPU: its per-sample modulation
gradients stay local) and needs no collective on the data path.  The only
communication is host-side plumbing: a barrier and the max-over-ranks time.
"""

from __future__ import annotations

import torch


def shard_sequences(num_sequences: int, world: int, rank: int) -> range:
    """Contiguous block of sequence indices owned by `rank`.

    The first ``num_sequences % world`` ranks take one extra sequence; the
    blocks are disjoint and cover ``range(num_sequences)`` in rank order.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    if num_sequences < 0:
        raise ValueError("num_sequences must be >= 0")
    base, extra = divmod(num_sequences, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def rows_of(seqs: range, seq_len: int) -> range:
    """Global row indices of a block of sequences ([B*S, D] row-major)."""
    return range(seqs.start * seq_len, seqs.stop * seq_len)


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    """Max of a per-rank scalar (e.g. a timed duration) over the process group."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
