"""Data-parallel decoding across GPUs: the host-side logic of the multi-GPU path.

Utterances are independent, so each rank (one process per GPU) decodes a contiguous slice of
them with its own session and no collective on the data path. The only collective is the
timing reduction (the max over ranks). The reference renders a batch of utterances in one
process (`drive_batch`, crates/syrinx-fish/src/common/dualar.rs:246-364); this splits the same
list across processes.
"""
from __future__ import annotations


def utterance_slice(n_utterances: int, rank: int, world: int) -> tuple[int, int]:
    """[start, end) of the utterances rank `rank` of `world` decodes: contiguous slices whose
    sizes differ by at most one, covering 0..n_utterances exactly once."""
    if world < 1 or not 0 <= rank < world or n_utterances < 0:
        raise ValueError(f"bad shard request n={n_utterances} rank={rank} world={world}")
    base, extra = divmod(n_utterances, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def rank_seed(base_seed: int, rank: int) -> int:
    """Seed of rank `rank`'s synthetic prompt: every rank decodes a different utterance."""
    return base_seed + rank


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """The max of `value` over all ranks (the slowest rank sets the job's time); `value` itself
    when not distributed. `device` is where the reduction tensor lives: a CUDA device under
    NCCL, the CPU under gloo."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
