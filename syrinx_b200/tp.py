"""Tensor-parallel decoding across the GPUs of one node (config 5): the host-side plumbing.

One process per GPU. Every rank loads the same weight blob as its shard
(`Model(..., tp_rank=r, tp_size=n)`): query and kv heads, FFN rows, and the matching input
columns of wo and w2 are split over the ranks; norms, embeddings and the heads are
replicated, so every rank computes the same greedy tokens without a collective. The only
cross-GPU step on the data path is the residual merge after wo and w2, done inside the
library's merge kernel over NVLink (peer pointers from CUDA IPC). This module only exchanges
the sessions' IPC handles, over torch.distributed (any backend).

The reference decodes on one device (`S2Pro`, crates/syrinx-fish/src/s2/mod.rs:119-167);
this splits the same per-frame step across ranks.
"""
from __future__ import annotations

from .configs import ModelConfig


def shard_dims(cfg: ModelConfig, tp: int) -> dict:
    """Per-rank sizes of the tensor-parallel split of `cfg`'s slow stack (the fast stack splits
    the same way). Raises when the split does not divide into whole 32-column blocks."""
    s = cfg.slow
    if tp < 1 or tp > 8:
        raise ValueError("tp must be 1..8")
    if s.n_head % tp or s.n_local_heads % tp or s.intermediate_size % tp:
        raise ValueError(f"heads {s.n_head}/{s.n_local_heads} and FFN {s.intermediate_size} must divide by tp={tp}")
    hl, fl = s.n_head // tp, s.intermediate_size // tp
    if (hl * s.head_dim) % 32 or fl % 32:
        raise ValueError("wo / w2 shards must be whole 32-column Q8_0 blocks")
    return {"n_head": hl, "n_local_heads": s.n_local_heads // tp, "intermediate_size": fl,
            "qkv_rows": (hl + 2 * (s.n_local_heads // tp)) * s.head_dim,
            "wo_cols": hl * s.head_dim, "w2_cols": fl}


def connect(session, dist=None) -> None:
    """Exchange `session`'s IPC handle with every rank of the default process group and map
    the peers (collective: every rank calls it). `session` is a B200DualAr of a TP model."""
    if dist is None:
        import torch.distributed as dist
    world = dist.get_world_size()
    mine = session.tp_handle()
    handles = [None] * world
    dist.all_gather_object(handles, mine)
    session.tp_connect(handles)


def reconnect(session, dist=None) -> None:
    """Recover a group after a failed residual exchange (collective): every rank unmaps its
    peers, the ranks meet, and the handle exchange runs again, which clears every rank's
    exchange state before any rank can push into it. Reset and prefill afterwards."""
    if dist is None:
        import torch.distributed as dist
    session.tp_disconnect()
    dist.barrier()
    connect(session, dist)


def close(session, model, dist=None) -> None:
    """Tear down a tensor-parallel rank: every rank unmaps its peers before any rank frees
    its own exchange region (collective)."""
    if dist is None:
        import torch.distributed as dist
    dist.barrier()
    session.tp_disconnect()
    dist.barrier()
    session.close()
    model.close()
