"""Data-parallel replicas of the encoder: one process per GPU, each holding
a full model, each embedding a contiguous slice of the length-sorted batch;
the embeddings meet on rank 0 in one gather, in the caller's order.

The reference embeds a batch on one process (models/gemma embed.go:15-80,
batching in embedBatch embed.go:118-157); sequences never interact, so the
batch shards with no collective in the forward. The split and the gather
here are the multi-GPU layer around that call.

Cost model for the split: a slice padded to its longest sequence costs its
padded tokens in the projections plus the attention's pairs; with the batch
sorted by length (longest first) a contiguous slice pads little, and the
split points put about 1/world of the total cost in each slice.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import numpy as np

# Attention work per token relative to the projections at these shapes:
# 3072 FLOP per (query, key) pair against 202.9 MFLOP of projections per
# token, i.e. one key costs ~1/66 000 of a token; a sequence of length L
# costs L·(1 + L/ATTN_TOKENS).
ATTN_TOKENS = 66_000.0


def sequence_cost(lengths: np.ndarray) -> np.ndarray:
    L = np.asarray(lengths, dtype=np.float64)
    return L * (1.0 + L / ATTN_TOKENS) + 1.0  # +1: a length-0 sequence still runs


def plan_slices(lengths: Sequence[int], world: int) -> List[np.ndarray]:
    """Indices of each rank's sequences: contiguous runs of the batch sorted
    by decreasing length (stable), cut where the running cost crosses
    k/world of the total. Every index appears exactly once; a rank may get
    none when the batch is smaller than the world."""
    if world < 1:
        raise ValueError(f"world size {world} < 1")
    lengths = np.asarray(lengths, dtype=np.int64)
    order = np.argsort(-lengths, kind="stable")
    if len(order) == 0:
        return [order[:0] for _ in range(world)]
    cum = np.cumsum(sequence_cost(lengths[order]))
    total = cum[-1]
    cuts = [0]
    for k in range(1, world):
        # first position whose prefix reaches k/world of the cost
        c = int(np.searchsorted(cum, total * k / world, side="left")) + 1
        cuts.append(min(max(c, cuts[-1]), len(order)))
    cuts.append(len(order))
    return [order[cuts[r]:cuts[r + 1]] for r in range(world)]


def embed_replicated(model, seqs: Sequence[Sequence[int]], dim: Optional[int] = None,
                     group=None, device=None) -> Optional[np.ndarray]:
    """Embeds `seqs` across the process group: each rank runs
    ``model.embed_ids`` on its slice (plan_slices) and rank 0 receives every
    embedding in one gather. Returns the [len(seqs), dim] array on rank 0
    and None elsewhere. Every rank must pass the same `seqs`. `device` is
    where the gather buffers live (the rank's GPU for NCCL; CPU for gloo)."""
    import torch
    import torch.distributed as dist

    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    slices = plan_slices([len(s) for s in seqs], world)
    mine = slices[rank]
    width = int(dim) if dim else int(model.Dim())
    rows = max(len(s) for s in slices)
    buf = torch.zeros((max(rows, 1), width), dtype=torch.float32, device=device)
    if len(mine):
        emb = np.stack(model.embed_ids([seqs[i] for i in mine], width))
        buf[: len(mine)] = torch.from_numpy(emb).to(buf.device)
    dst = dist.get_global_rank(group, 0) if group is not None else 0
    parts = [torch.empty_like(buf) for _ in range(world)] if rank == 0 else None
    dist.gather(buf, parts, dst=dst, group=group)
    if rank != 0:
        return None
    out = np.empty((len(seqs), width), dtype=np.float32)
    for r, idx in enumerate(slices):
        if len(idx):
            out[idx] = parts[r][: len(idx)].cpu().numpy()
    return out
