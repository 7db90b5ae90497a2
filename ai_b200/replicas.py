"""Data-parallel replicas of the encoder: one process per GPU, each holding
a full model, each embedding a contiguous slice of the length-sorted batch;
the embeddings meet on rank 0 in one gather, in the caller's order.

The reference embeds a batch on one process (models/gemma embed.go:15-80,
batching in embedBatch embed.go:118-157); sequences never interact, so the
batch shards with no collective in the forward. The split and the gather
here are the multi-GPU layer around that call.

The split is the library's (fg_plan_split, the one fg_embed_many_multi
uses inside one process): the batch stably sorted by increasing length, as
sortIndex sorts it (models/gemma/model.go:412), cut into contiguous runs of
about equal estimated GPU time (fg_sequence_cost: a sequence of L tokens
costs L·t(L), t the measured time per token of full-length batches of that
length on a B200). Contiguous runs of the sorted order pad little.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import numpy as np

def sequence_cost(lengths) -> np.ndarray:
    """Estimated GPU time of each sequence (units: one token of a 512-token
    sequence), the library's fg_sequence_cost."""
    from .gemma import sequence_cost as cost

    return cost(lengths)


def plan_slices(lengths: Sequence[int], world: int) -> List[np.ndarray]:
    """Indices of each rank's sequences: contiguous runs of the batch sorted
    by increasing length (stable), cut where the running cost crosses
    k/world of the total (fg_plan_split). Every index appears exactly once;
    a rank may get none when the batch is smaller than the world."""
    if world < 1:
        raise ValueError(f"world size {world} < 1")
    from .gemma import plan_split

    return plan_split(np.asarray(lengths, dtype=np.int64), world)


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
