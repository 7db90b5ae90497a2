"""Data-parallel replicas of the encoder: one process per GPU, each holding
a full model, each embedding a contiguous slice of the length-sorted batch;
the embeddings meet on rank 0 in one gather, in the caller's order.

The reference embeds a batch on one process (models/gemma embed.go:15-80,
batching in embedBatch embed.go:118-157); sequences never interact, so the
batch shards with no collective in the forward. The split and the gather
here are the multi-GPU layer around that call.

Cost model for the split: a sequence of length L costs L·t(L) GPU time,
t(L) the time per token of full-length batches of that length, measured on
a B200 (131 072-token batches of EmbeddingGemma-300m, split-TF32):
short sequences cost more per token (per-sequence attention tiles and
pooling), long ones more through the quadratic global layers. The
survey's FLOP estimate (projections + 3072 FLOP per allowed pair) missed
the short-sequence overhead: with it the 4-GPU config-3 ranks at the
extremes ran 17% longer than the middle ones. With the batch sorted by
length (longest first) a contiguous slice pads little, and the split
points put about 1/world of the total cost in each slice.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import numpy as np

# EmbeddingGemma-300m: 4 global and 20 sliding layers, window bound 257
# (|i − j| < 257), 202 899 456 FLOP of projections per token.
PROJ_FLOPS_PER_TOKEN = 202_899_456.0
ATTN_FLOPS_PER_PAIR = 3072.0

# Measured ns per token of full-length 131 072-token batches (B200,
# split-TF32, EmbeddingGemma-300m), by sequence length.
NS_PER_TOKEN = ((16, 959.4), (32, 805.2), (64, 730.1), (128, 688.3), (192, 730.0), (256, 704.1),
                (384, 732.0), (512, 751.2), (768, 771.9), (1024, 784.0), (1280, 788.0),
                (1536, 809.8), (1792, 811.1), (2048, 822.0))


def window_pairs(L: np.ndarray, w: int) -> np.ndarray:
    """(query, key) pairs with |i − j| < w in a sequence of length L."""
    L = np.asarray(L, dtype=np.float64)
    # Σ_i (min(L-1, i+w-1) − max(0, i−w+1) + 1) = L·(2w−1) − (w−1)·w for L ≥ w
    full = L * (2 * w - 1) - (w - 1) * w
    return np.where(L >= w, full, L * L) if w > 0 else L * L


def sequence_flops(lengths, n_global: int = 4, n_local: int = 20, window: int = 257) -> np.ndarray:
    """Algorithmic FLOPs of each sequence: projections + attention pairs."""
    L = np.asarray(lengths, dtype=np.float64)
    pairs = n_global * L * L + n_local * window_pairs(L, window)
    return PROJ_FLOPS_PER_TOKEN * L + ATTN_FLOPS_PER_PAIR * pairs


def sequence_cost(lengths) -> np.ndarray:
    """Estimated GPU time of each sequence in units of one 512-token
    sequence's tokens: L·t(L)/t(512), t interpolated in NS_PER_TOKEN
    (held constant outside the measured lengths). A length-0 sequence runs
    as one token."""
    L = np.maximum(np.asarray(lengths, dtype=np.float64), 1.0)
    xs = np.array([x for x, _ in NS_PER_TOKEN], np.float64)
    ys = np.array([y for _, y in NS_PER_TOKEN], np.float64)
    return L * np.interp(L, xs, ys) / np.interp(512.0, xs, ys)


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
