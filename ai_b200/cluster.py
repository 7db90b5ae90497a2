"""fiber/ai's ``cluster`` package on the GPU: k-means, nearest centres and
similarity matrices over embedding rows (cluster/cluster.go), through
libfgemma's C ABI on float32 CUDA tensors.

- ``Normalize`` (cluster.go:19-28), ``Similarities`` (:185-190),
  ``Nearest`` (:136-148), ``KMeans`` → ``Result`` with ``Inertia``
  (:43-133, :150-160) run on the device; the similarity products are the
  split-TF32 tensor-core GEMM, as the reference builds them on its matrix
  product.
- ``Cosine`` (:165-179) of two host vectors stays on the host.

Argument errors raise ``ClusterError`` where the reference panics.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass
from typing import List, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import PREC_SPLIT, PREC_SPLIT_TF32, PREC_TF32  # noqa: F401


class ClusterError(ValueError):
    """An argument error, raised where the reference panics."""


def _rows(name: str, x: torch.Tensor) -> None:
    if not isinstance(x, torch.Tensor) or x.dtype != torch.float32 or not x.is_cuda or x.dim() != 2:
        raise ClusterError(f"cluster: {name} must be a 2-D float32 CUDA tensor")
    if x.stride(1) != 1:
        raise ClusterError(f"cluster: {name} rows must be contiguous")


def _stream(x: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)


def Normalize(x: torch.Tensor) -> torch.Tensor:
    """x with every row scaled to unit length; zero rows stay zero."""
    _rows("Normalize", x)
    out = torch.empty_like(x, memory_format=torch.contiguous_format)
    _lib.check(_lib.lib().fg_normalize_rows(x.shape[0], x.shape[1], C.c_void_p(x.data_ptr()), x.stride(0),
                                            C.c_void_p(out.data_ptr()), out.stride(0), _stream(x)))
    return out


def Similarities(queries: torch.Tensor, docs: torch.Tensor, precision: int = PREC_SPLIT) -> torch.Tensor:
    """The [q, n] cosine similarities of unit-length rows: queries · docsᵀ."""
    _rows("Similarities", queries)
    _rows("Similarities", docs)
    if queries.shape[1] != docs.shape[1]:
        raise ClusterError(f"cluster: Similarities: shapes {list(queries.shape)} and {list(docs.shape)}")
    q, n = queries.shape[0], docs.shape[0]
    ld = max(4, (n + 3) // 4 * 4)
    buf = torch.empty((q, ld), dtype=torch.float32, device=queries.device)
    _lib.check(_lib.lib().fg_similarities(q, n, queries.shape[1], C.c_void_p(queries.data_ptr()),
                                          queries.stride(0), C.c_void_p(docs.data_ptr()), docs.stride(0),
                                          C.c_void_p(buf.data_ptr()), ld, precision, _stream(queries)))
    return buf[:, :n]


def Nearest(x: torch.Tensor, centres: torch.Tensor,
            precision: int = PREC_SPLIT) -> Tuple[List[int], List[float]]:
    """For every row of x, the index of the most similar centre (first on
    ties) and that similarity."""
    _rows("Nearest", x)
    _rows("Nearest", centres)
    if x.shape[1] != centres.shape[1] or centres.shape[0] == 0:
        raise ClusterError(f"cluster: Nearest: shapes {list(x.shape)} and {list(centres.shape)}")
    n = x.shape[0]
    idx = torch.empty(n, dtype=torch.int32, device=x.device)
    sim = torch.empty(n, dtype=torch.float32, device=x.device)
    _lib.check(_lib.lib().fg_nearest(n, centres.shape[0], x.shape[1], C.c_void_p(x.data_ptr()), x.stride(0),
                                     C.c_void_p(centres.data_ptr()), centres.stride(0),
                                     C.c_void_p(idx.data_ptr()), C.c_void_p(sim.data_ptr()), precision,
                                     _stream(x)))
    return idx.cpu().tolist(), sim.cpu().tolist()


@dataclass
class Result:
    """cluster.Result: centres [k, d] (unit rows, on the device), the
    centre of each row, each row's similarity to it, rows per centre."""
    Centres: torch.Tensor
    Assignment: List[int]
    Similarity: List[float]
    Sizes: List[int]
    Iterations: int

    def Inertia(self) -> float:
        """Mean cosine distance of rows to their centres (lower is tighter)."""
        if not self.Similarity:
            return math.nan
        s = np.asarray(self.Similarity, np.float32).astype(np.float64)
        return float(np.sum(1.0 - s) / len(s))


def KMeans(x: torch.Tensor, k: int, iters: int, seed: int, precision: int = PREC_SPLIT) -> Result:
    """k-means of the unit-length rows of x by cosine similarity:
    k-means++ seeding, then up to iters rounds, stopping early when no row
    changes centre."""
    _rows("KMeans", x)
    n, d = x.shape
    if k <= 0 or k > n:
        raise ClusterError("cluster: k must be between 1 and the number of rows")
    dev = x.device
    centres = torch.empty((k, d), dtype=torch.float32, device=dev)
    assign = torch.empty(n, dtype=torch.int32, device=dev)
    sim = torch.empty(n, dtype=torch.float32, device=dev)
    sizes = torch.empty(k, dtype=torch.int32, device=dev)
    it = C.c_int(0)
    _lib.check(_lib.lib().fg_kmeans(n, d, C.c_void_p(x.data_ptr()), x.stride(0), int(k), int(iters),
                                    C.c_uint64(int(seed) & ((1 << 64) - 1)), C.c_void_p(centres.data_ptr()),
                                    C.c_void_p(assign.data_ptr()), C.c_void_p(sim.data_ptr()),
                                    C.c_void_p(sizes.data_ptr()), C.byref(it), precision, _stream(x)))
    return Result(centres, assign.cpu().tolist(), sim.cpu().tolist(), sizes.cpu().tolist(), int(it.value))


def Cosine(a: Sequence[float], b: Sequence[float]) -> float:
    """Cosine similarity of two equal-length host vectors: 1 same direction,
    −1 opposite, 0 orthogonal or when either is all zero. float32 sums of
    a·b, a·a, b·b, then a float64 quotient (cluster.go:165-179)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    if a.shape != b.shape:
        raise ClusterError(f"cluster: Cosine: lengths {a.size} and {b.size} differ")
    if a.size == 0:
        return 0.0
    dot = np.float32(np.dot(a, b))
    na = np.float32(np.dot(a, a))
    nb = np.float32(np.dot(b, b))
    if na == 0 or nb == 0:
        return 0.0
    return float(np.float32(float(dot) / math.sqrt(float(na) * float(nb))))
