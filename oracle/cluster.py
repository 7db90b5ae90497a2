"""CPU restatement of fiber/ai's cluster package (cluster/cluster.go), the
checker for the device versions in ai_b200/csrc/fg_cluster.cu.

TEST INFRASTRUCTURE ONLY: imported by tests/ (and nothing that ships). It
follows the reference line by line:

- ``normalize``: cluster.go:19-28 (zero rows stay zero);
- ``kmeans``: cluster.go:43-133 — k-means++ with the weighted pick walked in
  float64 (:57-83), assignment by one product and a first-maximum argmax
  (:88-99, tensor/reduce.go:269-297), float32 row sums in row order
  (:101-108), empty centres restarted on the worst-fitting row (:110-118),
  the stop rule ``changed == 0 && it > 1`` (:120-122);
- ``nearest``: cluster.go:136-148; ``inertia``: :150-160;
- ``cosine``: cluster.go:165-179 (float64 division of float32 sums);
- ``GoRand``: Go's math/rand/v2 PCG (a 128-bit LCG with O'Neill's DXSM
  output, published PCG constants) with Rand.IntN (Lemire's
  multiply-and-reject) and Rand.Float64 (53 bits). Go is not installed here,
  so the stream is **parity unpinned**: it is a restatement of the published
  algorithm, not checked against Go's output.

Products are float64 (rounded to float32 where the reference keeps float32
results), so the oracle sits at or above the reference's precision.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import numpy as np

M64 = (1 << 64) - 1
M128 = (1 << 128) - 1
PCG_MUL = (0x2360ED051FC65DA4 << 64) | 0x4385DF649FCCF645
PCG_INC = (0x5851F42D4C957F2D << 64) | 0x14057B7EF767814F
DXSM_MUL = 0xDA942042E4DD58B5


class GoRand:
    """rand.New(rand.NewPCG(seed1, seed2)) — the methods KMeans draws from."""

    def __init__(self, seed1: int, seed2: int):
        self.hi = seed1 & M64
        self.lo = seed2 & M64

    def uint64(self) -> int:
        st = ((((self.hi << 64) | self.lo) * PCG_MUL) + PCG_INC) & M128
        self.hi, self.lo = st >> 64, st & M64
        h = self.hi
        h ^= h >> 32
        h = (h * DXSM_MUL) & M64
        h ^= h >> 48
        h = (h * (self.lo | 1)) & M64
        return h

    def uint64n(self, n: int) -> int:
        if n & (n - 1) == 0:
            return self.uint64() & (n - 1)
        p = self.uint64() * n
        lo = p & M64
        if lo < n:
            thresh = ((1 << 64) - n) % n
            while lo < thresh:
                p = self.uint64() * n
                lo = p & M64
        return p >> 64

    def intn(self, n: int) -> int:
        if n <= 0:
            raise ValueError("invalid argument to IntN")
        return self.uint64n(n)

    def float64(self) -> float:
        return float((self.uint64() << 11 & M64) >> 11) / float(1 << 53)


def normalize(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32)
    norm = np.sqrt((x.astype(np.float64) ** 2).sum(1)).astype(np.float32)
    norm[norm == 0] = 1
    return (x / norm[:, None]).astype(np.float32)


def _product(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """a · bᵀ in float64, kept as float32 as the reference's MatMul is."""
    return (np.asarray(a, np.float64) @ np.asarray(b, np.float64).T).astype(np.float32)


def argmax_rows(sim: np.ndarray) -> np.ndarray:
    """tensor.Argmax(1): the first index whose value beats every earlier one
    (`v > best`), so a NaN in column 0 keeps 0 and later NaNs are skipped."""
    sim = np.asarray(sim)
    # without NaNs the scan finds the first maximum; later NaNs never win
    out = np.argmax(np.where(np.isnan(sim), -np.inf, sim), axis=1).astype(np.int64)
    out[np.isnan(sim[:, 0])] = 0  # a NaN at column 0 is never beaten
    return out


def similarities(queries: np.ndarray, docs: np.ndarray) -> np.ndarray:
    return _product(queries, docs)


def nearest(x: np.ndarray, centres: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    sim = _product(x, centres)
    idx = argmax_rows(sim)
    return idx, sim[np.arange(len(idx)), idx]


def cosine(a, b) -> float:
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    if a.shape != b.shape:
        raise ValueError(f"cluster: Cosine: lengths {a.size} and {b.size} differ")
    if a.size == 0:
        return 0.0
    dot = np.float32(np.dot(a.astype(np.float64), b.astype(np.float64)))
    na = np.float32(np.dot(a.astype(np.float64), a.astype(np.float64)))
    nb = np.float32(np.dot(b.astype(np.float64), b.astype(np.float64)))
    if na == 0 or nb == 0:
        return 0.0
    return float(np.float32(float(dot) / np.sqrt(float(na) * float(nb))))


@dataclass
class Result:
    centres: np.ndarray      # [k, d] float32, unit rows
    assignment: np.ndarray   # [n] int
    similarity: np.ndarray   # [n] float32
    sizes: np.ndarray        # [k] int
    iterations: int

    def inertia(self) -> float:
        if len(self.similarity) == 0:
            return float("nan")
        return float(np.sum(1.0 - self.similarity.astype(np.float64)) / len(self.similarity))


def kmeans(x: np.ndarray, k: int, iters: int, seed: int) -> Result:
    x = np.asarray(x, np.float32)
    n, d = x.shape
    if k <= 0 or k > n:
        raise ValueError("cluster: k must be between 1 and the number of rows")
    r = GoRand(seed, seed ^ 0x9E3779B97F4A7C15)

    centres: List[np.ndarray] = [x[r.intn(n)].copy()]
    best = np.full(n, -1.0, np.float32)
    while len(centres) < k:
        sim = _product(x, centres[-1][None, :])[:, 0]
        upd = sim > best
        best[upd] = sim[upd]
        w = (np.float32(1) - best).astype(np.float64)  # float32 difference, then widened
        weights = w * w
        total = 0.0
        for v in weights:  # sequential float64 sum, as the reference's loop
            total += float(v)
        pick = r.float64() * total
        idx = n - 1
        for i in range(n):
            pick -= float(weights[i])
            if pick <= 0:
                idx = i
                break
        centres.append(x[idx].copy())
    cs = normalize(np.stack(centres))

    assignment = np.zeros(n, np.int64)
    similarity = np.zeros(n, np.float32)
    sizes = np.zeros(k, np.int64)
    iterations = 0
    for it in range(1, iters + 1):
        iterations = it
        sim = _product(x, cs)
        new = argmax_rows(sim)
        similarity = sim[np.arange(n), new].astype(np.float32)
        changed = int(np.sum(new != assignment))
        assignment = new
        sums = np.zeros((k, d), np.float32)
        np.add.at(sums, assignment, x)  # float32, rows added in order
        sizes = np.bincount(assignment, minlength=k).astype(np.int64)
        for c in range(k):
            if sizes[c] == 0:
                worst = 0
                for i in range(n):
                    if similarity[i] < similarity[worst]:
                        worst = i
                sums[c] = x[worst]
                similarity[worst] = 1
        cs = normalize(sums)
        if changed == 0 and it > 1:
            break
    return Result(cs, assignment, similarity, sizes, iterations)
