"""float64 torch restatement of the Lloyd oracle, for parity checks at the benchmark sizes.

TEST INFRASTRUCTURE ONLY (a checker, never the thing measured). It restates
the same reference semantics as ``oracle/lloyd.py`` -- assign =
``argmin_k (||x||^2 + ||c||^2 - 2 x.c)`` with ties to the lowest index
(``flash_kmeans_cuda/csrc/assign/assign_common.cuh:20-28``), update = exact
per-cluster sums and counts (``csrc/update/update_sorted.cu:97-110``),
finalize = ``where(count > 0, sum / count, old)`` rounded through fp32 to the
compute dtype (``csrc/update/update_finalize.cu:39-66``), shift =
``max ||new - old||`` (``kmeans.py:102-104``) -- in float64 torch, so that the
checks of c2/c3/c4/c5-sized problems can run on the GPU (cuBLAS DGEMM and
torch reductions; no code of this library is involved). At small sizes it is
pinned to ``oracle/lloyd.py`` by ``tests/test_oracle_torch.py``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple

import torch

TORCH_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


@dataclass
class Assign:
    ids: torch.Tensor      # (B, N) int64
    best: torch.Tensor     # (B, N) float64 smallest squared distance
    second: torch.Tensor   # (B, N) float64 second smallest (inf when K == 1)
    x_sq: torch.Tensor     # (B, N) float64

    def gap_mask(self, rel: float = 1e-3) -> torch.Tensor:
        """Rows whose top-2 distance gap exceeds rel * ||x||^2 (labels must match there)."""
        return (self.second - self.best) > rel * self.x_sq


def assign(x: torch.Tensor, c: torch.Tensor, chunk_elems: int = 1 << 28) -> Assign:
    """x (B, N, D), c (B, K, D) of any float dtype, on any device; float64 inside.

    Rows are processed in chunks of about ``chunk_elems`` distances. Ties: the
    lowest index among equal float64 distances (``argmin`` returns the first
    occurrence; exact float64 ties only arise for duplicate centroids)."""
    B, N, D = x.shape
    K = c.shape[1]
    x64 = x.to(torch.float64)
    c64 = c.to(torch.float64)
    x_sq = (x64 * x64).sum(-1)
    c_sq = (c64 * c64).sum(-1)
    ids = torch.empty((B, N), dtype=torch.int64, device=x.device)
    best = torch.empty((B, N), dtype=torch.float64, device=x.device)
    second = torch.full((B, N), float("inf"), dtype=torch.float64, device=x.device)
    rows = max(1, min(N, chunk_elems // max(K, 1)))
    for b in range(B):
        for n0 in range(0, N, rows):
            xb = x64[b, n0:n0 + rows]
            dist = x_sq[b, n0:n0 + rows, None] + c_sq[b][None, :] - 2.0 * (xb @ c64[b].T)
            k = torch.argmin(dist, dim=1)
            r = torch.arange(dist.shape[0], device=x.device)
            ids[b, n0:n0 + rows] = k
            best[b, n0:n0 + rows] = dist[r, k]
            if K > 1:
                dist[r, k] = float("inf")
                second[b, n0:n0 + rows] = dist.min(dim=1).values
            del dist
    return Assign(ids=ids, best=best, second=second, x_sq=x_sq)


def update(x: torch.Tensor, ids: torch.Tensor, K: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """float64 sums (B, K, D) and int64 counts (B, K); labels outside [0, K) skipped."""
    B, N, D = x.shape
    sums = torch.zeros((B, K, D), dtype=torch.float64, device=x.device)
    counts = torch.zeros((B, K), dtype=torch.int64, device=x.device)
    for b in range(B):
        lab = ids[b].to(torch.int64)
        ok = (lab >= 0) & (lab < K)
        sums[b].index_add_(0, lab[ok], x[b][ok].to(torch.float64))
        counts[b] = torch.bincount(lab[ok], minlength=K)
    return sums, counts


def abs_sums(x: torch.Tensor, ids: torch.Tensor, K: int) -> torch.Tensor:
    """Per-cluster sums of |x| (the scale of fp32 summation error)."""
    return update(x.abs(), ids, K)[0]


def round_to(a: torch.Tensor, dtype: str) -> torch.Tensor:
    """Round float64 values through fp32 to the compute dtype (round to nearest even)."""
    return a.to(torch.float32).to(TORCH_DTYPES[dtype]).to(torch.float32)


def finalize(sums: torch.Tensor, counts: torch.Tensor, old: torch.Tensor,
             dtype: str) -> torch.Tensor:
    """where(count > 0, sum / count, old) in the compute dtype, returned as float32."""
    cnt = counts.unsqueeze(-1)
    mean = sums / cnt.clamp(min=1).to(torch.float64)
    return torch.where(cnt > 0, round_to(mean, dtype), old.to(torch.float32))


def shift(new: torch.Tensor, old: torch.Tensor) -> float:
    d = new.to(torch.float64) - old.to(torch.float64)
    return float(torch.sqrt((d * d).sum(-1)).max())


def inertia(x: torch.Tensor, c: torch.Tensor, ids: torch.Tensor) -> float:
    """Sum of squared distances of each point to its assigned centroid (float64)."""
    tot = 0.0
    for b in range(x.shape[0]):
        d = x[b].to(torch.float64) - c[b].to(torch.float64)[ids[b].to(torch.int64)]
        tot += float((d * d).sum())
    return tot


def lloyd(x: torch.Tensor, init: torch.Tensor, iters: int,
          dtype: str) -> Tuple[torch.Tensor, torch.Tensor]:
    """``iters`` exact Lloyd iterations from ``init`` (tol = 0); returns the labels of the
    last assignment (against the pre-update centroids, as ``kmeans.py:195``) and the
    final centroids (float32 holding dtype values)."""
    cur = init.to(torch.float32)
    K = cur.shape[1]
    ids = None
    for _ in range(iters):
        a = assign(x, cur)
        s, n = update(x, a.ids, K)
        ids = a.ids
        cur = finalize(s, n, cur, dtype)
    return ids, cur
