"""CPU restatement of the reference's Euclidean Lloyd iteration.

TEST INFRASTRUCTURE ONLY. This module is the parity checker: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / ``--impl
reference`` legs may import it. The product path (``flash_kmeans_cuda``) never
does, and has no CPU fallback.

numpy, float64 arithmetic. Each function cites the reference code it restates
(paths inside OpsiClear/flash-kmeans-cuda):

* ``assign``: ``argmin_k (||x||^2 + ||c||^2 - 2 x.c)`` with ties to the lowest
  index -- ``flash_kmeans_cuda/csrc/assign/assign_common.cuh:20-28`` (strict "<"
  update), ``tests/test_mma_optin.py:29-32`` (fp32 einsum reference),
  ``tests/cpp/smoke.cpp:21-29``. ``c_sq`` from the dtype-rounded centroids
  (``flash_kmeans_cuda/kmeans.py:94``).
* ``update``: per-cluster sums and counts -- ``csrc/update/update_sorted.cu:97-110``
  (sum of the rows of each run, count = run length), labels outside [0, K)
  skipped (``update_sorted.cu:94``).
* ``finalize``: ``where(count > 0, sum / count, old)`` cast to the compute
  dtype -- ``csrc/update/update_finalize.cu:39-66``, ``tests/cpp/smoke.cpp:89-93``.
* ``shift``: ``max ||new - old||_2`` -- ``kmeans.py:102-104``.
* ``lloyd``: the loop of ``kmeans.py:108-195`` (labels returned are those of
  the last assignment, made against the pre-update centroids).

Parity pins: the reference ships no golden vectors (its label tests are
statistical, see ``tests/test_oracle.py``); ``tests/golden/`` holds fixtures
produced by the reference's own CUDA kernels (built from source by
``oracle/build_ref.sh``) on a B200, against which this module is checked.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import numpy as np

DTYPES = ("float16", "bfloat16", "float32")


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round to the compute dtype through fp32 (the reference divides in fp32 and then
    casts, update_finalize.cu:60-62); round-to-nearest-even; returns float32 values."""
    a32 = np.asarray(a, dtype=np.float64).astype(np.float32)
    if dtype == "float32":
        return a32
    if dtype == "float16":
        return a32.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        u = a32.view(np.uint32).astype(np.uint64)
        bias = ((u >> 16) & 1) + 0x7FFF
        r = ((u + bias) & 0xFFFF0000).astype(np.uint32)
        nan = np.isnan(a32)
        out = r.view(np.float32).copy()
        out[nan] = np.nan
        return out
    raise ValueError(f"unknown dtype {dtype}")


def sq_norms(a: np.ndarray) -> np.ndarray:
    """Row squared norms in float64; a is (..., D)."""
    a64 = np.asarray(a, dtype=np.float64)
    return np.einsum("...d,...d->...", a64, a64)


@dataclass
class AssignResult:
    ids: np.ndarray     # (B, N) int32
    best: np.ndarray    # (B, N) float64 smallest squared distance
    second: np.ndarray  # (B, N) float64 second smallest (inf when K == 1)
    x_sq: np.ndarray    # (B, N) float64

    def gap_mask(self, rel: float = 1e-3) -> np.ndarray:
        """Rows whose top-2 distance gap exceeds rel * ||x||^2 (labels must match there)."""
        return (self.second - self.best) > rel * self.x_sq


def assign(x: np.ndarray, c: np.ndarray, c_sq: Optional[np.ndarray] = None,
           chunk: int = 8192) -> AssignResult:
    """x (B, N, D), c (B, K, D) float arrays holding dtype values."""
    x = np.asarray(x, dtype=np.float64)
    c = np.asarray(c, dtype=np.float64)
    B, N, D = x.shape
    K = c.shape[1]
    x_sq = sq_norms(x)
    if c_sq is None:
        c_sq = sq_norms(c)
    c_sq = np.asarray(c_sq, dtype=np.float64)
    ids = np.empty((B, N), dtype=np.int32)
    best = np.empty((B, N))
    second = np.full((B, N), np.inf)
    for b in range(B):
        cb = c[b]
        for n0 in range(0, N, chunk):
            xb = x[b, n0:n0 + chunk]
            dist = x_sq[b, n0:n0 + chunk, None] + c_sq[b][None, :] - 2.0 * (xb @ cb.T)
            k = np.argmin(dist, axis=1)  # first occurrence == lowest index on ties
            rows = np.arange(dist.shape[0])
            ids[b, n0:n0 + chunk] = k
            best[b, n0:n0 + chunk] = dist[rows, k]
            if K > 1:
                dist[rows, k] = np.inf
                second[b, n0:n0 + chunk] = dist.min(axis=1)
    return AssignResult(ids=ids, best=best, second=second, x_sq=x_sq)


def update(x: np.ndarray, ids: np.ndarray, K: int) -> Tuple[np.ndarray, np.ndarray]:
    """Per-cluster float64 sums (B, K, D) and int64 counts (B, K)."""
    x = np.asarray(x, dtype=np.float64)
    B, N, D = x.shape
    sums = np.zeros((B, K, D))
    counts = np.zeros((B, K), dtype=np.int64)
    for b in range(B):
        lab = np.asarray(ids[b], dtype=np.int64)
        ok = (lab >= 0) & (lab < K)
        np.add.at(sums[b], lab[ok], x[b][ok])
        counts[b] = np.bincount(lab[ok], minlength=K)
    return sums, counts


def finalize(sums: np.ndarray, counts: np.ndarray, old: np.ndarray, dtype: str) -> np.ndarray:
    """where(count > 0, sum / count, old), rounded to dtype."""
    cnt = np.asarray(counts)[..., None]
    mean = np.asarray(sums, dtype=np.float64) / np.maximum(cnt, 1)
    new = np.where(cnt > 0, round_to(mean, dtype), np.asarray(old, dtype=np.float32))
    return new.astype(np.float32)


def shift(new: np.ndarray, old: np.ndarray) -> float:
    d = np.asarray(new, dtype=np.float64) - np.asarray(old, dtype=np.float64)
    return float(np.sqrt(np.einsum("...d,...d->...", d, d)).max())


def inertia(x: np.ndarray, c: np.ndarray, ids: np.ndarray) -> float:
    """Sum of squared distances of each point to its assigned centroid (float64)."""
    x = np.asarray(x, dtype=np.float64)
    c = np.asarray(c, dtype=np.float64)
    tot = 0.0
    for b in range(x.shape[0]):
        d = x[b] - c[b][np.asarray(ids[b], dtype=np.int64)]
        tot += float(np.einsum("nd,nd->", d, d))
    return tot


@dataclass
class LloydResult:
    ids: np.ndarray
    centroids: np.ndarray
    n_iters: int
    history: List[dict] = field(default_factory=list)


def lloyd(x: np.ndarray, init: np.ndarray, max_iters: int, tol: float, dtype: str,
          keep_history: bool = False) -> LloydResult:
    """The reference loop (kmeans.py:108-195) with exact float64 steps."""
    x = round_to(x, dtype)
    cur = round_to(init, dtype)
    K = cur.shape[1]
    ids = np.zeros(x.shape[:2], dtype=np.int32)
    hist: List[dict] = []
    n_run = 0
    for it in range(max_iters):
        a = assign(x, cur)
        sums, counts = update(x, a.ids, K)
        new = finalize(sums, counts, cur, dtype)
        s = shift(new, cur)
        ids = a.ids
        n_run = it + 1
        if keep_history:
            hist.append(dict(ids=a.ids, gap_mask=a.gap_mask(), sums=sums, counts=counts,
                             centroids_in=cur, centroids_out=new, shift=s))
        cur = new
        if tol > 0 and s < tol:
            break
    return LloydResult(ids=ids, centroids=cur, n_iters=n_run, history=hist)
