"""Multi-threaded CPU Lloyd loop in PyTorch: the CPU baseline.

TEST / BENCHMARK INFRASTRUCTURE ONLY (see ``oracle/lloyd.py`` for the rule on
who may import ``oracle/``). The reference has no CPU implementation of its
path; its upstream ships a PyTorch fallback that is absent from the reference
tree, so this restates the same loop (``flash_kmeans_cuda/kmeans.py:73-105``)
with CPU PyTorch ops in fp32, using every host core:

  assign: argmin_k (||c||^2 - 2 x @ c^T)      (MKL/OpenMP matmul + argmin)
  update: index_add_ of rows, bincount        (scatter-add)
  finalize: where(count > 0, sum / count, old)
"""

from __future__ import annotations

import os
import time
from typing import Tuple

import torch


def lloyd_cpu(x: torch.Tensor, init: torch.Tensor, max_iters: int,
              chunk: int = 16384) -> Tuple[torch.Tensor, torch.Tensor]:
    """x (B, N, D) and init (B, K, D) float32 CPU tensors."""
    B, N, D = x.shape
    K = init.shape[1]
    cur = init.clone()
    ids = torch.empty((B, N), dtype=torch.int64)
    for _ in range(max_iters):
        c_sq = (cur * cur).sum(-1)  # (B, K)
        for b in range(B):
            for n0 in range(0, N, chunk):
                xb = x[b, n0:n0 + chunk]
                score = torch.addmm(c_sq[b].unsqueeze(0), xb, cur[b].t(), beta=1.0, alpha=-2.0)
                ids[b, n0:n0 + chunk] = score.argmin(dim=1)
        new = torch.empty_like(cur)
        for b in range(B):
            sums = torch.zeros((K, D), dtype=torch.float32)
            sums.index_add_(0, ids[b], x[b])
            counts = torch.bincount(ids[b], minlength=K).to(torch.float32).unsqueeze(1)
            new[b] = torch.where(counts > 0, sums / counts.clamp_min(1), cur[b])
        cur = new
    return ids, cur


def time_lloyd_cpu(B: int, N: int, K: int, D: int, iters: int, seed: int = 0,
                   threads: int | None = None, repeats: int = 3) -> dict:
    """Median wall time of ``iters`` CPU iterations on seeded N(0,1) data."""
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((B, N, D), generator=g, dtype=torch.float32)
    init = torch.stack([x[b, torch.randperm(N, generator=g)[:K]] for b in range(B)])
    lloyd_cpu(x, init, 1)  # warm-up (thread pool, allocator)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        lloyd_cpu(x, init, iters)
        times.append(time.perf_counter() - t0)
    times.sort()
    med = times[len(times) // 2]
    return dict(seconds=med, ms_per_iter=1e3 * med / iters, threads=threads,
                flops=2.0 * B * N * K * D * iters)
