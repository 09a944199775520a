"""Multi-GPU Lloyd iteration: one process per GPU, ``torch.distributed`` over NCCL.

The reference is single-GPU (it has no collective). Two partitions are
provided, matching how the problem shards:

* ``shard="N"`` - every rank holds a contiguous slice of the points of each
  batch element and a replica of the centroids. Per iteration: local assign +
  counting-sort update into local sums (B, K, D) fp32 and counts (B, K) int32,
  ONE all-reduce (sum) of each, then the same finalize on every rank (same
  inputs -> bit-identical centroids everywhere). Counts stay int32, so they
  are exact for any N < 2^31.
* ``shard="B"`` - every rank owns whole batch elements; there is no
  per-iteration collective except a max-reduction of the shift when ``tol > 0``
  so that all ranks stop at the same iteration (the reference stops on the
  maximum shift over all batch elements, ``kmeans.py:104``).

Labels stay on the rank that owns the points. ``gather=True`` all-gathers them
(and, for ``shard="B"``, the centroids) at the end.

The per-rank compute is a ``LloydState`` (``flash_kmeans_cuda.kmeans``); the
``state_factory`` argument exists so the orchestration can be exercised with
another implementation of the same four methods (the CPU tests use gloo ranks
and an oracle-backed state).
"""

from __future__ import annotations

import datetime
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist


def shard_bounds(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [begin, end) of ``total`` items for ``rank`` (sizes differ by <= 1)."""
    base, rem = divmod(total, world)
    begin = rank * base + min(rank, rem)
    return begin, begin + base + (1 if rank < rem else 0)


def init_process_group_from_env(backend: str = "nccl", timeout_s: float = 120.0) -> None:
    """torchrun-style init with a bounded timeout (ranks that lose a peer fail, not hang)."""
    if not dist.is_initialized():
        dist.init_process_group(backend=backend,
                                timeout=datetime.timedelta(seconds=timeout_s))


def _default_state_factory(x_local: torch.Tensor, n_clusters: int):
    from .kmeans import LloydState

    return LloydState(x_local, n_clusters)


def _broadcast_init(x_local: torch.Tensor, n_clusters: int, group) -> torch.Tensor:
    """Rank 0 picks K random rows of its shard (with replacement); everyone receives them."""
    B, n_local, D = x_local.shape
    if dist.get_rank(group) == 0:
        idx = torch.randint(0, n_local, (B, n_clusters), device=x_local.device)
        c = torch.gather(x_local, 1, idx.unsqueeze(-1).expand(-1, -1, D)).contiguous()
    else:
        c = torch.empty((B, n_clusters, D), dtype=x_local.dtype, device=x_local.device)
    dist.broadcast(c, src=dist.get_global_rank(group, 0) if group is not None else 0,
                   group=group)
    return c


def allreduce_sums_counts(sums: torch.Tensor, counts: torch.Tensor, group=None) -> None:
    """Sum ``sums`` (fp32) and ``counts`` (int32) over the group (two all-reduces:
    the collectives cannot be grouped across dtypes, and counts stay int32, exact
    for any point count below 2**31)."""
    dist.all_reduce(sums, op=dist.ReduceOp.SUM, group=group)
    dist.all_reduce(counts, op=dist.ReduceOp.SUM, group=group)


def batch_kmeans_Euclid_sharded(
    x_local: torch.Tensor,
    n_clusters: int,
    max_iters: int = 100,
    tol: float = 0.0,
    init_centroids: Optional[torch.Tensor] = None,
    verbose: bool = False,
    *,
    shard: str = "N",
    group=None,
    gather: bool = False,
    state_factory: Callable = _default_state_factory,
) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Sharded ``batch_kmeans_Euclid``.

    Args:
        x_local: this rank's points: (B, N_local, D) for ``shard="N"``,
            (B_local, N, D) for ``shard="B"``.
        init_centroids: (B, K, D) identical on all ranks for ``shard="N"``
            (rank 0's value is broadcast), or this rank's (B_local, K, D) for
            ``shard="B"``. None: random rows (rank 0's shard for ``"N"``).
        gather: all-gather labels (and centroids for ``"B"``) to every rank.

    Returns:
        (labels, centroids, n_iters): labels of this rank's points unless
        ``gather``; centroids (B, K, D) replicated for ``"N"``, this rank's
        batch elements for ``"B"`` unless ``gather``.
    """
    if shard not in ("N", "B"):
        raise ValueError("shard must be 'N' or 'B'")
    assert x_local.dim() == 3, "x must be (B, N, D)"
    x_local = x_local.contiguous()
    B, n_local, D = x_local.shape
    K = int(n_clusters)
    world = dist.get_world_size(group)

    if init_centroids is None:
        if shard == "N":
            cur = _broadcast_init(x_local, K, group)
        else:
            from .kmeans import init_centroids_random

            cur = init_centroids_random(x_local, K)
    else:
        cur = init_centroids.contiguous().clone().view(B, K, D)
        if shard == "N":
            dist.broadcast(cur, src=dist.get_global_rank(group, 0) if group is not None else 0,
                           group=group)

    need_shift = tol > 0 or verbose
    state = state_factory(x_local, K)
    state.set_centroids(cur)
    nxt = torch.empty_like(cur)
    n_iters_run = 0
    for it in range(max_iters):
        if shard == "N":
            state.local(cur)
            if world > 1:
                allreduce_sums_counts(state.sums, state.counts, group)
            state.finalize(cur, nxt, need_shift)
        else:
            state.step(cur, nxt, need_shift)
            if need_shift and world > 1:
                dist.all_reduce(state.shift, op=dist.ReduceOp.MAX, group=group)
        n_iters_run = it + 1
        if need_shift:
            s = float(state.shift.item())
            if verbose and dist.get_rank(group) == 0:
                print(f"Iter {it}, center shift: {s:.6f}")
            if s < tol:
                cur = nxt
                break
        cur, nxt = nxt, cur

    labels = state.ids
    if gather and world > 1:
        if shard == "N":
            labels = _all_gather_var(labels, dim=1, group=group)
        else:
            labels = _all_gather_var(labels, dim=0, group=group)
            cur = _all_gather_var(cur, dim=0, group=group)
    return labels, cur, n_iters_run


def _all_gather_var(t: torch.Tensor, dim: int, group) -> torch.Tensor:
    """All-gather along ``dim`` with per-rank sizes that may differ by one."""
    world = dist.get_world_size(group)
    size = torch.tensor([t.shape[dim]], device=t.device, dtype=torch.int64)
    sizes = [torch.zeros_like(size) for _ in range(world)]
    dist.all_gather(sizes, size, group=group)
    sizes = [int(s.item()) for s in sizes]
    mx = max(sizes)
    pad_shape = list(t.shape)
    pad_shape[dim] = mx
    padded = torch.zeros(pad_shape, dtype=t.dtype, device=t.device)
    padded.narrow(dim, 0, t.shape[dim]).copy_(t)
    bufs = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(bufs, padded, group=group)
    return torch.cat([b.narrow(dim, 0, s) for b, s in zip(bufs, sizes)], dim=dim)
