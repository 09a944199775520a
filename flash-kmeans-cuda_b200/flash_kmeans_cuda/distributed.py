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

from ._trace import nvtx


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
    with nvtx("fkc.allreduce"):
        dist.all_reduce(sums, op=dist.ReduceOp.SUM, group=group)
        dist.all_reduce(counts, op=dist.ReduceOp.SUM, group=group)


def multimem_enabled() -> bool:
    """FKC_MULTIMEM=0 selects the NCCL all-reduce path for sharded runs."""
    import os

    return os.environ.get("FKC_MULTIMEM", "1") != "0"


class MultimemLloyd:
    """Data-parallel Lloyd step (points sharded over ranks) whose all-reduce of
    sums/counts is fused into the finalize over NVLink multicast.

    Workspace, sums, counts, centroids and the shift live in ONE symmetric
    buffer (torch symmetric memory, same layout on every rank, one multicast
    object). A step is: ``fkc_lloyd_local`` (local sums/counts) -> barrier ->
    ``fkc_lloyd_finalize_multimem`` on this rank's slice of the centroid rows
    (the NVSwitch sums the ranks' copies; new rows go to every rank) ->
    barrier. No NCCL call per iteration.
    """

    # Symmetric buffers are allocated and rendezvoused once per (group, shapes):
    # both are collective and cost milliseconds, so repeated runs reuse them.
    _cache: dict = {}

    @classmethod
    def cached(cls, x_local: torch.Tensor, n_clusters: int, n_max: int,
               group=None) -> "MultimemLloyd":
        """A MultimemLloyd for ``x_local`` whose symmetric buffers are reused
        across calls with the same group and shapes (x may change)."""
        from .kmeans import LloydState

        key = (id(group), x_local.device.index, tuple(x_local.shape), x_local.dtype,
               int(n_clusters), int(n_max))
        mm = cls._cache.get(key)
        if mm is None:
            mm = cls(x_local, n_clusters, n_max, group)
            cls._cache[key] = mm
        else:  # per-point terms of this call's x (its contents may have changed)
            mm.state = LloydState(x_local, int(n_clusters), ws=mm.ws, sums=mm.sums,
                                  counts=mm.counts)
        return mm

    @classmethod
    def release_all(cls) -> None:
        """Drops the cached buffers (call on every rank, before the process
        group is destroyed)."""
        for mm in cls._cache.values():
            mm.release()
        cls._cache.clear()

    @staticmethod
    def available(x_local: torch.Tensor, group=None) -> bool:
        try:
            import torch.distributed._symmetric_memory as symm
        except ImportError:
            return False
        if dist.get_backend(group) != "nccl" or int(x_local.shape[-1]) % 4 != 0:
            return False
        try:
            return bool(symm._SymmetricMemory.has_multicast_support(
                symm.DeviceType.CUDA, x_local.device.index))
        except Exception:
            return False

    def __init__(self, x_local: torch.Tensor, n_clusters: int, n_max: int, group=None):
        import torch.distributed._symmetric_memory as symm

        from . import _tensors
        from ._lib import lib
        from .kmeans import LloydState

        B, N, D = (int(v) for v in x_local.shape)
        K = int(n_clusters)
        dev = x_local.device
        code = _tensors.dtype_code(x_local)
        es = x_local.element_size()
        ws_bytes = int(lib.fkc_lloyd_workspace_size(B, n_max, K, D, code))

        def up(v):
            return (v + 255) // 256 * 256

        off_ws = 0
        off_sums = up(off_ws + ws_bytes)
        off_counts = up(off_sums + B * K * D * 4)
        off_c = up(off_counts + B * K * 4)
        off_shift = up(off_c + B * K * D * es)
        off_bar = up(off_shift + 8)  # the step's barrier words (fkc_lloyd_finalize_multimem_synced)
        total = up(off_bar + 16)
        self.buf = symm.empty(total, dtype=torch.uint8, device=dev)
        self.handle = symm.rendezvous(self.buf, group if group is not None else dist.group.WORLD)
        mc = int(self.handle.multicast_ptr)
        if mc == 0:
            raise RuntimeError("symmetric memory has no multicast address")
        self.buf.zero_()
        b = self.buf
        self.ws = b[off_ws:off_ws + ws_bytes]
        self.sums = b[off_sums:off_sums + B * K * D * 4].view(torch.float32).view(B, K, D)
        self.counts = b[off_counts:off_counts + B * K * 4].view(torch.int32).view(B, K)
        self.centroids = b[off_c:off_c + B * K * D * es].view(x_local.dtype).view(B, K, D)
        self.shift = b[off_shift:off_shift + 8].view(torch.float32)
        self.bar = b[off_bar:off_bar + 16]
        self.mc_ws, self.mc_sums, self.mc_counts = mc + off_ws, mc + off_sums, mc + off_counts
        self.mc_c, self.mc_shift, self.mc_bar = mc + off_c, mc + off_shift, mc + off_bar
        self.epoch = 0  # steps run (the barrier words count arrivals per step)
        self.state = LloydState(x_local, K, ws=self.ws, sums=self.sums, counts=self.counts)
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        self.world = world
        self.rows = shard_bounds(B * K, world, rank)
        self.dims = (B, K, D, code)
        self._barrier()

    def _barrier(self) -> None:
        self.handle.barrier(channel=0, timeout_ms=20000)

    def release(self) -> None:
        """Ends the symmetric-memory use: every rank passes a last barrier with
        no kernel of this object in flight before the buffer can be freed."""
        self.wait_previous()
        self._barrier()
        torch.cuda.synchronize(self.buf.device)

    def set_centroids(self, c: torch.Tensor) -> None:
        # the other ranks' last finalize may still be writing into these buffers
        self.wait_previous()
        self.centroids.copy_(c)
        self.state.set_centroids(self.centroids)

    def reduce_finalize(self, it: int, want_shift: bool) -> None:
        """This rank's slice of the centroid rows: the ranks' sums and counts summed
        through the NVSwitch, new rows written to every rank (between two barriers)."""
        from ._lib import check, lib

        p = it & 1
        st = self.state
        B, K, D, code = self.dims
        with torch.cuda.device(st.device):
            check(lib.fkc_lloyd_finalize_multimem(
                self.mc_sums, self.mc_counts, self.centroids.data_ptr(), self.mc_c, self.mc_ws,
                (self.mc_shift + 4 * p) if want_shift else None,
                self.shift[1 - p:2 - p].data_ptr() if want_shift else None,
                self.rows[0], self.rows[1], B, K, D, code, st._stream()),
                "fkc_lloyd_finalize_multimem")

    def wait_previous(self) -> None:
        """Stream-ordered wait until every rank finished the previous step's finalize."""
        from ._lib import check, lib

        if self.epoch > 0:
            with torch.cuda.device(self.state.device):
                check(lib.fkc_multimem_step_wait(self.bar.data_ptr(), self.epoch, self.world,
                                                 self.state._stream()), "fkc_multimem_step_wait")

    def reduce_finalize_synced(self, it: int, want_shift: bool) -> None:
        """reduce_finalize with the step's cross-GPU barriers folded into the kernel
        (every rank arrives, waits for all, finalizes its rows, signals completion)."""
        from ._lib import check, lib

        p = it & 1
        st = self.state
        B, K, D, code = self.dims
        self.epoch += 1
        if self.rows[0] == self.rows[1]:
            raise RuntimeError("synced multicast finalize needs at least one row per rank")
        with torch.cuda.device(st.device):
            check(lib.fkc_lloyd_finalize_multimem_synced(
                self.mc_sums, self.mc_counts, self.centroids.data_ptr(), self.mc_c, self.mc_ws,
                (self.mc_shift + 4 * p) if want_shift else None,
                self.shift[1 - p:2 - p].data_ptr() if want_shift else None,
                self.rows[0], self.rows[1], B, K, D, code, self.bar.data_ptr(), self.mc_bar,
                self.epoch, self.world, st._stream()),
                "fkc_lloyd_finalize_multimem_synced")

    def step(self, it: int, want_shift: bool) -> Optional[torch.Tensor]:
        """One iteration in place on ``self.centroids``; returns the (1,) shift
        tensor when ``want_shift`` (valid once the stream reaches it). With at
        least one centroid row per rank the two barriers of the step run inside
        device code (no separate barrier launches)."""
        if self.rows[0] < self.rows[1]:
            self.wait_previous()
            self.state.local(self.centroids)
            self.reduce_finalize_synced(it, want_shift)
        else:
            self.state.local(self.centroids)
            self._barrier()
            self.reduce_finalize(it, want_shift)
            self._barrier()
        p = it & 1
        return self.shift[p:p + 1] if want_shift else None


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
    if world > 1:
        _check_shards(x_local, K, shard, group)

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
    if (shard == "N" and world > 1 and state_factory is _default_state_factory
            and multimem_enabled() and MultimemLloyd.available(x_local, group)):
        n_max = torch.tensor([n_local], device=x_local.device, dtype=torch.int64)
        dist.all_reduce(n_max, op=dist.ReduceOp.MAX, group=group)
        mm = MultimemLloyd.cached(x_local, K, int(n_max.item()), group)
        mm.set_centroids(cur)
        n_iters_run = 0
        for it in range(max_iters):
            sh = mm.step(it, need_shift)
            n_iters_run = it + 1
            if need_shift:
                s = float(sh.item())
                if verbose and dist.get_rank(group) == 0:
                    print(f"Iter {it}, center shift: {s:.6f}")
                if s < tol:
                    break
        labels = mm.state.ids.clone()
        cur = mm.centroids.clone()
        if gather:
            labels = _all_gather_var(labels, dim=1, group=group)
        return labels, cur, n_iters_run

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


def _check_shards(x_local: torch.Tensor, K: int, shard: str, group) -> None:
    """Every rank must agree on K, D, the shard mode and the unsharded extent (B for
    ``shard="N"``, N for ``shard="B"``); a mismatch raises ValueError on every rank (each
    rank sees all ranks' shapes) instead of a hang or a garbled all-reduce."""
    world = dist.get_world_size(group)
    B, N, D = (int(v) for v in x_local.shape)
    mine = torch.tensor([B, N, D, K, 0 if shard == "N" else 1], device=x_local.device,
                        dtype=torch.int64)
    alls = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(alls, mine, group=group)
    rows = [tuple(int(v) for v in t.tolist()) for t in alls]
    keep = (0, 2, 3, 4) if shard == "N" else (1, 2, 3, 4)  # what must match
    ref = rows[0]
    for r, row in enumerate(rows):
        if any(row[i] != ref[i] for i in keep):
            raise ValueError(
                f"sharded K-Means: rank {r} has (B, N, D, K, shard) = {row}, rank 0 has {ref}; "
                f"ranks must agree on " + ("B, D and K" if shard == "N" else "N, D and K"))


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
