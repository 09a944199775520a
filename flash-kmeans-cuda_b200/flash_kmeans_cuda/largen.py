"""K-Means over host-resident points streamed through one or more GPUs.

For x that does not fit in device memory: the points stay in (pinned) host
memory as an (N, D) tensor and every Lloyd iteration streams them through the
GPUs in blocks. This follows the design the reference's documentation gives
for the upstream ``kmeans_largeN`` (``docs/development_notes.md``, "Large-N
streaming with multi-GPU"; its source is not part of the reference):

* the N rows are cut into contiguous blocks, dealt to the GPUs in contiguous
  runs (one host thread per GPU);
* each GPU runs a double-buffered pipeline on two streams: the host-to-device
  copy of block j+1 overlaps the assignment and accumulation of block j, and
  the labels of a block go back to host memory while the next one computes;
* the per-GPU partial sums and counts (fp32 / int32, K x D) are gathered onto
  the first GPU with peer copies and added there (no collective library: the
  partials are a few MB), the first GPU finalizes (empty clusters keep their
  old centroid, as the reference does) and the next iteration copies the new
  centroids to every GPU;
* batched input (B > 1) is not supported on this path, as upstream.

Per block the work is this library's own kernels through the C-ABI:
``fkc_lloyd_prepare`` (per-row norm terms of the block), ``fkc_lloyd_local``
(tcgen05 assignment with the fused histogram, counting sort, gather-accumulate)
and, once per iteration, ``fkc_finalize`` with the shift.
"""

from __future__ import annotations

import threading
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib, _tensors
from ._lib import lib

_DEFAULT_BLOCK_BYTES = 256 << 20


def plan_blocks(n: int, block_rows: int, n_devices: int) -> List[List[Tuple[int, int]]]:
    """Row ranges [r0, r1) of each device: blocks of ``block_rows`` rows (the last one may
    be shorter), dealt in contiguous runs whose sizes differ by at most one block."""
    if n < 1 or block_rows < 1 or n_devices < 1:
        raise ValueError("n, block_rows and n_devices must be >= 1")
    blocks = [(r, min(r + block_rows, n)) for r in range(0, n, block_rows)]
    per, extra = divmod(len(blocks), n_devices)
    out, i = [], 0
    for d in range(n_devices):
        take = per + (1 if d < extra else 0)
        out.append(blocks[i:i + take])
        i += take
    return out


class _Worker:
    """One GPU's buffers and streams for the streamed Lloyd pass."""

    def __init__(self, device: torch.device, block_rows: int, K: int, D: int,
                 dtype: torch.dtype):
        self.device = device
        self.block_rows, self.K, self.D = block_rows, K, D
        self.code = _tensors.dtype_code(torch.empty((), dtype=dtype))
        with torch.cuda.device(device):
            self.ws_bytes = int(lib.fkc_lloyd_workspace_size(1, block_rows, K, D, self.code))
            self.ws = _tensors.workspace(self.ws_bytes, device)
            self.x = [torch.empty((1, block_rows, D), dtype=dtype, device=device)
                      for _ in range(2)]
            self.ids = [torch.empty((1, block_rows), dtype=torch.int32, device=device)
                        for _ in range(2)]
            self.c = torch.empty((1, K, D), dtype=dtype, device=device)
            self.sums_blk = torch.empty((1, K, D), dtype=torch.float32, device=device)
            self.counts_blk = torch.empty((1, K), dtype=torch.int32, device=device)
            self.sums = torch.empty((1, K, D), dtype=torch.float32, device=device)
            self.counts = torch.empty((1, K), dtype=torch.int32, device=device)
            self.copy_stream = torch.cuda.Stream(device)
            self.compute_stream = torch.cuda.Stream(device)
            self.copied = [torch.cuda.Event() for _ in range(2)]
            self.computed = [torch.cuda.Event() for _ in range(2)]
            self.freed = [torch.cuda.Event() for _ in range(2)]
        self.error: Optional[BaseException] = None

    def _call(self, fn, *args, what: str) -> None:
        _lib.check(fn(*args), what)

    def run(self, x_host: torch.Tensor, ids_host: Optional[torch.Tensor],
            blocks: Sequence[Tuple[int, int]], centroids: torch.Tensor,
            accumulate: bool) -> None:
        """Streams ``blocks`` of ``x_host``: labels into ``ids_host`` (if given) and, with
        ``accumulate``, the sums/counts of the blocks into ``self.sums``/``self.counts``."""
        try:
            self._run(x_host, ids_host, blocks, centroids, accumulate)
        except BaseException as e:  # re-raised by the caller's thread
            self.error = e

    def _run(self, x_host, ids_host, blocks, centroids, accumulate):
        dev, K, D, code = self.device, self.K, self.D, self.code
        with torch.cuda.device(dev):
            cs, ps = self.compute_stream, self.copy_stream
            cs_ptr, ps_ptr = cs.cuda_stream, ps.cuda_stream
            with torch.cuda.stream(cs):
                self.c.copy_(centroids.view(1, K, D), non_blocking=True)
                if accumulate:
                    self.sums.zero_()
                    self.counts.zero_()
            ws, wsb = self.ws.data_ptr(), self.ws_bytes
            # Centroid terms (norm rows) of this iteration's centroids, in the part of the
            # workspace that does not depend on the block's row count.
            self._call(lib.fkc_lloyd_set_centroids, self.c.data_ptr(), 1, self.block_rows, K, D,
                       code, ws, wsb, cs_ptr, what="fkc_lloyd_set_centroids")
            def load(j):
                # copy stream: block j into buffer j % 2 once block j-2 has released it
                r0, r1 = blocks[j]
                bj = j % 2
                if j >= 2:
                    ps.wait_event(self.freed[bj])
                with torch.cuda.stream(ps):
                    self.x[bj][0, :r1 - r0].copy_(x_host[r0:r1], non_blocking=True)
                    self.copied[bj].record(ps)

            if blocks:
                load(0)
            for j, (r0, r1) in enumerate(blocks):
                b, n = j % 2, r1 - r0
                xb, ib = self.x[b], self.ids[b]
                if j + 1 < len(blocks):
                    load(j + 1)  # overlaps the compute of block j
                # compute stream: norm terms, assignment + accumulation of block j
                cs.wait_event(self.copied[b])
                self._call(lib.fkc_lloyd_prepare, xb.data_ptr(), 1, n, K, D, code, ws, wsb,
                           cs_ptr, what="fkc_lloyd_prepare")
                if accumulate:
                    self._call(lib.fkc_lloyd_local, xb.data_ptr(), self.c.data_ptr(),
                               ib.data_ptr(), self.sums_blk.data_ptr(),
                               self.counts_blk.data_ptr(), 1, n, K, D, code, ws, wsb, cs_ptr,
                               what="fkc_lloyd_local")
                    with torch.cuda.stream(cs):
                        self.sums.add_(self.sums_blk)
                        self.counts.add_(self.counts_blk)
                else:
                    self._call(lib.fkc_lloyd_assign, xb.data_ptr(), self.c.data_ptr(),
                               ib.data_ptr(), self.counts_blk.data_ptr(), 1, n, K, D, code,
                               ws, wsb, cs_ptr, what="fkc_lloyd_assign")
                self.computed[b].record(cs)
                # copy stream: labels of block j back to the host; then buffer b is free
                ps.wait_event(self.computed[b])
                if ids_host is not None:
                    with torch.cuda.stream(ps):
                        ids_host[r0:r1].copy_(ib[0, :n], non_blocking=True)
                self.freed[b].record(ps)
            ps.synchronize()
            cs.synchronize()


def _resolve_devices(devices) -> List[torch.device]:
    if not torch.cuda.is_available():
        raise RuntimeError("kmeans_largeN needs a CUDA device")
    if devices is None:
        return [torch.device("cuda", i) for i in range(torch.cuda.device_count())]
    if isinstance(devices, (int, str, torch.device)):
        devices = [devices]
    out = []
    for d in devices:
        d = torch.device("cuda", d) if isinstance(d, int) else torch.device(d)
        if d.type != "cuda":
            raise ValueError(f"devices must be CUDA devices (got {d})")
        out.append(torch.device("cuda", d.index if d.index is not None else 0))
    if not out:
        raise ValueError("devices is empty")
    return out


def _check_host_x(x: torch.Tensor) -> None:
    if x.is_cuda:
        raise ValueError("kmeans_largeN streams host-resident x: pass a CPU tensor "
                         "(device-resident x goes to batch_kmeans_Euclid)")
    if x.dim() != 2:
        raise ValueError("x must be (N, D): batched input is not supported on the streamed path")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError(f"unsupported dtype {x.dtype}")


def _pinned(x: torch.Tensor) -> torch.Tensor:
    x = x.contiguous()
    return x if x.is_pinned() else x.pin_memory()


class _Pool:
    def __init__(self, devs, block_rows, K, D, dtype):
        self.workers = [_Worker(d, block_rows, K, D, dtype) for d in devs]

    def run(self, plan, x_host, ids_host, centroids_per_dev, accumulate):
        threads = []
        for w, blocks, c in zip(self.workers, plan, centroids_per_dev):
            w.error = None
            t = threading.Thread(target=w.run, args=(x_host, ids_host, blocks, c, accumulate))
            t.start()
            threads.append(t)
        for t in threads:
            t.join()
        for w in self.workers:
            if w.error is not None:
                raise w.error


def kmeans_largeN(
    x: torch.Tensor,
    n_clusters: int,
    max_iters: int = 100,
    tol: float = 0.0,
    init_centroids: Optional[torch.Tensor] = None,
    devices=None,
    block_rows: Optional[int] = None,
    verbose: bool = False,
) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Lloyd K-Means of host-resident ``x`` (N, D) streamed through ``devices``.

    Returns ``(ids (N,) int32 on the host (pinned), centroids (K, D) of x's dtype on the
    first device, iterations run)``. ``devices=None`` uses every visible GPU; a single
    device runs the same pipeline without the reduction. ``init_centroids`` (K, D) (any
    device); default: K rows of x drawn with replacement (kmeans.py:153-157). Iterations
    stop after ``max_iters`` or once the centroid shift is below ``tol`` (> 0).
    """
    _check_host_x(x)
    N, D = (int(s) for s in x.shape)
    K = int(n_clusters)
    if K < 1 or max_iters < 0:
        raise ValueError("n_clusters must be >= 1 and max_iters >= 0")
    if N >= 2 ** 31:
        raise ValueError("N must be < 2^31")
    devs = _resolve_devices(devices)
    es = x.element_size()
    if block_rows is None:
        block_rows = max(1, _DEFAULT_BLOCK_BYTES // (D * es))
    block_rows = int(min(block_rows, N))
    x_host = _pinned(x)
    dev0 = devs[0]
    if init_centroids is None:
        idx = torch.randint(0, N, (K,))
        c = x_host[idx].to(dev0)
    else:
        if tuple(init_centroids.shape) != (K, D) or init_centroids.dtype != x.dtype:
            raise ValueError("init_centroids must be (K, D) of x's dtype")
        c = init_centroids.to(dev0).contiguous().clone()
    c = c.contiguous()
    plan = plan_blocks(N, block_rows, len(devs))
    pool = _Pool(devs, block_rows, K, D, x.dtype)
    ids_host = torch.empty((N,), dtype=torch.int32).pin_memory()
    code = _tensors.dtype_code(x)
    c_next = torch.empty_like(c)
    shift = torch.zeros((1,), dtype=torch.float32, device=dev0)
    sums = torch.empty((1, K, D), dtype=torch.float32, device=dev0)
    counts = torch.empty((1, K), dtype=torch.int32, device=dev0)
    n_run = 0
    torch.cuda.synchronize(dev0)  # c is read by the workers' own streams
    for it in range(max_iters):
        pool.run(plan, x_host, ids_host, [c] * len(devs), accumulate=True)
        with torch.cuda.device(dev0):
            # gather-reduce of the per-GPU partials onto the first GPU (peer copies)
            sums.copy_(pool.workers[0].sums)
            counts.copy_(pool.workers[0].counts)
            for w in pool.workers[1:]:
                sums.add_(w.sums.to(dev0, non_blocking=True))
                counts.add_(w.counts.to(dev0, non_blocking=True))
            _lib.check(lib.fkc_finalize(sums.data_ptr(), counts.data_ptr(), c.data_ptr(),
                                        c_next.data_ptr(), None, shift.data_ptr(), 1, K, D,
                                        code, _tensors.stream_ptr(dev0)), "fkc_finalize")
            torch.cuda.synchronize(dev0)
        c, c_next = c_next, c
        n_run = it + 1
        if verbose or tol > 0:
            s = float(shift.item())
            if verbose:
                print(f"Iter {it}, center shift: {s:.6f}")
            if tol > 0 and s < tol:
                break
    return ids_host, c.view(K, D), n_run


def kmeans_largeN_assign(
    x: torch.Tensor,
    centroids: torch.Tensor,
    devices=None,
    block_rows: Optional[int] = None,
) -> torch.Tensor:
    """Labels (N,) int32 (host, pinned) of host-resident ``x`` (N, D) against ``centroids``
    (K, D), streamed through ``devices`` like ``kmeans_largeN``."""
    _check_host_x(x)
    N, D = (int(s) for s in x.shape)
    if centroids.dim() != 2 or int(centroids.shape[1]) != D or centroids.dtype != x.dtype:
        raise ValueError("centroids must be (K, D) of x's dtype")
    K = int(centroids.shape[0])
    devs = _resolve_devices(devices)
    if block_rows is None:
        block_rows = max(1, _DEFAULT_BLOCK_BYTES // (D * x.element_size()))
    block_rows = int(min(block_rows, N))
    x_host = _pinned(x)
    plan = plan_blocks(N, block_rows, len(devs))
    pool = _Pool(devs, block_rows, K, D, x.dtype)
    ids_host = torch.empty((N,), dtype=torch.int32).pin_memory()
    per_dev = [centroids.to(d).contiguous() for d in devs]
    for d in devs:
        torch.cuda.synchronize(d)
    pool.run(plan, x_host, ids_host, per_dev, accumulate=False)
    return ids_host


_OVERLAP_MIN_WORK = 10 ** 11


def batch_kmeans_Euclid_host(
    x: torch.Tensor,
    n_clusters: int,
    max_iters: int = 100,
    tol: float = 0.0,
    init_centroids: Optional[torch.Tensor] = None,
    device=None,
    block_rows: int = 65536,
    overlap: Optional[bool] = None,
) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """``batch_kmeans_Euclid`` for x (B, N, D) in pinned host memory, on one GPU.

    Same results contract as ``batch_kmeans_Euclid`` (labels of the last
    assignment, final centroids, iterations run; the outputs and the device copy
    of x stay on ``device``, default the current one), with the host-to-device
    copy of x overlapped with the first iteration: x is copied on a side stream
    in blocks of ``block_rows`` rows straight into its resident device tensor,
    and every block is assigned and accumulated as soon as it has landed
    (``fkc_lloyd_prepare`` + ``fkc_lloyd_local`` of the block, partial sums and
    counts added up). The first iteration's finalize follows the last block;
    the remaining iterations run on the resident x as one CUDA-graph launch
    (``fkc_lloyd_run``). The first iteration's sums are added up per block, so
    its centroids can differ from a one-pass update in the last bits of the
    fp32 sums (labels of the first iteration are the same).
    With ``overlap=None``, problems with B*N*K*D below ``_OVERLAP_MIN_WORK`` (about 60 us of assignment
    per 65,536-row block at D = 128) copy x first and call
    ``batch_kmeans_Euclid``: the per-block launches would cost more than the
    overlap saves (measured on B200: c2, B=1 N=131072 K=2048 D=128, 0.170
    against 0.165 ms/iter; c3, N=524288 K=8192, 1.152 against 1.218);
    ``overlap=True`` / ``False`` force one route.
    ``init_centroids`` (B, K, D) of x's dtype, any device; default: K rows of x
    per batch element drawn with replacement (kmeans.py:153-157).
    """
    from .kmeans import LloydState

    if x.is_cuda or x.dim() != 3:
        raise ValueError("x must be a (B, N, D) tensor in host memory")
    B, N, D = (int(s) for s in x.shape)
    K = int(n_clusters)
    if K < 1 or max_iters < 0 or block_rows < 1:
        raise ValueError("n_clusters and block_rows must be >= 1 and max_iters >= 0")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else \
        torch.device(device)
    x_host = _pinned(x.contiguous())
    code = _tensors.dtype_code(x_host)
    if init_centroids is None:
        idx = torch.randint(0, N, (B, K))
        c0 = torch.gather(x_host, 1, idx.unsqueeze(-1).expand(-1, -1, D))
    else:
        if tuple(init_centroids.shape) != (B, K, D) or init_centroids.dtype != x.dtype:
            raise ValueError("init_centroids must be (B, K, D) of x's dtype")
        c0 = init_centroids
    with torch.cuda.device(dev):
        cs = torch.cuda.current_stream(dev)
        ps = torch.cuda.Stream(dev)
        xd = torch.empty((B, N, D), dtype=x.dtype, device=dev)
        c = c0.to(dev, non_blocking=True).contiguous().clone()
        if overlap is None:
            overlap = B * N * K * D >= _OVERLAP_MIN_WORK
        if max_iters == 0 or not overlap:
            from .kmeans import batch_kmeans_Euclid

            xd.copy_(x_host, non_blocking=True)
            return batch_kmeans_Euclid(xd, K, max_iters=max_iters, tol=tol, init_centroids=c)
        rows = min(block_rows, N)
        blocks = [(b, r0, min(r0 + rows, N)) for b in range(B) for r0 in range(0, N, rows)]
        ws_bytes = int(lib.fkc_lloyd_workspace_size(1, rows, K, D, code))
        ws = _tensors.workspace(ws_bytes, dev)
        ids = torch.empty((B, N), dtype=torch.int32, device=dev)
        sums = torch.zeros((B, K, D), dtype=torch.float32, device=dev)
        counts = torch.zeros((B, K), dtype=torch.int32, device=dev)
        sums_blk = torch.empty((1, K, D), dtype=torch.float32, device=dev)
        counts_blk = torch.empty((1, K), dtype=torch.int32, device=dev)
        landed = [torch.cuda.Event() for _ in blocks]
        # copies: all blocks back to back on the side stream, into x's final place
        ps.wait_stream(cs)
        with torch.cuda.stream(ps):
            for e, (b, r0, r1) in zip(landed, blocks):
                xd[b, r0:r1].copy_(x_host[b, r0:r1], non_blocking=True)
                e.record(ps)
        st = cs.cuda_stream
        cur_b = -1
        for e, (b, r0, r1) in zip(landed, blocks):
            cs.wait_event(e)
            n = r1 - r0
            xb = xd[b, r0:r1]
            cb = c[b]
            args = (1, n, K, D, code, ws.data_ptr(), ws_bytes, st)
            _lib.check(lib.fkc_lloyd_prepare(xb.data_ptr(), *args), "fkc_lloyd_prepare")
            if b != cur_b or n != rows:
                # centroid terms of batch element b (N-independent part of the workspace)
                _lib.check(lib.fkc_lloyd_set_centroids(cb.data_ptr(), *args),
                           "fkc_lloyd_set_centroids")
                cur_b = b
            _lib.check(lib.fkc_lloyd_local(xb.data_ptr(), cb.data_ptr(),
                                           ids[b, r0:r1].data_ptr(), sums_blk.data_ptr(),
                                           counts_blk.data_ptr(), *args), "fkc_lloyd_local")
            sums[b].add_(sums_blk[0])
            counts[b].add_(counts_blk[0])
        # first iteration's finalize: new centroids and the shift
        c1 = torch.empty_like(c)
        shift = torch.zeros((1,), dtype=torch.float32, device=dev)
        _lib.check(lib.fkc_finalize(sums.data_ptr(), counts.data_ptr(), c.data_ptr(),
                                    c1.data_ptr(), None, shift.data_ptr(), B, K, D, code, st),
                   "fkc_finalize")
        state = LloydState(xd, K)
        state.ids.copy_(ids)
        if max_iters == 1 or (tol > 0 and float(shift.item()) < tol):
            return state.ids, c1, 1
        n_more = state.run(c1, max_iters - 1, tol)
        return state.ids, c1, 1 + int(n_more.item())
