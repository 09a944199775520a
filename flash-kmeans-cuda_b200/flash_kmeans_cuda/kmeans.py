"""Lloyd loop for batched Euclidean K-Means (reference: ``flash_kmeans_cuda/kmeans.py:108-195``).

The iteration (``_euclid_iter``, kmeans.py:73-105: c_sq -> assign -> sort ->
accumulate -> finalize -> shift) is one C-ABI call, ``fkc_lloyd_iter``, whose
kernels all run on the current stream:

  assign (tcgen05, labels + fused label histogram) -> scan -> scatter
  -> gather-accumulate -> finalize (+ next ||c||^2 terms, + shift)

``batch_kmeans_Euclid`` runs the whole loop as one CUDA graph launch
(``fkc_lloyd_run``: a device-side while loop that also applies ``tol``), and
synchronises once, at the end, to read the number of iterations. With
``verbose=True`` it steps iteration by iteration instead, reading the shift
after each one as the reference does.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib, _tensors
from ._trace import nvtx
from ._lib import lib


class LloydState:
    """Device buffers and workspace of a Lloyd run over a fixed ``x`` (B, N, D).

    ``ids`` (B, N) int32, ``sums`` (B, K, D) fp32, ``counts`` (B, K) int32 and
    ``shift`` (1,) fp32 are overwritten by every step. ``local`` + ``finalize``
    split a step around a reduction of ``sums``/``counts`` (multi-GPU).
    """

    def __init__(self, x: torch.Tensor, n_clusters: int, *, ws: Optional[torch.Tensor] = None,
                 sums: Optional[torch.Tensor] = None, counts: Optional[torch.Tensor] = None):
        """``ws`` (uint8, 256-byte aligned, at least ``fkc_lloyd_workspace_size`` bytes),
        ``sums`` and ``counts`` may be supplied by the caller (e.g. in symmetric
        memory for the multi-GPU multicast finalize)."""
        if not x.is_contiguous():
            raise RuntimeError("x must be contiguous")
        self.x = x
        self.device = x.device
        self.B, self.N, self.D = (int(s) for s in x.shape)
        self.K = int(n_clusters)
        self.code = _tensors.dtype_code(x)
        dev = self.device
        with torch.cuda.device(dev):
            need = int(lib.fkc_lloyd_workspace_size(self.B, self.N, self.K, self.D, self.code))
            if ws is None:
                self.ws_bytes = need
                self.ws = _tensors.workspace(self.ws_bytes, dev)
            else:
                if ws.numel() < need:
                    raise RuntimeError(f"workspace needs {need} bytes (got {ws.numel()})")
                self.ws, self.ws_bytes = ws, int(ws.numel())
            self.ids = torch.empty((self.B, self.N), dtype=torch.int32, device=dev)
            self.sums = (sums if sums is not None else
                         torch.empty((self.B, self.K, self.D), dtype=torch.float32, device=dev))
            self.counts = (counts if counts is not None else
                           torch.empty((self.B, self.K), dtype=torch.int32, device=dev))
            self.shift = torch.zeros((1,), dtype=torch.float32, device=dev)
            _lib.check(lib.fkc_lloyd_prepare(x.data_ptr(), self.B, self.N, self.K, self.D,
                                             self.code, self.ws.data_ptr(), self.ws_bytes,
                                             self._stream()), "fkc_lloyd_prepare")

    def _stream(self) -> int:
        return _tensors.stream_ptr(self.device)

    def _dims(self):
        return (self.B, self.N, self.K, self.D, self.code, self.ws.data_ptr(), self.ws_bytes,
                self._stream())

    def _check_c(self, c: torch.Tensor) -> None:
        if c.dtype != self.x.dtype:
            raise RuntimeError("x and centroids must share dtype")
        if c.numel() != self.B * self.K * self.D or not c.is_contiguous() or not c.is_cuda:
            raise RuntimeError("centroids must be a contiguous CUDA (B, K, D) tensor")

    def set_centroids(self, c: torch.Tensor) -> None:
        """Declares ``c`` the centroids of the next ``local``/``step`` (initial centroids)."""
        self._check_c(c)
        with torch.cuda.device(self.device):
            _lib.check(lib.fkc_lloyd_set_centroids(c.data_ptr(), *self._dims()),
                       "fkc_lloyd_set_centroids")

    def local(self, c: torch.Tensor) -> None:
        """Assign + counting-sort update of this state's x against ``c``."""
        with nvtx("fkc.local"), torch.cuda.device(self.device):
            _lib.check(lib.fkc_lloyd_local(self.x.data_ptr(), c.data_ptr(), self.ids.data_ptr(),
                                           self.sums.data_ptr(), self.counts.data_ptr(),
                                           *self._dims()), "fkc_lloyd_local")

    def finalize(self, old: torch.Tensor, new: torch.Tensor, want_shift: bool) -> None:
        with nvtx("fkc.finalize"), torch.cuda.device(self.device):
            _lib.check(lib.fkc_lloyd_finalize(self.sums.data_ptr(), self.counts.data_ptr(),
                                              old.data_ptr(), new.data_ptr(),
                                              self.shift.data_ptr() if want_shift else None,
                                              *self._dims()), "fkc_lloyd_finalize")

    def run(self, c: torch.Tensor, max_iters: int, tol: float) -> torch.Tensor:
        """The whole loop on the device, centroids ``c`` updated in place.

        Returns the number of iterations run as a (1,) int32 device tensor.
        """
        self._check_c(c)
        n = torch.zeros((1,), dtype=torch.int32, device=self.device)
        with nvtx("fkc.run"), torch.cuda.device(self.device):
            _lib.check(lib.fkc_lloyd_run(self.x.data_ptr(), c.data_ptr(), self.ids.data_ptr(),
                                         self.sums.data_ptr(), self.counts.data_ptr(),
                                         self.shift.data_ptr(), n.data_ptr(), int(max_iters),
                                         float(tol), *self._dims()), "fkc_lloyd_run")
        return n

    def step(self, old: torch.Tensor, new: torch.Tensor, want_shift: bool) -> None:
        """One full Lloyd iteration: ids/sums/counts from ``old``, centroids into ``new``."""
        with nvtx("fkc.step"), torch.cuda.device(self.device):
            _lib.check(lib.fkc_lloyd_iter(self.x.data_ptr(), old.data_ptr(), new.data_ptr(),
                                          self.ids.data_ptr(), self.sums.data_ptr(),
                                          self.counts.data_ptr(),
                                          self.shift.data_ptr() if want_shift else None,
                                          *self._dims()), "fkc_lloyd_iter")


def _can_skip_x_sq_for_assign(x: torch.Tensor, n_clusters: int) -> bool:
    """True when the assignment of ``x`` never reads ``x_sq`` (the reference's helper of
    the same name, kmeans.py:48-70, answers it for its D=128 raw path). Here the
    tensor-core route computes its own row norms: fp16/bf16 with D % 16 == 0 and D <= 512,
    fp32 with D % 16 == 0 and D <= 384, unless FKC_ASSIGN_FORCE_SAFE=1 selects the
    CUDA-core kernel (which reads x_sq). ``n_clusters`` does not matter here."""
    del n_clusters
    import os

    if os.environ.get("FKC_ASSIGN_FORCE_SAFE", "") in ("1", "true"):
        return False
    D = int(x.shape[-1])
    if D < 16 or D % 16 != 0:
        return False
    if x.dtype in (torch.float16, torch.bfloat16):
        return D <= 512
    return x.dtype == torch.float32 and D <= 384


def _euclid_iter(
    x: torch.Tensor,
    x_sq: torch.Tensor,
    centroids: torch.Tensor,
    *,
    compute_shift: bool = True,
    cluster_ids_buf: Optional[torch.Tensor] = None,
    sums_buf: Optional[torch.Tensor] = None,
    counts_buf: Optional[torch.Tensor] = None,
    new_centroids_buf: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, Optional[torch.Tensor], torch.Tensor]:
    """One assign + update + finalize step through the public ops (the reference's
    helper of the same name and contract, kmeans.py:73-105): returns
    ``(new_centroids, shift, cluster_ids)``, ``shift`` the max over centroids of
    ||new - old|| as a 0-d fp32 tensor, or None without ``compute_shift``. The
    ``*_buf`` arguments are written in place when given. ``batch_kmeans_Euclid`` does not
    use it: its loop runs as one CUDA graph over the fused iteration."""
    from .ops import centroid_finalize, centroid_update_sorted, euclid_assign

    B, K, D = centroids.shape
    c_sq = (centroids.float() ** 2).sum(dim=-1).contiguous()
    cluster_ids = euclid_assign(x, centroids, x_sq, c_sq=c_sq, out=cluster_ids_buf)
    sums, counts = centroid_update_sorted(x, cluster_ids, K, sums_out=sums_buf,
                                          counts_out=counts_buf)
    new_centroids = centroid_finalize(sums, counts, centroids, out=new_centroids_buf)
    shift = None
    if compute_shift:
        shift = (new_centroids.float() - centroids.float()).norm(dim=-1).max()
    return new_centroids, shift, cluster_ids


def init_centroids_random(x: torch.Tensor, n_clusters: int) -> torch.Tensor:
    """K random points per batch element, drawn WITH replacement (kmeans.py:153-157)."""
    B, N, D = x.shape
    idx = torch.randint(0, N, (B, n_clusters), device=x.device)
    return torch.gather(x, dim=1, index=idx.unsqueeze(-1).expand(-1, -1, D)).contiguous()


def batch_kmeans_Euclid(
    x: torch.Tensor,
    n_clusters: int,
    max_iters: int = 100,
    tol: float = 0.0,
    init_centroids: Optional[torch.Tensor] = None,
    verbose: bool = False,
    *,
    use_heuristic: bool = True,  # accepted for API parity, ignored
) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Batched K-Means clustering using Euclidean distance.

    Drop-in replacement for ``flash_kmeans_cuda.batch_kmeans_Euclid``.

    Args:
        x: (B, N, D) fp16 / bf16 / fp32, CUDA.
        n_clusters: K.
        max_iters: maximum number of iterations.
        tol: stop when the max centroid shift falls below ``tol``; <= 0 runs
            all ``max_iters``.
        init_centroids: optional (B, K, D) initial centroids (same dtype as x).
            If None, K random points of x per batch element (with replacement).
            The tensor is not modified.
        verbose: print the per-iteration shift.
        use_heuristic: ignored.

    Returns:
        (cluster_ids (B, N) int32, centroids (B, K, D) x.dtype, n_iters_run).
        cluster_ids are the assignment against the centroids entering the last
        iteration, as in the reference.
    """
    del use_heuristic
    assert x.is_cuda, "flash_kmeans_cuda requires a CUDA input"
    assert x.dim() == 3, "x must be (B, N, D)"
    x = x.contiguous()
    B, N, D = x.shape
    if init_centroids is None:
        centroids = init_centroids_random(x, n_clusters)
    else:
        centroids = init_centroids.contiguous().clone()
    centroids = centroids.view(B, n_clusters, D)

    state = LloydState(x, n_clusters)
    state._check_c(centroids)
    if not verbose:
        n = state.run(centroids, max_iters, tol)
        return state.ids, centroids, int(n.item())
    need_shift = True
    cur, nxt = centroids, torch.empty_like(centroids)
    state.set_centroids(cur)
    n_iters_run = 0
    for it in range(max_iters):
        state.step(cur, nxt, need_shift)
        n_iters_run = it + 1
        if need_shift:
            shift = state.shift.item()
            if verbose:
                print(f"Iter {it}, center shift: {shift:.6f}")
            if shift < tol:
                cur = nxt
                break
        cur, nxt = nxt, cur
    return state.ids, cur, n_iters_run
