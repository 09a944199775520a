"""Python op wrappers with the reference's signatures (``flash_kmeans_cuda/ops.py:30-129``).

``centroid_update_sorted`` keeps its name and arguments but no longer calls
``torch.sort`` + ``gather``: labels go through the library's counting sort
(``fkc_update``), which writes the permutation in a workspace and accumulates
straight from the original-order ``x``.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _C, _lib
from ._lib import lib


def _ensure_contig(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device})")
    if not t.is_contiguous():
        return t.contiguous()
    return t


def euclid_assign(
    x: torch.Tensor,
    centroids: torch.Tensor,
    x_sq: torch.Tensor,
    c_sq: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Assign each point to its nearest centroid (Euclidean); ties -> lowest index.

    Args:
        x: (B, N, D) fp16/bf16/fp32, CUDA.
        centroids: (B, K, D) same dtype as x.
        x_sq: (B, N) fp32 ||x||^2 (read only by the fp32 / odd-D kernel).
        c_sq: (B, K) fp32 ||c||^2; computed from ``centroids`` if None.
        out: optional (B, N) int32 output buffer.

    Returns:
        cluster_ids: (B, N) int32.
    """
    x = _ensure_contig(x, "x")
    centroids = _ensure_contig(centroids, "centroids")
    x_sq = _ensure_contig(x_sq, "x_sq").to(torch.float32)
    if c_sq is None:
        c_sq = (centroids.float() ** 2).sum(dim=-1)
    c_sq = _ensure_contig(c_sq, "c_sq").to(torch.float32)
    return _C.euclid_assign(x, centroids, x_sq, c_sq, out)


def centroid_update_sorted(
    x: torch.Tensor,
    cluster_ids: torch.Tensor,
    K: int,
    *,
    sums_out: Optional[torch.Tensor] = None,
    counts_out: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-cluster sums (B, K, D) fp32 and counts (B, K) int32 of x by label.

    Labels must lie in [0, K). ``sums_out`` / ``counts_out`` are overwritten
    (they need not be zeroed).
    """
    x = _ensure_contig(x, "x")
    cluster_ids = _ensure_contig(cluster_ids, "cluster_ids")
    if cluster_ids.dtype != torch.int32:
        cluster_ids = cluster_ids.to(torch.int32)
    B, N, D = x.shape
    if sums_out is None:
        sums_out = torch.empty((B, K, D), device=x.device, dtype=torch.float32)
    if counts_out is None:
        counts_out = torch.empty((B, K), device=x.device, dtype=torch.int32)
    if not (sums_out.is_contiguous() and counts_out.is_contiguous()):
        raise RuntimeError("sums_out and counts_out must be contiguous")
    if sums_out.numel() != B * K * D or counts_out.numel() != B * K:
        raise RuntimeError("sums_out must be (B, K, D) and counts_out (B, K)")
    code = _C.dtype_code(x)
    with torch.cuda.device(x.device):
        ws_bytes = lib.fkc_update_workspace_size(B, N, K)
        ws = _C.workspace(ws_bytes, x.device)
        _lib.check(
            lib.fkc_update(x.data_ptr(), cluster_ids.data_ptr(), sums_out.data_ptr(),
                           counts_out.data_ptr(), B, N, K, D, code, ws.data_ptr(), ws_bytes,
                           _C.stream_ptr(x.device)),
            "centroid_update_sorted")
    return sums_out, counts_out


def centroid_finalize(
    centroid_sums: torch.Tensor,
    centroid_counts: torch.Tensor,
    old_centroids: torch.Tensor,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """new[b,k] = sums[b,k] / counts[b,k] if counts > 0 else old_centroids[b,k].

    Casts back to old_centroids.dtype.
    """
    return _C.centroid_finalize(
        centroid_sums.contiguous(),
        centroid_counts.contiguous(),
        old_centroids.contiguous(),
        out,
    )
