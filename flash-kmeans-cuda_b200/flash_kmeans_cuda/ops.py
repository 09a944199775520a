"""Python op wrappers with the reference's names, arguments and errors
(``flash_kmeans_cuda/ops.py:30-129``).

``centroid_update_sorted`` keeps its name and arguments but no longer calls
``torch.sort`` + ``gather``: labels go through the library's counting sort
(``fkc_update``), which writes the permutation in a workspace and accumulates
straight from the original-order ``x``.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _C, _lib, _tensors
from ._lib import lib


def _ensure_contig(t: torch.Tensor, name: str) -> torch.Tensor:
    # Error contract of the reference (ops.py:22-27): ValueError naming the
    # argument when it is not on a CUDA device; a contiguous copy otherwise.
    if t.is_cuda:
        return t if t.is_contiguous() else t.contiguous()
    raise ValueError(f"{name} must be a CUDA tensor (got {t.device})")


def euclid_assign(
    x: torch.Tensor,
    centroids: torch.Tensor,
    x_sq: torch.Tensor,
    c_sq: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Label of the nearest centroid for every point; equal distances go to the
    lower centroid index.

    ``x`` is (B, N, D) and ``centroids`` (B, K, D), both CUDA tensors of one
    dtype (float16, bfloat16 or float32). ``x_sq`` (B, N) and ``c_sq`` (B, K)
    are float32 squared row norms; the tensor-core kernel computes its own norms
    and ignores both, the CUDA-core kernel (float32, odd D) reads them, and a
    missing ``c_sq`` is computed here. ``out``, when given, is the (B, N) int32
    tensor the labels are written into and returned; otherwise a new one is.
    """
    xs = [_ensure_contig(t, n) for t, n in ((x, "x"), (centroids, "centroids"), (x_sq, "x_sq"))]
    x, centroids, x_sq = xs[0], xs[1], xs[2].float()
    if c_sq is None:
        c_sq = centroids.float().square().sum(-1)
    return _C.euclid_assign(x, centroids, x_sq, _ensure_contig(c_sq, "c_sq").float(), out)


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
    code = _tensors.dtype_code(x)
    with torch.cuda.device(x.device):
        ws_bytes = lib.fkc_update_workspace_size(B, N, K)
        ws = _tensors.workspace(ws_bytes, x.device)
        _lib.check(
            lib.fkc_update(x.data_ptr(), cluster_ids.data_ptr(), sums_out.data_ptr(),
                           counts_out.data_ptr(), B, N, K, D, code, ws.data_ptr(), ws_bytes,
                           _tensors.stream_ptr(x.device)),
            "centroid_update_sorted")
    return sums_out, counts_out


def centroid_finalize(
    centroid_sums: torch.Tensor,
    centroid_counts: torch.Tensor,
    old_centroids: torch.Tensor,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Mean of every non-empty cluster (sums / counts, computed in fp32) in the
    dtype of ``old_centroids``; an empty cluster keeps its old centroid. Written
    into ``out`` when it is given."""
    args = [t if t.is_contiguous() else t.contiguous()
            for t in (centroid_sums, centroid_counts, old_centroids)]
    return _C.centroid_finalize(*args, out)
