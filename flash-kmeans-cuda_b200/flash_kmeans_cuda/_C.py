"""Drop-in for the reference's compiled ``flash_kmeans_cuda._C`` module.

Same four functions, positional/keyword names and defaults as the reference
nanobind module (``flash_kmeans_cuda/csrc/bindings.cpp:107-127``), with the
same in-place semantics:

* ``euclid_assign(x, centroids, x_sq, c_sq, out=None)`` -> (B, N) int32
* ``centroid_update_sorted(x_sorted, cluster_ids_sorted, centroid_sums, centroid_counts)``
  accumulates INTO pre-zeroed sums/counts (the reference ``_C`` does not zero)
* ``centroid_update_sorted_indexed(x, sorted_idx, cluster_ids_sorted, centroid_sums, centroid_counts)``
* ``centroid_finalize(centroid_sums, centroid_counts, old_centroids, out=None)``

Each call goes through the C-ABI of ``libfkc_b200.so`` on the current torch
stream of the input's device. Argument errors raise ``RuntimeError`` like the
reference's ``TORCH_CHECK``.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._lib import lib

_DTYPE_CODE = {
    torch.float16: _lib.FKC_DTYPE_F16,
    torch.bfloat16: _lib.FKC_DTYPE_BF16,
    torch.float32: _lib.FKC_DTYPE_F32,
}


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def dtype_code(t: torch.Tensor) -> int:
    code = _DTYPE_CODE.get(t.dtype)
    if code is None:
        raise RuntimeError(f"unsupported dtype {t.dtype} (expected float16, bfloat16 or float32)")
    return code


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Scratch buffer from torch's caching allocator (blocks are >= 512-byte aligned)."""
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def euclid_assign(
    x: torch.Tensor,
    centroids: torch.Tensor,
    x_sq: torch.Tensor,
    c_sq: torch.Tensor,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """argmin_k ||x - c_k||^2 per point; returns (B, N) int32 (bindings.cpp:43-71)."""
    _check(x.is_cuda, "x must be a CUDA tensor")
    _check(centroids.is_cuda, "centroids must be a CUDA tensor")
    _check(x.dim() == 3 and centroids.dim() == 3, "x and centroids must be 3D (B,N,D)/(B,K,D)")
    B, N, D = x.shape
    K = centroids.shape[1]
    _check(x.dtype == centroids.dtype, "x and centroids must share dtype")
    _check(centroids.shape[0] == B and centroids.shape[2] == D,
           "centroids must be (B, K, D) matching x")
    _check(x_sq.dtype == torch.float32 and c_sq.dtype == torch.float32,
           "x_sq and c_sq must be fp32")
    if out is not None:
        _check(out.dtype == torch.int32, "out must be int32")
        _check(out.dim() == 2 and out.shape[0] == B and out.shape[1] == N,
               "out must be (B, N) int32")
        ids = out
    else:
        ids = torch.empty((B, N), dtype=torch.int32, device=x.device)
    _check(x.is_contiguous() and centroids.is_contiguous() and x_sq.is_contiguous()
           and c_sq.is_contiguous() and ids.is_contiguous(), "all tensors must be contiguous")
    _check(c_sq.numel() == B * K, "c_sq must be (B, K)")
    code = dtype_code(x)
    with torch.cuda.device(x.device):
        ws_bytes = lib.fkc_assign_workspace_size(B, N, K, D, code)
        ws = workspace(ws_bytes, x.device)
        _lib.check(
            lib.fkc_assign(x.data_ptr(), centroids.data_ptr(),
                           x_sq.data_ptr() if x_sq.numel() == B * N else None,
                           c_sq.data_ptr(), ids.data_ptr(), B, N, K, D, code,
                           ws.data_ptr(), ws_bytes, stream_ptr(x.device)),
            "euclid_assign")
    return ids


def _check_update(x, ids_sorted, sums, counts, what: str):
    _check(x.is_cuda, f"{what} must be CUDA")
    _check(x.dim() == 3, f"{what} must be (B, N, D)")
    _check(ids_sorted.dtype == torch.int32, "cluster_ids must be int32")
    _check(sums.dtype == torch.float32, "centroid_sums must be fp32")
    _check(counts.dtype == torch.int32, "centroid_counts must be int32")
    _check(x.is_contiguous() and ids_sorted.is_contiguous() and sums.is_contiguous()
           and counts.is_contiguous(), "all tensors must be contiguous")
    B, N, D = x.shape
    _check(sums.dim() == 3 and sums.shape[0] == B and sums.shape[2] == D,
           "centroid_sums must be (B, K, D)")
    K = sums.shape[1]
    _check(counts.numel() == B * K, "centroid_counts must be (B, K)")
    _check(ids_sorted.numel() == B * N, "cluster_ids_sorted must be (B, N)")
    return B, N, K, D


def centroid_update_sorted(
    x_sorted: torch.Tensor,
    cluster_ids_sorted: torch.Tensor,
    centroid_sums: torch.Tensor,
    centroid_counts: torch.Tensor,
) -> None:
    """Sorted-run accumulate into pre-zeroed sums/counts (bindings.cpp:73-80)."""
    B, N, K, D = _check_update(x_sorted, cluster_ids_sorted, centroid_sums, centroid_counts,
                               "x_sorted")
    code = dtype_code(x_sorted)
    with torch.cuda.device(x_sorted.device):
        _lib.check(
            lib.fkc_update_sorted(x_sorted.data_ptr(), cluster_ids_sorted.data_ptr(),
                                  centroid_sums.data_ptr(), centroid_counts.data_ptr(),
                                  B, N, K, D, code, stream_ptr(x_sorted.device)),
            "centroid_update_sorted")


def centroid_update_sorted_indexed(
    x: torch.Tensor,
    sorted_idx: torch.Tensor,
    cluster_ids_sorted: torch.Tensor,
    centroid_sums: torch.Tensor,
    centroid_counts: torch.Tensor,
) -> None:
    """Sorted-run accumulate reading x[b, sorted_idx[b, i]] (bindings.cpp:82-90)."""
    _check(sorted_idx.dtype == torch.int32, "sorted_idx must be int32")
    B, N, K, D = _check_update(x, cluster_ids_sorted, centroid_sums, centroid_counts, "x")
    _check(sorted_idx.is_contiguous() and sorted_idx.numel() == B * N, "sorted_idx must be (B, N)")
    code = dtype_code(x)
    with torch.cuda.device(x.device):
        _lib.check(
            lib.fkc_update_sorted_indexed(x.data_ptr(), sorted_idx.data_ptr(),
                                          cluster_ids_sorted.data_ptr(), centroid_sums.data_ptr(),
                                          centroid_counts.data_ptr(), B, N, K, D, code,
                                          stream_ptr(x.device)),
            "centroid_update_sorted_indexed")


def centroid_finalize(
    centroid_sums: torch.Tensor,
    centroid_counts: torch.Tensor,
    old_centroids: torch.Tensor,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """new = counts > 0 ? sums / counts : old, cast to old's dtype (bindings.cpp:92-102)."""
    _check(centroid_sums.is_cuda, "all tensors must be CUDA")
    _check(centroid_sums.dtype == torch.float32, "sums must be fp32")
    _check(centroid_counts.dtype == torch.int32, "counts must be int32")
    new = out if out is not None else torch.empty_like(old_centroids)
    _check(old_centroids.dtype == new.dtype, "old and new centroids must share dtype")
    _check(centroid_sums.is_contiguous() and centroid_counts.is_contiguous()
           and old_centroids.is_contiguous() and new.is_contiguous(),
           "all tensors must be contiguous")
    _check(centroid_sums.dim() == 3, "sums must be (B, K, D)")
    B, K, D = centroid_sums.shape
    _check(old_centroids.numel() == B * K * D and new.numel() == B * K * D,
           "old/new centroids must be (B, K, D)")
    _check(centroid_counts.numel() == B * K, "counts must be (B, K)")
    code = dtype_code(old_centroids)
    with torch.cuda.device(centroid_sums.device):
        _lib.check(
            lib.fkc_finalize(centroid_sums.data_ptr(), centroid_counts.data_ptr(),
                             old_centroids.data_ptr(), new.data_ptr(), None, None, B, K, D, code,
                             stream_ptr(centroid_sums.device)),
            "centroid_finalize")
    return new
