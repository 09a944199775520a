"""Tensor-side helpers of the Python layers over the C-ABI (``include/fkc_capi.h``).

The C-ABI dtype code of a tensor, the raw handle of a device's current PyTorch
stream (every C-ABI call takes one) and scratch buffers from PyTorch's caching
allocator (the workspaces the C-ABI asks its callers for).
"""

from __future__ import annotations

import torch

from . import _lib

_DTYPE_CODE = {
    torch.float16: _lib.FKC_DTYPE_F16,
    torch.bfloat16: _lib.FKC_DTYPE_BF16,
    torch.float32: _lib.FKC_DTYPE_F32,
}


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
