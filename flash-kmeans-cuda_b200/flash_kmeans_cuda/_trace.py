"""Optional NVTX ranges around the host-side phases (assign+update, finalize, whole
steps, all-reduce, streamed blocks), for Nsight timelines and ncu NVTX filtering.

Off unless FKC_NVTX=1 in the environment when the package is imported; when off, ``nvtx``
is a no-op context manager and nothing is pushed."""

from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("FKC_NVTX", "0") == "1"


@contextlib.contextmanager
def nvtx(name: str):
    if not ENABLED:
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
