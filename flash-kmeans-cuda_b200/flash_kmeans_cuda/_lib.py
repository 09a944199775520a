"""ctypes binding of ``libfkc_b200.so`` (the C-ABI declared in ``include/fkc_capi.h``).

This module is the only place that touches the shared library. It has no
fallback: if the library is missing or fails to load, importing it raises
``ImportError`` (the reference raises ``ImportError`` when its ``_C`` extension
is missing, ``flash_kmeans_cuda/ops.py:12-19``), and every failing call raises
``RuntimeError`` carrying ``fkc_last_error()`` (the reference surfaces
``TORCH_CHECK`` failures as ``RuntimeError``).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_NAME = "libfkc_b200.so"
LIB_PATH = Path(os.environ.get("FKC_LIB_PATH", _HERE / LIB_NAME))

FKC_OK = 0
FKC_DTYPE_F16 = 0
FKC_DTYPE_BF16 = 1
FKC_DTYPE_F32 = 2

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_size = ctypes.c_size_t
c_vp = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/fkc_capi.h.
_SIGNATURES = {
    "fkc_abi_version": (c_int, []),
    "fkc_kernel_launches": (ctypes.c_uint64, []),
    "fkc_last_error": (ctypes.c_char_p, []),
    "fkc_status_string": (ctypes.c_char_p, [c_int]),
    "fkc_device_supported": (c_int, []),
    "fkc_device_status": (c_int, []),
    "fkc_selftest_wait_timeout": (c_int, [ctypes.c_uint32, c_vp]),
    "fkc_assign_workspace_size": (c_size, [c_i64, c_i64, c_i64, c_i64, c_int]),
    "fkc_assign": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_int,
                           c_vp, c_size, c_vp]),
    "fkc_assign_noalloc": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64,
                                   c_int, c_vp]),
    "fkc_update_sorted": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_int,
                                  c_vp]),
    "fkc_update_sorted_indexed": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64,
                                          c_i64, c_int, c_vp]),
    "fkc_update_workspace_size": (c_size, [c_i64, c_i64, c_i64]),
    "fkc_update": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp,
                           c_size, c_vp]),
    "fkc_finalize": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_int,
                             c_vp]),
    "fkc_lloyd_workspace_size": (c_size, [c_i64, c_i64, c_i64, c_i64, c_int]),
    "fkc_lloyd_prepare": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_size, c_vp]),
    "fkc_lloyd_set_centroids": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_size,
                                        c_vp]),
    "fkc_lloyd_assign": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_int,
                                 c_vp, c_size, c_vp]),
    "fkc_lloyd_update": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_int,
                                 c_vp, c_size, c_vp]),
    "fkc_lloyd_local": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_int,
                                c_vp, c_size, c_vp]),
    "fkc_lloyd_finalize": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64,
                                   c_int, c_vp, c_size, c_vp]),
    "fkc_lloyd_iter": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64,
                               c_i64, c_int, c_vp, c_size, c_vp]),
    "fkc_lloyd_finalize_multimem": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64,
                                            c_i64, c_i64, c_i64, c_i64, c_int, c_vp]),
    "fkc_lloyd_finalize_multimem_synced": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                   c_i64, c_i64, c_i64, c_i64, c_i64, c_int,
                                                   c_vp, c_vp, ctypes.c_uint32, c_int, c_vp]),
    "fkc_multimem_step_wait": (c_int, [c_vp, ctypes.c_uint32, c_int, c_vp]),
    "fkc_lloyd_run": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, ctypes.c_float,
                              c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_size, c_vp]),
}

EXPORTED = tuple(_SIGNATURES)


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"flash_kmeans_cuda native library not found at {LIB_PATH}. Build it with "
            "`python flash-kmeans-cuda_b200/build.py` (or __graft_entry__.build())."
        )
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as e:  # pragma: no cover - depends on the host
        raise ImportError(f"failed to load {LIB_PATH}: {e}") from e
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error() -> str:
    return (lib.fkc_last_error() or b"").decode(errors="replace")


def check(status: int, what: str) -> None:
    """Raise RuntimeError for a non-zero C-ABI status."""
    if status != FKC_OK:
        name = (lib.fkc_status_string(status) or b"?").decode()
        raise RuntimeError(f"{what}: {name}: {last_error()}")


def device_status() -> None:
    """Synchronise the current device and raise if a kernel recorded an expired wait."""
    check(lib.fkc_device_status(), "fkc_device_status")
