"""CPU tests of the C-ABI boundary: libfkc_b200.so loads, exports every function
declared in include/fkc_capi.h, and rejects bad arguments on the host with the
documented status codes before touching a GPU."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "fkc_capi.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"FKC_CAPI_EXPORT\s+[\w\s\*]+?\b(fkc_\w+)\s*\(", text))


def test_header_declares_the_path():
    names = declared_functions()
    for required in ("fkc_assign", "fkc_update", "fkc_update_sorted", "fkc_update_sorted_indexed",
                     "fkc_finalize", "fkc_lloyd_iter", "fkc_lloyd_local", "fkc_lloyd_finalize",
                     "fkc_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from flash_kmeans_cuda import _lib

    raw = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in sorted(declared_functions()) if not hasattr(raw, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert set(_lib.EXPORTED) == declared_functions(), "ctypes signatures out of sync with header"


def test_status_strings_and_version():
    from flash_kmeans_cuda import _lib

    assert _lib.lib.fkc_abi_version() == 1
    assert _lib.lib.fkc_status_string(-5) == b"FKC_EWORKSPACE"
    assert _lib.lib.fkc_status_string(0) == b"FKC_OK"


@pytest.mark.parametrize("args,code,msg", [
    ((0, 1, 1, 1, 0), -1, "must be >= 1"),
    ((1, 1, 1, 1, 9), -1, "dtype"),
    ((1, 1 << 31, 1, 1, 0), -1, "int32"),
])
def test_assign_rejects_bad_dims(args, code, msg):
    from flash_kmeans_cuda import _lib

    B, N, K, D, dt = args
    st = _lib.lib.fkc_assign(1, 1, None, None, 1, B, N, K, D, dt, None, 0, None)
    assert st == code and msg in _lib.last_error()


def test_null_pointers_and_workspace_checks():
    from flash_kmeans_cuda import _lib

    L = _lib.lib
    assert L.fkc_assign(None, 1, None, None, 1, 1, 8, 2, 16, 0, None, 0, None) == -1
    assert "non-null" in _lib.last_error()
    assert L.fkc_update(1, 1, 1, 1, 1, 10, 4, 8, 0, None, 0, None) == -5
    need = L.fkc_lloyd_workspace_size(1, 10, 4, 16, 0)
    assert L.fkc_lloyd_local(1, 1, 1, 1, 1, 1, 10, 4, 16, 0, 256, need - 1, None) == -5
    assert L.fkc_lloyd_local(1, 1, 1, 1, 1, 1, 10, 4, 16, 0, 8, need, None) == -1
    assert "256-byte aligned" in _lib.last_error()


def test_workspace_sizes_are_device_independent():
    from flash_kmeans_cuda import _lib

    L = _lib.lib
    # tensor-core shapes carry the norm-extension rows (32 B per point and per centroid)
    a = L.fkc_assign_workspace_size(1, 1000, 100, 128, 0)
    assert a >= 1000 * 32 + 100 * 32
    # fp32 with D <= 384: plus the split bf16 operand rows ([hi | lo], 2 * Dp bf16 per point
    # and centroid, Dp = D rounded up to 64)
    al = lambda v: (v + 255) // 256 * 256
    assert L.fkc_assign_workspace_size(1, 1000, 100, 128, 2) == a + al(1000 * 256 * 2) + al(
        100 * 256 * 2)
    a144 = L.fkc_assign_workspace_size(1, 1000, 100, 144, 0)
    assert L.fkc_assign_workspace_size(1, 1000, 100, 144, 2) == a144 + al(1000 * 384 * 2) + al(
        100 * 384 * 2)
    a272 = L.fkc_assign_workspace_size(1, 1000, 100, 272, 0)
    assert L.fkc_assign_workspace_size(1, 1000, 100, 272, 2) == a272 + al(1000 * 640 * 2) + al(
        100 * 640 * 2)  # fp32, 256 < D <= 384: x streamed through the stages
    assert L.fkc_assign_workspace_size(1, 1000, 100, 400, 2) == 0  # fp32, D > 384: CUDA cores
    assert L.fkc_assign_workspace_size(1, 1000, 100, 512, 1) > 0   # bf16 up to D = 512
    assert L.fkc_assign_workspace_size(1, 1000, 100, 528, 1) == 0
    assert L.fkc_assign_workspace_size(1, 1000, 100, 100, 0) == 0  # D % 16 != 0
    u = L.fkc_update_workspace_size(2, 1000, 100)
    assert u >= 2 * (2 * 1000 * 4 + 2 * 100 * 4)
    assert L.fkc_lloyd_workspace_size(1, 1000, 100, 128, 0) >= (
        a + L.fkc_update_workspace_size(1, 1000, 100))


def test_device_queries_without_gpu():
    import torch

    from flash_kmeans_cuda import _lib

    if torch.cuda.is_available():
        pytest.skip("host has a GPU")
    assert _lib.lib.fkc_device_supported() == 0
    assert _lib.lib.fkc_kernel_launches() == 0


def test_noalloc_rejects_oversize_before_any_cuda_call():
    """fkc_assign_noalloc checks its static-scratch limit on the host first."""
    from flash_kmeans_cuda import _lib

    L = _lib.lib
    limit = 32 * 1024 * 1024
    assert L.fkc_assign_workspace_size(1, limit // 32 - 8192, 8192, 64, 0) == limit
    # 16-byte aligned stand-in pointers and a null ids: nothing could be launched either way
    st = L.fkc_assign_noalloc(4096, 8192, None, None, None, 1, limit // 32 - 8192 + 1, 8192, 64,
                              0, None)
    assert st == -5 and "static scratch" in _lib.last_error()
    # exactly at the limit: past the size check (no device here: -3; with one: null ids, -1)
    st = L.fkc_assign_noalloc(4096, 8192, None, None, None, 1, limit // 32 - 8192, 8192, 64,
                              0, None)
    assert st in (-1, -3) and "static scratch" not in _lib.last_error()
    # fp32 beyond the scratch falls back to the CUDA-core kernel: the limit does not apply
    st = L.fkc_assign_noalloc(None, 1, None, None, 1, 1, 1 << 24, 8192, 64, 2, None)
    assert st == -1 and "non-null" in _lib.last_error()
    st = L.fkc_assign_noalloc(None, 1, None, None, 1, 1, 1 << 24, 8192, 72, 2, None)
    assert st == -1 and "non-null" in _lib.last_error()


def test_noalloc_limit_skipped_for_cuda_core_route():
    """A call that fkc_assign routes to the CUDA-core kernel (x or centroids not 16-byte
    aligned) needs no scratch, so the size limit does not apply: the oversize call gets
    past it to fkc_assign's own argument checks (null ids here; nothing is launched)."""
    from flash_kmeans_cuda import _lib

    L = _lib.lib
    n = 1 << 24  # far beyond the 32 MiB scratch at fp16, D=64
    st = L.fkc_assign_noalloc(16 + 2, 4096, None, None, None, 1, n, 8192, 64, 0, None)
    assert st == -1 and "non-null" in _lib.last_error()
    st = L.fkc_assign_noalloc(4096, 16 + 8, None, None, None, 1, n, 8192, 64, 0, None)
    assert st == -1 and "non-null" in _lib.last_error()
    # 16-byte aligned: the tensor-core route, whose scratch need is checked first
    st = L.fkc_assign_noalloc(4096, 8192, None, None, None, 1, n, 8192, 64, 0, None)
    assert st == -5 and "static scratch" in _lib.last_error()


def test_noalloc_limit_skipped_when_forced_safe():
    """FKC_ASSIGN_FORCE_SAFE=1 (read once per process) routes every call to the CUDA-core
    kernel: no scratch, no limit (checked in a child process)."""
    import os
    import subprocess
    import sys

    pkg = str(ROOT / "flash-kmeans-cuda_b200")
    code = (
        "import sys; sys.path[:0] = [%r, %r]\n"
        "from flash_kmeans_cuda import _lib\n"
        "st = _lib.lib.fkc_assign_noalloc(4096, 8192, None, None, None, 1, 1 << 24, 8192, 64,"
        " 0, None)\n"
        "print(st, _lib.last_error())\n" % (pkg, str(ROOT)))
    env = dict(os.environ, FKC_ASSIGN_FORCE_SAFE="1")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    st, msg = out.stdout.strip().split(" ", 1)
    assert int(st) == -1 and "non-null" in msg


def test_selftest_timeout_checked_before_any_cuda_call():
    from flash_kmeans_cuda import _lib

    assert _lib.lib.fkc_selftest_wait_timeout(0, None) == -1
    assert "timeout_us" in _lib.last_error()
    assert _lib.lib.fkc_selftest_wait_timeout(20_000_000, None) == -1


def test_lloyd_entry_points_check_arguments_on_the_host():
    """Argument errors of the Lloyd entry points come back before any CUDA call."""
    from flash_kmeans_cuda import _lib

    L = _lib.lib
    # fkc_lloyd_run: negative max_iters
    st = L.fkc_lloyd_run(1, 1, 1, 1, 1, 1, None, -1, 0.0, 1, 100, 8, 16, 0, 1, 1 << 20, None)
    assert st == -1 and "max_iters" in _lib.last_error()
    # fkc_lloyd_run: null centroids
    st = L.fkc_lloyd_run(1, None, 1, 1, 1, 1, None, 5, 0.0, 1, 100, 8, 16, 0, 1, 1 << 20, None)
    assert st == -1
    # fkc_lloyd_iter without a workspace of the documented size
    need = L.fkc_lloyd_workspace_size(1, 100, 8, 16, 0)
    st = L.fkc_lloyd_iter(1, 1, 1, 1, 1, 1, None, 1, 100, 8, 16, 0, 256, need - 1, None)
    assert st == -5 and "workspace" in _lib.last_error()
    # fkc_lloyd_finalize_multimem: row slice outside [0, B*K)
    st = L.fkc_lloyd_finalize_multimem(1, 1, 1, 1, 1, None, None, 0, 17, 2, 8, 16, 0, None)
    assert st == -1 and "rows" in _lib.last_error()
    # fkc_update: workspace too small
    st = L.fkc_update(1, 1, 1, 1, 1, 100, 8, 16, 0, 256, 1, None)
    assert st == -5 and "workspace" in _lib.last_error()
    # bad dtype code
    st = L.fkc_lloyd_assign(1, 1, 1, 1, 1, 100, 8, 16, 7, 256, 1 << 20, None)
    assert st == -1 and "dtype" in _lib.last_error()


def test_fp32_workspace_grows_with_the_split_rows():
    """fp32 rows of D <= 384 add 2 * Dp bf16 per point and per centroid to the Lloyd
    workspace (the [hi | lo] split operands of the tensor-core path, Dp = D rounded up
    to 64); D > 384 does not."""
    from flash_kmeans_cuda import _lib

    L = _lib.lib
    al = lambda v: (v + 255) // 256 * 256

    f16 = L.fkc_lloyd_workspace_size(1, 5000, 300, 128, 0)
    f32 = L.fkc_lloyd_workspace_size(1, 5000, 300, 128, 2)
    # the rest of the layout is the same for both types (both rows are 64..512 bytes)
    assert f32 - f16 == al(5000 * 256 * 2) + al(300 * 256 * 2)
    f16 = L.fkc_lloyd_workspace_size(1, 5000, 300, 64, 0)
    f32 = L.fkc_lloyd_workspace_size(1, 5000, 300, 64, 2)
    assert f32 - f16 == al(5000 * 128 * 2) + al(300 * 128 * 2)
    w272_16 = L.fkc_lloyd_workspace_size(1, 5000, 300, 272, 0)
    w272_32 = L.fkc_lloyd_workspace_size(1, 5000, 300, 272, 2)
    assert w272_32 >= w272_16 + al(5000 * 640 * 2) + al(300 * 640 * 2)  # Dp = 320
    w400_16 = L.fkc_lloyd_workspace_size(1, 5000, 300, 400, 0)
    w400_32 = L.fkc_lloyd_workspace_size(1, 5000, 300, 400, 2)
    assert w400_32 < w400_16  # fp32 D=400: no tensor-core rows at all
