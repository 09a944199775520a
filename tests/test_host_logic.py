"""CPU tests of the host-side Python layer: argument checks with the reference's
error types (ops.py:22-27 ValueError, kmeans.py:141-142 AssertionError,
TORCH_CHECK -> RuntimeError), sharding arithmetic and the no-fallback rule."""

from __future__ import annotations

import importlib
import subprocess
import sys

import pytest
import torch


def test_public_api_matches_reference_exports():
    import flash_kmeans_cuda as f

    assert f.__version__ == "0.1.0"
    assert set(f.__all__) == {"__version__", "batch_kmeans_Euclid", "euclid_assign",
                              "centroid_update_sorted", "centroid_finalize"}
    from flash_kmeans_cuda import _C

    # a compiled extension module, like the reference's nanobind _C
    assert _C.__file__.endswith(".so")
    for name in ("euclid_assign", "centroid_update_sorted", "centroid_update_sorted_indexed",
                 "centroid_finalize"):
        assert callable(getattr(_C, name))


def test_ops_reject_cpu_tensors():
    from flash_kmeans_cuda import euclid_assign

    x = torch.randn(1, 8, 16, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        euclid_assign(x, x[:, :2], torch.zeros(1, 8))


def test_kmeans_asserts_cuda_and_rank():
    from flash_kmeans_cuda import batch_kmeans_Euclid

    with pytest.raises(AssertionError):
        batch_kmeans_Euclid(torch.randn(1, 8, 16), 2)


def test_c_module_checks_like_torch_check():
    from flash_kmeans_cuda import _C, _tensors

    x = torch.randn(1, 8, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.euclid_assign(x, x[:, :2], torch.zeros(1, 8), torch.zeros(1, 2), None)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.euclid_assign(x, x[:, :2], torch.zeros(1, 8), torch.zeros(1, 2))  # out defaults to None
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.centroid_finalize(torch.zeros(1, 2, 16), torch.zeros(1, 2, dtype=torch.int32), x[:, :2])
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.centroid_update_sorted(x, torch.zeros(1, 8, dtype=torch.int32), torch.zeros(1, 2, 16),
                                  torch.zeros(1, 2, dtype=torch.int32))
    with pytest.raises(TypeError):
        _C.euclid_assign(x, x[:, :2])  # missing arguments, as with the reference's module
    with pytest.raises(RuntimeError, match="unsupported dtype"):
        _tensors.dtype_code(torch.zeros(1, dtype=torch.float64))


@pytest.mark.parametrize("total,world", [(10, 3), (524288, 8), (7, 8), (1, 2)])
def test_shard_bounds_cover_exactly(total, world):
    from flash_kmeans_cuda.distributed import shard_bounds

    spans = [shard_bounds(total, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == total
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    sizes = [e - b for b, e in spans]
    assert max(sizes) - min(sizes) <= 1


def test_import_fails_loudly_without_library(tmp_path):
    """No silent fallback: a missing libfkc_b200.so is an ImportError."""
    code = ("import os, sys; os.environ['FKC_LIB_PATH']='/nonexistent/libfkc_b200.so';"
            f"sys.path.insert(0, {str(importlib.util.find_spec('flash_kmeans_cuda').submodule_search_locations[0] + '/..')!r});"
            "import flash_kmeans_cuda")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    assert r.returncode != 0 and "ImportError" in r.stderr


def test_nvtx_ranges_are_noops_unless_enabled(monkeypatch):
    from flash_kmeans_cuda import _trace

    monkeypatch.setattr(_trace, "ENABLED", False)
    with _trace.nvtx("x"):
        pass
    monkeypatch.setattr(_trace, "ENABLED", True)
    with _trace.nvtx("y"):  # pushes and pops a range (works without a GPU)
        pass
    with pytest.raises(ZeroDivisionError):
        with _trace.nvtx("z"):
            1 / 0  # the range is popped on the way out


def test_iteration_helpers_keep_the_reference_signatures():
    """kmeans._euclid_iter / _can_skip_x_sq_for_assign (reference kmeans.py:48-105)."""
    import inspect

    from flash_kmeans_cuda import kmeans

    sig = inspect.signature(kmeans._euclid_iter)
    assert list(sig.parameters)[:3] == ["x", "x_sq", "centroids"]
    for name in ("compute_shift", "cluster_ids_buf", "sums_buf", "counts_buf",
                 "new_centroids_buf"):
        assert sig.parameters[name].kind is inspect.Parameter.KEYWORD_ONLY
    skip = kmeans._can_skip_x_sq_for_assign
    assert skip(torch.zeros(1, 4, 128, dtype=torch.float16), 8)
    assert skip(torch.zeros(1, 4, 512, dtype=torch.bfloat16), 8)
    assert skip(torch.zeros(1, 4, 256, dtype=torch.float32), 8)
    assert skip(torch.zeros(1, 4, 384, dtype=torch.float32), 8)  # x streamed with the stages
    assert not skip(torch.zeros(1, 4, 400, dtype=torch.float32), 8)  # CUDA-core kernel
    assert not skip(torch.zeros(1, 4, 100, dtype=torch.float16), 8)  # D % 16 != 0
    assert not skip(torch.zeros(1, 4, 640, dtype=torch.float16), 8)  # D > 512
