"""The CMake package (flash-kmeans-cuda_b200/cmake): a downstream project finds
flash_kmeans_cuda with find_package and links both namespaced targets, as the
reference's installed package is consumed (CMakeLists.txt:100-125). Configure
and build run on the CPU; the C consumer's host-side checks run too (no GPU
call). Running the libtorch consumer on a GPU is tests/test_cpp_api_gpu.py."""

from __future__ import annotations

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_CMAKE = os.path.join(ROOT, "flash-kmeans-cuda_b200", "cmake")
CONSUMER = os.path.join(ROOT, "tests", "cmake_consumer")


@pytest.mark.timeout(600)
def test_find_package_and_link(tmp_path):
    if shutil.which("cmake") is None:
        pytest.skip("cmake not available")
    import torch
    from torch.utils import cmake_prefix_path

    lib = os.path.join(ROOT, "flash-kmeans-cuda_b200", "flash_kmeans_cuda", "libfkc_b200.so")
    if not os.path.exists(lib):
        pytest.fail("libfkc_b200.so not built")
    build = tmp_path / "build"
    env = dict(os.environ)
    cfg = subprocess.run(
        ["cmake", "-S", CONSUMER, "-B", str(build), f"-DCMAKE_PREFIX_PATH={PKG_CMAKE};{cmake_prefix_path}",
         "-DCMAKE_BUILD_TYPE=Release", "-DCMAKE_CUDA_COMPILER=/usr/local/cuda/bin/nvcc",
         "-DCUDAToolkit_ROOT=/usr/local/cuda", f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"],
        capture_output=True, text=True, env=env)
    assert cfg.returncode == 0, (cfg.stdout + cfg.stderr)[-4000:]
    bld = subprocess.run(["cmake", "--build", str(build), "-j", "4"], capture_output=True,
                         text=True, env=env)
    assert bld.returncode == 0, (bld.stdout + bld.stderr)[-4000:]
    exe = build / "capi_consumer"
    assert exe.exists()
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "capi consumer ok" in run.stdout
    # the libtorch target exists when Torch is found (it is, in this image)
    assert (build / "api_consumer").exists()
