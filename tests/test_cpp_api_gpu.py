"""Compiles tests/cpp/api_smoke.cpp against libflash_kmeans_cuda.so (the fkc::
libtorch API) and runs it on the GPU (the reference's tests/cpp/smoke.cpp checks)."""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "flash-kmeans-cuda_b200", "flash_kmeans_cuda")


def test_cpp_api_smoke(tmp_path, cuda_device):
    import torch
    from torch.utils import cpp_extension

    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    if not os.path.exists(os.path.join(LIBDIR, "libflash_kmeans_cuda.so")):
        pytest.fail("libflash_kmeans_cuda.so not built")
    tlib = os.path.join(os.path.dirname(torch.__file__), "lib")
    exe = str(tmp_path / "api_smoke")
    cmd = ["g++", "-O1", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *[f"-I{p}" for p in cpp_extension.include_paths()], "-I/usr/local/cuda/include",
           f"-I{os.path.join(ROOT, 'include')}", os.path.join(ROOT, "tests", "cpp", "api_smoke.cpp"),
           "-o", exe, "-Wl,--no-as-needed", f"-L{LIBDIR}", "-lflash_kmeans_cuda", "-lfkc_b200",
           f"-L{tlib}", "-lc10",
           "-ltorch_cpu", "-ltorch_cuda", "-lc10_cuda", "-L/usr/local/cuda/lib64", "-lcudart",
           f"-Wl,-rpath,{LIBDIR}", f"-Wl,-rpath,{tlib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    sys.stdout.write(r.stdout)
    assert r.returncode == 0, (r.stdout + r.stderr)[-4000:]
    assert "passed" in r.stdout
