"""Build recipe for the native parts of flash-kmeans-cuda_b200.

Produces, next to the Python package (``flash_kmeans_cuda/``):
  * ``libfkc_b200.so``       - the CUDA kernels behind the C-ABI of
                               ``include/fkc_capi.h`` (sm_100a only);
  * ``libflash_kmeans_cuda.so`` - the libtorch ``fkc::`` API of
                               ``include/flash_kmeans_cuda/flash_kmeans_cuda.h``
                               layered on the C-ABI (optional, needs torch headers).

Usage: ``python flash-kmeans-cuda_b200/build.py [--force] [--no-torch-api]``.
nvcc cross-compiles for sm_100a without a GPU.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
OUT_DIR = PKG_ROOT / "flash_kmeans_cuda"
BUILD_DIR = PKG_ROOT / "_build"
INCLUDE = REPO_ROOT / "include"

CORE_SOURCES = ["capi.cu", "assign_tc.cu", "norm_ext.cu", "assign_simt.cu", "update.cu",
                "update_det.cu",
                "finalize.cu", "lloyd_graph.cu", "assign_noalloc.cu", "selftest.cu"]
CORE_LIB = OUT_DIR / "libfkc_b200.so"
TORCH_API_LIB = OUT_DIR / "libflash_kmeans_cuda.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler=-fPIC",
    "-Xcompiler=-fvisibility=hidden",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.rglob("*.h"))


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build_core(force: bool = False, verbose: bool = False) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    hdrs = _headers()
    objs = []
    jobs = []
    for src in CORE_SOURCES:
        s = CSRC / src
        o = BUILD_DIR / (s.stem + ".o")
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(s), "-o", str(o)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(_run, jobs))
    if force or jobs or _newer(CORE_LIB, objs):
        _run([nvcc(), *ARCH_FLAGS, "-shared", "-o", str(CORE_LIB), *map(str, objs), "-lcuda"])
    return CORE_LIB


def build_torch_api(force: bool = False) -> Path | None:
    """libtorch fkc:: API over the C-ABI (reference: flash_kmeans_cuda/csrc/api.cpp)."""
    try:
        import torch
        from torch.utils import cpp_extension
    except Exception:  # pragma: no cover - torch is part of the image
        return None
    src = CSRC / "torch_api.cpp"
    hdr = INCLUDE / "flash_kmeans_cuda" / "flash_kmeans_cuda.h"
    if not src.exists():
        return None
    if not (force or _newer(TORCH_API_LIB, [src, hdr, CORE_LIB])):
        return TORCH_API_LIB
    inc = cpp_extension.include_paths()
    cuda_inc = "/usr/local/cuda/include"
    libdir = Path(torch.__file__).parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [
        "g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DFKC_BUILD_SHARED",
        *[f"-I{p}" for p in inc], f"-I{cuda_inc}", f"-I{INCLUDE}",
        str(src), "-o", str(TORCH_API_LIB),
        f"-L{libdir}", "-lc10", "-ltorch_cpu", "-lc10_cuda", "-ltorch_cuda",
        f"-L{OUT_DIR}", "-lfkc_b200",
        "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{libdir}",
    ]
    _run(cmd)
    return TORCH_API_LIB


def build_py_module(force: bool = False) -> Path | None:
    """The compiled ``flash_kmeans_cuda._C`` module (reference: flash_kmeans_cuda/csrc/bindings.cpp),
    a PyTorch extension over the C-ABI of libfkc_b200.so."""
    try:
        import sysconfig

        import torch
        from torch.utils import cpp_extension
    except Exception:  # pragma: no cover - torch is part of the image
        return None
    src = CSRC / "py_C.cpp"
    out = OUT_DIR / ("_C" + sysconfig.get_config_var("EXT_SUFFIX"))
    if not (force or _newer(out, [src, INCLUDE / "fkc_capi.h", CORE_LIB])):
        return out
    libdir = Path(torch.__file__).parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [
        "g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        *[f"-I{p}" for p in cpp_extension.include_paths()],
        f"-I{sysconfig.get_paths()['include']}", "-I/usr/local/cuda/include", f"-I{INCLUDE}",
        str(src), "-o", str(out),
        f"-L{libdir}", "-lc10", "-ltorch_cpu", "-ltorch", "-ltorch_python", "-lc10_cuda",
        "-ltorch_cuda", f"-L{OUT_DIR}", "-lfkc_b200",
        "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{libdir}",
    ]
    _run(cmd)
    return out


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--no-torch-api", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args(argv)
    lib = build_core(force=args.force, verbose=args.ptxas_verbose)
    print(f"built {lib}")
    if not args.no_torch_api:
        t = build_torch_api(force=args.force)
        if t is not None:
            print(f"built {t}")
        m = build_py_module(force=args.force)
        if m is not None:
            print(f"built {m}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
