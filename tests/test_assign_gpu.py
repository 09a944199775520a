"""Assignment parity on the GPU, through the C-ABI, against the float64 oracle.

Bar (per config): labels identical wherever the top-2 distance gap exceeds
1e-3 * ||x||^2, and >= 99.9% identical overall. Shapes cover the reference's
edge cases (tests/test_shapes.py:14-20, tests/test_persistent.py:26-118,
tests/test_mma_optin.py:35-42): tail tiles, K = 1, K around chunk widths,
D = 16..512, B > 1.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle.lloyd as orc
from _data import iid, mixture, subset_init, to_np

pytestmark = pytest.mark.gpu

GAP = 1e-3
MIN_AGREE = 0.999


def _assign_gpu(x, c, c_sq=None):
    from flash_kmeans_cuda import _C

    xd, cd = x.cuda(), c.cuda()
    if c_sq is None:
        c_sq = (cd.float() ** 2).sum(-1)
    x_sq = (xd.float() ** 2).sum(-1)
    ids = _C.euclid_assign(xd, cd, x_sq.contiguous(), c_sq.contiguous(), None)
    torch.cuda.synchronize()
    return ids.cpu().numpy()


def _check(ids, ref: orc.AssignResult, tag=""):
    mask = ref.gap_mask(GAP)
    bad = (ids != ref.ids) & mask
    agree = float((ids == ref.ids).mean())
    assert not bad.any(), f"{tag}: {int(bad.sum())} label mismatches above the gap threshold"
    assert agree >= MIN_AGREE, f"{tag}: agreement {agree:.5f} < {MIN_AGREE}"


SHAPES = [
    (1, 1024, 64, 64),
    (1, 4096, 128, 128),
    (2, 8192, 256, 128),
    (1, 100, 8, 64),
    (1, 257, 16, 128),
    (1, 1024, 1, 64),
    (1, 1024, 63, 64),
    (1, 1024, 65, 64),
    (1, 1024, 255, 128),
    (1, 1024, 257, 128),
    (1, 1024, 32, 256),
    (3, 2048, 32, 64),
    (1, 1000, 300, 96),
    (1, 777, 513, 192),
    (1, 513, 129, 16),
    (1, 2048, 4096, 128),
    (1, 1500, 300, 320),    # D > 256: CTA-pair kernel, 64 centroid rows per CTA
    (2, 3000, 700, 384),
    (1, 1200, 200, 400),    # D > 384: x streamed with the centroid stages (last block partial)
    (1, 2000, 500, 448),
    (2, 1700, 333, 512),
    (1, 70000, 600, 512),   # more row tiles than SMs (two x buffers in turn)
]


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("B,N,K,D", SHAPES)
def test_assign_matches_oracle(cuda_device, dtype, B, N, K, D):
    x = iid(B, N, D, seed=B * 7 + N + K + D, dtype=dtype)
    c = subset_init(x, K, seed=1) if K <= N else iid(B, K, D, seed=3, dtype=dtype)
    ids = _assign_gpu(x, c)
    ref = orc.assign(to_np(x), to_np(c))
    _check(ids, ref, f"{dtype} {B}x{N}x{K}x{D}")


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_assign_mixture_large_k(cuda_device, dtype):
    x = mixture(1, 16384, 128, 2048, seed=5, dtype=dtype)
    c = subset_init(x, 2048, seed=6)
    ids = _assign_gpu(x, c)
    _check(ids, orc.assign(to_np(x), to_np(c)), f"mixture {dtype}")


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_identity_centroids(cuda_device, dtype):
    """Rows 0..K-1 are the centroids: each must map to itself (test_persistent.py:35-48)."""
    x = iid(1, 4096, 128, seed=7, dtype=dtype)
    K = 300
    c = x[:, :K].contiguous()
    ids = _assign_gpu(x, c)
    assert (ids[0, :K] == np.arange(K)).all()


def test_duplicate_centroids_lowest_index(cuda_device):
    """Exact ties (duplicated centroids) resolve to the lowest index (assign_common.cuh:20-28)."""
    x = iid(1, 2048, 128, seed=8, dtype="float16")
    base = subset_init(x, 100, seed=9)
    # centroid k and k + 100 and k + 300 are identical; 200..299 are far away
    far = base + 50.0
    c = torch.cat([base, base, far.to(base.dtype), base], dim=1).contiguous()
    ids = _assign_gpu(x, c)
    assert ids.max() < 100, "a duplicate with a higher index won an exact tie"
    ref = orc.assign(to_np(x), to_np(c))
    _check(ids, ref, "duplicates")


def test_determinism(cuda_device):
    x = iid(1, 8192, 128, seed=10, dtype="float16")
    c = subset_init(x, 1000, seed=11)
    a = _assign_gpu(x, c)
    b = _assign_gpu(x, c)
    assert np.array_equal(a, b)


def test_user_c_sq_is_used(cuda_device):
    """The raw-distance path scores with the caller's c_sq (assign_sm80.cu:437-441)."""
    x = iid(1, 1024, 64, seed=12, dtype="float16")
    c = subset_init(x, 64, seed=13)
    cd = c.cuda()
    c_sq = (cd.float() ** 2).sum(-1)
    c_sq[0, 5] -= 1e6  # makes centroid 5 the nearest for every point
    ids = _assign_gpu(x, c, c_sq)
    assert (ids == 5).all()


@pytest.mark.parametrize("B,N,K,D", [(1, 1000, 37, 7), (2, 513, 65, 33), (1, 2048, 64, 64)])
def test_fp32_and_odd_d(cuda_device, B, N, K, D):
    """fp32 / odd D take the CUDA-core kernel (reference safe path semantics)."""
    for dtype in (["float32", "float16"] if D % 16 else ["float32"]):
        x = iid(B, N, D, seed=N + K, dtype=dtype)
        c = subset_init(x, K, seed=2)
        ids = _assign_gpu(x, c)
        _check(ids, orc.assign(to_np(x), to_np(c)), f"{dtype} D={D}")


@pytest.mark.parametrize("B,N,K,D", [(1, 3000, 500, 144), (2, 2000, 300, 192),
                                     (1, 2500, 700, 256), (1, 3000, 260, 272),
                                     (2, 1500, 333, 320), (1, 5000, 1000, 384),
                                     (1, 1000, 100, 400)])
def test_fp32_tensor_core_widths(cuda_device, B, N, K, D):
    """fp32 up to D = 384 runs on the tensor cores as split bf16 rows ([hi | lo] halves,
    hi.hi + hi.lo + lo.hi K steps; above D = 256 x is streamed through the centroid
    stages); D = 400 keeps the CUDA-core kernel. The assignment workspace is non-zero
    exactly for the tensor-core route."""
    from flash_kmeans_cuda import _lib

    x = mixture(B, N, D, max(K // 4, 2), seed=N + D, dtype="float32")
    c = subset_init(x, K, seed=4)
    assert (_lib.lib.fkc_assign_workspace_size(B, N, K, D, 2) > 0) == (D <= 384)
    ids = _assign_gpu(x, c)
    _check(ids, orc.assign(to_np(x), to_np(c)), f"float32 D={D}")


def test_out_buffer_and_errors(cuda_device):
    from flash_kmeans_cuda import _C, euclid_assign

    x = iid(1, 300, 64, seed=1).cuda()
    c = x[:, :10].contiguous()
    x_sq = (x.float() ** 2).sum(-1)
    out = torch.full((1, 300), -1, dtype=torch.int32, device="cuda")
    r = euclid_assign(x, c, x_sq, out=out)
    assert r.data_ptr() == out.data_ptr() and (out >= 0).all()
    with pytest.raises(RuntimeError, match="out must be"):
        _C.euclid_assign(x, c, x_sq, (c.float() ** 2).sum(-1), torch.empty(5, dtype=torch.int32,
                                                                           device="cuda"))
    with pytest.raises(RuntimeError, match="share dtype"):
        _C.euclid_assign(x, c.float(), x_sq, (c.float() ** 2).sum(-1), None)
    with pytest.raises(ValueError):
        euclid_assign(x.cpu(), c, x_sq)


_PAIR_SCRIPT = r"""
import sys, numpy as np, torch
sys.path[:0] = sys.argv[2:4]
from _data import iid, subset_init
from flash_kmeans_cuda import _C
out = {}
for i, (B, N, K, D, dt) in enumerate(eval(sys.argv[4])):
    x = iid(B, N, D, seed=B * 7 + N + K + D, dtype=dt)
    c = subset_init(x, K, seed=1) if K <= N else iid(B, K, D, seed=3, dtype=dt)
    xd, cd = x.cuda(), c.cuda()
    ids = _C.euclid_assign(xd, cd, (xd.float() ** 2).sum(-1), (cd.float() ** 2).sum(-1), None)
    out[f"ids{i}"] = ids.cpu().numpy()
np.savez(sys.argv[1], **out)
"""

PAIR_SHAPES = [(1, 1024, 64, 64, "float16"), (2, 8192, 256, 128, "bfloat16"),
               (1, 777, 513, 192, "float16"), (1, 1024, 32, 256, "bfloat16"),
               (1, 4100, 1000, 128, "float16")]


def test_cta_pair_kernel_matches_oracle(cuda_device, tmp_path):
    """The opt-in CTA-pair (cta_group::2) kernel, in a fresh process with
    FKC_ASSIGN_CTA_GROUP=2 (the choice is read once per process)."""
    import os
    import subprocess
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    pkg = os.path.join(os.path.dirname(here), "flash-kmeans-cuda_b200")
    out = tmp_path / "pair.npz"
    env = dict(os.environ, FKC_ASSIGN_CTA_GROUP="2")
    r = subprocess.run([sys.executable, "-c", _PAIR_SCRIPT, str(out), here, pkg,
                        repr(PAIR_SHAPES)], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    got = np.load(out)
    for i, (B, N, K, D, dt) in enumerate(PAIR_SHAPES):
        x = iid(B, N, D, seed=B * 7 + N + K + D, dtype=dt)
        c = subset_init(x, K, seed=1) if K <= N else iid(B, K, D, seed=3, dtype=dt)
        _check(got[f"ids{i}"], orc.assign(to_np(x), to_np(c)), f"pair {dt} {B}x{N}x{K}x{D}")
