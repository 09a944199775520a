"""fkc_assign_noalloc (static-scratch assignment) against fkc_assign, through the C-ABI.

Collected last on purpose (file name): the entry point must give the same
labels whether it is the first CUDA work of a fresh process or runs after every
other test. Each call's labels must be identical to fkc_assign's on the same
inputs, for two calls in a row whose shapes differ (the second call reuses the
scratch the first one wrote).
"""

from __future__ import annotations

import pytest
import torch

import oracle.lloyd as orc
from _data import iid, subset_init, to_np

pytestmark = pytest.mark.gpu

F16, BF16, F32 = 0, 1, 2
CODES = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}


def _lib():
    from flash_kmeans_cuda import _lib as L

    return L


def _inputs(B, N, K, D, dtype, seed):
    x = iid(B, N, D, seed=seed, dtype=dtype).cuda()
    c = subset_init(x.cpu(), K, seed=seed + 1).cuda()
    return x, c


def _assign_ws(x, c):
    """The existing entry point, with a workspace the test allocates."""
    L = _lib()
    B, N, D = x.shape
    K = c.shape[1]
    code = CODES[x.dtype]
    need = L.lib.fkc_assign_workspace_size(B, N, K, D, code)
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device=x.device)
    ids = torch.full((B, N), -1, dtype=torch.int32, device=x.device)
    st = torch.cuda.current_stream().cuda_stream
    L.check(L.lib.fkc_assign(x.data_ptr(), c.data_ptr(), None, None, ids.data_ptr(), B, N, K, D,
                             code, ws.data_ptr(), need, st), "fkc_assign")
    return ids


def _assign_noalloc(x, c, out=None):
    L = _lib()
    B, N, D = x.shape
    K = c.shape[1]
    ids = out if out is not None else torch.full((B, N), -1, dtype=torch.int32, device=x.device)
    st = torch.cuda.current_stream().cuda_stream
    L.check(L.lib.fkc_assign_noalloc(x.data_ptr(), c.data_ptr(), None, None, ids.data_ptr(), B,
                                     N, K, D, CODES[x.dtype], st), "fkc_assign_noalloc")
    return ids


def test_noalloc_matches_fkc_assign_two_calls(cuda_device):
    # First call: the larger shape; second call: a smaller one with other data,
    # reading the scratch rows the first call left behind.
    calls = [((2, 20000, 1000, 128), "float16", 11), ((1, 3000, 70, 64), "bfloat16", 23)]
    for (B, N, K, D), dt, seed in calls:
        x, c = _inputs(B, N, K, D, dt, seed)
        got = _assign_noalloc(x, c)
        want = _assign_ws(x, c)
        torch.cuda.synchronize()
        _lib().device_status()
        assert torch.equal(got, want), f"{dt} {B}x{N}x{K}x{D}: labels differ from fkc_assign"
        # and both agree with the float64 oracle where the top-2 gap is clear
        ref = orc.assign(to_np(x.cpu()), to_np(c.cpu()))
        g = got.cpu().numpy()
        assert not ((g != ref.ids) & ref.gap_mask(1e-3)).any()


def test_noalloc_allocates_nothing_after_setup(cuda_device):
    x, c = _inputs(1, 50000, 512, 128, "float16", 31)
    want = _assign_ws(x, c)
    out = torch.full_like(want, -1)
    _assign_noalloc(x, c, out)  # set-up (first call on this device) already done or done here
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        out.fill_(-1)
        _assign_noalloc(x, c, out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.equal(out, want)
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"


def test_noalloc_size_limit(cuda_device):
    """Exactly the maximum scratch is accepted; one more point is rejected."""
    L = _lib()
    limit = 32 * 1024 * 1024
    K, D = 8192, 64
    N = (limit - K * 32) // 32  # 1040384 points: aext + cext fill the scratch exactly
    assert L.lib.fkc_assign_workspace_size(1, N, K, D, F16) == limit
    x, c = _inputs(1, N, K, D, "float16", 41)
    got = _assign_noalloc(x, c)
    want = _assign_ws(x, c)
    torch.cuda.synchronize()
    assert torch.equal(got, want)

    before = L.lib.fkc_kernel_launches()
    ids = torch.empty((1, N + 1), dtype=torch.int32, device="cuda")
    x1 = torch.cat([x, x[:, :1]], dim=1)
    st = L.lib.fkc_assign_noalloc(x1.data_ptr(), c.data_ptr(), None, None, ids.data_ptr(), 1,
                                  N + 1, K, D, F16, None)
    assert st == -5 and "static scratch" in L.last_error()
    assert L.lib.fkc_kernel_launches() == before, "a rejected call launched kernels"


def test_noalloc_cuda_core_path(cuda_device):
    """fp32 and odd D take the CUDA-core kernel, which needs no scratch at all."""
    for dt, D in (("float32", 64), ("float16", 33)):
        x, c = _inputs(1, 4000, 100, D, dt, 51)
        got = _assign_noalloc(x, c)
        want = _assign_ws(x, c)
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"{dt} D={D}"
