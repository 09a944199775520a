"""fkc_assign_noalloc (static-scratch assignment) against fkc_assign, through the C-ABI.

The entry point exists for callers that cannot allocate device memory (FFI
bindings that only receive device pointers, hosts whose device memory a
pooling allocator owns, pipelines that cannot take cudaFree's device-wide
sync). Its labels must be identical to fkc_assign's on the same inputs:
for two calls in a row whose shapes differ (the second call reuses the
scratch the first one wrote), after every other test of the suite (this file
is collected last), and as the library's first CUDA work in a fresh process
(a child process).
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
    # What this process holds through torch's allocator must not move at all; the
    # device-wide free figure also counts other processes, so it gets a loose bound
    # (far below the 32 MiB a workspace of this shape would take).
    reserved0, allocated0 = torch.cuda.memory_reserved(), torch.cuda.memory_allocated()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        out.fill_(-1)
        _assign_noalloc(x, c, out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.equal(out, want)
    assert torch.cuda.memory_reserved() == reserved0
    assert torch.cuda.memory_allocated() == allocated0
    assert abs(free0 - free1) < (1 << 20), f"device free memory moved by {free0 - free1} bytes"


_FRESH_CHILD = r"""
import sys
sys.path[:0] = [{pkg!r}, {root!r}, {tests!r}]
import torch
from _data import iid, subset_init
from flash_kmeans_cuda import _lib as L
assert L.lib.fkc_kernel_launches() == 0
x = iid(1, 30000, 128, seed=61, dtype="float16").cuda()
c = subset_init(x.cpu(), 300, seed=62).cuda()
st = torch.cuda.current_stream().cuda_stream
got = torch.full((1, 30000), -1, dtype=torch.int32, device="cuda")
# the library's first CUDA work in this process: module load + scratch lookup + launch
L.check(L.lib.fkc_assign_noalloc(x.data_ptr(), c.data_ptr(), None, None, got.data_ptr(), 1,
                                 30000, 300, 128, 0, st), "fkc_assign_noalloc")
need = L.lib.fkc_assign_workspace_size(1, 30000, 300, 128, 0)
ws = torch.empty(need, dtype=torch.uint8, device="cuda")
want = torch.full_like(got, -1)
L.check(L.lib.fkc_assign(x.data_ptr(), c.data_ptr(), None, None, want.data_ptr(), 1, 30000, 300,
                         128, 0, ws.data_ptr(), need, st), "fkc_assign")
torch.cuda.synchronize()
L.device_status()
assert torch.equal(got, want), "labels differ"
print("fresh-ok", L.lib.fkc_kernel_launches())
"""


def test_noalloc_first_call_in_fresh_process(cuda_device):
    """fkc_assign_noalloc as the library's first CUDA work in a new process (the set-up
    path: lazy module load and scratch lookup) gives fkc_assign's labels."""
    import os
    import subprocess
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = _FRESH_CHILD.format(pkg=os.path.join(root, "flash-kmeans-cuda_b200"), root=root,
                               tests=here)
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-4000:]
    assert "fresh-ok" in out.stdout


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
    """fp32 at D > 128 and odd D take the CUDA-core kernel, which needs no scratch; fp32 at
    D <= 128 takes the split-bf16 tensor-core route through the scratch. All equal
    fkc_assign's labels."""
    for dt, D in (("float32", 64), ("float32", 144), ("float16", 33)):
        x, c = _inputs(1, 4000, 100, D, dt, 51)
        got = _assign_noalloc(x, c)
        want = _assign_ws(x, c)
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"{dt} D={D}"


def test_noalloc_unaligned_input_has_no_limit(cuda_device):
    """x not 16-byte aligned: fkc_assign takes the CUDA-core kernel, so the no-alloc call
    needs no scratch and has no size limit (1.1 M points would need 35 MB of tensor-core
    scratch); labels equal fkc_assign's on the same (unaligned) view."""
    n = 1_100_000
    base = iid(1, n * 64 + 1, 1, seed=57, dtype="float16").cuda().view(-1)
    x = base[1:].view(1, n, 64)  # starts 2 bytes past an aligned address
    assert x.data_ptr() % 16 != 0
    c = subset_init(x.cpu(), 50, seed=58).cuda()
    got = _assign_noalloc(x, c)
    want = _assign_ws(x, c)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
