"""FKC_DETERMINISTIC=1: the Lloyd update gives bit-identical results run to run.

With the variable set (read once per process, so the checks run in a child
process), the update is a stable counting sort of the labels, a span gather and
an ordered join of the clusters split between spans: every float addition
happens in an order fixed by the labels. The child checks, through the Python
API over the C-ABI:

* the whole-loop graph and the host-driven loop give identical labels and
  centroids (fp16, bf16, fp32; with and without tol);
* two runs of one step on fresh state give identical labels, counts, sums,
  centroids and shift (c3 and c4 shapes, fp32, K > 32768), and the multi-GPU
  rank's step (sums only) gives the step's sums;
* the deterministic path agrees with the float64 oracle (teacher-forced steps:
  labels above the top-2 gap, counts exact, sums, centroids).
"""

from __future__ import annotations

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

_CHILD = r"""
import sys
sys.path[:0] = [{pkg!r}, {root!r}, {tests!r}]
import numpy as np
import torch
import oracle.lloyd as orc
from _data import mixture, subset_init, to_np
from flash_kmeans_cuda import batch_kmeans_Euclid, _lib
from flash_kmeans_cuda.kmeans import LloydState

def stepwise(x, init, iters, tol):
    st = LloydState(x, init.shape[1])
    cur, nxt = init.clone(), torch.empty_like(init)
    st.set_centroids(cur)
    n = 0
    for it in range(iters):
        st.step(cur, nxt, True)
        n = it + 1
        if tol > 0 and st.shift.item() < tol:
            cur = nxt
            break
        cur, nxt = nxt, cur
    return st.ids.clone(), cur, n

for dtype in ("float16", "bfloat16", "float32"):
    for tol in (0.0, 1e-3):
        x = mixture(1, 16384, 64, 32, seed=21, dtype=dtype).cuda()
        init = subset_init(x.cpu(), 32, seed=22).cuda()
        ig, cg, ng = batch_kmeans_Euclid(x, 32, max_iters=30, tol=tol, init_centroids=init)
        is_, cs, ns = stepwise(x, init, 30, tol)
        torch.cuda.synchronize()
        assert ng == ns, (dtype, tol, ng, ns)
        assert torch.equal(ig, is_) and torch.equal(cg, cs), ("graph vs stepwise", dtype, tol)

for dtype, B, N, K, D, zipf in [("float16", 1, 524288, 8192, 128, 1.1),
                                ("bfloat16", 32, 16384, 1024, 64, 0.0),
                                ("float32", 2, 50000, 3000, 32, 1.1),
                                ("float16", 1, 200000, 40000, 64, 0.0)]:
    x = mixture(B, N, D, K, seed=N % 977, zipf=zipf, dtype=dtype).cuda()
    c = subset_init(x.cpu(), K, seed=5).cuda()
    outs = []
    for _ in range(2):
        st = LloydState(x, K)
        st.set_centroids(c)
        nxt = torch.empty_like(c)
        st.step(c, nxt, True)
        torch.cuda.synchronize()
        outs.append((st.ids.clone(), st.counts.clone(), st.sums.clone(), nxt, st.shift.clone()))
        st.set_centroids(c)  # the step left the norm terms of nxt in the workspace
        st.local(c)
        torch.cuda.synchronize()
        assert torch.equal(st.sums, outs[-1][2]), ("local vs step sums", dtype, K)
    for u, v, what in zip(outs[0], outs[1], ("labels", "counts", "sums", "centroids", "shift")):
        assert torch.equal(u, v), (what, dtype, B, N, K, D)

ULP = {{"float16": 2.0 ** -10, "bfloat16": 2.0 ** -7, "float32": 2.0 ** -23}}
for dtype in ("float16", "bfloat16", "float32"):
    B, N, K, D = 2, 20000, 700, 64
    x = mixture(B, N, D, K, seed=3, zipf=1.1, dtype=dtype)
    c = subset_init(x, K, seed=4)
    st = LloydState(x.cuda(), K)
    cur = c.cuda()
    st.set_centroids(cur)
    xn = to_np(x)
    for it in range(3):
        nxt = torch.empty_like(cur)
        st.step(cur, nxt, True)
        torch.cuda.synchronize()
        cn = to_np(cur)
        ref = orc.assign(xn, cn)
        ids = st.ids.cpu().numpy()
        assert not ((ids != ref.ids) & ref.gap_mask()).any()
        s_ref, c_ref = orc.update(xn, ids, K)
        assert np.array_equal(st.counts.cpu().numpy(), c_ref)
        s_abs, _ = orc.update(np.abs(xn), ids, K)
        assert (np.abs(st.sums.cpu().numpy() - s_ref) <= 1e-5 * s_abs + 1e-6).all()
        fin = orc.finalize(s_ref, c_ref, cn, dtype)
        got = to_np(nxt)
        assert (np.abs(got - fin) <= 1e-3 * np.abs(fin) + ULP[dtype] * np.abs(fin) + 1e-6).all()
        cur = nxt
_lib.device_status()
print("deterministic-ok")
"""


def test_deterministic_update_bit_identical(cuda_device):
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = _CHILD.format(pkg=os.path.join(root, "flash-kmeans-cuda_b200"), root=root, tests=here)
    env = dict(os.environ, FKC_DETERMINISTIC="1")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=900)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-4000:]
    assert "deterministic-ok" in out.stdout
