"""Parity at the benchmark configurations, against float64.

The north-star bar: labels bit-exact wherever the exact top-2 distance gap
exceeds 1e-3 * ||x||^2 and >= 99.9% equal overall, counts exact, fp32 sums
within 1e-5 of the sum of magnitudes, centroids within 1e-3 relative (plus
one ulp of the compute dtype), final inertia of a free-running loop within
0.05% of the exact loop's. The float64 checker is ``tests/_oracle_torch.py``
(pinned to ``oracle/lloyd.py`` on the CPU), run on the GPU because these
problems are too large for a CPU oracle in a test run.

* c2 (B=1, N=131072, K=2048, D=128 fp16 mixture): 20 teacher-forced steps and
  a free-running 20-iteration ``batch_kmeans_Euclid`` call.
* c3 (B=1, N=524288, K=8192, D=128 fp16, Zipf(1.1) cluster sizes): two
  teacher-forced steps (the timed bench workload), and the multi-GPU rank's
  step (assign + counting-sort accumulate, ``fkc_lloyd_local``).
* c4 (B=32, N=16384, K=1024, D=64 bf16): teacher-forced steps (the fused
  update + finalize pass) and a free-running 10-iteration call.
* c5 regime (iid N(0, I), K=65536, D=128 fp16; N=266240 >= 2^18, whose 1040
  row tiles leave the last wave of 148 CTAs short, so the assignment runs in
  split mode): one step through the fused pass and one through the
  accumulator (scatter with per-row atomics for K > 16384), near ties common.
"""

from __future__ import annotations

import pytest
import torch

import _oracle_torch as ot
from _data import TORCH_DTYPES, iid, mixture, subset_init

pytestmark = pytest.mark.gpu

ULP = {"float16": 2.0 ** -10, "bfloat16": 2.0 ** -7, "float32": 2.0 ** -23}


def _check_assign(ids, x, c, what):
    a = ot.assign(x, c)
    got = ids.to(torch.int64)
    bad = ((got != a.ids) & a.gap_mask()).sum().item()
    agree = (got == a.ids).double().mean().item()
    assert bad == 0, f"{what}: {bad} labels differ where the top-2 gap exceeds 1e-3 |x|^2"
    assert agree >= 0.999, f"{what}: label agreement {agree:.6f}"
    return a


def _check_update(st, x, c, nxt, dtype, what, sums_too=True):
    """counts exact, sums and next centroids of the GPU labels against float64."""
    K = c.shape[1]
    s_ref, n_ref = ot.update(x, st.ids, K)
    assert torch.equal(st.counts.to(torch.int64), n_ref), f"{what}: counts differ"
    if sums_too:
        s_abs = ot.abs_sums(x, st.ids, K)
        err = (st.sums.to(torch.float64) - s_ref).abs()
        assert bool((err <= 1e-5 * s_abs + 1e-6).all()), f"{what}: sums off by {err.max():.3g}"
    if nxt is not None:
        fin = ot.finalize(s_ref, n_ref, c, dtype)
        got = nxt.to(torch.float32)
        tol = 1e-3 * fin.abs() + ULP[dtype] * fin.abs() + 1e-6
        nbad = int(((got - fin).abs() > tol).sum())
        assert nbad == 0, f"{what}: {nbad} centroid entries off"
        return fin
    return None


def _teacher_forced(x, c0, steps, dtype, what):
    from flash_kmeans_cuda.kmeans import LloydState

    K = c0.shape[1]
    st = LloydState(x, K)
    cur = c0.clone()
    st.set_centroids(cur)
    for it in range(steps):
        nxt = torch.empty_like(cur)
        st.step(cur, nxt, True)
        torch.cuda.synchronize()
        _check_assign(st.ids, x, cur, f"{what} iter {it}")
        _check_update(st, x, cur, nxt, dtype, f"{what} iter {it}")
        ref_shift = ot.shift(nxt, cur)
        assert abs(st.shift.item() - ref_shift) <= 1e-3 * ref_shift + 1e-3
        cur = nxt
    return st, cur


def _free_running(x, init, iters, dtype, what):
    from flash_kmeans_cuda import batch_kmeans_Euclid

    ids, cents, n = batch_kmeans_Euclid(x, init.shape[1], max_iters=iters, tol=0.0,
                                        init_centroids=init)
    torch.cuda.synchronize()
    assert n == iters and cents.dtype == TORCH_DTYPES[dtype]
    ref_ids, ref_c = ot.lloyd(x, init, iters, dtype)
    inert = ot.inertia(x, cents, ids)
    inert_ref = ot.inertia(x, ref_c, ref_ids)
    assert abs(inert - inert_ref) <= 5e-4 * inert_ref, (
        f"{what}: inertia {inert:.6g} vs exact {inert_ref:.6g}")
    agree = (ids.to(torch.int64) == ref_ids).double().mean().item()
    assert agree >= 0.999, f"{what}: label agreement {agree:.6f} after {iters} iterations"


def test_c2_teacher_forced_20_iterations(cuda_device):
    x = mixture(1, 131072, 128, 2048, seed=2, dtype="float16").cuda()
    c0 = subset_init(x.cpu(), 2048, seed=3).cuda()
    _teacher_forced(x, c0, 20, "float16", "c2")


def test_c2_free_running_20_iterations(cuda_device):
    x = mixture(1, 131072, 128, 2048, seed=2, dtype="float16").cuda()
    init = subset_init(x.cpu(), 2048, seed=3).cuda()
    _free_running(x, init, 20, "float16", "c2")


def test_c3_teacher_forced(cuda_device):
    x = mixture(1, 524288, 128, 8192, seed=5, zipf=1.1, dtype="float16").cuda()
    c0 = subset_init(x.cpu(), 8192, seed=6).cuda()
    st, cur = _teacher_forced(x, c0, 2, "float16", "c3")
    # Zipf-sized clusters: the counts are far from uniform (the random-subset init
    # spreads many centroids over the heavy mixture components)
    assert int(st.counts.max()) > 8 * 524288 // 8192
    # the multi-GPU rank's step: assign + counting sort + accumulate into sums
    st.local(cur)
    torch.cuda.synchronize()
    _check_assign(st.ids, x, cur, "c3 local")
    _check_update(st, x, cur, None, "float16", "c3 local")


def test_c4_teacher_forced(cuda_device):
    x = mixture(32, 16384, 64, 1024, seed=40, dtype="bfloat16").cuda()
    c0 = subset_init(x.cpu(), 1024, seed=41).cuda()
    _teacher_forced(x, c0, 3, "bfloat16", "c4")


def test_c4_free_running_10_iterations(cuda_device):
    x = mixture(32, 16384, 64, 1024, seed=40, dtype="bfloat16").cuda()
    init = subset_init(x.cpu(), 1024, seed=41).cuda()
    _free_running(x, init, 10, "bfloat16", "c4")


def test_c5_regime_k65536(cuda_device):
    from flash_kmeans_cuda.kmeans import LloydState

    N, K = 266240, 65536
    x = iid(1, N, 128, seed=0, dtype="float16").cuda()
    c0 = subset_init(x.cpu(), K, seed=1).cuda()
    st = LloydState(x, K)
    st.set_centroids(c0)
    # fused update + finalize pass (about 4 rows per cluster)
    nxt = torch.empty_like(c0)
    st.step(c0, nxt, True)
    torch.cuda.synchronize()
    a = _check_assign(st.ids, x, c0, "c5 step")
    near = (~a.gap_mask()).double().mean().item()
    _check_update(st, x, c0, nxt, "float16", "c5 step")
    # accumulator path (the multi-GPU rank's local step) on the new centroids
    st.local(nxt)
    torch.cuda.synchronize()
    _check_assign(st.ids, x, nxt, "c5 local")
    _check_update(st, x, nxt, None, "float16", "c5 local")
    print(f"c5 regime: {near:.2e} of the rows have a top-2 gap below 1e-3 |x|^2")
