"""End-to-end batch_kmeans_Euclid parity on the GPU against the float64 oracle.

Two kinds of checks:
* teacher-forced: every iteration of the GPU loop is replayed by the oracle
  from the GPU's own input centroids, so one near-tie flip cannot cascade;
  labels must match above the gap threshold, counts exactly, centroids within
  1e-3 relative (+ one ulp of the compute dtype);
* free-running: both loops from the same initial centroids; final inertia
  within 0.05% and label agreement >= 99.9% on well-separated mixtures.
Also restates the reference's API tests (tests/test_shapes.py,
tests/test_dtypes.py, tests/test_correctness.py:16-25 init convention).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle.lloyd as orc
from _data import TORCH_DTYPES, iid, mixture, subset_init, to_np

pytestmark = pytest.mark.gpu

ULP = {"float16": 2.0 ** -10, "bfloat16": 2.0 ** -7, "float32": 2.0 ** -23}


def _close_centroids(got, ref, dtype, rel=1e-3):
    tol = rel * np.abs(ref) + ULP[dtype] * np.abs(ref) + 1e-6
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{int(bad.sum())} centroid entries off (max {np.abs(got - ref).max()})"


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("B,N,K,D,zipf", [
    (1, 20000, 256, 128, 0.0),
    (1, 30000, 1024, 128, 1.1),
    (4, 4096, 64, 64, 0.0),
    (1, 5000, 100, 96, 0.0),
    # fewer row tiles than SMs with several centroid chunks: the assignment
    # shares tiles between CTAs (split mode) and merges them in a fixup pass
    (2, 10000, 700, 64, 0.0),
    (1, 9000, 2000, 128, 1.1),
    (1, 6000, 300, 384, 0.0),  # D > 256: CTA pairs (fp32: split rows, x streamed)
    (1, 5000, 256, 512, 0.0),  # D = 512: x streamed with the stages (fp32: CUDA cores)
    (1, 8000, 300, 256, 1.1),  # D = 256: fp32 as split [hi | lo] rows, x streamed
    # small clusters on average (the fused update + finalize pass) with a few
    # hot ones split into 64-row units that the cluster's last unit finishes
    (2, 20000, 700, 64, 1.1),
])
def test_teacher_forced_iterations(cuda_device, dtype, B, N, K, D, zipf):
    from flash_kmeans_cuda.kmeans import LloydState

    x = mixture(B, N, D, K, seed=N + K, zipf=zipf, dtype=dtype)
    c = subset_init(x, K, seed=2)
    xd = x.cuda()
    st = LloydState(xd, K)
    cur = c.cuda()
    st.set_centroids(cur)
    xn = to_np(x)
    for it in range(4):
        nxt = torch.empty_like(cur)
        st.step(cur, nxt, True)
        torch.cuda.synchronize()
        cn = to_np(cur)
        ref = orc.assign(xn, cn)
        ids = st.ids.cpu().numpy()
        assert not ((ids != ref.ids) & ref.gap_mask()).any(), f"iter {it}: label mismatch"
        assert (ids == ref.ids).mean() >= 0.999
        counts = st.counts.cpu().numpy()
        s_ref, c_ref = orc.update(xn, ids, K)
        assert np.array_equal(counts, c_ref), f"iter {it}: counts"
        # fp32 sums against float64, relative to the sum of magnitudes
        s_abs, _ = orc.update(np.abs(xn), ids, K)
        s_err = np.abs(st.sums.cpu().numpy() - s_ref)
        assert (s_err <= 1e-5 * s_abs + 1e-6).all(), f"iter {it}: sums off by {s_err.max()}"
        fin = orc.finalize(s_ref, c_ref, cn, dtype)
        _close_centroids(to_np(nxt), fin, dtype)
        assert abs(st.shift.item() - orc.shift(to_np(nxt), cn)) <= 1e-3 * orc.shift(fin, cn) + 1e-3
        cur = nxt


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
def test_step_empty_and_split_clusters(cuda_device, dtype):
    """One Lloyd step of the fused update + finalize pass (20 rows per cluster on
    average) where all but 10 centroids are far from every point: 990 empty
    clusters keep their centroid and the 10 others hold about 2000 rows each
    (split into units). Sums, counts, centroids, norms and shift against the
    oracle."""
    from flash_kmeans_cuda.kmeans import LloydState

    B, N, K, D = 2, 20000, 1000, 128
    x = mixture(B, N, D, 10, seed=71, dtype=dtype)
    c = subset_init(x, K, seed=72).float()
    c[:, 10:] += 50.0
    c = c.to(x.dtype)
    xd = x.cuda()
    st = LloydState(xd, K)
    cur = c.cuda()
    st.set_centroids(cur)
    nxt = torch.empty_like(cur)
    st.step(cur, nxt, True)
    torch.cuda.synchronize()
    xn, cn = to_np(x), to_np(c)
    ids = st.ids.cpu().numpy()
    ref = orc.assign(xn, cn)
    assert not ((ids != ref.ids) & ref.gap_mask()).any()
    s_ref, c_ref = orc.update(xn, ids, K)
    counts = st.counts.cpu().numpy()
    assert np.array_equal(counts, c_ref)
    assert (counts[:, 10:] == 0).all() and counts.max() > 1000
    s_abs, _ = orc.update(np.abs(xn), ids, K)
    assert (np.abs(st.sums.cpu().numpy() - s_ref) <= 1e-5 * s_abs + 1e-6).all()
    fin = orc.finalize(s_ref, c_ref, cn, dtype)
    got = to_np(nxt)
    _close_centroids(got, fin, dtype)
    assert np.array_equal(got[:, 10:], cn[:, 10:])  # empty clusters keep the old centroid
    assert abs(st.shift.item() - orc.shift(got, cn)) <= 1e-3 * orc.shift(fin, cn) + 1e-3
    # the next assignment uses the norms written with the new centroids
    st.step(nxt, cur, False)
    torch.cuda.synchronize()
    ref2 = orc.assign(xn, got)
    assert not ((st.ids.cpu().numpy() != ref2.ids) & ref2.gap_mask()).any()


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
def test_local_update_small_clusters(cuda_device, dtype):
    """fkc_lloyd_local (the multi-GPU rank's step before the sums reduction) on small,
    skewed clusters with empty ones: sums and counts against the oracle, twice in a row."""
    from flash_kmeans_cuda.kmeans import LloydState

    B, N, K, D = 2, 12000, 600, 64
    x = mixture(B, N, D, 40, seed=101, zipf=1.1, dtype=dtype)
    c = subset_init(x, K, seed=102).float()
    c[:, 500:] += 50.0  # 100 empty clusters per batch element
    c = c.to(x.dtype)
    st = LloydState(x.cuda(), K)
    cd = c.cuda()
    st.set_centroids(cd)
    for _ in range(2):
        st.local(cd)
        torch.cuda.synchronize()
        ids = st.ids.cpu().numpy()
        s_ref, c_ref = orc.update(to_np(x), ids, K)
        counts = st.counts.cpu().numpy()
        assert np.array_equal(counts, c_ref)
        assert counts.max() > 64 and (counts[:, 500:] == 0).all()
        s_abs, _ = orc.update(np.abs(to_np(x)), ids, K)
        assert (np.abs(st.sums.cpu().numpy() - s_ref) <= 1e-5 * s_abs + 1e-6).all()


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_free_running_inertia(cuda_device, dtype):
    from flash_kmeans_cuda import batch_kmeans_Euclid

    B, N, K, D = 1, 32768, 256, 128
    x = mixture(B, N, D, K, seed=11, dtype=dtype)
    init = subset_init(x, K, seed=12)
    ids, cents, n = batch_kmeans_Euclid(x.cuda(), K, max_iters=10, tol=0.0,
                                        init_centroids=init.cuda())
    torch.cuda.synchronize()
    assert n == 10 and ids.dtype == torch.int32 and cents.dtype == TORCH_DTYPES[dtype]
    ref = orc.lloyd(to_np(x), to_np(init), 10, 0.0, dtype)
    xn = to_np(x)
    inert_gpu = orc.inertia(xn, to_np(cents), ids.cpu().numpy())
    inert_ref = orc.inertia(xn, ref.centroids, ref.ids)
    assert abs(inert_gpu - inert_ref) <= 5e-4 * inert_ref
    assert (ids.cpu().numpy() == ref.ids).mean() >= 0.999


@pytest.mark.parametrize("B,N,K,D", [
    (1, 100, 8, 64), (1, 257, 16, 128), (1, 1024, 1, 64), (1, 1024, 63, 64),
    (1, 1024, 65, 64), (1, 1024, 32, 256), (3, 2048, 32, 64),
])
def test_shapes(cuda_device, B, N, K, D):
    """tests/test_shapes.py:11-31 of the reference."""
    from flash_kmeans_cuda import batch_kmeans_Euclid

    x = torch.randn(B, N, D, device="cuda", dtype=torch.float16)
    ids, cents, n_iters = batch_kmeans_Euclid(x, K, max_iters=3, tol=0.0)
    assert ids.shape == (B, N) and ids.dtype == torch.int32
    assert cents.shape == (B, K, D) and cents.dtype == torch.float16
    assert (ids >= 0).all() and (ids < K).all()
    assert n_iters == 3


@pytest.mark.parametrize("K", [256, 2048, 4096, 8192])
def test_large_k_single_iteration(cuda_device, K):
    """tests/test_shapes.py:34-53: one iteration against the exact assignment."""
    from flash_kmeans_cuda import batch_kmeans_Euclid

    torch.manual_seed(123)
    x = torch.randn(1, 256, 128, device="cuda", dtype=torch.float16)
    init = torch.randn(1, K, 128, device="cuda", dtype=torch.float16)
    ids, cents, n = batch_kmeans_Euclid(x, K, max_iters=1, tol=0.0, init_centroids=init)
    ref = orc.assign(to_np(x), to_np(init))
    got = ids.cpu().numpy()
    assert n == 1 and not ((got != ref.ids) & ref.gap_mask()).any()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_kmeans_dtype(cuda_device, dtype):
    from flash_kmeans_cuda import batch_kmeans_Euclid

    x = torch.randn(2, 2048, 64, device="cuda", dtype=dtype)
    ids, cents, n_iters = batch_kmeans_Euclid(x, 32, max_iters=5, tol=0.0)
    assert cents.dtype == dtype and n_iters == 5


def test_tol_stops_early_and_init_untouched(cuda_device, capsys):
    from flash_kmeans_cuda import batch_kmeans_Euclid

    x = mixture(1, 8192, 64, 16, seed=4).cuda()
    init = subset_init(x.cpu(), 16, seed=5).cuda()
    keep = init.clone()
    ids, cents, n = batch_kmeans_Euclid(x, 16, max_iters=200, tol=1e-4, init_centroids=init,
                                        verbose=True)
    assert 1 <= n < 200
    assert torch.equal(init, keep)
    out = capsys.readouterr().out
    assert out.count("center shift") == n
    # converged: one more iteration from the result moves nothing
    ids2, cents2, _ = batch_kmeans_Euclid(x, 16, max_iters=1, init_centroids=cents)
    assert torch.equal(ids, ids2)


def test_kmeans_rejects_bad_input(cuda_device):
    from flash_kmeans_cuda import batch_kmeans_Euclid

    with pytest.raises(AssertionError):
        batch_kmeans_Euclid(torch.randn(1, 10, 4), 2)
    with pytest.raises(AssertionError):
        batch_kmeans_Euclid(torch.randn(10, 4, device="cuda"), 2)
    with pytest.raises(RuntimeError, match="share dtype"):
        batch_kmeans_Euclid(torch.randn(1, 10, 16, device="cuda", dtype=torch.float16), 2,
                            init_centroids=torch.randn(1, 2, 16, device="cuda"))


def _stepwise(x, init, max_iters, tol):
    """Iteration-by-iteration loop (fkc_lloyd_iter per step, shift read each step)."""
    from flash_kmeans_cuda.kmeans import LloydState

    st = LloydState(x, init.shape[1])
    cur, nxt = init.clone(), torch.empty_like(init)
    st.set_centroids(cur)
    n = 0
    for it in range(max_iters):
        st.step(cur, nxt, True)
        n = it + 1
        if tol > 0 and st.shift.item() < tol:
            cur = nxt
            break
        cur, nxt = nxt, cur
    return st.ids.clone(), cur, n


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("tol", [0.0, 1e-3])
def test_graph_loop_matches_stepwise(cuda_device, dtype, tol):
    """The whole-loop graph (device-side while + tol) runs the same iterations as
    the host-driven loop: same iteration count, labels >= 99.9% equal and
    centroids within 1e-3 (the default update accumulates with atomics, so the
    last bits may differ; FKC_DETERMINISTIC=1 makes them identical, see
    tests/test_deterministic_gpu.py)."""
    from flash_kmeans_cuda import batch_kmeans_Euclid

    x = mixture(1, 16384, 64, 32, seed=21, dtype=dtype).cuda()
    init = subset_init(x.cpu(), 32, seed=22).cuda()
    ids_g, c_g, n_g = batch_kmeans_Euclid(x, 32, max_iters=30, tol=tol, init_centroids=init)
    ids_s, c_s, n_s = _stepwise(x, init, 30, tol)
    torch.cuda.synchronize()
    assert n_g == n_s
    assert (ids_g == ids_s).float().mean().item() >= 0.999
    _close_centroids(to_np(c_g.cpu()), to_np(c_s.cpu()), dtype)


def test_graph_loop_replay_and_edges(cuda_device):
    """Second call on the same buffers replays the cached graph; max_iters=0 and
    tol larger than any shift are handled on the device."""
    from flash_kmeans_cuda import _lib
    from flash_kmeans_cuda.kmeans import LloydState

    x = mixture(2, 8192, 128, 64, seed=31).cuda()
    init = subset_init(x.cpu(), 64, seed=32).cuda()
    st = LloydState(x, 64)
    results = []
    for _ in range(2):
        c = init.clone()
        n = st.run(c, 6, 0.0)
        torch.cuda.synchronize()
        results.append((st.ids.clone(), c, int(n.item())))
    assert results[0][2] == results[1][2] == 6
    assert torch.equal(results[0][0], results[1][0])
    _close_centroids(to_np(results[0][1].cpu()), to_np(results[1][1].cpu()), "float16")
    c = init.clone()
    assert int(st.run(c, 0, 0.0).item()) == 0 and torch.equal(c, init)
    c = init.clone()
    assert int(st.run(c, 50, 1e30).item()) == 1  # every shift is below tol: one iteration
    _lib.device_status()


@pytest.mark.parametrize("dtype", ["float16", "float32"])
def test_euclid_iter_helper(cuda_device, dtype):
    """kmeans._euclid_iter (the reference's one-step helper) against the float64 oracle,
    with and without caller buffers."""
    from flash_kmeans_cuda.kmeans import _euclid_iter

    B, N, K, D = 2, 5000, 64, 128
    x = mixture(B, N, D, K, seed=17, dtype=dtype)
    c = subset_init(x, K, seed=18)
    xd, cd = x.cuda(), c.cuda()
    x_sq = (xd.float() ** 2).sum(-1)
    new_c, shift, ids = _euclid_iter(xd, x_sq, cd)
    torch.cuda.synchronize()
    xn, cn = to_np(x), to_np(c)
    ref = orc.assign(xn, cn)
    got = ids.cpu().numpy()
    assert not ((got != ref.ids) & ref.gap_mask()).any()
    s_ref, c_ref = orc.update(xn, got, K)
    fin = orc.finalize(s_ref, c_ref, cn, dtype)
    _close_centroids(to_np(new_c), fin, dtype)
    assert abs(float(shift) - orc.shift(to_np(new_c), cn)) <= 1e-5 + 1e-5 * float(shift)
    # caller buffers are written in place and returned; no shift without compute_shift
    bufs = dict(cluster_ids_buf=torch.empty_like(ids), sums_buf=torch.empty(
        B, K, D, device="cuda"), counts_buf=torch.empty(B, K, dtype=torch.int32, device="cuda"),
        new_centroids_buf=torch.empty_like(cd))
    nc2, sh2, ids2 = _euclid_iter(xd, x_sq, cd, compute_shift=False, **bufs)
    torch.cuda.synchronize()
    assert sh2 is None
    assert nc2.data_ptr() == bufs["new_centroids_buf"].data_ptr()
    assert ids2.data_ptr() == bufs["cluster_ids_buf"].data_ptr()
    assert torch.equal(ids2, ids)
