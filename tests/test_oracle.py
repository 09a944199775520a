"""CPU tests of the oracle (oracle/lloyd.py): known answers, the reference's
semantics, and the reference's own statistical pins restated.

The reference ships no golden vectors; its label checks are statistical
(tests/test_mma_optin.py:60-67, tests/test_shapes.py:52,
tests/test_persistent.py:35-48). Fixtures produced by the reference's CUDA
kernels are checked in tests/test_golden.py.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle.lloyd as orc


def test_known_answer_2d():
    x = np.array([[[0.0, 0.0], [1.0, 0.1], [9.0, 9.0], [10.0, 10.0], [0.2, 0.9]]])
    c = np.array([[[0.0, 0.0], [10.0, 10.0], [100.0, 100.0]]])
    a = orc.assign(x, c)
    assert a.ids.tolist() == [[0, 0, 1, 1, 0]]
    assert a.best[0, 0] == 0.0 and a.best[0, 3] == 0.0
    sums, counts = orc.update(x, a.ids, 3)
    assert counts.tolist() == [[3, 2, 0]]
    np.testing.assert_allclose(sums[0, 0], [1.2, 1.0])
    new = orc.finalize(sums, counts, c, "float32")
    np.testing.assert_allclose(new[0, 0], [0.4, 1.0 / 3.0], rtol=1e-6)
    np.testing.assert_allclose(new[0, 1], [9.5, 9.5])
    assert np.array_equal(new[0, 2], c[0, 2]), "empty cluster keeps its centroid"
    assert orc.shift(new, c) == pytest.approx(np.sqrt(0.5), rel=1e-6)  # cluster 1 moved most


def test_ties_go_to_lowest_index():
    x = np.array([[[1.0, 1.0], [3.0, 3.0]]])
    c = np.array([[[2.0, 2.0], [2.0, 2.0], [0.0, 0.0], [2.0, 2.0]]])
    a = orc.assign(x, c)
    # point 0 is equidistant to c0, c1, c2 and c3 (dist 2): lowest index wins
    assert a.ids.tolist() == [[0, 0]]
    assert not a.gap_mask().any()


def test_labels_out_of_range_are_skipped():
    """update_sorted.cu:94: runs whose id is outside [0, K) are not accumulated."""
    x = np.ones((1, 4, 3))
    sums, counts = orc.update(x, np.array([[0, -1, 5, 1]]), 2)
    assert counts.tolist() == [[1, 1]]


def test_round_to_matches_torch():
    g = torch.Generator().manual_seed(0)
    v = torch.randn(10000, generator=g, dtype=torch.float64) * 100
    for name, dt in (("float16", torch.float16), ("bfloat16", torch.bfloat16)):
        ref = v.float().to(dt).float().numpy()  # fp32 value -> dtype, as the kernels do
        assert np.array_equal(orc.round_to(v.numpy(), name), ref), name


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("B,N,K,D", [(1, 1024, 64, 64), (1, 4096, 128, 128)])
def test_matches_fp32_einsum_reference(dtype, B, N, K, D):
    """The reference's own pin (tests/test_mma_optin.py:29-67): <3% vs an fp32 einsum."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(B, N, D, generator=g).to(getattr(torch, dtype)).float()
    c = x[:, :K].contiguous()
    x_sq = (x ** 2).sum(-1)
    c_sq = (c ** 2).sum(-1)
    cross = torch.einsum("bnd,bkd->bnk", x, c)
    ref = (x_sq.unsqueeze(-1) + c_sq.unsqueeze(1) - 2 * cross).argmin(-1).numpy()
    a = orc.assign(x.numpy(), c.numpy())
    assert (a.ids != ref).mean() < 3e-2
    assert (a.ids[:, :K] == np.arange(K)).all(), "identity centroids (test_persistent.py:35-48)"


def test_gap_mask_rows_are_stable():
    """Rows above the gap threshold keep their label under fp32 rounding of the inputs."""
    g = np.random.default_rng(1)
    x = g.standard_normal((1, 2000, 32))
    c = g.standard_normal((1, 50, 32))
    a = orc.assign(x, c)
    b = orc.assign(x.astype(np.float32) * (1 + 1e-7), c.astype(np.float32))
    m = a.gap_mask()
    assert m.mean() > 0.9
    assert (a.ids[m] == b.ids[m]).all()


def test_lloyd_tol_and_history():
    g = np.random.default_rng(2)
    centres = g.standard_normal((4, 8)) * 10
    x = (centres[g.integers(0, 4, 400)] + g.standard_normal((400, 8)))[None]
    init = x[:, :4].copy()
    r = orc.lloyd(x, init, 100, 1e-6, "float32", keep_history=True)
    assert r.n_iters < 100
    assert r.history[-1]["shift"] < 1e-6
    assert r.history[0]["counts"].sum() == 400
    r2 = orc.lloyd(x, init, 3, 0.0, "float32")
    assert r2.n_iters == 3
    # labels are those of the last assignment (against the pre-update centroids)
    assert np.array_equal(r2.ids, orc.lloyd(x, init, 3, 0.0, "float32", True).history[-1]["ids"])


def test_inertia_decreases():
    g = np.random.default_rng(3)
    x = g.standard_normal((1, 3000, 16)).astype(np.float32)
    cur = x[:, :40].copy()
    prev = np.inf
    for _ in range(5):
        a = orc.assign(x, cur)
        val = orc.inertia(x, cur, a.ids)
        assert val <= prev + 1e-6
        prev = val
        s, n = orc.update(x, a.ids, 40)
        cur = orc.finalize(s, n, cur, "float32")
