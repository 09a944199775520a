"""Pins the float64 torch restatement (tests/_oracle_torch.py, used by the GPU parity
tests at the benchmark sizes) to the numpy oracle (oracle/lloyd.py) on the CPU."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import _oracle_torch as ot
import oracle.lloyd as orc
from _data import iid, mixture, subset_init, to_np


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("B,N,K,D,zipf", [(1, 3000, 64, 32, 0.0), (2, 2500, 40, 64, 1.1),
                                          (1, 2000, 1, 16, 0.0)])
def test_torch_oracle_matches_numpy_oracle(dtype, B, N, K, D, zipf):
    x = mixture(B, N, D, max(K, 2), seed=N + D, zipf=zipf, dtype=dtype)
    c = subset_init(x, K, seed=3)
    a_t = ot.assign(x, c, chunk_elems=1 << 14)  # several row chunks
    a_n = orc.assign(to_np(x), to_np(c))
    assert np.array_equal(a_t.ids.numpy(), a_n.ids)
    assert np.allclose(a_t.best.numpy(), a_n.best, rtol=1e-12, atol=1e-9)
    assert np.array_equal(np.isinf(a_t.second.numpy()), np.isinf(a_n.second))
    fin = np.isfinite(a_n.second)
    assert np.allclose(a_t.second.numpy()[fin], a_n.second[fin], rtol=1e-12, atol=1e-9)
    assert np.array_equal(a_t.gap_mask().numpy(), a_n.gap_mask())
    s_t, n_t = ot.update(x, a_t.ids, K)
    s_n, n_n = orc.update(to_np(x), a_n.ids, K)
    assert np.array_equal(n_t.numpy(), n_n)
    assert np.allclose(s_t.numpy(), s_n, rtol=1e-12, atol=1e-9)
    f_t = ot.finalize(s_t, n_t, c, dtype)
    f_n = orc.finalize(s_n, n_n, to_np(c), dtype)
    assert np.array_equal(f_t.numpy(), f_n)
    assert ot.shift(f_t, c) == pytest.approx(orc.shift(f_n, to_np(c)), rel=1e-12)
    assert ot.inertia(x, f_t, a_t.ids) == pytest.approx(
        orc.inertia(to_np(x), f_n, a_n.ids), rel=1e-12)


def test_torch_oracle_ties_lowest_index():
    x = iid(1, 64, 16, seed=5, dtype="float32")
    c = torch.cat([x[:, :8], x[:, :8]], dim=1)  # every centroid duplicated at k and k + 8
    a = ot.assign(x, c)
    assert (a.ids[0, :8] == torch.arange(8)).all()
    assert not a.gap_mask()[0, :8].any()  # exact ties: outside the gap mask


def test_torch_oracle_lloyd_matches_numpy():
    x = mixture(1, 4000, 32, 16, seed=9, dtype="float16")
    init = subset_init(x, 16, seed=10)
    ids_t, c_t = ot.lloyd(x, init, 5, "float16")
    ref = orc.lloyd(to_np(x), to_np(init), 5, 0.0, "float16")
    assert np.array_equal(ids_t.numpy(), ref.ids)
    assert np.array_equal(c_t.numpy(), ref.centroids)
