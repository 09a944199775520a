"""The fused update's split-cluster protocol, simulated on the CPU (no GPU).

update.cu, gather_finalize_kernel: a cluster of more than 64 rows is cut into
ceil(count / 64) units. Each unit adds its partial sum into the cluster's accumulator row
(vector atomics), fences, and increments the cluster's done counter; the unit that sees
the counter at nunits - 1 reads the row, finishes the cluster and writes zeros back to the
row and the counter. Under any interleaving of units: exactly one unit finishes each
cluster, it sees the complete sum, and the accumulator and counter are zero again for
the next pass (they are zeroed only when the workspace is prepared)."""

from __future__ import annotations

import numpy as np
import pytest

UNIT = 64


@pytest.mark.parametrize("seed", range(25))
def test_last_unit_finishes_each_cluster_once(seed):
    rng = np.random.default_rng(seed)
    K, D = int(rng.integers(1, 40)), 4
    counts = rng.integers(0, 700, K)
    x_sums = rng.standard_normal((K, D))
    acc = np.zeros((K, D))
    done = np.zeros(K, dtype=np.int64)
    for _ in range(3):  # passes in a row: the state must come back to zero each time
        units = []
        for k in range(K):
            if counts[k] > UNIT:
                n = (counts[k] + UNIT - 1) // UNIT
                parts = rng.dirichlet(np.ones(n))[:, None] * x_sums[k]
                units += [(k, n, p) for p in parts]
        order = rng.permutation(len(units))
        finished = {}
        for i in order:  # each unit's atomics, then its counter increment
            k, n, part = units[i]
            acc[k] += part
            prev = done[k]
            done[k] += 1
            if prev == n - 1:
                assert k not in finished
                finished[k] = acc[k].copy()
                acc[k] = 0.0
                done[k] = 0
        split = [k for k in range(K) if counts[k] > UNIT]
        assert sorted(finished) == split
        for k in split:
            assert np.allclose(finished[k], x_sums[k])
        assert not acc.any() and not done.any()
