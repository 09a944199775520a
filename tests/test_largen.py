"""Host-side logic of the streamed large-N path (no GPU): block plan and argument checks."""

from __future__ import annotations

import pytest
import torch

from flash_kmeans_cuda.largen import _check_host_x, plan_blocks


def test_plan_blocks_covers_rows_in_order():
    for n, rows, devs in [(100, 16, 3), (10, 100, 2), (1, 1, 1), (1000, 7, 8), (64, 64, 4)]:
        plan = plan_blocks(n, rows, devs)
        assert len(plan) == devs
        flat = [r for d in plan for r in d]
        assert flat[0][0] == 0 and flat[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(flat, flat[1:]))  # contiguous, in order
        assert all(0 < r1 - r0 <= rows for r0, r1 in flat)
        sizes = [len(d) for d in plan]
        assert max(sizes) - min(sizes) <= 1  # balanced to one block


def test_plan_blocks_rejects_bad_sizes():
    with pytest.raises(ValueError):
        plan_blocks(0, 4, 1)
    with pytest.raises(ValueError):
        plan_blocks(10, 0, 1)


def test_host_x_checks():
    _check_host_x(torch.zeros((8, 16), dtype=torch.float16))
    with pytest.raises(ValueError, match="batched"):
        _check_host_x(torch.zeros((2, 8, 16), dtype=torch.float16))
    with pytest.raises(ValueError, match="dtype"):
        _check_host_x(torch.zeros((8, 16), dtype=torch.float64))


def test_host_input_rejects_bad_x():
    from flash_kmeans_cuda.largen import batch_kmeans_Euclid_host

    with pytest.raises(ValueError, match="host memory"):
        batch_kmeans_Euclid_host(torch.zeros(8, 4), 2)  # not (B, N, D)
    with pytest.raises(ValueError):
        batch_kmeans_Euclid_host(torch.zeros(1, 8, 4), 0)
