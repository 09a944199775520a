"""Capacity of the fused update's unit table (no GPU).

The scan lays out, per batch row, ceil(count / 64) units for every cluster holding more
than 64 rows, in a table of cap = 2 * ceil(N / 64) entries (update.cu: plan_cap). The
device code writes without a bound check, so the bound must hold for every histogram
of N rows: sum over clusters with c > 64 of ceil(c / 64) <= N/64 + #(c > 64) <= 2N/64."""

from __future__ import annotations

import numpy as np
import pytest

UNIT = 64


def units_needed(counts: np.ndarray) -> int:
    big = counts[counts > UNIT]
    return int(((big + UNIT - 1) // UNIT).sum())


def cap(n: int) -> int:
    return 2 * ((n + UNIT - 1) // UNIT)


@pytest.mark.parametrize("seed", range(20))
def test_random_histograms_fit(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 200_000))
    k = int(rng.integers(1, 5000))
    p = rng.dirichlet(np.full(k, float(rng.choice([0.05, 0.5, 5.0]))))
    counts = rng.multinomial(n, p)
    assert units_needed(counts) <= cap(n)


@pytest.mark.parametrize("n", [65, 129, 6500, 65 * 1000, 2 ** 20 + 3])
def test_adversarial_histograms_fit(n):
    # clusters of 65 rows (just above one unit) maximise units per row
    k, rem = divmod(n, UNIT + 1)
    counts = np.array([UNIT + 1] * k + ([rem] if rem else []))
    assert counts.sum() == n
    assert units_needed(counts) <= cap(n)
    # one cluster holding everything
    assert units_needed(np.array([n])) <= cap(n)
    # 128-row clusters (exactly two units each)
    k2, rem2 = divmod(n, 2 * UNIT)
    counts2 = np.array([2 * UNIT] * k2 + ([rem2] if rem2 else []))
    assert units_needed(counts2) <= cap(n)
