"""The counting sort behind the centroid update, restated in Python (no GPU).

update.cu: the histogram (fused into the assignment) gives counts; scan_kernel writes
offsets = exclusive prefix of counts and cursor = offsets; scatter_chunk_kernel ranks the
rows of each chunk per cluster in shared memory, claims [base, base + local count) of each
cluster it holds with one atomic add on cursor, and writes perm[base + rank] = row.
Whatever order the chunks claim in, the result must place every row once, inside its
cluster's range [offset, offset + count)."""

from __future__ import annotations

import numpy as np
import pytest


def counting_sort(ids: np.ndarray, K: int, chunk: int, claim_order: np.ndarray) -> np.ndarray:
    N = ids.shape[0]
    counts = np.bincount(ids, minlength=K)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]])
    cursor = offsets.copy()
    perm = np.full(N, -1, dtype=np.int64)
    nchunks = (N + chunk - 1) // chunk
    for c in claim_order[:nchunks]:
        r0, r1 = c * chunk, min((c + 1) * chunk, N)
        lab = ids[r0:r1]
        local = np.zeros(K, dtype=np.int64)
        rank = np.empty(r1 - r0, dtype=np.int64)
        for i, k in enumerate(lab):  # shared-memory atomics in the kernel
            rank[i] = local[k]
            local[k] += 1
        base = np.zeros(K, dtype=np.int64)
        for k in np.nonzero(local)[0]:  # one global claim per (chunk, cluster)
            base[k] = cursor[k]
            cursor[k] += local[k]
        pos = base[lab] + rank
        assert (pos < N).all()
        perm[pos] = np.arange(r0, r1)
    return perm, offsets, counts


@pytest.mark.parametrize("seed", range(10))
def test_every_row_lands_once_in_its_cluster_range(seed):
    rng = np.random.default_rng(seed)
    N = int(rng.integers(1, 20000))
    K = int(rng.integers(1, 3000))
    p = rng.dirichlet(np.full(K, 0.3))
    ids = rng.choice(K, size=N, p=p)
    chunk = int(rng.choice([512, 1024, 4096]))
    order = rng.permutation((N + chunk - 1) // chunk)  # any claim order
    perm, offsets, counts = counting_sort(ids, K, chunk, order)
    assert sorted(perm.tolist()) == list(range(N))
    for k in np.nonzero(counts)[0][:200]:
        rows = perm[offsets[k]:offsets[k] + counts[k]]
        assert (ids[rows] == k).all()
