"""The epilogue's packed-key argmax, restated in numpy (no GPU).

Scores are negative floats (-||x-c||^2/2 - delta). Per group of 32 columns the epilogue
replaces the 5 low mantissa bits of each score with the column's position j
((bits & ~31) | j, one lop3), takes the float max, and folds the group winner into the
running best per row only if its truncated score is strictly larger (assign_tc.cu:
pack_key, group_max, merge_best). So the result is the exact argmax wherever the best
score beats the runner-up by more than 32 ulps, and exact ties go to the lowest column."""

from __future__ import annotations

import numpy as np


def packed_argmax(scores: np.ndarray) -> np.ndarray:
    rows, cols = scores.shape
    assert (scores < 0).all()
    bits = scores.astype(np.float32).view(np.uint32)
    best_val = np.full(rows, -np.inf, dtype=np.float32)
    best_idx = np.zeros(rows, dtype=np.int64)
    for g0 in range(0, cols, 32):
        blk = bits[:, g0:g0 + 32]
        j = np.arange(blk.shape[1], dtype=np.uint32)
        keys = ((blk & np.uint32(0xFFFFFFE0)) | j).view(np.float32)
        m = keys.max(axis=1).view(np.uint32)
        mt = (m & np.uint32(0xFFFFFFE0)).view(np.float32)
        cand = g0 + (m & np.uint32(31)).astype(np.int64)
        take = mt > best_val
        best_val = np.where(take, mt, best_val)
        best_idx = np.where(take, cand, best_idx)
    return best_idx


def test_matches_exact_argmax_outside_32_ulps():
    rng = np.random.default_rng(0)
    s = -(rng.uniform(0.01, 100.0, (3000, 300))).astype(np.float32)
    got = packed_argmax(s)
    exact = s.argmax(axis=1)
    srt = np.sort(s.astype(np.float64), axis=1)
    gap = srt[:, -1] - srt[:, -2]
    clear = gap > 2.0 ** -18 * np.abs(srt[:, -1])
    assert clear.mean() > 0.9
    assert (got[clear] == exact[clear]).all()


def test_exact_ties_go_to_the_lowest_column():
    rng = np.random.default_rng(1)
    s = -(rng.uniform(1.0, 2.0, (500, 256))).astype(np.float32)
    for r in range(500):
        cols = np.sort(rng.choice(256, size=3, replace=False))
        s[r, cols] = np.float32(-0.5)  # three equal best scores, in different groups or not
        assert packed_argmax(s[r:r + 1])[0] == cols[0]
