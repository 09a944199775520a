"""Pins the oracle (oracle/lloyd.py) against outputs of the reference's own CUDA
kernels (tests/golden/ref_*.npz, produced by tests/golden/make_golden.py on a
B200 from the reference built by oracle/build_ref.sh). CPU only.

The reference accumulates x.c in fp16 (flash_kmeans_cuda/csrc/common/ptx.cuh:151-170),
so its labels are only pinned where the exact top-2 gap is large; its own
tests allow 3% disagreement with an fp32 einsum (tests/test_mma_optin.py:60-67).
Its update and finalize are pinned exactly (counts) and to fp32 rounding
(sums, centroids), teacher-forced on the reference's own labels.
"""

from __future__ import annotations

import glob
import json
import os

import numpy as np
import pytest

import oracle.lloyd as orc
from _data import subset_init, to_np

HERE = os.path.dirname(os.path.abspath(__file__))
FILES = sorted(glob.glob(os.path.join(HERE, "golden", "ref_*.npz")))

# Rows whose exact top-2 gap exceeds this fraction of ||x||^2 must carry the
# same label in the reference (fp16 accumulation error stays well below it).
REF_GAP = 3e-2
DTYPE_ULP = {"float16": 2.0 ** -10, "bfloat16": 2.0 ** -7, "float32": 2.0 ** -23}


def _load(path):
    import sys

    sys.path.insert(0, os.path.join(HERE, "golden"))
    from make_golden import checksum, make_input

    z = np.load(path)
    meta = json.loads(str(z["meta"]))
    x = make_input(meta["spec"])
    assert checksum(x) == meta["x_sha"], "input generator drifted from the fixture"
    init = subset_init(x, meta["K"], seed=meta["spec"]["seed"] + 1000)
    assert checksum(init) == meta["init_sha"]
    return meta, z, to_np(x), to_np(init)


def test_fixtures_present():
    if not FILES:
        pytest.skip("no golden fixtures (generate with tests/golden/make_golden.py on a GPU)")
    assert len(FILES) >= 6


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(f)[4:-4] for f in FILES])
def test_oracle_matches_reference_outputs(path):
    meta, z, x, init = _load(path)
    dtype = meta["spec"]["dtype"]
    K = meta["K"]
    if meta["kind"] == "assign":
        a = orc.assign(x, init)
        ref_ids = z["ids"]
        sure = a.gap_mask(REF_GAP)
        assert (ref_ids[sure] == a.ids[sure]).all()
        assert (ref_ids == a.ids).mean() >= 0.97
        return
    cur = init
    for i in range(meta["iters"]):
        ref_ids = z[f"ids_{i}"]
        a = orc.assign(x, cur)
        sure = a.gap_mask(REF_GAP)
        assert (ref_ids[sure] == a.ids[sure]).all(), f"iter {i}: labels"
        assert (ref_ids == a.ids).mean() >= 0.97
        # update + finalize teacher-forced on the reference's labels
        sums, counts = orc.update(x, ref_ids, K)
        assert np.array_equal(counts, z[f"counts_{i}"]), f"iter {i}: counts"
        scale = orc.update(np.abs(x), ref_ids, K)[0] + 1e-6
        assert (np.abs(sums - z[f"sums_{i}"]) / scale).max() < 1e-5, f"iter {i}: sums"
        new = orc.finalize(sums, counts, cur, dtype)
        ref_new = z[f"cents_{i}"]
        tol = (1e-3 + DTYPE_ULP[dtype]) * np.abs(ref_new) + 1e-6
        assert (np.abs(new - ref_new) <= tol).all(), f"iter {i}: centroids"
        cur = ref_new  # follow the reference's trajectory
