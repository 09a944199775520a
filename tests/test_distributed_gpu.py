"""NCCL multi-GPU run (2 ranks, child processes) of the sharded Lloyd loop against
the single-GPU loop on the same data and initial centroids. Skipped with < 2 GPUs."""

from __future__ import annotations

import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("shard,multimem,tol", [
    ("N", True, 0.0),    # sums/counts reduced inside the finalize over NVLink multicast
    ("N", True, 1e-3),   # ... with the shift max-reduced over multicast and tol applied
    ("N", False, 0.0),   # NCCL all-reduce of sums/counts
    ("B", True, 0.0),    # independent batch elements: no per-iteration collective
])
def test_two_gpu_sharded_matches_single_gpu(tmp_path, shard, multimem, tol):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from _data import mixture, subset_init
    from _dist_gpu_workers import sharded_rank

    from flash_kmeans_cuda import batch_kmeans_Euclid

    out = str(tmp_path / "r.npz")
    mp.start_processes(sharded_rank, args=(2, _port(), shard, out, multimem, tol), nprocs=2,
                       start_method="spawn", join=True)
    r = np.load(out)
    B, N, D, K = (1, 40000, 128, 512) if shard == "N" else (4, 8192, 64, 64)
    x = mixture(B, N, D, K, seed=61, zipf=1.1 if shard == "N" else 0.0)
    init = subset_init(x, K, seed=62)
    ids, cents, n = batch_kmeans_Euclid(x.cuda(), K, max_iters=6 if tol == 0 else 40, tol=tol,
                                        init_centroids=init.cuda())
    assert int(r["n"]) == n
    agree = (r["ids"] == ids.cpu().numpy()).mean()
    assert agree >= 0.999, agree
    c1 = cents.float().cpu().numpy()
    close = np.abs(r["cents"] - c1) <= 2e-3 * np.abs(c1) + 2 ** -9
    assert close.mean() >= 0.999
