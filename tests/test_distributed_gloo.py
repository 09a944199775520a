"""World-size-2 gloo tests (CPU) of the multi-GPU driver's host logic.

The per-rank compute is the CPU oracle (tests/_dist_workers.py:OracleState);
what is under test is flash_kmeans_cuda.distributed: N-sharding with one
all-reduce of sums and counts per iteration, B-sharding with a max-reduced
shift, replicated finalize, consistent early stop, label gathering, and
failure surfacing when a rank dies (no hang).
"""

from __future__ import annotations

import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

import oracle.lloyd as orc


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("shard,tol", [("N", 0.0), ("N", 1e-5), ("B", 0.0), ("B", 1e-5)])
def test_sharded_matches_single_process(tmp_path, shard, tol):
    from _dist_workers import kmeans_rank

    out = str(tmp_path / "r.npz")
    mp.start_processes(kmeans_rank, args=(2, _port(), shard, out, tol), nprocs=2,
                       start_method="spawn", join=True)
    r = np.load(out)
    ref = orc.lloyd(r["x"], r["init"], 30, tol, "float32")
    assert int(r["n"]) == ref.n_iters
    assert (r["ids"] == ref.ids).mean() >= 0.999
    np.testing.assert_allclose(r["cents"], ref.centroids, rtol=1e-4, atol=1e-4)


def test_dead_rank_surfaces_as_error(tmp_path):
    from _dist_workers import failing_rank

    out = str(tmp_path / "status.txt")
    t0 = time.time()
    ctx = mp.start_processes(failing_rank, args=(2, _port(), out), nprocs=2,
                             start_method="spawn", join=False)
    deadline = t0 + 120
    while time.time() < deadline and not all(not p.is_alive() for p in ctx.processes):
        time.sleep(0.2)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    assert os.path.exists(out), "rank 0 neither finished nor reported"
    assert open(out).read().startswith("error:")
    assert time.time() - t0 < 120


def _run(fn, args, deadline_s):
    t0 = time.time()
    ctx = mp.start_processes(fn, args=args, nprocs=2, start_method="spawn", join=False)
    while time.time() - t0 < deadline_s and any(p.is_alive() for p in ctx.processes):
        time.sleep(0.2)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    return time.time() - t0


def test_mismatched_shards_raise_on_every_rank(tmp_path):
    from _dist_workers import mismatched_rank

    out = str(tmp_path / "status")
    elapsed = _run(mismatched_rank, (2, _port(), out), 90)
    for r in range(2):
        status = open(f"{out}.{r}").read()
        assert status.startswith("error:ValueError"), status
        assert "rank 1" in status
    assert elapsed < 90


def test_stalled_rank_times_out_instead_of_hanging(tmp_path):
    from _dist_workers import stalled_rank

    out = str(tmp_path / "status.txt")
    elapsed = _run(stalled_rank, (2, _port(), out), 90)
    status = open(out).read()
    assert status.startswith("error:"), status
    waited = float(status.rsplit(":", 1)[1])
    assert 2.0 <= waited < 20.0  # the 3 s process-group timeout, not the peer's 20 s stall
    assert elapsed < 90

