"""Rank bodies for the gloo multi-rank tests (spawned processes, CPU only).

``OracleState`` implements the four methods of ``flash_kmeans_cuda.kmeans.LloydState``
with the CPU oracle, so ``batch_kmeans_Euclid_sharded``'s host orchestration
(sharding, init broadcast, the per-iteration all-reduce of sums and counts,
replicated finalize, consistent early stop, label gather) runs on gloo ranks.
"""

from __future__ import annotations

import datetime
import os
import sys
import traceback

import numpy as np
import torch
import torch.distributed as dist


class OracleState:
    def __init__(self, x_local: torch.Tensor, K: int):
        import oracle.lloyd as orc

        self.orc = orc
        self.x = x_local.float().numpy()
        self.K = K
        B, N, D = x_local.shape
        self.ids = torch.empty((B, N), dtype=torch.int32)
        self.sums = torch.empty((B, K, D), dtype=torch.float32)
        self.counts = torch.empty((B, K), dtype=torch.int32)
        self.shift = torch.zeros((1,), dtype=torch.float32)

    def set_centroids(self, c):
        pass

    def local(self, c):
        a = self.orc.assign(self.x, c.float().numpy())
        s, n = self.orc.update(self.x, a.ids, self.K)
        self.ids.copy_(torch.from_numpy(a.ids))
        self.sums.copy_(torch.from_numpy(s.astype(np.float32)))
        self.counts.copy_(torch.from_numpy(n.astype(np.int32)))

    def finalize(self, old, new, want_shift):
        out = self.orc.finalize(self.sums.double().numpy(), self.counts.numpy(),
                                old.float().numpy(), "float32")
        new.copy_(torch.from_numpy(out))
        if want_shift:
            self.shift.fill_(self.orc.shift(out, old.float().numpy()))

    def step(self, old, new, want_shift):
        self.local(old)
        self.finalize(old, new, want_shift)


def _init(rank: int, world: int, port: int, timeout_s: float) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def kmeans_rank(rank: int, world: int, port: int, shard: str, out_path: str, tol: float) -> None:
    from flash_kmeans_cuda.distributed import batch_kmeans_Euclid_sharded, shard_bounds

    _init(rank, world, port, 60.0)
    g = np.random.default_rng(0)
    B, N, D, K = (1, 3001, 8, 12) if shard == "N" else (3, 700, 8, 6)
    centres = g.standard_normal((B, K, D)) * 6
    lab = g.integers(0, K, (B, N))
    x = np.stack([centres[b][lab[b]] for b in range(B)]) + g.standard_normal((B, N, D))
    x = torch.from_numpy(x.astype(np.float32))
    init = x[:, :K].clone()
    if shard == "N":
        n0, n1 = shard_bounds(N, world, rank)
        xl, il = x[:, n0:n1].contiguous(), init
    else:
        b0, b1 = shard_bounds(B, world, rank)
        xl, il = x[b0:b1].contiguous(), init[b0:b1].contiguous()
    ids, cents, n = batch_kmeans_Euclid_sharded(xl, K, max_iters=30, tol=tol, init_centroids=il,
                                                shard=shard, gather=True,
                                                state_factory=OracleState)
    if rank == 0:
        np.savez(out_path, ids=ids.numpy(), cents=cents.numpy(), n=n, x=x.numpy(),
                 init=init.numpy())
    dist.barrier()
    dist.destroy_process_group()


def failing_rank(rank: int, world: int, port: int, out_path: str) -> None:
    """Rank 1 dies before the first all-reduce; rank 0 must get an error, not hang."""
    from flash_kmeans_cuda.distributed import batch_kmeans_Euclid_sharded

    _init(rank, world, port, 10.0)
    x = torch.randn(1, 100, 4)
    if rank == 1:
        os._exit(3)
    try:
        batch_kmeans_Euclid_sharded(x, 4, max_iters=5, init_centroids=x[:, :4].clone(),
                                    state_factory=OracleState)
        status = "no-error"
    except Exception as e:  # noqa: BLE001
        status = "error:" + type(e).__name__
    with open(out_path, "w") as f:
        f.write(status)
    os._exit(0)


def mismatched_rank(rank: int, world: int, port: int, out_path: str) -> None:
    """Rank 1 holds rows of another width: every rank must raise, none may hang."""
    from flash_kmeans_cuda.distributed import batch_kmeans_Euclid_sharded

    _init(rank, world, port, 20.0)
    x = torch.randn(1, 100, 4 if rank == 0 else 5)
    try:
        batch_kmeans_Euclid_sharded(x, 4, max_iters=3, state_factory=OracleState)
        status = "no-error"
    except ValueError as e:
        status = "error:ValueError:" + str(e)
    except Exception as e:  # noqa: BLE001
        status = "error:" + type(e).__name__
    with open(f"{out_path}.{rank}", "w") as f:
        f.write(status)
    os._exit(0)


def stalled_rank(rank: int, world: int, port: int, out_path: str) -> None:
    """Rank 1 stalls longer than the process-group timeout before its first collective:
    rank 0's collective must end with an error after the timeout, not hang."""
    import time

    from flash_kmeans_cuda.distributed import batch_kmeans_Euclid_sharded

    _init(rank, world, port, 3.0)
    x = torch.randn(1, 100, 4)
    if rank == 1:
        time.sleep(20.0)
        os._exit(0)
    t0 = time.time()
    try:
        batch_kmeans_Euclid_sharded(x, 4, max_iters=3, state_factory=OracleState)
        status = "no-error"
    except Exception as e:  # noqa: BLE001
        status = f"error:{type(e).__name__}:{time.time() - t0:.1f}"
    with open(out_path, "w") as f:
        f.write(status)
    os._exit(0)

