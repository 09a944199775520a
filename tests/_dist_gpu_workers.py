"""Rank body for the NCCL multi-GPU test (spawned child processes, one GPU each)."""

from __future__ import annotations

import datetime
import os

import numpy as np
import torch
import torch.distributed as dist


def sharded_rank(rank: int, world: int, port: int, shard: str, out_path: str,
                 multimem: bool = True, tol: float = 0.0) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["FKC_MULTIMEM"] = "1" if multimem else "0"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from _data import mixture, subset_init
    from flash_kmeans_cuda.distributed import (MultimemLloyd, batch_kmeans_Euclid_sharded,
                                               shard_bounds)

    B, N, D, K = (1, 40000, 128, 512) if shard == "N" else (4, 8192, 64, 64)
    x = mixture(B, N, D, K, seed=61, zipf=1.1 if shard == "N" else 0.0)
    init = subset_init(x, K, seed=62)
    if shard == "N":
        n0, n1 = shard_bounds(N, world, rank)
        xl, il = x[:, n0:n1], init
    else:
        b0, b1 = shard_bounds(B, world, rank)
        xl, il = x[b0:b1], init[b0:b1]
    ids, cents, n = batch_kmeans_Euclid_sharded(xl.cuda(), K, max_iters=6 if tol == 0 else 40,
                                                tol=tol, init_centroids=il.cuda(), shard=shard,
                                                gather=True)
    torch.cuda.synchronize()
    if rank == 0:
        np.savez(out_path, ids=ids.cpu().numpy(), cents=cents.float().cpu().numpy(), n=n)
    dist.barrier()
    MultimemLloyd.release_all()
    dist.destroy_process_group()
