"""The reference's Lloyd iteration driven through the reference's own CUDA kernels.

TEST INFRASTRUCTURE ONLY (see ``oracle/lloyd.py`` for the rule on who may
import ``oracle/``). Requires ``oracle/_ref/`` built by ``oracle/build_ref.sh``
and a CUDA device. The glue restates the reference's Python layer, step by step:

* assign:   ``ops.euclid_assign`` (flash_kmeans_cuda/ops.py:30-55): c_sq
            defaults to ``(c.float()**2).sum(-1)``; x_sq as computed fp32 norms.
* update:   ``ops.centroid_update_sorted`` (ops.py:58-112): ``torch.sort`` of the
            labels, then the indexed kernel for fp16 / D == 128 / K >= 256, else a
            ``gather``-materialised ``x_sorted`` and the sorted kernel. The
            libtorch ``fkc::`` entry points zero sums/counts (api.cpp:74-95).
* finalize: ``fkc::centroid_finalize_out`` (api.cpp:105-113).
* loop:     ``kmeans.py:73-105,165-195`` with explicit initial centroids.
"""

from __future__ import annotations

import importlib
import os
import sys
from typing import List, Optional, Tuple

import torch

REF_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref")


def available() -> bool:
    return os.path.isdir(REF_DIR) and any(f.startswith("fkc_ref_shim") for f in os.listdir(REF_DIR))


def load():
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    return importlib.import_module("fkc_ref_shim")


class Reference:
    def __init__(self):
        self.m = load()

    def assign(self, x: torch.Tensor, c: torch.Tensor, x_sq: Optional[torch.Tensor] = None,
               c_sq: Optional[torch.Tensor] = None) -> torch.Tensor:
        if c_sq is None:
            c_sq = (c.float() ** 2).sum(dim=-1).contiguous()
        if x_sq is None:
            x_sq = (x.float() ** 2).sum(dim=-1).contiguous()
        return self.m.euclid_assign(x.contiguous(), c.contiguous(), x_sq, c_sq)

    def update(self, x: torch.Tensor, ids: torch.Tensor, K: int) -> Tuple[torch.Tensor, torch.Tensor]:
        B, N, D = x.shape
        ids = ids.to(torch.int32).contiguous()
        sorted_ids, perm = torch.sort(ids, dim=1, stable=False)
        sorted_ids = sorted_ids.contiguous()
        sums = torch.empty((B, K, D), device=x.device, dtype=torch.float32)
        counts = torch.empty((B, K), device=x.device, dtype=torch.int32)
        if x.dtype == torch.float16 and D == 128 and K >= 256:
            self.m.centroid_update_sorted_indexed(x, perm.contiguous().to(torch.int32), sorted_ids,
                                                  sums, counts)
        else:
            x_sorted = torch.gather(x, 1, perm.unsqueeze(-1).expand(-1, -1, D)).contiguous()
            self.m.centroid_update_sorted(x_sorted, sorted_ids, sums, counts)
        return sums, counts

    def finalize(self, sums: torch.Tensor, counts: torch.Tensor, old: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(old)
        self.m.centroid_finalize_out(sums, counts, old.contiguous(), out)
        return out

    def lloyd(self, x: torch.Tensor, init: torch.Tensor, max_iters: int, tol: float = 0.0,
              keep_history: bool = False):
        """Returns (ids, centroids, n_iters, history)."""
        x = x.contiguous()
        K = init.shape[1]
        x_sq = (x.float() ** 2).sum(dim=-1).contiguous()
        cur = init.contiguous().clone()
        ids = None
        hist: List[dict] = []
        n = 0
        for it in range(max_iters):
            ids = self.assign(x, cur, x_sq=x_sq)
            sums, counts = self.update(x, ids, K)
            new = self.finalize(sums, counts, cur)
            n = it + 1
            if keep_history:
                hist.append(dict(c_in=cur, ids=ids, sums=sums, counts=counts, c_out=new))
            shift = (new.float() - cur.float()).norm(dim=-1).max().item() if tol > 0 else None
            cur = new
            if tol > 0 and shift < tol:
                break
        return ids, cur, n, hist
