"""Seeded synthetic inputs shaped like the benchmark configurations (test helper).

The reference benchmarks on synthetic data; these generators follow the
shapes and distributions of its configurations: Gaussian mixtures with
centres ~ N(0, 4 I) and unit noise, optionally Zipf(1.1)-sized clusters,
or iid N(0, 1) points. Data are generated on the CPU with torch.Generator so
the oracle and the GPU path see identical values.
"""

from __future__ import annotations

import numpy as np
import torch

TORCH_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def mixture(B: int, N: int, D: int, n_centres: int, seed: int, zipf: float = 0.0,
            dtype: str = "float16") -> torch.Tensor:
    """(B, N, D) CPU tensor of `dtype`: centre ~ N(0, 4I) + N(0, I) noise."""
    out = []
    for b in range(B):
        g = torch.Generator().manual_seed(seed + b)
        centres = 2.0 * torch.randn((n_centres, D), generator=g)
        if zipf > 0:
            p = torch.arange(1, n_centres + 1, dtype=torch.float64) ** (-zipf)
            p = p / p.sum()
            lab = torch.multinomial(p, N, replacement=True, generator=g)
            lab = torch.randperm(n_centres, generator=g)[lab]
        else:
            lab = torch.randint(0, n_centres, (N,), generator=g)
        out.append(centres[lab] + torch.randn((N, D), generator=g))
    return torch.stack(out).to(TORCH_DTYPES[dtype])


def iid(B: int, N: int, D: int, seed: int, dtype: str = "float16") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn((B, N, D), generator=g).to(TORCH_DTYPES[dtype])


def subset_init(x: torch.Tensor, K: int, seed: int) -> torch.Tensor:
    """K distinct rows of each batch element (seeded randperm)."""
    B, N, D = x.shape
    g = torch.Generator().manual_seed(seed)
    return torch.stack([x[b, torch.randperm(N, generator=g)[:K]] for b in range(B)]).contiguous()


def to_np(t: torch.Tensor) -> np.ndarray:
    """float32 numpy copy of a (CPU or CUDA) tensor of any float dtype."""
    return t.detach().float().cpu().numpy()
