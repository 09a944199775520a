"""Generates tests/golden/*.npz from the reference's own CUDA kernels.

Run on a GPU box with ``oracle/_ref`` built (``oracle/build_ref.sh``):

    python tests/golden/make_golden.py [outdir]

Inputs are NOT stored: each fixture records the generator call (seeded CPU
torch.Generator, tests/_data.py) plus a checksum of the generated inputs, and
the reference's outputs (labels, sums, counts, centroids). tests/test_golden.py
regenerates the inputs on the CPU, checks the checksum and pins the oracle
(oracle/lloyd.py) against these outputs.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, ROOT)

from _data import iid, mixture, subset_init  # noqa: E402

from oracle.ref_lloyd import Reference  # noqa: E402

# (name, kind, generator spec, K, iterations)
CASES = [
    ("assign_fp16_iid", "assign", dict(fn="iid", B=1, N=4096, D=128, seed=21, dtype="float16"), 256, 0),
    ("assign_bf16_iid", "assign", dict(fn="iid", B=1, N=2048, D=64, seed=22, dtype="bfloat16"), 64, 0),
    ("assign_fp16_mix_k2048", "assign",
     dict(fn="mixture", B=1, N=8192, D=128, n_centres=2048, seed=23, dtype="float16"), 2048, 0),
    ("assign_fp16_d96", "assign", dict(fn="iid", B=2, N=1000, D=96, seed=24, dtype="float16"), 100, 0),
    ("lloyd_fp16_mix", "lloyd",
     dict(fn="mixture", B=1, N=8192, D=128, n_centres=256, seed=25, dtype="float16"), 256, 3),
    ("lloyd_bf16_batched", "lloyd",
     dict(fn="mixture", B=2, N=2048, D=64, n_centres=32, seed=26, dtype="bfloat16"), 32, 3),
    ("lloyd_fp16_zipf_small", "lloyd",
     dict(fn="mixture", B=1, N=4096, D=128, n_centres=300, seed=27, dtype="float16", zipf=1.1),
     300, 2),
    ("lloyd_fp32", "lloyd", dict(fn="iid", B=1, N=2048, D=32, seed=28, dtype="float32"), 16, 2),
]


def make_input(spec: dict) -> torch.Tensor:
    spec = dict(spec)
    fn = spec.pop("fn")
    if fn == "iid":
        return iid(spec["B"], spec["N"], spec["D"], spec["seed"], spec["dtype"])
    return mixture(spec["B"], spec["N"], spec["D"], spec["n_centres"], spec["seed"],
                   spec.get("zipf", 0.0), spec["dtype"])


def checksum(t: torch.Tensor) -> str:
    return hashlib.sha256(t.float().numpy().tobytes()).hexdigest()[:16]


def main(outdir: str = HERE) -> None:
    ref = Reference()
    dev = torch.device("cuda", 0)
    for name, kind, spec, K, iters in CASES:
        x = make_input(spec)
        init = subset_init(x, K, seed=spec["seed"] + 1000)
        meta = dict(name=name, kind=kind, spec=spec, K=K, iters=iters, x_sha=checksum(x),
                    init_sha=checksum(init), torch=torch.__version__,
                    gpu=torch.cuda.get_device_name(0))
        out = {}
        xd, cd = x.to(dev), init.to(dev)
        if kind == "assign":
            out["ids"] = ref.assign(xd, cd).cpu().numpy()
        else:
            ids, cents, n, hist = ref.lloyd(xd, cd, iters, keep_history=True)
            for i, h in enumerate(hist):
                out[f"ids_{i}"] = h["ids"].cpu().numpy()
                out[f"counts_{i}"] = h["counts"].cpu().numpy()
                out[f"sums_{i}"] = h["sums"].cpu().numpy()
                out[f"cents_{i}"] = h["c_out"].float().cpu().numpy()
        np.savez_compressed(os.path.join(outdir, f"ref_{name}.npz"), meta=json.dumps(meta), **out)
        print("wrote", name, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
