"""Benchmark of the B200 Lloyd iteration (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c3] [--impl ours|reference]

A *step* is one Lloyd iteration (assign -> counting-sort update -> finalize)
over the whole problem of the workload. ``value`` is ms per iteration of the
whole job (max over ranks, CUDA events, inputs resident in HBM); for N > 1
the points are sharded over the ranks (strong scaling: fixed total problem)
with one NCCL all-reduce of sums and counts per iteration.

Workloads (seeded synthetic data of those shapes and
distributions, generated on the device):
  c2  B=1  N=131072   K=2048  D=128 fp16, mixture N(0,4I)+N(0,I)
  c3  B=1  N=524288   K=8192  D=128 fp16, mixture with Zipf(1.1) cluster sizes  [default]
  c4  B=32 N=16384    K=1024  D=64  bf16, independent mixtures per b (sharded over B)
  c5  B=1  N=2^24     K=65536 D=128 fp16, iid N(0,1)

Extra keys: ``roofline`` for the assignment kernel (tensor-bound, against the
measured bf16/fp16 dense peak), ``update`` (HBM-bound, GB/s), ``e2e`` (the same
metric through ``batch_kmeans_Euclid`` with host-resident inputs copied in and
results copied out inside the timed region), ``e2e_device`` (whole
``batch_kmeans_Euclid`` calls on device-resident x, the reference's own
end-to-end definition), ``parity`` (labels of the last timed step on a fixed
row subset against a float64 assignment, counts against the label histogram),
``per_rank`` (N > 1: each rank's local step, reduction and barrier times),
``cpu_baseline`` (multi-threaded CPU Lloyd loop on a bounded sample, scaled to
the whole workload), ``cpu_baseline_c1`` (BASELINE config 1 in full on the host
cores), ``clocks`` (nvidia-smi samples during the timed region) and
``gpu_launches``.

``--impl reference`` times the reference's loop on the host cores (its CPU
port on a sample of the workload's own distribution) and adds
``reference_gpu``: the reference's own CUDA kernels, built from its sources
under oracle/_ref, on the whole workload on GPU 0.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "flash-kmeans-cuda_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

WORKLOADS = {
    "c2": dict(B=1, N=131072, K=2048, D=128, dtype="float16", data="mixture", zipf=0.0,
               shard="N", iters=20),
    "c3": dict(B=1, N=524288, K=8192, D=128, dtype="float16", data="mixture", zipf=1.1,
               shard="N", iters=10),
    "c4": dict(B=32, N=16384, K=1024, D=64, dtype="bfloat16", data="mixture", zipf=0.0,
               shard="B", iters=10),
    "c5": dict(B=1, N=1 << 24, K=65536, D=128, dtype="float16", data="iid", zipf=0.0,
               shard="N", iters=5),
}
TDT = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}
DT_SHORT = {"float16": "fp16", "bfloat16": "bf16", "float32": "fp32"}
L2_BYTES = 126 * 1024 * 1024


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# --------------------------------------------------------------------------- data
def make_data(w: dict, device, seed: int = 0, n_rows=None, dtype=None):
    """(B, N, D) points and (B, K, D) initial centroids (seeded subset of the points).

    ``n_rows`` draws that many points per batch element from the same distribution
    (a sample, for the CPU timings); ``dtype`` overrides the workload's dtype."""
    B, N, K, D = w["B"], w["N"], w["K"], w["D"]
    if n_rows is not None:
        N = int(n_rows)
    g = torch.Generator(device=device).manual_seed(seed)
    xs = []
    for b in range(B):
        if w["data"] == "iid":
            xb = torch.randn((N, D), generator=g, device=device)
        else:
            nc = K
            centres = 2.0 * torch.randn((nc, D), generator=g, device=device)
            if w["zipf"] > 0:
                p = torch.arange(1, nc + 1, device=device, dtype=torch.float64) ** (-w["zipf"])
                lab = torch.multinomial((p / p.sum()).float(), N, replacement=True, generator=g)
                lab = torch.randperm(nc, generator=g, device=device)[lab]
            else:
                lab = torch.randint(0, nc, (N,), generator=g, device=device)
            xb = centres[lab]
            xb.add_(torch.randn((N, D), generator=g, device=device))
        xs.append(xb.to(dtype or TDT[w["dtype"]]))
        del xb
    x = torch.stack(xs)
    del xs
    init = torch.stack([x[b, torch.randperm(N, generator=g, device=device)[:K]]
                        for b in range(B)]).contiguous()
    return x, init


# ------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (every 200 ms) of the bench's GPU during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu), "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append(dict(sm=float(parts[1]), smax=float(parts[2]),
                                     power=float(parts[3]), hw=parts[5], hwt=parts[6],
                                     swt=parts[7], pcap=parts[8]))
                except ValueError:
                    continue
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        loaded = [r for r in rows if r["power"] > 250] or rows
        reasons = set()
        for r in loaded:
            for k, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                            ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[k].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded),
                "sm_max_mhz": max(r["smax"] for r in rows), "reasons": sorted(reasons),
                "samples": len(rows), "samples_under_load": len(loaded),
                "power_w_max": max(r["power"] for r in rows)}


# ---------------------------------------------------------------------- helpers
def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(tflops=d["bf16_tflops"], tflops_sustained=d.get("bf16_tflops_sustained"),
                    hbm=d["hbm_gbs"], src="measured")
    return dict(tflops=1590.0, tflops_sustained=1400.0, hbm=6650.0, src="fallback")


def tensor_peak(peaks: dict, launch_ms: float):
    """Roofline denominator for an assign launch of launch_ms: the burst GEMM figure for
    launches about as long as the measured burst GEMMs, the sustained (power-capped) one
    for launches of tens of milliseconds and more (c5), which run under the power cap."""
    if launch_ms > 20.0 and peaks.get("tflops_sustained"):
        return peaks["tflops_sustained"], f"{peaks['src']} bf16 dense sustained"
    return peaks["tflops"], f"{peaks['src']} bf16 dense burst"


def profiled_traffic(workload: str):
    """DRAM bytes per assign launch from the committed ncu summary, if present."""
    p = ROOT / "profiles" / f"assign_tc_{workload}.md"
    if not p.exists():
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


def max_over_ranks(v: float, device) -> float:
    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return v


def barrier_sync(device):
    torch.cuda.synchronize(device)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
    torch.cuda.synchronize(device)


# ------------------------------------------------------------------ CPU timings
def cpu_sample_rows(w: dict, target_s: float) -> tuple:
    """Rows of one batch element whose CPU iteration takes ~target_s seconds."""
    from oracle.cpu_lloyd import time_lloyd_cpu

    n = 4096
    t = time_lloyd_cpu(1, n, w["K"], w["D"], 1, repeats=1)["seconds"]
    n2 = int(min(w["N"], max(1024, n * target_s / max(t, 1e-3))))
    return n2, t * n2 / n


def cpu_baseline(w: dict, workload: str) -> dict:
    from oracle.cpu_lloyd import time_lloyd_cpu

    n_s, _ = cpu_sample_rows(w, target_s=3.0)
    r = time_lloyd_cpu(1, n_s, w["K"], w["D"], iters=1, repeats=3)
    scale = (w["B"] * w["N"]) / n_s
    return {"value": r["ms_per_iter"] * scale, "unit": "ms/iter", "cores": r["threads"],
            "kind": "port",
            "sample": (f"{workload}: 1 iteration on {n_s} of {w['B'] * w['N']} points "
                       f"(full K={w['K']}, D={w['D']}, fp32 CPU PyTorch Lloyd loop, "
                       f"oracle/cpu_lloyd.py), median of 3, scaled by {scale:.1f}x")}


def cpu_baseline_c1() -> dict:
    """BASELINE config 1 in full on the host cores: B=1, N=32768, K=256, D=128 fp32, iid
    N(0, 1) from seed 0, K rows of a seeded randperm as initial centroids, 10 iterations,
    median of 3 (the CPU PyTorch Lloyd loop of oracle/cpu_lloyd.py)."""
    from oracle.cpu_lloyd import time_lloyd_cpu

    r = time_lloyd_cpu(1, 32768, 256, 128, iters=10, seed=0, repeats=3)
    return {"value": r["ms_per_iter"], "unit": "ms/iter", "cores": r["threads"], "kind": "port",
            "sample": "c1 in full: B=1 N=32768 K=256 D=128 fp32 iid, 10 iterations, median of 3"}


def sample_parity(x: torch.Tensor, c: torch.Tensor, ids: torch.Tensor, counts: torch.Tensor,
                  max_rows: int = 8192) -> dict:
    """Labels of a fixed, evenly strided subset of rows against a float64 restatement
    of the assignment (argmin_k ||x||^2 + ||c||^2 - 2 x.c, ties to the lowest index)
    computed on the device with torch (no code of this library), and the counts
    against the histogram of all labels (exact)."""
    B, N, D = x.shape
    K = c.shape[1]
    total = B * N
    n_s = int(min(total, max_rows, max(256, (1 << 27) // K)))
    flat = torch.linspace(0, total - 1, n_s, device=x.device).round().to(torch.int64).unique()
    bb, nn = flat // N, flat % N
    mismatch, agree, near = 0, 0, 0
    for b in bb.unique().tolist():
        sel = nn[bb == b]
        xr = x[b, sel].to(torch.float64)
        cb = c[b].to(torch.float64)
        x_sq = (xr * xr).sum(-1)
        dist = x_sq[:, None] + (cb * cb).sum(-1)[None, :] - 2.0 * (xr @ cb.T)
        best, exact = dist.min(dim=1)  # first occurrence: the lowest index on ties
        if K > 1:
            dist[torch.arange(dist.shape[0], device=x.device), exact] = float("inf")
            gap_ok = (dist.min(dim=1).values - best) > 1e-3 * x_sq
        else:
            gap_ok = torch.ones_like(best, dtype=torch.bool)
        got = ids[b, sel].to(torch.int64)
        mismatch += int(((got != exact) & gap_ok).sum())
        agree += int((got == exact).sum())
        near += int((~gap_ok).sum())
        del dist
    hist_ok = all(torch.equal(torch.bincount(ids[b].to(torch.int64), minlength=K).to(torch.int32),
                              counts[b]) for b in range(B))
    return {"rows": int(flat.numel()), "labels_above_gap_mismatch": mismatch,
            "agree": agree / max(1, int(flat.numel())), "near_tie_rows": near,
            "counts_exact": bool(hist_ok)}


def reduce_parity(p: dict, device) -> dict:
    """Sums the per-rank parity counts (every rank calls it)."""
    if not (dist.is_initialized() and dist.get_world_size() > 1):
        return p
    t = torch.tensor([p["rows"], p["labels_above_gap_mismatch"], round(p["agree"] * p["rows"]),
                      p["near_tie_rows"], 0 if p["counts_exact"] else 1], device=device,
                     dtype=torch.float64)
    dist.all_reduce(t)
    rows = int(t[0].item())
    return {"rows": rows, "labels_above_gap_mismatch": int(t[1].item()),
            "agree": float(t[2].item()) / max(1, rows), "near_tie_rows": int(t[3].item()),
            "counts_exact": int(t[4].item()) == 0}


def time_reference_gpu(w: dict, steps: int, warmup: int, device) -> dict:
    """The reference's own CUDA kernels (oracle/_ref, built from its sources) on the whole
    workload on one GPU: a step is one iteration of the reference's loop (c_sq,
    fkc::euclid_assign, torch.sort + sorted/indexed accumulate, finalize)."""
    from oracle import ref_lloyd

    if not ref_lloyd.available():
        return {"unavailable": "oracle/_ref not built (oracle/build_ref.sh needs the reference "
                               "sources)"}
    ref = ref_lloyd.Reference()
    x, init = make_data(w, device, seed=0)
    K = w["K"]
    x_sq = (x.float() ** 2).sum(-1).contiguous()
    cur = [init.clone()]

    def step():
        c = cur[0]
        c_sq = (c.float() ** 2).sum(dim=-1).contiguous()
        ids = ref.assign(x, c, x_sq=x_sq, c_sq=c_sq)
        sums, counts = ref.update(x, ids, K)
        cur[0] = ref.finalize(sums, counts, c)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clk:
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / steps
    c = cur[0]
    c_sq = (c.float() ** 2).sum(dim=-1).contiguous()
    reps = 3
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ref.assign(x, c, x_sq=x_sq, c_sq=c_sq)
    a0.record()
    for _ in range(reps):
        ref.assign(x, c, x_sq=x_sq, c_sq=c_sq)
    a1.record()
    torch.cuda.synchronize(device)
    t_assign = a0.elapsed_time(a1) / reps
    flops = 2.0 * w["B"] * w["N"] * K * w["D"]
    peaks = measured_peaks()
    tf = flops / (t_assign * 1e-3) / 1e12
    peak, peak_src = tensor_peak(peaks, t_assign)
    del x, init, x_sq, cur
    torch.cuda.empty_cache()
    return {"ms_per_iter": ms, "assign_ms": t_assign, "assign_tflops": tf,
            "assign_frac": tf / peak, "peak_src": peak_src, "steps": steps, "warmup": warmup,
            "kernel": "reference assign_sm80_kernel (mma.sync, fp16 accumulation), built from "
                      "its sources for sm_100",
            "clocks": clk.summary()}


def run_reference_gpu(args, w: dict) -> None:
    """``--ref-device cuda``: the reference's own CUDA kernels as the line's value."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    r = time_reference_gpu(w, args.steps, args.warmup, dev)
    if "unavailable" in r:
        print(json.dumps({"impl": "reference", "unavailable": r["unavailable"]}))
        return
    ms = r["ms_per_iter"]
    print(json.dumps({
        "metric": "K-Means ms/iter", "value": ms, "unit": "ms/iter", "impl": "reference",
        "device": "cuda", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": DT_SHORT[w["dtype"]], "data": "synthetic",
        "config": {"workload": args.workload, "B": w["B"], "N": w["N"], "K": w["K"],
                   "D": w["D"], "parallelism": "dp1"},
        "assign_ms": r["assign_ms"], "assign_tflops": r["assign_tflops"],
        "roofline": {"bound": "tensor", "achieved": r["assign_tflops"],
                     "peak": r["assign_tflops"] / r["assign_frac"], "unit": "TFLOP/s",
                     "frac": r["assign_frac"], "kernel": r["kernel"]},
        "clocks": r["clocks"],
    }), flush=True)


def run_reference_arm(args, w: dict) -> None:
    """The reference's loop on the host cores (rank 0 only): the CPU port of its Lloyd
    iteration (the reference has no CPU path of its own) on a bounded sample of the
    workload's own data distribution, plus, as ``reference_gpu``, the reference's own
    CUDA kernels (built from its sources) on the whole workload on GPU 0."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.ref_device == "cuda":
        run_reference_gpu(args, w)
        return
    from oracle.cpu_lloyd import lloyd_cpu

    # About a second per step, less for long runs: the whole arm stays near two minutes.
    target = min(1.0, 120.0 / max(1, args.steps + args.warmup))
    n_s, _ = cpu_sample_rows(w, target_s=target)
    torch.set_num_threads(os.cpu_count() or 1)
    # one batch element's worth of points drawn from the workload's distribution
    w1 = dict(w, B=1)
    x, init = make_data(w1, torch.device("cpu"), seed=0, n_rows=n_s, dtype=torch.float32)
    for _ in range(args.warmup):
        lloyd_cpu(x, init, 1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        lloyd_cpu(x, init, 1)
    dt = time.perf_counter() - t0
    scale = (w["B"] * w["N"]) / n_s
    ms = 1e3 * dt / args.steps * scale
    cores = torch.get_num_threads()
    del x, init
    ref_gpu = None
    if torch.cuda.is_available() and not args.no_ref_gpu:
        try:
            dev = torch.device("cuda", 0)
            torch.cuda.set_device(dev)
            long = w["N"] * w["B"] * w["K"] > (1 << 33)  # c5: about a second per iteration
            ref_gpu = time_reference_gpu(w, 2 if long else 5, 1, dev)
        except Exception as e:  # the CPU line stands on its own
            ref_gpu = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    line = {
        "metric": "K-Means ms/iter", "value": ms, "unit": "ms/iter", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "B": w["B"], "N": w["N"], "K": w["K"],
                   "D": w["D"], "parallelism": "cpu"},
        "cpu_baseline": {"value": ms, "unit": "ms/iter", "cores": cores, "kind": "port",
                         "sample": (f"each step: 1 iteration on {n_s} of {w['B'] * w['N']} "
                                    f"points drawn from the {args.workload} distribution "
                                    f"({w['data']}" + (f", Zipf({w['zipf']})" if w["zipf"] else "")
                                    + f"; full K, D), fp32 CPU PyTorch Lloyd loop "
                                    f"(oracle/cpu_lloyd.py; the reference has no CPU path), "
                                    f"scaled by {scale:.1f}x")},
        "cpu_baseline_c1": cpu_baseline_c1(),
        "e2e": {"value": ms, "unit": "ms/iter", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "reference_gpu": ref_gpu,
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- our arm
def run_ours(args, w: dict) -> None:
    import flash_kmeans_cuda as fkc
    from flash_kmeans_cuda import _lib
    from flash_kmeans_cuda.distributed import (MultimemLloyd, allreduce_sums_counts,
                                               batch_kmeans_Euclid_sharded, multimem_enabled,
                                               shard_bounds)
    from flash_kmeans_cuda.kmeans import LloydState
    from flash_kmeans_cuda.largen import batch_kmeans_Euclid_host

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from flash_kmeans_cuda.distributed import init_process_group_from_env

        init_process_group_from_env("nccl", timeout_s=300.0)

    B, N, K, D = w["B"], w["N"], w["K"], w["D"]
    x_full, init_full = make_data(w, dev, seed=0)
    if w["shard"] == "N":
        n0, n1 = shard_bounds(N, world, rank)
        x = x_full[:, n0:n1].contiguous()
        init = init_full
    else:
        b0, b1 = shard_bounds(B, world, rank)
        x = x_full[b0:b1].contiguous()
        init = init_full[b0:b1].contiguous()
    del x_full
    torch.cuda.empty_cache()
    Bl, Nl = x.shape[0], x.shape[1]

    mm = None
    if w["shard"] == "N" and world > 1 and multimem_enabled() and MultimemLloyd.available(x):
        # sums/counts all-reduce fused into the finalize over NVLink multicast
        n_max = max(b1 - b0 for b0, b1 in (shard_bounds(N, world, r) for r in range(world)))
        mm = MultimemLloyd(x, K, n_max)
        mm.set_centroids(init)
        st = mm.state
        bufs = [mm.centroids, mm.centroids]
    else:
        st = LloydState(x, K)
        cur = init.clone()
        nxt = torch.empty_like(cur)
        st.set_centroids(cur)
        bufs = [cur, nxt]

    def step(i):
        a, b = bufs[i % 2], bufs[(i + 1) % 2]
        if mm is not None:
            mm.step(i, False)
        elif w["shard"] == "N" and world > 1:
            st.local(a)
            allreduce_sums_counts(st.sums, st.counts)
            st.finalize(a, b, False)
        else:
            st.step(a, b, False)

    for i in range(args.warmup):
        step(i)
    barrier_sync(dev)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _lib.lib.fkc_kernel_launches()
    with ClockSampler(dev.index) as clk:
        barrier_sync(dev)
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record(stream)
        barrier_sync(dev)
    launches = int(_lib.lib.fkc_kernel_launches() - launches0)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, dev)
    parity = None
    if mm is None and not args.no_parity:
        # the labels and counts of the last timed step, made against its input centroids
        parity = sample_parity(x, bufs[(args.warmup + args.steps - 1) % 2], st.ids, st.counts)

    # Per-rank split of the multi-GPU step (5 reps after the timed loop): local assign +
    # update, the sums/counts reduction (+ finalize for the multicast path), barriers.
    per_rank = None
    if world > 1:
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        acc = torch.zeros(4, dtype=torch.float64)
        for r in range(6):
            barrier_sync(dev)
            i = args.warmup + args.steps + r
            a, b = bufs[i % 2], bufs[(i + 1) % 2]
            if mm is not None:
                # the timed step: wait for the previous step's finalize everywhere, local
                # step, finalize with the arrival barrier folded in
                evs[0].record(stream)
                mm.wait_previous()
                evs[2].record(stream)
                st.local(a)
                evs[1].record(stream)
                mm.reduce_finalize_synced(i, False)
                evs[3].record(stream)
                evs[4].record(stream)
                torch.cuda.synchronize(dev)
                if r == 0:
                    continue
                acc += torch.tensor([evs[2].elapsed_time(evs[1]), evs[0].elapsed_time(evs[2]),
                                     evs[1].elapsed_time(evs[3]), 0.0], dtype=torch.float64) / 5
                continue
            evs[0].record(stream)
            st.local(a)
            evs[1].record(stream)
            if w["shard"] == "N":
                evs[2].record(stream)
                allreduce_sums_counts(st.sums, st.counts)
                evs[3].record(stream)
                st.finalize(a, b, False)
            else:
                evs[2].record(stream)
                evs[3].record(stream)
                st.finalize(a, b, False)
            evs[4].record(stream)
            torch.cuda.synchronize(dev)
            if r == 0:
                continue
            acc += torch.tensor([evs[0].elapsed_time(evs[1]), evs[1].elapsed_time(evs[2]),
                                 evs[2].elapsed_time(evs[3]), evs[3].elapsed_time(evs[4])],
                                dtype=torch.float64) / 5
        mine = acc.to(dev)
        alls = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(alls, mine)
        rows = [t.tolist() for t in alls]
        if mm is not None:
            per_rank = {"local_ms": [r_[0] for r_ in rows],
                        "step_wait_ms": [r_[1] for r_ in rows],
                        "reduce_finalize_ms": [r_[2] for r_ in rows],
                        "path": "multicast finalize with the arrival barrier in the kernel "
                                "(fkc_lloyd_finalize_multimem_synced) + the completion wait "
                                "before the next local step (fkc_multimem_step_wait); "
                                "reduce_finalize_ms includes waiting for the slowest rank"}
        else:
            per_rank = {"local_ms": [r_[0] for r_ in rows],
                        "allreduce_ms": [r_[2] for r_ in rows],
                        "finalize_ms": [r_[3] for r_ in rows],
                        "path": "NCCL all-reduce of sums and counts + replicated finalize"
                                if w["shard"] == "N" else "B-sharded, no collective"}
    if mm is not None:
        mm.release()  # every rank past the last multicast kernel before phase timings

    # Per-phase timings on the resident data (assign / update / finalize).
    cur_c = bufs[(args.warmup + args.steps) % 2]   # centroids produced by the last step
    other = bufs[(args.warmup + args.steps + 1) % 2]
    reps = 5
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    t_assign = t_update = t_fin = t_iter = 0.0
    dims = (Bl, Nl, K, D, st.code, st.ws.data_ptr(), st.ws_bytes)
    ev.append(torch.cuda.Event(enable_timing=True))
    for _ in range(reps + 1):
        barrier_sync(dev)
        sp = stream.cuda_stream
        ev[0].record(stream)
        _lib.check(_lib.lib.fkc_lloyd_assign(x.data_ptr(), cur_c.data_ptr(), st.ids.data_ptr(),
                                             st.counts.data_ptr(), *dims, sp), "assign")
        ev[1].record(stream)
        _lib.check(_lib.lib.fkc_lloyd_update(x.data_ptr(), st.ids.data_ptr(),
                                             st.counts.data_ptr(), st.sums.data_ptr(), *dims,
                                             sp), "update")
        ev[2].record(stream)
        _lib.check(_lib.lib.fkc_lloyd_finalize(st.sums.data_ptr(), st.counts.data_ptr(),
                                               cur_c.data_ptr(), other.data_ptr(), None, *dims,
                                               sp), "finalize")
        ev[3].record(stream)
        if world == 1:
            # the whole step as timed above (fkc_lloyd_iter; its update + finalize is one
            # fused pass when clusters are small)
            _lib.check(_lib.lib.fkc_lloyd_iter(x.data_ptr(), cur_c.data_ptr(), other.data_ptr(),
                                               st.ids.data_ptr(), st.sums.data_ptr(),
                                               st.counts.data_ptr(), None, *dims, sp), "iter")
        ev[4].record(stream)
        torch.cuda.synchronize(dev)
        if _ == 0:
            continue  # warm-up rep
        t_assign += ev[0].elapsed_time(ev[1]) / reps
        t_update += ev[1].elapsed_time(ev[2]) / reps
        t_fin += ev[2].elapsed_time(ev[3]) / reps
        t_iter += ev[3].elapsed_time(ev[4]) / reps
    if mm is not None and not args.no_parity:
        # the phase reps updated the multicast centroids in place: label them once more
        _lib.check(_lib.lib.fkc_lloyd_assign(x.data_ptr(), cur_c.data_ptr(), st.ids.data_ptr(),
                                             st.counts.data_ptr(), *dims, stream.cuda_stream),
                   "assign")
        torch.cuda.synchronize(dev)
        parity = sample_parity(x, cur_c, st.ids, st.counts)
    if parity is not None:
        parity = reduce_parity(parity, dev)
    t_assign = max_over_ranks(t_assign, dev)
    t_update = max_over_ranks(t_update, dev)
    t_fin = max_over_ranks(t_fin, dev)
    esz = 2
    assign_flops = 2.0 * Bl * Nl * K * D
    update_bytes = Bl * Nl * D * esz + 4 * Bl * Nl + Bl * K * (4 * D + 4)
    peaks = measured_peaks()
    tflops = assign_flops / (t_assign * 1e-3) / 1e12
    peak, peak_src = tensor_peak(peaks, t_assign)
    traffic = profiled_traffic(args.workload)

    # End-to-end through the public API: host inputs in, host results out.
    e2e = None
    if not args.no_e2e:
        x_host = x.cpu().pin_memory()
        init_host = init.cpu().pin_memory()
        ids_out = torch.empty((Bl, Nl), dtype=torch.int32).pin_memory()
        cents_out = torch.empty(tuple(init.shape), dtype=init.dtype).pin_memory()
        iters = w["iters"]

        def copy_out(ids, cents):
            # results into pinned host buffers, on the stream the timing events use
            if tuple(ids.shape) == tuple(ids_out.shape):
                ids_out.copy_(ids, non_blocking=True)
            else:
                ids.to("cpu")
            if tuple(cents.shape) == tuple(cents_out.shape):
                cents_out.copy_(cents, non_blocking=True)
            else:
                cents.to("cpu")

        def copy_then_call():
            xd = x_host.to(dev, non_blocking=True)
            cd = init_host.to(dev, non_blocking=True)
            if world == 1:
                ids, cents, n = fkc.batch_kmeans_Euclid(xd, K, max_iters=iters, tol=0.0,
                                                        init_centroids=cd)
            else:
                ids, cents, n = batch_kmeans_Euclid_sharded(xd, K, max_iters=iters, tol=0.0,
                                                            init_centroids=cd, shard=w["shard"])
            copy_out(ids, cents)

        def host_call():
            # pinned host x in, the copy overlapped with the first iteration
            ids, cents, n = batch_kmeans_Euclid_host(x_host, K, max_iters=iters, tol=0.0,
                                                     init_centroids=init_host, device=dev)
            copy_out(ids, cents)

        def time_calls(call, reps=2):
            call()
            barrier_sync(dev)
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            for _ in range(reps):
                call()
            f1.record(stream)
            barrier_sync(dev)
            return max_over_ranks(f0.elapsed_time(f1) / (reps * iters), dev)

        copy_then_ms = time_calls(copy_then_call)
        e2e_ms = time_calls(host_call) if world == 1 else copy_then_ms
        h2d = (x_host.numel() * x_host.element_size() + init_host.numel() *
               init_host.element_size())
        d2h = Bl * Nl * 4 + init.numel() * init.element_size()
        e2e = {"value": e2e_ms, "unit": "ms/iter",
               "h2d_bytes_per_step": h2d / iters, "d2h_bytes_per_step": d2h / iters,
               "copy_then_call_ms": copy_then_ms,
               "note": (f"one call of {iters} iterations per {iters} steps with pinned-host x "
                        f"and init in, labels + centroids copied out, inside the timed region: "
                        + ("batch_kmeans_Euclid_host (copy of x overlapped with the first "
                           "iteration); copy_then_call_ms = x copied first, then "
                           "batch_kmeans_Euclid" if world == 1 else
                           "x copied, then the sharded batch_kmeans_Euclid"))}
        del x_host, init_host

    # The reference's own end-to-end definition (benchmarks/bench_vs_triton.py:52-67):
    # whole batch_kmeans_Euclid calls on device-resident x (set-up per call included),
    # total time / iterations.
    e2e_device = None
    if not args.no_e2e:
        iters = w["iters"]

        def dev_call():
            if world == 1:
                return fkc.batch_kmeans_Euclid(x, K, max_iters=iters, tol=0.0,
                                               init_centroids=init)
            return batch_kmeans_Euclid_sharded(x, K, max_iters=iters, tol=0.0,
                                               init_centroids=init, shard=w["shard"])

        dev_call()
        barrier_sync(dev)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps_dev = 3
        g0.record(stream)
        for _ in range(reps_dev):
            dev_call()
        g1.record(stream)
        barrier_sync(dev)
        e2e_device = {"value": max_over_ranks(g0.elapsed_time(g1) / (reps_dev * iters), dev),
                      "unit": "ms/iter", "calls": reps_dev, "iters_per_call": iters,
                      "note": "whole batch_kmeans_Euclid calls on device-resident x (workspace, "
                              "norm rows and graph launch per call), as the reference's "
                              "bench_vs_triton.py times them"}

    if rank == 0:
        cpu = cpu_c1 = None
        if world == 1 and not args.no_cpu_baseline:
            try:
                cpu = cpu_baseline(w, args.workload)
                cpu_c1 = cpu_baseline_c1()
            except Exception as e:  # pragma: no cover
                cpu = {"value": None, "error": str(e)}
        line = {
            "metric": "K-Means ms/iter", "value": ms, "unit": "ms/iter", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": DT_SHORT[w["dtype"]], "data": "synthetic",
            "config": {"workload": args.workload, "B": B, "N": N, "K": K, "D": D,
                       "parallelism": (f"dp{world}-shard{w['shard']}"
                                       + ("-multimem" if mm is not None else "")),
                       "l2": (f"x ({B * N * D * esz / 1e6:.0f} MB) > L2 (126 MB): no flush"
                              if B * N * D * esz > L2_BYTES else "x fits in L2")},
            "assign_tflops": tflops,
            "assign_ms": t_assign, "update_ms": t_update, "finalize_ms": t_fin,
            # one whole step (assign + update + finalize) timed alone, and what the step
            # spends after its assign (the fused pass when clusters are small)
            "step_ms": (t_iter if world == 1 else None),
            "step_after_assign_ms": (max(t_iter - t_assign, 0.0) if world == 1 else None),
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak,
                         "unit": "TFLOP/s", "frac": tflops / peak,
                         "traffic": traffic, "kernel": "assign_tc_kernel",
                         "peak_src": f"{peak_src} (fp16 dense is equal)"},
            "update": {"bound": "hbm", "achieved_gbs": update_bytes / (t_update * 1e-3) / 1e9,
                       "peak_gbs": peaks["hbm"],
                       "frac": update_bytes / (t_update * 1e-3) / 1e9 / peaks["hbm"],
                       "algorithmic_bytes": update_bytes,
                       "note": "phase times of the stepwise entry points (fkc_lloyd_update, "
                               "fkc_lloyd_finalize); "
                               + ("the timed step (fkc_lloyd_iter) fuses update and finalize "
                                  "into one pass over the clusters"
                                  if world == 1 and Nl <= 32 * K else
                                  "the timed step (fkc_lloyd_iter) runs the same update and "
                                  "finalize" if world == 1 else
                                  "the timed step runs this rank's update, then reduces sums and "
                                  "counts across ranks inside the finalize")},
            "e2e": e2e,
            "e2e_device": e2e_device,
            "parity": parity,
            "per_rank": per_rank,
            "cpu_baseline": cpu,
            "cpu_baseline_c1": cpu_c1,
            "clocks": clk.summary(),
            "gpu_launches": launches,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        MultimemLloyd.release_all()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="c3", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the float64 label check of the last timed step")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="reference arm: skip the reference_gpu timing of its CUDA kernels")
    ap.add_argument("--ref-device", default="cpu", choices=["cpu", "cuda"],
                    help="reference arm: the CPU port of its loop (default) or its own CUDA "
                         "kernels built from source under oracle/_ref")
    args = ap.parse_args()
    if args.warmup < 3:
        log("warmup raised to 3 (minimum)")
        args.warmup = 3
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference_arm(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
