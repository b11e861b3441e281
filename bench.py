"""Benchmark of the B200 render + train hot path (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload train|sort]

Workloads (BASELINE.json metric "train-step Mpix/s (fwd+bwd+Adam) and sort keys/s"):
  train -- config C5 (6M Gaussians, SH3, 32 views of 1920x1080 split over the ranks,
           owner-sharded sparse Adam with the gradient sum and parameter broadcast over
           NVLink); a step is one full training step. Metric: Mpix/s = 32 * 1920 * 1080 /
           step time. The line also carries `sort_c2`: the sort workload below measured
           in the same process at the same N (--no-sort skips it).
  sort  -- config C2 (2^24 Zipf (uint64 key, uint32 value) pairs, 45 key bits); a step is
           one stable sort per rank (independent per-GPU sorts, weak scaling).
           Metric: sorted pairs/s over all ranks.

The reference arm (--impl reference) runs the reference's CPU implementation of the same
workload (oracle/baseline.py) on rank 0 and loads nothing of this repository's library.

Timing: W untimed steps, then K steps between barrier + synchronize, CUDA events on the
launching stream, max over ranks. `value` has inputs resident in HBM; `e2e` goes through
the public API with pinned host buffers and the host<->device copies inside the timed
region. `roofline` is computed from the dominant kernel's average launch time, measured
with the library's CUDA-event kernel timer (gs_timing_*) in a separate loop after the
timed one. `cpu_baseline` times the reference's CPU implementation on this host.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "200"], stdout=open(self.path, "w"),
                stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------- distributed

def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "b200":
        torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        if args.impl == "b200":  # bound to this rank's GPU (no device guessing in barriers)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t)
    return float(t.item())


# ---------------------------------------------------------------- sort workload

SORT_N = 1 << 24
SORT_KEY_BITS = 45


def sort_pass_bytes(key_bits: int) -> list[int]:
    """Bytes per pair that each onesweep pass of this implementation's values-only sort of
    64-bit keys moves: a pass on 64-bit keys reads 12 B (key + value) and writes 12 B;
    above 32 key bits the last 64-bit pass writes its keys narrowed to 32 bits (8 B), the
    later passes read and write 8 B; the last pass writes the values only (4 B)."""
    npass = (key_bits + 7) // 8
    wide = (key_bits - 32 + 7) // 8 if key_bits > 32 else npass
    out = []
    for p in range(npass):
        rd = 12 if p < wide else 8
        wr = 4 if p == npass - 1 else 12 if p < wide - 1 or (p == wide - 1 and wide == npass) else 8
        out.append(rd + wr)
    return out


def sort_algorithmic_bytes(n: int, key_bits: int) -> tuple[float, float]:
    """(mean bytes per onesweep pass launch, bytes per sort with the histogram's 8 B/pair
    read) of this implementation's passes."""
    pb = sort_pass_bytes(key_bits)
    return n * sum(pb) / len(pb), n * sum(pb) + 8.0 * n


SORT_PASS_BYTES_PER_PAIR = 24  # scope table (d): 12 B read + 12 B written per LSD pass
SORT_METRIC = "sort keys/s (C2: 2^24 Zipf uint64/uint32 pairs, 45 key bits)"


def sort_config(world: int) -> dict:
    return {"workload": "C2 radix sort, one 2^24-pair instance per GPU",
            "pairs_per_gpu": SORT_N, "key_bits": SORT_KEY_BITS, "tiles": 8160,
            "l2": "inputs larger than L2 (201 MB keys+values per GPU)",
            "parallelism": f"independent sorts x{world}"}


def run_sort(args, rank, world, local) -> dict:
    import torch
    from gsplat_tt_b200 import scenes
    from gsplat_tt_b200._lib import lib, check, timing_report
    dev = torch.device("cuda", local)
    keys, vals = scenes.c2_pairs(seed=rank)  # one independent C2 instance per rank
    n = keys.size
    kd = torch.from_numpy(keys.view(np.int64)).to(dev)
    vd = torch.from_numpy(vals.view(np.int32)).to(dev)
    vo = torch.empty_like(vd)
    ws = torch.empty(lib.gs_sort_pairs_workspace_size(n, SORT_KEY_BITS), dtype=torch.uint8,
                     device=dev)
    st = torch.cuda.current_stream()

    def step():
        check(lib.gs_sort_pairs(kd.data_ptr(), vd.data_ptr(), n, SORT_KEY_BITS, None,
                                vo.data_ptr(), ws.data_ptr(), ws.numel(), st.cuda_stream))

    for _ in range(args.warmup):
        step()
    check(lib.gs_workspace_error(ws.data_ptr(), st.cuda_stream))
    torch.cuda.synchronize()
    # correctness guard on the benchmarked data: values are a permutation of 0..n-1, so
    # key_by_value[sorted values] must be non-decreasing.
    key_by_value = torch.empty_like(kd)
    key_by_value[vd.long()] = kd
    ks = key_by_value[vo.long()]
    if not bool((ks[1:] >= ks[:-1]).all()):
        raise RuntimeError("sort output is not sorted")
    del key_by_value, ks
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(world)
        torch.cuda.synchronize()
        l0 = lib.gs_launch_count()
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        launches = lib.gs_launch_count() - l0
        torch.cuda.synchronize()
        barrier(world)
    check(lib.gs_workspace_error(ws.data_ptr(), st.cuda_stream))
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    total_pairs = sum_over_ranks(float(n), world)
    value = total_pairs / (ms / 1e3)

    # e2e through the public API: pinned host in, sorted values back to the host.
    kh = torch.from_numpy(keys.view(np.int64)).pin_memory()
    vh = torch.from_numpy(vals.view(np.int32)).pin_memory()
    oh = torch.empty(n, dtype=torch.int32).pin_memory()
    for _ in range(2):
        kd.copy_(kh, non_blocking=True); vd.copy_(vh, non_blocking=True); step()
        oh.copy_(vo, non_blocking=True)
    barrier(world)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps):
        kd.copy_(kh, non_blocking=True)
        vd.copy_(vh, non_blocking=True)
        step()
        oh.copy_(vo, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)

    # dominant kernel (onesweep pass) launch times, live, with CUDA events
    lib.gs_timing_reset()
    lib.gs_timing_enable(1)
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    lib.gs_timing_enable(0)
    rep = timing_report()
    lib.gs_timing_reset()
    # every onesweep pass: those on 64-bit keys, then those on the narrowed 32-bit keys
    pass_ms = sum(rep.get(k, (0.0, 0))[0] for k in ("radix_pass", "radix_pass_n32"))
    pass_launches = sum(rep.get(k, (0.0, 0))[1] for k in ("radix_pass", "radix_pass_n32"))
    own_bytes, _ = sort_algorithmic_bytes(n, SORT_KEY_BITS)
    avg_ms = pass_ms / pass_launches if pass_launches else float("nan")
    peaks = measured_peaks()
    # the scope table's per-unit figure: an LSD pass over (64-bit key, 32-bit value) pairs
    # reads and writes 12 B per pair (24 B; 152 B per pair over six passes and the
    # histogram read). Narrowed keys make a pass move fewer; the own-bytes figure counts those
    per_launch_bytes = SORT_PASS_BYTES_PER_PAIR * n
    achieved = per_launch_bytes / (avg_ms / 1e3) / 1e9
    achieved_own = own_bytes / (avg_ms / 1e3) / 1e9
    out = {
        "metric": SORT_METRIC,
        "value": value, "unit": "pairs/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
        "config": sort_config(world),
        "e2e": {"value": sum_over_ranks(float(n), world) / (e2e_ms / 1e3), "unit": "pairs/s",
                "h2d_bytes_per_step": 12 * n, "d2h_bytes_per_step": 4 * n},
        # the library's kernels launched in the timed region, summed over the ranks
        "gpu_launches": int(sum_over_ranks(float(launches), world)),
        "roofline": {"bound": "hbm",
                     "kernel": "k_onesweep_pass (64-bit keys, then keys narrowed to 32 bits)",
                     "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"],
                     "traffic": None,
                     "traffic_source": "null: no ncu capture of the passes since the keys "
                                       "are narrowed (the last one measured a 64-bit pass)",
                     "peak_source": peaks["source"], "avg_launch_ms": avg_ms,
                     "pass_launches_per_sort": pass_launches / args.steps,
                     "algorithmic_bytes_per_launch": per_launch_bytes,
                     "bytes_per_pair_per_pass": SORT_PASS_BYTES_PER_PAIR,
                     "own_bytes_per_pair_by_pass": sort_pass_bytes(SORT_KEY_BITS),
                     "achieved_own_bytes": achieved_own,
                     "frac_own_bytes": achieved_own / peaks["hbm_gbs"]},
        "kernel_ms": {k: v[0] / v[1] for k, v in rep.items()},
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.baseline import cpu_sort_baseline
        out["cpu_baseline"] = cpu_sort_baseline(keys, vals)
    return out


def run_sort_reference(args) -> dict:
    from gsplat_tt_b200 import scenes
    from oracle.baseline import cpu_sort_baseline
    keys, vals = scenes.c2_pairs()
    b = cpu_sort_baseline(keys, vals, budget_s=max(5.0, 2.0 * args.steps))
    return {"impl": "reference", "metric": SORT_METRIC,
            "value": b["value"], "unit": "pairs/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": keys.size / b["value"] * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u64",
            "data": "synthetic", "config": sort_config(1), "cpu_baseline": b,
            "e2e": {"value": b["value"], "unit": "pairs/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------- train workload

TRAIN_METRIC = "train-step Mpix/s (fwd+bwd+Adam)"


def train_config(name: str, views: int | None = None) -> dict:
    """The training workload's config keys, shared by both arms."""
    from gsplat_tt_b200 import scenes
    c = scenes.CONFIGS[name]
    V = c["views"] if views is None else views
    return {"workload": f"{name.upper()} train step: {c['n']} Gaussians SH3, {V} views "
                        f"{c['width']}x{c['height']}, "
                        f"{'L1+SSIM' if c['ssim'] else 'L1'}, sparse Adam",
            "gaussians": c["n"], "views": V, "width": c["width"], "height": c["height"],
            "tile": 16, "l2": "inputs larger than L2 (params 1.4 GB, pairs per view > 100 MB)"}


def run_train_reference(args) -> dict:
    """The reference arm of the training workload: the oracle port of the reference's numpy
    training models on the host's cores, on a bounded sample of the same workload."""
    from oracle.baseline import train_cpu_baseline
    name = os.environ.get("GS_BENCH_CONFIG", "c5")
    b = train_cpu_baseline(name, budget_s=max(10.0, 3.0 * args.steps))
    cfg = train_config(name)
    cfg["parallelism"] = f"CPU: {b['cores']} worker processes, one view each"
    return {"impl": "reference", "metric": TRAIN_METRIC, "value": b["value"],
            "unit": "Mpix/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "cpu_baseline": b,
            "e2e": {"value": b["value"], "unit": "Mpix/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def sort_summary(s: dict) -> dict:
    """The C2 sort measurement carried inside the training line (every N, every rank)."""
    keys = ("metric", "value", "unit", "ms_per_step", "scaling", "config", "e2e", "roofline",
            "gpu_launches", "clocks", "cpu_baseline")
    return {k: s[k] for k in keys if k in s}


# ---------------------------------------------------------------- main

def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["train", "sort"], default="train")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sort", action="store_true",
                    help="train workload: skip the C2 sort measurement carried in the line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world, local = dist_setup(args)
    if args.impl == "reference":
        # the reference's CPU implementation only: nothing here loads libgs200.so
        if rank == 0:
            out = run_sort_reference(args) if args.workload == "sort" else run_train_reference(args)
            if args.workload == "train" and not args.no_sort:
                out["sort_c2"] = sort_summary(run_sort_reference(args))
            print(json.dumps(out), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    if args.workload == "sort":
        out = run_sort(args, rank, world, local)
    else:
        from gsplat_tt_b200 import train_bench
        out = train_bench.run(args, rank, world, local)
        if not args.no_sort:
            import torch
            torch.cuda.empty_cache()
            out["sort_c2"] = sort_summary(run_sort(args, rank, world, local))
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
