"""Training-step benchmark (bench.py --workload train).

Config ("C5"): 6,000,000 Gaussians, SH degree 3, 64-cluster
distributions of gsplat_tt_b200.scenes; 32 views of 1920x1080 (f = 1500) on a sphere of
radius 5 looking at the origin; loss 0.8 L1 + 0.2 (1 - SSIM); sparse Adam with betas
(0.9, 0.999), eps 1e-15 and the per-group learning rates of configs[3]. The views are split
evenly over the ranks (strong scaling: the step's total work is fixed); gradients are
reduce-scattered to the rows' owners, each rank runs sparse Adam on its own rows and the
parameters are all-gathered (``GS_BENCH_SHARDED=0``: one allreduce and replicated Adam
instead). ``GS_BENCH_CONFIG=c4`` selects configs[3] (3M Gaussians, 8 views of
1600x1056, f = 1300, radius 4) instead; ``GS_BENCH_VIEWS=k`` keeps only the first k views (for
small ncu captures; the benchmark line then names the reduced workload).
"""
from __future__ import annotations

import os
import time

import numpy as np
import torch

from . import scenes
from ._lib import check, lib, timing_report
from .dist import view_slice
from .train import TrainConfig, Trainer

LR_BASELINE = {"means": 1.6e-4, "log_scales": 5e-3, "quats": 1e-3, "opacity_logits": 5e-2,
               "sh_dc": 2.5e-3, "sh_rest": 2.5e-3 / 20.0}


def config_name() -> str:
    return os.environ.get("GS_BENCH_CONFIG", "c5")


def view_targets(cams, first_index: int) -> list[np.ndarray]:
    out = []
    for i, c in enumerate(cams):
        rng = np.random.default_rng(1000 + first_index + i)
        out.append(rng.uniform(0.0, 1.0, (c.height, c.width, 3)).astype(np.float32))
    return out


def train_cfg() -> TrainConfig:
    return TrainConfig(sh_degree=3, tile_size=16, use_ssim=True, lambda_dssim=0.2,
                       lr=dict(LR_BASELINE), betas=(0.9, 0.999), eps=1e-15)


def _kernel_bytes(name: str, n: int, views: int, pairs: float, px: int) -> float | None:
    """Algorithmic DRAM bytes of one timed launch of the HBM-bound kernels (the minimum the
    algorithm moves, not what the implementation happens to move):

    * train_project (one launch for all of the rank's views): the SH3 parameters once
      (236 B per Gaussian) and per view the 52 B record (mean 8, conic 12, colour 12,
      opacity 4, depth key 4, rectangle 8, pair count 4);
    * radix_pass32 (one pass of the depth sort over N): 4 B key + 4 B value read and written;
    * tile_sort_emit (pair emission fused into the first tile-sort pass): 16 B per Gaussian
      read (depth order, first-pair offset, rectangle), 8 B per pair written;
    * tile_sort_pass (the second tile-sort pass): 8 B per pair read, 4 B per pair written;
    * sparse_adam (the five group launches under one timer): 28 B per parameter value
      (p, m, v, g read; p, m, v written) for the 59 values of each row;
    * param_bwd: the parameters read and their gradients written (236 B each per Gaussian)
      and the 2D-gradient rows (36 B) of every view.
    The rasterisers and the loss filters are SM-issue bound and have no entry."""
    if name == "train_project":
        return n * 236.0 + views * n * 52.0
    if name == "radix_pass32":
        return n * 16.0
    if name == "tile_sort_emit":
        return pairs * 8.0 + n * 16.0
    if name == "tile_sort_pass":
        return pairs * 12.0
    if name == "sparse_adam":
        return n * 59 * 28.0
    if name == "param_bwd":
        return n * 472.0 + views * n * 36.0
    return None


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch measured by ncu on
# the C4 scene with one view (3M Gaussians, 21,898,068 pairs), and the unit the traffic
# scales with when the bench's workload is larger (profiles/train_kernels_c4_1view.md).
NCU_TRAFFIC_C4_1VIEW = {
    "tile_sort_emit": (172.1e6, "pairs"),
    "tile_sort_pass": (247.2e6, "pairs"),
}
C4_1VIEW_PAIRS = 21898068.0


def _traffic(name: str, pairs: float) -> float | None:
    t = NCU_TRAFFIC_C4_1VIEW.get(name)
    if t is None:
        return None
    return t[0] * pairs / C4_1VIEW_PAIRS


def summarize_kernels(rep: dict, ksteps: int, n: int, views: int, pairs: float, px: int,
                      peaks: dict):
    """Per-kernel figures from the library's timer report ({name: (total ms, launches)} over
    ksteps steps), the roofline object for the largest kernel with an HBM byte model, and
    the sort's share of the step."""
    per_kernel = {}
    for k, (tot, cnt) in rep.items():
        avg = tot / cnt
        entry = {"ms_per_launch": avg, "launches_per_step": cnt / ksteps,
                 "ms_per_step": tot / ksteps}
        b = _kernel_bytes(k, n, views, pairs, px)
        if b is not None:
            gbs = b / (avg / 1e3) / 1e9
            entry.update({"algorithmic_bytes": b, "achieved_gbs": gbs,
                          "frac_hbm": gbs / peaks["hbm_gbs"]})
        per_kernel[k] = entry
    # the largest kernel with an HBM byte model (the rasterisers, which take more time, are
    # SM-issue bound: about 72 % issue-active at 1-2 % of DRAM bandwidth per ncu)
    hbm = {k: v for k, v in per_kernel.items() if "achieved_gbs" in v}
    dom_name, d = max(hbm.items(), key=lambda kv: kv[1]["ms_per_step"])
    raster = {k: per_kernel[k]["ms_per_step"] for k in ("raster_fwd", "raster_bwd") if k in per_kernel}
    roofline = {"bound": "hbm", "kernel": dom_name, "achieved": d["achieved_gbs"],
                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": d["frac_hbm"],
                "traffic": _traffic(dom_name, pairs),
                "traffic_source": "ncu dram bytes of one launch at C4 / 1 view, scaled by pairs",
                "peak_source": peaks["source"],
                "note": "largest HBM-bound kernel of the step; the rasterisers "
                        f"({', '.join(f'{k} {v:.1f} ms' for k, v in raster.items())} per step) "
                        "are SM-issue bound and have no HBM roofline"}
    sort_parts = {k: per_kernel[k] for k in ("radix_hist", "radix_pass32", "pair_offsets",
                                             "tile_counts", "tile_sort_emit", "tile_sort_pass")
                  if k in per_kernel}
    sort_in_step = None
    if sort_parts:
        sort_in_step = {"ms_per_step": sum(v["ms_per_step"] for v in sort_parts.values()),
                        "parts": sorted(sort_parts)}
    return per_kernel, roofline, sort_in_step


def run(args, rank: int, world: int, local: int) -> dict:
    from bench import ClockSampler, barrier, max_over_ranks, measured_peaks  # noqa: E402
    name = config_name()
    c = scenes.CONFIGS[name]
    dev = torch.device("cuda", local)
    V = int(os.environ.get("GS_BENCH_VIEWS", c["views"]))  # fewer views: profiling runs only
    lo, hi = view_slice(V, world, rank)
    per = hi - lo
    cams_all = scenes.training_cameras(name)
    mine = cams_all[lo:hi]
    H, W = c["height"], c["width"]
    params = scenes.cluster_scene(c["n"], sh_degree=3, seed=0)
    targets_host = view_targets(mine, rank * per)
    cfg = train_cfg()
    # GS_BENCH_SHARDED=0: allreduce + replicated Adam instead of the owner-sharded optimizer
    sharded = os.environ.get("GS_BENCH_SHARDED", "1") != "0"
    # GS_BENCH_MULTICAST=0: the sharded update through NCCL instead of NVLink multicast
    multicast = os.environ.get("GS_BENCH_MULTICAST", "1") != "0"
    tr = Trainer(params, cfg, per, H, W, device=dev, sharded_optimizer=sharded, multicast=multicast)
    del params
    cams = [(cm.w2c, cm.K, H, W) for cm in mine]
    pairs0 = tr.count_pairs(cams)
    tr._alloc(int(max(pairs0) * 1.3) + 4096)
    targets = [torch.from_numpy(t).to(dev) for t in targets_host]
    st = torch.cuda.current_stream()

    for i in range(args.warmup):
        tr.step(cams, targets, check_errors=(i == 0))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(world)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            tr.step(cams, targets)
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
    if lib.gs_workspace_error(tr.ws.data_ptr(), st.cuda_stream) != 0:
        raise RuntimeError("a timed step overflowed its pair buffers or timed out")
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    total_px = V * H * W
    value = total_px / (ms / 1e3) / 1e6
    loss_now = float(tr.losses.sum().item())

    # e2e: the public API given the step's inputs (target images) in pinned host memory --
    # the library copies every view's target host -> device each step, on its own stream
    # overlapped with the other views' work -- and the loss read back to the host.
    pinned = [torch.from_numpy(t).pin_memory() for t in targets_host]
    for _ in range(2):
        tr.step(cams, pinned)
        loss_host = tr.losses.sum().item()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e0.record()
    for _ in range(args.steps):
        tr.step(cams, pinned)
        loss_host = tr.losses.sum().item()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    del loss_host, t0

    # per-kernel device times (CUDA events on the launching stream), one more short loop;
    # with the timer on the library runs the views on one stream, so launches do not overlap
    # and their sum is the serial step time (the timed step above overlaps two views)
    lib.gs_timing_reset()
    lib.gs_timing_enable(1)
    ksteps = max(2, min(args.steps, 5))
    for _ in range(ksteps):
        tr.step(cams, targets)
    torch.cuda.synchronize()
    lib.gs_timing_enable(0)
    rep = timing_report()
    lib.gs_timing_reset()
    pairs = tr.pairs.float().mean().item()
    peaks = measured_peaks()
    per_kernel, roofline, sort_in_step = summarize_kernels(rep, ksteps, tr.n, per, pairs, H * W, peaks)
    out = {
        "metric": "train-step Mpix/s (fwd+bwd+Adam)",
        "value": value, "unit": "Mpix/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{name.upper()} train step: {c['n']} Gaussians SH3, {V} views "
                               f"{W}x{H} ({per} per GPU), L1+SSIM, sparse Adam",
                   "gaussians": c["n"], "views": V, "width": W, "height": H, "tile": 16,
                   "parallelism": f"dp{world} over views" + (
                       "" if world == 1 else
                       " + owner-sharded Adam with NVLink-multicast gradient sum and parameter "
                       f"broadcast (gs_sparse_adam_multicast), pipelined over {tr.chunks} row chunks "
                       "with the projection backward" if tr.multicast else
                       " + NCCL reduce-scatter / all-gather, owner-sharded Adam" if tr.sharded
                       else " + NCCL allreduce, replicated Adam"),
                   "l2": "inputs larger than L2 (params 1.4 GB, pairs per view > 100 MB)"},
        "e2e": {"value": total_px / (e2e_ms / 1e3) / 1e6, "unit": "Mpix/s",
                "h2d_bytes_per_step": int(sum(t.size * 4 for t in targets_host)),
                "d2h_bytes_per_step": 4},
        "gpu_launches": int(sum(v["launches_per_step"] for v in per_kernel.values())),
        "pairs_per_view": pairs, "loss": loss_now,
        "kernels": per_kernel,
        "clocks": clk.summary(),
    }
    out["roofline"] = roofline
    if sort_in_step is not None:
        out["sort_in_step"] = sort_in_step
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(name)
    return out


def _oracle_sample(name: str, scale: int, views: int = 1):
    """The config at 1/scale^2 of the pixels and Gaussians (same density), `views` views."""
    c = scenes.CONFIGS[name]
    n = c["n"] // (scale * scale)
    H, W = c["height"] // scale, c["width"] // scale
    f = c["f"] / scale
    cams = scenes.sphere_cameras(views, c["radius"], f, W, H)
    params = scenes.cluster_scene(n, sh_degree=3, seed=0)
    tgts = [np.random.default_rng(1000 + i).uniform(0, 1, (H, W, 3)).astype(np.float32)
            for i in range(views)]
    return params, cams, tgts, n, H, W


def cpu_baseline(name: str, budget_s: float = 20.0, workers: int | None = None) -> dict:
    """The oracle port of the reference's numpy training models (the reference's CPU
    implementation of this path is numpy) on this host's cores: a multi-view step at
    reduced size with one view per worker process (oracle.train_pool), gradients summed
    and sparse Adam applied once per step, as the reference's per-view loop does."""
    from oracle import train as ot
    from oracle.train_pool import ViewPool
    scale = 8
    c = scenes.CONFIGS[name]
    if workers is None:  # the cores this process may run on, up to one per view of the step
        avail = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
        workers = max(1, min(avail or 1, c["views"]))
    params, cams, tgts, n, H, W = _oracle_sample(name, scale, views=workers)
    cfg = ot.Cfg(sh_degree=3, tile=16)
    zeros = {k: np.zeros_like(v) for k, v in params.items()}
    vcams = [(cm.w2c, cm.K, H, W) for cm in cams]
    with ViewPool(params, cfg, workers) as pool:
        pool.step(zeros, zeros, 0, vcams[:workers], tgts[:workers], lr=LR_BASELINE)  # warm-up
        t0 = time.perf_counter()
        iters = 0
        while True:
            pool.step(zeros, zeros, 0, vcams, tgts, lr=LR_BASELINE)
            iters += 1
            el = time.perf_counter() - t0
            if el > budget_s or iters >= 3:
                break
    return {"value": workers * H * W * iters / el / 1e6, "unit": "Mpix/s", "cores": workers,
            "kind": "port",
            "sample": f"{iters} oracle steps of {workers} views {W}x{H} (one per worker process) "
                      f"with {n} Gaussians ({name.upper()} at 1/{scale * scale} pixels and "
                      "Gaussians)"}


def run_reference(args) -> dict:
    name = config_name()
    b = cpu_baseline(name, budget_s=max(10.0, 3.0 * args.steps))
    return {"impl": "reference", "metric": "train-step Mpix/s (fwd+bwd+Adam)", "value": b["value"],
            "unit": "Mpix/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{name.upper()} train step (oracle port, reduced sample)"},
            "cpu_baseline": b,
            "e2e": {"value": b["value"], "unit": "Mpix/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
