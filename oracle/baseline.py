"""CPU baselines and the reference arm of bench.py (TEST INFRASTRUCTURE ONLY: bench.py's
cpu_baseline leg and its --impl reference arm call this module; the product never does).

Neither function loads libgs200.so: the reference arm must time the reference's own CPU
implementation only.

* sort  -- the reference's compiled sort_and_bin (src/gsplat_cpu/sort.cpp:89-263, built
  into oracle/_ref by oracle/Makefile) on the host's cores, else the C port's stable LSD
  sort (oracle/gs_oracle.c).
* train -- the oracle port of the reference's numpy training models (the reference's CPU
  implementation of this path is numpy: gsplat/blend_backward_dev.py forward_fast /
  ref_slots_fast, gsplat/train_loss.py, gsplat/t2_param_backward.py), one view per
  spawned worker process (oracle.train_pool), on a reduced sample of the config: 1/8 of
  the width and height and 1/64 of the Gaussians (the same Gaussian density per pixel).
"""
from __future__ import annotations

import os
import platform
import time

import numpy as np

# Worker processes of the training baseline: one view each, pinned so that the figure does
# not move with the host's core count (fewer when the process may use fewer cores).
TRAIN_WORKERS = 16
SAMPLE_SCALE = 8


def cpu_info() -> dict:
    """nproc (cores this process may use) and the CPU model of this host."""
    avail = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    model = platform.processor() or ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"nproc": int(avail or 1), "cpu_model": model}


def cpu_sort_baseline(keys, vals, budget_s: float = 15.0) -> dict:
    """The reference's sort_and_bin (oracle/_ref) on this host's cores, else the C port."""
    from . import display as od
    info = cpu_info()
    os.environ.setdefault("GSPLAT_TT_NUM_THREADS", str(info["nproc"]))
    ref = od.reference_module()
    n = keys.size
    if ref is not None:
        tiles = (keys >> np.uint64(32)).astype(np.int64)
        depth = (keys & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
        dv = np.empty(n, np.float32)
        dv[vals] = depth
        gids = vals.astype(np.int64)
        fn = lambda: ref.sort(gids, tiles, dv, 120, 68)  # noqa: E731
        kind, cores = "reference", int(os.environ["GSPLAT_TT_NUM_THREADS"])
    else:
        fn = lambda: od.sort_pairs(keys, vals)  # noqa: E731
        kind, cores = "port", 1
    fn()
    t0, iters = time.perf_counter(), 0
    while True:
        fn()
        iters += 1
        el = time.perf_counter() - t0
        if el > budget_s or iters >= 20:
            break
    v = n * iters / el
    # per core as well: the host's core count differs between boxes
    return {"value": v, "unit": "pairs/s", "cores": cores, "value_per_core": v / cores,
            "kind": kind, "sample": f"{iters} full C2 sorts of {n} pairs", **info}


def _train_sample(name: str, views: int):
    """The config at 1/SAMPLE_SCALE of the width and height and 1/SAMPLE_SCALE^2 of the
    Gaussians, `views` views (the same sphere of cameras)."""
    from gsplat_tt_b200 import scenes
    c = scenes.CONFIGS[name]
    s = SAMPLE_SCALE
    n = c["n"] // (s * s)
    H, W = c["height"] // s, c["width"] // s
    cams = scenes.sphere_cameras(views, c["radius"], c["f"] / s, W, H)
    params = scenes.cluster_scene(n, sh_degree=3, seed=0)
    tgts = [np.random.default_rng(1000 + i).uniform(0, 1, (H, W, 3)).astype(np.float32)
            for i in range(views)]
    return params, cams, tgts, n, H, W


def train_cpu_baseline(name: str, budget_s: float = 20.0, max_steps: int = 3) -> dict:
    """Multi-view oracle training steps on the sample (one view per worker process,
    gradients summed and sparse Adam applied once per step), timed end to end."""
    from gsplat_tt_b200 import scenes
    from . import train as ot
    from .train_pool import ViewPool
    info = cpu_info()
    c = scenes.CONFIGS[name]
    workers = max(1, min(info["nproc"], TRAIN_WORKERS, c["views"]))
    params, cams, tgts, n, H, W = _train_sample(name, workers)
    cfg = ot.Cfg(sh_degree=3, tile=16)
    zeros = {k: np.zeros_like(v) for k, v in params.items()}
    vcams = [(cm.w2c, cm.K, H, W) for cm in cams]
    lr = scenes.LR_BASELINE
    with ViewPool(params, cfg, workers, ssim=c["ssim"]) as pool:
        pool.step(zeros, zeros, 0, vcams, tgts, lr=lr)  # warm-up
        t0, iters = time.perf_counter(), 0
        while True:
            pool.step(zeros, zeros, 0, vcams, tgts, lr=lr)
            iters += 1
            el = time.perf_counter() - t0
            if el > budget_s or iters >= max_steps:
                break
    s = SAMPLE_SCALE
    v = workers * H * W * iters / el / 1e6
    return {"value": v, "unit": "Mpix/s", "cores": workers, "value_per_core": v / workers,
            "kind": "port",
            "sample": f"{iters} oracle steps of {workers} views {W}x{H} (one per worker process) "
                      f"with {n} Gaussians ({name.upper()} at 1/{s * s} of the pixels and "
                      "Gaussians, the same density)", **info}
