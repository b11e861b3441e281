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

import numpy as np
import torch

from . import scenes
from ._lib import check, lib, timing_report
from .dist import view_slice
from .train import TrainConfig, Trainer

LR_BASELINE = scenes.LR_BASELINE


def config_name() -> str:
    return os.environ.get("GS_BENCH_CONFIG", "c5")


def view_targets(cams, first_index: int) -> list[np.ndarray]:
    out = []
    for i, c in enumerate(cams):
        rng = np.random.default_rng(1000 + first_index + i)
        out.append(rng.uniform(0.0, 1.0, (c.height, c.width, 3)).astype(np.float32))
    return out


def train_cfg() -> TrainConfig:
    # GS_BENCH_DETERMINISTIC=1 times the fixed-order (slot) gradient sums instead of the
    # atomics; the bench line then says so in its config
    det = os.environ.get("GS_BENCH_DETERMINISTIC", "0") == "1"
    return TrainConfig(sh_degree=3, tile_size=16, use_ssim=True, lambda_dssim=0.2,
                       lr=dict(LR_BASELINE), betas=(0.9, 0.999), eps=1e-15, deterministic=det)


# Measured NVLink rate used as the multicast update's denominator: a peer copy of 770 GB/s
# per direction per GPU on this pool's B200s (900 GB/s nominal).
NVLINK_GBS = 770.0


def _kernel_bytes(name: str, n: int, views: int, pairs: float, launches_per_step: float,
                  adam_rows: int, world: int, q: int) -> float | None:
    """Algorithmic bytes of ONE timed launch of the kernels with a byte model (the minimum
    the algorithm moves, not what the implementation happens to move):

    * train_project (all of the rank's views in one pass over the rows; the step's
      launches split the N rows -- one launch, or one per row chunk when the next step's
      projection follows the multicast update chunk by chunk): the SH3 parameters once
      (236 B per Gaussian) and per view the 48 B record (mean 8, conic 12, colour 12,
      opacity 4, depth key 4, rectangle 8);
    * radix_pass32 (one pass of the depth sort over N): 4 B key + 4 B value read and written;
    * tile_filter (the per-tile lists from the sorted super-tile lists): 4 B per (Gaussian,
      tile) pair written, a lower bound (its reads are per super-tile item);
    * param_bwd: per row the parameters read and their gradients written (236 B each) and
      the 2D-gradient rows (36 B) of every view; the step's launches split the N rows
      (one launch on one GPU, one per row chunk with the pipelined multicast update);
    * sparse_adam (the five group launches under one timer): 28 B per parameter value
      (p, m, v, g read; p, m, v written) for the 59 values of each row this rank updates
      (all N rows on one GPU, its owned rows with the NCCL owner-sharded update);
    * sparse_adam_mc (NVLink, bytes per direction per GPU): in a launch this GPU owns q
      rows of a chunk of world * q rows; its partial gradients and count of every row of the
      chunk leave it for the switch's load-reduce (world * q * 240 B) and its q updated
      rows leave it for the multicast store (q * 236 B); the same amount arrives.
    The rasterisers and the loss filters are SM-issue bound and have no entry; the two
    passes of the super-tile sort (tile_sort_emit, tile_sort_pass) move per super-tile item
    bytes whose count the timer does not see, and have no entry either."""
    if name == "train_project":
        return (n * 236.0 + views * n * 48.0) / max(launches_per_step, 1.0)
    if name == "radix_pass32":
        return n * 16.0
    if name == "tile_filter":
        return pairs * 4.0
    if name == "param_bwd":
        return (n * 472.0 + views * n * 36.0) / max(launches_per_step, 1.0)
    if name == "sparse_adam":
        return adam_rows * 59 * 28.0 / max(launches_per_step, 1.0)
    if name == "sparse_adam_mc":
        return q * (world * 240.0 + 236.0)
    return None


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of a byte-modelled
# kernel, measured by ncu on the C4 scene with one view, and the unit it scales with at the
# bench's size. Empty: the depth-sort pass, the largest such kernel, keeps its keys and
# values in L2 at C4 (24 MB) but not at C5 (96 MB), so no scaled C4 figure describes the
# bench's launch, and the roofline object reports traffic null with that reason.
NCU_TRAFFIC_C4_1VIEW: dict = {}
C4_1VIEW_PAIRS = 21898068.0


def _traffic(name: str, pairs: float) -> float | None:
    t = NCU_TRAFFIC_C4_1VIEW.get(name)
    if t is None:
        return None
    return t[0] * pairs / C4_1VIEW_PAIRS


def summarize_kernels(rep: dict, ksteps: int, n: int, views: int, pairs: float, px: int,
                      peaks: dict, adam_rows: int | None = None, world: int = 1, q: int = 0):
    """Per-kernel figures from the library's timer report ({name: (total ms, launches)} over
    ksteps steps), the roofline object for the largest kernel with an HBM byte model, and
    the sort's share of the step. adam_rows: rows this rank's sparse Adam updates per step
    (default n); world, q: GPUs and owned rows per chunk of the multicast update."""
    adam_rows = n if adam_rows is None else adam_rows
    per_kernel = {}
    for k, (tot, cnt) in rep.items():
        avg = tot / cnt
        lps = cnt / ksteps
        entry = {"ms_per_launch": avg, "launches_per_step": lps, "ms_per_step": tot / ksteps}
        b = _kernel_bytes(k, n, views, pairs, lps, adam_rows, world, q)
        if b is not None:
            gbs = b / (avg / 1e3) / 1e9
            if k == "sparse_adam_mc":
                entry.update({"link_bytes_per_direction": b, "achieved_link_gbs": gbs,
                              "frac_nvlink": gbs / NVLINK_GBS})
            else:
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
                "traffic_source": ("ncu dram bytes of one launch at C4 / 1 view, scaled by pairs"
                                   if dom_name in NCU_TRAFFIC_C4_1VIEW else
                                   "null: no ncu capture of this launch at the bench's size (the "
                                   "C4 capture's keys stay in L2, the C5 launch's do not)"),
                "peak_source": peaks["source"],
                "note": "largest HBM-bound kernel of the step; the rasterisers "
                        f"({', '.join(f'{k} {v:.1f} ms' for k, v in raster.items())} per step) "
                        "are SM-issue bound and have no HBM roofline"}
    sort_parts = {k: per_kernel[k] for k in ("radix_hist", "radix_pass32", "pair_offsets",
                                             "tile_counts", "tile_sort_emit", "tile_sort_pass",
                                             "tile_filter")
                  if k in per_kernel}
    sort_in_step = None
    if sort_parts:
        sort_in_step = {"ms_per_step": sum(v["ms_per_step"] for v in sort_parts.values()),
                        "parts": sorted(sort_parts)}
    return per_kernel, roofline, sort_in_step


def ranks_list(x: float, world: int) -> list[float]:
    """x of every rank, in rank order (one small allreduce)."""
    if world == 1:
        return [x]
    import torch.distributed as dist
    t = torch.zeros(world, dtype=torch.float64, device="cuda")
    t[dist.get_rank()] = x
    dist.all_reduce(t)
    return [float(v) for v in t.tolist()]


def run(args, rank: int, world: int, local: int) -> dict:
    from bench import ClockSampler, barrier, max_over_ranks, measured_peaks, sum_over_ranks  # noqa: E402
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
    # GS_BENCH_MC_CHUNKS: row chunks of the pipelined multicast update (default 4)
    chunks = int(os.environ.get("GS_BENCH_MC_CHUNKS", "4"))
    tr = Trainer(params, cfg, per, H, W, device=dev, sharded_optimizer=sharded, multicast=multicast,
                 mc_chunks=chunks)
    del params
    cams = [(cm.w2c, cm.K, H, W) for cm in mine]
    # Every step trains on the same views, so each step hands them on as the next step's
    # cameras: their projection runs at the end of the step, behind the update
    # (GS_BENCH_PREFETCH=0: each step projects its own views at its start).
    nxt = cams if os.environ.get("GS_BENCH_PREFETCH", "1") != "0" else None
    pairs0 = tr.count_pairs(cams)
    tr._alloc(int(max(pairs0) * 1.3) + 4096)
    targets = [torch.from_numpy(t).to(dev) for t in targets_host]
    st = torch.cuda.current_stream()

    for i in range(args.warmup):
        tr.step(cams, targets, check_errors=(i == 0), next_cams=nxt)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(world)
        torch.cuda.synchronize()
        l0 = lib.gs_launch_count()
        e0.record()
        for _ in range(args.steps):
            tr.step(cams, targets, next_cams=nxt)
        e1.record()
        launches = lib.gs_launch_count() - l0
        torch.cuda.synchronize()
        barrier(world)
    if lib.gs_workspace_error(tr.ws.data_ptr(), st.cuda_stream) != 0:
        raise RuntimeError("a timed step overflowed its pair buffers or timed out")
    ms_rank = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(ms_rank, world)
    ms_by_rank = ranks_list(ms_rank, world)
    total_px = V * H * W
    value = total_px / (ms / 1e3) / 1e6
    loss_now = float(tr.losses.sum().item())

    # e2e: the public API given the step's inputs (target images) in pinned host memory --
    # the library copies every view's target host -> device each step, on its own stream
    # overlapped with the other views' work -- and every step's loss read back to the host.
    # The loss of step i is copied to pinned memory at the end of step i and read on the
    # host once step i + 1 has been enqueued (as a training loop that logs its losses does),
    # so the GPU is not left idle while the host waits; the last step's loss is read inside
    # the timed region too. The same loop with a blocking read after every step is reported
    # beside it.
    pinned = [torch.from_numpy(t).pin_memory() for t in targets_host]
    loss_pin = torch.zeros(args.steps, dtype=torch.float32).pin_memory()
    done = [torch.cuda.Event() for _ in range(args.steps)]
    losses_read = []

    def e2e_loop(blocking: bool) -> float:
        for _ in range(2):
            tr.step(cams, pinned, next_cams=nxt)
            tr.losses.sum().item()
        barrier(world)
        torch.cuda.synchronize()
        losses_read.clear()
        e0.record()
        for i in range(args.steps):
            tr.step(cams, pinned, next_cams=nxt)
            if blocking:
                losses_read.append(tr.losses.sum().item())
                continue
            loss_pin[i:i + 1].copy_(tr.losses.sum().reshape(1), non_blocking=True)
            done[i].record()
            if i > 0:
                done[i - 1].synchronize()
                losses_read.append(float(loss_pin[i - 1]))
        if not blocking:
            done[args.steps - 1].synchronize()
            losses_read.append(float(loss_pin[args.steps - 1]))
        e1.record()
        torch.cuda.synchronize()
        assert len(losses_read) == args.steps and all(np.isfinite(losses_read))
        return max_over_ranks(e0.elapsed_time(e1) / args.steps, world)

    e2e_ms = e2e_loop(blocking=False)
    e2e_blocking_ms = e2e_loop(blocking=True)

    # per-kernel device times (CUDA events on the launching stream), one more short loop;
    # with the timer on the library runs the views on one stream, so launches do not overlap
    # and their sum is the serial step time (the timed step above overlaps two views)
    lib.gs_timing_reset()
    lib.gs_timing_enable(1)
    ksteps = max(2, min(args.steps, 5))
    for _ in range(ksteps):
        tr.step(cams, targets, next_cams=nxt)
    torch.cuda.synchronize()
    lib.gs_timing_enable(0)
    rep = timing_report()
    lib.gs_timing_reset()
    pairs = tr.pairs.float().mean().item()
    peaks = measured_peaks()
    adam_rows = tr.n if world == 1 else (tr.chunks * tr.q if tr.multicast else tr.rows_per)
    per_kernel, roofline, sort_in_step = summarize_kernels(rep, ksteps, tr.n, per, pairs, H * W,
                                                           peaks, adam_rows, world, tr.q)
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
                       else " + NCCL allreduce, replicated Adam") + (
                       "; each step projects the next step's views after its update"
                       + (", row chunk by row chunk as the chunks land" if tr.multicast else "")
                       if nxt is not None else ""),
                   "gradient_sums": "fixed-order slots (deterministic mode)" if cfg.deterministic
                   else "float atomics",
                   "l2": "inputs larger than L2 (params 1.4 GB, pairs per view > 100 MB)"},
        "e2e": {"value": total_px / (e2e_ms / 1e3) / 1e6, "unit": "Mpix/s",
                "h2d_bytes_per_step": int(sum(t.size * 4 for t in targets_host)),
                "d2h_bytes_per_step": 4,
                "loss_read": "every step; step i's loss read on the host after step i + 1 is enqueued",
                "value_blocking_read": total_px / (e2e_blocking_ms / 1e3) / 1e6},
        # the library's kernels launched in the timed region, summed over the ranks
        "gpu_launches": int(sum_over_ranks(float(launches), world)),
        "ms_per_step_by_rank": ms_by_rank,
        "pairs_per_view": pairs, "loss": loss_now,
        "kernels": per_kernel,
        "clocks": clk.summary(),
    }
    out["roofline"] = roofline
    if sort_in_step is not None:
        out["sort_in_step"] = sort_in_step
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.baseline import train_cpu_baseline
        out["cpu_baseline"] = train_cpu_baseline(name)
    return out
