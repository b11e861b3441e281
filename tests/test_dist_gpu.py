"""View-parallel training on 2 GPUs: the owner-sharded optimizer -- through NVLink
multicast (gs_sparse_adam_multicast) where the GPUs support it, and through NCCL
reduce-scatter / all-gather -- gives every rank the same parameters as the allreduce +
replicated Adam, after two steps. Skipped with fewer than 2 GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from gsplat_tt_b200 import scenes
    from gsplat_tt_b200.dist import view_slice
    from gsplat_tt_b200.train import TrainConfig, Trainer
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        params = scenes.cluster_scene(5001, sh_degree=3, seed=11)
        params["means"] = (params["means"] * 0.5).astype(np.float32)
        params["log_scales"] = (params["log_scales"] + 1.5).astype(np.float32)
        H, W = 72, 100
        rng = np.random.default_rng(2)
        cams, tgts = [], []
        for _ in range(4):
            d = rng.standard_normal(3)
            d /= np.linalg.norm(d)
            cams.append((scenes.look_at(3.5 * d), scenes.intrinsics(90.0, W, H), H, W))
            tgts.append(rng.uniform(0, 1, (H, W, 3)).astype(np.float32))
        lo, hi = view_slice(4, world, rank)
        cfg = TrainConfig(sh_degree=3, tile_size=16)
        out, used_mc = {}, False
        for mode in ("multicast", "nccl", "allreduce"):
            tr = Trainer(params, cfg, hi - lo, H, W, sharded_optimizer=mode != "allreduce",
                         multicast=mode == "multicast")
            if mode == "multicast":
                used_mc = tr.multicast
            tr.ensure_capacity(cams[lo:hi])
            for _ in range(2):
                tr.step(cams[lo:hi], tgts[lo:hi], check_errors=True)
            torch.cuda.synchronize()
            out[mode] = tr.params.numpy()
            del tr
        ref = out["allreduce"]
        diff = {m: max(float(np.abs(out[m][k] - ref[k]).max()) for k in ref) for m in ("multicast", "nccl")}
        moved = max(float(np.abs(ref[k] - np.asarray(params[k], np.float32).reshape(ref[k].shape)).max())
                    for k in ref)
        q.put((rank, diff, moved, used_mc))
        dist.barrier()
    except Exception:  # report at once instead of leaving the parent waiting on the queue
        import traceback
        q.put((rank, "error", traceback.format_exc(), None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_optimizer_matches_allreduce_on_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = []
    while len(res) < 2:
        res.append(q.get(timeout=300))
        if res[-1][1] == "error":  # the other rank ends through its process-group timeout
            break
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    errors = [r for r in res if r[1] == "error"]
    assert not errors, errors[0][2]
    for p in procs:
        assert p.exitcode == 0
    for rank, diff, moved, used_mc in res:
        print(f"rank {rank}: multicast update {'used' if used_mc else 'unavailable'}; "
              f"max diff vs allreduce {diff}")
        assert moved > 0.0, "Adam did not update the parameters"
        # the sums of two ranks are order-free, but the backward rasteriser accumulates
        # per-Gaussian gradients with float atomics, so two runs differ in the last bits
        assert diff["multicast"] <= 1e-6 and diff["nccl"] <= 1e-6, (rank, diff)
