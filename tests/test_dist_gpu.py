"""View-parallel training on 2 GPUs: the owner-sharded optimizer -- through NVLink
multicast (gs_sparse_adam_multicast) where the GPUs support it, and through NCCL
reduce-scatter / all-gather, each also with the next step's projection run behind the
update (next_cams) -- gives every rank the same parameters as the allreduce + replicated
Adam, after two steps, bit for bit: the ranks' gradient sums use the deterministic mode
(fixed-order per-Gaussian sums on each GPU), and a sum of two ranks' partial gradients has
one result whichever path adds them. Skipped with fewer than 2 GPUs."""
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


def _run(rank, world, params, live):
    """The comparison itself; every Trainer is appended to `live`, so none is freed (and
    none of its symmetric buffers unmapped) before every rank has passed its GPU work."""
    from gsplat_tt_b200 import scenes
    from gsplat_tt_b200.dist import view_slice
    from gsplat_tt_b200.train import TrainConfig, Trainer
    H, W = 72, 100
    rng = np.random.default_rng(2)
    cams, tgts = [], []
    for _ in range(4):
        d = rng.standard_normal(3)
        d /= np.linalg.norm(d)
        cams.append((scenes.look_at(3.5 * d), scenes.intrinsics(90.0, W, H), H, W))
        tgts.append(rng.uniform(0, 1, (H, W, 3)).astype(np.float32))
    lo, hi = view_slice(4, world, rank)
    cfg = TrainConfig(sh_degree=3, tile_size=16, deterministic=True)
    out, used_mc = {}, False
    for mode in ("multicast", "multicast_ahead", "nccl", "nccl_ahead", "allreduce"):
        tr = Trainer(params, cfg, hi - lo, H, W, sharded_optimizer=mode != "allreduce",
                     multicast=mode.startswith("multicast"), mc_chunks=3)
        live.append(tr)
        if mode == "multicast":
            used_mc = tr.multicast
        tr.ensure_capacity(cams[lo:hi])
        for _ in range(2):
            if mode.endswith("_ahead"):
                # the next step's projection, chunk by chunk behind the update (multicast) or
                # after it (NCCL); the second step starts from it
                tr.step(cams[lo:hi], tgts[lo:hi], next_cams=cams[lo:hi])
                assert tr._projected is not None
            else:
                tr.step(cams[lo:hi], tgts[lo:hi], check_errors=True)
        torch.cuda.synchronize()
        out[mode] = tr.params.numpy()
    ref = out["allreduce"]
    diff = {m: max(float(np.abs(out[m][k] - ref[k]).max()) for k in ref)
            for m in ("multicast", "multicast_ahead", "nccl", "nccl_ahead")}
    moved = max(float(np.abs(ref[k] - np.asarray(params[k], np.float32).reshape(ref[k].shape)).max())
                for k in ref)
    return diff, moved, used_mc


def _worker(rank, world, port, q):
    """One rank. Whatever happens, it reports on the queue, then meets the other ranks at a
    host-side (gloo) barrier before it frees any buffer bound to the NVLink multicast object,
    and only then tears down: a rank must never exit, or be killed, while a peer may still
    reach its memory through the multicast mapping. NCCL timeouts abort the communicator
    and raise in this process (error handling mode 2) instead of ending it."""
    os.environ["TORCH_NCCL_ASYNC_ERROR_HANDLING"] = "2"
    import torch.distributed as dist
    from gsplat_tt_b200 import scenes
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    host = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=600))
    live = []
    try:
        params = scenes.cluster_scene(5001, sh_degree=3, seed=11)
        params["means"] = (params["means"] * 0.5).astype(np.float32)
        params["log_scales"] = (params["log_scales"] + 1.5).astype(np.float32)
        diff, moved, used_mc = _run(rank, world, params, live)
        status = (rank, diff, moved, used_mc)
    except Exception:  # reported on the host; the teardown below is the same either way
        import traceback
        status = (rank, "error", traceback.format_exc(), None)
    q.put(status)
    try:  # this rank's own GPU work has ended before it waits for the others
        torch.cuda.synchronize()
    except Exception:
        pass
    dist.barrier(group=host)   # every rank is past its GPU work: nobody reads peer memory now
    live.clear()               # frees the Trainers and their symmetric buffers
    torch.cuda.synchronize()
    dist.barrier(group=host)   # every rank has freed its buffers before anyone exits
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_optimizer_matches_allreduce_on_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    # every rank reports, error or not, and then tears down on its own after the host-side
    # barrier; the ranks are never killed (they may hold multicast-bound memory)
    res = [q.get(timeout=900) for _ in range(2)]
    for p in procs:
        p.join(timeout=900)
    assert not any(p.is_alive() for p in procs), "a rank did not finish its teardown"
    errors = [r for r in res if r[1] == "error"]
    assert not errors, errors[0][2]
    for p in procs:
        assert p.exitcode == 0
    for rank, diff, moved, used_mc in res:
        print(f"rank {rank}: multicast update {'used' if used_mc else 'unavailable'}; "
              f"max diff vs allreduce {diff}")
        assert moved > 0.0, "Adam did not update the parameters"
        # each GPU's sums are deterministic and a sum of two ranks is order-free
        assert max(diff.values()) == 0.0, (rank, diff)
