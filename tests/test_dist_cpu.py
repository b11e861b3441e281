"""The view-parallel trainer's host plumbing on CPU with gloo, world size 2: the view split,
the single allreduce of gradients + visibility counts + error flags (every rank takes the
same skip decision), and a rank that dies before the collective (the survivor's collective
fails within the process-group timeout instead of hanging)."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from gsplat_tt_b200.dist import reduce_step_buffer, view_slice


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _reduce_worker(rank, world, port, fail_rank, q):
    dist = _init(rank, world, port, 30)
    n = 5
    flat = torch.full((3 * n + n + 1,), float(rank + 1))
    err_slot = flat[-1:]
    skip = torch.zeros(1, dtype=torch.int32)
    local_err = torch.tensor([1 if rank == fail_rank else 0], dtype=torch.int32)
    reduce_step_buffer(flat, err_slot, local_err, skip)
    q.put((rank, flat[:-1].tolist(), float(err_slot.item()), int(skip.item())))
    dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_allreduce_sums_and_agrees_on_skip(fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_reduce_worker, args=(r, 2, port, fail_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, vals, err, skip in res:
        assert all(v == 3.0 for v in vals)  # 1 + 2 on both ranks
        assert skip == (1 if fail_rank >= 0 else 0)
        assert err == (1.0 if fail_rank >= 0 else 0.0)


def _dead_worker(rank, world, port, q):
    dist = _init(rank, world, port, 5)
    if rank == 1:
        os._exit(0)  # leaves between steps, before the step's collective
    flat = torch.ones(8)
    try:
        dist.all_reduce(flat)
        q.put("completed")
    except Exception as exc:  # noqa: BLE001
        q.put(f"error: {type(exc).__name__}")


def test_dead_rank_fails_the_survivors_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_dead_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg.startswith("error"), msg


def test_view_slice():
    assert [view_slice(32, 4, r) for r in range(4)] == [(0, 8), (8, 16), (16, 24), (24, 32)]
    with pytest.raises(ValueError):
        view_slice(32, 3, 0)
