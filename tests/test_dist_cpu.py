"""The view-parallel trainer's host plumbing on CPU with gloo, world size 2: the view split,
the single allreduce of gradients + visibility counts + error flags (every rank takes the
same skip decision), the owner-sharded update (reduce-scatter, Adam on owned rows,
all-gather) against the allreduce, the chunked row ownership of the multicast update, the
symmetric-buffer host logic against a fake of torch's API, and a rank that dies before the
collective (the survivor's collective fails within the process-group timeout)."""
import datetime
import os
import socket

import numpy as np
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
        if p.is_alive():  # a CPU-only gloo rank: it holds no GPU memory
            p.kill()
    assert msg.startswith("error"), msg


def test_view_slice():
    assert [view_slice(32, 4, r) for r in range(4)] == [(0, 8), (8, 16), (16, 24), (24, 32)]
    with pytest.raises(ValueError):
        view_slice(32, 3, 0)


def _adam_rows(p, g, m, v, vis, skip, lr=0.1, b1=0.9, b2=0.999, eps=1e-8):
    """Sparse Adam stand-in over rows (rows with a zero count are left alone)."""
    if int(skip.item()):
        return
    w = p.numel() // vis.numel()
    sel = (vis > 0).repeat_interleave(w)
    m[sel] = b1 * m[sel] + (1 - b1) * g[sel]
    v[sel] = b2 * v[sel] + (1 - b2) * g[sel] * g[sel]
    p[sel] -= lr * m[sel] / (v[sel].sqrt() + eps)


def _sharded_worker(rank, world, port, fail_rank, q):
    from gsplat_tt_b200.dist import shard_rows, sharded_update
    dist = _init(rank, world, port, 30)
    n, widths = 7, (3, 4, 1)
    rows = shard_rows(n, world)
    total = rows * world
    torch.manual_seed(0)
    params0 = [torch.zeros(total * w) for w in widths]
    for t, w in zip(params0, widths):
        t[:n * w] = torch.randn(n * w)
    gen = torch.Generator().manual_seed(100 + rank)
    grads = [torch.zeros(total * w) for w in widths]
    for t, w in zip(grads, widths):
        t[:n * w] = torch.randn(n * w, generator=gen)
    vis = torch.zeros(total)
    vis[:n] = (torch.rand(n, generator=gen) > 0.3).float()
    local_err = torch.tensor([1 if rank == fail_rank else 0], dtype=torch.int32)

    # allreduce reference: every rank updates every row
    ref_p = [t.clone() for t in params0]
    ref_g = [t.clone() for t in grads]
    ref_vis = vis.clone()
    for t in ref_g + [ref_vis]:
        dist.all_reduce(t)
    ref_err = local_err.clone().float()
    dist.all_reduce(ref_err)
    ref_skip = (ref_err > 0).to(torch.int32)
    for p, g, w in zip(ref_p, ref_g, widths):
        _adam_rows(p, g, torch.zeros_like(p), torch.zeros_like(p), ref_vis, ref_skip)

    # owner-sharded: reduce-scatter, Adam on this rank's rows, all-gather
    params = [t.clone() for t in params0]
    shards = [torch.zeros(rows * w) for w in widths] + [torch.zeros(rows)]
    moments = [(torch.zeros(rows * w), torch.zeros(rows * w)) for w in widths]
    err = torch.zeros(1)
    skip = torch.zeros(1, dtype=torch.int32)

    def adam(skip_flag):
        for p, g, (m, v), w in zip(params, shards, moments, widths):
            own = p[rank * rows * w:(rank + 1) * rows * w]
            _adam_rows(own, g, m, v, shards[-1], skip_flag)

    sharded_update(grads + [vis], shards, params, local_err, err, skip, rank, world, adam)
    diff = max(float((a - b).abs().max()) for a, b in zip(params, ref_p))
    pad_ok = all(float(p[n * w:].abs().max()) == 0.0 for p, w in zip(params, widths))
    q.put((rank, diff, pad_ok, int(skip.item()), float(err.item()),
           max(float((a - b).abs().max()) for a, b in zip(params, params0))))
    dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank", [-1, 0])
def test_sharded_update_matches_allreduce_update(fail_rank):
    """Reduce-scatter + owner Adam + all-gather gives every rank the same parameters as the
    allreduce + replicated Adam; a failed rank makes every rank skip the update."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, 2, port, fail_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, diff, pad_ok, skip, err, moved in res:
        assert diff <= 1e-6, (rank, diff)
        assert pad_ok
        assert skip == (1 if fail_rank >= 0 else 0) and err == (1.0 if fail_rank >= 0 else 0.0)
        assert (moved == 0.0) == (fail_rank >= 0)


def test_shard_rows():
    from gsplat_tt_b200.dist import shard_rows
    assert shard_rows(7, 2) == 4 and shard_rows(8, 2) == 4 and shard_rows(9, 2) == 8
    assert shard_rows(1, 8) == 4 and shard_rows(6_000_001, 8) % 4 == 0
    for n in (1, 5, 1000, 12345):
        for w in (1, 2, 4, 8):
            assert shard_rows(n, w) * w >= n


class _FakeHandle:
    """Stands in for torch's symmetric-memory handle with the interface of its type stub
    (properties rank / buffer_ptrs / buffer_size / multicast_ptr)."""

    def __init__(self, t, mc):
        self._t, self._mc = t, mc

    @property
    def rank(self):
        return 0

    @property
    def buffer_ptrs(self):
        return [self._t.data_ptr()]

    @property
    def buffer_size(self):
        return self._t.numel() * 4

    @property
    def multicast_ptr(self):
        return self._mc


@pytest.mark.parametrize("supported", [True, False])
def test_symmetric_buffer_host_logic(monkeypatch, supported):
    """symmetric_buffer against a fake of the symmetric-memory API (the real one needs CUDA):
    the static multicast query takes (device type, index), the handle's fields are properties."""
    import torch.distributed._symmetric_memory as symm
    from gsplat_tt_b200 import dist as gd

    class FakeSM:
        @staticmethod
        def empty_strided_p2p(size, stride, dtype, device, group_name=None, alloc_id=None):
            assert stride == (1,) and dtype == torch.float32
            return torch.full(size, 7.0)

        @staticmethod
        def has_multicast_support(device_type, device_idx):
            assert isinstance(device_idx, int)
            return supported

    monkeypatch.setattr(symm, "_SymmetricMemory", FakeSM)
    monkeypatch.setattr(symm, "rendezvous", lambda t, g: _FakeHandle(t, 0x7F0000000000))
    monkeypatch.setattr(torch.distributed, "group",
                        type("G", (), {"WORLD": type("PG", (), {"group_name": "0"})()}))
    t, h, mc = gd.symmetric_buffer(16, "cpu:0")
    assert t.numel() == 16 and float(t.abs().max()) == 0.0  # zeroed
    assert mc == (0x7F0000000000 if supported else None)


@pytest.mark.parametrize("n,world,chunks", [(5001, 2, 4), (6_000_000, 8, 4), (7, 4, 4), (1000, 3, 1)])
def test_owned_rows_partition_the_padded_rows(n, world, chunks):
    """Chunked ownership of the multicast update: every padded row has exactly one owner,
    every owner's range starts on a 16-byte boundary, and the padding covers n."""
    from gsplat_tt_b200.dist import owned_rows, shard_rows
    q = shard_rows(-(-n // chunks), world)
    total = chunks * world * q
    assert total >= n and q % 4 == 0
    seen = np.zeros(total, np.int32) if total < 10_000_000 else None
    spans = sorted(owned_rows(c, r, world, q) for c in range(chunks) for r in range(world))
    assert spans[0][0] == 0 and spans[-1][1] == total
    for (b0, e0), (b1, _) in zip(spans, spans[1:]):
        assert e0 == b1 and b0 % 4 == 0
    if seen is not None:
        for b, e in spans:
            seen[b:e] += 1
        assert (seen == 1).all()
