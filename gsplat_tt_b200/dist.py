"""Host-side plumbing of the view-parallel trainer (device-agnostic, so it runs on gloo/CPU
in tests and on NCCL/CUDA in training).

The reference has no multi-device trainer (its multi-chip mode is alternate-frame
rendering over process pipes, render/afr.py:1-33); here every rank holds the full
parameters and renders a contiguous share of the step's views. The gradients are then
combined in one of two ways:

* `reduce_step_buffer`: one allreduce sums the per-Gaussian gradients, visibility counts
  and the ranks' error flags, and every rank runs the identical sparse Adam on all rows;
* `sharded_update` (the owner-sharded optimizer): each rank owns a contiguous range of
  Gaussian rows; a reduce-scatter gives it the summed gradients and counts of its rows
  only, it runs sparse Adam on those rows (its Adam moments are only ever touched there),
  and an in-place all-gather of the parameters brings every rank's updated rows to all.
  The same bytes cross the links as with the allreduce, but the Adam work and the moment
  traffic are divided by the number of ranks.
"""
from __future__ import annotations

import torch


def view_slice(n_views: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's views; the views must split evenly."""
    if n_views % world != 0:
        raise ValueError(f"{n_views} views do not split evenly over {world} ranks")
    per = n_views // world
    return rank * per, (rank + 1) * per


def reduce_step_buffer(flat: torch.Tensor, err_slot: torch.Tensor, local_error: torch.Tensor,
                       skip_out: torch.Tensor, group=None) -> None:
    """Sum `flat` (gradients, visibility counts and the trailing error slot) over ranks.

    `err_slot` is a view of the last element(s) of `flat`; it is set from this rank's
    `local_error` (non-zero: the step failed here) before the reduction, so afterwards every
    rank sees the same total and `skip_out` (int32) is 1 on all ranks when any rank failed.
    Enqueued asynchronously on the current stream (no host synchronisation)."""
    import torch.distributed as dist
    err_slot.copy_((local_error != 0).to(err_slot.dtype).reshape(err_slot.shape))
    dist.all_reduce(flat, group=group)
    skip_out.copy_((err_slot.reshape(-1)[:1] > 0).to(torch.int32))


def shard_rows(n: int, world: int) -> int:
    """Rows per rank of the owner-sharded optimizer: rank r owns Gaussian rows
    [r * rows, (r + 1) * rows); arrays are padded to world * rows rows (padding rows have
    a zero visibility count, so Adam never updates them). A multiple of 4, so every rank's
    first row of every group starts on a 16-byte boundary (vectorised Adam loads)."""
    return max(4, -(-n // (4 * world)) * 4)


def owned_rows(chunk: int, rank: int, world: int, q: int) -> tuple[int, int]:
    """[begin, end) of the rows rank owns in row chunk `chunk` of the pipelined multicast
    update: chunk c spans rows [c * world * q, (c + 1) * world * q) and rank r owns the q
    rows at offset r * q inside it."""
    b = chunk * world * q + rank * q
    return b, b + q


def sharded_update(grad_groups, grad_shards, param_groups, local_error, err, skip_out, rank: int,
                   world: int, adam_fn, group=None) -> None:
    """One owner-sharded optimizer update, enqueued asynchronously on the current stream.

    grad_groups / param_groups: per parameter group (and, last in grad_groups, the
    visibility counts) a flat view of world * rows * width elements; grad_shards: the
    matching rows * width buffers that receive this rank's reduced rows. `err` (1 float)
    receives the number of ranks whose step failed (from `local_error`, non-zero = failed);
    `skip_out` (int32) is 1 on every rank when any failed. adam_fn(skip_out) updates this
    rank's parameter rows from grad_shards (and must honour skip_out). Every rank takes
    the same collectives in the same order, also when the step is skipped."""
    import torch.distributed as dist
    from torch.distributed.distributed_c10d import _coalescing_manager
    err.copy_((local_error != 0).to(err.dtype).reshape(err.shape))
    dist.all_reduce(err, group=group)
    skip_out.copy_((err.reshape(-1)[:1] > 0).to(torch.int32))
    # each set of per-group collectives goes to the backend as one coalesced call (one NCCL
    # group launch instead of one launch per parameter group)
    with _coalescing_manager(group=group):
        for full, shard in zip(grad_groups, grad_shards):
            dist.reduce_scatter_tensor(shard, full, group=group)
    adam_fn(skip_out)
    with _coalescing_manager(group=group):
        for full in param_groups:
            chunk = full.numel() // world
            dist.all_gather_into_tensor(full, full[rank * chunk:(rank + 1) * chunk], group=group)



def symmetric_buffer(numel: int, device, group=None):
    """A zeroed fp32 buffer of `numel` elements in CUDA symmetric memory -- mapped by every
    rank of `group` and bound to an NVLink multicast object when the GPUs support one --
    its handle, and its multicast address (None without multicast support). Collective:
    every rank calls it with the same `numel`, in the same order. The buffer is its own
    allocation (not carved from a pool), so the multicast address maps the tensor's bytes
    from its first one; that is checked through the handle's view of this rank's buffer."""
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm
    from torch._C._autograd import DeviceType
    device = torch.device(device)
    t = symm._SymmetricMemory.empty_strided_p2p((numel,), (1,), torch.float32, device)
    t.zero_()
    h = symm.rendezvous(t, group if group is not None else dist.group.WORLD)
    ok = (symm._SymmetricMemory.has_multicast_support(DeviceType.CUDA, device.index)
          and int(h.buffer_ptrs[h.rank]) == t.data_ptr()
          and int(h.buffer_size) >= 4 * numel)
    mc = int(h.multicast_ptr) if ok else 0
    return t, h, (mc if mc else None)
