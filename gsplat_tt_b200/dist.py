"""Host-side plumbing of the view-parallel trainer (device-agnostic, so it runs on gloo/CPU
in tests and on NCCL/CUDA in training).

The reference has no multi-device trainer (its multi-chip mode is alternate-frame
rendering over process pipes, render/afr.py:1-33); here every rank holds the full
parameters, renders a contiguous share of the step's views, and one allreduce sums the
per-Gaussian gradients, visibility counts and the ranks' error flags.
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
