"""Process-parallel driver of the oracle training step (TEST INFRASTRUCTURE ONLY: used by
the CPU baseline of bench.py and by the tests, never by the product).

A multi-view step's views are independent until their gradients are summed
(oracle.train.train_step, which restates gsplat/train_oracle.py's per-view loop and
sparse_adam_step). ViewPool gives each worker process one view at a time -- projection,
forward, loss, blend backward and projection backward, the same calls train_step makes --
and the parent sums the per-view gradients in view order and applies sparse Adam once, so
the result equals train_step's. The pool uses the spawn start method (safe in a process
that has already used the GPU) and one BLAS thread per worker.
"""
from __future__ import annotations

import multiprocessing as mp
import os

import numpy as np

from . import train as ot

_P = None
_CFG = None
_SSIM = True
_LAMBDA = 0.2


def _init(params, cfg, ssim, lambda_dssim):
    global _P, _CFG, _SSIM, _LAMBDA
    _P, _CFG, _SSIM, _LAMBDA = params, cfg, ssim, lambda_dssim


def _view(task):
    w2c, K, H, W, tgt = task
    pr = ot.project(_P, w2c, K, H, W, _CFG)
    fw = ot.forward(pr, H, W, _CFG)
    L, dimg = (ot.loss_ssim if _SSIM else ot.loss_l1)(fw["image"], tgt, _LAMBDA)
    g2 = ot.backward_2d(pr, fw["image"], dimg, H, W, _CFG)
    gp = ot.param_backward(_P, g2, w2c, K, H, W, _CFG)
    return gp, np.asarray(pr["visible"], bool), float(L)


_THREAD_VARS = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")


class ViewPool:
    """`workers` spawned processes holding `params` (fixed for the pool's lifetime)."""

    def __init__(self, params, cfg, workers: int, ssim: bool = True, lambda_dssim: float = 0.2):
        self.params = params
        self.workers = max(1, int(workers))
        saved = {k: os.environ.get(k) for k in _THREAD_VARS}
        for k in _THREAD_VARS:  # inherited by the children at spawn
            os.environ[k] = "1"
        try:
            self.pool = mp.get_context("spawn").Pool(self.workers, initializer=_init,
                                                     initargs=(params, cfg, ssim, lambda_dssim))
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v

    def step(self, m, v, step, cams, targets, lr=None, betas=(0.9, 0.999), eps=1e-15,
             bf16_moments=False):
        """train_step with the views spread over the workers; returns params, m, v, loss,
        grads and visible like oracle.train.train_step."""
        tasks = [(w2c, K, H, W, t) for (w2c, K, H, W), t in zip(cams, targets)]
        res = self.pool.map(_view, tasks, chunksize=1)
        N = np.asarray(self.params["means"]).shape[0]
        total = {k: np.zeros_like(np.asarray(self.params[k], np.float32)) for k in ot.PARAM_NAMES}
        vis = np.zeros(N, bool)
        loss = 0.0
        for gp, vv, L in res:  # view order, as train_step sums
            for k in ot.PARAM_NAMES:
                total[k] += gp[k]
            vis |= vv
            loss += L
        P, Mo, Vo = ot.sparse_adam(self.params, total, m, v, step, vis, lr, betas, eps, bf16_moments)
        return {"params": P, "m": Mo, "v": Vo, "loss": loss, "grads": total, "visible": vis}

    def close(self):
        self.pool.close()
        self.pool.join()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
