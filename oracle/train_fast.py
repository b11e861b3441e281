"""ctypes front end of the C training rasteriser oracle (oracle/gs_train_oracle.c).

TEST INFRASTRUCTURE ONLY. Same signatures and results as oracle.train.forward and
oracle.train.backward_2d_exact (the numpy restatements of the reference's
gsplat/blend_backward_dev.py:404-438 forward_fast and of its 2D-gradient terms,
gsplat/blend_backward_ref.py:134-249), multithreaded in C so the parity tests can run
them on a full view of the benchmark configurations (millions of Gaussians, tens of
millions of pairs), where the numpy models take hours.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import display as _display
from . import train as ot

_f = ctypes.POINTER(ctypes.c_float)
_d = ctypes.POINTER(ctypes.c_double)
_i64 = ctypes.POINTER(ctypes.c_int64)
_i32 = ctypes.POINTER(ctypes.c_int32)
_u8 = ctypes.POINTER(ctypes.c_uint8)
_BOUND = False


def _lib():
    global _BOUND
    L = _display.lib()
    if not _BOUND:
        c_i, c_f = ctypes.c_int, ctypes.c_float
        L.gso_train_forward.argtypes = [_f, _f, _f, _f, _i64, _i64, c_i, c_i, c_i, c_f, c_f, c_f,
                                        _f, _f, _f, _i32, _u8, _i64, c_i]
        L.gso_train_forward.restype = ctypes.c_int64
        L.gso_train_backward.argtypes = [_f, _f, _f, _f, _i64, _i64, c_i, c_i, c_i, c_f, c_f, c_f,
                                         _f, _f, ctypes.c_int64, _d, _u8, c_i]
        L.gso_train_backward.restype = ctypes.c_int
        _BOUND = True
    return L


def _p(a, t):
    return a.ctypes.data_as(t)


def threads() -> int:
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return max(1, int(n or 1))


def sorted_pairs(proj, H, W, tile):
    """(Gaussian ids sorted by tile then depth bits, tile ranges (tiles, 2) int64):
    oracle.train.pair_lists with its per-tile [start, end) table."""
    tx, ty = (W + tile - 1) // tile, (H + tile - 1) // tile
    pl = ot.pair_lists(proj["rects"], proj["depth"], tx)
    return pair_table(pl["g"], pl["tid"], tx * ty)


def pair_table(ids, tids, ntiles):
    ids = np.ascontiguousarray(ids, np.int64)
    tids = np.asarray(tids, np.int64)
    r = np.zeros((ntiles, 2), np.int64)
    if tids.size:
        t = np.arange(ntiles)
        st = np.searchsorted(tids, t, "left")
        en = np.searchsorted(tids, t, "right")
        nz = en > st
        r[nz, 0], r[nz, 1] = st[nz], en[nz]
    return ids, r


def _common(proj, cfg):
    m2 = np.ascontiguousarray(proj["means2d"], np.float32)
    con = np.ascontiguousarray(proj["conic"], np.float32)
    op = np.ascontiguousarray(proj["opacity"], np.float32)
    col = np.ascontiguousarray(proj["colors"], np.float32)
    bg = np.ascontiguousarray(cfg.background, np.float32)
    return m2, con, op, col, bg


def forward(proj, H, W, cfg: ot.Cfg, pairs=None, nthreads: int | None = None) -> dict:
    """oracle.train.forward: image, final_T, n_contrib, ties, n_pairs, n_live, and
    tile_reach (per tile, the leading pairs read before every pixel stopped). `pairs`:
    (sorted ids, tile ranges) when the caller has them (sorted_pairs otherwise)."""
    ids, rng = sorted_pairs(proj, H, W, cfg.tile) if pairs is None else pairs
    m2, con, op, col, bg = _common(proj, cfg)
    img = np.empty((H, W, 3), np.float32)
    T = np.empty((H, W), np.float32)
    nc = np.empty((H, W), np.int32)
    ties = np.empty((H, W), np.uint8)
    reach = np.zeros(rng.shape[0], np.int64)
    nl = _lib().gso_train_forward(_p(m2, _f), _p(con, _f), _p(op, _f), _p(col, _f), _p(ids, _i64),
                                  _p(rng, _i64), H, W, cfg.tile, cfg.alpha_max, cfg.alpha_min,
                                  cfg.t_min, _p(bg, _f), _p(img, _f), _p(T, _f), _p(nc, _i32),
                                  _p(ties, _u8), _p(reach, _i64), nthreads or threads())
    if nl < 0:
        raise ValueError("tile size above 32")
    return {"image": img, "final_T": T, "n_contrib": nc, "ties": ties.astype(bool),
            "n_pairs": int(ids.size), "n_live": int(nl), "tile_reach": reach}


def backward_2d_exact(proj, dL_dimage, H, W, cfg: ot.Cfg, ties: bool = False, pairs=None,
                      nthreads: int | None = None):
    """oracle.train.backward_2d_exact: (N, 9) float64 2D gradients (and the (N,) tie mask)."""
    ids, rng = sorted_pairs(proj, H, W, cfg.tile) if pairs is None else pairs
    m2, con, op, col, bg = _common(proj, cfg)
    n = m2.shape[0]
    g = np.empty((n, 9), np.float64)
    tie = np.empty(n, np.uint8) if ties else None
    dimg = np.ascontiguousarray(dL_dimage, np.float32)
    rc = _lib().gso_train_backward(_p(m2, _f), _p(con, _f), _p(op, _f), _p(col, _f), _p(ids, _i64),
                                   _p(rng, _i64), H, W, cfg.tile, cfg.alpha_max, cfg.alpha_min,
                                   cfg.t_min, _p(bg, _f), _p(dimg, _f), n, _p(g, _d),
                                   None if tie is None else _p(tie, _u8), nthreads or threads())
    if rc != 0:
        raise ValueError("tile size above 32")
    return (g, tie.astype(bool)) if ties else g
