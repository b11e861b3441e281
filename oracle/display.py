"""ctypes front end of the C display-path oracle (oracle/gs_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker the CUDA path is compared against. Function
names and argument meanings follow the reference's pybind module
(backends/cpu_cpp/pybind_module.cpp: compute_cov3d 1895, project_full_with_cov3d 1901,
tile_assign 2008, sort 2020, blend 2029), returning numpy arrays.
"""
from __future__ import annotations

import ctypes
import glob
import importlib
import os
import subprocess
import sys

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_f = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.POINTER(ctypes.c_int64)
_u8 = ctypes.POINTER(ctypes.c_uint8)
_u32 = ctypes.POINTER(ctypes.c_uint32)
_u64 = ctypes.POINTER(ctypes.c_uint64)


def build(ref: bool = False, ref_root: str | None = None) -> None:
    """Compile liboracle.so (and, with ref=True, oracle/_ref from the reference sources at
    ref_root, default $GSPLAT_TT_REFERENCE)."""
    targets = ["oracle"] + (["ref"] if ref else [])
    extra = [f"REF={ref_root}"] if ref_root else []
    subprocess.check_call(["make", "-s", "-C", _HERE, *targets,
                           f"PY={sys.executable}", *extra])


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        L.gso_compute_cov3d.argtypes = [_f, _f, ctypes.c_int64, _f]
        L.gso_project.argtypes = [_f, _f, _f, _f, _f, _f, ctypes.c_float, ctypes.c_int64,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                  ctypes.c_float, _f, _f, _f, _f, _u8, _f, _f]
        L.gso_project.restype = ctypes.c_int64
        L.gso_tile_assign.argtypes = [_f, _f, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, _f, _f, ctypes.c_float, _i64, _i64, _i64]
        L.gso_tile_assign.restype = ctypes.c_int64
        L.gso_sort_and_bin.argtypes = [_i64, _i64, _f, ctypes.c_int64, ctypes.c_int,
                                       ctypes.c_int, _i64, _i64]
        L.gso_sort_pairs.argtypes = [_u64, _u32, ctypes.c_int64, _u64, _u32]
        L.gso_logf_array.argtypes = [_f, _f, ctypes.c_int64]
        L.gso_blend.argtypes = [_f, _f, _f, _f, _i64, _i64, ctypes.c_int64, ctypes.c_int,
                                ctypes.c_int, ctypes.c_int, _f, _f]
        L.gso_cull_and_blend.argtypes = [_f, _f, _f, _f, _i64, _i64, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_float, ctypes.c_int, ctypes.c_float, _f, _i64]
        _LIB = L
    return _LIB


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


def _c(a, dt):
    return None if a is None else np.ascontiguousarray(a, dtype=dt)


def compute_cov3d(scales, rotations):
    s, q = _c(scales, np.float32), _c(rotations, np.float32)
    out = np.empty((s.shape[0], 3, 3), np.float32)
    lib().gso_compute_cov3d(_p(s, _f), _p(q, _f), s.shape[0], _p(out, _f))
    return out


def project_full_with_cov3d(means, cov3d, extrinsics, intrinsics, image_height, image_width,
                            opacities=None, min_opacity=1.0 / 255.0, colors=None,
                            max_radius=0, contrib_floor=1.0 / 16384.0, k_cap=3.0):
    """(means_2d (M,2), covs_2d (M,2,2), depths (M,), radii (M,2), valid_mask (N,) bool);
    with colors given, also the gathered colours (M,3) and opacities (M,)."""
    m = _c(means, np.float32)
    n = m.shape[0]
    c3 = _c(cov3d, np.float32).reshape(n, 9)
    e, k = _c(extrinsics, np.float32), _c(intrinsics, np.float32)
    op, col = _c(opacities, np.float32), _c(colors, np.float32)
    m2 = np.empty((n, 2), np.float32)
    cv = np.empty((n, 4), np.float32)
    d = np.empty(n, np.float32)
    r = np.empty((n, 2), np.float32)
    v = np.empty(n, np.uint8)
    co = np.empty((n, 3), np.float32)
    oo = np.empty(n, np.float32)
    M = lib().gso_project(_p(m, _f), _p(c3, _f), _p(e, _f), _p(k, _f), _p(col, _f), _p(op, _f),
                          float(min_opacity), n, int(image_height), int(image_width),
                          int(max_radius), float(contrib_floor), float(k_cap), _p(m2, _f),
                          _p(cv, _f), _p(d, _f), _p(r, _f), _p(v, _u8), _p(co, _f), _p(oo, _f))
    out = (m2[:M].copy(), cv[:M].reshape(M, 2, 2).copy(), d[:M].copy(), r[:M].copy(),
           v.astype(bool))
    if colors is not None:
        out = out + (co[:M].copy(), oo[:M].copy() if opacities is not None else None)
    return out


def tile_assign(means_2d, radii, image_height, image_width, tile_size, covs_2d=None,
                opacities=None, contrib_floor=15.0 / 255.0):
    m2, r = _c(means_2d, np.float32), _c(radii, np.float32).reshape(-1, 2)
    M = m2.shape[0]
    cv = None if covs_2d is None else _c(covs_2d, np.float32).reshape(M, 4)
    op = _c(opacities, np.float32)
    L = lib()
    bound = L.gso_tile_assign(_p(m2, _f), _p(r, _f), M, int(image_height), int(image_width),
                              int(tile_size), None, None, 0.0, None, None, None)
    gids = np.empty(max(bound, 1), np.int64)
    tids = np.empty(max(bound, 1), np.int64)
    tpg = np.empty(max(M, 1), np.int64)
    P = L.gso_tile_assign(_p(m2, _f), _p(r, _f), M, int(image_height), int(image_width),
                          int(tile_size), _p(cv, _f), _p(op, _f), float(contrib_floor),
                          _p(gids, _i64), _p(tids, _i64), _p(tpg, _i64))
    return gids[:P].copy(), tids[:P].copy(), tpg[:M].copy()


def sort(gaussian_ids, tile_ids, depths, tiles_x, tiles_y):
    g, t, d = _c(gaussian_ids, np.int64), _c(tile_ids, np.int64), _c(depths, np.float32)
    P = g.shape[0]
    sg = np.empty(max(P, 1), np.int64)
    rng = np.empty((tiles_x * tiles_y, 2), np.int64)
    lib().gso_sort_and_bin(_p(g, _i64), _p(t, _i64), _p(d, _f), P, int(tiles_x), int(tiles_y),
                           _p(sg, _i64), _p(rng, _i64))
    return sg[:P].copy(), rng


def sort_pairs(keys, values):
    k, v = _c(keys, np.uint64), _c(values, np.uint32)
    ko, vo = np.empty_like(k), np.empty_like(v)
    lib().gso_sort_pairs(_p(k, _u64), _p(v, _u32), k.shape[0], _p(ko, _u64), _p(vo, _u32))
    return ko, vo


def blend(means_2d, covs_2d, colors, opacities, sorted_gaussian_ids, tile_ranges,
          image_height, image_width, tile_size=32, return_alpha=False):
    m2 = _c(means_2d, np.float32)
    M = m2.shape[0]
    cv = _c(covs_2d, np.float32).reshape(M, 4)
    col, op = _c(colors, np.float32), _c(opacities, np.float32)
    sg, rng = _c(sorted_gaussian_ids, np.int64), _c(tile_ranges, np.int64)
    img = np.empty((image_height, image_width, 3), np.float32)
    alpha = np.empty((image_height, image_width), np.float32)
    lib().gso_blend(_p(m2, _f), _p(cv, _f), _p(col, _f), _p(op, _f), _p(sg, _i64),
                    _p(rng, _i64), M, int(image_height), int(image_width), int(tile_size),
                    _p(img, _f), _p(alpha, _f))
    return (img, alpha) if return_alpha else img


def cull_and_blend(means_2d, covs_2d, colors, opacities, sorted_gaussian_ids, tile_ranges,
                   tiles_x, tiles_y, tile_size, image_height, image_width,
                   mb_contrib_floor=1.0 / 16384.0, cull_disabled=False,
                   transmittance_threshold=1.0 / 255.0):
    """Microblock cull + blend (cull_and_blend.cpp, scalar build) -> (image, stats)."""
    m2 = _c(means_2d, np.float32)
    M = m2.shape[0]
    cv = _c(covs_2d, np.float32).reshape(M, 4)
    col, op = _c(colors, np.float32), _c(opacities, np.float32)
    sg, rng = _c(sorted_gaussian_ids, np.int64), _c(tile_ranges, np.int64)
    img = np.zeros((image_height, image_width, 3), np.float32)
    st = np.zeros(3, np.int64)
    lib().gso_cull_and_blend(_p(m2, _f), _p(cv, _f), _p(col, _f), _p(op, _f), _p(sg, _i64),
                             _p(rng, _i64), M, sg.shape[0], int(tiles_x), int(tiles_y),
                             int(tile_size), int(image_height), int(image_width),
                             float(mb_contrib_floor), int(bool(cull_disabled)),
                             float(transmittance_threshold), _p(img, _f), _p(st, _i64))
    return img, {"pairs_in": int(st[0]), "pairs_dropped": int(st[1]),
                 "pairs_kept_per_mb": int(st[2])}


def logf_array(x):
    """Host C library logf of a float32 array."""
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().gso_logf_array(_p(x, _f), _p(y, _f), x.shape[0])
    return y


def reference_module():
    """The reference's own ``_gsplat_cpu`` pybind module built into oracle/_ref, or None."""
    ref_dir = os.path.join(_HERE, "_ref")
    if not glob.glob(os.path.join(ref_dir, "_gsplat_cpu*.so")):
        return None
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    return importlib.import_module("_gsplat_cpu")
