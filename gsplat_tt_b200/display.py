"""Display-path stages on the GPU: torch front end of the libgs200 C ABI.

Function names, argument names and defaults follow the reference's pybind module
``_gsplat_cpu`` (backends/cpu_cpp/pybind_module.cpp:1880-2091): compute_cov3d,
project_full_with_cov3d, tile_assign, sort, blend, render_full. Inputs may be numpy
arrays or torch tensors on any device; they are moved to the current CUDA device.
Outputs are CUDA torch tensors (render_full returns a numpy image like the reference).
Shape errors raise ValueError, as the reference's std::invalid_argument does.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from . import _lib
from ._lib import check, lib

__all__ = ["compute_cov3d", "project_full_with_cov3d", "tile_assign", "sort", "sort_pairs",
           "blend", "render_full"]


def _dev():
    if not torch.cuda.is_available():
        raise RuntimeError("gsplat_tt_b200 needs a CUDA device (sm_100a); none is available")
    return torch.device("cuda", torch.cuda.current_device())


def _t(x, dtype, name, shape_tail=None):
    """Contiguous CUDA tensor of `dtype` (None passes through)."""
    if x is None:
        return None
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(np.ascontiguousarray(x))
    if not isinstance(x, torch.Tensor):
        x = torch.as_tensor(x)
    x = x.detach().to(device=_dev(), dtype=dtype).contiguous()
    if shape_tail is not None:
        if x.dim() < 1 or tuple(x.shape[1:]) != tuple(shape_tail):
            raise ValueError(f"{name} must have shape (N, {', '.join(map(str, shape_tail))}), "
                             f"got {tuple(x.shape)}")
    return x


def _host_mat(x, n):
    a = x.detach().cpu().numpy() if isinstance(x, torch.Tensor) else np.asarray(x)
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    if a.size != n:
        raise ValueError(f"expected {n} matrix entries, got {a.size}")
    return a


def _p(t):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _workspace(nbytes: int) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=_dev())


def compute_cov3d(scales, rotations) -> torch.Tensor:
    """(N,3,3) world covariances R S^2 R^T (project.cpp:190-202)."""
    s = _t(scales, torch.float32, "scales", (3,))
    q = _t(rotations, torch.float32, "rotations", (4,))
    if s.shape[0] != q.shape[0]:
        raise ValueError("scales and rotations must share N")
    out = torch.empty((s.shape[0], 3, 3), dtype=torch.float32, device=_dev())
    check(lib.gs_compute_cov3d(_p(s), _p(q), s.shape[0], _p(out), _stream()))
    return out


def project_full_with_cov3d(means, cov3d, extrinsics, intrinsics, image_height, image_width,
                            opacities=None, min_opacity=1.0 / 255.0, colors=None,
                            max_radius=0, contrib_floor=1.0 / 16384.0, k_cap=3.0,
                            use_isoellipse=False):
    """(means_2d (M,2), covs_2d (M,2,2), depths (M,), radii (M,2), valid_mask (N,) bool);
    with ``colors`` also (colors (M,3), opacities (M,)) gathered in the same pass
    (project_full_fused, project.cpp:484-798)."""
    m = _t(means, torch.float32, "means", (3,))
    n = m.shape[0]
    c3 = _t(cov3d, torch.float32, "cov3d").reshape(n, 9)
    op = _t(opacities, torch.float32, "opacities")
    if op is not None and op.numel() != n:
        raise ValueError("opacities must have shape (N,)")
    col = _t(colors, torch.float32, "colors", (3,)) if colors is not None else None
    e = _host_mat(extrinsics, 16)
    K = _host_mat(intrinsics, 9)
    d = _dev()
    m2 = torch.empty((n, 2), dtype=torch.float32, device=d)
    cv = torch.empty((n, 4), dtype=torch.float32, device=d)
    dp = torch.empty(n, dtype=torch.float32, device=d)
    r = torch.empty((n, 2), dtype=torch.float32, device=d)
    v = torch.empty(n, dtype=torch.uint8, device=d)
    co = torch.empty((n, 3), dtype=torch.float32, device=d) if col is not None else None
    oo = torch.empty(n, dtype=torch.float32, device=d) if (col is not None and op is not None) else None
    nv = torch.empty(1, dtype=torch.int64, device=d)
    ws = _workspace(lib.gs_project_workspace_size(n))
    host_m = _lib.i64(0)
    check(lib.gs_project(_p(m), _p(c3), e.ctypes.data, K.ctypes.data, _p(col), _p(op),
                         float(min_opacity), n, int(image_height), int(image_width),
                         int(max_radius), float(contrib_floor), float(k_cap),
                         int(bool(use_isoellipse)), _p(m2), _p(cv), _p(dp), _p(r), _p(v),
                         _p(co), _p(oo), _p(nv), _lib.ctypes.addressof(host_m), _p(ws),
                         ws.numel(), _stream()))
    M = host_m.value
    out = (m2[:M], cv[:M].reshape(M, 2, 2), dp[:M], r[:M], v.bool())
    if col is not None:
        out = out + (co[:M], oo[:M] if oo is not None else None)
    return out


def tile_assign(means_2d, radii, image_height, image_width, tile_size, covs_2d=None,
                opacities=None, contrib_floor=15.0 / 255.0, capacity: int | None = None):
    """(gaussian_ids (P,), tile_ids (P,), tiles_per_gaussian (M,)) int64
    (tile_assign.cpp:26-368). The pair buffers start at ``capacity`` (default 8 M) and
    grow on GS_ERR_OVERFLOW, as the reference's overflow-retry ladder does."""
    m2 = _t(means_2d, torch.float32, "means_2d", (2,))
    M = m2.shape[0]
    r = _t(radii, torch.float32, "radii").reshape(-1, 2)
    if r.shape[0] != M:
        raise ValueError("radii must have shape (M, 2)")
    cv = None
    if covs_2d is not None:
        cv = _t(covs_2d, torch.float32, "covs_2d")
        if cv.numel() != 4 * M:
            raise ValueError("covs_2d must have shape (M, 2, 2) or (M, 4)")
        cv = cv.reshape(M, 4)
    op = _t(opacities, torch.float32, "opacities")
    if (cv is None) != (op is None):
        cv, op = None, None  # the reference culls only when both are given
    d = _dev()
    cap = int(capacity) if capacity else max(1 << 23, 8 * M)
    while True:
        gids = torch.empty(max(cap, 1), dtype=torch.int64, device=d)
        tids = torch.empty(max(cap, 1), dtype=torch.int64, device=d)
        tpg = torch.empty(max(M, 1), dtype=torch.int64, device=d)
        npd = torch.empty(1, dtype=torch.int64, device=d)
        ws = _workspace(lib.gs_tile_assign_workspace_size(M, cap))
        host_p = _lib.i64(0)
        code = lib.gs_tile_assign(_p(m2), _p(r), M, int(image_height), int(image_width),
                                  int(tile_size), _p(cv), _p(op), float(contrib_floor),
                                  _p(gids), _p(tids), cap, _p(tpg), _p(npd),
                                  _lib.ctypes.addressof(host_p), _p(ws), ws.numel(), _stream())
        if code == _lib.GS_ERR_OVERFLOW:
            cap = int(host_p.value) + 1
            continue
        check(code)
        P = host_p.value
        return gids[:P], tids[:P], tpg[:M]


def sort(gaussian_ids, tile_ids, depths, tiles_x, tiles_y):
    """(sorted_gaussian_ids (P,) int64, tile_ranges (tiles, 2) int64), stable by
    (tile, depth bits) (sort.cpp:89-263)."""
    g = _t(gaussian_ids, torch.int64, "gaussian_ids").reshape(-1)
    t = _t(tile_ids, torch.int64, "tile_ids").reshape(-1)
    dp = _t(depths, torch.float32, "depths").reshape(-1)
    if g.shape[0] != t.shape[0]:
        raise ValueError("gaussian_ids and tile_ids must be 1-D arrays of equal length")
    P = g.shape[0]
    d = _dev()
    out = torch.empty(max(P, 1), dtype=torch.int64, device=d)
    rng = torch.empty((tiles_x * tiles_y, 2), dtype=torch.int64, device=d)
    ws = _workspace(lib.gs_sort_and_bin_workspace_size(P, tiles_x, tiles_y))
    check(lib.gs_sort_and_bin(_p(g), _p(t), _p(dp), P, int(tiles_x), int(tiles_y), _p(out),
                              _p(rng), _p(ws), ws.numel(), _stream()))
    if P:
        check(lib.gs_workspace_error(_p(ws), _stream()))
    return out[:P], rng


def sort_pairs(keys, values, key_bits: int = 64, return_keys: bool = False, workspace=None):
    """Stable sort of (uint64 key, uint32 value) pairs on the low ``key_bits`` bits.
    Keys/values are int64/int32 tensors holding the bit patterns. Returns sorted values
    (and keys)."""
    k = _t(keys, torch.int64, "keys").reshape(-1)
    v = _t(values, torch.int32, "values").reshape(-1)
    n = k.shape[0]
    d = _dev()
    vo = torch.empty(max(n, 1), dtype=torch.int32, device=d)
    ko = torch.empty(max(n, 1), dtype=torch.int64, device=d) if return_keys else None
    ws = workspace if workspace is not None else _workspace(
        lib.gs_sort_pairs_workspace_size(n, key_bits))
    check(lib.gs_sort_pairs(_p(k), _p(v), n, int(key_bits), _p(ko), _p(vo), _p(ws), ws.numel(),
                            _stream()))
    if n:
        check(lib.gs_workspace_error(_p(ws), _stream()))
    return (vo[:n], ko[:n]) if return_keys else vo[:n]


def blend(means_2d, covs_2d, colors, opacities, sorted_gaussian_ids, tile_ranges,
          image_height, image_width, tile_size=32, return_alpha=False):
    """(H,W,3) fp32 CUDA image with the display rules (blend.cpp:14-156); with
    return_alpha also (H,W) alpha = 1 - final T."""
    m2 = _t(means_2d, torch.float32, "means_2d", (2,))
    M = m2.shape[0]
    cv = _t(covs_2d, torch.float32, "covs_2d")
    if cv.numel() != 4 * M:
        raise ValueError("covs_2d must have shape (M, 4)")
    col = _t(colors, torch.float32, "colors", (3,))
    op = _t(opacities, torch.float32, "opacities").reshape(-1)
    if col.shape[0] != M or op.shape[0] != M:
        raise ValueError("means_2d, covs_2d, colors, opacities must share M")
    sg = _t(sorted_gaussian_ids, torch.int64, "sorted_gaussian_ids").reshape(-1)
    rng = _t(tile_ranges, torch.int64, "tile_ranges")
    if rng.dim() != 2 or rng.shape[1] != 2:
        raise ValueError("tile_ranges must have shape (num_tiles, 2)")
    tiles_x = (image_width + tile_size - 1) // tile_size
    tiles_y = (image_height + tile_size - 1) // tile_size
    if rng.shape[0] != tiles_x * tiles_y:
        raise ValueError("tile_ranges must have one row per tile")
    d = _dev()
    img = torch.empty((image_height, image_width, 3), dtype=torch.float32, device=d)
    alpha = torch.empty((image_height, image_width), dtype=torch.float32, device=d) if return_alpha else None
    check(lib.gs_blend(_p(m2), _p(cv), _p(col), _p(op), _p(sg), _p(rng), M, int(image_height),
                       int(image_width), int(tile_size), _p(img), _p(alpha), _stream()))
    return (img, alpha) if return_alpha else img


def cull_and_blend(means_2d, covs_2d, colors, opacities, sorted_gaussian_ids, tile_ranges,
                   tiles_x, tiles_y, tile_size, image_height, image_width,
                   mb_contrib_floor=1.0 / 16384.0, cull_disabled=False,
                   transmittance_threshold=1.0 / 255.0):
    """Microblock cull + blend, the reference's default CPU display blend
    (cull_and_blend.cpp:316-840; pybind cull_and_blend, pybind_module.cpp:764-820).
    Returns ((H,W,3) fp32 CUDA image, stats dict with pairs_in, pairs_dropped,
    pairs_kept_per_mb). cull_disabled / transmittance_threshold are the render_full
    parameters the pybind entry fixes at False / 1/255."""
    m2 = _t(means_2d, torch.float32, "means_2d", (2,))
    M = m2.shape[0]
    cv = _t(covs_2d, torch.float32, "covs_2d")
    if cv.numel() != 4 * M:
        raise ValueError("covs_2d must have shape (M, 4)")
    col = _t(colors, torch.float32, "colors", (3,))
    op = _t(opacities, torch.float32, "opacities").reshape(-1)
    if col.shape[0] != M or op.shape[0] != M:
        raise ValueError("means_2d, covs_2d, colors, opacities must share M")
    sg = _t(sorted_gaussian_ids, torch.int64, "sorted_gaussian_ids").reshape(-1)
    rng = _t(tile_ranges, torch.int64, "tile_ranges")
    if rng.dim() != 2 or rng.shape[1] != 2 or rng.shape[0] != tiles_x * tiles_y:
        raise ValueError("tile_ranges must have shape (tiles_x * tiles_y, 2)")
    d = _dev()
    img = torch.empty((image_height, image_width, 3), dtype=torch.float32, device=d)
    st = torch.empty(3, dtype=torch.int64, device=d)
    ws = _workspace(lib.gs_cull_and_blend_workspace_size(M))
    check(lib.gs_cull_and_blend(_p(m2), _p(cv), _p(col), _p(op), _p(sg), _p(rng), M, sg.shape[0],
                                int(tiles_x), int(tiles_y), int(tile_size), int(image_height),
                                int(image_width), float(mb_contrib_floor), int(bool(cull_disabled)),
                                float(transmittance_threshold), _p(img), _p(st), _p(ws), ws.numel(),
                                _stream()))
    s = st.cpu().tolist()
    return img, {"pairs_in": s[0], "pairs_dropped": s[1], "pairs_kept_per_mb": s[2]}


def render_full(means, cov3d, opacities, colors, extrinsics, intrinsics, image_height,
                image_width, tile_size=32, min_opacity=1.0 / 255.0, contrib_floor=1.0 / 16384.0,
                mb_contrib_floor=1.0 / 16384.0, cull_disabled=False,
                transmittance_threshold=1.0 / 255.0, max_radius=0, k_cap=3.0,
                use_isoellipse=False, blend_mode=0, return_alpha=False):
    """One call for project -> tile_assign -> sort -> microblock cull + blend (pybind
    render_full, pybind_module.cpp:1149-1575, CPU path: cull_and_blend). Returns (image
    (H,W,3) float32 numpy, stats dict with the reference's keys). blend_mode selects
    Tenstorrent device blends in the reference and is ignored. With return_alpha the
    plain per-tile blend (blend.cpp) also runs to give stats["alpha"] = 1 - final T,
    which the reference's render_full does not output."""
    del blend_mode
    t0 = time.perf_counter()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    ev[0].record()
    m2, cv, dp, r, v, col, op = project_full_with_cov3d(
        means, cov3d, extrinsics, intrinsics, image_height, image_width, opacities,
        min_opacity, colors=colors, max_radius=max_radius, contrib_floor=contrib_floor,
        k_cap=k_cap, use_isoellipse=use_isoellipse)
    ev[1].record()
    gids, tids, _ = tile_assign(m2, r, image_height, image_width, tile_size,
                                None if cull_disabled else cv,
                                None if cull_disabled else op, contrib_floor)
    ev[2].record()
    tiles_x = (image_width + tile_size - 1) // tile_size
    tiles_y = (image_height + tile_size - 1) // tile_size
    sg, rng = sort(gids, tids, dp, tiles_x, tiles_y)
    ev[3].record()
    img, cb = cull_and_blend(m2, cv.reshape(-1, 4), col, op, sg, rng, tiles_x, tiles_y, tile_size,
                             image_height, image_width, mb_contrib_floor, cull_disabled,
                             transmittance_threshold)
    ev[4].record()
    alpha = None
    if return_alpha:
        _, alpha = blend(m2, cv.reshape(-1, 4), col, op, sg, rng, image_height, image_width,
                         tile_size, return_alpha=True)
    img_np = img.cpu().numpy()
    stats = {
        "num_visible": int(m2.shape[0]),
        "num_entries": int(sg.shape[0]),
        "pairs_in": cb["pairs_in"],
        "pairs_dropped": cb["pairs_dropped"],
        "pairs_kept_per_mb": cb["pairs_kept_per_mb"],
        "project_ms": ev[0].elapsed_time(ev[1]),
        "tile_assign_ms": ev[1].elapsed_time(ev[2]),
        "sort_ms": ev[2].elapsed_time(ev[3]),
        "cull_ms": 0.0,
        "blend_ms": ev[3].elapsed_time(ev[4]),
        "total_ms": (time.perf_counter() - t0) * 1000.0,
    }
    if return_alpha:
        stats["alpha"] = alpha.cpu().numpy()
    return img_np, stats
