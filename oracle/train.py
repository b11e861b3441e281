"""numpy restatement of the reference's training-path models (TEST INFRASTRUCTURE ONLY).

The checker the CUDA training kernels are compared against; the product never imports
it. Each function cites the reference function it restates (paths relative to the
reference project root):

* project        -- gsplat/t2_param_backward.py:81-120 forward_lanes (fp32 lanes) plus
                    SH colour (gsplat/train_oracle.py:99-122, 163-173) and the tile
                    rectangles of gsplat/blend_backward_dev.py:76-92 (float64 from the conic).
* pair_lists     -- gsplat/blend_backward_dev.py:95-112 (per tile, front to back).
* forward        -- gsplat/blend_backward_dev.py:404-438 forward_fast: tiled fp32 forward,
                    tile-centred power (gsplat/blend_backward_ref.py:68-92), alpha clamp,
                    alpha_min skip, t_min stop; generalised to any tile size.
* loss_l1 / loss_ssim -- gsplat/train_loss.py:166-171 and :126-165 (fp32 scheme).
* backward_2d    -- gsplat/blend_backward_dev.py:444-517 ref_slots_fast summed per
                    Gaussian (gsplat/t2_param_backward.py:50-61).
* param_backward -- gsplat/t2_param_backward.py:123-192 projection_backward_sh0, extended
                    with SH bands 1-3 and the view-direction term into the means (the
                    derivative of gsplat/train_oracle.py:99-122 sh_eval, which the
                    reference covers only through fp64 autograd).
* sparse_adam    -- gsplat/train_oracle.py:434-470 sparse_adam_step (fp32 or bf16 moments).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

f32 = np.float32
SH_C0 = 0.28209479177387814
SH_C1 = 0.4886025119029199
SH_C2 = (1.0925484305920792, -1.0925484305920792, 0.31539156525252005,
         -1.0925484305920792, 0.5462742152960396)
SH_C3 = (-0.5900435899266435, 2.890611442640554, -0.4570457994644658,
         0.3731763325901154, -0.4570457994644658, 1.445305721320277,
         -0.5900435899266435)
PARAM_NAMES = ("means", "log_scales", "quats", "opacity_logits", "sh")
TIE_RTOL = 4e-6  # gsplat/blend_backward_dev.py:441 (about 32 fp32 ulp)
DEFAULT_LR = {"means": 1.6e-4, "log_scales": 5e-3, "quats": 1e-3, "opacity_logits": 0.05,
              "sh_dc": 2.5e-3, "sh_rest": 2.5e-3 / 20.0}


@dataclass
class Cfg:
    """gsplat/train_oracle.py:64-71 RenderConfig, plus the tile size."""
    sh_degree: int = 0
    near: float = 0.2
    lowpass: float = 0.3
    alpha_max: float = 0.99
    alpha_min: float = 1.0 / 255.0
    t_min: float = 1e-4
    background: tuple = (0.0, 0.0, 0.0)
    tile: int = 16


def _cam(w2c, K, ft=f32):
    w = np.asarray(w2c, np.float64)
    k = np.asarray(K, np.float64)
    R = w[:3, :3].astype(ft)
    t = w[:3, 3].astype(ft)
    cc = (-(w[:3, :3].T @ w[:3, 3])).astype(ft)   # camera centre, float64 then rounded
    return R, t, ft(k[0, 0]), ft(k[1, 1]), ft(k[0, 2]), ft(k[1, 2]), cc


def _quat_rot(w, x, y, z):
    two, one = f32(2), f32(1)
    return [one - two * (y * y + z * z), two * (x * y - w * z), two * (x * z + w * y),
            two * (x * y + w * z), one - two * (x * x + z * z), two * (y * z - w * x),
            two * (x * z - w * y), two * (y * z + w * x), one - two * (x * x + y * y)]


def sh_basis(dirs, degree):
    """(N, K) real SH basis of gsplat/train_oracle.py:99-122 (coefficients per band)."""
    x, y, z = dirs[:, 0], dirs[:, 1], dirs[:, 2]
    dt = dirs.dtype.type
    cols = [np.full_like(x, dt(SH_C0))]
    if degree >= 1:
        cols += [dt(-SH_C1) * y, dt(SH_C1) * z, dt(-SH_C1) * x]
    if degree >= 2:
        xx, yy, zz = x * x, y * y, z * z
        cols += [dt(SH_C2[0]) * (x * y), dt(SH_C2[1]) * (y * z),
                 dt(SH_C2[2]) * (dt(2) * zz - xx - yy), dt(SH_C2[3]) * (x * z),
                 dt(SH_C2[4]) * (xx - yy)]
    if degree >= 3:
        cols += [dt(SH_C3[0]) * y * (dt(3) * xx - yy), dt(SH_C3[1]) * (x * y) * z,
                 dt(SH_C3[2]) * y * (dt(4) * zz - xx - yy),
                 dt(SH_C3[3]) * z * (dt(2) * zz - dt(3) * xx - dt(3) * yy),
                 dt(SH_C3[4]) * x * (dt(4) * zz - xx - yy), dt(SH_C3[5]) * z * (xx - yy),
                 dt(SH_C3[6]) * x * (xx - dt(3) * yy)]
    return np.stack(cols, 1)


def sh_basis_grad(dirs, degree):
    """(N, K, 3) derivative of each basis function with respect to (x, y, z)."""
    x, y, z = dirs[:, 0], dirs[:, 1], dirs[:, 2]
    dt = dirs.dtype.type
    zero = np.zeros_like(x)
    g = [(zero, zero, zero)]
    if degree >= 1:
        c1 = dt(SH_C1)
        g += [(zero, -c1 + zero, zero), (zero, zero, c1 + zero), (-c1 + zero, zero, zero)]
    if degree >= 2:
        c = [dt(v) for v in SH_C2]
        g += [(c[0] * y, c[0] * x, zero), (zero, c[1] * z, c[1] * y),
              (c[2] * dt(-2) * x, c[2] * dt(-2) * y, c[2] * dt(4) * z),
              (c[3] * z, zero, c[3] * x), (c[4] * dt(2) * x, c[4] * dt(-2) * y, zero)]
    if degree >= 3:
        c = [dt(v) for v in SH_C3]
        xx, yy, zz = x * x, y * y, z * z
        g += [(c[0] * dt(6) * x * y, c[0] * (dt(3) * xx - dt(3) * yy), zero),
              (c[1] * y * z, c[1] * x * z, c[1] * x * y),
              (c[2] * dt(-2) * x * y, c[2] * (dt(4) * zz - xx - dt(3) * yy), c[2] * dt(8) * y * z),
              (c[3] * dt(-6) * x * z, c[3] * dt(-6) * y * z, c[3] * (dt(6) * zz - dt(3) * xx - dt(3) * yy)),
              (c[4] * (dt(4) * zz - dt(3) * xx - yy), c[4] * dt(-2) * x * y, c[4] * dt(8) * x * z),
              (c[5] * dt(2) * x * z, c[5] * dt(-2) * y * z, c[5] * (xx - yy)),
              (c[6] * (dt(3) * xx - dt(3) * yy), c[6] * dt(-6) * x * y, zero)]
    return np.stack([np.stack(v, 1) for v in g], 1)


def _exp(x, ft):
    """exp rounded once to `ft` (computed in float64): the correctly rounded value, in place
    of numpy's float32 exp (whose last bit is implementation-defined), for the projection's
    scales and opacities (which the device reproduces) and the rasteriser's Gaussian
    weights (which the device evaluates with its own exp, covered by the tolerances)."""
    return np.exp(np.asarray(x, np.float64)).astype(ft)


def project(params, w2c, K, H, W, cfg: Cfg, ft=f32) -> dict:
    """Per-Gaussian projection for one view (fp32 lanes). Every sum is written out in
    order so the device kernel (compiled without FMA contraction) rounds identically."""
    R, t, fx, fy, cx, cy, cc = _cam(w2c, K, ft)
    m = np.asarray(params["means"], ft)
    x, y, z = (R[i, 0] * m[:, 0] + R[i, 1] * m[:, 1] + R[i, 2] * m[:, 2] + t[i] for i in range(3))
    valid = z > ft(cfg.near)
    iz = ft(1) / np.where(valid, z, ft(1))
    mx, my = fx * x * iz + cx, fy * y * iz + cy
    q = np.asarray(params["quats"], ft)
    qinv = ft(1) / np.sqrt(q[:, 0] * q[:, 0] + q[:, 1] * q[:, 1] + q[:, 2] * q[:, 2]
                           + q[:, 3] * q[:, 3])
    qn = [q[:, i] * qinv for i in range(4)]
    Rq = _quat_rot(*qn)
    s = _exp(params["log_scales"], ft)
    M = [Rq[3 * i + j] * s[:, j] for i in range(3) for j in range(3)]
    S = {(i, k): M[3 * i] * M[3 * k] + M[3 * i + 1] * M[3 * k + 1] + M[3 * i + 2] * M[3 * k + 2]
         for i in range(3) for k in range(i, 3)}
    c3 = lambda i, k: S[(min(i, k), max(i, k))]  # noqa: E731
    j00, j02 = fx * iz, -fx * x * iz * iz
    j11, j12 = fy * iz, -fy * y * iz * iz
    T0 = [j00 * R[0, k] + j02 * R[2, k] for k in range(3)]
    T1 = [j11 * R[1, k] + j12 * R[2, k] for k in range(3)]
    CT0 = [c3(i, 0) * T0[0] + c3(i, 1) * T0[1] + c3(i, 2) * T0[2] for i in range(3)]
    CT1 = [c3(i, 0) * T1[0] + c3(i, 1) * T1[1] + c3(i, 2) * T1[2] for i in range(3)]
    a = T0[0] * CT0[0] + T0[1] * CT0[1] + T0[2] * CT0[2] + ft(cfg.lowpass)
    b = T1[0] * CT0[0] + T1[1] * CT0[1] + T1[2] * CT0[2]
    c = T1[0] * CT1[0] + T1[1] * CT1[1] + T1[2] * CT1[2] + ft(cfg.lowpass)
    idet = ft(1) / (a * c - b * b)
    A, B, C = c * idet, -b * idet, a * idet
    rx = np.ceil(ft(3) * np.sqrt(np.maximum(a, ft(0))))
    ry = np.ceil(ft(3) * np.sqrt(np.maximum(c, ft(0))))
    visible = valid & (mx + rx > 0) & (mx - rx < W) & (my + ry > 0) & (my - ry < H)
    op = ft(1) / (ft(1) + _exp(-np.asarray(params["opacity_logits"], ft), ft))
    d = m - cc
    dn = np.sqrt(d[:, 0] * d[:, 0] + d[:, 1] * d[:, 1] + d[:, 2] * d[:, 2])
    dirs = d / dn[:, None]
    basis = sh_basis(dirs, cfg.sh_degree)
    sh = np.asarray(params["sh"], ft)[:, :basis.shape[1]]
    raw = basis[:, 0, None] * sh[:, 0]
    for k in range(1, basis.shape[1]):
        raw = raw + basis[:, k, None] * sh[:, k]
    raw = raw + ft(0.5)
    colors = np.maximum(raw, ft(0))
    out = dict(R=R, t=t, fx=fx, fy=fy, x=x, y=y, z=z, iz=iz, valid=valid, visible=visible,
               qn=qn, qinv=qinv, Rq=Rq, s=s, M=M, c3=c3, T0=T0, T1=T1, A=A, B=B, C=C,
               means2d=np.stack([mx, my], 1), conic=np.stack([A, B, C], 1), opacity=op,
               colors=colors, raw=raw, dirs=dirs, dnorm=dn, basis=basis, depth=z)
    out["rects"] = tile_rects(out["means2d"], valid, out["conic"], H, W, cfg.tile)
    return out


def tile_rects(means2d, valid, conic, H, W, tile):
    """(N,4) inclusive tile rectangle [x0, x1, y0, y1] (x1 < x0: none), computed in float64
    from the conic as gsplat/blend_backward_dev.py:76-92 does; a degenerate conic (non-finite
    radius) gets no rectangle."""
    con = np.asarray(conic, np.float64)
    A, B, C = con[:, 0], con[:, 1], con[:, 2]
    with np.errstate(divide="ignore", invalid="ignore"):
        det = A * C - B * B
        ca, cc = C / det, A / det
        rx = np.ceil(3.0 * np.sqrt(np.maximum(ca, 0.0)))
        ry = np.ceil(3.0 * np.sqrt(np.maximum(cc, 0.0)))
        m = np.asarray(means2d, np.float64)
        px, py = m[:, 0], m[:, 1]
        ok = (np.asarray(valid, bool) & ~(px + rx <= 0) & ~(px - rx >= W)
              & ~(py + ry <= 0) & ~(py - ry >= H) & np.isfinite(rx) & np.isfinite(ry))
    tx, ty = (W + tile - 1) // tile, (H + tile - 1) // tile
    out = np.zeros((m.shape[0], 4), np.int64)
    out[:, 1] = -1

    def cl(v, hi):
        return np.clip(np.trunc(v[ok]), 0, hi).astype(np.int64)
    out[ok] = np.stack([cl((px - rx) / tile, tx - 1), cl((px + rx) / tile, tx - 1),
                        cl((py - ry) / tile, ty - 1), cl((py + ry) / tile, ty - 1)], 1)
    return out


def pair_lists(rects, depth, tiles_x):
    """All (tile, Gaussian) pairs sorted by tile, then depth bits, then Gaussian id --
    the order a stable sort of tile << 32 | bits(depth) over Gaussian-major pairs gives."""
    x0, x1, y0, y1 = (rects[:, i] for i in range(4))
    w = x1 - x0 + 1
    counts = np.where(x1 >= x0, w * (y1 - y0 + 1), 0).astype(np.int64)
    g = np.repeat(np.arange(rects.shape[0]), counts)
    j = np.arange(g.size, dtype=np.int64) - np.repeat(np.cumsum(counts) - counts, counts)
    tid = (y0[g] + j // w[g]) * tiles_x + x0[g] + j % w[g]
    dbits = np.asarray(depth, f32).view(np.uint32)[g].astype(np.uint64)
    key = (tid.astype(np.uint64) << np.uint64(32)) | dbits
    o = np.argsort(key, kind="stable")
    return {"g": g[o], "tid": tid[o], "counts": counts}


def _centred(A, B, C, mxl, myl, centre):
    """gsplat/blend_backward_ref.py:68-85 centred_power_coeffs, tile centre `centre`."""
    Af, Bf, Cf = f32(-0.5) * f32(A), -f32(B), f32(-0.5) * f32(C)
    a, b, c = (np.asarray(v, np.float64) for v in (Af, Bf, Cf))
    U0 = centre - np.asarray(mxl, np.float64)
    V0 = centre - np.asarray(myl, np.float64)
    P0 = a * U0 * U0 + b * U0 * V0 + c * V0 * V0
    Lx = 2.0 * a * U0 + b * V0
    Ly = b * U0 + 2.0 * c * V0
    return Af, Bf, Cf, f32(P0), f32(Lx), f32(Ly)


def _sweep(proj, H, W, tile):
    """Per-tile pair streams (tiles ordered by descending pair count) as forward_fast."""
    tx, ty = (W + tile - 1) // tile, (H + tile - 1) // tile
    pl = pair_lists(proj["rects"], proj["depth"], tx)
    utid, start, cnt = np.unique(pl["tid"], return_index=True, return_counts=True)
    s = np.argsort(-cnt, kind="stable")
    utid, start, cnt = utid[s], start[s], cnt[s]
    ox = (utid % tx * tile).astype(f32)[:, None, None]
    oy = (utid // tx * tile).astype(f32)[:, None, None]
    yy, xx = np.meshgrid(np.arange(tile, dtype=f32) + f32(0.5),
                         np.arange(tile, dtype=f32) + f32(0.5), indexing="ij")
    inside = np.zeros((ty * tile, tx * tile), bool)
    inside[:H, :W] = True
    inside = inside.reshape(ty, tile, tx, tile).swapaxes(1, 2).reshape(-1, tile, tile)[utid]
    return pl, utid, start, cnt, ox, oy, xx, yy, tx, ty, inside


def _untile(a, utid, tx, ty, tile, H, W, fill):
    full = np.empty((ty * tx, tile, tile) + a.shape[3:], a.dtype)
    full[...] = fill
    full[utid] = a
    full = full.reshape((ty, tx, tile, tile) + a.shape[3:]).swapaxes(1, 2)
    return full.reshape((ty * tile, tx * tile) + a.shape[3:])[:H, :W]


def forward(proj, H, W, cfg: Cfg) -> dict:
    """Tiled fp32 forward with the training rules; image (H,W,3), final_T (H,W), the
    per-pixel count of processed pairs up to the last blended one (n_contrib), and `ties`
    (H,W): pixels where a decision (alpha >= alpha_min, the alpha clamp, the t_min stop)
    came within TIE_RTOL of its threshold, where either outcome is a valid fp32 result
    (gsplat/blend_backward_dev.py:441-449)."""
    tile = cfg.tile
    m2, con = np.asarray(proj["means2d"], f32), np.asarray(proj["conic"], f32)
    op, col = np.asarray(proj["opacity"], f32), np.asarray(proj["colors"], f32)
    pl, utid, start, cnt, ox, oy, xx, yy, tx, ty, inside = _sweep(proj, H, W, tile)
    nt = utid.size
    centre = f32(tile / 2)
    done = ~inside
    T = np.ones((nt, tile, tile), f32)
    Cc = np.zeros((nt, tile, tile, 3), f32)
    ncon = np.zeros((nt, tile, tile), np.int32)
    amax, amin, tmin, one = f32(cfg.alpha_max), f32(cfg.alpha_min), f32(cfg.t_min), f32(1)
    n_live = 0
    taint = np.zeros((nt, tile, tile), bool)
    near = lambda q, th: np.abs(q / th - 1.0) < TIE_RTOL  # noqa: E731
    for k in range(int(cnt.max()) if nt else 0):
        n = int(np.searchsorted(-cnt, -k, side="left"))
        g = pl["g"][start[:n] + k]
        cf = _centred(*(con[g, i][:, None, None] for i in range(3)),
                      m2[g, 0][:, None, None] - ox[:n], m2[g, 1][:, None, None] - oy[:n], centre)
        Af, Bf, Cf, P0, Lx, Ly = cf
        du, dv = xx - centre, yy - centre
        pw = (P0 + du * (Lx + Af * du + Bf * dv) + dv * (Ly + Cf * dv)).astype(f32)
        raw = op[g][:, None, None] * _exp(np.minimum(pw, f32(0)), f32)
        al = np.minimum(raw, amax).astype(f32)
        Tn = T[:n] * (one - al)
        taint[:n] |= ~done[:n] & (near(al, amin) | near(raw, amax)
                                  | ((al >= amin) & near(Tn, tmin)))
        act = (al >= amin) & ~done[:n]
        live = act & (Tn >= tmin)
        n_live += int(live.sum())
        Cc[:n] += np.where(live, al * T[:n], f32(0))[..., None] * col[g][:, None, None, :]
        T[:n] = np.where(live, Tn, T[:n])
        ncon[:n] = np.where(live, k + 1, ncon[:n])
        done[:n] |= act & ~live
    bg = np.asarray(cfg.background, f32)
    img = _untile(Cc + T[..., None] * bg, utid, tx, ty, tile, H, W, bg)
    return {"image": img, "final_T": _untile(T, utid, tx, ty, tile, H, W, f32(1)),
            "n_contrib": _untile(ncon, utid, tx, ty, tile, H, W, 0),
            "ties": _untile(taint, utid, tx, ty, tile, H, W, False),
            "n_pairs": int(pl["g"].size), "n_live": n_live}


def backward_2d(proj, image, dL_dimage, H, W, cfg: Cfg, ties: bool = False):
    """Per-Gaussian (N, 9) = (dmx, dmy, dA, dB, dC, dopacity, dr, dg, db): the reference's
    front-to-back slot formula, summed per Gaussian. With ties=True also an (N,) bool of
    Gaussians one of whose pixels made a forward decision within 4e-6 relative of its
    threshold (either side is a valid fp32 outcome there)."""
    tile = cfg.tile
    m2, con = np.asarray(proj["means2d"], f32), np.asarray(proj["conic"], f32)
    op, col = np.asarray(proj["opacity"], f32), np.asarray(proj["colors"], f32)
    N = m2.shape[0]
    pl, utid, start, cnt, ox, oy, xx, yy, tx, ty, inside = _sweep(proj, H, W, tile)
    nt = utid.size
    centre = f32(tile / 2)

    def tiles_of(a):
        pad = np.zeros((ty * tile, tx * tile) + a.shape[2:], f32)
        pad[:H, :W] = a
        t = pad.reshape((ty, tile, tx, tile) + a.shape[2:]).swapaxes(1, 2)
        return t.reshape((ty * tx, tile, tile) + a.shape[2:])[utid]
    Gp = tiles_of(np.asarray(dL_dimage, f32))
    Ig = (tiles_of(np.asarray(image, f32)) * Gp).sum(-1, dtype=f32)
    alive = inside.copy()
    T = np.ones((nt, tile, tile), f32)
    s_acc = np.zeros((nt, tile, tile), f32)
    grads = np.zeros((N, 9), np.float64)
    tie_g = np.zeros(N, bool)
    taint = np.zeros((nt, tile, tile), bool)
    amax, amin, tmin, one = f32(cfg.alpha_max), f32(cfg.alpha_min), f32(cfg.t_min), f32(1)
    near = lambda q, th: np.abs(q / th - one) < TIE_RTOL  # noqa: E731
    for k in range(int(cnt.max()) if nt else 0):
        n = int(np.searchsorted(-cnt, -k, side="left"))
        g = pl["g"][start[:n] + k]
        mxl, myl = m2[g, 0][:, None, None] - ox[:n], m2[g, 1][:, None, None] - oy[:n]
        u, v = xx - mxl, yy - myl
        Af, Bf, Cf, P0, Lx, Ly = _centred(*(con[g, i][:, None, None] for i in range(3)),
                                          mxl, myl, centre)
        du, dv = xx - centre, yy - centre
        power = (P0 + du * (Lx + Af * du + Bf * dv) + dv * (Ly + Cf * dv)).astype(f32)
        wgt = _exp(np.minimum(power, f32(0)), f32)
        raw = op[g][:, None, None] * wgt
        clamp = raw > amax
        alpha = np.where(clamp, amax, raw).astype(f32)
        Tk = T[:n]
        live = alive[:n] & (alpha >= amin)
        if ties:
            taint[:n] |= alive[:n] & (near(alpha, amin) | near(raw, amax)
                                      | (live & near(Tk * (one - alpha), tmin)))
            tie_g[g[(taint[:n] & (alpha >= amin * (one - f32(TIE_RTOL)))).any((1, 2))]] = True
        stop = live & (Tk * (one - alpha) < tmin)
        live &= ~stop
        alive[:n] &= ~stop
        at = np.where(live, alpha * Tk, f32(0)).astype(f32)
        Gk = Gp[:n]
        cg = (col[g][:, None, None, :] * Gk).sum(-1, dtype=f32)
        s_acc[:n] = s_acc[:n] + at * cg
        behind = Ig[:n] - s_acc[:n]
        dalpha = Tk * cg - behind / (one - alpha)
        T[:n] = np.where(live, Tk * (one - alpha), Tk).astype(f32)
        act = live & ~clamp & (power <= f32(0))
        G = np.where(act, dalpha * alpha, f32(0)).astype(f32)
        terms = np.stack([np.where(live & ~clamp, dalpha * wgt, f32(0)),
                          at * Gk[..., 0], at * Gk[..., 1], at * Gk[..., 2],
                          G * u * u, G * u * v, G * v * v, G * u, G * v], -1).astype(f32)
        s = terms.reshape(n, -1, 9).sum(1, dtype=np.float64)
        Ac, Bc, Cc_ = (con[g, i].astype(np.float64) for i in range(3))
        Suu, Suv, Svv, Su, Sv = s[:, 4], s[:, 5], s[:, 6], s[:, 7], s[:, 8]
        pair = np.stack([Ac * Su + Bc * Sv, Bc * Su + Cc_ * Sv, -0.5 * Suu, -Suv, -0.5 * Svv,
                         s[:, 0], s[:, 1], s[:, 2], s[:, 3]], 1)
        np.add.at(grads, g, pair)
    out = grads.astype(f32)
    return (out, tie_g) if ties else out


def backward_2d_exact(proj, dL_dimage, H, W, cfg: Cfg, ties: bool = False):
    """The same per-Gaussian 2D gradients as backward_2d, with the forward decisions
    (alphas, clamps, live masks, stops) taken in fp32 exactly as the forward makes them and
    every gradient term evaluated in float64. In exact arithmetic the reference's
    front-to-back formula, dalpha_i = T_i c.g - (I.g - C_acc(<=i).g) / (1 - a_i), equals a
    back-to-front accumulation of the colour behind each pair; evaluated in fp32 the
    former cancels (I.g and C_acc.g are both O(1) while their difference is small behind
    opaque layers) and loses up to a few 1e-3 relative on opaque scenes. This function
    accumulates back to front in float64: the exact gradient of the fp32 forward."""
    tile = cfg.tile
    m2, con = np.asarray(proj["means2d"], f32), np.asarray(proj["conic"], f32)
    op, col = np.asarray(proj["opacity"], f32), np.asarray(proj["colors"], f32)
    N = m2.shape[0]
    pl, utid, start, cnt, ox, oy, xx, yy, tx, ty, inside = _sweep(proj, H, W, tile)
    nt = utid.size
    centre = f32(tile / 2)

    def tiles_of(a):
        pad = np.zeros((ty * tile, tx * tile) + a.shape[2:], f32)
        pad[:H, :W] = a
        t = pad.reshape((ty, tile, tx, tile) + a.shape[2:]).swapaxes(1, 2)
        return t.reshape((ty * tx, tile, tile) + a.shape[2:])[utid]
    Gp = tiles_of(np.asarray(dL_dimage, f32)).astype(np.float64)
    amax, amin, tmin, one = f32(cfg.alpha_max), f32(cfg.alpha_min), f32(cfg.t_min), f32(1)
    near = lambda q, th: np.abs(q / th - 1.0) < TIE_RTOL  # noqa: E731
    alive = inside.copy()
    T = np.ones((nt, tile, tile), f32)
    taint = np.zeros((nt, tile, tile), bool)
    tie_g = np.zeros(N, bool)
    recs = []
    for k in range(int(cnt.max()) if nt else 0):   # fp32 forward: the decisions
        n = int(np.searchsorted(-cnt, -k, side="left"))
        g = pl["g"][start[:n] + k]
        mxl, myl = m2[g, 0][:, None, None] - ox[:n], m2[g, 1][:, None, None] - oy[:n]
        Af, Bf, Cf, P0, Lx, Ly = _centred(*(con[g, i][:, None, None] for i in range(3)),
                                          mxl, myl, centre)
        du, dv = xx - centre, yy - centre
        power = (P0 + du * (Lx + Af * du + Bf * dv) + dv * (Ly + Cf * dv)).astype(f32)
        wgt = _exp(np.minimum(power, f32(0)), f32)
        raw = op[g][:, None, None] * wgt
        clamp = raw > amax
        alpha = np.where(clamp, amax, raw).astype(f32)
        live = alive[:n] & (alpha >= amin)
        if ties:
            taint[:n] |= alive[:n] & (near(alpha, amin) | near(raw, amax)
                                      | (live & near(T[:n] * (one - alpha), tmin)))
            tie_g[g[(taint[:n] & (alpha >= amin * (one - f32(TIE_RTOL)))).any((1, 2))]] = True
        stop = live & (T[:n] * (one - alpha) < tmin)
        live &= ~stop
        alive[:n] &= ~stop
        T[:n] = np.where(live, T[:n] * (one - alpha), T[:n])
        recs.append((n, g, mxl, myl, power, wgt, clamp, alpha, live))
    Tc = T.astype(np.float64)
    behind = Tc * (Gp * np.asarray(cfg.background, f32).astype(np.float64)).sum(-1)
    grads = np.zeros((N, 9), np.float64)
    for (n, g, mxl, myl, power, wgt, clamp, alpha, live) in reversed(recs):
        a, w = alpha.astype(np.float64), wgt.astype(np.float64)
        Gk = Gp[:n]
        cg = (col[g][:, None, None, :].astype(np.float64) * Gk).sum(-1)
        Ti = np.where(live, Tc[:n] / (1.0 - a), Tc[:n])
        dal = Ti * cg - behind[:n] / (1.0 - a)
        at = np.where(live, a * Ti, 0.0)
        behind[:n] += at * cg
        Tc[:n] = Ti
        u = (xx - mxl).astype(np.float64)
        v = (yy - myl).astype(np.float64)
        G = np.where(live & ~clamp & (power <= 0), dal * a, 0.0)
        terms = np.stack([np.where(live & ~clamp, dal * w, 0.0), at * Gk[..., 0], at * Gk[..., 1],
                          at * Gk[..., 2], G * u * u, G * u * v, G * v * v, G * u, G * v], -1)
        s = terms.reshape(n, -1, 9).sum(1)
        Ac, Bc, Cc_ = (con[g, i].astype(np.float64) for i in range(3))
        pair = np.stack([Ac * s[:, 7] + Bc * s[:, 8], Bc * s[:, 7] + Cc_ * s[:, 8], -0.5 * s[:, 4],
                         -s[:, 5], -0.5 * s[:, 6], s[:, 0], s[:, 1], s[:, 2], s[:, 3]], 1)
        np.add.at(grads, g, pair)
    return (grads, tie_g) if ties else grads


# ------------------------------------------------------------------ loss

WIN, SIGMA = 11, 1.5
C1, C2 = 0.01 ** 2, 0.03 ** 2


def _gauss():
    x = np.arange(WIN, dtype=np.float64) - WIN // 2
    g = np.exp(-(x * x) / (2.0 * SIGMA * SIGMA))
    return g / g.sum()


def filt(z):
    """Separable 11-tap Gaussian (sigma 1.5) with zero padding over (H, W, C), float64
    accumulation rounded to fp32 once (3DGS ssim's conv2d, gsplat/train_oracle.py:253-273)."""
    g = _gauss()
    z = np.asarray(z, np.float64)
    H, W = z.shape[:2]
    p = np.pad(z, ((0, 0), (5, 5), (0, 0)))
    r = sum(g[k] * p[:, k:k + W] for k in range(WIN))
    p = np.pad(r, ((5, 5), (0, 0), (0, 0)))
    return sum(g[k] * p[k:k + H] for k in range(WIN)).astype(f32)


def loss_l1(image, target, lambda_dssim=0.2):
    """gsplat/train_loss.py:166-171: (0.8 * L1, its dL/dimage)."""
    n = float(image.size)
    d = np.asarray(image, f32) - np.asarray(target, f32)
    w = f32((1.0 - lambda_dssim) / n)
    return (1.0 - lambda_dssim) * float(np.abs(d).astype(np.float64).sum() / n), w * np.sign(d)


def loss_ssim(image, target, lambda_dssim=0.2):
    """gsplat/train_loss.py:126-165 in fp32: (loss, dL/dimage) of
    (1 - lambda) L1 + lambda (1 - SSIM)."""
    x, y = np.asarray(image, f32), np.asarray(target, f32)
    n = f32(x.size)
    mu_x, mu_y = filt(x), filt(y)
    e_xx, e_yy, e_xy = filt(x * x), filt(y * y), filt(x * y)
    mxy = mu_x * mu_y
    A = f32(2) * mxy + f32(C1)
    B = f32(2) * (e_xy - mxy) + f32(C2)
    C = mu_x * mu_x + mu_y * mu_y + f32(C1)
    D = (e_xx - mu_x * mu_x) + (e_yy - mu_y * mu_y) + f32(C2)
    S = (A * B) / (C * D)
    w = f32(-lambda_dssim) / n
    Sw = S * w
    d_mu = Sw * (f32(2) * mu_y / A - f32(2) * mu_y / B - f32(2) * mu_x / C + f32(2) * mu_x / D)
    d_xx = -Sw / D
    d_xy = f32(2) * Sw / B
    grad = filt(d_mu) + f32(2) * x * filt(d_xx) + y * filt(d_xy)
    diff = x - y
    grad = grad + f32((1.0 - lambda_dssim)) / n * np.sign(diff)
    l1 = float(np.abs(diff).astype(np.float64).sum() / float(n))
    ssim = float(S.astype(np.float64).sum() / float(n))
    return (1.0 - lambda_dssim) * l1 + lambda_dssim * (1.0 - ssim), grad.astype(f32)


# ------------------------------------------------------------------ projection backward

def param_backward(params, g2d, w2c, K, H, W, cfg: Cfg, ft=f32) -> dict:
    """(N,9) 2D grads of one view -> optimizer-space grads (same shapes as params)."""
    F = project(params, w2c, K, H, W, cfg, ft)
    g = np.asarray(g2d, ft)
    gmx, gmy, gA, gB, gC, gop = (g[:, i] for i in range(6))
    A, B, C = F["A"], F["B"], F["C"]
    two = ft(2)
    ga = -(A * A * gA + A * B * gB + B * B * gC)
    gc = -(B * B * gA + B * C * gB + C * C * gC)
    gb = -(two * A * B * gA + (A * C + B * B) * gB + two * B * C * gC)
    T0, T1, c3, R = F["T0"], F["T1"], F["c3"], F["R"]
    hb = ft(0.5) * gb
    G3 = {(i, k): ga * T0[i] * T0[k] + hb * (T0[i] * T1[k] + T1[i] * T0[k]) + gc * T1[i] * T1[k]
          for i in range(3) for k in range(3)}
    TC0 = [T0[0] * c3(0, k) + T0[1] * c3(1, k) + T0[2] * c3(2, k) for k in range(3)]
    TC1 = [T1[0] * c3(0, k) + T1[1] * c3(1, k) + T1[2] * c3(2, k) for k in range(3)]
    dT0 = [two * (ga * TC0[k] + hb * TC1[k]) for k in range(3)]
    dT1 = [two * (hb * TC0[k] + gc * TC1[k]) for k in range(3)]
    gj00 = dT0[0] * R[0, 0] + dT0[1] * R[0, 1] + dT0[2] * R[0, 2]
    gj02 = dT0[0] * R[2, 0] + dT0[1] * R[2, 1] + dT0[2] * R[2, 2]
    gj11 = dT1[0] * R[1, 0] + dT1[1] * R[1, 1] + dT1[2] * R[1, 2]
    gj12 = dT1[0] * R[2, 0] + dT1[1] * R[2, 1] + dT1[2] * R[2, 2]
    fx, fy, x, y, iz = F["fx"], F["fy"], F["x"], F["y"], F["iz"]
    iz2 = iz * iz
    gx = gmx * fx * iz - gj02 * fx * iz2
    gy = gmy * fy * iz - gj12 * fy * iz2
    gz = (-(gmx * fx * x + gmy * fy * y + gj00 * fx + gj11 * fy) * iz2
          + two * (gj02 * fx * x + gj12 * fy * y) * iz2 * iz)
    v = F["valid"]
    gx, gy, gz = (np.where(v, a, ft(0)) for a in (gx, gy, gz))
    gmeans = np.stack([R[0, k] * gx + R[1, k] * gy + R[2, k] * gz for k in range(3)], 1)
    M, s, Rq = F["M"], F["s"], F["Rq"]
    dM = [two * (G3[(i, 0)] * M[j] + G3[(i, 1)] * M[3 + j] + G3[(i, 2)] * M[6 + j])
          for i in range(3) for j in range(3)]
    gls = np.stack([(dM[j] * Rq[j] + dM[3 + j] * Rq[3 + j] + dM[6 + j] * Rq[6 + j]) * s[:, j]
                    for j in range(3)], 1)
    g00, g01, g02, g10, g11, g12, g20, g21, g22 = [dM[3 * i + j] * s[:, j]
                                                   for i in range(3) for j in range(3)]
    w, qx, qy, qz = F["qn"]
    gqn = [two * (-qz * g01 + qy * g02 + qz * g10 - qx * g12 - qy * g20 + qx * g21),
           two * (qy * g01 + qz * g02 + qy * g10 - two * qx * g11 - w * g12 + qz * g20
                  + w * g21 - two * qx * g22),
           two * (-two * qy * g00 + qx * g01 + w * g02 + qx * g10 + qz * g12 - w * g20
                  + qz * g21 - two * qy * g22),
           two * (-two * qz * g00 - w * g01 + qx * g02 + w * g10 - two * qz * g11 + qy * g12
                  + qx * g20 + qy * g21)]
    dot = w * gqn[0] + qx * gqn[1] + qy * gqn[2] + qz * gqn[3]
    gq = np.stack([(gqn[i] - F["qn"][i] * dot) * F["qinv"] for i in range(4)], 1)
    op = F["opacity"]
    gol = gop * op * (ft(1) - op)
    keep = F["raw"] >= ft(0)
    gcol = np.where(keep, g[:, 6:9], ft(0))
    sh_all = np.asarray(params["sh"], ft)
    gsh = np.zeros_like(sh_all)
    Kd = F["basis"].shape[1]
    gsh[:, :Kd] = F["basis"][:, :, None] * gcol[:, None, :]
    if cfg.sh_degree > 0:
        db = sh_basis_grad(F["dirs"], cfg.sh_degree)                    # (N, K, 3xyz)
        gbasis = (sh_all[:, :Kd] * gcol[:, None, :]).sum(2, dtype=ft)   # (N, K)
        gdir = (db * gbasis[:, :, None]).sum(1, dtype=ft)               # (N, 3)
        dirs = F["dirs"]
        proj_d = (dirs * gdir).sum(1, dtype=ft)
        gmeans = gmeans + (gdir - dirs * proj_d[:, None]) / F["dnorm"][:, None]
    grads = {"means": gmeans, "log_scales": gls, "quats": gq, "opacity_logits": gol, "sh": gsh}
    zero = ~(g != 0).any(1)
    if zero.any():
        grads = {k: np.where(zero.reshape((-1,) + (1,) * (a.ndim - 1)), ft(0), a).astype(ft)
                 for k, a in grads.items()}
    return grads


# ------------------------------------------------------------------ Adam

def bf16_round(x):
    u = np.ascontiguousarray(x, f32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(f32)


def sparse_adam(params, grads, m, v, step, visible, lr=None, betas=(0.9, 0.999), eps=1e-15,
                bf16_moments=False):
    """Adam over visible rows; other rows unchanged. Returns new (params, m, v)."""
    lr = DEFAULT_LR if lr is None else lr
    b1, b2 = f32(betas[0]), f32(betas[1])
    t = step + 1
    bc1, bc2 = 1.0 - betas[0] ** t, 1.0 - betas[1] ** t
    isq = f32(1.0 / math.sqrt(bc2))
    rows = np.asarray(visible, bool)
    P, Mo, Vo = {}, {}, {}
    for name in PARAM_NAMES:
        p = np.array(params[name], f32)
        mm = np.array(m[name], f32)
        vv = np.array(v[name], f32)
        g = np.asarray(grads[name], f32)
        if name == "sh":
            ss = np.full((1, p.shape[1], 1), f32(lr["sh_rest"] / bc1), f32)
            ss[:, 0] = f32(lr["sh_dc"] / bc1)
            ss = np.broadcast_to(ss, p.shape)[rows]
        else:
            ss = f32(lr[name] / bc1)
        m1 = b1 * mm[rows] + (f32(1) - b1) * g[rows]
        v1 = b2 * vv[rows] + (f32(1) - b2) * g[rows] * g[rows]
        den = np.sqrt(v1) * isq + f32(eps)
        p[rows] = p[rows] - ss * (m1 / den)
        mm[rows] = bf16_round(m1) if bf16_moments else m1
        vv[rows] = bf16_round(v1) if bf16_moments else v1
        P[name], Mo[name], Vo[name] = p, mm, vv
    return P, Mo, Vo


# ------------------------------------------------------------------ whole step

def train_step(params, m, v, step, cams, targets, cfg: Cfg, lr=None, ssim=True,
               lambda_dssim=0.2, betas=(0.9, 0.999), eps=1e-15, bf16_moments=False):
    """One multi-view step: per view forward, loss, blend backward, projection backward;
    gradients and losses summed over views; sparse Adam over rows visible in >= 1 view.
    cams: list of (w2c, K, H, W). Returns dict(params, m, v, loss, grads, visible, views)."""
    N = np.asarray(params["means"]).shape[0]
    total = {k: np.zeros_like(np.asarray(params[k], f32)) for k in PARAM_NAMES}
    vis = np.zeros(N, bool)
    loss = 0.0
    views = []
    for (w2c, K, H, W), tgt in zip(cams, targets):
        pr = project(params, w2c, K, H, W, cfg)
        fw = forward(pr, H, W, cfg)
        L, dimg = (loss_ssim if ssim else loss_l1)(fw["image"], tgt, lambda_dssim)
        g2 = backward_2d(pr, fw["image"], dimg, H, W, cfg)
        gp = param_backward(params, g2, w2c, K, H, W, cfg)
        for k in PARAM_NAMES:
            total[k] += gp[k]
        vis |= pr["visible"]
        loss += L
        views.append({"image": fw["image"], "loss": L, "g2d": g2, "n_pairs": fw["n_pairs"]})
    P, Mo, Vo = sparse_adam(params, total, m, v, step, vis, lr, betas, eps, bf16_moments)
    return {"params": P, "m": Mo, "v": Vo, "loss": loss, "grads": total, "visible": vis,
            "views": views}


def rel_error(ad, ref, floor_frac=1e-4):
    """gsplat/train_oracle.py:406-417: max |ad - ref| / max(|ref|, floor * max|ref|)."""
    a, f = np.asarray(ad, np.float64).ravel(), np.asarray(ref, np.float64).ravel()
    scale = np.abs(f).max() if f.size else 0.0
    if scale == 0.0:
        return float(np.abs(a).max()) if a.size else 0.0
    return float((np.abs(a - f) / np.maximum(np.abs(f), floor_frac * scale)).max())
