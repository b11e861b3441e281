"""Display path on the B200 through the C ABI vs the oracle and the reference's golden
vectors: projection, pair counts, sorted orders and tile ranges bit-exact; image and
alpha within 1e-4 max-abs (fp32 exp differs between libraries)."""
import hashlib
import os

import numpy as np
import pytest

from gsplat_tt_b200 import scenes
from oracle import display as od

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
IMG_TOL = 1e-4


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a)).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def gd():
    from gsplat_tt_b200 import display
    return display


def np_(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("cull", [False, True])
def test_c1_bit_exact_vs_reference_golden(gd, cull):
    G = np.load(os.path.join(GOLDEN, "display.npz"))
    tag = "cull" if cull else "nocull"
    sc, cam = scenes.c1_scene(), scenes.c1_camera()
    cov3d = gd.compute_cov3d(sc["scales"], sc["rotations"])
    assert sha(np_(cov3d)) == str(G["sha_cov3d"])
    m2, cv, d, r, v, col, op = gd.project_full_with_cov3d(
        sc["means"], cov3d, cam.w2c, cam.K, 256, 256, sc["opacities"], colors=sc["colors"])
    assert m2.shape[0] == int(G["M"])
    assert sha(np_(m2)) == str(G["sha_means_2d"])
    assert sha(np_(cv)) == str(G["sha_covs_2d"])
    assert sha(np_(d)) == str(G["sha_depths"])
    assert sha(np_(r)) == str(G["sha_radii"])
    assert sha(np_(v).astype(np.uint8)) == str(G["sha_valid"])
    np.testing.assert_array_equal(np_(col), sc["colors"][np_(v)])
    np.testing.assert_array_equal(np_(op), sc["opacities"][np_(v)])
    kw = dict(covs_2d=cv, opacities=op, contrib_floor=1.0 / 16384.0) if cull else {}
    g, t, n = gd.tile_assign(m2, r, 256, 256, 16, **kw)
    assert g.shape[0] == int(G[f"P_{tag}"])
    assert sha(np_(g)) == str(G[f"sha_gids_{tag}"])
    assert sha(np_(t)) == str(G[f"sha_tids_{tag}"])
    assert sha(np_(n)) == str(G[f"sha_tpg_{tag}"])
    s, rg = gd.sort(g, t, d, 16, 16)
    assert sha(np_(s)) == str(G[f"sha_sorted_{tag}"])
    np.testing.assert_array_equal(np_(rg), G[f"ranges_{tag}"])
    img, alpha = gd.blend(m2, cv.reshape(-1, 4), col, op, s, rg, 256, 256, 16, return_alpha=True)
    ref_img = od.blend(np_(m2), np_(cv), np_(col), np_(op), np_(s), np_(rg), 256, 256, 16,
                       return_alpha=True)
    assert np.abs(np_(img) - ref_img[0]).max() <= IMG_TOL
    assert np.abs(np_(alpha) - ref_img[1]).max() <= IMG_TOL
    if not cull:
        assert np.abs(np_(img) - G["image"]).max() <= IMG_TOL


def ragged_scene(n, H, W, seed):
    rng = np.random.default_rng(seed)
    means = rng.uniform(-1, 1, (n, 3)).astype(np.float32)
    scales = np.exp(rng.normal(-3.5, 0.8, (n, 3))).astype(np.float32)
    q = rng.standard_normal((n, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    op = (1 / (1 + np.exp(-rng.normal(-1, 2, n)))).astype(np.float32)
    col = rng.uniform(0, 1, (n, 3)).astype(np.float32)
    w2c = scenes.look_at(rng.normal(0, 1, 3) * 0.3 + np.array([0, 0, -2.5]))
    K = scenes.intrinsics(0.9 * max(H, W), W, H)
    return means, scales, q, op, col, w2c, K


@pytest.mark.parametrize("H,W,tile,seed,n", [(64, 48, 16, 1, 3000), (100, 37, 32, 2, 3000),
                                             (33, 65, 8, 3, 3000), (128, 128, 16, 4, 20000),
                                             (720, 1280, 16, 5, 200000)])
def test_ragged_vs_oracle(gd, H, W, tile, seed, n):
    means, scales, q, op, col, w2c, K = ragged_scene(n, H, W, seed)
    c_o = od.compute_cov3d(scales, q)
    c_g = gd.compute_cov3d(scales, q)
    np.testing.assert_array_equal(np_(c_g).view(np.uint32), c_o.view(np.uint32))
    o = od.project_full_with_cov3d(means, c_o, w2c, K, H, W, op)
    g = gd.project_full_with_cov3d(means, c_g, w2c, K, H, W, op)
    for a, b in zip(o, g):
        np.testing.assert_array_equal(a, np_(b))
    m2, cv, d, rad, v = o
    for cull in (False, True):
        kw = dict(covs_2d=cv, opacities=op[v], contrib_floor=1.0 / 16384.0) if cull else {}
        to = od.tile_assign(m2, rad, H, W, tile, **kw)
        tg = gd.tile_assign(m2, rad, H, W, tile, **kw)
        for a, b in zip(to, tg):
            np.testing.assert_array_equal(a, np_(b))
        tx, ty = (W + tile - 1) // tile, (H + tile - 1) // tile
        so = od.sort(to[0], to[1], d, tx, ty)
        sg = gd.sort(tg[0], tg[1], d, tx, ty)
        np.testing.assert_array_equal(so[0], np_(sg[0]))
        np.testing.assert_array_equal(so[1], np_(sg[1]))
        io, ao = od.blend(m2, cv, col[v], op[v], so[0], so[1], H, W, tile, return_alpha=True)
        ig, ag = gd.blend(m2, cv.reshape(-1, 4), col[v], op[v], sg[0], sg[1], H, W, tile,
                          return_alpha=True)
        assert np.abs(io - np_(ig)).max() <= IMG_TOL
        assert np.abs(ao - np_(ag)).max() <= IMG_TOL


def test_kats_on_gpu(gd):
    from tests.test_oracle_display import blend_kat_cases
    for a, chk in blend_kat_cases():
        img = np_(gd.blend(a["m2"], a["cv"], a["col"], a["op"], a["ids"], a["rg"], a["H"],
                           a["W"], a["tile"]))
        assert chk(img)
    s, _ = gd.sort([0, 1, 2], [5, 5, 5], np.array([0.5, 0.3, 0.7], np.float32), 8, 8)
    assert np_(s).tolist() == [1, 0, 2]
    _, r = gd.sort([0, 1, 2, 3, 4], [2, 2, 7, 7, 10],
                   np.array([0.4, 0.6, 0.5, 0.8, 0.3, 0.9], np.float32), 4, 3)
    r = np_(r)
    assert r[2].tolist() == [0, 2] and r[7].tolist() == [2, 4] and r[10].tolist() == [4, 5]
    s, r = gd.sort(np.zeros(0, np.int64), np.zeros(0, np.int64), np.array([1.0], np.float32), 2, 2)
    assert s.numel() == 0 and not np_(r).any()
    g, t, n = gd.tile_assign(np.array([[48.0, 48.0]], np.float32),
                             np.array([[8.0, 8.0]], np.float32), 256, 256, 32)
    assert np_(g).tolist() == [0] and np_(t).tolist() == [9] and np_(n).tolist() == [1]


def test_empty_and_fully_culled(gd):
    cam = scenes.c1_camera()
    z = np.zeros((0, 3), np.float32)
    m2, cv, d, r, v = gd.project_full_with_cov3d(z, np.zeros((0, 9), np.float32), cam.w2c, cam.K,
                                                 64, 64, np.zeros(0, np.float32))
    assert m2.shape[0] == 0 and v.numel() == 0
    # every Gaussian behind the near plane
    means = np.tile(np.array([[0, 0, -3.0]], np.float32), (10, 1))
    c3 = np.tile(np.eye(3, dtype=np.float32).reshape(1, 9) * 1e-4, (10, 1))
    m2, cv, d, r, v = gd.project_full_with_cov3d(means, c3, cam.w2c, cam.K, 64, 64)
    assert m2.shape[0] == 0 and not np_(v).any()
    g, t, n = gd.tile_assign(m2, r, 64, 64, 16)
    assert g.numel() == 0


def test_tile_assign_overflow_retry(gd):
    m2 = np.array([[128.0, 128.0]] * 50, np.float32)
    r = np.array([[100.0, 100.0]] * 50, np.float32)
    g, t, n = gd.tile_assign(m2, r, 256, 256, 16, capacity=10)
    o = od.tile_assign(m2, r, 256, 256, 16)
    np.testing.assert_array_equal(np_(g), o[0])
    np.testing.assert_array_equal(np_(t), o[1])


def test_backend_plugin_stages(gd):
    import torch
    from gsplat_tt_b200.backend import get_backend
    be = get_backend("b200", tile_size=16)
    sc, cam = scenes.c1_scene(2000), scenes.c1_camera()
    T = {k: torch.from_numpy(v) for k, v in sc.items()}
    m2, cv, d, r, v = be.project(T["means"], T["scales"], T["rotations"],
                                 torch.from_numpy(cam.w2c), torch.from_numpy(cam.K), 256, 256,
                                 opacities=T["opacities"])
    assert m2.device.type == "cpu" and cv.shape[1:] == (2, 2)
    g, t, _ = be.tile_assign(m2, r, 256, 256, 16)
    s, rg = be.sort(g, t, d, 16, 16)
    img, sub = be.blend(m2, cv, T["colors"][v], T["opacities"][v], s, rg, 256, 256)
    assert img.shape == (256, 256, 3) and img.dtype == np.float32 and "kernel" in sub

    class G:  # the reference's Gaussians record (gsplat/data_structures.py)
        pass
    gg = G()
    for k, val in T.items():
        setattr(gg, k, val)
    # the fused render is the reference's render_full: 32-pixel tiles, pair cull, microblock
    # cull + blend -- checked against the oracle's chain of the same stages
    img2, stats = be.render_fused(gg, torch.from_numpy(cam.w2c), torch.from_numpy(cam.K), 256, 256)
    cov3d = od.compute_cov3d(sc["scales"], sc["rotations"])
    om2, ocv, od_, orad, ov = od.project_full_with_cov3d(sc["means"], cov3d, cam.w2c, cam.K, 256,
                                                         256, sc["opacities"])
    og, ot_, _ = od.tile_assign(om2, orad, 256, 256, 32, covs_2d=ocv, opacities=sc["opacities"][ov],
                                contrib_floor=1.0 / 16384.0)
    os_, org = od.sort(og, ot_, od_, 8, 8)
    oimg, ost = od.cull_and_blend(om2, ocv, sc["colors"][ov], sc["opacities"][ov], os_, org, 8, 8,
                                  32, 256, 256)
    assert np.abs(img2 - oimg).max() <= IMG_TOL
    assert stats["num_visible"] == om2.shape[0] and stats["num_entries"] == os_.shape[0]
    for k in ("pairs_in", "pairs_dropped", "pairs_kept_per_mb"):
        assert stats[k] == ost[k], k
    be.close()


@pytest.mark.parametrize("H,W,tile,seed,n,floor,cull_off", [
    (64, 48, 16, 11, 3000, 1.0 / 16384.0, False), (100, 37, 32, 12, 3000, 1.0 / 255.0, False),
    (128, 128, 32, 13, 20000, 1.0 / 16384.0, False), (33, 65, 8, 14, 3000, 1.0 / 16384.0, True),
    (720, 1280, 32, 15, 200000, 1.0 / 16384.0, False)])
def test_cull_and_blend_vs_oracle(gd, H, W, tile, seed, n, floor, cull_off):
    """Microblock cull + blend on the device against the oracle restatement (itself
    bit-exact against the reference's compiled cull_and_blend): cull statistics exact,
    image within 1e-4."""
    means, scales, q, op, col, w2c, K = ragged_scene(n, H, W, seed)
    c = od.compute_cov3d(scales, q)
    m2, cv, d, rad, v = od.project_full_with_cov3d(means, c, w2c, K, H, W, op)
    g, t, _ = od.tile_assign(m2, rad, H, W, tile, covs_2d=cv, opacities=op[v],
                             contrib_floor=1.0 / 16384.0)
    tx, ty = (W + tile - 1) // tile, (H + tile - 1) // tile
    s, rg = od.sort(g, t, d, tx, ty)
    for thr in (1.0 / 255.0, 1e-4):
        io, so = od.cull_and_blend(m2, cv, col[v], op[v], s, rg, tx, ty, tile, H, W, floor,
                                   cull_off, thr)
        ig, sg = gd.cull_and_blend(m2, cv.reshape(-1, 4), col[v], op[v], s, rg, tx, ty, tile, H, W,
                                   floor, cull_off, thr)
        assert sg == so
        assert np.abs(np_(ig) - io).max() <= IMG_TOL


def test_render_full_matches_oracle_chain(gd):
    """render_full (tile 32 default) = project -> pair cull -> sort -> microblock cull +
    blend, against the same chain on the oracle, on C1."""
    sc, cam = scenes.c1_scene(), scenes.c1_camera()
    cov3d = od.compute_cov3d(sc["scales"], sc["rotations"])
    img, st = gd.render_full(sc["means"], cov3d, sc["opacities"], sc["colors"], cam.w2c, cam.K,
                             256, 256)
    m2, cv, d, rad, v = od.project_full_with_cov3d(sc["means"], cov3d, cam.w2c, cam.K, 256, 256,
                                                   sc["opacities"])
    g, t, _ = od.tile_assign(m2, rad, 256, 256, 32, covs_2d=cv, opacities=sc["opacities"][v],
                             contrib_floor=1.0 / 16384.0)
    s, rg = od.sort(g, t, d, 8, 8)
    io, so = od.cull_and_blend(m2, cv, sc["colors"][v], sc["opacities"][v], s, rg, 8, 8, 32, 256,
                               256)
    assert np.abs(img - io).max() <= IMG_TOL
    assert st["num_visible"] == m2.shape[0] and st["num_entries"] == s.shape[0]
    for k in ("pairs_in", "pairs_dropped", "pairs_kept_per_mb"):
        assert st[k] == so[k], k
