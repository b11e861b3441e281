"""The C display-path oracle against the reference's golden vectors and known answers.

Pins oracle/gs_oracle.c (the checker of the CUDA path) to the reference: bit-exact on
config C1 and on the C2 sort against fixtures generated from the reference's own
compiled pipeline (tests/golden/make_golden.py), on the reference's C++ known-answer
cases (tests/unit/test_sort.cpp, test_tile_assign.cpp, test_blend.cpp), and -- when
oracle/_ref is built -- directly against the reference on ragged random cases.
"""
import hashlib
import os

import numpy as np
import pytest

from gsplat_tt_b200 import scenes
from oracle import display as od

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a)).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def golden_display():
    return np.load(os.path.join(GOLDEN, "display.npz"))


def c1_oracle(cull):
    sc, cam = scenes.c1_scene(), scenes.c1_camera()
    cov3d = od.compute_cov3d(sc["scales"], sc["rotations"])
    m2, cv, d, r, v = od.project_full_with_cov3d(sc["means"], cov3d, cam.w2c, cam.K, 256, 256,
                                                 sc["opacities"])
    col, op = sc["colors"][v], sc["opacities"][v]
    kw = dict(covs_2d=cv, opacities=op, contrib_floor=1.0 / 16384.0) if cull else {}
    g, t, n = od.tile_assign(m2, r, 256, 256, 16, **kw)
    s, rg = od.sort(g, t, d, 16, 16)
    img = od.blend(m2, cv, col, op, s, rg, 256, 256, 16)
    return dict(cov3d=cov3d, m2=m2, cv=cv, d=d, r=r, v=v, g=g, t=t, n=n, s=s, rg=rg, img=img)


@pytest.mark.parametrize("cull", [False, True])
def test_c1_oracle_matches_reference_golden(golden_display, cull):
    G = golden_display
    tag = "cull" if cull else "nocull"
    o = c1_oracle(cull)
    assert o["m2"].shape[0] == int(G["M"]) == 9940
    assert sha(o["cov3d"]) == str(G["sha_cov3d"])
    for k, gk in (("m2", "means_2d"), ("cv", "covs_2d"), ("d", "depths"), ("r", "radii")):
        assert sha(o[k]) == str(G[f"sha_{gk}"]), k
    assert sha(o["v"].astype(np.uint8)) == str(G["sha_valid"])
    assert o["g"].shape[0] == int(G[f"P_{tag}"])
    assert sha(o["g"]) == str(G[f"sha_gids_{tag}"])
    assert sha(o["t"]) == str(G[f"sha_tids_{tag}"])
    assert sha(o["n"]) == str(G[f"sha_tpg_{tag}"])
    assert sha(o["s"]) == str(G[f"sha_sorted_{tag}"])
    np.testing.assert_array_equal(o["rg"], G[f"ranges_{tag}"])
    assert sha(o["img"]) == str(G[f"sha_image_{tag}"])
    if not cull:
        np.testing.assert_array_equal(o["img"], G["image"])


def test_c2_sort_oracle_matches_reference_golden():
    G = np.load(os.path.join(GOLDEN, "sort.npz"))
    keys, vals = scenes.c2_pairs()
    assert keys.size == int(G["n"])
    _, vo = od.sort_pairs(keys, vals)
    assert sha(vo) == str(G["sha_sorted_values"])
    ks, vs = scenes.c2_pairs(n=1 << 16, seed=3)
    _, v2 = od.sort_pairs(ks, vs)
    np.testing.assert_array_equal(v2, G["sample_sorted_values"])
    assert keys.size - np.unique(keys).size == int(G["duplicates"]) == 208520


# --- known answers restated from the reference's C++ unit tests --------------------

def test_sort_kats():
    # tests/unit/test_sort.cpp:5-18 same tile sorted by depth
    s, _ = od.sort([0, 1, 2], [5, 5, 5], np.array([0.5, 0.3, 0.7], np.float32), 8, 8)
    assert s.tolist() == [1, 0, 2]
    # :20-36 ranges of three populated tiles
    _, r = od.sort([0, 1, 2, 3, 4], [2, 2, 7, 7, 10],
                   np.array([0.4, 0.6, 0.5, 0.8, 0.3, 0.9], np.float32), 4, 3)
    assert r[2].tolist() == [0, 2] and r[7].tolist() == [2, 4] and r[10].tolist() == [4, 5]
    # :38-50 empty tiles keep zero ranges
    _, r = od.sort([0], [3], np.array([1.0], np.float32), 4, 4)
    assert r[0].tolist() == [0, 0] and r[3].tolist() == [0, 1] and r[5].tolist() == [0, 0]
    # :52-62 same tile orders by depth, not by Gaussian id
    s, _ = od.sort([5, 1], [4, 4], np.array([0.2, 0.9, 0.4, 0.6, 0.1, 0.8], np.float32), 4, 4)
    assert s.tolist() == [5, 1]
    # :64-75 empty input
    s, r = od.sort(np.zeros(0, np.int64), np.zeros(0, np.int64), np.array([1.0], np.float32), 2, 2)
    assert s.size == 0 and r.shape == (4, 2) and not r.any()


def test_tile_assign_kats():
    # tests/unit/test_tile_assign.cpp:17-32 one Gaussian at a tile centre -> one tile
    g, t, n = od.tile_assign(np.array([[48.0, 48.0]], np.float32),
                             np.array([[8.0, 8.0]], np.float32), 256, 256, 32)
    assert g.tolist() == [0] and t.tolist() == [1 * 8 + 1] and n.tolist() == [1]
    # :34-46 straddling four tiles
    g, t, n = od.tile_assign(np.array([[32.0, 32.0]], np.float32),
                             np.array([[16.0, 16.0]], np.float32), 256, 256, 32)
    assert g.size == 4 and n.tolist() == [4]
    # :48-66 the Mahalanobis cull drops low-contribution pairs; counts stay consistent
    m2 = np.array([[16, 16], [240, 240]], np.float32)
    r = np.full((2, 2), 20.0, np.float32)
    cv = np.array([[0.01, 0, 0, 0.01]] * 2, np.float32)
    op = np.array([0.5, 0.5], np.float32)
    g0, _, _ = od.tile_assign(m2, r, 256, 256, 32)
    g1, _, n1 = od.tile_assign(m2, r, 256, 256, 32, cv, op, 15.0 / 255.0)
    assert g1.size < g0.size and n1.sum() == g1.size


def blend_kat_cases():
    """Known answers of tests/unit/test_blend.cpp:29-107 as (inputs, check) pairs; shared
    with the GPU tests."""
    cases = []
    # :29-53 single Gaussian at the pixel centre -> alpha clamp 0.99 of its colour
    cases.append((dict(m2=[[16.5, 16.5]], cv=[[50, 0, 0, 50]], col=[[1, 0, 0]], op=[1.0],
                       ids=[0], rg=[[0, 1]], H=32, W=32, tile=32),
                  lambda im: abs(im[16, 16, 0] - 0.99) < 1e-3 and abs(im[16, 16, 1]) < 1e-3
                  and abs(im[16, 16, 2]) < 1e-3))
    # :55-77 front to back: a faint red in front of an opaque green
    cases.append((dict(m2=[[16.5, 16.5]] * 2, cv=[[50, 0, 0, 50]] * 2, col=[[1, 0, 0], [0, 1, 0]],
                       op=[0.01, 1.0], ids=[0, 1], rg=[[0, 2]], H=32, W=32, tile=32),
                  lambda im: im[16, 16, 0] < 0.05 and im[16, 16, 1] > 0.95))
    # :79-107 early termination: 100 stacked opaque Gaussians saturate T; pixels stay finite
    cases.append((dict(m2=[[16.5, 16.5]] * 100, cv=[[400, 0, 0, 400]] * 100,
                       col=[[0.2, 0.4, 0.6]] * 100, op=[0.99] * 100, ids=list(range(100)),
                       rg=[[0, 100]], H=32, W=32, tile=32),
                  lambda im: np.all(np.isfinite(im)) and abs(im[16, 16, 1] - 0.4) < 1e-3))
    # empty tile (second tile of a 64x32 image) stays black
    cases.append((dict(m2=[[16.5, 16.5]], cv=[[50, 0, 0, 50]], col=[[1, 1, 1]], op=[1.0],
                       ids=[0], rg=[[0, 1], [0, 0]], H=32, W=64, tile=32),
                  lambda im: not im[:, 32:].any()))
    out = []
    for kw, chk in cases:
        a = {k: (np.asarray(v, np.float32) if k in ("m2", "cv", "col", "op") else v)
             for k, v in kw.items()}
        a["ids"] = np.asarray(a["ids"], np.int64)
        a["rg"] = np.asarray(a["rg"], np.int64)
        out.append((a, chk))
    return out


def test_blend_kats():
    for a, chk in blend_kat_cases():
        img = od.blend(a["m2"], a["cv"], a["col"], a["op"], a["ids"], a["rg"], a["H"], a["W"],
                       a["tile"])
        assert chk(img)


# --- direct comparison with the compiled reference, when present -------------------

def random_scene(n, H, W, seed):
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


@pytest.mark.parametrize("H,W,tile,seed", [(64, 48, 16, 1), (100, 37, 32, 2), (33, 65, 8, 3),
                                           (128, 128, 16, 4)])
def test_oracle_vs_compiled_reference_ragged(H, W, tile, seed):
    ref = od.reference_module()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    means, scales, q, op, col, w2c, K = random_scene(3000, H, W, seed)
    c_o = od.compute_cov3d(scales, q)
    c_r = np.asarray(ref.compute_cov3d(scales, q))
    assert np.array_equal(c_o.view(np.uint32), c_r.view(np.uint32))
    o = od.project_full_with_cov3d(means, c_o, w2c, K, H, W, op)
    r = [np.asarray(x) for x in ref.project_full_with_cov3d(means, c_r, w2c, K, H, W, op)]
    for a, b in zip(o, r):
        assert np.array_equal(a, b)
    m2, cv, d, rad, v = r
    for kw in ({}, dict(covs_2d=cv, opacities=op[v], contrib_floor=1.0 / 16384.0)):
        go = od.tile_assign(m2, rad, H, W, tile, **kw)
        gr = [np.asarray(x) for x in ref.tile_assign(m2, rad, H, W, tile, **kw)]
        for a, b in zip(go, gr):
            assert np.array_equal(a, b)
        tx, ty = (W + tile - 1) // tile, (H + tile - 1) // tile
        so = od.sort(go[0], go[1], d, tx, ty)
        sr = [np.asarray(x) for x in ref.sort(gr[0], gr[1], d, tx, ty)]
        assert np.array_equal(so[0], sr[0]) and np.array_equal(so[1], sr[1])
        io = od.blend(m2, cv, col[v], op[v], so[0], so[1], H, W, tile)
        ir = np.asarray(ref.blend(m2, cv.reshape(-1, 4), col[v], op[v], sr[0], sr[1], H, W, tile))
        assert np.array_equal(io, ir)


@pytest.mark.parametrize("H,W,tile,seed", [(64, 48, 16, 5), (100, 37, 32, 6), (128, 128, 32, 7),
                                           (256, 256, 16, 8)])
def test_cull_and_blend_oracle_vs_compiled_reference(H, W, tile, seed):
    """The microblock cull + blend restatement against the reference's compiled
    cull_and_blend (scalar build): image and cull statistics bit-exact."""
    ref = od.reference_module()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    means, scales, q, op, col, w2c, K = random_scene(4000, H, W, seed)
    c = od.compute_cov3d(scales, q)
    m2, cv, d, rad, v = od.project_full_with_cov3d(means, c, w2c, K, H, W, op)
    g, t, _ = od.tile_assign(m2, rad, H, W, tile, covs_2d=cv, opacities=op[v],
                             contrib_floor=1.0 / 16384.0)
    tx, ty = (W + tile - 1) // tile, (H + tile - 1) // tile
    s, rg = od.sort(g, t, d, tx, ty)
    for floor in (1.0 / 16384.0, 1.0 / 255.0):
        io, so = od.cull_and_blend(m2, cv, col[v], op[v], s, rg, tx, ty, tile, H, W, floor)
        ir, sr = ref.cull_and_blend(m2, cv.reshape(-1, 4), col[v], op[v], s, rg, tx, ty, tile,
                                    H, W, floor)
        assert np.array_equal(io, np.asarray(ir))
        assert so == {k: int(sr[k]) for k in ("pairs_in", "pairs_dropped", "pairs_kept_per_mb")}
        assert so["pairs_kept_per_mb"] > 0


def test_render_full_chain_matches_reference_render_full():
    """The oracle's staged chain (project -> tile_assign with pair cull -> sort ->
    microblock cull + blend) reproduces the reference's render_full on C1, tile 32."""
    ref = od.reference_module()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    sc, cam = scenes.c1_scene(), scenes.c1_camera()
    cov3d = od.compute_cov3d(sc["scales"], sc["rotations"])
    img_r, st_r = ref.render_full(sc["means"], cov3d, sc["opacities"], sc["colors"], cam.w2c,
                                  cam.K, 256, 256)
    m2, cv, d, rad, v = od.project_full_with_cov3d(sc["means"], cov3d, cam.w2c, cam.K, 256, 256,
                                                   sc["opacities"])
    g, t, _ = od.tile_assign(m2, rad, 256, 256, 32, covs_2d=cv, opacities=sc["opacities"][v],
                             contrib_floor=1.0 / 16384.0)
    s, rg = od.sort(g, t, d, 8, 8)
    img_o, st_o = od.cull_and_blend(m2, cv, sc["colors"][v], sc["opacities"][v], s, rg, 8, 8, 32,
                                    256, 256)
    assert np.array_equal(img_o, np.asarray(img_r))
    assert int(st_r["num_visible"]) == m2.shape[0] and int(st_r["num_entries"]) == s.shape[0]
    for k in ("pairs_in", "pairs_dropped", "pairs_kept_per_mb"):
        assert st_o[k] == int(st_r[k]), k
