"""The numpy training oracle (oracle/train.py) against the reference's own models.

Fixtures (tests/golden/make_golden_train.py) hold the reference's outputs: its fp32 tiled
forward, SSIM/L1 loss, blend backward slots and SH0 projection backward + Adam on a
seeded scene, and its fp64-autograd T0 gradient-oracle cases (SH0 and SH3)."""
import json
import os

import numpy as np
import pytest

from oracle import train as ot

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def tiled():
    return np.load(os.path.join(GOLDEN, "train_tiled.npz"))


def tiled_inputs(G):
    params = {k: G[f"param_{k}"] for k in ot.PARAM_NAMES}
    return params, G["w2c"], G["K"], int(G["H"]), int(G["W"])


def test_forward_matches_reference_forward_fast(tiled):
    params, w2c, K, H, W = tiled_inputs(tiled)
    cfg = ot.Cfg(sh_degree=0, tile=32)
    pr = ot.project(params, w2c, K, H, W, cfg)
    fw = ot.forward(pr, H, W, cfg)
    assert fw["n_live"] == int(tiled["n_live"])
    assert np.abs(fw["image"] - tiled["image"]).max() <= 1e-6


def test_loss_matches_reference(tiled):
    L, g = ot.loss_ssim(tiled["image"], tiled["target"])
    assert abs(L - float(tiled["loss"])) <= 1e-6 * abs(float(tiled["loss"]))
    assert np.abs(g - tiled["dL_dimage"]).max() <= 1e-5 * np.abs(tiled["dL_dimage"]).max()
    L1, g1 = ot.loss_l1(tiled["image"], tiled["target"])
    assert abs(L1 - float(tiled["loss_l1"])) <= 1e-9
    np.testing.assert_array_equal(g1, tiled["dL_dimage_l1"])


def test_blend_backward_matches_reference_slots(tiled):
    params, w2c, K, H, W = tiled_inputs(tiled)
    cfg = ot.Cfg(sh_degree=0, tile=32)
    pr = ot.project(params, w2c, K, H, W, cfg)
    g2d = ot.backward_2d(pr, tiled["image"], tiled["dL_dimage"], H, W, cfg)
    ok = ~tiled["tie_g"]
    assert ot.rel_error(g2d[ok], tiled["g2d"][ok]) <= 1e-3


def test_projection_backward_and_adam_match_reference(tiled):
    params, w2c, K, H, W = tiled_inputs(tiled)
    cfg = ot.Cfg(sh_degree=0, tile=32)
    grads = ot.param_backward(params, tiled["g2d"], w2c, K, H, W, cfg)
    # the reference evaluates exp in float32 and sums with numpy's reductions; the oracle
    # rounds exp once from float64 and sums in a fixed order (cancellation-prone elements
    # then differ by up to ~2e-4 relative; the gradient bar is 1e-3)
    for k in ot.PARAM_NAMES:
        assert ot.rel_error(grads[k], tiled[f"grad_{k}"]) <= 1e-3, k
    from tests.golden.make_golden_train import adam_state
    m_in, v_in = adam_state(params)
    lr = json.loads(str(tiled["adam_lr_json"]))
    vis = ot.project(params, w2c, K, H, W, cfg)["visible"]
    np.testing.assert_array_equal(vis, tiled["visible"])
    p1, m1, v1 = ot.sparse_adam(params, {k: tiled[f"grad_{k}"] for k in ot.PARAM_NAMES},
                                m_in, v_in, int(tiled["adam_step"]), vis, lr)
    for k in ot.PARAM_NAMES:
        np.testing.assert_array_equal(p1[k], tiled[f"adam_param_{k}"])
        np.testing.assert_array_equal(m1[k], tiled[f"adam_m_{k}"])
        np.testing.assert_array_equal(v1[k], tiled[f"adam_v_{k}"])


@pytest.mark.parametrize("deg", [0, 3])
def test_param_backward_matches_fp64_autograd(deg):
    """SH0 and SH3 (with the view-direction term into the means): the oracle's analytic
    backward fed the fp64 oracle's 2D grads reproduces its autograd parameter grads."""
    d = np.load(os.path.join(GOLDEN, f"train_t0_sh{deg}.npz"))
    params = {k: d[f"param_{k}"] for k in ot.PARAM_NAMES}
    g2d = np.concatenate([d["dL_dmeans2d"], d["dL_dconic"], d["dL_dopacity"][:, None],
                          d["dL_dcolors"]], 1)
    H, W = int(d["H"]), int(d["W"])
    cfg = ot.Cfg(sh_degree=deg, tile=32)
    for ft, bar in ((np.float64, 1e-9), (np.float32, 1e-3)):
        grads = ot.param_backward(params, g2d, d["w2c"], d["K"], H, W, cfg, ft=ft)
        for k in ot.PARAM_NAMES:
            err = ot.rel_error(grads[k], d[f"grad_{k}"])
            assert err <= bar, (k, ft, err)


@pytest.mark.parametrize("deg", [0, 3])
@pytest.mark.parametrize("bf16", [False, True])
def test_sparse_adam_matches_reference_dump(deg, bf16):
    d = np.load(os.path.join(GOLDEN, f"train_t0_sh{deg}.npz"))
    params = {k: d[f"param_{k}"].astype(np.float32) for k in ot.PARAM_NAMES}
    grads = {k: d[f"grad_{k}"].astype(np.float32) for k in ot.PARAM_NAMES}
    tag = "bf16" if bf16 else "fp32"
    mi = {k: d[f"adam_bf16_m_in_{k}" if bf16 else f"adam_m_in_{k}"] for k in ot.PARAM_NAMES}
    vi = {k: d[f"adam_bf16_v_in_{k}" if bf16 else f"adam_v_in_{k}"] for k in ot.PARAM_NAMES}
    lr = json.loads(str(d["adam_lr_json"]))
    p1, m1, v1 = ot.sparse_adam(params, grads, mi, vi, int(d["adam_step_in"]), d["visible"],
                                lr, tuple(d["adam_betas"]), float(d["adam_eps"]), bf16)
    for k in ot.PARAM_NAMES:
        assert ot.rel_error(p1[k] - params[k], d[f"adam_{tag}_param_{k}"] - params[k]) <= 1e-3
        assert ot.rel_error(m1[k], d[f"adam_{tag}_m_{k}"]) <= 1e-3
        assert ot.rel_error(v1[k], d[f"adam_{tag}_v_{k}"]) <= 1e-3


@pytest.mark.parametrize("deg", [0, 3])
def test_tiled_forward_vs_dense_fp64_oracle(deg):
    """The tiled fp32 forward (3-sigma tile rectangles) against the reference's dense fp64
    render of the same params: the image within 1e-4 max-abs and the projected 2D
    parameters within fp32 rounding."""
    d = np.load(os.path.join(GOLDEN, f"train_t0_sh{deg}.npz"))
    params = {k: d[f"param_{k}"] for k in ot.PARAM_NAMES}
    H, W = int(d["H"]), int(d["W"])
    for tile in (16, 32):
        cfg = ot.Cfg(sh_degree=deg, tile=tile)
        pr = ot.project(params, d["w2c"], d["K"], H, W, cfg)
        v = d["valid"]
        assert ot.rel_error(pr["means2d"][v], d["means2d"][v]) <= 1e-5
        assert ot.rel_error(pr["conic"][v], d["conic"][v]) <= 1e-4
        assert ot.rel_error(pr["colors"][v], d["colors"][v]) <= 1e-4
        np.testing.assert_array_equal(pr["visible"], d["visible"])
        fw = ot.forward(pr, H, W, cfg)
        assert np.abs(fw["image"] - d["image"]).max() <= 1e-4
        assert np.abs(fw["final_T"] - d["final_T"]).max() <= 1e-4


def test_blend_backward_vs_dense_fp64_oracle():
    """Tiled fp32 blend backward vs the fp64 autograd 2D grads (the reference's T1 bar is
    1e-2 relative on these cases, gsplat/blend_backward_ref.py:285)."""
    for deg in (0, 3):
        d = np.load(os.path.join(GOLDEN, f"train_t0_sh{deg}.npz"))
        params = {k: d[f"param_{k}"] for k in ot.PARAM_NAMES}
        H, W = int(d["H"]), int(d["W"])
        cfg = ot.Cfg(sh_degree=deg, tile=32)
        pr = ot.project(params, d["w2c"], d["K"], H, W, cfg)
        g2d = ot.backward_2d(pr, d["image"], d["dL_dimage"], H, W, cfg)
        vis = d["visible"]
        ref = np.concatenate([d["dL_dmeans2d"], d["dL_dconic"], d["dL_dopacity"][:, None],
                              d["dL_dcolors"]], 1)
        assert ot.rel_error(g2d[vis], ref[vis]) <= 1e-2


def test_exact_backward_agrees_with_reference_formula(tiled):
    """float64 back-to-front (backward_2d_exact) vs the reference's fp32 front-to-back slots
    on the reference-pinned tiled case: the same gradient up to the fp32 formula's error."""
    params, w2c, K, H, W = tiled_inputs(tiled)
    cfg = ot.Cfg(sh_degree=0, tile=32)
    pr = ot.project(params, w2c, K, H, W, cfg)
    g64 = ot.backward_2d_exact(pr, tiled["dL_dimage"], H, W, cfg)
    ok = ~tiled["tie_g"]
    assert ot.rel_error(g64[ok], tiled["g2d"][ok]) <= 2e-3


def test_view_pool_step_equals_sequential_train_step():
    """The process-parallel oracle step (the CPU baseline's driver) gives train_step's
    result exactly: per-view work in worker processes, gradients summed in view order."""
    from gsplat_tt_b200 import scenes
    from oracle.train_pool import ViewPool
    params = scenes.cluster_scene(1500, sh_degree=3, seed=7)
    params["means"] = (params["means"] * 0.5).astype(np.float32)
    params["log_scales"] = (params["log_scales"] + 1.5).astype(np.float32)
    H, W = 32, 48
    cams = [(c.w2c, c.K, H, W) for c in scenes.sphere_cameras(3, 3.5, 40.0, W, H)]
    tg = [np.random.default_rng(i).uniform(0, 1, (H, W, 3)).astype(np.float32) for i in range(3)]
    cfg = ot.Cfg(sh_degree=3, tile=16)
    zeros = {k: np.zeros_like(np.asarray(v, np.float32)) for k, v in params.items()}
    ref = ot.train_step(params, zeros, zeros, 0, cams, tg, cfg)
    with ViewPool(params, cfg, workers=2) as pool:
        got = pool.step(zeros, zeros, 0, cams, tg)
    assert got["loss"] == ref["loss"]
    np.testing.assert_array_equal(got["visible"], ref["visible"])
    for k in ot.PARAM_NAMES:
        np.testing.assert_array_equal(got["grads"][k], ref["grads"][k])
        np.testing.assert_array_equal(got["params"][k], ref["params"][k])
