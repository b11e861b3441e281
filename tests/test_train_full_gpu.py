"""The training path at the benchmark configurations' full sizes, through the C ABI, against
the oracle: one full view of C3 (500k Gaussians SH3, 1024x1024, L1) and of C4 (3M Gaussians
SH3, 1600x1056, 0.8 L1 + 0.2 D-SSIM) through gs_train_project_view and gs_train_step, and
one view of C5 (6M Gaussians, 1920x1080) through the projection and the sort.

Bars, as in the small-scene tests: projection records, visibility, tile rectangles, the
pair count, the sorted Gaussian ids and the tile ranges bit-exact (oracle/train.py project
and pair_lists); the image within 1e-4 max-abs away from pixels whose forward decisions sit
within 4e-6 of a threshold; the loss within 1e-5 relative; 2D gradients within 1e-3
relative (rel_error) of the exact float64 backward away from Gaussians touched by such a
decision; parameter gradients within 1e-3 of the float64 projection backward of the
device's own 2D gradients and the Adam update within 1e-3, the moments within 1e-6 (on a
seeded sample of rows above 600k Gaussians: both are per-row maps). The
rasteriser and its backward are checked with the C restatement of the numpy models
(oracle/gs_train_oracle.c, reproduced bit for bit by tests/test_oracle_train_c.py), which
finishes a full view in seconds."""
import numpy as np
import pytest

from gsplat_tt_b200 import scenes
from oracle import train as ot
from oracle import train_fast as tf

pytestmark = pytest.mark.gpu
IMG_TOL = 1e-4
GRAD_TOL = 1e-3


def _view(name, index=0):
    c = scenes.CONFIGS[name]
    cam = scenes.training_cameras(name)[index]
    return c, (cam.w2c, cam.K, c["height"], c["width"])


def _check_projection(tr, params, cam, cfg):
    """Device projection, rectangles, pairs, sorted ids and ranges against the oracle,
    bit for bit. Returns the oracle projection and its (sorted ids, tile ranges)."""
    w2c, K, H, W = cam
    tile = cfg.tile
    dv = tr.project_view(w2c, K, H, W)
    pr = ot.project(params, w2c, K, H, W, cfg)
    v = pr["valid"]
    for k in ("means2d", "conic", "opacity", "colors"):
        a = dv[k].cpu().numpy()[v]
        np.testing.assert_array_equal(a.view(np.uint32),
                                      np.asarray(pr[k], np.float32)[v].view(np.uint32), k)
    np.testing.assert_array_equal(dv["depth"].cpu().numpy().view(np.uint32),
                                  np.asarray(pr["depth"], np.float32).view(np.uint32))
    np.testing.assert_array_equal(dv["visible"].cpu().numpy() > 0, pr["visible"])
    rects = dv["rects"].cpu().numpy()
    has = pr["rects"][:, 1] >= pr["rects"][:, 0]
    np.testing.assert_array_equal(rects[has], pr["rects"][has])
    assert not (rects[~has][:, 1] >= rects[~has][:, 0]).any()
    del dv["means2d"], dv["conic"], dv["colors"], rects
    tx, ty = (W + tile - 1) // tile, (H + tile - 1) // tile
    pl = ot.pair_lists(pr["rects"], pr["depth"], tx)
    assert dv["pairs"] == pl["g"].size
    np.testing.assert_array_equal(dv["sorted_ids"].cpu().numpy(), pl["g"].astype(np.int32))
    ids, ranges = tf.pair_table(pl["g"], pl["tid"], tx * ty)
    del pl
    np.testing.assert_array_equal(dv["tile_ranges"].cpu().numpy(), ranges)
    return pr, (ids, ranges)


def _full_view(name, ssim):
    import torch
    from gsplat_tt_b200.train import TrainConfig, Trainer
    c, cam = _view(name)
    w2c, K, H, W = cam
    params = scenes.cluster_scene(c["n"], sh_degree=3, seed=0)
    lam = 0.2 if ssim else 0.0
    cfg = TrainConfig(sh_degree=3, tile_size=16, use_ssim=ssim, lambda_dssim=lam,
                      lr=dict(scenes.LR_BASELINE))
    tr = Trainer(params, cfg, 1, H, W)
    tr.ensure_capacity([cam])
    ocfg = ot.Cfg(sh_degree=3, tile=16)
    pr, pairs = _check_projection(tr, params, cam, ocfg)
    print(f"{name}: {pairs[0].size} pairs, {int(pr['visible'].sum())} visible")

    target = np.random.default_rng(1).uniform(0, 1, (H, W, 3)).astype(np.float32)
    img = torch.zeros((1, H, W, 3), device=tr.device)
    g2d = torch.zeros((1, tr.n, 9), device=tr.device)
    tr.step([cam], [target], check_errors=True, images=img, grad2d=g2d)
    torch.cuda.synchronize()
    img = img[0].cpu().numpy()
    g2d = g2d[0].cpu().numpy()

    fw = tf.forward(pr, H, W, ocfg, pairs=pairs)
    ok = ~fw["ties"]
    assert ok.mean() > 0.99
    img_err = float(np.abs(img - fw["image"])[ok].max())
    print(f"{name}: image max-abs {img_err:.2e} on {ok.mean():.4%} of pixels")
    assert img_err <= IMG_TOL
    # the loss and the 2D backward are evaluated on the device's own image
    L, dimg = (ot.loss_ssim if ssim else ot.loss_l1)(img, target, lam)
    assert abs(float(tr.losses[0].item()) - L) <= 1e-5 * abs(L)
    gref, ties = tf.backward_2d_exact(pr, dimg, H, W, ocfg, ties=True, pairs=pairs)
    keep = ~ties
    assert keep.mean() > 0.85  # a tainted pixel marks every later pair reaching it
    g_err = ot.rel_error(g2d[keep], gref[keep])
    print(f"{name}: 2D gradients rel {g_err:.2e} on {keep.mean():.2%} of Gaussians")
    assert g_err <= GRAD_TOL
    del gref, fw
    # The projection backward and Adam are per-row maps (a row's result depends on its own
    # parameters and 2D gradient only), so above 600k Gaussians they are checked on a
    # seeded sample of 400k rows plus the 2,000 rows with the largest 2D gradients (which
    # set rel_error's floor), to keep the float64 oracle within seconds.
    vis = pr["visible"]
    np.testing.assert_array_equal(tr.vis_counts.cpu().numpy() > 0, vis)
    n = tr.n
    if n > 600_000:
        big = np.argpartition(np.abs(g2d).max(1), n - 2000)[n - 2000:]
        idx = np.union1d(np.random.default_rng(7).choice(n, 400_000, replace=False), big)
    else:
        idx = np.arange(n)
    sub = {k: np.asarray(params[k], np.float32)[idx] for k in ot.PARAM_NAMES}
    del pr
    gp = ot.param_backward(sub, g2d[idx], w2c, K, H, W, ocfg, ft=np.float64)
    dev = {k: v[idx] for k, v in tr.grads.numpy().items()}
    errs = {k: ot.rel_error(dev[k], gp[k]) for k in ot.PARAM_NAMES}
    print(f"{name}: parameter gradients rel " + ", ".join(f"{k} {e:.2e}" for k, e in errs.items()))
    for k in ot.PARAM_NAMES:
        assert errs[k] <= GRAD_TOL, k
    del gp
    zeros = {k: np.zeros_like(v) for k, v in sub.items()}
    p1, m1, v1 = ot.sparse_adam(sub, dev, zeros, zeros, 0, vis[idx], tr.cfg.lr)
    got = {k: v[idx] for k, v in tr.params.numpy().items()}
    gm = {k: v[idx] for k, v in tr.m.numpy().items()}
    gv = {k: v[idx] for k, v in tr.v.numpy().items()}
    for k in ot.PARAM_NAMES:
        assert ot.rel_error(got[k] - sub[k], p1[k] - sub[k]) <= GRAD_TOL, k
        assert ot.rel_error(gm[k], m1[k]) <= 1e-6, k
        assert ot.rel_error(gv[k], v1[k]) <= 1e-6, k


def test_c3_full_view_train_step_vs_oracle():
    _full_view("c3", ssim=False)


def test_c4_full_view_train_step_vs_oracle():
    _full_view("c4", ssim=True)


def test_c5_view_projection_and_sort_vs_oracle():
    from gsplat_tt_b200.train import TrainConfig, Trainer
    c, cam = _view("c5")
    params = scenes.cluster_scene(c["n"], sh_degree=3, seed=0)
    tr = Trainer(params, TrainConfig(sh_degree=3, tile_size=16), 1, cam[2], cam[3])
    tr.ensure_capacity([cam])
    pr, (ids, _) = _check_projection(tr, params, cam, ot.Cfg(sh_degree=3, tile=16))
    print(f"c5: {ids.size} pairs, {int(pr['visible'].sum())} visible")
