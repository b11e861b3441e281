"""Training path on the B200 through the C ABI vs the oracle (oracle/train.py, itself
pinned to the reference's models): projection, intersections, sorted pairs and tile
ranges bit-exact; images within 1e-4 max-abs and gradients within 1e-3 relative
(train_oracle.rel_error), skipping pixels / Gaussians whose forward decisions sit within
4e-6 of a threshold (either side is a valid fp32 result there)."""
import os

import numpy as np
import pytest

from gsplat_tt_b200 import scenes
from oracle import train as ot

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
IMG_TOL = 1e-4
GRAD_TOL = 1e-3


def small_scene(n, deg, seed, aniso=False):
    p = scenes.cluster_scene(n, sh_degree=deg, seed=seed)
    p["means"] = (p["means"] * 0.5).astype(np.float32)
    p["log_scales"] = (p["log_scales"] + 1.5).astype(np.float32)
    if aniso:  # needle-like, opaque Gaussians: thin tilted ellipses stress the reach masks
        p["log_scales"][:, 0] += 1.5
        p["log_scales"][:, 2] -= 2.0
        p["opacity_logits"] = (np.abs(p["opacity_logits"]) + 2.0).astype(np.float32)
    return p


def cams_for(k, H, W, f, seed=4, radius=3.5):
    out = []
    rng = np.random.default_rng(seed)
    for _ in range(k):
        d = rng.standard_normal(3)
        d /= np.linalg.norm(d)
        out.append((scenes.look_at(radius * d), scenes.intrinsics(f, W, H), H, W))
    return out


def trainer(params, deg, tile, views, H, W, **kw):
    from gsplat_tt_b200.train import TrainConfig, Trainer
    cfg = TrainConfig(sh_degree=deg, tile_size=tile, **kw)
    return Trainer(params, cfg, views, H, W), cfg


@pytest.mark.parametrize("deg,tile,H,W", [(0, 16, 64, 96), (3, 16, 97, 130), (3, 32, 120, 72),
                                          (1, 16, 256, 256)])
def test_project_view_bit_exact(deg, tile, H, W):
    params = small_scene(20000, deg, seed=deg + tile)
    tr, _ = trainer(params, deg, tile, 1, H, W)
    (w2c, K, _, _), = cams_for(1, H, W, 0.9 * max(H, W), seed=deg)
    tr.ensure_capacity([(w2c, K, H, W)])
    dv = tr.project_view(w2c, K, H, W)
    cfg = ot.Cfg(sh_degree=deg, tile=tile)
    pr = ot.project(params, w2c, K, H, W, cfg)
    v = pr["valid"]
    for k in ("means2d", "conic", "opacity", "colors"):
        a = dv[k].cpu().numpy()[v]
        np.testing.assert_array_equal(a.view(np.uint32), np.asarray(pr[k], np.float32)[v].view(np.uint32), k)
    np.testing.assert_array_equal(dv["depth"].cpu().numpy().view(np.uint32),
                                  np.asarray(pr["depth"], np.float32).view(np.uint32))
    np.testing.assert_array_equal(dv["visible"].cpu().numpy() > 0, pr["visible"])
    rects = dv["rects"].cpu().numpy()
    has = pr["rects"][:, 1] >= pr["rects"][:, 0]
    np.testing.assert_array_equal(rects[has], pr["rects"][has])
    assert not (rects[~has][:, 1] >= rects[~has][:, 0]).any()
    tx = (W + tile - 1) // tile
    pl = ot.pair_lists(pr["rects"], pr["depth"], tx)
    assert dv["pairs"] == pl["g"].size
    np.testing.assert_array_equal(dv["sorted_ids"].cpu().numpy(), pl["g"].astype(np.int32))
    ranges = dv["tile_ranges"].cpu().numpy()
    tid = pl["tid"]
    ntiles = tx * ((H + tile - 1) // tile)
    exp = np.zeros((ntiles, 2), np.int64)
    if tid.size:
        starts = np.searchsorted(tid, np.arange(ntiles), "left")
        ends = np.searchsorted(tid, np.arange(ntiles), "right")
        nz = ends > starts
        exp[nz, 0], exp[nz, 1] = starts[nz], ends[nz]
    np.testing.assert_array_equal(ranges, exp)


@pytest.mark.parametrize("cells", ["4x2", "2x2", "1x1"])
def test_tile_lists_bit_exact_for_every_sort_cell_shape(cells, monkeypatch):
    """The per-tile lists (sorted ids) and ranges are the reference's stable (tile, depth,
    id) order whichever cells the tile sort sorts by: 4x2-tile super-tiles (the default
    below 2^24 Gaussians), 2x2-tile super-tiles (below 2^28) or the (Gaussian, tile) pairs
    themselves (GS_TILE_SORT_CELLS selects the shape; the library reads it on every call).
    Odd tile counts leave partial super-tiles on the right and bottom edges."""
    monkeypatch.setenv("GS_TILE_SORT_CELLS", cells)
    test_project_view_bit_exact(3, 16, 168, 200)


def run_step(params, deg, tile, cams, targets, ssim=True, lam=0.2, **kw):
    import torch
    H, W = cams[0][2], cams[0][3]
    tr, cfg = trainer(params, deg, tile, len(cams), H, W, use_ssim=ssim, lambda_dssim=lam, **kw)
    tr.ensure_capacity(cams)
    imgs = torch.zeros((len(cams), H, W, 3), device=tr.device)
    g2d = torch.zeros((len(cams), tr.n, 9), device=tr.device)
    tr.step(cams, targets, check_errors=True, images=imgs, grad2d=g2d)
    torch.cuda.synchronize()
    return tr, imgs.cpu().numpy(), g2d.cpu().numpy()


@pytest.mark.parametrize("deg,tile,ssim,aniso", [(3, 16, True, False), (0, 32, True, False),
                                                (3, 16, False, False), (2, 16, True, True),
                                                (1, 32, False, True)])
def test_train_step_vs_oracle(deg, tile, ssim, aniso):
    params = small_scene(8000, deg, seed=7 + deg, aniso=aniso)
    H, W = 72, 104
    cams = cams_for(2, H, W, 100.0)
    targets = scenes.random_targets([scenes.Camera(c[0], c[1], H, W) for c in cams], seed=9)
    lam = 0.2 if ssim else 0.0
    tr, imgs, g2d = run_step(params, deg, tile, cams, targets, ssim=ssim, lam=lam)
    cfg = ot.Cfg(sh_degree=deg, tile=tile)
    total = {k: np.zeros_like(np.asarray(params[k], np.float64)) for k in ot.PARAM_NAMES}
    vis = np.zeros(tr.n, bool)
    tie_any = np.zeros(tr.n, bool)
    for i, (w2c, K, _, _) in enumerate(cams):
        pr = ot.project(params, w2c, K, H, W, cfg)
        fw = ot.forward(pr, H, W, cfg)
        ok = ~fw["ties"]
        assert np.abs(imgs[i] - fw["image"])[ok].max() <= IMG_TOL
        # the loss and the 2D backward are evaluated on the device's own image
        L, dimg = (ot.loss_ssim if ssim else ot.loss_l1)(imgs[i], targets[i], lam)
        assert abs(float(tr.losses[i].item()) - L) <= 1e-5 * abs(L)
        # the reference's 2D-gradient formula evaluated exactly (float64, back to front) on
        # the fp32 forward's decisions; its fp32 front-to-back form (oracle.backward_2d)
        # cancels behind opaque layers and is itself ~3e-3 off on the anisotropic scene
        gref, ties = ot.backward_2d_exact(pr, dimg, H, W, cfg, ties=True)
        keep = ~ties
        assert ot.rel_error(g2d[i][keep], gref[keep]) <= GRAD_TOL
        # fp64 projection backward of the device's own 2D gradients: the exact parameter
        # gradient those 2D gradients imply (fp32 would cancel to ~1e-2 here)
        gp = ot.param_backward(params, g2d[i], w2c, K, H, W, cfg, ft=np.float64)
        for k in ot.PARAM_NAMES:
            total[k] = total[k] + gp[k]
        vis |= pr["visible"]
        tie_any |= ties
    np.testing.assert_array_equal(tr.vis_counts.cpu().numpy() > 0, vis)
    dev_grads = tr.grads.numpy()
    for k in ot.PARAM_NAMES:
        assert ot.rel_error(dev_grads[k], total[k]) <= GRAD_TOL, k
    # sparse Adam on the device's gradients, from zero moments at step 0
    zeros = {k: np.zeros_like(total[k], dtype=np.float32) for k in ot.PARAM_NAMES}
    p1, m1, v1 = ot.sparse_adam(params, dev_grads, zeros, zeros, 0, vis, tr.cfg.lr)
    got = tr.params.numpy()
    for k in ot.PARAM_NAMES:
        d_ref = p1[k] - np.asarray(params[k], np.float32)
        d_dev = got[k] - np.asarray(params[k], np.float32)
        assert ot.rel_error(d_dev, d_ref) <= GRAD_TOL, k
        assert ot.rel_error(tr.m.numpy()[k], m1[k]) <= 1e-6
        assert ot.rel_error(tr.v.numpy()[k], v1[k]) <= 1e-6


@pytest.mark.parametrize("deg", [0, 3])
def test_train_step_vs_reference_fp64_dump(deg):
    """The reference's T0 case (64x64, 50 Gaussians, 0.8 L1 + 0.2 D-SSIM) against its fp64
    autograd: image 1e-4, 2D and parameter gradients within the reference's 1e-2 tiled-vs-
    dense bar (gsplat/blend_backward_ref.py:285; the dense oracle has no tile rectangles)."""
    d = np.load(os.path.join(GOLDEN, f"train_t0_sh{deg}.npz"))
    params = {k: d[f"param_{k}"].astype(np.float32) for k in ot.PARAM_NAMES}
    H, W = int(d["H"]), int(d["W"])
    cams = [(d["w2c"], d["K"], H, W)]
    tr, imgs, g2d = run_step(params, deg, 32, cams, [d["target"].astype(np.float32)])
    assert np.abs(imgs[0] - d["image"]).max() <= IMG_TOL
    assert abs(float(tr.losses[0].item()) - float(d["loss"])) <= 1e-4 * float(d["loss"])
    vis = d["visible"]
    ref2d = np.concatenate([d["dL_dmeans2d"], d["dL_dconic"], d["dL_dopacity"][:, None],
                            d["dL_dcolors"]], 1)
    assert ot.rel_error(g2d[0][vis], ref2d[vis]) <= 1e-2
    dev = tr.grads.numpy()
    for k in ot.PARAM_NAMES:
        assert ot.rel_error(dev[k], d[f"grad_{k}"]) <= 1e-2, k


def test_overflow_retry_and_multi_step():
    import torch
    from gsplat_tt_b200.train import TrainConfig, Trainer
    params = small_scene(6000, 3, seed=21)
    H, W = 64, 64
    cams = cams_for(3, H, W, 70.0, seed=5)
    cfg = TrainConfig(sh_degree=3, tile_size=16)
    # targets rendered from the unperturbed scene; train the perturbed copy toward them
    ref = Trainer(params, cfg, 3, H, W)
    ref.ensure_capacity(cams)
    imgs = torch.zeros((3, H, W, 3), device=ref.device)
    ref.step(cams, [np.zeros((H, W, 3), np.float32)] * 3, check_errors=True, images=imgs)
    targets = [imgs[i].clone() for i in range(3)]
    rng = np.random.default_rng(0)
    pert = {k: (v + 0.02 * rng.standard_normal(v.shape)).astype(np.float32) for k, v in params.items()}
    tr = Trainer(pert, cfg, 3, H, W, pair_capacity=16)  # far too small: exercises the retry
    losses = []
    for _ in range(15):
        losses.append(float(tr.step(cams, targets, check_errors=True).sum().item()))
    assert tr.capacity > 16
    assert np.isfinite(losses).all() and losses[-1] < losses[0]


def test_projection_ahead_matches_projection_in_step():
    """next_cams: a step projects the next step's views after its update
    (gs_train_project_rows) and the next step starts at the pair-count scan
    (GS_STEP_PROJECTED). From the same parameters and moments, that next step gives the
    loss, gradients and parameters of a step that projects its views itself, bit for bit
    (deterministic gradient sums); a projection made for other cameras is discarded and the
    step projects its own. The second trainer starts from a copy of the first's state after
    the first step, so the comparison covers one step."""
    import torch
    params = small_scene(6000, 3, seed=21)
    H, W = 64, 96
    cams = cams_for(3, H, W, 90.0)
    other = cams_for(3, H, W, 90.0, seed=9)
    targets = [torch.from_numpy(t).cuda() for t in
               scenes.random_targets([scenes.Camera(c[0], c[1], H, W) for c in cams], seed=22)]
    for nxt in (cams, other):
        ahead, _ = trainer(params, 3, 16, len(cams), H, W, deterministic=True)
        plain, _ = trainer(params, 3, 16, len(cams), H, W, deterministic=True)
        for tr in (ahead, plain):
            tr.ensure_capacity(cams)
        ahead.step(cams, targets, next_cams=nxt)
        assert ahead._projected is not None
        for a, b in ((plain.params, ahead.params), (plain.m, ahead.m), (plain.v, ahead.v)):
            a.flat.copy_(b.flat)
        plain.step_count = ahead.step_count
        la = ahead.step(cams, targets).cpu().numpy()
        lp = plain.step(cams, targets).cpu().numpy()
        torch.cuda.synchronize()
        assert lib_error(ahead) == 0 and lib_error(plain) == 0
        np.testing.assert_allclose(la, lp, rtol=1e-6)
        ga, gp = ahead.grads.numpy(), plain.grads.numpy()
        pa, pp = ahead.params.numpy(), plain.params.numpy()
        for k in ot.PARAM_NAMES:
            np.testing.assert_array_equal(ga[k], gp[k], k)
            np.testing.assert_array_equal(pa[k], pp[k], k)


def lib_error(tr):
    import torch
    from gsplat_tt_b200._lib import lib
    return lib.gs_workspace_error(tr.ws.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_project_rows_argument_errors():
    """gs_train_project_rows rejects row ranges off the GS_PROJECT_ROW_ALIGN grid."""
    import torch
    from gsplat_tt_b200.train import GS_PROJECT_ROW_ALIGN
    params = small_scene(1000, 3, seed=3)
    H, W = 32, 48
    cams = cams_for(1, H, W, 40.0)
    tr, _ = trainer(params, 3, 16, 1, H, W)
    arr = tr._cams(cams)
    st = torch.cuda.current_stream().cuda_stream
    for b, e in ((1, 1000), (0, 300), (GS_PROJECT_ROW_ALIGN, 1001), (512, 256)):
        with pytest.raises(ValueError):
            tr._project_rows(arr, b, e, st)
    tr._project_rows(arr, 0, GS_PROJECT_ROW_ALIGN, st)
    tr._project_rows(arr, GS_PROJECT_ROW_ALIGN, 1000, st)
    torch.cuda.synchronize()
    # the projected rows feed a step: counts of the visible Gaussians are set
    assert float(tr.vis_counts.sum().item()) > 0.0


def test_bf16_moments_match_the_oracle_bf16_mode():
    """bf16 moment storage (gsplat/train_oracle.py:434-470, bf16 mode): the moments live in
    2-byte arrays, and two steps of the device's sparse Adam match the oracle's bf16 mode
    applied to the device's own gradients and previous state: the moments equal up to one
    bf16 unit where an fp32 rounding difference crossed a bf16 rounding boundary (at most
    0.1 % of them), the parameters equal up to two fp32 units of the parameter (the device
    fuses p - lr m / den into one rounding) plus one bf16 unit of the step."""
    import torch
    from gsplat_tt_b200.train import TrainConfig, Trainer
    params = small_scene(5000, 3, seed=2)
    H, W = 48, 64
    cams = cams_for(2, H, W, 60.0, seed=8)
    targets = scenes.random_targets([scenes.Camera(c[0], c[1], H, W) for c in cams], seed=4)
    cfg = TrainConfig(sh_degree=3, tile_size=16, bf16_moments=True)
    tr = Trainer(params, cfg, 2, H, W)
    assert tr.m.flat.dtype == torch.bfloat16 and tr.v.flat.element_size() == 2
    tr.ensure_capacity(cams)
    for step in range(2):
        p0, m0, v0 = tr.params.numpy(), tr.m.numpy(), tr.v.numpy()
        tr.step(cams, targets, check_errors=True)
        torch.cuda.synchronize()
        g = tr.grads.numpy()
        vis = tr.vis_counts.cpu().numpy() > 0
        p1, m1, v1 = ot.sparse_adam(p0, g, m0, v0, step, vis, cfg.lr, bf16_moments=True)
        got_p, got_m, got_v = tr.params.numpy(), tr.m.numpy(), tr.v.numpy()
        for k in ot.PARAM_NAMES:
            np.testing.assert_array_equal(got_m[k], ot.bf16_round(got_m[k]))
            bound = 2.0 * np.spacing(np.abs(p1[k])) + 2.0 ** -7 * np.abs(p1[k] - p0[k])
            assert (np.abs(got_p[k] - p1[k]) <= bound).all(), (step, k)
            for dev, ref in ((got_m[k], m1[k]), (got_v[k], v1[k])):
                diff = dev != ref
                assert diff.mean() <= 1e-3, (step, k, diff.mean())
                assert (np.abs(dev - ref) <= 2.0 ** -7 * np.abs(ref) + 1e-30)[diff].all(), (step, k)


def test_host_targets_match_device_targets():
    """Pinned host targets (copied by the library on its own stream, overlapped with the
    lanes) and pageable numpy targets give the same step as device targets over several
    views: the same losses and, with deterministic gradient sums, the same gradients bit for
    bit."""
    import torch
    params = small_scene(6000, 3, seed=21)
    H, W = 64, 96
    cams = cams_for(5, H, W, 90.0)
    targets = scenes.random_targets([scenes.Camera(c[0], c[1], H, W) for c in cams], seed=22)
    results = []
    for kind in ("device", "pinned", "numpy"):
        tr, _ = trainer(params, 3, 16, len(cams), H, W, deterministic=True)
        tr.ensure_capacity(cams)
        if kind == "device":
            tg = [torch.from_numpy(t).cuda() for t in targets]
        elif kind == "pinned":
            tg = [torch.from_numpy(t).pin_memory() for t in targets]
        else:
            tg = targets
        tr.step(cams, tg, check_errors=True)
        torch.cuda.synchronize()
        results.append((tr.losses.cpu().numpy(), tr.grads.numpy()))
    for losses, g in results[1:]:
        np.testing.assert_allclose(losses, results[0][0], rtol=1e-6)
        for k in ot.PARAM_NAMES:
            np.testing.assert_array_equal(g[k], results[0][1][k], k)


@pytest.mark.parametrize("deg,tile,ssim", [(3, 16, True), (1, 32, False)])
def test_staged_chain_matches_train_step_and_oracle(deg, tile, ssim):
    """gs_render_fwd -> gs_loss -> gs_render_bwd -> gs_train_param_backward -> gs_sparse_adam
    through the C ABI: the same image and loss as gs_train_step on the view (the same
    kernels); with 16x16 tiles (deterministic gradient sums on both sides) the same 2D and
    parameter gradients and Adam update bit for bit; with 32x32 tiles (float atomics) the
    same 2D gradients up to their summation order, and parameter gradients and the Adam
    update checked against the oracle on the staged chain's own 2D gradients (the atomics
    noise, amplified where the projection backward cancels, reaches 1e-4 there); and the
    oracle's image, loss and 2D gradients."""
    import torch
    from gsplat_tt_b200.train import StagedView
    params = small_scene(8000, deg, seed=40 + deg)
    H, W = 72, 104
    cams = cams_for(1, H, W, 100.0, seed=6)
    target = scenes.random_targets([scenes.Camera(cams[0][0], cams[0][1], H, W)], seed=3)[0]
    lam = 0.2 if ssim else 0.0
    det = tile == 16
    ref, img_ref, g2d_ref = run_step(params, deg, tile, cams, [target], ssim=ssim, lam=lam,
                                     deterministic=det)

    tr, _ = trainer(params, deg, tile, 1, H, W, use_ssim=ssim, lambda_dssim=lam, deterministic=det)
    tr.ensure_capacity(cams)
    sv = StagedView(tr, H, W)
    img = sv.forward(cams[0][0], cams[0][1])
    assert not sv.overflowed()
    loss, dimg = sv.loss(img, target)
    g2d = sv.backward(dimg)
    sv.param_backward()
    sv.adam(0)
    torch.cuda.synchronize()
    img_np = img.cpu().numpy()
    np.testing.assert_array_equal(img_np, img_ref[0])
    assert float(loss.item()) == float(ref.losses[0].item())
    np.testing.assert_array_equal(tr.vis_counts.cpu().numpy(), ref.vis_counts.cpu().numpy())
    cfg = ot.Cfg(sh_degree=deg, tile=tile)
    if det:
        np.testing.assert_array_equal(g2d.cpu().numpy(), g2d_ref[0])
        for k in ot.PARAM_NAMES:
            np.testing.assert_array_equal(tr.grads.numpy()[k], ref.grads.numpy()[k], k)
            np.testing.assert_array_equal(tr.params.numpy()[k], ref.params.numpy()[k], k)
    else:
        assert ot.rel_error(g2d.cpu().numpy(), g2d_ref[0]) <= 1e-4
        # fp64 projection backward of the staged chain's own 2D gradients, then sparse Adam
        # on its own parameter gradients from zero moments at step 0
        gp = ot.param_backward(params, g2d.cpu().numpy(), cams[0][0], cams[0][1], H, W, cfg,
                               ft=np.float64)
        dev_grads = tr.grads.numpy()
        vis = tr.vis_counts.cpu().numpy() > 0
        zeros = {k: np.zeros_like(np.asarray(params[k], np.float32)) for k in ot.PARAM_NAMES}
        p1, _, _ = ot.sparse_adam(params, dev_grads, zeros, zeros, 0, vis, tr.cfg.lr)
        for k in ot.PARAM_NAMES:
            assert ot.rel_error(dev_grads[k], gp[k]) <= GRAD_TOL, k
            d_ref = p1[k] - np.asarray(params[k], np.float32)
            d_dev = tr.params.numpy()[k] - np.asarray(params[k], np.float32)
            assert ot.rel_error(d_dev, d_ref) <= GRAD_TOL, k
    # the oracle: forward, loss and the exact 2D backward
    pr = ot.project(params, cams[0][0], cams[0][1], H, W, cfg)
    fw = ot.forward(pr, H, W, cfg)
    ok = ~fw["ties"]
    assert np.abs(img_np - fw["image"])[ok].max() <= IMG_TOL
    np.testing.assert_array_equal(sv.n_contrib.cpu().numpy()[ok], fw["n_contrib"][ok])
    L, dref = (ot.loss_ssim if ssim else ot.loss_l1)(img_np, target, lam)
    assert abs(float(loss.item()) - L) <= 1e-5 * abs(L)
    assert np.abs(dimg.cpu().numpy() - dref).max() <= 1e-5 * np.abs(dref).max()
    gex, ties = ot.backward_2d_exact(pr, dimg.cpu().numpy(), H, W, cfg, ties=True)
    assert ot.rel_error(g2d.cpu().numpy()[~ties], gex[~ties]) <= GRAD_TOL
