"""Training-path golden fixtures from the reference's own Python models.

Called by make_golden.py (``--only train``); needs the reference tree (not available on
the GPU box -- the fixtures it writes are committed):

* train_t0_sh{0,3}.npz -- the reference's T0 gradient-oracle cases (fp64 autograd forward,
  L1+SSIM loss, 2D and parameter gradients, one sparse Adam step with fp32 and bf16
  moments), regenerated with gsplat/train_oracle.py:475-541 build_case and checked equal
  to the copies the reference commits (benchmarks/train_oracle/*.npz).
* train_tiled.npz -- a seeded SH0 cluster scene (gsplat_tt_b200.scenes.cluster_scene)
  projected by this repository's oracle, then run through the reference's fp32 tiled
  models on those exact inputs: forward_fast image (gsplat/blend_backward_dev.py:404),
  loss_and_grad_device / loss_and_grad_l1 (gsplat/train_loss.py:126,166), ref_slots_fast
  summed per Gaussian (gsplat/blend_backward_dev.py:444 with t2_param_backward.py:50),
  projection_backward_sh0 and adam_step (gsplat/t2_param_backward.py:123,195).
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _import_ref(ref_root: str):
    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)
    import gsplat.blend_backward_dev as bbd
    import gsplat.t2_param_backward as t2
    import gsplat.train_loss as tl
    import gsplat.train_oracle as to
    return to, bbd, tl, t2


def make_t0(ref_root: str, to) -> None:
    for deg in (0, 3):
        d = to.build_case(deg, n=50, height=64, width=64)
        committed = np.load(os.path.join(ref_root, "benchmarks", "train_oracle",
                                         f"t0_sh{deg}_64x64_n50.npz"))
        worst = 0.0
        for k in committed.files:
            a, b = np.asarray(d[k]), np.asarray(committed[k])
            if a.dtype.kind in "fc":
                worst = max(worst, float(np.max(np.abs(a - b) / np.maximum(np.abs(b), 1e-30)))
                            if a.size else 0.0)
            else:
                assert np.array_equal(a, b), k
        # the reference's own test tolerates one fp32 element at 7e-8 relative (libm)
        assert worst < 1e-6, worst
        np.savez_compressed(os.path.join(HERE, f"train_t0_sh{deg}.npz"), **d)
        print(f"train_t0_sh{deg}.npz: regenerated, max rel diff vs committed {worst:.1e}")


def adam_state(params):
    """Seeded Adam moments for the tiled case (the tests rebuild the same arrays)."""
    gen = np.random.default_rng(6)
    m_in = {k: (0.01 * gen.standard_normal(np.shape(v))).astype(np.float32)
            for k, v in params.items()}
    v_in = {k: (1e-4 * gen.random(np.shape(v))).astype(np.float32) for k, v in params.items()}
    return m_in, v_in


def tiled_scene():
    """The seeded SH0 scene and camera of train_tiled.npz."""
    sys.path.insert(0, ROOT)
    from gsplat_tt_b200 import scenes
    H, W = 96, 128
    params = scenes.cluster_scene(3000, sh_degree=0, seed=11)
    params["means"] = (params["means"] * np.float32(0.6)).astype(np.float32)
    params["log_scales"] = (params["log_scales"] + np.float32(1.2)).astype(np.float32)
    cam = scenes.look_at((0.3, -0.2, -4.0))
    K = scenes.intrinsics(150.0, W, H)
    return params, cam, K, H, W


def make_tiled(bbd, tl, t2) -> None:
    from oracle import train as ot
    params, cam, K, H, W = tiled_scene()
    cfg = ot.Cfg(sh_degree=0, tile=32)
    pr = ot.project(params, cam, K, H, W, cfg)
    order = np.argsort(pr["depth"], kind="stable")
    bcfg = bbd.BlendCfg()
    img, st = bbd.forward_fast(pr["means2d"], pr["conic"], pr["opacity"], pr["colors"], order,
                               pr["valid"], H, W, bcfg)
    rng = np.random.default_rng(5)
    target = rng.uniform(0, 1, (H, W, 3)).astype(np.float32)
    loss, l1, ssim, dimg = tl.loss_and_grad_device(img, target)
    loss_l1, dimg_l1 = tl.loss_and_grad_l1(img, target)
    d = {"image": img, "dL_dimage": dimg, "means2d": pr["means2d"], "conic": pr["conic"],
         "opacity": pr["opacity"], "colors": pr["colors"], "valid": pr["valid"],
         "order": order}
    slots, ties = bbd.ref_slots_fast(d, bcfg, ties=True)
    rects = bbd.tile_rects_vec(pr["means2d"], pr["valid"], pr["conic"], H, W)
    counts = np.where(rects[:, 1] >= rects[:, 0],
                      (rects[:, 1] - rects[:, 0] + 1) * (rects[:, 3] - rects[:, 2] + 1), 0)
    P = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int64)
    g2d = t2.segment_reduce(slots, P, counts)
    tie_g = np.zeros(counts.size, bool)
    for g in np.nonzero(counts)[0]:
        tie_g[g] = ties[P[g]:P[g] + counts[g]].any()
    grads, vis = t2.projection_backward_sh0(params, g2d, cam, K, H, W)
    m_in, v_in = adam_state(params)
    lr = {"means": 1.6e-4, "log_scales": 5e-3, "quats": 1e-3, "opacity_logits": 0.05,
          "sh_dc": 2.5e-3, "sh_rest": 1.25e-4}
    p1, m1, v1 = t2.adam_step(params, grads, m_in, v_in, 7, vis, lr, bf16_moments=False)
    out = {"H": H, "W": W, "tile": 32, "w2c": cam, "K": K, "target": target,
           "image": img, "n_live": st["n_live_px"], "loss": loss, "l1": l1, "ssim": ssim,
           "dL_dimage": dimg, "loss_l1": loss_l1, "dL_dimage_l1": dimg_l1, "g2d": g2d,
           "tie_g": tie_g, "visible": vis, "adam_step": 7, "adam_lr_json": json.dumps(lr)}
    for k in params:
        out[f"param_{k}"] = params[k]
        out[f"grad_{k}"] = grads[k]
        out[f"adam_param_{k}"], out[f"adam_m_{k}"], out[f"adam_v_{k}"] = p1[k], m1[k], v1[k]
    np.savez_compressed(os.path.join(HERE, "train_tiled.npz"), **out)
    print("train_tiled.npz: pairs", st["n_pairs"], "live px", st["n_live_px"],
          "tie Gaussians", int(tie_g.sum()), "visible", int(vis.sum()))


def main(ref_root: str) -> None:
    to, bbd, tl, t2 = _import_ref(ref_root)
    make_t0(ref_root, to)
    make_tiled(bbd, tl, t2)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GSPLAT_TT_REFERENCE")
    if not root:
        sys.exit("usage: make_golden_train.py <reference root> (or set GSPLAT_TT_REFERENCE)")
    main(root)
