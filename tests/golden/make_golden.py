"""Regenerate the golden fixtures in tests/golden/ from the reference itself.

Run in a container where the reference is available (it is not on the GPU box):

    python tests/golden/make_golden.py --ref <reference root> [--only display,sort,train]

(--ref defaults to $GSPLAT_TT_REFERENCE.)

* display.npz -- config C1 (seeded scene of gsplat_tt_b200.scenes.c1_scene) through
  the reference's own compiled CPU pipeline (oracle/_ref/_gsplat_cpu, built from the
  reference sources by oracle/Makefile): visible count, pair counts with and without the
  pair cull, SHA-256 of every bit-exact output, tile ranges, and the rendered image.
* sort.npz -- config C2 (2^24 Zipf pairs, seed 0) through the reference's sort_and_bin:
  SHA-256 of the sorted values and of the tile ranges, plus a 64 Ki-pair sample (seed 3) in full.
* train_*.npz -- written by the training section (reference Python training models).

The fixtures are committed; tests compare the repository's oracle and its CUDA path
against them without needing the reference at run time.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from gsplat_tt_b200 import scenes  # noqa: E402
from oracle import display as od  # noqa: E402


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a)).tobytes()).hexdigest()


def make_display(ref) -> None:
    sc, cam = scenes.c1_scene(), scenes.c1_camera()
    H, W, tile = cam.height, cam.width, 16
    cov3d = np.asarray(ref.compute_cov3d(sc["scales"], sc["rotations"]))
    m2, cv, d, r, v = (np.asarray(x) for x in ref.project_full_with_cov3d(
        sc["means"], cov3d, cam.w2c, cam.K, H, W, sc["opacities"]))
    col, op = sc["colors"][v], sc["opacities"][v]
    out = {"M": np.int64(m2.shape[0]), "sha_cov3d": sha(cov3d), "sha_means_2d": sha(m2),
           "sha_covs_2d": sha(cv), "sha_depths": sha(d), "sha_radii": sha(r),
           "sha_valid": sha(v.astype(np.uint8))}
    for tag, kw in (("nocull", {}), ("cull", dict(covs_2d=cv, opacities=op,
                                                   contrib_floor=1.0 / 16384.0))):
        g, t, n = (np.asarray(x) for x in ref.tile_assign(m2, r, H, W, tile, **kw))
        s, rg = (np.asarray(x) for x in ref.sort(g, t, d, (W + tile - 1) // tile,
                                                  (H + tile - 1) // tile))
        img = np.asarray(ref.blend(m2, cv.reshape(-1, 4), col, op, s, rg, H, W, tile))
        out.update({f"P_{tag}": np.int64(g.shape[0]), f"sha_gids_{tag}": sha(g),
                    f"sha_tids_{tag}": sha(t), f"sha_tpg_{tag}": sha(n),
                    f"sha_sorted_{tag}": sha(s), f"ranges_{tag}": rg, f"sha_image_{tag}": sha(img)})
        if tag == "nocull":
            out["image"] = img
    np.savez_compressed(os.path.join(HERE, "display.npz"), **out)
    print("display.npz:", {k: (int(v) if np.ndim(v) == 0 and not isinstance(v, str) else "...")
                           for k, v in out.items() if k.startswith(("M", "P_"))})


def make_sort(ref) -> None:
    keys, vals = scenes.c2_pairs()
    n_tiles = 8160
    tiles = (keys >> np.uint64(32)).astype(np.int64)
    depth = (keys & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
    dv = np.empty(vals.shape[0], np.float32)
    dv[vals] = depth  # values are a permutation: depth indexed by value
    s, rg = (np.asarray(x) for x in ref.sort(vals.astype(np.int64), tiles, dv, 120, 68))
    counts = np.bincount(tiles, minlength=n_tiles)
    dup = int(keys.size - np.unique(keys).size)
    ks, vs = scenes.c2_pairs(n=1 << 16, seed=3)
    t2 = (ks >> np.uint64(32)).astype(np.int64)
    d2 = (ks & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
    dv2 = np.empty(vs.shape[0], np.float32)
    dv2[vs] = d2
    s2, _ = (np.asarray(x) for x in ref.sort(vs.astype(np.int64), t2, dv2, 120, 68))
    np.savez_compressed(os.path.join(HERE, "sort.npz"),
                        sha_sorted_values=sha(s.astype(np.uint32)), sha_ranges=sha(rg),
                        ranges=rg, n=np.int64(keys.size), duplicates=np.int64(dup),
                        max_tile=np.int64(counts.max()),
                        sample_sorted_values=s2.astype(np.uint32))
    print("sort.npz: duplicates", dup, "largest tile", int(counts.max()))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GSPLAT_TT_REFERENCE"),
                    required="GSPLAT_TT_REFERENCE" not in os.environ)
    ap.add_argument("--only", default="display,sort,train")
    a = ap.parse_args()
    parts = a.only.split(",")
    od.build(ref=True, ref_root=a.ref)
    ref = od.reference_module()
    if ref is None:
        sys.exit("oracle/_ref was not built (is the reference at --ref?)")
    if "display" in parts:
        make_display(ref)
    if "sort" in parts:
        make_sort(ref)
    if "train" in parts:
        from tests.golden import make_golden_train  # noqa: E402
        make_golden_train.main(a.ref)


if __name__ == "__main__":
    main()
