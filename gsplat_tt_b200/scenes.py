"""Seeded synthetic scenes and cameras for the five benchmark configurations.

The reference benchmarks these paths on synthetic scenes only; these generators give
the same shapes, sizes and value distributions (numpy ``default_rng``, fp32 storage):

* ``c1``   -- N=10k forward render: means U[-1,1]^3, log-scales N(-4, 0.5), quats
  N(0,1)^4 normalised (w, x, y, z), opacity logits N(0,1), SH degree 0 RGB U[0,1];
  camera at (0,0,-3) looking along +z, f=300, 256x256, principal point at the centre.
* ``c2``   -- 2^24 (uint64 key, uint32 value) sort pairs: key = tile << 32 | bits(depth),
  tile = a fixed permutation of 8,160 tiles indexed by a Zipf(1.1) rank, depth U[0.1, 50],
  values a shuffle of 0..N-1.
* ``c3..c5`` -- 64 isotropic clusters (centres U[-2,2]^3, sigma 0.3), log-scales
  N(-4.5, 0.7), random unit quats, opacity logits N(0, 1.5), SH degree 3 (DC U[0,1],
  higher bands N(0, 0.05)); cameras on a sphere looking at the origin (OpenCV axes:
  x right, y down, z forward; world up -y).

Parameters use the reference trainer's optimizer-space names and layouts
(gsplat/train_oracle.py:8-20): means (N,3), log_scales (N,3), quats (N,4, w first),
opacity_logits (N,), sh (N,K,3).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

SH_C0 = 0.28209479177387814


@dataclass
class Camera:
    """World-to-camera 4x4 ``w2c``, 3x3 intrinsics ``K``, image size."""
    w2c: np.ndarray
    K: np.ndarray
    height: int
    width: int


def intrinsics(f: float, width: int, height: int) -> np.ndarray:
    return np.array([[f, 0.0, width / 2.0], [0.0, f, height / 2.0], [0.0, 0.0, 1.0]],
                    np.float32)


def look_at(position, target=(0.0, 0.0, 0.0)) -> np.ndarray:
    """w2c of a camera at ``position`` looking at ``target`` (OpenCV axes, world up -y)."""
    p = np.asarray(position, np.float64)
    fwd = np.asarray(target, np.float64) - p
    fwd /= np.linalg.norm(fwd)
    up = np.array([0.0, -1.0, 0.0])
    if abs(np.dot(fwd, up)) > 0.999:
        up = np.array([0.0, 0.0, 1.0])
    right = np.cross(fwd, up)
    right /= np.linalg.norm(right)
    down = np.cross(fwd, right)
    R = np.stack([right, down, fwd])
    w2c = np.eye(4)
    w2c[:3, :3] = R
    w2c[:3, 3] = -R @ p
    return w2c.astype(np.float32)


def sphere_cameras(n_views: int, radius: float, f: float, width: int, height: int,
                   seed: int = 2) -> list[Camera]:
    rng = np.random.default_rng(seed)
    d = rng.standard_normal((n_views, 3))
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    K = intrinsics(f, width, height)
    return [Camera(look_at(radius * d[i]), K, height, width) for i in range(n_views)]


def c1_scene(n: int = 10_000, seed: int = 0) -> dict:
    """Display-path scene: activated params (means, scales, rotations, opacities, colors)
    as the reference's ``Gaussians`` holds them (gsplat/data_structures.py)."""
    rng = np.random.default_rng(seed)
    means = rng.uniform(-1.0, 1.0, (n, 3)).astype(np.float32)
    log_scales = rng.normal(-4.0, 0.5, (n, 3)).astype(np.float32)
    q = rng.standard_normal((n, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    logits = rng.standard_normal(n).astype(np.float32)
    colors = rng.uniform(0.0, 1.0, (n, 3)).astype(np.float32)
    return {
        "means": means,
        "scales": np.exp(log_scales).astype(np.float32),
        "rotations": q.astype(np.float32),
        "opacities": (1.0 / (1.0 + np.exp(-logits.astype(np.float64)))).astype(np.float32),
        "colors": colors,
    }


def c1_camera() -> Camera:
    w2c = np.eye(4, dtype=np.float32)
    w2c[2, 3] = 3.0  # camera centre at (0, 0, -3)
    return Camera(w2c, intrinsics(300.0, 256, 256), 256, 256)


def c2_pairs(n: int = 1 << 24, n_tiles: int = 8160, s: float = 1.1, seed: int = 0):
    """(keys uint64, values uint32) of the sort microbenchmark."""
    rng = np.random.default_rng(seed)
    r = np.arange(1, n_tiles + 1, dtype=np.float64)
    p = r ** (-s)
    p /= p.sum()
    perm = rng.permutation(n_tiles).astype(np.uint64)
    rank = rng.choice(n_tiles, size=n, p=p)
    tile = perm[rank]
    depth = rng.uniform(0.1, 50.0, n).astype(np.float32)
    keys = (tile << np.uint64(32)) | depth.view(np.uint32).astype(np.uint64)
    values = rng.permutation(n).astype(np.uint32)
    return keys, values


def cluster_scene(n: int, sh_degree: int = 3, seed: int = 0, n_clusters: int = 64) -> dict:
    """Optimizer-space training params of configs C3-C5 (fp32)."""
    rng = np.random.default_rng(seed)
    centres = rng.uniform(-2.0, 2.0, (n_clusters, 3))
    idx = rng.integers(0, n_clusters, n)
    means = (centres[idx] + 0.3 * rng.standard_normal((n, 3))).astype(np.float32)
    log_scales = rng.normal(-4.5, 0.7, (n, 3)).astype(np.float32)
    q = rng.standard_normal((n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    logits = rng.normal(0.0, 1.5, n).astype(np.float32)
    K = (sh_degree + 1) ** 2
    sh = np.empty((n, K, 3), np.float32)
    sh[:, 0] = rng.uniform(0.0, 1.0, (n, 3))
    if K > 1:
        sh[:, 1:] = rng.normal(0.0, 0.05, (n, K - 1, 3))
    return {"means": means, "log_scales": log_scales, "quats": q.astype(np.float32),
            "opacity_logits": logits, "sh": sh}


def random_targets(cams: list[Camera], seed: int = 1) -> list[np.ndarray]:
    rng = np.random.default_rng(seed)
    return [rng.uniform(0.0, 1.0, (c.height, c.width, 3)).astype(np.float32) for c in cams]


# Per-group Adam learning rates of configs[3] (C4; C5 uses the same): SH band 0 at 2.5e-3
# and bands 1-3 at 1/20 of it, as the reference's DEFAULT_LR (gsplat/train_oracle.py:422-423).
LR_BASELINE = {"means": 1.6e-4, "log_scales": 5e-3, "quats": 1e-3, "opacity_logits": 5e-2,
               "sh_dc": 2.5e-3, "sh_rest": 2.5e-3 / 20.0}

CONFIGS = {
    # name: (N, views, width, height, focal, radius, loss)
    "c3": dict(n=500_000, views=1, width=1024, height=1024, f=900.0, radius=4.0,
               ssim=False),
    "c4": dict(n=3_000_000, views=8, width=1600, height=1056, f=1300.0, radius=4.0,
               ssim=True),
    "c5": dict(n=6_000_000, views=32, width=1920, height=1080, f=1500.0, radius=5.0,
               ssim=True),
}


def training_cameras(name: str, views: int | None = None) -> list[Camera]:
    c = CONFIGS[name]
    v = c["views"] if views is None else views
    if name == "c3":
        K = intrinsics(c["f"], c["width"], c["height"])
        return [Camera(look_at((0.0, 0.0, -c["radius"])), K, c["height"], c["width"])]
    return sphere_cameras(v, c["radius"], c["f"], c["width"], c["height"])
