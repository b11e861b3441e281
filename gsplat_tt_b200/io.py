"""Scene and camera input formats: 3D-Gaussian-splatting `.ply` files and the reference's
camera JSON (`benchmarks/cameras_*.json`).

* `load_ply` reads a binary little-endian (or ASCII) PLY whose `vertex` element carries the
  usual splat properties (x y z, scale_0..2, rot_0..3, opacity, f_dc_0..2 and optionally
  f_rest_*) and returns them in the optimizer space the trainer uses: log-scales, raw
  quaternions (w, x, y, z), opacity logits, SH coefficients (N, K, 3). The reference's
  loader (gsplat/loading_gaussians.py:32-75) reads the same properties and reads the DC
  band only; `f_rest_*`, when present, are taken in the layout 3DGS writers use (all of
  channel 0's higher-band coefficients, then channel 1's, then channel 2's).
* `activate` applies the reference's activations for the display path
  (gsplat/loading_gaussians.py:7-29): scales = exp, unit quaternions,
  colour = clamp(0.5 + C0 * f_dc, 0, 1), opacity = sigmoid.
* `save_ply` writes the same layout (binary little-endian), e.g. after training.
* `load_cameras` turns one scene entry of a camera JSON into (w2c, K, H, W) tuples: OpenCV
  camera-to-world matrices (+z forward, +y down) inverted in closed form (R^T, -R^T t) as
  gsplat/utils.py:133-153 does, intrinsics from the entry's `intrinsics` block or, without
  one, from `fov_deg` over the longer image side (gsplat/viewer.py:190-200).

Host-side numpy only; nothing here touches the GPU.
"""
from __future__ import annotations

import json
import math
import re

import numpy as np

SH_C0 = 0.28209479177387814

_PLY_TYPES = {
    "char": "i1", "int8": "i1", "uchar": "u1", "uint8": "u1",
    "short": "i2", "int16": "i2", "ushort": "u2", "uint16": "u2",
    "int": "i4", "int32": "i4", "uint": "u4", "uint32": "u4",
    "float": "f4", "float32": "f4", "double": "f8", "float64": "f8",
}


def _read_header(f):
    if f.readline().strip() != b"ply":
        raise ValueError("not a PLY file")
    fmt = None
    elements = []  # (name, count, [(prop, dtype)])
    while True:
        line = f.readline()
        if not line:
            raise ValueError("PLY header not terminated")
        tok = line.decode("ascii", "replace").split()
        if not tok or tok[0] in ("comment", "obj_info"):
            continue
        if tok[0] == "format":
            fmt = tok[1]
        elif tok[0] == "element":
            elements.append((tok[1], int(tok[2]), []))
        elif tok[0] == "property":
            if tok[1] == "list":
                raise ValueError(f"PLY list property {tok[-1]!r} is not supported")
            if tok[1] not in _PLY_TYPES:
                raise ValueError(f"unknown PLY type {tok[1]!r}")
            elements[-1][2].append((tok[2], _PLY_TYPES[tok[1]]))
        elif tok[0] == "end_header":
            break
    if fmt not in ("binary_little_endian", "binary_big_endian", "ascii"):
        raise ValueError(f"unsupported PLY format {fmt!r}")
    return fmt, elements


def read_ply_vertices(path: str) -> dict[str, np.ndarray]:
    """Every property of the PLY's `vertex` element as a 1-D array."""
    with open(path, "rb") as f:
        fmt, elements = _read_header(f)
        out = None
        for name, count, props in elements:
            end = "<" if fmt == "binary_little_endian" else ">"
            dt = np.dtype([(p, end + t) for p, t in props])
            if fmt == "ascii":
                rows = [f.readline().split() for _ in range(count)]
                arr = np.array(rows, dtype=np.float64).reshape(count, len(props))
                data = {p: arr[:, i].astype(np.dtype(t)) for i, (p, t) in enumerate(props)}
            else:
                raw = np.frombuffer(f.read(dt.itemsize * count), dtype=dt, count=count)
                data = {p: np.asarray(raw[p]).astype(np.dtype(t).newbyteorder("=")) for p, t in props}
            if name == "vertex":
                out = data
                break
    if out is None:
        raise ValueError("PLY has no vertex element")
    return out


def load_ply(path: str) -> dict[str, np.ndarray]:
    """Optimizer-space parameters: means (N,3), log_scales (N,3), quats (N,4) w x y z,
    opacity_logits (N,), sh (N,K,3) float32 (K = 1 + number of f_rest per channel)."""
    v = read_ply_vertices(path)
    need = ["x", "y", "z", "scale_0", "scale_1", "scale_2", "rot_0", "rot_1", "rot_2", "rot_3",
            "opacity", "f_dc_0", "f_dc_1", "f_dc_2"]
    missing = [k for k in need if k not in v]
    if missing:
        raise ValueError(f"PLY vertex element lacks {missing}")
    f32 = lambda *ks: np.stack([v[k] for k in ks], axis=-1).astype(np.float32)  # noqa: E731
    n = v["x"].shape[0]
    rest_keys = sorted((k for k in v if re.fullmatch(r"f_rest_\d+", k)), key=lambda k: int(k[7:]))
    if len(rest_keys) % 3:
        raise ValueError(f"{len(rest_keys)} f_rest properties is not a multiple of 3")
    per_ch = len(rest_keys) // 3
    K = 1 + per_ch
    if int(round(math.sqrt(K))) ** 2 != K:
        raise ValueError(f"{K} SH coefficients per channel is not a full degree")
    sh = np.zeros((n, K, 3), np.float32)
    sh[:, 0, :] = f32("f_dc_0", "f_dc_1", "f_dc_2")
    if per_ch:
        rest = f32(*rest_keys).reshape(n, 3, per_ch)  # channel-major
        sh[:, 1:, :] = np.transpose(rest, (0, 2, 1))
    return {
        "means": f32("x", "y", "z"),
        "log_scales": f32("scale_0", "scale_1", "scale_2"),
        "quats": f32("rot_0", "rot_1", "rot_2", "rot_3"),
        "opacity_logits": v["opacity"].astype(np.float32),
        "sh": sh,
    }


def save_ply(path: str, params: dict[str, np.ndarray]) -> None:
    """Write optimizer-space parameters in the layout `load_ply` reads."""
    means = np.asarray(params["means"], np.float32)
    n = means.shape[0]
    sh = np.asarray(params["sh"], np.float32).reshape(n, -1, 3)
    per_ch = sh.shape[1] - 1
    cols = [("x", means[:, 0]), ("y", means[:, 1]), ("z", means[:, 2])]
    cols += [(f"f_dc_{c}", sh[:, 0, c]) for c in range(3)]
    rest = np.transpose(sh[:, 1:, :], (0, 2, 1)).reshape(n, 3 * per_ch)
    cols += [(f"f_rest_{i}", rest[:, i]) for i in range(3 * per_ch)]
    cols += [("opacity", np.asarray(params["opacity_logits"], np.float32).reshape(n))]
    ls = np.asarray(params["log_scales"], np.float32)
    cols += [(f"scale_{i}", ls[:, i]) for i in range(3)]
    q = np.asarray(params["quats"], np.float32)
    cols += [(f"rot_{i}", q[:, i]) for i in range(4)]
    dt = np.dtype([(k, "<f4") for k, _ in cols])
    rec = np.empty(n, dtype=dt)
    for k, a in cols:
        rec[k] = a
    header = ["ply", "format binary_little_endian 1.0", f"element vertex {n}"]
    header += [f"property float {k}" for k, _ in cols]
    header += ["end_header"]
    with open(path, "wb") as f:
        f.write(("\n".join(header) + "\n").encode("ascii"))
        f.write(rec.tobytes())


def activate(params: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """The reference's display activations: scales, unit quaternions, colours in [0, 1] from
    the DC band, opacities in (0, 1)."""
    q = np.asarray(params["quats"], np.float32)
    sh = np.asarray(params["sh"], np.float32)
    return {
        "means": np.asarray(params["means"], np.float32),
        "scales": np.exp(np.asarray(params["log_scales"], np.float32)),
        "rotations": (q / np.linalg.norm(q, axis=-1, keepdims=True)).astype(np.float32),
        "colors": np.clip(np.float32(0.5) + np.float32(SH_C0) * sh[:, 0, :], 0.0, 1.0).astype(np.float32),
        "opacities": (1.0 / (1.0 + np.exp(-np.asarray(params["opacity_logits"], np.float32)))).astype(np.float32),
    }


def intrinsics_from_fov(width: int, height: int, fov_deg: float) -> np.ndarray:
    """Square-pixel K with the field of view over the longer image side, principal point
    at the image centre."""
    f = 0.5 * max(width, height) / math.tan(0.5 * math.radians(fov_deg))
    return np.array([[f, 0.0, width * 0.5], [0.0, f, height * 0.5], [0.0, 0.0, 1.0]], np.float32)


def c2w_to_w2c(c2w) -> np.ndarray:
    """Closed-form inverse of a rigid camera-to-world matrix, float32 (4, 4)."""
    c2w = np.asarray(c2w, np.float64)
    if c2w.shape != (4, 4):
        raise ValueError(f"c2w must be 4x4, got {c2w.shape}")
    R, t = c2w[:3, :3], c2w[:3, 3]
    w2c = np.eye(4, dtype=np.float32)
    w2c[:3, :3] = R.T
    w2c[:3, 3] = -R.T @ t
    return w2c


def load_cameras(path: str, scene: str | None = None, views=None):
    """(w2c, K, H, W) per view of one scene entry, in the entry's `order` (or every view).

    scene: the entry's key (default: the only / first entry). views: optional list of view
    names to keep, in that order."""
    with open(path) as f:
        cat = json.load(f)
    if not isinstance(cat, dict) or not cat:
        raise ValueError("camera file must map scene names to entries")
    if scene is None:
        scene = next(iter(cat))
    if scene not in cat:
        raise KeyError(f"scene {scene!r} not in {sorted(cat)}")
    e = cat[scene]
    W, H = (int(x) for x in e["image_size"])
    if "intrinsics" in e:
        i = e["intrinsics"]
        K = np.array([[i["fx"], 0.0, i["cx"]], [0.0, i["fy"], i["cy"]], [0.0, 0.0, 1.0]], np.float32)
    else:
        K = intrinsics_from_fov(W, H, float(e.get("fov_deg", 50.0)))
    names = list(views) if views is not None else list(e.get("order") or e["views"].keys())
    out = []
    for name in names:
        if name not in e["views"]:
            raise KeyError(f"view {name!r} not in scene {scene!r}")
        out.append((c2w_to_w2c(e["views"][name]["c2w"]), K.copy(), H, W))
    return out
