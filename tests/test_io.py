"""Scene / camera input formats (host only): PLY round trip, the reference's activations,
and camera JSON parsing in the reference's `benchmarks/cameras_*.json` layout."""
import json
import math

import numpy as np
import pytest

from gsplat_tt_b200 import io, scenes


def test_ply_round_trip_sh3(tmp_path):
    params = scenes.cluster_scene(1000, sh_degree=3, seed=4)
    p = tmp_path / "s.ply"
    io.save_ply(str(p), params)
    back = io.load_ply(str(p))
    for k in ("means", "log_scales", "quats", "opacity_logits"):
        np.testing.assert_array_equal(back[k], np.asarray(params[k], np.float32))
    np.testing.assert_array_equal(back["sh"], np.asarray(params["sh"], np.float32).reshape(1000, 16, 3))


def test_ply_dc_only_and_rest_layout(tmp_path):
    """f_rest_* are channel-major: rest index c * (K - 1) + (k - 1) is band k of channel c."""
    n = 3
    props = ["x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2"] + [f"f_rest_{i}" for i in range(9)] + \
        ["opacity", "scale_0", "scale_1", "scale_2", "rot_0", "rot_1", "rot_2", "rot_3"]
    vals = np.arange(n * len(props), dtype=np.float32).reshape(n, len(props))
    header = "ply\nformat binary_little_endian 1.0\ncomment test\nelement vertex 3\n" + \
        "".join(f"property float {q}\n" for q in props) + "end_header\n"
    p = tmp_path / "r.ply"
    p.write_bytes(header.encode() + vals.astype("<f4").tobytes())
    d = io.load_ply(str(p))
    assert d["sh"].shape == (3, 4, 3)
    col = {q: i for i, q in enumerate(props)}
    for c in range(3):
        assert d["sh"][1, 0, c] == vals[1, col[f"f_dc_{c}"]]
        for k in range(1, 4):
            assert d["sh"][1, k, c] == vals[1, col[f"f_rest_{c * 3 + (k - 1)}"]]
    np.testing.assert_array_equal(d["quats"][2], vals[2, [col[f"rot_{i}"] for i in range(4)]])


def test_ply_ascii_and_errors(tmp_path):
    p = tmp_path / "a.ply"
    props = ["x", "y", "z", "scale_0", "scale_1", "scale_2", "rot_0", "rot_1", "rot_2", "rot_3",
             "opacity", "f_dc_0", "f_dc_1", "f_dc_2"]
    p.write_text("ply\nformat ascii 1.0\nelement vertex 1\n" +
                 "".join(f"property float {q}\n" for q in props) + "end_header\n" +
                 " ".join(str(float(i)) for i in range(len(props))) + "\n")
    d = io.load_ply(str(p))
    assert d["means"].tolist() == [[0.0, 1.0, 2.0]] and d["sh"].shape == (1, 1, 3)
    bad = tmp_path / "b.ply"
    bad.write_text("ply\nformat ascii 1.0\nelement vertex 1\nproperty float x\nend_header\n0\n")
    with pytest.raises(ValueError):
        io.load_ply(str(bad))


def test_activate_matches_reference_rules():
    params = scenes.cluster_scene(200, sh_degree=0, seed=1)
    a = io.activate(params)
    np.testing.assert_allclose(a["scales"], np.exp(params["log_scales"]), rtol=1e-6)
    np.testing.assert_allclose(np.linalg.norm(a["rotations"], axis=1), 1.0, rtol=1e-6)
    dc = np.asarray(params["sh"], np.float32).reshape(200, -1, 3)[:, 0, :]
    np.testing.assert_allclose(a["colors"], np.clip(0.5 + io.SH_C0 * dc, 0, 1), rtol=1e-6)
    assert a["opacities"].min() > 0 and a["opacities"].max() < 1


def test_load_cameras_json(tmp_path):
    rng = np.random.default_rng(0)
    Q, _ = np.linalg.qr(rng.standard_normal((3, 3)))
    c2w = np.eye(4)
    c2w[:3, :3] = Q
    c2w[:3, 3] = [1.0, -2.0, 3.0]
    cat = {"bicycle": {"ply": "scenes/bicycle.ply", "image_size": [1237, 822],
                       "fov_deg": 56.0, "intrinsics": {"fx": 1162.8, "fy": 1157.5, "cx": 618.5, "cy": 411.0},
                       "order": ["b", "a"],
                       "views": {"a": {"c2w": np.eye(4).tolist()}, "b": {"c2w": c2w.tolist()}}}}
    p = tmp_path / "cams.json"
    p.write_text(json.dumps(cat))
    cams = io.load_cameras(str(p))
    assert [c[2:] for c in cams] == [(822, 1237), (822, 1237)]
    w2c, K, H, W = cams[0]
    np.testing.assert_allclose(w2c @ c2w, np.eye(4), atol=1e-6)
    assert K[0, 0] == np.float32(1162.8) and K[1, 2] == np.float32(411.0)
    # without an intrinsics block: fov over the longer side, centred principal point
    del cat["bicycle"]["intrinsics"]
    p.write_text(json.dumps(cat))
    _, K2, _, _ = io.load_cameras(str(p), views=["a"])[0]
    f = 0.5 * 1237 / math.tan(math.radians(28.0))
    np.testing.assert_allclose(K2, [[f, 0, 618.5], [0, f, 411.0], [0, 0, 1]], rtol=1e-6)
    with pytest.raises(KeyError):
        io.load_cameras(str(p), views=["missing"])
