"""gs_project_noalloc, the projection entry point for callers that cannot allocate device
memory (a plug-in inside an application that owns all device buffers, or a real-time loop
that may not call the synchronising cudaMalloc): it keeps its scratch in a fixed array
inside the library instead of a caller workspace.

Checked through the C ABI against gs_project on two calls in a row with different scene
sizes (the second call reuses the shared array the first one left behind); the results
must be identical, the bar every projection test uses. Collected last on purpose, so a run
that stops at its first failure has run every other test before this one."""
import ctypes

import numpy as np
import pytest

from gsplat_tt_b200 import scenes

pytestmark = pytest.mark.gpu


def _project(lib, name, means, cov3d, w2c, K, opac, cols, H, W):
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    n = means.shape[0]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
    m, c3, op, col = t(means), t(cov3d.reshape(n, 9)), t(opac), t(cols)
    out = {"m2": torch.empty((n, 2), device=dev), "cov": torch.empty((n, 4), device=dev),
           "depth": torch.empty(n, device=dev), "radii": torch.empty((n, 2), device=dev),
           "valid": torch.empty(n, dtype=torch.uint8, device=dev),
           "col": torch.empty((n, 3), device=dev), "op": torch.empty(n, device=dev)}
    nv = torch.empty(1, dtype=torch.int64, device=dev)
    e = np.ascontiguousarray(w2c, np.float32).reshape(16)
    k = np.ascontiguousarray(K, np.float32).reshape(9)
    host_m = ctypes.c_int64(-1)
    st = torch.cuda.current_stream().cuda_stream
    common = [m.data_ptr(), c3.data_ptr(), e.ctypes.data, k.ctypes.data, col.data_ptr(),
              op.data_ptr(), 1.0 / 255.0, n, H, W, 0, 1.0 / 16384.0, 3.0, 0,
              out["m2"].data_ptr(), out["cov"].data_ptr(), out["depth"].data_ptr(),
              out["radii"].data_ptr(), out["valid"].data_ptr(), out["col"].data_ptr(),
              out["op"].data_ptr(), nv.data_ptr(), ctypes.addressof(host_m)]
    if name == "gs_project":
        ws = torch.empty(lib.gs_project_workspace_size(n), dtype=torch.uint8, device=dev)
        code = lib.gs_project(*common, ws.data_ptr(), ws.numel(), st)
    else:
        code = lib.gs_project_noalloc(*common, st)
    assert code == 0, lib.gs_last_error()
    M = host_m.value
    res = {k_: v[:M].cpu().numpy() for k_, v in out.items() if k_ != "valid"}
    res["valid"] = out["valid"].cpu().numpy()
    res["M"] = M
    return res


def _scene(n, seed, H, W):
    from oracle import display as od
    sc = scenes.c1_scene(n=n, seed=seed)
    cam = scenes.c1_camera()
    K = scenes.intrinsics(300.0 * W / 256.0, W, H)
    return sc, od.compute_cov3d(sc["scales"], sc["rotations"]), cam.w2c, K


def test_noalloc_projection_matches_gs_project_on_two_calls_in_a_row():
    from gsplat_tt_b200._lib import lib
    for n, seed, H, W in ((10_000, 0, 256, 256), (3_001, 5, 100, 37)):
        sc, cov3d, w2c, K = _scene(n, seed, H, W)
        ref = _project(lib, "gs_project", sc["means"], cov3d, w2c, K, sc["opacities"],
                       sc["colors"], H, W)
        got = _project(lib, "gs_project_noalloc", sc["means"], cov3d, w2c, K, sc["opacities"],
                       sc["colors"], H, W)
        assert got["M"] == ref["M"] > 0
        for key in ("m2", "cov", "depth", "radii", "valid", "col", "op"):
            np.testing.assert_array_equal(got[key], ref[key], err_msg=key)


def test_noalloc_projection_rejects_more_gaussians_than_its_scratch_holds():
    from gsplat_tt_b200._lib import lib
    e = (ctypes.c_float * 16)()
    k = (ctypes.c_float * 9)()
    code = lib.gs_project_noalloc(None, None, e, k, None, None, 0.0, (1 << 24) + 1, 8, 8, 0,
                                  1e-4, 3.0, 0, None, None, None, None, None, None, None, None,
                                  None, None)
    assert code == 1  # GS_ERR_ARG
    assert b"at most 16777216" in lib.gs_last_error()
    # the same checks in the same order as gs_project: the unsupported option first, then
    # a negative size as a bad size
    code = lib.gs_project_noalloc(None, None, e, k, None, None, 0.0, (1 << 24) + 1, 8, 8, 0,
                                  1e-4, 3.0, 1, None, None, None, None, None, None, None, None,
                                  None, None)
    assert code == 5  # GS_ERR_UNSUPPORTED
    code = lib.gs_project_noalloc(None, None, e, k, None, None, 0.0, -1, 8, 8, 0, 1e-4, 3.0, 0,
                                  None, None, None, None, None, None, None, None, None, None)
    assert code == 1 and b"bad sizes" in lib.gs_last_error()
