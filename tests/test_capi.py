"""libgs200.so host-side checks that need no GPU: it loads, exports every entry point
include/gs200.h declares, sizes workspaces, and rejects bad arguments before touching
the device (the reference's std::invalid_argument cases map to GS_ERR_ARG)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            text = open(os.path.join(ROOT, "include", f)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(gs_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "gs_sort_pairs" in names and "gs_project" in names and len(names) >= 10


def test_library_exports_every_declared_symbol():
    from gsplat_tt_b200 import _lib
    missing = [n for n in declared_symbols() if not hasattr(_lib.lib, n)]
    assert not missing, missing
    assert _lib.version().startswith("gs200")


def test_workspace_queries():
    from gsplat_tt_b200._lib import lib
    assert lib.gs_sort_pairs_workspace_size(1 << 24, 45) > (1 << 24) * 24
    assert lib.gs_project_workspace_size(10000) > 0
    assert lib.gs_tile_assign_workspace_size(10000, 1 << 20) > (1 << 20) * 8
    assert lib.gs_sort_and_bin_workspace_size(1000, 16, 16) > 1000 * 24


def test_argument_errors_need_no_device():
    from gsplat_tt_b200._lib import lib, GS_ERR_ARG, GS_ERR_UNSUPPORTED
    assert lib.gs_sort_pairs(None, None, -1, 45, None, None, None, 0, None) == GS_ERR_ARG
    assert b"n must be" in lib.gs_last_error()
    assert lib.gs_sort_pairs(None, None, 10, 0, None, None, None, 0, None) == GS_ERR_ARG
    assert lib.gs_blend(None, None, None, None, None, None, 0, 64, 64, 33, None, None,
                        None) == GS_ERR_ARG
    e = (ctypes.c_float * 16)()
    k = (ctypes.c_float * 9)()
    assert lib.gs_project(None, None, e, k, None, None, 0.0, 0, 8, 8, 0, 1e-4, 3.0, 1,
                          None, None, None, None, None, None, None, None, None, None, 0,
                          None) == GS_ERR_UNSUPPORTED
    assert lib.gs_tile_assign(None, None, 0, 8, 8, 16, ctypes.c_void_p(1), None, 0.0, None,
                              None, 0, None, ctypes.c_void_p(1), None, None, 0,
                              None) == GS_ERR_ARG


def test_product_path_fails_loudly_without_library(tmp_path, monkeypatch):
    import gsplat_tt_b200._lib as L
    monkeypatch.setattr(L, "LIB_PATH", str(tmp_path / "missing.so"))
    src = open(L.__file__).read()
    ns = {"__file__": str(tmp_path / "_lib.py"), "__name__": "x"}
    with pytest.raises(ImportError):
        exec(compile(src, "x", "exec"), ns)
    # the module itself is untouched (the copy ran in its own namespace): no reload, which
    # would replace the library handle whose signatures other modules have declared


def test_training_update_argument_errors_need_no_device():
    """The row-range projection backward and the multicast update reject bad arguments on
    the host (no device call is made before the checks)."""
    from gsplat_tt_b200._lib import GS_ERR_ARG
    from gsplat_tt_b200.train import GsCamera, GsGaussians, TrainConfig, camera_struct, lib
    import numpy as np
    cfg = TrainConfig(sh_degree=3).c_struct()
    g = GsGaussians(16, 16, 16, 16, 16)  # fake aligned addresses: never dereferenced
    cams = (GsCamera * 1)(camera_struct(np.eye(4), np.eye(3), 64, 64))
    ws = ctypes.c_void_p(256)
    # rows outside [0, n)
    assert lib.gs_train_param_backward(ctypes.byref(g), ctypes.byref(g), 100, 50, 101, cams, 1,
                                       ctypes.byref(cfg), 1000, ws, 1 << 30, None) == GS_ERR_ARG
    assert b"outside" in lib.gs_last_error()
    assert lib.gs_train_param_backward(ctypes.byref(g), ctypes.byref(g), 100, 60, 50, cams, 1,
                                       ctypes.byref(cfg), 1000, ws, 1 << 30, None) == GS_ERR_ARG
    # workspace too small for the layout
    assert lib.gs_train_param_backward(ctypes.byref(g), ctypes.byref(g), 100, 0, 100, cams, 1,
                                       ctypes.byref(cfg), 1000, ws, 16, None) == GS_ERR_ARG
    assert b"workspace" in lib.gs_last_error()
    # multicast update: rows must be a multiple of 4, pointers 16-byte aligned
    skip = ctypes.c_void_p(16)
    args = [ctypes.byref(g)] * 5
    assert lib.gs_sparse_adam_multicast(*args, ctypes.c_void_p(16), ctypes.c_void_p(16), 6, 0,
                                        ctypes.byref(cfg), skip, None) == GS_ERR_ARG
    assert b"multiple of 4" in lib.gs_last_error()
    bad = GsGaussians(16, 16, 20, 16, 16)
    assert lib.gs_sparse_adam_multicast(ctypes.byref(bad), *args[1:], ctypes.c_void_p(16),
                                        ctypes.c_void_p(16), 8, 0, ctypes.byref(cfg), skip,
                                        None) == GS_ERR_ARG
    assert b"16-byte" in lib.gs_last_error()
    # a deferred step mode outside {0, 1, 2}
    tg = (ctypes.c_void_p * 1)(16)
    assert lib.gs_train_step(ctypes.byref(g), ctypes.byref(g), ctypes.byref(g), ctypes.byref(g),
                             ctypes.c_void_p(16), 100, 0, cams, tg, 1, ctypes.byref(cfg), 3,
                             ctypes.c_void_p(16), None, None, None, 1000, ws, 1 << 30,
                             None) == GS_ERR_ARG


def test_stage_entry_points_argument_errors_need_no_device():
    """gs_render_fwd / gs_loss / gs_render_bwd check their arguments and workspace sizes on
    the host before any device call."""
    from gsplat_tt_b200._lib import GS_ERR_ARG
    from gsplat_tt_b200.train import GsGaussians, TrainConfig, camera_struct, lib
    import numpy as np
    cfg = TrainConfig(sh_degree=3).c_struct()
    g = GsGaussians(16, 16, 16, 16, 16)
    cam = camera_struct(np.eye(4), np.eye(3), 64, 64)
    ws = ctypes.c_void_p(256)
    p = ctypes.c_void_p(16)
    assert lib.gs_render_fwd(None, 100, ctypes.byref(cam), ctypes.byref(cfg), p, None, None, None,
                             None, 1000, ws, 1 << 30, None) == GS_ERR_ARG
    assert lib.gs_render_fwd(ctypes.byref(g), 100, ctypes.byref(cam), ctypes.byref(cfg), p, None,
                             None, None, None, 1000, ws, 16, None) == GS_ERR_ARG
    assert b"workspace too small" in lib.gs_last_error()
    bad = GsGaussians(16, 16, 20, 16, 16)
    assert lib.gs_render_fwd(ctypes.byref(bad), 100, ctypes.byref(cam), ctypes.byref(cfg), p, None,
                             None, None, None, 1000, ws, 1 << 30, None) == GS_ERR_ARG
    assert b"16-byte" in lib.gs_last_error()
    big = camera_struct(np.eye(4), np.eye(3), 64, 70000 * 16)
    assert lib.gs_render_bwd(100, ctypes.byref(big), ctypes.byref(cfg), p, None, 1000, ws, 1 << 30,
                             None) == GS_ERR_ARG
    assert lib.gs_render_bwd(100, ctypes.byref(cam), ctypes.byref(cfg), None, None, 1000, ws,
                             1 << 30, None) == GS_ERR_ARG
    assert lib.gs_loss_workspace_size(64, 64) >= 3 * 64 * 64 * 3 * 4
    assert lib.gs_loss(p, p, 64, 64, ctypes.byref(cfg), p, p, ws, 16, None) == GS_ERR_ARG
    assert b"workspace too small" in lib.gs_last_error()
    assert lib.gs_loss(p, None, 64, 64, ctypes.byref(cfg), p, p, ws, 1 << 30, None) == GS_ERR_ARG


def test_deterministic_mode_checks_and_workspace_need_no_device():
    """deterministic = 1 asks for 16x16 tiles (GS_ERR_UNSUPPORTED with 32) and a workspace
    with one 48-byte slot per pair and one 8-byte offset per Gaussian in every lane; the
    workspace before the slots is the default layout, and a default-sized workspace is
    rejected on the host before any device call."""
    from gsplat_tt_b200._lib import GS_ERR_ARG, GS_ERR_UNSUPPORTED
    from gsplat_tt_b200.train import GsCamera, GsGaussians, TrainConfig, camera_struct, lib
    import numpy as np
    n, cap, H, W = 1000, 50000, 64, 64
    for views, lanes in ((1, 1), (3, 3), (9, 4)):
        base = lib.gs_train_workspace_size(n, 3, views, H, W, 16, cap)
        det = lib.gs_train_deterministic_workspace_size(n, 3, views, H, W, 16, cap)
        extra = det - base
        assert lanes * (cap * 48 + n * 8) <= extra <= lanes * (cap * 48 + n * 8 + 2 * 256)
        assert TrainConfig(deterministic=True).workspace_size(n, views, H, W, cap) == det
        assert TrainConfig().workspace_size(n, views, H, W, cap) == base
    g = GsGaussians(16, 16, 16, 16, 16)  # fake aligned addresses: never dereferenced
    cams = (GsCamera * 1)(camera_struct(np.eye(4), np.eye(3), H, W))
    tg = (ctypes.c_void_p * 1)(16)
    ws = ctypes.c_void_p(256)

    def step(cfg, ws_bytes):
        return lib.gs_train_step(ctypes.byref(g), ctypes.byref(g), ctypes.byref(g),
                                 ctypes.byref(g), ctypes.c_void_p(16), n, 0, cams, tg, 1,
                                 ctypes.byref(cfg), 1, ctypes.c_void_p(16), None, None, None, cap,
                                 ws, ws_bytes, None)
    assert step(TrainConfig(tile_size=32, deterministic=True).c_struct(), 1 << 40) == GS_ERR_UNSUPPORTED
    assert b"tile_size 16" in lib.gs_last_error()
    bad = TrainConfig().c_struct()
    bad.deterministic = 2
    assert step(bad, 1 << 40) == GS_ERR_ARG
    assert b"deterministic" in lib.gs_last_error()
    base = lib.gs_train_workspace_size(n, 3, 1, H, W, 16, cap)
    assert step(TrainConfig(deterministic=True).c_struct(), base) == GS_ERR_ARG
    assert b"workspace too small" in lib.gs_last_error()
    cam = camera_struct(np.eye(4), np.eye(3), H, W)
    assert lib.gs_render_bwd(n, ctypes.byref(cam), ctypes.byref(TrainConfig(deterministic=True).c_struct()),
                             ctypes.c_void_p(16), None, cap, ws, base, None) == GS_ERR_ARG
    assert b"workspace too small" in lib.gs_last_error()
