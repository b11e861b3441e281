"""ctypes binding of libgs200.so (the C ABI declared in include/gs200.h).

The product path has no fallback: if the library is missing or fails to load,
importing this module raises ImportError. Build it with
``python -m gsplat_tt_b200.build`` (``__graft_entry__.build()`` does the same).
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgs200.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"libgs200.so not found at {LIB_PATH}; build it with "
                      "`python -m gsplat_tt_b200.build`")
try:
    lib = ctypes.CDLL(LIB_PATH)
except OSError as exc:  # pragma: no cover - depends on the host
    raise ImportError(f"cannot load {LIB_PATH}: {exc}") from exc

GS_OK, GS_ERR_ARG, GS_ERR_OVERFLOW, GS_ERR_CUDA, GS_ERR_TIMEOUT, GS_ERR_UNSUPPORTED = range(6)

vp = ctypes.c_void_p
i64 = ctypes.c_int64
i32 = ctypes.c_int32
f32 = ctypes.c_float
sz = ctypes.c_size_t
status = ctypes.c_int


class GsError(RuntimeError):
    """A libgs200 call failed; ``code`` is the gs_status value."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"gs200 error {code}: {msg}")
        self.code = code


class GsOverflow(GsError):
    """A data-dependent output exceeded the caller's capacity (GS_ERR_OVERFLOW)."""


def _sig(name, restype, *argtypes):
    fn = getattr(lib, name)
    fn.restype = restype
    fn.argtypes = list(argtypes)
    return fn


_sig("gs_last_error", ctypes.c_char_p)
_sig("gs_version", ctypes.c_char_p)
_sig("gs_workspace_error", status, vp, vp)
_sig("gs_debug_logf_host", status, vp, vp, i64, vp)
_sig("gs_compute_cov3d", status, vp, vp, i64, vp, vp)
_sig("gs_project", status, vp, vp, vp, vp, vp, vp, f32, i64, i32, i32, i32, f32, f32, i32,
     vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, sz, vp)
_sig("gs_project_workspace_size", sz, i64)
_sig("gs_project_noalloc", status, vp, vp, vp, vp, vp, vp, f32, i64, i32, i32, i32, f32, f32, i32,
     vp, vp, vp, vp, vp, vp, vp, vp, vp, vp)
_sig("gs_tile_assign", status, vp, vp, i64, i32, i32, i32, vp, vp, f32, vp, vp, i64, vp, vp,
     vp, vp, sz, vp)
_sig("gs_tile_assign_workspace_size", sz, i64, i64)
_sig("gs_sort_and_bin", status, vp, vp, vp, i64, i32, i32, vp, vp, vp, sz, vp)
_sig("gs_sort_and_bin_workspace_size", sz, i64, i32, i32)
_sig("gs_sort_pairs", status, vp, vp, i64, i32, vp, vp, vp, sz, vp)
_sig("gs_sort_pairs_workspace_size", sz, i64, i32)
_sig("gs_launch_count", i64)
_sig("gs_timing_enable", None, i32)
_sig("gs_timing_reset", None)
_sig("gs_timing_report", i32, ctypes.c_char_p, sz, ctypes.POINTER(ctypes.c_double),
     ctypes.POINTER(i64), i32)
_sig("gs_blend", status, vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, vp, vp, vp)
_sig("gs_cull_and_blend_workspace_size", sz, i64)
_sig("gs_cull_and_blend", status, vp, vp, vp, vp, vp, vp, i64, i64, i32, i32, i32, i32, i32, f32,
     i32, f32, vp, vp, vp, sz, vp)


def check(code: int) -> None:
    """Raise for a non-zero gs_status, with the library's message. Shape errors map to
    ValueError as the reference's pybind layer raises std::invalid_argument."""
    if code == GS_OK:
        return
    msg = lib.gs_last_error().decode(errors="replace")
    if code == GS_ERR_ARG:
        raise ValueError(msg)
    if code == GS_ERR_OVERFLOW:
        raise GsOverflow(code, msg)
    raise GsError(code, msg)


def version() -> str:
    return lib.gs_version().decode()


def timing_report(max_kernels: int = 64) -> dict[str, tuple[float, int]]:
    """{kernel name: (total ms, launches)} recorded since gs_timing_reset()."""
    names = ctypes.create_string_buffer(8192)
    tot = (ctypes.c_double * max_kernels)()
    cnt = (i64 * max_kernels)()
    k = lib.gs_timing_report(names, 8192, tot, cnt, max_kernels)
    keys = names.value.decode().split("\n")[:k]
    return {keys[i]: (tot[i], int(cnt[i])) for i in range(k)}
