"""``b200`` backend: the reference's Backend plugin interface served by libgs200.

Mirrors gsplat/backend.py:41-158 (project / tile_assign / sort / blend / close) and the
optional fused fast path the Pipeline probes (gsplat/pipeline.py:149-182:
has_render_fused / render_fused), with the same argument names, defaults, return
shapes and error behaviour. When the reference's ``gsplat`` package is importable the
class subclasses its ``Backend`` ABC, so ``backends.REGISTRY["b200"] = B200Backend``
(backends/__init__.py:20-60) drops it into the reference's Pipeline and viewer; without
it a local stand-in with the same abstract interface is used.

Stage outputs are returned on the device of the stage's first input (CPU tensors in,
CPU tensors out, as the reference's backends return), and every call synchronises
before returning, as the ABC requires of asynchronous backends
(gsplat/backend.py:25-29).
"""
from __future__ import annotations

import numpy as np
import torch

from . import display as _d

try:  # the reference's plugin ABC, when its package is on the path
    from gsplat.backend import Backend as _BackendBase  # type: ignore
except Exception:  # pragma: no cover - the reference is optional at run time
    from abc import ABC, abstractmethod

    class _BackendBase(ABC):  # same abstract surface as gsplat/backend.py:41-158
        @abstractmethod
        def blend(self, means_2d, covs_2d, colors, opacities, sorted_gaussian_ids,
                  tile_ranges, image_height, image_width):
            ...

        def close(self) -> None:
            """Release any resources held by the backend."""


def _like(t: torch.Tensor, ref) -> torch.Tensor:
    dev = ref.device if isinstance(ref, torch.Tensor) else torch.device("cpu")
    return t.to(dev)


class B200Backend(_BackendBase):
    """All four display stages on the B200, plus the one-call fused render."""

    def __init__(self, tile_size: int = 32, render_fused: bool = True,
                 cull_disabled: bool = False, min_opacity: float = 1.0 / 255.0,
                 max_radius: int = 0, contrib_floor: float | None = None,
                 k_cap: float = 3.0, use_isoellipse: bool = False,
                 transmittance_threshold: float = 1.0 / 255.0,
                 mb_contrib_floor: float = 1.0 / 16384.0, verbose: bool = False):
        if not torch.cuda.is_available():
            raise RuntimeError("B200Backend needs a CUDA device")
        self.tile_size = int(tile_size)
        self._render_fused = bool(render_fused)
        # Knobs the Pipeline pushes into fused backends (gsplat/pipeline.py:91-110).
        self.cull_disabled = bool(cull_disabled)
        self.min_opacity = float(min_opacity)
        self.max_radius = int(max_radius)
        self.contrib_floor_override = contrib_floor
        self.k_cap = float(k_cap)
        self.use_isoellipse = bool(use_isoellipse)
        self.transmittance_threshold = float(transmittance_threshold)
        self._mb_contrib_floor = float(mb_contrib_floor)
        self.verbose = verbose
        self._cov3d_key = None
        self._cov3d = None

    # -------------------------------------------------------------- stages

    def _cached_cov3d(self, scales, rotations) -> torch.Tensor:
        key = (getattr(scales, "data_ptr", lambda: id(scales))(), tuple(scales.shape),
               getattr(rotations, "data_ptr", lambda: id(rotations))(), tuple(rotations.shape))
        if key != self._cov3d_key:
            self._cov3d = _d.compute_cov3d(scales, rotations)
            self._cov3d_key = key
        return self._cov3d

    def project(self, means, scales, rotations, extrinsics, intrinsics, image_height,
                image_width, opacities=None, sub_timings=None):
        """(means_2d, covs_2d (M,2,2), depths, radii, valid_mask): project_full_with_cov3d
        with the CPU C++ backend's settings (min_opacity 1/255, k cap 3,
        backends/cpu_cpp/backend.py:142-154)."""
        del sub_timings
        cov3d = self._cached_cov3d(scales, rotations)
        m2, cv, d, r, v = _d.project_full_with_cov3d(
            means, cov3d, extrinsics, intrinsics, image_height, image_width, opacities,
            self.min_opacity, max_radius=self.max_radius, k_cap=self.k_cap)
        torch.cuda.synchronize()
        return tuple(_like(t, means) for t in (m2, cv, d, r, v))

    def tile_assign(self, means_2d, radii, image_height, image_width, tile_size=32,
                    covs_2d=None, opacities=None, contrib_floor=1.0 / 16384.0,
                    sub_timings=None):
        del sub_timings
        if self.cull_disabled:
            covs_2d, opacities = None, None
        g, t, n = _d.tile_assign(means_2d, radii, image_height, image_width, tile_size,
                                 covs_2d, opacities, contrib_floor)
        torch.cuda.synchronize()
        return tuple(_like(x, means_2d) for x in (g, t, n))

    def sort(self, gaussian_ids, tile_ids, depths, tiles_x, tiles_y, sub_timings=None):
        del sub_timings
        s, r = _d.sort(gaussian_ids, tile_ids, depths, tiles_x, tiles_y)
        torch.cuda.synchronize()
        return _like(s, gaussian_ids), _like(r, gaussian_ids)

    def blend(self, means_2d, covs_2d, colors, opacities, sorted_gaussian_ids, tile_ranges,
              image_height, image_width):
        """(H,W,3) float32 numpy image and {"kernel": ms}. The tile size is derived from
        tile_ranges (the Pipeline sorts with its own tile size)."""
        n_tiles = int(tile_ranges.shape[0])
        ts = self._tile_size_for(n_tiles, image_height, image_width)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        img = _d.blend(means_2d, covs_2d.reshape(-1, 4) if covs_2d.dim() == 3 else covs_2d,
                       colors, opacities, sorted_gaussian_ids, tile_ranges, image_height,
                       image_width, ts)
        ev1.record()
        out = img.cpu().numpy()
        return out, {"kernel": ev0.elapsed_time(ev1)}

    def _tile_size_for(self, n_tiles, H, W) -> int:
        for ts in (self.tile_size, 32, 16, 8, 24):
            if ((W + ts - 1) // ts) * ((H + ts - 1) // ts) == n_tiles:
                return ts
        raise ValueError(f"tile_ranges has {n_tiles} rows, which matches no tile size <= 32")

    # -------------------------------------------------------------- fused path

    def has_render_fused(self) -> bool:
        return self._render_fused

    def render_fused(self, gaussians, extrinsics, intrinsics, image_height, image_width,
                     contrib_floor=None, k_cap=3.0, use_isoellipse=False):
        """(image (H,W,3) float32 numpy, stats) in one library call per stage, all on the
        device (backends/cpu_cpp/backend.py:319-383)."""
        cov3d = self._cached_cov3d(gaussians.scales, gaussians.rotations)
        floor_ = (self._mb_contrib_floor if self.contrib_floor_override is None
                  else float(self.contrib_floor_override))
        # the reference's fused call renders with 32-pixel tiles whatever tile_size the
        # staged path uses (backends/cpu_cpp/backend.py:364-381)
        return _d.render_full(gaussians.means, cov3d, gaussians.opacities, gaussians.colors,
                              extrinsics, intrinsics, image_height, image_width,
                              tile_size=32, min_opacity=self.min_opacity,
                              contrib_floor=floor_, mb_contrib_floor=self._mb_contrib_floor,
                              cull_disabled=self.cull_disabled,
                              transmittance_threshold=self.transmittance_threshold,
                              max_radius=self.max_radius, k_cap=self.k_cap,
                              use_isoellipse=self.use_isoellipse)

    def close(self) -> None:
        self._cov3d = None
        self._cov3d_key = None


REGISTRY = {"b200": B200Backend}


def get_backend(name: str, **kwargs):
    """backends/__init__.py:48-60 get_backend, for this package's backends."""
    try:
        cls = REGISTRY[name]
    except KeyError:
        raise KeyError(f"unknown backend {name!r}; available: {', '.join(sorted(REGISTRY))}") from None
    return cls(**kwargs)
