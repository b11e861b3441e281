"""Training step on the B200: torch front end of the libgs200 training C ABI.

Names follow the reference trainer (gsplat/train_oracle.py): optimizer-space params
``means, log_scales, quats, opacity_logits, sh``; ``RenderConfig``-style render rules;
``DEFAULT_LR``; ``sparse_adam_step``. One ``Trainer.step`` runs, for every view of this
rank, projection + SH -> key emission -> radix sort -> tile ranges -> forward raster ->
loss -> backward raster, then one fused projection backward over all views and (on one
GPU) the sparse Adam update, all on one CUDA stream through ``gs_train_step``.

Multi-GPU (data parallel over views): each rank renders its own views. By default the
optimizer is owner-sharded (dist.sharded_update): the per-Gaussian gradients and
visibility counts are reduce-scattered so each rank holds the sums of its own contiguous
range of rows, each rank runs sparse Adam on those rows (holding Adam moments only there
in use), and an in-place all-gather of the parameters brings every rank the updated
rows. With ``sharded_optimizer=False`` one allreduce sums gradients + counts (one
contiguous fp32 buffer) and every rank applies the identical sparse Adam step.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from ._lib import check, lib
from .dist import owned_rows, reduce_step_buffer

PARAM_NAMES = ("means", "log_scales", "quats", "opacity_logits", "sh")
DEFAULT_LR = {"means": 1.6e-4, "log_scales": 5e-3, "quats": 1e-3, "opacity_logits": 0.05,
              "sh_dc": 2.5e-3, "sh_rest": 2.5e-3 / 20.0}


class GsGaussians(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in PARAM_NAMES]


class GsCamera(ctypes.Structure):
    _fields_ = [("w2c", ctypes.c_float * 16), ("K", ctypes.c_float * 9),
                ("height", ctypes.c_int32), ("width", ctypes.c_int32)]


class GsTrainConfig(ctypes.Structure):
    _fields_ = [("sh_degree", ctypes.c_int32), ("tile_size", ctypes.c_int32),
                ("near_plane", ctypes.c_float), ("lowpass", ctypes.c_float),
                ("alpha_max", ctypes.c_float), ("alpha_min", ctypes.c_float),
                ("t_min", ctypes.c_float), ("background", ctypes.c_float * 3),
                ("use_ssim", ctypes.c_int32), ("lambda_dssim", ctypes.c_float),
                ("lr_means", ctypes.c_float), ("lr_log_scales", ctypes.c_float),
                ("lr_quats", ctypes.c_float), ("lr_opacity", ctypes.c_float),
                ("lr_sh_dc", ctypes.c_float), ("lr_sh_rest", ctypes.c_float),
                ("beta1", ctypes.c_float), ("beta2", ctypes.c_float), ("eps", ctypes.c_float),
                ("bf16_moments", ctypes.c_int32), ("deterministic", ctypes.c_int32)]


_G = ctypes.POINTER(GsGaussians)
_C = ctypes.POINTER(GsCamera)
_CFG = ctypes.POINTER(GsTrainConfig)
_vp, _i64, _i32, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_size_t
lib.gs_train_step.restype = ctypes.c_int
lib.gs_train_step.argtypes = [_G, _G, _G, _G, _vp, _i64, _i64, _C, ctypes.POINTER(_vp), _i32,
                              _CFG, _i32, _vp, _vp, _vp, _vp, _i64, _vp, _sz, _vp]
lib.gs_train_workspace_size.restype = _sz
lib.gs_train_workspace_size.argtypes = [_i64, _i32, _i32, _i32, _i32, _i32, _i64]
lib.gs_train_deterministic_workspace_size.restype = _sz
lib.gs_train_deterministic_workspace_size.argtypes = [_i64, _i32, _i32, _i32, _i32, _i32, _i64]
lib.gs_train_count_pairs.restype = ctypes.c_int
lib.gs_train_count_pairs.argtypes = [_G, _i64, _C, _i32, _CFG, ctypes.POINTER(_i64), _vp, _sz, _vp]
lib.gs_sparse_adam.restype = ctypes.c_int
lib.gs_sparse_adam.argtypes = [_G, _G, _G, _G, _vp, _i64, _i64, _CFG, _vp, _vp]
lib.gs_sparse_adam_multicast.restype = ctypes.c_int
lib.gs_sparse_adam_multicast.argtypes = [_G, _G, _G, _G, _G, _vp, _vp, _i64, _i64, _CFG, _vp, _vp]
lib.gs_train_param_backward.restype = ctypes.c_int
lib.gs_train_param_backward.argtypes = [_G, _G, _i64, _i64, _i64, _C, _i32, _CFG, _i64, _vp, _sz, _vp]
lib.gs_train_project_rows.restype = ctypes.c_int
lib.gs_train_project_rows.argtypes = [_G, _vp, _i64, _i64, _i64, _C, _i32, _CFG, _i64, _vp, _sz, _vp]
GS_STEP_DEFER_PARAM_BWD = 2
GS_STEP_PROJECTED = 4
GS_PROJECT_ROW_ALIGN = 256
lib.gs_render_fwd.restype = ctypes.c_int
lib.gs_render_fwd.argtypes = [_G, _i64, _C, _CFG, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _sz, _vp]
lib.gs_loss.restype = ctypes.c_int
lib.gs_loss.argtypes = [_vp, _vp, _i32, _i32, _CFG, _vp, _vp, _vp, _sz, _vp]
lib.gs_loss_workspace_size.restype = _sz
lib.gs_loss_workspace_size.argtypes = [_i32, _i32]
lib.gs_render_bwd.restype = ctypes.c_int
lib.gs_render_bwd.argtypes = [_i64, _C, _CFG, _vp, _vp, _i64, _vp, _sz, _vp]
lib.gs_train_project_view.restype = ctypes.c_int
lib.gs_train_project_view.argtypes = [_G, _i64, _C, _CFG, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                      _vp, _vp, _i64, ctypes.POINTER(_i64), _vp, _sz, _vp]


@dataclass
class TrainConfig:
    """gsplat/train_oracle.py:64-71 RenderConfig + loss + Adam settings."""
    sh_degree: int = 3
    tile_size: int = 16
    near: float = 0.2
    lowpass: float = 0.3
    alpha_max: float = 0.99
    alpha_min: float = 1.0 / 255.0
    t_min: float = 1e-4
    background: tuple = (0.0, 0.0, 0.0)
    use_ssim: bool = True
    lambda_dssim: float = 0.2
    lr: dict = field(default_factory=lambda: dict(DEFAULT_LR))
    betas: tuple = (0.9, 0.999)
    eps: float = 1e-15
    bf16_moments: bool = False
    # fixed-order gradient sums in the backward rasteriser (same bits on every run; tile 16)
    deterministic: bool = False

    def workspace_size(self, n: int, n_views: int, height: int, width: int, cap: int) -> int:
        """Bytes of the training workspace a call with this config needs."""
        fn = (lib.gs_train_deterministic_workspace_size if self.deterministic
              else lib.gs_train_workspace_size)
        return int(fn(n, self.sh_degree, n_views, height, width, self.tile_size, cap))

    def c_struct(self) -> GsTrainConfig:
        c = GsTrainConfig()
        c.sh_degree, c.tile_size = int(self.sh_degree), int(self.tile_size)
        c.near_plane, c.lowpass = self.near, self.lowpass
        c.alpha_max, c.alpha_min, c.t_min = self.alpha_max, self.alpha_min, self.t_min
        for i in range(3):
            c.background[i] = float(self.background[i])
        c.use_ssim, c.lambda_dssim = int(bool(self.use_ssim)), float(self.lambda_dssim)
        c.lr_means, c.lr_log_scales = self.lr["means"], self.lr["log_scales"]
        c.lr_quats, c.lr_opacity = self.lr["quats"], self.lr["opacity_logits"]
        c.lr_sh_dc, c.lr_sh_rest = self.lr["sh_dc"], self.lr["sh_rest"]
        c.beta1, c.beta2, c.eps = self.betas[0], self.betas[1], self.eps
        c.bf16_moments = int(bool(self.bf16_moments))
        c.deterministic = int(bool(self.deterministic))
        return c


def camera_struct(w2c, K, height, width) -> GsCamera:
    c = GsCamera()
    w = np.asarray(w2c, np.float32).reshape(16)
    k = np.asarray(K, np.float32).reshape(9)
    for i in range(16):
        c.w2c[i] = float(w[i])
    for i in range(9):
        c.K[i] = float(k[i])
    c.height, c.width = int(height), int(width)
    return c


def _group_sizes(n: int, K: int) -> list[int]:
    return [3 * n, 3 * n, 4 * n, n, 3 * K * n]


class GroupBuffer:
    """The five parameter groups (or moments, or gradients) of N Gaussians in one flat
    device buffer (fp32, or bfloat16 for bf16-stored Adam moments), each group starting on
    a 16-byte boundary. ``extra`` values after the groups hold the visibility counts of a
    gradient buffer, so one allreduce covers gradients and counts."""

    def __init__(self, n: int, sh_degree: int, device, extra: int = 0, rows: int | None = None,
                 alloc=None, dtype=torch.float32):
        """rows >= n: rows allocated per group (the owner-sharded optimizer pads every group
        to world * rows-per-rank rows; the padding rows stay zero). alloc(numel), when given,
        returns the zeroed flat fp32 buffer (symmetric memory for multicast updates)."""
        self.n, self.K = n, (sh_degree + 1) ** 2
        self.rows = n if rows is None else int(rows)
        self.dtype = dtype
        self.esz = torch.empty(0, dtype=dtype).element_size()
        align = 16 // self.esz
        sizes = _group_sizes(self.rows, self.K)
        self.widths = [s // self.rows for s in sizes]
        self.offsets = []
        off = 0
        for s in sizes:
            self.offsets.append(off)
            off += (s + align - 1) // align * align
        self.extra_offset = off
        self.flat = torch.zeros(off + extra, dtype=dtype, device=device) if alloc is None \
            else alloc(off + extra)
        shapes = [(n, 3), (n, 3), (n, 4), (n,), (n, self.K, 3)]
        self.views = {name: self.flat[o:o + int(np.prod(shape))].view(*shape)
                      for name, o, shape in zip(PARAM_NAMES, self.offsets, shapes)}
        # every group's rows including padding, flat
        self.padded = {name: self.flat[o:o + s] for name, o, s in zip(PARAM_NAMES, self.offsets, sizes)}
        self.extra = self.flat[off:off + extra]

    def __getitem__(self, k):
        return self.views[k]

    def c_struct(self, row0: int = 0, base: int | None = None) -> GsGaussians:
        """Group pointers, optionally starting at row `row0` of every group; `base` replaces
        the buffer's own address (e.g. by its multicast address)."""
        b = self.flat.data_ptr() if base is None else base
        return GsGaussians(*[b + self.esz * (o + row0 * w) for o, w in zip(self.offsets, self.widths)])

    def load(self, params: dict) -> None:
        for k in PARAM_NAMES:
            src = params[k]
            src = torch.from_numpy(np.ascontiguousarray(src, np.float32)) if isinstance(src, np.ndarray) else src
            self.views[k].copy_(src.reshape(self.views[k].shape))

    def numpy(self) -> dict:
        """Host fp32 copies of the groups (bfloat16 values widen exactly)."""
        return {k: v.detach().float().cpu().numpy() for k, v in self.views.items()}


class Trainer:
    """Training state (params, Adam moments, gradients, workspace) of one rank.

    ``step(cams, targets)`` runs one step over this rank's views; cams is a list of
    (w2c, K, H, W) and targets a list of (H, W, 3) fp32 device tensors (or numpy arrays).
    Returns the per-view losses as a device tensor (no host synchronisation unless
    ``check`` is set, which also retries with a larger pair capacity on overflow).
    """

    def __init__(self, params: dict, cfg: TrainConfig, n_views: int, height: int, width: int,
                 pair_capacity: int | None = None, device=None, process_group=None,
                 sharded_optimizer: bool = True, multicast: bool = True, mc_chunks: int = 4):
        if not torch.cuda.is_available():
            raise RuntimeError("Trainer needs a CUDA device")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        self.cfg = cfg
        self.ccfg = cfg.c_struct()
        self.n = int(np.asarray(params["means"]).shape[0]) if not isinstance(params["means"], torch.Tensor) \
            else int(params["means"].shape[0])
        self.n_views, self.H, self.W = int(n_views), int(height), int(width)
        self.pg = process_group
        dist_on = torch.distributed.is_available() and torch.distributed.is_initialized()
        self.world = torch.distributed.get_world_size(process_group) if dist_on else 1
        self.rank = torch.distributed.get_rank(process_group) if dist_on else 0
        self.sharded = bool(sharded_optimizer) and self.world > 1
        # Row layout of the sharded update: the rows are padded to chunks * world * q rows.
        # Through multicast, chunk c's rows [c * world * q, (c + 1) * world * q) are updated
        # once every GPU has finished their projection backward, rank r owning the q rows
        # at offset r * q, so the update of one chunk overlaps the backward of the next.
        # Through NCCL, rank r owns the contiguous rows [r * rows_per, (r + 1) * rows_per).
        from .dist import shard_rows
        self.chunks = max(1, int(mc_chunks)) if (self.sharded and multicast) else 1
        self.q = shard_rows(-(-self.n // self.chunks), self.world) if self.sharded else self.n
        rows = self.chunks * self.world * self.q if self.sharded else self.n
        self.rows_per = rows // self.world if self.sharded else self.n
        # parameters and gradients in symmetric memory when the update can go through NVLink
        # multicast (gs_sparse_adam_multicast); otherwise NCCL collectives
        self._symm = {}
        alloc = {}
        if self.sharded and multicast and self.device.type == "cuda":
            from .dist import symmetric_buffer

            def symm_alloc(key):
                def f(numel):
                    t, h, mc = symmetric_buffer(numel, self.device, self.pg)
                    self._symm[key] = (h, mc)
                    return t
                return f
            alloc = {"params": symm_alloc("params"), "grads": symm_alloc("grads")}
        self.params = GroupBuffer(self.n, cfg.sh_degree, self.device, rows=rows, alloc=alloc.get("params"))
        self.params.load(params)
        # bf16 moments are stored as 2-byte values (half the moment bytes Adam moves)
        mdt = torch.bfloat16 if cfg.bf16_moments else torch.float32
        self.m = GroupBuffer(self.n, cfg.sh_degree, self.device, rows=rows, dtype=mdt)
        self.v = GroupBuffer(self.n, cfg.sh_degree, self.device, rows=rows, dtype=mdt)
        self.grads = GroupBuffer(self.n, cfg.sh_degree, self.device, extra=rows + 1, rows=rows,
                                 alloc=alloc.get("grads"))
        self.multicast = bool(self._symm) and all(mc for _, mc in self._symm.values())
        if self.multicast:
            self._vis_scratch = torch.zeros(self.q, dtype=torch.float32, device=self.device)
            self._fence = torch.zeros(1, dtype=torch.float32, device=self.device)
            # The update's stream and its barriers' NCCL stream run at high priority, so
            # their blocks are scheduled ahead of the pending blocks of the backward of the
            # next chunk instead of after all of them.
            self._comm = torch.cuda.Stream(device=self.device, priority=-1)
            self._chunk_done = [torch.cuda.Event() for _ in range(self.chunks)]
            self._chunk_updated = [torch.cuda.Event() for _ in range(self.chunks)]
            self._barrier_pg = self.pg
            if self.pg is None and torch.distributed.get_backend() == "nccl":
                opts = torch.distributed.ProcessGroupNCCL.Options()
                opts.is_high_priority_stream = True
                self._barrier_pg = torch.distributed.new_group(pg_options=opts,
                                                               device_id=self.device)
        self.vis_counts = self.grads.extra[:self.n]
        self.err_slot = self.grads.extra[rows:]
        if self.sharded:
            # this rank's reduced rows of every gradient group and of the visibility counts
            self._grad_shards = [torch.zeros(self.rows_per * w, dtype=torch.float32, device=self.device)
                                 for w in self.grads.widths] + \
                                [torch.zeros(self.rows_per, dtype=torch.float32, device=self.device)]
        self.losses = torch.zeros(self.n_views, dtype=torch.float32, device=self.device)
        self.pairs = torch.zeros(self.n_views, dtype=torch.int64, device=self.device)
        self.step_count = 0
        self._err_i32 = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.capacity = int(pair_capacity) if pair_capacity else 0
        self.ws = None
        # cameras whose projection the previous step already left in the workspace
        self._projected = None
        self._alloc(max(self.capacity, 1))

    def _alloc(self, capacity: int) -> None:
        self._projected = None
        self.capacity = capacity
        nb = self.cfg.workspace_size(self.n, self.n_views, self.H, self.W, capacity)
        self.ws = None
        torch.cuda.empty_cache()
        self.ws = torch.empty(nb, dtype=torch.uint8, device=self.device)

    def _cams(self, cams):
        arr = (GsCamera * len(cams))()
        for i, (w2c, K, H, W) in enumerate(cams):
            arr[i] = camera_struct(w2c, K, H, W)
        return arr

    def count_pairs(self, cams) -> list[int]:
        self._projected = None  # the count projects into the step workspace
        arr = self._cams(cams)
        out = (_i64 * len(cams))()
        p = self.params.c_struct()
        check(lib.gs_train_count_pairs(ctypes.byref(p), self.n, arr, len(cams), ctypes.byref(self.ccfg),
                                       out, self.ws.data_ptr(), self.ws.numel(),
                                       torch.cuda.current_stream().cuda_stream))
        return [int(x) for x in out]

    def ensure_capacity(self, cams, headroom: float = 1.2) -> None:
        need = max(self.count_pairs(cams))
        if need > self.capacity:
            self._alloc(int(need * headroom) + 4096)

    def _targets(self, targets):
        """Device tensors pass through; pinned host fp32 tensors also pass through (the
        library copies each view's target on its own stream, overlapped with the other
        views' work); numpy arrays and other host tensors are copied here."""
        ts = []
        for t in targets:
            if isinstance(t, np.ndarray):
                t = torch.from_numpy(np.ascontiguousarray(t, np.float32))
            if (t.device.type == "cpu" and t.is_pinned() and t.dtype == torch.float32
                    and t.is_contiguous()):
                ts.append(t)
            else:
                ts.append(t.to(self.device, torch.float32).contiguous())
        return ts

    @staticmethod
    def _cams_key(cams) -> tuple:
        return tuple((np.asarray(w2c, np.float32).tobytes(), np.asarray(K, np.float32).tobytes(),
                      int(H), int(W)) for (w2c, K, H, W) in cams)

    def step(self, cams, targets, check_errors: bool = False, images=None, grad2d=None,
             next_cams=None):
        """One step. next_cams (the next step's views, optional): project them at the end
        of this step, after the update -- through multicast, row chunk by row chunk as each
        chunk's update lands on every GPU, overlapped with the update of the later chunks --
        so that the next call with those cameras starts at the sort."""
        if len(cams) != self.n_views:
            raise ValueError(f"expected {self.n_views} views, got {len(cams)}")
        if next_cams is not None and len(next_cams) != self.n_views:
            raise ValueError(f"expected {self.n_views} next views, got {len(next_cams)}")
        tg = self._targets(targets)
        self._keep = tg
        tptr = (ctypes.c_void_p * len(tg))(*[t.data_ptr() for t in tg])
        arr = self._cams(cams)
        st = torch.cuda.current_stream().cuda_stream
        p, m, v, g = (b.c_struct() for b in (self.params, self.m, self.v, self.grads))
        single = self.world == 1
        mode = 1 if single else (GS_STEP_DEFER_PARAM_BWD if self.multicast else 0)
        key = self._cams_key(cams)
        projected, self._projected = self._projected == key, None
        # a step that may be redone (check_errors) does not project ahead
        nxt = None if (next_cams is None or check_errors) else self._cams(next_cams)
        while True:
            flags = mode | (GS_STEP_PROJECTED if projected else 0)
            code = lib.gs_train_step(ctypes.byref(p), ctypes.byref(m), ctypes.byref(v), ctypes.byref(g),
                                     self.vis_counts.data_ptr(), self.n, self.step_count, arr, tptr,
                                     len(cams), ctypes.byref(self.ccfg), flags,
                                     self.losses.data_ptr(),
                                     None if images is None else images.data_ptr(),
                                     None if grad2d is None else grad2d.data_ptr(),
                                     self.pairs.data_ptr(), self.capacity, self.ws.data_ptr(),
                                     self.ws.numel(), st)
            check(code)
            if not single:
                self._allreduce_and_adam(st, arr, nxt)
            elif nxt is not None:
                self._project_rows(nxt, 0, self.n, st)
            if nxt is not None:
                self._projected = self._cams_key(next_cams)
            if not check_errors:
                break
            projected = False
            if single:
                code = lib.gs_workspace_error(self.ws.data_ptr(), st)
                failed = code != _lib.GS_OK
            else:  # the reduced flag: every rank takes the same branch
                failed = bool(self.err_slot.item() > 0)
                code = lib.gs_workspace_error(self.ws.data_ptr(), st) if failed else _lib.GS_OK
            if failed and (code in (_lib.GS_ERR_OVERFLOW, _lib.GS_OK)):
                # Adam was skipped on the device: grow the pair buffers and redo the step.
                self._alloc(max(int(self.pairs.max().item() * 1.25) + 4096, self.capacity))
                continue
            check(code)
            break
        self.step_count += 1
        return self.losses

    def _project_rows(self, arr, b: int, e: int, st) -> None:
        p = self.params.c_struct()
        check(lib.gs_train_project_rows(ctypes.byref(p), self.vis_counts.data_ptr(), self.n, b, e,
                                        arr, len(arr), ctypes.byref(self.ccfg), self.capacity,
                                        self.ws.data_ptr(), self.ws.numel(), st))

    def _allreduce_and_adam(self, st, arr, nxt=None) -> None:
        # error word of this rank's step (first 4 bytes at the workspace's first 256-byte
        # boundary) rides along so every rank agrees on skipping Adam
        off = (-self.ws.data_ptr()) % 256
        errw = self.ws[off:off + 4].view(torch.int32)
        if self.multicast:
            self._multicast_adam(errw, arr, nxt)
            return
        if self.sharded:
            self._sharded_adam(errw, st)
        else:
            reduce_step_buffer(self.grads.flat, self.err_slot, errw, self._err_i32, self.pg)
            p, m, v, g = (b.c_struct() for b in (self.params, self.m, self.v, self.grads))
            check(lib.gs_sparse_adam(ctypes.byref(p), ctypes.byref(m), ctypes.byref(v), ctypes.byref(g),
                                     self.vis_counts.data_ptr(), self.n, self.step_count,
                                     ctypes.byref(self.ccfg), self._err_i32.data_ptr(), st))
        if nxt is not None:
            self._project_rows(nxt, 0, self.n, st)

    def _sharded_adam(self, errw, st) -> None:
        """Owner-sharded update (dist.sharded_update): reduce-scatter gradients and counts,
        sparse Adam on this rank's rows only, in-place all-gather of the parameters."""
        from .dist import sharded_update
        row0 = self.rank * self.rows_per
        shards = self._grad_shards

        def adam(skip):
            p, m, v = (b.c_struct(row0) for b in (self.params, self.m, self.v))
            g = GsGaussians(*[t.data_ptr() for t in shards[:5]])
            check(lib.gs_sparse_adam(ctypes.byref(p), ctypes.byref(m), ctypes.byref(v),
                                     ctypes.byref(g), shards[5].data_ptr(), self.rows_per,
                                     self.step_count, ctypes.byref(self.ccfg), skip.data_ptr(), st))

        grad_groups = [self.grads.padded[k] for k in PARAM_NAMES] + \
            [self.grads.extra[:self.rows_per * self.world]]
        param_groups = [self.params.padded[k] for k in PARAM_NAMES]
        sharded_update(grad_groups, shards, param_groups, errw, self.err_slot, self._err_i32,
                       self.rank, self.world, adam, self.pg)

    def _multicast_adam(self, errw, arr, nxt=None) -> None:
        """Owner-sharded update through NVLink multicast (gs_sparse_adam_multicast),
        pipelined over row chunks: the projection backward of chunk c runs on the step's
        stream; on a second stream a one-float allreduce (the barrier after which every
        GPU's chunk-c gradients are complete; for chunk 0 it also sums the ranks' error
        flags) is followed by the multicast update of this rank's rows of chunk c, while
        the backward of chunk c + 1 proceeds. Without next-step cameras (nxt), a last
        allreduce keeps every GPU from reading parameters or rewriting gradients before all
        updates have landed. With them, each chunk's update is followed by its own
        allreduce (every GPU's update of the chunk has landed, and every GPU has read its
        gradients and visibility counts), after which the step's stream projects the next
        step's views over the chunk's rows (gs_train_project_rows, which also zeroes their
        visibility counts) while the later chunks are still being updated."""
        import torch.distributed as dist
        cur = torch.cuda.current_stream()
        comm = self._comm
        span = self.world * self.q
        p, g = self.params.c_struct(), self.grads.c_struct()
        mc_p, mc_g = self._symm["params"][1], self._symm["grads"][1]
        self.err_slot.copy_((errw != 0).to(torch.float32).reshape(1))
        for c in range(self.chunks):
            b, e = c * span, min((c + 1) * span, self.n)
            if e > b:
                check(lib.gs_train_param_backward(ctypes.byref(p), ctypes.byref(g), self.n, b, e, arr,
                                                  len(arr), ctypes.byref(self.ccfg), self.capacity,
                                                  self.ws.data_ptr(), self.ws.numel(), cur.cuda_stream))
            self._chunk_done[c].record(cur)
            with torch.cuda.stream(comm):
                comm.wait_event(self._chunk_done[c])
                if c == 0:
                    dist.all_reduce(self.err_slot, group=self._barrier_pg)
                    self._err_i32.copy_((self.err_slot > 0).to(torch.int32))
                else:
                    dist.all_reduce(self._fence, group=self._barrier_pg)
                row0 = owned_rows(c, self.rank, self.world, self.q)[0]
                pr, mr, vr = (buf.c_struct(row0) for buf in (self.params, self.m, self.v))
                pm = self.params.c_struct(row0, base=mc_p)
                gm = self.grads.c_struct(row0, base=mc_g)
                vis_mc = mc_g + 4 * (self.grads.extra_offset + row0)
                check(lib.gs_sparse_adam_multicast(ctypes.byref(pr), ctypes.byref(pm), ctypes.byref(mr),
                                                   ctypes.byref(vr), ctypes.byref(gm), vis_mc,
                                                   self._vis_scratch.data_ptr(), self.q,
                                                   self.step_count, ctypes.byref(self.ccfg),
                                                   self._err_i32.data_ptr(), comm.cuda_stream))
                if nxt is not None:
                    dist.all_reduce(self._fence, group=self._barrier_pg)
                    self._chunk_updated[c].record(comm)
        if nxt is None:
            cur.wait_stream(comm)
            dist.all_reduce(self._fence, group=self._barrier_pg)
            return
        # Projection chunks start on block boundaries: chunk c's rows lie in update chunks
        # <= c, all of which have landed once chunk c's event has fired.
        A = GS_PROJECT_ROW_ALIGN
        for c in range(self.chunks):
            b = min(c * span // A * A, self.n)
            e = self.n if c == self.chunks - 1 else min((c + 1) * span // A * A, self.n)
            cur.wait_event(self._chunk_updated[c])
            if e > b:
                self._project_rows(nxt, b, e, cur.cuda_stream)
        cur.wait_stream(comm)

    def project_view(self, w2c, K, H, W) -> dict:
        """Projection, intersections, sorted pairs and tile ranges of one view (parity API)."""
        n, d = self.n, self.device
        out = {"means2d": torch.empty((n, 2), device=d), "conic": torch.empty((n, 3), device=d),
               "opacity": torch.empty(n, device=d), "colors": torch.empty((n, 3), device=d),
               "depth": torch.empty(n, device=d),
               "rects": torch.empty((n, 4), dtype=torch.int32, device=d),
               "visible": torch.empty(n, device=d)}
        ts = self.cfg.tile_size
        tiles = ((W + ts - 1) // ts) * ((H + ts - 1) // ts)
        cap = max(self.capacity, 1)
        sids = torch.empty(cap, dtype=torch.int32, device=d)
        rng = torch.empty((tiles, 2), dtype=torch.int32, device=d)
        P = _i64(0)
        ws = torch.empty(lib.gs_train_workspace_size(n, self.cfg.sh_degree, 1, H, W, ts, cap),
                         dtype=torch.uint8, device=d)
        p = self.params.c_struct()
        cam = camera_struct(w2c, K, H, W)
        check(lib.gs_train_project_view(
            ctypes.byref(p), n, ctypes.byref(cam), ctypes.byref(self.ccfg),
            *[out[k].data_ptr() for k in ("means2d", "conic", "opacity", "colors", "depth", "rects",
                                          "visible")],
            sids.data_ptr(), rng.data_ptr(), cap, ctypes.byref(P), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream().cuda_stream))
        out["sorted_ids"] = sids[:P.value]
        out["tile_ranges"] = rng
        out["pairs"] = P.value
        return out


class StagedView:
    """One view's training step as separate stage calls, in the order of the reference's
    staged chain: ``forward`` (gsplat/blend_backward_dev.py:404 forward_fast, through
    gs_render_fwd), ``loss`` (gsplat/train_loss.py:126 loss_and_grad_device / :166
    loss_and_grad_l1, gs_loss), ``backward`` (blend_backward_dev.py:444 ref_slots_fast
    summed per Gaussian, gs_render_bwd), ``param_backward`` (gsplat/t2_param_backward.py:123
    projection backward into ``trainer.grads``, gs_train_param_backward) and ``adam``
    (gsplat/train_oracle.py:434 sparse_adam_step, gs_sparse_adam). It works on the
    parameters, moments and gradients of a single-GPU ``Trainer`` and keeps its own one-view
    workspace; each stage must follow the previous one on the same view."""

    def __init__(self, trainer: "Trainer", height: int, width: int):
        self.tr = trainer
        self.H, self.W = int(height), int(width)
        cfg = trainer.cfg
        self.ws = torch.empty(cfg.workspace_size(trainer.n, 1, self.H, self.W, trainer.capacity),
                              dtype=torch.uint8, device=trainer.device)
        self.lws = torch.empty(lib.gs_loss_workspace_size(self.H, self.W), dtype=torch.uint8,
                               device=trainer.device)
        self.cam = None
        self.pairs = torch.zeros(1, dtype=torch.int64, device=trainer.device)

    def forward(self, w2c, K):
        """Image (H, W, 3) of the view; also sets trainer.vis_counts for this view."""
        tr = self.tr
        tr._projected = None  # vis_counts are rewritten
        self.cam = camera_struct(w2c, K, self.H, self.W)
        img = torch.empty((self.H, self.W, 3), dtype=torch.float32, device=tr.device)
        self.final_T = torch.empty((self.H, self.W), dtype=torch.float32, device=tr.device)
        self.n_contrib = torch.empty((self.H, self.W), dtype=torch.int32, device=tr.device)
        p = tr.params.c_struct()
        check(lib.gs_render_fwd(ctypes.byref(p), tr.n, ctypes.byref(self.cam), ctypes.byref(tr.ccfg),
                                img.data_ptr(), self.final_T.data_ptr(), self.n_contrib.data_ptr(),
                                tr.vis_counts.data_ptr(), self.pairs.data_ptr(), tr.capacity,
                                self.ws.data_ptr(), self.ws.numel(),
                                torch.cuda.current_stream().cuda_stream))
        return img

    def overflowed(self) -> bool:
        """True when the forward's pairs exceeded the trainer's pair capacity."""
        code = lib.gs_workspace_error(self.ws.data_ptr(), torch.cuda.current_stream().cuda_stream)
        if code not in (_lib.GS_OK, _lib.GS_ERR_OVERFLOW):
            check(code)
        return code == _lib.GS_ERR_OVERFLOW

    def loss(self, image, target):
        """(loss as a 1-element device tensor, dL/dimage (H, W, 3))."""
        tr = self.tr
        t = target if isinstance(target, torch.Tensor) else torch.from_numpy(
            np.ascontiguousarray(target, np.float32))
        t = t.to(tr.device, torch.float32).contiguous()
        loss = torch.empty(1, dtype=torch.float32, device=tr.device)
        dimg = torch.empty_like(image)
        check(lib.gs_loss(image.data_ptr(), t.data_ptr(), self.H, self.W, ctypes.byref(tr.ccfg),
                          loss.data_ptr(), dimg.data_ptr(), self.lws.data_ptr(), self.lws.numel(),
                          torch.cuda.current_stream().cuda_stream))
        return loss, dimg

    def backward(self, dL_dimage):
        """Per-Gaussian 2D gradients (N, 9): dmx, dmy, dA, dB, dC, dopacity, dr, dg, db."""
        tr = self.tr
        g2d = torch.empty((tr.n, 9), dtype=torch.float32, device=tr.device)
        check(lib.gs_render_bwd(tr.n, ctypes.byref(self.cam), ctypes.byref(tr.ccfg),
                                dL_dimage.contiguous().data_ptr(), g2d.data_ptr(), tr.capacity,
                                self.ws.data_ptr(), self.ws.numel(),
                                torch.cuda.current_stream().cuda_stream))
        return g2d

    def param_backward(self) -> None:
        """Parameter gradients of the view into trainer.grads."""
        tr = self.tr
        p, g = tr.params.c_struct(), tr.grads.c_struct()
        check(lib.gs_train_param_backward(ctypes.byref(p), ctypes.byref(g), tr.n, 0, tr.n,
                                          ctypes.byref(self.cam), 1, ctypes.byref(tr.ccfg),
                                          tr.capacity, self.ws.data_ptr(), self.ws.numel(),
                                          torch.cuda.current_stream().cuda_stream))

    def adam(self, step: int) -> None:
        """Sparse Adam over the rows visible in the view."""
        tr = self.tr
        tr._projected = None  # the parameters change
        p, m, v, g = (b.c_struct() for b in (tr.params, tr.m, tr.v, tr.grads))
        check(lib.gs_sparse_adam(ctypes.byref(p), ctypes.byref(m), ctypes.byref(v), ctypes.byref(g),
                                 tr.vis_counts.data_ptr(), tr.n, int(step), ctypes.byref(tr.ccfg),
                                 None, torch.cuda.current_stream().cuda_stream))
