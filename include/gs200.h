/*
 * gs200.h -- C ABI of libgs200.so, the B200 (sm_100a) implementation of gsplat_tt's
 * per-step render + train path.
 *
 * Conventions
 *   - Every entry point returns a gs_status; on failure gs_last_error() (thread local)
 *     holds a message.
 *   - Array arguments are DEVICE pointers owned by the caller (fp32 / int64 / uint8
 *     row-major, the reference's layouts) unless documented as host memory. Small
 *     per-call constants (camera matrices) are host memory.
 *   - The library allocates no device memory. Entry points that need scratch take a
 *     caller-provided workspace sized by the matching *_workspace_size() query.
 *   - All work is enqueued on `stream` (a cudaStream_t, NULL = legacy default stream).
 *     Entry points return without synchronising unless an argument asks for a host
 *     copy of a data-dependent count (e.g. num_visible_host != NULL), in which case
 *     they synchronise the stream before returning.
 *   - Data-dependent outputs that do not fit the caller's capacity return
 *     GS_ERR_OVERFLOW with the required count written to the *_host argument when
 *     one is given (the reference's overflow-retry contract: grow and call again).
 *
 * Reference interfaces replaced (paths relative to the reference project root) are
 * cited beside each declaration.
 */
#ifndef GS200_H
#define GS200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum gs_status {
    GS_OK = 0,
    GS_ERR_ARG = 1,          /* shape / argument error (reference: std::invalid_argument) */
    GS_ERR_OVERFLOW = 2,     /* caller capacity too small; required size reported */
    GS_ERR_CUDA = 3,         /* CUDA runtime error */
    GS_ERR_TIMEOUT = 4,      /* a bounded device-side wait gave up */
    GS_ERR_UNSUPPORTED = 5   /* option not implemented by this library */
} gs_status;

/* Message of the last failing call on this host thread ("" if none). */
const char* gs_last_error(void);

/* Library version string, e.g. "gs200 0.1 sm_100a". */
const char* gs_version(void);

/* Synchronise `stream` and report the device error word of the last call that used
 * `workspace` (calls whose kernels wait on one another -- the radix sort's look-back --
 * record bounded-wait timeouts there instead of hanging): GS_OK, GS_ERR_TIMEOUT or
 * GS_ERR_OVERFLOW. Valid for gs_sort_pairs and gs_sort_and_bin workspaces. Replaces the
 * reference's hard-fail on device errors (backends/cpu_cpp/pybind_module.cpp:1433-1460). */
gs_status gs_workspace_error(const void* workspace, void* stream);

/* Device reproduction of the host C library's logf over [2^-30, 2^30] (the function the
 * reference's k and pair-cull thresholds use, src/gsplat_cpu/types.h:141-144,
 * src/gsplat_cpu/tile_assign.cpp:177); exposed so tests can sweep it exhaustively. */
gs_status gs_debug_logf_host(const float* x, float* y, int64_t n, void* stream);

/* Per-kernel device timing for benchmarks (no counterpart in the reference, whose
 * stage timers are host-side, render/host/stage_timers.h:1-20). While enabled on a host
 * thread, the library records a CUDA event pair on the launching stream around each
 * instrumented kernel launch. gs_timing_report synchronises the recorded events and
 * writes up to max_kernels entries: kernel names ('\n'-separated) into `names`, total
 * milliseconds and launch counts; it returns the number of entries. */
/* Kernels the library has launched in this process, on every device and thread (for
 * benchmarks: launches inside a timed region). */
int64_t gs_launch_count(void);
void gs_timing_enable(int32_t on);
void gs_timing_reset(void);
int32_t gs_timing_report(char* names, size_t names_len, double* total_ms, int64_t* launches,
                         int32_t max_kernels);

/* ------------------------------------------------------------------------------
 * Display path: project -> tile_assign -> sort_and_bin -> blend
 * ------------------------------------------------------------------------------ */

/* compute_cov3d_batch (src/gsplat_cpu/project.cpp:190-202; pybind compute_cov3d,
 * backends/cpu_cpp/pybind_module.cpp:177-192): cov3d[i] = R(q_i) S_i^2 R(q_i)^T,
 * row-major 3x3, quats (w, x, y, z) used as given (not normalised). */
gs_status gs_compute_cov3d(const float* scales, const float* quats, int64_t n, float* cov3d,
                           void* stream);

/* project_full_fused (src/gsplat_cpu/project.cpp:484-798; pybind
 * project_full_with_cov3d, backends/cpu_cpp/pybind_module.cpp:194-260).
 *   means N*3, cov3d N*9, extrinsics (HOST, 16 floats, row-major world-to-camera),
 *   intrinsics (HOST, 9 floats). colors N*3 and opacities N may be NULL.
 *   max_radius: 0 = min(H,W)/2, >0 = cap, <0 = off. k_cap <= 0 disables the cap.
 *   Outputs (capacity N rows each; compacted to the M visible Gaussians in input order):
 *   means_2d M*2, covs_2d M*4 [a,b,b,c], depths M, radii M*2, colors_out M*3 and
 *   opacities_out M (skipped when the input or output pointer is NULL), valid_mask N.
 *   M is written to *num_visible_dev (device int64) and, if num_visible_host != NULL,
 *   to host memory after a stream synchronisation.
 *   use_isoellipse != 0 returns GS_ERR_UNSUPPORTED. */
gs_status gs_project(const float* means, const float* cov3d, const float* extrinsics,
                     const float* intrinsics, const float* colors, const float* opacities,
                     float min_opacity, int64_t n, int32_t height, int32_t width,
                     int32_t max_radius, float contrib_floor, float k_cap,
                     int32_t use_isoellipse, float* means_2d, float* covs_2d, float* depths,
                     float* radii, uint8_t* valid_mask, float* colors_out,
                     float* opacities_out, int64_t* num_visible_dev,
                     int64_t* num_visible_host, void* workspace, size_t workspace_bytes,
                     void* stream);
size_t gs_project_workspace_size(int64_t n);

/* gs_project without a workspace, for callers that cannot allocate device memory -- a
 * plug-in running inside a host application that owns every device buffer, or a real-time
 * loop where the synchronising cudaMalloc is not allowed. No counterpart in the reference
 * (its CPU stages allocate std::vectors freely).
 *   Same arguments, results and errors as gs_project, minus the workspace. Its scratch is a
 *   fixed 512 KB array inside libgs200.so, present on every device that loads the library
 *   until the process exits; it bounds n to at most 16,777,216 (2^24) Gaussians, and a
 *   larger n returns GS_ERR_ARG. It calls no allocator.
 *   Every call looks up that array's device address in the calling thread's current
 *   context (cudaGetSymbolAddress, which allocates nothing); the first call in a context
 *   also loads the library's device code there, so make that first call before any stream
 *   capture. Arguments are checked in gs_project's order.
 *   All calls share the one array: calls that may overlap on the GPU (different streams or
 *   host threads without ordering between them) race and corrupt each other's results.
 *   Nothing is left over between calls that a later call depends on. */
gs_status gs_project_noalloc(const float* means, const float* cov3d, const float* extrinsics,
                             const float* intrinsics, const float* colors, const float* opacities,
                             float min_opacity, int64_t n, int32_t height, int32_t width,
                             int32_t max_radius, float contrib_floor, float k_cap,
                             int32_t use_isoellipse, float* means_2d, float* covs_2d,
                             float* depths, float* radii, uint8_t* valid_mask,
                             float* colors_out, float* opacities_out, int64_t* num_visible_dev,
                             int64_t* num_visible_host, void* stream);

/* tile_assign (src/gsplat_cpu/tile_assign.cpp:26-368; pybind tile_assign,
 * backends/cpu_cpp/pybind_module.cpp:318-392).
 *   means_2d M*2, radii M*2; covs_2d M*4 and opacities M are both NULL (no pair cull)
 *   or both set (exact min-Mahalanobis cull against contrib_floor).
 *   Outputs: gaussian_ids / tile_ids (capacity `capacity` pairs, Gaussian-major,
 *   row-major within a Gaussian's rectangle, culled pairs removed in order) and
 *   tiles_per_gaussian M (NULL to skip). P is written to *num_pairs_dev and, when
 *   num_pairs_host != NULL, to host memory after a synchronisation; if the pre-cull
 *   pair count exceeds `capacity` the call returns GS_ERR_OVERFLOW with that count in
 *   *num_pairs_host (synchronising in that case even when the pointer is NULL). */
gs_status gs_tile_assign(const float* means_2d, const float* radii, int64_t m, int32_t height,
                         int32_t width, int32_t tile_size, const float* covs_2d,
                         const float* opacities, float contrib_floor, int64_t* gaussian_ids,
                         int64_t* tile_ids, int64_t capacity, int64_t* tiles_per_gaussian,
                         int64_t* num_pairs_dev, int64_t* num_pairs_host, void* workspace,
                         size_t workspace_bytes, void* stream);
size_t gs_tile_assign_workspace_size(int64_t m, int64_t capacity);

/* sort_and_bin (src/gsplat_cpu/sort.cpp:89-263; pybind sort,
 * backends/cpu_cpp/pybind_module.cpp:415-447): stable sort of the P pairs by
 * (tile_id, bits of depths[gaussian_id]); tile_ranges (tiles_x*tiles_y rows of
 * [start, end), (0, 0) for an empty tile). Gaussian ids must be < 2^32 and
 * tiles_x*tiles_y <= 2^31. */
gs_status gs_sort_and_bin(const int64_t* gaussian_ids, const int64_t* tile_ids,
                          const float* depths, int64_t p, int32_t tiles_x, int32_t tiles_y,
                          int64_t* sorted_gaussian_ids, int64_t* tile_ranges,
                          void* workspace, size_t workspace_bytes, void* stream);
size_t gs_sort_and_bin_workspace_size(int64_t p, int32_t tiles_x, int32_t tiles_y);

/* Stable ascending LSD radix sort of (uint64 key, uint32 value) pairs over the low
 * `key_bits` bits of the key (the higher bits must be zero); the order sort_and_bin
 * produces for key = tile << 32 | depth bits (src/gsplat_cpu/sort.cpp:24-27, the
 * reference's sort microbenchmark input). keys_out may be NULL: with more than 32 key
 * bits the sort then narrows its keys to 32 bits once only bits below bit 8 w + 32 are
 * left to sort (w = ceil((key_bits - 32) / 8) passes on 64-bit keys), so the later passes
 * move 4-byte keys; the values come out in the same order. */
gs_status gs_sort_pairs(const uint64_t* keys, const uint32_t* values, int64_t n,
                        int32_t key_bits, uint64_t* keys_out, uint32_t* values_out,
                        void* workspace, size_t workspace_bytes, void* stream);
size_t gs_sort_pairs_workspace_size(int64_t n, int32_t key_bits);

/* blend (src/gsplat_cpu/blend.cpp:14-156; pybind blend,
 * backends/cpu_cpp/pybind_module.cpp:527-600), display rules: conic with determinant
 * clamp 1e-6, alpha = min(o * exp(min(power, 0)), 0.99), front to back, tile-level stop
 * once every pixel of the tile has T < 1e-4. image H*W*3 (black background);
 * alpha H*W (1 - final T; NULL to skip). tile_size <= 32. */
gs_status gs_blend(const float* means_2d, const float* covs_2d, const float* colors,
                   const float* opacities, const int64_t* sorted_gaussian_ids,
                   const int64_t* tile_ranges, int64_t m, int32_t height, int32_t width,
                   int32_t tile_size, float* image, float* alpha, void* stream);

/* src/gsplat_cpu/cull_and_blend.cpp:678-840 cull_and_blend (the reference's default CPU
 * display blend, pybind_module.cpp:764-820 and render_full's CPU path): each tile cut into
 * 8x4-pixel microblocks; a Gaussian of the tile list is kept in each microblock where its
 * exact minimum Mahalanobis distance over the microblock reaches mb_contrib_floor
 * (cull_disabled: every microblock its bounding box overlaps); each microblock blends its
 * list front to back, alpha = min(o * exp(min(power, 0)), 0.99), and stops after the first
 * Gaussian that leaves every pixel's T below transmittance_threshold. image H*W*3 is
 * zeroed first (pixels no Gaussian reaches stay 0). stats (device, 3 int64): pairs_in,
 * pairs_dropped (pairs kept in no microblock), pairs_kept_per_mb. tile_size <= 32;
 * workspace: gs_cull_and_blend_workspace_size(m) bytes. */
size_t gs_cull_and_blend_workspace_size(int64_t m);
gs_status gs_cull_and_blend(const float* means_2d, const float* covs_2d, const float* colors,
                            const float* opacities, const int64_t* sorted_gaussian_ids,
                            const int64_t* tile_ranges, int64_t m, int64_t p, int32_t tiles_x,
                            int32_t tiles_y, int32_t tile_size, int32_t height, int32_t width,
                            float mb_contrib_floor, int32_t cull_disabled,
                            float transmittance_threshold, float* image, int64_t* stats,
                            void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------
 * Training path: per view project -> key emission -> sort -> ranges -> forward raster
 * -> loss -> backward raster; then one projection backward over all views and a
 * sparse Adam step.
 * ------------------------------------------------------------------------------ */

/* Optimizer-space Gaussian parameters (or Adam moments, or gradients), device fp32, in
 * the reference trainer's layouts (gsplat/train_oracle.py:8-20): means N*3, log_scales
 * N*3, quats N*4 (w, x, y, z; unnormalised), opacity_logits N, sh N*K*3 with
 * K = (sh_degree + 1)^2. The five arrays may live anywhere; quats must be 16-byte aligned. */
typedef struct gs_gaussians {
    float* means;
    float* log_scales;
    float* quats;
    float* opacity_logits;
    float* sh;
} gs_gaussians;

/* One pinhole view: world-to-camera w2c (row-major 4x4) and intrinsics K (row-major
 * 3x3), image size (gsplat/train_oracle.py:56-61 Camera). Host memory. */
typedef struct gs_camera {
    float w2c[16];
    float K[9];
    int32_t height;
    int32_t width;
} gs_camera;

/* Render rules (gsplat/train_oracle.py:64-71 RenderConfig), loss (train_oracle.py:276-279
 * loss_fn, gsplat/train_loss.py:126-171) and Adam settings
 * (train_oracle.py:422-470 DEFAULT_LR / sparse_adam_step). */
typedef struct gs_train_config {
    int32_t sh_degree;       /* 0..3 */
    int32_t tile_size;       /* 16 or 32 */
    float near_plane;        /* 0.2 */
    float lowpass;           /* 0.3 */
    float alpha_max;         /* 0.99 */
    float alpha_min;         /* 1/255 */
    float t_min;             /* 1e-4 */
    float background[3];
    int32_t use_ssim;        /* 0: loss = (1 - lambda) L1; 1: (1 - lambda) L1 + lambda (1 - SSIM) */
    float lambda_dssim;      /* 0.2 */
    float lr_means, lr_log_scales, lr_quats, lr_opacity, lr_sh_dc, lr_sh_rest;
    float beta1, beta2, eps;
    int32_t bf16_moments;    /* moments stored as bfloat16 (round to nearest even): the
                                exp_avg / exp_avg_sq arrays then hold 2-byte values and their
                                gs_gaussians pointers are read as 16-bit arrays */
    int32_t deterministic;   /* 1: the backward rasteriser sums each Gaussian's per-tile
                                gradient terms in a fixed order instead of with float
                                atomics, so the same inputs give the same bits on every run
                                (the reference's slot layout, gsplat/blend_backward_ref.py:32-36,
                                239-244: pair (g, tile) writes slot P[g] + j, j the tile's
                                row-major index in g's rectangle, P the exclusive prefix of the
                                Gaussians' tile counts; the slots are then summed j ascending).
                                A debugging mode: slower, tile_size 16 only (GS_ERR_UNSUPPORTED
                                otherwise), and the workspace of
                                gs_train_deterministic_workspace_size. 0: atomics (default). */
} gs_train_config;

/* One training step over n_views views (<= 64) of one rank.
 *   params / exp_avg / exp_avg_sq: parameters and Adam moments, updated in place when
 *   apply_adam != 0 (rows visible in at least one view only, bias correction with
 *   step + 1). grads: written with the gradients summed over the views;
 *   vis_counts (N floats): number of views in which each Gaussian is visible. These two
 *   are the buffers a multi-GPU caller sums across ranks before calling gs_sparse_adam
 *   (apply_adam = 0 here).
 *   targets: n_views pointers to H*W*3 fp32 target images (host array of pointers), each
 *   in device memory (read in place) or in host memory (copied into the workspace; from
 *   pinned memory the copies run on an internal stream, overlapped with other views' work,
 *   and the host buffers must stay unchanged until the step completes on `stream`).
 *   view_losses (device, n_views floats): per-view loss. images (nullable, device,
 *   n_views*H*W*3) and grad2d (nullable, device, n_views*N*9 of dmx, dmy, dA, dB, dC,
 *   dopacity, dr, dg, db) export intermediates for parity tests. pairs (nullable, device
 *   int64, n_views): pair count of each view.
 *   pair_capacity bounds the (Gaussian, tile) pairs of one view; if a view needs more,
 *   the step leaves params and moments untouched and gs_workspace_error() reports
 *   GS_ERR_OVERFLOW (grow the capacity with gs_train_count_pairs and retry).
 *   apply_adam = GS_STEP_DEFER_PARAM_BWD stops after the views: the projection backward
 *   (grads) is left to gs_train_param_backward, called with the same workspace and
 *   arguments, over row ranges (a multi-GPU caller overlaps the update of one range with
 *   the backward of the next); vis_counts are written as usual.
 *   All work is ordered on `stream`: with two or more views, views go round-robin over
 *   up to four lanes -- `stream` and internal streams of the library (created once per
 *   device) forked from `stream` after the projection and joined back to it before the
 *   parameter backward -- so the call stays capturable into a CUDA graph.
 * No counterpart in one reference call: it chains gsplat/blend_backward_dev.py:404
 * forward_fast, gsplat/train_loss.py:126 loss_and_grad_device, blend_backward_dev.py:444
 * ref_slots_fast, gsplat/t2_param_backward.py:244 t2_step (extended to SH1-3 and
 * multiple views) and gsplat/train_oracle.py:434 sparse_adam_step. */
#define GS_STEP_DEFER_PARAM_BWD 2
/* OR-ed into apply_adam: every row of these views was already projected into the
 * workspace by gs_train_project_rows (same params, n, cams, n_views, cfg, vis_counts,
 * pair_capacity and workspace), so the step starts at the pair-count scan. */
#define GS_STEP_PROJECTED 4

gs_status gs_train_step(const gs_gaussians* params, const gs_gaussians* exp_avg,
                        const gs_gaussians* exp_avg_sq, const gs_gaussians* grads,
                        float* vis_counts, int64_t n, int64_t step, const gs_camera* cams,
                        const float* const* targets, int32_t n_views,
                        const gs_train_config* cfg, int32_t apply_adam, float* view_losses,
                        float* images, float* grad2d, int64_t* pairs, int64_t pair_capacity,
                        void* workspace, size_t workspace_bytes, void* stream);
/* The projection of rows [row_begin, row_end) of a step's views into the workspace, for a
 * following gs_train_step with GS_STEP_PROJECTED: zeroes those rows of vis_counts and of
 * the workspace's touched-view masks, uploads the cameras, and projects (2D mean, conic,
 * opacity, colour, depth key, tile rectangle, pair count per view; visibility counts).
 * row_begin and row_end lie on multiples of GS_PROJECT_ROW_ALIGN (row_end may be n). A
 * multi-GPU caller projects the next step's views one row chunk at a time as soon as the
 * chunk's parameters have been updated on every GPU, overlapping the projection with the
 * update of the later chunks. Same stream rules as gs_train_step.
 * No reference counterpart as one call: the projection half of
 * gsplat/t2_param_backward.py:81-120 forward_lanes, split by rows. */
#define GS_PROJECT_ROW_ALIGN 256
gs_status gs_train_project_rows(const gs_gaussians* params, float* vis_counts, int64_t n,
                                int64_t row_begin, int64_t row_end, const gs_camera* cams,
                                int32_t n_views, const gs_train_config* cfg,
                                int64_t pair_capacity, void* workspace, size_t workspace_bytes,
                                void* stream);
size_t gs_train_workspace_size(int64_t n, int32_t sh_degree, int32_t n_views, int32_t height,
                               int32_t width, int32_t tile_size, int64_t pair_capacity);
/* The workspace of a step, gs_render_fwd or gs_render_bwd whose config sets
 * deterministic = 1: gs_train_workspace_size plus, per lane, pair_capacity 48-byte gradient
 * slots and n slot offsets (the layout before them is the same, so every other call taking
 * the workspace accepts it too). gsplat/blend_backward_ref.py:239-244 slot array. */
size_t gs_train_deterministic_workspace_size(int64_t n, int32_t sh_degree, int32_t n_views,
                                             int32_t height, int32_t width, int32_t tile_size,
                                             int64_t pair_capacity);

/* Pair count of each view (projection + tile rectangles only), synchronising, to size
 * pair_capacity. pairs_host: n_views int64 in host memory. */
gs_status gs_train_count_pairs(const gs_gaussians* params, int64_t n, const gs_camera* cams,
                               int32_t n_views, const gs_train_config* cfg,
                               int64_t* pairs_host, void* workspace, size_t workspace_bytes,
                               void* stream);

/* One view's projection and intersections with every intermediate exported, for parity
 * checks of the training path: means2d N*2, conic N*3 (A, B, C of the inverse low-passed
 * 2D covariance), opacity N, colors N*3 (max(SH + 0.5, 0)), depth N (camera z), rects
 * N*4 int32 (inclusive tile rectangle x0, x1, y0, y1; x1 < x0 when the Gaussian has no
 * pairs), vis_counts N (1 where visible for sparse Adam), sorted_ids (pair_capacity
 * uint32: Gaussian ids sorted by tile then depth bits), tile_ranges (tiles*2 int32
 * [start, end)), P in *pairs_host (synchronises). Mirrors gsplat/t2_param_backward.py:81-120
 * forward_lanes, gsplat/blend_backward_dev.py:76-112 tile_rects_vec / pair_lists. */
gs_status gs_train_project_view(const gs_gaussians* params, int64_t n, const gs_camera* cam,
                                const gs_train_config* cfg, float* means2d, float* conic,
                                float* opacity, float* colors, float* depth, int32_t* rects,
                                float* vis_counts, uint32_t* sorted_ids, int32_t* tile_ranges,
                                int64_t pair_capacity, int64_t* pairs_host, void* workspace,
                                size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------
 * Training stages of one view, as separate calls (the reference's staged chain):
 * gs_render_fwd -> gs_loss -> gs_render_bwd -> gs_train_param_backward (rows [0, n),
 * n_views = 1) -> gs_sparse_adam. The forward leaves the view's projected records, sorted
 * pairs, tile ranges, final transmittance and per-pixel pair counts in `workspace` (a
 * training workspace of gs_train_workspace_size(n, sh_degree, 1, H, W, tile, pair_capacity)
 * bytes); the backward and gs_train_param_backward read them from there, so they take the
 * same workspace, n, cam, cfg and pair_capacity, with no other call on that workspace in
 * between. A pair overflow is reported by gs_workspace_error(workspace) after the forward.
 * ------------------------------------------------------------------------------ */

/* gsplat/blend_backward_dev.py:404-438 forward_fast (with the projection of
 * gsplat/t2_param_backward.py:81-120 and the pairs of blend_backward_dev.py:76-112):
 * projection + SH colour, tile intersection, sort, tile ranges and the training-rule
 * forward rasteriser of one view. image H*W*3 (device); final_T H*W and n_contrib H*W
 * (pairs up to the last blended one) are optional copies of the state the backward uses;
 * vis_counts (nullable, N floats) is set to 1 where the Gaussian is visible (for
 * gs_sparse_adam); pairs (nullable, device int64) receives the pair count. */
gs_status gs_render_fwd(const gs_gaussians* params, int64_t n, const gs_camera* cam,
                        const gs_train_config* cfg, float* image, float* final_T,
                        int32_t* n_contrib, float* vis_counts, int64_t* pairs,
                        int64_t pair_capacity, void* workspace, size_t workspace_bytes,
                        void* stream);

/* gsplat/train_loss.py:126-165 loss_and_grad_device ((1 - lambda) L1 + lambda (1 - SSIM),
 * 11x11 Gaussian window, sigma 1.5, zero padding) when cfg->use_ssim, else
 * train_loss.py:166-171 loss_and_grad_l1 ((1 - lambda) L1): the loss of image against
 * target (both H*W*3, device) into *loss (device float) and its gradient into dL_dimage
 * (H*W*3). workspace: gs_loss_workspace_size(height, width) bytes. */
gs_status gs_loss(const float* image, const float* target, int32_t height, int32_t width,
                  const gs_train_config* cfg, float* loss, float* dL_dimage, void* workspace,
                  size_t workspace_bytes, void* stream);
size_t gs_loss_workspace_size(int32_t height, int32_t width);

/* gsplat/blend_backward_dev.py:444-517 ref_slots_fast summed per Gaussian
 * (gsplat/t2_param_backward.py:50-61 segment_reduce): the blend backward of the view of the
 * last gs_render_fwd on `workspace`, replayed back to front from its final transmittance,
 * given dL_dimage (H*W*3, device). The per-Gaussian 2D gradients stay in the workspace for
 * gs_train_param_backward; grad2d (nullable, device, N*9: dmx, dmy, dA, dB, dC, dopacity,
 * dr, dg, db) receives a copy. */
gs_status gs_render_bwd(int64_t n, const gs_camera* cam, const gs_train_config* cfg,
                        const float* dL_dimage, float* grad2d, int64_t pair_capacity,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Sparse Adam over rows with vis_counts > 0 (gsplat/train_oracle.py:434-470
 * sparse_adam_step; gsplat/t2_param_backward.py:195-223 adam_step): fp32 arithmetic,
 * moments stored as fp32 arrays or, with cfg->bf16_moments, as bfloat16 arrays (2 bytes a
 * value, rounded to nearest even after each update, the reference's bf16 mode), lr per
 * group with SH band 0 at lr_sh_dc and bands >= 1 at lr_sh_rest. `error_word` (nullable, device) is checked
 * first: a non-zero value (a failed gs_train_step) skips the update. */
gs_status gs_sparse_adam(const gs_gaussians* params, const gs_gaussians* exp_avg,
                         const gs_gaussians* exp_avg_sq, const gs_gaussians* grads,
                         const float* vis_counts, int64_t n, int64_t step,
                         const gs_train_config* cfg, const unsigned int* error_word,
                         void* stream);

/* Projection backward (2D gradients -> grads of means, log-scales, quaternions, opacity
 * logits and SH) of Gaussian rows [row_begin, row_end) after a gs_train_step call with
 * apply_adam = GS_STEP_DEFER_PARAM_BWD on the same workspace, n, cams, n_views, cfg and
 * pair_capacity, or after gs_render_fwd + gs_render_bwd (n_views = 1). Rows outside the range are not touched. gsplat/t2_param_backward.py:123-192
 * projection_backward_sh0, extended to SH1-3 and summed over the step's views. */
gs_status gs_train_param_backward(const gs_gaussians* params, const gs_gaussians* grads,
                                  int64_t n, int64_t row_begin, int64_t row_end,
                                  const gs_camera* cams, int32_t n_views,
                                  const gs_train_config* cfg, int64_t pair_capacity,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* Owner-sharded sparse Adam of one GPU of a multi-GPU step, with the gradient sum and the
 * parameter broadcast done through NVLink multicast (NVSwitch) inside the kernels. Replaces
 * the allreduce + gs_sparse_adam pair of the view-parallel trainer (the reference has no
 * multi-GPU trainer; its per-step optimizer is gsplat/train_oracle.py:434-470).
 *   params / exp_avg / exp_avg_sq: this GPU's `rows` rows (local memory);
 *   params_mc: the same parameter rows through the parameters' multicast mapping (the
 *     update is written there, i.e. into every GPU's copy);
 *   grads_mc / vis_counts_mc: the same rows of every GPU's partial gradients / visibility
 *     counts through their multicast mapping (read as sums over the GPUs);
 *   vis_scratch: `rows` floats of local device scratch (receives the summed counts);
 *   skip: device word, non-zero = skip the update (a failed step on any GPU).
 * rows is a multiple of 4 and every pointer 16-byte aligned. The caller synchronises the
 * GPUs before the call (every partial gradient written) and after it (no GPU reads the
 * parameters or rewrites its gradients while another is still in the call). */
gs_status gs_sparse_adam_multicast(const gs_gaussians* params, const gs_gaussians* params_mc,
                                   const gs_gaussians* exp_avg, const gs_gaussians* exp_avg_sq,
                                   const gs_gaussians* grads_mc, const float* vis_counts_mc,
                                   float* vis_scratch, int64_t rows, int64_t step,
                                   const gs_train_config* cfg, const unsigned int* skip,
                                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GS200_H */
