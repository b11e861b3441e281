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
 * reference's sort microbenchmark input). keys_out may be NULL. */
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

#ifdef __cplusplus
}
#endif

#endif /* GS200_H */
