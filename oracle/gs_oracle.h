/*
 * gs_oracle.h -- CPU restatement of the reference's display-path stages.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the parity tests,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg compare the CUDA path
 * against. The product library (libgs200.so) never links or loads it.
 *
 * Each function restates one function of the reference's gsplat_cpu library
 * (paths relative to the reference project root) in plain serial C with the same
 * fp32 operation order; compiled with -ffp-contract=off like the reference's
 * Release build (src/CMakeLists.txt:90) so every intermediate rounds as it does.
 * Parity of this restatement is pinned against the reference's own compiled
 * pipeline (oracle/_ref) by tests/test_oracle_display.py.
 */
#ifndef GS_ORACLE_H
#define GS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* src/gsplat_cpu/project.cpp:190-202 compute_cov3d_batch (N*9 row-major). */
void gso_compute_cov3d(const float* scales, const float* quats, int64_t n, float* cov3d);

/*
 * src/gsplat_cpu/project.cpp:484-798 project_full_fused. Outputs are compacted to the
 * M visible Gaussians in input order; every output buffer must hold N rows.
 * Returns M.  colors / opacities may be NULL (no colour gather / no opacity cull,
 * k = 3).  max_radius: 0 = min(H,W)/2, >0 = cap, <0 = off.
 */
int64_t gso_project(const float* means, const float* cov3d, const float* extrinsics,
                    const float* intrinsics, const float* colors, const float* opacities,
                    float min_opacity, int64_t n, int height, int width, int max_radius,
                    float contrib_floor_k, float k_cap, float* means_2d, float* covs_2d,
                    float* depths, float* radii, uint8_t* valid_mask, float* colors_out,
                    float* opacities_out);

/*
 * src/gsplat_cpu/tile_assign.cpp:26-368 tile_assign (recompute_tiles_per_gaussian =
 * true). First call with gaussian_ids == NULL to get the uncull pair count bound;
 * buffers must hold that many rows.  Returns P (after the optional cull).
 */
int64_t gso_tile_assign(const float* means_2d, const float* radii, int64_t m, int height,
                        int width, int tile_size, const float* covs_2d, const float* opacities,
                        float contrib_floor, int64_t* gaussian_ids, int64_t* tile_ids,
                        int64_t* tiles_per_gaussian);

/* src/gsplat_cpu/sort.cpp:89-263 sort_and_bin: stable by (tile_id, depth bits). */
void gso_sort_and_bin(const int64_t* gaussian_ids, const int64_t* tile_ids, const float* depths,
                      int64_t p, int tiles_x, int tiles_y, int64_t* sorted_gaussian_ids,
                      int64_t* tile_ranges);

/* Stable ascending sort of (uint64 key, uint32 value) pairs; the order sort_and_bin
 * produces when key = tile << 32 | depth bits (sort.cpp:24-27). */
void gso_sort_pairs(const uint64_t* keys, const uint32_t* values, int64_t n,
                    uint64_t* keys_out, uint32_t* values_out);

/*
 * src/gsplat_cpu/blend.cpp:14-156 blend (display rules: det clamp 1e-6, alpha <= 0.99,
 * tile-level stop when max T < 1e-4). image is H*W*3; alpha_out (H*W, may be NULL)
 * receives 1 - T_final, an addition the reference's display path does not output.
 */
void gso_blend(const float* means_2d, const float* covs_2d, const float* colors,
               const float* opacities, const int64_t* sorted_gaussian_ids,
               const int64_t* tile_ranges, int64_t m, int height, int width, int tile_size,
               float* image, float* alpha_out);

/*
 * src/gsplat_cpu/cull_and_blend.cpp:316-840 cull_and_blend, scalar build (8x4-pixel
 * microblocks, exact per-microblock cull, per-microblock stop at transmittance_threshold).
 * image (H*W*3) must be zeroed by the caller (pixels of microblocks with no kept Gaussian
 * are not written). stats[0..2] = pairs_in, pairs_dropped_all_mb, pairs_kept_per_mb.
 */
void gso_cull_and_blend(const float* means_2d, const float* covs_2d, const float* colors,
                        const float* opacities, const int64_t* sorted_ids,
                        const int64_t* tile_ranges, int64_t m, int64_t p, int tiles_x,
                        int tiles_y, int tile_size, int height, int width,
                        float mb_contrib_floor, int cull_disabled,
                        float transmittance_threshold, float* image, int64_t* stats);

/* ------------------------------------------------------------------------------
 * Training path (oracle/gs_train_oracle.c): C restatement of the numpy training models
 * of oracle/train.py (forward and backward_2d_exact), multithreaded over tiles, for the
 * parity checks at full benchmark sizes. sorted_ids: Gaussian ids sorted by tile, then
 * depth bits; tile_ranges: tiles_x * tiles_y rows of [start, end).
 * ------------------------------------------------------------------------------ */

/* gsplat/blend_backward_dev.py:404-438 forward_fast (oracle/train.py forward): image
 * H*W*3, final_T H*W, n_contrib H*W (pairs up to the last blended one), ties H*W (a
 * decision within 4e-6 relative of its threshold); tile_reach (nullable, one per tile):
 * the number of leading pairs of the tile's list read before every pixel stopped (the
 * whole list when one never did). Returns the number of blended (pair, pixel)
 * evaluations, or -1 for tile > 32. */
int64_t gso_train_forward(const float* means2d, const float* conic, const float* opacity,
                          const float* colors, const int64_t* sorted_ids,
                          const int64_t* tile_ranges, int height, int width, int tile,
                          float alpha_max, float alpha_min, float t_min, const float* background,
                          float* image, float* final_T, int32_t* n_contrib, uint8_t* ties,
                          int64_t* tile_reach, int threads);

/* gsplat/blend_backward_ref.py:134-249 terms, float64 back to front (oracle/train.py
 * backward_2d_exact): grads N*9 float64 (dmx, dmy, dA, dB, dC, dopacity, dr, dg, db);
 * tie_gaussians (N, may be NULL) marks Gaussians touched by a near-threshold decision.
 * Returns 0, or -1 for tile > 32. */
int gso_train_backward(const float* means2d, const float* conic, const float* opacity,
                       const float* colors, const int64_t* sorted_ids,
                       const int64_t* tile_ranges, int height, int width, int tile,
                       float alpha_max, float alpha_min, float t_min, const float* background,
                       const float* dL_dimage, int64_t n, double* grads, uint8_t* tie_gaussians,
                       int threads);

/* y[i] = logf(x[i]) with the host C library (checks the device logf reproduction). */
void gso_logf_array(const float* x, float* y, int64_t n);

#ifdef __cplusplus
}
#endif

#endif
