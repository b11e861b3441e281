// train.cuh -- shared definitions of the training-path kernels.
#pragma once

#include "common.cuh"

namespace gs {

// Per-view camera in device form (row-major rotation, translation, intrinsics, centre).
struct TCam {
    float R[9];
    float t[3];
    float fx, fy, cx, cy;
    float cc[3];  // camera centre -R^T t (computed in double on the host)
    int H, W;
};

struct TCfg {
    int sh_degree, K, tile, tiles_x, tiles_y;
    float near_plane, lowpass, amax, amin, tmin;
    float bg[3];
};

struct GConst {
    const float* means;
    const float* ls;
    const float* q;
    const float* ol;
    const float* sh;
};

// Projected records of the Gaussians for one view (or, for the projection kernel, all of a
// step's views back to back, [view][n]), as the rasterisers read them:
// p0 = (mean x, mean y, conic A, conic B), p1 = (conic C, opacity, r, g), p2 = b.
struct ProjView {
    float4* p0;
    float4* p1;
    float* p2;
    uint32_t* dkey;   // bits of the camera-space depth
    uint32_t* dsort;  // depth-sort key: dkey, or 0xffffffff for a Gaussian without pairs
    ushort4* rect;    // inclusive tile rectangle x0, x1, y0, y1 (x1 < x0: no pairs)

    // View v's records inside the [view][n] arrays.
    ProjView view(int v, int64_t n) const {
        const size_t o = (size_t)v * n;
        return ProjView{p0 + o, p1 + o, p2 + o, dkey ? dkey + o : nullptr, dsort + o, rect + o};
    }
};

constexpr int kGradStride = 12;  // floats per Gaussian in a view's 2D-gradient rows

TCam make_tcam(const gs_camera& c);
TCfg make_tcfg(const gs_train_config& c, int H, int W);

// train_project.cu (compiled without FMA contraction)
// Projects every view (cams: device array of n_views cameras) in one pass; pv arrays are
// [n_views][n], blk holds each view's per-block pair totals at v * blk_stride.
// Rows [row_begin, row_end) of the n; row_begin a multiple of kProjThreads.
void launch_project(const GConst& P, int64_t n, int64_t row_begin, int64_t row_end,
                    const TCam* cams, int n_views, const TCfg& cfg, const ProjView& pv,
                    int64_t* blk, int64_t blk_stride, uint64_t* touch, float* vis_counts,
                    float* grad2d, cudaStream_t st);
// Super-tiles of 2^sx x 2^sy tiles: cells along an axis of `tiles` tiles.
__host__ __device__ __forceinline__ int super_cells(int tiles, int s) {
    return (tiles + (1 << s) - 1) >> s;
}
// Per depth-ordered Gaussian: its rectangle and tile-sort item count (the 2^sx x 2^sy-tile
// super-tiles it touches; its tiles with sx = sy = 0), and block totals; then the items'
// offsets from those counts.
void launch_sorted_count(const ProjView& pv, const uint32_t* order, int64_t n, int sx, int sy,
                         ushort4* rect_d, uint32_t* ccnt, int64_t* blk, cudaStream_t st);
void launch_pair_offsets(const uint32_t* ccnt, int64_t n, const int64_t* blk_offsets,
                         int64_t capacity, uint32_t* goff, uint32_t* tfirst, int64_t tfirst_len,
                         uint32_t* last, int64_t* total, unsigned int* err, cudaStream_t st);
// ints of the two row-wise difference arrays (tile grid, then a super-tile grid of at most
// the 2x2-tile grid's size)
int tile_diff_ints(int tiles_x, int tiles_y);
// Tile ranges, super-tile ranges and the tile sort's digit offsets (of the super-tile grid,
// or of the tile grid with sx = sy = 0) from the projected rectangles.
gs_status launch_tile_counts(const ProjView& pv, int64_t n, int tiles_x, int tiles_y, int sx,
                             int sy, int npass, const int64_t* pairs, int64_t capacity, int* diff,
                             int2* ranges, int2* super_ranges, uint32_t* digit_offsets,
                             unsigned int* err, cudaStream_t st);
// Super-tile shapes 2x2 (sx = sy = 1) and 4x2 (sx = 2, sy = 1).
gs_status launch_tile_filter(const uint32_t* super_sorted, const int2* super_ranges,
                             const int2* ranges, int tiles_x, int tiles_y, int sx, int sy,
                             const int64_t* pairs, int64_t capacity, uint32_t* svals,
                             cudaStream_t st);
constexpr int kProjThreads = 256;
#ifndef GS_FILTER_THREADS
#define GS_FILTER_THREADS 256
#endif
constexpr int kFilterThreads = GS_FILTER_THREADS;  // warps x 32 sharing a super-tile in the tile filter
#ifndef GS_FILTER_AHEAD
#define GS_FILTER_AHEAD 8
#endif
constexpr int kFilterAhead = GS_FILTER_AHEAD;  // 32-item steps whose loads the filter issues together
constexpr int kMaxViews = 64;  // views per training step (one bit each in the touched mask)
constexpr int kMaxTileRows = 4096;  // tile rows the tile-count kernel handles

}  // namespace gs
