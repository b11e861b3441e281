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

// Projected record of one Gaussian for one view, as the rasterisers read it:
// p0 = (mean x, mean y, conic A, conic B), p1 = (conic C, opacity, r, g), p2 = b.
struct ProjView {
    float4* p0;
    float4* p1;
    float* p2;
    uint32_t* dkey;   // bits of the camera-space depth
    uint32_t* dsort;  // depth-sort key: dkey, or 0xffffffff for a Gaussian without pairs
    ushort4* rect;    // inclusive tile rectangle x0, x1, y0, y1
    uint32_t* cnt;    // tiles in the rectangle (0 = no pairs)
};

constexpr int kGradStride = 12;  // floats per Gaussian in a view's 2D-gradient rows

TCam make_tcam(const gs_camera& c);
TCfg make_tcfg(const gs_train_config& c, int H, int W);

// train_project.cu (compiled without FMA contraction)
void launch_project(const GConst& P, int64_t n, const TCam& cam, const TCfg& cfg, int view,
                    const ProjView& pv, int64_t* blk, uint64_t* touch, float* vis_counts,
                    float* grad2d, cudaStream_t st);
void launch_sorted_count(const ProjView& pv, const uint32_t* order, int64_t n, int64_t* blk,
                         cudaStream_t st);
void launch_emit(const ProjView& pv, const uint32_t* order, int64_t n, const TCfg& cfg,
                 const int64_t* blk_offsets, int64_t capacity, uint32_t* keys, uint32_t* vals,
                 unsigned int* err, cudaStream_t st);
constexpr int kProjThreads = 256;

}  // namespace gs
