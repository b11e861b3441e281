// display.cu -- display-path stages: cov3d, projection, tile assignment, blend.
//
// This translation unit is compiled with -fmad=false (plus IEEE division and square
// root, the nvcc defaults): every float product and sum rounds separately, in the
// operation order of the reference's CPU pipeline, which is built with
// -ffp-contract=off (src/CMakeLists.txt:90). That makes projected means, covariances,
// radii, tile rectangles and pair-cull decisions bit-identical to the reference, the
// precondition for bit-exact pair counts, sorted orders and tile ranges.
#include <cstdarg>
#include <cstring>

#include "common.cuh"
#include "scan.cuh"

namespace gs {

// ------------------------------------------------------------------ host-exact logf

// d_logf_exceptions[] and GS_LOGF_TABLE_{LO,HI,N}, generated at build time from the
// host's logf by gen_logf_table.c.
#include "logf_table.inc"

// logf as the host C library computes it (see gen_logf_table.c): the correctly
// rounded value, nudged by one ulp for the tabulated inputs.
__device__ __forceinline__ float logf_host(float x) {
    float r = (float)log((double)x);
    const unsigned int u = __float_as_uint(x);
    if (u >= GS_LOGF_TABLE_LO && u <= GS_LOGF_TABLE_HI) {
        int lo = 0, hi = (int)GS_LOGF_TABLE_N - 1;
        while (lo <= hi) {
            const int mid = (lo + hi) >> 1;
            const unsigned int e = d_logf_exceptions[mid];
            const unsigned int k = e & 0x7fffffffu;
            if (k == u) {
                const unsigned int rb = __float_as_uint(r);
                r = __uint_as_float((e >> 31) ? rb + 1u : rb - 1u);
                break;
            }
            if (k < u) lo = mid + 1; else hi = mid - 1;
        }
    }
    return r;
}

__global__ void k_logf_host(const float* x, float* y, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = logf_host(x[i]);
}

__device__ __forceinline__ float max_ref(float a, float b) { return (a < b) ? b : a; }
__device__ __forceinline__ float min_ref(float a, float b) { return (b < a) ? b : a; }

// ------------------------------------------------------------------ cov3d

// types.h:68-97 quat_to_rotation_matrix + build_covariance_3d (operation order kept).
__device__ __forceinline__ void cov3d_one(const float* s, float4 q, float* c) {
    const float w = q.x, x = q.y, y = q.z, z = q.w;
    float r[9];
    r[0] = 1.0f - 2.0f * (y * y + z * z);
    r[1] = 2.0f * (x * y - w * z);
    r[2] = 2.0f * (x * z + w * y);
    r[3] = 2.0f * (x * y + w * z);
    r[4] = 1.0f - 2.0f * (x * x + z * z);
    r[5] = 2.0f * (y * z - w * x);
    r[6] = 2.0f * (x * z - w * y);
    r[7] = 2.0f * (y * z + w * x);
    r[8] = 1.0f - 2.0f * (x * x + y * y);
#pragma unroll
    for (int col = 0; col < 3; ++col)
#pragma unroll
        for (int row = 0; row < 3; ++row) r[row * 3 + col] *= s[col];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            c[i * 3 + j] = r[i * 3 + 0] * r[j * 3 + 0] + r[i * 3 + 1] * r[j * 3 + 1] +
                           r[i * 3 + 2] * r[j * 3 + 2];
}

__global__ void k_cov3d(const float* __restrict__ scales, const float4* __restrict__ quats,
                        int64_t n, float* __restrict__ cov3d) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float s[3] = {scales[3 * i], scales[3 * i + 1], scales[3 * i + 2]};
    float c[9];
    cov3d_one(s, quats[i], c);
#pragma unroll
    for (int k = 0; k < 9; ++k) cov3d[9 * i + k] = c[k];
}

// ------------------------------------------------------------------ projection

struct ProjCam {
    float r[9];
    float t[3];
    float fx, fy, cx, cy;
    int height, width;
    float max_r;
    float min_opacity, contrib_floor, k_cap;
};

struct ProjOut {
    float mx, my, a, b, c, depth, rx, ry;
    bool valid;
};

// project.cpp:537-686: per-Gaussian fused projection (isoellipse off).
__device__ __forceinline__ ProjOut project_one(const ProjCam& P, const float* __restrict__ means,
                                               const float* __restrict__ cov3d,
                                               const float* __restrict__ opacities, int64_t i) {
    ProjOut o;
    o.valid = false;
    const float mx = means[3 * i], my = means[3 * i + 1], mz = means[3 * i + 2];
    const float tx = (mx * P.r[0] + my * P.r[1] + mz * P.r[2]) + P.t[0];
    const float ty = (mx * P.r[3] + my * P.r[4] + mz * P.r[5]) + P.t[1];
    const float tz = (mx * P.r[6] + my * P.r[7] + mz * P.r[8]) + P.t[2];
    o.depth = tz;
    if (tz <= 0.2f || (opacities != nullptr && opacities[i] < P.min_opacity)) return o;
    const float inv_tz = 1.0f / tz;
    o.mx = P.fx * tx * inv_tz + P.cx;
    o.my = P.fy * ty * inv_tz + P.cy;
    const float tz2 = tz * tz;
    const float j00 = P.fx / tz, j02 = -P.fx * tx / tz2;
    const float j11 = P.fy / tz, j12 = -P.fy * ty / tz2;
    const float* c3 = cov3d + 9 * i;
    const float c00 = c3[0], c01 = c3[1], c02 = c3[2], c11 = c3[4], c12 = c3[5], c22 = c3[8];
    const float r00 = P.r[0], r01 = P.r[1], r02 = P.r[2];
    const float r10 = P.r[3], r11 = P.r[4], r12 = P.r[5];
    const float r20 = P.r[6], r21 = P.r[7], r22 = P.r[8];
    const float v00 = c00 * r00 + c01 * r01 + c02 * r02;
    const float v01 = c01 * r00 + c11 * r01 + c12 * r02;
    const float v02 = c02 * r00 + c12 * r01 + c22 * r02;
    const float v10 = c00 * r10 + c01 * r11 + c02 * r12;
    const float v11 = c01 * r10 + c11 * r11 + c12 * r12;
    const float v12 = c02 * r10 + c12 * r11 + c22 * r12;
    const float v20 = c00 * r20 + c01 * r21 + c02 * r22;
    const float v21 = c01 * r20 + c11 * r21 + c12 * r22;
    const float v22 = c02 * r20 + c12 * r21 + c22 * r22;
    const float cc00 = r00 * v00 + r01 * v01 + r02 * v02;
    const float cc01 = r00 * v10 + r01 * v11 + r02 * v12;
    const float cc02 = r00 * v20 + r01 * v21 + r02 * v22;
    const float cc11 = r10 * v10 + r11 * v11 + r12 * v12;
    const float cc12 = r10 * v20 + r11 * v21 + r12 * v22;
    const float cc22 = r20 * v20 + r21 * v21 + r22 * v22;
    const float m00 = j00 * cc00 + j02 * cc02;
    const float m01 = j00 * cc01 + j02 * cc12;
    const float m02 = j00 * cc02 + j02 * cc22;
    const float m11 = j11 * cc11 + j12 * cc12;
    const float m12 = j11 * cc12 + j12 * cc22;
    o.a = m00 * j00 + m02 * j02 + 0.3f;
    o.b = m01 * j11 + m02 * j12;
    o.c = m11 * j11 + m12 * j12 + 0.3f;
    float k = 3.0f;
    if (opacities != nullptr) {
        // types.h:141-144 opacity_aware_k
        const float arg = max_ref(opacities[i] / P.contrib_floor, 1.0f);
        k = sqrtf(2.0f * logf_host(arg));
    }
    if (P.k_cap > 0.0f) k = min_ref(k, P.k_cap);
    o.rx = ceilf(k * sqrtf(max_ref(o.a, 0.0f)));
    o.ry = ceilf(k * sqrtf(max_ref(o.c, 0.0f)));
    o.valid = (o.mx + o.rx > 0.0f) && (o.mx - o.rx < (float)P.width) && (o.my + o.ry > 0.0f) &&
              (o.my - o.ry < (float)P.height) && (o.rx > 0.0f) && (o.ry > 0.0f) &&
              (o.rx <= P.max_r) && (o.ry <= P.max_r);
    return o;
}

constexpr int kProjBlock = 256;

// Pass 1: validity mask and per-block visible counts.
__global__ void k_project_count(ProjCam P, const float* __restrict__ means,
                                const float* __restrict__ cov3d,
                                const float* __restrict__ opacities, int64_t n,
                                uint8_t* __restrict__ valid_mask, int64_t* __restrict__ block_counts) {
    __shared__ int64_t smem[33];
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int v = 0;
    if (i < n) {
        v = project_one(P, means, cov3d, opacities, i).valid ? 1 : 0;
        valid_mask[i] = (uint8_t)v;
    }
    int64_t total;
    block_exclusive_scan<int64_t>((int64_t)v, smem, &total);
    if (threadIdx.x == 0) block_counts[blockIdx.x] = total;
}

// Pass 2 (after the block-offset scan): recompute and write the compacted rows in
// input order (project.cpp:710-797).
__global__ void k_project_emit(ProjCam P, const float* __restrict__ means,
                               const float* __restrict__ cov3d,
                               const float* __restrict__ opacities,
                               const float* __restrict__ colors, int64_t n,
                               const uint8_t* __restrict__ valid_mask,
                               const int64_t* __restrict__ block_offsets,
                               float* __restrict__ means_2d, float* __restrict__ covs_2d,
                               float* __restrict__ depths, float* __restrict__ radii,
                               float* __restrict__ colors_out,
                               float* __restrict__ opacities_out) {
    __shared__ int64_t smem[33];
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int v = (i < n) ? valid_mask[i] : 0;
    int64_t total;
    const int64_t rank = block_exclusive_scan<int64_t>((int64_t)v, smem, &total);
    if (!v) return;
    const int64_t o = block_offsets[blockIdx.x] + rank;
    const ProjOut p = project_one(P, means, cov3d, opacities, i);
    means_2d[2 * o] = p.mx;
    means_2d[2 * o + 1] = p.my;
    covs_2d[4 * o] = p.a;
    covs_2d[4 * o + 1] = p.b;
    covs_2d[4 * o + 2] = p.b;
    covs_2d[4 * o + 3] = p.c;
    depths[o] = p.depth;
    radii[2 * o] = p.rx;
    radii[2 * o + 1] = p.ry;
    if (opacities_out != nullptr && opacities != nullptr) opacities_out[o] = opacities[i];
    if (colors_out != nullptr && colors != nullptr) {
        colors_out[3 * o] = colors[3 * i];
        colors_out[3 * o + 1] = colors[3 * i + 1];
        colors_out[3 * o + 2] = colors[3 * i + 2];
    }
}

// ------------------------------------------------------------------ tile assignment

struct TileGrid {
    int tile_size, tiles_x, tiles_y;
    float ts;
};

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// tile_assign.cpp:60-86: inclusive tile rectangle from truncated (p +- r) / tile.
__device__ __forceinline__ void tile_rect(const TileGrid& G, float px, float py, float rx, float ry,
                                          int& x0, int& x1, int& y0, int& y1) {
    x0 = clampi((int)((px - rx) / G.ts), 0, G.tiles_x - 1);
    x1 = clampi((int)((px + rx) / G.ts), 0, G.tiles_x - 1);
    y0 = clampi((int)((py - ry) / G.ts), 0, G.tiles_y - 1);
    y1 = clampi((int)((py + ry) / G.ts), 0, G.tiles_y - 1);
}

__global__ void k_tile_count(TileGrid G, const float* __restrict__ means_2d,
                             const float* __restrict__ radii, int64_t m,
                             int64_t* __restrict__ counts, int64_t* __restrict__ block_counts) {
    __shared__ int64_t smem[33];
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t c = 0;
    if (g < m) {
        int x0, x1, y0, y1;
        tile_rect(G, means_2d[2 * g], means_2d[2 * g + 1], radii[2 * g], radii[2 * g + 1], x0, x1, y0, y1);
        c = (int64_t)(x1 - x0 + 1) * (int64_t)(y1 - y0 + 1);
        counts[g] = c;
    }
    int64_t total;
    block_exclusive_scan<int64_t>(c, smem, &total);
    if (threadIdx.x == 0) block_counts[blockIdx.x] = total;
}

// Gaussian-major, row-major pair emission (tile_assign.cpp:121-135) into 32-bit
// scratch; pairs past `capacity` are dropped and flagged.
__global__ void k_tile_emit(TileGrid G, const float* __restrict__ means_2d,
                            const float* __restrict__ radii, int64_t m,
                            const int64_t* __restrict__ counts,
                            const int64_t* __restrict__ block_offsets, int64_t capacity,
                            uint32_t* __restrict__ gid32, uint32_t* __restrict__ tid32,
                            unsigned int* __restrict__ err) {
    __shared__ int64_t smem[33];
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t c = (g < m) ? counts[g] : 0;
    int64_t total;
    const int64_t off = block_offsets[blockIdx.x] + block_exclusive_scan<int64_t>(c, smem, &total);
    if (g >= m) return;
    if (off + c > capacity) {
        atomicOr(err, DEV_OVERFLOW);
        return;
    }
    int x0, x1, y0, y1;
    tile_rect(G, means_2d[2 * g], means_2d[2 * g + 1], radii[2 * g], radii[2 * g + 1], x0, x1, y0, y1);
    int64_t pos = off;
    for (int y = y0; y <= y1; ++y)
        for (int x = x0; x <= x1; ++x) {
            gid32[pos] = (uint32_t)g;
            tid32[pos] = (uint32_t)(y * G.tiles_x + x);
            ++pos;
        }
}

// tile_assign.cpp:157-171 per-Gaussian threshold m2 <= -2 ln(floor / opacity).
__global__ void k_cull_thresh(const float* __restrict__ opacities, int64_t m, float floor_,
                              float* __restrict__ thresh) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= m) return;
    const float op = opacities[g];
    thresh[g] = (op > floor_) ? -2.0f * logf_host(floor_ / op) : -1.0f;  // -1: never kept
}

// tile_assign.cpp:211-282 exact min-Mahalanobis test of one (Gaussian, tile) pair.
__device__ __forceinline__ bool keep_pair(const TileGrid& G, uint32_t tile, float px, float py,
                                          float a, float b, float c, float thresh) {
    if (thresh < 0.0f) return false;
    const float det = max_ref(a * c - b * b, 1e-6f);
    const float tx0 = (float)(int)(tile % (uint32_t)G.tiles_x) * G.ts;
    const float ty0 = (float)(int)(tile / (uint32_t)G.tiles_x) * G.ts;
    const float u_lo = tx0 - px, u_hi = u_lo + G.ts;
    const float v_lo = ty0 - py, v_hi = v_lo + G.ts;
    const bool x_in = (u_lo <= 0.0f) && (0.0f <= u_hi);
    const bool y_in = (v_lo <= 0.0f) && (0.0f <= v_hi);
    const float scaled = det * thresh;
    if (x_in && y_in) return true;
    float m2v = __int_as_float(0x7f800000), m2h = __int_as_float(0x7f800000);
    if (!x_in) {
        const float uf = (u_lo > 0.0f) ? u_lo : u_hi;
        float vs = (b * uf) / max_ref(a, 1e-12f);
        vs = max_ref(v_lo, min_ref(vs, v_hi));
        m2v = c * uf * uf - 2.0f * b * uf * vs + a * vs * vs;
    }
    if (!y_in) {
        const float vf = (v_lo > 0.0f) ? v_lo : v_hi;
        float us = (b * vf) / max_ref(c, 1e-12f);
        us = max_ref(u_lo, min_ref(us, u_hi));
        m2h = c * us * us - 2.0f * b * us * vf + a * vf * vf;
    }
    return min_ref(m2v, m2h) <= scaled;
}

constexpr int kPairBlock = 256;
constexpr int kPairItems = 8;  // pairs per thread in the cull passes

__global__ void k_cull_count(TileGrid G, const float* __restrict__ means_2d,
                             const float* __restrict__ covs_2d,
                             const float* __restrict__ thresh, const uint32_t* __restrict__ gid32,
                             const uint32_t* __restrict__ tid32, const int64_t* __restrict__ p_dev,
                             uint8_t* __restrict__ keep, int64_t* __restrict__ block_counts) {
    __shared__ int64_t smem[33];
    const int64_t p = *p_dev;
    const int64_t base = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * kPairItems;
    int64_t c = 0;
    for (int k = 0; k < kPairItems; ++k) {
        const int64_t i = base + k;
        if (i >= p) break;
        const uint32_t g = gid32[i];
        const bool kp = keep_pair(G, tid32[i], means_2d[2 * g], means_2d[2 * g + 1], covs_2d[4 * g],
                                  covs_2d[4 * g + 1], covs_2d[4 * g + 3], thresh[g]);
        keep[i] = kp;
        c += kp;
    }
    int64_t total;
    block_exclusive_scan<int64_t>(c, smem, &total);
    if (threadIdx.x == 0) block_counts[blockIdx.x] = total;
}

// Order-preserving compaction (tile_assign.cpp:291-338) into the int64 outputs; with
// keep == null every pair is kept (no cull).
__global__ void k_pairs_write(const uint32_t* __restrict__ gid32, const uint32_t* __restrict__ tid32,
                              const int64_t* __restrict__ p_dev, const uint8_t* __restrict__ keep,
                              const int64_t* __restrict__ block_offsets,
                              int64_t* __restrict__ gids, int64_t* __restrict__ tids,
                              unsigned long long* __restrict__ tpg) {
    __shared__ int64_t smem[33];
    const int64_t p = *p_dev;
    const int64_t base = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * kPairItems;
    int64_t c = 0;
    if (keep != nullptr) {
        for (int k = 0; k < kPairItems; ++k) {
            const int64_t i = base + k;
            if (i >= p) break;
            c += keep[i];
        }
    }
    int64_t total;
    int64_t out = block_exclusive_scan<int64_t>(c, smem, &total);
    if (keep == nullptr) {
        out = base;
    } else {
        out += block_offsets[blockIdx.x];
    }
    for (int k = 0; k < kPairItems; ++k) {
        const int64_t i = base + k;
        if (i >= p) break;
        if (keep != nullptr && !keep[i]) continue;
        gids[out] = (int64_t)gid32[i];
        tids[out] = (int64_t)tid32[i];
        if (tpg != nullptr) atomicAdd(&tpg[gid32[i]], 1ull);
        ++out;
    }
}

__global__ void k_copy_i64(const int64_t* src, int64_t* dst) { *dst = *src; }

// ------------------------------------------------------------------ display blend

struct BlendPair {
    float mx, my, ia, ib, ic, op, cr, cg, cb;
};

// blend.cpp:14-156. One block per tile, one thread per pixel (tile_size^2 threads).
// The tile stops after the first pair at which every in-image pixel has T < 1e-4.
// Each pixel records the first batch-local pair after which its own T < 1e-4; the
// tile's stop pair is the maximum of those, and since T never increases, a batch in
// which that maximum is finite is replayed from its saved state up to the stop pair.
__global__ void k_blend_display(const float* __restrict__ means_2d, const float* __restrict__ covs_2d,
                                const float* __restrict__ colors, const float* __restrict__ opacities,
                                const int64_t* __restrict__ sorted_ids,
                                const int64_t* __restrict__ ranges, int height, int width,
                                int tile_size, int tiles_x, float* __restrict__ image,
                                float* __restrict__ alpha_out) {
    extern __shared__ BlendPair sp[];
    __shared__ int s_red[32];
    const int tile = blockIdx.x;
    const int tx = tile % tiles_x, ty = tile / tiles_x;
    const int lx = threadIdx.x % tile_size, ly = threadIdx.x / tile_size;
    const int x = tx * tile_size + lx, y = ty * tile_size + ly;
    const bool inside = (ly < tile_size) && (x < width) && (y < height);
    const float px = (float)x + 0.5f, py = (float)y + 0.5f;
    const int64_t start = ranges[2 * tile], end = ranges[2 * tile + 1];
    float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f;
    const int nthr = blockDim.x;
    for (int64_t b0 = start; b0 < end; b0 += nthr) {
        const int nb = (int)min((int64_t)nthr, end - b0);
        __syncthreads();
        if (threadIdx.x < nb) {
            const int64_t g = sorted_ids[b0 + threadIdx.x];
            const float a = covs_2d[4 * g], bb = covs_2d[4 * g + 1], c = covs_2d[4 * g + 3];
            const float det = max_ref(a * c - bb * bb, 1e-6f);
            BlendPair q;
            q.mx = means_2d[2 * g];
            q.my = means_2d[2 * g + 1];
            q.ia = c / det;
            q.ib = -bb / det;
            q.ic = a / det;
            q.op = opacities[g];
            q.cr = colors[3 * g];
            q.cg = colors[3 * g + 1];
            q.cb = colors[3 * g + 2];
            sp[threadIdx.x] = q;
        }
        __syncthreads();
        const float T0 = T, r0 = ar, g0 = ag, bl0 = ab;
        int first = 0x7fffffff;
        for (int j = 0; j < nb; ++j) {
            const BlendPair q = sp[j];
            const float dx = px - q.mx, dy = py - q.my;
            const float power = -0.5f * (q.ia * dx * dx + 2.0f * q.ib * dx * dy + q.ic * dy * dy);
            const float gw = expf(min_ref(power, 0.0f));
            const float alpha = min_ref(q.op * gw, 0.99f);
            const float at = alpha * T;
            ar += at * q.cr;
            ag += at * q.cg;
            ab += at * q.cb;
            T = T * (1.0f - alpha);
            if (first == 0x7fffffff && T < 0.0001f) first = j;
        }
        // Tile stop pair within this batch = max over in-image pixels of `first`.
        int v = inside ? first : -1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
        if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
        __syncthreads();
        int stop = -1;
        for (int w = 0; w < (nthr + 31) / 32; ++w) stop = max(stop, s_red[w]);
        if (stop != 0x7fffffff) {
            T = T0; ar = r0; ag = g0; ab = bl0;
            for (int j = 0; j <= stop; ++j) {
                const BlendPair q = sp[j];
                const float dx = px - q.mx, dy = py - q.my;
                const float power = -0.5f * (q.ia * dx * dx + 2.0f * q.ib * dx * dy + q.ic * dy * dy);
                const float gw = expf(min_ref(power, 0.0f));
                const float alpha = min_ref(q.op * gw, 0.99f);
                const float at = alpha * T;
                ar += at * q.cr;
                ag += at * q.cg;
                ab += at * q.cb;
                T = T * (1.0f - alpha);
            }
            break;
        }
    }
    if (!inside) return;
    const int64_t o = (int64_t)y * width + x;
    image[3 * o] = ar;
    image[3 * o + 1] = ag;
    image[3 * o + 2] = ab;
    if (alpha_out != nullptr) alpha_out[o] = 1.0f - T;
}

}  // namespace gs

using namespace gs;

// ================================================================== C ABI

extern "C" gs_status gs_compute_cov3d(const float* scales, const float* quats, int64_t n,
                                      float* cov3d, void* stream) {
    clear_error();
    GS_ARG_CHECK(n >= 0, "gs_compute_cov3d: n must be >= 0");
    if (n == 0) return GS_OK;
    GS_ARG_CHECK(scales && quats && cov3d, "gs_compute_cov3d: null pointer");
    GS_ARG_CHECK(((uintptr_t)quats & 15) == 0, "gs_compute_cov3d: quats must be 16-byte aligned");
    k_cov3d<<<div_up(n, 256), 256, 0, (cudaStream_t)stream>>>(scales, (const float4*)quats, n, cov3d);
    GS_CHECK_LAUNCH();
    return GS_OK;
}

static void proj_layout(int64_t n, WorkspaceSizer& s) {
    s.take<int64_t>(div_up(n, kProjBlock) + 1);
}

extern "C" size_t gs_project_workspace_size(int64_t n) {
    WorkspaceSizer s;
    proj_layout(n < 1 ? 1 : n, s);
    return s.bytes();
}

extern "C" gs_status gs_project(const float* means, const float* cov3d, const float* e,
                                const float* K, const float* colors, const float* opacities,
                                float min_opacity, int64_t n, int32_t height, int32_t width,
                                int32_t max_radius, float contrib_floor, float k_cap,
                                int32_t use_isoellipse, float* means_2d, float* covs_2d,
                                float* depths, float* radii, uint8_t* valid_mask,
                                float* colors_out, float* opacities_out,
                                int64_t* num_visible_dev, int64_t* num_visible_host,
                                void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    if (use_isoellipse) {
        set_error("gs_project: use_isoellipse is not supported");
        return GS_ERR_UNSUPPORTED;
    }
    GS_ARG_CHECK(n >= 0 && height > 0 && width > 0, "gs_project: bad sizes");
    GS_ARG_CHECK(e && K, "gs_project: extrinsics/intrinsics (host) required");
    GS_ARG_CHECK(num_visible_dev, "gs_project: num_visible_dev required");
    if (n > 0)
        GS_ARG_CHECK(means && cov3d && means_2d && covs_2d && depths && radii && valid_mask,
                     "gs_project: null pointer");
    GS_ARG_CHECK(contrib_floor > 0.0f, "gs_project: contrib_floor must be > 0");
    ProjCam P;
    const float r[9] = {e[0], e[1], e[2], e[4], e[5], e[6], e[8], e[9], e[10]};
    memcpy(P.r, r, sizeof(r));
    P.t[0] = e[3]; P.t[1] = e[7]; P.t[2] = e[11];
    P.fx = K[0]; P.fy = K[4]; P.cx = K[2]; P.cy = K[5];
    P.height = height; P.width = width;
    const int mr = max_radius < 0 ? 0x7fffffff
                                   : (max_radius > 0 ? max_radius : (height < width ? height : width) / 2);
    P.max_r = (float)mr;
    P.min_opacity = min_opacity; P.contrib_floor = contrib_floor; P.k_cap = k_cap;
    if (n == 0) {
        GS_CUDA_CHECK(cudaMemsetAsync(num_visible_dev, 0, sizeof(int64_t), st));
        if (num_visible_host) *num_visible_host = 0;
        return GS_OK;
    }
    Workspace ws(workspace, workspace_bytes);
    const unsigned int nb = div_up(n, kProjBlock);
    int64_t* blocks = ws.take<int64_t>(nb + 1);
    GS_ARG_CHECK(ws.ok(), "gs_project: workspace too small (%zu < %zu)", workspace_bytes,
                 gs_project_workspace_size(n));
    k_project_count<<<nb, kProjBlock, 0, st>>>(P, means, cov3d, opacities, n, valid_mask, blocks);
    GS_CHECK_LAUNCH();
    scan_block_totals<int64_t><<<1, 1024, 0, st>>>(blocks, nb, num_visible_dev);
    GS_CHECK_LAUNCH();
    k_project_emit<<<nb, kProjBlock, 0, st>>>(P, means, cov3d, opacities, colors, n, valid_mask,
                                              blocks, means_2d, covs_2d, depths, radii, colors_out,
                                              opacities_out);
    GS_CHECK_LAUNCH();
    if (num_visible_host) {
        GS_CUDA_CHECK(cudaMemcpyAsync(num_visible_host, num_visible_dev, sizeof(int64_t),
                                      cudaMemcpyDeviceToHost, st));
        GS_CUDA_CHECK(cudaStreamSynchronize(st));
    }
    return GS_OK;
}

static void ta_layout(int64_t m, int64_t cap, WorkspaceSizer& s) {
    const int64_t nb_g = div_up(m, kProjBlock) + 1;
    const int64_t nb_p = div_up(cap, (int64_t)kPairBlock * kPairItems) + 1;
    s.take<int64_t>(m);        // counts
    s.take<int64_t>(nb_g);     // per-block totals (Gaussians)
    s.take<int64_t>(nb_p);     // per-block totals (pairs)
    s.take<int64_t>(2);        // pre-cull P, kept P
    s.take<float>(m);          // cull thresholds
    s.take<uint32_t>(cap);     // gid32
    s.take<uint32_t>(cap);     // tid32
    s.take<uint8_t>(cap);      // keep
    s.take<unsigned int>(1);   // error word
}

extern "C" size_t gs_tile_assign_workspace_size(int64_t m, int64_t capacity) {
    WorkspaceSizer s;
    ta_layout(m < 1 ? 1 : m, capacity < 1 ? 1 : capacity, s);
    return s.bytes();
}

extern "C" gs_status gs_tile_assign(const float* means_2d, const float* radii, int64_t m,
                                    int32_t height, int32_t width, int32_t tile_size,
                                    const float* covs_2d, const float* opacities,
                                    float contrib_floor, int64_t* gaussian_ids,
                                    int64_t* tile_ids, int64_t capacity,
                                    int64_t* tiles_per_gaussian, int64_t* num_pairs_dev,
                                    int64_t* num_pairs_host, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    GS_ARG_CHECK(m >= 0 && height > 0 && width > 0 && tile_size > 0, "gs_tile_assign: bad sizes");
    GS_ARG_CHECK((covs_2d == nullptr) == (opacities == nullptr),
                 "gs_tile_assign: covs_2d and opacities must both be given or both be NULL");
    GS_ARG_CHECK(num_pairs_dev, "gs_tile_assign: num_pairs_dev required");
    GS_ARG_CHECK(capacity >= 0 && capacity < (1ll << 40), "gs_tile_assign: bad capacity");
    const bool cull = covs_2d != nullptr;
    TileGrid G;
    G.tile_size = tile_size;
    G.tiles_x = (width + tile_size - 1) / tile_size;
    G.tiles_y = (height + tile_size - 1) / tile_size;
    G.ts = (float)tile_size;
    if (m == 0) {
        GS_CUDA_CHECK(cudaMemsetAsync(num_pairs_dev, 0, sizeof(int64_t), st));
        if (num_pairs_host) *num_pairs_host = 0;
        return GS_OK;
    }
    GS_ARG_CHECK(means_2d && radii, "gs_tile_assign: null pointer");
    GS_ARG_CHECK((int64_t)G.tiles_x * G.tiles_y < (1ll << 31), "gs_tile_assign: too many tiles");
    GS_ARG_CHECK(m < (1ll << 32), "gs_tile_assign: m must be < 2^32");
    Workspace ws(workspace, workspace_bytes);
    const unsigned int nb_g = div_up(m, kProjBlock);
    const int64_t cap = capacity < 1 ? 1 : capacity;
    const unsigned int nb_p = div_up(cap, (int64_t)kPairBlock * kPairItems);
    int64_t* counts = ws.take<int64_t>(m);
    int64_t* blk_g = ws.take<int64_t>(nb_g + 1);
    int64_t* blk_p = ws.take<int64_t>(nb_p + 1);
    int64_t* pcount = ws.take<int64_t>(2);
    float* thresh = ws.take<float>(m);
    uint32_t* gid32 = ws.take<uint32_t>(cap);
    uint32_t* tid32 = ws.take<uint32_t>(cap);
    uint8_t* keep = ws.take<uint8_t>(cap);
    unsigned int* err = ws.take<unsigned int>(1);
    GS_ARG_CHECK(ws.ok(), "gs_tile_assign: workspace too small (%zu < %zu)", workspace_bytes,
                 gs_tile_assign_workspace_size(m, capacity));
    GS_CUDA_CHECK(cudaMemsetAsync(err, 0, sizeof(unsigned int), st));
    k_tile_count<<<nb_g, kProjBlock, 0, st>>>(G, means_2d, radii, m, counts, blk_g);
    GS_CHECK_LAUNCH();
    scan_block_totals<int64_t><<<1, 1024, 0, st>>>(blk_g, nb_g, pcount);
    GS_CHECK_LAUNCH();
    k_tile_emit<<<nb_g, kProjBlock, 0, st>>>(G, means_2d, radii, m, counts, blk_g, capacity, gid32,
                                             tid32, err);
    GS_CHECK_LAUNCH();
    // Pre-cull P is needed on the host to check the capacity (and to size the launch
    // of the pair passes): one synchronisation, as the reference's vectors imply.
    int64_t p_pre = 0;
    unsigned int herr = 0;
    GS_CUDA_CHECK(cudaMemcpyAsync(&p_pre, pcount, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
    GS_CUDA_CHECK(cudaMemcpyAsync(&herr, err, sizeof(unsigned int), cudaMemcpyDeviceToHost, st));
    GS_CUDA_CHECK(cudaStreamSynchronize(st));
    if (p_pre > capacity || (herr & DEV_OVERFLOW)) {
        if (num_pairs_host) *num_pairs_host = p_pre;
        set_error("gs_tile_assign: %lld pairs exceed capacity %lld", (long long)p_pre,
                  (long long)capacity);
        return GS_ERR_OVERFLOW;
    }
    if (p_pre > 0) GS_ARG_CHECK(gaussian_ids && tile_ids, "gs_tile_assign: null output");
    if (tiles_per_gaussian != nullptr) {
        if (cull) {
            GS_CUDA_CHECK(cudaMemsetAsync(tiles_per_gaussian, 0, m * sizeof(int64_t), st));
        } else {
            GS_CUDA_CHECK(cudaMemcpyAsync(tiles_per_gaussian, counts, m * sizeof(int64_t),
                                          cudaMemcpyDeviceToDevice, st));
        }
    }
    const unsigned int nb_run = div_up(p_pre < 1 ? 1 : p_pre, (int64_t)kPairBlock * kPairItems);
    if (cull && p_pre > 0) {
        k_cull_thresh<<<nb_g, kProjBlock, 0, st>>>(opacities, m, contrib_floor, thresh);
        GS_CHECK_LAUNCH();
        k_cull_count<<<nb_run, kPairBlock, 0, st>>>(G, means_2d, covs_2d, thresh, gid32, tid32,
                                                    pcount, keep, blk_p);
        GS_CHECK_LAUNCH();
        scan_block_totals<int64_t><<<1, 1024, 0, st>>>(blk_p, nb_run, pcount + 1);
        GS_CHECK_LAUNCH();
        k_pairs_write<<<nb_run, kPairBlock, 0, st>>>(gid32, tid32, pcount, keep, blk_p, gaussian_ids,
                                                     tile_ids, (unsigned long long*)tiles_per_gaussian);
        GS_CHECK_LAUNCH();
        k_copy_i64<<<1, 1, 0, st>>>(pcount + 1, num_pairs_dev);
    } else {
        if (p_pre > 0) {
            k_pairs_write<<<nb_run, kPairBlock, 0, st>>>(gid32, tid32, pcount, nullptr, nullptr,
                                                         gaussian_ids, tile_ids, nullptr);
            GS_CHECK_LAUNCH();
        }
        k_copy_i64<<<1, 1, 0, st>>>(pcount, num_pairs_dev);
    }
    GS_CHECK_LAUNCH();
    if (num_pairs_host) {
        GS_CUDA_CHECK(cudaMemcpyAsync(num_pairs_host, num_pairs_dev, sizeof(int64_t),
                                      cudaMemcpyDeviceToHost, st));
        GS_CUDA_CHECK(cudaStreamSynchronize(st));
    }
    return GS_OK;
}

// ================================================================== allocation-free projection
//
// A second entry to the projection for callers that cannot allocate device memory, whose
// only scratch (one int64 visible count per 256-Gaussian block) lives in the array below.
// The array is ordinary module memory: every device that loads the library holds it
// (512 KB) until the process exits.

static constexpr int64_t kNoAllocMaxGaussians = 1ll << 24;
static constexpr int64_t kNoAllocScratch = (kNoAllocMaxGaussians + kProjBlock - 1) / kProjBlock + 1;
static __device__ __align__(256) int64_t g_project_scratch[kNoAllocScratch];

// Device address of g_project_scratch in the current device's current context. In host
// code the array's name is only a host-side stand-in, so the address is looked up on every
// call (cudaGetSymbolAddress allocates nothing): module memory belongs to a CUDA context,
// and a cached address would go stale after a device reset or under another context.
static gs_status project_scratch_address(int64_t** out) {
    int64_t* ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress((void**)&ptr, g_project_scratch);
    if (err != cudaSuccess || ptr == nullptr) {
        int dev = -1;
        cudaGetDevice(&dev);
        set_error("gs_project_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                  cudaGetErrorString(err));
        return GS_ERR_CUDA;
    }
    *out = ptr;
    return GS_OK;
}

extern "C" gs_status gs_project_noalloc(const float* means, const float* cov3d, const float* e,
                                        const float* K, const float* colors,
                                        const float* opacities, float min_opacity, int64_t n,
                                        int32_t height, int32_t width, int32_t max_radius,
                                        float contrib_floor, float k_cap, int32_t use_isoellipse,
                                        float* means_2d, float* covs_2d, float* depths,
                                        float* radii, uint8_t* valid_mask, float* colors_out,
                                        float* opacities_out, int64_t* num_visible_dev,
                                        int64_t* num_visible_host, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    if (use_isoellipse) {
        set_error("gs_project_noalloc: use_isoellipse is not supported");
        return GS_ERR_UNSUPPORTED;
    }
    GS_ARG_CHECK(n >= 0 && height > 0 && width > 0, "gs_project_noalloc: bad sizes");
    GS_ARG_CHECK(n <= kNoAllocMaxGaussians,
                 "gs_project_noalloc: n = %lld, but at most %lld Gaussians fit its fixed "
                 "scratch; use gs_project with a workspace for more",
                 (long long)n, (long long)kNoAllocMaxGaussians);
    GS_ARG_CHECK(e && K, "gs_project_noalloc: extrinsics/intrinsics (host) required");
    GS_ARG_CHECK(num_visible_dev, "gs_project_noalloc: num_visible_dev required");
    if (n > 0)
        GS_ARG_CHECK(means && cov3d && means_2d && covs_2d && depths && radii && valid_mask,
                     "gs_project_noalloc: null pointer");
    GS_ARG_CHECK(contrib_floor > 0.0f, "gs_project_noalloc: contrib_floor must be > 0");
    int64_t* blocks = nullptr;
    gs_status s = project_scratch_address(&blocks);
    if (s != GS_OK) return s;
    ProjCam P;
    const float r[9] = {e[0], e[1], e[2], e[4], e[5], e[6], e[8], e[9], e[10]};
    memcpy(P.r, r, sizeof(r));
    P.t[0] = e[3]; P.t[1] = e[7]; P.t[2] = e[11];
    P.fx = K[0]; P.fy = K[4]; P.cx = K[2]; P.cy = K[5];
    P.height = height; P.width = width;
    const int mr = max_radius < 0 ? 0x7fffffff
                                   : (max_radius > 0 ? max_radius : (height < width ? height : width) / 2);
    P.max_r = (float)mr;
    P.min_opacity = min_opacity; P.contrib_floor = contrib_floor; P.k_cap = k_cap;
    if (n == 0) {
        GS_CUDA_CHECK(cudaMemsetAsync(num_visible_dev, 0, sizeof(int64_t), st));
        if (num_visible_host) *num_visible_host = 0;
        return GS_OK;
    }
    // Every scratch entry this call reads is written earlier in the same call (one count
    // per block, then the in-place scan), so nothing needs clearing between calls.
    const unsigned int nb = div_up(n, kProjBlock);
    k_project_count<<<nb, kProjBlock, 0, st>>>(P, means, cov3d, opacities, n, valid_mask, blocks);
    GS_CHECK_LAUNCH();
    scan_block_totals<int64_t><<<1, 1024, 0, st>>>(blocks, nb, num_visible_dev);
    GS_CHECK_LAUNCH();
    k_project_emit<<<nb, kProjBlock, 0, st>>>(P, means, cov3d, opacities, colors, n, valid_mask,
                                              blocks, means_2d, covs_2d, depths, radii, colors_out,
                                              opacities_out);
    GS_CHECK_LAUNCH();
    if (num_visible_host) {
        GS_CUDA_CHECK(cudaMemcpyAsync(num_visible_host, num_visible_dev, sizeof(int64_t),
                                      cudaMemcpyDeviceToHost, st));
        GS_CUDA_CHECK(cudaStreamSynchronize(st));
    }
    return GS_OK;
}

extern "C" gs_status gs_blend(const float* means_2d, const float* covs_2d, const float* colors,
                              const float* opacities, const int64_t* sorted_gaussian_ids,
                              const int64_t* tile_ranges, int64_t m, int32_t height, int32_t width,
                              int32_t tile_size, float* image, float* alpha, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    GS_ARG_CHECK(height > 0 && width > 0, "gs_blend: bad image size");
    GS_ARG_CHECK(tile_size >= 1 && tile_size <= 32, "gs_blend: tile_size must be in [1, 32]");
    GS_ARG_CHECK(image && tile_ranges, "gs_blend: null pointer");
    if (m > 0) GS_ARG_CHECK(means_2d && covs_2d && colors && opacities && sorted_gaussian_ids,
                            "gs_blend: null pointer");
    const int tiles_x = (width + tile_size - 1) / tile_size;
    const int tiles_y = (height + tile_size - 1) / tile_size;
    int threads = tile_size * tile_size;
    threads = (threads + 31) / 32 * 32;
    const size_t smem = (size_t)threads * sizeof(BlendPair);
    k_blend_display<<<tiles_x * tiles_y, threads, smem, st>>>(means_2d, covs_2d, colors, opacities,
                                                              sorted_gaussian_ids, tile_ranges, height,
                                                              width, tile_size, tiles_x, image, alpha);
    GS_CHECK_LAUNCH();
    return GS_OK;
}

// ------------------------------------------------------------------ microblock cull + blend

// Per-Gaussian record of the cull (cull_and_blend.cpp:718-748): screen mean, inverse 2D
// covariance (det clamped at 1e-6), log(floor / opacity) (>= 0: never kept), the
// opacity-scaled bounding-box half extents, opacity and colour.
struct CullRec {
    float mx, my, ia, ib, ic, lt, xh, yh, op, cr, cg, cb;
};
static_assert(sizeof(CullRec) == 48, "CullRec is three 16-byte words");

__global__ void k_cull_records(const float* __restrict__ means_2d, const float* __restrict__ covs_2d,
                               const float* __restrict__ colors, const float* __restrict__ opacities,
                               int64_t m, float floor_, CullRec* __restrict__ rec) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const float a = covs_2d[4 * i], b = covs_2d[4 * i + 1], c = covs_2d[4 * i + 3];
    const float det = max_ref(a * c - b * b, 1e-6f);
    CullRec r;
    r.mx = means_2d[2 * i];
    r.my = means_2d[2 * i + 1];
    r.ia = c / det;
    r.ib = -b / det;
    r.ic = a / det;
    r.op = opacities[i];
    r.cr = colors[3 * i];
    r.cg = colors[3 * i + 1];
    r.cb = colors[3 * i + 2];
    if (r.op <= floor_) {
        r.lt = 0.0f;
        r.xh = r.yh = 0.0f;
    } else {
        r.lt = logf_host(floor_ / r.op);
        const float rd = sqrtf(-2.0f * r.lt);
        r.xh = rd * sqrtf(max_ref(a, 0.0f));
        r.yh = rd * sqrtf(max_ref(c, 0.0f));
    }
    rec[i] = r;
}

constexpr int kMbBatch = 128;  // Gaussians of the tile list staged per batch

// cull_and_blend.cpp:316-675 (scalar build). One block of 32 warps per tile; warp w owns
// microblock w = (my << 2) | mx (8 x 4 pixels, one per lane). Per batch of the tile's
// sorted list, each warp keeps, in list order, the Gaussians whose exact minimum
// Mahalanobis distance over its microblock reaches the floor (ballot compaction), then
// blends them; a warp stops blending after the first Gaussian that leaves every pixel of
// its microblock below transmittance_threshold, but keeps culling to the end of the list
// so the kept / dropped statistics count every pair, as the reference's cull pass does.
// Microblocks outside the tile or image (tiles narrower than 32) are culled for the
// statistics and never blended.
__global__ void __launch_bounds__(1024)
k_cull_blend(const CullRec* __restrict__ rec, const int64_t* __restrict__ sorted_ids,
             const int64_t* __restrict__ ranges, int tiles_x, int tile_size, int height, int width,
             int cull_disabled, float tthresh, float* __restrict__ image,
             unsigned long long* __restrict__ counts) {
    __shared__ CullRec s_rec[kMbBatch];
    __shared__ uint32_t s_rng[kMbBatch];  // mx_lo | mx_hi << 8 | my_lo << 16 | my_hi << 24; ~0: dropped
    __shared__ int s_any[kMbBatch];
    __shared__ uint8_t s_list[32][kMbBatch];
    __shared__ unsigned long long s_kept, s_drop;
    const int tile = blockIdx.x;
    const int64_t start = ranges[2 * tile], end = ranges[2 * tile + 1];
    if (start == end) return;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int ty = tile / tiles_x, tx = tile % tiles_x;
    const float txt = (float)(tx * tile_size), tyt = (float)(ty * tile_size);
    const int mbx = w & 3, mby = w >> 2;
    const int py_tile = ty * tile_size, px_tile = tx * tile_size;
    const int py_end = min(py_tile + tile_size, height), px_end = min(px_tile + tile_size, width);
    const int py0 = py_tile + mby * 4, px0 = px_tile + mbx * 8;
    const int py1 = min(py0 + 4, py_end), px1 = min(px0 + 8, px_end);
    const bool mb_live = py0 < py1 && px0 < px1;
    const int pi = lane >> 3, pj = lane & 7;
    const bool pix = mb_live && pi < py1 - py0 && pj < px1 - px0;
    const float py = (float)(py0 + pi) + 0.5f, px = (float)(px0 + pj) + 0.5f;
    const float v_lo = (tyt + (float)(mby * 4));  // minus the mean per Gaussian
    const float u_lo = (txt + (float)(mbx * 8));
    float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f;
    bool saturated = false;
    int kept_total = 0;
    if (tid == 0) s_kept = s_drop = 0ull;
    for (int64_t b0 = start; b0 < end; b0 += kMbBatch) {
        const int nb = (int)min((int64_t)kMbBatch, end - b0);
        __syncthreads();
        if (tid < nb) {
            const CullRec r = rec[sorted_ids[b0 + tid]];
            s_rec[tid] = r;
            s_any[tid] = 0;
            uint32_t rg = 0xffffffffu;
            if (r.lt < 0.0f) {
                const int mx_lo = max(0, (int)floorf(((r.mx - r.xh) - txt) / 8.0f));
                const int mx_hi = min(3, (int)floorf(((r.mx + r.xh) - txt) / 8.0f));
                const int my_lo = max(0, (int)floorf(((r.my - r.yh) - tyt) / 4.0f));
                const int my_hi = min(7, (int)floorf(((r.my + r.yh) - tyt) / 4.0f));
                if (mx_lo <= mx_hi && my_lo <= my_hi)
                    rg = (uint32_t)mx_lo | (uint32_t)mx_hi << 8 | (uint32_t)my_lo << 16 |
                         (uint32_t)my_hi << 24;
            }
            s_rng[tid] = rg;
        }
        __syncthreads();
        // cull: this warp's microblock against the batch, list order kept by the ballot
        int cnt = 0;
        for (int c0 = 0; c0 < nb; c0 += 32) {
            const int k = c0 + lane;
            bool keep = false;
            if (k < nb) {
                const uint32_t rg = s_rng[k];
                if (rg != 0xffffffffu && mbx >= (int)(rg & 0xff) && mbx <= (int)((rg >> 8) & 0xff) &&
                    mby >= (int)((rg >> 16) & 0xff) && mby <= (int)(rg >> 24)) {
                    const CullRec& r = s_rec[k];
                    const float vl = v_lo - r.my, vh = vl + 4.0f;
                    const bool y_in = (vl <= 0.0f) && (0.0f <= vh);
                    const float v_fix = (vl > 0.0f) ? vl : vh;
                    const float ul = u_lo - r.mx, uh = ul + 8.0f;
                    const bool x_in = (ul <= 0.0f) && (0.0f <= uh);
                    float m2;
                    if (cull_disabled || (x_in && y_in)) {
                        m2 = 0.0f;
                    } else {
                        float m2v = INFINITY, m2h = INFINITY;
                        if (!x_in) {
                            const float uf = (ul > 0.0f) ? ul : uh;
                            float vs = -r.ib * uf / max_ref(r.ic, 1e-12f);
                            vs = vs < vl ? vl : (vh < vs ? vh : vs);
                            m2v = r.ia * uf * uf + 2.0f * r.ib * uf * vs + r.ic * vs * vs;
                        }
                        if (!y_in) {
                            float us = -r.ib * v_fix / max_ref(r.ia, 1e-12f);
                            us = us < ul ? ul : (uh < us ? uh : us);
                            m2h = r.ia * us * us + 2.0f * r.ib * us * v_fix + r.ic * v_fix * v_fix;
                        }
                        m2 = min_ref(m2v, m2h);
                    }
                    keep = m2 <= -2.0f * r.lt;
                }
            }
            const uint32_t bal = __ballot_sync(0xffffffffu, keep);
            if (keep) {
                s_list[w][cnt + __popc(bal & ((1u << lane) - 1u))] = (uint8_t)k;
                s_any[k] = 1;
            }
            cnt += __popc(bal);
        }
        kept_total += cnt;
        __syncwarp();
        // blend this batch's kept list in order until the microblock saturates
        if (mb_live && !saturated) {
            for (int q = 0; q < cnt; ++q) {
                const CullRec& r = s_rec[s_list[w][q]];
                if (pix) {
                    const float dx = px - r.mx, dy = py - r.my;
                    const float power =
                        -0.5f * (r.ia * dx * dx + 2.0f * r.ib * dx * dy + r.ic * dy * dy);
                    const float gw = (float)exp((double)min_ref(power, 0.0f));
                    const float alpha = min_ref(r.op * gw, 0.99f);
                    const float at = alpha * T;
                    ar += at * r.cr;
                    ag += at * r.cg;
                    ab += at * r.cb;
                    T = T * (1.0f - alpha);
                }
                if (__all_sync(0xffffffffu, !pix || T < tthresh)) {
                    saturated = true;
                    break;
                }
            }
        }
        __syncthreads();
        // statistics: Gaussians kept by no microblock (or dropped before the cull)
        if (tid < nb && (s_rng[tid] == 0xffffffffu || s_any[tid] == 0)) atomicAdd(&s_drop, 1ull);
    }
    if (lane == 0 && kept_total > 0) atomicAdd(&s_kept, (unsigned long long)kept_total);
    if (pix && kept_total > 0) {
        const size_t o = ((size_t)(py0 + pi) * width + (px0 + pj)) * 3;
        image[o] = ar;
        image[o + 1] = ag;
        image[o + 2] = ab;
    }
    __syncthreads();
    if (tid == 0) {
        atomicAdd(&counts[0], s_drop);
        atomicAdd(&counts[1], s_kept);
    }
}

__global__ void k_cull_stats(const unsigned long long* __restrict__ counts, int64_t p,
                             int64_t* __restrict__ stats) {
    stats[0] = p;
    stats[1] = (int64_t)counts[0];
    stats[2] = (int64_t)counts[1];
}

extern "C" size_t gs_cull_and_blend_workspace_size(int64_t m) {
    WorkspaceSizer s;
    s.take<unsigned long long>(2);
    s.take<CullRec>(m > 0 ? m : 1);
    return s.bytes();
}

extern "C" gs_status gs_cull_and_blend(const float* means_2d, const float* covs_2d,
                                       const float* colors, const float* opacities,
                                       const int64_t* sorted_gaussian_ids,
                                       const int64_t* tile_ranges, int64_t m, int64_t p,
                                       int32_t tiles_x, int32_t tiles_y, int32_t tile_size,
                                       int32_t height, int32_t width, float mb_contrib_floor,
                                       int32_t cull_disabled, float transmittance_threshold,
                                       float* image, int64_t* stats, void* workspace,
                                       size_t workspace_bytes, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    GS_ARG_CHECK(height > 0 && width > 0 && m >= 0 && p >= 0, "gs_cull_and_blend: bad sizes");
    GS_ARG_CHECK(tile_size >= 1 && tile_size <= 32,
                 "gs_cull_and_blend: tile_size must be in [1, 32] (8x4 microblocks of a 32x32 tile)");
    GS_ARG_CHECK(tiles_x == (width + tile_size - 1) / tile_size &&
                     tiles_y == (height + tile_size - 1) / tile_size,
                 "gs_cull_and_blend: tile grid does not match the image");
    GS_ARG_CHECK(image && tile_ranges && stats, "gs_cull_and_blend: null pointer");
    if (m > 0 && p > 0)
        GS_ARG_CHECK(means_2d && covs_2d && colors && opacities && sorted_gaussian_ids,
                     "gs_cull_and_blend: null pointer");
    Workspace ws(workspace, workspace_bytes);
    unsigned long long* counts = ws.take<unsigned long long>(2);
    CullRec* rec = ws.take<CullRec>(m > 0 ? m : 1);
    GS_ARG_CHECK(ws.ok(), "gs_cull_and_blend: workspace too small (%zu < %zu)", workspace_bytes,
                 gs_cull_and_blend_workspace_size(m));
    GS_CUDA_CHECK(cudaMemsetAsync(image, 0, (size_t)height * width * 3 * sizeof(float), st));
    GS_CUDA_CHECK(cudaMemsetAsync(counts, 0, 2 * sizeof(unsigned long long), st));
    if (m > 0 && p > 0) {
        k_cull_records<<<div_up(m, 256), 256, 0, st>>>(means_2d, covs_2d, colors, opacities, m,
                                                       mb_contrib_floor, rec);
        GS_CHECK_LAUNCH();
        k_cull_blend<<<tiles_x * tiles_y, 1024, 0, st>>>(rec, sorted_gaussian_ids, tile_ranges,
                                                         tiles_x, tile_size, height, width,
                                                         cull_disabled, transmittance_threshold,
                                                         image, counts);
        GS_CHECK_LAUNCH();
    }
    k_cull_stats<<<1, 1, 0, st>>>(counts, p, stats);
    GS_CHECK_LAUNCH();
    return GS_OK;
}

// Device logf reproduction, exposed for the exhaustive parity test of the table.
extern "C" gs_status gs_debug_logf_host(const float* x, float* y, int64_t n, void* stream) {
    clear_error();
    if (n <= 0) return GS_OK;
    k_logf_host<<<div_up(n, 256), 256, 0, (cudaStream_t)stream>>>(x, y, n);
    GS_CHECK_LAUNCH();
    return GS_OK;
}
