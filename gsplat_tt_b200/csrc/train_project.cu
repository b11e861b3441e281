// train_project.cu -- training-path projection and (Gaussian, tile) key emission.
//
// Compiled with -fmad=false: every fp32 product and sum rounds separately, in the
// operation order of the oracle's projection (the reference's fp32 lane model,
// gsplat/t2_param_backward.py:81-120, with its sums written out), and exp is evaluated
// in double and rounded once. Projected means, conics and tile rectangles -- hence pair
// counts, keys and tile ranges -- are then bit-identical to the oracle's.
#include "onesweep.cuh"
#include "scan.cuh"
#include "train.cuh"

namespace gs {

__device__ __forceinline__ float exp_rounded(float x) { return (float)exp((double)x); }

// All of a step's views in one pass over the parameters: a thread reads its Gaussian once
// (means, quaternion, log-scales, opacity logit; the block's SH rows are staged in shared
// memory with coalesced 16-byte loads), forms the view-independent parts (rotation,
// scales, 3D covariance, opacity), then projects it into every view. View v's records go
// to pv arrays at [v * n + g], its per-block pair totals to blk[v * blk_stride + block].
// The Gaussian's Adam visibility count is added once and its touched-view mask written
// once; a touched view's 2D-gradient row is zeroed for the backward's atomics. The launch
// covers rows [row_begin, row_end) of the n, row_begin a multiple of the block size, so a
// block's totals land in the same blk slot whichever row range launched it.
template <int DEG>
__global__ void __launch_bounds__(kProjThreads, 4)
k_train_project(GConst P, int64_t n, int64_t row_begin, int64_t row_end,
                const TCam* __restrict__ cams, int n_views, TCfg cfg,
                ProjView pv, int64_t* __restrict__ blk, int64_t blk_stride,
                uint64_t* __restrict__ touch, float* __restrict__ vis_counts,
                float* __restrict__ grad2d) {
    constexpr int K = (DEG + 1) * (DEG + 1);
    constexpr int ROW = 3 * K;  // floats of SH per Gaussian
    extern __shared__ __align__(16) float s_sh[];
    __shared__ unsigned long long s_tot[kMaxViews];  // the block's pairs per view
    __shared__ TCam s_cam[kMaxViews];
    for (int i = threadIdx.x; i < n_views * (int)(sizeof(TCam) / 4); i += blockDim.x)
        reinterpret_cast<uint32_t*>(s_cam)[i] = reinterpret_cast<const uint32_t*>(cams)[i];
    for (int i = threadIdx.x; i < n_views; i += blockDim.x) s_tot[i] = 0ull;
    const int64_t g = row_begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    {
        const int64_t g0 = row_begin + (int64_t)blockIdx.x * blockDim.x;
        const int rows = (int)min((int64_t)blockDim.x, row_end - g0);
        const float* src = P.sh + (size_t)g0 * ROW;
        const int total = rows * ROW;
        if (((uintptr_t)src & 15u) == 0) {
            const int nv = total >> 2;
            for (int i = threadIdx.x; i < nv; i += blockDim.x)
                reinterpret_cast<float4*>(s_sh)[i] = reinterpret_cast<const float4*>(src)[i];
            for (int i = (nv << 2) + threadIdx.x; i < total; i += blockDim.x) s_sh[i] = src[i];
        } else {
            for (int i = threadIdx.x; i < total; i += blockDim.x) s_sh[i] = src[i];
        }
        __syncthreads();
    }
    const bool live = g < row_end;
    float m0 = 0.f, m1 = 0.f, m2 = 0.f, op = 0.f;
    float S[3][3];
    if (live) {
        m0 = P.means[3 * g];
        m1 = P.means[3 * g + 1];
        m2 = P.means[3 * g + 2];
        const float4 q = reinterpret_cast<const float4*>(P.q)[g];
        const float qinv = 1.0f / sqrtf(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w);
        const float w = q.x * qinv, qx = q.y * qinv, qy = q.z * qinv, qz = q.w * qinv;
        float Rq[9];
        Rq[0] = 1.0f - 2.0f * (qy * qy + qz * qz);
        Rq[1] = 2.0f * (qx * qy - w * qz);
        Rq[2] = 2.0f * (qx * qz + w * qy);
        Rq[3] = 2.0f * (qx * qy + w * qz);
        Rq[4] = 1.0f - 2.0f * (qx * qx + qz * qz);
        Rq[5] = 2.0f * (qy * qz - w * qx);
        Rq[6] = 2.0f * (qx * qz - w * qy);
        Rq[7] = 2.0f * (qy * qz + w * qx);
        Rq[8] = 1.0f - 2.0f * (qx * qx + qy * qy);
        const float s3[3] = {exp_rounded(P.ls[3 * g]), exp_rounded(P.ls[3 * g + 1]),
                             exp_rounded(P.ls[3 * g + 2])};
        float M[9];
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) M[3 * i + j] = Rq[3 * i + j] * s3[j];
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int k = i; k < 3; ++k) {
                S[i][k] = M[3 * i] * M[3 * k] + M[3 * i + 1] * M[3 * k + 1] +
                          M[3 * i + 2] * M[3 * k + 2];
                S[k][i] = S[i][k];
            }
        op = 1.0f / (1.0f + exp_rounded(-P.ol[g]));
    } else {
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int k = 0; k < 3; ++k) S[i][k] = 0.0f;
    }
    const float* sh = s_sh + threadIdx.x * ROW;
    uint64_t touched = 0;
    float nvis = 0.0f;
    for (int v = 0; v < n_views; ++v) {
        const TCam& cam = s_cam[v];
        const int tiles_x = (cam.W + cfg.tile - 1) / cfg.tile;
        const int tiles_y = (cam.H + cfg.tile - 1) / cfg.tile;
        uint32_t count = 0;
        if (live) {
            const float* R = cam.R;
            const float x = R[0] * m0 + R[1] * m1 + R[2] * m2 + cam.t[0];
            const float y = R[3] * m0 + R[4] * m1 + R[5] * m2 + cam.t[1];
            const float z = R[6] * m0 + R[7] * m1 + R[8] * m2 + cam.t[2];
            const bool valid = z > cfg.near_plane;
            float mx = 0.f, my = 0.f, A = 0.f, B = 0.f, C = 0.f, opv = 0.f;
            float col[3] = {0.f, 0.f, 0.f};
            bool visible = false;
            ushort4 rc = make_ushort4(1, 0, 1, 0);
            if (valid) {
                const float iz = 1.0f / z;
                mx = cam.fx * x * iz + cam.cx;
                my = cam.fy * y * iz + cam.cy;
                const float j00 = cam.fx * iz, j02 = -cam.fx * x * iz * iz;
                const float j11 = cam.fy * iz, j12 = -cam.fy * y * iz * iz;
                float T0[3], T1[3];
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    T0[k] = j00 * R[k] + j02 * R[6 + k];
                    T1[k] = j11 * R[3 + k] + j12 * R[6 + k];
                }
                float CT0[3], CT1[3];
#pragma unroll
                for (int i = 0; i < 3; ++i) {
                    CT0[i] = S[i][0] * T0[0] + S[i][1] * T0[1] + S[i][2] * T0[2];
                    CT1[i] = S[i][0] * T1[0] + S[i][1] * T1[1] + S[i][2] * T1[2];
                }
                const float a = T0[0] * CT0[0] + T0[1] * CT0[1] + T0[2] * CT0[2] + cfg.lowpass;
                const float b = T1[0] * CT0[0] + T1[1] * CT0[1] + T1[2] * CT0[2];
                const float c = T1[0] * CT1[0] + T1[1] * CT1[1] + T1[2] * CT1[2] + cfg.lowpass;
                const float idet = 1.0f / (a * c - b * b);
                A = c * idet;
                B = -b * idet;
                C = a * idet;
                // Adam visibility: 3-sigma box of the low-passed covariance overlaps the image.
                const float rxf = ceilf(3.0f * sqrtf(fmaxf(a, 0.0f)));
                const float ryf = ceilf(3.0f * sqrtf(fmaxf(c, 0.0f)));
                visible = (mx + rxf > 0.0f) && (mx - rxf < (float)cam.W) && (my + ryf > 0.0f) &&
                          (my - ryf < (float)cam.H);
                opv = op;
                // SH colour, dir = normalize(mean - camera centre); colour = max(SH + 0.5, 0).
                const float d0 = m0 - cam.cc[0], d1 = m1 - cam.cc[1], d2 = m2 - cam.cc[2];
                const float dn = sqrtf(d0 * d0 + d1 * d1 + d2 * d2);
                const float dx = d0 / dn, dy = d1 / dn, dz = d2 / dn;
                float basis[16];
                basis[0] = 0.28209479177387814f;
                if (DEG >= 1) {
                    basis[1] = -0.4886025119029199f * dy;
                    basis[2] = 0.4886025119029199f * dz;
                    basis[3] = -0.4886025119029199f * dx;
                }
                if (DEG >= 2) {
                    const float xx = dx * dx, yy = dy * dy, zz = dz * dz;
                    basis[4] = 1.0925484305920792f * (dx * dy);
                    basis[5] = -1.0925484305920792f * (dy * dz);
                    basis[6] = 0.31539156525252005f * (2.0f * zz - xx - yy);
                    basis[7] = -1.0925484305920792f * (dx * dz);
                    basis[8] = 0.5462742152960396f * (xx - yy);
                    if (DEG >= 3) {
                        basis[9] = -0.5900435899266435f * dy * (3.0f * xx - yy);
                        basis[10] = 2.890611442640554f * (dx * dy) * dz;
                        basis[11] = -0.4570457994644658f * dy * (4.0f * zz - xx - yy);
                        basis[12] = 0.3731763325901154f * dz * (2.0f * zz - 3.0f * xx - 3.0f * yy);
                        basis[13] = -0.4570457994644658f * dx * (4.0f * zz - xx - yy);
                        basis[14] = 1.445305721320277f * dz * (xx - yy);
                        basis[15] = -0.5900435899266435f * dx * (xx - 3.0f * yy);
                    }
                }
#pragma unroll
                for (int ch = 0; ch < 3; ++ch) {
                    float r = basis[0] * sh[ch];
#pragma unroll
                    for (int k = 1; k < K; ++k) r = r + basis[k] * sh[3 * k + ch];
                    r = r + 0.5f;
                    col[ch] = fmaxf(r, 0.0f);
                }
                // Tile rectangle in float64 from the fp32 conic (gsplat/blend_backward_dev.py:76-92).
                const double Ad = A, Bd = B, Cd = C;
                const double det = Ad * Cd - Bd * Bd;
                const double ca = Cd / det, cc = Ad / det;
                const double rx = ceil(3.0 * sqrt(fmax(ca, 0.0)));
                const double ry = ceil(3.0 * sqrt(fmax(cc, 0.0)));
                const double px = mx, py = my;
                const bool ok = !(px + rx <= 0.0) && !(px - rx >= (double)cam.W) &&
                                !(py + ry <= 0.0) && !(py - ry >= (double)cam.H) && isfinite(rx) &&
                                isfinite(ry);
                if (ok) {
                    // The tile size is a power of two, so x / ts == x * (1 / ts) exactly.
                    const double its = 1.0 / (double)cfg.tile;
                    const double hx = (double)(tiles_x - 1), hy = (double)(tiles_y - 1);
                    const int x0 = (int)fmin(fmax(trunc((px - rx) * its), 0.0), hx);
                    const int x1 = (int)fmin(fmax(trunc((px + rx) * its), 0.0), hx);
                    const int y0 = (int)fmin(fmax(trunc((py - ry) * its), 0.0), hy);
                    const int y1 = (int)fmin(fmax(trunc((py + ry) * its), 0.0), hy);
                    rc = make_ushort4((unsigned short)x0, (unsigned short)x1, (unsigned short)y0,
                                      (unsigned short)y1);
                    count = (uint32_t)((x1 - x0 + 1) * (y1 - y0 + 1));
                }
            }
            const size_t o = (size_t)v * n + g;
            pv.p0[o] = make_float4(mx, my, A, B);
            pv.p1[o] = make_float4(C, opv, col[0], col[1]);
            pv.p2[o] = col[2];
            if (pv.dkey != nullptr) pv.dkey[o] = __float_as_uint(z);
            pv.dsort[o] = count > 0 ? __float_as_uint(z) : 0xffffffffu;
            pv.rect[o] = rc;
            if (visible) nvis += 1.0f;
            if (count > 0) {
                touched |= 1ull << v;
                if (grad2d != nullptr) {
                    float4* gr = reinterpret_cast<float4*>(grad2d + o * kGradStride);
                    gr[0] = make_float4(0.f, 0.f, 0.f, 0.f);
                    gr[1] = make_float4(0.f, 0.f, 0.f, 0.f);
                    gr[2] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
        uint32_t wsum = count;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
        if ((threadIdx.x & 31) == 0 && wsum != 0u) atomicAdd(&s_tot[v], (unsigned long long)wsum);
    }
    if (live) {
        if (touch != nullptr) touch[g] = touched;
        if (vis_counts != nullptr && nvis > 0.0f) vis_counts[g] += nvis;
    }
    __syncthreads();
    const int64_t b = row_begin / kProjThreads + blockIdx.x;
    for (int v = threadIdx.x; v < n_views; v += blockDim.x)
        blk[v * blk_stride + b] = (int64_t)s_tot[v];
}

// The Gaussians in depth order (`order` = ids sorted by depth bits, stable): each one's
// tile rectangle (rect_d) and its number of tile-sort items (ccnt: the 2^sx x 2^sy-tile
// super-tiles its rectangle touches, its tiles with sx = sy = 0, 0 without tiles),
// gathered once, and the per-block item totals for the offset scan.
__global__ void __launch_bounds__(kProjThreads)
k_sorted_count(const ushort4* __restrict__ rect,
               const uint32_t* __restrict__ order, int64_t n, int sx, int sy,
               ushort4* __restrict__ rect_d, uint32_t* __restrict__ ccnt,
               int64_t* __restrict__ blk) {
    __shared__ int64_t smem[33];
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint32_t c = 0u;
    if (i < n) {
        const uint32_t g = order[i];
        const ushort4 r = rect[g];
        // the tile count follows from the rectangle (x1 < x0 for a Gaussian without tiles),
        // so one 8-byte gather per Gaussian suffices
        const uint32_t t = (r.y >= r.x) ? (uint32_t)(r.y - r.x + 1) * (uint32_t)(r.w - r.z + 1) : 0u;
        c = (t == 0u || (sx | sy) == 0)
                ? t
                : (uint32_t)((r.y >> sx) - (r.x >> sx) + 1) * (uint32_t)((r.w >> sy) - (r.z >> sy) + 1);
        rect_d[i] = r;
        ccnt[i] = c;
    }
    int64_t total;
    block_exclusive_scan<int64_t>((int64_t)c, smem, &total);
    if (threadIdx.x == 0) blk[blockIdx.x] = total;
}

// First tile-sort item of each Gaussian in depth order (goff, n + 1 entries; goff[n] =
// items), clamped to the pair capacity (DEV_OVERFLOW when they exceed it). Also, per
// 4096-item tile of the tile sort, the depth index of the Gaussian holding the tile's first
// item (tfirst), the depth index of the last Gaussian with pairs (Gaussians without pairs
// sort after every Gaussian with pairs), and the number of items (total).
__global__ void __launch_bounds__(kProjThreads)
k_pair_offsets(const uint32_t* __restrict__ ccnt, int64_t n,
               const int64_t* __restrict__ blk_offsets, int64_t capacity,
               uint32_t* __restrict__ goff, uint32_t* __restrict__ tfirst, int64_t tfirst_len,
               uint32_t* __restrict__ last, int64_t* __restrict__ total_out,
               unsigned int* __restrict__ err) {
    __shared__ int64_t smem[33];
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t c = (i < n) ? ccnt[i] : 0u;
    int64_t total;
    const int64_t off = blk_offsets[blockIdx.x] + block_exclusive_scan<int64_t>((int64_t)c, smem, &total);
    if (i >= n) return;
    const uint32_t cn = (i + 1 < n) ? ccnt[i + 1] : 0u;
    goff[i] = (uint32_t)min(off, capacity);
    if (i == n - 1) {
        goff[n] = (uint32_t)min(off + (int64_t)c, capacity);
        *total_out = off + (int64_t)c;
    }
    if (c == 0) return;
    if (off + (int64_t)c > capacity) atomicOr(err, DEV_OVERFLOW);
    for (int64_t b = (off + kTileItems - 1) / kTileItems;
         b * kTileItems < off + (int64_t)c && b < tfirst_len; ++b)
        tfirst[b] = (uint32_t)i;
    if (cn == 0) *last = (uint32_t)i;
}

// Per tile row, +1 at column x0 and -1 at column x1 + 1 for every row of every Gaussian's
// tile rectangle (a row-wise difference array, (tiles_x + 1) x tiles_y ints): a prefix
// sum along each row then gives the pairs per tile. The same for the grid of 2^sx x 2^sy
// super-tiles ((cells_x + 1) x cells_y ints, after the tile grid's). Summed in shared
// memory per block when both grids fit `smem_bins`, then added to the global arrays.
__global__ void __launch_bounds__(1024)
k_tile_diff(const ushort4* __restrict__ rect, int64_t n,
            int tiles_x, int tiles_y, int sx, int sy, int smem_bins, int* __restrict__ diff) {
    extern __shared__ int s_diff[];
    const int gw = tiles_x + 1;
    const int sgw = super_cells(tiles_x, sx) + 1, sgh = super_cells(tiles_y, sy);
    const int tbins = gw * tiles_y;
    const int bins = tbins + sgw * sgh;
    const bool local = bins <= smem_bins;
    int* d = local ? s_diff : diff;
    int* ds = d + tbins;
    if (local) {
        for (int i = threadIdx.x; i < bins; i += blockDim.x) s_diff[i] = 0;
        __syncthreads();
    }
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n;
         g += (int64_t)gridDim.x * blockDim.x) {
        const ushort4 r = rect[g];
        if (r.y < r.x) continue;  // no tiles
        for (int y = r.z; y <= (int)r.w; ++y) {
            atomicAdd(&d[y * gw + r.x], 1);
            atomicAdd(&d[y * gw + r.y + 1], -1);
        }
        for (int y = r.z >> sy; y <= (int)(r.w >> sy); ++y) {
            atomicAdd(&ds[y * sgw + (r.x >> sx)], 1);
            atomicAdd(&ds[y * sgw + (r.y >> sx) + 1], -1);
        }
    }
    if (local) {
        __syncthreads();
        for (int i = threadIdx.x; i < bins; i += blockDim.x) {
            const int v = s_diff[i];
            if (v != 0) atomicAdd(&diff[i], v);
        }
    }
}

// One block of 1024 threads: pairs per tile from the row-wise difference array (a warp
// per tile row), tile ranges [start, end) in row-major tile order ((0, 0) when empty), and
// each tile-sort pass's exclusive digit offsets: digit d of pass p collects the tiles t
// with (t >> 8p) & 255 == d. When the view's pairs exceed the capacity (reported through
// DEV_OVERFLOW by k_pair_offsets) every range is left empty, so no later kernel reads
// past the sorted-pair buffer.
struct GridFinish {
    const int* diff;
    int tiles_x, tiles_y, npass;
    int2* ranges;
    uint32_t* digit_offsets;
    unsigned int* err;
};

__global__ void __launch_bounds__(1024)
k_tile_finish(GridFinish g0, GridFinish g1, const int64_t* __restrict__ pairs, int64_t capacity) {
    const GridFinish& G = blockIdx.x == 0 ? g0 : g1;  // one block per grid
    const int* __restrict__ diff = G.diff;
    const int tiles_x = G.tiles_x, tiles_y = G.tiles_y, npass = G.npass;
    int2* __restrict__ ranges = G.ranges;
    uint32_t* __restrict__ digit_offsets = G.digit_offsets;
    unsigned int* __restrict__ err = G.err;
    __shared__ uint32_t s_rows[kMaxTileRows];
    __shared__ uint32_t s_hist[4][256];
    __shared__ uint32_t smem[33];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int gw = tiles_x + 1;
    if (*pairs > capacity) {
        if (threadIdx.x == 0 && err != nullptr) atomicOr(err, DEV_OVERFLOW);
        for (int t = threadIdx.x; t < tiles_x * tiles_y; t += blockDim.x) ranges[t] = make_int2(0, 0);
        for (int i = threadIdx.x; i < npass * 256; i += blockDim.x) digit_offsets[i] = 0u;
        return;
    }
    for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) (&s_hist[0][0])[i] = 0u;
    __syncthreads();
    for (int y = warp; y < tiles_y; y += nwarps) {
        int carry_c = 0;
        uint32_t carry_s = 0u;
        for (int x0 = 0; x0 < tiles_x; x0 += 32) {
            const int x = x0 + lane;
            int v = (x < tiles_x) ? diff[y * gw + x] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += t;
            }
            const int c = v + carry_c;
            carry_c = __shfl_sync(0xffffffffu, c, 31);
            const uint32_t cu = (x < tiles_x) ? (uint32_t)c : 0u;
            uint32_t s = cu;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += t;
            }
            const uint32_t ex = carry_s + s - cu;
            carry_s += __shfl_sync(0xffffffffu, s, 31);
            if (x < tiles_x) {
                const uint32_t t = (uint32_t)(y * tiles_x + x);
                ranges[t] = make_int2((int)ex, (int)cu);
                if (cu != 0u)
                    for (int p = 0; p < npass; ++p) atomicAdd(&s_hist[p][(t >> (8 * p)) & 255u], cu);
            }
        }
        if (lane == 0) s_rows[y] = carry_s;
    }
    __syncthreads();
    {   // exclusive scan of the row totals, up to 4 rows per thread
        constexpr int kPer = kMaxTileRows / 1024;
        uint32_t loc[kPer], sum = 0u;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int y = threadIdx.x * kPer + k;
            loc[k] = (y < tiles_y) ? s_rows[y] : 0u;
            sum += loc[k];
        }
        uint32_t tot;
        uint32_t ex = block_exclusive_scan<uint32_t>(sum, smem, &tot);
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int y = threadIdx.x * kPer + k;
            if (y < tiles_y) s_rows[y] = ex;
            ex += loc[k];
        }
    }
    __syncthreads();
    const int T = tiles_x * tiles_y;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const int2 r = ranges[t];
        const int start = (int)s_rows[t / tiles_x] + r.x;
        ranges[t] = (r.y != 0) ? make_int2(start, start + r.y) : make_int2(0, 0);
    }
    for (int p = 0; p < npass; ++p) {
        uint32_t v = (threadIdx.x < 256) ? s_hist[p][threadIdx.x] : 0u;
        uint32_t tot;
        const uint32_t ex = block_exclusive_scan<uint32_t>(v, smem, &tot);
        if (threadIdx.x < 256) digit_offsets[p * 256 + threadIdx.x] = ex;
    }
}

void launch_project(const GConst& P, int64_t n, int64_t row_begin, int64_t row_end,
                    const TCam* cams, int n_views, const TCfg& cfg, const ProjView& pv,
                    int64_t* blk, int64_t blk_stride, uint64_t* touch, float* vis_counts,
                    float* grad2d, cudaStream_t st) {
    if (row_end <= row_begin) return;
    const unsigned int nb = div_up(row_end - row_begin, kProjThreads);
    const size_t smem = (size_t)kProjThreads * 3 * cfg.K * sizeof(float);
#define GS_PROJ(D_)                                                                        \
    k_train_project<D_><<<nb, kProjThreads, smem, st>>>(P, n, row_begin, row_end, cams,     \
                                                        n_views, cfg, pv, blk, blk_stride, \
                                                        touch, vis_counts, grad2d)
    switch (cfg.sh_degree) {
        case 0: GS_PROJ(0); break;
        case 1: GS_PROJ(1); break;
        case 2: GS_PROJ(2); break;
        default:
            cudaFuncSetAttribute(k_train_project<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            GS_PROJ(3);
            break;
    }
#undef GS_PROJ
}

// The per-tile lists from the super-tile lists: one block per super-tile of 2^SX x 2^SY
// tiles, its items (Gaussian id << Q | mask of the super-tile's Q tiles its rectangle
// covers, in depth order) split into one contiguous part per warp. Each warp counts its part's items per
// tile, one barrier gives every warp its offsets, and each warp walks its part again 32
// items at a time, appending each item to the lists of the tiles in its mask, in order (a
// ballot per tile gives every lane its slot; the lanes of a tile store to consecutive ids).
// Every tile's list is then the depth-ordered list of the Gaussians covering it, exactly
// what a stable sort of all (tile, Gaussian) pairs by tile gives. Loads run kFilterAhead
// steps ahead. Nothing is written when the view's pairs exceed the capacity (the ranges are
// empty then).
template <int SX, int SY>
__global__ void __launch_bounds__(kFilterThreads)
k_tile_filter(const uint32_t* __restrict__ super_sorted, const int2* __restrict__ sranges,
              const int2* __restrict__ ranges, int tiles_x, int tiles_y,
              const int64_t* __restrict__ pairs, int64_t capacity,
              uint32_t* __restrict__ svals) {
    constexpr int NW = kFilterThreads / 32;
    constexpr int Q = (1 << SX) * (1 << SY);  // tiles per super-tile = mask bits
    __shared__ uint32_t s_cnt[NW][Q];
    if (*pairs > capacity) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sid = blockIdx.x;
    const int2 sr = sranges[sid];
    if (sr.y <= sr.x) return;
    const int len = sr.y - sr.x;
    const int beg = sr.x + (int)((int64_t)len * warp / NW);
    const int end = sr.x + (int)((int64_t)len * (warp + 1) / NW);
    const uint32_t lt = (1u << lane) - 1u;
    uint32_t c[Q];
#pragma unroll
    for (int q = 0; q < Q; ++q) c[q] = 0u;
    for (int k0 = beg; k0 < end; k0 += 32 * kFilterAhead) {
        uint32_t v[kFilterAhead];
#pragma unroll
        for (int a = 0; a < kFilterAhead; ++a) {
            const int k = k0 + a * 32 + lane;
            v[a] = (k < end) ? super_sorted[k] : 0u;
        }
#pragma unroll
        for (int a = 0; a < kFilterAhead; ++a)
#pragma unroll
            for (int q = 0; q < Q; ++q) c[q] += (v[a] >> q) & 1u;
    }
#pragma unroll
    for (int q = 0; q < Q; ++q) {
        const uint32_t t = __reduce_add_sync(0xffffffffu, c[q]);
        if (lane == 0) s_cnt[warp][q] = t;
    }
    __syncthreads();
    const int sx_n = super_cells(tiles_x, SX);
    const int tx0 = (sid % sx_n) << SX, ty0 = (sid / sx_n) << SY;
    uint32_t* dst[Q];
#pragma unroll
    for (int q = 0; q < Q; ++q) {
        const int tx = tx0 + (q & ((1 << SX) - 1)), ty = ty0 + (q >> SX);
        uint32_t off = 0u;
        for (int w = 0; w < warp; ++w) off += s_cnt[w][q];
        // a tile outside the grid is in no item's mask
        dst[q] = svals + ((tx < tiles_x && ty < tiles_y) ? ranges[ty * tiles_x + tx].x : 0) + off;
    }
    for (int k0 = beg; k0 < end; k0 += 32 * kFilterAhead) {
        uint32_t v[kFilterAhead];
#pragma unroll
        for (int a = 0; a < kFilterAhead; ++a) {
            const int k = k0 + a * 32 + lane;
            v[a] = (k < end) ? super_sorted[k] : 0u;
        }
#pragma unroll
        for (int a = 0; a < kFilterAhead; ++a) {
            // an item's mask is a rectangle of the super-tile's tiles, so the lanes holding
            // tile (row, column) are those covering the row and the column: W + H ballots
            // instead of one per tile
            constexpr int W = 1 << SX, H = 1 << SY;
            constexpr uint32_t kRow = (1u << W) - 1u;
            uint32_t spread = 0u;  // bit r * W of every row r
#pragma unroll
            for (int r = 0; r < H; ++r) spread |= 1u << (r * W);
            uint32_t br[H], bc[W];
#pragma unroll
            for (int r = 0; r < H; ++r) br[r] = __ballot_sync(0xffffffffu, (v[a] >> (r * W)) & kRow);
#pragma unroll
            for (int c = 0; c < W; ++c) bc[c] = __ballot_sync(0xffffffffu, (v[a] >> c) & spread);
            const uint32_t gid = v[a] >> Q;
#pragma unroll
            for (int q = 0; q < Q; ++q) {
                const uint32_t b = br[q / W] & bc[q % W];
                if ((b >> lane) & 1u) dst[q][__popc(b & lt)] = gid;
                dst[q] += __popc(b);
            }
        }
    }
}

void launch_sorted_count(const ProjView& pv, const uint32_t* order, int64_t n, int sx, int sy,
                         ushort4* rect_d, uint32_t* ccnt, int64_t* blk, cudaStream_t st) {
    k_sorted_count<<<div_up(n, kProjThreads), kProjThreads, 0, st>>>(pv.rect, order, n,
                                                                    sx, sy, rect_d, ccnt, blk);
}

void launch_pair_offsets(const uint32_t* ccnt, int64_t n, const int64_t* blk_offsets,
                         int64_t capacity, uint32_t* goff, uint32_t* tfirst, int64_t tfirst_len,
                         uint32_t* last, int64_t* total, unsigned int* err, cudaStream_t st) {
    k_pair_offsets<<<div_up(n, kProjThreads), kProjThreads, 0, st>>>(
        ccnt, n, blk_offsets, capacity, goff, tfirst, tfirst_len, last, total, err);
}

// Sized for the finest super-tile grid (2x2 tiles); coarser grids use less of it.
int tile_diff_ints(int tiles_x, int tiles_y) {
    return (tiles_x + 1) * tiles_y + (super_cells(tiles_x, 1) + 1) * super_cells(tiles_y, 1);
}

gs_status launch_tile_counts(const ProjView& pv, int64_t n, int tiles_x, int tiles_y, int sx,
                             int sy, int npass, const int64_t* pairs, int64_t capacity, int* diff,
                             int2* ranges, int2* super_ranges, uint32_t* digit_offsets,
                             unsigned int* err, cudaStream_t st) {
    // the direct (Gaussian, tile) sort (sx = sy = 0) sorts by tiles; the super-tile ranges
    // it does not use are still formed on the 2x2 grid
    const bool direct = (sx | sy) == 0;
    if (direct) sx = sy = 1;
    const int bins = tile_diff_ints(tiles_x, tiles_y);
    constexpr int kSmemBins = 40960;  // 160 KB
    const size_t smem = bins <= kSmemBins ? (size_t)bins * sizeof(int) : 0;
    GS_CUDA_CHECK(cudaMemsetAsync(diff, 0, (size_t)bins * sizeof(int), st));
    GS_CUDA_CHECK(cudaFuncSetAttribute(k_tile_diff, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)(kSmemBins * sizeof(int))));
#ifndef GS_TILE_DIFF_BLOCKS_PER_SM
#define GS_TILE_DIFF_BLOCKS_PER_SM 2
#endif
    // every block merges its shared copy into the global arrays with atomics, so fewer
    // blocks mean fewer merges
    const int grid = (int)std::min<int64_t>(GS_TILE_DIFF_BLOCKS_PER_SM * kNumSMs, div_up(n, 1024));
    k_tile_diff<<<grid, 1024, smem, st>>>(pv.rect, n, tiles_x, tiles_y, sx, sy,
                                          smem ? kSmemBins : 0, diff);
    GS_CHECK_LAUNCH();
    // block 0: tile ranges; block 1: super-tile ranges; the sort's digit offsets from the
    // grid it sorts by
    const int sx_n = super_cells(tiles_x, sx), sy_n = super_cells(tiles_y, sy);
    const GridFinish tiles{diff, tiles_x, tiles_y, direct ? npass : 0, ranges,
                           direct ? digit_offsets : nullptr, err};
    const GridFinish supers{diff + (tiles_x + 1) * tiles_y, sx_n, sy_n, direct ? 0 : npass,
                            super_ranges, direct ? nullptr : digit_offsets, nullptr};
    k_tile_finish<<<2, 1024, 0, st>>>(tiles, supers, pairs, capacity);
    GS_CHECK_LAUNCH();
    return GS_OK;
}

gs_status launch_tile_filter(const uint32_t* super_sorted, const int2* super_ranges,
                             const int2* ranges, int tiles_x, int tiles_y, int sx, int sy,
                             const int64_t* pairs, int64_t capacity, uint32_t* svals,
                             cudaStream_t st) {
    const int nsuper = super_cells(tiles_x, sx) * super_cells(tiles_y, sy);
#define GS_FILTER(SX_, SY_)                                                                  \
    k_tile_filter<SX_, SY_><<<nsuper, kFilterThreads, 0, st>>>(super_sorted, super_ranges,   \
                                                               ranges, tiles_x, tiles_y,     \
                                                               pairs, capacity, svals)
    if (sx == 1 && sy == 1) {
        GS_FILTER(1, 1);
    } else if (sx == 2 && sy == 1) {
        GS_FILTER(2, 1);
    } else {
        set_error("tile filter: unsupported super-tile shape %dx%d", 1 << sx, 1 << sy);
        return GS_ERR_ARG;
    }
#undef GS_FILTER
    GS_CHECK_LAUNCH();
    return GS_OK;
}

}  // namespace gs
