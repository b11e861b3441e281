// train_project.cu -- training-path projection and (Gaussian, tile) key emission.
//
// Compiled with -fmad=false: every fp32 product and sum rounds separately, in the
// operation order of the oracle's projection (the reference's fp32 lane model,
// gsplat/t2_param_backward.py:81-120, with its sums written out), and exp is evaluated
// in double and rounded once. Projected means, conics and tile rectangles -- hence pair
// counts, keys and tile ranges -- are then bit-identical to the oracle's.
#include "scan.cuh"
#include "train.cuh"

namespace gs {

__device__ __forceinline__ float exp_rounded(float x) { return (float)exp((double)x); }

// SH coefficients of a block's Gaussians are staged in shared memory with coalesced 16-byte
// loads (the block's rows are one contiguous run of 3 K floats each); each thread then
// reads its own row from shared memory.
template <int DEG>
__global__ void __launch_bounds__(kProjThreads)
k_train_project(GConst P, int64_t n, TCam cam, TCfg cfg, int view, ProjView pv,
                int64_t* __restrict__ blk, uint64_t* __restrict__ touch,
                float* __restrict__ vis_counts, float* __restrict__ grad2d) {
    constexpr int K = (DEG + 1) * (DEG + 1);
    constexpr int ROW = 3 * K;  // floats of SH per Gaussian
    extern __shared__ __align__(16) float s_sh[];
    __shared__ int64_t smem[33];
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    {
        const int64_t g0 = (int64_t)blockIdx.x * blockDim.x;
        const int rows = (int)min((int64_t)blockDim.x, n - g0);
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
    uint32_t count = 0;
    if (g < n) {
        const float m0 = P.means[3 * g], m1 = P.means[3 * g + 1], m2 = P.means[3 * g + 2];
        const float* R = cam.R;
        const float x = R[0] * m0 + R[1] * m1 + R[2] * m2 + cam.t[0];
        const float y = R[3] * m0 + R[4] * m1 + R[5] * m2 + cam.t[1];
        const float z = R[6] * m0 + R[7] * m1 + R[8] * m2 + cam.t[2];
        const bool valid = z > cfg.near_plane;
        float mx = 0.f, my = 0.f, A = 0.f, B = 0.f, C = 0.f, op = 0.f;
        float col[3] = {0.f, 0.f, 0.f};
        bool visible = false;
        ushort4 rc = make_ushort4(1, 0, 1, 0);
        if (valid) {
            const float iz = 1.0f / z;
            mx = cam.fx * x * iz + cam.cx;
            my = cam.fy * y * iz + cam.cy;
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
            const float s[3] = {exp_rounded(P.ls[3 * g]), exp_rounded(P.ls[3 * g + 1]),
                                exp_rounded(P.ls[3 * g + 2])};
            float M[9];
#pragma unroll
            for (int i = 0; i < 3; ++i)
#pragma unroll
                for (int j = 0; j < 3; ++j) M[3 * i + j] = Rq[3 * i + j] * s[j];
            float S[3][3];
#pragma unroll
            for (int i = 0; i < 3; ++i)
#pragma unroll
                for (int k = i; k < 3; ++k) {
                    S[i][k] = M[3 * i] * M[3 * k] + M[3 * i + 1] * M[3 * k + 1] +
                              M[3 * i + 2] * M[3 * k + 2];
                    S[k][i] = S[i][k];
                }
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
            op = 1.0f / (1.0f + exp_rounded(-P.ol[g]));
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
            const float* sh = s_sh + threadIdx.x * ROW;
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
                const double ts = (double)cfg.tile;
                const double hx = (double)(cfg.tiles_x - 1), hy = (double)(cfg.tiles_y - 1);
                const int x0 = (int)fmin(fmax(trunc((px - rx) / ts), 0.0), hx);
                const int x1 = (int)fmin(fmax(trunc((px + rx) / ts), 0.0), hx);
                const int y0 = (int)fmin(fmax(trunc((py - ry) / ts), 0.0), hy);
                const int y1 = (int)fmin(fmax(trunc((py + ry) / ts), 0.0), hy);
                rc = make_ushort4((unsigned short)x0, (unsigned short)x1, (unsigned short)y0,
                                  (unsigned short)y1);
                count = (uint32_t)((x1 - x0 + 1) * (y1 - y0 + 1));
            }
        }
        pv.p0[g] = make_float4(mx, my, A, B);
        pv.p1[g] = make_float4(C, op, col[0], col[1]);
        pv.p2[g] = col[2];
        pv.dkey[g] = __float_as_uint(z);
        pv.dsort[g] = count > 0 ? __float_as_uint(z) : 0xffffffffu;
        pv.rect[g] = rc;
        pv.cnt[g] = count;
        if (vis_counts != nullptr && visible) vis_counts[g] += 1.0f;
        if (grad2d != nullptr && count > 0) {
            float4* gr = reinterpret_cast<float4*>(grad2d + (size_t)g * kGradStride);
            gr[0] = make_float4(0.f, 0.f, 0.f, 0.f);
            gr[1] = make_float4(0.f, 0.f, 0.f, 0.f);
            gr[2] = make_float4(0.f, 0.f, 0.f, 0.f);
            touch[g] |= (1ull << view);
        }
    }
    int64_t total;
    block_exclusive_scan<int64_t>((int64_t)count, smem, &total);
    if (threadIdx.x == 0) blk[blockIdx.x] = total;
}

// Pair counts of the Gaussians in depth order (`order` = Gaussian ids sorted by depth
// bits, stable), one total per block for the offset scan.
__global__ void __launch_bounds__(kProjThreads)
k_sorted_count(const uint32_t* __restrict__ cnt, const uint32_t* __restrict__ order, int64_t n,
               int64_t* __restrict__ blk) {
    __shared__ int64_t smem[33];
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t c = (i < n) ? cnt[order[i]] : 0u;
    int64_t total;
    block_exclusive_scan<int64_t>((int64_t)c, smem, &total);
    if (threadIdx.x == 0) blk[blockIdx.x] = total;
}

// Pairs of the Gaussians in depth order, each Gaussian's tiles row-major: key = tile id,
// value = Gaussian id. A stable sort on the tile id then yields the reference's
// (tile, depth bits, Gaussian id) order (src/gsplat_cpu/sort.cpp:24-27).
// Warp-cooperative: the warp's 32 Gaussians own one contiguous run of pairs, and lane l
// writes pairs l, l + 32, ... of that run (finding its Gaussian by a binary search over
// the warp's offsets), so consecutive lanes store to consecutive addresses.
__global__ void __launch_bounds__(kProjThreads)
k_train_emit(ProjView pv, const uint32_t* __restrict__ order, int64_t n, int tiles_x,
             const int64_t* __restrict__ blk_offsets, int64_t capacity,
             uint32_t* __restrict__ keys, uint32_t* __restrict__ vals,
             unsigned int* __restrict__ err) {
    __shared__ int64_t smem[33];
    __shared__ int64_t s_off[kProjThreads];   // first pair of each thread's Gaussian
    __shared__ uint32_t s_gid[kProjThreads];
    __shared__ ushort4 s_rect[kProjThreads];
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t g = (i < n) ? order[i] : 0u;
    const uint32_t c = (i < n) ? pv.cnt[g] : 0u;
    int64_t total;
    const int64_t off = blk_offsets[blockIdx.x] + block_exclusive_scan<int64_t>((int64_t)c, smem, &total);
    s_off[threadIdx.x] = off;
    s_gid[threadIdx.x] = g;
    s_rect[threadIdx.x] = (c > 0) ? pv.rect[g] : make_ushort4(0, 0, 0, 0);
    __syncwarp();
    const int lane = threadIdx.x & 31, wbase = threadIdx.x & ~31;
    const int64_t run0 = __shfl_sync(0xffffffffu, off, 0);
    const int64_t run1 = __shfl_sync(0xffffffffu, off + (int64_t)c, 31);
    if (run1 > capacity) {
        if (c > 0 && off + (int64_t)c > capacity) atomicOr(err, DEV_OVERFLOW);
        return;
    }
    for (int64_t p = run0 + lane; p < run1; p += 32) {
        int lo = 0, hi = 31;  // last lane of the warp whose first pair is <= p
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s_off[wbase + mid] <= p) lo = mid; else hi = mid - 1;
        }
        const ushort4 r = s_rect[wbase + lo];
        const int w = r.y - r.x + 1;
        const int j = (int)(p - s_off[wbase + lo]);
        const int ty = r.z + j / w, tx = r.x + j % w;
        keys[p] = (uint32_t)(ty * tiles_x + tx);
        vals[p] = s_gid[wbase + lo];
    }
}

void launch_project(const GConst& P, int64_t n, const TCam& cam, const TCfg& cfg, int view,
                    const ProjView& pv, int64_t* blk, uint64_t* touch, float* vis_counts,
                    float* grad2d, cudaStream_t st) {
    const unsigned int nb = div_up(n, kProjThreads);
    const size_t smem = (size_t)kProjThreads * 3 * cfg.K * sizeof(float);
    switch (cfg.sh_degree) {
        case 0:
            k_train_project<0><<<nb, kProjThreads, smem, st>>>(P, n, cam, cfg, view, pv, blk, touch, vis_counts, grad2d);
            break;
        case 1:
            k_train_project<1><<<nb, kProjThreads, smem, st>>>(P, n, cam, cfg, view, pv, blk, touch, vis_counts, grad2d);
            break;
        case 2:
            k_train_project<2><<<nb, kProjThreads, smem, st>>>(P, n, cam, cfg, view, pv, blk, touch, vis_counts, grad2d);
            break;
        default:
            cudaFuncSetAttribute(k_train_project<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            k_train_project<3><<<nb, kProjThreads, smem, st>>>(P, n, cam, cfg, view, pv, blk, touch, vis_counts, grad2d);
            break;
    }
}

void launch_sorted_count(const ProjView& pv, const uint32_t* order, int64_t n, int64_t* blk,
                         cudaStream_t st) {
    k_sorted_count<<<div_up(n, kProjThreads), kProjThreads, 0, st>>>(pv.cnt, order, n, blk);
}

void launch_emit(const ProjView& pv, const uint32_t* order, int64_t n, const TCfg& cfg,
                 const int64_t* blk_offsets, int64_t capacity, uint32_t* keys, uint32_t* vals,
                 unsigned int* err, cudaStream_t st) {
    k_train_emit<<<div_up(n, kProjThreads), kProjThreads, 0, st>>>(pv, order, n, cfg.tiles_x,
                                                                   blk_offsets, capacity, keys,
                                                                   vals, err);
}

}  // namespace gs
