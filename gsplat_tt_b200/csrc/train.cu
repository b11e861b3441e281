// train.cu -- training path: rasterisers, loss, projection backward, sparse Adam and
// the gs_train_step orchestration (one stream, no host synchronisation inside a step).
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "radix_sort.cuh"
#include "rect_pairs.cuh"
#include "scan.cuh"
#include "train.cuh"

namespace gs {

// ------------------------------------------------------------------ host helpers

TCam make_tcam(const gs_camera& c) {
    TCam t;
    const float* w = c.w2c;
    const float R[9] = {w[0], w[1], w[2], w[4], w[5], w[6], w[8], w[9], w[10]};
    memcpy(t.R, R, sizeof(R));
    t.t[0] = w[3];
    t.t[1] = w[7];
    t.t[2] = w[11];
    t.fx = c.K[0];
    t.fy = c.K[4];
    t.cx = c.K[2];
    t.cy = c.K[5];
    for (int j = 0; j < 3; ++j) {  // camera centre -R^T t, in double, rounded once
        double acc = 0.0;
        for (int i = 0; i < 3; ++i) acc += (double)R[3 * i + j] * (double)t.t[i];
        t.cc[j] = (float)(-acc);
    }
    t.H = c.height;
    t.W = c.width;
    return t;
}

TCfg make_tcfg(const gs_train_config& c, int H, int W) {
    TCfg t;
    t.sh_degree = c.sh_degree;
    t.K = (c.sh_degree + 1) * (c.sh_degree + 1);
    t.tile = c.tile_size;
    t.tiles_x = (W + c.tile_size - 1) / c.tile_size;
    t.tiles_y = (H + c.tile_size - 1) / c.tile_size;
    t.near_plane = c.near_plane;
    t.lowpass = c.lowpass;
    t.amax = c.alpha_max;
    t.amin = c.alpha_min;
    t.tmin = c.t_min;
    for (int i = 0; i < 3; ++i) t.bg[i] = c.background[i];
    return t;
}

// ------------------------------------------------------------------ rasterisers

// One pair staged in shared memory: the tile-centred power polynomial
// (gsplat/blend_backward_ref.py:68-92), opacity and colour.
struct __align__(16) RPair {
    float Af, Bf, Cf, P0, Lx, Ly, op, r, g, b;
    uint32_t rows, cols;  // tile rows / columns with a pixel centre that can reach alpha_min
};

// Rows and columns of a TILE x TILE tile whose pixel centres can reach alpha >= amin for
// this pair: alpha <= op exp(-m2 / 2), so a pixel can be live only if
// m2 <= 2 ln(op / amin). Per row (column) the minimum of the quadratic form over the
// row's (column's) centres is taken exactly; the test keeps a slack far above the fp32
// error of both this bound and the per-pixel power (1e-4 of the form's magnitude plus
// 0.02), so a skipped pixel is one the per-pixel test would skip too: results do not change.
template <int TILE>
__device__ __forceinline__ void reach_masks(float A, float B, float C, float op, float mxl,
                                            float myl, float amin, uint32_t& rows,
                                            uint32_t& cols) {
    rows = 0u;
    cols = 0u;
    if (!(op >= amin)) return;
    if (!(A > 0.0f) || !(C > 0.0f) || !(A * C - B * B > 0.0f)) {
        rows = cols = (TILE == 32) ? 0xffffffffu : ((1u << TILE) - 1u);
        return;
    }
    const float th = 2.0f * __logf(op / amin) + 0.02f;
    const float ulo = 0.5f - mxl, uhi = (float)TILE - 0.5f - mxl;
    const float vlo = 0.5f - myl, vhi = (float)TILE - 0.5f - myl;
    const float iA = 1.0f / A, iC = 1.0f / C;
#pragma unroll 4
    for (int k = 0; k < TILE; ++k) {
        {   // row k: v fixed, minimise over u
            const float v = ((float)k + 0.5f) - myl;
            const float us = fminf(fmaxf(-B * v * iA, ulo), uhi);
            const float m2 = A * us * us + 2.0f * B * us * v + C * v * v;
            const float mag = A * us * us + 2.0f * fabsf(B * us * v) + C * v * v;
            if (m2 - 1e-4f * mag <= th) rows |= 1u << k;
        }
        {   // column k: u fixed, minimise over v
            const float u = ((float)k + 0.5f) - mxl;
            const float vs = fminf(fmaxf(-B * u * iC, vlo), vhi);
            const float m2 = A * u * u + 2.0f * B * u * vs + C * vs * vs;
            const float mag = A * u * u + 2.0f * fabsf(B * u * vs) + C * vs * vs;
            if (m2 - 1e-4f * mag <= th) cols |= 1u << k;
        }
    }
}

// Coefficients in float64 from the fp32 conic and tile-local mean, rounded once.
template <int TILE>
__device__ __forceinline__ RPair stage_pair(float4 p0, float4 p1, float p2, float ox, float oy,
                                            float centre, float amin, float& mxl, float& myl) {
    RPair q;
    mxl = __fsub_rn(p0.x, ox);
    myl = __fsub_rn(p0.y, oy);
    q.Af = __fmul_rn(-0.5f, p0.z);
    q.Bf = -p0.w;
    q.Cf = __fmul_rn(-0.5f, p1.x);
    // float64 without contraction, in the reference's operation order
    // (gsplat/blend_backward_ref.py:79-84), rounded once to fp32.
    const double a = q.Af, b = q.Bf, c = q.Cf;
    const double U0 = __dsub_rn((double)centre, (double)mxl);
    const double V0 = __dsub_rn((double)centre, (double)myl);
    q.P0 = (float)__dadd_rn(__dadd_rn(__dmul_rn(__dmul_rn(a, U0), U0), __dmul_rn(__dmul_rn(b, U0), V0)),
                            __dmul_rn(__dmul_rn(c, V0), V0));
    q.Lx = (float)__dadd_rn(__dmul_rn(__dmul_rn(2.0, a), U0), __dmul_rn(b, V0));
    q.Ly = (float)__dadd_rn(__dmul_rn(b, U0), __dmul_rn(__dmul_rn(2.0, c), V0));
    q.op = p1.y;
    q.r = p1.z;
    q.g = p1.w;
    q.b = p2;
    reach_masks<TILE>(p0.z, p0.w, p1.x, p1.y, mxl, myl, amin, q.rows, q.cols);
    return q;
}

// The forward rasteriser keeps, per pair it stages (at the pair's position in the tile's
// sorted list), the float64-derived coefficients and the reach masks: qc = (P0, Lx, Ly,
// bits of the row mask), qcols = the column mask. The backward, which only replays pairs
// the forward staged, takes them from there instead of recomputing them; the opacity,
// colour and conic are read from the projected records as in stage_pair, so every value
// is identical to the forward's.
__device__ __forceinline__ float4 pack_cache(const RPair& q) {
    return make_float4(q.P0, q.Lx, q.Ly, __uint_as_float(q.rows));
}

__device__ __forceinline__ RPair stage_pair_cached(float4 p0, float4 p1, float p2, float4 qc,
                                                   uint32_t qcols, float ox, float oy,
                                                   float& mxl, float& myl) {
    RPair q;
    mxl = __fsub_rn(p0.x, ox);
    myl = __fsub_rn(p0.y, oy);
    q.Af = __fmul_rn(-0.5f, p0.z);
    q.Bf = -p0.w;
    q.Cf = __fmul_rn(-0.5f, p1.x);
    q.P0 = qc.x;
    q.Lx = qc.y;
    q.Ly = qc.z;
    q.op = p1.y;
    q.r = p1.z;
    q.g = p1.w;
    q.b = p2;
    q.rows = __float_as_uint(qc.w);
    q.cols = qcols;
    return q;
}

// power = P0 + du (Lx + Af du + Bf dv) + dv (Ly + Cf dv), every product and sum rounded
// separately in the reference's order (gsplat/blend_backward_ref.py:88-92): the forward and
// backward kernels and the oracle evaluate bit-identical powers, so only exp can move a
// forward decision. `lx_af` = Lx + Af du is shared by the pixels of one column.
__device__ __forceinline__ float centred_power(const RPair& q, float lx_af, float du, float dv) {
    const float inner = __fadd_rn(lx_af, __fmul_rn(q.Bf, dv));
    const float e6 = __fadd_rn(q.P0, __fmul_rn(du, inner));
    const float e8 = __fadd_rn(q.Ly, __fmul_rn(q.Cf, dv));
    return __fadd_rn(e6, __fmul_rn(dv, e8));
}
__device__ __forceinline__ float lx_plus_af_du(const RPair& q, float du) {
    return __fadd_rn(q.Lx, __fmul_rn(q.Af, du));
}

// centred_power for two pixels of one column at once with Blackwell's packed fp32x2
// operations: each lane rounds exactly as the scalar version does.
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 centred_power2(const RPair& q, float lx_af, float du, float2 dv) {
    const float2 inner = __fadd2_rn(f2(lx_af), __fmul2_rn(f2(q.Bf), dv));
    const float2 e6 = __fadd2_rn(f2(q.P0), __fmul2_rn(f2(du), inner));
    const float2 e8 = __fadd2_rn(f2(q.Ly), __fmul2_rn(f2(q.Cf), dv));
    return __fadd2_rn(e6, __fmul2_rn(dv, e8));
}

// Pixel layout of the rasterisers: a TILE x TILE tile is covered by TILE*TILE/PPT threads;
// thread t owns column t % TILE and the PPT consecutive rows (t / TILE) * PPT + i. One pair
// read from shared memory then serves PPT pixels, and the pair's row/column reach masks
// decide per thread (and per warp) whether any of them needs evaluating.
template <int TILE, int PPT>
struct PixLayout {
    static constexpr int kThreads = TILE * TILE / PPT;
    static constexpr uint32_t kBandMask = (1u << PPT) - 1u;
};

// Pixels per thread and pairs staged per batch of the forward and backward rasterisers
// (4 pixels per thread: 64 threads per 16x16 tile).
#ifndef GS_FWD_PPT
#define GS_FWD_PPT 4
#endif
#ifndef GS_BWD_PPT
#define GS_BWD_PPT 4
#endif
#ifndef GS_FWD_BATCH
#define GS_FWD_BATCH 128
#endif
#ifndef GS_BWD_BATCH
#define GS_BWD_BATCH 128
#endif
constexpr int kFwdPPT = GS_FWD_PPT;
constexpr int kBwdPPT = GS_BWD_PPT;
constexpr int kFwdBatch = GS_FWD_BATCH;
constexpr int kBwdBatch = GS_BWD_BATCH;

template <int TILE, int PPT>
__global__ void __launch_bounds__(TILE * TILE / PPT)
k_train_fwd(const int2* __restrict__ ranges, const uint32_t* __restrict__ svals, ProjView pv,
            TCfg cfg, int H, int W, float* __restrict__ image, float* __restrict__ final_T,
            int32_t* __restrict__ n_contrib, float4* __restrict__ qc,
            uint32_t* __restrict__ qcols) {
    using LY = PixLayout<TILE, PPT>;
    constexpr int NB = kFwdBatch;
    constexpr int NP = PPT / 2;  // pixel pairs per thread, each blended with packed fp32x2 math
    static_assert(PPT % 2 == 0, "pixels are processed in pairs");
    __shared__ RPair sp[NB];
    const int tile = blockIdx.x;
    const int tx = tile % cfg.tiles_x, ty = tile / cfg.tiles_x;
    const int lx = threadIdx.x % TILE, ly0 = (threadIdx.x / TILE) * PPT;
    const int x = tx * TILE + lx;
    const float centre = 0.5f * TILE;
    const float du = ((float)lx + 0.5f) - centre;
    const float ox = (float)(tx * TILE), oy = (float)(ty * TILE);
    const int2 rg = ranges[tile];
    const float amax = cfg.amax, amin = cfg.amin, tmin = cfg.tmin;
    float2 dv[NP], T[NP], cr[NP], cg[NP], cb[NP];
    int last[PPT];
    unsigned live_mask = 0;  // pixels still blending
#pragma unroll
    for (int h = 0; h < NP; ++h) {
        dv[h] = make_float2(((float)(ly0 + 2 * h) + 0.5f) - centre,
                            ((float)(ly0 + 2 * h + 1) + 0.5f) - centre);
        T[h] = f2(1.0f);
        cr[h] = cg[h] = cb[h] = f2(0.0f);
    }
#pragma unroll
    for (int i = 0; i < PPT; ++i) {
        last[i] = 0;
        if (x < W && ty * TILE + ly0 + i < H) live_mask |= 1u << i;
    }
    for (int b0 = rg.x; b0 < rg.y; b0 += NB) {
        __syncthreads();
        for (int s = threadIdx.x; s < NB && b0 + s < rg.y; s += LY::kThreads) {
            const uint32_t g = svals[b0 + s];
            float mxl, myl;
            const RPair q = stage_pair<TILE>(pv.p0[g], pv.p1[g], pv.p2[g], ox, oy, centre, amin, mxl, myl);
            sp[s] = q;
            qc[b0 + s] = pack_cache(q);
            qcols[b0 + s] = q.cols;
        }
        __syncthreads();
        const int nb = min(NB, rg.y - b0);
        for (int j = 0; j < nb && live_mask; ++j) {
            const RPair q = sp[j];
            const uint32_t reach = ((q.cols >> lx) & 1u) ? (q.rows >> ly0) & LY::kBandMask : 0u;
            const uint32_t todo = reach & live_mask;
            if (!todo) continue;
            const float t1 = lx_plus_af_du(q, du);  // shared by the thread's pixels
#pragma unroll
            for (int h = 0; h < NP; ++h) {
                const uint32_t tb = (todo >> (2 * h)) & 3u;
                if (!tb) continue;
                const float2 power = centred_power2(q, t1, du, dv[h]);
                const float2 w = make_float2(__expf(fminf(power.x, 0.0f)), __expf(fminf(power.y, 0.0f)));
                const float2 ow = __fmul2_rn(f2(q.op), w);
                const float2 alpha = make_float2(fminf(ow.x, amax), fminf(ow.y, amax));
                const float2 Tn = __fmul2_rn(T[h], __fadd2_rn(f2(1.0f), make_float2(-alpha.x, -alpha.y)));
                const bool h0 = (tb & 1u) && alpha.x >= amin, h1 = (tb & 2u) && alpha.y >= amin;
                const bool s0 = h0 && Tn.x < tmin, s1 = h1 && Tn.y < tmin;  // pixel stops
                const bool u0 = h0 && !s0, u1 = h1 && !s1;                  // pixel blends
                if (s0) live_mask &= ~(1u << (2 * h));
                if (s1) live_mask &= ~(1u << (2 * h + 1));
                if (!(u0 || u1)) continue;
                const float2 at0 = __fmul2_rn(alpha, T[h]);
                const float2 at = make_float2(u0 ? at0.x : 0.0f, u1 ? at0.y : 0.0f);
                cr[h] = __ffma2_rn(at, f2(q.r), cr[h]);
                cg[h] = __ffma2_rn(at, f2(q.g), cg[h]);
                cb[h] = __ffma2_rn(at, f2(q.b), cb[h]);
                T[h] = make_float2(u0 ? Tn.x : T[h].x, u1 ? Tn.y : T[h].y);
                const int idx = b0 - rg.x + j + 1;
                if (u0) last[2 * h] = idx;
                if (u1) last[2 * h + 1] = idx;
            }
        }
        if (__syncthreads_count(live_mask != 0) == 0) break;
    }
#pragma unroll
    for (int i = 0; i < PPT; ++i) {
        const int y = ty * TILE + ly0 + i;
        if (x >= W || y >= H) continue;
        const int h = i >> 1;
        const bool hi = i & 1;
        const float Ti = hi ? T[h].y : T[h].x;
        const size_t o = (size_t)y * W + x;
        image[3 * o] = (hi ? cr[h].y : cr[h].x) + Ti * cfg.bg[0];
        image[3 * o + 1] = (hi ? cg[h].y : cg[h].x) + Ti * cfg.bg[1];
        image[3 * o + 2] = (hi ? cb[h].y : cb[h].x) + Ti * cfg.bg[2];
        final_T[o] = Ti;
        n_contrib[o] = last[i];
    }
}

// Warp sums of nine per-lane values in 14 shuffles instead of 45: a halving transpose
// for values 0-7 (at each step a lane keeps half of its partial sums and sends the other
// half to its partner), a butterfly for value 8. On return lane l with (l & 3) == 0 holds
// the sum of value l >> 2 in s8, and every lane holds the sum of value 8 in s1.
__device__ __forceinline__ void warp_sum9(const float (&v)[9], int lane, float& s8, float& s1) {
    constexpr unsigned kAll = 0xffffffffu;
    const bool b4 = (lane & 16) != 0, b3 = (lane & 8) != 0, b2 = (lane & 4) != 0;
    float a[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float send = b4 ? v[k] : v[k + 4];
        const float keep = b4 ? v[k + 4] : v[k];
        a[k] = keep + __shfl_xor_sync(kAll, send, 16);
    }
    float b[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const float send = b3 ? a[k] : a[k + 2];
        const float keep = b3 ? a[k + 2] : a[k];
        b[k] = keep + __shfl_xor_sync(kAll, send, 8);
    }
    float c = (b2 ? b[1] : b[0]) + __shfl_xor_sync(kAll, b2 ? b[0] : b[1], 4);
    c += __shfl_xor_sync(kAll, c, 2);
    c += __shfl_xor_sync(kAll, c, 1);
    s8 = c;
    float d = v[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(kAll, d, o);
    s1 = d;
}

// The backward's pair records as copied from global memory, before staging: projected
// records p0 / p1 / p2, the forward's coefficient cache qc / qcols, and the Gaussian id.
struct __align__(16) BRaw {  // 64 bytes
    float4 p0, p1, qc;
    float p2;
    uint32_t qcols, gid, pad;
};

// Asynchronous global -> shared copies (cp.async): 16 bytes through L2 only, or 4 bytes.
__device__ __forceinline__ void cp_async16_cg(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4_ca(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem) : "memory");
}

// 1: the backward copies the next batch's pair records into shared memory with cp.async
// while it replays the current batch, and loads the Gaussian ids of the batch after that
// into registers; 0: each batch's records are loaded synchronously between two barriers.
#ifndef GS_BWD_PREFETCH
#define GS_BWD_PREFETCH 0
#endif
// Minimum resident blocks per SM the backward's register budget is set for (0: none).
#ifndef GS_BWD_MIN_BLOCKS
#define GS_BWD_MIN_BLOCKS 0
#endif

struct __align__(16) BPair {  // 80 bytes: five 16-byte shared-memory loads
    RPair q;
    float mxl, myl, A, B, C;
    uint32_t gid;
    float pad[2];
};

// Back-to-front replay (gsplat/blend_backward_ref.py:134-249 terms, recomputed from the
// stored final T and count of processed pairs): per pixel and live pair
//   T_i = T_{i+1} / (1 - a_i),  da = T_i (c.g) - behind / (1 - a_i),  behind += a T_i (c.g)
// with behind starting at T_final (bg.g). The nine per-pixel terms (dopacity, dcolour,
// G u^2, G uv, G v^2, G u, G v with G = dL/dpower) are summed over the thread's PPT pixels
// in registers, over the warp with shuffles, over the tile in shared memory, and added once
// per pair into the view's per-Gaussian rows with float4 atomics.
//
// DET (deterministic mode): instead of the atomics, pair (g, tile) stores its sums in slot
// doff[g] + j, j the tile's row-major index inside g's rectangle (every staged pair, zero
// sums included; the caller zeroes the slots first), and k_det_reduce adds each Gaussian's
// slots in j order. Only for 16x16 tiles: the two warps of such a block add onto zero in
// shared memory, which gives the same bits in either order.
template <int TILE, int PPT, bool DET>
__global__ void __launch_bounds__(TILE * TILE / PPT, TILE == 16 ? GS_BWD_MIN_BLOCKS : 0)
k_train_bwd(const int2* __restrict__ ranges, const uint32_t* __restrict__ svals, ProjView pv,
            TCfg cfg, int H, int W, const float* __restrict__ dimg,
            const float* __restrict__ final_T, const int32_t* __restrict__ n_contrib,
            const float4* __restrict__ qc, const uint32_t* __restrict__ qcols,
            float* __restrict__ grad2d, const int64_t* __restrict__ doff,
            float4* __restrict__ dslots, int64_t slot_cap) {
    static_assert(!DET || (TILE == 16 && TILE * TILE / PPT <= 64),
                  "the deterministic mode needs at most two warps per tile");
    using LY = PixLayout<TILE, PPT>;
    constexpr int NB = kBwdBatch;
    constexpr int NP = PPT / 2;  // pixel pairs per thread (packed fp32x2 math)
    static_assert(PPT % 2 == 0, "pixels are processed in pairs");
    __shared__ BPair sp[NB];
    __shared__ float acc[9][NB + 1];  // rows one bank apart: the 8-lane atomics hit 8 banks
    __shared__ int s_max;
    const int tile = blockIdx.x;
    const int tx = tile % cfg.tiles_x, ty = tile / cfg.tiles_x;
    const int lx = threadIdx.x % TILE, ly0 = (threadIdx.x / TILE) * PPT;
    const int x = tx * TILE + lx;
    const float centre = 0.5f * TILE;
    const float du = ((float)lx + 0.5f) - centre;
    const float xx = (float)lx + 0.5f;
    const float ox = (float)(tx * TILE), oy = (float)(ty * TILE);
    const int2 rg = ranges[tile];
    const int lane = threadIdx.x & 31;
    const float amax = cfg.amax, amin = cfg.amin;
    float2 dv[NP], yy[NP], T[NP], g0[NP], g1[NP], g2[NP], behind[NP];
    int last[PPT];
    int my_max = 0;
#pragma unroll
    for (int i = 0; i < PPT; ++i) {
        const int ly = ly0 + i;
        const int y = ty * TILE + ly;
        float Ti = 1.0f, a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, bh = 0.0f;
        last[i] = 0;
        if (x < W && y < H) {
            const size_t o = (size_t)y * W + x;
            Ti = final_T[o];
            last[i] = n_contrib[o];
            a0 = dimg[3 * o];
            a1 = dimg[3 * o + 1];
            a2 = dimg[3 * o + 2];
            bh = Ti * (cfg.bg[0] * a0 + cfg.bg[1] * a1 + cfg.bg[2] * a2);
            my_max = max(my_max, last[i]);
        }
        float2& d2 = dv[i >> 1];
        float2& y2 = yy[i >> 1];
        float2& t2 = T[i >> 1];
        float2& e0 = g0[i >> 1];
        float2& e1 = g1[i >> 1];
        float2& e2 = g2[i >> 1];
        float2& b2 = behind[i >> 1];
        if (i & 1) {
            d2.y = ((float)ly + 0.5f) - centre; y2.y = (float)ly + 0.5f; t2.y = Ti;
            e0.y = a0; e1.y = a1; e2.y = a2; b2.y = bh;
        } else {
            d2.x = ((float)ly + 0.5f) - centre; y2.x = (float)ly + 0.5f; t2.x = Ti;
            e0.x = a0; e1.x = a1; e2.x = a2; b2.x = bh;
        }
    }
    if (threadIdx.x == 0) s_max = 0;
    __syncthreads();
    if (my_max > 0) atomicMax(&s_max, my_max);
    __syncthreads();
    const int maxl = s_max;
#if GS_BWD_PREFETCH
    // Batches run back to front: batch b is [max(0, maxl - (b + 1) NB), maxl - b NB). Thread t
    // stages slots t + k kThreads of a batch. While batch b is replayed, batch b + 1's
    // records are in flight (cp.async into raw) and batch b + 2's ids in registers.
    constexpr int kSPT = (NB + LY::kThreads - 1) / LY::kThreads;
    __shared__ BRaw raw[NB];
    uint32_t gnext[kSPT];
    auto load_ids = [&](int hi_) {
        const int lo_ = max(0, hi_ - NB);
#pragma unroll
        for (int k = 0; k < kSPT; ++k) {
            const int s = threadIdx.x + k * LY::kThreads;
            gnext[k] = (hi_ > 0 && s < hi_ - lo_) ? svals[rg.x + lo_ + s] : 0u;
        }
    };
    auto issue = [&](int hi_) {
        const int lo_ = max(0, hi_ - NB);
#pragma unroll
        for (int k = 0; k < kSPT; ++k) {
            const int s = threadIdx.x + k * LY::kThreads;
            if (hi_ > 0 && s < hi_ - lo_) {
                const uint32_t g = gnext[k];
                const int64_t pi = (int64_t)rg.x + lo_ + s;
                raw[s].gid = g;
                cp_async16_cg(&raw[s].p0, &pv.p0[g]);
                cp_async16_cg(&raw[s].p1, &pv.p1[g]);
                cp_async16_cg(&raw[s].qc, &qc[pi]);
                cp_async4_ca(&raw[s].p2, &pv.p2[g]);
                cp_async4_ca(&raw[s].qcols, &qcols[pi]);
            }
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };
    if (maxl > 0) {
        load_ids(maxl);
        issue(maxl);
        load_ids(maxl - NB);
    }
#endif
    for (int hi = maxl; hi > 0; hi -= NB) {
        const int lo = max(0, hi - NB);
        const int nb = hi - lo;
#if GS_BWD_PREFETCH
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        __syncthreads();  // every thread's copies of this batch landed; the last epilogue is done
        for (int s = threadIdx.x; s < nb; s += LY::kThreads) {
            const BRaw& r = raw[s];
            const float4 p0 = r.p0, p1 = r.p1;
            BPair bp;
            bp.q = stage_pair_cached(p0, p1, r.p2, r.qc, r.qcols, ox, oy, bp.mxl, bp.myl);
            bp.A = p0.z;
            bp.B = p0.w;
            bp.C = p1.x;
            bp.gid = r.gid;
            sp[s] = bp;
#pragma unroll
            for (int k = 0; k < 9; ++k) acc[k][s] = 0.0f;
        }
        __syncthreads();  // the batch is staged; raw may be refilled
        if (lo > 0) {
            issue(lo);
            load_ids(lo - NB);
        }
#else
        __syncthreads();
        for (int s = threadIdx.x; s < nb; s += LY::kThreads) {
            const uint32_t g = svals[rg.x + lo + s];
            const float4 p0 = pv.p0[g], p1 = pv.p1[g];
            BPair bp;
            bp.q = stage_pair_cached(p0, p1, pv.p2[g], qc[rg.x + lo + s], qcols[rg.x + lo + s], ox,
                                     oy, bp.mxl, bp.myl);
            bp.A = p0.z;
            bp.B = p0.w;
            bp.C = p1.x;
            bp.gid = g;
            sp[s] = bp;
#pragma unroll
            for (int k = 0; k < 9; ++k) acc[k][s] = 0.0f;
        }
        __syncthreads();
#endif
        for (int j = nb - 1; j >= 0; --j) {
            const int idx = lo + j;
            float2 v[9];
#pragma unroll
            for (int k = 0; k < 9; ++k) v[k] = f2(0.0f);
            bool live_any = false;
            const BPair& bp = sp[j];
            const uint32_t reach = (idx < my_max && ((bp.q.cols >> lx) & 1u))
                                       ? (bp.q.rows >> ly0) & LY::kBandMask : 0u;
            if (reach) {
                const RPair q = bp.q;
                const float t1 = lx_plus_af_du(q, du);
                const float u = xx - bp.mxl;
#pragma unroll
                for (int h = 0; h < NP; ++h) {
                    const bool r0 = ((reach >> (2 * h)) & 1u) && idx < last[2 * h];
                    const bool r1 = ((reach >> (2 * h + 1)) & 1u) && idx < last[2 * h + 1];
                    if (!(r0 || r1)) continue;
                    const float2 power = centred_power2(q, t1, du, dv[h]);
                    const float2 w = make_float2(__expf(fminf(power.x, 0.0f)), __expf(fminf(power.y, 0.0f)));
                    const float2 raw = __fmul2_rn(f2(q.op), w);
                    const float2 alpha = make_float2(fminf(raw.x, amax), fminf(raw.y, amax));
                    const bool l0 = r0 && alpha.x >= amin, l1 = r1 && alpha.y >= amin;
                    if (!(l0 || l1)) continue;
                    live_any = true;
                    // d alpha / d power and d alpha / d opacity vanish where alpha is clamped
                    const bool c0 = l0 && !(raw.x > amax), c1 = l1 && !(raw.y > amax);
                    const float2 rr = make_float2(__fdividef(1.0f, 1.0f - alpha.x),
                                                  __fdividef(1.0f, 1.0f - alpha.y));
                    const float2 Ti = __fmul2_rn(T[h], rr);
                    const float2 cgv = __ffma2_rn(f2(q.b), g2[h], __ffma2_rn(f2(q.g), g1[h], __fmul2_rn(f2(q.r), g0[h])));
                    const float2 dalpha = __ffma2_rn(Ti, cgv, make_float2(-behind[h].x * rr.x, -behind[h].y * rr.y));
                    const float2 at0 = __fmul2_rn(alpha, Ti);
                    const float2 at = make_float2(l0 ? at0.x : 0.0f, l1 ? at0.y : 0.0f);
                    behind[h] = __ffma2_rn(at, cgv, behind[h]);
                    T[h] = make_float2(l0 ? Ti.x : T[h].x, l1 ? Ti.y : T[h].y);
                    const float2 dd = make_float2(c0 ? dalpha.x : 0.0f, c1 ? dalpha.y : 0.0f);
                    const float2 G = make_float2(power.x <= 0.0f ? dd.x * alpha.x : 0.0f,
                                                 power.y <= 0.0f ? dd.y * alpha.y : 0.0f);
                    const float2 vv = __fadd2_rn(yy[h], f2(-bp.myl));
                    const float2 Gu = __fmul2_rn(G, f2(u)), Gv = __fmul2_rn(G, vv);
                    v[0] = __ffma2_rn(dd, w, v[0]);
                    v[1] = __ffma2_rn(at, g0[h], v[1]);
                    v[2] = __ffma2_rn(at, g1[h], v[2]);
                    v[3] = __ffma2_rn(at, g2[h], v[3]);
                    v[4] = __ffma2_rn(Gu, f2(u), v[4]);
                    v[5] = __ffma2_rn(Gu, vv, v[5]);
                    v[6] = __ffma2_rn(Gv, vv, v[6]);
                    v[7] = __fadd2_rn(v[7], Gu);
                    v[8] = __fadd2_rn(v[8], Gv);
                }
            }
            if (__any_sync(0xffffffffu, live_any)) {
                float vs[9];
#pragma unroll
                for (int k = 0; k < 9; ++k) vs[k] = v[k].x + v[k].y;
                float s8, s1;
                warp_sum9(vs, lane, s8, s1);
                if ((lane & 3) == 0) atomicAdd(&acc[lane >> 2][j], s8);
                if (lane == 1) atomicAdd(&acc[8][j], s1);
            }
        }
        __syncthreads();
        for (int s = threadIdx.x; s < nb; s += LY::kThreads) {
            const BPair& bp = sp[s];
            const float s0 = acc[0][s], s1 = acc[1][s], s2 = acc[2][s], s3 = acc[3][s];
            const float Suu = acc[4][s], Suv = acc[5][s], Svv = acc[6][s], Su = acc[7][s];
            const float Sv = acc[8][s];
            if constexpr (DET) {
                const ushort4 r = pv.rect[bp.gid];
                const int64_t slot = doff[bp.gid] + (int64_t)(ty - (int)r.z) * ((int)r.y - (int)r.x + 1) +
                                     (tx - (int)r.x);
                if (slot >= 0 && slot < slot_cap) {
                    float4* d = dslots + 3 * slot;
                    d[0] = make_float4(bp.A * Su + bp.B * Sv, bp.B * Su + bp.C * Sv, -0.5f * Suu, -Suv);
                    d[1] = make_float4(-0.5f * Svv, s0, s1, s2);
                    d[2] = make_float4(s3, 0.0f, 0.0f, 0.0f);
                }
            } else if (s0 != 0.0f || s1 != 0.0f || s2 != 0.0f || s3 != 0.0f || Su != 0.0f ||
                       Sv != 0.0f || Suu != 0.0f || Suv != 0.0f || Svv != 0.0f) {
                float4* gr = reinterpret_cast<float4*>(grad2d + (size_t)bp.gid * kGradStride);
                atomicAdd(&gr[0], make_float4(bp.A * Su + bp.B * Sv, bp.B * Su + bp.C * Sv,
                                              -0.5f * Suu, -Suv));
                atomicAdd(&gr[1], make_float4(-0.5f * Svv, s0, s1, s2));
                atomicAdd(&gr[2], make_float4(s3, 0.0f, 0.0f, 0.0f));
            }
        }
    }
}

// Tiles of an inclusive tile rectangle (x0, x1, y0, y1); x1 < x0 means none.
__device__ __forceinline__ int64_t rect_tiles(ushort4 r) {
    return (r.y >= r.x) ? (int64_t)(r.y - r.x + 1) * (int64_t)(r.w - r.z + 1) : 0;
}

// Deterministic mode: each Gaussian's first slot, the exclusive prefix of the tile counts
// in Gaussian order (gsplat/blend_backward_ref.py:32-36 P[g]); blk_off holds the exclusive
// offsets of the projection's 256-Gaussian blocks.
__global__ void __launch_bounds__(kProjThreads)
k_det_offsets(const ushort4* __restrict__ rect, int64_t n, const int64_t* __restrict__ blk_off,
              int64_t* __restrict__ doff) {
    __shared__ int64_t smem[33];
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t c = (i < n) ? rect_tiles(rect[i]) : 0;
    int64_t total;
    const int64_t ex = block_exclusive_scan<int64_t>(c, smem, &total);
    if (i < n) doff[i] = blk_off[blockIdx.x] + ex;
}

// Zero the view's used slots: 3 float4 per pair, pairs = min(*pairs, cap).
__global__ void k_det_zero(float4* __restrict__ slots, const int64_t* __restrict__ pairs,
                           int64_t cap) {
    const int64_t m = 3 * min(*pairs, cap);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m;
         i += (int64_t)gridDim.x * blockDim.x)
        slots[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
}

// Deterministic mode: each Gaussian's 2D-gradient row = its slots summed j = 0, 1, ... in
// fp32 (gsplat/blend_backward_ref.py:239-244), stored over the row the projection zeroed.
__global__ void k_det_reduce(const ushort4* __restrict__ rect, const int64_t* __restrict__ doff,
                             const float4* __restrict__ slots, int64_t n, int64_t cap,
                             float* __restrict__ grad2d) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    const int64_t c = rect_tiles(rect[g]);
    if (c == 0) return;
    const int64_t o = doff[g];
    if (o + c > cap) return;  // overflowed view: its tile lists are empty, nothing was written
    float4 a[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) a[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int64_t j = 0; j < c; ++j) {
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const float4 s = slots[3 * (o + j) + k];
            a[k].x = __fadd_rn(a[k].x, s.x);
            a[k].y = __fadd_rn(a[k].y, s.y);
            a[k].z = __fadd_rn(a[k].z, s.z);
            a[k].w = __fadd_rn(a[k].w, s.w);
        }
    }
    float4* gr = reinterpret_cast<float4*>(grad2d + (size_t)g * kGradStride);
#pragma unroll
    for (int k = 0; k < 3; ++k) gr[k] = a[k];
}

// ------------------------------------------------------------------ loss

constexpr int kHalo = 5;  // half-width of the 11-tap SSIM window

struct LossCfg {
    float taps[11];
    float lambda;   // lambda_dssim
    float inv_n;    // 1 / (3 H W)
    int H, W;
};

// Pure L1 (gsplat/train_loss.py:166-171): grad = (1 - lambda) / n sign(x - y).
__global__ void k_loss_l1(const float* __restrict__ img, const float* __restrict__ tgt, int64_t n3,
                          LossCfg L, float* __restrict__ dimg, double* __restrict__ acc) {
    __shared__ double red[32];
    double s = 0.0;
    const float w = (1.0f - L.lambda) * L.inv_n;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n3;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float d = img[i] - tgt[i];
        s += fabsf(d);
        dimg[i] = w * (float)((d > 0.0f) - (d < 0.0f));
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += red[k];
        atomicAdd(&acc[0], t);
    }
}

// 4-byte asynchronous global -> shared copy (cp.async, no register staging), zero-filled
// when `in` is false (nothing is read then; the source must still be a valid address).
__device__ __forceinline__ void cp_async4(float* smem, const float* gmem, bool in) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem),
                 "r"(in ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// SSIM tiles: 32 x 32 outputs per block of 256 threads, from a (42 x 42) patch (halo 5
// for the 11-tap window). Horizontal pass: a thread filters 4 adjacent outputs of a patch
// row from 14 values held in registers; vertical pass: a thread filters 4 adjacent rows
// of an output column from 14 values. Shared rows are padded to 45 floats, which keeps the
// horizontal pass's four rows per warp on distinct banks.
constexpr int kSsimT = 32;                    // output tile edge
constexpr int kSsimP = kSsimT + 2 * kHalo;    // 42
constexpr int kSsimS = 45;                    // padded patch row stride
constexpr int kSsimHItems = kSsimP * (kSsimT / 4);  // 336 horizontal items of 4 outputs

struct SsimFwdSmem {
    float px[kSsimP][kSsimS];  // one channel's patch of each image
    float py[kSsimP][kSsimS];
    float h[5][kSsimP][kSsimT];
};
struct SsimBwdSmem {
    float p[3][kSsimP][kSsimS];
    float h[3][kSsimP][kSsimT];
};

// SSIM forward + its partial derivatives (gsplat/train_loss.py:126-165): per pixel and
// channel mu_x, mu_y, E_xx, E_yy, E_xy (zero padding), S, and the maps d_mu, d_xx, d_xy
// (scaled by -lambda / n; planar [3][H][W]) that the second pass filters. Sums |x - y|
// and S. The image patch is read once for all three channels, row segments contiguous.
#ifndef GS_SSIM_FWD_BLOCKS
#define GS_SSIM_FWD_BLOCKS 1
#endif
__global__ void __launch_bounds__(256, GS_SSIM_FWD_BLOCKS)
k_ssim_fwd(const float* __restrict__ img, const float* __restrict__ tgt, LossCfg L,
           float* __restrict__ dmu, float* __restrict__ dxx, float* __restrict__ dxy,
           double* __restrict__ acc) {
    extern __shared__ __align__(16) unsigned char ssim_raw[];
    SsimFwdSmem& S = *reinterpret_cast<SsimFwdSmem*>(ssim_raw);
    __shared__ double red[2][8];
    const int tid = threadIdx.x;
    const int x0 = blockIdx.x * kSsimT, y0 = blockIdx.y * kSsimT;
    // One channel's patch of both images at a time, copied asynchronously: channel 0 before
    // the loop, channel ch + 1 once the horizontal pass of channel ch has consumed the
    // patch, so the copies overlap the vertical pass (the other channels' bytes of the
    // interleaved rows are L2 hits by then).
    auto load_patch = [&](int ch) {
        for (int i = tid; i < kSsimP * kSsimP; i += 256) {
            const int r = i / kSsimP, c = i - r * kSsimP;
            const int yy = y0 - kHalo + r, xx = x0 - kHalo + c;
            const bool in = yy >= 0 && yy < L.H && xx >= 0 && xx < L.W;
            const size_t o = in ? ((size_t)yy * L.W + xx) * 3 + ch : 0;
            cp_async4(&S.px[r][c], img + o, in);
            cp_async4(&S.py[r][c], tgt + o, in);
        }
        cp_async_commit();
    };
    load_patch(0);
    double s_l1 = 0.0, s_ssim = 0.0;
    const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
    const float w = -L.lambda * L.inv_n;
    const int vc = tid & 31, vr0 = (tid >> 5) * 4;  // vertical item: column, first of 4 rows
    for (int ch = 0; ch < 3; ++ch) {
        cp_async_wait_all();
        __syncthreads();
        for (int it = tid; it < kSsimHItems; it += 256) {
            const int r = it >> 3, c0 = (it & 7) * 4;
            // (x, y) and (x^2, y^2) filtered as packed fp32x2 pairs, x y on its own
            float2 xy[14], sq[14];
            float pr[14];
#pragma unroll
            for (int k = 0; k < 14; ++k) {
                xy[k] = make_float2(S.px[r][c0 + k], S.py[r][c0 + k]);
                sq[k] = __fmul2_rn(xy[k], xy[k]);
                pr[k] = __fmul_rn(xy[k].x, xy[k].y);
            }
#pragma unroll
            for (int o = 0; o < 4; ++o) {
                float2 a01 = f2(0.0f), a23 = f2(0.0f);
                float a4 = 0.0f;
#pragma unroll
                for (int k = 0; k < 11; ++k) {
                    const float t = L.taps[k];
                    a01 = __ffma2_rn(f2(t), xy[o + k], a01);
                    a23 = __ffma2_rn(f2(t), sq[o + k], a23);
                    a4 = __fmaf_rn(t, pr[o + k], a4);
                }
                S.h[0][r][c0 + o] = a01.x;
                S.h[1][r][c0 + o] = a01.y;
                S.h[2][r][c0 + o] = a23.x;
                S.h[3][r][c0 + o] = a23.y;
                S.h[4][r][c0 + o] = a4;
            }
        }
        float ad[4];  // |x - y| of this thread's 4 pixels, before the patch is overwritten
#pragma unroll
        for (int o = 0; o < 4; ++o)
            ad[o] = fabsf(S.px[vr0 + o + kHalo][vc + kHalo] - S.py[vr0 + o + kHalo][vc + kHalo]);
        __syncthreads();
        if (ch + 1 < 3) load_patch(ch + 1);
        float m[5][4];
#pragma unroll
        for (int q = 0; q < 4; q += 2) {  // quantities (0, 1) and (2, 3) packed
            float2 v[14];
#pragma unroll
            for (int k = 0; k < 14; ++k) v[k] = make_float2(S.h[q][vr0 + k][vc], S.h[q + 1][vr0 + k][vc]);
#pragma unroll
            for (int o = 0; o < 4; ++o) {
                float2 a = f2(0.0f);
#pragma unroll
                for (int k = 0; k < 11; ++k) a = __ffma2_rn(f2(L.taps[k]), v[o + k], a);
                m[q][o] = a.x;
                m[q + 1][o] = a.y;
            }
        }
        {
            float v[14];
#pragma unroll
            for (int k = 0; k < 14; ++k) v[k] = S.h[4][vr0 + k][vc];
#pragma unroll
            for (int o = 0; o < 4; ++o) {
                float a = 0.0f;
#pragma unroll
                for (int k = 0; k < 11; ++k) a = __fmaf_rn(L.taps[k], v[o + k], a);
                m[4][o] = a;
            }
        }
#pragma unroll
        for (int o = 0; o < 4; ++o) {
            const int x = x0 + vc, y = y0 + vr0 + o;
            if (x >= L.W || y >= L.H) continue;
            const float mx = m[0][o], my = m[1][o], exx = m[2][o], eyy = m[3][o], exy = m[4][o];
            const float mxy = mx * my;
            const float A = 2.0f * mxy + C1;
            const float B = 2.0f * (exy - mxy) + C2;
            const float C = mx * mx + my * my + C1;
            const float D = (exx - mx * mx) + (eyy - my * my) + C2;
            const float Sv = (A * B) / (C * D);
            const float Sw = Sv * w;
            const size_t po = ((size_t)ch * L.H + y) * L.W + x;
            dmu[po] = Sw * (2.0f * my / A - 2.0f * my / B - 2.0f * mx / C + 2.0f * mx / D);
            dxx[po] = -Sw / D;
            dxy[po] = 2.0f * Sw / B;
            s_ssim += Sv;
            s_l1 += ad[o];
        }
        __syncthreads();
    }
    for (int o = 16; o > 0; o >>= 1) {
        s_l1 += __shfl_xor_sync(0xffffffffu, s_l1, o);
        s_ssim += __shfl_xor_sync(0xffffffffu, s_ssim, o);
    }
    if ((tid & 31) == 0) {
        red[0][tid >> 5] = s_l1;
        red[1][tid >> 5] = s_ssim;
    }
    __syncthreads();
    if (tid == 0) {
        double a = 0.0, b = 0.0;
        for (int k = 0; k < 8; ++k) { a += red[0][k]; b += red[1][k]; }
        atomicAdd(&acc[0], a);
        atomicAdd(&acc[1], b);
    }
}

// dL/dx = G*d_mu + 2 x G*d_xx + y G*d_xy + (1 - lambda)/n sign(x - y), per channel from
// (42 x 42) patches of the planar maps; written interleaved (H, W, 3) like the image.
__global__ void __launch_bounds__(256, 5)
k_ssim_bwd(const float* __restrict__ img, const float* __restrict__ tgt,
           const float* __restrict__ dmu, const float* __restrict__ dxx,
           const float* __restrict__ dxy, LossCfg L, float* __restrict__ dimg) {
    extern __shared__ __align__(16) unsigned char ssim_raw[];
    SsimBwdSmem& S = *reinterpret_cast<SsimBwdSmem*>(ssim_raw);
    const int tid = threadIdx.x;
    const int x0 = blockIdx.x * kSsimT, y0 = blockIdx.y * kSsimT;
    const float wl1 = (1.0f - L.lambda) * L.inv_n;
    const int vc = tid & 31, vr0 = (tid >> 5) * 4;
    // The three maps' patch of a channel, copied asynchronously: channel 0 before the loop,
    // channel ch + 1 once the horizontal pass of channel ch has consumed the patch, so the
    // copies overlap the vertical pass.
    auto load_patch = [&](int ch) {
        const size_t plane = (size_t)ch * L.H * L.W;
        for (int i = tid; i < kSsimP * kSsimP; i += 256) {
            const int r = i / kSsimP, c = i - r * kSsimP;
            const int yy = y0 - kHalo + r, xx = x0 - kHalo + c;
            const bool in = yy >= 0 && yy < L.H && xx >= 0 && xx < L.W;
            const size_t o = in ? plane + (size_t)yy * L.W + xx : 0;
            cp_async4(&S.p[0][r][c], dmu + o, in);
            cp_async4(&S.p[1][r][c], dxx + o, in);
            cp_async4(&S.p[2][r][c], dxy + o, in);
        }
        cp_async_commit();
    };
    load_patch(0);
    for (int ch = 0; ch < 3; ++ch) {
        cp_async_wait_all();
        __syncthreads();
        for (int it = tid; it < kSsimHItems; it += 256) {
            const int r = it >> 3, c0 = (it & 7) * 4;
            {   // maps 0 and 1 packed
                float2 v[14];
#pragma unroll
                for (int k = 0; k < 14; ++k) v[k] = make_float2(S.p[0][r][c0 + k], S.p[1][r][c0 + k]);
#pragma unroll
                for (int o = 0; o < 4; ++o) {
                    float2 a = f2(0.0f);
#pragma unroll
                    for (int k = 0; k < 11; ++k) a = __ffma2_rn(f2(L.taps[k]), v[o + k], a);
                    S.h[0][r][c0 + o] = a.x;
                    S.h[1][r][c0 + o] = a.y;
                }
            }
            {
                float v[14];
#pragma unroll
                for (int k = 0; k < 14; ++k) v[k] = S.p[2][r][c0 + k];
#pragma unroll
                for (int o = 0; o < 4; ++o) {
                    float a = 0.0f;
#pragma unroll
                    for (int k = 0; k < 11; ++k) a = __fmaf_rn(L.taps[k], v[o + k], a);
                    S.h[2][r][c0 + o] = a;
                }
            }
        }
        __syncthreads();
        if (ch + 1 < 3) load_patch(ch + 1);  // the patch is free: S.h holds this channel now
        // this thread's pixels of the channel, loaded ahead of the vertical pass
        float xv4[4], yv4[4];
#pragma unroll
        for (int o = 0; o < 4; ++o) {
            const int x = x0 + vc, y = y0 + vr0 + o;
            const bool in = x < L.W && y < L.H;
            const size_t io = in ? ((size_t)y * L.W + x) * 3 + ch : 0;
            xv4[o] = in ? img[io] : 0.0f;
            yv4[o] = in ? tgt[io] : 0.0f;
        }
        float m[3][4];
        {
            float2 v[14];
#pragma unroll
            for (int k = 0; k < 14; ++k) v[k] = make_float2(S.h[0][vr0 + k][vc], S.h[1][vr0 + k][vc]);
#pragma unroll
            for (int o = 0; o < 4; ++o) {
                float2 a = f2(0.0f);
#pragma unroll
                for (int k = 0; k < 11; ++k) a = __ffma2_rn(f2(L.taps[k]), v[o + k], a);
                m[0][o] = a.x;
                m[1][o] = a.y;
            }
        }
        {
            float v[14];
#pragma unroll
            for (int k = 0; k < 14; ++k) v[k] = S.h[2][vr0 + k][vc];
#pragma unroll
            for (int o = 0; o < 4; ++o) {
                float a = 0.0f;
#pragma unroll
                for (int k = 0; k < 11; ++k) a = __fmaf_rn(L.taps[k], v[o + k], a);
                m[2][o] = a;
            }
        }
#pragma unroll
        for (int o = 0; o < 4; ++o) {
            const int x = x0 + vc, y = y0 + vr0 + o;
            if (x >= L.W || y >= L.H) continue;
            const size_t io = ((size_t)y * L.W + x) * 3 + ch;
            const float xv = xv4[o], yv = yv4[o];
            const float d = xv - yv;
            dimg[io] = m[0][o] + 2.0f * xv * m[1][o] + yv * m[2][o] +
                       wl1 * (float)((d > 0.0f) - (d < 0.0f));
        }
        __syncthreads();
    }
}

__global__ void k_loss_finalize(const double* __restrict__ acc, LossCfg L, int use_ssim,
                                float* __restrict__ out) {
    const double n = 1.0 / (double)L.inv_n;
    const double l1 = acc[0] / n;
    double loss = (1.0 - (double)L.lambda) * l1;
    if (use_ssim) loss += (double)L.lambda * (1.0 - acc[1] / n);
    *out = (float)loss;
}

// ------------------------------------------------------------------ projection backward

constexpr float kC0 = 0.28209479177387814f, kC1 = 0.4886025119029199f;
__constant__ float c_C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                              -1.0925484305920792f, 0.5462742152960396f};
__constant__ float c_C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                              0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
                              -0.5900435899266435f};

// Real SH basis up to degree `deg` at unit direction (x, y, z) (gsplat/train_oracle.py:99-122).
__device__ __forceinline__ void sh_basis(int deg, float x, float y, float z, float* b) {
    b[0] = kC0;
    if (deg < 1) return;
    b[1] = -kC1 * y;
    b[2] = kC1 * z;
    b[3] = -kC1 * x;
    if (deg < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    const float* c = c_C2;
    b[4] = c[0] * (x * y);
    b[5] = c[1] * (y * z);
    b[6] = c[2] * (2.0f * zz - xx - yy);
    b[7] = c[3] * (x * z);
    b[8] = c[4] * (xx - yy);
    if (deg < 3) return;
    const float* e = c_C3;
    b[9] = e[0] * y * (3.0f * xx - yy);
    b[10] = e[1] * (x * y) * z;
    b[11] = e[2] * y * (4.0f * zz - xx - yy);
    b[12] = e[3] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
    b[13] = e[4] * x * (4.0f * zz - xx - yy);
    b[14] = e[5] * z * (xx - yy);
    b[15] = e[6] * x * (xx - 3.0f * yy);
}

// Gradient with respect to the direction of sum_k w[k] basis_k(x, y, z), term by term.
__device__ __forceinline__ void sh_dir_grad(int deg, float x, float y, float z, const float* w,
                                            float* g) {
    g[0] = g[1] = g[2] = 0.0f;
    if (deg < 1) return;
    g[1] += -kC1 * w[1];
    g[2] += kC1 * w[2];
    g[0] += -kC1 * w[3];
    if (deg < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    const float* c = c_C2;
    g[0] += c[0] * y * w[4]; g[1] += c[0] * x * w[4];
    g[1] += c[1] * z * w[5]; g[2] += c[1] * y * w[5];
    g[0] += -2.0f * c[2] * x * w[6]; g[1] += -2.0f * c[2] * y * w[6]; g[2] += 4.0f * c[2] * z * w[6];
    g[0] += c[3] * z * w[7]; g[2] += c[3] * x * w[7];
    g[0] += 2.0f * c[4] * x * w[8]; g[1] += -2.0f * c[4] * y * w[8];
    if (deg < 3) return;
    const float* e = c_C3;
    g[0] += e[0] * 6.0f * x * y * w[9]; g[1] += e[0] * (3.0f * xx - 3.0f * yy) * w[9];
    g[0] += e[1] * y * z * w[10]; g[1] += e[1] * x * z * w[10]; g[2] += e[1] * x * y * w[10];
    g[0] += -2.0f * e[2] * x * y * w[11]; g[1] += e[2] * (4.0f * zz - xx - 3.0f * yy) * w[11];
    g[2] += 8.0f * e[2] * y * z * w[11];
    g[0] += -6.0f * e[3] * x * z * w[12]; g[1] += -6.0f * e[3] * y * z * w[12];
    g[2] += e[3] * (6.0f * zz - 3.0f * xx - 3.0f * yy) * w[12];
    g[0] += e[4] * (4.0f * zz - 3.0f * xx - yy) * w[13]; g[1] += -2.0f * e[4] * x * y * w[13];
    g[2] += 8.0f * e[4] * x * z * w[13];
    g[0] += 2.0f * e[5] * x * z * w[14]; g[1] += -2.0f * e[5] * y * z * w[14];
    g[2] += e[5] * (xx - yy) * w[14];
    g[0] += e[6] * (3.0f * xx - 3.0f * yy) * w[15]; g[1] += -6.0f * e[6] * x * y * w[15];
}

struct GMut {
    float* means;
    float* ls;
    float* q;
    float* ol;
    float* sh;
};

// Per Gaussian, over every view that gave it 2D gradients: the analytic projection
// backward of gsplat/t2_param_backward.py:123-192 extended with SH bands 1-3 and the
// view-direction term, summed over views. dL/dcov3d, dL/dopacity and the SH gradient
// accumulate across views; the log-scale, quaternion and logit gradients are formed once.
// The geometric part runs in fp64: the covariance gradient cancels strongly along the
// viewing direction (the part of cov3d a view cannot see), and fp32 there leaves errors
// of ~1e-2 relative to the group's largest gradient. SH terms stay fp32. The block's SH
// rows and SH-gradient accumulators live in shared memory (coefficient-major, one padded
// row per coefficient), which keeps the per-thread register state to the fp64 geometry.
constexpr int kParamThreads = 128;
constexpr int kParamStride = kParamThreads + 1;  // shared row stride: consecutive rows one bank apart

template <int DEG>
__global__ void __launch_bounds__(kParamThreads, 4)
k_param_bwd(GConst P, int64_t n, int64_t row_begin, int64_t row_end, const TCam* __restrict__ cams,
            int n_views, TCfg cfg, const float* __restrict__ grad2d,
            const uint64_t* __restrict__ touch, GMut G) {
    // rows [row_begin, row_end) of the n Gaussians (n is the stride of the per-view arrays)
    constexpr int K = (DEG + 1) * (DEG + 1);
    constexpr int ROW = 3 * K;
    extern __shared__ float s_param[];
    float* s_sh = s_param;                          // [ROW][kParamStride]
    float* s_gsh = s_param + ROW * kParamStride;    // [ROW][kParamStride]
    const int tid = threadIdx.x;
    const int64_t g0 = row_begin + (int64_t)blockIdx.x * kParamThreads;
    const int rows = (int)min((int64_t)kParamThreads, row_end - g0);
    for (int i = tid; i < rows * ROW; i += kParamThreads) {
        const int t = i / ROW, c = i - t * ROW;
        s_sh[c * kParamStride + t] = P.sh[g0 * ROW + i];
    }
    for (int c = 0; c < ROW; ++c) s_gsh[c * kParamStride + tid] = 0.0f;
    __syncthreads();
    const int64_t g = g0 + tid;
    if (g < row_end) {
        const uint64_t mask = touch[g];
        double gm[3] = {0.0, 0.0, 0.0};
        double G3[6] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0};  // 00 01 02 11 12 22
        float gop = 0.0f;
        const double m0 = P.means[3 * g], m1 = P.means[3 * g + 1], m2 = P.means[3 * g + 2];
        const float4 q = reinterpret_cast<const float4*>(P.q)[g];
        const double qinv = 1.0 / sqrt((double)q.x * q.x + (double)q.y * q.y + (double)q.z * q.z +
                                       (double)q.w * q.w);
        const double qw = q.x * qinv, qx = q.y * qinv, qy = q.z * qinv, qz = q.w * qinv;
        double Rq[9];
        Rq[0] = 1.0 - 2.0 * (qy * qy + qz * qz);
        Rq[1] = 2.0 * (qx * qy - qw * qz);
        Rq[2] = 2.0 * (qx * qz + qw * qy);
        Rq[3] = 2.0 * (qx * qy + qw * qz);
        Rq[4] = 1.0 - 2.0 * (qx * qx + qz * qz);
        Rq[5] = 2.0 * (qy * qz - qw * qx);
        Rq[6] = 2.0 * (qx * qz - qw * qy);
        Rq[7] = 2.0 * (qy * qz + qw * qx);
        Rq[8] = 1.0 - 2.0 * (qx * qx + qy * qy);
        const double s[3] = {exp((double)P.ls[3 * g]), exp((double)P.ls[3 * g + 1]),
                             exp((double)P.ls[3 * g + 2])};
        double M[9];
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) M[3 * i + j] = Rq[3 * i + j] * s[j];
        double S[6];  // 00 01 02 11 12 22
        S[0] = M[0] * M[0] + M[1] * M[1] + M[2] * M[2];
        S[1] = M[0] * M[3] + M[1] * M[4] + M[2] * M[5];
        S[2] = M[0] * M[6] + M[1] * M[7] + M[2] * M[8];
        S[3] = M[3] * M[3] + M[4] * M[4] + M[5] * M[5];
        S[4] = M[3] * M[6] + M[4] * M[7] + M[5] * M[8];
        S[5] = M[6] * M[6] + M[7] * M[7] + M[8] * M[8];
        for (int v = 0; v < n_views; ++v) {
            if (!((mask >> v) & 1ull)) continue;
            const float* gr = grad2d + ((size_t)v * n + g) * kGradStride;
            const float4 ga4 = reinterpret_cast<const float4*>(gr)[0];
            const float4 gb4 = reinterpret_cast<const float4*>(gr)[1];
            const float gbl = gr[8];
            if (ga4.x == 0.f && ga4.y == 0.f && ga4.z == 0.f && ga4.w == 0.f && gb4.x == 0.f &&
                gb4.y == 0.f && gb4.z == 0.f && gb4.w == 0.f && gbl == 0.f)
                continue;
            const double gmx = ga4.x, gmy = ga4.y, gA = ga4.z, gB = ga4.w, gC = gb4.x;
            const TCam& cam = cams[v];
            double R[9];
#pragma unroll
            for (int k = 0; k < 9; ++k) R[k] = cam.R[k];
            const double x = R[0] * m0 + R[1] * m1 + R[2] * m2 + (double)cam.t[0];
            const double y = R[3] * m0 + R[4] * m1 + R[5] * m2 + (double)cam.t[1];
            const double z = R[6] * m0 + R[7] * m1 + R[8] * m2 + (double)cam.t[2];
            if (!(z > (double)cfg.near_plane)) continue;
            const double fx = cam.fx, fy = cam.fy;
            const double iz = 1.0 / z, iz2 = iz * iz;
            const double j00 = fx * iz, j02 = -fx * x * iz2;
            const double j11 = fy * iz, j12 = -fy * y * iz2;
            double T0[3], T1[3];
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                T0[k] = j00 * R[k] + j02 * R[6 + k];
                T1[k] = j11 * R[3 + k] + j12 * R[6 + k];
            }
            double TC0[3], TC1[3];
            TC0[0] = T0[0] * S[0] + T0[1] * S[1] + T0[2] * S[2];
            TC0[1] = T0[0] * S[1] + T0[1] * S[3] + T0[2] * S[4];
            TC0[2] = T0[0] * S[2] + T0[1] * S[4] + T0[2] * S[5];
            TC1[0] = T1[0] * S[0] + T1[1] * S[1] + T1[2] * S[2];
            TC1[1] = T1[0] * S[1] + T1[1] * S[3] + T1[2] * S[4];
            TC1[2] = T1[0] * S[2] + T1[1] * S[4] + T1[2] * S[5];
            const double lp = cfg.lowpass;
            const double a = T0[0] * TC0[0] + T0[1] * TC0[1] + T0[2] * TC0[2] + lp;
            const double b = T1[0] * TC0[0] + T1[1] * TC0[1] + T1[2] * TC0[2];
            const double c = T1[0] * TC1[0] + T1[1] * TC1[1] + T1[2] * TC1[2] + lp;
            const double idet = 1.0 / (a * c - b * b);
            const double A = c * idet, B = -b * idet, C = a * idet;
            // conic -> 2D covariance
            const double ga = -(A * A * gA + A * B * gB + B * B * gC);
            const double gc = -(B * B * gA + B * C * gB + C * C * gC);
            const double hb = -0.5 * (2.0 * A * B * gA + (A * C + B * B) * gB + 2.0 * B * C * gC);
            // dL/dcov3d += T^T Gs T
            G3[0] += ga * T0[0] * T0[0] + 2.0 * hb * T0[0] * T1[0] + gc * T1[0] * T1[0];
            G3[1] += ga * T0[0] * T0[1] + hb * (T0[0] * T1[1] + T1[0] * T0[1]) + gc * T1[0] * T1[1];
            G3[2] += ga * T0[0] * T0[2] + hb * (T0[0] * T1[2] + T1[0] * T0[2]) + gc * T1[0] * T1[2];
            G3[3] += ga * T0[1] * T0[1] + 2.0 * hb * T0[1] * T1[1] + gc * T1[1] * T1[1];
            G3[4] += ga * T0[1] * T0[2] + hb * (T0[1] * T1[2] + T1[1] * T0[2]) + gc * T1[1] * T1[2];
            G3[5] += ga * T0[2] * T0[2] + 2.0 * hb * T0[2] * T1[2] + gc * T1[2] * T1[2];
            // dL/dT = 2 Gs T Sigma -> Jacobian entries -> camera-space mean
            double dT0[3], dT1[3];
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                dT0[k] = 2.0 * (ga * TC0[k] + hb * TC1[k]);
                dT1[k] = 2.0 * (hb * TC0[k] + gc * TC1[k]);
            }
            const double gj00 = dT0[0] * R[0] + dT0[1] * R[1] + dT0[2] * R[2];
            const double gj02 = dT0[0] * R[6] + dT0[1] * R[7] + dT0[2] * R[8];
            const double gj11 = dT1[0] * R[3] + dT1[1] * R[4] + dT1[2] * R[5];
            const double gj12 = dT1[0] * R[6] + dT1[1] * R[7] + dT1[2] * R[8];
            const double gx = gmx * fx * iz - gj02 * fx * iz2;
            const double gy = gmy * fy * iz - gj12 * fy * iz2;
            const double gz = -(gmx * fx * x + gmy * fy * y + gj00 * fx + gj11 * fy) * iz2 +
                              2.0 * (gj02 * fx * x + gj12 * fy * y) * iz2 * iz;
            gm[0] += R[0] * gx + R[3] * gy + R[6] * gz;
            gm[1] += R[1] * gx + R[4] * gy + R[7] * gz;
            gm[2] += R[2] * gx + R[5] * gy + R[8] * gz;
            gop += gb4.y;
            // SH colour backward (colour = max(raw, 0)) and the view-direction term.
            const double d0 = m0 - (double)cam.cc[0], d1 = m1 - (double)cam.cc[1], d2 = m2 - (double)cam.cc[2];
            const double idn = 1.0 / sqrt(d0 * d0 + d1 * d1 + d2 * d2);
            const float dx = (float)(d0 * idn), dy = (float)(d1 * idn), dz = (float)(d2 * idn);
            float basis[16];
            sh_basis(DEG, dx, dy, dz, basis);
            const float gcol_in[3] = {gb4.z, gb4.w, gbl};
            float gcol[3];
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                float raw = 0.5f;
#pragma unroll
                for (int k = 0; k < K; ++k) raw += basis[k] * s_sh[(3 * k + ch) * kParamStride + tid];
                gcol[ch] = (raw >= 0.0f) ? gcol_in[ch] : 0.0f;
            }
            float gbk[16];
#pragma unroll
            for (int k = 0; k < K; ++k) {
                float* acc = s_gsh + 3 * k * kParamStride + tid;
                acc[0] += basis[k] * gcol[0];
                acc[kParamStride] += basis[k] * gcol[1];
                acc[2 * kParamStride] += basis[k] * gcol[2];
                const float* sk = s_sh + 3 * k * kParamStride + tid;
                gbk[k] = sk[0] * gcol[0] + sk[kParamStride] * gcol[1] + sk[2 * kParamStride] * gcol[2];
            }
            if (K > 1) {
                float gdir[3];
                sh_dir_grad(DEG, dx, dy, dz, gbk, gdir);
                const double pd = (double)dx * gdir[0] + (double)dy * gdir[1] + (double)dz * gdir[2];
                gm[0] += ((double)gdir[0] - dx * pd) * idn;
                gm[1] += ((double)gdir[1] - dy * pd) * idn;
                gm[2] += ((double)gdir[2] - dz * pd) * idn;
            }
        }
        // cov3d = M M^T: dM = 2 G3 M, M = Rq diag(s).
        const double Gf[3][3] = {{G3[0], G3[1], G3[2]}, {G3[1], G3[3], G3[4]}, {G3[2], G3[4], G3[5]}};
        double dM[9];
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j)
                dM[3 * i + j] = 2.0 * (Gf[i][0] * M[j] + Gf[i][1] * M[3 + j] + Gf[i][2] * M[6 + j]);
        double gls[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) gls[j] = (dM[j] * Rq[j] + dM[3 + j] * Rq[3 + j] + dM[6 + j] * Rq[6 + j]) * s[j];
        double gR[9];
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) gR[3 * i + j] = dM[3 * i + j] * s[j];
        const double g00 = gR[0], g01 = gR[1], g02 = gR[2], g10 = gR[3], g11 = gR[4], g12 = gR[5];
        const double g20 = gR[6], g21 = gR[7], g22 = gR[8];
        const double gqn0 = 2.0 * (-qz * g01 + qy * g02 + qz * g10 - qx * g12 - qy * g20 + qx * g21);
        const double gqn1 = 2.0 * (qy * g01 + qz * g02 + qy * g10 - 2.0 * qx * g11 - qw * g12 + qz * g20 +
                                   qw * g21 - 2.0 * qx * g22);
        const double gqn2 = 2.0 * (-2.0 * qy * g00 + qx * g01 + qw * g02 + qx * g10 + qz * g12 - qw * g20 +
                                   qz * g21 - 2.0 * qy * g22);
        const double gqn3 = 2.0 * (-2.0 * qz * g00 - qw * g01 + qx * g02 + qw * g10 - 2.0 * qz * g11 +
                                   qy * g12 + qx * g20 + qy * g21);
        const double dot = qw * gqn0 + qx * gqn1 + qy * gqn2 + qz * gqn3;
        const float op = 1.0f / (1.0f + __expf(-P.ol[g]));
        G.means[3 * g] = (float)gm[0];
        G.means[3 * g + 1] = (float)gm[1];
        G.means[3 * g + 2] = (float)gm[2];
        G.ls[3 * g] = (float)gls[0];
        G.ls[3 * g + 1] = (float)gls[1];
        G.ls[3 * g + 2] = (float)gls[2];
        reinterpret_cast<float4*>(G.q)[g] =
            make_float4((float)((gqn0 - qw * dot) * qinv), (float)((gqn1 - qx * dot) * qinv),
                        (float)((gqn2 - qy * dot) * qinv), (float)((gqn3 - qz * dot) * qinv));
        G.ol[g] = gop * op * (1.0f - op);
    }
    __syncthreads();
    for (int i = tid; i < rows * ROW; i += kParamThreads) {
        const int t = i / ROW, c = i - t * ROW;
        G.sh[g0 * ROW + i] = s_gsh[c * kParamStride + t];
    }
}

// View v's 2D gradient rows in the reference's (N, 9) layout (zero where untouched).
__global__ void k_export_grad2d(const float* __restrict__ grad2d, const uint64_t* __restrict__ touch,
                                int64_t n, int view, float* __restrict__ out) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    const bool t = (touch[g] >> view) & 1ull;
    const float* src = grad2d + ((size_t)view * n + g) * kGradStride;
#pragma unroll
    for (int k = 0; k < 9; ++k) out[9 * g + k] = t ? src[k] : 0.0f;
}

// ------------------------------------------------------------------ sparse Adam

struct AdamGroup {
    float* p;
    void* m;             // fp32 values, or bf16 values when AdamParams::bf16 is set
    void* v;
    const float* g;
    int64_t count;       // elements
    int width;           // elements per Gaussian row
    float step_size;     // lr / (1 - beta1^t)
    float step_size_rest;
    int sh_band_split;   // 1 for the SH group: element j of a row is band j / 3
};

struct AdamParams {
    AdamGroup grp[5];
    float b1, b2, isq_bc2, eps;
    int bf16;
};

__device__ __forceinline__ float bf16_round(float x) {
    uint32_t u = __float_as_uint(x);
    u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
    return __uint_as_float(u);
}

// Adam moments in memory: fp32 (4 bytes a value) or bfloat16 (2 bytes a value; the stored
// bits are the upper half of an fp32 that adam_update has already rounded to bf16, so
// storing truncates nothing and loading shifts the bits back).
template <bool BF>
struct MomentStore;

template <>
struct MomentStore<false> {
    static constexpr unsigned kAlign4 = 16;  // bytes of four values
    __device__ __forceinline__ static float4 ld4(const void* p, uint32_t i) {
        return reinterpret_cast<const float4*>(p)[i];
    }
    __device__ __forceinline__ static void st4(void* p, uint32_t i, const float4& v) {
        reinterpret_cast<float4*>(p)[i] = v;
    }
    __device__ __forceinline__ static float ld(const void* p, uint32_t e) {
        return reinterpret_cast<const float*>(p)[e];
    }
    __device__ __forceinline__ static void st(void* p, uint32_t e, float v) {
        reinterpret_cast<float*>(p)[e] = v;
    }
};

template <>
struct MomentStore<true> {
    static constexpr unsigned kAlign4 = 8;
    __device__ __forceinline__ static float lo(uint32_t w) { return __uint_as_float(w << 16); }
    __device__ __forceinline__ static float hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
    __device__ __forceinline__ static uint32_t pack(float a, float b) {
        return (__float_as_uint(a) >> 16) | (__float_as_uint(b) & 0xFFFF0000u);
    }
    __device__ __forceinline__ static float4 ld4(const void* p, uint32_t i) {
        const uint2 w = reinterpret_cast<const uint2*>(p)[i];
        return make_float4(lo(w.x), hi(w.x), lo(w.y), hi(w.y));
    }
    __device__ __forceinline__ static void st4(void* p, uint32_t i, const float4& v) {
        reinterpret_cast<uint2*>(p)[i] = make_uint2(pack(v.x, v.y), pack(v.z, v.w));
    }
    __device__ __forceinline__ static float ld(const void* p, uint32_t e) {
        return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(p)[e] << 16);
    }
    __device__ __forceinline__ static void st(void* p, uint32_t e, float v) {
        reinterpret_cast<uint16_t*>(p)[e] = (uint16_t)(__float_as_uint(v) >> 16);
    }
};

// One Adam update of element e (column col of its row) when its row is visible.
__device__ __forceinline__ void adam_update(const AdamParams& A, const AdamGroup& G, int col,
                                            float g, float& p, float& m, float& v) {
    const float m1 = A.b1 * m + (1.0f - A.b1) * g;
    const float v1 = A.b2 * v + (1.0f - A.b2) * g * g;
    const float den = sqrtf(v1) * A.isq_bc2 + A.eps;
    const float ss = (G.sh_band_split && col >= 3) ? G.step_size_rest : G.step_size;
    p = p - ss * (m1 / den);
    m = A.bf16 ? bf16_round(m1) : m1;
    v = A.bf16 ? bf16_round(v1) : v1;
}

// Rows with a visibility count > 0 (gsplat/t2_param_backward.py:195-223), W elements per row
// (a compile-time width turns the row / column split into a multiply-shift). With VEC, four
// consecutive elements per thread through 16-byte loads and stores (the group's arrays are
// 16-byte aligned); the count's remainder modulo 4 is done element by element.
template <int W, bool VEC, bool BF>
__global__ void __launch_bounds__(256)
k_sparse_adam(AdamParams A, const float* __restrict__ vis, const unsigned int* __restrict__ err,
              int group) {
    using MS = MomentStore<BF>;
    if (err != nullptr && *err != 0u) return;
    const AdamGroup& G = A.grp[group];
    const uint32_t count = (uint32_t)G.count;
    const uint32_t stride = gridDim.x * blockDim.x;
    const uint32_t t0 = blockIdx.x * blockDim.x + threadIdx.x;
    uint32_t done = 0;
    if (VEC) {
        const uint32_t n4 = count / 4u;
        for (uint32_t i = t0; i < n4; i += stride) {
            const uint32_t e = 4u * i;
            const uint32_t r0 = e / W, r3 = (e + 3u) / W;
            bool any = false;
            for (uint32_t r = r0; r <= r3; ++r) any |= vis[r] > 0.0f;
            if (!any) continue;
            const float4 g4 = reinterpret_cast<const float4*>(G.g)[i];
            float4 p4 = reinterpret_cast<const float4*>(G.p)[i];
            float4 m4 = MS::ld4(G.m, i);
            float4 v4 = MS::ld4(G.v, i);
            float* pp = &p4.x;
            float* mm = &m4.x;
            float* vv = &v4.x;
            const float* gg = &g4.x;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t ek = e + (uint32_t)k;
                const uint32_t row = ek / W;
                if (vis[row] > 0.0f) adam_update(A, G, (int)(ek - row * W), gg[k], pp[k], mm[k], vv[k]);
            }
            reinterpret_cast<float4*>(G.p)[i] = p4;
            MS::st4(G.m, i, m4);
            MS::st4(G.v, i, v4);
        }
        done = n4 * 4u;
    }
    for (uint32_t e = done + t0; e < count; e += stride) {
        const uint32_t row = e / W;
        if (!(vis[row] > 0.0f)) continue;
        float p = G.p[e], m = MS::ld(G.m, e), v = MS::ld(G.v, e);
        adam_update(A, G, (int)(e - row * W), G.g[e], p, m, v);
        G.p[e] = p;
        MS::st(G.m, e, m);
        MS::st(G.v, e, v);
    }
}

// ------------------------------------------------ owner-sharded Adam through NVSwitch multicast
//
// Multi-GPU update with the reduction and the broadcast inside the Adam kernel. Every GPU
// holds its partial gradients (its own views) in a buffer bound to an NVLink multicast
// object, and the parameters likewise. The GPU that owns a range of rows reads each
// gradient element with multimem.ld_reduce -- the switch returns the sum over all GPUs --
// updates the row with its own moments, and writes the new parameter with multimem.st,
// which lands in every GPU's copy. The gradient sums cross the links once (to the owner)
// and each updated parameter once (out of the owner); no gradient or parameter is staged.
// The caller orders the kernel between two cross-GPU synchronisation points: all partial
// gradients written before it starts, and every GPU's kernel finished before any GPU
// reads parameters or overwrites gradients again.

__device__ __forceinline__ float4 mc_ld_add_v4(const float* a) {
    float4 r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(a)
                 : "memory");
    return r;
}

__device__ __forceinline__ void mc_st_v4(float* a, const float4& v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(a),
                 "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// Stores through the multicast alias are made visible system-wide before the kernel ends.
__device__ __forceinline__ void mc_release() {
    asm volatile("fence.proxy.alias;" ::: "memory");
    __threadfence_system();
}

// counts[i] = sum over GPUs of counts_mc[i] for this GPU's rows (rows4 float4s).
__global__ void __launch_bounds__(256)
k_mc_reduce_counts(const float* __restrict__ counts_mc, float* __restrict__ counts,
                   uint32_t rows4, const unsigned int* __restrict__ skip) {
    if (*skip != 0u) return;
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < rows4; i += stride)
        reinterpret_cast<float4*>(counts)[i] = mc_ld_add_v4(counts_mc + 4ull * i);
}

// One parameter group of this GPU's rows: G.p / G.m / G.v point at the rows' local copies,
// g_mc / p_mc at the same rows through the gradient / parameter multicast mappings. The
// group's element count is a multiple of 4 and every pointer 16-byte aligned. The update
// arithmetic is adam_update's, element for element, as in k_sparse_adam. Each thread
// issues the load-reduces of kMcUnroll float4s (grid-strided slabs) before using any. The
// link, not the SMs, bounds the kernel: two 256-thread blocks per SM with four requests in
// flight per thread move the same bytes per second as sixteen blocks with one, and leave
// most of each SM to the projection backward of the next row chunk running beside it.
#ifndef GS_MC_UNROLL
#define GS_MC_UNROLL 4
#endif
#ifndef GS_MC_BLOCKS_PER_SM
#define GS_MC_BLOCKS_PER_SM 2
#endif
constexpr int kMcUnroll = GS_MC_UNROLL;
constexpr int kMcBlocksPerSm = GS_MC_BLOCKS_PER_SM;

template <int W, bool BF>
__global__ void __launch_bounds__(256)
k_sparse_adam_mc(AdamParams A, const float* __restrict__ vis, const unsigned int* __restrict__ skip,
                 int group, const float* g_mc, float* p_mc) {
    using MS = MomentStore<BF>;
    if (*skip != 0u) return;
    const AdamGroup& G = A.grp[group];
    const uint32_t n4 = (uint32_t)(G.count / 4);
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t base = blockIdx.x * blockDim.x + threadIdx.x; base < n4;
         base += stride * (uint32_t)kMcUnroll) {
        float4 g4[kMcUnroll];
        bool live[kMcUnroll];
#pragma unroll
        for (int u = 0; u < kMcUnroll; ++u) {
            const uint32_t i = base + (uint32_t)u * stride;
            live[u] = false;
            if (i < n4) {
                const uint32_t e = 4u * i;
                const uint32_t r0 = e / W, r3 = (e + 3u) / W;
                for (uint32_t r = r0; r <= r3; ++r) live[u] |= vis[r] > 0.0f;
            }
            if (live[u]) g4[u] = mc_ld_add_v4(g_mc + 4ull * i);
        }
#pragma unroll
        for (int u = 0; u < kMcUnroll; ++u) {
            if (!live[u]) continue;
            const uint32_t i = base + (uint32_t)u * stride;
            const uint32_t e = 4u * i;
            float4 p4 = reinterpret_cast<const float4*>(G.p)[i];
            float4 m4 = MS::ld4(G.m, i);
            float4 v4 = MS::ld4(G.v, i);
            float* pp = &p4.x;
            float* mm = &m4.x;
            float* vv = &v4.x;
            const float* gg = &g4[u].x;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t ek = e + (uint32_t)k;
                const uint32_t row = ek / W;
                if (vis[row] > 0.0f) adam_update(A, G, (int)(ek - row * W), gg[k], pp[k], mm[k], vv[k]);
            }
            mc_st_v4(p_mc + e, p4);
            MS::st4(G.m, i, m4);
            MS::st4(G.v, i, v4);
        }
    }
    mc_release();
}

// ------------------------------------------------------------------ workspace layout

// Per-view scratch. A step's views are spread over kLanes lanes, each with its own stream
// (the caller's stream for lane 0) and its own copy of these buffers, so one view's
// rasterisers run while the next view sorts.
#ifndef GS_TRAIN_LANES
#define GS_TRAIN_LANES 4
#endif
constexpr int kLanes = GS_TRAIN_LANES;

struct ViewLane {
    int64_t* blk2;
    uint32_t* order;   // Gaussian ids sorted by depth
    uint32_t* goff;    // first tile-sort item of each depth-ordered Gaussian (n + 1)
    ushort4* rect_d;   // tile rectangle of each depth-ordered Gaussian
    uint32_t* ccnt;    // tile-sort items of each depth-ordered Gaussian
    uint32_t* tfirst;  // per 4096-item super-tile sort tile: depth index of its first item's Gaussian
    int64_t tfirst_len;
    uint32_t* tlast;   // depth index of the last Gaussian with pairs
    int64_t* stotal;   // (Gaussian, 2x2-tile super-tile) pairs of the view
    int* tdiff;        // row-wise difference arrays of the per-tile and per-super-tile counts
    uint32_t* tdig;    // super-tile sort digit offsets, 4 passes x 256
    int2* sranges;     // per super-tile [start, end) into ssorted
    uint32_t* ssorted; // depth indices sorted by (super-tile, depth order)
    uint32_t* svals;   // Gaussian ids sorted by (tile, depth bits, id)
    float4* qc;        // per sorted pair the forward staged: P0, Lx, Ly, row mask (for the backward)
    uint32_t* qcols;   // per sorted pair the forward staged: column mask
    char* radix;
    size_t radix_bytes;
    int2* ranges;
    float* image;
    float* final_T;
    int32_t* ncon;
    float* dimg;
    float* dmu;
    float* dxx;
    float* dxy;
    float* target;     // staging copy of a view's target when the caller passes host memory
    // deterministic mode only (null otherwise): slot offset of each Gaussian (exclusive
    // prefix of the tile counts, Gaussian order) and the per-pair gradient slots, 3 float4
    int64_t* doff;
    float4* dslots;
};

struct TrainWs {
    unsigned int* err;
    uint64_t* touch;
    TCam* cams;
    float* grad2d;
    int64_t* blk;      // per-view block pair totals, view v at v * blk_stride
    int64_t blk_stride;
    int64_t* pairs;
    ProjView pv;       // every view's projected records, [view][n]
    double* loss_acc;
    int nlanes;
    ViewLane lane[kLanes];
};

template <typename WS>
static void train_layout(WS& ws, TrainWs& L, int64_t n, int n_views, int H, int W, int tile,
                         int64_t cap, bool det = false) {
    const int tiles = ((W + tile - 1) / tile) * ((H + tile - 1) / tile);
    const int tile_bits = bits_for(tiles > 1 ? tiles - 1 : 1);
    const int64_t nb = div_up(n, kProjThreads) + 1;
    const int64_t px = (int64_t)H * W;
    L.err = ws.template take<unsigned int>(1);
    L.touch = ws.template take<uint64_t>(n);
    L.cams = ws.template take<TCam>(n_views);
    L.grad2d = ws.template take<float>((size_t)n_views * n * kGradStride);
    L.blk_stride = nb;
    L.blk = ws.template take<int64_t>((size_t)n_views * nb);
    L.pairs = ws.template take<int64_t>(n_views);
    const size_t nv = (size_t)n_views * n;  // projected records of every view, [view][n]
    L.pv.p0 = ws.template take<float4>(nv);
    L.pv.p1 = ws.template take<float4>(nv);
    L.pv.p2 = ws.template take<float>(nv);
    L.pv.dkey = ws.template take<uint32_t>(nv);
    L.pv.dsort = ws.template take<uint32_t>(nv);
    L.pv.rect = ws.template take<ushort4>(nv);
    L.nlanes = std::min(kLanes, n_views);
    for (int l = 0; l < L.nlanes; ++l) {
        ViewLane& V = L.lane[l];
        V.blk2 = ws.template take<int64_t>(nb);
        V.order = ws.template take<uint32_t>(n);
        V.goff = ws.template take<uint32_t>(n + 1);
        V.rect_d = ws.template take<ushort4>(n);
        V.ccnt = ws.template take<uint32_t>(n);
        V.tfirst_len = div_up(cap, kTileItems) + 1;
        V.tfirst = ws.template take<uint32_t>(V.tfirst_len);
        V.tlast = ws.template take<uint32_t>(1);
        V.stotal = ws.template take<int64_t>(1);
        V.tdiff = ws.template take<int>(tile_diff_ints((W + tile - 1) / tile, (H + tile - 1) / tile));
        V.tdig = ws.template take<uint32_t>(4 * 256);
        V.sranges = ws.template take<int2>(((W / tile + 2) / 2) * ((H / tile + 2) / 2));
        V.ssorted = ws.template take<uint32_t>(cap);
        V.svals = ws.template take<uint32_t>(cap);
        V.qc = ws.template take<float4>(cap);
        V.qcols = ws.template take<uint32_t>(cap);
        // one scratch region serves the depth sort (N, 32 bits) and the tile sort (P, tile bits)
        V.radix_bytes = std::max(radix_workspace_bytes(n, 32, 4), radix_workspace_bytes(cap, tile_bits, 4));
        V.radix = ws.template take<char>(V.radix_bytes);
        V.ranges = ws.template take<int2>(tiles);
        V.image = ws.template take<float>(px * 3);
        V.final_T = ws.template take<float>(px);
        V.ncon = ws.template take<int32_t>(px);
        V.dimg = ws.template take<float>(px * 3);
        V.dmu = ws.template take<float>(px * 3);
        V.dxx = ws.template take<float>(px * 3);
        V.dxy = ws.template take<float>(px * 3);
        V.target = ws.template take<float>(px * 3);
    }
    L.loss_acc = ws.template take<double>(2 * (size_t)n_views);
    // The deterministic mode's slots come last, so the layout before them does not depend on
    // the mode and a deterministic workspace serves every other call unchanged.
    for (int l = 0; l < L.nlanes; ++l) {
        ViewLane& V = L.lane[l];
        V.doff = det ? ws.template take<int64_t>(n) : nullptr;
        V.dslots = det ? ws.template take<float4>(3 * (size_t)cap) : nullptr;
    }
}

struct SizerAdapter {
    WorkspaceSizer s;
    template <typename T>
    T* take(size_t c) {
        s.take<T>(c);
        return nullptr;
    }
};

// Auxiliary streams of lanes 1.. (non-blocking, created once per device) and the events
// that fork them from and join them to the caller's stream.
struct LaneStreams {
    cudaStream_t s[kLanes];
    cudaEvent_t fork;
    cudaEvent_t join[kLanes];
    // host-target staging: copies run on their own stream; per lane, `staged` marks the
    // copy done and `consumed` the loss kernels that read the lane's staging buffer
    cudaStream_t copy;
    cudaEvent_t staged[kLanes];
    cudaEvent_t consumed[kLanes];
};

static gs_status lane_streams(LaneStreams** out) {
    static std::mutex mu;
    static LaneStreams* per_dev[64] = {};
    int dev = 0;
    GS_CUDA_CHECK(cudaGetDevice(&dev));
    GS_ARG_CHECK(dev >= 0 && dev < 64, "train: device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (per_dev[dev] == nullptr) {
        LaneStreams* ls = new LaneStreams();
        ls->s[0] = nullptr;
        for (int l = 1; l < kLanes; ++l)
            GS_CUDA_CHECK(cudaStreamCreateWithFlags(&ls->s[l], cudaStreamNonBlocking));
        GS_CUDA_CHECK(cudaEventCreateWithFlags(&ls->fork, cudaEventDisableTiming));
        for (int l = 0; l < kLanes; ++l) {
            GS_CUDA_CHECK(cudaEventCreateWithFlags(&ls->join[l], cudaEventDisableTiming));
            GS_CUDA_CHECK(cudaEventCreateWithFlags(&ls->staged[l], cudaEventDisableTiming));
            GS_CUDA_CHECK(cudaEventCreateWithFlags(&ls->consumed[l], cudaEventDisableTiming));
        }
        GS_CUDA_CHECK(cudaStreamCreateWithFlags(&ls->copy, cudaStreamNonBlocking));
        per_dev[dev] = ls;
    }
    *out = per_dev[dev];
    return GS_OK;
}

static gs_status check_cfg(const gs_train_config* cfg) {
    GS_ARG_CHECK(cfg != nullptr, "train: null config");
    GS_ARG_CHECK(cfg->sh_degree >= 0 && cfg->sh_degree <= 3, "train: sh_degree must be 0..3");
    GS_ARG_CHECK(cfg->tile_size == 16 || cfg->tile_size == 32, "train: tile_size must be 16 or 32");
    GS_ARG_CHECK(cfg->deterministic == 0 || cfg->deterministic == 1,
                 "train: deterministic must be 0 or 1");
    if (cfg->deterministic && cfg->tile_size != 16) {
        // a 32x32 tile's backward block has eight warps adding into the same shared-memory
        // sums in whatever order they arrive; with 16x16 tiles two warps add onto zero, which
        // is order-independent
        set_error("train: deterministic mode needs tile_size 16");
        return GS_ERR_UNSUPPORTED;
    }
    return GS_OK;
}

// Tile rows are bounded by the tile-count kernel, tile columns by the 16-bit rectangles.
static bool image_fits(int32_t h, int32_t w, int tile) {
    return h > 0 && w > 0 && (h + tile - 1) / tile <= kMaxTileRows && (w + tile - 1) / tile <= 65535;
}

static GConst gconst(const gs_gaussians* p) {
    return GConst{p->means, p->log_scales, p->quats, p->opacity_logits, p->sh};
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_train_workspace_size(int64_t n, int32_t sh_degree, int32_t n_views,
                                          int32_t height, int32_t width, int32_t tile_size,
                                          int64_t pair_capacity) {
    (void)sh_degree;
    if (n < 1) n = 1;
    if (n_views < 1) n_views = 1;
    if (tile_size < 1) tile_size = 16;
    if (pair_capacity < 1) pair_capacity = 1;
    SizerAdapter s;
    TrainWs L;
    train_layout(s, L, n, n_views, height, width, tile_size, pair_capacity);
    return s.s.bytes();
}

extern "C" size_t gs_train_deterministic_workspace_size(int64_t n, int32_t sh_degree,
                                                        int32_t n_views, int32_t height,
                                                        int32_t width, int32_t tile_size,
                                                        int64_t pair_capacity) {
    (void)sh_degree;
    if (n < 1) n = 1;
    if (n_views < 1) n_views = 1;
    if (tile_size < 1) tile_size = 16;
    if (pair_capacity < 1) pair_capacity = 1;
    SizerAdapter s;
    TrainWs L;
    train_layout(s, L, n, n_views, height, width, tile_size, pair_capacity, true);
    return s.s.bytes();
}

// Size of the workspace a call with this config lays out.
static size_t train_ws_bytes(const gs_train_config& cfg, int64_t n, int n_views, int H, int W,
                             int64_t cap) {
    return cfg.deterministic
               ? gs_train_deterministic_workspace_size(n, cfg.sh_degree, n_views, H, W,
                                                       cfg.tile_size, cap)
               : gs_train_workspace_size(n, cfg.sh_degree, n_views, H, W, cfg.tile_size, cap);
}

// Every view's projection in one pass over the parameters (cameras already in L.cams),
// then each view's pair total in L.pairs[v].
static_assert(GS_PROJECT_ROW_ALIGN % kProjThreads == 0, "row chunks must start on a projection block");

// The projection kernel over rows [row_begin, row_end) of every view.
static gs_status project_rows(const GConst& P, int64_t n, int64_t row_begin, int64_t row_end,
                              int n_views, const TCfg& cfg, TrainWs& L, float* vis_counts,
                              bool with_grad, cudaStream_t st) {
    KernelTimer kt("train_project", st);
    ProjView pv = L.pv;
    if (with_grad) pv.dkey = nullptr;  // raw depth bits are only exported by project_view
    launch_project(P, n, row_begin, row_end, L.cams, n_views, cfg, pv, L.blk, L.blk_stride,
                   L.touch, vis_counts, with_grad ? L.grad2d : nullptr, st);
    GS_CHECK_LAUNCH();
    return GS_OK;
}

// Every view's pair total from the projection's per-block totals.
static gs_status scan_view_pairs(int64_t n, int n_views, TrainWs& L, cudaStream_t st) {
    scan_block_totals_segments<int64_t><<<n_views, 1024, 0, st>>>(L.blk, div_up(n, kProjThreads),
                                                                  L.blk_stride, L.pairs);
    GS_CHECK_LAUNCH();
    return GS_OK;
}

static gs_status project_views(const GConst& P, int64_t n, int n_views, const TCfg& cfg,
                               TrainWs& L, float* vis_counts, bool with_grad, cudaStream_t st) {
    gs_status s = project_rows(P, n, 0, n, n_views, cfg, L, vis_counts, with_grad, st);
    if (s != GS_OK) return s;
    return scan_view_pairs(n, n_views, L, st);
}

// Largest Gaussian counts (exclusive) sorted through 4x2-tile super-tiles (the packed sort
// value holds id << 8, so 2^24) and through 2x2-tile super-tiles (id << 4, 2^28); above
// them the (Gaussian, tile) pairs are sorted directly. Build options, so the 2x2 path and
// the direct tile sort can be exercised on small scenes too.
#ifndef GS_WIDE_SUPER_TILE_MAX_N
#define GS_WIDE_SUPER_TILE_MAX_N (1ll << 24)
#endif
#ifndef GS_SUPER_TILE_MAX_N
#define GS_SUPER_TILE_MAX_N (1ll << 28)
#endif

// The tile sort's cell shape for n Gaussians: log2 of the super-tile width and height in
// tiles (0, 0: the (Gaussian, tile) pairs themselves). GS_TILE_SORT_CELLS=4x2|2x2|1x1 in
// the environment selects a shape for testing, where n allows it (read on every call).
static void tile_sort_shape(int64_t n, int& sx, int& sy) {
    sx = (n < (int64_t)GS_WIDE_SUPER_TILE_MAX_N) ? 2 : (n < (int64_t)GS_SUPER_TILE_MAX_N) ? 1 : 0;
    const char* e = getenv("GS_TILE_SORT_CELLS");
    if (e != nullptr) {
        if (strcmp(e, "2x2") == 0 && n < (int64_t)GS_SUPER_TILE_MAX_N) sx = 1;
        else if (strcmp(e, "1x1") == 0) sx = 0;
    }
    sy = sx ? 1 : 0;
}

// Depth order, pair offsets, tile counts / ranges and the tile sort of one projected view.
static gs_status sort_view(int64_t n, const TCfg& cfg, int view, TrainWs& L, ViewLane& V,
                           int64_t cap, cudaStream_t st) {
    const unsigned int nb = div_up(n, kProjThreads);
    const ProjView pv = L.pv.view(view, n);
    // The tile lists come from a stable sort of the (Gaussian, super-tile) pairs and a filter
    // that hands each super-tile's depth-ordered items to its tiles. Super-tiles are 4x2
    // tiles (about 0.32 of the (Gaussian, tile) pairs at the benchmark sizes) while the
    // Gaussian ids fit the 24 bits the packed sort value leaves, else 2x2 tiles (0.43; 28
    // bits), else the (Gaussian, tile) pairs themselves are sorted (sx = sy = 0).
    int sx, sy;
    tile_sort_shape(n, sx, sy);
    const bool super = sx != 0;
    // Gaussians in (depth bits, id) order, those without pairs last.
    unsigned int* rerr = nullptr;
    gs_status s = radix_sort_pairs32(pv.dsort, nullptr, nullptr, n, 32, nullptr, V.order, V.radix,
                                     V.radix_bytes, st, &rerr, L.err);
    if (s != GS_OK) return s;
    // each one's rectangle and tile-sort item count in depth order (one gather), and the
    // per-block item totals
    launch_sorted_count(pv, V.order, n, sx, sy, V.rect_d, V.ccnt, V.blk2, st);
    GS_CHECK_LAUNCH();
    scan_block_totals<int64_t><<<1, 1024, 0, st>>>(V.blk2, nb, nullptr);
    GS_CHECK_LAUNCH();
    const int cells_x = super_cells(cfg.tiles_x, sx);
    const int cells = cells_x * super_cells(cfg.tiles_y, sy);
    const int key_bits = bits_for(cells > 1 ? cells - 1 : 1);
    const int npass = radix_num_passes(key_bits);
    {
        KernelTimer kt("pair_offsets", st);
        GS_CUDA_CHECK(cudaMemsetAsync(V.tlast, 0, sizeof(uint32_t), st));
        launch_pair_offsets(V.ccnt, n, V.blk2, cap, V.goff, V.tfirst, V.tfirst_len, V.tlast,
                            V.stotal, L.err, st);
        GS_CHECK_LAUNCH();
    }
    {
        KernelTimer kt("tile_counts", st);
        s = launch_tile_counts(pv, n, cfg.tiles_x, cfg.tiles_y, sx, sy, npass, L.pairs + view,
                               cap, V.tdiff, V.ranges, V.sranges, V.tdig, L.err, st);
        if (s != GS_OK) return s;
    }
    const RectPairArgs src{V.order, V.goff, V.tfirst, V.tlast, V.rect_d, cells_x, sx, sy};
    s = radix_sort_rect_pairs(src, V.stotal, cap, key_bits, V.tdig, super ? V.ssorted : V.svals,
                              V.radix, V.radix_bytes, st, L.err);
    if (s != GS_OK) return s;
    if (super) {
        KernelTimer kt("tile_filter", st);
        s = launch_tile_filter(V.ssorted, V.sranges, V.ranges, cfg.tiles_x, cfg.tiles_y, sx, sy,
                               L.pairs + view, cap, V.svals, st);
        if (s != GS_OK) return s;
    }
    return GS_OK;
}

// One view after the projection: sort, forward, loss, backward into the view's 2D-gradient
// rows (and the optional exports), all on stream st with lane V's scratch.
// True for host memory (pinned or pageable), which the step stages through the lane's
// device buffer; device and managed memory are read in place.
static bool is_host_pointer(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return true;
    }
    return a.type == cudaMemoryTypeHost || a.type == cudaMemoryTypeUnregistered;
}

// The loss's constants: 11-tap Gaussian (sigma 1.5) filter weights and lambda_dssim.
static LossCfg make_loss_cfg(const gs_train_config& cfg) {
    LossCfg LC;
    double taps[11], sum = 0.0;
    for (int k = 0; k < 11; ++k) {
        const double xk = k - 5;
        taps[k] = std::exp(-(xk * xk) / (2.0 * 1.5 * 1.5));
        sum += taps[k];
    }
    for (int k = 0; k < 11; ++k) LC.taps[k] = (float)(taps[k] / sum);
    // (1 - lambda) L1 [+ lambda (1 - SSIM)]; a pure L1 loss is lambda = 0 without SSIM.
    LC.lambda = cfg.lambda_dssim;
    LC.H = LC.W = 0;
    LC.inv_n = 0.0f;
    return LC;
}

static gs_status ssim_smem_attributes() {
    GS_CUDA_CHECK(cudaFuncSetAttribute(k_ssim_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sizeof(SsimFwdSmem)));
    GS_CUDA_CHECK(cudaFuncSetAttribute(k_ssim_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sizeof(SsimBwdSmem)));
    return GS_OK;
}

// Forward rasteriser of one sorted view into img (H*W*3) and the lane's final T / counts.
static gs_status launch_raster_fwd(const TCfg& c, const ViewLane& V, const ProjView& pvv, int vh,
                                   int vw, float* img, cudaStream_t st) {
    KernelTimer kt("raster_fwd", st);
    const unsigned int tiles = (unsigned int)(c.tiles_x * c.tiles_y);
    if (c.tile == 16)
        k_train_fwd<16, kFwdPPT><<<tiles, 256 / kFwdPPT, 0, st>>>(V.ranges, V.svals, pvv, c, vh, vw, img, V.final_T, V.ncon, V.qc, V.qcols);
    else
        k_train_fwd<32, kFwdPPT><<<tiles, 1024 / kFwdPPT, 0, st>>>(V.ranges, V.svals, pvv, c, vh, vw, img, V.final_T, V.ncon, V.qc, V.qcols);
    GS_CHECK_LAUNCH();
    return GS_OK;
}

// Loss of one view and its gradient dimg; the loss lands in *loss_out (device) from the
// two float64 accumulators at acc (zeroed by the caller). dmu / dxx / dxy: SSIM scratch.
static gs_status launch_loss(const float* img, const float* target, int vh, int vw, int use_ssim,
                             LossCfg LC, float* dmu, float* dxx, float* dxy, float* dimg,
                             double* acc, float* loss_out, cudaStream_t st) {
    KernelTimer kt("loss", st);
    LC.H = vh;
    LC.W = vw;
    LC.inv_n = (float)(1.0 / (3.0 * vh * vw));
    const int64_t n3 = (int64_t)vh * vw * 3;
    if (use_ssim) {
        dim3 grid(div_up(vw, kSsimT), div_up(vh, kSsimT));
        k_ssim_fwd<<<grid, 256, sizeof(SsimFwdSmem), st>>>(img, target, LC, dmu, dxx, dxy, acc);
        GS_CHECK_LAUNCH();
        k_ssim_bwd<<<grid, 256, sizeof(SsimBwdSmem), st>>>(img, target, dmu, dxx, dxy, LC, dimg);
    } else {
        k_loss_l1<<<(unsigned int)std::min<int64_t>(div_up(n3, 256), kNumSMs * 8), 256, 0, st>>>(
            img, target, n3, LC, dimg, acc);
    }
    GS_CHECK_LAUNCH();
    k_loss_finalize<<<1, 1, 0, st>>>(acc, LC, use_ssim, loss_out);
    GS_CHECK_LAUNCH();
    return GS_OK;
}

// Backward rasteriser of one view: 2D-gradient rows g2 from dimg and the lane's final T /
// counts of the same view's forward.
// With the workspace's deterministic slots (V.doff non-null: cfg.deterministic), the
// per-pair sums go through the slots instead of atomics; blk_off = the view's scanned
// projection block offsets, pairs = its pair total (device), n Gaussians, cap the capacity.
static gs_status launch_raster_bwd(const TCfg& c, const ViewLane& V, const ProjView& pvv, int vh,
                                   int vw, const float* dimg, float* g2, const int64_t* blk_off,
                                   const int64_t* pairs, int64_t n, int64_t cap, cudaStream_t st) {
    KernelTimer kt("raster_bwd", st);
    const unsigned int tiles = (unsigned int)(c.tiles_x * c.tiles_y);
    if (V.doff != nullptr) {
        if (c.tile != 16) {
            set_error("train: deterministic mode needs tile_size 16");
            return GS_ERR_UNSUPPORTED;
        }
        k_det_offsets<<<div_up(n, kProjThreads), kProjThreads, 0, st>>>(pvv.rect, n, blk_off, V.doff);
        GS_CHECK_LAUNCH();
        k_det_zero<<<kNumSMs * 4, 256, 0, st>>>(V.dslots, pairs, cap);
        GS_CHECK_LAUNCH();
        k_train_bwd<16, kBwdPPT, true><<<tiles, 256 / kBwdPPT, 0, st>>>(
            V.ranges, V.svals, pvv, c, vh, vw, dimg, V.final_T, V.ncon, V.qc, V.qcols, g2, V.doff,
            V.dslots, cap);
        GS_CHECK_LAUNCH();
        k_det_reduce<<<div_up(n, 256), 256, 0, st>>>(pvv.rect, V.doff, V.dslots, n, cap, g2);
        GS_CHECK_LAUNCH();
        return GS_OK;
    }
    if (c.tile == 16)
        k_train_bwd<16, kBwdPPT, false><<<tiles, 256 / kBwdPPT, 0, st>>>(
            V.ranges, V.svals, pvv, c, vh, vw, dimg, V.final_T, V.ncon, V.qc, V.qcols, g2, nullptr,
            nullptr, 0);
    else
        k_train_bwd<32, kBwdPPT, false><<<tiles, 1024 / kBwdPPT, 0, st>>>(
            V.ranges, V.svals, pvv, c, vh, vw, dimg, V.final_T, V.ncon, V.qc, V.qcols, g2, nullptr,
            nullptr, 0);
    GS_CHECK_LAUNCH();
    return GS_OK;
}

static gs_status run_view(int64_t n, int v, const gs_camera& cam, const gs_train_config& cfg,
                          LossCfg LC, const float* target, float* images, float* grad2d_out,
                          float* view_losses, TrainWs& L, ViewLane& V, int64_t cap,
                          cudaStream_t st, LaneStreams* LS, int lane) {
    const int vh = cam.height, vw = cam.width;
    const TCfg c = make_tcfg(cfg, vh, vw);
    // A host target is copied into the lane's staging buffer: with lanes, on the copy
    // stream while this view sorts and blends (after the loss kernels of the lane's previous
    // view have read the buffer); without, in order on st.
    const bool host_target = is_host_pointer(target);
    const size_t tbytes = (size_t)vh * vw * 3 * sizeof(float);
    if (host_target) {
        if (LS != nullptr) {
            // a lane's first view in this call reuses the buffer after the fork, which already
            // follows every earlier use (the previous call joined its lanes to st)
            if (v != lane) GS_CUDA_CHECK(cudaStreamWaitEvent(LS->copy, LS->consumed[lane], 0));
            GS_CUDA_CHECK(cudaMemcpyAsync(V.target, target, tbytes, cudaMemcpyHostToDevice, LS->copy));
            GS_CUDA_CHECK(cudaEventRecord(LS->staged[lane], LS->copy));
        } else {
            GS_CUDA_CHECK(cudaMemcpyAsync(V.target, target, tbytes, cudaMemcpyHostToDevice, st));
        }
        target = V.target;
    }
    gs_status s = sort_view(n, c, v, L, V, cap, st);
    if (s != GS_OK) return s;
    const ProjView pvv = L.pv.view(v, n);
    float* img = images ? images + (size_t)v * vh * vw * 3 : V.image;
    s = launch_raster_fwd(c, V, pvv, vh, vw, img, st);
    if (s != GS_OK) return s;
    if (host_target && LS != nullptr) GS_CUDA_CHECK(cudaStreamWaitEvent(st, LS->staged[lane], 0));
    s = launch_loss(img, target, vh, vw, cfg.use_ssim, LC, V.dmu, V.dxx, V.dxy, V.dimg,
                    L.loss_acc + 2 * v, view_losses + v, st);
    if (s != GS_OK) return s;
    if (host_target && LS != nullptr) GS_CUDA_CHECK(cudaEventRecord(LS->consumed[lane], st));
    s = launch_raster_bwd(c, V, pvv, vh, vw, V.dimg, L.grad2d + (size_t)v * n * kGradStride,
                          L.blk + (size_t)v * L.blk_stride, L.pairs + v, n, cap, st);
    if (s != GS_OK) return s;
    if (grad2d_out) {
        k_export_grad2d<<<div_up(n, 256), 256, 0, st>>>(L.grad2d, L.touch, n, v,
                                                        grad2d_out + (size_t)v * n * 9);
        GS_CHECK_LAUNCH();
    }
    return GS_OK;
}

extern "C" gs_status gs_train_count_pairs(const gs_gaussians* params, int64_t n,
                                          const gs_camera* cams, int32_t n_views,
                                          const gs_train_config* cfg, int64_t* pairs_host,
                                          void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    gs_status cs = check_cfg(cfg);
    if (cs != GS_OK) return cs;
    GS_ARG_CHECK(params && cams && pairs_host && n > 0 && n_views > 0 && n_views <= 64,
                 "gs_train_count_pairs: bad arguments");
    int H = 0, W = 0;
    for (int v = 0; v < n_views; ++v) {
        H = std::max(H, (int)cams[v].height);
        W = std::max(W, (int)cams[v].width);
    }
    Workspace ws(workspace, workspace_bytes);
    TrainWs L;
    train_layout(ws, L, n, n_views, H, W, cfg->tile_size, 1);
    GS_ARG_CHECK(ws.ok(), "gs_train_count_pairs: workspace too small");
    std::vector<TCam> hc(n_views);
    for (int v = 0; v < n_views; ++v) hc[v] = make_tcam(cams[v]);
    GS_CUDA_CHECK(cudaMemcpyAsync(L.cams, hc.data(), n_views * sizeof(TCam), cudaMemcpyHostToDevice, st));
    gs_status s = project_views(gconst(params), n, n_views, make_tcfg(*cfg, H, W), L, nullptr, false, st);
    if (s != GS_OK) return s;
    GS_CUDA_CHECK(cudaMemcpyAsync(pairs_host, L.pairs, n_views * sizeof(int64_t),
                                  cudaMemcpyDeviceToHost, st));
    GS_CUDA_CHECK(cudaStreamSynchronize(st));
    return GS_OK;
}

__global__ void k_export_projection(ProjView pv, int64_t n, float* __restrict__ means2d,
                                    float* __restrict__ conic, float* __restrict__ opacity,
                                    float* __restrict__ colors, float* __restrict__ depth,
                                    int32_t* __restrict__ rects) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    const float4 p0 = pv.p0[g], p1 = pv.p1[g];
    means2d[2 * g] = p0.x;
    means2d[2 * g + 1] = p0.y;
    conic[3 * g] = p0.z;
    conic[3 * g + 1] = p0.w;
    conic[3 * g + 2] = p1.x;
    opacity[g] = p1.y;
    colors[3 * g] = p1.z;
    colors[3 * g + 1] = p1.w;
    colors[3 * g + 2] = pv.p2[g];
    depth[g] = __uint_as_float(pv.dkey[g]);
    const ushort4 r = pv.rect[g];
    const bool any = r.y >= r.x;  // x1 < x0: no tiles
    rects[4 * g] = any ? r.x : 0;
    rects[4 * g + 1] = any ? r.y : -1;
    rects[4 * g + 2] = any ? r.z : 0;
    rects[4 * g + 3] = any ? r.w : -1;
}

extern "C" gs_status gs_train_project_view(const gs_gaussians* params, int64_t n,
                                           const gs_camera* cam, const gs_train_config* cfg,
                                           float* means2d, float* conic, float* opacity,
                                           float* colors, float* depth, int32_t* rects,
                                           float* vis_counts, uint32_t* sorted_ids,
                                           int32_t* tile_ranges, int64_t pair_capacity,
                                           int64_t* pairs_host, void* workspace,
                                           size_t workspace_bytes, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    gs_status cs = check_cfg(cfg);
    if (cs != GS_OK) return cs;
    GS_ARG_CHECK(params && cam && means2d && conic && opacity && colors && depth && rects &&
                 vis_counts && sorted_ids && tile_ranges && pairs_host && n > 0,
                 "gs_train_project_view: bad arguments");
    GS_ARG_CHECK(pair_capacity >= 1 && pair_capacity < (1ll << 30),
                 "gs_train_project_view: bad pair_capacity");
    GS_ARG_CHECK(n < (1ll << 32), "gs_train_project_view: n must be below 2^32");
    GS_ARG_CHECK(image_fits(cam->height, cam->width, cfg->tile_size),
                 "gs_train_project_view: image must be 1..%d tile rows and 1..65535 tile columns",
                 kMaxTileRows);
    Workspace ws(workspace, workspace_bytes);
    TrainWs L;
    train_layout(ws, L, n, 1, cam->height, cam->width, cfg->tile_size, pair_capacity);
    GS_ARG_CHECK(ws.ok(), "gs_train_project_view: workspace too small");
    GS_CUDA_CHECK(cudaMemsetAsync(L.err, 0, sizeof(unsigned int), st));
    GS_CUDA_CHECK(cudaMemsetAsync(L.touch, 0, n * sizeof(uint64_t), st));
    GS_CUDA_CHECK(cudaMemsetAsync(vis_counts, 0, n * sizeof(float), st));
    const TCam tc = make_tcam(*cam);
    const TCfg c = make_tcfg(*cfg, cam->height, cam->width);
    GS_CUDA_CHECK(cudaMemcpyAsync(L.cams, &tc, sizeof(TCam), cudaMemcpyHostToDevice, st));
    gs_status s = project_views(gconst(params), n, 1, c, L, vis_counts, false, st);
    if (s != GS_OK) return s;
    ViewLane& V = L.lane[0];
    s = sort_view(n, c, 0, L, V, pair_capacity, st);
    if (s != GS_OK) return s;
    k_export_projection<<<div_up(n, 256), 256, 0, st>>>(L.pv, n, means2d, conic, opacity, colors,
                                                        depth, rects);
    GS_CHECK_LAUNCH();
    const int tiles = c.tiles_x * c.tiles_y;
    GS_CUDA_CHECK(cudaMemcpyAsync(tile_ranges, V.ranges, tiles * sizeof(int2), cudaMemcpyDeviceToDevice, st));
    unsigned int herr = 0;
    GS_CUDA_CHECK(cudaMemcpyAsync(pairs_host, L.pairs, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
    GS_CUDA_CHECK(cudaMemcpyAsync(&herr, L.err, sizeof(unsigned int), cudaMemcpyDeviceToHost, st));
    GS_CUDA_CHECK(cudaStreamSynchronize(st));
    if (herr & DEV_OVERFLOW) {
        set_error("gs_train_project_view: %lld pairs exceed capacity %lld", (long long)*pairs_host,
                  (long long)pair_capacity);
        return GS_ERR_OVERFLOW;
    }
    if (herr & DEV_TIMEOUT) {
        set_error("gs_train_project_view: radix sort look-back timed out");
        return GS_ERR_TIMEOUT;
    }
    if (*pairs_host > 0)
        GS_CUDA_CHECK(cudaMemcpyAsync(sorted_ids, V.svals, *pairs_host * sizeof(uint32_t),
                                      cudaMemcpyDeviceToDevice, st));
    return GS_OK;
}

// ------------------------------------------------------------------ stage entry points
//
// One view's forward, loss and backward as separate calls, in the order of the reference's
// staged chain (forward_fast -> loss_and_grad_device -> ref_slots_fast -> t2_step). The
// forward leaves the view's projected records, sorted pairs, tile ranges, final
// transmittance and per-pixel counts in a training workspace laid out for one view; the
// backward and gs_train_param_backward read them from there.

static gs_status stage_layout(const char* who, int64_t n, const gs_camera* cam,
                              const gs_train_config* cfg, int64_t cap, void* workspace,
                              size_t workspace_bytes, TrainWs& L) {
    gs_status cs = check_cfg(cfg);
    if (cs != GS_OK) return cs;
    GS_ARG_CHECK(cam != nullptr && workspace != nullptr, "%s: null argument", who);
    GS_ARG_CHECK(n > 0 && n < (1ll << 32), "%s: n must be in [1, 2^32)", who);
    GS_ARG_CHECK(cap >= 1 && cap < (1ll << 30), "%s: pair_capacity must be in [1, 2^30)", who);
    GS_ARG_CHECK(image_fits(cam->height, cam->width, cfg->tile_size),
                 "%s: image must be 1..%d tile rows and 1..65535 tile columns", who, kMaxTileRows);
    Workspace ws(workspace, workspace_bytes);
    train_layout(ws, L, n, 1, cam->height, cam->width, cfg->tile_size, cap, cfg->deterministic != 0);
    GS_ARG_CHECK(ws.ok(), "%s: workspace too small (%zu < %zu)", who, workspace_bytes,
                 train_ws_bytes(*cfg, n, 1, cam->height, cam->width, cap));
    return GS_OK;
}

extern "C" gs_status gs_render_fwd(const gs_gaussians* params, int64_t n, const gs_camera* cam,
                                   const gs_train_config* cfg, float* image, float* final_T,
                                   int32_t* n_contrib, float* vis_counts, int64_t* pairs,
                                   int64_t pair_capacity, void* workspace,
                                   size_t workspace_bytes, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    GS_ARG_CHECK(params && image, "gs_render_fwd: null argument");
    GS_ARG_CHECK(((uintptr_t)params->quats & 15) == 0, "gs_render_fwd: quats must be 16-byte aligned");
    TrainWs L;
    gs_status s = stage_layout("gs_render_fwd", n, cam, cfg, pair_capacity, workspace,
                               workspace_bytes, L);
    if (s != GS_OK) return s;
    const int H = cam->height, W = cam->width;
    GS_CUDA_CHECK(cudaMemsetAsync(L.err, 0, sizeof(unsigned int), st));
    GS_CUDA_CHECK(cudaMemsetAsync(L.touch, 0, n * sizeof(uint64_t), st));
    if (vis_counts) GS_CUDA_CHECK(cudaMemsetAsync(vis_counts, 0, n * sizeof(float), st));
    const TCam tc = make_tcam(*cam);
    const TCfg c = make_tcfg(*cfg, H, W);
    GS_CUDA_CHECK(cudaMemcpyAsync(L.cams, &tc, sizeof(TCam), cudaMemcpyHostToDevice, st));
    // with_grad: the view's 2D-gradient rows are zeroed for the later gs_render_bwd
    s = project_views(gconst(params), n, 1, c, L, vis_counts, true, st);
    if (s != GS_OK) return s;
    ViewLane& V = L.lane[0];
    s = sort_view(n, c, 0, L, V, pair_capacity, st);
    if (s != GS_OK) return s;
    s = launch_raster_fwd(c, V, L.pv.view(0, n), H, W, image, st);
    if (s != GS_OK) return s;
    const size_t px = (size_t)H * W;
    if (final_T)
        GS_CUDA_CHECK(cudaMemcpyAsync(final_T, V.final_T, px * sizeof(float), cudaMemcpyDeviceToDevice, st));
    if (n_contrib)
        GS_CUDA_CHECK(cudaMemcpyAsync(n_contrib, V.ncon, px * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
    if (pairs)
        GS_CUDA_CHECK(cudaMemcpyAsync(pairs, L.pairs, sizeof(int64_t), cudaMemcpyDeviceToDevice, st));
    return GS_OK;
}

static void loss_layout(Workspace& ws, int32_t height, int32_t width, double** acc, float** dmu,
                        float** dxx, float** dxy) {
    const size_t px3 = (size_t)height * width * 3;
    *acc = ws.take<double>(2);
    *dmu = ws.take<float>(px3);
    *dxx = ws.take<float>(px3);
    *dxy = ws.take<float>(px3);
}

extern "C" size_t gs_loss_workspace_size(int32_t height, int32_t width) {
    if (height < 1) height = 1;
    if (width < 1) width = 1;
    WorkspaceSizer z;
    const size_t px3 = (size_t)height * width * 3;
    z.take<double>(2);
    z.take<float>(px3);
    z.take<float>(px3);
    z.take<float>(px3);
    return z.bytes();
}

extern "C" gs_status gs_loss(const float* image, const float* target, int32_t height,
                             int32_t width, const gs_train_config* cfg, float* loss,
                             float* dL_dimage, void* workspace, size_t workspace_bytes,
                             void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    gs_status cs = check_cfg(cfg);
    if (cs != GS_OK) return cs;
    GS_ARG_CHECK(image && target && loss && dL_dimage && workspace, "gs_loss: null argument");
    GS_ARG_CHECK(height > 0 && width > 0, "gs_loss: bad sizes");
    Workspace ws(workspace, workspace_bytes);
    double* acc;
    float *dmu, *dxx, *dxy;
    loss_layout(ws, height, width, &acc, &dmu, &dxx, &dxy);
    GS_ARG_CHECK(ws.ok(), "gs_loss: workspace too small (%zu < %zu)", workspace_bytes,
                 gs_loss_workspace_size(height, width));
    if (cfg->use_ssim) {
        gs_status ss = ssim_smem_attributes();
        if (ss != GS_OK) return ss;
    }
    GS_CUDA_CHECK(cudaMemsetAsync(acc, 0, 2 * sizeof(double), st));
    return launch_loss(image, target, height, width, cfg->use_ssim, make_loss_cfg(*cfg), dmu, dxx,
                       dxy, dL_dimage, acc, loss, st);
}

extern "C" gs_status gs_render_bwd(int64_t n, const gs_camera* cam, const gs_train_config* cfg,
                                   const float* dL_dimage, float* grad2d, int64_t pair_capacity,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    GS_ARG_CHECK(dL_dimage, "gs_render_bwd: null dL_dimage");
    TrainWs L;
    gs_status s = stage_layout("gs_render_bwd", n, cam, cfg, pair_capacity, workspace,
                               workspace_bytes, L);
    if (s != GS_OK) return s;
    const int H = cam->height, W = cam->width;
    const TCfg c = make_tcfg(*cfg, H, W);
    s = launch_raster_bwd(c, L.lane[0], L.pv.view(0, n), H, W, dL_dimage, L.grad2d, L.blk, L.pairs,
                          n, pair_capacity, st);
    if (s != GS_OK) return s;
    if (grad2d) {
        k_export_grad2d<<<div_up(n, 256), 256, 0, st>>>(L.grad2d, L.touch, n, 0, grad2d);
        GS_CHECK_LAUNCH();
    }
    return GS_OK;
}

static AdamParams make_adam(const gs_gaussians* p, const gs_gaussians* m, const gs_gaussians* v,
                            const gs_gaussians* g, int64_t n, int64_t step,
                            const gs_train_config* cfg) {
    AdamParams A;
    const int K = (cfg->sh_degree + 1) * (cfg->sh_degree + 1);
    const double t = (double)step + 1.0;
    const double bc1 = 1.0 - std::pow((double)cfg->beta1, t);
    const double bc2 = 1.0 - std::pow((double)cfg->beta2, t);
    A.b1 = cfg->beta1;
    A.b2 = cfg->beta2;
    A.isq_bc2 = (float)(1.0 / std::sqrt(bc2));
    A.eps = cfg->eps;
    A.bf16 = cfg->bf16_moments;
    float* P[5] = {p->means, p->log_scales, p->quats, p->opacity_logits, p->sh};
    float* Mm[5] = {m->means, m->log_scales, m->quats, m->opacity_logits, m->sh};
    float* Vv[5] = {v->means, v->log_scales, v->quats, v->opacity_logits, v->sh};
    const float* Gg[5] = {g->means, g->log_scales, g->quats, g->opacity_logits, g->sh};
    const int width[5] = {3, 3, 4, 1, 3 * K};
    const double lr[5] = {cfg->lr_means, cfg->lr_log_scales, cfg->lr_quats, cfg->lr_opacity,
                          cfg->lr_sh_dc};
    for (int i = 0; i < 5; ++i) {
        A.grp[i].p = P[i];
        A.grp[i].m = Mm[i];
        A.grp[i].v = Vv[i];
        A.grp[i].g = Gg[i];
        A.grp[i].count = n * width[i];
        A.grp[i].width = width[i];
        A.grp[i].step_size = (float)(lr[i] / bc1);
        A.grp[i].step_size_rest = (float)((double)cfg->lr_sh_rest / bc1);
        A.grp[i].sh_band_split = (i == 4) ? 1 : 0;
    }
    return A;
}

static gs_status launch_adam(const AdamParams& A, const float* vis, const unsigned int* err,
                             cudaStream_t st) {
    KernelTimer kt("sparse_adam", st);
    for (int i = 0; i < 5; ++i) {
        const AdamGroup& G = A.grp[i];
        const int64_t cnt = G.count;
        GS_ARG_CHECK(cnt < (1ll << 32), "sparse Adam: a parameter group exceeds 2^32 elements");
        const uintptr_t mom_align = A.bf16 ? 7u : 15u;  // four moments: 8 or 16 bytes
        const bool vec = (((uintptr_t)G.p | (uintptr_t)G.g) & 15u) == 0 &&
                         (((uintptr_t)G.m | (uintptr_t)G.v) & mom_align) == 0;
        const unsigned int blocks =
            (unsigned int)std::min<int64_t>(div_up(vec ? div_up(cnt, 4) : cnt, 256), kNumSMs * 16);
#define GS_ADAM(W_)                                                                             \
    (A.bf16 ? (vec ? k_sparse_adam<W_, true, true><<<blocks, 256, 0, st>>>(A, vis, err, i)      \
                   : k_sparse_adam<W_, false, true><<<blocks, 256, 0, st>>>(A, vis, err, i))    \
            : (vec ? k_sparse_adam<W_, true, false><<<blocks, 256, 0, st>>>(A, vis, err, i)     \
                   : k_sparse_adam<W_, false, false><<<blocks, 256, 0, st>>>(A, vis, err, i)))
        switch (G.width) {
            case 1: GS_ADAM(1); break;
            case 3: GS_ADAM(3); break;
            case 4: GS_ADAM(4); break;
            case 12: GS_ADAM(12); break;
            case 27: GS_ADAM(27); break;
            case 48: GS_ADAM(48); break;
            default: set_error("sparse Adam: unsupported row width %d", G.width); return GS_ERR_ARG;
        }
#undef GS_ADAM
        GS_CHECK_LAUNCH();
    }
    return GS_OK;
}

extern "C" gs_status gs_sparse_adam(const gs_gaussians* params, const gs_gaussians* exp_avg,
                                    const gs_gaussians* exp_avg_sq, const gs_gaussians* grads,
                                    const float* vis_counts, int64_t n, int64_t step,
                                    const gs_train_config* cfg, const unsigned int* error_word,
                                    void* stream) {
    clear_error();
    gs_status cs = check_cfg(cfg);
    if (cs != GS_OK) return cs;
    GS_ARG_CHECK(params && exp_avg && exp_avg_sq && grads && vis_counts && n >= 0 && step >= 0,
                 "gs_sparse_adam: bad arguments");
    if (n == 0) return GS_OK;
    const AdamParams A = make_adam(params, exp_avg, exp_avg_sq, grads, n, step, cfg);
    return launch_adam(A, vis_counts, error_word, (cudaStream_t)stream);
}

// Projection backward of rows [row_begin, row_end) from the per-view 2D gradients that
// the step's views left in the workspace.
static gs_status launch_param_bwd(const gs_gaussians* params, const gs_gaussians* grads, int64_t n,
                                  int64_t row_begin, int64_t row_end, int n_views,
                                  const gs_train_config& cfg, int H, int W, const TrainWs& L,
                                  cudaStream_t st) {
    if (row_end <= row_begin) return GS_OK;
    KernelTimer kt("param_bwd", st);
    const GConst P = gconst(params);
    const TCfg c = make_tcfg(cfg, H, W);
    GMut G{grads->means, grads->log_scales, grads->quats, grads->opacity_logits, grads->sh};
    const unsigned int nb = div_up(row_end - row_begin, kParamThreads);
    const int K = (cfg.sh_degree + 1) * (cfg.sh_degree + 1);
    const size_t smem = 2 * (size_t)3 * K * kParamStride * sizeof(float);
#define GS_PBWD(D_) k_param_bwd<D_><<<nb, kParamThreads, smem, st>>>(P, n, row_begin, row_end, L.cams, n_views, c, L.grad2d, L.touch, G)
    switch (cfg.sh_degree) {
        case 0: GS_PBWD(0); break;
        case 1: GS_PBWD(1); break;
        case 2: GS_PBWD(2); break;
        default:
            GS_CUDA_CHECK(cudaFuncSetAttribute(k_param_bwd<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            GS_PBWD(3);
            break;
    }
#undef GS_PBWD
    GS_CHECK_LAUNCH();
    return GS_OK;
}

extern "C" gs_status gs_sparse_adam_multicast(const gs_gaussians* params,
                                              const gs_gaussians* params_mc,
                                              const gs_gaussians* exp_avg,
                                              const gs_gaussians* exp_avg_sq,
                                              const gs_gaussians* grads_mc,
                                              const float* vis_counts_mc, float* vis_scratch,
                                              int64_t rows, int64_t step,
                                              const gs_train_config* cfg,
                                              const unsigned int* skip, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    gs_status cs = check_cfg(cfg);
    if (cs != GS_OK) return cs;
    GS_ARG_CHECK(params && params_mc && exp_avg && exp_avg_sq && grads_mc && vis_counts_mc &&
                 vis_scratch && skip && rows >= 0 && step >= 0,
                 "gs_sparse_adam_multicast: bad arguments");
    GS_ARG_CHECK(rows % 4 == 0 && rows < (1ll << 30),
                 "gs_sparse_adam_multicast: rows must be a multiple of 4 below 2^30");
    if (rows == 0) return GS_OK;
    const AdamParams A = make_adam(params, exp_avg, exp_avg_sq, grads_mc, rows, step, cfg);
    const float* Gm[5] = {grads_mc->means, grads_mc->log_scales, grads_mc->quats,
                          grads_mc->opacity_logits, grads_mc->sh};
    float* Pm[5] = {params_mc->means, params_mc->log_scales, params_mc->quats,
                    params_mc->opacity_logits, params_mc->sh};
    uintptr_t all = (uintptr_t)vis_counts_mc | (uintptr_t)vis_scratch, mom = 0;
    for (int i = 0; i < 5; ++i) {
        all |= (uintptr_t)A.grp[i].p | (uintptr_t)Gm[i] | (uintptr_t)Pm[i];
        mom |= (uintptr_t)A.grp[i].m | (uintptr_t)A.grp[i].v;
    }
    GS_ARG_CHECK((all & 15u) == 0 && (mom & (A.bf16 ? 7u : 15u)) == 0,
                 "gs_sparse_adam_multicast: every pointer must be 16-byte aligned (bf16 moments: 8)");
    KernelTimer kt("sparse_adam_mc", st);
    const uint32_t rows4 = (uint32_t)(rows / 4);
    k_mc_reduce_counts<<<(unsigned)std::min<int64_t>(div_up(rows4, 256), kNumSMs * 8), 256, 0, st>>>(
        vis_counts_mc, vis_scratch, rows4, skip);
    GS_CHECK_LAUNCH();
    for (int i = 0; i < 5; ++i) {
        const AdamGroup& G = A.grp[i];
        const unsigned int blocks =
            (unsigned int)std::min<int64_t>(div_up(div_up(G.count, 4), 256 * kMcUnroll),
                                            kNumSMs * kMcBlocksPerSm);
#define GS_ADAM_MC(W_)                                                                         \
    (A.bf16 ? k_sparse_adam_mc<W_, true><<<blocks, 256, 0, st>>>(A, vis_scratch, skip, i, Gm[i], Pm[i]) \
            : k_sparse_adam_mc<W_, false><<<blocks, 256, 0, st>>>(A, vis_scratch, skip, i, Gm[i], Pm[i]))
        switch (G.width) {
            case 1: GS_ADAM_MC(1); break;
            case 3: GS_ADAM_MC(3); break;
            case 4: GS_ADAM_MC(4); break;
            case 12: GS_ADAM_MC(12); break;
            case 27: GS_ADAM_MC(27); break;
            case 48: GS_ADAM_MC(48); break;
            default: set_error("sparse Adam: unsupported row width %d", G.width); return GS_ERR_ARG;
        }
#undef GS_ADAM_MC
        GS_CHECK_LAUNCH();
    }
    return GS_OK;
}

extern "C" gs_status gs_train_param_backward(const gs_gaussians* params,
                                             const gs_gaussians* grads, int64_t n,
                                             int64_t row_begin, int64_t row_end,
                                             const gs_camera* cams, int32_t n_views,
                                             const gs_train_config* cfg, int64_t pair_capacity,
                                             void* workspace, size_t workspace_bytes,
                                             void* stream) {
    clear_error();
    gs_status cs = check_cfg(cfg);
    if (cs != GS_OK) return cs;
    GS_ARG_CHECK(params && grads && cams && workspace, "gs_train_param_backward: null argument");
    GS_ARG_CHECK(n > 0 && n < (1ll << 32) && n_views >= 1 && n_views <= 64,
                 "gs_train_param_backward: bad n or n_views");
    GS_ARG_CHECK(row_begin >= 0 && row_begin <= row_end && row_end <= n,
                 "gs_train_param_backward: rows [%lld, %lld) outside [0, %lld)",
                 (long long)row_begin, (long long)row_end, (long long)n);
    GS_ARG_CHECK(pair_capacity >= 1 && pair_capacity < (1ll << 30),
                 "gs_train_param_backward: pair_capacity must be in [1, 2^30)");
    GS_ARG_CHECK(((uintptr_t)params->quats & 15) == 0 && ((uintptr_t)grads->quats & 15) == 0,
                 "gs_train_param_backward: quats must be 16-byte aligned");
    int H = 0, W = 0;
    for (int v = 0; v < n_views; ++v) {
        GS_ARG_CHECK(image_fits(cams[v].height, cams[v].width, cfg->tile_size),
                     "gs_train_param_backward: bad camera %d", v);
        H = std::max(H, (int)cams[v].height);
        W = std::max(W, (int)cams[v].width);
    }
    Workspace ws(workspace, workspace_bytes);
    TrainWs L;
    train_layout(ws, L, n, n_views, H, W, cfg->tile_size, pair_capacity);
    GS_ARG_CHECK(ws.ok(), "gs_train_param_backward: workspace too small");
    return launch_param_bwd(params, grads, n, row_begin, row_end, n_views, *cfg, H, W, L,
                            (cudaStream_t)stream);
}

// The views' cameras into the workspace. A copy from pageable memory returns once the
// source has been staged, so the host vector may go out of scope afterwards.
static gs_status upload_cams(const gs_camera* cams, int n_views, TrainWs& L, cudaStream_t st) {
    std::vector<TCam> hc(n_views);
    for (int v = 0; v < n_views; ++v) hc[v] = make_tcam(cams[v]);
    GS_CUDA_CHECK(cudaMemcpyAsync(L.cams, hc.data(), n_views * sizeof(TCam), cudaMemcpyHostToDevice, st));
    return GS_OK;
}

extern "C" gs_status gs_train_project_rows(const gs_gaussians* params, float* vis_counts,
                                           int64_t n, int64_t row_begin, int64_t row_end,
                                           const gs_camera* cams, int32_t n_views,
                                           const gs_train_config* cfg, int64_t pair_capacity,
                                           void* workspace, size_t workspace_bytes,
                                           void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    gs_status cs = check_cfg(cfg);
    if (cs != GS_OK) return cs;
    GS_ARG_CHECK(params && vis_counts && cams && workspace, "gs_train_project_rows: null argument");
    GS_ARG_CHECK(n > 0 && n < (1ll << 32) && n_views >= 1 && n_views <= 64,
                 "gs_train_project_rows: bad n or n_views");
    GS_ARG_CHECK(row_begin >= 0 && row_begin <= row_end && row_end <= n &&
                     row_begin % GS_PROJECT_ROW_ALIGN == 0 &&
                     (row_end % GS_PROJECT_ROW_ALIGN == 0 || row_end == n),
                 "gs_train_project_rows: rows [%lld, %lld) must lie in [0, %lld) on multiples "
                 "of %d", (long long)row_begin, (long long)row_end, (long long)n,
                 GS_PROJECT_ROW_ALIGN);
    GS_ARG_CHECK(pair_capacity >= 1 && pair_capacity < (1ll << 30),
                 "gs_train_project_rows: pair_capacity must be in [1, 2^30)");
    GS_ARG_CHECK(((uintptr_t)params->quats & 15) == 0,
                 "gs_train_project_rows: quats must be 16-byte aligned");
    int H = 0, W = 0;
    for (int v = 0; v < n_views; ++v) {
        GS_ARG_CHECK(image_fits(cams[v].height, cams[v].width, cfg->tile_size),
                     "gs_train_project_rows: bad camera %d", v);
        H = std::max(H, (int)cams[v].height);
        W = std::max(W, (int)cams[v].width);
    }
    Workspace ws(workspace, workspace_bytes);
    TrainWs L;
    train_layout(ws, L, n, n_views, H, W, cfg->tile_size, pair_capacity);
    GS_ARG_CHECK(ws.ok(), "gs_train_project_rows: workspace too small");
    if (row_end == row_begin) return GS_OK;
    const int64_t rows = row_end - row_begin;
    GS_CUDA_CHECK(cudaMemsetAsync(L.touch + row_begin, 0, rows * sizeof(uint64_t), st));
    GS_CUDA_CHECK(cudaMemsetAsync(vis_counts + row_begin, 0, rows * sizeof(float), st));
    gs_status s = upload_cams(cams, n_views, L, st);
    if (s != GS_OK) return s;
    return project_rows(gconst(params), n, row_begin, row_end, n_views, make_tcfg(*cfg, H, W), L,
                        vis_counts, true, st);
}

extern "C" gs_status gs_train_step(const gs_gaussians* params, const gs_gaussians* exp_avg,
                                   const gs_gaussians* exp_avg_sq, const gs_gaussians* grads,
                                   float* vis_counts, int64_t n, int64_t step,
                                   const gs_camera* cams, const float* const* targets,
                                   int32_t n_views, const gs_train_config* cfg,
                                   int32_t apply_adam, float* view_losses, float* images,
                                   float* grad2d_out, int64_t* pairs, int64_t pair_capacity,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    gs_status cs = check_cfg(cfg);
    if (cs != GS_OK) return cs;
    GS_ARG_CHECK(params && grads && vis_counts && cams && targets && view_losses,
                 "gs_train_step: null argument");
    const bool projected = (apply_adam & GS_STEP_PROJECTED) != 0;
    apply_adam &= ~GS_STEP_PROJECTED;
    GS_ARG_CHECK(apply_adam >= 0 && apply_adam <= GS_STEP_DEFER_PARAM_BWD,
                 "gs_train_step: apply_adam must be 0, 1 or GS_STEP_DEFER_PARAM_BWD, "
                 "optionally with GS_STEP_PROJECTED");
    GS_ARG_CHECK(apply_adam != 1 || (exp_avg && exp_avg_sq), "gs_train_step: Adam needs moments");
    GS_ARG_CHECK(n > 0 && n < (1ll << 32), "gs_train_step: n must be in [1, 2^32)");
    GS_ARG_CHECK(n_views >= 1 && n_views <= 64, "gs_train_step: n_views must be in [1, 64]");
    GS_ARG_CHECK(pair_capacity >= 1 && pair_capacity < (1ll << 30),
                 "gs_train_step: pair_capacity must be in [1, 2^30)");
    GS_ARG_CHECK(((uintptr_t)params->quats & 15) == 0 && ((uintptr_t)grads->quats & 15) == 0,
                 "gs_train_step: quats must be 16-byte aligned");
    int H = 0, W = 0;
    for (int v = 0; v < n_views; ++v) {
        GS_ARG_CHECK(image_fits(cams[v].height, cams[v].width, cfg->tile_size),
                     "gs_train_step: image must be 1..%d tile rows and 1..65535 tile columns",
                     kMaxTileRows);
        GS_ARG_CHECK(targets[v] != nullptr, "gs_train_step: null target");
        H = std::max(H, (int)cams[v].height);
        W = std::max(W, (int)cams[v].width);
    }
    Workspace ws(workspace, workspace_bytes);
    TrainWs L;
    train_layout(ws, L, n, n_views, H, W, cfg->tile_size, pair_capacity, cfg->deterministic != 0);
    GS_ARG_CHECK(ws.ok(), "gs_train_step: workspace too small (%zu < %zu)", workspace_bytes,
                 train_ws_bytes(*cfg, n, n_views, H, W, pair_capacity));
    const GConst P = gconst(params);
    GS_CUDA_CHECK(cudaMemsetAsync(L.err, 0, sizeof(unsigned int), st));
    GS_CUDA_CHECK(cudaMemsetAsync(L.loss_acc, 0, 2 * n_views * sizeof(double), st));
    const LossCfg LC = make_loss_cfg(*cfg);
    if (cfg->use_ssim) {
        gs_status ss = ssim_smem_attributes();
        if (ss != GS_OK) return ss;
    }
    if (projected) {
        // gs_train_project_rows has projected every row of these views into the workspace
        gs_status s = scan_view_pairs(n, n_views, L, st);
        if (s != GS_OK) return s;
    } else {
        GS_CUDA_CHECK(cudaMemsetAsync(L.touch, 0, n * sizeof(uint64_t), st));
        GS_CUDA_CHECK(cudaMemsetAsync(vis_counts, 0, n * sizeof(float), st));
        gs_status s = upload_cams(cams, n_views, L, st);
        if (s != GS_OK) return s;
        s = project_views(P, n, n_views, make_tcfg(*cfg, H, W), L, vis_counts, true, st);
        if (s != GS_OK) return s;
    }
    // Views round-robin over the lanes; lanes 1.. run on auxiliary streams forked from the
    // caller's stream after the projection and joined back before the parameter backward.
    // With the kernel timer on, every view runs on the caller's stream, so the timed
    // launches do not overlap and each event pair measures one kernel alone.
    const int nlanes = timing_enabled() ? 1 : L.nlanes;
    LaneStreams* LS = nullptr;
    cudaStream_t lst[kLanes] = {st};
    if (nlanes > 1) {
        gs_status ls = lane_streams(&LS);
        if (ls != GS_OK) return ls;
        GS_CUDA_CHECK(cudaEventRecord(LS->fork, st));
        for (int l = 1; l < nlanes; ++l) {
            lst[l] = LS->s[l];
            GS_CUDA_CHECK(cudaStreamWaitEvent(lst[l], LS->fork, 0));
        }
        GS_CUDA_CHECK(cudaStreamWaitEvent(LS->copy, LS->fork, 0));
    }
    gs_status vs = GS_OK;
    for (int v = 0; v < n_views && vs == GS_OK; ++v) {
        ViewLane& V = L.lane[v % nlanes];
        const cudaStream_t vst = lst[v % nlanes];
        vs = run_view(n, v, cams[v], *cfg, LC, targets[v], images, grad2d_out, view_losses, L, V,
                      pair_capacity, vst, nlanes > 1 ? LS : nullptr, v % nlanes);
    }
    if (nlanes > 1) {  // join every lane, also after an error, before anything else runs on st
        for (int l = 1; l < nlanes; ++l) {
            GS_CUDA_CHECK(cudaEventRecord(LS->join[l], lst[l]));
            GS_CUDA_CHECK(cudaStreamWaitEvent(st, LS->join[l], 0));
        }
    }
    if (vs != GS_OK) return vs;
    if (pairs) {
        GS_CUDA_CHECK(cudaMemcpyAsync(pairs, L.pairs, n_views * sizeof(int64_t),
                                      cudaMemcpyDeviceToDevice, st));
    }
    if (apply_adam == GS_STEP_DEFER_PARAM_BWD) return GS_OK;
    {
        gs_status ps = launch_param_bwd(params, grads, n, 0, n, n_views, *cfg, H, W, L, st);
        if (ps != GS_OK) return ps;
    }
    if (apply_adam) {
        const AdamParams A = make_adam(params, exp_avg, exp_avg_sq, grads, n, step, cfg);
        gs_status s = launch_adam(A, vis_counts, L.err, st);
        if (s != GS_OK) return s;
    }
    return GS_OK;
}
