// rect_pairs.cuh -- (Gaussian, tile) pairs generated from tile rectangles, as a onesweep
// item source: the first pass of the training tile sort emits its items itself.
//
// Pair order before the sort (the order the stable sort must preserve within a tile):
// Gaussians in depth order, each Gaussian's tiles row-major inside its rectangle. The
// rectangle is taken at a coarser grid of super-tiles 2^sx tiles wide and 2^sy high (tile
// column >> sx, row >> sy), key = cell id (cy * cells_x + cx). With sx = sy = 0 the value
// is the Gaussian id and sorting stably by cell id gives the reference's (tile, depth bits,
// Gaussian id) order (src/gsplat_cpu/sort.cpp:24-27); otherwise the value is Gaussian id
// << Q | the mask of the super-tile's Q = 2^(sx + sy) tiles the Gaussian's rectangle
// covers (bit row * 2^sx + column), from which the tile filter (train_project.cu) derives
// each tile's list.
#pragma once

#include "onesweep.cuh"

namespace gs {

// The host's description of the items; radix_sort_rect_pairs instantiates the source for
// the super-tile shape (sx, sy).
struct RectPairArgs {
    const uint32_t* order;   // Gaussian ids in depth order
    const uint32_t* goff;    // first pair of each depth-ordered Gaussian; n + 1 entries
    const uint32_t* tfirst;  // per 4096-pair tile: depth index of the Gaussian holding its first pair
    const uint32_t* last;    // [0]: depth index of the last Gaussian with pairs
    const ushort4* rect;     // per depth-ordered Gaussian: tile columns x0..x1, rows y0..y1
    int tiles_x;             // cells per row of the (coarser) grid the keys index
    int sx, sy;              // cell = (tile column >> sx, tile row >> sy)
};

template <int SX, int SY>
struct RectPairSource : RectPairArgs {

    // The tile's pairs come from depth-ordered Gaussians gf..gl (at most `valid` of them,
    // each has at least one pair), taken in chunks of kGaussPerThread per thread. A thread writes
    // the pairs of its Gaussian that fall in the tile into the tile's shared key / value
    // arrays itself, walking the rectangle row-major, when there are at most kOwnPairs of
    // them; longer runs are queued and written by whole warps (lanes striding over the
    // run), so one large Gaussian does not serialise its warp. The thread then takes its
    // warp-striped items from shared memory.
    static constexpr uint32_t kOwnPairs = 32;
#ifndef GS_EMIT_GAUSS_PER_THREAD
#define GS_EMIT_GAUSS_PER_THREAD 2
#endif
    static constexpr uint32_t kGaussPerThread = GS_EMIT_GAUSS_PER_THREAD;

    // Value of the item of (depth-ordered Gaussian with id gid and tile rectangle r0, cell
    // (cx, cy)).
    __device__ __forceinline__ uint32_t value(uint32_t gid, ushort4 r0, uint32_t cx,
                                              uint32_t cy) const {
        if constexpr (SX == 0 && SY == 0) {
            return gid;
        } else {
            constexpr uint32_t W = 1u << SX, H = 1u << SY;
            // the rectangle's columns c0..c1 and rows q0..q1 inside the cell (it meets the cell)
            const uint32_t x = cx << SX, y = cy << SY;
            const uint32_t c0 = max((uint32_t)r0.x, x) - x, c1 = min((uint32_t)r0.y - x, W - 1u);
            const uint32_t q0 = max((uint32_t)r0.z, y) - y, q1 = min((uint32_t)r0.w - y, H - 1u);
            const uint32_t cols = ((2u << c1) - 1u) & ~((1u << c0) - 1u);
            uint32_t rows = 0u;  // bit q * W for each covered row q
#pragma unroll
            for (uint32_t q = 0; q < H; ++q) rows |= (q >= q0 && q <= q1) ? 1u << (q * W) : 0u;
            return (gid << (W * H)) | (cols * rows);
        }
    }

    static constexpr bool kValsInSmem = true;  // load_vals reads the staged S.vals

    __device__ __forceinline__ void load_vals(const SortSmem<uint32_t>& S, int64_t base, int valid,
                                              uint32_t (&val)[kSortItems]) const {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
        for (int j = 0; j < kSortItems; ++j) {
            const int li = warp * (kSortItems * 32) + j * 32 + lane;
            val[j] = (li < valid) ? S.vals[li] : 0u;
        }
    }

    __device__ __forceinline__ void load(SortSmem<uint32_t>& S, uint32_t tile, int64_t base,
                                         int valid, int64_t n, uint32_t pad,
                                         uint32_t (&key)[kSortItems]) const {
        // Queue of long runs, double-buffered by chunk parity: chunk k writes buffer k & 1
        // before its first barrier, and chunk k + 2 (the next writer of that buffer) starts
        // only after every warp has passed chunk k + 1's first barrier. Each counter is
        // read by all threads between chunk k's two barriers and cleared after the second.
        // A chunk is kGaussPerThread Gaussians per thread (most have a handful of items).
        constexpr uint32_t kChunk = kSortThreads * kGaussPerThread;
        __shared__ uint32_t s_big[2][kChunk];
        __shared__ uint32_t s_nbig[2];
        const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
        const uint32_t lo_p = (uint32_t)base, hi_p = (uint32_t)(base + valid);
        const uint32_t gf = tfirst[tile];
        const uint32_t gnext = (base + kTileItems < n) ? tfirst[tile + 1] : last[0];
        const uint32_t gl = min(gnext, gf + (uint32_t)valid - 1u);
        const uint32_t tx_n = (uint32_t)tiles_x;
        if (tid < 2) s_nbig[tid] = 0u;
        __syncthreads();
        int par = 0;
        for (uint32_t c0 = gf; c0 <= gl; c0 += kChunk, par ^= 1) {
#pragma unroll
            for (uint32_t u = 0; u < kGaussPerThread; ++u) {
                const uint32_t i = c0 + u * kSortThreads + (uint32_t)tid;
                if (i > gl) continue;
                const uint32_t off = goff[i], end = goff[i + 1], gid = order[i];
                const ushort4 r0 = rect[i];
                const ushort4 r = make_ushort4(r0.x >> SX, r0.y >> SX, r0.z >> SY, r0.w >> SY);
                const uint32_t p0 = max(off, lo_p), p1 = min(end, hi_p);
                if (p1 > p0 && p1 - p0 <= kOwnPairs) {
                    const uint32_t w = (uint32_t)r.y - (uint32_t)r.x + 1u;
                    const uint32_t j0 = p0 - off;
                    uint32_t ty = r.z + j0 / w, tx = r.x + j0 % w;
                    for (uint32_t p = p0; p < p1; ++p) {
                        S.keys[p - lo_p] = ty * tx_n + tx;
                        S.vals[p - lo_p] = value(gid, r0, tx, ty);
                        if (++tx > r.y) {
                            tx = r.x;
                            ++ty;
                        }
                    }
                } else if (p1 > p0) {
                    s_big[par][atomicAdd(&s_nbig[par], 1u)] = i;
                }
            }
            __syncthreads();
            const uint32_t nbig = s_nbig[par];
            __syncthreads();
            if (tid == 0) s_nbig[par] = 0u;
            for (uint32_t q = (uint32_t)warp; q < nbig; q += kSortWarps) {
                const uint32_t bi = s_big[par][q];
                const uint32_t off = goff[bi], end = goff[bi + 1], gid = order[bi];
                const ushort4 r0 = rect[bi];
                const ushort4 r = make_ushort4(r0.x >> SX, r0.y >> SX, r0.z >> SY, r0.w >> SY);
                const uint32_t p0 = max(off, lo_p), p1 = min(end, hi_p);
                const uint32_t w = (uint32_t)r.y - (uint32_t)r.x + 1u;
                for (uint32_t p = p0 + (uint32_t)lane; p < p1; p += 32u) {
                    const uint32_t j = p - off;
                    const uint32_t cy = r.z + j / w, cx = r.x + j % w;
                    S.keys[p - lo_p] = cy * tx_n + cx;
                    S.vals[p - lo_p] = value(gid, r0, cx, cy);
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kSortItems; ++j) {
            const int li = warp * (kSortItems * 32) + j * 32 + lane;
            // pads get the largest digit so they rank after every real item; the values stay
            // in S.vals until load_vals
            key[j] = (li < valid) ? S.keys[li] : pad;
        }
    }
};

}  // namespace gs
