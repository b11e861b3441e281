// scan.cuh -- block-level and device-wide (reduce-then-scan) prefix sums.
//
// Device-wide scans here never spin on another block: each producing kernel writes
// one total per block, scan_block_totals turns those into exclusive block offsets
// in a single block, and the consuming kernel adds its block's offset to an
// in-block scan. Deterministic and free of inter-block waits.
#pragma once

#include <stdint.h>

namespace gs {

// Exclusive scan of one value per thread across the block; returns the thread's
// exclusive prefix and writes the block total to *total (all threads see it).
// Requires blockDim.x a multiple of 32 and <= 1024; `smem` holds 33 T.
template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* smem, T* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    T x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) smem[warp] = x;
    __syncthreads();
    if (warp == 0) {
        T w = (lane < nwarps) ? smem[lane] : T(0);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            T y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < nwarps) smem[lane] = w;  // inclusive warp totals
        if (lane == nwarps - 1) smem[32] = w;
    }
    __syncthreads();
    T base = (warp > 0) ? smem[warp - 1] : T(0);
    T res = base + x - v;
    *total = smem[32];
    __syncthreads();
    return res;
}

// In-place exclusive scan of totals[0..n) by one block of 1024 threads; the grand
// total goes to *grand (may be null). Used on per-block counts (n up to ~1e6).
template <typename T>
__global__ void scan_block_totals(T* totals, int64_t n, T* grand) {
    __shared__ T smem[33];
    T carry = 0;
    for (int64_t base = 0; base < n; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        T v = (i < n) ? totals[i] : T(0);
        T tot;
        T ex = block_exclusive_scan<T>(v, smem, &tot);
        if (i < n) totals[i] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0 && grand != nullptr) *grand = carry;
}

// scan_block_totals over gridDim.x independent segments, one block each: segment s is
// totals[s * stride, s * stride + n), its grand total goes to grand[s].
template <typename T>
__global__ void scan_block_totals_segments(T* totals, int64_t n, int64_t stride, T* grand) {
    __shared__ T smem[33];
    T* seg = totals + (int64_t)blockIdx.x * stride;
    T carry = 0;
    for (int64_t base = 0; base < n; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        T v = (i < n) ? seg[i] : T(0);
        T tot;
        T ex = block_exclusive_scan<T>(v, smem, &tot);
        if (i < n) seg[i] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) grand[blockIdx.x] = carry;
}

}  // namespace gs
