// onesweep.cuh -- one pass of the onesweep LSD radix sort, with a pluggable item source.
//
// A pass ranks a 4096-item tile in shared memory (warp-level multisplit: one ballot per
// digit bit finds each item's peers, one shared atomic per peer group claims their slots
// in item order), publishes the tile's per-digit counts, resolves its global digit
// offsets with a decoupled look-back over earlier tiles, and writes the tile out in
// digit-sorted runs so the global stores are coalesced.
//
// The source fills a thread's kSortItems items (warp-striped: warp w owns items
// [512 w, 512 w + 512) of the tile). GlobalSource reads them from key / value arrays;
// RectPairSource (rect_pairs.cuh) generates them from per-Gaussian tile rectangles, which
// fuses pair emission into the first pass of the training tile sort.
//
// Every look-back wait is bounded; on timeout the kernel raises DEV_TIMEOUT in the error
// word and continues with the offsets it has, so the host reports GS_ERR_TIMEOUT instead
// of the GPU hanging.
#pragma once

#include "common.cuh"

namespace gs {

constexpr int kRadixBits = 8;
constexpr int kRadix = 1 << kRadixBits;
constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 16;
constexpr int kTileItems = kSortThreads * kSortItems;  // 4096 (32-bit keys)
// Items per thread and per tile by key width: 64-bit keys may take fewer per thread, which
// shrinks their shared staging so more blocks fit an SM.
#ifndef GS_SORT_ITEMS_U64
#define GS_SORT_ITEMS_U64 16
#endif
template <typename KeyT>
struct SortShape {
    static constexpr int kItems = sizeof(KeyT) == 8 ? GS_SORT_ITEMS_U64 : kSortItems;
    static constexpr int kTile = kSortThreads * kItems;
};
__host__ __device__ constexpr int sort_tile_items(int key_bytes) {
    return key_bytes == 8 ? SortShape<uint64_t>::kTile : SortShape<uint32_t>::kTile;
}
constexpr unsigned int kFlagAgg = 1u << 30;
constexpr unsigned int kFlagInc = 2u << 30;
constexpr unsigned int kValueMask = (1u << 30) - 1;
constexpr int kSpinLimit = 1 << 22;
#ifndef GS_LOOK_WINDOW
#define GS_LOOK_WINDOW 4
#endif
#ifndef GS_LOOK_SLEEP
#define GS_LOOK_SLEEP 32
#endif
constexpr int kLookWindow = GS_LOOK_WINDOW;  // predecessors read per look-back round trip
constexpr int kLookSleep = GS_LOOK_SLEEP;    // ns to back off after an unpublished predecessor

static_assert(kSortThreads == kRadix, "one thread per digit in the look-back");

template <typename KeyT>
struct SortSmem {
    KeyT keys[SortShape<KeyT>::kTile];
    uint32_t vals[SortShape<KeyT>::kTile];
    uint32_t warp_hist[kSortWarps][kRadix];
    uint32_t local_off[kRadix];
    uint32_t gbase[kRadix];  // digit's global offset minus its block-local offset
    uint32_t scan[kRadix];
    uint32_t tile;
};

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
    return *(const volatile uint32_t*)p;
}
__device__ __forceinline__ void st_volatile(uint32_t* p, uint32_t v) { *(volatile uint32_t*)p = v; }

// Items from global key / value arrays; vals == null stands for the item's index (iota).
// A source fills a thread's keys first (load) and its values only after the ranking and
// the look-back (load_vals), so the values do not hold registers across them.
template <typename KeyT>
struct GlobalSource {
    const KeyT* keys;
    const uint32_t* vals;
    static constexpr bool kValsInSmem = false;  // load_vals reads global memory only

    static constexpr int kItems = SortShape<KeyT>::kItems;

    __device__ __forceinline__ void load(SortSmem<KeyT>& S, uint32_t tile, int64_t base, int valid,
                                         int64_t n, KeyT pad, KeyT (&key)[kItems]) const {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
        for (int j = 0; j < kItems; ++j) {
            const int li = warp * (kItems * 32) + j * 32 + lane;
            // pads get the largest digit so they rank after every real item
            key[j] = (li < valid) ? keys[base + li] : pad;
        }
    }

    __device__ __forceinline__ void load_vals(const SortSmem<KeyT>& S, int64_t base, int valid,
                                              uint32_t (&val)[kItems]) const {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
        for (int j = 0; j < kItems; ++j) {
            const int li = warp * (kItems * 32) + j * 32 + lane;
            val[j] = (li < valid) ? (vals ? vals[base + li] : (uint32_t)(base + li)) : 0u;
        }
    }
};

// One pass over the digit_bits-bit digit at `shift` (key bits above it are ignored). The
// item count is n_host when n_dev is null, else *n_dev if
// it is at most n_host; a larger *n_dev (a capacity overflow, which the caller reports)
// sorts nothing, so no write can land past the caller's buffers. keys_out may be null on
// the last pass (values only).
// Resident blocks per SM the register budget is set for: 64-bit keys 3 (their shared
// staging allows no more), 32-bit keys from global arrays GS_SORT_BLOCKS_U32, 32-bit keys
// from a generating source (more shared memory) 4.
#ifndef GS_SORT_BLOCKS_U32
#define GS_SORT_BLOCKS_U32 4
#endif
#ifndef GS_SORT_BLOCKS_U64
#define GS_SORT_BLOCKS_U64 3
#endif
template <typename KeyT, typename Src>
constexpr int sort_min_blocks() {
    return sizeof(KeyT) == 8 ? GS_SORT_BLOCKS_U64 : (Src::kValsInSmem ? 4 : GS_SORT_BLOCKS_U32);
}

// The pass writes keys as KeyOutT, shifted right by out_shift: a 64-bit sort whose caller
// wants only the values narrows its keys to 32 bits once the bits below
// key_bits - 32 are sorted, so the remaining passes move 4-byte keys.
template <typename KeyT, typename Src, typename KeyOutT = KeyT>
__global__ void __launch_bounds__(kSortThreads, (sort_min_blocks<KeyT, Src>()))
k_onesweep_pass(Src src, KeyOutT* __restrict__ keys_out, uint32_t* __restrict__ vals_out,
                const int64_t* __restrict__ n_dev, int64_t n_host, int shift, int digit_bits,
                const uint32_t* __restrict__ digit_offsets, uint32_t* __restrict__ lookback,
                uint32_t* __restrict__ tile_counter, unsigned int* __restrict__ err,
                int out_shift) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SortSmem<KeyT>& S = *reinterpret_cast<SortSmem<KeyT>*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t nd = n_dev ? *n_dev : n_host;
    const int64_t n = nd <= n_host ? nd : 0;

    if (tid == 0) S.tile = atomicAdd(tile_counter, 1u);
    for (int i = tid; i < kSortWarps * kRadix; i += kSortThreads) (&S.warp_hist[0][0])[i] = 0;
    __syncthreads();
    const uint32_t tile = S.tile;
    constexpr int kItems = SortShape<KeyT>::kItems, kTile = SortShape<KeyT>::kTile;
    const int64_t base = (int64_t)tile * kTile;
    if (base >= n) return;
    const int valid = (int)min((int64_t)kTile, n - base);

    KeyT key[kItems];
    const uint32_t dmax = (1u << digit_bits) - 1u;  // pads' digit
    src.load(S, tile, base, valid, n, (KeyT)dmax << shift, key);
#define GS_DIGIT(k) ((uint32_t)((k) >> shift) & dmax)

    // Warp-level multisplit: rank of each item among the warp's items of its digit.
    // Peers are found with one ballot per digit bit (pure ALU, pipelines across items);
    // each peer group's leader claims the group's slots with one shared atomic, kept in
    // item order by __syncwarp.
    uint32_t rank[kItems];
    const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
        const uint32_t d = GS_DIGIT(key[j]);
        uint32_t peers = 0xffffffffu;
        if (digit_bits == kRadixBits) {
#pragma unroll
            for (int b = 0; b < kRadixBits; ++b) {
                const uint32_t bit = (d >> b) & 1u;
                const uint32_t m = __ballot_sync(0xffffffffu, bit);
                peers &= bit ? m : ~m;
            }
        } else {  // a narrower last digit needs fewer ballots (higher bits are 0 in every lane)
            for (int b = 0; b < digit_bits; ++b) {
                const uint32_t bit = (d >> b) & 1u;
                const uint32_t m = __ballot_sync(0xffffffffu, bit);
                peers &= bit ? m : ~m;
            }
        }
        const int leader = 31 - __clz(peers);
        uint32_t old = 0;
        if (lane == leader) old = atomicAdd(&S.warp_hist[warp][d], (uint32_t)__popc(peers));
        rank[j] = __shfl_sync(0xffffffffu, old, leader) + __popc(peers & lt_mask);
        __syncwarp();
    }
    __syncthreads();

    // Per digit (thread = digit): warp prefix, tile count, then the tile's offset.
    const int d = tid;
    uint32_t count = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
        const uint32_t c = S.warp_hist[w][d];
        S.warp_hist[w][d] = count;
        count += c;
    }
    const uint32_t pads = ((uint32_t)d == dmax) ? (uint32_t)(kTile - valid) : 0u;
    count -= pads;

    // Decoupled look-back over earlier tiles of this pass, kLookWindow predecessors per
    // round trip: their words are loaded together and consumed in order up to the first
    // inclusive prefix (done) or the first tile that has not published yet (retry there).
    uint32_t* my = lookback + (size_t)tile * kRadix + d;
    uint32_t excl = 0;
    if (tile == 0) {
        st_volatile(my, kFlagInc | count);
    } else {
        st_volatile(my, kFlagAgg | count);
        int64_t k = (int64_t)tile - 1;
        int spins = 0;
        while (true) {
            uint32_t v[kLookWindow];
#pragma unroll
            for (int q = 0; q < kLookWindow; ++q)
                v[q] = (k - q >= 0) ? ld_volatile(lookback + (size_t)(k - q) * kRadix + d) : kFlagInc;
            int q = 0;
            bool done = false;
#pragma unroll
            for (; q < kLookWindow; ++q) {
                const uint32_t flag = v[q] & ~kValueMask;
                if (flag == 0u) break;
                excl += v[q] & kValueMask;
                if (flag == kFlagInc) {
                    done = true;
                    break;
                }
            }
            if (done) break;
            k -= q;
            if (q < kLookWindow) {
                if (++spins > kSpinLimit) {
                    atomicOr(err, DEV_TIMEOUT);
                    break;
                }
                if (kLookSleep > 0) __nanosleep(kLookSleep);
            }
        }
        st_volatile(my, kFlagInc | (excl + count));
    }
    S.gbase[d] = digit_offsets[d] + excl;

    // Block-local exclusive offsets of the digits (tile-sorted order): warp scans, then
    // the eight warp totals.
    {
        const uint32_t own = count + pads;
        uint32_t x = own;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) S.scan[warp] = x;
        __syncthreads();
        uint32_t wbase = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) wbase += (w < warp) ? S.scan[w] : 0u;
        const uint32_t lo = wbase + x - own;
        S.local_off[d] = lo;
        S.gbase[d] -= lo;  // the write-out then needs one word per item
    }
    __syncthreads();

    // Scatter into shared memory in digit-sorted order: the keys, then the values, which are
    // loaded only now (each item's slot stays in rank[]).
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
        const uint32_t dj = GS_DIGIT(key[j]);
        rank[j] += S.local_off[dj] + S.warp_hist[warp][dj];
        S.keys[rank[j]] = key[j];
    }
    {
        uint32_t val[kItems];
        src.load_vals(S, base, valid, val);
        // a source that staged its values in S.vals: every thread has read its own before
        // any slot is overwritten
        if (Src::kValsInSmem) __syncthreads();
#pragma unroll
        for (int j = 0; j < kItems; ++j) S.vals[rank[j]] = val[j];
    }
    __syncthreads();

    // Coalesced write-out: consecutive threads write consecutive items of a digit run.
#pragma unroll 4
    for (int i = tid; i < valid; i += kSortThreads) {
        const KeyT k = S.keys[i];
        const uint32_t dd = GS_DIGIT(k);
        const uint32_t out = S.gbase[dd] + (uint32_t)i;
        if (keys_out) keys_out[out] = (KeyOutT)(k >> out_shift);
        vals_out[out] = S.vals[i];
    }
#undef GS_DIGIT
}

}  // namespace gs
