// radix_sort.cu -- stable LSD radix sort of (uint64 key, uint32 value) pairs.
//
// Onesweep structure: one up-front kernel reads every key once and builds the digit
// histograms of all passes; each pass is then a single kernel that ranks a 4096-item
// tile in shared memory (warp-level multisplit with __match_any_sync), publishes the
// tile's per-digit counts, resolves its global digit offsets with a decoupled
// look-back over earlier tiles, and writes the tile out in digit-sorted runs so the
// global stores are coalesced. Only the low `key_bits` bits are sorted: passes above
// the tile-id bit width are skipped (45 bits for 8,160 tiles -> 6 passes).
//
// Every look-back wait is bounded; on timeout the kernel raises DEV_TIMEOUT in the
// error word and continues with the offsets it has, so the host reports
// GS_ERR_TIMEOUT instead of the GPU hanging.
#include "common.cuh"
#include "radix_sort.cuh"

namespace gs {

constexpr int kRadixBits = 8;
constexpr int kRadix = 1 << kRadixBits;
constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 16;
constexpr int kTileItems = kSortThreads * kSortItems;  // 4096
constexpr unsigned int kFlagAgg = 1u << 30;
constexpr unsigned int kFlagInc = 2u << 30;
constexpr unsigned int kValueMask = (1u << 30) - 1;
constexpr int kSpinLimit = 1 << 22;

static_assert(kSortThreads == kRadix, "one thread per digit in the look-back");

template <typename KeyT>
struct SortSmem {
    KeyT keys[kTileItems];
    uint32_t vals[kTileItems];
    uint32_t warp_hist[kSortWarps][kRadix];
    uint32_t local_off[kRadix];
    uint32_t gbase[kRadix];
    uint32_t tile;
};

// Digit histograms of every pass in one read of the keys.
template <typename KeyT>
__global__ void k_radix_hist(const KeyT* __restrict__ keys, const int64_t* __restrict__ n_dev,
                             int64_t n_host, int npass, uint32_t* __restrict__ hist) {
    __shared__ uint32_t sh[8][kRadix];
    const int64_t n = n_dev ? min(*n_dev, n_host) : n_host;  // device count, capped
    for (int i = threadIdx.x; i < 8 * kRadix; i += blockDim.x) (&sh[0][0])[i] = 0;
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const KeyT k = keys[i];
        for (int p = 0; p < npass; ++p) atomicAdd(&sh[p][(uint32_t)(k >> (p * kRadixBits)) & (kRadix - 1)], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < npass * kRadix; i += blockDim.x) {
        const uint32_t c = (&sh[0][0])[i];
        if (c) atomicAdd(&hist[i], c);
    }
}

// Exclusive scan of each pass's 256-bin histogram (one block of 256 threads).
__global__ void k_radix_hist_scan(uint32_t* __restrict__ hist, int npass) {
    __shared__ uint32_t s[kRadix];
    for (int p = 0; p < npass; ++p) {
        const uint32_t v = hist[p * kRadix + threadIdx.x];
        s[threadIdx.x] = v;
        __syncthreads();
        for (int o = 1; o < kRadix; o <<= 1) {
            const uint32_t t = (threadIdx.x >= o) ? s[threadIdx.x - o] : 0u;
            __syncthreads();
            s[threadIdx.x] += t;
            __syncthreads();
        }
        hist[p * kRadix + threadIdx.x] = s[threadIdx.x] - v;
        __syncthreads();
    }
}

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
    return *(const volatile uint32_t*)p;
}
__device__ __forceinline__ void st_volatile(uint32_t* p, uint32_t v) { *(volatile uint32_t*)p = v; }

// One onesweep pass over digit `shift`.
template <typename KeyT>
__global__ void __launch_bounds__(kSortThreads, 3)
k_radix_pass(const KeyT* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
             KeyT* __restrict__ keys_out, uint32_t* __restrict__ vals_out,
             const int64_t* __restrict__ n_dev, int64_t n_host, int shift,
             const uint32_t* __restrict__ digit_offsets, uint32_t* __restrict__ lookback,
             uint32_t* __restrict__ tile_counter, unsigned int* __restrict__ err) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SortSmem<KeyT>& S = *reinterpret_cast<SortSmem<KeyT>*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t n = n_dev ? min(*n_dev, n_host) : n_host;  // device count, capped

    if (tid == 0) S.tile = atomicAdd(tile_counter, 1u);
    for (int i = tid; i < kSortWarps * kRadix; i += kSortThreads) (&S.warp_hist[0][0])[i] = 0;
    __syncthreads();
    const uint32_t tile = S.tile;
    const int64_t base = (int64_t)tile * kTileItems;
    if (base >= n) return;
    const int valid = (int)min((int64_t)kTileItems, n - base);

    // Load (warp-striped: warp w owns items [512 w, 512 w + 512) of the tile). Pads
    // past the end get an all-ones digit so they rank after every real item.
    KeyT key[kSortItems];
    uint32_t val[kSortItems];
#pragma unroll
    for (int j = 0; j < kSortItems; ++j) {
        const int li = warp * (kSortItems * 32) + j * 32 + lane;
        if (li < valid) {
            key[j] = keys_in[base + li];
            val[j] = vals_in ? vals_in[base + li] : (uint32_t)(base + li);  // null: iota
        } else {
            key[j] = (KeyT)(kRadix - 1) << shift;
            val[j] = 0;
        }
    }
#define GS_DIGIT(k) ((uint32_t)((k) >> shift) & (uint32_t)(kRadix - 1))

    // Warp-level multisplit: rank of each item among the warp's items of its digit.
    // Peers are found with one ballot per digit bit (pure ALU, pipelines across items);
    // each peer group's leader claims the group's slots with one shared atomic, kept in
    // item order by __syncwarp.
    uint32_t rank[kSortItems];
    const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int j = 0; j < kSortItems; ++j) {
        const uint32_t d = GS_DIGIT(key[j]);
        uint32_t peers = 0xffffffffu;
#pragma unroll
        for (int b = 0; b < kRadixBits; ++b) {
            const uint32_t bit = (d >> b) & 1u;
            const uint32_t m = __ballot_sync(0xffffffffu, bit);
            peers &= bit ? m : ~m;
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
    if (d == kRadix - 1) count -= (uint32_t)(kTileItems - valid);

    // Decoupled look-back over earlier tiles of this pass.
    uint32_t* my = lookback + (size_t)tile * kRadix + d;
    uint32_t excl = 0;
    if (tile == 0) {
        st_volatile(my, kFlagInc | count);
    } else {
        st_volatile(my, kFlagAgg | count);
        int64_t k = (int64_t)tile - 1;
        int spins = 0;
        while (k >= 0) {
            const uint32_t v = ld_volatile(lookback + (size_t)k * kRadix + d);
            const uint32_t flag = v & ~kValueMask;
            if (flag == 0u) {
                if (++spins > kSpinLimit) {
                    atomicOr(err, DEV_TIMEOUT);
                    break;
                }
                __nanosleep(32);
                continue;
            }
            excl += v & kValueMask;
            if (flag == kFlagInc) break;
            --k;
        }
        st_volatile(my, kFlagInc | (excl + count));
    }
    S.gbase[d] = digit_offsets[d] + excl;

    // Block-local exclusive offsets of the digits (tile-sorted order).
    {
        __shared__ uint32_t scan_s[kRadix];
        scan_s[d] = count + (d == kRadix - 1 ? (uint32_t)(kTileItems - valid) : 0u);
        __syncthreads();
        for (int o = 1; o < kRadix; o <<= 1) {
            const uint32_t t = (d >= o) ? scan_s[d - o] : 0u;
            __syncthreads();
            scan_s[d] += t;
            __syncthreads();
        }
        const uint32_t tot = count + (d == kRadix - 1 ? (uint32_t)(kTileItems - valid) : 0u);
        S.local_off[d] = scan_s[d] - tot;
    }
    __syncthreads();

    // Scatter into shared memory in digit-sorted order.
#pragma unroll
    for (int j = 0; j < kSortItems; ++j) {
        const uint32_t d = GS_DIGIT(key[j]);
        const uint32_t pos = S.local_off[d] + S.warp_hist[warp][d] + rank[j];
        S.keys[pos] = key[j];
        S.vals[pos] = val[j];
    }
    __syncthreads();

    // Coalesced write-out: consecutive threads write consecutive items of a digit run.
#pragma unroll 4
    for (int i = tid; i < valid; i += kSortThreads) {
        const KeyT k = S.keys[i];
        const uint32_t dd = GS_DIGIT(k);
        const uint32_t out = S.gbase[dd] + ((uint32_t)i - S.local_off[dd]);
        if (keys_out) keys_out[out] = k;
        vals_out[out] = S.vals[i];
    }
#undef GS_DIGIT
}

size_t radix_workspace_bytes(int64_t n, int key_bits, int key_bytes) {
    const int npass = (key_bits + kRadixBits - 1) / kRadixBits;
    const int64_t ntiles = (n + kTileItems - 1) / kTileItems + 1;
    WorkspaceSizer s;
    s.take<unsigned int>(1);                            // error word (first: see gs_workspace_error)
    s.take<uint32_t>((size_t)npass * kRadix);          // histograms / offsets
    s.take<uint32_t>((size_t)npass * ntiles * kRadix);  // look-back words
    s.take<uint32_t>(npass);                            // tile counters
    s.take<char>((size_t)n * key_bytes); s.take<uint32_t>(n);  // ping
    s.take<char>((size_t)n * key_bytes); s.take<uint32_t>(n);  // pong
    return s.bytes();
}

int radix_num_passes(int key_bits) { return (key_bits + kRadixBits - 1) / kRadixBits; }

template <typename KeyT>
gs_status radix_sort_pairs_t(const KeyT* keys, const uint32_t* vals, const int64_t* n_dev,
                             int64_t n_cap, int key_bits, KeyT* keys_out, uint32_t* vals_out,
                             void* workspace, size_t workspace_bytes, cudaStream_t st,
                             unsigned int** err_out, unsigned int* err_ext) {
    const int npass = radix_num_passes(key_bits);
    const int64_t ntiles = (n_cap + kTileItems - 1) / kTileItems + 1;
    Workspace ws(workspace, workspace_bytes);
    unsigned int* err = ws.take<unsigned int>(1);
    uint32_t* hist = ws.take<uint32_t>((size_t)npass * kRadix);
    uint32_t* look = ws.take<uint32_t>((size_t)npass * ntiles * kRadix);
    uint32_t* counters = ws.take<uint32_t>(npass);
    KeyT* ka = (KeyT*)ws.take<char>((size_t)n_cap * sizeof(KeyT));
    uint32_t* va = ws.take<uint32_t>(n_cap);
    KeyT* kb = (KeyT*)ws.take<char>((size_t)n_cap * sizeof(KeyT));
    uint32_t* vb = ws.take<uint32_t>(n_cap);
    if (!ws.ok()) {
        set_error("radix sort: workspace too small (%zu < %zu)", workspace_bytes,
                  radix_workspace_bytes(n_cap, key_bits, (int)sizeof(KeyT)));
        return GS_ERR_ARG;
    }
    // err .. counters are contiguous: one memset clears all of them. A caller-owned
    // error word (err_ext) is OR-ed into, never cleared here.
    GS_CUDA_CHECK(cudaMemsetAsync(err, 0, (char*)(counters + npass) - (char*)err, st));
    if (err_ext) err = err_ext;
    if (err_out) *err_out = err;
    const int hist_blocks = (int)std::min<int64_t>(kNumSMs * 4, std::max<int64_t>(1, (n_cap + 4095) / 4096));
    {
        KernelTimer kt("radix_hist", st);
        k_radix_hist<KeyT><<<hist_blocks, 512, 0, st>>>(keys, n_dev, n_cap, npass, hist);
        GS_CHECK_LAUNCH();
        k_radix_hist_scan<<<1, kRadix, 0, st>>>(hist, npass);
        GS_CHECK_LAUNCH();
    }
    const size_t smem = sizeof(SortSmem<KeyT>);
    GS_CUDA_CHECK(cudaFuncSetAttribute(k_radix_pass<KeyT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const KeyT* kin = keys;
    const uint32_t* vin = vals;
    for (int p = 0; p < npass; ++p) {
        const bool last = (p == npass - 1);
        KeyT* kout = last ? keys_out : ((p & 1) ? kb : ka);
        uint32_t* vout = last ? vals_out : ((p & 1) ? vb : va);
        KernelTimer kt(sizeof(KeyT) == 8 ? "radix_pass" : "radix_pass32", st);
        k_radix_pass<KeyT><<<(unsigned int)(ntiles - 1 > 0 ? ntiles - 1 : 1), kSortThreads, smem, st>>>(
            kin, vin, kout, vout, n_dev, n_cap, p * kRadixBits, hist + p * kRadix,
            look + (size_t)p * ntiles * kRadix, counters + p, err);
        GS_CHECK_LAUNCH();
        kin = kout;
        vin = vout;
    }
    return GS_OK;
}

gs_status radix_sort_pairs(const uint64_t* keys, const uint32_t* vals, const int64_t* n_dev,
                           int64_t n_cap, int key_bits, uint64_t* keys_out, uint32_t* vals_out,
                           void* workspace, size_t workspace_bytes, cudaStream_t st,
                           unsigned int** err_out, unsigned int* err_ext) {
    return radix_sort_pairs_t<uint64_t>(keys, vals, n_dev, n_cap, key_bits, keys_out, vals_out,
                                        workspace, workspace_bytes, st, err_out, err_ext);
}

gs_status radix_sort_pairs32(const uint32_t* keys, const uint32_t* vals, const int64_t* n_dev,
                             int64_t n_cap, int key_bits, uint32_t* keys_out, uint32_t* vals_out,
                             void* workspace, size_t workspace_bytes, cudaStream_t st,
                             unsigned int** err_out, unsigned int* err_ext) {
    return radix_sort_pairs_t<uint32_t>(keys, vals, n_dev, n_cap, key_bits, keys_out, vals_out,
                                        workspace, workspace_bytes, st, err_out, err_ext);
}

// ------------------------------------------------------------------ sort_and_bin

__global__ void k_make_keys(const int64_t* __restrict__ gids, const int64_t* __restrict__ tids,
                            const float* __restrict__ depths, int64_t p, uint64_t* __restrict__ keys,
                            uint32_t* __restrict__ vals) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= p) return;
    const int64_t g = gids[i];
    keys[i] = ((uint64_t)tids[i] << 32) | (uint64_t)__float_as_uint(depths[g]);
    vals[i] = (uint32_t)g;
}

__global__ void k_widen(const uint32_t* __restrict__ v, int64_t p, int64_t* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < p) out[i] = (int64_t)v[i];
}

// sort.cpp:146-165 tile ranges: [lower_bound(t), lower_bound(t+1)) of the sorted keys,
// (0, 0) for an empty tile.
__global__ void k_tile_ranges(const uint64_t* __restrict__ sorted_keys, int64_t p, int64_t ntiles,
                              int64_t* __restrict__ ranges) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= ntiles) return;
    auto lower = [&](uint64_t target) {
        int64_t lo = 0, hi = p;
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (sorted_keys[mid] < target) lo = mid + 1; else hi = mid;
        }
        return lo;
    };
    const int64_t s = lower((uint64_t)t << 32), e = lower((uint64_t)(t + 1) << 32);
    ranges[2 * t] = (e > s) ? s : 0;
    ranges[2 * t + 1] = (e > s) ? e : 0;
}

int bits_for(int64_t v) {
    int b = 0;
    while (b < 63 && (v >> b) > 0) ++b;
    return b;
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_sort_pairs_workspace_size(int64_t n, int32_t key_bits) {
    if (n < 1) n = 1;
    if (key_bits < 1) key_bits = 1;
    return radix_workspace_bytes(n, key_bits, 8);
}

extern "C" gs_status gs_sort_pairs(const uint64_t* keys, const uint32_t* values, int64_t n,
                                   int32_t key_bits, uint64_t* keys_out, uint32_t* values_out,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    GS_ARG_CHECK(n >= 0 && n <= (int64_t)kValueMask, "gs_sort_pairs: n must be in [0, 2^30)");
    GS_ARG_CHECK(key_bits >= 1 && key_bits <= 64, "gs_sort_pairs: key_bits must be in [1, 64]");
    if (n == 0) return GS_OK;
    GS_ARG_CHECK(keys && values && values_out, "gs_sort_pairs: null pointer");
    unsigned int* err = nullptr;
    gs_status s = radix_sort_pairs(keys, values, nullptr, n, key_bits, keys_out, values_out,
                                   workspace, workspace_bytes, st, &err);
    return s;
}

extern "C" size_t gs_sort_and_bin_workspace_size(int64_t p, int32_t tiles_x, int32_t tiles_y) {
    if (p < 1) p = 1;
    const int kb = 32 + bits_for((int64_t)tiles_x * tiles_y - 1);
    WorkspaceSizer s;
    s.take<char>(radix_workspace_bytes(p, kb, 8));  // first, so its error word leads
    s.take<uint64_t>(p);  // keys
    s.take<uint32_t>(p);  // values
    s.take<uint64_t>(p);  // sorted keys
    s.take<uint32_t>(p);  // sorted values
    return s.bytes();
}

extern "C" gs_status gs_sort_and_bin(const int64_t* gaussian_ids, const int64_t* tile_ids,
                                     const float* depths, int64_t p, int32_t tiles_x,
                                     int32_t tiles_y, int64_t* sorted_gaussian_ids,
                                     int64_t* tile_ranges, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    clear_error();
    cudaStream_t st = (cudaStream_t)stream;
    GS_ARG_CHECK(p >= 0 && p <= (int64_t)kValueMask, "gs_sort_and_bin: P must be in [0, 2^30)");
    GS_ARG_CHECK(tiles_x > 0 && tiles_y > 0 && (int64_t)tiles_x * tiles_y < (1ll << 31),
                 "gs_sort_and_bin: bad tile grid");
    GS_ARG_CHECK(tile_ranges, "gs_sort_and_bin: null tile_ranges");
    const int64_t ntiles = (int64_t)tiles_x * tiles_y;
    if (p == 0) {
        GS_CUDA_CHECK(cudaMemsetAsync(tile_ranges, 0, ntiles * 2 * sizeof(int64_t), st));
        return GS_OK;
    }
    GS_ARG_CHECK(gaussian_ids && tile_ids && depths && sorted_gaussian_ids,
                 "gs_sort_and_bin: null pointer");
    const int kb = 32 + bits_for(ntiles - 1);
    Workspace ws(workspace, workspace_bytes);
    const size_t rbytes = radix_workspace_bytes(p, kb, 8);
    char* rws = ws.take<char>(rbytes);
    uint64_t* keys = ws.take<uint64_t>(p);
    uint32_t* vals = ws.take<uint32_t>(p);
    uint64_t* skeys = ws.take<uint64_t>(p);
    uint32_t* svals = ws.take<uint32_t>(p);
    GS_ARG_CHECK(ws.ok(), "gs_sort_and_bin: workspace too small (%zu < %zu)", workspace_bytes,
                 gs_sort_and_bin_workspace_size(p, tiles_x, tiles_y));
    k_make_keys<<<div_up(p, 256), 256, 0, st>>>(gaussian_ids, tile_ids, depths, p, keys, vals);
    GS_CHECK_LAUNCH();
    unsigned int* err = nullptr;
    gs_status s = radix_sort_pairs(keys, vals, nullptr, p, kb, skeys, svals, rws, rbytes, st, &err);
    if (s != GS_OK) return s;
    k_widen<<<div_up(p, 256), 256, 0, st>>>(svals, p, sorted_gaussian_ids);
    GS_CHECK_LAUNCH();
    k_tile_ranges<<<div_up(ntiles, 256), 256, 0, st>>>(skeys, p, ntiles, tile_ranges);
    GS_CHECK_LAUNCH();
    return GS_OK;
}
