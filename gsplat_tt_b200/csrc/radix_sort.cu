// radix_sort.cu -- stable LSD radix sort of (key, uint32 value) pairs, 64- or 32-bit keys.
//
// One up-front kernel reads every key once and builds the digit histograms of all passes;
// each pass is then one onesweep kernel (onesweep.cuh). Only the low `key_bits` bits are
// sorted: passes above the key's bit width are skipped (45 bits for 8,160 display tiles
// -> 6 passes).
#include "common.cuh"
#include "onesweep.cuh"
#include "radix_sort.cuh"
#include "rect_pairs.cuh"

namespace gs {

// Digit histograms of every pass in one read of the keys (only the low key_bits bits).
template <typename KeyT>
__global__ void k_radix_hist(const KeyT* __restrict__ keys, const int64_t* __restrict__ n_dev,
                             int64_t n_host, int npass, int key_bits, uint32_t* __restrict__ hist) {
    __shared__ uint32_t sh[8][kRadix];
    const int64_t nd = n_dev ? *n_dev : n_host;
    const int64_t n = nd <= n_host ? nd : 0;  // over capacity: nothing (see k_onesweep_pass)
    for (int i = threadIdx.x; i < 8 * kRadix; i += blockDim.x) (&sh[0][0])[i] = 0;
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const KeyT k = keys[i];
        for (int p = 0; p < npass; ++p) {
            const uint32_t mask = (1u << min(kRadixBits, key_bits - p * kRadixBits)) - 1u;
            atomicAdd(&sh[p][(uint32_t)(k >> (p * kRadixBits)) & mask], 1u);
        }
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

size_t radix_workspace_bytes(int64_t n, int key_bits, int key_bytes) {
    const int npass = (key_bits + kRadixBits - 1) / kRadixBits;
    const int tile_items = sort_tile_items(key_bytes);
    const int64_t ntiles = (n + tile_items - 1) / tile_items + 1;
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
    constexpr int kTile = SortShape<KeyT>::kTile;
    const int64_t ntiles = (n_cap + kTile - 1) / kTile + 1;
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
        k_radix_hist<KeyT><<<hist_blocks, 512, 0, st>>>(keys, n_dev, n_cap, npass, key_bits, hist);
        GS_CHECK_LAUNCH();
        k_radix_hist_scan<<<1, kRadix, 0, st>>>(hist, npass);
        GS_CHECK_LAUNCH();
    }
    const size_t smem = sizeof(SortSmem<KeyT>);
    GS_CUDA_CHECK(cudaFuncSetAttribute(k_onesweep_pass<KeyT, GlobalSource<KeyT>>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    // all of the SM's unified memory as shared memory: the passes are occupancy-bound and
    // read their inputs once
    GS_CUDA_CHECK(cudaFuncSetAttribute(k_onesweep_pass<KeyT, GlobalSource<KeyT>>,
                                       cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    const KeyT* kin = keys;
    const uint32_t* vin = vals;
    const unsigned int grid = (unsigned int)(ntiles - 1 > 0 ? ntiles - 1 : 1);
    // Only the values wanted and more than 32 key bits: the first `wide` passes sort the
    // 64-bit keys, the last of them writes each key's bits [8 wide, 8 wide + 32) -- every
    // bit a later pass reads -- as a 32-bit key, and the remaining passes move 4-byte keys.
    // Same digits, same stable passes: the same order as sorting the 64-bit keys throughout.
    const int wide = (sizeof(KeyT) == 8 && keys_out == nullptr && key_bits > 32)
                         ? (key_bits - 32 + kRadixBits - 1) / kRadixBits : npass;
    if (wide < npass) {
        GS_CUDA_CHECK(cudaFuncSetAttribute(k_onesweep_pass<KeyT, GlobalSource<KeyT>, uint32_t>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        GS_CUDA_CHECK(cudaFuncSetAttribute(k_onesweep_pass<KeyT, GlobalSource<KeyT>, uint32_t>,
                                           cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    }
    for (int p = 0; p < wide; ++p) {
        const bool last = (p == npass - 1);
        KeyT* kout = last ? keys_out : ((p & 1) ? kb : ka);
        uint32_t* vout = last ? vals_out : ((p & 1) ? vb : va);
        KernelTimer kt(sizeof(KeyT) == 8 ? "radix_pass" : "radix_pass32", st);
        if (p == wide - 1 && wide < npass) {
            k_onesweep_pass<KeyT, GlobalSource<KeyT>, uint32_t><<<grid, kSortThreads, smem, st>>>(
                GlobalSource<KeyT>{kin, vin}, (uint32_t*)kout, vout, n_dev, n_cap, p * kRadixBits,
                kRadixBits, hist + p * kRadix, look + (size_t)p * ntiles * kRadix, counters + p,
                err, wide * kRadixBits);
        } else {
            k_onesweep_pass<KeyT><<<grid, kSortThreads, smem, st>>>(
                GlobalSource<KeyT>{kin, vin}, kout, vout, n_dev, n_cap, p * kRadixBits,
                std::min(kRadixBits, key_bits - p * kRadixBits), hist + p * kRadix,
                look + (size_t)p * ntiles * kRadix, counters + p, err, 0);
        }
        GS_CHECK_LAUNCH();
        kin = kout;
        vin = vout;
    }
    if (wide < npass) {
        const size_t smem32 = sizeof(SortSmem<uint32_t>);
        GS_CUDA_CHECK(cudaFuncSetAttribute(k_onesweep_pass<uint32_t, GlobalSource<uint32_t>>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem32));
        GS_CUDA_CHECK(cudaFuncSetAttribute(k_onesweep_pass<uint32_t, GlobalSource<uint32_t>>,
                                           cudaFuncAttributePreferredSharedMemoryCarveout, 100));
        const unsigned int grid32 = (unsigned int)std::max<int64_t>(1, div_up(n_cap, kTileItems));
        const uint32_t* kin32 = (const uint32_t*)kin;
        for (int p = wide; p < npass; ++p) {
            const bool last = (p == npass - 1);
            uint32_t* kout = last ? nullptr : (uint32_t*)((p & 1) ? kb : ka);
            uint32_t* vout = last ? vals_out : ((p & 1) ? vb : va);
            KernelTimer kt("radix_pass_n32", st);
            k_onesweep_pass<uint32_t><<<grid32, kSortThreads, smem32, st>>>(
                GlobalSource<uint32_t>{kin32, vin}, kout, vout, n_dev, n_cap,
                (p - wide) * kRadixBits, std::min(kRadixBits, key_bits - p * kRadixBits),
                hist + p * kRadix, look + (size_t)p * ntiles * kRadix, counters + p, err, 0);
            GS_CHECK_LAUNCH();
            kin32 = kout;
            vin = vout;
        }
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

// Training tile sort: the first pass draws its items from the Gaussians' tile rectangles
// (pair emission fused into the pass); later passes read the previous pass's output. The
// caller supplies every pass's exclusive digit offsets (npass x 256), derived from the
// per-tile pair counts, so no histogram pass over the pairs is needed; only values are
// written by the last pass.
// The first pass of the tile sort for one super-tile shape.
template <int SX, int SY>
static gs_status launch_rect_pass(const RectPairArgs& a, uint32_t* keys_out, uint32_t* vals_out,
                                  const int64_t* n_dev, int64_t n_cap, int digit_bits,
                                  const uint32_t* digit_offsets, uint32_t* look,
                                  uint32_t* counter, unsigned int* err, unsigned int grid,
                                  cudaStream_t st) {
    const size_t smem = sizeof(SortSmem<uint32_t>);
    GS_CUDA_CHECK(cudaFuncSetAttribute(k_onesweep_pass<uint32_t, RectPairSource<SX, SY>>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    RectPairSource<SX, SY> src;
    static_cast<RectPairArgs&>(src) = a;
    k_onesweep_pass<uint32_t, RectPairSource<SX, SY>><<<grid, kSortThreads, smem, st>>>(
        src, keys_out, vals_out, n_dev, n_cap, 0, digit_bits, digit_offsets, look, counter, err, 0);
    GS_CHECK_LAUNCH();
    return GS_OK;
}

gs_status radix_sort_rect_pairs(const RectPairArgs& src, const int64_t* n_dev, int64_t n_cap,
                                int key_bits, const uint32_t* digit_offsets, uint32_t* vals_out,
                                void* workspace, size_t workspace_bytes, cudaStream_t st,
                                unsigned int* err_ext) {
    const int npass = radix_num_passes(key_bits);
    const int64_t ntiles = (n_cap + kTileItems - 1) / kTileItems + 1;
    Workspace ws(workspace, workspace_bytes);
    unsigned int* err = ws.take<unsigned int>(1);
    ws.take<uint32_t>((size_t)npass * kRadix);
    uint32_t* look = ws.take<uint32_t>((size_t)npass * ntiles * kRadix);
    uint32_t* counters = ws.take<uint32_t>(npass);
    uint32_t* ka = (uint32_t*)ws.take<char>((size_t)n_cap * sizeof(uint32_t));
    uint32_t* va = ws.take<uint32_t>(n_cap);
    uint32_t* kb = (uint32_t*)ws.take<char>((size_t)n_cap * sizeof(uint32_t));
    uint32_t* vb = ws.take<uint32_t>(n_cap);
    if (!ws.ok()) {
        set_error("tile sort: workspace too small (%zu < %zu)", workspace_bytes,
                  radix_workspace_bytes(n_cap, key_bits, 4));
        return GS_ERR_ARG;
    }
    GS_CUDA_CHECK(cudaMemsetAsync(err, 0, (char*)(counters + npass) - (char*)err, st));
    if (err_ext) err = err_ext;
    const size_t smem = sizeof(SortSmem<uint32_t>);
    GS_CUDA_CHECK(cudaFuncSetAttribute(k_onesweep_pass<uint32_t, GlobalSource<uint32_t>>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    GS_CUDA_CHECK(cudaFuncSetAttribute(k_onesweep_pass<uint32_t, GlobalSource<uint32_t>>,
                                       cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    const unsigned int grid = (unsigned int)(ntiles - 1 > 0 ? ntiles - 1 : 1);
    {
        KernelTimer kt("tile_sort_emit", st);
        uint32_t* k1 = npass == 1 ? nullptr : ka;
        uint32_t* v1 = npass == 1 ? vals_out : va;
        const int db = std::min(kRadixBits, key_bits);
        gs_status ls;
        if (src.sx == 0 && src.sy == 0)
            ls = launch_rect_pass<0, 0>(src, k1, v1, n_dev, n_cap, db, digit_offsets, look, counters, err, grid, st);
        else if (src.sx == 1 && src.sy == 1)
            ls = launch_rect_pass<1, 1>(src, k1, v1, n_dev, n_cap, db, digit_offsets, look, counters, err, grid, st);
        else if (src.sx == 2 && src.sy == 1)
            ls = launch_rect_pass<2, 1>(src, k1, v1, n_dev, n_cap, db, digit_offsets, look, counters, err, grid, st);
        else {
            set_error("tile sort: unsupported super-tile shape %dx%d", 1 << src.sx, 1 << src.sy);
            return GS_ERR_ARG;
        }
        if (ls != GS_OK) return ls;
    }
    const uint32_t* kin = ka;
    const uint32_t* vin = va;
    for (int p = 1; p < npass; ++p) {
        const bool lastp = (p == npass - 1);
        uint32_t* kout = lastp ? nullptr : ((p & 1) ? kb : ka);
        uint32_t* vout = lastp ? vals_out : ((p & 1) ? vb : va);
        KernelTimer kt("tile_sort_pass", st);
        k_onesweep_pass<uint32_t, GlobalSource<uint32_t>><<<grid, kSortThreads, smem, st>>>(
            GlobalSource<uint32_t>{kin, vin}, kout, vout, n_dev, n_cap, p * kRadixBits,
            std::min(kRadixBits, key_bits - p * kRadixBits), digit_offsets + p * kRadix,
            look + (size_t)p * ntiles * kRadix, counters + p, err, 0);
        GS_CHECK_LAUNCH();
        kin = kout;
        vin = vout;
    }
    return GS_OK;
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
