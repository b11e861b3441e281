// radix_sort.cuh -- internal interface of the onesweep LSD radix sort.
#pragma once

#include "common.cuh"

namespace gs {

// Bytes of scratch for sorting up to n pairs on the low key_bits bits. The first
// word of the scratch is the sort's device error word.
size_t radix_workspace_bytes(int64_t n, int key_bits, int key_bytes);
int radix_num_passes(int key_bits);
int bits_for(int64_t v);

// Enqueue a stable sort of (keys, vals); vals == null sorts (key, index) pairs. The element
// count is *n_dev when n_dev is non-null (device-resident; above n_cap nothing is sorted),
// else n_cap. keys_out may be null
// (values only). *err_out receives the device error word (DEV_TIMEOUT on a
// look-back timeout).
gs_status radix_sort_pairs(const uint64_t* keys, const uint32_t* vals, const int64_t* n_dev,
                           int64_t n_cap, int key_bits, uint64_t* keys_out, uint32_t* vals_out,
                           void* workspace, size_t workspace_bytes, cudaStream_t st,
                           unsigned int** err_out, unsigned int* err_ext = nullptr);
gs_status radix_sort_pairs32(const uint32_t* keys, const uint32_t* vals, const int64_t* n_dev,
                             int64_t n_cap, int key_bits, uint32_t* keys_out, uint32_t* vals_out,
                             void* workspace, size_t workspace_bytes, cudaStream_t st,
                             unsigned int** err_out, unsigned int* err_ext = nullptr);

struct RectPairArgs;
// Stable sort by cell id of the (Gaussian, cell) items that `src` describes (rect_pairs.cuh;
// cells of 2^sx x 2^sy tiles, sx and sy in {0, 1, 2}), *n_dev items (at most n_cap);
// digit_offsets holds each pass's exclusive digit offsets.
gs_status radix_sort_rect_pairs(const RectPairArgs& src, const int64_t* n_dev, int64_t n_cap,
                                int key_bits, const uint32_t* digit_offsets, uint32_t* vals_out,
                                void* workspace, size_t workspace_bytes, cudaStream_t st,
                                unsigned int* err_ext);

}  // namespace gs
