// common.cuh -- shared definitions for the gs200 CUDA library (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>

#include "../../include/gs200.h"

namespace gs {

// Thread-local message read back through gs_last_error().
void set_error(const char* fmt, ...);
void clear_error();

// Device-side error word (one per call site family). Kernels OR error bits into
// it; the host reads it after the call and maps it to a status code.
enum DeviceError : unsigned int {
    DEV_OK = 0u,
    DEV_OVERFLOW = 1u,       // a data-dependent count exceeded a buffer's capacity
    DEV_TIMEOUT = 2u,        // a bounded spin wait gave up
};

#define GS_CUDA_CHECK(expr)                                                        \
    do {                                                                           \
        cudaError_t err__ = (expr);                                                \
        if (err__ != cudaSuccess) {                                                \
            ::gs::set_error("%s:%d: %s: %s", __FILE__, __LINE__, #expr,            \
                            cudaGetErrorString(err__));                            \
            return GS_ERR_CUDA;                                                    \
        }                                                                          \
    } while (0)

// Every kernel launch of the library is followed by exactly one GS_CHECK_LAUNCH, which
// also counts it (gs_launch_count).
void count_launch();
#define GS_CHECK_LAUNCH()                                                          \
    do {                                                                           \
        ::gs::count_launch();                                                      \
        cudaError_t err__ = cudaGetLastError();                                    \
        if (err__ != cudaSuccess) {                                                \
            ::gs::set_error("%s:%d: kernel launch: %s", __FILE__, __LINE__,        \
                            cudaGetErrorString(err__));                            \
            return GS_ERR_CUDA;                                                    \
        }                                                                          \
    } while (0)

#define GS_ARG_CHECK(cond, ...)                                                    \
    do {                                                                           \
        if (!(cond)) {                                                             \
            ::gs::set_error(__VA_ARGS__);                                          \
            return GS_ERR_ARG;                                                     \
        }                                                                          \
    } while (0)

constexpr int kNumSMs = 148;

// RAII CUDA-event pair around a launch site, recorded only while gs_timing_enable(1)
// is in effect on this host thread (see gs_timing_report).
class KernelTimer {
  public:
    KernelTimer(const char* name, cudaStream_t st);
    ~KernelTimer();
    KernelTimer(const KernelTimer&) = delete;
    KernelTimer& operator=(const KernelTimer&) = delete;

  private:
    const char* name_;
    cudaStream_t st_;
    bool on_;
    void* start_ = nullptr;
};
bool timing_enabled();

inline unsigned int div_up(int64_t a, int64_t b) { return (unsigned int)((a + b - 1) / b); }

// Sub-allocator over a caller-provided workspace: every piece is 256-byte aligned.
struct Workspace {
    char* base;
    size_t size;
    size_t used;
    __host__ Workspace(void* p, size_t n) : base((char*)p), size(n), used(0) {}
    template <typename T>
    __host__ T* take(size_t count) {
        size_t off = (used + 255) & ~(size_t)255;
        used = off + count * sizeof(T);
        if (base == nullptr || used > size) return nullptr;
        return (T*)(base + off);
    }
    __host__ bool ok() const { return base != nullptr && used <= size; }
};

// Sizes a workspace layout with the same calls as Workspace::take.
struct WorkspaceSizer {
    size_t used = 0;
    template <typename T>
    void take(size_t count) {
        used = ((used + 255) & ~(size_t)255) + count * sizeof(T);
    }
    size_t bytes() const { return used + 256; }
};

}  // namespace gs
