// runtime.cu -- error reporting and library-level queries of libgs200.so.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace gs {

static thread_local char t_error[1024] = {0};

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_error, sizeof(t_error), fmt, ap);
    va_end(ap);
}

void clear_error() { t_error[0] = '\0'; }

}  // namespace gs

extern "C" const char* gs_last_error(void) { return gs::t_error; }

extern "C" const char* gs_version(void) { return "gs200 0.1 sm_100a"; }

extern "C" gs_status gs_workspace_error(const void* workspace, void* stream) {
    gs::clear_error();
    GS_ARG_CHECK(workspace != nullptr, "gs_workspace_error: null workspace");
    // Workspace layouts start at the first 256-byte boundary (Workspace::take).
    const char* p = (const char*)(((uintptr_t)workspace + 255) & ~(uintptr_t)255);
    unsigned int err = 0;
    GS_CUDA_CHECK(cudaMemcpyAsync(&err, p, sizeof(err), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    GS_CUDA_CHECK(cudaStreamSynchronize((cudaStream_t)stream));
    if (err & gs::DEV_TIMEOUT) {
        gs::set_error("a bounded device wait timed out (look-back)");
        return GS_ERR_TIMEOUT;
    }
    if (err & gs::DEV_OVERFLOW) {
        gs::set_error("a device-side capacity was exceeded");
        return GS_ERR_OVERFLOW;
    }
    return GS_OK;
}

// ------------------------------------------------------------------ kernel timing
//
// Off by default. When enabled, launch sites wrapped in gs::KernelTimer record a CUDA
// event pair on the launching stream; gs_timing_report() synchronises those events
// and returns per-kernel totals. bench.py uses it to time the dominant kernel live.
#include <atomic>
#include <map>
#include <string>
#include <vector>

namespace gs {

struct TimingLog {
    bool enabled = false;
    std::vector<cudaEvent_t> pool;
    size_t next = 0;
    std::vector<std::pair<std::string, std::pair<cudaEvent_t, cudaEvent_t>>> marks;
};
static thread_local TimingLog t_timing;

static cudaEvent_t timing_event() {
    TimingLog& L = t_timing;
    if (L.next == L.pool.size()) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        L.pool.push_back(e);
    }
    return L.pool[L.next++];
}

bool timing_enabled() { return t_timing.enabled; }

KernelTimer::KernelTimer(const char* name, cudaStream_t st) : name_(name), st_(st), on_(t_timing.enabled) {
    if (on_) {
        start_ = timing_event();
        cudaEventRecord((cudaEvent_t)start_, st_);
    }
}

KernelTimer::~KernelTimer() {
    if (!on_) return;
    cudaEvent_t end = timing_event();
    cudaEventRecord(end, st_);
    t_timing.marks.push_back({name_, {(cudaEvent_t)start_, end}});
}

static std::atomic<int64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

}  // namespace gs

extern "C" int64_t gs_launch_count(void) { return gs::g_launches.load(std::memory_order_relaxed); }

extern "C" void gs_timing_enable(int32_t on) {
    gs::t_timing.enabled = on != 0;
}

extern "C" void gs_timing_reset(void) {
    gs::t_timing.marks.clear();
    gs::t_timing.next = 0;
}

extern "C" int32_t gs_timing_report(char* names, size_t names_len, double* total_ms,
                                    int64_t* launches, int32_t max_kernels) {
    gs::TimingLog& L = gs::t_timing;
    std::map<std::string, std::pair<double, int64_t>> agg;
    std::vector<std::string> order;
    for (auto& m : L.marks) {
        float ms = 0.0f;
        cudaEventSynchronize(m.second.second);
        cudaEventElapsedTime(&ms, m.second.first, m.second.second);
        auto it = agg.find(m.first);
        if (it == agg.end()) {
            order.push_back(m.first);
            agg[m.first] = {ms, 1};
        } else {
            it->second.first += ms;
            it->second.second += 1;
        }
    }
    std::string joined;
    int k = 0;
    for (auto& name : order) {
        if (k >= max_kernels) break;
        total_ms[k] = agg[name].first;
        launches[k] = agg[name].second;
        joined += name;
        joined += '\n';
        ++k;
    }
    if (names && names_len) {
        size_t n = joined.size() < names_len - 1 ? joined.size() : names_len - 1;
        memcpy(names, joined.data(), n);
        names[n] = '\0';
    }
    return k;
}
