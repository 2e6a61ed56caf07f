// C-ABI plumbing: the per-thread error message and version query.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>
#include <vector>

#include "common.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

namespace f2s {

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess)
        return fail(F2S_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(err));
    return F2S_OK;
}

int sm_count() {
    static std::mutex cache_mutex;
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(cache_mutex);
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

namespace {

struct TraceRecord {
    int tag;
    cudaEvent_t start, stop;
};

std::mutex g_trace_mutex;
bool g_trace_enabled = false;
std::vector<TraceRecord> g_trace_records;
std::vector<cudaEvent_t> g_event_pool;

cudaEvent_t take_event() {
    if (!g_event_pool.empty()) {
        cudaEvent_t e = g_event_pool.back();
        g_event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    return e;
}

void release_records() {
    for (auto& r : g_trace_records) {
        g_event_pool.push_back(r.start);
        g_event_pool.push_back(r.stop);
    }
    g_trace_records.clear();
}

const char* const kTagNames[kTagCount] = {
    "knn",          "input_embed",  "condition",     "gemm_content", "edge_stage",
    "gemm_head",    "row_norm",     "gemm_qkv",      "attn_colstats", "attn_output",
    "gemm_proj",    "gemm_swiglu",  "gemm_ff2",      "gemm_decoder", "fps",
    "patch_index",  "fusion_build", "gather",        "fuse_euler",   "nearest",
    "transpose",    "training"};

}  // namespace

TraceScope::TraceScope(int tag, cudaStream_t stream) : tag_(tag), stream_(stream) {
    std::lock_guard<std::mutex> lock(g_trace_mutex);
    if (!g_trace_enabled) return;
    start_ = take_event();
    if (start_) cudaEventRecord(start_, stream_);
}

TraceScope::~TraceScope() {
    if (!start_) return;
    std::lock_guard<std::mutex> lock(g_trace_mutex);
    cudaEvent_t stop = take_event();
    if (!stop) {
        g_event_pool.push_back(start_);
        return;
    }
    cudaEventRecord(stop, stream_);
    g_trace_records.push_back({tag_, start_, stop});
}

}  // namespace f2s

extern "C" int f2s_trace_enable(int on) {
    std::lock_guard<std::mutex> lock(f2s::g_trace_mutex);
    f2s::release_records();
    f2s::g_trace_enabled = on != 0;
    return F2S_OK;
}

extern "C" int f2s_trace_tag_count(void) { return f2s::kTagCount; }

extern "C" const char* f2s_trace_tag_name(int tag) {
    return tag >= 0 && tag < f2s::kTagCount ? f2s::kTagNames[tag] : "";
}

extern "C" int f2s_trace_collect(double* total_ms, int64_t* launches) {
    std::lock_guard<std::mutex> lock(f2s::g_trace_mutex);
    if (!total_ms || !launches) return f2s::fail(F2S_ERR_INVALID_ARGUMENT, "trace: null pointer");
    for (int t = 0; t < f2s::kTagCount; ++t) {
        total_ms[t] = 0.0;
        launches[t] = 0;
    }
    for (auto& r : f2s::g_trace_records) {
        cudaError_t err = cudaEventSynchronize(r.stop);
        if (err != cudaSuccess)
            return f2s::fail(F2S_ERR_CUDA, "trace: %s", cudaGetErrorString(err));
        float ms = 0.0f;
        err = cudaEventElapsedTime(&ms, r.start, r.stop);
        if (err != cudaSuccess)
            return f2s::fail(F2S_ERR_CUDA, "trace: %s", cudaGetErrorString(err));
        total_ms[r.tag] += ms;
        launches[r.tag] += 1;
    }
    f2s::release_records();
    return F2S_OK;
}

extern "C" const char* f2s_last_error(void) { return g_last_error; }

extern "C" int f2s_version(void) { return 100; }
