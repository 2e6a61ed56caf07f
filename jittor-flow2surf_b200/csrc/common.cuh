// Shared helpers for the sm_100a kernels and the C-ABI: status codes, the
// per-thread error message, launch checks and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "flow2surf_b200.h"

namespace f2s {

// Record a formatted message for f2s_last_error() and return `code`.
int fail(int code, const char* fmt, ...);

// Return F2S_OK, or F2S_ERR_CUDA with the pending launch error named.
int check_launch(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Number of SMs on the current device (cached per device).
int sm_count();

// Per-launch device timing (CUDA events around each kernel launch), off by
// default; f2s_trace_enable / f2s_trace_collect expose it through the C-ABI.
enum TraceTag {
    kTagKnn = 0,
    kTagInputEmbed,
    kTagCondition,
    kTagGemmContent,
    kTagEdge,
    kTagGemmHead,
    kTagRowNorm,
    kTagGemmQkv,
    kTagAttnColstats,
    kTagAttnOutput,
    kTagGemmProj,
    kTagGemmSwiGlu,
    kTagGemmFf2,
    kTagGemmDecoder,
    kTagFps,
    kTagPatchIndex,
    kTagFusionBuild,
    kTagGather,
    kTagFuseEuler,
    kTagNearest,
    kTagTranspose,
    kTagTraining,
    kTagCount
};

class TraceScope {
  public:
    TraceScope(int tag, cudaStream_t stream);
    ~TraceScope();
    TraceScope(const TraceScope&) = delete;
    TraceScope& operator=(const TraceScope&) = delete;

  private:
    int tag_;
    cudaStream_t stream_;
    cudaEvent_t start_ = nullptr;
};

}  // namespace f2s

#define F2S_REQUIRE(cond, ...)                                        \
    do {                                                              \
        if (!(cond)) return f2s::fail(F2S_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
    } while (0)

#define F2S_LIMIT(cond, ...)                                          \
    do {                                                              \
        if (!(cond)) return f2s::fail(F2S_ERR_UNSUPPORTED, __VA_ARGS__); \
    } while (0)

#define F2S_CUDA_TRY(expr)                                            \
    do {                                                              \
        cudaError_t err_ = (expr);                                    \
        if (err_ != cudaSuccess)                                      \
            return f2s::fail(F2S_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(err_)); \
    } while (0)

#define F2S_TRY(expr)                                                 \
    do {                                                              \
        int st_ = (expr);                                             \
        if (st_ != F2S_OK) return st_;                                \
    } while (0)

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

// Order-preserving map from float bits to uint32 (the key of the reference's
// flow2surf_neighbor_key, knn.cuh:7-17): -0 is folded onto +0 first, negative
// values flip all bits, non-negative values flip the sign bit.
__device__ __forceinline__ uint32_t f2s_ordered_bits(float d) {
    const float canonical = d == 0.0f ? 0.0f : d;
    const uint32_t bits = __float_as_uint(canonical);
    return bits ^ ((bits & 0x80000000u) ? 0xffffffffu : 0x80000000u);
}

__device__ __forceinline__ float f2s_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float f2s_warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float f2s_gelu_erf(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

__device__ __forceinline__ float f2s_silu(float x) { return x / (1.0f + expf(-x)); }

// Approximate reciprocal / base-2 exponential (the hardware's approximate
// instructions, denormals flushed): for tensor-core paths whose operands are
// rounded far more coarsely than these results.
__device__ __forceinline__ float f2s_rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ float f2s_ex2_approx(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// silu(x) = x / (1 + 2^(-x log2 e)) on the approximate instructions.
__device__ __forceinline__ float f2s_silu_approx(float x) {
    return x * f2s_rcp_approx(1.0f + f2s_ex2_approx(-1.44269504088896341f * x));
}

__device__ __forceinline__ float f2s_leaky(float x) { return x > 0.0f ? x : 0.2f * x; }

// Round to the nearest tf32 value (10-bit mantissa, ties away from zero).
// Tensor cores read an fp32 operand as tf32 by dropping the low 13 mantissa
// bits; rounding first makes that error unbiased and half as large.
__device__ __forceinline__ float f2s_round_tf32(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & 0xffffe000u;
    return __uint_as_float(u);
}
