// Row-wise channel LayerNorms of the point-major activations (one warp per
// point). All follow ChannelLayerNorm (flow2surf/models/layers.py:20-27):
// two-pass mean / variance over channels, eps 1e-6.
#include <cuda_fp16.h>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace f2s {
namespace {

__device__ __forceinline__ void row_stats(const float* x, int C, int lane, float& mean,
                                          float& rstd) {
    float s = 0.0f;
    for (int c = lane; c < C; c += 32) s += x[c];
    mean = f2s_warp_sum(s) / (float)C;
    float q = 0.0f;
    for (int c = lane; c < C; c += 32) {
        const float d = x[c] - mean;
        q = fmaf(d, d, q);
    }
    rstd = rsqrtf(f2s_warp_sum(q) / (float)C + 1e-6f);
}

// Rows of up to 256 channels held in registers: lane `l` owns the float2
// pairs (l + 32 i) for i < kPairs, so a row is read from HBM once with
// coalesced 8-byte loads.
constexpr int kPairs = 4;

__device__ __forceinline__ void row_load(const float* x, int C, int lane, float2 (&v)[kPairs]) {
#pragma unroll
    for (int i = 0; i < kPairs; ++i) {
        const int c = 2 * (lane + 32 * i);
        v[i] = c < C ? *reinterpret_cast<const float2*>(x + c) : make_float2(0.0f, 0.0f);
    }
}

__device__ __forceinline__ void row_stats_reg(const float2 (&v)[kPairs], int C, int lane,
                                              float& mean, float& rstd) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kPairs; ++i) s += v[i].x + v[i].y;
    mean = f2s_warp_sum(s) / (float)C;
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < kPairs; ++i) {
        if (2 * (lane + 32 * i) < C) {
            const float d0 = v[i].x - mean, d1 = v[i].y - mean;
            q = fmaf(d0, d0, q);
            q = fmaf(d1, d1, q);
        }
    }
    rstd = rsqrtf(f2s_warp_sum(q) / (float)C + 1e-6f);
}

// AdaLN-Zero modulate(norm(x), shift, scale) (transformer.py:10-12,85,88).
// kPaired: C even, C <= 256, 8-byte aligned rows (the register path).
// kHalf (paired only): h is fp16, values out of its range set *err.
template <bool kPaired, bool kHalf = false>
__global__ void ln_modulate_kernel(const float* __restrict__ x, int ldx, void* __restrict__ h_out,
                                   int ldh, const float* __restrict__ mod, int mod_stride,
                                   int scale_off, int shift_off, int rows, int rows_per_patch,
                                   int C, bool round_tf32, int* err) {
    float* h = static_cast<float*>(h_out);
    const int lane = threadIdx.x & 31;
    if constexpr (kPaired) {
        // two rows per warp, both loaded before either is reduced
        const int row0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 2;
        if (row0 >= rows) return;
        float2 v[2][kPairs];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            if (row0 + q < rows) row_load(x + (size_t)(row0 + q) * ldx, C, lane, v[q]);
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int row = row0 + q;
            if (row >= rows) break;
            float mean, rstd;
            row_stats_reg(v[q], C, lane, mean, rstd);
            const float* m = mod + (size_t)(row / rows_per_patch) * mod_stride;
            float* hr = h + (size_t)row * ldh;
            __half* hr16 = static_cast<__half*>(h_out) + (size_t)row * ldh;
            bool out_of_range = false;
#pragma unroll
            for (int i = 0; i < kPairs; ++i) {
                const int c = 2 * (lane + 32 * i);
                if (c < C) {
                    const float2 sc = *reinterpret_cast<const float2*>(m + scale_off + c);
                    const float2 sh = *reinterpret_cast<const float2*>(m + shift_off + c);
                    float a = (v[q][i].x - mean) * rstd * (1.0f + sc.x) + sh.x;
                    float b = (v[q][i].y - mean) * rstd * (1.0f + sc.y) + sh.y;
                    if constexpr (kHalf) {
                        out_of_range |= !(fabsf(a) < 65504.0f) || !(fabsf(b) < 65504.0f);
                        *reinterpret_cast<__half2*>(hr16 + c) = __floats2half2_rn(a, b);
                    } else {
                        if (round_tf32) {
                            a = f2s_round_tf32(a);
                            b = f2s_round_tf32(b);
                        }
                        *reinterpret_cast<float2*>(hr + c) = make_float2(a, b);
                    }
                }
            }
            if (kHalf && out_of_range) atomicExch(err, tc::kTcFp16Range);
        }
    } else {
        const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
        if (row >= rows) return;
        const float* xr = x + (size_t)row * ldx;
        const float* m = mod + (size_t)(row / rows_per_patch) * mod_stride;
        float* hr = h + (size_t)row * ldh;
        float mean, rstd;
        row_stats(xr, C, lane, mean, rstd);
        for (int c = lane; c < C; c += 32) {
            const float v = (xr[c] - mean) * rstd * (1.0f + m[scale_off + c]) + m[shift_off + c];
            hr[c] = round_tf32 ? f2s_round_tf32(v) : v;
        }
    }
}

// Affine ChannelLayerNorm + LeakyReLU(0.2) (encoder.py:118-123, decoder.py:18-22).
template <bool kPaired>
__global__ void ln_affine_leaky_kernel(float* __restrict__ y, int ldy,
                                       const float* __restrict__ gamma,
                                       const float* __restrict__ beta, int rows, int C,
                                       bool round_tf32) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float* yr = y + (size_t)row * ldy;
    float mean, rstd;
    if constexpr (kPaired) {
        float2 v[kPairs];
        row_load(yr, C, lane, v);
        row_stats_reg(v, C, lane, mean, rstd);
#pragma unroll
        for (int i = 0; i < kPairs; ++i) {
            const int c = 2 * (lane + 32 * i);
            if (c < C) {
                float a = f2s_leaky((v[i].x - mean) * rstd * gamma[c] + beta[c]);
                float b = f2s_leaky((v[i].y - mean) * rstd * gamma[c + 1] + beta[c + 1]);
                if (round_tf32) {
                    a = f2s_round_tf32(a);
                    b = f2s_round_tf32(b);
                }
                *reinterpret_cast<float2*>(yr + c) = make_float2(a, b);
            }
        }
    } else {
        row_stats(yr, C, lane, mean, rstd);
        for (int c = lane; c < C; c += 32) {
            const float v = f2s_leaky((yr[c] - mean) * rstd * gamma[c] + beta[c]);
            yr[c] = round_tf32 ? f2s_round_tf32(v) : v;
        }
    }
}

// qk_norm on the query and key blocks of qkv (transformer.py:59-63).
__global__ void qk_norm_kernel(float* __restrict__ qkv, int ld, int rows, int d) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    for (int part = 0; part < 2; ++part) {
        float* r = qkv + (size_t)row * ld + part * d;
        float mean, rstd;
        row_stats(r, d, lane, mean, rstd);
        for (int c = lane; c < d; c += 32) r[c] = (r[c] - mean) * rstd;
    }
}

constexpr int kRowsPerCta = 8;

}  // namespace

int ln_modulate(const float* x, int ldx, float* h, int ldh, const float* mod, int mod_stride,
                int scale_off, int shift_off, int rows, int rows_per_patch, int C,
                bool round_tf32, cudaStream_t stream) {
    if (rows == 0) return F2S_OK;
    TraceScope trace(kTagRowNorm, stream);
    const bool paired = C % 2 == 0 && C <= 64 * kPairs && ldx % 2 == 0 && ldh % 2 == 0 &&
                        ((uintptr_t)x & 7) == 0 && ((uintptr_t)h & 7) == 0 &&
                        ((uintptr_t)mod & 7) == 0 && mod_stride % 2 == 0 && scale_off % 2 == 0 &&
                        shift_off % 2 == 0;
    auto kernel = paired ? ln_modulate_kernel<true> : ln_modulate_kernel<false>;
    const int rows_per_cta = paired ? 2 * kRowsPerCta : kRowsPerCta;
    kernel<<<ceil_div(rows, rows_per_cta), kRowsPerCta * 32, 0, stream>>>(
        x, ldx, h, ldh, mod, mod_stride, scale_off, shift_off, rows, rows_per_patch, C, round_tf32,
        nullptr);
    return check_launch("ln_modulate_kernel");
}

int ln_modulate_f16(const float* x, int ldx, void* h, int ldh, const float* mod, int mod_stride,
                    int scale_off, int shift_off, int rows, int rows_per_patch, int C,
                    cudaStream_t stream) {
    if (rows == 0) return F2S_OK;
    const bool paired = C % 2 == 0 && C <= 64 * kPairs && ldx % 2 == 0 && ldh % 2 == 0 &&
                        ((uintptr_t)x & 7) == 0 && ((uintptr_t)h & 3) == 0 &&
                        ((uintptr_t)mod & 7) == 0 && mod_stride % 2 == 0 && scale_off % 2 == 0 &&
                        shift_off % 2 == 0;
    if (!paired) return fail(F2S_ERR_UNSUPPORTED, "ln_modulate_f16: shape outside the register path");
    int* err = tc_error_word();
    if (!err) return fail(F2S_ERR_CUDA, "ln_modulate_f16: device error word unavailable");
    TraceScope trace(kTagRowNorm, stream);
    ln_modulate_kernel<true, true><<<ceil_div(rows, 2 * kRowsPerCta), kRowsPerCta * 32, 0, stream>>>(
        x, ldx, h, ldh, mod, mod_stride, scale_off, shift_off, rows, rows_per_patch, C, false, err);
    return check_launch("ln_modulate_kernel");
}

int ln_affine_leaky(float* y, int ldy, const float* gamma, const float* beta, int rows, int C,
                    bool round_tf32, cudaStream_t stream) {
    if (rows == 0) return F2S_OK;
    TraceScope trace(kTagRowNorm, stream);
    const bool paired = C % 2 == 0 && C <= 64 * kPairs && ldy % 2 == 0 && ((uintptr_t)y & 7) == 0;
    auto kernel = paired ? ln_affine_leaky_kernel<true> : ln_affine_leaky_kernel<false>;
    kernel<<<ceil_div(rows, kRowsPerCta), kRowsPerCta * 32, 0, stream>>>(
        y, ldy, gamma, beta, rows, C, round_tf32);
    return check_launch("ln_affine_leaky_kernel");
}

int qk_norm(float* qkv, int ld, int rows, int d, cudaStream_t stream) {
    if (rows == 0) return F2S_OK;
    TraceScope trace(kTagRowNorm, stream);
    qk_norm_kernel<<<ceil_div(rows, kRowsPerCta), kRowsPerCta * 32, 0, stream>>>(qkv, ld, rows,
                                                                                 d);
    return check_launch("qk_norm_kernel");
}

}  // namespace f2s
