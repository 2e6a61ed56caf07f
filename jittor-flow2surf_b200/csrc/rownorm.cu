// Row-wise channel LayerNorms of the point-major activations (one warp per
// point). All follow ChannelLayerNorm (flow2surf/models/layers.py:20-27):
// two-pass mean / variance over channels, eps 1e-6.
#include "kernels.cuh"

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

// AdaLN-Zero modulate(norm(x), shift, scale) (transformer.py:10-12,85,88).
__global__ void ln_modulate_kernel(const float* __restrict__ x, int ldx, float* __restrict__ h,
                                   int ldh, const float* __restrict__ mod, int mod_stride,
                                   int scale_off, int shift_off, int rows, int rows_per_patch,
                                   int C, bool round_tf32) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + (size_t)row * ldx;
    float mean, rstd;
    row_stats(xr, C, lane, mean, rstd);
    const float* m = mod + (size_t)(row / rows_per_patch) * mod_stride;
    float* hr = h + (size_t)row * ldh;
    for (int c = lane; c < C; c += 32) {
        const float v = (xr[c] - mean) * rstd * (1.0f + m[scale_off + c]) + m[shift_off + c];
        hr[c] = round_tf32 ? f2s_round_tf32(v) : v;
    }
}

// Affine ChannelLayerNorm + LeakyReLU(0.2) (encoder.py:118-123, decoder.py:18-22).
__global__ void ln_affine_leaky_kernel(float* __restrict__ y, int ldy,
                                       const float* __restrict__ gamma,
                                       const float* __restrict__ beta, int rows, int C,
                                       bool round_tf32) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float* yr = y + (size_t)row * ldy;
    float mean, rstd;
    row_stats(yr, C, lane, mean, rstd);
    for (int c = lane; c < C; c += 32) {
        const float v = f2s_leaky((yr[c] - mean) * rstd * gamma[c] + beta[c]);
        yr[c] = round_tf32 ? f2s_round_tf32(v) : v;
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
    ln_modulate_kernel<<<ceil_div(rows, kRowsPerCta), kRowsPerCta * 32, 0, stream>>>(
        x, ldx, h, ldh, mod, mod_stride, scale_off, shift_off, rows, rows_per_patch, C, round_tf32);
    return check_launch("ln_modulate_kernel");
}

int ln_affine_leaky(float* y, int ldy, const float* gamma, const float* beta, int rows, int C,
                    bool round_tf32, cudaStream_t stream) {
    if (rows == 0) return F2S_OK;
    TraceScope trace(kTagRowNorm, stream);
    ln_affine_leaky_kernel<<<ceil_div(rows, kRowsPerCta), kRowsPerCta * 32, 0, stream>>>(
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
