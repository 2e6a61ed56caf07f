// Building blocks shared by the tensor-core neighbour-stage kernels
// (edge_tc.cu, edge_tcu.cu): shared-memory layouts and copies, packed fp32x2
// arithmetic, the GELU of the hidden rows, and the per-CTA preparation of the
// weights (the HPE LayerNorm folded into the pre-activation contraction, the
// composed projection W_po in bf16 halves, the message-norm affine).
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace f2s {
namespace edge {

constexpr int kRows = 128;  // edge rows per tile (the MMA's M)
constexpr uint32_t kUBytes = kRows * 32;  // one 128 x 8 tf32 operand in the interleaved layout

// Byte offset of 16-byte chunk `chunk` of row `row` inside a K-block of
// 128-byte rows in the 128-byte-swizzle layout (8-row atoms of 1024 bytes).
__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 16-byte global -> shared copy through L2 only (the content rows are read
// once per tile), tracked per thread by commit groups.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// Bring `bytes` (a multiple of 16) at a 16-byte aligned global address into L2.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ float4 lds128(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ float lds32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// wait until at most `pending` (0 .. 3) of this thread's groups are in flight
__device__ __forceinline__ void cp_async_wait(int pending) {
    switch (pending) {
        case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    }
}

__device__ __forceinline__ uint32_t pack_bf16(float lo_elem, float hi_elem) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(lo_elem, hi_elem);
    return *reinterpret_cast<const uint32_t*>(&b);
}

// Byte offset of 16-byte chunk `chunk` of row `row` in the interleaved
// (no-swizzle) K-major layout of 32-byte rows: 8-row core matrices of 128
// bytes, the two K chunks 128 bytes apart, 8-row groups 256 bytes apart.
__device__ __forceinline__ uint32_t interleaved_offset(int row, int chunk) {
    return (uint32_t)((row >> 3) * 256 + chunk * 128 + (row & 7) * 16);
}

// Packed fp32x2 arithmetic of sm_100 (one instruction, two lanes of fp32,
// each rounded as the scalar operation is): the per-edge CUDA-core work of
// this kernel is issue-bound, so pairs of channels go through one issue slot.
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }


// GELU(x) = x * Phi(x) with Phi from the erf approximation of Abramowitz and
// Stegun, Handbook of Mathematical Functions, eq. 7.1.26 (after Hastings):
//   erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2),
//   t = 1 / (1 + p z), z >= 0, |error| <= 1.5e-7.
// With z = |x| / sqrt(2) and q = (1 - erf(z)) / 2, Phi(x) = q for x < 0 and
// 1 - q otherwise, so GELU(x) = max(x, 0) - |x| q for every x (no select, no
// cancellation in the negative tail). The constants fold in 1/2, 1/sqrt(2)
// and log2(e) / 2 (exp(-x^2 / 2) = 2^(-x^2 log2(e) / 2)). Within 3.5e-7 of
// the exact GELU in float32, far below the operand rounding of the
// tensor-core contraction the hidden rows feed (2^-18 relative at best).
// Applied to two values at once; the polynomial's coefficients are negated
// so that the final step is max(x, 0) + |x| (-q t e).
__device__ __forceinline__ float2 gelu_as2(float2 x) {
    const float2 ax = make_float2(fabsf(x.x), fabsf(x.y));
    const float2 den = fma2(f2(0.23164189f), ax, f2(1.0f));
    const float2 t = make_float2(f2s_rcp_approx(den.x), f2s_rcp_approx(den.y));
    float2 q = fma2(t, f2(-0.5307027145f), f2(0.7265760135f));
    q = fma2(t, q, f2(-0.7107068705f));
    q = fma2(t, q, f2(0.142248368f));
    q = fma2(t, q, f2(-0.127414796f));
    const float2 s = mul2(x, mul2(x, f2(-0.72134752f)));
    const float2 e = make_float2(f2s_ex2_approx(s.x), f2s_ex2_approx(s.y));
    const float2 nqte = mul2(mul2(q, t), e);
    return fma2(ax, nqte, make_float2(fmaxf(x.x, 0.0f), fmaxf(x.y, 0.0f)));
}

// The HPE LayerNorm is folded into the pre-activation contraction. The mean
// over the hidden channels of h = W_in g + b_in is linear in g, so with
// column-centred weights W~ = W_in - mean_c(W_in), b~ = b_in - mean_c(b_in),
// h - mean(h) = W~ g + b~ and
//   LN(h)_c = gamma_c rstd (W~_c g + b~_c) + beta_c
//           = [gamma_c W~_c | gamma_c b~_c | beta_c] . [rstd g | rstd | 1],
// a K = 8 row product whose u row carries the per-edge 1/std; the variance is
// g^T G g + 2 a.g + c with G, a, c the moments of the centred rows.
// Writes the B operand of that product (H rows of 8 as tf32 hi, then lo, in
// the interleaved layout) to sWu and G, a, c to sGram[43]; `mean_scratch`
// holds 7 doubles. Every thread of the CTA calls it (one __syncthreads inside).
__device__ __forceinline__ void prepare_pre_activation(const float* hpe_w, const float* hpe_b,
                                                       const float* hpe_ln_w,
                                                       const float* hpe_ln_b, int H,
                                                       double* mean_scratch, unsigned char* sWu,
                                                       float* sGram, int tid, int nthreads) {
    double* sMean = mean_scratch;
    if (tid < 7) {
        double acc = 0.0;
        for (int c = 0; c < H; ++c)
            acc += tid < 6 ? (double)hpe_w[(size_t)c * 6 + tid] : (double)hpe_b[c];
        sMean[tid] = acc / (double)H;
    }
    __syncthreads();
    for (int c = tid; c < H; c += nthreads) {
        const float* w = hpe_w + (size_t)c * 6;
        const double gamma = hpe_ln_w[c];
        float row8[8];
#pragma unroll
        for (int e = 0; e < 6; ++e) row8[e] = (float)(gamma * ((double)w[e] - sMean[e]));
        row8[6] = (float)(gamma * ((double)hpe_b[c] - sMean[6]));
        row8[7] = hpe_ln_b[c];
        float hi[8], lo[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            hi[e] = f2s_round_tf32(row8[e]);
            lo[e] = row8[e] - hi[e];
        }
        for (int ch = 0; ch < 2; ++ch) {
            const uint32_t off = interleaved_offset(c, ch);
            *reinterpret_cast<float4*>(sWu + off) =
                make_float4(hi[4 * ch], hi[4 * ch + 1], hi[4 * ch + 2], hi[4 * ch + 3]);
            *reinterpret_cast<float4*>(sWu + (size_t)H * 32 + off) =
                make_float4(lo[4 * ch], lo[4 * ch + 1], lo[4 * ch + 2], lo[4 * ch + 3]);
        }
    }
    if (tid < 43) {
        // moments of the centred rows over the hidden channels, in double:
        // G (36), a (6), c
        double acc = 0.0;
        for (int c = 0; c < H; ++c) {
            const float* w = hpe_w + (size_t)c * 6;
            const double bt = (double)hpe_b[c] - sMean[6];
            if (tid < 36) {
                const int d = tid / 6, e = tid % 6;
                acc += ((double)w[d] - sMean[d]) * ((double)w[e] - sMean[e]);
            } else if (tid < 42) {
                acc += ((double)w[tid - 36] - sMean[tid - 36]) * bt;
            } else {
                acc += bt * bt;
            }
        }
        sGram[tid] = (float)(acc / (double)H);
    }
}

// The message norm's per-channel constants: the projection bias, |gain| and
// shift, and the sign of the gain (the epilogues take the max over the K edge
// rows of sign * normalised value, then apply |gain| and the shift).
__device__ __forceinline__ void prepare_message_norm(const float* contrib_b, const float* ln_w,
                                                     const float* ln_b, int cout, float* sCb,
                                                     float* sLn, float* sSgn, int tid,
                                                     int nthreads) {
    for (int c = tid; c < cout; c += nthreads) {
        sCb[c] = contrib_b[c];
        sLn[2 * c] = fabsf(ln_w[c]);
        sLn[2 * c + 1] = ln_b[c];
        sSgn[c] = ln_w[c] < 0.0f ? -1.0f : 1.0f;
    }
}

// W_po (cout x H fp32) as bf16 high parts into sB and, when sBlo is given, the
// bf16 rounding of the remainders into sBlo: K-major, 128-byte swizzled
// K-blocks of 64 channels (cout rows of 128 bytes each), as TMA would write.
__device__ __forceinline__ void convert_projection(const float* contrib_w, int H, int cout,
                                                   unsigned char* sB, unsigned char* sBlo,
                                                   int tid, int nthreads) {
    const int chunks_per_row = H / 8;
    for (int t = tid; t < cout * chunks_per_row; t += nthreads) {
        const int n = t / chunks_per_row, q = t - n * chunks_per_row;
        const float4 w0 = *reinterpret_cast<const float4*>(contrib_w + (size_t)n * H + q * 8);
        const float4 w1 = *reinterpret_cast<const float4*>(contrib_w + (size_t)n * H + q * 8 + 4);
        const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(w[2 * e], w[2 * e + 1]);
            hi[e] = *reinterpret_cast<const uint32_t*>(&h2);
            lo[e] = pack_bf16(w[2 * e] - __bfloat162float(h2.x),
                              w[2 * e + 1] - __bfloat162float(h2.y));
        }
        const size_t off = (size_t)(q / 8) * cout * 128 + sw128_offset(n, q % 8);
        *reinterpret_cast<uint4*>(sB + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        if (sBlo) *reinterpret_cast<uint4*>(sBlo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// The u row [rstd g, rstd, 1] of edge row `row` from its geometry g (rstd =
// 1 / sqrt(var + 1e-5) of its pre-activations, the variance from the moments
// in sGram) as tf32 hi at sU and lo at sU + kUBytes.
__device__ __forceinline__ void write_u_row_g(unsigned char* sU, const float* sGram, int row,
                                              const float (&g)[6]) {
    float var = sGram[42];
#pragma unroll
    for (int d = 0; d < 6; ++d) {
        float t = 2.0f * sGram[36 + d];
#pragma unroll
        for (int e = 0; e < 6; ++e) t = fmaf(sGram[d * 6 + e], g[e], t);
        var = fmaf(t, g[d], var);
    }
    const float rstd = rsqrtf(fmaxf(var, 0.0f) + 1e-5f);
    const float u8[8] = {rstd * g[0], rstd * g[1], rstd * g[2], rstd * g[3],
                         rstd * g[4], rstd * g[5], rstd,        1.0f};
    float hi[8], lo[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        hi[e] = f2s_round_tf32(u8[e]);
        lo[e] = u8[e] - hi[e];
    }
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
        const uint32_t off = interleaved_offset(row, ch);
        *reinterpret_cast<float4*>(sU + off) =
            make_float4(hi[4 * ch], hi[4 * ch + 1], hi[4 * ch + 2], hi[4 * ch + 3]);
        *reinterpret_cast<float4*>(sU + kUBytes + off) =
            make_float4(lo[4 * ch], lo[4 * ch + 1], lo[4 * ch + 2], lo[4 * ch + 3]);
    }
}

// The same for g = [x_j - x_i, x_i] of centre point pi and neighbour pj.
__device__ __forceinline__ void write_u_row(unsigned char* sU, const float* sGram, int row,
                                            const float4& pi, const float4& pj) {
    const float g[6] = {pj.x - pi.x, pj.y - pi.y, pj.z - pi.z, pi.x, pi.y, pi.z};
    write_u_row_g(sU, sGram, row, g);
}

}  // namespace edge
}  // namespace f2s
