// Offset attention, fp32 SIMT two-pass form.
//
// Reference semantics (flow2surf/models/ops/attention.py:15-19):
//   S = Q K (no 1/sqrt(d) scale), P = softmax of S over the QUERY axis,
//   W = P / (row sum of P over keys + 1e-9), A = W V.
// Column softmax means every key j needs a statistic over all queries, so the
// N x N matrix is never stored: pass 1 computes each key's log-sum-exp
// L_j = max_i S_ij + log sum_i exp(S_ij - max_i S_ij); pass 2 streams key
// tiles and accumulates, per query, sum_j exp(S_ij - L_j) V_j and
// sum_j exp(S_ij - L_j) (each term <= 1, so no online rescaling), then divides.
// The trunk fuses the offset h - A (transformer.py:66-68) into pass 2.
#include <cfloat>

#include "kernels.cuh"

namespace f2s {
namespace {

constexpr int TQ = 64;  // queries per tile
constexpr int TK = 64;  // keys per tile

// Pass 1: one CTA per (patch, 64 keys); streams all query tiles.
__global__ void __launch_bounds__(256)
attn_colstats_kernel(const float* __restrict__ q, const float* __restrict__ k, int ld, int N,
                     int d, int key_tiles, float* __restrict__ L) {
    extern __shared__ __align__(16) float sm[];
    const int dp = d + 1;
    float* Ks = sm;                 // [TK][dp]
    float* Qs = Ks + TK * dp;       // [TQ][dp]
    float* Ss = Qs + TQ * dp;       // [TQ][TK + 1]
    const int b = blockIdx.x / key_tiles;
    const int k0 = (blockIdx.x - b * key_tiles) * TK;
    const size_t base = (size_t)b * N;
    const int tid = threadIdx.x;

    for (int i = tid; i < TK * d; i += 256) {
        const int r = i / d, c = i - r * d;
        Ks[r * dp + c] = (k0 + r < N) ? k[(base + k0 + r) * ld + c] : 0.0f;
    }
    // online (max, sum) for key column `col`, 4 threads per column
    const int col = tid >> 2, part = tid & 3;
    float m = -FLT_MAX, s = 0.0f;
    const int ty = tid >> 4, tx = tid & 15;

    for (int q0 = 0; q0 < N; q0 += TQ) {
        __syncthreads();
        for (int i = tid; i < TQ * d; i += 256) {
            const int r = i / d, c = i - r * d;
            Qs[r * dp + c] = (q0 + r < N) ? q[(base + q0 + r) * ld + c] : 0.0f;
        }
        __syncthreads();
        float acc[4][4] = {};
        for (int c = 0; c < d; ++c) {
            float a[4], bb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = Qs[(ty * 4 + i) * dp + c];
#pragma unroll
            for (int j = 0; j < 4; ++j) bb[j] = Ks[(tx + 16 * j) * dp + c];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) Ss[(ty * 4 + i) * (TK + 1) + tx + 16 * j] = acc[i][j];
        __syncthreads();
        for (int r = part * 16; r < part * 16 + 16; ++r) {
            if (q0 + r >= N) break;
            const float v = Ss[r * (TK + 1) + col];
            if (v > m) {
                s = s * expf(m - v) + 1.0f;
                m = v;
            } else {
                s += expf(v - m);
            }
        }
    }
    // combine the 4 partial (max, sum) of each column
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        const float mm = fmaxf(m, m2);
        s = (s > 0.0f ? s * expf(m - mm) : 0.0f) + (s2 > 0.0f ? s2 * expf(m2 - mm) : 0.0f);
        m = mm;
    }
    if (part == 0 && k0 + col < N) L[base + k0 + col] = m + logf(s);
}

// Pass 2: one CTA per (patch, 64 queries); streams all key tiles.
// out = (h ? h - A : A), A = sum_j p_ij V_j / (sum_j p_ij + 1e-9).
template <int CJ>  // value columns per thread: C <= 16 * CJ
__global__ void __launch_bounds__(256)
attn_output_kernel(const float* __restrict__ q, const float* __restrict__ k, int ldqk,
                   const float* __restrict__ v, int ldv, const float* __restrict__ L,
                   const float* __restrict__ h, int ldh, float* __restrict__ out, int ldo,
                   int N, int d, int C, int query_tiles, bool round_tf32) {
    extern __shared__ __align__(16) float sm[];
    const int dp = d + 1;
    float* Qs = sm;                    // [TQ][dp]
    float* Ks = Qs + TQ * dp;          // [TK][dp]
    float* Vs = Ks + TK * dp;          // [TK][C]
    float* Ps = Vs + TK * C;           // [TQ][TK + 1]
    float* Ls = Ps + TQ * (TK + 1);    // [TK]
    const int b = blockIdx.x / query_tiles;
    const int q0 = (blockIdx.x - b * query_tiles) * TQ;
    const size_t base = (size_t)b * N;
    const int tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;

    for (int i = tid; i < TQ * d; i += 256) {
        const int r = i / d, c = i - r * d;
        Qs[r * dp + c] = (q0 + r < N) ? q[(base + q0 + r) * ldqk + c] : 0.0f;
    }
    float acc[4][CJ];
    float den[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        den[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < CJ; ++j) acc[i][j] = 0.0f;
    }

    for (int k0 = 0; k0 < N; k0 += TK) {
        __syncthreads();
        for (int i = tid; i < TK * d; i += 256) {
            const int r = i / d, c = i - r * d;
            Ks[r * dp + c] = (k0 + r < N) ? k[(base + k0 + r) * ldqk + c] : 0.0f;
        }
        for (int i = tid; i < TK * C; i += 256) {
            const int r = i / C, c = i - r * C;
            Vs[i] = (k0 + r < N) ? v[(base + k0 + r) * ldv + c] : 0.0f;
        }
        if (tid < TK) Ls[tid] = (k0 + tid < N) ? L[base + k0 + tid] : 0.0f;
        __syncthreads();
        float s[4][4] = {};
        for (int c = 0; c < d; ++c) {
            float a[4], bb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = Qs[(ty * 4 + i) * dp + c];
#pragma unroll
            for (int j = 0; j < 4; ++j) bb[j] = Ks[(tx + 16 * j) * dp + c];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[i][j] = fmaf(a[i], bb[j], s[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kc = tx + 16 * j;
                Ps[(ty * 4 + i) * (TK + 1) + kc] =
                    (k0 + kc < N) ? expf(s[i][j] - Ls[kc]) : 0.0f;
            }
        __syncthreads();
        for (int kk = 0; kk < TK; ++kk) {
            float p[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                p[i] = Ps[(ty * 4 + i) * (TK + 1) + kk];
                den[i] += p[i];
            }
#pragma unroll
            for (int j = 0; j < CJ; ++j) {
                const int c = tx + 16 * j;
                const float vv = c < C ? Vs[kk * C + c] : 0.0f;
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[i][j] = fmaf(p[i], vv, acc[i][j]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = q0 + ty * 4 + i;
        if (r >= N) continue;
        const float inv = 1.0f / (den[i] + 1e-9f);
#pragma unroll
        for (int j = 0; j < CJ; ++j) {
            const int c = tx + 16 * j;
            if (c >= C) continue;
            const float a = acc[i][j] * inv;
            const float o = h ? h[(base + r) * ldh + c] - a : a;
            out[(base + r) * ldo + c] = round_tf32 ? f2s_round_tf32(o) : o;
        }
    }
}

template <int CJ>
int launch_output(const float* q, const float* k, int ldqk, const float* v, int ldv,
                  const float* L, const float* h, int ldh, float* out, int ldo, int B, int N,
                  int d, int C, bool round_tf32, cudaStream_t stream) {
    const int dp = d + 1;
    const size_t smem = sizeof(float) * ((size_t)TQ * dp + TK * dp + (size_t)TK * C +
                                         TQ * (TK + 1) + TK);
    auto kernel = attn_output_kernel<CJ>;
    F2S_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
    const int tiles = ceil_div(N, TQ);
    TraceScope trace(kTagAttnOutput, stream);
    kernel<<<B * tiles, 256, smem, stream>>>(q, k, ldqk, v, ldv, L, h, ldh, out, ldo, N, d, C,
                                             tiles, round_tf32);
    return check_launch("attn_output_kernel");
}

}  // namespace

int attention_f32(const float* q, const float* k, int ldqk, const float* v, int ldv,
                  const float* h, int ldh, float* out, int ldo, float* colstats, int B, int N,
                  int d, int C, bool round_tf32, cudaStream_t stream) {
    if (B == 0 || N == 0) return F2S_OK;
    F2S_LIMIT(d >= 1 && d <= 128, "attention: query/key width %d outside [1, 128]", d);
    F2S_LIMIT(C >= 1 && C <= 256, "attention: value width %d outside [1, 256]", C);
    const int dp = d + 1;
    const size_t smem1 = sizeof(float) * ((size_t)TK * dp + TQ * dp + TQ * (TK + 1));
    F2S_CUDA_TRY(cudaFuncSetAttribute(attn_colstats_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1));
    const int key_tiles = ceil_div(N, TK);
    {
    TraceScope trace(kTagAttnColstats, stream);
    attn_colstats_kernel<<<B * key_tiles, 256, smem1, stream>>>(q, k, ldqk, N, d, key_tiles,
                                                                colstats);
    F2S_TRY(check_launch("attn_colstats_kernel"));
    }
    const int cj = ceil_div(C, 16);
    if (cj <= 4) return launch_output<4>(q, k, ldqk, v, ldv, colstats, h, ldh, out, ldo, B, N, d, C, round_tf32, stream);
    if (cj <= 8) return launch_output<8>(q, k, ldqk, v, ldv, colstats, h, ldh, out, ldo, B, N, d, C, round_tf32, stream);
    if (cj <= 12) return launch_output<12>(q, k, ldqk, v, ldv, colstats, h, ldh, out, ldo, B, N, d, C, round_tf32, stream);
    return launch_output<16>(q, k, ldqk, v, ldv, colstats, h, ldh, out, ldo, B, N, d, C, round_tf32, stream);
}

}  // namespace f2s
