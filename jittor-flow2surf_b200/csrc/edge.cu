// Fused neighbour stage, fp32 SIMT version: gather + HPE hidden + composed
// edge projection + content terms + LayerNorm + LeakyReLU + max over k, in
// one kernel. Nothing per-edge is written to HBM.
//
// Reference pieces fused here (the reference runs them as three kernels and
// writes the (B,N,K,H) hidden and (B,N,K,C) contribution tensors to HBM):
//   geometry [xyz_j - xyz_i, xyz_i]        flow2surf/models/encoder.py:26-37,85
//   hidden = GELU(LN(W_in g + b_in))       flow2surf/models/ops/hpe.py:14-43,
//     LN with var = max(E[h^2]-E[h]^2, 0), eps 1e-5   hpe_hidden_forward.cu:11-33
//   contrib = W_po hidden + b_po           hpe.py:46-50 (W_po = P W_out, encoder.py:99-101)
//   message = content[j, :C] + content[i, C:] + contrib, two-pass LN over C
//     (eps 1e-6), affine, LeakyReLU 0.2, max over k
//                                          neighbor_reduce_forward.cu:13-33
//
// CTA = 256 threads handles ppc = max(1, 64 / K) points (<= 64 edges).
// Phase 1: warp per edge computes the H hidden values into shared memory.
// Phase 2: warp w owns 8 edges, lane owns channels lane + 32 t; W_po streams
// through shared memory 32 hidden rows at a time; the message LN is a warp
// reduction; the max over k goes through a shared-memory atomic max.
#include <cfloat>

#include "kernels.cuh"

namespace f2s {
namespace {

constexpr int kEdgesPerCta = 64;
constexpr int kHChunk = 32;
constexpr int kMaxD = 8;

// Atomic max of floats in shared memory (sign-split integer ordering).
__device__ __forceinline__ void smem_atomic_max(float* addr, float v) {
    v = v + 0.0f;  // fold -0 onto +0
    if (v >= 0.0f)
        atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
    else
        atomicMin(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

template <int CT>  // channel chunks of 32 per lane: cout <= 32 * CT
__global__ void __launch_bounds__(256) edge_kernel(const EdgeArgs a, int ppc) {
    extern __shared__ __align__(16) float sm[];
    const int H = a.H, cout = a.cout, K = a.K;
    const int E = ppc * K;
    float* hid = sm;                                   // [64][H]
    float* wch = hid + kEdgesPerCta * H;               // [32][cout + 1]
    float* mx = wch + kHChunk * (cout + 1);            // [ppc][cout]
    int* erow = reinterpret_cast<int*>(mx + ppc * cout);  // [64] neighbour row or -1

    const int R = a.B * a.M;
    const int p0 = blockIdx.x * ppc;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    for (int i = tid; i < ppc * cout; i += 256) mx[i] = -FLT_MAX;

    // ---- phase 1: hidden activations -------------------------------------
    for (int e = warp; e < kEdgesPerCta; e += 8) {
        const int p = p0 + e / K;
        const bool valid = e < E && p < R;
        if (!valid) {
            for (int c = lane; c < H; c += 32) hid[e * H + c] = 0.0f;
            if (lane == 0) erow[e] = -1;
            continue;
        }
        const int kk = e - (e / K) * K;
        const int b = p / a.M;
        const int jrow = b * a.M + a.idx[(size_t)p * K + kk];
        float g[kMaxD];
        if (a.geometry) {
#pragma unroll
            for (int d = 0; d < kMaxD; ++d)
                g[d] = d < a.D ? a.geometry[((size_t)p * K + kk) * a.D + d] : 0.0f;
        } else {
            const float4 xi = *reinterpret_cast<const float4*>(a.xyz4 + (size_t)p * 4);
            const float4 xj = *reinterpret_cast<const float4*>(a.xyz4 + (size_t)jrow * 4);
            g[0] = xj.x - xi.x; g[1] = xj.y - xi.y; g[2] = xj.z - xi.z;
            g[3] = xi.x; g[4] = xi.y; g[5] = xi.z; g[6] = 0.0f; g[7] = 0.0f;
        }
        float s = 0.0f, s2 = 0.0f;
        for (int c = lane; c < H; c += 32) {
            float v = a.hpe_b[c];
            for (int d = 0; d < a.D; ++d) v = fmaf(g[d], a.hpe_w[c * a.D + d], v);
            hid[e * H + c] = v;
            s += v;
            s2 = fmaf(v, v, s2);
        }
        const float mean = f2s_warp_sum(s) / (float)H;
        const float var = fmaxf(f2s_warp_sum(s2) / (float)H - mean * mean, 0.0f);
        const float rstd = rsqrtf(var + 1e-5f);
        for (int c = lane; c < H; c += 32) {
            const float v = hid[e * H + c];
            hid[e * H + c] = f2s_gelu_erf((v - mean) * rstd * a.hpe_ln_w[c] + a.hpe_ln_b[c]);
        }
        if (lane == 0) erow[e] = jrow;
    }

    // ---- phase 2: composed projection + message + max ---------------------
    float acc[8][CT];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int t = 0; t < CT; ++t) acc[i][t] = 0.0f;
    const int e0 = warp * 8;
    for (int h0 = 0; h0 < H; h0 += kHChunk) {
        __syncthreads();
        for (int i = tid; i < kHChunk * cout; i += 256) {
            const int c = i / kHChunk, hh = i - c * kHChunk;
            wch[hh * (cout + 1) + c] = (h0 + hh < H) ? a.contrib_w[(size_t)c * H + h0 + hh] : 0.0f;
        }
        __syncthreads();
        const int hn = min(kHChunk, H - h0);
        for (int hh = 0; hh < hn; ++hh) {
            float w[CT];
#pragma unroll
            for (int t = 0; t < CT; ++t) {
                const int c = lane + 32 * t;
                w[t] = c < cout ? wch[hh * (cout + 1) + c] : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float hv = hid[(e0 + i) * H + h0 + hh];
#pragma unroll
                for (int t = 0; t < CT; ++t) acc[i][t] = fmaf(hv, w[t], acc[i][t]);
            }
        }
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = e0 + i;
        const int jrow = erow[e];
        if (jrow < 0) continue;  // warp-uniform
        const int pl = e / K;
        const int p = p0 + pl;
        const float* cj = a.content + (size_t)jrow * a.ldc;
        const float* ci = a.content + (size_t)p * a.ldc + cout;
        float v[CT];
        float s = 0.0f;
#pragma unroll
        for (int t = 0; t < CT; ++t) {
            const int c = lane + 32 * t;
            v[t] = c < cout ? cj[c] + ci[c] + (acc[i][t] + a.contrib_b[c]) : 0.0f;
            s += v[t];
        }
        const float mean = f2s_warp_sum(s) / (float)cout;
        float q = 0.0f;
#pragma unroll
        for (int t = 0; t < CT; ++t) {
            const int c = lane + 32 * t;
            const float dlt = c < cout ? v[t] - mean : 0.0f;
            q = fmaf(dlt, dlt, q);
        }
        const float rstd = rsqrtf(f2s_warp_sum(q) / (float)cout + 1e-6f);
#pragma unroll
        for (int t = 0; t < CT; ++t) {
            const int c = lane + 32 * t;
            if (c < cout)
                smem_atomic_max(&mx[pl * cout + c],
                                f2s_leaky((v[t] - mean) * rstd * a.ln_w[c] + a.ln_b[c]));
        }
    }
    __syncthreads();
    for (int i = tid; i < ppc * cout; i += 256) {
        const int pl = i / cout, c = i - pl * cout;
        const int p = p0 + pl;
        if (p < R) a.out[(size_t)p * a.ldo + c] = mx[i];
    }
}

template <int CT>
int launch_edge(const EdgeArgs& a, cudaStream_t stream) {
    const int ppc = a.K >= kEdgesPerCta ? 1 : kEdgesPerCta / a.K;
    const size_t smem = sizeof(float) * ((size_t)kEdgesPerCta * a.H +
                                         (size_t)kHChunk * (a.cout + 1) + (size_t)ppc * a.cout) +
                        sizeof(int) * kEdgesPerCta;
    auto kernel = edge_kernel<CT>;
    F2S_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
    const int R = a.B * a.M;
    TraceScope trace(kTagEdge, stream);
    kernel<<<ceil_div(R, ppc), 256, smem, stream>>>(a, ppc);
    return check_launch("edge_kernel");
}

}  // namespace

int edge_stage_f32(const EdgeArgs& a, cudaStream_t stream) {
    if (a.B == 0 || a.M == 0) return F2S_OK;
    F2S_LIMIT(a.K >= 1 && a.K <= kEdgesPerCta, "edge stage: K=%d outside [1, %d]", a.K,
              kEdgesPerCta);
    F2S_LIMIT(a.H >= 1 && a.H <= 256, "edge stage: hidden width %d outside [1, 256]", a.H);
    F2S_LIMIT(a.cout >= 1 && a.cout <= 256, "edge stage: width %d outside [1, 256]", a.cout);
    F2S_LIMIT(a.D >= 1 && a.D <= kMaxD, "edge stage: geometry width %d outside [1, %d]", a.D,
              kMaxD);
    F2S_REQUIRE(a.xyz4 != nullptr || a.geometry != nullptr, "edge stage: no geometry source");
    const int ct = ceil_div(a.cout, 32);
    if (ct <= 2) return launch_edge<2>(a, stream);
    if (ct <= 4) return launch_edge<4>(a, stream);
    if (ct <= 6) return launch_edge<6>(a, stream);
    return launch_edge<8>(a, stream);
}

}  // namespace f2s
