// Flow2SurfNet forward (flow2surf/models/network.py:75-82) as a sequence of
// sm_100a kernels over point-major activations, plus the parameter-blob and
// workspace layouts and the operator entry points that share its kernels.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cfloat>
#include <vector>

#include "kernels.cuh"

namespace f2s {

int transpose_batched(const float* in, float* out, int B, int rows, int cols,
                      cudaStream_t stream);

namespace {

constexpr int kMaxStages = F2S_MAX_STAGES;
constexpr int kMaxBlocks = F2S_MAX_BLOCKS;
constexpr int kMaxDecoder = F2S_MAX_DECODER;

// ---------------------------------------------------------------------------
// Parameter blob: float32 segments, each 16-byte aligned, in a fixed order.
// ---------------------------------------------------------------------------
struct StageParams {
    int64_t content_w, hpe_w, hpe_b, hpe_ln_w, hpe_ln_b, contrib_w, contrib_b, ln_w, ln_b;
};
struct BlockParams {
    int64_t mod_w, mod_b, qkv_w, proj_w, gate_w, gate_b, ff1_w, ff1_b, ff2_w, ff2_b;
};
struct DecParams {
    int64_t w, ln_w, ln_b;
};

struct Layout {
    int64_t alpha_w1, alpha_b1, alpha_w2, alpha_b2;
    int64_t in_w, in_b, in_ln_w, in_ln_b, in_out_w, in_out_b;
    StageParams stage[kMaxStages];
    int64_t proj_w, proj_ln_w, proj_ln_b;
    BlockParams block[kMaxBlocks];
    DecParams dec[kMaxDecoder];
    int64_t dec_out_w;
    std::vector<int64_t> offsets, sizes;
    int64_t total = 0;

    int64_t add(int64_t n) {
        const int64_t off = total;
        offsets.push_back(off);
        sizes.push_back(n);
        total += (n + 3) & ~int64_t(3);
        return off;
    }
};

struct Dims {
    int K, C, NB, A, Hf, qk, S, ndec;
    int sd[kMaxStages], si[kMaxStages], dd[kMaxDecoder];
    int sum_stage, max_cout, max_dec;
    int max_gemm_in;    // widest K of the encoder GEMMs (content, projection head)
    int max_gemm_w;     // largest weight matrix of the encoder GEMMs
    int precision;      // trunk + decoder
    int enc_precision;  // neighbour stages + projection head
    int enc_gemm_precision;
};

// tf32 tensor cores for the trunk (with fp16 or fp32 FFN rows)
bool trunk_on_tensor_cores(int precision) {
    return precision == F2S_PRECISION_TF32 || precision == F2S_PRECISION_TF32_WIDE;
}

int check_config(const f2s_model_config* cfg, Dims& d) {
    F2S_REQUIRE(cfg != nullptr, "model config is null");
    d.K = cfg->k_neighbors;
    d.C = cfg->feat_dim;
    d.NB = cfg->num_blocks;
    d.A = cfg->alpha_dim;
    F2S_REQUIRE(d.K >= 1, "k_neighbors must be >= 1, got %d", d.K);
    F2S_LIMIT(d.K <= F2S_KNN_MAX_K, "k_neighbors %d exceeds %d", d.K, F2S_KNN_MAX_K);
    F2S_REQUIRE(d.NB >= 0, "num_blocks must be >= 0, got %d", d.NB);
    F2S_LIMIT(d.NB <= kMaxBlocks, "num_blocks %d exceeds %d", d.NB, kMaxBlocks);
    F2S_REQUIRE(cfg->ffn_ratio >= 1, "ffn_ratio must be >= 1, got %d", cfg->ffn_ratio);
    F2S_REQUIRE(d.A >= 1, "alpha_dim must be >= 1, got %d", d.A);
    F2S_REQUIRE(d.C >= 4, "channels must be >= 4, got %d", d.C);
    F2S_LIMIT(d.C <= 256, "feat_dim %d exceeds 256", d.C);
    F2S_LIMIT(d.A <= 256, "alpha_dim %d exceeds 256", d.A);
    d.qk = d.C / 4;
    d.Hf = d.C * cfg->ffn_ratio;
    d.S = cfg->num_stages;
    F2S_REQUIRE(d.S >= 1 && d.S <= kMaxStages, "num_stages %d outside [1, %d]", d.S, kMaxStages);
    F2S_REQUIRE(cfg->stage_dims[d.S - 1] == d.C, "last stage width must equal feat_dim");
    d.sum_stage = 0;
    d.max_cout = 0;
    for (int s = 0; s < d.S; ++s) {
        d.sd[s] = cfg->stage_dims[s];
        d.si[s] = s == 0 ? cfg->stage_dims[0] : cfg->stage_dims[s - 1];
        F2S_REQUIRE(d.sd[s] >= 1, "stage width must be >= 1");
        F2S_LIMIT(d.sd[s] <= 256, "stage width %d exceeds 256", d.sd[s]);
        d.sum_stage += d.sd[s];
        d.max_cout = d.sd[s] > d.max_cout ? d.sd[s] : d.max_cout;
    }
    d.precision = cfg->precision;
    d.enc_precision = cfg->encoder_precision;
    F2S_REQUIRE(d.precision == F2S_PRECISION_FP32 || d.precision == F2S_PRECISION_TF32 ||
                    d.precision == F2S_PRECISION_TF32_WIDE,
                "trunk precision %d is not F2S_PRECISION_FP32, _TF32 or _TF32_WIDE", d.precision);
    F2S_REQUIRE(d.enc_precision == F2S_PRECISION_FP32 || d.enc_precision == F2S_PRECISION_TF32 ||
                    d.enc_precision == F2S_PRECISION_BF16X3,
                "encoder precision %d is not F2S_PRECISION_FP32, _TF32 or _BF16X3",
                d.enc_precision);
    // the encoder's plain GEMMs (content, projection head): tf32 with a tf32
    // encoder, 3xTF32 (denoted F2S_PRECISION_BF16X3 here) with a split-bf16
    // one, fp32 CUDA cores with an fp32 one
    d.enc_gemm_precision = d.enc_precision;
    d.max_gemm_in = d.sum_stage;
    d.max_gemm_w = d.C * d.sum_stage;
    for (int s = 0; s < d.S; ++s) {
        d.max_gemm_in = d.si[s] > d.max_gemm_in ? d.si[s] : d.max_gemm_in;
        const int wsize = 2 * d.sd[s] * d.si[s];
        d.max_gemm_w = wsize > d.max_gemm_w ? wsize : d.max_gemm_w;
    }
    d.ndec = cfg->num_decoder;
    F2S_REQUIRE(d.ndec >= 0 && d.ndec <= kMaxDecoder, "num_decoder %d outside [0, %d]", d.ndec,
                kMaxDecoder);
    d.max_dec = 0;
    for (int i = 0; i < d.ndec; ++i) {
        d.dd[i] = cfg->decoder_dims[i];
        F2S_REQUIRE(d.dd[i] >= 1, "decoder width must be >= 1");
        d.max_dec = d.dd[i] > d.max_dec ? d.dd[i] : d.max_dec;
    }
    return F2S_OK;
}

Layout make_layout(const Dims& d) {
    Layout L;
    const int A4 = 4 * d.A, S0 = d.sd[0];
    L.alpha_w1 = L.add(A4);
    L.alpha_b1 = L.add(A4);
    L.alpha_w2 = L.add((int64_t)d.A * A4);
    L.alpha_b2 = L.add(d.A);
    L.in_w = L.add((int64_t)S0 * 3);
    L.in_b = L.add(S0);
    L.in_ln_w = L.add(S0);
    L.in_ln_b = L.add(S0);
    L.in_out_w = L.add((int64_t)S0 * S0);
    L.in_out_b = L.add(S0);
    for (int s = 0; s < d.S; ++s) {
        const int cin = d.si[s], cout = d.sd[s], H = cin;
        StageParams& p = L.stage[s];
        p.content_w = L.add((int64_t)2 * cout * cin);
        p.hpe_w = L.add((int64_t)H * 6);
        p.hpe_b = L.add(H);
        p.hpe_ln_w = L.add(H);
        p.hpe_ln_b = L.add(H);
        p.contrib_w = L.add((int64_t)cout * H);
        p.contrib_b = L.add(cout);
        p.ln_w = L.add(cout);
        p.ln_b = L.add(cout);
    }
    L.proj_w = L.add((int64_t)d.C * d.sum_stage);
    L.proj_ln_w = L.add(d.C);
    L.proj_ln_b = L.add(d.C);
    for (int i = 0; i < d.NB; ++i) {
        BlockParams& p = L.block[i];
        p.mod_w = L.add((int64_t)6 * d.C * d.A);
        p.mod_b = L.add(6 * d.C);
        p.qkv_w = L.add((int64_t)(d.C + 2 * d.qk) * d.C);
        p.proj_w = L.add((int64_t)d.C * d.C);
        p.gate_w = L.add((int64_t)d.Hf * d.C);
        p.gate_b = L.add(d.Hf);
        p.ff1_w = L.add((int64_t)d.Hf * d.C);
        p.ff1_b = L.add(d.Hf);
        p.ff2_w = L.add((int64_t)d.C * d.Hf);
        p.ff2_b = L.add(d.C);
    }
    int in_dim = d.C;
    for (int i = 0; i < d.ndec; ++i) {
        L.dec[i].w = L.add((int64_t)d.dd[i] * in_dim);
        L.dec[i].ln_w = L.add(d.dd[i]);
        L.dec[i].ln_b = L.add(d.dd[i]);
        in_dim = d.dd[i];
    }
    L.dec_out_w = L.add((int64_t)3 * in_dim);
    return L;
}

// ---------------------------------------------------------------------------
// Workspace carve-up (all regions 256-byte aligned).
// ---------------------------------------------------------------------------
struct Workspace {
    float *xyz4, *feat0, *content, *cat, *x, *h, *qkv, *colstats, *offs, *ffh, *dec0, *dec1;
    float *cond, *mod, *attn;
    float* split_w;  // split-bf16 encoder: bf16 high and low parts of a GEMM's weights
    // tf32 trunk: the FFN input (w.h after the second modulation) and hidden
    // rows (w.ffh) are fp16, and the FFN GEMMs read fp16 copies of their
    // weights made at the start of every forward: per block gate, value
    // (Hf x C each) and ff2 (C x Hf)
    __half* ffn_w16;
    int32_t* idx;
    size_t bytes;
};

Workspace carve(const Dims& d, int B, int M, char* base) {
    Workspace w{};
    size_t off = 0;
    const size_t R = (size_t)B * M;
    auto take = [&](size_t count) -> char* {
        char* p = base ? base + off : nullptr;
        off += (count * 4 + 255) & ~size_t(255);
        return p;
    };
    w.xyz4 = (float*)take(R * 4);
    w.feat0 = (float*)take(R * d.sd[0]);
    w.idx = (int32_t*)take(R * d.K);
    w.content = (float*)take(R * 2 * d.max_cout);
    w.cat = (float*)take(R * d.sum_stage);
    w.x = (float*)take(R * d.C);
    w.h = (float*)take(R * d.C);
    w.qkv = (float*)take(R * (d.C + 2 * d.qk));
    w.colstats = (float*)take(R);
    w.offs = (float*)take(R * d.C);
    w.ffh = (float*)take(R * d.Hf);
    w.dec0 = (float*)take(R * (d.max_dec > 0 ? d.max_dec : 1));
    w.dec1 = (float*)take(R * (d.max_dec > 0 ? d.max_dec : 1));
    w.cond = (float*)take((size_t)B * d.A);
    w.mod = (float*)take((size_t)B * (d.NB > 0 ? d.NB : 1) * 6 * d.C);
    w.attn = (float*)take((size_t)attention_tc_workspace_floats(B, M, d.C));
    const bool split = d.enc_gemm_precision == F2S_PRECISION_BF16X3;
    w.split_w = split ? (float*)take((size_t)d.max_gemm_w) : nullptr;  // 2 x bf16 per weight
    const bool tf32_trunk = trunk_on_tensor_cores(d.precision);
    w.ffn_w16 = tf32_trunk ? (__half*)take(((size_t)(d.NB > 0 ? d.NB : 1) * 3 * d.C * d.Hf + 1) / 2)
                           : nullptr;
    w.bytes = off;
    return w;
}

// ---------------------------------------------------------------------------
// Small kernels: conditioning and the input embedding.
// ---------------------------------------------------------------------------
struct CondArgs {
    const float* P;
    int64_t w1, b1, w2, b2;
    int64_t mod_w[kMaxBlocks], mod_b[kMaxBlocks];
    int A, NB, C;
};

// AlphaEmbed (network.py:10-26) and every block's AdaLN modulation
// Linear(SiLU(cond)) (transformer.py:51-54,77-83); one CTA per patch.
__global__ void cond_mod_kernel(const CondArgs a, const float* __restrict__ alpha,
                                float* __restrict__ cond, float* __restrict__ mod) {
    extern __shared__ float sm[];
    const int A = a.A, A4 = 4 * a.A;
    float* t = sm;            // [A4]
    float* sc = sm + A4;      // [A]
    const int b = blockIdx.x;
    const float e = 2.0f * alpha[b] - 1.0f;
    for (int j = threadIdx.x; j < A4; j += blockDim.x)
        t[j] = f2s_silu(fmaf(a.P[a.w1 + j], e, a.P[a.b1 + j]));
    __syncthreads();
    for (int i = threadIdx.x; i < A; i += blockDim.x) {
        float v = a.P[a.b2 + i];
        for (int j = 0; j < A4; ++j) v = fmaf(a.P[a.w2 + (int64_t)i * A4 + j], t[j], v);
        cond[(size_t)b * A + i] = v;
        sc[i] = f2s_silu(v);
    }
    __syncthreads();
    const int n6 = 6 * a.C;
    for (int blk = 0; blk < a.NB; ++blk) {
        for (int n = threadIdx.x; n < n6; n += blockDim.x) {
            float v = a.P[a.mod_b[blk] + n];
            const float* w = a.P + a.mod_w[blk] + (int64_t)n * A;
            for (int j = 0; j < A; ++j) v = fmaf(w[j], sc[j], v);
            mod[((size_t)b * a.NB + blk) * n6 + n] = v;
        }
    }
}

// xyz (B, 3, M) -> point-major xyz4, and the input HPE (encoder.py:40-71,177):
// Linear(3 -> S0), Jittor LayerNorm (var = max(E[x^2]-E[x]^2, 0), eps 1e-5),
// erf GELU, Linear(S0 -> S0). One warp per point; persistent CTAs load the
// output weights into shared memory once and loop over groups of 8 points.
__global__ void input_embed_kernel(const float* __restrict__ x, int B, int M,
                                   const float* __restrict__ w, const float* __restrict__ bia,
                                   const float* __restrict__ lnw, const float* __restrict__ lnb,
                                   const float* __restrict__ ow, const float* __restrict__ ob,
                                   int S0, float* __restrict__ xyz4, float* __restrict__ feat) {
    extern __shared__ float sm[];
    float* owT = sm;                         // [S0][S0] transposed (h-major)
    float* hid = sm + (size_t)S0 * S0;       // [8][S0]
    for (int i = threadIdx.x; i < S0 * S0; i += blockDim.x) {
        const int c = i / S0, hh = i - c * S0;
        owT[hh * S0 + c] = ow[i];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = B * M;
    for (int p = blockIdx.x * 8 + warp; p < R; p += gridDim.x * 8) {
    const int b = p / M, m = p - b * M;
    const float* xb = x + (size_t)b * 3 * M;
    const float x0 = xb[m], x1 = xb[M + m], x2 = xb[2 * M + m];
    if (lane == 0) *reinterpret_cast<float4*>(xyz4 + (size_t)p * 4) = make_float4(x0, x1, x2, 0.0f);
    float* hw = hid + warp * S0;
    float s = 0.0f, s2 = 0.0f;
    for (int c = lane; c < S0; c += 32) {
        float v = bia[c];
        v = fmaf(w[c * 3 + 0], x0, v);
        v = fmaf(w[c * 3 + 1], x1, v);
        v = fmaf(w[c * 3 + 2], x2, v);
        hw[c] = v;
        s += v;
        s2 = fmaf(v, v, s2);
    }
    const float mean = f2s_warp_sum(s) / (float)S0;
    const float var = fmaxf(f2s_warp_sum(s2) / (float)S0 - mean * mean, 0.0f);
    const float rstd = rsqrtf(var + 1e-5f);
    for (int c = lane; c < S0; c += 32)
        hw[c] = f2s_gelu_erf((hw[c] - mean) * rstd * lnw[c] + lnb[c]);
    __syncwarp();
    float* fr = feat + (size_t)p * S0;
    for (int c = lane; c < S0; c += 32) {
        float v = ob[c];
        for (int hh = 0; hh < S0; ++hh) v = fmaf(owT[hh * S0 + c], hw[hh], v);
        fr[c] = v;
    }
    __syncwarp();  // hw is rewritten for the next point
    }
}

// The same input embedding with one point per lane: the S0 hidden values of
// the lane's point stay in registers and every weight is a warp-wide
// broadcast read from shared memory (a float4 per four multiply-adds), so
// the S0 x S0 output projection runs at the FMA rate. S0 <= S, channels past
// S0 predicated off. Per output channel the projection accumulates in the
// same order as input_embed_kernel (ob[c] + sum over hh = 0, 1, ...).
template <int S>
__global__ void __launch_bounds__(256, 1)
input_embed_lane_kernel(const float* __restrict__ x, int B, int M, const float* __restrict__ w,
                        const float* __restrict__ bia, const float* __restrict__ lnw,
                        const float* __restrict__ lnb, const float* __restrict__ ow,
                        const float* __restrict__ ob, int S0, float* __restrict__ xyz4,
                        float* __restrict__ feat, float* __restrict__ feat_lo) {
    extern __shared__ __align__(16) float sm[];
    float* sOw = sm;                    // [S][S]: row c = output channel, zero-padded
    float* sW = sOw + S * S;            // [S][4]: w0, w1, w2, bias
    float* sLn = sW + 4 * S;            // [S][2]: gain, shift
    float* sOb = sLn + 2 * S;           // [S]
    for (int i = threadIdx.x; i < S * S; i += blockDim.x) {
        const int c = i / S, hh = i - c * S;
        sOw[i] = (c < S0 && hh < S0) ? ow[c * S0 + hh] : 0.0f;
    }
    for (int c = threadIdx.x; c < S; c += blockDim.x) {
        const bool on = c < S0;
        sW[4 * c + 0] = on ? w[c * 3 + 0] : 0.0f;
        sW[4 * c + 1] = on ? w[c * 3 + 1] : 0.0f;
        sW[4 * c + 2] = on ? w[c * 3 + 2] : 0.0f;
        sW[4 * c + 3] = on ? bia[c] : 0.0f;
        sLn[2 * c] = on ? lnw[c] : 0.0f;
        sLn[2 * c + 1] = on ? lnb[c] : 0.0f;
        sOb[c] = on ? ob[c] : 0.0f;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = B * M;
    for (int p0 = (blockIdx.x * 8 + warp) * 32; p0 < R; p0 += gridDim.x * 8 * 32) {
        const int p = p0 + lane;
        const bool ok = p < R;
        float x0 = 0.0f, x1 = 0.0f, x2 = 0.0f;
        if (ok) {
            const int b = p / M, m = p - b * M;
            const float* xb = x + (size_t)b * 3 * M;
            x0 = xb[m];
            x1 = xb[M + m];
            x2 = xb[2 * M + m];
            *reinterpret_cast<float4*>(xyz4 + (size_t)p * 4) = make_float4(x0, x1, x2, 0.0f);
        }
        float h[S];
        float s = 0.0f, s2 = 0.0f;
#pragma unroll
        for (int c = 0; c < S; ++c) {
            const float4 wc = *reinterpret_cast<const float4*>(sW + 4 * c);
            float v = wc.w;
            v = fmaf(wc.x, x0, v);
            v = fmaf(wc.y, x1, v);
            v = fmaf(wc.z, x2, v);
            h[c] = v;
            if (c < S0) {
                s += v;
                s2 = fmaf(v, v, s2);
            }
        }
        const float mean = s / (float)S0;
        const float var = fmaxf(s2 / (float)S0 - mean * mean, 0.0f);
        const float rstd = rsqrtf(var + 1e-5f);
#pragma unroll
        for (int c = 0; c < S; ++c) {
            const float2 g = *reinterpret_cast<const float2*>(sLn + 2 * c);
            h[c] = f2s_gelu_erf((h[c] - mean) * rstd * g.x + g.y);  // padded channels: gain 0
        }
        if (!ok) continue;
        float* fr = feat + (size_t)p * S0;
        float* fl = feat_lo ? feat_lo + (size_t)p * S0 : nullptr;
        for (int c = 0; c < S0; c += 4) {
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float* wr = sOw + (c + e) * S;
                float v = sOb[c + e];
#pragma unroll
                for (int hh = 0; hh < S; hh += 4) {
                    const float4 q = *reinterpret_cast<const float4*>(wr + hh);
                    v = fmaf(q.x, h[hh], v);
                    v = fmaf(q.y, h[hh + 1], v);
                    v = fmaf(q.z, h[hh + 2], v);
                    v = fmaf(q.w, h[hh + 3], v);
                }
                o[e] = v;
            }
            float lo[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (fl) {
                // tf32 high part here, the remainder in feat_lo (the operand
                // split of the 3xTF32 GEMM that reads the features)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float hi = f2s_round_tf32(o[e]);
                    lo[e] = o[e] - hi;
                    o[e] = hi;
                }
            }
            if (c + 4 <= S0 && (S0 & 3) == 0) {
                *reinterpret_cast<float4*>(fr + c) = make_float4(o[0], o[1], o[2], o[3]);
                if (fl) *reinterpret_cast<float4*>(fl + c) = make_float4(lo[0], lo[1], lo[2], lo[3]);
            } else {
                for (int e = 0; e < 4 && c + e < S0; ++e) {
                    fr[c + e] = o[e];
                    if (fl) fl[c + e] = lo[e];
                }
            }
        }
    }
}

// fp16 copy (round to nearest) of n floats.
__global__ void to_half_kernel(const float* __restrict__ src, __half* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}

GemmArgs gemm_args(const float* A, int lda, const float* W, const float* bias, float* Y, int ldy,
                   int rows, int cols, int K) {
    GemmArgs g{};
    g.A = A;
    g.lda = lda;
    g.W = W;
    g.bias = bias;
    g.Y = Y;
    g.ldy = ldy;
    g.rows = rows;
    g.cols = cols;
    g.K = K;
    g.rows_per_patch = 1;
    g.epilogue = kEpiStore;
    g.tag = kTagGemmContent;
    return g;
}

// One dense contraction of the forward at the configured precision: the fp32
// CUDA-core kernel, the tcgen05 kernel reading the fp32 operands as tf32, or
// (F2S_PRECISION_BF16X3 here) the split-bf16 tcgen05 kernel, which splits the
// fp32 A rows into bf16 high and low parts in shared memory; the weights'
// parts are made here into split_w (2 x cols x K bf16).
int linear_op(const GemmArgs& g, int precision, cudaStream_t st, void* split_w = nullptr) {
    if (precision == F2S_PRECISION_FP32) return gemm_f32(g, st);
    if (precision == F2S_PRECISION_BF16X3) {
        // fp32 A rows and bf16 weight rows by TMA: 16-byte pitches and base
        if (g.K % 8 != 0 || g.lda % 4 != 0 || ((uintptr_t)g.A & 15) != 0 ||
            g.epilogue != kEpiStore || !split_w)
            return gemm_f32(g, st);
        __nv_bfloat16* w_hi = static_cast<__nv_bfloat16*>(split_w);
        __nv_bfloat16* w_lo = w_hi + (size_t)g.cols * g.K;
        {
            TraceScope trace(g.tag, st);
            F2S_TRY(split_bf16(g.W, g.K, g.cols, g.K, w_hi, w_lo, st));
        }
        TcGemmOp op{};
        op.A = g.A;
        op.lda = g.lda;
        op.W = w_hi;
        op.W_lo = w_lo;
        op.split_in = true;
        op.bias = g.bias;
        op.Y = g.Y;
        op.ldy = g.ldy;
        op.rows_per_patch = 1;
        op.rows = g.rows;
        op.cols = g.cols;
        op.K = g.K;
        // N tiles up to 192: two stages of fp32 A (32 KB) and the W parts fit
        op.bn = tc_pick_bn(g.cols, false);
        if (op.bn > 192) op.bn = tc_pick_bn(g.cols, true);
        op.tf32 = false;
        op.epilogue = kEpiStore;
        op.tag = g.tag;
        return tc_gemm(op, st);
    }
    TcGemmOp op{};
    op.A = g.A;
    op.lda = g.lda;
    op.W = g.W;
    op.W2 = g.W2;
    op.bias = g.bias;
    op.bias2 = g.bias2;
    op.Y = g.Y;
    op.ldy = g.ldy;
    op.gate = g.gate;
    op.gate_stride = g.gate_stride;
    op.rows_per_patch = g.rows_per_patch;
    op.rows = g.rows;
    op.cols = g.cols;
    op.K = g.K;
    op.bn = tc_pick_bn(g.cols, g.epilogue == kEpiSwiGlu);
    op.tf32 = !g.fp16_operands;
    op.fp16 = g.fp16_operands;
    if (g.fp16_operands) {
        op.W = g.W16;
        op.W2 = g.W2_16;
    }
    op.y_fp16 = g.y_fp16;
    op.vt = g.vt;
    op.vt_col0 = g.vt_col0;
    op.vt_C = g.vt_C;
    op.vt_npad = g.vt_npad;
    op.vt_M = g.vt_M;
    op.qk_hi = g.qk_hi;
    op.qk_lo = g.qk_lo;
    op.round_tf32 = g.round_tf32;
    op.epilogue = g.epilogue;
    op.tag = g.tag;
    return tc_gemm(op, st);
}

// AlphaEmbed (network.py:10-26, :75-76) and every block's AdaLN modulation
// (transformer.py:48-54) into w.cond, w.mod.
int condition(const Dims& d, const Layout& L, const float* P, const float* alpha, int B,
              const Workspace& w, cudaStream_t st) {
    const int C = d.C;
    {
        CondArgs ca{};
        ca.P = P;
        ca.w1 = L.alpha_w1;
        ca.b1 = L.alpha_b1;
        ca.w2 = L.alpha_w2;
        ca.b2 = L.alpha_b2;
        for (int i = 0; i < d.NB; ++i) {
            ca.mod_w[i] = L.block[i].mod_w;
            ca.mod_b[i] = L.block[i].mod_b;
        }
        ca.A = d.A;
        ca.NB = d.NB;
        ca.C = C;
        TraceScope trace(kTagCondition, st);
        cond_mod_kernel<<<B, 256, sizeof(float) * 5 * d.A, st>>>(ca, alpha, w.cond, w.mod);
        F2S_TRY(check_launch("cond_mod_kernel"));
    }
    return F2S_OK;
}

int trunk(const Dims& d, const Layout& L, const float* P, int B, int M, float* x,
          const Workspace& w, cudaStream_t st);

int forward(const Dims& d, const Layout& L, const float* P, const float* x_in, const float* alpha,
            int B, int M, float* velocity, const Workspace& w, cudaStream_t st) {
    const int R = B * M;
    const int C = d.C;
    F2S_TRY(condition(d, L, P, alpha, B, w, st));
    // input embedding + xyz
    if (d.sd[0] <= 64) {
        const int S0 = d.sd[0];
        TraceScope trace(kTagInputEmbed, st);
        const int warps = ceil_div(R, 32);
        const int blocks = ceil_div(warps, 8);
        const int grid = blocks < 4 * sm_count() ? blocks : 4 * sm_count();
        auto launch = [&](auto kernel, int S) -> int {
            const size_t smem = sizeof(float) * ((size_t)S * S + 7 * (size_t)S);
            F2S_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)smem));
            kernel<<<grid, 256, smem, st>>>(x_in, B, M, P + L.in_w, P + L.in_b, P + L.in_ln_w,
                                            P + L.in_ln_b, P + L.in_out_w, P + L.in_out_b, S0,
                                            w.xyz4, w.feat0, nullptr);
            return check_launch("input_embed_lane_kernel");
        };
        if (S0 <= 16) F2S_TRY(launch(input_embed_lane_kernel<16>, 16));
        else if (S0 <= 32) F2S_TRY(launch(input_embed_lane_kernel<32>, 32));
        else F2S_TRY(launch(input_embed_lane_kernel<64>, 64));
    } else {
        const int S0 = d.sd[0];
        const size_t smem = sizeof(float) * ((size_t)S0 * S0 + 8 * S0);
        F2S_CUDA_TRY(cudaFuncSetAttribute(input_embed_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        TraceScope trace(kTagInputEmbed, st);
        const int groups = ceil_div(R, 8);
        const int grid = groups < 4 * sm_count() ? groups : 4 * sm_count();
        input_embed_kernel<<<grid, 256, smem, st>>>(
            x_in, B, M, P + L.in_w, P + L.in_b, P + L.in_ln_w, P + L.in_ln_b, P + L.in_out_w,
            P + L.in_out_b, S0, w.xyz4, w.feat0);
        F2S_TRY(check_launch("input_embed_kernel"));
    }
    F2S_TRY(knn_launch(x_in, B, 3, M, d.K, w.idx, st));
    // neighbour stages (the split encoder's GEMMs split their fp32 inputs
    // into bf16 parts in shared memory)
    int col = 0;
    const float* fin = w.feat0;
    int ldin = d.sd[0];
    for (int s = 0; s < d.S; ++s) {
        const StageParams& sp = L.stage[s];
        const int cin = d.si[s], cout = d.sd[s];
        GemmArgs gc = gemm_args(fin, ldin, P + sp.content_w, nullptr, w.content, 2 * cout, R,
                                2 * cout, cin);  // tag: gemm_content
        F2S_TRY(linear_op(gc, d.enc_gemm_precision, st, w.split_w));
        EdgeArgs ea{};
        ea.content = w.content;
        ea.ldc = 2 * cout;
        ea.xyz4 = w.xyz4;
        ea.D = 6;
        ea.idx = w.idx;
        ea.B = B;
        ea.M = M;
        ea.K = d.K;
        ea.H = cin;
        ea.cout = cout;
        ea.hpe_w = P + sp.hpe_w;
        ea.hpe_b = P + sp.hpe_b;
        ea.hpe_ln_w = P + sp.hpe_ln_w;
        ea.hpe_ln_b = P + sp.hpe_ln_b;
        ea.contrib_w = P + sp.contrib_w;
        ea.contrib_b = P + sp.contrib_b;
        ea.ln_w = P + sp.ln_w;
        ea.ln_b = P + sp.ln_b;
        ea.out = w.cat + col;
        ea.ldo = d.sum_stage;
        int edge_status = F2S_ERR_UNSUPPORTED;
        if (d.enc_precision != F2S_PRECISION_FP32)
            edge_status = edge_stage_tc(ea, d.enc_precision, st);
        // shapes the tensor-core kernel does not take run on the CUDA-core kernel
        if (edge_status == F2S_ERR_UNSUPPORTED) edge_status = edge_stage_f32(ea, st);
        F2S_TRY(edge_status);
        fin = w.cat + col;
        ldin = d.sum_stage;
        col += cout;
    }
    // projection head (encoder.py:118-123,184)
    {
        GemmArgs g = gemm_args(w.cat, d.sum_stage, P + L.proj_w, nullptr, w.x, C, R, C,
                               d.sum_stage);
        g.tag = kTagGemmHead;
        F2S_TRY(linear_op(g, d.enc_gemm_precision, st, w.split_w));
    }
    F2S_TRY(ln_affine_leaky(w.x, C, P + L.proj_ln_w, P + L.proj_ln_b, R, C, false, st));
    F2S_TRY(trunk(d, L, P, B, M, w.x, w, st));
    // decoder (decoder.py:8-32)
    const bool tf32_trunk = trunk_on_tensor_cores(d.precision);
    const float* cur = w.x;
    int in_dim = C;
    float* bufs[2] = {w.dec0, w.dec1};
    for (int i = 0; i < d.ndec; ++i) {
        float* out = bufs[i & 1];
        GemmArgs gd = gemm_args(cur, in_dim, P + L.dec[i].w, nullptr, out, d.dd[i], R, d.dd[i],
                                in_dim);
        gd.tag = kTagGemmDecoder;
        F2S_TRY(linear_op(gd, d.precision, st));
        F2S_TRY(ln_affine_leaky(out, d.dd[i], P + L.dec[i].ln_w, P + L.dec[i].ln_b, R, d.dd[i],
                                tf32_trunk, st));
        cur = out;
        in_dim = d.dd[i];
    }
    GemmArgs go = gemm_args(cur, in_dim, P + L.dec_out_w, nullptr, velocity, 3, R, 3, in_dim);
    go.tag = kTagGemmDecoder;
    return linear_op(go, d.precision, st);
}

// The AdaLN-Zero blocks (transformer.py:75-89) on the point-major residual
// stream x (B*M rows of C), in place; w.mod holds the blocks' modulation.
int trunk(const Dims& d, const Layout& L, const float* P, int B, int M, float* x,
          const Workspace& w, cudaStream_t st) {
    const int R = B * M;
    const int C = d.C;
    const int ld_qkv = C + 2 * d.qk;
    // operands of tf32 contractions are rounded to the nearest tf32 where made
    const bool tf32_trunk = trunk_on_tensor_cores(d.precision);
    const int mstride = d.NB * 6 * C;
    // fp16 FFN operands (tf32 trunk; 16-byte fp16 rows, the register LN path)
    const bool ffn_fp16 = d.precision == F2S_PRECISION_TF32 && d.Hf % 8 == 0 && C % 8 == 0 &&
                          C <= 256 &&
                          w.ffn_w16 != nullptr;
    const int64_t ffn_n = (int64_t)C * d.Hf;  // elements of one FFN weight matrix
    if (ffn_fp16) {
        TraceScope trace(kTagGemmSwiGlu, st);
        for (int i = 0; i < d.NB; ++i) {
            const int64_t srcs[3] = {L.block[i].gate_w, L.block[i].ff1_w, L.block[i].ff2_w};
            for (int m = 0; m < 3; ++m) {
                to_half_kernel<<<(unsigned)((ffn_n + 255) / 256 < 1024 ? (ffn_n + 255) / 256 : 1024),
                                 256, 0, st>>>(P + srcs[m], w.ffn_w16 + (size_t)(3 * i + m) * ffn_n,
                                               ffn_n);
                F2S_TRY(check_launch("to_half_kernel"));
            }
        }
    }
    for (int i = 0; i < d.NB; ++i) {
        const BlockParams& bp = L.block[i];
        const float* mod = w.mod + (size_t)i * 6 * C;
        F2S_TRY(ln_modulate(x, C, w.h, C, mod, mstride, 0, C, R, M, C, tf32_trunk, st));
        GemmArgs gq = gemm_args(w.h, C, P + bp.qkv_w, nullptr, w.qkv, ld_qkv, R, ld_qkv, C);
        gq.tag = kTagGemmQkv;
        // with the tensor-core attention, the GEMM writes V straight into the
        // attention's fp16 V^T (V starts at column 2 qk, a multiple of 32)
        const bool attn_tc = tf32_trunk && attention_tc_supported(w.qkv, w.qkv + d.qk, ld_qkv, d.qk, C);
        const bool vt_fused = attn_tc && (2 * d.qk) % 32 == 0 && ld_qkv % 4 == 0;
        if (vt_fused) {
            gq.vt = attention_tc_vt(w.attn, B, M);
            gq.vt_col0 = 2 * d.qk;
            gq.vt_C = C;
            gq.vt_npad = (M + 7) & ~7;
            gq.vt_M = M;
            // and, at the q / k width the fused epilogue has, the q and k
            // rows LayerNorm'd and split for the attention as well
            if (d.qk == 48) attention_tc_qk(w.attn, B, M, &gq.qk_hi, &gq.qk_lo);
        }
        F2S_TRY(linear_op(gq, d.precision, st));
        int attn_status = F2S_ERR_UNSUPPORTED;
        if (attn_tc)  // q, k LayerNorm inside the tensor-core path's prep kernel
            attn_status = attention_tc(w.qkv, w.qkv + d.qk, ld_qkv, w.qkv + 2 * d.qk, ld_qkv,
                                       w.h, C, w.offs, C, w.attn, B, M, d.qk, C, true, true, st,
                                       vt_fused, gq.qk_hi != nullptr);
        if (attn_status == F2S_ERR_UNSUPPORTED) {
            // (never with V already in V^T form: attention_tc takes every shape
            // attention_tc_supported accepts)
            if (vt_fused) return fail(F2S_ERR_INVALID_ARGUMENT, "attention: V only in V^T form");
            F2S_TRY(qk_norm(w.qkv, ld_qkv, R, d.qk, st));
            attn_status = attention_f32(w.qkv, w.qkv + d.qk, ld_qkv, w.qkv + 2 * d.qk, ld_qkv,
                                        w.h, C, w.offs, C, w.colstats, B, M, d.qk, C, tf32_trunk,
                                        st);
        }
        F2S_TRY(attn_status);
        GemmArgs g = gemm_args(w.offs, C, P + bp.proj_w, nullptr, x, C, R, C, C);
        g.epilogue = kEpiGatedResidual;
        g.gate = mod + 2 * C;
        g.gate_stride = mstride;
        g.rows_per_patch = M;
        g.tag = kTagGemmProj;
        F2S_TRY(linear_op(g, d.precision, st));
        if (ffn_fp16)
            F2S_TRY(ln_modulate_f16(x, C, w.h, C, mod, mstride, 3 * C, 4 * C, R, M, C, st));
        else
            F2S_TRY(ln_modulate(x, C, w.h, C, mod, mstride, 3 * C, 4 * C, R, M, C, tf32_trunk, st));
        GemmArgs sw = gemm_args(w.h, C, P + bp.gate_w, P + bp.gate_b, w.ffh, d.Hf, R, d.Hf, C);
        sw.epilogue = kEpiSwiGlu;
        sw.W2 = P + bp.ff1_w;
        sw.bias2 = P + bp.ff1_b;
        sw.tag = kTagGemmSwiGlu;
        sw.round_tf32 = tf32_trunk;
        // the tf32 trunk keeps the FFN input and hidden rows in fp16 (the same
        // 10-bit mantissa as the tf32 operands they replace, half the bytes
        // each way) and runs both FFN GEMMs as kind::f16 on them
        sw.y_fp16 = ffn_fp16;
        sw.fp16_operands = ffn_fp16;
        sw.W16 = ffn_fp16 ? (const void*)(w.ffn_w16 + (size_t)(3 * i) * ffn_n) : nullptr;
        sw.W2_16 = ffn_fp16 ? (const void*)(w.ffn_w16 + (size_t)(3 * i + 1) * ffn_n) : nullptr;
        F2S_TRY(linear_op(sw, d.precision, st));
        GemmArgs f2 = gemm_args(w.ffh, d.Hf, P + bp.ff2_w, P + bp.ff2_b, x, C, R, C, d.Hf);
        f2.epilogue = kEpiGatedResidual;
        f2.gate = mod + 5 * C;
        f2.gate_stride = mstride;
        f2.rows_per_patch = M;
        f2.tag = kTagGemmFf2;
        f2.fp16_operands = ffn_fp16;
        f2.W16 = ffn_fp16 ? (const void*)(w.ffn_w16 + (size_t)(3 * i + 2) * ffn_n) : nullptr;
        F2S_TRY(linear_op(f2, d.precision, st));
    }
    return F2S_OK;
}

}  // namespace
}  // namespace f2s

using namespace f2s;

extern "C" int f2s_model_param_segments(const f2s_model_config* cfg, int64_t* offsets,
                                        int64_t* sizes, int capacity, int64_t* total_floats) {
    Dims d;
    F2S_TRY(check_config(cfg, d));
    const Layout L = make_layout(d);
    const int n = (int)L.offsets.size();
    if (offsets && sizes) {
        F2S_REQUIRE(capacity >= n, "segment arrays hold %d entries, %d needed", capacity, n);
        for (int i = 0; i < n; ++i) {
            offsets[i] = L.offsets[i];
            sizes[i] = L.sizes[i];
        }
    }
    if (total_floats) *total_floats = L.total;
    return n;
}

extern "C" int f2s_model_workspace_bytes(const f2s_model_config* cfg, int B, int M,
                                         size_t* bytes) {
    Dims d;
    F2S_TRY(check_config(cfg, d));
    F2S_REQUIRE(B >= 0 && M >= 0 && bytes != nullptr, "bad workspace query");
    *bytes = carve(d, B, M, nullptr).bytes;
    return F2S_OK;
}

extern "C" int f2s_model_forward(const f2s_model_config* cfg, const float* params,
                                 const float* x, const float* alpha, int B, int M,
                                 float* velocity, void* workspace, size_t workspace_bytes,
                                 void* stream) {
    Dims d;
    F2S_TRY(check_config(cfg, d));
    F2S_REQUIRE(B >= 0 && M >= 0, "bad shape B=%d M=%d", B, M);
    if (B == 0 || M == 0) return F2S_OK;
    F2S_LIMIT(M <= F2S_KNN_MAX_POINTS, "patch of %d points exceeds %d", M, F2S_KNN_MAX_POINTS);
    F2S_LIMIT((int64_t)B * M < (1ll << 31) / 2048, "too many points in one call: B*M=%lld",
              (long long)B * M);
    F2S_REQUIRE(params && x && alpha && velocity && workspace, "model forward: null pointer");
    const Layout L = make_layout(d);
    const Workspace w = carve(d, B, M, static_cast<char*>(workspace));
    if (workspace_bytes < w.bytes)
        return fail(F2S_ERR_WORKSPACE, "model forward needs %zu workspace bytes, got %zu", w.bytes,
                    workspace_bytes);
    return forward(d, L, params, x, alpha, B, M, velocity, w, as_stream(stream));
}

extern "C" int f2s_trunk_forward(const f2s_model_config* cfg, const float* params, float* x,
                                 const float* alpha, int B, int M, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    Dims d;
    F2S_TRY(check_config(cfg, d));
    F2S_REQUIRE(B >= 0 && M >= 0, "bad shape B=%d M=%d", B, M);
    if (B == 0 || M == 0) return F2S_OK;
    F2S_LIMIT(M <= F2S_KNN_MAX_POINTS, "patch of %d points exceeds %d", M, F2S_KNN_MAX_POINTS);
    F2S_LIMIT((int64_t)B * M < (1ll << 31) / 2048, "too many points in one call: B*M=%lld",
              (long long)B * M);
    F2S_REQUIRE(params && x && alpha && workspace, "trunk forward: null pointer");
    F2S_REQUIRE(((uintptr_t)x & 15) == 0, "trunk forward: x must be 16-byte aligned");
    const Layout L = make_layout(d);
    const Workspace w = carve(d, B, M, static_cast<char*>(workspace));
    if (workspace_bytes < w.bytes)
        return fail(F2S_ERR_WORKSPACE, "trunk forward needs %zu workspace bytes, got %zu", w.bytes,
                    workspace_bytes);
    cudaStream_t st = as_stream(stream);
    F2S_TRY(condition(d, L, params, alpha, B, w, st));
    return trunk(d, L, params, B, M, x, w, st);
}

extern "C" int f2s_neighbor_reduce_workspace_bytes(int B, int N, int C, size_t* bytes) {
    F2S_REQUIRE(B >= 0 && N >= 0 && C >= 0 && bytes, "bad workspace query");
    *bytes = (size_t)B * N * 3 * C * sizeof(float);
    return F2S_OK;
}

namespace {
// The reduce_neighbor_messages operator on the fp32 CUDA-core kernel or (tc)
// the split-bf16 tensor-core kernel: content (B, 2C, N) and the output
// (B, C, N) channel-major as the reference has them, transposed point-major
// through the workspace around the kernel.
int neighbor_reduce_op(const float* content, const float* geometry, const int32_t* indices,
                       const float* hpe_input_weight, const float* hpe_input_bias,
                       const float* hpe_output_weight, const float* hpe_output_bias,
                       const float* hpe_norm_weight, const float* hpe_norm_bias,
                       const float* message_norm_weight, const float* message_norm_bias, int B,
                       int N, int K, int D, int H, int C, float* out, void* workspace,
                       size_t workspace_bytes, void* stream, bool tc) {
    F2S_REQUIRE(B >= 0 && N >= 0 && K >= 1 && D >= 1 && H >= 1 && C >= 1,
                "neighbor_reduce: bad shape B=%d N=%d K=%d D=%d H=%d C=%d", B, N, K, D, H, C);
    if (B == 0 || N == 0) return F2S_OK;
    F2S_REQUIRE(content && geometry && indices && hpe_input_weight && hpe_input_bias &&
                    hpe_output_weight && hpe_output_bias && hpe_norm_weight && hpe_norm_bias &&
                    message_norm_weight && message_norm_bias && out && workspace,
                "neighbor_reduce: null pointer");
    const size_t need = (size_t)B * N * 3 * C * sizeof(float);
    if (workspace_bytes < need)
        return fail(F2S_ERR_WORKSPACE, "neighbor_reduce needs %zu workspace bytes, got %zu", need,
                    workspace_bytes);
    cudaStream_t st = as_stream(stream);
    float* content_pm = static_cast<float*>(workspace);       // (B*N, 2C)
    float* out_pm = content_pm + (size_t)B * N * 2 * C;         // (B*N, C)
    EdgeArgs ea{};
    ea.content = content_pm;
    ea.ldc = 2 * C;
    ea.geometry = geometry;
    ea.D = D;
    ea.idx = indices;
    ea.B = B;
    ea.M = N;
    ea.K = K;
    ea.H = H;
    ea.cout = C;
    ea.hpe_w = hpe_input_weight;
    ea.hpe_b = hpe_input_bias;
    ea.hpe_ln_w = hpe_norm_weight;
    ea.hpe_ln_b = hpe_norm_bias;
    ea.contrib_w = hpe_output_weight;
    ea.contrib_b = hpe_output_bias;
    ea.ln_w = message_norm_weight;
    ea.ln_b = message_norm_bias;
    ea.out = out_pm;
    ea.ldo = C;
    if (tc) {
        // the shape check first, so an unsupported shape launches nothing
        int log2K = 0;
        while ((1 << log2K) < K) ++log2K;
        F2S_LIMIT(D == 6 && (H == 64 || H == 128) && (C == 64 || C == 128 || C == 192) &&
                      (1 << log2K) == K && K >= 8 && K <= 32 &&
                      ((uintptr_t)hpe_output_weight & 15) == 0,
                  "neighbor_reduce_tc: D=%d H=%d C=%d K=%d outside the tensor-core kernel "
                  "(D 6, H 64 or 128, C 64, 128 or 192, K 8, 16 or 32)", D, H, C, K);
    }
    F2S_TRY(transpose_batched(content, content_pm, B, 2 * C, N, st));
    F2S_TRY(tc ? edge_stage_unified(ea, st) : edge_stage_f32(ea, st));
    return transpose_batched(out_pm, out, B, N, C, st);
}
}  // namespace

extern "C" int f2s_neighbor_reduce(const float* content, const float* geometry,
                                   const int32_t* indices, const float* hpe_input_weight,
                                   const float* hpe_input_bias, const float* hpe_output_weight,
                                   const float* hpe_output_bias, const float* hpe_norm_weight,
                                   const float* hpe_norm_bias, const float* message_norm_weight,
                                   const float* message_norm_bias, int B, int N, int K, int D,
                                   int H, int C, float* out, void* workspace,
                                   size_t workspace_bytes, void* stream) {
    return neighbor_reduce_op(content, geometry, indices, hpe_input_weight, hpe_input_bias,
                              hpe_output_weight, hpe_output_bias, hpe_norm_weight, hpe_norm_bias,
                              message_norm_weight, message_norm_bias, B, N, K, D, H, C, out,
                              workspace, workspace_bytes, stream, false);
}

extern "C" int f2s_neighbor_reduce_tc(const float* content, const float* geometry,
                                      const int32_t* indices, const float* hpe_input_weight,
                                      const float* hpe_input_bias, const float* hpe_output_weight,
                                      const float* hpe_output_bias, const float* hpe_norm_weight,
                                      const float* hpe_norm_bias, const float* message_norm_weight,
                                      const float* message_norm_bias, int B, int N, int K, int D,
                                      int H, int C, float* out, void* workspace,
                                      size_t workspace_bytes, void* stream) {
    return neighbor_reduce_op(content, geometry, indices, hpe_input_weight, hpe_input_bias,
                              hpe_output_weight, hpe_output_bias, hpe_norm_weight, hpe_norm_bias,
                              message_norm_weight, message_norm_bias, B, N, K, D, H, C, out,
                              workspace, workspace_bytes, stream, true);
}

extern "C" int f2s_offset_attention_workspace_bytes(int B, int N, int d, size_t* bytes) {
    F2S_REQUIRE(B >= 0 && N >= 0 && d >= 0 && bytes, "bad workspace query");
    *bytes = (size_t)B * N * (d + 1) * sizeof(float);
    return F2S_OK;
}

extern "C" int f2s_offset_attention(const float* query, const float* key, const float* value,
                                    int B, int N, int d, int C, float* out, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    F2S_REQUIRE(B >= 0 && N >= 0 && d >= 1 && C >= 1,
                "offset_attention: bad shape B=%d N=%d d=%d C=%d", B, N, d, C);
    if (B == 0 || N == 0) return F2S_OK;
    F2S_REQUIRE(query && key && value && out && workspace, "offset_attention: null pointer");
    const size_t need = (size_t)B * N * (d + 1) * sizeof(float);
    if (workspace_bytes < need)
        return fail(F2S_ERR_WORKSPACE, "offset_attention needs %zu workspace bytes, got %zu",
                    need, workspace_bytes);
    cudaStream_t st = as_stream(stream);
    float* key_pm = static_cast<float*>(workspace);           // (B*N, d)
    float* colstats = key_pm + (size_t)B * N * d;             // (B*N)
    F2S_TRY(transpose_batched(key, key_pm, B, d, N, st));
    return attention_f32(query, key_pm, d, value, C, nullptr, 0, out, C, colstats, B, N, d, C,
                         false, st);
}

extern "C" int f2s_offset_attention_tc_workspace_bytes(int B, int N, int d, int C,
                                                       size_t* bytes) {
    F2S_REQUIRE(B >= 0 && N >= 0 && d >= 0 && C >= 0 && bytes, "bad workspace query");
    const size_t key_floats = ((size_t)B * N * d + 63) & ~size_t(63);
    *bytes = (key_floats + (size_t)attention_tc_workspace_floats(B, N, C)) * sizeof(float);
    return F2S_OK;
}

extern "C" int f2s_offset_attention_tc(const float* query, const float* key, const float* value,
                                       int B, int N, int d, int C, float* out, void* workspace,
                                       size_t workspace_bytes, void* stream) {
    F2S_REQUIRE(B >= 0 && N >= 0 && d >= 1 && C >= 1,
                "offset_attention: bad shape B=%d N=%d d=%d C=%d", B, N, d, C);
    if (B == 0 || N == 0) return F2S_OK;
    F2S_REQUIRE(query && key && value && out && workspace, "offset_attention: null pointer");
    F2S_LIMIT(d <= 64 && d % 4 == 0 && C % 64 == 0 && C <= 256 && ((uintptr_t)query & 15) == 0,
              "offset_attention_tc: d=%d C=%d outside the tensor-core kernel (d a multiple of 4 "
              "up to 64, C a multiple of 64 up to 256)", d, C);
    size_t need = 0;
    F2S_TRY(f2s_offset_attention_tc_workspace_bytes(B, N, d, C, &need));
    if (workspace_bytes < need)
        return fail(F2S_ERR_WORKSPACE, "offset_attention_tc needs %zu workspace bytes, got %zu",
                    need, workspace_bytes);
    cudaStream_t st = as_stream(stream);
    float* key_pm = static_cast<float*>(workspace);  // (B*N, d)
    float* attn_ws = key_pm + (((size_t)B * N * d + 63) & ~size_t(63));
    F2S_TRY(transpose_batched(key, key_pm, B, d, N, st));
    // the query rows and the transposed key rows share the pitch d
    return attention_tc(query, key_pm, d, value, C, nullptr, 0, out, C, attn_ws, B, N, d, C,
                        false, false, st);
}
