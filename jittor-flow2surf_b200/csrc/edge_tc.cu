// Fused neighbour stage on tcgen05 tensor cores.
//
// Same arithmetic as edge.cu (encoder.py:83-115, neighbor_reduce.py:244-337,
// hpe.py:14-50, hpe_hidden_forward.cu, neighbor_reduce_forward.cu); the
// per-edge composed projection W_po h (the stage's only contraction) runs as
// a tcgen05 MMA with the hidden rows as the A operand. Nothing per edge
// reaches HBM.
//
// Persistent CTA of 512 threads; W_po resident in shared memory (TMA,
// 128-byte swizzle, K-major), every per-channel parameter staged in shared
// memory; per tile of 128 edge rows (128 / K points):
//   1. hidden: 4 threads per edge row gather xyz_i, xyz_j and evaluate
//      W_in g + b_in, the HPE LayerNorm (E[h^2] - E[h]^2, eps 1e-5) and GELU
//      for a quarter of the H channels, writing them straight into shared
//      memory in the swizzled layout the MMA reads (generic-proxy writes
//      fenced for the async proxy);
//   2. one thread issues the MMAs (M = 128, N = C_out) into TMEM;
//   3. 16 warps = 4 TMEM lane quarters x 4 column groups: the message
//      content[j] + content[i] + (acc + b_po) is formed once and written back
//      to TMEM, the two-pass LayerNorm (eps 1e-6) reads only TMEM, and after
//      the affine + LeakyReLU the max over each point's K edge rows (K lanes)
//      is a register butterfly across lanes that leaves lane = channel, so the
//      output row is stored coalesced.
#include <cfloat>
#include <cstring>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace f2s {
namespace {

constexpr int kThreads = 512;
constexpr int kRows = 128;
constexpr int kParts = 4;    // threads per row in phase 1, column groups in phase 3
constexpr int kMaxPer = 32;  // hidden channels per thread: H <= 128
constexpr unsigned kFull = 0xffffffffu;

struct EdgeTcArgs {
    const float* content;
    int ldc;
    const float* xyz4;
    const int32_t* idx;
    int B, M, K, log2K, H, cout;
    int ppt;  // points per tile (128 / K)
    const float* hpe_w;
    const float* hpe_b;
    const float* hpe_ln_w;
    const float* hpe_ln_b;
    const float* contrib_b;
    const float* contrib_w;  // fp32 (cout x H): converted in-kernel for the bf16 modes
    const float* ln_w;
    const float* ln_b;
    float* out;
    int ldo;
    uint32_t idesc;
    int* err;
};

// Byte offset of 16-byte chunk `chunk` of row `row` inside a K-block of
// 128-byte rows in the 128-byte-swizzle layout (8-row atoms of 1024 bytes).
__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Operand modes of the edge contraction.
enum EdgeMode : int {
    kModeTf32 = 0,   // fp32 hidden rows and weights read as tf32
    kModeBf16 = 1,   // bf16 hidden rows and weights
    kModeSplit = 2,  // x = hi + lo with hi, lo bf16; hi*hi + hi*lo + lo*hi (3 MMAs)
};

template <int kMode>
__global__ void __launch_bounds__(kThreads, 1)
edge_tc_kernel(const __grid_constant__ CUtensorMap map_w, const EdgeTcArgs a) {
    extern __shared__ __align__(1024) unsigned char edge_smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(edge_smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr bool kTf32 = kMode == kModeTf32;
    constexpr bool kSplit = kMode == kModeSplit;
    constexpr int kElem = kTf32 ? 4 : 2;
    constexpr int kBk = 128 / kElem;   // K elements per 128-byte row
    constexpr int kPer = 16 / kElem;   // elements per 16-byte chunk
    const int H = a.H, cout = a.cout, K = a.K;
    const int kblocks = (H + kBk - 1) / kBk;
    const size_t a_bytes = (size_t)kblocks * kRows * 128;
    const size_t b_bytes = (size_t)kblocks * cout * 128;
    unsigned char* sA = smem;                     // kblocks x 16 KB
    unsigned char* sAlo = sA + a_bytes;           // split mode: low halves
    unsigned char* sB = sAlo + (kSplit ? a_bytes : 0);
    unsigned char* sBlo = sB + b_bytes;
    float* sW = reinterpret_cast<float*>(sBlo + (kSplit ? b_bytes : 0));  // H x 6
    float* sHb = sW + H * 6;
    float* sHg = sHb + H;
    float* sHs = sHg + H;
    float* sCb = sHs + H;                                         // cout
    float* sLg = sCb + cout;
    float* sLs = sLg + cout;
    float* sStat = sLs + cout;                                    // [2][kParts][128]
    int* sJ = reinterpret_cast<int*>(sStat + 2 * kParts * kRows); // [128]
    uint64_t* bars = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(sJ + kRows) + 7) & ~uintptr_t(7));  // [0] weights, [1] mma
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
    int* sFlag = reinterpret_cast<int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int R = a.B * a.M;
    const int n_tiles = (R + a.ppt - 1) / a.ppt;
    uint32_t tmem_cols = 32;
    while (tmem_cols < (uint32_t)cout) tmem_cols <<= 1;

    for (int i = tid; i < H * 6; i += kThreads) sW[i] = a.hpe_w[i];
    for (int i = tid; i < H; i += kThreads) {
        sHb[i] = a.hpe_b[i];
        sHg[i] = a.hpe_ln_w[i];
        sHs[i] = a.hpe_ln_b[i];
    }
    for (int i = tid; i < cout; i += kThreads) {
        sCb[i] = a.contrib_b[i];
        sLg[i] = a.ln_w[i];
        sLs[i] = a.ln_b[i];
    }
    if (tid == 0) {
        tc::mbar_init(&bars[0], 1);
        tc::mbar_init(&bars[1], 1);
        tc::fence_barrier_init();
    }
    if (warp == 0) tc::tmem_alloc(tmem_slot, tmem_cols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    bool ok = true;
    if constexpr (kTf32) {
        if (tid == 0) {
            tc::mbar_arrive_expect_tx(&bars[0], (uint32_t)(kblocks * cout * 128));
            for (int kb = 0; kb < kblocks; ++kb)
                tc::tma_load_2d(sB + (size_t)kb * cout * 128, &map_w, &bars[0], kb * kBk, 0);
            ok = tc::mbar_wait(&bars[0], 0, a.err);
        }
    } else {
        // bf16 weights (and their residuals in split mode), swizzled like TMA would
        const int chunks_per_row = H / 8;
        for (int t = tid; t < cout * chunks_per_row; t += kThreads) {
            const int n = t / chunks_per_row, q = t - n * chunks_per_row;
            const float4 w0 = *reinterpret_cast<const float4*>(a.contrib_w + (size_t)n * H + q * 8);
            const float4 w1 = *reinterpret_cast<const float4*>(a.contrib_w + (size_t)n * H + q * 8 + 4);
            const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 h2 = __floats2bfloat162_rn(w[2 * e], w[2 * e + 1]);
                const __nv_bfloat162 l2 = __floats2bfloat162_rn(
                    w[2 * e] - __bfloat162float(h2.x), w[2 * e + 1] - __bfloat162float(h2.y));
                hi[e] = *reinterpret_cast<const uint32_t*>(&h2);
                lo[e] = *reinterpret_cast<const uint32_t*>(&l2);
            }
            const size_t off = (size_t)(q / 8) * cout * 128 + sw128_offset(n, q % 8);
            *reinterpret_cast<uint4*>(sB + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            if (kSplit) *reinterpret_cast<uint4*>(sBlo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        fence_proxy_async();
        __syncthreads();
    }

    const int hper = H / kParts;
    uint32_t mma_phase = 0;

    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        // one thread decides whether to go on; every thread follows it
        if (tid == 0) *sFlag = *reinterpret_cast<volatile int*>(a.err) != tc::kTcOk;
        __syncthreads();
        if (*sFlag) break;
        const int p0 = tile * a.ppt;
        // ---- 1. hidden rows -> A operand --------------------------------
        {
            const int row = tid & (kRows - 1);
            const int part = tid >> 7;
            const int pl = row >> a.log2K;
            const int p = p0 + pl;
            const bool valid = pl < a.ppt && p < R;
            float g[6] = {0, 0, 0, 0, 0, 0};
            if (valid) {
                const int kk = row - (pl << a.log2K);
                const int b = p / a.M;
                const int jrow = b * a.M + a.idx[(size_t)p * K + kk];
                const float4 xi = *reinterpret_cast<const float4*>(a.xyz4 + (size_t)p * 4);
                const float4 xj = *reinterpret_cast<const float4*>(a.xyz4 + (size_t)jrow * 4);
                g[0] = xj.x - xi.x; g[1] = xj.y - xi.y; g[2] = xj.z - xi.z;
                g[3] = xi.x; g[4] = xi.y; g[5] = xi.z;
                if (part == 0) sJ[row] = jrow;
            } else if (part == 0) {
                sJ[row] = -1;
            }
            const int ch0 = part * hper;
            float pre[kMaxPer];
            float s = 0.0f, s2 = 0.0f;
#pragma unroll
            for (int i = 0; i < kMaxPer; ++i) {
                if (i < hper) {
                    const int c = ch0 + i;
                    float v = sHb[c];
#pragma unroll
                    for (int d = 0; d < 6; ++d) v = fmaf(g[d], sW[c * 6 + d], v);
                    pre[i] = v;
                    s += v;
                    s2 = fmaf(v, v, s2);
                }
            }
            sStat[part * kRows + row] = s;
            sStat[(kParts + part) * kRows + row] = s2;
            __syncthreads();
            float ts = 0.0f, ts2 = 0.0f;
#pragma unroll
            for (int q = 0; q < kParts; ++q) {
                ts += sStat[q * kRows + row];
                ts2 += sStat[(kParts + q) * kRows + row];
            }
            const float mean = ts / (float)H;
            const float var = fmaxf(ts2 / (float)H - mean * mean, 0.0f);
            const float rstd = rsqrtf(var + 1e-5f);
#pragma unroll
            for (int i0 = 0; i0 < kMaxPer; i0 += kPer) {
                if (i0 < hper) {
                    float o[kPer];
#pragma unroll
                    for (int e = 0; e < kPer; ++e) {
                        const int c = ch0 + i0 + e;
                        o[e] = valid ? f2s_gelu_erf((pre[i0 + e] - mean) * rstd * sHg[c] + sHs[c])
                                     : 0.0f;
                    }
                    const int c = ch0 + i0;
                    unsigned char* dst = sA + (size_t)(c / kBk) * kRows * 128 +
                                         sw128_offset(row, (c % kBk) / kPer);
                    if constexpr (kTf32) {
                        *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
                    } else {
                        uint32_t w[4], wl[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const __nv_bfloat162 b2 = __floats2bfloat162_rn(o[2 * e], o[2 * e + 1]);
                            w[e] = *reinterpret_cast<const uint32_t*>(&b2);
                            if (kSplit) {
                                const __nv_bfloat162 l2 = __floats2bfloat162_rn(
                                    o[2 * e] - __bfloat162float(b2.x),
                                    o[2 * e + 1] - __bfloat162float(b2.y));
                                wl[e] = *reinterpret_cast<const uint32_t*>(&l2);
                            }
                        }
                        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
                        if (kSplit)
                            *reinterpret_cast<uint4*>(dst + (sAlo - sA)) =
                                make_uint4(wl[0], wl[1], wl[2], wl[3]);
                    }
                }
            }
        }
        fence_proxy_async();
        tc::tc_fence_before();
        __syncthreads();
        // ---- 2. MMA -------------------------------------------------------
        if (tid == 0) {
            tc::tc_fence_after();
            if (ok) {
                const uint32_t a0 = tc::smem_u32(sA), b0 = tc::smem_u32(sB);
                const uint32_t a_lo = tc::smem_u32(sAlo), b_lo = tc::smem_u32(sBlo);
                for (int kb = 0; kb < kblocks; ++kb)
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if ((kb * kBk + k * (32 / kElem)) >= H) break;
                        const uint32_t ao = kb * kRows * 128 + k * 32;
                        const uint32_t bo = kb * cout * 128 + k * 32;
                        const uint64_t da = tc::sw128_desc(a0 + ao);
                        const uint64_t db = tc::sw128_desc(b0 + bo);
                        tc::umma<kTf32>(tmem_base, da, db, a.idesc, (kb | k) ? 1u : 0u);
                        if (kSplit) {
                            tc::umma<false>(tmem_base, da, tc::sw128_desc(b_lo + bo), a.idesc, 1u);
                            tc::umma<false>(tmem_base, tc::sw128_desc(a_lo + ao), db, a.idesc, 1u);
                        }
                    }
            }
            tc::umma_commit(&bars[1]);
            *sFlag = tc::mbar_wait(&bars[1], mma_phase, a.err) ? 0 : 1;
        }
        __syncthreads();
        if (*sFlag) break;
        mma_phase ^= 1u;
        tc::tc_fence_after();
        // ---- 3. message LayerNorm, LeakyReLU, max over k --------------------
        {
            const int quarter = warp & 3;
            const int cpart = warp >> 2;
            const int erow = quarter * 32 + lane;  // TMEM lane = edge row
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16);
            const int ej = sJ[erow];
            const int ep = p0 + (erow >> a.log2K);
            const float* cj = a.content + (size_t)(ej < 0 ? 0 : ej) * a.ldc;
            // centre terms: one point per K consecutive lanes, mostly a broadcast
            const float* ci = a.content + (size_t)(ej < 0 ? 0 : ep) * a.ldc + cout;
            const int nchunks = cout / 32;
            // pass 1: message = content[j] + content[i] + (acc + b_po) -> TMEM
            float sum = 0.0f;
            for (int ch = cpart; ch < nchunks; ch += kParts) {
                const int cb = ch * 32;
                float v[32];
                tc::tmem_ld32(taddr + (uint32_t)cb, v);
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    const float4 nj = *reinterpret_cast<const float4*>(cj + cb + i);
                    const float4 ni = *reinterpret_cast<const float4*>(ci + cb + i);
                    v[i + 0] = nj.x + ni.x + (v[i + 0] + sCb[cb + i + 0]);
                    v[i + 1] = nj.y + ni.y + (v[i + 1] + sCb[cb + i + 1]);
                    v[i + 2] = nj.z + ni.z + (v[i + 2] + sCb[cb + i + 2]);
                    v[i + 3] = nj.w + ni.w + (v[i + 3] + sCb[cb + i + 3]);
                    sum += (v[i] + v[i + 1]) + (v[i + 2] + v[i + 3]);
                }
                tc::tmem_st32(taddr + (uint32_t)cb, v);
            }
            sStat[cpart * kRows + erow] = sum;
            __syncthreads();
            float tot = 0.0f;
#pragma unroll
            for (int q = 0; q < kParts; ++q) tot += sStat[q * kRows + erow];
            const float mean = tot / (float)cout;
            // pass 2: centred second moment
            float q2 = 0.0f;
            for (int ch = cpart; ch < nchunks; ch += kParts) {
                float v[32];
                tc::tmem_ld32(taddr + (uint32_t)(ch * 32), v);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float d = v[i] - mean;
                    q2 = fmaf(d, d, q2);
                }
            }
            sStat[(kParts + cpart) * kRows + erow] = q2;
            __syncthreads();
            float totq = 0.0f;
#pragma unroll
            for (int q = 0; q < kParts; ++q) totq += sStat[(kParts + q) * kRows + erow];
            const float rstd = rsqrtf(totq / (float)cout + 1e-6f);
            // pass 3: affine + LeakyReLU, then max over the K lanes of each point
            for (int ch = cpart; ch < nchunks; ch += kParts) {
                const int cb = ch * 32;
                float y[32];
                tc::tmem_ld32(taddr + (uint32_t)cb, y);
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    y[i] = ej >= 0 ? f2s_leaky((y[i] - mean) * rstd * sLg[cb + i] + sLs[cb + i])
                                   : -FLT_MAX;
                int off = 0;
#pragma unroll
                for (int s = 0; s < 5; ++s) {
                    if (s < a.log2K) {
                        const int m = K >> (s + 1);
                        const bool hi = (lane & m) != 0;
                        const int h = 16 >> s;
#pragma unroll
                        for (int i = 0; i < h; ++i) {
                            const float send = hi ? y[i] : y[h + i];
                            const float keep = hi ? y[h + i] : y[i];
                            y[i] = fmaxf(keep, __shfl_xor_sync(kFull, send, m));
                        }
                        off += hi ? h : 0;
                    }
                }
                if (ep < R) {
                    const int nv = 32 >> a.log2K;
                    float* o = a.out + (size_t)ep * a.ldo + cb + off;
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (i < nv) o[i] = y[i];
                }
            }
        }
        tc::tc_fence_before();
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, tmem_cols);
    }
}

}  // namespace

// Tensor-core edge stage at `precision` (F2S_PRECISION_TF32, _BF16 or
// _BF16X3); returns F2S_ERR_UNSUPPORTED for shapes it does not cover (the
// caller then uses the CUDA-core kernel).
int edge_stage_tc(const EdgeArgs& e, int precision, cudaStream_t st) {
    if (e.B == 0 || e.M == 0) return F2S_OK;
    int log2K = 0;
    while ((1 << log2K) < e.K) ++log2K;
    if (e.geometry != nullptr || e.xyz4 == nullptr || e.D != 6 || e.H > kParts * kMaxPer ||
        e.H % 32 != 0 || e.cout % 32 != 0 || e.cout > 256 || (1 << log2K) != e.K || e.K > 32 ||
        ((uintptr_t)e.content & 15) != 0 || e.ldc % 4 != 0 || ((uintptr_t)e.contrib_w & 15) != 0)
        return fail(F2S_ERR_UNSUPPORTED, "edge stage shape outside the tensor-core kernel");
    const int mode = precision == F2S_PRECISION_TF32   ? kModeTf32
                     : precision == F2S_PRECISION_BF16 ? kModeBf16
                                                       : kModeSplit;
    F2S_REQUIRE(precision == F2S_PRECISION_TF32 || precision == F2S_PRECISION_BF16 ||
                    precision == F2S_PRECISION_BF16X3,
                "edge_tc: precision %d", precision);
    int* err = tc_error_word();
    if (!err) return fail(F2S_ERR_CUDA, "edge_tc: device error word unavailable");
    const bool tf32 = mode == kModeTf32;
    const int elem = tf32 ? 4 : 2;
    const int bk = 128 / elem;
    const int kblocks = ceil_div(e.H, bk);
    CUtensorMap map;
    if (tf32) F2S_TRY(make_tensor_map_2d(&map, e.contrib_w, true, e.cout, e.H, e.H, e.cout, bk));
    else memset(&map, 0, sizeof(map));
    EdgeTcArgs a{};
    a.content = e.content;
    a.ldc = e.ldc;
    a.xyz4 = e.xyz4;
    a.idx = e.idx;
    a.B = e.B;
    a.M = e.M;
    a.K = e.K;
    a.log2K = log2K;
    a.H = e.H;
    a.cout = e.cout;
    a.ppt = kRows / e.K;
    a.hpe_w = e.hpe_w;
    a.hpe_b = e.hpe_b;
    a.hpe_ln_w = e.hpe_ln_w;
    a.hpe_ln_b = e.hpe_ln_b;
    a.contrib_b = e.contrib_b;
    a.contrib_w = e.contrib_w;
    a.ln_w = e.ln_w;
    a.ln_b = e.ln_b;
    a.out = e.out;
    a.ldo = e.ldo;
    a.idesc = tc::make_idesc(kRows, e.cout, tf32 ? 2u : 1u);
    a.err = err;
    const size_t copies = mode == kModeSplit ? 2 : 1;
    const size_t smem = 1024 + copies * ((size_t)kblocks * kRows * 128 +
                                         (size_t)kblocks * e.cout * 128) +
                        sizeof(float) * ((size_t)e.H * 9 + (size_t)e.cout * 3 + 2 * kParts * kRows) +
                        sizeof(int) * kRows + 64;
    F2S_LIMIT(smem <= 227 * 1024, "edge_tc: %zu bytes of shared memory", smem);
    const int R = e.B * e.M;
    const int tiles = ceil_div(R, a.ppt);
    const int grid = tiles < sm_count() ? tiles : sm_count();
    TraceScope trace(kTagEdge, st);
    auto launch = [&](auto kernel) -> int {
        F2S_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
        kernel<<<grid, kThreads, smem, st>>>(map, a);
        return check_launch("edge_tc_kernel");
    };
    if (mode == kModeTf32) return launch(edge_tc_kernel<kModeTf32>);
    if (mode == kModeBf16) return launch(edge_tc_kernel<kModeBf16>);
    return launch(edge_tc_kernel<kModeSplit>);
}

}  // namespace f2s
