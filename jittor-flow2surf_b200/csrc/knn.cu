// k nearest non-self neighbours in feature space, bit-exact to the reference's
// global_knn kernel (flow2surf/models/ops/cuda/knn_global.cu:1-53).
//
// Semantics restated from the reference:
//   - per (query q, candidate j != q) in fp32, accumulated over channels in
//     order with fused multiply-adds: qn = sum f_qc^2, rn = sum f_jc^2,
//     ip = sum f_qc f_jc (knn_global.cu:19-28, nvcc contracts `x += a*b`);
//     d = qn + rn - 2 ip (knn_global.cu:29);
//   - key = (order-preserving bits of d with -0 -> +0, j) compared
//     lexicographically (knn.cuh:7-17); the k smallest keys, ascending.
//
// B200 design (not the reference's one-block-per-query, K rounds of block-min):
//   - one CTA per (patch, 64 queries); the patch's features and per-point
//     squared norms are staged once in shared memory;
//   - one warp per query: each lane holds ceil(N/32) keys in registers;
//   - a candidate filter: the k-th smallest of the 64 minima of half-lane
//     slot groups bounds the k-th key from above; the (typically ~50) keys at
//     or below it are compacted with ballots and sorted as (key, index)
//     pairs by a 64-wide warp bitonic network, whose first k are the answer;
//   - when more than 64 keys pass, the k-th smallest key is found exactly by
//     a 4-pass, 8-bit radix select over a per-warp shared-memory histogram;
//     keys below it and the lowest-index ties are compacted in index order
//     with ballots; the <= 32 survivors are sorted by a warp bitonic network
//     and written coalesced.
// Work per query is O(N/32 + log^2 64) lane steps on the filter path (plus
// 4*256/32 on the radix path) instead of the
// reference's k block-wide reductions.
#include "common.cuh"

using f2s::TraceScope;
using f2s::kTagKnn;

namespace {

constexpr int kWarps = 8;
constexpr int kQueriesPerCta = 64;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ uint64_t warp_bitonic_sort_u64(uint64_t v, int lane) {
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const uint64_t other = __shfl_xor_sync(kFull, v, stride);
            const bool ascending = (lane & size) == 0;
            const bool lower = (lane & stride) == 0;
            const uint64_t lo = other < v ? other : v;
            const uint64_t hi = other < v ? v : other;
            v = (lower == ascending) ? lo : hi;
        }
    }
    return v;
}

// Ascending bitonic sort of 64 values held two per lane (element lane and
// element 32 + lane).
template <typename T>
__device__ __forceinline__ void warp_bitonic_sort64(T& v0, T& v1, int lane) {
#pragma unroll
    for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride == 32) {  // elements lane and 32 + lane; size 64 sorts ascending
                const T lo = v1 < v0 ? v1 : v0;
                const T hi = v1 < v0 ? v0 : v1;
                v0 = lo;
                v1 = hi;
            } else {
                const bool lower = (lane & stride) == 0;
                {
                    const T other = __shfl_xor_sync(kFull, v0, stride);
                    const bool asc = (lane & size) == 0;  // element index lane
                    const T lo = other < v0 ? other : v0, hi = other < v0 ? v0 : other;
                    v0 = (lower == asc) ? lo : hi;
                }
                {
                    const T other = __shfl_xor_sync(kFull, v1, stride);
                    const bool asc = ((32 + lane) & size) == 0;  // element index 32 + lane
                    const T lo = other < v1 ? other : v1, hi = other < v1 ? v1 : other;
                    v1 = (lower == asc) ? lo : hi;
                }
            }
        }
    }
}

// CFIX = 3 specialises the channel loop for xyz; CFIX = 0 takes C at run time.
template <int SLOTS, int CFIX>
__global__ void __launch_bounds__(kWarps * 32)
knn_kernel(const float* __restrict__ features, int C_runtime, int N, int k, int actual_k,
           int tiles_per_patch, int32_t* __restrict__ out) {
    const int C = CFIX > 0 ? CFIX : C_runtime;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int n_pad = (N + 3) & ~3;
    float* s_norm = reinterpret_cast<float*>(smem_raw);
    uint32_t* s_hist = reinterpret_cast<uint32_t*>(s_norm + n_pad);
    uint64_t* s_list = reinterpret_cast<uint64_t*>(s_hist + kWarps * 256);
    float* s_feat = reinterpret_cast<float*>(s_list + kWarps * 64);

    const int b = blockIdx.x / tiles_per_patch;
    const int tile = blockIdx.x - b * tiles_per_patch;
    const float* f = features + (size_t)b * C * N;

    // xyz (CFIX = 3): one float4 (x, y, z, |p|^2) per point, zero padded to
    // SLOTS * 32, so a slot is one 16-byte load with no bounds check
    float4* s_pts = reinterpret_cast<float4*>(s_feat);
    if constexpr (CFIX == 3) {
        for (int j = threadIdx.x; j < SLOTS * 32; j += blockDim.x) {
            float4 p = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (j < N) {
                p.x = f[j];
                p.y = f[(size_t)N + j];
                p.z = f[2 * (size_t)N + j];
                float norm = 0.0f;
                norm = __fmaf_rn(p.x, p.x, norm);
                norm = __fmaf_rn(p.y, p.y, norm);
                norm = __fmaf_rn(p.z, p.z, norm);
                p.w = norm;
            }
            s_pts[j] = p;
        }
    } else {
        for (int j = threadIdx.x; j < N; j += blockDim.x) {
            float norm = 0.0f;
            for (int c = 0; c < C; ++c) {
                const float v = f[(size_t)c * N + j];
                s_feat[(size_t)c * N + j] = v;
                norm = __fmaf_rn(v, v, norm);
            }
            s_norm[j] = norm;
        }
    }
    __syncthreads();
    const float* fe = s_feat;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const unsigned lanes_below = (1u << lane) - 1u;
    uint32_t* hist = s_hist + warp * 256;
    uint64_t* list = s_list + warp * 64;  // selected keys (32) or filter candidates (64)
    uint64_t* cl = list;

    const int q_begin = tile * kQueriesPerCta;
    const int q_end = min(N, q_begin + kQueriesPerCta);
    for (int q = q_begin + warp; q < q_end; q += kWarps) {
        float qn;
        // Inner products accumulate channel by channel; per (q, j) the order
        // is c = 0, 1, ... as in the reference.
        // ip[r] becomes the slot's d = |q|^2 + |p|^2 - 2 q.p
        float ip[SLOTS];
        if constexpr (CFIX == 3) {
            const float4 qp = s_pts[q];
            qn = qp.w;
#pragma unroll
            for (int r = 0; r < SLOTS; ++r) {
                const float4 p = s_pts[r * 32 + lane];
                float t = __fmaf_rn(qp.x, p.x, 0.0f);
                t = __fmaf_rn(qp.y, p.y, t);
                t = __fmaf_rn(qp.z, p.z, t);
                ip[r] = __fmaf_rn(-2.0f, t, __fadd_rn(qn, p.w));
            }
        } else {
            qn = s_norm[q];
            // channel-outer loop so the slot loop unrolls
#pragma unroll
            for (int r = 0; r < SLOTS; ++r) ip[r] = 0.0f;
            for (int c = 0; c < C; ++c) {
                const float* row = fe + (size_t)c * N;
                const float qc = row[q];
#pragma unroll
                for (int r = 0; r < SLOTS; ++r) {
                    const int j = r * 32 + lane;
                    const float fj = j < N ? row[j] : 0.0f;
                    ip[r] = __fmaf_rn(qc, fj, ip[r]);
                }
            }
#pragma unroll
            for (int r = 0; r < SLOTS; ++r) {
                const int j = r * 32 + lane;
                ip[r] = __fmaf_rn(-2.0f, ip[r], __fadd_rn(qn, j < N ? s_norm[j] : 0.0f));
            }
        }
        uint32_t key[SLOTS];
#pragma unroll
        for (int r = 0; r < SLOTS; ++r) {
            const int j = r * 32 + lane;
            uint32_t kk = 0xffffffffu;
            if (j < N && j != q) {
                const float d = ip[r];
                kk = f2s_ordered_bits(d);
            }
            key[r] = kk;
        }

        // Candidate filter. Each lane's slots form two groups (even and odd
        // slots); the
        // actual_k-th smallest of the 64 group minima is a key T with at
        // least actual_k distinct elements at or below it, so every selected
        // element has key <= T (ties at T included). Typically ~5% of the
        // keys pass; up to 64 candidates are sorted as (key, index) pairs,
        // which is the final order, and more fall back to the radix select.
        {
            uint32_t g0 = 0xffffffffu, g1 = 0xffffffffu;
#pragma unroll
            for (int r = 0; r < SLOTS; ++r) {
                const uint32_t kv = key[r];  // 0xffffffff for the query itself and slots past N
                // even / odd slots: both groups sample every part of the index
                // range (patch points are stored in radial order)
                if ((r & 1) == 0) g0 = kv < g0 ? kv : g0;
                else g1 = kv < g1 ? kv : g1;
            }
            warp_bitonic_sort64<uint32_t>(g0, g1, lane);
            const int src = actual_k - 1;  // element index of the threshold (< 32)
            const uint32_t T = __shfl_sync(kFull, g0, src);
            int c = 0;
            // below the all-ones key the threshold already excludes the slots
            // that are not candidates; only T = 0xffffffff needs the check
            const bool check_valid = T == 0xffffffffu;
#pragma unroll
            for (int r = 0; r < SLOTS; ++r) {
                const int j = r * 32 + lane;
                const bool cand = key[r] <= T && (!check_valid || (j < N && j != q));
                const unsigned m = __ballot_sync(kFull, cand);
                const int pos = c + __popc(m & lanes_below);
                if (cand && pos < 64) cl[pos] = ((uint64_t)key[r] << 32) | (uint32_t)j;
                c += __popc(m);
            }
            if (c <= 64) {
                __syncwarp();
                uint64_t v0 = lane < c ? cl[lane] : ~0ull;
                uint64_t v1 = lane + 32 < c ? cl[lane + 32] : ~0ull;
                __syncwarp();
                warp_bitonic_sort64<uint64_t>(v0, v1, lane);
                const int idx = (int)(uint32_t)(v0 & 0xffffffffu);
                const int last = __shfl_sync(kFull, idx, actual_k - 1);
                if (lane < k) out[((size_t)b * N + q) * k + lane] = lane < actual_k ? idx : last;
                continue;
            }
            __syncwarp();
        }

        // Exact radix select of the actual_k-th smallest key among valid ones.
        uint32_t prefix = 0u, pmask = 0u;
        uint32_t need = (uint32_t)actual_k;
#pragma unroll 1
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
#pragma unroll
            for (int i = 0; i < 8; ++i) hist[lane + 32 * i] = 0u;
            __syncwarp();
#pragma unroll
            for (int r = 0; r < SLOTS; ++r) {
                const int j = r * 32 + lane;
                if (j < N && j != q && (key[r] & pmask) == prefix)
                    atomicAdd(&hist[(key[r] >> shift) & 255u], 1u);
            }
            __syncwarp();
            uint32_t cnt[8];
            uint32_t sum = 0u;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                cnt[i] = hist[lane * 8 + i];
                sum += cnt[i];
            }
            uint32_t incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(kFull, incl, o);
                if (lane >= o) incl += t;
            }
            const uint32_t excl = incl - sum;
            const bool owner = excl < need && need <= incl;
            const unsigned owners = __ballot_sync(kFull, owner);
            const int src = __ffs(owners) - 1;
            uint32_t digit = 0u, below = excl;
            if (owner) {
                bool found = false;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (!found) {
                        if (below + cnt[i] >= need) {
                            digit = (uint32_t)(lane * 8 + i);
                            found = true;
                        } else {
                            below += cnt[i];
                        }
                    }
                }
            }
            digit = __shfl_sync(kFull, digit, src);
            below = __shfl_sync(kFull, below, src);
            need -= below;
            prefix |= digit << shift;
            pmask |= 0xffu << shift;
            __syncwarp();
        }

        // Compact keys < T, then the lowest-index ties == T, in index order.
        const uint32_t threshold = prefix;
        const int n_less = actual_k - (int)need;
        int nl = 0, ne = 0;
#pragma unroll
        for (int r = 0; r < SLOTS; ++r) {
            const int j = r * 32 + lane;
            const bool valid = j < N && j != q;
            const bool less = valid && key[r] < threshold;
            const bool equal = valid && key[r] == threshold;
            const unsigned ml = __ballot_sync(kFull, less);
            const unsigned me = __ballot_sync(kFull, equal);
            if (less) list[nl + __popc(ml & lanes_below)] = ((uint64_t)key[r] << 32) | (uint32_t)j;
            if (equal) {
                const int e = ne + __popc(me & lanes_below);
                if (e < (int)need) list[n_less + e] = ((uint64_t)threshold << 32) | (uint32_t)j;
            }
            nl += __popc(ml);
            ne += __popc(me);
        }
        __syncwarp();
        uint64_t v = lane < actual_k ? list[lane] : ~0ull;
        __syncwarp();
        v = warp_bitonic_sort_u64(v, lane);
        const int idx = (int)(uint32_t)(v & 0xffffffffu);
        const int last = __shfl_sync(kFull, idx, actual_k - 1);
        if (lane < k) out[((size_t)b * N + q) * k + lane] = lane < actual_k ? idx : last;
    }
}

template <int SLOTS, int CFIX>
int launch_knn(const float* features, int B, int C, int N, int k, int actual_k, int32_t* out,
               cudaStream_t stream) {
    const int n_pad = (N + 3) & ~3;
    // the features: (C, N) floats, or for xyz one float4 per slot position
    const size_t feat = CFIX == 3 ? (size_t)SLOTS * 32 * 16 : (size_t)C * N * 4;
    const size_t smem = (size_t)n_pad * 4 + (size_t)kWarps * 256 * 4 + (size_t)kWarps * 64 * 8 + feat;
    auto kernel = knn_kernel<SLOTS, CFIX>;
    if (smem > 48 * 1024)
        F2S_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int tiles = f2s::ceil_div(N, kQueriesPerCta);
    const int64_t grid = (int64_t)B * tiles;
    F2S_LIMIT(grid < (1ll << 31), "knn grid too large: B=%d N=%d", B, N);
    TraceScope trace(kTagKnn, stream);
    kernel<<<(unsigned)grid, kWarps * 32, smem, stream>>>(features, C, N, k, actual_k, tiles, out);
    return f2s::check_launch("knn_kernel");
}

template <int CFIX>
int dispatch_slots(const float* features, int B, int C, int N, int k, int actual_k, int32_t* out,
                   cudaStream_t stream) {
    const int slots = f2s::ceil_div(N, 32);
    if (slots <= 8) return launch_knn<8, CFIX>(features, B, C, N, k, actual_k, out, stream);
    if (slots <= 32) return launch_knn<32, CFIX>(features, B, C, N, k, actual_k, out, stream);
    return launch_knn<64, CFIX>(features, B, C, N, k, actual_k, out, stream);
}

}  // namespace

namespace f2s {
// Entry used by the model forward as well as the public operator.
int knn_launch(const float* features, int B, int C, int N, int k, int32_t* indices,
               cudaStream_t stream) {
    F2S_REQUIRE(B >= 0 && C >= 1 && N >= 0, "knn: bad shape B=%d C=%d N=%d", B, C, N);
    F2S_REQUIRE(k >= 1, "k must be >= 1, got %d", k);
    F2S_LIMIT(k <= F2S_KNN_MAX_K, "knn: k=%d exceeds the limit %d", k, F2S_KNN_MAX_K);
    F2S_LIMIT(N <= F2S_KNN_MAX_POINTS, "knn: N=%d exceeds the limit %d", N, F2S_KNN_MAX_POINTS);
    if (B == 0 || N == 0) return F2S_OK;
    F2S_REQUIRE(features != nullptr && indices != nullptr, "knn: null pointer");
    if (N <= 1) {
        F2S_CUDA_TRY(cudaMemsetAsync(indices, 0, (size_t)B * N * k * sizeof(int32_t), stream));
        return F2S_OK;
    }
    const int actual_k = k < N - 1 ? k : N - 1;
    F2S_LIMIT((size_t)C * N * 4 <= F2S_KNN_MAX_FEATURE_BYTES,
              "knn: C*N*4=%zu bytes of features exceed the %d-byte shared-memory stage",
              (size_t)C * N * 4, F2S_KNN_MAX_FEATURE_BYTES);
    if (C == 3) return dispatch_slots<3>(features, B, C, N, k, actual_k, indices, stream);
    return dispatch_slots<0>(features, B, C, N, k, actual_k, indices, stream);
}
}  // namespace f2s

extern "C" int f2s_knn(const float* features, int B, int C, int N, int k, int32_t* indices,
                       void* stream) {
    return f2s::knn_launch(features, B, C, N, k, indices, f2s::as_stream(stream));
}
