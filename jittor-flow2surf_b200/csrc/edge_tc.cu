// Fused neighbour stage on tcgen05 tensor cores.
//
// Same arithmetic as edge.cu (encoder.py:83-115, neighbor_reduce.py:244-337,
// hpe.py:14-50, hpe_hidden_forward.cu, neighbor_reduce_forward.cu); the
// per-edge composed projection W_po h (the stage's only contraction) runs as
// a tcgen05 MMA with the hidden rows as the A operand. Nothing per edge
// reaches HBM.
//
// Persistent CTA of 16 warps, specialised and pipelined over tiles of 128
// edge rows (128 / K points); W_po resident in shared memory (TMA or an
// in-kernel bf16 conversion, 128-byte swizzle, K-major):
//   warps 0-7   hidden producers, two lanes per edge row. The geometry g =
//               [xyz_j - xyz_i, xyz_i] of the next tile is loaded while this
//               tile is processed. The HPE LayerNorm (eps 1e-5) rides on the
//               pre-activation MMA: the per-channel mean of h = W_in g + b_in
//               is linear in g, so with column-centred weights the centred,
//               scaled and shifted h is one K = 8 product [gamma W~ | gamma b~
//               | beta] . [rstd g | rstd | 1], and the variance is a quadratic
//               form in g (the centred rows' 6 x 6 moment matrix, computed
//               once per CTA): O(36) per edge row, no pass over H. Once the A
//               buffer is free (one or two buffers, whatever shared memory
//               holds) they apply GELU to the normalised pre-activations and
//               write the rows into the swizzled buffer; then one lane issues
//               the MMAs (M = 128, N = C_out) into one of two TMEM
//               accumulators and commits "A free" and "accumulator ready".
//               Warp 0 owns the TMEM allocation.
//   warps 8-15  epilogue, two warps per TMEM lane quarter splitting the
//               output channels: the message content[j] + content[i] +
//               (acc + b_po) is formed once from content rows staged in
//               shared memory by coalesced asynchronous copies (a chunk or a
//               tile ahead; the rows two grid rounds ahead are prefetched into
//               L2) and written back to TMEM with its moments about a
//               per-warp shift (one pass, the channel halves combined
//               pairwise); the LayerNorm (eps 1e-6) then reads only TMEM, and
//               after the
//               affine + LeakyReLU the max over each point's K edge rows (K
//               lanes) is a register butterfly across lanes that leaves
//               lane = channel, so the output row is stored coalesced.
// So the hidden rows of tile t + 1 are computed while the epilogue of tile t
// runs, and the MMAs overlap both. Each role has one polling lane per wait;
// the role's other warps wait on a named barrier and issue nothing.
#include <algorithm>
#include <cfloat>
#include <cstring>

#include "edge_common.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace f2s {
namespace {

using namespace edge;
constexpr int kProducerWarps = 8;
constexpr int kEpilogueWarps = 8;
constexpr int kEpiWarp0 = kProducerWarps;
constexpr int kThreads = (kProducerWarps + kEpilogueWarps) * 32;
constexpr int kProducerThreads = kProducerWarps * 32;
constexpr int kEpilogueThreads = kEpilogueWarps * 32;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kEpiBarrier = 1;   // named barrier of the epilogue warps
constexpr int kProdBarrier = 2;  // named barrier of the producer warps

struct EdgeTcArgs {
    const float* content;
    int ldc;
    const float* xyz4;
    const int32_t* idx;
    int B, M, K, log2K, H, cout;
    int ppt;     // points per tile (128 / K)
    int a_bufs;  // hidden-row buffers (1 or 2)
    int stage_bufs;   // content staging buffers per epilogue warp (1 .. 4)
    int stage_bytes;  // bytes of one staging buffer: 32 neighbour rows + the warp's centre rows
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
    uint32_t idesc_pre;  // tf32, M = 128, N = H: the pre-activation MMA
    int* err;
};

__device__ __forceinline__ void epi_barrier() {
    asm volatile("bar.sync %0, %1;" ::"n"(kEpiBarrier), "n"(kEpilogueThreads) : "memory");
}

__device__ __forceinline__ void prod_barrier() {
    asm volatile("bar.sync %0, %1;" ::"n"(kProdBarrier), "n"(kProducerThreads) : "memory");
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
    const size_t a_bytes = (size_t)kblocks * kRows * 128;  // one operand copy of a tile
    const size_t a_buf_bytes = a_bytes * (kSplit ? 2 : 1);  // + low halves
    const size_t b_bytes = (size_t)kblocks * cout * 128;
    unsigned char* sA = smem;                               // a_bufs x a_buf_bytes
    unsigned char* sB = sA + (size_t)a.a_bufs * a_buf_bytes;
    unsigned char* sBlo = sB + b_bytes;
    // the normalised pre-activations LN(W_in g + b_in) as a K = 8 tf32 MMA in
    // the interleaved (no-swizzle) K-major layout: A_u = 128 rows of
    // [rstd g0..g5, rstd, 1], B_w = H rows of [gamma W~ (6), gamma b~, beta]
    // (column-centred weights), each as tf32 hi and lo
    unsigned char* sU = sBlo + (kSplit ? b_bytes : 0);  // 2 x 4 KB
    unsigned char* sWu = sU + 2 * kUBytes;               // 2 x H x 32 bytes
    float* sHn = reinterpret_cast<float*>(sWu + 2 * (size_t)H * 32);  // H x 2 floats of set-up scratch
    // LayerNorm moments of the pre-activations as functions of g:
    // sum = bsum + wsum . g, sum of squares = bsq + g . (2 u + G g)
    float* sGram = sHn + H * 2;  // moments of the centred HPE rows: G[36], a[6], c (16-byte aligned)
    float* sCb = sGram + 52;                                              // cout
    float* sLn = sCb + cout;      // cout x {|gain|, shift}
    float* sSgn = sLn + cout * 2;  // cout: sign of the gain (+1 / -1)
    float* sStat = sSgn + cout;    // [2][2][128]
    float* sRed = sStat + 4 * kRows;  // [8 epilogue warps][32]: per-channel maxima (K = 32)
    uint64_t* bars = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(sRed + kEpilogueWarps * 32) + 7) & ~uintptr_t(7));
    uint64_t* a_empty = bars + 2;   // [2]
    uint64_t* t_full = bars + 4;    // [2]
    uint64_t* t_empty = bars + 6;   // [2]
    uint64_t* w_bar = bars + 8;
    uint64_t* mma_done = bars + 9;
    uint64_t* pre_full = bars + 10;  // pre-activation MMA of the tile done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
    // failure flags of the epilogue and (per tile parity) producer warps:
    // written by the role's one polling lane before the role's named barrier,
    // read by every warp of the role after it
    int* sEpiFail = reinterpret_cast<int*>(tmem_slot + 1);
    int* sProdFail = sEpiFail + 1;  // [2]
    // content staging of the epilogue warps: per warp `stage_bufs` buffers of
    // 32 neighbour rows x 32 channels (128-byte rows, 16-byte chunks swizzled
    // by row & 7) followed by the warp's centre rows (same swizzle by point)
    unsigned char* sStage = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(sProdFail + 2) + 127) & ~uintptr_t(127));

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int R = a.B * a.M;
    const int n_tiles = (R + a.ppt - 1) / a.ppt;
    // TMEM: two accumulators (columns [0, 2 C_out)), the pre-activations
    // (columns [2 C_out, 2 C_out + H))
    uint32_t tmem_cols = 32;
    while (tmem_cols < (uint32_t)(2 * cout + H)) tmem_cols <<= 1;
    const uint32_t pre_col = (uint32_t)(2 * cout);

    const int hh = H >> 1;
    prepare_pre_activation(a.hpe_w, a.hpe_b, a.hpe_ln_w, a.hpe_ln_b, H,
                           reinterpret_cast<double*>(sHn), sWu, sGram, tid, kThreads);
    prepare_message_norm(a.contrib_b, a.ln_w, a.ln_b, cout, sCb, sLn, sSgn, tid, kThreads);
    if (tid == 0) {
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&a_empty[b], 1);
            tc::mbar_init(&t_full[b], 1);
            tc::mbar_init(&t_empty[b], kEpilogueThreads);
        }
        tc::mbar_init(w_bar, 1);
        tc::mbar_init(mma_done, 1);
        tc::mbar_init(pre_full, 1);
        *sEpiFail = 0;
        sProdFail[0] = sProdFail[1] = 0;
        tc::fence_barrier_init();
    }
    if constexpr (!kTf32) convert_projection(a.contrib_w, H, cout, sB, kSplit ? sBlo : nullptr, tid, kThreads);
    fence_proxy_async();  // the split B_w (and bf16 W_po) for the tensor cores
    if (warp == 0) tc::tmem_alloc(tmem_slot, tmem_cols);
    if constexpr (kTf32) {
        if (tid == 0) {
            tc::mbar_arrive_expect_tx(w_bar, (uint32_t)(kblocks * cout * 128));
            for (int kb = 0; kb < kblocks; ++kb)
                tc::tma_load_2d(sB + (size_t)kb * cout * 128, &map_w, w_bar, kb * kBk, 0);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp < kProducerWarps) {
        // ---------------- hidden producers + MMA issue ----------------
        // thread = edge row (TMEM lane) for one half of the hidden channels
        const int quarter = warp & 3;
        const int half = warp >> 2;
        const int row = quarter * 32 + lane;
        const int ch0 = half * hh;
        const uint32_t t_lane = (uint32_t)(quarter * 32) << 16;
        const int pl = row >> a.log2K;
        const int kk = row & (K - 1);
        // geometry of the first tile; later tiles' loads are issued one tile ahead
        bool valid = false;
        float4 xi = make_float4(0.f, 0.f, 0.f, 0.f), xj = xi;
        {
            const int p = blockIdx.x * a.ppt + pl;
            if (blockIdx.x < n_tiles && p < R) {
                valid = true;
                xi = *reinterpret_cast<const float4*>(a.xyz4 + (size_t)p * 4);
                const int jrow = (p / a.M) * a.M + a.idx[(size_t)p * K + kk];
                xj = *reinterpret_cast<const float4*>(a.xyz4 + (size_t)jrow * 4);
            }
        }
        // u = [rstd g, rstd, 1] of this row as tf32 hi / lo (the lanes of one
        // half), rstd = 1 / sqrt(var + 1e-5) of the row's pre-activations
        auto write_u = [&](const float4& pi, const float4& pj) {
            write_u_row(sU, sGram, row, pi, pj);
        };
        // pre = LN(W_in g + b_in) as the row product above, in 3xTF32 (hi hi +
        // hi lo + lo hi), into TMEM
        auto issue_pre = [&]() {
            const uint32_t u0 = tc::smem_u32(sU), w0 = tc::smem_u32(sWu);
            const uint64_t du = tc::interleaved_desc(u0, 128, 256);
            const uint64_t du_lo = tc::interleaved_desc(u0 + kUBytes, 128, 256);
            const uint64_t dw = tc::interleaved_desc(w0, 128, 256);
            const uint64_t dw_lo = tc::interleaved_desc(w0 + (uint32_t)H * 32, 128, 256);
            const uint32_t dpre = tmem_base + pre_col;
            tc::umma<true>(dpre, du, dw, a.idesc_pre, 0u);
            tc::umma<true>(dpre, du, dw_lo, a.idesc_pre, 1u);
            tc::umma<true>(dpre, du_lo, dw, a.idesc_pre, 1u);
            tc::umma_commit(pre_full);
        };
        // the first tile's pre-activations; later tiles' are issued with the
        // previous tile's main MMAs
        if (half == 0) {
            write_u(xi, xj);
            fence_proxy_async();
        }
        prod_barrier();
        if (tid == 0 && blockIdx.x < n_tiles) {
            tc::tc_fence_after();
            issue_pre();
        }
        bool weights_ready = !kTf32;
        int it = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
            const bool has_next = tile + (int)gridDim.x < n_tiles;
            // next tile: neighbour index and centre point now, the neighbour
            // point after the wait below
            const int np = (tile + gridDim.x) * a.ppt + pl;
            valid = has_next && np < R;
            int nidx = 0;
            if (valid) {
                nidx = a.idx[(size_t)np * K + kk];
                xi = *reinterpret_cast<const float4*>(a.xyz4 + (size_t)np * 4);
            }
            // wait until the MMAs of the tile that last used this A buffer are
            // done and this tile's pre-activations are in TMEM; one lane polls,
            // the other producer warps wait on the named barrier
            const int abuf = a.a_bufs == 2 ? (it & 1) : 0;
            const uint32_t round = a.a_bufs == 2 ? (uint32_t)(it >> 1) : (uint32_t)it;
            volatile int* fail = sProdFail + (it & 1);
            if (tid == 0 && !(tc::mbar_wait(&a_empty[abuf], (round & 1u) ^ 1u, a.err) &&
                              tc::mbar_wait(pre_full, (uint32_t)it & 1u, a.err)))
                *fail = 1;
            prod_barrier();
            if (*fail) break;
            tc::tc_fence_after();
            if (valid) xj = *reinterpret_cast<const float4*>(
                           a.xyz4 + (size_t)((np / a.M) * a.M + nidx) * 4);
            unsigned char* dA = sA + (size_t)abuf * a_buf_bytes;
            // GELU of the normalised pre-activations, packed as the main MMA
            // reads it (rows past the end hold finite values the epilogue
            // ignores)
            for (int c0 = 0; c0 < hh; c0 += 32) {
                float v[32];
                tc::tmem_ld32(tmem_base + t_lane + pre_col + (uint32_t)(ch0 + c0), v);
#pragma unroll
                for (int i0 = 0; i0 < 32; i0 += kPer) {
                    float2 o[kPer / 2];
#pragma unroll
                    for (int e = 0; e < kPer / 2; ++e)
                        o[e] = gelu_as2(make_float2(v[i0 + 2 * e], v[i0 + 2 * e + 1]));
                    const int c = ch0 + c0 + i0;
                    unsigned char* dst =
                        dA + (size_t)(c / kBk) * kRows * 128 + sw128_offset(row, (c % kBk) / kPer);
                    if constexpr (kTf32) {
                        *reinterpret_cast<float4*>(dst) = make_float4(o[0].x, o[0].y, o[1].x, o[1].y);
                    } else {
                        uint32_t hi[4], lo[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const __nv_bfloat162 h2 = __floats2bfloat162_rn(o[e].x, o[e].y);
                            hi[e] = *reinterpret_cast<const uint32_t*>(&h2);
                            if (kSplit) {
                                // o - hi exactly (Sterbenz), then rounded to bf16
                                const float2 hf = make_float2(__uint_as_float(hi[e] << 16),
                                                              __uint_as_float(hi[e] & 0xffff0000u));
                                const float2 r = fma2(hf, f2(-1.0f), o[e]);
                                lo[e] = pack_bf16(r.x, r.y);
                            }
                        }
                        *reinterpret_cast<uint4*>(dst) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        if (kSplit)
                            *reinterpret_cast<uint4*>(dst + a_bytes) =
                                make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    }
                }
            }
            // the next tile's u rows (its geometry has landed by now)
            if (half == 0 && has_next) write_u(xi, xj);
            fence_proxy_async();
            tc::tc_fence_before();  // this tile's pre-activations have been read
            prod_barrier();  // the whole A tile (and the next u) is written
            if (tid == 0) {
                // issue the tile's MMAs once its accumulator buffer is free; a
                // failure stops the producers at the next tile's decision
                const int tbuf = it & 1;
                const uint32_t tph = (uint32_t)(it >> 1) & 1u;
                bool ok = true;
                if (!weights_ready) {
                    ok = tc::mbar_wait(w_bar, 0, a.err);
                    if (!ok) tc::mbar_drain(w_bar, 0);
                    weights_ready = true;
                }
                ok = ok && tc::mbar_wait(&t_empty[tbuf], tph ^ 1u, a.err);
                if (ok) {
                    tc::tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(tbuf * cout);
                    const uint32_t a0 = tc::smem_u32(dA);
                    const uint32_t b0 = tc::smem_u32(sB), b_lo = tc::smem_u32(sBlo);
                    for (int kb = 0; kb < kblocks; ++kb) {
                        // the K block's descriptors once; K step k adds 32 bytes
                        // = 2 in the start-address field (address >> 4)
                        const uint64_t da0 = tc::sw128_desc(a0 + kb * kRows * 128);
                        const uint64_t db0 = tc::sw128_desc(b0 + kb * cout * 128);
                        const uint64_t dal0 = tc::sw128_desc(a0 + (uint32_t)a_bytes + kb * kRows * 128);
                        const uint64_t dbl0 = tc::sw128_desc(b_lo + kb * cout * 128);
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            if ((kb * kBk + k * (32 / kElem)) >= H) break;
                            tc::umma<kTf32>(d, da0 + 2 * k, db0 + 2 * k, a.idesc, (kb | k) ? 1u : 0u);
                            if (kSplit) {
                                tc::umma<false>(d, da0 + 2 * k, dbl0 + 2 * k, a.idesc, 1u);
                                tc::umma<false>(d, dal0 + 2 * k, db0 + 2 * k, a.idesc, 1u);
                            }
                        }
                    }
                    tc::umma_commit(&a_empty[abuf]);
                    tc::umma_commit(&t_full[tbuf]);
                    if (has_next) issue_pre();
                } else {
                    reinterpret_cast<volatile int*>(sProdFail)[(it + 1) & 1] = 1;
                }
            }
        }
        if (tid == 0) {
            // the weight copies and every MMA issued complete before the CTA
            // releases its shared and tensor memory
            if (!weights_ready) tc::mbar_drain(w_bar, 0);
            tc::umma_commit(mma_done);
            tc::mbar_drain(mma_done, 0);
        }
    } else {
        // ---------------- epilogue ----------------
        const int quarter = warp & 3;
        const int cpart = (warp - kEpiWarp0) >> 2;
        const int erow = quarter * 32 + lane;  // TMEM lane = edge row
        const int nchunks = cout / 32;
        const int kk = erow & (K - 1);
        const int ptw = lane >> a.log2K;    // point of this lane's edge row within the warp
        const int ppw = 32 >> a.log2K;      // points whose edge rows the warp holds
        // this warp's 32-channel chunks of a tile: cpart, cpart + 2, ...
        const int nmine = (nchunks - cpart + 1) >> 1;
        const int nbuf = a.stage_bufs < nmine ? a.stage_bufs : nmine;
        const uint32_t stage =
            tc::smem_u32(sStage) + (uint32_t)((warp - kEpiWarp0) * a.stage_bufs * a.stage_bytes);
        // neighbour row of this lane's edge row in tile t (-1 past the end)
        auto neighbour_row = [&](int t) -> int {
            const int p = t * a.ppt + (erow >> a.log2K);
            if (t >= n_tiles || p >= R) return -1;
            return (p / a.M) * a.M + a.idx[(size_t)p * K + kk];
        };
        int jcur = neighbour_row(blockIdx.x);
        int jnext = neighbour_row(blockIdx.x + gridDim.x);
        int it = 0;
        // Stage this warp's k-th chunk of tile `tile_s` (the current tile, or
        // the next one when `next`) into buffer b with coalesced 16-byte
        // copies: eight lanes per 128-byte row segment, four rows per
        // instruction, so a warp instruction touches 4 lines instead of 32.
        // One commit group per chunk (empty past the last tile), so `nbuf`
        // groups are always in flight before a wait.
        auto issue = [&](int tile_s, bool next, int k, int b) {
            if (tile_s < n_tiles) {
                const int ch = cpart + 2 * k;
                const int jl = max(next ? jnext : jcur, 0);
                const uint32_t buf = stage + (uint32_t)(b * a.stage_bytes);
                const int q = lane & 7;
                const float* src = a.content + ch * 32 + q * 4;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int r = 4 * i + (lane >> 3);
                    const int j = __shfl_sync(kFull, jl, r);
                    cp_async16(buf + (uint32_t)(r * 128 + ((q ^ (r & 7)) << 4)), src + (size_t)j * a.ldc);
                }
                const int pbase = tile_s * a.ppt + ((quarter * 32) >> a.log2K);
                for (int i = lane; i < ppw * 8; i += 32) {
                    const int pt = i >> 3, qq = i & 7;
                    const int p = pbase + pt < R ? pbase + pt : 0;
                    cp_async16(buf + (uint32_t)(4096 + pt * 128 + ((qq ^ (pt & 7)) << 4)),
                               a.content + (size_t)p * a.ldc + cout + ch * 32 + qq * 4);
                }
            }
            cp_async_commit();
        };
        // The content rows of a patch are first read by the tiles of that
        // patch in the same grid round, from DRAM when the matrix exceeds L2;
        // each CTA brings the rows of its points two rounds ahead into L2 (the
        // points of a round span a patch or more, so a patch's rows are in L2
        // before its tiles gather them).
        auto prefetch_rows = [&](int t) {
            if (t < n_tiles) {
                const int p = t * a.ppt;
                const int n = min(a.ppt, R - p);
                prefetch_l2(a.content + (size_t)p * a.ldc, (uint32_t)(n * a.ldc * 4));
            }
        };
        if (warp == kEpiWarp0 && lane == 0) {
            prefetch_rows(blockIdx.x);
            prefetch_rows(blockIdx.x + gridDim.x);
        }
        if (nmine > 0)
            for (int k = 0; k < nbuf; ++k) issue(blockIdx.x, false, k, k);
        int cons = 0;  // buffer of the next chunk to consume
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
            const int tbuf = it & 1;
            const uint32_t tph = (uint32_t)(it >> 1) & 1u;
            if (warp == kEpiWarp0 && lane == 0) prefetch_rows(tile + 2 * (int)gridDim.x);
            // one lane polls, the other epilogue warps wait on the named
            // barrier; the flag is next written after two more barriers of
            // this tile, so every warp reads this tile's decision
            if (warp == kEpiWarp0 && lane == 0 && !tc::mbar_wait(&t_full[tbuf], tph, a.err))
                *reinterpret_cast<volatile int*>(sEpiFail) = 1;
            epi_barrier();
            if (*reinterpret_cast<volatile int*>(sEpiFail)) break;
            tc::tc_fence_after();
            const int ep = tile * a.ppt + (erow >> a.log2K);
            const int ej = jcur;
            const uint32_t taddr =
                tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(tbuf * cout);
            // pass 1: message = content[j] + content[i] + (acc + b_po) -> TMEM,
            // content rows from the staging buffers, with the moments of this
            // warp's channels taken about the mean of its first chunk (one
            // pass; the two channel halves are combined below)
            float shift = 0.0f, s1 = 0.0f, s2 = 0.0f;
            for (int k = 0; k < nmine; ++k) {
                const int cb = (cpart + 2 * k) * 32;
                uint32_t r[32];
                tc::tmem_ld32_issue(taddr + (uint32_t)cb, r);
                cp_async_wait(nbuf - 1);
                __syncwarp();  // every lane's copies of this chunk have landed
                const uint32_t buf = stage + (uint32_t)(cons * a.stage_bytes);
                const uint32_t rj = buf + (uint32_t)(lane * 128);
                const uint32_t ri = buf + (uint32_t)(4096 + ptw * 128);
                tc::tmem_ld32_wait(r);
                float2 v2[16];
                float2 csum = f2(0.0f);
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    const float4 nj = lds128(rj + (uint32_t)(((i >> 2) ^ (lane & 7)) << 4));
                    const float4 ni = lds128(ri + (uint32_t)(((i >> 2) ^ (ptw & 7)) << 4));
                    const float4 bb = *reinterpret_cast<const float4*>(sCb + cb + i);
                    const float2 a0 = make_float2(__uint_as_float(r[i + 0]), __uint_as_float(r[i + 1]));
                    const float2 a1 = make_float2(__uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
                    v2[i / 2] = add2(add2(make_float2(nj.x, nj.y), make_float2(ni.x, ni.y)),
                                     add2(a0, make_float2(bb.x, bb.y)));
                    v2[i / 2 + 1] = add2(add2(make_float2(nj.z, nj.w), make_float2(ni.z, ni.w)),
                                         add2(a1, make_float2(bb.z, bb.w)));
                    if (k == 0) csum = add2(csum, add2(v2[i / 2], v2[i / 2 + 1]));
                }
                tc::tmem_st32_async(taddr + (uint32_t)cb, *reinterpret_cast<const float(*)[32]>(v2));
                if (k == 0) shift = (csum.x + csum.y) * (1.0f / 32.0f);
                const float2 nshift = f2(-shift);
                float2 s1p = f2(0.0f), s2p = f2(0.0f);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float2 d = add2(v2[i], nshift);
                    s1p = add2(s1p, d);
                    s2p = fma2(d, d, s2p);
                }
                s1 += s1p.x + s1p.y;
                s2 += s2p.x + s2p.y;
                __syncwarp();  // the buffer has been read: refill it
                const int kn = k + nbuf;
                if (kn < nmine) issue(tile, false, kn, cons);
                else issue(tile + (int)gridDim.x, true, kn - nmine, cons);
                cons = cons + 1 == nbuf ? 0 : cons + 1;
            }
            {
                // this half's mean and centred sum of squares (Chan et al.'s
                // pairwise update combines the halves)
                const float n_p = (float)(32 * nmine);
                const float m_p = nmine > 0 ? shift + s1 / n_p : 0.0f;
                const float q_p = nmine > 0 ? fmaxf(s2 - s1 * (s1 / n_p), 0.0f) : 0.0f;
                sStat[(2 * cpart) * kRows + erow] = m_p;
                sStat[(2 * cpart + 1) * kRows + erow] = q_p;
            }
            tc::tmem_st_wait();  // the messages are in TMEM before pass 3 reads them
            epi_barrier();
            const float n0 = (float)(32 * ((nchunks + 1) >> 1)), n1 = (float)(32 * (nchunks >> 1));
            const float m0 = sStat[erow], q0 = sStat[kRows + erow];
            const float m1 = sStat[2 * kRows + erow], q1 = sStat[3 * kRows + erow];
            const float dm = m1 - m0;
            const float mean = m0 + dm * (n1 / (float)cout);
            const float m2 = q0 + q1 + dm * dm * (n0 * n1 / (float)cout);
            const float rstd = rsqrtf(m2 / (float)cout + 1e-6f);
            const float nmr = -mean * rstd;
            // pass 3: max over the K lanes of each point of the normalised value,
            // then the affine + LeakyReLU once per point and channel. Both are
            // monotone (and rounding is monotone), so they commute exactly with
            // the max; a negative gain reverses the order, which the sign
            // folded into the normalised value undoes (|g| s n + b with s n
            // maximised).
            for (int ch = cpart; ch < nchunks; ch += 2) {
                const int cb = ch * 32;
                float y[32];
                tc::tmem_ld32(taddr + (uint32_t)cb, y);
                if (ej >= 0) {
                    const float2 rstd2 = f2(rstd), nmr2 = f2(nmr);
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        const float4 sg = *reinterpret_cast<const float4*>(sSgn + cb + i);
                        const float2 y0 = mul2(fma2(make_float2(y[i], y[i + 1]), rstd2, nmr2),
                                               make_float2(sg.x, sg.y));
                        const float2 y1 = mul2(fma2(make_float2(y[i + 2], y[i + 3]), rstd2, nmr2),
                                               make_float2(sg.z, sg.w));
                        y[i + 0] = y0.x;
                        y[i + 1] = y0.y;
                        y[i + 2] = y1.x;
                        y[i + 3] = y1.y;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) y[i] = -FLT_MAX;
                }
                int off = 0;
                if (K == 32) {
                    // one point per warp: a warp-wide max per channel; lane 0
                    // writes the 32 maxima to the warp's slots and lane c reads
                    // channel c back
                    float* red = sRed + (warp - kEpiWarp0) * 32;
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        float r[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r[e]) : "f"(y[i + e]));
                        if (lane == 0) *reinterpret_cast<float4*>(red + i) = make_float4(r[0], r[1], r[2], r[3]);
                    }
                    __syncwarp();
                    y[0] = red[lane];
                    __syncwarp();  // read before the next chunk's maxima overwrite the slots
                    off = lane;
                } else
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
                    for (int i = 0; i < 32; ++i) {
                        if (i < nv) {
                            const float2 gs = *reinterpret_cast<const float2*>(sLn + 2 * (cb + off + i));
                            const float t = fmaf(y[i], gs.x, gs.y);
                            o[i] = fmaxf(t, 0.2f * t);  // LeakyReLU(0.2)
                        }
                    }
                }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&t_empty[tbuf]);
            jcur = jnext;
            jnext = neighbour_row(tile + 2 * (int)gridDim.x);
        }
        cp_async_wait(0);  // no copy into shared memory outlives the loop
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, tmem_cols);
    }
}

// Shared memory of the kernel for `bufs` hidden-row buffers and `stage_bufs`
// content staging buffers of `stage_bytes` per epilogue warp.
size_t edge_tc_smem(int mode, int H, int cout, int bufs, int stage_bufs, int stage_bytes) {
    const int elem = mode == kModeTf32 ? 4 : 2;
    const size_t kblocks = (size_t)ceil_div(H, 128 / elem);
    const size_t copies = mode == kModeSplit ? 2 : 1;
    return 1024 + copies * kblocks * 128 * ((size_t)bufs * kRows + cout) + 2 * (size_t)kUBytes +
           2 * (size_t)H * 32 +
           sizeof(float) * ((size_t)H * 2 + 52 + (size_t)cout * 4 + 4 * kRows + kEpilogueWarps * 32) +
           128 + 128 + (size_t)kEpilogueWarps * stage_bufs * stage_bytes;
}

}  // namespace

// Tensor-core edge stage at `precision` (F2S_PRECISION_TF32, _BF16 or
// _BF16X3); returns F2S_ERR_UNSUPPORTED for shapes it does not cover (the
// caller then uses the CUDA-core kernel).
int edge_stage_tc(const EdgeArgs& e, int precision, cudaStream_t st) {
    if (e.B == 0 || e.M == 0) return F2S_OK;
    int log2K = 0;
    while ((1 << log2K) < e.K) ++log2K;
    // H: a multiple of 64 (each producer half reads 32-column TMEM chunks);
    // TMEM holds two C_out accumulators and the H pre-activations
    if (e.geometry != nullptr || e.xyz4 == nullptr || e.D != 6 || e.H > 128 || e.H % 64 != 0 ||
        e.cout % 32 != 0 || e.cout > 256 || 2 * e.cout + e.H > 512 || (1 << log2K) != e.K || e.K > 32 ||
        ((uintptr_t)e.content & 15) != 0 || e.ldc % 4 != 0 || ((uintptr_t)e.contrib_w & 15) != 0)
        return fail(F2S_ERR_UNSUPPORTED, "edge stage shape outside the tensor-core kernel");
    F2S_REQUIRE(precision == F2S_PRECISION_TF32 || precision == F2S_PRECISION_BF16 ||
                    precision == F2S_PRECISION_BF16X3,
                "edge_tc: precision %d", precision);
    if (precision == F2S_PRECISION_BF16X3) {
        const int status = edge_stage_unified(e, st);
        if (status != F2S_ERR_UNSUPPORTED) return status;
    }
    const int mode = precision == F2S_PRECISION_TF32   ? kModeTf32
                     : precision == F2S_PRECISION_BF16 ? kModeBf16
                                                       : kModeSplit;
    int* err = tc_error_word();
    if (!err) return fail(F2S_ERR_CUDA, "edge_tc: device error word unavailable");
    const bool tf32 = mode == kModeTf32;
    const int bk = tf32 ? 32 : 64;
    CUtensorMap map;
    if (tf32) F2S_TRY(make_tensor_map_2d(&map, e.contrib_w, true, e.cout, e.H, e.H, e.cout, bk));
    else memset(&map, 0, sizeof(map));
    // shared memory: as many content staging buffers per epilogue warp as
    // the warp has chunks per tile (at most 4), then two hidden-row buffers
    // if they still fit
    constexpr size_t kSmemLimit = 227 * 1024;
    const int stage_bytes = 4096 + (32 / e.K) * 128;
    const int stage_max = std::min((e.cout / 32 + 1) / 2, 4);
    int bufs = 0, stage_bufs = 0;
    size_t smem = 0;
    for (int sb = stage_max; sb >= 1 && bufs == 0; --sb)
        for (int ab = 2; ab >= 1 && bufs == 0; --ab)
            if (edge_tc_smem(mode, e.H, e.cout, ab, sb, stage_bytes) <= kSmemLimit) {
                bufs = ab;
                stage_bufs = sb;
                smem = edge_tc_smem(mode, e.H, e.cout, ab, sb, stage_bytes);
            }
    if (bufs == 0) return fail(F2S_ERR_UNSUPPORTED, "edge_tc: shape needs more shared memory");
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
    a.a_bufs = bufs;
    a.stage_bufs = stage_bufs;
    a.stage_bytes = stage_bytes;
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
    a.idesc_pre = tc::make_idesc(kRows, e.H, 2u);
    a.err = err;
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
