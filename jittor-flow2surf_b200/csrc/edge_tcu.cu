// Fused neighbour stage, split-bf16 precision, with every compute warp in both
// roles.
//
// Same arithmetic as edge_tc.cu (encoder.py:83-115, neighbor_reduce.py:244-337,
// hpe.py:14-50, hpe_hidden_forward.cu, neighbor_reduce_forward.cu): per edge
// row, the LayerNorm'd HPE pre-activations (a K = 8 3xTF32 MMA), GELU, the
// composed projection W_po h as hi*hi + hi*lo + lo*hi bf16 MMAs, the message
// content[j] + content[i] + W_po h + b_po, its LayerNorm, and the max over the
// K edge rows of each point after the affine + LeakyReLU.
//
// Work of a tile of 128 edge rows, per CTA (persistent, one per SM):
//   16 compute warps, four per TMEM lane quarter (edge rows 32q .. 32q + 31),
//   each owning a quarter of the hidden channels and a quarter of the output
//   channels. Per tile they
//     1. turn the pre-activations of the NEXT tile into hidden rows in place
//        in TMEM: each warp reads its H/4 fp32 columns, applies GELU and
//        writes the bf16 high and low halves over the same columns (the MMA
//        reads its A operand from tensor memory, so the hidden rows never
//        touch shared memory), then arrives on "A ready";
//     2. run the epilogue of THIS tile: the accumulator columns of the warp's
//        output channels go to registers at once (the accumulator is then
//        released to the next MMA), the neighbour and centre content rows
//        come from shared memory (staged by the warp's own cp.async copies a
//        whole tile ahead), the message moments of the four warps of a lane
//        quarter are combined through TMEM and a named barrier, and the
//        normalised messages are reduced over the K rows of each point.
//   1 control warp: computes the u rows [rstd g, rstd, 1] of the tile after
//   next from the geometry, issues the pre-activation MMAs (into the TMEM
//   slot the MMA of the tile before has released) and the main MMAs (one
//   lane; a tcgen05.mma holds its issuing thread until the tensor pipe takes
//   it, so no compute warp waits on that).
// So the tensor pipe runs the MMAs of tile t while the compute warps turn
// tile t + 1's pre-activations into hidden rows and finish tile t - 1: per
// tile the compute warps issue one GELU pass and one epilogue pass and wait
// on nothing else in steady state.
//
// TMEM columns: n_acc accumulators of C_out columns, two pre-activation /
// hidden-row slots of H columns, 16 columns of message moments.
#include <cfloat>
#include <cstring>

#include "edge_common.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace f2s {
namespace {

using namespace edge;

constexpr int kComputeWarps = 16;
constexpr int kControlWarp = kComputeWarps;
constexpr int kThreads = (kComputeWarps + 1) * 32;
constexpr unsigned kFull = 0xffffffffu;

struct UArgs {
    const float* content;
    int ldc;
    const float* xyz4;
    const int32_t* idx;
    int B, M, K, log2K, H, cout;
    int ppt;    // points per tile (128 / K)
    int n_acc;  // TMEM accumulators (1 or 2)
    uint32_t tmem_cols;
    const float* hpe_w;
    const float* hpe_b;
    const float* hpe_ln_w;
    const float* hpe_ln_b;
    const float* contrib_b;
    const float* contrib_w;
    const float* ln_w;
    const float* ln_b;
    float* out;
    int ldo;
    uint32_t idesc;      // bf16 operands, M = 128, N = C_out
    uint32_t idesc_pre;  // tf32, M = 128, N = H
    int* err;
};

// Shared-memory layout (byte offsets from the 1024-byte aligned base).
struct Layout {
    uint32_t b_hi, b_lo, u, wu, gram, cb, ln, sgn, bars, fails, stage;
    uint32_t stage_bytes;  // per compute warp: 32 neighbour rows + the centre rows of its points
    uint32_t total;
};

__host__ __device__ inline Layout layout(int H, int cout, int K) {
    Layout L{};
    const uint32_t cw = (uint32_t)cout / 4;  // output channels of one compute warp
    const uint32_t ppw = 32u / (uint32_t)K;  // points whose rows one warp holds
    const uint32_t b_bytes = (uint32_t)cout * (uint32_t)H * 2u;
    L.b_hi = 0;
    L.b_lo = b_bytes;
    L.u = 2 * b_bytes;
    L.wu = L.u + 2 * kUBytes;
    L.gram = L.wu + 2u * (uint32_t)H * 32u;
    L.cb = L.gram + 64 * 4;
    L.ln = L.cb + (uint32_t)cout * 4;
    L.sgn = L.ln + (uint32_t)cout * 8;
    L.bars = (L.sgn + (uint32_t)cout * 4 + 7) & ~7u;
    L.fails = L.bars + 16 * 8 + 8;
    L.stage = (L.fails + 2 * kComputeWarps * 4 + 127) & ~127u;
    L.stage_bytes = 32u * cw * 4u + ppw * cw * 4u;
    L.total = L.stage + kComputeWarps * L.stage_bytes;
    return L;
}

// 16-byte chunk position of chunk c of staged row r (rows of nc chunks): XOR
// swizzles under which the eight lanes of one quarter-warp phase, reading
// chunk c of eight consecutive rows, hit eight distinct 16-byte bank groups
// for row pitches of 4, 8 and 12 chunks.
__device__ __forceinline__ int stage_swizzle(int r, int c, int nc) {
    if (nc >= 8 && c < 8) return c ^ (r & 7);
    const int base = nc >= 8 ? 8 : 0;
    return base + ((c - base) ^ ((r >> 1) & 3));
}

__device__ __forceinline__ void quarter_barrier(int q) {
    asm volatile("bar.sync %0, 128;" ::"r"(q + 1) : "memory");
}

// Bounded mbarrier wait by lane 0 of the warp, result shared by the warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int lane) {
    int ok = 1;
    if (lane == 0) ok = tc::mbar_wait_spin(bar, parity, err) ? 1 : 0;
    return __shfl_sync(kFull, ok, 0) != 0;
}

template <int kNch, bool kK32>
__global__ void __launch_bounds__(kThreads, 1)
edge_unified_kernel(const UArgs a) {
    extern __shared__ __align__(1024) unsigned char edge_u_smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(edge_u_smem_raw) + 1023) & ~uintptr_t(1023));
    const int H = a.H, cout = a.cout, K = a.K;
    const Layout L = layout(H, cout, K);
    unsigned char* sB = smem + L.b_hi;
    unsigned char* sBlo = smem + L.b_lo;
    unsigned char* sU = smem + L.u;
    unsigned char* sWu = smem + L.wu;
    float* sGram = reinterpret_cast<float*>(smem + L.gram);
    float* sCb = reinterpret_cast<float*>(smem + L.cb);
    float* sLn = reinterpret_cast<float*>(smem + L.ln);
    float* sSgn = reinterpret_cast<float*>(smem + L.sgn);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint64_t* pre_full = bars + 0;   // [2] pre-activations of a slot's tile in TMEM
    uint64_t* a_ready = bars + 2;    // [2] hidden rows of a slot written (16 arrivals)
    uint64_t* slot_free = bars + 4;  // [2] the MMAs reading a slot are done
    uint64_t* acc_full = bars + 6;   // [2] accumulator holds its tile
    uint64_t* acc_free = bars + 8;   // [2] accumulator read out (16 arrivals)
    uint64_t* mma_done = bars + 10;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
    volatile int* sFail = reinterpret_cast<volatile int*>(smem + L.fails);  // [2][16]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int R = a.B * a.M;
    const int n_tiles = (R + a.ppt - 1) / a.ppt;
    const uint32_t slot_col0 = (uint32_t)(a.n_acc * cout);
    const uint32_t stat_col = slot_col0 + 2u * (uint32_t)H;

    // ---- per-CTA preparation (the staging area doubles as set-up scratch) ----
    prepare_pre_activation(a.hpe_w, a.hpe_b, a.hpe_ln_w, a.hpe_ln_b, H,
                           reinterpret_cast<double*>(smem + L.stage), sWu, sGram, tid, kThreads);
    prepare_message_norm(a.contrib_b, a.ln_w, a.ln_b, cout, sCb, sLn, sSgn, tid, kThreads);
    convert_projection(a.contrib_w, H, cout, sB, sBlo, tid, kThreads);
    if (tid == 0) {
        for (int s = 0; s < 2; ++s) {
            tc::mbar_init(&pre_full[s], 1);
            tc::mbar_init(&a_ready[s], kComputeWarps);
            tc::mbar_init(&slot_free[s], 1);
            tc::mbar_init(&acc_full[s], 1);
            tc::mbar_init(&acc_free[s], kComputeWarps);
        }
        tc::mbar_init(mma_done, 1);
        tc::fence_barrier_init();
    }
    if (tid < 2 * kComputeWarps) sFail[tid] = 0;
    fence_proxy_async();  // the weights written above, for the tensor cores
    if (warp == kControlWarp) tc::tmem_alloc(tmem_slot, a.tmem_cols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == kControlWarp) {
        // ---------------- control: u rows, pre-activation and main MMAs ----------------
        // geometry of the four rows this lane computes u for (rows lane + 32 m),
        // fetched in two stages a tile apart so that no load waits on another:
        // stage 1 reads the neighbour indices and centre points of a tile,
        // stage 2 (one tile later) the neighbour points they name
        float4 gi[4], gj[4], ni[4];
        int nj[4];
        bool gvalid[4], nvalid[4];
        auto fetch_indices = [&](int t) {
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int row = lane + 32 * m;
                const int p = t * a.ppt + (row >> a.log2K);
                nvalid[m] = t < n_tiles && p < R;
                const int pc = nvalid[m] ? p : 0;
                ni[m] = *reinterpret_cast<const float4*>(a.xyz4 + (size_t)pc * 4);
                nj[m] = (pc / a.M) * a.M + a.idx[(size_t)pc * K + (row & (K - 1))];
            }
        };
        auto fetch_points = [&]() {
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                gi[m] = ni[m];
                gj[m] = *reinterpret_cast<const float4*>(a.xyz4 + (size_t)nj[m] * 4);
                gvalid[m] = nvalid[m];
            }
        };
        auto load_geometry = [&](int t) {  // both stages at once (start-up only)
            fetch_indices(t);
            fetch_points();
        };
        auto write_u = [&]() {
            const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int m = 0; m < 4; ++m)
                write_u_row(sU, sGram, lane + 32 * m, gvalid[m] ? gi[m] : zero,
                            gvalid[m] ? gj[m] : zero);
            fence_proxy_async();
            __syncwarp();
        };
        // pre = LN(W_in g + b_in) of the tile whose u rows are in sU, into slot s
        auto issue_pre = [&](int s) {
            const uint32_t u0 = tc::smem_u32(sU), w0 = tc::smem_u32(sWu);
            const uint64_t du = tc::interleaved_desc(u0, 128, 256);
            const uint64_t du_lo = tc::interleaved_desc(u0 + kUBytes, 128, 256);
            const uint64_t dw = tc::interleaved_desc(w0, 128, 256);
            const uint64_t dw_lo = tc::interleaved_desc(w0 + (uint32_t)H * 32, 128, 256);
            const uint32_t d = tmem_base + slot_col0 + (uint32_t)(s * H);
            tc::umma<true>(d, du, dw, a.idesc_pre, 0u);
            tc::umma<true>(d, du, dw_lo, a.idesc_pre, 1u);
            tc::umma<true>(d, du_lo, dw, a.idesc_pre, 1u);
            tc::umma_commit(&pre_full[s]);
        };
        const int hq = H / 4, steps_per_part = hq / 16;
        // W_po h of the tile in slot s into accumulator acc: per K step of 16
        // channels hi*hi + hi*lo + lo*hi, A (the hidden rows) from TMEM
        auto issue_main = [&](int s, int acc) {
            const uint32_t d = tmem_base + (uint32_t)(acc * cout);
            const uint32_t b0 = tc::smem_u32(sB), b1 = tc::smem_u32(sBlo);
            for (int k = 0; k < H / 16; ++k) {
                const int part = k / steps_per_part, j = k - part * steps_per_part;
                const uint32_t hi_col =
                    tmem_base + slot_col0 + (uint32_t)(s * H + part * hq + j * 8);
                const uint32_t lo_col = hi_col + (uint32_t)(hq / 2);
                const int kb = k >> 2, w = k & 3;
                const uint64_t db_hi = tc::sw128_desc(b0 + (uint32_t)(kb * cout * 128)) + 2 * w;
                const uint64_t db_lo = tc::sw128_desc(b1 + (uint32_t)(kb * cout * 128)) + 2 * w;
                tc::umma_tmem_a_f16(d, hi_col, db_hi, a.idesc, k > 0 ? 1u : 0u);
                tc::umma_tmem_a_f16(d, hi_col, db_lo, a.idesc, 1u);
                tc::umma_tmem_a_f16(d, lo_col, db_hi, a.idesc, 1u);
            }
        };
        bool ok = true;
        const int t0 = blockIdx.x, t1 = blockIdx.x + (int)gridDim.x;
        load_geometry(t0);
        write_u();
        if (lane == 0) issue_pre(0);
        load_geometry(t1);
        if (t1 < n_tiles) {
            ok = warp_wait(&pre_full[0], 0, a.err, lane);  // sU read by pre(t0)
            if (ok) {
                write_u();
                if (lane == 0) issue_pre(1);
            }
        }
        load_geometry(t1 + (int)gridDim.x);        // tile index 2
        fetch_indices(t1 + 2 * (int)gridDim.x);    // tile index 3, stage 1
        // per tile index it: the u rows of tile it + 2 (its geometry loaded
        // one iteration earlier) while the compute warps still produce the
        // hidden rows of tile it, then MMA(it), then the pre-activations of
        // tile it + 2 into the slot MMA(it) has released
        for (int it = 0; ok; ++it) {
            const int tile = blockIdx.x + it * (int)gridDim.x;
            if (tile >= n_tiles) break;
            const int s = it & 1, acc = it % a.n_acc;
            const int tile2 = tile + 2 * (int)gridDim.x;
            if (tile2 < n_tiles) {
                ok = warp_wait(&pre_full[s ^ 1], (uint32_t)((it + 1) >> 1) & 1u, a.err, lane);
                if (!ok) break;
                write_u();
                fetch_points();                               // tile index it + 3
                fetch_indices(tile2 + 2 * (int)gridDim.x);    // tile index it + 4
            }
            int good = 1;
            if (lane == 0) {
                good = tc::mbar_wait_spin(&a_ready[s], (uint32_t)(it >> 1) & 1u, a.err);
                if (good && it >= a.n_acc)
                    good = tc::mbar_wait_spin(&acc_free[acc], ((uint32_t)(it / a.n_acc) & 1u) ^ 1u,
                                              a.err);
                if (good) {
                    tc::tc_fence_after();
                    issue_main(s, acc);
                    tc::umma_commit(&slot_free[s]);
                    tc::umma_commit(&acc_full[acc]);
                }
            }
            ok = __shfl_sync(kFull, good, 0) != 0;
            if (!ok || tile2 >= n_tiles) continue;
            ok = warp_wait(&slot_free[s], (uint32_t)(it >> 1) & 1u, a.err, lane);
            if (ok && lane == 0) {
                tc::tc_fence_after();
                issue_pre(s);
            }
        }
        if (lane == 0) {
            // every MMA issued completes before the CTA frees its memory
            tc::umma_commit(mma_done);
            tc::mbar_drain(mma_done, 0);
        }
    } else {
        // ---------------- compute warps ----------------
        const int q = warp & 3, part = warp >> 2;
        const int erow = q * 32 + lane;  // TMEM lane = edge row
        const int kk = erow & (K - 1);
        const int ptw = lane >> a.log2K;  // this lane's point within the warp's points
        const int ppw = 32 >> a.log2K;
        constexpr int nch = kNch, cw = 16 * kNch, nc = cw / 4;
        const int ch0 = part * cw;
        const int hq = H / 4;
        const uint32_t lane_off = tmem_base + ((uint32_t)(q * 32) << 16);
        const uint32_t stage = tc::smem_u32(smem + L.stage) + (uint32_t)warp * L.stage_bytes;
        const uint32_t centre = stage + 32u * (uint32_t)cw * 4u;
        auto neighbour_row = [&](int t) -> int {
            const int p = t * a.ppt + (erow >> a.log2K);
            if (t >= n_tiles || p >= R) return -1;
            return (p / a.M) * a.M + a.idx[(size_t)p * K + kk];
        };
        // this warp's content of tile t: the neighbour rows (channels
        // [ch0, ch0 + cw)) of its 32 edge rows and the centre rows
        // (channels cout + [ch0, ch0 + cw)) of its points; one commit group
        auto issue_stage = [&](int t, int jrow) {
            if (t < n_tiles) {
                const int jl = max(jrow, 0);
                const float* src0 = a.content + ch0;
                for (int i = lane; i < 32 * nc; i += 32) {
                    const int r = i / nc, c = i - r * nc;
                    const int j = __shfl_sync(kFull, jl, r);
                    cp_async16(stage + (uint32_t)(r * cw * 4 + stage_swizzle(r, c, nc) * 16),
                               src0 + (size_t)j * a.ldc + c * 4);
                }
                const int pbase = t * a.ppt + ((q * 32) >> a.log2K);
                for (int i = lane; i < ppw * nc; i += 32) {
                    const int pt = i / nc, c = i - pt * nc;
                    const int p = pbase + pt < R ? pbase + pt : 0;
                    cp_async16(centre + (uint32_t)(pt * cw * 4 + c * 16),
                               src0 + (size_t)p * a.ldc + cout + c * 4);
                }
            }
            cp_async_commit();
        };
        // hidden rows of tile index it into slot it & 1
        auto gelu_tile = [&](int it) -> bool {
            const int s = it & 1;
            if (!warp_wait(&pre_full[s], (uint32_t)(it >> 1) & 1u, a.err, lane)) return false;
            tc::tc_fence_after();
            const uint32_t col = lane_off + slot_col0 + (uint32_t)(s * H + part * hq);
            // all of this warp's pre-activations are read before any hidden
            // row is written over them (the low halves of the first 16
            // channels land where the pre-activations of the next 16 were)
            uint32_t r[2][16];
            tc::tmem_ld<16>(col, r[0]);
            if (hq > 16) tc::tmem_ld<16>(col + 16u, r[1]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (h * 16 >= hq) break;
                uint32_t hi[8], lo[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float2 o = gelu_as2(
                        make_float2(__uint_as_float(r[h][2 * e]), __uint_as_float(r[h][2 * e + 1])));
                    const __nv_bfloat162 h2 = __floats2bfloat162_rn(o.x, o.y);
                    hi[e] = *reinterpret_cast<const uint32_t*>(&h2);
                    const float2 hf = make_float2(__uint_as_float(hi[e] << 16),
                                                  __uint_as_float(hi[e] & 0xffff0000u));
                    const float2 rem = fma2(hf, f2(-1.0f), o);  // o - hi, exact
                    lo[e] = pack_bf16(rem.x, rem.y);
                }
                // channels 16h .. 16h + 15 of this warp's hq: packed columns
                // 8h .. 8h + 7 of its high half, hq / 2 later the low half
                tc::tmem_st_async<8>(col + (uint32_t)(8 * h), hi);
                tc::tmem_st_async<8>(col + (uint32_t)(hq / 2 + 8 * h), lo);
            }
            tc::tmem_st_wait();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&a_ready[s]);
            return true;
        };

        int jcur = neighbour_row(blockIdx.x);
        issue_stage(blockIdx.x, jcur);
        // a failed wait is carried to the next moment exchange, where the
        // four warps of the lane quarter stop together (each warp reaches the
        // quarter's named barrier once per tile until then)
        bool ok = gelu_tile(0);
        for (int it = 0;; ++it) {
            const int tile = blockIdx.x + it * (int)gridDim.x;
            if (tile >= n_tiles) break;
            const int next = tile + (int)gridDim.x;
            if (ok && next < n_tiles) ok = gelu_tile(it + 1);
            // ---- epilogue of tile it ----
            const int acc = it % a.n_acc;
            const uint32_t rj = stage + (uint32_t)(lane * cw * 4);  // this lane's staged row
            const uint32_t ri = centre + (uint32_t)(ptw * cw * 4);
            if (ok) ok = warp_wait(&acc_full[acc], (uint32_t)(it / a.n_acc) & 1u, a.err, lane);
            if (ok) {
                tc::tc_fence_after();
                cp_async_wait(0);
                __syncwarp();  // every lane's copies of this tile have landed
                // message = (content[j] + content[i]) + (acc + b_po), written back
                // over the lane's own staged row (same chunk positions); moments
                // about the mean of the first 16 channels, in one pass
                const uint32_t acol = lane_off + (uint32_t)(acc * cout + ch0);
                float shift = 0.0f;
                float2 s1p = f2(0.0f), s2p = f2(0.0f);
#pragma unroll
                for (int k = 0; k < nch; ++k) {
                    uint32_t r[16];
                    tc::tmem_ld<16>(acol + (uint32_t)(16 * k), r);
                    float2 m[8];
                    float2 csum = f2(0.0f);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const int c = 4 * k + q4;
                        const uint32_t pos = rj + (uint32_t)(stage_swizzle(lane, c, nc) * 16);
                        const float4 nj = lds128(pos);
                        const float4 ni = lds128(ri + (uint32_t)(c * 16));
                        const float4 bb = *reinterpret_cast<const float4*>(sCb + ch0 + 4 * c);
                        m[2 * q4] = add2(add2(make_float2(nj.x, nj.y), make_float2(ni.x, ni.y)),
                                         add2(make_float2(__uint_as_float(r[4 * q4]),
                                                          __uint_as_float(r[4 * q4 + 1])),
                                              make_float2(bb.x, bb.y)));
                        m[2 * q4 + 1] = add2(add2(make_float2(nj.z, nj.w), make_float2(ni.z, ni.w)),
                                             add2(make_float2(__uint_as_float(r[4 * q4 + 2]),
                                                              __uint_as_float(r[4 * q4 + 3])),
                                                  make_float2(bb.z, bb.w)));
                        sts128(pos, make_float4(m[2 * q4].x, m[2 * q4].y, m[2 * q4 + 1].x,
                                                m[2 * q4 + 1].y));
                        csum = add2(csum, add2(m[2 * q4], m[2 * q4 + 1]));
                    }
                    if (k == 0) shift = (csum.x + csum.y) * (1.0f / 16.0f);
                    const float2 ns = f2(-shift);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float2 d = add2(m[i], ns);
                        s1p = add2(s1p, d);
                        s2p = fma2(d, d, s2p);
                    }
                }
                // the accumulator has been read: the next tile's MMA may use it
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&acc_free[acc]);
                const float s1 = s1p.x + s1p.y, s2 = s2p.x + s2p.y;
                // this warp's mean and centred sum of squares over its cw channels
                const float n_p = (float)cw;
                const uint32_t st[2] = {__float_as_uint(shift + s1 / n_p),
                                        __float_as_uint(fmaxf(s2 - s1 * (s1 / n_p), 0.0f))};
                tc::tmem_st_async<2>(lane_off + stat_col + (uint32_t)((it & 1) * 8 + part * 2), st);
                tc::tmem_st_wait();
            }
            if (lane == 0) sFail[(it & 1) * kComputeWarps + warp] = ok ? 0 : 1;
            tc::tc_fence_before();
            quarter_barrier(q);
            tc::tc_fence_after();
            bool quarter_ok = true;
#pragma unroll
            for (int p = 0; p < 4; ++p) quarter_ok &= sFail[(it & 1) * kComputeWarps + q + 4 * p] == 0;
            if (!quarter_ok) break;
            // the four warps' moments, combined pairwise (Chan et al.)
            uint32_t stats[8];
            tc::tmem_ld<8>(lane_off + stat_col + (uint32_t)((it & 1) * 8), stats);
            float mean = 0.0f;
#pragma unroll
            for (int p = 0; p < 4; ++p) mean += __uint_as_float(stats[2 * p]);
            mean *= 0.25f;
            float m2 = 0.0f;
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const float dm = __uint_as_float(stats[2 * p]) - mean;
                m2 += __uint_as_float(stats[2 * p + 1]) + (float)cw * dm * dm;
            }
            const float rstd = rsqrtf(m2 / (float)cout + 1e-6f);
            const float nmr = -mean * rstd;
            const int ep = tile * a.ppt + (erow >> a.log2K);
            const bool valid_row = jcur >= 0;
            // normalised message times the sign of the gain; its max over the
            // K rows of a point, then |gain| x + shift and LeakyReLU(0.2)
            const float2 rstd2 = f2(rstd), nmr2 = f2(nmr);
            auto normalised = [&](int k, float (&y)[16]) {
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const int c = 4 * k + q4;
                    const float4 mv = lds128(rj + (uint32_t)(stage_swizzle(lane, c, nc) * 16));
                    const float4 sg = *reinterpret_cast<const float4*>(sSgn + ch0 + 4 * c);
                    const float2 y0 = mul2(fma2(make_float2(mv.x, mv.y), rstd2, nmr2),
                                           make_float2(sg.x, sg.y));
                    const float2 y1 = mul2(fma2(make_float2(mv.z, mv.w), rstd2, nmr2),
                                           make_float2(sg.z, sg.w));
                    y[4 * q4 + 0] = valid_row ? y0.x : -FLT_MAX;
                    y[4 * q4 + 1] = valid_row ? y0.y : -FLT_MAX;
                    y[4 * q4 + 2] = valid_row ? y1.x : -FLT_MAX;
                    y[4 * q4 + 3] = valid_row ? y1.y : -FLT_MAX;
                }
            };
            if constexpr (kK32) {
                // one point per warp: warp-wide maxima; lane 0 parks those of
                // chunk k over the staged row 0 positions of chunk k (lane 0's
                // own row, already read) and lane c stores channel c
                float* red = reinterpret_cast<float*>(smem + L.stage + (size_t)warp * L.stage_bytes);
#pragma unroll
                for (int k = 0; k < nch; ++k) {
                    float y[16];
                    normalised(k, y);
#pragma unroll
                    for (int i = 0; i < 16; i += 4) {
                        float r4[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r4[e]) : "f"(y[i + e]));
                        if (lane == 0)
                            *reinterpret_cast<float4*>(red + 16 * k + i) =
                                make_float4(r4[0], r4[1], r4[2], r4[3]);
                    }
                }
                __syncwarp();
                if (ep < R) {
                    for (int c = lane; c < cw; c += 32) {
                        const float2 gs = *reinterpret_cast<const float2*>(sLn + 2 * (ch0 + c));
                        const float t = fmaf(red[c], gs.x, gs.y);
                        a.out[(size_t)ep * a.ldo + ch0 + c] = fmaxf(t, 0.2f * t);
                    }
                }
                __syncwarp();  // the maxima are read before the next copies land there
            } else {
                // K < 32: a butterfly over the K lanes of each point leaves
                // 16 / K channels of each 16-channel chunk per lane
#pragma unroll
                for (int k = 0; k < nch; ++k) {
                    float y[16];
                    normalised(k, y);
                    int off = 0;
#pragma unroll
                    for (int sdx = 0; sdx < 4; ++sdx) {
                        if (sdx < a.log2K) {
                            const int msk = K >> (sdx + 1);
                            const bool hi = (lane & msk) != 0;
                            const int h = 8 >> sdx;
#pragma unroll
                            for (int i = 0; i < h; ++i) {
                                const float send = hi ? y[i] : y[h + i];
                                const float keep = hi ? y[h + i] : y[i];
                                y[i] = fmaxf(keep, __shfl_xor_sync(kFull, send, msk));
                            }
                            off += hi ? h : 0;
                        }
                    }
                    if (ep < R) {
                        const int nv = 16 >> a.log2K;
                        float* o = a.out + (size_t)ep * a.ldo + ch0 + 16 * k + off;
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            if (i < nv) {
                                const float2 gs = *reinterpret_cast<const float2*>(
                                    sLn + 2 * (ch0 + 16 * k + off + i));
                                const float t = fmaf(y[i], gs.x, gs.y);
                                o[i] = fmaxf(t, 0.2f * t);
                            }
                        }
                    }
                }
                __syncwarp();
            }
            // this tile's staging has been read: bring in the next tile's
            jcur = neighbour_row(next);
            issue_stage(next, jcur);
        }
        cp_async_wait(0);  // no copy into shared memory outlives the loop
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == kControlWarp) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, a.tmem_cols);
    }
}

}  // namespace

// The split-bf16 neighbour stage on the unified kernel when its shape allows:
// H in {64, 128}, C_out in {64, 128, 192}, K in {8, 16, 32}, xyz4 geometry;
// F2S_ERR_UNSUPPORTED otherwise (the caller then uses edge_tc_kernel).
int edge_stage_unified(const EdgeArgs& e, cudaStream_t st) {
    if (e.B == 0 || e.M == 0) return F2S_OK;
    int log2K = 0;
    while ((1 << log2K) < e.K) ++log2K;
    if (e.geometry != nullptr || e.xyz4 == nullptr || e.D != 6 || (e.H != 64 && e.H != 128) ||
        (e.cout != 64 && e.cout != 128 && e.cout != 192) || (1 << log2K) != e.K || e.K < 8 ||
        e.K > 32 || ((uintptr_t)e.content & 15) != 0 || e.ldc % 4 != 0 ||
        ((uintptr_t)e.contrib_w & 15) != 0)
        return fail(F2S_ERR_UNSUPPORTED, "edge stage shape outside the unified kernel");
    int* err = tc_error_word();
    if (!err) return fail(F2S_ERR_CUDA, "edge_unified: device error word unavailable");
    const Layout L = layout(e.H, e.cout, e.K);
    const size_t smem = (size_t)L.total + 1024;
    if (smem > 227 * 1024) return fail(F2S_ERR_UNSUPPORTED, "edge_unified: shared memory");
    UArgs a{};
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
    a.n_acc = 2 * e.cout + 2 * e.H + 16 <= 512 ? 2 : 1;
    const int cols = a.n_acc * e.cout + 2 * e.H + 16;
    uint32_t tcols = 32;
    while (tcols < (uint32_t)cols) tcols <<= 1;
    a.tmem_cols = tcols;
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
    a.idesc = tc::make_idesc(kRows, e.cout, 1u);
    a.idesc_pre = tc::make_idesc(kRows, e.H, 2u);
    a.err = err;
    const int R = e.B * e.M;
    const int tiles = ceil_div(R, a.ppt);
    const int grid = tiles < sm_count() ? tiles : sm_count();
    TraceScope trace(kTagEdge, st);
    auto launch = [&](auto kernel) -> int {
        F2S_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
        kernel<<<grid, kThreads, smem, st>>>(a);
        return check_launch("edge_unified_kernel");
    };
    const bool k32 = e.K == 32;
    switch (e.cout / 64) {
        case 1: return k32 ? launch(edge_unified_kernel<1, true>) : launch(edge_unified_kernel<1, false>);
        case 2: return k32 ? launch(edge_unified_kernel<2, true>) : launch(edge_unified_kernel<2, false>);
        default: return k32 ? launch(edge_unified_kernel<3, true>) : launch(edge_unified_kernel<3, false>);
    }
}

}  // namespace f2s
