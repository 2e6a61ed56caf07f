// Fused neighbour stage, split-bf16 precision, as three concurrent roles.
//
// Same arithmetic as edge_tc.cu (encoder.py:83-115, neighbor_reduce.py:244-337,
// hpe.py:14-50, hpe_hidden_forward.cu, neighbor_reduce_forward.cu): per edge
// row, the LayerNorm'd HPE pre-activations (a K = 8 3xTF32 MMA), GELU, the
// composed projection W_po h as hi*hi + hi*lo + lo*hi bf16 MMAs, the message
// content[j] + content[i] + W_po h + b_po, its LayerNorm, and the max over the
// K edge rows of each point after the affine + LeakyReLU.
//
// Persistent CTA (one per SM) over tiles of 128 edge rows, 20 warps:
//   warps 0-7   hidden rows: two warps per TMEM lane quarter, each half of the
//               hidden channels. A warp turns the fp32 pre-activations of a
//               tile into GELU'd bf16 high and low halves in place in TMEM
//               (each 16-channel chunk: high halves in its first 8 columns,
//               low halves in the next 8), the A operand the MMA reads from
//               tensor memory; the hidden rows never touch shared memory.
//   warps 8-15  epilogue: two warps per lane quarter, each half of the output
//               channels. The accumulator goes through registers once (then
//               the next MMA may use it), with the neighbour and centre
//               content rows staged in shared memory by the warp's own
//               cp.async copies a whole tile ahead; the messages are written
//               back over the consumed staged rows, the two halves' moments
//               meet through TMEM and a named barrier, and the normalised
//               messages are reduced over the K rows of each point.
//   warps 16-19 control: warps 16-18 compute the u rows [rstd g, rstd, 1]
//               two tiles ahead (geometry prefetched a further tile ahead);
//               lane 0 of warp 19 issues the pre-activation MMAs into the
//               TMEM slot the MMA before has released and the main MMAs (a
//               tcgen05.mma holds its issuing thread until the tensor pipe
//               takes it, so no other role waits on that).
// The hidden-row warps (MUFU-heavy GELU), the epilogue warps (FMA, shared
// memory) and the tensor pipe work on consecutive tiles at once.
//
// TMEM columns: n_acc accumulators of C_out columns, two pre-activation /
// hidden-row slots of H columns, 8 columns of message moments.
#include <cfloat>
#include <cstring>

#include "edge_common.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace f2s {
namespace {

using namespace edge;

constexpr int kHiddenWarps = 8;
constexpr int kEpilogueWarps = 8;
constexpr int kEpiWarp0 = kHiddenWarps;
constexpr int kControlWarp0 = kHiddenWarps + kEpilogueWarps;
constexpr int kControlWarps = 4;  // three u-row writers and the MMA issuer
constexpr int kWriterWarps = 3;
constexpr int kThreads = (kControlWarp0 + kControlWarps) * 32;
constexpr unsigned kFull = 0xffffffffu;

struct UArgs {
    const float* content;
    int ldc;
    const float* xyz4;      // (B*M, 4) points, or null with geometry
    const float* geometry;  // (B*M*K, 6) explicit g = [x_j - x_i, x_i], or null
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
    uint32_t b_hi, b_lo, u, wu, gram, cb, ln, sgn, bars, fails, rn, stage;
    uint32_t stage_bytes;  // per epilogue warp: 32 neighbour rows + the centre rows of its points
    uint32_t total;
};

__host__ __device__ inline Layout layout(int H, int cout, int K) {
    Layout L{};
    const uint32_t cw = (uint32_t)cout / 2;  // output channels of one epilogue warp
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
    // per epilogue warp, its 32 rows' (rstd, -mean rstd) for the column pass
    L.rn = (L.fails + 2 * kEpilogueWarps * 4 + 16 + 15) & ~15u;
    L.stage = (L.rn + kEpilogueWarps * 32 * 8 + 127) & ~127u;
    L.stage_bytes = 32u * cw * 4u + ppw * cw * 4u;
    L.total = L.stage + kEpilogueWarps * L.stage_bytes;
    return L;
}

// 16-byte chunk position of chunk c of staged row r (rows of a multiple of 8
// chunks, i.e. of 128 bytes): XOR within each 8-chunk block, so the eight
// lanes of a quarter-warp phase reading chunk c of eight consecutive rows hit
// eight distinct 16-byte bank groups.
__device__ __forceinline__ int stage_swizzle(int r, int c) { return (c & ~7) | ((c ^ r) & 7); }

// The two epilogue warps of lane quarter q.
__device__ __forceinline__ void quarter_barrier(int q) {
    asm volatile("bar.sync %0, 64;" ::"r"(q + 1) : "memory");
}

// Bounded mbarrier wait by lane 0 of the warp, result shared by the warp;
// kPoll waits without the suspend hint (the control warps).
template <bool kPoll = false>
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int lane) {
    int ok = 1;
    if (lane == 0)
        ok = (kPoll ? tc::mbar_wait_poll(bar, parity, err) : tc::mbar_wait_spin(bar, parity, err)) ? 1 : 0;
    return __shfl_sync(kFull, ok, 0) != 0;
}

template <int kNch>  // 16-channel chunks of an epilogue warp (cw / 16)
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
    uint64_t* a_ready = bars + 2;    // [2] hidden rows of a slot written (8 arrivals)
    uint64_t* slot_free = bars + 4;  // [2] the MMAs reading a slot are done
    uint64_t* acc_full = bars + 6;   // [2] accumulator holds its tile
    uint64_t* acc_free = bars + 8;   // [2] accumulator read out (8 arrivals)
    uint64_t* mma_done = bars + 10;
    uint64_t* u_full = bars + 11;    // [1] u rows of the next tile in sU (one arrival per writer)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
    volatile int* sFail = reinterpret_cast<volatile int*>(smem + L.fails);  // [2][8]

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
            tc::mbar_init(&a_ready[s], kHiddenWarps);
            tc::mbar_init(&slot_free[s], 1);
            tc::mbar_init(&acc_full[s], 1);
            tc::mbar_init(&acc_free[s], kEpilogueWarps);
        }
        tc::mbar_init(mma_done, 1);
        tc::mbar_init(u_full, kWriterWarps * 32);
        tc::fence_barrier_init();
    }
    if (tid < 2 * kEpilogueWarps) sFail[tid] = 0;
    fence_proxy_async();  // the weights written above, for the tensor cores
    if (warp == kControlWarp0) tc::tmem_alloc(tmem_slot, a.tmem_cols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp >= kControlWarp0) {
        // ---------------- control: u rows, pre-activation and main MMAs ----------------
        // Control warps 0-2 write the 128 u rows of a tile (warp 0 two rows
        // per lane: rows lane and 96 + lane; warps 1 and 2 one row each) and
        // signal them on an mbarrier; lane 0 of control warp 3 issues the
        // MMAs.
        const int cwarp = warp - kControlWarp0;
        // g = [x_j - x_i, x_i] of the row, from the points (model) or read as
        // given (operator). Stage 1 (fetch_indices) loads the centre point and
        // the neighbour index (or the given g) of a tile; stage 2
        // (fetch_points, one tile later) the neighbour point; write_u (one
        // more tile later) forms g, so no instruction waits on a load issued
        // in the same iteration.
        struct RowGeo {
            float4 pj;
            float3 pi, ni;
            float g6[6], ng6[6];
            int nj, nbase;  // neighbour index within its patch, the patch's first row
            bool gvalid, nvalid;
            int row;        // TMEM lane / u row
        };
        auto fetch_indices = [&](RowGeo& r, int t) {
            const int p = t * a.ppt + (r.row >> a.log2K);
            r.nvalid = t < n_tiles && p < R;
            const int pc = r.nvalid ? p : 0;
            if (a.geometry) {
                const float* gp = a.geometry + ((size_t)pc * K + (r.row & (K - 1))) * 6;
#pragma unroll
                for (int e = 0; e < 6; ++e) r.ng6[e] = gp[e];
            } else {
                const float4 v = *reinterpret_cast<const float4*>(a.xyz4 + (size_t)pc * 4);
                r.ni = make_float3(v.x, v.y, v.z);
                r.nbase = (pc / a.M) * a.M;
                r.nj = a.idx[(size_t)pc * K + (r.row & (K - 1))];
            }
        };
        auto fetch_points = [&](RowGeo& r) {
            if (a.geometry) {
#pragma unroll
                for (int e = 0; e < 6; ++e) r.g6[e] = r.ng6[e];
            } else {
                r.pi = r.ni;
                r.pj = *reinterpret_cast<const float4*>(a.xyz4 + (size_t)(r.nbase + r.nj) * 4);
            }
            r.gvalid = r.nvalid;
        };
        auto write_u = [&](RowGeo& r) {
            float g[6];
            if (!a.geometry) {
                r.g6[0] = r.pj.x - r.pi.x;
                r.g6[1] = r.pj.y - r.pi.y;
                r.g6[2] = r.pj.z - r.pi.z;
                r.g6[3] = r.pi.x;
                r.g6[4] = r.pi.y;
                r.g6[5] = r.pi.z;
            }
#pragma unroll
            for (int e = 0; e < 6; ++e) g[e] = r.gvalid ? r.g6[e] : 0.0f;
            write_u_row_g(sU, sGram, r.row, g);
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
        // W_po h of the tile in slot s into accumulator acc: per K step of 16
        // channels hi*hi + hi*lo + lo*hi, A (the hidden rows) from TMEM
        auto issue_main = [&](int s, int acc) {
            const uint32_t d = tmem_base + (uint32_t)(acc * cout);
            const uint32_t b0 = tc::smem_u32(sB), b1 = tc::smem_u32(sBlo);
            for (int k = 0; k < H / 16; ++k) {
                const uint32_t hi_col = tmem_base + slot_col0 + (uint32_t)(s * H + 16 * k);
                const uint32_t lo_col = hi_col + 8u;
                const int kb = k >> 2, w = k & 3;
                const uint64_t db_hi = tc::sw128_desc(b0 + (uint32_t)(kb * cout * 128)) + 2 * w;
                const uint64_t db_lo = tc::sw128_desc(b1 + (uint32_t)(kb * cout * 128)) + 2 * w;
                tc::umma_tmem_a_f16(d, hi_col, db_hi, a.idesc, k > 0 ? 1u : 0u);
                tc::umma_tmem_a_f16(d, hi_col, db_lo, a.idesc, 1u);
                tc::umma_tmem_a_f16(d, lo_col, db_hi, a.idesc, 1u);
            }
        };
        const int G = (int)gridDim.x;
        const int t0 = blockIdx.x, t1 = blockIdx.x + G;
        if (cwarp == kWriterWarps) {
            // ---- issuer: per tile index it, MMA(it) once its hidden rows are
            // in TMEM, then the pre-activations of tile it + 2 into the slot
            // MMA(it) releases, once the writers have its u rows in sU ----
            if (lane == 0) {
                bool good = tc::mbar_wait_poll(u_full, 0u, a.err);  // u rows of t0
                if (good) {
                    tc::tc_fence_after();
                    issue_pre(0);
                }
                if (good && t1 < n_tiles) {
                    good = tc::mbar_wait_poll(u_full, 1u, a.err);
                    if (good) {
                        tc::tc_fence_after();
                        issue_pre(1);
                    }
                }
                for (int it = 0; good; ++it) {
                    const int tile = blockIdx.x + it * G;
                    if (tile >= n_tiles) break;
                    const int s = it & 1, acc = it % a.n_acc;
                    good = tc::mbar_wait_poll(&a_ready[s], (uint32_t)(it >> 1) & 1u, a.err);
                    if (good && it >= a.n_acc)
                        good = tc::mbar_wait_poll(&acc_free[acc], ((uint32_t)(it / a.n_acc) & 1u) ^ 1u,
                                                  a.err);
                    if (!good) break;
                    tc::tc_fence_after();
                    issue_main(s, acc);
                    tc::umma_commit(&slot_free[s]);
                    tc::umma_commit(&acc_full[acc]);
                    if (tile + 2 * G < n_tiles) {
                        // u rows of tile index it + 2: the (it + 2)-th phase of u_full
                        good = tc::mbar_wait_poll(u_full, (uint32_t)it & 1u, a.err) &&
                               tc::mbar_wait_poll(&slot_free[s], (uint32_t)(it >> 1) & 1u, a.err);
                        if (good) {
                            tc::tc_fence_after();
                            issue_pre(s);
                        }
                    }
                }
                // every MMA issued completes before the CTA frees its memory
                tc::umma_commit(mma_done);
                tc::mbar_drain(mma_done, 0);
            }
            __syncwarp();
        } else {
            // ---- u-row writers: rows cwarp * 32 + lane, and for the first
            // writer also 96 + lane; the u rows of tile index it + 2
            // (geometry loaded one iteration earlier) as soon as pre(it + 1)
            // has read sU, each thread fencing its rows and arriving on u_full ----
            RowGeo rg[2] = {};
            rg[0].row = cwarp * 32 + lane;
            rg[1].row = 96 + lane;
            const bool two = cwarp == 0;  // warp-uniform
            auto each = [&](auto&& f) {
                f(rg[0]);
                if (two) f(rg[1]);
            };
            auto write_all = [&]() {
                each(write_u);
                // the rows for the tensor cores, before the next prefetch loads
                fence_proxy_async();
                tc::mbar_arrive(u_full);
            };
            each([&](RowGeo& r) { fetch_indices(r, t0); fetch_points(r); });
            write_all();
            bool ok = true;
            if (t1 < n_tiles) {
                each([&](RowGeo& r) { fetch_indices(r, t1); fetch_points(r); });
                ok = warp_wait<true>(&pre_full[0], 0, a.err, lane);  // sU read by pre(t0)
                if (ok) write_all();
            }
            each([&](RowGeo& r) { fetch_indices(r, t1 + G); fetch_points(r); });  // tile index 2
            each([&](RowGeo& r) { fetch_indices(r, t1 + 2 * G); });              // tile index 3, stage 1
            for (int it = 0; ok; ++it) {
                const int tile2 = blockIdx.x + (it + 2) * G;
                if (tile2 >= n_tiles) break;
                if (!warp_wait<true>(&pre_full[(it & 1) ^ 1], (uint32_t)((it + 1) >> 1) & 1u, a.err, lane))
                    break;
                write_all();
                // tile index it + 3, stage 2; tile index it + 4, stage 1
                each([&](RowGeo& r) { fetch_points(r); fetch_indices(r, tile2 + 2 * G); });
            }
        }
    } else if (warp < kHiddenWarps) {
        // ---------------- hidden rows ----------------
        const int q = warp & 3, half = warp >> 2;
        const uint32_t lane_off = tmem_base + ((uint32_t)(q * 32) << 16);
        const int chunks = H / 32;  // 16-channel chunks of this warp's half
        for (int it = 0;; ++it) {
            const int tile = blockIdx.x + it * (int)gridDim.x;
            if (tile >= n_tiles) break;
            const int s = it & 1;
            if (!warp_wait(&pre_full[s], (uint32_t)(it >> 1) & 1u, a.err, lane)) break;
            tc::tc_fence_after();
            const uint32_t col0 = lane_off + slot_col0 + (uint32_t)(s * H + half * (H / 2));
            // chunk c: fp32 pre-activations in its 16 columns, replaced by the
            // bf16 high halves (first 8 columns) and low halves (next 8); the
            // next chunk's load is in flight while this one is computed
            uint32_t r[2][16];
            tc::tmem_ld16_issue(col0, r[0]);
            tc::tmem_ld16_wait(r[0]);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                if (c >= chunks) break;
                uint32_t(&cur)[16] = r[c & 1];
                if (c + 1 < chunks) tc::tmem_ld16_issue(col0 + (uint32_t)(16 * (c + 1)), r[(c + 1) & 1]);
                uint32_t hi[8], lo[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float2 o = gelu_as2(
                        make_float2(__uint_as_float(cur[2 * e]), __uint_as_float(cur[2 * e + 1])));
                    const __nv_bfloat162 h2 = __floats2bfloat162_rn(o.x, o.y);
                    hi[e] = *reinterpret_cast<const uint32_t*>(&h2);
                    const float2 hf = make_float2(__uint_as_float(hi[e] << 16),
                                                  __uint_as_float(hi[e] & 0xffff0000u));
                    const float2 rem = fma2(hf, f2(-1.0f), o);  // o - hi, exact
                    lo[e] = pack_bf16(rem.x, rem.y);
                }
                tc::tmem_st_async<8>(col0 + (uint32_t)(16 * c), hi);
                tc::tmem_st_async<8>(col0 + (uint32_t)(16 * c + 8), lo);
                if (c + 1 < chunks) tc::tmem_ld16_wait(r[(c + 1) & 1]);
            }
            tc::tmem_st_wait();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&a_ready[s]);
        }
    } else {
        // ---------------- epilogue ----------------
        const int ew = warp - kEpiWarp0;
        const int q = ew & 3, half = ew >> 2;
        const int erow = q * 32 + lane;  // TMEM lane = edge row
        const int kk = erow & (K - 1);
        const int ptw = lane >> a.log2K;  // this lane's point within the warp's points
        const int ppw = 32 >> a.log2K;
        constexpr int nch = kNch, cw = 16 * kNch, nc = cw / 4;
        const int ch0 = half * cw;
        const uint32_t lane_off = tmem_base + ((uint32_t)(q * 32) << 16);
        const uint32_t stage = tc::smem_u32(smem + L.stage) + (uint32_t)ew * L.stage_bytes;
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
#pragma unroll 4
                for (int i = lane; i < 32 * nc; i += 32) {
                    const int r = i / nc, c = i - r * nc;
                    const int j = __shfl_sync(kFull, jl, r);
                    cp_async16(stage + (uint32_t)(r * cw * 4 + stage_swizzle(r, c) * 16),
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

        int jcur = neighbour_row(blockIdx.x);
        int jnext = neighbour_row(blockIdx.x + (int)gridDim.x);  // read a tile ahead
        issue_stage(blockIdx.x, jcur);
        for (int it = 0;; ++it) {
            const int tile = blockIdx.x + it * (int)gridDim.x;
            if (tile >= n_tiles) break;
            const int next = tile + (int)gridDim.x;
            const int acc = it % a.n_acc;
            const uint32_t rj = stage + (uint32_t)(lane * cw * 4);  // this lane's staged row
            const uint32_t ri = centre + (uint32_t)(ptw * cw * 4);
            // a failed wait is carried to the moment exchange below, where
            // the two warps of the lane quarter stop together (each reaches
            // the quarter's named barrier once per tile until then)
            bool ok = warp_wait(&acc_full[acc], (uint32_t)(it / a.n_acc) & 1u, a.err, lane);
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
                uint32_t racc[2][16];
                tc::tmem_ld16_issue(acol, racc[0]);
                tc::tmem_ld16_wait(racc[0]);
#pragma unroll 2
                for (int k = 0; k < nch; ++k) {
                    uint32_t(&r)[16] = racc[k & 1];
                    if (k + 1 < nch) tc::tmem_ld16_issue(acol + (uint32_t)(16 * (k + 1)), racc[(k + 1) & 1]);
                    float2 m[8];
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const int c = 4 * k + q4;
                        const uint32_t pos = rj + (uint32_t)(stage_swizzle(lane, c) * 16);
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
                    }
                    if (k == 0) {  // the shift: the mean of the first 16 channels
                        float2 csum = f2(0.0f);
#pragma unroll
                        for (int i = 0; i < 8; i += 2) csum = add2(csum, add2(m[i], m[i + 1]));
                        shift = (csum.x + csum.y) * (1.0f / 16.0f);
                    }
                    const float2 ns = f2(-shift);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float2 d = add2(m[i], ns);
                        s1p = add2(s1p, d);
                        s2p = fma2(d, d, s2p);
                    }
                    if (k + 1 < nch) tc::tmem_ld16_wait(racc[(k + 1) & 1]);
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
                tc::tmem_st_async<2>(lane_off + stat_col + (uint32_t)((it & 1) * 4 + half * 2), st);
                tc::tmem_st_wait();
            }
            if (lane == 0) sFail[(it & 1) * kEpilogueWarps + ew] = ok ? 0 : 1;
            tc::tc_fence_before();
            quarter_barrier(q);
            tc::tc_fence_after();
            if (sFail[(it & 1) * kEpilogueWarps + q] != 0 ||
                sFail[(it & 1) * kEpilogueWarps + q + 4] != 0)
                break;
            // the two halves' moments, combined pairwise (Chan et al.)
            uint32_t stats[2][2];
            {
                uint32_t s4[8];
                tc::tmem_ld<8>(lane_off + stat_col, s4);  // both parities; this tile's 4 columns
                const bool odd = (it & 1) != 0;  // (selects keep s4 in registers)
                stats[0][0] = odd ? s4[4] : s4[0];
                stats[0][1] = odd ? s4[5] : s4[1];
                stats[1][0] = odd ? s4[6] : s4[2];
                stats[1][1] = odd ? s4[7] : s4[3];
            }
            const float m0 = __uint_as_float(stats[0][0]), m1 = __uint_as_float(stats[1][0]);
            const float mean = 0.5f * (m0 + m1);
            const float dm = m1 - m0;
            const float m2 = __uint_as_float(stats[0][1]) + __uint_as_float(stats[1][1]) +
                             dm * dm * (0.5f * (float)cw);
            const float rstd = rsqrtf(m2 / (float)cout + 1e-6f);
            const float nmr = -mean * rstd;
            // the max over the K rows of each point of the normalised message,
            // by columns: lane l takes channels l, l + 32, ... of this warp's
            // cw and walks the rows of each point in the staged messages,
            // keeping the max and min of (m - mean) rstd (the row's rstd and
            // -mean rstd come by shuffle); the sign of the gain picks max or
            // -min, then |gain| x + shift and LeakyReLU(0.2), stored coalesced
            // the row's normalisation, read back by every lane as one broadcast
            float2* rn_w = reinterpret_cast<float2*>(smem + L.rn) + ew * 32;
            rn_w[lane] = make_float2(rstd, nmr);
            __syncwarp();  // every lane's messages and normalisation are in shared memory
            // channel lane + 32 j of staged row r: chunk (lane / 4 + 8 j), stored
            // at chunk 8 j + ((lane / 4) ^ (r & 7)) of the row (rows start on
            // 128-byte boundaries), element lane % 4
            const uint32_t lane_part = (uint32_t)(((lane >> 2) << 4) | ((lane & 3) << 2));
            uint32_t lp[8];  // this lane's offset in a row with r & 7 = i
#pragma unroll
            for (int i = 0; i < 8; ++i) lp[i] = lane_part ^ (uint32_t)(i << 4);
            constexpr int nj = cw / 32;  // channels per lane (1, 2, 3)
            float gain[nj], shift_c[nj], sgn[nj];
#pragma unroll
            for (int j = 0; j < nj; ++j) {
                const int c = ch0 + lane + 32 * j;
                gain[j] = sLn[2 * c];
                shift_c[j] = sLn[2 * c + 1];
                sgn[j] = sSgn[c];
            }
            const int pbase = tile * a.ppt + ((q * 32) >> a.log2K);
            for (int pt = 0; pt < ppw; ++pt) {
                // even and odd rows in separate max / min chains
                float mx[2][nj], mn[2][nj];
#pragma unroll
                for (int j = 0; j < nj; ++j) {
                    mx[0][j] = mx[1][j] = -FLT_MAX;
                    mn[0][j] = mn[1][j] = FLT_MAX;
                }
#pragma unroll 1
                for (int e0 = 0; e0 < K; e0 += 8) {  // K is a multiple of 8: row & 7 = i
                    const uint32_t base = stage + (uint32_t)((pt * K + e0) * cw * 4);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float2 rn = rn_w[pt * K + e0 + i];
                        const uint32_t rowa = base + (uint32_t)(i * cw * 4) + lp[i];
#pragma unroll
                        for (int j = 0; j < nj; ++j) {
                            const float x = fmaf(lds32(rowa + (uint32_t)(128 * j)), rn.x, rn.y);
                            mx[i & 1][j] = fmaxf(mx[i & 1][j], x);
                            mn[i & 1][j] = fminf(mn[i & 1][j], x);
                        }
                    }
                }
                const int p = pbase + pt;
                if (p < R) {
#pragma unroll
                    for (int j = 0; j < nj; ++j) {
                        const float v = sgn[j] > 0.0f ? fmaxf(mx[0][j], mx[1][j])
                                                      : -fminf(mn[0][j], mn[1][j]);
                        const float t = fmaf(v, gain[j], shift_c[j]);
                        a.out[(size_t)p * a.ldo + ch0 + lane + 32 * j] = fmaxf(t, 0.2f * t);
                    }
                }
            }
            __syncwarp();  // the messages are read before the next copies land there
            // this tile's staging has been read: bring in the next tile's
            jcur = jnext;
            issue_stage(next, jcur);
            jnext = neighbour_row(next + (int)gridDim.x);
        }
        cp_async_wait(0);  // no copy into shared memory outlives the loop
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == kControlWarp0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, a.tmem_cols);
    }
}

}  // namespace

// The split-bf16 neighbour stage on the three-role kernel when its shape allows:
// H in {64, 128}, C_out in {64, 128, 192}, K in {8, 16, 32}, geometry from the
// points (xyz4) or given;
// F2S_ERR_UNSUPPORTED otherwise (the caller then uses edge_tc_kernel).
int edge_stage_unified(const EdgeArgs& e, cudaStream_t st) {
    if (e.B == 0 || e.M == 0) return F2S_OK;
    int log2K = 0;
    while ((1 << log2K) < e.K) ++log2K;
    if ((e.geometry == nullptr) == (e.xyz4 == nullptr) || e.D != 6 || (e.H != 64 && e.H != 128) ||
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
    a.geometry = e.geometry;
    a.idx = e.idx;
    a.B = e.B;
    a.M = e.M;
    a.K = e.K;
    a.log2K = log2K;
    a.H = e.H;
    a.cout = e.cout;
    a.ppt = kRows / e.K;
    a.n_acc = 2 * e.cout + 2 * e.H + 8 <= 512 ? 2 : 1;
    const int cols = a.n_acc * e.cout + 2 * e.H + 8;
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
    switch (e.cout / 64) {
        case 1: return launch(edge_unified_kernel<2>);
        case 2: return launch(edge_unified_kernel<4>);
        default: return launch(edge_unified_kernel<6>);
    }
}

}  // namespace f2s
