// Tensor-core (tcgen05 / TMEM / TMA) GEMM for the point-wise contractions,
// Y (rows x cols) = A (rows x K) * W^T (W: cols x K), both K-major, with the
// model's epilogues fused: bias, gated residual x += g * (acc + b), and SwiGLU
// silu(acc_gate + b) * (acc_value + b2) from two weight matrices sharing A.
//
// Structure (one CTA per SM, persistent over 128 x BN output tiles):
//   warp 0      TMA producer: A and W tiles (128-byte swizzle) into a ring of
//               shared-memory stages, each completing on a "full" mbarrier;
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma (M = 128, N = BN,
//               K = 32 bytes per instruction) into one of two TMEM
//               accumulators and commits stage releases / accumulator-ready;
//   warps 2-9   epilogue: two warps per TMEM lane quarter, each taking every
//               other 32-column chunk; a chunk is read with tcgen05.ld (thread
//               = accumulator row), transposed through shared memory (lane =
//               column, so bias / gate loads and stores are coalesced), the
//               epilogue applied and stored; then the accumulator buffer is
//               freed, so the MMAs of the next tile overlap this epilogue.
// Operands are bf16 (kind::f16) or fp32 read as tf32 (kind::tf32), or
// (3xTF32) pairs x = hi + lo of tf32 values with the products hi*hi + hi*lo +
// lo*hi accumulated, which leaves only the lo*lo term (2^-22 relative) out.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace f2s {

// Library-wide device error word of the tensor-core kernels (bounded waits
// that ran out). Read and cleared through f2s_device_error().
__device__ int g_tc_error = 0;

namespace {

constexpr int kEpilogueThreads = 256;
constexpr int kTileM = 128;
constexpr size_t kSmemLimit = 227 * 1024;

struct TcGemmArgs {
    int rows, cols, K;
    int bn;
    int k_blocks;
    int stages;
    int b_res;          // the CTA's weight tiles (all K) stay in shared memory
    int acc_cols;       // TMEM columns of one accumulator buffer
    uint32_t idesc;
    uint32_t idesc_dual;  // SwiGLU: N = 2 BN over the adjacent W / W2 tiles
    const float* bias;
    const float* bias2;
    void* Y;
    int ldy;
    int y_bf16;
    int y_fp16;         // fp16 boxes (32 x 32, 64-byte swizzle) on the TMA path
    const float* gate;
    int gate_stride;
    int rows_per_patch;
    int round_tf32;
    int tma_epi;        // fp32 output written by TMA store / reduce-add boxes
    __half* vt;         // columns >= vt_col0: fp16, transposed per patch of vt_M rows
    int vt_col0, vt_C, vt_npad, vt_M;
    // columns [0, 2 kQkD): the attention's q and k rows, LayerNorm'd and split
    // into bf16 high / low parts (rows of [q 64 | k 64], zero padded)
    __nv_bfloat16* qk_hi;
    __nv_bfloat16* qk_lo;
    int* err;
};

// q / k width of the fused q/k epilogue: three 32-column chunks hold q and k.
constexpr int kQkD = 48;

constexpr uint32_t kEpiBox = 32 * 128;  // one 32-row x 32-column fp32 box, 128-byte swizzle

__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

// Byte offset of 16-byte chunk `chunk` (0..3) of row `row` in a box of
// 64-byte rows with the 64-byte swizzle (box base 512-byte aligned).
__device__ __forceinline__ uint32_t sw64_offset(int row, int chunk) {
    return (uint32_t)(row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4));
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(tc::smem_u32(src)), "r"(c0), "r"(c1)
                 : "memory");
}

// global += box, element by element in L2 (each element once: deterministic)
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int c0,
                                                  int c1) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(tc::smem_u32(src)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

template <int kPending>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kPending) : "memory");
}

// 16 consecutive values of a per-column vector from `col0` (zeros past `cols`;
// cols is a multiple of 4 on the TMA path).
__device__ __forceinline__ void load_cols16(const float* v, int col0, int cols, float (&out)[16]) {
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
        const float4 x = v && col0 + i < cols ? __ldg(reinterpret_cast<const float4*>(v + col0 + i))
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
        out[i] = x.x;
        out[i + 1] = x.y;
        out[i + 2] = x.z;
        out[i + 3] = x.w;
    }
}

// 32 consecutive values of a per-column vector from `col0` (zeros past `cols`;
// cols is a multiple of 4 on the TMA path).
__device__ __forceinline__ void load_cols32(const float* v, int col0, int cols, float (&out)[32]) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
        const float4 x = v && col0 + i < cols ? __ldg(reinterpret_cast<const float4*>(v + col0 + i))
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
        out[i] = x.x;
        out[i + 1] = x.y;
        out[i + 2] = x.z;
        out[i + 3] = x.w;
    }
}

// Threads of one CTA: TMA producer and MMA warps, kEW epilogue warps, and for
// the split-bf16 form four operand-split warps.
template <bool kTf32, bool kSplit, int kEW>
constexpr int gemm_threads() {
    return 64 + 32 * kEW + ((kSplit && !kTf32) ? 128 : 0);
}

// kSplit with kTf32 (3xTF32): map_a2 / map_b2 hold the low parts of A / W.
// kSplit without kTf32 (split bf16): A is fp32, loaded by TMA as two 32-column
// boxes per 64-column K block; four split warps turn each row of a stage into
// its bf16 high and low parts in place (the row's 256 fp32 bytes become 128
// bytes of each, in the same swizzled 128-byte slots of the two boxes, so a
// thread only ever overwrites its own row); map_b / map_b2 hold the bf16
// high and low parts of W; the MMA issues hi*hi + hi*lo + lo*hi.
// kEW: epilogue warps, 8, or 16 for the SwiGLU epilogue with fp16 rows (its
// SiLU on the special-function unit needs four warps per SM sub-partition to
// hide the latency of the exponential and reciprocal).
template <bool kTf32, int kEpi, bool kSplit, int kEW = 8>
__global__ void __launch_bounds__(gemm_threads<kTf32, kSplit, kEW>(), 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a2,
               const __grid_constant__ CUtensorMap map_b, const __grid_constant__ CUtensorMap map_b2,
               const __grid_constant__ CUtensorMap map_y, const TcGemmArgs g) {
    constexpr bool kDual = kEpi == kEpiSwiGlu;
    constexpr bool kSplitIn = kSplit && !kTf32;
    static_assert(!(kSplit && (kDual || kEpi != kEpiStore)), "split forms: the plain epilogue");
    static_assert(kEW == 8 || (kEW == 16 && kDual), "16 epilogue warps: the SwiGLU form only");
    constexpr int kEpiThreads = 32 * kEW;
    extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
    // 1024-byte alignment of the tile region (SWIZZLE_128B atoms)
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = g.stages;
    const uint32_t a_bytes = kTileM * 128;
    const uint32_t b_bytes = (uint32_t)g.bn * 128;
    // stage: A (A_lo), then W (W2 for SwiGLU, W_lo for 3xTF32). With b_res
    // the W tiles of every K block are loaded once, after the stages, and a
    // stage holds A only.
    const uint32_t a_stage = a_bytes * (kSplit ? 2 : 1);
    const uint32_t b_stage = b_bytes * ((kDual || kSplit) ? 2 : 1);
    const uint32_t stage_bytes = a_stage + (g.b_res ? 0u : b_stage);
    unsigned char* b_region = smem + (size_t)S * stage_bytes;
    const size_t tiles_bytes = (size_t)S * stage_bytes + (g.b_res ? (size_t)g.k_blocks * b_stage : 0);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + tiles_bytes);
    uint64_t* empty = full + S;
    uint64_t* tfull = empty + S;      // [2]
    uint64_t* tempty = tfull + 2;     // [2]
    uint64_t* mma_done = tempty + 2;  // [1]
    uint64_t* b_full = mma_done + 1;  // [1] the resident W tiles
    uint64_t* conv = b_full + 1;      // [S] split bf16: the stage's A split
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(conv + S);
    // per tile parity: set by the one polling epilogue lane when its wait
    // failed, read by every epilogue warp after their named barrier
    int* epi_fail = reinterpret_cast<int*>(tmem_slot + 1);  // [2]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles_n = (g.cols + g.bn - 1) / g.bn;
    const int m_tiles = (g.rows + kTileM - 1) / kTileM;
    // the i-th output tile of this CTA; false past its last. Streaming W:
    // tiles in row-major order, strided by the grid. Resident W: the grid is
    // n_tiles_n x groups, CTA c keeps N tile c % n_tiles_n and walks the row
    // blocks c / n_tiles_n, + groups, ...
    auto tile_at = [&](int i, int& m0, int& n0) -> bool {
        int mb, nb;
        if (g.b_res) {
            nb = (int)blockIdx.x % n_tiles_n;
            mb = (int)blockIdx.x / n_tiles_n + i * ((int)gridDim.x / n_tiles_n);
        } else {
            const int t = (int)blockIdx.x + i * (int)gridDim.x;
            mb = t / n_tiles_n;
            nb = t - mb * n_tiles_n;
        }
        m0 = mb * kTileM;
        n0 = nb * g.bn;
        return mb < m_tiles;
    };
    uint32_t tmem_cols = 32;
    while (tmem_cols < (uint32_t)(2 * g.acc_cols)) tmem_cols <<= 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
            if (kSplitIn) tc::mbar_init(&conv[s], 128);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], kEpiThreads);
        }
        tc::mbar_init(mma_done, 1);
        tc::mbar_init(b_full, 1);
        epi_fail[0] = epi_fail[1] = 0;
        tc::fence_barrier_init();
        tc::prefetch_tensormap(&map_a);
        tc::prefetch_tensormap(&map_b);
        if (kSplit) tc::prefetch_tensormap(&map_a2);
        if (kDual || kSplit) tc::prefetch_tensormap(&map_b2);
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, tmem_cols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t pending = 0;        // stages whose last load may still be in flight
            uint32_t pending_phase = 0;  // the phase each of those loads completes
            bool ok = true;
            if (g.b_res) {
                // the CTA's W tiles, every K block, once
                int m0, n0;
                tile_at(0, m0, n0);
                tc::mbar_arrive_expect_tx(b_full, (uint32_t)g.k_blocks * b_stage);
                for (int kb = 0; kb < g.k_blocks; ++kb) {
                    unsigned char* bs = b_region + (size_t)kb * b_stage;
                    const int k0 = kb * (kTf32 ? 32 : 64);
                    tc::tma_load_2d(bs, &map_b, b_full, k0, n0);
                    if (kDual || kSplit) tc::tma_load_2d(bs + b_bytes, &map_b2, b_full, k0, n0);
                }
            }
            for (int i = 0; ok; ++i) {
                int m0, n0;
                if (!tile_at(i, m0, n0)) break;
                for (int kb = 0; kb < g.k_blocks; ++kb) {
                    if (!tc::mbar_wait(&empty[stage], phase ^ 1u, g.err)) {
                        ok = false;
                        break;
                    }
                    pending &= ~(1u << stage);
                    unsigned char* st = smem + (size_t)stage * stage_bytes;
                    tc::mbar_arrive_expect_tx(&full[stage], stage_bytes);
                    const int k0 = kb * (kTf32 ? 32 : 64);
                    if constexpr (kSplitIn) {  // fp32 A: two boxes of 32 columns
                        tc::tma_load_2d(st, &map_a, &full[stage], k0, m0);
                        tc::tma_load_2d(st + a_bytes, &map_a, &full[stage], k0 + 32, m0);
                    } else {
                        tc::tma_load_2d(st, &map_a, &full[stage], k0, m0);
                        if (kSplit) tc::tma_load_2d(st + a_bytes, &map_a2, &full[stage], k0, m0);
                    }
                    if (!g.b_res) {
                        tc::tma_load_2d(st + a_stage, &map_b, &full[stage], k0, n0);
                        if (kDual || kSplit)
                            tc::tma_load_2d(st + a_stage + b_bytes, &map_b2, &full[stage], k0, n0);
                    }
                    pending |= 1u << stage;
                    pending_phase = (pending_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // let the copies already issued land before the CTA exits
                for (int s = 0; s < S; ++s)
                    if (pending & (1u << s)) tc::mbar_drain(&full[s], (pending_phase >> s) & 1u);
                if (g.b_res) tc::mbar_drain(b_full, 0);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int iter = 0;
            bool ok = true;
            constexpr int kSteps = 4;  // 128 bytes of K per stage / 32 bytes per instruction
            if (g.b_res && !tc::mbar_wait(b_full, 0, g.err)) ok = false;
            for (int i = 0; ok; ++i, ++iter) {
                int m0, n0;
                if (!tile_at(i, m0, n0)) break;
                const int buf = iter & 1;
                const uint32_t tph = (uint32_t)(iter >> 1) & 1u;
                if (!tc::mbar_wait(&tempty[buf], tph ^ 1u, g.err)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * g.acc_cols);
                for (int kb = 0; kb < g.k_blocks; ++kb) {
                    if (!tc::mbar_wait(&full[stage], phase, g.err) ||
                        (kSplitIn && !tc::mbar_wait_poll(&conv[stage], phase, g.err))) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t st = tc::smem_u32(smem + (size_t)stage * stage_bytes);
                    const uint32_t sb = g.b_res ? tc::smem_u32(b_region + (size_t)kb * b_stage)
                                                : st + a_stage;
                    // the stage's descriptors once; K step k adds 32 bytes = 2 in
                    // the start-address field (address >> 4)
                    const uint64_t a0 = tc::sw128_desc(st);
                    const uint64_t b0 = tc::sw128_desc(sb);
                    const uint64_t a_lo0 = kSplit ? tc::sw128_desc(st + a_bytes) : 0;
                    const uint64_t b_lo0 = kSplit ? tc::sw128_desc(sb + b_bytes) : 0;
                    const uint32_t idesc = kDual ? g.idesc_dual : g.idesc;
#pragma unroll
                    for (int k = 0; k < kSteps; ++k) {
                        const uint32_t acc = (kb | k) ? 1u : 0u;
                        // SwiGLU: W and W2 tiles are adjacent swizzled row blocks,
                        // so one N = 2 BN instruction fills both accumulators
                        tc::umma<kTf32>(d, a0 + 2 * k, b0 + 2 * k, idesc, acc);
                        if (kSplit) {
                            tc::umma<kTf32>(d, a0 + 2 * k, b_lo0 + 2 * k, g.idesc, 1u);
                            tc::umma<kTf32>(d, a_lo0 + 2 * k, b0 + 2 * k, g.idesc, 1u);
                        }
                    }
                    tc::umma_commit(&empty[stage]);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) tc::umma_commit(&tfull[buf]);
            }
            // every MMA this thread issued has completed before TMEM is freed
            tc::umma_commit(mma_done);
            tc::mbar_drain(mma_done, 0);
        }
        __syncwarp();
    } else if (kSplitIn && warp >= 2 + kEW) {
        // ---------------- operand split (warps 2 + kEW .. 5 + kEW) ----------------
        // thread = row of the A tile: the row's 64 fp32 values of the stage
        // (two boxes, 128-byte swizzle) are read, then its bf16 high parts are
        // written over the first box's row and the low parts over the second's
        const int r = (int)threadIdx.x - (64 + kEpiThreads);
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int i = 0; ok; ++i) {
            int m0, n0;
            if (!tile_at(i, m0, n0)) break;
            for (int kb = 0; kb < g.k_blocks; ++kb) {
                int landed = 1;
                if (lane == 0) landed = tc::mbar_wait_poll(&full[stage], phase, g.err) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, landed, 0)) {
                    ok = false;
                    break;
                }
                unsigned char* st = smem + (size_t)stage * stage_bytes;
                float4 x[16];  // x[q] = K columns 4q .. 4q + 3 of the block
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    x[c] = *reinterpret_cast<const float4*>(st + sw128_offset(r, c));
                    x[8 + c] = *reinterpret_cast<const float4*>(st + a_bytes + sw128_offset(r, c));
                }
#pragma unroll
                for (int c = 0; c < 8; ++c) {  // bf16 chunk c: K columns 8c .. 8c + 7
                    const float v[8] = {x[2 * c].x,     x[2 * c].y,     x[2 * c].z,     x[2 * c].w,
                                        x[2 * c + 1].x, x[2 * c + 1].y, x[2 * c + 1].z, x[2 * c + 1].w};
                    uint32_t h[4], l[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const __nv_bfloat162 hb = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
                        const float2 hf = __bfloat1622float2(hb);
                        const __nv_bfloat162 lb =
                            __floats2bfloat162_rn(v[2 * e] - hf.x, v[2 * e + 1] - hf.y);
                        h[e] = *reinterpret_cast<const uint32_t*>(&hb);
                        l[e] = *reinterpret_cast<const uint32_t*>(&lb);
                    }
                    *reinterpret_cast<uint4*>(st + sw128_offset(r, c)) = make_uint4(h[0], h[1], h[2], h[3]);
                    *reinterpret_cast<uint4*>(st + a_bytes + sw128_offset(r, c)) =
                        make_uint4(l[0], l[1], l[2], l[3]);
                }
                // the parts are read by the tensor cores (async proxy)
                fence_proxy_async_shared();
                tc::mbar_arrive(&conv[stage]);
                if (++stage == S) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 2 .. 1 + kEW) ----------------
        // kEW / 4 warps per TMEM lane quarter, taking alternate 32-column chunks
        const int quarter = warp & 3;
        const int ew = warp - 2;
        const int chunk_half = ew >> 2;  // the warp's place in its quarter
        unsigned char* epi_smem = smem + tiles_bytes + 1024;  // 1024-byte aligned
        // TMA path: two swizzled 32 x 32 boxes per warp, alternating (fp32
        // boxes of kEpiBox bytes); with 16 warps one 2 KB fp16 box per warp
        // (a warp stores one box per tile, so its previous store has long
        // finished reading when the next tile's box is written, and the
        // shared memory goes to operand stages instead)
        constexpr uint32_t kBoxSlot = kEW == 16 ? 2048u : kEpiBox;
        constexpr int kSlots = kEW == 16 ? 1 : 2;
        unsigned char* boxes = epi_smem + (size_t)ew * kSlots * kBoxSlot;
        // transposing path: 32 x 33 staging buffers (two for SwiGLU)
        float* stage_buf = reinterpret_cast<float*>(epi_smem) + ew * (kDual ? 2 : 1) * 32 * 33;
        float* stage_buf2 = stage_buf + 32 * 33;  // SwiGLU value accumulator
        int iter = 0;
        int boxes_sent = 0;
        for (int i = 0;; ++i, ++iter) {
            int m0, n0;
            if (!tile_at(i, m0, n0)) break;
            const int buf = iter & 1;
            const uint32_t tph = (uint32_t)(iter >> 1) & 1u;
            // one lane polls, the other epilogue warps wait on the named barrier
            volatile int* fail = epi_fail + (iter & 1);
            if (ew == 0 && lane == 0 && !tc::mbar_wait(&tfull[buf], tph, g.err)) *fail = 1;
            asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
            if (*fail) break;
            tc::tc_fence_after();
            const int row0 = m0 + quarter * 32;  // first of this warp's 32 rows
            const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) +
                                   (uint32_t)(buf * g.acc_cols);
            if constexpr (kEW == 16) {
                // SwiGLU into fp16 rows: warp place c of its quarter takes the
                // 32-column chunks c, c + 4, ... in two halves of 16 columns
                // (gate and value accumulators and both biases of a half in
                // registers), one 32 x 32 fp16 box per chunk, stored by TMA
                for (int c0 = chunk_half * 32; c0 < g.bn; c0 += 32 * (kEW / 4)) {
                    const int col0 = n0 + c0;
                    if (col0 >= g.cols) break;  // warp-uniform
                    unsigned char* box = boxes;
                    // the box's previous store must have read it
                    if (lane == 0 && boxes_sent >= 1) bulk_wait_read<0>();
                    __syncwarp();
                    bool out_of_range = false;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint32_t rv[16], ru[16];
                        tc::tmem_ld16_issue(t_row + (uint32_t)(c0 + 16 * h), rv);
                        tc::tmem_ld16_issue(t_row + (uint32_t)(g.bn + c0 + 16 * h), ru);
                        float b[16], b2[16];
                        load_cols16(g.bias, col0 + 16 * h, g.cols, b);
                        load_cols16(g.bias2, col0 + 16 * h, g.cols, b2);
                        tc::tmem_ld16_wait(rv);
                        tc::tmem_ld16_wait(ru);
                        float o[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            o[j] = f2s_silu_approx(__uint_as_float(rv[j]) + b[j]) *
                                   (__uint_as_float(ru[j]) + b2[j]);
                            // fp16 keeps tf32's 10-bit mantissa; a value the
                            // format cannot hold is reported, not clamped
                            out_of_range |= !(fabsf(o[j]) < 65504.0f);
                        }
#pragma unroll
                        for (int ch = 0; ch < 2; ++ch)
                            *reinterpret_cast<uint4*>(box + sw64_offset(lane, 2 * h + ch)) = make_uint4(
                                pack_half2(o[8 * ch], o[8 * ch + 1]), pack_half2(o[8 * ch + 2], o[8 * ch + 3]),
                                pack_half2(o[8 * ch + 4], o[8 * ch + 5]), pack_half2(o[8 * ch + 6], o[8 * ch + 7]));
                    }
                    if (out_of_range) atomicExch(g.err, tc::kTcFp16Range);
                    fence_proxy_async_shared();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&map_y, box, col0, row0);
                        bulk_commit();
                    }
                    ++boxes_sent;
                }
            } else if (g.tma_epi) {
                // thread = row: the epilogue in registers, one swizzled box per
                // 32 columns, written to global memory by one TMA store (or
                // reduce-add for the residual, so y is never read here)
                const int row = min(row0 + lane, g.rows - 1);
                int c_begin = chunk_half * 32, c_step = 64;
                if constexpr (kEpi == kEpiStore) {
                    if (g.qk_hi && n0 == 0) {
                        // the q and k columns: the first warp of the quarter
                        // takes all three chunks (a row's LayerNorm needs all
                        // of its q or k), the second the tile's other chunks
                        if (chunk_half == 0) {
                            float x[3][32];
#pragma unroll
                            for (int ch = 0; ch < 3; ++ch) {
                                tc::tmem_ld32(t_row + (uint32_t)(32 * ch), x[ch]);
                                if (g.bias) {
                                    float b[32];
                                    load_cols32(g.bias, 32 * ch, g.cols, b);
#pragma unroll
                                    for (int i = 0; i < 32; ++i) x[ch][i] += b[i];
                                }
                            }
                            {  // every lane: rows past the end are clipped by the stores
#pragma unroll
                                for (int part = 0; part < 2; ++part) {
                                    // ChannelLayerNorm without affine, eps 1e-6
                                    // (layers.py:20-27, transformer.py:59-63)
                                    float y[kQkD];
#pragma unroll
                                    for (int i = 0; i < kQkD; ++i)
                                        y[i] = x[(part * kQkD + i) >> 5][(part * kQkD + i) & 31];
                                    float sum = 0.0f;
#pragma unroll
                                    for (int i = 0; i < kQkD; ++i) sum += y[i];
                                    const float mean = sum / (float)kQkD;
                                    float qq = 0.0f;
#pragma unroll
                                    for (int i = 0; i < kQkD; ++i) qq = fmaf(y[i] - mean, y[i] - mean, qq);
                                    const float rstd = rsqrtf(qq / (float)kQkD + 1e-6f);
                                    uint32_t h[32], l[32];  // 64 bf16 of each part, zero padded
#pragma unroll
                                    for (int e = 0; e < 32; ++e) {
                                        const float v0 = 2 * e < kQkD ? (y[2 * e] - mean) * rstd : 0.0f;
                                        const float v1 = 2 * e + 1 < kQkD ? (y[2 * e + 1] - mean) * rstd : 0.0f;
                                        const __nv_bfloat162 hb = __floats2bfloat162_rn(v0, v1);
                                        const __nv_bfloat162 lb = __floats2bfloat162_rn(
                                            v0 - __bfloat162float(hb.x), v1 - __bfloat162float(hb.y));
                                        h[e] = *reinterpret_cast<const uint32_t*>(&hb);
                                        l[e] = *reinterpret_cast<const uint32_t*>(&lb);
                                    }
                                    // the warp's 32 rows x 64 bf16 of each part as one
                                    // swizzled box, stored by TMA (map_a2: high
                                    // parts, map_b2: low parts; unused by this form)
#pragma unroll
                                    for (int w = 0; w < 2; ++w) {
                                        const uint32_t* src = w == 0 ? h : l;
                                        unsigned char* box = boxes + (boxes_sent & 1) * kBoxSlot;
                                        if (lane == 0 && boxes_sent >= 2) bulk_wait_read<1>();
                                        __syncwarp();
#pragma unroll
                                        for (int j = 0; j < 8; ++j)
                                            *reinterpret_cast<uint4*>(box + sw128_offset(lane, j)) =
                                                make_uint4(src[4 * j], src[4 * j + 1], src[4 * j + 2], src[4 * j + 3]);
                                        fence_proxy_async_shared();
                                        __syncwarp();
                                        if (lane == 0) {
                                            tma_store_2d(w == 0 ? &map_a2 : &map_b2, box, part * 64, row0);
                                            bulk_commit();
                                        }
                                        ++boxes_sent;
                                    }
                                }
                            }
                            c_begin = g.bn;  // nothing else for this warp
                        } else {
                            c_begin = 2 * kQkD;
                            c_step = 32;
                        }
                    }
                }
                for (int c0 = c_begin; c0 < g.bn; c0 += c_step) {
                    const int col0 = n0 + c0;
                    float v[32];
                    tc::tmem_ld32(t_row + (uint32_t)c0, v);
                    if (col0 >= g.cols) continue;  // warp-uniform
                    float b[32];
                    load_cols32(g.bias, col0, g.cols, b);
                    if constexpr (kDual) {
                        float u[32], b2[32];
                        tc::tmem_ld32(t_row + (uint32_t)(g.bn + c0), u);
                        load_cols32(g.bias2, col0, g.cols, b2);
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = f2s_silu_approx(v[i] + b[i]) * (u[i] + b2[i]);
                    } else if constexpr (kEpi == kEpiGatedResidual) {
                        float gt[32];
                        load_cols32(g.gate + (size_t)(row / g.rows_per_patch) * g.gate_stride, col0,
                                    g.cols, gt);
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = gt[i] * (v[i] + b[i]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            v[i] += b[i];
                            if (g.round_tf32) v[i] = f2s_round_tf32(v[i]);
                        }
                        if (g.vt && col0 >= g.vt_col0) {
                            // a chunk of V: column c of this row goes to
                            // vt[patch][c][row in patch] in fp16; a warp's 32
                            // rows of one column are contiguous there
                            const int pb0 = row0 / g.vt_M, key0 = row0 - pb0 * g.vt_M;
                            if (key0 + 32 <= g.vt_M && (key0 & 7) == 0 && row0 + 32 <= g.rows &&
                                col0 + 32 <= g.cols) {  // warp-uniform
                                // 32 rows of one patch, 16-byte aligned there: the
                                // chunk transposed through this warp's box slot
                                // (rows of 40 halves: the 16-byte reads of eight
                                // consecutive columns hit distinct banks), then
                                // each lane stores one column's 32 keys as four
                                // 16-byte stores
                                __half* t = reinterpret_cast<__half*>(boxes + (boxes_sent & 1) * kBoxSlot);
                                if (lane == 0) bulk_wait_read<0>();  // no box store still reads the slot
                                __syncwarp();
                                bool out_of_range = false;
#pragma unroll
                                for (int i = 0; i < 32; ++i) {
                                    out_of_range |= !(fabsf(v[i]) < 65504.0f);
                                    t[i * 40 + lane] = __float2half_rn(v[i]);
                                }
                                if (out_of_range) atomicExch(g.err, tc::kTcFp16Range);
                                __syncwarp();
                                const uint4* src = reinterpret_cast<const uint4*>(t + lane * 40);
                                uint4* dst = reinterpret_cast<uint4*>(
                                    g.vt + ((size_t)pb0 * g.vt_C + (col0 - g.vt_col0 + lane)) * g.vt_npad + key0);
#pragma unroll
                                for (int j = 0; j < 4; ++j) dst[j] = src[j];
                                __syncwarp();  // the slot is read before it is written again
                                continue;
                            }
                            const int r = row0 + lane;
                            if (r < g.rows) {
                                const int pb = r / g.vt_M;
                                __half* dst = g.vt + ((size_t)pb * g.vt_C + (col0 - g.vt_col0)) * g.vt_npad +
                                              (r - pb * g.vt_M);
                                bool out_of_range = false;
#pragma unroll
                                for (int i = 0; i < 32; ++i) {
                                    if (col0 + i < g.cols) {
                                        out_of_range |= !(fabsf(v[i]) < 65504.0f);
                                        dst[(size_t)i * g.vt_npad] = __float2half_rn(v[i]);
                                    }
                                }
                                if (out_of_range) atomicExch(g.err, tc::kTcFp16Range);
                            }
                            continue;  // nothing of this chunk goes to Y
                        }
                    }
                    unsigned char* box = boxes + (boxes_sent & 1) * kBoxSlot;
                    // the box's previous store must have read it
                    if (lane == 0 && boxes_sent >= 2) bulk_wait_read<1>();
                    __syncwarp();
                    if (g.y_fp16) {
                        // fp16 values keep tf32's 10-bit mantissa; a value the
                        // format cannot hold is reported, not clamped
                        bool out_of_range = false;
#pragma unroll
                        for (int i = 0; i < 32; ++i) out_of_range |= !(fabsf(v[i]) < 65504.0f);
                        if (out_of_range) atomicExch(g.err, tc::kTcFp16Range);
#pragma unroll
                        for (int ch = 0; ch < 4; ++ch)
                            *reinterpret_cast<uint4*>(box + sw64_offset(lane, ch)) = make_uint4(
                                pack_half2(v[8 * ch], v[8 * ch + 1]), pack_half2(v[8 * ch + 2], v[8 * ch + 3]),
                                pack_half2(v[8 * ch + 4], v[8 * ch + 5]), pack_half2(v[8 * ch + 6], v[8 * ch + 7]));
                    } else {
#pragma unroll
                        for (int ch = 0; ch < 8; ++ch)
                            *reinterpret_cast<float4*>(box + sw128_offset(lane, ch)) =
                                make_float4(v[4 * ch], v[4 * ch + 1], v[4 * ch + 2], v[4 * ch + 3]);
                    }
                    fence_proxy_async_shared();
                    __syncwarp();
                    if (lane == 0) {
                        if constexpr (kEpi == kEpiGatedResidual) tma_reduce_add_2d(&map_y, box, col0, row0);
                        else tma_store_2d(&map_y, box, col0, row0);
                        bulk_commit();
                    }
                    ++boxes_sent;
                }
            } else {
            for (int c0 = chunk_half * 32; c0 < g.bn; c0 += 64) {
                // thread = row in TMEM; through the staging buffer, lane = column
                // for coalesced global access and one bias / gate load per lane
                float v[32];
                tc::tmem_ld32(t_row + (uint32_t)c0, v);
#pragma unroll
                for (int i = 0; i < 32; ++i) stage_buf[lane * 33 + i] = v[i];
                if constexpr (kDual) {
                    tc::tmem_ld32(t_row + (uint32_t)(g.bn + c0), v);
#pragma unroll
                    for (int i = 0; i < 32; ++i) stage_buf2[lane * 33 + i] = v[i];
                }
                __syncwarp();
                const int col = n0 + c0 + lane;
                if (col < g.cols) {
                    const float b = g.bias ? g.bias[col] : 0.0f;
                    const float b2 = (kDual && g.bias2) ? g.bias2[col] : 0.0f;
                    const int r_end = min(32, g.rows - row0);
                    // gated residual: patch of the current row and the row
                    // where the next patch starts
                    int patch = row0 / g.rows_per_patch;
                    int next_patch_row = (patch + 1) * g.rows_per_patch;
                    float gt = 0.0f;
                    if constexpr (kEpi == kEpiGatedResidual)
                        gt = g.gate[(size_t)patch * g.gate_stride + col];
                    // eight rows at a time: all loads of a group are issued
                    // before its stores (rows are distinct, but the compiler
                    // cannot tell that the residual loads do not alias them)
                    for (int r0 = 0; r0 < r_end; r0 += 8) {
                        float yv[8];
                        if constexpr (kEpi == kEpiGatedResidual) {
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                yv[j] = r0 + j < r_end
                                            ? static_cast<const float*>(g.Y)[(size_t)(row0 + r0 + j) * g.ldy + col]
                                            : 0.0f;
                        }
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int r = r0 + j;
                            if (r >= r_end) break;
                            const int row = row0 + r;
                            float out = stage_buf[r * 33 + lane] + b;
                            if constexpr (kDual) {
                                const float u = stage_buf2[r * 33 + lane] + b2;
                                out = f2s_silu_approx(out) * u;
                            }
                            const size_t o = (size_t)row * g.ldy + col;
                            if constexpr (kEpi == kEpiGatedResidual) {
                                if (row >= next_patch_row) {
                                    patch = row / g.rows_per_patch;
                                    next_patch_row = (patch + 1) * g.rows_per_patch;
                                    gt = g.gate[(size_t)patch * g.gate_stride + col];
                                }
                                static_cast<float*>(g.Y)[o] = fmaf(gt, out, yv[j]);
                            } else if (g.y_bf16) {
                                static_cast<__nv_bfloat16*>(g.Y)[o] = __float2bfloat16_rn(out);
                            } else {
                                static_cast<float*>(g.Y)[o] = g.round_tf32 ? f2s_round_tf32(out) : out;
                            }
                        }
                    }
                }
                __syncwarp();
            }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&tempty[buf]);
        }
        // every box store has read its shared memory before the CTA exits
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
    }

    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, tmem_cols);
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

template <bool kTf32, int kEpi, bool kSplit = false, int kEW = 8>
int launch_tc(const CUtensorMap& ma, const CUtensorMap& ma2, const CUtensorMap& mb,
              const CUtensorMap& mb2, const CUtensorMap& my, const TcGemmArgs& g, size_t smem,
              int grid, cudaStream_t st) {
    auto kernel = tc_gemm_kernel<kTf32, kEpi, kSplit, kEW>;
    F2S_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kernel<<<grid, gemm_threads<kTf32, kSplit, kEW>(), smem, st>>>(ma, ma2, mb, mb2, my, g);
    return check_launch("tc_gemm_kernel");
}

}  // namespace

int* tc_error_word() {
    static int* addr[64] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_tc_error) != cudaSuccess) return nullptr;
        addr[dev] = static_cast<int*>(p);
    }
    return addr[dev];
}

int make_tensor_map_2d_typed(CUtensorMap* map, const void* base, TmaType type, int swizzle_bytes,
                             int64_t rows, int64_t cols, int64_t ld, int box_rows, int box_cols) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(F2S_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const int64_t elem = type == kTmaF32 ? 4 : 2;
    F2S_REQUIRE(((uintptr_t)base & 15) == 0, "tensor map base must be 16-byte aligned");
    F2S_REQUIRE((ld * elem) % 16 == 0, "tensor map row pitch must be a multiple of 16 bytes");
    F2S_REQUIRE(swizzle_bytes == 128 || swizzle_bytes == 64, "tensor map swizzle %d", swizzle_bytes);
    F2S_REQUIRE(box_cols * elem <= swizzle_bytes, "tensor map box row wider than its swizzle span");
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(ld * elem)};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = type == kTmaF32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : type == kTmaBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(F2S_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return F2S_OK;
}

int make_tensor_map_2d(CUtensorMap* map, const void* base, bool fp32, int64_t rows, int64_t cols,
                       int64_t ld, int box_rows, int box_cols) {
    return make_tensor_map_2d_typed(map, base, fp32 ? kTmaF32 : kTmaBF16, 128, rows, cols, ld,
                                    box_rows, box_cols);
}

int make_tensor_map_3d(CUtensorMap* map, const void* base, bool fp32, int64_t d0, int64_t d1,
                       int64_t d2, int64_t stride1_bytes, int64_t stride2_bytes, int box0,
                       int box1) {
    return make_tensor_map_3d_typed(map, base, fp32 ? kTmaF32 : kTmaBF16, d0, d1, d2,
                                    stride1_bytes, stride2_bytes, box0, box1);
}

int make_tensor_map_3d_typed(CUtensorMap* map, const void* base, TmaType type, int64_t d0,
                             int64_t d1, int64_t d2, int64_t stride1_bytes, int64_t stride2_bytes,
                             int box0, int box1) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(F2S_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    F2S_REQUIRE(((uintptr_t)base & 15) == 0, "tensor map base must be 16-byte aligned");
    F2S_REQUIRE(stride1_bytes % 16 == 0 && stride2_bytes % 16 == 0,
                "tensor map strides must be multiples of 16 bytes");
    const cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
    const cuuint64_t strides[2] = {(cuuint64_t)stride1_bytes, (cuuint64_t)stride2_bytes};
    const cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType dt = type == kTmaF32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : type == kTmaBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(F2S_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
    return F2S_OK;
}

// Y = A W^T (+ epilogue) on tcgen05. A: rows x K (lda), W: cols x K (K
// contiguous), W2 the SwiGLU value weights. `tf32`: A/W are fp32 and the MMA
// runs kind::tf32; otherwise bf16 and kind::f16. bn: N tile (multiple of 32,
// <= 256; <= 128 for SwiGLU).
int tc_gemm(const TcGemmOp& op, cudaStream_t st) {
    if (op.rows == 0 || op.cols == 0) return F2S_OK;
    F2S_REQUIRE(op.A && op.W && op.Y && op.K > 0, "tc_gemm: bad operands");
    const bool dual = op.epilogue == kEpiSwiGlu;
    const bool split = op.A_lo != nullptr;
    const bool split_in = op.split_in;
    F2S_REQUIRE(!dual || op.W2, "tc_gemm: SwiGLU needs W2");
    F2S_REQUIRE(!split || (op.W_lo && op.tf32 && op.epilogue == kEpiStore && !split_in),
                "tc_gemm: 3xTF32 needs W_lo, tf32 operands and the plain epilogue");
    F2S_REQUIRE(!split_in || (op.W_lo && !op.tf32 && !op.fp16 && op.epilogue == kEpiStore &&
                              op.lda % 4 == 0 && ((uintptr_t)op.A & 15) == 0),
                "tc_gemm: split bf16 needs fp32 A rows of 16-byte pitch, W / W_lo in bf16 and "
                "the plain epilogue");
    F2S_REQUIRE(op.epilogue != kEpiGatedResidual || (op.gate && op.rows_per_patch > 0 && !op.y_bf16),
                "tc_gemm: gated residual needs a gate and an fp32 output");
    int bn = op.bn;
    F2S_REQUIRE(bn >= 32 && bn <= 256 && bn % 32 == 0 && (!dual || bn <= 128),
                "tc_gemm: bad N tile %d", bn);
    int* err = tc_error_word();
    if (!err) return fail(F2S_ERR_CUDA, "tc_gemm: device error word unavailable");
    F2S_REQUIRE(!(op.fp16 && op.tf32), "tc_gemm: fp16 operands run kind::f16, not tf32");
    F2S_REQUIRE(!(op.y_fp16 && op.y_bf16), "tc_gemm: one output type");
    CUtensorMap ma, ma2, mb, mb2;
    const int bk = op.tf32 ? 32 : 64;
    const TmaType ot = op.tf32 ? kTmaF32 : op.fp16 ? kTmaF16 : kTmaBF16;
    // split bf16: fp32 A in boxes of 32 columns (two per 64-column K block)
    if (split_in) F2S_TRY(make_tensor_map_2d_typed(&ma, op.A, kTmaF32, 128, op.rows, op.K, op.lda, kTileM, 32));
    else F2S_TRY(make_tensor_map_2d_typed(&ma, op.A, ot, 128, op.rows, op.K, op.lda, kTileM, bk));
    F2S_TRY(make_tensor_map_2d_typed(&mb, op.W, ot, 128, op.cols, op.K, op.K, bn, bk));
    if (dual) F2S_TRY(make_tensor_map_2d_typed(&mb2, op.W2, ot, 128, op.cols, op.K, op.K, bn, bk));
    else if (split) F2S_TRY(make_tensor_map_2d(&mb2, op.W_lo, true, op.cols, op.K, op.K, bn, bk));
    else if (split_in) F2S_TRY(make_tensor_map_2d_typed(&mb2, op.W_lo, kTmaBF16, 128, op.cols, op.K, op.K, bn, bk));
    else mb2 = mb;
    if (split) F2S_TRY(make_tensor_map_2d(&ma2, op.A_lo, true, op.rows, op.K, op.lda, kTileM, bk));
    else ma2 = ma;
    if (op.qk_hi && op.qk_lo && !dual && !split && !split_in) {
        // the fused q/k rows (bf16, 128 per row): 32-row x 64-column boxes
        F2S_TRY(make_tensor_map_2d_typed(&ma2, op.qk_hi, kTmaBF16, 128, op.rows, 128, 128, 32, 64));
        F2S_TRY(make_tensor_map_2d_typed(&mb2, op.qk_lo, kTmaBF16, 128, op.rows, 128, 128, 32, 64));
    }

    TcGemmArgs g{};
    g.rows = op.rows;
    g.cols = op.cols;
    g.K = op.K;
    g.bn = bn;
    g.k_blocks = ceil_div(op.K, bk);
    g.acc_cols = bn * (dual ? 2 : 1);
    // operand format of the instruction descriptor: 0 fp16, 1 bf16 (kind::f16), 2 tf32
    const uint32_t fmt = op.tf32 ? 2u : op.fp16 ? 0u : 1u;
    g.idesc = tc::make_idesc(kTileM, bn, fmt);
    g.idesc_dual = tc::make_idesc(kTileM, 2 * bn, fmt);
    g.bias = op.bias;
    g.bias2 = op.bias2;
    g.Y = op.Y;
    g.ldy = op.ldy;
    g.y_bf16 = op.y_bf16 ? 1 : 0;
    g.y_fp16 = op.y_fp16 ? 1 : 0;
    g.gate = op.gate;
    g.gate_stride = op.gate_stride;
    g.rows_per_patch = op.rows_per_patch > 0 ? op.rows_per_patch : 1;
    g.round_tf32 = op.round_tf32 ? 1 : 0;
    g.vt = op.vt;
    g.vt_col0 = op.vt_col0;
    g.vt_C = op.vt_C;
    g.vt_npad = op.vt_npad;
    g.vt_M = op.vt_M > 0 ? op.vt_M : 1;
    g.qk_hi = static_cast<__nv_bfloat16*>(op.qk_hi);
    g.qk_lo = static_cast<__nv_bfloat16*>(op.qk_lo);
    g.err = err;
    // fp32 output with 16-byte rows, columns and per-column vectors: the
    // epilogue writes 32 x 32 boxes by TMA (store, or reduce-add for the residual)
    auto aligned16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    g.tma_epi = !op.y_bf16 && op.ldy % (op.y_fp16 ? 8 : 4) == 0 && op.cols % 4 == 0 && aligned16(op.Y) &&
                aligned16(op.bias) && aligned16(op.bias2) &&
                (op.epilogue != kEpiGatedResidual || (aligned16(op.gate) && op.gate_stride % 4 == 0));
    F2S_REQUIRE(!op.y_fp16 || (g.tma_epi && op.epilogue != kEpiGatedResidual),
                "tc_gemm: fp16 output needs the TMA epilogue (16-byte rows and vectors), no residual");
    F2S_REQUIRE(!op.vt || (g.tma_epi && op.epilogue == kEpiStore && !split && !split_in &&
                           !op.y_fp16 && op.vt_col0 % 32 == 0 && op.vt_M > 0 &&
                           op.vt_npad >= op.vt_M),
                "tc_gemm: the V^T output needs the plain TMA epilogue and a 32-aligned first column");
    F2S_REQUIRE(!op.qk_hi || (op.vt && op.qk_lo && op.vt_col0 == 2 * kQkD && bn >= 2 * kQkD &&
                              op.cols >= 2 * kQkD),
                "tc_gemm: the q/k output needs the V^T output at column %d and an N tile of >= %d",
                2 * kQkD, 2 * kQkD);
    CUtensorMap my;
    if (g.tma_epi)
        F2S_TRY(make_tensor_map_2d_typed(&my, op.Y, op.y_fp16 ? kTmaF16 : kTmaF32, op.y_fp16 ? 64 : 128,
                                         op.rows, op.cols, op.ldy, 32, 32));
    else my = ma;
    const size_t a_stage_bytes = (size_t)kTileM * 128 * ((split || split_in) ? 2 : 1);
    const size_t b_stage_bytes = (size_t)bn * 128 * ((dual || split || split_in) ? 2 : 1);
    // epilogue region: the TMA path's two 4 KB boxes per warp, or the
    // transposing path's 32 x 33 buffers
    // SwiGLU into fp16 rows runs 16 epilogue warps with 2 KB boxes
    const bool wide_epi = dual && op.y_fp16 && g.tma_epi;
    const size_t stage_buf_bytes =
        wide_epi    ? (size_t)16 * 2048
        : g.tma_epi ? (size_t)(kEpilogueThreads / 32) * 2 * kEpiBox
                    : (size_t)(kEpilogueThreads / 32) * (dual ? 2 : 1) * 32 * 33 * sizeof(float);
    const size_t fixed = 1024 + 1024 + stage_buf_bytes;  // alignment slack, barriers, epilogue
    const int m_tiles = ceil_div(op.rows, kTileM), n_tiles_n = ceil_div(op.cols, bn);
    const int sms = sm_count();
    // Resident W: when one N tile's weights over all of K fit beside two A
    // stages and every CTA gets at least two row blocks, each CTA loads its
    // W tiles once instead of once per output tile (a small-K GEMM otherwise
    // moves more W than A bytes from L2 into shared memory).
    const size_t b_region = (size_t)g.k_blocks * b_stage_bytes;
    int groups = n_tiles_n <= sms ? sms / n_tiles_n : 0;
    groups = groups < m_tiles ? groups : m_tiles;
    g.b_res = groups >= 1 && m_tiles >= 2 * groups &&
              fixed + b_region + 4 * a_stage_bytes <= kSmemLimit;
    const size_t stage_bytes = a_stage_bytes + (g.b_res ? 0 : b_stage_bytes);
    const size_t resident = g.b_res ? b_region : 0;
    int stages = (int)((kSmemLimit - fixed - resident) / stage_bytes);
    stages = stages > 8 ? 8 : stages;
    F2S_LIMIT(stages >= 2, "tc_gemm: tile too large for shared memory");
    g.stages = stages;
    // alignment slack, tiles (+ resident W), barriers + TMEM slot (< 1 KB,
    // keeping the epilogue region 1024-byte aligned for its swizzled boxes),
    // epilogue region
    const size_t smem = 1024 + stages * stage_bytes + resident + 1024 + stage_buf_bytes;
    const int tiles = m_tiles * n_tiles_n;
    const int grid = g.b_res ? n_tiles_n * groups : (tiles < sms ? tiles : sms);
    TraceScope trace(op.tag, st);
    if (split) return launch_tc<true, kEpiStore, true>(ma, ma2, mb, mb2, my, g, smem, grid, st);
    if (split_in) return launch_tc<false, kEpiStore, true>(ma, ma2, mb, mb2, my, g, smem, grid, st);
    if (op.tf32) {
        switch (op.epilogue) {
            case kEpiStore: return launch_tc<true, kEpiStore>(ma, ma2, mb, mb2, my, g, smem, grid, st);
            case kEpiGatedResidual: return launch_tc<true, kEpiGatedResidual>(ma, ma2, mb, mb2, my, g, smem, grid, st);
            case kEpiSwiGlu:
                if (wide_epi) return launch_tc<true, kEpiSwiGlu, false, 16>(ma, ma2, mb, mb2, my, g, smem, grid, st);
                return launch_tc<true, kEpiSwiGlu>(ma, ma2, mb, mb2, my, g, smem, grid, st);
        }
    } else {
        switch (op.epilogue) {
            case kEpiStore: return launch_tc<false, kEpiStore>(ma, ma2, mb, mb2, my, g, smem, grid, st);
            case kEpiGatedResidual: return launch_tc<false, kEpiGatedResidual>(ma, ma2, mb, mb2, my, g, smem, grid, st);
            case kEpiSwiGlu:
                if (wide_epi) return launch_tc<false, kEpiSwiGlu, false, 16>(ma, ma2, mb, mb2, my, g, smem, grid, st);
                return launch_tc<false, kEpiSwiGlu>(ma, ma2, mb, mb2, my, g, smem, grid, st);
        }
    }
    return fail(F2S_ERR_INVALID_ARGUMENT, "tc_gemm: bad epilogue");
}

namespace {
// hi = x rounded to the nearest tf32, lo = x - hi (exact), both (rows, K).
__global__ void split_tf32_kernel(const float* __restrict__ x, int ldx, int rows, int K,
                                  float* __restrict__ hi, float* __restrict__ lo) {
    const int64_t total = (int64_t)rows * K;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / K, c = i - r * K;
        const float v = x[r * ldx + c];
        const float h = f2s_round_tf32(v);
        hi[i] = h;
        lo[i] = v - h;
    }
}

// The same four columns at a time (K and ldx multiples of 4, 16-byte aligned
// arrays, fewer than 2^31 groups): 16-byte accesses, 32-bit index arithmetic.
__global__ void split_tf32_x4_kernel(const float4* __restrict__ x, int ldx4, int rows, int K4,
                                     float4* __restrict__ hi, float4* __restrict__ lo) {
    const int total = rows * K4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int r = i / K4, c = i - r * K4;
        const float4 v = x[(size_t)r * ldx4 + c];
        const float4 h = make_float4(f2s_round_tf32(v.x), f2s_round_tf32(v.y), f2s_round_tf32(v.z),
                                     f2s_round_tf32(v.w));
        hi[i] = h;
        lo[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
    }
}
}  // namespace

namespace {
// hi = bf16(x), lo = bf16(x - hi), both (rows, K) with leading dimension K.
__global__ void split_bf16_kernel(const float* __restrict__ x, int ldx, int rows, int K,
                                  __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    const int64_t total = (int64_t)rows * K;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / K, c = i - r * K;
        const float v = x[r * ldx + c];
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        hi[i] = h;
        lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
}
}  // namespace

int split_bf16(const float* x, int ldx, int rows, int K, void* hi, void* lo, cudaStream_t st) {
    if (rows == 0 || K == 0) return F2S_OK;
    const int64_t total = (int64_t)rows * K;
    const int64_t cap = (int64_t)sm_count() * 16;
    int64_t blocks = (total + 255) / 256;
    blocks = blocks < cap ? blocks : cap;
    split_bf16_kernel<<<(int)blocks, 256, 0, st>>>(x, ldx, rows, K, static_cast<__nv_bfloat16*>(hi),
                                                   static_cast<__nv_bfloat16*>(lo));
    return check_launch("split_bf16_kernel");
}

int split_tf32(const float* x, int ldx, int rows, int K, float* hi, float* lo, cudaStream_t st) {
    if (rows == 0 || K == 0) return F2S_OK;
    const int64_t total = (int64_t)rows * K;
    const int64_t cap = (int64_t)sm_count() * 16;
    auto aligned16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    if (K % 4 == 0 && ldx % 4 == 0 && aligned16(x) && aligned16(hi) && aligned16(lo) &&
        total / 4 < (int64_t)INT32_MAX) {
        int64_t blocks = (total / 4 + 255) / 256;
        blocks = blocks < cap ? blocks : cap;
        split_tf32_x4_kernel<<<(int)blocks, 256, 0, st>>>(
            reinterpret_cast<const float4*>(x), ldx / 4, rows, K / 4, reinterpret_cast<float4*>(hi),
            reinterpret_cast<float4*>(lo));
        return check_launch("split_tf32_x4_kernel");
    }
    int64_t blocks = (total + 255) / 256;
    blocks = blocks < cap ? blocks : cap;
    split_tf32_kernel<<<(int)blocks, 256, 0, st>>>(x, ldx, rows, K, hi, lo);
    return check_launch("split_tf32_kernel");
}

int tc_pick_bn(int cols, bool swiglu) {
    // One tcgen05 MMA (M = 128) takes about 64 ns for every N up to ~176 and
    // about 0.36 ns per column beyond (measured on B200: 64 ns at N <= 128,
    // 93 ns at N = 256): minimise N tiles x that time, larger tiles on ties.
    // On ties, the least padding, then the larger tile. SwiGLU tiles pair W
    // and W2 in one N = 2 BN instruction, so BN <= 128.
    static const int kCandidates[] = {256, 224, 192, 160, 128, 96, 64, 32};
    int best = 32, best_waste = 1 << 30;
    double best_cost = 1e30;
    for (int bn : kCandidates) {
        if (swiglu && bn > 128) continue;
        const int n_eff = swiglu ? 2 * bn : bn;
        const double per_mma = 0.3625 * n_eff > 64.0 ? 0.3625 * n_eff : 64.0;
        const int tiles = ceil_div(cols, bn);
        const double cost = tiles * per_mma;
        const int waste = tiles * bn - cols;
        if (cost < best_cost - 1e-9 || (cost < best_cost + 1e-9 && waste < best_waste)) {
            best = bn;
            best_cost = cost;
            best_waste = waste;
        }
    }
    return best;
}

}  // namespace f2s

extern "C" int f2s_linear(const void* x, int ldx, const void* weight, const float* bias, float* y,
                          int ldy, int rows, int cols, int K, int precision, void* stream) {
    F2S_REQUIRE(rows >= 0 && cols >= 1 && K >= 1 && ldx >= K && ldy >= cols,
                "linear: bad shape rows=%d cols=%d K=%d ldx=%d ldy=%d", rows, cols, K, ldx, ldy);
    if (rows == 0) return F2S_OK;
    F2S_REQUIRE(x && weight && y, "linear: null pointer");
    cudaStream_t st = f2s::as_stream(stream);
    if (precision == F2S_PRECISION_FP32) {
        f2s::GemmArgs g{};
        g.A = static_cast<const float*>(x);
        g.lda = ldx;
        g.W = static_cast<const float*>(weight);
        g.bias = bias;
        g.Y = y;
        g.ldy = ldy;
        g.rows = rows;
        g.cols = cols;
        g.K = K;
        g.rows_per_patch = 1;
        g.epilogue = f2s::kEpiStore;
        g.tag = f2s::kTagGemmContent;
        return f2s::gemm_f32(g, st);
    }
    F2S_REQUIRE(precision == F2S_PRECISION_TF32 || precision == F2S_PRECISION_BF16 ||
                    precision == F2S_PRECISION_BF16X3,
                "linear: unknown precision %d", precision);
    f2s::TcGemmOp op{};
    op.A = x;
    op.lda = ldx;
    op.W = weight;
    if (precision == F2S_PRECISION_BF16X3) {
        // fp32 x split in the kernel; weight = bf16 high parts then low parts
        op.split_in = true;
        op.W_lo = static_cast<const __nv_bfloat16*>(weight) + (size_t)cols * K;
    }
    op.bias = bias;
    op.Y = y;
    op.ldy = ldy;
    op.rows = rows;
    op.cols = cols;
    op.K = K;
    op.bn = f2s::tc_pick_bn(cols, false);
    if (op.split_in && op.bn > 192) op.bn = f2s::tc_pick_bn(cols, true);
    op.tf32 = precision == F2S_PRECISION_TF32;
    op.epilogue = f2s::kEpiStore;
    op.rows_per_patch = 1;
    op.tag = f2s::kTagGemmContent;
    return f2s::tc_gemm(op, st);
}

namespace f2s {
namespace {
// One thread waits, with a bound of `polls`, on an mbarrier that expects one
// arrival that never comes: the bounded-wait path of every tensor-core kernel
// (give up, record kTcWaitTimeout in the error word, return) without a real
// pipeline behind it.
__global__ void wait_timeout_kernel(int* err, uint32_t polls) {
    __shared__ uint64_t bar;
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
    tc::mbar_wait(&bar, 0, err, polls);
}
}  // namespace
}  // namespace f2s

extern "C" int f2s_selftest_wait_timeout(int polls, void* stream) {
    F2S_REQUIRE(polls >= 1 && polls <= (1 << 20), "selftest: polls %d outside [1, 2^20]", polls);
    int* word = f2s::tc_error_word();
    if (!word) return f2s::fail(F2S_ERR_CUDA, "device error word unavailable");
    f2s::wait_timeout_kernel<<<1, 1, 0, f2s::as_stream(stream)>>>(word, (uint32_t)polls);
    return f2s::check_launch("wait_timeout_kernel");
}

extern "C" int f2s_device_error(int* value, int reset, void* stream) {
    F2S_REQUIRE(value != nullptr, "device_error: null pointer");
    int* word = f2s::tc_error_word();
    if (!word) return f2s::fail(F2S_ERR_CUDA, "device error word unavailable");
    cudaStream_t st = f2s::as_stream(stream);
    F2S_CUDA_TRY(cudaMemcpyAsync(value, word, sizeof(int), cudaMemcpyDeviceToHost, st));
    F2S_CUDA_TRY(cudaStreamSynchronize(st));
    if (reset) F2S_CUDA_TRY(cudaMemsetAsync(word, 0, sizeof(int), st));
    return F2S_OK;
}
