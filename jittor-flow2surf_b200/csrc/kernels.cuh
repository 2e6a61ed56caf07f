// Internal launch functions shared by the C-ABI translation units.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace f2s {

// ---- knn.cu ----
int knn_launch(const float* features, int B, int C, int N, int k, int32_t* indices,
               cudaStream_t stream);

// ---- gemm.cu ----
// Y[r, n] = sum_k A[r, k] * W[n, k] for r < rows, n < cols (A row-major with
// leading dimension lda, W row-major (cols x K)), followed by an epilogue.
enum GemmEpilogue {
    kEpiStore = 0,          // Y = acc (+ bias)
    kEpiGatedResidual = 1,  // Y += gate[r / rows_per_patch, n] * (acc (+ bias))
    kEpiSwiGlu = 2,         // Y = silu(acc_W + bias) * (acc_W2 + bias2)
};

struct GemmArgs {
    const float* A;
    int lda;
    const float* W;
    const float* bias;     // may be null
    const float* W2;       // SwiGLU value weights
    const float* bias2;    // SwiGLU value bias
    float* Y;
    int ldy;
    const float* gate;     // gated residual: (patches, gate_stride) rows
    int gate_stride;
    int rows_per_patch;
    int rows, cols, K;
    GemmEpilogue epilogue;
    int tag;               // TraceTag of this launch
    bool round_tf32;       // tensor-core path: round fp32 outputs to the nearest tf32
    // tensor-core path only: Y written as fp16 (y_fp16); A read as fp16 with the
    // fp16 copy W16 of W (fp16_operands), the MMA then kind::f16
    bool y_fp16;
    bool fp16_operands;
    const void* W16;
    const void* W2_16;     // fp16 copy of W2 (SwiGLU)
    // tensor-core plain-store path: output columns >= vt_col0 (a multiple of
    // 32) are not stored in Y but, in fp16, transposed per patch of vt_M rows
    // into vt (patch, column - vt_col0, row in patch) with row pitch vt_npad
    // (the V^T operand of attention_tc); values outside the fp16 range set
    // the device error word to 2
    __half* vt;
    int vt_col0, vt_C, vt_npad, vt_M;
    // with vt: the q and k columns [0, 96) (q / k width 48) LayerNorm'd and
    // split into the attention's bf16 rows (attention_tc_qk) instead of Y
    void* qk_hi;
    void* qk_lo;
};
int gemm_f32(const GemmArgs& args, cudaStream_t stream);

// ---- tc_gemm.cu ----
// The same contraction on tcgen05 tensor cores (TMA-fed, TMEM accumulators).
// A, W, W2 are bf16 or (tf32 = true) fp32; Y is fp32 or (y_bf16) bf16.
struct TcGemmOp {
    const void* A;
    int lda;
    const void* W;           // cols x K, K contiguous
    const void* W2;          // SwiGLU value weights (cols x K)
    const void* A_lo;        // 3xTF32: low parts of A (rows x K, lda) and W (cols x K);
    const void* W_lo;        //   A and W then hold the tf32-rounded high parts
    __half* vt;              // as GemmArgs::vt (plain store, TMA epilogue)
    int vt_col0, vt_C, vt_npad, vt_M;
    void* qk_hi;             // as GemmArgs::qk_hi / qk_lo
    void* qk_lo;
    bool split_in;           // split bf16: A is fp32 (split into bf16 high and low parts
                             //   in shared memory), W / W_lo the bf16 parts of the weights
    const float* bias;
    const float* bias2;
    void* Y;
    int ldy;
    bool y_bf16;
    bool y_fp16;             // fp16 output (TMA epilogue; out-of-range values set the error word)
    const float* gate;       // gated residual
    int gate_stride;
    int rows_per_patch;
    int rows, cols, K;
    int bn;                  // N tile: multiple of 32, <= 256 (<= 128 for SwiGLU)
    bool tf32;
    bool fp16;               // !tf32: operands are fp16 (kind::f16, F16) rather than bf16
    bool round_tf32;         // round fp32 outputs to the nearest tf32
    GemmEpilogue epilogue;
    int tag;
};
int tc_gemm(const TcGemmOp& op, cudaStream_t stream);
// hi = x rounded to the nearest tf32, lo = x - hi; hi and lo are (rows, K)
// with leading dimension K: the operand split of the 3xTF32 GEMM.
int split_tf32(const float* x, int ldx, int rows, int K, float* hi, float* lo, cudaStream_t stream);
// hi = bf16(x), lo = bf16(x - hi) (round to nearest), (rows, K) each with
// leading dimension K: the weight split of the split-bf16 GEMM.
int split_bf16(const float* x, int ldx, int rows, int K, void* hi, void* lo, cudaStream_t stream);
// N tile with the least padding for `cols` output columns.
int tc_pick_bn(int cols, bool swiglu);

// ---- rownorm.cu ----
// h = LN(x) * (1 + scale[p]) + shift[p]; LN two-pass over C, eps 1e-6.
// round_tf32: round the output to the nearest tf32 (it feeds a tf32 GEMM).
int ln_modulate(const float* x, int ldx, float* h, int ldh, const float* mod, int mod_stride,
                int scale_off, int shift_off, int rows, int rows_per_patch, int C,
                bool round_tf32, cudaStream_t stream);
// The same with h in fp16 (C even, <= 256); values out of the fp16 range set
// the device error word to 2. F2S_ERR_UNSUPPORTED outside that shape.
int ln_modulate_f16(const float* x, int ldx, void* h, int ldh, const float* mod, int mod_stride,
                    int scale_off, int shift_off, int rows, int rows_per_patch, int C,
                    cudaStream_t stream);
// y = LeakyReLU_0.2(LN(y) * gamma + beta) in place (two-pass, eps 1e-6).
int ln_affine_leaky(float* y, int ldy, const float* gamma, const float* beta, int rows, int C,
                    bool round_tf32, cudaStream_t stream);
// LN (no affine, eps 1e-6) of columns [0, d) and [d, 2d) of each row, in place.
int qk_norm(float* qkv, int ld, int rows, int d, cudaStream_t stream);

// ---- attention.cu ----
// Offset attention over point-major q, k (rows B*N, leading dim ldqk, width d)
// and v (ldv, width C); out = h - A when h is given, else A. colstats holds
// B*N floats of scratch (per-key log-sum-exp over queries).
int attention_f32(const float* q, const float* k, int ldqk, const float* v, int ldv,
                  const float* h, int ldh, float* out, int ldo, float* colstats, int B, int N,
                  int d, int C, bool round_tf32, cudaStream_t stream);

// ---- attention_tc.cu ----
// The same on tcgen05 tensor cores: q, k (width d <= 64, LayerNorm'd first
// when normalize_qk) contracted as split bf16, P V as tf32. workspace holds
// attention_tc_workspace_floats(B, N, C) floats. F2S_ERR_UNSUPPORTED for
// shapes it does not cover.
int attention_tc_workspace_floats(int B, int N, int C);
// Whether attention_tc takes this shape (else it returns F2S_ERR_UNSUPPORTED).
bool attention_tc_supported(const float* q, const float* k, int ldqk, int d, int C);
// Where attention_tc keeps V^T (fp16, (B, C, (N + 7) & ~7)) in its workspace;
// a producer that writes it there passes vt_ready.
__half* attention_tc_vt(float* workspace, int B, int N);
// Where attention_tc keeps the LayerNorm'd q / k rows as bf16 high and low
// parts (rows of [q 64 | k 64], zero padded); a producer that writes them
// passes qk_ready.
void attention_tc_qk(float* workspace, int B, int N, void** hi, void** lo);
int attention_tc(const float* q, const float* k, int ldqk, const float* v, int ldv,
                 const float* h, int ldh, float* out, int ldo, float* workspace, int B, int N,
                 int d, int C, bool normalize_qk, bool round_tf32, cudaStream_t stream,
                 bool vt_ready = false, bool qk_ready = false);

// ---- edge.cu ----
// Fused neighbour stage: per edge (i, j = idx[i, k]) the HPE hidden
// GELU(LN(W_in g + b_in)) of g = [xyz_j - xyz_i, xyz_i] (or a given geometry
// row), the composed projection W_po h + b_po, plus the content terms, LN,
// affine, LeakyReLU and the max over k.
struct EdgeArgs {
    const float* content;   // (B*M, ldc): [0, cout) neighbour term, [cout, 2cout) centre term
    int ldc;
    const float* xyz4;      // (B*M, 4) point-major xyz (model path), or null
    const float* geometry;  // (B*M*K, D) explicit geometry (operator path), or null
    int D;
    const int32_t* idx;     // (B*M, K) indices local to each patch
    int B, M, K, H, cout;
    const float* hpe_w;     // (H, D)
    const float* hpe_b;
    const float* hpe_ln_w;
    const float* hpe_ln_b;
    const float* contrib_w; // (cout, H)
    const float* contrib_b;
    const float* ln_w;
    const float* ln_b;
    float* out;             // (B*M, ldo) row-major, already offset to its column
    int ldo;
};
int edge_stage_f32(const EdgeArgs& args, cudaStream_t stream);
// The stage on tcgen05 tensor cores at F2S_PRECISION_TF32, _BF16 or _BF16X3
// (args.contrib_w is fp32 in every case). F2S_ERR_UNSUPPORTED for shapes it
// does not cover.
int edge_stage_tc(const EdgeArgs& args, int precision, cudaStream_t stream);
// The split-bf16 stage on the kernel whose warps each take both the hidden-row
// and the epilogue work (edge_tcu.cu); F2S_ERR_UNSUPPORTED for shapes it does
// not cover.
int edge_stage_unified(const EdgeArgs& args, cudaStream_t stream);

}  // namespace f2s
