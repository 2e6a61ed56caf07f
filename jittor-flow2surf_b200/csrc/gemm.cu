// fp32 SIMT GEMM for the point-wise 1x1 convolutions / linears of the model,
// with the reference's residual and SwiGLU arithmetic fused into the epilogue.
//
// Y (rows x cols) = A (rows x K, row-major) * W^T (W is cols x K, row-major):
// activations are point-major so every 1x1 conv of the reference
// (transformer.py:37-48, encoder.py:98,118-123, decoder.py:18,26) is this
// product with the conv weight used as stored.
//
// Tile 128 x 64 x 16 per CTA of 256 threads, 8 x 4 outputs per thread; the A
// tile is stored k-major in shared memory so both operands are read as float4.
#include "kernels.cuh"

namespace f2s {
namespace {

constexpr int BM = 128, BN = 64, BK = 16;

template <int EPI>
__global__ void __launch_bounds__(256) gemm_f32_kernel(const GemmArgs g) {
    __shared__ __align__(16) float As[BK][BM + 4];
    __shared__ __align__(16) float Ws[BK][BN + 4];
    __shared__ __align__(16) float W2s[EPI == kEpiSwiGlu ? BK : 1][BN + 4];

    const int tid = threadIdx.x;
    const int row0 = blockIdx.x * BM;
    const int col0 = blockIdx.y * BN;
    const int tm = tid >> 4, tn = tid & 15;

    float acc[8][4];
    float acc2[EPI == kEpiSwiGlu ? 8 : 1][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            acc[i][j] = 0.0f;
            if (EPI == kEpiSwiGlu) acc2[i][j] = 0.0f;
        }

    const int a_row = tid >> 1, a_k = (tid & 1) * 8;
    const int w_col = tid >> 2, w_k = (tid & 3) * 4;
    const int ar = row0 + a_row;
    const int wn = col0 + w_col;

    for (int k0 = 0; k0 < g.K; k0 += BK) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int k = k0 + a_k + i;
            As[a_k + i][a_row] = (ar < g.rows && k < g.K) ? g.A[(size_t)ar * g.lda + k] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = k0 + w_k + i;
            const bool in = wn < g.cols && k < g.K;
            Ws[w_k + i][w_col] = in ? g.W[(size_t)wn * g.K + k] : 0.0f;
            if (EPI == kEpiSwiGlu) W2s[w_k + i][w_col] = in ? g.W2[(size_t)wn * g.K + k] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][tm * 8]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][tm * 8 + 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float4 b = *reinterpret_cast<const float4*>(&Ws[kk][tn * 4]);
            const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            if (EPI == kEpiSwiGlu) {
                const float4 c = *reinterpret_cast<const float4*>(&W2s[kk][tn * 4]);
                const float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc2[i][j] = fmaf(av[i], cv[j], acc2[i][j]);
            }
        }
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = row0 + tm * 8 + i;
        if (r >= g.rows) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = col0 + tn * 4 + j;
            if (n >= g.cols) continue;
            float v = acc[i][j] + (g.bias ? g.bias[n] : 0.0f);
            float* y = g.Y + (size_t)r * g.ldy + n;
            if (EPI == kEpiStore) {
                *y = v;
            } else if (EPI == kEpiGatedResidual) {
                const float gate = g.gate[(size_t)(r / g.rows_per_patch) * g.gate_stride + n];
                *y = *y + gate * v;
            } else {
                const float u = acc2[i][j] + (g.bias2 ? g.bias2[n] : 0.0f);
                *y = f2s_silu(v) * u;
            }
        }
    }
}

}  // namespace

int gemm_f32(const GemmArgs& g, cudaStream_t stream) {
    if (g.rows == 0 || g.cols == 0) return F2S_OK;
    F2S_REQUIRE(g.A && g.W && g.Y && g.K > 0, "gemm: bad operands");
    F2S_REQUIRE(g.epilogue != kEpiSwiGlu || g.W2, "gemm: SwiGLU needs W2");
    F2S_REQUIRE(g.epilogue != kEpiGatedResidual || (g.gate && g.rows_per_patch > 0),
                "gemm: gated residual needs gate");
    dim3 grid(ceil_div(g.rows, BM), ceil_div(g.cols, BN));
    TraceScope trace(g.tag, stream);
    F2S_LIMIT(grid.y <= 65535, "gemm: cols too large");
    switch (g.epilogue) {
        case kEpiStore: gemm_f32_kernel<kEpiStore><<<grid, 256, 0, stream>>>(g); break;
        case kEpiGatedResidual:
            gemm_f32_kernel<kEpiGatedResidual><<<grid, 256, 0, stream>>>(g);
            break;
        case kEpiSwiGlu: gemm_f32_kernel<kEpiSwiGlu><<<grid, 256, 0, stream>>>(g); break;
    }
    return check_launch("gemm_f32_kernel");
}

}  // namespace f2s
