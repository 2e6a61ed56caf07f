// Training gradients and losses: the backward passes of the reference's
// custom operators and its point-set losses.
//
// Reference semantics:
//   nearest_distance_backward.cu:11-40 (training/distances.py:40-62)
//   training/losses.py:8-47 (dcd_loss, velocity_loss)
//   hpe_activation_backward.cu:10-66 (models/ops/hpe.py:54-84)
//   neighbor_reduce_backward.cu:20-84 and neighbor_reduce.py:155-237
//   offset_attention_backward.cu + offset_attention.cuh:130-208
//
// B200 design: CUDA-core fp32 kernels (the reference's arithmetic), a warp
// per row for the normalisation backwards with the row held in registers,
// per-block partial sums reduced in a fixed order for every parameter
// gradient (deterministic; only the scatters into shared inputs -- the
// nearest backward's and the neighbour rows' -- use float atomics, as the
// reference's kernels do), and the attention backward as tiled batched
// products over a materialised probability tile per batch item.
#include <cfloat>

#include "kernels.cuh"

namespace f2s {

int transpose_batched(const float* in, float* out, int B, int rows, int cols,
                      cudaStream_t stream);

namespace {

constexpr int kBlock = 256;

int blocks_for(int64_t work, int per_block = kBlock) {
    const int64_t b = (work + per_block - 1) / per_block;
    const int64_t cap = (int64_t)sm_count() * 32;
    return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ---------------------------------------------------------------------------
// Column sums of per-block partials in a fixed order: out[c] = sum over p of
// part[p * pitch + c], in float64.
// ---------------------------------------------------------------------------
__global__ void sum_partials_kernel(const float* __restrict__ part, int parts, int cols,
                                    int pitch, float* __restrict__ out) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    double s = 0.0;
    for (int p = 0; p < parts; ++p) s += (double)part[(size_t)p * pitch + c];
    out[c] = (float)s;
}

int sum_partials(const float* part, int parts, int cols, float* out, cudaStream_t st) {
    sum_partials_kernel<<<(cols + 255) / 256, 256, 0, st>>>(part, parts, cols, cols, out);
    return check_launch("sum_partials_kernel");
}

// the same with partial rows pitch floats apart (cols <= pitch)
int sum_partials_strided(const float* part, int parts, int cols, int pitch, float* out,
                         cudaStream_t st) {
    sum_partials_kernel<<<(cols + 255) / 256, 256, 0, st>>>(part, parts, cols, pitch, out);
    return check_launch("sum_partials_kernel");
}

// ---------------------------------------------------------------------------
// Nearest squared distances: coordinate gradients
// ---------------------------------------------------------------------------

// Own terms, stored: grad_first[b, i] = 2 g1 (first_i - second_j(i)), and the
// same for the second set (a missing distance gradient counts as zero).
__global__ void nearest_grad_own_kernel(const float* __restrict__ first,
                                        const float* __restrict__ second, int B, int M, int N,
                                        const int32_t* __restrict__ second_index,
                                        const int32_t* __restrict__ first_index,
                                        const float* __restrict__ g1, const float* __restrict__ g2,
                                        float* __restrict__ grad_first,
                                        float* __restrict__ grad_second) {
    const int64_t n1 = (int64_t)B * M, total = n1 + (int64_t)B * N;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const bool one = e < n1;
        const int64_t r = one ? e : e - n1;
        const int b = (int)(r / (one ? M : N));
        const float* self = one ? first + r * 3 : second + r * 3;
        const float g = one ? (g1 ? g1[r] : 0.0f) : (g2 ? g2[r] : 0.0f);
        const int j = one ? second_index[r] : first_index[r];
        const int other_n = one ? N : M;
        float* out = one ? grad_first + r * 3 : grad_second + r * 3;
        if (j < 0 || j >= other_n) {
            out[0] = out[1] = out[2] = 0.0f;
            continue;
        }
        const float* o = (one ? second : first) + ((int64_t)b * other_n + j) * 3;
        const float scale = 2.0f * g;
        for (int c = 0; c < 3; ++c) out[c] = scale * (self[c] - o[c]);
    }
}

// The matched points' terms, added: grad_second[b, j(i)] -= 2 g1 (first_i -
// second_j), and the same the other way.
__global__ void nearest_grad_scatter_kernel(const float* __restrict__ first,
                                            const float* __restrict__ second, int B, int M, int N,
                                            const int32_t* __restrict__ second_index,
                                            const int32_t* __restrict__ first_index,
                                            const float* __restrict__ g1,
                                            const float* __restrict__ g2,
                                            float* __restrict__ grad_first,
                                            float* __restrict__ grad_second) {
    const int64_t n1 = (int64_t)B * M, total = n1 + (int64_t)B * N;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const bool one = e < n1;
        const int64_t r = one ? e : e - n1;
        const float* gv = one ? g1 : g2;
        if (!gv) continue;
        const int b = (int)(r / (one ? M : N));
        const int j = one ? second_index[r] : first_index[r];
        const int other_n = one ? N : M;
        if (j < 0 || j >= other_n) continue;
        const float* self = one ? first + r * 3 : second + r * 3;
        const float* o = (one ? second : first) + ((int64_t)b * other_n + j) * 3;
        float* out = (one ? grad_second : grad_first) + ((int64_t)b * other_n + j) * 3;
        const float scale = 2.0f * gv[r];
        for (int c = 0; c < 3; ++c) atomicAdd(&out[c], -(scale * (self[c] - o[c])));
    }
}

int nearest_backward(const float* first, const float* second, int B, int M, int N,
                     const int32_t* second_index, const int32_t* first_index, const float* g1,
                     const float* g2, float* grad_first, float* grad_second, cudaStream_t st) {
    const int64_t total = (int64_t)B * ((int64_t)M + N);
    nearest_grad_own_kernel<<<blocks_for(total), kBlock, 0, st>>>(
        first, second, B, M, N, second_index, first_index, g1, g2, grad_first, grad_second);
    F2S_TRY(check_launch("nearest_grad_own_kernel"));
    nearest_grad_scatter_kernel<<<blocks_for(total), kBlock, 0, st>>>(
        first, second, B, M, N, second_index, first_index, g1, g2, grad_first, grad_second);
    return check_launch("nearest_grad_scatter_kernel");
}

// ---------------------------------------------------------------------------
// Density-aware Chamfer loss (training/losses.py:8-41)
// ---------------------------------------------------------------------------

// Nearest-neighbour multiplicities: how many points of the other set chose
// each point.
__global__ void dcd_count_kernel(const int32_t* __restrict__ second_index,
                                 const int32_t* __restrict__ first_index, int B, int M, int N,
                                 int* __restrict__ target_mult, int* __restrict__ pred_mult) {
    const int64_t n1 = (int64_t)B * M, total = n1 + (int64_t)B * N;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        if (e < n1) {
            const int b = (int)(e / M);
            const int j = second_index[e];
            if (j >= 0 && j < N) atomicAdd(&target_mult[(int64_t)b * N + j], 1);
        } else {
            const int64_t r = e - n1;
            const int b = (int)(r / N);
            const int i = first_index[r];
            if (i >= 0 && i < M) atomicAdd(&pred_mult[(int64_t)b * M + i], 1);
        }
    }
}

// One block per batch item: loss[b] = 0.5 (mean_i (1 - w1 e^{-alpha d1}) +
// mean_j (1 - w2 e^{-alpha d2})) with w = 1 / max(multiplicity, 1), summed in
// float64 in a fixed order; with gd1 / gd2, the loss's derivative with
// respect to each distance times grad_loss[b] (one when absent).
__global__ void __launch_bounds__(1024)
dcd_terms_kernel(const float* __restrict__ d1, const int32_t* __restrict__ i2,
                 const float* __restrict__ d2, const int32_t* __restrict__ i1, int M, int N,
                 const int* __restrict__ target_mult, const int* __restrict__ pred_mult,
                 float alpha, const float* __restrict__ grad_loss, float* __restrict__ loss,
                 float* __restrict__ gd1, float* __restrict__ gd2) {
    __shared__ double red[32];
    const int b = blockIdx.x;
    const float gl = grad_loss ? grad_loss[b] : 1.0f;
    const float s1 = 0.5f / (float)M, s2 = 0.5f / (float)N;
    double a1 = 0.0, a2 = 0.0;
    for (int i = threadIdx.x; i < M; i += blockDim.x) {
        const int64_t r = (int64_t)b * M + i;
        const int j = i2[r];
        const int m = (j >= 0 && j < N) ? target_mult[(int64_t)b * N + j] : 0;
        const float w = 1.0f / fmaxf((float)m, 1.0f);
        const float e = expf(-alpha * d1[r]);
        a1 += (double)(1.0f - w * e);
        if (gd1) gd1[r] = gl * s1 * w * alpha * e;
    }
    for (int j = threadIdx.x; j < N; j += blockDim.x) {
        const int64_t r = (int64_t)b * N + j;
        const int i = i1[r];
        const int m = (i >= 0 && i < M) ? pred_mult[(int64_t)b * M + i] : 0;
        const float w = 1.0f / fmaxf((float)m, 1.0f);
        const float e = expf(-alpha * d2[r]);
        a2 += (double)(1.0f - w * e);
        if (gd2) gd2[r] = gl * s2 * w * alpha * e;
    }
    double v = a1 / (double)M + a2 / (double)N;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) loss[b] = (float)(0.5 * v);
    }
}

struct DcdSpace {
    size_t d1, i2, d2, i1, tm, pm, gd1, gd2, nearest, bytes;
};

DcdSpace dcd_space(int B, int M, int N) {
    DcdSpace s;
    const size_t bm = (size_t)B * M, bn = (size_t)B * N;
    s.d1 = 0;
    s.i2 = align256(s.d1 + bm * 4);
    s.d2 = align256(s.i2 + bm * 4);
    s.i1 = align256(s.d2 + bn * 4);
    s.tm = align256(s.i1 + bn * 4);
    s.pm = align256(s.tm + bn * 4);
    s.gd1 = align256(s.pm + bm * 4);
    s.gd2 = align256(s.gd1 + bm * 4);
    s.nearest = align256(s.gd2 + bn * 4);
    size_t nb = 0;
    f2s_nearest_workspace_bytes(B, M, N, &nb);
    s.bytes = s.nearest + nb;
    return s;
}

// ---------------------------------------------------------------------------
// Velocity loss (training/losses.py:44-47)
// ---------------------------------------------------------------------------

// One block per batch item: loss[b] = mean_m sum_c (p - t)^2 (float64 sums,
// fixed order); the gradients 2 (p - t) / M grad_loss[b] and its negative.
__global__ void __launch_bounds__(1024)
velocity_loss_kernel(const float* __restrict__ pred, const float* __restrict__ target, int M,
                     const float* __restrict__ grad_loss, float* __restrict__ loss,
                     float* __restrict__ grad_pred, float* __restrict__ grad_target) {
    __shared__ double red[32];
    const int b = blockIdx.x;
    const float gl = grad_loss ? grad_loss[b] : 1.0f;
    const float scale = 2.0f / (float)M * gl;
    double acc = 0.0;
    for (int e = threadIdx.x; e < 3 * M; e += blockDim.x) {
        const int64_t r = (int64_t)b * 3 * M + e;
        const float d = pred[r] - target[r];
        acc += (double)(d * d);
        if (grad_pred) grad_pred[r] = scale * d;
        if (grad_target) grad_target[r] = -(scale * d);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        acc = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (threadIdx.x == 0 && loss) loss[b] = (float)(acc / (double)M);
    }
}

// ---------------------------------------------------------------------------
// Warp helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// The per-lane channel accumulators of the warps of a block summed into one
// row of part (cols channels, lane + 32 t of each warp; red: 8 x cols floats).
template <int kCPL>
__device__ __forceinline__ void block_channel_partial(const float (&acc)[kCPL], int cols,
                                                      float* red, float* part_row) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int t = 0; t < kCPL; ++t) {
        const int c = lane + 32 * t;
        if (c < cols) red[warp * cols + c] = acc[t];
    }
    __syncthreads();
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        float s = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w * cols + c];
        part_row[c] = s;
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// HPE activation backward (hpe_activation_backward.cu:10-66)
// ---------------------------------------------------------------------------

// A warp per row of H <= 32 kCPL channels: the moment LayerNorm (eps 1e-5,
// raw variance clamped at zero) and the exact GELU recomputed, then
// grad_pre = inv_std (gn - mean(gn) - [var > 0] normalized mean(gn normalized))
// with gn = grad_hidden GELU'(affine) weight; the weight and bias gradients
// into per-block partial rows.
template <int kCPL>
__global__ void __launch_bounds__(kBlock)
hpe_grad_kernel(const float* __restrict__ pre, int64_t rows, int H,
                const float* __restrict__ weight, const float* __restrict__ bias,
                const float* grad_hidden, float* grad_pre,  // may be the same rows
                float* __restrict__ part_w, float* __restrict__ part_b) {
    extern __shared__ float red[];  // [8][H]
    const int lane = threadIdx.x & 31;
    const int wpb = blockDim.x >> 5;
    float wv[kCPL], bv[kCPL], aw[kCPL], ab[kCPL];
#pragma unroll
    for (int t = 0; t < kCPL; ++t) {
        const int c = lane + 32 * t;
        wv[t] = c < H ? weight[c] : 0.0f;
        bv[t] = c < H ? bias[c] : 0.0f;
        aw[t] = ab[t] = 0.0f;
    }
    const float inv_h = 1.0f / (float)H;
    for (int64_t row = (int64_t)blockIdx.x * wpb + (threadIdx.x >> 5); row < rows;
         row += (int64_t)gridDim.x * wpb) {
        float v[kCPL], g[kCPL];
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
        for (int t = 0; t < kCPL; ++t) {
            const int c = lane + 32 * t;
            v[t] = c < H ? pre[row * H + c] : 0.0f;
            g[t] = c < H ? grad_hidden[row * H + c] : 0.0f;
            s1 += v[t];
            s2 += v[t] * v[t];
        }
        s1 = warp_sum(s1);
        s2 = warp_sum(s2);
        const float mean = s1 * inv_h;
        const float raw_var = s2 * inv_h - mean * mean;
        const float inv_std = rsqrtf(fmaxf(raw_var, 0.0f) + 1e-5f);
        float nrm[kCPL], gn[kCPL];
        float t1 = 0.0f, t2 = 0.0f;
#pragma unroll
        for (int t = 0; t < kCPL; ++t) {
            const int c = lane + 32 * t;
            nrm[t] = 0.0f;
            gn[t] = 0.0f;
            if (c < H) {
                nrm[t] = (v[t] - mean) * inv_std;
                const float a = nrm[t] * wv[t] + bv[t];
                const float cdf = 0.5f * (erff(a * 0.7071067811865475f) + 1.0f);
                const float density = expf(-0.5f * a * a) * 0.3989422804014327f;
                const float ga = g[t] * (cdf + a * density);
                aw[t] += ga * nrm[t];
                ab[t] += ga;
                gn[t] = ga * wv[t];
            }
            t1 += gn[t];
            t2 += gn[t] * nrm[t];
        }
        t1 = warp_sum(t1);
        t2 = warp_sum(t2);
#pragma unroll
        for (int t = 0; t < kCPL; ++t) {
            const int c = lane + 32 * t;
            if (c < H) {
                const float vg = raw_var > 0.0f ? nrm[t] * t2 * inv_h : 0.0f;
                grad_pre[row * H + c] = inv_std * (gn[t] - t1 * inv_h - vg);
            }
        }
    }
    block_channel_partial<kCPL>(aw, H, red, part_w + (size_t)blockIdx.x * H);
    block_channel_partial<kCPL>(ab, H, red, part_b + (size_t)blockIdx.x * H);
}

int hpe_grad_blocks(int64_t rows) {
    const int64_t b = (rows + 7) / 8;
    const int64_t cap = (int64_t)sm_count() * 8;
    return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

int hpe_activation_backward(const float* pre, int64_t rows, int H, const float* w,
                            const float* b, const float* grad_hidden, float* grad_pre,
                            float* grad_w, float* grad_b, float* part, cudaStream_t st) {
    const int blocks = hpe_grad_blocks(rows);
    float* part_w = part;
    float* part_b = part + (size_t)blocks * H;
    const size_t smem = (size_t)8 * H * sizeof(float);
#define F2S_HPE_GRAD(CPL)                                                                   \
    hpe_grad_kernel<CPL><<<blocks, kBlock, smem, st>>>(pre, rows, H, w, b, grad_hidden,    \
                                                       grad_pre, part_w, part_b)
    const int cpl = (H + 31) / 32;
    if (cpl <= 1) F2S_HPE_GRAD(1);
    else if (cpl <= 2) F2S_HPE_GRAD(2);
    else if (cpl <= 4) F2S_HPE_GRAD(4);
    else F2S_HPE_GRAD(8);
#undef F2S_HPE_GRAD
    F2S_TRY(check_launch("hpe_grad_kernel"));
    F2S_TRY(sum_partials(part_w, blocks, H, grad_w, st));
    return sum_partials(part_b, blocks, H, grad_b, st);
}

// ---------------------------------------------------------------------------
// Neighbour-message reduction backward (neighbor_reduce_backward.cu:20-84)
// ---------------------------------------------------------------------------

// The message of edge k of point n, channels lane + 32 t, normalised: returns
// the activation in act (LeakyReLU 0.2 of the affine LayerNorm, two-pass,
// eps 1e-6), the normalised values, slope and inv_std.
template <int kCPL>
__device__ __forceinline__ void edge_message(const float* __restrict__ content_pm,
                                             const float* __restrict__ contribution, int64_t b,
                                             int n, int j, int64_t edge, int C, int N,
                                             const float (&center)[kCPL], const float (&wv)[kCPL],
                                             const float (&bv)[kCPL], float (&nrm)[kCPL],
                                             float (&act)[kCPL], float (&slope)[kCPL],
                                             float& inv_std) {
    const int lane = threadIdx.x & 31;
    const float inv_c = 1.0f / (float)C;
    float m[kCPL];
    float s = 0.0f;
#pragma unroll
    for (int t = 0; t < kCPL; ++t) {
        const int c = lane + 32 * t;
        m[t] = c < C ? content_pm[(b * N + j) * 2 * C + c] + center[t] + contribution[edge * C + c]
                     : 0.0f;
        s += m[t];
    }
    const float mean = warp_sum(s) * inv_c;
    float q = 0.0f;
#pragma unroll
    for (int t = 0; t < kCPL; ++t) {
        const int c = lane + 32 * t;
        m[t] = c < C ? m[t] - mean : 0.0f;
        q += m[t] * m[t];
    }
    inv_std = rsqrtf(warp_sum(q) * inv_c + 1e-6f);
#pragma unroll
    for (int t = 0; t < kCPL; ++t) {
        nrm[t] = m[t] * inv_std;
        const float a = nrm[t] * wv[t] + bv[t];
        act[t] = a > 0.0f ? a : 0.2f * a;
        slope[t] = a > 0.0f ? 1.0f : 0.2f;
    }
}

// A warp per point, on a point-major copy of the content (B, N, 2C): the K
// edges' activations recomputed once for the maximum of each channel, then
// again to route the upstream gradient to every edge that reaches it (all
// exact ties), through the LayerNorm to the message: grad_contribution[edge]
// stored, the neighbour part added into row j of the point-major gradient
// grad_pm (B, N, 2C) (atomics, channels [0, C)), the centre part summed into
// channels [C, 2C) of row n; the norm weight / bias gradients into per-block
// partial rows. A neighbour index outside [0, N) reads the point itself and
// scatters nothing.
template <int kCPL>
__global__ void __launch_bounds__(kBlock)
messages_grad_kernel(const float* __restrict__ content, const float* __restrict__ contribution,
                     const int32_t* __restrict__ indices, int B, int N, int K, int C,
                     const float* __restrict__ weight, const float* __restrict__ bias,
                     const float* __restrict__ grad_output, float* __restrict__ grad_pm,
                     float* __restrict__ grad_contribution, float* __restrict__ part_w,
                     float* __restrict__ part_b) {
    extern __shared__ float red[];  // [8][C]
    const int lane = threadIdx.x & 31;
    const int wpb = blockDim.x >> 5;
    float wv[kCPL], bv[kCPL], aw[kCPL], ab[kCPL];
#pragma unroll
    for (int t = 0; t < kCPL; ++t) {
        const int c = lane + 32 * t;
        wv[t] = c < C ? weight[c] : 0.0f;
        bv[t] = c < C ? bias[c] : 0.0f;
        aw[t] = ab[t] = 0.0f;
    }
    const float inv_c = 1.0f / (float)C;
    const int64_t points = (int64_t)B * N;
    for (int64_t p = (int64_t)blockIdx.x * wpb + (threadIdx.x >> 5); p < points;
         p += (int64_t)gridDim.x * wpb) {
        const int64_t b = p / N;
        const int n = (int)(p - b * N);
        float center[kCPL], up[kCPL], mx[kCPL], csum[kCPL];
#pragma unroll
        for (int t = 0; t < kCPL; ++t) {
            const int c = lane + 32 * t;
            center[t] = c < C ? content[(b * N + n) * 2 * C + C + c] : 0.0f;
            up[t] = c < C ? grad_output[(b * C + c) * N + n] : 0.0f;
            mx[t] = -FLT_MAX;
            csum[t] = 0.0f;
        }
        float nrm[kCPL], act[kCPL], slope[kCPL], inv_std;
        for (int k = 0; k < K; ++k) {
            const int64_t edge = p * K + k;
            int j = indices[edge];
            j = (j >= 0 && j < N) ? j : n;
            edge_message<kCPL>(content, contribution, b, n, j, edge, C, N, center, wv, bv, nrm, act,
                               slope, inv_std);
#pragma unroll
            for (int t = 0; t < kCPL; ++t) mx[t] = fmaxf(mx[t], act[t]);
        }
        for (int k = 0; k < K; ++k) {
            const int64_t edge = p * K + k;
            const int jr = indices[edge];
            const bool valid = jr >= 0 && jr < N;
            const int j = valid ? jr : n;
            edge_message<kCPL>(content, contribution, b, n, j, edge, C, N, center, wv, bv, nrm, act,
                               slope, inv_std);
            float wt[kCPL];
            float t1 = 0.0f, t2 = 0.0f;
#pragma unroll
            for (int t = 0; t < kCPL; ++t) {
                const int c = lane + 32 * t;
                const float u = (c < C && act[t] == mx[t]) ? up[t] * slope[t] : 0.0f;
                aw[t] += u * nrm[t];
                ab[t] += u;
                wt[t] = u * wv[t];
                t1 += wt[t];
                t2 += wt[t] * nrm[t];
            }
            t1 = warp_sum(t1) * inv_c;
            t2 = warp_sum(t2) * inv_c;
#pragma unroll
            for (int t = 0; t < kCPL; ++t) {
                const int c = lane + 32 * t;
                if (c < C) {
                    const float gr = inv_std * (wt[t] - t1 - nrm[t] * t2);
                    grad_contribution[edge * C + c] = gr;
                    if (valid) atomicAdd(&grad_pm[(b * N + j) * 2 * C + c], gr);
                    csum[t] += gr;
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kCPL; ++t) {
            const int c = lane + 32 * t;
            if (c < C) grad_pm[(b * N + n) * 2 * C + C + c] = csum[t];
        }
    }
    block_channel_partial<kCPL>(aw, C, red, part_w + (size_t)blockIdx.x * C);
    block_channel_partial<kCPL>(ab, C, red, part_b + (size_t)blockIdx.x * C);
}

int messages_grad_blocks(int64_t points) {
    const int64_t b = (points + 7) / 8;
    const int64_t cap = (int64_t)sm_count() * 8;
    return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

// content_pm and grad_pm: B * N * 2C floats each of workspace.
int messages_backward(const float* content, const float* contribution, const int32_t* indices,
                      int B, int N, int K, int C, const float* w, const float* b,
                      const float* grad_output, float* grad_content, float* grad_contribution,
                      float* grad_w, float* grad_b, float* part, float* content_pm,
                      float* grad_pm, cudaStream_t st) {
    const int64_t points = (int64_t)B * N;
    F2S_TRY(transpose_batched(content, content_pm, B, 2 * C, N, st));
    F2S_CUDA_TRY(cudaMemsetAsync(grad_pm, 0, (size_t)points * 2 * C * sizeof(float), st));
    const int blocks = messages_grad_blocks(points);
    float* part_w = part;
    float* part_b = part + (size_t)blocks * C;
    const size_t smem = (size_t)8 * C * sizeof(float);
#define F2S_MSG_GRAD(CPL)                                                                      \
    messages_grad_kernel<CPL><<<blocks, kBlock, smem, st>>>(content_pm, contribution, indices, \
                                                            B, N, K, C, w, b, grad_output,     \
                                                            grad_pm, grad_contribution,        \
                                                            part_w, part_b)
    const int cpl = (C + 31) / 32;
    if (cpl <= 1) F2S_MSG_GRAD(1);
    else if (cpl <= 2) F2S_MSG_GRAD(2);
    else if (cpl <= 4) F2S_MSG_GRAD(4);
    else if (cpl <= 6) F2S_MSG_GRAD(6);
    else F2S_MSG_GRAD(8);
#undef F2S_MSG_GRAD
    F2S_TRY(check_launch("messages_grad_kernel"));
    F2S_TRY(transpose_batched(grad_pm, grad_content, B, N, 2 * C, st));
    F2S_TRY(sum_partials(part_w, blocks, C, grad_w, st));
    return sum_partials(part_b, blocks, C, grad_b, st);
}

// ---------------------------------------------------------------------------
// The full reduce_neighbor_messages backward (neighbor_reduce.py:155-237):
// HPE recompute, the projection products and the parameter reductions
// ---------------------------------------------------------------------------

// A warp per edge row: pre = W_in g + b_in (D <= 8 inputs), then the moment
// LayerNorm (eps 1e-5) and the exact GELU (hpe.py:14-27); pre and hidden
// stored (R x H).
template <int kCPL>
__global__ void __launch_bounds__(kBlock)
hpe_forward_rows_kernel(const float* __restrict__ geometry, int64_t rows, int D, int H,
                        const float* __restrict__ w_in, const float* __restrict__ b_in,
                        const float* __restrict__ norm_w, const float* __restrict__ norm_b,
                        float* __restrict__ pre_out, float* __restrict__ hidden) {
    const int lane = threadIdx.x & 31;
    const int wpb = blockDim.x >> 5;
    const float inv_h = 1.0f / (float)H;
    for (int64_t row = (int64_t)blockIdx.x * wpb + (threadIdx.x >> 5); row < rows;
         row += (int64_t)gridDim.x * wpb) {
        float g[8];
#pragma unroll
        for (int d = 0; d < 8; ++d) g[d] = d < D ? geometry[row * D + d] : 0.0f;
        float v[kCPL];
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
        for (int t = 0; t < kCPL; ++t) {
            const int h = lane + 32 * t;
            float a = 0.0f;
            if (h < H) {
                a = b_in[h];
#pragma unroll
                for (int d = 0; d < 8; ++d)
                    if (d < D) a += w_in[h * D + d] * g[d];
                pre_out[row * H + h] = a;
            }
            v[t] = a;
            s1 += a;
            s2 += a * a;
        }
        const float mean = warp_sum(s1) * inv_h;
        const float var = fmaxf(warp_sum(s2) * inv_h - mean * mean, 0.0f);
        const float inv_std = rsqrtf(var + 1e-5f);
#pragma unroll
        for (int t = 0; t < kCPL; ++t) {
            const int h = lane + 32 * t;
            if (h < H) {
                const float x = (v[t] - mean) * inv_std * norm_w[h] + norm_b[h];
                hidden[row * H + h] = 0.5f * x * (1.0f + erff(x * 0.7071067811865475f));
            }
        }
    }
}

// out (cols x rows) = in (rows x cols) transposed (small weights)
__global__ void transpose_small_kernel(const float* __restrict__ in, int rows, int cols,
                                       float* __restrict__ out) {
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < rows * cols;
         e += gridDim.x * blockDim.x) {
        const int r = e / cols, c = e - r * cols;
        out[(size_t)c * rows + r] = in[e];
    }
}

// Partial sums over a slice of rows of X^T Y (X: R x I, Y: R x J, row-major):
// part[s][i][j], and with colsum the slice's column sums of X into
// colsum[s][i] (from the blocks of the first j tile); blockIdx.z = slice s
// of rows_per_slice rows, a 96 x 128 tile of (i, j) per block of 256 threads
// (16 x 16, 6 x 8 outputs each), 16 rows a step, the next step's rows
// loaded into registers while the current one is multiplied (two
// shared-memory buffers).
constexpr int kXtyI = 96, kXtyJ = 128;

__global__ void __launch_bounds__(256)
xty_partial_kernel(const float* __restrict__ X, int I, const float* __restrict__ Y, int J,
                   int64_t R, int64_t rows_per_slice, float* __restrict__ part,
                   float* __restrict__ colsum) {
    __shared__ __align__(16) float xs[2][16][kXtyI + 4], ys[2][16][kXtyJ + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int i0 = blockIdx.x * kXtyI, j0 = blockIdx.y * kXtyJ;
    const int64_t r_lo = (int64_t)blockIdx.z * rows_per_slice;
    const int64_t r_hi = r_lo + rows_per_slice < R ? r_lo + rows_per_slice : R;
    float acc[6][8] = {};
    float cs[6] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    const bool sums = colsum != nullptr && blockIdx.y == 0 && tx == 0;
    // staging: X rows 16 x 96 (6 per thread), Y rows 16 x 128 (8 per thread)
    float xr[6], yr[8];
    auto fetch = [&](int64_t r0) {
#pragma unroll
        for (int u = 0; u < 6; ++u) {
            const int e = threadIdx.x + 256 * u, rr = e / kXtyI, cc = e - rr * kXtyI;
            const int64_t r = r0 + rr;
            xr[u] = (r < r_hi && i0 + cc < I) ? X[r * I + i0 + cc] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int e = threadIdx.x + 256 * u, rr = e >> 7, cc = e & 127;
            const int64_t r = r0 + rr;
            yr[u] = (r < r_hi && j0 + cc < J) ? Y[r * J + j0 + cc] : 0.0f;
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int u = 0; u < 6; ++u) {
            const int e = threadIdx.x + 256 * u, rr = e / kXtyI, cc = e - rr * kXtyI;
            xs[buf][rr][cc] = xr[u];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int e = threadIdx.x + 256 * u, rr = e >> 7, cc = e & 127;
            ys[buf][rr][cc] = yr[u];
        }
    };
    fetch(r_lo);
    stash(0);
    __syncthreads();
    int buf = 0;
    for (int64_t r0 = r_lo; r0 < r_hi; r0 += 16) {
        const bool more = r0 + 16 < r_hi;
        if (more) fetch(r0 + 16);
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
            // this thread's rows i0 + 6 ty .. + 5 and columns j0 + 4 tx, + 64
            // (6 ty floats = 24 ty bytes: 8-byte aligned, so three 8-byte
            // loads; the Y columns 4 tx and 64 + 4 tx are 16-byte aligned)
            const float2 a0 = *reinterpret_cast<const float2*>(&xs[buf][rr][ty * 6]);
            const float2 a1 = *reinterpret_cast<const float2*>(&xs[buf][rr][ty * 6 + 2]);
            const float2 a2 = *reinterpret_cast<const float2*>(&xs[buf][rr][ty * 6 + 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&ys[buf][rr][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&ys[buf][rr][64 + tx * 4]);
            const float a[6] = {a0.x, a0.y, a1.x, a1.y, a2.x, a2.y};
            const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int u = 0; u < 6; ++u) {
                cs[u] += a[u];
#pragma unroll
                for (int v = 0; v < 8; ++v) acc[u][v] += a[u] * bv[v];
            }
        }
        if (more) {
            stash(buf ^ 1);  // the other buffer: its last readers passed the barrier below
            __syncthreads();
            buf ^= 1;
        }
    }
#pragma unroll
    for (int u = 0; u < 6; ++u) {
        const int i = i0 + ty * 6 + u;
        if (i >= I) continue;
        if (sums) colsum[(size_t)blockIdx.z * I + i] = cs[u];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const int j = j0 + (v < 4 ? tx * 4 + v : 64 + tx * 4 + v - 4);
            if (j < J) part[((size_t)blockIdx.z * I + i) * J + j] = acc[u][v];
        }
    }
}

constexpr int kSlices = 256;  // row slices of the parameter reductions
constexpr int kWgradSlices = 2048;  // row slices of the input projection's weight gradient

int64_t slice_rows(int64_t R) { return (R + kSlices - 1) / kSlices; }

// out (I x J) = X^T Y and, with colsum, colsum = the column sums of X
// (part: slices x (I x J + I) floats).
int xty(const float* X, int I, const float* Y, int J, int64_t R, float* out, float* colsum,
        float* part, cudaStream_t st) {
    const int64_t per = slice_rows(R);
    const int slices = (int)((R + per - 1) / per);
    float* part_cs = part + (size_t)slices * I * J;
    xty_partial_kernel<<<dim3((I + kXtyI - 1) / kXtyI, (J + kXtyJ - 1) / kXtyJ, slices), 256, 0, st>>>(
        X, I, Y, J, R, per, part, colsum ? part_cs : nullptr);
    F2S_TRY(check_launch("xty_partial_kernel"));
    F2S_TRY(sum_partials(part, slices, I * J, out, st));
    if (!colsum) return F2S_OK;
    return sum_partials(part_cs, slices, I, colsum, st);
}

// One thread per edge row: grad_geometry[r][d] = sum_h grad_pre[r][h]
// W_in[h][d] (D <= 8), W_in broadcast from shared memory; the row read as
// 16-byte chunks when H is a multiple of 4 (rows 16-byte aligned), else by
// single floats.
__global__ void __launch_bounds__(kBlock)
geometry_grad_kernel(const float* __restrict__ grad_pre, int64_t rows, int H, int D,
                     const float* __restrict__ w_in, float* __restrict__ grad_geometry) {
    extern __shared__ float wsm[];  // [H][D]
    for (int e = threadIdx.x; e < H * D; e += blockDim.x) wsm[e] = w_in[e];
    __syncthreads();
    const bool vec = (H & 3) == 0;
    for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < rows;
         row += (int64_t)gridDim.x * blockDim.x) {
        const float* gr = grad_pre + row * H;
        float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        for (int h4 = 0; h4 < (H + 3) / 4; ++h4) {
            float gv[4];
            if (vec) {
                const float4 g = reinterpret_cast<const float4*>(gr)[h4];
                gv[0] = g.x;
                gv[1] = g.y;
                gv[2] = g.z;
                gv[3] = g.w;
            } else {
#pragma unroll
                for (int u = 0; u < 4; ++u) gv[u] = 4 * h4 + u < H ? gr[4 * h4 + u] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (4 * h4 + u >= H) break;
                const float* w = wsm + (4 * h4 + u) * D;
#pragma unroll
                for (int d = 0; d < 8; ++d)
                    if (d < D) acc[d] = fmaf(gv[u], w[d], acc[d]);
            }
        }
#pragma unroll
        for (int d = 0; d < 8; ++d)
            if (d < D) grad_geometry[row * D + d] = acc[d];
    }
}

// One thread per hidden channel h over a slice of edge rows (blockIdx.x): the
// input projection's weight gradient sum_r grad_pre[r][h] geometry[r][d] and
// bias gradient sum_r grad_pre[r][h], as one partial row per slice (H x D,
// then H).
__global__ void __launch_bounds__(256)
input_weight_grad_kernel(const float* __restrict__ grad_pre, const float* __restrict__ geometry,
                         int64_t rows, int64_t rows_per_slice, int H, int D,
                         float* __restrict__ part) {
    const int h = threadIdx.x;
    const int64_t r_lo = (int64_t)blockIdx.x * rows_per_slice;
    const int64_t r_hi = r_lo + rows_per_slice < rows ? r_lo + rows_per_slice : rows;
    float aw[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    float ab = 0.0f;
    if (h < H) {
#pragma unroll 4
        for (int64_t r = r_lo; r < r_hi; ++r) {
            const float g = grad_pre[r * H + h];
            ab += g;
#pragma unroll
            for (int d = 0; d < 8; ++d)
                if (d < D) aw[d] = fmaf(g, geometry[r * D + d], aw[d]);
        }
        float* out = part + (size_t)blockIdx.x * H * (D + 1);
#pragma unroll
        for (int d = 0; d < 8; ++d)
            if (d < D) out[h * D + d] = aw[d];
        out[H * D + h] = ab;
    }
}

// ---------------------------------------------------------------------------
// Offset-attention backward (offset_attention_backward.cu,
// offset_attention.cuh:130-208), per chunk of batch items with the N x N
// probabilities held in the workspace
// ---------------------------------------------------------------------------

// Strided batched product: C[b][m][n] = sum_k A(b, m, k) B(b, k, n), with
// A(b, m, k) = A[b sAb + m sAm + k sAk] and B(b, k, n) = B[b sBb + k sBk +
// n sBn]; C row-major (ldc) per item at b sCb. 64 x 64 tiles, 16-deep k
// steps, 4 x 4 outputs per thread.
struct Bmm {
    const float* A;
    int64_t sAb, sAm, sAk;
    const float* B;
    int64_t sBb, sBk, sBn;
    float* C;
    int64_t sCb, ldc;
    int M, N, K;
};

__global__ void __launch_bounds__(256) bmm_kernel(const Bmm p) {
    __shared__ __align__(16) float As[2][16][64 + 4], Bs[2][16][64 + 4];
    const int b = blockIdx.z;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const float* A = p.A + b * p.sAb;
    const float* Bp = p.B + b * p.sBb;
    float acc[4][4] = {};
    // staging slots of this thread: k rows e >> 6, m / n columns e & 63; the
    // next 16-deep step is loaded into registers while the current one is
    // multiplied (two shared-memory buffers)
    float ar[4], br[4];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = threadIdx.x + 256 * u, kk = e >> 6, mm = e & 63;
            const int k = k0 + kk, m = m0 + mm, n = n0 + mm;
            ar[u] = (m < p.M && k < p.K) ? A[m * p.sAm + k * p.sAk] : 0.0f;
            br[u] = (n < p.N && k < p.K) ? Bp[k * p.sBk + n * p.sBn] : 0.0f;
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = threadIdx.x + 256 * u, kk = e >> 6, mm = e & 63;
            As[buf][kk][mm] = ar[u];
            Bs[buf][kk][mm] = br[u];
        }
    };
    fetch(0);
    stash(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < p.K; k0 += 16) {
        const bool more = k0 + 16 < p.K;
        if (more) fetch(k0 + 16);
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            const float4 a4 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            const float4 b4 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
            const float a[4] = {a4.x, a4.y, a4.z, a4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int v = 0; v < 4; ++v) acc[u][v] += a[u] * bv[v];
        }
        if (more) {
            stash(buf ^ 1);  // the other buffer: its last readers passed the barrier below
            __syncthreads();
            buf ^= 1;
        }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int m = m0 + ty * 4 + u;
        if (m >= p.M) continue;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            const int n = n0 + tx * 4 + v;
            if (n < p.N) p.C[b * p.sCb + m * p.ldc + n] = acc[u][v];
        }
    }
}

int bmm(const Bmm& p, int batch, cudaStream_t st) {
    const dim3 grid((p.N + 63) / 64, (p.M + 63) / 64, batch);
    F2S_LIMIT(grid.y <= 65535 && grid.z <= 65535, "attention backward: product too large");
    bmm_kernel<<<grid, 256, 0, st>>>(p);
    return check_launch("bmm_kernel");
}

// Softmax over the queries (rows) of each key column of S, in place: a block
// of 32 columns x 8 row groups per (column tile, item).
__global__ void __launch_bounds__(256) column_softmax_kernel(float* __restrict__ P, int N) {
    __shared__ float red[8][32];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int j = blockIdx.x * 32 + tx;
    float* col = P + (size_t)blockIdx.y * N * N;
    float m = -FLT_MAX;
    if (j < N)
        for (int i = ty; i < N; i += 8) m = fmaxf(m, col[(size_t)i * N + j]);
    red[ty][tx] = m;
    __syncthreads();
    m = red[0][tx];
    for (int g = 1; g < 8; ++g) m = fmaxf(m, red[g][tx]);
    __syncthreads();
    float s = 0.0f;
    if (j < N)
        for (int i = ty; i < N; i += 8) {
            const float e = expf(col[(size_t)i * N + j] - m);
            col[(size_t)i * N + j] = e;
            s += e;
        }
    red[ty][tx] = s;
    __syncthreads();
    s = 0.0f;
    for (int g = 0; g < 8; ++g) s += red[g][tx];
    const float inv = 1.0f / s;
    if (j < N)
        for (int i = ty; i < N; i += 8) col[(size_t)i * N + j] *= inv;
}

// A warp per query row: z = sum over keys of P, G^ = G / (z + 1e-9), r = <G^, O>.
__global__ void __launch_bounds__(256)
attention_rows_kernel(const float* __restrict__ P, const float* __restrict__ G,
                      const float* __restrict__ O, int N, int C, int rows,
                      float* __restrict__ Gh, float* __restrict__ r) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int b = row / N, i = row - b * N;
    const float* p = P + ((size_t)b * N + i) * N;
    float z = 0.0f;
    for (int j = lane; j < N; j += 32) z += p[j];
    z = warp_sum(z);
    const float inv = 1.0f / (z + 1e-9f);
    float acc = 0.0f;
    for (int c = lane; c < C; c += 32) {
        const float gh = G[(size_t)row * C + c] * inv;
        Gh[(size_t)row * C + c] = gh;
        acc += gh * O[(size_t)row * C + c];
    }
    acc = warp_sum(acc);
    if (lane == 0) r[row] = acc;
}

// Per key column j: c_j = sum_i P[i][j] (D[i][j] - r_i), then in place
// D[i][j] = dS = P[i][j] (D[i][j] - r_i - c_j).
__global__ void __launch_bounds__(256)
column_jacobian_kernel(const float* __restrict__ P, float* __restrict__ D,
                       const float* __restrict__ r, int N) {
    __shared__ float red[8][32];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int j = blockIdx.x * 32 + tx;
    const size_t base = (size_t)blockIdx.y * N * N;
    const float* rr = r + (size_t)blockIdx.y * N;
    float s = 0.0f;
    if (j < N)
        for (int i = ty; i < N; i += 8) s += P[base + (size_t)i * N + j] * (D[base + (size_t)i * N + j] - rr[i]);
    red[ty][tx] = s;
    __syncthreads();
    s = 0.0f;
    for (int g = 0; g < 8; ++g) s += red[g][tx];
    if (j < N)
        for (int i = ty; i < N; i += 8) {
            const size_t e = base + (size_t)i * N + j;
            D[e] = P[e] * (D[e] - rr[i] - s);
        }
}

constexpr int kAttnChunk = 8;  // batch items per pass (2 N^2 floats each)

struct AttnSpace {
    size_t P, D, Gh, r, GhT, VT, KT, bytes;
};

AttnSpace attn_space(int B, int N, int d, int C) {
    const size_t chunk = (size_t)(B < kAttnChunk ? B : kAttnChunk);
    AttnSpace s;
    s.P = 0;
    s.D = align256(s.P + chunk * N * N * 4);
    s.Gh = align256(s.D + chunk * N * N * 4);
    s.r = align256(s.Gh + chunk * N * C * 4);
    s.GhT = align256(s.r + chunk * N * 4);      // G^ transposed, (C, N) per item
    s.VT = align256(s.GhT + chunk * N * C * 4);  // V transposed, (C, N) per item
    s.KT = align256(s.VT + chunk * N * C * 4);   // K transposed, (N, d) per item
    s.bytes = align256(s.KT + chunk * N * d * 4);
    return s;
}

// ---------------------------------------------------------------------------
// The full neighbour-reduction backward: workspace layout
// ---------------------------------------------------------------------------
struct NrSpace {
    size_t pre, hidden, contrib, gcontrib, ghidden, wout_t, win_t, wsplit, wtsplit, content_pm,
        grad_pm, part, bytes;
};

NrSpace nr_space(int B, int N, int K, int D, int H, int C) {
    const size_t R = (size_t)B * N * K;
    NrSpace s;
    s.pre = 0;
    s.hidden = align256(s.pre + R * H * 4);
    s.contrib = align256(s.hidden + R * H * 4);
    s.gcontrib = align256(s.contrib + R * C * 4);
    s.ghidden = align256(s.gcontrib + R * C * 4);
    s.wout_t = align256(s.ghidden + R * H * 4);
    s.win_t = align256(s.wout_t + (size_t)C * H * 4);
    s.wsplit = align256(s.win_t + (size_t)H * D * 4);      // W_out as bf16 high, low
    s.wtsplit = align256(s.wsplit + (size_t)C * H * 4);    // W_out^T as bf16 high, low
    s.content_pm = align256(s.wtsplit + (size_t)C * H * 4);
    s.grad_pm = align256(s.content_pm + (size_t)B * N * 2 * C * 4);
    s.part = align256(s.grad_pm + (size_t)B * N * 2 * C * 4);
    // partial rows: the per-block kernels (<= 8 per SM) and the row slices
    const size_t blocks = (size_t)sm_count() * 8;
    size_t part = 2 * blocks * (size_t)(H > C ? H : C);
    const size_t geo = (size_t)kWgradSlices * H * (D + 1);
    part = part > geo ? part : geo;
    const size_t ch = (size_t)C * H + C, hd = (size_t)H * D + H;
    const size_t slices = (size_t)kSlices * (ch > hd ? ch : hd);
    part = part > slices ? part : slices;
    s.bytes = align256(s.part + part * 4);
    return s;
}

}  // namespace
}  // namespace f2s

using namespace f2s;

extern "C" int f2s_nearest_backward(const float* first, const float* second, int B, int M, int N,
                                    const int32_t* second_index, const int32_t* first_index,
                                    const float* grad_first_distance,
                                    const float* grad_second_distance, float* grad_first,
                                    float* grad_second, void* stream) {
    F2S_REQUIRE(B >= 0 && M >= 1 && N >= 1, "nearest_backward: bad sizes B=%d M=%d N=%d", B, M, N);
    if (B == 0) return F2S_OK;
    F2S_REQUIRE(first && second && second_index && first_index && grad_first && grad_second,
                "nearest_backward: null pointer");
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagTraining, st);
    return nearest_backward(first, second, B, M, N, second_index, first_index,
                            grad_first_distance, grad_second_distance, grad_first, grad_second, st);
}

extern "C" int f2s_dcd_loss_workspace_bytes(int B, int M, int N, size_t* bytes) {
    F2S_REQUIRE(B >= 0 && M >= 0 && N >= 0 && bytes, "bad workspace query");
    *bytes = dcd_space(B, M, N).bytes;
    return F2S_OK;
}

extern "C" int f2s_dcd_loss(const float* pred, const float* target, int B, int M, int N,
                            float alpha, float* loss, const float* grad_loss, float* grad_pred,
                            float* grad_target, void* workspace, size_t workspace_bytes,
                            void* stream) {
    F2S_REQUIRE(B >= 0 && M >= 1 && N >= 1, "dcd_loss: bad sizes B=%d M=%d N=%d", B, M, N);
    if (B == 0) return F2S_OK;
    F2S_REQUIRE(pred && target && loss && workspace, "dcd_loss: null pointer");
    F2S_REQUIRE((grad_pred == nullptr) == (grad_target == nullptr),
                "dcd_loss: give both gradient outputs or neither");
    const DcdSpace s = dcd_space(B, M, N);
    if (workspace_bytes < s.bytes)
        return fail(F2S_ERR_WORKSPACE, "dcd_loss needs %zu workspace bytes, got %zu", s.bytes,
                    workspace_bytes);
    char* ws = static_cast<char*>(workspace);
    float* d1 = reinterpret_cast<float*>(ws + s.d1);
    int32_t* i2 = reinterpret_cast<int32_t*>(ws + s.i2);
    float* d2 = reinterpret_cast<float*>(ws + s.d2);
    int32_t* i1 = reinterpret_cast<int32_t*>(ws + s.i1);
    int* tm = reinterpret_cast<int*>(ws + s.tm);
    int* pm = reinterpret_cast<int*>(ws + s.pm);
    float* gd1 = grad_pred ? reinterpret_cast<float*>(ws + s.gd1) : nullptr;
    float* gd2 = grad_pred ? reinterpret_cast<float*>(ws + s.gd2) : nullptr;
    cudaStream_t st = as_stream(stream);
    F2S_TRY(f2s_nearest(pred, target, B, M, N, d1, i2, d2, i1, ws + s.nearest,
                        workspace_bytes - s.nearest, stream));
    TraceScope trace(kTagTraining, st);
    F2S_CUDA_TRY(cudaMemsetAsync(tm, 0, s.gd1 - s.tm, st));  // both multiplicity arrays
    const int64_t total = (int64_t)B * ((int64_t)M + N);
    dcd_count_kernel<<<blocks_for(total), kBlock, 0, st>>>(i2, i1, B, M, N, tm, pm);
    F2S_TRY(check_launch("dcd_count_kernel"));
    dcd_terms_kernel<<<B, 1024, 0, st>>>(d1, i2, d2, i1, M, N, tm, pm, alpha, grad_loss, loss,
                                         gd1, gd2);
    F2S_TRY(check_launch("dcd_terms_kernel"));
    if (!grad_pred) return F2S_OK;
    return nearest_backward(pred, target, B, M, N, i2, i1, gd1, gd2, grad_pred, grad_target, st);
}

extern "C" int f2s_velocity_loss(const float* pred, const float* target, int B, int M,
                                 float* loss, const float* grad_loss, float* grad_pred,
                                 float* grad_target, void* stream) {
    F2S_REQUIRE(B >= 0 && M >= 1, "velocity_loss: bad sizes B=%d M=%d", B, M);
    if (B == 0) return F2S_OK;
    F2S_REQUIRE(pred && target, "velocity_loss: null pointer");
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagTraining, st);
    velocity_loss_kernel<<<B, 1024, 0, st>>>(pred, target, M, grad_loss, loss, grad_pred,
                                             grad_target);
    return check_launch("velocity_loss_kernel");
}

extern "C" int f2s_hpe_activation_backward_workspace_bytes(int64_t rows, int H, size_t* bytes) {
    F2S_REQUIRE(rows >= 0 && H >= 1 && bytes, "bad workspace query");
    *bytes = (size_t)2 * hpe_grad_blocks(rows) * H * sizeof(float);
    return F2S_OK;
}

extern "C" int f2s_hpe_activation_backward(const float* preactivation, int64_t rows, int H,
                                           const float* norm_weight, const float* norm_bias,
                                           const float* grad_hidden, float* grad_preactivation,
                                           float* grad_norm_weight, float* grad_norm_bias,
                                           void* workspace, size_t workspace_bytes,
                                           void* stream) {
    F2S_REQUIRE(rows >= 0 && H >= 1, "hpe_activation_backward: bad sizes");
    F2S_LIMIT(H <= 256, "hpe_activation_backward: %d hidden channels (at most 256)", H);
    F2S_REQUIRE(preactivation && norm_weight && norm_bias && grad_hidden && grad_preactivation &&
                    grad_norm_weight && grad_norm_bias && workspace,
                "hpe_activation_backward: null pointer");
    size_t need = 0;
    F2S_TRY(f2s_hpe_activation_backward_workspace_bytes(rows, H, &need));
    if (workspace_bytes < need)
        return fail(F2S_ERR_WORKSPACE, "hpe_activation_backward needs %zu workspace bytes, got %zu",
                    need, workspace_bytes);
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagTraining, st);
    return hpe_activation_backward(preactivation, rows, H, norm_weight, norm_bias, grad_hidden,
                                   grad_preactivation, grad_norm_weight, grad_norm_bias,
                                   static_cast<float*>(workspace), st);
}

extern "C" int f2s_neighbor_messages_backward_workspace_bytes(int B, int N, int C,
                                                              size_t* bytes) {
    F2S_REQUIRE(B >= 0 && N >= 0 && C >= 1 && bytes, "bad workspace query");
    const size_t part = align256((size_t)2 * messages_grad_blocks((int64_t)B * N) * C * 4);
    const size_t pm = align256((size_t)B * N * 2 * C * 4);
    *bytes = part + 2 * pm;
    return F2S_OK;
}

extern "C" int f2s_neighbor_messages_backward(const float* content, const float* contribution,
                                              const int32_t* indices, int B, int N, int K, int C,
                                              const float* norm_weight, const float* norm_bias,
                                              const float* grad_output, float* grad_content,
                                              float* grad_contribution, float* grad_norm_weight,
                                              float* grad_norm_bias, void* workspace,
                                              size_t workspace_bytes, void* stream) {
    F2S_REQUIRE(B >= 0 && N >= 1 && K >= 1 && C >= 1, "neighbor_messages_backward: bad sizes");
    F2S_LIMIT(C <= 256, "neighbor_messages_backward: %d channels (at most 256)", C);
    if (B == 0) return F2S_OK;
    F2S_REQUIRE(content && contribution && indices && norm_weight && norm_bias && grad_output &&
                    grad_content && grad_contribution && grad_norm_weight && grad_norm_bias &&
                    workspace,
                "neighbor_messages_backward: null pointer");
    size_t need = 0;
    F2S_TRY(f2s_neighbor_messages_backward_workspace_bytes(B, N, C, &need));
    if (workspace_bytes < need)
        return fail(F2S_ERR_WORKSPACE,
                    "neighbor_messages_backward needs %zu workspace bytes, got %zu", need,
                    workspace_bytes);
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagTraining, st);
    char* ws = static_cast<char*>(workspace);
    const size_t part = align256((size_t)2 * messages_grad_blocks((int64_t)B * N) * C * 4);
    const size_t pm = align256((size_t)B * N * 2 * C * 4);
    return messages_backward(content, contribution, indices, B, N, K, C, norm_weight, norm_bias,
                             grad_output, grad_content, grad_contribution, grad_norm_weight,
                             grad_norm_bias, reinterpret_cast<float*>(ws),
                             reinterpret_cast<float*>(ws + part),
                             reinterpret_cast<float*>(ws + part + pm), st);
}

extern "C" int f2s_neighbor_reduce_backward_workspace_bytes(int B, int N, int K, int D, int H,
                                                            int C, size_t* bytes) {
    F2S_REQUIRE(B >= 0 && N >= 0 && K >= 0 && D >= 1 && H >= 1 && C >= 1 && bytes,
                "bad workspace query");
    *bytes = nr_space(B, N, K, D, H, C).bytes;
    return F2S_OK;
}

extern "C" int f2s_neighbor_reduce_backward(
    const float* content, const float* geometry, const int32_t* indices,
    const float* hpe_input_weight, const float* hpe_input_bias, const float* hpe_output_weight,
    const float* hpe_output_bias, const float* hpe_norm_weight, const float* hpe_norm_bias,
    const float* message_norm_weight, const float* message_norm_bias, int B, int N, int K, int D,
    int H, int C, const float* grad_output, float* grad_content, float* grad_geometry,
    float* grad_hpe_input_weight, float* grad_hpe_input_bias, float* grad_hpe_output_weight,
    float* grad_hpe_output_bias, float* grad_hpe_norm_weight, float* grad_hpe_norm_bias,
    float* grad_message_norm_weight, float* grad_message_norm_bias, void* workspace,
    size_t workspace_bytes, void* stream) {
    F2S_REQUIRE(B >= 0 && N >= 1 && K >= 1 && D >= 1 && H >= 1 && C >= 1,
                "neighbor_reduce_backward: bad sizes");
    F2S_LIMIT(D <= 8 && H <= 256 && C <= 256,
              "neighbor_reduce_backward: D=%d H=%d C=%d (at most 8, 256, 256)", D, H, C);
    if (B == 0) return F2S_OK;
    const void* need_ptrs[] = {content, geometry, indices, hpe_input_weight, hpe_input_bias,
                               hpe_output_weight, hpe_output_bias, hpe_norm_weight,
                               hpe_norm_bias, message_norm_weight, message_norm_bias,
                               grad_output, grad_content, grad_geometry, grad_hpe_input_weight,
                               grad_hpe_input_bias, grad_hpe_output_weight,
                               grad_hpe_output_bias, grad_hpe_norm_weight, grad_hpe_norm_bias,
                               grad_message_norm_weight, grad_message_norm_bias, workspace};
    for (const void* q : need_ptrs) F2S_REQUIRE(q != nullptr, "neighbor_reduce_backward: null pointer");
    const NrSpace s = nr_space(B, N, K, D, H, C);
    if (workspace_bytes < s.bytes)
        return fail(F2S_ERR_WORKSPACE, "neighbor_reduce_backward needs %zu workspace bytes, got %zu",
                    s.bytes, workspace_bytes);
    char* ws = static_cast<char*>(workspace);
    float* pre = reinterpret_cast<float*>(ws + s.pre);
    float* hidden = reinterpret_cast<float*>(ws + s.hidden);
    float* contrib = reinterpret_cast<float*>(ws + s.contrib);
    float* gcontrib = reinterpret_cast<float*>(ws + s.gcontrib);
    float* ghidden = reinterpret_cast<float*>(ws + s.ghidden);
    float* wout_t = reinterpret_cast<float*>(ws + s.wout_t);
    float* part = reinterpret_cast<float*>(ws + s.part);
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagTraining, st);
    const int64_t R = (int64_t)B * N * K;
    const int rb = hpe_grad_blocks(R);
    // recompute the HPE rows and the contribution (neighbor_reduce.py:174-184)
#define F2S_HPE_FWD(CPL)                                                                         \
    hpe_forward_rows_kernel<CPL><<<rb, kBlock, 0, st>>>(geometry, R, D, H, hpe_input_weight,    \
                                                        hpe_input_bias, hpe_norm_weight,         \
                                                        hpe_norm_bias, pre, hidden)
    const int hcpl = (H + 31) / 32;
    if (hcpl <= 1) F2S_HPE_FWD(1);
    else if (hcpl <= 2) F2S_HPE_FWD(2);
    else if (hcpl <= 4) F2S_HPE_FWD(4);
    else F2S_HPE_FWD(8);
#undef F2S_HPE_FWD
    F2S_TRY(check_launch("hpe_forward_rows_kernel"));
    // the two projection products on the tensor cores as split bf16 (the
    // fp32 rows split in the GEMM, W_out and its transpose split here;
    // about 1e-5 relative to sum |x| |w|), which need 16-byte bf16 rows;
    // other widths on the fp32 CUDA-core GEMM
    F2S_LIMIT(R <= INT32_MAX, "neighbor_reduce_backward: %lld edge rows", (long long)R);
    const bool tensor = H % 8 == 0 && C % 8 == 0;
    void* wsplit = ws + s.wsplit;
    void* wtsplit = ws + s.wtsplit;
    if (tensor) {
        F2S_TRY(split_bf16(hpe_output_weight, H, C, H, wsplit,
                           static_cast<char*>(wsplit) + (size_t)C * H * 2, st));
        F2S_TRY(f2s_linear(hidden, H, wsplit, hpe_output_bias, contrib, C, (int)R, C, H,
                           F2S_PRECISION_BF16X3, stream));
    } else {
        F2S_TRY(f2s_linear(hidden, H, hpe_output_weight, hpe_output_bias, contrib, C, (int)R, C,
                           H, F2S_PRECISION_FP32, stream));
    }
    // the message reduction's backward (neighbor_reduce.py:186-202)
    F2S_TRY(messages_backward(content, contrib, indices, B, N, K, C, message_norm_weight,
                              message_norm_bias, grad_output, grad_content, gcontrib,
                              grad_message_norm_weight, grad_message_norm_bias, part,
                              reinterpret_cast<float*>(ws + s.content_pm),
                              reinterpret_cast<float*>(ws + s.grad_pm), st));
    // grad_hidden = grad_contribution W_out; the output projection's gradients
    transpose_small_kernel<<<blocks_for((int64_t)C * H), kBlock, 0, st>>>(hpe_output_weight, C, H,
                                                                          wout_t);
    F2S_TRY(check_launch("transpose_small_kernel"));
    if (tensor) {
        F2S_TRY(split_bf16(wout_t, C, H, C, wtsplit,
                           static_cast<char*>(wtsplit) + (size_t)C * H * 2, st));
        F2S_TRY(f2s_linear(gcontrib, C, wtsplit, nullptr, ghidden, H, (int)R, H, C,
                           F2S_PRECISION_BF16X3, stream));
    } else {
        F2S_TRY(f2s_linear(gcontrib, C, wout_t, nullptr, ghidden, H, (int)R, H, C,
                           F2S_PRECISION_FP32, stream));
    }
    F2S_TRY(xty(gcontrib, C, hidden, H, R, grad_hpe_output_weight, grad_hpe_output_bias, part, st));
    // the HPE activation's backward, in place over grad_hidden (its rows are
    // read before they are written, one warp per row)
    F2S_TRY(hpe_activation_backward(pre, R, H, hpe_norm_weight, hpe_norm_bias, ghidden, ghidden,
                                    grad_hpe_norm_weight, grad_hpe_norm_bias, part, st));
    // the input projection's gradients (neighbor_reduce.py:219-224)
    const size_t gsmem = (size_t)H * D * sizeof(float);
    geometry_grad_kernel<<<blocks_for(R), kBlock, gsmem, st>>>(ghidden, R, H, D, hpe_input_weight,
                                                                grad_geometry);
    F2S_TRY(check_launch("geometry_grad_kernel"));
    const int64_t per = (R + kWgradSlices - 1) / kWgradSlices;
    const int slices = (int)((R + per - 1) / per);
    input_weight_grad_kernel<<<slices, 256, 0, st>>>(ghidden, geometry, R, per, H, D, part);
    F2S_TRY(check_launch("input_weight_grad_kernel"));
    F2S_TRY(sum_partials_strided(part, slices, H * D, H * (D + 1), grad_hpe_input_weight, st));
    return sum_partials_strided(part + H * D, slices, H, H * (D + 1), grad_hpe_input_bias, st);
}

extern "C" int f2s_offset_attention_backward_workspace_bytes(int B, int N, int d, int C,
                                                             size_t* bytes) {
    F2S_REQUIRE(B >= 0 && N >= 0 && d >= 1 && C >= 1 && bytes, "bad workspace query");
    *bytes = attn_space(B, N, d, C).bytes;
    return F2S_OK;
}

extern "C" int f2s_offset_attention_backward(const float* query, const float* key,
                                             const float* value, int B, int N, int d, int C,
                                             const float* output, const float* grad_output,
                                             float* grad_query, float* grad_key,
                                             float* grad_value, void* workspace,
                                             size_t workspace_bytes, void* stream) {
    F2S_REQUIRE(B >= 0 && N >= 1 && d >= 1 && C >= 1, "offset_attention_backward: bad sizes");
    if (B == 0) return F2S_OK;
    F2S_REQUIRE(query && key && value && output && grad_output && grad_query && grad_key &&
                    grad_value && workspace,
                "offset_attention_backward: null pointer");
    const AttnSpace s = attn_space(B, N, d, C);
    if (workspace_bytes < s.bytes)
        return fail(F2S_ERR_WORKSPACE,
                    "offset_attention_backward needs %zu workspace bytes, got %zu", s.bytes,
                    workspace_bytes);
    char* ws = static_cast<char*>(workspace);
    float* P = reinterpret_cast<float*>(ws + s.P);
    float* D = reinterpret_cast<float*>(ws + s.D);
    float* Gh = reinterpret_cast<float*>(ws + s.Gh);
    float* r = reinterpret_cast<float*>(ws + s.r);
    float* GhT = reinterpret_cast<float*>(ws + s.GhT);
    float* VT = reinterpret_cast<float*>(ws + s.VT);
    float* KT = reinterpret_cast<float*>(ws + s.KT);
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagTraining, st);
    const int64_t NN = (int64_t)N * N;
    for (int b0 = 0; b0 < B; b0 += kAttnChunk) {
        const int nb = B - b0 < kAttnChunk ? B - b0 : kAttnChunk;
        const float* q = query + (size_t)b0 * N * d;
        const float* k = key + (size_t)b0 * d * N;
        const float* v = value + (size_t)b0 * N * C;
        // S = Q K, then the softmax over queries of each key column
        F2S_TRY(bmm(Bmm{q, (int64_t)N * d, d, 1, k, (int64_t)d * N, N, 1, P, NN, N, N, N, d}, nb,
                    st));
        column_softmax_kernel<<<dim3((N + 31) / 32, nb), 256, 0, st>>>(P, N);
        F2S_TRY(check_launch("column_softmax_kernel"));
        // z, G^ = G / (z + 1e-9), r = <G^, O>
        attention_rows_kernel<<<(nb * N + 7) / 8, 256, 0, st>>>(
            P, grad_output + (size_t)b0 * N * C, output + (size_t)b0 * N * C, N, C, nb * N, Gh, r);
        F2S_TRY(check_launch("attention_rows_kernel"));
        // dV = P^T G^
        F2S_TRY(bmm(Bmm{P, NN, 1, N, Gh, (int64_t)N * C, C, 1, grad_value + (size_t)b0 * N * C,
                        (int64_t)N * C, C, N, C, N},
                    nb, st));
        // D = G^ V^T on transposed copies of G^ and V, so both operands are
        // read along rows (i and j contiguous); then dS = P (D - r - c) per
        // key column
        F2S_TRY(transpose_batched(Gh, GhT, nb, N, C, st));
        F2S_TRY(transpose_batched(v, VT, nb, N, C, st));
        F2S_TRY(bmm(Bmm{GhT, (int64_t)C * N, 1, N, VT, (int64_t)C * N, N, 1, D, NN, N, N, N, C},
                    nb, st));
        column_jacobian_kernel<<<dim3((N + 31) / 32, nb), 256, 0, st>>>(P, D, r, N);
        F2S_TRY(check_launch("column_jacobian_kernel"));
        // dQ = dS K^T from dS transposed (into P, which is no longer needed)
        // and K transposed, so both operands are read along rows; dK = Q^T dS
        F2S_TRY(transpose_batched(D, P, nb, N, N, st));
        F2S_TRY(transpose_batched(k, KT, nb, d, N, st));
        F2S_TRY(bmm(Bmm{P, NN, 1, N, KT, (int64_t)N * d, d, 1, grad_query + (size_t)b0 * N * d,
                        (int64_t)N * d, d, N, d, N},
                    nb, st));
        F2S_TRY(bmm(Bmm{q, (int64_t)N * d, 1, d, D, NN, N, 1, grad_key + (size_t)b0 * d * N,
                        (int64_t)d * N, N, d, N, N},
                    nb, st));
    }
    return F2S_OK;
}
