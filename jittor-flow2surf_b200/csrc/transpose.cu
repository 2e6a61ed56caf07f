// Batched 2-D transpose (B, rows, cols) -> (B, cols, rows) through 32 x 33
// shared-memory tiles; converts the reference's channel-major (B, C, N)
// operator layouts to the point-major rows the kernels read, and back.
#include "kernels.cuh"

namespace f2s {
namespace {

__global__ void transpose_kernel(const float* __restrict__ in, float* __restrict__ out,
                                 int rows, int cols, int tiles_c) {
    __shared__ float tile[32][33];
    const int b = blockIdx.z;
    const int tr = blockIdx.y, tc = blockIdx.x;
    const float* src = in + (size_t)b * rows * cols;
    float* dst = out + (size_t)b * rows * cols;
    const int x = tc * 32 + threadIdx.x;
    for (int y = threadIdx.y; y < 32; y += 8) {
        const int r = tr * 32 + y;
        if (r < rows && x < cols) tile[y][threadIdx.x] = src[(size_t)r * cols + x];
    }
    __syncthreads();
    const int xr = tr * 32 + threadIdx.x;
    for (int y = threadIdx.y; y < 32; y += 8) {
        const int c = tc * 32 + y;
        if (c < cols && xr < rows) dst[(size_t)c * rows + xr] = tile[threadIdx.x][y];
    }
    (void)tiles_c;
}

}  // namespace

int transpose_batched(const float* in, float* out, int B, int rows, int cols,
                      cudaStream_t stream) {
    if (B == 0 || rows == 0 || cols == 0) return F2S_OK;
    F2S_LIMIT(B <= 65535, "transpose: batch %d too large", B);
    dim3 grid(ceil_div(cols, 32), ceil_div(rows, 32), B);
    F2S_LIMIT(grid.y <= 65535, "transpose: too many rows");
    TraceScope trace(kTagTranspose, stream);
    transpose_kernel<<<grid, dim3(32, 8), 0, stream>>>(in, out, rows, cols, grid.x);
    return check_launch("transpose_kernel");
}

}  // namespace f2s
