// Bidirectional nearest squared distances and the Chamfer distance.
//
// Reference semantics (flow2surf/training/cuda/nearest_distance_forward.cu:1-93):
// for each query point, scan the other set in index order keeping the smallest
// d = dx*dx + dy*dy + dz*dz (nvcc contracts it to fma(dz, dz, fma(dx, dx,
// dy*dy)), dx = query - reference), starting from (FLT_MAX, index = N) and
// replacing only on a strictly smaller distance (ties keep the lower index).
// Chamfer: mean d(p -> q) + mean d(q -> p) (flow2surf/evaluation.py:24-28).
//
// B200 design: each thread keeps 4 queries in registers, the reference set
// streams through shared memory as float4 tiles, and the reference set is split
// across CTAs when the query count alone cannot fill 148 SMs. Each split's
// (distance, index) winner is folded into a 64-bit key
// (order-preserving distance bits << 32 | index) with atomicMin, which is
// exactly the lexicographic rule above, so the split changes no result.
#include <cfloat>

#include "kernels.cuh"

namespace f2s {
namespace {

constexpr int kThreads = 256;
constexpr int kQpt = 4;
constexpr int kQueriesPerCta = kThreads * kQpt;
constexpr int kTile = 1024;

__device__ __forceinline__ unsigned long long dist_key(float d, int j) {
    return ((unsigned long long)f2s_ordered_bits(d) << 32) | (unsigned)j;
}

// A uniform grid over one batch item of a point set (the grid search below).
struct GridInfo {
    float ox, oy, oz;  // the minimum corner of the finite points
    float inv_h, h;    // cell edge and its reciprocal
    float margin;      // rounding allowance of a computed cell index, in cells
    int gx, gy, gz;
    int dense;  // some cell holds more than 1/32 of the points: plain scan instead
};

__global__ void init_keys_kernel(unsigned long long* keys, int64_t count, int reference_count) {
    const unsigned long long k0 = dist_key(FLT_MAX, reference_count);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x)
        keys[i] = k0;
}

__global__ void __launch_bounds__(kThreads)
nearest_kernel(const float* __restrict__ query, const float* __restrict__ ref, int M, int N,
               int ref_chunk, unsigned long long* __restrict__ keys,
               const GridInfo* __restrict__ only_dense) {
    __shared__ float4 tile[kTile];
    const int b = blockIdx.z;
    // beside the grid search: only the items whose grid is too dense
    if (only_dense != nullptr && !only_dense[b].dense) return;
    const int q0 = blockIdx.x * kQueriesPerCta;
    const int j_lo = blockIdx.y * ref_chunk;
    const int j_hi = min(N, j_lo + ref_chunk);
    const float* qb = query + (size_t)b * M * 3;
    const float* rb = ref + (size_t)b * N * 3;
    float qx[kQpt], qy[kQpt], qz[kQpt], best[kQpt];
    int bj[kQpt];
#pragma unroll
    for (int t = 0; t < kQpt; ++t) {
        const int i = q0 + threadIdx.x + kThreads * t;
        const bool in = i < M;
        qx[t] = in ? qb[3 * i] : 0.0f;
        qy[t] = in ? qb[3 * i + 1] : 0.0f;
        qz[t] = in ? qb[3 * i + 2] : 0.0f;
        best[t] = INFINITY;
        bj[t] = -1;
    }
    for (int t0 = j_lo; t0 < j_hi; t0 += kTile) {
        const int count = min(kTile, j_hi - t0);
        __syncthreads();
        for (int j = threadIdx.x; j < count; j += kThreads) {
            const float* p = rb + 3 * (size_t)(t0 + j);
            tile[j] = make_float4(p[0], p[1], p[2], 0.0f);
        }
        __syncthreads();
        for (int j = 0; j < count; ++j) {
            const float4 r = tile[j];
#pragma unroll
            for (int t = 0; t < kQpt; ++t) {
                const float dx = __fsub_rn(qx[t], r.x);
                const float dy = __fsub_rn(qy[t], r.y);
                const float dz = __fsub_rn(qz[t], r.z);
                const float d = __fmaf_rn(dz, dz, __fmaf_rn(dx, dx, __fmul_rn(dy, dy)));
                if (d < best[t]) {
                    best[t] = d;
                    bj[t] = t0 + j;
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < kQpt; ++t) {
        const int i = q0 + threadIdx.x + kThreads * t;
        if (i < M && bj[t] >= 0) atomicMin(&keys[(size_t)b * M + i], dist_key(best[t], bj[t]));
    }
}

__global__ void unpack_kernel(const unsigned long long* __restrict__ keys, int64_t count,
                              float* __restrict__ dist, int32_t* __restrict__ index) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x) {
        const unsigned long long k = keys[i];
        dist[i] = __uint_as_float((unsigned)(k >> 32) ^ 0x80000000u);
        index[i] = (int32_t)(unsigned)(k & 0xffffffffu);
    }
}

// chamfer[b] = mean_i d1[b, i] + mean_j d2[b, j], float64, fixed reduction order.
__global__ void __launch_bounds__(1024)
chamfer_reduce_kernel(const unsigned long long* __restrict__ k1, int M,
                      const unsigned long long* __restrict__ k2, int N, double* __restrict__ out) {
    __shared__ double red[32];
    const int b = blockIdx.x;
    // four independent partial sums per thread (loads in flight together),
    // combined in a fixed order
    double s1[4] = {0.0, 0.0, 0.0, 0.0}, s2[4] = {0.0, 0.0, 0.0, 0.0};
    for (int i = threadIdx.x; i < M; i += 4096)
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (i + 1024 * u < M)
                s1[u] += (double)__uint_as_float(
                    (unsigned)(k1[(size_t)b * M + i + 1024 * u] >> 32) ^ 0x80000000u);
    for (int j = threadIdx.x; j < N; j += 4096)
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (j + 1024 * u < N)
                s2[u] += (double)__uint_as_float(
                    (unsigned)(k2[(size_t)b * N + j + 1024 * u] >> 32) ^ 0x80000000u);
    double v = ((s1[0] + s1[1]) + (s1[2] + s1[3])) / (double)M +
               ((s2[0] + s2[1]) + (s2[2] + s2[3])) / (double)N;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        v = red[threadIdx.x];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) out[b] = v;
    }
}

int grid_1d(int64_t work) {
    const int64_t blocks = (work + 255) / 256;
    const int64_t cap = (int64_t)sm_count() * 16;
    return (int)(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

// keys[b, i] = min over j of dist_key(d(query_i, ref_j), j), starting at (FLT_MAX, N).
// With only_dense, only the items whose grid there is flagged dense; with
// init false, the keys have been started already.
int one_way(const float* query, const float* ref, int B, int M, int N, unsigned long long* keys,
            cudaStream_t st, const GridInfo* only_dense = nullptr, bool init = true) {
    if (init) {
        const int64_t count = (int64_t)B * M;
        init_keys_kernel<<<grid_1d(count), 256, 0, st>>>(keys, count, N);
        F2S_TRY(check_launch("init_keys_kernel"));
    }
    const int qblocks = ceil_div(M, kQueriesPerCta);
    const int64_t base = (int64_t)qblocks * B;
    int splits = (int)((4ll * sm_count() + base - 1) / base);
    const int max_splits = ceil_div(N, kTile);
    splits = splits < 1 ? 1 : (splits > max_splits ? max_splits : splits);
    const int ref_chunk = ceil_div(ceil_div(N, splits), kTile) * kTile;
    dim3 grid(qblocks, ceil_div(N, ref_chunk), B);
    F2S_LIMIT(grid.y <= 65535 && grid.z <= 65535, "nearest: grid too large");
    nearest_kernel<<<grid, kThreads, 0, st>>>(query, ref, M, N, ref_chunk, keys, only_dense);
    return check_launch("nearest_kernel");
}

// ---------------------------------------------------------------------------
// Exact nearest search on a uniform grid, for large sets (the 100k-point
// Chamfer of the evaluation): the same (distance, index) winner as the
// brute-force scan above, from a few hundred candidates per query instead of
// all of them.
//
// Each set is counting-sorted into the cells of a grid over the bounding box
// of its finite points (about two cells per point, at most 4096 per axis):
// the points of a row of cells (fixed y and z) are then one contiguous range.
// A query visits the cells around its own cell in Chebyshev rings r = 0, 1,
// ... and stops after ring r once its best distance is below a lower bound on
// the squared distance of every point outside the visited box: a point in a
// cell at index distance r + 1 along an axis is at least (r + f - 2 m) cells
// away along it, f being the query's distance to its own cell's face in that
// direction (in cells) and m the rounding allowance of a computed cell
// index, and no nearer along the other two axes than the grid's slabs are;
// its computed distance is within 4e-7 (relative) of the exact one, so a
// best below lb^2 (1 - 4e-6) cannot be beaten or tied by any point not
// visited. Points with a non-finite coordinate take part in no bounding
// box; their distances are never below a finite best, as in the scan.
// Results do not depend on the order of points within a cell: the winner is
// the lexicographic minimum of (distance, index).
// ---------------------------------------------------------------------------


constexpr int kGridMinPoints = 4096;   // both sets at least this large
constexpr int kGridMaxAxis = 4096;     // cells along one axis
constexpr int kScanTile = 4096;        // cells per 1024-thread scan block, four per thread

int64_t grid_cell_cap(int n) {
    const int64_t c = 2 * (int64_t)n;
    return c < 64 ? 64 : (c > (1 << 22) ? (1 << 22) : c);
}

bool use_grid(int M, int N) { return M >= kGridMinPoints && N >= kGridMinPoints; }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int grid_tiles(int n) { return (int)((grid_cell_cap(n) + kScanTile - 1) / kScanTile); }  // <= 1024

// a query left to the far search: batch item, sorted position, best key so far
struct HardQuery {
    int b, i;
    unsigned long long key;
};

// One point set's grid and its part of the workspace. The grid kernels take
// both sets at once (GridPair), blockIdx.z choosing the set; in the search,
// set d is the query set and set 1 - d the reference set.
struct GridSet {
    const float* pts;  // (B, n, 3)
    int n;             // points per batch item
    int other_n;       // the other set's, the index of the starting key
    int64_t cap1;      // cells per item + 1
    int tiles;         // scan tiles per item
    GridInfo* info;    // [B]
    uint32_t* box;     // [B][6] order-preserving keys of the finite points' box
    uint32_t* tile_sum;  // [B][tiles]: tile sums, then tile offsets
    uint32_t* tile_max;  // [B][tiles]
    int* cellid;       // [B][n], -1 for a non-finite point
    int* counts;       // [B][cap1]
    int* starts;       // [B][cap1]
    float4* sorted;    // [B][n] (x, y, z, index bits) in cell order
    unsigned long long* keys;  // [B][n], this set as the query set
    HardQuery* hard;   // [B][n] its queries left to the far search
};

struct GridPair {
    GridSet s[2];
    int B;
    unsigned* counters;  // [0], [1]: hard queries of each set; [2]: the next one taken
};

// Byte offsets of one set's arrays from base.
struct GridSpace {
    size_t info, box, tile_sum, tile_max, cellid, counts, starts, sorted, hard, bytes;
};

GridSpace grid_space(int B, int n, size_t base) {
    GridSpace g;
    const size_t cap1 = (size_t)grid_cell_cap(n) + 1;
    const size_t tiles = (size_t)B * grid_tiles(n);
    g.info = align256(base);
    g.box = align256(g.info + (size_t)B * sizeof(GridInfo));
    g.tile_sum = align256(g.box + (size_t)B * 6 * sizeof(uint32_t));
    g.tile_max = align256(g.tile_sum + tiles * sizeof(uint32_t));
    g.cellid = align256(g.tile_max + tiles * sizeof(uint32_t));
    g.counts = align256(g.cellid + (size_t)B * n * sizeof(int));
    g.starts = align256(g.counts + (size_t)B * cap1 * sizeof(int));
    g.sorted = align256(g.starts + (size_t)B * cap1 * sizeof(int));
    g.hard = align256(g.sorted + (size_t)B * n * sizeof(float4));
    g.bytes = align256(g.hard + (size_t)B * n * sizeof(HardQuery));
    return g;
}

__device__ __forceinline__ bool finite3(float x, float y, float z) {
    return isfinite(x) && isfinite(y) && isfinite(z);
}

// Zeroes the counts and the hard-query counters, and starts the boxes at all
// ones (grid: blocks x 2 sets).
__global__ void grid_prepare_kernel(const GridPair P) {
    const GridSet& S = P.s[blockIdx.y];
    const int64_t cells = (int64_t)P.B * S.cap1;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < cells;
         i += (int64_t)gridDim.x * blockDim.x)
        S.counts[i] = 0;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    for (int e = t; e < 6 * P.B; e += gridDim.x * blockDim.x) S.box[e] = 0xffffffffu;
    if (blockIdx.y == 0 && t < 3) P.counters[t] = 0u;
}

// Bounding box of the finite points of each batch item: blocks over the
// points (grid: blocks x B x 2 sets), each folding its minima and maxima
// into the item's six keys with atomicMin (minima as order-preserving keys,
// maxima as their complements).
__global__ void __launch_bounds__(256) grid_box_kernel(const GridPair P) {
    __shared__ float red[8][6];
    const GridSet& S = P.s[blockIdx.z];
    const int b = blockIdx.y;
    const float* p = S.pts + (size_t)b * S.n * 3;
    float v[6] = {INFINITY, INFINITY, INFINITY, -INFINITY, -INFINITY, -INFINITY};
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < S.n; i += gridDim.x * blockDim.x) {
        const float x = p[3 * i], y = p[3 * i + 1], z = p[3 * i + 2];
        if (!finite3(x, y, z)) continue;
        v[0] = fminf(v[0], x);
        v[1] = fminf(v[1], y);
        v[2] = fminf(v[2], z);
        v[3] = fmaxf(v[3], x);
        v[4] = fmaxf(v[4], y);
        v[5] = fmaxf(v[5], z);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            v[a] = fminf(v[a], __shfl_xor_sync(0xffffffffu, v[a], o));
            v[a + 3] = fmaxf(v[a + 3], __shfl_xor_sync(0xffffffffu, v[a + 3], o));
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0)
        for (int a = 0; a < 6; ++a) red[warp][a] = v[a];
    __syncthreads();
    if (threadIdx.x >= 6) return;
    const int a = threadIdx.x;
    float m = red[0][a];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        m = a < 3 ? fminf(m, red[w][a]) : fmaxf(m, red[w][a]);
    if (isfinite(m)) {
        const uint32_t k = f2s_ordered_bits(m);
        atomicMin(&S.box[b * 6 + a], a < 3 ? k : ~k);
    }
}

__device__ __forceinline__ float unordered(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k ^ 0x80000000u) : ~k);
}

// Cells along the three axes at edge h (at least one each).
__device__ __forceinline__ int64_t grid_cells_at(const float* ext, float h, int* g) {
    const float inv = 1.0f / h;
    int64_t prod = 1;
    for (int a = 0; a < 3; ++a) {
        const float c = fminf(fmaxf(ceilf(ext[a] * inv), 1.0f), (float)kGridMaxAxis);
        g[a] = (int)c;
        prod *= g[a];
    }
    return prod;
}

// One thread per batch item and set: the grid over the item's box (the
// smallest cell edge whose cell count stays within the cap).
__global__ void grid_param_kernel(const GridPair P) {
    const GridSet& S = P.s[blockIdx.y];
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= P.B) return;
    const int64_t cap = S.cap1 - 1;
    GridInfo g{};
    g.ox = g.oy = g.oz = 0.0f;
    g.h = g.inv_h = 1.0f;
    g.margin = 0.0f;
    g.gx = g.gy = g.gz = 1;
    g.dense = 0;
    const uint32_t* k = S.box + b * 6;
    // all ones: no finite point
    if (k[0] != 0xffffffffu) {
        float v[6];
        for (int a = 0; a < 3; ++a) {
            v[a] = unordered(k[a]);
            v[a + 3] = unordered(~k[a + 3]);
        }
        const float ext[3] = {v[3] - v[0], v[4] - v[1], v[5] - v[2]};
        const float emax = fmaxf(ext[0], fmaxf(ext[1], ext[2]));
        // one cell when all points coincide or the extent overflows float:
        // the search is then the plain scan (a grid that falls short of the
        // box by rounding only puts the last points in the last cell, which
        // the search allows for)
        if (emax > 0.0f && emax < 1e37f) {
            int gd[3];
            // below emax / kGridMaxAxis the longest axis would be cut short
            float lo = emax / (float)(cap < kGridMaxAxis ? cap : kGridMaxAxis), hi = emax;
            for (int it = 0; it < 40; ++it) {  // cells(hi) <= cap throughout
                const float mid = 0.5f * (lo + hi);
                if (grid_cells_at(ext, mid, gd) > cap) lo = mid; else hi = mid;
            }
            grid_cells_at(ext, hi, gd);
            g.ox = v[0];
            g.oy = v[1];
            g.oz = v[2];
            g.h = hi;
            g.inv_h = 1.0f / hi;
            g.gx = gd[0];
            g.gy = gd[1];
            g.gz = gd[2];
            // index error: the subtraction's (half an ulp of the largest
            // magnitude, in cells), the product's (relative 2^-23 of an index
            // below 4096, and of inv_h itself)
            double amax = 0.0;
            for (int a = 0; a < 6; ++a) amax = fmax(amax, fabs((double)v[a]));
            g.margin = (float)(amax * 0x1p-23 / (double)hi + 0x1p-9);
        }
    }
    S.info[b] = g;
}

__device__ __forceinline__ int grid_axis(float t, int g) {
    // floor, saturating; NaN -> 0
    const int c = __float2int_rd(t);
    return c < 0 ? 0 : (c >= g ? g - 1 : c);
}

__device__ __forceinline__ int grid_cell(const GridInfo& g, float x, float y, float z) {
    const int cx = grid_axis(__fmul_rn(__fsub_rn(x, g.ox), g.inv_h), g.gx);
    const int cy = grid_axis(__fmul_rn(__fsub_rn(y, g.oy), g.inv_h), g.gy);
    const int cz = grid_axis(__fmul_rn(__fsub_rn(z, g.oz), g.inv_h), g.gz);
    return (cz * g.gy + cy) * g.gx + cx;
}

// cell of each point (-1: a non-finite coordinate, left out) and the counts
// (grid: point blocks x B x 2 sets)
__global__ void grid_count_kernel(const GridPair P) {
    const GridSet& S = P.s[blockIdx.z];
    const int b = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= S.n) return;
    const float* p = S.pts + ((size_t)b * S.n + i) * 3;
    const float x = p[0], y = p[1], z = p[2];
    int c = -1;
    if (finite3(x, y, z)) {
        c = grid_cell(S.info[b], x, y, z);
        atomicAdd(&S.counts[(size_t)b * S.cap1 + c], 1);
    }
    S.cellid[(size_t)b * S.n + i] = c;
}

__device__ unsigned grid_block_scan(unsigned v, unsigned* sm33, unsigned& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) sm33[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const unsigned w = lane < (int)(blockDim.x >> 5) ? sm33[lane] : 0u;
        unsigned wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        sm33[lane] = wi - w;
        if (lane == 31) sm33[32] = wi;
    }
    __syncthreads();
    const unsigned out = sm33[warp] + incl - v;
    total = sm33[32];
    __syncthreads();
    return out;
}

// Exclusive scan of each item's cell counts into starts (starts[cells] = the
// finite points), in tiles of kScanTile cells: per-tile sums and maxima, a
// scan of the tile sums per item (which also flags an item whose fullest
// cell holds more than 1/32 of its points), then each tile's scan.
// (grid: tiles x B x 2 sets)
__global__ void __launch_bounds__(1024) grid_tile_sums_kernel(const GridPair P) {
    __shared__ uint32_t red_s[32], red_m[32];
    const GridSet& S = P.s[blockIdx.z];
    const int b = blockIdx.y, tile = blockIdx.x;
    if (tile >= S.tiles) return;  // (whole block)
    const GridInfo g = S.info[b];
    const int cells = g.gx * g.gy * g.gz;
    const int i0 = tile * kScanTile + 4 * threadIdx.x;
    const int* c = S.counts + (size_t)b * S.cap1;
    uint32_t s = 0, m = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint32_t v = i0 + t < cells ? (uint32_t)c[i0 + t] : 0u;
        s += v;
        m = max(m, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        red_s[warp] = s;
        red_m[warp] = m;
    }
    __syncthreads();
    if (warp == 0) {
        s = red_s[lane];
        m = red_m[lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            s += __shfl_xor_sync(0xffffffffu, s, o);
            m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
        }
        if (lane == 0) {
            S.tile_sum[(size_t)b * S.tiles + tile] = s;
            S.tile_max[(size_t)b * S.tiles + tile] = m;
        }
    }
}

// one block per item and set (tiles <= 1024): tile sums -> tile offsets in
// place (grid: B x 2 sets)
__global__ void __launch_bounds__(1024) grid_tile_offsets_kernel(const GridPair P) {
    __shared__ unsigned sm33[33];
    __shared__ unsigned smax;
    const GridSet& S = P.s[blockIdx.y];
    const int b = blockIdx.x;
    const GridInfo g = S.info[b];
    const int cells = g.gx * g.gy * g.gz;
    const int used = (cells + kScanTile - 1) / kScanTile;
    if (threadIdx.x == 0) smax = 0u;
    const int t = threadIdx.x;
    const unsigned v = t < used ? S.tile_sum[(size_t)b * S.tiles + t] : 0u;
    const unsigned m = t < used ? S.tile_max[(size_t)b * S.tiles + t] : 0u;
    unsigned total;
    const unsigned off = grid_block_scan(v, sm33, total);  // (synchronises the block)
    if (t < used) S.tile_sum[(size_t)b * S.tiles + t] = off;
    atomicMax(&smax, m);
    __syncthreads();
    if (t == 0) {
        S.starts[(size_t)b * S.cap1 + cells] = (int)total;
        S.info[b].dense = (int64_t)smax * 32 > (int64_t)S.n ? 1 : 0;
    }
}

// (grid: tiles x B x 2 sets)
__global__ void __launch_bounds__(1024) grid_tile_scan_kernel(const GridPair P) {
    __shared__ unsigned sm33[33];
    const GridSet& S = P.s[blockIdx.z];
    const int b = blockIdx.y, tile = blockIdx.x;
    if (tile >= S.tiles) return;  // (whole block)
    const GridInfo g = S.info[b];
    const int cells = g.gx * g.gy * g.gz;
    if (tile * kScanTile >= cells) return;  // (whole block)
    const int i0 = tile * kScanTile + 4 * threadIdx.x;
    const int* c = S.counts + (size_t)b * S.cap1;
    int* s = S.starts + (size_t)b * S.cap1;
    unsigned v[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) v[t] = i0 + t < cells ? (unsigned)c[i0 + t] : 0u;
    unsigned total;
    unsigned o = S.tile_sum[(size_t)b * S.tiles + tile] +
                 grid_block_scan(v[0] + v[1] + v[2] + v[3], sm33, total);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        if (i0 + t < cells) s[i0 + t] = (int)o;
        o += v[t];
    }
}

// The finite points in cell order as (x, y, z, index bits), the counts
// running down to zero as the slots of each cell are taken; and every
// point's starting key as a query, (FLT_MAX, the other set's size).
// (grid: point blocks x B x 2 sets)
__global__ void grid_scatter_kernel(const GridPair P) {
    const GridSet& S = P.s[blockIdx.z];
    const int b = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= S.n) return;
    S.keys[(size_t)b * S.n + i] = dist_key(FLT_MAX, S.other_n);
    const int c = S.cellid[(size_t)b * S.n + i];
    if (c < 0) return;
    const int slot =
        S.starts[(size_t)b * S.cap1 + c] + atomicSub(&S.counts[(size_t)b * S.cap1 + c], 1) - 1;
    const float* p = S.pts + ((size_t)b * S.n + i) * 3;
    S.sorted[(size_t)b * S.n + slot] = make_float4(p[0], p[1], p[2], __int_as_float(i));
}

__device__ __forceinline__ void grid_scan_range(const float4* __restrict__ pts, int lo, int hi,
                                                float qx, float qy, float qz, float& best,
                                                int& bj) {
    for (int p = lo; p < hi; ++p) {
        const float4 r = pts[p];
        const float dx = __fsub_rn(qx, r.x);
        const float dy = __fsub_rn(qy, r.y);
        const float dz = __fsub_rn(qz, r.z);
        const float d = __fmaf_rn(dz, dz, __fmaf_rn(dx, dx, __fmul_rn(dy, dy)));
        const int j = __float_as_int(r.w);
        if (d < best || (d == best && j < bj)) {
            best = d;
            bj = j;
        }
    }
}

// the lexicographic minimum of (d, j) pairs over a group of kGroup lanes
// (aligned, a power of two up to 32; mask = the group's lanes); no candidate
// is (INFINITY, -1), which every candidate beats
template <int kGroup>
__device__ __forceinline__ void group_min_pair(float& best, int& bj, unsigned mask) {
    unsigned long long k = bj >= 0 ? dist_key(best, bj) : ~0ull;
#pragma unroll
    for (int o = kGroup / 2; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(mask, k, o);
        k = other < k ? other : k;
    }
    if (k != ~0ull) {
        best = __uint_as_float((unsigned)(k >> 32) ^ 0x80000000u);
        bj = (int)(unsigned)(k & 0xffffffffu);
    }
}

// the same over a whole block of kGroup (> 32) threads, through red (one
// entry per warp); every thread of the block calls it
template <int kGroup>
__device__ __forceinline__ void block_min_pair(float& best, int& bj, unsigned long long* red) {
    group_min_pair<32>(best, bj, 0xffffffffu);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = bj >= 0 ? dist_key(best, bj) : ~0ull;
    __syncthreads();
    unsigned long long k = red[0];
#pragma unroll
    for (int w = 1; w < kGroup / 32; ++w) k = red[w] < k ? red[w] : k;
    __syncthreads();  // red is free again
    if (k != ~0ull) {
        best = __uint_as_float((unsigned)(k >> 32) ^ 0x80000000u);
        bj = (int)(unsigned)(k & 0xffffffffu);
    }
}

// Gap (in cells, made smaller by the rounding allowance) between the query
// at t and cell k along an axis.
__device__ __forceinline__ float cell_gap(float t, int k, float m2) {
    return fmaxf(fmaxf((float)k - t, t - (float)(k + 1)) - m2, 0.0f);
}

// The search of one query in the reference grid g: rings r0 .. r1 of cells
// around the query's cell, the rows of a ring spread over a group of kGroup
// threads (sub = the thread's place in it; up to 32: aligned lanes of a warp,
// mask = the group's lanes; more: the whole block, red = kGroup / 32 entries
// of shared memory), which takes the minimum after each ring. A row, or the cells of a row, whose gap to the
// query already puts every point in it beyond the thread's best distance is
// skipped. Returns true once no point outside the visited box can beat or tie
// the best (best, bj) found.
struct QueryGeo {
    float x, y, z;
    float t[3];      // position in cells
    int c[3];        // cell (clamped to the grid)
    float fl[3], fu[3];  // distance to the cell's lower / upper face, in cells
    float og2[3];    // squared distance to the grid's slab along the axis, in cells
    float og_sum;
};

__device__ __forceinline__ QueryGeo query_geo(const GridInfo& g, float4 q) {
    QueryGeo Q;
    Q.x = q.x;
    Q.y = q.y;
    Q.z = q.z;
    Q.t[0] = __fmul_rn(__fsub_rn(q.x, g.ox), g.inv_h);
    Q.t[1] = __fmul_rn(__fsub_rn(q.y, g.oy), g.inv_h);
    Q.t[2] = __fmul_rn(__fsub_rn(q.z, g.oz), g.inv_h);
    const int gd[3] = {g.gx, g.gy, g.gz};
    const float m2 = 2.0f * g.margin;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        Q.c[a] = grid_axis(Q.t[a], gd[a]);
        Q.fl[a] = Q.t[a] - (float)Q.c[a];
        Q.fu[a] = (float)(Q.c[a] + 1) - Q.t[a];
        const float o = fmaxf(fmaxf(-Q.t[a], Q.t[a] - (float)gd[a]) - m2, 0.0f);
        Q.og2[a] = o * o;
    }
    Q.og_sum = (Q.og2[0] + Q.og2[1]) + Q.og2[2];
    return Q;
}

template <int kGroup>
__device__ __forceinline__ bool search_rings(const GridInfo& g, const int* __restrict__ st,
                                             const float4* __restrict__ pts, const QueryGeo& Q,
                                             int r0, int r1, float& best, int& bj, int sub,
                                             unsigned mask, unsigned long long* red = nullptr) {
    const float m2 = 2.0f * g.margin;
    const int gd[3] = {g.gx, g.gy, g.gz};
    // a cell is skipped when (its gap)^2 h^2 (1 - 4e-6) > best
    const float skip_scale = g.h * g.h * (1.0f - 4e-6f);
    for (int r = r0; r <= r1; ++r) {
        const int z0 = max(Q.c[2] - r, 0), z1 = min(Q.c[2] + r, g.gz - 1);
        const int y0 = max(Q.c[1] - r, 0), y1 = min(Q.c[1] + r, g.gy - 1);
        const int ny = y1 - y0 + 1, rows = (z1 - z0 + 1) * ny;
        for (int k = sub; k < rows; k += kGroup) {
            const int z = z0 + k / ny, y = y0 + k % ny;
            const float gy = cell_gap(Q.t[1], y, m2), gz = cell_gap(Q.t[2], z, m2);
            // squared x gap (in cells^2) below which a cell of this row can
            // still hold a point no farther than best (no skipping while best
            // is so small that distances may be subnormal, where the relative
            // rounding bound does not hold)
            const float room = best >= 1e-30f ? best / skip_scale - (gy * gy + gz * gz) : INFINITY;
            if (room < 0.0f) continue;
            int xa = max(Q.c[0] - r, 0), xb = min(Q.c[0] + r, g.gx - 1);
            if (room < 1e12f) {  // trim the row to the cells within reach
                const float w = sqrtf(room) + m2;
                xa = max(xa, __float2int_rd(Q.t[0] - w) - 1);
                xb = min(xb, __float2int_rd(Q.t[0] + w) + 1);
            }
            const int row = (z * g.gy + y) * g.gx;
            if (z == Q.c[2] - r || z == Q.c[2] + r || y == Q.c[1] - r || y == Q.c[1] + r) {
                if (xa <= xb)
                    grid_scan_range(pts, st[row + xa], st[row + xb + 1], Q.x, Q.y, Q.z, best, bj);
            } else {  // inner rows: only the ring's two cells
                const int xl = Q.c[0] - r, xr = Q.c[0] + r;
                if (xl >= xa && xl <= xb)
                    grid_scan_range(pts, st[row + xl], st[row + xl + 1], Q.x, Q.y, Q.z, best, bj);
                if (xr >= xa && xr <= xb)
                    grid_scan_range(pts, st[row + xr], st[row + xr + 1], Q.x, Q.y, Q.z, best, bj);
            }
        }
        if (kGroup > 32) block_min_pair<kGroup>(best, bj, red);
        else if (kGroup > 1) group_min_pair<kGroup>(best, bj, mask);
        // a point not visited lies beyond a face of the visited box that has
        // cells behind it (along axis a: at least r + the query's distance to
        // its cell's face, in cells) and inside the grid's slabs along the
        // other two axes
        float lbc = INFINITY;
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            float e = INFINITY;
            if (Q.c[a] - r > 0) e = fminf(e, Q.fl[a]);
            if (Q.c[a] + r < gd[a] - 1) e = fminf(e, Q.fu[a]);
            if (e == INFINITY) continue;
            const float x = fmaxf((float)r + e - m2, 0.0f);
            lbc = fminf(lbc, x * x + (Q.og_sum - Q.og2[a]));
        }
        if (lbc == INFINITY) return true;  // the box holds every cell
        const float lb2 = lbc * g.h * g.h;
        if (lb2 >= 1e-30f && best < lb2 * (1.0f - 4e-6f)) return true;
    }
    return false;
}

constexpr int kThreadRings = 2;  // rings 0 .. 2 by kNearGroup lanes, the rest by a block
constexpr int kNearGroup = 4;
constexpr int kNearThreads = 256;
constexpr int kFarThreads = 256;

// Near search: kNearGroup lanes per query, the queries of set d taken in the
// cell order of their own grid (neighbouring lanes search neighbouring
// cells) against the grid of set 1 - d, over rings 0 .. kThreadRings; a
// query not settled by then goes to its set's hard list with its best so
// far. A query's key is written only when some distance is below infinity
// (it starts at (FLT_MAX, the other set's size)).
// (grid: query blocks x B x 2 directions)
__global__ void __launch_bounds__(kNearThreads) grid_near_kernel(const GridPair P) {
    const int d = blockIdx.z;
    const GridSet& Qs = P.s[d];
    const GridSet& Rs = P.s[1 - d];
    const int b = blockIdx.y;
    const int i = (blockIdx.x * blockDim.x + threadIdx.x) / kNearGroup;
    const int sub = threadIdx.x & (kNearGroup - 1);
    const unsigned mask = ((1u << kNearGroup) - 1u) << (threadIdx.x & 31 & ~(kNearGroup - 1));
    const GridInfo g = Rs.info[b];
    if (g.dense) return;  // the plain scan serves this item (whole block)
    // the finite queries are the sorted ones; the others keep the starting
    // key, which no distance from them can replace (whole group)
    {
        const GridInfo qg = Qs.info[b];
        if (i >= Qs.n || i >= Qs.starts[(size_t)b * Qs.cap1 + qg.gx * qg.gy * qg.gz]) return;
    }
    const float4 q = Qs.sorted[(size_t)b * Qs.n + i];
    const QueryGeo Q = query_geo(g, q);
    float best = INFINITY;
    int bj = -1;
    const bool done = search_rings<kNearGroup>(g, Rs.starts + (size_t)b * Rs.cap1,
                                               Rs.sorted + (size_t)b * Rs.n, Q, 0, kThreadRings,
                                               best, bj, sub, mask);
    if (sub != 0) return;
    const unsigned long long key = bj >= 0 ? dist_key(best, bj) : ~0ull;
    if (done) {
        if (bj >= 0) Qs.keys[(size_t)b * Qs.n + __float_as_int(q.w)] = key;
    } else {
        const unsigned slot = atomicAdd(&P.counters[d], 1u);
        Qs.hard[slot] = HardQuery{b, i, key};
    }
}

// Far search: persistent blocks over both hard lists, each taking the next
// query and resuming its search at ring kThreadRings + 1 with its threads
// sharing the rows.
__global__ void __launch_bounds__(kFarThreads) grid_far_kernel(const GridPair P) {
    __shared__ unsigned long long red[kFarThreads / 32];
    __shared__ unsigned next;
    const unsigned count0 = P.counters[0], count = count0 + P.counters[1];
    for (;;) {
        if (threadIdx.x == 0) next = atomicAdd(&P.counters[2], 1u);
        __syncthreads();
        const unsigned idx = next;
        __syncthreads();  // next is read before thread 0 writes it again
        if (idx >= count) break;
        const int d = idx < count0 ? 0 : 1;
        const GridSet& Qs = P.s[d];
        const GridSet& Rs = P.s[1 - d];
        const HardQuery h = Qs.hard[d == 0 ? idx : idx - count0];
        const GridInfo g = Rs.info[h.b];
        const float4 q = Qs.sorted[(size_t)h.b * Qs.n + h.i];
        const QueryGeo Q = query_geo(g, q);
        float best = INFINITY;
        int bj = -1;
        if (h.key != ~0ull) {
            best = __uint_as_float((unsigned)(h.key >> 32) ^ 0x80000000u);
            bj = (int)(unsigned)(h.key & 0xffffffffu);
        }
        search_rings<kFarThreads>(g, Rs.starts + (size_t)h.b * Rs.cap1,
                                  Rs.sorted + (size_t)h.b * Rs.n, Q, kThreadRings + 1, INT_MAX,
                                  best, bj, threadIdx.x, 0u, red);
        if (threadIdx.x == 0 && bj >= 0)
            Qs.keys[(size_t)h.b * Qs.n + __float_as_int(q.w)] = dist_key(best, bj);
    }
}

// Workspace of the nearest / Chamfer entries: the 64-bit keys of both sets,
// then (for sets large enough for the grid search) the grid arrays of both
// sets and the three hard-query counters.
size_t nearest_space(int B, int M, int N, GridSpace* ga, GridSpace* gb, size_t* counters) {
    const size_t keys = (size_t)B * ((size_t)M + N) * sizeof(unsigned long long);
    if (!use_grid(M, N)) return keys;
    const GridSpace a = grid_space(B, M, keys);
    const GridSpace b = grid_space(B, N, a.bytes);
    if (ga) *ga = a;
    if (gb) *gb = b;
    if (counters) *counters = b.bytes;
    return b.bytes + 256;
}

GridSet grid_set(char* ws, const GridSpace& gs, const float* pts, int B, int n, int other_n,
                 unsigned long long* keys) {
    GridSet S;
    S.pts = pts;
    S.n = n;
    S.other_n = other_n;
    S.cap1 = grid_cell_cap(n) + 1;
    S.tiles = grid_tiles(n);
    S.info = reinterpret_cast<GridInfo*>(ws + gs.info);
    S.box = reinterpret_cast<uint32_t*>(ws + gs.box);
    S.tile_sum = reinterpret_cast<uint32_t*>(ws + gs.tile_sum);
    S.tile_max = reinterpret_cast<uint32_t*>(ws + gs.tile_max);
    S.cellid = reinterpret_cast<int*>(ws + gs.cellid);
    S.counts = reinterpret_cast<int*>(ws + gs.counts);
    S.starts = reinterpret_cast<int*>(ws + gs.starts);
    S.sorted = reinterpret_cast<float4*>(ws + gs.sorted);
    S.keys = keys;
    S.hard = reinterpret_cast<HardQuery*>(ws + gs.hard);
    (void)B;
    return S;
}

// Both directions into k1 (first -> second) and k2 (second -> first): the
// plain scan for small sets; otherwise both grids, the plain scan for the
// items whose reference grid is too dense, and the near and far searches.
int both_ways(const float* first, const float* second, int B, int M, int N, void* workspace,
              unsigned long long* k1, unsigned long long* k2, cudaStream_t st) {
    if (!use_grid(M, N)) {
        F2S_TRY(one_way(first, second, B, M, N, k1, st));
        return one_way(second, first, B, N, M, k2, st);
    }
    F2S_LIMIT(B <= 65535, "nearest: batch %d too large for the grid search", B);
    GridSpace ga, gb;
    size_t counters_at = 0;
    nearest_space(B, M, N, &ga, &gb, &counters_at);
    char* ws = static_cast<char*>(workspace);
    GridPair P;
    P.s[0] = grid_set(ws, ga, first, B, M, N, k1);
    P.s[1] = grid_set(ws, gb, second, B, N, M, k2);
    P.B = B;
    P.counters = reinterpret_cast<unsigned*>(ws + counters_at);
    const int nmax = M > N ? M : N;
    const int tmax = P.s[0].tiles > P.s[1].tiles ? P.s[0].tiles : P.s[1].tiles;
    const int64_t cells = (int64_t)B * (P.s[0].cap1 > P.s[1].cap1 ? P.s[0].cap1 : P.s[1].cap1);
    int prep = (int)((cells + 255) / 256);
    prep = prep < ceil_div(6 * B, 256) ? ceil_div(6 * B, 256) : prep;
    prep = prep > 8 * sm_count() ? 8 * sm_count() : prep;
    grid_prepare_kernel<<<dim3(prep, 2), 256, 0, st>>>(P);
    F2S_TRY(check_launch("grid_prepare_kernel"));
    const int box_blocks = ceil_div(nmax, 256 * 16) < 64 ? ceil_div(nmax, 256 * 16) : 64;
    grid_box_kernel<<<dim3(box_blocks, B, 2), 256, 0, st>>>(P);
    F2S_TRY(check_launch("grid_box_kernel"));
    grid_param_kernel<<<dim3(ceil_div(B, 128), 2), 128, 0, st>>>(P);
    F2S_TRY(check_launch("grid_param_kernel"));
    const dim3 pg(ceil_div(nmax, 256), B, 2);
    grid_count_kernel<<<pg, 256, 0, st>>>(P);
    F2S_TRY(check_launch("grid_count_kernel"));
    grid_tile_sums_kernel<<<dim3(tmax, B, 2), 1024, 0, st>>>(P);
    F2S_TRY(check_launch("grid_tile_sums_kernel"));
    grid_tile_offsets_kernel<<<dim3(B, 2), 1024, 0, st>>>(P);
    F2S_TRY(check_launch("grid_tile_offsets_kernel"));
    grid_tile_scan_kernel<<<dim3(tmax, B, 2), 1024, 0, st>>>(P);
    F2S_TRY(check_launch("grid_tile_scan_kernel"));
    grid_scatter_kernel<<<pg, 256, 0, st>>>(P);
    F2S_TRY(check_launch("grid_scatter_kernel"));
    // the items whose reference grid is too dense (their keys were started above)
    F2S_TRY(one_way(first, second, B, M, N, k1, st, P.s[1].info, false));
    F2S_TRY(one_way(second, first, B, N, M, k2, st, P.s[0].info, false));
    grid_near_kernel<<<dim3(ceil_div(nmax, kNearThreads / kNearGroup), B, 2), kNearThreads, 0,
                       st>>>(P);
    F2S_TRY(check_launch("grid_near_kernel"));
    grid_far_kernel<<<4 * sm_count(), kFarThreads, 0, st>>>(P);
    return check_launch("grid_far_kernel");
}

// ---------------------------------------------------------------------------
// Point-to-triangle-mesh distance (flow2surf/evaluation.py:31-34, which takes
// it from point_cloud_utils' closest_points_on_mesh): for each point the
// squared distance to the closest point of the closest triangle. The closest
// point on a triangle follows the region classification of Ericson,
// Real-Time Collision Detection (2005), sec. 5.1.5: the point's dot products
// with the two edges from a vertex decide whether the closest feature is a
// vertex, an edge or the face, in a fixed order; here written without
// branches (every region's barycentric pair is formed and the first region
// that holds is selected), with the per-triangle dot products precomputed.
// ---------------------------------------------------------------------------
constexpr int kTriTile = 512;
constexpr int kTriFloats = 12;  // a (3), ab (3), ac (3), |ab|^2, |ac|^2, ab.ac

__global__ void triangle_prep_kernel(const float* __restrict__ vertices, int V,
                                     const int32_t* __restrict__ faces, int F,
                                     float* __restrict__ tri) {
    for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F; f += gridDim.x * blockDim.x) {
        int i[3];
#pragma unroll
        for (int e = 0; e < 3; ++e) {
            const int v = faces[3 * (size_t)f + e];
            i[e] = v < 0 ? 0 : (v >= V ? V - 1 : v);  // the host checks the range first
        }
        const float* a = vertices + 3 * (size_t)i[0];
        const float* b = vertices + 3 * (size_t)i[1];
        const float* c = vertices + 3 * (size_t)i[2];
        const float ab[3] = {b[0] - a[0], b[1] - a[1], b[2] - a[2]};
        const float ac[3] = {c[0] - a[0], c[1] - a[1], c[2] - a[2]};
        float* o = tri + (size_t)f * kTriFloats;
        o[0] = a[0];
        o[1] = a[1];
        o[2] = a[2];
        o[3] = ab[0];
        o[4] = ab[1];
        o[5] = ab[2];
        o[6] = ac[0];
        o[7] = ac[1];
        o[8] = ac[2];
        o[9] = ab[0] * ab[0] + ab[1] * ab[1] + ab[2] * ab[2];
        o[10] = ac[0] * ac[0] + ac[1] * ac[1] + ac[2] * ac[2];
        o[11] = ab[0] * ac[0] + ab[1] * ac[1] + ab[2] * ac[2];
    }
}

// Squared distance from p to the triangle (a, a + ab, a + ac).
__device__ __forceinline__ float point_triangle_sq(float px, float py, float pz, const float* t) {
    const float apx = px - t[0], apy = py - t[1], apz = pz - t[2];
    const float d1 = t[3] * apx + t[4] * apy + t[5] * apz;  // ab . ap
    const float d2 = t[6] * apx + t[7] * apy + t[8] * apz;  // ac . ap
    const float d3 = d1 - t[9];                             // ab . bp
    const float d4 = d2 - t[11];                            // ac . bp
    const float d5 = d1 - t[11];                            // ab . cp
    const float d6 = d2 - t[10];                            // ac . cp
    const float vc = d1 * d4 - d3 * d2;
    const float vb = d5 * d2 - d1 * d6;
    const float va = d3 * d6 - d5 * d4;
    // face region by default, then the edge and vertex regions in reverse
    // order of precedence, so the first region that holds wins
    // (__fdividef: ~2 ulp, a displacement of ~1e-7 of an edge along it)
    const float inv = __fdividef(1.0f, va + vb + vc);
    float v = vb * inv, w = vc * inv;
    const float e43 = d4 - d3, e56 = d5 - d6;
    if (va <= 0.0f && e43 >= 0.0f && e56 >= 0.0f) {  // edge bc
        w = __fdividef(e43, e43 + e56);
        v = 1.0f - w;
    }
    if (vb <= 0.0f && d2 >= 0.0f && d6 <= 0.0f) {  // edge ac
        v = 0.0f;
        w = __fdividef(d2, d2 - d6);
    }
    if (d6 >= 0.0f && d5 <= d6) {  // vertex c
        v = 0.0f;
        w = 1.0f;
    }
    if (vc <= 0.0f && d1 >= 0.0f && d3 <= 0.0f) {  // edge ab
        v = __fdividef(d1, d1 - d3);
        w = 0.0f;
    }
    if (d3 >= 0.0f && d4 <= d3) {  // vertex b
        v = 1.0f;
        w = 0.0f;
    }
    if (d1 <= 0.0f && d2 <= 0.0f) {  // vertex a
        v = 0.0f;
        w = 0.0f;
    }
    const float dx = apx - (v * t[3] + w * t[6]);
    const float dy = apy - (v * t[4] + w * t[7]);
    const float dz = apz - (v * t[5] + w * t[8]);
    return dx * dx + dy * dy + dz * dz;
}

// keys[i] = min over triangles f of dist_key(d^2(point_i, f), f); the
// triangles split across blockIdx.y chunks and folded with atomicMin.
__global__ void __launch_bounds__(kThreads)
point_mesh_kernel(const float* __restrict__ points, int M, const float* __restrict__ tri, int F,
                  int tri_chunk, unsigned long long* __restrict__ keys) {
    __shared__ float tile[kTriTile * kTriFloats];
    const int q0 = blockIdx.x * kQueriesPerCta;
    const int f_lo = blockIdx.y * tri_chunk;
    const int f_hi = min(F, f_lo + tri_chunk);
    float px[kQpt], py[kQpt], pz[kQpt], best[kQpt];
    int bf[kQpt];
#pragma unroll
    for (int t = 0; t < kQpt; ++t) {
        const int i = q0 + threadIdx.x + kThreads * t;
        const bool in = i < M;
        px[t] = in ? points[3 * (size_t)i] : 0.0f;
        py[t] = in ? points[3 * (size_t)i + 1] : 0.0f;
        pz[t] = in ? points[3 * (size_t)i + 2] : 0.0f;
        best[t] = INFINITY;
        bf[t] = -1;
    }
    for (int f0 = f_lo; f0 < f_hi; f0 += kTriTile) {
        const int count = min(kTriTile, f_hi - f0);
        __syncthreads();
        for (int j = threadIdx.x; j < count * kTriFloats; j += kThreads)
            tile[j] = tri[(size_t)f0 * kTriFloats + j];
        __syncthreads();
        for (int f = 0; f < count; ++f) {
            const float* tr = tile + f * kTriFloats;
#pragma unroll
            for (int t = 0; t < kQpt; ++t) {
                const float d = point_triangle_sq(px[t], py[t], pz[t], tr);
                if (d < best[t]) {
                    best[t] = d;
                    bf[t] = f0 + f;
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < kQpt; ++t) {
        const int i = q0 + threadIdx.x + kThreads * t;
        if (i < M && bf[t] >= 0) atomicMin(&keys[i], dist_key(best[t], bf[t]));
    }
}

int check_sets(const float* first, const float* second, int B, int M, int N) {
    F2S_REQUIRE(B >= 0, "batch must be >= 0");
    F2S_REQUIRE(M >= 1 && N >= 1, "Point sets must be nonempty");
    F2S_REQUIRE(first && second, "nearest: null pointer");
    return F2S_OK;
}

}  // namespace
}  // namespace f2s

using namespace f2s;

extern "C" int f2s_nearest_workspace_bytes(int B, int M, int N, size_t* bytes) {
    F2S_REQUIRE(B >= 0 && M >= 0 && N >= 0 && bytes, "bad workspace query");
    *bytes = nearest_space(B, M, N, nullptr, nullptr, nullptr);
    return F2S_OK;
}

extern "C" int f2s_nearest(const float* first, const float* second, int B, int M, int N,
                           float* first_distance, int32_t* second_index, float* second_distance,
                           int32_t* first_index, void* workspace, size_t workspace_bytes,
                           void* stream) {
    F2S_TRY(check_sets(first, second, B, M, N));
    if (B == 0) return F2S_OK;
    F2S_REQUIRE(first_distance && second_index && second_distance && first_index && workspace,
                "nearest: null pointer");
    const size_t need = nearest_space(B, M, N, nullptr, nullptr, nullptr);
    if (workspace_bytes < need)
        return fail(F2S_ERR_WORKSPACE, "nearest needs %zu workspace bytes, got %zu", need,
                    workspace_bytes);
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagNearest, st);
    unsigned long long* k1 = static_cast<unsigned long long*>(workspace);
    unsigned long long* k2 = k1 + (size_t)B * M;
    F2S_TRY(both_ways(first, second, B, M, N, workspace, k1, k2, st));
    unpack_kernel<<<grid_1d((int64_t)B * M), 256, 0, st>>>(k1, (int64_t)B * M, first_distance,
                                                           second_index);
    F2S_TRY(check_launch("unpack_kernel"));
    unpack_kernel<<<grid_1d((int64_t)B * N), 256, 0, st>>>(k2, (int64_t)B * N, second_distance,
                                                           first_index);
    return check_launch("unpack_kernel");
}

extern "C" int f2s_chamfer(const float* pred, const float* target, int B, int M, int N,
                           double* chamfer, void* workspace, size_t workspace_bytes,
                           void* stream) {
    F2S_TRY(check_sets(pred, target, B, M, N));
    if (B == 0) return F2S_OK;
    F2S_REQUIRE(chamfer && workspace, "chamfer: null pointer");
    const size_t need = nearest_space(B, M, N, nullptr, nullptr, nullptr);
    if (workspace_bytes < need)
        return fail(F2S_ERR_WORKSPACE, "chamfer needs %zu workspace bytes, got %zu", need,
                    workspace_bytes);
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagNearest, st);
    unsigned long long* k1 = static_cast<unsigned long long*>(workspace);
    unsigned long long* k2 = k1 + (size_t)B * M;
    F2S_TRY(both_ways(pred, target, B, M, N, workspace, k1, k2, st));
    chamfer_reduce_kernel<<<B, 1024, 0, st>>>(k1, M, k2, N, chamfer);
    return check_launch("chamfer_reduce_kernel");
}

// ---------------------------------------------------------------------------
// Chamfer without any allocation, for callers that cannot call cudaMalloc:
// code running inside a caching allocator's out-of-memory handler, a host
// that forbids device allocation after start-up, or a caller in the middle of
// other work that must not synchronise the device (cudaMalloc/cudaFree can).
// The 64-bit distance keys live in one file-scope device array of
// F2S_CHAMFER_STATIC_MAX_POINTS entries (16 MiB), which every GPU that loads
// this library keeps until the process exits.
// ---------------------------------------------------------------------------
#include <mutex>

static __device__ __align__(256) unsigned long long
    g_chamfer_scratch[F2S_CHAMFER_STATIC_MAX_POINTS];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
unsigned long long* g_scratch_address[kMaxDevices] = {nullptr};

// The device address of g_chamfer_scratch on the current device. In host code
// the array's name is only a host-side stand-in, so the address is looked up
// once per device (with that device current) and cached. With CUDA's lazy
// module loading (the default) that first look-up is also what loads this
// file's module on the device and so reserves the array; the kernels the
// entry launches are loaded here too (cudaFuncGetAttributes loads a
// function), so later calls load and reserve nothing.
int chamfer_scratch(unsigned long long** out) {
    int dev = 0;
    F2S_CUDA_TRY(cudaGetDevice(&dev));
    F2S_LIMIT(dev >= 0 && dev < kMaxDevices, "device ordinal %d beyond %d", dev, kMaxDevices);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (g_scratch_address[dev] == nullptr) {
        void* ptr = nullptr;
        F2S_CUDA_TRY(cudaGetSymbolAddress(&ptr, g_chamfer_scratch));
        cudaFuncAttributes attr;
        F2S_CUDA_TRY(cudaFuncGetAttributes(&attr, init_keys_kernel));
        F2S_CUDA_TRY(cudaFuncGetAttributes(&attr, nearest_kernel));
        F2S_CUDA_TRY(cudaFuncGetAttributes(&attr, chamfer_reduce_kernel));
        g_scratch_address[dev] = static_cast<unsigned long long*>(ptr);
    }
    *out = g_scratch_address[dev];
    return F2S_OK;
}
}  // namespace

extern "C" int f2s_chamfer_static(const float* pred, const float* target, int B, int M, int N,
                                  double* chamfer, void* stream) {
    F2S_TRY(check_sets(pred, target, B, M, N));
    // the per-device set-up comes first, so that a call with B = 0 does it and
    // nothing else: the way to prepare a device before allocation is ruled out
    unsigned long long* k1 = nullptr;
    F2S_TRY(chamfer_scratch(&k1));
    if (B == 0) return F2S_OK;
    F2S_REQUIRE(chamfer != nullptr, "chamfer: null pointer");
    const int64_t keys = (int64_t)B * ((int64_t)M + N);
    F2S_LIMIT(keys <= F2S_CHAMFER_STATIC_MAX_POINTS,
              "chamfer_static: B*(M+N) = %lld points exceed the built-in scratch of %d; use "
              "f2s_chamfer with a caller workspace",
              (long long)keys, F2S_CHAMFER_STATIC_MAX_POINTS);
    unsigned long long* k2 = k1 + (size_t)B * M;
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagNearest, st);
    // one_way() rewrites every key it uses with its starting value first, so
    // whatever an earlier call left in the array does not matter.
    F2S_TRY(one_way(pred, target, B, M, N, k1, st));
    F2S_TRY(one_way(target, pred, B, N, M, k2, st));
    chamfer_reduce_kernel<<<B, 1024, 0, st>>>(k1, M, k2, N, chamfer);
    return check_launch("chamfer_reduce_kernel");
}

extern "C" int f2s_point_to_mesh_workspace_bytes(int M, int F, size_t* bytes) {
    F2S_REQUIRE(M >= 0 && F >= 0 && bytes, "bad workspace query");
    *bytes = (((size_t)F * kTriFloats * sizeof(float) + 255) & ~size_t(255)) +
             (size_t)M * sizeof(unsigned long long);
    return F2S_OK;
}

extern "C" int f2s_point_to_mesh(const float* points, int M, const float* vertices, int V,
                                 const int32_t* faces, int F, float* sq_distance,
                                 int32_t* face_index, void* workspace, size_t workspace_bytes,
                                 void* stream) {
    F2S_REQUIRE(M >= 0 && V >= 0 && F >= 0, "point_to_mesh: bad sizes M=%d V=%d F=%d", M, V, F);
    if (M == 0) return F2S_OK;
    F2S_REQUIRE(V >= 1 && F >= 1, "point_to_mesh: the mesh is empty (V=%d, F=%d)", V, F);
    F2S_REQUIRE(points && vertices && faces && sq_distance && face_index && workspace,
                "point_to_mesh: null pointer");
    size_t need = 0;
    F2S_TRY(f2s_point_to_mesh_workspace_bytes(M, F, &need));
    if (workspace_bytes < need)
        return fail(F2S_ERR_WORKSPACE, "point_to_mesh needs %zu workspace bytes, got %zu", need,
                    workspace_bytes);
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagNearest, st);
    float* tri = static_cast<float*>(workspace);
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(
        static_cast<char*>(workspace) + (((size_t)F * kTriFloats * sizeof(float) + 255) & ~size_t(255)));
    triangle_prep_kernel<<<grid_1d(F), 256, 0, st>>>(vertices, V, faces, F, tri);
    F2S_TRY(check_launch("triangle_prep_kernel"));
    init_keys_kernel<<<grid_1d(M), 256, 0, st>>>(keys, M, F);
    F2S_TRY(check_launch("init_keys_kernel"));
    const int qblocks = ceil_div(M, kQueriesPerCta);
    int splits = (4 * sm_count() + qblocks - 1) / qblocks;
    const int max_splits = ceil_div(F, kTriTile);
    splits = splits < 1 ? 1 : (splits > max_splits ? max_splits : splits);
    const int chunk = ceil_div(ceil_div(F, splits), kTriTile) * kTriTile;
    dim3 grid(qblocks, ceil_div(F, chunk));
    F2S_LIMIT(grid.y <= 65535, "point_to_mesh: grid too large");
    point_mesh_kernel<<<grid, kThreads, 0, st>>>(points, M, tri, F, chunk, keys);
    F2S_TRY(check_launch("point_mesh_kernel"));
    unpack_kernel<<<grid_1d(M), 256, 0, st>>>(keys, M, sq_distance, face_index);
    return check_launch("unpack_kernel");
}
