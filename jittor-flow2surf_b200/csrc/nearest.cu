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

__global__ void init_keys_kernel(unsigned long long* keys, int64_t count, int reference_count) {
    const unsigned long long k0 = dist_key(FLT_MAX, reference_count);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x)
        keys[i] = k0;
}

__global__ void __launch_bounds__(kThreads)
nearest_kernel(const float* __restrict__ query, const float* __restrict__ ref, int M, int N,
               int ref_chunk, unsigned long long* __restrict__ keys) {
    __shared__ float4 tile[kTile];
    const int b = blockIdx.z;
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
    double s1 = 0.0, s2 = 0.0;
    for (int i = threadIdx.x; i < M; i += 1024)
        s1 += (double)__uint_as_float((unsigned)(k1[(size_t)b * M + i] >> 32) ^ 0x80000000u);
    for (int j = threadIdx.x; j < N; j += 1024)
        s2 += (double)__uint_as_float((unsigned)(k2[(size_t)b * N + j] >> 32) ^ 0x80000000u);
    double v = s1 / (double)M + s2 / (double)N;
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
int one_way(const float* query, const float* ref, int B, int M, int N, unsigned long long* keys,
            cudaStream_t st) {
    const int64_t count = (int64_t)B * M;
    init_keys_kernel<<<grid_1d(count), 256, 0, st>>>(keys, count, N);
    F2S_TRY(check_launch("init_keys_kernel"));
    const int qblocks = ceil_div(M, kQueriesPerCta);
    const int64_t base = (int64_t)qblocks * B;
    int splits = (int)((4ll * sm_count() + base - 1) / base);
    const int max_splits = ceil_div(N, kTile);
    splits = splits < 1 ? 1 : (splits > max_splits ? max_splits : splits);
    const int ref_chunk = ceil_div(ceil_div(N, splits), kTile) * kTile;
    dim3 grid(qblocks, ceil_div(N, ref_chunk), B);
    F2S_LIMIT(grid.y <= 65535 && grid.z <= 65535, "nearest: grid too large");
    nearest_kernel<<<grid, kThreads, 0, st>>>(query, ref, M, N, ref_chunk, keys);
    return check_launch("nearest_kernel");
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
    *bytes = (size_t)B * ((size_t)M + N) * sizeof(unsigned long long);
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
    const size_t need = (size_t)B * ((size_t)M + N) * sizeof(unsigned long long);
    if (workspace_bytes < need)
        return fail(F2S_ERR_WORKSPACE, "nearest needs %zu workspace bytes, got %zu", need,
                    workspace_bytes);
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagNearest, st);
    unsigned long long* k1 = static_cast<unsigned long long*>(workspace);
    unsigned long long* k2 = k1 + (size_t)B * M;
    F2S_TRY(one_way(first, second, B, M, N, k1, st));
    F2S_TRY(one_way(second, first, B, N, M, k2, st));
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
    const size_t need = (size_t)B * ((size_t)M + N) * sizeof(unsigned long long);
    if (workspace_bytes < need)
        return fail(F2S_ERR_WORKSPACE, "chamfer needs %zu workspace bytes, got %zu", need,
                    workspace_bytes);
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagNearest, st);
    unsigned long long* k1 = static_cast<unsigned long long*>(workspace);
    unsigned long long* k2 = k1 + (size_t)B * M;
    F2S_TRY(one_way(pred, target, B, M, N, k1, st));
    F2S_TRY(one_way(target, pred, B, N, M, k2, st));
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
