// Device-resident patch_denoise pieces (flow2surf/inference.py:19-198):
// farthest-point seeds, the patch index, the centre-weighted fusion structure,
// the per-step patch gather and the fused vote aggregation + Euler update.
#include <cfloat>
#include <cooperative_groups.h>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace f2s {
namespace {

constexpr int kFpsThreads = 1024;
constexpr int kFpsMaxCluster = 8;
// x, y, z and the running minimum per point in shared memory (16 bytes).
constexpr int kFpsSmemPoints = (224 * 1024) / 16;

__device__ __forceinline__ unsigned long long u64max(unsigned long long a,
                                                     unsigned long long b) {
    return a > b ? a : b;
}

__device__ unsigned long long block_max_u64(unsigned long long v, unsigned long long* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = u64max(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = u64max(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[32] = v;
    }
    __syncthreads();
    return red[32];
}

// Farthest-point sampling, bit-exact to _farthest_point_indices
// (inference.py:19-41): each ufunc of the NumPy loop is a separately rounded
// float32 operation, d = ((x-cx)^2 + (y-cy)^2) + (z-cz)^2 (:30-37); the
// running minimum only ever holds float32 values (:24,38); argmax takes the
// first maximum (:39), i.e. the largest (value, -index) key.
// A cluster of up to 8 CTAs splits the points; per iteration each CTA reduces
// its slice and every CTA reads all partial maxima over distributed shared
// memory (double-buffered, one cluster barrier per selected seed).
template <bool SMEM>
__global__ void __launch_bounds__(kFpsThreads)
fps_kernel(const float* __restrict__ pts, int N, int count, int first, int slice,
           float* __restrict__ gmin, int32_t* __restrict__ sel) {
    extern __shared__ __align__(16) float4 fps_sm[];
    __shared__ unsigned long long red[33];
    __shared__ unsigned long long part[2];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int csize = (int)cluster.num_blocks();
    const int lo = rank * slice;
    const int hi = min(N, lo + slice);
    const int tid = threadIdx.x;

    if (SMEM) {
        for (int n = lo + tid; n < hi; n += kFpsThreads)
            fps_sm[n - lo] = make_float4(pts[3 * n], pts[3 * n + 1], pts[3 * n + 2], INFINITY);
    } else {
        for (int n = lo + tid; n < hi; n += kFpsThreads) gmin[n] = INFINITY;
    }
    if (rank == 0 && tid == 0) sel[0] = first;
    int cur = first;
    __syncthreads();

    for (int i = 1; i < count; ++i) {
        const float cx = pts[3 * cur], cy = pts[3 * cur + 1], cz = pts[3 * cur + 2];
        unsigned long long best = 0ull;
        for (int n = lo + tid; n < hi; n += kFpsThreads) {
            float x, y, z, m;
            if (SMEM) {
                const float4 p = fps_sm[n - lo];
                x = p.x; y = p.y; z = p.z; m = p.w;
            } else {
                x = pts[3 * n]; y = pts[3 * n + 1]; z = pts[3 * n + 2]; m = gmin[n];
            }
            float d = __fsub_rn(x, cx);
            d = __fmul_rn(d, d);
            float w = __fsub_rn(y, cy);
            w = __fmul_rn(w, w);
            d = __fadd_rn(d, w);
            w = __fsub_rn(z, cz);
            w = __fmul_rn(w, w);
            d = __fadd_rn(d, w);
            m = d < m ? d : m;
            if (SMEM)
                fps_sm[n - lo].w = m;
            else
                gmin[n] = m;
            const unsigned long long key =
                ((unsigned long long)__float_as_uint(m) << 32) | (0xffffffffu - (unsigned)n);
            best = u64max(best, key);
        }
        best = block_max_u64(best, red);
        if (tid == 0) part[i & 1] = best;
        cluster.sync();
        unsigned long long g = 0ull;
        if (tid < 32) {
            unsigned long long v = 0ull;
            if (tid < csize) v = *cluster.map_shared_rank(&part[i & 1], tid);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = u64max(v, __shfl_xor_sync(0xffffffffu, v, o));
            g = v;
            if (tid == 0) red[32] = g;
        }
        __syncthreads();
        g = red[32];
        cur = (int)(0xffffffffu - (unsigned)(g & 0xffffffffu));
        if (rank == 0 && tid == 0) sel[i] = cur;
        __syncthreads();
    }
    cluster.sync();  // no CTA exits while a peer may still read its `part`
}

// The same sampling for clouds beyond one cluster's shared memory: one
// cooperative grid of up to one CTA per SM, each CTA's slice (xyz and the
// running minimum) resident in its shared memory. Per seed every CTA reduces
// its slice to one (distance, -index) key, folds it into the seed's slot in
// global memory with a 64-bit atomicMax and counts itself in on an arrival
// counter; one thread per CTA polls the counter (a bounded wait: it gives up
// after kFpsPollLimit polls, records kTcWaitTimeout in the device error word
// and the grid returns) and reads the winner. Same arithmetic and tie-break
// as fps_kernel, so the seeds are identical; slots and counter are zeroed by
// the host before the launch.
constexpr int kFpsGridThreads = 512;
constexpr uint32_t kFpsPollLimit = 1u << 22;

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kFpsGridThreads)
fps_grid_kernel(const float* __restrict__ pts, int N, int count, int first, int slice,
                unsigned long long* __restrict__ slots, unsigned* __restrict__ arrived,
                int32_t* __restrict__ sel, int* __restrict__ err) {
    extern __shared__ __align__(16) float4 fps_sm[];
    __shared__ unsigned long long red[33];
    __shared__ int s_cur;
    const int lo = blockIdx.x * slice;
    const int hi = min(N, lo + slice);
    const int tid = threadIdx.x;
    for (int n = lo + tid; n < hi; n += kFpsGridThreads)
        fps_sm[n - lo] = make_float4(pts[3 * n], pts[3 * n + 1], pts[3 * n + 2], INFINITY);
    if (blockIdx.x == 0 && tid == 0) sel[0] = first;
    int cur = first;
    __syncthreads();
    const unsigned grid = gridDim.x;
    for (int i = 1; i < count; ++i) {
        const float cx = pts[3 * cur], cy = pts[3 * cur + 1], cz = pts[3 * cur + 2];
        unsigned long long best = 0ull;
        for (int n = lo + tid; n < hi; n += kFpsGridThreads) {
            const float4 p = fps_sm[n - lo];
            float d = __fsub_rn(p.x, cx);
            d = __fmul_rn(d, d);
            float w = __fsub_rn(p.y, cy);
            w = __fmul_rn(w, w);
            d = __fadd_rn(d, w);
            w = __fsub_rn(p.z, cz);
            w = __fmul_rn(w, w);
            d = __fadd_rn(d, w);
            const float m = d < p.w ? d : p.w;
            fps_sm[n - lo].w = m;
            best = u64max(best, ((unsigned long long)__float_as_uint(m) << 32) |
                                    (0xffffffffu - (unsigned)n));
        }
        best = block_max_u64(best, red);
        if (tid == 0) {
            atomicMax(&slots[i], best);
            __threadfence();  // the slot's update is visible before the arrival
            atomicAdd(arrived, 1u);
            const unsigned target = (unsigned)i * grid;
            int next = -1;
            uint32_t poll = 0;
            for (; poll < kFpsPollLimit; ++poll) {
                if (ld_acquire_gpu(arrived) >= target) {
                    next = (int)(0xffffffffu - (unsigned)(ld_relaxed_gpu(&slots[i]) & 0xffffffffu));
                    break;
                }
                if ((poll & 255u) == 255u && *reinterpret_cast<volatile int*>(err) != tc::kTcOk)
                    break;
            }
            if (poll == kFpsPollLimit) atomicExch(err, tc::kTcWaitTimeout);
            s_cur = next;
        }
        __syncthreads();
        cur = s_cur;
        if (cur < 0) return;  // a wait gave up: the whole CTA leaves
        if (blockIdx.x == 0 && tid == 0) sel[i] = cur;
    }
}

// ---------------------------------------------------------------------------
// Patch index: per seed, the k nearest points by float64 squared distance
// ((dx^2 + dy^2) + dz^2 of float32 coordinates, as scipy's cKDTree computes
// it for p = 2), ordered by (distance, index); radial positions
// r = d / (d_max + 1e-8) (inference.py:110-122) and vote weights
// w = exp(-beta r r) (:124-127). One CTA per seed: exact 8-pass radix select
// of the k-th 64-bit key, ordered compaction, bitonic sort in shared memory.
// The histogram passes walk the points with the block's stride, so a warp's
// coordinate loads are coalesced (the ordered compaction keeps contiguous
// per-thread ranges); the distances from one seed share their high bytes, so
// the histogram adds of a warp mostly hit one bin and are aggregated per
// distinct bin (__match_any_sync) before the shared-memory atomic.
// ---------------------------------------------------------------------------
constexpr int kPiThreads = 1024;

__device__ __forceinline__ double sqdist64(const float* p, double sx, double sy, double sz) {
    const double dx = (double)p[0] - sx, dy = (double)p[1] - sy, dz = (double)p[2] - sz;
    return __dadd_rn(__dadd_rn(__dmul_rn(dx, dx), __dmul_rn(dy, dy)), __dmul_rn(dz, dz));
}

__device__ unsigned block_exclusive_scan(unsigned v, unsigned* sm32, unsigned& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) sm32[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        unsigned w = lane < (int)(blockDim.x >> 5) ? sm32[lane] : 0u;
        unsigned wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        sm32[lane] = wi - w;
        if (lane == 31) sm32[32] = wi;
    }
    __syncthreads();
    const unsigned out = sm32[warp] + incl - v;
    total = sm32[32];
    __syncthreads();
    return out;
}

__global__ void __launch_bounds__(kPiThreads)
patch_index_kernel(const float* __restrict__ pts, int N, const int32_t* __restrict__ seeds,
                   int k, int kpow2, double beta, int32_t* __restrict__ nbr,
                   double* __restrict__ radial, double* __restrict__ wts) {
    extern __shared__ __align__(16) unsigned char pi_sm[];
    unsigned long long* skey = reinterpret_cast<unsigned long long*>(pi_sm);   // [kpow2]
    int* sidx = reinterpret_cast<int*>(skey + kpow2);                           // [kpow2]
    __shared__ unsigned hist[256];
    __shared__ unsigned scan32[33];
    __shared__ unsigned long long bcast[2];

    const int s = blockIdx.x;
    const int tid = threadIdx.x;
    const int sp = seeds[s];
    const double sx = pts[3 * sp], sy = pts[3 * sp + 1], sz = pts[3 * sp + 2];
    const unsigned lanes_below = (1u << (tid & 31)) - 1u;
    unsigned long long prefix = 0ull, mask = 0ull;
    unsigned need = (unsigned)k;
    for (int pass = 0; pass < 8; ++pass) {
        const int shift = 56 - 8 * pass;
        if (tid < 256) hist[tid] = 0u;
        __syncthreads();
        // the same trip count in every thread, so whole warps vote together
        for (int base = 0; base < N; base += kPiThreads) {
            const int n = base + tid;
            unsigned long long key = 0ull;
            if (n < N) key = (unsigned long long)__double_as_longlong(sqdist64(pts + 3 * n, sx, sy, sz));
            const bool act = n < N && (key & mask) == prefix;
            const unsigned bin = (unsigned)((key >> shift) & 255ull);
            const unsigned am = __ballot_sync(0xffffffffu, act);
            if (act) {
                const unsigned peers = __match_any_sync(am, bin);
                if ((peers & lanes_below) == 0u) atomicAdd(&hist[bin], (unsigned)__popc(peers));
            }
        }
        __syncthreads();
        if (tid < 32) {
            unsigned c[8], sum = 0u;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                c[i] = hist[tid * 8 + i];
                sum += c[i];
            }
            unsigned incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
                if (tid >= o) incl += t;
            }
            const unsigned excl = incl - sum;
            const bool owner = excl < need && need <= incl;
            if (owner) {
                unsigned below = excl, digit = 0u;
                bool found = false;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (!found) {
                        if (below + c[i] >= need) {
                            digit = (unsigned)(tid * 8 + i);
                            found = true;
                        } else {
                            below += c[i];
                        }
                    }
                }
                bcast[0] = digit;
                bcast[1] = below;
            }
        }
        __syncthreads();
        need -= (unsigned)bcast[1];
        prefix |= bcast[0] << shift;
        mask |= 0xffull << shift;
        __syncthreads();
    }
    const unsigned long long T = prefix;
    const unsigned n_less = (unsigned)k - need;

    const int chunk = (N + kPiThreads - 1) / kPiThreads;
    const int lo = min(N, tid * chunk), hi = min(N, lo + chunk);
    unsigned cl = 0u, ce = 0u;
    for (int n = lo; n < hi; ++n) {
        const unsigned long long key =
            (unsigned long long)__double_as_longlong(sqdist64(pts + 3 * n, sx, sy, sz));
        cl += key < T;
        ce += key == T;
    }
    unsigned tot;
    unsigned ol = block_exclusive_scan(cl, scan32, tot);
    unsigned oe = block_exclusive_scan(ce, scan32, tot);
    for (int n = lo; n < hi; ++n) {
        const unsigned long long key =
            (unsigned long long)__double_as_longlong(sqdist64(pts + 3 * n, sx, sy, sz));
        if (key < T) {
            skey[ol] = key;
            sidx[ol] = n;
            ++ol;
        } else if (key == T) {
            if (oe < need) {
                skey[n_less + oe] = key;
                sidx[n_less + oe] = n;
            }
            ++oe;
        }
    }
    for (int i = k + tid; i < kpow2; i += kPiThreads) {
        skey[i] = ~0ull;
        sidx[i] = 0x7fffffff;
    }
    __syncthreads();
    // bitonic sort by (key, index)
    for (int size = 2; size <= kpow2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < kpow2; i += kPiThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    const unsigned long long ki = skey[i], kj = skey[j];
                    const int ii = sidx[i], ij = sidx[j];
                    const bool gt = ki > kj || (ki == kj && ii > ij);
                    if (gt == up) {
                        skey[i] = kj; skey[j] = ki;
                        sidx[i] = ij; sidx[j] = ii;
                    }
                }
            }
            __syncthreads();
        }
    }
    const double dmax = sqrt(__longlong_as_double((long long)skey[k - 1]));
    const double denom = dmax + 1e-8;
    for (int i = tid; i < k; i += kPiThreads) {
        const double d = sqrt(__longlong_as_double((long long)skey[i]));
        const double r = d / denom;
        const size_t o = (size_t)s * k + i;
        nbr[o] = sidx[i];
        radial[o] = r;
        wts[o] = exp(__dmul_rn(__dmul_rn(-beta, r), r));
    }
}

// ---------------------------------------------------------------------------
// Fusion structure: per point, the flat (patch, slot) entries that vote for
// it, in increasing flat order -- the order np.bincount accumulates in
// (inference.py:128-132,160-170) -- and the float64 weight sums.
// ---------------------------------------------------------------------------
__global__ void count_kernel(const int32_t* __restrict__ nbr, int64_t total, int N,
                             int* __restrict__ counts, int* __restrict__ bad) {
    for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < total;
         f += (int64_t)gridDim.x * blockDim.x) {
        const int n = nbr[f];
        if (n < 0 || n >= N) {
            atomicExch(bad, 1);
            continue;
        }
        atomicAdd(&counts[n], 1);
    }
}

__global__ void __launch_bounds__(1024) scan_kernel(const int* __restrict__ counts, int N,
                                                    int32_t* __restrict__ offsets) {
    __shared__ unsigned scan32[33];
    const int tid = threadIdx.x;
    const int chunk = (N + 1023) / 1024;
    const int lo = min(N, tid * chunk), hi = min(N, lo + chunk);
    unsigned s = 0u;
    for (int n = lo; n < hi; ++n) s += (unsigned)counts[n];
    unsigned tot;
    unsigned o = block_exclusive_scan(s, scan32, tot);
    for (int n = lo; n < hi; ++n) {
        offsets[n] = (int32_t)o;
        o += (unsigned)counts[n];
    }
    if (tid == 0) offsets[N] = (int32_t)tot;
}

__global__ void fill_kernel(const int32_t* __restrict__ nbr, int64_t total, int N,
                            const int32_t* __restrict__ offsets, int* __restrict__ cursor,
                            int32_t* __restrict__ entries) {
    for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < total;
         f += (int64_t)gridDim.x * blockDim.x) {
        const int n = nbr[f];
        if (n < 0 || n >= N) continue;
        const int pos = atomicAdd(&cursor[n], 1);
        entries[offsets[n] + pos] = (int32_t)f;
    }
}

__global__ void sort_sum_kernel(const int32_t* __restrict__ offsets, int32_t* __restrict__ entries,
                                const double* __restrict__ wts, int N,
                                double* __restrict__ wsum) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const int a = offsets[n], b = offsets[n + 1];
    for (int i = a + 1; i < b; ++i) {
        const int32_t v = entries[i];
        int j = i - 1;
        while (j >= a && entries[j] > v) {
            entries[j + 1] = entries[j];
            --j;
        }
        entries[j + 1] = v;
    }
    double s = 0.0;
    for (int i = a; i < b; ++i) s = __dadd_rn(s, wts[entries[i]]);
    wsum[n] = s;
}

// x[p, c, m] = points[nbr[p, m], c] - points[seed[p], c] (inference.py:142-150).
__global__ void gather_kernel(const float* __restrict__ pts, const int32_t* __restrict__ nbr,
                              const int32_t* __restrict__ seeds, int P, int k,
                              float* __restrict__ x) {
    const int64_t total = (int64_t)P * k;
    for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < total;
         f += (int64_t)gridDim.x * blockDim.x) {
        const int p = (int)(f / k), m = (int)(f - (int64_t)p * k);
        const int n = nbr[f], s = seeds[p];
        float* xp = x + (size_t)p * 3 * k;
#pragma unroll
        for (int c = 0; c < 3; ++c) xp[(size_t)c * k + m] = __fsub_rn(pts[3 * n + c], pts[3 * s + c]);
    }
}

// Per point: v = sum_f w_f * vote_f / (wsum + 1e-8) in float64, in flat order
// (inference.py:158-171), cast to float32; x' = x - alpha_step * v as two
// separately rounded float32 operations; points no patch covers keep x
// (:193-195).
__global__ void fuse_euler_kernel(const float* __restrict__ pts, const float* __restrict__ votes,
                                  const int32_t* __restrict__ offsets,
                                  const int32_t* __restrict__ entries,
                                  const double* __restrict__ wts, const double* __restrict__ wsum,
                                  int N, float alpha_step, float* __restrict__ out,
                                  float* __restrict__ velocity) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const int a = offsets[n], b = offsets[n + 1];
    double s0 = 0.0, s1 = 0.0, s2 = 0.0;
    for (int i = a; i < b; ++i) {
        const int f = entries[i];
        const double w = wts[f];
        s0 = __dadd_rn(s0, __dmul_rn(w, (double)votes[3 * (size_t)f]));
        s1 = __dadd_rn(s1, __dmul_rn(w, (double)votes[3 * (size_t)f + 1]));
        s2 = __dadd_rn(s2, __dmul_rn(w, (double)votes[3 * (size_t)f + 2]));
    }
    const double den = __dadd_rn(wsum[n], 1e-8);
    const float v[3] = {(float)__ddiv_rn(s0, den), (float)__ddiv_rn(s1, den),
                        (float)__ddiv_rn(s2, den)};
    const bool covered = b > a && wsum[n] != 0.0;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const float x = pts[3 * n + c];
        out[3 * n + c] = covered ? __fsub_rn(x, __fmul_rn(alpha_step, v[c])) : x;
        if (velocity) velocity[3 * n + c] = v[c];
    }
}

// Patch-sharded form of the same fusion, for one cloud whose patches are
// split across GPUs: the weighted vote sums of the entries whose patch lies in
// [patch_begin, patch_end), in entry order, float64 (N, 3). Summed over the
// ranks (an all-reduce) they give the sums fuse_euler_kernel forms; with one
// rank the result is the same sum bit for bit.
__global__ void fuse_partial_kernel(const float* __restrict__ votes,
                                    const int32_t* __restrict__ offsets,
                                    const int32_t* __restrict__ entries,
                                    const double* __restrict__ wts, int N, int k,
                                    int patch_begin, int patch_end, double* __restrict__ vsum) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const int a = offsets[n], b = offsets[n + 1];
    const int f_begin = patch_begin * k, f_end = patch_end * k;
    double s0 = 0.0, s1 = 0.0, s2 = 0.0;
    for (int i = a; i < b; ++i) {
        const int f = entries[i];
        if (f < f_begin || f >= f_end) continue;
        const double w = wts[f];
        s0 = __dadd_rn(s0, __dmul_rn(w, (double)votes[3 * (size_t)f]));
        s1 = __dadd_rn(s1, __dmul_rn(w, (double)votes[3 * (size_t)f + 1]));
        s2 = __dadd_rn(s2, __dmul_rn(w, (double)votes[3 * (size_t)f + 2]));
    }
    vsum[3 * (size_t)n] = s0;
    vsum[3 * (size_t)n + 1] = s1;
    vsum[3 * (size_t)n + 2] = s2;
}

// Normalisation and Euler update from summed votes (the second half of
// fuse_euler_kernel).
__global__ void euler_from_sum_kernel(const float* __restrict__ pts,
                                      const double* __restrict__ vsum,
                                      const double* __restrict__ wsum,
                                      const int32_t* __restrict__ offsets, int N,
                                      float alpha_step, float* __restrict__ out,
                                      float* __restrict__ velocity) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const double den = __dadd_rn(wsum[n], 1e-8);
    const bool covered = offsets[n + 1] > offsets[n] && wsum[n] != 0.0;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const float v = (float)__ddiv_rn(vsum[3 * (size_t)n + c], den);
        const float x = pts[3 * n + c];
        out[3 * n + c] = covered ? __fsub_rn(x, __fmul_rn(alpha_step, v)) : x;
        if (velocity) velocity[3 * n + c] = v;
    }
}

int grid_for(int64_t work, int threads) {
    const int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * 32;
    return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

}  // namespace
}  // namespace f2s

using namespace f2s;

extern "C" int f2s_fps_workspace_bytes(int64_t N, size_t* bytes) {
    F2S_REQUIRE(N >= 0 && bytes, "bad workspace query");
    // the larger of: a running minimum per point (cluster path beyond the
    // grid's shared memory), a 64-bit slot per seed plus the arrival counter
    // (cooperative grid path)
    *bytes = ((size_t)N + 2) * sizeof(unsigned long long);
    return F2S_OK;
}

extern "C" int f2s_fps(const float* points, int64_t N, int64_t count, int64_t first,
                       int32_t* selected, void* workspace, size_t workspace_bytes,
                       void* stream) {
    F2S_REQUIRE(N >= 1, "num_points must be >= 1, got %lld", (long long)N);
    F2S_REQUIRE(count >= 1 && count <= N, "count %lld outside [1, %lld]", (long long)count,
                (long long)N);
    F2S_REQUIRE(first >= 0 && first < N, "first index %lld out of range", (long long)first);
    F2S_LIMIT(N < (1ll << 31) - 1, "too many points: %lld", (long long)N);
    F2S_REQUIRE(points && selected, "fps: null pointer");
    const int n = (int)N;
    int cs = ceil_div(n, 4 * kFpsThreads);
    cs = cs < 1 ? 1 : (cs > kFpsMaxCluster ? kFpsMaxCluster : cs);
    const int slice = ceil_div(n, cs);
    const bool smem = slice <= kFpsSmemPoints;
    const int grid = sm_count();
    const int grid_slice = ceil_div(n, grid > 0 ? grid : 1);
    if (!smem && grid > 0 && grid_slice <= kFpsSmemPoints &&
        (int64_t)count * grid < (1ll << 32)) {
        // cooperative grid, one CTA per SM, every slice in shared memory
        const size_t need = ((size_t)count + 2) * sizeof(unsigned long long);
        F2S_REQUIRE(workspace != nullptr, "fps: a workspace is needed for %d points", n);
        if (workspace_bytes < need)
            return fail(F2S_ERR_WORKSPACE, "fps needs %zu workspace bytes, got %zu", need,
                        workspace_bytes);
        int* err = tc_error_word();
        if (!err) return fail(F2S_ERR_CUDA, "device error word unavailable");
        cudaStream_t st = as_stream(stream);
        auto* slots = static_cast<unsigned long long*>(workspace);
        auto* arrived = reinterpret_cast<unsigned*>(slots + count);
        TraceScope trace(kTagFps, st);
        F2S_CUDA_TRY(cudaMemsetAsync(workspace, 0, need, st));
        const size_t smem_bytes = (size_t)grid_slice * 16;
        F2S_CUDA_TRY(cudaFuncSetAttribute(fps_grid_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem_bytes));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kFpsGridThreads);
        cfg.dynamicSmemBytes = smem_bytes;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        F2S_CUDA_TRY(cudaLaunchKernelEx(&cfg, fps_grid_kernel, points, n, (int)count,
                                        (int)first, grid_slice, slots, arrived, selected, err));
        return check_launch("fps_grid_kernel");
    }
    if (!smem) {
        F2S_REQUIRE(workspace != nullptr, "fps: a workspace is needed for %d points", n);
        if (workspace_bytes < (size_t)N * sizeof(float))
            return fail(F2S_ERR_WORKSPACE, "fps needs %zu workspace bytes, got %zu",
                        (size_t)N * sizeof(float), workspace_bytes);
    }
    TraceScope trace(kTagFps, as_stream(stream));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs);
    cfg.blockDim = dim3(kFpsThreads);
    cfg.dynamicSmemBytes = smem ? (size_t)slice * 16 : 0;
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    float* gmin = static_cast<float*>(workspace);
    if (smem) {
        F2S_CUDA_TRY(cudaFuncSetAttribute(fps_kernel<true>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)cfg.dynamicSmemBytes));
        F2S_CUDA_TRY(cudaLaunchKernelEx(&cfg, fps_kernel<true>, points, n, (int)count, (int)first,
                                        slice, gmin, selected));
    } else {
        F2S_CUDA_TRY(cudaLaunchKernelEx(&cfg, fps_kernel<false>, points, n, (int)count,
                                        (int)first, slice, gmin, selected));
    }
    return check_launch("fps_kernel");
}

extern "C" int f2s_patch_index(const float* points, int64_t N, const int32_t* seeds, int P,
                               int k, double beta, int32_t* neighbors, double* radial,
                               double* weights, void* stream) {
    F2S_REQUIRE(N >= 1 && P >= 0, "patch_index: bad sizes N=%lld P=%d", (long long)N, P);
    F2S_REQUIRE(k >= 1 && k <= N, "patch_size %d outside [1, %lld]", k, (long long)N);
    F2S_LIMIT(k <= F2S_KNN_MAX_POINTS, "patch_size %d exceeds %d", k, F2S_KNN_MAX_POINTS);
    F2S_LIMIT(N < (1ll << 31) - 1, "too many points: %lld", (long long)N);
    if (P == 0) return F2S_OK;
    F2S_REQUIRE(points && seeds && neighbors && radial && weights, "patch_index: null pointer");
    int kpow2 = 1;
    while (kpow2 < k) kpow2 <<= 1;
    const size_t smem = (size_t)kpow2 * (sizeof(unsigned long long) + sizeof(int));
    F2S_CUDA_TRY(cudaFuncSetAttribute(patch_index_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    TraceScope trace(kTagPatchIndex, as_stream(stream));
    patch_index_kernel<<<P, kPiThreads, smem, as_stream(stream)>>>(
        points, (int)N, seeds, k, kpow2, beta, neighbors, radial, weights);
    return check_launch("patch_index_kernel");
}

extern "C" int f2s_fusion_workspace_bytes(int64_t N, size_t* bytes) {
    F2S_REQUIRE(N >= 0 && bytes, "bad workspace query");
    *bytes = ((size_t)N * 2 + 64) * sizeof(int);
    return F2S_OK;
}

extern "C" int f2s_fusion_build(const int32_t* neighbors, const double* weights, int P, int k,
                                int64_t N, int32_t* offsets, int32_t* entries,
                                double* weight_sum, void* workspace, size_t workspace_bytes,
                                void* stream) {
    F2S_REQUIRE(N >= 1 && P >= 0 && k >= 1, "fusion_build: bad sizes");
    F2S_LIMIT((int64_t)P * k < (1ll << 31) - 1 && N < (1ll << 31) - 1,
              "fusion_build: too many entries");
    F2S_REQUIRE(neighbors && weights && offsets && entries && weight_sum && workspace,
                "fusion_build: null pointer");
    const size_t need = ((size_t)N * 2 + 64) * sizeof(int);
    if (workspace_bytes < need)
        return fail(F2S_ERR_WORKSPACE, "fusion_build needs %zu workspace bytes, got %zu", need,
                    workspace_bytes);
    cudaStream_t st = as_stream(stream);
    TraceScope trace(kTagFusionBuild, st);
    int* counts = static_cast<int*>(workspace);
    int* cursor = counts + N;
    int* bad = cursor + N;
    F2S_CUDA_TRY(cudaMemsetAsync(workspace, 0, need, st));
    const int64_t total = (int64_t)P * k;
    count_kernel<<<grid_for(total, 256), 256, 0, st>>>(neighbors, total, (int)N, counts, bad);
    F2S_TRY(check_launch("count_kernel"));
    scan_kernel<<<1, 1024, 0, st>>>(counts, (int)N, offsets);
    F2S_TRY(check_launch("scan_kernel"));
    fill_kernel<<<grid_for(total, 256), 256, 0, st>>>(neighbors, total, (int)N, offsets, cursor,
                                                       entries);
    F2S_TRY(check_launch("fill_kernel"));
    sort_sum_kernel<<<ceil_div((int)N, 256), 256, 0, st>>>(offsets, entries, weights, (int)N,
                                                           weight_sum);
    return check_launch("sort_sum_kernel");
}

extern "C" int f2s_gather_patches(const float* points, const int32_t* neighbors,
                                  const int32_t* seeds, int P, int k, float* x, void* stream) {
    F2S_REQUIRE(P >= 0 && k >= 1, "gather_patches: bad sizes");
    if (P == 0) return F2S_OK;
    F2S_REQUIRE(points && neighbors && seeds && x, "gather_patches: null pointer");
    const int64_t total = (int64_t)P * k;
    TraceScope trace(kTagGather, as_stream(stream));
    gather_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(points, neighbors, seeds,
                                                                         P, k, x);
    return check_launch("gather_kernel");
}

extern "C" int f2s_fuse_euler(const float* points, const float* votes, const int32_t* offsets,
                              const int32_t* entries, const double* weights,
                              const double* weight_sum, int64_t N, float alpha_step, float* out,
                              float* velocity, void* stream) {
    F2S_REQUIRE(N >= 0, "fuse_euler: bad size");
    if (N == 0) return F2S_OK;
    F2S_LIMIT(N < (1ll << 31) - 1, "too many points");
    F2S_REQUIRE(points && votes && offsets && entries && weights && weight_sum && out,
                "fuse_euler: null pointer");
    TraceScope trace(kTagFuseEuler, as_stream(stream));
    fuse_euler_kernel<<<ceil_div((int)N, 256), 256, 0, as_stream(stream)>>>(
        points, votes, offsets, entries, weights, weight_sum, (int)N, alpha_step, out, velocity);
    return check_launch("fuse_euler_kernel");
}

extern "C" int f2s_fuse_partial(const float* votes, const int32_t* offsets,
                                const int32_t* entries, const double* weights, int64_t N, int k,
                                int patch_begin, int patch_end, double* vote_sum, void* stream) {
    F2S_REQUIRE(N >= 0 && k >= 1 && 0 <= patch_begin && patch_begin <= patch_end,
                "fuse_partial: bad size N=%lld k=%d patches [%d, %d)", (long long)N, k,
                patch_begin, patch_end);
    if (N == 0) return F2S_OK;
    F2S_LIMIT(N < (1ll << 31) - 1 && (int64_t)patch_end * k < (1ll << 31) - 1, "too many points");
    F2S_REQUIRE(offsets && entries && weights && vote_sum && (votes || patch_begin == patch_end),
                "fuse_partial: null pointer");
    f2s::TraceScope trace(f2s::kTagFuseEuler, f2s::as_stream(stream));
    f2s::fuse_partial_kernel<<<f2s::ceil_div((int)N, 256), 256, 0, f2s::as_stream(stream)>>>(
        votes, offsets, entries, weights, (int)N, k, patch_begin, patch_end, vote_sum);
    return f2s::check_launch("fuse_partial_kernel");
}

extern "C" int f2s_euler_from_sum(const float* points, const double* vote_sum,
                                  const double* weight_sum, const int32_t* offsets, int64_t N,
                                  float alpha_step, float* out, float* velocity, void* stream) {
    F2S_REQUIRE(N >= 0, "euler_from_sum: bad size");
    if (N == 0) return F2S_OK;
    F2S_LIMIT(N < (1ll << 31) - 1, "too many points");
    F2S_REQUIRE(points && vote_sum && weight_sum && offsets && out,
                "euler_from_sum: null pointer");
    f2s::TraceScope trace(f2s::kTagFuseEuler, f2s::as_stream(stream));
    f2s::euler_from_sum_kernel<<<f2s::ceil_div((int)N, 256), 256, 0, f2s::as_stream(stream)>>>(
        points, vote_sum, weight_sum, offsets, (int)N, alpha_step, out, velocity);
    return f2s::check_launch("euler_from_sum_kernel");
}
