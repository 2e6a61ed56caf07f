/*
 * ORACLE -- test infrastructure only. CPU restatement of the reference's
 * integer/index-exact kernels, used by tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py as the checker. Never linked into the product.
 *
 * Build with -ffp-contract=off: every fused multiply-add below is spelled out
 * with fmaf() where the reference's CUDA source contracts one, and no other
 * expression may be contracted.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Order-preserving float -> uint32 map with -0 folded onto +0
 * (flow2surf/models/ops/cuda/knn.cuh:11-16). */
static uint32_t ordered_bits(float d) {
    float canonical = d == 0.0f ? 0.0f : d;
    uint32_t bits;
    memcpy(&bits, &canonical, 4);
    return bits ^ ((bits & 0x80000000u) ? 0xffffffffu : 0x80000000u);
}

/*
 * k nearest non-self neighbours (flow2surf/models/ops/cuda/knn_global.cu:1-53,
 * flow2surf/models/ops/knn.py:55-86).
 *   features (B, C, N) f32 -> indices (B, N, k) int32.
 * Per pair: qn, rn, ip accumulate over channels in order with fmaf
 * (knn_global.cu:22-28 under nvcc's default contraction), then
 * d = (qn + rn) - 2*ip (knn_global.cu:29; 2*ip is exact so one rounding).
 * Selection: the actual_k = min(k, N-1) smallest (ordered_bits(d), j) keys in
 * ascending order (knn_global.cu:35-52); padded by repeating the last index
 * (knn.py:83-85); N <= 1 gives zeros (knn.py:64-65).
 */
void oracle_knn(const float* features, int64_t B, int64_t C, int64_t N, int64_t k,
                int32_t* out) {
    if (N <= 1) {
        memset(out, 0, (size_t)(B * N * k) * sizeof(int32_t));
        return;
    }
    const int64_t actual_k = k < N - 1 ? k : N - 1;
#pragma omp parallel
    {
        float* norm = (float*)malloc((size_t)N * sizeof(float));
        uint64_t* best = (uint64_t*)malloc((size_t)(actual_k + 1) * sizeof(uint64_t));
        int64_t last_b = -1;
#pragma omp for schedule(static)
        for (int64_t bq = 0; bq < B * N; ++bq) {
            const int64_t b = bq / N, q = bq % N;
            const float* f = features + b * C * N;
            if (b != last_b) {
                for (int64_t j = 0; j < N; ++j) {
                    float n = 0.0f;
                    for (int64_t c = 0; c < C; ++c) n = fmaf(f[c * N + j], f[c * N + j], n);
                    norm[j] = n;
                }
                last_b = b;
            }
            int64_t filled = 0;
            for (int64_t j = 0; j < N; ++j) {
                if (j == q) continue;
                float ip = 0.0f;
                for (int64_t c = 0; c < C; ++c) ip = fmaf(f[c * N + q], f[c * N + j], ip);
                const float d = fmaf(-2.0f, ip, norm[q] + norm[j]);
                const uint64_t key = ((uint64_t)ordered_bits(d) << 32) | (uint32_t)j;
                if (filled == actual_k && key >= best[actual_k - 1]) continue;
                int64_t pos = filled < actual_k ? filled++ : actual_k - 1;
                while (pos > 0 && best[pos - 1] > key) {
                    best[pos] = best[pos - 1];
                    --pos;
                }
                best[pos] = key;
            }
            int32_t* o = out + bq * k;
            for (int64_t r = 0; r < k; ++r) {
                const int64_t s = r < actual_k ? r : actual_k - 1;
                o[r] = (int32_t)(best[s] & 0xffffffffu);
            }
        }
        free(norm);
        free(best);
    }
}

/*
 * Squared distance of the reference's nearest-distance kernel,
 * `dx * dx + dy * dy + dz * dz` (flow2surf/training/cuda/nearest_distance_forward.cu:29).
 * mode 0: nvcc's contraction fmaf(dz, dz, fmaf(dx, dx, dy*dy));
 * mode 1: fmaf(dz, dz, fmaf(dy, dy, dx*dx)); mode 2: no contraction.
 */
static float nearest_sq(float dx, float dy, float dz, int mode) {
    if (mode == 0) return fmaf(dz, dz, fmaf(dx, dx, dy * dy));
    if (mode == 1) return fmaf(dz, dz, fmaf(dy, dy, dx * dx));
    return (dx * dx + dy * dy) + dz * dz;
}

/*
 * Bidirectional nearest squared distances (nearest_distance_forward.cu:1-93):
 * for each point of `query` (B, M, 3) the smallest distance to `points`
 * (B, N, 3) and its index, scanning j in order with strict `<` so ties keep
 * the lower index (:31-36); best starts at FLT_MAX with index N (:10-11).
 */
void oracle_nearest_one_way(const float* query, const float* points, int64_t B, int64_t M,
                            int64_t N, int mode, float* dist, int32_t* index) {
#pragma omp parallel for schedule(static)
    for (int64_t bi = 0; bi < B * M; ++bi) {
        const int64_t b = bi / M;
        const float* p = query + bi * 3;
        const float* r = points + b * N * 3;
        float best = 3.402823466e+38f;
        int64_t best_index = N;
        for (int64_t j = 0; j < N; ++j) {
            const float dx = p[0] - r[j * 3 + 0];
            const float dy = p[1] - r[j * 3 + 1];
            const float dz = p[2] - r[j * 3 + 2];
            const float d = nearest_sq(dx, dy, dz, mode);
            if (d < best || (d == best && j < best_index)) {
                best = d;
                best_index = j;
            }
        }
        dist[bi] = best;
        index[bi] = (int32_t)best_index;
    }
}

/*
 * Farthest-point sampling (flow2surf/inference.py:19-41). Every operation is a
 * separately rounded float32 NumPy ufunc: d = ((x-cx)^2 + (y-cy)^2) + (z-cz)^2
 * (:30-37); the running minimum is float64 in the reference (:24) but only
 * ever holds float32 values (or +inf), so float32 storage is exact; argmax
 * returns the first maximum (:39).
 */
void oracle_fps(const float* points, int64_t N, int64_t count, int64_t first,
                int64_t* selected) {
    float* mind = (float*)malloc((size_t)N * sizeof(float));
    for (int64_t n = 0; n < N; ++n) mind[n] = INFINITY;
    selected[0] = first;
    for (int64_t i = 1; i < count; ++i) {
        const float* c = points + selected[i - 1] * 3;
        int64_t best = 0;
        float best_value = -INFINITY;
        for (int64_t n = 0; n < N; ++n) {
            const float* p = points + n * 3;
            float d = p[0] - c[0];
            d = d * d;
            float w = p[1] - c[1];
            w = w * w;
            d = d + w;
            w = p[2] - c[2];
            w = w * w;
            d = d + w;
            if (d < mind[n]) mind[n] = d;
            if (mind[n] > best_value) {
                best_value = mind[n];
                best = n;
            }
        }
        selected[i] = best;
    }
    free(mind);
}
