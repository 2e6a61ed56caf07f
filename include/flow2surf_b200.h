/*
 * flow2surf_b200.h -- C-ABI of the B200 (sm_100a) reverse-flow denoising path.
 *
 * Every entry point:
 *   - takes plain device pointers, sizes and a CUDA stream (passed as void*,
 *     a cudaStream_t; NULL means the legacy default stream);
 *   - never allocates device memory: the caller owns every buffer, including
 *     any workspace, whose size a *_workspace_bytes() query reports;
 *   - is stream-ordered: it enqueues kernels and returns without a device sync;
 *   - returns F2S_OK or an f2s_status code and never aborts; the message of
 *     the last failure on the calling host thread is in f2s_last_error().
 *
 * Layouts are row-major, dimensions named as in the reference's Python
 * operators (flow2surf/models/ops/*.py, flow2surf/training/distances.py,
 * flow2surf/inference.py). Each declaration names the reference interface it
 * replaces as path:line inside the reference project.
 */
#ifndef FLOW2SURF_B200_H
#define FLOW2SURF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum f2s_status {
    F2S_OK = 0,
    F2S_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad rank/shape, bad config */
    F2S_ERR_UNSUPPORTED = 2,      /* size beyond a kernel's stated limit      */
    F2S_ERR_CUDA = 3,             /* a CUDA launch or runtime call failed     */
    F2S_ERR_WORKSPACE = 4         /* caller workspace smaller than required   */
} f2s_status;

/* Message of the last failed call on this host thread ("" if none). */
const char* f2s_last_error(void);

/* ABI version: major * 10000 + minor * 100 + patch. */
int f2s_version(void);

/* ------------------------------------------------------------------------ */
/* Operators (flow2surf/models/ops/__init__.py:3-11)                        */
/* ------------------------------------------------------------------------ */

/*
 * k nearest non-self neighbours in feature space.
 * Replaces knn_indices (flow2surf/models/ops/knn.py:55-86) and its kernel
 * global_knn (flow2surf/models/ops/cuda/knn_global.cu:1-57, keys from
 * flow2surf/models/ops/cuda/knn.cuh:7-17).
 *   features : (B, C, N) float32
 *   indices  : (B, N, k) int32, ascending (distance, index); when k > N-1 the
 *              last real neighbour is repeated (knn.py:83-85); N <= 1 gives 0.
 * Distances are the reference kernel's fp32 expression, bit for bit.
 * Limits: 1 <= k <= 32 (F2S_KNN_MAX_K), N <= 2048 (F2S_KNN_MAX_POINTS) and
 * C*N*4 <= F2S_KNN_MAX_FEATURE_BYTES (one patch's features are staged in
 * shared memory). Beyond them the call returns F2S_ERR_UNSUPPORTED.
 */
#define F2S_KNN_MAX_K 32
#define F2S_KNN_MAX_POINTS 2048
#define F2S_KNN_MAX_FEATURE_BYTES (96 * 1024)
int f2s_knn(const float* features, int B, int C, int N, int k,
            int32_t* indices, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLOW2SURF_B200_H */
