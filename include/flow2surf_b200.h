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

/*
 * Per-launch device timing (no counterpart in the reference, which has no
 * profiling hooks). While enabled, every kernel launch of this library is
 * bracketed by CUDA events on its stream; f2s_trace_collect waits for them,
 * returns per-kernel-class totals (arrays of f2s_trace_tag_count() entries,
 * milliseconds and launch counts) and clears the records.
 * f2s_trace_enable(0|1) also clears them.
 */
int f2s_trace_enable(int on);
int f2s_trace_tag_count(void);
const char* f2s_trace_tag_name(int tag);
int f2s_trace_collect(double* total_ms, int64_t* launches);

/* ------------------------------------------------------------------------ */
/* Operators (flow2surf/models/ops/__init__.py:3-11)                        */
/* ------------------------------------------------------------------------ */

/*
 * k nearest non-self neighbours in feature space.
 * Replaces knn_indices (flow2surf/models/ops/knn.py:35-66) and its kernel
 * global_knn (flow2surf/models/ops/cuda/knn_global.cu:1-57, keys from
 * flow2surf/models/ops/cuda/knn.cuh:7-17).
 *   features : (B, C, N) float32
 *   indices  : (B, N, k) int32, ascending (distance, index); when k > N-1 the
 *              last real neighbour is repeated (knn.py:63-65); N <= 1 gives 0.
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

/*
 * Offset-attention aggregate: column softmax over queries, then row
 * normalisation over keys, then the value product, without ever storing the
 * N x N matrix.
 * Replaces offset_attention_aggregate (flow2surf/models/ops/attention.py:84-106;
 * semantics of _aggregate_jittor, attention.py:15-19).
 *   query (B, N, d), key (B, d, N), value (B, N, C) float32 -> out (B, N, C)
 *   workspace: f2s_offset_attention_workspace_bytes() bytes (key transposed
 *   point-major and one log-sum-exp per key).
 * Limits: d <= 128, C <= 256.
 */
int f2s_offset_attention_workspace_bytes(int B, int N, int d, size_t* bytes);
int f2s_offset_attention(const float* query, const float* key, const float* value,
                         int B, int N, int d, int C, float* out,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * f2s_offset_attention on tcgen05 tensor cores: S = q k^T as split-bf16 MMAs,
 * the column softmax in two passes (per-key log-sum-exp, then P = exp(S - L)
 * per key tile with P V as fp16 MMAs from tensor memory); the N x N scores
 * never reach global memory. d a multiple of 4 up to 64, C a multiple of 64 up
 * to 256, else F2S_ERR_UNSUPPORTED. Results within ~1e-3 relative of the fp32
 * entry (fp16 P and V).
 *   workspace: f2s_offset_attention_tc_workspace_bytes(B, N, d, C) bytes.
 */
int f2s_offset_attention_tc_workspace_bytes(int B, int N, int d, int C, size_t* bytes);
int f2s_offset_attention_tc(const float* query, const float* key, const float* value, int B,
                            int N, int d, int C, float* out, void* workspace,
                            size_t workspace_bytes, void* stream);

/*
 * Normalised neighbour-message reduction with HPE geometry, fused into one
 * kernel (hidden and per-edge contributions never reach HBM).
 * Replaces reduce_neighbor_messages (flow2surf/models/ops/neighbor_reduce.py:244-337)
 * with its no-grad CUDA branch hpe_hidden (hpe.py:35-43, hpe_hidden_forward.cu),
 * project_hpe_output (hpe.py:46-50) and neighbor_reduce (neighbor_reduce_forward.cu).
 *   content (B, 2C, N), geometry (B, N, K, D), indices (B, N, K) int32,
 *   hpe_input_weight (H, D), hpe_input_bias (H), hpe_output_weight (C, H),
 *   hpe_output_bias (C), hpe_norm_weight/bias (H), message_norm_weight/bias (C)
 *   -> out (B, C, N).
 *   workspace: f2s_neighbor_reduce_workspace_bytes() bytes.
 * Limits: K <= 64, D <= 8, H <= 256, C <= 256.
 */
int f2s_neighbor_reduce_workspace_bytes(int B, int N, int C, size_t* bytes);
int f2s_neighbor_reduce(const float* content, const float* geometry, const int32_t* indices,
                        const float* hpe_input_weight, const float* hpe_input_bias,
                        const float* hpe_output_weight, const float* hpe_output_bias,
                        const float* hpe_norm_weight, const float* hpe_norm_bias,
                        const float* message_norm_weight, const float* message_norm_bias,
                        int B, int N, int K, int D, int H, int C, float* out,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * f2s_neighbor_reduce on tcgen05 tensor cores: the HPE output projection as
 * split-bf16 MMAs (hi*hi + hi*lo + lo*hi, close to fp32), the hidden rows and
 * the message reduce fused around it in one kernel. Same arguments, workspace
 * and layouts; D = 6, H in {64, 128}, C in {64, 128, 192}, K in {8, 16, 32},
 * F2S_ERR_UNSUPPORTED otherwise (nothing is launched then).
 */
int f2s_neighbor_reduce_tc(const float* content, const float* geometry, const int32_t* indices,
                           const float* hpe_input_weight, const float* hpe_input_bias,
                           const float* hpe_output_weight, const float* hpe_output_bias,
                           const float* hpe_norm_weight, const float* hpe_norm_bias,
                           const float* message_norm_weight, const float* message_norm_bias,
                           int B, int N, int K, int D, int H, int C, float* out, void* workspace,
                           size_t workspace_bytes, void* stream);

/*
 * Point-wise linear map y = x W^T + b over rows of points: the 1x1
 * Conv1d / Linear of the reference's modules (e.g. transformer.py:37-48 via
 * Jittor's conv/linear) with point-major activations.
 *   x (rows, ldx >= K), weight (cols, K), bias (cols) or NULL -> y (rows, ldy) fp32.
 *   precision F2S_PRECISION_FP32: fp32 CUDA-core kernel;
 *   F2S_PRECISION_TF32: tcgen05 tensor cores reading fp32 x/weight as tf32;
 *   F2S_PRECISION_BF16: tcgen05 tensor cores, x and weight are bf16;
 *   F2S_PRECISION_BF16X3: x is fp32, split into bf16 high and low parts in
 *   shared memory by the kernel; weight points at the bf16 high parts of W
 *   (cols, K) followed by its bf16 low parts (cols, K); y = hi*hi + hi*lo +
 *   lo*hi on tensor cores (about 1e-5 relative to sum |x||w|).
 * Rows (ldx, ldy) must be 16-byte pitched for the tensor-core precisions.
 */
#define F2S_PRECISION_FP32 0
#define F2S_PRECISION_TF32 1
#define F2S_PRECISION_BF16 2
/* Operands split as x = hi + lo (both bf16) and contracted as
 * hi*hi + hi*lo + lo*hi on tensor cores: close to fp32 accuracy. The model's
 * encoder_precision (edge contraction, content and head GEMMs) and
 * f2s_linear. */
#define F2S_PRECISION_BF16X3 3
/* Trunk only: tf32 tensor cores as F2S_PRECISION_TF32, but the FFN input and
 * hidden rows stay fp32 (F2S_PRECISION_TF32 stores them as fp16, which
 * carries tf32's 10-bit mantissa in half the bytes but only fp16's range).
 * The denoise entry points rerun a denoise in this mode when the fp16 rows
 * overflowed (device error word 2). */
#define F2S_PRECISION_TF32_WIDE 4
int f2s_linear(const void* x, int ldx, const void* weight, const float* bias, float* y, int ldy,
               int rows, int cols, int K, int precision, void* stream);

/*
 * The library's device error word: 1 when a tensor-core kernel gave up on a
 * bounded wait (it then returned without finishing its tile), 2 when an fp16
 * intermediate of the tf32 trunk (the FFN hidden rows, which keep tf32's
 * 10-bit mantissa in half the bytes) was out of the fp16 range; 0 otherwise.
 * Copies it to *value (synchronising `stream`) and clears it when `reset` is
 * non-zero. The Python denoise entry points check it after every denoise.
 */
int f2s_device_error(int* value, int reset, void* stream);

/*
 * Self-test of the failure path above (no counterpart in the reference): one
 * thread waits on an mbarrier that nothing arrives on, bounded by `polls`
 * (1 .. 2^20; each poll parks the thread for at most ~1 us), gives up and
 * sets the device error word to 1, as a tensor-core kernel does when a wait
 * runs out. Nothing faults or hangs; the context stays usable.
 */
int f2s_selftest_wait_timeout(int polls, void* stream);

/* ------------------------------------------------------------------------ */
/* Model (flow2surf/models/network.py:29-95)                                */
/* ------------------------------------------------------------------------ */

#define F2S_MAX_STAGES 6
#define F2S_MAX_BLOCKS 16
#define F2S_MAX_DECODER 4

/* The architecture keys of build_model(cfg) (network.py:85-95). */
typedef struct f2s_model_config {
    int32_t k_neighbors;                     /* cfg["k_neighbors"]             */
    int32_t feat_dim;                        /* cfg["feat_dim"]                */
    int32_t num_blocks;                      /* cfg["num_blocks"]              */
    int32_t alpha_dim;                       /* cfg["alpha_dim"]               */
    int32_t ffn_ratio;                       /* cfg["ffn_ratio"]               */
    int32_t num_stages;                      /* len(encoder_dims) + 1          */
    int32_t stage_dims[F2S_MAX_STAGES];      /* encoder_dims + [feat_dim]      */
    int32_t num_decoder;                     /* len(decoder_dims)              */
    int32_t decoder_dims[F2S_MAX_DECODER];   /* cfg["decoder_dims"]            */
    int32_t precision;                       /* trunk and decoder contractions:
                                                F2S_PRECISION_FP32 (CUDA cores),
                                                F2S_PRECISION_TF32 or _TF32_WIDE
                                                (tcgen05)                      */
    int32_t encoder_precision;               /* neighbour stages and projection
                                                head: the choices above or
                                                F2S_PRECISION_BF16X3 (edge
                                                contraction on split-bf16
                                                tensor cores, the rest fp32) */
} f2s_model_config;

/*
 * Layout of the packed parameter blob (float32). On success returns the
 * number of segments (always > F2S_ERR_WORKSPACE, a valid config has at least
 * 20) and, when the arrays are given, each segment's float offset and element
 * count; *total_floats gets the blob size. On failure returns an f2s_status. Segment order (composed exactly as encoder.py:88-101 composes
 * them):
 *   alpha_emb.mlp.0.{weight,bias}, alpha_emb.mlp.2.{weight,bias},
 *   input_embed.net.{0.weight, 0.bias, 1.weight, 1.bias, 3.weight, 3.bias},
 *   per stage: [Wd; Wc - Wd] (2C_out x C_in), position_embed.net.0.{weight,bias},
 *     position_embed.net.1.{weight,bias}, P W_out (C_out x H), P b_out,
 *     norm.{weight,bias}   (P = projection.weight[:, 2 C_in:], W_out/b_out =
 *     position_embed.net.3)
 *   proj.0.weight, proj.1.{weight,bias},
 *   per block: mod.1.{weight,bias}, qkv_conv.weight, proj.weight,
 *     ff_gate.{weight,bias}, ff1.{weight,bias}, ff2.{weight,bias},
 *   per decoder layer: net.{3i}.weight, net.{3i+1}.{weight,bias}; output weight.
 */
int f2s_model_param_segments(const f2s_model_config* cfg, int64_t* offsets, int64_t* sizes,
                             int capacity, int64_t* total_floats);

/* Workspace bytes f2s_model_forward needs for B patches of M points. */
int f2s_model_workspace_bytes(const f2s_model_config* cfg, int B, int M, size_t* bytes);

/*
 * Flow2SurfNet forward: x (B, 3, M) float32 patch coordinates, alpha (B)
 * float32 -> velocity (B, M, 3) float32.
 * Replaces Flow2SurfNet.execute (network.py:75-82) under jt.no_grad().
 * Limits: M <= F2S_KNN_MAX_POINTS, stage widths and feat_dim <= 256.
 */
int f2s_model_forward(const f2s_model_config* cfg, const float* params, const float* x,
                      const float* alpha, int B, int M, float* velocity,
                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * The transformer trunk alone: AlphaEmbed and the num_blocks AdaLN-Zero
 * blocks (offset attention + SwiGLU FFN) of the model above
 * (flow2surf/models/network.py:75-80, transformer.py:75-89), in place on the
 * residual stream; the cfg->precision arithmetic (fp32 CUDA cores or tf32
 * tensor cores). For the trunk micro-benchmark and for callers that run the
 * encoder elsewhere.
 *   params : the same blob as f2s_model_forward (only the alpha embedding and
 *            block segments are read)
 *   x      : (B, M, feat_dim) float32 POINT-MAJOR (the reference's (B, C, M)
 *            transposed), 16-byte aligned; updated in place
 *   alpha  : (B,) float32
 *   workspace: f2s_model_workspace_bytes(cfg, B, M) bytes.
 */
int f2s_trunk_forward(const f2s_model_config* cfg, const float* params, float* x,
                      const float* alpha, int B, int M, void* workspace, size_t workspace_bytes,
                      void* stream);

/* ------------------------------------------------------------------------ */
/* Patch-wise reverse flow (flow2surf/inference.py:19-198)                  */
/* ------------------------------------------------------------------------ */

/*
 * Farthest-point sampling, bit-exact to _farthest_point_indices
 * (inference.py:19-41) given its first index (the reference's
 * rng.integers(N), drawn by the caller).
 *   points (N, 3) float32 -> selected (count,) int32.
 *   workspace: f2s_fps_workspace_bytes() bytes (used only when an 8-CTA
 *   cluster's shared memory cannot hold the cloud, N > 114,688).
 * Up to 114,688 points one thread-block cluster runs the loop; up to one
 * CTA per SM x 14,336 points (2.1 M on a B200) a cooperative grid with one
 * bounded grid-wide wait per seed (a wait that runs out sets the device
 * error word, f2s_device_error, to 1 and the selection is not valid);
 * beyond that the cluster keeps the running minima in the workspace.
 */
int f2s_fps_workspace_bytes(int64_t N, size_t* bytes);
int f2s_fps(const float* points, int64_t N, int64_t count, int64_t first, int32_t* selected,
            void* workspace, size_t workspace_bytes, void* stream);

/*
 * Patch index and vote weights (build_patch_index + build_aggregation,
 * inference.py:110-134): for each seed the k = patch_size nearest points by
 * float64 squared distance, ascending (ties by index);
 * radial = d / (d_max + 1e-8); weights = exp(-beta * radial^2).
 *   seeds (P,) int32 -> neighbors (P, k) int32, radial (P, k) float64,
 *   weights (P, k) float64.   Limit: k <= F2S_KNN_MAX_POINTS.
 */
int f2s_patch_index(const float* points, int64_t N, const int32_t* seeds, int P, int k,
                    double beta, int32_t* neighbors, double* radial, double* weights,
                    void* stream);

/*
 * Fusion structure (the grouping np.bincount performs, inference.py:128-132):
 * offsets (N + 1,) int32, entries (P * k,) int32 -- for every point, the flat
 * (patch * k + slot) positions voting for it in increasing order -- and
 * weight_sum (N,) float64 summed in that order.
 *   workspace: f2s_fusion_workspace_bytes() bytes.
 */
int f2s_fusion_workspace_bytes(int64_t N, size_t* bytes);
int f2s_fusion_build(const int32_t* neighbors, const double* weights, int P, int k, int64_t N,
                     int32_t* offsets, int32_t* entries, double* weight_sum,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * Model input of every patch (inference.py:142-150):
 * x[p, c, m] = points[neighbors[p, m], c] - points[seeds[p], c], x (P, 3, k).
 */
int f2s_gather_patches(const float* points, const int32_t* neighbors, const int32_t* seeds,
                       int P, int k, float* x, void* stream);

/*
 * Centre-weighted fusion of the patch votes (P * k, 3) and the Euler update
 * (aggregate_votes + update, inference.py:158-171,193-195):
 * v = (float)(sum_f w_f vote_f / (weight_sum + 1e-8)) in float64 in entry
 * order; out = points - alpha_step * v (float32, two roundings); points with
 * weight_sum == 0 are copied. `velocity` (N, 3) may be NULL.
 */
int f2s_fuse_euler(const float* points, const float* votes, const int32_t* offsets,
                   const int32_t* entries, const double* weights, const double* weight_sum,
                   int64_t N, float alpha_step, float* out, float* velocity, void* stream);

/*
 * Patch-sharded fusion, for one cloud whose patches are split across GPUs
 * (no counterpart in the reference, which runs one process; it splits the
 * bincount sum of aggregate_votes, inference.py:158-171, by patch):
 * vote_sum (N, 3) float64 = sum, in entry order, of w_f * vote_f over the
 * entries f whose patch p = f / k lies in [patch_begin, patch_end). Only those
 * patches' votes are read. Summing the ranks' vote_sum (an all-reduce) and
 * calling f2s_euler_from_sum gives f2s_fuse_euler's result; with a single
 * range [0, P) it is bit-identical.
 */
int f2s_fuse_partial(const float* votes, const int32_t* offsets, const int32_t* entries,
                     const double* weights, int64_t N, int k, int patch_begin, int patch_end,
                     double* vote_sum, void* stream);

/*
 * Second half of f2s_fuse_euler from summed votes: v = (float)(vote_sum /
 * (weight_sum + 1e-8)), out = points - alpha_step * v; uncovered points are
 * copied. `velocity` (N, 3) may be NULL.
 */
int f2s_euler_from_sum(const float* points, const double* vote_sum, const double* weight_sum,
                       const int32_t* offsets, int64_t N, float alpha_step, float* out,
                       float* velocity, void* stream);

/* ------------------------------------------------------------------------ */
/* Nearest distances and Chamfer                                            */
/* ------------------------------------------------------------------------ */

/*
 * Bidirectional nearest squared distances, bit-exact to the reference kernels
 * nearest_first / nearest_second (flow2surf/training/cuda/nearest_distance_forward.cu:1-93)
 * behind nearest_squared_distances (flow2surf/training/distances.py:70-87).
 *   first (B, M, 3), second (B, N, 3) float32 ->
 *   first_distance (B, M), second_index (B, M) int32,
 *   second_distance (B, N), first_index (B, N) int32.
 *   When both sets hold 4096 points or more, each is sorted into a uniform
 *   grid over its bounding box and a query searches rings of cells around
 *   its own until no unvisited point can beat or tie its best; the results
 *   are the all-pairs scan's, bit for bit (the lexicographic minimum of
 *   (distance, index); points with a non-finite coordinate are never
 *   nearest).
 *   workspace: f2s_nearest_workspace_bytes() bytes (a 64-bit key per point,
 *   and for the grid search about 52 bytes more per point).
 */
int f2s_nearest_workspace_bytes(int B, int M, int N, size_t* bytes);
int f2s_nearest(const float* first, const float* second, int B, int M, int N,
                float* first_distance, int32_t* second_index, float* second_distance,
                int32_t* first_index, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Chamfer distance per batch item: mean of the float32 nearest squared
 * distances pred -> target plus target -> pred, accumulated in float64
 * (chamfer_distance, flow2surf/evaluation.py:24-28, with the kernel's
 * distances). pred (B, M, 3), target (B, N, 3) -> chamfer (B,) float64.
 *   workspace: f2s_nearest_workspace_bytes(B, M, N) bytes.
 */
int f2s_chamfer(const float* pred, const float* target, int B, int M, int N, double* chamfer,
                void* workspace, size_t workspace_bytes, void* stream);

/*
 * Point-to-surface distance: for each point, the squared distance to the
 * closest point of a triangle mesh and that triangle's index (the smaller
 * index on ties), in float32. Replaces point_cloud_utils'
 * closest_points_on_mesh as flow2surf/evaluation.py:31-34 (point_to_surface =
 * the mean of these squared distances) uses it; the closest point on each
 * triangle by the region tests of Ericson, Real-Time Collision Detection
 * (2005), sec. 5.1.5.
 *   points (M, 3) float32, vertices (V, 3) float32, faces (F, 3) int32 with
 *   every index in [0, V) (the caller checks; out-of-range indices are clamped
 *   so nothing is read out of bounds) -> sq_distance (M,) float32,
 *   face_index (M,) int32.
 *   workspace: f2s_point_to_mesh_workspace_bytes(M, F) bytes.
 */
int f2s_point_to_mesh_workspace_bytes(int M, int F, size_t* bytes);
int f2s_point_to_mesh(const float* points, int M, const float* vertices, int V,
                      const int32_t* faces, int F, float* sq_distance, int32_t* face_index,
                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * f2s_chamfer for callers that cannot allocate device memory. No counterpart
 * in the reference: it exists for code that must not call cudaMalloc -- an
 * out-of-memory handler, a host that forbids device allocation once running,
 * or work that must not risk the device synchronisation cudaMalloc/cudaFree
 * can cause. Same inputs, outputs and results as f2s_chamfer, but the
 * distance keys live in a built-in device array of
 * F2S_CHAMFER_STATIC_MAX_POINTS 64-bit entries (16 MiB, held by every GPU
 * that loads this library until the process exits) instead of a workspace.
 *   Requires B * (M + N) <= F2S_CHAMFER_STATIC_MAX_POINTS, else
 *   F2S_ERR_UNSUPPORTED. Allocates nothing.
 *   The first call on each device (with that device current) looks up the
 *   array's device address; under CUDA's lazy module loading (the default)
 *   that first call is also what loads the library's module on the device,
 *   which reserves the array, and it loads the entry's kernels. So make one
 *   call per device before the phase in which nothing may be allocated, and
 *   before any stream capture: a call with B = 0 (any non-null pointers,
 *   M, N >= 1) does only this set-up.
 *   All calls share the one array: calls that overlap on the GPU (other
 *   streams, other host threads) race and must be serialised by the caller.
 */
#define F2S_CHAMFER_STATIC_MAX_POINTS (1 << 21)
int f2s_chamfer_static(const float* pred, const float* target, int B, int M, int N,
                       double* chamfer, void* stream);

/* ------------------------------------------------------------------------ */
/* Training gradients and losses                                            */
/* ------------------------------------------------------------------------ */

/*
 * Coordinate gradients of the nearest squared distances: the backward of
 * f2s_nearest (flow2surf/training/cuda/nearest_distance_backward.cu:11-40,
 * _NearestDistanceFunction.grad, training/distances.py:40-62).
 * second_index (B, M) / first_index (B, N) are f2s_nearest's index outputs;
 * grad_first_distance (B, M) / grad_second_distance (B, N) may be NULL (zero).
 * grad_first (B, M, 3), grad_second (B, N, 3) are written (the matched
 * points' terms added with float atomics, as in the reference).
 */
int f2s_nearest_backward(const float* first, const float* second, int B, int M, int N,
                         const int32_t* second_index, const int32_t* first_index,
                         const float* grad_first_distance, const float* grad_second_distance,
                         float* grad_first, float* grad_second, void* stream);

/*
 * Density-aware Chamfer loss per batch item (dcd_loss, training/losses.py:8-41):
 * loss (B,) float32 (float64 sums). With grad_pred / grad_target (both or
 * neither), also the gradients of sum_b grad_loss[b] loss[b] (grad_loss NULL
 * = ones) with respect to pred (B, M, 3) and target (B, N, 3); the
 * reciprocal multiplicities are constants, as under the reference's autograd.
 *   workspace: f2s_dcd_loss_workspace_bytes(B, M, N) bytes.
 */
int f2s_dcd_loss_workspace_bytes(int B, int M, int N, size_t* bytes);
int f2s_dcd_loss(const float* pred, const float* target, int B, int M, int N, float alpha,
                 float* loss, const float* grad_loss, float* grad_pred, float* grad_target,
                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * Velocity loss per batch item (velocity_loss, training/losses.py:44-47):
 * mean over M of the squared L2 error of (B, M, 3) velocities; loss,
 * grad_pred and grad_target may each be NULL (grad_loss NULL = ones).
 */
int f2s_velocity_loss(const float* pred, const float* target, int B, int M, float* loss,
                      const float* grad_loss, float* grad_pred, float* grad_target,
                      void* stream);

/*
 * Backward of the HPE activation, moment LayerNorm (eps 1e-5) + exact GELU
 * (hpe_activation_grad, flow2surf/models/ops/hpe.py:82-96 and
 * cuda/hpe_activation_backward.cu:10-66): preactivation and grad_hidden
 * (rows, H), H <= 256 -> grad_preactivation (rows, H) (may be grad_hidden
 * itself), grad_norm_weight (H), grad_norm_bias (H) (summed in a fixed order).
 */
int f2s_hpe_activation_backward_workspace_bytes(int64_t rows, int H, size_t* bytes);
int f2s_hpe_activation_backward(const float* preactivation, int64_t rows, int H,
                                const float* norm_weight, const float* norm_bias,
                                const float* grad_hidden, float* grad_preactivation,
                                float* grad_norm_weight, float* grad_norm_bias, void* workspace,
                                size_t workspace_bytes, void* stream);

/*
 * Backward of the normalised message max-reduction
 * (_reduce_messages_grad, flow2surf/models/ops/neighbor_reduce.py:57-72 and
 * cuda/neighbor_reduce_backward.cu:20-84): content (B, 2C, N), contribution
 * (B, N, K, C), indices (B, N, K) int32, the message norm weight / bias (C),
 * grad_output (B, C, N) -> grad_content (B, 2C, N), grad_contribution
 * (B, N, K, C), grad_norm_weight / grad_norm_bias (C). The upstream gradient
 * of a (point, channel) goes to every edge whose recomputed activation
 * equals the maximum over the point's edges (all exact ties). C <= 256.
 */
int f2s_neighbor_messages_backward_workspace_bytes(int B, int N, int C, size_t* bytes);
int f2s_neighbor_messages_backward(const float* content, const float* contribution,
                                   const int32_t* indices, int B, int N, int K, int C,
                                   const float* norm_weight, const float* norm_bias,
                                   const float* grad_output, float* grad_content,
                                   float* grad_contribution, float* grad_norm_weight,
                                   float* grad_norm_bias, void* workspace, size_t workspace_bytes,
                                   void* stream);

/*
 * The whole backward of reduce_neighbor_messages
 * (_NeighborMessageFunction.grad, neighbor_reduce.py:155-237): the HPE rows
 * and the contribution recomputed, the message backward, then through the
 * output projection, the HPE activation and the input projection. Same
 * operand layouts as f2s_neighbor_reduce; every gradient output is written.
 * D <= 8, H <= 256, C <= 256.
 */
int f2s_neighbor_reduce_backward_workspace_bytes(int B, int N, int K, int D, int H, int C,
                                                 size_t* bytes);
int f2s_neighbor_reduce_backward(
    const float* content, const float* geometry, const int32_t* indices,
    const float* hpe_input_weight, const float* hpe_input_bias, const float* hpe_output_weight,
    const float* hpe_output_bias, const float* hpe_norm_weight, const float* hpe_norm_bias,
    const float* message_norm_weight, const float* message_norm_bias, int B, int N, int K, int D,
    int H, int C, const float* grad_output, float* grad_content, float* grad_geometry,
    float* grad_hpe_input_weight, float* grad_hpe_input_bias, float* grad_hpe_output_weight,
    float* grad_hpe_output_bias, float* grad_hpe_norm_weight, float* grad_hpe_norm_bias,
    float* grad_message_norm_weight, float* grad_message_norm_bias, void* workspace,
    size_t workspace_bytes, void* stream);

/*
 * Backward of offset_attention_aggregate (_aggregate_cuda_grad,
 * flow2surf/models/ops/attention.py:46-63 and cuda/offset_attention_backward.cu):
 * query (B, N, d), key (B, d, N), value (B, N, C), the forward's output
 * (B, N, C) and grad_output (B, N, C) -> grad_query, grad_key, grad_value
 * (same shapes as the inputs), fp32. The N x N probabilities of up to 8
 * batch items at a time are held in the workspace.
 */
int f2s_offset_attention_backward_workspace_bytes(int B, int N, int d, int C, size_t* bytes);
int f2s_offset_attention_backward(const float* query, const float* key, const float* value,
                                  int B, int N, int d, int C, const float* output,
                                  const float* grad_output, float* grad_query, float* grad_key,
                                  float* grad_value, void* workspace, size_t workspace_bytes,
                                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLOW2SURF_B200_H */
