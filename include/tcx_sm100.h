/*
 * tcx_sm100.h — C ABI of the B200 (sm_100a) CUDA backend for tensor.cx.
 *
 * This is the drop-in boundary under tensor.cx's backend execution ABI
 * (`Backend::execute(const BackendExecution&)`, cpp/tensorcx/core/backend.h:67-73).
 * Each entry point replaces one `launch_*` function of the reference CUDA backend
 * (cpp/tensorcx/backends/cuda/cuda_kernels.h, cuda_math.h) or one composite that the
 * reference runs as several backend calls (cpp/tensorcx/core/inference.cpp). The
 * citation above each declaration names the interface it replaces.
 *
 * Conventions
 *  - Plain device pointers and sizes; no C++ or torch types. Element counts and
 *    extents are int64_t, like tensorcx::Dim (cpp/tensorcx/core/shape.h:8).
 *  - Every call is stream-ordered on `stream` (a cudaStream_t; NULL is the legacy
 *    default stream) and returns once the work is enqueued. The reference launches
 *    finish with cudaDeviceSynchronize (cuda_profiling.h:66-77); the host backend
 *    keeps that synchronous contract by synchronizing its own stream instead.
 *  - Calls never allocate device memory. Where a kernel needs scratch, the caller
 *    passes `workspace` of at least the size the matching *_workspace_bytes query
 *    returns (the host backend takes it from its stream-ordered pool).
 *  - Metadata arrays (shapes, strides) are HOST pointers read during the call; they
 *    travel to the GPU as kernel parameters. The reference instead allocated and
 *    copied them with cudaMalloc + cudaMemcpy on every call (cuda_backend.cpp:590-599).
 *  - Return value: TCX_OK, or a status mirroring tensorcx::StatusCode
 *    (cpp/tensorcx/core/status.h:8-13). TCX_INVALID_ARGUMENT is raised before any
 *    work is enqueued, so outputs are untouched, as the reference requires of failed
 *    execution (cuda_backend.cpp:612-613). The message of the last failure on the
 *    calling thread is returned by tcx_sm100_last_error().
 */
#ifndef TCX_SM100_H_
#define TCX_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* tcx_stream_t;

/* tensorcx::StatusCode */
enum { TCX_OK = 0, TCX_INVALID_ARGUMENT = 1, TCX_UNAVAILABLE = 2, TCX_INTERNAL = 3 };

/* tensorcx::DType (cpp/tensorcx/core/dtype.h:8-12); bool (one byte, 0 or 1) only in
 * the tensor operations at the end of this header. */
enum { TCX_FLOAT32 = 0, TCX_INT32 = 1, TCX_BOOL = 2 };

/* tensorcx::OpKind values (cpp/tensorcx/core/operation.h:12-63) for the ops on this
 * path, so a host backend can pass OpDesc::kind through unchanged. */
enum {
  TCX_OP_ADD = 1, TCX_OP_MULTIPLY = 2, TCX_OP_MATMUL = 3, TCX_OP_SUM = 4, TCX_OP_MAX = 5,
  TCX_OP_MEAN = 6, TCX_OP_EXP = 7, TCX_OP_GELU = 8, TCX_OP_SILU = 9, TCX_OP_SOFTMAX = 10,
  TCX_OP_RMSNORM = 11, TCX_OP_LAYERNORM = 12, TCX_OP_SUBTRACT = 13, TCX_OP_DIVIDE = 14,
  TCX_OP_NEGATE = 15, TCX_OP_ADD_SCALAR = 16, TCX_OP_SUBTRACT_SCALAR = 17, TCX_OP_MULTIPLY_SCALAR = 18,
  TCX_OP_DIVIDE_SCALAR = 19, TCX_OP_EQUAL = 24, TCX_OP_NOT_EQUAL = 25, TCX_OP_LESS = 26,
  TCX_OP_LESS_EQUAL = 27, TCX_OP_GREATER = 28, TCX_OP_GREATER_EQUAL = 29, TCX_OP_LOGICAL_AND = 30,
  TCX_OP_LOGICAL_OR = 31, TCX_OP_LOGICAL_XOR = 32, TCX_OP_LOGICAL_NOT = 33, TCX_OP_WHERE = 34,
  TCX_OP_ANY = 35, TCX_OP_ALL = 36, TCX_OP_LOG = 38, TCX_OP_SQRT = 39, TCX_OP_ABS = 40,
  TCX_OP_MIN = 41, TCX_OP_ARGMAX = 42, TCX_OP_CLIP = 43, TCX_OP_TOPK = 44
};

/* Activation applied after the bias add in fused chains. ReLU is tensor.cx's
 * clip(x, lower=0) (python/tensorcx/tensor.py:858-876; cpu_math.cpp:42-47). */
enum { TCX_ACT_NONE = 0, TCX_ACT_SILU = 1, TCX_ACT_RELU = 2 };

/* Matmul kernel selection: automatic, the SIMT FFMA kernel, or the tcgen05 3xTF32
 * tensor-core kernel (the latter two for tests and measurement). */
enum { TCX_MATMUL_AUTO = 0, TCX_MATMUL_FFMA = 1, TCX_MATMUL_TENSOR = 2 };

/* ------------------------------------------------------------------ runtime --- */

/* Thread-local message of the last failed call on this thread ("" if none). */
const char* tcx_sm100_last_error(void);

/* ABI revision of this library (bumped on any signature change). */
int tcx_sm100_abi_version(void);

/* TCX_OK when `device` is an sm_100 GPU this library's kernels can run on.
 * Replaces the availability probe of cuda::available() (cuda_backend.cpp:166-169). */
int tcx_sm100_device_supported(int device);

/* Reads and clears the device-side error word of `device`: kernels with bounded
 * waits record a timeout there instead of hanging (0 = no error). */
int tcx_sm100_device_error(int device, int* code);

/* Device timing of this library's kernel launches, the reference's DeviceTimer
 * contract (cpp/tensorcx/backends/cuda/cuda_profiling.h:23-64): while enabled on the
 * calling thread, every kernel the entry points launch is bracketed by CUDA events
 * on its own stream. tcx_sm100_timer_read waits for the recorded events and returns
 * one entry per kernel name: launch count and total device milliseconds. `names`
 * receives up to `capacity` NUL-separated names (each at most 63 bytes). Reading
 * clears the records. Disabled by default; costs nothing when disabled. */
int tcx_sm100_timer_enable(int enable);
int tcx_sm100_timer_read(char* names, size_t names_bytes, int64_t* launches, double* total_ms,
                         int32_t capacity, int32_t* entries);

/* --------------------------------------------------------------- reductions --- */

/* One-axis reduction or normalization over a contiguous tensor viewed as
 * [outer, reduce, inner] (axis extent `reduce`, element stride `inner`).
 * Replaces launch_axis (cuda_kernels.h:34-36; primitives.cu:290-306).
 *   op  TCX_OP_SUM / TCX_OP_MAX (float32, int32), TCX_OP_MEAN (float32): output
 *       [outer, inner]. For float32 sum/mean the order of additions is the CPU
 *       reference's left-to-right order, bit for bit, whenever reduce <= 65536 or
 *       there are at least 4096 independent rows; otherwise (few very long rows) a
 *       fixed-shape pairwise tree (relative error <= 1e-5 against the CPU result).
 *       Max is exact in every case (first NaN, first of equal values).
 *   op  TCX_OP_SOFTMAX / TCX_OP_RMSNORM / TCX_OP_LAYERNORM (float32): output has the
 *       input's shape; `epsilon` is the already-validated float32 epsilon
 *       (cpu_backend.cpp:30-42 checks it on the host side). */
int tcx_sm100_axis(tcx_stream_t stream, int op, int dtype, const void* input, void* output,
                   int64_t outer, int64_t reduce, int64_t inner, float epsilon,
                   void* workspace, size_t workspace_bytes);

/* Scratch for tcx_sm100_axis (non-zero only for sum/max/mean over few long rows,
 * which run the parallel tree; with less workspace those run the ordered kernel). */
size_t tcx_sm100_axis_workspace_bytes(int op, int64_t outer, int64_t reduce, int64_t inner);

/* Affine normalization fused into one pass: normalize, multiply by weight[reduce]
 * (if non-NULL), then add bias[reduce] (if non-NULL), each a separately rounded
 * float32 operation. Replaces the three-call kAffineRmsNorm / kAffineLayerNorm
 * composite (core/inference.cpp:103-122). op is TCX_OP_RMSNORM or TCX_OP_LAYERNORM. */
int tcx_sm100_affine_norm(tcx_stream_t stream, int op, const float* input, float* output,
                          int64_t outer, int64_t reduce, int64_t inner, float epsilon,
                          const float* weight, const float* bias);

/* Multi-axis reduction (sum / max / mean) described by the reduction plan's index
 * metadata: `rank` (extent, element stride) pairs, kept axes first, reduced axes last
 * (core/shape.h:59-70). groups = number of outputs, reduction_size = elements per
 * output. Replaces launch_reduce_axes (cuda_kernels.h:37-40). A reduction over every
 * axis (groups == 1) runs the bandwidth-bound two-stage kernel: exact for int32 and
 * max, fixed-order pairwise tree for float32 sum/mean (relative error <= 1e-5).
 * Other selections keep the CPU order exactly. `workspace` >= the bytes returned by
 * tcx_sm100_reduce_workspace_bytes(groups * reduction_size). */
int tcx_sm100_reduce_axes(tcx_stream_t stream, int op, int dtype, const void* input,
                          void* output, int64_t groups, int64_t reduction_size,
                          const int64_t* index_metadata, int32_t outer_rank, int32_t rank,
                          void* workspace, size_t workspace_bytes);

/* min (op TCX_OP_MIN, output dtype = input dtype) or argmax (TCX_OP_ARGMAX, int32
 * output) over the plan's metadata, as make_math_plan builds it (core/math.cpp:39-56).
 * Replaces math_kernel codes 3 and 4 (math.cu:56-60). The first NaN wins; otherwise
 * the first extremum (lowest index) wins, with -0 == +0, as cpu_math.cpp:48-54. */
int tcx_sm100_min_argmax(tcx_stream_t stream, int op, int dtype, const void* input,
                         void* output, int64_t groups, int64_t reduction_size,
                         const int64_t* index_metadata, int32_t rank, void* workspace,
                         size_t workspace_bytes);

/* Scratch needed by the full-tensor reduction kernels for `count` input elements. */
size_t tcx_sm100_reduce_workspace_bytes(int64_t count);

/* Full-tensor reduction of a contiguous buffer of `count` elements:
 * op in {SUM, MAX, MEAN, MIN, ARGMAX}. Equivalent to tcx_sm100_reduce_axes /
 * tcx_sm100_min_argmax over every axis; `output` holds one element (int32 for
 * ARGMAX). */
int tcx_sm100_reduce_all(tcx_stream_t stream, int op, int dtype, const void* input,
                         int64_t count, void* output, void* workspace,
                         size_t workspace_bytes);

/* tcx_sm100_reduce_all for callers that cannot allocate device memory (no
 * counterpart in the reference). Some hosts own the whole device memory budget and
 * forbid any other allocation, and some loops cannot pay the device-wide
 * synchronization of cudaMalloc/cudaFree; this entry point needs no workspace. Its
 * scratch is a fixed 16 KiB device array inside the library (1024 partial records),
 * held on every device that loads the library until the process exits. The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress), so
 * make that first call before any stream capture. A failed lookup is not kept (the
 * next call retries it), and after the device's context is destroyed and recreated
 * (cudaDeviceReset) the next call looks the address up again. Calls share the one array: two
 * calls that overlap on the GPU (e.g. on different streams) race and must be
 * serialized by the caller. Inputs whose stage-1 grid needs more than 1024 records
 * are rejected with TCX_INVALID_ARGUMENT (never on GPUs with up to 256 SMs). */
int tcx_sm100_reduce_all_noalloc(tcx_stream_t stream, int op, int dtype, const void* input,
                                 int64_t count, void* output);

/* Per-shard partial of a full-tensor reduction, for combining across GPUs. The
 * record is produced on the device; shards are combined in rank order by
 * tcx_sm100_reduce_combine, so the result does not depend on collective ordering.
 * `index_base` is the global index of this shard's first element. */
typedef struct tcx_partial {
  uint32_t key;    /* order key of the best element (min/max/argmax) */
  uint32_t bits;   /* raw bits of the best element, or of the float32/int32 sum */
  int64_t index;   /* global index of the best element (lowest among ties) */
} tcx_partial;

int tcx_sm100_reduce_partial(tcx_stream_t stream, int op, int dtype, const void* input,
                             int64_t count, int64_t index_base, tcx_partial* partial,
                             void* workspace, size_t workspace_bytes);

/* Combines `nparts` device records in order into the final one-element output of
 * a reduction over `total_count` elements (the mean divides by it once). */
int tcx_sm100_reduce_combine(tcx_stream_t stream, int op, int dtype,
                             const tcx_partial* partials, int32_t nparts,
                             int64_t total_count, void* output);

/* ------------------------------------------ cross-GPU fold over peer memory --- */

/* The multi-GPU full reduction with its exchange step inside the kernel, in place of
 * reduce_partial + an all-gather of the records + reduce_combine (the sharded helper
 * of the 2/4/8-GPU path; the reference runs one device, cuda_backend.cpp:272-274).
 * Each rank owns a mailbox: a device allocation of tcx_sm100_mailbox_bytes(world)
 * that every rank maps through CUDA IPC (one process per GPU, peer access over
 * NVLink / NVSwitch). The calling rank's kernel folds its shard to one record, stores
 * it with a system-scope release into slot `rank` of every rank's mailbox, waits until
 * all `world` records of this `epoch` are in its own mailbox (bounded by
 * `wait_limit_ns`; on expiry the device error word is set, see
 * tcx_sm100_device_error, and the output is undefined), and folds them in rank order
 * exactly as tcx_sm100_reduce_combine, so every rank gets the same value.
 * Epochs start at 1 and rise by 1 per call on every rank (two slot sets, by epoch
 * parity, let a rank run one call ahead of a slower peer). */
size_t tcx_sm100_mailbox_bytes(int32_t world);
/* Allocates and zeroes a mailbox; writes its IPC handle (64 bytes) to ipc_handle. */
int tcx_sm100_mailbox_create(int32_t world, void** mailbox, void* ipc_handle);
/* Maps a peer's mailbox from its IPC handle; tcx_sm100_mailbox_close unmaps it. */
int tcx_sm100_mailbox_open(const void* ipc_handle, void** peer_mailbox);
int tcx_sm100_mailbox_close(void* peer_mailbox);
int tcx_sm100_mailbox_free(void* mailbox);
/* `mailboxes` is a host array of `world` device pointers: the mapped mailbox of each
 * rank, this rank's own at [rank]. `workspace` as for tcx_sm100_reduce_partial. */
int tcx_sm100_reduce_sharded(tcx_stream_t stream, int op, int dtype, const void* input,
                             int64_t count, int64_t index_base, void* const* mailboxes,
                             int32_t rank, int32_t world, uint64_t epoch, uint64_t wait_limit_ns,
                             int64_t total_count, void* output, void* workspace,
                             size_t workspace_bytes);

/* -------------------------------------------------------------- elementwise --- */

/* exp / gelu (tanh form) / silu, float32. Replaces launch_unary (cuda_kernels.h:32-33;
 * primitives.cu:14-27). Arithmetic follows cpu_backend.cpp:990-1010 operation by
 * operation (no contraction into FMA). */
int tcx_sm100_unary(tcx_stream_t stream, int op, const float* input, float* output,
                    int64_t count);

/* add / subtract / multiply / divide with NumPy broadcasting. `metadata` holds the
 * output shape, then the lhs element strides, then the rhs element strides (zero for
 * broadcast axes), 3*rank values (core/shape.h:14-22). rank 0 or identical shapes may
 * pass metadata = NULL, rank = 0. int32 wraps through uint32; divide is float32 only.
 * Replaces launch_binary / launch_broadcast_binary (cuda_kernels.h:15-22). */
int tcx_sm100_binary(tcx_stream_t stream, int op, int dtype, const void* lhs,
                     const void* rhs, void* output, int64_t count, const int64_t* metadata,
                     int32_t rank);

/* clip(x, lower, upper) with broadcast bounds: metadata = output shape then the
 * element strides of x, lower and upper (4*rank values), as make_math_plan builds it
 * (core/math.cpp:33-38). Replaces math_kernel code 5 (math.cu:51-55). */
int tcx_sm100_clip(tcx_stream_t stream, int dtype, const void* input, const void* lower,
                   const void* upper, void* output, int64_t count, const int64_t* metadata,
                   int32_t rank);

/* Fused elementwise chain out[r, c] = act(x[r, c] + bias[c]) over a [rows, cols]
 * buffer (bias may be NULL). Replaces the broadcast add + activation pair of calls
 * (cuda_backend.cpp:557-578 then 604-605) with one read and one write. */
int tcx_sm100_bias_act(tcx_stream_t stream, const float* input, const float* bias,
                       float* output, int64_t rows, int64_t cols, int act);

/* Fills `count` 32-bit elements with the raw word `bits` (float32 or int32 value as
 * stored). Replaces launch_fill (cuda_kernels.h:13-14). */
int tcx_sm100_fill(tcx_stream_t stream, void* output, int64_t count, uint32_t bits);

/* ------------------------------------------------------------------- matmul --- */

/* Scratch for tcx_sm100_matmul: the tf32 hi/lo split of both operands (K-major), or,
 * when k and n are multiples of 4 and both operands are 16-byte aligned, only their lo
 * terms in the operands' own layouts (the tensor cores then read the operands
 * themselves as the hi terms); the size covers either. It also covers the partial
 * accumulators of small products split over k (split-K) or, for products large enough
 * for the two-SM (CTA-pair) tiles, of tiles split between two SM pairs (stream-K: 256
 * KiB per SM pair). A workspace sized before those areas existed is still accepted (no
 * split is made then). lhs_batches / rhs_batches are the operands' own batch counts
 * (numel / (m*k), numel / (k*n)). Zero when the FFMA kernel will be used. Calls that
 * share one workspace must not overlap on the GPU. */
size_t tcx_sm100_matmul_workspace_bytes(int64_t m, int64_t n, int64_t k,
                                        int64_t lhs_batches, int64_t rhs_batches, int path);

/* Batched float32 matmul with NumPy broadcasting, as planned by make_matmul_plan
 * (core/shape.cpp:49-76): output [batches, m, n] contiguous; batch b reads
 * lhs + offset(b, lhs_batch_strides) and rhs + offset(b, rhs_batch_strides), offsets
 * as matmul_batch_offset (shape.cpp:78-85) over `batch_shape` (batch_rank entries;
 * batches = its product). Optional fused epilogue: out = act(acc + bias[n]) when
 * bias != NULL or act != TCX_ACT_NONE. Replaces launch_matmul (cuda_kernels.h:43-45)
 * and, with an epilogue, the matmul -> add -> activation call chain.
 * Large products run on tcgen05 tensor cores with a 3xTF32 split
 * (hi*hi + hi*lo + lo*hi, float32 accumulation; hi = the tf32 truncation of x when the
 * operands are read in place, else its rounding): relative Frobenius error
 * <= 1e-4 * sqrt(k / 1024) against the CPU reference. Inputs holding inf or NaN are
 * computed by the FFMA kernel instead (IEEE semantics), decided on the device. */
int tcx_sm100_matmul(tcx_stream_t stream, const float* lhs, const float* rhs, float* output,
                     int64_t m, int64_t n, int64_t k, int64_t batches,
                     const int64_t* batch_shape, const int64_t* lhs_batch_strides,
                     const int64_t* rhs_batch_strides, int32_t batch_rank,
                     const float* bias, int act, int path, void* workspace,
                     size_t workspace_bytes);

/* C = A @ B for HOST buffers A [m, k], B [k, n], C [m, n] (row-major float32), the
 * transfer-inclusive form of tcx_sm100_matmul. B is uploaded once; A and C move in
 * row chunks through three streams (upload, compute, download) so copies in both
 * directions overlap the GEMMs of neighbouring chunks. Synchronous: returns when C is
 * complete in host memory. Host buffers should be page-locked (cudaHostAlloc or
 * cudaHostRegister); pageable buffers still work, without overlap. `workspace` is
 * device memory of at least tcx_sm100_matmul_host_workspace_bytes(m, n, k). Uses the
 * current device. (The reference's equivalent is from_cpu, matmul and to_cpu in
 * sequence, cuda_backend.cpp:215-264.) */
size_t tcx_sm100_matmul_host_workspace_bytes(int64_t m, int64_t n, int64_t k);
int tcx_sm100_matmul_host(const float* a_host, const float* b_host, float* c_host, int64_t m, int64_t n,
                          int64_t k, void* workspace, size_t workspace_bytes);

/* linear(x, w, bias): out[r, o] = act(sum_k x[r, k] * w[o, k] + bias[o]) for x [rows, in],
 * w [out_features, in] (the nn.Linear layout, i.e. K-major), bias [out_features] or
 * NULL. One GEMM with the bias (and activation) in its epilogue; the weight is used
 * in place, without the transpose copy of the reference's kLinear composite
 * (core/inference.cpp:89-102: transpose, matmul, add). Same kernels, accuracy and
 * workspace rules as tcx_sm100_matmul. */
size_t tcx_sm100_linear_workspace_bytes(int64_t rows, int64_t in_features, int64_t out_features, int path);
int tcx_sm100_linear(tcx_stream_t stream, const float* x, const float* w, const float* bias, float* output,
                     int64_t rows, int64_t in_features, int64_t out_features, int act, int path,
                     void* workspace, size_t workspace_bytes);

/* Masked, scaled row softmax of attention scores (kAttentionSoftmax; plan
 * make_attention_softmax_plan, core/inference.cpp:56-83; CPU semantics
 * cpu_inference.cpp:22-45; replaces launch_attention_softmax, kernels/inference.cu:53).
 * The target is `shape` [..., queries, keys] (rank 2..32), output contiguous. `scores`
 * and `mask` are read through broadcast strides over that shape (0 = broadcast; the
 * last-axis stride must be 0 or 1). mask_kind: 0 none, 1 bool (one byte per element,
 * nonzero = allowed), 2 float32 added to the scaled score. Per row: score = -inf where
 * causal and key > query, where a bool mask is false or a float mask is -inf; otherwise
 * scores * scale + mask. A row whose maximum is -inf is all zeros; a NaN makes the row
 * NaN; else exp(score - max) / sum. `scale` must be finite. */
int tcx_sm100_attention_softmax(tcx_stream_t stream, const float* scores, const void* mask, int32_t mask_kind,
                                float* output, const int64_t* shape, const int64_t* score_strides,
                                const int64_t* mask_strides, int32_t rank, float scale, int32_t causal);

/* Scaled dot-product attention (kAttention, core/inference.cpp:123-160): out =
 * attention_softmax(Q·Kᵀ, mask, scale, causal) · V. Without a mask, with features and
 * value_features multiples of 32 up to 128 and a 16-byte aligned output, one fused
 * tcgen05 kernel computes it (scores and probabilities stay in TMEM; the workspace holds
 * only the 3xTF32 split planes of q, k and v, or k's lo terms, and for products with few
 * 256-query items the partial rows of items cut into key ranges); otherwise the
 * composite below runs. Inputs
 * holding inf / NaN are computed by an IEEE row kernel (decided on the device).
 * q [batch..., queries, features],
 * k [batch..., keys, features], v [batch..., keys, value_features], each batch-broadcast
 * to `batch_shape` through its batch strides (element units, 0 = broadcast, as
 * tcx_sm100_matmul). mask_strides: batch_rank + 2 strides of the mask over
 * [batch..., queries, keys] (ignored when mask_kind is 0). The keys are read K-major by
 * the GEMM (no transpose copy); the scores live in the workspace. Output contiguous
 * [batch..., queries, value_features]. q/k/v_batches = the number of distinct batch
 * matrices of each operand (the product of its own batch extents). */
size_t tcx_sm100_attention_workspace_bytes(int64_t batches, int64_t queries, int64_t keys, int64_t features,
                                           int64_t value_features, int64_t q_batches, int64_t k_batches,
                                           int64_t v_batches, int32_t mask_kind);
int tcx_sm100_attention(tcx_stream_t stream, const float* q, const float* k, const float* v, const void* mask,
                        int32_t mask_kind, float* output, int64_t queries, int64_t keys, int64_t features,
                        int64_t value_features, const int64_t* batch_shape, const int64_t* q_batch_strides,
                        const int64_t* k_batch_strides, const int64_t* v_batch_strides, int32_t batch_rank,
                        const int64_t* mask_strides, float scale, int32_t causal, void* workspace,
                        size_t workspace_bytes);

/* Synchronous copies between host and device memory of the current device (the
 * transfers of from_cpu / to_cpu, cuda_backend.cpp:215-264 of the reference). Pageable
 * host buffers of 4 MiB and more are staged through two page-locked 32 MiB slots per
 * device, with several host threads copying one slot while the DMA engine moves the
 * other; page-locked buffers and small copies use one cudaMemcpyAsync. `stream` orders
 * the copy after earlier work on it; the call returns when the copy is complete. */
int tcx_sm100_copy_to_device(tcx_stream_t stream, void* dst, const void* src, size_t bytes);
int tcx_sm100_copy_to_host(tcx_stream_t stream, void* dst, const void* src, size_t bytes);

/* Seeded float32 generation on the device, in place of drawing on the host and
 * uploading: tensor.cx's randn (python/tensorcx/tensor.py:485-497) draws with NumPy
 * and copies through from_cpu (cpp/tensorcx/backends/cuda/cuda_backend.cpp:215-236).
 * Writes elements [offset, offset + count) of the stream of `seed` into out[0, count).
 * The stream is counter-based (Philox4x32-10): element e depends only on (seed, e),
 * so slices generated at different offsets (e.g. one per GPU) concatenate to the
 * stream generated whole. NORMAL: mean a, standard deviation b (Box-Muller); UNIFORM:
 * [a, b) with 24 random bits per value. The numbers differ from NumPy's generator
 * (PCG64 + ziggurat), which no device generator reproduces. */
enum { TCX_RANDOM_NORMAL = 0, TCX_RANDOM_UNIFORM = 1 };
int tcx_sm100_random(tcx_stream_t stream, int distribution, float* out, int64_t count, uint64_t seed,
                     uint64_t offset, float a, float b);

/* -------------------------------------------------------- tensor operations --- */
/* The reference CUDA backend's remaining primitives (data movement, predicates, casts,
 * scalar arithmetic, topk, embedding), off the hot path but needed for a drop-in
 * device="cuda". Stream-ordered like the rest; results as the reference's kernels and
 * CPU backend, bit for bit (log within 1 ulp: CUDA's logf against std::log). */

/* One-input elementwise ops over `count` float32 or int32 words: TCX_OP_NEGATE,
 * TCX_OP_{ADD,SUBTRACT,MULTIPLY,DIVIDE}_SCALAR (scalar rounded to float32, or an int32
 * value; scalar_left puts it on the left; no int32 divide), TCX_OP_LOG / TCX_OP_SQRT
 * (float32), TCX_OP_ABS (float32: sign cleared; int32: wraps at INT_MIN). Replaces
 * launch_unary's negate, launch_scalar and math_kernel codes 0-2 (primitives.cu:14-32,
 * elementwise.cu:110-116, math.cu:29-41). */
int tcx_sm100_map(tcx_stream_t stream, int op, int dtype, const void* input, void* output, int64_t count,
                  double scalar, int32_t scalar_left);

/* Cast between TCX_FLOAT32, TCX_INT32 and TCX_BOOL. float32 -> int32 truncates toward
 * zero; a value that is not finite or lies outside [-2^31, 2^31) raises the device int
 * *invalid_flag (cleared first; required for this pair), which the caller reads before
 * using the output. Same dtype copies. Replaces launch_validate_int32_cast, launch_cast
 * and launch_bool_cast (elementwise.cu:85-107, predicate.cu:62-71). */
int tcx_sm100_cast(tcx_stream_t stream, int src_dtype, int dst_dtype, const void* input, void* output,
                   int64_t count, int* invalid_flag);

/* Comparisons (TCX_OP_EQUAL .. TCX_OP_GREATER_EQUAL: float32, int32 or bool inputs, bool
 * output), logical ops (bool) and TCX_OP_WHERE (bool condition a, branches b and c of
 * `dtype`, output `dtype`), with broadcasting: metadata = output shape, then the element
 * strides of each input (0 = broadcast), (1 + inputs) * rank values, as
 * make_predicate_plan builds them (core/predicate.cpp). Replaces launch_predicate
 * (predicate.cu:19-61). */
int tcx_sm100_predicate(tcx_stream_t stream, int op, int dtype, const void* a, const void* b, const void* c,
                        void* output, int64_t count, const int64_t* metadata, int32_t rank);

/* any (TCX_OP_ANY) / all (TCX_OP_ALL) of bool elements over the reduction plan's
 * (extent, stride) pairs (make_boolean_reduction_plan). Replaces launch_bool_reduce. */
int tcx_sm100_bool_reduce(tcx_stream_t stream, int op, const void* input, void* output, int64_t groups,
                          int64_t reduction_size, const int64_t* index_metadata, int32_t rank);

/* Transpose / slice: output element i (contiguous over `shape`) = input[offset +
 * sum(coord * input_strides)], 1- or 4-byte elements (make_transpose_plan /
 * make_slice_plan). A transpose of the last two axes goes through 32 x 32 shared-memory
 * tiles. Replaces launch_transpose (elementwise.cu:62-76). */
int tcx_sm100_index_copy(tcx_stream_t stream, int32_t element_bytes, const void* input, void* output, int64_t count,
                         const int64_t* shape, const int64_t* input_strides, int32_t rank, int64_t offset);

/* One input of a concat: input element i goes to output (i / block) * output_block +
 * offset + i % block (make_concat_plan). Replaces launch_concat (elementwise.cu:78-83). */
int tcx_sm100_concat(tcx_stream_t stream, int32_t element_bytes, const void* input, void* output, int64_t count,
                     int64_t block, int64_t output_block, int64_t offset);

/* masked_select (make_masked_select_plan): first the number of selected mask positions
 * into the device int64 *selected (the output's leading extent; the caller reads it and
 * sizes the output), then the copy of each selected position's block of `block`
 * elements in order. Both calls take the same workspace, which carries the per-tile
 * offsets from the first to the second. Replaces launch_mask_prefix / launch_prefix_step
 * / launch_mask_copy (predicate.cu:76-101). */
size_t tcx_sm100_masked_select_workspace_bytes(int64_t mask_count);
int tcx_sm100_masked_select_count(tcx_stream_t stream, const void* mask, int64_t mask_count, int64_t* selected,
                                  void* workspace, size_t workspace_bytes);
int tcx_sm100_masked_select(tcx_stream_t stream, int32_t element_bytes, const void* input, const void* mask,
                            int64_t mask_count, int64_t block, void* output, const void* workspace,
                            size_t workspace_bytes);

/* topk along one axis (make_math_plan code 6): `groups` output groups of k values (the
 * input's dtype) and int32 indices, group g reading elements base + j * inner. Order as
 * the reference: largest: NaN first, then larger, ties to the lower index; smallest:
 * smaller first, NaN last; unsorted: the selected indices ascending. Replaces
 * math_kernel code 6 (math.cu:61-76). */
int tcx_sm100_topk(tcx_stream_t stream, int dtype, const void* input, void* values, int32_t* indices, int64_t groups,
                   int64_t reduction_size, int64_t inner, int64_t k, int32_t largest, int32_t sorted);

/* Embedding gather: output row i = weight row indices[i] (float32 rows of `width`); an
 * index outside [0, vocabulary) raises the device int *invalid_flag (cleared first),
 * which the caller reads. Replaces launch_embedding_validate / launch_embedding_gather
 * (inference.cu:8-15). */
int tcx_sm100_embedding(tcx_stream_t stream, const int32_t* indices, int64_t rows, const float* weight,
                        int64_t vocabulary, int64_t width, float* output, int* invalid_flag);

#ifdef __cplusplus
}  /* extern "C" */
#endif
#endif  /* TCX_SM100_H_ */
