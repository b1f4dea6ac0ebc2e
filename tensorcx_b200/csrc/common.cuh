// Shared helpers of the sm_100a backend: error reporting across the C ABI, launch
// geometry and the float32/int32 order keys used by the reductions.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "tcx_sm100.h"

namespace tcx {

// Thread-local last-error message behind tcx_sm100_last_error().
void set_error(const std::string& message);
void clear_error();

inline int invalid(const char* message) {
  set_error(message);
  return TCX_INVALID_ARGUMENT;
}

// Maps the launch status of the kernels just enqueued to a C-ABI status.
inline int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return TCX_OK;
  set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return TCX_INTERNAL;
}

// Number of SMs of the current device (cached per device).
int sm_count();

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization (launch_after) may start while the kernel before it in the stream is
// still running; dependents_may_launch() in that earlier kernel lets it be scheduled,
// and wait_for_prior_grid() in it blocks until the earlier grid has finished and its
// memory is visible (a no-op for a kernel launched the ordinary way). The later
// kernel's launch and set-up then overlap the earlier kernel's tail.
__device__ __forceinline__ void dependents_may_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void wait_for_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launches `kernel` with programmatic stream serialization (see above); `dynamic_smem`
// bytes of dynamic shared memory.
template <typename... Params, typename... Args>
void launch_after(void (*kernel)(Params...), dim3 grid, dim3 block, cudaStream_t s, size_t dynamic_smem,
                  Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = dynamic_smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

// Device-side error word (see tcx_sm100_device_error); bounded waits set it.
__device__ __forceinline__ void record_device_error(int* word, int code) {
  if (word) atomicCAS(word, 0, code);
}
int* device_error_word();

// Brackets the kernel launches of its scope with CUDA events when the calling
// thread enabled tcx_sm100_timer_enable (runtime.cu); otherwise does nothing.
class TimedLaunch {
 public:
  TimedLaunch(const char* name, cudaStream_t stream);
  ~TimedLaunch();
  TimedLaunch(const TimedLaunch&) = delete;
  TimedLaunch& operator=(const TimedLaunch&) = delete;

 private:
  const char* name_;
  cudaStream_t stream_;
  cudaEvent_t start_ = nullptr;
};

constexpr int kMaxRank = 16;

// Small by-value metadata block passed as a kernel parameter (no per-call
// device allocation, unlike the reference's cudaMalloc + cudaMemcpy uploads).
struct Meta {
  int32_t rank;
  int64_t v[4 * kMaxRank];
};

// ------------------------------------------------------------ order keys
// 32-bit keys whose unsigned order is the reduction's preference order:
// a larger key wins; equal keys fall back to the lower index. NaN maps to the
// largest key (the first NaN wins), both zeros share one key (they compare equal),
// as cpu_math.cpp:14-21 and std::max in cpu_backend.cpp:1190-1196.
__device__ __forceinline__ uint32_t ordered_f32(uint32_t b) {
  if ((b & 0x7fffffffu) == 0) b = 0;  // -0 == +0
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ bool is_nan_bits(uint32_t b) {
  return (b & 0x7fffffffu) > 0x7f800000u;
}
// key for "largest wins" (max, argmax)
__device__ __forceinline__ uint32_t key_max(uint32_t b, bool fp) {
  if (!fp) return b ^ 0x80000000u;
  return is_nan_bits(b) ? 0xffffffffu : ordered_f32(b);
}
// key for "smallest wins" (min); NaN still wins.
__device__ __forceinline__ uint32_t key_min(uint32_t b, bool fp) {
  if (!fp) return ~(b ^ 0x80000000u);
  return is_nan_bits(b) ? 0xffffffffu : ~ordered_f32(b);
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Merges adjacent axes that stay affine for every operand and drops unit axes
// (elementwise.cu): strides[k] is operand k's stride vector over `shape` (rank entries);
// on return out_shape and strides hold the collapsed axes. Returns the collapsed rank.
int collapse(const int64_t* shape, std::vector<std::vector<int64_t>>& strides, int rank,
             std::vector<int64_t>& out_shape);

// One-axis sum/max/mean over [outer, reduce, inner] (reduce.cu).
int axis_reduce(cudaStream_t s, int op, int dtype, const void* input, void* output,
                int64_t outer, int64_t reduce, int64_t inner, void* ws, size_t ws_bytes);
size_t axis_reduce_workspace(int64_t outer, int64_t reduce, int64_t inner);

// Batched matmul of tcx_sm100_matmul (gemm.cu) for composites; rhs_kmajor reads the
// right operand as [batch..., n, k]. Workspace as tcx_sm100_matmul_workspace_bytes.
int matmul_run(cudaStream_t stream, const float* lhs, const float* rhs, float* output, int64_t m, int64_t n,
               int64_t k, int64_t batches, const int64_t* batch_shape, const int64_t* lhs_batch_strides,
               const int64_t* rhs_batch_strides, int32_t batch_rank, bool rhs_kmajor, void* workspace,
               size_t workspace_bytes);

// Split pre-pass of the 3xTF32 tensor path (gemm.cu): nb matrices [rows, k] -> K-major
// hi/lo planes [2 * nb, rows, kp]; the column form transposes nb matrices [k, n] into
// [2 * nb, n, kp]. Both raise *flag on inf / NaN. encode_planes_map builds the TMA map
// (box {32, box_rows, 1}, 128-byte swizzle) over such planes, or over any stack of
// `planes` row-major [rows, kp] float32 matrices; with mn_atom32 the swizzle has 32-byte
// atoms (the layout of MN-major tf32 MMA operands). `map` is a CUtensorMap*.
void split_rows_planes(cudaStream_t s, const float* x, float* planes, int64_t nb, int64_t rows, int64_t k,
                       int64_t kp, int* flag);
// Two row splits with the same K in one launch (x1 and x2 as split_rows_planes).
void split_rows_planes2(cudaStream_t s, const float* x1, float* planes1, int64_t nb1, int64_t rows1,
                        const float* x2, float* planes2, int64_t nb2, int64_t rows2, int64_t k, int64_t kp,
                        int* flag);
void split_cols_planes(cudaStream_t s, const float* x, float* planes, int64_t nb, int64_t k, int64_t n,
                       int64_t kp, int* flag);
bool encode_planes_map(void* map, const float* base, int64_t planes, int64_t rows, int64_t kp, int box_rows,
                       bool mn_atom32 = false);
// Raw-mode lo terms (gemm.cu split_lo): lo[i] = rna_tf32(x[i] - trunc_tf32(x[i])) for n4
// 16-byte words, elementwise in x's own layout; raises *flag on inf / NaN.
void split_lo_planes(cudaStream_t s, const float* x, float* lo, int64_t n4, int* flag);

// Fused attention (flash.cu): eligibility, workspace and launch.
bool flash_eligible(int64_t queries, int64_t keys, int64_t features, int64_t value_features, int mask_kind,
                    int batch_rank);
size_t flash_workspace_bytes(int64_t queries, int64_t keys, int64_t features, int64_t value_features,
                             int64_t q_batches, int64_t k_batches, int64_t v_batches, int64_t batches,
                             int mask_kind);
int attention_fused(cudaStream_t s, const float* q, const float* k, const float* v, const void* mask,
                    int mask_kind, const int64_t* mask_strides, float* out, int64_t L, int64_t S, int64_t d,
                    int64_t dv, int64_t batches, const int64_t* batch_shape, const int64_t* q_strides,
                    const int64_t* k_strides, const int64_t* v_strides, int32_t rank, float scale, int causal,
                    void* workspace, size_t workspace_bytes);

}  // namespace tcx
