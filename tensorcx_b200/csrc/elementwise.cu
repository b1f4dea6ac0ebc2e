// Elementwise kernels: exp / gelu / silu, broadcast arithmetic, clip (ReLU), and the
// fused bias-add + activation chain. All are HBM-bound streams: 128-bit accesses
// where alignment allows, a grid sized to the SM count, broadcast metadata collapsed
// on the host to the fewest axes and passed by value.
//
// Arithmetic mirrors the CPU reference operation by operation (cpu_backend.cpp:
// 990-1010 unary, 1014-1097 binary; cpu_math.cpp:42-47 clip), with _rn intrinsics
// where nvcc would otherwise contract a multiply and an add into one FMA.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <vector>

#include "common.cuh"

namespace tcx {
namespace {

__device__ __forceinline__ float gelu_f(float v) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;  // cpu_backend.cpp:27-28
  const float cube = __fmul_rn(__fmul_rn(__fmul_rn(k1, v), v), v);
  const float inner = __fmul_rn(k0, __fadd_rn(v, cube));
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(inner)));
}
__device__ __forceinline__ float silu_f(float v) { return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v))); }

// clip on raw words (cpu_math.cpp:14-21, 42-47)
__device__ __forceinline__ bool w_nan(uint32_t a, bool fp) { return fp && (a & 0x7fffffffu) > 0x7f800000u; }
__device__ __forceinline__ bool w_less(uint32_t a, uint32_t b, bool fp) {
  if (!fp) return static_cast<int32_t>(a) < static_cast<int32_t>(b);
  if (!(a & 0x7fffffffu)) a = 0;
  if (!(b & 0x7fffffffu)) b = 0;
  const uint32_t ka = (a & 0x80000000u) ? ~a : (a ^ 0x80000000u);
  const uint32_t kb = (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
  return ka < kb;
}
__device__ __forceinline__ uint32_t clip_w(uint32_t a, uint32_t lo, uint32_t hi, bool fp) {
  if (!w_nan(a, fp)) a = (w_nan(lo, fp) || !w_less(lo, a, fp)) ? lo : a;
  if (!w_nan(a, fp)) a = (w_nan(hi, fp) || !w_less(a, hi, fp)) ? hi : a;
  return a;
}
// ReLU = clip(x, +0, +inf) on a float32 word.
__device__ __forceinline__ float relu_f(float v) {
  return __uint_as_float(clip_w(__float_as_uint(v), 0u, 0x7f800000u, true));
}

template <int OP>
__device__ __forceinline__ float unary_f(float v) {
  if (OP == TCX_OP_EXP) return expf(v);
  if (OP == TCX_OP_GELU) return gelu_f(v);
  return silu_f(v);
}

template <int OP>
__global__ void unary_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const bool vec = (reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) % 16 == 0;
  int64_t done = 0;
  if (vec) {
    const int64_t n4 = n >> 2;
    for (int64_t i = tid; i < n4; i += stride) {
      float4 v = __ldcs(reinterpret_cast<const float4*>(x) + i);
      v.x = unary_f<OP>(v.x); v.y = unary_f<OP>(v.y); v.z = unary_f<OP>(v.z); v.w = unary_f<OP>(v.w);
      __stcs(reinterpret_cast<float4*>(out) + i, v);
    }
    done = n4 * 4;
  }
  for (int64_t i = done + tid; i < n; i += stride) out[i] = unary_f<OP>(x[i]);
}

template <typename T>
__device__ __forceinline__ T arith(int op, T a, T b) {
  if constexpr (std::is_same<T, float>::value) {
    switch (op) {
      case TCX_OP_ADD: return __fadd_rn(a, b);
      case TCX_OP_SUBTRACT: return __fsub_rn(a, b);
      case TCX_OP_MULTIPLY: return __fmul_rn(a, b);
      default: return __fdiv_rn(a, b);
    }
  } else {
    const uint32_t x = static_cast<uint32_t>(a), y = static_cast<uint32_t>(b);
    switch (op) {
      case TCX_OP_ADD: return static_cast<T>(x + y);
      case TCX_OP_SUBTRACT: return static_cast<T>(x - y);
      default: return static_cast<T>(x * y);
    }
  }
}

template <typename T>
__global__ void binary_same(int op, const T* __restrict__ a, const T* __restrict__ b,
                            T* __restrict__ out, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  for (int64_t i = tid; i < n; i += stride) out[i] = arith<T>(op, a[i], b[i]);
}

// Collapsed broadcast: meta = out shape, lhs strides, rhs strides (rank <= kMaxRank).
template <typename T>
__global__ void binary_bcast(int op, const T* __restrict__ a, const T* __restrict__ b,
                             T* __restrict__ out, int64_t n, Meta m) {
  const int r = m.rank;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    int64_t idx = i, l = 0, rr = 0;
    for (int axis = r - 1; axis >= 0; --axis) {
      const int64_t c = idx % m.v[axis];
      idx /= m.v[axis];
      l += c * m.v[r + axis];
      rr += c * m.v[2 * r + axis];
    }
    out[i] = arith<T>(op, a[l], b[rr]);
  }
}

__global__ void clip_kernel(bool fp, const uint32_t* __restrict__ x, const uint32_t* __restrict__ lo,
                            const uint32_t* __restrict__ hi, uint32_t* __restrict__ out, int64_t n,
                            Meta m) {
  const int r = m.rank;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    int64_t idx = i, o0 = 0, o1 = 0, o2 = 0;
    for (int axis = r - 1; axis >= 0; --axis) {
      const int64_t c = idx % m.v[axis];
      idx /= m.v[axis];
      o0 += c * m.v[r + axis];
      o1 += c * m.v[2 * r + axis];
      o2 += c * m.v[3 * r + axis];
    }
    out[i] = clip_w(x[o0], lo[o1], hi[o2], fp);
  }
}

template <int ACT>
__device__ __forceinline__ float act_f(float v) {
  if (ACT == TCX_ACT_SILU) return silu_f(v);
  if (ACT == TCX_ACT_RELU) return relu_f(v);
  return v;
}

// out[r, c] = act(x[r, c] + bias[c]); VEC requires cols % 4 == 0 and aligned buffers.
template <int ACT, bool VEC>
__global__ void bias_act_kernel(const float* __restrict__ x, const float* __restrict__ bias,
                                float* __restrict__ out, int64_t rows, int64_t cols) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (VEC) {
    const int64_t c4 = cols >> 2, n4 = rows * c4;
    for (int64_t i = tid; i < n4; i += stride) {
      float4 v = __ldcs(reinterpret_cast<const float4*>(x) + i);
      if (bias) {
        const float4 bb = __ldg(reinterpret_cast<const float4*>(bias) + (i % c4));
        v.x = __fadd_rn(v.x, bb.x); v.y = __fadd_rn(v.y, bb.y);
        v.z = __fadd_rn(v.z, bb.z); v.w = __fadd_rn(v.w, bb.w);
      }
      v.x = act_f<ACT>(v.x); v.y = act_f<ACT>(v.y); v.z = act_f<ACT>(v.z); v.w = act_f<ACT>(v.w);
      __stcs(reinterpret_cast<float4*>(out) + i, v);
    }
  } else {
    const int64_t n = rows * cols;
    for (int64_t i = tid; i < n; i += stride) {
      float v = x[i];
      if (bias) v = __fadd_rn(v, bias[i % cols]);
      out[i] = act_f<ACT>(v);
    }
  }
}

__global__ void fill_kernel(uint32_t* __restrict__ out, int64_t n, uint32_t bits) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  int64_t done = 0;
  if (reinterpret_cast<uintptr_t>(out) % 16 == 0) {
    const uint4 v = make_uint4(bits, bits, bits, bits);
    for (int64_t i = tid; i < (n >> 2); i += stride) reinterpret_cast<uint4*>(out)[i] = v;
    done = (n >> 2) << 2;
  }
  for (int64_t i = done + tid; i < n; i += stride) out[i] = bits;
}

int ew_grid(int64_t n) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256 * 4), 8LL * sm_count() * 4)));
}

}  // namespace

// Merges adjacent axes that stay affine for every operand; drops unit axes.
// groups[k] are stride vectors (one per operand), all of `rank` entries.
int collapse(const int64_t* shape, std::vector<std::vector<int64_t>>& strides, int rank,
             std::vector<int64_t>& out_shape) {
  out_shape.clear();
  std::vector<std::vector<int64_t>> s(strides.size());
  for (int a = 0; a < rank; ++a) {
    if (shape[a] == 1) continue;
    if (!out_shape.empty()) {
      bool merge = true;
      for (size_t k = 0; k < strides.size(); ++k)
        if (s[k].back() != strides[k][a] * shape[a]) merge = false;
      if (merge) {
        out_shape.back() *= shape[a];
        for (size_t k = 0; k < strides.size(); ++k) s[k].back() = strides[k][a];
        continue;
      }
    }
    out_shape.push_back(shape[a]);
    for (size_t k = 0; k < strides.size(); ++k) s[k].push_back(strides[k][a]);
  }
  strides = s;
  return static_cast<int>(out_shape.size());
}

}  // namespace tcx

using namespace tcx;

extern "C" {

int tcx_sm100_fill(tcx_stream_t stream, void* output, int64_t count, uint32_t bits) {
  clear_error();
  if (count < 0) return invalid("negative element count");
  if (count == 0) return TCX_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  TimedLaunch timer("fill", s);
  fill_kernel<<<ew_grid(count), 256, 0, s>>>(static_cast<uint32_t*>(output), count, bits);
  return launch_status("fill");
}

int tcx_sm100_unary(tcx_stream_t stream, int op, const float* input, float* output, int64_t count) {
  clear_error();
  if (count < 0) return invalid("negative element count");
  if (op != TCX_OP_EXP && op != TCX_OP_GELU && op != TCX_OP_SILU) return invalid("unsupported unary operation");
  if (count == 0) return TCX_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid = ew_grid(count);
  TimedLaunch timer("unary", s);
  if (op == TCX_OP_EXP) unary_kernel<TCX_OP_EXP><<<grid, 256, 0, s>>>(input, output, count);
  else if (op == TCX_OP_GELU) unary_kernel<TCX_OP_GELU><<<grid, 256, 0, s>>>(input, output, count);
  else unary_kernel<TCX_OP_SILU><<<grid, 256, 0, s>>>(input, output, count);
  return launch_status("unary");
}

int tcx_sm100_binary(tcx_stream_t stream, int op, int dtype, const void* lhs, const void* rhs,
                     void* output, int64_t count, const int64_t* metadata, int32_t rank) {
  clear_error();
  if (op != TCX_OP_ADD && op != TCX_OP_SUBTRACT && op != TCX_OP_MULTIPLY && op != TCX_OP_DIVIDE)
    return invalid("unsupported binary operation");
  if (dtype != TCX_FLOAT32 && dtype != TCX_INT32) return invalid("CUDA operations only support float32");
  if (dtype == TCX_INT32 && op == TCX_OP_DIVIDE) return invalid("division only supports float32 tensors");
  if (count < 0 || rank < 0) return invalid("negative extents");
  if (count == 0) return TCX_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid = ew_grid(count);
  bool same = rank == 0 || !metadata;
  Meta m;
  m.rank = 0;
  if (!same) {
    std::vector<std::vector<int64_t>> st = {
        std::vector<int64_t>(metadata + rank, metadata + 2 * rank),
        std::vector<int64_t>(metadata + 2 * rank, metadata + 3 * rank)};
    std::vector<int64_t> shape;
    const int r = collapse(metadata, st, rank, shape);
    if (r > kMaxRank) return invalid("broadcast rank exceeds 16 after collapsing");
    same = r == 0 || (r == 1 && st[0][0] == 1 && st[1][0] == 1);
    m.rank = r;
    for (int a = 0; a < r; ++a) { m.v[a] = shape[a]; m.v[r + a] = st[0][a]; m.v[2 * r + a] = st[1][a]; }
  }
  TimedLaunch timer("binary", s);
  if (dtype == TCX_FLOAT32) {
    auto* a = static_cast<const float*>(lhs); auto* b = static_cast<const float*>(rhs);
    auto* o = static_cast<float*>(output);
    if (same) binary_same<float><<<grid, 256, 0, s>>>(op, a, b, o, count);
    else binary_bcast<float><<<grid, 256, 0, s>>>(op, a, b, o, count, m);
  } else {
    auto* a = static_cast<const int32_t*>(lhs); auto* b = static_cast<const int32_t*>(rhs);
    auto* o = static_cast<int32_t*>(output);
    if (same) binary_same<int32_t><<<grid, 256, 0, s>>>(op, a, b, o, count);
    else binary_bcast<int32_t><<<grid, 256, 0, s>>>(op, a, b, o, count, m);
  }
  return launch_status("binary");
}

int tcx_sm100_clip(tcx_stream_t stream, int dtype, const void* input, const void* lower,
                   const void* upper, void* output, int64_t count, const int64_t* metadata,
                   int32_t rank) {
  clear_error();
  if (dtype != TCX_FLOAT32 && dtype != TCX_INT32) return invalid("math operations require float32 or int32 tensors");
  if (count < 0 || rank < 0) return invalid("negative extents");
  if (count == 0) return TCX_OK;
  if (rank > 0 && !metadata) return invalid("missing clip metadata");
  std::vector<std::vector<int64_t>> st(3);
  for (int k = 0; k < 3; ++k) st[k].assign(metadata + (k + 1) * rank, metadata + (k + 2) * rank);
  std::vector<int64_t> shape;
  const int r = collapse(metadata, st, rank, shape);
  if (r > kMaxRank) return invalid("clip rank exceeds 16 after collapsing");
  Meta m;
  m.rank = r;
  for (int a = 0; a < r; ++a) {
    m.v[a] = shape[a];
    for (int k = 0; k < 3; ++k) m.v[(k + 1) * r + a] = st[k][a];
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  TimedLaunch timer("clip", s);
  clip_kernel<<<ew_grid(count), 256, 0, s>>>(dtype == TCX_FLOAT32, static_cast<const uint32_t*>(input),
                                             static_cast<const uint32_t*>(lower),
                                             static_cast<const uint32_t*>(upper),
                                             static_cast<uint32_t*>(output), count, m);
  return launch_status("clip");
}

int tcx_sm100_bias_act(tcx_stream_t stream, const float* input, const float* bias, float* output,
                       int64_t rows, int64_t cols, int act) {
  clear_error();
  if (rows < 0 || cols < 0) return invalid("negative extents");
  if (act != TCX_ACT_NONE && act != TCX_ACT_SILU && act != TCX_ACT_RELU) return invalid("unsupported activation");
  if (rows * cols == 0) return TCX_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = cols % 4 == 0 &&
                   ((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(output) |
                     reinterpret_cast<uintptr_t>(bias)) % 16) == 0;
  const int grid = ew_grid(rows * cols);
  TimedLaunch timer("bias_act", s);
#define TCX_BA(A)                                                                              \
  if (vec) bias_act_kernel<A, true><<<grid, 256, 0, s>>>(input, bias, output, rows, cols);     \
  else bias_act_kernel<A, false><<<grid, 256, 0, s>>>(input, bias, output, rows, cols);
  if (act == TCX_ACT_SILU) { TCX_BA(TCX_ACT_SILU) }
  else if (act == TCX_ACT_RELU) { TCX_BA(TCX_ACT_RELU) }
  else { TCX_BA(TCX_ACT_NONE) }
#undef TCX_BA
  return launch_status("bias_act");
}

}  // extern "C"
