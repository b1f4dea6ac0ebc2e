// Row-statistics helpers shared by the row kernels (rows.cu) and the attention
// softmax (attention.cu): an ex2-based exponential, a NaN-propagating max and
// CTA-wide sum / max reductions built from warp shuffles plus one shared-memory hop.
#pragma once

#include <cuda_runtime.h>
#include <math.h>

namespace tcx {
namespace rowmath {

// e^x through the base-2 identity e^x = 2^(x * log2 e) and the hardware ex2.approx
// instruction (relative error ~2^-22 on the ex2 step, plus |x| * 2^-24 from rounding
// x * log2 e: < 2e-6 for the |x| <= 60 a softmax row can feed it before underflow).
__device__ __forceinline__ float exp_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(__fmul_rn(x, 1.4426950408889634f)));
  return y;
}

__device__ __forceinline__ float nan_max(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  return a < b ? b : a;
}

// CTA-wide reductions; every thread receives the result.
template <int THREADS>
struct Block {
  static constexpr int kWarps = THREADS / 32;
  __device__ static float sum(float v, float* smem) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (kWarps == 1) return v;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) smem[warp] = v;
    __syncthreads();
    float t = lane < kWarps ? smem[lane] : 0.0f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, off));
    return t;
  }
  __device__ static float max(float v, float* smem) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = nan_max(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (kWarps == 1) return v;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) smem[warp] = v;
    __syncthreads();
    float t = lane < kWarps ? smem[lane] : -INFINITY;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) t = nan_max(t, __shfl_xor_sync(0xffffffffu, t, off));
    return t;
  }
  // Sums two values in one pass (one pair of barriers instead of two).
  __device__ static float2 sum2(float a, float b, float* smem) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, off));
      b = __fadd_rn(b, __shfl_xor_sync(0xffffffffu, b, off));
    }
    if (kWarps == 1) return make_float2(a, b);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) { smem[warp] = a; smem[32 + warp] = b; }
    __syncthreads();
    float ta = lane < kWarps ? smem[lane] : 0.0f, tb = lane < kWarps ? smem[32 + lane] : 0.0f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      ta = __fadd_rn(ta, __shfl_xor_sync(0xffffffffu, ta, off));
      tb = __fadd_rn(tb, __shfl_xor_sync(0xffffffffu, tb, off));
    }
    return make_float2(ta, tb);
  }
  __device__ static bool all(bool v, float* smem) {
    v = __all_sync(0xffffffffu, v);
    if (kWarps == 1) return v;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) smem[warp] = v ? 1.0f : 0.0f;
    __syncthreads();
    return __all_sync(0xffffffffu, lane < kWarps ? smem[lane] != 0.0f : true);
  }
};

}  // namespace rowmath
}  // namespace tcx
