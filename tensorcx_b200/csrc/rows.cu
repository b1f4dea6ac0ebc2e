// Row softmax / rmsnorm / layernorm (+ fused affine) on sm_100a, and the
// tcx_sm100_axis dispatcher.
//
// Contiguous rows (axis = -1, inner == 1) up to 32768 elements stay in registers
// (128-bit loads when the row is 16-byte aligned), so every element is read from HBM
// once and written once: 8 bytes per element, the roofline minimum. Rows up to 16384
// take one small CTA per row (a warp for rows up to 2048) with 16-64 values per thread;
// longer rows take a persistent CTA per SM that prefetches the next row into shared
// memory, or a CTA pair per row. Statistics use warp shuffles plus one shared-memory
// hop. Rows over 32768 stream from global memory in 2-3 passes; strided axes run one
// thread per (outer, inner) column in the reference's own order.
//
// Special cases follow the CPU reference (cpu_backend.cpp:125-240): a NaN anywhere in
// a softmax row makes the row NaN; a constant finite layernorm row gives 0 (NaN when
// epsilon is 0); a zero layernorm denominator gives NaN. Elementwise products and sums
// that the reference performs as separate float32 operations use _rn intrinsics so
// nvcc does not contract them into FMAs.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <string>

#include "common.cuh"
#include "ptx.cuh"
#include "rowmath.cuh"


namespace tcx {
namespace {

enum RowOp { kSoftmax = 0, kRms = 1, kLayer = 2 };

using rowmath::Block;
using rowmath::exp_ex2;
using rowmath::nan_max;

// Per-row math on values held by the CTA's threads. E = elements per thread; valid(q)
// tells whether slot q of this thread holds an element of the row. Callers fill the
// other slots with the padding pad_value<OP>() gives (-inf for softmax, 0 for the norms),
// which leaves every max and sum unchanged, so only layernorm's equality count and
// deviation sum test valid(q).
template <int OP, int THREADS, int E, typename Valid>
__device__ __forceinline__ void row_math(float (&v)[E], Valid valid, int64_t n, float first, float eps,
                                         float* smem) {
  using B = Block<THREADS>;
  if (OP == kSoftmax) {
    // fmaxf skips NaN elements; a NaN still makes the whole row NaN, as the reference
    // does, because its exponential enters the row sum that divides every element.
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < E; ++i) m = fmaxf(m, v[i]);
    m = B::max(m, smem);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      v[i] = exp_ex2(__fsub_rn(v[i], m));
      s = __fadd_rn(s, v[i]);
    }
    s = B::sum(s, smem);
    // one IEEE reciprocal per row, then a multiply per element (<= 1.5 ulp vs division)
    const float inv = __frcp_rn(s);
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = __fmul_rn(v[i], inv);
  } else if (OP == kRms) {
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < E; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    ss = B::sum(ss, smem);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(n)), eps)));
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = __fmul_rn(v[i], scale);
  } else {
    float s = 0.0f, neq = 0.0f;  // neq counts elements != first (exact below 2^24 per thread)
#pragma unroll
    for (int i = 0; i < E; ++i) {
      s = __fadd_rn(s, v[i]);
      if (valid(i)) neq += (v[i] == first) ? 0.0f : 1.0f;
    }
    const float2 r = B::sum2(s, neq, smem);
    s = r.x;
    const bool eq = r.y == 0.0f;
    if (eq && isfinite(first)) {
      const float value = eps == 0.0f ? __int_as_float(0x7fc00000) : 0.0f;
#pragma unroll
      for (int i = 0; i < E; ++i) v[i] = value;
      return;
    }
    const float mean = __fdiv_rn(s, static_cast<float>(n));
    float ssd = 0.0f;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      if (valid(i)) {
        const float d = __fsub_rn(v[i], mean);
        ssd = __fadd_rn(ssd, __fmul_rn(d, d));
      }
    }
    ssd = B::sum(ssd, smem);
    const float denom = __fadd_rn(__fdiv_rn(ssd, static_cast<float>(n)), eps);
    if (denom == 0.0f) {
#pragma unroll
      for (int i = 0; i < E; ++i) v[i] = __int_as_float(0x7fc00000);
      return;
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(denom));
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = __fmul_rn(__fsub_rn(v[i], mean), scale);
  }
}

// Value of the slots past the end of a row: neutral for the row's max and sums.
template <int OP>
__device__ __forceinline__ float pad_value() {
  return OP == kSoftmax ? -INFINITY : 0.0f;
}

__device__ __forceinline__ float affine(float y, const float* w, const float* b, int64_t c) {
  if (w) y = __fmul_rn(y, __ldg(w + c));
  if (b) y = __fadd_rn(y, __ldg(b + c));
  return y;
}

// One CTA per row, the row held in registers. VEC: float4 accesses (row length % 4 == 0
// and 16-byte aligned rows); otherwise scalar accesses, element tid + THREADS*q.
// FULL: n == THREADS * VPT * 4 exactly (every slot valid; no bounds checks). Rows are
// at most 32768 elements here, so column indices fit 32 bits.
template <int OP, int THREADS, int VPT, bool VEC, bool FULL = false>
__global__ void __launch_bounds__(THREADS)
row_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t rows, int64_t n,
           float eps, const float* __restrict__ w, const float* __restrict__ b) {
  constexpr int E = VPT * 4;
  __shared__ float smem[64];
  const int n32 = static_cast<int>(n), n4 = n32 >> 2;
  const int tid = static_cast<int>(threadIdx.x);
  const float pad = pad_value<OP>();
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * n;
    float* orow = out + row * n;
    float v[E];
    if (VEC) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int i4 = tid + j * THREADS;
        float4 t = make_float4(pad, pad, pad, pad);
        if (FULL || i4 < n4) t = __ldcs(reinterpret_cast<const float4*>(xr) + i4);
        v[4 * j + 0] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < E; ++q) {
        const int i = tid + q * THREADS;
        v[q] = i < n32 ? __ldcs(xr + i) : pad;
      }
    }
    const float first = OP == kLayer ? __ldg(xr) : 0.0f;
    auto valid = [&](int q) -> bool {
      if (FULL) return true;
      return VEC ? tid + (q >> 2) * THREADS < n4 : tid + q * THREADS < n32;
    };
    row_math<OP, THREADS, E>(v, valid, n, first, eps, smem);
    if (VEC) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int i4 = tid + j * THREADS;
        if (FULL || i4 < n4) {
          float4 t = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          if (w || b) {
            t.x = affine(t.x, w, b, 4 * i4 + 0); t.y = affine(t.y, w, b, 4 * i4 + 1);
            t.z = affine(t.z, w, b, 4 * i4 + 2); t.w = affine(t.w, w, b, 4 * i4 + 3);
          }
          __stcs(reinterpret_cast<float4*>(orow) + i4, t);
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < E; ++q) {
        const int i = tid + q * THREADS;
        if (i < n32) __stcs(orow + i, (w || b) ? affine(v[q], w, b, i) : v[q]);
      }
    }
  }
}

// Long rows (16384 < n <= 32768 outside the paired kernel's reach, and layernorm rows of
// 8192 < n <= 32768; n % 4 == 0, 16-byte aligned): a persistent kernel, one
// 1024-thread CTA per SM. The CTA holds the current row in registers while the next
// row streams into shared memory through one cp.async.bulk (TMA bulk) copy that
// completes on an mbarrier, so the SM's HBM reads never pause for the row's
// reductions, exponentials and stores.
template <int OP, int VPT>
__global__ void __launch_bounds__(1024, 1)
row_staged_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t rows, int64_t n, float eps,
                  const float* __restrict__ w, const float* __restrict__ b, int* err) {
  constexpr int THREADS = 1024, E = VPT * 4;
  extern __shared__ __align__(128) float stage[];  // one row (n floats)
  __shared__ float smem[64];
  __shared__ uint64_t bar;
  const uint32_t bar_addr = ptx::smem_u32(&bar);
  const uint32_t stage_addr = ptx::smem_u32(stage);
  const uint32_t bytes = static_cast<uint32_t>(n * 4);
  if (threadIdx.x == 0) {
    ptx::mbar_init(bar_addr, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  auto issue = [&](int64_t row) {  // thread 0 only
    ptx::mbar_expect_tx(bar_addr, bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     stage_addr),
                 "l"(x + row * n), "r"(bytes), "r"(bar_addr)
                 : "memory");
  };
  int64_t row = blockIdx.x;
  if (threadIdx.x == 0 && row < rows) issue(row);
  const int n4 = static_cast<int>(n >> 2);
  const int tid = static_cast<int>(threadIdx.x);
  const float pad = pad_value<OP>();
  for (uint32_t it = 0; row < rows; row += gridDim.x, ++it) {
    ptx::wait_or_give_up(bar_addr, it & 1u, err, 0x301);
    float v[E];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int i4 = tid + j * THREADS;
      float4 t = make_float4(pad, pad, pad, pad);
      if (i4 < n4) t = reinterpret_cast<const float4*>(stage)[i4];
      v[4 * j + 0] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
    }
    __syncthreads();  // the whole row is in registers: the stage may be refilled
    if (threadIdx.x == 0 && row + gridDim.x < rows) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(row + gridDim.x);
    }
    const float first = OP == kLayer ? __ldg(x + row * n) : 0.0f;
    auto valid = [&](int q) -> bool { return tid + (q >> 2) * THREADS < n4; };
    row_math<OP, THREADS, E>(v, valid, n, first, eps, smem);
    float* orow = out + row * n;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int i4 = tid + j * THREADS;
      if (i4 < n4) {
        float4 t = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        if (w || b) {
          t.x = affine(t.x, w, b, 4LL * i4 + 0); t.y = affine(t.y, w, b, 4LL * i4 + 1);
          t.z = affine(t.z, w, b, 4LL * i4 + 2); t.w = affine(t.w, w, b, 4LL * i4 + 3);
        }
        __stcs(reinterpret_cast<float4*>(orow) + i4, t);
      }
    }
  }
}

template <int OP, int VPT>
int launch_staged_row(cudaStream_t s, const float* x, float* out, int64_t rows, int64_t n, float eps,
                      const float* w, const float* b) {
  const int smem = static_cast<int>(n * 4);
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(row_staged_kernel<OP, VPT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             4 * 32768) != cudaSuccess)
      return launch_status("staged row smem attribute");
    attr_done[dev] = true;
  }
  const int grid = static_cast<int>(std::min<int64_t>(rows, sm_count()));
  TimedLaunch timer("row_staged", s);
  row_staged_kernel<OP, VPT><<<grid, 1024, smem, s>>>(x, out, rows, n, eps, w, b, device_error_word());
  return launch_status("staged row op");
}

// Softmax and rmsnorm rows of 16384 < n <= 32768 (n % 8 == 0, 16-byte aligned): each
// row is split between the two CTAs of a cluster (one 1024-thread CTA per SM), each
// holding its half of the row in registers while the next row's half streams into its
// shared-memory stage through one cp.async.bulk copy. The halves' statistics cross over
// once per row as one 16-byte st.async store into the peer CTA's shared memory that
// completes on the peer's mbarrier: there is no cluster barrier inside the loop, so
// neither CTA waits for the other's output stores to drain.
//
// Softmax combines the halves as (max_h, sum_h of e^(x - max_h)): the row sum is
// sum_h * e^(max_h - max) added in rank order, and an element is e^(x - max_h) *
// (e^(max_h - max) / sum). A NaN anywhere still reaches every element through the sum;
// a half whose elements are all -inf contributes zeros (NaN if the row is all -inf, as
// the reference's e^(-inf - -inf)). Rmsnorm adds the halves' sums of squares in rank
// order, so both CTAs derive identical row statistics.
template <int OP>
__global__ void __launch_bounds__(1024, 1)
row_pair_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t rows, int64_t n, float eps,
                const float* __restrict__ w, const float* __restrict__ b, int* err) {
  constexpr int THREADS = 1024, VPT = 4, E = VPT * 4;
  using B = Block<THREADS>;
  extern __shared__ __align__(128) float stage[];  // this CTA's half of one row
  __shared__ float smem[64];
  __shared__ __align__(16) float4 inbox[2];  // the peer's statistics, by exchange parity
  __shared__ uint64_t bar, xbar[2];
  const uint32_t rank = ptx::cluster_rank(), peer = rank ^ 1u;
  const int64_t half = n >> 1;
  const int h4 = static_cast<int>(half >> 2);
  const int64_t col0 = static_cast<int64_t>(rank) * half;
  const uint32_t bar_addr = ptx::smem_u32(&bar), stage_addr = ptx::smem_u32(stage);
  const uint32_t bytes = static_cast<uint32_t>(half * 4);
  if (threadIdx.x == 0) {
    ptx::mbar_init(bar_addr, 1);
    ptx::mbar_init(ptx::smem_u32(&xbar[0]), 1);
    ptx::mbar_init(ptx::smem_u32(&xbar[1]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  ptx::cluster_sync_all();  // the peer's barriers exist before the first st.async reaches them
  const uint32_t peer_inbox = ptx::map_rank(ptx::smem_u32(&inbox[0]), peer);
  const uint32_t peer_xbar = ptx::map_rank(ptx::smem_u32(&xbar[0]), peer);
  bool live = true;  // false once a wait gave up (error recorded): later waits are skipped
  uint32_t xseq = 0;
  // Sends (a, c, d) to the peer and returns the peer's values. Every thread calls it once
  // per row after a CTA reduction, so all threads have read this inbox slot's previous
  // contents (two rows back) before the peer can send into it again.
  auto exchange = [&](float a, float c, float d) -> float4 {
    const uint32_t slot = xseq & 1u, parity = (xseq >> 1) & 1u;
    ++xseq;
    const uint32_t mine = ptx::smem_u32(&xbar[slot]);
    if (threadIdx.x == 0) {
      ptx::mbar_expect_tx(mine, 16);
      ptx::st_async_v4(peer_inbox + 16 * slot, a, c, d, 0.0f, peer_xbar + 8 * slot);
    }
    if (live) live = ptx::wait_or_give_up(mine, parity, err, 0x303);
    return inbox[slot];
  };
  auto issue = [&](int64_t row) {  // thread 0 only
    ptx::mbar_expect_tx(bar_addr, bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     stage_addr),
                 "l"(x + row * n + col0), "r"(bytes), "r"(bar_addr)
                 : "memory");
  };
  const int64_t first_row = ptx::cluster_index(), stride = ptx::cluster_count();
  if (threadIdx.x == 0 && first_row < rows) issue(first_row);
  const int tid = static_cast<int>(threadIdx.x);
  const float pad = pad_value<OP>();
  uint32_t it = 0;
  for (int64_t row = first_row; row < rows; row += stride, ++it) {
    if (live) live = ptx::wait_or_give_up(bar_addr, it & 1u, err, 0x302);
    float v[E];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int i4 = tid + j * THREADS;
      float4 t = make_float4(pad, pad, pad, pad);
      if (i4 < h4) t = reinterpret_cast<const float4*>(stage)[i4];
      v[4 * j + 0] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
    }
    __syncthreads();  // this half is in registers: the stage may be refilled
    if (threadIdx.x == 0 && row + stride < rows) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(row + stride);
    }
    if (OP == kSoftmax) {
      float m = -INFINITY;
#pragma unroll
      for (int i = 0; i < E; ++i) m = fmaxf(m, v[i]);
      m = B::max(m, smem);
      const float base = m == -INFINITY ? 0.0f : m;
      float s = 0.0f;
#pragma unroll
      for (int i = 0; i < E; ++i) {
        v[i] = exp_ex2(__fsub_rn(v[i], base));
        s = __fadd_rn(s, v[i]);
      }
      s = B::sum(s, smem);
      const float4 other = exchange(m, s, 0.0f);
      const float m0 = rank == 0 ? m : other.x, s0 = rank == 0 ? s : other.y;
      const float m1 = rank == 0 ? other.x : m, s1 = rank == 0 ? other.y : s;
      const float mx = fmaxf(m0, m1);
      const float total = __fadd_rn(__fmul_rn(s0, exp_ex2(__fsub_rn(m0, mx))),
                                    __fmul_rn(s1, exp_ex2(__fsub_rn(m1, mx))));
      const float inv = __frcp_rn(total);
      const float f = m == -INFINITY ? __fmul_rn(0.0f, inv) : __fmul_rn(exp_ex2(__fsub_rn(m, mx)), inv);
#pragma unroll
      for (int i = 0; i < E; ++i) v[i] = __fmul_rn(v[i], f);
    } else {
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < E; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
      ss = B::sum(ss, smem);
      const float4 other = exchange(ss, 0.0f, 0.0f);
      const float total = rank == 0 ? __fadd_rn(ss, other.x) : __fadd_rn(other.x, ss);
      const float scale =
          __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(n)), eps)));
#pragma unroll
      for (int i = 0; i < E; ++i) v[i] = __fmul_rn(v[i], scale);
    }
    float* orow = out + row * n + col0;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int i4 = tid + j * THREADS;
      if (i4 < h4) {
        float4 t = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        if (w || b) {
          const int64_t c = col0 + 4LL * i4;
          t.x = affine(t.x, w, b, c + 0); t.y = affine(t.y, w, b, c + 1);
          t.z = affine(t.z, w, b, c + 2); t.w = affine(t.w, w, b, c + 3);
        }
        __stcs(reinterpret_cast<float4*>(orow) + i4, t);
      }
    }
  }
  ptx::cluster_sync_all();  // neither CTA leaves while the other may still write its inbox
}

template <int OP>
int launch_pair_row(cudaStream_t s, const float* x, float* out, int64_t rows, int64_t n, float eps,
                    const float* w, const float* b) {
  constexpr int kStageBytes = 4 * 16384;
  static int clusters_fit[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(1024);
  cfg.dynamicSmemBytes = static_cast<size_t>(n / 2) * 4;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (dev < 0 || dev >= 64) dev = 0;
  if (clusters_fit[dev] == 0) {
    if (cudaFuncSetAttribute(row_pair_kernel<OP>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStageBytes) !=
        cudaSuccess)
      return launch_status("paired row smem attribute");
    // how many clusters are co-resident: the persistent grid never exceeds one wave
    cudaLaunchConfig_t probe = cfg;
    probe.dynamicSmemBytes = kStageBytes;
    probe.gridDim = dim3(2 * (sm_count() / 2));
    int fit = 0;
    if (cudaOccupancyMaxActiveClusters(&fit, row_pair_kernel<OP>, &probe) != cudaSuccess || fit < 1)
      return launch_status("paired row occupancy");
    clusters_fit[dev] = fit;
  }
  const int clusters = static_cast<int>(std::min<int64_t>(rows, clusters_fit[dev]));
  cfg.gridDim = dim3(2 * clusters);
  TimedLaunch timer("row_pair", s);
  cudaLaunchKernelEx(&cfg, row_pair_kernel<OP>, x, out, rows, n, eps, w, b, device_error_word());
  return launch_status("paired row op");
}

// Rows longer than the register-resident limit: CTA per row, streaming passes.
template <int OP>
__global__ void __launch_bounds__(1024)
row_stream(const float* __restrict__ x, float* __restrict__ out, int64_t rows, int64_t n,
           float eps, const float* __restrict__ w, const float* __restrict__ b) {
  using B = Block<1024>;
  __shared__ float smem[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * n;
    float* orow = out + row * n;
    if (OP == kSoftmax) {
      float m = -INFINITY;
      for (int64_t i = threadIdx.x; i < n; i += 1024) m = nan_max(m, xr[i]);
      m = B::max(m, smem);
      float s = 0.0f;
      for (int64_t i = threadIdx.x; i < n; i += 1024) s = __fadd_rn(s, exp_ex2(__fsub_rn(xr[i], m)));
      s = B::sum(s, smem);
      const float inv = __frcp_rn(s);
      for (int64_t i = threadIdx.x; i < n; i += 1024) orow[i] = __fmul_rn(exp_ex2(__fsub_rn(xr[i], m)), inv);
    } else if (OP == kRms) {
      float ss = 0.0f;
      for (int64_t i = threadIdx.x; i < n; i += 1024) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
      ss = B::sum(ss, smem);
      const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(n)), eps)));
      for (int64_t i = threadIdx.x; i < n; i += 1024) orow[i] = affine(__fmul_rn(xr[i], scale), w, b, i);
    } else {
      const float first = xr[0];
      float s = 0.0f;
      bool eq = true;
      for (int64_t i = threadIdx.x; i < n; i += 1024) { s = __fadd_rn(s, xr[i]); eq = eq && xr[i] == first; }
      s = B::sum(s, smem);
      eq = B::all(eq, smem);
      if (eq && isfinite(first)) {
        const float value = eps == 0.0f ? __int_as_float(0x7fc00000) : 0.0f;
        for (int64_t i = threadIdx.x; i < n; i += 1024) orow[i] = affine(value, w, b, i);
        continue;
      }
      const float mean = __fdiv_rn(s, static_cast<float>(n));
      float ssd = 0.0f;
      for (int64_t i = threadIdx.x; i < n; i += 1024) {
        const float d = __fsub_rn(xr[i], mean);
        ssd = __fadd_rn(ssd, __fmul_rn(d, d));
      }
      ssd = B::sum(ssd, smem);
      const float denom = __fadd_rn(__fdiv_rn(ssd, static_cast<float>(n)), eps);
      const float scale = denom == 0.0f ? __int_as_float(0x7fc00000) : __fdiv_rn(1.0f, __fsqrt_rn(denom));
      for (int64_t i = threadIdx.x; i < n; i += 1024)
        orow[i] = affine(denom == 0.0f ? scale : __fmul_rn(__fsub_rn(xr[i], mean), scale), w, b, i);
    }
  }
}

// Strided axis: one thread per (outer, inner) column, the reference's sequential order.
template <int OP>
__global__ void row_strided(const float* __restrict__ x, float* __restrict__ out, int64_t outer,
                            int64_t reduce, int64_t inner, float eps, const float* __restrict__ w,
                            const float* __restrict__ b) {
  const int64_t count = outer * inner;
  for (int64_t id = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; id < count;
       id += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t base = (id / inner) * reduce * inner + id % inner;
    if (OP == kSoftmax) {
      float m = -INFINITY;
      for (int64_t r = 0; r < reduce; ++r) {
        const float v = x[base + r * inner];
        if (isnan(v)) { m = v; break; }
        m = m < v ? v : m;
      }
      float d = 0.0f;
      for (int64_t r = 0; r < reduce; ++r) d = __fadd_rn(d, expf(__fsub_rn(x[base + r * inner], m)));
      for (int64_t r = 0; r < reduce; ++r) {
        const int64_t i = base + r * inner;
        out[i] = __fdiv_rn(expf(__fsub_rn(x[i], m)), d);
      }
    } else if (OP == kRms) {
      float ss = 0.0f;
      for (int64_t r = 0; r < reduce; ++r) {
        const float v = x[base + r * inner];
        ss = __fadd_rn(ss, __fmul_rn(v, v));
      }
      const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(reduce)), eps)));
      for (int64_t r = 0; r < reduce; ++r) {
        const int64_t i = base + r * inner;
        out[i] = affine(__fmul_rn(x[i], scale), w, b, r);
      }
    } else {
      float s = 0.0f;
      const float first = x[base];
      bool eq = true;
      for (int64_t r = 0; r < reduce; ++r) {
        const float v = x[base + r * inner];
        s = __fadd_rn(s, v);
        eq = eq && v == first;
      }
      if (eq && isfinite(first)) {
        const float value = eps == 0.0f ? __int_as_float(0x7fc00000) : 0.0f;
        for (int64_t r = 0; r < reduce; ++r) out[base + r * inner] = affine(value, w, b, r);
        continue;
      }
      const float mean = __fdiv_rn(s, static_cast<float>(reduce));
      float ssd = 0.0f;
      for (int64_t r = 0; r < reduce; ++r) {
        const float d = __fsub_rn(x[base + r * inner], mean);
        ssd = __fadd_rn(ssd, __fmul_rn(d, d));
      }
      const float denom = __fadd_rn(__fdiv_rn(ssd, static_cast<float>(reduce)), eps);
      if (denom == 0.0f) {
        for (int64_t r = 0; r < reduce; ++r) out[base + r * inner] = affine(__int_as_float(0x7fc00000), w, b, r);
        continue;
      }
      const float scale = __fdiv_rn(1.0f, __fsqrt_rn(denom));
      for (int64_t r = 0; r < reduce; ++r) {
        const int64_t i = base + r * inner;
        out[i] = affine(__fmul_rn(__fsub_rn(x[i], mean), scale), w, b, r);
      }
    }
  }
}

template <int OP, int THREADS, int VPT>
void launch_row(cudaStream_t s, const float* x, float* out, int64_t rows, int64_t n, float eps,
                const float* w, const float* b, bool vec) {
  const int grid = static_cast<int>(std::min<int64_t>(rows, 1LL << 20));
  TimedLaunch timer("row_kernel", s);
  if (vec && n == static_cast<int64_t>(THREADS) * VPT * 4)
    row_kernel<OP, THREADS, VPT, true, true><<<grid, THREADS, 0, s>>>(x, out, rows, n, eps, w, b);
  else if (vec) row_kernel<OP, THREADS, VPT, true><<<grid, THREADS, 0, s>>>(x, out, rows, n, eps, w, b);
  else row_kernel<OP, THREADS, VPT, false><<<grid, THREADS, 0, s>>>(x, out, rows, n, eps, w, b);
}

template <int OP>
int run_rows(cudaStream_t s, const float* x, float* out, int64_t outer, int64_t reduce,
             int64_t inner, float eps, const float* w, const float* b) {
  if (outer * inner == 0 || reduce == 0) return TCX_OK;
  if (inner != 1) {
    const int64_t count = outer * inner;
    const int grid = static_cast<int>(std::min<int64_t>(ceil_div(count, 256), 32LL * sm_count()));
    {
      TimedLaunch timer("row_strided", s);
      row_strided<OP><<<grid, 256, 0, s>>>(x, out, outer, reduce, inner, eps, w, b);
    }
    return launch_status("strided row op");
  }
  const int64_t n = reduce;
  const bool vec = n % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0;
  // Few threads per row, many values per thread: a warp (or two) per row needs no CTA
  // barrier, or one, per statistic, and 10-16 rows stay in flight per SM.
  if (n <= 1024) {
    launch_row<OP, 32, 8>(s, x, out, outer, n, eps, w, b, vec);
  } else if (n <= 2048) {
    launch_row<OP, 32, 16>(s, x, out, outer, n, eps, w, b, vec);
  } else if (n <= 4096) {
    launch_row<OP, 64, 16>(s, x, out, outer, n, eps, w, b, vec);
  } else if (n <= 8192) {
    launch_row<OP, 128, 16>(s, x, out, outer, n, eps, w, b, vec);
  } else if (n <= 32768) {
    if constexpr (OP != kLayer) {
      if (n <= 16384) {
        launch_row<OP, 256, 16>(s, x, out, outer, n, eps, w, b, vec);
        return launch_status("row op");
      }
      if (vec && n % 8 == 0) return launch_pair_row<OP>(s, x, out, outer, n, eps, w, b);
      if (vec) return launch_staged_row<OP, 8>(s, x, out, outer, n, eps, w, b);
    } else {
      // layernorm's deviation pass runs out of registers at 64 values per thread in
      // 256-thread rows, and its second statistic would cost the paired kernel a second
      // exchange per row: it streams through the staged kernel
      if (vec && n <= 16384) return launch_staged_row<OP, 4>(s, x, out, outer, n, eps, w, b);
      if (vec) return launch_staged_row<OP, 8>(s, x, out, outer, n, eps, w, b);
      if (n <= 16384) {
        launch_row<OP, 512, 8>(s, x, out, outer, n, eps, w, b, vec);
        return launch_status("row op");
      }
    }
    launch_row<OP, 1024, 8>(s, x, out, outer, n, eps, w, b, vec);
  } else {
    const int grid = static_cast<int>(std::min<int64_t>(outer, 1LL << 20));
    TimedLaunch timer("row_stream", s);
    row_stream<OP><<<grid, 1024, 0, s>>>(x, out, outer, n, eps, w, b);
  }
  return launch_status("row op");
}

int rows_dispatch(cudaStream_t s, int op, const float* x, float* out, int64_t outer,
                  int64_t reduce, int64_t inner, float eps, const float* w, const float* b) {
  switch (op) {
    case TCX_OP_SOFTMAX: return run_rows<kSoftmax>(s, x, out, outer, reduce, inner, eps, w, b);
    case TCX_OP_RMSNORM: return run_rows<kRms>(s, x, out, outer, reduce, inner, eps, w, b);
    default: return run_rows<kLayer>(s, x, out, outer, reduce, inner, eps, w, b);
  }
}

bool valid_dims(int64_t outer, int64_t reduce, int64_t inner) {
  return outer >= 0 && reduce >= 0 && inner >= 0;
}

}  // namespace
}  // namespace tcx

using namespace tcx;

extern "C" {

size_t tcx_sm100_axis_workspace_bytes(int op, int64_t outer, int64_t reduce, int64_t inner) {
  if (op != TCX_OP_SUM && op != TCX_OP_MAX && op != TCX_OP_MEAN) return 0;
  return axis_reduce_workspace(outer, reduce, inner);
}

int tcx_sm100_axis(tcx_stream_t stream, int op, int dtype, const void* input, void* output,
                   int64_t outer, int64_t reduce, int64_t inner, float epsilon, void* workspace,
                   size_t workspace_bytes) {
  clear_error();
  if (!valid_dims(outer, reduce, inner)) return invalid("negative axis extents");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (op) {
    case TCX_OP_SUM:
    case TCX_OP_MAX:
      if (dtype != TCX_FLOAT32 && dtype != TCX_INT32) return invalid("CUDA operations only support float32");
      if (op == TCX_OP_MAX && reduce == 0) return invalid("max reduction requires a non-empty axis");
      return axis_reduce(s, op, dtype, input, output, outer, reduce, inner, workspace, workspace_bytes);
    case TCX_OP_MEAN:
      if (dtype != TCX_FLOAT32) return invalid("mean only supports float32 tensors");
      return axis_reduce(s, op, dtype, input, output, outer, reduce, inner, workspace, workspace_bytes);
    case TCX_OP_SOFTMAX:
    case TCX_OP_RMSNORM:
    case TCX_OP_LAYERNORM:
      if (dtype != TCX_FLOAT32) return invalid("CUDA operation only supports float32 for this dtype");
      if (!(epsilon >= 0.0f) || isinf(epsilon)) return invalid("epsilon must be finite and non-negative and representable as float32");
      return rows_dispatch(s, op, static_cast<const float*>(input), static_cast<float*>(output), outer,
                           reduce, inner, epsilon, nullptr, nullptr);
    default:
      return invalid("unsupported axis operation");
  }
}

int tcx_sm100_affine_norm(tcx_stream_t stream, int op, const float* input, float* output,
                          int64_t outer, int64_t reduce, int64_t inner, float epsilon,
                          const float* weight, const float* bias) {
  clear_error();
  if (!valid_dims(outer, reduce, inner)) return invalid("negative axis extents");
  if (op != TCX_OP_RMSNORM && op != TCX_OP_LAYERNORM) return invalid("affine norm supports rmsnorm and layernorm");
  if (op == TCX_OP_RMSNORM && bias) return invalid("invalid affine normalization parameters");
  if (!(epsilon >= 0.0f) || isinf(epsilon)) return invalid("epsilon must be finite, non-negative and representable as float32");
  return rows_dispatch(reinterpret_cast<cudaStream_t>(stream), op, input, output, outer, reduce, inner,
                       epsilon, weight, bias);
}

}  // extern "C"
