// Attention on sm_100a: the masked, scaled row softmax primitive (kAttentionSoftmax)
// and the scaled dot-product attention composite (kAttention) built from it and the
// tcgen05 3xTF32 GEMM.
//
// Semantics follow the reference CPU backend (cpu_inference.cpp:22-45) and plan
// (core/inference.cpp:56-83): for row r of the [batch..., queries, keys] scores and
// column c,
//   score = -inf                      if causal and c > r % queries,
//         = -inf                      if a bool mask is false there,
//         = -inf                      if a float mask is -inf there,
//         = scores * scale + mask     otherwise (one float32 multiply, then one add);
// a row whose maximum is -inf (everything masked, or no keys) is all zeros; a NaN
// anywhere makes the row NaN; otherwise exp(score - max) / sum. Scores and mask are
// read through broadcast strides; the last-axis stride is 0 or 1, so each row is a
// base offset plus a column stride, computed once per row.
//
// The composite (core/inference.cpp:123-160) is three stream-ordered launches with no
// transpose copy and no metadata upload: S = Q·Kᵀ with K read K-major by the GEMM
// (keys are already [keys, features]), the softmax in place on S, then O = P·V.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "rowmath.cuh"

namespace tcx {
namespace {

using rowmath::Block;
using rowmath::exp_ex2;
using rowmath::nan_max;

constexpr int kAttnMaxRank = 32;

struct AttnMeta {
  int32_t rank;                       // rank of the [batch..., queries, keys] target
  int32_t narrow;                     // every row index fits 32 bits
  int64_t shape[kAttnMaxRank];
  int64_t s_stride[kAttnMaxRank];     // broadcast strides of the scores
  int64_t m_stride[kAttnMaxRank];     // broadcast strides of the mask (0 without one)
};

struct RowBase {
  int64_t s, m, query;
};

// Offsets of row `row` (an index over [batch..., queries]); 32-bit index arithmetic
// when the row count allows it (meta.narrow), as a 64-bit divide costs ~70 instructions.
__device__ __forceinline__ RowBase row_base(const AttnMeta& meta, int64_t row) {
  RowBase b{0, 0, 0};
  if (meta.narrow) {
    uint32_t i = static_cast<uint32_t>(row);
    for (int a = meta.rank - 2; a >= 0; --a) {
      const uint32_t e = static_cast<uint32_t>(meta.shape[a]);
      const uint32_t idx = i % e;
      i /= e;
      b.s += idx * meta.s_stride[a];
      b.m += idx * meta.m_stride[a];
      if (a == meta.rank - 2) b.query = idx;
    }
    return b;
  }
  int64_t i = row;
  for (int a = meta.rank - 2; a >= 0; --a) {
    const int64_t e = meta.shape[a];
    const int64_t idx = i % e;
    i /= e;
    b.s += idx * meta.s_stride[a];
    b.m += idx * meta.m_stride[a];
    if (a == meta.rank - 2) b.query = idx;
  }
  return b;
}

// Merges neighbouring batch axes (never the query or key axis) whose score and mask
// strides are both contiguous across them, drops extent-1 batch axes, and marks the
// metadata narrow when every row index fits 32 bits.
void collapse_rows(AttnMeta& meta) {
  const int r = meta.rank;
  AttnMeta c{};
  int n = 0;
  for (int a = 0; a < r - 2; ++a) {
    if (meta.shape[a] == 1) continue;
    if (n > 0 && c.s_stride[n - 1] == meta.s_stride[a] * meta.shape[a] &&
        c.m_stride[n - 1] == meta.m_stride[a] * meta.shape[a]) {
      c.shape[n - 1] *= meta.shape[a];
      c.s_stride[n - 1] = meta.s_stride[a];
      c.m_stride[n - 1] = meta.m_stride[a];
      continue;
    }
    c.shape[n] = meta.shape[a];
    c.s_stride[n] = meta.s_stride[a];
    c.m_stride[n] = meta.m_stride[a];
    ++n;
  }
  for (int a = r - 2; a < r; ++a, ++n) {
    c.shape[n] = meta.shape[a];
    c.s_stride[n] = meta.s_stride[a];
    c.m_stride[n] = meta.m_stride[a];
  }
  c.rank = n;
  int64_t rows = 1;
  for (int a = 0; a < n - 1; ++a) rows *= c.shape[a];
  c.narrow = rows <= static_cast<int64_t>(UINT32_MAX);
  meta = c;
}

struct Scorer {
  const float* s;
  const void* mask;
  int kind;      // 0 none, 1 bool (one byte, nonzero = allowed), 2 float32 additive
  int causal;
  float scale;
  int64_t cs, ms;  // last-axis strides (0 or 1)

  __device__ __forceinline__ float operator()(const RowBase& b, int64_t col) const {
    if (causal && col > b.query) return -INFINITY;
    float bias = 0.0f;
    if (kind == 1) {
      if (!static_cast<const unsigned char*>(mask)[b.m + col * ms]) return -INFINITY;
    } else if (kind == 2) {
      bias = static_cast<const float*>(mask)[b.m + col * ms];
      if (bias == -INFINITY) return bias;
    }
    return __fadd_rn(__fmul_rn(s[b.s + col * cs], scale), bias);
  }
};

// One CTA per row, the row's scores in registers (cols <= THREADS * VPT).
template <int THREADS, int VPT>
__global__ void __launch_bounds__(THREADS)
attention_softmax_rows(Scorer sc, float* out, AttnMeta meta, int64_t rows, int64_t cols) {
  __shared__ float smem[64];
  using B = Block<THREADS>;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const RowBase base = row_base(meta, row);
    float v[VPT];
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int64_t c = threadIdx.x + static_cast<int64_t>(q) * THREADS;
      v[q] = c < cols ? sc(base, c) : -INFINITY;
      m = nan_max(m, v[q]);
    }
    m = B::max(m, smem);
    float* orow = out + row * cols;
    if (m == -INFINITY) {  // the whole row is masked: zeros (uniform across the CTA)
#pragma unroll
      for (int q = 0; q < VPT; ++q) {
        const int64_t c = threadIdx.x + static_cast<int64_t>(q) * THREADS;
        if (c < cols) orow[c] = 0.0f;
      }
      continue;
    }
    float total = 0.0f;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int64_t c = threadIdx.x + static_cast<int64_t>(q) * THREADS;
      v[q] = c < cols ? exp_ex2(__fsub_rn(v[q], m)) : 0.0f;
      total = __fadd_rn(total, v[q]);
    }
    total = B::sum(total, smem);
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int64_t c = threadIdx.x + static_cast<int64_t>(q) * THREADS;
      if (c < cols) orow[c] = __fdiv_rn(v[q], total);
    }
  }
}

// Contiguous rows (score column stride 1, rows 16-byte aligned, cols % 4 == 0), the
// layout of every composite call: float4 score loads, mask loads of 4 entries (KIND 1:
// 4 bytes, KIND 2: a float4) when the mask varies along the row (MCOL), one value per
// row otherwise; 32-bit column arithmetic. TPR threads share a row: 32 (a warp per
// row, shuffles only, no barriers) for rows up to 2048, the whole CTA beyond. Same
// math as attention_softmax_rows except that the final division is a multiply by one
// correctly rounded reciprocal per row (<= 1.5 ulp from the quotient).
template <int TPR, int THREADS>
struct RowReduce {
  __device__ static float max(float v, float* smem) {
    if constexpr (TPR == 32) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v = nan_max(v, __shfl_xor_sync(0xffffffffu, v, off));
      return v;
    } else {
      return Block<THREADS>::max(v, smem);
    }
  }
  __device__ static float sum(float v, float* smem) {
    if constexpr (TPR == 32) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
      return v;
    } else {
      return Block<THREADS>::sum(v, smem);
    }
  }
};

// The mask entries of one float4 group of scores, loaded beside the scores.
template <int KIND>
struct MaskGroup;
template <>
struct MaskGroup<0> {
  __device__ void load(const Scorer&, const RowBase&, int32_t, bool) {}
  __device__ bool keep(int) const { return true; }
  __device__ float bias(int) const { return 0.0f; }
};
template <>
struct MaskGroup<1> {
  uchar4 b;
  __device__ void load(const Scorer& sc, const RowBase& base, int32_t i4, bool mcol) {
    const unsigned char* m = static_cast<const unsigned char*>(sc.mask) + base.m;
    if (mcol) {
      b = reinterpret_cast<const uchar4*>(m)[i4];
    } else {
      const unsigned char k = *m;
      b = make_uchar4(k, k, k, k);
    }
  }
  __device__ bool keep(int e) const { return (e == 0 ? b.x : e == 1 ? b.y : e == 2 ? b.z : b.w) != 0; }
  __device__ float bias(int) const { return 0.0f; }
};
template <>
struct MaskGroup<2> {
  float4 f;
  __device__ void load(const Scorer& sc, const RowBase& base, int32_t i4, bool mcol) {
    const float* m = static_cast<const float*>(sc.mask) + base.m;
    if (mcol) {
      f = reinterpret_cast<const float4*>(m)[i4];
    } else {
      const float k = *m;
      f = make_float4(k, k, k, k);
    }
  }
  __device__ bool keep(int) const { return true; }
  __device__ float bias(int e) const { return e == 0 ? f.x : e == 1 ? f.y : e == 2 ? f.z : f.w; }
};

template <int TPR, int THREADS, int VPT, int KIND, bool MCOL>
__global__ void __launch_bounds__(THREADS)
attention_softmax_vec(Scorer sc, float* out, AttnMeta meta, int64_t rows, int32_t cols) {
  __shared__ float smem[64];
  using R = RowReduce<TPR, THREADS>;
  constexpr int E = 4 * VPT;
  constexpr int kRowsPerCta = THREADS / TPR;
  const int32_t n4 = cols >> 2;
  const int lane = threadIdx.x % TPR;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerCta + threadIdx.x / TPR; row < rows;
       row += static_cast<int64_t>(gridDim.x) * kRowsPerCta) {
    const RowBase base = row_base(meta, row);
    const float4* srow = reinterpret_cast<const float4*>(sc.s + base.s);
    // all loads first (predicated, no branches), then the arithmetic
    float4 t[VPT];
    MaskGroup<KIND> mk[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int32_t i4 = lane + j * TPR;
      const bool in = i4 < n4;
      t[j] = in ? srow[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
      if (in) mk[j].load(sc, base, i4, MCOL);
    }
    // causal limit as a 32-bit column bound (columns are < 2^31)
    const int32_t last = sc.causal ? static_cast<int32_t>(base.query < INT32_MAX ? base.query : INT32_MAX) : INT32_MAX;
    float v[E];
    float m = -INFINITY;
    bool nan = false;  // fmaxf drops NaN: track it apart, the row becomes NaN anyway
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int32_t i4 = lane + j * TPR;
      const float raw[4] = {t[j].x, t[j].y, t[j].z, t[j].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int32_t c = 4 * i4 + e;
        const float bias = mk[j].bias(e);
        const bool masked = i4 >= n4 || c > last || !mk[j].keep(e) || (KIND == 2 && bias == -INFINITY);
        const float x = masked ? -INFINITY : __fadd_rn(__fmul_rn(raw[e], sc.scale), bias);
        v[4 * j + e] = x;
        m = fmaxf(m, x);
        nan |= x != x;
      }
    }
    if (nan) m = __int_as_float(0x7fc00000);
    m = R::max(m, smem);
    float4* orow = reinterpret_cast<float4*>(out + row * static_cast<int64_t>(cols));
    if (m == -INFINITY) {  // uniform across the row's threads
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int32_t i4 = lane + j * TPR;
        if (i4 < n4) orow[i4] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      continue;
    }
    float total = 0.0f;
#pragma unroll
    for (int q = 0; q < E; ++q) {
      v[q] = exp_ex2(__fsub_rn(v[q], m));  // -inf slots (masked, padding) give +0
      total = __fadd_rn(total, v[q]);
    }
    total = R::sum(total, smem);
    const float inv = __frcp_rn(total);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int32_t i4 = lane + j * TPR;
      if (i4 < n4)
        orow[i4] = make_float4(__fmul_rn(v[4 * j], inv), __fmul_rn(v[4 * j + 1], inv), __fmul_rn(v[4 * j + 2], inv),
                               __fmul_rn(v[4 * j + 3], inv));
    }
  }
}

// Rows longer than the register path: three passes over the row (max, sum, write),
// the second and third served from L2 for rows up to a few MB.
template <int THREADS>
__global__ void __launch_bounds__(THREADS)
attention_softmax_stream(Scorer sc, float* out, AttnMeta meta, int64_t rows, int64_t cols) {
  __shared__ float smem[64];
  using B = Block<THREADS>;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const RowBase base = row_base(meta, row);
    float m = -INFINITY;
    for (int64_t c = threadIdx.x; c < cols; c += THREADS) m = nan_max(m, sc(base, c));
    m = B::max(m, smem);
    float* orow = out + row * cols;
    if (m == -INFINITY) {
      for (int64_t c = threadIdx.x; c < cols; c += THREADS) orow[c] = 0.0f;
      continue;
    }
    float total = 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += THREADS) total = __fadd_rn(total, exp_ex2(__fsub_rn(sc(base, c), m)));
    total = B::sum(total, smem);
    __syncthreads();  // in-place use: every thread has read the row before any write
    for (int64_t c = threadIdx.x; c < cols; c += THREADS) orow[c] = __fdiv_rn(exp_ex2(__fsub_rn(sc(base, c), m)), total);
  }
}

template <int THREADS, int VPT>
void launch_rows(cudaStream_t s, const Scorer& sc, float* out, const AttnMeta& meta, int64_t rows, int64_t cols) {
  const int per_sm = std::max(1, 2048 / THREADS);
  const int grid = static_cast<int>(std::min<int64_t>(rows, static_cast<int64_t>(sm_count()) * per_sm));
  attention_softmax_rows<THREADS, VPT><<<grid, THREADS, 0, s>>>(sc, out, meta, rows, cols);
}

template <int TPR, int THREADS, int VPT>
void launch_vec(cudaStream_t s, const Scorer& sc, float* out, const AttnMeta& meta, int64_t rows, int64_t cols) {
  const int per_sm = std::max(1, 2048 / THREADS);
  const int64_t ctas = ceil_div(rows, THREADS / TPR);
  const int grid = static_cast<int>(std::min<int64_t>(ctas, static_cast<int64_t>(sm_count()) * per_sm));
  const int32_t c = static_cast<int32_t>(cols);
  const bool mcol = sc.ms == 1;
  if (sc.kind == 0)
    attention_softmax_vec<TPR, THREADS, VPT, 0, false><<<grid, THREADS, 0, s>>>(sc, out, meta, rows, c);
  else if (sc.kind == 1 && mcol)
    attention_softmax_vec<TPR, THREADS, VPT, 1, true><<<grid, THREADS, 0, s>>>(sc, out, meta, rows, c);
  else if (sc.kind == 1)
    attention_softmax_vec<TPR, THREADS, VPT, 1, false><<<grid, THREADS, 0, s>>>(sc, out, meta, rows, c);
  else if (mcol)
    attention_softmax_vec<TPR, THREADS, VPT, 2, true><<<grid, THREADS, 0, s>>>(sc, out, meta, rows, c);
  else
    attention_softmax_vec<TPR, THREADS, VPT, 2, false><<<grid, THREADS, 0, s>>>(sc, out, meta, rows, c);
}

// Every row base (scores and mask) a multiple of 4 elements and 16-byte aligned, the
// scores contiguous along the row: what the vector kernel needs.
bool vec_rows(const float* scores, const void* mask, int kind, const float* out, const AttnMeta& meta,
              int64_t cols) {
  const int r = meta.rank;
  if (cols % 4 || cols > INT32_MAX || meta.s_stride[r - 1] != 1) return false;
  if (reinterpret_cast<uintptr_t>(scores) % 16 || reinterpret_cast<uintptr_t>(out) % 16) return false;
  if (kind && meta.m_stride[r - 1] == 1 && reinterpret_cast<uintptr_t>(mask) % 16) return false;
  for (int a = 0; a < r - 1; ++a) {
    if (meta.s_stride[a] % 4) return false;
    if (kind && meta.m_stride[r - 1] == 1 && meta.m_stride[a] % 4) return false;
  }
  return true;
}

int attention_softmax(cudaStream_t s, const float* scores, const void* mask, int kind, float* out,
                      const AttnMeta& meta_in, int64_t rows, int64_t cols, float scale, int causal) {
  if (rows == 0 || cols == 0) return TCX_OK;
  AttnMeta meta = meta_in;
  collapse_rows(meta);
  Scorer sc{scores, mask, kind, causal, scale, meta.s_stride[meta.rank - 1], meta.m_stride[meta.rank - 1]};
  TimedLaunch timer("attention_softmax", s);
  if (vec_rows(scores, mask, kind, out, meta, cols) && cols <= 8192) {
    // 4 to 16 values per thread: more per thread and the compiler trades load
    // batching for registers (serialized row loads)
    if (cols <= 128) launch_vec<32, 256, 1>(s, sc, out, meta, rows, cols);
    else if (cols <= 256) launch_vec<32, 256, 2>(s, sc, out, meta, rows, cols);
    else if (cols <= 512) launch_vec<32, 256, 4>(s, sc, out, meta, rows, cols);
    else if (cols <= 1024) launch_vec<64, 64, 4>(s, sc, out, meta, rows, cols);
    else if (cols <= 2048) launch_vec<128, 128, 4>(s, sc, out, meta, rows, cols);
    else if (cols <= 4096) launch_vec<256, 256, 4>(s, sc, out, meta, rows, cols);
    else launch_vec<512, 512, 4>(s, sc, out, meta, rows, cols);
    return launch_status("attention softmax");
  }
  if (cols <= 128) launch_rows<128, 1>(s, sc, out, meta, rows, cols);
  else if (cols <= 512) launch_rows<128, 4>(s, sc, out, meta, rows, cols);
  else if (cols <= 1024) launch_rows<256, 4>(s, sc, out, meta, rows, cols);
  else if (cols <= 2048) launch_rows<512, 4>(s, sc, out, meta, rows, cols);
  else if (cols <= 4096) launch_rows<512, 8>(s, sc, out, meta, rows, cols);
  else if (cols <= 8192) launch_rows<1024, 8>(s, sc, out, meta, rows, cols);
  else {
    const int grid = static_cast<int>(std::min<int64_t>(rows, static_cast<int64_t>(sm_count()) * 2));
    attention_softmax_stream<1024><<<grid, 1024, 0, s>>>(sc, out, meta, rows, cols);
  }
  return launch_status("attention softmax");
}

// Checked product of non-negative extents; -1 on a negative extent or overflow.
int64_t checked_numel(const int64_t* dims, int rank) {
  for (int a = 0; a < rank; ++a)
    if (dims[a] == 0) return 0;  // an empty axis leaves the rest unvisited
  int64_t n = 1;
  for (int a = 0; a < rank; ++a) {
    if (dims[a] < 0) return -1;
    if (dims[a] && n > INT64_MAX / dims[a]) return -1;
    n *= dims[a];
  }
  return n;
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace
}  // namespace tcx

using namespace tcx;

extern "C" {

int tcx_sm100_attention_softmax(tcx_stream_t stream, const float* scores, const void* mask, int32_t mask_kind,
                                float* output, const int64_t* shape, const int64_t* score_strides,
                                const int64_t* mask_strides, int32_t rank, float scale, int32_t causal) {
  clear_error();
  if (rank < 2 || rank > kAttnMaxRank) return invalid("attention scores must have rank 2..32");
  if (!shape || !score_strides) return invalid("missing attention metadata");
  if (mask_kind < 0 || mask_kind > 2) return invalid("attention mask must be bool or float32");
  if (mask_kind != 0 && !mask_strides) return invalid("missing attention mask strides");
  if (!std::isfinite(scale)) return invalid("attention scale must be finite and representable as float32");
  const int64_t count = checked_numel(shape, rank);
  if (count < 0) return invalid("attention shape overflows");
  AttnMeta meta{};
  meta.rank = rank;
  for (int a = 0; a < rank; ++a) {
    meta.shape[a] = shape[a];
    meta.s_stride[a] = score_strides[a];
    meta.m_stride[a] = mask_kind ? mask_strides[a] : 0;
    if (meta.s_stride[a] < 0 || meta.m_stride[a] < 0) return invalid("negative attention strides");
  }
  if (meta.s_stride[rank - 1] > 1 || meta.m_stride[rank - 1] > 1)
    return invalid("attention last-axis strides must be 0 or 1");
  const int64_t cols = shape[rank - 1];
  const int64_t rows = cols ? count / cols : 0;
  if (count && (!scores || !output || (mask_kind && !mask))) return invalid("missing attention buffer");
  return attention_softmax(reinterpret_cast<cudaStream_t>(stream), scores, mask, mask_kind, output, meta,
                           rows, cols, scale, causal != 0);
}

size_t tcx_sm100_attention_workspace_bytes(int64_t batches, int64_t queries, int64_t keys, int64_t features,
                                           int64_t value_features, int64_t q_batches, int64_t k_batches,
                                           int64_t v_batches, int32_t mask_kind) {
  if (batches < 0 || queries < 0 || keys < 0 || features < 0 || value_features < 0) return 0;
  if (flash_eligible(queries, keys, features, value_features, mask_kind, 0))
    return flash_workspace_bytes(queries, keys, features, value_features, q_batches, k_batches, v_batches, batches,
                                 mask_kind);
  const size_t scores = round_up(static_cast<size_t>(batches) * queries * keys * sizeof(float), 1024);
  const size_t g1 = tcx_sm100_matmul_workspace_bytes(queries, keys, features, q_batches, k_batches, TCX_MATMUL_AUTO);
  const size_t g2 = tcx_sm100_matmul_workspace_bytes(queries, value_features, keys, batches, v_batches,
                                                     TCX_MATMUL_AUTO);
  return scores + std::max(g1, g2);
}

int tcx_sm100_attention(tcx_stream_t stream, const float* q, const float* k, const float* v, const void* mask,
                        int32_t mask_kind, float* output, int64_t queries, int64_t keys, int64_t features,
                        int64_t value_features, const int64_t* batch_shape, const int64_t* q_batch_strides,
                        const int64_t* k_batch_strides, const int64_t* v_batch_strides, int32_t batch_rank,
                        const int64_t* mask_strides, float scale, int32_t causal, void* workspace,
                        size_t workspace_bytes) {
  clear_error();
  if (queries < 0 || keys < 0 || features <= 0 || value_features < 0)
    return invalid("attention query/key features and key/value sequence sizes must match; features must be positive");
  if (batch_rank < 0 || batch_rank + 2 > kAttnMaxRank) return invalid("attention batch rank exceeds 30");
  if (batch_rank > 0 && (!batch_shape || !q_batch_strides || !k_batch_strides || !v_batch_strides))
    return invalid("missing attention batch metadata");
  if (mask_kind < 0 || mask_kind > 2) return invalid("attention mask must be bool or float32");
  if (mask_kind != 0 && (!mask_strides)) return invalid("missing attention mask strides");
  if (!std::isfinite(scale)) return invalid("attention scale must be finite and representable as float32");
  const int64_t batches = checked_numel(batch_shape, batch_rank);
  if (batches < 0) return invalid("attention batch shape overflows");
  if (batches == 0 || queries == 0 || value_features == 0) return TCX_OK;
  if (!q || !output || (keys > 0 && (!k || !v || (mask_kind && !mask)))) return invalid("missing attention buffer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  // scores [batch..., queries, keys] at the front of the workspace, GEMM scratch after
  int64_t dims[kAttnMaxRank], cstr[kAttnMaxRank], pstr[kAttnMaxRank];
  const int rank = batch_rank + 2;
  for (int a = 0; a < batch_rank; ++a) dims[a] = batch_shape[a];
  dims[batch_rank] = queries;
  dims[batch_rank + 1] = keys;
  int64_t st = 1;
  for (int a = rank - 1; a >= 0; --a) {
    cstr[a] = st;
    st *= dims[a];
  }
  for (int a = 0; a < batch_rank; ++a) pstr[a] = cstr[a];
  int64_t qn = 1, kn = 1, vn = 1;  // distinct batches of each operand
  for (int a = 0; a < batch_rank; ++a) {
    if (q_batch_strides[a]) qn *= batch_shape[a];
    if (k_batch_strides[a]) kn *= batch_shape[a];
    if (v_batch_strides[a]) vn *= batch_shape[a];
  }
  if (flash_eligible(queries, keys, features, value_features, mask_kind, batch_rank) &&
      reinterpret_cast<uintptr_t>(output) % 16 == 0) {
    const size_t need = flash_workspace_bytes(queries, keys, features, value_features, qn, kn, vn, batches, mask_kind);
    if (!workspace || workspace_bytes < need) return invalid("attention workspace is missing or too small");
    if (reinterpret_cast<uintptr_t>(workspace) % 1024) return invalid("attention workspace must be 1024-byte aligned");
    return attention_fused(s, q, k, v, mask, mask_kind, mask_strides, output, queries, keys, features,
                           value_features, batches, batch_shape, q_batch_strides, k_batch_strides, v_batch_strides,
                           batch_rank, scale, causal != 0, workspace, workspace_bytes);
  }
  const size_t need = tcx_sm100_attention_workspace_bytes(batches, queries, keys, features, value_features, qn, kn, vn,
                                                          mask_kind);
  if (need && (!workspace || workspace_bytes < need)) return invalid("attention workspace is missing or too small");
  if (reinterpret_cast<uintptr_t>(workspace) % 1024) return invalid("attention workspace must be 1024-byte aligned");
  float* scores = static_cast<float*>(workspace);
  const size_t score_bytes = round_up(static_cast<size_t>(batches) * queries * keys * sizeof(float), 1024);
  uint8_t* gemm_ws = static_cast<uint8_t*>(workspace) + score_bytes;
  const size_t gemm_bytes = workspace_bytes - score_bytes;

  if (keys > 0) {
    if (int rc = matmul_run(s, q, k, scores, queries, keys, features, batches, batch_shape, q_batch_strides,
                            k_batch_strides, batch_rank, /*rhs_kmajor=*/true, gemm_ws, gemm_bytes))
      return rc;
    AttnMeta meta{};
    meta.rank = rank;
    for (int a = 0; a < rank; ++a) {
      meta.shape[a] = dims[a];
      meta.s_stride[a] = cstr[a];
      meta.m_stride[a] = mask_kind ? mask_strides[a] : 0;
      if (meta.m_stride[a] < 0) return invalid("negative attention strides");
    }
    if (meta.m_stride[rank - 1] > 1) return invalid("attention last-axis strides must be 0 or 1");
    if (int rc = attention_softmax(s, scores, mask, mask_kind, scores, meta, batches * queries, keys, scale,
                                   causal != 0))
      return rc;
  }
  // O = P·V (keys == 0 gives zeros: an empty contraction)
  return matmul_run(s, scores, v, output, queries, value_features, keys, batches, batch_shape, pstr,
                    v_batch_strides, batch_rank, /*rhs_kmajor=*/false, gemm_ws, gemm_bytes);
}

}  // extern "C"
