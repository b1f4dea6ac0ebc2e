// float32 matmul / batched matmul for sm_100a.
//
// Tensor-core path (3xTF32 on tcgen05):
//   1. Split pre-pass (HBM-bound): every operand element x becomes
//      hi = rna_tf32(x), lo = rna_tf32(x - hi), written K-major into the caller's
//      workspace ([plane][rows][Kp], planes hi/lo per operand batch, K padded with
//      zeros to a multiple of 32). B is transposed on the way, so both operands are
//      K-major. The pass also flags any inf/NaN input.
//      Raw mode (tcx_sm100_matmul and tcx_sm100_matmul_host with a row-major B, K and N
//      multiples of 4, 16-byte aligned operands): kind::tf32 reads fp32 words and drops
//      their low 13 mantissa bits (measured on sm_100a), so the operands themselves
//      are the hi terms, hi = trunc_tf32(x). The pre-pass (split_lo) then writes only
//      lo = rna_tf32(x - trunc_tf32(x)), elementwise in each operand's own layout:
//      8 B per element instead of 12, no transpose. The GEMM reads A K-major as
//      before and B MN-major: 32-column chunks of 32 k rows (4 KB TMA boxes with the
//      128-byte / 32-byte-atom swizzle, layout type 1 in the MMA descriptor; the plain
//      128-byte swizzle gives zeros for MN-major tf32 operands).
//   2. GEMM: a persistent, warp-specialized kernel, one CTA per SM:
//        warp 0      TMA producer: 4 tiles per k-block (A hi/lo 128x32, B hi/lo 256x32,
//                    128B-swizzled) into a 2-stage shared-memory ring (mbarriers);
//        warp 1      MMA issuer: per 8-wide k step, three tcgen05.mma.kind::tf32
//                    (lo*hi, hi*lo, hi*hi) into one float32 TMEM accumulator;
//                    tcgen05.commit releases the stage / publishes the accumulator;
//        warps 2-9   epilogue, two warps per SM sub-partition (a warp may read only
//                    its TMEM lane quarter; warps 2-5 take columns 0-127, 6-9 the
//                    rest): tcgen05.ld 32x32b with the next chunk's load in flight,
//                    bias + activation, and row-coalesced stores through a 4 KB
//                    shared-memory slice per warp. Two TMEM accumulators (2 x 256
//                    columns) let the epilogue of tile t overlap the main loop of t+1.
//      No TMA multicast anywhere (this code also runs in multi-GPU jobs).
//   3. If the pre-pass saw inf/NaN, the GEMM exits at once and the FFMA kernel
//      (launched behind it, idle otherwise) computes the product with IEEE
//      semantics: 3xTF32 cross terms would turn inf*0 into NaN.
// FFMA path: a 64x64x16 register-blocked SIMT kernel for skinny or small products.
//
// Every spin-wait is bounded (a few seconds of %globaltimer); on expiry the kernel
// records the site in the device error word, stops issuing, drains what it issued
// and frees its TMEM before returning.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "ptx.cuh"

namespace tcx {
namespace {

constexpr int kMaxBatchRank = 8;

struct BatchMap {
  int32_t rank;
  int64_t shape[kMaxBatchRank];
  int64_t lhs[kMaxBatchRank];  // element strides (plan strides)
  int64_t rhs[kMaxBatchRank];
};

__device__ __forceinline__ int64_t batch_off(int64_t b, const int64_t* shape, const int64_t* st, int rank) {
  int64_t off = 0;
  for (int a = rank - 1; a >= 0; --a) {
    off += (b % shape[a]) * st[a];
    b /= shape[a];
  }
  return off;
}

// PTX helpers (mbarriers, bounded waits, TMA, tcgen05): ptx.cuh
using namespace ptx;

__device__ __forceinline__ float silu_e(float v) { return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v))); }
__device__ __forceinline__ float relu_e(float v) {
  // clip(v, +0, +inf) of cpu_math.cpp:42-47: NaN kept, v <= 0 (incl. -0) -> +0
  return (v != v) ? v : (v > 0.0f ? v : 0.0f);
}
__device__ __forceinline__ float epilogue_op(float v, const float* bias, int64_t col, int act) {
  if (bias) v = __fadd_rn(v, __ldg(bias + col));
  if (act == TCX_ACT_SILU) v = silu_e(v);
  else if (act == TCX_ACT_RELU) v = relu_e(v);
  return v;
}

// ------------------------------------------------------------------- pre-pass

__device__ __forceinline__ void split_one(float x, float& hi, float& lo, bool& bad) {
  bad |= !isfinite(x);
  hi = tf32_rna(x);
  lo = tf32_rna(__fsub_rn(x, hi));
}

__device__ __forceinline__ float4 ldg_f4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}

// lo term of the raw mode: the tensor core takes x itself as hi (it drops the low 13
// mantissa bits), so lo = rna_tf32(x - trunc_tf32(x)); x - trunc_tf32(x) is exact.
__device__ __forceinline__ float lo_one(float x, bool& bad) {
  bad |= !isfinite(x);
  return tf32_rna(__fsub_rn(x, __uint_as_float(__float_as_uint(x) & 0xFFFFE000u)));
}

// Raw-mode pre-pass of both operands in one launch: A [na4 float4s] -> wa and
// B [nb4 float4s] -> wb elementwise, in place of layout (each operand's own); raises
// *nonfinite on inf / NaN. Both operands 16-byte aligned with element counts that are
// multiples of 4 (K % 4 == 0 and N % 4 == 0).
__global__ void __launch_bounds__(256)
split_lo(const float4* __restrict__ a, float4* __restrict__ wa, int64_t na4, const float4* __restrict__ b,
         float4* __restrict__ wb, int64_t nb4, int* __restrict__ nonfinite) {
  bool bad = false;
  const int64_t total = na4 + nb4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  // four independent 128-bit loads in flight per thread
  for (; i + 3 * stride < total; i += 4 * stride) {
    float4 x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t j = i + u * stride;
      x[u] = __ldg(j < na4 ? a + j : b + (j - na4));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t j = i + u * stride;
      const float4 l = make_float4(lo_one(x[u].x, bad), lo_one(x[u].y, bad), lo_one(x[u].z, bad), lo_one(x[u].w, bad));
      if (j < na4) wa[j] = l;
      else wb[j - na4] = l;
    }
  }
  for (; i < total; i += stride) {
    const float4 x = __ldg(i < na4 ? a + i : b + (i - na4));
    const float4 l = make_float4(lo_one(x.x, bad), lo_one(x.y, bad), lo_one(x.z, bad), lo_one(x.w, bad));
    if (i < na4) wa[i] = l;
    else wb[i - na4] = l;
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(nonfinite, 1);
  dependents_may_launch();  // the GEMM behind may start its set-up
}

// A [nb][rows][K] -> W [2*nb][rows][Kp] (plane 2b hi, 2b+1 lo), zero padded in K.
// A flat grid-stride walk over 4-wide K chunks of all rows; each thread issues 4
// independent 128-bit loads before converting (VEC: K % 4 == 0, 16-byte aligned A),
// so enough bytes are in flight per SM to run at HBM speed.
// The body runs as block `bid` of `nblk` (a kernel of its own, or part of split_pair).
template <bool VEC>
__device__ __forceinline__ void split_rows_body(const float* __restrict__ a, float* __restrict__ w, int64_t nb,
                                                int64_t rows, int64_t k, int64_t kp, int* __restrict__ nonfinite,
                                                int64_t bid, int64_t nblk) {
  constexpr int U = 4;
  const int64_t plane = rows * kp;
  const int64_t kq = kp >> 2;                // 4-wide chunks per row
  const int64_t total = nb * rows * kq;
  const int64_t stride = nblk * blockDim.x;
  bool bad = false;
  for (int64_t base = bid * static_cast<int64_t>(blockDim.x) + threadIdx.x; base < total;
       base += stride * U) {
    float4 x[U];
    int64_t row[U], c[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t q = base + u * stride;
      x[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      row[u] = q / kq;
      c[u] = (q - row[u] * kq) * 4;
      if (q < total) {
        const float* src = a + row[u] * k;
        if (VEC) {
          if (c[u] < k) x[u] = ldg_f4(src + c[u]);
        } else {
          if (c[u] + 0 < k) x[u].x = __ldg(src + c[u] + 0);
          if (c[u] + 1 < k) x[u].y = __ldg(src + c[u] + 1);
          if (c[u] + 2 < k) x[u].z = __ldg(src + c[u] + 2);
          if (c[u] + 3 < k) x[u].w = __ldg(src + c[u] + 3);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (base + u * stride >= total) continue;
      const int64_t b = row[u] / rows, r = row[u] - b * rows;
      float4 h, l;
      split_one(x[u].x, h.x, l.x, bad);
      split_one(x[u].y, h.y, l.y, bad);
      split_one(x[u].z, h.z, l.z, bad);
      split_one(x[u].w, h.w, l.w, bad);
      float* dhi = w + (2 * b) * plane + r * kp + c[u];
      *reinterpret_cast<float4*>(dhi) = h;
      *reinterpret_cast<float4*>(dhi + plane) = l;
    }
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(nonfinite, 1);
}

template <bool VEC>
__global__ void __launch_bounds__(256)
split_rows(const float* __restrict__ a, float* __restrict__ w, int64_t nb, int64_t rows, int64_t k,
           int64_t kp, int* __restrict__ nonfinite) {
  split_rows_body<VEC>(a, w, nb, rows, k, kp, nonfinite, blockIdx.x, gridDim.x);
  dependents_may_launch();
}

// B [nb][K][N] -> W [2*nb][N][Kp] (transposed to K-major, zero padded in K).
// A CTA moves a 32 (k) x 128 (n) tile: coalesced 128-bit loads along n (VEC: N % 4 == 0
// and 16-byte aligned B), scalar shared-memory transpose (pitch 129: conflict-free
// reads), 128-bit stores along k.
template <bool VEC>
__device__ __forceinline__ void split_cols_body(const float* __restrict__ bsrc, float* __restrict__ w, int64_t nb,
                                                int64_t k, int64_t n, int64_t kp, int* __restrict__ nonfinite,
                                                int64_t bid, int64_t nblk) {
  __shared__ float tile[32][129];
  const int64_t plane = n * kp;
  const int64_t tiles_n = (n + 127) / 128, tiles_k = kp / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  bool bad = false;
  for (int64_t t = bid; t < nb * tiles_n * tiles_k; t += nblk) {
    const int64_t b = t / (tiles_n * tiles_k), rem = t % (tiles_n * tiles_k);
    const int64_t n0 = (rem % tiles_n) * 128, k0 = (rem / tiles_n) * 32;
    const float* src = bsrc + b * k * n;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kk = warp * 4 + j;
      const int64_t gk = k0 + kk, gn = n0 + lane * 4;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (gk < k) {
        if (VEC) {
          if (gn < n) x = ldg_f4(src + gk * n + gn);
        } else {
          const float* p = src + gk * n + gn;
          if (gn + 0 < n) x.x = __ldg(p + 0);
          if (gn + 1 < n) x.y = __ldg(p + 1);
          if (gn + 2 < n) x.z = __ldg(p + 2);
          if (gn + 3 < n) x.w = __ldg(p + 3);
        }
      }
      tile[kk][lane * 4 + 0] = x.x;
      tile[kk][lane * 4 + 1] = x.y;
      tile[kk][lane * 4 + 2] = x.z;
      tile[kk][lane * 4 + 3] = x.w;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int nn = (threadIdx.x >> 3) + 32 * j;
      const int k4 = threadIdx.x & 7;
      const int64_t gn = n0 + nn;
      float4 h, l;
      split_one(tile[4 * k4 + 0][nn], h.x, l.x, bad);
      split_one(tile[4 * k4 + 1][nn], h.y, l.y, bad);
      split_one(tile[4 * k4 + 2][nn], h.z, l.z, bad);
      split_one(tile[4 * k4 + 3][nn], h.w, l.w, bad);
      if (gn < n) {
        float* dhi = w + (2 * b) * plane + gn * kp + k0 + 4 * k4;
        *reinterpret_cast<float4*>(dhi) = h;
        *reinterpret_cast<float4*>(dhi + plane) = l;
      }
    }
    __syncthreads();
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(nonfinite, 1);
}

template <bool VEC>
__global__ void __launch_bounds__(256)
split_cols(const float* __restrict__ bsrc, float* __restrict__ w, int64_t nb, int64_t k, int64_t n,
           int64_t kp, int* __restrict__ nonfinite) {
  split_cols_body<VEC>(bsrc, w, nb, k, n, kp, nonfinite, blockIdx.x, gridDim.x);
  dependents_may_launch();
}

// Both operands' pre-passes in one launch: blocks [0, ga) split A's rows, the others B
// (a row split when B is K-major, else the transposing split).
template <bool VA, bool BK, bool VB>
__global__ void __launch_bounds__(256)
split_pair(const float* __restrict__ a, float* __restrict__ wa, int64_t nba, int64_t m, const float* __restrict__ b,
           float* __restrict__ wb, int64_t nbb, int64_t n, int64_t k, int64_t kp, int* __restrict__ nonfinite,
           int ga) {
  if (static_cast<int>(blockIdx.x) < ga) {
    split_rows_body<VA>(a, wa, nba, m, k, kp, nonfinite, blockIdx.x, ga);
  } else if (BK) {
    split_rows_body<VB>(b, wb, nbb, n, k, kp, nonfinite, blockIdx.x - ga, gridDim.x - ga);
  } else {
    split_cols_body<VB>(b, wb, nbb, k, n, kp, nonfinite, blockIdx.x - ga, gridDim.x - ga);
  }
  dependents_may_launch();
}

// ------------------------------------------------------------ tcgen05 GEMM
constexpr int kBM = 128, kBN = 256, kBK = 32;
constexpr int kTileA = kBM * kBK * 4;                   // 16 KB
constexpr int kGemmThreads = 320;  // TMA warp, MMA warp, 8 epilogue warps
constexpr int kTmemCols = 2 * kBN;                      // two 256-column accumulators (CTA-pair kernel)
constexpr int kEpiWarps = 8;
constexpr int kStoreStage = kEpiWarps * 32 * 32 * 4;     // 32 KB: a 32 x 32 staging block per epilogue warp
constexpr int kGroupM = 8;
constexpr int kChunkB = 32 * kBK * 4;  // 4 KB: 32 columns of B x 32 k rows, one TMA box

// Starts the TMA unit's fetch of the four tensor maps (kernel parameters) while the
// CTA sets up, so the first loads do not wait for them.
__device__ __forceinline__ void prefetch_maps(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c,
                                              const CUtensorMap& d) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a)) : "memory");
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&b)) : "memory");
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&c)) : "memory");
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&d)) : "memory");
}

// Tile shape of the single-SM kernel: 128 x BN outputs per work item, BN = 256 (large
// products, two 96 KB stages) or 128 (products whose 128 x 256 tiles leave SMs idle:
// twice the work items, half the epilogue per item, three 64 KB stages). Narrower N
// tiles would be shared-memory bound: each MMA reads its 128 x 8 A slice again, and at
// N = 64 that is ~21 flop per byte read against the ~32 the tensor pipe needs at
// 128 B/clock.
template <int BN>
struct SingleTile {
  static constexpr int kTileB = BN * kBK * 4;
  static constexpr int kStages = BN == 256 ? 2 : 3;
  static constexpr int kStageBytes = 2 * kTileA + 2 * kTileB;
  static constexpr int kTmemCols = 2 * BN;  // two accumulators
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 1024 + kStoreStage;  // slack, barriers, slices
  // instruction descriptor: kind::tf32, D f32, A/B tf32, both K-major, M = 128, N = BN;
  // the MN variant sets bit 16 (B MN-major, the raw mode)
  static constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                                     (static_cast<uint32_t>(kBM >> 4) << 24);
  static constexpr uint32_t kIdescMN = kIdesc | (1u << 16);
  static constexpr int kChunks = BN / 64;  // 32-column chunks per epilogue warp (two warps per lane quarter)
  static_assert(kSmem <= 232448, "shared memory per CTA");
};

struct GemmArgs {
  float* c;
  const float* bias;
  const int* nonfinite;
  int* err;
  int64_t m, n, k_elems;  // output extents
  int64_t lhs_mk, rhs_kn; // elements per operand batch (m*k, k*n)
  int32_t num_kb, tiles_m, tiles_n, act, vec_store;
  int64_t batches;
  BatchMap bm;
  // split-K (single-SM kernel, one output batch): work item t covers tile t / splits and
  // k-blocks [(t % splits) * kb_per_split, +kb_per_split); its raw partial tile goes to
  // partial + (t % splits) * m * n, summed by splitk_reduce
  int32_t splits, kb_per_split;
  float* partial;
  // raw (1): the hi terms are the operands themselves (tcgen05 kind::tf32 reads fp32
  // and drops the low 13 mantissa bits: hi = trunc_tf32(x)); map_a / map_b then hold
  // only lo = rna_tf32(x - trunc_tf32(x)) in the operands' own layouts, and B (hi and
  // lo) is read MN-major in 32-column chunks. raw (0): split planes, both K-major.
  int32_t raw;
  // CTA-pair kernel: the output leaves through TMA tile stores (map_c over [batches][m][n]
  // float32, 32 x 32 boxes, 128-byte swizzle); needs n % 4 == 0 and a 16-byte aligned c
  int32_t tma_out;
  // Stream-K tail of the CTA-pair kernel. Tiles [0, dp_tiles) go round-robin over the
  // clusters (whole waves); the k-blocks of tiles [dp_tiles, total) form one sequence
  // (tile-major) cut into equal contiguous ranges, one per cluster (sk_range). A tile
  // whose k-blocks fall into several ranges is finished by the cluster holding its last
  // k-block: the clusters before it store their raw partial accumulators in their slot
  // of sk_partial (256 x 256 floats per cluster, in epilogue-warp order) and count their
  // epilogue warps in sk_count[2 * cluster + rank] (zeroed before the launch); the
  // finishing cluster waits for the counts, adds the partials in k order, then applies
  // bias / activation and stores. dp_tiles == total: no stream-K.
  int64_t dp_tiles;
  float* sk_partial;
  unsigned* sk_count;
};

// ------------------------------------------------------------ stream-K ranges
constexpr int kMaxSkSources = 4;       // partial slots a finishing cluster may add (ring refills beyond 6 images)
constexpr int kSkSlotFloats = 256 * 256;

// Cluster c's range of the stream-K k-block sequence (U k-blocks over ncl clusters).
__host__ __device__ __forceinline__ int64_t sk_bound(int64_t c, int64_t u, int64_t ncl) { return c * u / ncl; }

// The clusters before `cid` holding the first k-blocks of stream-K tile `ta` (up to
// where cid's range starts) are [first, cid), in k order; this returns `first`. Every
// range is non-empty (u >= ncl), so they are consecutive.
__host__ __device__ __forceinline__ int64_t sk_first_source(int64_t cid, int64_t ta, int64_t kb, int64_t u,
                                                           int64_t ncl) {
  int64_t c = cid - 1;
  while (c > 0 && sk_bound(c, u, ncl) > ta * kb) --c;
  return c;
}

// What one work unit of the CTA-pair kernel does with its accumulator.
enum UnitKind { kWhole = 0, kPartial = 1, kFinish = 2 };

struct PairUnit {
  int64_t tile;
  int kb0, kb1;  // k-blocks [kb0, kb1)
  int kind;
};

// Unit i of cluster cid, in the order all three roles of the cluster walk them: its
// round-robin whole tiles, then its stream-K range as (1) the first k-blocks of the tile
// the range ends in (a partial: the rest of that tile lies in later ranges), (2) the
// whole tiles inside the range, (3) the last k-blocks of the tile the range starts in
// (finishing it with the partials of earlier ranges, stored long before). false: no unit i.
__device__ __forceinline__ bool pair_unit(const GemmArgs& g, int64_t total, int64_t cid, int64_t ncl, int64_t i,
                                          PairUnit& u) {
  const int64_t dp = g.dp_tiles < total ? g.dp_tiles : total;
  const int64_t n_dp = cid < dp ? (dp - cid + ncl - 1) / ncl : 0;
  const int kb = g.num_kb;
  if (i < n_dp) {
    u.tile = cid + i * ncl;
    u.kb0 = 0;
    u.kb1 = kb;
    u.kind = kWhole;
    return true;
  }
  int64_t j = i - n_dp;
  const int64_t sk = total - dp, un = sk * kb;
  if (sk <= 0) return false;
  const int64_t lo = sk_bound(cid, un, ncl), hi = sk_bound(cid + 1, un, ncl);
  if (lo >= hi) return false;
  const int64_t ta = lo / kb, tb = (hi - 1) / kb;
  const int ka = static_cast<int>(lo - ta * kb), ke = static_cast<int>(hi - tb * kb);  // ke in [1, kb]
  if (ta == tb) {
    if (j > 0) return false;
    u.tile = dp + ta;
    u.kb0 = ka;
    u.kb1 = ke;
    u.kind = (ka == 0 && ke == kb) ? kWhole : (ke == kb ? kFinish : kPartial);
    return true;
  }
  const bool head = ke < kb, tail = ka > 0;
  const int64_t f0 = tail ? ta + 1 : ta, f1 = head ? tb - 1 : tb;  // whole tiles [f0, f1]
  const int64_t nf = f1 >= f0 ? f1 - f0 + 1 : 0;
  if (head) {
    if (j == 0) {
      u.tile = dp + tb;
      u.kb0 = 0;
      u.kb1 = ke;
      u.kind = kPartial;
      return true;
    }
    --j;
  }
  if (j < nf) {
    u.tile = dp + f0 + j;
    u.kb0 = 0;
    u.kb1 = kb;
    u.kind = kWhole;
    return true;
  }
  if (tail && j == nf) {
    u.tile = dp + ta;
    u.kb0 = ka;
    u.kb1 = kb;
    u.kind = kFinish;
    return true;
  }
  return false;
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// k-block range of work item t
__device__ __forceinline__ void split_range(int64_t t, const GemmArgs& g, int64_t& tile, int& split, int& kb0, int& kb1) {
  tile = t / g.splits;
  split = static_cast<int>(t - tile * g.splits);
  kb0 = split * g.kb_per_split;
  kb1 = min(g.num_kb, kb0 + g.kb_per_split);
}

__device__ __forceinline__ void tile_coords(int64_t t, const GemmArgs& g, int64_t& batch, int& mt, int& nt) {
  const int64_t per_batch = static_cast<int64_t>(g.tiles_m) * g.tiles_n;
  batch = t / per_batch;
  const int64_t r = t % per_batch;
  const int64_t group_span = static_cast<int64_t>(kGroupM) * g.tiles_n;
  const int64_t group = r / group_span;
  const int first_m = static_cast<int>(group * kGroupM);
  const int gsize = min(kGroupM, g.tiles_m - first_m);
  const int64_t in_group = r % group_span;
  mt = first_m + static_cast<int>(in_group % gsize);
  nt = static_cast<int>(in_group / gsize);
}

// Stores one epilogue warp's 32 x 32 block of the output (lane = row, v = 32 consecutive
// columns of that row) through a 4 KB slice of shared memory, so that each global store
// instruction writes four whole 128-byte row segments instead of 32 half-used sectors
// of 32 different rows (writing rows straight from the TMEM lane layout held the
// epilogue of a 128 x 256 tile at ~10 GB/s per SM). Float4 chunks are XOR-swizzled by
// row: conflict-free both ways. `tile` points at the block's (row 0, column 0); rows
// >= rows_valid and columns >= cols_valid are not written; vec: 16-byte stores allowed
// (the row pitch and base are 16-byte aligned).
__device__ __forceinline__ void store_block_staged(float4* stage, const float (&v)[32], int lane, float* tile,
                                                   int64_t ld, int rows_valid, int64_t cols_valid, bool vec) {
#pragma unroll
  for (int jj = 0; jj < 8; ++jj)
    stage[lane * 8 + (jj ^ (lane & 7))] = make_float4(v[4 * jj], v[4 * jj + 1], v[4 * jj + 2], v[4 * jj + 3]);
  __syncwarp();
  const int jj = lane & 7;
  const int64_t cv = cols_valid - 4 * jj;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int rr = 4 * i + (lane >> 3);
    const float4 x = stage[rr * 8 + (jj ^ (rr & 7))];
    if (rr < rows_valid && cv > 0) {
      float* p = tile + rr * ld + 4 * jj;
      if (vec && cv >= 4) {
        *reinterpret_cast<float4*>(p) = x;
      } else {
        p[0] = x.x;
        if (cv > 1) p[1] = x.y;
        if (cv > 2) p[2] = x.z;
        if (cv > 3) p[3] = x.w;
      }
    }
  }
  __syncwarp();  // the slice is rewritten by the next block
}

// One epilogue warp's share of an accumulator tile: TMEM lanes [32 q, 32 q + 32) (the
// quarter the warp may access) x 32 NCH columns starting at TMEM column `tcol` and output
// column `col0`, as NCH 32-column chunks with the next chunk's tcgen05.ld in flight
// while the current one is finished and stored. `release` runs once every TMEM read of
// the share is done. `block` points at output (row 0, column 0) of the share.
template <int NCH = 4, typename Release>
__device__ __forceinline__ void drain_share(uint32_t tcol, float4* stage, int lane, float* block, int64_t ld,
                                            int rows_valid, int64_t cols_left, int64_t col0, const float* bias,
                                            int act, bool vec, bool skip, Release release) {
  const bool plain = bias == nullptr && act == TCX_ACT_NONE;
  uint32_t r0[32], r1[32];
  TCX_LD32(r0, tcol);
#pragma unroll
  for (int ci = 0; ci < NCH; ++ci) {
    uint32_t (&cur)[32] = (ci & 1) ? r1 : r0;
    uint32_t (&nxt)[32] = (ci & 1) ? r0 : r1;
    TCX_WAIT_LD32(cur);
    if (ci + 1 < NCH) {
      TCX_LD32(nxt, tcol + static_cast<uint32_t>((ci + 1) * 32));
    } else {
      release();
    }
    const int64_t left = cols_left - ci * 32;
    if (left > 0 && rows_valid > 0 && !skip) {
      float v[32];
      if (plain) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(cur[j]);
      } else {
        const int64_t c = col0 + ci * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = j < left ? epilogue_op(__uint_as_float(cur[j]), bias, c + j, act) : 0.0f;
      }
      store_block_staged(stage, v, lane, block + ci * 32, ld, rows_valid, left, vec);
    }
  }
}

// ------------------------------------------------ CTA-pair epilogue (bulk stores)
// Each epilogue warp of the pair kernel owns a 4 KB staging slice (1024-byte aligned):
// a 32 x 32 float block in the 128-byte-swizzled image (row = lane, 16-byte chunk j of
// the row at position j ^ (row & 7)), which is both what a SWIZZLE_128B tensor map
// stores from and conflict-free for the lanes' 16-byte writes. Output blocks leave the
// slice through one TMA tile store (the map clips the tensor's edges); stream-K partial
// blocks through one plain bulk store of the image itself. Before rewriting the slice,
// lane 0 waits until the previous bulk store has read it.
__device__ __forceinline__ void stage_image(float4* slice, const uint32_t (&r)[32], int lane) {
  if (lane == 0) bulk_wait_read();
  __syncwarp();
#pragma unroll
  for (int jj = 0; jj < 8; ++jj)
    slice[lane * 8 + (jj ^ (lane & 7))] = make_float4(__uint_as_float(r[4 * jj]), __uint_as_float(r[4 * jj + 1]),
                                                      __uint_as_float(r[4 * jj + 2]), __uint_as_float(r[4 * jj + 3]));
  fence_async_shared();  // the writes become visible to the bulk copy
  __syncwarp();
}

// What one pair-kernel epilogue warp does with its share (4 chunks of 32 x 32) of a
// work unit's accumulator (PairUnit kinds), when the output leaves through TMA tile
// stores (otherwise the kernel drains with drain_share and runs without stream-K):
//   kWhole   bias / activation, then TMA tile stores through map_c;
//   kPartial the raw accumulator to the stream-K partial slot `part` (4 KB images, chunk
//            ci at part + 1024 ci), as bulk stores;
//   kFinish  first adds the partial images of the nsrc clusters holding the tile's earlier
//            k-blocks (src, src + kSkSlotFloats, ..., in k order), which `ring` (this
//            warp's 24 KB of the idle pipeline stages: six 4 KB slots with one mbarrier
//            each at ring_bars) receives by bulk loads, then as kWhole.
struct PairOut {
  const CUtensorMap* map_c;
  int rows_valid, cols_left;  // of the share, from its (row 0, column 0)
  int col0, row0, batch;      // the share's column, row and batch in map_c
};

template <int MODE, int NCH = 4, typename Release>
__device__ __forceinline__ void drain_pair(uint32_t tcol, float4* slice, int lane, const PairOut& o, const float* bias,
                                           int act, bool skip, Release release, float* part, const float* src,
                                           int nsrc, float4* ring, uint32_t ring_bars, int* err) {
  const bool plain = bias == nullptr && act == TCX_ACT_NONE;
  const int items = MODE == kFinish ? 4 * nsrc : 0;  // (chunk, source) images, chunk-major
  if constexpr (MODE == kFinish) {
    if (lane == 0) {
      fence_async_global();  // the sources' counts were acquired: their images are visible
      for (int q = 0; q < items && q < 6; ++q) {
        const uint32_t bar = ring_bars + 8 * q;
        mbar_expect_tx(bar, 4096);
        bulk_load(smem_u32(ring + 256 * q), src + (q % nsrc) * kSkSlotFloats + (q / nsrc) * 1024, 4096, bar);
      }
    }
  }
  uint32_t r0[32], r1[32];
  TCX_LD32(r0, tcol);
#pragma unroll
  for (int ci = 0; ci < NCH; ++ci) {
    uint32_t (&cur)[32] = (ci & 1) ? r1 : r0;
    uint32_t (&nxt)[32] = (ci & 1) ? r0 : r1;
    TCX_WAIT_LD32(cur);
    if (ci + 1 < NCH) {
      TCX_LD32(nxt, tcol + static_cast<uint32_t>((ci + 1) * 32));
    } else {
      release();
    }
    if constexpr (MODE == kPartial) {
      stage_image(slice, cur, lane);
      if (lane == 0) {
        bulk_store(part + ci * 1024, smem_u32(slice), 4096);
        bulk_commit();
      }
      continue;
    }
    if (MODE == kFinish && nsrc > 0) {
      // (source 0 + source 1 + ...) + own accumulator
      float t[32];
      for (int p = 0; p < nsrc; ++p) {
        const int q = ci * nsrc + p;
        const uint32_t bar = ring_bars + 8 * (q % 6);
        wait_or_give_up(bar, static_cast<uint32_t>((q / 6) & 1), err, 0x207);
        const float4* img = ring + 256 * (q % 6);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const float4 x = img[lane * 8 + (jj ^ (lane & 7))];
          if (p == 0) {
            t[4 * jj] = x.x; t[4 * jj + 1] = x.y; t[4 * jj + 2] = x.z; t[4 * jj + 3] = x.w;
          } else {
            t[4 * jj] = __fadd_rn(t[4 * jj], x.x);
            t[4 * jj + 1] = __fadd_rn(t[4 * jj + 1], x.y);
            t[4 * jj + 2] = __fadd_rn(t[4 * jj + 2], x.z);
            t[4 * jj + 3] = __fadd_rn(t[4 * jj + 3], x.w);
          }
        }
        __syncwarp();
        if (lane == 0 && q + 6 < items) {  // refill the slot just read
          fence_async_shared();
          const int q2 = q + 6;
          mbar_expect_tx(bar, 4096);
          bulk_load(smem_u32(ring + 256 * (q2 % 6)), src + (q2 % nsrc) * kSkSlotFloats + (q2 / nsrc) * 1024, 4096,
                    bar);
        }
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) cur[j] = __float_as_uint(__fadd_rn(t[j], __uint_as_float(cur[j])));
    }
    const int left = o.cols_left - ci * 32;
    if (left > 0 && o.rows_valid > 0 && !skip) {
      if (!plain) {
        const int64_t c = o.col0 + ci * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          cur[j] = __float_as_uint(j < left ? epilogue_op(__uint_as_float(cur[j]), bias, c + j, act) : 0.0f);
      }
      stage_image(slice, cur, lane);
      if (lane == 0) {
        tma_store_3d(o.map_c, smem_u32(slice), o.col0 + ci * 32, o.row0, o.batch);
        bulk_commit();
      }
    }
  }
}

// The finishing drain of a stream-K tile (once per cluster and call), kept out of line so
// that its partial loads do not raise the register pressure of the kernel's other paths.
template <typename Release>
__device__ __noinline__ void drain_finish(uint32_t tcol, float4* slice, int lane, const PairOut o, const float* bias,
                                          int act, bool skip, Release release, const float* src, int nsrc,
                                          float4* ring, uint32_t ring_bars, int* err) {
  drain_pair<kFinish>(tcol, slice, lane, o, bias, act, skip, release, nullptr, src, nsrc, ring, ring_bars, err);
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_a_hi, const __grid_constant__ CUtensorMap map_b_hi,
                   const __grid_constant__ CUtensorMap map_c, const GemmArgs g) {
  using T = SingleTile<BN>;
  constexpr int kStages = T::kStages, kStageBytes = T::kStageBytes, kTileB = T::kTileB, kTmemCols = T::kTmemCols;
  if (threadIdx.x == 0) {
    prefetch_maps(map_a, map_b, map_a_hi, map_b_hi);
    if (g.tma_out) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_c)) : "memory");
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* full = bars;                  // [kStages]
  uint64_t* empty = bars + kStages;       // [kStages]
  uint64_t* acc_full = bars + 2 * kStages;      // [2]
  uint64_t* acc_empty = bars + 2 * kStages + 2; // [2]
  uint64_t* drain = bars + 2 * kStages + 4;     // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float4* stage = reinterpret_cast<float4*>(smem + kStages * kStageBytes + 1024) + ((threadIdx.x >> 5) - 2) * 256;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) { mbar_init(smem_u32(&full[s]), 1); mbar_init(smem_u32(&empty[s]), 1); }
    for (int s = 0; s < 2; ++s) { mbar_init(smem_u32(&acc_full[s]), 1); mbar_init(smem_u32(&acc_empty[s]), kEpiWarps); }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Set-up is done; the pre-pass launched before this kernel must now be complete. With
  // inf / NaN in the inputs it raised the flag: no work here, the FFMA kernel queued
  // behind this one computes the product.
  wait_for_prior_grid();
  const int64_t total_work = *g.nonfinite ? 0 : g.batches * g.tiles_m * g.tiles_n * g.splits;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- TMA producer
      int64_t kb_global = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < total_work && ok; t += gridDim.x) {
        int64_t tile; int split, kb0, kb1;
        split_range(t, g, tile, split, kb0, kb1);
        int64_t batch; int mt, nt;
        tile_coords(tile, g, batch, mt, nt);
        const int64_t pa = batch_off(batch, g.bm.shape, g.bm.lhs, g.bm.rank) / (g.lhs_mk > 0 ? g.lhs_mk : 1);
        const int64_t pb = batch_off(batch, g.bm.shape, g.bm.rhs, g.bm.rank) / (g.rhs_kn > 0 ? g.rhs_kn : 1);
        for (int kb = kb0; kb < kb1; ++kb, ++kb_global) {
          const int s = static_cast<int>(kb_global % kStages);
          const uint32_t phase = static_cast<uint32_t>((kb_global / kStages) & 1);
          if (!wait_bounded(smem_u32(&empty[s]), phase ^ 1u, abort_flag, g.err, 0x101)) { ok = false; break; }
          uint8_t* st = smem + s * kStageBytes;
          const uint32_t fb = smem_u32(&full[s]);
          mbar_expect_tx(fb, kStageBytes);
          const int kc = kb * kBK;
          if (g.raw) {
            // A: raw rows (hi) and lo rows, K-major; B: raw (hi) and lo, each as BN / 32
            // MN-major chunks of 32 columns x 32 k rows (columns past N read as zeros)
            tma_load_3d(smem_u32(st), &map_a_hi, fb, kc, mt * kBM, static_cast<int>(pa));
            tma_load_3d(smem_u32(st + kTileA), &map_a, fb, kc, mt * kBM, static_cast<int>(pa));
            for (int j = 0; j < BN / 32; ++j) {
              tma_load_3d(smem_u32(st + 2 * kTileA + j * kChunkB), &map_b_hi, fb, nt * BN + 32 * j, kc,
                          static_cast<int>(pb));
              tma_load_3d(smem_u32(st + 2 * kTileA + kTileB + j * kChunkB), &map_b, fb, nt * BN + 32 * j, kc,
                          static_cast<int>(pb));
            }
          } else {
            tma_load_3d(smem_u32(st), &map_a, fb, kc, mt * kBM, static_cast<int>(2 * pa));
            tma_load_3d(smem_u32(st + kTileA), &map_a, fb, kc, mt * kBM, static_cast<int>(2 * pa + 1));
            tma_load_3d(smem_u32(st + 2 * kTileA), &map_b, fb, kc, nt * BN, static_cast<int>(2 * pb));
            tma_load_3d(smem_u32(st + 2 * kTileA + kTileB), &map_b, fb, kc, nt * BN, static_cast<int>(2 * pb + 1));
          }
        }
      }
      // Drain: every stage this thread filled must have landed before the CTA exits.
      if (!ok) {
        for (int s = 0; s < kStages; ++s) {
          const int64_t fills = kb_global > s ? (kb_global - s + kStages - 1) / kStages : 0;
          if (fills == 0) continue;
          const uint32_t parity = static_cast<uint32_t>((fills - 1) & 1);
          const uint64_t start = globaltimer();
          while (!mbar_try_wait(smem_u32(&full[s]), parity))
            if (globaltimer() - start > kWaitLimitNs) { record_device_error(g.err, 0x1ff); break; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      int64_t kb_global = 0;
      int64_t local = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < total_work && ok; t += gridDim.x, ++local) {
        int64_t tile; int split, kb0, kb1;
        split_range(t, g, tile, split, kb0, kb1);
        const int acc = static_cast<int>(local & 1);
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!wait_bounded(smem_u32(&acc_empty[acc]), acc_phase ^ 1u, abort_flag, g.err, 0x102)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb, ++kb_global) {
          const int s = static_cast<int>(kb_global % kStages);
          const uint32_t phase = static_cast<uint32_t>((kb_global / kStages) & 1);
          if (!wait_bounded(smem_u32(&full[s]), phase, abort_flag, g.err, 0x103)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_hi = smem_u32(smem + s * kStageBytes);
          const uint32_t a_lo = a_hi + kTileA;
          const uint32_t b_hi = a_hi + 2 * kTileA;
          const uint32_t b_lo = b_hi + kTileB;
          const uint64_t da_hi = smem_desc_sw128(a_hi), da_lo = smem_desc_sw128(a_lo);
          // 8 k per MMA: 32 bytes along a K-major row (2 in the >> 4 address field), or
          // 8 rows of 128 bytes in an MN-major chunk (64)
          const uint64_t db_hi = g.raw ? smem_desc_sw128_mn(b_hi, kChunkB) : smem_desc_sw128(b_hi);
          const uint64_t db_lo = g.raw ? smem_desc_sw128_mn(b_lo, kChunkB) : smem_desc_sw128(b_lo);
          const uint64_t b_step = g.raw ? 64u : 2u;
          const uint32_t idesc = g.raw ? T::kIdescMN : T::kIdesc;
#pragma unroll
          for (int kk = 0; kk < kBK / 8; ++kk) {
            const uint32_t first = (kb == kb0 && kk == 0) ? 0u : 1u;
            const uint64_t ka = 2u * kk, kbo = b_step * kk;
            mma_tf32(d_tmem, da_lo + ka, db_hi + kbo, idesc, first);
            mma_tf32(d_tmem, da_hi + ka, db_lo + kbo, idesc, 1u);
            mma_tf32(d_tmem, da_hi + ka, db_hi + kbo, idesc, 1u);
          }
          mma_commit(smem_u32(&empty[s]));  // stage free once these MMAs have read it
        }
        mma_commit(smem_u32(&acc_full[acc]));  // accumulator ready (or drained on abort)
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue
    // Eight warps, two per SM sub-partition: warp w drains TMEM lane quarter w & 3 (the
    // lanes it may access), columns [0, BN / 2) for warps 2-5 and [BN / 2, BN) for 6-9.
    const int q = warp & 3;
    const int part = warp >= 6 ? 1 : 0;
    int64_t local = 0;
    for (int64_t t = blockIdx.x; t < total_work; t += gridDim.x, ++local) {
      const int acc = static_cast<int>(local & 1);
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      if (!wait_bounded(smem_u32(&acc_full[acc]), acc_phase, abort_flag, g.err, 0x104)) break;
      tc_fence_after();
      int64_t tile; int split, kb0, kb1;
      split_range(t, g, tile, split, kb0, kb1);
      int64_t batch; int mt, nt;
      tile_coords(tile, g, batch, mt, nt);
      const int64_t row0 = static_cast<int64_t>(mt) * kBM + q * 32;  // this warp's first row
      const int64_t col0 = static_cast<int64_t>(nt) * BN + part * (BN / 2);
      // split-K: the raw partial sums go to this split's slice of the workspace
      const bool raw = g.splits > 1;
      float* block = (raw ? g.partial + (static_cast<int64_t>(split) * g.m + row0) * g.n
                          : g.c + (batch * g.m + row0) * g.n) + col0;
      const int rows_valid = static_cast<int>(g.m - row0 < 32 ? g.m - row0 : 32);
      const uint32_t tcol = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            static_cast<uint32_t>(acc * BN + part * (BN / 2));
      auto release = [&] {
        // all TMEM reads of this accumulator are done: hand it back to the MMA warp
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&acc_empty[acc]));
      };
      if (g.tma_out) {
        // TMA tile stores: map_c covers the output [batches][m][n], or with split-K the
        // partial slices [splits][m][n]
        PairOut o;
        o.map_c = &map_c;
        o.rows_valid = rows_valid;
        o.cols_left = static_cast<int>(g.n - col0);
        o.col0 = static_cast<int>(col0);
        o.row0 = static_cast<int>(row0);
        o.batch = static_cast<int>(raw ? split : batch);
        drain_pair<kWhole, T::kChunks>(tcol, stage, lane, o, raw ? nullptr : g.bias, raw ? TCX_ACT_NONE : g.act,
                                       *abort_flag != 0, release, nullptr, nullptr, 0, nullptr, 0, g.err);
      } else {
        drain_share<T::kChunks>(tcol, stage, lane, block, g.n, rows_valid, g.n - col0, col0, raw ? nullptr : g.bias,
                                raw ? TCX_ACT_NONE : g.act, g.vec_store != 0, *abort_flag != 0, release);
      }
    }
    if (lane == 0) bulk_wait();  // this warp's bulk stores complete before the CTA exits
    __syncwarp();
  }

  dependents_may_launch();  // the split-K reduce / fallback behind may start its set-up
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) {
      // every MMA this thread issued must complete before TMEM is released
      mma_commit(smem_u32(drain));
      const uint64_t start = globaltimer();
      while (!mbar_try_wait(smem_u32(drain), 0))
        if (globaltimer() - start > kWaitLimitNs) { record_device_error(g.err, 0x1fe); break; }
    }
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------- 2-SM (CTA pair) GEMM
// The same 3xTF32 product on 256 x 256 tiles computed by a cluster of two CTAs on two
// SMs with tcgen05.mma.cta_group::2 (M = 256): CTA r of the pair holds rows
// [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128) of the B tile (its
// half of N) in its own shared memory, at the same offsets; the leader CTA (rank 0)
// issues every MMA, each SM's TMEM receives its 128 rows of the 256 x 256 accumulator.
// Per SM and k step the tensor core reads 24 KB of operands instead of 36 KB, and the
// stages shrink to 64 KB, so three fit: the single-SM kernel's shared-memory traffic
// (operand reads plus TMA writes, ~150 B/clock against 128) drops to ~100 B/clock.
// Both CTAs' TMA loads complete on the leader's full barrier (which expects both
// halves); the leader's commits arrive on both CTAs' barriers (one commit per CTA, no
// multicast); the peer's epilogue warps arrive on the leader's accumulator-empty
// barrier remotely. No TMA multicast.
constexpr int kStages2 = 3;
constexpr int kHalf = 128;                                  // rows of A and of B per CTA
constexpr int kTile2 = kHalf * kBK * 4;                     // 16 KB
constexpr int kStage2Bytes = 4 * kTile2;                    // A hi/lo, B hi/lo: 64 KB
// stages, alignment slack, 1 KB of barriers (and the stream-K ring's), staging slices
constexpr int kGemm2Smem = kStages2 * kStage2Bytes + 1024 + 1024 + kStoreStage;
constexpr int kRingSlots = 6;  // stream-K partial images in flight per epilogue warp (24 KB of the stages)
static_assert(kEpiWarps * kRingSlots * 4096 <= kStages2 * kStage2Bytes, "stream-K ring in the pipeline stages");
static_assert(kGemm2Smem <= 232448, "shared memory per CTA");
constexpr uint32_t kIdesc2 = (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(256 >> 3) << 17) |
                             (static_cast<uint32_t>(256 >> 4) << 24);
constexpr uint32_t kIdesc2MN = kIdesc2 | (1u << 16);  // B MN-major (raw mode)

__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_tf32x3_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_a_hi, const __grid_constant__ CUtensorMap map_b_hi,
                        const __grid_constant__ CUtensorMap map_c, const GemmArgs g) {
  // g.tiles_m counts 256-row tiles here; both CTAs of a pair return together
  if (threadIdx.x == 0) {
    prefetch_maps(map_a, map_b, map_a_hi, map_b_hi);
    if (g.tma_out) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_c)) : "memory");
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages2 * kStage2Bytes);
  uint64_t* full = bars;                          // [kStages2] (the leader's are used)
  uint64_t* empty = bars + kStages2;              // [kStages2]
  uint64_t* acc_full = bars + 2 * kStages2;       // [2]
  uint64_t* acc_empty = bars + 2 * kStages2 + 2;  // [2] (the leader's, 8 warps arrive)
  uint64_t* drain = bars + 2 * kStages2 + 4;      // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages2 + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* ring_bars = bars + 2 * kStages2 + 6;  // [kEpiWarps][kRingSlots] (stream-K finishing)
  // this epilogue warp's staging slice (4 KB, 1024-byte aligned) and stream-K ring
  float4* stage = reinterpret_cast<float4*>(smem + kStages2 * kStage2Bytes + 1024) + ((threadIdx.x >> 5) - 2) * 256;
  float4* ring = reinterpret_cast<float4*>(smem) + ((threadIdx.x >> 5) - 2) * kRingSlots * 256;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) { mbar_init(smem_u32(&full[s]), 1); mbar_init(smem_u32(&empty[s]), 1); }
    for (int s = 0; s < 2; ++s) { mbar_init(smem_u32(&acc_full[s]), 1); mbar_init(smem_u32(&acc_empty[s]), 2 * kEpiWarps); }
    mbar_init(smem_u32(drain), 1);
    for (int i = 0; i < kEpiWarps * kRingSlots; ++i) mbar_init(smem_u32(&ring_bars[i]), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrive or load
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // as in the single-SM kernel: the pre-pass must be complete; the flag means no work
  wait_for_prior_grid();
  const int64_t total_tiles = *g.nonfinite ? 0 : g.batches * g.tiles_m * g.tiles_n;
  const int64_t cid = cluster_index(), ncl = cluster_count();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer (both CTAs)
      int64_t kb_global = 0;
      bool ok = true;
      PairUnit u;
      for (int64_t i = 0; ok && pair_unit(g, total_tiles, cid, ncl, i, u); ++i) {
        int64_t batch; int mt, nt;
        tile_coords(u.tile, g, batch, mt, nt);
        const int64_t pa = batch_off(batch, g.bm.shape, g.bm.lhs, g.bm.rank) / (g.lhs_mk > 0 ? g.lhs_mk : 1);
        const int64_t pb = batch_off(batch, g.bm.shape, g.bm.rhs, g.bm.rank) / (g.rhs_kn > 0 ? g.rhs_kn : 1);
        const int row_a = mt * 2 * kHalf + static_cast<int>(rank) * kHalf;
        const int row_b = nt * 2 * kHalf + static_cast<int>(rank) * kHalf;
        for (int kb = u.kb0; kb < u.kb1; ++kb, ++kb_global) {
          const int s = static_cast<int>(kb_global % kStages2);
          const uint32_t phase = static_cast<uint32_t>((kb_global / kStages2) & 1);
          if (!wait_bounded(smem_u32(&empty[s]), phase ^ 1u, abort_flag, g.err, 0x201)) { ok = false; break; }
          uint8_t* st = smem + s * kStage2Bytes;
          const uint32_t fb_local = smem_u32(&full[s]);
          if (leader) mbar_expect_tx(fb_local, 2 * kStage2Bytes);  // both CTAs' halves
          const uint32_t fb = map_rank(fb_local, 0);
          const int kc = kb * kBK;
          if (g.raw) {  // this CTA's half of B: kHalf / 32 MN-major chunks per term
            tma_load_3d_pair(smem_u32(st), &map_a_hi, fb, kc, row_a, static_cast<int>(pa));
            tma_load_3d_pair(smem_u32(st + kTile2), &map_a, fb, kc, row_a, static_cast<int>(pa));
            for (int j = 0; j < kHalf / 32; ++j) {
              tma_load_3d_pair(smem_u32(st + 2 * kTile2 + j * kChunkB), &map_b_hi, fb, row_b + 32 * j, kc,
                               static_cast<int>(pb));
              tma_load_3d_pair(smem_u32(st + 3 * kTile2 + j * kChunkB), &map_b, fb, row_b + 32 * j, kc,
                               static_cast<int>(pb));
            }
          } else {
            tma_load_3d_pair(smem_u32(st), &map_a, fb, kc, row_a, static_cast<int>(2 * pa));
            tma_load_3d_pair(smem_u32(st + kTile2), &map_a, fb, kc, row_a, static_cast<int>(2 * pa + 1));
            tma_load_3d_pair(smem_u32(st + 2 * kTile2), &map_b, fb, kc, row_b, static_cast<int>(2 * pb));
            tma_load_3d_pair(smem_u32(st + 3 * kTile2), &map_b, fb, kc, row_b, static_cast<int>(2 * pb + 1));
          }
        }
      }
      if (!ok && leader) {  // the leader's fills must land before the CTA exits
        for (int s = 0; s < kStages2; ++s) {
          const int64_t fills = kb_global > s ? (kb_global - s + kStages2 - 1) / kStages2 : 0;
          if (fills == 0) continue;
          const uint32_t parity = static_cast<uint32_t>((fills - 1) & 1);
          const uint64_t start = globaltimer();
          while (!mbar_try_wait(smem_u32(&full[s]), parity))
            if (globaltimer() - start > kWaitLimitNs) { record_device_error(g.err, 0x2ff); break; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------ MMA issuer (leader only)
      int64_t kb_global = 0, local = 0;
      bool ok = true;
      PairUnit u;
      for (int64_t i = 0; ok && pair_unit(g, total_tiles, cid, ncl, i, u); ++i, ++local) {
        const int acc = static_cast<int>(local & 1);
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!wait_bounded(smem_u32(&acc_empty[acc]), acc_phase ^ 1u, abort_flag, g.err, 0x202)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kb = u.kb0; kb < u.kb1; ++kb, ++kb_global) {
          const int s = static_cast<int>(kb_global % kStages2);
          const uint32_t phase = static_cast<uint32_t>((kb_global / kStages2) & 1);
          if (!wait_bounded(smem_u32(&full[s]), phase, abort_flag, g.err, 0x203)) { ok = false; break; }
          tc_fence_after();
          const uint64_t a_hi = smem_desc_sw128(smem_u32(smem + s * kStage2Bytes));
          const uint64_t a_lo = smem_desc_sw128(smem_u32(smem + s * kStage2Bytes + kTile2));
          const uint32_t sb_hi = smem_u32(smem + s * kStage2Bytes + 2 * kTile2);
          const uint32_t sb_lo = smem_u32(smem + s * kStage2Bytes + 3 * kTile2);
          const uint64_t b_hi = g.raw ? smem_desc_sw128_mn(sb_hi, kChunkB) : smem_desc_sw128(sb_hi);
          const uint64_t b_lo = g.raw ? smem_desc_sw128_mn(sb_lo, kChunkB) : smem_desc_sw128(sb_lo);
          const uint64_t b_step = g.raw ? 64u : 2u;  // 8 rows of 128 B (MN-major) or 32 B (K-major)
          const uint32_t idesc = g.raw ? kIdesc2MN : kIdesc2;
#pragma unroll
          for (int kk = 0; kk < kBK / 8; ++kk) {  // 8 tf32 = 32 bytes = 2 in the >> 4 address field
            const uint32_t first = (kb == u.kb0 && kk == 0) ? 0u : 1u;
            mma_tf32_pair(d_tmem, a_lo + 2 * kk, b_hi + b_step * kk, idesc, first);
            mma_tf32_pair(d_tmem, a_hi + 2 * kk, b_lo + b_step * kk, idesc, 1u);
            mma_tf32_pair(d_tmem, a_hi + 2 * kk, b_hi + b_step * kk, idesc, 1u);
          }
          const uint32_t e = smem_u32(&empty[s]);
          mma_commit_pair(e);               // both CTAs' stages are free once these MMAs
          mma_commit_pair(map_rank(e, 1));  // have read them
        }
        const uint32_t af = smem_u32(&acc_full[acc]);
        mma_commit_pair(af);
        mma_commit_pair(map_rank(af, 1));
      }
    }
  } else {
    // ------------------------------------------------------ epilogue (both CTAs)
    // Eight warps per CTA as in the single-SM kernel: lane quarter w & 3, columns
    // [0, 128) for warps 2-5 and [128, 256) for 6-9.
    const int q = warp & 3;
    const int part = warp >= 6 ? 1 : 0;
    // this warp's share of a 256 x 256 partial slot: four 4 KB block images
    const int64_t share = (static_cast<int64_t>(rank) * kEpiWarps + (warp - 2)) * 4096;
    const uint32_t my_ring_bars = smem_u32(ring_bars + (warp - 2) * kRingSlots);
    int64_t local = 0;
    PairUnit u;
    for (int64_t i = 0; pair_unit(g, total_tiles, cid, ncl, i, u); ++i, ++local) {
      const int acc = static_cast<int>(local & 1);
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      if (!wait_bounded(smem_u32(&acc_full[acc]), acc_phase, abort_flag, g.err, 0x204)) break;
      tc_fence_after();
      int64_t batch; int mt, nt;
      tile_coords(u.tile, g, batch, mt, nt);
      const int64_t row0 = static_cast<int64_t>(mt) * 2 * kHalf + static_cast<int64_t>(rank) * kHalf + q * 32;
      const int64_t col0 = static_cast<int64_t>(nt) * kBN + part * 128;
      const int rows_valid = static_cast<int>(g.m - row0 < 32 ? g.m - row0 : 32);
      const uint32_t tcol = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            static_cast<uint32_t>(acc * kBN + part * 128);
      auto release = [&] {
        // all TMEM reads of this accumulator are done: tell the leader's MMA warp
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_rank(smem_u32(&acc_empty[acc]), 0));
      };
      const bool skip = *abort_flag != 0;
      PairOut o;
      o.map_c = &map_c;
      o.rows_valid = rows_valid;
      o.cols_left = static_cast<int>(g.n - col0);
      o.col0 = static_cast<int>(col0);
      o.row0 = static_cast<int>(row0);
      o.batch = static_cast<int>(batch);
      if (u.kind == kPartial) {
        // raw partial of the tile's first k-blocks into this cluster's slot; the count is
        // raised once the stores have completed (even after an abort, so that the
        // finishing cluster does not wait out its limit)
        drain_pair<kPartial>(tcol, stage, lane, o, g.bias, g.act, skip, release,
                             g.sk_partial + cid * kSkSlotFloats + share, nullptr, 0, ring, my_ring_bars, g.err);
        if (lane == 0) {
          bulk_wait();
          fence_async_global();
          __threadfence();
          red_release_add(g.sk_count + 2 * cid + rank, 1u);
        }
        __syncwarp();
      } else if (u.kind == kFinish) {
        // the clusters holding the tile's first k-blocks stored their partials first
        // thing in their stream-K ranges; wait for their counts (bounded), then add
        const int64_t dp = g.dp_tiles < total_tiles ? g.dp_tiles : total_tiles;
        const int64_t first = sk_first_source(cid, u.tile - dp, g.num_kb, (total_tiles - dp) * g.num_kb, ncl);
        const int n = static_cast<int>(cid - first);  // 1 or 2: the host keeps it <= kMaxSkSources
        bool waited = true;
        if (lane == 0) {
          for (int64_t c = first; c < cid && waited; ++c) {
            const unsigned* cnt = g.sk_count + 2 * c + rank;
            const uint64_t start = globaltimer();
            while (ld_acquire_u32(cnt) < static_cast<unsigned>(kEpiWarps)) {
              if (globaltimer() - start > kWaitLimitNs) {
                record_device_error(g.err, 0x205);
                waited = false;
                break;
              }
            }
          }
        }
        waited = __shfl_sync(0xffffffffu, waited ? 1 : 0, 0) != 0;
        drain_finish(tcol, stage, lane, o, g.bias, g.act, skip || !waited, release,
                     g.sk_partial + first * kSkSlotFloats + share, waited ? n : 0, ring, my_ring_bars, g.err);
      } else if (g.tma_out) {
        drain_pair<kWhole>(tcol, stage, lane, o, g.bias, g.act, skip, release, nullptr, nullptr, 0, ring,
                           my_ring_bars, g.err);
      } else {
        float* block = g.c + (batch * g.m + row0) * g.n + col0;
        drain_share(tcol, stage, lane, block, g.n, rows_valid, g.n - col0, col0, g.bias, g.act, g.vec_store != 0,
                    skip, release);
      }
    }
    if (lane == 0) bulk_wait();  // this warp's bulk stores complete before the CTA exits
    __syncwarp();
  }

  dependents_may_launch();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) {
      // every MMA of the pair must complete before either CTA releases its TMEM
      if (leader) {
        mma_commit_pair(smem_u32(drain));
        mma_commit_pair(map_rank(smem_u32(drain), 1));
      }
      const uint64_t start = globaltimer();
      while (!mbar_try_wait(smem_u32(drain), 0))
        if (globaltimer() - start > kWaitLimitNs) { record_device_error(g.err, 0x2fe); break; }
    }
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
  cluster_sync_all();  // neither CTA leaves while the other may still touch its barriers
}

// --------------------------------------------------------------- FFMA GEMM
constexpr int kFM = 64, kFN = 64, kFK = 16;

// mode 0: always compute; mode 1: only when *nonfinite is set (fallback behind the
// tensor-core kernel). BT: B is stored transposed ([n][k], K-major), as a linear weight.
template <bool BT>
__global__ void __launch_bounds__(256)
gemm_ffma_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ c,
                 int64_t m, int64_t n, int64_t k, int64_t batches, BatchMap bm,
                 const float* __restrict__ bias, int act, const int* __restrict__ nonfinite, int mode) {
  wait_for_prior_grid();
  if (mode == 1 && !*nonfinite) return;
  __shared__ float as[kFK][kFM + 4];
  __shared__ float bs[kFK][kFN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t tiles_m = (m + kFM - 1) / kFM, tiles_n = (n + kFN - 1) / kFN;
  const int64_t total = batches * tiles_m * tiles_n;
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    const int64_t batch = t / (tiles_m * tiles_n), r = t % (tiles_m * tiles_n);
    const int64_t m0 = (r / tiles_n) * kFM, n0 = (r % tiles_n) * kFN;
    const float* ab = a + batch_off(batch, bm.shape, bm.lhs, bm.rank);
    const float* bb = b + batch_off(batch, bm.shape, bm.rhs, bm.rank);
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int64_t k0 = 0; k0 < k; k0 += kFK) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int e = threadIdx.x + i * 256;
        const int rr = e / kFK, cc = e % kFK;
        const int64_t gm = m0 + rr, gk = k0 + cc;
        as[cc][rr] = (gm < m && gk < k) ? __ldg(ab + gm * k + gk) : 0.0f;
        const int br = e / kFN, bc = e % kFN;
        const int64_t bk = k0 + br, bn = n0 + bc;
        if (BT) {
          // transposed B: consecutive threads walk k for one n (coalesced along k)
          const int tk = e % kFK, tn = e / kFK;
          const int64_t gk = k0 + tk, gn = n0 + tn;
          bs[tk][tn] = (gk < k && gn < n) ? __ldg(bb + gn * k + gk) : 0.0f;
        } else {
          bs[br][bc] = (bk < k && bn < n) ? __ldg(bb + bk * n + bn) : 0.0f;
        }
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < kFK; ++kk) {
        float av[4], bv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) av[i] = as[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[j] = bs[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t gm = m0 + ty * 4 + i;
      if (gm >= m) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gn = n0 + tx * 4 + j;
        if (gn < n) c[(batch * m + gm) * n + gn] = epilogue_op(acc[i][j], bias, gn, act);
      }
    }
  }
}

// Split-K epilogue: out = act(sum over splits, in split order, of the raw partial
// tiles + bias). When the pre-pass flagged inf / NaN the tensor-core kernel left no
// partials, and this kernel computes the IEEE product instead: every output element
// accumulates a[row, kk] * b[kk, col] with fmaf in ascending kk, as the FFMA fallback
// kernel does, so the split-K path needs no separate fallback launch.
// VEC: n % 4 == 0 and 16-byte aligned buffers.
template <bool VEC>
__global__ void __launch_bounds__(256)
splitk_reduce(const float* __restrict__ partial, float* __restrict__ out, int64_t mn, int64_t n, int splits,
              const float* __restrict__ bias, int act, const int* __restrict__ nonfinite,
              const float* __restrict__ lhs, const float* __restrict__ rhs, int64_t k, int rhs_kmajor) {
  wait_for_prior_grid();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (*nonfinite) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < mn; i += stride) {
      const int64_t r = i / n, c = i - r * n;
      float acc = 0.0f;
      for (int64_t kk = 0; kk < k; ++kk)
        acc = fmaf(__ldg(lhs + r * k + kk), __ldg(rhs_kmajor ? rhs + c * k + kk : rhs + kk * n + c), acc);
      out[i] = epilogue_op(acc, bias, c, act);
    }
    return;
  }
  if (VEC) {
    for (int64_t i = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) * 4; i < mn; i += stride * 4) {
      float4 v = __ldcs(reinterpret_cast<const float4*>(partial + i));
      for (int sp = 1; sp < splits; ++sp) {
        const float4 w = __ldcs(reinterpret_cast<const float4*>(partial + sp * mn + i));
        v.x = __fadd_rn(v.x, w.x); v.y = __fadd_rn(v.y, w.y); v.z = __fadd_rn(v.z, w.z); v.w = __fadd_rn(v.w, w.w);
      }
      const int64_t c = i % n;
      v.x = epilogue_op(v.x, bias, c + 0, act); v.y = epilogue_op(v.y, bias, c + 1, act);
      v.z = epilogue_op(v.z, bias, c + 2, act); v.w = epilogue_op(v.w, bias, c + 3, act);
      *reinterpret_cast<float4*>(out + i) = v;
    }
  } else {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < mn; i += stride) {
      float v = partial[i];
      for (int sp = 1; sp < splits; ++sp) v = __fadd_rn(v, partial[sp * mn + i]);
      out[i] = epilogue_op(v, bias, i % n, act);
    }
  }
}

// Skinny products (n <= 32, FFMA path): one warp per output row. Lane l accumulates
// the k indices l, l + 32, ... for every output column in registers, then a butterfly
// of shuffles sums each column and lane j stores column j. A rows are read coalesced;
// the small B stays in L1.
template <bool BT, int NMAX>
__global__ void __launch_bounds__(256)
gemm_skinny_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ c, int64_t m,
                   int64_t n, int64_t k, int64_t batches, BatchMap bm, const float* __restrict__ bias, int act) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int nn = static_cast<int>(n);
  for (int64_t rg = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); rg < batches * m;
       rg += warps) {
    const int64_t batch = rg / m, row = rg - batch * m;
    const float* ar = a + batch_off(batch, bm.shape, bm.lhs, bm.rank) + row * k;
    const float* bb = b + batch_off(batch, bm.shape, bm.rhs, bm.rank);
    float acc[NMAX];
#pragma unroll
    for (int j = 0; j < NMAX; ++j) acc[j] = 0.0f;
#pragma unroll 4
    for (int64_t kk = lane; kk < k; kk += 32) {
      const float av = __ldg(ar + kk);
#pragma unroll
      for (int j = 0; j < NMAX; ++j)
        if (j < nn) acc[j] = fmaf(av, BT ? __ldg(bb + j * k + kk) : __ldg(bb + kk * n + j), acc[j]);
    }
    float mine = 0.0f;
#pragma unroll
    for (int j = 0; j < NMAX; ++j) {
      if (j >= nn) break;
      float v = acc[j];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == j) mine = v;
    }
    if (lane < nn) c[(batch * m + row) * n + lane] = epilogue_op(mine, bias, lane, act);
  }
}

// ------------------------------------------------------------------ host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D map over [planes][rows][kp] float32, box {32, box_rows, 1}, 128-byte swizzle
// (with 32-byte atoms for MN-major tf32 operands: swizzle_atom32).
bool make_map(CUtensorMap* map, const float* base, int64_t planes, int64_t rows, int64_t kp, int box_rows,
              bool swizzle_atom32 = false) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kp), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(planes)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kp * 4), static_cast<cuuint64_t>(rows * kp * 4)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows), 1};
  const cuuint32_t elem[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle_atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D map over the output [batches][m][n] float32 for the pair kernel's TMA tile stores:
// 32 x 32 boxes in the 128-byte swizzle (the epilogue's staging image). n % 4 == 0 and c
// 16-byte aligned.
bool make_out_map(CUtensorMap* map, float* c, int64_t batches, int64_t m, int64_t n) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(m),
                              static_cast<cuuint64_t>(batches)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(n * 4), static_cast<cuuint64_t>(m * n * 4)};
  const cuuint32_t box[3] = {32, 32, 1};
  const cuuint32_t elem[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, c, dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Layout {
  int64_t kp;
  size_t off_flag, off_a, off_b, off_partial, total;
  int splits;    // split-K factor of the single-SM kernel (1: none)
  int sk_slots;  // stream-K partial slots of the CTA-pair kernel at off_partial (0: none)
};

// The workspace's first 1024 bytes: the inf / NaN flag (int at 0) and, from byte
// kSkCountOff, the stream-K counters (two per cluster), all zeroed by one memset per call.
constexpr size_t kSkCountOff = 64;
constexpr int kMaxSkSlots = static_cast<int>((1024 - kSkCountOff) / 8);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// CTA pairs (256 x 256 tiles, tcgen05 cta_group::2) once the tiles keep at least half
// of the SM pairs busy (a pair tile takes no longer than a single-SM 128 x 256 tile).
bool use_pair(int64_t m, int64_t n, int64_t batches, int sms) {
  const int64_t pair_tiles = batches * ceil_div(m, 2 * kHalf) * ceil_div(n, kBN);
  return m >= 2 * kHalf && n >= kBN && pair_tiles >= sms / 4;
}

// N tile of the single-SM kernel: 128 when 128 x 256 tiles would leave SMs without a
// tile (small products: more, smaller work items, each with half the epilogue) or when
// N <= 128 (a 256-wide tile would be half empty), else 256.
int single_bn(int64_t m, int64_t n, int64_t batches, int sms) {
  return n <= 128 || batches * ceil_div(m, kBM) * ceil_div(n, kBN) < sms ? 128 : kBN;
}

// Split-K factor for a single-batch product whose 128 x BN tiles fill less than half
// of the SMs: each split keeps >= 4 k-blocks, and tiles x splits stays within the SMs.
int split_count(int64_t m, int64_t n, int64_t kp, int64_t batches, int sms) {
  if (batches != 1 || use_pair(m, n, batches, sms)) return 1;
  const int64_t tiles = ceil_div(m, kBM) * ceil_div(n, single_bn(m, n, batches, sms));
  const int64_t num_kb = kp / kBK;
  if (2 * tiles > sms || num_kb < 8) return 1;
  const int64_t want = std::max<int64_t>(1, std::min<int64_t>(num_kb / 4, sms / tiles));
  const int64_t per = ceil_div(num_kb, want);
  return static_cast<int>(ceil_div(num_kb, per));  // no empty split
}

Layout tensor_layout(int64_t m, int64_t n, int64_t k, int64_t nba, int64_t nbb) {
  Layout l;
  l.kp = (k + kBK - 1) / kBK * kBK;
  l.off_flag = 0;
  l.off_a = 1024;
  l.off_b = align_up(l.off_a + static_cast<size_t>(2 * nba * m * l.kp) * 4, 1024);
  l.off_partial = align_up(l.off_b + static_cast<size_t>(2 * nbb * n * l.kp) * 4, 1024);
  l.splits = (nba == 1 && nbb == 1) ? split_count(m, n, l.kp, 1, sm_count()) : 1;
  // products that run on CTA pairs get one stream-K slot per cluster (judged on the
  // operand batches; a product that reaches the pair kernel only through broadcast
  // batches runs without stream-K)
  l.sk_slots = (l.splits == 1 && use_pair(m, n, std::max(nba, nbb), sm_count()))
                   ? std::min(sm_count() / 2, kMaxSkSlots) : 0;
  l.total = l.off_partial + (l.splits > 1 ? align_up(static_cast<size_t>(l.splits * m * n) * 4, 1024)
                                          : static_cast<size_t>(l.sk_slots) * kSkSlotFloats * 4);
  return l;
}

// Stream-K split of `tiles` pair tiles of kb k-blocks over `clusters` clusters: the number
// of tiles left to whole round-robin waves (dp_tiles; == tiles: no stream-K). Used only
// when the last wave would leave at least half of the clusters idle and the balance saves
// each cluster at least 16 k-blocks (the finishing epilogue's partial read costs about
// eight): the stream-K part is that partial wave plus one whole wave, so
// every range covers one to one and a half tiles, a tile spans at most two ranges, and
// the partial of a split tile is the first thing its cluster computes (the finishing
// cluster never waits for it). Measured on one B200: with fewer tiles than clusters, or a
// last wave more than half full, the finishing epilogue's extra partial read, and the
// clusters' loss of lock-step k positions (the operand panels fall out of L2 when they
// exceed it), cost as much as the balance gains.
int64_t sk_dp_tiles(int64_t tiles, int64_t kb, int64_t clusters) {
  const int64_t r = tiles % clusters;
  if (tiles <= clusters || r == 0 || 2 * r > clusters || (clusters - r) * kb < 16 * clusters) return tiles;
  const int64_t sk = r + clusters, un = sk * kb;
  for (int64_t c = 0; c < clusters; ++c) {
    const int64_t lo = sk_bound(c, un, clusters), hi = sk_bound(c + 1, un, clusters);
    const int64_t ta = lo / kb;
    if (lo % kb != 0 && hi >= (ta + 1) * kb && c - sk_first_source(c, ta, kb, un, clusters) > kMaxSkSources)
      return tiles;
  }
  return tiles - sk;
}

bool use_tensor(int64_t m, int64_t n, int64_t k, int path) {
  if (path == TCX_MATMUL_FFMA) return false;
  if (m == 0 || n == 0 || k == 0) return false;
  if (path == TCX_MATMUL_TENSOR) return true;
  return m >= 128 && n >= 128 && k >= 128 && static_cast<double>(m) * n >= 4.0 * kBM * kBN;
}

int collapse_batches(int64_t batches, const int64_t* shape, const int64_t* ls, const int64_t* rs, int rank,
                     BatchMap& bm) {
  bm.rank = 0;
  for (int a = 0; a < rank; ++a) {
    if (shape[a] == 1) continue;
    if (bm.rank > 0) {
      const int p = bm.rank - 1;
      if (bm.lhs[p] == ls[a] * shape[a] && bm.rhs[p] == rs[a] * shape[a]) {
        bm.shape[p] *= shape[a];
        bm.lhs[p] = ls[a];
        bm.rhs[p] = rs[a];
        continue;
      }
    }
    if (bm.rank == kMaxBatchRank) return invalid("matmul batch rank exceeds 8 after collapsing");
    bm.shape[bm.rank] = shape[a];
    bm.lhs[bm.rank] = ls[a];
    bm.rhs[bm.rank] = rs[a];
    ++bm.rank;
  }
  (void)batches;
  return TCX_OK;
}

}  // namespace
}  // namespace tcx

using namespace tcx;

namespace {
// Number of distinct operand batches = (largest offset / batch size) + 1.
int64_t distinct_batches(const BatchMap& bm, bool lhs, int64_t per) {
  if (per == 0) return 1;
  int64_t max_off = 0;
  for (int a = 0; a < bm.rank; ++a) max_off += (bm.shape[a] - 1) * (lhs ? bm.lhs[a] : bm.rhs[a]);
  return max_off / per + 1;
}

// ------------------------------------------------------------ tensor-path phases
// Split pre-pass of the left operand: nba matrices [m, k] -> hi/lo planes
// [2 * nba, m, kp] (K-major); raises *flag on inf / NaN.
void split_a(cudaStream_t s, const float* lhs, float* wa, int64_t nba, int64_t m, int64_t k, int64_t kp,
             int* flag, int sms) {
  const bool vec_a = k % 4 == 0 && reinterpret_cast<uintptr_t>(lhs) % 16 == 0;
  const int grid_a = static_cast<int>(std::min<int64_t>(ceil_div(nba * m * (kp / 4), 256 * 4), 16LL * sms));
  TimedLaunch timer("split_rows", s);
  if (vec_a) split_rows<true><<<grid_a, 256, 0, s>>>(lhs, wa, nba, m, k, kp, flag);
  else split_rows<false><<<grid_a, 256, 0, s>>>(lhs, wa, nba, m, k, kp, flag);
}

// Both pre-passes (split_a's and split_b's work) in one launch.
void split_both(cudaStream_t s, const float* lhs, float* wa, int64_t nba, int64_t m, const float* rhs, float* wb,
                int64_t nbb, int64_t n, int64_t k, int64_t kp, int* flag, bool kmajor, int sms) {
  const bool va = k % 4 == 0 && reinterpret_cast<uintptr_t>(lhs) % 16 == 0;
  const bool vb = (kmajor ? k : n) % 4 == 0 && reinterpret_cast<uintptr_t>(rhs) % 16 == 0;
  const int ga = static_cast<int>(std::min<int64_t>(ceil_div(nba * m * (kp / 4), 256 * 4), 16LL * sms));
  const int64_t b_work = kmajor ? ceil_div(nbb * n * (kp / 4), 256 * 4) : nbb * ceil_div(n, 128) * (kp / 32);
  const int gb = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(b_work, 16LL * sms)));
  TimedLaunch timer("split_pair", s);
  auto go = [&](auto kernel) { kernel<<<ga + gb, 256, 0, s>>>(lhs, wa, nba, m, rhs, wb, nbb, n, k, kp, flag, ga); };
  if (kmajor) {
    if (va) { if (vb) go(split_pair<true, true, true>); else go(split_pair<true, true, false>); }
    else { if (vb) go(split_pair<false, true, true>); else go(split_pair<false, true, false>); }
  } else {
    if (va) { if (vb) go(split_pair<true, false, true>); else go(split_pair<true, false, false>); }
    else { if (vb) go(split_pair<false, false, true>); else go(split_pair<false, false, false>); }
  }
}

// Split pre-pass of the right operand into K-major planes [2 * nbb, n, kp]: a row split
// when it is already K-major ([n][k], a linear weight or key matrix), else a transpose.
void split_b(cudaStream_t s, const float* rhs, float* wb, int64_t nbb, int64_t n, int64_t k, int64_t kp, int* flag,
             bool kmajor, int sms) {
  if (kmajor) {
    const bool vec_w = k % 4 == 0 && reinterpret_cast<uintptr_t>(rhs) % 16 == 0;
    const int grid_w = static_cast<int>(std::min<int64_t>(ceil_div(nbb * n * (kp / 4), 256 * 4), 16LL * sms));
    TimedLaunch timer("split_rows", s);
    if (vec_w) split_rows<true><<<grid_w, 256, 0, s>>>(rhs, wb, nbb, n, k, kp, flag);
    else split_rows<false><<<grid_w, 256, 0, s>>>(rhs, wb, nbb, n, k, kp, flag);
  } else {
    const bool vec_b = n % 4 == 0 && reinterpret_cast<uintptr_t>(rhs) % 16 == 0;
    const int64_t tiles = nbb * ceil_div(n, 128) * (kp / 32);
    const int grid_b = static_cast<int>(std::min<int64_t>(tiles, 16LL * sms));
    TimedLaunch timer("split_cols", s);
    if (vec_b) split_cols<true><<<grid_b, 256, 0, s>>>(rhs, wb, nbb, k, n, kp, flag);
    else split_cols<false><<<grid_b, 256, 0, s>>>(rhs, wb, nbb, k, n, kp, flag);
  }
}

// Raw-mode pre-pass: lo terms of A (na4 float4s) and B (nb4 float4s) in their own
// layouts, one launch (either count may be 0).
void split_lo_launch(cudaStream_t s, const float* a, float* wa, int64_t na4, const float* b, float* wb, int64_t nb4,
                     int* flag, int sms) {
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(na4 + nb4, 256 * 4), 16LL * sms)));
  TimedLaunch timer("split_lo", s);
  split_lo<<<grid, 256, 0, s>>>(reinterpret_cast<const float4*>(a), reinterpret_cast<float4*>(wa), na4,
                                reinterpret_cast<const float4*>(b), reinterpret_cast<float4*>(wb), nb4, flag);
}

// The tcgen05 GEMM over split planes, then the IEEE FFMA fallback that runs only when
// the pre-pass raised *flag (reading the original lhs / rhs). splits > 1 (single-SM
// kernel, one output batch) needs `partial`: splits * m * n floats of workspace.
int gemm_planes(cudaStream_t s, float* wa, float* wb, int64_t nba, int64_t nbb, int64_t m, int64_t n, int64_t k,
                int64_t kp, int64_t batches, const BatchMap& bm, float* output, const float* bias, int act, int* flag,
                const float* lhs, const float* rhs, bool rhs_kmajor, int sms, int splits = 1,
                float* partial = nullptr, bool raw = false, int sk_slots = 0) {
  const int64_t pair_tiles = batches * ceil_div(m, 2 * kHalf) * ceil_div(n, kBN);
  const bool pair = use_pair(m, n, batches, sms);
  const int bn = pair ? kBN : single_bn(m, n, batches, sms);
  if (pair || batches != 1 || !partial) splits = 1;
  alignas(64) CUtensorMap map_a, map_b, map_a_hi, map_b_hi;
  if (raw) {
    // A and its lo [nba][m][k], boxes of 32 k x 128 rows; B and its lo [nbb][k][n],
    // boxes of 32 columns x 32 k rows (one MN-major chunk); zeros past k and n
    if (!make_map(&map_a, wa, nba, m, k, kBM) || !make_map(&map_a_hi, lhs, nba, m, k, kBM) ||
        !make_map(&map_b, wb, nbb, k, n, kBK, true) || !make_map(&map_b_hi, rhs, nbb, k, n, kBK, true))
      return (set_error("cuTensorMapEncodeTiled failed"), TCX_INTERNAL);
  } else {
    if (!make_map(&map_a, wa, 2 * nba, m, kp, kBM) || !make_map(&map_b, wb, 2 * nbb, n, kp, pair ? kHalf : bn))
      return (set_error("cuTensorMapEncodeTiled failed"), TCX_INTERNAL);
    map_a_hi = map_a;
    map_b_hi = map_b;
  }

  static bool attr_done[64] = {false};
  static int pair_fit[64] = {0};  // co-resident pair clusters (stream-K waits need them all resident)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(gemm_tf32x3_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SingleTile<256>::kSmem) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_tf32x3_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SingleTile<128>::kSmem) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_tf32x3_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemm2Smem) !=
            cudaSuccess)
      return launch_status("gemm smem attribute");
    cudaLaunchConfig_t probe = {};
    probe.gridDim = dim3(2 * (sms / 2));
    probe.blockDim = dim3(kGemmThreads);
    probe.dynamicSmemBytes = kGemm2Smem;
    cudaLaunchAttribute pattr[1];
    pattr[0].id = cudaLaunchAttributeClusterDimension;
    pattr[0].val.clusterDim.x = 2;
    pattr[0].val.clusterDim.y = 1;
    pattr[0].val.clusterDim.z = 1;
    probe.attrs = pattr;
    probe.numAttrs = 1;
    int fit = 0;
    if (cudaOccupancyMaxActiveClusters(&fit, gemm_tf32x3_pair_kernel, &probe) != cudaSuccess) {
      cudaGetLastError();
      fit = 0;  // unknown: no stream-K
    }
    pair_fit[dev] = fit;
    attr_done[dev] = true;
  }
  const int sk_clusters = (dev >= 0 && dev < 64) ? std::min(pair_fit[dev], sms / 2) : 0;
  GemmArgs g;
  g.c = output;
  g.bias = bias;
  g.nonfinite = flag;
  g.err = device_error_word();
  g.m = m; g.n = n; g.k_elems = k;
  g.lhs_mk = m * k; g.rhs_kn = k * n;
  g.num_kb = static_cast<int32_t>(kp / kBK);
  g.tiles_m = static_cast<int32_t>(ceil_div(m, kBM));
  g.tiles_n = static_cast<int32_t>(ceil_div(n, bn));
  g.act = act;
  g.vec_store = (n % 4 == 0 && reinterpret_cast<uintptr_t>(output) % 16 == 0) ? 1 : 0;
  g.batches = batches;
  g.bm = bm;
  g.splits = std::max(1, splits);
  g.kb_per_split = static_cast<int32_t>(ceil_div(g.num_kb, g.splits));
  g.partial = partial;
  g.raw = raw ? 1 : 0;
  if (g.splits > 1) g.vec_store = (n % 4 == 0 && reinterpret_cast<uintptr_t>(partial) % 16 == 0) ? 1 : 0;
  g.dp_tiles = pair_tiles;
  g.sk_partial = nullptr;
  g.sk_count = nullptr;
  g.tma_out = 0;
  alignas(64) CUtensorMap map_c;
  memset(&map_c, 0, sizeof(map_c));
  if (g.splits > 1) {  // single-SM split-K: the stores go to the partial slices [splits][m][n]
    if (n % 4 == 0 && reinterpret_cast<uintptr_t>(partial) % 16 == 0 && make_out_map(&map_c, partial, g.splits, m, n))
      g.tma_out = 1;
  } else if (n % 4 == 0 && reinterpret_cast<uintptr_t>(output) % 16 == 0 &&
             make_out_map(&map_c, output, batches, m, n)) {
    g.tma_out = 1;
  }
  if (pair) {
    g.tiles_n = static_cast<int32_t>(ceil_div(n, kBN));
    g.tiles_m = static_cast<int32_t>(ceil_div(m, 2 * kHalf));
    int clusters = static_cast<int>(std::min<int64_t>(pair_tiles, sms / 2));
    // stream-K over the last waves' tiles: partial slots at `partial`, counters beside
    // the flag (both in the workspace, the counters zeroed with the flag)
    if (g.tma_out && partial && sk_clusters >= 1 && sk_slots >= sk_clusters) {
      const int64_t dp = sk_dp_tiles(pair_tiles, g.num_kb, sk_clusters);
      if (dp < pair_tiles) {
        g.dp_tiles = dp;
        g.sk_partial = partial;
        g.sk_count = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(flag) + kSkCountOff);
        clusters = sk_clusters;
      }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = kGemm2Smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // set-up overlaps the pre-pass
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    TimedLaunch timer("gemm_tf32x3", s);
    cudaLaunchKernelEx(&cfg, gemm_tf32x3_pair_kernel, map_a, map_b, map_a_hi, map_b_hi, map_c, g);
  } else {
    const int64_t work = batches * g.tiles_m * g.tiles_n * g.splits;
    const int grid = static_cast<int>(std::min<int64_t>(work, sms));
    TimedLaunch timer("gemm_tf32x3", s);
    // launched behind the pre-pass so that its set-up overlaps the pre-pass's tail
    if (bn == 128)
      launch_after(gemm_tf32x3_kernel<128>, grid, kGemmThreads, s, SingleTile<128>::kSmem, map_a, map_b, map_a_hi,
                   map_b_hi, map_c, g);
    else
      launch_after(gemm_tf32x3_kernel<256>, grid, kGemmThreads, s, SingleTile<256>::kSmem, map_a, map_b, map_a_hi,
                   map_b_hi, map_c, g);
  }
  if (int st = launch_status("tcgen05 matmul")) return st;
  if (g.splits > 1) {
    const int64_t mn = m * n;
    const bool vec = n % 4 == 0 && reinterpret_cast<uintptr_t>(output) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(partial) % 16 == 0;
    const int grid = static_cast<int>(std::min<int64_t>(ceil_div(vec ? mn / 4 : mn, 256), 4LL * sms));
    TimedLaunch timer("splitk_reduce", s);
    if (vec)
      launch_after(splitk_reduce<true>, grid, 256, s, 0, partial, output, mn, n, g.splits, bias, act, flag, lhs, rhs,
                   k, rhs_kmajor ? 1 : 0);
    else
      launch_after(splitk_reduce<false>, grid, 256, s, 0, partial, output, mn, n, g.splits, bias, act, flag, lhs, rhs,
                   k, rhs_kmajor ? 1 : 0);
    // the reduce kernel computes the IEEE product itself when the pre-pass saw inf / NaN
    return launch_status("split-K reduce");
  }
  // IEEE fallback for inputs with inf/NaN (idle unless the pre-pass raised the flag)
  const int64_t ftiles = batches * ceil_div(m, kFM) * ceil_div(n, kFN);
  const int fgrid = static_cast<int>(std::min<int64_t>(ftiles, 16LL * sms));
  {
    TimedLaunch timer("gemm_ffma_fallback", s);
    if (rhs_kmajor) launch_after(gemm_ffma_kernel<true>, fgrid, 256, s, 0, lhs, rhs, output, m, n, k, batches, bm, bias, act, flag, 1);
    else launch_after(gemm_ffma_kernel<false>, fgrid, 256, s, 0, lhs, rhs, output, m, n, k, batches, bm, bias, act, flag, 1);
  }
  return launch_status("matmul fallback");
}
}  // namespace

extern "C" {

size_t tcx_sm100_matmul_workspace_bytes(int64_t m, int64_t n, int64_t k, int64_t lhs_batches,
                                        int64_t rhs_batches, int path) {
  if (!use_tensor(m, n, k, path)) return 0;
  return tensor_layout(m, n, k, std::max<int64_t>(lhs_batches, 1), std::max<int64_t>(rhs_batches, 1)).total;
}

static int run_matmul(tcx_stream_t stream, const float* lhs, const float* rhs, float* output, int64_t m,
                      int64_t n, int64_t k, int64_t batches, const int64_t* batch_shape,
                      const int64_t* lhs_batch_strides, const int64_t* rhs_batch_strides, int32_t batch_rank,
                      const float* bias, int act, int path, void* workspace, size_t workspace_bytes,
                      bool rhs_kmajor) {
  clear_error();
  if (m < 0 || n < 0 || k < 0 || batches < 0 || batch_rank < 0) return invalid("negative matmul extents");
  if (act != TCX_ACT_NONE && act != TCX_ACT_SILU && act != TCX_ACT_RELU) return invalid("unsupported activation");
  if (path != TCX_MATMUL_AUTO && path != TCX_MATMUL_FFMA && path != TCX_MATMUL_TENSOR)
    return invalid("unknown matmul path");
  if (batch_rank > 0 && (!batch_shape || !lhs_batch_strides || !rhs_batch_strides))
    return invalid("missing matmul batch metadata");
  BatchMap bm;
  if (int st = collapse_batches(batches, batch_shape, lhs_batch_strides, rhs_batch_strides, batch_rank, bm)) return st;
  if (m == 0 || n == 0 || batches == 0) return TCX_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int sms = sm_count();

  if (!use_tensor(m, n, k, path)) {
    if (n <= 32) {
      const int grid = static_cast<int>(std::min<int64_t>(ceil_div(batches * m, 8), 64LL * sms));
      TimedLaunch timer("gemm_skinny", s);
      if (n <= 8) {
        if (rhs_kmajor) gemm_skinny_kernel<true, 8><<<grid, 256, 0, s>>>(lhs, rhs, output, m, n, k, batches, bm, bias, act);
        else gemm_skinny_kernel<false, 8><<<grid, 256, 0, s>>>(lhs, rhs, output, m, n, k, batches, bm, bias, act);
      } else if (n <= 16) {
        if (rhs_kmajor) gemm_skinny_kernel<true, 16><<<grid, 256, 0, s>>>(lhs, rhs, output, m, n, k, batches, bm, bias, act);
        else gemm_skinny_kernel<false, 16><<<grid, 256, 0, s>>>(lhs, rhs, output, m, n, k, batches, bm, bias, act);
      } else {
        if (rhs_kmajor) gemm_skinny_kernel<true, 32><<<grid, 256, 0, s>>>(lhs, rhs, output, m, n, k, batches, bm, bias, act);
        else gemm_skinny_kernel<false, 32><<<grid, 256, 0, s>>>(lhs, rhs, output, m, n, k, batches, bm, bias, act);
      }
      return launch_status("skinny matmul");
    }
    const int64_t tiles = batches * ceil_div(m, kFM) * ceil_div(n, kFN);
    const int grid = static_cast<int>(std::min<int64_t>(tiles, 16LL * sms));
    {
      TimedLaunch timer("gemm_ffma", s);
      if (rhs_kmajor) gemm_ffma_kernel<true><<<grid, 256, 0, s>>>(lhs, rhs, output, m, n, k, batches, bm, bias, act, nullptr, 0);
      else gemm_ffma_kernel<false><<<grid, 256, 0, s>>>(lhs, rhs, output, m, n, k, batches, bm, bias, act, nullptr, 0);
    }
    return launch_status("ffma matmul");
  }
  if (m > INT32_MAX / 2 || n > INT32_MAX / 2 || k > INT32_MAX / 2) return invalid("matmul extent too large for the tensor path");
  const int64_t nba = distinct_batches(bm, true, m * k), nbb = distinct_batches(bm, false, k * n);
  Layout lay = tensor_layout(m, n, k, nba, nbb);
  if (lay.splits > 1 && batches != 1) {
    lay.splits = 1;  // no split-K with several output batches
    lay.total = lay.off_partial;
  }
  if (workspace && workspace_bytes < lay.total && workspace_bytes >= lay.off_partial) {
    lay.splits = 1;  // a workspace sized without the split-K / stream-K area: neither
    lay.sk_slots = 0;
    lay.total = lay.off_partial;
  }
  if (!workspace || workspace_bytes < lay.total) return invalid("matmul workspace is missing or too small");
  if (reinterpret_cast<uintptr_t>(workspace) % 1024) return invalid("matmul workspace must be 1024-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* flag = reinterpret_cast<int*>(ws + lay.off_flag);
  float* wa = reinterpret_cast<float*>(ws + lay.off_a);
  float* wb = reinterpret_cast<float*>(ws + lay.off_b);
  if (2 * std::max(nba, nbb) > INT32_MAX) return invalid("too many operand batches for the tensor path");

  // the flag and, with stream-K slots, the stream-K counters beside it
  const size_t reset = lay.sk_slots > 0 ? kSkCountOff + 8 * static_cast<size_t>(lay.sk_slots) : sizeof(int);
  if (cudaMemsetAsync(flag, 0, reset, s) != cudaSuccess) return launch_status("matmul flag reset");
  // Raw mode (row-major B, K and N multiples of 4, 16-byte aligned operands): the GEMM
  // reads A and B themselves as the hi terms and the pre-pass writes only their lo
  // terms, in the operands' own layouts (8 B per element instead of 12, no transpose).
  // The lo arrays fit in the split planes' workspace areas.
  const bool raw = !rhs_kmajor && k % 4 == 0 && n % 4 == 0 && reinterpret_cast<uintptr_t>(lhs) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(rhs) % 16 == 0;
  if (raw) {
    split_lo_launch(s, lhs, wa, nba * m * k / 4, rhs, wb, nbb * k * n / 4, flag, sms);
  } else {
    split_both(s, lhs, wa, nba, m, rhs, wb, nbb, n, k, lay.kp, flag, rhs_kmajor, sms);
  }
  if (int st = launch_status("matmul split pre-pass")) return st;
  float* partial = (lay.splits > 1 || lay.sk_slots > 0) ? reinterpret_cast<float*>(ws + lay.off_partial) : nullptr;
  return gemm_planes(s, wa, wb, nba, nbb, m, n, k, lay.kp, batches, bm, output, bias, act, flag, lhs, rhs,
                     rhs_kmajor, sms, lay.splits, partial, raw, lay.sk_slots);
}

int tcx_sm100_matmul(tcx_stream_t stream, const float* lhs, const float* rhs, float* output, int64_t m,
                     int64_t n, int64_t k, int64_t batches, const int64_t* batch_shape,
                     const int64_t* lhs_batch_strides, const int64_t* rhs_batch_strides, int32_t batch_rank,
                     const float* bias, int act, int path, void* workspace, size_t workspace_bytes) {
  return run_matmul(stream, lhs, rhs, output, m, n, k, batches, batch_shape, lhs_batch_strides,
                    rhs_batch_strides, batch_rank, bias, act, path, workspace, workspace_bytes, false);
}

size_t tcx_sm100_linear_workspace_bytes(int64_t rows, int64_t in_features, int64_t out_features, int path) {
  return tcx_sm100_matmul_workspace_bytes(rows, out_features, in_features, 1, 1, path);
}

int tcx_sm100_linear(tcx_stream_t stream, const float* x, const float* w, const float* bias, float* output,
                     int64_t rows, int64_t in_features, int64_t out_features, int act, int path,
                     void* workspace, size_t workspace_bytes) {
  return run_matmul(stream, x, w, output, rows, out_features, in_features, 1, nullptr, nullptr, nullptr, 0, bias,
                    act, path, workspace, workspace_bytes, true);
}

}  // extern "C"

// ------------------------------------------------------------ host-buffer matmul
namespace {
constexpr int kHostSlots = 3;

struct HostPlan {
  int64_t chunk_m, chunks, kp;
  bool tensor;  // chunks run the tcgen05 path with B split once; else run_matmul per chunk
  size_t off_b, off_bp, off_bflag, off_a[kHostSlots], off_ap[kHostSlots], off_c[kHostSlots],
      off_flag[kHostSlots], off_ws, off_sk, ws_bytes, total;
  int sk_slots;  // stream-K slots shared by the chunks' GEMMs (they run one after another)
};

// Row chunks of A (and C). The PCIe uploads are the floor of the whole call; chunks
// of 256 rows keep each chunk's GEMM (B split once) about as long as the next chunk's
// upload, and keep the tail that nothing overlaps (the last GEMM and download) short.
// Measured at 8192^3 on one B200, the variants interleaved in one process: 256-row
// chunks 11.02-11.31 ms per call, 512 rows 11.25-11.64, 1024 rows 11.55, 128 rows 16.1
// (the per-chunk launches no longer hide behind the uploads).
HostPlan host_plan(int64_t m, int64_t n, int64_t k) {
  HostPlan p;
  p.chunk_m = m >= 2048 ? 256 : m;
  p.chunks = (m + p.chunk_m - 1) / p.chunk_m;
  p.kp = (k + kBK - 1) / kBK * kBK;
  p.tensor = use_tensor(p.chunk_m, n, k, TCX_MATMUL_AUTO);
  size_t off = 0;
  p.off_b = off;
  off = align_up(off + static_cast<size_t>(k * n) * 4, 1024);
  p.off_bp = p.off_bflag = off;
  if (p.tensor) {
    off = align_up(off + static_cast<size_t>(2 * n * p.kp) * 4, 1024);
    p.off_bflag = off;
    off += 1024;
  }
  for (int s = 0; s < kHostSlots; ++s) {
    p.off_a[s] = off;
    off = align_up(off + static_cast<size_t>(p.chunk_m * k) * 4, 1024);
    p.off_c[s] = off;
    off = align_up(off + static_cast<size_t>(p.chunk_m * n) * 4, 1024);
    p.off_ap[s] = p.off_flag[s] = off;
    if (p.tensor) {
      off = align_up(off + static_cast<size_t>(2 * p.chunk_m * p.kp) * 4, 1024);
      p.off_flag[s] = off;
      off += 1024;
    }
  }
  p.off_ws = off;
  p.ws_bytes = p.tensor ? 0 : tcx_sm100_matmul_workspace_bytes(p.chunk_m, n, k, 1, 1, TCX_MATMUL_AUTO);
  off = align_up(off + p.ws_bytes, 1024);
  p.off_sk = off;
  p.sk_slots = (p.tensor && use_pair(p.chunk_m, n, 1, sm_count())) ? std::min(sm_count() / 2, kMaxSkSlots) : 0;
  p.total = align_up(off + static_cast<size_t>(p.sk_slots) * kSkSlotFloats * 4, 1024);
  return p;
}

struct Streams {
  cudaStream_t in = nullptr, comp = nullptr, out = nullptr;
  cudaEvent_t b_ready = nullptr, a_ready = nullptr, c_ready = nullptr, a_free[kHostSlots] = {},
              c_free[kHostSlots] = {};
  cudaError_t create() {
    cudaError_t e = cudaSuccess;
    for (cudaStream_t* st : {&in, &comp, &out})
      if (e == cudaSuccess) e = cudaStreamCreateWithFlags(st, cudaStreamNonBlocking);
    for (cudaEvent_t* ev : {&b_ready, &a_ready, &c_ready})
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
    for (int i = 0; i < kHostSlots; ++i) {
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&a_free[i], cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c_free[i], cudaEventDisableTiming);
    }
    return e;
  }
  void release() {
    for (cudaEvent_t* ev : {&b_ready, &a_ready, &c_ready})
      if (*ev) cudaEventDestroy(*ev), *ev = nullptr;
    for (int i = 0; i < kHostSlots; ++i) {
      if (a_free[i]) cudaEventDestroy(a_free[i]), a_free[i] = nullptr;
      if (c_free[i]) cudaEventDestroy(c_free[i]), c_free[i] = nullptr;
    }
    for (cudaStream_t* st : {&in, &comp, &out})
      if (*st) cudaStreamDestroy(*st), *st = nullptr;
  }
  ~Streams() { release(); }
};

// The calling thread's upload / compute / download streams and events for the current
// device, created on its first call and kept until the thread ends (each call returns
// with all three streams idle, so the next call may reuse them as they are).
Streams* host_streams() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return nullptr;
  }
  thread_local Streams lanes[64];
  thread_local bool made[64] = {};
  if (!made[dev]) {
    if (lanes[dev].create() != cudaSuccess) {
      cudaGetLastError();
      lanes[dev].release();
      return nullptr;
    }
    made[dev] = true;
  }
  return &lanes[dev];
}
}  // namespace

extern "C" {

size_t tcx_sm100_matmul_host_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k < 0) return 0;
  return host_plan(m, n, k).total;
}

int tcx_sm100_matmul_host(const float* a_host, const float* b_host, float* c_host, int64_t m, int64_t n,
                          int64_t k, void* workspace, size_t workspace_bytes) {
  clear_error();
  if (m < 0 || n < 0 || k < 0) return invalid("negative matmul extents");
  if (m == 0 || n == 0) return TCX_OK;
  if (!c_host || (k > 0 && (!a_host || !b_host))) return invalid("missing host buffer");
  const HostPlan p = host_plan(m, n, k);
  if (!workspace || workspace_bytes < p.total) return invalid("matmul workspace is missing or too small");
  if (reinterpret_cast<uintptr_t>(workspace) % 1024) return invalid("matmul workspace must be 1024-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* b_dev = reinterpret_cast<float*>(ws + p.off_b);
  Streams* lane = host_streams();
  if (!lane) {
    set_error("matmul_host: could not create its streams and events");
    return TCX_INTERNAL;
  }
  Streams& st = *lane;
  auto fail = [](cudaError_t e, const char* what) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return TCX_INTERNAL;
  };
  if (k > 0) {
    if (cudaError_t e = cudaMemcpyAsync(b_dev, b_host, static_cast<size_t>(k * n) * 4, cudaMemcpyHostToDevice, st.in);
        e != cudaSuccess)
      return fail(e, "matmul_host B upload");
  }
  cudaEventRecord(st.b_ready, st.in);
  cudaStreamWaitEvent(st.comp, st.b_ready, 0);
  cudaStream_t comp = st.comp;
  const int sms = sm_count();
  float* b_planes = reinterpret_cast<float*>(ws + p.off_bp);
  int* b_flag = reinterpret_cast<int*>(ws + p.off_bflag);
  // raw mode as the device-buffer path takes it (the staging buffers are 1024-byte
  // aligned), so both paths run the same kernels and give identical results
  const bool raw = p.tensor && k % 4 == 0 && n % 4 == 0;
  // a chunk's flag area starts as a copy of B's: B's inf / NaN flag, then zeros (the
  // stream-K counters)
  const size_t flag_bytes = p.sk_slots > 0 ? kSkCountOff + 8 * static_cast<size_t>(p.sk_slots) : sizeof(int);
  if (p.tensor) {  // B's split pre-pass once, shared by every chunk
    if (cudaError_t e = cudaMemsetAsync(b_flag, 0, flag_bytes, comp); e != cudaSuccess)
      return fail(e, "matmul_host flag reset");
    if (raw) split_lo_launch(comp, nullptr, nullptr, 0, b_dev, b_planes, k * n / 4, b_flag, sms);
    else split_b(comp, b_dev, b_planes, 1, n, k, p.kp, b_flag, false, sms);
  }
  BatchMap one;
  one.rank = 0;
  for (int64_t i = 0; i < p.chunks; ++i) {
    const int slot = static_cast<int>(i % kHostSlots);
    const int64_t r0 = i * p.chunk_m;
    const int64_t rows = std::min<int64_t>(p.chunk_m, m - r0);
    float* a_dev = reinterpret_cast<float*>(ws + p.off_a[slot]);
    float* c_dev = reinterpret_cast<float*>(ws + p.off_c[slot]);
    // upload A chunk once the GEMM that last used this slot has finished with it
    if (i >= kHostSlots) cudaStreamWaitEvent(st.in, st.a_free[slot], 0);
    if (k > 0) {
      if (cudaError_t e = cudaMemcpyAsync(a_dev, a_host + r0 * k, static_cast<size_t>(rows * k) * 4,
                                          cudaMemcpyHostToDevice, st.in);
          e != cudaSuccess)
        return fail(e, "matmul_host A upload");
    }
    cudaEventRecord(st.a_ready, st.in);
    cudaStreamWaitEvent(comp, st.a_ready, 0);
    if (i >= kHostSlots) cudaStreamWaitEvent(comp, st.c_free[slot], 0);  // C slot downloaded
    if (p.tensor) {
      // the chunk's flag starts as B's (inf / NaN anywhere in B), then A's split adds to it
      float* a_planes = reinterpret_cast<float*>(ws + p.off_ap[slot]);
      int* flag = reinterpret_cast<int*>(ws + p.off_flag[slot]);
      if (cudaError_t e = cudaMemcpyAsync(flag, b_flag, flag_bytes, cudaMemcpyDeviceToDevice, comp); e != cudaSuccess)
        return fail(e, "matmul_host flag copy");
      if (raw) split_lo_launch(comp, a_dev, a_planes, rows * k / 4, nullptr, nullptr, 0, flag, sms);
      else split_a(comp, a_dev, a_planes, 1, rows, k, p.kp, flag, sms);
      if (int rc = launch_status("matmul_host split pre-pass")) return rc;
      float* sk_area = p.sk_slots > 0 ? reinterpret_cast<float*>(ws + p.off_sk) : nullptr;
      if (int rc = gemm_planes(comp, a_planes, b_planes, 1, 1, rows, n, k, p.kp, 1, one, c_dev, nullptr,
                               TCX_ACT_NONE, flag, a_dev, b_dev, false, sms, 1, sk_area, raw, p.sk_slots))
        return rc;
    } else {
      const int rc = run_matmul(reinterpret_cast<tcx_stream_t>(comp), a_dev, b_dev, c_dev, rows, n, k, 1, nullptr,
                                nullptr, nullptr, 0, nullptr, TCX_ACT_NONE, TCX_MATMUL_AUTO, ws + p.off_ws, p.ws_bytes,
                                false);
      if (rc != TCX_OK) return rc;
    }
    cudaEventRecord(st.a_free[slot], comp);
    cudaEventRecord(st.c_ready, comp);
    cudaStreamWaitEvent(st.out, st.c_ready, 0);
    if (cudaError_t e = cudaMemcpyAsync(c_host + r0 * n, c_dev, static_cast<size_t>(rows * n) * 4,
                                        cudaMemcpyDeviceToHost, st.out);
        e != cudaSuccess)
      return fail(e, "matmul_host C download");
    cudaEventRecord(st.c_free[slot], st.out);
  }
  if (cudaError_t e = cudaStreamSynchronize(st.out); e != cudaSuccess) return fail(e, "matmul_host synchronize");
  if (cudaError_t e = cudaStreamSynchronize(st.comp); e != cudaSuccess) return fail(e, "matmul_host synchronize");
  return launch_status("matmul_host");
}

}  // extern "C"

namespace tcx {
// In-library entry for composites (attention.cu): the matmul of tcx_sm100_matmul with
// the right operand optionally K-major ([batch..., n, k], the layout of a key matrix).
int matmul_run(cudaStream_t stream, const float* lhs, const float* rhs, float* output, int64_t m, int64_t n,
               int64_t k, int64_t batches, const int64_t* batch_shape, const int64_t* lhs_batch_strides,
               const int64_t* rhs_batch_strides, int32_t batch_rank, bool rhs_kmajor, void* workspace,
               size_t workspace_bytes) {
  return run_matmul(reinterpret_cast<tcx_stream_t>(stream), lhs, rhs, output, m, n, k, batches, batch_shape,
                    lhs_batch_strides, rhs_batch_strides, batch_rank, nullptr, TCX_ACT_NONE, TCX_MATMUL_AUTO,
                    workspace, workspace_bytes, rhs_kmajor);
}
}  // namespace tcx

namespace tcx {
void split_rows_planes(cudaStream_t s, const float* x, float* planes, int64_t nb, int64_t rows, int64_t k,
                       int64_t kp, int* flag) {
  split_a(s, x, planes, nb, rows, k, kp, flag, sm_count());
}
void split_rows_planes2(cudaStream_t s, const float* x1, float* planes1, int64_t nb1, int64_t rows1,
                        const float* x2, float* planes2, int64_t nb2, int64_t rows2, int64_t k, int64_t kp,
                        int* flag) {
  split_both(s, x1, planes1, nb1, rows1, x2, planes2, nb2, rows2, k, kp, flag, true, sm_count());
}
void split_cols_planes(cudaStream_t s, const float* x, float* planes, int64_t nb, int64_t k, int64_t n,
                       int64_t kp, int* flag) {
  split_b(s, x, planes, nb, n, k, kp, flag, false, sm_count());
}
void split_lo_planes(cudaStream_t s, const float* x, float* lo, int64_t n4, int* flag) {
  split_lo_launch(s, x, lo, n4, nullptr, nullptr, 0, flag, sm_count());
}
bool encode_planes_map(void* map, const float* base, int64_t planes, int64_t rows, int64_t kp, int box_rows,
                       bool mn_atom32) {
  return make_map(static_cast<CUtensorMap*>(map), base, planes, rows, kp, box_rows, mn_atom32);
}
}  // namespace tcx
