// Reductions of the tensor.cx hot path on sm_100a.
//
//  * Full-tensor and long-row reductions (sum / mean / max / min / argmax, float32
//    and int32): a two-stage, bandwidth-bound design. Stage 1 runs a fixed grid of
//    4 CTAs per SM; each CTA streams one contiguous chunk with 128-bit
//    non-allocating loads, 4 loads in flight per thread, and reduces it to one
//    16-byte record (warp shuffles, then shared memory). Stage 2 folds the records
//    of each row in a fixed tree order. Shape-fixed order => results are
//    deterministic run to run. Index-carrying keys keep the reference semantics:
//    the first NaN wins, both zeros compare equal, ties go to the lowest index
//    (cpu_math.cpp:48-54; cpu_backend.cpp:1184-1196).
//  * Ordered row reductions (float32 sum / mean where the CPU order must be kept
//    bit for bit, tests/python/test_cuda_primitives.py:114-125 of the reference):
//    32 rows per CTA staged through shared memory in coalesced 32x128 tiles, one
//    thread per row adding left to right.
//  * Strided axes and general multi-axis selections: one thread per output, walking
//    the reduction in the reference's index order (exact).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "ptx.cuh"

namespace tcx {
namespace {

constexpr int kStage1Threads = 512;
constexpr int kUnroll = 4;

enum Kind { kSumF = 0, kSumI = 1, kBestMax = 2, kBestMin = 3 };

// Max / min / argmax load the next kUnroll vectors before folding the current ones (their
// compare-and-select chain is serial), so a thread always has a batch of loads in
// flight; the sums keep their 16 independent accumulators and higher occupancy instead.
template <int K>
__host__ __device__ constexpr bool prefetch_kind() { return K == kBestMax || K == kBestMin; }

template <typename T>
__device__ __forceinline__ T max_identity() {
  if constexpr (std::is_same<T, float>::value) return -INFINITY;
  else return INT32_MIN;
}

// 128-bit streaming load into integer registers. The words stay integers end to end:
// routed through float registers, `bits ^ 0x80000000` may be folded into a float
// negation, which is free to canonicalize NaN payloads (and int32 words that look
// like NaNs), breaking both exact int32 keys and first-NaN-payload semantics.
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

struct Acc {
  float f[4 * kUnroll];
  uint32_t u[4 * kUnroll];
  uint32_t key;
  int64_t idx;
};

// Per-thread best element for max / min / argmax, tracked as a value plus a 32-bit
// offset from the chunk start: one compare and two selects per element. A thread
// visits its elements in increasing index order, so the strict compare keeps the
// first of equal values (and -0 == +0 compare equal). NaN is handled apart: the first
// NaN wins outright, and one check per four elements (their sum is NaN if any is NaN,
// or for +inf + -inf, which the exact slow path then rules out) keeps it off the
// common path. The exact order key (key_max / key_min) is formed once per thread.
template <int K, bool FP>
struct BestRun {
  using V = typename std::conditional<FP, float, int32_t>::type;
  V bv;
  int32_t bi = -1;          // offset of bv, -1 while nothing beat the identity
  int32_t first = -1;       // offset of the first element this thread saw
  int32_t nan_at = -1;      // offset of the first NaN, -1 if none
  __device__ BestRun() {
    if constexpr (FP) bv = (K == kBestMax) ? -INFINITY : INFINITY;
    else bv = (K == kBestMax) ? INT32_MIN : INT32_MAX;
  }
  __device__ __forceinline__ void one(uint32_t bits, int32_t off) {
    V v;
    if constexpr (FP) v = __uint_as_float(bits);
    else v = static_cast<int32_t>(bits);
    const bool better = (K == kBestMax) ? (v > bv) : (v < bv);
    bv = better ? v : bv;
    bi = better ? off : bi;
  }
  __device__ __forceinline__ void four(uint4 w, int32_t off) {
    if (first < 0) first = off;
    one(w.x, off + 0);
    one(w.y, off + 1);
    one(w.z, off + 2);
    one(w.w, off + 3);
    if constexpr (FP) {
      const float s = __fadd_rn(__fadd_rn(__uint_as_float(w.x), __uint_as_float(w.y)),
                                __fadd_rn(__uint_as_float(w.z), __uint_as_float(w.w)));
      if (s != s && nan_at < 0) {
        if (is_nan_bits(w.x)) nan_at = off;
        else if (is_nan_bits(w.y)) nan_at = off + 1;
        else if (is_nan_bits(w.z)) nan_at = off + 2;
        else if (is_nan_bits(w.w)) nan_at = off + 3;
      }
    }
  }
  __device__ __forceinline__ void single(uint32_t bits, int32_t off) {
    if (first < 0) first = off;
    one(bits, off);
    if constexpr (FP) {
      if (nan_at < 0 && is_nan_bits(bits)) nan_at = off;
    }
  }
  // (key, global index) of this thread's best; key 0 / INT64_MAX when it saw nothing.
  // The winning value's bits are still in bv (selects only); the chunk is read again
  // only for a NaN or when no element beat the identity.
  __device__ __forceinline__ void result(const uint32_t* chunk, int64_t base, uint32_t& key, int64_t& idx) const {
    int32_t at = nan_at >= 0 ? nan_at : (bi >= 0 ? bi : first);
    if (at < 0) { key = 0; idx = INT64_MAX; return; }
    uint32_t bits;
    if (nan_at < 0 && bi >= 0) {
      if constexpr (FP) bits = __float_as_uint(bv);
      else bits = static_cast<uint32_t>(bv);
    } else {
      bits = chunk[at];
    }
    key = (K == kBestMax) ? key_max(bits, FP) : key_min(bits, FP);
    idx = base + at;
  }
};

template <int K, bool FP>
__device__ __forceinline__ void take(Acc& a, int slot, uint32_t bits, int64_t index) {
  if (K == kSumF) {
    a.f[slot] = __fadd_rn(a.f[slot], __uint_as_float(bits));
  } else if (K == kSumI) {
    a.u[slot] += bits;
  } else {
    const uint32_t k = (K == kBestMax) ? key_max(bits, FP) : key_min(bits, FP);
    if (k > a.key || a.idx == INT64_MAX) {  // strict: earlier indices win ties within a thread
      a.key = k;
      a.idx = index;
    }
  }
}

__device__ __forceinline__ bool better(uint32_t ka, int64_t ia, uint32_t kb, int64_t ib) {
  // an empty slot (index INT64_MAX) never beats a real element
  return ka > kb || (ka == kb && ia < ib) || (ib == INT64_MAX && ia != INT64_MAX);
}

// Folds (sum or key/index) across the CTA in a fixed order; result in thread 0.
template <int K>
__device__ __forceinline__ void block_fold(uint32_t& bits, uint32_t& key, int64_t& idx) {
  __shared__ uint32_t s_bits[32], s_key[32];
  __shared__ int64_t s_idx[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const uint32_t ob = __shfl_xor_sync(0xffffffffu, bits, off);
    const uint32_t ok = __shfl_xor_sync(0xffffffffu, key, off);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, off);
    if (K == kSumF) bits = __float_as_uint(__fadd_rn(__uint_as_float(bits), __uint_as_float(ob)));
    else if (K == kSumI) bits += ob;
    else if (better(ok, oi, key, idx)) { key = ok; idx = oi; }
  }
  if (lane == 0) { s_bits[warp] = bits; s_key[warp] = key; s_idx[warp] = idx; }
  __syncthreads();
  if (warp == 0) {
    if (lane < nwarps) { bits = s_bits[lane]; key = s_key[lane]; idx = s_idx[lane]; }
    else { bits = K == kSumF ? __float_as_uint(0.0f) : 0u; key = 0; idx = INT64_MAX; }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const uint32_t ob = __shfl_xor_sync(0xffffffffu, bits, off);
      const uint32_t ok = __shfl_xor_sync(0xffffffffu, key, off);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, off);
      if (K == kSumF) bits = __float_as_uint(__fadd_rn(__uint_as_float(bits), __uint_as_float(ob)));
      else if (K == kSumI) bits += ob;
      else if (better(ok, oi, key, idx)) { key = ok; idx = oi; }
    }
  }
  __syncthreads();
}

// Stage 1: CTA (blockIdx.x, row) reduces elements [blockIdx.x*chunk, +chunk) of a
// row of `n` elements into part[row * gridDim.x + blockIdx.x]. `chunk` is a multiple
// of 4 so every chunk starts 16-byte aligned when VEC (row start aligned).
template <int K, bool FP, bool VEC>
__global__ void __launch_bounds__(kStage1Threads)
reduce_stage1(const uint32_t* __restrict__ x, int64_t rows, int64_t n, int64_t chunk,
              int64_t index_base, tcx_partial* __restrict__ part) {
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    const uint32_t* xr = x + row * n;
    const int64_t begin = static_cast<int64_t>(blockIdx.x) * chunk;
    const int64_t end = min(begin + chunk, n);
    Acc a;
#pragma unroll
    for (int s = 0; s < 4 * kUnroll; ++s) { a.f[s] = 0.0f; a.u[s] = 0u; }
    a.key = 0; a.idx = INT64_MAX;
    BestRun<K, FP> best;
    constexpr bool kBestKind = K == kBestMax || K == kBestMin;
    constexpr bool kPrefetch = prefetch_kind<K>();
    const int tid = threadIdx.x;
    int64_t tail_begin = begin;
    if (VEC && end > begin) {
      const uint4* xv = reinterpret_cast<const uint4*>(xr + begin);
      const int64_t nvec = (end - begin) >> 2;
      int64_t i = tid;
      uint4 v[kUnroll];
      if (kPrefetch && i + (kUnroll - 1) * kStage1Threads < nvec) {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) v[u] = ldg_stream(xv + i + u * kStage1Threads);
      }
      for (; i + (kUnroll - 1) * kStage1Threads < nvec; i += kUnroll * kStage1Threads) {
        uint4 nv[kUnroll];
        if (kPrefetch) {
          const int64_t ni = i + kUnroll * kStage1Threads;
          if (ni + (kUnroll - 1) * kStage1Threads < nvec) {
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) nv[u] = ldg_stream(xv + ni + u * kStage1Threads);
          }
        } else {
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) v[u] = ldg_stream(xv + i + u * kStage1Threads);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int64_t e = begin + 4 * (i + u * kStage1Threads) + index_base;
          if constexpr (kBestKind) {
            best.four(v[u], static_cast<int32_t>(4 * (i + u * kStage1Threads)));
          } else {
            take<K, FP>(a, 4 * u + 0, v[u].x, e + 0);
            take<K, FP>(a, 4 * u + 1, v[u].y, e + 1);
            take<K, FP>(a, 4 * u + 2, v[u].z, e + 2);
            take<K, FP>(a, 4 * u + 3, v[u].w, e + 3);
          }
        }
        if (kPrefetch) {
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) v[u] = nv[u];
        }
      }
      for (; i < nvec; i += kStage1Threads) {
        const uint4 v = ldg_stream(xv + i);
        const int64_t e = begin + 4 * i + index_base;
        if constexpr (kBestKind) {
          best.four(v, static_cast<int32_t>(4 * i));
        } else {
          take<K, FP>(a, 0, v.x, e + 0);
          take<K, FP>(a, 1, v.y, e + 1);
          take<K, FP>(a, 2, v.z, e + 2);
          take<K, FP>(a, 3, v.w, e + 3);
        }
      }
      tail_begin = begin + nvec * 4;
    }
    for (int64_t j = tail_begin + tid; j < end; j += kStage1Threads) {
      if constexpr (kBestKind) best.single(__ldg(xr + j), static_cast<int32_t>(j - begin));
      else take<K, FP>(a, 0, __ldg(xr + j), j + index_base);
    }

    if (row + gridDim.y >= rows) dependents_may_launch();  // this CTA's last row: its loads are done
    uint32_t bits = 0, key = a.key;
    int64_t idx = a.idx;
    if constexpr (kBestKind) best.result(xr + begin, begin + index_base, key, idx);
    if (K == kSumF) {
      // fixed pairwise order over the 16 accumulators
      float t[4 * kUnroll];
#pragma unroll
      for (int s = 0; s < 4 * kUnroll; ++s) t[s] = a.f[s];
#pragma unroll
      for (int w = 4 * kUnroll / 2; w > 0; w >>= 1)
#pragma unroll
        for (int s = 0; s < w; ++s) t[s] = __fadd_rn(t[s], t[s + w]);
      bits = __float_as_uint(t[0]);
    } else if (K == kSumI) {
      uint32_t s = 0;
#pragma unroll
      for (int q = 0; q < 4 * kUnroll; ++q) s += a.u[q];
      bits = s;
    }
    block_fold<K>(bits, key, idx);
    if (threadIdx.x == 0) {
      tcx_partial p;
      p.key = key;
      p.bits = bits;
      p.index = idx;
      part[row * gridDim.x + blockIdx.x] = p;
    }
  }
}

// Output modes of stage 2 and the rank combine.
enum OutMode { kOutValue = 0, kOutMean = 1, kOutIndex = 2, kOutRecord = 3 };

__device__ __forceinline__ void emit(int mode, const uint32_t* xr, int64_t index_base,
                                     uint32_t bits, uint32_t key, int64_t idx, int64_t count,
                                     bool sum_kind, void* out, int64_t slot) {
  if (mode == kOutRecord) {
    tcx_partial p;
    p.key = key;
    p.index = idx;
    p.bits = sum_kind ? bits : (idx == INT64_MAX ? 0u : xr[idx - index_base]);
    static_cast<tcx_partial*>(out)[slot] = p;
  } else if (mode == kOutIndex) {
    static_cast<int32_t*>(out)[slot] = static_cast<int32_t>(idx - index_base);
  } else if (mode == kOutMean) {
    static_cast<float*>(out)[slot] =
        count ? __fdiv_rn(__uint_as_float(bits), static_cast<float>(count)) : __int_as_float(0x7fc00000);
  } else {
    static_cast<uint32_t*>(out)[slot] = sum_kind ? bits : xr[idx - index_base];
  }
}

// Stage 2: one CTA per row folds that row's `nparts` records in a fixed order.
template <int K>
__global__ void __launch_bounds__(1024)
reduce_stage2(const tcx_partial* __restrict__ part, int nparts, int64_t rows, int64_t n,
              const uint32_t* __restrict__ x, int64_t index_base, int mode, void* out) {
  wait_for_prior_grid();
  dependents_may_launch();
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    uint32_t bits = K == kSumF ? __float_as_uint(0.0f) : 0u, key = 0;
    int64_t idx = INT64_MAX;
    // Each thread folds a strided subset in increasing order, then the CTA tree.
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
      const tcx_partial p = part[row * nparts + i];
      if (K == kSumF) bits = __float_as_uint(__fadd_rn(__uint_as_float(bits), __uint_as_float(p.bits)));
      else if (K == kSumI) bits += p.bits;
      else if (better(p.key, p.index, key, idx)) { key = p.key; idx = p.index; }
    }
    block_fold<K>(bits, key, idx);
    if (threadIdx.x == 0)
      emit(mode, x + row * n, index_base, bits, key, idx, n, K <= kSumI, out, row);
  }
}

// Folds per-rank records in rank order (one thread; nparts is the world size).
template <int K>
__global__ void combine_records(const tcx_partial* __restrict__ parts, int nparts,
                                int64_t total, int mode, void* out) {
  wait_for_prior_grid();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  uint32_t bits = K == kSumF ? __float_as_uint(0.0f) : 0u, key = 0, best_bits = 0;
  int64_t idx = INT64_MAX;
  for (int i = 0; i < nparts; ++i) {
    const tcx_partial p = parts[i];
    if (K == kSumF) bits = __float_as_uint(__fadd_rn(__uint_as_float(bits), __uint_as_float(p.bits)));
    else if (K == kSumI) bits += p.bits;
    else if (better(p.key, p.index, key, idx)) { key = p.key; idx = p.index; best_bits = p.bits; }
  }
  if (mode == kOutIndex) static_cast<int32_t*>(out)[0] = static_cast<int32_t>(idx);
  else if (mode == kOutMean)
    static_cast<float*>(out)[0] =
        total ? __fdiv_rn(__uint_as_float(bits), static_cast<float>(total)) : __int_as_float(0x7fc00000);
  else static_cast<uint32_t*>(out)[0] = K <= kSumI ? bits : best_bits;
}

// ------------------------------------------------- cross-GPU fold (peer memory)
// Mailbox of one rank: 2 slot sets (epoch parity) x world slots of 32 bytes: the
// sender's tcx_partial (16 B), then the epoch it belongs to (8 B).
constexpr int kMaxRanks = 64;
constexpr int kSlotBytes = 32;
constexpr uint64_t kDefaultExchangeWaitNs = 2000000000ull;  // 2 s

struct Mailboxes {
  char* box[kMaxRanks];  // each rank's mailbox, mapped into this process; own at [rank]
};

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Stage 2 of a sharded reduction fused with the exchange: the CTA folds this rank's
// stage-1 records (as reduce_stage2), thread 0 stores the rank's record into slot
// `rank` of every mailbox (peer stores over NVLink), releases it with the epoch at
// system scope, waits (bounded) for all ranks' epochs in its own mailbox and folds the
// records in rank order with the combine_records rule.
template <int K>
__global__ void __launch_bounds__(1024)
reduce_stage2_exchange(const tcx_partial* __restrict__ part, int nparts, const uint32_t* __restrict__ x,
                       int64_t index_base, Mailboxes mb, int rank, int world, uint64_t epoch, uint64_t limit_ns,
                       int64_t total, int mode, void* out, int* err) {
  wait_for_prior_grid();
  uint32_t bits = K == kSumF ? __float_as_uint(0.0f) : 0u, key = 0;
  int64_t idx = INT64_MAX;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
    const tcx_partial p = part[i];
    if (K == kSumF) bits = __float_as_uint(__fadd_rn(__uint_as_float(bits), __uint_as_float(p.bits)));
    else if (K == kSumI) bits += p.bits;
    else if (better(p.key, p.index, key, idx)) { key = p.key; idx = p.index; }
  }
  block_fold<K>(bits, key, idx);
  const bool sum_kind = K <= kSumI;
  const int64_t set = static_cast<int64_t>(epoch & 1) * world;
  __shared__ uint64_t s_rec[2];
  __shared__ int s_late;
  if (threadIdx.x == 0) {
    const uint32_t rec_bits = sum_kind ? bits : (idx == INT64_MAX ? 0u : x[idx - index_base]);
    s_rec[0] = static_cast<uint64_t>(key) | (static_cast<uint64_t>(rec_bits) << 32);
    s_rec[1] = static_cast<uint64_t>(idx);
    s_late = 0;
  }
  __syncthreads();
  // one thread per rank: store this rank's record into slot `rank` of rank r's mailbox
  // (a peer store over NVLink), release it with the epoch, then wait (bounded) for rank
  // r's record in this rank's own mailbox
  const char* mine = mb.box[rank] + set * kSlotBytes;
  if (threadIdx.x < world) {
    const int r = threadIdx.x;
    uint64_t* slot = reinterpret_cast<uint64_t*>(mb.box[r] + (set + rank) * kSlotBytes);
    asm volatile("st.global.v2.u64 [%0], {%1, %2};" ::"l"(slot), "l"(s_rec[0]), "l"(s_rec[1]) : "memory");
    st_release_sys(slot + 2, epoch);
    const uint64_t* flag = reinterpret_cast<const uint64_t*>(mine + r * kSlotBytes) + 2;
    const uint64_t start = ptx::globaltimer();
    while (ld_acquire_sys(flag) != epoch) {
      if (ptx::globaltimer() - start > limit_ns) {
        atomicExch(&s_late, 1);
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  if (s_late) record_device_error(err, 0x501);
  uint32_t fbits = K == kSumF ? __float_as_uint(0.0f) : 0u, fkey = 0, best_bits = 0;
  int64_t fidx = INT64_MAX;
  for (int r = 0; r < world; ++r) {
    const uint64_t* slot = reinterpret_cast<const uint64_t*>(mine + r * kSlotBytes);
    (void)ld_acquire_sys(slot + 2);  // pairs with rank r's release (its waiter saw the epoch)
    uint64_t lo, hi;
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(lo), "=l"(hi) : "l"(slot) : "memory");
    const uint32_t pkey = static_cast<uint32_t>(lo), pbits = static_cast<uint32_t>(lo >> 32);
    const int64_t pidx = static_cast<int64_t>(hi);
    if (K == kSumF) fbits = __float_as_uint(__fadd_rn(__uint_as_float(fbits), __uint_as_float(pbits)));
    else if (K == kSumI) fbits += pbits;
    else if (better(pkey, pidx, fkey, fidx)) { fkey = pkey; fidx = pidx; best_bits = pbits; }
  }
  if (mode == kOutIndex) static_cast<int32_t*>(out)[0] = static_cast<int32_t>(fidx);
  else if (mode == kOutMean)
    static_cast<float*>(out)[0] =
        total ? __fdiv_rn(__uint_as_float(fbits), static_cast<float>(total)) : __int_as_float(0x7fc00000);
  else static_cast<uint32_t*>(out)[0] = sum_kind ? fbits : best_bits;
}

// ---------------------------------------------------------------- ordered rows
constexpr int kRowsPerCta = 32, kTileCols = 128;

// One thread per row, left-to-right in float32 (sum/mean) or the reference's max.
template <typename T, int OP>  // OP: 0 sum, 1 max, 2 mean
__global__ void __launch_bounds__(256)
rows_ordered(const T* __restrict__ x, T* __restrict__ out, int64_t rows, int64_t n) {
  __shared__ T tile[kRowsPerCta][kTileCols + 1];
  for (int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRowsPerCta; row0 < rows;
       row0 += static_cast<int64_t>(gridDim.x) * kRowsPerCta) {
    T acc;
    bool seen_nan = false;
    acc = OP == 1 ? max_identity<T>() : static_cast<T>(0);
    for (int64_t c0 = 0; c0 < n; c0 += kTileCols) {
#pragma unroll
      for (int k = 0; k < kRowsPerCta * kTileCols / 256; ++k) {
        const int e = threadIdx.x + k * 256;
        const int r = e / kTileCols, c = e % kTileCols;
        const int64_t gr = row0 + r, gc = c0 + c;
        tile[r][c] = (gr < rows && gc < n) ? x[gr * n + gc] : static_cast<T>(0);
      }
      __syncthreads();
      if (threadIdx.x < kRowsPerCta) {
        const int r = threadIdx.x;
        const int cols = static_cast<int>(n - c0 < kTileCols ? n - c0 : kTileCols);
        for (int c = 0; c < cols; ++c) {
          const T v = tile[r][c];
          if (OP == 1) {
            if constexpr (std::is_same<T, float>::value) {
              if (!seen_nan) {
                if (isnan(v)) { acc = v; seen_nan = true; }
                else acc = (acc < v) ? v : acc;
              }
            } else {
              acc = (acc < v) ? v : acc;
            }
          } else {
            if constexpr (std::is_same<T, float>::value) acc = __fadd_rn(acc, v);
            else acc = static_cast<T>(static_cast<uint32_t>(acc) + static_cast<uint32_t>(v));
          }
        }
      }
      __syncthreads();
    }
    if (threadIdx.x < kRowsPerCta && row0 + threadIdx.x < rows) {
      if constexpr (std::is_same<T, float>::value) {
        if (OP == 2) acc = n ? __fdiv_rn(acc, static_cast<float>(n)) : __int_as_float(0x7fc00000);
      }
      out[row0 + threadIdx.x] = acc;
    }
  }
}

// Strided axis: one thread per (outer, inner) output, reduce in index order.
template <typename T, int OP>
__global__ void axis_strided(const T* __restrict__ x, T* __restrict__ out, int64_t outer,
                             int64_t reduce, int64_t inner) {
  const int64_t count = outer * inner;
  for (int64_t id = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; id < count;
       id += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t base = (id / inner) * reduce * inner + id % inner;
    T acc;
    acc = OP == 1 ? max_identity<T>() : static_cast<T>(0);
    for (int64_t r = 0; r < reduce; ++r) {
      const T v = x[base + r * inner];
      if (OP == 1) {
        if constexpr (std::is_same<T, float>::value) {
          if (isnan(v)) { acc = v; break; }
        }
        acc = (acc < v) ? v : acc;
      } else {
        if constexpr (std::is_same<T, float>::value) acc = __fadd_rn(acc, v);
        else acc = static_cast<T>(static_cast<uint32_t>(acc) + static_cast<uint32_t>(v));
      }
    }
    if constexpr (std::is_same<T, float>::value) {
      if (OP == 2) acc = reduce ? __fdiv_rn(acc, static_cast<float>(reduce)) : __int_as_float(0x7fc00000);
    }
    out[id] = acc;
  }
}

__device__ __forceinline__ int64_t meta_offset(int64_t index, const Meta& m, int begin, int end) {
  int64_t value = 0;
  for (int a = end - 1; a >= begin; --a) {
    const int64_t extent = m.v[2 * a];
    value += (index % extent) * m.v[2 * a + 1];
    index /= extent;
  }
  return value;
}

// ------------------------------------------------------ chunked strided axis
// [outer, reduce, inner] with few (outer, inner) outputs: the reduce axis is cut into
// `nchunks` pieces; one thread per (outer, piece, inner) folds its piece in index order
// (coalesced along inner), then one thread per output folds the pieces in order with
// the same rule. Exact for int32 and for max (the first NaN and the first of equal
// values survive both folds); float sums are regrouped into pieces (deterministic).
template <typename T, int OP>  // OP: 0 sum, 1 max, 2 mean
__device__ __forceinline__ bool fold_one(T& acc, T v) {
  if (OP == 1) {
    if constexpr (std::is_same<T, float>::value) {
      if (isnan(v)) { acc = v; return true; }
    }
    acc = (acc < v) ? v : acc;
  } else {
    if constexpr (std::is_same<T, float>::value) acc = __fadd_rn(acc, v);
    else acc = static_cast<T>(static_cast<uint32_t>(acc) + static_cast<uint32_t>(v));
  }
  return false;
}

template <typename T, int OP, int W>  // W adjacent inner columns per thread (1 or 4)
__global__ void __launch_bounds__(256)
axis_chunks(const T* __restrict__ x, T* __restrict__ part, int64_t outer, int64_t reduce, int64_t inner,
            int64_t nchunks, int64_t chunk) {
  constexpr int kU = 8;  // rows in flight per thread
  const int64_t cols = inner / W;
  const int64_t items = outer * nchunks * cols;
  for (int64_t id = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; id < items;
       id += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t jw = id % cols, t = id / cols;
    const int64_t c = t % nchunks, o = t / nchunks;
    const int64_t r0 = c * chunk, r1 = min(r0 + chunk, reduce);
    const T* xp = x + (o * reduce + r0) * inner + jw * W;
    T acc[W];
    bool done[W];
#pragma unroll
    for (int w = 0; w < W; ++w) {
      acc[w] = OP == 1 ? max_identity<T>() : static_cast<T>(0);
      done[w] = false;
    }
    for (int64_t r = r0; r < r1; r += kU) {
      T v[kU][W];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (r + u < r1) {
          if constexpr (W == 4) {
            const auto q = *reinterpret_cast<const typename std::conditional<std::is_same<T, float>::value, float4, int4>::type*>(xp + u * inner);
            v[u][0] = q.x; v[u][1] = q.y; v[u][2] = q.z; v[u][3] = q.w;
          } else {
            v[u][0] = xp[u * inner];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (r + u < r1) {
#pragma unroll
          for (int w = 0; w < W; ++w)
            if (!done[w]) done[w] = fold_one<T, OP>(acc[w], v[u][w]);
        }
      }
      xp += kU * inner;
    }
#pragma unroll
    for (int w = 0; w < W; ++w) part[(o * nchunks + c) * inner + jw * W + w] = acc[w];
  }
}

template <typename T, int OP>
__global__ void __launch_bounds__(256)
axis_chunks_fold(const T* __restrict__ part, T* __restrict__ out, int64_t outer, int64_t reduce,
                 int64_t inner, int64_t nchunks) {
  const int64_t count = outer * inner;
  for (int64_t id = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; id < count;
       id += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t o = id / inner, j = id % inner;
    T acc;
    acc = OP == 1 ? max_identity<T>() : static_cast<T>(0);
    for (int64_t c = 0; c < nchunks; ++c)
      if (fold_one<T, OP>(acc, part[(o * nchunks + c) * inner + j])) break;
    if constexpr (std::is_same<T, float>::value) {
      if (OP == 2) acc = reduce ? __fdiv_rn(acc, static_cast<float>(reduce)) : __int_as_float(0x7fc00000);
    }
    out[id] = acc;
  }
}

// ------------------------------------------------------ chunked multi-axis
// General selections with long reductions: one warp per (group, piece of `chunk`
// reduction indices). Lanes take indices r = r0 + lane + 32 i; the innermost reduced
// axis is walked incrementally (coalesced when it is contiguous) and the other reduced
// axes are re-derived only when that axis wraps. Each warp leaves one 16-byte record
// (sum bits, or order key + index + bits), folded per group in piece order: exact for
// int32 and max (key order = the reference's first-NaN / first-of-equals rule), float
// sums regrouped (deterministic).
template <int K, bool FP, int V>  // V consecutive elements per lane and load (1, or 4 as a uint4)
__global__ void __launch_bounds__(256)
axes_chunks(const uint32_t* __restrict__ x, tcx_partial* __restrict__ part, int64_t groups, int64_t size,
            int64_t nchunks, int64_t chunk, Meta meta, int outer_rank) {
  const int lane = threadIdx.x & 31;
  const int64_t items = groups * nchunks;
  const int last = meta.rank - 1;
  const int64_t e_in = meta.v[2 * last], s_in = meta.v[2 * last + 1];
  constexpr int64_t kStep = 32 * V;
  for (int64_t item = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; item < items;
       item += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    const int64_t g = item / nchunks, c = item % nchunks;
    const int64_t base = meta_offset(g, meta, 0, outer_rank);
    const int64_t r0 = c * chunk, r1 = min(r0 + chunk, size);
    uint32_t bits = K == kSumF ? __float_as_uint(0.0f) : 0u, key = 0, best = 0;
    int64_t idx = INT64_MAX;
    auto fold = [&](uint32_t w, int64_t at) {
      if (K == kSumF) bits = __float_as_uint(__fadd_rn(__uint_as_float(bits), __uint_as_float(w)));
      else if (K == kSumI) bits += w;
      else {
        const uint32_t k = key_max(w, FP);
        if (k > key || idx == INT64_MAX) { key = k; idx = at; best = w; }
      }
    };
    int64_t r = r0 + V * lane;
    // one reduced axis besides the innermost, stepped by at most one index per load:
    // the walk carries into it with an add instead of re-deriving the offset
    const bool one_mid = last - outer_rank == 1 && kStep <= e_in;
    const int64_t s_mid = one_mid ? meta.v[2 * outer_rank + 1] : 0;
    if (r < r1) {
      int64_t q = r / e_in, p = r % e_in;
      int64_t run = base + meta_offset(q, meta, outer_rank, last);
      for (; r < r1; r += 4 * kStep) {
        // four addresses from the index walk, four loads in flight, then the folds
        uint32_t w[4][V];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (r + kStep * u < r1) {
            if constexpr (V == 4) {
              const uint4 t = *reinterpret_cast<const uint4*>(x + run + p);
              w[u][0] = t.x; w[u][1] = t.y; w[u][2] = t.z; w[u][3] = t.w;
            } else {
              w[u][0] = __ldg(x + run + p * s_in);
            }
          }
          p += kStep;
          if (p >= e_in) {
            if (one_mid) {
              p -= e_in;
              ++q;
              run += s_mid;
            } else {
              q += p / e_in;
              p %= e_in;
              run = base + meta_offset(q, meta, outer_rank, last);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t ru = r + kStep * u;
          if (ru >= r1) break;
#pragma unroll
          for (int e = 0; e < V; ++e) fold(w[u][e], ru + e);
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {  // fixed tree order across lanes
      const uint32_t ob = __shfl_xor_sync(0xffffffffu, bits, off);
      const uint32_t ok = __shfl_xor_sync(0xffffffffu, key, off);
      const uint32_t ow = __shfl_xor_sync(0xffffffffu, best, off);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, off);
      if (K == kSumF) bits = __float_as_uint(__fadd_rn(__uint_as_float(bits), __uint_as_float(ob)));
      else if (K == kSumI) bits += ob;
      else if (better(ok, oi, key, idx)) { key = ok; idx = oi; best = ow; }
    }
    if (lane == 0) {
      tcx_partial rec;
      rec.key = key;
      rec.bits = K <= kSumI ? bits : best;
      rec.index = idx;
      part[item] = rec;
    }
  }
}

template <int K>
__global__ void __launch_bounds__(256)
axes_chunks_fold(const tcx_partial* __restrict__ part, uint32_t* __restrict__ out, int64_t groups,
                 int64_t nchunks, int64_t size, int mean) {
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint32_t bits = K == kSumF ? __float_as_uint(0.0f) : 0u, key = 0, best = 0;
    int64_t idx = INT64_MAX;
    for (int64_t c = 0; c < nchunks; ++c) {
      const tcx_partial p = part[g * nchunks + c];
      if (K == kSumF) bits = __float_as_uint(__fadd_rn(__uint_as_float(bits), __uint_as_float(p.bits)));
      else if (K == kSumI) bits += p.bits;
      else if (better(p.key, p.index, key, idx)) { key = p.key; idx = p.index; best = p.bits; }
    }
    if (K <= kSumI) {
      out[g] = mean ? __float_as_uint(__fdiv_rn(__uint_as_float(bits), static_cast<float>(size))) : bits;
    } else {
      out[g] = best;
    }
  }
}

// General multi-axis sum/max/mean, one thread per output (cpu_backend.cpp:1123-1152).
template <typename T, int OP>
__global__ void reduce_axes_general(const T* __restrict__ x, T* __restrict__ out,
                                    int64_t groups, int64_t size, Meta meta, int outer_rank) {
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t base = meta_offset(g, meta, 0, outer_rank);
    T acc;
    acc = OP == 1 ? max_identity<T>() : static_cast<T>(0);
    for (int64_t r = 0; r < size; ++r) {
      const T v = x[base + meta_offset(r, meta, outer_rank, meta.rank)];
      if (OP == 1) {
        if constexpr (std::is_same<T, float>::value) {
          if (isnan(v)) { acc = v; break; }
        }
        acc = (acc < v) ? v : acc;
      } else {
        if constexpr (std::is_same<T, float>::value) acc = __fadd_rn(acc, v);
        else acc = static_cast<T>(static_cast<uint32_t>(acc) + static_cast<uint32_t>(v));
      }
    }
    if constexpr (std::is_same<T, float>::value) {
      if (OP == 2) acc = size ? __fdiv_rn(acc, static_cast<float>(size)) : __int_as_float(0x7fc00000);
    }
    out[g] = acc;
  }
}

// General min/argmax, one thread per output (cpu_math.cpp:48-54).
template <bool FP, bool ARGMAX>
__global__ void min_argmax_general(const uint32_t* __restrict__ x, uint32_t* __restrict__ out,
                                   int64_t groups, int64_t reduce, Meta meta) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < groups;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint32_t best = x[meta_offset(i * reduce, meta, 0, meta.rank)];
    uint32_t bkey = ARGMAX ? key_max(best, FP) : key_min(best, FP);
    int64_t index = 0;
    for (int64_t j = 1; j < reduce; ++j) {
      const uint32_t a = x[meta_offset(i * reduce + j, meta, 0, meta.rank)];
      const uint32_t k = ARGMAX ? key_max(a, FP) : key_min(a, FP);
      if (k > bkey) { best = a; bkey = k; index = j; }
    }
    out[i] = ARGMAX ? static_cast<uint32_t>(index) : best;
  }
}

__global__ void fill_word(uint32_t* out, uint32_t value) { *out = value; }


// ------------------------------------------------------------------- host side
int kind_of(int op, int dtype) {
  if (op == TCX_OP_SUM || op == TCX_OP_MEAN) return dtype == TCX_FLOAT32 ? kSumF : kSumI;
  if (op == TCX_OP_MAX || op == TCX_OP_ARGMAX) return kBestMax;
  return kBestMin;
}

struct Stage1Grid {
  int64_t chunk;
  int parts;
  int rows_y;
};

Stage1Grid stage1_grid(int64_t rows, int64_t n) {
  const int64_t target_ctas = 4LL * sm_count();
  int64_t per_row = rows >= target_ctas ? 1 : target_ctas / rows;
  per_row = std::max<int64_t>(1, std::min<int64_t>(per_row, ceil_div(n, 4096)));
  int64_t chunk = ceil_div(n, per_row);
  chunk = (chunk + 3) & ~int64_t(3);
  if (chunk == 0) chunk = 4;
  Stage1Grid g;
  g.chunk = chunk;
  g.parts = static_cast<int>(std::max<int64_t>(1, ceil_div(n, chunk)));
  g.rows_y = static_cast<int>(std::min<int64_t>(rows, 65535));
  return g;
}

size_t tree_workspace(int64_t rows, int64_t n) {
  const Stage1Grid g = stage1_grid(rows, n);
  return static_cast<size_t>(rows) * g.parts * sizeof(tcx_partial);
}

template <int K, bool FP>
void launch_stage1(cudaStream_t s, const uint32_t* x, int64_t rows, int64_t n, int64_t index_base,
                   tcx_partial* parts, const Stage1Grid& g) {
  const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (n % 4 == 0 || rows == 1);
  dim3 grid(g.parts, g.rows_y);
  TimedLaunch timer("reduce_stage1", s);
  if (vec) reduce_stage1<K, FP, true><<<grid, kStage1Threads, 0, s>>>(x, rows, n, g.chunk, index_base, parts);
  else reduce_stage1<K, FP, false><<<grid, kStage1Threads, 0, s>>>(x, rows, n, g.chunk, index_base, parts);
}

// Row-wise tree reduction of `rows` contiguous rows of `n` elements.
int tree_reduce(cudaStream_t s, int op, int dtype, const void* input, int64_t rows, int64_t n,
                int64_t index_base, int mode, void* out, void* ws, size_t ws_bytes) {
  const Stage1Grid g = stage1_grid(rows, n);
  const size_t need = static_cast<size_t>(rows) * g.parts * sizeof(tcx_partial);
  if (!ws || ws_bytes < need) return invalid("reduction workspace is missing or too small");
  if (g.chunk > INT32_MAX) return invalid("reduction chunk exceeds 2^31 elements");
  auto* parts = static_cast<tcx_partial*>(ws);
  const auto* x = static_cast<const uint32_t*>(input);
  const bool fp = dtype == TCX_FLOAT32;
  const int kind = kind_of(op, dtype);
  const int grid2 = static_cast<int>(std::min<int64_t>(rows, 65535));
  TimedLaunch timer("reduce_tree", s);
  switch (kind) {
    case kSumF:
      launch_stage1<kSumF, true>(s, x, rows, n, index_base, parts, g);
      launch_after(reduce_stage2<kSumF>, grid2, 1024, s, 0, parts, g.parts, rows, n, x, index_base, mode, out);
      break;
    case kSumI:
      launch_stage1<kSumI, false>(s, x, rows, n, index_base, parts, g);
      launch_after(reduce_stage2<kSumI>, grid2, 1024, s, 0, parts, g.parts, rows, n, x, index_base, mode, out);
      break;
    case kBestMax:
      if (fp) launch_stage1<kBestMax, true>(s, x, rows, n, index_base, parts, g);
      else launch_stage1<kBestMax, false>(s, x, rows, n, index_base, parts, g);
      launch_after(reduce_stage2<kBestMax>, grid2, 1024, s, 0, parts, g.parts, rows, n, x, index_base, mode, out);
      break;
    default:
      if (fp) launch_stage1<kBestMin, true>(s, x, rows, n, index_base, parts, g);
      else launch_stage1<kBestMin, false>(s, x, rows, n, index_base, parts, g);
      launch_after(reduce_stage2<kBestMin>, grid2, 1024, s, 0, parts, g.parts, rows, n, x, index_base, mode, out);
      break;
  }
  return launch_status("tree reduction");
}

int out_mode(int op) {
  if (op == TCX_OP_MEAN) return kOutMean;
  if (op == TCX_OP_ARGMAX) return kOutIndex;
  return kOutValue;
}

bool valid_reduce_op(int op, int dtype) {
  if (dtype != TCX_FLOAT32 && dtype != TCX_INT32) return false;
  switch (op) {
    case TCX_OP_SUM: case TCX_OP_MAX: case TCX_OP_MIN: case TCX_OP_ARGMAX: return true;
    case TCX_OP_MEAN: return dtype == TCX_FLOAT32;
    default: return false;
  }
}

int grid_for(int64_t work, int threads) {
  const int64_t blocks = ceil_div(std::max<int64_t>(work, 1), threads);
  return static_cast<int>(std::min<int64_t>(blocks, 32LL * sm_count()));
}

// True when the (extent, stride) pairs enumerate a contiguous buffer in order.
bool identity_metadata(const int64_t* meta, int rank) {
  int64_t expect = 1;
  for (int a = rank - 1; a >= 0; --a) {
    if (meta[2 * a] == 1) continue;
    if (meta[2 * a + 1] != expect) return false;
    expect *= meta[2 * a];
  }
  return true;
}

int load_meta(Meta& m, const int64_t* meta, int rank) {
  if (rank < 0 || rank > 2 * kMaxRank) return invalid("reduction metadata rank exceeds 32 axes");
  m.rank = rank;
  for (int i = 0; i < 2 * rank; ++i) m.v[i] = meta[i];
  return TCX_OK;
}

}  // namespace

// Pieces of a strided-axis reduction (1 = one thread per output): only when the
// outputs alone leave most of the GPU idle and each output has real work.
int64_t strided_chunks(int64_t outer, int64_t reduce, int64_t inner) {
  const int64_t count = outer * inner;
  if (inner <= 1 || count <= 0 || count >= 32768 || reduce < 256) return 1;
  // one wave of resident threads: axis_chunks holds 8 rows x 4 columns in flight per
  // thread (80 registers), 3 CTAs of 256 per SM; a thread covers 4 columns when inner % 4 == 0
  const int64_t target = 768LL * sm_count();
  const int64_t units = inner % 4 == 0 ? count / 4 : count;
  return std::max<int64_t>(1, std::min<int64_t>(ceil_div(reduce, 64), ceil_div(target, units)));
}

size_t axis_reduce_workspace(int64_t outer, int64_t reduce, int64_t inner) {
  if (inner != 1) {
    const int64_t pieces = strided_chunks(outer, reduce, inner);
    return pieces > 1 ? static_cast<size_t>(outer * pieces * inner) * 4 : 0;
  }
  if (reduce <= 65536 || outer >= 4096 || outer <= 0) return 0;
  return tree_workspace(outer, reduce);
}

// Shared by tcx_sm100_axis (rows.cu) and reduce_axes: sum/max/mean along one axis.
int axis_reduce(cudaStream_t s, int op, int dtype, const void* input, void* output,
                               int64_t outer, int64_t reduce, int64_t inner, void* ws,
                               size_t ws_bytes) {
  const int64_t count = outer * inner;
  if (count == 0) return TCX_OK;
  const bool f32 = dtype == TCX_FLOAT32;
  if (inner == 1) {
    const int64_t rows = outer;
    // Few long rows: the parallel tree (exact for int32 and max, 1e-5 for float sums).
    if (reduce > 65536 && rows < 4096 && ws) {
      const size_t need = tree_workspace(rows, reduce);
      if (ws_bytes >= need)
        return tree_reduce(s, op, dtype, input, rows, reduce, 0, out_mode(op), output, ws, ws_bytes);
    }
    const int grid = static_cast<int>(std::min<int64_t>(ceil_div(rows, kRowsPerCta), 65535LL * 16));
    TimedLaunch timer("rows_ordered", s);
    if (f32) {
      auto* x = static_cast<const float*>(input);
      auto* o = static_cast<float*>(output);
      if (op == TCX_OP_SUM) rows_ordered<float, 0><<<grid, 256, 0, s>>>(x, o, rows, reduce);
      else if (op == TCX_OP_MAX) rows_ordered<float, 1><<<grid, 256, 0, s>>>(x, o, rows, reduce);
      else rows_ordered<float, 2><<<grid, 256, 0, s>>>(x, o, rows, reduce);
    } else {
      auto* x = static_cast<const int32_t*>(input);
      auto* o = static_cast<int32_t*>(output);
      if (op == TCX_OP_SUM) rows_ordered<int32_t, 0><<<grid, 256, 0, s>>>(x, o, rows, reduce);
      else rows_ordered<int32_t, 1><<<grid, 256, 0, s>>>(x, o, rows, reduce);
    }
    return launch_status("ordered row reduction");
  }
  const int64_t pieces = strided_chunks(outer, reduce, inner);
  if (pieces > 1 && ws && ws_bytes >= static_cast<size_t>(outer * pieces * inner) * 4) {
    const int64_t chunk = ceil_div(reduce, pieces);
    const bool vec = inner % 4 == 0 && reinterpret_cast<uintptr_t>(input) % 16 == 0;
    const int grid1 = grid_for(outer * pieces * (vec ? inner / 4 : inner), 256), grid2 = grid_for(count, 256);
    TimedLaunch timer("axis_chunks", s);
    auto run = [&](auto zero, auto op_tag) {
      using T = decltype(zero);
      constexpr int OP = decltype(op_tag)::value;
      constexpr int FOLD = OP;
      const T* x = static_cast<const T*>(input);
      T* part = static_cast<T*>(ws);
      T* o = static_cast<T*>(output);
      if (vec) axis_chunks<T, OP == 2 ? 0 : OP, 4><<<grid1, 256, 0, s>>>(x, part, outer, reduce, inner, pieces, chunk);
      else axis_chunks<T, OP == 2 ? 0 : OP, 1><<<grid1, 256, 0, s>>>(x, part, outer, reduce, inner, pieces, chunk);
      axis_chunks_fold<T, FOLD><<<grid2, 256, 0, s>>>(part, o, outer, reduce, inner, pieces);
    };
    if (f32) {
      if (op == TCX_OP_MAX) run(0.0f, std::integral_constant<int, 1>());
      else if (op == TCX_OP_SUM) run(0.0f, std::integral_constant<int, 0>());
      else run(0.0f, std::integral_constant<int, 2>());
    } else {
      if (op == TCX_OP_MAX) run(int32_t(0), std::integral_constant<int, 1>());
      else run(int32_t(0), std::integral_constant<int, 0>());
    }
    return launch_status("chunked strided axis reduction");
  }
  const int grid = grid_for(count, 256);
  TimedLaunch timer("axis_strided", s);
  if (f32) {
    auto* x = static_cast<const float*>(input);
    auto* o = static_cast<float*>(output);
    if (op == TCX_OP_SUM) axis_strided<float, 0><<<grid, 256, 0, s>>>(x, o, outer, reduce, inner);
    else if (op == TCX_OP_MAX) axis_strided<float, 1><<<grid, 256, 0, s>>>(x, o, outer, reduce, inner);
    else axis_strided<float, 2><<<grid, 256, 0, s>>>(x, o, outer, reduce, inner);
  } else {
    auto* x = static_cast<const int32_t*>(input);
    auto* o = static_cast<int32_t*>(output);
    if (op == TCX_OP_SUM) axis_strided<int32_t, 0><<<grid, 256, 0, s>>>(x, o, outer, reduce, inner);
    else axis_strided<int32_t, 1><<<grid, 256, 0, s>>>(x, o, outer, reduce, inner);
  }
  return launch_status("strided axis reduction");
}


}  // namespace tcx

using namespace tcx;

extern "C" {

size_t tcx_sm100_reduce_workspace_bytes(int64_t count) {
  // Upper bound of tree_workspace(rows, n) over every split rows * n == count that
  // runs the tree (n >= 1024): fewer rows than the CTA target use at most that many
  // records; more rows use one record per row.
  // (chunked multi-axis selections need at most count / 1024 + groups records, with
  // groups <= count / 2048: covered by 2 * count / 1024.)
  const int64_t records = std::max<int64_t>(4LL * sm_count(), 2 * (count / 1024) + 1);
  return static_cast<size_t>(records) * sizeof(tcx_partial);
}

int tcx_sm100_reduce_all(tcx_stream_t stream, int op, int dtype, const void* input,
                         int64_t count, void* output, void* workspace, size_t workspace_bytes) {
  clear_error();
  if (!valid_reduce_op(op, dtype)) return invalid("unsupported full reduction op/dtype");
  if (count < 0) return invalid("negative element count");
  if (count == 0) {
    if (op == TCX_OP_MAX || op == TCX_OP_MIN || op == TCX_OP_ARGMAX)
      return invalid("reduction requires a non-empty input");
    // sum of nothing is 0, mean of nothing is NaN (cpu_backend.cpp:1146-1147)
    TimedLaunch timer("fill_word", reinterpret_cast<cudaStream_t>(stream));
    fill_word<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<uint32_t*>(output), op == TCX_OP_MEAN ? 0x7fc00000u : 0u);
    return launch_status("empty reduction");
  }
  if (op == TCX_OP_ARGMAX && count > INT32_MAX) return invalid("argmax index range exceeds int32");
  return tree_reduce(reinterpret_cast<cudaStream_t>(stream), op, dtype, input, 1, count, 0,
                     out_mode(op), output, workspace, workspace_bytes);
}

int tcx_sm100_reduce_partial(tcx_stream_t stream, int op, int dtype, const void* input,
                             int64_t count, int64_t index_base, tcx_partial* partial,
                             void* workspace, size_t workspace_bytes) {
  clear_error();
  if (!valid_reduce_op(op, dtype)) return invalid("unsupported partial reduction op/dtype");
  if (count <= 0) return invalid("partial reduction requires a non-empty shard");
  return tree_reduce(reinterpret_cast<cudaStream_t>(stream), op, dtype, input, 1, count, index_base,
                     kOutRecord, partial, workspace, workspace_bytes);
}

int tcx_sm100_reduce_combine(tcx_stream_t stream, int op, int dtype, const tcx_partial* partials,
                             int32_t nparts, int64_t total_count, void* output) {
  clear_error();
  if (!valid_reduce_op(op, dtype)) return invalid("unsupported combine op/dtype");
  if (nparts <= 0) return invalid("combine requires at least one record");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int mode = out_mode(op);
  TimedLaunch timer("reduce_combine", s);
  switch (kind_of(op, dtype)) {
    case kSumF: launch_after(combine_records<kSumF>, 1, 32, s, 0, partials, nparts, total_count, mode, output); break;
    case kSumI: launch_after(combine_records<kSumI>, 1, 32, s, 0, partials, nparts, total_count, mode, output); break;
    case kBestMax: launch_after(combine_records<kBestMax>, 1, 32, s, 0, partials, nparts, total_count, mode, output); break;
    default: launch_after(combine_records<kBestMin>, 1, 32, s, 0, partials, nparts, total_count, mode, output); break;
  }
  return launch_status("reduction combine");
}

size_t tcx_sm100_mailbox_bytes(int32_t world) {
  if (world <= 0 || world > kMaxRanks) return 0;
  return (static_cast<size_t>(2 * world * kSlotBytes) + 255) / 256 * 256;
}

int tcx_sm100_mailbox_create(int32_t world, void** mailbox, void* ipc_handle) {
  clear_error();
  if (world <= 0 || world > kMaxRanks) return invalid("mailbox world size must be in [1, 64]");
  if (!mailbox || !ipc_handle) return invalid("missing mailbox output");
  const size_t bytes = tcx_sm100_mailbox_bytes(world);
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return launch_status("mailbox allocation");
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return launch_status("mailbox setup");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle is 64 bytes");
  memcpy(ipc_handle, &h, sizeof(h));
  *mailbox = p;
  return TCX_OK;
}

int tcx_sm100_mailbox_open(const void* ipc_handle, void** peer_mailbox) {
  clear_error();
  if (!ipc_handle || !peer_mailbox) return invalid("missing mailbox handle");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  if (cudaIpcOpenMemHandle(peer_mailbox, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return launch_status("mailbox open (CUDA IPC)");
  return TCX_OK;
}

int tcx_sm100_mailbox_close(void* peer_mailbox) {
  clear_error();
  if (!peer_mailbox) return TCX_OK;
  if (cudaIpcCloseMemHandle(peer_mailbox) != cudaSuccess) return launch_status("mailbox close");
  return TCX_OK;
}

int tcx_sm100_mailbox_free(void* mailbox) {
  clear_error();
  if (!mailbox) return TCX_OK;
  if (cudaFree(mailbox) != cudaSuccess) return launch_status("mailbox free");
  return TCX_OK;
}

int tcx_sm100_reduce_sharded(tcx_stream_t stream, int op, int dtype, const void* input, int64_t count,
                             int64_t index_base, void* const* mailboxes, int32_t rank, int32_t world,
                             uint64_t epoch, uint64_t wait_limit_ns, int64_t total_count, void* output,
                             void* workspace, size_t workspace_bytes) {
  clear_error();
  if (!valid_reduce_op(op, dtype)) return invalid("unsupported sharded reduction op/dtype");
  if (count <= 0) return invalid("sharded reduction requires a non-empty shard");
  if (world <= 0 || world > kMaxRanks || rank < 0 || rank >= world) return invalid("rank / world out of range");
  if (epoch == 0) return invalid("exchange epochs start at 1");
  if (!mailboxes || !output) return invalid("missing mailboxes or output");
  Mailboxes mb = {};
  for (int r = 0; r < world; ++r) {
    if (!mailboxes[r]) return invalid("missing mailbox");
    mb.box[r] = static_cast<char*>(mailboxes[r]);
  }
  const Stage1Grid g = stage1_grid(1, count);
  const size_t need = static_cast<size_t>(g.parts) * sizeof(tcx_partial);
  if (!workspace || workspace_bytes < need) return invalid("reduction workspace is missing or too small");
  if (g.chunk > INT32_MAX) return invalid("reduction chunk exceeds 2^31 elements");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto* parts = static_cast<tcx_partial*>(workspace);
  const auto* x = static_cast<const uint32_t*>(input);
  const bool fp = dtype == TCX_FLOAT32;
  const int mode = out_mode(op);
  const uint64_t limit = wait_limit_ns ? wait_limit_ns : kDefaultExchangeWaitNs;
  int* err = device_error_word();
  // Two timer records: stage 1 (this rank's shard, HBM-bound) and the exchange
  // (record stores to every peer, the bounded wait for theirs, the rank-order fold),
  // so the time a call spends waiting on its peers shows on its own.
  const int kind = kind_of(op, dtype);
  {
    TimedLaunch timer("reduce_stage1", s);
    switch (kind) {
      case kSumF: launch_stage1<kSumF, true>(s, x, 1, count, index_base, parts, g); break;
      case kSumI: launch_stage1<kSumI, false>(s, x, 1, count, index_base, parts, g); break;
      case kBestMax:
        if (fp) launch_stage1<kBestMax, true>(s, x, 1, count, index_base, parts, g);
        else launch_stage1<kBestMax, false>(s, x, 1, count, index_base, parts, g);
        break;
      default:
        if (fp) launch_stage1<kBestMin, true>(s, x, 1, count, index_base, parts, g);
        else launch_stage1<kBestMin, false>(s, x, 1, count, index_base, parts, g);
        break;
    }
  }
  TimedLaunch timer("reduce_exchange", s);
  switch (kind) {
    case kSumF:
      launch_after(reduce_stage2_exchange<kSumF>, 1, 1024, s, 0, parts, g.parts, x, index_base, mb, rank, world, epoch, limit,
                                                      total_count, mode, output, err);
      break;
    case kSumI:
      launch_after(reduce_stage2_exchange<kSumI>, 1, 1024, s, 0, parts, g.parts, x, index_base, mb, rank, world, epoch, limit,
                                                      total_count, mode, output, err);
      break;
    case kBestMax:
      launch_after(reduce_stage2_exchange<kBestMax>, 1, 1024, s, 0, parts, g.parts, x, index_base, mb, rank, world, epoch,
                                                         limit, total_count, mode, output, err);
      break;
    default:
      launch_after(reduce_stage2_exchange<kBestMin>, 1, 1024, s, 0, parts, g.parts, x, index_base, mb, rank, world, epoch,
                                                         limit, total_count, mode, output, err);
      break;
  }
  return launch_status("sharded reduction");
}

int tcx_sm100_reduce_axes(tcx_stream_t stream, int op, int dtype, const void* input, void* output,
                          int64_t groups, int64_t reduction_size, const int64_t* index_metadata,
                          int32_t outer_rank, int32_t rank, void* workspace,
                          size_t workspace_bytes) {
  clear_error();
  if (op != TCX_OP_SUM && op != TCX_OP_MAX && op != TCX_OP_MEAN)
    return invalid("reduce_axes supports sum, max and mean");
  if (!valid_reduce_op(op, dtype)) return invalid("mean only supports float32 tensors");
  if (groups < 0 || reduction_size < 0 || outer_rank < 0 || outer_rank > rank)
    return invalid("malformed reduction plan");
  if (op == TCX_OP_MAX && reduction_size == 0) return invalid("max reduction requires non-empty axes");
  if (groups == 0) return TCX_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (rank > 0 && !index_metadata) return invalid("missing reduction metadata");
  // A selection whose metadata enumerates the buffer in order is `groups` contiguous
  // rows of `reduction_size`: the row kernels apply (all-axes is the 1-row case).
  if (reduction_size > 0 && identity_metadata(index_metadata, rank)) {
    if (groups == 1 && reduction_size > 65536)
      return tree_reduce(s, op, dtype, input, 1, reduction_size, 0, out_mode(op), output, workspace,
                         workspace_bytes);
    return axis_reduce(s, op, dtype, input, output, groups, reduction_size, 1,
                       workspace, workspace_bytes);
  }
  Meta meta;
  if (int st = load_meta(meta, index_metadata, rank)) return st;
  // long reductions over few groups: warps per (group, piece), records folded in order
  if (reduction_size >= 2048 && groups < 65536 && outer_rank < rank) {
    // about 8 waves of 8-warp CTAs (4 resident per SM): the last, partial wave costs
    // little, and a warp's piece stays >= 1024 elements
    const int64_t target = 256LL * sm_count();
    const int64_t pieces = std::max<int64_t>(1, std::min<int64_t>(ceil_div(reduction_size, 1024),
                                                                  ceil_div(target, groups)));
    const int last = rank - 1;
    // 16-byte loads when the innermost reduced axis is the contiguous last axis with an
    // extent divisible by 4 (every other stride is then a multiple of 4 as well)
    const bool vec = index_metadata[2 * last + 1] == 1 && index_metadata[2 * last] % 4 == 0 &&
                     reinterpret_cast<uintptr_t>(input) % 16 == 0;
    const int64_t chunk = vec ? ceil_div(ceil_div(reduction_size, pieces), 4) * 4 : ceil_div(reduction_size, pieces);
    const int64_t npieces = ceil_div(reduction_size, chunk);
    const size_t need = static_cast<size_t>(groups * npieces) * sizeof(tcx_partial);
    if (npieces > 1 && workspace && workspace_bytes >= need) {
      auto* part = static_cast<tcx_partial*>(workspace);
      const auto* x = static_cast<const uint32_t*>(input);
      auto* o = static_cast<uint32_t*>(output);
      // one (group, piece) per warp, CTAs scheduled as SMs free up
      const int grid1 = static_cast<int>(std::min<int64_t>(ceil_div(groups * npieces, 8), INT32_MAX));
      const int grid2 = grid_for(groups, 256);
      const bool fp = dtype == TCX_FLOAT32;
      TimedLaunch timer("axes_chunks", s);
      auto run = [&](auto kind_tag, auto fp_tag) {
        constexpr int K = decltype(kind_tag)::value;
        constexpr bool FP = decltype(fp_tag)::value;
        if (vec) axes_chunks<K, FP, 4><<<grid1, 256, 0, s>>>(x, part, groups, reduction_size, npieces, chunk, meta, outer_rank);
        else axes_chunks<K, FP, 1><<<grid1, 256, 0, s>>>(x, part, groups, reduction_size, npieces, chunk, meta, outer_rank);
        axes_chunks_fold<K><<<grid2, 256, 0, s>>>(part, o, groups, npieces, reduction_size, op == TCX_OP_MEAN);
      };
      using T0 = std::integral_constant<bool, false>;
      using T1 = std::integral_constant<bool, true>;
      if (op == TCX_OP_MAX) {
        if (fp) run(std::integral_constant<int, kBestMax>(), T1());
        else run(std::integral_constant<int, kBestMax>(), T0());
      } else if (fp) {
        run(std::integral_constant<int, kSumF>(), T1());
      } else {
        run(std::integral_constant<int, kSumI>(), T0());
      }
      return launch_status("chunked multi-axis reduction");
    }
  }
  const int grid = grid_for(groups, 256);
  TimedLaunch timer("reduce_axes_general", s);
  if (dtype == TCX_FLOAT32) {
    auto* x = static_cast<const float*>(input);
    auto* o = static_cast<float*>(output);
    if (op == TCX_OP_SUM) reduce_axes_general<float, 0><<<grid, 256, 0, s>>>(x, o, groups, reduction_size, meta, outer_rank);
    else if (op == TCX_OP_MAX) reduce_axes_general<float, 1><<<grid, 256, 0, s>>>(x, o, groups, reduction_size, meta, outer_rank);
    else reduce_axes_general<float, 2><<<grid, 256, 0, s>>>(x, o, groups, reduction_size, meta, outer_rank);
  } else {
    auto* x = static_cast<const int32_t*>(input);
    auto* o = static_cast<int32_t*>(output);
    if (op == TCX_OP_SUM) reduce_axes_general<int32_t, 0><<<grid, 256, 0, s>>>(x, o, groups, reduction_size, meta, outer_rank);
    else reduce_axes_general<int32_t, 1><<<grid, 256, 0, s>>>(x, o, groups, reduction_size, meta, outer_rank);
  }
  return launch_status("multi-axis reduction");
}

int tcx_sm100_min_argmax(tcx_stream_t stream, int op, int dtype, const void* input, void* output,
                         int64_t groups, int64_t reduction_size, const int64_t* index_metadata,
                         int32_t rank, void* workspace, size_t workspace_bytes) {
  clear_error();
  if (op != TCX_OP_MIN && op != TCX_OP_ARGMAX) return invalid("min_argmax supports min and argmax");
  if (dtype != TCX_FLOAT32 && dtype != TCX_INT32)
    return invalid("math operations require float32 or int32 tensors");
  if (reduction_size <= 0) return invalid("min/argmax require a non-empty reduction");
  if (op == TCX_OP_ARGMAX && reduction_size > INT32_MAX) return invalid("argmax index range exceeds int32");
  if (groups < 0) return invalid("malformed reduction plan");
  if (groups == 0) return TCX_OK;
  if (rank > 0 && !index_metadata) return invalid("missing reduction metadata");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool fp = dtype == TCX_FLOAT32;
  if (identity_metadata(index_metadata, rank) && reduction_size >= 1024) {
    // contiguous rows: parallel row reduction (exact: index-carrying keys)
    return tree_reduce(s, op, dtype, input, groups, reduction_size, 0, out_mode(op), output,
                       workspace, workspace_bytes);
  }
  Meta meta;
  if (int st = load_meta(meta, index_metadata, rank)) return st;
  const int grid = grid_for(groups, 256);
  TimedLaunch timer("min_argmax_general", s);
  auto* x = static_cast<const uint32_t*>(input);
  auto* o = static_cast<uint32_t*>(output);
  if (op == TCX_OP_ARGMAX) {
    if (fp) min_argmax_general<true, true><<<grid, 256, 0, s>>>(x, o, groups, reduction_size, meta);
    else min_argmax_general<false, true><<<grid, 256, 0, s>>>(x, o, groups, reduction_size, meta);
  } else {
    if (fp) min_argmax_general<true, false><<<grid, 256, 0, s>>>(x, o, groups, reduction_size, meta);
    else min_argmax_general<false, false><<<grid, 256, 0, s>>>(x, o, groups, reduction_size, meta);
  }
  return launch_status("min/argmax");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Full-tensor reduction without any allocation (no counterpart in the reference).
//
// For callers that may not allocate device memory at all: hosts that hand the whole
// GPU memory budget to their own allocator up front, or loops that cannot afford the
// device-wide synchronization cudaMalloc/cudaFree imply. The stage-1 records live in
// this fixed, file-scope device array instead of a caller-supplied workspace. Every
// device that loads the library holds the array (16 KiB) until the process exits.
namespace {
constexpr int kNoAllocRecords = 1024;
constexpr int kNoAllocMaxDevices = 64;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// The array's device address as last looked up on a device, and the id of the CUDA
// context it belongs to. A lookup that failed is not kept (the next call tries
// again), and an address whose context has since been destroyed and replaced (a
// device reset) is looked up anew, since the module, and with it the array, may now
// sit elsewhere.
struct NoAllocScratch {
  std::mutex mu;
  void* ptr = nullptr;
  unsigned long long context_id = 0;
};
NoAllocScratch g_noalloc[kNoAllocMaxDevices];

// Id of the calling thread's current context, or 0 when none is current or the
// driver offers no context ids.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}
}  // namespace

static __device__ __align__(256) tcx_partial tcx_noalloc_records[kNoAllocRecords];

extern "C" int tcx_sm100_reduce_all_noalloc(tcx_stream_t stream, int op, int dtype, const void* input,
                                            int64_t count, void* output) {
  clear_error();
  if (!valid_reduce_op(op, dtype)) return invalid("unsupported full reduction op/dtype");
  if (count < 0) return invalid("negative element count");
  if (op == TCX_OP_ARGMAX && count > INT32_MAX) return invalid("argmax index range exceeds int32");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return launch_status("cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices) return invalid("device index beyond the no-allocation table");
  // Set-up, with this device current: the host-side name of the array is only a
  // stand-in, so the kernels get the device address looked up here. It happens on
  // the first call on a device, and again only after that device's context changed.
  void* scratch = nullptr;
  {
    NoAllocScratch& slot = g_noalloc[dev];
    std::lock_guard<std::mutex> lock(slot.mu);
    const unsigned long long ctx = current_context_id();
    if (slot.ptr == nullptr || ctx == 0 || ctx != slot.context_id) {
      void* p = nullptr;
      const cudaError_t rc = cudaGetSymbolAddress(&p, tcx_noalloc_records);
      if (rc != cudaSuccess) {
        cudaGetLastError();
        slot.ptr = nullptr;  // not kept: the next call looks it up again
        set_error(std::string("cudaGetSymbolAddress(no-allocation scratch): ") + cudaGetErrorString(rc));
        return TCX_INTERNAL;
      }
      slot.ptr = p;
      slot.context_id = current_context_id();  // the lookup made the primary context current
    }
    scratch = slot.ptr;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (count == 0) {
    if (op == TCX_OP_MAX || op == TCX_OP_MIN || op == TCX_OP_ARGMAX)
      return invalid("reduction requires a non-empty input");
    fill_word<<<1, 1, 0, s>>>(static_cast<uint32_t*>(output), op == TCX_OP_MEAN ? 0x7fc00000u : 0u);
    return launch_status("empty reduction");
  }
  const size_t capacity = sizeof(tcx_partial) * kNoAllocRecords;
  const size_t need = tree_workspace(1, count);
  if (need > capacity)
    return invalid("input needs more partial records than the fixed no-allocation scratch holds (1024)");
  // Stage 1 writes every record stage 2 reads, so the previous call's contents never
  // leak into a result and nothing has to be cleared first.
  return tree_reduce(s, op, dtype, input, 1, count, 0, out_mode(op), output, scratch, capacity);
}
