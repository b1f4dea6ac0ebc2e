// Fused attention on sm_100a: O = softmax(scale * Q·Kᵀ) · V in one persistent,
// warp-specialized kernel, the scores and probabilities never leaving the SM.
//
// Two kernels. The single-SM kernel (masks, at most 128 queries, Dv 32 or 96, operands
// not 16-byte aligned) reads the 3xTF32 split planes (hi = rna_tf32(x),
// lo = rna_tf32(x - hi)) of Q [L, D], K [S, D] and Vᵀ [Dv, S], all K-major, made by the
// matmul pre-pass. The CTA-pair kernel below (the unmasked products over 128 queries)
// reads q, k and v in place and needs only K's lo terms from a pre-pass. One work item
// of the single-SM kernel is 128 queries of one batch, whose Q hi/lo stays in shared
// memory; key blocks of 64 are visited in order:
//   warp 0      TMA producer: the item's Q (D/32 pairs of 128x32 hi/lo tiles), then per
//               key block D/32 K hi/lo chunks (64x32) into a 2-deep ring and two Vᵀ
//               hi/lo chunks (Dv x 32) into another.
//   warp 1      S issuer, ahead of the softmax: S_j = Q·K_jᵀ into TMEM buffer j % 3
//               (three tcgen05.mma.kind::tf32 per 8-wide k step: lo·hi, hi·lo, hi·hi).
//   warp 6      P·V issuer: O += P_j·V_j once the softmax released P_j, with P read
//               straight from TMEM as the A operand, again as three products. Two
//               issuing threads keep the tensor pipe fed while either one waits on a
//               barrier (each wait costs its thread a few hundred cycles); the softmax
//               of block j overlaps the MMAs of blocks j+1 and j-1.
//   warps 2-5   softmax, one thread per query row (its TMEM lane): row maximum of the
//               scaled, causally masked scores (log2 domain), p = 2^(t - m), the row sum,
//               and p written back over S with tcgen05.st (the tensor core reads it as
//               tf32, the hi term) with p - trunc_tf32(p) beside it (the lo term). The
//               running maximum is raised only when a block's maximum exceeds it by more
//               than 8 (p stays <= 256), and only then is O (in TMEM) rescaled; at the end
//               O / sum is stored to HBM.
// TMEM (512 columns): buffer b in {0, 1, 2}: S / P_hi [128 b, 128 b + 64), P_lo
// [128 b + 64, 128 b + 128); O [384, 384 + Dv). Three buffers let S_{j+2} start while
// P_{j-1} is still being read, so the MMA issuer never drains the tensor pipe.
// Every wait is bounded (4 s of %globaltimer), with the same abort / drain / TMEM
// release discipline as the GEMM. No TMA multicast.
//
// Masks (the reference's kAttention mask input: bool, false = masked; or float32,
// added to the scaled scores, -inf = masked) are read inside the kernel: each softmax
// thread loads its row's 64 mask entries of the next key block while it waits for that
// block's S, through the mask's broadcast strides. A row with no unmasked key is all
// zeros, as in the reference.
//
// Non-finite inputs (flagged by the split pre-pass, by the pair kernel's converters and
// scan, and NaN / +inf in a float mask, flagged by a scan of the mask) hand the call to
// a row-wise IEEE kernel queued behind the fused one (idle otherwise), which computes
// the result the way the reference composite does (core/inference.cpp:123-160), mask
// included; the single-SM kernel exits at once when the pre-pass raised the flag.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "ptx.cuh"
#include "rowmath.cuh"

namespace tcx {
namespace {

using namespace ptx;

constexpr int kFQ = 128;     // queries per work item (MMA M)
constexpr int kFK = 64;      // keys per block (S tile N, P·V contraction per block)
constexpr int kFC = 32;      // one 128-byte swizzle row of float32: the TMA box width
constexpr int kKStages = 2;
constexpr int kVStages = 2;
constexpr int kMaxD = 128;
constexpr int kMaxDv = 128;
constexpr int kQTile = kFQ * kFC * 4;        // 16 KB: one 32-wide chunk of Q, hi or lo
constexpr int kQBytes = 2 * (kMaxD / kFC) * kQTile;  // 128 KB: all of Q hi/lo
constexpr int kKTile = kFK * kFC * 4;        // 8 KB
constexpr int kKStage = 2 * kKTile;          // 16 KB
constexpr int kVTileMax = kMaxDv * kFC * 4;  // 16 KB at Dv = 128
constexpr int kVStage = 2 * kVTileMax;       // 32 KB
constexpr int kFlashSmem = kQBytes + kKStages * kKStage + kVStages * kVStage + 1024 + 256;
constexpr int kFlashThreads = 224;
constexpr uint32_t kTmemCols = 512;
constexpr int kSBufs = 3;
constexpr uint32_t kColO = 384;
constexpr float kLog2e = 1.4426950408889634f;

__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

constexpr int kMaxFlashBatchRank = 30;  // the attention ABI's own batch-rank limit

struct FlashArgs {
  int64_t L, S;
  int32_t dp, dv;          // features (multiple of 32, <= 128) and value features (idem)
  int64_t batches;
  int32_t rank;            // merged batch rank; strides in matrix units (0 = broadcast)
  int64_t shape[kMaxFlashBatchRank], qs[kMaxFlashBatchRank], ks[kMaxFlashBatchRank], vs[kMaxFlashBatchRank];
  int32_t q_tiles, kv_blocks;
  float scale_log2;        // scale * log2(e)
  int32_t causal;
  int32_t vec8;            // out is 32-byte aligned: 32-byte stores
  float* out;              // [batches, L, dv]
  // mask (kind 1 bool, 2 float32): element strides per merged batch axis, along the
  // queries and along the keys (0 or 1); mask_vec: a row's 64 entries of a key block
  // may be read with 16-byte loads
  const void* mask;
  int64_t ms[kMaxFlashBatchRank];
  int64_t mq, mk;
  int32_t mask_vec;
  const int* nonfinite;
  int* err;
  // the CTA-pair kernel reads q, k, v in place ([planes][rows][features] float32,
  // 16-byte aligned), checks the Q and V tiles it loads for inf / NaN, scans the rows
  // [tail_row, S) of the v_planes V planes that no item loads, and raises *flag on a hit
  const float* v;
  int64_t v_planes;
  int64_t tail_row;
  int* flag;
  // the CTA-pair kernel's work units: items whole (kv_split == 0) or cut into units of
  // kv_split key blocks (when there are too few items for the SM pairs); a unit that is
  // not a whole item leaves its unnormalized O rows in part_o [units][256][dv] and each
  // row's reference maximum (log2 domain) and sum in part_ml [units][256][2], combined
  // by flash_combine_kernel
  int32_t kv_split;
  int64_t units;
  float* part_o;
  float* part_ml;
};

__device__ __forceinline__ void batch_planes(const FlashArgs& a, int64_t b, int64_t& pq, int64_t& pk, int64_t& pv) {
  pq = pk = pv = 0;
  for (int d = a.rank - 1; d >= 0; --d) {
    const int64_t i = b % a.shape[d];
    b /= a.shape[d];
    pq += i * a.qs[d];
    pk += i * a.ks[d];
    pv += i * a.vs[d];
  }
}

__device__ __forceinline__ int64_t mask_offset(const FlashArgs& a, int64_t b) {
  int64_t off = 0;
  for (int d = a.rank - 1; d >= 0; --d) {
    off += (b % a.shape[d]) * a.ms[d];
    b /= a.shape[d];
  }
  return off;
}

// One row's mask entries for key block [key0, key0 + 64): MK 1 as 64 keep bits (1 =
// unmasked), MK 2 as 64 biases already in log2 units (-inf = masked). Entries at or past
// `valid` are not read.
template <int MK>
struct MaskBlock {
  uint32_t keep[2];
  float bias[MK == 2 ? 64 : 1];
  __device__ __forceinline__ void load(const FlashArgs& a, int64_t row_off, int64_t key0, int valid) {
    if constexpr (MK == 1) {
      const unsigned char* m = static_cast<const unsigned char*>(a.mask) + row_off;
      if (a.mk == 0) {
        const uint32_t all = m[0] ? 0xffffffffu : 0u;
        keep[0] = keep[1] = all;
      } else if (a.mask_vec && valid == 64) {
        const uint4* v = reinterpret_cast<const uint4*>(m + key0);
        uint32_t bits[2] = {0u, 0u};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 w = __ldg(v + i);
          const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int byte = 0; byte < 4; ++byte)
              if ((words[j] >> (8 * byte)) & 0xffu) bits[i >> 1] |= 1u << (((i & 1) * 16) + j * 4 + byte);
        }
        keep[0] = bits[0];
        keep[1] = bits[1];
      } else {
        keep[0] = keep[1] = 0u;
        for (int e = 0; e < valid; ++e)
          if (m[key0 + e]) keep[e >> 5] |= 1u << (e & 31);
      }
    } else if constexpr (MK == 2) {
      const float* m = static_cast<const float*>(a.mask) + row_off;
      if (a.mk == 0) {
        const float v = __fmul_rn(m[0], kLog2e);
#pragma unroll
        for (int e = 0; e < 64; ++e) bias[e] = v;
      } else if (a.mask_vec && valid == 64) {
        const float4* v = reinterpret_cast<const float4*>(m + key0);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 w = __ldg(v + i);
          bias[4 * i] = __fmul_rn(w.x, kLog2e);
          bias[4 * i + 1] = __fmul_rn(w.y, kLog2e);
          bias[4 * i + 2] = __fmul_rn(w.z, kLog2e);
          bias[4 * i + 3] = __fmul_rn(w.w, kLog2e);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 64; ++e) bias[e] = e < valid ? __fmul_rn(m[key0 + e], kLog2e) : -INFINITY;
      }
    }
  }
  // the scaled score t of entry e with the mask applied
  __device__ __forceinline__ float apply(float t, int e) const {
    if constexpr (MK == 1) return (keep[e >> 5] >> (e & 31)) & 1u ? t : -INFINITY;
    else if constexpr (MK == 2) return bias[e] == -INFINITY ? -INFINITY : __fadd_rn(t, bias[e]);
    else return t;
  }
};

// Item of round r for this CTA: rounds alternate direction over the grid (a snake), so
// with items ordered longest first each CTA's total stays near the mean (causal items
// shrink with the query tile: round-robin leaves the busiest CTA 1.3x the mean on a
// 32 x 16-tile grid, the snake 1.05x). -1 when this CTA has no item in round r.
__device__ __forceinline__ int64_t snake_item(int64_t r, int64_t items) {
  const int64_t g = gridDim.x;
  const int64_t w = r * g + ((r & 1) ? g - 1 - blockIdx.x : blockIdx.x);
  return w < items ? w : -1;
}

// Work item w -> (batch, query tile); the longest causal items first.
__device__ __forceinline__ void item_coords(const FlashArgs& a, int64_t w, int64_t& b, int& qt, int& nkb) {
  qt = a.q_tiles - 1 - static_cast<int>(w / a.batches);
  b = w % a.batches;
  // causal: keys up to the tile's last query, (qt + 1) * 128 - 1
  nkb = a.causal ? min(a.kv_blocks, (qt + 1) * (kFQ / kFK)) : a.kv_blocks;
}

template <int MK>
__global__ void __launch_bounds__(kFlashThreads, 1)
flash_tf32x3_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, const FlashArgs a) {
  if (*a.nonfinite) return;  // the IEEE row kernel queued behind this one does the work
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_res = smem;                                   // chunk c: hi at 2c, lo at 2c + 1
  uint8_t* k_ring = smem + kQBytes;
  uint8_t* v_ring = k_ring + kKStages * kKStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(v_ring + kVStages * kVStage);
  uint64_t* k_full = bars;                       // [kKStages]
  uint64_t* k_empty = k_full + kKStages;         // [kKStages]
  uint64_t* v_full = k_empty + kKStages;         // [kVStages]
  uint64_t* v_empty = v_full + kVStages;         // [kVStages]
  uint64_t* s_full = v_empty + kVStages;         // [kSBufs] S of the block is in its TMEM buffer
  uint64_t* p_full = s_full + kSBufs;            // [kSBufs] P (and the rescaled O) are in TMEM
  uint64_t* pv_done = p_full + kSBufs;           // [kSBufs] P·V of the buffer's block has completed
  uint64_t* q_full = pv_done + kSBufs;           // the item's Q has landed
  uint64_t* q_empty = q_full + 1;                // the item's last S has read Q
  uint64_t* o_free = q_empty + 1;                // the item's O has been read out
  uint64_t* drain = o_free + 1;                  // [2]: the S issuer's and the P·V issuer's MMAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dchunks = a.dp / kFC;
  const uint32_t v_tile = static_cast<uint32_t>(a.dv) * kFC * 4;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kKStages; ++s) { mbar_init(smem_u32(&k_full[s]), 1); mbar_init(smem_u32(&k_empty[s]), 1); }
    for (int s = 0; s < kVStages; ++s) { mbar_init(smem_u32(&v_full[s]), 1); mbar_init(smem_u32(&v_empty[s]), 1); }
    for (int b = 0; b < kSBufs; ++b) {
      mbar_init(smem_u32(&s_full[b]), 1);
      mbar_init(smem_u32(&p_full[b]), 4);
      mbar_init(smem_u32(&pv_done[b]), 1);
    }
    mbar_init(smem_u32(q_full), 1);
    mbar_init(smem_u32(q_empty), 1);
    mbar_init(smem_u32(o_free), 4);
    mbar_init(smem_u32(&drain[0]), 1);
    mbar_init(smem_u32(&drain[1]), 1);
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
  const uint32_t tmem = *tmem_slot;
  const int64_t items = a.batches * a.q_tiles;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      int64_t k_n = 0, v_n = 0, local = 0;
      bool ok = true;
      for (int64_t r = 0; r * gridDim.x < items && ok; ++r) {
        const int64_t w = snake_item(r, items);
        if (w < 0) continue;
        int64_t b; int qt, nkb;
        item_coords(a, w, b, qt, nkb);
        int64_t pq, pk, pv;
        batch_planes(a, b, pq, pk, pv);
        // Q of this item, once the previous item's S products have read the old one
        if (!wait_bounded(smem_u32(q_empty), static_cast<uint32_t>(local & 1) ^ 1u, abort_flag, a.err, 0x400)) break;
        ++local;
        {
          const uint32_t fb = smem_u32(q_full);
          mbar_expect_tx(fb, static_cast<uint32_t>(2 * dchunks * kQTile));
          for (int c = 0; c < dchunks; ++c) {
            tma_load_3d(smem_u32(q_res + (2 * c) * kQTile), &map_q, fb, c * kFC, qt * kFQ, static_cast<int>(2 * pq));
            tma_load_3d(smem_u32(q_res + (2 * c + 1) * kQTile), &map_q, fb, c * kFC, qt * kFQ,
                        static_cast<int>(2 * pq + 1));
          }
        }
        // the MMA issuer's order: K_j, then V_{j-1} (its P·V follows S_j), V_last at the end
        auto load_k = [&](int j) {
          for (int c = 0; c < dchunks; ++c, ++k_n) {
            const int s = static_cast<int>(k_n % kKStages);
            const uint32_t ph = static_cast<uint32_t>((k_n / kKStages) & 1);
            if (!wait_bounded(smem_u32(&k_empty[s]), ph ^ 1u, abort_flag, a.err, 0x401)) return false;
            uint8_t* st = k_ring + s * kKStage;
            const uint32_t fb = smem_u32(&k_full[s]);
            mbar_expect_tx(fb, kKStage);
            tma_load_3d(smem_u32(st), &map_k, fb, c * kFC, j * kFK, static_cast<int>(2 * pk));
            tma_load_3d(smem_u32(st + kKTile), &map_k, fb, c * kFC, j * kFK, static_cast<int>(2 * pk + 1));
          }
          return true;
        };
        auto load_v = [&](int j) {
          for (int c = 0; c < kFK / kFC; ++c, ++v_n) {
            const int s = static_cast<int>(v_n % kVStages);
            const uint32_t ph = static_cast<uint32_t>((v_n / kVStages) & 1);
            if (!wait_bounded(smem_u32(&v_empty[s]), ph ^ 1u, abort_flag, a.err, 0x402)) return false;
            uint8_t* st = v_ring + s * kVStage;
            const uint32_t fb = smem_u32(&v_full[s]);
            mbar_expect_tx(fb, 2 * v_tile);
            tma_load_3d(smem_u32(st), &map_v, fb, j * kFK + c * kFC, 0, static_cast<int>(2 * pv));
            tma_load_3d(smem_u32(st + kVTileMax), &map_v, fb, j * kFK + c * kFC, 0, static_cast<int>(2 * pv + 1));
          }
          return true;
        };
        for (int j = 0; j < nkb && ok; ++j) {
          ok = load_k(j);
          if (ok && j >= 1) ok = load_v(j - 1);
        }
        if (ok && nkb >= 1) ok = load_v(nkb - 1);
      }
      if (!ok || *abort_flag) {  // every fill this thread issued must land before the CTA exits
        auto settle = [&](uint64_t* full, int stages, int64_t n, int site) {
          for (int s = 0; s < stages; ++s) {
            const int64_t fills = n > s ? (n - s + stages - 1) / stages : 0;
            if (!fills) continue;
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(smem_u32(&full[s]), static_cast<uint32_t>((fills - 1) & 1)))
              if (globaltimer() - t0 > kWaitLimitNs) { record_device_error(a.err, site); break; }
          }
        };
        settle(k_full, kKStages, k_n, 0x4f1);
        settle(v_full, kVStages, v_n, 0x4f2);
        settle(q_full, 1, local, 0x4f3);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- S = Q·Kᵀ issuer
      const uint32_t id_s = idesc_tf32(kFQ, kFK);
      int64_t k_n = 0, g = 0, local = 0;  // g: blocks issued by this CTA so far
      bool ok = true;
      for (int64_t r = 0; r * gridDim.x < items && ok; ++r) {
        const int64_t w = snake_item(r, items);
        if (w < 0) continue;
        int64_t b; int qt, nkb;
        item_coords(a, w, b, qt, nkb);
        if (!wait_bounded(smem_u32(q_full), static_cast<uint32_t>(local & 1), abort_flag, a.err, 0x410)) break;
        ++local;
        tc_fence_after();
        for (int j = 0; j < nkb && ok; ++j, ++g) {
          const int buf = static_cast<int>(g % kSBufs);
          if (g >= kSBufs) {  // S overwrites the buffer's previous P: that block's P·V must be done
            if (!wait_bounded(smem_u32(&pv_done[buf]), static_cast<uint32_t>(((g - kSBufs) / kSBufs) & 1), abort_flag, a.err,
                              0x412)) { ok = false; break; }
            tc_fence_after();
          }
          const uint32_t d_s = tmem + static_cast<uint32_t>(buf * 128);
          for (int c = 0; c < dchunks; ++c, ++k_n) {
            const int s = static_cast<int>(k_n % kKStages);
            const uint32_t ph = static_cast<uint32_t>((k_n / kKStages) & 1);
            if (!wait_bounded(smem_u32(&k_full[s]), ph, abort_flag, a.err, 0x413)) { ok = false; break; }
            tc_fence_after();
            const uint64_t dq_hi = smem_desc_sw128(smem_u32(q_res + (2 * c) * kQTile));
            const uint64_t dq_lo = smem_desc_sw128(smem_u32(q_res + (2 * c + 1) * kQTile));
            const uint64_t dk_hi = smem_desc_sw128(smem_u32(k_ring + s * kKStage));
            const uint64_t dk_lo = smem_desc_sw128(smem_u32(k_ring + s * kKStage + kKTile));
#pragma unroll
            for (int kk = 0; kk < kFC / 8; ++kk) {
              const uint32_t acc = (c == 0 && kk == 0) ? 0u : 1u;
              mma_tf32(d_s, dq_lo + 2 * kk, dk_hi + 2 * kk, id_s, acc);
              mma_tf32(d_s, dq_hi + 2 * kk, dk_lo + 2 * kk, id_s, 1u);
              mma_tf32(d_s, dq_hi + 2 * kk, dk_hi + 2 * kk, id_s, 1u);
            }
            mma_commit(smem_u32(&k_empty[s]));
          }
          if (!ok) break;
          mma_commit(smem_u32(&s_full[buf]));
          if (j == nkb - 1) mma_commit(smem_u32(q_empty));  // the item's Q is no longer read
        }
      }
    }
  } else if (warp == 6) {
    if (lane == 0) {
      // ------------------------------------------------------ O += P·V issuer
      // A second issuing thread: the tensor pipe takes its P·V products while the S
      // issuer waits on the K ring, and the S products while this one waits on V or P.
      const uint32_t id_o = idesc_tf32(kFQ, a.dv);
      const uint32_t d_o = tmem + kColO;
      int64_t v_n = 0, g = 0, local = 0;
      bool ok = true;
      for (int64_t r = 0; r * gridDim.x < items && ok; ++r) {
        const int64_t w = snake_item(r, items);
        if (w < 0) continue;
        int64_t b; int qt, nkb;
        item_coords(a, w, b, qt, nkb);
        const int64_t item = local++;
        for (int j = 0; j < nkb && ok; ++j, ++g) {
          const int buf = static_cast<int>(g % kSBufs);
          if (!wait_bounded(smem_u32(&p_full[buf]), static_cast<uint32_t>((g / kSBufs) & 1), abort_flag, a.err, 0x414)) {
            ok = false;
            break;
          }
          // the item's first P·V overwrites O: the previous item's O must have been read out
          if (j == 0 && !wait_bounded(smem_u32(o_free), static_cast<uint32_t>(item & 1) ^ 1u, abort_flag, a.err, 0x411)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t p_hi = tmem + static_cast<uint32_t>(buf * 128), p_lo = p_hi + kFK;
          for (int c = 0; c < kFK / kFC && ok; ++c, ++v_n) {
            const int s = static_cast<int>(v_n % kVStages);
            const uint32_t ph = static_cast<uint32_t>((v_n / kVStages) & 1);
            if (!wait_bounded(smem_u32(&v_full[s]), ph, abort_flag, a.err, 0x415)) { ok = false; break; }
            tc_fence_after();
            // descriptors built once per chunk; a k step adds 32 bytes (2 in the >> 4 field)
            const uint64_t dv_hi = smem_desc_sw128(smem_u32(v_ring + s * kVStage));
            const uint64_t dv_lo = smem_desc_sw128(smem_u32(v_ring + s * kVStage + kVTileMax));
#pragma unroll
            for (int kk = 0; kk < kFC / 8; ++kk) {
              const uint32_t col = static_cast<uint32_t>(c * kFC + kk * 8);
              const uint32_t acc = (j == 0 && c == 0 && kk == 0) ? 0u : 1u;
              mma_tf32_ta(d_o, p_lo + col, dv_hi + 2 * kk, id_o, acc);
              mma_tf32_ta(d_o, p_hi + col, dv_lo + 2 * kk, id_o, 1u);
              mma_tf32_ta(d_o, p_hi + col, dv_hi + 2 * kk, id_o, 1u);
            }
            mma_commit(smem_u32(&v_empty[s]));
          }
          if (!ok) break;
          mma_commit(smem_u32(&pv_done[buf]));
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax
    const int quarter = warp & 3;  // the TMEM lane quarter this warp may access
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int row_in_tile = quarter * 32 + lane;
    int64_t g = 0;
    for (int64_t r = 0; r * gridDim.x < items; ++r) {
      const int64_t w = snake_item(r, items);
      if (w < 0) continue;
      int64_t b; int qt, nkb;
      item_coords(a, w, b, qt, nkb);
      const int64_t query = static_cast<int64_t>(qt) * kFQ + row_in_tile;
      const bool row_ok = query < a.L;
      const int64_t mrow = MK ? mask_offset(a, b) + (row_ok ? query : 0) * a.mq : 0;
      float m_use = -INFINITY, l = 0.0f;
      bool aborted = false;
      for (int j = 0; j < nkb; ++j, ++g) {
        const int buf = static_cast<int>(g % kSBufs);
        const uint32_t col_s = static_cast<uint32_t>(buf * 128), col_lo = col_s + kFK;
        const int64_t key0 = static_cast<int64_t>(j) * kFK;
        // keys allowed for this row in this block: [0, lim)
        int64_t lim64 = a.S - key0;
        if (a.causal) lim64 = min(lim64, query - key0 + 1);
        const int lim = static_cast<int>(lim64 < 0 ? 0 : (lim64 > kFK ? kFK : lim64));
        // this row's mask entries of the block, loaded while S is still being computed
        MaskBlock<MK> mb;
        if constexpr (MK != 0) {
          const int64_t left = a.S - key0;
          mb.load(a, mrow, key0, row_ok ? static_cast<int>(left < kFK ? left : kFK) : 0);
        }
        if (!wait_bounded(smem_u32(&s_full[buf]), static_cast<uint32_t>((g / kSBufs) & 1), abort_flag, a.err, 0x421)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        // the block's 64 scores of this row, both halves loaded before one wait, kept in
        // registers for both passes (one TMEM round trip per block), scaled to log2 units
        uint32_t s0[32], s1[32];
        TCX_LD32(s0, tmem + lane_base + col_s);
        TCX_LD32(s1, tmem + lane_base + col_s + 32);
        TCX_WAIT_LD32(s0);
        TCX_TIE32(s1);
        // pass 1: the block's row maximum (log2 domain)
        float mxv[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four independent chains
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float t = mb.apply(__fmul_rn(__uint_as_float(s0[e]), a.scale_log2), e);
          s0[e] = __float_as_uint(t);
          if (e < lim) mxv[e & 3] = fmaxf(mxv[e & 3], t);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float t = mb.apply(__fmul_rn(__uint_as_float(s1[e]), a.scale_log2), 32 + e);
          s1[e] = __float_as_uint(t);
          if (32 + e < lim) mxv[e & 3] = fmaxf(mxv[e & 3], t);
        }
        const float mx = fmaxf(fmaxf(mxv[0], mxv[1]), fmaxf(mxv[2], mxv[3]));
        // raise the running maximum only when p would exceed 2^8; rescale O then
        const bool need = mx > m_use + 8.0f;
        float alpha = 1.0f;
        if (need) {
          alpha = j == 0 ? 0.0f : exp2f(m_use - mx);
          m_use = mx;
        }
        l = __fmul_rn(l, alpha);
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // O holds blocks < j only once the previous block's P·V has completed
          const int64_t gp = g - 1;
          if (!wait_bounded(smem_u32(&pv_done[gp % kSBufs]), static_cast<uint32_t>((gp / kSBufs) & 1), abort_flag, a.err,
                            0x423)) {
            aborted = true;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < a.dv; cc += 32) {
            uint32_t rr[32];
            TCX_LD32(rr, tmem + lane_base + kColO + cc);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int e = 0; e < 32; ++e) rr[e] = __float_as_uint(__fmul_rn(__uint_as_float(rr[e]), alpha));
            TCX_ST32(tmem + lane_base + kColO + cc, rr);
          }
        }
        // pass 2: p = 2^(t - m), the row sum, P_hi over S and P_lo beside it
        // The tensor core reads float32 operands as tf32 by dropping the low 13 mantissa
        // bits, so p itself is the hi term of the 3xTF32 split and p - trunc_tf32(p)
        // (exact) the lo term: no conversions (two per element were most of this loop's
        // time), at most 2^-20 of p lost against a rounded split.
        float lsum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        auto emit = [&](uint32_t (&sv)[32], int c0) {
          uint32_t lo[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float p = 0.0f;
            // masked entries (-inf) give 0, also while every earlier key was masked (m_use -inf)
            if (c0 + e < lim && (MK == 0 || __uint_as_float(sv[e]) != -INFINITY)) {
              asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(p) : "f"(__fsub_rn(__uint_as_float(sv[e]), m_use)));
            }
            lsum[e & 3] = __fadd_rn(lsum[e & 3], p);
            sv[e] = __float_as_uint(p);
            lo[e] = __float_as_uint(__fsub_rn(p, __uint_as_float(__float_as_uint(p) & 0xFFFFE000u)));
          }
          TCX_ST32(tmem + lane_base + col_s + c0, sv);
          TCX_ST32(tmem + lane_base + col_lo + c0, lo);
        };
        emit(s0, 0);
        emit(s1, 32);
        l = __fadd_rn(l, __fadd_rn(__fadd_rn(lsum[0], lsum[1]), __fadd_rn(lsum[2], lsum[3])));
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&p_full[buf]));
      }
      if (aborted) break;
      // the item's last P·V, then O / l to HBM
      const int64_t gl = g - 1;
      if (!wait_bounded(smem_u32(&pv_done[gl % kSBufs]), static_cast<uint32_t>((gl / kSBufs) & 1), abort_flag, a.err, 0x422))
        break;
      tc_fence_after();
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;  // no unmasked key: a zero row
      float* orow = a.out + (b * a.L + query) * a.dv;
      // O drained in 32-column chunks with the next chunk's TMEM load in flight
      const int nch = a.dv / 32;
      uint32_t o0[32], o1[32];
      TCX_LD32(o0, tmem + lane_base + kColO);
#pragma unroll
      for (int ci = 0; ci < kMaxDv / 32; ++ci) {
        if (ci >= nch) break;
        uint32_t (&cur)[32] = (ci & 1) ? o1 : o0;
        uint32_t (&nxt)[32] = (ci & 1) ? o0 : o1;
        TCX_WAIT_LD32(cur);
        if (ci + 1 < nch) TCX_LD32(nxt, tmem + lane_base + kColO + static_cast<uint32_t>((ci + 1) * 32));
        if (row_ok) {
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __fmul_rn(__uint_as_float(cur[e]), inv);
          // each thread writes its own row: whole 32-byte sectors per store when the
          // output allows, instead of half sectors
          float* dst = orow + ci * 32;
          if (a.vec8) {
#pragma unroll
            for (int e = 0; e < 32; e += 8)
              st_global_v8(dst + e, v[e], v[e + 1], v[e + 2], v[e + 3], v[e + 4], v[e + 5], v[e + 6], v[e + 7]);
          } else {
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              *reinterpret_cast<float4*>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(o_free));
    }
  }

  dependents_may_launch();  // the fallback kernel behind may start launching
  // every MMA either issuer started completes before TMEM is released
  if ((warp == 1 || warp == 6) && lane == 0) {
    uint64_t* d = &drain[warp == 1 ? 0 : 1];
    mma_commit(smem_u32(d));
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(smem_u32(d), 0))
      if (globaltimer() - t0 > kWaitLimitNs) { record_device_error(a.err, 0x4fe); break; }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ------------------------------------------------------------- CTA-pair form
// The same fused attention on work items of 256 queries computed by a cluster of two
// CTAs on two SMs with tcgen05.mma.cta_group::2 (M = 256), reading q, k and v where they
// lie, with no pre-pass: CTA r holds queries [256 t + 128 r, +128) of Q, of every
// 64-key block the keys [32 r, 32 r + 32) of K, and the value columns
// [Dv r / 2, Dv (r + 1) / 2) of V (MN-major: V's rows are the P·V contraction), at the
// same shared-memory offsets; each SM's TMEM receives its 128 query rows of S, P and O.
// TMA brings the float32 tiles themselves, which the tensor core reads as the hi terms
// (kind::tf32 drops the low 13 mantissa bits). K's lo terms, lo = rna_tf32(x -
// trunc_tf32(x)), come from a pre-pass ([nk][S][D] beside K's layout, which also checks
// K for inf / NaN); for Q (once per item) and V four converter warps per CTA write each
// tile's lo terms beside it, checking it on the way, and arrive on the leader's ready
// barriers, on which the MMA issuers wait. A scanner warp checks the V rows no item
// loads (causal, keys past the last query tile). On a hit the row-wise IEEE kernel
// queued behind this one recomputes the whole result. (Converting K in the kernel too
// made it 15-18 % slower: the K ring is two stages deep and each stage is consumed in
// ~1.2 us, and the conversion sat between the TMA landing and the S products.)
// The leader's S and P·V issuers drive both SMs: every instruction does twice the work
// of the single-SM kernel's, and a K stage holds two 32-feature chunks, so one barrier
// wait covers 24 MMAs instead of 12. The leader's commits arrive on both CTAs' barriers
// (one commit per CTA, no multicast), both CTAs' softmax warps arrive on the leader's
// P-ready barriers and both CTAs' converter warps on its O-free barrier. Softmax,
// rescaling and the bounded waits are the single-SM kernel's; the item epilogue is not:
// the softmax warps hand each row's 1 / sum over shared memory and go on to the next
// item, and the converter warps drain, normalize and store O.
//   warp 0      TMA producer (Q and V on this CTA's barriers, K on the leader's)
//   warp 1      S issuer (leader)          warp 6      P·V issuer (leader)
//   warps 2-5   softmax                    warps 7-10  lo-term converters, item epilogue
//   warp 11     non-finite scan
constexpr int kPQ = 2 * kFQ;                   // queries per pair item
constexpr int kPKeys = kFK / 2;                // keys of a block per CTA (32)
constexpr int kPKC = 2;                        // feature chunks per K stage
constexpr int kPKStages = 2;
constexpr int kPKTile = kPKeys * kFC * 4;      // 4 KB: 32 keys x 32 features
constexpr int kPKStage = kPKC * 2 * kPKTile;   // 16 KB
constexpr int kPVStages = 2;
constexpr int kPVTile = 32 * kFC * 4;          // 4 KB: 32 keys x 32 value columns, MN-major
constexpr int kPVHalf = 2 * (kMaxDv / 64) * kPVTile;  // 16 KB: a block's hi (or lo) tiles
constexpr int kPVStage = 2 * kPVHalf;          // 32 KB: hi tiles, then lo tiles
constexpr int kPairThreads = 384;
constexpr int kConvWarp0 = 7, kScanWarp = 11;
constexpr int kPairSmem = kQBytes + kPKStages * kPKStage + kPVStages * kPVStage + 1024 + 512 + 1024;
static_assert(kPairSmem <= 232448, "shared memory per CTA");

__device__ __forceinline__ void mma_tf32_pair_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Commit to the barrier at `bar` in both CTAs of the pair.
__device__ __forceinline__ void commit_both(uint32_t bar) {
  mma_commit_pair(bar);
  mma_commit_pair(map_rank(bar, 1));
}

__device__ __forceinline__ int64_t snake_item_pair(int64_t r, int64_t items, int64_t cid, int64_t ncl) {
  const int64_t w = r * ncl + ((r & 1) ? ncl - 1 - cid : cid);
  return w < items ? w : -1;
}

__device__ __forceinline__ void item_coords_pair(const FlashArgs& a, int64_t w, int64_t& b, int& qt, int& nkb) {
  qt = a.q_tiles - 1 - static_cast<int>(w / a.batches);  // q_tiles counts 256-query tiles here
  b = w % a.batches;
  nkb = a.causal ? min(a.kv_blocks, (qt + 1) * (kPQ / kFK)) : a.kv_blocks;
}

// Key blocks of an item of query tile qt (256 queries): all, or up to the causal diagonal.
__device__ __forceinline__ int item_blocks_pair(const FlashArgs& a, int qt) {
  return a.causal ? min(a.kv_blocks, (qt + 1) * (kPQ / kFK)) : a.kv_blocks;
}

// Work unit u of the pair kernel: key blocks [j0, j1) of the item (batch b, query tile qt)
// of nkb blocks. Units follow the item order (longest query tiles first); an item's units
// are consecutive.
__device__ __forceinline__ void unit_coords_pair(const FlashArgs& a, int64_t u, int64_t& b, int& qt, int& j0,
                                                 int& j1, int& nkb) {
  if (a.kv_split == 0) {
    item_coords_pair(a, u, b, qt, nkb);
    j0 = 0;
    j1 = nkb;
    return;
  }
  int64_t rest = u;
  for (int r = 0; r < a.q_tiles; ++r) {
    qt = a.q_tiles - 1 - r;
    nkb = item_blocks_pair(a, qt);
    const int per = (nkb + a.kv_split - 1) / a.kv_split;
    const int64_t group = a.batches * per;
    if (rest < group || r == a.q_tiles - 1) {
      b = rest / per;
      j0 = static_cast<int>(rest % per) * a.kv_split;
      j1 = min(nkb, j0 + a.kv_split);
      return;
    }
    rest -= group;
  }
}

// The lo term of a float32 word x: x - trunc_tf32(x) (exact), rounded to tf32 (to
// nearest, ties away from zero, as cvt.rna.tf32.f32) by adding half a tf32 ulp to the
// magnitude bits and dropping the low 13.
__device__ __forceinline__ uint32_t lo_term(uint32_t x) {
  const uint32_t d = __float_as_uint(__fsub_rn(__uint_as_float(x), __uint_as_float(x & 0xFFFFE000u)));
  return (d + 0x1000u) & 0xFFFFE000u;
}

__device__ __forceinline__ uint32_t nonfinite4(uint4 w) {
  const uint32_t e = 0x7F800000u;
  return ((w.x & e) == e) | ((w.y & e) == e) | ((w.z & e) == e) | ((w.w & e) == e);
}

// Converter thread t (0..127) writes the lo terms of the 16-byte words t, t + 128, ... of
// the `bytes` of float32 tiles at shared address hi into the same offsets from lo, and
// notes an inf / NaN among them in `bad`.
__device__ __forceinline__ void write_lo(uint32_t hi, uint32_t lo, int bytes, int t, uint32_t& bad) {
#pragma unroll 4
  for (int off = t * 16; off < bytes; off += 128 * 16) {
    uint4 x;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(x.x), "=r"(x.y), "=r"(x.z), "=r"(x.w) : "r"(hi + off));
    bad |= nonfinite4(x);
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(lo + off), "r"(lo_term(x.x)), "r"(lo_term(x.y)),
                 "r"(lo_term(x.z)), "r"(lo_term(x.w))
                 : "memory");
  }
}

// A converter warp's lo writes become visible to the tensor core (the async proxy), then
// its lane 0 arrives on the leader's copy of the ready barrier `bar` (four warps of each
// CTA arrive: count 8).
__device__ __forceinline__ void publish_lo(uint32_t bar, int lane) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) mbar_arrive_cluster(map_rank(bar, 0));
}

template <int MK>
__global__ void __launch_bounds__(kPairThreads, 1)
flash_pair_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                  const __grid_constant__ CUtensorMap map_klo, const __grid_constant__ CUtensorMap map_v,
                  const FlashArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_res = smem;
  uint8_t* k_ring = smem + kQBytes;
  uint8_t* v_ring = k_ring + kPKStages * kPKStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(v_ring + kPVStages * kPVStage);
  uint64_t* k_full = bars;                       // [kPKStages] (the leader's count both CTAs' bytes)
  uint64_t* k_empty = k_full + kPKStages;        // [kPKStages]
  uint64_t* v_full = k_empty + kPKStages;        // [kPVStages] this CTA's V tiles landed
  uint64_t* v_empty = v_full + kPVStages;        // [kPVStages]
  uint64_t* v_ready = v_empty + kPVStages;       // [kPVStages] (the leader's: 8 converter warps)
  uint64_t* s_full = v_ready + kPVStages;        // [kSBufs]
  uint64_t* p_full = s_full + kSBufs;            // [kSBufs] (the leader's: 8 softmax warps)
  uint64_t* pv_done = p_full + kSBufs;           // [kSBufs]
  uint64_t* q_full = pv_done + kSBufs;
  uint64_t* q_ready = q_full + 1;                // (the leader's: 8 converter warps)
  uint64_t* q_empty = q_ready + 1;
  uint64_t* o_free = q_empty + 1;                // (the leader's: 8 softmax warps)
  uint64_t* drain = o_free + 1;                  // [2]
  uint64_t* l_ready = drain + 2;                 // [2] an item's row inverses written (4 softmax warps)
  uint64_t* inv_free = l_ready + 2;              // [2] ... and read by the converters (4 warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(inv_free + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* row_inv = reinterpret_cast<float*>(bars) + 128;  // [2][kFQ], past the 512-byte barrier area

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int dchunks = a.dp / kFC;
  const int kfills = (dchunks + kPKC - 1) / kPKC;  // K stage fills per key block
  const int nvc = a.dv / 64;                      // 32-column V chunks per CTA
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPKStages; ++s) { mbar_init(smem_u32(&k_full[s]), 1); mbar_init(smem_u32(&k_empty[s]), 1); }
    for (int s = 0; s < kPVStages; ++s) {
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
      mbar_init(smem_u32(&v_ready[s]), 8);
    }
    for (int b = 0; b < kSBufs; ++b) {
      mbar_init(smem_u32(&s_full[b]), 1);
      mbar_init(smem_u32(&p_full[b]), 8);
      mbar_init(smem_u32(&pv_done[b]), 1);
    }
    mbar_init(smem_u32(q_full), 1);
    mbar_init(smem_u32(q_ready), 8);
    mbar_init(smem_u32(q_empty), 1);
    mbar_init(smem_u32(o_free), 8);
    mbar_init(smem_u32(&drain[0]), 1);
    mbar_init(smem_u32(&drain[1]), 1);
    for (int i = 0; i < 2; ++i) { mbar_init(smem_u32(&l_ready[i]), 4); mbar_init(smem_u32(&inv_free[i]), 4); }
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
  const uint32_t tmem = *tmem_slot;
  const int64_t items = a.units;  // work units: items, or key ranges of items (kv_split)
  const int64_t cid = cluster_index(), ncl = cluster_count();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------- TMA producer (both CTAs)
      int64_t kf = 0, vf = 0, local = 0;  // K and V stage fills, items
      bool ok = true;
      for (int64_t r = 0; r * ncl < items && ok; ++r) {
        const int64_t w = snake_item_pair(r, items, cid, ncl);
        if (w < 0) continue;
        int64_t b; int qt, j0, j1, nkb;
        unit_coords_pair(a, w, b, qt, j0, j1, nkb);
        int64_t pq, pk, pv;
        batch_planes(a, b, pq, pk, pv);
        if (!wait_bounded(smem_u32(q_empty), static_cast<uint32_t>(local & 1) ^ 1u, abort_flag, a.err, 0x480)) break;
        ++local;
        {
          const uint32_t fb = smem_u32(q_full);
          mbar_expect_tx(fb, static_cast<uint32_t>(dchunks * kQTile));
          const int row = qt * kPQ + static_cast<int>(rank) * kFQ;
          for (int c = 0; c < dchunks; ++c)
            tma_load_3d(smem_u32(q_res + (2 * c) * kQTile), &map_q, fb, c * kFC, row, static_cast<int>(pq));
        }
        auto load_k = [&](int j) {
          const int key = j * kFK + static_cast<int>(rank) * kPKeys;
          for (int f = 0; f < kfills; ++f, ++kf) {
            const int s = static_cast<int>(kf % kPKStages);
            const uint32_t ph = static_cast<uint32_t>((kf / kPKStages) & 1);
            if (!wait_bounded(smem_u32(&k_empty[s]), ph ^ 1u, abort_flag, a.err, 0x481)) return false;
            const int c0 = f * kPKC, nc = min(kPKC, dchunks - c0);
            uint8_t* st = k_ring + s * kPKStage;
            const uint32_t fb_local = smem_u32(&k_full[s]);
            if (leader) mbar_expect_tx(fb_local, static_cast<uint32_t>(2 * nc * 2 * kPKTile));
            const uint32_t fb = map_rank(fb_local, 0);
            for (int c = 0; c < nc; ++c) {
              tma_load_3d_pair(smem_u32(st + (2 * c) * kPKTile), &map_k, fb, (c0 + c) * kFC, key, static_cast<int>(pk));
              tma_load_3d_pair(smem_u32(st + (2 * c + 1) * kPKTile), &map_klo, fb, (c0 + c) * kFC, key,
                               static_cast<int>(pk));
            }
          }
          return true;
        };
        // V of block j: this CTA's value columns as nvc MN-major chunks, for each half of
        // the block's keys, tiles [key half][chunk]; keys past S read as zeros
        auto load_v = [&](int j) {
          const int s = static_cast<int>(vf % kPVStages);
          const uint32_t ph = static_cast<uint32_t>((vf / kPVStages) & 1);
          if (!wait_bounded(smem_u32(&v_empty[s]), ph ^ 1u, abort_flag, a.err, 0x482)) return false;
          ++vf;  // counted once issued: an aborting producer settles only the fills made
          uint8_t* st = v_ring + s * kPVStage;
          const uint32_t fb = smem_u32(&v_full[s]);
          mbar_expect_tx(fb, static_cast<uint32_t>(2 * nvc * kPVTile));
          const int col = static_cast<int>(rank) * (a.dv / 2);
          for (int h = 0; h < 2; ++h)
            for (int c = 0; c < nvc; ++c)
              tma_load_3d(smem_u32(st + (h * nvc + c) * kPVTile), &map_v, fb, col + c * kFC, j * kFK + h * 32,
                          static_cast<int>(pv));
          return true;
        };
        for (int j = j0; j < j1 && ok; ++j) {
          ok = load_k(j);
          if (ok && j > j0) ok = load_v(j - 1);
        }
        if (ok && j1 > j0) ok = load_v(j1 - 1);
      }
      if (!ok || *abort_flag) {  // Q and V fills land on this CTA's barriers, K on the leader's
        auto settle = [&](uint64_t* full, int stages, int64_t n, int site) {
          for (int s = 0; s < stages; ++s) {
            const int64_t fills = n > s ? (n - s + stages - 1) / stages : 0;
            if (!fills) continue;
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(smem_u32(&full[s]), static_cast<uint32_t>((fills - 1) & 1)))
              if (globaltimer() - t0 > kWaitLimitNs) { record_device_error(a.err, site); break; }
          }
        };
        if (leader) settle(k_full, kPKStages, kf, 0x4f4);
        settle(v_full, kPVStages, vf, 0x4f5);
        settle(q_full, 1, local, 0x4f6);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // --------------------------------------------------- S = Q·Kᵀ issuer (leader)
      const uint32_t id_s = idesc_tf32(kPQ, kFK);
      int64_t kf = 0, g = 0, local = 0;
      bool ok = true;
      for (int64_t r = 0; r * ncl < items && ok; ++r) {
        const int64_t w = snake_item_pair(r, items, cid, ncl);
        if (w < 0) continue;
        int64_t b; int qt, j0, j1, nkb;
        unit_coords_pair(a, w, b, qt, j0, j1, nkb);
        if (!wait_bounded(smem_u32(q_ready), static_cast<uint32_t>(local & 1), abort_flag, a.err, 0x490)) break;
        ++local;
        tc_fence_after();
        for (int j = j0; j < j1 && ok; ++j, ++g) {
          const int buf = static_cast<int>(g % kSBufs);
          if (g >= kSBufs) {
            if (!wait_bounded(smem_u32(&pv_done[buf]), static_cast<uint32_t>(((g - kSBufs) / kSBufs) & 1), abort_flag,
                              a.err, 0x492)) { ok = false; break; }
            tc_fence_after();
          }
          const uint32_t d_s = tmem + static_cast<uint32_t>(buf * 128);
          for (int f = 0; f < kfills; ++f, ++kf) {
            const int s = static_cast<int>(kf % kPKStages);
            const uint32_t ph = static_cast<uint32_t>((kf / kPKStages) & 1);
            if (!wait_bounded(smem_u32(&k_full[s]), ph, abort_flag, a.err, 0x493)) { ok = false; break; }
            tc_fence_after();
            const int c0 = f * kPKC, nc = min(kPKC, dchunks - c0);
            for (int c = 0; c < nc; ++c) {
              const uint64_t dq_hi = smem_desc_sw128(smem_u32(q_res + (2 * (c0 + c)) * kQTile));
              const uint64_t dq_lo = smem_desc_sw128(smem_u32(q_res + (2 * (c0 + c) + 1) * kQTile));
              const uint64_t dk_hi = smem_desc_sw128(smem_u32(k_ring + s * kPKStage + (2 * c) * kPKTile));
              const uint64_t dk_lo = smem_desc_sw128(smem_u32(k_ring + s * kPKStage + (2 * c + 1) * kPKTile));
#pragma unroll
              for (int kk = 0; kk < kFC / 8; ++kk) {
                const uint32_t acc = (c0 + c == 0 && kk == 0) ? 0u : 1u;
                mma_tf32_pair(d_s, dq_lo + 2 * kk, dk_hi + 2 * kk, id_s, acc);
                mma_tf32_pair(d_s, dq_hi + 2 * kk, dk_lo + 2 * kk, id_s, 1u);
                mma_tf32_pair(d_s, dq_hi + 2 * kk, dk_hi + 2 * kk, id_s, 1u);
              }
            }
            commit_both(smem_u32(&k_empty[s]));
          }
          if (!ok) break;
          commit_both(smem_u32(&s_full[buf]));
          if (j == j1 - 1) commit_both(smem_u32(q_empty));
        }
      }
    }
  } else if (warp == 6) {
    if (lane == 0 && leader) {
      // --------------------------------------------------- O += P·V issuer (leader)
      const uint32_t id_o = idesc_tf32(kPQ, a.dv) | (1u << 16);  // B (V) MN-major
      const uint32_t d_o = tmem + kColO;
      int64_t vf = 0, g = 0, local = 0;
      bool ok = true;
      for (int64_t r = 0; r * ncl < items && ok; ++r) {
        const int64_t w = snake_item_pair(r, items, cid, ncl);
        if (w < 0) continue;
        int64_t b; int qt, j0, j1, nkb;
        unit_coords_pair(a, w, b, qt, j0, j1, nkb);
        const int64_t item = local++;
        for (int j = j0; j < j1 && ok; ++j, ++g) {
          const int buf = static_cast<int>(g % kSBufs);
          if (!wait_bounded(smem_u32(&p_full[buf]), static_cast<uint32_t>((g / kSBufs) & 1), abort_flag, a.err, 0x494)) {
            ok = false;
            break;
          }
          if (j == j0 && !wait_bounded(smem_u32(o_free), static_cast<uint32_t>(item & 1) ^ 1u, abort_flag, a.err, 0x491)) {
            ok = false;
            break;
          }
          const uint32_t p_hi = tmem + static_cast<uint32_t>(buf * 128), p_lo = p_hi + kFK;
          {
            const int s = static_cast<int>(vf % kPVStages);
            const uint32_t ph = static_cast<uint32_t>((vf / kPVStages) & 1);
            ++vf;
            if (!wait_bounded(smem_u32(&v_ready[s]), ph, abort_flag, a.err, 0x495)) { ok = false; break; }
            tc_fence_after();
            const uint32_t v_hi = smem_u32(v_ring + s * kPVStage), v_lo = v_hi + kPVHalf;
#pragma unroll
            for (int t = 0; t < kFK / 8; ++t) {  // 8 keys per MMA: 8 rows of 128 B in a chunk
              const uint32_t off = static_cast<uint32_t>((t >> 2) * nvc * kPVTile + (t & 3) * 1024);
              const uint64_t dv_hi = smem_desc_sw128_mn(v_hi + off, kPVTile);
              const uint64_t dv_lo = smem_desc_sw128_mn(v_lo + off, kPVTile);
              const uint32_t col = static_cast<uint32_t>(t * 8);
              const uint32_t acc = (j == j0 && t == 0) ? 0u : 1u;
              mma_tf32_pair_ta(d_o, p_lo + col, dv_hi, id_o, acc);
              mma_tf32_pair_ta(d_o, p_hi + col, dv_lo, id_o, 1u);
              mma_tf32_pair_ta(d_o, p_hi + col, dv_hi, id_o, 1u);
            }
            commit_both(smem_u32(&v_empty[s]));
          }
          if (!ok) break;
          commit_both(smem_u32(&pv_done[buf]));
        }
      }
    }
  } else if (warp >= 2 && warp <= 5) {
    // -------------------------------------------------------- softmax (both CTAs)
    const int quarter = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int row_in_tile = quarter * 32 + lane;
    int64_t g = 0, sitem = 0;
    for (int64_t r = 0; r * ncl < items; ++r) {
      const int64_t w = snake_item_pair(r, items, cid, ncl);
      if (w < 0) continue;
      int64_t b; int qt, j0, j1, nkb;
      unit_coords_pair(a, w, b, qt, j0, j1, nkb);
      const int64_t query = static_cast<int64_t>(qt) * kPQ + static_cast<int64_t>(rank) * kFQ + row_in_tile;
      const bool row_ok = query < a.L;
      const int64_t mrow = MK ? mask_offset(a, b) + (row_ok ? query : 0) * a.mq : 0;
      float m_use = -INFINITY, l = 0.0f;
      bool aborted = false;
      for (int j = j0; j < j1; ++j, ++g) {
        const int buf = static_cast<int>(g % kSBufs);
        const uint32_t col_s = static_cast<uint32_t>(buf * 128), col_lo = col_s + kFK;
        const int64_t key0 = static_cast<int64_t>(j) * kFK;
        int64_t lim64 = a.S - key0;
        if (a.causal) lim64 = min(lim64, query - key0 + 1);
        const int lim = static_cast<int>(lim64 < 0 ? 0 : (lim64 > kFK ? kFK : lim64));
        MaskBlock<MK> mb;
        if constexpr (MK != 0) {
          const int64_t left = a.S - key0;
          mb.load(a, mrow, key0, row_ok ? static_cast<int>(left < kFK ? left : kFK) : 0);
        }
        if (!wait_bounded(smem_u32(&s_full[buf]), static_cast<uint32_t>((g / kSBufs) & 1), abort_flag, a.err, 0x4a1)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        uint32_t s0[32], s1[32];
        TCX_LD32(s0, tmem + lane_base + col_s);
        TCX_LD32(s1, tmem + lane_base + col_s + 32);
        TCX_WAIT_LD32(s0);
        TCX_TIE32(s1);
        float mxv[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four independent chains
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float t = mb.apply(__fmul_rn(__uint_as_float(s0[e]), a.scale_log2), e);
          s0[e] = __float_as_uint(t);
          if (e < lim) mxv[e & 3] = fmaxf(mxv[e & 3], t);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float t = mb.apply(__fmul_rn(__uint_as_float(s1[e]), a.scale_log2), 32 + e);
          s1[e] = __float_as_uint(t);
          if (32 + e < lim) mxv[e & 3] = fmaxf(mxv[e & 3], t);
        }
        const float mx = fmaxf(fmaxf(mxv[0], mxv[1]), fmaxf(mxv[2], mxv[3]));
        const bool need = mx > m_use + 8.0f;
        float alpha = 1.0f;
        if (need) {
          alpha = j == j0 ? 0.0f : exp2f(m_use - mx);
          m_use = mx;
        }
        l = __fmul_rn(l, alpha);
        if (j > j0 && __any_sync(0xffffffffu, need)) {
          const int64_t gp = g - 1;
          if (!wait_bounded(smem_u32(&pv_done[gp % kSBufs]), static_cast<uint32_t>((gp / kSBufs) & 1), abort_flag, a.err,
                            0x4a3)) {
            aborted = true;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < a.dv; cc += 32) {
            uint32_t rr[32];
            TCX_LD32(rr, tmem + lane_base + kColO + cc);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int e = 0; e < 32; ++e) rr[e] = __float_as_uint(__fmul_rn(__uint_as_float(rr[e]), alpha));
            TCX_ST32(tmem + lane_base + kColO + cc, rr);
          }
        }
        // The tensor core reads float32 operands as tf32 by dropping the low 13 mantissa
        // bits, so p itself is the hi term of the 3xTF32 split and p - trunc_tf32(p)
        // (exact) the lo term: no conversions (two per element were most of this loop's
        // time), at most 2^-20 of p lost against a rounded split.
        float lsum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        auto emit = [&](uint32_t (&sv)[32], int c0) {
          uint32_t lo[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float p = 0.0f;
            if (c0 + e < lim && (MK == 0 || __uint_as_float(sv[e]) != -INFINITY)) {
              asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(p) : "f"(__fsub_rn(__uint_as_float(sv[e]), m_use)));
            }
            lsum[e & 3] = __fadd_rn(lsum[e & 3], p);
            sv[e] = __float_as_uint(p);
            lo[e] = __float_as_uint(__fsub_rn(p, __uint_as_float(__float_as_uint(p) & 0xFFFFE000u)));
          }
          TCX_ST32(tmem + lane_base + col_s + c0, sv);
          TCX_ST32(tmem + lane_base + col_lo + c0, lo);
        };
        emit(s0, 0);
        emit(s1, 32);
        l = __fadd_rn(l, __fadd_rn(__fadd_rn(lsum[0], lsum[1]), __fadd_rn(lsum[2], lsum[3])));
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_rank(smem_u32(&p_full[buf]), 0));
      }
      if (aborted) break;
      // Hand the row's 1 / sum to the converter warps, which drain, normalize and store O
      // once the item's last P·V has completed; the softmax moves on to the next item.
      const int ib = static_cast<int>(sitem & 1);
      if (sitem >= 2 && !wait_bounded(smem_u32(&inv_free[ib]), static_cast<uint32_t>(((sitem >> 1) - 1) & 1),
                                      abort_flag, a.err, 0x4a2))
        break;
      if (j0 == 0 && j1 == nkb) {
        row_inv[ib * kFQ + row_in_tile] = l > 0.0f ? 1.0f / l : 0.0f;
      } else {  // a key range of the item: O stays unnormalized, the row's statistics go out
        row_inv[ib * kFQ + row_in_tile] = 1.0f;
        float* ml = a.part_ml + (w * kPQ + static_cast<int64_t>(rank) * kFQ + row_in_tile) * 2;
        ml[0] = m_use;
        ml[1] = l;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&l_ready[ib]));
      ++sitem;
    }
  } else if (warp >= kConvWarp0 && warp < kScanWarp) {
    // ------------------------------------------------ lo-term converters (both CTAs)
    // The producer's Q and V fills in its order (K's lo terms come from the pre-pass),
    // and the output: after converting item i's Q, these warps drain item i - 1's O
    // (its last P·V done, its row inverses handed over by the softmax warps), release
    // the accumulator to the next item's P·V and store the rows; then item i's V.
    const int t = static_cast<int>(threadIdx.x) - kConvWarp0 * 32;
    const int quarter = warp & 3;  // the TMEM lane quarter this warp may read
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int row_in_tile = quarter * 32 + lane;
    int64_t vf = 0, local = 0, g_end = 0;
    uint32_t bad = 0;
    bool ok = true;
    int64_t pb = 0, pw = 0;
    int pqt = 0;
    bool pwhole = true;
    // O of this CTA's `it`-th unit (unit index uw: batch b, query tile qt; whole: the
    // item's every key block, else a key range whose O goes to part_o), whose last key
    // block is block gl of this cluster's sequence
    auto drain_o = [&](int64_t it, int64_t uw, bool whole, int64_t b, int qt, int64_t gl) {
      if (!wait_bounded(smem_u32(&pv_done[gl % kSBufs]), static_cast<uint32_t>((gl / kSBufs) & 1), abort_flag, a.err,
                        0x4b4))
        return false;
      const int ib = static_cast<int>(it & 1);
      if (!wait_bounded(smem_u32(&l_ready[ib]), static_cast<uint32_t>((it >> 1) & 1), abort_flag, a.err, 0x4b5))
        return false;
      tc_fence_after();
      const float inv = row_inv[ib * kFQ + row_in_tile];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&inv_free[ib]));
      const int64_t query = static_cast<int64_t>(qt) * kPQ + static_cast<int64_t>(rank) * kFQ + row_in_tile;
      const bool row_ok = query < a.L;
      float* orow = whole ? a.out + (b * a.L + query) * a.dv
                          : a.part_o + (uw * kPQ + static_cast<int64_t>(rank) * kFQ + row_in_tile) * a.dv;
      const int nch = a.dv / 32;
      // two 32-column chunks at a time (registers): the accumulator is released after the
      // last pair's TMEM load, before its stores
      auto store_chunk = [&](const uint32_t (&oc)[32], int ci) {
        if (!row_ok) return;
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = __fmul_rn(__uint_as_float(oc[e]), inv);
        float* dst = orow + ci * 32;
        if (a.vec8) {
#pragma unroll
          for (int e = 0; e < 32; e += 8)
            st_global_v8(dst + e, v[e], v[e + 1], v[e + 2], v[e + 3], v[e + 4], v[e + 5], v[e + 6], v[e + 7]);
        } else {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
        }
      };
      for (int c0 = 0; c0 < nch; c0 += 2) {
        const bool two = c0 + 1 < nch;
        uint32_t o0[32], o1[32];
        TCX_LD32(o0, tmem + lane_base + kColO + static_cast<uint32_t>(c0 * 32));
        if (two) TCX_LD32(o1, tmem + lane_base + kColO + static_cast<uint32_t>((c0 + 1) * 32));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        TCX_TIE32(o0);
        TCX_TIE32(o1);
        if (c0 + 2 >= nch) {
          // every TMEM read of O is done: the next item's first P·V may overwrite it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(map_rank(smem_u32(o_free), 0));
        }
        store_chunk(o0, c0);
        if (two) store_chunk(o1, c0 + 1);
      }
      return true;
    };
    for (int64_t r = 0; r * ncl < items && ok; ++r) {
      const int64_t w = snake_item_pair(r, items, cid, ncl);
      if (w < 0) continue;
      int64_t b; int qt, j0, j1, nkb;
      unit_coords_pair(a, w, b, qt, j0, j1, nkb);
      if (!wait_bounded(smem_u32(q_full), static_cast<uint32_t>(local & 1), abort_flag, a.err, 0x4b0)) break;
      for (int c = 0; c < dchunks; ++c)
        write_lo(smem_u32(q_res + (2 * c) * kQTile), smem_u32(q_res + (2 * c + 1) * kQTile), kQTile, t, bad);
      publish_lo(smem_u32(q_ready), lane);
      if (local > 0 && !(ok = drain_o(local - 1, pw, pwhole, pb, pqt, g_end - 1))) break;
      ++local;
      auto conv_v = [&]() {
        const int s = static_cast<int>(vf % kPVStages);
        const uint32_t ph = static_cast<uint32_t>((vf / kPVStages) & 1);
        ++vf;
        if (!wait_bounded(smem_u32(&v_full[s]), ph, abort_flag, a.err, 0x4b2)) return false;
        const uint32_t st = smem_u32(v_ring + s * kPVStage);
        write_lo(st, st + kPVHalf, 2 * nvc * kPVTile, t, bad);
        publish_lo(smem_u32(&v_ready[s]), lane);
        return true;
      };
      for (int j = j0; j < j1 && ok; ++j) ok = conv_v();
      g_end += j1 - j0;
      pb = b;
      pqt = qt;
      pw = w;
      pwhole = j0 == 0 && j1 == nkb;
    }
    if (ok && local > 0) drain_o(local - 1, pw, pwhole, pb, pqt, g_end - 1);
    // every tile this CTA loaded was checked on the way: Q whole, V up to the last key
    // any item reaches (the pre-pass checked all of K)
    if (__any_sync(0xffffffffu, bad != 0) && lane == 0) atomicExch(a.flag, 1);
  } else if (warp == kScanWarp) {
    // ------------------------------------------------------ non-finite scan (both CTAs)
    // The V rows no item loads (causal, keys past the last query tile): rows
    // [a.tail_row, S) of every plane, 16-byte words split evenly over the CTAs.
    uint32_t bad = 0;
    const int64_t cta = blockIdx.x, nct = gridDim.x, rows = a.S - a.tail_row;
    if (rows > 0) {
      const uint4* p = reinterpret_cast<const uint4*>(a.v);
      const int64_t row_words = a.dv / 4, per_plane = rows * row_words;
      const int64_t n = a.v_planes * per_plane, lo = n * cta / nct, hi = n * (cta + 1) / nct;
      for (int64_t i = lo + lane; i < hi; i += 32) {
        const int64_t plane = i / per_plane;
        bad |= nonfinite4(__ldg(p + (plane * a.S + a.tail_row) * row_words + (i - plane * per_plane)));
      }
    }
    if (__any_sync(0xffffffffu, bad != 0) && lane == 0) atomicExch(a.flag, 1);
  }

  dependents_may_launch();  // the fallback kernel behind may start launching
  // every MMA the leader's issuers started completes before either CTA releases its TMEM
  if ((warp == 1 || warp == 6) && lane == 0) {
    uint64_t* d = &drain[warp == 1 ? 0 : 1];
    if (leader) commit_both(smem_u32(d));
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(smem_u32(d), 0))
      if (globaltimer() - t0 > kWaitLimitNs) { record_device_error(a.err, 0x4fd); break; }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
  cluster_sync_all();  // neither CTA leaves while the other may still touch its barriers
}

// Combines the units of the items the pair kernel cut into key ranges (kv_split): per
// row, O = (sum_u 2^(m_u - M) O_u) / (sum_u 2^(m_u - M) l_u) with M the largest m_u
// (log2 domain; a unit with no key for the row has m_u = -inf and weight 0). One warp per
// row, launched behind the pair kernel (programmatic dependent: waits for its grid).
constexpr int kCombineThreads = 256;

__global__ void __launch_bounds__(kCombineThreads) flash_combine_kernel(const FlashArgs a) {
  wait_for_prior_grid();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kCombineThreads / 32);
  const int64_t jobs = a.batches * a.q_tiles * kPQ;
  for (int64_t job = static_cast<int64_t>(blockIdx.x) * (kCombineThreads / 32) + (threadIdx.x >> 5); job < jobs;
       job += warps) {
    const int64_t item = job / kPQ;
    const int row = static_cast<int>(job % kPQ);
    const int r = static_cast<int>(item / a.batches);
    const int64_t b = item % a.batches;
    const int qt = a.q_tiles - 1 - r;
    const int per = (item_blocks_pair(a, qt) + a.kv_split - 1) / a.kv_split;
    const int64_t query = static_cast<int64_t>(qt) * kPQ + row;
    if (per == 1 || query >= a.L) continue;  // whole items were written by the pair kernel
    int64_t u0 = b * per;  // the item's first unit: all units of the longer groups first
    for (int rr = 0; rr < r; ++rr)
      u0 += a.batches * ((item_blocks_pair(a, a.q_tiles - 1 - rr) + a.kv_split - 1) / a.kv_split);
    float mx = -INFINITY;
    for (int u = 0; u < per; ++u) mx = fmaxf(mx, __ldcg(a.part_ml + ((u0 + u) * kPQ + row) * 2));
    float den = 0.0f, acc[kMaxDv / 32];
#pragma unroll
    for (int c = 0; c < kMaxDv / 32; ++c) acc[c] = 0.0f;
    for (int u = 0; u < per; ++u) {
      const float* ml = a.part_ml + ((u0 + u) * kPQ + row) * 2;
      const float mu = __ldcg(ml);
      const float wgt = mu == -INFINITY ? 0.0f : exp2f(__fsub_rn(mu, mx));
      den = __fmaf_rn(wgt, __ldcg(ml + 1), den);
      const float* o = a.part_o + ((u0 + u) * kPQ + row) * a.dv;
#pragma unroll
      for (int c = 0; c < kMaxDv / 32; ++c)
        if (32 * c + lane < a.dv) acc[c] = __fmaf_rn(wgt, __ldcg(o + 32 * c + lane), acc[c]);
    }
    const float inv = den > 0.0f ? 1.0f / den : 0.0f;
    float* out = a.out + (b * a.L + query) * a.dv;
#pragma unroll
    for (int c = 0; c < kMaxDv / 32; ++c)
      if (32 * c + lane < a.dv) out[32 * c + lane] = __fmul_rn(acc[c], inv);
  }
  dependents_may_launch();
}

// IEEE fallback, used only when the pre-pass or the pair kernel's scan saw inf / NaN
// (launched behind the fused kernel with programmatic stream serialization: it waits
// for that grid before reading the flag): one CTA per (batch, query) row computes the scores as float32 dot products in feature order (as the reference
// matmul), the masked softmax of core/inference.cpp / cpu_inference.cpp, and P·V summed
// over keys in order, recomputing the dot products per pass instead of storing them.
constexpr int kRowThreads = 128;

template <int MK>
__global__ void __launch_bounds__(kRowThreads)
flash_rows_fallback(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                    FlashArgs a, int64_t d, float scale, const int* __restrict__ flag) {
  wait_for_prior_grid();
  if (!*flag) return;
  __shared__ float qrow[kMaxDv];
  __shared__ float p_chunk[kRowThreads];
  __shared__ float red[64];
  using B = rowmath::Block<kRowThreads>;
  const int64_t rows = a.batches * a.L;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t b = row / a.L, query = row % a.L;
    int64_t pq, pk, pv;
    batch_planes(a, b, pq, pk, pv);
    const float* qr = q + (pq * a.L + query) * d;
    const float* kb = k + pk * a.S * d;
    const float* vb = v + pv * a.S * a.dv;
    __syncthreads();
    for (int i = threadIdx.x; i < d; i += kRowThreads) qrow[i] = qr[i];
    __syncthreads();
    const int64_t keys = a.causal ? (query + 1 < a.S ? query + 1 : a.S) : a.S;
    const int64_t mrow = MK ? mask_offset(a, b) + query * a.mq : 0;
    // cpu_inference.cpp:26-33: a false bool entry or a -inf float entry masks the key;
    // otherwise score * scale + bias
    auto score = [&](int64_t key) {
      float bias = 0.0f;
      if constexpr (MK == 1) {
        if (!static_cast<const unsigned char*>(a.mask)[mrow + key * a.mk]) return -INFINITY;
      } else if constexpr (MK == 2) {
        bias = static_cast<const float*>(a.mask)[mrow + key * a.mk];
        if (bias == -INFINITY) return -INFINITY;
      }
      float acc = 0.0f;
      const float* kr = kb + key * d;
      for (int64_t i = 0; i < d; ++i) acc = __fadd_rn(acc, __fmul_rn(qrow[i], kr[i]));
      return MK == 2 ? __fadd_rn(__fmul_rn(acc, scale), bias) : __fmul_rn(acc, scale);
    };
    float mx = -INFINITY;
    bool nan = false;
    for (int64_t key = threadIdx.x; key < keys; key += kRowThreads) {
      const float s = score(key);
      nan |= s != s;
      mx = fmaxf(mx, s);
    }
    if (nan) mx = __int_as_float(0x7fc00000);
    mx = B::max(mx, red);
    float* orow = a.out + row * a.dv;
    if (mx == -INFINITY) {  // every score -inf: the reference's all-zero row
      for (int c = threadIdx.x; c < a.dv; c += kRowThreads) orow[c] = 0.0f;
      continue;
    }
    float total = 0.0f;
    for (int64_t key = threadIdx.x; key < keys; key += kRowThreads) total = __fadd_rn(total, expf(score(key) - mx));
    total = B::sum(total, red);
    // P·V over every key, masked ones with p = 0 (as the reference's dense product, so a
    // non-finite value under a masked key still propagates)
    float acc[kMaxDv / kRowThreads + 1] = {0.0f};
    for (int64_t k0 = 0; k0 < a.S; k0 += kRowThreads) {
      __syncthreads();
      const int64_t key = k0 + threadIdx.x;
      p_chunk[threadIdx.x] = key < keys ? __fdiv_rn(expf(score(key) - mx), total) : 0.0f;
      __syncthreads();
      const int64_t n = a.S - k0 < kRowThreads ? a.S - k0 : kRowThreads;
      for (int c = threadIdx.x, slot = 0; c < a.dv; c += kRowThreads, ++slot)
        for (int64_t i = 0; i < n; ++i) acc[slot] = __fadd_rn(acc[slot], __fmul_rn(p_chunk[i], vb[(k0 + i) * a.dv + c]));
    }
    for (int c = threadIdx.x, slot = 0; c < a.dv; c += kRowThreads, ++slot) orow[c] = acc[slot];
  }
}

// NaN or +inf anywhere in a float mask raises *flag (the fused kernel's arithmetic
// assumes finite or -inf biases; the IEEE row kernel then gives the reference's NaN rows).
__global__ void __launch_bounds__(256) mask_scan(const float* __restrict__ m, int64_t n, int* __restrict__ flag) {
  bool bad = false;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float x = __ldg(m + i);
    bad |= x != x || x == INFINITY;
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flag, 1);
}

size_t round_up(size_t v, size_t m) { return (v + m - 1) / m * m; }

struct FlashLayout {
  size_t off_flag, off_q, off_k, off_v, off_po, off_pml, total;
  int64_t sp;
  int64_t part_units;  // key-range units the partial areas hold (0: no split possible)
};

// Unmasked products that may run on CTA pairs with fewer items (256 queries of one batch)
// than twice the SM pairs get room for key-range units: at most two per SM pair beyond
// one per item (the split keeps units >= total key blocks / (2 x pairs) blocks long).
FlashLayout flash_layout(int64_t L, int64_t S, int64_t d, int64_t dv, int64_t nq, int64_t nk, int64_t nv,
                         int64_t batches, int mask_kind) {
  FlashLayout f;
  f.sp = (S + kFC - 1) / kFC * kFC;
  f.off_flag = 0;
  f.off_q = 1024;
  f.off_k = round_up(f.off_q + static_cast<size_t>(2 * nq * L * d) * 4, 1024);
  f.off_v = round_up(f.off_k + static_cast<size_t>(2 * nk * S * d) * 4, 1024);
  f.off_po = round_up(f.off_v + static_cast<size_t>(2 * nv * dv * f.sp) * 4, 1024);
  const int64_t pairs = sm_count() / 2;
  const int64_t items = batches * ((L + kPQ - 1) / kPQ);
  f.part_units = (mask_kind == 0 && dv % 64 == 0 && L > kFQ && items < 2 * pairs) ? 2 * pairs + items : 0;
  f.off_pml = round_up(f.off_po + static_cast<size_t>(f.part_units * kPQ * dv) * 4, 1024);
  f.total = round_up(f.off_pml + static_cast<size_t>(f.part_units * kPQ * 2) * 4, 1024);
  return f;
}

}  // namespace

bool flash_eligible(int64_t queries, int64_t keys, int64_t features, int64_t value_features, int mask_kind,
                    int batch_rank) {
  return mask_kind >= 0 && mask_kind <= 2 && queries > 0 && keys > 0 && features % kFC == 0 && features <= 128 &&
         value_features % kFC == 0 && value_features > 0 && value_features <= kMaxDv &&
         batch_rank <= kMaxFlashBatchRank && queries <= INT32_MAX / 2 && keys <= INT32_MAX / 2;
}

size_t flash_workspace_bytes(int64_t queries, int64_t keys, int64_t features, int64_t value_features,
                             int64_t q_batches, int64_t k_batches, int64_t v_batches, int64_t batches,
                             int mask_kind) {
  return flash_layout(queries, keys, features, value_features, q_batches, k_batches, v_batches, batches, mask_kind)
      .total;
}

int attention_fused(cudaStream_t s, const float* q, const float* k, const float* v, const void* mask,
                    int mask_kind, const int64_t* mask_strides, float* out, int64_t L, int64_t S, int64_t d,
                    int64_t dv, int64_t batches, const int64_t* batch_shape, const int64_t* q_strides,
                    const int64_t* k_strides, const int64_t* v_strides, int32_t rank, float scale, int causal,
                    void* workspace, size_t workspace_bytes) {
  FlashArgs fa{};
  // mask strides (elements) over [batch..., L, S]: the keys' must be 0 or 1
  if (mask_kind) {
    for (int i = 0; i < rank + 2; ++i)
      if (mask_strides[i] < 0) return invalid("negative attention strides");
    if (mask_strides[rank + 1] > 1) return invalid("attention last-axis strides must be 0 or 1");
    fa.mask = mask;
    fa.mq = mask_strides[rank];
    fa.mk = mask_strides[rank + 1];
  }
  fa.L = L; fa.S = S; fa.dp = static_cast<int32_t>(d); fa.dv = static_cast<int32_t>(dv);
  fa.batches = batches;
  // batch strides in matrix units; collapse extent-1 axes
  int64_t nq = 1, nk = 1, nv = 1;
  fa.rank = 0;
  for (int i = 0; i < rank; ++i) {
    if (batch_shape[i] == 1) continue;
    if (fa.rank == kMaxFlashBatchRank) return invalid("attention batch rank exceeds 30");
    fa.shape[fa.rank] = batch_shape[i];
    fa.qs[fa.rank] = q_strides[i] / (L * d);
    fa.ks[fa.rank] = k_strides[i] / (S * d);
    fa.vs[fa.rank] = v_strides[i] / (S * dv);
    fa.ms[fa.rank] = mask_kind ? mask_strides[i] : 0;
    if (q_strides[i]) nq *= batch_shape[i];
    if (k_strides[i]) nk *= batch_shape[i];
    if (v_strides[i]) nv *= batch_shape[i];
    ++fa.rank;
  }
  FlashLayout lay = flash_layout(L, S, d, dv, nq, nk, nv, batches, mask_kind);
  if (workspace && workspace_bytes < lay.total && workspace_bytes >= lay.off_po) {
    lay.part_units = 0;  // a workspace sized without the key-range partials: no split
    lay.total = lay.off_po;
  }
  if (!workspace || workspace_bytes < lay.total) return invalid("attention workspace is missing or too small");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* flag = reinterpret_cast<int*>(ws + lay.off_flag);
  float* wq = reinterpret_cast<float*>(ws + lay.off_q);
  float* wk = reinterpret_cast<float*>(ws + lay.off_k);
  float* wv = reinterpret_cast<float*>(ws + lay.off_v);
  if (cudaMemsetAsync(flag, 0, sizeof(int), s) != cudaSuccess) return launch_status("attention flag reset");
  // CTA pairs (256 queries per item) for unmasked products with more than one 128-query
  // tile, reading q, k, v in place (no pre-pass): they need 16-byte aligned operands and
  // whole 32-column V chunks per CTA (Dv 64 or 128). Measured on [32, 2048, 2048, 128]
  // with the split pre-pass: 0.487 against 0.512 ms per call without a mask, 0.302
  // against 0.306 causal; with a float mask the pair is slower (0.674 against 0.636 ms
  // kernel), its two SMs' softmax warps both gating every P·V. Measured again with the
  // pair reading q, k, v in place (no split pre-pass): masked calls 0.610 against 0.577 ms
  // (float mask) and 0.531 against 0.487 ms (bool mask), so masks keep the single-SM
  // kernel.
  auto aligned16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const bool pair = L > kFQ && mask_kind == 0 && dv % 64 == 0 && aligned16(q) && aligned16(k) && aligned16(v);
  if (pair) {
    split_lo_planes(s, k, wk, nk * S * d / 4, flag);  // K's lo terms [nk][S][d]
  } else {
    // K-major split planes: Q [2nq][L][d], K [2nk][S][d] (rows already K-major), Vᵀ [2nv][dv][Sp]
    split_rows_planes2(s, q, wq, nq, L, k, wk, nk, S, d, d, flag);
    split_cols_planes(s, v, wv, nv, S, dv, lay.sp, flag);
  }
  const int sms = sm_count();
  if (mask_kind == 2) {
    // the mask's storage: 1 + sum of (extent - 1) * stride over [batch..., L, S]
    int64_t extent = 1 + (L - 1) * fa.mq + (S - 1) * fa.mk;
    for (int i = 0; i < rank; ++i) extent += (batch_shape[i] - 1) * mask_strides[i];
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(extent, 256 * 8), 8LL * sms)));
    mask_scan<<<grid, 256, 0, s>>>(static_cast<const float*>(mask), extent, flag);
  }
  if (int st = launch_status("attention split pre-pass")) return st;
  if (mask_kind) {
    const int64_t unit = mask_kind == 1 ? 16 : 4;  // elements per 16 bytes
    bool vec = reinterpret_cast<uintptr_t>(mask) % 16 == 0 && fa.mq % unit == 0;
    for (int i = 0; i < fa.rank; ++i) vec = vec && fa.ms[i] % unit == 0;
    fa.mask_vec = vec ? 1 : 0;
  }

  alignas(64) CUtensorMap map_q, map_k, map_klo, map_v;
  const bool mapped =
      pair ? encode_planes_map(&map_q, q, nq, L, d, kFQ) && encode_planes_map(&map_k, k, nk, S, d, kPKeys) &&
                 encode_planes_map(&map_klo, wk, nk, S, d, kPKeys) && encode_planes_map(&map_v, v, nv, S, dv, 32, true)
           : encode_planes_map(&map_q, wq, 2 * nq, L, d, kFQ) && encode_planes_map(&map_k, wk, 2 * nk, S, d, kFK) &&
                 encode_planes_map(&map_v, wv, 2 * nv, dv, lay.sp, static_cast<int>(dv));
  if (!mapped) return (set_error("cuTensorMapEncodeTiled failed"), TCX_INTERNAL);
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(flash_tf32x3_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFlashSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(flash_tf32x3_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFlashSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(flash_tf32x3_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFlashSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(flash_pair_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmem) !=
            cudaSuccess)
      return launch_status("flash smem attribute");
    attr_done[dev] = true;
  }
  fa.q_tiles = static_cast<int32_t>(ceil_div(L, pair ? kPQ : kFQ));
  fa.kv_blocks = static_cast<int32_t>(ceil_div(S, kFK));
  fa.scale_log2 = scale * kLog2e;
  fa.causal = causal;
  fa.out = out;
  fa.vec8 = reinterpret_cast<uintptr_t>(out) % 32 == 0;
  fa.nonfinite = flag;
  fa.err = device_error_word();
  fa.v = v;
  fa.v_planes = nv;
  fa.tail_row = causal ? std::min<int64_t>(S, static_cast<int64_t>(fa.q_tiles) * kPQ) : S;
  fa.flag = flag;
  const int64_t items = batches * fa.q_tiles;
  fa.kv_split = 0;
  fa.units = items;
  fa.part_o = fa.part_ml = nullptr;
  if (pair && items < sms && lay.part_units > 0) {
    // Few items for the SM pairs (heads sharded over GPUs, short sequences) and the
    // longest item more than three times the work per SM pair: cut the items' key blocks
    // into units of >= 4 blocks, about two per SM pair, and combine the units' partial
    // rows afterwards. Measured on [heads, 2048, 2048, 128] (per call): causal 4 heads
    // 118 -> 71 µs; where the longest item is not that far above the average, the units'
    // extra transitions, partial stores and the combining pass cost more than the balance
    // gains (8 heads full 126 -> 179 µs, 16 heads causal 132 -> 186 µs), so those stay whole.
    int64_t total = 0;
    int longest = 0;
    for (int qt = 0; qt < fa.q_tiles; ++qt) {
      const int nkb = causal ? static_cast<int>(std::min<int64_t>(fa.kv_blocks, (qt + 1) * (kPQ / kFK))) : fa.kv_blocks;
      total += batches * nkb;
      longest = std::max(longest, nkb);
    }
    const int split = static_cast<int>(std::max<int64_t>(4, ceil_div(total, sms)));
    if (split < longest && static_cast<int64_t>(longest) * (sms / 2) > 3 * total) {
      int64_t units = 0;
      for (int qt = 0; qt < fa.q_tiles; ++qt) {
        const int nkb = causal ? static_cast<int>(std::min<int64_t>(fa.kv_blocks, (qt + 1) * (kPQ / kFK))) : fa.kv_blocks;
        units += batches * ceil_div(nkb, split);
      }
      if (units <= lay.part_units) {
        fa.kv_split = split;
        fa.units = units;
        fa.part_o = reinterpret_cast<float*>(ws + lay.off_po);
        fa.part_ml = reinterpret_cast<float*>(ws + lay.off_pml);
      }
    }
  }
  if (pair) {
    TimedLaunch timer("flash_tf32x3", s);
    const int clusters = static_cast<int>(std::min<int64_t>(fa.units, sms / 2));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(kPairThreads);
    cfg.dynamicSmemBytes = kPairSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, flash_pair_kernel<0>, map_q, map_k, map_klo, map_v, fa);  // unmasked only
  } else {
    TimedLaunch timer("flash_tf32x3", s);
    const int grid = static_cast<int>(std::min<int64_t>(items, sms));
    if (mask_kind == 1) flash_tf32x3_kernel<1><<<grid, kFlashThreads, kFlashSmem, s>>>(map_q, map_k, map_v, fa);
    else if (mask_kind == 2) flash_tf32x3_kernel<2><<<grid, kFlashThreads, kFlashSmem, s>>>(map_q, map_k, map_v, fa);
    else flash_tf32x3_kernel<0><<<grid, kFlashThreads, kFlashSmem, s>>>(map_q, map_k, map_v, fa);
  }
  if (int st = launch_status("fused attention")) return st;
  if (fa.kv_split > 0) {  // merge the key-range units' rows
    TimedLaunch timer("flash_combine", s);
    const int64_t rows = items * kPQ;
    const int grid = static_cast<int>(std::min<int64_t>(ceil_div(rows, kCombineThreads / 32), 4LL * sms));
    launch_after(flash_combine_kernel, grid, kCombineThreads, s, 0, fa);
    if (int st = launch_status("attention combine")) return st;
  }
  {
    TimedLaunch timer("flash_rows_fallback", s);
    // idle unless a non-finite input was seen: a small grid (rows in a grid-stride loop)
    // keeps its launch and exit short
    const int grid = static_cast<int>(std::min<int64_t>(batches * L, 2LL * sms));
    const int* f = flag;
    if (mask_kind == 1) launch_after(flash_rows_fallback<1>, grid, kRowThreads, s, 0, q, k, v, fa, d, scale, f);
    else if (mask_kind == 2) launch_after(flash_rows_fallback<2>, grid, kRowThreads, s, 0, q, k, v, fa, d, scale, f);
    else launch_after(flash_rows_fallback<0>, grid, kRowThreads, s, 0, q, k, v, fa, d, scale, f);
  }
  return launch_status("attention fallback");
}

}  // namespace tcx
