// The rest of the reference CUDA backend's primitives, so that a tensor.cx program on
// device="cuda" finds every op it had: negate and scalar arithmetic, log / sqrt / abs,
// casts, comparisons, logical ops and where, any / all, masked_select, transpose and
// slice (index copies), concat, topk and embedding. All are HBM-bound streams (topk a
// per-group selection): grids sized to the SM count, 16-byte accesses where the layout
// allows, broadcast metadata collapsed on the host and passed by value. Results match
// the reference bit for bit (cited per op) except log, which calls CUDA's logf against
// the CPU backend's std::log (within 1 ulp of each other).
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <vector>

#include "common.cuh"

namespace tcx {
namespace {

constexpr int kThreads = 256;

// ------------------------------------------------------------ map (one input)
// cpu_backend.cpp / primitives.cu:14-32 (negate), elementwise.cu:19-31 and 110-116
// (scalar arithmetic: the scalar rounded to float32 once, or wrapped to int32), and
// math.cu:29-41 / cpu_math.cpp:36-40 (log, sqrt on float32; abs on the sign bit, or
// with int32 wrap).
template <int OP>
__device__ __forceinline__ uint32_t map_f32(uint32_t w, float scalar, bool left) {
  const float v = __uint_as_float(w);
  switch (OP) {
    case TCX_OP_NEGATE: return w ^ 0x80000000u;
    case TCX_OP_ADD_SCALAR: return __float_as_uint(left ? __fadd_rn(scalar, v) : __fadd_rn(v, scalar));
    case TCX_OP_SUBTRACT_SCALAR: return __float_as_uint(left ? __fsub_rn(scalar, v) : __fsub_rn(v, scalar));
    case TCX_OP_MULTIPLY_SCALAR: return __float_as_uint(left ? __fmul_rn(scalar, v) : __fmul_rn(v, scalar));
    case TCX_OP_DIVIDE_SCALAR: return __float_as_uint(left ? __fdiv_rn(scalar, v) : __fdiv_rn(v, scalar));
    case TCX_OP_LOG: return __float_as_uint(logf(v));
    case TCX_OP_SQRT: return __float_as_uint(sqrtf(v));
    default: return w & 0x7fffffffu;  // abs
  }
}
template <int OP>
__device__ __forceinline__ uint32_t map_i32(uint32_t w, uint32_t scalar, bool left) {
  switch (OP) {
    case TCX_OP_NEGATE: return 0u - w;
    case TCX_OP_ADD_SCALAR: return w + scalar;
    case TCX_OP_SUBTRACT_SCALAR: return left ? scalar - w : w - scalar;
    case TCX_OP_MULTIPLY_SCALAR: return w * scalar;
    default: return (w & 0x80000000u) ? 0u - w : w;  // abs, INT_MIN stays INT_MIN
  }
}
template <int OP, bool FP>
__device__ __forceinline__ uint32_t map_word(uint32_t w, float fs, uint32_t is, bool left) {
  if constexpr (FP) return map_f32<OP>(w, fs, left);
  else return map_i32<OP>(w, is, left);
}

template <int OP, bool FP>
__global__ void __launch_bounds__(kThreads)
map_kernel(const uint32_t* __restrict__ x, uint32_t* __restrict__ out, int64_t n, float fs, uint32_t is, bool left) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  int64_t done = 0;
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
    const int64_t n4 = n >> 2;
    for (int64_t i = tid; i < n4; i += stride) {
      uint4 v = __ldcs(reinterpret_cast<const uint4*>(x) + i);
      v.x = map_word<OP, FP>(v.x, fs, is, left);
      v.y = map_word<OP, FP>(v.y, fs, is, left);
      v.z = map_word<OP, FP>(v.z, fs, is, left);
      v.w = map_word<OP, FP>(v.w, fs, is, left);
      __stcs(reinterpret_cast<uint4*>(out) + i, v);
    }
    done = n4 << 2;
  }
  for (int64_t i = done + tid; i < n; i += stride) out[i] = map_word<OP, FP>(x[i], fs, is, left);
}

// ------------------------------------------------------------------------ cast
// elementwise.cu:85-107 and predicate.cu:62-71: float32 -> int32 truncates toward zero
// after a range check (finite, in [-2^31, 2^31)), int32 -> float32 rounds to nearest,
// anything -> bool is "!= 0", bool -> numbers is 0 / 1.
__device__ __forceinline__ bool cast_src_nonzero(const void* x, int64_t i, int src) {
  if (src == TCX_FLOAT32) return static_cast<const float*>(x)[i] != 0.0f;
  if (src == TCX_INT32) return static_cast<const int32_t*>(x)[i] != 0;
  return static_cast<const uint8_t*>(x)[i] != 0;
}
__global__ void __launch_bounds__(kThreads)
cast_kernel(const void* __restrict__ x, void* __restrict__ out, int64_t n, int src, int dst, int* __restrict__ bad) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  bool invalid_seen = false;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    if (src == TCX_FLOAT32 && dst == TCX_INT32) {
      const float v = static_cast<const float*>(x)[i];
      if (!(v >= -2147483648.0f && v < 2147483648.0f)) {
        invalid_seen = true;
        static_cast<int32_t*>(out)[i] = 0;
      } else {
        static_cast<int32_t*>(out)[i] = __float2int_rz(v);
      }
    } else if (src == TCX_INT32 && dst == TCX_FLOAT32) {
      static_cast<float*>(out)[i] = __int2float_rn(static_cast<const int32_t*>(x)[i]);
    } else {
      const bool v = cast_src_nonzero(x, i, src);
      if (dst == TCX_BOOL) static_cast<uint8_t*>(out)[i] = v;
      else if (dst == TCX_FLOAT32) static_cast<float*>(out)[i] = v ? 1.0f : 0.0f;
      else static_cast<int32_t*>(out)[i] = v;
    }
  }
  if (invalid_seen) atomicExch(bad, 1);
}

// ------------------------------------------------------------------ predicates
// predicate.cu:19-61 / cpu_predicate.cpp: comparisons of float32 (IEEE: NaN compares
// unequal), int32, or bools (as "!= 0"); logical ops on bools; where selects stored
// words (no float arithmetic, NaN payloads kept). Operand offsets through collapsed
// broadcast strides: m.v = out shape, then strides of a, b, c.
template <typename T>
__device__ __forceinline__ bool compare(int op, T a, T b) {
  switch (op) {
    case TCX_OP_EQUAL: return a == b;
    case TCX_OP_NOT_EQUAL: return a != b;
    case TCX_OP_LESS: return a < b;
    case TCX_OP_LESS_EQUAL: return a <= b;
    case TCX_OP_GREATER: return a > b;
    default: return a >= b;
  }
}

__device__ __forceinline__ void offsets3(int64_t i, const Meta& m, int64_t& oa, int64_t& ob, int64_t& oc) {
  const int r = m.rank;
  oa = ob = oc = 0;
  for (int axis = r - 1; axis >= 0; --axis) {
    const int64_t c = i % m.v[axis];
    i /= m.v[axis];
    oa += c * m.v[r + axis];
    ob += c * m.v[2 * r + axis];
    oc += c * m.v[3 * r + axis];
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
predicate_kernel(int op, const T* __restrict__ a, const T* __restrict__ b, uint8_t* __restrict__ out, int64_t n,
                 Meta m) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    int64_t oa, ob, oc;
    offsets3(i, m, oa, ob, oc);
    bool r;
    if (op == TCX_OP_LOGICAL_NOT) {
      r = a[oa] == T(0);
    } else if (op == TCX_OP_LOGICAL_AND || op == TCX_OP_LOGICAL_OR || op == TCX_OP_LOGICAL_XOR) {
      const bool x = a[oa] != T(0), y = b[ob] != T(0);
      r = op == TCX_OP_LOGICAL_AND ? (x && y) : op == TCX_OP_LOGICAL_OR ? (x || y) : (x != y);
    } else if constexpr (sizeof(T) == 1) {
      r = compare<bool>(op, a[oa] != 0, b[ob] != 0);
    } else {
      r = compare<T>(op, a[oa], b[ob]);
    }
    out[i] = r;
  }
}

template <typename W>
__global__ void __launch_bounds__(kThreads)
where_kernel(const uint8_t* __restrict__ cond, const W* __restrict__ b, const W* __restrict__ c, W* __restrict__ out,
             int64_t n, Meta m) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    int64_t oa, ob, oc;
    offsets3(i, m, oa, ob, oc);
    out[i] = cond[oa] ? b[ob] : c[oc];
  }
}

// ------------------------------------------------------------------- any / all
// predicate.cu:62-75: group g reduces elements g * reduce + j (j < reduce) of the
// plan's flat order, whose source offsets come from (extent, stride) pairs, innermost
// last (core/shape.cpp make_reduction_plan). One warp per group.
__device__ __forceinline__ int64_t pair_offset(int64_t flat, const Meta& m) {
  int64_t off = 0;
  for (int axis = m.rank - 1; axis >= 0; --axis) {
    off += (flat % m.v[2 * axis]) * m.v[2 * axis + 1];
    flat /= m.v[2 * axis];
  }
  return off;
}

__global__ void __launch_bounds__(kThreads)
bool_reduce_kernel(const uint8_t* __restrict__ x, uint8_t* __restrict__ out, int64_t groups, int64_t reduce, Meta m,
                   bool all) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); g < groups; g += warps) {
    bool v = all;
    for (int64_t j = lane; j < reduce; j += 32) {
      const bool e = x[pair_offset(g * reduce + j, m)] != 0;
      v = all ? (v && e) : (v || e);
    }
    const bool r = all ? __all_sync(0xffffffffu, v) : __any_sync(0xffffffffu, v);
    if (lane == 0) out[g] = r;
  }
}

// ----------------------------------------------------------- index copies
// Transpose and slice (elementwise.cu:62-76): output element i (contiguous) reads the
// input at offset + sum(coord_a * stride_a). Metadata collapsed: m.v = out shape, then
// input strides.
template <typename W>
__global__ void __launch_bounds__(kThreads)
gather_kernel(const W* __restrict__ x, W* __restrict__ out, int64_t n, Meta m, int64_t offset) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int r = m.rank;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    int64_t idx = i, src = offset;
    for (int axis = r - 1; axis >= 0; --axis) {
      src += (idx % m.v[axis]) * m.v[r + axis];
      idx /= m.v[axis];
    }
    out[i] = x[src];
  }
}

// The last two output axes read a transposed input (input stride 1 along the output's
// second-to-last axis): 32 x 32 tiles through shared memory, so both the reads (along
// the input's contiguous axis) and the writes (along the output's) are coalesced.
// m.v = out shape, then input strides; the outer axes (all but the last two) index the
// tile's batch.
template <typename W>
__global__ void __launch_bounds__(32 * 8)
transpose_tiles(const W* __restrict__ x, W* __restrict__ out, Meta m, int64_t offset, int64_t tiles_r,
                int64_t tiles_c, int64_t batches) {
  __shared__ W tile[32][33];
  const int r = m.rank;
  const int64_t rows = m.v[r - 2], cols = m.v[r - 1];
  const int64_t in_col_stride = m.v[2 * r - 1];  // input stride of the output's last axis
  const int64_t total = batches * tiles_r * tiles_c;
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    const int64_t bt = t / (tiles_r * tiles_c), rt = (t / tiles_c) % tiles_r, ct = t % tiles_c;
    int64_t idx = bt, base = offset;
    for (int axis = r - 3; axis >= 0; --axis) {
      base += (idx % m.v[axis]) * m.v[r + axis];
      idx /= m.v[axis];
    }
    // read: tile rows are output columns (input rows), lanes run along output rows
    // (input stride 1)
    for (int k = threadIdx.y; k < 32; k += 8) {
      const int64_t oc = ct * 32 + k, orow = rt * 32 + threadIdx.x;
      if (oc < cols && orow < rows) tile[k][threadIdx.x] = x[base + oc * in_col_stride + orow];
    }
    __syncthreads();
    const int64_t obase = bt * rows * cols;
    for (int k = threadIdx.y; k < 32; k += 8) {
      const int64_t orow = rt * 32 + k, oc = ct * 32 + threadIdx.x;
      if (orow < rows && oc < cols) out[obase + orow * cols + oc] = tile[threadIdx.x][k];
    }
    __syncthreads();
  }
}

// concat (elementwise.cu:78-83): input element i goes to output
// (i / block) * out_block + offset + i % block; U words per thread step when every
// run is a multiple of U words and the buffers are aligned for it.
template <typename W>
__global__ void __launch_bounds__(kThreads)
concat_kernel(const W* __restrict__ x, W* __restrict__ out, int64_t n, int64_t block, int64_t out_block,
              int64_t offset) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
    out[(i / block) * out_block + offset + i % block] = x[i];
}

// --------------------------------------------------------------- masked select
// predicate.cu:76-101: positions m of the mask with mask[m] != 0, in order, each copy a
// block of `block` elements. Three passes: per-tile counts, an exclusive scan of the
// tile counts (one CTA; also the total), then each tile compacts its own positions and
// copies their blocks.
constexpr int kMaskTile = 4096;  // mask bytes per tile
constexpr int kScanThreads = 1024;

__global__ void __launch_bounds__(kThreads)
mask_count_kernel(const uint8_t* __restrict__ mask, int64_t n, int64_t* __restrict__ counts) {
  const int64_t t = blockIdx.x, begin = t * kMaskTile, end = min(n, begin + kMaskTile);
  int c = 0;
  for (int64_t i = begin + threadIdx.x; i < end; i += blockDim.x) c += mask[i] != 0;
  c = __reduce_add_sync(0xffffffffu, c);
  __shared__ int part[kThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int w = 0; w < kThreads / 32; ++w) s += part[w];
    counts[t] = s;
  }
}

// Exclusive scan of `tiles` counts in place (counts[t] becomes the first output slot of
// tile t); *total receives the sum.
__global__ void __launch_bounds__(kScanThreads)
mask_scan_kernel(int64_t* __restrict__ counts, int64_t tiles, int64_t* __restrict__ total) {
  __shared__ int64_t warp_sum[kScanThreads / 32];
  __shared__ int64_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t base = 0; base < tiles; base += kScanThreads) {
    const int64_t i = base + threadIdx.x;
    const int64_t v = i < tiles ? counts[i] : 0;
    int64_t inc = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, inc, d);
      if (lane >= d) inc += y;
    }
    if (lane == 31) warp_sum[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      int64_t w = warp_sum[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += y;
      }
      warp_sum[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int64_t before = carry + (warp ? warp_sum[warp - 1] : 0) + inc - v;
    if (i < tiles) counts[i] = before;
    __syncthreads();
    if (threadIdx.x == kScanThreads - 1) carry = before + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = carry;
}

template <typename W>
__global__ void __launch_bounds__(kThreads)
mask_copy_kernel(const W* __restrict__ x, const uint8_t* __restrict__ mask, int64_t n, int64_t block,
                 const int64_t* __restrict__ first, W* __restrict__ out) {
  __shared__ int positions[kMaskTile];
  __shared__ int warp_count[kThreads / 32];
  __shared__ int taken;
  const int64_t t = blockIdx.x, begin = t * kMaskTile, end = min(n, begin + kMaskTile);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) taken = 0;
  __syncthreads();
  // compact this tile's selected positions, in order, kThreads positions per round
  for (int64_t r = begin; r < end; r += kThreads) {
    const int64_t i = r + threadIdx.x;
    const bool sel = i < end && mask[i] != 0;
    const unsigned bits = __ballot_sync(0xffffffffu, sel);
    if (lane == 0) warp_count[warp] = __popc(bits);
    __syncthreads();
    int before = taken;
    for (int w = 0; w < warp; ++w) before += warp_count[w];
    if (sel) positions[before + __popc(bits & ((1u << lane) - 1u))] = static_cast<int>(i - begin);
    __syncthreads();
    if (threadIdx.x == 0) {
      int s = 0;
      for (int w = 0; w < kThreads / 32; ++w) s += warp_count[w];
      taken += s;
    }
    __syncthreads();
  }
  const int64_t count = taken, dst0 = first[t];
  for (int64_t e = threadIdx.x; e < count * block; e += blockDim.x) {
    const int64_t p = e / block, within = e - p * block;
    out[(dst0 + p) * block + within] = x[(begin + positions[p]) * block + within];
  }
}

// ------------------------------------------------------------------------ topk
// math.cu:61-76 / cpu_math.cpp: k rounds of selection in a fixed order: for `largest`,
// NaN first, then larger values, ties (-0 == +0, NaN == NaN) to the lower index; for
// smallest, smaller values first and NaN last. Here each element becomes a unique
// 64-bit key whose descending order is that order (value key high, ~index low), and
// round s picks the largest key below round s-1's. One warp per group. sorted: the
// selection order; otherwise the k selected indices ascending (the reference's
// insertion sort), values gathered by index.
__device__ __forceinline__ uint64_t topk_key(uint32_t w, int64_t j, bool fp, bool largest) {
  uint32_t vk;
  if (fp) {
    if ((w & 0x7fffffffu) > 0x7f800000u) vk = largest ? 0xffffffffu : 0u;
    else vk = largest ? ordered_f32(w) : ~ordered_f32(w);
  } else {
    const uint32_t o = w ^ 0x80000000u;
    vk = largest ? o : ~o;
  }
  return (static_cast<uint64_t>(vk) << 32) | (0xffffffffu - static_cast<uint32_t>(j));
}

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    const uint64_t o = __shfl_xor_sync(0xffffffffu, v, d);
    v = o > v ? o : v;
  }
  return v;
}

__global__ void __launch_bounds__(kThreads)
topk_kernel(const uint32_t* __restrict__ x, uint32_t* __restrict__ values, int32_t* __restrict__ indices,
            int64_t groups, int64_t reduce, int64_t inner, int64_t k, bool fp, bool largest, bool sorted) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); g < groups; g += warps) {
    const int64_t base = (g / inner) * reduce * inner + g % inner;
    const int64_t dest = (g / inner) * k * inner + g % inner;
    uint64_t bound = ~0ull;  // keys are unique and below all-ones (index field < 2^32 - 1)
    for (int64_t s = 0; s < k; ++s) {
      uint64_t best = 0;
      bool found = false;
      for (int64_t j = lane; j < reduce; j += 32) {
        const uint64_t key = topk_key(x[base + j * inner], j, fp, largest);
        if (key < bound && (!found || key > best)) { best = key; found = true; }
      }
      if (!found) best = 0;
      best = warp_max_u64(best);
      bound = best;
      if (sorted && lane == 0) {
        const int64_t j = 0xffffffffu - static_cast<uint32_t>(best);
        indices[dest + s * inner] = static_cast<int32_t>(j);
        values[dest + s * inner] = x[base + j * inner];
      }
    }
    if (!sorted && k > 0) {
      // the selected set is every key >= the k-th one: write it in index order
      int64_t written = 0;
      for (int64_t j0 = 0; j0 < reduce; j0 += 32) {
        const int64_t j = j0 + lane;
        const bool sel = j < reduce && topk_key(x[base + j * inner], j, fp, largest) >= bound;
        const unsigned bits = __ballot_sync(0xffffffffu, sel);
        if (sel) {
          const int64_t slot = written + __popc(bits & ((1u << lane) - 1u));
          indices[dest + slot * inner] = static_cast<int32_t>(j);
          values[dest + slot * inner] = x[base + j * inner];
        }
        written += __popc(bits);
      }
    }
  }
}

// ------------------------------------------------------------------- embedding
// inference.cu:8-15 / cpu_inference.cpp:13-20: output row i is weight row indices[i];
// an index outside [0, vocabulary) raises *bad (its row is left unwritten).
template <bool VEC>
__global__ void __launch_bounds__(kThreads)
embedding_kernel(const int32_t* __restrict__ indices, int64_t rows, const float* __restrict__ weight,
                 int64_t vocabulary, int64_t width, float* __restrict__ out, int* __restrict__ bad) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t w = VEC ? width / 4 : width;
  bool invalid_seen = false;
  for (int64_t e = tid; e < rows * w; e += stride) {
    const int64_t r = e / w, c = e - r * w;
    const int32_t idx = __ldg(indices + r);
    if (idx < 0 || idx >= vocabulary) {
      invalid_seen = true;
      continue;
    }
    if constexpr (VEC) reinterpret_cast<float4*>(out)[e] = __ldg(reinterpret_cast<const float4*>(weight) + idx * w + c);
    else out[e] = __ldg(weight + idx * width + c);
  }
  if (invalid_seen) atomicExch(bad, 1);
}

int grid_for_count(int64_t n, int per_thread = 4) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, int64_t(kThreads) * per_thread),
                                                                 8LL * sm_count() * 4)));
}

// Collapses `operands` stride vectors (each `rank` long) over `shape` into m (m.v = shape,
// then each operand's strides); fails past kMaxRank axes.
int load_collapsed(Meta& m, const int64_t* shape, std::vector<std::vector<int64_t>>& strides, int rank) {
  std::vector<int64_t> out_shape;
  const int r = collapse(shape, strides, rank, out_shape);
  if (r > kMaxRank || static_cast<size_t>(r) * (strides.size() + 1) > sizeof(m.v) / sizeof(m.v[0]))
    return invalid("tensor rank exceeds 16 after collapsing");
  m.rank = r;
  for (int a = 0; a < r; ++a) {
    m.v[a] = out_shape[a];
    for (size_t k = 0; k < strides.size(); ++k) m.v[(k + 1) * r + a] = strides[k][a];
  }
  return TCX_OK;
}

bool fp_dtype(int d) { return d == TCX_FLOAT32; }

}  // namespace
}  // namespace tcx

using namespace tcx;

extern "C" {

int tcx_sm100_map(tcx_stream_t stream, int op, int dtype, const void* input, void* output, int64_t count,
                  double scalar, int32_t scalar_left) {
  clear_error();
  const bool scalar_op = op == TCX_OP_ADD_SCALAR || op == TCX_OP_SUBTRACT_SCALAR || op == TCX_OP_MULTIPLY_SCALAR ||
                         op == TCX_OP_DIVIDE_SCALAR;
  if (!scalar_op && op != TCX_OP_NEGATE && op != TCX_OP_LOG && op != TCX_OP_SQRT && op != TCX_OP_ABS)
    return invalid("unsupported elementwise operation");
  if (dtype != TCX_FLOAT32 && dtype != TCX_INT32) return invalid("CUDA operations only support float32");
  if (dtype == TCX_INT32 && (op == TCX_OP_LOG || op == TCX_OP_SQRT)) return invalid("log/sqrt only support float32 tensors");
  if (dtype == TCX_INT32 && op == TCX_OP_DIVIDE_SCALAR) return invalid("CUDA operation only supports float32 for this dtype");
  if (dtype == TCX_INT32 && scalar_op &&
      !(scalar == static_cast<double>(static_cast<int64_t>(scalar)) && scalar >= -2147483648.0 && scalar <= 2147483647.0))
    return invalid("fill/arithmetic scalar must be an integer in int32 range");
  if (count < 0) return invalid("negative element count");
  if (count == 0) return TCX_OK;
  if (!input || !output) return invalid("missing buffer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const float fs = static_cast<float>(scalar);
  const uint32_t is = scalar_op && dtype == TCX_INT32 ? static_cast<uint32_t>(static_cast<int32_t>(scalar)) : 0u;
  const bool left = scalar_left != 0;
  auto* x = static_cast<const uint32_t*>(input);
  auto* o = static_cast<uint32_t*>(output);
  const int grid = grid_for_count(count);
  TimedLaunch timer("map", s);
#define TCX_MAP(OPC)                                                                          \
  case OPC:                                                                                   \
    if (dtype == TCX_FLOAT32) map_kernel<OPC, true><<<grid, kThreads, 0, s>>>(x, o, count, fs, is, left);  \
    else map_kernel<OPC, false><<<grid, kThreads, 0, s>>>(x, o, count, fs, is, left);         \
    break;
  switch (op) {
    TCX_MAP(TCX_OP_NEGATE)
    TCX_MAP(TCX_OP_ADD_SCALAR)
    TCX_MAP(TCX_OP_SUBTRACT_SCALAR)
    TCX_MAP(TCX_OP_MULTIPLY_SCALAR)
    TCX_MAP(TCX_OP_ABS)
    case TCX_OP_DIVIDE_SCALAR: map_kernel<TCX_OP_DIVIDE_SCALAR, true><<<grid, kThreads, 0, s>>>(x, o, count, fs, is, left); break;
    case TCX_OP_LOG: map_kernel<TCX_OP_LOG, true><<<grid, kThreads, 0, s>>>(x, o, count, fs, is, left); break;
    default: map_kernel<TCX_OP_SQRT, true><<<grid, kThreads, 0, s>>>(x, o, count, fs, is, left); break;
  }
#undef TCX_MAP
  return launch_status("elementwise map");
}

int tcx_sm100_cast(tcx_stream_t stream, int src_dtype, int dst_dtype, const void* input, void* output, int64_t count,
                   int* invalid_flag) {
  clear_error();
  auto known = [](int d) { return d == TCX_FLOAT32 || d == TCX_INT32 || d == TCX_BOOL; };
  if (!known(src_dtype) || !known(dst_dtype)) return invalid("unsupported cast target dtype");
  if (count < 0) return invalid("negative element count");
  const bool checked = src_dtype == TCX_FLOAT32 && dst_dtype == TCX_INT32;
  if (checked && !invalid_flag) return invalid("float32 to int32 casts need a device flag");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (checked && cudaMemsetAsync(invalid_flag, 0, sizeof(int), s) != cudaSuccess) return launch_status("cast flag reset");
  if (count == 0) return TCX_OK;
  if (!input || !output) return invalid("missing buffer");
  if (src_dtype == dst_dtype) {
    const size_t bytes = static_cast<size_t>(count) * (src_dtype == TCX_BOOL ? 1 : 4);
    if (cudaMemcpyAsync(output, input, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return launch_status("cast copy");
    return TCX_OK;
  }
  TimedLaunch timer("cast", s);
  cast_kernel<<<grid_for_count(count, 2), kThreads, 0, s>>>(input, output, count, src_dtype, dst_dtype, invalid_flag);
  return launch_status("cast");
}

int tcx_sm100_predicate(tcx_stream_t stream, int op, int dtype, const void* a, const void* b, const void* c,
                        void* output, int64_t count, const int64_t* metadata, int32_t rank) {
  clear_error();
  const bool where = op == TCX_OP_WHERE;
  const bool logical = op == TCX_OP_LOGICAL_AND || op == TCX_OP_LOGICAL_OR || op == TCX_OP_LOGICAL_XOR ||
                       op == TCX_OP_LOGICAL_NOT;
  const bool comparison = op >= TCX_OP_EQUAL && op <= TCX_OP_GREATER_EQUAL;
  if (!where && !logical && !comparison) return invalid("invalid predicate operation or input count");
  if (dtype != TCX_FLOAT32 && dtype != TCX_INT32 && dtype != TCX_BOOL) return invalid("unsupported dtype");
  if (logical && dtype != TCX_BOOL) return invalid("logical operations require bool tensors");
  if (count < 0 || rank < 0) return invalid("negative extents");
  if (count == 0) return TCX_OK;
  if (rank > 0 && !metadata) return invalid("missing predicate metadata");
  const int operands = where ? 3 : op == TCX_OP_LOGICAL_NOT ? 1 : 2;
  std::vector<std::vector<int64_t>> st(3, std::vector<int64_t>(rank, 0));
  for (int k = 0; k < operands; ++k) st[k].assign(metadata + (k + 1) * rank, metadata + (k + 2) * rank);
  Meta m;
  if (int rc = load_collapsed(m, metadata, st, rank)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid = grid_for_count(count, 2);
  TimedLaunch timer("predicate", s);
  if (where) {
    if (dtype == TCX_BOOL)
      where_kernel<uint8_t><<<grid, kThreads, 0, s>>>(static_cast<const uint8_t*>(a), static_cast<const uint8_t*>(b),
                                                      static_cast<const uint8_t*>(c), static_cast<uint8_t*>(output),
                                                      count, m);
    else
      where_kernel<uint32_t><<<grid, kThreads, 0, s>>>(static_cast<const uint8_t*>(a), static_cast<const uint32_t*>(b),
                                                       static_cast<const uint32_t*>(c), static_cast<uint32_t*>(output),
                                                       count, m);
  } else if (dtype == TCX_FLOAT32) {
    predicate_kernel<float><<<grid, kThreads, 0, s>>>(op, static_cast<const float*>(a), static_cast<const float*>(b),
                                                      static_cast<uint8_t*>(output), count, m);
  } else if (dtype == TCX_INT32) {
    predicate_kernel<int32_t><<<grid, kThreads, 0, s>>>(op, static_cast<const int32_t*>(a),
                                                        static_cast<const int32_t*>(b),
                                                        static_cast<uint8_t*>(output), count, m);
  } else {
    predicate_kernel<uint8_t><<<grid, kThreads, 0, s>>>(op, static_cast<const uint8_t*>(a),
                                                        static_cast<const uint8_t*>(b),
                                                        static_cast<uint8_t*>(output), count, m);
  }
  return launch_status("predicate");
}

int tcx_sm100_bool_reduce(tcx_stream_t stream, int op, const void* input, void* output, int64_t groups,
                          int64_t reduction_size, const int64_t* index_metadata, int32_t rank) {
  clear_error();
  if (op != TCX_OP_ANY && op != TCX_OP_ALL) return invalid("expected a boolean reduction operation");
  if (groups < 0 || reduction_size < 0 || rank < 0) return invalid("malformed reduction plan");
  if (groups == 0) return TCX_OK;
  if (rank > kMaxRank || (rank > 0 && !index_metadata)) return invalid("missing or oversized reduction metadata");
  Meta m;
  m.rank = rank;
  for (int i = 0; i < 2 * rank; ++i) m.v[i] = index_metadata[i];
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(groups, kThreads / 32),
                                                                           8LL * sm_count())));
  TimedLaunch timer("bool_reduce", s);
  bool_reduce_kernel<<<grid, kThreads, 0, s>>>(static_cast<const uint8_t*>(input), static_cast<uint8_t*>(output),
                                                groups, reduction_size, m, op == TCX_OP_ALL);
  return launch_status("bool reduction");
}

int tcx_sm100_index_copy(tcx_stream_t stream, int32_t element_bytes, const void* input, void* output, int64_t count,
                         const int64_t* shape, const int64_t* input_strides, int32_t rank, int64_t offset) {
  clear_error();
  if (element_bytes != 1 && element_bytes != 4) return invalid("index copies move 1- or 4-byte elements");
  if (count < 0 || rank < 0 || offset < 0) return invalid("negative extents");
  if (count == 0) return TCX_OK;
  if (rank > 0 && (!shape || !input_strides)) return invalid("missing index-copy metadata");
  std::vector<std::vector<int64_t>> st = {std::vector<int64_t>(input_strides, input_strides + rank)};
  std::vector<int64_t> sh(shape, shape + rank);
  Meta m;
  if (int rc = load_collapsed(m, sh.data(), st, rank)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int r = m.rank;
  if (element_bytes == 4 && r >= 2 && m.v[2 * r - 2] == 1 && m.v[2 * r - 1] != 1 && m.v[r - 2] >= 16 &&
      m.v[r - 1] >= 16) {
    const int64_t tr = ceil_div(m.v[r - 2], 32), tc = ceil_div(m.v[r - 1], 32);
    const int64_t batches = count / (m.v[r - 2] * m.v[r - 1]);
    const int grid = static_cast<int>(std::min<int64_t>(batches * tr * tc, 16LL * sm_count()));
    TimedLaunch timer("transpose_tiles", s);
    transpose_tiles<uint32_t><<<grid, dim3(32, 8), 0, s>>>(static_cast<const uint32_t*>(input),
                                                           static_cast<uint32_t*>(output), m, offset, tr, tc, batches);
    return launch_status("transpose");
  }
  TimedLaunch timer("index_copy", s);
  if (element_bytes == 4)
    gather_kernel<uint32_t><<<grid_for_count(count, 2), kThreads, 0, s>>>(
        static_cast<const uint32_t*>(input), static_cast<uint32_t*>(output), count, m, offset);
  else
    gather_kernel<uint8_t><<<grid_for_count(count, 2), kThreads, 0, s>>>(
        static_cast<const uint8_t*>(input), static_cast<uint8_t*>(output), count, m, offset);
  return launch_status("index copy");
}

int tcx_sm100_concat(tcx_stream_t stream, int32_t element_bytes, const void* input, void* output, int64_t count,
                     int64_t block, int64_t output_block, int64_t offset) {
  clear_error();
  if (element_bytes != 1 && element_bytes != 4) return invalid("concat moves 1- or 4-byte elements");
  if (count < 0 || block < 0 || output_block < block || offset < 0 || offset + block > output_block)
    return invalid("malformed concat plan");
  if (count == 0) return TCX_OK;
  if (block == 0 || count % block) return invalid("malformed concat plan");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  TimedLaunch timer("concat", s);
  const int64_t unit = 16 / element_bytes;  // elements per 16 bytes
  const bool vec = block % unit == 0 && output_block % unit == 0 && offset % unit == 0 &&
                   ((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(output)) & 15) == 0;
  if (vec)
    concat_kernel<uint4><<<grid_for_count(count / unit, 1), kThreads, 0, s>>>(
        static_cast<const uint4*>(input), static_cast<uint4*>(output), count / unit, block / unit,
        output_block / unit, offset / unit);
  else if (element_bytes == 4)
    concat_kernel<uint32_t><<<grid_for_count(count, 2), kThreads, 0, s>>>(
        static_cast<const uint32_t*>(input), static_cast<uint32_t*>(output), count, block, output_block, offset);
  else
    concat_kernel<uint8_t><<<grid_for_count(count, 2), kThreads, 0, s>>>(
        static_cast<const uint8_t*>(input), static_cast<uint8_t*>(output), count, block, output_block, offset);
  return launch_status("concat");
}

size_t tcx_sm100_masked_select_workspace_bytes(int64_t mask_count) {
  if (mask_count <= 0) return 0;
  return static_cast<size_t>(ceil_div(mask_count, kMaskTile) + 1) * sizeof(int64_t);
}

int tcx_sm100_masked_select_count(tcx_stream_t stream, const void* mask, int64_t mask_count, int64_t* selected,
                                  void* workspace, size_t workspace_bytes) {
  clear_error();
  if (mask_count < 0) return invalid("negative element count");
  if (!selected) return invalid("missing count output");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (mask_count == 0) {
    if (cudaMemsetAsync(selected, 0, sizeof(int64_t), s) != cudaSuccess) return launch_status("mask count");
    return TCX_OK;
  }
  if (!mask || !workspace || workspace_bytes < tcx_sm100_masked_select_workspace_bytes(mask_count))
    return invalid("masked select workspace is missing or too small");
  const int64_t tiles = ceil_div(mask_count, kMaskTile);
  auto* counts = static_cast<int64_t*>(workspace);
  TimedLaunch timer("mask_count", s);
  mask_count_kernel<<<static_cast<unsigned>(tiles), kThreads, 0, s>>>(static_cast<const uint8_t*>(mask), mask_count,
                                                                      counts);
  mask_scan_kernel<<<1, kScanThreads, 0, s>>>(counts, tiles, selected);
  return launch_status("mask count");
}

int tcx_sm100_masked_select(tcx_stream_t stream, int32_t element_bytes, const void* input, const void* mask,
                            int64_t mask_count, int64_t block, void* output, const void* workspace,
                            size_t workspace_bytes) {
  clear_error();
  if (element_bytes != 1 && element_bytes != 4) return invalid("masked select moves 1- or 4-byte elements");
  if (mask_count < 0 || block < 0) return invalid("negative extents");
  if (mask_count == 0 || block == 0) return TCX_OK;
  if (!input || !mask || !output || !workspace ||
      workspace_bytes < tcx_sm100_masked_select_workspace_bytes(mask_count))
    return invalid("masked select workspace is missing or too small");
  const int64_t tiles = ceil_div(mask_count, kMaskTile);
  if (tiles > INT32_MAX) return invalid("mask too large");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto* first = static_cast<const int64_t*>(workspace);
  TimedLaunch timer("mask_copy", s);
  if (element_bytes == 4)
    mask_copy_kernel<uint32_t><<<static_cast<unsigned>(tiles), kThreads, 0, s>>>(
        static_cast<const uint32_t*>(input), static_cast<const uint8_t*>(mask), mask_count, block, first,
        static_cast<uint32_t*>(output));
  else
    mask_copy_kernel<uint8_t><<<static_cast<unsigned>(tiles), kThreads, 0, s>>>(
        static_cast<const uint8_t*>(input), static_cast<const uint8_t*>(mask), mask_count, block, first,
        static_cast<uint8_t*>(output));
  return launch_status("masked select");
}

int tcx_sm100_topk(tcx_stream_t stream, int dtype, const void* input, void* values, int32_t* indices, int64_t groups,
                   int64_t reduction_size, int64_t inner, int64_t k, int32_t largest, int32_t sorted) {
  clear_error();
  if (dtype != TCX_FLOAT32 && dtype != TCX_INT32) return invalid("math operations require float32 or int32 tensors");
  if (groups < 0 || reduction_size < 0 || inner < 0 || k < 0 || k > reduction_size)
    return invalid("topk k must be between zero and the axis size");
  if (reduction_size > INT32_MAX) return invalid("topk index range exceeds int32");
  if (groups == 0 || k == 0) return TCX_OK;
  if (inner <= 0 || !input || !values || !indices) return invalid("missing topk buffer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(groups, kThreads / 32),
                                                                           8LL * sm_count())));
  TimedLaunch timer("topk", s);
  topk_kernel<<<grid, kThreads, 0, s>>>(static_cast<const uint32_t*>(input), static_cast<uint32_t*>(values), indices,
                                        groups, reduction_size, inner, k, fp_dtype(dtype), largest != 0, sorted != 0);
  return launch_status("topk");
}

int tcx_sm100_embedding(tcx_stream_t stream, const int32_t* indices, int64_t rows, const float* weight,
                        int64_t vocabulary, int64_t width, float* output, int* invalid_flag) {
  clear_error();
  if (rows < 0 || vocabulary < 0 || width < 0) return invalid("negative extents");
  if (!invalid_flag) return invalid("embedding needs a device flag");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(invalid_flag, 0, sizeof(int), s) != cudaSuccess) return launch_status("embedding flag reset");
  if (rows == 0) return TCX_OK;
  if (!indices || (width > 0 && (!weight || !output))) return invalid("missing embedding buffer");
  const bool vec = width % 4 == 0 &&
                   ((reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(output)) & 15) == 0;
  const int64_t work = rows * std::max<int64_t>(1, vec ? width / 4 : width);
  TimedLaunch timer("embedding", s);
  if (vec)
    embedding_kernel<true><<<grid_for_count(work, 1), kThreads, 0, s>>>(indices, rows, weight, vocabulary, width, output,
                                                                        invalid_flag);
  else
    embedding_kernel<false><<<grid_for_count(work, 1), kThreads, 0, s>>>(indices, rows, weight, vocabulary, width,
                                                                         output, invalid_flag);
  return launch_status("embedding");
}

}  // extern "C"
