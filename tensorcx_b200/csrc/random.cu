// Seeded float32 generation on the device (the reference draws its randn values on
// the host with NumPy and uploads them: python/tensorcx/tensor.py:485-497,
// cpp/tensorcx/backends/cuda/cuda_backend.cpp:215-236).
//
// Bit stream: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC'11), counter-based: element e of the logical stream takes word
// e % 4 of Philox(counter = (e / 4 as a 64-bit number, 0, 0), key = seed). A value
// depends only on (seed, e), so any grid shape, and any split of the stream into
// slices (shards at offsets), gives the same numbers. It does not reproduce NumPy's
// PCG64 / ziggurat stream bit for bit; nothing on the device can.
//
// Distributions:
//  * uniform [a, b): u = (w >> 8) * 2^-24 (24 random bits, exact), value = fma(b - a, u, a);
//  * normal (mean a, std b): Box-Muller on the pair of words (2p, 2p + 1) of a block,
//    u1 = ((w0 >> 8) + 1) * 2^-24 in (0, 1], u2 = (w1 >> 8) * 2^-24,
//    r = sqrt(-2 ln u1), t = fma(u2, 2 pi, -pi) in [-pi, pi) (a uniform angle),
//    element 2p gets r cos t, element 2p + 1 r sin t, value = fma(b, z, a). The sine and
//    cosine are the SFU's (__sincosf: absolute error at most 2^-21.41 on [-pi, pi]).
//    -ln u1 comes from the SFU's log2 (lg2.approx) times ln 2 while v = 1 - u1 >= 2^-5,
//    and from the series -ln(1 - v) = v + v^2/2 + ... + v^6/6 (first omitted term under
//    2^-30 of the sum) below that, where a coarse logarithm's absolute error would be
//    magnified: r = sqrt(y) near 0 carries y's error divided by 2r. The square root is
//    y * rsqrt(y) (rsqrt.approx; y = 0 gives 0). Against double precision the values
//    stay within 1e-6 + 4e-7 |z|.
//
// The kernel is bound by instruction issue (Philox-10 is ~40 integer instructions per
// four values), not by the 4 bytes written per value: the round keys are computed once
// per thread, each round's two products are 32 x 32 -> 64-bit multiplies (high and low
// halves from one product), the full blocks of an aligned output take a loop without
// bounds tests, two blocks per iteration (one 128-bit streaming store each), and the
// ragged ends another.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace tcx {
namespace {

constexpr uint32_t kPhiloxM0 = 0xD2511F53u, kPhiloxM1 = 0xCD9E8D57u;  // round multipliers
constexpr uint32_t kPhiloxW0 = 0x9E3779B9u, kPhiloxW1 = 0xBB67AE85u;  // key schedule (Weyl)
constexpr float kTwoPow24Inv = 5.9604644775390625e-08f;               // 2^-24
constexpr float kPi = 3.14159265358979323846f, kTwoPi = 6.28318530717958647692f;

// The ten round keys of `key` (the Weyl sequence), computed once per thread.
struct RoundKeys {
  uint32_t x[10], y[10];
};
__device__ __forceinline__ RoundKeys round_keys(uint2 k) {
  RoundKeys rk;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    rk.x[r] = k.x + static_cast<uint32_t>(r) * kPhiloxW0;
    rk.y[r] = k.y + static_cast<uint32_t>(r) * kPhiloxW1;
  }
  return rk;
}

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, const RoundKeys& rk) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = static_cast<uint64_t>(kPhiloxM0) * c.x, p1 = static_cast<uint64_t>(kPhiloxM1) * c.z;
    const uint32_t hi0 = static_cast<uint32_t>(p0 >> 32), lo0 = static_cast<uint32_t>(p0);
    const uint32_t hi1 = static_cast<uint32_t>(p1 >> 32), lo1 = static_cast<uint32_t>(p1);
    c = make_uint4(hi1 ^ c.y ^ rk.x[r], lo1, hi0 ^ c.w ^ rk.y[r], lo0);
  }
  return c;
}

// -ln u for u in (0, 1] as described above (v = 1 - u is exact for u >= 1/2).
__device__ __forceinline__ float neg_ln(float u) {
  constexpr float kLn2 = 0.69314718055994531f;
  float l2;
  asm("lg2.approx.f32 %0, %1;" : "=f"(l2) : "f"(u));
  const float v = __fsub_rn(1.0f, u);
  float sr = __fmaf_rn(v, 1.0f / 6.0f, 0.2f);
  sr = __fmaf_rn(v, sr, 0.25f);
  sr = __fmaf_rn(v, sr, 1.0f / 3.0f);
  sr = __fmaf_rn(v, sr, 0.5f);
  sr = __fmaf_rn(v, sr, 1.0f);
  sr = __fmul_rn(v, sr);
  return v < 0.03125f ? sr : __fmul_rn(-kLn2, l2);
}

__device__ __forceinline__ float sqrt_approx(float y) {
  float r;
  asm("rsqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(y));
  return y > 0.0f ? __fmul_rn(y, r) : 0.0f;
}

template <bool NORMAL>
__device__ __forceinline__ float4 block_values(uint4 w, float a, float b) {
  float4 v;
  if constexpr (NORMAL) {
    const float u1a = __fmul_rn(static_cast<float>((w.x >> 8) + 1u), kTwoPow24Inv);
    const float u2a = __fmul_rn(static_cast<float>(w.y >> 8), kTwoPow24Inv);
    const float u1b = __fmul_rn(static_cast<float>((w.z >> 8) + 1u), kTwoPow24Inv);
    const float u2b = __fmul_rn(static_cast<float>(w.w >> 8), kTwoPow24Inv);
    const float ra = sqrt_approx(2.0f * neg_ln(u1a)), rb = sqrt_approx(2.0f * neg_ln(u1b));
    float sa, ca, sb, cb;
    __sincosf(__fmaf_rn(u2a, kTwoPi, -kPi), &sa, &ca);
    __sincosf(__fmaf_rn(u2b, kTwoPi, -kPi), &sb, &cb);
    v.x = __fmaf_rn(b, __fmul_rn(ra, ca), a);
    v.y = __fmaf_rn(b, __fmul_rn(ra, sa), a);
    v.z = __fmaf_rn(b, __fmul_rn(rb, cb), a);
    v.w = __fmaf_rn(b, __fmul_rn(rb, sb), a);
  } else {
    const float span = __fsub_rn(b, a);
    v.x = __fmaf_rn(span, __fmul_rn(static_cast<float>(w.x >> 8), kTwoPow24Inv), a);
    v.y = __fmaf_rn(span, __fmul_rn(static_cast<float>(w.y >> 8), kTwoPow24Inv), a);
    v.z = __fmaf_rn(span, __fmul_rn(static_cast<float>(w.z >> 8), kTwoPow24Inv), a);
    v.w = __fmaf_rn(span, __fmul_rn(static_cast<float>(w.w >> 8), kTwoPow24Inv), a);
  }
  return v;
}

__device__ __forceinline__ uint4 block_words(uint64_t blk, const RoundKeys& rk) {
  return philox4x32_10(make_uint4(static_cast<uint32_t>(blk), static_cast<uint32_t>(blk >> 32), 0u, 0u), rk);
}

// Elements [offset, offset + count) of the stream into out[0, count); element e is word
// e % 4 of Philox block e / 4. With a 16-byte aligned output and offset % 4 == 0, the
// full blocks go through a loop of 128-bit streaming stores (written once, read later)
// and the partial last block element by element; otherwise every block is stored
// element by element with its bounds tested.
template <bool NORMAL, bool ALIGNED>
__global__ void __launch_bounds__(256)
random_kernel(float* __restrict__ out, int64_t count, uint64_t offset, uint2 key, float a, float b) {
  const RoundKeys rk = round_keys(key);
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t first_block = offset >> 2;
  if constexpr (ALIGNED) {
    const uint64_t full = static_cast<uint64_t>(count) >> 2;
    float4* out4 = reinterpret_cast<float4*>(out);
    // two blocks per iteration (independent instruction streams); the second is computed
    // past the end on the last iteration and not stored
    for (uint64_t i = tid; i < full; i += 2 * stride) {
      const uint64_t j = i + stride;
      const float4 v0 = block_values<NORMAL>(block_words(first_block + i, rk), a, b);
      const float4 v1 = block_values<NORMAL>(block_words(first_block + j, rk), a, b);
      __stcs(out4 + i, v0);
      if (j < full) __stcs(out4 + j, v1);
    }
    const int rest = static_cast<int>(count & 3);
    if (rest && tid == 0) {
      const float4 v = block_values<NORMAL>(block_words(first_block + full, rk), a, b);
      const float vals[4] = {v.x, v.y, v.z, v.w};
      for (int j = 0; j < rest; ++j) out[4 * full + j] = vals[j];
    }
  } else {
    const uint64_t end = offset + static_cast<uint64_t>(count);
    const uint64_t blocks = ((end + 3) >> 2) - first_block;
    for (uint64_t i = tid; i < blocks; i += stride) {
      const uint64_t blk = first_block + i;
      const float4 v = block_values<NORMAL>(block_words(blk, rk), a, b);
      const float vals[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint64_t e = (blk << 2) + j;
        if (e >= offset && e < end) out[e - offset] = vals[j];
      }
    }
  }
}

}  // namespace
}  // namespace tcx

using namespace tcx;

extern "C" int tcx_sm100_random(tcx_stream_t stream, int distribution, float* out, int64_t count, uint64_t seed,
                                uint64_t offset, float a, float b) {
  clear_error();
  if (distribution != TCX_RANDOM_NORMAL && distribution != TCX_RANDOM_UNIFORM)
    return invalid("unknown random distribution");
  if (count < 0) return invalid("negative element count");
  if (count == 0) return TCX_OK;
  if (!out) return invalid("missing output");
  if (offset > UINT64_MAX - static_cast<uint64_t>(count) - 3) return invalid("stream offset overflows");
  if (!(a == a) || !(b == b) || a == INFINITY || a == -INFINITY || b == INFINITY || b == -INFINITY)
    return invalid("distribution parameters must be finite");
  if (distribution == TCX_RANDOM_NORMAL && b < 0) return invalid("normal standard deviation must be non-negative");
  if (distribution == TCX_RANDOM_UNIFORM && !(a <= b)) return invalid("uniform bounds need low <= high");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const uint64_t blocks = ((offset + static_cast<uint64_t>(count) + 3) >> 2) - (offset >> 2);
  const uint64_t want = (blocks + 255) / 256;
  const int grid = static_cast<int>(want < static_cast<uint64_t>(8 * sm_count()) ? want : 8 * sm_count());
  const uint2 key = make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  const bool aligned = (reinterpret_cast<uintptr_t>(out) & 15) == 0 && (offset & 3) == 0;
  TimedLaunch timer("random", s);
  if (distribution == TCX_RANDOM_NORMAL) {
    if (aligned) random_kernel<true, true><<<grid, 256, 0, s>>>(out, count, offset, key, a, b);
    else random_kernel<true, false><<<grid, 256, 0, s>>>(out, count, offset, key, a, b);
  } else {
    if (aligned) random_kernel<false, true><<<grid, 256, 0, s>>>(out, count, offset, key, a, b);
    else random_kernel<false, false><<<grid, 256, 0, s>>>(out, count, offset, key, a, b);
  }
  return launch_status("random generation");
}
