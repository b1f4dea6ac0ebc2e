/* TEST INFRASTRUCTURE ONLY — the CPU oracle for the tensor.cx hot path.
 *
 * A plain-C restatement of the reference CPU backend's arithmetic, used by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker. It is
 * never linked into, loaded by or called from the product library.
 *
 * Each function follows one reference function (paths relative to the tensor.cx
 * repository) operation by operation, in the same order and in float32, so that a
 * build with the reference's flags (-O3, no fast-math, x86-64 baseline: no FMA
 * contraction) reproduces its results bit for bit. Shape planning (outer/reduce/
 * inner, index metadata, batch offsets) is restated in oracle/oracle.py.
 *
 * Parity pin: tests/test_oracle.py compares every function here with the
 * reference itself (oracle/_ref/libtcx_ref.so, built from the reference sources)
 * and with the committed golden fixtures in tests/golden/.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

typedef uint32_t word;

static word fbits(float f) { word w; memcpy(&w, &f, 4); return w; }
static float bitsf(word w) { float f; memcpy(&f, &w, 4); return f; }

/* Single-axis float32 reduction over (outer, reduce, inner):
 * cpu::reduce, cpu_backend.cpp:1178-1221. op: 0 sum, 1 max, 2 mean. */
void tcxo_reduce_axis_f32(int op, const float* x, float* out, int64_t outer,
                          int64_t reduce, int64_t inner) {
  const int64_t count = outer * inner;
  for (int64_t id = 0; id < count; ++id) {
    const int64_t base = (id / inner) * reduce * inner + id % inner;
    if (op == 1) {
      float m = -INFINITY;
      for (int64_t r = 0; r < reduce; ++r) {
        const float v = x[base + r * inner];
        if (isnan(v)) { m = v; break; }
        m = (m < v) ? v : m; /* std::max keeps the first argument on ties */
      }
      out[id] = m;
    } else {
      if (op == 2 && reduce == 0) { out[id] = NAN; continue; }
      float s = 0.0f;
      for (int64_t r = 0; r < reduce; ++r) s += x[base + r * inner];
      out[id] = op == 2 ? s / (float)reduce : s;
    }
  }
}

/* Single-axis int32 reduction: cpu::reduce, cpu_backend.cpp:1223-1247.
 * op: 0 sum (uint32 wraparound), 1 max. */
void tcxo_reduce_axis_i32(int op, const int32_t* x, int32_t* out, int64_t outer,
                          int64_t reduce, int64_t inner) {
  const int64_t count = outer * inner;
  for (int64_t id = 0; id < count; ++id) {
    const int64_t base = (id / inner) * reduce * inner + id % inner;
    if (op == 1) {
      int32_t m = INT32_MIN;
      for (int64_t r = 0; r < reduce; ++r) {
        const int32_t v = x[base + r * inner];
        m = m < v ? v : m;
      }
      out[id] = m;
    } else {
      uint32_t s = 0;
      for (int64_t r = 0; r < reduce; ++r) s += (uint32_t)x[base + r * inner];
      out[id] = (int32_t)s;
    }
  }
}

/* Index-metadata offset used by multi-axis reductions and min/argmax:
 * cpu::reduce's `offset` lambda, cpu_backend.cpp:1114-1122 (pairs of
 * extent/stride, innermost pair last). */
static int64_t meta_offset(int64_t index, const int64_t* meta, int64_t begin, int64_t end) {
  int64_t value = 0;
  for (int64_t axis = end; axis-- > begin;) {
    const int64_t extent = meta[2 * axis];
    value += (index % extent) * meta[2 * axis + 1];
    index /= extent;
  }
  return value;
}

/* Multi-axis reduction over metadata (kept pairs first, reduced pairs last):
 * cpu::reduce, cpu_backend.cpp:1123-1152. op: 0 sum, 1 max, 2 mean;
 * dtype 0 float32, 1 int32. A full-tensor reduction is the all-axes case. */
void tcxo_reduce_axes(int op, int dtype, const void* x, void* out, int64_t groups,
                      int64_t reduction_size, const int64_t* meta, int64_t outer_rank,
                      int64_t rank) {
  for (int64_t g = 0; g < groups; ++g) {
    const int64_t base = meta_offset(g, meta, 0, outer_rank);
    if (dtype == 0) {
      const float* xf = (const float*)x;
      float value = op == 1 ? -INFINITY : 0.0f;
      for (int64_t r = 0; r < reduction_size; ++r) {
        const float item = xf[base + meta_offset(r, meta, outer_rank, rank)];
        if (op == 1) {
          if (isnan(item)) { value = item; break; }
          value = (value < item) ? item : value;
        } else {
          value += item;
        }
      }
      if (op == 2) value = reduction_size ? value / (float)reduction_size : NAN;
      ((float*)out)[g] = value;
    } else {
      const int32_t* xi = (const int32_t*)x;
      uint32_t sum = 0;
      int32_t maximum = INT32_MIN;
      for (int64_t r = 0; r < reduction_size; ++r) {
        const int32_t item = xi[base + meta_offset(r, meta, outer_rank, rank)];
        if (op == 1) maximum = maximum < item ? item : maximum;
        else sum += (uint32_t)item;
      }
      ((int32_t*)out)[g] = op == 1 ? maximum : (int32_t)sum;
    }
  }
}

/* Total order helpers of cpu_math.cpp:14-21: NaN test and `less` with both
 * zeros equal, on raw 32-bit words. */
static int word_nan(word a, int fp) { return fp && (a & 0x7fffffffu) > 0x7f800000u; }
static int word_less(word a, word b, int fp) {
  if (!fp) return (int32_t)a < (int32_t)b;
  if (!(a & 0x7fffffffu)) a = 0;
  if (!(b & 0x7fffffffu)) b = 0;
  const word ka = (a & 0x80000000u) ? ~a : (a ^ 0x80000000u);
  const word kb = (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
  return ka < kb;
}

/* min (code 3) / argmax (code 4) over metadata: cpu::execute_math,
 * cpu_math.cpp:48-54. The first NaN wins; otherwise the first extremum wins
 * (strict comparison), with both zeros comparing equal. */
void tcxo_min_argmax(int code, int fp, const void* x, void* out, int64_t groups,
                     int64_t reduce, const int64_t* meta, int64_t rank) {
  const word* xw = (const word*)x;
  word* ow = (word*)out;
  for (int64_t i = 0; i < groups; ++i) {
    word best = xw[meta_offset(i * reduce, meta, 0, rank)];
    int64_t index = 0;
    for (int64_t j = 1; j < reduce; ++j) {
      const word a = xw[meta_offset(i * reduce + j, meta, 0, rank)];
      if (!word_nan(best, fp) &&
          (word_nan(a, fp) || (code == 3 ? word_less(a, best, fp) : word_less(best, a, fp)))) {
        best = a;
        index = j;
      }
    }
    ow[i] = code == 4 ? (word)index : best;
  }
}

/* clip (code 5) with broadcast metadata (shape, then the element strides of x,
 * lower and upper): cpu_math.cpp:42-47. */
void tcxo_clip(int fp, const void* x, const void* lo, const void* hi, void* out,
               int64_t count, const int64_t* meta, int64_t rank) {
  const word* in[3] = {(const word*)x, (const word*)lo, (const word*)hi};
  word* ow = (word*)out;
  for (int64_t i = 0; i < count; ++i) {
    int64_t off[3] = {0, 0, 0};
    for (int arg = 0; arg < 3; ++arg) {
      int64_t flat = i;
      for (int64_t a = rank; a-- > 0;) {
        off[arg] += flat % meta[a] * meta[(arg + 1) * rank + a];
        flat /= meta[a];
      }
    }
    word a = in[0][off[0]];
    const word l = in[1][off[1]], h = in[2][off[2]];
    if (!word_nan(a, fp)) a = (word_nan(l, fp) || !word_less(l, a, fp)) ? l : a;
    if (!word_nan(a, fp)) a = (word_nan(h, fp) || !word_less(a, h, fp)) ? h : a;
    ow[i] = a;
  }
}

/* softmax over (outer, reduce, inner): compute_softmax, cpu_backend.cpp:125-155. */
void tcxo_softmax(const float* x, float* out, int64_t outer, int64_t reduce, int64_t inner) {
  for (int64_t o = 0; o < outer; ++o) {
    for (int64_t in = 0; in < inner; ++in) {
      const int64_t base = o * reduce * inner + in;
      float maxv = -INFINITY;
      for (int64_t r = 0; r < reduce; ++r) {
        const float v = x[base + r * inner];
        if (isnan(v)) { maxv = v; break; }
        maxv = (maxv < v) ? v : maxv;
      }
      float denom = 0.0f;
      for (int64_t r = 0; r < reduce; ++r) denom += expf(x[base + r * inner] - maxv);
      for (int64_t r = 0; r < reduce; ++r) {
        const int64_t idx = base + r * inner;
        out[idx] = expf(x[idx] - maxv) / denom;
      }
    }
  }
}

/* rmsnorm: compute_rmsnorm, cpu_backend.cpp:157-183. */
void tcxo_rmsnorm(const float* x, float* out, int64_t outer, int64_t reduce, int64_t inner,
                  float epsilon) {
  for (int64_t o = 0; o < outer; ++o) {
    for (int64_t in = 0; in < inner; ++in) {
      const int64_t base = o * reduce * inner + in;
      float ss = 0.0f;
      for (int64_t r = 0; r < reduce; ++r) {
        const float v = x[base + r * inner];
        ss += v * v;
      }
      const float scale = 1.0f / sqrtf((ss / (float)reduce) + epsilon);
      for (int64_t r = 0; r < reduce; ++r) {
        const int64_t idx = base + r * inner;
        out[idx] = x[idx] * scale;
      }
    }
  }
}

/* layernorm: compute_layernorm, cpu_backend.cpp:185-240, including the constant
 * finite row (0, or NaN when epsilon is 0) and zero-denominator (NaN) cases. */
void tcxo_layernorm(const float* x, float* out, int64_t outer, int64_t reduce, int64_t inner,
                    float epsilon) {
  for (int64_t o = 0; o < outer; ++o) {
    for (int64_t in = 0; in < inner; ++in) {
      const int64_t base = o * reduce * inner + in;
      float sum = 0.0f;
      const float first = x[base];
      int all_equal = 1;
      for (int64_t r = 0; r < reduce; ++r) {
        const float v = x[base + r * inner];
        sum += v;
        all_equal = all_equal && v == first;
      }
      if (all_equal && isfinite(first)) {
        const float value = epsilon == 0.0f ? NAN : 0.0f;
        for (int64_t r = 0; r < reduce; ++r) out[base + r * inner] = value;
        continue;
      }
      const float mean = sum / (float)reduce;
      float ssd = 0.0f;
      for (int64_t r = 0; r < reduce; ++r) {
        const float d = x[base + r * inner] - mean;
        ssd += d * d;
      }
      const float variance = ssd / (float)reduce;
      const float denom = variance + epsilon;
      if (denom == 0.0f) {
        for (int64_t r = 0; r < reduce; ++r) out[base + r * inner] = NAN;
        continue;
      }
      const float scale = 1.0f / sqrtf(denom);
      for (int64_t r = 0; r < reduce; ++r) {
        const int64_t idx = base + r * inner;
        out[idx] = (x[idx] - mean) * scale;
      }
    }
  }
}

/* exp / gelu(tanh) / silu: cpu::execute_unary, cpu_backend.cpp:990-1010.
 * op: 0 exp, 1 gelu, 2 silu. */
void tcxo_unary(int op, const float* x, float* out, int64_t count) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f; /* cpu_backend.cpp:27-28 */
  for (int64_t i = 0; i < count; ++i) {
    const float v = x[i];
    if (op == 0) {
      out[i] = expf(v);
    } else if (op == 1) {
      const float inner = k0 * (v + k1 * v * v * v);
      out[i] = 0.5f * v * (1.0f + tanhf(inner));
    } else {
      out[i] = v / (1.0f + expf(-v));
    }
  }
}

/* Broadcast binary arithmetic: cpu::execute_binary, cpu_backend.cpp:1014-1097.
 * op: 0 add, 1 subtract, 2 multiply, 3 divide; meta = output shape, lhs strides,
 * rhs strides (zero for broadcast axes). int32 wraps through uint32. */
void tcxo_binary(int op, int dtype, const void* a, const void* b, void* out, int64_t count,
                 const int64_t* meta, int64_t rank) {
  for (int64_t i = 0; i < count; ++i) {
    int64_t idx = i, l = 0, r = 0;
    for (int64_t axis = rank; axis > 0; --axis) {
      const int64_t c = idx % meta[axis - 1];
      idx /= meta[axis - 1];
      l += c * meta[rank + axis - 1];
      r += c * meta[2 * rank + axis - 1];
    }
    if (dtype == 0) {
      const float x = ((const float*)a)[l], y = ((const float*)b)[r];
      float v = 0.0f;
      switch (op) {
        case 0: v = x + y; break;
        case 1: v = x - y; break;
        case 2: v = x * y; break;
        default: v = x / y; break;
      }
      ((float*)out)[i] = v;
    } else {
      const uint32_t x = (uint32_t)((const int32_t*)a)[l], y = (uint32_t)((const int32_t*)b)[r];
      uint32_t v = 0;
      switch (op) {
        case 0: v = x + y; break;
        case 1: v = x - y; break;
        default: v = x * y; break;
      }
      ((int32_t*)out)[i] = (int32_t)v;
    }
  }
}

/* Rows [row_begin, row_end) of one batch of C = A·B, A [m,k], B [k,n] row-major:
 * cpu::matmul, cpu_backend.cpp:1264-1273 (float sum += a*b in k order). */
void tcxo_matmul_rows(const float* a, const float* b, float* out, int64_t m, int64_t n,
                      int64_t k, int64_t row_begin, int64_t row_end) {
  (void)m;
  for (int64_t row = row_begin; row < row_end; ++row) {
    for (int64_t col = 0; col < n; ++col) {
      float sum = 0.0f;
      for (int64_t inner = 0; inner < k; ++inner) sum += a[row * k + inner] * b[inner * n + col];
      out[(row - row_begin) * n + col] = sum;
    }
  }
}

/* Exact (float64) sum, used as a secondary accuracy reference for the
 * full-tensor float32 sum (not a reference function). */
/* Masked, scaled attention softmax over the target `shape` [..., queries, keys]:
 * execute_inference_primitive, cpu_inference.cpp:22-45 (plan: core/inference.cpp:56-83).
 * scores / mask are read through broadcast strides (sstr / mstr, element units);
 * mask_kind 0 none, 1 bool bytes, 2 float32. Output contiguous. */
static int64_t attn_offset(int64_t i, const int64_t* shape, const int64_t* strides, int rank) {
  int64_t off = 0;
  for (int a = rank - 1; a >= 0; --a) {
    off += (i % shape[a]) * strides[a];
    i /= shape[a];
  }
  return off;
}

static float attn_score(const float* scores, const void* mask, int mask_kind, const int64_t* shape,
                        const int64_t* sstr, const int64_t* mstr, int rank, int64_t i, int64_t col,
                        int64_t query, float scale, int causal) {
  if (causal && col > query) return -INFINITY;
  if (mask_kind == 1 && !((const unsigned char*)mask)[attn_offset(i, shape, mstr, rank)]) return -INFINITY;
  const float bias = mask_kind == 2 ? ((const float*)mask)[attn_offset(i, shape, mstr, rank)] : 0.0f;
  if (bias == -INFINITY) return bias;
  return scores[attn_offset(i, shape, sstr, rank)] * scale + bias;
}

void tcxo_attention_softmax(const float* scores, const void* mask, int mask_kind, float* out,
                            const int64_t* shape, const int64_t* sstr, const int64_t* mstr, int rank,
                            float scale, int causal) {
  int64_t count = 1;
  for (int a = 0; a < rank; ++a) count *= shape[a];
  const int64_t columns = shape[rank - 1];
  const int64_t rows = columns ? count / columns : 0;
  for (int64_t row = 0; row < rows; ++row) {
    const int64_t query = row % shape[rank - 2];
    float maximum = -INFINITY;
    for (int64_t col = 0; col < columns; ++col) {
      const float v = attn_score(scores, mask, mask_kind, shape, sstr, mstr, rank, row * columns + col, col,
                                 query, scale, causal);
      if (isnan(v)) { maximum = v; break; }
      maximum = (maximum < v) ? v : maximum;
    }
    if (maximum == -INFINITY) {
      for (int64_t col = 0; col < columns; ++col) out[row * columns + col] = 0.0f;
      continue;
    }
    float total = 0.0f;
    for (int64_t col = 0; col < columns; ++col)
      total += expf(attn_score(scores, mask, mask_kind, shape, sstr, mstr, rank, row * columns + col, col, query,
                               scale, causal) - maximum);
    for (int64_t col = 0; col < columns; ++col)
      out[row * columns + col] = expf(attn_score(scores, mask, mask_kind, shape, sstr, mstr, rank,
                                                 row * columns + col, col, query, scale, causal) - maximum) / total;
  }
}

double tcxo_sum_f64(const float* x, int64_t count) {
  double s = 0.0;
  for (int64_t i = 0; i < count; ++i) s += (double)x[i];
  return s;
}

/* word helpers exported for the Python side's self-checks */
uint32_t tcxo_float_bits(float f) { return fbits(f); }
float tcxo_bits_float(uint32_t w) { return bitsf(w); }

/* ------------------------------------------------------------------ generation
 * Checker of tcx_sm100_random (no reference counterpart: tensor.cx draws randn on the
 * host with NumPy, python/tensorcx/tensor.py:485-497). Restates the published
 * Philox4x32-10 (Salmon et al., SC'11) and the generator's value mapping; the Philox
 * words, the uniform values and the Box-Muller angle are bit-exact, the normal values
 * use double precision logarithm / square root / sine / cosine (the device uses float32
 * ones and the SFU's sine and cosine, so they agree within a few 1e-6, not bit for
 * bit). Pinned by known answers in
 * tests/test_oracle.py: Philox4x32-10 of a zero counter and key, and the C++26
 * std::philox4x32 requirement that its 10000th output after default seeding (key
 * 20111115) is 1955073260. */
void tcxo_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
  uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3], k0 = key[0], k1 = key[1];
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0, n1 = (uint32_t)p1;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1, n3 = (uint32_t)p0;
    c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* Elements [offset, offset + count) of the stream of `seed`: dist 0 normal (mean a,
 * std b), 1 uniform [a, b). */
void tcxo_random(int dist, float* out, int64_t count, uint64_t seed, uint64_t offset, float a, float b) {
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  const float inv24 = 5.9604644775390625e-08f;
  for (int64_t i = 0; i < count; ++i) {
    const uint64_t e = offset + (uint64_t)i, blk = e >> 2;
    const uint32_t ctr[4] = {(uint32_t)blk, (uint32_t)(blk >> 32), 0u, 0u};
    uint32_t w[4];
    tcxo_philox4x32_10(ctr, key, w);
    const int lane = (int)(e & 3);
    if (dist == 1) {
      const float u = (float)(w[lane] >> 8) * inv24;
      out[i] = fmaf(b - a, u, a);
    } else {
      const int p = lane >> 1;
      const float u1 = (float)((w[2 * p] >> 8) + 1u) * inv24, u2 = (float)(w[2 * p + 1] >> 8) * inv24;
      const double r = sqrt(-2.0 * log((double)u1));
      const double t = (double)fmaf(u2, 6.28318530717958647692f, -3.14159265358979323846f);
      const float z = (float)((lane & 1) ? r * sin(t) : r * cos(t));
      out[i] = fmaf(b, z, a);
    }
  }
}
