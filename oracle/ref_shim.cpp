// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// C-ABI shim over the reference's own CPU backend (tensor.cx), compiled from the
// reference sources where they lie (oracle/Makefile) into oracle/_ref/libtcx_ref.so.
// It lets the tests, the golden-vector generator and bench.py's reference arm call
// the unmodified upstream `CpuBackend::execute` (cpp/tensorcx/backends/cpu/
// cpu_backend.cpp:246-366) and `cpu::execute_math` (cpu_math.cpp:27-76) with plain
// host pointers. Every entry returns 0 on success, 1 for kInvalidArgument, 2 for
// kUnavailable and 3 for kInternal, mirroring tensorcx::StatusCode
// (cpp/tensorcx/core/status.h:8-13). The message of the last failure on the
// calling thread is available from tcxref_last_error().
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "tensorcx/backends/cpu/cpu_backend.h"
#include "tensorcx/core/backend.h"

namespace {
using namespace tensorcx;
thread_local std::string g_error;

Shape shape_of(const std::int64_t* dims, int rank) {
  return Shape(dims, dims + rank);
}

Tensor make_tensor(int dtype, const void* data, const std::int64_t* dims, int rank) {
  Shape shape = shape_of(dims, rank);
  const auto n = static_cast<std::size_t>(numel(shape));
  if (dtype == 0) {
    std::vector<float> v(n);
    if (n) std::memcpy(v.data(), data, n * 4);
    return cpu::to_core_tensor(cpu::CpuTensor(shape, std::move(v)));
  }
  if (dtype == 2) {  // bool, one byte per element
    std::vector<std::uint8_t> v(n);
    if (n) std::memcpy(v.data(), data, n);
    return cpu::to_core_tensor(cpu::CpuTensor(shape, std::move(v)));
  }
  std::vector<std::int32_t> v(n);
  if (n) std::memcpy(v.data(), data, n * 4);
  return cpu::to_core_tensor(cpu::CpuTensor(shape, std::move(v)));
}

int finish(const Status& status, const Tensor& out, void* dst, std::int64_t capacity,
           std::int64_t* out_shape, int* out_rank) {
  if (!status.ok()) {
    g_error = status.message();
    return static_cast<int>(status.code());
  }
  const auto host = cpu::from_core_tensor(out);
  if (host.size() > capacity) {
    g_error = "output capacity too small";
    return 3;
  }
  if (out_rank) {
    *out_rank = static_cast<int>(host.shape().size());
    for (std::size_t i = 0; i < host.shape().size() && i < 64; ++i) out_shape[i] = host.shape()[i];
  }
  if (host.size()) std::memcpy(dst, host.data(), static_cast<std::size_t>(host.size()) * 4);
  return 0;
}

template <typename F>
int guarded(F&& body) {
  try {
    return body();
  } catch (const std::invalid_argument& e) {
    g_error = e.what();
    return 1;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 3;
  }
}

int run(OpDesc op, std::vector<Tensor> inputs, void* dst, std::int64_t capacity,
        std::int64_t* out_shape, int* out_rank) {
  cpu::CpuBackend backend;
  std::vector<Tensor> outputs(1);
  BackendExecution e{BackendOpClass::kPrimitive, op, inputs, outputs, std::nullopt, std::nullopt, {}};
  const Status status = backend.execute(e);
  return finish(status, outputs[0], dst, capacity, out_shape, out_rank);
}
}  // namespace

extern "C" {

const char* tcxref_last_error() { return g_error.c_str(); }

// OpKind values follow tensorcx::OpKind (cpp/tensorcx/core/operation.h:12-63).
// Generic single-input primitive: reductions (axis or axes), unary, softmax, norms,
// min/argmax. naxes < 0 selects the original single-axis path (op.axis).
int tcxref_unary_op(int kind, int dtype, const void* x, const std::int64_t* dims, int rank,
                    std::int64_t axis, int naxes, const std::int64_t* axes, double epsilon,
                    void* out, std::int64_t capacity, std::int64_t* out_shape, int* out_rank) {
  return guarded([&] {
    OpDesc op{static_cast<OpKind>(kind)};
    op.axis = axis;
    op.epsilon = epsilon;
    if (naxes >= 0) op.reduction_axes = Shape(axes, axes + naxes);
    return run(op, {make_tensor(dtype, x, dims, rank)}, out, capacity, out_shape, out_rank);
  });
}

// Two-input primitive: add/subtract/multiply/divide with broadcasting, matmul.
int tcxref_binary_op(int kind, int dtype, const void* a, const std::int64_t* adims, int arank,
                     const void* b, const std::int64_t* bdims, int brank, void* out,
                     std::int64_t capacity, std::int64_t* out_shape, int* out_rank) {
  return guarded([&] {
    OpDesc op{static_cast<OpKind>(kind)};
    return run(op, {make_tensor(dtype, a, adims, arank), make_tensor(dtype, b, bdims, brank)},
               out, capacity, out_shape, out_rank);
  });
}

// clip(x, lower, upper) with broadcast bounds (cpu_math.cpp:42-47).
int tcxref_clip(int dtype, const void* x, const std::int64_t* xd, int xr, const void* lo,
                const std::int64_t* lod, int lor, const void* hi, const std::int64_t* hid,
                int hir, void* out, std::int64_t capacity, std::int64_t* out_shape,
                int* out_rank) {
  return guarded([&] {
    OpDesc op{OpKind::kClip};
    return run(op, {make_tensor(dtype, x, xd, xr), make_tensor(dtype, lo, lod, lor),
                    make_tensor(dtype, hi, hid, hir)},
               out, capacity, out_shape, out_rank);
  });
}

// Affine normalization composite (cpp/tensorcx/core/inference.cpp:103-122).
int tcxref_affine_norm(int rms, const float* x, const std::int64_t* dims, int rank,
                       std::int64_t axis, double epsilon, const float* weight,
                       const float* bias, float* out, std::int64_t capacity) {
  return guarded([&] {
    OpDesc op{rms ? OpKind::kAffineRmsNorm : OpKind::kAffineLayerNorm};
    op.axis = axis;
    op.epsilon = epsilon;
    op.has_weight = weight != nullptr;
    op.has_bias = bias != nullptr;
    std::vector<Tensor> inputs{make_tensor(0, x, dims, rank)};
    std::int64_t n = rank ? dims[(axis < 0 ? axis + rank : axis)] : 1;
    std::int64_t pdims[1] = {n};
    if (weight) inputs.push_back(make_tensor(0, weight, pdims, rank ? 1 : 0));
    if (bias) inputs.push_back(make_tensor(0, bias, pdims, rank ? 1 : 0));
    return run(op, inputs, out, capacity, nullptr, nullptr);
  });
}

// linear(x, w, b) composite (cpp/tensorcx/core/inference.cpp:89-102).
int tcxref_linear(const float* x, const std::int64_t* xd, int xr, const float* w,
                  const std::int64_t* wd, const float* bias, float* out,
                  std::int64_t capacity) {
  return guarded([&] {
    OpDesc op{OpKind::kLinear};
    std::vector<Tensor> inputs{make_tensor(0, x, xd, xr), make_tensor(0, w, wd, 2)};
    std::int64_t bd[1] = {wd[0]};
    if (bias) inputs.push_back(make_tensor(0, bias, bd, 1));
    return run(op, inputs, out, capacity, nullptr, nullptr);
  });
}

// Attention composite (cpp/tensorcx/core/inference.cpp:123-160): query, key, value and
// an optional mask (mask_kind 0 none, 1 bool, 2 float32).
// has_scale = 0 uses the default 1/sqrt(features).
int tcxref_attention(const float* q, const std::int64_t* qd, int qr, const float* k, const std::int64_t* kd,
                     int kr, const float* v, const std::int64_t* vd, int vr, const void* mask,
                     int mask_kind, const std::int64_t* md, int mr, int causal, int has_scale, double scale,
                     float* out, std::int64_t capacity, std::int64_t* out_shape, int* out_rank) {
  return guarded([&] {
    OpDesc op{OpKind::kAttention};
    op.causal = causal != 0;
    if (has_scale) op.attention_scale = scale;
    std::vector<Tensor> inputs{make_tensor(0, q, qd, qr), make_tensor(0, k, kd, kr), make_tensor(0, v, vd, vr)};
    if (mask_kind == 1) inputs.push_back(make_tensor(2, mask, md, mr));
    if (mask_kind == 2) inputs.push_back(make_tensor(0, mask, md, mr));
    return run(op, inputs, out, capacity, out_shape, out_rank);
  });
}

// Attention softmax primitive (kAttentionSoftmax, cpu_inference.cpp:22-45) of scores
// broadcast to the target shape td, with an optional mask (mask_kind 1 bool, 2 float).
int tcxref_attention_softmax(const float* scores, const std::int64_t* sd, int sr, const void* mask,
                             int mask_kind, const std::int64_t* md, int mr, const std::int64_t* td, int tr,
                             int causal, double scale, float* out, std::int64_t capacity) {
  return guarded([&] {
    OpDesc op{OpKind::kAttentionSoftmax};
    op.causal = causal != 0;
    op.attention_scale = scale;
    op.attention_shape = Shape(td, td + tr);
    std::vector<Tensor> inputs{make_tensor(0, scores, sd, sr)};
    if (mask_kind == 1) inputs.push_back(make_tensor(2, mask, md, mr));
    if (mask_kind == 2) inputs.push_back(make_tensor(0, mask, md, mr));
    return run(op, inputs, out, capacity, nullptr, nullptr);
  });
}

// The right operand of the row-sliced CPU baseline, copied into a CpuTensor once
// (tcxref_matmul_bind_rhs, outside any timed region) and shared read-only by every
// thread's tcxref_matmul_rows call on the same B. Without it each call copies the
// whole of B (256 MiB at 8192^3) next to a few rows of arithmetic.
struct BoundRhs {
  const float* src = nullptr;
  std::int64_t k = 0, n = 0;
  std::shared_ptr<const cpu::CpuTensor> tensor;
};
std::mutex g_rhs_mu;
BoundRhs g_rhs;

int tcxref_matmul_bind_rhs(const float* b, std::int64_t k, std::int64_t n) {
  return guarded([&] {
    auto t = std::make_shared<const cpu::CpuTensor>(Shape{k, n}, std::vector<float>(b, b + k * n));
    std::lock_guard<std::mutex> lock(g_rhs_mu);
    g_rhs = BoundRhs{b, k, n, std::move(t)};
    return 0;
  });
}

// Row-slice matmul for the timed CPU baseline: cpu::matmul over rows
// [row_begin, row_end) of a 2-D lhs, which performs exactly the per-element
// arithmetic of the full product (cpu_backend.cpp:1251-1276). B comes from the bound
// copy when it is the bound operand, else it is copied for this call.
int tcxref_matmul_rows(const float* a, const float* b, float* out, std::int64_t m,
                       std::int64_t k, std::int64_t n, std::int64_t row_begin,
                       std::int64_t row_end) {
  return guarded([&] {
    const std::int64_t rows = row_end - row_begin;
    if (rows < 0 || row_end > m) { g_error = "bad row range"; return 1; }
    std::vector<float> slice(static_cast<std::size_t>(rows * k));
    if (rows * k) std::memcpy(slice.data(), a + row_begin * k, static_cast<std::size_t>(rows * k) * 4);
    std::shared_ptr<const cpu::CpuTensor> rhs_t;
    {
      std::lock_guard<std::mutex> lock(g_rhs_mu);
      if (g_rhs.src == b && g_rhs.k == k && g_rhs.n == n) rhs_t = g_rhs.tensor;
    }
    if (!rhs_t) rhs_t = std::make_shared<const cpu::CpuTensor>(Shape{k, n}, std::vector<float>(b, b + k * n));
    const cpu::CpuTensor lhs_t(Shape{rows, k}, std::move(slice));
    const auto result = cpu::matmul(lhs_t, *rhs_t);
    if (result.size()) std::memcpy(out, result.data(), static_cast<std::size_t>(result.size()) * 4);
    return 0;
  });
}

}  // extern "C"
