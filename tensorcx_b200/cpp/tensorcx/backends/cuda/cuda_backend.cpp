// CudaBackend::execute for the sm100 backend: validation and planning with the
// unchanged tensor.cx core (validate_primitive_execution_contract, make_*_plan), then
// one C-ABI call per primitive (include/tcx_sm100.h) on the calling thread's stream for
// the device, a synchronize of that stream (the ABI stays synchronous, docs/BACKENDS.md:178-180)
// and publication of the result slot only on success (cuda_backend.cpp:612-613 of the
// reference). Validation messages follow the reference CUDA backend so the bindings
// raise the same errors.
#include "tensorcx/backends/cuda/cuda_backend.h"

#include <cuda_runtime_api.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <numeric>
#include <stdexcept>
#include <string>
#include <vector>

#include "tcx_sm100.h"
#include "tensorcx/backends/cuda/cuda_context.h"
#include "tensorcx/backends/cuda/cuda_device.h"
#include "tensorcx/backends/cuda/cuda_external_storage.h"
#include "tensorcx/backends/cuda/cuda_kernel.h"
#include "tensorcx/backends/cuda/cuda_memory_pool.h"
#include "tensorcx/backends/cuda/cuda_profile.h"
#include "tensorcx/core/inference.h"
#include "tensorcx/core/math.h"
#include "tensorcx/core/predicate.h"
#include "tensorcx/core/shape.h"

namespace tensorcx::cuda {
namespace {

Status invalid(std::string message) { return {StatusCode::kInvalidArgument, std::move(message)}; }

Status abi_status(int rc, const char* what) {
  if (rc == TCX_OK) return Status::Ok();
  const auto code = rc == TCX_INVALID_ARGUMENT ? StatusCode::kInvalidArgument
                    : rc == TCX_UNAVAILABLE   ? StatusCode::kUnavailable
                                              : StatusCode::kInternal;
  return Status(code, std::string(what) + ": " + tcx_sm100_last_error());
}

Expected<std::size_t> byte_size(DType dtype, const Shape& shape) {
  if (dtype != DType::kFloat32 && dtype != DType::kInt32 && dtype != DType::kBool)
    return invalid("unsupported CUDA dtype");
  const auto count = static_cast<std::uint64_t>(numel(shape));
  if (count > std::numeric_limits<std::size_t>::max() / dtype_size(dtype)) return invalid("CUDA buffer size overflow");
  return static_cast<std::size_t>(count) * dtype_size(dtype);
}

tcx_stream_t abi_stream(const DeviceScope& scope) { return reinterpret_cast<tcx_stream_t>(scope.stream()); }

// Stream-ordered scratch for one call: from the thread's pool when one is entered,
// otherwise from the device's default stream-ordered pool. Released (stream-ordered)
// when the call's work is queued, so no explicit wait is needed.
class Scratch {
 public:
  Scratch(std::size_t bytes, const DeviceScope& scope) : bytes_(bytes), stream_(scope.stream()) {
    if (!bytes_) return;
    const std::size_t padded = bytes_ + 1024;
    pool_ = active_memory_pool();
    if (pool_) {
      auto p = pool_->allocate(padded);
      if (!p) { status_ = p.status(); return; }
      raw_ = p.value();
    } else {
      status_ = runtime_status(cudaMallocAsync(&raw_, padded, stream_), "CUDA workspace allocation");
      if (!status_.ok()) return;
    }
    aligned_ = reinterpret_cast<void*>((reinterpret_cast<std::uintptr_t>(raw_) + 1023) & ~std::uintptr_t(1023));
  }
  ~Scratch() {
    if (!raw_) return;
    if (pool_) pool_->release(raw_, bytes_ + 1024, true);
    else (void)cudaFreeAsync(raw_, stream_);
  }
  Scratch(const Scratch&) = delete;
  Scratch& operator=(const Scratch&) = delete;
  const Status& status() const { return status_; }
  void* data() const { return aligned_; }
  std::size_t bytes() const { return bytes_; }

 private:
  std::size_t bytes_;
  cudaStream_t stream_;
  std::shared_ptr<MemoryPool> pool_;
  void* raw_{nullptr};
  void* aligned_{nullptr};
  Status status_;
};

struct Axis {
  Shape reduced_shape;
  std::int64_t outer{1}, reduce{1}, inner{1};
};

// One-axis view (cpu_backend.cpp:76-123 and cuda_backend.cpp:520-534 of the reference).
Expected<Axis> axis_view(const Tensor& t, std::int64_t axis) {
  Axis a;
  const auto rank = static_cast<std::int64_t>(t.shape.size());
  if (!rank) {
    if (axis != 0 && axis != -1) return invalid("reduction axis is out of range");
    return a;
  }
  if (axis < 0) axis += rank;
  if (axis < 0 || axis >= rank) return invalid("reduction axis is out of range");
  a.outer = numel(Shape(t.shape.begin(), t.shape.begin() + axis));
  a.inner = t.strides[axis];
  a.reduce = t.shape[axis];
  a.reduced_shape = t.shape;
  a.reduced_shape.erase(a.reduced_shape.begin() + axis);
  return a;
}

Expected<float> checked_epsilon(double eps) {
  if (!std::isfinite(eps) || eps < 0 || eps > std::numeric_limits<float>::max() ||
      (eps > 0 && static_cast<float>(eps) == 0))
    return invalid("epsilon must be finite and non-negative and representable as float32");
  return static_cast<float>(eps);
}

bool is_binary(OpKind k) {
  return k == OpKind::kAdd || k == OpKind::kSubtract || k == OpKind::kMultiply || k == OpKind::kDivide;
}

bool is_scalar_map(OpKind k) {
  return k == OpKind::kNegate || k == OpKind::kAddScalar || k == OpKind::kSubtractScalar ||
         k == OpKind::kMultiplyScalar || k == OpKind::kDivideScalar;
}

int abi_dtype(DType d) { return d == DType::kFloat32 ? TCX_FLOAT32 : d == DType::kInt32 ? TCX_INT32 : TCX_BOOL; }

class Executor {
 public:
  Executor(const BackendExecution& e, std::vector<CudaTensor>& in, const DeviceScope& scope)
      : e_(e), in_(in), scope_(scope) {}

  // `second` receives topk's indices (the op's second output); other ops leave it.
  Status run(Tensor& out, Tensor& second) {
    const auto kind = e_.op.kind;
    if (kind == OpKind::kFill) return fill(out);
    if (is_scalar_map(kind)) return scalar_map(out);
    if (kind == OpKind::kLog || kind == OpKind::kSqrt || kind == OpKind::kAbs) return unary_math(out);
    if (kind == OpKind::kTopK) return topk(out, second);
    if (kind == OpKind::kCast) return cast(out);
    if (kind == OpKind::kTranspose || kind == OpKind::kSlice) return index_copy(out);
    if (kind == OpKind::kConcat) return concat(out);
    if (is_predicate_elementwise(kind)) return predicate(out);
    if (kind == OpKind::kAny || kind == OpKind::kAll) return bool_reduce(out);
    if (kind == OpKind::kMaskedSelect) return masked_select(out);
    if (kind == OpKind::kEmbedding) return embedding(out);
    if (kind == OpKind::kMatmul) return matmul(out);
    if (kind == OpKind::kLinear) return linear(out);
    if (kind == OpKind::kSum || kind == OpKind::kMax || kind == OpKind::kMean) return reduction(out);
    if (kind == OpKind::kSoftmax || kind == OpKind::kRmsNorm || kind == OpKind::kLayerNorm) return row_op(out);
    if (kind == OpKind::kAffineRmsNorm || kind == OpKind::kAffineLayerNorm) return affine_norm(out);
    if (kind == OpKind::kExp || kind == OpKind::kGelu || kind == OpKind::kSilu) return unary(out);
    if (is_binary(kind)) return binary(out);
    if (kind == OpKind::kMin || kind == OpKind::kArgmax || kind == OpKind::kClip) return math(out);
    if (kind == OpKind::kAttentionSoftmax) return attention_softmax(out);
    if (kind == OpKind::kAttention) return attention(out);
    return {StatusCode::kUnavailable, "unsupported CUDA operation"};
  }

 private:
  const BackendExecution& e_;
  std::vector<CudaTensor>& in_;
  const DeviceScope& scope_;

  void* ptr(std::size_t i) const { return in_[i].buffer()->data(); }

  // One C-ABI call inside the profiler's compute span and device interval named `name`
  // (the reference's launch_* names); its completion wait happens inside the span.
  template <typename Call>
  Status launch(const char* name, const char* what, Call&& call) {
    ProfiledLaunch profiled(name, scope_.stream());
    return profiled.complete(abi_status(call(), what));
  }

  Expected<std::shared_ptr<CudaBuffer>> output(DType dtype, const Shape& shape) {
    return CudaBuffer::create(dtype, shape, scope_.device());
  }

  Status publish(Tensor& out, DType dtype, const Shape& shape, std::shared_ptr<CudaBuffer> buffer) {
    out = to_core_tensor(CudaTensor(dtype, shape, std::move(buffer)));
    return Status::Ok();
  }

  Status require_float32() {
    for (const auto& t : in_)
      if (t.dtype() != DType::kFloat32) return invalid("CUDA operation only supports float32 for this dtype");
    return Status::Ok();
  }

  Status fill(Tensor& out) {
    const auto& desc = e_.outputs[0];
    auto buffer = output(desc.dtype, desc.shape);
    if (!buffer) return buffer.status();
    const auto count = numel(desc.shape);
    if (count) {
      if (desc.dtype == DType::kBool) {
        ProfileScope span(ProfileCategory::kMemset, "cudaMemsetAsync", "cuda", buffer.value()->nbytes());
        auto st = runtime_status(cudaMemsetAsync(buffer.value()->data(), e_.op.scalar_value != 0,
                                                 buffer.value()->nbytes(), scope_.stream()),
                                 "CUDA bool fill");
        if (!st.ok()) return st;
      } else {
        std::uint32_t bits;
        if (desc.dtype == DType::kInt32) {
          if (!is_int32_representable(e_.op.scalar_value))
            return invalid("fill/arithmetic scalar must be an integer in int32 range");
          const auto v = static_cast<std::int32_t>(e_.op.scalar_value);
          std::memcpy(&bits, &v, 4);
        } else {
          const auto v = static_cast<float>(e_.op.scalar_value);
          std::memcpy(&bits, &v, 4);
        }
        auto st = launch("launch_fill", "CUDA fill", [&] {
          return tcx_sm100_fill(abi_stream(scope_), buffer.value()->data(), count, bits); });
        if (!st.ok()) return st;
      }
    }
    return publish(out, desc.dtype, desc.shape, buffer.move_value());
  }

  Status matmul(Tensor& out) {
    if (e_.op.matmul_preference != MatmulPreference::kAuto && e_.op.matmul_preference != MatmulPreference::kCustom)
      return invalid("CUDA matmul supports auto or custom");
    if (auto st = require_float32(); !st.ok()) return st;
    const auto plan = make_matmul_plan(in_[0].shape(), in_[1].shape());
    auto buffer = output(DType::kFloat32, plan.output_shape);
    if (!buffer) return buffer.status();
    const auto count = numel(plan.output_shape);
    if (count) {
      const auto batches = count / plan.n / plan.m;
      const auto nba = plan.m * plan.k != 0 ? numel(in_[0].shape()) / (plan.m * plan.k) : 1;
      const auto nbb = plan.k * plan.n != 0 ? numel(in_[1].shape()) / (plan.k * plan.n) : 1;
      Scratch ws(tcx_sm100_matmul_workspace_bytes(plan.m, plan.n, plan.k, nba, nbb, TCX_MATMUL_AUTO), scope_);
      if (!ws.status().ok()) return ws.status();
      auto st = launch("launch_matmul", "CUDA matmul", [&] {
        return tcx_sm100_matmul(abi_stream(scope_), static_cast<const float*>(ptr(0)), static_cast<const float*>(ptr(1)),
                           static_cast<float*>(buffer.value()->data()), plan.m, plan.n, plan.k, batches,
                           plan.batch_shape.data(), plan.lhs_batch_strides.data(), plan.rhs_batch_strides.data(),
                           static_cast<std::int32_t>(plan.batch_shape.size()), nullptr, TCX_ACT_NONE,
                           TCX_MATMUL_AUTO, ws.data(), ws.bytes()); });
      if (!st.ok()) return st;
    }
    return publish(out, DType::kFloat32, plan.output_shape, buffer.move_value());
  }

  // kLinear (core/inference.cpp:89-102) in one GEMM: weight read in place, bias fused.
  Status linear(Tensor& out) {
    if (in_.size() < 2 || in_.size() > 3) return invalid("linear requires input, weight and optional bias");
    for (const auto& t : in_)
      if (t.dtype() != DType::kFloat32) return invalid("inference values require float32 tensors");
    const auto& x = in_[0].shape();
    const auto& w = in_[1].shape();
    if (x.empty() || w.size() != 2 || x.back() != w[1])
      return invalid("linear requires (..., in_features) and (out_features, in_features)");
    if (in_.size() == 3 && in_[2].shape() != Shape{w[0]}) return invalid("linear bias must have shape (out_features,)");
    Shape shape = x;
    shape.back() = w[0];
    (void)numel(shape);
    auto buffer = output(DType::kFloat32, shape);
    if (!buffer) return buffer.status();
    const auto rows = numel(Shape(x.begin(), x.end() - 1));
    if (numel(shape)) {
      Scratch ws(tcx_sm100_linear_workspace_bytes(rows, w[1], w[0], TCX_MATMUL_AUTO), scope_);
      if (!ws.status().ok()) return ws.status();
      auto st = launch("launch_matmul", "CUDA linear", [&] {
        return tcx_sm100_linear(abi_stream(scope_), static_cast<const float*>(ptr(0)),
                                            static_cast<const float*>(ptr(1)),
                                            in_.size() == 3 ? static_cast<const float*>(ptr(2)) : nullptr,
                                            static_cast<float*>(buffer.value()->data()), rows, w[1], w[0],
                                            TCX_ACT_NONE, TCX_MATMUL_AUTO, ws.data(), ws.bytes()); });
      if (!st.ok()) return st;
    }
    return publish(out, DType::kFloat32, shape, buffer.move_value());
  }

  // kAttentionSoftmax (plan core/inference.cpp:56-83): one masked-softmax kernel reading
  // the scores and mask through the plan's broadcast strides.
  Status attention_softmax(Tensor& out) {
    const auto plan = make_attention_softmax_plan(e_.op, e_.inputs);
    auto buffer = output(DType::kFloat32, plan.shape);
    if (!buffer) return buffer.status();
    const auto rank = plan.shape.size();
    if (numel(plan.shape)) {
      auto st = launch("launch_attention_softmax", "CUDA attention softmax", [&] {
        return tcx_sm100_attention_softmax(abi_stream(scope_), static_cast<const float*>(ptr(0)),
                                      plan.mask_kind ? ptr(1) : nullptr, static_cast<std::int32_t>(plan.mask_kind),
                                      static_cast<float*>(buffer.value()->data()), plan.shape.data(),
                                      plan.metadata.data() + rank,
                                      plan.mask_kind ? plan.metadata.data() + 2 * rank : nullptr,
                                      static_cast<std::int32_t>(rank), plan.scale, e_.op.causal ? 1 : 0); });
      if (!st.ok()) return st;
    }
    return publish(out, DType::kFloat32, plan.shape, buffer.move_value());
  }

  // kAttention (core/inference.cpp:123-160) as one C-ABI call: the two GEMMs read the
  // keys K-major (no transpose launch) and the scores stay in stream-ordered scratch.
  Status attention(Tensor& out) {
    if (in_.size() < 3 || in_.size() > 4) return invalid("attention requires query, key, value and optional mask");
    for (std::size_t i = 0; i < 3; ++i) {
      if (in_[i].dtype() != DType::kFloat32) return invalid("inference values require float32 tensors");
      if (in_[i].shape().size() < 2) return invalid("attention tensors require rank >= 2");
    }
    const auto& q = in_[0].shape();
    const auto& k = in_[1].shape();
    const auto& v = in_[2].shape();
    const Dim features = q.back(), queries = q[q.size() - 2], keys = k[k.size() - 2];
    if (features <= 0 || features != k.back() || keys != v[v.size() - 2])
      return invalid("attention query/key features and key/value sequence sizes must match; features must be positive");
    Shape batch;
    for (const auto* s : {&q, &k, &v}) {
      const std::size_t own = s->size() - 2;
      const std::size_t rank = std::max(batch.size(), own);
      Shape merged(rank, 1);
      for (std::size_t a = 0; a < rank; ++a) {
        const Dim left = a < rank - batch.size() ? 1 : batch[a - (rank - batch.size())];
        const Dim right = a < rank - own ? 1 : (*s)[a - (rank - own)];
        if (left != right && left != 1 && right != 1) return invalid("attention batch dimensions cannot broadcast");
        merged[a] = left == 1 ? right : left;
      }
      batch = std::move(merged);
    }
    Shape scores = batch;
    scores.push_back(queries);
    scores.push_back(keys);
    Shape shape = batch;
    shape.push_back(queries);
    shape.push_back(v.back());
    (void)numel(scores), (void)contiguous_strides(scores), (void)numel(shape), (void)contiguous_strides(shape);
    const double requested = e_.op.attention_scale.value_or(1.0 / std::sqrt(static_cast<double>(features)));
    const float scale = static_cast<float>(requested);
    if (!std::isfinite(requested) || !std::isfinite(scale) || (requested != 0 && scale == 0))
      return invalid("attention scale must be finite and representable as float32");
    // mask dtype / broadcast checks of the softmax plan, before any allocation
    OpDesc softmax{OpKind::kAttentionSoftmax};
    softmax.attention_shape = scores;
    softmax.causal = e_.op.causal;
    softmax.attention_scale = scale;
    Tensor descriptor = e_.inputs[0];
    descriptor.shape = scores;
    descriptor.strides = contiguous_strides(scores);
    std::vector<Tensor> preview{descriptor};
    if (in_.size() == 4) preview.push_back(e_.inputs[3]);
    const auto plan = make_attention_softmax_plan(softmax, preview);
    auto buffer = output(DType::kFloat32, shape);
    if (!buffer) return buffer.status();
    if (!numel(shape)) return publish(out, DType::kFloat32, shape, buffer.move_value());
    const std::size_t rank = batch.size();
    auto batch_strides = [&](const Shape& s) {
      const auto own = contiguous_strides(s);
      const std::size_t r = s.size() - 2;
      Shape st(rank, 0);
      for (std::size_t a = rank - r; a < rank; ++a)
        if (s[a - (rank - r)] != 1) st[a] = own[a - (rank - r)];
      return st;
    };
    const Shape qs = batch_strides(q), ks = batch_strides(k), vs = batch_strides(v);
    const Dim nb = numel(batch);
    const Dim qn = numel(Shape(q.begin(), q.end() - 2)), kn = numel(Shape(k.begin(), k.end() - 2)),
              vn = numel(Shape(v.begin(), v.end() - 2));
    Scratch ws(tcx_sm100_attention_workspace_bytes(nb, queries, keys, features, v.back(), qn, kn, vn,
                                                   static_cast<std::int32_t>(plan.mask_kind)),
               scope_);
    if (!ws.status().ok()) return ws.status();
    const auto srank = scores.size();
    auto st = launch("launch_attention", "CUDA attention", [&] {
      return tcx_sm100_attention(abi_stream(scope_), static_cast<const float*>(ptr(0)), static_cast<const float*>(ptr(1)),
                            static_cast<const float*>(ptr(2)), plan.mask_kind ? ptr(3) : nullptr,
                            static_cast<std::int32_t>(plan.mask_kind), static_cast<float*>(buffer.value()->data()),
                            queries, keys, features, v.back(), batch.data(), qs.data(), ks.data(), vs.data(),
                            static_cast<std::int32_t>(rank),
                            plan.mask_kind ? plan.metadata.data() + 2 * srank : nullptr, scale,
                            e_.op.causal ? 1 : 0, ws.data(), ws.bytes()); });
    if (!st.ok()) return st;
    return publish(out, DType::kFloat32, shape, buffer.move_value());
  }

  Status reduction(Tensor& out) {
    const auto kind = e_.op.kind;
    const auto& t = e_.inputs[0];
    const auto dtype = t.dtype;
    if (dtype != DType::kFloat32 && !(dtype == DType::kInt32 && kind != OpKind::kMean))
      return invalid("CUDA operation only supports float32 for this dtype");
    const int code = static_cast<int>(kind);
    const int dt = dtype == DType::kFloat32 ? TCX_FLOAT32 : TCX_INT32;
    if (e_.op.reduction_axes) {
      const auto plan = make_reduction_plan(t.shape, *e_.op.reduction_axes);
      if (kind == OpKind::kMax && plan.reduction_size == 0) return invalid("max reduction requires non-empty axes");
      auto buffer = output(dtype, e_.op.reduction_axes->empty() ? t.shape : plan.output_shape);
      if (!buffer) return buffer.status();
      if (e_.op.reduction_axes->empty()) {  // no axes: an independent copy
        ProfileScope span(ProfileCategory::kCopy, "device_to_device", "cuda", in_[0].nbytes());
        auto st = runtime_status(cudaMemcpyAsync(buffer.value()->data(), ptr(0), in_[0].nbytes(),
                                                 cudaMemcpyDeviceToDevice, scope_.stream()),
                                 "CUDA copy");
        if (!st.ok()) return st;
        return publish(out, dtype, t.shape, buffer.move_value());
      }
      const auto groups = numel(plan.output_shape);
      if (groups) {
        Scratch ws(tcx_sm100_reduce_workspace_bytes(groups * plan.reduction_size), scope_);
        if (!ws.status().ok()) return ws.status();
        auto st = launch("launch_reduce_axes", "CUDA multi-axis reduction", [&] {
          return tcx_sm100_reduce_axes(abi_stream(scope_), code, dt, ptr(0), buffer.value()->data(), groups,
                                  plan.reduction_size, plan.index_metadata.data(),
                                  static_cast<std::int32_t>(plan.output_shape.size()),
                                  static_cast<std::int32_t>(t.shape.size()), ws.data(), ws.bytes()); });
        if (!st.ok()) return st;
      }
      return publish(out, dtype, plan.output_shape, buffer.move_value());
    }
    auto a = axis_view(t, e_.op.axis);
    if (!a) return a.status();
    if (kind == OpKind::kMax && !a.value().reduce) return invalid("max reduction requires a non-empty axis");
    auto buffer = output(dtype, a.value().reduced_shape);
    if (!buffer) return buffer.status();
    if (a.value().outer * a.value().inner != 0) {
      Scratch ws(tcx_sm100_axis_workspace_bytes(code, a.value().outer, a.value().reduce, a.value().inner), scope_);
      if (!ws.status().ok()) return ws.status();
      auto st = launch("launch_axis", "CUDA axis reduction", [&] {
        return tcx_sm100_axis(abi_stream(scope_), code, dt, ptr(0), buffer.value()->data(),
                                          a.value().outer, a.value().reduce, a.value().inner, 0.0f, ws.data(),
                                          ws.bytes()); });
      if (!st.ok()) return st;
    }
    return publish(out, dtype, a.value().reduced_shape, buffer.move_value());
  }

  Status row_op(Tensor& out) {
    if (auto st = require_float32(); !st.ok()) return st;
    const auto& t = e_.inputs[0];
    auto a = axis_view(t, e_.op.axis);
    if (!a) return a.status();
    float eps = 0.0f;
    if (e_.op.kind != OpKind::kSoftmax) {
      auto e = checked_epsilon(e_.op.epsilon);
      if (!e) return e.status();
      eps = e.value();
    }
    auto buffer = output(DType::kFloat32, t.shape);
    if (!buffer) return buffer.status();
    if (numel(t.shape)) {
      auto st = launch("launch_axis", "CUDA row operation", [&] {
        return tcx_sm100_axis(abi_stream(scope_), static_cast<int>(e_.op.kind), TCX_FLOAT32, ptr(0),
                                          buffer.value()->data(), a.value().outer, a.value().reduce,
                                          a.value().inner, eps, nullptr, 0); });
      if (!st.ok()) return st;
    }
    return publish(out, DType::kFloat32, t.shape, buffer.move_value());
  }

  // kAffineRmsNorm / kAffineLayerNorm (core/inference.cpp:103-122) in one kernel.
  Status affine_norm(Tensor& out) {
    const auto& op = e_.op;
    if (e_.inputs.size() != 1U + op.has_weight + op.has_bias || (op.kind == OpKind::kAffineRmsNorm && op.has_bias))
      return invalid("invalid affine normalization parameters");
    for (const auto& t : in_)
      if (t.dtype() != DType::kFloat32) return invalid("inference values require float32 tensors");
    const auto& x = e_.inputs[0];
    auto a = axis_view(x, op.axis);
    if (!a) return invalid("normalization axis out of range");
    const Shape expected = x.shape.empty() ? Shape{} : Shape{a.value().reduce};
    for (std::size_t i = 1; i < e_.inputs.size(); ++i)
      if (e_.inputs[i].shape != expected) return invalid("affine parameters must match the normalized axis");
    auto eps = checked_epsilon(op.epsilon);
    if (!eps) return invalid("epsilon must be finite, non-negative and representable as float32");
    auto buffer = output(DType::kFloat32, x.shape);
    if (!buffer) return buffer.status();
    if (numel(x.shape)) {
      std::size_t next = 1;
      const float* w = op.has_weight ? static_cast<const float*>(ptr(next++)) : nullptr;
      const float* b = op.has_bias ? static_cast<const float*>(ptr(next)) : nullptr;
      auto st = launch("launch_axis", "CUDA affine normalization", [&] {
        return tcx_sm100_affine_norm(abi_stream(scope_), op.kind == OpKind::kAffineRmsNorm ? TCX_OP_RMSNORM : TCX_OP_LAYERNORM,
                                static_cast<const float*>(ptr(0)), static_cast<float*>(buffer.value()->data()),
                                a.value().outer, a.value().reduce, a.value().inner, eps.value(), w, b); });
      if (!st.ok()) return st;
    }
    return publish(out, DType::kFloat32, x.shape, buffer.move_value());
  }

  Status unary(Tensor& out) {
    if (auto st = require_float32(); !st.ok()) return st;
    const auto& t = e_.inputs[0];
    auto buffer = output(DType::kFloat32, t.shape);
    if (!buffer) return buffer.status();
    auto st = launch("launch_unary", "CUDA unary", [&] {
      return tcx_sm100_unary(abi_stream(scope_), static_cast<int>(e_.op.kind),
                                         static_cast<const float*>(ptr(0)),
                                         static_cast<float*>(buffer.value()->data()), numel(t.shape)); });
    if (!st.ok()) return st;
    return publish(out, DType::kFloat32, t.shape, buffer.move_value());
  }

  Status binary(Tensor& out) {
    const auto kind = e_.op.kind;
    const auto& l = e_.inputs[0];
    const auto& r = e_.inputs[1];
    if (l.dtype != r.dtype) return invalid("dtype mismatch for binary operation");
    if (l.dtype != DType::kFloat32 && !(l.dtype == DType::kInt32 && kind != OpKind::kDivide))
      return invalid("CUDA operation only supports float32 for this dtype");
    Shape shape = l.shape;
    Shape metadata;
    if (l.shape != r.shape) {
      const auto plan = make_broadcast_plan(l.shape, r.shape);
      shape = plan.output_shape;
      metadata = plan.output_shape;
      metadata.insert(metadata.end(), plan.lhs_strides.begin(), plan.lhs_strides.end());
      metadata.insert(metadata.end(), plan.rhs_strides.begin(), plan.rhs_strides.end());
    }
    auto buffer = output(l.dtype, shape);
    if (!buffer) return buffer.status();
    auto st = launch(metadata.empty() ? "launch_binary" : "launch_broadcast_binary", "CUDA binary", [&] {
      return tcx_sm100_binary(abi_stream(scope_), static_cast<int>(kind),
                                          l.dtype == DType::kFloat32 ? TCX_FLOAT32 : TCX_INT32, ptr(0), ptr(1),
                                          buffer.value()->data(), numel(shape),
                                          metadata.empty() ? nullptr : metadata.data(),
                                          metadata.empty() ? 0 : static_cast<std::int32_t>(shape.size())); });
    if (!st.ok()) return st;
    return publish(out, l.dtype, shape, buffer.move_value());
  }

  // min / argmax / clip through make_math_plan (core/math.cpp:13-71).
  Status math(Tensor& out) {
    const auto plan = make_math_plan(e_.op, e_.inputs);
    auto buffer = output(plan.dtype, plan.shape);
    if (!buffer) return buffer.status();
    const int dt = e_.inputs[0].dtype == DType::kFloat32 ? TCX_FLOAT32 : TCX_INT32;
    if (plan.groups) {
      Status st;
      if (e_.op.kind == OpKind::kClip) {
        st = launch("launch_math", "CUDA clip", [&] {
          return tcx_sm100_clip(abi_stream(scope_), dt, ptr(0), ptr(1), ptr(2), buffer.value()->data(),
                                       plan.groups, plan.metadata.data(), static_cast<std::int32_t>(plan.rank)); });
      } else {
        Scratch ws(tcx_sm100_reduce_workspace_bytes(plan.groups * plan.reduce), scope_);
        if (!ws.status().ok()) return ws.status();
        st = launch("launch_math", "CUDA min/argmax", [&] {
          return tcx_sm100_min_argmax(abi_stream(scope_), static_cast<int>(e_.op.kind), dt, ptr(0),
                                             buffer.value()->data(), plan.groups, plan.reduce,
                                             plan.metadata.data(), static_cast<std::int32_t>(plan.rank),
                                             ws.data(), ws.bytes()); });
      }
      if (!st.ok()) return st;
    }
    return publish(out, plan.dtype, plan.shape, buffer.move_value());
  }

  // The host reads a device int the previous launch wrote (cast range, embedding index).
  Expected<int> read_flag(const Scratch& flag) {
    int value = 0;
    ProfileScope span(ProfileCategory::kCopy, "device_to_host", "cuda", sizeof(int));
    auto st = runtime_status(cudaMemcpyAsync(&value, flag.data(), sizeof(int), cudaMemcpyDeviceToHost, scope_.stream()),
                             "CUDA flag readback");
    if (!st.ok()) return st;
    st = runtime_status(cudaStreamSynchronize(scope_.stream()), "CUDA flag readback");
    if (!st.ok()) return st;
    return value;
  }

  // negate and scalar arithmetic (cuda_backend.cpp:452-466 and 585-587 of the reference):
  // float32, or int32 except divide, with an integral int32 scalar.
  Status scalar_map(Tensor& out) {
    const auto kind = e_.op.kind;
    const auto& t = e_.inputs[0];
    const bool integer_ok = kind != OpKind::kDivideScalar;
    if (t.dtype != DType::kFloat32 && !(t.dtype == DType::kInt32 && integer_ok))
      return invalid("CUDA operation only supports float32 for this dtype");
    if (t.dtype == DType::kInt32 && kind != OpKind::kNegate && !is_int32_representable(e_.op.scalar_value))
      return invalid("fill/arithmetic scalar must be an integer in int32 range");
    auto buffer = output(t.dtype, t.shape);
    if (!buffer) return buffer.status();
    if (numel(t.shape)) {
      auto st = launch(kind == OpKind::kNegate ? "launch_unary" : "launch_scalar", "CUDA elementwise", [&] {
        return tcx_sm100_map(abi_stream(scope_), static_cast<int>(kind), abi_dtype(t.dtype), ptr(0),
                             buffer.value()->data(), numel(t.shape), e_.op.scalar_value, e_.op.scalar_left ? 1 : 0); });
      if (!st.ok()) return st;
    }
    return publish(out, t.dtype, t.shape, buffer.move_value());
  }

  // log / sqrt / abs through make_math_plan (codes 0-2).
  Status unary_math(Tensor& out) {
    const auto plan = make_math_plan(e_.op, e_.inputs);
    auto buffer = output(plan.dtype, plan.shape);
    if (!buffer) return buffer.status();
    if (plan.groups) {
      auto st = launch("launch_math", "CUDA math", [&] {
        return tcx_sm100_map(abi_stream(scope_), static_cast<int>(e_.op.kind), abi_dtype(plan.dtype), ptr(0),
                             buffer.value()->data(), plan.groups, 0.0, 0); });
      if (!st.ok()) return st;
    }
    return publish(out, plan.dtype, plan.shape, buffer.move_value());
  }

  // topk through make_math_plan (code 6): values and int32 indices.
  Status topk(Tensor& out, Tensor& indices_out) {
    const auto plan = make_math_plan(e_.op, e_.inputs);
    auto values = output(plan.dtype, plan.shape);
    if (!values) return values.status();
    auto indices = output(DType::kInt32, plan.shape);
    if (!indices) return indices.status();
    if (plan.groups) {
      auto st = launch("launch_math", "CUDA topk", [&] {
        return tcx_sm100_topk(abi_stream(scope_), abi_dtype(plan.dtype), ptr(0), values.value()->data(),
                              static_cast<std::int32_t*>(indices.value()->data()), plan.groups, plan.reduce, plan.inner,
                              plan.k, e_.op.largest ? 1 : 0, e_.op.sorted ? 1 : 0); });
      if (!st.ok()) return st;
    }
    indices_out = to_core_tensor(CudaTensor(DType::kInt32, plan.shape, indices.move_value()));
    return publish(out, plan.dtype, plan.shape, values.move_value());
  }

  // cast (cuda_backend.cpp:399-440 of the reference): float32 / int32 / bool; a
  // float32 -> int32 cast checks the range on the device and fails before publishing.
  Status cast(Tensor& out) {
    const auto& t = e_.inputs[0];
    const auto target = e_.op.target_dtype;
    if (target != DType::kFloat32 && target != DType::kInt32 && target != DType::kBool)
      return invalid("unsupported cast target dtype");
    auto buffer = output(target, t.shape);
    if (!buffer) return buffer.status();
    const auto count = numel(t.shape);
    if (count) {
      const bool checked = t.dtype == DType::kFloat32 && target == DType::kInt32;
      Scratch flag(checked ? sizeof(int) : 0, scope_);
      if (!flag.status().ok()) return flag.status();
      auto st = launch("launch_cast", "CUDA tensor cast", [&] {
        return tcx_sm100_cast(abi_stream(scope_), abi_dtype(t.dtype), abi_dtype(target), ptr(0), buffer.value()->data(),
                              count, checked ? static_cast<int*>(flag.data()) : nullptr); });
      if (!st.ok()) return st;
      if (checked) {
        auto bad = read_flag(flag);
        if (!bad) return bad.status();
        if (bad.value()) return invalid("float32 to int32 cast requires finite values in [-2147483648, 2147483648)");
      }
    }
    return publish(out, target, t.shape, buffer.move_value());
  }

  // transpose / slice (cuda_backend.cpp:342-375 of the reference): one index copy.
  Status index_copy(Tensor& out) {
    const auto& t = e_.inputs[0];
    const auto plan = e_.op.kind == OpKind::kTranspose
                          ? make_transpose_plan(t.shape, e_.op.axes)
                          : make_slice_plan(t.shape, e_.op.slice_starts, e_.op.slice_steps, e_.op.slice_shape);
    auto buffer = output(t.dtype, plan.output_shape);
    if (!buffer) return buffer.status();
    const auto count = numel(plan.output_shape);
    if (count) {
      auto st = launch("launch_transpose", "CUDA index copy", [&] {
        return tcx_sm100_index_copy(abi_stream(scope_), static_cast<std::int32_t>(dtype_size(t.dtype)), ptr(0),
                                    buffer.value()->data(), count, plan.output_shape.data(), plan.input_strides.data(),
                                    static_cast<std::int32_t>(plan.output_shape.size()), plan.offset); });
      if (!st.ok()) return st;
    }
    return publish(out, t.dtype, plan.output_shape, buffer.move_value());
  }

  // concat (cuda_backend.cpp:376-398 of the reference): one block copy per input.
  Status concat(Tensor& out) {
    const auto dtype = e_.inputs[0].dtype;
    std::vector<Shape> shapes;
    for (const auto& t : e_.inputs) {
      if (t.dtype != dtype) return invalid("concat dtypes must match");
      shapes.push_back(t.shape);
    }
    const auto plan = make_concat_plan(shapes, e_.op.axis);
    auto buffer = output(dtype, plan.output_shape);
    if (!buffer) return buffer.status();
    if (numel(plan.output_shape)) {
      const Dim output_block = plan.output_shape[plan.axis] * plan.inner;
      Dim offset = 0;
      for (std::size_t i = 0; i < e_.inputs.size(); ++i) {
        const Dim block = e_.inputs[i].shape[plan.axis] * plan.inner;
        const Dim count = numel(e_.inputs[i].shape);
        if (count) {
          auto st = launch("launch_concat", "CUDA concat", [&] {
            return tcx_sm100_concat(abi_stream(scope_), static_cast<std::int32_t>(dtype_size(dtype)), ptr(i),
                                    buffer.value()->data(), count, block, output_block, offset); });
          if (!st.ok()) return st;
        }
        offset += block;
      }
    }
    return publish(out, dtype, plan.output_shape, buffer.move_value());
  }

  // comparisons, logical ops and where (make_predicate_plan).
  Status predicate(Tensor& out) {
    const auto plan = make_predicate_plan(e_.op, e_.inputs);
    auto buffer = output(plan.output_dtype, plan.output_shape);
    if (!buffer) return buffer.status();
    const auto count = numel(plan.output_shape);
    if (count) {
      Shape metadata = plan.output_shape;
      for (const auto& strides : plan.input_strides) metadata.insert(metadata.end(), strides.begin(), strides.end());
      const auto kind = e_.op.kind;
      const auto dtype = e_.inputs[kind == OpKind::kWhere ? 1 : 0].dtype;
      auto st = launch("launch_predicate", "CUDA predicate", [&] {
        return tcx_sm100_predicate(abi_stream(scope_), static_cast<int>(kind), abi_dtype(dtype), ptr(0),
                                   e_.inputs.size() > 1 ? ptr(1) : nullptr, e_.inputs.size() > 2 ? ptr(2) : nullptr,
                                   buffer.value()->data(), count, metadata.data(),
                                   static_cast<std::int32_t>(plan.output_shape.size())); });
      if (!st.ok()) return st;
    }
    return publish(out, plan.output_dtype, plan.output_shape, buffer.move_value());
  }

  // any / all (make_boolean_reduction_plan).
  Status bool_reduce(Tensor& out) {
    const auto& t = e_.inputs[0];
    if (t.dtype != DType::kBool) return invalid("any/all require bool tensors");
    const auto plan = make_boolean_reduction_plan(e_.op, t.shape);
    auto buffer = output(DType::kBool, plan.output_shape);
    if (!buffer) return buffer.status();
    const auto groups = numel(plan.output_shape);
    if (groups) {
      auto st = launch("launch_bool_reduce", "CUDA bool reduction", [&] {
        return tcx_sm100_bool_reduce(abi_stream(scope_), static_cast<int>(e_.op.kind), ptr(0), buffer.value()->data(),
                                     groups, plan.reduction_size, plan.index_metadata.data(),
                                     static_cast<std::int32_t>(t.shape.size())); });
      if (!st.ok()) return st;
    }
    return publish(out, DType::kBool, plan.output_shape, buffer.move_value());
  }

  // masked_select (make_masked_select_plan): count on the device, read it, then copy.
  Status masked_select(Tensor& out) {
    const auto& t = e_.inputs[0];
    const auto& mask = e_.inputs[1];
    const auto plan = make_masked_select_plan(t, mask);
    const auto count = numel(mask.shape);
    Scratch ws(tcx_sm100_masked_select_workspace_bytes(count) + 64, scope_);
    if (!ws.status().ok()) return ws.status();
    auto* selected_dev = reinterpret_cast<std::int64_t*>(static_cast<char*>(ws.data()) + ws.bytes() - 64);
    Dim selected = 0;
    if (count) {
      auto st = launch("launch_mask_prefix", "CUDA mask count", [&] {
        return tcx_sm100_masked_select_count(abi_stream(scope_), ptr(1), count, selected_dev, ws.data(),
                                             ws.bytes() - 64); });
      if (!st.ok()) return st;
      ProfileScope span(ProfileCategory::kCopy, "device_to_host", "cuda", sizeof(Dim));
      st = runtime_status(cudaMemcpyAsync(&selected, selected_dev, sizeof(Dim), cudaMemcpyDeviceToHost, scope_.stream()),
                          "CUDA mask result count");
      if (!st.ok()) return st;
      st = runtime_status(cudaStreamSynchronize(scope_.stream()), "CUDA mask result count");
      if (!st.ok()) return st;
    }
    Shape shape{selected};
    shape.insert(shape.end(), plan.tail_shape.begin(), plan.tail_shape.end());
    auto buffer = output(t.dtype, shape);
    if (!buffer) return buffer.status();
    if (selected && numel(t.shape)) {
      auto st = launch("launch_mask_copy", "CUDA masked selection", [&] {
        return tcx_sm100_masked_select(abi_stream(scope_), static_cast<std::int32_t>(dtype_size(t.dtype)), ptr(0),
                                       ptr(1), count, plan.block_size, buffer.value()->data(), ws.data(),
                                       ws.bytes() - 64); });
      if (!st.ok()) return st;
    }
    return publish(out, t.dtype, shape, buffer.move_value());
  }

  // embedding (make_embedding_plan): gather with the index range checked on the device.
  Status embedding(Tensor& out) {
    const auto plan = make_embedding_plan(e_.inputs);
    auto buffer = output(DType::kFloat32, plan.shape);
    if (!buffer) return buffer.status();
    if (plan.indices) {
      Scratch flag(sizeof(int), scope_);
      if (!flag.status().ok()) return flag.status();
      auto st = launch("launch_embedding_gather", "CUDA embedding", [&] {
        return tcx_sm100_embedding(abi_stream(scope_), static_cast<const std::int32_t*>(ptr(0)), plan.indices,
                                   static_cast<const float*>(ptr(1)), plan.vocabulary, plan.width,
                                   static_cast<float*>(buffer.value()->data()), static_cast<int*>(flag.data())); });
      if (!st.ok()) return st;
      auto bad = read_flag(flag);
      if (!bad) return bad.status();
      if (bad.value()) return invalid("embedding index out of range");
    }
    return publish(out, DType::kFloat32, plan.shape, buffer.move_value());
  }
};

}  // namespace

// ------------------------------------------------------------------ buffers
Expected<std::shared_ptr<CudaBuffer>> CudaBuffer::create(DType dtype, const Shape& shape, int device) {
  auto bytes = byte_size(dtype, shape);
  if (!bytes) return bytes.status();
  DeviceScope scope(device);
  if (!scope.ready()) return scope.status();
  auto buffer = std::make_shared<CudaBuffer>();
  buffer->dtype_ = dtype;
  buffer->bytes_ = bytes.value();
  buffer->device_ = device;
  if (buffer->bytes_) {
    auto pool = active_memory_pool();
    if (pool) {
      auto p = pool->allocate(buffer->bytes_);
      if (!p) return p.status();
      buffer->data_ = p.value();
      buffer->pool_ = std::move(pool);
    } else {
      ProfileScope span(ProfileCategory::kAllocation, "cudaMallocAsync", "cuda", buffer->bytes_);
      auto st = runtime_status(cudaMallocAsync(&buffer->data_, buffer->bytes_, scope.stream()), "CUDA allocation");
      if (!st.ok()) return st;
    }
  }
  return buffer;
}

Expected<std::shared_ptr<CudaBuffer>> CudaBuffer::borrow(DType dtype, const Shape& shape, void* data,
                                                        std::shared_ptr<void> owner, int device) {
  auto bytes = byte_size(dtype, shape);
  if (!bytes) return bytes.status();
  if (bytes.value() && !data) return invalid("borrowed CUDA memory requires a pointer");
  auto buffer = std::make_shared<CudaBuffer>();
  buffer->dtype_ = dtype;
  buffer->bytes_ = bytes.value();
  buffer->device_ = device;
  buffer->data_ = data;
  buffer->external_owner_ = owner ? std::move(owner) : std::shared_ptr<void>(data, [](void*) {});
  return buffer;
}

Expected<std::shared_ptr<CudaBuffer>> CudaBuffer::borrow(DType dtype, const Shape& shape, void* data,
                                                        std::shared_ptr<void> owner,
                                                        std::shared_ptr<ExternalStorage> storage) {
  int device = 0;
  if (data) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, data) == cudaSuccess && attr.type == cudaMemoryTypeDevice) device = attr.device;
    else cudaGetLastError();
  }
  auto bytes = byte_size(dtype, shape);
  if (!bytes) return bytes.status();
  if (storage) {
    if (auto st = storage->validate_range(data, dtype, bytes.value()); !st.ok()) return st;
  }
  auto buffer = borrow(dtype, shape, data, std::move(owner), device);
  if (!buffer) return buffer.status();
  buffer.value()->external_storage_ = std::move(storage);
  return buffer;
}

StorageIdentity CudaBuffer::storage_identity() const {
  if (external_storage_) return external_storage_->identity(data_, bytes_);
  return {this, 0, bytes_};
}

std::shared_ptr<StorageAccess> CudaBuffer::access() const {
  return external_storage_ ? external_storage_->access() : nullptr;
}

const std::shared_ptr<PrimaryContext>& CudaBuffer::context() const {
  if (!context_) {
    DeviceScope scope(device_);
    if (scope.ready()) {
      auto ctx = PrimaryContext::acquire();
      if (ctx) context_ = ctx.move_value();
    }
  }
  return context_;
}

CudaBuffer::~CudaBuffer() {
  if (external_owner_ || !data_) return;
  DeviceScope scope(device_);
  if (!scope.ready()) return;
  const bool exported = exported_.load(std::memory_order_relaxed);
  if (pool_) {
    pool_->release(data_, bytes_, !exported);
    return;
  }
  // Backend work on this buffer has completed (every execute synchronizes its stream
  // before returning), so a stream-ordered free on this thread's stream is safe. An
  // exported buffer may still be read by a foreign consumer on a stream this backend
  // does not track: wait for the device first.
  ProfileScope span(ProfileCategory::kDeallocation, "cudaFreeAsync", "cuda", bytes_);
  if (exported) {
    (void)cudaDeviceSynchronize();
    cudaGetLastError();
  }
  (void)cudaFreeAsync(data_, scope.stream());
}

StorageRelation CudaBuffer::storage_relation(const Buffer& other) const {
  const auto* rhs = dynamic_cast<const CudaBuffer*>(&other);
  if (!rhs || external_storage_ || rhs->external_storage_) return Buffer::storage_relation(other);
  if (device_ != rhs->device_) return StorageRelation::kDisjoint;
  if (this == rhs) return StorageRelation::kSameRange;
  if (!nbytes() || !rhs->nbytes()) return StorageRelation::kDisjoint;
  const auto a = reinterpret_cast<std::uintptr_t>(data_), b = reinterpret_cast<std::uintptr_t>(rhs->data_);
  if (a == b && nbytes() == rhs->nbytes()) return StorageRelation::kSameRange;
  const bool overlap = a <= b ? b - a < nbytes() : a - b < rhs->nbytes();
  return overlap ? StorageRelation::kPartialOverlap : StorageRelation::kDisjoint;
}

// ------------------------------------------------------------------ tensors
CudaTensor::CudaTensor(DType dtype, Shape shape, std::shared_ptr<CudaBuffer> buffer)
    : dtype_(dtype), shape_(std::move(shape)), strides_(contiguous_strides(shape_)), buffer_(std::move(buffer)) {}

std::size_t CudaTensor::nbytes() const { return buffer_ ? buffer_->nbytes() : 0; }

Tensor to_core_tensor(const CudaTensor& t) {
  return Tensor{t.dtype(), t.shape(), t.strides(), Device{"cuda", t.buffer()->device()},
                std::static_pointer_cast<Buffer>(t.buffer()), 0};
}

Expected<CudaTensor> from_core_tensor(const Tensor& t) {
  try {
    if (t.device.type != "cuda") return invalid("CUDA tensor metadata requires device='cuda'");
    if (t.device.index < 0 || t.device.index >= device_count())
      return invalid("CUDA tensor metadata requires an available device index");
    if (t.offset != 0) return invalid("CUDA tensor metadata with non-zero offset is unsupported");
    if (t.strides != contiguous_strides(t.shape)) return invalid("CUDA tensor metadata must be contiguous");
    auto buffer = std::dynamic_pointer_cast<CudaBuffer>(t.buffer);
    if (!buffer) return invalid("CUDA tensor metadata requires a CUDA buffer");
    auto bytes = byte_size(t.dtype, t.shape);
    if (!bytes) return bytes.status();
    if (buffer->nbytes() != bytes.value() || buffer->dtype() != t.dtype)
      return invalid("CUDA buffer does not match tensor metadata");
    if (buffer->device() != t.device.index) return invalid("CUDA buffer device does not match tensor device");
    return CudaTensor(t.dtype, t.shape, std::move(buffer));
  } catch (const std::invalid_argument& e) {
    return invalid(e.what());
  }
}

// ------------------------------------------------------------------ device API
bool available() { return device_count() > 0 && tcx_sm100_device_supported(0) == TCX_OK; }

Expected<std::string> device_name() {
  auto info = device_info();
  if (!info) return info.status();
  return info.value().name;
}

Expected<DeviceInfo> device_info() {
  DeviceScope scope(0);
  if (!scope.ready()) return scope.status();
  cudaDeviceProp prop{};
  auto st = runtime_status(cudaGetDeviceProperties(&prop, 0), "cudaGetDeviceProperties");
  if (!st.ok()) return st;
  DeviceInfo info;
  info.name = prop.name;
  info.major = prop.major;
  info.minor = prop.minor;
  (void)cudaRuntimeGetVersion(&info.runtime_version);
  (void)cudaDriverGetVersion(&info.driver_version);
  (void)cudaMemGetInfo(&info.free_bytes, &info.total_bytes);
  cudaGetLastError();
  return info;
}

Expected<CudaTensor> empty(Shape shape, DType dtype, int device) {
  try {
    (void)contiguous_strides(shape);
    auto buffer = CudaBuffer::create(dtype, shape, device);
    if (!buffer) return buffer.status();
    if (buffer.value()->nbytes()) {
      // the allocation is ordered on this thread's stream; complete it before the
      // tensor can reach another thread's stream
      DeviceScope scope(device);
      if (!scope.ready()) return scope.status();
      ProfileScope wait(ProfileCategory::kSynchronize, "cudaStreamSynchronize", "cuda");
      if (auto st = runtime_status(cudaStreamSynchronize(scope.stream()), "CUDA allocation"); !st.ok()) return st;
    }
    return CudaTensor(dtype, std::move(shape), buffer.move_value());
  } catch (const std::invalid_argument& e) {
    return invalid(e.what());
  }
}

Expected<CudaTensor> from_cpu(const cpu::CpuTensor& tensor, int device) {
  auto buffer = CudaBuffer::create(tensor.dtype(), tensor.shape(), device);
  if (!buffer) return buffer.status();
  if (buffer.value()->nbytes()) {
    DeviceScope scope(device);
    if (!scope.ready()) return scope.status();
    // pinned staging with parallel host copies for large pageable tensors (synchronous)
    ProfileScope span(ProfileCategory::kCopy, "host_to_device", "cuda", buffer.value()->nbytes());
    auto st = abi_status(tcx_sm100_copy_to_device(abi_stream(scope), buffer.value()->data(), tensor.data(),
                                                  buffer.value()->nbytes()),
                         "CUDA upload");
    if (!st.ok()) return st;
  }
  return CudaTensor(tensor.dtype(), tensor.shape(), buffer.move_value());
}

Expected<cpu::CpuTensor> to_cpu(const CudaTensor& tensor) {
  cpu::CpuTensor result(tensor.dtype(), tensor.shape());
  if (tensor.nbytes()) {
    DeviceScope scope(tensor.buffer()->device());
    if (!scope.ready()) return scope.status();
    ProfileScope span(ProfileCategory::kCopy, "device_to_host", "cuda", tensor.nbytes());
    auto st = abi_status(tcx_sm100_copy_to_host(abi_stream(scope), result.mutable_data(), tensor.buffer()->data(),
                                                tensor.nbytes()),
                         "CUDA download");
    if (!st.ok()) return st;
  }
  return result;
}

// ------------------------------------------------------------------ execute
Status CudaBackend::execute(const BackendExecution& e) {
  ProfileScope profile(ProfileCategory::kDispatch, "execute", "cuda", std::nullopt,
                       e.op_class == BackendOpClass::kPrimitive ? std::optional{e.op.kind} : std::nullopt);
  try {
    if (e.op_class == BackendOpClass::kKernel) return execute_compiled_kernel(e);
    if (auto st = validate_primitive_execution_contract(e, "cuda"); !st.ok()) return st;
    std::vector<CudaTensor> in;
    in.reserve(e.inputs.size());
    for (const auto& t : e.inputs) {
      auto c = from_core_tensor(t);
      if (!c) return c.status();
      in.push_back(c.move_value());
    }
    const int device = e.op.kind == OpKind::kFill ? e.outputs[0].device.index : in.empty() ? 0 : in[0].buffer()->device();
    for (const auto& t : in)
      if (t.buffer()->device() != device) return invalid("device mismatch between CUDA inputs");
    DeviceScope scope(device);
    if (!scope.ready()) return scope.status();
    Tensor result, second;
    Executor ex(e, in, scope);
    if (auto st = ex.run(result, second); !st.ok()) return st;
    // every launch already waited inside its span; this only catches stray work (a copy)
    if (auto st = runtime_status(cudaStreamSynchronize(scope.stream()), "CUDA stream synchronize"); !st.ok())
      return st;
    e.outputs[0] = std::move(result);  // publish only on success
    if (e.op.kind == OpKind::kTopK && e.outputs.size() > 1) e.outputs[1] = std::move(second);
    return Status::Ok();
  } catch (const std::invalid_argument& err) {
    return invalid(err.what());
  } catch (const std::exception& err) {
    return {StatusCode::kInternal, err.what()};
  }
}

}  // namespace tensorcx::cuda
