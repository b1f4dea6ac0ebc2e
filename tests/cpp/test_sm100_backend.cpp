// TEST INFRASTRUCTURE: contract test of the sm100 CudaBackend, in the style of the
// reference's tests/cpp/test_cuda_backend_contract.cpp (returns 77 to skip without a
// GPU). Every hot-path primitive runs through CudaBackend::execute on device tensors
// and is compared with the reference CpuBackend on the same inputs; malformed
// descriptors must fail with kInvalidArgument and leave result slots untouched; the
// memory pool's OOM / free-failure accounting is driven by an injected PoolRuntime
// (host fakes, no GPU memory exhausted).
#include <array>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>
#include <thread>
#include <atomic>
#include <chrono>
#include <mutex>
#include <set>

#include "tensorcx/backends/cpu/cpu_backend.h"
#include "tensorcx/backends/cuda/cuda_backend.h"
#include "tensorcx/backends/cuda/cuda_context.h"
#include "tensorcx/backends/cuda/cuda_external_storage.h"
#include "tensorcx/backends/cuda/cuda_kernel.h"
#include "tensorcx/backends/cuda/cuda_device.h"
#include "tensorcx/backends/cuda/cuda_memory_pool.h"
#include "tensorcx/core/profiling.h"

using namespace tensorcx;

namespace {
int failures = 0;
void check(bool ok, const std::string& what) {
  if (!ok) {
    std::fprintf(stderr, "FAIL: %s\n", what.c_str());
    ++failures;
  }
}

cpu::CpuTensor randn(Shape shape, std::uint32_t seed, float scale = 1.0f) {
  std::mt19937 gen(seed);
  std::normal_distribution<float> dist(0.0f, scale);
  std::vector<float> v(static_cast<std::size_t>(numel(shape)));
  for (auto& x : v) x = dist(gen);
  return cpu::CpuTensor(shape, std::move(v));
}

cpu::CpuTensor randi(Shape shape, std::uint32_t seed) {
  std::mt19937 gen(seed);
  std::uniform_int_distribution<std::int32_t> dist(-1000, 1000);
  std::vector<std::int32_t> v(static_cast<std::size_t>(numel(shape)));
  for (auto& x : v) x = dist(gen);
  return cpu::CpuTensor(shape, std::move(v));
}

cpu::CpuTensor randb(Shape shape, std::uint32_t seed) {
  std::mt19937 g(seed);
  std::vector<std::uint8_t> v(static_cast<std::size_t>(numel(shape)));
  for (auto& x : v) x = (g() % 10) < 7;
  return cpu::CpuTensor(shape, std::move(v));
}

Tensor on_gpu(const cpu::CpuTensor& t, int device = 0) {
  auto c = cuda::from_cpu(t, device);
  if (!c) {
    std::fprintf(stderr, "upload failed: %s\n", c.status().message().c_str());
    std::exit(1);
  }
  return cuda::to_core_tensor(c.value());
}

Status run(Backend& backend, OpDesc op, std::vector<Tensor> inputs, Tensor& out, Tensor* second = nullptr) {
  std::vector<Tensor> outputs(second ? 2 : 1);
  BackendExecution e{BackendOpClass::kPrimitive, op, inputs, outputs, std::nullopt, std::nullopt, {}};
  auto st = backend.execute(e);
  if (st.ok()) {
    out = outputs[0];
    if (second) *second = outputs[1];
  }
  return st;
}

cpu::CpuTensor download(const Tensor& t) {
  auto c = cuda::from_core_tensor(t);
  if (!c) { std::fprintf(stderr, "bad result: %s\n", c.status().message().c_str()); std::exit(1); }
  auto h = cuda::to_cpu(c.value());
  if (!h) { std::fprintf(stderr, "download failed: %s\n", h.status().message().c_str()); std::exit(1); }
  return h.move_value();
}

// |gpu - cpu| <= atol + rtol |cpu| elementwise (NaN == NaN), or exact for int32 and bool.
bool close(const cpu::CpuTensor& a, const cpu::CpuTensor& b, double rtol, double atol) {
  if (a.shape() != b.shape() || a.dtype() != b.dtype()) return false;
  if (a.dtype() != DType::kFloat32) {
    return std::memcmp(a.data(), b.data(), static_cast<std::size_t>(a.size()) * dtype_size(a.dtype())) == 0;
  }
  auto x = a.float_data(), y = b.float_data();
  for (std::size_t i = 0; i < x.size(); ++i) {
    if (std::isnan(x[i]) || std::isnan(y[i])) {
      if (std::isnan(x[i]) != std::isnan(y[i])) return false;
      continue;
    }
    if (std::fabs(double(x[i]) - y[i]) > atol + rtol * std::fabs(double(y[i]))) return false;
  }
  return true;
}

struct Case {
  std::string name;
  OpDesc op;
  std::vector<cpu::CpuTensor> inputs;
  double rtol, atol;
  // float32 full-tensor sum: the CPU adds left to right in float32 and can itself be
  // off by more than 1e-5; accept a GPU result closer to the exact sum than the CPU's.
  bool full_sum = false;
};

bool sum_close(const cpu::CpuTensor& gpu, const cpu::CpuTensor& cpu_result, const cpu::CpuTensor& input, double divisor) {
  double exact = 0.0;
  for (float v : input.float_data()) exact += v;
  exact /= divisor;
  const double g = gpu.float_data()[0], c = cpu_result.float_data()[0];
  return std::fabs(g - c) <= 1e-5 * std::fabs(c) || std::fabs(g - exact) <= std::fabs(c - exact);
}

void compare(Backend& gpu, Backend& ref, const Case& c, int device = 0) {
  std::vector<Tensor> gin, cin;
  for (const auto& t : c.inputs) {
    gin.push_back(on_gpu(t, device));
    cin.push_back(cpu::to_core_tensor(t));
  }
  Tensor g, r, g2, r2;
  const bool two = c.op.kind == OpKind::kTopK;
  auto gs = run(gpu, c.op, gin, g, two ? &g2 : nullptr);
  auto rs = run(ref, c.op, cin, r, two ? &r2 : nullptr);
  if (!rs.ok()) {
    check(!gs.ok() && gs.code() == rs.code(), c.name + ": CPU rejects (" + rs.message() + "), GPU must too");
    return;
  }
  if (!gs.ok()) { check(false, c.name + ": " + gs.message()); return; }
  check(g.device.type == "cuda" && g.device.index == device, c.name + ": result device");
  if (c.full_sum) {
    const double n = c.op.kind == OpKind::kMean ? static_cast<double>(c.inputs[0].size()) : 1.0;
    check(sum_close(download(g), cpu::from_core_tensor(r), c.inputs[0], n), c.name + ": full sum vs CPU / exact");
  } else {
    check(close(download(g), cpu::from_core_tensor(r), c.rtol, c.atol), c.name + ": parity with CpuBackend");
    if (two) check(close(download(g2), cpu::from_core_tensor(r2), 0, 0), c.name + ": indices parity with CpuBackend");
  }
}

// inputs with the float32 edge values of the elementwise ops: signed zeros, infinities,
// NaN, subnormals, negatives and values near the int32 range limits
cpu::CpuTensor specials(std::uint32_t seed) {
  auto t = randn({4, 64}, seed, 3.0f);
  std::vector<float> v(t.float_data().begin(), t.float_data().end());
  const float edge[] = {0.0f, -0.0f, INFINITY, -INFINITY, NAN, 1e-40f, -1e-40f, 2147483520.0f, -2147483648.0f,
                        2147483648.0f, 1e30f, -7.5f, 7.5f, 0.4999f, -0.5f, 1.0f};
  for (std::size_t i = 0; i < sizeof(edge) / sizeof(edge[0]); ++i) v[i * 13 % v.size()] = edge[i];
  return cpu::CpuTensor(t.shape(), std::move(v));
}

cpu::CpuTensor randk(Shape shape, std::uint32_t seed, int distinct) {  // many ties
  std::mt19937 g(seed);
  std::vector<float> v(static_cast<std::size_t>(numel(shape)));
  for (auto& x : v) x = static_cast<float>(static_cast<int>(g() % distinct) - distinct / 2);
  return cpu::CpuTensor(shape, std::move(v));
}

cpu::CpuTensor indices_i32(Shape shape, std::uint32_t seed, int vocabulary, bool out_of_range = false) {
  std::mt19937 g(seed);
  std::vector<std::int32_t> v(static_cast<std::size_t>(numel(shape)));
  for (auto& x : v) x = static_cast<std::int32_t>(g() % vocabulary);
  if (out_of_range && !v.empty()) v[v.size() / 2] = vocabulary;
  return cpu::CpuTensor(shape, std::move(v));
}

OpDesc desc(OpKind k) { OpDesc op; op.kind = k; return op; }
OpDesc axis_op(OpKind k, std::int64_t axis, double eps = 1e-5) { OpDesc op; op.kind = k; op.axis = axis; op.epsilon = eps; return op; }
OpDesc axes_op(OpKind k, Shape axes) { OpDesc op; op.kind = k; op.reduction_axes = axes; return op; }

// host fakes for the pool contract
int fake_oom_left = 0;
int fake_free_errors = 0;
std::vector<void*> fake_blocks;
cudaError_t fake_allocate(void** p, std::size_t bytes) {
  if (fake_oom_left > 0) { --fake_oom_left; return cudaErrorMemoryAllocation; }
  *p = std::malloc(bytes);
  fake_blocks.push_back(*p);
  return cudaSuccess;
}
cudaError_t fake_free(void* p) {
  std::free(p);
  if (fake_free_errors > 0) { --fake_free_errors; return cudaErrorInvalidValue; }
  return cudaSuccess;
}
cudaError_t fake_clear() { return cudaSuccess; }

void pool_contract() {
  using cuda::MemoryPool;
  using cuda::PoolRuntime;
  auto pool = std::make_shared<MemoryPool>(1024, 4, PoolRuntime{fake_allocate, fake_free, fake_clear});
  check(pool->enter().ok(), "pool enter");
  check(!std::make_shared<MemoryPool>(1024, 4, PoolRuntime{fake_allocate, fake_free, fake_clear})->enter().ok(),
        "nested pool rejected");
  auto a = pool->allocate(128);
  check(a.has_value(), "pool allocate");
  void* address = a.value();
  pool->release(address, 128, true);
  auto b = pool->allocate(128);
  check(b.has_value() && b.value() == address && pool->stats().hits == 1, "exact-size reuse");
  pool->release(b.value(), 128, true);
  fake_oom_left = 1;  // next miss runs out: the cache is drained and the allocation retried once
  auto c = pool->allocate(256);
  check(c.has_value() && pool->stats().oom_retries == 1 && pool->stats().free_calls == 1, "OOM drain and retry");
  pool->release(c.value(), 256, false);
  check(pool->stats().uncached_returns == 1, "non-reusable block returned, not cached");
  fake_oom_left = 2;  // a retry that also fails is one allocation failure
  auto d = pool->allocate(64);
  check(!d.has_value() && pool->stats().allocation_failures == 1, "failed retry accounting (no cache: no retry)");
  fake_oom_left = 0;
  auto e = pool->allocate(32);
  pool->release(e.value(), 32, true);
  fake_free_errors = 1;
  check(!pool->trim().ok() && pool->stats().free_failures == 1 && pool->stats().cached_bytes == 0,
        "trim reports free failure and gives ownership up");
  check(pool->exit().ok(), "pool exit");
  check(!pool->enter().ok(), "pools are single-use");
  check(pool->stats().in_use_bytes == 0, "nothing left in use");
}

void error_contract(Backend& gpu) {
  auto a = on_gpu(randn({2, 3}, 1));
  Tensor sentinel;
  sentinel.device = Device{"sentinel", 7};
  std::vector<Tensor> outputs{sentinel};
  // matmul contracting mismatch
  std::vector<Tensor> in{a, a};
  BackendExecution e{BackendOpClass::kPrimitive, desc(OpKind::kMatmul), in, outputs, std::nullopt, std::nullopt, {}};
  auto st = gpu.execute(e);
  check(st.code() == StatusCode::kInvalidArgument, "matmul shape mismatch -> invalid argument");
  check(outputs[0].device.type == "sentinel", "failed matmul leaves the result slot untouched");
  // bad epsilon
  std::vector<Tensor> one{a};
  BackendExecution n{BackendOpClass::kPrimitive, axis_op(OpKind::kRmsNorm, -1, -1.0), one, outputs, std::nullopt,
                     std::nullopt, {}};
  st = gpu.execute(n);
  check(st.code() == StatusCode::kInvalidArgument && st.message().find("epsilon") != std::string::npos,
        "bad epsilon -> invalid argument");
  check(outputs[0].device.type == "sentinel", "failed norm leaves the result slot untouched");
  // axis out of range, wrong input count, CPU tensor handed to the CUDA backend
  BackendExecution r{BackendOpClass::kPrimitive, axis_op(OpKind::kSum, 2), one, outputs, std::nullopt, std::nullopt, {}};
  check(gpu.execute(r).code() == StatusCode::kInvalidArgument, "axis out of range");
  BackendExecution wrong{BackendOpClass::kPrimitive, desc(OpKind::kAdd), one, outputs, std::nullopt, std::nullopt, {}};
  check(gpu.execute(wrong).code() == StatusCode::kInvalidArgument, "input count mismatch");
  std::vector<Tensor> host{cpu::to_core_tensor(randn({2, 3}, 2))};
  BackendExecution h{BackendOpClass::kPrimitive, desc(OpKind::kExp), host, outputs, std::nullopt, std::nullopt, {}};
  check(gpu.execute(h).code() == StatusCode::kInvalidArgument, "CPU tensor rejected");
  check(outputs[0].device.type == "sentinel", "rejected calls leave the result slot untouched");
}

// The rest of the reference's backend surface: driver contexts and the
// external-storage registry and lease.
struct FakeAccess final : StorageAccess {
  Status validate() const override { return Status::Ok(); }
};
struct FakeStorage final : cuda::ExternalStorage {
  void* base{};
  std::size_t size{};
  int completions{};
  std::shared_ptr<StorageAccess> lock = std::make_shared<FakeAccess>();
  std::shared_ptr<StorageAccess> access() override { return lock; }
  std::uintptr_t begin() const override { return reinterpret_cast<std::uintptr_t>(base); }
  std::size_t bytes() const override { return size; }
  std::size_t mapped_bytes() const override { return size; }
  Status validate_range(void* data, DType, std::size_t n) const override {
    const auto a = reinterpret_cast<std::uintptr_t>(data);
    return a >= begin() && a + n <= begin() + size ? Status::Ok()
                                                   : Status(StatusCode::kInvalidArgument, "outside the storage");
  }
  StorageIdentity identity(void* data, std::size_t n) const override {
    return {this, reinterpret_cast<std::uintptr_t>(data) - begin(), n};
  }
  Status complete_cuda() override {
    ++completions;
    return Status::Ok();
  }
  void poison() noexcept override {}
};

// ---------------------------------------------------------------- compiled kernels
// A generated elementwise add as a producer would emit it for sm_100a: one guarded
// store per thread, no output reads (written by hand here; the body is plain PTX).
const char* kAddBody = R"(.version 8.7
.target sm_100a
.address_size 64

.visible .entry tensorcx_add_v1(
	.param .u64 p_a,
	.param .u64 p_b,
	.param .u64 p_out,
	.param .u32 p_n
)
{
	.reg .pred 	%p<2>;
	.reg .b32 	%r<6>;
	.reg .f32 	%f<4>;
	.reg .b64 	%rd<8>;

	ld.param.u64 	%rd1, [p_a];
	ld.param.u64 	%rd2, [p_b];
	ld.param.u64 	%rd3, [p_out];
	ld.param.u32 	%r1, [p_n];
	mov.u32 	%r2, %ctaid.x;
	mov.u32 	%r3, %ntid.x;
	mov.u32 	%r4, %tid.x;
	mad.lo.s32 	%r5, %r2, %r3, %r4;
	setp.ge.u32 	%p1, %r5, %r1;
	@%p1 bra 	$L_done;
	cvta.to.global.u64 	%rd4, %rd1;
	cvta.to.global.u64 	%rd5, %rd2;
	cvta.to.global.u64 	%rd6, %rd3;
	mul.wide.u32 	%rd7, %r5, 4;
	add.s64 	%rd4, %rd4, %rd7;
	add.s64 	%rd5, %rd5, %rd7;
	add.s64 	%rd6, %rd6, %rd7;
	ld.global.f32 	%f1, [%rd4];
	ld.global.f32 	%f2, [%rd5];
	add.rn.f32 	%f3, %f1, %f2;
	st.global.f32 	[%rd6], %f3;
$L_done:
	ret;
}
)";

std::string add_ptx(bool v2, const std::string& body = kAddBody) {
  return "// " + cuda::kernel_manifest(cuda::KernelSignature{"tttu", 2, 3}, "add", v2) + "\n" + body;
}

std::vector<KernelArgument> add_args(const Tensor& a, const Tensor& b, const Tensor& out, std::uint32_t n) {
  std::vector<KernelArgument> args(4);
  args[0] = {KernelArgumentKind::kTensor, &a, 0};
  args[1] = {KernelArgumentKind::kTensor, &b, 0};
  args[2] = {KernelArgumentKind::kTensor, &out, 0};
  args[3] = {KernelArgumentKind::kUInt32, nullptr, n};
  return args;
}

std::size_t count_named(const ProfileResult& r, const char* name) {
  std::size_t n = 0;
  for (const auto& e : r.events) n += std::strcmp(e.name, name) == 0;
  return n;
}

void compiled_kernel_contract() {
  check(cuda::compiled_kernel_support().ok(), "compiled kernels supported on sm_100");
  const cuda::KernelSignature sig{"tttu", 2, 3};
  // rejected before any JIT: target, manifest, signature, entry
  std::string wrong_target = add_ptx(true);
  wrong_target.replace(wrong_target.find("sm_100a\n.address"), 7, "sm_90a ");
  check(cuda::CudaKernelModule::load(wrong_target, "tensorcx_add_v1", sig).status().code() ==
            StatusCode::kInvalidArgument, "PTX for another target rejected");
  check(!cuda::CudaKernelModule::load(kAddBody, "tensorcx_add_v1", sig), "PTX without a manifest rejected");
  check(!cuda::CudaKernelModule::load(add_ptx(true), "tensorcx_add_v1", cuda::KernelSignature{"tttt", 2, 3}),
        "malformed signature rejected");
  check(!cuda::CudaKernelModule::load(add_ptx(true), "tensorcx_relu_v1", sig), "unknown entry rejected");
  auto v2 = cuda::CudaKernelModule::load(add_ptx(true), "tensorcx_add_v1", sig);
  auto v1 = cuda::CudaKernelModule::load(add_ptx(false), "tensorcx_add_v1", sig);
  check(v2.has_value() && v1.has_value(), "v1 and v2 modules load");
  if (!v2 || !v1) return;
  check(v2.value()->artifact_id() != v1.value()->artifact_id(), "distinct artifact ids");

  const std::uint32_t n = 1000;
  const auto ha = randn({n}, 151), hb = randn({n}, 152);
  std::vector<float> seven(n, 7.0f);
  const Tensor a = on_gpu(ha), b = on_gpu(hb), templ = on_gpu(cpu::CpuTensor(Shape{n}, seven));
  auto sum_of = [&](const cpu::CpuTensor& x, const cpu::CpuTensor& y, std::uint32_t upto, const std::vector<float>& rest) {
    std::vector<float> v(n);
    for (std::uint32_t i = 0; i < n; ++i) v[i] = i < upto ? x.float_data()[i] + y.float_data()[i] : rest[i];
    return cpu::CpuTensor(Shape{n}, std::move(v));
  };

  // v2, every element written: no template copy, a private result, template untouched
  auto token = begin_profile(1000, true);
  auto full = cuda::launch_compiled_kernel(v2.value(), add_args(a, b, templ, n), n, 128);
  auto prof = end_profile(token);
  check(full.has_value() && close(download(cuda::to_core_tensor(full.value())), sum_of(ha, hb, n, seven), 0, 0),
        "v2 full write: a + b");
  check(count_named(prof, "device_to_device") == 0, "v2 full write: no output template copy");
  bool timed = false;
  for (const auto& d : prof.device_events) timed = timed || (std::strcmp(d.name, "generated_kernel") == 0 && !d.error);
  check(timed, "generated kernel launch has a device interval");
  check(close(download(templ), cpu::CpuTensor(Shape{n}, seven), 0, 0), "output template unchanged");

  // v2, an input aliasing the template keeps reading the template's values
  auto alias = cuda::launch_compiled_kernel(v2.value(), add_args(templ, b, templ, n), n, 256);
  check(alias.has_value() &&
            close(download(cuda::to_core_tensor(alias.value())), sum_of(cpu::CpuTensor(Shape{n}, seven), hb, n, seven), 0, 0),
        "v2 full write: aliased input reads the template");

  // v1: the result starts as a copy of the template, aliased inputs read the copy
  token = begin_profile(1000, true);
  auto copied = cuda::launch_compiled_kernel(v1.value(), add_args(templ, b, templ, n), n, 128);
  prof = end_profile(token);
  check(copied.has_value() &&
            close(download(cuda::to_core_tensor(copied.value())), sum_of(cpu::CpuTensor(Shape{n}, seven), hb, n, seven), 0, 0),
        "v1: aliased input reads the template copy");
  check(count_named(prof, "device_to_device") == 1, "v1: one output template copy");

  // v2 but partial work: the untouched suffix keeps the template's bits
  auto partial = cuda::launch_compiled_kernel(v2.value(), add_args(a, b, templ, n - 37), n - 37, 96);
  check(partial.has_value() &&
            close(download(cuda::to_core_tensor(partial.value())), sum_of(ha, hb, n - 37, seven), 0, 0),
        "partial launch: suffix keeps the template");

  // zero work: no launch, a distinct copy of the template
  auto zero = cuda::launch_compiled_kernel(v2.value(), add_args(a, b, templ, 0), 0, 32);
  check(zero.has_value() && zero.value().buffer()->data() != cuda::from_core_tensor(templ).value().buffer()->data() &&
            close(download(cuda::to_core_tensor(zero.value())), cpu::CpuTensor(Shape{n}, seven), 0, 0),
        "zero work: a private copy of the template");

  // guard and block limits
  check(!cuda::launch_compiled_kernel(v2.value(), add_args(a, b, templ, n - 1), n, 128), "guard must equal threads");
  check(!cuda::launch_compiled_kernel(v2.value(), add_args(a, b, templ, n), n, 4096), "block size limit");
  // an unknown artifact id through the backend
  std::array<Tensor, 1> outs{templ};
  const auto args = add_args(a, b, templ, n);
  BackendExecution e{BackendOpClass::kKernel, {}, {}, outs, LaunchConfig{n, 1, 1, 128, 1, 1},
                     CompilationTarget{KernelArtifactKind::kBinary, "no-such-artifact", "tensorcx_add_v1"}, args};
  cuda::CudaBackend backend;
  check(backend.execute(e).code() == StatusCode::kInvalidArgument, "unknown artifact rejected");
}

// ---------------------------------------------------------------- profiling records
// With a profile active, every execute is a dispatch span, every launch a compute_sync
// span with a device interval of the same name, pool traffic pool_acquire/_release.
void profiling_contract(Backend& gpu) {
  const Tensor a = on_gpu(randn({64, 96}, 161)), b = on_gpu(randn({96, 80}, 162));
  auto pool = std::make_shared<cuda::MemoryPool>(1 << 24, 16);
  check(pool->enter().ok(), "profiling pool enter");
  const auto token = begin_profile(4096, true);
  Tensor m, s, sum, add;
  check(run(gpu, desc(OpKind::kMatmul), {a, b}, m).ok(), "profiled matmul");
  check(run(gpu, axis_op(OpKind::kSoftmax, -1), {m}, s).ok(), "profiled softmax");
  check(run(gpu, desc(OpKind::kAdd), {s, s}, add).ok(), "profiled add");
  check(run(gpu, axes_op(OpKind::kSum, {0, 1}), {add}, sum).ok(), "profiled sum");
  m = s = add = sum = Tensor{};
  const auto r = end_profile(token);
  check(pool->exit().ok(), "profiling pool exit");
  check(count_named(r, "execute") == 4, "one dispatch span per execute");
  for (const auto& e : r.events)
    if (std::strcmp(e.name, "execute") == 0) check(e.operation.has_value(), "dispatch span carries the operation");
  check(count_named(r, "pool_acquire") >= 4 && count_named(r, "pool_release") >= 4, "pool spans");
  std::set<std::string> names;
  for (const auto& d : r.device_events) {
    names.insert(d.name);
    check(d.error == nullptr && d.elapsed_ms && *d.elapsed_ms >= 0, std::string("device interval measured: ") + d.name);
    bool paired = false;
    for (const auto& h : r.events)
      paired = paired || (h.id == d.host_event_id && h.category == ProfileCategory::kCompute &&
                          std::strcmp(h.name, d.name) == 0);
    check(paired, std::string("device interval belongs to its compute_sync span: ") + d.name);
  }
  check(names.count("launch_matmul") && names.count("launch_axis") && names.count("launch_binary") &&
            names.count("launch_reduce_axes"),
        "launch names of the reference backend");
  check(r.device_events.size() == 4, "one device interval per launch");
  // no profile: nothing recorded, nothing timed
  Tensor quiet;
  check(run(gpu, desc(OpKind::kExp), {a}, quiet).ok(), "unprofiled call");
}

void surface_contract() {
  check(cuda::current_process(), "current process");
  auto ctx = cuda::PrimaryContext::acquire();
  check(ctx.has_value() && ctx.value()->get() != nullptr, "primary context retained");
  if (ctx) {
    cuda::ContextScope scope(ctx.value());
    check(scope.ready(), "context scope pushes the primary context");
  }
  // external storage: registry lookups, borrowed buffers that report its identity and
  // lock, and a lease that completes its CUDA work
  auto fake = std::make_shared<FakeStorage>();
  fake->size = 1 << 16;
  auto backing = cuda::empty({static_cast<Dim>(fake->size / 4)}, DType::kFloat32);  // device memory to "own"
  if (!backing) { check(false, "device memory for the external storage"); return; }
  fake->base = backing.value().buffer()->data();
  cuda::register_external_storage(fake);
  auto hit = cuda::find_external_storage(static_cast<char*>(fake->base) + 256, 1024);
  check(hit.has_value() && hit.value().get() == fake.get(), "registry finds the owner of a range");
  auto miss = cuda::find_external_storage(static_cast<char*>(fake->base) + fake->size - 4, 64);
  check(!miss && miss.status().code() == StatusCode::kInvalidArgument, "registry rejects a range past the end");
  auto buf = cuda::CudaBuffer::borrow(DType::kFloat32, {16}, static_cast<char*>(fake->base) + 512, nullptr,
                                      std::shared_ptr<cuda::ExternalStorage>(fake));
  check(buf.has_value(), "borrow from external storage");
  if (buf) {
    const auto id = buf.value()->storage_identity();
    check(id.token == fake.get() && id.offset == 512 && id.bytes == 64, "borrowed buffer reports the storage identity");
    check(buf.value()->access() == fake->lock, "borrowed buffer reports the storage lock");
    check(buf.value()->context() != nullptr, "buffer context");
    Tensor t{DType::kFloat32, {16}, contiguous_strides({16}), Device{"cuda", 0}, buf.value(), 0};
    std::vector<Tensor> ins{t}, outs(1);
    BackendExecution e{BackendOpClass::kPrimitive, desc(OpKind::kExp), ins, outs, std::nullopt, std::nullopt, {}};
    auto owners = cuda::external_owners(e);
    check(owners.size() == 1 && owners[0].get() == fake.get(), "external owners of an execution");
    {
      cuda::ExternalLease lease(owners);
      check(lease.status().ok(), "lease taken");
      check(lease.finish().ok() && fake->completions == 1, "lease completes the owner's CUDA work");
    }
    check(fake->completions == 1, "a finished lease does not complete twice");
  }
  auto bad = cuda::CudaBuffer::borrow(DType::kFloat32, {1 << 20}, fake->base, nullptr,
                                      std::shared_ptr<cuda::ExternalStorage>(fake));
  check(!bad, "borrow beyond the storage is rejected");
  cuda::unregister_external_storage(fake->begin(), fake.get());
  check(!cuda::find_external_storage(fake->base, 4), "unregistered storage is no longer found");
}

// Calls arrive concurrently from many threads (the bindings release the GIL around
// execute): four threads each run matmul -> softmax chains and check their results.
void concurrency_contract(Backend& gpu, Backend& ref) {
  const auto a = randn({64, 96}, 131), b = randn({96, 80}, 132);
  Tensor rm, rs;
  check(run(ref, desc(OpKind::kMatmul), {cpu::to_core_tensor(a), cpu::to_core_tensor(b)}, rm).ok(), "reference matmul");
  check(run(ref, axis_op(OpKind::kSoftmax, -1), {rm}, rs).ok(), "reference softmax");
  const auto expected = cpu::from_core_tensor(rs);
  std::atomic<int> bad{0};
  std::vector<std::thread> threads;
  for (int t = 0; t < 4; ++t) {
    threads.emplace_back([&] {
      for (int i = 0; i < 8; ++i) {
        Tensor m, s;
        if (!run(gpu, desc(OpKind::kMatmul), {on_gpu(a), on_gpu(b)}, m).ok() ||
            !run(gpu, axis_op(OpKind::kSoftmax, -1), {m}, s).ok() || !close(download(s), expected, 1e-4, 1e-5))
          ++bad;
      }
    });
  }
  for (auto& th : threads) th.join();
  check(bad.load() == 0, "concurrent executes from four threads");

  // every thread gets its own stream per device
  std::set<cudaStream_t> streams;
  std::mutex mu;
  std::vector<std::thread> probes;
  for (int t = 0; t < 4; ++t)
    probes.emplace_back([&] {
      cuda::DeviceScope scope(0);
      std::lock_guard lock(mu);
      streams.insert(scope.stream());
    });
  for (auto& th : probes) th.join();
  check(streams.size() == 4 && !streams.count(nullptr), "one stream per host thread");

  // calls from four threads overlap: four threads doing K calls each take far less
  // than four times one thread doing K calls (one shared, synchronized stream would
  // serialize them)
  const auto la = on_gpu(randn({256, 1024}, 133)), lb = on_gpu(randn({1024, 256}, 134));
  const int calls = 200;
  auto wall = [&](int nthreads) {
    std::atomic<int> errors{0};
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; ++t)
      pool.emplace_back([&] {
        for (int i = 0; i < calls; ++i) {
          Tensor m;
          if (!run(gpu, desc(OpKind::kMatmul), {la, lb}, m).ok()) ++errors;
        }
      });
    for (auto& th : pool) th.join();
    check(errors.load() == 0, "overlap calls succeed");
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  };
  (void)wall(4);  // warm every thread's stream and allocations
  const double one = wall(1), four = wall(4);
  std::printf("concurrency: %d matmul [256,1024]x[1024,256] calls: 1 thread %.2f ms, 4 threads x %d calls %.2f ms "
              "(%.2fx the work in %.2fx the time)\n", calls, one, calls, four, 4.0, four / one);
  check(four < 3.0 * one, "four threads' calls overlap (wall < 3x one thread's)");
}

// A block returned to the pool from another thread is reused behind that thread's
// work: the owner's stream waits on the event recorded at the return.
void cross_thread_pool_contract(Backend& gpu, Backend& ref) {
  auto pool = std::make_shared<cuda::MemoryPool>(1 << 26, 16);
  check(pool->enter().ok(), "cross-thread pool enter");
  const auto a = randn({128, 64}, 141), b = randn({64, 96}, 142);
  Tensor made;
  check(run(gpu, desc(OpKind::kMatmul), {on_gpu(a), on_gpu(b)}, made).ok(), "pool matmul");
  const auto hits_before = pool->stats().hits;
  std::thread other([&] {
    Tensor scaled;
    (void)run(gpu, axis_op(OpKind::kSoftmax, -1), {made}, scaled);  // work on this thread's stream
    made = Tensor{};  // the last owner dies here: the block goes back from this thread
  });
  other.join();
  check(pool->stats().cached_blocks >= 1 && pool->stats().readiness_failures == 0,
        "block returned from another thread is cached with its event");
  Tensor again;
  check(run(gpu, desc(OpKind::kMatmul), {on_gpu(a), on_gpu(b)}, again).ok(), "pool matmul again");
  check(pool->stats().hits > hits_before, "the returned block is reused");
  Tensor r;
  check(run(ref, desc(OpKind::kMatmul), {cpu::to_core_tensor(a), cpu::to_core_tensor(b)}, r).ok(), "reference matmul");
  check(close(download(again), cpu::from_core_tensor(r), 1e-4, 1e-4), "result in the reused block");
  again = Tensor{};
  check(pool->exit().ok() && pool->stats().in_use_bytes == 0, "cross-thread pool exit");
}
}  // namespace

int main() {
  if (!cuda::available()) {
    std::printf("no sm_100 GPU: skipped\n");
    return 77;
  }
  cuda::CudaBackend gpu;
  cpu::CpuBackend ref;
  check(gpu.name() == "cuda", "backend name");
  std::vector<Case> cases;
  // matmul: reference test shapes, batched broadcast, and sizes that take the tcgen05 path
  for (auto [a, b] : std::vector<std::pair<Shape, Shape>>{
           {{2, 3}, {3, 4}}, {{15, 17}, {17, 31}}, {{65, 129}, {129, 67}}, {{3}, {3}}, {{2, 3, 4}, {4}},
           {{2, 1, 3, 4}, {1, 5, 4, 6}}, {{2, 17, 19}, {1, 19, 33}}, {{256, 512}, {512, 384}},
           {{3, 200, 160}, {160, 300}}, {{0, 3}, {3, 4}}, {{3, 0}, {0, 4}}})
    cases.push_back({"matmul", desc(OpKind::kMatmul), {randn(a, 11), randn(b, 12)}, 1e-4, 1e-4});
  // reductions: one axis, multi-axis, full; float32 and int32
  for (auto k : {OpKind::kSum, OpKind::kMax, OpKind::kMean}) {
    for (std::int64_t ax : {0, 1, -1}) cases.push_back({"axis", axis_op(k, ax), {randn({7, 300}, 21)}, 1e-5, 1e-5});
    cases.push_back({"row65536", axis_op(k, -1), {randn({2, 3, 65536}, 22)}, 0, 0});  // bit-exact order
    cases.push_back({"axes", axes_op(k, {0, 2}), {randn({4, 5, 6}, 23)}, 1e-5, 1e-5});
    cases.push_back({"full", axes_op(k, {0, 1}), {randn({512, 1025}, 24)}, 1e-5, 1e-5, k != OpKind::kMax});
    if (k != OpKind::kMean) {
      cases.push_back({"i32 axis", axis_op(k, 1), {randi({9, 777}, 25)}, 0, 0});
      cases.push_back({"i32 full", axes_op(k, {0, 1}), {randi({300, 1000}, 26)}, 0, 0});
    }
  }
  cases.push_back({"mean int32 rejected", axis_op(OpKind::kMean, 0), {randi({4}, 27)}, 0, 0});
  for (auto k : {OpKind::kMin, OpKind::kArgmax}) {
    cases.push_back({"math axis", axes_op(k, {1}), {randn({5, 3000}, 31)}, 0, 0});
    cases.push_back({"math full", axes_op(k, {0, 1}), {randn({64, 4100}, 32)}, 0, 0});
    cases.push_back({"math i32", axes_op(k, {0}), {randi({6, 9}, 33)}, 0, 0});
  }
  {
    OpDesc clip = desc(OpKind::kClip);
    std::vector<float> lo{0.0f}, hi{INFINITY};
    cases.push_back({"relu = clip(lower=0)", clip,
                     {randn({33, 7}, 34), cpu::CpuTensor(Shape{}, lo), cpu::CpuTensor(Shape{}, hi)}, 0, 0});
  }
  for (auto k : {OpKind::kSoftmax, OpKind::kRmsNorm, OpKind::kLayerNorm}) {
    for (auto s : std::vector<Shape>{{16, 4096}, {4, 300}, {3, 33}})
      cases.push_back({"row op", axis_op(k, -1), {randn(s, 41, 3.0f)}, 1e-5, 1e-5});
    cases.push_back({"row op axis 0", axis_op(k, 0), {randn({50, 3}, 42)}, 1e-5, 1e-5});
  }
  {
    OpDesc aff = axis_op(OpKind::kAffineLayerNorm, -1);
    aff.has_weight = aff.has_bias = true;
    cases.push_back({"affine layernorm", aff, {randn({8, 1024}, 51, 3.0f), randn({1024}, 52), randn({1024}, 53)}, 1e-5, 1e-5});
    OpDesc rms = axis_op(OpKind::kAffineRmsNorm, -1);
    rms.has_weight = true;
    cases.push_back({"affine rmsnorm", rms, {randn({8, 1024}, 54, 3.0f), randn({1024}, 55)}, 1e-5, 1e-5});
  }
  for (auto k : {OpKind::kExp, OpKind::kGelu, OpKind::kSilu})
    cases.push_back({"unary", desc(k), {randn({1000}, 61, 3.0f)}, 1e-6, 1e-6});
  for (auto k : {OpKind::kAdd, OpKind::kSubtract, OpKind::kMultiply, OpKind::kDivide}) {
    cases.push_back({"binary bcast", desc(k), {randn({64, 37}, 71), randn({37}, 72)}, 0, 0});
    cases.push_back({"binary same", desc(k), {randn({5, 6}, 73), randn({5, 6}, 74)}, 0, 0});
  }
  cases.push_back({"int add wrap", desc(OpKind::kAdd), {randi({100}, 75), randi({100}, 76)}, 0, 0});
  cases.push_back({"linear", desc(OpKind::kLinear), {randn({256, 784}, 81), randn({512, 784}, 82, 0.03f), randn({512}, 83)},
                   1e-4, 1e-4});
  cases.push_back({"linear no bias", desc(OpKind::kLinear), {randn({3, 5}, 84), randn({7, 5}, 85)}, 1e-4, 1e-4});
  // attention composite and its softmax primitive (core/inference.cpp:56-160)
  {
    OpDesc att = desc(OpKind::kAttention);
    cases.push_back({"attention", att, {randn({2, 64, 32}, 101), randn({2, 300, 32}, 102), randn({2, 300, 16}, 103)},
                     2e-4, 2e-5});
    cases.push_back({"attention tensor path", att,
                     {randn({4, 256, 64}, 104), randn({4, 1024, 64}, 105), randn({4, 1024, 64}, 106)}, 2e-4, 2e-5});
    OpDesc causal = att;
    causal.causal = true;
    cases.push_back({"attention causal bool mask", causal,
                     {randn({2, 40, 16}, 107), randn({1, 50, 16}, 108), randn({2, 50, 8}, 109), randb({40, 50}, 110)},
                     2e-4, 2e-5});
    OpDesc scaled = att;
    scaled.attention_scale = 0.3;
    cases.push_back({"attention additive mask", scaled,
                     {randn({2, 1, 3, 4}, 111), randn({1, 3, 5, 4}, 112), randn({2, 3, 5, 2}, 113), randn({3, 5}, 114)},
                     2e-4, 2e-5});
    cases.push_back({"attention empty keys", att, {randn({3, 4}, 115), randn({0, 4}, 116), randn({0, 2}, 117)}, 0, 0});
    OpDesc sm = desc(OpKind::kAttentionSoftmax);
    sm.attention_shape = Shape{2, 5, 600};
    sm.attention_scale = 0.7;
    sm.causal = true;
    cases.push_back({"attention softmax", sm, {randn({2, 5, 600}, 118, 4.0f), randn({600}, 119)}, 1e-5, 1e-7});
    OpDesc bad = att;
    cases.push_back({"attention feature mismatch", bad, {randn({3, 4}, 120), randn({5, 3}, 121), randn({5, 2}, 122)}, 0, 0});
  }
  // the rest of the reference CUDA backend's primitives (tensor_ops.cu)
  {
    for (auto k : {OpKind::kNegate, OpKind::kAddScalar, OpKind::kSubtractScalar, OpKind::kMultiplyScalar,
                   OpKind::kDivideScalar}) {
      for (bool left : {false, true}) {
        OpDesc op = desc(k);
        op.scalar_value = 0.3;
        op.scalar_left = left;
        cases.push_back({"scalar f32", op, {specials(131)}, 0, 0});
        op.scalar_value = -7;
        cases.push_back({"scalar i32", op, {randi({1000}, 132)}, 0, 0});
        op.scalar_value = 2.5;
        cases.push_back({"scalar i32 fractional rejected", op, {randi({10}, 133)}, 0, 0});
      }
    }
    cases.push_back({"log", desc(OpKind::kLog), {specials(134)}, 1.2e-7, 0});
    cases.push_back({"sqrt", desc(OpKind::kSqrt), {specials(135)}, 0, 0});
    cases.push_back({"abs f32", desc(OpKind::kAbs), {specials(136)}, 0, 0});
    {
      std::vector<std::int32_t> w{INT32_MIN, -1, 0, 1, INT32_MAX, -5};
      cases.push_back({"abs i32 wrap", desc(OpKind::kAbs), {cpu::CpuTensor(Shape{6}, w)}, 0, 0});
    }
    cases.push_back({"log i32 rejected", desc(OpKind::kLog), {randi({8}, 137)}, 0, 0});
    for (auto [from, to] : std::vector<std::pair<DType, DType>>{
             {DType::kInt32, DType::kFloat32}, {DType::kFloat32, DType::kBool}, {DType::kBool, DType::kFloat32},
             {DType::kInt32, DType::kBool}, {DType::kBool, DType::kInt32}, {DType::kFloat32, DType::kFloat32},
             {DType::kBool, DType::kBool}}) {
      OpDesc op = desc(OpKind::kCast);
      op.target_dtype = to;
      const auto in = from == DType::kFloat32 ? specials(138) : from == DType::kInt32 ? randi({3, 70}, 139) : randb({3, 70}, 140);
      cases.push_back({"cast", op, {in}, 0, 0});
    }
    {
      OpDesc op = desc(OpKind::kCast);
      op.target_dtype = DType::kInt32;
      cases.push_back({"cast f32->i32", op, {randn({5, 77}, 141, 1e6f)}, 0, 0});
      cases.push_back({"cast f32->i32 out of range rejected", op, {specials(142)}, 0, 0});
    }
    for (auto axes : std::vector<Shape>{{1, 0}, {0, 2, 1}, {2, 0, 1}, {1, 2, 0}}) {
      OpDesc op = desc(OpKind::kTranspose);
      op.axes = axes;
      const Shape shape = axes.size() == 2 ? Shape{300, 77} : Shape{6, 130, 70};
      cases.push_back({"transpose", op, {randn(shape, 143)}, 0, 0});
      cases.push_back({"transpose bool", op, {randb(shape, 144)}, 0, 0});
    }
    {
      OpDesc op = desc(OpKind::kSlice);
      op.slice_starts = {1, 0, 5};
      op.slice_steps = {2, 1, 3};
      op.slice_shape = {3, 9, 20};
      cases.push_back({"slice", op, {randn({7, 9, 70}, 145)}, 0, 0});
      cases.push_back({"slice i32", op, {randi({7, 9, 70}, 146)}, 0, 0});
    }
    for (std::int64_t axis : {0, 1, -1}) {
      OpDesc op = desc(OpKind::kConcat);
      op.axis = axis;
      const auto a = axis == 0 ? Shape{3, 8, 12} : axis == 1 ? Shape{4, 5, 12} : Shape{4, 8, 5};
      const auto b = axis == 0 ? Shape{2, 8, 12} : axis == 1 ? Shape{4, 3, 12} : Shape{4, 8, 16};
      cases.push_back({"concat", op, {randn(a, 147), randn(b, 148), randn(a, 149)}, 0, 0});
      cases.push_back({"concat bool", op, {randb(a, 150), randb(b, 151)}, 0, 0});
    }
    {
      OpDesc op = desc(OpKind::kConcat);
      op.axis = 0;
      cases.push_back({"concat dtype mismatch", op, {randn({2, 3}, 152), randi({2, 3}, 153)}, 0, 0});
    }
    for (auto k : {OpKind::kEqual, OpKind::kNotEqual, OpKind::kLess, OpKind::kLessEqual, OpKind::kGreater,
                   OpKind::kGreaterEqual}) {
      cases.push_back({"compare f32", desc(k), {randk({40, 33}, 154, 7), randk({33}, 155, 7)}, 0, 0});
      cases.push_back({"compare specials", desc(k), {specials(156), specials(157)}, 0, 0});
      cases.push_back({"compare i32", desc(k), {randi({5, 1, 9}, 158), randi({7, 9}, 159)}, 0, 0});
      cases.push_back({"compare bool", desc(k), {randb({6, 10}, 160), randb({6, 10}, 161)}, 0, 0});
    }
    for (auto k : {OpKind::kLogicalAnd, OpKind::kLogicalOr, OpKind::kLogicalXor})
      cases.push_back({"logical", desc(k), {randb({8, 1, 50}, 162), randb({3, 50}, 163)}, 0, 0});
    cases.push_back({"logical not", desc(OpKind::kLogicalNot), {randb({300}, 164)}, 0, 0});
    cases.push_back({"logical on f32 rejected", desc(OpKind::kLogicalAnd), {randn({3}, 165), randn({3}, 166)}, 0, 0});
    cases.push_back({"where f32", desc(OpKind::kWhere), {randb({4, 1}, 167), specials(168), randn({64}, 170)}, 0, 0});
    cases.push_back({"where i32", desc(OpKind::kWhere), {randb({5, 7}, 171), randi({5, 7}, 172), randi({1, 7}, 173)}, 0, 0});
    cases.push_back({"where bool", desc(OpKind::kWhere), {randb({9}, 174), randb({9}, 175), randb({9}, 176)}, 0, 0});
    for (auto k : {OpKind::kAny, OpKind::kAll}) {
      cases.push_back({"bool reduce axis", axis_op(k, 1), {randb({7, 100, 3}, 177)}, 0, 0});
      cases.push_back({"bool reduce axes", axes_op(k, {0, 2}), {randb({7, 100, 3}, 178)}, 0, 0});
      cases.push_back({"bool reduce all axes", axes_op(k, {0, 1, 2}), {randb({7, 100, 3}, 179)}, 0, 0});
      cases.push_back({"bool reduce f32 rejected", axis_op(k, 0), {randn({4}, 180)}, 0, 0});
    }
    cases.push_back({"masked select rows", desc(OpKind::kMaskedSelect), {randn({50, 7, 3}, 181), randb({50}, 182)}, 0, 0});
    cases.push_back({"masked select elements", desc(OpKind::kMaskedSelect),
                     {randi({300, 41}, 183), randb({300, 41}, 184)}, 0, 0});
    cases.push_back({"masked select many tiles", desc(OpKind::kMaskedSelect),
                     {randn({20000}, 185), randb({20000}, 186)}, 0, 0});
    cases.push_back({"masked select bool", desc(OpKind::kMaskedSelect), {randb({64, 2}, 187), randb({64}, 188)}, 0, 0});
    for (bool largest : {true, false}) {
      for (bool sorted : {true, false}) {
        OpDesc op = desc(OpKind::kTopK);
        op.k = 5;
        op.largest = largest;
        op.sorted = sorted;
        op.axis = -1;
        cases.push_back({"topk ties", op, {randk({6, 40}, 189, 9)}, 0, 0});
        cases.push_back({"topk specials", op, {specials(190)}, 0, 0});
        op.axis = 0;
        cases.push_back({"topk axis 0", op, {randn({33, 4, 6}, 191)}, 0, 0});
        op.k = 33;
        cases.push_back({"topk k = axis", op, {randi({33, 5}, 192)}, 0, 0});
      }
    }
    {
      OpDesc op = desc(OpKind::kTopK);
      op.k = 0;
      op.axis = 1;
      cases.push_back({"topk k = 0", op, {randn({3, 9}, 193)}, 0, 0});
      op.k = 10;
      cases.push_back({"topk k too large rejected", op, {randn({3, 9}, 194)}, 0, 0});
    }
    cases.push_back({"embedding", desc(OpKind::kEmbedding), {indices_i32({4, 33}, 195, 500), randn({500, 64}, 196)}, 0, 0});
    cases.push_back({"embedding odd width", desc(OpKind::kEmbedding), {indices_i32({70}, 197, 9), randn({9, 7}, 198)}, 0, 0});
    cases.push_back({"embedding out of range rejected", desc(OpKind::kEmbedding),
                     {indices_i32({10}, 199, 20, true), randn({20, 8}, 200)}, 0, 0});
  }
  for (const auto& c : cases) compare(gpu, ref, c);

  // fill descriptor
  {
    OpDesc f = desc(OpKind::kFill);
    f.scalar_value = 2.5;
    Tensor d{DType::kFloat32, {3, 5}, contiguous_strides({3, 5}), Device{"cuda", 0}, nullptr, 0};
    std::vector<Tensor> outputs{d};
    BackendExecution e{BackendOpClass::kPrimitive, f, {}, outputs, std::nullopt, std::nullopt, {}};
    auto st = gpu.execute(e);
    check(st.ok(), "fill: " + st.message());
    if (st.ok()) {
      auto h = download(outputs[0]);
      bool ok = true;
      for (float v : h.float_data()) ok = ok && v == 2.5f;
      check(ok, "fill values");
    }
  }
  error_contract(gpu);
  pool_contract();
  surface_contract();
  compiled_kernel_contract();
  profiling_contract(gpu);
  concurrency_contract(gpu, ref);
  cross_thread_pool_contract(gpu, ref);
  // the same ops inside a real stream-ordered pool scope
  {
    auto pool = std::make_shared<cuda::MemoryPool>(1 << 28, 64);
    check(pool->enter().ok(), "real pool enter");
    for (int i = 0; i < 3; ++i)
      compare(gpu, ref, {"matmul in pool", desc(OpKind::kMatmul), {randn({256, 300}, 91), randn({300, 260}, 92)}, 1e-4, 1e-4});
    check(pool->stats().hits > 0, "pool reuses blocks across calls");
    check(pool->exit().ok(), "real pool exit");
  }
  // multi-device: a second GPU when present
  if (cuda::device_count() > 1) {
    compare(gpu, ref, {"matmul dev1", desc(OpKind::kMatmul), {randn({256, 512}, 93), randn({512, 384}, 94)}, 1e-4, 1e-4}, 1);
    compare(gpu, ref, {"sum dev1", axes_op(OpKind::kSum, {0, 1}), {randi({700, 999}, 95)}, 0, 0}, 1);
  }
  std::printf("%zu parity cases, %d failures\n", cases.size(), failures);
  return failures ? 1 : 0;
}
