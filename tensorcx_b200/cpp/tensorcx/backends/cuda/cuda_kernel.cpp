// Compiled (generated) kernels on the sm100 backend: caller-provided PTX for sm_100a,
// loaded with the driver's JIT, launched on the calling thread's stream.
//
// Behaviour follows the reference loader (cpp/tensorcx/backends/cuda/cuda_kernel.cpp:
// 47-300, docs/CUDA_OUTPUT_COPY_ELISION.md): a module holds exactly one entry
// (tensorcx_{add,sub,mul,expr}_v1) with four parameters (three float32 tensors and
// one uint32 guard equal to the thread count); the PTX starts with a manifest line
// naming the producer contract. Each launch returns a fresh private result tensor:
//
//  * v1 manifests (and v2 launches that do not cover every element) start the result
//    as a copy of the output template, and inputs that alias the template read that
//    copy;
//  * a v2 manifest (write-per-thread-no-output-read: every thread stores its element
//    once and never reads the output) with thread_count == numel(output) skips the
//    template copy; inputs that alias the template keep reading the template.
//
// B200 form: the private result comes from the stream-ordered allocator (the thread's
// memory pool when one is entered), the template copy is a stream-ordered
// device-to-device copy on the same stream as the launch (no wait of its own), and
// the one completion wait is the launch's. The target line must be sm_100a.
#include "tensorcx/backends/cuda/cuda_kernel.h"

#include <algorithm>
#include <array>
#include <atomic>
#include <mutex>
#include <regex>
#include <unordered_map>

#include "tensorcx/backends/cuda/cuda_context.h"
#include "tensorcx/backends/cuda/cuda_device.h"
#include "tensorcx/backends/cuda/cuda_external_storage.h"
#include "tensorcx/backends/cuda/cuda_profile.h"

namespace tensorcx::cuda {
namespace {

Status invalid(std::string message) { return {StatusCode::kInvalidArgument, std::move(message)}; }

template <typename F>
F driver_entry(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return reinterpret_cast<F>(p);
}

// Driver calls of the module path, resolved at run time (the runtime loads the driver).
struct ModuleApi {
  decltype(&cuModuleLoadDataEx) load = driver_entry<decltype(&cuModuleLoadDataEx)>("cuModuleLoadDataEx");
  decltype(&cuModuleUnload) unload = driver_entry<decltype(&cuModuleUnload)>("cuModuleUnload");
  decltype(&cuModuleGetFunction) function = driver_entry<decltype(&cuModuleGetFunction)>("cuModuleGetFunction");
  decltype(&cuModuleGetFunctionCount) count =
      driver_entry<decltype(&cuModuleGetFunctionCount)>("cuModuleGetFunctionCount");
  decltype(&cuFuncGetParamInfo) param = driver_entry<decltype(&cuFuncGetParamInfo)>("cuFuncGetParamInfo");
  decltype(&cuFuncGetAttribute) attribute = driver_entry<decltype(&cuFuncGetAttribute)>("cuFuncGetAttribute");
  decltype(&cuLaunchKernel) launch = driver_entry<decltype(&cuLaunchKernel)>("cuLaunchKernel");
  bool ok() const { return load && unload && function && count && param && attribute && launch; }
};
const ModuleApi& api() {
  static const ModuleApi a;
  return a;
}

// Loaded modules by artifact id; the id is what a BackendExecution carries.
std::mutex g_registry_mutex;
std::unordered_map<std::string, std::weak_ptr<CudaKernelModule>> g_registry;
std::atomic<std::uint64_t> g_next_artifact{1};

Expected<std::shared_ptr<CudaKernelModule>> find_module(const std::string& id) {
  std::lock_guard lock(g_registry_mutex);
  if (const auto it = g_registry.find(id); it != g_registry.end())
    if (auto module = it->second.lock()) return module;
  return invalid("unknown or expired CUDA kernel artifact");
}

// Three float32 tensor slots and one uint32 guard; the output is a tensor slot.
bool well_formed(const KernelSignature& s) {
  if (s.kinds.size() != 4 || s.output_index >= 4 || s.guard_index >= 4) return false;
  if (std::count(s.kinds.begin(), s.kinds.end(), 't') != 3 || std::count(s.kinds.begin(), s.kinds.end(), 'u') != 1)
    return false;
  return s.kinds[s.output_index] == 't' && s.kinds[s.guard_index] == 'u';
}

const char* operation_of(const std::string& entry) {
  if (entry == "tensorcx_add_v1") return "add";
  if (entry == "tensorcx_sub_v1") return "sub";
  if (entry == "tensorcx_mul_v1") return "mul";
  if (entry == "tensorcx_expr_v1") return "expr";
  return nullptr;
}

// The directive occurs on exactly one line of the PTX.
bool single_directive(const std::string& ptx, const char* pattern) {
  const std::regex re(pattern);
  return std::distance(std::sregex_iterator(ptx.begin(), ptx.end(), re), std::sregex_iterator()) == 1;
}

}  // namespace

std::string kernel_manifest(const KernelSignature& signature, const std::string& operation,
                            bool write_per_thread_no_output_read) {
  std::string m = write_per_thread_no_output_read ? "tensorcx.cuda.v2" : "tensorcx.cuda.v1";
  m += "|linux-x86_64|sm_100a|" + operation + "-f32-v1|" + signature.kinds + "|" +
       std::to_string(signature.output_index) + "|" + std::to_string(signature.guard_index);
  if (write_per_thread_no_output_read) m += "|write-per-thread-no-output-read-v1";
  return m;
}

Status compiled_kernel_support() {
#if !defined(__linux__) || !defined(__x86_64__)
  return {StatusCode::kUnavailable, "compiled CUDA kernels need Linux x86_64"};
#else
  if (!api().ok()) return {StatusCode::kUnavailable, "CUDA driver module entry points are unavailable"};
  DeviceScope scope(0);
  if (!scope.ready()) return scope.status();
  cudaDeviceProp prop{};
  if (auto st = runtime_status(cudaGetDeviceProperties(&prop, 0), "cudaGetDeviceProperties"); !st.ok()) return st;
  int driver = 0;
  (void)cudaDriverGetVersion(&driver);
  if (prop.major != 10 || prop.minor != 0 || driver < 12080)
    return {StatusCode::kUnavailable, "compiled CUDA kernels need an sm_100 device and a CUDA 12.8+ driver"};
  return Status::Ok();
#endif
}

struct CudaKernelModule::Impl {
  std::shared_ptr<PrimaryContext> context;
  int device{0};
  CUmodule module{};
  CUfunction function{};
  int max_block{}, max_grid{};
  bool write_per_thread{false};
  ~Impl() {
    if (!module || !current_process()) return;
    ContextScope scope(context);
    if (scope.ready()) (void)api().unload(module);
  }
};

CudaKernelModule::CudaKernelModule() : impl_(std::make_unique<Impl>()) {}

CudaKernelModule::~CudaKernelModule() {
  if (id_.empty() || !current_process()) return;
  std::lock_guard lock(g_registry_mutex);
  g_registry.erase(id_);
}

Expected<std::shared_ptr<CudaKernelModule>> CudaKernelModule::load(const std::string& ptx, const std::string& entry,
                                                                   KernelSignature signature) {
  try {
    if (!well_formed(signature)) return invalid("invalid CUDA kernel signature");
    const char* operation = operation_of(entry);
    if (!operation) return invalid("unsupported CUDA entry point");
    const bool v2 = ptx.starts_with("// " + kernel_manifest(signature, operation, true) + "\n");
    const bool v1 = ptx.starts_with("// " + kernel_manifest(signature, operation, false) + "\n");
    if (ptx.size() > (1u << 20) || ptx.find('\0') != std::string::npos || (!v1 && !v2) ||
        !single_directive(ptx, R"((^|\n)\.version 8\.[6-9]\r?\n)") ||
        !single_directive(ptx, R"((^|\n)\.target sm_100a\r?\n)") ||
        !single_directive(ptx, R"((^|\n)\.address_size 64\r?\n)"))
      return invalid("CUDA PTX target/ABI manifest mismatch");
    if (auto st = compiled_kernel_support(); !st.ok()) return st;
    int device = 0;
    if (auto st = runtime_status(cudaGetDevice(&device), "cudaGetDevice"); !st.ok()) return st;
    ContextScope scope;
    if (!scope.ready()) return scope.status();
    std::shared_ptr<CudaKernelModule> module(new CudaKernelModule);
    Impl& m = *module->impl_;
    m.context = scope.owner();
    m.device = device;
    m.write_per_thread = v2;
    std::array<char, 4096> log{};
    CUjit_option options[] = {CU_JIT_ERROR_LOG_BUFFER, CU_JIT_ERROR_LOG_BUFFER_SIZE_BYTES};
    void* values[] = {log.data(), reinterpret_cast<void*>(static_cast<std::uintptr_t>(log.size()))};
    if (const CUresult rc = api().load(&m.module, ptx.c_str(), 2, options, values); rc != CUDA_SUCCESS) {
      m.module = nullptr;
      log.back() = '\0';
      return invalid(driver_status(rc, "CUDA PTX JIT").message() + ": " + log.data());
    }
    unsigned functions = 0;
    if (auto st = driver_status(api().count(&functions, m.module), "CUDA module function count"); !st.ok()) return st;
    if (functions != 1) return invalid("CUDA module must contain exactly one kernel");
    if (auto st = driver_status(api().function(&m.function, m.module, entry.c_str()), "CUDA entry lookup"); !st.ok())
      return st;
    // parameter layout: 8-byte pointers and 4-byte guards at their natural offsets
    std::size_t offset = 0;
    for (unsigned i = 0; i < 4; ++i) {
      const std::size_t size = signature.kinds[i] == 't' ? 8 : 4;
      offset = (offset + size - 1) / size * size;
      std::size_t got_offset = 0, got_size = 0;
      if (api().param(m.function, i, &got_offset, &got_size) != CUDA_SUCCESS || got_offset != offset ||
          got_size != size)
        return invalid("CUDA entry parameter ABI mismatch");
      offset += size;
    }
    std::size_t extra_offset = 0, extra_size = 0;
    if (api().param(m.function, 4, &extra_offset, &extra_size) != CUDA_ERROR_INVALID_VALUE)
      return invalid("CUDA entry parameter count mismatch");
    int function_block = 0;
    if (auto st = driver_status(api().attribute(&function_block, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, m.function),
                                "CUDA function block limit");
        !st.ok())
      return st;
    cudaDeviceProp prop{};
    if (auto st = runtime_status(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties"); !st.ok())
      return st;
    m.max_block = std::min({prop.maxThreadsPerBlock, prop.maxThreadsDim[0], function_block});
    m.max_grid = prop.maxGridSize[0];
    module->entry_ = entry;
    module->signature_ = std::move(signature);
    module->id_ = "sm100-kernel-" + std::to_string(g_next_artifact.fetch_add(1));
    {
      std::lock_guard lock(g_registry_mutex);
      g_registry.emplace(module->id_, module);
    }
    return module;
  } catch (const std::exception& error) {
    return Status(StatusCode::kInternal, error.what());
  }
}

Expected<CudaTensor> CudaKernelModule::launch(std::span<const KernelArgument> arguments, const Tensor& output,
                                              std::uint32_t threads, std::uint32_t block) const {
  try {
    if (!current_process()) return Status(StatusCode::kUnavailable, "CUDA kernels need a fresh process after fork");
    BackendExecution described;
    described.inputs = std::span(&output, 1);
    described.kernel_arguments = arguments;
    ExternalLease lease(external_owners(described));
    if (!lease.status().ok()) return lease.status();
    auto run = [&]() -> Expected<CudaTensor> {
      const Impl& m = *impl_;
      if (arguments.size() != 4) return invalid("CUDA kernel argument count mismatch");
      if (block == 0 || block > static_cast<std::uint32_t>(m.max_block)) return invalid("CUDA block size exceeds limits");
      const std::uint64_t blocks = threads ? (static_cast<std::uint64_t>(threads) + block - 1) / block : 0;
      if (blocks > static_cast<std::uint64_t>(m.max_grid)) return invalid("CUDA grid size exceeds limits");
      auto templ = from_core_tensor(output);
      if (!templ) return templ.status();
      const auto elements = static_cast<std::uint64_t>(numel(output.shape));
      if (output.dtype != DType::kFloat32 || threads > elements) return invalid("CUDA kernel output dtype/size mismatch");
      if (templ.value().buffer()->device() != m.device) return invalid("CUDA kernel output is on another device");
      const auto& out_buffer = *templ.value().buffer();
      for (std::size_t i = 0; i < 4; ++i) {
        const KernelArgument& arg = arguments[i];
        if (signature_.kinds[i] == 'u') {
          if (arg.kind != KernelArgumentKind::kUInt32 || arg.tensor || arg.uint32_value != threads)
            return invalid("CUDA guard argument must equal thread_count");
          continue;
        }
        if (arg.kind != KernelArgumentKind::kTensor || !arg.tensor) return invalid("CUDA tensor argument kind mismatch");
        auto t = from_core_tensor(*arg.tensor);
        if (!t) return t.status();
        if (t.value().dtype() != DType::kFloat32 || t.value().shape() != output.shape ||
            t.value().buffer()->device() != m.device)
          return invalid("CUDA tensor dtype/shape/context mismatch");
        if (t.value().buffer()->storage_relation(out_buffer) == StorageRelation::kPartialOverlap)
          return invalid("CUDA kernel arguments have unsupported partial storage overlap");
        if (i == signature_.output_index && t.value().buffer().get() != &out_buffer)
          return invalid("CUDA output argument mismatch");
      }
      DeviceScope scope(m.device);
      if (!scope.ready()) return scope.status();
      ContextScope context(m.context);
      if (!context.ready()) return context.status();
      auto result = CudaBuffer::create(DType::kFloat32, output.shape, m.device);
      if (!result) return result.status();
      const bool full_write = m.write_per_thread && threads != 0 && threads == elements;
      if (!full_write && result.value()->nbytes()) {
        ProfileScope span(ProfileCategory::kCopy, "device_to_device", "cuda", result.value()->nbytes());
        if (auto st = runtime_status(cudaMemcpyAsync(result.value()->data(), out_buffer.data(), result.value()->nbytes(),
                                                     cudaMemcpyDeviceToDevice, scope.stream()),
                                     "CUDA output template copy");
            !st.ok())
          return st;
      }
      std::array<CUdeviceptr, 4> pointers{};
      std::array<std::uint32_t, 4> guards{};
      std::array<void*, 4> params{};
      for (std::size_t i = 0; i < 4; ++i) {
        if (signature_.kinds[i] == 'u') {
          guards[i] = arguments[i].uint32_value;
          params[i] = &guards[i];
          continue;
        }
        const auto* buffer = static_cast<const CudaBuffer*>(arguments[i].tensor->buffer.get());
        void* data = buffer->data();
        // the output slot always writes the private result; on the copy path an input
        // that aliases the template reads the copy (its initialized contents), on the
        // full-write path it keeps reading the template
        if (i == signature_.output_index ||
            (!full_write && buffer->storage_relation(out_buffer) == StorageRelation::kSameRange))
          data = result.value()->data();
        pointers[i] = reinterpret_cast<CUdeviceptr>(data);
        params[i] = &pointers[i];
      }
      if (threads) {
        ProfiledLaunch profiled("generated_kernel", scope.stream());
        const Status launched =
            driver_status(api().launch(m.function, static_cast<unsigned>(blocks), 1, 1, block, 1, 1, 0,
                                       reinterpret_cast<CUstream>(scope.stream()), params.data(), nullptr),
                          "CUDA generated kernel launch");
        if (auto st = profiled.complete(launched); !st.ok()) return st;
      } else if (!full_write && result.value()->nbytes()) {
        ProfileScope wait(ProfileCategory::kSynchronize, "cudaStreamSynchronize", "cuda");
        if (auto st = runtime_status(cudaStreamSynchronize(scope.stream()), "CUDA output template copy"); !st.ok())
          return st;
      }
      return CudaTensor(DType::kFloat32, output.shape, result.move_value());
    };
    auto launched = run();
    if (auto done = lease.finish(); !done.ok()) return done;
    return launched;
  } catch (const std::invalid_argument& error) {
    return invalid(error.what());
  } catch (const std::exception& error) {
    return Status(StatusCode::kInternal, error.what());
  }
}

Status execute_compiled_kernel(const BackendExecution& e) {
  if (auto st = validate_kernel_execution_contract(e); !st.ok()) return st;
  if (e.outputs.size() != 1 || e.compilation_target->artifact_kind != KernelArtifactKind::kBinary)
    return invalid("unsupported CUDA kernel artifact/output");
  const LaunchConfig& l = *e.launch;
  if (l.grid_y != 1 || l.grid_z != 1 || l.threads_per_group_y != 1 || l.threads_per_group_z != 1)
    return invalid("CUDA kernel requires one-dimensional launch");
  auto module = find_module(e.compilation_target->artifact);
  if (!module) return module.status();
  if (e.compilation_target->entry_point != module.value()->entry_point())
    return invalid("CUDA kernel entry does not match artifact");
  auto result = module.value()->launch(e.kernel_arguments, e.outputs[0], l.grid_x, l.threads_per_group_x);
  if (!result) return result.status();
  e.outputs[0] = to_core_tensor(result.value());  // published only on success
  return Status::Ok();
}

Expected<CudaTensor> launch_compiled_kernel(const std::shared_ptr<CudaKernelModule>& module,
                                            std::span<const KernelArgument> arguments, std::uint32_t threads,
                                            std::uint32_t block) {
  if (!module) return invalid("missing CUDA module");
  const auto out = module->signature().output_index;
  if (arguments.size() != 4 || !arguments[out].tensor || arguments[out].kind != KernelArgumentKind::kTensor)
    return invalid("missing CUDA output");
  std::array<Tensor, 1> outputs{*arguments[out].tensor};
  if (!threads) return module->launch(arguments, outputs[0], threads, block);  // zero work: no launch record
  BackendExecution e{BackendOpClass::kKernel, {}, {}, outputs, LaunchConfig{threads, 1, 1, block, 1, 1},
                     CompilationTarget{KernelArtifactKind::kBinary, module->artifact_id(), module->entry_point()},
                     arguments};
  CudaBackend backend;
  if (auto st = backend.execute(e); !st.ok()) return st;
  return from_core_tensor(outputs[0]);
}

}  // namespace tensorcx::cuda
