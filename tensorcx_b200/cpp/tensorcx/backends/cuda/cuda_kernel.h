// Compiled-kernel surface of the reference backend (cpp/tensorcx/backends/cuda/
// cuda_kernel.h:7-37), kept so the bindings that load DSL-compiled PTX link unchanged.
// Compiled kernels are not part of this backend's data path: every entry reports
// kUnavailable with a message saying so, and modules are never created.
#pragma once

#include <memory>
#include <span>
#include <string>

#include "tensorcx/backends/cuda/cuda_backend.h"

namespace tensorcx::cuda {

struct KernelSignature {
  std::string kinds;
  std::uint32_t output_index{0}, guard_index{0};
};

// A textual description of a compiled kernel's interface (argument kinds, operation,
// output and guard positions), stable for equal inputs.
std::string kernel_manifest(const KernelSignature& signature, const std::string& operation = "add",
                            bool write_per_thread_no_output_read = false);
Status compiled_kernel_support();

class CudaKernelModule {
 public:
  ~CudaKernelModule();
  CudaKernelModule(const CudaKernelModule&) = delete;
  CudaKernelModule& operator=(const CudaKernelModule&) = delete;
  static Expected<std::shared_ptr<CudaKernelModule>> load(const std::string& ptx, const std::string& entry,
                                                          KernelSignature signature);
  const std::string& artifact_id() const { return id_; }
  const std::string& entry_point() const { return entry_; }
  const KernelSignature& signature() const { return signature_; }
  Expected<CudaTensor> launch(std::span<const KernelArgument> arguments, const Tensor& output,
                              std::uint32_t threads, std::uint32_t block) const;

 private:
  CudaKernelModule() = default;
  KernelSignature signature_;
  std::string id_, entry_;
};

Status execute_compiled_kernel(const BackendExecution& execution);
Expected<CudaTensor> launch_compiled_kernel(const std::shared_ptr<CudaKernelModule>& module,
                                            std::span<const KernelArgument> arguments, std::uint32_t threads,
                                            std::uint32_t block);

}  // namespace tensorcx::cuda
