// Compiled-kernel surface of the reference backend (cpp/tensorcx/backends/cuda/
// cuda_kernel.h:7-37), which the bindings that load generated PTX link against: PTX
// for sm_100a with a manifest line, one entry with three float32 tensor slots and a
// uint32 guard, launched on the calling thread's stream into a private result
// (the output template copy is skipped when the manifest promises a full per-thread
// write; see cuda_kernel.cpp).
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

// The manifest line a producer writes at the top of the PTX ("// " + manifest): the
// contract version (v2 = write-per-thread-no-output-read), platform, target, operation,
// argument kinds, output and guard positions.
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
  CudaKernelModule();
  struct Impl;
  std::unique_ptr<Impl> impl_;
  KernelSignature signature_;
  std::string id_, entry_;
};

Status execute_compiled_kernel(const BackendExecution& execution);
Expected<CudaTensor> launch_compiled_kernel(const std::shared_ptr<CudaKernelModule>& module,
                                            std::span<const KernelArgument> arguments, std::uint32_t threads,
                                            std::uint32_t block);

}  // namespace tensorcx::cuda
