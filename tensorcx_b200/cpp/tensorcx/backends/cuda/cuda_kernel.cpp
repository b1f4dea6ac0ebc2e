// Compiled-kernel entries of the sm100 backend: unavailable by design (the backend
// serves the primitive hot path; DSL-compiled PTX is not loaded).
#include "tensorcx/backends/cuda/cuda_kernel.h"

namespace tensorcx::cuda {
namespace {
Status unavailable() {
  return Status(StatusCode::kUnavailable,
                "compiled kernels are not supported by the sm100 backend (it serves the primitive hot path)");
}
}  // namespace

std::string kernel_manifest(const KernelSignature& signature, const std::string& operation,
                            bool write_per_thread_no_output_read) {
  return "kinds=" + signature.kinds + ";operation=" + operation + ";output=" +
         std::to_string(signature.output_index) + ";guard=" + std::to_string(signature.guard_index) +
         ";per_thread_write=" + (write_per_thread_no_output_read ? "1" : "0");
}

Status compiled_kernel_support() { return unavailable(); }

CudaKernelModule::~CudaKernelModule() = default;

Expected<std::shared_ptr<CudaKernelModule>> CudaKernelModule::load(const std::string&, const std::string&,
                                                                   KernelSignature) {
  return unavailable();
}

Expected<CudaTensor> CudaKernelModule::launch(std::span<const KernelArgument>, const Tensor&, std::uint32_t,
                                              std::uint32_t) const {
  return unavailable();
}

Status execute_compiled_kernel(const BackendExecution&) { return unavailable(); }

Expected<CudaTensor> launch_compiled_kernel(const std::shared_ptr<CudaKernelModule>&, std::span<const KernelArgument>,
                                            std::uint32_t, std::uint32_t) {
  return unavailable();
}

}  // namespace tensorcx::cuda
