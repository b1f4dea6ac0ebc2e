// Driver-context surface of the sm100 backend, as the reference declares it
// (cpp/tensorcx/backends/cuda/cuda_context.h:10-43): status mapping of runtime and
// driver errors, a retained primary context that is never reset (other users in the
// process may share it), and a scope that makes it current on the calling thread and
// restores whatever was current before. The compute path itself selects devices with
// DeviceScope (cuda_device.h); this class serves callers that work at the driver
// level (DLPack import, interop).
#pragma once

#include <cuda.h>
#include <cuda_runtime_api.h>

#include <memory>

#include "tensorcx/core/expected.h"

namespace tensorcx::cuda {

// False in a child process forked after the parent initialized CUDA: CUDA state does
// not survive fork, so such a child must not touch the inherited contexts.
bool current_process();
Status driver_status(CUresult error, const char* operation);
Status runtime_status(cudaError_t error, const char* operation);

class PrimaryContext {
 public:
  // Retains the primary context of the calling thread's current device.
  static Expected<std::shared_ptr<PrimaryContext>> acquire();
  ~PrimaryContext();
  PrimaryContext(const PrimaryContext&) = delete;
  PrimaryContext& operator=(const PrimaryContext&) = delete;
  CUcontext get() const { return context_; }
  CUdevice device() const { return device_; }

 private:
  PrimaryContext() = default;
  CUcontext context_{};
  CUdevice device_{};
};

// Pushes the owner's context on the calling thread for its lifetime (a foreign
// driver context that was current stays below it and is current again afterwards).
class ContextScope {
 public:
  ContextScope();  // the primary context of the current device
  explicit ContextScope(std::shared_ptr<PrimaryContext> owner);
  ~ContextScope();
  ContextScope(const ContextScope&) = delete;
  ContextScope& operator=(const ContextScope&) = delete;
  const Status& status() const { return status_; }
  bool ready() const { return status_.ok(); }
  const std::shared_ptr<PrimaryContext>& owner() const { return owner_; }

 private:
  std::shared_ptr<PrimaryContext> owner_;
  Status status_;
  bool pushed_{false};
  void push();
};

}  // namespace tensorcx::cuda
