// Per-device execution state of the sm100 backend: one non-blocking stream per device
// (0..N-1) for each host thread, created on first use, plus the device's default
// stream-ordered memory pool with a release threshold that keeps freed memory
// reserved in the driver.
// The reference pins everything to device 0 and the legacy stream
// (cuda_context.cpp:37-47); here a tensor's Device.index selects the GPU.
#pragma once

#include <cuda_runtime_api.h>

#include "tensorcx/core/expected.h"

namespace tensorcx::cuda {

Status runtime_status(cudaError_t error, const char* operation);

// Makes `device` current on the calling thread for its lifetime (restoring the previous
// device) and exposes the device's stream.
class DeviceScope {
 public:
  explicit DeviceScope(int device);
  ~DeviceScope();
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;
  const Status& status() const { return status_; }
  bool ready() const { return status_.ok(); }
  int device() const { return device_; }
  cudaStream_t stream() const { return stream_; }

 private:
  int device_{0}, previous_{-1};
  cudaStream_t stream_{nullptr};
  Status status_;
};

int device_count();
// The calling thread's stream for its current device (creating it on first use).
cudaStream_t current_device_stream();

}  // namespace tensorcx::cuda
