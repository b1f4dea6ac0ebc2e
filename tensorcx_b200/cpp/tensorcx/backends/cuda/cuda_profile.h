// Profiling records of the sm100 backend, written into the tensor.cx core profiler
// (core/profiling.h: ProfileScope host spans, reserve/finish_device_profile device
// slots). The record names and categories are the reference backend's
// (cuda_backend.cpp:291 "execute" dispatch span, cuda_profiling.h:23-77 launch
// intervals, cuda_memory_pool.cpp:55,103 pool spans), so cx.profile() reports read the
// same. With no profile active on the thread nothing is created or timed.
#pragma once

#include <cuda_runtime_api.h>

#include <cmath>
#include <optional>
#include <string>

#include "tensorcx/core/expected.h"
#include "tensorcx/core/profiling.h"

namespace tensorcx::cuda {

// One launch of the backend: a host span of category compute_sync named `name` that
// covers the launch and its completion wait, and, when the active profile times the
// device, a device interval of the same name bracketed by two CUDA events on the
// launching stream. complete() records the end event, synchronizes the stream (the
// backend's calls are synchronous) and fills the device slot; it returns the launch's
// own status, or the wait's error.
class ProfiledLaunch {
 public:
  ProfiledLaunch(const char* name, cudaStream_t stream) noexcept
      : host_(ProfileCategory::kCompute, name, "cuda"), stream_(stream), token_(reserve_device_profile(name, "cuda")) {
    if (!token_) return;
    if (cudaEventCreate(&start_) != cudaSuccess || cudaEventCreate(&stop_) != cudaSuccess ||
        cudaEventRecord(start_, stream_) != cudaSuccess) {
      cudaGetLastError();
      error_ = "event_setup_failed";
    }
  }
  ~ProfiledLaunch() noexcept { settle(std::nullopt, error_ ? error_ : "incomplete"); }
  ProfiledLaunch(const ProfiledLaunch&) = delete;
  ProfiledLaunch& operator=(const ProfiledLaunch&) = delete;

  Status complete(Status launched) noexcept {
    if (!launched.ok()) {
      settle(std::nullopt, "operation_failed");
      return launched;
    }
    const bool timed = token_ && !error_;
    if (timed && cudaEventRecord(stop_, stream_) != cudaSuccess) {
      cudaGetLastError();
      error_ = "record_stop_failed";
    }
    cudaError_t waited;
    {
      ProfileScope wait(ProfileCategory::kSynchronize, "cudaStreamSynchronize", "cuda");
      waited = cudaStreamSynchronize(stream_);
    }
    if (waited != cudaSuccess) {
      const char* text = cudaGetErrorString(waited);
      cudaGetLastError();
      settle(std::nullopt, "operation_failed");
      return Status(StatusCode::kInternal, std::string("CUDA launch completion: ") + text);
    }
    std::optional<float> ms;
    if (token_ && !error_) {
      float v = 0.0f;
      if (cudaEventElapsedTime(&v, start_, stop_) == cudaSuccess && std::isfinite(v) && v >= 0) ms = v;
      else {
        cudaGetLastError();
        error_ = "elapsed_failed";
      }
    }
    settle(ms, error_);
    return launched;
  }

 private:
  void settle(std::optional<float> ms, const char* error) noexcept {
    if (start_) (void)cudaEventDestroy(start_);
    if (stop_) (void)cudaEventDestroy(stop_);
    start_ = stop_ = nullptr;
    if (token_) finish_device_profile(token_, error ? std::nullopt : ms, error);
    token_ = {};
  }

  ProfileScope host_;
  cudaStream_t stream_;
  DeviceProfileToken token_;
  cudaEvent_t start_{}, stop_{};
  const char* error_{};
};

}  // namespace tensorcx::cuda
