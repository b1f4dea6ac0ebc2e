#include "tensorcx/backends/cuda/cuda_device.h"

#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

namespace tensorcx::cuda {
namespace {
constexpr int kMaxDevices = 64;

// Once per device: memory freed back to the device's default stream-ordered pool
// stays reserved there, so repeated same-size allocations cost no driver call.
std::once_flag g_pool_once[kMaxDevices];

void keep_freed_memory_reserved(int device) {
  std::call_once(g_pool_once[device], [device] {
    cudaMemPool_t pool = nullptr;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
      std::uint64_t threshold = UINT64_MAX;
      (void)cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    }
    cudaGetLastError();
  });
}

// One non-blocking stream per device for each host thread: concurrent executes from
// different threads (the bindings release the GIL around them) run on different
// streams, and each waits only for its own work. Destroyed when the thread ends
// (work still queued on a destroyed stream completes first).
struct ThreadStreams {
  std::vector<cudaStream_t> by_device;
  ~ThreadStreams() {
    for (cudaStream_t s : by_device)
      if (s) (void)cudaStreamDestroy(s);
  }
};

Expected<cudaStream_t> stream_for(int device) {
  if (device < 0 || device >= kMaxDevices) return Status(StatusCode::kInvalidArgument, "CUDA device index out of range");
  thread_local ThreadStreams streams;
  if (static_cast<std::size_t>(device) >= streams.by_device.size()) streams.by_device.resize(device + 1, nullptr);
  cudaStream_t& s = streams.by_device[device];
  if (!s) {
    keep_freed_memory_reserved(device);
    auto status = runtime_status(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "CUDA stream creation");
    if (!status.ok()) {
      s = nullptr;
      return status;
    }
  }
  return s;
}
}  // namespace

Status runtime_status(cudaError_t error, const char* operation) {
  if (error == cudaSuccess) return Status::Ok();
  cudaGetLastError();  // never leave a sticky error behind for unrelated calls
  return Status(StatusCode::kInternal, std::string(operation) + ": " + cudaGetErrorString(error));
}

int device_count() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

DeviceScope::DeviceScope(int device) : device_(device) {
  if (device < 0 || device >= device_count()) {
    status_ = Status(StatusCode::kInvalidArgument, "CUDA device index " + std::to_string(device) + " is not available");
    return;
  }
  if (cudaGetDevice(&previous_) != cudaSuccess) {
    cudaGetLastError();
    previous_ = -1;
  }
  status_ = runtime_status(cudaSetDevice(device), "cudaSetDevice");
  if (!status_.ok()) return;
  auto s = stream_for(device);
  if (!s) { status_ = s.status(); return; }
  stream_ = s.value();
}

DeviceScope::~DeviceScope() {
  if (previous_ >= 0 && previous_ != device_) (void)cudaSetDevice(previous_);
}

cudaStream_t current_device_stream() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) {
    cudaGetLastError();
    d = 0;
  }
  auto s = stream_for(d);
  return s ? s.value() : nullptr;
}

}  // namespace tensorcx::cuda
