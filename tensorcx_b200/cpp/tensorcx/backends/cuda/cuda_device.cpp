#include "tensorcx/backends/cuda/cuda_device.h"

#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

namespace tensorcx::cuda {
namespace {
std::mutex g_mutex;
std::vector<cudaStream_t> g_streams;

Expected<cudaStream_t> stream_for(int device) {
  std::lock_guard lock(g_mutex);
  if (device < 0) return Status(StatusCode::kInvalidArgument, "negative CUDA device index");
  if (static_cast<std::size_t>(device) >= g_streams.size()) g_streams.resize(device + 1, nullptr);
  if (!g_streams[device]) {
    cudaStream_t s = nullptr;
    auto status = runtime_status(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "CUDA stream creation");
    if (!status.ok()) return status;
    // Keep memory freed back to the device's stream-ordered pool cached in the
    // driver: repeated same-size allocations then cost no cudaMalloc.
    cudaMemPool_t pool = nullptr;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
      std::uint64_t threshold = UINT64_MAX;
      (void)cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    }
    cudaGetLastError();
    g_streams[device] = s;
  }
  return g_streams[device];
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
