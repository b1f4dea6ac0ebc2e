// C-ABI runtime entry points: error reporting, device checks, the device error word.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace tcx {
namespace {
thread_local std::string g_last_error;

struct TimerRecord {
  const char* name;
  cudaEvent_t start, stop;
};
struct TimerState {
  bool enabled = false;
  std::vector<TimerRecord> records;
};
thread_local TimerState g_timer;
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices];
std::once_flag g_sm_once[kMaxDevices];
}  // namespace

// Per-device error word written by kernels whose waits are bounded (a wait that
// runs out records its site here and returns instead of spinning forever).
__device__ int g_device_error;

void set_error(const std::string& message) { g_last_error = message; }
void clear_error() { g_last_error.clear(); }

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::call_once(g_sm_once[dev], [dev] {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  });
  return g_sm_count[dev];
}

TimedLaunch::TimedLaunch(const char* name, cudaStream_t stream) : name_(name), stream_(stream) {
  if (!g_timer.enabled) return;
  if (cudaEventCreate(&start_) != cudaSuccess || cudaEventRecord(start_, stream_) != cudaSuccess) {
    cudaGetLastError();
    start_ = nullptr;
  }
}

TimedLaunch::~TimedLaunch() {
  if (!start_) return;
  cudaEvent_t stop = nullptr;
  if (cudaEventCreate(&stop) == cudaSuccess && cudaEventRecord(stop, stream_) == cudaSuccess) {
    g_timer.records.push_back({name_, start_, stop});
  } else {
    cudaGetLastError();
    cudaEventDestroy(start_);
    if (stop) cudaEventDestroy(stop);
  }
}

int* device_error_word() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return static_cast<int*>(p);
}

}  // namespace tcx

extern "C" {

const char* tcx_sm100_last_error(void) { return tcx::g_last_error.c_str(); }

int tcx_sm100_abi_version(void) { return 1; }

int tcx_sm100_device_supported(int device) {
  cudaDeviceProp prop;
  const cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) {
    tcx::set_error(std::string("cudaGetDeviceProperties: ") + cudaGetErrorString(e));
    return TCX_UNAVAILABLE;
  }
  if (prop.major != 10 || prop.minor != 0) {
    tcx::set_error("tensorcx_b200 kernels are built for sm_100a (B200) only");
    return TCX_UNAVAILABLE;
  }
  return TCX_OK;
}

int tcx_sm100_timer_enable(int enable) {
  tcx::g_timer.enabled = enable != 0;
  return TCX_OK;
}

int tcx_sm100_timer_read(char* names, size_t names_bytes, int64_t* launches, double* total_ms,
                         int32_t capacity, int32_t* entries) {
  tcx::clear_error();
  std::vector<std::string> order;
  std::map<std::string, std::pair<int64_t, double>> sums;
  int status = TCX_OK;
  for (auto& r : tcx::g_timer.records) {
    float ms = 0.0f;
    if (cudaEventSynchronize(r.stop) != cudaSuccess || cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess) {
      tcx::set_error("timer event failed");
      status = TCX_INTERNAL;
      cudaGetLastError();
    }
    if (!sums.count(r.name)) order.push_back(r.name);
    auto& e = sums[r.name];
    e.first += 1;
    e.second += ms;
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  tcx::g_timer.records.clear();
  int32_t n = 0;
  size_t used = 0;
  for (const auto& name : order) {
    if (n >= capacity) break;
    const size_t len = std::min<size_t>(name.size(), 63);
    if (names && used + len + 1 <= names_bytes) {
      std::memcpy(names + used, name.data(), len);
      names[used + len] = '\0';
      used += len + 1;
    }
    if (launches) launches[n] = sums[name].first;
    if (total_ms) total_ms[n] = sums[name].second;
    ++n;
  }
  if (entries) *entries = n;
  return status;
}

int tcx_sm100_device_error(int device, int* code) {
  int previous = 0;
  if (cudaGetDevice(&previous) != cudaSuccess) return TCX_INTERNAL;
  if (cudaSetDevice(device) != cudaSuccess) return TCX_INTERNAL;
  int value = 0;
  const int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&value, tcx::g_device_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(tcx::g_device_error, &zero, sizeof(int));
  cudaSetDevice(previous);
  if (e != cudaSuccess) {
    tcx::set_error(std::string("device error word: ") + cudaGetErrorString(e));
    return TCX_INTERNAL;
  }
  if (code) *code = value;
  return TCX_OK;
}

}  // extern "C"
