// Host <-> device copies for pageable host memory through pinned staging.
//
// A copy from or to ordinary (pageable) host memory runs at the speed of the CUDA
// driver's own single-threaded staging (about 11 GB/s host to device and 21 GB/s back
// on a B200 host, against 55 GB/s for page-locked memory). These entries stage through
// a per-device ring of two page-locked 32 MiB slots instead: several host threads copy
// between the caller's buffer and one slot while the DMA engine moves the other, so
// the host side runs at memory bandwidth and overlaps the PCIe transfer. Page-locked
// caller buffers and small copies go straight to cudaMemcpyAsync. Both entries are
// synchronous, as the reference's from_cpu / to_cpu (cuda_backend.cpp:215-264).
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"

namespace tcx {
namespace {

constexpr size_t kSlotBytes = 32u << 20;
constexpr size_t kDirectBelow = 4u << 20;

// Persistent host workers for parallel memcpy (created once, never joined: they park
// on a condition variable between jobs and are reclaimed with the process).
class CopyPool {
 public:
  static CopyPool& get() {
    static CopyPool* pool = new CopyPool();
    return *pool;
  }

  // Copies n bytes with every worker plus the calling thread; returns when done.
  // One job at a time (callers on other devices wait here).
  void copy(void* dst, const void* src, size_t n) {
    std::lock_guard<std::mutex> job(job_mu_);
    const int parts = static_cast<int>(workers_.size()) + 1;
    if (n < (1u << 20) || parts == 1) {
      memcpy(dst, src, n);
      return;
    }
    const size_t step = ((n + parts - 1) / parts + 4095) & ~size_t(4095);
    {
      std::lock_guard<std::mutex> lock(mu_);
      dst_ = static_cast<char*>(dst);
      src_ = static_cast<const char*>(src);
      n_ = n;
      step_ = step;
      pending_ = parts - 1;
      ++generation_;
    }
    cv_.notify_all();
    piece(0);
    std::unique_lock<std::mutex> lock(mu_);
    done_.wait(lock, [&] { return pending_ == 0; });
  }

 private:
  CopyPool() {
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const int n = static_cast<int>(std::min(8u, std::max(1u, hw / 2))) - 1;
    for (int i = 0; i < n; ++i) workers_.emplace_back([this, i] { loop(i + 1); });
    for (auto& t : workers_) t.detach();
  }

  void piece(int k) {
    const size_t begin = std::min(n_, static_cast<size_t>(k) * step_);
    const size_t end = std::min(n_, begin + step_);
    if (end > begin) memcpy(dst_ + begin, src_ + begin, end - begin);
  }

  void loop(int k) {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lock(mu_);
        cv_.wait(lock, [&] { return generation_ != seen; });
        seen = generation_;
      }
      piece(k);
      {
        std::lock_guard<std::mutex> lock(mu_);
        if (--pending_ == 0) done_.notify_one();
      }
    }
  }

  std::vector<std::thread> workers_;
  std::mutex job_mu_, mu_;
  std::condition_variable cv_, done_;
  uint64_t generation_ = 0;
  int pending_ = 0;
  char* dst_ = nullptr;
  const char* src_ = nullptr;
  size_t n_ = 0, step_ = 0;
};

struct Stager {
  std::mutex mu;
  char* slot[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  bool ready = false;
};

Stager& stager(int device) {
  static Stager stagers[64];
  return stagers[device & 63];
}

int stage_init(Stager& st) {
  if (st.ready) return TCX_OK;
  for (int i = 0; i < 2; ++i) {
    if (cudaHostAlloc(reinterpret_cast<void**>(&st.slot[i]), kSlotBytes, cudaHostAllocPortable) != cudaSuccess ||
        cudaEventCreateWithFlags(&st.done[i], cudaEventDisableTiming) != cudaSuccess)
      return launch_status("pinned staging allocation");
  }
  st.ready = true;
  return TCX_OK;
}

bool page_locked(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();  // unregistered memory may report an error on some drivers
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

int fail(cudaError_t e, const char* what) {
  set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return TCX_INTERNAL;
}

// Host to device through the two slots: the host copy of chunk i+1 overlaps the DMA of chunk i.
int staged_to_device(cudaStream_t s, void* dst, const void* src, size_t bytes) {
  int device = 0;
  cudaGetDevice(&device);
  Stager& st = stager(device);
  std::lock_guard<std::mutex> lock(st.mu);
  if (int rc = stage_init(st)) return rc;
  const char* in = static_cast<const char*>(src);
  char* out = static_cast<char*>(dst);
  size_t i = 0;
  for (size_t off = 0; off < bytes; off += kSlotBytes, ++i) {
    const int k = static_cast<int>(i & 1);
    const size_t n = std::min(kSlotBytes, bytes - off);
    if (i >= 2)  // the DMA that last read this slot has finished
      if (cudaError_t e = cudaEventSynchronize(st.done[k])) return fail(e, "staging slot wait");
    CopyPool::get().copy(st.slot[k], in + off, n);
    if (cudaError_t e = cudaMemcpyAsync(out + off, st.slot[k], n, cudaMemcpyHostToDevice, s))
      return fail(e, "staged host to device copy");
    cudaEventRecord(st.done[k], s);
  }
  if (cudaError_t e = cudaStreamSynchronize(s)) return fail(e, "host to device synchronize");
  return TCX_OK;
}

// Device to host: two DMAs ahead of the host copies out of the slots.
int staged_to_host(cudaStream_t s, void* dst, const void* src, size_t bytes) {
  int device = 0;
  cudaGetDevice(&device);
  Stager& st = stager(device);
  std::lock_guard<std::mutex> lock(st.mu);
  if (int rc = stage_init(st)) return rc;
  const char* in = static_cast<const char*>(src);
  char* out = static_cast<char*>(dst);
  const size_t chunks = (bytes + kSlotBytes - 1) / kSlotBytes;
  auto issue = [&](size_t c) -> int {
    const int k = static_cast<int>(c & 1);
    const size_t off = c * kSlotBytes, n = std::min(kSlotBytes, bytes - off);
    if (cudaError_t e = cudaMemcpyAsync(st.slot[k], in + off, n, cudaMemcpyDeviceToHost, s))
      return fail(e, "staged device to host copy");
    cudaEventRecord(st.done[k], s);
    return TCX_OK;
  };
  for (size_t c = 0; c < std::min<size_t>(2, chunks); ++c)
    if (int rc = issue(c)) return rc;
  for (size_t c = 0; c < chunks; ++c) {
    const int k = static_cast<int>(c & 1);
    const size_t off = c * kSlotBytes, n = std::min(kSlotBytes, bytes - off);
    if (cudaError_t e = cudaEventSynchronize(st.done[k])) return fail(e, "staging slot wait");
    CopyPool::get().copy(out + off, st.slot[k], n);
    if (c + 2 < chunks)
      if (int rc = issue(c + 2)) return rc;
  }
  return TCX_OK;
}

}  // namespace
}  // namespace tcx

using namespace tcx;

extern "C" {

int tcx_sm100_copy_to_device(tcx_stream_t stream, void* dst, const void* src, size_t bytes) {
  clear_error();
  if (bytes == 0) return TCX_OK;
  if (!dst || !src) return invalid("missing copy buffer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (bytes < kDirectBelow || page_locked(src)) {
    if (cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s)) return fail(e, "host to device copy");
    if (cudaError_t e = cudaStreamSynchronize(s)) return fail(e, "host to device synchronize");
    return TCX_OK;
  }
  try {
    return staged_to_device(s, dst, src, bytes);
  } catch (const std::exception& e) {
    set_error(std::string("staged host to device copy: ") + e.what());
    return TCX_INTERNAL;
  }
}

int tcx_sm100_copy_to_host(tcx_stream_t stream, void* dst, const void* src, size_t bytes) {
  clear_error();
  if (bytes == 0) return TCX_OK;
  if (!dst || !src) return invalid("missing copy buffer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (bytes < kDirectBelow || page_locked(dst)) {
    if (cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s)) return fail(e, "device to host copy");
    if (cudaError_t e = cudaStreamSynchronize(s)) return fail(e, "device to host synchronize");
    return TCX_OK;
  }
  try {
    return staged_to_host(s, dst, src, bytes);
  } catch (const std::exception& e) {
    set_error(std::string("staged device to host copy: ") + e.what());
    return TCX_INTERNAL;
  }
}

}  // extern "C"
