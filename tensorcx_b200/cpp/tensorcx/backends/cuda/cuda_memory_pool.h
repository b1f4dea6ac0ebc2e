// Memory pool of the sm100 CUDA backend.
//
// Interface kept from the reference (cpp/tensorcx/backends/cuda/cuda_memory_pool.h:12-54,
// bound by bindings/python_module.cpp:1152-1183): the PoolStats fields, the injectable
// PoolRuntime, and a single-use, thread-scoped MemoryPool with enter / exit / trim /
// stats. Behind it, a stream-ordered design:
//
//  * Blocks come from cudaMallocAsync on the calling thread's stream for the current
//    device and go back with cudaFreeAsync (the device's default memory pool keeps the
//    bytes reserved, so a later cudaMallocAsync of them costs no driver call).
//  * Idle blocks are kept per (device, byte size) as LIFO stacks: a hit returns the
//    most recently released block of exactly that size on that device (warm in L2,
//    never another GPU's memory).
//  * Every thread has its own stream per device (cuda_device.h), so work from
//    different threads overlaps. A block released on the pool's owning thread is
//    reused on that same stream, where stream order already puts the new work after
//    the old. A block released from another thread carries an event recorded on that
//    thread's stream; the next user's stream waits on it (a device-side wait, no host
//    synchronization), and so does a stream-ordered free of it.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <thread>
#include <utility>
#include <vector>

#include "tensorcx/core/expected.h"

namespace tensorcx::cuda {

struct PoolStats {
  std::size_t max_cached_bytes{}, max_cached_blocks{}, cached_bytes{}, cached_blocks{};
  std::size_t in_use_bytes{}, peak_in_use_bytes{}, peak_cached_bytes{};
  std::uint64_t hits{}, misses{}, allocation_calls{}, free_calls{}, allocation_failures{},
      oom_retries{}, uncached_returns{}, readiness_failures{}, free_failures{}, failed_free_bytes{};
  bool active{};
};

// Injectable runtime calls (allocation, free, clearing a recoverable error), so OOM
// and free-failure paths are tested on the host without exhausting a shared GPU.
struct PoolRuntime {
  cudaError_t (*allocate)(void**, std::size_t);
  cudaError_t (*free)(void*);
  cudaError_t (*clear_error)();
};
// Production runtime: cudaMallocAsync / cudaFreeAsync on the calling thread's stream
// for the current device.
PoolRuntime default_pool_runtime();

class MemoryPool : public std::enable_shared_from_this<MemoryPool> {
 public:
  MemoryPool(std::size_t bytes, std::size_t blocks, PoolRuntime runtime = default_pool_runtime());
  ~MemoryPool();
  Status enter();
  Status exit();
  Status trim();
  PoolStats stats() const;
  // Backend use, on the owning thread inside the scope, with the target device current.
  Expected<void*> allocate(std::size_t bytes);
  // Any thread, with the block's device current. `reusable` false (e.g. storage that
  // was exported to a foreign consumer) frees the block instead of keeping it.
  // `context_ready` is kept for the reference's signature; blocks are freed
  // stream-ordered on the releasing thread's stream, which needs no extra context.
  void release(void* pointer, std::size_t bytes, bool reusable, bool context_ready = true) noexcept;
  void close_noexcept() noexcept;

 private:
  struct IdleBlock {
    void* pointer;
    cudaEvent_t ready;  // end of its last use on another thread's stream; null otherwise
  };
  using SizeKey = std::pair<int, std::size_t>;  // (device, bytes)

  Status close();
  void* take_idle_locked(int device, std::size_t bytes);
  bool has_idle_locked(int device) const;
  Status drop_idle_locked(int device, bool every_device);
  cudaError_t free_block_locked(void* pointer, cudaEvent_t ready, std::size_t bytes);

  mutable std::mutex mutex_;
  PoolRuntime runtime_;
  PoolStats stats_;
  std::map<SizeKey, std::vector<IdleBlock>> idle_;
  std::thread::id owner_;
  bool entered_once_{};
};

// The pool entered on the calling thread, if any.
std::shared_ptr<MemoryPool> active_memory_pool();

}  // namespace tensorcx::cuda
