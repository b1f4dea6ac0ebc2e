// Memory pool of the sm100 CUDA backend: the public surface of the reference's
// cpp/tensorcx/backends/cuda/cuda_memory_pool.h:12-54 (PoolStats fields, injectable
// PoolRuntime, single-use thread-scoped MemoryPool), rebuilt on stream-ordered
// allocation: blocks come from cudaMallocAsync and go back with cudaFreeAsync on the
// backend's per-device stream, so a cached block can be handed out again at once
// (stream order already separates its previous use from the next one).
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>
#include <memory>
#include <mutex>
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
// Stream-ordered production runtime: cudaMallocAsync / cudaFreeAsync on the calling
// thread's current device stream (cuda_device.h).
PoolRuntime default_pool_runtime();

class MemoryPool : public std::enable_shared_from_this<MemoryPool> {
 public:
  MemoryPool(std::size_t bytes, std::size_t blocks, PoolRuntime runtime = default_pool_runtime());
  ~MemoryPool();
  Status enter();
  Status exit();
  Status trim();
  PoolStats stats() const;
  Expected<void*> allocate(std::size_t bytes);
  // context_ready: the reference's flag that the pool's context is current (always true
  // here: blocks are freed stream-ordered on the backend's per-device stream).
  void release(void* pointer, std::size_t bytes, bool reusable, bool context_ready = true) noexcept;
  void close_noexcept() noexcept;

 private:
  struct Block { void* pointer; std::size_t bytes; };
  Status close();
  Status trim_locked();
  cudaError_t free_locked(void* pointer, std::size_t bytes);
  mutable std::mutex mutex_;
  PoolRuntime runtime_;
  PoolStats stats_;
  std::vector<Block> cached_;
  bool used_{};
};

// The pool entered on the calling thread, if any.
std::shared_ptr<MemoryPool> active_memory_pool();

}  // namespace tensorcx::cuda
