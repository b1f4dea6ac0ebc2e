// Stream-ordered memory pool of the sm100 backend (design in cuda_memory_pool.h).
//
// Observable contract kept from the reference pool (docs/CUDA_MEMORY_POOL.md): exact
// byte-size reuse, the byte and block caps on idle storage (a return that does not fit
// is freed rather than evicting others), single-use scopes entered on one thread and
// never nested, an allocation that runs out of memory while idle blocks exist hands
// them back and is retried exactly once, and a free that was attempted gives the block
// up even when it reports an error.
#include "tensorcx/backends/cuda/cuda_memory_pool.h"

#include <algorithm>
#include <stdexcept>

#include "tensorcx/backends/cuda/cuda_device.h"
#include "tensorcx/core/profiling.h"

namespace tensorcx::cuda {
namespace {

// The pool entered on this thread. A plain pointer (trivially destructible), so that a
// buffer destroyed late in the thread's teardown can still read it after the slot
// below is gone.
thread_local MemoryPool* t_entered = nullptr;

// Holds the entered pool alive for the thread, and closes a pool that was entered but
// never exited when the thread ends (its idle blocks are freed, later returns of its
// live blocks are freed directly).
struct ThreadPoolSlot {
  std::shared_ptr<MemoryPool> pool;
  ~ThreadPoolSlot() {
    t_entered = nullptr;
    if (pool) pool->close_noexcept();
  }
};
ThreadPoolSlot& thread_slot() {
  thread_local ThreadPoolSlot slot;
  return slot;
}

Status invalid(const char* message) { return {StatusCode::kInvalidArgument, message}; }

int current_device() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    cudaGetLastError();
    device = 0;
  }
  return device;
}

cudaError_t stream_ordered_allocate(void** pointer, std::size_t bytes) {
  return cudaMallocAsync(pointer, bytes, current_device_stream());
}
cudaError_t stream_ordered_free(void* pointer) { return cudaFreeAsync(pointer, current_device_stream()); }

// The calling thread's stream for the current device waits for `ready` (device side;
// on the host only when the wait cannot be queued), then the event is released.
void wait_for(cudaEvent_t ready) {
  if (!ready) return;
  if (cudaStreamWaitEvent(current_device_stream(), ready, 0) != cudaSuccess) {
    cudaGetLastError();
    (void)cudaEventSynchronize(ready);
    cudaGetLastError();
  }
  (void)cudaEventDestroy(ready);  // the queued wait keeps what it needs
}

}  // namespace

PoolRuntime default_pool_runtime() { return {stream_ordered_allocate, stream_ordered_free, cudaGetLastError}; }

MemoryPool::MemoryPool(std::size_t bytes, std::size_t blocks, PoolRuntime runtime) : runtime_(runtime) {
  if (blocks == 0 || blocks > 4096) throw std::invalid_argument("max_cached_blocks must be in [1, 4096]");
  if (!runtime.allocate || !runtime.free || !runtime.clear_error)
    throw std::invalid_argument("memory pool runtime needs allocate, free and clear_error");
  stats_.max_cached_bytes = bytes;
  stats_.max_cached_blocks = blocks;
}

MemoryPool::~MemoryPool() { close_noexcept(); }

Status MemoryPool::enter() {
  std::lock_guard lock(mutex_);
  if (t_entered) return invalid("memory pools cannot be nested on one thread");
  if (entered_once_) return invalid("memory pool scopes are single-use");
  entered_once_ = true;
  owner_ = std::this_thread::get_id();
  stats_.active = true;
  thread_slot().pool = shared_from_this();
  t_entered = this;
  return Status::Ok();
}

Status MemoryPool::exit() {
  if (t_entered != this) return invalid("memory pool must exit on its owning thread");
  t_entered = nullptr;
  const auto keep_alive = std::move(thread_slot().pool);  // lives until close() is done
  return close();
}

std::shared_ptr<MemoryPool> active_memory_pool() { return t_entered ? t_entered->shared_from_this() : nullptr; }

void* MemoryPool::take_idle_locked(int device, std::size_t bytes) {
  const auto found = idle_.find({device, bytes});
  if (found == idle_.end()) return nullptr;
  const IdleBlock block = found->second.back();
  found->second.pop_back();
  if (found->second.empty()) idle_.erase(found);
  stats_.cached_bytes -= bytes;
  stats_.cached_blocks -= 1;
  wait_for(block.ready);  // last used on another thread's stream
  return block.pointer;
}

bool MemoryPool::has_idle_locked(int device) const {
  const auto first = idle_.lower_bound({device, 0});
  return first != idle_.end() && first->first.first == device;
}

cudaError_t MemoryPool::free_block_locked(void* pointer, cudaEvent_t ready, std::size_t bytes) {
  wait_for(ready);
  ++stats_.free_calls;
  const cudaError_t rc = runtime_.free(pointer);
  if (rc != cudaSuccess) {
    ++stats_.free_failures;
    stats_.failed_free_bytes += bytes;
  }
  return rc;
}

Status MemoryPool::drop_idle_locked(int device, bool every_device) {
  Status first = Status::Ok();
  for (auto it = every_device ? idle_.begin() : idle_.lower_bound({device, 0}); it != idle_.end();) {
    const auto [dev, bytes] = it->first;
    if (!every_device && dev != device) break;
    DeviceScope on(dev);  // stream-ordered frees on this thread's stream of that device
    for (const IdleBlock& block : it->second) {
      stats_.cached_bytes -= bytes;
      stats_.cached_blocks -= 1;
      const cudaError_t rc = on.ready() ? free_block_locked(block.pointer, block.ready, bytes) : cudaErrorInvalidDevice;
      if (!on.ready()) {
        ++stats_.free_failures;
        stats_.failed_free_bytes += bytes;
      }
      if (rc != cudaSuccess && first.ok()) first = runtime_status(rc, "CUDA pool free of idle blocks");
    }
    it = idle_.erase(it);
  }
  return first;
}

Expected<void*> MemoryPool::allocate(std::size_t bytes) {
  ProfileScope span(ProfileCategory::kMemoryPool, "pool_acquire", "cuda", bytes);
  std::lock_guard lock(mutex_);
  if (t_entered != this || !stats_.active) return invalid("memory pool allocation outside its active scope");
  if (bytes == 0) return invalid("memory pool allocation of zero bytes");
  const int device = current_device();
  void* pointer = take_idle_locked(device, bytes);
  if (pointer) {
    ++stats_.hits;
  } else {
    ++stats_.misses;
    ++stats_.allocation_calls;
    cudaError_t rc = runtime_.allocate(&pointer, bytes);
    if (rc == cudaErrorMemoryAllocation && has_idle_locked(device)) {
      // Out of memory while this device has idle blocks: hand them back (stream
      // ordered, so the retry on the same stream can reuse their bytes) and try once
      // more. Only the out-of-memory error itself is cleared.
      const cudaError_t pending = runtime_.clear_error();
      if (pending != cudaSuccess && pending != cudaErrorMemoryAllocation) {
        ++stats_.allocation_failures;
        return runtime_status(pending, "CUDA error pending before the pool's out-of-memory retry");
      }
      if (auto dropped = drop_idle_locked(device, false); !dropped.ok()) {
        ++stats_.allocation_failures;
        return dropped;
      }
      ++stats_.oom_retries;
      ++stats_.allocation_calls;
      rc = runtime_.allocate(&pointer, bytes);
    }
    if (rc != cudaSuccess) {
      ++stats_.allocation_failures;
      return runtime_status(rc, "CUDA pool allocation");
    }
  }
  stats_.in_use_bytes += bytes;
  stats_.peak_in_use_bytes = std::max(stats_.peak_in_use_bytes, stats_.in_use_bytes);
  return pointer;
}

void MemoryPool::release(void* pointer, std::size_t bytes, bool reusable, bool /*context_ready*/) noexcept {
  try {
    ProfileScope span(ProfileCategory::kMemoryPool, "pool_release", "cuda", bytes);
    std::lock_guard lock(mutex_);
    stats_.in_use_bytes -= bytes;
    const bool fits = stats_.cached_blocks < stats_.max_cached_blocks &&
                      bytes <= stats_.max_cached_bytes - stats_.cached_bytes;
    if (stats_.active && reusable && fits) {
      cudaEvent_t ready = nullptr;
      bool marked = true;
      if (std::this_thread::get_id() != owner_) {
        // returned from another thread: mark the end of its use on this thread's stream
        marked = cudaEventCreateWithFlags(&ready, cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventRecord(ready, current_device_stream()) == cudaSuccess;
        if (!marked) {
          cudaGetLastError();
          if (ready) (void)cudaEventDestroy(ready);
          ready = nullptr;
          ++stats_.readiness_failures;
        }
      }
      if (marked) {
        idle_[{current_device(), bytes}].push_back({pointer, ready});
        stats_.cached_bytes += bytes;
        stats_.cached_blocks += 1;
        stats_.peak_cached_bytes = std::max(stats_.peak_cached_bytes, stats_.cached_bytes);
        return;
      }
    }
    ++stats_.uncached_returns;
    if (!reusable) {
      // storage a foreign consumer may still read on a stream this backend does not
      // track: wait for the device before the free
      (void)cudaDeviceSynchronize();
      cudaGetLastError();
    }
    (void)free_block_locked(pointer, nullptr, bytes);
  } catch (...) {
    (void)runtime_.free(pointer);
  }
}

Status MemoryPool::trim() {
  if (t_entered != this) return invalid("memory pool trim is only allowed on its active owning thread");
  std::lock_guard lock(mutex_);
  return drop_idle_locked(0, true);
}

Status MemoryPool::close() {
  std::lock_guard lock(mutex_);
  stats_.active = false;
  return drop_idle_locked(0, true);
}

void MemoryPool::close_noexcept() noexcept {
  try {
    (void)close();
  } catch (...) {
  }
}

PoolStats MemoryPool::stats() const {
  std::lock_guard lock(mutex_);
  return stats_;
}

}  // namespace tensorcx::cuda
