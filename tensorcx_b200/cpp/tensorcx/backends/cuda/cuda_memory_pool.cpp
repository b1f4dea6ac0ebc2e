// Stream-ordered rebuild of the reference memory pool (cuda_memory_pool.cpp:21-163):
// same scope rules (thread-local, single-use, not nested), same exact-size block cache
// with byte and block caps, same OOM drain-and-retry-once and failure accounting. The
// production runtime allocates with cudaMallocAsync and frees with cudaFreeAsync on the
// device stream, so a released block is reusable immediately (no readiness query).
#include "tensorcx/backends/cuda/cuda_memory_pool.h"

#include <algorithm>
#include <stdexcept>

#include "tensorcx/backends/cuda/cuda_device.h"

namespace tensorcx::cuda {
namespace {
thread_local MemoryPool* active{};
struct Holder {
  std::shared_ptr<MemoryPool> pool;
  ~Holder() { active = nullptr; if (pool) pool->close_noexcept(); }
};
Holder& holder() { static thread_local Holder value; return value; }
Status invalid(const char* message) { return {StatusCode::kInvalidArgument, message}; }

cudaError_t async_allocate(void** pointer, std::size_t bytes) {
  return cudaMallocAsync(pointer, bytes, current_device_stream());
}
cudaError_t async_free(void* pointer) { return cudaFreeAsync(pointer, current_device_stream()); }
}  // namespace

PoolRuntime default_pool_runtime() { return {async_allocate, async_free, cudaGetLastError}; }

MemoryPool::MemoryPool(std::size_t bytes, std::size_t blocks, PoolRuntime runtime) : runtime_(runtime) {
  if (!blocks || blocks > 4096) throw std::invalid_argument("max_cached_blocks must be in [1, 4096]");
  if (!runtime.allocate || !runtime.free || !runtime.clear_error) throw std::invalid_argument("invalid pool runtime");
  stats_.max_cached_bytes = bytes;
  stats_.max_cached_blocks = blocks;
  cached_.reserve(blocks);
}

MemoryPool::~MemoryPool() { close_noexcept(); }

Status MemoryPool::enter() {
  std::lock_guard lock(mutex_);
  if (active) return invalid("memory pools cannot be nested on the same thread");
  if (used_) return invalid("memory pool contexts are single-use");
  holder().pool = shared_from_this();
  used_ = true;
  stats_.active = true;
  active = this;
  return Status::Ok();
}

Status MemoryPool::exit() {
  if (active != this) return invalid("memory pool must exit on its owning thread");
  active = nullptr;
  auto keep_alive = std::move(holder().pool);
  return close();
}

std::shared_ptr<MemoryPool> active_memory_pool() { return active ? active->shared_from_this() : nullptr; }

Expected<void*> MemoryPool::allocate(std::size_t bytes) {
  std::lock_guard lock(mutex_);
  if (active != this || !stats_.active || !bytes) return invalid("inactive pool or zero-byte allocation");
  const auto found = std::find_if(cached_.begin(), cached_.end(), [=](const Block& b) { return b.bytes == bytes; });
  void* pointer{};
  if (found != cached_.end()) {
    pointer = found->pointer;
    stats_.cached_bytes -= bytes;
    cached_.erase(found);
    ++stats_.hits;
  } else {
    ++stats_.misses;
    ++stats_.allocation_calls;
    auto error = runtime_.allocate(&pointer, bytes);
    if (error == cudaErrorMemoryAllocation && !cached_.empty()) {
      // Only a recoverable OOM is retried (after returning every cached block).
      const auto pending = runtime_.clear_error();
      if (pending != cudaSuccess && pending != cudaErrorMemoryAllocation) {
        ++stats_.allocation_failures;
        return runtime_status(pending, "CUDA pool allocation prior error");
      }
      const auto drained = trim_locked();
      if (!drained.ok()) { ++stats_.allocation_failures; return drained; }
      ++stats_.oom_retries;
      ++stats_.allocation_calls;
      error = runtime_.allocate(&pointer, bytes);
    }
    if (error != cudaSuccess) {
      ++stats_.allocation_failures;
      return runtime_status(error, "CUDA pool allocation");
    }
  }
  stats_.cached_blocks = cached_.size();
  stats_.in_use_bytes += bytes;
  stats_.peak_in_use_bytes = std::max(stats_.peak_in_use_bytes, stats_.in_use_bytes);
  return pointer;
}

cudaError_t MemoryPool::free_locked(void* pointer, std::size_t bytes) {
  ++stats_.free_calls;
  const auto error = runtime_.free(pointer);
  if (error != cudaSuccess) { ++stats_.free_failures; stats_.failed_free_bytes += bytes; }
  return error;
}

void MemoryPool::release(void* pointer, std::size_t bytes, bool reusable, bool /*context_ready*/) noexcept {
  try {
    std::lock_guard lock(mutex_);
    stats_.in_use_bytes -= bytes;
    if (stats_.active && reusable && cached_.size() < stats_.max_cached_blocks &&
        bytes <= stats_.max_cached_bytes - stats_.cached_bytes) {
      // Stream order makes the block safe to hand out again right away: work that
      // reuses it is queued behind every use of its previous owner.
      cached_.push_back({pointer, bytes});
      stats_.cached_bytes += bytes;
      stats_.cached_blocks = cached_.size();
      stats_.peak_cached_bytes = std::max(stats_.peak_cached_bytes, stats_.cached_bytes);
      return;
    }
    ++stats_.uncached_returns;
    (void)free_locked(pointer, bytes);
  } catch (...) {
    (void)runtime_.free(pointer);
  }
}

Status MemoryPool::trim_locked() {
  Status first = Status::Ok();
  while (!cached_.empty()) {
    const auto block = cached_.back();
    cached_.pop_back();
    stats_.cached_bytes -= block.bytes;
    stats_.cached_blocks = cached_.size();
    const auto error = free_locked(block.pointer, block.bytes);
    // ownership is given up once a free was attempted: never retry it
    if (first.ok() && error != cudaSuccess) first = runtime_status(error, "CUDA pool trim");
  }
  return first;
}

Status MemoryPool::trim() {
  if (active != this) return invalid("memory pool trim requires its active owning thread");
  std::lock_guard lock(mutex_);
  return trim_locked();
}

Status MemoryPool::close() {
  std::lock_guard lock(mutex_);
  stats_.active = false;
  return trim_locked();
}

void MemoryPool::close_noexcept() noexcept {
  try { (void)close(); } catch (...) {}
}

PoolStats MemoryPool::stats() const {
  std::lock_guard lock(mutex_);
  return stats_;
}

}  // namespace tensorcx::cuda
