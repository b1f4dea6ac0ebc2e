// External-storage registry and lease of the sm100 backend.
#include "tensorcx/backends/cuda/cuda_external_storage.h"

#include <map>
#include <mutex>

#include "tensorcx/backends/cuda/cuda_backend.h"

namespace tensorcx::cuda {
namespace {
struct Registry {
  std::mutex mutex;
  std::map<std::uintptr_t, std::weak_ptr<ExternalStorage>> by_begin;
};
Registry& registry() {
  static Registry* r = new Registry();  // outlives static destruction order
  return *r;
}

std::vector<std::shared_ptr<StorageAccess>> accesses(const std::vector<std::shared_ptr<ExternalStorage>>& owners) {
  std::vector<std::shared_ptr<StorageAccess>> out;
  out.reserve(owners.size());
  for (const auto& o : owners)
    if (o) out.push_back(o->access());
  return out;
}
}  // namespace

void register_external_storage(const std::shared_ptr<ExternalStorage>& owner) {
  if (!owner) return;
  auto& r = registry();
  std::lock_guard<std::mutex> lock(r.mutex);
  r.by_begin[owner->begin()] = owner;
}

void unregister_external_storage(std::uintptr_t begin, const ExternalStorage* owner) noexcept {
  auto& r = registry();
  std::lock_guard<std::mutex> lock(r.mutex);
  auto it = r.by_begin.find(begin);
  if (it == r.by_begin.end()) return;
  auto live = it->second.lock();
  if (!live || live.get() == owner) r.by_begin.erase(it);
}

Expected<std::shared_ptr<ExternalStorage>> find_external_storage(void* data, std::size_t bytes) {
  const auto addr = reinterpret_cast<std::uintptr_t>(data);
  auto& r = registry();
  std::lock_guard<std::mutex> lock(r.mutex);
  auto it = r.by_begin.upper_bound(addr);
  if (it != r.by_begin.begin()) {
    --it;
    if (auto owner = it->second.lock()) {
      const std::uintptr_t begin = owner->begin();
      if (addr >= begin && addr - begin <= owner->mapped_bytes() && bytes <= owner->mapped_bytes() - (addr - begin))
        return owner;
    }
  }
  return Status(StatusCode::kInvalidArgument, "no registered external CUDA storage holds this range");
}

ExternalLease::ExternalLease(std::vector<std::shared_ptr<ExternalStorage>> owners)
    : owners_(std::move(owners)), lease_(accesses(owners_)) {}

Status ExternalLease::finish() {
  if (finished_) return completion_;
  finished_ = true;
  for (const auto& owner : owners_) {
    if (!owner) continue;
    if (auto st = owner->complete_cuda(); !st.ok() && completion_.ok()) completion_ = st;
  }
  return completion_;
}

ExternalLease::~ExternalLease() { (void)finish(); }

std::vector<std::shared_ptr<ExternalStorage>> external_owners(const BackendExecution& execution) {
  std::vector<std::shared_ptr<ExternalStorage>> owners;
  auto add = [&](const Tensor& t) {
    if (t.device.type != "cuda" || !t.buffer) return;
    if (auto* b = dynamic_cast<const CudaBuffer*>(t.buffer.get()); b && b->external_storage())
      owners.push_back(b->external_storage());
  };
  for (const auto& t : execution.inputs) add(t);
  for (const auto& t : execution.outputs) add(t);
  return owners;
}

}  // namespace tensorcx::cuda
