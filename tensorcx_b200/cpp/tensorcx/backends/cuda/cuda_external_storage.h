// External device storage (memory a DLPack producer or a graphics interop owns) as the
// reference declares it (cpp/tensorcx/backends/cuda/cuda_external_storage.h): a typed
// provider interface, a process-wide registry keyed by address range, and a lease that
// holds the owners' storage locks for one operation and completes their CUDA work
// before releasing them.
#pragma once

#include <cstdint>
#include <memory>
#include <span>
#include <vector>

#include "tensorcx/core/backend.h"
#include "tensorcx/core/dtype.h"
#include "tensorcx/core/expected.h"
#include "tensorcx/core/storage_access.h"

namespace tensorcx::cuda {

class ExternalStorage {
 public:
  virtual ~ExternalStorage() = default;
  virtual std::shared_ptr<StorageAccess> access() = 0;
  virtual std::uintptr_t begin() const = 0;
  virtual std::size_t bytes() const = 0;
  virtual std::size_t mapped_bytes() const = 0;
  virtual Status validate_range(void* data, DType dtype, std::size_t bytes) const = 0;
  virtual StorageIdentity identity(void* data, std::size_t bytes) const = 0;
  virtual Status complete_cuda() = 0;
  virtual void poison() noexcept = 0;
};

void register_external_storage(const std::shared_ptr<ExternalStorage>& owner);
void unregister_external_storage(std::uintptr_t begin, const ExternalStorage* owner) noexcept;
// The registered owner whose mapped range contains [data, data + bytes); kInvalidArgument
// when none does.
Expected<std::shared_ptr<ExternalStorage>> find_external_storage(void* data, std::size_t bytes);

class ExternalLease {
 public:
  explicit ExternalLease(std::vector<std::shared_ptr<ExternalStorage>> owners);
  ~ExternalLease();
  const Status& status() const { return lease_.status(); }
  // Completes every owner's outstanding CUDA work (first failure reported).
  Status finish();

 private:
  std::vector<std::shared_ptr<ExternalStorage>> owners_;
  StorageLease lease_;
  bool finished_ = false;
  Status completion_;
};

// The external owners of an execution's CUDA inputs and outputs.
std::vector<std::shared_ptr<ExternalStorage>> external_owners(const BackendExecution& execution);

}  // namespace tensorcx::cuda
