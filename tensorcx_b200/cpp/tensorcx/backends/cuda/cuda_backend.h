// The sm100 CUDA backend behind tensor.cx's backend execution ABI. Same public
// surface as the reference's cpp/tensorcx/backends/cuda/cuda_backend.h:15-49 and
// cuda_buffer.h:22-45, so bindings and core composites link against it unchanged;
// the hot-path primitives run the sm_100a kernels of libtcx_sm100.so through the C
// ABI in include/tcx_sm100.h.
#pragma once

#include <atomic>
#include <memory>
#include <string>

#include "tensorcx/backends/cpu/cpu_tensor.h"
#include "tensorcx/core/backend.h"
#include "tensorcx/core/buffer.h"
#include "tensorcx/core/expected.h"

namespace tensorcx::cuda {

class MemoryPool;
class ExternalStorage;
class PrimaryContext;

// Device memory of one tensor: owned (stream-ordered pool or the device's default
// stream-ordered pool) or borrowed from an external owner (a DLPack producer, or a
// registered ExternalStorage whose storage identity and lock it then reports).
class CudaBuffer final : public Buffer {
 public:
  static Expected<std::shared_ptr<CudaBuffer>> create(DType dtype, const Shape& shape, int device = 0);
  static Expected<std::shared_ptr<CudaBuffer>> borrow(DType dtype, const Shape& shape, void* data,
                                                     std::shared_ptr<void> owner, int device = 0);
  // The reference's form (cuda_buffer.h:22-45): the device is the one the pointer lives on.
  static Expected<std::shared_ptr<CudaBuffer>> borrow(DType dtype, const Shape& shape, void* data,
                                                     std::shared_ptr<void> owner,
                                                     std::shared_ptr<ExternalStorage> storage);
  ~CudaBuffer() override;
  std::size_t nbytes() const override { return bytes_; }
  StorageRelation storage_relation(const Buffer& other) const override;
  StorageIdentity storage_identity() const override;
  std::shared_ptr<StorageAccess> access() const override;
  const std::shared_ptr<ExternalStorage>& external_storage() const { return external_storage_; }
  // The retained primary context of the buffer's device (acquired on first use).
  const std::shared_ptr<PrimaryContext>& context() const;
  DType dtype() const { return dtype_; }
  void* data() const { return data_; }
  int device() const { return device_; }
  void mark_exported() { exported_.store(true, std::memory_order_relaxed); }

  CudaBuffer() = default;

 private:
  DType dtype_{DType::kFloat32};
  std::size_t bytes_{0};
  int device_{0};
  void* data_{nullptr};
  std::atomic<bool> exported_{false};
  std::shared_ptr<MemoryPool> pool_;
  std::shared_ptr<void> external_owner_;
  std::shared_ptr<ExternalStorage> external_storage_;
  mutable std::shared_ptr<PrimaryContext> context_;
};

class CudaTensor {
 public:
  CudaTensor(DType dtype, Shape shape, std::shared_ptr<CudaBuffer> buffer);
  DType dtype() const { return dtype_; }
  const Shape& shape() const { return shape_; }
  const Shape& strides() const { return strides_; }
  const std::shared_ptr<CudaBuffer>& buffer() const { return buffer_; }
  std::size_t nbytes() const;

 private:
  DType dtype_;
  Shape shape_;
  Shape strides_;
  std::shared_ptr<CudaBuffer> buffer_;
};

class CudaBackend final : public Backend {
 public:
  std::string name() const override { return "cuda"; }
  Status execute(const BackendExecution& execution) override;
};

bool available();
Expected<std::string> device_name();
struct DeviceInfo {
  std::string name;
  int major{0}, minor{0}, runtime_version{0}, driver_version{0};
  std::size_t free_bytes{0}, total_bytes{0};
};
Expected<DeviceInfo> device_info();
Expected<CudaTensor> empty(Shape shape, DType dtype, int device = 0);
Expected<CudaTensor> from_cpu(const cpu::CpuTensor& tensor, int device = 0);
Expected<cpu::CpuTensor> to_cpu(const CudaTensor& tensor);
Tensor to_core_tensor(const CudaTensor& tensor);
Expected<CudaTensor> from_core_tensor(const Tensor& tensor);

}  // namespace tensorcx::cuda
