// Primary-context retention and scoped push/pop for the sm100 backend
// (surface of the reference's cuda_context.h:10-43).
#include "tensorcx/backends/cuda/cuda_context.h"

#include <unistd.h>

#include <string>

namespace tensorcx::cuda {
namespace {
const pid_t g_loaded_pid = getpid();

// Driver entry points resolved through the runtime (no link-time dependency on the
// driver library, which the CUDA runtime loads itself).
template <typename F>
F driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<F>(p);
}
struct Driver {
  decltype(&cuInit) init = driver_fn<decltype(&cuInit)>("cuInit");
  decltype(&cuDeviceGet) device_get = driver_fn<decltype(&cuDeviceGet)>("cuDeviceGet");
  decltype(&cuDevicePrimaryCtxRetain) retain = driver_fn<decltype(&cuDevicePrimaryCtxRetain)>("cuDevicePrimaryCtxRetain");
  decltype(&cuDevicePrimaryCtxRelease) release =
      driver_fn<decltype(&cuDevicePrimaryCtxRelease)>("cuDevicePrimaryCtxRelease");
  decltype(&cuCtxPushCurrent) push = driver_fn<decltype(&cuCtxPushCurrent)>("cuCtxPushCurrent");
  decltype(&cuCtxPopCurrent) pop = driver_fn<decltype(&cuCtxPopCurrent)>("cuCtxPopCurrent");
  decltype(&cuGetErrorName) error_name = driver_fn<decltype(&cuGetErrorName)>("cuGetErrorName");
  decltype(&cuGetErrorString) error_string = driver_fn<decltype(&cuGetErrorString)>("cuGetErrorString");
  bool ok() const { return init && device_get && retain && release && push && pop; }
};
const Driver& driver() {
  static const Driver d;
  return d;
}
}  // namespace

bool current_process() { return getpid() == g_loaded_pid; }

Status driver_status(CUresult error, const char* operation) {
  if (error == CUDA_SUCCESS) return Status::Ok();
  const char* name = nullptr;
  const char* text = nullptr;
  if (driver().error_name) driver().error_name(error, &name);
  if (driver().error_string) driver().error_string(error, &text);
  const StatusCode code = error == CUDA_ERROR_INVALID_VALUE ? StatusCode::kInvalidArgument
                          : error == CUDA_ERROR_NO_DEVICE || error == CUDA_ERROR_NOT_INITIALIZED ||
                                    error == CUDA_ERROR_DEINITIALIZED
                              ? StatusCode::kUnavailable
                              : StatusCode::kInternal;
  return Status(code, std::string(operation) + " failed: " + (name ? name : "CUDA driver error") + ": " +
                          (text ? text : ""));
}

Expected<std::shared_ptr<PrimaryContext>> PrimaryContext::acquire() {
  if (!current_process()) return Status(StatusCode::kUnavailable, "CUDA is not usable in a forked child");
  const Driver& d = driver();
  if (!d.ok()) return Status(StatusCode::kUnavailable, "CUDA driver entry points are unavailable");
  if (auto st = driver_status(d.init(0), "cuInit"); !st.ok()) return st;
  int ordinal = 0;
  if (auto st = runtime_status(cudaGetDevice(&ordinal), "cudaGetDevice"); !st.ok()) return st;
  std::shared_ptr<PrimaryContext> ctx(new PrimaryContext());
  if (auto st = driver_status(d.device_get(&ctx->device_, ordinal), "cuDeviceGet"); !st.ok()) return st;
  if (auto st = driver_status(d.retain(&ctx->context_, ctx->device_),
                              "cuDevicePrimaryCtxRetain");
      !st.ok()) {
    ctx->context_ = nullptr;
    return st;
  }
  return ctx;
}

PrimaryContext::~PrimaryContext() {
  // release only: never reset a primary context that other users may hold
  if (context_ && current_process() && driver().release) (void)driver().release(device_);
}

ContextScope::ContextScope() {
  auto owner = PrimaryContext::acquire();
  if (!owner) {
    status_ = owner.status();
    return;
  }
  owner_ = owner.move_value();
  push();
}

ContextScope::ContextScope(std::shared_ptr<PrimaryContext> owner) : owner_(std::move(owner)) {
  if (!owner_) {
    status_ = Status(StatusCode::kInvalidArgument, "missing CUDA context owner");
    return;
  }
  push();
}

void ContextScope::push() {
  if (!current_process()) {
    status_ = Status(StatusCode::kUnavailable, "CUDA is not usable in a forked child");
    return;
  }
  if (!driver().push) {
    status_ = Status(StatusCode::kUnavailable, "CUDA driver entry points are unavailable");
    return;
  }
  status_ = driver_status(driver().push(owner_->get()), "cuCtxPushCurrent");
  pushed_ = status_.ok();
}

ContextScope::~ContextScope() {
  if (pushed_) {
    CUcontext popped = nullptr;
    (void)driver().pop(&popped);
  }
}

}  // namespace tensorcx::cuda
