// C++ PrivateUse1 plumbing for the `matrixman` device, built as a small torch
// extension (torch.utils.cpp_extension) in-tree.
//
// Replaces drivers/matrixman/native/autograd_privateuse1.cpp of the reference
// (lines 7-66), whose hooks and DeviceGuard hard-wired one device and a no-op
// default stream.  Here the guard reports the real CUDA device count, switches
// the current CUDA device, and maps the c10 default stream of each device onto
// the runtime stream of libmatrixman_b200 (queried / synchronised through the
// C ABI).  The library is resolved at run time with dlsym, so this extension
// links against neither CUDA nor libmatrixman_b200 directly.
#include <ATen/detail/PrivateUse1HooksInterface.h>
#include <c10/core/impl/DeviceGuardImplInterface.h>
#include <dlfcn.h>
#include <torch/extension.h>

#include <atomic>
#include <cstring>

namespace {

using count_fn = int (*)(int*);
using dev_fn = int (*)(int);
using stream_fn = int (*)(int, void**);
using sync_fn = int (*)(void*, int64_t);
using query_fn = int (*)(void*, int*);

template <class F>
F resolve(const char* name) {
  void* p = dlsym(RTLD_DEFAULT, name);
  TORCH_CHECK(p != nullptr, "matrixman hooks: libmatrixman_b200 symbol ", name,
              " not loaded (import matrixman_b200 first)");
  return reinterpret_cast<F>(p);
}

thread_local int t_current_device = 0;

// Upper bound of every stream wait the guard makes (matrixman.config
// waitTimeoutMs, passed in at backend init; the config is locked from then on).
std::atomic<int64_t> g_wait_timeout_ms{600000};

int device_count() {
  int n = 0;
  if (resolve<count_fn>("mm_device_count")(&n) != 0) return 0;
  return n;
}

void* runtime_stream(int device) {
  void* s = nullptr;
  resolve<dev_fn>("mm_init")(device);
  resolve<stream_fn>("mm_runtime_stream")(device, &s);
  return s;
}

constexpr int MM_STATUS_TIMEOUT = 5;  // MM_ERR_TIMEOUT of the C ABI

// Bounded synchronisation of a device's runtime stream: raises with the C
// ABI's message when the wait gives up (MM_ERR_TIMEOUT) or fails.
void sync_runtime_stream(int device, const char* what) {
  const int rc = resolve<sync_fn>("mm_stream_sync")(runtime_stream(device), g_wait_timeout_ms.load());
  if (rc == 0) return;
  char msg[512] = {0};
  using err_fn = int (*)(char*, size_t);
  if (void* p = dlsym(RTLD_DEFAULT, "mm_last_error")) reinterpret_cast<err_fn>(p)(msg, sizeof(msg));
  TORCH_CHECK(rc != MM_STATUS_TIMEOUT, "matrixman guard: ", what, " of device ", device,
              " did not finish within ", g_wait_timeout_ms.load(), " ms (waitTimeoutMs): ", msg);
  TORCH_CHECK(false, "matrixman guard: ", what, " of device ", device, " failed: ", msg);
}

using pin_alloc_fn = int (*)(size_t, void**);
using pin_free_fn = int (*)(void*);
using is_pinned_fn = int (*)(const void*, int*);

void free_pinned(void* p) {
  if (p) resolve<pin_free_fn>("mm_host_free_pinned")(p);
}

// Page-locked host memory for Tensor.pin_memory() on this backend, so that
// uploads from pinned buffers run as asynchronous copy-engine transfers.
class PinnedAllocator final : public c10::Allocator {
 public:
  c10::DataPtr allocate(size_t n) override {
    void* p = nullptr;
    if (n > 0) {
      TORCH_CHECK(resolve<pin_alloc_fn>("mm_host_alloc_pinned")(n, &p) == 0,
                  "matrixman: pinned host allocation of ", n, " bytes failed");
    }
    return {p, p, &free_pinned, c10::Device(c10::DeviceType::CPU)};
  }
  c10::DeleterFnPtr raw_deleter() const override { return &free_pinned; }
  void copy_data(void* dst, const void* src, std::size_t count) const override {
    std::memcpy(dst, src, count);
  }
};

PinnedAllocator g_pinned;

class MatrixManHooks final : public at::PrivateUse1HooksInterface {
 public:
  bool isBuilt() const override { return true; }
  bool isAvailable() const override { return device_count() > 0; }
  bool hasPrimaryContext(c10::DeviceIndex) const override { return true; }
  c10::Device getDeviceFromPtr(void*) const override {
    return c10::Device(c10::DeviceType::PrivateUse1, (c10::DeviceIndex)t_current_device);
  }
  bool isPinnedPtr(const void* data) const override {
    int pinned = 0;
    resolve<is_pinned_fn>("mm_host_is_pinned")(data, &pinned);
    return pinned != 0;
  }
  c10::Allocator* getPinnedMemoryAllocator() const override { return &g_pinned; }
};

class MatrixManGuardImpl final : public c10::impl::DeviceGuardImplInterface {
 public:
  c10::DeviceType type() const override { return c10::DeviceType::PrivateUse1; }

  c10::Device exchangeDevice(c10::Device d) const override {
    c10::Device old = getDevice();
    if (d.index() != old.index()) setDevice(d);
    return old;
  }

  c10::Device getDevice() const override {
    return c10::Device(c10::DeviceType::PrivateUse1, (c10::DeviceIndex)t_current_device);
  }

  void setDevice(c10::Device d) const override {
    TORCH_CHECK(d.type() == c10::DeviceType::PrivateUse1, "matrixman guard: wrong device type");
    int idx = d.index() < 0 ? 0 : d.index();
    TORCH_CHECK(resolve<dev_fn>("mm_set_device")(idx) == 0, "matrixman guard: cannot select device ", idx);
    t_current_device = idx;
  }

  void uncheckedSetDevice(c10::Device d) const noexcept override {
    int idx = d.index() < 0 ? 0 : d.index();
    void* p = dlsym(RTLD_DEFAULT, "mm_set_device");
    if (p) reinterpret_cast<dev_fn>(p)(idx);
    t_current_device = idx;
  }

  // One runtime stream per device (id 0 == the libmatrixman_b200 runtime stream).
  c10::Stream getStream(c10::Device d) const override {
    return c10::Stream(c10::Stream::DEFAULT, d);
  }
  c10::Stream getNewStream(c10::Device d, int) const override {
    return c10::Stream(c10::Stream::DEFAULT, d);
  }
  c10::Stream exchangeStream(c10::Stream s) const noexcept override { return s; }

  c10::DeviceIndex deviceCount() const noexcept override {
    void* p = dlsym(RTLD_DEFAULT, "mm_device_count");
    if (!p) return 0;
    int n = 0;
    if (reinterpret_cast<count_fn>(p)(&n) != 0) return 0;
    return (c10::DeviceIndex)n;
  }

  bool queryStream(const c10::Stream& s) const override {
    int done = 1;
    resolve<query_fn>("mm_stream_query")(runtime_stream(s.device_index()), &done);
    return done != 0;
  }

  void synchronizeStream(const c10::Stream& s) const override {
    sync_runtime_stream(s.device_index(), "stream synchronize");
  }

  void synchronizeDevice(const c10::DeviceIndex idx) const override {
    sync_runtime_stream(idx, "device synchronize");
  }
};

C10_REGISTER_GUARD_IMPL(PrivateUse1, MatrixManGuardImpl);

MatrixManHooks g_hooks;
std::atomic<bool> g_registered{false};

void register_hooks() {
  bool expected = false;
  if (g_registered.compare_exchange_strong(expected, true)) {
    at::RegisterPrivateUse1HooksInterface(&g_hooks);
  }
}

int guard_device_count() { return (int)MatrixManGuardImpl().deviceCount(); }

void set_wait_timeout_ms(int64_t ms) {
  TORCH_CHECK(ms > 0, "matrixman hooks: wait timeout must be positive");
  g_wait_timeout_ms.store(ms);
}

int64_t wait_timeout_ms() { return g_wait_timeout_ms.load(); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("register_hooks", &register_hooks, "Register the matrixman PrivateUse1 hooks");
  m.def("device_count", &guard_device_count, "Device count seen by the DeviceGuard");
  m.def("set_wait_timeout_ms", &set_wait_timeout_ms, "Bound of the guard's stream waits (ms)");
  m.def("wait_timeout_ms", &wait_timeout_ms, "Bound of the guard's stream waits (ms)");
}
