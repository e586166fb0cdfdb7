// Runtime part of libmatrixman_b200: errors, devices, streams, events, the
// caching arena, copies and CUDA graphs.  See include/matrixman_b200.h.
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>

#include "mm_arena.hpp"
#include "mm_common.cuh"

namespace mm {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t err, const char* action) {
  std::string msg = std::string(action) + ": " + cudaGetErrorName(err) + " (" +
                    cudaGetErrorString(err) + ")";
  g_last_error = msg;
  if (err == cudaErrorMemoryAllocation) return MM_ERR_OOM;
  return MM_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Arena backends
// ---------------------------------------------------------------------------

struct CudaArenaBackend {
  using Event = cudaEvent_t;
  using Stream = cudaStream_t;
  int device = 0;
  bool malloc(void** p, size_t n) {
    cudaError_t e = cudaMalloc(p, n);
    if (e != cudaSuccess) {
      cudaGetLastError();  // clear the sticky-free error state of a failed malloc
      return false;
    }
    return true;
  }
  void free(void* p) { cudaFree(p); }
  bool event_create(Event* e) {
    return cudaEventCreateWithFlags(e, cudaEventDisableTiming) == cudaSuccess;
  }
  void event_destroy(Event e) { cudaEventDestroy(e); }
  void event_record(Event e, Stream s) { cudaEventRecord(e, s); }
  bool event_done(Event e) {
    cudaError_t r = cudaEventQuery(e);
    if (r == cudaErrorNotReady) {
      cudaGetLastError();
      return false;
    }
    return true;
  }
  void stream_wait(Stream s, Event e) { cudaStreamWaitEvent(s, e, 0); }
  void stream_sync(Stream s) { cudaStreamSynchronize(s); }
  void device_sync() { cudaDeviceSynchronize(); }
};

// Host memory with simulated events: a record stamps the current generation;
// the event counts as complete once complete(g >= stamp) has been called.
struct HostArenaState {
  int64_t capacity = 0;
  int64_t used = 0;
  int64_t generation = 1;
  int64_t completed = 0;
  std::unordered_map<void*, size_t> sizes;
};

struct HostArenaBackend {
  using Event = int64_t;
  using Stream = int;
  HostArenaState* st = nullptr;
  bool malloc(void** p, size_t n) {
    if (st->capacity > 0 && st->used + (int64_t)n > st->capacity) return false;
    *p = std::malloc(n);
    if (*p == nullptr) return false;
    st->used += (int64_t)n;
    st->sizes[*p] = n;
    return true;
  }
  void free(void* p) {
    auto it = st->sizes.find(p);
    if (it != st->sizes.end()) {
      st->used -= (int64_t)it->second;
      st->sizes.erase(it);
    }
    std::free(p);
  }
  bool event_create(Event* e) {
    *e = 0;
    return true;
  }
  void event_destroy(Event) {}
  void event_record(Event& e, Stream) { e = st->generation++; }
  bool event_done(Event e) { return e <= st->completed; }
  void stream_wait(Stream, Event) {}
  void stream_sync(Stream) {}
  void device_sync() { st->completed = st->generation; }
};

// ---------------------------------------------------------------------------
// Per-device runtime
// ---------------------------------------------------------------------------

struct DeviceRuntime {
  int device = -1;
  cudaStream_t stream = nullptr;
  std::unique_ptr<Arena<CudaArenaBackend>> arena;
  int sm_count = 0;
  std::atomic<int64_t> next_capture{1};
};

static std::mutex g_rt_mu;
static DeviceRuntime* g_rt[64] = {nullptr};

static DeviceRuntime* runtime_for(int device) {
  if (device < 0 || device >= 64) return nullptr;
  return g_rt[device];
}

static int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

cudaStream_t resolve_stream(void* stream) {
  if (stream != nullptr) return (cudaStream_t)stream;
  DeviceRuntime* rt = runtime_for(current_device());
  return rt ? rt->stream : nullptr;
}

int sm_count() {
  int d = current_device();
  DeviceRuntime* rt = runtime_for(d);
  if (rt && rt->sm_count > 0) return rt->sm_count;
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
  return n;
}

int validate(const mm_tensor_t* t, const char* name, int want_dtype) {
  if (t == nullptr) return fail(MM_ERR_INVALID, std::string(name) + ": null tensor descriptor");
  if (t->ndim < 0 || t->ndim > MM_MAX_DIMS)
    return fail(MM_ERR_UNSUPPORTED, std::string(name) + ": rank " + std::to_string(t->ndim) +
                                        " exceeds " + std::to_string(MM_MAX_DIMS));
  if (want_dtype >= 0 && t->dtype != want_dtype)
    return fail(MM_ERR_UNSUPPORTED, std::string(name) + ": unsupported dtype");
  for (int i = 0; i < t->ndim; ++i) {
    if (t->size[i] < 0 || t->stride[i] < 0)
      return fail(MM_ERR_INVALID, std::string(name) + ": negative size or stride");
  }
  if (numel(t) > 0 && t->data == nullptr)
    return fail(MM_ERR_INVALID, std::string(name) + ": null data pointer");
  return MM_OK;
}

int collapse(int nops, const mm_tensor_t* const* ops, Geom* g) {
  const mm_tensor_t* r = ops[0];
  for (int k = 1; k < nops; ++k) {
    if (ops[k]->ndim != r->ndim) return fail(MM_ERR_INVALID, "collapse: rank mismatch");
    for (int i = 0; i < r->ndim; ++i)
      if (ops[k]->size[i] != r->size[i]) return fail(MM_ERR_INVALID, "collapse: shape mismatch");
  }
  // Drop size-1 dims.
  int nd = 0;
  int64_t size[MM_MAX_DIMS];
  int64_t st[4][MM_MAX_DIMS];
  for (int i = 0; i < r->ndim; ++i) {
    if (r->size[i] == 1) continue;
    size[nd] = r->size[i];
    for (int k = 0; k < nops; ++k) st[k][nd] = ops[k]->stride[i];
    ++nd;
  }
  // Merge dim i-1 into i when contiguous in every operand.
  int out_nd = 0;
  int64_t osize[MM_MAX_DIMS];
  int64_t ost[4][MM_MAX_DIMS];
  for (int i = 0; i < nd; ++i) {
    if (out_nd > 0) {
      bool merge = true;
      for (int k = 0; k < nops; ++k)
        if (ost[k][out_nd - 1] != st[k][i] * size[i]) merge = false;
      if (merge) {
        osize[out_nd - 1] *= size[i];
        for (int k = 0; k < nops; ++k) ost[k][out_nd - 1] = st[k][i];
        continue;
      }
    }
    osize[out_nd] = size[i];
    for (int k = 0; k < nops; ++k) ost[k][out_nd] = st[k][i];
    ++out_nd;
  }
  for (int k = 0; k < nops; ++k) {
    g[k].nd = out_nd;
    for (int i = 0; i < out_nd; ++i) {
      g[k].size[i] = osize[i];
      g[k].stride[i] = ost[k][i];
    }
  }
  return MM_OK;
}

}  // namespace mm

using namespace mm;

// ---------------------------------------------------------------------------
// C ABI: errors and devices
// ---------------------------------------------------------------------------

extern "C" int mm_abi_version(void) { return MM_ABI_VERSION; }

extern "C" int mm_last_error(char* buf, size_t n) {
  if (buf == nullptr || n == 0) return MM_ERR_INVALID;
  const std::string& s = g_last_error;
  size_t len = s.size() < n - 1 ? s.size() : n - 1;
  std::memcpy(buf, s.data(), len);
  buf[len] = '\0';
  return MM_OK;
}

extern "C" int mm_device_count(int* out) {
  if (out == nullptr) return fail(MM_ERR_INVALID, "mm_device_count: null output");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *out = 0;
    return cuda_fail(e, "cudaGetDeviceCount");
  }
  *out = n;
  return MM_OK;
}

extern "C" int mm_device_info(int device, mm_device_info_t* out) {
  if (out == nullptr) return fail(MM_ERR_INVALID, "mm_device_info: null output");
  cudaDeviceProp prop;
  MM_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  std::memset(out, 0, sizeof(*out));
  std::strncpy(out->name, prop.name, sizeof(out->name) - 1);
  out->cc_major = prop.major;
  out->cc_minor = prop.minor;
  out->sm_count = prop.multiProcessorCount;
  out->total_bytes = (int64_t)prop.totalGlobalMem;
  int prev = current_device();
  if (cudaSetDevice(device) == cudaSuccess) {
    size_t fr = 0, tot = 0;
    if (cudaMemGetInfo(&fr, &tot) == cudaSuccess) out->free_bytes = (int64_t)fr;
    cudaSetDevice(prev);
  }
  return MM_OK;
}

extern "C" int mm_init(int device) {
  std::lock_guard<std::mutex> g(g_rt_mu);
  if (device < 0 || device >= 64) return fail(MM_ERR_INVALID, "mm_init: device index out of range");
  if (g_rt[device] != nullptr) {
    MM_CUDA(cudaSetDevice(device), "cudaSetDevice");
    return MM_OK;
  }
  int count = 0;
  MM_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (device >= count)
    return fail(MM_ERR_STATE, "mm_init: device " + std::to_string(device) + " not present (" +
                                  std::to_string(count) + " visible)");
  MM_CUDA(cudaSetDevice(device), "cudaSetDevice");
  cudaDeviceProp prop;
  MM_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(MM_ERR_UNSUPPORTED, std::string("mm_init: ") + prop.name +
                                        " is not an sm_100 (B200) device; this build targets sm_100a only");
  auto* rt = new DeviceRuntime();
  rt->device = device;
  rt->sm_count = prop.multiProcessorCount;
  cudaError_t e = cudaStreamCreateWithFlags(&rt->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete rt;
    return cuda_fail(e, "cudaStreamCreate");
  }
  CudaArenaBackend be;
  be.device = device;
  rt->arena.reset(new Arena<CudaArenaBackend>(be));
  if (const char* env = std::getenv("MATRIXMAN_TEST_FAIL_ALLOC_AFTER")) {
    rt->arena->set_fail_after(std::atoll(env));
  }
  g_rt[device] = rt;
  return MM_OK;
}

extern "C" int mm_shutdown(int device) {
  std::lock_guard<std::mutex> g(g_rt_mu);
  DeviceRuntime* rt = runtime_for(device);
  if (rt == nullptr) return MM_OK;
  cudaSetDevice(device);
  cudaStreamSynchronize(rt->stream);
  rt->arena->release_all();
  cudaStreamDestroy(rt->stream);
  delete rt;
  g_rt[device] = nullptr;
  return MM_OK;
}

extern "C" int mm_set_device(int device) {
  MM_CUDA(cudaSetDevice(device), "cudaSetDevice");
  return MM_OK;
}

extern "C" int mm_runtime_stream(int device, void** stream_out) {
  DeviceRuntime* rt = runtime_for(device);
  if (rt == nullptr) return fail(MM_ERR_STATE, "mm_runtime_stream: device not initialised");
  *stream_out = rt->stream;
  return MM_OK;
}

extern "C" int mm_stream_create(int device, void** stream_out) {
  MM_CUDA(cudaSetDevice(device), "cudaSetDevice");
  cudaStream_t s;
  MM_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
  *stream_out = s;
  return MM_OK;
}

extern "C" int mm_stream_destroy(void* stream) {
  if (stream == nullptr) return MM_OK;
  MM_CUDA(cudaStreamDestroy((cudaStream_t)stream), "cudaStreamDestroy");
  return MM_OK;
}

static int bounded_poll(std::function<cudaError_t()> query, int64_t timeout_ms, const char* what) {
  auto start = std::chrono::steady_clock::now();
  int spins = 0;
  while (true) {
    cudaError_t e = query();
    if (e == cudaSuccess) return MM_OK;
    if (e != cudaErrorNotReady) return cuda_fail(e, what);
    cudaGetLastError();
    if (timeout_ms >= 0) {
      auto el = std::chrono::duration_cast<std::chrono::milliseconds>(
                    std::chrono::steady_clock::now() - start)
                    .count();
      if (el >= timeout_ms)
        return fail(MM_ERR_TIMEOUT, std::string(what) + ": timed out after " +
                                        std::to_string(timeout_ms) + " ms");
    }
    if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

extern "C" int mm_stream_sync(void* stream, int64_t timeout_ms) {
  cudaStream_t s = resolve_stream(stream);
  if (timeout_ms < 0) {
    MM_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    return MM_OK;
  }
  return bounded_poll([s]() { return cudaStreamQuery(s); }, timeout_ms, "stream synchronize");
}

extern "C" int mm_stream_query(void* stream, int* done) {
  cudaError_t e = cudaStreamQuery(resolve_stream(stream));
  if (e == cudaSuccess) {
    *done = 1;
    return MM_OK;
  }
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    *done = 0;
    return MM_OK;
  }
  return cuda_fail(e, "cudaStreamQuery");
}

extern "C" int mm_event_create(void** event_out, int timing) {
  cudaEvent_t e;
  MM_CUDA(cudaEventCreateWithFlags(&e, timing ? cudaEventDefault : cudaEventDisableTiming),
          "cudaEventCreate");
  *event_out = e;
  return MM_OK;
}

extern "C" int mm_event_destroy(void* event) {
  if (event) MM_CUDA(cudaEventDestroy((cudaEvent_t)event), "cudaEventDestroy");
  return MM_OK;
}

extern "C" int mm_event_record(void* event, void* stream) {
  MM_CUDA(cudaEventRecord((cudaEvent_t)event, resolve_stream(stream)), "cudaEventRecord");
  return MM_OK;
}

extern "C" int mm_event_sync(void* event, int64_t timeout_ms) {
  cudaEvent_t e = (cudaEvent_t)event;
  if (timeout_ms < 0) {
    MM_CUDA(cudaEventSynchronize(e), "cudaEventSynchronize");
    return MM_OK;
  }
  return bounded_poll([e]() { return cudaEventQuery(e); }, timeout_ms, "event synchronize");
}

extern "C" int mm_stream_wait_event(void* stream, void* event) {
  MM_CUDA(cudaStreamWaitEvent(resolve_stream(stream), (cudaEvent_t)event, 0), "cudaStreamWaitEvent");
  return MM_OK;
}

extern "C" int mm_event_elapsed_ms(void* start, void* stop, float* ms) {
  MM_CUDA(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)stop), "cudaEventElapsedTime");
  return MM_OK;
}

// ---------------------------------------------------------------------------
// C ABI: arena
// ---------------------------------------------------------------------------

extern "C" int mm_pool_configure(int device, int sync_safe, int deferred_activation,
                                 int deferred_scratch, int disable_pool) {
  DeviceRuntime* rt = runtime_for(device);
  if (rt == nullptr) return fail(MM_ERR_STATE, "mm_pool_configure: device not initialised");
  rt->arena->configure(sync_safe != 0, deferred_activation != 0, deferred_scratch != 0,
                       disable_pool != 0);
  return MM_OK;
}

extern "C" int mm_alloc(int device, size_t bytes, int kind, void* stream, void** out) {
  if (out == nullptr) return fail(MM_ERR_INVALID, "mm_alloc: null output");
  DeviceRuntime* rt = runtime_for(device);
  if (rt == nullptr) return fail(MM_ERR_STATE, "mm_alloc: device not initialised");
  int prev = current_device();
  if (prev != device) cudaSetDevice(device);
  std::string msg;
  cudaStream_t s = stream ? (cudaStream_t)stream : rt->stream;
  int rc = rt->arena->alloc(bytes, kind, s, out, &msg);
  if (prev != device) cudaSetDevice(prev);
  if (rc != MM_OK) return fail(rc, msg);
  return MM_OK;
}

static DeviceRuntime* runtime_owning(void* ptr) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return runtime_for(attr.device);
}

extern "C" int mm_free(void* ptr, void* stream) {
  if (ptr == nullptr) return MM_OK;
  DeviceRuntime* rt = runtime_owning(ptr);
  if (rt == nullptr) return fail(MM_ERR_STATE, "mm_free: pointer's device has no runtime");
  int prev = current_device();
  if (prev != rt->device) cudaSetDevice(rt->device);
  std::string msg;
  cudaStream_t s = stream ? (cudaStream_t)stream : rt->stream;
  int rc = rt->arena->free(ptr, s, &msg);
  if (prev != rt->device) cudaSetDevice(prev);
  if (rc != MM_OK) return fail(rc, msg);
  return MM_OK;
}

extern "C" int mm_pool_trim(int device) {
  DeviceRuntime* rt = runtime_for(device);
  if (rt == nullptr) return fail(MM_ERR_STATE, "mm_pool_trim: device not initialised");
  int prev = current_device();
  cudaSetDevice(device);
  rt->arena->trim();
  cudaSetDevice(prev);
  return MM_OK;
}

extern "C" int mm_pool_stats(int device, mm_pool_stats_t* out) {
  DeviceRuntime* rt = runtime_for(device);
  if (rt == nullptr) return fail(MM_ERR_STATE, "mm_pool_stats: device not initialised");
  *out = rt->arena->stats();
  return MM_OK;
}

extern "C" int mm_debug_fail_alloc_after(int device, int64_t n) {
  DeviceRuntime* rt = runtime_for(device);
  if (rt == nullptr) return fail(MM_ERR_STATE, "mm_debug_fail_alloc_after: device not initialised");
  rt->arena->set_fail_after(n);
  return MM_OK;
}

// Host-backed arena for CPU tests.
struct HostArena {
  HostArenaState state;
  std::unique_ptr<Arena<HostArenaBackend>> arena;
};

extern "C" int mm_host_arena_create(int64_t capacity_bytes, int deferred, void** arena_out) {
  auto* h = new HostArena();
  h->state.capacity = capacity_bytes;
  HostArenaBackend be;
  be.st = &h->state;
  h->arena.reset(new Arena<HostArenaBackend>(be));
  h->arena->configure(true, deferred != 0, deferred != 0, false);
  *arena_out = h;
  return MM_OK;
}

extern "C" int mm_host_arena_destroy(void* arena) {
  delete (HostArena*)arena;
  return MM_OK;
}

extern "C" int mm_host_arena_alloc(void* arena, size_t bytes, int kind, void** out) {
  std::string msg;
  int rc = ((HostArena*)arena)->arena->alloc(bytes, kind, 0, out, &msg);
  return rc == MM_OK ? MM_OK : fail(rc, msg);
}

extern "C" int mm_host_arena_free(void* arena, void* ptr) {
  std::string msg;
  int rc = ((HostArena*)arena)->arena->free(ptr, 0, &msg);
  return rc == MM_OK ? MM_OK : fail(rc, msg);
}

extern "C" int mm_host_arena_complete(void* arena, int64_t generation) {
  auto* h = (HostArena*)arena;
  if (generation > h->state.completed) h->state.completed = generation;
  return MM_OK;
}

extern "C" int mm_host_arena_generation(void* arena, int64_t* out) {
  *out = ((HostArena*)arena)->state.generation;
  return MM_OK;
}

extern "C" int mm_host_arena_fail_after(void* arena, int64_t n) {
  ((HostArena*)arena)->arena->set_fail_after(n);
  return MM_OK;
}

extern "C" int mm_host_arena_stats(void* arena, mm_pool_stats_t* out) {
  *out = ((HostArena*)arena)->arena->stats();
  return MM_OK;
}

// ---------------------------------------------------------------------------
// C ABI: copies
// ---------------------------------------------------------------------------

extern "C" int mm_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream, int sync) {
  if (bytes == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  MM_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s), "host-to-device copy");
  if (sync) MM_CUDA(cudaStreamSynchronize(s), "host-to-device copy synchronize");
  return MM_OK;
}

extern "C" int mm_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream, int sync) {
  if (bytes == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  MM_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s), "device-to-host copy");
  if (sync) MM_CUDA(cudaStreamSynchronize(s), "device-to-host copy synchronize");
  return MM_OK;
}

extern "C" int mm_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return MM_OK;
  MM_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, resolve_stream(stream)),
          "device-to-device copy");
  return MM_OK;
}

extern "C" int mm_memcpy_peer(void* dst, int dst_device, const void* src, int src_device,
                              size_t bytes, void* stream) {
  if (bytes == 0) return MM_OK;
  MM_CUDA(cudaMemcpyPeerAsync(dst, dst_device, src, src_device, bytes, resolve_stream(stream)),
          "peer copy");
  return MM_OK;
}

extern "C" int mm_enable_peer_access(int device, int peer) {
  int can = 0;
  MM_CUDA(cudaDeviceCanAccessPeer(&can, device, peer), "cudaDeviceCanAccessPeer");
  if (!can) return fail(MM_ERR_UNSUPPORTED, "peer access not available between these devices");
  int prev = current_device();
  cudaSetDevice(device);
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  cudaSetDevice(prev);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return MM_OK;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceEnablePeerAccess");
  return MM_OK;
}

// Device memory shared between processes (one process per GPU): the owner
// allocates it and exports a CUDA IPC handle; the other processes open the
// handle and write into it with copy-engine copies (NVLink between GPUs).
extern "C" int mm_ipc_alloc(int device, size_t bytes, void** ptr_out, void* handle_out) {
  if (ptr_out == nullptr || handle_out == nullptr || bytes == 0)
    return fail(MM_ERR_INVALID, "mm_ipc_alloc: bad arguments");
  int prev = current_device();
  MM_CUDA(cudaSetDevice(device), "cudaSetDevice");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) {
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) {
      memcpy(handle_out, &h, sizeof(h));
      *ptr_out = p;
    } else {
      cudaFree(p);
    }
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "mm_ipc_alloc");
  return MM_OK;
}

extern "C" int mm_ipc_free(int device, void* ptr) {
  if (ptr == nullptr) return MM_OK;
  int prev = current_device();
  MM_CUDA(cudaSetDevice(device), "cudaSetDevice");
  cudaError_t e = cudaFree(ptr);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "mm_ipc_free");
  return MM_OK;
}

extern "C" int mm_ipc_open(int device, const void* handle, void** ptr_out) {
  if (ptr_out == nullptr || handle == nullptr) return fail(MM_ERR_INVALID, "mm_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  int prev = current_device();
  MM_CUDA(cudaSetDevice(device), "cudaSetDevice");
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "mm_ipc_open");
  *ptr_out = p;
  return MM_OK;
}

extern "C" int mm_ipc_close(int device, void* ptr) {
  if (ptr == nullptr) return MM_OK;
  int prev = current_device();
  MM_CUDA(cudaSetDevice(device), "cudaSetDevice");
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "mm_ipc_close");
  return MM_OK;
}

extern "C" int mm_host_alloc_pinned(size_t bytes, void** out) {
  MM_CUDA(cudaHostAlloc(out, bytes, cudaHostAllocPortable), "cudaHostAlloc");
  return MM_OK;
}

extern "C" int mm_host_free_pinned(void* ptr) {
  if (ptr) MM_CUDA(cudaFreeHost(ptr), "cudaFreeHost");
  return MM_OK;
}

extern "C" int mm_host_is_pinned(const void* ptr, int* out) {
  if (out == nullptr) return fail(MM_ERR_INVALID, "mm_host_is_pinned: null output");
  *out = 0;
  if (ptr == nullptr) return MM_OK;
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return MM_OK;
  }
  *out = attr.type == cudaMemoryTypeHost ? 1 : 0;
  return MM_OK;
}

// ---------------------------------------------------------------------------
// C ABI: graphs
// ---------------------------------------------------------------------------

struct GraphHandle {
  int device;
  int64_t capture_id;
  cudaGraph_t graph;
  cudaGraphExec_t exec;
};

extern "C" int mm_graph_capture_begin(int device, void* stream) {
  DeviceRuntime* rt = runtime_for(device);
  if (rt == nullptr) return fail(MM_ERR_STATE, "mm_graph_capture_begin: device not initialised");
  cudaStream_t s = stream ? (cudaStream_t)stream : rt->stream;
  int64_t id = rt->next_capture.fetch_add(1);
  rt->arena->begin_capture(id);
  cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed);
  if (e != cudaSuccess) {
    rt->arena->end_capture();
    rt->arena->destroy_capture(id);
    return cuda_fail(e, "cudaStreamBeginCapture");
  }
  return MM_OK;
}

extern "C" int mm_graph_capture_end(int device, void* stream, void** graph_out) {
  DeviceRuntime* rt = runtime_for(device);
  if (rt == nullptr) return fail(MM_ERR_STATE, "mm_graph_capture_end: device not initialised");
  cudaStream_t s = stream ? (cudaStream_t)stream : rt->stream;
  // The capture id is the most recent one handed out on this device.
  int64_t id = rt->next_capture.load() - 1;
  rt->arena->end_capture();
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(s, &graph);
  if (e != cudaSuccess) {
    rt->arena->destroy_capture(id);
    return cuda_fail(e, "cudaStreamEndCapture");
  }
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(graph);
    rt->arena->destroy_capture(id);
    return cuda_fail(e, "cudaGraphInstantiate");
  }
  auto* h = new GraphHandle{device, id, graph, exec};
  *graph_out = h;
  return MM_OK;
}

extern "C" int mm_graph_launch(void* graph, void* stream) {
  auto* h = (GraphHandle*)graph;
  if (h == nullptr) return fail(MM_ERR_INVALID, "mm_graph_launch: null graph");
  DeviceRuntime* rt = runtime_for(h->device);
  cudaStream_t s = stream ? (cudaStream_t)stream : (rt ? rt->stream : nullptr);
  MM_CUDA(cudaGraphLaunch(h->exec, s), "cudaGraphLaunch");
  return MM_OK;
}

extern "C" int mm_graph_destroy(void* graph) {
  auto* h = (GraphHandle*)graph;
  if (h == nullptr) return MM_OK;
  DeviceRuntime* rt = runtime_for(h->device);
  int prev = current_device();
  cudaSetDevice(h->device);
  cudaDeviceSynchronize();
  cudaGraphExecDestroy(h->exec);
  cudaGraphDestroy(h->graph);
  if (rt) rt->arena->destroy_capture(h->capture_id);
  cudaSetDevice(prev);
  delete h;
  return MM_OK;
}
