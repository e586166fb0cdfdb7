// Caching arena behind matrixman.config.activation_pool / scratch_pool.
//
// Policy code is templated on a backend so that the same state machine runs
// on CUDA (CudaBackend in mm_runtime.cu) and on host memory with simulated
// events (HostBackend in mm_runtime.cu) for CPU-only tests.
//
// State machine of a pooled block (activation / scratch kinds):
//   live --free--> pending (deferred policy: until its release event completes)
//                  cached  (safe policy: immediately, reuse ordered by the event)
//   cached --alloc of the same size class--> live
// Parameter blocks are never pooled: free returns them to the device.
// During CUDA-graph capture, allocations and frees on the capturing device go
// to a private pool owned by the graph (see CapturePool) so that replays never
// race with eager work.
#pragma once

#include <stdint.h>

#include <deque>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/matrixman_b200.h"

namespace mm {

// Size classes: 512-byte granularity below 1 MiB, then 8 classes per power
// of two (at most 12.5% internal waste).
inline size_t size_class(size_t bytes) {
  if (bytes == 0) bytes = 1;
  if (bytes <= (1u << 20)) return (bytes + 511) & ~size_t(511);
  size_t p = 1;
  while (p < bytes) p <<= 1;
  size_t step = p >> 4;  // p/2 .. p in steps of p/16
  return (bytes + step - 1) / step * step;
}

template <class Backend>
class Arena {
 public:
  using Event = typename Backend::Event;
  using Stream = typename Backend::Stream;

  struct Block {
    void* ptr = nullptr;
    size_t size = 0;       // class size
    int kind = 0;
    Event ev{};
    bool has_event = false;
    Stream release_stream{};
    int64_t capture_id = 0;  // 0 = global pool
  };

  struct CapturePool {
    std::map<size_t, std::vector<Block*>> free_blocks;
    std::vector<Block*> owned;  // every block the graph may touch
  };

  explicit Arena(Backend backend) : be_(backend) {}
  ~Arena() { release_all(); }

  void configure(bool sync_safe, bool deferred_act, bool deferred_scratch, bool disable_pool) {
    std::lock_guard<std::mutex> g(mu_);
    sync_safe_ = sync_safe;
    deferred_[MM_POOL_ACTIVATION] = deferred_act;
    deferred_[MM_POOL_SCRATCH] = deferred_scratch;
    disable_pool_ = disable_pool;
  }

  void set_fail_after(int64_t n) {
    std::lock_guard<std::mutex> g(mu_);
    fail_after_ = n;
  }

  // Returns MM_OK / MM_ERR_OOM / MM_ERR_INVALID / MM_ERR_CUDA; msg on failure.
  int alloc(size_t bytes, int kind, Stream stream, void** out, std::string* msg) {
    if (kind < 0 || kind > MM_POOL_PARAMETER) {
      *msg = "mm_alloc: invalid pool kind";
      return MM_ERR_INVALID;
    }
    std::lock_guard<std::mutex> g(mu_);
    size_t cls = size_class(bytes);
    ++stats_.alloc_calls[kind];
    if (capture_id_ != 0 && kind != MM_POOL_PARAMETER) {
      CapturePool& cp = captures_[capture_id_];
      auto it = cp.free_blocks.find(cls);
      if (it != cp.free_blocks.end() && !it->second.empty()) {
        Block* b = it->second.back();
        it->second.pop_back();
        b->kind = kind;
        live_[b->ptr] = b;
        account_live(b, +1);
        ++stats_.pool_hits[kind];
        *out = b->ptr;
        return MM_OK;
      }
      Block* b = nullptr;
      int rc = device_alloc(cls, kind, &b, msg);
      if (rc != MM_OK) return rc;
      b->capture_id = capture_id_;
      cp.owned.push_back(b);
      live_[b->ptr] = b;
      account_live(b, +1);
      *out = b->ptr;
      return MM_OK;
    }
    if (kind != MM_POOL_PARAMETER && !disable_pool_) {
      drain_pending_locked(kind);
      auto it = cached_[kind].find(cls);
      if (it != cached_[kind].end() && !it->second.empty()) {
        Block* b = it->second.back();
        it->second.pop_back();
        stats_.cached_bytes[kind] -= (int64_t)b->size;
        if (sync_safe_ && b->has_event) be_.stream_wait(stream, b->ev);
        live_[b->ptr] = b;
        account_live(b, +1);
        ++stats_.pool_hits[kind];
        *out = b->ptr;
        return MM_OK;
      }
    }
    Block* b = nullptr;
    int rc = device_alloc(cls, kind, &b, msg);
    if (rc != MM_OK) return rc;
    live_[b->ptr] = b;
    account_live(b, +1);
    *out = b->ptr;
    return MM_OK;
  }

  int free(void* ptr, Stream stream, std::string* msg) {
    if (ptr == nullptr) return MM_OK;
    std::lock_guard<std::mutex> g(mu_);
    auto it = live_.find(ptr);
    if (it == live_.end()) {
      *msg = "mm_free: pointer is not a live arena block (double free or foreign pointer)";
      return MM_ERR_INVALID;
    }
    Block* b = it->second;
    live_.erase(it);
    account_live(b, -1);
    int kind = b->kind;
    // A block freed while a capture is active, or owned by a capture pool,
    // belongs to that graph until the graph is destroyed.
    int64_t owner = b->capture_id != 0 ? b->capture_id : capture_id_;
    if (owner != 0 && kind != MM_POOL_PARAMETER) {
      auto cit = captures_.find(owner);
      if (cit != captures_.end()) {
        if (b->capture_id == 0) {
          b->capture_id = owner;
          cit->second.owned.push_back(b);
        }
        cit->second.free_blocks[b->size].push_back(b);
        return MM_OK;
      }
    }
    if (kind == MM_POOL_PARAMETER || disable_pool_) {
      be_.stream_sync(stream);
      be_.free(b->ptr);
      ++stats_.device_frees;
      if (b->has_event) be_.event_destroy(b->ev);
      delete b;
      return MM_OK;
    }
    if (!b->has_event) {
      if (!be_.event_create(&b->ev)) {
        *msg = "mm_free: event creation failed";
        return MM_ERR_CUDA;
      }
      b->has_event = true;
    }
    be_.event_record(b->ev, stream);
    b->release_stream = stream;
    if (deferred_[kind]) {
      pending_[kind].push_back(b);
      stats_.pending_bytes[kind] += (int64_t)b->size;
    } else {
      cached_[kind][b->size].push_back(b);
      stats_.cached_bytes[kind] += (int64_t)b->size;
    }
    return MM_OK;
  }

  // Move completed pending blocks to the cache and return cached blocks to the
  // device.  Pending blocks whose events have not completed stay pending.
  void trim() {
    std::lock_guard<std::mutex> g(mu_);
    for (int k = 0; k < 2; ++k) drain_pending_locked(k);
    release_cached_locked();
  }

  void begin_capture(int64_t id) {
    std::lock_guard<std::mutex> g(mu_);
    capture_id_ = id;
    captures_[id];
    ++stats_.capture_pools;
  }

  void end_capture() {
    std::lock_guard<std::mutex> g(mu_);
    capture_id_ = 0;
  }

  // Free every block owned by a capture pool (the graph is gone).
  void destroy_capture(int64_t id) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = captures_.find(id);
    if (it == captures_.end()) return;
    for (Block* b : it->second.owned) {
      auto lit = live_.find(b->ptr);
      if (lit != live_.end()) {
        // Still referenced by a tensor: hand it to the global pool on its
        // eventual free instead of releasing it now.
        b->capture_id = 0;
        continue;
      }
      be_.free(b->ptr);
      ++stats_.device_frees;
      if (b->has_event) be_.event_destroy(b->ev);
      delete b;
    }
    captures_.erase(it);
    --stats_.capture_pools;
  }

  mm_pool_stats_t stats() {
    std::lock_guard<std::mutex> g(mu_);
    return stats_;
  }

  void release_all() {
    std::lock_guard<std::mutex> g(mu_);
    for (int k = 0; k < 2; ++k) {
      for (Block* b : pending_[k]) cached_[k][b->size].push_back(b);
      pending_[k].clear();
      stats_.pending_bytes[k] = 0;
    }
    release_cached_locked();
  }

  Backend& backend() { return be_; }

 private:
  void account_live(Block* b, int sign) {
    stats_.live_bytes[b->kind] += sign * (int64_t)b->size;
    if (stats_.live_bytes[b->kind] > stats_.peak_live_bytes[b->kind])
      stats_.peak_live_bytes[b->kind] = stats_.live_bytes[b->kind];
  }

  void drain_pending_locked(int kind) {
    auto& q = pending_[kind];
    while (!q.empty()) {
      Block* b = q.front();
      if (!be_.event_done(b->ev)) break;  // FIFO: later releases are newer
      q.pop_front();
      stats_.pending_bytes[kind] -= (int64_t)b->size;
      cached_[kind][b->size].push_back(b);
      stats_.cached_bytes[kind] += (int64_t)b->size;
    }
  }

  void release_cached_locked() {
    for (int k = 0; k < 2; ++k) {
      for (auto& kv : cached_[k]) {
        for (Block* b : kv.second) {
          be_.free(b->ptr);
          ++stats_.device_frees;
          if (b->has_event) be_.event_destroy(b->ev);
          delete b;
        }
      }
      cached_[k].clear();
      stats_.cached_bytes[k] = 0;
    }
  }

  int device_alloc(size_t cls, int kind, Block** out, std::string* msg) {
    void* p = nullptr;
    bool ok = try_device_malloc(cls, &p);
    if (!ok) {
      // OOM recovery: wait for the device, make every pending block reusable,
      // return the cache to the device and retry once (gpumatrix.py:4913-4923).
      ++stats_.oom_recoveries;
      be_.device_sync();
      for (int k = 0; k < 2; ++k) {
        for (Block* b : pending_[k]) cached_[k][b->size].push_back(b);
        pending_[k].clear();
        stats_.pending_bytes[k] = 0;
      }
      release_cached_locked();
      ok = try_device_malloc(cls, &p);
    }
    if (!ok) {
      *msg = "mm_alloc: out of device memory allocating " + std::to_string(cls) +
             " bytes after draining the pool";
      return MM_ERR_OOM;
    }
    ++stats_.device_mallocs;
    Block* b = new Block();
    b->ptr = p;
    b->size = cls;
    b->kind = kind;
    *out = b;
    return MM_OK;
  }

  bool try_device_malloc(size_t cls, void** p) {
    if (fail_after_ == 0) return false;
    if (!be_.malloc(p, cls)) return false;
    if (fail_after_ > 0) --fail_after_;
    return true;
  }

  Backend be_;
  std::mutex mu_;
  bool sync_safe_ = true;
  bool deferred_[2] = {false, false};
  bool disable_pool_ = false;
  int64_t fail_after_ = -1;
  int64_t capture_id_ = 0;
  std::unordered_map<void*, Block*> live_;
  std::map<size_t, std::vector<Block*>> cached_[2];
  std::deque<Block*> pending_[2];
  std::map<int64_t, CapturePool> captures_;
  mm_pool_stats_t stats_{};
};

}  // namespace mm
