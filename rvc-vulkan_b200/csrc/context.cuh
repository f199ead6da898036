// Per-device context: stream, device error flag, accounted device memory,
// optional per-launch profiling of the tensor-core convolutions.
#pragma once

#include "common.cuh"

#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace rvc {

struct Context : std::enable_shared_from_this<Context> {
  int device = 0;
  cudaStream_t stream = nullptr;
  int* d_err = nullptr;
  std::mutex mu;
  int64_t mem_cap = 0;   // 0 = unlimited
  int64_t mem_used = 0;
  std::unordered_map<void*, size_t> allocs;  // live blocks -> block size
  // Freed blocks kept for reuse (by size).  All device work of a context is
  // ordered on its one stream, so a block freed by one call can be handed to
  // the next without waiting: the new owner's work queues after the old one's.
  std::multimap<size_t, void*> pool;
  size_t pool_bytes = 0;
  void release_pool();
  // profiling: totals cover the tensor-core conv launches; other labelled
  // kernels (attention) are kept per label only
  bool prof = false;
  struct ProfRec { cudaEvent_t a, b; double flops; std::string label; bool tc; };
  std::vector<ProfRec> prof_ev;
  struct ProfAgg { long long n = 0; double ms = 0, flops = 0; };
  std::map<std::string, ProfAgg> prof_by_label;
  std::vector<cudaEvent_t> ev_pool;
  int64_t prof_launches = 0;
  double prof_ms = 0.0, prof_flops = 0.0;

  int sms = 0;
  int num_sms() {
    if (sms == 0 && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) sms = 148;
    return sms;
  }

  explicit Context(int dev);
  ~Context();
  void* alloc(size_t bytes);  // zero-filled
  void free(void* p);
  void prof_begin(cudaEvent_t* a, cudaEvent_t* b);
  // tc = false: recorded per label only, outside the tensor-core totals.
  void prof_end(cudaEvent_t a, cudaEvent_t b, double flops, const std::string& label, bool tc = true);
  void prof_collect();
  // Polls the stream (bounded) and the device error flag.
  int32_t sync(int timeout_ms);
};

// RAII device buffer owned by a context.
struct DevBuf {
  Context* ctx = nullptr;
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(Context* c, size_t n) : ctx(c), p(c->alloc(n)), bytes(n) {}
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : ctx(o.ctx), p(o.p), bytes(o.bytes) { o.p = nullptr; }
  DevBuf& operator=(DevBuf&& o) noexcept {
    if (this != &o) {
      reset();
      ctx = o.ctx; p = o.p; bytes = o.bytes; o.p = nullptr;
    }
    return *this;
  }
  ~DevBuf() { reset(); }
  void reset() {
    if (p && ctx) ctx->free(p);
    p = nullptr;
    bytes = 0;
  }
  template <typename T> T* as() const { return static_cast<T*>(p); }
  float* f() const { return static_cast<float*>(p); }
};

// Sets the calling thread's current device for the duration of a call.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace rvc
