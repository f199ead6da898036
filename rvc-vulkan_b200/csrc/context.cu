#include "context.cuh"

#include <atomic>
#include <chrono>
#include <thread>

namespace rvc {

static thread_local std::string g_last_error;
static std::atomic<long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(); }
void set_error(const std::string& msg) { g_last_error = msg; }
const std::string& get_error() { return g_last_error; }

Context::Context(int dev) : device(dev) {
  DeviceGuard g(dev);
  RVC_CUDA_TRY(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  RVC_CUDA_TRY(cudaMalloc(&d_err, sizeof(int) * 4));
  RVC_CUDA_TRY(cudaMemset(d_err, 0, sizeof(int) * 4));
}

Context::~Context() {
  DeviceGuard g(device);
  cudaStreamSynchronize(stream);
  for (auto& kv : allocs) cudaFree(kv.first);
  allocs.clear();
  for (auto& kv : pool) cudaFree(kv.second);
  pool.clear();
  for (auto& e : prof_ev) {
    cudaEventDestroy(e.a);
    cudaEventDestroy(e.b);
  }
  for (auto e : ev_pool) cudaEventDestroy(e);
  if (d_err) cudaFree(d_err);
  if (stream) cudaStreamDestroy(stream);
}

namespace {
constexpr size_t kPoolMaxBytes = size_t(16) << 30;  // cached free blocks above this are returned
size_t block_size(size_t bytes) {
  const size_t g = bytes >= (size_t(1) << 20) ? (size_t(1) << 20) : 512;  // 1 MiB granules for large blocks
  return (bytes + g - 1) / g * g;
}
}  // namespace

void Context::release_pool() {
  if (pool.empty()) return;
  cudaStreamSynchronize(stream);
  for (auto& kv : pool) cudaFree(kv.second);
  pool.clear();
  pool_bytes = 0;
}

void* Context::alloc(size_t bytes) {
  if (bytes == 0) bytes = 16;
  const size_t bs = block_size(bytes);
  if (mem_cap > 0 && mem_used + (int64_t)bs > mem_cap)
    throw Error{kErrOom, "device memory cap exceeded: need " + std::to_string(bs) + " B, used " +
                             std::to_string(mem_used) + " of " + std::to_string(mem_cap)};
  void* p = nullptr;
  size_t got = bs;
  auto it = pool.lower_bound(bs);
  if (it != pool.end() && it->first <= bs + bs / 4) {  // reuse a cached block of about this size
    got = it->first;
    p = it->second;
    pool_bytes -= got;
    pool.erase(it);
  } else {
    cudaError_t e = cudaMalloc(&p, bs);
    if (e != cudaSuccess) {  // give the cached blocks back and retry once
      cudaGetLastError();
      release_pool();
      e = cudaMalloc(&p, bs);
    }
    if (e != cudaSuccess) {
      cudaGetLastError();
      throw Error{kErrOom, std::string("cudaMalloc failed: ") + cudaGetErrorString(e)};
    }
  }
  // Zero-filled: padding rows of activation buffers must read as zeros.
  RVC_CUDA_TRY(cudaMemsetAsync(p, 0, bytes, stream));
  allocs[p] = got;
  mem_used += (int64_t)got;
  return p;
}

void Context::free(void* p) {
  auto it = allocs.find(p);
  if (it == allocs.end()) return;
  const size_t bs = it->second;
  mem_used -= (int64_t)bs;
  allocs.erase(it);
  pool.emplace(bs, p);
  pool_bytes += bs;
  if (pool_bytes > kPoolMaxBytes) {  // return the largest cached blocks
    cudaStreamSynchronize(stream);
    while (pool_bytes > kPoolMaxBytes / 2 && !pool.empty()) {
      auto last = std::prev(pool.end());
      cudaFree(last->second);
      pool_bytes -= last->first;
      pool.erase(last);
    }
  }
}

void Context::prof_begin(cudaEvent_t* a, cudaEvent_t* b) {
  auto get = [&]() {
    cudaEvent_t e;
    if (!ev_pool.empty()) {
      e = ev_pool.back();
      ev_pool.pop_back();
    } else {
      RVC_CUDA_TRY(cudaEventCreate(&e));
    }
    return e;
  };
  *a = get();
  *b = get();
  RVC_CUDA_TRY(cudaEventRecord(*a, stream));
}

void Context::prof_end(cudaEvent_t a, cudaEvent_t b, double flops, const std::string& label, bool tc) {
  RVC_CUDA_TRY(cudaEventRecord(b, stream));
  prof_ev.push_back(ProfRec{a, b, flops, label, tc});
  if (tc) {
    prof_launches += 1;
    prof_flops += flops;
  }
  if (prof_ev.size() > 4096) prof_collect();
}

void Context::prof_collect() {
  RVC_CUDA_TRY(cudaStreamSynchronize(stream));
  for (auto& e : prof_ev) {
    float ms = 0.f;
    RVC_CUDA_TRY(cudaEventElapsedTime(&ms, e.a, e.b));
    if (e.tc) prof_ms += ms;
    auto& g = prof_by_label[e.label];
    g.n += 1;
    g.ms += ms;
    g.flops += e.flops;
    ev_pool.push_back(e.a);
    ev_pool.push_back(e.b);
  }
  prof_ev.clear();
}

int32_t Context::sync(int timeout_ms) {
  if (timeout_ms <= 0) timeout_ms = 60000;
  auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t e = cudaStreamQuery(stream);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) {
      set_error(std::string("stream error: ") + cudaGetErrorString(e));
      return kErrCuda;
    }
    auto el = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (el.count() > timeout_ms) {
      set_error("rvc_cuda_sync: stream did not drain within " + std::to_string(timeout_ms) + " ms");
      return kErrTimeout;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  int herr[4] = {0, 0, 0, 0};
  cudaError_t e = cudaMemcpy(herr, d_err, sizeof(herr), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    set_error(std::string("error-flag read: ") + cudaGetErrorString(e));
    return kErrCuda;
  }
  if (herr[0] != 0) {
    cudaMemset(d_err, 0, sizeof(int) * 4);
    set_error("device wait gave up inside a kernel (code " + std::to_string(herr[0]) + ")");
    return kErrTimeout;
  }
  return kOk;
}

}  // namespace rvc
