// rvc_cuda_rel_attention_noalloc: the text-encoder attention operator for
// callers that must not allocate device memory.
//
// Some hosts cannot call cudaMalloc on the path that runs this operator: an
// audio callback with a hard latency budget (cudaMalloc/cudaFree can
// synchronise the whole device), or a process that has handed all device
// memory to its own arena and forbids allocations outside it.  This entry
// point takes device buffers the caller already owns and keeps its
// intermediates (the channels-last q/k/v pack and the attention output before
// it is transposed back) in one fixed array in device global memory, declared
// at file scope below.  It calls no cudaMalloc, cudaFree or allocating library
// routine.
//
// Limits and sharing rules:
//   * the array holds kNoAllocScratchFloats floats (8 MiB); every GPU that
//     loads the library keeps that much reserved until the process exits;
//   * a call needs 4 * B * heads * kc * P floats of it, larger calls are
//     rejected with RVC_E_ARG before any work is queued;
//   * every call on a device shares the one array and it keeps the last
//     call's contents; each call overwrites every element it reads before
//     reading it, so nothing has to start at zero;
//   * calls queued on different streams of the same device can overlap on
//     the GPU and would then race on the array: issue them on one context
//     (one stream), where they run one after another.
//   * the first call on a device looks up the array's device address with
//     that device current (cudaGetSymbolAddress); make that first call before
//     any stream capture begins on the device.
#include "../../include/rvc_cuda.h"
#include "context.cuh"
#include "kernels.cuh"

#include <mutex>

namespace rvc {

constexpr size_t kNoAllocScratchFloats = size_t(1) << 21;  // 8 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// In host code g_noalloc_scratch names a host-side stand-in, not device memory:
// kernels get the address resolved here, once per device, with it current.
static float* noalloc_scratch(int device) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  RVC_CHECK_ARG(device >= 0 && device < 64, "noalloc: device index out of range");
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[device]) {
    float* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress((void**)&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      throw Error{kErrCuda, std::string("noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e)};
    }
    addr[device] = p;
  }
  return addr[device];
}

}  // namespace rvc

using namespace rvc;

// Declared in the registry of capi.cu; looked up the same way.
std::shared_ptr<Context> rvc_capi_context(int64_t h);

extern "C" int32_t rvc_cuda_rel_attention_noalloc(int64_t ctx, const float* q, const float* k, const float* v,
                                                  const float* emb_k, const float* emb_v, int32_t B, int32_t heads,
                                                  int32_t kc, int32_t P, int32_t window, float* y) {
  try {
    std::shared_ptr<Context> c = rvc_capi_context(ctx);
    std::lock_guard<std::mutex> lk(c->mu);
    DeviceGuard dg(c->device);
    RVC_CHECK_ARG(B >= 0 && heads > 0 && kc > 0 && P >= 0 && window >= 0, "rel_attention_noalloc: bad shape");
    RVC_CHECK_ARG(q && k && v && emb_k && emb_v && y, "rel_attention_noalloc: null device pointer");
    RVC_CHECK_ARG(kc <= 128 && window <= 16, "rel_attention_noalloc: head dim <= 128 and window <= 16 supported");
    if ((long long)B * P == 0) return kOk;
    const long long H = (long long)heads * kc;
    const long long need = 4LL * B * H * P;
    if (need > (long long)kNoAllocScratchFloats)
      throw Error{kErrArg, "rel_attention_noalloc: needs " + std::to_string(need) + " scratch floats, the fixed array holds " +
                               std::to_string(kNoAllocScratchFloats) + " (4*B*heads*kc*P must not exceed it)"};
    float* scratch = noalloc_scratch(c->device);
    float* qkv = scratch;                  // [B, P, 3H]
    float* yt = scratch + 3LL * B * H * P;  // [B, P, H]
    const int h = (int)H;
    for (int b = 0; b < B; ++b) {
      k_nct_to_ntc(q + (size_t)b * H * P, qkv + (size_t)b * P * 3 * H, 1, h, P, 3 * h, c->stream);
      k_nct_to_ntc(k + (size_t)b * H * P, qkv + (size_t)b * P * 3 * H + H, 1, h, P, 3 * h, c->stream);
      k_nct_to_ntc(v + (size_t)b * H * P, qkv + (size_t)b * P * 3 * H + 2 * H, 1, h, P, 3 * h, c->stream);
    }
    k_rel_attention(qkv, 3 * h, 0, h, 2 * h, emb_k, emb_v, B, heads, kc, P, window, nullptr, yt, h, c->stream);
    k_ntc_to_nct(yt, h, y, B, h, P, c->stream);
    return kOk;
  } catch (const Error& e) {
    set_error(e.msg);
    return e.code;
  } catch (const std::exception& e) {
    set_error(std::string("internal error: ") + e.what());
    return kErrState;
  }
}
