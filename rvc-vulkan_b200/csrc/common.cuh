// Shared device/host helpers for librvc_cuda (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

namespace rvc {

// ---------------------------------------------------------------- errors
// Host-side status plumbing: every C-ABI call returns an int32 status and
// leaves a thread-local message (same convention as the reference's
// rvc_last_error, engine/src/ffi.zig:1110 / runtime/_vulkan.py:313-324).
enum Status : int32_t {
  kOk = 0,
  kErrArg = -1,        // bad argument / shape (Python raises ValueError)
  kErrCuda = -2,       // CUDA runtime error
  kErrTimeout = -3,    // a bounded device wait gave up
  kErrState = -4,      // object in the wrong state (missing weight, freed handle)
  kErrOom = -5,        // device allocation failed / over the caller's cap
};

void set_error(const std::string& msg);
// Counts kernel launches made by this library (all devices, all threads).
void note_launch();
long long launch_count();
const std::string& get_error();

struct Error {
  int32_t code;
  std::string msg;
};

#define RVC_CUDA_TRY(expr)                                                     \
  do {                                                                         \
    cudaError_t _e = (expr);                                                   \
    if (_e != cudaSuccess) {                                                   \
      throw ::rvc::Error{::rvc::kErrCuda, std::string(#expr) + ": " +          \
                                              cudaGetErrorString(_e)};         \
    }                                                                          \
  } while (0)

#define RVC_CHECK_ARG(cond, msg)                                               \
  do {                                                                         \
    if (!(cond)) throw ::rvc::Error{::rvc::kErrArg, std::string(msg)};         \
  } while (0)

// ---------------------------------------------------------------- device
// Activation codes shared by kernel prologues/epilogues.
enum Act : int32_t { kActNone = 0, kActLeaky = 1, kActRelu = 2, kActTanh = 3, kActGelu = 4 };

__device__ __forceinline__ float act_apply(float v, int act, float slope) {
  switch (act) {
    case kActLeaky: return v >= 0.f ? v : slope * v;
    case kActRelu: return v > 0.f ? v : 0.f;
    case kActTanh: return tanhf(v);
    case kActGelu: return 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
    default: return v;
  }
}

// fp32 -> (hi, lo) bf16 pair with hi = RN(x), lo = RN(x - hi).  x ~ hi + lo to
// ~2^-17 relative; the three products hi*hi + hi*lo + lo*hi recover fp32-grade
// GEMM accuracy on the bf16 tensor pipe.
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

__device__ __forceinline__ uint32_t pack_bf16x2(__nv_bfloat16 a, __nv_bfloat16 b) {
  return (uint32_t)__bfloat16_as_ushort(a) | ((uint32_t)__bfloat16_as_ushort(b) << 16);
}

template <typename T>
__host__ __device__ __forceinline__ T cdiv(T a, T b) { return (a + b - 1) / b; }

}  // namespace rvc
