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

// GELU 0.5 x (1 + erf(x / sqrt 2)) with erf from Abramowitz & Stegun 7.1.26
// (|error| <= 1.5e-7), the formula the reference's HuBERT uses
// (runtime/models/hubert.py:168-176, :194-210): t = 1 / (1 + p|u|),
// erf(|u|) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-u^2), odd in u.
__device__ __forceinline__ float gelu_as(float x) {
  const float u = x * 0.70710678118654752f;
  const float au = fabsf(u);
  const float t = 1.f / (1.f + 0.3275911f * au);
  const float poly = ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t +
                      0.254829592f) * t;
  float e = 1.f - poly * expf(-au * au);
  e = u < 0.f ? -e : e;
  return 0.5f * x * (1.f + e);
}

__device__ __forceinline__ float act_apply(float v, int act, float slope) {
  switch (act) {
    case kActLeaky: return v >= 0.f ? v : slope * v;
    case kActRelu: return v > 0.f ? v : 0.f;
    case kActTanh: return tanhf(v);
    case kActGelu: return gelu_as(v);
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
