// GeneratorNSF pieces that are not GEMMs: the NSF sine source and conv_post.
#include "kernels.cuh"

#include <algorithm>

namespace rvc {

// NSF source (runtime/models/vits.py:1468-1501).  Phase carry between frames:
// a float32 running sum over frames of fmod(rad_last + 0.5, 1) - 0.5 (numpy's
// cumsum is sequential, so is this), then fmod(., 1) of each prefix.  One CTA
// per chunk: the per-frame terms are computed in parallel into shared memory,
// the sequential sum runs in one thread over shared memory.
__global__ void __launch_bounds__(256) sine_phase_kernel(const float* __restrict__ f0, int P, int upp, float srf,
                                                         float* __restrict__ phase) {
  extern __shared__ float r2[];
  const int b = blockIdx.x;
  const float last = (float)upp;
  for (int t = threadIdx.x; t < P; t += blockDim.x) {
    const float rl = (f0[(long long)b * P + t] / srf) * last;
    r2[t] = fmodf(rl + 0.5f, 1.0f) - 0.5f;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float acc = 0.f;
    for (int t = 0; t < P; ++t) {
      acc = acc + r2[t];
      r2[t] = fmodf(acc, 1.0f);
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < P; t += blockDim.x) phase[(long long)b * P + t] = r2[t];
}

__global__ void sine_source_kernel(const float* __restrict__ f0, const float* __restrict__ ns,
                                   const float* __restrict__ phase, int B, int P, int upp, float srf, float lw,
                                   float lb, float* __restrict__ har) {
  const long long N = (long long)P * upp;
  const long long n = (long long)B * N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(i / N);
    const long long s = i % N;
    const int t = (int)(s / upp), j = (int)(s % upp);
    const float f = f0[(long long)b * P + t];
    float rad = (f / srf) * (float)(j + 1);
    if (t > 0) rad = rad + phase[(long long)b * P + t - 1];
    float sine = sinf(6.2831855f * rad) * 0.1f;  // float32(2*pi) * rad, as numpy
    const float uv = f > 0.f ? 1.f : 0.f;
    const float amp = uv * 0.003f + ((1.f - uv) * 0.1f) / 3.f;
    sine = sine * uv + amp * ns[i];
    har[i] = tanhf(sine * lw + lb);
  }
}

void k_sine_source(const float* f0, const float* ns, int B, int P, int upp, int sr, float lin_w, float lin_b,
                   float* phase_scratch, float* har, cudaStream_t st) {
  if (B * P == 0) return;
  RVC_CHECK_ARG((size_t)P * 4 <= 200 * 1024, "sine source: chunk longer than 51200 frames");
  if ((size_t)P * 4 > 48 * 1024)
    RVC_CUDA_TRY(cudaFuncSetAttribute(sine_phase_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  sine_phase_kernel<<<B, 256, (size_t)P * 4, st>>>(f0, P, upp, (float)sr, phase_scratch);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
  const long long n = (long long)B * P * upp;
  const int grid = (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, 148 * 32));
  sine_source_kernel<<<grid, 256, 0, st>>>(f0, ns, phase_scratch, B, P, upp, (float)sr, lin_w, lin_b, har);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

// conv_post + tanh (runtime/models/vits.py:2228-2231): one output channel, no
// bias, leaky(0.01) on the input.  A CTA stages 256 + K - 1 input rows
// (coalesced, activation applied) in shared memory; each thread then forms
// one output from shared memory.
constexpr int kPostRows = 256;
__global__ void __launch_bounds__(kPostRows) conv_post_kernel(const float* __restrict__ x, long long x_bs, int T,
                                                             int C, const float* __restrict__ w, int K, int pad,
                                                             float slope, float* __restrict__ y) {
  extern __shared__ float sx[];  // [(256+K-1)][C+1]
  float* sw = sx + (size_t)(kPostRows + K - 1) * (C + 1);  // [K][C]
  const int b = blockIdx.y;
  const int t0 = blockIdx.x * kPostRows;
  const float* xb = x + (long long)b * x_bs;
  const int rows = kPostRows + K - 1;
  for (int e = threadIdx.x; e < rows * C; e += blockDim.x) {
    const int r = e / C, c = e % C;
    const int src = t0 - pad + r;
    float v = 0.f;
    if (src >= 0 && src < T) {
      v = xb[(long long)src * C + c];
      v = v >= 0.f ? v : slope * v;
    }
    sx[r * (C + 1) + c] = v;
  }
  for (int e = threadIdx.x; e < K * C; e += blockDim.x) {
    const int k = e / C, c = e % C;
    sw[e] = w[c * K + k];
  }
  __syncthreads();
  const int t = t0 + threadIdx.x;
  if (t >= T) return;
  float s = 0.f;
  for (int k = 0; k < K; ++k) {
    const float* xr = sx + (threadIdx.x + k) * (C + 1);
    const float* wk = sw + k * C;
    for (int c = 0; c < C; ++c) s = fmaf(xr[c], wk[c], s);
  }
  y[(long long)b * T + t] = tanhf(s);
}

void k_conv_post_tanh(const float* x, long long x_bs, int B, int T, int C, const float* w, int K, int pad,
                      float slope, float* y, cudaStream_t st) {
  if ((long long)B * T == 0) return;
  const size_t smem = sizeof(float) * ((size_t)(kPostRows + K - 1) * (C + 1) + (size_t)K * C);
  RVC_CHECK_ARG(smem <= 48 * 1024, "conv_post: too many channels");
  dim3 g(cdiv(T, kPostRows), B);
  conv_post_kernel<<<g, kPostRows, smem, st>>>(x, x_bs, T, C, w, K, pad, slope, y);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

}  // namespace rvc
