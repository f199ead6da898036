// Tier-1 operators without a model-level counterpart: 2-D convolution and
// RMSNorm for the reference's operator dispatcher (runtime/backend.py:254,
// :309).  Plain fp32 kernels: these run per op on the caller's arrays.
#include "kernels.cuh"

namespace rvc {

namespace {

// One thread per output element y[b][o][ho][wo] of a 2-D cross-correlation
// (torch.nn.functional.conv2d semantics, zero padding): the sum runs over
// input channels, then kernel rows, then kernel columns, in fp32.
__global__ void conv2d_direct_kernel(const float* __restrict__ x, int B, int C, int H, int W,
                                     const float* __restrict__ w, int O, int KH, int KW,
                                     const float* __restrict__ bias, int sh, int sw, int ph, int pw, int Ho, int Wo,
                                     float* __restrict__ y) {
  const long long total = (long long)B * O * Ho * Wo;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int wo = (int)(i % Wo);
    long long r = i / Wo;
    const int ho = (int)(r % Ho);
    r /= Ho;
    const int o = (int)(r % O);
    const int b = (int)(r / O);
    const int h0 = ho * sh - ph, w0 = wo * sw - pw;
    float acc = 0.f;
    for (int c = 0; c < C; ++c) {
      const float* xc = x + ((long long)b * C + c) * H * W;
      const float* wc = w + ((long long)o * C + c) * KH * KW;
      for (int kh = 0; kh < KH; ++kh) {
        const int hh = h0 + kh;
        if (hh < 0 || hh >= H) continue;
        for (int kw = 0; kw < KW; ++kw) {
          const int ww = w0 + kw;
          if (ww < 0 || ww >= W) continue;
          acc = fmaf(__ldg(xc + (long long)hh * W + ww), __ldg(wc + kh * KW + kw), acc);
        }
      }
    }
    y[i] = bias ? acc + __ldg(bias + o) : acc;
  }
}

// One warp per row: y = x / sqrt(mean(x^2) + eps) * gamma, the mean of squares
// accumulated in double.
__global__ void rmsnorm_kernel(const float* __restrict__ x, long long rows, int C, const float* __restrict__ g,
                               float eps, float* __restrict__ y) {
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float* xr = x + r * C;
  double s = 0.0;
  for (int k = lane; k < C; k += 32) s += (double)xr[k] * (double)xr[k];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float inv = (float)(1.0 / sqrt(s / C + (double)eps));
  for (int k = lane; k < C; k += 32) y[r * C + k] = xr[k] * inv * g[k];
}

}  // namespace

void k_conv2d(const float* x, int B, int C, int H, int W, const float* w, int O, int KH, int KW, const float* bias,
              int sh, int sw, int ph, int pw, float* y, cudaStream_t st) {
  const int Ho = (H + 2 * ph - KH) / sh + 1, Wo = (W + 2 * pw - KW) / sw + 1;
  const long long total = (long long)B * O * Ho * Wo;
  if (total <= 0) return;
  const int grid = (int)std::min<long long>(cdiv<long long>(total, 256), 148LL * 32);
  conv2d_direct_kernel<<<grid, 256, 0, st>>>(x, B, C, H, W, w, O, KH, KW, bias, sh, sw, ph, pw, Ho, Wo, y);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

void k_rmsnorm(const float* x, long long rows, int C, const float* g, float eps, float* y, cudaStream_t st) {
  if (rows <= 0) return;
  rmsnorm_kernel<<<(unsigned)cdiv<long long>(rows, 8), 256, 0, st>>>(x, rows, C, g, eps, y);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

}  // namespace rvc
