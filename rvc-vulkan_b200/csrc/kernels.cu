// SIMT kernels for the non-GEMM parts of the hot path (see kernels.cuh).
#include "kernels.cuh"

#include <algorithm>
#include <atomic>
#include <cmath>

namespace rvc {

static inline int grid_for(long long n, int block, int cap = 148 * 32) {
  long long g = (n + block - 1) / block;
  return (int)std::max<long long>(1, std::min<long long>(g, cap));
}

#define RVC_LAUNCH_CHECK() \
  do {                      \
    note_launch();          \
    RVC_CUDA_TRY(cudaGetLastError()); \
  } while (0)

// ------------------------------------------------------------------ layout
__global__ void nct_to_ntc_kernel(const float* __restrict__ x, float* __restrict__ y, int C, int T, int y_ld) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const float* xb = x + (long long)b * C * T;
  float* yb = y + (long long)b * T * y_ld;
  for (int i = threadIdx.y; i < 32; i += 8) {
    int c = c0 + i, t = t0 + threadIdx.x;
    tile[i][threadIdx.x] = (c < C && t < T) ? xb[(long long)c * T + t] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    int t = t0 + i, c = c0 + threadIdx.x;
    if (c < C && t < T) yb[(long long)t * y_ld + c] = tile[threadIdx.x][i];
  }
}
void k_nct_to_ntc(const float* x, float* y, int B, int C, int T, int y_ld, cudaStream_t st) {
  if (B * C * T == 0) return;
  dim3 g(cdiv(T, 32), cdiv(C, 32), B);
  nct_to_ntc_kernel<<<g, dim3(32, 8), 0, st>>>(x, y, C, T, y_ld);
  RVC_LAUNCH_CHECK();
}

__global__ void ntc_to_nct_kernel(const float* __restrict__ x, int x_ld, float* __restrict__ y, int C, int T) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const float* xb = x + (long long)b * T * x_ld;
  float* yb = y + (long long)b * C * T;
  for (int i = threadIdx.y; i < 32; i += 8) {
    int t = t0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (c < C && t < T) ? xb[(long long)t * x_ld + c] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    int c = c0 + i, t = t0 + threadIdx.x;
    if (c < C && t < T) yb[(long long)c * T + t] = tile[threadIdx.x][i];
  }
}
void k_ntc_to_nct(const float* x, int x_ld, float* y, int B, int C, int T, cudaStream_t st) {
  if (B * C * T == 0) return;
  dim3 g(cdiv(T, 32), cdiv(C, 32), B);
  ntc_to_nct_kernel<<<g, dim3(32, 8), 0, st>>>(x, x_ld, y, C, T);
  RVC_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ norms
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One warp per row, two passes over registers (mean, then centred variance),
// the same two-pass formula as numpy's x.mean()/x.var() (runtime/backend.py:292-296).
template <int MAXV>
__global__ void layernorm_kernel(const float* __restrict__ x, int x_ld, const float* __restrict__ res, int res_ld,
                                 long long rows, int C, const float* __restrict__ gamma,
                                 const float* __restrict__ beta, float eps, float* __restrict__ y, int y_ld) {
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float v[MAXV];
  const float* xr = x + r * x_ld;
  const float* rr = res ? res + r * res_ld : nullptr;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    int c = lane + 32 * i;
    float a = 0.f;
    if (c < C) {
      a = xr[c];
      if (rr) a = a + rr[c];
    }
    v[i] = a;
    s += a;
  }
  const float mean = warp_sum(s) / (float)C;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    int c = lane + 32 * i;
    if (c < C) {
      float d = v[i] - mean;
      q += d * d;
    }
  }
  const float var = warp_sum(q) / (float)C;
  const float den = sqrtf(var + eps);
  float* yr = y + r * y_ld;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    int c = lane + 32 * i;
    if (c < C) yr[c] = (v[i] - mean) / den * gamma[c] + beta[c];
  }
}
void k_layernorm(const float* x, int x_ld, const float* res, int res_ld, long long rows, int C, const float* gamma,
                 const float* beta, float eps, float* y, int y_ld, cudaStream_t st) {
  if (rows == 0) return;
  RVC_CHECK_ARG(C <= 1024, "layer_norm: C > 1024 unsupported");
  int grid = (int)((rows + 7) / 8);
  if (C <= 256)
    layernorm_kernel<8><<<grid, 256, 0, st>>>(x, x_ld, res, res_ld, rows, C, gamma, beta, eps, y, y_ld);
  else
    layernorm_kernel<32><<<grid, 256, 0, st>>>(x, x_ld, res, res_ld, rows, C, gamma, beta, eps, y, y_ld);
  RVC_LAUNCH_CHECK();
}

// exp(x - max) / sum, one warp per row (runtime/backend.py:298-306).
__global__ void softmax_kernel(const float* __restrict__ x, float* __restrict__ y, long long rows, int C) {
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float* xr = x + r * C;
  float* yr = y + r * C;
  float m = -INFINITY;
  for (int c = lane; c < C; c += 32) m = fmaxf(m, xr[c]);
  m = warp_max(m);
  float s = 0.f;
  for (int c = lane; c < C; c += 32) {
    float e = expf(xr[c] - m);
    yr[c] = e;
    s += e;
  }
  s = warp_sum(s);
  for (int c = lane; c < C; c += 32) yr[c] = yr[c] / s;
}
void k_softmax_rows(const float* x, float* y, long long rows, int C, cudaStream_t st) {
  if (rows == 0) return;
  softmax_kernel<<<(int)((rows + 7) / 8), 256, 0, st>>>(x, y, rows, C);
  RVC_LAUNCH_CHECK();
}

__device__ __forceinline__ float sigmoid_np(float x) {
  // two-sided form of runtime/nn.py:520-523
  if (x >= 0.f) return 1.f / (1.f + expf(-x));
  float e = expf(x);
  return e / (1.f + e);
}

__global__ void elementwise_kernel(int op, const float* __restrict__ a, const float* __restrict__ b, long long n,
                                   float alpha, float* __restrict__ y) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    float v = a[i], r;
    switch (op) {
      case 0: r = v + b[i]; break;
      case 1: r = v * b[i]; break;
      case 2: r = v > 0.f ? v : 0.f; break;
      case 3: r = v >= 0.f ? v : alpha * v; break;
      case 4: r = gelu_as(v); break;
      case 5: r = tanhf(v); break;
      default: r = sigmoid_np(v); break;
    }
    y[i] = r;
  }
}
void k_elementwise(int op, const float* a, const float* b, long long n, float alpha, float* y, cudaStream_t st) {
  if (n == 0) return;
  elementwise_kernel<<<grid_for(n, 256), 256, 0, st>>>(op, a, b, n, alpha, y);
  RVC_LAUNCH_CHECK();
}

__global__ void embedding_kernel(const long long* __restrict__ ids, long long n, const float* __restrict__ table,
                                 int V, int E, float* __restrict__ y) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n * E; i += (long long)gridDim.x * blockDim.x) {
    long long r = i / E;
    int c = (int)(i % E);
    long long id = ids[r];
    if (id < 0) id += V;
    y[i] = table[id * E + c];
  }
}
void k_embedding(const long long* ids, long long n, const float* table, int V, int E, float* y, cudaStream_t st) {
  if (n == 0) return;
  embedding_kernel<<<grid_for(n * E, 256), 256, 0, st>>>(ids, n, table, V, E, y);
  RVC_LAUNCH_CHECK();
}

__global__ void gating_nct_kernel(const float* __restrict__ x, const float* __restrict__ g, int B, int H, int T,
                                  float* __restrict__ y) {
  long long n = (long long)B * H * T;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    int t = (int)(i % T);
    long long r = i / T;
    int c = (int)(r % H);
    int b = (int)(r / H);
    const float* xb = x + (long long)b * 2 * H * T;
    float a = xb[(long long)c * T + t], s = xb[(long long)(H + c) * T + t];
    if (g) {
      a = a + g[(long long)b * 2 * H + c];
      s = s + g[(long long)b * 2 * H + H + c];
    }
    y[i] = tanhf(a) * sigmoid_np(s);
  }
}
void k_gating_nct(const float* x, const float* g, int B, int H, int T, float* y, cudaStream_t st) {
  long long n = (long long)B * H * T;
  if (n == 0) return;
  gating_nct_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, g, B, H, T, y);
  RVC_LAUNCH_CHECK();
}

__global__ void im2col1d_kernel(const float* __restrict__ x, int B, int C, int T, int K, int stride, int pad_l,
                                int dil, int oL, float* __restrict__ cols) {
  long long n = (long long)B * oL * C * K;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    int k = (int)(i % K);
    long long r = i / K;
    int c = (int)(r % C);
    r /= C;
    int t = (int)(r % oL);
    int b = (int)(r / oL);
    int src = t * stride + k * dil - pad_l;
    cols[i] = (src >= 0 && src < T) ? x[((long long)b * C + c) * T + src] : 0.f;
  }
}
void k_im2col1d(const float* x, int B, int C, int T, int K, int stride, int pad_l, int dil, int oL, float* cols,
                cudaStream_t st) {
  long long n = (long long)B * oL * C * K;
  if (n == 0) return;
  im2col1d_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, B, C, T, K, stride, pad_l, dil, oL, cols);
  RVC_LAUNCH_CHECK();
}

// ------------------------------------------------------------ weight prep
__global__ void fold_wn_kernel(const float* __restrict__ v, const float* __restrict__ g, float* __restrict__ out,
                               int inner) {
  const int r = blockIdx.x;
  const float* vr = v + (long long)r * inner;
  float s = 0.f;
  for (int i = threadIdx.x; i < inner; i += blockDim.x) s += vr[i] * vr[i];
  __shared__ float red[32];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float norm = fmaxf(sqrtf(red[0]), 1e-12f);
  const float sc = g[r] / norm;   // w_g / ||w_v|| first, then times w_v (vits.py:440-441)
  for (int i = threadIdx.x; i < inner; i += blockDim.x) out[(long long)r * inner + i] = vr[i] * sc;
}
void k_fold_weight_norm(const float* v, const float* g, float* out, int rows, int inner, cudaStream_t st) {
  if (rows == 0) return;
  fold_wn_kernel<<<rows, 256, 0, st>>>(v, g, out, inner);
  RVC_LAUNCH_CHECK();
}

__global__ void gather_taps_kernel(const float* __restrict__ W, float* __restrict__ Wg, int O, int I, int K,
                                   int layout, const int* __restrict__ tap_k, int ntaps) {
  long long n = (long long)ntaps * I * O;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    int o = (int)(i % O);
    long long r = i / O;
    int ci = (int)(r % I);
    int j = (int)(r / I);
    int k = tap_k[j];
    Wg[i] = layout == 0 ? W[((long long)o * I + ci) * K + k] : W[((long long)ci * O + o) * K + k];
  }
}
void k_gather_taps(const float* W, float* Wg, int O, int I, int K, int layout, const int* tap_k_dev, int ntaps,
                   cudaStream_t st) {
  long long n = (long long)ntaps * I * O;
  if (n == 0) return;
  gather_taps_kernel<<<grid_for(n, 256), 256, 0, st>>>(W, Wg, O, I, K, layout, tap_k_dev, ntaps);
  RVC_LAUNCH_CHECK();
}

__global__ void gemv_rows_kernel(const float* __restrict__ W, const float* __restrict__ bias,
                                 const float* __restrict__ x, int B, int O, int I, float* __restrict__ y) {
  long long n = (long long)B * O;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    int o = (int)(i % O), b = (int)(i / O);
    float s = 0.f;
    for (int k = 0; k < I; ++k) s = fmaf(W[(long long)o * I + k], x[(long long)b * I + k], s);
    y[i] = s + (bias ? bias[o] : 0.f);
  }
}
void k_gemv_rows(const float* W, const float* bias, const float* x, int B, int O, int I, float* y, cudaStream_t st) {
  if (B * O == 0) return;
  gemv_rows_kernel<<<grid_for((long long)B * O, 128), 128, 0, st>>>(W, bias, x, B, O, I, y);
  RVC_LAUNCH_CHECK();
}

// --------------------------------------------------------- synthesizer
__global__ void enc_embed_finish_kernel(float* __restrict__ lin, const long long* __restrict__ pitch,
                                        const float* __restrict__ E, long long rows, int H, float scale) {
  long long n = rows * H;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long r = i / H;
    int c = (int)(i % H);
    long long p = pitch[r];
    if (p < 0) p += 256;
    float v = (lin[i] + E[p * H + c]) * scale;
    lin[i] = v >= 0.f ? v : 0.1f * v;
  }
}
void k_enc_embed_finish(float* lin, const long long* pitch, const float* E, long long rows, int H, float scale,
                        cudaStream_t st) {
  if (rows == 0) return;
  enc_embed_finish_kernel<<<grid_for(rows * H, 256), 256, 0, st>>>(lin, pitch, E, rows, H, scale);
  RVC_LAUNCH_CHECK();
}

// k_rel_attention lives in attention.cu.

__global__ void zp_kernel(const float* __restrict__ stats, const float* __restrict__ nz, int P, int H,
                          float* __restrict__ z, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    int c = (int)(i % H);
    long long r = i / H;
    int t = (int)(r % P);
    int b = (int)(r / P);
    const float* s = stats + r * 2 * H;
    float nzv = nz[((long long)b * H + c) * P + t];
    z[i] = s[c] + expf(s[H + c]) * nzv * 0.66666f;
  }
}
void k_zp(const float* stats, const float* nz, int B, int P, int H, float* z, cudaStream_t st) {
  long long n = (long long)B * P * H;
  if (n == 0) return;
  zp_kernel<<<grid_for(n, 256), 256, 0, st>>>(stats, nz, P, H, z, n);
  RVC_LAUNCH_CHECK();
}

__global__ void flip_kernel(const float* __restrict__ x, float* __restrict__ y, long long n, int C) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long r = i / C;
    int c = (int)(i % C);
    y[i] = x[r * C + (C - 1 - c)];
  }
}
void k_flip_channels(const float* x, float* y, long long rows, int C, cudaStream_t st) {
  if (rows == 0) return;
  flip_kernel<<<grid_for(rows * C, 256), 256, 0, st>>>(x, y, rows * C, C);
  RVC_LAUNCH_CHECK();
}

__global__ void gate_rows_kernel(const float* __restrict__ xin, long long n, int H, float* __restrict__ acts) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long r = i / H;
    int c = (int)(i % H);
    const float* xr = xin + r * 2 * H;
    acts[i] = tanhf(xr[c]) * sigmoid_np(xr[H + c]);
  }
}
void k_gate_rows(const float* xin, long long rows, int H, float* acts, cudaStream_t st) {
  if (rows == 0) return;
  gate_rows_kernel<<<grid_for(rows * H, 256), 256, 0, st>>>(xin, rows * H, H, acts);
  RVC_LAUNCH_CHECK();
}

__global__ void wn_update_kernel(float* __restrict__ h, float* __restrict__ skip, const float* __restrict__ rs,
                                 long long n, int H, int first, int last) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long r = i / H;
    int c = (int)(i % H);
    if (last) {
      skip[i] = skip[i] + rs[r * H + c];
    } else {
      const float* rr = rs + r * 2 * H;
      h[i] = h[i] + rr[c];
      skip[i] = (first ? 0.f : skip[i]) + rr[H + c];
    }
  }
}
void k_wn_update(float* h, float* skip, const float* rs, long long rows, int H, int first, int last,
                 cudaStream_t st) {
  if (rows == 0) return;
  wn_update_kernel<<<grid_for(rows * H, 256), 256, 0, st>>>(h, skip, rs, rows * H, H, first, last);
  RVC_LAUNCH_CHECK();
}

// k_sine_source, k_conv_post_tanh live in dec_kernels.cu.

// NSF noise conv (runtime/models/vits.py:1616-1636 noise_convs): a tile of
// ROWS output rows x COLS channels per CTA (COLS = 32 for 32-channel stages so
// no thread idles, else 64), each thread 4 consecutive rows x 4 channels with
// one 16-byte store per row; the source window and the weights staged in
// shared memory (weights transposed to [k][co] for conflict-free reads).  Per
// output: sum over k in order, then the bias.
constexpr int kNzMaxK = 128, kNzRpt = 4;
template <int COLS>
__global__ void __launch_bounds__(256) noise_conv_kernel(const float* __restrict__ har, long long har_bs, int har_len,
                                                         const float* __restrict__ w, const float* __restrict__ bias,
                                                         int C, int nk, int str, int pad, int T_out,
                                                         float* __restrict__ y, long long y_bs) {
  constexpr int TX = COLS / 4, TY = 256 / TX, ROWS = TY * kNzRpt;
  extern __shared__ float sm[];
  const int span = (ROWS - 1) * str + nk;
  float* hs = sm;                      // [span]
  float* ws = sm + ((span + 3) & ~3);  // [nk][COLS], 16-byte aligned for float4 reads
  const int b = blockIdx.z;
  const int t0 = blockIdx.x * ROWS, c0 = blockIdx.y * COLS;
  const float* hb = har + (long long)b * har_bs;
  const int base = t0 * str - pad;
  for (int i = threadIdx.x; i < span; i += blockDim.x) {
    const int idx = base + i;
    hs[i] = (idx >= 0 && idx < har_len) ? hb[idx] : 0.f;
  }
  for (int i = threadIdx.x; i < nk * COLS; i += blockDim.x) {
    const int k = i / COLS, c = i % COLS;
    ws[i] = (c0 + c < C) ? w[(long long)(c0 + c) * nk + k] : 0.f;
  }
  __syncthreads();
  const int tx = threadIdx.x % TX, ty = threadIdx.x / TX;
  float acc[kNzRpt][4];
#pragma unroll
  for (int r = 0; r < kNzRpt; ++r)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[r][j] = 0.f;
  for (int k = 0; k < nk; ++k) {
    const float4 wv = *reinterpret_cast<const float4*>(ws + k * COLS + tx * 4);
    const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int r = 0; r < kNzRpt; ++r) {
      const float h = hs[(ty * kNzRpt + r) * str + k];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[r][j] = fmaf(h, wa[j], acc[r][j]);
    }
  }
  const int c = c0 + tx * 4;
  float bv[4] = {0.f, 0.f, 0.f, 0.f};
  if (bias) {
#pragma unroll
    for (int j = 0; j < 4; ++j) bv[j] = c + j < C ? bias[c + j] : 0.f;
  }
#pragma unroll
  for (int r = 0; r < kNzRpt; ++r) {
    const int t = t0 + ty * kNzRpt + r;
    if (t >= T_out) continue;
    float* yr = y + (long long)b * y_bs + (long long)t * C;
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = bias ? acc[r][j] + bv[j] : acc[r][j];
    if (c + 3 < C && (C & 3) == 0) {
      *reinterpret_cast<float4*>(yr + c) = make_float4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (c + j < C) yr[c + j] = o[j];
    }
  }
}
void k_noise_conv(const float* har, long long har_bs, int har_len, const float* w, const float* bias, int C, int nk,
                  int str, int pad, int B, int T_out, float* y, long long y_bs, cudaStream_t st) {
  if (B * T_out == 0) return;
  RVC_CHECK_ARG(nk <= kNzMaxK * 4, "noise_conv: kernel too long");
  const bool narrow = C <= 32;
  const int cols = narrow ? 32 : 64, rows = (256 / (cols / 4)) * kNzRpt;
  const int span = (rows - 1) * str + nk;
  size_t smem = sizeof(float) * ((size_t)((span + 3) & ~3) + (size_t)nk * cols);
  RVC_CHECK_ARG(smem <= 200 * 1024, "noise_conv: tile does not fit in shared memory");
  RVC_CHECK_ARG(((uintptr_t)y & 15) == 0 && y_bs % 4 == 0, "noise_conv: output must be 16-byte aligned");
  static std::atomic<uint64_t> attr_done{0};
  int dev = 0;
  RVC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && !(attr_done.load() & (1ull << dev))) {
    RVC_CUDA_TRY(cudaFuncSetAttribute(noise_conv_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    RVC_CUDA_TRY(cudaFuncSetAttribute(noise_conv_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_done.fetch_or(1ull << dev);
  }
  dim3 g(cdiv(T_out, rows), cdiv(C, cols), B);
  if (narrow)
    noise_conv_kernel<32><<<g, 256, smem, st>>>(har, har_bs, har_len, w, bias, C, nk, str, pad, T_out, y, y_bs);
  else
    noise_conv_kernel<64><<<g, 256, smem, st>>>(har, har_bs, har_len, w, bias, C, nk, str, pad, T_out, y, y_bs);
  RVC_LAUNCH_CHECK();
}


// ------------------------------------------------------------------ HuBERT pieces
// GroupNorm with one group per channel over time (runtime/models/hubert.py:689-695,
// runtime/nn.py:415-440), channels-last x[b][t][c].  Stage 1: each block takes
// kGnSplit-th of the rows of one chunk, one thread per channel, and computes the
// slice mean and the centred sum of squares (two passes over its rows).
// Stage 2 merges the slices with Chan's pairwise update in double and stores
// mean and sqrt(var + eps), var = M2 / T (biased, as numpy's var).
constexpr int kGnSplit = 64;

__global__ void gn_partial_kernel(const float* __restrict__ x, long long x_bs, int T, int C, float* __restrict__ part) {
  const int b = blockIdx.y, sp = blockIdx.x;
  const int r0 = (int)((long long)T * sp / kGnSplit), r1 = (int)((long long)T * (sp + 1) / kGnSplit);
  const float* xb = x + (long long)b * x_bs;
  float* pb = part + ((long long)b * kGnSplit + sp) * 2 * C;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float s = 0.f;
    for (int r = r0; r < r1; ++r) s += xb[(long long)r * C + c];
    const int n = r1 - r0;
    const float m = n > 0 ? s / (float)n : 0.f;
    float q = 0.f;
    for (int r = r0; r < r1; ++r) {
      const float d = xb[(long long)r * C + c] - m;
      q = fmaf(d, d, q);
    }
    pb[c] = m;
    pb[C + c] = q;
  }
}

__global__ void gn_finalize_kernel(const float* __restrict__ part, int T, int C, float eps, float* __restrict__ mean,
                                   float* __restrict__ den) {
  const int b = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  double n = 0.0, m = 0.0, q = 0.0;
  for (int sp = 0; sp < kGnSplit; ++sp) {
    const int r0 = (int)((long long)T * sp / kGnSplit), r1 = (int)((long long)T * (sp + 1) / kGnSplit);
    const double nb = r1 - r0;
    if (nb == 0.0) continue;
    const float* pb = part + ((long long)b * kGnSplit + sp) * 2 * C;
    const double mb = pb[c], qb = pb[C + c];
    const double nt = n + nb, d = mb - m;
    m += d * nb / nt;
    q += qb + d * d * n * nb / nt;
    n = nt;
  }
  const float var = (float)(q / (n > 0.0 ? n : 1.0));
  mean[(long long)b * C + c] = (float)m;
  den[(long long)b * C + c] = sqrtf(var + eps);
}

__global__ void gn_apply_gelu_kernel(float* __restrict__ x, long long x_bs, int T, int C, int B,
                                     const float* __restrict__ mean, const float* __restrict__ den,
                                     const float* __restrict__ gamma, const float* __restrict__ beta) {
  const long long per = (long long)T * C / 4, n = per * B;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(i / per);
    const long long e = (i % per) * 4;
    const int c = (int)(e % C);
    float4* p = reinterpret_cast<float4*>(x + (long long)b * x_bs + e);
    float4 v = *p;
    float o[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const long long bc = (long long)b * C + c + j;
      o[j] = gelu_as((o[j] - mean[bc]) / den[bc] * gamma[c + j] + beta[c + j]);
    }
    *p = make_float4(o[0], o[1], o[2], o[3]);
  }
}

void k_groupnorm_chan_gelu(float* x, long long x_bs, int T, int C, int B, const float* gamma, const float* beta,
                           float eps, float* scratch, cudaStream_t st) {
  if (B * T == 0) return;
  RVC_CHECK_ARG(C % 4 == 0 && x_bs % 4 == 0 && ((uintptr_t)x & 15) == 0, "group_norm: C and strides must be x4");
  float* part = scratch;
  float* mean = part + (size_t)B * kGnSplit * 2 * C;
  float* den = mean + (size_t)B * C;
  gn_partial_kernel<<<dim3(kGnSplit, B), 512, 0, st>>>(x, x_bs, T, C, part);
  RVC_LAUNCH_CHECK();
  gn_finalize_kernel<<<dim3(cdiv(C, 128), B), 128, 0, st>>>(part, T, C, eps, mean, den);
  RVC_LAUNCH_CHECK();
  gn_apply_gelu_kernel<<<grid_for((long long)B * T * C / 4, 256), 256, 0, st>>>(x, x_bs, T, C, B, mean, den, gamma,
                                                                             beta);
  RVC_LAUNCH_CHECK();
}

size_t groupnorm_chan_scratch_floats(int B, int C) { return (size_t)B * kGnSplit * 2 * C + 2 * (size_t)B * C; }

// Weight norm over dims (0, 1) for each tap k (weight_norm dim=2):
// W[o][i][k] = g[k] * (v[o][i][k] / ||v[:, :, k]||), the norm summed in double
// and cast to float first (runtime/models/hubert.py:521-522).
__global__ void fold_wn_dim2_kernel(const float* __restrict__ v, const float* __restrict__ g, float* __restrict__ out,
                                    long long rows, int K) {
  const int k = blockIdx.x;
  double s = 0.0;
  for (long long r = threadIdx.x; r < rows; r += blockDim.x) {
    const double a = v[r * K + k];
    s += a * a;
  }
  __shared__ double red[256];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  const float norm = (float)sqrt(red[0]);
  const float gk = g[k];
  for (long long r = threadIdx.x; r < rows; r += blockDim.x) out[r * K + k] = gk * (v[r * K + k] / norm);
}
void k_fold_weight_norm_dim2(const float* v, const float* g, float* out, long long rows, int K, cudaStream_t st) {
  if (rows * K == 0) return;
  fold_wn_dim2_kernel<<<K, 256, 0, st>>>(v, g, out, rows, K);
  RVC_LAUNCH_CHECK();
}

// y[o][t*I + i] = W[o][i][j0 + t] for t < nt: taps j0..j0+nt-1 of a conv
// [O][I][K] become one 1-tap conv over nt*I channels (the stride-2 view).
__global__ void taps_to_channels_kernel(const float* __restrict__ W, int O, int I, int K, int j0, int nt,
                                        float* __restrict__ y) {
  const long long n = (long long)O * nt * I;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const int o = (int)(e / ((long long)nt * I));
    const int r = (int)(e % ((long long)nt * I));
    const int t = r / I, i = r % I;
    y[e] = W[((long long)o * I + i) * K + j0 + t];
  }
}
void k_taps_to_channels(const float* W, int O, int I, int K, int j0, int nt, float* y, cudaStream_t st) {
  if ((long long)O * I * nt == 0) return;
  taps_to_channels_kernel<<<grid_for((long long)O * I * nt, 256), 256, 0, st>>>(W, O, I, K, j0, nt, y);
  RVC_LAUNCH_CHECK();
}

}  // namespace rvc
