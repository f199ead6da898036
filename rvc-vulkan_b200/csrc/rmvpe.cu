// Device-resident RMVPE F0 estimator.
//
// Reference semantics: RMVPE.infer_from_audio (runtime/models/rmvpe.py:927-952):
// log-mel front end (:632-641, runtime/dsp/fft.py:59-113, runtime/dsp/mel.py:97-122),
// deep U-Net (:643-760) of ConvBlockRes (:518-547), 2x2 average pooling
// (:387-390), 3x3 stride-2 transposed convs (:319-384), cnn + BiGRU + linear +
// sigmoid (:878-897, :393-442) and the local-average decode (:899-925).
//
// Layout: channels-last images [B][H = frames][W = mel bins][C], fp32.  The
// argmax over 360 salience bins must reproduce the reference's, so the whole
// network runs in fp32 on the CUDA cores (no reduced-precision tensor-core
// split): 3x3 convs in a direct kernel over shared-memory halo tiles (row
// segments in registers, cp.async double buffering, channel-block splits for
// small grids), the stride-2 transposed convs split by output parity, 1x1
// convs and linears as an fp32 implicit GEMM; BatchNorm + ReLU + residual in
// every epilogue, in the reference's operation order.  The STFT is a batched
// cuFFT D2Z in float64 (the reference transforms in float64).  The BiGRU runs
// as one 8-CTA thread-block cluster per (direction, pair of clips): each CTA
// keeps 96 rows of the recurrent matrix in registers and broadcasts its 32 new
// hidden units to the other CTAs' shared memory every step.
#include "rmvpe.cuh"

#include <cooperative_groups.h>
#include <cufft.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>

namespace cg = cooperative_groups;

namespace rvc {

namespace {

__device__ __forceinline__ float sigmoid_two_sided(float x) {
  // runtime/nn.py:520-523
  if (x >= 0.f) return __fdiv_rn(1.f, __fadd_rn(1.f, expf(-x)));
  const float e = expf(x);
  return __fdiv_rn(e, __fadd_rn(1.f, e));
}

// numpy float32 sum of a short contiguous row (pairwise_sum, n < 128).
__device__ __forceinline__ float np_sum_small(const float* a, int n) {
  if (n < 8) {
    float s = 0.f;
    for (int i = 0; i < n; ++i) s = __fadd_rn(s, a[i]);
    return s;
  }
  float r[8];
  for (int j = 0; j < 8; ++j) r[j] = a[j];
  int i = 8;
  for (; i < n - (n % 8); i += 8)
    for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(r[j], a[i + j]);
  float s = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                      __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
  for (; i < n; ++i) s = __fadd_rn(s, a[i]);
  return s;
}

// ------------------------------------------------------------------ front end
// |rfft(frame * hann)| in float64, cast to float32: the windowed frames of the
// reflect-padded signal (pad 512 each side) go to frames[b][t][1024] (double),
// a batched cuFFT D2Z gives spec[b][t][513], then mag[b][t][k].
__global__ void stft_frames_kernel(const float* __restrict__ x, long long T, int F, const double* __restrict__ window,
                                   double* __restrict__ frames, int B) {
  const long long n_all = (long long)B * F * 1024;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n_all;
       e += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(e & 1023);
    const long long bt = e >> 10;
    const int b = (int)(bt / F), t = (int)(bt - (long long)b * F);
    long long p = (long long)t * 160 + n - 512;
    if (p < 0) p = -p;
    if (p >= T) p = 2 * (T - 1) - p;
    frames[e] = (double)x[(long long)b * T + p] * window[n];
  }
}

__global__ void stft_mag_kernel(const double2* __restrict__ spec, long long n, float* __restrict__ mag) {
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const double2 v = spec[e];
    mag[e] = (float)sqrt(v.x * v.x + v.y * v.y);
  }
}

// After the mel projection s = basis @ mag (the fp32 implicit GEMM, frames < F):
// log(clip(s, 1e-5)) per (frame, mel bin); frames >= F are the zero padding to
// a multiple of 32 (mel2hidden, :861-867).  Writes the raw log-mel [B][Fp][128]
// in place and the encoder's input BatchNorm of it.
__global__ void mel_finish_kernel(float* __restrict__ mel, int F, int Fp, int B, const float* __restrict__ s_in,
                                  const float* __restrict__ t_in, float* __restrict__ x0) {
  const long long n = (long long)B * Fp * 128;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const int t = (int)((e / 128) % Fp);
    const float v = t < F ? logf(fmaxf(mel[e], 1e-5f)) : 0.f;
    mel[e] = v;
    x0[e] = __fadd_rn(__fmul_rn(v, s_in[0]), t_in[0]);
  }
}

// ------------------------------------------------------------------ conv
struct C2Args {
  const float* x;
  long long x_bs;
  int H, W, ldi;
  int C_in, C_out, taps, transposed;
  const float* w;  // [taps][C_in][C_out]
  int OH, OW;
  float* y;
  long long y_bs, oh_s;
  int ow_s, oc_s;
  const float *bias, *scale, *shift;
  int relu, sigm;
  const float* res;
  long long res_bs;
  int ldr;
  int splits, kit;
  float* part;
  int B;
};

__device__ __forceinline__ void c2_store(const C2Args& a, int b, int m, int co, float v) {
  if (a.bias) v = __fadd_rn(v, a.bias[co]);
  if (a.scale) v = __fadd_rn(__fmul_rn(v, a.scale[co]), a.shift[co]);
  if (a.relu) v = v > 0.f ? v : 0.f;
  if (a.sigm) v = sigmoid_two_sided(v);
  if (a.res) v = __fadd_rn(v, a.res[(long long)b * a.res_bs + (long long)m * a.ldr + co]);
  const int oh = m / a.OW, ow = m - oh * a.OW;
  a.y[(long long)b * a.y_bs + (long long)oh * a.oh_s + (long long)ow * a.ow_s + (long long)co * a.oc_s] = v;
}

constexpr int kBK = 16, kTileElems = 4096;  // BM x BN output tile, 4 x 4 per thread, 256 threads

// BM x BN in {64 x 64, 128 x 32, 256 x 16}: narrow layers (16 / 32 output
// channels) take taller pixel tiles instead of idle columns.
template <int BM, int BN>
__global__ void __launch_bounds__(256) conv2d_kernel(const C2Args a) {
  constexpr int QA = BM / 16, QB = BN / 16, BS = 256 / BN;
  __shared__ __align__(16) float As[2][kBK][BM + 4];
  __shared__ __align__(16) float Bs[2][kBK][BN];
  const int tid = threadIdx.x;
  const int M = a.OH * a.OW;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int b = blockIdx.z / a.splits, sp = blockIdx.z - (blockIdx.z / a.splits) * a.splits;
  const int nci = (a.C_in + kBK - 1) / kBK;
  const int it0 = (int)((long long)a.kit * sp / a.splits), it1 = (int)((long long)a.kit * (sp + 1) / a.splits);
  const float* xb = a.x + (long long)b * a.x_bs;
  // A-load slots: pixel px = (tid >> 4) + 16 q, channel c = tid & 15
  const int ac = tid & 15;
  int aoh[QA], aow[QA];
  bool am[QA];
#pragma unroll
  for (int q = 0; q < QA; ++q) {
    const int m = m0 + (tid >> 4) + 16 * q;
    am[q] = m < M;
    aoh[q] = am[q] ? m / a.OW : 0;
    aow[q] = am[q] ? m - aoh[q] * a.OW : 0;
  }
  // B-load slots: c = tid / BN + BS q, column n = tid % BN
  const int bn = tid % BN, bco = n0 + bn;
  float ra[QA], rb[QB];
  auto load = [&](int it) {
    const int tap = it / nci, cb = it - (it / nci) * nci;
    const int ci = cb * kBK + ac;
    int dy, dx;
    if (a.taps == 9) {
      dy = tap / 3;
      dx = tap - dy * 3;
    } else {
      dy = dx = 1;
    }
#pragma unroll
    for (int q = 0; q < QA; ++q) {
      float v = 0.f;
      int ih, iw;
      bool ok = am[q] && ci < a.C_in;
      if (a.transposed) {  // out (oh, ow) takes in ((oh + 1 - ky) / 2, (ow + 1 - kx) / 2) when even
        const int h2 = aoh[q] + 1 - dy, w2 = aow[q] + 1 - dx;
        // the reference computes rows/cols < 2H-1 / 2W-1 and zero-fills the
        // output-padding row and column (runtime/models/rmvpe.py:378-384)
        ok = ok && h2 >= 0 && w2 >= 0 && !(h2 & 1) && !(w2 & 1) && aoh[q] < 2 * a.H - 1 && aow[q] < 2 * a.W - 1;
        ih = h2 >> 1;
        iw = w2 >> 1;
      } else {
        ih = aoh[q] + dy - 1;
        iw = aow[q] + dx - 1;
      }
      ok = ok && ih >= 0 && ih < a.H && iw >= 0 && iw < a.W;
      if (ok) v = __ldg(xb + ((long long)ih * a.W + iw) * a.ldi + ci);
      ra[q] = v;
    }
#pragma unroll
    for (int q = 0; q < QB; ++q) {
      const int c = cb * kBK + tid / BN + BS * q;
      rb[q] = (c < a.C_in && bco < a.C_out) ? __ldg(a.w + ((long long)tap * a.C_in + c) * a.C_out + bco) : 0.f;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int q = 0; q < QA; ++q) As[buf][ac][(tid >> 4) + 16 * q] = ra[q];
#pragma unroll
    for (int q = 0; q < QB; ++q) Bs[buf][tid / BN + BS * q][bn] = rb[q];
  };
  const int tx = tid % (BN / 4), ty = tid / (BN / 4);
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  if (it0 < it1) {
    load(it0);
    store(0);
    __syncthreads();
    for (int it = it0; it < it1; ++it) {
      const int cur = (it - it0) & 1;
      const bool more = it + 1 < it1;
      if (more) load(it + 1);
#pragma unroll
      for (int c = 0; c < kBK; ++c) {
        const float4 av = *reinterpret_cast<const float4*>(&As[cur][c][ty * 4]);
        const float4 bv = *reinterpret_cast<const float4*>(&Bs[cur][c][tx * 4]);
        const float aa[4] = {av.x, av.y, av.z, av.w}, bb[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(aa[i], bb[j], acc[i][j]);
      }
      if (more) store(cur ^ 1);
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int co = n0 + tx * 4 + j;
      if (co >= a.C_out) continue;
      if (a.splits > 1)
        a.part[(((long long)sp * a.B + b) * M + m) * a.C_out + co] = acc[i][j];
      else
        c2_store(a, b, m, co, acc[i][j]);
    }
  }
}

// Register-blocked variant for the narrow stride-1 convs: TM x TN outputs per
// thread (8 x 4), channel blocks of 8.  The per-output accumulation runs over
// (tap, input channel) in the same order as conv2d_kernel, so both kernels give
// the same sums.
constexpr int kBK8 = 8;
template <int BM, int BN, int TM, int TN>
__global__ void __launch_bounds__(256) conv2d_rb_kernel(const C2Args a) {
  static_assert((BM / TM) * (BN / TN) == 256, "256 threads");
  constexpr int QA = BM * kBK8 / 256, QB = (BN * kBK8 + 255) / 256;
  __shared__ __align__(16) float As[2][kBK8][BM + 4];
  __shared__ __align__(16) float Bs[2][kBK8][BN];
  const int tid = threadIdx.x;
  const int M = a.OH * a.OW;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int b = blockIdx.z / a.splits, sp = blockIdx.z - (blockIdx.z / a.splits) * a.splits;
  const int nci = (a.C_in + kBK8 - 1) / kBK8;
  const int it0 = (int)((long long)a.kit * sp / a.splits), it1 = (int)((long long)a.kit * (sp + 1) / a.splits);
  const float* xb = a.x + (long long)b * a.x_bs;
  // A-load slots: pixel (tid >> 3) + 32 q, channel tid & 7
  const int ac = tid & 7;
  int aoh[QA], aow[QA];
#pragma unroll
  for (int q = 0; q < QA; ++q) {
    const int m = m0 + (tid >> 3) + 32 * q;
    aoh[q] = m < M ? m / a.OW : -100000;  // out-of-range pixels never pass the bounds test
    aow[q] = m < M ? m - (m / a.OW) * a.OW : 0;
  }
  float ra[QA], rb[QB];
  auto load = [&](int it) {
    const int tap = it / nci, cb = it - (it / nci) * nci;
    const int ci = cb * kBK8 + ac;
    int dy = 1, dx = 1;
    if (a.taps == 9) {
      dy = tap / 3;
      dx = tap - dy * 3;
    }
#pragma unroll
    for (int q = 0; q < QA; ++q) {
      const int ih = aoh[q] + dy - 1, iw = aow[q] + dx - 1;
      const bool ok = ci < a.C_in && ih >= 0 && ih < a.H && iw >= 0 && iw < a.W;
      ra[q] = ok ? __ldg(xb + ((long long)ih * a.W + iw) * a.ldi + ci) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < QB; ++q) {
      const int e = tid + 256 * q;
      const int c = cb * kBK8 + e / BN, n = n0 + e % BN;
      rb[q] = (e < BN * kBK8 && c < a.C_in && n < a.C_out) ? __ldg(a.w + ((long long)tap * a.C_in + c) * a.C_out + n)
                                                            : 0.f;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int q = 0; q < QA; ++q) As[buf][ac][(tid >> 3) + 32 * q] = ra[q];
#pragma unroll
    for (int q = 0; q < QB; ++q) {
      const int e = tid + 256 * q;
      if (e < BN * kBK8) Bs[buf][e / BN][e % BN] = rb[q];
    }
  };
  const int tx = tid % (BN / TN), ty = tid / (BN / TN);
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
  if (it0 < it1) {
    load(it0);
    store(0);
    __syncthreads();
    for (int it = it0; it < it1; ++it) {
      const int cur = (it - it0) & 1;
      const bool more = it + 1 < it1;
      if (more) load(it + 1);
#pragma unroll
      for (int c = 0; c < kBK8; ++c) {
        float aa[TM], bb[TN];
#pragma unroll
        for (int i = 0; i < TM; i += 4) {
          const float4 v = *reinterpret_cast<const float4*>(&As[cur][c][ty * TM + i]);
          aa[i] = v.x; aa[i + 1] = v.y; aa[i + 2] = v.z; aa[i + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < TN; j += 4) {
          const float4 v = *reinterpret_cast<const float4*>(&Bs[cur][c][tx * TN + j]);
          bb[j] = v.x; bb[j + 1] = v.y; bb[j + 2] = v.z; bb[j + 3] = v.w;
        }
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(aa[i], bb[j], acc[i][j]);
      }
      if (more) store(cur ^ 1);
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + ty * TM + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int co = n0 + tx * TN + j;
      if (co >= a.C_out) continue;
      if (a.splits > 1)
        a.part[(((long long)sp * a.B + b) * M + m) * a.C_out + co] = acc[i][j];
      else
        c2_store(a, b, m, co, acc[i][j]);
    }
  }
}

// Packed fp32 pairs for the sm_100 fma.rn.f32x2 instruction: two independent
// fused multiply-adds, round to nearest, in one instruction; each half's
// result is the one fmaf gives.
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ void fma2(unsigned long long& c, unsigned long long a, unsigned long long b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c) : "l"(a), "l"(b));
}

// 4-byte global -> shared copy without a register round trip; n = 0 copies
// nothing and writes zero (the source must still be a valid address).
__device__ __forceinline__ void cp_async4(float* dst, const float* src, int n) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Direct 3x3 stride-1 conv over a shared-memory halo tile: per block of CK
// input channels the (TH+2) x (TW+2) input pixels of a TH x TW output tile are
// loaded once and serve all nine taps (the implicit-GEMM kernels re-read them
// per tap).  Each thread owns TMP consecutive pixels of one output row x TNC
// channels (in quads NT x 4 apart, so a warp's float4 weight loads are
// contiguous); per input channel and kernel row it reads the TMP + 2 halo
// values of that row into registers once and applies the three kernel columns
// from there.  Halo and weights are double-buffered: cp.async fills channel
// block cb + 1 while block cb is summed.  Optional split over the channel
// blocks (blockIdx.z = clip x split): partial sums go to a.part and
// conv2d_reduce_kernel adds them in split order.
// Accumulation order per output: channel block, channel, kernel row, column.
template <int BN, int TNC, int TMP, int CK>
__global__ void __launch_bounds__(256, 2) conv3x3_direct_kernel(const C2Args a, int TW) {
  constexpr int NT = BN / TNC;         // threads across the channel block
  constexpr int TPX = 256 / NT * TMP;  // pixels per tile
  constexpr int WST = 9 * CK * BN;     // one weight stage [9][CK][BN]
  extern __shared__ __align__(16) float dsm[];
  const int TH = TPX / TW;
  const int HW = TW + 2;
  const int npx = (TH + 2) * HW;
  const int HST = (npx * (CK + 1) + 3) & ~3;  // one halo stage [(TH+2)(TW+2)][CK+1], 16-byte multiple
  float* wts = dsm;                           // [2][WST]
  float* halo = dsm + 2 * WST;                // [2][HST]
  const int tid = threadIdx.x;
  const int tilesW = (a.OW + TW - 1) / TW;
  const int h0 = (blockIdx.x / tilesW) * TH, w0 = (blockIdx.x % tilesW) * TW;
  const int n0 = blockIdx.y * BN;
  const int b = blockIdx.z / a.splits, sp = blockIdx.z - b * a.splits;
  const int ncb = (a.C_in + CK - 1) / CK;
  const int cb0 = (int)((long long)ncb * sp / a.splits), cb1 = (int)((long long)ncb * (sp + 1) / a.splits);
  const float* xb = a.x + (long long)b * a.x_bs;
  const int tn = tid % NT, tg = tid / NT;
  const int p0 = tg * TMP, pr = p0 / TW, pc = p0 % TW;  // first pixel of this thread (tile coordinates)
  auto issue = [&](int cb, int st) {
    const int c0 = cb * CK;
    float* hs = halo + st * HST;
    for (int e = tid; e < npx * CK; e += 256) {
      const int px = e / CK, c = e % CK;
      const int ih = h0 - 1 + px / HW, iw = w0 - 1 + px % HW;
      const bool ok = ih >= 0 && ih < a.H && iw >= 0 && iw < a.W && c0 + c < a.C_in;
      cp_async4(hs + px * (CK + 1) + c, ok ? xb + ((long long)ih * a.W + iw) * a.ldi + c0 + c : xb, ok ? 4 : 0);
    }
    float* ws = wts + st * WST;
    for (int e = tid; e < WST; e += 256) {
      const int n = e % BN, c = (e / BN) % CK, tap = e / (BN * CK);
      const bool ok = c0 + c < a.C_in && n0 + n < a.C_out;
      cp_async4(ws + e, ok ? a.w + ((long long)tap * a.C_in + c0 + c) * a.C_out + n0 + n : a.w, ok ? 4 : 0);
    }
    cp_async_commit();
  };
  // channel pairs (j, j + 1) packed for fma.rn.f32x2 (zero bits = (0.f, 0.f))
  unsigned long long acc2[TMP][TNC / 2];
#pragma unroll
  for (int i = 0; i < TMP; ++i)
#pragma unroll
    for (int j = 0; j < TNC / 2; ++j) acc2[i][j] = 0ull;
  if (cb0 < cb1) issue(cb0, 0);
  for (int cb = cb0; cb < cb1; ++cb) {
    const int st = (cb - cb0) & 1;
    if (cb + 1 < cb1) {
      issue(cb + 1, st ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* hs = halo + st * HST;
    const float* ws = wts + st * WST;
#pragma unroll 2
    for (int c = 0; c < CK; ++c) {
#pragma unroll
      for (int dy = 0; dy < 3; ++dy) {
        float r[TMP + 2];
        const float* hp = hs + ((pr + dy) * HW + pc) * (CK + 1) + c;
#pragma unroll
        for (int k = 0; k < TMP + 2; ++k) r[k] = hp[k * (CK + 1)];
#pragma unroll
        for (int dx = 0; dx < 3; ++dx) {
          unsigned long long wv2[TNC / 2];
#pragma unroll
          for (int q = 0; q < TNC / 4; ++q) {
            const float4 v = *reinterpret_cast<const float4*>(ws + ((dy * 3 + dx) * CK + c) * BN + q * NT * 4 + tn * 4);
            wv2[2 * q] = pack2(v.x, v.y);
            wv2[2 * q + 1] = pack2(v.z, v.w);
          }
          // two channels per packed FMA: acc += r * w per output, as fmaf in the same order
#pragma unroll
          for (int i = 0; i < TMP; ++i) {
            const unsigned long long x2 = pack2(r[i + dx], r[i + dx]);
#pragma unroll
            for (int j = 0; j < TNC / 2; ++j) fma2(acc2[i][j], x2, wv2[j]);
          }
        }
      }
    }
    __syncthreads();  // stage st is refilled by the next iteration's issue
  }
  const int oh = h0 + pr;
  if (oh >= a.OH) return;
  const long long M = (long long)a.OH * a.OW;
  float acc[TMP][TNC];
#pragma unroll
  for (int i = 0; i < TMP; ++i)
#pragma unroll
    for (int j = 0; j < TNC / 2; ++j) unpack2(acc2[i][j], acc[i][2 * j], acc[i][2 * j + 1]);
#pragma unroll
  for (int i = 0; i < TMP; ++i) {
    const int ow = w0 + pc + i;
    if (ow >= a.OW) continue;
#pragma unroll
    for (int j = 0; j < TNC; ++j) {
      const int co = n0 + (j / 4) * (NT * 4) + tn * 4 + (j % 4);
      if (co >= a.C_out) continue;
      if (a.splits > 1)
        a.part[(((long long)sp * a.B + b) * M + (long long)oh * a.OW + ow) * a.C_out + co] = acc[i][j];
      else
        c2_store(a, b, oh * a.OW + ow, co, acc[i][j]);
    }
  }
}

// Direct 3x3 stride-2 transposed conv, split by output parity: output
// (2i + ph, 2j + pw) takes kernel row 1 from input row i when ph = 0, rows 0
// and 2 from input rows i + 1 and i when ph = 1 (columns likewise), so each
// output sums 1, 2, 2 or 4 taps instead of masking nine.  Each thread owns one
// output row x TMP input columns (2 TMP output columns) x TNC channels; pixel
// groups are ordered by row parity so a warp's branch is uniform.  The
// reference computes rows / columns < 2H - 1 / 2W - 1 only and zero-fills the
// output-padding row and column (runtime/models/rmvpe.py:378-384): those sums
// are zeroed before the epilogue.  Same double-buffered halo / weights and
// channel-block split as conv3x3_direct_kernel.
// Accumulation order per output: channel block, channel, kernel row, column.
template <int BN, int TNC, int TMP, int CK>
__global__ void __launch_bounds__(256, 2) convT3x3_direct_kernel(const C2Args a, int TW) {
  constexpr int NT = BN / TNC;
  constexpr int G = 256 / NT;  // pixel groups per tile
  constexpr int WST = 9 * CK * BN;
  extern __shared__ __align__(16) float dsm[];
  const int gpr = TW / TMP;  // groups per output row
  const int OHt = G / gpr;   // output rows per tile (even)
  const int IR = OHt / 2 + 1, IW = TW + 1;
  const int npx = IR * IW;
  const int HST = (npx * (CK + 1) + 3) & ~3;
  float* wts = dsm;
  float* halo = dsm + 2 * WST;
  const int tid = threadIdx.x;
  const int tilesW = (a.W + TW - 1) / TW;
  const int oh0 = (blockIdx.x / tilesW) * OHt, w0 = (blockIdx.x % tilesW) * TW;  // w0: input column
  const int i0 = oh0 / 2;
  const int n0 = blockIdx.y * BN;
  const int b = blockIdx.z / a.splits, sp = blockIdx.z - b * a.splits;
  const int ncb = (a.C_in + CK - 1) / CK;
  const int cb0 = (int)((long long)ncb * sp / a.splits), cb1 = (int)((long long)ncb * (sp + 1) / a.splits);
  const float* xb = a.x + (long long)b * a.x_bs;
  const int tn = tid % NT, g = tid / NT;
  const int ph = g / (G / 2), rem = g % (G / 2);
  const int rr = rem / gpr, pc = (rem % gpr) * TMP;
  const int oh = oh0 + 2 * rr + ph;  // input row i0 + rr is local halo row rr
  auto issue = [&](int cb, int st) {
    const int c0 = cb * CK;
    float* hs = halo + st * HST;
    for (int e = tid; e < npx * CK; e += 256) {
      const int px = e / CK, c = e % CK;
      const int ih = i0 + px / IW, iw = w0 + px % IW;
      const bool ok = ih < a.H && iw < a.W && c0 + c < a.C_in;
      cp_async4(hs + px * (CK + 1) + c, ok ? xb + ((long long)ih * a.W + iw) * a.ldi + c0 + c : xb, ok ? 4 : 0);
    }
    float* ws = wts + st * WST;
    for (int e = tid; e < WST; e += 256) {
      const int n = e % BN, c = (e / BN) % CK, tap = e / (BN * CK);
      const bool ok = c0 + c < a.C_in && n0 + n < a.C_out;
      cp_async4(ws + e, ok ? a.w + ((long long)tap * a.C_in + c0 + c) * a.C_out + n0 + n : a.w, ok ? 4 : 0);
    }
    cp_async_commit();
  };
  float acc[TMP][2][TNC];
#pragma unroll
  for (int i = 0; i < TMP; ++i)
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
      for (int j = 0; j < TNC; ++j) acc[i][p][j] = 0.f;
  if (cb0 < cb1) issue(cb0, 0);
  for (int cb = cb0; cb < cb1; ++cb) {
    const int st = (cb - cb0) & 1;
    if (cb + 1 < cb1) {
      issue(cb + 1, st ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* hs = halo + st * HST;
    const float* ws = wts + st * WST;
#pragma unroll 2
    for (int c = 0; c < CK; ++c) {
      // kernel row ky read from local input row lr: column taps kx = 1 (even
      // outputs, column j), then kx = 0 (column j + 1) and kx = 2 (column j)
      auto krow = [&](int ky, int lr) {
        float r[TMP + 1];
        const float* hp = hs + (lr * IW + pc) * (CK + 1) + c;
#pragma unroll
        for (int k = 0; k < TMP + 1; ++k) r[k] = hp[k * (CK + 1)];
        float wv[TNC];
        auto wload = [&](int kx) {
#pragma unroll
          for (int q = 0; q < TNC / 4; ++q) {
            const float4 v = *reinterpret_cast<const float4*>(ws + ((ky * 3 + kx) * CK + c) * BN + q * NT * 4 + tn * 4);
            wv[4 * q] = v.x; wv[4 * q + 1] = v.y; wv[4 * q + 2] = v.z; wv[4 * q + 3] = v.w;
          }
        };
        wload(1);
#pragma unroll
        for (int t = 0; t < TMP; ++t)
#pragma unroll
          for (int j = 0; j < TNC; ++j) acc[t][0][j] = fmaf(r[t], wv[j], acc[t][0][j]);
        wload(0);
#pragma unroll
        for (int t = 0; t < TMP; ++t)
#pragma unroll
          for (int j = 0; j < TNC; ++j) acc[t][1][j] = fmaf(r[t + 1], wv[j], acc[t][1][j]);
        wload(2);
#pragma unroll
        for (int t = 0; t < TMP; ++t)
#pragma unroll
          for (int j = 0; j < TNC; ++j) acc[t][1][j] = fmaf(r[t], wv[j], acc[t][1][j]);
      };
      if (ph == 0) {
        krow(1, rr);
      } else {
        krow(0, rr + 1);
        krow(2, rr);
      }
    }
    __syncthreads();  // stage st is refilled by the next iteration's issue
  }
  if (oh >= a.OH) return;
  const bool zrow = oh == 2 * a.H - 1;
  const long long M = (long long)a.OH * a.OW;
#pragma unroll
  for (int t = 0; t < TMP; ++t) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int ow = 2 * (w0 + pc + t) + p;
      if (ow >= a.OW) continue;
      const bool zero = zrow || ow == 2 * a.W - 1;
#pragma unroll
      for (int j = 0; j < TNC; ++j) {
        const int co = n0 + (j / 4) * (NT * 4) + tn * 4 + (j % 4);
        if (co >= a.C_out) continue;
        const float v = zero ? 0.f : acc[t][p][j];
        if (a.splits > 1)
          a.part[(((long long)sp * a.B + b) * M + (long long)oh * a.OW + ow) * a.C_out + co] = v;
        else
          c2_store(a, b, oh * a.OW + ow, co, v);
      }
    }
  }
}

// Split-K: partial sums added in split order, then the epilogue.
__global__ void conv2d_reduce_kernel(const C2Args a) {
  const long long M = (long long)a.OH * a.OW, per = M * a.C_out, n = per * a.B;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(e / per);
    const long long r = e - (long long)b * per;
    const int m = (int)(r / a.C_out), co = (int)(r - (long long)m * a.C_out);
    float v = a.part[e];
    for (int s = 1; s < a.splits; ++s) v = __fadd_rn(v, a.part[(long long)s * n + e]);
    c2_store(a, b, m, co, v);
  }
}

// 2x2 average pooling: ((x00 + x01) + x10) + x11, times 1/4 (numpy's reduce order
// over the two pooled axes, then the mean's division by 4).
__global__ void avgpool_kernel(const float* __restrict__ x, long long x_bs, int H, int W, int C, int ldi,
                               float* __restrict__ y, long long y_bs, int B) {
  const int OH = H / 2, OW = W / 2;
  const long long per = (long long)OH * OW * C, n = per * B;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(e / per);
    long long r = e - (long long)b * per;
    const int c = (int)(r % C);
    r /= C;
    const int ow = (int)(r % OW), oh = (int)(r / OW);
    const float* p = x + (long long)b * x_bs + ((long long)(2 * oh) * W + 2 * ow) * ldi + c;
    const float s = __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[ldi]), p[(long long)W * ldi]), p[(long long)W * ldi + ldi]);
    y[(long long)b * y_bs + ((long long)oh * OW + ow) * C + c] = __fmul_rn(s, 0.25f);
  }
}

// ------------------------------------------------------------------ BiGRU
// One 8-CTA cluster per (direction, group of kGruBg sequences).  CTA `rank`
// owns hidden units [32 rank, 32 rank + 32): the 96 rows g*256 + unit of the
// recurrent matrix for the gates g = r, z, n, held in registers (warp w: rows
// 8w..8w+7, lane l: columns l + 32k).  Per step: gh = W_hh h + b_hh for those
// rows, the gate update of its 32 units, a store of the new units into every
// CTA's next h buffer (distributed shared memory), then one cluster barrier.
// gx = x W_ih^T + b_ih is precomputed for both directions.
constexpr int kGruCta = 8, kGruUnits = 32, kGruRows = 96, kGruThreads = 384, kGruBg = 2;

__global__ void __cluster_dims__(kGruCta, 1, 1) __launch_bounds__(kGruThreads)
    gru_kernel(const float* __restrict__ gx, const float* __restrict__ whh, const float* __restrict__ bhh, int B,
               int T, float* __restrict__ out) {
  __shared__ float hb[2][kGruBg][256];
  __shared__ float gh[kGruBg][kGruRows];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int cid = blockIdx.x / kGruCta;
  const int dir = cid & 1, b0 = (cid >> 1) * kGruBg;
  const int nb = min(kGruBg, B - b0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* W = whh + (long long)dir * 768 * 256;
  float w[8][8], bias_row[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int rr = warp * 8 + q;
    const int row = (rr / kGruUnits) * 256 + rank * kGruUnits + (rr % kGruUnits);
#pragma unroll
    for (int k = 0; k < 8; ++k) w[q][k] = W[(long long)row * 256 + lane + 32 * k];
    bias_row[q] = bhh[dir * 768 + row];
  }
  for (int e = tid; e < 2 * kGruBg * 256; e += kGruThreads) (&hb[0][0][0])[e] = 0.f;
  cluster.sync();
  const int gu = tid % kGruUnits, gb = tid / kGruUnits;  // gate threads: unit, sequence
  const bool gate = gb < nb;
  const int j = rank * kGruUnits + gu;
  // the input gates of step s + 1 are loaded during step s, so the recurrence
  // does not wait on a global load
  float nx[3] = {0.f, 0.f, 0.f};
  auto fetch = [&](int s2) {
    if (gate && s2 < T) {
      const int t2 = dir == 0 ? s2 : T - 1 - s2;
      const float* g = gx + ((long long)(b0 + gb) * T + t2) * 1536 + dir * 768;
      nx[0] = g[j];
      nx[1] = g[256 + j];
      nx[2] = g[512 + j];
    }
  };
  fetch(0);
  for (int s = 0; s < T; ++s) {
    const int tt = dir == 0 ? s : T - 1 - s;
    const int cur = s & 1, nxt = cur ^ 1;
    const float gxr = nx[0], gxz = nx[1], gxn = nx[2];
    fetch(s + 1);
    for (int bb = 0; bb < nb; ++bb) {
      float hv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) hv[k] = hb[cur][bb][lane + 32 * k];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) acc = fmaf(w[q][k], hv[k], acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) gh[bb][warp * 8 + q] = __fadd_rn(acc, bias_row[q]);
      }
    }
    __syncthreads();
    if (gate) {
      const float r = sigmoid_two_sided(__fadd_rn(gxr, gh[gb][gu]));
      const float z = sigmoid_two_sided(__fadd_rn(gxz, gh[gb][kGruUnits + gu]));
      const float n = tanhf(__fadd_rn(gxn, __fmul_rn(r, gh[gb][2 * kGruUnits + gu])));
      const float hp = hb[cur][gb][j];
      const float hn = __fadd_rn(__fmul_rn(__fsub_rn(1.f, z), n), __fmul_rn(z, hp));
      out[((long long)(b0 + gb) * T + tt) * 512 + dir * 256 + j] = hn;
      float* dst = &hb[nxt][gb][j];
#pragma unroll
      for (int r2 = 0; r2 < kGruCta; ++r2) *cluster.map_shared_rank(dst, r2) = hn;
    }
    cluster.sync();
  }
}

// ------------------------------------------------------------------ decode
__global__ void decode_kernel(const float* __restrict__ sal, int Fp, int F, float thred, float* __restrict__ f0,
                              int* __restrict__ amax, int B) {
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= (long long)B * F) return;
  const int b = (int)(row / F), t = (int)(row - (long long)b * F);
  const float* s = sal + ((long long)b * Fp + t) * 360;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = lane; c < 360; c += 32) {
    const float v = s[c];
    if (v > best || (v == best && c < bi)) {
      best = v;
      bi = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (lane != 0) return;
  float ts[9], pr[9];
  for (int q = 0; q < 9; ++q) {
    const int c = bi + q - 4;  // window in unpadded bins; the 4-bin zero pads read 0
    const int p = bi + q;      // padded cents index
    const float v = (c >= 0 && c < 360) ? s[c] : 0.f;
    const float cents = (p >= 4 && p < 364) ? (float)(20.0 * (p - 4) + 1997.3794084376191) : 0.f;
    ts[q] = v;
    pr[q] = __fmul_rn(v, cents);
  }
  float cents = __fdiv_rn(np_sum_small(pr, 9), np_sum_small(ts, 9));
  const float maxx = best > 0.f ? best : 0.f;  // the max of the zero-padded row
  if (maxx <= thred) cents = 0.f;
  float f = __fmul_rn(10.f, powf(2.f, __fdiv_rn(cents, 1200.f)));
  if (f == 10.f) f = 0.f;
  f0[(long long)b * F + t] = f;
  if (amax) amax[(long long)b * F + t] = bi;
}

int grid_for(long long n, int block) {
  return (int)std::max<long long>(1, std::min<long long>((n + block - 1) / block, 148ll * 16));
}

}  // namespace

// ================================================================== model
RmvpeModel::RmvpeModel(Context* c) : ctx(c) {}

RmvpeModel::~RmvpeModel() {
  if (!fft_plans_.empty()) cudaStreamSynchronize(ctx->stream);  // no transform still in flight
  for (auto& kv : fft_plans_) cufftDestroy((cufftHandle)kv.second);
}

void RmvpeModel::set_weight(const std::string& key, const float* host, const std::vector<int64_t>& shape) {
  RmvpeTensor t;
  t.shape = shape;
  t.buf = DevBuf(ctx, sizeof(float) * (size_t)std::max<int64_t>(1, t.numel()));
  RVC_CUDA_TRY(cudaMemcpyAsync(t.buf.p, host, sizeof(float) * t.numel(), cudaMemcpyHostToDevice, ctx->stream));
  RVC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  raw_[key] = std::move(t);
  finalized_ = false;
}

const RmvpeTensor& RmvpeModel::W(const std::string& key) const {
  auto it = raw_.find(key);
  if (it == raw_.end()) throw Error{kErrState, "rmvpe: missing weight '" + key + "'"};
  return it->second;
}

namespace {
// scale = gamma / sqrt(var + 1e-5), shift = beta - mean * scale (float32, :507-515)
__global__ void bn_fold_kernel(const float* g, const float* bt, const float* rm, const float* rv, int C, float* s,
                               float* t) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const float sc = __fdiv_rn(g[c], __fsqrt_rn(__fadd_rn(rv[c], 1e-5f)));
  s[c] = sc;
  t[c] = __fsub_rn(bt[c], __fmul_rn(rm[c], sc));
}
// w [O][I][kh][kw] (conv) or [I][O][kh][kw] (transposed) -> [kh*kw][I][O]
__global__ void conv_w_kernel(const float* w, int O, int I, int taps, int transposed, float* out) {
  const long long n = (long long)taps * I * O;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const int o = (int)(e % O);
    const long long r = e / O;
    const int i = (int)(r % I), tap = (int)(r / I);
    out[e] = transposed ? w[((long long)i * O + o) * taps + tap] : w[((long long)o * I + i) * taps + tap];
  }
}
}  // namespace

void RmvpeModel::bn_fold(const std::string& p, DevBuf& scale, DevBuf& shift, int C) {
  for (const char* s : {".weight", ".bias", ".running_mean", ".running_var"})
    RVC_CHECK_ARG(W(p + s).numel() == C, "rmvpe: BatchNorm '" + p + "' does not have " + std::to_string(C) + " channels");
  scale = DevBuf(ctx, sizeof(float) * C);
  shift = DevBuf(ctx, sizeof(float) * C);
  bn_fold_kernel<<<(C + 127) / 128, 128, 0, ctx->stream>>>(W(p + ".weight").buf.f(), W(p + ".bias").buf.f(),
                                                            W(p + ".running_mean").buf.f(),
                                                            W(p + ".running_var").buf.f(), C, scale.f(), shift.f());
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

static Conv2dW make_conv(Context* ctx, const RmvpeTensor& w, bool transposed, const std::string& key) {
  RVC_CHECK_ARG(w.shape.size() == 4 && w.shape[2] == w.shape[3] && (w.shape[2] == 3 || w.shape[2] == 1),
                "rmvpe: conv weight '" + key + "' must be [*, *, 3, 3] or [*, *, 1, 1]");
  Conv2dW L;
  L.transposed = transposed;
  L.taps = (int)(w.shape[2] * w.shape[3]);
  L.C_out = (int)(transposed ? w.shape[1] : w.shape[0]);
  L.C_in = (int)(transposed ? w.shape[0] : w.shape[1]);
  L.w = DevBuf(ctx, sizeof(float) * (size_t)L.taps * L.C_in * L.C_out);
  conv_w_kernel<<<grid_for(w.numel(), 256), 256, 0, ctx->stream>>>(w.buf.f(), L.C_out, L.C_in, L.taps, transposed,
                                                                   L.w.f());
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
  return L;
}

void RmvpeModel::build_block(const std::string& p, int cin, int cout) {
  Conv2dW c0 = make_conv(ctx, W(p + ".conv.0.weight"), false, p + ".conv.0.weight");
  RVC_CHECK_ARG(c0.C_in == cin && c0.C_out == cout && c0.taps == 9, "rmvpe: unexpected shape of " + p + ".conv.0");
  bn_fold(p + ".conv.1", c0.scale, c0.shift, cout);
  Conv2dW c3 = make_conv(ctx, W(p + ".conv.3.weight"), false, p + ".conv.3.weight");
  RVC_CHECK_ARG(c3.C_in == cout && c3.C_out == cout && c3.taps == 9, "rmvpe: unexpected shape of " + p + ".conv.3");
  bn_fold(p + ".conv.4", c3.scale, c3.shift, cout);
  convs_[p + ".conv.0"] = std::move(c0);
  convs_[p + ".conv.3"] = std::move(c3);
  if (cin != cout) {
    Conv2dW sc = make_conv(ctx, W(p + ".shortcut.weight"), false, p + ".shortcut.weight");
    RVC_CHECK_ARG(sc.taps == 1 && sc.C_in == cin && sc.C_out == cout, "rmvpe: unexpected shortcut shape in " + p);
    if (raw_.count(p + ".shortcut.bias")) {
      sc.bias = DevBuf(ctx, sizeof(float) * cout);
      RVC_CUDA_TRY(cudaMemcpyAsync(sc.bias.p, W(p + ".shortcut.bias").buf.p, sizeof(float) * cout,
                                   cudaMemcpyDeviceToDevice, ctx->stream));
    }
    convs_[p + ".shortcut"] = std::move(sc);
  } else {
    RVC_CHECK_ARG(!raw_.count(p + ".shortcut.weight"), "rmvpe: shortcut in an equal-width block " + p);
  }
}

static const int kEnc[5][2] = {{1, 16}, {16, 32}, {32, 64}, {64, 128}, {128, 256}};
static const int kInter[4][2] = {{256, 512}, {512, 512}, {512, 512}, {512, 512}};
static const int kDec[5][2] = {{512, 256}, {256, 128}, {128, 64}, {64, 32}, {32, 16}};

void RmvpeModel::finalize() {
  cudaStream_t st = ctx->stream;
  convs_.clear();
  bn_fold("unet.encoder.bn", in_scale_, in_shift_, 1);
  for (int i = 0; i < 5; ++i)
    for (int j = 0; j < 4; ++j)
      build_block("unet.encoder.layers." + std::to_string(i) + ".conv." + std::to_string(j), j == 0 ? kEnc[i][0] : kEnc[i][1],
                  kEnc[i][1]);
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 4; ++j)
      build_block("unet.intermediate.layers." + std::to_string(i) + ".conv." + std::to_string(j),
                  j == 0 ? kInter[i][0] : kInter[i][1], kInter[i][1]);
  for (int i = 0; i < 5; ++i) {
    const std::string p = "unet.decoder.layers." + std::to_string(i);
    Conv2dW ct = make_conv(ctx, W(p + ".conv1.0.weight"), true, p + ".conv1.0.weight");
    RVC_CHECK_ARG(ct.taps == 9 && ct.C_in == kDec[i][0] && ct.C_out == kDec[i][1], "rmvpe: unexpected " + p + ".conv1.0");
    bn_fold(p + ".conv1.1", ct.scale, ct.shift, kDec[i][1]);
    convs_[p + ".conv1"] = std::move(ct);
    for (int j = 0; j < 4; ++j)
      build_block(p + ".conv2." + std::to_string(j), j == 0 ? 2 * kDec[i][1] : kDec[i][1], kDec[i][1]);
  }
  {
    Conv2dW cnn = make_conv(ctx, W("cnn.weight"), false, "cnn.weight");
    RVC_CHECK_ARG(cnn.C_in == 16 && cnn.C_out == 3 && cnn.taps == 9, "rmvpe: cnn.weight must be [3,16,3,3]");
    cnn.bias = DevBuf(ctx, sizeof(float) * 3);
    RVC_CUDA_TRY(cudaMemcpyAsync(cnn.bias.p, W("cnn.bias").buf.p, sizeof(float) * 3, cudaMemcpyDeviceToDevice, st));
    convs_["cnn"] = std::move(cnn);
  }
  {
    // GRU input projection of both directions as one [384 -> 1536] 1x1 conv
    Conv2dW gi;
    gi.C_in = 384;
    gi.C_out = 1536;
    gi.taps = 1;
    std::vector<float> w((size_t)384 * 1536), bsum(1536);
    std::vector<float> wf((size_t)768 * 384), bf(768);
    for (int d = 0; d < 2; ++d) {
      const std::string sfx = d ? "_reverse" : "";
      const auto& wi = W("fc.0.gru.weight_ih_l0" + sfx);
      RVC_CHECK_ARG(wi.numel() == 768 * 384, "rmvpe: fc.0.gru.weight_ih_l0" + sfx + " must be [768, 384]");
      RVC_CUDA_TRY(cudaMemcpy(wf.data(), wi.buf.p, sizeof(float) * wf.size(), cudaMemcpyDeviceToHost));
      RVC_CUDA_TRY(cudaMemcpy(bf.data(), W("fc.0.gru.bias_ih_l0" + sfx).buf.p, sizeof(float) * 768,
                              cudaMemcpyDeviceToHost));
      for (int o = 0; o < 768; ++o) {
        for (int i = 0; i < 384; ++i) w[(size_t)i * 1536 + d * 768 + o] = wf[(size_t)o * 384 + i];
        bsum[d * 768 + o] = bf[o];
      }
    }
    gi.w = DevBuf(ctx, sizeof(float) * w.size());
    gi.bias = DevBuf(ctx, sizeof(float) * 1536);
    RVC_CUDA_TRY(cudaMemcpy(gi.w.p, w.data(), sizeof(float) * w.size(), cudaMemcpyHostToDevice));
    RVC_CUDA_TRY(cudaMemcpy(gi.bias.p, bsum.data(), sizeof(float) * 1536, cudaMemcpyHostToDevice));
    convs_["gru_in"] = std::move(gi);
    w_hh_ = DevBuf(ctx, sizeof(float) * 2 * 768 * 256);
    b_hh_ = DevBuf(ctx, sizeof(float) * 2 * 768);
    for (int d = 0; d < 2; ++d) {
      const std::string sfx = d ? "_reverse" : "";
      RVC_CHECK_ARG(W("fc.0.gru.weight_hh_l0" + sfx).numel() == 768 * 256, "rmvpe: GRU hidden size must be 256");
      RVC_CUDA_TRY(cudaMemcpyAsync(w_hh_.f() + (size_t)d * 768 * 256, W("fc.0.gru.weight_hh_l0" + sfx).buf.p,
                                   sizeof(float) * 768 * 256, cudaMemcpyDeviceToDevice, st));
      RVC_CUDA_TRY(cudaMemcpyAsync(b_hh_.f() + (size_t)d * 768, W("fc.0.gru.bias_hh_l0" + sfx).buf.p,
                                   sizeof(float) * 768, cudaMemcpyDeviceToDevice, st));
    }
  }
  {
    // fc.1: Linear(512 -> 360) as a 1x1 conv ([O][I] == [O][I][1][1])
    const auto& wf = W("fc.1.weight");
    RVC_CHECK_ARG(wf.numel() == 360 * 512, "rmvpe: fc.1.weight must be [360, 512]");
    RmvpeTensor t4;
    t4.shape = {360, 512, 1, 1};
    t4.buf = DevBuf(ctx, sizeof(float) * 360 * 512);
    RVC_CUDA_TRY(cudaMemcpyAsync(t4.buf.p, wf.buf.p, t4.buf.bytes, cudaMemcpyDeviceToDevice, st));
    Conv2dW fc = make_conv(ctx, t4, false, "fc.1.weight");
    fc.bias = DevBuf(ctx, sizeof(float) * 360);
    RVC_CUDA_TRY(cudaMemcpyAsync(fc.bias.p, W("fc.1.bias").buf.p, sizeof(float) * 360, cudaMemcpyDeviceToDevice, st));
    RVC_CUDA_TRY(cudaStreamSynchronize(st));  // t4 is freed on return
    convs_["fc"] = std::move(fc);
  }
  // front-end tables: HTK mel filters (rows normalised to sum 1) and numpy's
  // symmetric Hann window (runtime/dsp/mel.py:97-122, runtime/dsp/fft.py:16-56)
  {
    const int nb = kBins;
    std::vector<double> fftf(nb);
    for (int k = 0; k < nb; ++k) fftf[k] = (nb == 1) ? 0.0 : 8000.0 * k / (nb - 1);
    const double mlo = 1127.0 * std::log1p(30.0 / 700.0), mhi = 1127.0 * std::log1p(8000.0 / 700.0);
    std::vector<double> fpts(kMels + 2);
    const double step = (mhi - mlo) / (kMels + 1);  // numpy.linspace: i * step + start, exact end point
    for (int i = 0; i < kMels + 2; ++i) {
      const double m = i == kMels + 1 ? mhi : i * step + mlo;
      fpts[i] = 700.0 * std::expm1(m / 1127.0);
    }
    std::vector<float> basis((size_t)kMels * nb);
    for (int i = 0; i < kMels; ++i) {
      const double lo = fpts[i], c = fpts[i + 1], hi = fpts[i + 2];
      std::vector<double> tri(nb);
      double s = 0.0;
      for (int k = 0; k < nb; ++k) {
        const double up = c - lo > 0 ? (fftf[k] - lo) / (c - lo) : 0.0;
        const double dn = hi - c > 0 ? (hi - fftf[k]) / (hi - c) : 0.0;
        tri[k] = std::max(0.0, std::min(up, dn));
        s += tri[k];
      }
      for (int k = 0; k < nb; ++k) basis[(size_t)i * nb + k] = (float)(s > 0 ? tri[k] / s : tri[k]);
    }
    std::vector<double> win(kNFFT);
    const double pi = 3.14159265358979323846;
    for (int k = 0; k < kNFFT; ++k) {
      const double n = 1.0 - kNFFT + 2.0 * k;  // numpy.hanning: 0.5 + 0.5 cos(pi n / (M - 1))
      win[k] = 0.5 + 0.5 * std::cos(pi * n / (kNFFT - 1));
    }
    // the projection runs as a 1x1 conv: weights [1][513 bins][128 mels]
    std::vector<float> basis_t(basis.size());
    for (int m = 0; m < kMels; ++m)
      for (int k = 0; k < nb; ++k) basis_t[(size_t)k * kMels + m] = basis[(size_t)m * nb + k];
    mel_basis_ = DevBuf(ctx, sizeof(float) * basis_t.size());
    window_ = DevBuf(ctx, sizeof(double) * win.size());
    RVC_CUDA_TRY(cudaMemcpy(mel_basis_.p, basis_t.data(), mel_basis_.bytes, cudaMemcpyHostToDevice));
    RVC_CUDA_TRY(cudaMemcpy(window_.p, win.data(), window_.bytes, cudaMemcpyHostToDevice));
  }
  RVC_CUDA_TRY(cudaStreamSynchronize(st));
  finalized_ = true;
}

void RmvpeModel::ensure_ws(int B, int64_t T) {
  if (B <= ws_B && T <= ws_T) return;
  B = std::max(B, ws_B);
  T = std::max(T, ws_T);
  ws_.clear();
  const int64_t F = frames(T), Fp = 32 * ((F - 1) / 32 + 1);
  const int64_t big = Fp * 128 * 16;  // widest activation: level 0, 16 channels
  auto add = [&](const std::string& n, long long per_chunk) {
    ws_.emplace(n, DevBuf(ctx, sizeof(float) * (size_t)B * std::max<long long>(1, per_chunk)));
  };
  add("x", T);
  add("mag", F * kBins);
  add("mel", Fp * 128);
  add("x0", Fp * 128);
  add("A", big);
  add("Bb", big);
  add("Tt", big);
  add("P", big / 2);
  for (int l = 0; l < 5; ++l) add("cat" + std::to_string(l), (Fp >> l) * (128 >> l) * 2 * kEnc[l][1]);
  add("feat", Fp * 384);
  add("gx", Fp * 1536);
  add("hg", Fp * 512);
  add("sal", Fp * 360);
  add("f0", F);
  ws_.emplace("amax", DevBuf(ctx, sizeof(int32_t) * (size_t)B * F));
  ws_.emplace("frames", DevBuf(ctx, sizeof(double) * (size_t)B * F * kNFFT));
  ws_.emplace("spec", DevBuf(ctx, 2 * sizeof(double) * (size_t)B * F * kBins));
  // split partials: the direct conv splits while the batch's tiles x splits <
  // 2 x 148, so the partials hold < 4 x 148 tiles x 256 pixels x 64 channels
  ws_.emplace("part", DevBuf(ctx, sizeof(float) * (size_t)4 * 148 * 256 * 64));
  ws_B = B;
  ws_T = T;
}

void RmvpeModel::save_tap(const std::string& name, const float* d, int64_t n) {
  if (!keep_taps) return;
  std::vector<float> h((size_t)n);
  RVC_CUDA_TRY(cudaMemcpyAsync(h.data(), d, sizeof(float) * n, cudaMemcpyDeviceToHost, ctx->stream));
  RVC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  taps_[name] = std::move(h);
}

bool RmvpeModel::tap(const std::string& name, float* host, int64_t n) {
  auto it = taps_.find(name);
  if (it == taps_.end() || (int64_t)it->second.size() < n) return false;
  std::copy(it->second.begin(), it->second.begin() + n, host);
  return true;
}

void RmvpeModel::conv(const Conv2dW& L, int B, const float* x, long long x_bs, int H, int Wd, int ldi, float* y,
                      long long y_bs, long long oh_s, int ow_s, int oc_s, bool relu, const float* res,
                      long long res_bs, int ldr, bool sigmoid) {
  C2Args a{};
  a.x = x; a.x_bs = x_bs; a.H = H; a.W = Wd; a.ldi = ldi;
  a.C_in = L.C_in; a.C_out = L.C_out; a.taps = L.taps; a.transposed = L.transposed ? 1 : 0;
  a.w = L.w.f();
  a.OH = L.transposed ? 2 * H : H;
  a.OW = L.transposed ? 2 * Wd : Wd;
  a.y = y; a.y_bs = y_bs; a.oh_s = oh_s; a.ow_s = ow_s; a.oc_s = oc_s;
  a.bias = L.bias.p ? L.bias.f() : nullptr;
  a.scale = L.scale.p ? L.scale.f() : nullptr;
  a.shift = L.shift.p ? L.shift.f() : nullptr;
  a.relu = relu ? 1 : 0;
  a.sigm = sigmoid ? 1 : 0;
  a.res = res; a.res_bs = res_bs; a.ldr = ldr;
  a.B = B;
  const long long M = (long long)a.OH * a.OW;
  // direct kernel: <BN, TNC, TMP, CK> by output channels and row width (a
  // thread's TMP pixels lie in one row, so rows narrower than TMP go below)
  static const int kBN[4] = {16, 32, 64, 64}, kTNC[4] = {4, 4, 8, 8}, kTMP[4] = {8, 8, 8, 4}, kCK[4] = {8, 8, 8, 8};
  const int v = L.C_out <= 16 ? 0 : (L.C_out <= 32 ? 1 : (a.OW >= 8 ? 2 : 3));
  if (!L.transposed && L.taps == 9 && a.OW >= kTMP[v]) {
    const int BNd = kBN[v], TMP = kTMP[v], CK = kCK[v];
    const int TPX = 256 / (BNd / kTNC[v]) * TMP;
    const int TW = std::min(32, a.OW) / TMP * TMP;
    const int TH = TPX / TW;
    const int ncb = (L.C_in + CK - 1) / CK;
    const long long tiles = (long long)((a.OH + TH - 1) / TH) * ((a.OW + TW - 1) / TW) * ((L.C_out + BNd - 1) / BNd);
    // split the channel blocks when the batch's tiles fill less than two waves
    // (sums then differ from the unsplit order by fp32 rounding only)
    int splits = 1;
    while (tiles * B * splits < 2 * 148 && ncb / (splits * 2) >= 2 && splits < 16) splits *= 2;
    if (splits > 1 && (size_t)splits * B * M * L.C_out * sizeof(float) > ws_.at("part").bytes) splits = 1;
    a.splits = splits;
    a.part = ws_.at("part").f();
    dim3 g((unsigned)(((a.OH + TH - 1) / TH) * ((a.OW + TW - 1) / TW)), (unsigned)((L.C_out + BNd - 1) / BNd),
           (unsigned)(B * splits));
    // dynamic shared memory: two stages of weights [9][CK][BN] and halo
    const size_t hs = sizeof(float) * 2 * ((size_t)9 * CK * BNd + (((size_t)(TH + 2) * (TW + 2) * (CK + 1) + 3) & ~(size_t)3));
    static std::atomic<uint64_t> attr_done{0};  // the attribute is per device
    if (ctx->device < 64 && !(attr_done.load() & (1ull << ctx->device))) {
      RVC_CUDA_TRY(cudaFuncSetAttribute(conv3x3_direct_kernel<16, 4, 8, 8>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
      RVC_CUDA_TRY(cudaFuncSetAttribute(conv3x3_direct_kernel<32, 4, 8, 8>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
      RVC_CUDA_TRY(cudaFuncSetAttribute(conv3x3_direct_kernel<64, 8, 8, 8>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
      RVC_CUDA_TRY(cudaFuncSetAttribute(conv3x3_direct_kernel<64, 8, 4, 8>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
      attr_done.fetch_or(1ull << ctx->device);
    }
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ctx->prof) ctx->prof_begin(&e0, &e1);
    if (v == 0)
      conv3x3_direct_kernel<16, 4, 8, 8><<<g, 256, hs, ctx->stream>>>(a, TW);
    else if (v == 1)
      conv3x3_direct_kernel<32, 4, 8, 8><<<g, 256, hs, ctx->stream>>>(a, TW);
    else if (v == 2)
      conv3x3_direct_kernel<64, 8, 8, 8><<<g, 256, hs, ctx->stream>>>(a, TW);
    else
      conv3x3_direct_kernel<64, 8, 4, 8><<<g, 256, hs, ctx->stream>>>(a, TW);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
    if (splits > 1) {
      conv2d_reduce_kernel<<<grid_for(B * M * L.C_out, 256), 256, 0, ctx->stream>>>(a);
      note_launch();
      RVC_CUDA_TRY(cudaGetLastError());
    }
    if (ctx->prof) {
      char lab[160];
      snprintf(lab, sizeof(lab), "rmvpe conv Cin=%d Cout=%d taps=9 %dx%d B=%d direct split=%d", L.C_in, L.C_out,
               a.OH, a.OW, B, splits);
      ctx->prof_end(e0, e1, 2.0 * B * M * L.C_out * L.C_in * 9.0, lab, false);
    }
    return;
  }
  if (L.transposed && L.taps == 9 && Wd >= 4) {
    // parity-split direct transposed conv: <BN, TNC, TMP = 4, CK = 8>
    const int vt = L.C_out <= 16 ? 0 : (L.C_out <= 32 ? 1 : 2);
    static const int kTBN[3] = {16, 32, 64}, kTTNC[3] = {4, 4, 8};
    const int BNd = kTBN[vt], TMP = 4, CK = 8;
    const int G = 256 / (BNd / kTTNC[vt]);
    const int TW = std::min(32, Wd) / TMP * TMP;
    const int OHt = G / (TW / TMP);
    const int ncb = (L.C_in + CK - 1) / CK;
    const long long tiles = (long long)((a.OH + OHt - 1) / OHt) * ((Wd + TW - 1) / TW) * ((L.C_out + BNd - 1) / BNd);
    int splits = 1;
    while (tiles * B * splits < 2 * 148 && ncb / (splits * 2) >= 2 && splits < 16) splits *= 2;
    if (splits > 1 && (size_t)splits * B * M * L.C_out * sizeof(float) > ws_.at("part").bytes) splits = 1;
    a.splits = splits;
    a.part = ws_.at("part").f();
    dim3 g((unsigned)(((a.OH + OHt - 1) / OHt) * ((Wd + TW - 1) / TW)), (unsigned)((L.C_out + BNd - 1) / BNd),
           (unsigned)(B * splits));
    const size_t hs =
        sizeof(float) * 2 * ((size_t)9 * CK * BNd + (((size_t)(OHt / 2 + 1) * (TW + 1) * (CK + 1) + 3) & ~(size_t)3));
    static std::atomic<uint64_t> attr_done{0};  // the attribute is per device
    if (ctx->device < 64 && !(attr_done.load() & (1ull << ctx->device))) {
      RVC_CUDA_TRY(cudaFuncSetAttribute(convT3x3_direct_kernel<16, 4, 4, 8>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
      RVC_CUDA_TRY(cudaFuncSetAttribute(convT3x3_direct_kernel<32, 4, 4, 8>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
      RVC_CUDA_TRY(cudaFuncSetAttribute(convT3x3_direct_kernel<64, 8, 4, 8>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
      attr_done.fetch_or(1ull << ctx->device);
    }
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ctx->prof) ctx->prof_begin(&e0, &e1);
    if (vt == 0)
      convT3x3_direct_kernel<16, 4, 4, 8><<<g, 256, hs, ctx->stream>>>(a, TW);
    else if (vt == 1)
      convT3x3_direct_kernel<32, 4, 4, 8><<<g, 256, hs, ctx->stream>>>(a, TW);
    else
      convT3x3_direct_kernel<64, 8, 4, 8><<<g, 256, hs, ctx->stream>>>(a, TW);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
    if (splits > 1) {
      conv2d_reduce_kernel<<<grid_for(B * M * L.C_out, 256), 256, 0, ctx->stream>>>(a);
      note_launch();
      RVC_CUDA_TRY(cudaGetLastError());
    }
    if (ctx->prof) {
      char lab[160];
      snprintf(lab, sizeof(lab), "rmvpe convT Cin=%d Cout=%d taps=9 %dx%d B=%d direct split=%d", L.C_in, L.C_out,
               a.OH, a.OW, B, splits);
      ctx->prof_end(e0, e1, 2.0 * B * M * L.C_out * L.C_in * 2.25, lab, false);
    }
    return;
  }
  // narrow stride-1 convs (<= 32 output channels, the tall full-resolution
  // levels): register-blocked 8 x 4 tiles; the rest (measured faster there:
  // fewer registers, more resident blocks) the 4 x 4 kernel
  const bool rb = !L.transposed && L.C_out <= 32;
  int BN, BM;
  if (rb) {
    BN = L.C_out <= 16 ? 16 : 32;
    BM = BN == 16 ? 512 : 256;
    a.kit = L.taps * ((L.C_in + kBK8 - 1) / kBK8);
  } else {
    BN = L.C_out <= 16 ? 16 : (L.C_out <= 32 ? 32 : 64);
    BM = kTileElems / BN;
    a.kit = L.taps * ((L.C_in + kBK - 1) / kBK);
  }
  const int mt = (int)((M + BM - 1) / BM), nt = (L.C_out + BN - 1) / BN;
  const long long tiles = (long long)mt * nt * B;
  int splits = 1;
  // few output tiles and a long K loop: split K so ~2 waves of blocks run
  while (tiles * splits < 2 * 148 && a.kit / (splits * 2) >= 8 && splits < 16) splits *= 2;
  if (splits > 1) {
    const size_t need = (size_t)splits * B * M * L.C_out;
    if (need * sizeof(float) > ws_.at("part").bytes) splits = 1;
  }
  a.splits = splits;
  a.part = ws_.at("part").f();
  dim3 g(mt, nt, B * splits);
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (ctx->prof) ctx->prof_begin(&e0, &e1);
  if (rb) {
    if (BN == 16)
      conv2d_rb_kernel<512, 16, 8, 4><<<g, 256, 0, ctx->stream>>>(a);
    else
      conv2d_rb_kernel<256, 32, 8, 4><<<g, 256, 0, ctx->stream>>>(a);
  } else if (BN == 16) {
    conv2d_kernel<256, 16><<<g, 256, 0, ctx->stream>>>(a);
  } else if (BN == 32) {
    conv2d_kernel<128, 32><<<g, 256, 0, ctx->stream>>>(a);
  } else {
    conv2d_kernel<64, 64><<<g, 256, 0, ctx->stream>>>(a);
  }
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
  if (splits > 1) {
    conv2d_reduce_kernel<<<grid_for(B * M * L.C_out, 256), 256, 0, ctx->stream>>>(a);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
  }
  if (ctx->prof) {
    char lab[160];
    snprintf(lab, sizeof(lab), "rmvpe %s Cin=%d Cout=%d taps=%d %dx%d B=%d split=%d", L.transposed ? "convT" : "conv",
             L.C_in, L.C_out, L.taps, a.OH, a.OW, B, splits);
    ctx->prof_end(e0, e1, 2.0 * B * M * L.C_out * L.C_in * (L.transposed ? 2.25 : (double)L.taps), lab, false);
  }
}

void RmvpeModel::block(const std::string& p, int B, const float* x, long long x_bs, int H, int Wd, int ldi,
                       float* out, long long out_bs, int ldo, float* tmp, long long tmp_bs) {
  const Conv2dW& c0 = convs_.at(p + ".conv.0");
  const Conv2dW& c3 = convs_.at(p + ".conv.3");
  const int co = c0.C_out;
  const long long ohs_o = (long long)Wd * ldo, ohs_t = (long long)Wd * co;
  auto sc = convs_.find(p + ".shortcut");
  if (sc != convs_.end())  // shortcut = conv1x1(x) + b, written first, then added to the main branch
    conv(sc->second, B, x, x_bs, H, Wd, ldi, out, out_bs, ohs_o, ldo, 1, false, nullptr, 0, 0);
  conv(c0, B, x, x_bs, H, Wd, ldi, tmp, tmp_bs, ohs_t, co, 1, true, nullptr, 0, 0);
  if (sc != convs_.end())
    conv(c3, B, tmp, tmp_bs, H, Wd, co, out, out_bs, ohs_o, ldo, 1, true, out, out_bs, ldo);
  else
    conv(c3, B, tmp, tmp_bs, H, Wd, co, out, out_bs, ohs_o, ldo, 1, true, x, x_bs, ldi);
}

void RmvpeModel::infer_device(int B, int64_t T, const float* x, float thred, float* f0, int32_t* argmax) {
  if (!finalized_) throw Error{kErrState, "rmvpe: finalize() not called after the last weight upload"};
  RVC_CHECK_ARG(B >= 1, "rmvpe: B must be positive");
  RVC_CHECK_ARG(T > kNFFT / 2, "rmvpe: audio must be longer than 512 samples (reflect padding)");
  RVC_CHECK_ARG(T <= (1ll << 31), "rmvpe: audio too long");
  ensure_ws(B, T);
  taps_.clear();
  cudaStream_t st = ctx->stream;
  const int F = (int)frames(T), Fp = 32 * ((F - 1) / 32 + 1);
  const long long bs_big = (long long)(ws_.at("A").bytes / sizeof(float) / ws_B);
  // ---------------- front end
  {
    const long long nfr = (long long)B * F;
    auto it = fft_plans_.find(nfr);
    if (it == fft_plans_.end()) {
      cufftHandle h = 0;
      int n = kNFFT;
      if (cufftPlanMany(&h, 1, &n, nullptr, 1, kNFFT, nullptr, 1, kBins, CUFFT_D2Z, (int)nfr) != CUFFT_SUCCESS)
        throw Error{kErrCuda, "rmvpe: cuFFT plan failed"};
      it = fft_plans_.emplace(nfr, (int)h).first;
    }
    const cufftHandle h = (cufftHandle)it->second;
    double* fr = reinterpret_cast<double*>(ws_.at("frames").p);
    stft_frames_kernel<<<(unsigned)std::min<long long>((nfr * 1024 + 255) / 256, 148ll * 16), 256, 0, st>>>(
        x, T, F, (const double*)window_.p, fr, B);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
    if (cufftSetStream(h, st) != CUFFT_SUCCESS ||
        cufftExecD2Z(h, (cufftDoubleReal*)fr, (cufftDoubleComplex*)ws_.at("spec").p) != CUFFT_SUCCESS)
      throw Error{kErrCuda, "rmvpe: cuFFT transform failed"};
    stft_mag_kernel<<<(unsigned)std::min<long long>((nfr * kBins + 255) / 256, 148ll * 16), 256, 0, st>>>(
        (const double2*)ws_.at("spec").p, nfr * kBins, buf("mag"));
    note_launch();
  }
  {
    // mel projection s[t][m] = sum_k basis[m][k] mag[t][k] as an unsplit fp32
    // 1x1 implicit GEMM: each sum runs over k in ascending order from 0, one
    // fmaf per bin, as a per-(frame, mel) loop would
    C2Args a{};
    a.x = buf("mag"); a.x_bs = (long long)F * kBins; a.H = F; a.W = 1; a.ldi = kBins;
    a.C_in = kBins; a.C_out = kMels; a.taps = 1; a.transposed = 0;
    a.w = mel_basis_.f();
    a.OH = F; a.OW = 1;
    a.y = buf("mel"); a.y_bs = (long long)Fp * kMels; a.oh_s = kMels; a.ow_s = kMels; a.oc_s = 1;
    a.B = B; a.splits = 1; a.kit = (kBins + kBK - 1) / kBK;
    conv2d_kernel<64, 64><<<dim3((unsigned)((F + 63) / 64), (unsigned)(kMels / 64), (unsigned)B), 256, 0, st>>>(a);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
    const long long n = (long long)B * Fp * kMels;
    mel_finish_kernel<<<(unsigned)std::min<long long>((n + 255) / 256, 148ll * 16), 256, 0, st>>>(
        buf("mel"), F, Fp, B, in_scale_.f(), in_shift_.f(), buf("x0"));
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
  }
  save_tap("mel", buf("mel"), (long long)B * Fp * 128);
  // ---------------- encoder
  float *A = buf("A"), *Bb = buf("Bb"), *Tt = buf("Tt"), *P = buf("P");
  const float* lin = buf("x0");
  long long lin_bs = (long long)Fp * 128;
  int ldin = 1;
  for (int l = 0; l < 5; ++l) {
    const int H = Fp >> l, Wd = 128 >> l, co = kEnc[l][1];
    float* cat = buf(("cat" + std::to_string(l)).c_str());
    const long long cat_bs = (long long)(ws_.at("cat" + std::to_string(l)).bytes / sizeof(float) / ws_B);
    const std::string p = "unet.encoder.layers." + std::to_string(l) + ".conv.";
    block(p + "0", B, lin, lin_bs, H, Wd, ldin, A, bs_big, co, Tt, bs_big);
    block(p + "1", B, A, bs_big, H, Wd, co, Bb, bs_big, co, Tt, bs_big);
    block(p + "2", B, Bb, bs_big, H, Wd, co, A, bs_big, co, Tt, bs_big);
    block(p + "3", B, A, bs_big, H, Wd, co, cat + co, cat_bs, 2 * co, Tt, bs_big);  // skip half of the concat
    save_tap("enc" + std::to_string(l), cat, (long long)B * cat_bs);  // skip = channels [co, 2co)
    const long long pn = (long long)(H / 2) * (Wd / 2) * co;
    avgpool_kernel<<<grid_for(pn * B, 256), 256, 0, st>>>(cat + co, cat_bs, H, Wd, co, 2 * co, P, bs_big / 2, B);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
    lin = P;
    lin_bs = bs_big / 2;
    ldin = co;
  }
  // ---------------- intermediate: [Fp/32][4]
  {
    const int H = Fp >> 5, Wd = 4;
    float* bufs[2] = {A, Bb};
    const float* cur = P;
    long long cur_bs = bs_big / 2;
    int ldc = 256, k = 0;
    for (int i = 0; i < 4; ++i)
      for (int j = 0; j < 4; ++j, ++k) {
        float* o = bufs[k & 1];
        block("unet.intermediate.layers." + std::to_string(i) + ".conv." + std::to_string(j), B, cur, cur_bs, H, Wd,
              ldc, o, bs_big, 512, Tt, bs_big);
        cur = o;
        cur_bs = bs_big;
        ldc = 512;
      }
    lin = cur;  // == bufs[1] after 16 blocks
    lin_bs = bs_big;
    ldin = 512;
    save_tap("inter", lin, (long long)B * bs_big);
  }
  // ---------------- decoder
  for (int i = 0; i < 5; ++i) {
    const int l = 4 - i, H = Fp >> l, Wd = 128 >> l, co = kDec[i][1];
    float* cat = buf(("cat" + std::to_string(l)).c_str());
    const long long cat_bs = (long long)(ws_.at("cat" + std::to_string(l)).bytes / sizeof(float) / ws_B);
    const std::string p = "unet.decoder.layers." + std::to_string(i);
    // convT + BN + ReLU into the first half of the concat buffer
    conv(convs_.at(p + ".conv1"), B, lin, lin_bs, H / 2, Wd / 2, ldin, cat, cat_bs, (long long)Wd * 2 * co, 2 * co, 1,
         true, nullptr, 0, 0);
    float* outb = (lin == A) ? Bb : A;
    float* other = (outb == A) ? Bb : A;
    block(p + ".conv2.0", B, cat, cat_bs, H, Wd, 2 * co, outb, bs_big, co, Tt, bs_big);
    block(p + ".conv2.1", B, outb, bs_big, H, Wd, co, other, bs_big, co, Tt, bs_big);
    block(p + ".conv2.2", B, other, bs_big, H, Wd, co, outb, bs_big, co, Tt, bs_big);
    block(p + ".conv2.3", B, outb, bs_big, H, Wd, co, other, bs_big, co, Tt, bs_big);
    lin = other;
    lin_bs = bs_big;
    ldin = co;
    save_tap("dec" + std::to_string(i), lin, (long long)B * bs_big);
  }
  // ---------------- cnn (16 -> 3, bias) written as [Fp][3 * 128] (channel-major within a frame)
  conv(convs_.at("cnn"), B, lin, lin_bs, Fp, 128, 16, buf("feat"), (long long)Fp * 384, 384, 1, 128, false, nullptr,
       0, 0);
  save_tap("cnn", buf("feat"), (long long)B * Fp * 384);
  // ---------------- BiGRU: gx for both directions, then the recurrence
  conv(convs_.at("gru_in"), B, buf("feat"), (long long)Fp * 384, Fp, 1, 384, buf("gx"), (long long)Fp * 1536, 1536,
       1536, 1, false, nullptr, 0, 0);
  {
    const int groups = (B + kGruBg - 1) / kGruBg;  // every (direction, sequence group) cluster runs at once
    gru_kernel<<<2 * groups * kGruCta, kGruThreads, 0, st>>>(buf("gx"), w_hh_.f(), b_hh_.f(), B, Fp, buf("hg"));
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
  }
  save_tap("gru", buf("hg"), (long long)B * Fp * 512);
  // ---------------- fc: Linear(512 -> 360) + sigmoid
  conv(convs_.at("fc"), B, buf("hg"), (long long)Fp * 512, Fp, 1, 512, buf("sal"), (long long)Fp * 360, 360, 360, 1,
       false, nullptr, 0, 0, true);
  save_tap("salience", buf("sal"), (long long)B * Fp * 360);
  // ---------------- decode
  decode_kernel<<<(unsigned)(((long long)B * F + 7) / 8), 256, 0, st>>>(buf("sal"), Fp, F, thred, f0, argmax, B);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

void RmvpeModel::infer_host(int B, int64_t T, const float* x, float thred, float* f0, int32_t* argmax) {
  RVC_CHECK_ARG(T > kNFFT / 2, "rmvpe: audio must be longer than 512 samples (reflect padding)");
  ensure_ws(B, T);
  cudaStream_t st = ctx->stream;
  const int64_t F = frames(T);
  RVC_CUDA_TRY(cudaMemcpyAsync(buf("x"), x, sizeof(float) * (size_t)B * T, cudaMemcpyHostToDevice, st));
  infer_device(B, T, buf("x"), thred, buf("f0"), ws_.at("amax").as<int32_t>());
  RVC_CUDA_TRY(cudaMemcpyAsync(f0, buf("f0"), sizeof(float) * (size_t)B * F, cudaMemcpyDeviceToHost, st));
  if (argmax)
    RVC_CUDA_TRY(cudaMemcpyAsync(argmax, ws_.at("amax").p, sizeof(int32_t) * (size_t)B * F, cudaMemcpyDeviceToHost,
                                 st));
}

}  // namespace rvc
