// Fused self-attention for the text encoder (T5 relative positions) and,
// with window < 0, plain scaled-dot-product attention.
//
// Reference semantics (runtime/models/vits.py:993-1014):
//   qs     = q / sqrt(kc)
//   scores = qs . k^T + rel_to_abs(qs . used_k^T)   (bias non-zero only for |j-i| <= window)
//   p      = softmax(scores)
//   out    = p . v + abs_to_rel(p) . used_v          (again only the band |j-i| <= window)
//
// One CTA = 64 queries of one head of one chunk, 256 threads.  Keys stream in
// blocks of 64: S = Qs K^T on a 4x4-per-thread register tile, the band bias
// from precomputed qs . emb_k rows, online softmax (running max / sum per
// row), O += P V on a 4x6 register tile.  The band term of the output is
// recomputed at the end from the final row max and sum.  fp32 throughout.
#include "kernels.cuh"

#include <atomic>
#include <cmath>

namespace rvc {

constexpr int kQB = 64;      // queries per CTA
constexpr int kKB = 64;      // keys per block
constexpr int kMaxD = 128;   // head dim (kc) supported
constexpr int kMaxW = 16;    // relative window supported

struct AttnSmem {
  // sizes in floats, for D = head dim
  static size_t floats(int D, int W) {
    const int dp = D + 1;
    return (size_t)kQB * dp + (size_t)kKB * dp + (size_t)kKB * D + (size_t)kQB * (kKB + 1) +
           (size_t)kQB * (2 * kMaxW + 1) + 3 * kQB;
  }
};

__global__ void __launch_bounds__(256) flash_rel_attn_kernel(const float* __restrict__ qkv, int ld, int q_off,
                                                             int k_off, int v_off, const float* __restrict__ emb_k,
                                                             const float* __restrict__ emb_v, int heads, int D,
                                                             int P, int W, float q_div, float* __restrict__ y,
                                                             int y_ld) {
  extern __shared__ float sm[];
  const int dp = D + 1;
  float* Qs = sm;                         // [64][D+1]
  float* Ks = Qs + kQB * dp;              // [64][D+1]
  float* Vs = Ks + kKB * dp;              // [64][D]
  float* S = Vs + kKB * D;                // [64][65]
  float* Rk = S + kQB * (kKB + 1);        // [64][2W+1]  qs . emb_k[r]
  float* mrow = Rk + kQB * (2 * kMaxW + 1);
  float* lrow = mrow + kQB;
  float* arow = lrow + kQB;

  const int bh = blockIdx.y;
  const int b = bh / heads, h = bh % heads;
  const int i0 = blockIdx.x * kQB;
  const float* base = qkv + (long long)b * P * ld;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int nb = 2 * W + 1;

  for (int e = tid; e < kQB * D; e += 256) {
    const int r = e / D, d = e % D;
    const int i = i0 + r;
    Qs[r * dp + d] = i < P ? base[(long long)i * ld + q_off + h * D + d] / q_div : 0.f;
  }
  if (tid < kQB) {
    mrow[tid] = -INFINITY;
    lrow[tid] = 0.f;
  }
  __syncthreads();
  if (W >= 0) {
    for (int e = tid; e < kQB * nb; e += 256) {
      const int r = e / nb, k = e % nb;
      float s = 0.f;
      for (int d = 0; d < D; ++d) s = fmaf(Qs[r * dp + d], emb_k[(long long)k * D + d], s);
      Rk[r * (2 * kMaxW + 1) + k] = s;
    }
  }
  // output accumulator: rows ty*4..+3, columns tx + 16*c (c < 6; D <= 96 per 16-col stripe ... up to 8)
  constexpr int kCols = kMaxD / 16;
  float o[4][kCols];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < kCols; ++c) o[r][c] = 0.f;

  for (int j0 = 0; j0 < P; j0 += kKB) {
    __syncthreads();  // previous block's S / Vs fully consumed
    for (int e = tid; e < kKB * D; e += 256) {
      const int r = e / D, d = e % D;
      const int j = j0 + r;
      const bool ok = j < P;
      Ks[r * dp + d] = ok ? base[(long long)j * ld + k_off + h * D + d] : 0.f;
      Vs[r * D + d] = ok ? base[(long long)j * ld + v_off + h * D + d] : 0.f;
    }
    __syncthreads();
    // S tile: rows ty*4+a, cols tx*4+c
    float s[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[a][c] = 0.f;
    for (int d = 0; d < D; ++d) {
      float qa[4], kb[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) qa[a] = Qs[(ty * 4 + a) * dp + d];
#pragma unroll
      for (int c = 0; c < 4; ++c) kb[c] = Ks[(tx * 4 + c) * dp + d];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[a][c] = fmaf(qa[a], kb[c], s[a][c]);
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int r = ty * 4 + a, cc = tx * 4 + c;
        const int i = i0 + r, j = j0 + cc;
        float v = s[a][c];
        if (W >= 0) {
          const int rel = j - i;
          if (rel >= -W && rel <= W) v = v + Rk[r * (2 * kMaxW + 1) + rel + W];
        }
        S[r * (kKB + 1) + cc] = (j < P) ? v : -INFINITY;
      }
    __syncthreads();
    // online softmax: 4 threads per row, 16 columns each
    {
      const int r = tid >> 2, part = tid & 3;
      float mx = -INFINITY;
      for (int c = part * 16; c < part * 16 + 16; ++c) mx = fmaxf(mx, S[r * (kKB + 1) + c]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mold = mrow[r];
      const float mnew = fmaxf(mold, mx);
      float sum = 0.f;
      for (int c = part * 16; c < part * 16 + 16; ++c) {
        const float pv = expf(S[r * (kKB + 1) + c] - mnew);
        S[r * (kKB + 1) + c] = pv;
        sum += pv;
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      __syncwarp();
      if (part == 0) {
        const float alpha = (mold == -INFINITY) ? 0.f : expf(mold - mnew);
        lrow[r] = lrow[r] * alpha + sum;
        mrow[r] = mnew;
        arow[r] = alpha;
      }
    }
    __syncthreads();
    // O = O*alpha + P V
    float al[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) al[a] = arow[ty * 4 + a];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < kCols; ++c) o[a][c] *= al[a];
    for (int jj = 0; jj < kKB; ++jj) {
      float pa[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) pa[a] = S[(ty * 4 + a) * (kKB + 1) + jj];
#pragma unroll
      for (int c = 0; c < kCols; ++c) {
        const int d = tx + 16 * c;
        if (d < D) {
          const float vv = Vs[jj * D + d];
#pragma unroll
          for (int a = 0; a < 4; ++a) o[a][c] = fmaf(pa[a], vv, o[a][c]);
        }
      }
    }
  }
  __syncthreads();
  // band probabilities p[i, i+k-W] from the final row max / sum (S is free now)
  float* Pb = S;  // [64][2W+1]
  if (W >= 0) {
    for (int e = tid; e < kQB * nb; e += 256) {
      const int r = e / nb, k = e % nb;
      const int i = i0 + r, j = i + k - W;
      float pb = 0.f;
      if (i < P && j >= 0 && j < P) {
        const float* kr = base + (long long)j * ld + k_off + h * D;
        float sc = 0.f;
        for (int d = 0; d < D; ++d) sc = fmaf(Qs[r * dp + d], kr[d], sc);
        sc = sc + Rk[r * (2 * kMaxW + 1) + k];
        pb = expf(sc - mrow[r]) / lrow[r];
      }
      Pb[r * (2 * kMaxW + 1) + k] = pb;
    }
    __syncthreads();
  }
  // out = O / l + band(p) . emb_v
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int r = ty * 4 + a, i = i0 + r;
    if (i >= P) continue;
    const float l = lrow[r];
#pragma unroll
    for (int c = 0; c < kCols; ++c) {
      const int d = tx + 16 * c;
      if (d >= D) continue;
      float v = o[a][c] / l;
      if (W >= 0) {
        float band = 0.f;
        for (int k = 0; k < nb; ++k) band = fmaf(Pb[r * (2 * kMaxW + 1) + k], emb_v[(long long)k * D + d], band);
        v = v + band;
      }
      y[((long long)b * P + i) * y_ld + h * D + d] = v;
    }
  }
}

static void launch_attn(const float* qkv, int ld, int q_off, int k_off, int v_off, const float* emb_k,
                        const float* emb_v, int B, int heads, int D, int P, int window, float q_div, float* y, int y_ld,
                        cudaStream_t st) {
  if (B * P == 0) return;
  RVC_CHECK_ARG(D <= kMaxD && window <= kMaxW, "attention: head dim <= 128 and window <= 16 supported");
  const size_t smem = sizeof(float) * AttnSmem::floats(D, window);
  static std::atomic<uint64_t> attr_done{0};  // the attribute is per device
  int dev = 0;
  RVC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && !(attr_done.load() & (1ull << dev))) {
    RVC_CUDA_TRY(cudaFuncSetAttribute(flash_rel_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_done.fetch_or(1ull << dev);
  }
  dim3 g(cdiv(P, kQB), B * heads);
  flash_rel_attn_kernel<<<g, 256, smem, st>>>(qkv, ld, q_off, k_off, v_off, emb_k, emb_v, heads, D, P, window, q_div,
                                               y, y_ld);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

void k_rel_attention(const float* qkv, int qkv_ld, int q_off, int k_off, int v_off, const float* emb_k,
                     const float* emb_v, int B, int heads, int kc, int P, int window, float* scratch, float* y,
                     int y_ld, cudaStream_t st) {
  (void)scratch;
  const float qdiv = window >= 0 ? (float)std::sqrt((double)kc) : 1.f;
  launch_attn(qkv, qkv_ld, q_off, k_off, v_off, emb_k, emb_v, B, heads, kc, P, window, qdiv, y, y_ld, st);
}

void k_attention(const float* qkv, int qkv_ld, int q_off, int k_off, int v_off, int B, int heads, int D, int P,
                 float q_div, float* y, int y_ld, cudaStream_t st) {
  launch_attn(qkv, qkv_ld, q_off, k_off, v_off, nullptr, nullptr, B, heads, D, P, -1, q_div, y, y_ld, st);
}

}  // namespace rvc
