// Tensor-core (tcgen05) scaled-dot-product attention, BF16x3, for the HuBERT
// encoder (runtime/models/hubert.py:1315-1400: softmax(q k^T / 8) v over 12
// heads of 64) and, with a relative-position band, the text encoder
// (runtime/models/vits.py:993-1014).
//
// Pack step: q / q_div, k and v of every (chunk, head) are split into bf16
// hi + lo planes and written in the tcgen05 K-major core-matrix layouts the
// MMAs read, so tiles reach shared memory with plain bulk copies:
//   Q tile [128 rows][D]           : (k/8)*128*16 + r*16 + (k%8)*2 per plane
//   K tile [hi 128 keys | lo 128]  : (k/8)*256*16 + n*16 + (k%8)*2   (stacked N = 256)
//   V tile [hi D rows | lo D rows] : (j/8)*2D*16 + n*16 + (j%8)*2   (keys are the K dim)
// Main kernel, one 128-query tile per work item (persistent CTAs):
//   warp 0  bulk-copies Q once per item and K per 128-key tile; warp 10 V;
//   warp 1  issues S = Qhi.Khi + Qhi.Klo + Qlo.Khi (three N = 128 MMAs into one
//           of two TMEM buffers), then O_t = Phi.[Vhi|Vlo] + Plo.Vhi (N = 2D
//           and D), in the order S_0, S_1, PV_0, S_2, PV_1, ... so the next
//           tile's S is on the tensor pipe while the softmax warps work;
//   warps 2-9 (one query row per thread, two warps per row: each half of the
//           tile's keys and of the head dimensions) read S, keep the running
//           max / sum, write P = exp(s - m) as bf16 hi / lo planes for the
//           second MMA and fold each tile's O_t into a register accumulator
//           (rescaled when the running max moves); band bias and band output
//           term added on the CUDA cores when a window is given.
// Every mbarrier wait is bounded; on a timeout the kernel records an error and
// winds down.
#include "context.cuh"
#include "kernels.cuh"
#include "tc_ptx.cuh"

#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>
#include <cmath>

namespace rvc {

namespace {

constexpr int kTQ = 128;   // queries per tile
constexpr int kTK = 128;   // keys per tile
constexpr int kAThreads = 352;
constexpr uint64_t kAttnWaitNs = 2000000000ull;
constexpr int kMaxWin = 16;

__device__ __forceinline__ void split2(float v, uint16_t& hi, uint16_t& lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  hi = __bfloat16_as_ushort(h);
  lo = __bfloat16_as_ushort(__float2bfloat16_rn(v - __bfloat162float(h)));
}

// q/k/v [B][P][ld] fp32 -> packed tiles.  One thread per (bh, row, 8-element chunk).
__global__ void attn_pack_kernel(const float* __restrict__ qkv, int ld, int q_off, int k_off, int v_off, int heads,
                                 int D, int P, int nq, int nk, float q_div, uint16_t* __restrict__ Qp,
                                 uint16_t* __restrict__ Kp, uint16_t* __restrict__ Vp, long long total) {
  const int dc = D / 8;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(e % dc);
    const long long rest = e / dc;
    const int r = (int)(rest % (nq * kTQ));  // padded row (queries and keys share the padded length)
    const int bh = (int)(rest / (nq * kTQ));
    const int b = bh / heads, h = bh % heads;
    const bool ok = r < P;
    const float* row = qkv + ((long long)b * P + (ok ? r : 0)) * ld;
    uint16_t qh[8], ql[8], kh[8], kl[8], vh[8], vl[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = c * 8 + i;
      const float q = ok ? row[q_off + h * D + d] / q_div : 0.f;
      const float k = ok ? row[k_off + h * D + d] : 0.f;
      const float v = ok ? row[v_off + h * D + d] : 0.f;
      split2(q, qh[i], ql[i]);
      split2(k, kh[i], kl[i]);
      split2(v, vh[i], vl[i]);
    }
    // Q: tile qt = r / 128, plane-major
    {
      const int qt = r / kTQ, rr = r % kTQ;
      uint16_t* base = Qp + ((long long)bh * nq + qt) * 2 * (kTQ * D);
      const long long off = (long long)c * kTQ * 8 + rr * 8;
      *reinterpret_cast<uint4*>(base + off) = *reinterpret_cast<const uint4*>(qh);
      *reinterpret_cast<uint4*>(base + kTQ * D + off) = *reinterpret_cast<const uint4*>(ql);
    }
    if (r < nk * kTK) {
      const int kt = r / kTK, rr = r % kTK;
      uint16_t* kb = Kp + ((long long)bh * nk + kt) * (2 * kTK * D);
      const long long off = (long long)c * (2 * kTK) * 8;
      *reinterpret_cast<uint4*>(kb + off + rr * 8) = *reinterpret_cast<const uint4*>(kh);
      *reinterpret_cast<uint4*>(kb + off + (kTK + rr) * 8) = *reinterpret_cast<const uint4*>(kl);
      // V: key rr is element (rr % 8) of key chunk rr / 8; rows n = d (hi) and D + d (lo)
      uint16_t* vb = Vp + ((long long)bh * nk + kt) * (2 * kTK * D);
      const long long vchunk = (long long)(rr / 8) * (2 * D) * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d = c * 8 + i;
        vb[vchunk + (long long)d * 8 + (rr % 8)] = vh[i];
        vb[vchunk + (long long)(D + d) * 8 + (rr % 8)] = vl[i];
      }
    }
  }
}

struct AttnArgs {
  const uint16_t* Qp;
  const uint16_t* Kp;
  const uint16_t* Vp;
  int heads, D, P, nq, nk;
  float* y;
  int y_ld;
  // relative band (window < 0: none)
  int window;
  const float* rk;     // [B*heads][P][2W+1] qs . emb_k[r]
  const float* sb;     // [B*heads][P][2W+1] band logits qs . k[i + r - W] + rk (-inf outside)
  const float* emb_v;  // [2W+1][D]
  int* err;
  int BH;              // chunks x heads
  // key split: item = (query tile, key range); with nsplit > 1 each item
  // writes its unnormalised O and (row max, row sum) for attn_combine_kernel
  int nsplit;
  float* po;           // [BH][nsplit][P][D]
  float* pml;          // [BH][nsplit][P][2]
};

template <int D>
__global__ void __launch_bounds__(kAThreads, 1) tc_attn_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t q_plane = (uint32_t)kTQ * D * 2u;      // bytes per Q plane
  const uint32_t k_bytes = (uint32_t)2 * kTK * D * 2u;  // stacked hi|lo
  const uint32_t v_bytes = (uint32_t)2 * kTK * D * 2u;
  const uint32_t p_plane = (uint32_t)kTQ * kTK * 2u;
  const uint32_t sbase = ptx::smem_u32(smem);
  const uint32_t off_q = 0, off_k = off_q + 2 * q_plane, off_v = off_k + k_bytes, off_p = off_v + v_bytes;
  const uint32_t off_bar = off_p + 2 * p_plane, off_red = off_bar + 128;  // red: softmax pair exchange, 3 KB
  // barriers; tiles are counted over the whole CTA (g), S alternates between two TMEM buffers
  const uint32_t Q_FULL = sbase + off_bar, Q_EMPTY = Q_FULL + 8, K_FULL = Q_FULL + 16, K_EMPTY = Q_FULL + 24;
  const uint32_t V_FULL = Q_FULL + 32, V_EMPTY = Q_FULL + 40, S_FULL = Q_FULL + 48 /* [2] */,
                 S_EMPTY = Q_FULL + 64 /* [2] */, P_FULL = Q_FULL + 80, PV_FULL = Q_FULL + 88,
                 PV_EMPTY = Q_FULL + 96, DRAIN = Q_FULL + 104;
  uint32_t* tmem_slot = (uint32_t*)(smem + off_bar + 112);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    ptx::mbar_init(Q_FULL, 1);
    ptx::mbar_init(Q_EMPTY, 1);
    ptx::mbar_init(K_FULL, 1);
    ptx::mbar_init(K_EMPTY, 1);
    ptx::mbar_init(V_FULL, 1);
    ptx::mbar_init(V_EMPTY, 1);
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(S_FULL + 8 * b, 1);
      ptx::mbar_init(S_EMPTY + 8 * b, 8);
    }
    ptx::mbar_init(P_FULL, 8);
    ptx::mbar_init(PV_FULL, 1);
    ptx::mbar_init(PV_EMPTY, 8);
    ptx::mbar_init(DRAIN, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // S of tile g: columns (g & 1) * 128 .. + 127; O_t: 2D columns from 256
  const uint32_t PV_COL = 256;
  const int total_items = a.BH * a.nq * a.nsplit;

  if (warp == 0) {
    // ------------------------------------------------ Q and K loader
    if (lane == 0) {
      int qi = 0, g = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < total_items && ok; it += gridDim.x) {
        const int sp = it % a.nsplit, bq = it / a.nsplit;
        const int bh = bq / a.nq, qt = bq % a.nq;
        const int kt0 = a.nk * sp / a.nsplit, kt1 = a.nk * (sp + 1) / a.nsplit;
        if (!ptx::mbar_wait(Q_EMPTY, (qi & 1) ^ 1, kAttnWaitNs)) {
          atomicExch(a.err, 21);
          ok = false;
          break;
        }
        ++qi;
        ptx::mbar_expect_tx(Q_FULL, 2 * q_plane);
        ptx::bulk_g2s(sbase + off_q, a.Qp + ((long long)bh * a.nq + qt) * 2 * (kTQ * D), 2 * q_plane, Q_FULL);
        for (int kt = kt0; kt < kt1; ++kt, ++g) {
          // the K tile is free once the previous tile's S MMAs have read it
          if (!ptx::mbar_wait(K_EMPTY, (g & 1) ^ 1, kAttnWaitNs)) {
            atomicExch(a.err, 22);
            ok = false;
            break;
          }
          ptx::mbar_expect_tx(K_FULL, k_bytes);
          ptx::bulk_g2s(sbase + off_k, a.Kp + ((long long)bh * a.nk + kt) * (2 * kTK * D), k_bytes, K_FULL);
        }
      }
      // no copy left in flight
      if (qi > 0) ptx::mbar_wait(Q_FULL, (qi - 1) & 1, kAttnWaitNs);
      if (g > 0) ptx::mbar_wait(K_FULL, (g - 1) & 1, kAttnWaitNs);
    }
    __syncwarp();
  } else if (warp == 10) {
    // ------------------------------------------------ V loader
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < total_items && ok; it += gridDim.x) {
        const int sp = it % a.nsplit, bq = it / a.nsplit;
        const int bh = bq / a.nq;
        const int kt0 = a.nk * sp / a.nsplit, kt1 = a.nk * (sp + 1) / a.nsplit;
        for (int kt = kt0; kt < kt1; ++kt, ++g) {
          // free once the previous tile's P.V MMAs have read it
          if (!ptx::mbar_wait(V_EMPTY, (g & 1) ^ 1, kAttnWaitNs)) {
            atomicExch(a.err, 29);
            ok = false;
            break;
          }
          ptx::mbar_expect_tx(V_FULL, v_bytes);
          ptx::bulk_g2s(sbase + off_v, a.Vp + ((long long)bh * a.nk + kt) * (2 * kTK * D), v_bytes, V_FULL);
        }
      }
      if (g > 0) ptx::mbar_wait(V_FULL, (g - 1) & 1, kAttnWaitNs);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    // Order: S_0, S_1, PV_0, S_2, PV_1, ...: the next tile's S is computed while
    // the softmax warps work on this one (S double-buffered in TMEM).
    if (lane == 0) {
      const uint32_t id_s = ptx::idesc_bf16_f32(128, kTK);
      const uint32_t id_v2 = ptx::idesc_bf16_f32(128, 2 * D), id_v1 = ptx::idesc_bf16_f32(128, D);
      const uint32_t lbo_q = (uint32_t)kTQ * 16u, lbo_k = (uint32_t)2 * kTK * 16u;
      const uint32_t lbo_p = (uint32_t)kTQ * 16u, lbo_v = (uint32_t)2 * D * 16u;
      int qi = 0, g = 0;
      bool ok = true;
      // O_h = Phi.[Vhi|Vlo] (N = 2D) + Plo.Vhi (N = D), K = 128 keys in steps of 16
      auto issue_pv = [&](int h) {
        if (!ptx::mbar_wait(P_FULL, h & 1, kAttnWaitNs) || !ptx::mbar_wait(V_FULL, h & 1, kAttnWaitNs) ||
            !ptx::mbar_wait(PV_EMPTY, (h & 1) ^ 1, kAttnWaitNs)) {
          atomicExch(a.err, 25);
          ok = false;
          return;
        }
        ptx::tc_fence_after();
        for (int kk = 0; kk < kTK / 16; ++kk) {
          const uint64_t dph = ptx::smem_desc(sbase + off_p + (uint32_t)kk * 2u * lbo_p, lbo_p, 128);
          const uint64_t dpl = ptx::smem_desc(sbase + off_p + p_plane + (uint32_t)kk * 2u * lbo_p, lbo_p, 128);
          const uint64_t dv = ptx::smem_desc(sbase + off_v + (uint32_t)kk * 2u * lbo_v, lbo_v, 128);
          ptx::mma_bf16(tmem + PV_COL, dph, dv, id_v2, kk > 0 ? 1u : 0u);
          ptx::mma_bf16(tmem + PV_COL, dpl, dv, id_v1, 1u);
        }
        ptx::mma_commit(PV_FULL);
        ptx::mma_commit(V_EMPTY);
      };
      for (int it = blockIdx.x; it < total_items && ok; it += gridDim.x) {
        const int sp = it % a.nsplit;
        const int kt0 = a.nk * sp / a.nsplit, kt1 = a.nk * (sp + 1) / a.nsplit;
        if (!ptx::mbar_wait(Q_FULL, qi & 1, kAttnWaitNs)) {
          atomicExch(a.err, 23);
          ok = false;
          break;
        }
        ++qi;
        for (int kt = kt0; kt < kt1 && ok; ++kt, ++g) {
          const int b = g & 1;
          if (!ptx::mbar_wait(K_FULL, g & 1, kAttnWaitNs) ||
              !ptx::mbar_wait(S_EMPTY + 8 * b, ((g >> 1) & 1) ^ 1, kAttnWaitNs)) {
            atomicExch(a.err, 24);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          // S = Qhi.Khi + Qhi.Klo + Qlo.Khi (N = 128 each; K tile rows 0-127 hi, 128-255 lo)
          const uint32_t s_col = tmem + (uint32_t)(b * kTK);
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t dqh = ptx::smem_desc(sbase + off_q + (uint32_t)kk * 2u * lbo_q, lbo_q, 128);
            const uint64_t dql = ptx::smem_desc(sbase + off_q + q_plane + (uint32_t)kk * 2u * lbo_q, lbo_q, 128);
            const uint64_t dkh = ptx::smem_desc(sbase + off_k + (uint32_t)kk * 2u * lbo_k, lbo_k, 128);
            const uint64_t dkl = ptx::smem_desc(sbase + off_k + kTK * 16u + (uint32_t)kk * 2u * lbo_k, lbo_k, 128);
            ptx::mma_bf16(s_col, dqh, dkh, id_s, kk > 0 ? 1u : 0u);
            ptx::mma_bf16(s_col, dqh, dkl, id_s, 1u);
            ptx::mma_bf16(s_col, dql, dkh, id_s, 1u);
          }
          ptx::mma_commit(S_FULL + 8 * b);
          ptx::mma_commit(K_EMPTY);
          if (kt + 1 == kt1) ptx::mma_commit(Q_EMPTY);
          if (g > 0) issue_pv(g - 1);
        }
      }
      if (ok && g > 0) issue_pv(g - 1);
      ptx::mma_commit(DRAIN);
      ptx::mbar_wait(DRAIN, 0, kAttnWaitNs);  // every MMA done before TMEM is freed
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ softmax warps 2-9
    // Two warps per TMEM lane quarter: warp w reads lanes 32 (w % 4) .. +31
    // (one query row per thread); half hf = (w - 2) / 4 takes key columns
    // [64 hf, 64 hf + 64) of every tile and head dimensions [hf D/2, (hf+1) D/2)
    // of O.  The pair exchanges its row maxima through shared memory (named
    // barrier 1 + quarter, 64 threads) once per tile and its row sums once per
    // item; everything else is per half.
    constexpr int DH = D / 2;
    constexpr int CH = kTK / 2;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int hf = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t pair_bar = 1u + (uint32_t)quarter;
    float* red_m = reinterpret_cast<float*>(smem + off_red);  // [tile parity][half][128 rows]
    float* red_l = red_m + 2 * 2 * kTQ;                       // [half][128 rows]
    const int nb = 2 * a.window + 1;
    int kvi = 0;  // tiles seen by this CTA (g)
    bool ok = true;
    for (int it = blockIdx.x; it < total_items && ok; it += gridDim.x) {
      const int sp = it % a.nsplit, bq = it / a.nsplit;
      const int bh = bq / a.nq, qt = bq % a.nq;
      const int kt0 = a.nk * sp / a.nsplit, kt1 = a.nk * (sp + 1) / a.nsplit;
      const int i = qt * kTQ + row;  // query index
      float o[DH];
#pragma unroll
      for (int d = 0; d < DH; ++d) o[d] = 0.f;
      float m = -INFINITY, l = 0.f;
      float rk[2 * kMaxWin + 1];
      if (a.window >= 0) {
        const float* rr = a.rk + ((long long)bh * a.P + (i < a.P ? i : 0)) * nb;
        for (int r = 0; r < nb; ++r) rk[r] = rr[r];
      }
      for (int kt = kt0; kt < kt1; ++kt, ++kvi) {
        const int b = kvi & 1;
        const bool got = __all_sync(0xffffffffu, ptx::mbar_wait(S_FULL + 8 * b, (kvi >> 1) & 1, kAttnWaitNs));
        if (!got) {
          if (lane == 0) atomicExch(a.err, 26);
          ok = false;
        }
        // The pair takes every named barrier together: an error in either half
        // (a bounded wait that ran out) ends both here, never between barriers.
        ok = ptx::named_bar_and(pair_bar, 64, ok);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint32_t s_col = tmem + lane_base + (uint32_t)(b * kTK + hf * CH);
        const int j0 = kt * kTK + hf * CH;
        // pass A: row max of this half tile, then of the tile through the pair
        float tmax = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < CH; c += 32) {
          float s1[32];
          ptx::tmem_ld32(s_col + (uint32_t)c, s1);
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const int j = j0 + c + k;
            float s = s1[k];
            if (a.window >= 0) {
              const int rel = j - i;
              if (rel >= -a.window && rel <= a.window) s = s + rk[rel + a.window];
            }
            if (j >= a.P) s = -INFINITY;
            tmax = fmaxf(tmax, s);
          }
        }
        red_m[(b * 2 + hf) * kTQ + row] = tmax;
        ptx::named_bar(pair_bar, 64);
        tmax = fmaxf(tmax, red_m[(b * 2 + (hf ^ 1)) * kTQ + row]);
        const float m_new = fmaxf(m, tmax);
        // fold the previous tile's O_t (computed with exp(s - m)) into this half's dimensions
        if (kt > kt0) {
          const bool pv = __all_sync(0xffffffffu, ptx::mbar_wait(PV_FULL, (kvi - 1) & 1, kAttnWaitNs));
          if (!pv) {
            if (lane == 0) atomicExch(a.err, 27);
            ok = false;
            continue;  // to the next tile's pair barrier, which ends the item for both halves
          }
          ptx::tc_fence_after();
#pragma unroll
          for (int c = 0; c < DH; c += 16) {
            float u1[16], u2[16];
            ptx::tmem_ld16(tmem + lane_base + PV_COL + (uint32_t)(hf * DH + c), u1);
            ptx::tmem_ld16(tmem + lane_base + PV_COL + (uint32_t)(D + hf * DH + c), u2);
#pragma unroll
            for (int k = 0; k < 16; ++k) o[c + k] = o[c + k] + (u1[k] + u2[k]);
          }
          ptx::tc_fence_before();
          if (lane == 0) ptx::mbar_arrive(PV_EMPTY);
        }
        // rescale the accumulator (all earlier tiles) to the new max
        const float scale = (m == -INFINITY) ? 0.f : expf(m - m_new);
#pragma unroll
        for (int d = 0; d < DH; ++d) o[d] *= scale;
        l *= scale;
        // pass B: p = exp(s - m_new) -> bf16 hi / lo planes, this half's row sum.
        // The P planes are free: the previous tile's P.V MMAs finished (folded
        // above, or at the end of the previous item).
        float sum = 0.f;
#pragma unroll 1
        for (int c = 0; c < CH; c += 32) {
          float s1[32];
          ptx::tmem_ld32(s_col + (uint32_t)c, s1);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint16_t ph16[16], pl16[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const int j = j0 + c + 16 * h + k;
              float s = s1[16 * h + k];
              if (a.window >= 0) {
                const int rel = j - i;
                if (rel >= -a.window && rel <= a.window) s = s + rk[rel + a.window];
              }
              const float p = (j < a.P && m_new != -INFINITY) ? expf(s - m_new) : 0.f;
              sum += p;
              split2(p, ph16[k], pl16[k]);
            }
#pragma unroll
            for (int g2 = 0; g2 < 2; ++g2) {
              const int jc = (hf * CH + c + 16 * h) / 8 + g2;  // key chunk
              const uint32_t off = (uint32_t)jc * (kTQ * 16u) + (uint32_t)row * 16u;
              const uint4 vh = *reinterpret_cast<const uint4*>(ph16 + 8 * g2);
              const uint4 vl = *reinterpret_cast<const uint4*>(pl16 + 8 * g2);
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + off_p + off), "r"(vh.x), "r"(vh.y),
                           "r"(vh.z), "r"(vh.w)
                           : "memory");
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + off_p + p_plane + off), "r"(vl.x),
                           "r"(vl.y), "r"(vl.z), "r"(vl.w)
                           : "memory");
            }
          }
        }
        l += sum;
        m = m_new;
        ptx::fence_proxy_async_smem();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          ptx::mbar_arrive(S_EMPTY + 8 * b);
          ptx::mbar_arrive(P_FULL);
        }
      }
      // the last tile's O_t (an error in the tile loop skips it; the pair
      // barrier below then ends the item for both halves)
      if (ok) {
        const uint32_t ph = (kvi - 1) & 1;
        const bool pv = __all_sync(0xffffffffu, ptx::mbar_wait(PV_FULL, ph, kAttnWaitNs));
        if (!pv) {
          if (lane == 0) atomicExch(a.err, 28);
          ok = false;
        } else {
          ptx::tc_fence_after();
#pragma unroll
          for (int c = 0; c < DH; c += 16) {
            float u1[16], u2[16];
            ptx::tmem_ld16(tmem + lane_base + PV_COL + (uint32_t)(hf * DH + c), u1);
            ptx::tmem_ld16(tmem + lane_base + PV_COL + (uint32_t)(D + hf * DH + c), u2);
#pragma unroll
            for (int k = 0; k < 16; ++k) o[c + k] = o[c + k] + (u1[k] + u2[k]);
          }
          ptx::tc_fence_before();
          if (lane == 0) ptx::mbar_arrive(PV_EMPTY);
        }
      }
      // the row sum: this half's plus the partner's (same max, same rescaling)
      red_l[hf * kTQ + row] = l;
      ok = ptx::named_bar_and(pair_bar, 64, ok);
      if (!ok) break;
      l = red_l[row] + red_l[kTQ + row];
      if (i < a.P && a.nsplit > 1) {
        // partial result of this key range: unnormalised O, row max and sum
        const long long pr = ((long long)bh * a.nsplit + sp) * a.P + i;
        float* po = a.po + pr * D + hf * DH;
#pragma unroll
        for (int d = 0; d < DH; d += 4) *reinterpret_cast<float4*>(po + d) = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
        if (hf == 0) {
          a.pml[2 * pr] = m;
          a.pml[2 * pr + 1] = l;
        }
      } else if (i < a.P) {
        const int b = bh / a.heads, h = bh % a.heads;
        float* yr = a.y + ((long long)b * a.P + i) * a.y_ld + h * D + hf * DH;
        const float inv_l = 1.f / l;
        if (a.window >= 0) {
          // band term: p(i, i + r - W) from the final max / sum, times emb_v[r]
          const float* sbr = a.sb + ((long long)bh * a.P + i) * nb;
          float pb[2 * kMaxWin + 1];
          for (int r = 0; r < nb; ++r) pb[r] = expf(sbr[r] - m) * inv_l;
#pragma unroll
          for (int d = 0; d < DH; ++d) {
            float band = 0.f;
            for (int r = 0; r < nb; ++r) band = fmaf(pb[r], a.emb_v[(long long)r * D + hf * DH + d], band);
            o[d] = o[d] * inv_l + band;
          }
        } else {
#pragma unroll
          for (int d = 0; d < DH; ++d) o[d] = o[d] * inv_l;
        }
#pragma unroll
        for (int d = 0; d < DH; d += 4) *reinterpret_cast<float4*>(yr + d) = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, 512);
}

// Merge of the key ranges of one (chunk x head, query row), one warp, lanes
// over the head dimension: M = max m_s, L = sum exp(m_s - M) l_s, O = sum
// exp(m_s - M) O_s; then y = O / L plus the band term p(i, i + r - W) emb_v[r]
// with p from the final M and L, as in the one-range epilogue.
__global__ void attn_combine_kernel(const float* __restrict__ po, const float* __restrict__ pml, int nsplit, int P,
                                    int heads, int D, int W, const float* __restrict__ sb,
                                    const float* __restrict__ emb_v, float* __restrict__ y, int y_ld,
                                    long long rows) {
  const long long wr = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wr >= rows) return;
  const int i = (int)(wr % P);
  const int bh = (int)(wr / P);
  const int b = bh / heads, h = bh % heads;
  float M = -INFINITY;
  for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, pml[2 * (((long long)bh * nsplit + sp) * P + i)]);
  float L = 0.f, o[3] = {0.f, 0.f, 0.f};
  for (int sp = 0; sp < nsplit; ++sp) {
    const long long pr = ((long long)bh * nsplit + sp) * P + i;
    const float ms = pml[2 * pr];
    const float f = ms == -INFINITY ? 0.f : expf(ms - M);
    L += f * pml[2 * pr + 1];
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      const int d = lane + 32 * t;
      if (d < D) o[t] = fmaf(f, po[pr * D + d], o[t]);
    }
  }
  const float inv_l = 1.f / L;
  float* yr = y + ((long long)b * P + i) * y_ld + h * D;
  const int nb = 2 * W + 1;
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    const int d = lane + 32 * t;
    if (d >= D) continue;
    float v = o[t] * inv_l;
    if (W >= 0) {
      const float* sbr = sb + ((long long)bh * P + i) * nb;
      float band = 0.f;
      for (int r = 0; r < nb; ++r) band = fmaf(expf(sbr[r] - M) * inv_l, emb_v[(long long)r * D + d], band);
      v = v + band;
    }
    yr[d] = v;
  }
}

// One warp per (chunk x head, query row): rk[r] = qs . emb_k[r] (added to the
// band of S) and sb[r] = qs . k[i + r - W] + rk[r] (the band logits the output
// term uses), r < 2W + 1, lanes over the head dimension.
__global__ void attn_band_kernel(const float* __restrict__ qkv, int ld, int q_off, int k_off, int heads, int D,
                                 int P, int W, float q_div, const float* __restrict__ emb_k, float* __restrict__ rk,
                                 float* __restrict__ sb, long long rows) {
  const long long wr = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wr >= rows) return;
  const int i = (int)(wr % P);
  const int bh = (int)(wr / P);
  const int b = bh / heads, h = bh % heads;
  const float* q = qkv + ((long long)b * P + i) * ld + q_off + h * D;
  const int nb = 2 * W + 1;
  float qs[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) qs[t] = lane + 32 * t < D ? q[lane + 32 * t] / q_div : 0.f;
  for (int r = 0; r < nb; ++r) {
    const int j = i + r - W;
    float se = 0.f, sk = 0.f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int d = lane + 32 * t;
      if (d < D) {
        se = fmaf(qs[t], emb_k[(long long)r * D + d], se);
        if (j >= 0 && j < P) sk = fmaf(qs[t], qkv[((long long)b * P + j) * ld + k_off + h * D + d], sk);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      se += __shfl_xor_sync(0xffffffffu, se, o);
      sk += __shfl_xor_sync(0xffffffffu, sk, o);
    }
    if (lane == 0) {
      rk[wr * nb + r] = se;
      sb[wr * nb + r] = (j >= 0 && j < P) ? sk + se : -INFINITY;
    }
  }
}

}  // namespace

// Returns false when the shape is not served (the caller then runs the SIMT kernel).
bool k_attention_tc(Context* ctx, const float* qkv, int ld, int q_off, int k_off, int v_off, const float* emb_k,
                    const float* emb_v, int B, int heads, int D, int P, int window, float q_div, float* y, int y_ld) {
  if (B * P == 0) return true;
  if ((D != 64 && D != 96) || window > kMaxWin) return false;
  cudaStream_t st = ctx->stream;
  const int nq = (P + kTQ - 1) / kTQ, nk = (P + kTK - 1) / kTK;
  const int BH = B * heads;
  const size_t tile_elems = (size_t)2 * kTQ * D;  // one Q tile (2 planes) == one K or V tile
  DevBuf Qp(ctx, sizeof(uint16_t) * tile_elems * BH * nq), Kp(ctx, sizeof(uint16_t) * tile_elems * BH * nk),
      Vp(ctx, sizeof(uint16_t) * tile_elems * BH * nk);
  const long long total = (long long)BH * nq * kTQ * (D / 8);
  attn_pack_kernel<<<(int)std::min<long long>((total + 255) / 256, 148ll * 32), 256, 0, st>>>(
      qkv, ld, q_off, k_off, v_off, heads, D, P, nq, nk, q_div, Qp.as<uint16_t>(), Kp.as<uint16_t>(),
      Vp.as<uint16_t>(), total);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
  DevBuf rk, sb;
  if (window >= 0) {
    const long long rows = (long long)BH * P, n = rows * (2 * window + 1);
    rk = DevBuf(ctx, sizeof(float) * (size_t)n);
    sb = DevBuf(ctx, sizeof(float) * (size_t)n);
    attn_band_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(qkv, ld, q_off, k_off, heads, D, P, window, q_div,
                                                                 emb_k, rk.f(), sb.f(), rows);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
  }
  AttnArgs a;
  a.Qp = Qp.as<uint16_t>();
  a.Kp = Kp.as<uint16_t>();
  a.Vp = Vp.as<uint16_t>();
  a.heads = heads;
  a.D = D;
  a.P = P;
  a.nq = nq;
  a.nk = nk;
  a.y = y;
  a.y_ld = y_ld;
  a.window = window;
  a.rk = rk.f();
  a.sb = sb.f();
  a.emb_v = emb_v;
  a.err = ctx->d_err;  // reported by the context's bounded sync
  a.BH = BH;
  const size_t smem = 1024 + (size_t)2 * kTQ * D * 2 + (size_t)2 * kTK * D * 2 * 2 + (size_t)2 * kTQ * kTK * 2 + 128 + 3 * kTQ * sizeof(float) * 2;
  static std::atomic<uint64_t> attr_done{0};
  int dev = 0;
  RVC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && !(attr_done.load() & (1ull << dev))) {
    RVC_CUDA_TRY(cudaFuncSetAttribute(tc_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    RVC_CUDA_TRY(cudaFuncSetAttribute(tc_attn_kernel<96>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    attr_done.fetch_or(1ull << dev);
  }
  // Split the keys when the (query tile) items fill the SMs' waves poorly (one
  // sequence, few heads): the split count maximises items / (waves x SMs),
  // at least 2 key tiles per split and a charge of 0.05 per extra split for the
  // partial results and the merge.
  const int sms = ctx->num_sms();
  int nsplit = 1;
  {
    const long long base = (long long)BH * nq;
    double best = -1.0;
    for (int ns = 1; ns <= std::max(1, nk / 2); ++ns) {
      const long long it = base * ns, waves = (it + sms - 1) / sms;
      const double score = (double)it / (double)(waves * sms) - 0.05 * (ns - 1);
      if (score > best + 1e-9) {
        best = score;
        nsplit = ns;
      }
    }
  }
  a.nsplit = nsplit;
  DevBuf po, pml;
  if (nsplit > 1) {
    po = DevBuf(ctx, sizeof(float) * (size_t)BH * nsplit * P * D);
    pml = DevBuf(ctx, sizeof(float) * (size_t)BH * nsplit * P * 2);
  }
  a.po = po.p ? po.f() : nullptr;
  a.pml = pml.p ? pml.f() : nullptr;
  const int items = BH * nq * nsplit;
  if (D == 64)
    tc_attn_kernel<64><<<std::min(items, sms), kAThreads, smem, st>>>(a);
  else
    tc_attn_kernel<96><<<std::min(items, sms), kAThreads, smem, st>>>(a);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
  if (nsplit > 1) {
    const long long rows = (long long)BH * P;
    attn_combine_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(po.f(), pml.f(), nsplit, P, heads, D, window,
                                                                     sb.p ? sb.f() : nullptr, emb_v, y, y_ld, rows);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
  }
  return true;  // the packed tiles are released to the stream-ordered cache: later work queues behind this kernel
}

}  // namespace rvc
