// tcgen05 implicit-GEMM convolution: persistent, TMA-fed, BF16x3 split
// precision with fp32 accumulation in TMEM.  Operator contract in conv.cuh.
//
// A CTA loops over tiles of msub*128 output rows x bn output channels.  Each
// weight stage (one tap x one cb-channel block, bf16 hi and lo planes) feeds
// msub MMAs, one per 128-row subtile, so weights stream through shared memory
// once per msub*128 rows.  Accumulators live in TMEM: nacc sets of msub*bn
// columns, so the epilogue of one tile overlaps the main loop of the next.
//
//   warp 0       weight producer: cp.async.bulk of packed hi/lo planes into a
//                `stages`-deep ring
//   warp 1       TMEM owner + single-thread tcgen05.mma issuer
//   warp 2       activation loader: TMA (cp.async.bulk.tensor) of the fp32 halo
//                tile (out-of-range rows zero-filled = conv padding) into a
//                staging buffer
//   warps 3..6   converters: staging fp32 -> prologue activation -> bf16 hi/lo
//                MMA planes (the halo tile serves every tap of the block)
//   warps 7..10  epilogue: TMEM -> registers; residual / accumulator tiles
//                arrive by TMA into 128B-swizzled slots (prefetched one step
//                ahead), the result is written in place and stored by TMA.
//                Transposed-conv phases (strided output rows) and unaligned
//                cases use direct vector stores instead.
#include "conv.cuh"
#include "tc_ptx.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>

namespace rvc {

constexpr int kTM = 128;
constexpr int kWarps = 11;
constexpr int kThreads = kWarps * 32;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per barrier wait
constexpr int kEpiCols = 32;
constexpr uint32_t kSlotBytes = kTM * kEpiCols * 4;  // one 128 x 32 fp32 tile
constexpr int kEpiRows = 32;                           // rows per epilogue warp (its TMEM lane quarter)
constexpr uint32_t kWarpSlotBytes = kEpiRows * kEpiCols * 4;  // a warp's 32 x 32 part of a slot
constexpr int kBarriers = 22 + 16;                     // fixed barriers + EPI_W[4 slots][4 warps]

struct TcMaps {
  CUtensorMap a, res, acc, y;
};

struct TcPlan {
  int msub, nacc, arows_pad, stages;
  int nstg, box_rows, nbox;
  int nslot, acc_slot, tma_epi;
  uint32_t a_plane, b_plane, stg_bytes;
  uint32_t off_a, off_stg, off_b, off_epi, off_bar, smem_bytes;
  uint32_t off_bias;  // bias staged in shared memory (0: read from global)
  int bias_n;
  int w_res;          // whole packed weight tensor resident in shared memory
  uint32_t off_w, w_bytes;
  int ephase;         // epilogue maps are 4-D {ch, phase, q, b} (transposed conv)
  uint32_t tmem_cols;
  int tiles_m, ntiles, total_tiles;
  int vec;
};

// Direct epilogue for N (16 or 32) consecutive output channels of one row;
// every global load of the step is issued before any is used.
// Terms of the prologue / epilogue a launch uses, as compile-time flags of
// tc_conv_kernel: the models' layers use a handful of combinations, and with
// only those terms compiled the epilogue warps skip the instruction fetch and
// branches of the unused ones (the activation switch alone was unrolled 32x).
// kTGeneric reads the terms from ConvArgs at run time.  Same operations in
// the same order either way.
constexpr int kTBias = 1, kTBias2 = 2, kTRes = 4, kTResSub = 8, kTAcc = 16, kTDiv = 32, kTLeaky = 64, kTRelu = 128,
              kTGelu = 256, kTGeneric = 512;

// the output activation of one value (act_apply's formulas)
template <int F>
__device__ __forceinline__ float act_val(float x, const ConvArgs& a) {
  if constexpr ((F & kTGeneric) != 0) return act_apply(x, a.out_act, a.out_slope);
  else if constexpr ((F & kTLeaky) != 0) return act_apply(x, kActLeaky, a.out_slope);
  else if constexpr ((F & kTRelu) != 0) return act_apply(x, kActRelu, 0.f);
  else if constexpr ((F & kTGelu) != 0) return gelu_as(x);
  else return x;
}

template <int N, int F>
__device__ __forceinline__ void epi_direct(const ConvArgs& a, int b, int prow, int cg0, float (&v)[N], int vec) {
  constexpr bool gen = (F & kTGeneric) != 0;
  const bool t_bias = gen ? a.bias != nullptr : (F & kTBias) != 0;
  const bool t_bias2 = gen ? a.bias2 != nullptr : (F & kTBias2) != 0;
  const bool t_res = gen ? a.res != nullptr : (F & kTRes) != 0;
  const bool t_sub = gen ? a.res_sub != 0 : (F & kTResSub) != 0;
  const bool t_acc = gen ? a.accin != nullptr : (F & kTAcc) != 0;
  const bool t_div = gen ? a.out_div != 0.f : (F & kTDiv) != 0;
  if (!vec) {
#pragma unroll
    for (int i = 0; i < N; ++i) conv_epilogue(a, b, prow, cg0 + i, v[i]);
    return;
  }
  constexpr int Q = N / 4;
  float4 rb[Q], ra[Q];
  if (t_res) {
    const float4* p =
        reinterpret_cast<const float4*>(a.res + (long long)b * a.res_bs + (long long)prow * a.res_ld + cg0);
#pragma unroll
    for (int q = 0; q < Q; ++q) rb[q] = p[q];
  }
  if (t_acc) {
    const float4* p =
        reinterpret_cast<const float4*>(a.accin + (long long)b * a.acc_bs + (long long)prow * a.acc_ld + cg0);
#pragma unroll
    for (int q = 0; q < Q; ++q) ra[q] = p[q];
  }
  float out[N];
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    float x[4] = {v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]};
    const float4 bi = t_bias ? __ldg(reinterpret_cast<const float4*>(a.bias + cg0) + q) : make_float4(0, 0, 0, 0);
    const float4 b2 = t_bias2 ? __ldg(reinterpret_cast<const float4*>(a.bias2 + (long long)b * a.bias2_bs + cg0) + q)
                              : make_float4(0, 0, 0, 0);
    const float bb[4] = {bi.x, bi.y, bi.z, bi.w}, b22[4] = {b2.x, b2.y, b2.z, b2.w};
    const float rr[4] = {rb[q].x, rb[q].y, rb[q].z, rb[q].w}, aa[4] = {ra[q].x, ra[q].y, ra[q].z, ra[q].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float t = x[e];
      if (t_bias) t += bb[e];
      if (t_bias2) t += b22[e];
      if (t_res) t = t_sub ? (rr[e] - t) : (t + rr[e]);
      if (t_acc) t = aa[e] + t;
      if (t_div) t = t / a.out_div;
      out[4 * q + e] = t;
    }
  }
  const long long o = (long long)b * a.y_bs + (long long)prow * a.y_ld + cg0;
  if (a.y_raw) {
    float4* p = reinterpret_cast<float4*>(a.y_raw + o);
#pragma unroll
    for (int q = 0; q < Q; ++q) p[q] = make_float4(out[4 * q], out[4 * q + 1], out[4 * q + 2], out[4 * q + 3]);
  }
  float4* p = reinterpret_cast<float4*>(a.y + o);
#pragma unroll
  for (int q = 0; q < Q; ++q)
    p[q] = make_float4(act_val<F>(out[4 * q], a), act_val<F>(out[4 * q + 1], a), act_val<F>(out[4 * q + 2], a),
                       act_val<F>(out[4 * q + 3], a));
}

// Issues the BF16x3 MMAs of one weight stage: for each 16-wide k step and each
// 128-row subtile, D += Ahi*Bhi + Ahi*Blo + Alo*Bhi.  Descriptors are built once
// and advanced by adding encoded offsets (the start-address field holds
// addr >> 4; shared addresses stay below 256 KB, so an add never carries out of
// the 14-bit field), which keeps the single issuing thread at a few
// instructions per MMA.
template <int MSUB, int KK>
__device__ __forceinline__ void issue_stage(uint32_t dbase, uint64_t dah0, uint64_t dal0, uint64_t dbh0,
                                            uint64_t dbl0, uint32_t lbo_a, uint32_t lbo_b, int bn, uint32_t idesc,
                                            bool first) {
#pragma unroll
  for (int kk = 0; kk < KK; ++kk) {
    const uint64_t ka = (uint64_t)((2u * (uint32_t)kk * lbo_a) >> 4);
    const uint64_t kb = (uint64_t)((2u * (uint32_t)kk * lbo_b) >> 4);
    // products grouped across subtiles: an MMA's accumulator was last written
    // MSUB instructions earlier (sa: 128 rows x 16 B, >> 4)
#pragma unroll
    for (int sub = 0; sub < MSUB; ++sub)
      ptx::mma_bf16(dbase + (uint32_t)(sub * bn), dah0 + ka + (uint64_t)(sub * kTM), dbh0 + kb, idesc,
                    (first && kk == 0) ? 0u : 1u);
#pragma unroll
    for (int sub = 0; sub < MSUB; ++sub)
      ptx::mma_bf16(dbase + (uint32_t)(sub * bn), dah0 + ka + (uint64_t)(sub * kTM), dbl0 + kb, idesc, 1u);
#pragma unroll
    for (int sub = 0; sub < MSUB; ++sub)
      ptx::mma_bf16(dbase + (uint32_t)(sub * bn), dal0 + ka + (uint64_t)(sub * kTM), dbh0 + kb, idesc, 1u);
  }
}

// Stacked form: per 16-wide k step and subtile, D[0:2bn) += Ahi.[Bhi|Blo] (one
// N = 2bn MMA) and D[0:bn) += Alo.Bhi; the epilogue adds D[bn:2bn) to D[0:bn).
template <int MSUB, int KK>
__device__ __forceinline__ void issue_stacked(uint32_t dbase, uint64_t dah0, uint64_t dal0, uint64_t db0,
                                              uint32_t lbo_a, uint32_t lbo_b, int bn, uint32_t idesc2,
                                              uint32_t idesc1, bool first) {
#pragma unroll
  for (int kk = 0; kk < KK; ++kk) {
    const uint64_t ka = (uint64_t)((2u * (uint32_t)kk * lbo_a) >> 4);
    const uint64_t kb = (uint64_t)((2u * (uint32_t)kk * lbo_b) >> 4);
    // the subtiles' MMAs interleave, so consecutive MMAs never accumulate into
    // the same TMEM columns (the accumulation chain of one subtile advances
    // every MSUB instructions)
#pragma unroll
    for (int sub = 0; sub < MSUB; ++sub)
      ptx::mma_bf16(dbase + (uint32_t)(sub * 2 * bn), dah0 + ka + (uint64_t)(sub * kTM), db0 + kb, idesc2,
                    (first && kk == 0) ? 0u : 1u);
#pragma unroll
    for (int sub = 0; sub < MSUB; ++sub)
      ptx::mma_bf16(dbase + (uint32_t)(sub * 2 * bn), dal0 + ka + (uint64_t)(sub * kTM), db0 + kb, idesc1, 1u);
  }
}

__device__ __forceinline__ void issue_stacked_any(int msub, int kk, uint32_t dbase, uint64_t dah0, uint64_t dal0,
                                                  uint64_t db0, uint32_t lbo_a, uint32_t lbo_b, int bn,
                                                  uint32_t idesc2, uint32_t idesc1, bool first) {
#define RVC_ISSUE_S(M, K)                                                                  \
  if (msub == M && kk == K) {                                                              \
    issue_stacked<M, K>(dbase, dah0, dal0, db0, lbo_a, lbo_b, bn, idesc2, idesc1, first); \
    return;                                                                                \
  }
  RVC_ISSUE_S(1, 1) RVC_ISSUE_S(1, 2) RVC_ISSUE_S(1, 3) RVC_ISSUE_S(1, 4)
  RVC_ISSUE_S(2, 1) RVC_ISSUE_S(2, 2) RVC_ISSUE_S(2, 3) RVC_ISSUE_S(2, 4)
  RVC_ISSUE_S(4, 1) RVC_ISSUE_S(4, 2) RVC_ISSUE_S(4, 3) RVC_ISSUE_S(4, 4)
#undef RVC_ISSUE_S
}

__device__ __forceinline__ void issue_any(int msub, int kk, uint32_t dbase, uint64_t dah0, uint64_t dal0,
                                          uint64_t dbh0, uint64_t dbl0, uint32_t lbo_a, uint32_t lbo_b, int bn,
                                          uint32_t idesc, bool first) {
#define RVC_ISSUE(M, K)                                                                    \
  if (msub == M && kk == K) {                                                              \
    issue_stage<M, K>(dbase, dah0, dal0, dbh0, dbl0, lbo_a, lbo_b, bn, idesc, first);      \
    return;                                                                                \
  }
  RVC_ISSUE(1, 1) RVC_ISSUE(1, 2) RVC_ISSUE(1, 3) RVC_ISSUE(1, 4)
  RVC_ISSUE(2, 1) RVC_ISSUE(2, 2) RVC_ISSUE(2, 3) RVC_ISSUE(2, 4)
  RVC_ISSUE(4, 1) RVC_ISSUE(4, 2) RVC_ISSUE(4, 3) RVC_ISSUE(4, 4)
#undef RVC_ISSUE
}

struct TileCoord {
  int b, s, nt, mt;
};
__device__ __forceinline__ TileCoord tile_coord(int tile, int nslices, int ntiles, int tiles_m) {
  TileCoord c;
  c.mt = tile % tiles_m;
  int r = tile / tiles_m;
  c.nt = r % ntiles;
  r /= ntiles;
  c.s = r % nslices;
  c.b = r / nslices;
  return c;
}

// Two fp32 values -> (hi, lo) bf16x2 words with hi = RN(x), lo = RN(x - hi),
// one paired conversion per word (same values as split_bf16 element by element).
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Activation of a whole 32-value epilogue row segment, the act chosen once.
// leaky_relu as max(x, s*x) when 0 <= s <= 1 (equal to x >= 0 ? x : s*x there).
__device__ __forceinline__ void act_row(float (&x)[32], int act, float slope) {
  switch (act) {
    case kActNone: return;
    case kActLeaky:
      if (slope >= 0.f && slope <= 1.f) {
#pragma unroll
        for (int k = 0; k < 32; ++k) x[k] = fmaxf(x[k], slope * x[k]);
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) x[k] = x[k] >= 0.f ? x[k] : slope * x[k];
      }
      return;
    default:
#pragma unroll
      for (int k = 0; k < 32; ++k) x[k] = act_apply(x[k], act, slope);
  }
}

template <int F>
__device__ __forceinline__ void act_row_t(float (&x)[32], const ConvArgs& a) {
  if constexpr ((F & kTGeneric) != 0) {
    act_row(x, a.out_act, a.out_slope);
  } else if constexpr ((F & kTLeaky) != 0) {  // slope in [0, 1] (tc_flags)
    const float sl = a.out_slope;
#pragma unroll
    for (int k = 0; k < 32; ++k) x[k] = fmaxf(x[k], sl * x[k]);
  } else if constexpr ((F & kTRelu) != 0) {
#pragma unroll
    for (int k = 0; k < 32; ++k) x[k] = act_apply(x[k], kActRelu, 0.f);
  } else if constexpr ((F & kTGelu) != 0) {
#pragma unroll
    for (int k = 0; k < 32; ++k) x[k] = gelu_as(x[k]);
  }
}

template <int F>
__global__ void __launch_bounds__(kThreads, 1)
    tc_conv_kernel(const __grid_constant__ ConvArgs a, const __grid_constant__ TcMaps maps, TcPlan g) {
  constexpr bool gen = (F & kTGeneric) != 0;
  const bool t_bias = gen ? a.bias != nullptr : (F & kTBias) != 0;
  const bool t_bias2 = gen ? a.bias2 != nullptr : (F & kTBias2) != 0;
  const bool t_res = gen ? a.res != nullptr : (F & kTRes) != 0;
  const bool t_sub = gen ? a.res_sub != 0 : (F & kTResSub) != 0;
  const bool t_acc = gen ? a.accin != nullptr : (F & kTAcc) != 0;
  const bool t_div = gen ? a.out_div != 0.f : (F & kTDiv) != 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int BN = a.bn, CB = a.cb;
  const int nblk = a.C_in / CB;
  const int MT = g.msub * kTM;
  const uint32_t LBO_A = (uint32_t)g.arows_pad * 16u;
  const bool STK = tc_stacked(BN);
  const int ACW = STK ? 2 * BN : BN;  // TMEM columns per 128-row subtile
  const uint32_t LBO_B = (uint32_t)(STK ? 2 * BN : BN) * 16u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = ptx::smem_u32(smem);
  const uint32_t bar0 = sbase + g.off_bar;
  // barriers: A_FULL[2] A_EMPTY[2] STG_FULL[4] STG_EMPTY[4] ACC_FULL[2] ACC_EMPTY[2] (4 unused) DRAIN
  //           W_FULL EPI_W[4 slots][4 epilogue warps] B_FULL[stages] B_EMPTY[stages], then the TMEM
  //           address slot
  const uint32_t A_FULL = bar0, A_EMPTY = bar0 + 16, STG_FULL = bar0 + 32, STG_EMPTY = bar0 + 64;
  const uint32_t ACC_FULL = bar0 + 96, ACC_EMPTY = bar0 + 112, DRAIN = bar0 + 160;
  const uint32_t W_FULL = bar0 + 168, EPI_W = bar0 + 176;
  const uint32_t B_FULL = EPI_W + 8u * 16, B_EMPTY = B_FULL + 8u * g.stages;
  uint32_t* tmem_slot = (uint32_t*)(smem + g.off_bar + 8 * (kBarriers + 2 * g.stages));
  auto a_plane = [&](int buf, int lo) { return sbase + g.off_a + (uint32_t)(2 * buf + lo) * g.a_plane; };
  auto b_plane = [&](int st, int lo) { return sbase + g.off_b + (uint32_t)(2 * st + lo) * g.b_plane; };
  auto stg = [&](int sb) { return g.off_stg + (uint32_t)sb * g.stg_bytes; };  // offset from smem
  const uint32_t slot_span = kSlotBytes * (g.acc_slot ? 2u : 1u);
  auto slot_main = [&](int s) { return g.off_epi + (uint32_t)s * slot_span; };
  auto slot_aux = [&](int s) { return g.off_epi + (uint32_t)s * slot_span + kSlotBytes; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(A_FULL + 8 * i, 128);
      ptx::mbar_init(A_EMPTY + 8 * i, 1);
      ptx::mbar_init(ACC_FULL + 8 * i, 1);
      ptx::mbar_init(ACC_EMPTY + 8 * i, 128);
    }
    for (int i = 0; i < 4; ++i) {
      ptx::mbar_init(STG_FULL + 8 * i, 1);
      ptx::mbar_init(STG_EMPTY + 8 * i, 128);
    }
    for (int i = 0; i < 16; ++i) ptx::mbar_init(EPI_W + 8 * i, 1);
    ptx::mbar_init(DRAIN, 1);
    ptx::mbar_init(W_FULL, 1);
    for (int i = 0; i < g.stages; ++i) {
      ptx::mbar_init(B_FULL + 8 * i, 1);
      ptx::mbar_init(B_EMPTY + 8 * i, 1);
    }
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), g.tmem_cols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ weight producer
    if (lane == 0 && g.w_res) {
      // whole packed tensor once per CTA (n-tile 0 is the only n-tile)
      ptx::mbar_expect_tx(W_FULL, g.w_bytes);
      const uint8_t* src = reinterpret_cast<const uint8_t*>(a.wpk);
      for (uint32_t o = 0; o < g.w_bytes; o += 32768u)
        ptx::bulk_g2s(sbase + g.off_w + o, src + o, min(32768u, g.w_bytes - o), W_FULL);
      ptx::mbar_wait(W_FULL, 0, kWaitNs);  // never exit with the copy in flight
    } else if (lane == 0) {
      const size_t blk_elems = 2u * (size_t)CB * BN;
      int ks = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
        const TileCoord c = tile_coord(tile, a.nslices, g.ntiles, g.tiles_m);
        const ConvSlice& S = a.sl[c.s];
        if (c.mt * MT >= S.rows) continue;
        for (int kb = 0; kb < nblk && ok; ++kb)
          for (int j = 0; j < S.ntaps; ++j, ++ks) {
            const int st = ks % g.stages, round = ks / g.stages;
            if (!ptx::mbar_wait(B_EMPTY + 8 * st, (round & 1) ^ 1, kWaitNs)) {
              ok = false;
              atomicExch(a.err, 1);
              break;
            }
            const uint16_t* src = a.wpk + ((size_t)((S.wtap0 + j) * g.ntiles + c.nt) * nblk + kb) * blk_elems;
            ptx::mbar_expect_tx(B_FULL + 8 * st, 2u * g.b_plane);
            ptx::bulk_g2s(b_plane(st, 0), src, g.b_plane, B_FULL + 8 * st);
            ptx::bulk_g2s(b_plane(st, 1), src + (size_t)CB * BN, g.b_plane, B_FULL + 8 * st);
          }
      }
      for (int k = (ks > g.stages ? ks - g.stages : 0); k < ks; ++k)  // no copy left in flight
        ptx::mbar_wait(B_FULL + 8 * (k % g.stages), (k / g.stages) & 1, kWaitNs);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = ptx::idesc_bf16_f32(kTM, BN);
      const uint32_t idesc2 = ptx::idesc_bf16_f32(kTM, 2 * BN);
      int ab = 0, it = 0;
      int st = 0, round = 0;  // weight ring stage and phase, counted (no per-tap division)
      // descriptor bases: start address >> 4 in the low bits and every offset
      // below a multiple of 16 B inside shared memory, so offsets are added
      const uint64_t d_a0 = ptx::smem_desc(a_plane(0, 0), LBO_A, 128), s_aplane = (uint64_t)(g.a_plane >> 4);
      const uint64_t d_b0 = ptx::smem_desc(b_plane(0, 0), LBO_B, 128), s_bplane = (uint64_t)(g.b_plane >> 4);
      const uint64_t d_w0 = ptx::smem_desc(sbase + g.off_w, LBO_B, 128);
      bool ok = true;
      if (g.w_res && !ptx::mbar_wait(W_FULL, 0, kWaitNs)) {
        ok = false;
        atomicExch(a.err, 10);
      }
      for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
        const TileCoord c = tile_coord(tile, a.nslices, g.ntiles, g.tiles_m);
        const ConvSlice& S = a.sl[c.s];
        if (c.mt * MT >= S.rows) continue;
        const int set = it % g.nacc;
        if (!ptx::mbar_wait(ACC_EMPTY + 8 * set, ((it / g.nacc) & 1) ^ 1, kWaitNs)) {
          ok = false;
          atomicExch(a.err, 2);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t dbase = tmem + (uint32_t)(set * g.msub * ACW);
        const int span = (S.ntaps - 1) * S.tap_step;
        const int shift = span < 0 ? -span : 0;
        bool first = true;
        for (int kb = 0; kb < nblk && ok; ++kb, ++ab) {
          const int buf = ab & 1;
          if (!ptx::mbar_wait(A_FULL + 8 * buf, (ab >> 1) & 1, kWaitNs)) {
            ok = false;
            atomicExch(a.err, 3);
            break;
          }
          const uint64_t da_buf = d_a0 + (uint64_t)(2 * buf) * s_aplane;
          for (int j = 0; j < S.ntaps; ++j) {
            uint64_t dbh0;
            if (g.w_res) {
              dbh0 = d_w0 + (uint64_t)((S.wtap0 + j) * nblk + kb) * 2u * s_bplane;
            } else {
              if (!ptx::mbar_wait(B_FULL + 8 * st, round & 1, kWaitNs)) {
                ok = false;
                atomicExch(a.err, 4);
                break;
              }
              ptx::tc_fence_after();
              dbh0 = d_b0 + (uint64_t)(2 * st) * s_bplane;
            }
            const uint64_t dah0 = da_buf + (uint64_t)(uint32_t)(j * S.tap_step + shift);
            const uint64_t dal0 = dah0 + s_aplane;
            if (STK) {
              issue_stacked_any(g.msub, CB / 16, dbase, dah0, dal0, dbh0, LBO_A, LBO_B, BN, idesc2, idesc, first);
            } else {
              issue_any(g.msub, CB / 16, dbase, dah0, dal0, dbh0, dbh0 + s_bplane, LBO_A, LBO_B, BN, idesc, first);
            }
            first = false;
            if (!g.w_res) {
              ptx::mma_commit(B_EMPTY + 8 * st);
              if (++st == g.stages) {
                st = 0;
                ++round;
              }
            }
          }
          if (ok) ptx::mma_commit(A_EMPTY + 8 * buf);
        }
        if (ok) ptx::mma_commit(ACC_FULL + 8 * set);
        ++it;
      }
      ptx::mma_commit(DRAIN);
      ptx::mbar_wait(DRAIN, 0, kWaitNs);
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------ activation loader (TMA)
    if (lane == 0) {
      const uint32_t bytes = (uint32_t)g.nbox * g.box_rows * CB * 4u;
      int ab = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
        const TileCoord c = tile_coord(tile, a.nslices, g.ntiles, g.tiles_m);
        const ConvSlice& S = a.sl[c.s];
        const int t0 = c.mt * MT;
        if (t0 >= S.rows) continue;
        const int span = (S.ntaps - 1) * S.tap_step;
        const int r_start = t0 + S.tap_base + (span < 0 ? span : 0);
        for (int kb = 0; kb < nblk; ++kb, ++ab) {
          const int sb = ab % g.nstg;
          if (!ptx::mbar_wait(STG_EMPTY + 8 * sb, ((ab / g.nstg) & 1) ^ 1, kWaitNs)) {
            ok = false;
            atomicExch(a.err, 5);
            break;
          }
          ptx::mbar_expect_tx(STG_FULL + 8 * sb, bytes);
          for (int i = 0; i < g.nbox; ++i)
            ptx::tma_load_3d(sbase + stg(sb) + (uint32_t)i * g.box_rows * CB * 4u, &maps.a, S.ci_off + kb * CB,
                             r_start + i * g.box_rows, c.b, STG_FULL + 8 * sb);
        }
      }
      for (int k = (ab > g.nstg ? ab - g.nstg : 0); k < ab; ++k)  // no copy left in flight
        ptx::mbar_wait(STG_FULL + 8 * (k % g.nstg), (k / g.nstg) & 1, kWaitNs);
    }
  } else if (warp < 7) {
    // ------------------------------------------------ converters
    const int tp = threadIdx.x - 96;
    const int c4n = CB / 4;
    int ab = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
      const TileCoord c = tile_coord(tile, a.nslices, g.ntiles, g.tiles_m);
      const ConvSlice& S = a.sl[c.s];
      if (c.mt * MT >= S.rows) continue;
      const int span = (S.ntaps - 1) * S.tap_step;
      const int arows = MT + (span < 0 ? -span : span);
      const int total = arows * c4n;
      for (int kb = 0; kb < nblk; ++kb, ++ab) {
        const int sb = ab % g.nstg, buf = ab & 1;
        if (!ptx::mbar_wait(STG_FULL + 8 * sb, (ab / g.nstg) & 1, kWaitNs) ||
            !ptx::mbar_wait(A_EMPTY + 8 * buf, ((ab >> 1) & 1) ^ 1, kWaitNs)) {
          ok = false;
          atomicExch(a.err, 6);
          break;
        }
        const uint32_t src = sbase + stg(sb);
        const uint32_t phi = a_plane(buf, 0), plo = a_plane(buf, 1);
        const bool leaky_max = a.in_act == kActLeaky && a.in_slope >= 0.f && a.in_slope <= 1.f;
        if ((128 % c4n) == 0 && (a.in_act == kActNone || leaky_max)) {
          // each thread keeps one 4-channel column c4 and walks rows 128/c4n apart
          const int c4 = tp % c4n, rstep = 128 / c4n;
          const int niter = total > tp ? (total - tp + 127) / 128 : 0;
          uint32_t s_addr = src + (uint32_t)tp * 16u;
          uint32_t off = (uint32_t)(c4 >> 1) * LBO_A + (uint32_t)(tp / c4n) * 16u + (uint32_t)(c4 & 1) * 8u;
          const float sl = leaky_max ? a.in_slope : 1.f;
#pragma unroll 4
          for (int i = 0; i < niter; ++i) {
            float4 v = ptx::lds128(s_addr);
            if (leaky_max) {
              v.x = fmaxf(v.x, sl * v.x);
              v.y = fmaxf(v.y, sl * v.y);
              v.z = fmaxf(v.z, sl * v.z);
              v.w = fmaxf(v.w, sl * v.w);
            }
            uint32_t h01, l01, h23, l23;
            split_pair(v.x, v.y, h01, l01);
            split_pair(v.z, v.w, h23, l23);
            ptx::sts64(phi + off, h01, h23);
            ptx::sts64(plo + off, l01, l23);
            s_addr += 2048u;
            off += (uint32_t)rstep * 16u;
          }
        } else {
#pragma unroll 4
          for (int e = tp; e < total; e += 128) {
            const int r = e / c4n, c4 = e - r * c4n;
            float4 v = ptx::lds128(src + (uint32_t)e * 16u);
            if constexpr (gen) {
              if (a.in_act) {
                v.x = act_apply(v.x, a.in_act, a.in_slope);
                v.y = act_apply(v.y, a.in_act, a.in_slope);
                v.z = act_apply(v.z, a.in_act, a.in_slope);
                v.w = act_apply(v.w, a.in_act, a.in_slope);
              }
            } else if (a.in_act) {  // leaky with slope in [0, 1] (tc_flags)
              v.x = act_apply(v.x, kActLeaky, a.in_slope);
              v.y = act_apply(v.y, kActLeaky, a.in_slope);
              v.z = act_apply(v.z, kActLeaky, a.in_slope);
              v.w = act_apply(v.w, kActLeaky, a.in_slope);
            }
            uint32_t h01, l01, h23, l23;
            split_pair(v.x, v.y, h01, l01);
            split_pair(v.z, v.w, h23, l23);
            const uint32_t off = (uint32_t)(c4 >> 1) * LBO_A + (uint32_t)r * 16u + (uint32_t)(c4 & 1) * 8u;
            ptx::sts64(phi + off, h01, h23);
            ptx::sts64(plo + off, l01, l23);
          }
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(A_FULL + 8 * buf);
        ptx::mbar_arrive(STG_EMPTY + 8 * sb);
      }
    }
  } else {
    // ------------------------------------------------ epilogue
    const int wq = warp & 3;
    const int r_in = wq * 32 + lane;  // row within a 128-row subtile
    int it = 0;
    if (g.tma_epi) {
      // Each epilogue warp runs its own pipeline over its 32 TMEM lanes: its
      // residual / accumulator boxes (32 rows x 32 columns) arrive by TMA into its
      // 4 KB part of a slot, it writes the result there in place and its lane 0
      // stores the box.  No barrier across the four warps per step.
      const bool wlead = lane == 0;
      const int nch = BN / kEpiCols;
      const int spt = g.msub * nch;
      const int ntile_cta = (g.total_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
      const int total_steps = ntile_cta * spt;
      // prefetch distance: loads for step e + pdist are issued at step e; with
      // nslot >= 3 that slot's last store is not the one just committed
      const int pdist = g.nslot >= 3 ? g.nslot - 2 : g.nslot - 1;
      const uint32_t wslot = (uint32_t)wq * kWarpSlotBytes;
      auto epi_bar = [&](int sl) { return EPI_W + 8u * (uint32_t)(sl * 4 + wq); };
      int issued = 0;
      auto issue = [&](int f) {
        if (f >= total_steps) return;
        issued = f + 1;
        const int sl = f % g.nslot;
        const TileCoord c = tile_coord(blockIdx.x + (f / spt) * gridDim.x, a.nslices, g.ntiles, g.tiles_m);
        const ConvSlice& S = a.sl[c.s];
        const int q = f % spt, sub = q / nch, ch = q % nch;
        const int row0 = c.mt * MT + sub * kTM + wq * kEpiRows, col0 = S.co_off + c.nt * BN + ch * kEpiCols;
        // this warp's previous store from the slot (step f - nslot) has finished
        // reading it; the nslot - pdist - 1 newer stores may still be in flight
        ptx::bulk_wait_read(g.nslot - pdist - 1);
        const uint32_t bytes = (t_res ? kWarpSlotBytes : 0u) + (t_acc ? kWarpSlotBytes : 0u);
        ptx::mbar_expect_tx(epi_bar(sl), bytes);
        if (g.ephase) {  // transposed-conv phase p: rows q*up + p through the 4-D view
          if (t_res)
            ptx::tma_load_4d(sbase + slot_main(sl) + wslot, &maps.res, col0, S.out_r0, row0, c.b, epi_bar(sl));
          if (t_acc)
            ptx::tma_load_4d(sbase + slot_aux(sl) + wslot, &maps.acc, col0, S.out_r0, row0, c.b, epi_bar(sl));
        } else {
          if (t_res) ptx::tma_load_3d(sbase + slot_main(sl) + wslot, &maps.res, col0, row0, c.b, epi_bar(sl));
          if (t_acc) ptx::tma_load_3d(sbase + slot_aux(sl) + wslot, &maps.acc, col0, row0, c.b, epi_bar(sl));
        }
      };
      if (g.off_bias) {  // stage the bias vector once per CTA
        for (int i = r_in; i < g.bias_n; i += 128) {
          const float bv = a.bias[i];
          asm volatile("st.shared.f32 [%0], %1;" ::"r"(sbase + g.off_bias + 4u * (uint32_t)i), "f"(bv) : "memory");
        }
        ptx::named_bar(3, 128);
      }
      if (wlead)
        for (int f = 0; f < pdist; ++f) issue(f);
      int e = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
        const TileCoord c = tile_coord(tile, a.nslices, g.ntiles, g.tiles_m);
        const ConvSlice& S = a.sl[c.s];
        const int set = it % g.nacc;
        const bool got = __all_sync(0xffffffffu, ptx::mbar_wait(ACC_FULL + 8 * set, (it / g.nacc) & 1, kWaitNs));
        if (!got) {
          if (lane == 0) atomicExch(a.err, 7);
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t dbase = tmem + (uint32_t)(set * g.msub * ACW) + ((uint32_t)(wq * 32) << 16);
        for (int q = 0; q < spt; ++q, ++e) {
          if (wlead) issue(e + pdist);
          const int sl = e % g.nslot;
          const int sub = q / nch, ch = q % nch;
          const bool in = __all_sync(0xffffffffu, ptx::mbar_wait(epi_bar(sl), (e / g.nslot) & 1, kWaitNs));
          float v[32];
          ptx::tmem_ld32(dbase + (uint32_t)(sub * ACW + ch * kEpiCols), v);
          if (STK) {  // add the Ahi.Blo half, 16 columns at a time
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float w2[16];
              ptx::tmem_ld16(dbase + (uint32_t)(sub * ACW + BN + ch * kEpiCols + 16 * h), w2);
#pragma unroll
              for (int k = 0; k < 16; ++k) v[16 * h + k] += w2[k];
            }
          }
          if (q == spt - 1) {
            ptx::tc_fence_before();
            ptx::mbar_arrive(ACC_EMPTY + 8 * set);
          }
          if (!in) {
            if (lane == 0) atomicExch(a.err, 8);
            ok = false;
            break;
          }
          const int col0 = S.co_off + c.nt * BN + ch * kEpiCols;
          const uint32_t mainp = sbase + slot_main(sl) + wslot + (uint32_t)lane * 128u;
          const uint32_t auxp = sbase + slot_aux(sl) + wslot + (uint32_t)lane * 128u;
          // each optional term is one uniform branch per 32 values
          if (t_bias) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 t = g.off_bias ? ptx::lds128(sbase + g.off_bias + (uint32_t)(col0 + 4 * j) * 4u)
                                          : __ldg(reinterpret_cast<const float4*>(a.bias + col0) + j);
              v[4 * j] += t.x; v[4 * j + 1] += t.y; v[4 * j + 2] += t.z; v[4 * j + 3] += t.w;
            }
          }
          if (t_bias2) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 t = __ldg(reinterpret_cast<const float4*>(a.bias2 + (long long)c.b * a.bias2_bs + col0) + j);
              v[4 * j] += t.x; v[4 * j + 1] += t.y; v[4 * j + 2] += t.z; v[4 * j + 3] += t.w;
            }
          }
          if (t_res) {
            if (t_sub) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float4 t = ptx::lds128(mainp + (uint32_t)((j ^ (lane & 7)) << 4));
                v[4 * j] = t.x - v[4 * j]; v[4 * j + 1] = t.y - v[4 * j + 1];
                v[4 * j + 2] = t.z - v[4 * j + 2]; v[4 * j + 3] = t.w - v[4 * j + 3];
              }
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float4 t = ptx::lds128(mainp + (uint32_t)((j ^ (lane & 7)) << 4));
                v[4 * j] += t.x; v[4 * j + 1] += t.y; v[4 * j + 2] += t.z; v[4 * j + 3] += t.w;
              }
            }
          }
          if (t_acc) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 t = ptx::lds128(auxp + (uint32_t)((j ^ (lane & 7)) << 4));
              v[4 * j] = t.x + v[4 * j]; v[4 * j + 1] = t.y + v[4 * j + 1];
              v[4 * j + 2] = t.z + v[4 * j + 2]; v[4 * j + 3] = t.w + v[4 * j + 3];
            }
          }
          if (t_div) {
            const float dv = a.out_div, rd = __frcp_rn(dv);
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = div_by(v[k], dv, rd);
          }
          act_row_t<F>(v, a);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            ptx::sts128(mainp + (uint32_t)((j ^ (lane & 7)) << 4),
                        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (wlead) {
            const int row0 = c.mt * MT + sub * kTM + wq * kEpiRows;
            if (g.ephase)
              ptx::tma_store_4d(&maps.y, col0, S.out_r0, row0, c.b, sbase + slot_main(sl) + wslot);
            else
              ptx::tma_store_3d(&maps.y, col0, row0, c.b, sbase + slot_main(sl) + wslot);
            ptx::bulk_commit();
          }
        }
        ++it;
      }
      if (wlead) {
        // no TMA load left in flight into this warp's slots, no store still reading one
        for (int f = (issued > g.nslot ? issued - g.nslot : 0); f < issued; ++f)
          ptx::mbar_wait(epi_bar(f % g.nslot), (f / g.nslot) & 1, kWaitNs);
        ptx::bulk_wait0();
      }
      __syncwarp();
    } else {
      bool ok = true;
      for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
        const TileCoord c = tile_coord(tile, a.nslices, g.ntiles, g.tiles_m);
        const ConvSlice& S = a.sl[c.s];
        const int t0 = c.mt * MT;
        if (t0 >= S.rows) continue;
        const int set = it % g.nacc;
        bool got = ptx::mbar_wait(ACC_FULL + 8 * set, (it / g.nacc) & 1, kWaitNs);
        got = __all_sync(0xffffffffu, got);
        if (!got) {
          if (lane == 0) atomicExch(a.err, 9);
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t dbase = tmem + (uint32_t)(set * g.msub * ACW) + ((uint32_t)(wq * 32) << 16);
        for (int sub = 0; sub < g.msub; ++sub) {
          const int row = t0 + sub * kTM + r_in;
          const bool valid = row < S.rows;
          const int prow = row * a.out_rs + S.out_r0;
          int col = 0;
          for (; col + 32 <= BN; col += 32) {
            float v[32];
            ptx::tmem_ld32(dbase + (uint32_t)(sub * ACW + col), v);
            if (STK) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                float w2[16];
                ptx::tmem_ld16(dbase + (uint32_t)(sub * ACW + BN + col + 16 * h), w2);
#pragma unroll
                for (int k = 0; k < 16; ++k) v[16 * h + k] += w2[k];
              }
            }
            if (valid) epi_direct<32, F>(a, c.b, prow, S.co_off + c.nt * BN + col, v, g.vec);
          }
          if (col < BN) {
            float v[16];
            ptx::tmem_ld16(dbase + (uint32_t)(sub * ACW + col), v);
            if (STK) {
              float w2[16];
              ptx::tmem_ld16(dbase + (uint32_t)(sub * ACW + BN + col), w2);
#pragma unroll
              for (int k = 0; k < 16; ++k) v[k] += w2[k];
            }
            if (valid) epi_direct<16, F>(a, c.b, prow, S.co_off + c.nt * BN + col, v, g.vec);
          }
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(ACC_EMPTY + 8 * set);
        ++it;
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, g.tmem_cols);
}

// ----------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) throw Error{kErrCuda, "cuTensorMapEncodeTiled is not available from the driver"};
  return fn;
}

// The compile-time flags of a launch (kTGeneric when its terms are not
// expressible: a pre-activation copy, a prologue activation other than
// leaky / none, an activation other than leaky / relu / gelu).
static int tc_flags(const ConvArgs& a) {
  if (a.y_raw) return kTGeneric;
  if (a.in_act != kActNone && !(a.in_act == kActLeaky && a.in_slope >= 0.f && a.in_slope <= 1.f)) return kTGeneric;
  int f = 0;
  if (a.bias) f |= kTBias;
  if (a.bias2) f |= kTBias2;
  if (a.res) f |= kTRes | (a.res_sub ? kTResSub : 0);
  if (a.accin) f |= kTAcc;
  if (a.out_div != 0.f) f |= kTDiv;
  switch (a.out_act) {
    case kActNone: break;
    case kActLeaky:
      if (!(a.out_slope >= 0.f && a.out_slope <= 1.f)) return kTGeneric;
      f |= kTLeaky;
      break;
    case kActRelu: f |= kTRelu; break;
    case kActGelu: f |= kTGelu; break;
    default: return kTGeneric;
  }
  return f;
}

template <int F>
static void tc_launch(const ConvArgs& a, const TcMaps& maps, const TcPlan& g, int grid, int dev, cudaStream_t st) {
  static std::atomic<uint64_t> attr_done{0};  // per instantiation, one bit per device
  if (dev < 64 && !(attr_done.load() & (1ull << dev))) {
    RVC_CUDA_TRY(cudaFuncSetAttribute(tc_conv_kernel<F>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    attr_done.fetch_or(1ull << dev);
  }
  tc_conv_kernel<F><<<grid, kThreads, g.smem_bytes, st>>>(a, maps, g);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

// fp32 3-D map [B][rows][width] with row stride `ld` and batch stride `bs` (elements).
static void make_map(CUtensorMap* m, const float* base, int width, int rows, int B, long long ld, long long bs,
                     int box_w, int box_r, bool swz128) {
  cuuint64_t dims[3] = {(cuuint64_t)width, (cuuint64_t)rows, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)bs * 4};
  cuuint32_t box[3] = {(cuuint32_t)box_w, (cuuint32_t)box_r, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swz128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error{kErrCuda, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")"};
}

// fp32 4-D epilogue view of a transposed conv output: element (c, p, q, b) is
// row q*up + p, channel c of batch item b.  Box: 32 channels x 1 phase x 128 q.
static void make_phase_map(CUtensorMap* m, const float* base, int width, int up, int q_rows, int B, long long ld,
                           long long bs) {
  cuuint64_t dims[4] = {(cuuint64_t)width, (cuuint64_t)up, (cuuint64_t)q_rows, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)ld * 4, (cuuint64_t)ld * 4 * up, (cuuint64_t)bs * 4};
  cuuint32_t box[4] = {(cuuint32_t)kEpiCols, 1, (cuuint32_t)kEpiRows, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)base, dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error{kErrCuda, "cuTensorMapEncodeTiled (phase view) failed (" + std::to_string((int)r) + ")"};
}

static int g_num_sms = 0;

static TcPlan tc_plan(const ConvArgs& a) {
  TcPlan g{};
  int halo = 0, maxrows = 0, minrows = 1 << 30;
  for (int s = 0; s < a.nslices; ++s) {
    int span = (a.sl[s].ntaps - 1) * a.sl[s].tap_step;
    halo = std::max(halo, span < 0 ? -span : span);
    maxrows = std::max(maxrows, a.sl[s].rows);
    minrows = std::min(minrows, a.sl[s].rows);
  }
  auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  bool v = (a.y_ld % 4 == 0) && (a.y_bs % 4 == 0) && al16(a.y) && (!a.y_raw || al16(a.y_raw));
  v = v && (!a.res || (a.res_ld % 4 == 0 && a.res_bs % 4 == 0 && al16(a.res)));
  v = v && (!a.accin || (a.acc_ld % 4 == 0 && a.acc_bs % 4 == 0 && al16(a.accin)));
  v = v && (!a.bias || al16(a.bias)) && (!a.bias2 || (a.bias2_bs % 4 == 0 && al16(a.bias2)));
  for (int s = 0; s < a.nslices; ++s) v = v && (a.sl[s].co_off % 4 == 0);
  g.vec = v ? 1 : 0;
  // TMA epilogue: plain row mapping, whole 32-column steps, every tile valid.
  // Transposed convs qualify when every phase has the same row count (output
  // length a multiple of the stride): phase p's rows q*up+p are then a box of
  // the 4-D view {channel, phase, q, batch}.
  g.tma_epi = v && a.bn % kEpiCols == 0 && !a.y_raw && minrows == maxrows &&
              (a.out_rs == 1 || a.nslices == a.out_rs);
  g.ephase = a.out_rs > 1 ? 1 : 0;
  for (int s = 0; s < a.nslices; ++s) g.tma_epi = g.tma_epi && a.sl[s].out_r0 == (a.out_rs > 1 ? s : 0);

  const uint32_t limit = 227u * 1024u;
  g.b_plane = (uint32_t)a.cb * a.bn * 2u;
  const int acc_slot = (g.tma_epi && a.accin) ? 1 : 0;
  const uint32_t slot_span = kSlotBytes * (acc_slot ? 2u : 1u);
  int width = 0, ntaps_max = 1;
  for (int s = 0; s < a.nslices; ++s) {
    width = std::max(width, a.sl[s].co_off + a.C_out);
    ntaps_max = std::max(ntaps_max, a.sl[s].ntaps);
  }
  const uint32_t bias_bytes = (g.tma_epi && a.bias && width <= 2048) ? (uint32_t)((width * 4 + 127) & ~127) : 0u;
  // Candidate pipelines, best first.  Narrow convs (bn <= 64) are HBM-bound:
  // short tiles with deep activation/epilogue pipelines keep ~100 KB in
  // flight per SM.  Wide convs are tensor-bound: tall tiles reuse each
  // weight stage, and when one K block already keeps the MMA busy for
  // thousands of cycles a single staging buffer leaves room for more
  // weight stages.
  int taps_total = 0;
  for (int s = 0; s < a.nslices; ++s) taps_total = std::max(taps_total, a.sl[s].wtap0 + a.sl[s].ntaps);
  const uint32_t w_all = (uint32_t)taps_total * a.C_in * a.C_out * 4u;  // packed hi + lo
  const bool can_res = (a.C_out == a.bn) && w_all <= 120u * 1024u;
  // Candidate pipelines, best first.  Narrow convs (bn <= 64) are HBM-bound
  // and their weights are small: keep the whole packed weight tensor resident
  // (one bulk copy per CTA, no per-stage round trips), 256-row tiles, double
  // activation staging and epilogue slots.  Wide convs are tensor-bound: tall
  // tiles reuse each streamed weight stage, and when one K block already keeps
  // the MMA busy for thousands of cycles a single staging buffer leaves room
  // for more weight stages.
  struct Cand {
    int msub, nacc, nstg, nslot, min_stages, res;
  };
  Cand cands[12];
  int ncand = 0;
  if (a.bn <= 64) {
    const Cand c[] = {{2, 2, 2, 4, 0, 1}, {2, 2, 2, 3, 0, 1}, {2, 2, 1, 3, 0, 1}, {2, 2, 1, 2, 0, 1},
                      {1, 2, 2, 3, 0, 1}, {2, 2, 2, 3, 6, 0}, {2, 2, 1, 3, 6, 0}, {2, 2, 1, 2, 4, 0},
                      {1, 2, 2, 2, 2, 0}, {1, 1, 1, 1, 2, 0}};
    for (const Cand& x : c)
      if (!x.res || can_res) cands[ncand++] = x;
  } else {
    const long long blk_clk = (long long)ntaps_max * (a.cb / 16) * 2 * 3 * (a.bn / 2);
    const int ns = blk_clk >= 6000 ? 1 : 2;
    const Cand c[] = {{4, 2, ns, 3, 4, 0}, {2, 2, ns, 3, 4, 0}, {2, 1, ns, 3, 4, 0}, {2, 2, 1, 3, 3, 0},
                      {2, 2, 1, 2, 3, 0},  {2, 1, 1, 2, 3, 0},  {2, 1, 1, 1, 3, 0}, {1, 2, 2, 2, 2, 0},
                      {1, 1, 1, 1, 2, 0}};
    for (const Cand& x : c) cands[ncand++] = x;
  }
  auto try_cand = [&](const Cand& cd, int need_stages) -> bool {
    int cols = 32;
    const int acw = tc_stacked(a.bn) ? 2 * a.bn : a.bn;
    while (cols < cd.nacc * cd.msub * acw) cols <<= 1;
    if (cols > 512) return false;
    const int arows = cd.msub * kTM + halo;
    const int pad = arows + ((1 - arows % 8) + 8) % 8;  // == 1 (mod 8): spreads chunk planes over banks
    const uint32_t a_plane = (uint32_t)a.cb * pad * 2u;
    const int nbox = (arows + 255) / 256;
    // rows per TMA box: <= 256, multiple of 8 so every box lands 128B-aligned
    const int box_rows = std::min(256, ((arows + nbox - 1) / nbox + 7) / 8 * 8);
    const uint32_t stg_bytes = (uint32_t)nbox * box_rows * a.cb * 4u;
    const int nslot = g.tma_epi ? cd.nslot : 0;
    uint32_t off = 0;
    const uint32_t off_epi = off;
    off += (uint32_t)nslot * slot_span;  // slots first: 1024-aligned for the 128B swizzle
    const uint32_t off_bias = bias_bytes ? off : 0u;
    off += bias_bytes;
    off = (off + 1023u) & ~1023u;
    const uint32_t off_a = off;
    off += 4u * a_plane;
    off = (off + 1023u) & ~1023u;
    const uint32_t off_stg = off;
    off += (uint32_t)cd.nstg * stg_bytes;
    off = (off + 127u) & ~127u;
    const uint32_t off_w = off;
    if (cd.res) off += w_all;  // resident weights replace the streaming ring
    off = (off + 127u) & ~127u;
    const uint32_t off_b = off;
    int stages = cd.res ? 1 : 8;
    const uint32_t ring = cd.res ? 0u : 2u * g.b_plane;
    auto total = [&](int st) { return 1024u + off_b + (uint32_t)st * ring + 8u * (kBarriers + 2 * st) + 16u; };
    while (stages > 2 && total(stages) > limit) --stages;
    if (total(stages) > limit || (!cd.res && stages < need_stages)) return false;
    g.w_res = cd.res;
    g.off_w = off_w;
    g.w_bytes = cd.res ? w_all : 0u;
    g.msub = cd.msub;
    g.nacc = cd.nacc;
    g.arows_pad = pad;
    g.a_plane = a_plane;
    g.tmem_cols = (uint32_t)cols;
    g.nbox = nbox;
    g.box_rows = box_rows;
    g.stg_bytes = stg_bytes;
    g.nstg = cd.nstg;
    g.nslot = nslot;
    g.acc_slot = acc_slot;
    g.off_epi = off_epi;
    g.off_bias = off_bias;
    g.bias_n = bias_bytes ? width : 0;
    g.off_a = off_a;
    g.off_stg = off_stg;
    g.off_b = off_b;
    g.stages = stages;
    g.off_bar = off_b + (uint32_t)stages * ring;
    g.smem_bytes = total(stages);
    return true;
  };
  // Best-first, except that a plan whose tiles leave SMs idle (one long
  // sequence: few row tiles) gives way to the fitting candidate with fewer
  // 128-row subtiles per tile and so more tiles; a row's K order is the same
  // for every msub.
  const int sms = g_num_sms > 0 ? g_num_sms : 148;
  auto tiles_for = [&](int msub) {
    return (long long)a.B * a.nslices * (a.C_out / a.bn) * cdiv(maxrows, msub * kTM);
  };
  int pick = -1, pick_need = 0;
  long long pick_tiles = -1;
  for (int pass = 0; pass < 2 && (pick < 0 || pick_tiles < sms); ++pass) {
    for (int i = 0; i < ncand; ++i) {
      const int need = pass == 0 ? cands[i].min_stages : 2;
      if (!try_cand(cands[i], need)) continue;
      const long long t = tiles_for(cands[i].msub);
      if (t > pick_tiles) {
        pick = i;
        pick_need = need;
        pick_tiles = t;
      }
      if (t >= sms) break;
    }
  }
  RVC_CHECK_ARG(pick >= 0, "tc_conv: tile does not fit in shared memory");
  try_cand(cands[pick], pick_need);
  g.tiles_m = cdiv(maxrows, g.msub * kTM);
  g.ntiles = a.C_out / a.bn;
  g.total_tiles = a.B * a.nslices * g.ntiles * g.tiles_m;
  return g;
}

void launch_tc_conv(const ConvArgs& a, cudaStream_t st) {
  RVC_CHECK_ARG(a.stride == 1, "tc_conv: stride must be 1 (use the strided view)");
  RVC_CHECK_ARG(a.C_in % a.cb == 0 && a.C_out % a.bn == 0 && a.cb % 16 == 0 && a.bn % 16 == 0 && a.bn <= 256,
                "tc_conv: channel tiling");
  RVC_CHECK_ARG(a.x_ld % 4 == 0 && a.x_bs % 4 == 0 && ((uintptr_t)a.x & 15) == 0,
                "tc_conv: input rows must be 16-byte aligned");
  if (g_num_sms == 0) {
    int d = 0;
    RVC_CUDA_TRY(cudaGetDevice(&d));
    RVC_CUDA_TRY(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, d));
  }
  TcPlan g = tc_plan(a);
  if (g.total_tiles == 0) return;
  TcMaps maps;
  memset(&maps, 0, sizeof(maps));
  make_map(&maps.a, a.x, a.x_ld, a.T_in, a.B, a.x_ld, a.x_bs, a.cb, g.box_rows, false);
  if (g.tma_epi) {
    int width = 0;
    for (int s = 0; s < a.nslices; ++s) width = std::max(width, a.sl[s].co_off + a.C_out);
    const int rows = a.sl[0].rows;
    if (g.ephase) {
      make_phase_map(&maps.y, a.y, width, a.out_rs, rows, a.B, a.y_ld, a.y_bs);
      if (a.res) make_phase_map(&maps.res, a.res, width, a.out_rs, rows, a.B, a.res_ld, a.res_bs);
      if (a.accin) make_phase_map(&maps.acc, a.accin, width, a.out_rs, rows, a.B, a.acc_ld, a.acc_bs);
    } else {
      make_map(&maps.y, a.y, width, rows, a.B, a.y_ld, a.y_bs, kEpiCols, kEpiRows, true);
      if (a.res) make_map(&maps.res, a.res, width, rows, a.B, a.res_ld, a.res_bs, kEpiCols, kEpiRows, true);
      if (a.accin) make_map(&maps.acc, a.accin, width, rows, a.B, a.acc_ld, a.acc_bs, kEpiCols, kEpiRows, true);
    }
  }
  int dev = 0;
  RVC_CUDA_TRY(cudaGetDevice(&dev));
  if (g_num_sms == 0) RVC_CUDA_TRY(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = std::min(g.total_tiles, g_num_sms);
  switch (tc_flags(a)) {  // the combinations the models' layers use
    case 0: tc_launch<0>(a, maps, g, grid, dev, st); break;
    case kTBias: tc_launch<kTBias>(a, maps, g, grid, dev, st); break;
    case kTBias | kTRes: tc_launch<kTBias | kTRes>(a, maps, g, grid, dev, st); break;
    case kTBias | kTGelu: tc_launch<kTBias | kTGelu>(a, maps, g, grid, dev, st); break;
    case kTGelu: tc_launch<kTGelu>(a, maps, g, grid, dev, st); break;
    case kTAcc | kTGelu: tc_launch<kTAcc | kTGelu>(a, maps, g, grid, dev, st); break;
    case kTBias | kTRelu: tc_launch<kTBias | kTRelu>(a, maps, g, grid, dev, st); break;
    case kTBias | kTBias2: tc_launch<kTBias | kTBias2>(a, maps, g, grid, dev, st); break;
    case kTBias | kTRes | kTResSub: tc_launch<kTBias | kTRes | kTResSub>(a, maps, g, grid, dev, st); break;
    case kTBias | kTLeaky: tc_launch<kTBias | kTLeaky>(a, maps, g, grid, dev, st); break;
    case kTBias | kTRes | kTAcc: tc_launch<kTBias | kTRes | kTAcc>(a, maps, g, grid, dev, st); break;
    case kTBias | kTRes | kTAcc | kTDiv: tc_launch<kTBias | kTRes | kTAcc | kTDiv>(a, maps, g, grid, dev, st); break;
    default: tc_launch<kTGeneric>(a, maps, g, grid, dev, st); break;
  }
}

}  // namespace rvc
