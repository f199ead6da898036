// tcgen05 implicit-GEMM convolution with the time rows as the MMA's N
// dimension (N = 256) and the output channels as M = 128.  Operator contract
// in conv.cuh (ConvArgs); this kernel takes plain stride-1 convolutions of one
// slice (the GeneratorNSF ResBlock convs and the like).
//
// Why a second orientation: with time rows as M (tc_conv.cu) a narrow conv
// (C_out = 32..128) issues MMAs of N = C_out columns, and every tcgen05.mma
// costs the issuing thread and the pipe a fixed ~60-70 cycles however small
// its N.  Here each MMA is M = 128 x N = 256 x K = 16 (128 cycles of tensor
// work), so the fixed cost hides under the math:
//
//   mode 1 (C_out a multiple of 128): a tile is 128 output channels x 256
//     time rows; per 16-channel k step D += Wh.Xh + Wh.Xl + Wl.Xh (BF16x3).
//   mode 2 (C_out = 32 or 64): the weight operand stacks the split inside
//     each TMEM lane quarter: rows 32q + 0..15 = Wh, rows 32q + 16..31 = Wl
//     of channels 16q .. 16q + 15, so two MMAs D += A.Xh + A.Xl leave the
//     hi and lo products of one channel 16 lanes apart in the same warp; one
//     shuffle adds them (the extra Wl.Xl term is below fp32 rounding).  With
//     32 channels the upper two quarters repeat the lower two (free in the
//     MMA, which is M = 128 either way), so all four epilogue warps have
//     channels: warps 7-8 finish a tile's time rows 0-127, warps 9-10 rows
//     128-255.
//
// Warp roles (11 warps, one CTA per SM, persistent over tiles):
//   warp 0      weight producer: cp.async.bulk of one (tap, channel block)
//               stage of packed weights into a ring, or every stage once
//               (resident weights) when they fit
//   warp 1      TMEM owner (2 x 256 columns) + single-thread MMA issuer
//   warp 2      activation loader: TMA of the fp32 halo tile [rows][cb]
//               (out-of-range rows zero-filled = conv padding)
//   warps 3-6   converters: fp32 -> prologue activation -> bf16 hi/lo planes
//               (time-row-major, 16 B per row per 8 channels: the MMA's
//               K-major B operand, shifted per tap by the descriptor start)
//   warps 7-10  epilogue: TMEM lanes = output channels, columns = time rows;
//               residual / accumulator boxes in by TMA a few chunks ahead,
//               bias / residual / accumulate / divide / activation, results
//               straight from registers to global memory.
// Every mbarrier wait is bounded (2 s): on expiry the warp sets the device
// error flag and winds down; the MMA warp waits (bounded) for its MMAs before
// TMEM is freed.  No TMA multicast.
#include "conv.cuh"
#include "tc_ptx.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <atomic>
#include <mutex>

namespace rvc {

namespace {

constexpr int kNT = 256;           // time rows per tile = MMA N
constexpr int kMT = 128;           // MMA M
constexpr int kCB = 32;            // input channels per staged block
constexpr int kWarps = 11;
constexpr int kThreads = kWarps * 32;
constexpr uint64_t kWaitNs = 2000000000ull;

struct TnPlan {
  int mode, co_tiles, tiles_t, total_tiles;
  int resident;  // every weight stage in its own slot, loaded once per CTA
  int nst, st_shift, ts;  // weight stages per k block (taps), their row shift, output rows per tile
  int arows_pad, nbox, box_rows, nstg, stages, nslot;
  uint32_t x_plane, stg_bytes, w_stage;
  uint32_t off_x, off_stg, off_w, off_epi, off_bar, smem_bytes;
};

struct TnMaps {
  CUtensorMap x, res, acc;
};

__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

struct TileT {
  int b, ct, tt;
};
// Tiles ordered with the channel tiles of one time tile adjacent (its
// activation tile is fetched once from HBM, then from L2).
__device__ __forceinline__ TileT tile_of(int tile, int co_tiles, int tiles_t) {
  TileT c;
  c.ct = tile % co_tiles;
  const int r = tile / co_tiles;
  c.tt = r % tiles_t;
  c.b = r / tiles_t;
  return c;
}

// Terms of the prologue / epilogue a launch uses, as compile-time flags of
// tcn_conv_kernel.  The ResBlock convs need a handful of combinations; with
// only those terms unrolled the epilogue warps run about twice as fast as
// with every optional term behind a run-time branch (the unrolled code of the
// unused terms cost instruction fetch and branch stalls).  Any other
// combination runs the kFGeneric instantiation, which reads the terms from
// ConvArgs at run time.  Both compute the same operations in the same order.
constexpr int kFBias = 1, kFRes = 2, kFResSub = 4, kFAcc = 8, kFDiv = 16, kFOutLeaky = 32, kFOutRelu = 64,
              kFInLeaky = 128, kFGeneric = 256;

// Epilogue of N rows of this lane's output channel: v[i] = the accumulated
// sum of row r0 + i of the current chunk (r0 may differ between lanes); bias,
// then the residual and accumulator values from the chunk's TMA boxes (32 rows
// x BW channels of fp32, box column bc = this lane's channel; BW = 32 boxes
// are 128B-swizzled: row r, column c at r*128 + ((c/4) ^ (r%8))*16 + (c%4)*4;
// BW = 16 boxes are plain: r*64 + c*4), divide, activation; rows below nval
// are stored at y + i*y_ld.
template <int N, int BW, int F>
__device__ __forceinline__ void tn_finish(const ConvArgs& a, float (&v)[N], float bsum, uint32_t resp,
                                          int r0, int bc, float* y, int nval) {
  constexpr bool gen = (F & kFGeneric) != 0;
  const bool t_bias = gen ? (a.bias || a.bias2) : (F & kFBias) != 0;
  const bool t_res = gen ? a.res != nullptr : (F & kFRes) != 0;
  const bool t_sub = gen ? a.res_sub != 0 : (F & kFResSub) != 0;
  const bool t_acc = gen ? a.accin != nullptr : (F & kFAcc) != 0;
  const bool t_div = gen ? a.out_div != 0.f : (F & kFDiv) != 0;
  if (t_bias) {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] += bsum;
  }
  auto so = [&](int i) {
    const int r = r0 + i;
    return BW == 32 ? (uint32_t)(r * 128 + (((bc >> 2) ^ (r & 7)) << 4) + (bc & 3) * 4)
                    : (uint32_t)(r * 64 + bc * 4);
  };
  constexpr uint32_t kBox = 32u * BW * 4u;
  if (t_res) {
    if (t_sub) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float r;
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r) : "r"(resp + so(i)));
        v[i] = r - v[i];
      }
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float r;
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r) : "r"(resp + so(i)));
        v[i] += r;
      }
    }
  }
  if (t_acc) {
    const uint32_t accp = resp + (t_res ? kBox : 0u);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float qv;
      asm volatile("ld.shared.f32 %0, [%1];" : "=f"(qv) : "r"(accp + so(i)));
      v[i] = qv + v[i];
    }
  }
  if (t_div) {
    const float dv = a.out_div, rd = __frcp_rn(dv);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = div_by(v[i], dv, rd);
  }
  if constexpr (gen) {
    if (a.out_act == kActLeaky && a.out_slope >= 0.f && a.out_slope <= 1.f) {
      const float sl = a.out_slope;
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = fmaxf(v[i], sl * v[i]);
    } else if (a.out_act == kActRelu) {
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = fmaxf(v[i], 0.f);
    } else if (a.out_act != kActNone) {
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = act_apply(v[i], a.out_act, a.out_slope);
    }
  } else if constexpr ((F & kFOutLeaky) != 0) {
    const float sl = a.out_slope;
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = fmaxf(v[i], sl * v[i]);
  } else if constexpr ((F & kFOutRelu) != 0) {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = fmaxf(v[i], 0.f);
  }
  if (nval >= N) {
#pragma unroll
    for (int i = 0; i < N; ++i) y[(long long)i * a.y_ld] = v[i];
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (i < nval) y[(long long)i * a.y_ld] = v[i];
  }
}

template <int F>
__global__ void __launch_bounds__(kThreads, 1)
    tcn_conv_kernel(const __grid_constant__ ConvArgs a, const __grid_constant__ TnMaps maps, TnPlan g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int nblk = a.C_in / kCB;
  const ConvSlice& S = a.sl[0];
  const int arows = kNT + (g.nst - 1) * g.st_shift;
  const uint32_t LBO_X = (uint32_t)g.arows_pad * 16u;  // K-core stride of an activation plane
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = ptx::smem_u32(smem);
  const uint32_t bar0 = sbase + g.off_bar;
  // X_FULL[2] X_EMPTY[2] STG_FULL[2] STG_EMPTY[2] ACC_FULL[2] ACC_EMPTY[2] DRAIN W_FULL[st] W_EMPTY[st]
  // EPI[4 warps][nslot], then the TMEM address slot
  const uint32_t X_FULL = bar0, X_EMPTY = bar0 + 16, STG_FULL = bar0 + 32, STG_EMPTY = bar0 + 48;
  const uint32_t ACC_FULL = bar0 + 64, ACC_EMPTY = bar0 + 80, DRAIN = bar0 + 96;
  const uint32_t W_FULL = bar0 + 104, W_EMPTY = W_FULL + 8u * g.stages, EPI = W_EMPTY + 8u * g.stages;
  uint32_t* tmem_slot = (uint32_t*)(smem + g.off_bar + 104 + 16 * g.stages + 32 * g.nslot);
  auto x_plane = [&](int buf, int lo) { return sbase + g.off_x + (uint32_t)(2 * buf + lo) * g.x_plane; };
  auto w_slot = [&](int st) { return sbase + g.off_w + (uint32_t)st * g.w_stage; };
  auto stg = [&](int sb) { return sbase + g.off_stg + (uint32_t)sb * g.stg_bytes; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(X_FULL + 8 * i, 128);
      ptx::mbar_init(X_EMPTY + 8 * i, 1);
      ptx::mbar_init(STG_FULL + 8 * i, 1);
      ptx::mbar_init(STG_EMPTY + 8 * i, 128);
      ptx::mbar_init(ACC_FULL + 8 * i, 1);
      ptx::mbar_init(ACC_EMPTY + 8 * i, 128);
    }
    ptx::mbar_init(DRAIN, 1);
    for (int i = 0; i < g.stages; ++i) {
      ptx::mbar_init(W_FULL + 8 * i, 1);
      ptx::mbar_init(W_EMPTY + 8 * i, 1);
    }
    for (int i = 0; i < 4 * g.nslot; ++i) ptx::mbar_init(EPI + 8 * i, 1);
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

  if (warp == 0) {
    // ------------------------------------------------ weight producer
    if (lane == 0) {
      int ks = 0;
      bool ok = true;
      // resident weights: the first tile's pass loads every stage once
      const int tile_end = g.resident ? min(g.total_tiles, (int)blockIdx.x + 1) : g.total_tiles;
      for (int tile = blockIdx.x; tile < tile_end && ok; tile += gridDim.x) {
        const TileT c = tile_of(tile, g.co_tiles, g.tiles_t);
        for (int kb = 0; kb < nblk && ok; ++kb)
          for (int j = 0; j < g.nst; ++j, ++ks) {
            const int st = ks % g.stages, round = ks / g.stages;
            if (!ptx::mbar_wait(W_EMPTY + 8 * st, (round & 1) ^ 1, kWaitNs)) {
              ok = false;
              atomicExch(a.err, 21);
              break;
            }
            const uint8_t* src = reinterpret_cast<const uint8_t*>(a.wpk) +
                                 ((size_t)(c.ct * g.nst + j) * nblk + kb) * g.w_stage;
            ptx::mbar_expect_tx(W_FULL + 8 * st, g.w_stage);
            ptx::bulk_g2s(w_slot(st), src, g.w_stage, W_FULL + 8 * st);
          }
      }
      for (int k = (ks > g.stages ? ks - g.stages : 0); k < ks; ++k)  // no copy left in flight
        ptx::mbar_wait(W_FULL + 8 * (k % g.stages), (k / g.stages) & 1, kWaitNs);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = ptx::idesc_bf16_f32(kMT, kNT);
      const uint32_t W_PLANE = (uint32_t)kCB * kMT * 2u;  // one hi or lo weight plane (mode 1)
      int ab = 0, it = 0;
      bool ok = true;
      if (g.resident) {
        // every weight stage lands once: wait for all of them here, so the
        // tile loop below issues its MMAs without a barrier test and a
        // tcgen05 fence per tap (10-13 % of the issuing thread's cycles at
        // 32 / 64 channels, measured with per-role counters)
        for (int st = 0; st < g.stages && ok; ++st)
          if (!ptx::mbar_wait(W_FULL + 8 * st, 0, kWaitNs)) {
            ok = false;
            atomicExch(a.err, 24);
          }
        ptx::tc_fence_after();
      }
      // Resident weights: every descriptor is a per-CTA base plus multiples of
      // fixed strides (start address >> 4 in the low bits, all offsets
      // multiples of 16 B inside shared memory), so the loop below advances
      // them by additions and issues the MMAs of a tap back to back.
      const uint64_t d_x0 = ptx::smem_desc(x_plane(0, 0), LBO_X, 128);
      const uint64_t s_lo = (uint64_t)(g.x_plane >> 4), s_buf = (uint64_t)((2u * g.x_plane) >> 4);
      const uint64_t s_tap = (uint64_t)g.st_shift, s_kx = (uint64_t)((2u * LBO_X) >> 4);
      const uint64_t d_w0 = ptx::smem_desc(w_slot(0), 2048, 128), s_w = (uint64_t)(g.w_stage >> 4);
      const uint64_t s_ka = 4096u >> 4, s_wl = W_PLANE >> 4;
      for (int tile = blockIdx.x; tile < g.total_tiles && ok && g.resident; tile += gridDim.x) {
        const int set = it & 1;
        if (!ptx::mbar_wait(ACC_EMPTY + 8 * set, ((it >> 1) & 1) ^ 1, kWaitNs)) {
          ok = false;
          atomicExch(a.err, 22);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t dtm = tmem + (uint32_t)(set * kNT);
        uint64_t aw = d_w0;  // stage kb * nst + j
        for (int kb = 0; kb < nblk; ++kb, ++ab) {
          const int buf = ab & 1;
          if (!ptx::mbar_wait(X_FULL + 8 * buf, (ab >> 1) & 1, kWaitNs)) {
            ok = false;
            atomicExch(a.err, 23);
            break;
          }
          ptx::tc_fence_after();
          uint64_t bh = d_x0 + (uint64_t)buf * s_buf;
          if (g.mode == 1) {
            for (int j = 0; j < g.nst; ++j, bh += s_tap, aw += s_w) {
              ptx::mma_bf16(dtm, aw, bh, idesc, (kb | j) ? 1u : 0u);
              ptx::mma_bf16(dtm, aw, bh + s_lo, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_wl, bh, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_ka, bh + s_kx, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_ka, bh + s_lo + s_kx, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_wl + s_ka, bh + s_kx, idesc, 1u);
            }
          } else {
            for (int j = 0; j < g.nst; ++j, bh += s_tap, aw += s_w) {
              ptx::mma_bf16(dtm, aw, bh, idesc, (kb | j) ? 1u : 0u);
              ptx::mma_bf16(dtm, aw, bh + s_lo, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_ka, bh + s_kx, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_ka, bh + s_lo + s_kx, idesc, 1u);
            }
          }
          ptx::mma_commit(X_EMPTY + 8 * buf);
        }
        if (ok) ptx::mma_commit(ACC_FULL + 8 * set);
        ++it;
      }
      // Streamed weights: the ring stage st and its phase round are counted
      // per tap (the producer fills the stages in the same order); the
      // descriptors advance by additions as above.
      int st = 0, round = 0;
      uint64_t aw = d_w0;  // descriptor of stage st
      for (int tile = blockIdx.x; tile < g.total_tiles && ok && !g.resident; tile += gridDim.x) {
        const int set = it & 1;
        if (!ptx::mbar_wait(ACC_EMPTY + 8 * set, ((it >> 1) & 1) ^ 1, kWaitNs)) {
          ok = false;
          atomicExch(a.err, 22);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t dtm = tmem + (uint32_t)(set * kNT);
        for (int kb = 0; kb < nblk && ok; ++kb, ++ab) {
          const int buf = ab & 1;
          if (!ptx::mbar_wait(X_FULL + 8 * buf, (ab >> 1) & 1, kWaitNs)) {
            ok = false;
            atomicExch(a.err, 23);
            break;
          }
          ptx::tc_fence_after();
          uint64_t bh = d_x0 + (uint64_t)buf * s_buf;
          for (int j = 0; j < g.nst; ++j, bh += s_tap) {
            if (!ptx::mbar_wait(W_FULL + 8 * st, round & 1, kWaitNs)) {
              ok = false;
              atomicExch(a.err, 24);
              break;
            }
            ptx::tc_fence_after();
            const uint32_t acc0 = (kb | j) ? 1u : 0u;
            if (g.mode == 1) {
              ptx::mma_bf16(dtm, aw, bh, idesc, acc0);
              ptx::mma_bf16(dtm, aw, bh + s_lo, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_wl, bh, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_ka, bh + s_kx, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_ka, bh + s_lo + s_kx, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_wl + s_ka, bh + s_kx, idesc, 1u);
            } else {
              ptx::mma_bf16(dtm, aw, bh, idesc, acc0);
              ptx::mma_bf16(dtm, aw, bh + s_lo, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_ka, bh + s_kx, idesc, 1u);
              ptx::mma_bf16(dtm, aw + s_ka, bh + s_lo + s_kx, idesc, 1u);
            }
            ptx::mma_commit(W_EMPTY + 8 * st);
            if (++st == g.stages) {
              st = 0;
              ++round;
              aw = d_w0;
            } else {
              aw += s_w;
            }
          }
          if (ok) ptx::mma_commit(X_EMPTY + 8 * buf);
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
      const uint32_t bytes = (uint32_t)g.nbox * g.box_rows * kCB * 4u;
      int ab = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
        const TileT c = tile_of(tile, g.co_tiles, g.tiles_t);
        const int r_start = c.tt * g.ts + S.tap_base;
        for (int kb = 0; kb < nblk; ++kb, ++ab) {
          const int sb = ab % g.nstg;
          if (!ptx::mbar_wait(STG_EMPTY + 8 * sb, ((ab / g.nstg) & 1) ^ 1, kWaitNs)) {
            ok = false;
            atomicExch(a.err, 25);
            break;
          }
          ptx::mbar_expect_tx(STG_FULL + 8 * sb, bytes);
          for (int i = 0; i < g.nbox; ++i)
            ptx::tma_load_3d(stg(sb) + (uint32_t)i * g.box_rows * kCB * 4u, &maps.x, S.ci_off + kb * kCB,
                             r_start + i * g.box_rows, c.b, STG_FULL + 8 * sb);
        }
      }
      for (int k = (ab > g.nstg ? ab - g.nstg : 0); k < ab; ++k)  // no copy left in flight
        ptx::mbar_wait(STG_FULL + 8 * (k % g.nstg), (k / g.nstg) & 1, kWaitNs);
    }
  } else if (warp < 7) {
    // ------------------------------------------------ converters
    const int tp = threadIdx.x - 96;
    constexpr int c4n = kCB / 4;  // 8 four-channel columns
    const int total = arows * c4n;
    const bool leaky_max = a.in_act == kActLeaky && a.in_slope >= 0.f && a.in_slope <= 1.f;
    const bool plain = a.in_act == kActNone || leaky_max;
    const float sl = leaky_max ? a.in_slope : 1.f;
    constexpr bool gen = (F & kFGeneric) != 0;
    int ab = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < nblk; ++kb, ++ab) {
        const int sb = ab % g.nstg, buf = ab & 1;
        if (!ptx::mbar_wait(STG_FULL + 8 * sb, (ab / g.nstg) & 1, kWaitNs) ||
            !ptx::mbar_wait(X_EMPTY + 8 * buf, ((ab >> 1) & 1) ^ 1, kWaitNs)) {
          ok = false;
          atomicExch(a.err, 26);
          break;
        }
        const uint32_t src = stg(sb);
        const uint32_t phi = x_plane(buf, 0), plo = x_plane(buf, 1);
        // one thread keeps one 4-channel column c4 and walks rows 16 apart
        const int c4 = tp % c4n, r0 = tp / c4n;
        const int niter = total > tp ? (total - tp + 127) / 128 : 0;
        uint32_t s_addr = src + (uint32_t)tp * 16u;
        uint32_t off = (uint32_t)(c4 >> 1) * LBO_X + (uint32_t)r0 * 16u + (uint32_t)(c4 & 1) * 8u;
#pragma unroll 4
        for (int i = 0; i < niter; ++i) {
          float4 v = ptx::lds128(s_addr);
          if constexpr (gen) {
            if (plain) {
              v.x = fmaxf(v.x, sl * v.x);
              v.y = fmaxf(v.y, sl * v.y);
              v.z = fmaxf(v.z, sl * v.z);
              v.w = fmaxf(v.w, sl * v.w);
            } else {
              v.x = act_apply(v.x, a.in_act, a.in_slope);
              v.y = act_apply(v.y, a.in_act, a.in_slope);
              v.z = act_apply(v.z, a.in_act, a.in_slope);
              v.w = act_apply(v.w, a.in_act, a.in_slope);
            }
          } else if constexpr ((F & kFInLeaky) != 0) {
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
          off += 16u * 16u;
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(X_FULL + 8 * buf);
        ptx::mbar_arrive(STG_EMPTY + 8 * sb);
      }
    }
  } else {
    // ------------------------------------------------ epilogue
    // TMEM lanes = output channels, columns = time rows.  A warp's step
    // finishes one 32-row chunk of its lane quarter: mode 1 32 channels x 32
    // rows; mode 2 16 channels, lanes 0-15 rows 0-15 and lanes 16-31 rows
    // 16-31 after one shuffle swaps the halves' partial sums.  The chunk's
    // residual / accumulator boxes (32 rows x 32 channels, mode 2: x 16) are
    // loaded by the warp itself with TMA, a few chunks ahead, into its slots.
    const int wq = warp & 3;
    const bool m2 = g.mode == 2;
    // mode 2 with 32 channels: quarters 2-3 hold copies of quarters 0-1, so
    // warps 7-8 finish chunks 0-3 and warps 9-10 chunks 4-7 of every tile
    const bool split = m2 && a.C_out == 32;
    const int nch = split ? 4 : 8;            // chunks of a tile this warp finishes
    const int c0 = split ? (wq >> 1) * 4 : 0;  // its first chunk
    const int bw = m2 ? 16 : 32;             // box width (channels)
    auto col_of = [&](int ct) { return S.co_off + (m2 ? (split ? (wq & 1) : wq) * 16 : ct * kMT + wq * 32); };
    const int ntile_cta = (g.total_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const int total_steps = ntile_cta * nch;  // one step per chunk
    const bool has_in = a.res || a.accin;
    const uint32_t box_bytes = 32u * (uint32_t)bw * 4u;
    const uint32_t slot_bytes = box_bytes * ((a.res ? 1u : 0u) + (a.accin ? 1u : 0u));
    // input slots exist for the warps that hold channels (wq < 2 for 32 channels)
    auto slot_res = [&](int sl) { return sbase + g.off_epi + (uint32_t)(wq * g.nslot + sl) * slot_bytes; };
    auto epi_bar = [&](int sl) { return EPI + 8u * (uint32_t)(wq * g.nslot + sl); };
    const bool loader = lane == 0;  // issues this warp's input boxes
    const int pdist = g.nslot - 1;  // input boxes are loaded this many chunks ahead
    const int bc = m2 ? (lane & 15) : lane;  // this lane's column of the boxes
    float bias_r0 = 0.f, bias_r1 = 0.f;      // this lane's channel: constant but for the channel tile
    if (a.bias) {
      bias_r0 = __ldg(a.bias + col_of(0) + bc);
      if (g.co_tiles > 1) bias_r1 = __ldg(a.bias + col_of(1) + bc);
    }
    int issued = 0;
    auto issue = [&](int f) {  // input boxes of chunk step f (lane 0)
      if (!has_in || f >= total_steps) return;
      const int sl = f % g.nslot;
      const TileT c = tile_of(blockIdx.x + (f / nch) * gridDim.x, g.co_tiles, g.tiles_t);
      const int row0 = c.tt * g.ts + 32 * (c0 + f % nch), col0 = col_of(c.ct);
      issued = f + 1;
      // the slot was last read (generic proxy) at step f - nslot, finished by now
      ptx::fence_proxy_async_smem();
      ptx::mbar_expect_tx(epi_bar(sl), slot_bytes);
      uint32_t dst = slot_res(sl);
      if (a.res) {
        ptx::tma_load_3d(dst, &maps.res, col0, row0, c.b, epi_bar(sl));
        dst += box_bytes;
      }
      if (a.accin) ptx::tma_load_3d(dst, &maps.acc, col0, row0, c.b, epi_bar(sl));
    };
    if (loader)
      for (int f = 0; f < pdist; ++f) issue(f);
    int e = 0;  // this warp's next step
    bool ok = true;
    int it = 0;
    for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
      const TileT c = tile_of(tile, g.co_tiles, g.tiles_t);
      const int set = it & 1;
      if (!__all_sync(0xffffffffu, ptx::mbar_wait(ACC_FULL + 8 * set, (it >> 1) & 1, kWaitNs))) {
        if (lane == 0) atomicExch(a.err, 27);
        break;
      }
      ptx::tc_fence_after();
      const uint32_t dt = tmem + (uint32_t)(set * kNT) + ((uint32_t)(wq * 32) << 16);
      const int t_tile = c.tt * g.ts, t_end = min(S.rows, t_tile + g.ts);
      const int co = col_of(c.ct) + bc;
      const float br = (c.ct & 1) ? bias_r1 : bias_r0;
      const float bsum = a.bias2 ? br + __ldg(a.bias2 + (long long)c.b * a.bias2_bs + co) : br;
      float* ybase = a.y + (long long)c.b * a.y_bs + co;
      // chunk ch's results: the TMEM load of the next chunk is already in flight
      auto process = [&](int ch, const uint32_t (&r)[32]) {
        if (!ok) return;
        if (loader) issue(e + pdist);
        if (has_in) {
          const int sl = e % g.nslot;
          if (!__all_sync(0xffffffffu, ptx::mbar_wait(epi_bar(sl), (e / g.nslot) & 1, kWaitNs))) {
            if (lane == 0) atomicExch(a.err, 28);
            ok = false;
            return;
          }
        }
        const uint32_t resp = slot_res(e % g.nslot);
        if (!m2) {
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          const int row0 = t_tile + 32 * ch;
          tn_finish<32, 32, F>(a, v, bsum, resp, 0, bc, ybase + (long long)row0 * a.y_ld, min(32, t_end - row0));
        } else {
          // lane l < 16: hi part of channel l, rows 0-31; lane l + 16: its lo
          // part.  Lane l finishes rows 0-15 and lane l + 16 rows 16-31, each
          // as (hi part) + (lo part).
          const bool hi = lane < 16;
          float w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float a0 = __uint_as_float(r[i]), a1 = __uint_as_float(r[16 + i]);
            const float recv = __shfl_xor_sync(0xffffffffu, hi ? a1 : a0, 16);
            w[i] = hi ? a0 + recv : recv + a1;
          }
          const int r0 = hi ? 0 : 16;
          const int row0 = t_tile + 32 * ch + r0;
          tn_finish<16, 16, F>(a, w, bsum, resp, r0, bc, ybase + (long long)row0 * a.y_ld, min(16, t_end - row0));
        }
      };
      uint32_t ra[32], rb[32];
      const int c_end = c0 + nch;
      ptx::tmem_ld32_async(dt + (uint32_t)(c0 * 32), ra);
      ptx::tmem_wait_ld(ra);
#pragma unroll 1
      for (int ch = c0; ch < c_end; ch += 2) {
        ptx::tmem_ld32_async(dt + (uint32_t)((ch + 1) * 32), rb);
        process(ch, ra);
        ++e;
        ptx::tmem_wait_ld(rb);
        if (ch + 2 < c_end) {
          ptx::tmem_ld32_async(dt + (uint32_t)((ch + 2) * 32), ra);
        } else {  // every column of this accumulator set is in registers
          ptx::tc_fence_before();
          ptx::mbar_arrive(ACC_EMPTY + 8 * set);
        }
        process(ch + 1, rb);
        ++e;
        if (ch + 2 < c_end) ptx::tmem_wait_ld(ra);
      }
      ++it;
    }
    if (loader) {
      // no TMA load left in flight into this warp's slots
      for (int f = (issued > g.nslot ? issued - g.nslot : 0); f < issued; ++f)
        ptx::mbar_wait(epi_bar(f % g.nslot), (f / g.nslot) & 1, kWaitNs);
    }
    __syncwarp();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, 512);
}

// Packs fp32 weights [taps][C_in][C_out] into the M-major operand stages of
// this kernel: stage (ct, tap, kb) holds, for mode 1, a hi and a lo plane of
// [kstep (cb/16)][K-core 2][row 128][8 ch] bf16 (row m = channel ct*128 + m);
// for mode 2 one plane whose row 32q + j is the hi (j < 16) or lo (j >= 16)
// part of channel 16q + j % 16 (zero for channels >= C_out).
// hi = RN(w), lo = RN(w - hi).
__global__ void tcn_pack_kernel(const float* __restrict__ w, uint16_t* __restrict__ out, int taps, int C_in,
                                int C_out, int mode, long long total) {
  const int nblk = C_in / kCB;
  const int nhl = mode == 1 ? 2 : 1;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    long long r = i;
    const int e = (int)(r % 8); r /= 8;
    const int m = (int)(r % kMT); r /= kMT;
    const int core = (int)(r % 2); r /= 2;
    const int s = (int)(r % (kCB / 16)); r /= (kCB / 16);
    const int hl = (int)(r % nhl); r /= nhl;
    const int kb = (int)(r % nblk); r /= nblk;
    const int tap = (int)(r % taps); r /= taps;
    const int ct = (int)r;
    const int ci = kb * kCB + s * 16 + core * 8 + e;
    int co;
    bool lo;
    if (mode == 1) {
      co = ct * kMT + m;
      lo = hl == 1;
    } else {
      // 32 channels: lane quarters 2-3 repeat quarters 0-1 (the epilogue then
      // splits each tile's columns over all four warps)
      co = (C_out == 32 ? ((m >> 5) & 1) : (m >> 5)) * 16 + (m & 15);
      lo = (m & 16) != 0;
    }
    const float x = co < C_out ? w[((long long)tap * C_in + ci) * C_out + co] : 0.f;
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    const __nv_bfloat16 v = lo ? __float2bfloat16_rn(x - __bfloat162float(h)) : h;
    out[i] = *reinterpret_cast<const uint16_t*>(&v);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 tn_encode_fn() {
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

int tn_mode(int C_out) { return (C_out == 32 || C_out == 64) ? 2 : (C_out % kMT == 0 ? 1 : 0); }

bool tn_plan(const ConvArgs& a, int sms, TnPlan* out) {
  TnPlan g{};
  const ConvSlice& S = a.sl[0];
  g.mode = tn_mode(a.C_out);
  g.nst = S.ntaps;
  g.st_shift = S.tap_step;
  g.ts = kNT;
  g.co_tiles = g.mode == 1 ? a.C_out / kMT : 1;
  g.tiles_t = cdiv(S.rows, g.ts);
  g.total_tiles = a.B * g.tiles_t * g.co_tiles;
  const int arows = kNT + (g.nst - 1) * g.st_shift;
  g.arows_pad = arows + ((1 - arows % 8) + 8) % 8;  // == 1 (mod 8): spreads the planes over banks
  g.x_plane = (uint32_t)kCB * g.arows_pad * 2u;
  g.nbox = (arows + 255) / 256;
  g.box_rows = std::min(256, ((arows + g.nbox - 1) / g.nbox + 7) / 8 * 8);
  g.stg_bytes = (uint32_t)g.nbox * g.box_rows * kCB * 4u;
  g.w_stage = (uint32_t)(g.mode == 1 ? 2 : 1) * kCB * kMT * 2u;
  const uint32_t limit = 227u * 1024u;
  const uint32_t slot_bytes = (g.mode == 1 ? 4096u : 2048u) * ((a.res ? 1u : 0u) + (a.accin ? 1u : 0u));
  const uint32_t nact = 4u;  // epilogue warps with input slots
  // Preference: resident weights (a CTA reads its weights from L2 once
  // instead of once per tile; streaming them was the MMA warp's main wait)
  // with deep residual / accumulator prefetch in the epilogue (its box waits
  // were the next cost), then a ring of weight stages, then shallower
  // prefetch; two activation staging buffers where they fit.
  struct Cand {
    int resident, nslot, nstg, min_stages;
  };
  const Cand cands[] = {{1, 8, 2, 0}, {1, 8, 1, 0}, {1, 6, 1, 0}, {1, 4, 2, 0}, {1, 4, 1, 0},
                        {0, 8, 1, 4}, {0, 6, 1, 4}, {0, 4, 2, 4}, {0, 4, 1, 4}, {1, 3, 1, 0},
                        {1, 2, 1, 0}, {0, 3, 1, 4}, {0, 3, 1, 3}, {0, 2, 1, 3}, {0, 2, 1, 2}};
  const int all_stages = g.nst * (a.C_in / kCB);  // one channel tile's stages (resident: co_tiles == 1)
  for (Cand cd : cands) {
    if (cd.resident && g.co_tiles != 1) continue;
    if (slot_bytes == 0) {  // no input boxes: the slot count only sizes the barriers
      if (cd.nslot > 4) continue;
      cd.nslot = 1;
    }
    uint32_t off = 0;
    const uint32_t off_epi = off;  // 1024-aligned: 128B-swizzled boxes
    off += nact * (uint32_t)cd.nslot * slot_bytes;
    off = (off + 1023u) & ~1023u;
    const uint32_t off_x = off;
    off += 4u * g.x_plane;
    off = (off + 1023u) & ~1023u;
    const uint32_t off_stg = off;
    off += (uint32_t)cd.nstg * g.stg_bytes;
    off = (off + 127u) & ~127u;
    const uint32_t off_w = off;
    auto total = [&](int st) {
      return 1024u + off_w + (uint32_t)st * g.w_stage + 104u + 16u * st + 32u * cd.nslot + 16u;
    };
    int stages = cd.resident ? all_stages : 8;
    if (!cd.resident)
      while (stages > cd.min_stages && total(stages) > limit) --stages;
    if (total(stages) > limit) continue;
    g.resident = cd.resident;
    g.nslot = cd.nslot;
    g.nstg = cd.nstg;
    g.stages = stages;
    g.off_epi = off_epi;
    g.off_x = off_x;
    g.off_stg = off_stg;
    g.off_w = off_w;
    g.off_bar = off_w + (uint32_t)stages * g.w_stage;
    g.smem_bytes = total(stages);
    *out = g;
    (void)sms;
    return true;
  }
  return false;
}

}  // namespace

int tcn_enabled() {
  static const int mode = [] {
    const char* e = getenv("RVC_CUDA_TCN");
    if (e && e[0] == '0') return 0;
    if (e && e[0] == '2') return 2;
    return 1;
  }();
  return mode;
}

bool tcn_shape_ok(const ConvArgs& a) {
  if (a.nslices != 1 || a.stride != 1 || a.out_rs != 1 || a.y_raw) return false;
  const ConvSlice& S = a.sl[0];
  if (S.tap_step < 1 || S.ntaps < 1 || S.out_r0 != 0 || S.rows < 1) return false;
  if (a.C_in % kCB != 0 || tn_mode(a.C_out) == 0) return false;
  if ((S.ntaps - 1) * S.tap_step > 512) return false;
  // TMA epilogue boxes: 16-byte aligned rows and bases
  auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (a.y_ld % 4 || a.y_bs % 4 || !al16(a.y) || S.co_off % 4) return false;
  if (a.res && (a.res_ld % 4 || a.res_bs % 4 || !al16(a.res))) return false;
  if (a.accin && (a.acc_ld % 4 || a.acc_bs % 4 || !al16(a.accin))) return false;
  return true;
}

bool tcn_fits(const ConvArgs& a) {
  TnPlan g;
  return tcn_shape_ok(a) && tn_plan(a, 148, &g);
}

size_t tcn_packed_elems(int taps, int C_in, int C_out) {
  const int mode = tn_mode(C_out);
  const int co_tiles = mode == 1 ? C_out / kMT : 1;
  return (size_t)co_tiles * taps * (C_in / kCB) * (mode == 1 ? 2 : 1) * kCB * kMT;
}

void launch_tcn_pack(const float* w, uint16_t* out, int taps, int C_in, int C_out, cudaStream_t st) {
  RVC_CHECK_ARG(C_in % kCB == 0 && tn_mode(C_out) != 0, "tcn_pack: channel counts");
  const long long total = (long long)tcn_packed_elems(taps, C_in, C_out);
  const int grid = (int)std::min<long long>(cdiv<long long>(total, 256), 148 * 16);
  tcn_pack_kernel<<<grid, 256, 0, st>>>(w, out, taps, C_in, C_out, tn_mode(C_out), total);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

namespace {

// The compile-time flags of a launch (kFGeneric when its terms are not one
// of the instantiated combinations).
int tn_flags(const ConvArgs& a) {
  int f = 0;
  if (a.bias || a.bias2) f |= kFBias;
  if (a.res) f |= kFRes | (a.res_sub ? kFResSub : 0);
  if (a.accin) f |= kFAcc;
  if (a.out_div != 0.f) f |= kFDiv;
  if (a.out_act == kActLeaky && a.out_slope >= 0.f && a.out_slope <= 1.f) f |= kFOutLeaky;
  else if (a.out_act == kActRelu) f |= kFOutRelu;
  else if (a.out_act != kActNone) return kFGeneric;
  if (a.in_act == kActLeaky && a.in_slope >= 0.f && a.in_slope <= 1.f) f |= kFInLeaky;
  else if (a.in_act != kActNone) return kFGeneric;
  return f;
}

template <int F>
void tn_launch(const ConvArgs& a, const TnMaps& maps, const TnPlan& g, int grid, int dev, cudaStream_t st) {
  static std::atomic<uint64_t> attr_done{0};  // per instantiation, one bit per device
  if (dev < 64 && !(attr_done.load() & (1ull << dev))) {
    RVC_CUDA_TRY(cudaFuncSetAttribute(tcn_conv_kernel<F>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    attr_done.fetch_or(1ull << dev);
  }
  tcn_conv_kernel<F><<<grid, kThreads, g.smem_bytes, st>>>(a, maps, g);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

}  // namespace

void launch_tcn_conv(const ConvArgs& a, cudaStream_t st) {
  RVC_CHECK_ARG(tcn_shape_ok(a), "tcn_conv: unsupported conv shape");
  RVC_CHECK_ARG(a.x_ld % 4 == 0 && a.x_bs % 4 == 0 && ((uintptr_t)a.x & 15) == 0 && ((uintptr_t)a.wpk & 15) == 0,
                "tcn_conv: input rows and packed weights must be 16-byte aligned");
  int dev = 0;
  RVC_CUDA_TRY(cudaGetDevice(&dev));
  int sms = 0;
  RVC_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  TnPlan g;
  RVC_CHECK_ARG(tn_plan(a, sms, &g), "tcn_conv: tile does not fit in shared memory");
  if (g.total_tiles == 0) return;
  TnMaps maps;
  memset(&maps, 0, sizeof(maps));
  auto encode = [](CUtensorMap* m, const float* base, long long width, long long rows, int B, long long ld,
                   long long bs, int box_w, int box_r, bool swz) {
    cuuint64_t dims[3] = {(cuuint64_t)width, (cuuint64_t)rows, (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)bs * 4};
    cuuint32_t box[3] = {(cuuint32_t)box_w, (cuuint32_t)box_r, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = tn_encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box, es,
                                CU_TENSOR_MAP_INTERLEAVE_NONE,
                                swz ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error{kErrCuda, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")"};
  };
  encode(&maps.x, a.x, a.x_ld, a.T_in, a.B, a.x_ld, a.x_bs, kCB, g.box_rows, false);
  const int width = a.sl[0].co_off + a.C_out, rows = a.sl[0].rows;
  const int bw = g.mode == 1 ? 32 : 16;  // epilogue box: 32 rows x bw channels (32: 128B-swizzled)
  if (a.res) encode(&maps.res, a.res, width, rows, a.B, a.res_ld, a.res_bs, bw, 32, bw == 32);
  if (a.accin) encode(&maps.acc, a.accin, width, rows, a.B, a.acc_ld, a.acc_bs, bw, 32, bw == 32);
  const int grid = std::min(g.total_tiles, sms);
  switch (tn_flags(a)) {
    case kFBias: tn_launch<kFBias>(a, maps, g, grid, dev, st); break;
    case kFBias | kFInLeaky | kFOutLeaky: tn_launch<kFBias | kFInLeaky | kFOutLeaky>(a, maps, g, grid, dev, st); break;
    case kFBias | kFRes: tn_launch<kFBias | kFRes>(a, maps, g, grid, dev, st); break;
    case kFBias | kFRes | kFAcc: tn_launch<kFBias | kFRes | kFAcc>(a, maps, g, grid, dev, st); break;
    case kFBias | kFRes | kFAcc | kFDiv: tn_launch<kFBias | kFRes | kFAcc | kFDiv>(a, maps, g, grid, dev, st); break;
    default: tn_launch<kFGeneric>(a, maps, g, grid, dev, st); break;
  }
}

}  // namespace rvc
