// Implicit-GEMM convolution kernels (see conv.cuh for the operator contract).
#include "conv.cuh"
#include "tc_ptx.cuh"

#include <algorithm>
#include <atomic>

namespace rvc {

// =====================================================================
// SIMT fp32 kernel: 64x64 output tile, 256 threads, 4x4 per thread.
// =====================================================================
__global__ void __launch_bounds__(256) simt_conv_kernel(const __grid_constant__ ConvArgs a, int nrt_max) {
  const int s = blockIdx.z;
  const ConvSlice& S = a.sl[s];
  const int b = blockIdx.x / nrt_max;
  const int rt = blockIdx.x % nrt_max;
  const int t0 = rt * 64;
  const int c0 = blockIdx.y * 64;
  if (b >= a.B || t0 >= S.rows || c0 >= a.C_out) return;
  __shared__ float As[16][65];
  __shared__ float Ws[16][64];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  const float* xb = a.x + (long long)b * a.x_bs;
  for (int j = 0; j < S.ntaps; ++j) {
    const int roff = S.tap_base + j * S.tap_step;
    const float* wj = a.w + (long long)(S.wtap0 + j) * a.C_in * a.C_out;
    for (int ci0 = 0; ci0 < a.C_in; ci0 += 16) {
      for (int e = threadIdx.x; e < 1024; e += 256) {
        const int r = e >> 4, c = e & 15;
        const int t = t0 + r, ci = ci0 + c;
        const int irow = t * a.stride + roff;
        float v = 0.f;
        if (t < S.rows && irow >= 0 && irow < a.T_in && ci < a.C_in) {
          v = xb[(long long)irow * a.x_ld + S.ci_off + ci];
          if (a.in_act) v = act_apply(v, a.in_act, a.in_slope);
        }
        As[c][r] = v;
      }
      for (int e = threadIdx.x; e < 1024; e += 256) {
        const int c = e >> 6, n = e & 63;
        const int ci = ci0 + c, co = c0 + n;
        Ws[c][n] = (ci < a.C_in && co < a.C_out) ? wj[(long long)ci * a.C_out + co] : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float av[4], wv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) av[i] = As[c][ty * 4 + i];
#pragma unroll
        for (int i = 0; i < 4; ++i) wv[i] = Ws[c][tx * 4 + i];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) acc[i][jj] = fmaf(av[i], wv[jj], acc[i][jj]);
      }
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
    if (t >= S.rows) continue;
    const int prow = t * a.out_rs + S.out_r0;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int co = c0 + tx * 4 + jj;
      if (co < a.C_out) conv_epilogue(a, b, prow, S.co_off + co, acc[i][jj]);
    }
  }
}

void launch_simt_conv(const ConvArgs& a, cudaStream_t st) {
  int nrt_max = 0;
  for (int s = 0; s < a.nslices; ++s) nrt_max = std::max(nrt_max, cdiv(a.sl[s].rows, 64));
  if (nrt_max == 0 || a.B == 0) return;
  dim3 grid(a.B * nrt_max, cdiv(a.C_out, 64), a.nslices);
  simt_conv_kernel<<<grid, 256, 0, st>>>(a, nrt_max);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

// =====================================================================
// Weight packing for the tensor path.
// Layout per (tap, n-tile, k-block): [hi plane | lo plane], each plane
// [chunk c (cb/8)][row n (bn)][8 bf16]  == the K-major no-swizzle canonical
// layout with SBO = 128 B and LBO = bn*16 B, so one bulk copy per plane lands
// an MMA-ready B tile in shared memory.
// =====================================================================
bool tc_shape_ok(int C_in, int C_out) { return C_in % 16 == 0 && C_out % 16 == 0; }

int tc_pick_bn(int C_out) {
  for (int bn = 256; bn >= 16; bn -= 16)
    if (C_out % bn == 0) return bn;
  return 16;
}

int tc_pick_cb(int C_in) {
  // 32-channel K blocks keep the activation tile small enough for 2-4
  // 128-row subtiles per weight stage (weights are re-read per tile).
  for (int cb : {32, 48, 16})
    if (C_in % cb == 0) return cb;
  return 16;
}

size_t tc_packed_elems(int taps, int C_in, int C_out, int bn, int cb) {
  (void)bn;
  (void)cb;
  return (size_t)taps * C_in * C_out * 2;
}

__global__ void tc_pack_kernel(const float* __restrict__ w, uint16_t* __restrict__ wpk, int taps, int C_in,
                               int C_out, int bn, int cb) {
  const long long total = (long long)taps * C_in * C_out;
  const int ntiles = C_out / bn, nblk = C_in / cb;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int co = (int)(i % C_out);
    const long long r = i / C_out;
    const int ci = (int)(r % C_in);
    const int tap = (int)(r / C_in);
    const int nt = co / bn, n = co % bn;
    const int kb = ci / cb, cc = ci % cb;
    const int chunk = cc >> 3, e = cc & 7;
    const long long blk = ((long long)(tap * ntiles + nt) * nblk + kb) * (2LL * cb * bn);
    const long long off = ((long long)chunk * bn + n) * 8 + e;
    __nv_bfloat16 hi, lo;
    split_bf16(w[i], hi, lo);
    wpk[blk + off] = __bfloat16_as_ushort(hi);
    wpk[blk + (long long)cb * bn + off] = __bfloat16_as_ushort(lo);
  }
}

void launch_tc_pack(const float* w, uint16_t* wpk, int taps, int C_in, int C_out, int bn, int cb,
                    cudaStream_t st) {
  long long total = (long long)taps * C_in * C_out;
  int grid = (int)std::min<long long>(cdiv<long long>(total, 256), 148 * 16);
  tc_pack_kernel<<<grid, 256, 0, st>>>(w, wpk, taps, C_in, C_out, bn, cb);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

// =====================================================================
// tcgen05 implicit-GEMM kernel, persistent.
//
// A CTA loops over tiles of msub*128 output rows x bn output channels.  Each
// weight stage (one tap x one cb-channel block, hi and lo planes) feeds msub
// MMAs, one per 128-row subtile, so weights stream through shared memory once
// per msub*128 rows.  Accumulators live in TMEM: nacc sets of msub*bn columns,
// so the epilogue of one tile overlaps the main loop of the next.
//   warp 0      weight producer (cp.async.bulk, `stages`-deep ring)
//   warp 1      TMEM owner, single-thread MMA issuer
//   warps 2..5  activation producer: fp32 rows -> bf16 hi/lo halo tile, shared
//               by every tap of the block
//   warps 6..9  epilogue: TMEM -> registers -> fused epilogue -> HBM
// =====================================================================
constexpr int kTM = 128;
constexpr int kTcThreads = 320;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per barrier wait

struct TcPlan {
  int msub, nacc, arows_pad, stages;
  uint32_t a_plane, b_plane;
  uint32_t off_a, off_b, off_bar, smem_bytes;
  uint32_t tmem_cols;
  int tiles_m, ntiles, total_tiles;
  int vec;  // epilogue may use 16-byte accesses
};

// Epilogue for N (16 or 32) consecutive output channels [cg0, cg0+N) of one
// row; all global loads of the step are issued before any is used.
template <int N>
__device__ __forceinline__ void conv_epilogue_vec(const ConvArgs& a, int b, int prow, int cg0, float (&v)[N],
                                                  int vec) {
  if (!vec) {
#pragma unroll
    for (int i = 0; i < N; ++i) conv_epilogue(a, b, prow, cg0 + i, v[i]);
    return;
  }
  constexpr int Q = N / 4;
  float4 rb[Q], ra[Q];
  if (a.res) {
    const float4* p =
        reinterpret_cast<const float4*>(a.res + (long long)b * a.res_bs + (long long)prow * a.res_ld + cg0);
#pragma unroll
    for (int q = 0; q < Q; ++q) rb[q] = p[q];
  }
  if (a.accin) {
    const float4* p =
        reinterpret_cast<const float4*>(a.accin + (long long)b * a.acc_bs + (long long)prow * a.acc_ld + cg0);
#pragma unroll
    for (int q = 0; q < Q; ++q) ra[q] = p[q];
  }
  if (a.bias) {
    const float4* p = reinterpret_cast<const float4*>(a.bias + cg0);
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      float4 t = __ldg(p + q);
      v[4 * q] += t.x; v[4 * q + 1] += t.y; v[4 * q + 2] += t.z; v[4 * q + 3] += t.w;
    }
  }
  if (a.bias2) {
    const float4* p = reinterpret_cast<const float4*>(a.bias2 + (long long)b * a.bias2_bs + cg0);
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      float4 t = __ldg(p + q);
      v[4 * q] += t.x; v[4 * q + 1] += t.y; v[4 * q + 2] += t.z; v[4 * q + 3] += t.w;
    }
  }
  if (a.res) {
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      float r[4] = {rb[q].x, rb[q].y, rb[q].z, rb[q].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) v[4 * q + e] = a.res_sub ? (r[e] - v[4 * q + e]) : (v[4 * q + e] + r[e]);
    }
  }
  if (a.accin) {
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      v[4 * q] = ra[q].x + v[4 * q]; v[4 * q + 1] = ra[q].y + v[4 * q + 1];
      v[4 * q + 2] = ra[q].z + v[4 * q + 2]; v[4 * q + 3] = ra[q].w + v[4 * q + 3];
    }
  }
  if (a.out_div != 0.f) {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = v[i] / a.out_div;
  }
  const long long o = (long long)b * a.y_bs + (long long)prow * a.y_ld + cg0;
  if (a.y_raw) {
    float4* p = reinterpret_cast<float4*>(a.y_raw + o);
#pragma unroll
    for (int q = 0; q < Q; ++q) p[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  }
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = act_apply(v[i], a.out_act, a.out_slope);
  float4* p = reinterpret_cast<float4*>(a.y + o);
#pragma unroll
  for (int q = 0; q < Q; ++q) p[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
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

__global__ void __launch_bounds__(kTcThreads, 1) tc_conv_kernel(const __grid_constant__ ConvArgs a, TcPlan g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int BN = a.bn, CB = a.cb;
  const int nblk = a.C_in / CB;
  const int MT = g.msub * kTM;
  const uint32_t LBO_A = (uint32_t)g.arows_pad * 16u;
  const uint32_t LBO_B = (uint32_t)BN * 16u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = ptx::smem_u32(smem);
  const uint32_t bar0 = sbase + g.off_bar;
  // barriers: a_full[2] a_empty[2] b_full[S] b_empty[S] acc_full[2] acc_empty[2] drain
  const uint32_t A_FULL = bar0, A_EMPTY = bar0 + 16, B_FULL = bar0 + 32, B_EMPTY = B_FULL + 8u * g.stages;
  const uint32_t ACC_FULL = B_EMPTY + 8u * g.stages, ACC_EMPTY = ACC_FULL + 16, DRAIN = ACC_EMPTY + 16;
  uint32_t* tmem_slot = (uint32_t*)(smem + g.off_bar + 8 * (9 + 2 * g.stages));
  auto a_plane = [&](int buf, int lo) { return sbase + g.off_a + (uint32_t)(2 * buf + lo) * g.a_plane; };
  auto b_plane = [&](int st, int lo) { return sbase + g.off_b + (uint32_t)(2 * st + lo) * g.b_plane; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(A_FULL + 8 * i, 128);
      ptx::mbar_init(A_EMPTY + 8 * i, 1);
      ptx::mbar_init(ACC_FULL + 8 * i, 1);
      ptx::mbar_init(ACC_EMPTY + 8 * i, 128);
    }
    for (int i = 0; i < g.stages; ++i) {
      ptx::mbar_init(B_FULL + 8 * i, 1);
      ptx::mbar_init(B_EMPTY + 8 * i, 1);
    }
    ptx::mbar_init(DRAIN, 1);
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
    if (lane == 0) {
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
            if (!ptx::mbar_wait(B_EMPTY + 8 * st, (round & 1) ^ 1, kWaitLimitNs)) {
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
      // never exit with a copy in flight
      for (int k = (ks > g.stages ? ks - g.stages : 0); k < ks; ++k)
        ptx::mbar_wait(B_FULL + 8 * (k % g.stages), (k / g.stages) & 1, kWaitLimitNs);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = ptx::idesc_bf16_f32(kTM, BN);
      int ks = 0, ab = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
        const TileCoord c = tile_coord(tile, a.nslices, g.ntiles, g.tiles_m);
        const ConvSlice& S = a.sl[c.s];
        if (c.mt * MT >= S.rows) continue;
        const int set = it % g.nacc;
        if (!ptx::mbar_wait(ACC_EMPTY + 8 * set, ((it / g.nacc) & 1) ^ 1, kWaitLimitNs)) {
          ok = false;
          atomicExch(a.err, 2);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t dbase = tmem + (uint32_t)(set * g.msub * BN);
        const int span = (S.ntaps - 1) * S.tap_step;
        const int shift = span < 0 ? -span : 0;
        bool first = true;
        for (int kb = 0; kb < nblk && ok; ++kb, ++ab) {
          const int buf = ab & 1;
          if (!ptx::mbar_wait(A_FULL + 8 * buf, (ab >> 1) & 1, kWaitLimitNs)) {
            ok = false;
            atomicExch(a.err, 3);
            break;
          }
          for (int j = 0; j < S.ntaps; ++j, ++ks) {
            const int st = ks % g.stages, round = ks / g.stages;
            if (!ptx::mbar_wait(B_FULL + 8 * st, round & 1, kWaitLimitNs)) {
              ok = false;
              atomicExch(a.err, 4);
              break;
            }
            ptx::tc_fence_after();
            const uint32_t rowoff = (uint32_t)(j * S.tap_step + shift);
            const uint32_t bhi = b_plane(st, 0), blo = b_plane(st, 1);
            for (int kk = 0; kk < CB / 16; ++kk) {
              const uint32_t ko_b = (uint32_t)(2 * kk) * LBO_B;
              const uint64_t dbh = ptx::smem_desc(bhi + ko_b, LBO_B, 128);
              const uint64_t dbl = ptx::smem_desc(blo + ko_b, LBO_B, 128);
              for (int sub = 0; sub < g.msub; ++sub) {
                const uint32_t ao = (uint32_t)(2 * kk) * LBO_A + (rowoff + (uint32_t)(sub * kTM)) * 16u;
                const uint64_t dah = ptx::smem_desc(a_plane(buf, 0) + ao, LBO_A, 128);
                const uint64_t dal = ptx::smem_desc(a_plane(buf, 1) + ao, LBO_A, 128);
                const uint32_t d = dbase + (uint32_t)(sub * BN);
                ptx::mma_bf16(d, dah, dbh, idesc, first ? 0u : 1u);
                ptx::mma_bf16(d, dah, dbl, idesc, 1u);
                ptx::mma_bf16(d, dal, dbh, idesc, 1u);
              }
              first = false;
            }
            ptx::mma_commit(B_EMPTY + 8 * st);
          }
          if (ok) ptx::mma_commit(A_EMPTY + 8 * buf);
        }
        if (ok) ptx::mma_commit(ACC_FULL + 8 * set);
        ++it;
      }
      ptx::mma_commit(DRAIN);
      ptx::mbar_wait(DRAIN, 0, kWaitLimitNs);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ------------------------------------------------ activation producer
    const int tp = threadIdx.x - 64;
    const int c4n = CB / 4;
    int ab = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
      const TileCoord c = tile_coord(tile, a.nslices, g.ntiles, g.tiles_m);
      const ConvSlice& S = a.sl[c.s];
      const int t0 = c.mt * MT;
      if (t0 >= S.rows) continue;
      const int span = (S.ntaps - 1) * S.tap_step;
      const int rmin = S.tap_base + (span < 0 ? span : 0);
      const int arows = MT + (span < 0 ? -span : span);
      const int r_start = t0 * a.stride + rmin;
      const float* xb = a.x + (long long)c.b * a.x_bs;
      for (int kb = 0; kb < nblk; ++kb, ++ab) {
        const int buf = ab & 1;
        if (!ptx::mbar_wait(A_EMPTY + 8 * buf, ((ab >> 1) & 1) ^ 1, kWaitLimitNs)) {
          ok = false;
          atomicExch(a.err, 5);
          break;
        }
        const int ci0 = S.ci_off + kb * CB;
        const uint32_t phi = a_plane(buf, 0), plo = a_plane(buf, 1);
        const int total = arows * c4n;
        // 8 independent 16-byte loads in flight per thread before any use
        for (int e0 = tp; e0 < total; e0 += 128 * 8) {
          float4 v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int e = e0 + u * 128;
            v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e < total) {
              const int r = e / c4n, c4 = e - r * c4n;
              const int irow = r_start + r;
              if (irow >= 0 && irow < a.T_in)
                v[u] = __ldg(reinterpret_cast<const float4*>(xb + (long long)irow * a.x_ld + ci0 + c4 * 4));
            }
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int e = e0 + u * 128;
            if (e >= total) break;
            const int r = e / c4n, c4 = e - r * c4n;
            float4 w4 = v[u];
            if (a.in_act) {
              w4.x = act_apply(w4.x, a.in_act, a.in_slope);
              w4.y = act_apply(w4.y, a.in_act, a.in_slope);
              w4.z = act_apply(w4.z, a.in_act, a.in_slope);
              w4.w = act_apply(w4.w, a.in_act, a.in_slope);
            }
            __nv_bfloat16 h0, h1, h2, h3, l0, l1, l2, l3;
            split_bf16(w4.x, h0, l0);
            split_bf16(w4.y, h1, l1);
            split_bf16(w4.z, h2, l2);
            split_bf16(w4.w, h3, l3);
            const uint32_t off = (uint32_t)(c4 >> 1) * LBO_A + (uint32_t)r * 16u + (uint32_t)(c4 & 1) * 8u;
            asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(phi + off), "r"(pack_bf16x2(h0, h1)),
                         "r"(pack_bf16x2(h2, h3))
                         : "memory");
            asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(plo + off), "r"(pack_bf16x2(l0, l1)),
                         "r"(pack_bf16x2(l2, l3))
                         : "memory");
          }
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(A_FULL + 8 * buf);
      }
    }
  } else {
    // ------------------------------------------------ epilogue
    const int wq = warp & 3;
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < g.total_tiles && ok; tile += gridDim.x) {
      const TileCoord c = tile_coord(tile, a.nslices, g.ntiles, g.tiles_m);
      const ConvSlice& S = a.sl[c.s];
      const int t0 = c.mt * MT;
      if (t0 >= S.rows) continue;
      const int set = it % g.nacc;
      bool got = ptx::mbar_wait(ACC_FULL + 8 * set, (it / g.nacc) & 1, kWaitLimitNs);
      got = __all_sync(0xffffffffu, got);
      if (!got) {
        if (lane == 0) atomicExch(a.err, 6);
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      const uint32_t dbase = tmem + (uint32_t)(set * g.msub * BN) + ((uint32_t)(wq * 32) << 16);
      for (int sub = 0; sub < g.msub; ++sub) {
        const int row = t0 + sub * kTM + wq * 32 + lane;
        const bool valid = row < S.rows;
        const int prow = row * a.out_rs + S.out_r0;
        int col = 0;
        for (; col + 32 <= BN; col += 32) {
          float v[32];
          ptx::tmem_ld32(dbase + (uint32_t)(sub * BN + col), v);
          if (valid) conv_epilogue_vec<32>(a, c.b, prow, S.co_off + c.nt * BN + col, v, g.vec);
        }
        if (col < BN) {
          float v[16];
          ptx::tmem_ld16(dbase + (uint32_t)(sub * BN + col), v);
          if (valid) conv_epilogue_vec<16>(a, c.b, prow, S.co_off + c.nt * BN + col, v, g.vec);
        }
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(ACC_EMPTY + 8 * set);
      ++it;
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, g.tmem_cols);
}

static int g_num_sms = 0;

static TcPlan tc_plan(const ConvArgs& a, int B) {
  TcPlan g{};
  int halo = 0;
  for (int s = 0; s < a.nslices; ++s) {
    int span = (a.sl[s].ntaps - 1) * a.sl[s].tap_step;
    halo = std::max(halo, span < 0 ? -span : span);
  }
  const uint32_t limit = 227u * 1024u;
  // Largest msub in {4,2,1} whose accumulators fit TMEM (nacc*msub*bn <= 512),
  // preferring two accumulator sets, and whose A tiles + 2 weight stages fit.
  g.b_plane = (uint32_t)a.cb * a.bn * 2u;
  for (int msub : {4, 2, 1}) {
    for (int nacc : {2, 1}) {
      int cols = 32;
      while (cols < nacc * msub * a.bn) cols <<= 1;
      if (cols > 512) continue;
      int rows = msub * kTM + halo;
      int pad = rows + ((1 - rows % 8) + 8) % 8;  // == 1 (mod 8): spreads chunk planes over banks
      uint32_t a_plane = (uint32_t)a.cb * pad * 2u;
      uint32_t fixed = 1024u + 4u * a_plane + 512u;
      if (fixed + 2u * 2u * g.b_plane > limit) continue;
      g.msub = msub;
      g.nacc = nacc;
      g.arows_pad = pad;
      g.a_plane = a_plane;
      g.tmem_cols = (uint32_t)cols;
      break;
    }
    if (g.msub) break;
  }
  RVC_CHECK_ARG(g.msub > 0, "tc_conv: tile does not fit in shared memory");
  const uint32_t fixed = 1024u + 4u * g.a_plane + 512u;
  int stages = 8;
  while (stages > 2 && fixed + (uint32_t)stages * 2u * g.b_plane > limit) --stages;
  g.stages = stages;
  g.off_a = 0;
  g.off_b = 4u * g.a_plane;
  g.off_bar = g.off_b + (uint32_t)stages * 2u * g.b_plane;
  g.smem_bytes = 1024u + g.off_bar + 8u * (12 + 2 * stages);
  int maxrows = 0;
  for (int s = 0; s < a.nslices; ++s) maxrows = std::max(maxrows, a.sl[s].rows);
  g.tiles_m = cdiv(maxrows, g.msub * kTM);
  g.ntiles = a.C_out / a.bn;
  g.total_tiles = B * a.nslices * g.ntiles * g.tiles_m;
  auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  bool v = (a.y_ld % 4 == 0) && (a.y_bs % 4 == 0) && al16(a.y) && (!a.y_raw || al16(a.y_raw));
  v = v && (!a.res || (a.res_ld % 4 == 0 && a.res_bs % 4 == 0 && al16(a.res)));
  v = v && (!a.accin || (a.acc_ld % 4 == 0 && a.acc_bs % 4 == 0 && al16(a.accin)));
  v = v && (!a.bias || al16(a.bias)) && (!a.bias2 || (a.bias2_bs % 4 == 0 && al16(a.bias2)));
  for (int s = 0; s < a.nslices; ++s) v = v && (a.sl[s].co_off % 4 == 0);
  g.vec = v ? 1 : 0;
  return g;
}

void launch_tc_conv(const ConvArgs& a, cudaStream_t st) {
  RVC_CHECK_ARG(a.stride == 1, "tc_conv: stride must be 1 (use the strided view)");
  RVC_CHECK_ARG(a.C_in % a.cb == 0 && a.C_out % a.bn == 0 && a.cb % 16 == 0 && a.bn % 16 == 0 && a.bn <= 256,
                "tc_conv: channel tiling");
  RVC_CHECK_ARG(a.x_ld % 4 == 0 && a.x_bs % 4 == 0 && ((uintptr_t)a.x & 15) == 0,
                "tc_conv: input rows must be 16-byte aligned");
  TcPlan g = tc_plan(a, a.B);
  if (g.total_tiles == 0) return;
  int dev = 0;
  RVC_CUDA_TRY(cudaGetDevice(&dev));
  // The attribute is per device: set it once for every device we launch on.
  static std::atomic<uint64_t> attr_done{0};
  if (dev < 64 && !(attr_done.load() & (1ull << dev))) {
    RVC_CUDA_TRY(cudaFuncSetAttribute(tc_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    attr_done.fetch_or(1ull << dev);
  }
  if (g_num_sms == 0) RVC_CUDA_TRY(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = std::min(g.total_tiles, g_num_sms);
  tc_conv_kernel<<<grid, kTcThreads, g.smem_bytes, st>>>(a, g);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

}  // namespace rvc
