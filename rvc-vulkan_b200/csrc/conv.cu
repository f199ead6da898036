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
  for (int cb : {64, 48, 32, 16})
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
// tcgen05 implicit-GEMM kernel.
//   M = 128 output rows (time), N = bn output channels, K = C_in x taps.
//   warp 0      : weight producer (cp.async.bulk into a `stages`-deep ring)
//   warp 1      : TMEM owner + single-thread MMA issuer
//   warps 2..5  : activation producer (fp32 -> bf16 hi/lo, halo tile reused
//                 by every tap), then the epilogue (TMEM -> registers -> HBM)
// =====================================================================
constexpr int kTM = 128;
constexpr int kTcThreads = 192;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per barrier wait

struct TcGeom {
  int arows_pad;   // allocated A rows per plane (>= 128 + halo), % 8 == 1
  int stages;
  uint32_t a_plane, b_plane;  // bytes
  uint32_t off_a, off_b, off_bar, smem_bytes;
};

__global__ void __launch_bounds__(kTcThreads) tc_conv_kernel(const __grid_constant__ ConvArgs a, TcGeom g,
                                                             int nrt_max) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int s = blockIdx.z;
  const ConvSlice& S = a.sl[s];
  const int b = blockIdx.x / nrt_max;
  const int rt = blockIdx.x % nrt_max;
  const int t0 = rt * kTM;
  if (b >= a.B || t0 >= S.rows) return;
  const int BN = a.bn, CB = a.cb;
  const int nt = blockIdx.y;
  const int n0 = nt * BN;
  const int ntiles = a.C_out / BN;
  const int nblk = a.C_in / CB;
  const int ntaps = S.ntaps;
  const int nks = nblk * ntaps;
  const int span = (ntaps - 1) * S.tap_step;
  const int rmin = S.tap_base + (span < 0 ? span : 0);
  const int arows = kTM + (span < 0 ? -span : span);
  const uint32_t LBO_A = (uint32_t)g.arows_pad * 16u;
  const uint32_t LBO_B = (uint32_t)BN * 16u;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = ptx::smem_u32(smem);
  const uint32_t bar0 = sbase + g.off_bar;
  // barrier map: a_full[2], a_empty[2], b_full[stages], b_empty[stages], acc_full, drain
  auto a_full = [&](int i) { return bar0 + 8u * i; };
  auto a_empty = [&](int i) { return bar0 + 8u * (2 + i); };
  auto b_full = [&](int i) { return bar0 + 8u * (4 + i); };
  auto b_empty = [&](int i) { return bar0 + 8u * (4 + g.stages + i); };
  const uint32_t acc_full = bar0 + 8u * (4 + 2 * g.stages);
  const uint32_t drain = acc_full + 8u;
  uint32_t* tmem_slot = (uint32_t*)(smem + g.off_bar + 8 * (6 + 2 * g.stages));
  auto a_plane = [&](int buf, int lo) { return sbase + g.off_a + (uint32_t)(2 * buf + lo) * g.a_plane; };
  auto b_plane = [&](int st, int lo) { return sbase + g.off_b + (uint32_t)(2 * st + lo) * g.b_plane; };

  uint32_t ncols = 32;
  while ((int)ncols < BN) ncols <<= 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(a_full(i), 128);
      ptx::mbar_init(a_empty(i), 1);
    }
    for (int i = 0; i < g.stages; ++i) {
      ptx::mbar_init(b_full(i), 1);
      ptx::mbar_init(b_empty(i), 1);
    }
    ptx::mbar_init(acc_full, 1);
    ptx::mbar_init(drain, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), ncols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- weight producer
    if (lane == 0) {
      const uint32_t blk_elems = 2u * CB * BN;
      int issued = 0;
      bool ok = true;
      for (int ks = 0; ks < nks && ok; ++ks) {
        const int kb = ks / ntaps, j = ks % ntaps;
        const int st = ks % g.stages, round = ks / g.stages;
        if (!ptx::mbar_wait(b_empty(st), (round & 1) ^ 1, kWaitLimitNs)) {
          ok = false;
          atomicExch(a.err, 1);
          break;
        }
        const uint16_t* src =
            a.wpk + ((size_t)((S.wtap0 + j) * ntiles + nt) * nblk + kb) * blk_elems;
        ptx::mbar_expect_tx(b_full(st), 2u * g.b_plane);
        ptx::bulk_g2s(b_plane(st, 0), src, g.b_plane, b_full(st));
        ptx::bulk_g2s(b_plane(st, 1), src + (size_t)CB * BN, g.b_plane, b_full(st));
        ++issued;
      }
      // Never leave a copy in flight behind us: wait for the last ones to land.
      for (int ks = (issued > g.stages ? issued - g.stages : 0); ks < issued; ++ks)
        ptx::mbar_wait(b_full(ks % g.stages), (ks / g.stages) & 1, kWaitLimitNs);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = ptx::idesc_bf16_f32(kTM, BN);
      bool ok = true;
      int ks = 0;
      for (int kb = 0; kb < nblk && ok; ++kb) {
        const int buf = kb & 1;
        if (!ptx::mbar_wait(a_full(buf), (kb >> 1) & 1, kWaitLimitNs)) {
          ok = false;
          atomicExch(a.err, 2);
          break;
        }
        for (int j = 0; j < ntaps; ++j, ++ks) {
          const int st = ks % g.stages, round = ks / g.stages;
          if (!ptx::mbar_wait(b_full(st), round & 1, kWaitLimitNs)) {
            ok = false;
            atomicExch(a.err, 3);
            break;
          }
          ptx::tc_fence_after();
          const int rowoff = j * S.tap_step - (span < 0 ? span : 0);
          const uint32_t ahi = a_plane(buf, 0) + (uint32_t)rowoff * 16u;
          const uint32_t alo = a_plane(buf, 1) + (uint32_t)rowoff * 16u;
          const uint32_t bhi = b_plane(st, 0), blo = b_plane(st, 1);
          for (int kk = 0; kk < CB / 16; ++kk) {
            const uint32_t ko_a = (uint32_t)(2 * kk) * LBO_A, ko_b = (uint32_t)(2 * kk) * LBO_B;
            const uint64_t dah = ptx::smem_desc(ahi + ko_a, LBO_A, 128);
            const uint64_t dal = ptx::smem_desc(alo + ko_a, LBO_A, 128);
            const uint64_t dbh = ptx::smem_desc(bhi + ko_b, LBO_B, 128);
            const uint64_t dbl = ptx::smem_desc(blo + ko_b, LBO_B, 128);
            ptx::mma_bf16(tmem, dah, dbh, idesc, (ks | kk) != 0);
            ptx::mma_bf16(tmem, dah, dbl, idesc, 1);
            ptx::mma_bf16(tmem, dal, dbh, idesc, 1);
          }
          ptx::mma_commit(b_empty(st));
        }
        if (ok) ptx::mma_commit(a_empty(buf));
      }
      if (ok) ptx::mma_commit(acc_full);
      // Drain: all issued MMAs complete before TMEM can be released.
      ptx::mma_commit(drain);
      ptx::mbar_wait(drain, 0, kWaitLimitNs);
    }
    __syncwarp();
  } else {
    // ---------------- activation producer (128 threads), then epilogue
    const int tp = threadIdx.x - 64;
    const float* xb = a.x + (long long)b * a.x_bs;
    const int c4n = CB / 4;
    const int r_start = t0 + rmin;
    bool ok = true;
    for (int kb = 0; kb < nblk && ok; ++kb) {
      const int buf = kb & 1;
      if (!ptx::mbar_wait(a_empty(buf), ((kb >> 1) & 1) ^ 1, kWaitLimitNs)) {
        ok = false;
        atomicExch(a.err, 4);
        break;
      }
      const int ci0 = S.ci_off + kb * CB;
      const uint32_t phi = a_plane(buf, 0), plo = a_plane(buf, 1);
      for (int e = tp; e < arows * c4n; e += 128) {
        const int r = e / c4n, c4 = e - r * c4n;
        const int irow = r_start + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (irow >= 0 && irow < a.T_in) {
          v = *reinterpret_cast<const float4*>(xb + (long long)irow * a.x_ld + ci0 + c4 * 4);
          if (a.in_act) {
            v.x = act_apply(v.x, a.in_act, a.in_slope);
            v.y = act_apply(v.y, a.in_act, a.in_slope);
            v.z = act_apply(v.z, a.in_act, a.in_slope);
            v.w = act_apply(v.w, a.in_act, a.in_slope);
          }
        }
        __nv_bfloat16 h0, h1, h2, h3, l0, l1, l2, l3;
        split_bf16(v.x, h0, l0);
        split_bf16(v.y, h1, l1);
        split_bf16(v.z, h2, l2);
        split_bf16(v.w, h3, l3);
        const uint32_t off = (uint32_t)(c4 >> 1) * LBO_A + (uint32_t)r * 16u + (uint32_t)(c4 & 1) * 8u;
        asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(phi + off), "r"(pack_bf16x2(h0, h1)),
                     "r"(pack_bf16x2(h2, h3))
                     : "memory");
        asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(plo + off), "r"(pack_bf16x2(l0, l1)),
                     "r"(pack_bf16x2(l2, l3))
                     : "memory");
      }
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive(a_full(buf));
    }
    // epilogue
    bool acc_ok = ok && ptx::mbar_wait(acc_full, 0, kWaitLimitNs);
    acc_ok = __all_sync(0xffffffffu, acc_ok);
    if (!acc_ok) {
      if (lane == 0) atomicExch(a.err, 5);
    } else {
      ptx::tc_fence_after();
      const int wq = warp & 3;
      const int row = t0 + wq * 32 + lane;
      const bool valid = row < S.rows;
      const int prow = row * a.out_rs + S.out_r0;
      for (int col = 0; col < BN; col += 16) {
        float v[16];
        ptx::tmem_ld16(tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)col, v);
        if (valid) {
#pragma unroll
          for (int i = 0; i < 16; ++i) conv_epilogue(a, b, prow, S.co_off + n0 + col + i, v[i]);
        }
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, ncols);
}

static TcGeom tc_geom(const ConvArgs& a) {
  TcGeom g{};
  int halo = 0;
  for (int s = 0; s < a.nslices; ++s) {
    int span = (a.sl[s].ntaps - 1) * a.sl[s].tap_step;
    halo = std::max(halo, span < 0 ? -span : span);
  }
  int rows = kTM + halo;
  g.arows_pad = rows + ((1 - rows % 8) + 8) % 8;  // == 1 (mod 8): spreads chunk planes over banks
  g.a_plane = (uint32_t)a.cb * g.arows_pad * 2u;
  g.b_plane = (uint32_t)a.cb * a.bn * 2u;
  const uint32_t limit = 227u * 1024u;
  const uint32_t fixed = 1024u + 4u * g.a_plane + 256u;
  int stages = 8;
  while (stages > 2 && fixed + (uint32_t)stages * 2u * g.b_plane > limit) --stages;
  g.stages = stages;
  g.off_a = 0;
  g.off_b = 4u * g.a_plane;
  g.off_bar = g.off_b + (uint32_t)stages * 2u * g.b_plane;
  g.smem_bytes = 1024u + g.off_bar + 8u * (8 + 2 * stages);
  return g;
}

void launch_tc_conv(const ConvArgs& a, cudaStream_t st) {
  RVC_CHECK_ARG(a.stride == 1, "tc_conv: stride must be 1 (use the strided view)");
  RVC_CHECK_ARG(a.C_in % a.cb == 0 && a.C_out % a.bn == 0 && a.cb % 16 == 0 && a.bn % 16 == 0 &&
                    a.bn <= 256,
                "tc_conv: channel tiling");
  RVC_CHECK_ARG(a.x_ld % 4 == 0 && a.x_bs % 4 == 0, "tc_conv: input rows must be 16-byte aligned");
  TcGeom g = tc_geom(a);
  RVC_CHECK_ARG(g.smem_bytes <= 227u * 1024u, "tc_conv: tile does not fit in shared memory");
  int nrt_max = 0;
  for (int s = 0; s < a.nslices; ++s) nrt_max = std::max(nrt_max, cdiv(a.sl[s].rows, kTM));
  if (nrt_max == 0 || a.B == 0) return;
  // The attribute is per device: set it once for every device we launch on.
  static std::atomic<uint64_t> attr_done{0};
  int dev = 0;
  RVC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && !(attr_done.load() & (1ull << dev))) {
    RVC_CUDA_TRY(cudaFuncSetAttribute(tc_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      227 * 1024));
    attr_done.fetch_or(1ull << dev);
  }
  dim3 grid(a.B * nrt_max, a.C_out / a.bn, a.nslices);
  tc_conv_kernel<<<grid, kTcThreads, g.smem_bytes, st>>>(a, g, nrt_max);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

}  // namespace rvc
