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
// Layout per (tap, n-tile, k-block), 2*cb*bn bf16:
//  * bn > 64: [hi plane | lo plane], each plane [chunk c (cb/8)][row n (bn)][8 bf16]
//    == the K-major no-swizzle canonical layout with SBO = 128 B, LBO = bn*16 B;
//  * bn <= 64 (stacked): [chunk c][row: hi rows 0..bn-1, lo rows bn..2bn-1][8 bf16]
//    with LBO = 2*bn*16 B, so [B_hi | B_lo] is one N = 2*bn operand and B_hi alone
//    the first bn rows of it.
// One bulk copy per block lands an MMA-ready B tile in shared memory.
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

// Offsets of element (tap, ci, co)'s hi and lo halves in the packed layout for
// column tiles of bn and K blocks of cb: blocks (tap, column tile, K block) of
// 2 cb bn values; inside, 8-channel chunks of bn columns x 8, hi and lo either
// stacked per chunk (bn <= 64) or as two planes.
__device__ __forceinline__ void tc_pack_offsets(int tap, int ci, int co, int C_in, int C_out, int bn, int cb,
                                                long long& hi, long long& lo) {
  const int ntiles = C_out / bn, nblk = C_in / cb;
  const int nt = co / bn, n = co % bn;
  const int kb = ci / cb, cc = ci % cb;
  const int chunk = cc >> 3, e = cc & 7;
  const long long blk = ((long long)(tap * ntiles + nt) * nblk + kb) * (2LL * cb * bn);
  if (tc_stacked(bn)) {
    hi = blk + ((long long)chunk * 2 * bn + n) * 8 + e;
    lo = hi + (long long)bn * 8;
  } else {
    hi = blk + ((long long)chunk * bn + n) * 8 + e;
    lo = hi + (long long)cb * bn;
  }
}

__global__ void tc_pack_kernel(const float* __restrict__ w, uint16_t* __restrict__ wpk, int taps, int C_in,
                               int C_out, int bn, int cb) {
  const long long total = (long long)taps * C_in * C_out;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int co = (int)(i % C_out);
    const long long r = i / C_out;
    const int ci = (int)(r % C_in);
    const int tap = (int)(r / C_in);
    long long oh, ol;
    tc_pack_offsets(tap, ci, co, C_in, C_out, bn, cb, oh, ol);
    __nv_bfloat16 hi, lo;
    split_bf16(w[i], hi, lo);
    wpk[oh] = __bfloat16_as_ushort(hi);
    wpk[ol] = __bfloat16_as_ushort(lo);
  }
}

// The same hi / lo values moved from the layout for column tiles of bn_a to
// the one for bn_b (K blocks of cb in both).
__global__ void tc_repack_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int taps, int C_in,
                                 int C_out, int bn_a, int bn_b, int cb) {
  const long long total = (long long)taps * C_in * C_out;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int co = (int)(i % C_out);
    const long long r = i / C_out;
    const int ci = (int)(r % C_in);
    const int tap = (int)(r / C_in);
    long long ah, al, bh, bl;
    tc_pack_offsets(tap, ci, co, C_in, C_out, bn_a, cb, ah, al);
    tc_pack_offsets(tap, ci, co, C_in, C_out, bn_b, cb, bh, bl);
    dst[bh] = src[ah];
    dst[bl] = src[al];
  }
}

void launch_tc_repack(const uint16_t* src, uint16_t* dst, int taps, int C_in, int C_out, int bn_a, int bn_b, int cb,
                      cudaStream_t st) {
  long long total = (long long)taps * C_in * C_out;
  int grid = (int)std::min<long long>(cdiv<long long>(total, 256), 148 * 16);
  tc_repack_kernel<<<grid, 256, 0, st>>>(src, dst, taps, C_in, C_out, bn_a, bn_b, cb);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

void launch_tc_pack(const float* w, uint16_t* wpk, int taps, int C_in, int C_out, int bn, int cb,
                    cudaStream_t st) {
  long long total = (long long)taps * C_in * C_out;
  int grid = (int)std::min<long long>(cdiv<long long>(total, 256), 148 * 16);
  tc_pack_kernel<<<grid, 256, 0, st>>>(w, wpk, taps, C_in, C_out, bn, cb);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

}  // namespace rvc
