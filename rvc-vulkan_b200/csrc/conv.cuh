// Channels-last implicit-GEMM convolution for the RVC hot path.
//
// One description (ConvArgs) serves every GEMM-shaped op of the synthesizer and
// HuBERT: linears (K=1), same/valid convs with dilation, grouped convs (one
// "slice" per group) and transposed convs (one slice per output phase).
//
//   out[b, row(s,t), co_off(s)+co] = epilogue( sum_j sum_ci
//        act_in(x[b, t*stride + tap_base(s) + j*tap_step(s), ci_off(s)+ci]) * W[s][j][ci][co] )
//   row(s,t) = t*out_rs + out_r0(s)
//
// Activations are fp32 [B][T][C] (row stride x_ld).  Two kernels consume it:
//  * tc_conv_kernel: tcgen05.mma (kind::f16, BF16x3 split precision, fp32
//    accumulation in TMEM), weights streamed by cp.async.bulk, activations
//    split to bf16 hi/lo while staged to shared memory;
//  * simt_conv_kernel: plain fp32 FMA tiles, for shapes the tensor path does
//    not take (C_in or C_out not a multiple of 16) and as an in-library check.
#pragma once

#include "common.cuh"

namespace rvc {

constexpr int kMaxSlices = 16;

struct ConvSlice {
  int ntaps;       // taps in this slice
  int tap_base;    // input row offset of tap 0 (relative to t*stride)
  int tap_step;    // input row step between taps
  int out_r0;      // output physical row = t*out_rs + out_r0
  int rows;        // logical output rows t in [0, rows)
  int ci_off;      // input channel offset
  int co_off;      // output channel offset
  int wtap0;       // index of this slice's tap 0 in the weight tap axis
};

struct ConvArgs {
  // input
  const float* x;
  long long x_bs;  // batch stride (elements)
  int x_ld;        // row stride (elements)
  int T_in;        // valid input rows
  int C_in;        // channels contracted per slice
  int in_act;      // prologue activation (kActNone / kActLeaky)
  float in_slope;
  int stride;      // input rows per output row
  int out_rs;      // output row stride multiplier
  int C_out;       // output channels per slice
  int nslices;
  ConvSlice sl[kMaxSlices];
  int B;
  // weights: fp32 [taps_total][C_in][C_out] (SIMT) / packed bf16 hi-lo (tcgen05)
  const float* w;
  const uint16_t* wpk;
  int bn;          // tcgen05 N tile
  int cb;          // tcgen05 channel block (K per stage)
  // epilogue: v = acc + bias[c] + bias2[b][c] (+ res) ; v = accin + v ; v /= div ;
  //           y = act(v)   (optionally also y_raw = v before act)
  const float* bias;
  const float* bias2; long long bias2_bs;
  const float* res; long long res_bs; int res_ld;
  int res_sub;     // 0: v + res ; 1: res - v  (flow coupling x1 - m)
  const float* accin; long long acc_bs; int acc_ld;
  float out_div;   // 0: none
  int out_act; float out_slope;
  float* y; long long y_bs; int y_ld;
  float* y_raw;    // optional pre-activation copy (same strides as y)
  int* err;        // device error flag (bounded waits)
};

// v / d for a divisor d used across many values, with rd = __frcp_rn(d): the
// quotient q = RN(v * rd) corrected once by its remainder, RN(q + RN(v - q*d) * rd)
// (division by a constant known in advance: Markstein's correction step, as in
// Brisebarre, Muller and Raina, IEEE Trans. Computers 2004).  Checked on the
// host against IEEE v / d over every mantissa of 9 binades, both signs, for
// d = 2, 3, 5, 7: identical (so for every normal v and these d); 3 instructions
// instead of a full division per value.
__device__ __forceinline__ float div_by(float v, float d, float rd) {
  const float q = __fmul_rn(v, rd);
  const float r = __fmaf_rn(-q, d, v);
  return __fmaf_rn(r, rd, q);
}

// Epilogue for one output element (physical row `prow`, channel `c` in [0, C_out)
// of slice s).  `acc` is the raw dot product.
__device__ __forceinline__ void conv_epilogue(const ConvArgs& a, int b, int prow, int cg, float acc) {
  float v = acc;
  if (a.bias) v += a.bias[cg];
  if (a.bias2) v += a.bias2[(long long)b * a.bias2_bs + cg];
  if (a.res) {
    const float r = a.res[(long long)b * a.res_bs + (long long)prow * a.res_ld + cg];
    v = a.res_sub ? (r - v) : (v + r);
  }
  if (a.accin) v = a.accin[(long long)b * a.acc_bs + (long long)prow * a.acc_ld + cg] + v;
  if (a.out_div != 0.f) v = v / a.out_div;
  long long o = (long long)b * a.y_bs + (long long)prow * a.y_ld + cg;
  if (a.y_raw) a.y_raw[o] = v;
  a.y[o] = act_apply(v, a.out_act, a.out_slope);
}

// Host launchers (conv.cu).
void launch_simt_conv(const ConvArgs& a, cudaStream_t st);
void launch_tc_conv(const ConvArgs& a, cudaStream_t st);
// Pack fp32 [taps][C_in][C_out] into the tcgen05 operand layout (conv.cu).
size_t tc_packed_elems(int taps, int C_in, int C_out, int bn, int cb);
// Packed weights for column tiles of bn_a -> the layout for bn_b (same values).
void launch_tc_repack(const uint16_t* src, uint16_t* dst, int taps, int C_in, int C_out, int bn_a, int bn_b, int cb,
                      cudaStream_t st);
void launch_tc_pack(const float* w, uint16_t* wpk, int taps, int C_in, int C_out, int bn, int cb,
                    cudaStream_t st);
bool tc_shape_ok(int C_in, int C_out);
// Narrow N tiles issue A_hi.[B_hi | B_lo] as one N = 2*bn MMA plus A_lo.B_hi
// (two MMAs per k step instead of three); the packed weight layout follows.
__host__ __device__ __forceinline__ bool tc_stacked(int bn) { return bn <= 64; }
int tc_pick_bn(int C_out);
int tc_pick_cb(int C_in);
// Time-rows-as-N tensor-core conv (tcn_conv.cu): one slice, stride 1, dilated
// taps, C_in % 32 == 0, C_out == 32, 64 or a multiple of 128.
bool tcn_shape_ok(const ConvArgs& a);
// tcn_shape_ok and a pipeline plan that fits in shared memory
bool tcn_fits(const ConvArgs& a);
size_t tcn_packed_elems(int taps, int C_in, int C_out);
void launch_tcn_pack(const float* w, uint16_t* out, int taps, int C_in, int C_out, cudaStream_t st);
void launch_tcn_conv(const ConvArgs& a, cudaStream_t st);
// RVC_CUDA_TCN (read once): 0 = never use the time-as-N kernel, 2 = use it for
// every conv it can run (for timing both kernels), otherwise (default, 1) where
// ConvLayer::run's routing picks it.
int tcn_enabled();

}  // namespace rvc
