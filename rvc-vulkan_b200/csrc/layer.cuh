// ConvLayer: device-resident weights of one GEMM-shaped op in both operand
// forms (fp32 [taps][C_in][C_out] and the packed bf16 hi/lo tensor-core form),
// plus the slice geometry; run() binds activations and an epilogue.
#pragma once

#include "context.cuh"
#include "conv.cuh"
#include "kernels.cuh"

#include <string>
#include <vector>

namespace rvc {

// Epilogue/IO binding for one launch (everything ConvArgs needs besides weights).
struct ConvIO {
  const float* x = nullptr; long long x_bs = 0; int x_ld = 0; int T_in = 0;
  int in_act = kActNone; float in_slope = 0.f;
  float* y = nullptr; long long y_bs = 0; int y_ld = 0;
  float* y_raw = nullptr;
  const float* bias2 = nullptr; long long bias2_bs = 0;
  const float* res = nullptr; long long res_bs = 0; int res_ld = 0; int res_sub = 0;
  const float* accin = nullptr; long long acc_bs = 0; int acc_ld = 0;
  float out_div = 0.f;
  int out_act = kActNone; float out_slope = 0.f;
  int B = 1;
};

enum class LayerKind { kConv, kConvT };

struct ConvLayer {
  LayerKind kind = LayerKind::kConv;
  int C_in = 0, C_out = 0, K = 0;
  int dil = 1, pad_l = 0, pad_r = 0, stride = 1;  // conv
  int up = 1, up_pad = 0;                          // convT: stride, padding
  int groups = 1;                                  // conv: one slice per group (<= 16)
  int taps_total = 0;
  std::vector<ConvSlice> slices;  // rows filled per launch
  DevBuf Wg, wpk, bias;
  bool tc = false;
  int bn = 0, cb = 0;
  // narrower column tiles for launches whose row tiles leave SMs idle (one
  // short sequence), packed from wpk on first use
  mutable DevBuf wpk_n;
  mutable int bn_n = 0;
  // operand stages of the time-rows-as-N kernel (tcn_conv.cu), for convs it takes
  DevBuf wpk_t;
  bool tn = false;

  // W: conv [O,I,K] (I = input channels per group) or convT [I,O,K], device
  // fp32 (already weight-norm folded).
  void build(Context* ctx, LayerKind k, const float* W, const float* b, int O, int I, int Kk, bool use_tc);
  int out_len(int T_in) const;
  // Launch on ctx->stream.  force_simt: run the fp32 SIMT kernel.
  void run(Context* ctx, const ConvIO& io, bool force_simt = false) const;
  double flops(int B, int T_in) const;
  // Drops the fp32 weight copy when the tensor-core form exists (the SIMT
  // kernel, which reads it, is then unavailable for this layer).
  void release_fp32() {
    if (tc) Wg.reset();
  }
};

}  // namespace rvc
