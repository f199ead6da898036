#include "layer.cuh"

#include <algorithm>
#include <cstdio>

namespace rvc {

void ConvLayer::build(Context* ctx, LayerKind k, const float* W, const float* b, int O, int I, int Kk,
                      bool use_tc) {
  kind = k;
  K = Kk;
  cudaStream_t st = ctx->stream;
  std::vector<int> tap_k;
  slices.clear();
  if (k == LayerKind::kConv) {
    RVC_CHECK_ARG(groups >= 1 && groups <= kMaxSlices && O % groups == 0, "conv1d: groups must divide C_out, <= 16");
    C_in = I;
    C_out = O / groups;
    for (int g = 0; g < groups; ++g) {
      for (int j = 0; j < K; ++j) tap_k.push_back(j);
      ConvSlice s{};
      s.ntaps = K;
      s.tap_base = -pad_l;
      s.tap_step = dil;
      s.out_r0 = 0;
      s.ci_off = g * I;
      s.co_off = g * C_out;
      s.wtap0 = g * K;
      slices.push_back(s);
    }
  } else {
    // Transposed conv as `up` phase GEMMs: output row q*up + p takes taps
    // k = k0 + j*up with k0 = (p + pad) mod up, reading input row
    // q + (p + pad - k0)/up - j  (runtime/nn.py:294-346 scatter, gathered).
    C_in = I;
    C_out = O;
    RVC_CHECK_ARG(up >= 1 && up <= kMaxSlices, "conv_transpose1d: stride must be in [1,16]");
    for (int p = 0; p < up; ++p) {
      int k0 = (p + up_pad) % up;
      ConvSlice s{};
      s.wtap0 = (int)tap_k.size();
      int n = 0;
      for (int kk = k0; kk < K; kk += up) {
        tap_k.push_back(kk);
        ++n;
      }
      s.ntaps = n;
      s.tap_base = (p + up_pad - k0) / up;
      s.tap_step = -1;
      s.out_r0 = p;
      s.ci_off = 0;
      s.co_off = 0;
      slices.push_back(s);
    }
  }
  taps_total = (int)tap_k.size();
  DevBuf taps(ctx, sizeof(int) * std::max(1, taps_total));
  RVC_CUDA_TRY(cudaMemcpyAsync(taps.p, tap_k.data(), sizeof(int) * taps_total, cudaMemcpyHostToDevice, st));
  Wg = DevBuf(ctx, sizeof(float) * (size_t)std::max(1, taps_total) * C_in * C_out);
  if (k == LayerKind::kConv && groups > 1) {
    // group g: taps [g*K, (g+1)*K) of Wg hold W[g*C_out + o][i][k]
    for (int g = 0; g < groups; ++g)
      k_gather_taps(W + (size_t)g * C_out * I * K, Wg.f() + (size_t)g * K * I * C_out, C_out, I, K, 0, taps.as<int>(),
                    K, st);
  } else {
    k_gather_taps(W, Wg.f(), O, I, K, k == LayerKind::kConv ? 0 : 1, taps.as<int>(), taps_total, st);
  }
  if (b) {  // the epilogue indexes bias by the global output channel (co_off + co)
    const int nb = k == LayerKind::kConv ? O : C_out;
    bias = DevBuf(ctx, sizeof(float) * nb);
    RVC_CUDA_TRY(cudaMemcpyAsync(bias.p, b, sizeof(float) * nb, cudaMemcpyDeviceToDevice, st));
  }
  tc = use_tc && tc_shape_ok(C_in, C_out) && stride == 1;
  if (tc) {
    bn = tc_pick_bn(C_out);
    cb = tc_pick_cb(C_in);
    wpk = DevBuf(ctx, sizeof(uint16_t) * tc_packed_elems(taps_total, C_in, C_out, bn, cb));
    launch_tc_pack(Wg.f(), wpk.as<uint16_t>(), taps_total, C_in, C_out, bn, cb, st);
  }
  // square convs of the generator (ResBlocks: C_in == C_out) also get the
  // operand stages of the time-rows-as-N kernel
  tn = tc && k == LayerKind::kConv && groups == 1 && dil >= 1 && C_in == C_out && C_in % 32 == 0 &&
       (C_out == 32 || C_out == 64 || C_out % 128 == 0);
  if (tn) {
    wpk_t = DevBuf(ctx, sizeof(uint16_t) * tcn_packed_elems(taps_total, C_in, C_out));
    launch_tcn_pack(Wg.f(), wpk_t.as<uint16_t>(), taps_total, C_in, C_out, st);
  }
  RVC_CUDA_TRY(cudaStreamSynchronize(st));  // `taps` is freed on return
}

int ConvLayer::out_len(int T_in) const {
  if (kind == LayerKind::kConv) return (T_in + pad_l + pad_r - dil * (K - 1) - 1) / stride + 1;
  return (T_in - 1) * up - 2 * up_pad + (K - 1) + 1;
}

double ConvLayer::flops(int B, int T_in) const {
  return 2.0 * B * (double)out_len(T_in) * C_in * C_out * (kind == LayerKind::kConv ? (double)K * groups : (double)K / up);
}

void ConvLayer::run(Context* ctx, const ConvIO& io, bool force_simt) const {
  ConvArgs a{};
  a.x = io.x; a.x_bs = io.x_bs; a.x_ld = io.x_ld; a.T_in = io.T_in; a.C_in = C_in;
  a.in_act = io.in_act; a.in_slope = io.in_slope;
  a.stride = stride;
  a.out_rs = kind == LayerKind::kConv ? 1 : up;
  a.C_out = C_out;
  a.B = io.B;
  const int oL = out_len(io.T_in);
  RVC_CHECK_ARG(oL >= 0, "conv: negative output length");
  a.nslices = (int)slices.size();
  for (int s = 0; s < a.nslices; ++s) {
    a.sl[s] = slices[s];
    if (kind == LayerKind::kConv) {
      a.sl[s].rows = oL;
    } else {
      const int p = slices[s].out_r0;
      a.sl[s].rows = oL > p ? cdiv(oL - p, up) : 0;
    }
  }
  a.w = Wg.f();
  a.wpk = wpk.as<uint16_t>();
  a.bn = bn; a.cb = cb;
  a.bias = bias.p ? bias.f() : nullptr;
  a.bias2 = io.bias2; a.bias2_bs = io.bias2_bs;
  a.res = io.res; a.res_bs = io.res_bs; a.res_ld = io.res_ld; a.res_sub = io.res_sub;
  a.accin = io.accin; a.acc_bs = io.acc_bs; a.acc_ld = io.acc_ld;
  a.out_div = io.out_div;
  a.out_act = io.out_act; a.out_slope = io.out_slope;
  a.y = io.y; a.y_bs = io.y_bs; a.y_ld = io.y_ld; a.y_raw = io.y_raw;
  a.err = ctx->d_err;
  if (oL == 0 || io.B == 0) return;
  bool any_empty = false;  // a transposed-conv phase with no taps: output = epilogue(0)
  for (int s = 0; s < a.nslices; ++s) any_empty |= a.sl[s].ntaps == 0;
  const bool use_tc = tc && !force_simt && !any_empty && (io.x_ld % 4 == 0) && (io.x_bs % 4 == 0);
  RVC_CHECK_ARG(use_tc || Wg.p, "conv: fp32 weights were released; only the tensor-core path can run this layer");
  // Time rows as the MMA's N (tcn_conv.cu) where it measured faster than the
  // time-rows-as-M kernel (B200, both kernels on the same inputs in one
  // process, the v2-48k generator's ResBlock convs at 4 chunks per call):
  // C >= 128 always (0.54-0.87 of the time); C = 32 and 64 for K >= 7
  // (0.64-0.89) and for K = 3 without residual / accumulator inputs
  // (0.61-0.64).  At K = 3 with a residual input it is slower (1.1-1.4x).  At
  // least one wave of 256-row tiles.
  const int tcn_mode = tcn_enabled();
  const bool tn_pick = tcn_mode == 2 || C_out >= 128 || K >= 7 || (!io.res && !io.accin);
  if (use_tc && tn && tn_pick && tcn_mode != 0 && ((uintptr_t)io.x & 15) == 0 && tcn_fits(a)) {
    const long long tiles = (long long)io.B * cdiv(a.sl[0].rows, 256) * (C_out <= 64 ? 1 : C_out / 128);
    if (tiles >= ctx->num_sms()) {
      a.wpk = wpk_t.as<uint16_t>();
      cudaEvent_t e0 = nullptr, e1 = nullptr;
      if (ctx->prof) ctx->prof_begin(&e0, &e1);
      launch_tcn_conv(a, ctx->stream);
      if (ctx->prof) {
        char lab[160];
        snprintf(lab, sizeof(lab), "tcn conv Cin=%d Cout=%d K=%d dil=%d T=%d B=%d", C_in, C_out, K, dil, io.T_in,
                 io.B);
        ctx->prof_end(e0, e1, flops(io.B, io.T_in), lab);
      }
      return;
    }
  }
  if (use_tc) {
    // Few row tiles even at one 128-row subtile per tile: narrower column
    // tiles (the same weights repacked once) put more SMs to work.  Each
    // output's K order is unchanged.
    {
      int maxrows = 0;
      for (int s = 0; s < a.nslices; ++s) maxrows = std::max(maxrows, a.sl[s].rows);
      const long long row_tiles = (long long)io.B * a.nslices * cdiv(maxrows, 128);
      const int sms = ctx->num_sms();
      // only widths that keep the MMA efficient and the epilogue in whole
      // 32-column steps (narrower tiles measured slower)
      if (2 * row_tiles * (C_out / bn) < sms) {
        int want = 0;
        for (int c : {128, 64})
          if (c < bn && C_out % c == 0) {
            want = c;
            break;
          }
        if (want) {
          if (bn_n != want) {
            wpk_n = DevBuf(ctx, sizeof(uint16_t) * tc_packed_elems(taps_total, C_in, C_out, want, cb));
            launch_tc_repack(wpk.as<uint16_t>(), wpk_n.as<uint16_t>(), taps_total, C_in, C_out, bn, want, cb,
                             ctx->stream);
            bn_n = want;
          }
          a.wpk = wpk_n.as<uint16_t>();
          a.bn = bn_n;
        }
      }
    }
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ctx->prof) ctx->prof_begin(&e0, &e1);
    launch_tc_conv(a, ctx->stream);
    if (ctx->prof) {
      char lab[160];
      snprintf(lab, sizeof(lab), "%s Cin=%d Cout=%d K=%d dil=%d up=%d g=%d T=%d B=%d bn=%d cb=%d",
               kind == LayerKind::kConv ? "conv" : "convT", C_in, C_out, K, dil, up, groups, io.T_in, io.B, a.bn, cb);
      ctx->prof_end(e0, e1, flops(io.B, io.T_in), lab);
    }
  } else {
    launch_simt_conv(a, ctx->stream);
  }
}

}  // namespace rvc
