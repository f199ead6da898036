// Device-resident HuBERT-base encoder.
//
// Reference semantics: HubertEncoder.encode (runtime/models/hubert.py:564-589)
// with the numpy branches of _feature_extractor (:658-696), _feature_projection
// (:775-803), _pos_conv_embed (:838-857), _encoder (:928-968) and
// _encoder_layer (:1262-1287).  Layout: channels-last [B][T][C] fp32; the B
// chunks of one call have equal length and run as one launch per layer (the
// transformer GEMMs treat all B*L frames as one row block).
//
// Strided convs: a kernel-K, stride-2 conv over x[T][512] is a stride-1 conv
// over the view v[T/2][1024] (v[r] = x[2r] ++ x[2r+1]):
//   y[t] = [W0 W1] . v[t]  (+ W2 . v[t+1][0:512] for K = 3)
// so the tensor-core kernel runs it as one 1-tap GEMM over 1024 channels, plus,
// for K = 3, a second 1-tap GEMM that reads the first half of the next view
// row and accumulates into the first one's output in its epilogue.
#include "hubert.cuh"

#include <algorithm>
#include <cmath>

namespace rvc {

HubertModel::HubertModel(Context* c, int prec) : ctx(c), precision(prec) {
  RVC_CHECK_ARG(prec == 0 || prec == 1, "hubert: precision must be 0 (tensor cores) or 1 (fp32 SIMT)");
}

void HubertModel::set_weight(const std::string& key_in, const float* host, const std::vector<int64_t>& shape) {
  std::string key = key_in;
  // torch parametrized weight-norm names (runtime/models/hubert.py:512-518)
  if (key == "encoder.pos_conv_embed.conv.parametrizations.weight.original0")
    key = "encoder.pos_conv_embed.conv.weight_g";
  if (key == "encoder.pos_conv_embed.conv.parametrizations.weight.original1")
    key = "encoder.pos_conv_embed.conv.weight_v";
  HubertTensor t;
  t.shape = shape;
  t.buf = DevBuf(ctx, sizeof(float) * (size_t)std::max<int64_t>(1, t.numel()));
  RVC_CUDA_TRY(cudaMemcpyAsync(t.buf.p, host, sizeof(float) * t.numel(), cudaMemcpyHostToDevice, ctx->stream));
  RVC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  raw_[key] = std::move(t);
  finalized_ = false;
}

const HubertTensor& HubertModel::W(const std::string& key) const {
  auto it = raw_.find(key);
  if (it == raw_.end()) throw Error{kErrState, "hubert: missing weight '" + key + "'"};
  return it->second;
}

static void expect(const HubertTensor& t, std::vector<int64_t> s, const std::string& key) {
  // linear weights may come as [O, I] or [O, I, 1]
  std::vector<int64_t> a = t.shape;
  while (a.size() > s.size() && a.back() == 1) a.pop_back();
  if (a != s) {
    std::string x, y;
    for (auto v : t.shape) x += std::to_string(v) + ",";
    for (auto v : s) y += std::to_string(v) + ",";
    throw Error{kErrArg, "hubert: weight '" + key + "' has shape [" + x + "] expected [" + y + "]"};
  }
}

int64_t HubertModel::out_len(int64_t T) {
  static const int ks[7] = {10, 3, 3, 3, 3, 2, 2};
  int64_t L = T;
  for (int i = 0; i < 7; ++i) {
    const int s = i == 0 ? 5 : 2;
    if (L < ks[i]) return 0;
    L = (L - ks[i]) / s + 1;
  }
  return L;
}

void HubertModel::finalize() {
  const bool tc = precision == 0;
  cudaStream_t st = ctx->stream;
  const int C = kConvC, D = kD;
  // ---------------- conv feature extractor
  {
    const auto& w0 = W("feature_extractor.conv_layers.0.conv.weight");
    expect(w0, {C, 1, 10}, "feature_extractor.conv_layers.0.conv.weight");
    conv0_w_ = DevBuf(ctx, sizeof(float) * C * 10);
    RVC_CUDA_TRY(cudaMemcpyAsync(conv0_w_.p, w0.buf.p, sizeof(float) * C * 10, cudaMemcpyDeviceToDevice, st));
    expect(W("feature_extractor.conv_layers.0.layer_norm.weight"), {C}, "conv_layers.0.layer_norm.weight");
    expect(W("feature_extractor.conv_layers.0.layer_norm.bias"), {C}, "conv_layers.0.layer_norm.bias");
  }
  for (int i = 1; i < 7; ++i) {
    const std::string key = "feature_extractor.conv_layers." + std::to_string(i) + ".conv.weight";
    const int K = conv_k_[i];
    expect(W(key), {C, C, K}, key);
    DevBuf wa(ctx, sizeof(float) * (size_t)C * 2 * C);
    k_taps_to_channels(W(key).buf.f(), C, C, K, 0, 2, wa.f(), st);
    convA_[i] = ConvLayer();
    convA_[i].build(ctx, LayerKind::kConv, wa.f(), nullptr, C, 2 * C, 1, tc);
    if (K == 3) {
      DevBuf wb(ctx, sizeof(float) * (size_t)C * C);
      k_taps_to_channels(W(key).buf.f(), C, C, K, 2, 1, wb.f(), st);
      convB_[i] = ConvLayer();
      convB_[i].pad_l = -1;  // reads view row t + 1
      convB_[i].build(ctx, LayerKind::kConv, wb.f(), nullptr, C, C, 1, tc);
    }
  }
  // ---------------- feature projection
  expect(W("feature_projection.layer_norm.weight"), {C}, "feature_projection.layer_norm.weight");
  expect(W("feature_projection.projection.weight"), {D, C}, "feature_projection.projection.weight");
  proj_ = ConvLayer();
  proj_.build(ctx, LayerKind::kConv, W("feature_projection.projection.weight").buf.f(),
              W("feature_projection.projection.bias").buf.f(), D, C, 1, tc);
  // ---------------- positional conv (weight norm over dims 0,1, runtime/models/hubert.py:509-522)
  {
    const int I = D / kPosGroups;
    DevBuf wpos(ctx, sizeof(float) * (size_t)D * I * kPosK);
    auto it = raw_.find("_pos_conv_weight");
    if (it != raw_.end()) {
      expect(it->second, {D, I, kPosK}, "_pos_conv_weight");
      RVC_CUDA_TRY(cudaMemcpyAsync(wpos.p, it->second.buf.p, wpos.bytes, cudaMemcpyDeviceToDevice, st));
    } else {
      const auto& v = W("encoder.pos_conv_embed.conv.weight_v");
      const auto& g = W("encoder.pos_conv_embed.conv.weight_g");
      expect(v, {D, I, kPosK}, "encoder.pos_conv_embed.conv.weight_v");
      RVC_CHECK_ARG(g.numel() == kPosK, "hubert: pos_conv weight_g must hold 128 values");
      k_fold_weight_norm_dim2(v.buf.f(), g.buf.f(), wpos.f(), (long long)D * I, kPosK, st);
    }
    pos_ = ConvLayer();
    pos_.groups = kPosGroups;
    pos_.pad_l = kPosK / 2;
    pos_.pad_r = kPosK / 2 - 1;  // SamePad: the last output frame is dropped
    pos_.build(ctx, LayerKind::kConv, wpos.f(), W("encoder.pos_conv_embed.conv.bias").buf.f(), D, I, kPosK, tc);
  }
  expect(W("encoder.layer_norm.weight"), {D}, "encoder.layer_norm.weight");
  // ---------------- transformer layers
  for (int l = 0; l < kLayers; ++l) {
    const std::string p = "encoder.layers." + std::to_string(l) + ".";
    DevBuf wqkv(ctx, sizeof(float) * 3 * D * D), bqkv(ctx, sizeof(float) * 3 * D);
    const char* nm[3] = {"attention.q_proj", "attention.k_proj", "attention.v_proj"};
    for (int j = 0; j < 3; ++j) {
      expect(W(p + nm[j] + ".weight"), {D, D}, p + nm[j] + ".weight");
      RVC_CUDA_TRY(cudaMemcpyAsync(wqkv.f() + (size_t)j * D * D, W(p + nm[j] + ".weight").buf.p,
                                   sizeof(float) * D * D, cudaMemcpyDeviceToDevice, st));
      RVC_CUDA_TRY(cudaMemcpyAsync(bqkv.f() + (size_t)j * D, W(p + nm[j] + ".bias").buf.p, sizeof(float) * D,
                                   cudaMemcpyDeviceToDevice, st));
    }
    qkv_[l] = ConvLayer();
    qkv_[l].build(ctx, LayerKind::kConv, wqkv.f(), bqkv.f(), 3 * D, D, 1, tc);
    expect(W(p + "attention.out_proj.weight"), {D, D}, p + "attention.out_proj.weight");
    o_[l] = ConvLayer();
    o_[l].build(ctx, LayerKind::kConv, W(p + "attention.out_proj.weight").buf.f(),
                W(p + "attention.out_proj.bias").buf.f(), D, D, 1, tc);
    expect(W(p + "feed_forward.intermediate_dense.weight"), {kFF, D}, p + "feed_forward.intermediate_dense.weight");
    ff1_[l] = ConvLayer();
    ff1_[l].build(ctx, LayerKind::kConv, W(p + "feed_forward.intermediate_dense.weight").buf.f(),
                  W(p + "feed_forward.intermediate_dense.bias").buf.f(), kFF, D, 1, tc);
    expect(W(p + "feed_forward.output_dense.weight"), {D, kFF}, p + "feed_forward.output_dense.weight");
    ff2_[l] = ConvLayer();
    ff2_[l].build(ctx, LayerKind::kConv, W(p + "feed_forward.output_dense.weight").buf.f(),
                  W(p + "feed_forward.output_dense.bias").buf.f(), D, kFF, 1, tc);
    expect(W(p + "layer_norm.weight"), {D}, p + "layer_norm.weight");
    expect(W(p + "final_layer_norm.weight"), {D}, p + "final_layer_norm.weight");
  }
  final_ = ConvLayer();
  if (raw_.count("final_proj.weight")) {
    expect(W("final_proj.weight"), {kFinal, D}, "final_proj.weight");
    final_.build(ctx, LayerKind::kConv, W("final_proj.weight").buf.f(), W("final_proj.bias").buf.f(), kFinal, D, 1,
                 tc);
  }
  RVC_CUDA_TRY(cudaStreamSynchronize(st));
  finalized_ = true;
}

// Rows per chunk in the conv-stack buffers: even (whole view rows) plus one
// spare view row, so a view row never reaches into the next chunk.
static int64_t conv_rows(int64_t T) { return (T + 1) / 2 * 2 + 2; }

void HubertModel::ensure_ws(int B, int64_t T) {
  if (B <= ws_B && T <= ws_T) return;
  B = std::max(B, ws_B);
  T = std::max(T, ws_T);
  ws_.clear();
  const int64_t T0 = (T - 10) / 5 + 1, T1 = (T0 - 3) / 2 + 1, L = out_len(T);
  auto add = [&](const char* n, long long per_chunk) {
    ws_.emplace(n, DevBuf(ctx, sizeof(float) * (size_t)B * std::max<long long>(1, per_chunk)));
  };
  add("x", T);
  add("fa", conv_rows(T0) * kConvC);
  add("fb", conv_rows(T1) * kConvC);
  ws_.emplace("gn", DevBuf(ctx, sizeof(float) * groupnorm_chan_scratch_floats(B, kConvC)));
  add("c6", L * kConvC);
  add("ln", L * kConvC);
  for (const char* n : {"hp", "pos", "h", "att", "t1", "out"}) add(n, L * kD);
  add("qkv", L * 3 * kD);
  add("ff", L * kFF);
  ws_B = B;
  ws_T = T;
}

void HubertModel::save_tap(const std::string& name, const float* d, int64_t rows, int C, int ld, long long bs,
                           int B) {
  if (!keep_taps) return;
  std::vector<float> h((size_t)B * rows * C);
  for (int b = 0; b < B; ++b)
    RVC_CUDA_TRY(cudaMemcpy2DAsync(h.data() + (size_t)b * rows * C, sizeof(float) * C, d + (size_t)b * bs,
                                   sizeof(float) * ld, sizeof(float) * C, rows, cudaMemcpyDeviceToHost, ctx->stream));
  RVC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  taps_[name] = std::move(h);
}

bool HubertModel::tap(const std::string& name, float* host, int64_t n) {
  auto it = taps_.find(name);
  if (it == taps_.end() || (int64_t)it->second.size() < n) return false;
  std::copy(it->second.begin(), it->second.begin() + n, host);
  return true;
}

void HubertModel::run_conv(const ConvLayer& L, const ConvIO& io) { L.run(ctx, io, precision == 1); }

void HubertModel::encode_device(int B, int64_t T, const float* x, int version, float* out) {
  if (!finalized_) throw Error{kErrState, "hubert: finalize() not called after the last weight upload"};
  RVC_CHECK_ARG(version == 1 || version == 2, "hubert: version must be 1 or 2");
  RVC_CHECK_ARG(B >= 1, "hubert: B must be positive");
  RVC_CHECK_ARG(T <= (1ll << 30), "hubert: input too long");
  const int64_t L = out_len(T);
  RVC_CHECK_ARG(L >= 1, "hubert: input of " + std::to_string(T) + " samples is too short for the conv stack");
  if (version == 1) RVC_CHECK_ARG(final_.C_out == kFinal, "hubert: version 1 needs final_proj.weight/bias");
  ensure_ws(B, T);
  cudaStream_t st = ctx->stream;
  const int C = kConvC, D = kD;
  taps_.clear();
  // ---------------- conv feature extractor
  int64_t Tl[7];
  Tl[0] = (T - 10) / 5 + 1;
  for (int i = 1; i < 7; ++i) Tl[i] = (Tl[i - 1] - conv_k_[i]) / 2 + 1;
  const long long bs_a = (long long)(ws_.at("fa").bytes / sizeof(float) / ws_B);
  const long long bs_b = (long long)(ws_.at("fb").bytes / sizeof(float) / ws_B);
  float* fa = buf("fa");
  float* fb = buf("fb");
  k_noise_conv(x, T, (int)T, conv0_w_.f(), nullptr, C, 10, 5, 0, B, (int)Tl[0], fa, bs_a, st);
  k_groupnorm_chan_gelu(fa, bs_a, (int)Tl[0], C, B, W("feature_extractor.conv_layers.0.layer_norm.weight").buf.f(),
                        W("feature_extractor.conv_layers.0.layer_norm.bias").buf.f(), 1e-5f, buf("gn"), st);
  save_tap("conv0", fa, Tl[0], C, C, bs_a, B);
  for (int i = 1; i < 7; ++i) {
    const float* in = (i & 1) ? fa : fb;
    const long long in_bs = (i & 1) ? bs_a : bs_b;
    float* o = (i == 6) ? buf("c6") : ((i & 1) ? fb : fa);
    const long long o_bs = (i == 6) ? (long long)L * C : ((i & 1) ? bs_b : bs_a);
    const int To = (int)Tl[i];
    ConvIO a;
    a.x = in; a.x_ld = 2 * C; a.x_bs = in_bs; a.T_in = To;
    a.y = o; a.y_ld = C; a.y_bs = o_bs;
    a.B = B;
    if (conv_k_[i] == 2) a.out_act = kActGelu;
    run_conv(convA_[i], a);
    if (conv_k_[i] == 3) {
      ConvIO b2;
      b2.x = in; b2.x_ld = 2 * C; b2.x_bs = in_bs; b2.T_in = To + 1;
      b2.y = o; b2.y_ld = C; b2.y_bs = o_bs;
      b2.accin = o; b2.acc_ld = C; b2.acc_bs = o_bs;
      b2.out_act = kActGelu;
      b2.B = B;
      run_conv(convB_[i], b2);
    }
    save_tap("conv" + std::to_string(i), o, To, C, C, o_bs, B);
  }
  // ---------------- feature projection: LN(512) -> Linear(512 -> 768)
  const long long rows = (long long)B * L;
  k_layernorm(buf("c6"), C, nullptr, 0, rows, C, W("feature_projection.layer_norm.weight").buf.f(),
              W("feature_projection.layer_norm.bias").buf.f(), 1e-5f, buf("ln"), C, st);
  auto gemm_io = [&](const float* xin, int ld_in, float* y, int ld_out) {
    ConvIO io;
    io.x = xin; io.x_ld = ld_in; io.x_bs = rows * ld_in; io.T_in = (int)rows;
    io.y = y; io.y_ld = ld_out; io.y_bs = rows * ld_out;
    io.B = 1;
    return io;
  };
  run_conv(proj_, gemm_io(buf("ln"), C, buf("hp"), D));
  save_tap("proj", buf("hp"), rows, D, D, 0, 1);
  // ---------------- positional conv + GELU, residual, encoder LN
  {
    ConvIO io;
    io.x = buf("hp"); io.x_ld = D; io.x_bs = (long long)L * D; io.T_in = (int)L;
    io.y = buf("pos"); io.y_ld = D; io.y_bs = (long long)L * D;
    io.out_act = kActGelu;
    io.B = B;
    run_conv(pos_, io);
    save_tap("pos", buf("pos"), rows, D, D, 0, 1);
  }
  float* h = buf("h");
  k_layernorm(buf("hp"), D, buf("pos"), D, rows, D, W("encoder.layer_norm.weight").buf.f(),
              W("encoder.layer_norm.bias").buf.f(), 1e-5f, h, D, st);
  // ---------------- 12 post-LN transformer layers
  const int nl = version == 1 ? 9 : kLayers;
  for (int l = 0; l < nl; ++l) {
    const std::string p = "encoder.layers." + std::to_string(l) + ".";
    run_conv(qkv_[l], gemm_io(h, D, buf("qkv"), 3 * D));
    // q * 64^-0.5 == q / 8 exactly
    {
      cudaEvent_t e0 = nullptr, e1 = nullptr;
      if (ctx->prof) ctx->prof_begin(&e0, &e1);
      if (precision == 1 || !k_attention_tc(ctx, buf("qkv"), 3 * D, 0, D, 2 * D, nullptr, nullptr, B, kHeads, kHeadD,
                                             (int)L, -1, 8.f, buf("att"), D))
        k_attention(buf("qkv"), 3 * D, 0, D, 2 * D, B, kHeads, kHeadD, (int)L, 8.f, buf("att"), D, st);
      if (ctx->prof)
        ctx->prof_end(e0, e1, 4.0 * B * kHeads * (double)L * L * kHeadD,
                      "attn hubert B=" + std::to_string(B) + " L=" + std::to_string(L), false);
    }
    ConvIO o = gemm_io(buf("att"), D, buf("t1"), D);
    o.res = h; o.res_ld = D; o.res_bs = rows * D;
    run_conv(o_[l], o);
    k_layernorm(buf("t1"), D, nullptr, 0, rows, D, W(p + "layer_norm.weight").buf.f(),
                W(p + "layer_norm.bias").buf.f(), 1e-5f, h, D, st);
    ConvIO f1 = gemm_io(h, D, buf("ff"), kFF);
    f1.out_act = kActGelu;
    run_conv(ff1_[l], f1);
    ConvIO f2 = gemm_io(buf("ff"), kFF, buf("t1"), D);
    f2.res = h; f2.res_ld = D; f2.res_bs = rows * D;
    run_conv(ff2_[l], f2);
    float* dst = (version == 2 && l == nl - 1) ? out : h;
    k_layernorm(buf("t1"), D, nullptr, 0, rows, D, W(p + "final_layer_norm.weight").buf.f(),
                W(p + "final_layer_norm.bias").buf.f(), 1e-5f, dst, D, st);
    save_tap("layer" + std::to_string(l), dst, rows, D, D, 0, 1);
  }
  if (version == 1) run_conv(final_, gemm_io(h, D, out, kFinal));
}

void HubertModel::encode_host(int B, int64_t T, const float* x, int version, float* out) {
  const int64_t L = out_len(T);
  RVC_CHECK_ARG(L >= 1, "hubert: input of " + std::to_string(T) + " samples is too short for the conv stack");
  ensure_ws(B, T);
  cudaStream_t st = ctx->stream;
  RVC_CUDA_TRY(cudaMemcpyAsync(buf("x"), x, sizeof(float) * (size_t)B * T, cudaMemcpyHostToDevice, st));
  encode_device(B, T, buf("x"), version, buf("out"));
  const int Co = version == 1 ? kFinal : kD;
  RVC_CUDA_TRY(cudaMemcpyAsync(out, buf("out"), sizeof(float) * (size_t)B * L * Co, cudaMemcpyDeviceToHost, st));
}

}  // namespace rvc
