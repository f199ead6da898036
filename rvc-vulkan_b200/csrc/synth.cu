// Device-resident SynthesizerTrnMs768NSFsid inference.
//
// Reference semantics: SynthesizerTrn.infer_controlled
// (runtime/models/vits.py:2551-2598) with the numpy branches of
// _TextEncoder.embed/encode/stats (:499-538, :962-1059), _FlowBlock.reverse
// (:1086-1145, :1255-1268) and _GeneratorNSF.forward (:2133-2231).
// Layout: every activation is channels-last [B][T][C] fp32; the B chunks of
// one call are independent and run as one batched launch per layer.
#include "synth.cuh"

#include <cmath>
#include <stdexcept>

namespace rvc {

SynthModel::SynthModel(Context* c, const SynthConfig& cf) : ctx(c), cfg(cf) {
  RVC_CHECK_ARG(cfg.n_ups >= 1 && cfg.n_ups <= 8 && (int)cfg.rates.size() == cfg.n_ups &&
                    (int)cfg.kernels.size() == cfg.n_ups,
                "synth: bad upsample config");
  RVC_CHECK_ARG(cfg.layers >= 1 && cfg.layers <= 8, "synth: 1..8 encoder layers supported");
  RVC_CHECK_ARG(cfg.hidden == cfg.heads * cfg.kc, "synth: hidden != heads*kc");
}

void SynthModel::set_weight(const std::string& key, const float* host, const std::vector<int64_t>& shape) {
  RawTensor t;
  t.shape = shape;
  t.buf = DevBuf(ctx, sizeof(float) * (size_t)std::max<int64_t>(1, t.numel()));
  RVC_CUDA_TRY(cudaMemcpyAsync(t.buf.p, host, sizeof(float) * t.numel(), cudaMemcpyHostToDevice, ctx->stream));
  RVC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  raw_[key] = std::move(t);
  finalized_ = false;
}

const RawTensor& SynthModel::W(const std::string& key) const {
  auto it = raw_.find(key);
  if (it == raw_.end()) throw Error{kErrState, "synth: missing weight '" + key + "'"};
  return it->second;
}

DevBuf SynthModel::fold(const std::string& base) {
  const RawTensor& v = W(base + ".weight_v");
  const RawTensor& g = W(base + ".weight_g");
  const int rows = (int)v.shape[0];
  RVC_CHECK_ARG(g.numel() == rows, "synth: weight_g of " + base + " does not match weight_v rows");
  DevBuf out(ctx, sizeof(float) * v.numel());
  k_fold_weight_norm(v.buf.f(), g.buf.f(), out.f(), rows, (int)(v.numel() / rows), ctx->stream);
  return out;
}

static void expect_shape(const RawTensor& t, std::vector<int64_t> s, const std::string& key) {
  if (t.shape != s) {
    std::string a, b;
    for (auto v : t.shape) a += std::to_string(v) + ",";
    for (auto v : s) b += std::to_string(v) + ",";
    throw Error{kErrArg, "synth: weight '" + key + "' has shape [" + a + "] expected [" + b + "]"};
  }
}

void SynthModel::finalize() {
  const bool tc = cfg.precision == 0;
  const int H = cfg.hidden, F = cfg.filter;
  cudaStream_t st = ctx->stream;
  // ---------------- enc_p
  {
    const auto& w = W("enc_p.emb_phone.weight");
    expect_shape(w, {H, cfg.phone_dim}, "enc_p.emb_phone.weight");
    emb_phone_.build(ctx, LayerKind::kConv, w.buf.f(), W("enc_p.emb_phone.bias").buf.f(), H, cfg.phone_dim, 1, tc);
  }
  for (int i = 0; i < cfg.layers; ++i) {
    const std::string p = "enc_p.encoder.attn_layers." + std::to_string(i);
    DevBuf wqkv(ctx, sizeof(float) * 3 * H * H), bqkv(ctx, sizeof(float) * 3 * H);
    const char* nm[3] = {".conv_q", ".conv_k", ".conv_v"};
    for (int j = 0; j < 3; ++j) {
      const auto& w = W(p + nm[j] + ".weight");
      expect_shape(w, {H, H, 1}, p + nm[j] + ".weight");
      RVC_CUDA_TRY(cudaMemcpyAsync(wqkv.f() + (size_t)j * H * H, w.buf.p, sizeof(float) * H * H,
                                   cudaMemcpyDeviceToDevice, st));
      RVC_CUDA_TRY(cudaMemcpyAsync(bqkv.f() + (size_t)j * H, W(p + nm[j] + ".bias").buf.p, sizeof(float) * H,
                                   cudaMemcpyDeviceToDevice, st));
    }
    qkv_[i].build(ctx, LayerKind::kConv, wqkv.f(), bqkv.f(), 3 * H, H, 1, tc);
    o_[i].build(ctx, LayerKind::kConv, W(p + ".conv_o.weight").buf.f(), W(p + ".conv_o.bias").buf.f(), H, H, 1, tc);
    expect_shape(W(p + ".emb_rel_k"), {1, 2 * cfg.window + 1, cfg.kc}, p + ".emb_rel_k");
    const std::string f = "enc_p.encoder.ffn_layers." + std::to_string(i);
    ffn1_[i].pad_l = ffn1_[i].pad_r = 1;
    expect_shape(W(f + ".conv_1.weight"), {F, H, 3}, f + ".conv_1.weight");
    ffn1_[i].build(ctx, LayerKind::kConv, W(f + ".conv_1.weight").buf.f(), W(f + ".conv_1.bias").buf.f(), F, H, 3, tc);
    ffn2_[i].pad_l = ffn2_[i].pad_r = 1;
    ffn2_[i].build(ctx, LayerKind::kConv, W(f + ".conv_2.weight").buf.f(), W(f + ".conv_2.bias").buf.f(), H, F, 3, tc);
  }
  proj_.build(ctx, LayerKind::kConv, W("enc_p.proj.weight").buf.f(), W("enc_p.proj.bias").buf.f(), 2 * H, H, 1, tc);
  // ---------------- flow (coupling layers 0,2,4,6)
  for (int fi = 0; fi < 4; ++fi) {
    const std::string p = "flow.flows." + std::to_string(2 * fi);
    pre_[fi].build(ctx, LayerKind::kConv, W(p + ".pre.weight").buf.f(), W(p + ".pre.bias").buf.f(), H, H / 2, 1, tc);
    flow_cond_w_[fi] = fold(p + ".enc.cond_layer");
    flow_cond_b_[fi] = DevBuf(ctx, sizeof(float) * 6 * H);
    RVC_CUDA_TRY(cudaMemcpyAsync(flow_cond_b_[fi].p, W(p + ".enc.cond_layer.bias").buf.p, sizeof(float) * 6 * H,
                                 cudaMemcpyDeviceToDevice, st));
    for (int i = 0; i < 3; ++i) {
      const std::string li = p + ".enc.in_layers." + std::to_string(i);
      DevBuf wi = fold(li);
      in_[fi][i].pad_l = in_[fi][i].pad_r = 2;
      in_[fi][i].build(ctx, LayerKind::kConv, wi.f(), W(li + ".bias").buf.f(), 2 * H, H, 5, tc);
      const std::string lr = p + ".enc.res_skip_layers." + std::to_string(i);
      DevBuf wr = fold(lr);
      const int ro = i < 2 ? 2 * H : H;
      rs_[fi][i].build(ctx, LayerKind::kConv, wr.f(), W(lr + ".bias").buf.f(), ro, H, 1, tc);
    }
    post_[fi].build(ctx, LayerKind::kConv, W(p + ".post.weight").buf.f(), W(p + ".post.bias").buf.f(), H / 2, H, 1, tc);
  }
  // ---------------- dec
  conv_pre_.pad_l = conv_pre_.pad_r = 3;
  expect_shape(W("dec.conv_pre.weight"), {cfg.up0, H, 7}, "dec.conv_pre.weight");
  conv_pre_.build(ctx, LayerKind::kConv, W("dec.conv_pre.weight").buf.f(), W("dec.conv_pre.bias").buf.f(), cfg.up0,
                  H, 7, tc);
  for (int i = 0; i < cfg.n_ups; ++i) {
    const int cin = cfg.up0 >> i, cout = cfg.up0 >> (i + 1);
    const std::string u = "dec.ups." + std::to_string(i);
    expect_shape(W(u + ".weight_v"), {cin, cout, cfg.kernels[i]}, u + ".weight_v");
    DevBuf wu = fold(u);
    ups_[i].up = cfg.rates[i];
    ups_[i].up_pad = (cfg.kernels[i] - cfg.rates[i]) / 2;
    ups_[i].build(ctx, LayerKind::kConvT, wu.f(), W(u + ".bias").buf.f(), cout, cin, cfg.kernels[i], tc);
    const auto& nw = W("dec.noise_convs." + std::to_string(i) + ".weight");
    noise_k_[i] = (int)nw.shape[2];
    noise_s_[i] = i < cfg.n_ups - 1 ? noise_k_[i] / 2 : 1;
    const int ks[3] = {3, 7, 11}, ds[3] = {1, 3, 5};
    for (int j = 0; j < 3; ++j) {
      const std::string rb = "dec.resblocks." + std::to_string(i * 3 + j);
      for (int m = 0; m < 3; ++m) {
        const int k = ks[j], d = ds[m];
        DevBuf w1 = fold(rb + ".convs1." + std::to_string(m));
        rb1_[i][j][m].dil = d;
        rb1_[i][j][m].pad_l = rb1_[i][j][m].pad_r = (k * d - d) / 2;
        rb1_[i][j][m].build(ctx, LayerKind::kConv, w1.f(), W(rb + ".convs1." + std::to_string(m) + ".bias").buf.f(),
                            cout, cout, k, tc);
        DevBuf w2 = fold(rb + ".convs2." + std::to_string(m));
        rb2_[i][j][m].pad_l = rb2_[i][j][m].pad_r = (k - 1) / 2;
        rb2_[i][j][m].build(ctx, LayerKind::kConv, w2.f(), W(rb + ".convs2." + std::to_string(m) + ".bias").buf.f(),
                            cout, cout, k, tc);
      }
    }
  }
  expect_shape(W("dec.conv_post.weight"), {1, cfg.up0 >> cfg.n_ups, 7}, "dec.conv_post.weight");
  RVC_CUDA_TRY(cudaMemcpyAsync(&lin_w_, W("dec.m_source.l_linear.weight").buf.p, sizeof(float),
                               cudaMemcpyDeviceToHost, st));
  RVC_CUDA_TRY(cudaMemcpyAsync(&lin_b_, W("dec.m_source.l_linear.bias").buf.p, sizeof(float),
                               cudaMemcpyDeviceToHost, st));
  W("emb_g.weight");
  W("enc_p.emb_pitch.weight");
  RVC_CUDA_TRY(cudaStreamSynchronize(st));
  finalized_ = true;
}

void SynthModel::ensure_ws(int B, int P) {
  if (B <= ws_B && P <= ws_P) return;
  B = std::max(B, ws_B);
  P = std::max(P, ws_P);
  ws_.clear();
  const int H = cfg.hidden, F = cfg.filter, upp = cfg.upp();
  long long dmax = (long long)P * cfg.up0;
  long long L = P;
  for (int i = 0; i < cfg.n_ups; ++i) {
    L *= cfg.rates[i];
    dmax = std::max(dmax, L * (cfg.up0 >> (i + 1)));
  }
  auto add = [&](const char* n, long long per_chunk, size_t elem = sizeof(float)) {
    ws_.emplace(n, DevBuf(ctx, elem * (size_t)B * per_chunk));
  };
  add("in_phone", (long long)P * cfg.phone_dim);
  add("in_pitch", P, sizeof(long long));
  add("in_f0", P);
  add("in_sid", 1, sizeof(long long));
  add("in_nz", (long long)P * H);
  add("in_ns", (long long)P * upp);
  add("out_wave", (long long)P * upp);
  add("gvec", cfg.gin);
  add("dcond", cfg.up0);
  for (const char* n : {"fcond0", "fcond1", "fcond2", "fcond3"}) add(n, 6 * H);
  for (const char* n : {"ex", "att", "ao", "y2", "z", "zf", "h", "acts", "skip"}) add(n, (long long)P * H);
  add("qkv", (long long)P * 3 * H);
  add("y1", (long long)P * F);
  add("stats", (long long)P * 2 * H);
  add("xin", (long long)P * 2 * H);
  add("rs", (long long)P * 2 * H);
  add("har", (long long)P * upp);
  add("phase", P);
  for (const char* n : {"xo", "x0", "r", "t", "s", "noise"}) add(n, dmax);
  ws_B = B;
  ws_P = P;
}

void SynthModel::save_tap(const std::string& name, const float* d, int64_t per_chunk, int B) {
  if (!keep_taps) return;
  int64_t off = 0, n = per_chunk * B;
  if (keep_taps >= 2) {
    const int c = keep_taps - 2;
    if (c >= B) return;
    off = per_chunk * c;
    n = per_chunk;
  }
  std::vector<float> h((size_t)n);
  RVC_CUDA_TRY(cudaMemcpyAsync(h.data(), d + off, sizeof(float) * n, cudaMemcpyDeviceToHost, ctx->stream));
  RVC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  taps_[name] = std::move(h);
}

bool SynthModel::tap(const std::string& name, float* host, int64_t n) {
  auto it = taps_.find(name);
  if (it == taps_.end() || (int64_t)it->second.size() < n) return false;
  std::copy(it->second.begin(), it->second.begin() + n, host);
  return true;
}

void SynthModel::run_conv(const ConvLayer& L, const ConvIO& io) { L.run(ctx, io, cfg.precision == 1); }

static ConvIO io_rows(const float* x, int ld, int T, float* y, int y_ld, int B, long long x_bs, long long y_bs) {
  ConvIO io;
  io.x = x; io.x_ld = ld; io.T_in = T; io.x_bs = x_bs;
  io.y = y; io.y_ld = y_ld; io.y_bs = y_bs;
  io.B = B;
  return io;
}

// enc_p + speaker conditioning + z_p = m + exp(logs) * nz * 0.66666 into buf("z").
void SynthModel::enc_stage(int B, int P, const float* phone, const long long* pitch, const long long* sid,
                           const float* nz) {
  cudaStream_t st = ctx->stream;
  const int H = cfg.hidden, F = cfg.filter;
  const long long PH = (long long)P * H;
  // speaker conditioning g = emb_g(sid); dec.cond(g); flow cond layers
  k_embedding(sid, B, W("emb_g.weight").buf.f(), (int)W("emb_g.weight").shape[0], cfg.gin, buf("gvec"), st);
  k_gemv_rows(W("dec.cond.weight").buf.f(), W("dec.cond.bias").buf.f(), buf("gvec"), B, cfg.up0, cfg.gin,
              buf("dcond"), st);
  static const char* fc[4] = {"fcond0", "fcond1", "fcond2", "fcond3"};
  for (int fi = 0; fi < 4; ++fi)
    k_gemv_rows(flow_cond_w_[fi].f(), flow_cond_b_[fi].f(), buf("gvec"), B, 6 * H, cfg.gin, buf(fc[fi]), st);

  // ---------------- enc_p
  float* ex = buf("ex");
  run_conv(emb_phone_, io_rows(phone, cfg.phone_dim, P, ex, H, B, (long long)P * cfg.phone_dim, PH));
  k_enc_embed_finish(ex, pitch, W("enc_p.emb_pitch.weight").buf.f(), (long long)B * P, H,
                     (float)std::sqrt((double)H), st);
  save_tap("enc.embed", ex, PH, B);
  for (int i = 0; i < cfg.layers; ++i) {
    const std::string p = "enc_p.encoder.attn_layers." + std::to_string(i);
    run_conv(qkv_[i], io_rows(ex, H, P, buf("qkv"), 3 * H, B, PH, 3 * PH));
    {
      cudaEvent_t e0 = nullptr, e1 = nullptr;
      if (ctx->prof) ctx->prof_begin(&e0, &e1);
      if (cfg.precision == 1 ||
          !k_attention_tc(ctx, buf("qkv"), 3 * H, 0, H, 2 * H, W(p + ".emb_rel_k").buf.f(),
                          W(p + ".emb_rel_v").buf.f(), B, cfg.heads, cfg.kc, P, cfg.window,
                          (float)std::sqrt((double)cfg.kc), buf("att"), H))
        k_rel_attention(buf("qkv"), 3 * H, 0, H, 2 * H, W(p + ".emb_rel_k").buf.f(), W(p + ".emb_rel_v").buf.f(), B,
                        cfg.heads, cfg.kc, P, cfg.window, nullptr, buf("att"), H, st);
      if (ctx->prof)
        ctx->prof_end(e0, e1, 4.0 * B * cfg.heads * (double)P * P * cfg.kc,
                      "attn enc_p B=" + std::to_string(B) + " P=" + std::to_string(P), false);
    }
    run_conv(o_[i], io_rows(buf("att"), H, P, buf("ao"), H, B, PH, PH));
    save_tap("enc.l" + std::to_string(i) + ".attn", buf("ao"), PH, B);
    const std::string nl = "enc_p.encoder.norm_layers_";
    k_layernorm(ex, H, buf("ao"), H, (long long)B * P, H, W(nl + "1." + std::to_string(i) + ".gamma").buf.f(),
                W(nl + "1." + std::to_string(i) + ".beta").buf.f(), 1e-5f, ex, H, st);
    ConvIO f1 = io_rows(ex, H, P, buf("y1"), F, B, PH, (long long)P * F);
    f1.out_act = kActRelu;
    run_conv(ffn1_[i], f1);
    run_conv(ffn2_[i], io_rows(buf("y1"), F, P, buf("y2"), H, B, (long long)P * F, PH));
    k_layernorm(ex, H, buf("y2"), H, (long long)B * P, H, W(nl + "2." + std::to_string(i) + ".gamma").buf.f(),
                W(nl + "2." + std::to_string(i) + ".beta").buf.f(), 1e-5f, ex, H, st);
    save_tap("enc.l" + std::to_string(i), ex, PH, B);
  }
  run_conv(proj_, io_rows(ex, H, P, buf("stats"), 2 * H, B, PH, 2 * PH));
  k_zp(buf("stats"), nz, B, P, H, buf("z"), st);
  save_tap("enc.zp", buf("z"), PH, B);

}

// Flow reverse over P frames of z (rows of H channels, batch stride P*H); zf is
// scratch of the same size.  Returns the buffer holding the result.
float* SynthModel::flow_stage(int B, int P, float* z, float* zf) {
  cudaStream_t st = ctx->stream;
  const int H = cfg.hidden;
  const long long PH = (long long)P * H;
  static const char* fc[4] = {"fcond0", "fcond1", "fcond2", "fcond3"};
  // ---------------- flow reverse: Flip, RC(6), Flip, RC(4), Flip, RC(2), Flip, RC(0)
  for (int fi = 3; fi >= 0; --fi) {
    k_flip_channels(z, zf, (long long)B * P, H, st);
    run_conv(pre_[fi], io_rows(zf, H, P, buf("h"), H, B, PH, PH));
    for (int i = 0; i < 3; ++i) {
      ConvIO a = io_rows(buf("h"), H, P, buf("xin"), 2 * H, B, PH, 2 * PH);
      a.bias2 = buf(fc[fi]) + i * 2 * H;
      a.bias2_bs = 6 * H;
      run_conv(in_[fi][i], a);
      k_gate_rows(buf("xin"), (long long)B * P, H, buf("acts"), st);
      const int ro = i < 2 ? 2 * H : H;
      run_conv(rs_[fi][i], io_rows(buf("acts"), H, P, buf("rs"), ro, B, PH, (long long)P * ro));
      k_wn_update(buf("h"), buf("skip"), buf("rs"), (long long)B * P, H, i == 0, i == 2, st);
    }
    ConvIO pm = io_rows(buf("skip"), H, P, zf + H / 2, H, B, PH, PH);
    pm.res = zf + H / 2;
    pm.res_ld = H;
    pm.res_bs = PH;
    pm.res_sub = 1;
    run_conv(post_[fi], pm);
    std::swap(z, zf);
  }
  return z;
}

// GeneratorNSF over P frames of z (batch stride z_bs) with the harmonic source
// har (har_len samples per chunk, batch stride har_bs) -> wave [B][P*upp].
void SynthModel::dec_stage(int B, int P, const float* z, long long z_bs, const float* har, long long har_bs,
                           int har_len, float* wave) {
  cudaStream_t st = ctx->stream;
  const int H = cfg.hidden, upp = cfg.upp();
  const long long PH = z_bs;
  // ---------------- GeneratorNSF
  const long long N = (long long)P * upp;
  long long dmax = ws_.at("xo").bytes / sizeof(float) / ws_B;
  float *xo = buf("xo"), *x0 = buf("x0"), *r = buf("r"), *t = buf("t"), *s = buf("s");
  {
    ConvIO a = io_rows(z, H, P, xo, cfg.up0, B, PH, dmax);
    a.bias2 = buf("dcond");
    a.bias2_bs = cfg.up0;
    run_conv(conv_pre_, a);
    save_tap("dec.pre", xo, dmax, B);
  }
  int Lc = P;
  for (int i = 0; i < cfg.n_ups; ++i) {
    const int C = cfg.up0 >> (i + 1);
    const int Ln = ups_[i].out_len(Lc);
    {
      ConvIO a = io_rows(xo, cfg.up0 >> i, Lc, x0, C, B, dmax, dmax);
      a.in_act = kActLeaky;
      a.in_slope = 0.1f;
      // x = ups(x) + noise_conv(har): the noise conv (bias included) runs first
      // and enters the transposed conv's epilogue as its residual term.
      k_noise_conv(har, har_bs, har_len, W("dec.noise_convs." + std::to_string(i) + ".weight").buf.f(),
                   W("dec.noise_convs." + std::to_string(i) + ".bias").buf.f(), C, noise_k_[i], noise_s_[i],
                   noise_s_[i] / 2, B, Ln, buf("noise"), dmax, st);
      a.res = buf("noise");
      a.res_bs = dmax;
      a.res_ld = C;
      run_conv(ups_[i], a);
      save_tap("dec.s" + std::to_string(i) + ".ups", x0, dmax, B);
    }
    for (int j = 0; j < 3; ++j) {
      for (int m = 0; m < 3; ++m) {
        const float* in = m == 0 ? x0 : r;
        ConvIO a = io_rows(in, C, Ln, t, C, B, dmax, dmax);
        a.in_act = kActLeaky;
        a.in_slope = 0.1f;
        a.out_act = kActLeaky;
        a.out_slope = 0.1f;
        run_conv(rb1_[i][j][m], a);
        ConvIO c = io_rows(t, C, Ln, r, C, B, dmax, dmax);
        c.res = in;
        c.res_bs = dmax;
        c.res_ld = C;
        if (m == 2) {
          if (j == 0) {
            c.y = s;
          } else if (j == 1) {
            c.y = s;
            c.accin = s; c.acc_bs = dmax; c.acc_ld = C;
          } else {
            c.y = xo;
            c.accin = s; c.acc_bs = dmax; c.acc_ld = C;
            c.out_div = 3.f;
          }
        }
        run_conv(rb2_[i][j][m], c);
      }
    }
    save_tap("dec.s" + std::to_string(i) + ".out", xo, dmax, B);
    Lc = Ln;
  }
  const int Cl = cfg.up0 >> cfg.n_ups;
  k_conv_post_tanh(xo, dmax, B, Lc, Cl, W("dec.conv_post.weight").buf.f(), 7, 3, 0.01f, wave, st);
  save_tap("dec.wave", wave, N, B);
}

void SynthModel::infer_device(int B, int P, const float* phone, const long long* pitch, const float* nsff0,
                              const long long* sid, const float* nz, const float* ns, float* wave) {
  if (!finalized_) throw Error{kErrState, "synth: finalize() not called after the last weight upload"};
  RVC_CHECK_ARG(B >= 1 && P >= 1, "synth: B and P must be positive");
  ensure_ws(B, P);
  cudaStream_t st = ctx->stream;
  const int H = cfg.hidden, upp = cfg.upp();
  const long long PH = (long long)P * H, N = (long long)P * upp;
  taps_.clear();
  enc_stage(B, P, phone, pitch, sid, nz);
  float* z = flow_stage(B, P, buf("z"), buf("zf"));
  save_tap("flow.z", z, PH, B);
  k_sine_source(nsff0, ns, B, P, upp, cfg.sr, lin_w_, lin_b_, buf("phase"), buf("har"), st);
  save_tap("dec.har", buf("har"), N, B);
  dec_stage(B, P, z, PH, buf("har"), N, (int)N, wave);
}

// Partial synthesis of one chunk (runtime/models/vits.py:2404-2420, :2422-2476,
// :2539-2548): the text encoder over all P frames; the flow from
// flow_head = max(head - 24 - 16, 0); the generator over frames
// [zs, ze) = [max(head - 16, 0), min(P, head + length + 16)) with the harmonic
// source of those frames taken from the full-length source (its phase is the
// full-length phase at each absolute frame, which is what the reference's
// per-segment phase offsets reproduce); output samples [(head - zs) * upp,
// + length * upp) of that segment.
void SynthModel::infer_partial_device(int P, int head, int length, const float* phone, const long long* pitch,
                                      const float* nsff0, const long long* sid, const float* nz, const float* ns,
                                      float* wave) {
  if (!finalized_) throw Error{kErrState, "synth: finalize() not called after the last weight upload"};
  RVC_CHECK_ARG(P >= 1 && head >= 0 && head < P && length >= 1 && head + length <= P,
                "synth: skip_head/return_length out of range");
  ensure_ws(1, P);
  cudaStream_t st = ctx->stream;
  const int H = cfg.hidden, upp = cfg.upp();
  const long long N = (long long)P * upp;
  constexpr int kFlowPad = 24, kDecPad = 16;
  taps_.clear();
  enc_stage(1, P, phone, pitch, sid, nz);
  const int flow_head = std::max(head - kFlowPad - kDecPad, 0);
  float* z = flow_stage(1, P - flow_head, buf("z") + (size_t)flow_head * H, buf("zf") + (size_t)flow_head * H);
  k_sine_source(nsff0, ns, 1, P, upp, cfg.sr, lin_w_, lin_b_, buf("phase"), buf("har"), st);
  const int zs = std::max(head - kDecPad, 0), ze = std::min(P, head + length + kDecPad);
  const int nseg = ze - zs;
  // z rows are absolute frames offset by flow_head; the segment starts at frame zs
  const float* zseg = z + (size_t)(zs - flow_head) * H;
  float* wseg = buf("out_wave");
  dec_stage(1, nseg, zseg, (long long)nseg * H, buf("har") + (size_t)zs * upp, (long long)nseg * upp, nseg * upp,
            wseg);
  RVC_CUDA_TRY(cudaMemcpyAsync(wave, wseg + (size_t)(head - zs) * upp, sizeof(float) * (size_t)length * upp,
                               cudaMemcpyDeviceToDevice, st));
  (void)N;
}

void SynthModel::infer_host(int B, int P, const float* phone, const long long* pitch, const float* nsff0,
                            const long long* sid, const float* nz, const float* ns, float* wave) {
  ensure_ws(B, P);
  cudaStream_t st = ctx->stream;
  const int H = cfg.hidden, upp = cfg.upp();
  auto h2d = [&](const char* n, const void* src, size_t bytes) {
    RVC_CUDA_TRY(cudaMemcpyAsync(ws_.at(n).p, src, bytes, cudaMemcpyHostToDevice, st));
  };
  h2d("in_phone", phone, sizeof(float) * (size_t)B * P * cfg.phone_dim);
  h2d("in_pitch", pitch, sizeof(long long) * (size_t)B * P);
  h2d("in_f0", nsff0, sizeof(float) * (size_t)B * P);
  h2d("in_sid", sid, sizeof(long long) * (size_t)B);
  h2d("in_nz", nz, sizeof(float) * (size_t)B * H * P);
  h2d("in_ns", ns, sizeof(float) * (size_t)B * P * upp);
  infer_device(B, P, buf("in_phone"), ws_.at("in_pitch").as<long long>(), buf("in_f0"),
               ws_.at("in_sid").as<long long>(), buf("in_nz"), buf("in_ns"), buf("out_wave"));
  RVC_CUDA_TRY(cudaMemcpyAsync(wave, buf("out_wave"), sizeof(float) * (size_t)B * P * upp, cudaMemcpyDeviceToHost, st));
}

SynthModel::~SynthModel() {
  // every grouped call returns with its copies finished; nothing is in flight
  for (cudaEvent_t& e : ev_)
    if (e) cudaEventDestroy(e);
  if (up_st_) cudaStreamDestroy(up_st_);
  if (down_st_) cudaStreamDestroy(down_st_);
}

void SynthModel::infer_host_grouped(int B, int G, int P, const float* phone, const long long* pitch,
                                    const float* nsff0, const long long* sid, const float* nz, const float* ns,
                                    float* wave) {
  RVC_CHECK_ARG(B >= 1 && G >= 1 && P >= 1, "synth: B, G and P must be positive");
  if (G >= B) {
    infer_host(B, P, phone, pitch, nsff0, sid, nz, ns, wave);
    return;
  }
  if (!finalized_) throw Error{kErrState, "synth: finalize() not called after the last weight upload"};
  ensure_ws(G, P);
  const int H = cfg.hidden, upp = cfg.upp();
  if (!up_st_) {
    RVC_CUDA_TRY(cudaStreamCreateWithFlags(&up_st_, cudaStreamNonBlocking));
    RVC_CUDA_TRY(cudaStreamCreateWithFlags(&down_st_, cudaStreamNonBlocking));
    for (cudaEvent_t& e : ev_) RVC_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  cudaEvent_t* ev_up = ev_;
  cudaEvent_t* ev_done = ev_ + 2;
  cudaEvent_t* ev_down = ev_ + 4;
  // bytes per chunk of the six inputs and of the waveform
  const size_t per[6] = {sizeof(float) * (size_t)P * cfg.phone_dim, sizeof(long long) * (size_t)P,
                         sizeof(float) * (size_t)P, sizeof(long long), sizeof(float) * (size_t)H * P,
                         sizeof(float) * (size_t)P * upp};
  const size_t per_out = sizeof(float) * (size_t)P * upp;
  const uint8_t* src[6] = {(const uint8_t*)phone, (const uint8_t*)pitch, (const uint8_t*)nsff0,
                           (const uint8_t*)sid,   (const uint8_t*)nz,    (const uint8_t*)ns};
  if (G > g_G_ || P > g_P_) {  // no copy is in flight between calls
    g_G_ = std::max(G, g_G_);
    g_P_ = std::max(P, g_P_);
    const size_t per_max[6] = {sizeof(float) * (size_t)g_P_ * cfg.phone_dim, sizeof(long long) * (size_t)g_P_,
                               sizeof(float) * (size_t)g_P_, sizeof(long long), sizeof(float) * (size_t)H * g_P_,
                               sizeof(float) * (size_t)g_P_ * upp};
    for (int b = 0; b < 2; ++b) {
      for (int i = 0; i < 6; ++i) gin_[b][i] = DevBuf(ctx, per_max[i] * (size_t)g_G_);
      gout_[b] = DevBuf(ctx, sizeof(float) * (size_t)g_P_ * upp * (size_t)g_G_);
    }
    // the new buffers are zero-filled on ctx->stream: copies on the other
    // streams start after that
    RVC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  }
  const int ng = cdiv(B, G);
  auto count = [&](int g) { return std::min(G, B - g * G); };
  auto up = [&](int g) {  // group g's inputs, once group g - 2 has been computed from the same buffers
    const int b = g & 1, nb = count(g);
    if (g >= 2) RVC_CUDA_TRY(cudaStreamWaitEvent(up_st_, ev_done[b], 0));
    for (int i = 0; i < 6; ++i)
      RVC_CUDA_TRY(cudaMemcpyAsync(gin_[b][i].p, src[i] + (size_t)g * G * per[i], (size_t)nb * per[i],
                                   cudaMemcpyHostToDevice, up_st_));
    RVC_CUDA_TRY(cudaEventRecord(ev_up[b], up_st_));
  };
  auto compute = [&](int g) {  // after its inputs arrived and group g - 2's waveforms left
    const int b = g & 1, nb = count(g);
    RVC_CUDA_TRY(cudaStreamWaitEvent(ctx->stream, ev_up[b], 0));
    if (g >= 2) RVC_CUDA_TRY(cudaStreamWaitEvent(ctx->stream, ev_down[b], 0));
    infer_device(nb, P, gin_[b][0].f(), gin_[b][1].as<long long>(), gin_[b][2].f(), gin_[b][3].as<long long>(),
                 gin_[b][4].f(), gin_[b][5].f(), gout_[b].f());
    RVC_CUDA_TRY(cudaEventRecord(ev_done[b], ctx->stream));
  };
  auto down = [&](int g) {
    const int b = g & 1, nb = count(g);
    RVC_CUDA_TRY(cudaStreamWaitEvent(down_st_, ev_done[b], 0));
    RVC_CUDA_TRY(cudaMemcpyAsync(wave + (size_t)g * G * P * upp, gout_[b].p, (size_t)nb * per_out,
                                 cudaMemcpyDeviceToHost, down_st_));
    RVC_CUDA_TRY(cudaEventRecord(ev_down[b], down_st_));
  };
  // group g + 1 is queued before group g's download, so a download from
  // pageable memory (which returns only when done) leaves the next group
  // already queued on the device
  up(0);
  compute(0);
  for (int g = 0; g < ng; ++g) {
    if (g + 1 < ng) {
      up(g + 1);
      compute(g + 1);
    }
    down(g);
  }
  RVC_CUDA_TRY(cudaStreamSynchronize(up_st_));
  RVC_CUDA_TRY(cudaStreamSynchronize(down_st_));
}

}  // namespace rvc
