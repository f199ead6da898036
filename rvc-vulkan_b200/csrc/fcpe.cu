// Device-resident FCPE F0 estimator.
//
// Reference semantics: FCPE.infer (runtime/models/fcpe.py:344-369):
//   _wav2mel (:204-235): pad 432 / max(432, 1024 - T - 432) (reflect when the
//     right pad is shorter than the signal, else zeros), STFT with the periodic
//     Hann window, n_fft 1024, hop 160, no centring; sqrt(|X|^2 + 1e-9) in
//     float64 -> float32; Slaney mel filters (runtime/dsp/mel.py:118-146);
//     log(max(., 1e-5)); F = T / 160 + 1 frames (the last frame repeated when
//     the STFT has one fewer);
//   _input_stack (:237-255): conv k3 128 -> 512, GroupNorm(4), LeakyReLU(0.01),
//     conv k3 512 -> 512;
//   _encoder_layer x 6 (:257-282): x += conv1x1(SiLU(dwconv31(GLU(conv1x1(LN(x))))));
//   _latent (:290-302): LN, weight-normalised linear 512 -> 360, sigmoid;
//   _decode local_argmax (:304-342).
// Layout channels-last [B][F][C]; the convolutions and linears are tensor-core
// implicit GEMMs (BF16x3, fp32 accumulate), the rest SIMT fp32 (float64 for
// the STFT and the GroupNorm statistics).
#include "fcpe.cuh"

#include <cufft.h>

#include <algorithm>
#include <cmath>

namespace rvc {

namespace {

// |rfft(frame * window)|: mag[b][t][k] = sqrt(re^2 + im^2 + 1e-9), k < 513.
// The windowed frames (offset -432, reflect or zero padding) go to
// frames[b][t][1024] (double), a batched cuFFT D2Z gives spec[b][t][513].
__global__ void fcpe_frames_kernel(const float* __restrict__ x, long long T, int nf, bool reflect,
                                   const double* __restrict__ window, double* __restrict__ frames, int B) {
  const long long n_all = (long long)B * nf * 1024;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n_all;
       e += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(e & 1023);
    const long long bt = e >> 10;
    const int b = (int)(bt / nf), t = (int)(bt - (long long)b * nf);
    const float* xb = x + (long long)b * T;
    long long p = (long long)t * 160 + n - 432;
    double v;
    if (reflect) {
      if (p < 0) p = -p;
      if (p >= T) p = 2 * (T - 1) - p;
      v = (double)xb[p];
    } else {
      v = (p >= 0 && p < T) ? (double)xb[p] : 0.0;
    }
    frames[e] = v * window[n];
  }
}

__global__ void fcpe_mag_kernel(const double2* __restrict__ spec, long long n, float* __restrict__ mag) {
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const double2 v = spec[e];
    mag[e] = (float)sqrt(__dadd_rn(__dadd_rn(__dmul_rn(v.x, v.x), __dmul_rn(v.y, v.y)), 1e-9));
  }
}

// mel[b][t][m] = log(max(sum_k basis[m][k] mag[b][min(t, nf - 1)][k], 1e-5)), t < F
__global__ void fcpe_mel_kernel(const float* __restrict__ mag, const float* __restrict__ basis, int nf, int F,
                                float* __restrict__ mel) {
  const int t = blockIdx.x, b = blockIdx.y, m = threadIdx.x;
  const int tt = t < nf ? t : nf - 1;
  const float* mr = mag + ((long long)b * nf + tt) * 513;
  const float* br = basis + (long long)m * 513;
  float s = 0.f;
  for (int k = 0; k < 513; ++k) s = fmaf(br[k], mr[k], s);
  mel[((long long)b * F + t) * 128 + m] = logf(fmaxf(s, 1e-5f));
}

// GroupNorm statistics, pass 1: per (batch, group, row chunk) the float64 sum
// and sum of squares of x[b][t][g*Cg .. (g+1)*Cg).
constexpr int kGnRows = 64;
__global__ void gn_partial_kernel(const float* __restrict__ x, long long x_bs, int T, int C, int G,
                                  double* __restrict__ part, int chunks) {
  const int ch = blockIdx.x, bg = blockIdx.y;
  const int b = bg / G, g = bg % G, Cg = C / G;
  const float* xb = x + (long long)b * x_bs;
  const int r0 = ch * kGnRows, r1 = min(T, r0 + kGnRows);
  double s = 0.0, q = 0.0;
  for (int i = threadIdx.x; i < (r1 - r0) * Cg; i += blockDim.x) {
    const int r = r0 + i / Cg, c = g * Cg + i % Cg;
    const double v = (double)xb[(long long)r * C + c];
    s += v;
    q = fma(v, v, q);
  }
  __shared__ double ss[256], qq[256];
  ss[threadIdx.x] = s;
  qq[threadIdx.x] = q;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) {
      ss[threadIdx.x] += ss[threadIdx.x + o];
      qq[threadIdx.x] += qq[threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    part[((long long)bg * chunks + ch) * 2] = ss[0];
    part[((long long)bg * chunks + ch) * 2 + 1] = qq[0];
  }
}

// pass 2 (one thread per (batch, group)): mean and variance in float32 as the
// reference holds them.
__global__ void gn_stats_kernel(const double* __restrict__ part, int chunks, int BG, double count,
                                float* __restrict__ stats) {
  const int bg = blockIdx.x * blockDim.x + threadIdx.x;
  if (bg >= BG) return;
  double s = 0.0, q = 0.0;
  for (int c = 0; c < chunks; ++c) {
    s += part[((long long)bg * chunks + c) * 2];
    q += part[((long long)bg * chunks + c) * 2 + 1];
  }
  const double mean = s / count;
  const double var = fmax(q / count - mean * mean, 0.0);
  stats[bg * 2] = (float)mean;
  stats[bg * 2 + 1] = (float)var;
}

// y = leaky(((x - mean) / sqrt(var + eps)) * gamma + beta, slope), in place
__global__ void gn_apply_leaky_kernel(float* __restrict__ x, long long x_bs, int T, int C, int G, int B,
                                      const float* __restrict__ stats, const float* __restrict__ gamma,
                                      const float* __restrict__ beta, float eps, float slope) {
  const long long per = (long long)T * C, total = per * B;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(e / per);
    const long long r = e - (long long)b * per;
    const int c = (int)(r % C);
    const int bg = b * G + c / (C / G);
    float* p = x + (long long)b * x_bs + r;
    const float xn = __fdiv_rn(__fsub_rn(*p, stats[bg * 2]), sqrtf(__fadd_rn(stats[bg * 2 + 1], eps)));
    const float v = __fadd_rn(__fmul_rn(xn, gamma[c]), beta[c]);
    *p = v >= 0.f ? v : __fmul_rn(slope, v);
  }
}

__device__ __forceinline__ float sigmoid_ref(float x) {  // runtime/nn.py:520-523
  if (x >= 0.f) return __fdiv_rn(1.f, __fadd_rn(1.f, expf(-x)));
  const float e = expf(x);
  return __fdiv_rn(e, __fadd_rn(1.f, e));
}

// s[b][t][c] = SiLU(b_dw[c] + sum_k GLU(u)[b][t + k - 15][c] w_dw[c][k]),
// GLU(u)[c] = u[c] * sigmoid(u[c + 1024]), zero outside [0, T).
constexpr int kDwT = 64, kDwC = 64;
__global__ void __launch_bounds__(256) glu_dw_silu_kernel(const float* __restrict__ u, long long u_bs, int T,
                                                           const float* __restrict__ w, const float* __restrict__ bias,
                                                           float* __restrict__ s, long long s_bs) {
  __shared__ float g[kDwT + 30][kDwC];
  __shared__ float ws[kDwC][31];
  const int t0 = blockIdx.x * kDwT, c0 = blockIdx.y * kDwC, b = blockIdx.z;
  const float* ub = u + (long long)b * u_bs;
  for (int i = threadIdx.x; i < (kDwT + 30) * kDwC; i += blockDim.x) {
    const int r = i / kDwC, c = i % kDwC, t = t0 + r - 15;
    float v = 0.f;
    if (t >= 0 && t < T) {
      const float a = ub[(long long)t * 2048 + c0 + c], gt = ub[(long long)t * 2048 + 1024 + c0 + c];
      v = __fmul_rn(a, sigmoid_ref(gt));
    }
    g[r][c] = v;
  }
  for (int i = threadIdx.x; i < kDwC * 31; i += blockDim.x) ws[i / 31][i % 31] = w[(long long)(c0 + i / 31) * 31 + i % 31];
  __syncthreads();
  const int c = threadIdx.x % kDwC, ty = threadIdx.x / kDwC;  // 4 row groups of 16
  const float bc = bias[c0 + c];
  for (int j = 0; j < kDwT / 4; ++j) {
    const int r = ty * (kDwT / 4) + j, t = t0 + r;
    if (t >= T) break;
    float d = 0.f;
#pragma unroll
    for (int k = 0; k < 31; ++k) d = fmaf(g[r + k][c], ws[c][k], d);
    d = __fadd_rn(d, bc);
    s[(long long)b * s_bs + (long long)t * 1024 + c0 + c] = __fmul_rn(d, sigmoid_ref(d));
  }
}

// numpy's float32 pairwise sum of 9 values: eight running values, folded, then the ninth
__device__ __forceinline__ float np_sum9(const float* a) {
  const float s = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                            __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
  return __fadd_rn(s, a[8]);
}

// numpy's float32 pairwise sum of n <= 128 values (n >= 8): eight running
// values over the blocks of eight, folded ((0+1)+(2+3))+((4+5)+(6+7)), then
// the remainder in order
__device__ float np_sum_block(const float* a, int n) {
  float r[8];
  for (int j = 0; j < 8; ++j) r[j] = a[j];
  int i = 8;
  for (; i < n - (n % 8); i += 8)
    for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(r[j], a[i + j]);
  float s = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                      __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
  for (; i < n; ++i) s = __fadd_rn(s, a[i]);
  return s;
}
// ... of the 360 bins: numpy halves n > 128 at a multiple of 8:
// 360 -> 176 + 184, 176 -> 88 + 88, 184 -> 88 + 96
__device__ float np_sum360(const float* a) {
  return __fadd_rn(__fadd_rn(np_sum_block(a, 88), np_sum_block(a + 88, 88)),
                   __fadd_rn(np_sum_block(a + 176, 88), np_sum_block(a + 264, 96)));
}

// One warp per frame: latent = sigmoid(logits); decode (runtime/models/fcpe.py:
// 304-342): local argmax (mode 0: the cents-weighted mean of the 9 bins around
// the peak) or argmax (mode 1: over all 360 bins); f0 = 10 * 2^(decoded /
// 1200), 0 when the peak is <= threshold.  `wsum` holds 360 floats per frame
// for mode 1 (cents x latent).
__global__ void fcpe_decode_kernel(const float* __restrict__ logit, long long rows, const float* __restrict__ cents,
                                   float threshold, int mode, float* __restrict__ lat, float* __restrict__ wsum,
                                   float* __restrict__ f0, int32_t* __restrict__ argmax) {
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float* lr = logit + r * 360;
  float* lo = lat + r * 360;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int k = lane; k < 360; k += 32) {
    const float v = sigmoid_ref(lr[k]);
    lo[k] = v;
    if (v > bv || (v == bv && k < bi)) {
      bv = v;
      bi = k;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (mode == 1) {
    float* cw = wsum + r * 360;
    for (int k = lane; k < 360; k += 32) cw[k] = __fmul_rn(cents[k], lo[k]);
    __syncwarp();
    if (lane != 0) return;
    const float dec = __fdiv_rn(np_sum360(cw), np_sum360(lo));
    f0[r] = bv <= threshold ? 0.f : __fmul_rn(10.f, powf(2.f, __fdiv_rn(dec, 1200.f)));
    if (argmax) argmax[r] = bi;
    return;
  }
  __syncwarp();
  if (lane != 0) return;
  float y[9], cy[9];
  for (int j = 0; j < 9; ++j) {
    int idx = j + bi - 4;
    idx = idx < 0 ? 0 : (idx > 359 ? 359 : idx);
    y[j] = lo[idx];
    cy[j] = __fmul_rn(cents[idx], y[j]);
  }
  float den = np_sum9(y);
  if (den == 0.f) den = 1e-30f;
  const float dec = __fdiv_rn(np_sum9(cy), den);
  f0[r] = bv <= threshold ? 0.f : __fmul_rn(10.f, powf(2.f, __fdiv_rn(dec, 1200.f)));
  if (argmax) argmax[r] = bi;
}

int grid_n(long long n) { return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, 148ll * 16)); }

}  // namespace

FcpeModel::FcpeModel(Context* c, int prec) : ctx(c), precision(prec) {
  RVC_CHECK_ARG(prec == 0 || prec == 1, "fcpe: precision must be 0 (tensor cores) or 1 (fp32 SIMT)");
}

FcpeModel::~FcpeModel() {
  if (!fft_plans_.empty()) cudaStreamSynchronize(ctx->stream);  // no transform still in flight
  for (auto& kv : fft_plans_) cufftDestroy((cufftHandle)kv.second);
}

void FcpeModel::set_weight(const std::string& key, const float* host, const std::vector<int64_t>& shape) {
  Tensor t;
  t.shape = shape;
  t.buf = DevBuf(ctx, sizeof(float) * (size_t)std::max<int64_t>(1, t.numel()));
  RVC_CUDA_TRY(cudaMemcpyAsync(t.buf.p, host, sizeof(float) * t.numel(), cudaMemcpyHostToDevice, ctx->stream));
  RVC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  raw_[key] = std::move(t);
  finalized_ = false;
}

const FcpeModel::Tensor& FcpeModel::W(const std::string& key) const {
  auto it = raw_.find(key);
  if (it == raw_.end()) throw Error{kErrState, "fcpe: missing weight '" + key + "'"};
  return it->second;
}

static void expect_numel(const std::string& key, int64_t got, int64_t want) {
  RVC_CHECK_ARG(got == want, "fcpe: weight '" + key + "' holds " + std::to_string(got) + " values, expected " +
                                 std::to_string(want));
}

void FcpeModel::finalize() {
  const bool tc = precision == 0;
  cudaStream_t st = ctx->stream;
  auto chk = [&](const std::string& k, int64_t n) { expect_numel(k, W(k).numel(), n); };
  chk("input_stack.0.weight", (int64_t)kH * kMels * 3);
  chk("input_stack.3.weight", (int64_t)kH * kH * 3);
  for (const char* k : {"input_stack.0.bias", "input_stack.1.weight", "input_stack.1.bias", "input_stack.3.bias",
                        "norm.weight", "norm.bias"})
    chk(k, kH);
  in0_ = ConvLayer();
  in0_.pad_l = in0_.pad_r = 1;
  in0_.build(ctx, LayerKind::kConv, W("input_stack.0.weight").buf.f(), W("input_stack.0.bias").buf.f(), kH, kMels, 3,
             tc);
  in3_ = ConvLayer();
  in3_.pad_l = in3_.pad_r = 1;
  in3_.build(ctx, LayerKind::kConv, W("input_stack.3.weight").buf.f(), W("input_stack.3.bias").buf.f(), kH, kH, 3, tc);
  for (int l = 0; l < kLayers; ++l) {
    const std::string p = "net.encoder_layers." + std::to_string(l) + ".conformer.net";
    chk(p + ".0.weight", kH);
    chk(p + ".0.bias", kH);
    chk(p + ".2.weight", (int64_t)kFF * kH);
    chk(p + ".2.bias", kFF);
    chk(p + ".4.conv.weight", (int64_t)kDW * kDWK);
    chk(p + ".4.conv.bias", kDW);
    chk(p + ".6.weight", (int64_t)kH * kDW);
    chk(p + ".6.bias", kH);
    up_[l] = ConvLayer();
    up_[l].build(ctx, LayerKind::kConv, W(p + ".2.weight").buf.f(), W(p + ".2.bias").buf.f(), kFF, kH, 1, tc);
    down_[l] = ConvLayer();
    down_[l].build(ctx, LayerKind::kConv, W(p + ".6.weight").buf.f(), W(p + ".6.bias").buf.f(), kH, kDW, 1, tc);
  }
  chk("output_proj.weight_v", (int64_t)kOut * kH);
  chk("output_proj.weight_g", kOut);
  chk("output_proj.bias", kOut);
  chk("cent_table", kOut);
  wproj_ = DevBuf(ctx, sizeof(float) * (size_t)kOut * kH);
  k_fold_weight_norm(W("output_proj.weight_v").buf.f(), W("output_proj.weight_g").buf.f(), wproj_.f(), kOut, kH, st);
  proj_ = ConvLayer();
  proj_.build(ctx, LayerKind::kConv, wproj_.f(), W("output_proj.bias").buf.f(), kOut, kH, 1, tc);
  // front-end tables: periodic Hann (torch.hann_window), Slaney
  // mel filters with area normalisation (runtime/dsp/mel.py:118-146)
  {
    const double pi = 3.14159265358979323846;
    std::vector<double> win(kNFFT);
    for (int k = 0; k < kNFFT; ++k) win[k] = 0.5 - 0.5 * std::cos(2.0 * pi * k / kNFFT);
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    const double logstep = std::log(6.4) / 27.0;
    auto hz_to_mel = [&](double f) { return f >= min_log_hz ? min_log_mel + std::log(f / min_log_hz) / logstep : f / f_sp; };
    auto mel_to_hz = [&](double m) { return m >= min_log_mel ? min_log_hz * std::exp(logstep * (m - min_log_mel)) : f_sp * m; };
    const double mlo = hz_to_mel(0.0), mhi = hz_to_mel(8000.0);
    std::vector<double> mel_f(kMels + 2), fftf(kBins);
    const double step = (mhi - mlo) / (kMels + 1);  // numpy.linspace: i * step + start, exact end point
    for (int i = 0; i < kMels + 2; ++i) mel_f[i] = mel_to_hz(i == kMels + 1 ? mhi : i * step + mlo);
    for (int k = 0; k < kBins; ++k) fftf[k] = 8000.0 * k / (kBins - 1);
    std::vector<float> basis((size_t)kMels * kBins);
    for (int i = 0; i < kMels; ++i) {
      const double lo_d = mel_f[i + 1] - mel_f[i], hi_d = mel_f[i + 2] - mel_f[i + 1];
      const double enorm = 2.0 / (mel_f[i + 2] - mel_f[i]);
      for (int k = 0; k < kBins; ++k) {
        const double lower = -(mel_f[i] - fftf[k]) / lo_d, upper = (mel_f[i + 2] - fftf[k]) / hi_d;
        basis[(size_t)i * kBins + k] = (float)(std::max(0.0, std::min(lower, upper)) * enorm);
      }
    }
    window_ = DevBuf(ctx, sizeof(double) * win.size());
    basis_ = DevBuf(ctx, sizeof(float) * basis.size());
    RVC_CUDA_TRY(cudaMemcpyAsync(window_.p, win.data(), window_.bytes, cudaMemcpyHostToDevice, st));
    RVC_CUDA_TRY(cudaMemcpyAsync(basis_.p, basis.data(), basis_.bytes, cudaMemcpyHostToDevice, st));
  }
  RVC_CUDA_TRY(cudaStreamSynchronize(st));
  finalized_ = true;
}

void FcpeModel::ensure_ws(int B, int64_t T) {
  if (B <= ws_B && T <= ws_T) return;
  B = std::max(B, ws_B);
  T = std::max(T, ws_T);
  ws_.clear();
  const int64_t F = frames(T);
  auto add = [&](const char* n, long long per) {
    ws_.emplace(n, DevBuf(ctx, sizeof(float) * (size_t)B * std::max<long long>(1, per)));
  };
  add("x_in", T);
  add("mag", F * kBins);
  add("mel", F * kMels);
  add("h0", F * kH);
  add("xa", F * kH);
  add("xb", F * kH);
  add("xn", F * kH);
  add("u", F * kFF);
  add("s", F * kDW);
  add("logit", F * kOut);
  add("lat", F * kOut);
  add("wsum", F * kOut);
  add("f0", F);
  add("am", F);
  add("gn", 2 * kGroups * ((F + kGnRows - 1) / kGnRows) * 2 + 2 * kGroups);  // doubles in float units
  // STFT frames (nf <= F) as doubles and their D2Z spectra
  ws_.emplace("frames", DevBuf(ctx, sizeof(double) * (size_t)B * F * kNFFT));
  ws_.emplace("spec", DevBuf(ctx, 2 * sizeof(double) * (size_t)B * F * kBins));
  ws_B = B;
  ws_T = T;
}

void FcpeModel::save_tap(const std::string& name, const float* d, int64_t n) {
  if (!keep_taps) return;
  std::vector<float> h((size_t)n);
  RVC_CUDA_TRY(cudaMemcpyAsync(h.data(), d, sizeof(float) * (size_t)n, cudaMemcpyDeviceToHost, ctx->stream));
  RVC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  taps_[name] = std::move(h);
}

bool FcpeModel::tap(const std::string& name, float* host, int64_t n) {
  auto it = taps_.find(name);
  if (it == taps_.end() || (int64_t)it->second.size() < n) return false;
  std::copy(it->second.begin(), it->second.begin() + n, host);
  return true;
}

void FcpeModel::infer_device(int B, int64_t T, const float* x, float threshold, float* f0, int32_t* argmax,
                             int decoder_mode) {
  RVC_CHECK_ARG(decoder_mode == 0 || decoder_mode == 1, "fcpe: decoder_mode must be 0 (local_argmax) or 1 (argmax)");
  if (!finalized_) throw Error{kErrState, "fcpe: finalize() not called after the last weight upload"};
  RVC_CHECK_ARG(B >= 1 && T >= 1, "fcpe: need B >= 1 clips of T >= 1 samples");
  RVC_CHECK_ARG(T <= (1ll << 30), "fcpe: input too long");
  ensure_ws(B, T);
  taps_.clear();
  cudaStream_t st = ctx->stream;
  const int F = (int)frames(T);
  const int64_t pl = (kNFFT - kHop) / 2, pr = std::max<int64_t>((kNFFT - kHop + 1) / 2, kNFFT - T - pl);
  const bool reflect = pr < T;
  const int nf = (int)(1 + (T + pl + pr - kNFFT) / kHop);
  // ---------------- front end
  {
    const long long nfr = (long long)B * nf;
    auto it = fft_plans_.find(nfr);
    if (it == fft_plans_.end()) {
      cufftHandle h = 0;
      int n = kNFFT;
      if (cufftPlanMany(&h, 1, &n, nullptr, 1, kNFFT, nullptr, 1, kBins, CUFFT_D2Z, (int)nfr) != CUFFT_SUCCESS)
        throw Error{kErrCuda, "fcpe: cuFFT plan failed"};
      it = fft_plans_.emplace(nfr, (int)h).first;
    }
    const cufftHandle h = (cufftHandle)it->second;
    double* fr = reinterpret_cast<double*>(ws_.at("frames").p);
    fcpe_frames_kernel<<<(unsigned)std::min<long long>((nfr * 1024 + 255) / 256, 148ll * 16), 256, 0, st>>>(
        x, T, nf, reflect, (const double*)window_.p, fr, B);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
    if (cufftSetStream(h, st) != CUFFT_SUCCESS ||
        cufftExecD2Z(h, (cufftDoubleReal*)fr, (cufftDoubleComplex*)ws_.at("spec").p) != CUFFT_SUCCESS)
      throw Error{kErrCuda, "fcpe: cuFFT transform failed"};
    fcpe_mag_kernel<<<(unsigned)std::min<long long>((nfr * kBins + 255) / 256, 148ll * 16), 256, 0, st>>>(
        (const double2*)ws_.at("spec").p, nfr * kBins, buf("mag"));
    note_launch();
  }
  fcpe_mel_kernel<<<dim3(F, B), 128, 0, st>>>(buf("mag"), basis_.f(), nf, F, buf("mel"));
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
  save_tap("mel", buf("mel"), (int64_t)B * F * kMels);
  // ---------------- input stack
  const long long rows = (long long)B * F;
  {
    ConvIO io;
    io.x = buf("mel"); io.x_ld = kMels; io.x_bs = (long long)F * kMels; io.T_in = F;
    io.y = buf("h0"); io.y_ld = kH; io.y_bs = (long long)F * kH;
    io.B = B;
    run_conv(in0_, io);
    const int chunks = (F + kGnRows - 1) / kGnRows;
    double* part = (double*)buf("gn");
    float* stats = (float*)(part + (size_t)B * kGroups * chunks * 2);
    gn_partial_kernel<<<dim3(chunks, B * kGroups), 256, 0, st>>>(buf("h0"), (long long)F * kH, F, kH, kGroups, part,
                                                                 chunks);
    note_launch();
    gn_stats_kernel<<<(B * kGroups + 63) / 64, 64, 0, st>>>(part, chunks, B * kGroups, (double)F * (kH / kGroups),
                                                             stats);
    note_launch();
    gn_apply_leaky_kernel<<<grid_n(rows * kH), 256, 0, st>>>(buf("h0"), (long long)F * kH, F, kH, kGroups, B, stats,
                                                              W("input_stack.1.weight").buf.f(),
                                                              W("input_stack.1.bias").buf.f(), 1e-5f, 0.01f);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
    ConvIO io3 = io;
    io3.x = buf("h0"); io3.x_ld = kH; io3.x_bs = (long long)F * kH;
    io3.y = buf("xa");
    run_conv(in3_, io3);
  }
  save_tap("stack", buf("xa"), rows * kH);
  // ---------------- conformer conv layers
  auto gemm_io = [&](const float* xin, int ld_in, float* y, int ld_out) {
    ConvIO io;
    io.x = xin; io.x_ld = ld_in; io.x_bs = rows * ld_in; io.T_in = (int)rows;
    io.y = y; io.y_ld = ld_out; io.y_bs = rows * ld_out;
    io.B = 1;
    return io;
  };
  float* xc = buf("xa");
  float* xo = buf("xb");
  for (int l = 0; l < kLayers; ++l) {
    const std::string p = "net.encoder_layers." + std::to_string(l) + ".conformer.net";
    k_layernorm(xc, kH, nullptr, 0, rows, kH, W(p + ".0.weight").buf.f(), W(p + ".0.bias").buf.f(), 1e-5f, buf("xn"),
                kH, st);
    run_conv(up_[l], gemm_io(buf("xn"), kH, buf("u"), kFF));
    glu_dw_silu_kernel<<<dim3((F + kDwT - 1) / kDwT, kDW / kDwC, B), 256, 0, st>>>(
        buf("u"), (long long)F * kFF, F, W(p + ".4.conv.weight").buf.f(), W(p + ".4.conv.bias").buf.f(), buf("s"),
        (long long)F * kDW);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
    ConvIO dn = gemm_io(buf("s"), kDW, xo, kH);
    dn.res = xc; dn.res_ld = kH; dn.res_bs = rows * kH;
    run_conv(down_[l], dn);
    std::swap(xc, xo);
    save_tap("layer" + std::to_string(l), xc, rows * kH);
  }
  // ---------------- output norm, projection, sigmoid, decode
  k_layernorm(xc, kH, nullptr, 0, rows, kH, W("norm.weight").buf.f(), W("norm.bias").buf.f(), 1e-5f, buf("xn"), kH,
              st);
  run_conv(proj_, gemm_io(buf("xn"), kH, buf("logit"), kOut));
  fcpe_decode_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(buf("logit"), rows, W("cent_table").buf.f(),
                                                                  threshold, decoder_mode, buf("lat"),
                                                                  decoder_mode == 1 ? buf("wsum") : nullptr, f0,
                                                                  argmax);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
  save_tap("latent", buf("lat"), rows * kOut);
}

void FcpeModel::infer_host(int B, int64_t T, const float* x, float threshold, float* f0, int32_t* argmax,
                           int decoder_mode) {
  RVC_CHECK_ARG(B >= 1 && T >= 1, "fcpe: need B >= 1 clips of T >= 1 samples");
  ensure_ws(B, T);
  cudaStream_t st = ctx->stream;
  const int64_t F = frames(T);
  RVC_CUDA_TRY(cudaMemcpyAsync(buf("x_in"), x, sizeof(float) * (size_t)B * T, cudaMemcpyHostToDevice, st));
  infer_device(B, T, buf("x_in"), threshold, buf("f0"), argmax ? (int32_t*)buf("am") : nullptr, decoder_mode);
  RVC_CUDA_TRY(cudaMemcpyAsync(f0, buf("f0"), sizeof(float) * (size_t)B * F, cudaMemcpyDeviceToHost, st));
  if (argmax)
    RVC_CUDA_TRY(cudaMemcpyAsync(argmax, buf("am"), sizeof(int32_t) * (size_t)B * F, cudaMemcpyDeviceToHost, st));
}

}  // namespace rvc
