// SIMT kernels for the non-GEMM parts of the hot path (norms, attention,
// gates, the NSF source, weight preparation).  Host launchers; all run on the
// given stream.  Activations are channels-last [B][T][C] unless noted.
#pragma once

#include "common.cuh"

namespace rvc {

// ---- layout
void k_nct_to_ntc(const float* x, float* y, int B, int C, int T, int y_ld, cudaStream_t st);
void k_ntc_to_nct(const float* x, int x_ld, float* y, int B, int C, int T, cudaStream_t st);

// ---- norms / softmax / elementwise
// y[r] = LN(x[r] (+ res[r])) ; rows of C with lds.
void k_layernorm(const float* x, int x_ld, const float* res, int res_ld, long long rows, int C,
                 const float* gamma, const float* beta, float eps, float* y, int y_ld, cudaStream_t st);
void k_softmax_rows(const float* x, float* y, long long rows, int C, cudaStream_t st);
void k_elementwise(int op, const float* a, const float* b, long long n, float alpha, float* y, cudaStream_t st);
void k_embedding(const long long* ids, long long n, const float* table, int V, int E, float* y, cudaStream_t st);
void k_gating_nct(const float* x, const float* g, int B, int H, int T, float* y, cudaStream_t st);
void k_im2col1d(const float* x, int B, int C, int T, int K, int stride, int pad_l, int dil, int oL, float* cols,
                cudaStream_t st);

// ---- weight preparation
// out[r, :] = v[r, :] * (g[r] / max(||v[r, :]||, 1e-12)), rows of `inner` (weight_norm dim 0).
void k_fold_weight_norm(const float* v, const float* g, float* out, int rows, int inner, cudaStream_t st);
// Wg[j][i][o] = layout==0 ? W[o][i][tap_k[j]] : W[i][o][tap_k[j]]   (conv [O,I,K] / convT [I,O,K])
void k_gather_taps(const float* W, float* Wg, int O, int I, int K, int layout, const int* tap_k_dev, int ntaps,
                   cudaStream_t st);
// y[b][o] = sum_i W[o][i] x[b][i] + bias[o]  (1x1 conv on one frame)
void k_gemv_rows(const float* W, const float* bias, const float* x, int B, int O, int I, float* y,
                 cudaStream_t st);

// ---- synthesizer pieces
// x = leaky(((lin + E[pitch]) * scale), 0.1), in place on lin [B*P, H]
void k_enc_embed_finish(float* lin, const long long* pitch, const float* E, long long rows, int H, float scale,
                        cudaStream_t st);
// T5 relative attention, head-interleaved channels-last qkv [B,P,3*H*kc] -> y [B,P,H*kc]
void k_rel_attention(const float* qkv, int qkv_ld, int q_off, int k_off, int v_off, const float* emb_k,
                     const float* emb_v, int B, int heads, int kc, int P, int window, float* scratch, float* y,
                     int y_ld, cudaStream_t st);
// z[b,t,c] = m + exp(logs) * nz[b,c,t] * 0.66666   (stats [B,P,2H])
void k_zp(const float* stats, const float* nz, int B, int P, int H, float* z, cudaStream_t st);
void k_flip_channels(const float* x, float* y, long long rows, int C, cudaStream_t st);
// acts = tanh(xin[:, :H]) * sigmoid(xin[:, H:])   (g already added by the conv epilogue)
void k_gate_rows(const float* xin, long long rows, int H, float* acts, cudaStream_t st);
// i<last: h += rs[:, :H]; skip = (first ? 0 : skip) + rs[:, H:] ; last: skip += rs
void k_wn_update(float* h, float* skip, const float* rs, long long rows, int H, int first, int last,
                 cudaStream_t st);
// NSF sine source: har[b, n], n < P*upp
void k_sine_source(const float* f0, const float* ns, int B, int P, int upp, int sr, float lin_w, float lin_b,
                   float* phase_scratch, float* har, cudaStream_t st);
// NSF noise conv (conv1d with one input channel): y[b,t,co] = sum_k har[b, t*str - pad + k] * w[co][k] + bias[co]
// for t < T_out, written to y with batch stride y_bs and row stride C.
void k_noise_conv(const float* har, long long har_bs, int har_len, const float* w, const float* bias, int C, int nk,
                  int str, int pad, int B, int T_out, float* y, long long y_bs, cudaStream_t st);
// y[b,t] = tanh(sum_k sum_c leaky(x[b,t+k-pad,c],slope) * w[c][k])   (conv_post, C_out = 1, no bias)
void k_conv_post_tanh(const float* x, long long x_bs, int B, int T, int C, const float* w, int K, int pad, float slope,
                      float* y, cudaStream_t st);

// ---- HuBERT pieces
// Per-channel GroupNorm over time of channels-last x [B][T][C] (in place), then
// GELU; scratch holds groupnorm_chan_scratch_floats(B, C) floats.
void k_groupnorm_chan_gelu(float* x, long long x_bs, int T, int C, int B, const float* gamma, const float* beta,
                           float eps, float* scratch, cudaStream_t st);
size_t groupnorm_chan_scratch_floats(int B, int C);
// out[r][k] = g[k] * v[r][k] / ||v[:, k]||  for v viewed as [rows][K] (weight_norm dim=2)
void k_fold_weight_norm_dim2(const float* v, const float* g, float* out, long long rows, int K, cudaStream_t st);
// y[o][t*I + i] = W[o][i][j0 + t], t < nt  (taps folded into input channels)
void k_taps_to_channels(const float* W, int O, int I, int K, int j0, int nt, float* y, cudaStream_t st);
// Plain softmax(q k^T / q_div) v attention over head-interleaved channels-last rows.
void k_attention(const float* qkv, int qkv_ld, int q_off, int k_off, int v_off, int B, int heads, int D, int P,
                 float q_div, float* y, int y_ld, cudaStream_t st);

// ---- tensor-core attention (tc_attn.cu)
struct Context;
// Same contract as k_rel_attention (window >= 0, q / q_div) / k_attention
// (window < 0) on the tensor cores (BF16x3); false when the head size is not
// served (D % 16 != 0 or D > 96), the caller then runs the SIMT kernel.
bool k_attention_tc(Context* ctx, const float* qkv, int ld, int q_off, int k_off, int v_off, const float* emb_k,
                    const float* emb_v, int B, int heads, int D, int P, int window, float q_div, float* y, int y_ld);

// ---- pipeline signal processing (dsp.cu); device pointers unless noted
// scipy.signal.filtfilt(b, a, x) with padtype 'odd' (b, a host arrays), float64
void dsp_filtfilt(Context* ctx, const double* b, int nb, const double* a, int na, const double* x_dev, long long n,
                  bool ext_f32, double* y_dev);
// method 0: fft (factor = n_in sr_out / (sr_in n_out)), 1: linear, 2: sinc; y float32 [n_out]
void dsp_resample(Context* ctx, const double* x, long long n_in, long long n_out, int method, double factor,
                  float* y);
void dsp_f0_autocorr(Context* ctx, const double* x, long long n, int hop, int win, int lag_min, int lag_max,
                     const double* hann, double sr, double thr, float* f0, long long n_frames);
void dsp_f32_to_f64(Context* ctx, const float* x, long long n, double* y);
// first argmin of the 160-sample absolute sums around t = step, 2 step, ... (< n); -1 = empty window
long long dsp_split_points(Context* ctx, const double* audio, long long n, int window, long long t_query,
                           long long step, long long* out_dev);
void dsp_interp_time(Context* ctx, const float* x, long long L, int D, double scale, float* y, long long Lo);
void dsp_protect(Context* ctx, const float* feats, const float* feats0, const float* pitchf, long long P, int D,
                 float protect, float* out);
void dsp_change_rms(Context* ctx, const float* d1, long long n1, int sr1, const float* d2, long long n2, int sr2,
                    double rate, float* out);
void dsp_to_int16(Context* ctx, const float* x, long long n, short* y);

// Tier-1 2-D convolution (torch conv2d semantics, zero padding) and RMSNorm (ops2d.cu).
void k_conv2d(const float* x, int B, int C, int H, int W, const float* w, int O, int KH, int KW, const float* bias,
              int sh, int sw, int ph, int pw, float* y, cudaStream_t st);
void k_rmsnorm(const float* x, long long rows, int C, const float* g, float eps, float* y, cudaStream_t st);

}  // namespace rvc
