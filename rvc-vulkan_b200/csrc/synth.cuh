// Device-resident VITS synthesizer (SynthesizerTrnMs768NSFsid inference).
#pragma once

#include "layer.cuh"

#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace rvc {

struct SynthConfig {
  int sr = 40000, hidden = 192, filter = 768, heads = 2, layers = 6, kc = 96, window = 10;
  int gin = 256, up0 = 512, n_ups = 4;
  std::vector<int> rates, kernels;
  int phone_dim = 768, n_spk = 1;
  int precision = 0;  // 0 BF16x3 tensor cores, 1 SIMT fp32
  int upp() const {
    int u = 1;
    for (int r : rates) u *= r;
    return u;
  }
};

struct RawTensor {
  DevBuf buf;
  std::vector<int64_t> shape;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

class SynthModel {
 public:
  SynthModel(Context* ctx, const SynthConfig& cfg);
  void set_weight(const std::string& key, const float* host, const std::vector<int64_t>& shape);
  void finalize();
  // Device pointers; asynchronous on ctx->stream.
  void infer_device(int B, int P, const float* phone, const long long* pitch, const float* nsff0,
                    const long long* sid, const float* nz, const float* ns, float* wave);
  void infer_host(int B, int P, const float* phone, const long long* pitch, const float* nsff0,
                  const long long* sid, const float* nz, const float* ns, float* wave);
  // Host buffers, B chunks in groups of G (each group exactly as infer_host
  // of those chunks): a group's inputs go up on one copy stream and its
  // waveforms come down on another while the neighbouring groups compute on
  // ctx->stream (double-buffered device inputs and outputs, ordered by
  // events).  Returns with every copy finished.
  void infer_host_grouped(int B, int G, int P, const float* phone, const long long* pitch, const float* nsff0,
                          const long long* sid, const float* nz, const float* ns, float* wave);
  ~SynthModel();
  // Partial synthesis of one chunk: wave [length * upp] for frames [head, head + length).
  void infer_partial_device(int P, int head, int length, const float* phone, const long long* pitch,
                            const float* nsff0, const long long* sid, const float* nz, const float* ns,
                            float* wave);
  bool tap(const std::string& name, float* host, int64_t n);
  int keep_taps = 0;  // 0 off, 1 every chunk, 2 + c chunk c only
  Context* ctx;
  SynthConfig cfg;

 private:
  const RawTensor& W(const std::string& key) const;
  DevBuf fold(const std::string& base);  // weight_v/weight_g -> folded
  void ensure_ws(int B, int P);
  // records B chunks of `per_chunk` floats each (chunk stride per_chunk) from d
  void save_tap(const std::string& name, const float* d, int64_t per_chunk, int B);
  void run_conv(const ConvLayer& L, const ConvIO& io);
  void enc_stage(int B, int P, const float* phone, const long long* pitch, const long long* sid, const float* nz);
  float* flow_stage(int B, int P, float* z, float* zf);
  void dec_stage(int B, int P, const float* z, long long z_bs, const float* har, long long har_bs, int har_len,
                 float* wave);
  bool finalized_ = false;
  std::unordered_map<std::string, RawTensor> raw_;
  // enc
  ConvLayer emb_phone_, qkv_[8], o_[8], ffn1_[8], ffn2_[8], proj_;
  // flow
  ConvLayer pre_[4], in_[4][3], rs_[4][3], post_[4];
  DevBuf flow_cond_w_[4], flow_cond_b_[4];
  // dec
  ConvLayer conv_pre_, ups_[8], rb1_[8][3][3], rb2_[8][3][3];
  int noise_k_[8] = {0}, noise_s_[8] = {0};
  float lin_w_ = 0.f, lin_b_ = 0.f;  // dec.m_source.l_linear (1x1)
  // grouped host path: copy streams, events (inputs up [2], group computed
  // [2], waveforms down [2]) and the double-buffered group inputs / outputs
  cudaStream_t up_st_ = nullptr, down_st_ = nullptr;
  cudaEvent_t ev_[6] = {};
  DevBuf gin_[2][6], gout_[2];
  int g_G_ = 0, g_P_ = 0;
  // workspace
  int ws_B = 0, ws_P = 0;
  std::map<std::string, DevBuf> ws_;
  float* buf(const char* n) { return ws_.at(n).f(); }
  std::map<std::string, std::vector<float>> taps_;
};

}  // namespace rvc
