// Device-resident HuBERT-base encoder (HubertEncoder.encode inference).
#pragma once

#include "layer.cuh"

#include <map>
#include <string>
#include <unordered_map>
#include <vector>

namespace rvc {

struct HubertTensor {
  DevBuf buf;
  std::vector<int64_t> shape;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

class HubertModel {
 public:
  static constexpr int kConvC = 512, kD = 768, kHeads = 12, kHeadD = 64, kFF = 3072, kLayers = 12;
  static constexpr int kPosK = 128, kPosGroups = 16, kFinal = 256;

  HubertModel(Context* ctx, int precision);
  void set_weight(const std::string& key, const float* host, const std::vector<int64_t>& shape);
  void finalize();
  // Frames produced for T input samples (0 when T is too short for the conv stack).
  static int64_t out_len(int64_t T);
  // Device pointers; asynchronous on ctx->stream.  x [B][T] -> out [B][L][768] (version 2)
  // or [B][L][256] (version 1: layer 9 through final_proj).
  void encode_device(int B, int64_t T, const float* x, int version, float* out);
  void encode_host(int B, int64_t T, const float* x, int version, float* out);
  bool tap(const std::string& name, float* host, int64_t n);
  bool keep_taps = false;
  Context* ctx;
  int precision;  // 0 BF16x3 tensor cores, 1 fp32 SIMT

 private:
  const HubertTensor& W(const std::string& key) const;
  void ensure_ws(int B, int64_t T);
  void save_tap(const std::string& name, const float* d, int64_t rows, int C, int ld, long long bs, int B);
  void run_conv(const ConvLayer& L, const ConvIO& io);
  bool finalized_ = false;
  std::unordered_map<std::string, HubertTensor> raw_;
  // conv feature extractor: layer 0 is a one-channel conv (SIMT), layers 1..6
  // run on the stride-2 view [T/2][1024]: convA takes taps 0,1 as 1024 input
  // channels, convB tap 2 (kernel-3 layers only) from the next view row.
  DevBuf conv0_w_;
  ConvLayer convA_[7], convB_[7];
  int conv_k_[7] = {10, 3, 3, 3, 3, 2, 2};
  ConvLayer proj_, pos_, qkv_[kLayers], o_[kLayers], ff1_[kLayers], ff2_[kLayers], final_;
  // workspace
  int ws_B = 0;
  int64_t ws_T = 0;
  std::map<std::string, DevBuf> ws_;
  float* buf(const char* n) { return ws_.at(n).f(); }
  std::map<std::string, std::vector<float>> taps_;
};

}  // namespace rvc
