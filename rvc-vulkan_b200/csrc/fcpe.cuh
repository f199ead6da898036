// Device-resident FCPE F0 estimator (CFNaiveMelPE, conv-only), the model of
// runtime/models/fcpe.py:165-369.
#pragma once

#include "layer.cuh"

#include <map>
#include <string>
#include <unordered_map>
#include <vector>

namespace rvc {

class FcpeModel {
 public:
  static constexpr int kMels = 128, kBins = 513, kNFFT = 1024, kHop = 160, kH = 512, kFF = 2048, kDW = 1024;
  static constexpr int kDWK = 31, kLayers = 6, kOut = 360, kGroups = 4;

  FcpeModel(Context* ctx, int precision);
  ~FcpeModel();
  FcpeModel(const FcpeModel&) = delete;
  FcpeModel& operator=(const FcpeModel&) = delete;
  // Checkpoint tensors under the reference's keys (FCPE.W), incl. cent_table.
  void set_weight(const std::string& key, const float* host, const std::vector<int64_t>& shape);
  void finalize();
  static int64_t frames(int64_t T) { return T / kHop + 1; }
  // Device pointers, asynchronous on ctx->stream: x [B][T] -> f0 [B][F] Hz and,
  // when argmax != nullptr, the latent argmax [B][F].
  // decoder_mode: 0 local_argmax (the pipeline's), 1 argmax (runtime/models/fcpe.py:304-333)
  void infer_device(int B, int64_t T, const float* x, float threshold, float* f0, int32_t* argmax,
                    int decoder_mode = 0);
  void infer_host(int B, int64_t T, const float* x, float threshold, float* f0, int32_t* argmax,
                  int decoder_mode = 0);
  bool tap(const std::string& name, float* host, int64_t n);
  bool keep_taps = false;
  Context* ctx;
  int precision;  // 0 BF16x3 tensor cores, 1 fp32 SIMT

 private:
  struct Tensor {
    DevBuf buf;
    std::vector<int64_t> shape;
    int64_t numel() const {
      int64_t n = 1;
      for (auto s : shape) n *= s;
      return n;
    }
  };
  const Tensor& W(const std::string& key) const;
  void ensure_ws(int B, int64_t T);
  void save_tap(const std::string& name, const float* d, int64_t n);
  void run_conv(const ConvLayer& L, const ConvIO& io) { L.run(ctx, io, precision == 1); }
  bool finalized_ = false;
  std::unordered_map<std::string, Tensor> raw_;
  ConvLayer in0_, in3_, up_[kLayers], down_[kLayers], proj_;
  DevBuf window_, basis_, wproj_;
  std::map<long long, int> fft_plans_;  // cuFFT D2Z plans (n = 1024) by frame count
  int ws_B = 0;
  int64_t ws_T = 0;
  std::map<std::string, DevBuf> ws_;
  float* buf(const char* n) { return ws_.at(n).f(); }
  std::map<std::string, std::vector<float>> taps_;
};

}  // namespace rvc
