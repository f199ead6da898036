// Device-resident RMVPE F0 estimator (RMVPE.infer_from_audio inference).
#pragma once

#include "context.cuh"

#include <map>
#include <string>
#include <unordered_map>
#include <vector>

namespace rvc {

// One stride-1 3x3 / 1x1 convolution (or the 3x3, stride-2 transposed
// convolution of the decoder) over channels-last images, fp32 SIMT.
struct Conv2dW {
  int C_in = 0, C_out = 0, taps = 0;  // taps: 9 (3x3) or 1
  bool transposed = false;
  DevBuf w;                           // [taps][C_in][C_out]
  DevBuf bias, scale, shift;          // optional [C_out]
};

struct RmvpeTensor {
  DevBuf buf;
  std::vector<int64_t> shape;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

class RmvpeModel {
 public:
  static constexpr int kNFFT = 1024, kHop = 160, kBins = 513, kMels = 128, kHidden = 256, kClasses = 360;

  explicit RmvpeModel(Context* ctx);
  ~RmvpeModel();
  RmvpeModel(const RmvpeModel&) = delete;
  RmvpeModel& operator=(const RmvpeModel&) = delete;
  void set_weight(const std::string& key, const float* host, const std::vector<int64_t>& shape);
  void finalize();
  static int64_t frames(int64_t T) { return 1 + T / kHop; }
  // Device pointers, asynchronous: x [B][T] -> f0 [B][frames(T)] (Hz) and,
  // when argmax != nullptr, the salience argmax per frame [B][frames(T)].
  void infer_device(int B, int64_t T, const float* x, float thred, float* f0, int32_t* argmax);
  void infer_host(int B, int64_t T, const float* x, float thred, float* f0, int32_t* argmax);
  bool tap(const std::string& name, float* host, int64_t n);
  bool keep_taps = false;
  Context* ctx;

 private:
  const RmvpeTensor& W(const std::string& key) const;
  void bn_fold(const std::string& p, DevBuf& scale, DevBuf& shift, int C);
  void build_block(const std::string& p, int cin, int cout);
  void ensure_ws(int B, int64_t T);
  void save_tap(const std::string& name, const float* d, int64_t n);
  // conv launch helpers (rmvpe.cu)
  void conv(const Conv2dW& L, int B, const float* x, long long x_bs, int H, int Wd, int ldi, float* y, long long y_bs,
            long long oh_s, int ow_s, int oc_s, bool relu, const float* res, long long res_bs, int ldr,
            bool sigmoid = false);
  void block(const std::string& p, int B, const float* x, long long x_bs, int H, int Wd, int ldi, float* out,
             long long out_bs, int ldo, float* tmp, long long tmp_bs);

  bool finalized_ = false;
  std::unordered_map<std::string, RmvpeTensor> raw_;
  std::map<std::string, Conv2dW> convs_;  // by checkpoint prefix
  DevBuf in_scale_, in_shift_;            // unet.encoder.bn
  DevBuf mel_basis_, window_;             // front end tables
  std::map<long long, int> fft_plans_;    // cuFFT D2Z plans (n = 1024) by frame count
  DevBuf w_hh_, b_hh_;                    // GRU recurrent weights [2][768][256], biases [2][768]
  int ws_B = 0;
  int64_t ws_T = 0;
  std::map<std::string, DevBuf> ws_;
  float* buf(const char* n) { return ws_.at(n).f(); }
  std::map<std::string, std::vector<float>> taps_;
};

}  // namespace rvc
