// Device-resident feature index: brute-force L2 top-k search and the
// inverse-squared-distance blend of the retrieved vectors.
#pragma once

#include "layer.cuh"

#include <memory>

namespace rvc {

class IndexModel {
 public:
  static constexpr int kMaxK = 16;   // largest k served
  static constexpr int kExtra = 8;   // extra approximate candidates re-ranked exactly

  // db: host [N][D] float32 (copied to the device).
  IndexModel(Context* ctx, const float* db, int64_t N, int D, int precision);
  // Device pointers, asynchronous on ctx->stream: q [F][D] -> scores/inds [F][min(k, N)].
  void search_device(const float* q, int64_t F, int k, float* scores, int64_t* inds);
  // Device pointers: out [F][D] = blend (mode 0: w = (1/s)^2, the pipeline's formula;
  // mode 1: w = 1/max(s,1e-6)^2, weighted_blend), mixed with feats when feats != nullptr:
  // out = blend * c_blend + feats * c_feats.
  void blend_device(const float* q, int64_t F, int k, int mode, float c_blend, float c_feats, const float* feats,
                    float* out);
  // Host-pointer versions (inputs staged through buffers the model keeps).
  void search_host(const float* q, int64_t F, int k, float* scores, int64_t* inds);
  void blend_host(const float* q, int64_t F, int k, int mode, float c_blend, float c_feats, const float* feats,
                  float* out);
  // Inverted-file structure (runtime/ivf_index.py:121-483): centroids [nlist][D]
  // (host) and the bucket of every index row (host [N], values in [0, nlist)).
  void set_ivf(const float* centroids, int nlist, const int64_t* assignments);
  // runtime/pipeline.py:_ivf_strict_search (:66-161) on device pointers: per
  // query the nprobe nearest centroids, then the k nearest rows of those
  // buckets; scores/inds [F][k], inf / -1 where the buckets hold fewer rows.
  void ivf_search_device(const float* q, int64_t F, int k, int nprobe, float* scores, int64_t* inds);
  void ivf_blend_device(const float* q, int64_t F, int k, int nprobe, float c_blend, float c_feats,
                        const float* feats, float* out);
  void ivf_search_host(const float* q, int64_t F, int k, int nprobe, float* scores, int64_t* inds);
  void ivf_blend_host(const float* q, int64_t F, int k, int nprobe, float c_blend, float c_feats,
                      const float* feats, float* out);
  int64_t N = 0, Npad = 0;
  int D = 0;
  int nlist = 0;
  Context* ctx;
  int precision;

 private:
  void ensure_ws(int64_t rows);
  DevBuf db_, d2_;
  ConvLayer gemm_;
  int64_t ws_rows_ = 0;
  DevBuf dot_, q2_, cand_v_, cand_i_, sc_, ix_;
  DevBuf h_q_, h_f_, h_o_, h_s_, h_i_;  // staging for the host-pointer calls
  std::unique_ptr<IndexModel> cent_;    // brute-force index over the centroids
  DevBuf bucket_rows_, bucket_off_;     // row ids grouped by bucket (stable), bucket offsets [nlist + 1]
  DevBuf probe_sc_, probe_ix_, ivf_sc_, ivf_ix_;
  int64_t probe_rows_ = 0, ivf_rows_ = 0;
  void stage(DevBuf& b, size_t bytes);
};

}  // namespace rvc
