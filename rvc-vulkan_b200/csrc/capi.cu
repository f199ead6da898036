// extern "C" boundary of librvc_cuda (declared in include/rvc_cuda.h).
// Every entry point: look up handles, take the context lock, set the device,
// run, and turn any exception into an int32 status + thread-local message.
#include "../../include/rvc_cuda.h"
#include "fcpe.cuh"
#include "hubert.cuh"
#include "retrieval.cuh"
#include "rmvpe.cuh"
#include "synth.cuh"

#include <cstring>
#include <memory>
#include <unordered_map>
#include <vector>

using namespace rvc;

namespace {

std::mutex g_reg_mu;
// Registries hold shared ownership: a call in flight keeps its model (and the
// model keeps its context) alive, so a concurrent destroy only drops the
// registry's reference and the object goes away when the last call is done.
std::unordered_map<int64_t, std::shared_ptr<Context>> g_ctx;
std::unordered_map<int64_t, std::shared_ptr<SynthModel>> g_synth;
std::unordered_map<int64_t, std::shared_ptr<HubertModel>> g_hubert;
std::unordered_map<int64_t, std::shared_ptr<IndexModel>> g_index;
std::unordered_map<int64_t, std::shared_ptr<RmvpeModel>> g_rmvpe;
std::unordered_map<int64_t, std::shared_ptr<FcpeModel>> g_fcpe;
int64_t g_next = 1;

template <typename T>
std::shared_ptr<T> lookup(std::unordered_map<int64_t, std::shared_ptr<T>>& reg, int64_t h, const char* what) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  auto it = reg.find(h);
  if (it == reg.end()) throw Error{kErrState, std::string("invalid ") + what + " handle " + std::to_string(h)};
  return it->second;
}

std::shared_ptr<Context> get_ctx(int64_t h) { return lookup(g_ctx, h, "context"); }

// Shared ownership of a new model: the deleter keeps the model's context alive
// and frees the model's device buffers under the context lock, on its device.
// The last reference is never dropped by a thread holding that lock (callers
// release the lock before their reference).
template <typename T>
std::shared_ptr<T> own_model(Context* c, std::unique_ptr<T> m) {
  std::shared_ptr<Context> cref = c->shared_from_this();
  return std::shared_ptr<T>(m.release(), [cref](T* p) {
    std::lock_guard<std::mutex> lk(cref->mu);
    DeviceGuard dg(cref->device);
    delete p;
  });
}

// Removes a model from its registry; the caller drops the returned reference
// outside every lock.
template <typename T>
std::shared_ptr<T> take(std::unordered_map<int64_t, std::shared_ptr<T>>& reg, int64_t h, const char* what) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  auto it = reg.find(h);
  if (it == reg.end()) throw Error{kErrState, std::string("invalid ") + what + " handle " + std::to_string(h)};
  std::shared_ptr<T> m = std::move(it->second);
  reg.erase(it);
  return m;
}

template <typename F>
int32_t guarded(F&& f) {
  try {
    f();
    return kOk;
  } catch (const Error& e) {
    set_error(e.msg);
    return e.code;
  } catch (const std::exception& e) {
    set_error(std::string("internal error: ") + e.what());
    return kErrState;
  } catch (...) {
    set_error("internal error");
    return kErrState;
  }
}

// Runs `f` on the context's device under its lock.
template <typename F>
int32_t on_ctx(int64_t h, F&& f) {
  return guarded([&] {
    std::shared_ptr<Context> c = get_ctx(h);
    std::lock_guard<std::mutex> lk(c->mu);
    DeviceGuard dg(c->device);
    f(c.get());
  });
}

int32_t finish(Context* c) {
  int32_t rc = c->sync(0);
  if (rc != kOk) throw Error{rc, get_error()};
  return rc;
}

void h2d(Context* c, void* d, const void* h, size_t n) {
  if (n) RVC_CUDA_TRY(cudaMemcpyAsync(d, h, n, cudaMemcpyHostToDevice, c->stream));
}
void d2h(Context* c, void* h, const void* d, size_t n) {
  if (n) RVC_CUDA_TRY(cudaMemcpyAsync(h, d, n, cudaMemcpyDeviceToHost, c->stream));
}

template <typename F>
int32_t on_synth(int64_t model, F&& f) {
  return guarded([&] {
    std::shared_ptr<SynthModel> m = lookup(g_synth, model, "synthesizer");
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    DeviceGuard dg(m->ctx->device);
    f(m.get());
  });
}

template <typename F>
int32_t on_hubert(int64_t model, F&& f) {
  return guarded([&] {
    std::shared_ptr<HubertModel> m = lookup(g_hubert, model, "HuBERT");
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    DeviceGuard dg(m->ctx->device);
    f(m.get());
  });
}

template <typename F>
int32_t on_index(int64_t index, F&& f) {
  return guarded([&] {
    std::shared_ptr<IndexModel> m = lookup(g_index, index, "index");
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    DeviceGuard dg(m->ctx->device);
    f(m.get());
  });
}

template <typename F>
int32_t on_fcpe(int64_t model, F&& f) {
  return guarded([&] {
    std::shared_ptr<FcpeModel> m = lookup(g_fcpe, model, "FCPE");
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    DeviceGuard dg(m->ctx->device);
    f(m.get());
  });
}

template <typename F>
int32_t on_rmvpe(int64_t model, F&& f) {
  return guarded([&] {
    std::shared_ptr<RmvpeModel> m = lookup(g_rmvpe, model, "RMVPE");
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    DeviceGuard dg(m->ctx->device);
    f(m.get());
  });
}

}  // namespace

// Handle lookup for entry points defined in other translation units.
std::shared_ptr<rvc::Context> rvc_capi_context(int64_t h) { return get_ctx(h); }

extern "C" {

int32_t rvc_cuda_version(void) { return 100; }

int32_t rvc_cuda_launch_count(int64_t* n) {
  *n = launch_count();
  return kOk;
}

int32_t rvc_cuda_last_error(char* buf, int64_t n) {
  const std::string& m = get_error();
  if (buf && n > 0) {
    size_t k = std::min<size_t>((size_t)n - 1, m.size());
    std::memcpy(buf, m.data(), k);
    buf[k] = 0;
  }
  return (int32_t)m.size();
}

int32_t rvc_cuda_device_count(int32_t* n) {
  return guarded([&] {
    int c = 0;
    cudaError_t e = cudaGetDeviceCount(&c);
    if (e != cudaSuccess) {
      cudaGetLastError();
      c = 0;
    }
    *n = c;
  });
}

int32_t rvc_cuda_create(int32_t device, int64_t* ctx) {
  return guarded([&] {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
      cudaGetLastError();
      throw Error{kErrArg, "no CUDA device " + std::to_string(device) + " (" + std::to_string(n) + " visible)"};
    }
    cudaDeviceProp prop;
    RVC_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
      throw Error{kErrArg, std::string("librvc_cuda is built for sm_100a (B200); device is ") + prop.name};
    auto c = std::make_shared<Context>(device);
    std::lock_guard<std::mutex> lk(g_reg_mu);
    *ctx = g_next++;
    g_ctx[*ctx] = std::move(c);
  });
}

int32_t rvc_cuda_destroy(int64_t ctx) {
  return guarded([&] {
    std::shared_ptr<Context> c;
    std::vector<std::shared_ptr<void>> bound;
    {
      std::lock_guard<std::mutex> lk(g_reg_mu);
      auto it = g_ctx.find(ctx);
      if (it == g_ctx.end()) throw Error{kErrState, "invalid context handle " + std::to_string(ctx)};
      // every model bound to this context leaves the registry first
      const Context* cp = it->second.get();
      auto drop = [cp, &bound](auto& reg) {
        for (auto s = reg.begin(); s != reg.end();) {
          if (s->second->ctx == cp) {
            bound.push_back(std::move(s->second));
            s = reg.erase(s);
          } else {
            ++s;
          }
        }
      };
      drop(g_synth);
      drop(g_hubert);
      drop(g_index);
      drop(g_rmvpe);
      drop(g_fcpe);
      c = std::move(it->second);
      g_ctx.erase(it);
    }
    // models first (each deleter waits for the context lock, i.e. for calls in
    // flight on it), then the context once no call holds it any more
    bound.clear();
    { std::lock_guard<std::mutex> lk(c->mu); }
    c.reset();
  });
}

int32_t rvc_cuda_sync(int64_t ctx, int32_t timeout_ms) {
  return on_ctx(ctx, [&](Context* c) {
    int32_t rc = c->sync(timeout_ms);
    if (rc != kOk) throw Error{rc, get_error()};
  });
}

int32_t rvc_cuda_stream(int64_t ctx, void** stream) {
  return on_ctx(ctx, [&](Context* c) { *stream = (void*)c->stream; });
}

int32_t rvc_cuda_set_mem_cap(int64_t ctx, int64_t bytes) {
  return on_ctx(ctx, [&](Context* c) { c->mem_cap = bytes; });
}

int32_t rvc_cuda_release_pool(int64_t ctx) {
  return on_ctx(ctx, [&](Context* c) { c->release_pool(); });
}

int32_t rvc_cuda_alloc(int64_t ctx, int64_t bytes, void** dptr) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(bytes >= 0, "alloc: negative size");
    *dptr = c->alloc((size_t)bytes);
  });
}

int32_t rvc_cuda_free(int64_t ctx, void* dptr) {
  return on_ctx(ctx, [&](Context* c) { c->free(dptr); });
}

int32_t rvc_cuda_h2d(int64_t ctx, void* dst, const void* src, int64_t bytes) {
  return on_ctx(ctx, [&](Context* c) {
    h2d(c, dst, src, (size_t)bytes);
    finish(c);
  });
}

int32_t rvc_cuda_d2h(int64_t ctx, void* dst, const void* src, int64_t bytes) {
  return on_ctx(ctx, [&](Context* c) {
    d2h(c, dst, src, (size_t)bytes);
    finish(c);
  });
}

int32_t rvc_cuda_d2d(int64_t ctx, void* dst, const void* src, int64_t bytes) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(dst && src && bytes >= 0, "d2d: bad arguments");
    if (bytes) RVC_CUDA_TRY(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDeviceToDevice, c->stream));
  });
}

int32_t rvc_cuda_h2d_async(int64_t ctx, void* dst, const void* src, int64_t bytes) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(dst && src && bytes >= 0, "h2d_async: bad arguments");
    h2d(c, dst, src, (size_t)bytes);
  });
}

int32_t rvc_cuda_host_alloc(int64_t bytes, void** ptr) {
  return guarded([&] {
    RVC_CHECK_ARG(ptr && bytes > 0, "host_alloc: bad arguments");
    *ptr = nullptr;
    RVC_CUDA_TRY(cudaHostAlloc(ptr, (size_t)bytes, cudaHostAllocPortable));
  });
}

int32_t rvc_cuda_host_free(void* ptr) {
  return guarded([&] {
    if (ptr) RVC_CUDA_TRY(cudaFreeHost(ptr));
  });
}

int32_t rvc_cuda_profile(int64_t ctx, int32_t enable) {
  return on_ctx(ctx, [&](Context* c) {
    c->prof_collect();
    c->prof = enable != 0;
    c->prof_by_label.clear();
    c->prof_launches = 0;
    c->prof_ms = 0.0;
    c->prof_flops = 0.0;
  });
}

int32_t rvc_cuda_profile_dump(int64_t ctx, char* buf, int64_t n) {
  int32_t len = 0;
  int32_t rc = on_ctx(ctx, [&](Context* c) {
    c->prof_collect();
    std::string out = "label,launches,ms,flops\n";
    for (auto& kv : c->prof_by_label) {
      char line[256];
      snprintf(line, sizeof(line), "\"%s\",%lld,%.6f,%.6e\n", kv.first.c_str(), kv.second.n, kv.second.ms,
               kv.second.flops);
      out += line;
    }
    len = (int32_t)out.size();
    if (buf && n > 0) {
      size_t k = std::min<size_t>((size_t)n - 1, out.size());
      std::memcpy(buf, out.data(), k);
      buf[k] = 0;
    }
  });
  return rc == kOk ? len : rc;
}

int32_t rvc_cuda_profile_read(int64_t ctx, int64_t* launches, double* ms, double* flops) {
  return on_ctx(ctx, [&](Context* c) {
    c->prof_collect();
    *launches = c->prof_launches;
    *ms = c->prof_ms;
    *flops = c->prof_flops;
  });
}

// ----------------------------------------------------------------- tier 1
int32_t rvc_cuda_conv1d(int64_t ctx, const float* x, int32_t B, int32_t C, int32_t T, const float* w, int32_t O,
                        int32_t K, const float* b, int32_t stride, int32_t pad_l, int32_t pad_r, int32_t dilation,
                        float* y, int32_t oL) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(B >= 0 && C > 0 && T >= 0 && O > 0 && K > 0 && stride > 0 && dilation > 0 && pad_l >= 0 &&
                      pad_r >= 0,
                  "conv1d: bad arguments");
    RVC_CHECK_ARG(oL == (T + pad_l + pad_r - dilation * (K - 1) - 1) / stride + 1 || (oL == 0),
                  "conv1d: output length mismatch");
    if (B == 0 || oL <= 0) return;
    DevBuf dx(c, sizeof(float) * (size_t)B * C * T), dxt(c, sizeof(float) * (size_t)B * C * T);
    DevBuf dw(c, sizeof(float) * (size_t)O * C * K), dy(c, sizeof(float) * (size_t)B * O * oL),
        dyt(c, sizeof(float) * (size_t)B * O * oL);
    DevBuf db;
    h2d(c, dx.p, x, dx.bytes);
    h2d(c, dw.p, w, dw.bytes);
    if (b) {
      db = DevBuf(c, sizeof(float) * O);
      h2d(c, db.p, b, db.bytes);
    }
    k_nct_to_ntc(dx.f(), dxt.f(), B, C, T, C, c->stream);
    ConvLayer L;
    L.dil = dilation;
    L.pad_l = pad_l;
    L.pad_r = pad_r;
    L.stride = stride;
    L.build(c, LayerKind::kConv, dw.f(), db.p ? db.f() : nullptr, O, C, K, true);
    ConvIO io;
    io.x = dxt.f(); io.x_ld = C; io.x_bs = (long long)T * C; io.T_in = T;
    io.y = dy.f(); io.y_ld = O; io.y_bs = (long long)oL * O;
    io.B = B;
    L.run(c, io);
    k_ntc_to_nct(dy.f(), O, dyt.f(), B, O, oL, c->stream);
    d2h(c, y, dyt.p, dyt.bytes);
    finish(c);
  });
}

int32_t rvc_cuda_conv_transpose1d(int64_t ctx, const float* x, int32_t B, int32_t Ci, int32_t T, const float* w,
                                  int32_t Co, int32_t K, const float* b, int32_t stride, int32_t padding,
                                  int32_t output_padding, int32_t dilation, float* y, int32_t oL) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(B >= 0 && Ci > 0 && T >= 0 && Co > 0 && K > 0 && stride > 0 && padding >= 0,
                  "conv_transpose1d: bad arguments");
    RVC_CHECK_ARG(dilation == 1 && output_padding == 0,
                  "conv_transpose1d: only dilation=1, output_padding=0 are supported");
    RVC_CHECK_ARG(stride <= kMaxSlices, "conv_transpose1d: stride > 16 unsupported");
    RVC_CHECK_ARG(oL == (T - 1) * stride - 2 * padding + K, "conv_transpose1d: output length mismatch");
    if (B == 0 || oL <= 0) return;
    DevBuf dx(c, sizeof(float) * (size_t)B * Ci * T), dxt(c, sizeof(float) * (size_t)B * Ci * T);
    DevBuf dw(c, sizeof(float) * (size_t)Ci * Co * K), dy(c, sizeof(float) * (size_t)B * Co * oL),
        dyt(c, sizeof(float) * (size_t)B * Co * oL);
    DevBuf db;
    h2d(c, dx.p, x, dx.bytes);
    h2d(c, dw.p, w, dw.bytes);
    if (b) {
      db = DevBuf(c, sizeof(float) * Co);
      h2d(c, db.p, b, db.bytes);
    }
    k_nct_to_ntc(dx.f(), dxt.f(), B, Ci, T, Ci, c->stream);
    ConvLayer L;
    L.up = stride;
    L.up_pad = padding;
    L.build(c, LayerKind::kConvT, dw.f(), db.p ? db.f() : nullptr, Co, Ci, K, true);
    ConvIO io;
    io.x = dxt.f(); io.x_ld = Ci; io.x_bs = (long long)T * Ci; io.T_in = T;
    io.y = dy.f(); io.y_ld = Co; io.y_bs = (long long)oL * Co;
    io.B = B;
    L.run(c, io);
    k_ntc_to_nct(dy.f(), Co, dyt.f(), B, Co, oL, c->stream);
    d2h(c, y, dyt.p, dyt.bytes);
    finish(c);
  });
}

int32_t rvc_cuda_matmul(int64_t ctx, const float* a, const float* b, int32_t M, int32_t K, int32_t N, float* cc) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(M >= 0 && K > 0 && N > 0, "matmul: bad shape");
    if (M == 0) return;
    DevBuf da(c, sizeof(float) * (size_t)M * K), dw(c, sizeof(float) * (size_t)K * N),
        dc(c, sizeof(float) * (size_t)M * N);
    h2d(c, da.p, a, da.bytes);
    // b[K,N] row-major is exactly the [tap=1][C_in=K][C_out=N] weight layout;
    // build() expects [O,I,K]: upload as conv weight via an explicit transpose.
    DevBuf dbt(c, sizeof(float) * (size_t)K * N), dbn(c, sizeof(float) * (size_t)K * N);
    h2d(c, dbt.p, b, dbt.bytes);
    k_ntc_to_nct(dbt.f(), N, dbn.f(), 1, N, K, c->stream);  // [K][N] -> [N][K]
    ConvLayer L;
    L.build(c, LayerKind::kConv, dbn.f(), nullptr, N, K, 1, true);
    ConvIO io;
    io.x = da.f(); io.x_ld = K; io.x_bs = (long long)M * K; io.T_in = M;
    io.y = dc.f(); io.y_ld = N; io.y_bs = (long long)M * N;
    io.B = 1;
    L.run(c, io);
    d2h(c, cc, dc.p, dc.bytes);
    finish(c);
  });
}

int32_t rvc_cuda_layer_norm(int64_t ctx, const float* x, int64_t rows, int32_t C, const float* gamma,
                            const float* beta, float eps, float* y) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(rows >= 0 && C > 0 && C <= 1024, "layer_norm: bad shape (C <= 1024)");
    if (rows == 0) return;
    DevBuf dx(c, sizeof(float) * (size_t)rows * C), dg(c, sizeof(float) * C), dbb(c, sizeof(float) * C);
    h2d(c, dx.p, x, dx.bytes);
    h2d(c, dg.p, gamma, dg.bytes);
    h2d(c, dbb.p, beta, dbb.bytes);
    k_layernorm(dx.f(), C, nullptr, 0, rows, C, dg.f(), dbb.f(), eps, dx.f(), C, c->stream);
    d2h(c, y, dx.p, dx.bytes);
    finish(c);
  });
}

int32_t rvc_cuda_conv2d(int64_t ctx, const float* x, int32_t B, int32_t C, int32_t H, int32_t W, const float* w,
                        int32_t O, int32_t KH, int32_t KW, const float* b, int32_t sh, int32_t sw, int32_t ph,
                        int32_t pw, float* y) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(B >= 0 && C > 0 && H > 0 && W > 0 && O > 0 && KH > 0 && KW > 0 && sh > 0 && sw > 0 && ph >= 0 &&
                      pw >= 0,
                  "conv2d: bad shape");
    const int Ho = (H + 2 * ph - KH) / sh + 1, Wo = (W + 2 * pw - KW) / sw + 1;
    RVC_CHECK_ARG(H + 2 * ph >= KH && W + 2 * pw >= KW && Ho > 0 && Wo > 0, "conv2d: kernel larger than the input");
    if (B == 0) return;
    DevBuf dx(c, sizeof(float) * (size_t)B * C * H * W), dw(c, sizeof(float) * (size_t)O * C * KH * KW), db,
        dy(c, sizeof(float) * (size_t)B * O * Ho * Wo);
    h2d(c, dx.p, x, dx.bytes);
    h2d(c, dw.p, w, dw.bytes);
    if (b) {
      db = DevBuf(c, sizeof(float) * O);
      h2d(c, db.p, b, db.bytes);
    }
    k_conv2d(dx.f(), B, C, H, W, dw.f(), O, KH, KW, b ? db.f() : nullptr, sh, sw, ph, pw, dy.f(), c->stream);
    d2h(c, y, dy.p, dy.bytes);
    finish(c);
  });
}

int32_t rvc_cuda_rmsnorm(int64_t ctx, const float* x, int64_t rows, int32_t C, const float* gamma, float eps,
                         float* y) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(rows >= 0 && C > 0, "rmsnorm: bad shape");
    if (rows == 0) return;
    DevBuf dx(c, sizeof(float) * (size_t)rows * C), dg(c, sizeof(float) * C);
    h2d(c, dx.p, x, dx.bytes);
    h2d(c, dg.p, gamma, dg.bytes);
    k_rmsnorm(dx.f(), rows, C, dg.f(), eps, dx.f(), c->stream);
    d2h(c, y, dx.p, dx.bytes);
    finish(c);
  });
}

int32_t rvc_cuda_softmax(int64_t ctx, const float* x, int64_t rows, int32_t C, float* y) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(rows >= 0 && C > 0, "softmax: bad shape");
    if (rows == 0) return;
    DevBuf dx(c, sizeof(float) * (size_t)rows * C);
    h2d(c, dx.p, x, dx.bytes);
    k_softmax_rows(dx.f(), dx.f(), rows, C, c->stream);
    d2h(c, y, dx.p, dx.bytes);
    finish(c);
  });
}

int32_t rvc_cuda_elementwise(int64_t ctx, int32_t op, const float* a, const float* b, int64_t n, float alpha,
                             float* y) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(op >= 0 && op <= 6 && n >= 0, "elementwise: bad op or size");
    RVC_CHECK_ARG(op > 1 || b != nullptr, "elementwise: binary op needs b");
    if (n == 0) return;
    DevBuf da(c, sizeof(float) * (size_t)n), dbb;
    h2d(c, da.p, a, da.bytes);
    if (op <= 1) {
      dbb = DevBuf(c, sizeof(float) * (size_t)n);
      h2d(c, dbb.p, b, dbb.bytes);
    }
    k_elementwise(op, da.f(), dbb.p ? dbb.f() : nullptr, n, alpha, da.f(), c->stream);
    d2h(c, y, da.p, da.bytes);
    finish(c);
  });
}

int32_t rvc_cuda_embedding(int64_t ctx, const int64_t* ids, int64_t n, const float* table, int32_t V, int32_t E,
                           float* y) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(n >= 0 && V > 0 && E > 0, "embedding: bad shape");
    for (int64_t i = 0; i < n; ++i)
      RVC_CHECK_ARG(ids[i] >= -V && ids[i] < V, "embedding: id out of range");
    if (n == 0) return;
    DevBuf di(c, sizeof(int64_t) * (size_t)n), dt(c, sizeof(float) * (size_t)V * E), dy(c, sizeof(float) * (size_t)n * E);
    h2d(c, di.p, ids, di.bytes);
    h2d(c, dt.p, table, dt.bytes);
    k_embedding(di.as<long long>(), n, dt.f(), V, E, dy.f(), c->stream);
    d2h(c, y, dy.p, dy.bytes);
    finish(c);
  });
}

int32_t rvc_cuda_gating(int64_t ctx, const float* x, const float* g, int32_t B, int32_t H, int32_t T, float* y) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(B >= 0 && H > 0 && T >= 0, "gating: bad shape");
    if (B * T == 0) return;
    DevBuf dx(c, sizeof(float) * (size_t)B * 2 * H * T), dg, dy(c, sizeof(float) * (size_t)B * H * T);
    h2d(c, dx.p, x, dx.bytes);
    if (g) {
      dg = DevBuf(c, sizeof(float) * (size_t)B * 2 * H);
      h2d(c, dg.p, g, dg.bytes);
    }
    k_gating_nct(dx.f(), dg.p ? dg.f() : nullptr, B, H, T, dy.f(), c->stream);
    d2h(c, y, dy.p, dy.bytes);
    finish(c);
  });
}

int32_t rvc_cuda_rel_attention(int64_t ctx, const float* q, const float* k, const float* v, const float* emb_k,
                               const float* emb_v, int32_t B, int32_t heads, int32_t kc, int32_t P, int32_t window,
                               float* y) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(B >= 0 && heads > 0 && kc > 0 && P >= 0 && window >= 0, "rel_attention: bad shape");
    if (B * P == 0) return;
    const int H = heads * kc;
    const size_t n = (size_t)B * H * P;
    DevBuf dq(c, sizeof(float) * n), dk(c, sizeof(float) * n), dv(c, sizeof(float) * n);
    DevBuf qkv(c, sizeof(float) * 3 * n), ek(c, sizeof(float) * (2 * window + 1) * kc),
        ev(c, sizeof(float) * (2 * window + 1) * kc);
    DevBuf yt(c, sizeof(float) * n), yo(c, sizeof(float) * n);
    h2d(c, dq.p, q, dq.bytes);
    h2d(c, dk.p, k, dk.bytes);
    h2d(c, dv.p, v, dv.bytes);
    h2d(c, ek.p, emb_k, ek.bytes);
    h2d(c, ev.p, emb_v, ev.bytes);
    // pack [B, P, 3H] channels-last
    for (int bb = 0; bb < B; ++bb) {
      k_nct_to_ntc(dq.f() + (size_t)bb * H * P, qkv.f() + (size_t)bb * P * 3 * H, 1, H, P, 3 * H, c->stream);
      k_nct_to_ntc(dk.f() + (size_t)bb * H * P, qkv.f() + (size_t)bb * P * 3 * H + H, 1, H, P, 3 * H, c->stream);
      k_nct_to_ntc(dv.f() + (size_t)bb * H * P, qkv.f() + (size_t)bb * P * 3 * H + 2 * H, 1, H, P, 3 * H, c->stream);
    }
    k_rel_attention(qkv.f(), 3 * H, 0, H, 2 * H, ek.f(), ev.f(), B, heads, kc, P, window, nullptr, yt.f(), H,
                    c->stream);
    k_ntc_to_nct(yt.f(), H, yo.f(), B, H, P, c->stream);
    d2h(c, y, yo.p, yo.bytes);
    finish(c);
  });
}

int32_t rvc_cuda_im2col1d(int64_t ctx, const float* x, int32_t B, int32_t C, int32_t T, int32_t K, int32_t stride,
                          int32_t pad_l, int32_t dilation, int32_t oL, float* cols) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(B >= 0 && C > 0 && T >= 0 && K > 0 && stride > 0 && dilation > 0 && oL >= 0,
                  "im2col1d: bad shape");
    if (B * oL == 0) return;
    DevBuf dx(c, sizeof(float) * (size_t)B * C * T), dc(c, sizeof(float) * (size_t)B * oL * C * K);
    h2d(c, dx.p, x, dx.bytes);
    k_im2col1d(dx.f(), B, C, T, K, stride, pad_l, dilation, oL, dc.f(), c->stream);
    d2h(c, cols, dc.p, dc.bytes);
    finish(c);
  });
}

// ----------------------------------------------------------------- tier 2
int32_t rvc_cuda_synth_create(int64_t ctx, const int32_t* cfg, int32_t ncfg, int64_t* model) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(ncfg >= 10, "synth_create: config too short");
    SynthConfig s;
    int i = 0;
    s.sr = cfg[i++]; s.hidden = cfg[i++]; s.filter = cfg[i++]; s.heads = cfg[i++]; s.layers = cfg[i++];
    s.kc = cfg[i++]; s.window = cfg[i++]; s.gin = cfg[i++]; s.up0 = cfg[i++]; s.n_ups = cfg[i++];
    RVC_CHECK_ARG(s.n_ups >= 1 && s.n_ups <= 8 && ncfg >= 10 + 2 * s.n_ups + 3, "synth_create: config too short");
    for (int u = 0; u < s.n_ups; ++u) s.rates.push_back(cfg[i++]);
    for (int u = 0; u < s.n_ups; ++u) s.kernels.push_back(cfg[i++]);
    s.phone_dim = cfg[i++]; s.n_spk = cfg[i++]; s.precision = cfg[i++];
    RVC_CHECK_ARG(s.precision == 0 || s.precision == 1, "synth_create: precision must be 0 or 1");
    auto m = std::make_unique<SynthModel>(c, s);
    std::lock_guard<std::mutex> lk(g_reg_mu);
    *model = g_next++;
    g_synth[*model] = own_model(c, std::move(m));
  });
}

int32_t rvc_cuda_synth_destroy(int64_t model) {
  return guarded([&] {
    std::shared_ptr<SynthModel> m = take(g_synth, model, "synthesizer");
    m.reset();  // freed now, or when the last call in flight returns
  });
}

int32_t rvc_cuda_synth_set_weight(int64_t model, const char* key, const float* data, const int64_t* shape,
                                  int32_t ndim) {
  return on_synth(model, [&](SynthModel* m) {
    RVC_CHECK_ARG(key && data && ndim >= 0 && ndim <= 8, "synth_set_weight: bad arguments");
    std::vector<int64_t> s(shape, shape + ndim);
    m->set_weight(key, data, s);
  });
}

int32_t rvc_cuda_synth_finalize(int64_t model) {
  return on_synth(model, [&](SynthModel* m) {
    m->finalize();
    finish(m->ctx);
  });
}

int32_t rvc_cuda_synth_infer(int64_t model, int32_t B, int32_t P, const float* phone, const int64_t* pitch,
                             const float* nsff0, const int64_t* sid, const float* nz, const float* ns, float* wave) {
  return on_synth(model, [&](SynthModel* m) {
    RVC_CHECK_ARG(B >= 1 && P >= 1, "synth_infer: B and P must be positive");
    const int V = 256;
    for (int64_t i = 0; i < (int64_t)B * P; ++i)
      RVC_CHECK_ARG(pitch[i] >= -V && pitch[i] < V, "synth_infer: pitch id out of [0,256)");
    for (int i = 0; i < B; ++i)
      RVC_CHECK_ARG(sid[i] >= -m->cfg.n_spk && sid[i] < m->cfg.n_spk, "synth_infer: speaker id out of range");
    m->infer_host(B, P, phone, (const long long*)pitch, nsff0, (const long long*)sid, nz, ns, wave);
    finish(m->ctx);
  });
}

int32_t rvc_cuda_synth_infer_grouped(int64_t model, int32_t B, int32_t G, int32_t P, const float* phone,
                                     const int64_t* pitch, const float* nsff0, const int64_t* sid, const float* nz,
                                     const float* ns, float* wave) {
  return on_synth(model, [&](SynthModel* m) {
    RVC_CHECK_ARG(B >= 1 && G >= 1 && P >= 1, "synth_infer_grouped: B, G and P must be positive");
    for (int64_t i = 0; i < (int64_t)B * P; ++i)
      RVC_CHECK_ARG(pitch[i] >= -256 && pitch[i] < 256, "synth_infer_grouped: pitch id out of [0,256)");
    for (int i = 0; i < B; ++i)
      RVC_CHECK_ARG(sid[i] >= -m->cfg.n_spk && sid[i] < m->cfg.n_spk, "synth_infer_grouped: speaker id out of range");
    m->infer_host_grouped(B, G, P, phone, (const long long*)pitch, nsff0, (const long long*)sid, nz, ns, wave);
    finish(m->ctx);
  });
}

int32_t rvc_cuda_synth_infer_device(int64_t model, int32_t B, int32_t P, const float* phone, const int64_t* pitch,
                                    const float* nsff0, const int64_t* sid, const float* nz, const float* ns,
                                    float* wave) {
  return on_synth(model, [&](SynthModel* m) {
    m->infer_device(B, P, phone, (const long long*)pitch, nsff0, (const long long*)sid, nz, ns, wave);
  });
}

int32_t rvc_cuda_synth_infer_partial(int64_t model, int32_t P, int32_t skip_head, int32_t return_length,
                                     const float* phone, const int64_t* pitch, const float* nsff0, const int64_t* sid,
                                     const float* nz, const float* ns, float* wave) {
  return on_synth(model, [&](SynthModel* m) {
    RVC_CHECK_ARG(P >= 1 && skip_head >= 0 && skip_head < P && return_length >= 1 && skip_head + return_length <= P,
                  "synth_infer_partial: skip_head/return_length out of range");
    for (int64_t i = 0; i < P; ++i)
      RVC_CHECK_ARG(pitch[i] >= -256 && pitch[i] < 256, "synth_infer_partial: pitch id out of [0,256)");
    RVC_CHECK_ARG(sid[0] >= -m->cfg.n_spk && sid[0] < m->cfg.n_spk, "synth_infer_partial: speaker id out of range");
    const int H = m->cfg.hidden, upp = m->cfg.upp();
    const int Dp = m->cfg.phone_dim;
    DevBuf dph(m->ctx, sizeof(float) * (size_t)P * Dp), dpi(m->ctx, sizeof(int64_t) * P), df0(m->ctx, sizeof(float) * P),
        dsid(m->ctx, sizeof(int64_t)), dnz(m->ctx, sizeof(float) * (size_t)H * P),
        dns(m->ctx, sizeof(float) * (size_t)P * upp), dw(m->ctx, sizeof(float) * (size_t)return_length * upp);
    h2d(m->ctx, dph.p, phone, dph.bytes);
    h2d(m->ctx, dpi.p, pitch, dpi.bytes);
    h2d(m->ctx, df0.p, nsff0, df0.bytes);
    h2d(m->ctx, dsid.p, sid, dsid.bytes);
    h2d(m->ctx, dnz.p, nz, dnz.bytes);
    h2d(m->ctx, dns.p, ns, dns.bytes);
    m->infer_partial_device(P, skip_head, return_length, dph.f(), dpi.as<long long>(), df0.f(),
                            dsid.as<long long>(), dnz.f(), dns.f(), dw.f());
    d2h(m->ctx, wave, dw.p, dw.bytes);
    finish(m->ctx);
  });
}

int32_t rvc_cuda_synth_tap(int64_t model, const char* name, float* out, int64_t n) {
  return on_synth(model, [&](SynthModel* m) {
    if (!m->tap(name, out, n)) throw Error{kErrArg, std::string("synth_tap: no tap '") + name + "' of that size"};
  });
}

int32_t rvc_cuda_synth_keep_taps(int64_t model, int32_t enable) {
  return on_synth(model, [&](SynthModel* m) {
    RVC_CHECK_ARG(enable >= 0, "synth_keep_taps: enable must be >= 0");
    m->keep_taps = enable;
  });
}

// ----------------------------------------------------------------- HuBERT
int32_t rvc_cuda_hubert_create(int64_t ctx, int32_t precision, int64_t* model) {
  return on_ctx(ctx, [&](Context* c) {
    auto m = std::make_unique<HubertModel>(c, precision);
    std::lock_guard<std::mutex> lk(g_reg_mu);
    *model = g_next++;
    g_hubert[*model] = own_model(c, std::move(m));
  });
}

int32_t rvc_cuda_hubert_destroy(int64_t model) {
  return guarded([&] {
    std::shared_ptr<HubertModel> m = take(g_hubert, model, "HuBERT");
    m.reset();  // freed now, or when the last call in flight returns
  });
}

int32_t rvc_cuda_hubert_set_weight(int64_t model, const char* key, const float* data, const int64_t* shape,
                                   int32_t ndim) {
  return on_hubert(model, [&](HubertModel* m) {
    RVC_CHECK_ARG(key && data && ndim >= 0 && ndim <= 8, "hubert_set_weight: bad arguments");
    std::vector<int64_t> s(shape, shape + ndim);
    m->set_weight(key, data, s);
  });
}

int32_t rvc_cuda_hubert_finalize(int64_t model) {
  return on_hubert(model, [&](HubertModel* m) {
    m->finalize();
    finish(m->ctx);
  });
}

int32_t rvc_cuda_hubert_out_len(int64_t T, int64_t* L) {
  return guarded([&] {
    RVC_CHECK_ARG(T >= 0 && L, "hubert_out_len: bad arguments");
    *L = HubertModel::out_len(T);
  });
}

int32_t rvc_cuda_hubert_encode(int64_t model, int32_t B, int64_t T, const float* x, int32_t version, float* out) {
  return on_hubert(model, [&](HubertModel* m) {
    RVC_CHECK_ARG(B >= 1 && T >= 1 && x && out, "hubert_encode: bad arguments");
    m->encode_host(B, T, x, version, out);
    finish(m->ctx);
  });
}

int32_t rvc_cuda_hubert_encode_device(int64_t model, int32_t B, int64_t T, const float* x, int32_t version,
                                      float* out) {
  return on_hubert(model, [&](HubertModel* m) { m->encode_device(B, T, x, version, out); });
}

int32_t rvc_cuda_hubert_tap(int64_t model, const char* name, float* out, int64_t n) {
  return on_hubert(model, [&](HubertModel* m) {
    if (!m->tap(name, out, n)) throw Error{kErrArg, std::string("hubert_tap: no tap '") + name + "' of that size"};
  });
}

int32_t rvc_cuda_hubert_keep_taps(int64_t model, int32_t enable) {
  return on_hubert(model, [&](HubertModel* m) { m->keep_taps = enable != 0; });
}

// ----------------------------------------------------------------- retrieval
int32_t rvc_cuda_index_create(int64_t ctx, const float* db, int64_t N, int32_t D, int32_t precision,
                              int64_t* index) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(db && index && N >= 1 && D >= 1, "index_create: need N >= 1 rows of D >= 1 floats");
    auto m = std::make_unique<IndexModel>(c, db, N, D, precision);
    std::lock_guard<std::mutex> lk(g_reg_mu);
    *index = g_next++;
    g_index[*index] = own_model(c, std::move(m));
  });
}

int32_t rvc_cuda_index_destroy(int64_t index) {
  return guarded([&] {
    std::shared_ptr<IndexModel> m = take(g_index, index, "index");
    m.reset();  // freed now, or when the last call in flight returns
  });
}

int32_t rvc_cuda_index_search(int64_t index, const float* q, int64_t F, int32_t D, int32_t k, float* scores,
                              int64_t* inds) {
  return on_index(index, [&](IndexModel* m) {
    RVC_CHECK_ARG(D == m->D, "index_search: query width " + std::to_string(D) + " != index width " +
                                 std::to_string(m->D));
    RVC_CHECK_ARG(F >= 0 && (F == 0 || (q && scores && inds)), "index_search: bad arguments");
    m->search_host(q, F, k, scores, inds);
    finish(m->ctx);
  });
}

int32_t rvc_cuda_index_search_device(int64_t index, const float* q, int64_t F, int32_t D, int32_t k,
                                     float* scores, int64_t* inds) {
  return on_index(index, [&](IndexModel* m) {
    RVC_CHECK_ARG(D == m->D, "index_search: query width does not match the index");
    m->search_device(q, F, k, scores, inds);
  });
}

int32_t rvc_cuda_index_blend(int64_t index, const float* q, int64_t F, int32_t D, int32_t k, int32_t mode,
                             double index_rate, const float* feats, float* out) {
  return on_index(index, [&](IndexModel* m) {
    RVC_CHECK_ARG(D == m->D, "index_blend: query width does not match the index");
    RVC_CHECK_ARG(F >= 0 && (F == 0 || (q && out)), "index_blend: bad arguments");
    // blend * rate + feats * (1 - rate), each factor rounded to float32 as numpy does
    m->blend_host(q, F, k, mode, (float)index_rate, (float)(1.0 - index_rate), feats, out);
    finish(m->ctx);
  });
}

int32_t rvc_cuda_index_blend_device(int64_t index, const float* q, int64_t F, int32_t D, int32_t k, int32_t mode,
                                    double index_rate, const float* feats, float* out) {
  return on_index(index, [&](IndexModel* m) {
    RVC_CHECK_ARG(D == m->D, "index_blend: query width does not match the index");
    m->blend_device(q, F, k, mode, (float)index_rate, (float)(1.0 - index_rate), feats, out);
  });
}

int32_t rvc_cuda_index_set_ivf(int64_t index, const float* centroids, int32_t nlist, const int64_t* assignments) {
  return on_index(index, [&](IndexModel* m) {
    RVC_CHECK_ARG(centroids && assignments && nlist >= 1, "index_set_ivf: bad arguments");
    m->set_ivf(centroids, nlist, assignments);
  });
}

int32_t rvc_cuda_index_ivf_search(int64_t index, const float* q, int64_t F, int32_t D, int32_t k, int32_t nprobe,
                                  float* scores, int64_t* inds) {
  return on_index(index, [&](IndexModel* m) {
    RVC_CHECK_ARG(D == m->D, "index_ivf_search: query width does not match the index");
    RVC_CHECK_ARG(F >= 0 && (F == 0 || (q && scores && inds)), "index_ivf_search: bad arguments");
    m->ivf_search_host(q, F, k, nprobe, scores, inds);
    finish(m->ctx);
  });
}

int32_t rvc_cuda_index_ivf_blend_device(int64_t index, const float* q, int64_t F, int32_t D, int32_t k,
                                        int32_t nprobe, double index_rate, const float* feats, float* out) {
  return on_index(index, [&](IndexModel* m) {
    RVC_CHECK_ARG(D == m->D, "index_ivf_blend: query width does not match the index");
    m->ivf_blend_device(q, F, k, nprobe, (float)index_rate, (float)(1.0 - index_rate), feats, out);
  });
}

int32_t rvc_cuda_index_ivf_blend(int64_t index, const float* q, int64_t F, int32_t D, int32_t k, int32_t nprobe,
                                 double index_rate, const float* feats, float* out) {
  return on_index(index, [&](IndexModel* m) {
    RVC_CHECK_ARG(D == m->D, "index_ivf_blend: query width does not match the index");
    RVC_CHECK_ARG(F >= 0 && (F == 0 || (q && out)), "index_ivf_blend: bad arguments");
    m->ivf_blend_host(q, F, k, nprobe, (float)index_rate, (float)(1.0 - index_rate), feats, out);
    finish(m->ctx);
  });
}

// ----------------------------------------------------------------- RMVPE
int32_t rvc_cuda_rmvpe_create(int64_t ctx, int64_t* model) {
  return on_ctx(ctx, [&](Context* c) {
    auto m = std::make_unique<RmvpeModel>(c);
    std::lock_guard<std::mutex> lk(g_reg_mu);
    *model = g_next++;
    g_rmvpe[*model] = own_model(c, std::move(m));
  });
}

int32_t rvc_cuda_rmvpe_destroy(int64_t model) {
  return guarded([&] {
    std::shared_ptr<RmvpeModel> m = take(g_rmvpe, model, "RMVPE");
    m.reset();  // freed now, or when the last call in flight returns
  });
}

int32_t rvc_cuda_rmvpe_set_weight(int64_t model, const char* key, const float* data, const int64_t* shape,
                                  int32_t ndim) {
  return on_rmvpe(model, [&](RmvpeModel* m) {
    RVC_CHECK_ARG(key && data && ndim >= 0 && ndim <= 8, "rmvpe_set_weight: bad arguments");
    std::vector<int64_t> s(shape, shape + ndim);
    m->set_weight(key, data, s);
  });
}

int32_t rvc_cuda_rmvpe_finalize(int64_t model) {
  return on_rmvpe(model, [&](RmvpeModel* m) {
    m->finalize();
    finish(m->ctx);
  });
}

int32_t rvc_cuda_rmvpe_frames(int64_t T, int64_t* F) {
  return guarded([&] {
    RVC_CHECK_ARG(T >= 0 && F, "rmvpe_frames: bad arguments");
    *F = RmvpeModel::frames(T);
  });
}

int32_t rvc_cuda_rmvpe_infer(int64_t model, int32_t B, int64_t T, const float* x, float thred, float* f0,
                             int32_t* argmax) {
  return on_rmvpe(model, [&](RmvpeModel* m) {
    RVC_CHECK_ARG(B >= 1 && x && f0, "rmvpe_infer: bad arguments");
    m->infer_host(B, T, x, thred, f0, argmax);
    finish(m->ctx);
  });
}

int32_t rvc_cuda_rmvpe_infer_device(int64_t model, int32_t B, int64_t T, const float* x, float thred, float* f0,
                                    int32_t* argmax) {
  return on_rmvpe(model, [&](RmvpeModel* m) { m->infer_device(B, T, x, thred, f0, argmax); });
}

int32_t rvc_cuda_rmvpe_tap(int64_t model, const char* name, float* out, int64_t n) {
  return on_rmvpe(model, [&](RmvpeModel* m) {
    if (!m->tap(name, out, n)) throw Error{kErrArg, std::string("rmvpe_tap: no tap '") + name + "' of that size"};
  });
}

int32_t rvc_cuda_rmvpe_keep_taps(int64_t model, int32_t enable) {
  return on_rmvpe(model, [&](RmvpeModel* m) { m->keep_taps = enable != 0; });
}

// ----------------------------------------------------------------- FCPE
int32_t rvc_cuda_fcpe_create(int64_t ctx, int32_t precision, int64_t* model) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(model, "fcpe_create: null output handle");
    auto m = std::make_unique<FcpeModel>(c, precision);
    std::lock_guard<std::mutex> lk(g_reg_mu);
    *model = g_next++;
    g_fcpe[*model] = own_model(c, std::move(m));
  });
}

int32_t rvc_cuda_fcpe_destroy(int64_t model) {
  return guarded([&] {
    std::shared_ptr<FcpeModel> m = take(g_fcpe, model, "FCPE");
    m.reset();  // freed now, or when the last call in flight returns
  });
}

int32_t rvc_cuda_fcpe_set_weight(int64_t model, const char* key, const float* data, const int64_t* shape,
                                 int32_t ndim) {
  return on_fcpe(model, [&](FcpeModel* m) {
    RVC_CHECK_ARG(key && data && ndim >= 0 && ndim <= 8, "fcpe_set_weight: bad arguments");
    std::vector<int64_t> s(shape, shape + ndim);
    m->set_weight(key, data, s);
  });
}

int32_t rvc_cuda_fcpe_finalize(int64_t model) {
  return on_fcpe(model, [&](FcpeModel* m) {
    m->finalize();
    finish(m->ctx);
  });
}

int32_t rvc_cuda_fcpe_infer_mode(int64_t model, int32_t B, int64_t T, const float* x, float threshold,
                                 int32_t decoder_mode, float* f0, int32_t* argmax) {
  return on_fcpe(model, [&](FcpeModel* m) {
    RVC_CHECK_ARG(B >= 1 && x && f0, "fcpe_infer_mode: bad arguments");
    m->infer_host(B, T, x, threshold, f0, argmax, decoder_mode);
    finish(m->ctx);
  });
}

int32_t rvc_cuda_fcpe_infer(int64_t model, int32_t B, int64_t T, const float* x, float threshold, float* f0,
                            int32_t* argmax) {
  return on_fcpe(model, [&](FcpeModel* m) {
    RVC_CHECK_ARG(B >= 1 && x && f0, "fcpe_infer: bad arguments");
    m->infer_host(B, T, x, threshold, f0, argmax);
    finish(m->ctx);
  });
}

int32_t rvc_cuda_fcpe_infer_device(int64_t model, int32_t B, int64_t T, const float* x, float threshold, float* f0,
                                   int32_t* argmax) {
  return on_fcpe(model, [&](FcpeModel* m) { m->infer_device(B, T, x, threshold, f0, argmax); });
}

int32_t rvc_cuda_fcpe_tap(int64_t model, const char* name, float* out, int64_t n) {
  return on_fcpe(model, [&](FcpeModel* m) {
    if (!m->tap(name, out, n)) throw Error{kErrArg, std::string("fcpe_tap: no tap '") + name + "' of that size"};
  });
}

int32_t rvc_cuda_fcpe_keep_taps(int64_t model, int32_t enable) {
  return on_fcpe(model, [&](FcpeModel* m) { m->keep_taps = enable != 0; });
}

// ----------------------------------------------------------------- pipeline DSP
int32_t rvc_cuda_filtfilt(int64_t ctx, const double* b, int32_t nb, const double* a, int32_t na, const void* x,
                          int32_t x_f32, int64_t n, double* y) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(b && a && x && y && nb >= 1 && na >= 1 && n >= 0, "filtfilt: bad arguments");
    DevBuf dx(c, sizeof(double) * (size_t)std::max<int64_t>(1, n)), dy(c, sizeof(double) * (size_t)std::max<int64_t>(1, n));
    if (x_f32) {
      DevBuf xf(c, sizeof(float) * (size_t)std::max<int64_t>(1, n));
      h2d(c, xf.p, x, sizeof(float) * n);
      dsp_f32_to_f64(c, xf.f(), n, (double*)dx.p);
      RVC_CUDA_TRY(cudaStreamSynchronize(c->stream));
    } else {
      h2d(c, dx.p, x, sizeof(double) * n);
    }
    dsp_filtfilt(c, b, nb, a, na, (const double*)dx.p, n, x_f32 != 0, (double*)dy.p);
    d2h(c, y, dy.p, sizeof(double) * n);
    finish(c);
  });
}

int32_t rvc_cuda_split_points(int64_t ctx, const double* audio, int64_t n, int32_t window, int64_t t_query,
                              int64_t step, int64_t* out, int64_t cap, int64_t* count) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(audio && out && count && n >= 1 && cap >= 0, "split_points: bad arguments");
    const int64_t nq = n > step ? (n - 1) / step : 0;
    RVC_CHECK_ARG(nq <= cap, "split_points: output holds " + std::to_string(cap) + " points, " +
                                 std::to_string(nq) + " needed");
    DevBuf dx(c, sizeof(double) * (size_t)n), dout(c, sizeof(int64_t) * (size_t)std::max<int64_t>(1, nq));
    h2d(c, dx.p, audio, sizeof(double) * n);
    *count = dsp_split_points(c, (const double*)dx.p, n, window, t_query, step, (long long*)dout.p);
    d2h(c, out, dout.p, sizeof(int64_t) * (size_t)nq);
    finish(c);
  });
}

int32_t rvc_cuda_interp_linear(int64_t ctx, const float* x, int64_t L, int32_t D, double scale, float* y,
                               int64_t Lo) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(x && y && L >= 1 && D >= 1 && scale > 0.0 && Lo == (int64_t)((double)L * scale),
                  "interp_linear: bad arguments (Lo must be int(L * scale))");
    DevBuf dx(c, sizeof(float) * (size_t)L * D), dy(c, sizeof(float) * (size_t)std::max<int64_t>(1, Lo) * D);
    h2d(c, dx.p, x, dx.bytes);
    dsp_interp_time(c, dx.f(), L, D, scale, dy.f(), Lo);
    d2h(c, y, dy.p, sizeof(float) * (size_t)Lo * D);
    finish(c);
  });
}

int32_t rvc_cuda_protect(int64_t ctx, const float* feats, const float* feats0, const float* pitchf, int64_t P,
                         int32_t D, float protect, float* out) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(feats && feats0 && pitchf && out && P >= 0 && D >= 1, "protect: bad arguments");
    if (P == 0) return;
    const size_t nb = sizeof(float) * (size_t)P * D;
    DevBuf df(c, nb), df0(c, nb), dp(c, sizeof(float) * P), dout(c, nb);
    h2d(c, df.p, feats, nb);
    h2d(c, df0.p, feats0, nb);
    h2d(c, dp.p, pitchf, sizeof(float) * P);
    dsp_protect(c, df.f(), df0.f(), dp.f(), P, D, protect, dout.f());
    d2h(c, out, dout.p, nb);
    finish(c);
  });
}

int32_t rvc_cuda_change_rms(int64_t ctx, const float* d1, int64_t n1, int32_t sr1, const float* d2, int64_t n2,
                            int32_t sr2, double rate, float* out) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(d1 && d2 && out && n1 >= 0 && n2 >= 0, "change_rms: bad arguments");
    if (n2 == 0) return;
    DevBuf a(c, sizeof(float) * (size_t)std::max<int64_t>(1, n1)), b(c, sizeof(float) * (size_t)n2),
        o(c, sizeof(float) * (size_t)n2);
    h2d(c, a.p, d1, sizeof(float) * n1);
    h2d(c, b.p, d2, sizeof(float) * n2);
    dsp_change_rms(c, a.f(), n1, sr1, b.f(), n2, sr2, rate, o.f());
    d2h(c, out, o.p, sizeof(float) * n2);
    finish(c);
  });
}

int32_t rvc_cuda_f0_autocorr(int64_t ctx, const double* x, int64_t n, int32_t sr, int32_t hop, int32_t win,
                             int32_t lag_min, int32_t lag_max, const double* hann, double threshold, float* f0,
                             int64_t n_frames) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(x && hann && f0 && n >= 1 && sr >= 1 && n_frames >= 0, "f0_autocorr: bad arguments");
    DevBuf dx(c, sizeof(double) * (size_t)n), dw(c, sizeof(double) * (size_t)std::max(1, win)),
        df(c, sizeof(float) * (size_t)std::max<int64_t>(1, n_frames));
    h2d(c, dx.p, x, sizeof(double) * n);
    h2d(c, dw.p, hann, sizeof(double) * (size_t)win);
    dsp_f0_autocorr(c, (const double*)dx.p, n, hop, win, lag_min, lag_max, (const double*)dw.p, (double)sr,
                    threshold, df.f(), n_frames);
    d2h(c, f0, df.p, sizeof(float) * (size_t)n_frames);
    finish(c);
  });
}

int32_t rvc_cuda_interp_linear_device(int64_t ctx, const float* x, int64_t L, int32_t D, double scale, float* y,
                                      int64_t Lo) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(x && y && L >= 1 && D >= 1 && scale > 0.0 && Lo == (int64_t)((double)L * scale),
                  "interp_linear: bad arguments (Lo must be int(L * scale))");
    dsp_interp_time(c, x, L, D, scale, y, Lo);
  });
}

int32_t rvc_cuda_protect_device(int64_t ctx, const float* feats, const float* feats0, const float* pitchf, int64_t P,
                                int32_t D, float protect, float* out) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(feats && feats0 && pitchf && out && P >= 0 && D >= 1, "protect: bad arguments");
    if (P) dsp_protect(c, feats, feats0, pitchf, P, D, protect, out);
  });
}

int32_t rvc_cuda_change_rms_device(int64_t ctx, const float* d1, int64_t n1, int32_t sr1, const float* d2, int64_t n2,
                                   int32_t sr2, double rate, float* out) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(d1 && d2 && out && n1 >= 0 && n2 >= 0, "change_rms: bad arguments");
    dsp_change_rms(c, d1, n1, sr1, d2, n2, sr2, rate, out);
  });
}

int32_t rvc_cuda_to_int16_device(int64_t ctx, const float* x, int64_t n, int16_t* y) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(x && y && n >= 0, "to_int16: bad arguments");
    if (n) dsp_to_int16(c, x, n, (short*)y);
  });
}

int32_t rvc_cuda_resample(int64_t ctx, const void* x, int32_t x_f32, int64_t n_in, int32_t orig_sr,
                          int32_t target_sr, int32_t method, float* y, int64_t n_out) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(x && y && n_in >= 1 && n_out >= 1 && orig_sr > 0 && target_sr > 0, "resample: bad arguments");
    DevBuf dx(c, sizeof(double) * (size_t)n_in), dy(c, sizeof(float) * (size_t)n_out);
    if (x_f32) {
      DevBuf xf(c, sizeof(float) * (size_t)n_in);
      h2d(c, xf.p, x, sizeof(float) * n_in);
      dsp_f32_to_f64(c, xf.f(), n_in, (double*)dx.p);
      RVC_CUDA_TRY(cudaStreamSynchronize(c->stream));
    } else {
      h2d(c, dx.p, x, sizeof(double) * n_in);
    }
    // the fft method's bin-position factor, formed as the reference does: (n_in * sr_out) / (sr_in * n_out)
    const double factor = (double)(n_in * (int64_t)target_sr) / (double)((int64_t)orig_sr * n_out);
    dsp_resample(c, (const double*)dx.p, n_in, n_out, method, factor, dy.f());
    d2h(c, y, dy.p, sizeof(float) * (size_t)n_out);
    finish(c);
  });
}

int32_t rvc_cuda_to_int16(int64_t ctx, const float* x, int64_t n, int16_t* y) {
  return on_ctx(ctx, [&](Context* c) {
    RVC_CHECK_ARG(x && y && n >= 1, "to_int16: bad arguments");
    DevBuf dx(c, sizeof(float) * (size_t)n), dy(c, sizeof(int16_t) * (size_t)n);
    h2d(c, dx.p, x, dx.bytes);
    dsp_to_int16(c, dx.f(), n, (short*)dy.p);
    d2h(c, y, dy.p, dy.bytes);
    finish(c);
  });
}

}  // extern "C"
