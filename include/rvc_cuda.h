/* librvc_cuda: B200 (sm_100a) CUDA backend for the RVC inference hot path.
 *
 * C ABI reached from Python through ctypes, the same way the reference reaches
 * its Vulkan engine rvc_core.dll (runtime/_vulkan.py:127-279).  Conventions
 * follow the reference engine's FFI (engine/src/ffi.zig):
 *   - every call returns int32: 0 = ok, < 0 = error code (RVC_E_*);
 *   - the message of the last error of the calling thread is read with
 *     rvc_cuda_last_error (ffi.zig:1110 rvc_last_error; the reference turns
 *     rc != 0 into RuntimeError at runtime/_vulkan.py:320-324);
 *   - objects are opaque int64 handles (ffi.zig:50 rvc_engine_create);
 *   - host pointers are borrowed for the duration of the call only; device
 *     memory belongs to the context that allocated it;
 *   - one context per device; calls on a context are serialised by a mutex
 *     (the reference serialises on _BATCH_LIFECYCLE_LOCK,
 *     runtime/vulkan_ops.py:160); different devices may be driven from
 *     different host threads.
 * No C++ exception crosses this boundary.  All float tensors are float32,
 * C-contiguous, in the reference's layouts unless a function says otherwise.
 */
#ifndef RVC_CUDA_H
#define RVC_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RVC_OK 0
#define RVC_E_ARG (-1)     /* bad argument or shape (Python raises ValueError) */
#define RVC_E_CUDA (-2)    /* CUDA runtime error */
#define RVC_E_TIMEOUT (-3) /* a bounded device wait gave up */
#define RVC_E_STATE (-4)   /* missing weight, freed handle, not finalised */
#define RVC_E_OOM (-5)     /* device allocation failed or over the context cap */

/* ---------------------------------------------------------------- library */
/* Library ABI version (major*100 + minor). */
int32_t rvc_cuda_version(void);
/* Copies the calling thread's last error message (NUL-terminated, truncated to
 * n bytes); returns its full length.  Replaces rvc_last_error (ffi.zig:1110). */
int32_t rvc_cuda_last_error(char* buf, int64_t n);
/* Kernel launches issued by this library so far (process-wide). */
int32_t rvc_cuda_launch_count(int64_t* n);
/* Number of visible CUDA devices. */
int32_t rvc_cuda_device_count(int32_t* n);

/* ---------------------------------------------------------------- context */
/* Creates a context (stream, error flag, workspace) on `device`.
 * Replaces rvc_engine_create / rvc_engine_destroy (ffi.zig:50-74). */
int32_t rvc_cuda_create(int32_t device, int64_t* ctx);
int32_t rvc_cuda_destroy(int64_t ctx);
/* Waits for all work on the context's stream, polling at most timeout_ms
 * (<= 0: 60 s); returns RVC_E_TIMEOUT instead of blocking forever.  Also
 * reports a device-side wait that gave up inside a kernel (RVC_E_TIMEOUT). */
int32_t rvc_cuda_sync(int64_t ctx, int32_t timeout_ms);
/* The context's cudaStream_t, for callers that time work with CUDA events. */
int32_t rvc_cuda_stream(int64_t ctx, void** stream);
/* Caps the bytes the context may hold on the device (0 = no cap); a request
 * over the cap fails with RVC_E_OOM (host-side fault injection for tests). */
int32_t rvc_cuda_set_mem_cap(int64_t ctx, int64_t bytes);
/* Gives the context's cached free device blocks back to the driver; blocks in
 * use are untouched.  Counterpart of VulkanContext.clear_pool
 * (runtime/vulkan_ops.py:618-633), which VC.vc_single calls after every
 * conversion (runtime/vc.py:532-534). */
int32_t rvc_cuda_release_pool(int64_t ctx);
/* Device buffers owned by the context (for device-resident inputs). */
int32_t rvc_cuda_alloc(int64_t ctx, int64_t bytes, void** dptr);
int32_t rvc_cuda_free(int64_t ctx, void* dptr);
int32_t rvc_cuda_h2d(int64_t ctx, void* dst, const void* src, int64_t bytes);
int32_t rvc_cuda_d2h(int64_t ctx, void* dst, const void* src, int64_t bytes);
/* Device-to-device copy, asynchronous on the context's stream. */
int32_t rvc_cuda_d2d(int64_t ctx, void* dst, const void* src, int64_t bytes);
/* Host-to-device copy enqueued on the context's stream without waiting for it
 * (rvc_cuda_h2d waits for the stream).  From page-locked memory
 * (rvc_cuda_host_alloc) the copy runs in stream order after the call returns,
 * so the source must stay unchanged until the next rvc_cuda_sync / rvc_cuda_d2h. */
int32_t rvc_cuda_h2d_async(int64_t ctx, void* dst, const void* src, int64_t bytes);
/* Page-locked host memory (cudaHostAlloc, portable) for rvc_cuda_h2d_async. */
int32_t rvc_cuda_host_alloc(int64_t bytes, void** ptr);
int32_t rvc_cuda_host_free(void* ptr);
/* Per-kernel timing of the tensor-core convolutions: enable, then read the
 * accumulated launch count, device milliseconds and algorithmic FLOPs. */
int32_t rvc_cuda_profile(int64_t ctx, int32_t enable);
int32_t rvc_cuda_profile_read(int64_t ctx, int64_t* launches, double* ms, double* flops);
/* Per-layer breakdown as CSV text (label,launches,ms,flops); returns the full
 * length (>= 0) or an error status. */
int32_t rvc_cuda_profile_dump(int64_t ctx, char* buf, int64_t n);

/* ------------------------------------------------- tier 1: operator module
 * Numpy-semantics operators behind runtime.backend's RVC_BACKEND dispatch
 * (runtime/backend.py:205-319).  Host in, host out. */

/* conv1d, torch semantics: x[B,C,T], w[O,C,K], b[O] or NULL, asymmetric pad.
 * y[B,O,oL], oL = (T+pad_l+pad_r-dil*(K-1)-1)/stride+1.
 * Replaces backend.conv1d (runtime/backend.py:233) / rvc_conv1d (ffi.zig:294). */
int32_t rvc_cuda_conv1d(int64_t ctx, const float* x, int32_t B, int32_t C, int32_t T, const float* w,
                        int32_t O, int32_t K, const float* b, int32_t stride, int32_t pad_l, int32_t pad_r,
                        int32_t dilation, float* y, int32_t oL);
/* conv_transpose1d: x[B,Ci,T], w[Ci,Co,K], b[Co] or NULL,
 * oL = (T-1)*stride - 2*padding + dilation*(K-1) + output_padding + 1.
 * Replaces backend.conv_transpose1d (runtime/backend.py:242) / rvc_conv_t1d (ffi.zig:336). */
int32_t rvc_cuda_conv_transpose1d(int64_t ctx, const float* x, int32_t B, int32_t Ci, int32_t T,
                                  const float* w, int32_t Co, int32_t K, const float* b, int32_t stride,
                                  int32_t padding, int32_t output_padding, int32_t dilation, float* y,
                                  int32_t oL);
/* c[M,N] = a[M,K] @ b[K,N].  Replaces backend.matmul (runtime/backend.py:205) / rvc_matmul (ffi.zig:233). */
int32_t rvc_cuda_matmul(int64_t ctx, const float* a, const float* b, int32_t M, int32_t K, int32_t N,
                        float* c);
/* Row LayerNorm over the last axis (biased variance).  Replaces
 * backend.layer_norm (runtime/backend.py:286) / rvc_layernorm (ffi.zig:575). */
int32_t rvc_cuda_layer_norm(int64_t ctx, const float* x, int64_t rows, int32_t C, const float* gamma,
                            const float* beta, float eps, float* y);
/* 2-D convolution x[B,C,H,W] * w[O,C,KH,KW] (+ b[O] when not NULL), stride
 * (sh, sw), symmetric zero padding (ph, pw) -> y[B,O,Ho,Wo], fp32.  Replaces
 * backend.conv2d (runtime/backend.py:254) / the engine's conv2d. */
int32_t rvc_cuda_conv2d(int64_t ctx, const float* x, int32_t B, int32_t C, int32_t H, int32_t W, const float* w,
                        int32_t O, int32_t KH, int32_t KW, const float* b, int32_t sh, int32_t sw, int32_t ph,
                        int32_t pw, float* y);
/* Row RMSNorm over the last axis: y = x / sqrt(mean(x^2) + eps) * gamma.
 * Replaces backend.rmsnorm (runtime/backend.py:309). */
int32_t rvc_cuda_rmsnorm(int64_t ctx, const float* x, int64_t rows, int32_t C, const float* gamma, float eps,
                         float* y);
/* Row softmax over the last axis.  Replaces backend.softmax (runtime/backend.py:298) / rvc_softmax (ffi.zig:604). */
int32_t rvc_cuda_softmax(int64_t ctx, const float* x, int64_t rows, int32_t C, float* y);
/* Elementwise: op 0 add(a,b), 1 mul(a,b), 2 relu(a), 3 leaky_relu(a, alpha),
 * 4 gelu_erf(a), 5 tanh(a), 6 sigmoid(a).  b may be NULL for unary ops.
 * Replaces backend.add/mul/relu/add_inplace/mul_inplace (runtime/backend.py:212-284). */
int32_t rvc_cuda_elementwise(int64_t ctx, int32_t op, const float* a, const float* b, int64_t n,
                             float alpha, float* y);
/* Row gather y[n,E] = table[ids[n]] (negative ids count from the end).
 * Replaces backend.embedding (runtime/backend.py:263). */
int32_t rvc_cuda_embedding(int64_t ctx, const int64_t* ids, int64_t n, const float* table, int32_t V,
                           int32_t E, float* y);
/* WaveNet gate: x[B,2H,T] (+ g[B,2H,1] or NULL) -> tanh(x[:H]+g[:H]) * sigmoid(x[H:]+g[H:]) -> y[B,H,T]
 * (runtime/models/vits.py:1131-1132; engine/shaders/gating.comp). */
int32_t rvc_cuda_gating(int64_t ctx, const float* x, const float* g, int32_t B, int32_t H, int32_t T,
                        float* y);
/* T5 relative-position self-attention of the text encoder for one layer:
 * q,k,v[B,heads*kc,P] (projected, NCT) + emb_rel_k/v[2*window+1,kc] -> y[B,heads*kc,P]
 * (runtime/models/vits.py:993-1014; engine/shaders/banded_attn_qk/sv.comp). */
int32_t rvc_cuda_rel_attention(int64_t ctx, const float* q, const float* k, const float* v,
                               const float* emb_k, const float* emb_v, int32_t B, int32_t heads,
                               int32_t kc, int32_t P, int32_t window, float* y);
/* rvc_cuda_rel_attention for callers that cannot allocate device memory: no
 * counterpart in the reference.  Same math and layouts, but q, k, v, emb_k,
 * emb_v and y are DEVICE pointers the caller owns, and the intermediates live in
 * one fixed 8 MiB array in device global memory (held by every GPU that loads
 * the library until exit), so the call makes no cudaMalloc/cudaFree.  Requires
 * 4*B*heads*kc*P <= 2^21, else RVC_E_ARG.  Asynchronous on the context stream
 * (rvc_cuda_sync waits).  All calls on a device share the array: calls on
 * different streams of one device race; calls on one context run in order.
 * The first call on a device resolves the array's address (with that device
 * current) and should come before any stream capture on it. */
int32_t rvc_cuda_rel_attention_noalloc(int64_t ctx, const float* q, const float* k, const float* v,
                                       const float* emb_k, const float* emb_v, int32_t B, int32_t heads,
                                       int32_t kc, int32_t P, int32_t window, float* y);
/* im2col of a 1-D conv: x[B,C,T] -> cols[B,oL,C*K] (column index c*K+k).
 * Replaces BatchRunner.im2col_1d (runtime/vulkan_ops.py:2727). */
int32_t rvc_cuda_im2col1d(int64_t ctx, const float* x, int32_t B, int32_t C, int32_t T, int32_t K,
                          int32_t stride, int32_t pad_l, int32_t dilation, int32_t oL, float* cols);

/* ------------------------------------------------ tier 2: synthesizer model
 * Device-resident SynthesizerTrnMs768NSFsid (runtime/models/vits.py:2237-2598):
 * weights uploaded once under their checkpoint keys, weight norm folded on the
 * device, one call runs enc_p + flow + GeneratorNSF for B equal-length chunks. */

/* cfg: {sr, hidden, filter, heads, layers, kc, window, gin, up0, n_ups,
 *       rates[n_ups]..., kernels[n_ups]..., phone_dim, n_spk, precision}
 * precision: 0 = BF16x3 split (parity), 1 = SIMT fp32 (in-library check). */
int32_t rvc_cuda_synth_create(int64_t ctx, const int32_t* cfg, int32_t ncfg, int64_t* model);
int32_t rvc_cuda_synth_destroy(int64_t model);
/* Uploads one checkpoint tensor (key as in the reference state dict). */
int32_t rvc_cuda_synth_set_weight(int64_t model, const char* key, const float* data, const int64_t* shape,
                                  int32_t ndim);
/* Folds weight norm, packs tensor-core operands; required before infer. */
int32_t rvc_cuda_synth_finalize(int64_t model);
/* B chunks of P frames: phone[B,P,phone_dim], pitch[B,P] int64, nsff0[B,P],
 * sid[B] int64, nz[B,hidden,P], ns[B,P*upp] -> wave[B,P*upp].
 * Host buffers; same math as SynthesizerTrn.infer_controlled (vits.py:2551). */
int32_t rvc_cuda_synth_infer(int64_t model, int32_t B, int32_t P, const float* phone, const int64_t* pitch,
                             const float* nsff0, const int64_t* sid, const float* nz, const float* ns,
                             float* wave);
/* rvc_cuda_synth_infer over B chunks in groups of G chunks (each group's
 * result equals rvc_cuda_synth_infer of those chunks): a group's inputs are
 * copied up and its waveforms down on two copy streams while the neighbouring
 * groups compute, so the host<->device traffic overlaps the synthesis.  The
 * batched-decode loop of decode_batch (vits.py:1847-1878) over many chunks. */
int32_t rvc_cuda_synth_infer_grouped(int64_t model, int32_t B, int32_t G, int32_t P, const float* phone,
                                     const int64_t* pitch, const float* nsff0, const int64_t* sid, const float* nz,
                                     const float* ns, float* wave);
/* Same with device pointers (allocated by rvc_cuda_alloc); asynchronous on
 * the context stream (call rvc_cuda_sync before reading `wave`). */
int32_t rvc_cuda_synth_infer_device(int64_t model, int32_t B, int32_t P, const float* phone,
                                    const int64_t* pitch, const float* nsff0, const int64_t* sid,
                                    const float* nz, const float* ns, float* wave);
/* Partial synthesis of one chunk (SynthesizerTrn.infer with skip_head /
 * return_length, runtime/models/vits.py:2404-2420, :2422-2476, :2539-2548):
 * inputs as rvc_cuda_synth_infer with B = 1 -> wave[return_length*upp], the
 * samples of frames [skip_head, skip_head + return_length).  Host buffers. */
int32_t rvc_cuda_synth_infer_partial(int64_t model, int32_t P, int32_t skip_head, int32_t return_length,
                                     const float* phone, const int64_t* pitch, const float* nsff0, const int64_t* sid,
                                     const float* nz, const float* ns, float* wave);
/* Debug taps: copies the named intermediate of the last infer (e.g.
 * "enc.l5", "flow.z", "dec.s2.out") into out (n floats); RVC_E_ARG if unknown. */
int32_t rvc_cuda_synth_tap(int64_t model, const char* name, float* out, int64_t n);
/* Enables recording of debug taps (off by default: taps cost a copy).
 * enable: 0 off, 1 every chunk of the call (chunk-major), 2 + c only chunk c
 * of a batched call (the taps then hold that chunk's data alone). */
int32_t rvc_cuda_synth_keep_taps(int64_t model, int32_t enable);

/* ---------------------------------------------------------------- HuBERT
 * Device-resident HuBERT-base encoder; replaces HubertEncoder.encode /
 * encode_batch (runtime/models/hubert.py:564-589, :593-628) and its pieces
 * _feature_extractor (:658), _feature_projection (:775), _pos_conv_embed
 * (:838), _encoder (:928), _encoder_layer (:1262).
 * precision: 0 = BF16x3 tensor cores (default), 1 = fp32 SIMT check path. */
int32_t rvc_cuda_hubert_create(int64_t ctx, int32_t precision, int64_t* model);
int32_t rvc_cuda_hubert_destroy(int64_t model);
/* Weights by the reference's state-dict key (prefix-stripped transformers
 * names, runtime/models/hubert.py:499-559); the positional conv is given as
 * weight_g/weight_v (or parametrizations.weight.original0/1) and folded on the
 * device, or pre-folded as "_pos_conv_weight" [768,48,128]. */
int32_t rvc_cuda_hubert_set_weight(int64_t model, const char* key, const float* data, const int64_t* shape,
                                   int32_t ndim);
int32_t rvc_cuda_hubert_finalize(int64_t model);
/* Frames L produced for T samples (0 when T is too short for the conv stack). */
int32_t rvc_cuda_hubert_out_len(int64_t T, int64_t* L);
/* B equal-length chunks x [B,T] (host) -> out [B,L,768] (version 2,
 * last_hidden_state) or [B,L,256] (version 1, layer 9 through final_proj);
 * runtime/models/hubert.py:564-589.  Synchronous. */
int32_t rvc_cuda_hubert_encode(int64_t model, int32_t B, int64_t T, const float* x, int32_t version, float* out);
/* Same with device pointers, asynchronous on the context's stream. */
int32_t rvc_cuda_hubert_encode_device(int64_t model, int32_t B, int64_t T, const float* x, int32_t version,
                                      float* out);
/* Debug taps after an encode with taps enabled: "conv0".."conv6" [B,Ti,512],
 * "proj" and "pos" [B*L,768], "layer0".."layer11" [B*L,768]. */
int32_t rvc_cuda_hubert_tap(int64_t model, const char* name, float* out, int64_t n);
int32_t rvc_cuda_hubert_keep_taps(int64_t model, int32_t enable);

/* ---------------------------------------------------------------- RMVPE
 * Device-resident RMVPE F0 estimator; replaces RMVPE.infer_from_audio
 * (runtime/models/rmvpe.py:927-952) with its pieces _extract_mel (:632),
 * mel2hidden (:861), _unet (:727), _conv_block_res (:518), conv_transpose2d
 * (:319), _bgru (:393), decode / to_local_average_cents (:899-925).
 * fp32 throughout (float64 STFT) so the salience argmax follows the reference. */
int32_t rvc_cuda_rmvpe_create(int64_t ctx, int64_t* model);
int32_t rvc_cuda_rmvpe_destroy(int64_t model);
/* Checkpoint tensors under the reference's keys (RMVPE.W). */
int32_t rvc_cuda_rmvpe_set_weight(int64_t model, const char* key, const float* data, const int64_t* shape,
                                  int32_t ndim);
int32_t rvc_cuda_rmvpe_finalize(int64_t model);
/* F = 1 + T / 160 frames for T samples. */
int32_t rvc_cuda_rmvpe_frames(int64_t T, int64_t* F);
/* B equal-length clips x [B,T] (host, 16 kHz, T > 512) -> f0 [B,F] Hz and,
 * when argmax is not NULL, the per-frame salience argmax [B,F].  Synchronous. */
int32_t rvc_cuda_rmvpe_infer(int64_t model, int32_t B, int64_t T, const float* x, float thred, float* f0,
                             int32_t* argmax);
/* Same with device pointers, asynchronous on the context's stream. */
int32_t rvc_cuda_rmvpe_infer_device(int64_t model, int32_t B, int64_t T, const float* x, float thred, float* f0,
                                    int32_t* argmax);
/* Debug taps after an infer with taps enabled: "mel" [B,Fp,128], "enc0".."enc4",
 * "inter", "dec0".."dec4" (channels-last buffers), "cnn" [B,Fp,384],
 * "gru" [B,Fp,512], "salience" [B,Fp,360]; Fp = F rounded up to 32. */
int32_t rvc_cuda_rmvpe_tap(int64_t model, const char* name, float* out, int64_t n);
int32_t rvc_cuda_rmvpe_keep_taps(int64_t model, int32_t enable);

/* ---------------------------------------------------------------- FCPE
 * Device-resident FCPE F0 estimator (CFNaiveMelPE, conv-only); replaces
 * FCPE.infer (runtime/models/fcpe.py:344-369) with _wav2mel (:204), the input
 * stack (:237), the conformer conv layers (:257), _latent (:290) and the local
 * argmax decode (:304).  precision 0 = BF16x3 tensor cores, 1 = fp32 SIMT. */
int32_t rvc_cuda_fcpe_create(int64_t ctx, int32_t precision, int64_t* model);
int32_t rvc_cuda_fcpe_destroy(int64_t model);
/* Checkpoint tensors under the reference's keys (FCPE.W, cent_table included). */
int32_t rvc_cuda_fcpe_set_weight(int64_t model, const char* key, const float* data, const int64_t* shape,
                                 int32_t ndim);
int32_t rvc_cuda_fcpe_finalize(int64_t model);
/* B equal-length clips x [B,T] (host, 16 kHz) -> f0 [B,F] Hz, F = T / 160 + 1,
 * and, when argmax is not NULL, the latent argmax [B,F].  Synchronous. */
int32_t rvc_cuda_fcpe_infer(int64_t model, int32_t B, int64_t T, const float* x, float threshold, float* f0,
                            int32_t* argmax);
/* FCPE.infer with its decoder_mode (runtime/models/fcpe.py:304-342, :344-369):
 * 0 = "local_argmax" (what rvc_cuda_fcpe_infer runs), 1 = "argmax" (the
 * latent-weighted mean of the cents over all 360 bins).  Host buffers. */
int32_t rvc_cuda_fcpe_infer_mode(int64_t model, int32_t B, int64_t T, const float* x, float threshold,
                                 int32_t decoder_mode, float* f0, int32_t* argmax);
/* Same with device pointers, asynchronous on the context's stream. */
int32_t rvc_cuda_fcpe_infer_device(int64_t model, int32_t B, int64_t T, const float* x, float threshold, float* f0,
                                   int32_t* argmax);
/* Debug taps after an infer with taps enabled: "mel" [B,F,128], "stack" and
 * "layer0".."layer5" [B,F,512], "latent" [B,F,360]. */
int32_t rvc_cuda_fcpe_tap(int64_t model, const char* name, float* out, int64_t n);
int32_t rvc_cuda_fcpe_keep_taps(int64_t model, int32_t enable);

/* ---------------------------------------------------------------- retrieval
 * Device-resident feature index for brute-force L2 search; replaces
 * runtime.retrieval.search_l2 (runtime/retrieval.py:35-82), weighted_blend
 * (:85-108) and the pipeline's blend + mix (runtime/pipeline.py:545-551,
 * :563-566).  db [N,D] (host) is copied; precision 0 = tensor-core GEMM with an
 * exact float64 re-rank of the candidates, 1 = fp32 SIMT GEMM (same re-rank). */
int32_t rvc_cuda_index_create(int64_t ctx, const float* db, int64_t N, int32_t D, int32_t precision,
                              int64_t* index);
int32_t rvc_cuda_index_destroy(int64_t index);
/* q [F,D] -> scores [F,k'] (ascending squared L2 distance) and inds [F,k']
 * (int64), k' = min(k, N), 1 <= k <= 16; equal distances keep the lower index
 * first.  Synchronous, host pointers. */
int32_t rvc_cuda_index_search(int64_t index, const float* q, int64_t F, int32_t D, int32_t k, float* scores,
                              int64_t* inds);
/* Same with device pointers, asynchronous on the context's stream. */
int32_t rvc_cuda_index_search_device(int64_t index, const float* q, int64_t F, int32_t D, int32_t k,
                                     float* scores, int64_t* inds);
/* out [F,D] = sum_j w_j db[inds_j] with w = (1/score)^2 normalised (mode 0,
 * runtime/pipeline.py:547-551) or w = 1/max(score,1e-6)^2 normalised (mode 1,
 * weighted_blend); when feats [F,D] is given, out = blend * index_rate +
 * feats * (1 - index_rate) (runtime/pipeline.py:563-566).  Host pointers. */
int32_t rvc_cuda_index_blend(int64_t index, const float* q, int64_t F, int32_t D, int32_t k, int32_t mode,
                             double index_rate, const float* feats, float* out);
int32_t rvc_cuda_index_blend_device(int64_t index, const float* q, int64_t F, int32_t D, int32_t k, int32_t mode,
                                    double index_rate, const float* feats, float* out);
/* Inverted-file (IVF) structure of runtime/ivf_index.py:121-483: centroids
 * [nlist,D] and the bucket of every index row, assignments [N] in [0, nlist)
 * (IVFIndex.centroids / _assignments).  Host pointers. */
int32_t rvc_cuda_index_set_ivf(int64_t index, const float* centroids, int32_t nlist, const int64_t* assignments);
/* runtime/pipeline.py:_ivf_strict_search (:66-161): per query row its nprobe
 * nearest centroids (nprobe clipped to nlist, at most 16), then the k nearest
 * rows of the union of those buckets: scores [F,k] / inds [F,k], inf / -1
 * past the rows the buckets hold.  Host pointers. */
int32_t rvc_cuda_index_ivf_search(int64_t index, const float* q, int64_t F, int32_t D, int32_t k, int32_t nprobe,
                                  float* scores, int64_t* inds);
/* Same as rvc_cuda_index_ivf_blend with device pointers, asynchronous. */
int32_t rvc_cuda_index_ivf_blend_device(int64_t index, const float* q, int64_t F, int32_t D, int32_t k,
                                        int32_t nprobe, double index_rate, const float* feats, float* out);
/* The pipeline's blend (mode 0 above) over the IVF search results
 * (runtime/pipeline.py:523-527, :563-566).  Host pointers. */
int32_t rvc_cuda_index_ivf_blend(int64_t index, const float* q, int64_t F, int32_t D, int32_t k, int32_t nprobe,
                                 double index_rate, const float* feats, float* out);

/* ---------------------------------------------------------------- pipeline DSP
 * The signal-processing steps of Pipeline.pipeline / _vc_prepare run on the
 * device (host pointers, synchronous). */
/* scipy.signal.filtfilt(b, a, x) with padtype 'odd' (padlen 3*max(na, nb)),
 * float64 out; the 48 Hz high-pass of runtime/pipeline.py:49, :765.  x holds
 * float32 samples when x_f32 != 0 (the odd extension is then formed in
 * float32, as scipy does for a float32 signal), else float64. */
int32_t rvc_cuda_filtfilt(int64_t ctx, const double* b, int32_t nb, const double* a, int32_t na, const void* x,
                          int32_t x_f32, int64_t n, double* y);
/* Silence split (runtime/pipeline.py:767-790): for t = step, 2*step, ... < n,
 * the first argmin of the 160-sample absolute sums of the reflect-padded audio
 * over [max(0, t - t_query), min(n, t + t_query)); -1 for an empty window.
 * count = number of t values (<= cap). */
int32_t rvc_cuda_split_points(int64_t ctx, const double* audio, int64_t n, int32_t window, int64_t t_query,
                              int64_t step, int64_t* out, int64_t cap, int64_t* count);
/* runtime.nn.interpolate_linear along time (runtime/nn.py:734-758) of x [L, D]
 * (time-major) -> y [Lo, D], Lo = int(L * scale), float32. */
int32_t rvc_cuda_interp_linear(int64_t ctx, const float* x, int64_t L, int32_t D, double scale, float* y,
                               int64_t Lo);
/* Protect blend (runtime/pipeline.py:594-608): feats * w + feats0 * (1 - w),
 * w = protect where pitchf < 1 else 1; feats, feats0, out [P, D], pitchf [P]. */
int32_t rvc_cuda_protect(int64_t ctx, const float* feats, const float* feats0, const float* pitchf, int64_t P,
                         int32_t D, float protect, float* out);
/* change_rms(data1, data2, sr1, sr2, rate) (runtime/pipeline.py:164-235). */
int32_t rvc_cuda_change_rms(int64_t ctx, const float* d1, int64_t n1, int32_t sr1, const float* d2, int64_t n2,
                            int32_t sr2, double rate, float* out);
/* Autocorrelation f0 ("pm", runtime/dsp/f0.py:24-94): frame i centred on
 * i * hop, win samples (odd), mean removed, skipped (0) when its peak is below
 * 1e-7, weighted by hann [win]; f0 = sr / lag of the largest normalised
 * autocorrelation in [lag_min, lag_max] when above threshold, else 0.
 * x [n] float64 -> f0 [n_frames] float32.  Host pointers. */
int32_t rvc_cuda_f0_autocorr(int64_t ctx, const double* x, int64_t n, int32_t sr, int32_t hop, int32_t win,
                             int32_t lag_min, int32_t lag_max, const double* hann, double threshold, float* f0,
                             int64_t n_frames);
/* Device-pointer forms of interp_linear, protect, change_rms and to_int16
 * (same arguments), asynchronous on the context's stream: the device pipeline
 * keeps a conversion's features and waveform in HBM between the steps. */
int32_t rvc_cuda_interp_linear_device(int64_t ctx, const float* x, int64_t L, int32_t D, double scale, float* y,
                                      int64_t Lo);
int32_t rvc_cuda_protect_device(int64_t ctx, const float* feats, const float* feats0, const float* pitchf, int64_t P,
                                int32_t D, float protect, float* out);
int32_t rvc_cuda_change_rms_device(int64_t ctx, const float* d1, int64_t n1, int32_t sr1, const float* d2, int64_t n2,
                                   int32_t sr2, double rate, float* out);
int32_t rvc_cuda_to_int16_device(int64_t ctx, const float* x, int64_t n, int16_t* y);
/* runtime.dsp.resample.resample (runtime/dsp/resample.py:129): x [n_in]
 * (float32 when x_f32 != 0, else float64) from orig_sr to target_sr ->
 * y [n_out] float32, n_out = max(1, round(n_in * target_sr / orig_sr));
 * method 0 = fft (spectral Kaiser-sinc interpolation, the pipeline's), 1 =
 * linear (np.interp), 2 = sinc (time-domain Kaiser-sinc).  Host pointers. */
int32_t rvc_cuda_resample(int64_t ctx, const void* x, int32_t x_f32, int64_t n_in, int32_t orig_sr,
                          int32_t target_sr, int32_t method, float* y, int64_t n_out);
/* Peak-normalised int16 conversion (runtime/pipeline.py:1208-1213). */
int32_t rvc_cuda_to_int16(int64_t ctx, const float* x, int64_t n, int16_t* y);

#ifdef __cplusplus
}
#endif

#endif /* RVC_CUDA_H */
