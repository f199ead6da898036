// Pipeline signal processing on the device: the steps runtime/pipeline.py
// runs in numpy / scipy around the models.
//
//  * filtfilt (scipy.signal.filtfilt, padtype 'odd', method 'pad'), used for the
//    48 Hz high-pass (runtime/pipeline.py:49, :765).  The IIR recursion runs in
//    float64 in scipy's direct-form-II-transposed order, one thread per block
//    of kIirBlock outputs: each thread starts `warm` samples before its block
//    from a zero state (the first blocks from the true initial state) and runs
//    the recursion through the warm-up, so the state it enters its block with
//    differs from the sequential one by less than 1e-22 of the state's size
//    (warm is derived from the filter's zero-input decay on the host).  A
//    state-space block scan is not used: for this filter (poles at |z| = 0.994,
//    five zeros at z = 1) the DF2T zero-input responses grow to ~3e6 before
//    decaying, and combining block responses through them loses ~1e-5.
//  * silence split points (runtime/pipeline.py:767-790): 160-sample absolute
//    sums in float64 (same accumulation order), first argmin per query window.
//  * x2 linear interpolation of the features (runtime/nn.py:734-758) and the
//    protect blend (runtime/pipeline.py:594-608), float32 in numpy's order.
//  * change_rms (runtime/pipeline.py:164-235) and the int16 conversion
//    (runtime/pipeline.py:1208-1213).
#include "context.cuh"

#include <algorithm>
#include <cmath>
#include <vector>

namespace rvc {

namespace {

constexpr int kIirMax = 8;      // up to 7 states (order-7 filters)
constexpr int kIirBlock = 1024;
constexpr long long kIirMaxWarm = 1ll << 20;

struct IirCoef {
  int n;  // taps (= states + 1)
  double b[kIirMax], a[kIirMax], zi[kIirMax - 1];
};

// One direct-form-II-transposed step in scipy's lfilter order:
// y = z0 + b0 x ; z_k = (z_{k+1} + x b_{k+1}) - y a_{k+1} ; z_last = x b_last - y a_last
template <int N>
__device__ __forceinline__ double df2t(const IirCoef& f, double x, double (&z)[kIirMax - 1]) {
  const double y = __dadd_rn(z[0], __dmul_rn(f.b[0], x));
#pragma unroll
  for (int k = 0; k < N - 2; ++k) z[k] = __dsub_rn(__dadd_rn(z[k + 1], __dmul_rn(x, f.b[k + 1])), __dmul_rn(y, f.a[k + 1]));
  z[N - 2] = __dsub_rn(__dmul_rn(x, f.b[N - 1]), __dmul_rn(y, f.a[N - 1]));
  return y;
}

// Thread k writes y[kL, (k+1)L): it runs the recursion from max(0, kL - warm),
// from zi * (*scale_src) when that is sample 0 and from a zero state otherwise.
template <int N>
__global__ void iir_warm_kernel(const IirCoef f, const double* __restrict__ x, long long n,
                                const double* __restrict__ scale_src, long long L, long long warm,
                                double* __restrict__ y) {
  const long long s = (blockIdx.x * (long long)blockDim.x + threadIdx.x) * L;
  if (s >= n) return;
  const long long e = s + L < n ? s + L : n;
  long long t = s - warm > 0 ? s - warm : 0;
  double z[kIirMax - 1];
#pragma unroll
  for (int i = 0; i < kIirMax - 1; ++i) z[i] = 0.0;
  if (t == 0) {
    const double x0 = *scale_src;
#pragma unroll
    for (int i = 0; i < N - 1; ++i) z[i] = __dmul_rn(f.zi[i], x0);
  }
  // 16-sample chunks through 16-byte loads / stores, the next chunk loaded
  // while this one runs (each thread streams its own segment, so the loads
  // would otherwise stall the recursion); the recursion itself unchanged.
  // t and s are multiples of 16 here (L and warm are), so a chunk lies wholly
  // in the warm-up or wholly in the output range.
  const long long e16 = t + (e - t) / 16 * 16;
  double cur[16], nxt[16];
  auto load16 = [&](long long tt, double (&v)[16]) {
#pragma unroll
    for (int k = 0; k < 16; k += 2) {
      const double2 w = *reinterpret_cast<const double2*>(x + tt + k);
      v[k] = w.x;
      v[k + 1] = w.y;
    }
  };
  if (t < e16) load16(t, cur);
  for (; t < e16; t += 16) {
    if (t + 16 < e16) load16(t + 16, nxt);
    double yv[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) yv[k] = df2t<N>(f, cur[k], z);
    if (t >= s) {
#pragma unroll
      for (int k = 0; k < 16; k += 2) *reinterpret_cast<double2*>(y + t + k) = make_double2(yv[k], yv[k + 1]);
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) cur[k] = nxt[k];
  }
  for (; t < e; ++t) {
    const double yy = df2t<N>(f, x[t], z);
    if (t >= s) y[t] = yy;
  }
}

// odd extension: [2 x0 - x[pl..1], x, 2 x_last - x[n-2 .. n-1-pl]]; for a
// float32 signal scipy forms the extension in float32 (round_f32).
__global__ void odd_ext_kernel(const double* __restrict__ x, long long n, int pl, bool round_f32,
                               double* __restrict__ ext) {
  const long long m = n + 2 * pl;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < m; i += (long long)gridDim.x * blockDim.x) {
    double v;
    if (i < pl) v = 2.0 * x[0] - x[pl - i];
    else if (i < pl + n) v = x[i - pl];
    else v = 2.0 * x[n - 1] - x[n - 2 - (i - pl - n)];
    ext[i] = round_f32 ? (double)(float)v : v;
  }
}

__global__ void reverse_kernel(const double* __restrict__ x, long long n, double* __restrict__ y) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = x[n - 1 - i];
}

__global__ void f32_to_f64_kernel(const float* __restrict__ x, long long n, double* __restrict__ y) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = (double)x[i];
}

// ------------------------------------------------------------------ split
// audio_sum[j] = sum_{i<160} |pad[j + i]| over the reflect-padded signal
// (pad window/2 each side), accumulated in i order as the reference does.
__global__ void abs_window_sum_kernel(const double* __restrict__ x, long long n, int window,
                                      double* __restrict__ sum) {
  const int half = window / 2;
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < n; j += (long long)gridDim.x * blockDim.x) {
    double s = 0.0;
    for (int i = 0; i < window; ++i) {
      long long p = j + i - half;
      if (p < 0) p = -p;
      if (p >= n) p = 2 * (n - 1) - p;
      s += fabs(x[p]);
    }
    sum[j] = s;
  }
}

// One block per query point t = step * (q + 1): first index of the minimum of
// sum[max(0, t - tq) : min(n, t + tq)], or -1 for an empty window.
__global__ void window_argmin_kernel(const double* __restrict__ sum, long long n, long long step, long long tq,
                                     long long* __restrict__ out) {
  const long long t = step * (blockIdx.x + 1);
  const long long lo = t - tq > 0 ? t - tq : 0, hi = t + tq < n ? t + tq : n;
  __shared__ double sv[256];
  __shared__ long long si[256];
  double best = INFINITY;
  long long bi = -1;
  for (long long j = lo + threadIdx.x; j < hi; j += blockDim.x) {
    const double v = sum[j];
    if (v < best || (v == best && j < bi)) {
      best = v;
      bi = j;
    }
  }
  sv[threadIdx.x] = best;
  si[threadIdx.x] = bi;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) {
      const double v = sv[threadIdx.x + o];
      const long long i = si[threadIdx.x + o];
      if (i >= 0 && (si[threadIdx.x] < 0 || v < sv[threadIdx.x] || (v == sv[threadIdx.x] && i < si[threadIdx.x]))) {
        sv[threadIdx.x] = v;
        si[threadIdx.x] = i;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) out[blockIdx.x] = si[0];
}

// ------------------------------------------------------------------ features
// y[i][d] = x[lo][d] * (1 - frac) + x[hi][d] * frac, src = (i + 0.5) / scale - 0.5
// clipped to [0, L-1] in float64, frac rounded to float32 (runtime/nn.py:746-755).
__global__ void interp_time_kernel(const float* __restrict__ x, long long L, int D, long long Lo, double scale,
                                   float* __restrict__ y) {
  const long long total = Lo * D;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long i = e / D;
    const int d = (int)(e - i * D);
    double src = __dsub_rn(__ddiv_rn((double)i + 0.5, scale), 0.5);
    src = fmin(fmax(src, 0.0), (double)(L - 1));
    const long long lo = (long long)floor(src);
    const long long hi = lo + 1 < L - 1 ? lo + 1 : L - 1;
    const float frac = (float)(src - (double)lo);
    y[e] = __fadd_rn(__fmul_rn(x[lo * D + d], __fsub_rn(1.f, frac)), __fmul_rn(x[hi * D + d], frac));
  }
}

// feats * pitchff + feats0 * (1 - pitchff), pitchff = pitchf < 1 ? protect : 1
__global__ void protect_kernel(const float* __restrict__ feats, const float* __restrict__ feats0,
                               const float* __restrict__ pitchf, long long P, int D, float protect,
                               float* __restrict__ out) {
  const long long total = P * D;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const float pf = pitchf[e / D];
    const float w = pf < 1.f ? protect : (pf > 0.f ? 1.f : pf);
    out[e] = __fadd_rn(__fmul_rn(feats[e], w), __fmul_rn(feats0[e], __fsub_rn(1.f, w)));
  }
}

// ------------------------------------------------------------------ rms mix
// rms[f] = sqrt(mean(frame^2)), frames of length sr//2*2 every sr//2 samples of
// the zero-padded signal (pad = frame/2 each side); block per frame.
__global__ void rms_frames_kernel(const float* __restrict__ x, long long n, int sr, float* __restrict__ rms,
                                  long long nframes) {
  const long long f = blockIdx.x;
  if (f >= nframes) return;
  const int fl = sr / 2 * 2, hop = sr / 2, pad = fl / 2;
  double s = 0.0;
  for (int i = threadIdx.x; i < fl; i += blockDim.x) {
    const long long p = f * hop + i - pad;
    if (p >= 0 && p < n) {
      const float v = __fmul_rn(x[p], x[p]);
      s += (double)v;
    }
  }
  __shared__ double red[256];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) rms[f] = sqrtf(__fdiv_rn((float)red[0], (float)fl));
}

__device__ __forceinline__ float interp_size_at(const float* r, long long L, long long i, long long n_out) {
  if (L == n_out) return r[i];
  double src = __dsub_rn(__dmul_rn((double)i + 0.5, (double)L / (double)n_out), 0.5);
  src = fmin(fmax(src, 0.0), (double)(L - 1));
  const long long lo = (long long)floor(src);
  const long long hi = lo + 1 < L - 1 ? lo + 1 : L - 1;
  const double frac = src - (double)lo;
  return (float)__dadd_rn(__dmul_rn((double)r[lo], 1.0 - frac), __dmul_rn((double)r[hi], frac));
}

__global__ void rms_mix_kernel(const float* __restrict__ d2, long long n2, const float* __restrict__ r1, long long L1,
                               const float* __restrict__ r2, long long L2, float e1, float e2,
                               float* __restrict__ out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n2; i += (long long)gridDim.x * blockDim.x) {
    const float a = interp_size_at(r1, L1, i, n2);
    const float b = fmaxf(interp_size_at(r2, L2, i, n2), 1e-6f);
    out[i] = __fmul_rn(d2[i], __fmul_rn(powf(a, e1), powf(b, e2)));
  }
}

// ------------------------------------------------------------------ pm f0
// numpy's pairwise float64 sum (blocks of <= 128 with eight running sums,
// halves rounded down to a multiple of 8 above that), iterative.
__device__ double np_block_sum(const double* a, int n) {  // n <= 128
  if (n < 8) {
    double res = 0.0;
    for (int i = 0; i < n; ++i) res += a[i];
    return res;
  }
  double r[8];
  for (int j = 0; j < 8; ++j) r[j] = a[j];
  int i = 8;
  for (; i < n - (n % 8); i += 8)
    for (int j = 0; j < 8; ++j) r[j] += a[i + j];
  double res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
  for (; i < n; ++i) res += a[i];
  return res;
}

__device__ double np_pairwise_sum(const double* a, int n) {
  // explicit-stack form of sum(a, n) = n <= 128 ? block(a, n) : sum(a, h) + sum(a + h, n - h),
  // h = n / 2 rounded down to a multiple of 8
  struct Frame { int off, n, state; double left; };  // state 0: new, 1: left pending, 2: right pending
  Frame fr[24];
  int top = 0;
  fr[top++] = {0, n, 0, 0.0};
  double ret = 0.0;
  while (top > 0) {
    Frame& f = fr[top - 1];
    bool done = false;
    if (f.n <= 128) {
      ret = np_block_sum(a + f.off, f.n);
      done = true;
    } else {
      const int h = (f.n / 2) - (f.n / 2) % 8;
      if (f.state == 0) {
        f.state = 1;
        fr[top++] = {f.off, h, 0, 0.0};
      } else if (f.state == 1) {  // left finished: its sum is in ret
        f.left = ret;
        f.state = 2;
        fr[top++] = {f.off + h, f.n - h, 0, 0.0};
      } else {                    // right finished
        ret = f.left + ret;
        done = true;
      }
    }
    if (done) --top;
  }
  return ret;
}

// One block per frame (runtime/dsp/f0.py:24-94): the zero-padded window of
// `win` samples centred on i * hop, mean removed (numpy's pairwise mean),
// skipped when its peak is below 1e-7; Hann-weighted; autocorrelation at lag 0
// and at lag_min..lag_max (direct float64 sums); the first lag of the largest
// normalised value, voiced above the threshold: f0 = sr / lag.
__global__ void f0_autocorr_kernel(const double* __restrict__ x, long long n, int hop, int win, int lag_min,
                                   int lag_max, const double* __restrict__ hann, double sr, double thr,
                                   float* __restrict__ f0) {
  extern __shared__ double sm[];
  double* seg = sm;            // [win]
  double* r = sm + win;        // [lag_max + 1]
  __shared__ double s_mean, s_peak;
  const long long i = blockIdx.x;
  const long long s0 = i * hop - win / 2;
  for (int t = threadIdx.x; t < win; t += blockDim.x) {
    const long long p = s0 + t;
    seg[t] = (p >= 0 && p < n) ? x[p] : 0.0;
  }
  __syncthreads();
  if (threadIdx.x == 0) s_mean = np_pairwise_sum(seg, win) / (double)win;
  __syncthreads();
  const double mean = s_mean;
  for (int t = threadIdx.x; t < win; t += blockDim.x) seg[t] = seg[t] - mean;
  __syncthreads();
  if (threadIdx.x == 0) {
    double pk = 0.0;
    for (int t = 0; t < win; ++t) pk = fmax(pk, fabs(seg[t]));
    s_peak = pk;
  }
  __syncthreads();
  if (s_peak < 1e-7) {
    if (threadIdx.x == 0) f0[i] = 0.f;
    return;
  }
  for (int t = threadIdx.x; t < win; t += blockDim.x) seg[t] = seg[t] * hann[t];
  __syncthreads();
  for (int lag = threadIdx.x; lag <= lag_max; lag += blockDim.x) {
    if (lag != 0 && lag < lag_min) continue;
    double acc = 0.0;
    for (int t = 0; t + lag < win; ++t) acc = fma(seg[t], seg[t + lag], acc);
    r[lag] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const double r0 = r[0];
    float out = 0.f;
    if (r0 > 0.0) {
      int best = lag_min;
      double bv = r[lag_min] / r0;
      for (int lag = lag_min + 1; lag <= lag_max; ++lag) {
        const double v = r[lag] / r0;
        if (v > bv) {
          bv = v;
          best = lag;
        }
      }
      if (bv > thr) out = (float)(sr / (double)best);
    }
    f0[i] = out;
  }
}

// ------------------------------------------------------------------ int16
__global__ void absmax_kernel(const float* __restrict__ x, long long n, unsigned int* __restrict__ out) {
  float m = 0.f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(x[i]));
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));  // non-negative floats order as uints
}

__global__ void to_int16_kernel(const float* __restrict__ x, long long n, const unsigned int* __restrict__ amax,
                                short* __restrict__ y) {
  const float am = __fdiv_rn(__uint_as_float(*amax), 0.99f);
  const float scale = am > 1.f ? __fdiv_rn(32768.f, am) : 32768.f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = (short)__float2int_rz(__fmul_rn(x[i], scale));
}

int grid_for(long long n, int block) {
  return (int)std::max<long long>(1, std::min<long long>((n + block - 1) / block, 148ll * 16));
}

void check_launch() {
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

}  // namespace

// ------------------------------------------------------------------ host side
// Filter setup on the host in double: normalised coefficients, lfilter_zi
// (the steady state of a unit step) and the warm-up length.
struct IirPlan {
  IirCoef f{};
  int m = 0;
  long long warm = 0;  // < 0: no decay found, run sequentially
};

static IirPlan iir_plan(const double* b, int nb, const double* a, int na) {
  RVC_CHECK_ARG(na >= 1 && nb >= 1 && a[0] != 0.0, "filtfilt: a[0] must be non-zero");
  const int n = std::max(na, nb);
  RVC_CHECK_ARG(n >= 2 && n <= kIirMax, "filtfilt: filters of 2..8 taps supported");
  IirPlan p;
  p.f.n = n;
  p.m = n - 1;
  for (int i = 0; i < n; ++i) {
    p.f.b[i] = (i < nb ? b[i] : 0.0) / a[0];
    p.f.a[i] = (i < na ? a[i] : 0.0) / a[0];
  }
  const int m = p.m;
  // scipy 1.18's closed form: y_inf = sum(b) / sum(a) (the unit-step output in
  // steady state), zi[k] = sum_{j>k} (b_j - y_inf a_j) summed from the last tap.
  double sb = 0.0, sa = 0.0;
  for (int i = 0; i < n; ++i) {
    sb += p.f.b[i];
    sa += p.f.a[i];
  }
  RVC_CHECK_ARG(sa != 0.0, "filtfilt: filter not stable (sum(a) == 0, a pole at z = 1)");
  const double y_inf = sb / sa;
  double acc = 0.0;
  for (int k = n - 1; k >= 1; --k) {
    acc += p.f.b[k] - y_inf * p.f.a[k];
    p.f.zi[k - 1] = acc;
  }
  // Warm-up: zero-input responses of the m unit states until every state
  // component is below 1e-22 of the largest seen, plus a quarter for margin.
  std::vector<double> z((size_t)m * m, 0.0);
  for (int i = 0; i < m; ++i) z[(size_t)i * m + i] = 1.0;
  double peak = 1.0;
  p.warm = -1;
  for (long long t = 1; t <= kIirMaxWarm; ++t) {
    double cur = 0.0;
    for (int i = 0; i < m; ++i) {
      double* zz = &z[(size_t)i * m];
      const double y = zz[0];
      for (int k = 0; k < m - 1; ++k) zz[k] = zz[k + 1] - y * p.f.a[k + 1];
      zz[m - 1] = -y * p.f.a[m];
      for (int k = 0; k < m; ++k) cur = std::max(cur, std::fabs(zz[k]));
    }
    peak = std::max(peak, cur);
    if (!(cur == cur) || cur > 1e300) break;  // unstable
    if (cur < 1e-22 * peak) {
      p.warm = ((t + t / 4) + 255) / 256 * 256;
      break;
    }
  }
  return p;
}

// lfilter over x[n] (device) from the state zi * (*scale_src) -> y (device).
static void iir_run(Context* ctx, const IirPlan& p, const double* x, long long n, const double* scale_src,
                    double* y) {
  const long long L = p.warm < 0 ? n : kIirBlock, warm = p.warm < 0 ? 0 : p.warm;
  const long long threads = (n + L - 1) / L;
  // one warp per block: the sequential threads spread over as many SMs as possible
  const unsigned grid = (unsigned)((threads + 31) / 32);
  cudaStream_t st = ctx->stream;
  switch (p.f.n) {
#define RVC_IIR_CASE(N) \
  case N: iir_warm_kernel<N><<<grid, 32, 0, st>>>(p.f, x, n, scale_src, L, warm, y); break;
    RVC_IIR_CASE(2) RVC_IIR_CASE(3) RVC_IIR_CASE(4) RVC_IIR_CASE(5) RVC_IIR_CASE(6) RVC_IIR_CASE(7) RVC_IIR_CASE(8)
#undef RVC_IIR_CASE
    default: RVC_CHECK_ARG(false, "filtfilt: filters of 2..8 taps supported");
  }
  check_launch();
}

void dsp_filtfilt(Context* ctx, const double* b, int nb, const double* a, int na, const double* x_dev, long long n,
                  bool ext_f32, double* y_dev) {
  const IirPlan p = iir_plan(b, nb, a, na);
  const int pl = 3 * std::max(na, nb);
  RVC_CHECK_ARG(n > pl, "filtfilt: the input must be longer than padlen = 3 * max(len(a), len(b))");
  cudaStream_t st = ctx->stream;
  const long long m = n + 2 * pl;
  DevBuf ext(ctx, sizeof(double) * m), y1(ctx, sizeof(double) * m), r(ctx, sizeof(double) * m);
  odd_ext_kernel<<<grid_for(m, 256), 256, 0, st>>>(x_dev, n, pl, ext_f32, (double*)ext.p);
  check_launch();
  // forward from zi * ext[0], backward (on the reversed output) from zi * y1[last]
  iir_run(ctx, p, (const double*)ext.p, m, (const double*)ext.p, (double*)y1.p);
  reverse_kernel<<<grid_for(m, 256), 256, 0, st>>>((const double*)y1.p, m, (double*)r.p);
  check_launch();
  iir_run(ctx, p, (const double*)r.p, m, (const double*)r.p, (double*)ext.p);
  // y = reverse(ext)[pl : pl + n]
  reverse_kernel<<<grid_for(m, 256), 256, 0, st>>>((const double*)ext.p, m, (double*)y1.p);
  check_launch();
  RVC_CUDA_TRY(cudaMemcpyAsync(y_dev, (const double*)y1.p + pl, sizeof(double) * n, cudaMemcpyDeviceToDevice, st));
  RVC_CUDA_TRY(cudaStreamSynchronize(st));
}

void dsp_f32_to_f64(Context* ctx, const float* x, long long n, double* y) {
  f32_to_f64_kernel<<<grid_for(n, 256), 256, 0, ctx->stream>>>(x, n, y);
  check_launch();
}

long long dsp_split_points(Context* ctx, const double* audio, long long n, int window, long long t_query,
                           long long step, long long* out_dev) {
  RVC_CHECK_ARG(window >= 2 && step >= 1 && t_query >= 0 && n > window / 2, "split: bad arguments");
  cudaStream_t st = ctx->stream;
  DevBuf sum(ctx, sizeof(double) * (size_t)n);
  abs_window_sum_kernel<<<grid_for(n, 256), 256, 0, st>>>(audio, n, window, (double*)sum.p);
  check_launch();
  const long long nq = n > step ? (n - 1) / step : 0;  // t = step, 2 step, ... < n
  if (nq > 0) {
    window_argmin_kernel<<<(unsigned)nq, 256, 0, st>>>((const double*)sum.p, n, step, t_query, out_dev);
    check_launch();
  }
  RVC_CUDA_TRY(cudaStreamSynchronize(st));
  return nq;
}

void dsp_interp_time(Context* ctx, const float* x, long long L, int D, double scale, float* y, long long Lo) {
  interp_time_kernel<<<grid_for(Lo * D, 256), 256, 0, ctx->stream>>>(x, L, D, Lo, scale, y);
  check_launch();
}

void dsp_protect(Context* ctx, const float* feats, const float* feats0, const float* pitchf, long long P, int D,
                 float protect, float* out) {
  protect_kernel<<<grid_for(P * D, 256), 256, 0, ctx->stream>>>(feats, feats0, pitchf, P, D, protect, out);
  check_launch();
}

void dsp_change_rms(Context* ctx, const float* d1, long long n1, int sr1, const float* d2, long long n2, int sr2,
                    double rate, float* out) {
  RVC_CHECK_ARG(sr1 >= 2 && sr2 >= 2, "change_rms: sample rates must be >= 2");
  if (n2 == 0) return;
  cudaStream_t st = ctx->stream;
  const long long L1 = 1 + n1 / (sr1 / 2), L2 = 1 + n2 / (sr2 / 2);
  DevBuf r1(ctx, sizeof(float) * L1), r2(ctx, sizeof(float) * L2);
  rms_frames_kernel<<<(unsigned)L1, 256, 0, st>>>(d1, n1, sr1, r1.f(), L1);
  check_launch();
  rms_frames_kernel<<<(unsigned)L2, 256, 0, st>>>(d2, n2, sr2, r2.f(), L2);
  check_launch();
  // np.power(r, 1.0 - rate) with a float32 base: the exponent is rounded to float32
  rms_mix_kernel<<<grid_for(n2, 256), 256, 0, st>>>(d2, n2, r1.f(), L1, r2.f(), L2, (float)(1.0 - rate),
                                                   (float)(rate - 1.0), out);
  check_launch();  // r1 / r2 go back to the stream-ordered cache: later work queues behind this
}

void dsp_f0_autocorr(Context* ctx, const double* x, long long n, int hop, int win, int lag_min, int lag_max,
                     const double* hann, double sr, double thr, float* f0, long long n_frames) {
  RVC_CHECK_ARG(hop >= 1 && win >= 3 && win <= 8192 && lag_min >= 1 && lag_min <= lag_max && lag_max < win,
                "f0_autocorr: bad frame / lag parameters");
  if (n_frames <= 0) return;
  const size_t smem = sizeof(double) * ((size_t)win + lag_max + 1);
  if (smem > 48 * 1024)
    RVC_CUDA_TRY(cudaFuncSetAttribute(f0_autocorr_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  f0_autocorr_kernel<<<(unsigned)n_frames, 256, smem, ctx->stream>>>(x, n, hop, win, lag_min, lag_max, hann, sr, thr,
                                                                       f0);
  check_launch();
}

void dsp_to_int16(Context* ctx, const float* x, long long n, short* y) {
  cudaStream_t st = ctx->stream;
  DevBuf am(ctx, sizeof(unsigned int));
  RVC_CUDA_TRY(cudaMemsetAsync(am.p, 0, sizeof(unsigned int), st));
  absmax_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, n, (unsigned int*)am.p);
  check_launch();
  to_int16_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, n, (const unsigned int*)am.p, y);
  check_launch();
}

}  // namespace rvc
