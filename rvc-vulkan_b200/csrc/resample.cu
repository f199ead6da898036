// Output resampling on the device: runtime/dsp/resample.py (resample :129).
//
//  * fft (the pipeline's method, runtime/pipeline.py:1204-1205): the rfft of
//    the whole signal, the spectrum interpolated at the target bins' source
//    positions p_k = k * n_in sr_out / (sr_in n_out) with a 33-tap Kaiser-
//    windowed sinc (beta 12) over the edge-padded spectrum, zero above the
//    source Nyquist, irfft to n_out samples, scaled by n_out / n_in.  The two
//    transforms are cuFFT double-precision plans (plain FFTs); the spectral
//    interpolation is this file's kernel.  I0 is evaluated from its power
//    series.
//  * sinc: the time-domain 25-tap Kaiser-sinc interpolation (radius 12).
//  * linear: np.interp on np.linspace(0, n_in - 1, n_out).
// Everything is float64 as in the reference; the result is rounded to float32.
#include "context.cuh"
#include "kernels.cuh"

#include <cufft.h>

#include <algorithm>
#include <cmath>

namespace rvc {

namespace {

// Modified Bessel function of the first kind, order 0: sum_k ((z/2)^2)^k / (k!)^2.
__device__ double bessel_i0(double z) {
  const double q = 0.25 * z * z;
  double term = 1.0, sum = 1.0;
  for (int k = 1; k < 200; ++k) {
    term *= q / ((double)k * (double)k);
    sum += term;
    if (term < 1e-17 * sum) break;
  }
  return sum;
}

// np.sinc(t) * kaiser(t / radius) (runtime/dsp/resample.py:_kaiser_window_sinc)
__device__ double kaiser_sinc(double t, int radius, double beta, double i0_beta) {
  const double x = t / (double)radius;
  double kw = 0.0;
  if (fabs(x) <= 1.0) kw = bessel_i0(beta * sqrt(fmax(0.0, 1.0 - x * x))) / i0_beta;
  const double y = M_PI * (t == 0.0 ? 1.0e-20 : t);
  return sin(y) / y * kw;
}

__global__ void spectrum_interp_kernel(const double2* __restrict__ X, long long nbi, double2* __restrict__ Y,
                                       long long nbo, double factor, int radius, double beta, bool even_out) {
  const double i0b = bessel_i0(beta);
  const int pad = radius + 1;
  for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < nbo;
       k += (long long)gridDim.x * blockDim.x) {
    const double p = (double)k * factor;
    double re = 0.0, im = 0.0;
    if (p <= (double)(nbi - 1)) {
      const double pp = p + (double)pad;
      const long long fl = (long long)floor(pp);
      for (int j = -radius; j <= radius; ++j) {
        const long long b = fl + j;
        const double w = kaiser_sinc(pp - (double)b, radius, beta, i0b);
        long long src = b - pad;  // edge padding of the spectrum
        src = src < 0 ? 0 : (src > nbi - 1 ? nbi - 1 : src);
        re += X[src].x * w;
        im += X[src].y * w;
      }
    }
    // irfft ignores the imaginary parts of the DC and Nyquist bins
    if (k == 0 || (even_out && k == nbo - 1)) im = 0.0;
    Y[k] = make_double2(re, im);
  }
}

__global__ void scale_to_f32_kernel(const double* __restrict__ y, long long n, double inv_n, double gain,
                                    float* __restrict__ out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] = (float)((y[i] * inv_n) * gain);
}

__global__ void resample_sinc_kernel(const double* __restrict__ x, long long n_in, long long n_out, double ratio,
                                     int radius, double beta, float* __restrict__ out) {
  const double i0b = bessel_i0(beta);
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < n_out;
       j += (long long)gridDim.x * blockDim.x) {
    const double pos = (double)j * ratio;
    const long long base = (long long)pos;
    double acc = 0.0;
    for (int k = -radius; k <= radius; ++k) {
      long long idx = base + k;
      idx = idx < 0 ? 0 : (idx > n_in - 1 ? n_in - 1 : idx);
      acc = __dadd_rn(acc, __dmul_rn(x[idx], kaiser_sinc(pos - (double)(base + k), radius, beta, i0b)));
    }
    out[j] = (float)acc;
  }
}

// np.interp(np.linspace(0, n_in - 1, n_out), np.arange(n_in), x)
__global__ void resample_linear_kernel(const double* __restrict__ x, long long n_in, long long n_out, double step,
                                       float* __restrict__ out) {
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < n_out;
       j += (long long)gridDim.x * blockDim.x) {
    const double xv = (j == n_out - 1 && n_out > 1) ? (double)(n_in - 1) : __dmul_rn((double)j, step);
    long long i = (long long)floor(xv);
    i = i < 0 ? 0 : (i > n_in - 1 ? n_in - 1 : i);
    double r;
    if (i == n_in - 1 || (double)i == xv) {
      r = x[i];
    } else {
      const double slope = __dsub_rn(x[i + 1], x[i]);  // / (xp[i+1] - xp[i]) = / 1
      r = __dadd_rn(__dmul_rn(slope, __dsub_rn(xv, (double)i)), x[i]);
    }
    out[j] = (float)r;
  }
}

int grid_of(long long n) { return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, 148ll * 16)); }

void cufft_try(cufftResult r, const char* what) {
  if (r != CUFFT_SUCCESS) throw Error{kErrCuda, std::string("cuFFT ") + what + " failed (" + std::to_string((int)r) + ")"};
}

struct Plan {
  cufftHandle h = 0;
  bool ok = false;
  ~Plan() {
    if (ok) cufftDestroy(h);
  }
};

}  // namespace

void dsp_resample(Context* ctx, const double* x, long long n_in, long long n_out, int method, double factor,
                  float* y) {
  RVC_CHECK_ARG(n_in >= 1 && n_out >= 1, "resample: empty signal");
  cudaStream_t st = ctx->stream;
  if (method == 1) {  // linear
    const double step = n_out > 1 ? (double)(n_in - 1) / (double)(n_out - 1) : 0.0;
    resample_linear_kernel<<<grid_of(n_out), 256, 0, st>>>(x, n_in, n_out, step, y);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
    return;
  }
  if (method == 2) {  // sinc
    resample_sinc_kernel<<<grid_of(n_out), 256, 0, st>>>(x, n_in, n_out, (double)n_in / (double)n_out, 12, 12.0, y);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
    return;
  }
  RVC_CHECK_ARG(method == 0, "resample: method must be 0 (fft), 1 (linear) or 2 (sinc)");
  RVC_CHECK_ARG(n_in < (1ll << 31) && n_out < (1ll << 31), "resample: signals of at most 2^31 - 1 samples");
  const long long nbi = n_in / 2 + 1, nbo = n_out / 2 + 1;
  DevBuf X(ctx, sizeof(double2) * (size_t)nbi), Y(ctx, sizeof(double2) * (size_t)nbo),
      yr(ctx, sizeof(double) * (size_t)n_out), xin(ctx, sizeof(double) * (size_t)n_in);
  RVC_CUDA_TRY(cudaMemcpyAsync(xin.p, x, sizeof(double) * (size_t)n_in, cudaMemcpyDeviceToDevice, st));
  Plan fwd, inv;
  cufft_try(cufftPlan1d(&fwd.h, (int)n_in, CUFFT_D2Z, 1), "plan (forward)");
  fwd.ok = true;
  cufft_try(cufftPlan1d(&inv.h, (int)n_out, CUFFT_Z2D, 1), "plan (inverse)");
  inv.ok = true;
  cufft_try(cufftSetStream(fwd.h, st), "set stream");
  cufft_try(cufftSetStream(inv.h, st), "set stream");
  cufft_try(cufftExecD2Z(fwd.h, (cufftDoubleReal*)xin.p, (cufftDoubleComplex*)X.p), "forward transform");
  spectrum_interp_kernel<<<grid_of(nbo), 256, 0, st>>>((const double2*)X.p, nbi, (double2*)Y.p, nbo, factor, 16,
                                                       12.0, n_out % 2 == 0);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
  cufft_try(cufftExecZ2D(inv.h, (cufftDoubleComplex*)Y.p, (cufftDoubleReal*)yr.p), "inverse transform");
  scale_to_f32_kernel<<<grid_of(n_out), 256, 0, st>>>((const double*)yr.p, n_out, 1.0 / (double)n_out,
                                                      (double)n_out / (double)n_in, y);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
  RVC_CUDA_TRY(cudaStreamSynchronize(st));  // the plans and buffers are released on return
}

}  // namespace rvc
