// Brute-force L2 retrieval on the device.
//
// Reference semantics: runtime.retrieval.search_l2 (runtime/retrieval.py:35-82):
// dist = (||q||^2 + ||d||^2) - 2 q.d, clamped at 0, the k smallest per query in
// ascending order; the pipeline blend (runtime/pipeline.py:545-551, :563-566)
// and weighted_blend (runtime/retrieval.py:85-108).
//
// Plan per block of query rows:
//   1. q.d for every index row: one tensor-core GEMM (the implicit-GEMM conv
//      kernel with K = 1; the index is its resident "weight", packed once) into
//      a [rows][Npad] fp32 block (Npad = N rounded up to 256, pad rows have
//      ||d||^2 = +inf so they never win);
//   2. a warp per (query, column slice) scans its slice of the row, forms the
//      reference's fp32 distance and keeps the k + 8 smallest (value, index)
//      in registers, then merges lanes (slices keep the GPU full when a block
//      has few rows);
//   3. a warp per query takes the k + 8 smallest of its slices' lists and
//      re-ranks them with the exact distance sum((q - d)^2) in float64, writing
//      the k best, ties to the lower index.
// Step 3 makes the order independent of the GEMM's rounding: the result
// matches the reference wherever the reference's own fp32 rounding does not
// reorder two candidates.
#include "retrieval.cuh"

#include <cfloat>
#include <cmath>
#include <vector>

namespace rvc {

namespace {

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// out[r] = sum_d x[r][d]^2 (fp32), +inf for rows in [n_valid, rows).
__global__ void row_sqnorm_kernel(const float* __restrict__ x, long long rows, long long n_valid, int D,
                                  float* __restrict__ out) {
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  if (r >= n_valid) {
    if (lane == 0) out[r] = INFINITY;
    return;
  }
  float s = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float v = x[r * D + d];
    s = fmaf(v, v, s);
  }
  s = warp_sum_f(s);
  if (lane == 0) out[r] = s;
}

// Lexicographic (value, index, lane) order; the lane makes it total so every
// lane of a warp agrees on the winner.
__device__ __forceinline__ bool before(float d1, int i1, int l1, float d2, int i2, int l2) {
  if (d1 != d2) return d1 < d2;
  if (i1 != i2) return (unsigned)i1 < (unsigned)i2;  // -1 (empty) sorts last
  return l1 < l2;
}

constexpr int kTopkSlices = 16;  // column slices of one query row (candidate lists merged by the re-rank)
constexpr int kSliceCols = 512;  // slice granularity: one warp step (32 lanes x 4 float4 loads)

// Candidate scan, one warp per (query row, column slice [s*slice, (s+1)*slice)):
// the reference's fp32 distance (q2 + d2) - 2 q.d clamped at 0, the KC
// smallest (value, index) of the slice in (value, index) order, written to
// cv / ci [row][slice][KC] (inf / -1 where the slice has fewer entries).
// Splitting a row into slices keeps enough warps (and loads in flight) on the
// GPU when a query block has few rows; the union of the slices' exact lists
// holds the row's exact list, which the re-rank selects.
//
// The warp keeps ONE sorted list, lane j < KC holding the j-th smallest.  An
// element is a candidate only if its distance is <= the list's last value (a
// warp-uniform threshold), so after the list fills almost every element costs
// one compare and a ballot; candidates are inserted one at a time by the whole
// warp (compare, ballot, shift up by one lane).  The threshold before the list
// fills is the KC-th smallest of the first step's 32 lane minima (real
// elements, so at least KC elements of the slice are at or below it).  Ties
// are exact: the insertion compares (value, index).  The distance block is
// streamed once (evict-first loads, the next step's loads issued before this
// step's values are used); d2 is shared by the block's 8 rows through L1.
template <int KC>
__global__ void __launch_bounds__(256, 3) topk_slice_kernel(const float* __restrict__ dot, long long ld,
                                                          const float* __restrict__ q2, const float* __restrict__ d2,
                                                          long long rows, long long npad, long long slice,
                                                          float* __restrict__ cv, int* __restrict__ ci) {
  static_assert(KC <= 32, "one list entry per lane");
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const long long c_begin = (long long)blockIdx.y * slice;
  const long long c_end = min(npad, c_begin + slice);
  float lv = INFINITY;  // this lane's list entry (lane < KC)
  int li = -1;
  float tau = INFINITY;  // candidates: dist <= tau (warp-uniform)
  const float qq = q2[r];
  const float* row = dot + r * ld;
  auto insert = [&](float d, int c) {  // warp-wide; d, c uniform
    const bool gt = lane < KC && before(d, c, 0, lv, li, 0);
    const unsigned gm = __ballot_sync(0xffffffffu, gt);
    if (gm == 0) return;  // not better than the KC-th entry
    const int pos = __ffs(gm) - 1;
    const float uv = __shfl_up_sync(0xffffffffu, lv, 1);
    const int ui = __shfl_up_sync(0xffffffffu, li, 1);
    if (lane == pos) {
      lv = d;
      li = c;
    } else if (lane > pos && lane < KC) {
      lv = uv;
      li = ui;
    }
    tau = fminf(tau, __shfl_sync(0xffffffffu, lv, KC - 1));
  };
  // one warp step: lane columns base + 128 u + (0..3), u = 0..3
  auto load = [&](long long base, float4 (&v)[4], float4 (&n2)[4]) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long c0 = base + 128ll * u;
      if (c0 < c_end) {
        v[u] = __ldcs(reinterpret_cast<const float4*>(row + c0));
        n2[u] = __ldg(reinterpret_cast<const float4*>(d2 + c0));
      } else {
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        n2[u] = make_float4(INFINITY, INFINITY, INFINITY, INFINITY);  // inf: never a candidate
      }
    }
  };
  auto dist_of = [&](float x, float nn) { return fmaxf((qq + nn) - 2.f * x, 0.f); };  // the reference's fp32 order
  auto process = [&](long long base, const float4 (&v)[4], const float4 (&n2)[4]) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float x[4] = {v[u].x, v[u].y, v[u].z, v[u].w}, nn[4] = {n2[u].x, n2[u].y, n2[u].z, n2[u].w};
      float dd[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) dd[e] = dist_of(x[e], nn[e]);
      // one ballot per four elements: most groups hold no candidate
      const float m4 = fminf(fminf(dd[0], dd[1]), fminf(dd[2], dd[3]));
      if (!__any_sync(0xffffffffu, m4 <= tau && m4 < INFINITY)) continue;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float dist = dd[e];
        unsigned m = __ballot_sync(0xffffffffu, dist <= tau && dist < INFINITY);
        while (m) {  // warp-uniform
          const int l = __ffs(m) - 1;
          m &= m - 1;
          const float d = __shfl_sync(0xffffffffu, dist, l);
          const int c = __shfl_sync(0xffffffffu, (int)(base + 128ll * u + e), l);
          if (d <= tau) insert(d, c);
        }
      }
    }
  };
  float4 va[4], na[4], vb[4], nb[4];
  long long base = c_begin + 4ll * lane;
  load(base, va, na);
  {
    // threshold before the list fills: the KC-th smallest lane minimum of the first step
    float mn = INFINITY;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      mn = fminf(mn, fminf(fminf(dist_of(va[u].x, na[u].x), dist_of(va[u].y, na[u].y)),
                           fminf(dist_of(va[u].z, na[u].z), dist_of(va[u].w, na[u].w))));
    }
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {  // bitonic sort of the 32 lane minima, ascending
#pragma unroll
      for (int j = k >> 1; j > 0; j >>= 1) {
        const float o = __shfl_xor_sync(0xffffffffu, mn, j);
        const bool asc = (lane & k) == 0, lower = (lane & j) == 0;
        mn = (asc == lower) ? fminf(mn, o) : fmaxf(mn, o);
      }
    }
    tau = __shfl_sync(0xffffffffu, mn, KC - 1);
  }
  for (; base < c_end; base += 2 * kSliceCols) {
    load(base + kSliceCols, vb, nb);
    process(base, va, na);
    load(base + 2 * kSliceCols, va, na);
    process(base + kSliceCols, vb, nb);
  }
  if (lane < KC) {
    const long long o0 = (r * gridDim.y + blockIdx.y) * KC;
    cv[o0 + lane] = lv;
    ci[o0 + lane] = li;
  }
}

// Re-rank, one warp per query row: the KC smallest (value, index) of the
// row's nsl slice lists (the row's exact candidate list), then the exact
// float64 distance sum((q - d)^2) of each and the k best, ties to the lower
// index.
template <int KC>
__global__ void rerank_kernel(const float* __restrict__ q, const float* __restrict__ db, int D,
                              const float* __restrict__ cv, const int* __restrict__ cidx, int nsl, long long rows,
                              int k, float* __restrict__ scores, long long* __restrict__ inds) {
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float* qr = q + r * D;
  constexpr int kPer = kTopkSlices * KC / 32;  // slice-list entries per lane
  const int total = nsl * KC;
  float mv[kPer];
  int mi[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    mv[j] = e < total ? cv[r * total + e] : INFINITY;
    mi[j] = e < total ? cidx[r * total + e] : -1;
  }
  int ci[KC];
#pragma unroll
  for (int t = 0; t < KC; ++t) {
    float bd = mv[0];
    int bi = mi[0], bj = 0;
#pragma unroll
    for (int j = 1; j < kPer; ++j)
      if (before(mv[j], mi[j], 0, bd, bi, 0)) {
        bd = mv[j];
        bi = mi[j];
        bj = j;
      }
    int bl = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float od = __shfl_xor_sync(0xffffffffu, bd, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
      if (before(od, oi, ol, bd, bi, bl)) {
        bd = od;
        bi = oi;
        bl = ol;
      }
    }
    if (lane == bl) {
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (j == bj) {
          mv[j] = INFINITY;
          mi[j] = -1;
        }
    }
    ci[t] = bi;
  }
  double dd[KC];
#pragma unroll
  for (int j = 0; j < KC; ++j) {
    double s = 0.0;
    if (ci[j] >= 0) {
      const float* dr = db + (long long)ci[j] * D;
      for (int d = lane; d < D; d += 32) {
        const double t = (double)qr[d] - (double)dr[d];
        s = fma(t, t, s);
      }
      s = warp_sum_d(s);
    } else {
      s = INFINITY;
    }
    dd[j] = s;
  }
  if (lane != 0) return;
  bool used[KC];
#pragma unroll
  for (int j = 0; j < KC; ++j) used[j] = false;
  for (int t = 0; t < k; ++t) {
    int best = -1, bc = 0;
    double bd = 0.0;
#pragma unroll
    for (int j = 0; j < KC; ++j) {
      if (used[j] || ci[j] < 0) continue;
      if (best < 0 || dd[j] < bd || (dd[j] == bd && ci[j] < bc)) {
        best = j;
        bd = dd[j];
        bc = ci[j];
      }
    }
#pragma unroll
    for (int j = 0; j < KC; ++j)
      if (j == best) used[j] = true;
    const float sc = best >= 0 ? (float)bd : INFINITY;
    const long long ix = best >= 0 ? (long long)bc : -1;
    scores[r * k + t] = sc;
    inds[r * k + t] = ix;
  }
}

// numpy's float32 sum of a short contiguous row (pairwise_sum for n < 128):
// n < 8 sequential; otherwise eight running sums folded as
// ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)), then the tail in order.
__device__ __forceinline__ float np_sum(const float* a, int n) {
  if (n < 8) {
    float s = 0.f;
    for (int i = 0; i < n; ++i) s += a[i];
    return s;
  }
  float r[8];
  for (int j = 0; j < 8; ++j) r[j] = a[j];
  int i = 8;
  for (; i < n - (n % 8); i += 8)
    for (int j = 0; j < 8; ++j) r[j] += a[i + j];
  float s = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
  for (; i < n; ++i) s += a[i];
  return s;
}

__global__ void blend_kernel(const float* __restrict__ db, int D, const float* __restrict__ scores,
                             const long long* __restrict__ inds, long long rows, int k, int mode, float c_blend,
                             float c_feats, const float* __restrict__ feats, float* __restrict__ out) {
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float w[IndexModel::kMaxK];
  long long ix[IndexModel::kMaxK];
  for (int j = 0; j < k; ++j) {
    const float s = scores[r * k + j];
    ix[j] = inds[r * k + j];
    if (mode == 0) {
      const float t = 1.f / s;  // np.square(1.0 / sc)
      w[j] = t * t;
    } else {
      const float m = fmaxf(s, 1e-6f);  // 1.0 / np.maximum(s, 1e-6) ** 2, valid rows only
      w[j] = ix[j] >= 0 ? 1.f / (m * m) : 0.f;
    }
  }
  const float norm = fmaxf(np_sum(w, k), 1e-12f);
  for (int j = 0; j < k; ++j) w[j] = w[j] / norm;
  for (int d = lane; d < D; d += 32) {
    float acc = 0.f;
    bool first = true;
    for (int j = 0; j < k; ++j) {
      if (ix[j] < 0) continue;
      const float p = db[ix[j] * D + d] * w[j];
      acc = first ? p : acc + p;
      first = false;
    }
    float o = acc;
    if (feats) o = acc * c_blend + feats[r * D + d] * c_feats;
    out[r * D + d] = o;
  }
}

constexpr int kRows = 8;  // warps (query rows) per 256-thread block

// IVF bucket scan: one 256-thread block per query.  The query's rows are the
// union of its nprobe buckets; each warp takes every 8th row, forms the exact
// distance sum((q - v)^2) in float64 and keeps its k best (distance, row) in
// lanes 0..k-1 (ties to the lower row); the 8 lists are merged at the end.
constexpr int kIvfWarps = 8;

__device__ __forceinline__ bool before_d(double d1, int i1, double d2, int i2) {
  if (d1 != d2) return d1 < d2;
  return (unsigned)i1 < (unsigned)i2;  // -1 (empty) sorts last
}

__global__ void ivf_scan_kernel(const float* __restrict__ q, const float* __restrict__ db, int D,
                                const int* __restrict__ rows, const long long* __restrict__ off,
                                const long long* __restrict__ probe, int nprobe, int k,
                                float* __restrict__ scores, long long* __restrict__ inds) {
  extern __shared__ float qs[];
  __shared__ double md[kIvfWarps][IndexModel::kMaxK];
  __shared__ int mi[kIvfWarps][IndexModel::kMaxK];
  const long long f = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = q[f * D + d];
  __syncthreads();
  double bd = INFINITY;
  int bi = -1;
  long long seen = 0;  // running row count over the probed buckets (this warp's share is every 8th)
  for (int p = 0; p < nprobe; ++p) {
    const long long b = probe[f * nprobe + p];
    if (b < 0) continue;
    const long long r0 = off[b], r1 = off[b + 1];
    for (long long r = r0 + ((warp - seen) % kIvfWarps + kIvfWarps) % kIvfWarps; r < r1; r += kIvfWarps) {
      const int g = rows[r];
      const float* v = db + (long long)g * D;
      double s = 0.0;
      for (int d = lane; d < D; d += 32) {
        const double t = (double)qs[d] - (double)v[d];
        s = fma(t, t, s);
      }
      s = warp_sum_d(s);
      const double wd = __shfl_sync(0xffffffffu, bd, k - 1);
      const int wi = __shfl_sync(0xffffffffu, bi, k - 1);
      if (before_d(s, g, wd, wi)) {
        const bool gt = lane < k && before_d(s, g, bd, bi);  // the new entry goes before this lane's
        const unsigned m = __ballot_sync(0xffffffffu, gt);
        const int pos = m ? __ffs(m) - 1 : k;
        const double ud = __shfl_up_sync(0xffffffffu, bd, 1);
        const int ui = __shfl_up_sync(0xffffffffu, bi, 1);
        if (lane < k && lane > pos) {
          bd = ud;
          bi = ui;
        } else if (lane == pos) {
          bd = s;
          bi = g;
        }
      }
    }
    seen += r1 - r0;
  }
  if (lane < k) {
    md[warp][lane] = bd;
    mi[warp][lane] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int head[kIvfWarps];
    for (int w = 0; w < kIvfWarps; ++w) head[w] = 0;
    for (int t = 0; t < k; ++t) {
      int bw = -1;
      for (int w = 0; w < kIvfWarps; ++w) {
        if (head[w] >= k) continue;
        if (bw < 0 || before_d(md[w][head[w]], mi[w][head[w]], md[bw][head[bw]], mi[bw][head[bw]])) bw = w;
      }
      const double dd = md[bw][head[bw]];
      const int ii = mi[bw][head[bw]];
      ++head[bw];
      scores[f * k + t] = ii >= 0 ? (float)dd : INFINITY;
      inds[f * k + t] = ii;
    }
  }
}

}  // namespace

IndexModel::IndexModel(Context* c, const float* db, int64_t n, int d, int prec) : ctx(c), precision(prec) {
  RVC_CHECK_ARG(n >= 1 && d >= 1, "index: N and D must be positive");
  RVC_CHECK_ARG(n < (1ll << 31), "index: at most 2^31 - 1 rows");
  RVC_CHECK_ARG(prec == 0 || prec == 1, "index: precision must be 0 (tensor cores) or 1 (fp32 SIMT)");
  N = n;
  D = d;
  Npad = (n + 255) / 256 * 256;
  cudaStream_t st = ctx->stream;
  db_ = DevBuf(ctx, sizeof(float) * (size_t)N * D);
  RVC_CUDA_TRY(cudaMemcpyAsync(db_.p, db, db_.bytes, cudaMemcpyHostToDevice, st));
  d2_ = DevBuf(ctx, sizeof(float) * (size_t)Npad);
  row_sqnorm_kernel<<<(unsigned)((Npad + kRows - 1) / kRows), 32 * kRows, 0, st>>>(db_.f(), Npad, N, D, d2_.f());
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
  {
    // the GEMM's [C_out = Npad][C_in = D] operand: the index rows plus zero pad rows
    DevBuf padded(ctx, sizeof(float) * (size_t)Npad * D);  // zero-filled
    RVC_CUDA_TRY(cudaMemcpyAsync(padded.p, db_.p, db_.bytes, cudaMemcpyDeviceToDevice, st));
    gemm_.build(ctx, LayerKind::kConv, padded.f(), nullptr, (int)Npad, D, 1, precision == 0);
  }
  if (precision == 0) gemm_.release_fp32();  // the packed tensor-core copy is all the GEMM reads
  RVC_CUDA_TRY(cudaStreamSynchronize(st));
}

void IndexModel::ensure_ws(int64_t rows) {
  if (rows <= ws_rows_) return;
  dot_ = DevBuf();
  dot_ = DevBuf(ctx, sizeof(float) * (size_t)rows * Npad);
  q2_ = DevBuf(ctx, sizeof(float) * (size_t)rows);
  cand_v_ = DevBuf(ctx, sizeof(float) * (size_t)rows * kTopkSlices * (kMaxK + kExtra));
  cand_i_ = DevBuf(ctx, sizeof(int) * (size_t)rows * kTopkSlices * (kMaxK + kExtra));
  sc_ = DevBuf(ctx, sizeof(float) * (size_t)rows * kMaxK);
  ix_ = DevBuf(ctx, sizeof(long long) * (size_t)rows * kMaxK);
  ws_rows_ = rows;
}

namespace {
// Resident 256-thread blocks of topk_slice_kernel<KC> per SM (registers bound it).
int topk_blocks_per_sm(int KC) {
  static int n16 = 0, n24 = 0;
  int& n = KC == 16 ? n16 : n24;
  if (n == 0) {
    int b = 0;
    const cudaError_t e = KC == 16
                              ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, topk_slice_kernel<16>, 32 * kRows, 0)
                              : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, topk_slice_kernel<24>, 32 * kRows, 0);
    n = (e == cudaSuccess && b > 0) ? b : 1;
  }
  return n;
}
}  // namespace

void IndexModel::search_device(const float* q, int64_t F, int k, float* scores, int64_t* inds) {
  RVC_CHECK_ARG(k >= 1 && k <= kMaxK, "index_search: k must be in [1, 16]");
  RVC_CHECK_ARG(F >= 0, "index_search: negative query count");
  if (F == 0) return;
  const int kk = (int)std::min<int64_t>(k, N);
  cudaStream_t st = ctx->stream;
  // query rows per block: the distance block stays within ~2 GiB
  int64_t chunk = std::max<int64_t>(128, ((int64_t)1 << 29) / Npad);
  chunk = std::min<int64_t>(chunk, F);
  ensure_ws(chunk);
  const int KC = kk + kExtra <= 16 ? 16 : 24;
  for (int64_t r0 = 0; r0 < F; r0 += chunk) {
    const int64_t rows = std::min<int64_t>(chunk, F - r0);
    const float* qb = q + r0 * D;
    row_sqnorm_kernel<<<(unsigned)((rows + kRows - 1) / kRows), 32 * kRows, 0, st>>>(qb, rows, rows, D, q2_.f());
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
    ConvIO io;
    io.x = qb; io.x_ld = D; io.x_bs = rows * D; io.T_in = (int)rows;
    io.y = dot_.f(); io.y_ld = (int)Npad; io.y_bs = rows * Npad;
    io.B = 1;
    gemm_.run(ctx, io, precision == 1);
    // column slices per row: the count whose blocks fill the resident block
    // slots' waves best (the scan is bound by HBM: a half-empty last wave is
    // lost bandwidth), fewer slices on a tie
    const long long rb = cdiv<long long>(rows, kRows);
    const long long slots = (long long)ctx->num_sms() * topk_blocks_per_sm(KC);
    long long nsl = 1, slice = Npad;
    {
      double best = -1.0;
      const long long max_sl = std::max<long long>(1, std::min<long long>(kTopkSlices, Npad / kSliceCols));
      for (long long ns = 1; ns <= max_sl; ++ns) {
        const long long sl = cdiv<long long>(cdiv<long long>(Npad, ns), kSliceCols) * kSliceCols;
        const long long n_eff = cdiv<long long>(Npad, sl);  // no empty slice
        const long long blocks = rb * n_eff, waves = cdiv<long long>(blocks, slots);
        const double score = (double)blocks / (double)(waves * slots) - 0.01 * (double)n_eff;
        if (score > best + 1e-9) {
          best = score;
          nsl = n_eff;
          slice = sl;
        }
      }
    }
    const dim3 sgrid((unsigned)((rows + kRows - 1) / kRows), (unsigned)nsl);
    const unsigned grid = (unsigned)((rows + kRows - 1) / kRows);
    if (KC == 16) {
      topk_slice_kernel<16><<<sgrid, 32 * kRows, 0, st>>>(dot_.f(), Npad, q2_.f(), d2_.f(), rows, Npad, slice,
                                                          cand_v_.f(), cand_i_.as<int>());
      note_launch();
      rerank_kernel<16><<<grid, 32 * kRows, 0, st>>>(qb, db_.f(), D, cand_v_.f(), cand_i_.as<int>(), (int)nsl, rows,
                                                     kk, scores + r0 * kk, (long long*)inds + r0 * kk);
    } else {
      topk_slice_kernel<24><<<sgrid, 32 * kRows, 0, st>>>(dot_.f(), Npad, q2_.f(), d2_.f(), rows, Npad, slice,
                                                          cand_v_.f(), cand_i_.as<int>());
      note_launch();
      rerank_kernel<24><<<grid, 32 * kRows, 0, st>>>(qb, db_.f(), D, cand_v_.f(), cand_i_.as<int>(), (int)nsl, rows,
                                                     kk, scores + r0 * kk, (long long*)inds + r0 * kk);
    }
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
  }
}

void IndexModel::blend_device(const float* q, int64_t F, int k, int mode, float c_blend, float c_feats,
                              const float* feats, float* out) {
  RVC_CHECK_ARG(mode == 0 || mode == 1, "index_blend: mode must be 0 (pipeline) or 1 (weighted_blend)");
  RVC_CHECK_ARG(k >= 1 && k <= kMaxK, "index_blend: k must be in [1, 16]");
  if (F == 0) return;
  const int kk = (int)std::min<int64_t>(k, N);
  int64_t chunk = std::max<int64_t>(128, ((int64_t)1 << 29) / Npad);
  chunk = std::min<int64_t>(chunk, F);
  ensure_ws(chunk);
  cudaStream_t st = ctx->stream;
  for (int64_t r0 = 0; r0 < F; r0 += chunk) {
    const int64_t rows = std::min<int64_t>(chunk, F - r0);
    search_device(q + r0 * D, rows, kk, sc_.f(), ix_.as<int64_t>());
    blend_kernel<<<(unsigned)((rows + kRows - 1) / kRows), 32 * kRows, 0, st>>>(
        db_.f(), D, sc_.f(), ix_.as<long long>(), rows, kk, mode, c_blend, c_feats, feats ? feats + r0 * D : nullptr,
        out + r0 * D);
    note_launch();
    RVC_CUDA_TRY(cudaGetLastError());
  }
}

void IndexModel::set_ivf(const float* centroids, int nl, const int64_t* assignments) {
  RVC_CHECK_ARG(nl >= 1 && centroids && assignments, "index_set_ivf: need nlist >= 1 centroids and assignments");
  std::vector<int64_t> cnt((size_t)nl + 1, 0);
  for (int64_t i = 0; i < N; ++i) {
    RVC_CHECK_ARG(assignments[i] >= 0 && assignments[i] < nl, "index_set_ivf: assignment " +
                                                                   std::to_string(assignments[i]) + " of row " +
                                                                   std::to_string(i) + " outside [0, nlist)");
    ++cnt[(size_t)assignments[i] + 1];
  }
  for (int b = 0; b < nl; ++b) cnt[(size_t)b + 1] += cnt[(size_t)b];
  std::vector<int> order((size_t)N);
  std::vector<int64_t> fill(cnt.begin(), cnt.end() - 1);
  for (int64_t i = 0; i < N; ++i) order[(size_t)fill[(size_t)assignments[i]]++] = (int)i;  // stable, like argsort(kind="stable")
  cent_ = std::make_unique<IndexModel>(ctx, centroids, nl, D, precision);
  cudaStream_t st = ctx->stream;
  bucket_rows_ = DevBuf(ctx, sizeof(int) * (size_t)N);
  bucket_off_ = DevBuf(ctx, sizeof(int64_t) * ((size_t)nl + 1));
  RVC_CUDA_TRY(cudaMemcpyAsync(bucket_rows_.p, order.data(), bucket_rows_.bytes, cudaMemcpyHostToDevice, st));
  RVC_CUDA_TRY(cudaMemcpyAsync(bucket_off_.p, cnt.data(), bucket_off_.bytes, cudaMemcpyHostToDevice, st));
  RVC_CUDA_TRY(cudaStreamSynchronize(st));
  nlist = nl;
}

void IndexModel::ivf_search_device(const float* q, int64_t F, int k, int nprobe, float* scores, int64_t* inds) {
  RVC_CHECK_ARG(nlist > 0, "index_ivf_search: the index has no IVF structure (set_ivf first)");
  RVC_CHECK_ARG(k >= 1 && k <= kMaxK, "index_ivf_search: k must be in [1, 16]");
  RVC_CHECK_ARG(nprobe >= 1, "index_ivf_search: nprobe must be >= 1");
  RVC_CHECK_ARG(D <= 8192, "index_ivf_search: D above 8192");
  nprobe = std::min(nprobe, nlist);
  RVC_CHECK_ARG(nprobe <= kMaxK, "index_ivf_search: nprobe above 16 is not served");
  if (F == 0) return;
  if (F > probe_rows_) {
    probe_sc_ = DevBuf();
    probe_ix_ = DevBuf();
    probe_sc_ = DevBuf(ctx, sizeof(float) * (size_t)F * kMaxK);
    probe_ix_ = DevBuf(ctx, sizeof(int64_t) * (size_t)F * kMaxK);
    probe_rows_ = F;
  }
  cent_->search_device(q, F, nprobe, probe_sc_.f(), probe_ix_.as<int64_t>());
  ivf_scan_kernel<<<(unsigned)F, 32 * kIvfWarps, sizeof(float) * (size_t)D, ctx->stream>>>(
      q, db_.f(), D, bucket_rows_.as<int>(), bucket_off_.as<long long>(), probe_ix_.as<long long>(), nprobe, k,
      scores, (long long*)inds);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

void IndexModel::ivf_blend_device(const float* q, int64_t F, int k, int nprobe, float c_blend, float c_feats,
                                  const float* feats, float* out) {
  if (F == 0) return;
  if (F > ivf_rows_) {
    ivf_sc_ = DevBuf();
    ivf_ix_ = DevBuf();
    ivf_sc_ = DevBuf(ctx, sizeof(float) * (size_t)F * kMaxK);
    ivf_ix_ = DevBuf(ctx, sizeof(int64_t) * (size_t)F * kMaxK);
    ivf_rows_ = F;
  }
  ivf_search_device(q, F, k, nprobe, ivf_sc_.f(), ivf_ix_.as<int64_t>());
  blend_kernel<<<(unsigned)((F + kRows - 1) / kRows), 32 * kRows, 0, ctx->stream>>>(
      db_.f(), D, ivf_sc_.f(), ivf_ix_.as<long long>(), F, k, 0, c_blend, c_feats, feats, out);
  note_launch();
  RVC_CUDA_TRY(cudaGetLastError());
}

void IndexModel::ivf_search_host(const float* q, int64_t F, int k, int nprobe, float* scores, int64_t* inds) {
  if (F <= 0) return;
  cudaStream_t st = ctx->stream;
  stage(h_q_, sizeof(float) * (size_t)F * D);
  stage(h_s_, sizeof(float) * (size_t)F * k);
  stage(h_i_, sizeof(int64_t) * (size_t)F * k);
  RVC_CUDA_TRY(cudaMemcpyAsync(h_q_.p, q, sizeof(float) * (size_t)F * D, cudaMemcpyHostToDevice, st));
  ivf_search_device(h_q_.f(), F, k, nprobe, h_s_.f(), h_i_.as<int64_t>());
  RVC_CUDA_TRY(cudaMemcpyAsync(scores, h_s_.p, sizeof(float) * (size_t)F * k, cudaMemcpyDeviceToHost, st));
  RVC_CUDA_TRY(cudaMemcpyAsync(inds, h_i_.p, sizeof(int64_t) * (size_t)F * k, cudaMemcpyDeviceToHost, st));
}

void IndexModel::ivf_blend_host(const float* q, int64_t F, int k, int nprobe, float c_blend, float c_feats,
                                const float* feats, float* out) {
  if (F <= 0) return;
  cudaStream_t st = ctx->stream;
  const size_t nb = sizeof(float) * (size_t)F * D;
  stage(h_q_, nb);
  stage(h_o_, nb);
  RVC_CUDA_TRY(cudaMemcpyAsync(h_q_.p, q, nb, cudaMemcpyHostToDevice, st));
  if (feats) {
    stage(h_f_, nb);
    RVC_CUDA_TRY(cudaMemcpyAsync(h_f_.p, feats, nb, cudaMemcpyHostToDevice, st));
  }
  ivf_blend_device(h_q_.f(), F, k, nprobe, c_blend, c_feats, feats ? h_f_.f() : nullptr, h_o_.f());
  RVC_CUDA_TRY(cudaMemcpyAsync(out, h_o_.p, nb, cudaMemcpyDeviceToHost, st));
}

void IndexModel::stage(DevBuf& b, size_t bytes) {
  if (b.bytes < bytes) {
    b = DevBuf();
    b = DevBuf(ctx, bytes);
  }
}

void IndexModel::search_host(const float* q, int64_t F, int k, float* scores, int64_t* inds) {
  RVC_CHECK_ARG(k >= 1 && k <= kMaxK, "index_search: k must be in [1, 16]");
  if (F <= 0) return;
  const int kk = (int)std::min<int64_t>(k, N);
  cudaStream_t st = ctx->stream;
  stage(h_q_, sizeof(float) * (size_t)F * D);
  stage(h_s_, sizeof(float) * (size_t)F * kk);
  stage(h_i_, sizeof(int64_t) * (size_t)F * kk);
  RVC_CUDA_TRY(cudaMemcpyAsync(h_q_.p, q, sizeof(float) * (size_t)F * D, cudaMemcpyHostToDevice, st));
  search_device(h_q_.f(), F, k, h_s_.f(), h_i_.as<int64_t>());
  RVC_CUDA_TRY(cudaMemcpyAsync(scores, h_s_.p, sizeof(float) * (size_t)F * kk, cudaMemcpyDeviceToHost, st));
  RVC_CUDA_TRY(cudaMemcpyAsync(inds, h_i_.p, sizeof(int64_t) * (size_t)F * kk, cudaMemcpyDeviceToHost, st));
}

void IndexModel::blend_host(const float* q, int64_t F, int k, int mode, float c_blend, float c_feats,
                            const float* feats, float* out) {
  if (F <= 0) return;
  cudaStream_t st = ctx->stream;
  const size_t nb = sizeof(float) * (size_t)F * D;
  stage(h_q_, nb);
  stage(h_o_, nb);
  RVC_CUDA_TRY(cudaMemcpyAsync(h_q_.p, q, nb, cudaMemcpyHostToDevice, st));
  if (feats) {
    stage(h_f_, nb);
    RVC_CUDA_TRY(cudaMemcpyAsync(h_f_.p, feats, nb, cudaMemcpyHostToDevice, st));
  }
  blend_device(h_q_.f(), F, k, mode, c_blend, c_feats, feats ? h_f_.f() : nullptr, h_o_.f());
  RVC_CUDA_TRY(cudaMemcpyAsync(out, h_o_.p, nb, cudaMemcpyDeviceToHost, st));
}

}  // namespace rvc
