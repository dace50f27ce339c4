// Stage 1 (motion fields linear at the event), the exposure correction and the window counts.
//
//   velocity        Translation / Affine / DenseLinearFlow fields (atl/motion/parametric.py:148-312)
//   velocity_bwd    their gradient w.r.t. theta / the flow grid (torch autograd in the reference)
//   visible_fraction atl/objectives/ats.py:31-50 (16 transports per anchor fused into one thread)
//   window_counts   atl/ops/functional.py:210-217 (binary searches over the (b, t)-sorted events)
//
// The velocity bits feed the plan's cell keys, so the fields are evaluated with torch's eager CPU
// rounding sequence (each op rounded, no FMA; division by a Python scalar is an IEEE division).
#include "common.cuh"
#include "motion_math.cuh"

namespace atlb {
namespace {

constexpr int kThreads = 256;
inline int grid_for(long long n) { return clamp_grid(blocks_for(n, kThreads)); }

__global__ void __launch_bounds__(kThreads) k_velocity(MotionView Mv, const float2* __restrict__ xy,
                                                       const long long* __restrict__ b, long long N,
                                                       float2* __restrict__ v) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N; j += stride) {
    const float2 p = xy[j];
    const long long bj = b[j];
    v[j] = (bj >= 0 && bj < Mv.B) ? motion_field(Mv, p.x, p.y, bj)
                                  : make_float2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
  }
}

// Translation / Affine: per-batch sums of gv (and gv (x) (x - c)); block partials + atomics.
__global__ void __launch_bounds__(kThreads) k_velocity_bwd_param(MotionView Mv, const float2* __restrict__ gv,
                                                                 const float2* __restrict__ xy,
                                                                 const long long* __restrict__ b, long long N,
                                                                 float* __restrict__ gtheta) {
  const int np = Mv.kind == ATLB_MOTION_TRANSLATION ? 2 : 6;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N; j += stride) {
    const float2 g = gv[j];
    if ((g.x == 0.f && g.y == 0.f) || b[j] < 0 || b[j] >= Mv.B) continue;
    float* gt = gtheta + b[j] * np;
    atomicAdd(gt + 0, g.x);
    atomicAdd(gt + 1, g.y);
    if (np == 6) {
      const float2 p = xy[j];
      const float d0 = sub_rn(p.x, Mv.cx), d1 = sub_rn(p.y, Mv.cy);
      atomicAdd(gt + 2, g.x * d0);
      atomicAdd(gt + 3, g.x * d1);
      atomicAdd(gt + 4, g.y * d0);
      atomicAdd(gt + 5, g.y * d1);
    }
  }
}

// DenseLinearFlow: scatter of gv with the 4 bilinear weights into the (B, 2, Hg, Wg) grid gradient.
__global__ void __launch_bounds__(kThreads) k_velocity_bwd_dense(MotionView Mv, const float2* __restrict__ gv,
                                                                 const float2* __restrict__ xy,
                                                                 const long long* __restrict__ b, long long N,
                                                                 float* __restrict__ ggrid) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long plane = Mv.Hg * Mv.Wg;
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N; j += stride) {
    const float2 g = gv[j];
    if ((g.x == 0.f && g.y == 0.f) || b[j] < 0 || b[j] >= Mv.B) continue;
    const float2 p = xy[j];
    DenseTaps T;
    dense_taps(Mv, p.x, p.y, &T);
    float* G = ggrid + b[j] * 2 * plane;
    const long long idx[4] = {T.y0 * Mv.Wg + T.x0, T.y0 * Mv.Wg + T.x1, T.y1 * Mv.Wg + T.x0, T.y1 * Mv.Wg + T.x1};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (T.w[q] == 0.f) continue;
      red_add_f1(G + idx[q], g.x * T.w[q]);
      red_add_f1(G + plane + idx[q], g.y * T.w[q]);
    }
  }
}

// Per-(batch, slice) event counts (ats.py:39-41).  Events are time-sorted, so neighbouring threads hit
// the same counter: counts are aggregated in shared memory first (one global atomic per bin per CTA).
constexpr int kMaxSmemBins = 8192;
__global__ void __launch_bounds__(kThreads) k_slice_counts(const float* __restrict__ t,
                                                           const long long* __restrict__ b, long long N, long long B,
                                                           int n_check, int* __restrict__ counts) {
  __shared__ int hist[kMaxSmemBins];
  const long long nbins = B * n_check;
  const bool use_smem = nbins <= kMaxSmemBins;
  if (use_smem)
    for (long long i = threadIdx.x; i < nbins; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N; j += stride) {
    if (b[j] < 0 || b[j] >= B) continue;
    long long s = (long long)mul_rn(t[j], (float)n_check);  // (ev.t * n_check).long(): truncation
    s = s < 0 ? 0 : (s > n_check - 1 ? n_check - 1 : s);
    if (use_smem) atomicAdd(hist + b[j] * n_check + s, 1);
    else atomicAdd(counts + b[j] * n_check + s, 1);
  }
  __syncthreads();
  if (use_smem)
    for (long long i = threadIdx.x; i < nbins; i += blockDim.x)
      if (hist[i]) atomicAdd(counts + i, hist[i]);
}

__global__ void __launch_bounds__(kThreads) k_visible_fraction(MotionView Mv, const float2* __restrict__ xa,
                                                               const float* __restrict__ ta,
                                                               const long long* __restrict__ ba, long long M,
                                                               const int* __restrict__ counts, int n_check, float tau,
                                                               float wmax, float hmax, float* __restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M; i += stride) {
    const float2 p = xa[i];
    const float ti = ta[i];
    const long long bi = ba[i];
    if (bi < 0 || bi >= Mv.B) {
      out[i] = __int_as_float(0x7fc00000);
      continue;
    }
    out[i] = visible_fraction_one(Mv, p.x, p.y, ti, bi, counts + bi * n_check, n_check, tau, wmax, hmax);
  }
}

__device__ __forceinline__ double event_key(const float* t, const long long* b, long long j) {
  return (double)b[j] * 4.0 + (double)t[j];
}

__global__ void __launch_bounds__(kThreads) k_check_sorted(const float* __restrict__ t,
                                                           const long long* __restrict__ b, long long N,
                                                           int* __restrict__ flag) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j + 1 < N; j += stride) {
    const double k0 = event_key(t, b, j), k1 = event_key(t, b, j + 1);
    if (!(k0 <= k1)) atomicOr(flag, 1);
  }
}

// lower bound: first index with key >= q (left); upper: first index with key > q (right)
template <typename KeyF>
__device__ __forceinline__ long long search(KeyF key, long long N, double q, bool right) {
  long long lo = 0, hi = N;
  while (lo < hi) {
    const long long m = (lo + hi) >> 1;
    const double k = key(m);
    if (right ? (k <= q) : (k < q)) lo = m + 1; else hi = m;
  }
  return lo;
}

__global__ void __launch_bounds__(kThreads) k_window_counts(const float* __restrict__ t,
                                                            const long long* __restrict__ b, long long N,
                                                            const double* __restrict__ sorted_keys,
                                                            const long long* __restrict__ idx, long long M,
                                                            double tau, float* __restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < M; q += stride) {
    const long long i = idx[q];
    if (i < 0 || i >= N) {  // the reference raises on an out-of-range index; flag it with NaN
      out[q] = __int_as_float(0x7fc00000);
      continue;
    }
    const double ki = event_key(t, b, i);
    long long L, R;
    if (sorted_keys) {
      auto key = [&](long long m) { return sorted_keys[m]; };
      L = search(key, N, ki - tau, false);
      R = search(key, N, ki + tau, true);
    } else {
      auto key = [&](long long m) { return event_key(t, b, m); };
      L = search(key, N, ki - tau, false);
      R = search(key, N, ki + tau, true);
    }
    const long long c = R - L - 1;
    out[q] = (float)(c > 0 ? c : 0);
  }
}

}  // namespace

int velocity(const MotionView& Mv, const float* xy, const long long* b, long long N, float* v, cudaStream_t s) {
  if (N > 0) launch(k_velocity, grid_for(N), kThreads, 0, s, Mv, (const float2*)xy, b, N, (float2*)v);
  return launch_status("velocity");
}

int velocity_bwd(const MotionView& Mv, const float* gv, const float* xy, const long long* b, long long N,
                 float* gtheta, cudaStream_t s) {
  const size_t nth = Mv.kind == ATLB_MOTION_DENSE ? (size_t)(Mv.B * 2 * Mv.Hg * Mv.Wg)
                                                  : (size_t)(Mv.B * (Mv.kind == ATLB_MOTION_TRANSLATION ? 2 : 6));
  cudaMemsetAsync(gtheta, 0, nth * sizeof(float), s);
  if (N > 0) {
    if (Mv.kind == ATLB_MOTION_DENSE)
      launch(k_velocity_bwd_dense, grid_for(N), kThreads, 0, s, Mv, (const float2*)gv, (const float2*)xy, b, N, gtheta);
    else
      launch(k_velocity_bwd_param, grid_for(N), kThreads, 0, s, Mv, (const float2*)gv, (const float2*)xy, b, N, gtheta);
  }
  return launch_status("velocity_bwd");
}

int visible_fraction(const MotionView& Mv, const float* xa, const float* ta, const long long* ba, long long M,
                     const float* t, const long long* b, long long N, double tau, long long n_check, float* out,
                     void* scratch, cudaStream_t s) {
  int* counts = (int*)scratch;
  cudaMemsetAsync(counts, 0, (size_t)(Mv.B * n_check) * sizeof(int), s);
  if (N > 0) launch(k_slice_counts, clamp_grid(blocks_for(N, kThreads * 16)), kThreads, 0, s, t, b, N, Mv.B, (int)n_check, counts);
  if (M > 0)
    launch(k_visible_fraction, grid_for(M), kThreads, 0, s, Mv, (const float2*)xa, ta, ba, M, counts, (int)n_check,
                                                        (float)tau, (float)(Mv.W - 1), (float)(Mv.H - 1), out);
  return launch_status("visible_fraction");
}

int window_counts(const float* t, const long long* b, long long N, const long long* idx, long long M, double tau,
                  float* out, void* scratch, cudaStream_t s) {
  int* flag = (int*)scratch;
  cudaMemsetAsync(flag, 0, sizeof(int), s);
  if (N > 1) launch(k_check_sorted, grid_for(N), kThreads, 0, s, t, b, N, flag);
  if (M > 0) launch(k_window_counts, grid_for(M), kThreads, 0, s, t, b, N, nullptr, idx, M, tau, out);
  int host = 0;
  if (cudaMemcpyAsync(&host, flag, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return launch_status("window_counts copy");
  if (cudaStreamSynchronize(s) != cudaSuccess) return launch_status("window_counts sync");
  const int st = launch_status("window_counts");
  if (st) return st;
  if (host) {
    set_error("window_counts: events are not sorted by (b, t); pass sorted keys to atlb_window_counts_keys");
    return ATLB_ERR_UNSORTED;
  }
  return ATLB_OK;
}

int window_counts_keys(const double* keys, long long N, const float* t, const long long* b, const long long* idx,
                       long long M, double tau, float* out, cudaStream_t s) {
  if (M > 0) launch(k_window_counts, grid_for(M), kThreads, 0, s, t, b, N, keys, idx, M, tau, out);
  return launch_status("window_counts_keys");
}

}  // namespace atlb
