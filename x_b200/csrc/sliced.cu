// Per-anchor score of AnchoredSliced (atl/objectives/ats.py:154-169) for all anchors of all slices in one
// kernel, with its backward.
//
// Each anchor i carries a record of P transported positions (float2 slots) at its slice centre:
//   slot ia   a, the transported smoothed anchor position;
//   slot io   the transported unsmoothed position (the source copy of the anchor, ats.py:160-162), or io < 0:
//             the leave-one-out term is then the self term at a (atl/objectives/cmax.py:125-137);
//   slots ip .. ip+3   the transports of x + d e_x, x - d e_x, x + d e_y, x - d e_y of the finite-difference
//             log-determinant (atl/motion/base.py:43-50), or ip < 0 (logdet off).
// and the scalars val (slice density gathered at a), cnt (sources of the anchor's slice and batch minus
// src), vis (exposure correction, optional) and src (1 if the anchor is a source of its own slice, else 0):
//
//   own = src * sum_corners w(a, corner) norm exp(-|corner - c|^2 / (2 sigma^2))      (ats.py:186-200)
//   ls  = log(eps + max(val - own, 0) / max(cnt vis, 1)) + log(max(|det J|, 1e-12))
//
// with c = the own position (corners also within ceil(3 sigma) of its torch.round, half to even) or c = a.
// Products, sums and quotients are rounded one by one in the reference's order (its torch CPU ops), the
// exponential and logarithm are CUDA's.  The backward returns dL/dval and dL/d(record) -- the derivative of
// the record slots that feed the score (a, the own position, the probes).
#include "common.cuh"

namespace atlb {
namespace {

constexpr int kThreads = 256;

struct ScoreConsts {
  int P, ia, io, ip;  // record layout (slots of float2)
  float delta2;       // 2 d of the finite differences
  float two_s2;       // 2 sigma^2
  float norm;         // 1 / (2 pi sigma^2)
  float eps;
  float R;            // ceil(3 sigma)
  float H, W;
};

// Leave-one-out term at a with centre c (cross: corner window around round(c); else c = a), and its
// derivatives d/da (through the bilinear weights and, for the self term, the kernel) and d/dc.
__device__ __forceinline__ float loo_term(const ScoreConsts& K, float2 a, float2 c, bool cross, float2& ga,
                                          float2& gc) {
  const float x0 = floorf(a.x), y0 = floorf(a.y);
  const float ax = sub_rn(a.x, x0), ay = sub_rn(a.y, y0);
  const float cx0 = rintf(c.x), cy0 = rintf(c.y);
  float s = 0.f, gax = 0.f, gay = 0.f, gcx = 0.f, gcy = 0.f;
#pragma unroll
  for (int dy = 0; dy < 2; ++dy) {
    const float wy = dy ? ay : sub_rn(1.f, ay);
#pragma unroll
    for (int dx = 0; dx < 2; ++dx) {
      const float wx = dx ? ax : sub_rn(1.f, ax);
      const float px = add_rn(x0, (float)dx), py = add_rn(y0, (float)dy);
      bool ok = px >= 0.f && px < K.W && py >= 0.f && py < K.H;
      if (cross) ok = ok && fabsf(sub_rn(px, cx0)) <= K.R && fabsf(sub_rn(py, cy0)) <= K.R;
      if (!ok) continue;
      const float ex = sub_rn(px, c.x), ey = sub_rn(py, c.y);
      const float d2 = add_rn(mul_rn(ex, ex), mul_rn(ey, ey));
      const float e = expf(div_rn(-d2, K.two_s2));
      const float w = mul_rn(wx, wy);
      s = add_rn(s, mul_rn(mul_rn(w, K.norm), e));
      const float ke = K.norm * e;
      gax += (dx ? 1.f : -1.f) * wy * ke;  // d w / d a.x = +-wy
      gay += (dy ? 1.f : -1.f) * wx * ke;
      const float f = w * ke * 2.f / K.two_s2;  // d exp(-d2 / 2s^2) / d c = e (corner - c) / s^2
      gcx += f * ex;
      gcy += f * ey;
    }
  }
  if (!cross) {  // c = a: the kernel derivative acts on a as well
    gax += gcx;
    gay += gcy;
    gcx = gcy = 0.f;
  }
  ga = make_float2(gax, gay);
  gc = make_float2(gcx, gcy);
  return s;
}

struct LogDet {
  float ld;
  float jx0, jx1, jy0, jy1, det;
};

__device__ __forceinline__ LogDet logdet(const ScoreConsts& K, const float2* rec) {
  const float2 px = rec[K.ip], mx = rec[K.ip + 1], py = rec[K.ip + 2], my = rec[K.ip + 3];
  LogDet L;
  L.jx0 = div_rn(sub_rn(px.x, mx.x), K.delta2);
  L.jx1 = div_rn(sub_rn(px.y, mx.y), K.delta2);
  L.jy0 = div_rn(sub_rn(py.x, my.x), K.delta2);
  L.jy1 = div_rn(sub_rn(py.y, my.y), K.delta2);
  L.det = sub_rn(mul_rn(L.jx0, L.jy1), mul_rn(L.jx1, L.jy0));
  const float ad = fabsf(L.det);
  L.ld = logf(ad >= 1e-12f ? ad : 1e-12f);
  return L;
}

struct Score {
  float ls, num, nn, own;
  float2 ga, gc;
};

__device__ __forceinline__ Score score(const ScoreConsts& K, const float2* rec, float val, float cnt,
                                       const float* vis, float src, long long i, float ld) {
  Score S;
  S.ga = S.gc = make_float2(0.f, 0.f);
  const float2 a = rec[K.ia];
  S.own = 0.f;
  if (src != 0.f) S.own = mul_rn(src, loo_term(K, a, K.io >= 0 ? rec[K.io] : a, K.io >= 0, S.ga, S.gc));
  const float n = vis ? mul_rn(cnt, vis[i]) : cnt;
  S.nn = n >= 1.f ? n : 1.f;
  S.num = sub_rn(val, S.own);
  const float rho = div_rn(S.num >= 0.f ? S.num : 0.f, S.nn);
  S.ls = add_rn(logf(add_rn(K.eps, rho)), ld);
  return S;
}

__global__ void __launch_bounds__(kThreads) k_score_fwd(ScoreConsts K, long long N, const float2* __restrict__ pos,
                                                        const float* __restrict__ val, const float* __restrict__ cnt,
                                                        const float* __restrict__ vis, const float* __restrict__ src,
                                                        float* __restrict__ ls) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < N; i += stride) {
    const float2* rec = pos + i * K.P;
    const float ld = K.ip >= 0 ? logdet(K, rec).ld : 0.f;
    ls[i] = score(K, rec, val[i], cnt[i], vis, src[i], i, ld).ls;
  }
}

__global__ void __launch_bounds__(kThreads) k_score_bwd(ScoreConsts K, long long N, const float* __restrict__ gls,
                                                        const float2* __restrict__ pos, const float* __restrict__ val,
                                                        const float* __restrict__ cnt, const float* __restrict__ vis,
                                                        const float* __restrict__ src, float* __restrict__ gval,
                                                        float2* __restrict__ gpos) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < N; i += stride) {
    const float2* rec = pos + i * K.P;
    float2* grec = gpos + i * K.P;
    const float g = gls[i];
    const float sw = src[i];
    const Score S = score(K, rec, val[i], cnt[i], vis, sw, i, 0.f);
    const float grho = g / add_rn(K.eps, S.num >= 0.f ? div_rn(S.num, S.nn) : 0.f);
    const float gnum = S.num >= 0.f ? grho / S.nn : 0.f;  // clamp(min=0) passes the gradient where num >= 0
    gval[i] = gnum;
    const float go = -gnum * sw;
    for (int k = 0; k < K.P; ++k) grec[k] = make_float2(0.f, 0.f);
    grec[K.ia] = make_float2(go * S.ga.x, go * S.ga.y);
    if (K.io >= 0) grec[K.io] = make_float2(go * S.gc.x, go * S.gc.y);
    if (K.ip >= 0) {
      const LogDet L = logdet(K, rec);
      const float ad = fabsf(L.det);
      const float gdet = ad >= 1e-12f ? g / L.det : 0.f;  // d log|det| = d det / det
      const float gjx0 = gdet * L.jy1 / K.delta2, gjx1 = -gdet * L.jy0 / K.delta2;
      const float gjy0 = -gdet * L.jx1 / K.delta2, gjy1 = gdet * L.jx0 / K.delta2;
      grec[K.ip] = make_float2(gjx0, gjx1);
      grec[K.ip + 1] = make_float2(-gjx0, -gjx1);
      grec[K.ip + 2] = make_float2(gjy0, gjy1);
      grec[K.ip + 3] = make_float2(-gjy0, -gjy1);
    }
  }
}

// Counts of small keys: out[r][k] = #{n : key[n] == k, mask == NULL or mask[r * N + n] != 0} for R mask rows.
// The histograms of AnchoredSliced (anchors per slice, sources per slice and batch, events per check slice):
// keys of sorted events repeat along a warp, so each warp adds one count per distinct key (__match_any_sync)
// to shared counters, flushed once per block.
constexpr int kCountSmem = 8192;

__global__ void __launch_bounds__(kThreads) k_count_keys(const long long* __restrict__ key, long long N, int nbins,
                                                         const float* __restrict__ mask, int R,
                                                         unsigned long long* __restrict__ out) {
  __shared__ unsigned int hist[kCountSmem];
  const int total = nbins * R;
  const bool sm = total <= kCountSmem;
  if (sm)
    for (int i = threadIdx.x; i < total; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n0 = blockIdx.x * (long long)blockDim.x; n0 < N; n0 += stride) {  // warp-uniform
    const long long n = n0 + threadIdx.x;
    long long k = n < N ? key[n] : -1;
    if (k >= nbins) k = -1;
    const unsigned grp = __match_any_sync(0xffffffffu, k);
    const bool leader = lane == __ffs(grp) - 1;
    for (int r = 0; r < R; ++r) {
      const bool m = k >= 0 && (mask == nullptr || mask[(long long)r * N + n] != 0.f);
      const unsigned c = __popc(__ballot_sync(0xffffffffu, m) & grp);
      if (leader && k >= 0 && c) {
        if (sm) atomicAdd(hist + r * nbins + k, c);
        else atomicAdd(out + (long long)r * nbins + k, (unsigned long long)c);
      }
    }
  }
  __syncthreads();
  if (sm)
    for (int i = threadIdx.x; i < total; i += blockDim.x)
      if (hist[i]) atomicAdd(out + i, (unsigned long long)hist[i]);
}

ScoreConsts score_consts(int P, int ia, int io, int ip, double sigma, double delta, double eps, long long H,
                         long long W) {
  ScoreConsts K;
  K.P = P;
  K.ia = ia;
  K.io = io;
  K.ip = ip;
  K.delta2 = (float)(2 * delta);
  K.two_s2 = (float)(2 * sigma * sigma);
  K.norm = (float)(1.0 / (2 * M_PI * sigma * sigma));
  K.eps = (float)eps;
  K.R = (float)std::ceil(3 * sigma);
  K.H = (float)H;
  K.W = (float)W;
  return K;
}

}  // namespace

int sliced_score(long long N, int P, int ia, int io, int ip, const float* pos, const float* val, const float* cnt,
                 const float* vis, const float* src, double sigma, double delta, double eps, long long H, long long W,
                 float* ls, cudaStream_t s) {
  const ScoreConsts K = score_consts(P, ia, io, ip, sigma, delta, eps, H, W);
  if (N > 0)
    launch(k_score_fwd, clamp_grid(blocks_for(N, kThreads)), kThreads, 0, s, K, N, (const float2*)pos, val, cnt, vis,
           src, ls);
  return launch_status("sliced_score");
}

int sliced_score_bwd(long long N, int P, int ia, int io, int ip, const float* gls, const float* pos, const float* val,
                     const float* cnt, const float* vis, const float* src, double sigma, double delta, double eps,
                     long long H, long long W, float* gval, float* gpos, cudaStream_t s) {
  const ScoreConsts K = score_consts(P, ia, io, ip, sigma, delta, eps, H, W);
  if (N > 0)
    launch(k_score_bwd, clamp_grid(blocks_for(N, kThreads)), kThreads, 0, s, K, N, gls, (const float2*)pos, val, cnt,
           vis, src, gval, (float2*)gpos);
  return launch_status("sliced_score_bwd");
}

int count_keys(const long long* key, long long N, long long nbins, const float* mask, long long R, long long* out,
               cudaStream_t s) {
  cudaMemsetAsync(out, 0, (size_t)(nbins * R) * sizeof(long long), s);
  if (N > 0 && nbins > 0)
    launch(k_count_keys, clamp_grid(blocks_for(N, kThreads)), kThreads, 0, s, key, N, (int)nbins, mask, (int)R,
           (unsigned long long*)out);
  return launch_status("count_keys");
}

}  // namespace atlb
