// Gaussian splat, forward and backward, over shared-memory image tiles: the B200 replacement of
// splat_gauss_fwd / splat_gauss_bwd (csrc/atl_cpu.cpp:79-131).
//
// Reference semantics: event n with weight w at (x, y) adds w * exp(-(dx^2 + dy^2) / (2 s^2)) / (2 pi s^2) to
// every pixel (xx, yy) of the (2R+1)^2 window around (lround(x), lround(y)) that lies in the image,
// dx = xx - x, dy = yy - y; the backward returns d/dw and d/d(x, y) of sum(gimg * img).
//
// Here:
//   1. events are bucketed by the 32x32-pixel tile of their (clamped) window centre: a counting sort into
//      (x, y, w, index) records, tile-major;
//   2. one CTA per tile keeps the tile plus an R-pixel halo in shared memory.  Forward: one warp per event
//      and one private tile copy per warp, so the window is added with plain conflict-free load-add-stores
//      (no shared atomics); the separable factors exp(-dx^2 k) and exp(-dy^2 k) are evaluated once per
//      column / row (2(2R+1) exponentials instead of (2R+1)^2).  The warp copies are summed and flushed
//      to the image with vectorised red.global.add.v4.f32 (neighbouring tiles overlap by the halo).
//      Backward: the gradient image tile is staged in shared memory, each lane sums its event's window
//      row by row.
// A tap's value is w * exp(-dx^2 k) * exp(-dy^2 k) instead of w * exp(-(dx^2 + dy^2) k): the same pixels,
// values within a few ulp; sums are taken in a different order than the reference's atomics.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "pair_math.cuh"
#include "plan_math.cuh"
#include "scan.cuh"

namespace atlb {
namespace {

constexpr int kTS = 32;          // tile side (pixels)
constexpr int kTSLog = 5;
constexpr int kGThreads = 256;

struct GaussConsts {
  float inv2s2, norm, s2;
};

// 1 / (2 s^2) and 1 / (2 pi s^2) rounded as the reference computes them in fp32 (atl_cpu.cpp:83, 112).
GaussConsts gauss_consts(double sigma) {
  GaussConsts K;
  const float s2 = (float)(sigma * sigma);
  K.s2 = s2;
  volatile float d = 2.f * s2;
  K.inv2s2 = 1.f / d;
  volatile float n = 2.f * (float)M_PI;
  n = n * s2;
  K.norm = 1.f / n;
  return K;
}

// lround (half away from zero) for |x| < 2^23: x - trunc(x) is exact, so the tie test is exact too.
__device__ __forceinline__ int lround_small(float x) {
  const float t = truncf(x);
  const float r = fabsf(x - t) >= 0.5f ? t + copysignf(1.f, x) : t;
  return (int)r;
}

struct GTiles {
  long long B, H, W;
  int tw, th;  // tiles per image row / column
  int R;
  long long ntiles;
};

// The tile of event n, or -1 when it adds nothing: batch index outside [0, B), a non-finite position, a
// window with no pixel in the image, or (skip_zero) a zero weight times the normaliser (atl_cpu.cpp:89).
__device__ __forceinline__ long long gauss_tile(const GTiles& T, float x, float y, float wn, long long bb,
                                                bool skip_zero) {
  if ((skip_zero && wn == 0.f) || bb < 0 || bb >= T.B) return -1;
  if (!(fabsf(x) < 1e18f && fabsf(y) < 1e18f)) return -1;
  const long long cx = lroundf(x), cy = lroundf(y);
  if (cx < -T.R || cx > T.W - 1 + T.R || cy < -T.R || cy > T.H - 1 + T.R) return -1;
  const long long tx = min(max(cx, 0LL), T.W - 1) >> kTSLog, ty = min(max(cy, 0LL), T.H - 1) >> kTSLog;
  return (bb * T.th + ty) * T.tw + tx;
}

// Bucketing is a two-level counting sort: each CTA histograms a contiguous chunk of events in shared
// memory (one global atomic per tile it touches), then reserves one range per tile for its chunk and
// places its events with shared-memory cursors.  Tile counts above kSmemTiles use global counters directly.
constexpr int kSmemTiles = 12288;  // 48 KB of shared counters

__global__ void __launch_bounds__(kGThreads) k_gtile_count(GTiles T, const float2* __restrict__ P,
                                                           const float* __restrict__ Wt,
                                                           const long long* __restrict__ Bi, long long N, float norm,
                                                           bool skip_zero, long long chunk, int* __restrict__ counts) {
  extern __shared__ int hist[];
  const bool sm = T.ntiles <= kSmemTiles;
  if (sm)
    for (int i = threadIdx.x; i < T.ntiles; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const long long n0 = blockIdx.x * chunk, n1 = min(n0 + chunk, N);
  const int lane = threadIdx.x & 31;
  for (long long nb = n0; nb < n1; nb += blockDim.x) {  // warp-uniform: one atomic per distinct tile of a warp
    const long long n = nb + threadIdx.x;
    long long key = -1;
    if (n < n1) {
      const float2 p = P[n];
      key = gauss_tile(T, p.x, p.y, mul_rn(Wt[n], norm), Bi[n], skip_zero);
    }
    const unsigned grp = __match_any_sync(0xffffffffu, key);
    if (key >= 0 && lane == __ffs(grp) - 1) atomicAdd(sm ? hist + key : counts + key, __popc(grp));
  }
  __syncthreads();
  if (sm)
    for (int i = threadIdx.x; i < T.ntiles; i += blockDim.x)
      if (hist[i]) atomicAdd(counts + i, hist[i]);
}

// EV[slot] = (x, y, w, n) in tile order.
__global__ void __launch_bounds__(kGThreads) k_gtile_scatter(GTiles T, const float2* __restrict__ P,
                                                             const float* __restrict__ Wt,
                                                             const long long* __restrict__ Bi, long long N,
                                                             float norm, bool skip_zero, long long chunk,
                                                             const int* __restrict__ start, int* __restrict__ cursor,
                                                             float4* __restrict__ EV) {
  extern __shared__ int hist[];  // counts, then this CTA's base slot per tile
  const bool sm = T.ntiles <= kSmemTiles;
  const long long n0 = blockIdx.x * chunk, n1 = min(n0 + chunk, N);
  if (sm) {
    for (int i = threadIdx.x; i < T.ntiles; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (long long nb = n0; nb < n1; nb += blockDim.x) {  // warp-uniform, as in k_gtile_count
      const long long n = nb + threadIdx.x;
      long long key = -1;
      if (n < n1) {
        const float2 p = P[n];
        key = gauss_tile(T, p.x, p.y, mul_rn(Wt[n], norm), Bi[n], skip_zero);
      }
      const unsigned grp = __match_any_sync(0xffffffffu, key);
      if (key >= 0 && (threadIdx.x & 31) == __ffs(grp) - 1) atomicAdd(hist + key, __popc(grp));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < T.ntiles; i += blockDim.x) {
      const int c = hist[i];
      hist[i] = c ? start[i] + atomicAdd(cursor + i, c) : 0;
    }
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  for (long long nb = n0; nb < n1; nb += blockDim.x) {  // warp-uniform: the lanes of a tile take consecutive slots
    const long long n = nb + threadIdx.x;
    long long key = -1;
    float2 p = make_float2(0.f, 0.f);
    float w = 0.f;
    if (n < n1) {
      p = P[n];
      w = Wt[n];
      key = gauss_tile(T, p.x, p.y, mul_rn(w, norm), Bi[n], skip_zero);
    }
    const unsigned grp = __match_any_sync(0xffffffffu, key);
    const int leader = __ffs(grp) - 1;
    int base = 0;
    if (key >= 0 && lane == leader)
      base = sm ? atomicAdd(hist + key, __popc(grp)) : start[key] + atomicAdd(cursor + key, __popc(grp));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (key < 0) continue;
    EV[base + __popc(grp & ((1u << lane) - 1u))] = make_float4(p.x, p.y, w, __int_as_float((int)n));
  }
}

// Tile geometry: the shared tile covers pixels [ox, ox + side) x [oy, oy + side), side = 32 + 2R, with a
// row pitch of side + 1 floats.
struct TileView {
  int b, ox, oy, side, pitch;
};
__device__ __forceinline__ TileView tile_view(const GTiles& T, long long t) {
  TileView v;
  const long long per = (long long)T.th * T.tw;
  v.b = (int)(t / per);
  const int r = (int)(t - (long long)v.b * per);
  const int ty = r / T.tw, tx = r - ty * T.tw;
  v.ox = (tx << kTSLog) - T.R;
  v.oy = (ty << kTSLog) - T.R;
  v.side = kTS + 2 * T.R;
  v.pitch = v.side + 1;
  return v;
}

// Forward: one event per lane.  RT > 0: compile-time radius (window unrolled); RT == 0: runtime radius.
template <int RT>
__device__ __forceinline__ void splat_event(float* __restrict__ tile, const TileView& v, const GTiles& T,
                                            const GaussConsts& K, float4 q) {
  const int R = RT > 0 ? RT : T.R;
  constexpr int WMAX = RT > 0 ? 2 * RT + 1 : 1;
  const float x = q.x, y = q.y, wn = mul_rn(q.z, K.norm);
  const int cx = (int)lroundf(x), cy = (int)lroundf(y);
  const int lx0 = cx - R - v.ox, ly0 = cy - R - v.oy;  // window origin in the tile
  const bool inside = cx >= 0 && cx < T.W && cy >= 0 && cy < T.H;  // then the whole window is in the tile
  if (RT > 0) {
    float ex[WMAX], ey[WMAX];
#pragma unroll
    for (int d = 0; d < WMAX; ++d) {
      const float dx = sub_rn((float)(cx - R + d), x), dy = sub_rn((float)(cy - R + d), y);
      ex[d] = expf(-mul_rn(mul_rn(dx, dx), K.inv2s2));
      ey[d] = mul_rn(wn, expf(-mul_rn(mul_rn(dy, dy), K.inv2s2)));
    }
    float* row = tile + ly0 * v.pitch + lx0;
    if (inside) {
#pragma unroll
      for (int dy = 0; dy < WMAX; ++dy) {
#pragma unroll
        for (int dx = 0; dx < WMAX; ++dx) atomicAdd(row + dy * v.pitch + dx, ey[dy] * ex[dx]);
      }
    } else {
#pragma unroll
      for (int dy = 0; dy < WMAX; ++dy) {
        const int ly = ly0 + dy;
        if (ly < 0 || ly >= v.side) continue;
#pragma unroll
        for (int dx = 0; dx < WMAX; ++dx) {
          const int lx = lx0 + dx;
          if (lx >= 0 && lx < v.side) atomicAdd(row + dy * v.pitch + dx, ey[dy] * ex[dx]);
        }
      }
    }
  } else {
    const int w = 2 * R + 1;
    for (int dy = 0; dy < w; ++dy) {
      const int ly = ly0 + dy;
      if (ly < 0 || ly >= v.side) continue;
      const float fy = sub_rn((float)(cy - R + dy), y);
      const float ey = mul_rn(wn, expf(-mul_rn(mul_rn(fy, fy), K.inv2s2)));
      for (int dx = 0; dx < w; ++dx) {
        const int lx = lx0 + dx;
        if (lx < 0 || lx >= v.side) continue;
        const float fx = sub_rn((float)(cx - R + dx), x);
        atomicAdd(tile + ly * v.pitch + lx, ey * expf(-mul_rn(mul_rn(fx, fx), K.inv2s2)));
      }
    }
  }
}

// Forward, warp per event with one private tile per warp (no atomics).  The 32 lanes take 32 consecutive
// window taps t (dy = t / w, dx = t % w) per round; with the tile's row pitch = w (mod 32) the round's 32
// addresses fall in 32 distinct banks, and no two lanes of a warp touch the same pixel, so a plain
// load-add-store suffices.  The separable factors exp(-dx^2 k) and w_n exp(-dy^2 k) are computed by lanes
// 0..w-1 (ex2.approx) and fetched with shuffles.  RT: compile-time radius (1..12, w <= 25 <= 32).
template <int RT>
struct WarpTaps {
  static constexpr int WD = 2 * RT + 1, NT = WD * WD, ROUNDS = (NT + 31) / 32, PITCH = kTS + 2 * RT + 1;
  int dy[ROUNDS], dx[ROUNDS], off[ROUNDS];
  __device__ __forceinline__ explicit WarpTaps(int lane) {
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
      const int t = 32 * r + lane;
      dy[r] = t < NT ? t / WD : 0;
      dx[r] = t < NT ? t - (t / WD) * WD : 0;
      off[r] = dy[r] * PITCH + dx[r];
    }
  }
};

template <int RT>
__device__ __forceinline__ void splat_event_warp(float* __restrict__ tile, float* __restrict__ dummy,
                                                 const WarpTaps<RT>& tp, const TileView& v, const GTiles& T, float k2,
                                                 float norm, float x, float y, float w, int lane) {
  using TP = WarpTaps<RT>;
  constexpr int R = RT;
  const float wn = mul_rn(w, norm);
  const int cx = lround_small(x), cy = lround_small(y);  // |x|, |y| < W + R, H + R (bucketed events)
  const int lx0 = cx - R - v.ox, ly0 = cy - R - v.oy;
  const bool inside = cx >= 0 && cx < T.W && cy >= 0 && cy < T.H;  // warp-uniform
  const int l = min(lane, TP::WD - 1);
  const float dx = (float)(cx - R + l) - x, dy = (float)(cy - R + l) - y;
  const float exl = ex2_approx(-(dx * dx) * k2);
  const float eyl = wn * ex2_approx(-(dy * dy) * k2);
  float* org = tile + ly0 * TP::PITCH + lx0;
  if (inside) {
#pragma unroll
    for (int r = 0; r < TP::ROUNDS; ++r) {
      const float val = __shfl_sync(0xffffffffu, eyl, tp.dy[r]) * __shfl_sync(0xffffffffu, exl, tp.dx[r]);
      // lanes past the window's last tap add 0 to their own slot beyond the tile
      float* c = (32 * r + lane < TP::NT) ? org + tp.off[r] : dummy;
      *c += val;
    }
  } else {
#pragma unroll
    for (int r = 0; r < TP::ROUNDS; ++r) {
      const float val = __shfl_sync(0xffffffffu, eyl, tp.dy[r]) * __shfl_sync(0xffffffffu, exl, tp.dx[r]);
      const bool ok = 32 * r + lane < TP::NT && ly0 + tp.dy[r] >= 0 && ly0 + tp.dy[r] < v.side &&
                      lx0 + tp.dx[r] >= 0 && lx0 + tp.dx[r] < v.side;
      float* c = ok ? org + tp.off[r] : dummy;
      *c += val;
    }
  }
  __syncwarp();  // the next event's lanes read pixels this event's lanes wrote
}

template <int RT>
__global__ void __launch_bounds__(kGThreads) k_gsplat_fwd_tiles(GTiles T, GaussConsts K, const float4* __restrict__ EV,
                                                                const int* __restrict__ start,
                                                                float* __restrict__ img, bool vec4, int nwt) {
  extern __shared__ float tile[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float k2 = K.inv2s2 * 1.44269504088896341f;  // exp(-a k) = 2^(-a k log2 e)
  for (long long t = blockIdx.x; t < T.ntiles; t += gridDim.x) {
    const int e0 = start[t], e1 = start[t + 1];
    if (e0 == e1) continue;  // CTA-uniform
    const TileView v = tile_view(T, t);
    const int cells = v.side * v.pitch + 32;  // a warp's tile plus one dummy slot per lane
    for (int i = threadIdx.x; i < cells * nwt; i += blockDim.x) tile[i] = 0.f;
    __syncthreads();
    if (RT > 0) {
      if (warp < nwt) {
        const WarpTaps<(RT > 0 ? RT : 1)> tp(lane);
        float* mine = tile + warp * cells;
        float* dummy = mine + v.side * v.pitch + lane;
        // 32 events per coalesced load, broadcast to the warp one at a time
        for (int base = e0 + 32 * warp; base < e1; base += 32 * nwt) {
          const float4 q = base + lane < e1 ? __ldg(EV + base + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
          const int cnt = min(32, e1 - base);
          for (int j = 0; j < cnt; ++j) {
            const float x = __shfl_sync(0xffffffffu, q.x, j), y = __shfl_sync(0xffffffffu, q.y, j);
            const float w = __shfl_sync(0xffffffffu, q.z, j);
            splat_event_warp<(RT > 0 ? RT : 1)>(mine, dummy, tp, v, T, k2, K.norm, x, y, w, lane);
          }
        }
      }
    } else {
      for (int e = e0 + threadIdx.x; e < e1; e += blockDim.x) splat_event<0>(tile, v, T, K, __ldg(EV + e));
    }
    __syncthreads();
    // flush the in-image part: the warp tiles summed, groups of 4 columns aligned in the image row
    float* base = img + (long long)v.b * T.H * T.W;
    const int y0 = max(v.oy, 0), y1 = min(v.oy + v.side, (int)T.H);
    const int x0 = max(v.ox, 0) & ~3, x1 = min(v.ox + v.side, (int)T.W);
    const int ng = (x1 - x0 + 3) >> 2, nrow = y1 - y0;
    for (int i = threadIdx.x; i < nrow * ng; i += blockDim.x) {
      const int r = i / ng, gx = x0 + 4 * (i - r * ng), gy = y0 + r;
      const int off = (gy - v.oy) * v.pitch + (gx - v.ox);
      float a[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int lx = gx + k - v.ox;
        float sum = 0.f;
        if (lx >= 0 && lx < v.side && gx + k < T.W)
          for (int q = 0; q < nwt; ++q) sum += tile[q * cells + off + k];
        a[k] = sum;
      }
      if (a[0] == 0.f && a[1] == 0.f && a[2] == 0.f && a[3] == 0.f) continue;
      float* dst = base + (long long)gy * T.W + gx;
      if (vec4 && gx + 3 < T.W) {
        red_add_f4(dst, a[0], a[1], a[2], a[3]);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (a[k] != 0.f && gx + k < T.W) red_add_f1(dst + k, a[k]);
      }
    }
    __syncthreads();  // the tile buffers are reused by the next tile of this CTA
  }
}

// Backward of one event against the staged gradient tile: gw = sum gk, gpos = w * sum gk (dx, dy) / s^2 with
// gk = norm * exp(-dx^2 k) exp(-dy^2 k) * gimg (atl_cpu.cpp:115-127).
template <int RT>
__device__ __forceinline__ void splat_event_bwd(const float* __restrict__ tile, const TileView& v, const GTiles& T,
                                                const GaussConsts& K, float4 q, float* __restrict__ GW,
                                                float2* __restrict__ GP) {
  const int R = RT > 0 ? RT : T.R;
  constexpr int WMAX = RT > 0 ? 2 * RT + 1 : 1;
  const float x = q.x, y = q.y, w = q.z;
  const int n = __float_as_int(q.w);
  const int cx = lround_small(x), cy = lround_small(y);  // bucketed events: |x|, |y| < 2^31
  const int lx0 = cx - R - v.ox, ly0 = cy - R - v.oy;
  const bool inside = cx >= 0 && cx < T.W && cy >= 0 && cy < T.H;
  float sw = 0.f, sx = 0.f, sy = 0.f;
  if (RT > 0) {
    const float k2 = K.inv2s2 * 1.44269504088896341f;  // exp(-a k) = 2^(-a k log2 e)
    float ex[WMAX], fxs[WMAX];
#pragma unroll
    for (int d = 0; d < WMAX; ++d) {
      fxs[d] = sub_rn((float)(cx - R + d), x);
      ex[d] = ex2_approx(-(fxs[d] * fxs[d]) * k2);
    }
#pragma unroll
    for (int dy = 0; dy < WMAX; ++dy) {
      const int ly = ly0 + dy;
      if (!inside && (ly < 0 || ly >= v.side)) continue;
      const float fy = sub_rn((float)(cy - R + dy), y);
      const float ey = ex2_approx(-(fy * fy) * k2);
      const float* row = tile + ly * v.pitch + lx0;
      float rg = 0.f, rgx = 0.f;
#pragma unroll
      for (int dx = 0; dx < WMAX; ++dx) {
        if (!inside && (lx0 + dx < 0 || lx0 + dx >= v.side)) continue;
        const float g = ex[dx] * row[dx];
        rg += g;
        rgx = fmaf(g, fxs[dx], rgx);
      }
      sw = fmaf(ey, rg, sw);
      sx = fmaf(ey, rgx, sx);
      sy = fmaf(ey * fy, rg, sy);
    }
  } else {
    const int wdt = 2 * R + 1;
    for (int dy = 0; dy < wdt; ++dy) {
      const int ly = ly0 + dy;
      if (ly < 0 || ly >= v.side) continue;
      const float fy = sub_rn((float)(cy - R + dy), y);
      const float ey = expf(-mul_rn(mul_rn(fy, fy), K.inv2s2));
      float rg = 0.f, rgx = 0.f;
      for (int dx = 0; dx < wdt; ++dx) {
        const int lx = lx0 + dx;
        if (lx < 0 || lx >= v.side) continue;
        const float fx = sub_rn((float)(cx - R + dx), x);
        const float g = expf(-mul_rn(mul_rn(fx, fx), K.inv2s2)) * tile[ly * v.pitch + lx];
        rg += g;
        rgx = fmaf(g, fx, rgx);
      }
      sw = fmaf(ey, rg, sw);
      sx = fmaf(ey, rgx, sx);
      sy = fmaf(ey * fy, rg, sy);
    }
  }
  sw = mul_rn(K.norm, sw);
  if (GW) GW[n] = sw;
  GP[n] = make_float2(mul_rn(w, div_rn(mul_rn(K.norm, sx), K.s2)), mul_rn(w, div_rn(mul_rn(K.norm, sy), K.s2)));
}

template <int RT>
__global__ void __launch_bounds__(kGThreads) k_gsplat_bwd_tiles(GTiles T, GaussConsts K, const float4* __restrict__ EV,
                                                                const int* __restrict__ start,
                                                                const float* __restrict__ G, float* __restrict__ GW,
                                                                float2* __restrict__ GP) {
  extern __shared__ float tile[];
  for (long long t = blockIdx.x; t < T.ntiles; t += gridDim.x) {
    const int e0 = start[t], e1 = start[t + 1];
    if (e0 == e1) continue;  // CTA-uniform
    const TileView v = tile_view(T, t);
    const float* gb = G + (long long)v.b * T.H * T.W;
    for (int i = threadIdx.x; i < v.side * v.side; i += blockDim.x) {
      const int ly = i / v.side, lx = i - ly * v.side;
      const int gy = v.oy + ly, gx = v.ox + lx;
      tile[ly * v.pitch + lx] = (gy >= 0 && gy < T.H && gx >= 0 && gx < T.W) ? __ldg(gb + (long long)gy * T.W + gx) : 0.f;
    }
    __syncthreads();
    for (int e = e0 + threadIdx.x; e < e1; e += blockDim.x) splat_event_bwd<RT>(tile, v, T, K, __ldg(EV + e), GW, GP);
    __syncthreads();
  }
}

// Events that add nothing still get the reference's outputs: gw = 0, gpos = w * 0.
__global__ void __launch_bounds__(kGThreads) k_gsplat_bwd_init(const float* __restrict__ Wt, long long N,
                                                               float* __restrict__ GW, float2* __restrict__ GP) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    const float z = mul_rn(Wt[n], 0.f);
    if (GW) GW[n] = 0.f;
    GP[n] = make_float2(z, z);
  }
}

GTiles make_tiles(long long B, long long H, long long W, long long R) {
  GTiles T;
  T.B = B;
  T.H = H;
  T.W = W;
  T.R = (int)R;
  T.tw = (int)((W + kTS - 1) / kTS);
  T.th = (int)((H + kTS - 1) / kTS);
  T.ntiles = B * T.th * (long long)T.tw;
  return T;
}

struct GaussWs {
  int* counts;
  int* start;
  long long* partials;
  float4* EV;
};
GaussWs carve_gauss(void* ws, long long N, long long ntiles) {
  char* p = (char*)align_ptr(ws);
  GaussWs w;
  w.counts = (int*)p; p += align_up((size_t)ntiles * 4);
  w.start = (int*)p; p += align_up((size_t)(ntiles + 1) * 4);
  w.partials = (long long*)p; p += align_up(scan_partials_bytes(ntiles));
  w.EV = (float4*)p;
  return w;
}

inline int ggrid(long long n) { return clamp_grid(blocks_for(n, kGThreads)); }

size_t tile_smem(int R) { return (size_t)(kTS + 2 * R) * (kTS + 2 * R + 1) * sizeof(float); }

template <typename F>
void dispatch_radius(int R, F&& f) {
  switch (R) {
#define ATLB_R(r) \
  case r: f(std::integral_constant<int, r>{}); break;
    ATLB_R(1) ATLB_R(2) ATLB_R(3) ATLB_R(4) ATLB_R(5) ATLB_R(6)
    ATLB_R(7) ATLB_R(8) ATLB_R(9) ATLB_R(10) ATLB_R(11) ATLB_R(12)
#undef ATLB_R
    default: f(std::integral_constant<int, 0>{}); break;
  }
}

// Dynamic shared memory above 48 KB (radii beyond 12) needs the per-kernel opt-in.
template <typename K>
void allow_smem(K kernel, size_t bytes) {
  if (bytes > 48 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

void bucket(const GTiles& T, const GaussWs& w, const float* pos, const float* wt, const long long* b, long long N,
            float norm, bool skip_zero, cudaStream_t s) {
  cudaMemsetAsync(w.counts, 0, (size_t)T.ntiles * 4, s);
  // large chunks (4 CTAs per SM): each CTA then touches a tile a few thousand times, not a few times
  const int grid = (int)std::max<long long>(1, std::min<long long>(blocks_for(N, kGThreads), 148LL * 4));
  const long long chunk = (N + grid - 1) / grid;
  const size_t hsm = T.ntiles <= kSmemTiles ? (size_t)T.ntiles * 4 : 0;
  if (N > 0)
    launch(k_gtile_count, grid, kGThreads, hsm, s, T, (const float2*)pos, wt, b, N, norm, skip_zero, chunk, w.counts);
  exclusive_scan<int>(w.counts, T.ntiles, w.partials, w.start, s);
  if (N > 0)
    launch(k_gtile_scatter, grid, kGThreads, hsm, s, T, (const float2*)pos, wt, b, N, norm, skip_zero, chunk,
           (const int*)w.start, w.counts, w.EV);
}

}  // namespace

size_t splat_gauss_workspace_bytes(long long N, long long B, long long H, long long W) {
  const long long ntiles = B * ((H + kTS - 1) / kTS) * ((W + kTS - 1) / kTS);
  return align_up((size_t)ntiles * 4) + align_up((size_t)(ntiles + 1) * 4) + align_up(scan_partials_bytes(ntiles)) +
         align_up((size_t)N * 16) + 256;
}

int splat_gauss_fwd(const float* pos, const float* w, const long long* b, long long N, long long B, long long H,
                    long long W, double sigma, long long R, float* img, void* ws, cudaStream_t s) {
  cudaMemsetAsync(img, 0, (size_t)(B * H * W) * sizeof(float), s);
  const GTiles T = make_tiles(B, H, W, R);
  const GaussConsts K = gauss_consts(sigma);
  const GaussWs gw = carve_gauss(ws, N, T.ntiles);
  bucket(T, gw, pos, w, b, N, K.norm, true, s);
  if (N > 0 && T.ntiles > 0) {
    const size_t one = tile_smem((int)R);
    const bool vec4 = (W % 4 == 0) && ((uintptr_t)img % 16 == 0);
    const int grid = (int)(T.ntiles < 148LL * 16 ? T.ntiles : 148LL * 16);
    cudaEvent_t e0 = timing_begin(s);
    dispatch_radius((int)R, [&](auto rc) {
      constexpr int RT = decltype(rc)::value;
      // compiled radii: one private tile per warp (up to 8, within 200 KB); generic radius: one shared tile
      const size_t per = one + 32 * sizeof(float);  // tile + dummy slots
      const int nwt = RT > 0 ? (int)std::max<size_t>(1, std::min<size_t>(kGThreads / 32, (200u << 10) / per)) : 1;
      const size_t smem = per * nwt;
      allow_smem(k_gsplat_fwd_tiles<RT>, smem);
      launch(k_gsplat_fwd_tiles<RT>, grid, kGThreads, smem, s, T, K, (const float4*)gw.EV, (const int*)gw.start, img,
             vec4, nwt);
    });
    timing_end("k_gsplat_fwd", s, e0);
  }
  return launch_status("splat_gauss_fwd");
}

int splat_gauss_bwd(const float* g, const float* pos, const float* w, const long long* b, long long N, long long B,
                    long long H, long long W, double sigma, long long R, float* gpos, float* gw_out, void* ws,
                    cudaStream_t s) {
  const GTiles T = make_tiles(B, H, W, R);
  const GaussConsts K = gauss_consts(sigma);
  const GaussWs gw = carve_gauss(ws, N, T.ntiles);
  if (N > 0) launch(k_gsplat_bwd_init, ggrid(N), kGThreads, 0, s, w, N, gw_out, (float2*)gpos);
  bucket(T, gw, pos, w, b, N, K.norm, false, s);
  if (N > 0 && T.ntiles > 0) {
    const size_t smem = tile_smem((int)R);
    const int grid = (int)(T.ntiles < 148LL * 16 ? T.ntiles : 148LL * 16);
    cudaEvent_t e0 = timing_begin(s);
    dispatch_radius((int)R, [&](auto rc) {
      constexpr int RT = decltype(rc)::value;
      allow_smem(k_gsplat_bwd_tiles<RT>, smem);
      launch(k_gsplat_bwd_tiles<RT>, grid, kGThreads, smem, s, T, K, (const float4*)gw.EV, (const int*)gw.start, g,
             gw_out, (float2*)gpos);
    });
    timing_end("k_gsplat_bwd", s, e0);
  }
  return launch_status("splat_gauss_bwd");
}

// Backward w.r.t. the positions only, over the buckets that the preceding splat_gauss_fwd of the same
// (pos, w, b) left in ws: the forward's bucketing is reused, not redone.  Events the forward skipped (zero
// weight) get gpos = w * 0.
int splat_gauss_bwd_pos(const float* g, const float* w, long long N, long long B, long long H, long long W,
                        double sigma, long long R, float* gpos, void* ws, cudaStream_t s) {
  const GTiles T = make_tiles(B, H, W, R);
  const GaussConsts K = gauss_consts(sigma);
  const GaussWs gw = carve_gauss(ws, N, T.ntiles);
  if (N > 0) launch(k_gsplat_bwd_init, ggrid(N), kGThreads, 0, s, w, N, (float*)nullptr, (float2*)gpos);
  if (N > 0 && T.ntiles > 0) {
    const size_t smem = tile_smem((int)R);
    const int grid = (int)(T.ntiles < 148LL * 16 ? T.ntiles : 148LL * 16);
    cudaEvent_t e0 = timing_begin(s);
    dispatch_radius((int)R, [&](auto rc) {
      constexpr int RT = decltype(rc)::value;
      allow_smem(k_gsplat_bwd_tiles<RT>, smem);
      launch(k_gsplat_bwd_tiles<RT>, grid, kGThreads, smem, s, T, K, (const float4*)gw.EV, (const int*)gw.start, g,
             (float*)nullptr, (float2*)gpos);
    });
    timing_end("k_gsplat_bwd", s, e0);
  }
  return launch_status("splat_gauss_bwd_pos");
}

}  // namespace atlb
