// Bilinear splat, bilinear gather and the trilinear voxel grid over shared-memory image tiles, and a
// separable Gaussian blur: the B200 replacements of splat_bilinear_fwd/bwd (csrc/atl_cpu.cpp:37-76),
// gather_bilinear_fwd/bwd (csrc/atl_cpu.cpp:134-172), voxel_grid (csrc/atl_cpu.cpp:256-286) and blur
// (atl/ops/functional.py:99-110).
//
// Reference semantics of the bilinear corner set (csrc/atl_cpu.cpp:17-33): for a point (x, y), x0 = floor(x),
// ax = x - x0, wx = (1 - ax, ax) and likewise in y; the corners (y0 + j, x0 + i), j then i, that lie in the
// image carry the weight c = wx[i] wy[j] and the derivatives dc/dx = (-1, 1)[i] wy[j], dc/dy = wx[i] (-1, 1)[j].
//
// Design:
//   1. the points are bucketed by the 32 x 32-pixel tile of their (clamped) floor corner: a two-level counting
//      sort into (x, y, value, index) records, tile-major (every corner of a point then lies in its tile plus a
//      one-pixel halo on the right and at the bottom);
//   2. one CTA per tile.  Reads of an image (gather, and both backward passes) stage the tile and its halo,
//      33 x 33 pixels, in shared memory with one TMA copy (cp.async.bulk.tensor over a (W, H, B) tensor map,
//      zero fill outside the image; plain loads where the image cannot be described by a tensor map); then every
//      lane evaluates its point's corners from shared memory, in the reference's corner order and rounding,
//      so per-point results are bit-identical to the reference's.  Writes to an image (splat, gather's image
//      gradient, voxel grid) accumulate in a shared tile with shared atomics and leave with one vectorised
//      red.global.add.v4.f32 per 4 pixels (neighbouring tiles overlap by the halo).
//   3. The blur is two passes over (plane, 32 x 32 tile) blocks with the tile and its radius-r halo in shared
//      memory; its adjoint (the backward) is the same blur, the kernel being symmetric with zero padding.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "plan_math.cuh"
#include "scan.cuh"

namespace atlb {
namespace {

constexpr int kT = 32;          // tile side (pixels)
constexpr int kTLog = 5;
constexpr int kTS = kT + 1;     // staged side: the tile and a one-pixel halo
constexpr int kTP = 36;         // staged row pitch (floats): the TMA box width, 144 bytes (a multiple of 16)
constexpr int kThreads = 256;
constexpr int kSmemTiles = 12288;  // per-CTA shared tile histogram of the bucketing (48 KB)
constexpr long long kChunk = 1 << 14;  // points per bucketing CTA
constexpr int kVoxMaxC = 16;    // voxel channels accumulated in shared memory (more: global reds)

struct BTiles {
  long long B, H, W;
  int tw, th;
  long long ntiles;
};

BTiles make_tiles(long long B, long long H, long long W) {
  BTiles T;
  T.B = B; T.H = H; T.W = W;
  T.tw = (int)((W + kT - 1) / kT);
  T.th = (int)((H + kT - 1) / kT);
  T.ntiles = B * T.tw * T.th;
  return T;
}

// Tile of a point whose floor corner is (floor x, floor y), or -1 when none of its corners lies in the image
// (batch index outside [0, B), non-finite position, corner row / column outside [-1, H-1] / [-1, W-1]).
__device__ __forceinline__ long long bil_tile(const BTiles& T, float x, float y, long long b) {
  if (b < 0 || b >= T.B) return -1;
  if (!(fabsf(x) < 1e18f && fabsf(y) < 1e18f)) return -1;
  const long long x0 = (long long)floorf(x), y0 = (long long)floorf(y);
  if (x0 < -1 || x0 > T.W - 1 || y0 < -1 || y0 > T.H - 1) return -1;
  const long long tx = min(max(x0, 0LL), T.W - 1) >> kTLog, ty = min(max(y0, 0LL), T.H - 1) >> kTLog;
  return (b * T.th + ty) * T.tw + tx;
}

// ---- bucketing: per-CTA shared histograms, one global atomic per (CTA, tile) --------------------------------
// The value stored with a point: its weight (w), the upstream gradient (g) or its time and polarity (voxel).
__global__ void __launch_bounds__(kThreads) k_btile_count(BTiles T, const float2* __restrict__ P,
                                                          const long long* __restrict__ Bi, long long N,
                                                          long long chunk, const float* __restrict__ skip_zero,
                                                          int* __restrict__ counts) {
  extern __shared__ int hist[];
  const bool sm = T.ntiles <= kSmemTiles;
  if (sm)
    for (int i = threadIdx.x; i < T.ntiles; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const long long n0 = blockIdx.x * chunk, n1 = min(n0 + chunk, N);
  for (long long n = n0 + threadIdx.x; n < n1; n += blockDim.x) {
    if (skip_zero && skip_zero[n] == 0.f) continue;
    const float2 p = P[n];
    const long long key = bil_tile(T, p.x, p.y, Bi[n]);
    if (key >= 0) atomicAdd(sm ? hist + key : counts + key, 1);
  }
  __syncthreads();
  if (sm)
    for (int i = threadIdx.x; i < T.ntiles; i += blockDim.x)
      if (hist[i]) atomicAdd(counts + i, hist[i]);
}

// REC[slot] = (x, y, v0, v1): v0 = val0[n] (or 0), v1 = val1[n] (voxel) or the index bits.
__global__ void __launch_bounds__(kThreads) k_btile_scatter(BTiles T, const float2* __restrict__ P,
                                                            const long long* __restrict__ Bi, long long N,
                                                            long long chunk, const float* __restrict__ skip_zero,
                                                            const float* __restrict__ val0,
                                                            const float* __restrict__ val1,
                                                            const int* __restrict__ start, int* __restrict__ cursor,
                                                            float4* __restrict__ REC) {
  extern __shared__ int hist[];
  const bool sm = T.ntiles <= kSmemTiles;
  const long long n0 = blockIdx.x * chunk, n1 = min(n0 + chunk, N);
  if (sm) {
    for (int i = threadIdx.x; i < T.ntiles; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (long long n = n0 + threadIdx.x; n < n1; n += blockDim.x) {
      if (skip_zero && skip_zero[n] == 0.f) continue;
      const float2 p = P[n];
      const long long key = bil_tile(T, p.x, p.y, Bi[n]);
      if (key >= 0) atomicAdd(hist + key, 1);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < T.ntiles; i += blockDim.x) {
      const int c = hist[i];
      hist[i] = c ? start[i] + atomicAdd(cursor + i, c) : 0;
    }
    __syncthreads();
  }
  for (long long n = n0 + threadIdx.x; n < n1; n += blockDim.x) {
    if (skip_zero && skip_zero[n] == 0.f) continue;
    const float2 p = P[n];
    const long long key = bil_tile(T, p.x, p.y, Bi[n]);
    if (key < 0) continue;
    const int slot = sm ? atomicAdd(hist + key, 1) : start[key] + atomicAdd(cursor + key, 1);
    REC[slot] = make_float4(p.x, p.y, val0 ? val0[n] : 0.f, val1 ? val1[n] : __int_as_float((int)n));
  }
}

// ---- tiles ---------------------------------------------------------------------------------------------
struct TileOrigin {
  int b, x0, y0;  // image, first pixel column / row of the tile
};
__device__ __forceinline__ TileOrigin tile_origin(const BTiles& T, long long t) {
  const long long per = (long long)T.th * T.tw;
  TileOrigin o;
  o.b = (int)(t / per);
  const int r = (int)(t - (long long)o.b * per);
  const int ty = r / T.tw, tx = r - ty * T.tw;
  o.x0 = tx << kTLog;
  o.y0 = ty << kTLog;
  return o;
}

// Staging of a tile (kTS x kTS pixels from (x0, y0) of image b, zero outside the image) into tile[kTS][kTP].
__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

// mbarrier wait with an iteration limit: on timeout *err is set and false returned (never expected: the copy
// is a few KB).
__device__ __forceinline__ bool mbar_wait(unsigned bar, unsigned phase, int* err) {
  for (int it = 0; it < (1 << 22); ++it) {
    unsigned done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(phase)
        : "memory");
    if (done) return true;
  }
  if (err) atomicOr(err, 1);
  return false;
}

// TMA: the whole CTA calls it; returns false if the copy did not complete (the caller skips the tile).
__device__ __forceinline__ bool stage_tile_tma(float (*tile)[kTP], const CUtensorMap* map, const TileOrigin& o,
                                               unsigned long long* bar, int* err) {
  const unsigned b = smem_u32(bar);
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(b) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(kTS * kTP * 4) : "memory");
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(&tile[0][0])),
        "l"(map), "r"(o.x0), "r"(o.y0), "r"(o.b), "r"(b)
        : "memory");
  }
  return mbar_wait(b, 0, err);
}

__device__ __forceinline__ void stage_tile_plain(float (*tile)[kTP], const float* __restrict__ img, const BTiles& T,
                                                 const TileOrigin& o) {
  const float* im = img + (long long)o.b * T.H * T.W;
  for (int i = threadIdx.x; i < kTS * kTP; i += blockDim.x) {
    const int r = i / kTP, c = i - r * kTP;
    const long long y = o.y0 + r, x = o.x0 + c;
    tile[r][c] = (c < kTS && y < T.H && x < T.W) ? __ldg(im + y * T.W + x) : 0.f;
  }
  __syncthreads();
}

// The reference's corner loop (csrc/atl_cpu.cpp:17-33) over a staged tile: f(tile row, tile column, c, dc/dx,
// dc/dy) for the corners in the image, in the reference's order.
template <class F>
__device__ __forceinline__ void tile_corners(float x, float y, const BTiles& T, const TileOrigin& o, F&& f) {
  const float fx0 = floorf(x), fy0 = floorf(y);
  const int x0 = (int)fx0, y0 = (int)fy0;  // |x|, |y| < W + 1, H + 1: bucketed points
  const float ax = x - fx0, ay = y - fy0;
  const float wx[2] = {1.f - ax, ax}, wy[2] = {1.f - ay, ay};
  const float dwx[2] = {-1.f, 1.f}, dwy[2] = {-1.f, 1.f};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int yy = y0 + j;
    if (yy < 0 || yy >= T.H) continue;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int xx = x0 + i;
      if (xx < 0 || xx >= T.W) continue;
      f(yy - o.y0, xx - o.x0, __fmul_rn(wx[i], wy[j]), __fmul_rn(dwx[i], wy[j]), __fmul_rn(wx[i], dwy[j]));
    }
  }
}

// Shared accumulation tile -> image (red.global; v4 where four pixels of a row are 16-byte aligned in the image).
__device__ __forceinline__ void flush_tile(const float (*acc)[kTP], float* __restrict__ img, const BTiles& T,
                                           const TileOrigin& o) {
  float* im = img + (long long)o.b * T.H * T.W;
  const bool vec = (T.W % 4 == 0) && ((reinterpret_cast<uintptr_t>(img) & 15) == 0);
  for (int i = threadIdx.x; i < kTS * 9; i += blockDim.x) {  // 9 groups of <= 4 columns per row (33 columns)
    const int r = i / 9, q = i - r * 9;
    const long long y = o.y0 + r;
    if (y >= T.H) continue;
    const int c0 = q * 4;
    const long long x = o.x0 + c0;
    if (vec && c0 + 4 <= kT && x + 4 <= T.W) {
      const float a = acc[r][c0], b = acc[r][c0 + 1], c = acc[r][c0 + 2], d = acc[r][c0 + 3];
      if (a != 0.f || b != 0.f || c != 0.f || d != 0.f) red_add_f4(im + y * T.W + x, a, b, c, d);
    } else {
      for (int k = 0; k < 4 && c0 + k < kTS && x + k < T.W; ++k) {
        const float v = acc[r][c0 + k];
        if (v != 0.f) red_add_f1(im + y * T.W + x + k, v);
      }
    }
  }
}

__device__ __forceinline__ void zero_tile(float (*acc)[kTP]) {
  for (int i = threadIdx.x; i < kTS * kTP; i += blockDim.x) (&acc[0][0])[i] = 0.f;
}

struct __align__(128) StageSmem {
  float tile[kTS][kTP];
  unsigned long long bar;
};

// ---- bilinear splat ------------------------------------------------------------------------------------
// Forward: img[b] += w c over the corners (csrc/atl_cpu.cpp:37-53), REC = (x, y, w, n).
__global__ void __launch_bounds__(kThreads) k_bsplat_fwd(BTiles T, const float4* __restrict__ REC,
                                                         const int* __restrict__ start, float* __restrict__ img) {
  __shared__ float acc[kTS][kTP];
  const long long t = blockIdx.x;
  const int s0 = start[t], s1 = start[t + 1];
  if (s0 == s1) return;  // CTA-uniform
  const TileOrigin o = tile_origin(T, t);
  zero_tile(acc);
  __syncthreads();
  for (int s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
    const float4 q = REC[s];
    tile_corners(q.x, q.y, T, o, [&](int r, int c, float cw, float, float) { atomicAdd(&acc[r][c], q.z * cw); });
  }
  __syncthreads();
  flush_tile(acc, img, T, o);
}

// Backward: gw = sum g c, gpos = w (sum g dc/dx, sum g dc/dy) (csrc/atl_cpu.cpp:56-76), g staged.
template <bool TMA>
__global__ void __launch_bounds__(kThreads) k_bsplat_bwd(BTiles T, const __grid_constant__ CUtensorMap map,
                                                         const float* __restrict__ gimg, const float4* __restrict__ REC,
                                                         const int* __restrict__ start, float2* __restrict__ gpos,
                                                         float* __restrict__ gw, int* err) {
  __shared__ StageSmem S;
  const long long t = blockIdx.x;
  const int s0 = start[t], s1 = start[t + 1];
  if (s0 == s1) return;
  const TileOrigin o = tile_origin(T, t);
  if (TMA) {
    if (!stage_tile_tma(S.tile, &map, o, &S.bar, err)) return;
  } else {
    stage_tile_plain(S.tile, gimg, T, o);
  }
  for (int s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
    const float4 q = REC[s];
    float sx = 0.f, sy = 0.f, sw = 0.f;
    tile_corners(q.x, q.y, T, o, [&](int r, int c, float cw, float dcx, float dcy) {
      const float g = S.tile[r][c];
      sw = __fadd_rn(sw, __fmul_rn(g, cw));
      sx = __fadd_rn(sx, __fmul_rn(g, dcx));
      sy = __fadd_rn(sy, __fmul_rn(g, dcy));
    });
    const int n = __float_as_int(q.w);
    gw[n] = sw;
    gpos[n] = make_float2(__fmul_rn(q.z, sx), __fmul_rn(q.z, sy));
  }
}

// ---- bilinear gather -----------------------------------------------------------------------------------
// Forward: out = sum c img (csrc/atl_cpu.cpp:134-150), REC = (x, y, 0, n).
template <bool TMA>
__global__ void __launch_bounds__(kThreads) k_gather_fwd(BTiles T, const __grid_constant__ CUtensorMap map,
                                                         const float* __restrict__ img, const float4* __restrict__ REC,
                                                         const int* __restrict__ start, float* __restrict__ out,
                                                         int* err) {
  __shared__ StageSmem S;
  const long long t = blockIdx.x;
  const int s0 = start[t], s1 = start[t + 1];
  if (s0 == s1) return;
  const TileOrigin o = tile_origin(T, t);
  if (TMA) {
    if (!stage_tile_tma(S.tile, &map, o, &S.bar, err)) return;
  } else {
    stage_tile_plain(S.tile, img, T, o);
  }
  for (int s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
    const float4 q = REC[s];
    float acc = 0.f;
    tile_corners(q.x, q.y, T, o, [&](int r, int c, float cw, float, float) {
      acc = __fadd_rn(acc, __fmul_rn(cw, S.tile[r][c]));
    });
    out[__float_as_int(q.w)] = acc;
  }
}

// Backward: gimg += g c (shared tile, then red.global), gpos = g (sum dc/dx img, sum dc/dy img)
// (csrc/atl_cpu.cpp:152-172), REC = (x, y, g, n).
template <bool TMA>
__global__ void __launch_bounds__(kThreads) k_gather_bwd(BTiles T, const __grid_constant__ CUtensorMap map,
                                                         const float* __restrict__ img, const float4* __restrict__ REC,
                                                         const int* __restrict__ start, float* __restrict__ gimg,
                                                         float2* __restrict__ gpos, int* err) {
  __shared__ StageSmem S;
  __shared__ float acc[kTS][kTP];
  const long long t = blockIdx.x;
  const int s0 = start[t], s1 = start[t + 1];
  if (s0 == s1) return;
  const TileOrigin o = tile_origin(T, t);
  zero_tile(acc);
  if (TMA) {
    if (!stage_tile_tma(S.tile, &map, o, &S.bar, err)) return;
  } else {
    stage_tile_plain(S.tile, img, T, o);
  }
  __syncthreads();  // acc zeroed (the TMA path's wait does not order it)
  for (int s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
    const float4 q = REC[s];
    const float g = q.z;
    float sx = 0.f, sy = 0.f;
    tile_corners(q.x, q.y, T, o, [&](int r, int c, float cw, float dcx, float dcy) {
      const float v = S.tile[r][c];
      sx = __fadd_rn(sx, __fmul_rn(dcx, v));
      sy = __fadd_rn(sy, __fmul_rn(dcy, v));
      atomicAdd(&acc[r][c], __fmul_rn(g, cw));
    });
    gpos[__float_as_int(q.w)] = make_float2(__fmul_rn(g, sx), __fmul_rn(g, sy));
  }
  __syncthreads();
  flush_tile(acc, gimg, T, o);
}

// ---- voxel grid ----------------------------------------------------------------------------------------
// vox[b, tt, yy, xx] += p wt wy wx over the 8 corners of (t (C - 1), y, x) (csrc/atl_cpu.cpp:256-286),
// REC = (x, y, t, p).  Channels up to kVoxMaxC accumulate in shared memory, others with global reds.
__global__ void __launch_bounds__(kThreads) k_voxel(BTiles T, int C, const float4* __restrict__ REC,
                                                    const int* __restrict__ start, float* __restrict__ vox) {
  extern __shared__ float vacc[];  // [C][kTS][kTP] when C <= kVoxMaxC
  const long long t = blockIdx.x;
  const int s0 = start[t], s1 = start[t + 1];
  if (s0 == s1) return;
  const TileOrigin o = tile_origin(T, t);
  const bool sm = C <= kVoxMaxC;
  if (sm)
    for (int i = threadIdx.x; i < C * kTS * kTP; i += blockDim.x) vacc[i] = 0.f;
  __syncthreads();
  const long long plane = T.H * T.W;
  float* vb = vox + (long long)o.b * C * plane;
  for (int s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
    const float4 q = REC[s];
    const float x = q.x, y = q.y, tn = __fmul_rn(q.z, (float)(C - 1)), pol = q.w;
    const int x0 = (int)floorf(x), y0 = (int)floorf(y);
    const float ft0 = floorf(tn);
    if (!(fabsf(tn) < 1e9f)) continue;  // no time bin
    const int t0 = (int)ft0;
#pragma unroll
    for (int dt = 0; dt < 2; ++dt) {
      const int tt = t0 + dt;
      if (tt < 0 || tt >= C) continue;
      const float wt = __fsub_rn(1.f, fabsf(__fsub_rn((float)tt, tn)));
#pragma unroll
      for (int dy = 0; dy < 2; ++dy) {
        const int yy = y0 + dy;
        if (yy < 0 || yy >= T.H) continue;
        const float wy = __fsub_rn(1.f, fabsf(__fsub_rn((float)yy, y)));
#pragma unroll
        for (int dx = 0; dx < 2; ++dx) {
          const int xx = x0 + dx;
          if (xx < 0 || xx >= T.W) continue;
          const float wx = __fsub_rn(1.f, fabsf(__fsub_rn((float)xx, x)));
          const float v = __fmul_rn(__fmul_rn(__fmul_rn(pol, wt), wy), wx);
          if (sm)
            atomicAdd(vacc + (tt * kTS + (yy - o.y0)) * kTP + (xx - o.x0), v);
          else
            red_add_f1(vb + tt * plane + (long long)yy * T.W + xx, v);
        }
      }
    }
  }
  if (!sm) return;
  __syncthreads();
  for (int c = 0; c < C; ++c) {
    BTiles Tc = T;
    const TileOrigin oc{0, o.x0, o.y0};
    flush_tile(reinterpret_cast<const float(*)[kTP]>(vacc + c * kTS * kTP), vb + c * plane, Tc, oc);
  }
}

// ---- separable blur ------------------------------------------------------------------------------------
// out = K_y * (K_x * img) with zero padding (atl/ops/functional.py:99-110): one CTA per (plane, 32 x 32 tile);
// pass 1 convolves rows of the tile and an r-row halo, pass 2 the columns, both from shared memory.
constexpr int kBlurMaxR = 32;
struct BlurWeights {
  float k[2 * kBlurMaxR + 1];
};
__global__ void __launch_bounds__(kThreads) k_blur(const float* __restrict__ img, long long H, long long W, int tw,
                                                   int th, const BlurWeights kw, int r, float* __restrict__ out) {
  extern __shared__ float sb[];  // in: (32 + 2r) rows x (32 + 2r) cols; mid: (32 + 2r) rows x 32 cols
  __shared__ float k[2 * kBlurMaxR + 1];
  const int side = kT + 2 * r;
  float* in = sb;
  float* mid = sb + side * side;
  const long long blk = blockIdx.x;
  const long long plane = blk / ((long long)tw * th);
  const int rem = (int)(blk - plane * tw * th), ty = rem / tw, tx = rem - ty * tw;
  const long long x0 = (long long)tx * kT - r, y0 = (long long)ty * kT - r;
  const float* im = img + plane * H * W;
  for (int i = threadIdx.x; i < 2 * r + 1; i += blockDim.x) k[i] = kw.k[i];
  for (int i = threadIdx.x; i < side * side; i += blockDim.x) {
    const int rr = i / side, cc = i - rr * side;
    const long long y = y0 + rr, x = x0 + cc;
    in[i] = (y >= 0 && y < H && x >= 0 && x < W) ? __ldg(im + y * W + x) : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < side * kT; i += blockDim.x) {  // rows: every staged row, the tile's columns
    const int rr = i / kT, cc = i - rr * kT;
    float s = 0.f;
    for (int d = 0; d <= 2 * r; ++d) s = __fadd_rn(s, __fmul_rn(k[d], in[rr * side + cc + d]));
    mid[rr * kT + cc] = s;
  }
  __syncthreads();
  float* ob = out + plane * H * W;
  for (int i = threadIdx.x; i < kT * kT; i += blockDim.x) {  // columns: the tile's pixels
    const int rr = i / kT, cc = i - rr * kT;
    const long long y = (long long)ty * kT + rr, x = (long long)tx * kT + cc;
    if (y >= H || x >= W) continue;
    float s = 0.f;
    for (int d = 0; d <= 2 * r; ++d) s = __fadd_rn(s, __fmul_rn(k[d], mid[(rr + d) * kT + cc]));
    ob[y * W + x] = s;
  }
}

// ---- host side -----------------------------------------------------------------------------------------
struct TileWs {
  int* counts;
  int* start;
  long long* partials;
  float4* rec;
  int* err;
};

TileWs carve_tiles(void* ws, long long N, long long ntiles) {
  char* p = (char*)align_ptr(ws);
  TileWs w;
  w.counts = (int*)p; p += align_up((size_t)ntiles * 4);
  w.start = (int*)p; p += align_up((size_t)(ntiles + 1) * 4);
  w.partials = (long long*)p; p += align_up(scan_partials_bytes(ntiles));
  w.rec = (float4*)p; p += align_up((size_t)N * 16);
  w.err = (int*)p;
  return w;
}

inline size_t bucket_smem(const BTiles& T) { return T.ntiles <= kSmemTiles ? (size_t)T.ntiles * 4 : 0; }

// Buckets the N points by tile into w.rec with (val0, val1) as the record's third / fourth member.
void bucket(const BTiles& T, const float* pos, const long long* b, long long N, const float* skip_zero,
            const float* val0, const float* val1, const TileWs& w, cudaStream_t s) {
  cudaMemsetAsync(w.counts, 0, (size_t)T.ntiles * 4, s);
  // enough CTAs to fill the GPU (8 per SM), each with a contiguous chunk of at least kChunk / 16 points so its
  // shared histogram is reused: with a fixed chunk of kChunk points a 1M-point call had 61 CTAs
  long long grid_l = (N + kChunk / 16 - 1) / (kChunk / 16);
  grid_l = grid_l < 148LL * 8 ? grid_l : 148LL * 8;
  const unsigned grid = (unsigned)(grid_l > 0 ? grid_l : 1);
  const long long chunk = (N + grid - 1) / grid;
  if (N > 0)
    launch(k_btile_count, grid, kThreads, bucket_smem(T), s, T, (const float2*)pos, b, N, chunk, skip_zero,
           w.counts);
  exclusive_scan<int>(w.counts, T.ntiles, w.partials, w.start, s);
  if (N > 0)
    launch(k_btile_scatter, grid, kThreads, bucket_smem(T), s, T, (const float2*)pos, b, N, chunk, skip_zero, val0,
           val1, (const int*)w.start, w.counts, w.rec);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}

// A (W, H, B) tensor map of an image stack with a kTP x kTS x 1 box, or false when the layout does not allow
// one (row pitch not a multiple of 16 bytes, unaligned base): the kernels then stage with plain loads.
bool image_map(CUtensorMap* m, const float* img, const BTiles& T) {
  if (!img || (reinterpret_cast<uintptr_t>(img) & 15) || (T.W * 4) % 16 || T.W > (1LL << 31) ||
      T.H > (1LL << 31) || T.B > (1LL << 31))
    return false;
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)T.W, (cuuint64_t)T.H, (cuuint64_t)T.B};
  const cuuint64_t strides[2] = {(cuuint64_t)T.W * 4, (cuuint64_t)(T.H * T.W) * 4};
  const cuuint32_t box[3] = {kTP, kTS, 1}, es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(img), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Launches a staging kernel with a tensor map when one can be made, else with plain loads.
template <class KT, class KP, class... Args>
void launch_staged(KT k_tma, KP k_plain, const float* img, const BTiles& T, cudaStream_t s, Args... args) {
  CUtensorMap m;
  const bool tma = image_map(&m, img, T);
  if (!tma) memset(&m, 0, sizeof(m));
  if (tma)
    launch(k_tma, (unsigned)T.ntiles, kThreads, 0, s, T, m, args...);
  else
    launch(k_plain, (unsigned)T.ntiles, kThreads, 0, s, T, m, args...);
}

}  // namespace

size_t tile_ops_workspace_bytes(long long N, long long B, long long H, long long W) {
  const BTiles T = make_tiles(B, H, W);
  return align_up((size_t)T.ntiles * 4) + align_up((size_t)(T.ntiles + 1) * 4) + align_up(scan_partials_bytes(T.ntiles)) +
         align_up((size_t)N * 16) + align_up(16) + 256;
}

int splat_bilinear_fwd(const float* pos, const float* w, const long long* b, long long N, long long B, long long H,
                       long long W, float* img, void* ws, cudaStream_t s) {
  const BTiles T = make_tiles(B, H, W);
  cudaMemsetAsync(img, 0, (size_t)(B * H * W) * 4, s);
  if (T.ntiles == 0) return launch_status("splat_bilinear_fwd");
  const TileWs tw = carve_tiles(ws, N, T.ntiles);
  bucket(T, pos, b, N, w, w, nullptr, tw, s);  // a zero weight adds nothing (atl_cpu.cpp:46)
  launch(k_bsplat_fwd, (unsigned)T.ntiles, kThreads, 0, s, T, (const float4*)tw.rec, (const int*)tw.start, img);
  return launch_status("splat_bilinear_fwd");
}

int splat_bilinear_bwd(const float* g, const float* pos, const float* w, const long long* b, long long N, long long B,
                       long long H, long long W, float* gpos, float* gw, void* ws, cudaStream_t s) {
  const BTiles T = make_tiles(B, H, W);
  cudaMemsetAsync(gpos, 0, (size_t)N * 8, s);
  cudaMemsetAsync(gw, 0, (size_t)N * 4, s);
  if (T.ntiles == 0) return launch_status("splat_bilinear_bwd");
  const TileWs tw = carve_tiles(ws, N, T.ntiles);
  bucket(T, pos, b, N, nullptr, w, nullptr, tw, s);
  launch_staged(k_bsplat_bwd<true>, k_bsplat_bwd<false>, g, T, s, g, (const float4*)tw.rec, (const int*)tw.start,
                (float2*)gpos, gw, tw.err);
  return launch_status("splat_bilinear_bwd");
}

int gather_fwd(const float* img, const float* pos, const long long* b, long long N, long long B, long long H,
               long long W, float* out, void* ws, cudaStream_t s) {
  const BTiles T = make_tiles(B, H, W);
  cudaMemsetAsync(out, 0, (size_t)N * 4, s);
  if (T.ntiles == 0) return launch_status("gather_fwd");
  const TileWs tw = carve_tiles(ws, N, T.ntiles);
  bucket(T, pos, b, N, nullptr, nullptr, nullptr, tw, s);
  launch_staged(k_gather_fwd<true>, k_gather_fwd<false>, img, T, s, img, (const float4*)tw.rec, (const int*)tw.start,
                out, tw.err);
  return launch_status("gather_fwd");
}

int gather_bwd(const float* g, const float* img, const float* pos, const long long* b, long long N, long long B,
               long long H, long long W, float* gimg, float* gpos, void* ws, cudaStream_t s) {
  const BTiles T = make_tiles(B, H, W);
  cudaMemsetAsync(gimg, 0, (size_t)(B * H * W) * 4, s);
  cudaMemsetAsync(gpos, 0, (size_t)N * 8, s);
  if (T.ntiles == 0) return launch_status("gather_bwd");
  const TileWs tw = carve_tiles(ws, N, T.ntiles);
  bucket(T, pos, b, N, nullptr, g, nullptr, tw, s);
  launch_staged(k_gather_bwd<true>, k_gather_bwd<false>, img, T, s, img, (const float4*)tw.rec, (const int*)tw.start,
                gimg, (float2*)gpos, tw.err);
  return launch_status("gather_bwd");
}

int voxel_grid(const float* pos, const float* t, const float* p, const long long* b, long long N, long long B,
               long long C, long long H, long long W, float* vox, void* ws, cudaStream_t s) {
  const BTiles T = make_tiles(B, H, W);
  cudaMemsetAsync(vox, 0, (size_t)(B * C * H * W) * 4, s);
  if (T.ntiles == 0 || C <= 0) return launch_status("voxel_grid");
  const TileWs tw = carve_tiles(ws, N, T.ntiles);
  bucket(T, pos, b, N, nullptr, t, p, tw, s);
  const size_t smem = C <= kVoxMaxC ? (size_t)C * kTS * kTP * 4 : 0;
  static unsigned long long attr_done = 0;
  if (first_use_on_device(attr_done))
    cudaFuncSetAttribute(k_voxel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)((size_t)kVoxMaxC * kTS * kTP * 4));
  launch(k_voxel, (unsigned)T.ntiles, kThreads, smem, s, T, (int)C, (const float4*)tw.rec, (const int*)tw.start, vox);
  return launch_status("voxel_grid");
}

// Normalised 1-D Gaussian kernel of radius max(ceil(3 sigma), 1) (atl/ops/functional.py:89-96), in fp32.
int blur_weights(double sigma, std::vector<float>* k) {
  const int r = std::max((int)std::ceil(3 * sigma), 1);
  if (r > kBlurMaxR) return -1;
  k->resize(2 * r + 1);
  const float den = (float)(2 * sigma * sigma);
  float sum = 0.f;
  for (int i = -r; i <= r; ++i) {
    const float x = (float)i;
    (*k)[i + r] = std::exp(-(x * x) / den);
  }
  for (float v : *k) sum += v;
  for (float& v : *k) v /= sum;
  return r;
}

int blur(const float* img, long long P, long long H, long long W, double sigma, float* out, cudaStream_t s) {
  std::vector<float> k;
  const int r = blur_weights(sigma, &k);
  if (r < 0) {
    set_error("blur: sigma %g gives a radius above %d", sigma, kBlurMaxR);
    return ATLB_ERR_ARG;
  }
  BlurWeights kw;
  for (int i = 0; i < 2 * r + 1; ++i) kw.k[i] = k[i];
  const int tw = (int)((W + kT - 1) / kT), th = (int)((H + kT - 1) / kT);
  const int side = kT + 2 * r;
  const size_t smem = (size_t)(side * side + side * kT) * 4;
  static unsigned long long attr_done = 0;
  if (first_use_on_device(attr_done)) {
    const int mside = kT + 2 * kBlurMaxR;
    cudaFuncSetAttribute(k_blur, cudaFuncAttributeMaxDynamicSharedMemorySize, (mside * mside + mside * kT) * 4);
  }
  if (P * tw * th > 0) launch(k_blur, (unsigned)(P * tw * th), kThreads, smem, s, img, H, W, tw, th, kw, r, out);
  return launch_status("blur");
}

}  // namespace atlb
