// Pair-sum kernels shared by the drop-in path (reference plan layout) and the fused objective path
// (compact layout), templated on how entries and anchors are read.
//
// Forward: one warp per ANCHOR CELL.  The cell's anchors are processed in groups of NA (1..8, a
// compile-time size picked per group, so no lane evaluates an absent anchor); every lane streams one
// candidate source of the 3 neighbouring cell rows at a time (each row is one contiguous CSR range)
// and tests it against the NA anchors held in registers.  The per-anchor partial sums are reduced
// across the warp in double.
// Backward: one warp per SOURCE CELL, one source entry per lane; the anchors of the 3x3 neighbouring
// cells are broadcast from the bucketed anchor array.  The gradient of an entry is summed in
// registers and leaves with one vector red.global per entry.
#pragma once
#include "common.cuh"
#include "pair_math.cuh"

namespace atlb {

struct CellGrid {
  long long GW, GH, S, ncell;
};

// ---- entry accessors ---------------------------------------------------------------------------------
// Reference PairPlan layout (functional.py:114-129): SoA, int64 ids.
struct RefEntries {
  using Id = long long;
  const float2* SY;
  const float2* SV;
  const float* ST;
  const long long* SID;
  __device__ __forceinline__ void load(long long k, float2& y, float2& v, float& t, Id& id) const {
    y = __ldg(SY + k);
    v = __ldg(SV + k);
    t = __ldg(ST + k);
    id = __ldg(SID + k);
  }
  __device__ __forceinline__ float4 yv(long long k) const {
    const float2 y = __ldg(SY + k), v = __ldg(SV + k);
    return make_float4(y.x, y.y, v.x, v.y);
  }
  __device__ __forceinline__ float t(long long k) const { return __ldg(ST + k); }
  __device__ __forceinline__ int id(long long k) const { return (int)__ldg(SID + k); }
  __device__ __forceinline__ long long id64(long long k) const { return __ldg(SID + k); }
};

// Compact layout of the fused path: (y.x, y.y, v.x, v.y) + (t, id bits), 24 bytes per entry.
struct FastEntries {
  using Id = int;
  const float4* YV;
  const float2* TI;
  __device__ __forceinline__ void load(long long k, float2& y, float2& v, float& t, Id& id) const {
    const float4 a = __ldg(YV + k);
    const float2 b = __ldg(TI + k);
    y = make_float2(a.x, a.y);
    v = make_float2(a.z, a.w);
    t = b.x;
    id = __float_as_int(b.y);
  }
  __device__ __forceinline__ float4 yv(long long k) const { return __ldg(YV + k); }
  __device__ __forceinline__ float t(long long k) const { return __ldg(TI + k).x; }
  __device__ __forceinline__ int id(long long k) const { return __float_as_int(__ldg(TI + k).y); }
};

// ---- anchor accessors (bucketed by cell) -------------------------------------------------------------
struct RefAnchors {
  using Id = long long;
  const float2* xy;
  const float* t;
  const long long* id;
  const int* idx;  // original anchor index
  __device__ __forceinline__ void load(int p, float& x, float& y, float& ta, Id& aid) const {
    const float2 q = __ldg(xy + p);
    x = q.x; y = q.y;
    ta = __ldg(t + p);
    aid = __ldg(id + p);
  }
};

struct FastAnchors {
  using Id = int;
  const float4* XT;  // (x, y, t, id bits)
  const int* idx;
  __device__ __forceinline__ void load(int p, float& x, float& y, float& ta, Id& aid) const {
    const float4 q = __ldg(XT + p);
    x = q.x; y = q.y; ta = q.z;
    aid = __float_as_int(q.w);
  }
};

template <typename CS>
__device__ __forceinline__ void cell_coords(long long c, const CellGrid& G, long long* cx, long long* cy,
                                            long long* g) {
  *cx = c % G.GW;
  const long long r = c / G.GW;
  *cy = r % G.GH;
  *g = r / G.GH;
}

// ---- forward -----------------------------------------------------------------------------------------
template <int NA, class E, class A, typename CS, class Out>
__device__ __forceinline__ void fwd_group(const E& ent, const A& anc, int base, const CS* __restrict__ cstart,
                                          long long row0, long long GW, long long ylo, long long yhi, long long xlo,
                                          long long xhi, float cs, const PairConsts& C, Out& out, int lane) {
  float ax[NA], ay[NA], at[NA], adt[NA], acc[NA];
  typename A::Id aid[NA];
#pragma unroll
  for (int q = 0; q < NA; ++q) {
    anc.load(base + q, ax[q], ay[q], at[q], aid[q]);
    adt[q] = sub_rn(at[q], cs);
    acc[q] = 0.f;
  }
  for (long long yy = ylo; yy <= yhi; ++yy) {
    const long long row = row0 + yy * GW;
    const long long k0 = cstart[row + xlo], k1 = cstart[row + xhi + 1];
    for (long long k = k0 + lane; k < k1; k += 32) {
      float2 sy, sv;
      float st;
      typename E::Id sid;
      ent.load(k, sy, sv, st, sid);
#pragma unroll
      for (int q = 0; q < NA; ++q) {
        float rx, ry, d2, dt;
        if ((long long)sid != (long long)aid[q] &&
            pair_test(C, ax[q], ay[q], at[q], adt[q], sy, sv, st, &rx, &ry, &d2, &dt))
          acc[q] += pair_kernel(C, d2);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < NA; ++q) {
    const double s = warp_sum((double)acc[q]);
    if (lane == 0) out(base + q, s);
  }
}

template <class E, class A, typename CS, class Out>
__global__ void __launch_bounds__(256) k_pair_fwd_t(E ent, A anc, const int* __restrict__ astart,
                                                    const CS* __restrict__ cstart, CellGrid G,
                                                    const float* __restrict__ SC, PairConsts C, Out out) {
  const int lane = threadIdx.x & 31;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long c = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; c < G.ncell; c += nwarps) {
    const int a0 = astart[c], a1 = astart[c + 1];
    if (a0 == a1) continue;
    long long cx, cy, g;
    cell_coords<CS>(c, G, &cx, &cy, &g);
    const float cs = __ldg(SC + g % G.S);
    const long long row0 = g * G.GH * G.GW;
    const long long xlo = cx > 0 ? cx - 1 : 0, xhi = cx + 1 < G.GW ? cx + 1 : G.GW - 1;
    const long long ylo = cy > 0 ? cy - 1 : 0, yhi = cy + 1 < G.GH ? cy + 1 : G.GH - 1;
    for (int base = a0; base < a1; base += 8) {
      const int na = min(8, a1 - base);
      switch (na) {
#define ATLB_FWD_CASE(n)                                                                                      \
  case n:                                                                                                     \
    fwd_group<n>(ent, anc, base, cstart, row0, G.GW, ylo, yhi, xlo, xhi, cs, C, out, lane);                   \
    break;
        ATLB_FWD_CASE(1) ATLB_FWD_CASE(2) ATLB_FWD_CASE(3) ATLB_FWD_CASE(4)
        ATLB_FWD_CASE(5) ATLB_FWD_CASE(6) ATLB_FWD_CASE(7) ATLB_FWD_CASE(8)
#undef ATLB_FWD_CASE
        default: break;
      }
    }
  }
}

// ---- backward ----------------------------------------------------------------------------------------
// gSb: the anchors' dL/dS in bucket order.  gv (N,2) receives sum over pairs of gS k r dt / h^2.
template <class E, class A, typename CS>
__global__ void __launch_bounds__(256) k_pair_bwd_t(E ent, A anc, const int* __restrict__ astart,
                                                    const float* __restrict__ gSb, const CS* __restrict__ cstart,
                                                    CellGrid G, const float* __restrict__ SC, PairConsts C,
                                                    long long N, float* __restrict__ gv) {
  const int lane = threadIdx.x & 31;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long c = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; c < G.ncell; c += nwarps) {
    const long long k0 = cstart[c], k1 = cstart[c + 1];
    if (k0 == k1) continue;
    long long cx, cy, g;
    cell_coords<CS>(c, G, &cx, &cy, &g);
    const float cs = __ldg(SC + g % G.S);
    const long long row0 = g * G.GH * G.GW;
    const long long xlo = cx > 0 ? cx - 1 : 0, xhi = cx + 1 < G.GW ? cx + 1 : G.GW - 1;
    const long long ylo = cy > 0 ? cy - 1 : 0, yhi = cy + 1 < G.GH ? cy + 1 : G.GH - 1;
    for (long long kb = k0; kb < k1; kb += 32) {
      const long long k = kb + lane;
      const bool valid = k < k1;
      float2 sy, sv;
      float st;
      typename E::Id sid;
      ent.load(valid ? k : k0, sy, sv, st, sid);
      float gx = 0.f, gy = 0.f;
      for (long long yy = ylo; yy <= yhi; ++yy) {
        const long long row = row0 + yy * G.GW;
        const int p0 = astart[row + xlo], p1 = astart[row + xhi + 1];
        for (int p = p0; p < p1; ++p) {
          const float gi = __ldg(gSb + p);
          if (gi == 0.f) continue;  // warp-uniform
          float ax, ay, at;
          typename A::Id aid;
          anc.load(p, ax, ay, at, aid);
          const float adt = sub_rn(at, cs);
          float rx, ry, d2, dt;
          if ((long long)sid != (long long)aid && pair_test(C, ax, ay, at, adt, sy, sv, st, &rx, &ry, &d2, &dt)) {
            const float f = pair_grad_factor(C, gi, pair_kernel(C, d2), dt);
            gx += mul_rn(f, rx);
            gy += mul_rn(f, ry);
          }
        }
      }
      const long long j = (long long)sid;
      if (valid && (gx != 0.f || gy != 0.f) && j >= 0 && j < N) red_add_f2(gv + 2 * j, gx, gy);
    }
  }
}

}  // namespace atlb
