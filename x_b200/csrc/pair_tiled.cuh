// Shared-memory tiled pair kernels of the fused path (compact entry layout).
//
// A CTA owns a tile of TX x TY cells of one slice grid g.
//   forward : the entries of the (TX+2) x (TY+2) cells around the tile are staged once in shared memory
//             with cp.async (each row of cells is one contiguous CSR range); the warps then walk the
//             tile's anchor cells: a cell's anchors in register groups of NA, the candidate rows of its
//             3x3 neighbourhood read from shared memory.  A tile whose neighbourhood does not fit reads
//             its candidates from global memory instead (same code, other pointer).
//   backward: the anchors (and their dL/dS) of the (TX+2) x (TY+2) cells are staged; each lane takes one
//             source entry of the tile and sums its gradient over the staged anchors of its 3x3 cells.
// The prologue (row offsets of the staged cells) is computed by one warp in parallel; several CTAs per
// SM overlap one CTA's staging with another's arithmetic.
#pragma once
#include "common.cuh"
#include "pair_kernels.cuh"
#include "pair_math.cuh"

namespace atlb {

constexpr int kTileX = 8;
constexpr int kTileY = 4;
constexpr int kTileThreads = 512;
constexpr int kStageCap = 3584;  // staged entries per CTA (forward): 3584 * 24 B = 84 KB -> 2 CTAs / SM
constexpr int kAncCap = 1536;    // staged anchors per CTA (backward): 1536 * 20 B = 30 KB

constexpr int kSR = kTileY + 2;  // staged rows
constexpr int kSC = kTileX + 2;  // staged columns

struct TileSmemFwd {
  float4 yv[kStageCap];
  float2 ti[kStageCap];
  int cell_off[kSR][kSC + 1];  // staged offset of each cell of a staged row (+ end)
  int row_k0[kSR];
  int row_base[kSR];
  int total, any;
};

struct TileSmemBwd {
  float4 xt[kAncCap];
  float gs[kAncCap];
  int cell_off[kSR][kSC + 1];
  int row_p0[kSR];
  int row_base[kSR];
  int total;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// Tile geometry shared by both kernels.
struct TileGeo {
  int tx0, tx1, ty0, ty1;  // tile cells [tx0, tx1) x [ty0, ty1)
  int sx0, sx1, sy0, sy1;  // staged cells (tile + 1-cell halo, clipped)
  long long gbase;         // first cell of grid g
};

__device__ __forceinline__ TileGeo tile_geo(const CellGrid& G) {
  TileGeo t;
  const int tiles_x = (int)((G.GW + kTileX - 1) / kTileX);
  t.tx0 = (blockIdx.x % tiles_x) * kTileX;
  t.ty0 = (blockIdx.x / tiles_x) * kTileY;
  t.tx1 = (int)min((long long)t.tx0 + kTileX, G.GW);
  t.ty1 = (int)min((long long)t.ty0 + kTileY, G.GH);
  t.sx0 = t.tx0 > 0 ? t.tx0 - 1 : 0;
  t.sx1 = t.tx1 < G.GW ? t.tx1 + 1 : (int)G.GW;
  t.sy0 = t.ty0 > 0 ? t.ty0 - 1 : 0;
  t.sy1 = t.ty1 < G.GH ? t.ty1 + 1 : (int)G.GH;
  t.gbase = (long long)blockIdx.y * G.GH * G.GW;
  return t;
}

// Offsets (relative to a compact staging buffer) of every staged cell, from a CSR array:
// off[r][c] for staged row r and column c in [0, nsc]; row0[r] = CSR index of the row's first cell;
// rbase[r] = the row's first slot in the buffer.  Executed by one full warp; *total = staged count.
template <typename CSR>
__device__ __forceinline__ void stage_offsets(const TileGeo& t, long long GW, const CSR* __restrict__ csr,
                                              int (*off)[kSC + 1], int* row0, int* rbase, int* total) {
  const int lane = threadIdx.x & 31;
  const int nsr = t.sy1 - t.sy0, nsc = t.sx1 - t.sx0;
  int len = 0, k0 = 0;
  if (lane < nsr) {
    const long long row = t.gbase + (long long)(t.sy0 + lane) * GW;
    k0 = (int)csr[row + t.sx0];
    len = (int)csr[row + t.sx1] - k0;
  }
  int incl = len;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  const int tot = __shfl_sync(0xffffffffu, incl, nsr > 0 ? nsr - 1 : 0);
  if (lane < nsr) {
    row0[lane] = k0;
    rbase[lane] = incl - len;
  }
  if (lane == 0) *total = nsr > 0 ? tot : 0;
  __syncwarp();
  for (int i = lane; i < nsr * (nsc + 1); i += 32) {
    const int r = i / (nsc + 1), c = i % (nsc + 1);
    const long long row = t.gbase + (long long)(t.sy0 + r) * GW;
    off[r][c] = (int)csr[row + t.sx0 + c] - row0[r] + rbase[r];
  }
  __syncwarp();
}

// 3x3 neighbourhood of tile cell (cx, cy) as up to 3 ranges [lo, hi) of a staged buffer (or of the global
// CSR when not staged).
template <typename CSR>
__device__ __forceinline__ int neighbour_rows(const TileGeo& t, long long GW, long long GH, int cx, int cy,
                                              bool staged, const int (*off)[kSC + 1],
                                              const CSR* __restrict__ csr, int* lo, int* hi) {
  int nrows = 0;
  const int xl = (cx > 0 ? cx - 1 : 0) - t.sx0, xh = (cx + 1 < GW ? cx + 1 : (int)GW - 1) - t.sx0 + 1;
  for (int y = (cy > 0 ? cy - 1 : 0); y <= cy + 1 && y < GH; ++y) {
    const int r = y - t.sy0;
    if (staged) {
      lo[nrows] = off[r][xl];
      hi[nrows] = off[r][xh];
    } else {
      const long long row = t.gbase + (long long)y * GW;
      lo[nrows] = (int)csr[row + t.sx0 + xl];
      hi[nrows] = (int)csr[row + t.sx0 + xh];
    }
    ++nrows;
  }
  return nrows;
}

// Candidate reads from shared memory (staged) or global memory (overflow tiles).
struct CandView {
  const float4* yv;
  const float2* ti;
};

template <int NA, class Out>
__device__ __forceinline__ void fwd_group_tile(const FastAnchors& anc, int base, const CandView& cv,
                                               const int* lo, const int* hi, int nrows, float cs,
                                               const PairConsts& C, Out& out, int lane) {
  float ax[NA], ay[NA], at[NA], adt[NA], acc[NA];
  int aid[NA];
#pragma unroll
  for (int q = 0; q < NA; ++q) {
    anc.load(base + q, ax[q], ay[q], at[q], aid[q]);
    adt[q] = sub_rn(at[q], cs);
    acc[q] = 0.f;
  }
  for (int r = 0; r < nrows; ++r) {
    const int k1 = hi[r];
    for (int k = lo[r] + lane; k < k1; k += 32) {
      const float4 e = cv.yv[k];
      const float2 f = cv.ti[k];
      const float2 sy = make_float2(e.x, e.y), sv = make_float2(e.z, e.w);
      const int sid = __float_as_int(f.y);
#pragma unroll
      for (int q = 0; q < NA; ++q) {
        float rx, ry, dt;
        acc[q] += pair_eval(C, ax[q], ay[q], at[q], adt[q], sy, sv, f.x, sid == aid[q], &rx, &ry, &dt);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < NA; ++q) {
    const float s = warp_sum(acc[q]);
    if (lane == 0) out(base + q, (double)s);
  }
}

template <class Out>
__global__ void __launch_bounds__(kTileThreads) k_pair_fwd_tiled(FastEntries ent, FastAnchors anc,
                                                                 const int* __restrict__ astart,
                                                                 const int* __restrict__ cstart, CellGrid G,
                                                                 const float* __restrict__ SC, PairConsts C, Out out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TileSmemFwd& sm = *reinterpret_cast<TileSmemFwd*>(smem_raw);
  const TileGeo t = tile_geo(G);
  const long long GW = G.GW, GH = G.GH;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;

  if (warp == 0) {
    // anchors in the tile? (lane r < TY: one row of the tile each)
    int na = 0;
    if (lane < t.ty1 - t.ty0) {
      const long long row = t.gbase + (long long)(t.ty0 + lane) * GW;
      na = astart[row + t.tx1] - astart[row + t.tx0];
    }
    na = __reduce_add_sync(0xffffffffu, na);
    if (na > 0) stage_offsets(t, GW, cstart, sm.cell_off, sm.row_k0, sm.row_base, &sm.total);
    if (lane == 0) sm.any = na;
  }
  __syncthreads();
  if (sm.any == 0) return;
  const int nsr = t.sy1 - t.sy0, nsc = t.sx1 - t.sx0;
  const bool staged = sm.total <= kStageCap;
  if (staged) {
    for (int r = 0; r < nsr; ++r) {
      const int k0 = sm.row_k0[r], b0 = sm.cell_off[r][0], n = sm.cell_off[r][nsc] - b0;
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        cp_async16(&sm.yv[b0 + i], ent.YV + k0 + i);
        cp_async8(&sm.ti[b0 + i], ent.TI + k0 + i);
      }
    }
    cp_async_wait_all();
  }
  __syncthreads();

  const float cs = __ldg(SC + blockIdx.y % G.S);
  const int ncx = t.tx1 - t.tx0, ncells = ncx * (t.ty1 - t.ty0);
  const CandView cv = staged ? CandView{sm.yv, sm.ti} : CandView{ent.YV, ent.TI};
  for (int ci = warp; ci < ncells; ci += nwarps) {
    const int cx = t.tx0 + ci % ncx, cy = t.ty0 + ci / ncx;
    const long long c = t.gbase + (long long)cy * GW + cx;
    const int a0 = astart[c], a1 = astart[c + 1];
    if (a0 == a1) continue;
    int lo[3], hi[3];
    const int nrows = neighbour_rows(t, GW, GH, cx, cy, staged, sm.cell_off, cstart, lo, hi);
    int base = a0;
    for (; base + 4 <= a1; base += 4) fwd_group_tile<4>(anc, base, cv, lo, hi, nrows, cs, C, out, lane);
    switch (a1 - base) {
      case 3: fwd_group_tile<3>(anc, base, cv, lo, hi, nrows, cs, C, out, lane); break;
      case 2: fwd_group_tile<2>(anc, base, cv, lo, hi, nrows, cs, C, out, lane); break;
      case 1: fwd_group_tile<1>(anc, base, cv, lo, hi, nrows, cs, C, out, lane); break;
      default: break;
    }
  }
}

// Backward: source entries of the tile, anchors of the (TX+2) x (TY+2) cells staged.
__global__ void __launch_bounds__(kTileThreads) k_pair_bwd_tiled(FastEntries ent, FastAnchors anc,
                                                                 const int* __restrict__ astart,
                                                                 const float* __restrict__ gSb,
                                                                 const int* __restrict__ cstart, CellGrid G,
                                                                 const float* __restrict__ SC, PairConsts C,
                                                                 long long N, float* __restrict__ gv) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TileSmemBwd& sm = *reinterpret_cast<TileSmemBwd*>(smem_raw);
  const TileGeo t = tile_geo(G);
  const long long GW = G.GW, GH = G.GH;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;

  if (warp == 0) stage_offsets(t, GW, astart, sm.cell_off, sm.row_p0, sm.row_base, &sm.total);
  __syncthreads();
  const int nsr = t.sy1 - t.sy0, nsc = t.sx1 - t.sx0;
  const bool staged = sm.total <= kAncCap;
  if (staged) {
    for (int r = 0; r < nsr; ++r) {
      const int p0 = sm.row_p0[r], b0 = sm.cell_off[r][0], n = sm.cell_off[r][nsc] - b0;
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        cp_async16(&sm.xt[b0 + i], anc.XT + p0 + i);
        cp_async4(&sm.gs[b0 + i], gSb + p0 + i);
      }
    }
    cp_async_wait_all();
  }
  __syncthreads();

  const float cs = __ldg(SC + blockIdx.y % G.S);
  const int ncx = t.tx1 - t.tx0, ncells = ncx * (t.ty1 - t.ty0);
  const float4* XT = staged ? sm.xt : anc.XT;
  const float* GS = staged ? sm.gs : gSb;
  for (int ci = warp; ci < ncells; ci += nwarps) {
    const int cx = t.tx0 + ci % ncx, cy = t.ty0 + ci / ncx;
    const long long c = t.gbase + (long long)cy * GW + cx;
    const int k0 = cstart[c], k1 = cstart[c + 1];
    if (k0 == k1) continue;
    int lo[3], hi[3];
    const int nrows = neighbour_rows(t, GW, GH, cx, cy, staged, sm.cell_off, astart, lo, hi);
    for (int kb = k0; kb < k1; kb += 32) {
      const int k = kb + lane;
      const bool valid = k < k1;
      float2 sy, sv;
      float st;
      int sid;
      ent.load(valid ? k : k0, sy, sv, st, sid);
      float gx = 0.f, gy = 0.f;
      for (int r = 0; r < nrows; ++r) {
        for (int p = lo[r]; p < hi[r]; ++p) {
          const float4 a = XT[p];
          const float gi = GS[p];
          float rx, ry, dt;
          const float e = pair_eval(C, a.x, a.y, a.z, sub_rn(a.z, cs), sy, sv, st, sid == __float_as_int(a.w),
                                    &rx, &ry, &dt);
          const float f = mul_rn(mul_rn(mul_rn(gi, e), dt), C.invh2);  // gS k dt / h^2 (atl_cpu.cpp:244)
          const bool hit = e != 0.f;
          gx += hit ? f * rx : 0.f;
          gy += hit ? f * ry : 0.f;
        }
      }
      if (valid && (gx != 0.f || gy != 0.f) && sid >= 0 && sid < N) red_add_f2(gv + 2 * (long long)sid, gx, gy);
    }
  }
}

}  // namespace atlb
