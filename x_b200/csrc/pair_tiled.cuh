// Pair kernels: shared-memory tiled forward, cell-per-warp backward.  Templated on the entry layout: the
// fused path's compact records (FastEntries) or the reference's plan arrays (RefEntries, drop-in ops).
//
// Grid: (tile column, tile row, slice); each CTA walks the batches of its slice.  A tile is TX x TY cells.
//   forward : the entries of the (TX+2) x (TY+2) cells around the tile and the anchors of the tile are
//             staged in shared memory with cp.async (every row of cells is one contiguous CSR range);
//             each anchor record carries its leave-one-out term (fused layout) or its id (drop-in
//             layout, compared per pair).  Warps then walk the tile's
//             anchor cells: a cell's anchors in register groups of up to 4, the candidates of its 3x3
//             neighbourhood streamed by the lanes.  A tile whose neighbourhood does not fit reads its
//             candidates from global memory instead (same loop, global pointer); a tile with more anchors
//             than it stages is left to k_pair_fwd_overflow (warp per anchor cell, groups of up to 8).
//   backward: not tiled.  One warp per source cell, one entry per lane (a cell's last chunk of at most 16
//             entries spreads each entry over several lanes); the warp copies the anchor records of the
//             3x3 cells (prepared once per backward) into its own shared-memory list and the lanes walk it
//             (per warp: no CTA barriers, no per-tile set-up; a flat, unrolled walk with immediate offsets
//             instead of three row loops over global addresses).
// Index arithmetic is 32-bit and division-free (power-of-two tile width, one grid axis per coordinate):
// per-thread integer divisions by runtime values cost more than the pair arithmetic they surround.
#pragma once
#include "common.cuh"
#include "pair_kernels.cuh"
#include "pair_math.cuh"
#include "plan_math.cuh"

namespace atlb {

constexpr int kTileXLog = 3;
constexpr int kTileX = 1 << kTileXLog;  // 8
constexpr int kTileY = 4;
constexpr int kTileThreads = 512;
constexpr int kStageCap = 3456;   // staged entries per CTA (forward): 3456 * 16 B = 54 KB (+ 8 B each for t)
constexpr int kTileAncCap = 768;  // staged anchors per CTA (forward): 768 * 24 B = 18 KB

constexpr int kSR = kTileY + 2;  // staged rows
constexpr int kSC = kTileX + 2;  // staged columns

// Per-CTA work list: items (cell << 16 | part) sorted by decreasing cost, handed to warps by an atomic
// counter (longest-processing-time-first: the cost of a cell's work varies by ~40x across a tile).
constexpr int kMaxItems = 256;
struct WorkQueue {
  int item[kMaxItems];
  int cost[kMaxItems];
  int sorted[kMaxItems];
  int n, next;
};

// Sorts wq.item[0..n) by decreasing cost into wq.sorted (rank sort; n <= kMaxItems).  Whole CTA.
__device__ __forceinline__ void sort_items(WorkQueue& wq) {
  const int n = wq.n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int ci = wq.cost[i];
    int rank = 0;
    for (int j = 0; j < n; ++j) {
      const int cj = wq.cost[j];
      rank += (cj > ci) || (cj == ci && j < i);
    }
    wq.sorted[rank] = wq.item[i];
  }
  if (threadIdx.x == 0) wq.next = 0;
}

// Next item for this warp (-1 when done).
__device__ __forceinline__ int next_item(WorkQueue& wq, int lane) {
  int k = 0;
  if (lane == 0) k = atomicAdd(&wq.next, 1);
  k = __shfl_sync(0xffffffffu, k, 0);
  return k < wq.n ? wq.sorted[k] : -1;
}

struct TileSmemFwd {
  float4 yv[kStageCap];
  float4 anc[kTileAncCap];      // (x, y, t, a bits)
  int aidx[kTileAncCap];        // original anchor index
  int cell_off[kSR][kSC + 1];   // staged entry offset of each cell of a staged row (+ end)
  int row_k0[kSR];
  int row_base[kSR];
  int acell_off[kTileY][kTileX + 1];
  int arow_p0[kTileY];
  int arow_base[kTileY];
  int total, atotal;
  WorkQueue wq;
  float2 ti[kStageCap];  // entry times: staged only when tau does not cover the window (last member: the
                         // launch omits it from the dynamic shared memory otherwise)
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
__device__ __forceinline__ unsigned smem_addr(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ float4 lds128(unsigned a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float2 lds64(unsigned a) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
  return v;
}

// 32-bit grid shape of the tiled kernels (ncell < 2^31 is checked by the API).
struct TileGrid {
  int GW, GH, S, B;
};

struct TileGeo {
  int tx0, tx1, ty0, ty1;  // tile cells [tx0, tx1) x [ty0, ty1)
  int sx0, sx1, sy0, sy1;  // staged cells (tile + 1-cell halo, clipped)
};

__device__ __forceinline__ TileGeo tile_geo(const TileGrid& G) {
  TileGeo t;
  t.tx0 = (int)blockIdx.x << kTileXLog;
  t.ty0 = (int)blockIdx.y * kTileY;
  t.tx1 = min(t.tx0 + kTileX, G.GW);
  t.ty1 = min(t.ty0 + kTileY, G.GH);
  t.sx0 = max(t.tx0 - 1, 0);
  t.sx1 = min(t.tx1 + 1, G.GW);
  t.sy0 = max(t.ty0 - 1, 0);
  t.sy1 = min(t.ty1 + 1, G.GH);
  return t;
}

// Buffer offsets of a block of cells (rows [y0, y1), columns [x0, x1)) from a CSR array: off[r][c] = slot of
// cell (y0 + r, x0 + c) (c = x1 - x0 gives the row end), row0[r] = CSR index of the row's first cell,
// rbase[r] = the row's first slot.  Executed by one full warp; *total = the block's entries.
template <int NC, typename CS>
__device__ __forceinline__ void block_offsets(const CS* __restrict__ csr, int gbase, int GW, int y0, int y1, int x0,
                                              int x1, int (*off)[NC + 1], int* row0, int* rbase, int* total) {
  const int lane = threadIdx.x & 31;
  const int nr = y1 - y0, nc = x1 - x0;
  int len = 0, k0 = 0;
  if (lane < nr) {
    const int row = gbase + (y0 + lane) * GW;
    k0 = (int)csr[row + x0];
    len = (int)csr[row + x1] - k0;
  }
  int incl = len;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  const int tot = __shfl_sync(0xffffffffu, incl, nr > 0 ? nr - 1 : 0);
  if (lane < nr) {
    row0[lane] = k0;
    rbase[lane] = incl - len;
  }
  if (lane == 0) *total = nr > 0 ? tot : 0;
  __syncwarp();
  for (int r = 0; r < nr; ++r) {
    const int row = gbase + (y0 + r) * GW;
    for (int c = lane; c <= nc; c += 32) off[r][c] = (int)csr[row + x0 + c] - row0[r] + rbase[r];
  }
  __syncwarp();
}

// The 3x3 neighbourhood of tile cell (cx, cy) as up to 3 ranges [lo, hi) of the staged rows (or of the
// global CSR when not staged).
// The CSR ranges of the 3 cell rows (cy-1 .. cy+1, each spanning cells cx-1 .. cx+1 clipped to the grid)
// around cell (cx, cy); a row outside the grid gets an empty range.  Always 3 rows, so that callers
// unroll their row loops and lo/hi stay in registers.
template <typename CS>
__device__ __forceinline__ int neighbour_rows(const TileGeo& t, int gbase, int GW, int GH, int cx, int cy, bool staged,
                                              const int (*off)[kSC + 1], const CS* __restrict__ csr, int* lo,
                                              int* hi) {
  const int xl = max(cx - 1, 0), xh = min(cx + 1, GW - 1) + 1;
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const int y = cy - 1 + r;
    int l = 0, h = 0;
    if (y >= 0 && y < GH) {
      if (staged) {
        l = off[y - t.sy0][xl - t.sx0];
        h = off[y - t.sy0][xh - t.sx0];
      } else {
        const int row = gbase + y * GW;
        l = (int)csr[row + xl];
        h = (int)csr[row + xh];
      }
    }
    lo[r] = l;
    hi[r] = h;
  }
  return 3;
}

// Stage plan entry k into shared memory as (y, v) and, if asked, (t, id bits).  Compact layout: two copies;
// the reference's layout: four (its int64 id contributes its low word; ids are below 2^31).
__device__ __forceinline__ void stage_entry(const FastEntries& e, float4* dyv, float2* dti, int k, bool with_ti) {
  cp_async16(dyv, e.YV + k);
  if (with_ti) cp_async8(dti, e.TI + k);
}
__device__ __forceinline__ void stage_entry(const RefEntries& e, float4* dyv, float2* dti, int k, bool with_ti) {
  cp_async8(&dyv->x, e.SY + k);
  cp_async8(&dyv->z, e.SV + k);
  if (with_ti) {
    cp_async4(&dti->x, e.ST + k);
    cp_async4(&dti->y, e.SID + k);  // little-endian: the low 32 bits
  }
}

// Warp sums of NA (<= 8) values at once, by a transposing butterfly: each exchange step halves the values a lane
// holds, so NA sums cost about as many shuffles as two.  On return lane q * (32 / NP) holds the total of v[q]
// (NP = NA rounded up to a power of two); the other lanes hold partial sums.
template <int NA>
constexpr int sum_lane_stride() {
  return 32 / (NA <= 1 ? 1 : NA <= 2 ? 2 : NA <= 4 ? 4 : 8);
}
template <int NA>
__device__ __forceinline__ float warp_sum_many(const float (&v)[NA], int lane) {
  constexpr int NP = 32 / sum_lane_stride<NA>();
  float w[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) w[i] = i < NA ? v[i] : 0.f;
#pragma unroll
  for (int cnt = NP, off = 16; cnt > 1; cnt >>= 1, off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < cnt / 2; ++i) {
      const float send = upper ? w[i] : w[i + cnt / 2];
      const float keep = upper ? w[i + cnt / 2] : w[i];
      w[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
#pragma unroll
  for (int off = 16 / NP; off > 0; off >>= 1) w[0] += __shfl_xor_sync(0xffffffffu, w[0], off);
  return w[0];
}

// Leave-one-out: anchor a's own event appears among the candidates iff its entry of slice s exists and its
// cell lies in the anchor's 3x3 cells; returns that entry's (bit-identical) kernel value, else 0.
__device__ __forceinline__ float self_term(const PlanConsts& P, const PairConsts& C, const float4* __restrict__ ev4,
                                           int a, float xi, float yi, float ti, float dti, int b, int s, int cx,
                                           int cy) {
  if (a < P.src0 || a >= P.src1) return 0.f;  // the anchor's own event is not among this call's sources
  int s_lo, s_hi;
  slice_range(P, ti, &s_lo, &s_hi);
  if (s < s_lo || s > s_hi || b < 0 || b >= P.B) return 0.f;
  const float4 e = __ldg(ev4 + a);
  const float dtc = sub_rn(slice_centre(P, s), ti);
  const float yx = add_rn(e.x, mul_rn(e.z, dtc)), yy = add_rn(e.y, mul_rn(e.w, dtc));
  const float qx = floorf(div_rn(sub_rn(yx, P.ox_f), P.cell_f));
  const float qy = floorf(div_rn(sub_rn(yy, P.oy_f), P.cell_f));
  if (!(qx >= 0.f && qx < (float)P.GW && qy >= 0.f && qy < (float)P.GH)) return 0.f;
  const int ex = (int)qx, ey = (int)qy;
  if (ex < cx - 1 || ex > cx + 1 || ey < cy - 1 || ey > cy + 1) return 0.f;
  float2 r;
  const float d2 = residual2(pk2(xi, yi), pk2(dti, dti), pk2(yx, yy), pk2(e.z, e.w), &r);
  const float k = ex2_approx(-d2 * C.k2);
  return (d2 > C.r2max) ? 0.f : k;  // dt = 0: inside any tau
}

// ---- forward -----------------------------------------------------------------------------------------
// Anchor records (x, y, t, w).  Fused layout: w = the anchor's own pair value, self_term() evaluated once per
// anchor when the records are built, subtracted from the sum.  LOO_ID (the reference's plan layout, where an
// anchor's own entry cannot be located): w = the low 32 bits of the anchor's id, and pairs are excluded by
// comparing ids.
template <int NA, bool TAU_ALL, bool LOO_ID, bool STAGED, class E, class Out>
__device__ __forceinline__ void fwd_group_tile(const TileSmemFwd& sm, int p, const E& ent, const int* lo,
                                               const int* hi, float cs, const PairConsts& C, Out& out, int lane) {
  constexpr bool kTI = !TAU_ALL || LOO_ID;  // entry times / ids needed
  f32x2 axy[NA], adt2[NA];
  float at[NA], acc[NA];
  int aid[NA];
#pragma unroll
  for (int q = 0; q < NA; ++q) {
    const float4 a = sm.anc[p + q];
    const float adt = sub_rn(a.z, cs);
    axy[q] = pk2(a.x, a.y);
    adt2[q] = pk2(adt, adt);
    at[q] = a.z;
    aid[q] = __float_as_int(a.w);
    acc[q] = 0.f;
  }
  const unsigned yv_s = STAGED ? smem_addr(sm.yv) : 0u, ti_s = STAGED ? smem_addr(sm.ti) : 0u;
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const int k1 = hi[r];
    for (int k = lo[r] + lane; k < k1; k += 32) {
      float4 e;
      float st = 0.f;
      int eid = 0;
      if (STAGED) {
        e = lds128(yv_s + 16u * (unsigned)k);
        if (kTI) {
          const float2 q = lds64(ti_s + 8u * (unsigned)k);
          st = q.x;
          eid = __float_as_int(q.y);
        }
      } else {
        e = ent.yv(k);
        if (kTI) {
          st = ent.t(k);
          eid = ent.id(k);
        }
      }
      const f32x2 y = pk2(e.x, e.y), v = pk2(e.z, e.w);
#pragma unroll
      for (int q = 0; q < NA; ++q) {
        float2 rr;
        const float d2 = residual2(axy[q], adt2[q], y, v, &rr);
        bool ok = !(d2 > C.r2max);
        if (!TAU_ALL) ok = ok && !(fabsf(sub_rn(at[q], st)) > C.tau);
        if (LOO_ID) ok = ok && eid != aid[q];
        const float kv = ex2_approx(-d2 * C.k2);
        acc[q] += ok ? kv : 0.f;
      }
    }
  }
  const float sum = warp_sum_many<NA>(acc, lane);
  constexpr int kStride = sum_lane_stride<NA>();
  const int q = lane / kStride;
  if (lane % kStride == 0 && q < NA) out(sm.aidx[p + q], (double)(LOO_ID ? sum : sum - sm.anc[p + q].w));
}

// Bits of the overflow word shared by the tiled and untiled forward kernels.
constexpr int kOverflowTiles = 1;  // some tile has more anchors than the tiled kernel stages
constexpr int kOverflowAll = 2;    // set by the caller before the launch: the untiled kernel takes every cell

// out(i, S_i) with i the original anchor index.  A tile with more than kTileAncCap anchors sets *overflow
// and leaves its anchors to the caller's untiled pass.
template <bool TAU_ALL, bool LOO_ID, class E, typename CS, class Out>
__global__ void __launch_bounds__(kTileThreads) k_pair_fwd_tiled(E ent, FastAnchors anc,
                                                                 const int* __restrict__ astart,
                                                                 const CS* __restrict__ cstart, TileGrid G,
                                                                 const float* __restrict__ SC, PairConsts C, Out out,
                                                                 int* __restrict__ overflow) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TileSmemFwd& sm = *reinterpret_cast<TileSmemFwd*>(smem_raw);
  if (LOO_ID && (*overflow & kOverflowAll)) return;  // ids beyond 32 bits: every cell goes to the untiled kernel
  const TileGeo t = tile_geo(G);
  const int GW = G.GW, GH = G.GH, s = (int)blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const float cs = __ldg(SC + s);
  const int nsc = t.sx1 - t.sx0, ntx = t.tx1 - t.tx0, nty = t.ty1 - t.ty0;

  for (int b = 0; b < G.B; ++b) {
    const int gbase = (b * G.S + s) * GH * GW;
    if (warp == 0) {
      block_offsets<kTileX>(astart, gbase, GW, t.ty0, t.ty1, t.tx0, t.tx1, sm.acell_off, sm.arow_p0, sm.arow_base,
                            &sm.atotal);
      block_offsets<kSC>(cstart, gbase, GW, t.sy0, t.sy1, t.sx0, t.sx1, sm.cell_off, sm.row_k0, sm.row_base,
                         &sm.total);
    }
    __syncthreads();
    const int na = sm.atotal;
    const bool staged = sm.total <= kStageCap;
    if (na == 0 || na > kTileAncCap) {  // CTA-uniform
      if (na > kTileAncCap && threadIdx.x == 0) atomicOr(overflow, kOverflowTiles);
      __syncthreads();
      continue;
    }
    // stage the tile's anchors (contiguous per tile row) and, if they fit, the neighbourhood's entries
    for (int r = 0; r < nty; ++r) {
      const int p0 = sm.arow_p0[r], b0 = sm.acell_off[r][0], n = sm.acell_off[r][ntx] - b0;
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        cp_async16(&sm.anc[b0 + i], anc.XT + p0 + i);
        cp_async4(&sm.aidx[b0 + i], anc.idx + p0 + i);
      }
    }
    if (staged) {
      for (int r = 0; r < t.sy1 - t.sy0; ++r) {
        const int k0 = sm.row_k0[r], b0 = sm.cell_off[r][0], n = sm.cell_off[r][nsc] - b0;
        for (int i = threadIdx.x; i < n; i += blockDim.x)
          stage_entry(ent, &sm.yv[b0 + i], &sm.ti[b0 + i], k0 + i, !TAU_ALL || LOO_ID);
      }
    }
    // work items: (cell, group of <= 4 anchors), cost = anchors x candidates
    if (warp == 0) {
      int ng = 0, cand = 0, p0 = 0;
      const int cxo = lane & (kTileX - 1), cyo = lane >> kTileXLog;
      if (lane < kTileX * kTileY && cxo < ntx && cyo < nty) {
        p0 = sm.acell_off[cyo][cxo];
        ng = (sm.acell_off[cyo][cxo + 1] - p0 + 3) >> 2;
        int lo[3], hi[3];
        const int nr = neighbour_rows(t, gbase, GW, GH, t.tx0 + cxo, t.ty0 + cyo, staged, sm.cell_off, cstart, lo, hi);
#pragma unroll
        for (int r = 0; r < 3; ++r) cand += hi[r] - lo[r];
      }
      int incl = ng;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      const int total_items = __shfl_sync(0xffffffffu, incl, 31);
      const int p1 = lane < kTileX * kTileY && cxo < ntx && cyo < nty ? sm.acell_off[cyo][cxo + 1] : 0;
      for (int gi = 0; gi < ng; ++gi) {
        const int slot = incl - ng + gi;
        if (slot < kMaxItems) {
          sm.wq.item[slot] = (lane << 16) | gi;
          sm.wq.cost[slot] = min(4, p1 - (p0 + 4 * gi)) * cand;
        }
      }
      if (lane == 0) sm.wq.n = min(total_items, kMaxItems);
    }
    cp_async_wait_all();
    __syncthreads();
    sort_items(sm.wq);
    __syncthreads();
    for (int it = next_item(sm.wq, lane); it >= 0; it = next_item(sm.wq, lane)) {
      const int ci = it >> 16, gi = it & 0xffff;
      const int cxo = ci & (kTileX - 1), cyo = ci >> kTileXLog;
      const int p = sm.acell_off[cyo][cxo] + 4 * gi, p1 = sm.acell_off[cyo][cxo + 1];
      int lo[3], hi[3];
      const int nrows = neighbour_rows(t, gbase, GW, GH, t.tx0 + cxo, t.ty0 + cyo, staged, sm.cell_off, cstart, lo, hi);
      const int na_g = min(4, p1 - p);
      const int cx = t.tx0 + cxo, cy = t.ty0 + cyo;
#define ATLB_GROUP(n, st) fwd_group_tile<n, TAU_ALL, LOO_ID, st>(sm, p, ent, lo, hi, cs, C, out, lane)
      if (staged) {
        switch (na_g) {
          case 4: ATLB_GROUP(4, true); break;
          case 3: ATLB_GROUP(3, true); break;
          case 2: ATLB_GROUP(2, true); break;
          default: ATLB_GROUP(1, true); break;
        }
      } else {
        switch (na_g) {
          case 4: ATLB_GROUP(4, false); break;
          case 3: ATLB_GROUP(3, false); break;
          case 2: ATLB_GROUP(2, false); break;
          default: ATLB_GROUP(1, false); break;
        }
      }
#undef ATLB_GROUP
    }
    __syncthreads();  // the next batch reuses the shared buffers
  }
}

// ---- forward, untiled (cells the tiled kernel leaves: tiles with more anchors than it stages) -----------
// One warp per anchor cell: its anchors in register groups of up to 8, the candidates of the 3 neighbouring
// cell rows streamed from global memory (L1) by the lanes; the same arithmetic as the tiled kernel.  With
// LOO_ID the ids are compared at full width: AID holds the anchors' ids by original index.
template <int NA, bool TAU_ALL, bool LOO_ID, class E, class Out>
__device__ __forceinline__ void fwd_group_cells(const E& ent, const FastAnchors& anc,
                                                const long long* __restrict__ AID, int p, const int* lo,
                                                const int* hi, float cs, const PairConsts& C, Out& out, int lane) {
  f32x2 axy[NA], adt2[NA];
  float at[NA], acc[NA];
  long long aid[NA];
#pragma unroll
  for (int q = 0; q < NA; ++q) {
    const float4 a = __ldg(anc.XT + p + q);
    const float adt = sub_rn(a.z, cs);
    axy[q] = pk2(a.x, a.y);
    adt2[q] = pk2(adt, adt);
    at[q] = a.z;
    aid[q] = LOO_ID ? __ldg(AID + __ldg(anc.idx + p + q)) : 0;
    acc[q] = 0.f;
  }
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const int k1 = hi[r];
    for (int k = lo[r] + lane; k < k1; k += 32) {
      const float4 e = ent.yv(k);
      const float st = TAU_ALL ? 0.f : ent.t(k);
      long long eid = 0;
      if constexpr (LOO_ID) eid = ent.id64(k);
      const f32x2 y = pk2(e.x, e.y), v = pk2(e.z, e.w);
#pragma unroll
      for (int q = 0; q < NA; ++q) {
        float2 rr;
        const float d2 = residual2(axy[q], adt2[q], y, v, &rr);
        bool ok = !(d2 > C.r2max);
        if (!TAU_ALL) ok = ok && !(fabsf(sub_rn(at[q], st)) > C.tau);
        if (LOO_ID) ok = ok && eid != aid[q];
        const float kv = ex2_approx(-d2 * C.k2);
        acc[q] += ok ? kv : 0.f;
      }
    }
  }
  const float sum = warp_sum_many<NA>(acc, lane);
  constexpr int kStride = sum_lane_stride<NA>();
  const int q = lane / kStride;
  if (lane % kStride == 0 && q < NA)
    out(__ldg(anc.idx + p + q), (double)(LOO_ID ? sum : sum - __ldg(&anc.XT[p + q].w)));
}

// Anchor cells of the tiles with more than kTileAncCap anchors (the tiled kernel set kOverflowTiles), or of
// every tile when the caller set kOverflowAll.
template <bool TAU_ALL, bool LOO_ID, class E, typename CS, class Out>
__global__ void __launch_bounds__(256) k_pair_fwd_overflow(E ent, FastAnchors anc, const long long* __restrict__ AID,
                                                           const int* __restrict__ astart,
                                                           const CS* __restrict__ cstart, TileGrid G,
                                                           const float* __restrict__ SC, PairConsts C, Out out,
                                                           const int* __restrict__ overflow) {
  const int flags = *overflow;
  if (flags == 0) return;
  const bool all = LOO_ID && (flags & kOverflowAll);
  const int lane = threadIdx.x & 31;
  const long long ncell = (long long)G.B * G.S * G.GH * G.GW;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long c = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; c < ncell; c += nwarps) {
    const int a0 = astart[c], a1 = astart[c + 1];
    if (a0 == a1) continue;
    const int GW = G.GW, GH = G.GH;
    const int row = (int)(c / GW), cx = (int)(c - (long long)row * GW);
    const int g = row / GH, cy = row - g * GH;
    const int b = g / G.S, s = g - b * G.S;
    const int gbase = g * GH * GW;
    if (!all) {  // the cell's tile and its anchor count, as the tiled kernel saw it
      const int tx0 = (cx >> kTileXLog) << kTileXLog, ty0 = (cy / kTileY) * kTileY;
      const int tx1 = min(tx0 + kTileX, GW), ty1 = min(ty0 + kTileY, GH);
      int na = 0;
      for (int y = ty0; y < ty1; ++y) na += astart[gbase + y * GW + tx1] - astart[gbase + y * GW + tx0];
      if (na <= kTileAncCap) continue;
    }
    const int xl = max(cx - 1, 0), xh = min(cx + 1, GW - 1) + 1;
    int lo[3], hi[3];
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      const int y = cy - 1 + r;
      int l = 0, h = 0;
      if (y >= 0 && y < GH) {
        l = (int)cstart[gbase + y * GW + xl];
        h = (int)cstart[gbase + y * GW + xh];
      }
      lo[r] = l;
      hi[r] = h;
    }
    const float cs = __ldg(SC + s);
    for (int p = a0; p < a1; p += 8) {
      switch (min(8, a1 - p)) {
#define ATLB_OVF(n) \
  case n: fwd_group_cells<n, TAU_ALL, LOO_ID>(ent, anc, AID, p, lo, hi, cs, C, out, lane); break;
        ATLB_OVF(8) ATLB_OVF(7) ATLB_OVF(6) ATLB_OVF(5) ATLB_OVF(4) ATLB_OVF(3) ATLB_OVF(2)
#undef ATLB_OVF
        default: fwd_group_cells<1, TAU_ALL, LOO_ID>(ent, anc, AID, p, lo, hi, cs, C, out, lane); break;
      }
    }
  }
}

// ---- backward ----------------------------------------------------------------------------------------
constexpr int kBwdWarps = 8;   // warps (source cells) per CTA
constexpr int kBwdAnc = 128;   // anchor records a warp stages at a time

// Gradient of one entry (y, v, t, id) over the staged anchors i = g, g + G, ... < na (g = 0, G = 1: every
// anchor, a warp-uniform loop).
template <bool TAU_ALL, bool LOO_ID, bool STRIDED, typename Id>
__device__ __forceinline__ float2 bwd_entry(const float4* ab, const float2* gt, const long long* gid, int na,
                                            f32x2 y, f32x2 v, float st, Id sid, int g, int G, const PairConsts& C) {
  float gx = 0.f, gy = 0.f;
#pragma unroll 4
  for (int i = STRIDED ? g : 0; i < na; i += STRIDED ? G : 1) {
    const float4 a = ab[i];   // (x, y, t - c_s, t - c_s): both pairs are packed operands as loaded
    const float2 q = gt[i];   // (dL/dS / h^2, t)
    float2 rr;
    const float d2 = residual2(pk2(a.x, a.y), pk2(a.z, a.w), y, v, &rr);
    const float dt = sub_rn(q.y, st);
    bool ok = !(d2 > C.r2max);
    if (!TAU_ALL) ok = ok && !(fabsf(dt) > C.tau);
    if (LOO_ID) ok = ok && (long long)sid != gid[i];
    const float f = ok ? q.x * ex2_approx(-d2 * C.k2) * dt : 0.f;  // gS k dt / h^2
    gx = fmaf(f, rr.x, gx);
    gy = fmaf(f, rr.y, gy);
  }
  return make_float2(gx, gy);
}

// One warp per source cell (grid: x = groups of 8 cells of a cell row, y = cell rows of all (batch, slice)
// grids).  The anchor records of the 3 neighbouring cell rows, AB = (x, y, t - c_s, t - c_s) and
// GT = (dL/dS / h^2, t) in bucket order (prepared once per backward), are copied by the warp into its own
// shared-memory arrays, up to kBwdAnc at a time, as one flat list; the lanes then walk that list with
// broadcast shared loads, one entry of the cell per lane, in chunks of 32 entries.  A last chunk of m <= 16
// entries would leave most lanes idle: there each entry gets G = floor(32 / m) lanes, lane g of them taking
// every G-th anchor, and the G partial gradients are summed by shuffles.  Leave-one-out: the anchor's own
// pair has dt = 0 and adds nothing in the fused layout; with LOO_ID the pair is excluded by comparing the
// entry's id with the anchor's (GID, bucket order), as the reference does.
template <bool TAU_ALL, bool LOO_ID, class E, typename CS>
__global__ void __launch_bounds__(kBwdWarps * 32, LOO_ID ? 5 : 6) k_pair_bwd_cells(E ent, const float4* __restrict__ AB,
                                                                    const float2* __restrict__ GT,
                                                                    const long long* __restrict__ GID,
                                                                    const int* __restrict__ astart,
                                                                    const CS* __restrict__ cstart, int GW, int GH,
                                                                    int nrows, PairConsts C, long long N,
                                                                    float* __restrict__ gv) {
  __shared__ float4 s_ab[kBwdWarps][kBwdAnc];
  __shared__ float2 s_gt[kBwdWarps][kBwdAnc];
  __shared__ long long s_id[LOO_ID ? kBwdWarps : 1][LOO_ID ? kBwdAnc : 1];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int cx = blockIdx.x * kBwdWarps + w;
  if (cx >= GW) return;  // warp-uniform; no CTA-wide barrier follows
  float4* ab = s_ab[w];
  float2* gt = s_gt[w];
  long long* gid = s_id[LOO_ID ? w : 0];
  for (int row = blockIdx.y; row < nrows; row += gridDim.y) {  // row = (b * S + s) * GH + cy
    const int cy = row % GH;
    const int c = row * GW + cx;
    const int k0 = (int)cstart[c], k1 = (int)cstart[c + 1];
    if (k0 == k1) continue;
    const int gbase = (row - cy) * GW;
    const int xl = max(cx - 1, 0), xh = min(cx + 1, GW - 1) + 1;
    int lo[3], len[3];
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      const int y = cy - 1 + r;
      int l = 0, h = 0;
      if (y >= 0 && y < GH) {
        l = astart[gbase + y * GW + xl];
        h = astart[gbase + y * GW + xh];
      }
      lo[r] = l;
      len[r] = h - l;
    }
    const int A = len[0] + len[1] + len[2];
    for (int a0 = 0; a0 < A; a0 += kBwdAnc) {
      const int na = min(kBwdAnc, A - a0);
      __syncwarp();  // the previous batch of records is no longer read
      for (int i = lane; i < na; i += 32) {
        const int f = a0 + i;  // flat index over the 3 rows
        const int p = f < len[0] ? lo[0] + f : (f < len[0] + len[1] ? lo[1] + (f - len[0]) : lo[2] + (f - len[0] - len[1]));
        ab[i] = __ldg(AB + p);
        gt[i] = __ldg(GT + p);
        if (LOO_ID) gid[i] = __ldg(GID + p);
      }
      __syncwarp();
      for (int kb = k0; kb < k1; kb += 32) {
        const int m = min(32, k1 - kb);
        float2 sy, sv;
        float st;
        typename E::Id sid;
        if (m > 16) {  // warp-uniform: one entry per lane, every lane walks every anchor
          const bool valid = lane < m;
          ent.load(kb + (valid ? lane : 0), sy, sv, st, sid);
          const float2 gr = bwd_entry<TAU_ALL, LOO_ID, false>(ab, gt, gid, na, pk2(sy.x, sy.y), pk2(sv.x, sv.y), st,
                                                              sid, 0, 1, C);
          if (valid && (gr.x != 0.f || gr.y != 0.f) && sid >= 0 && (long long)sid < N)
            red_add_f2(gv + 2 * (long long)sid, gr.x, gr.y);
        } else {
          // G lanes per entry: entry e = lane / G, part g = lane % G.  The float quotients are exact after
          // truncation: 32.5 / m and (lane + 0.5) / G lie at least 1/64 from an integer.
          const int G = (int)__fdividef(32.5f, (float)m);
          const int e = (int)__fdividef((float)lane + 0.5f, (float)G);
          const int g = lane - e * G;
          const bool valid = e < m;
          ent.load(kb + (valid ? e : 0), sy, sv, st, sid);
          float2 gr = bwd_entry<TAU_ALL, LOO_ID, true>(ab, gt, gid, valid ? na : 0, pk2(sy.x, sy.y), pk2(sv.x, sv.y),
                                                       st, sid, g, G, C);
          for (int d = 1; d < G; d <<= 1) {  // tree sum of each entry's G partials into its lane g = 0
            const float ox = __shfl_down_sync(0xffffffffu, gr.x, d), oy = __shfl_down_sync(0xffffffffu, gr.y, d);
            if ((g & (2 * d - 1)) == 0 && g + d < G) {
              gr.x += ox;
              gr.y += oy;
            }
          }
          if (valid && g == 0 && (gr.x != 0.f || gr.y != 0.f) && sid >= 0 && (long long)sid < N)
            red_add_f2(gv + 2 * (long long)sid, gr.x, gr.y);
        }
      }
    }
  }
}

}  // namespace atlb
