/*
 * atl_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CPU algorithm for the anchored-transport-score path
 * (KAVYANSHTYAGI/x, package `atl`).  It is the checker that tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg compare the CUDA library against; nothing in the product path
 * calls, links or loads it.
 *
 * Parity pin: every function here is checked bit-for-bit (integer outputs) or within 1e-6 relative
 * (float outputs) against outputs of the reference itself -- its torch code plus its OpenMP
 * extension csrc/atl_cpu.cpp -- committed as fixtures under tests/golden/ by
 * tests/golden/gen_golden.py.
 *
 * Floating point: compiled with -ffp-contract=off, so every `a * b + c` below rounds twice, as
 * torch's eager CPU ops and the reference's -O3 x86-64 build (no FMA instructions) do.  The one
 * place torch itself fuses (the row norm in the cell-size computation) calls fmaf explicitly.
 * Division by a Python scalar is an IEEE fp32 division on torch CPU (checked), not a reciprocal
 * multiply.
 */
#define _GNU_SOURCE
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_API __attribute__((visibility("default")))

static inline int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }
static inline int64_t imax64(int64_t a, int64_t b) { return a > b ? a : b; }
static inline float fclampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* ------------------------------------------------------------------------------------------------
 * Pair plan geometry.  atl/ops/functional.py:136-149 (build_pair_plan).
 *   vmax = max_j |v_j| with torch's row norm: sqrt(fma(vy, vy, vx*vx)) (functional.py:139)
 *   cell = max(cut*h + vmax*delta/2 + 1e-3, 1)                         (functional.py:140)
 *   origin / extent from the anchors' bounding box +- one cell         (functional.py:142-149)
 * ---------------------------------------------------------------------------------------------- */
ORACLE_API float oracle_vmax(const float* v, int64_t N) {
  float m = 0.f;
  for (int64_t j = 0; j < N; ++j) {
    const float vx = v[2 * j], vy = v[2 * j + 1];
    const float n = sqrtf(fmaf(vy, vy, vx * vx));
    if (n > m || n != n) m = n;
  }
  return m;
}

/* out[0..4] = cell, ox, oy, (double)GW, (double)GH */
ORACLE_API void oracle_plan_geometry(float vmax, const float* xa, int64_t M, int64_t H, int64_t W, double h,
                                     double cut, int64_t S, double* out) {
  const double delta = 1.0 / (double)S;
  double cell = cut * h + (double)vmax * delta / 2 + 1e-3;
  if (cell < 1.0) cell = 1.0;
  double ox, oy, ex, ey;
  if (M > 0) {
    float mnx = xa[0], mny = xa[1], mxx = xa[0], mxy = xa[1];
    for (int64_t i = 1; i < M; ++i) {
      const float x = xa[2 * i], y = xa[2 * i + 1];
      mnx = x < mnx ? x : mnx; mxx = x > mxx ? x : mxx;
      mny = y < mny ? y : mny; mxy = y > mxy ? y : mxy;
    }
    ox = (double)mnx - cell; oy = (double)mny - cell;
    ex = (double)mxx + cell; ey = (double)mxy + cell;
  } else {
    ox = -cell; oy = -cell; ex = (double)W + cell; ey = (double)H + cell;
  }
  out[0] = cell; out[1] = ox; out[2] = oy;
  out[3] = (double)((int64_t)ceil((ex - ox) / cell) + 1);
  out[4] = (double)((int64_t)ceil((ey - oy) / cell) + 1);
}

/* Slice range of one source, functional.py:151-153.  Returns the count (>= 0). */
static inline int64_t slice_range(float t, float tau_f, float hd_f, float delta_f, int64_t S, int64_t* lo) {
  const float a = ceilf((t - tau_f - hd_f) / delta_f - 0.5f);
  const float b = floorf((t + tau_f + hd_f) / delta_f - 0.5f);
  const int64_t s_lo = (int64_t)fclampf(a, 0.f, (float)(S - 1));
  const int64_t s_hi = (int64_t)fclampf(b, 0.f, (float)(S - 1));
  *lo = s_lo;
  const int64_t c = s_hi - s_lo + 1;
  return c > 0 ? c : 0;
}

/* Cell of the transported source, functional.py:157-161.  Returns the key or -1 when dropped. */
static inline int64_t source_key(float xj, float yj, float vx, float vy, float tj, float cs, int64_t bj, int64_t s,
                                 int64_t S, float ox_f, float oy_f, float cell_f, int64_t GW, int64_t GH,
                                 float* yx_out, float* yy_out) {
  const float dtc = cs - tj;
  const float yx = xj + vx * dtc, yy = yj + vy * dtc;
  const int64_t cx = (int64_t)floorf((yx - ox_f) / cell_f);
  const int64_t cy = (int64_t)floorf((yy - oy_f) / cell_f);
  *yx_out = yx; *yy_out = yy;
  if (cx < 0 || cx >= GW || cy < 0 || cy >= GH) return -1;
  return ((bj * S + s) * GH + cy) * GW + cx;
}

/* Number of plan entries (sources kept in the grid), functional.py:150-162. */
ORACLE_API int64_t oracle_plan_count(const float* x, const float* t, const float* v, const int64_t* b, int64_t N,
                                     int64_t S, double tau, const double* geom) {
  const double delta = 1.0 / (double)S;
  const float tau_f = (float)tau, hd_f = (float)(delta / 2), delta_f = (float)delta;
  const float ox_f = (float)geom[1], oy_f = (float)geom[2], cell_f = (float)geom[0];
  const int64_t GW = (int64_t)geom[3], GH = (int64_t)geom[4];
  int64_t n = 0;
  for (int64_t j = 0; j < N; ++j) {
    int64_t lo;
    const int64_t c = slice_range(t[j], tau_f, hd_f, delta_f, S, &lo);
    for (int64_t q = 0; q < c; ++q) {
      const int64_t s = lo + q;
      const float cs = ((float)s + 0.5f) * delta_f;
      float yx, yy;
      if (source_key(x[2 * j], x[2 * j + 1], v[2 * j], v[2 * j + 1], t[j], cs, b[j], s, S, ox_f, oy_f, cell_f, GW,
                     GH, &yx, &yy) >= 0)
        ++n;
    }
  }
  return n;
}

/* Full plan, functional.py:150-178.  Entries are emitted in a STABLE key order (the reference's
 * argsort is unstable; only the within-cell order can differ, which the kernels do not depend on).
 * cell_start has B*S*GH*GW + 1 entries. */
ORACLE_API void oracle_plan_build(const float* x, const float* t, const float* v, const int64_t* b, int64_t N,
                                  int64_t B, int64_t S, double tau, const double* geom, const int64_t* anchors,
                                  const float* anchor_xy, int64_t M, float* src_y, float* src_v, float* src_t,
                                  int64_t* src_id, int64_t* cell_start, float* anc_x, float* anc_t,
                                  int64_t* anc_cell, int64_t* anc_id, float* slice_c) {
  const double delta = 1.0 / (double)S;
  const float tau_f = (float)tau, hd_f = (float)(delta / 2), delta_f = (float)delta;
  const float ox_f = (float)geom[1], oy_f = (float)geom[2], cell_f = (float)geom[0];
  const int64_t GW = (int64_t)geom[3], GH = (int64_t)geom[4];
  const int64_t ncell = B * S * GH * GW;
  for (int64_t s = 0; s < S; ++s) slice_c[s] = ((float)s + 0.5f) * delta_f;
  memset(cell_start, 0, sizeof(int64_t) * (size_t)(ncell + 1));
  /* pass 1: counts */
  for (int64_t j = 0; j < N; ++j) {
    int64_t lo;
    const int64_t c = slice_range(t[j], tau_f, hd_f, delta_f, S, &lo);
    for (int64_t q = 0; q < c; ++q) {
      const int64_t s = lo + q;
      float yx, yy;
      const int64_t key = source_key(x[2 * j], x[2 * j + 1], v[2 * j], v[2 * j + 1], t[j], slice_c[s], b[j], s, S,
                                     ox_f, oy_f, cell_f, GW, GH, &yx, &yy);
      if (key >= 0) cell_start[key + 1]++;
    }
  }
  for (int64_t k = 0; k < ncell; ++k) cell_start[k + 1] += cell_start[k];
  /* pass 2: stable scatter (j ascending, then s ascending) */
  int64_t* cur = (int64_t*)malloc(sizeof(int64_t) * (size_t)(ncell > 0 ? ncell : 1));
  memcpy(cur, cell_start, sizeof(int64_t) * (size_t)ncell);
  for (int64_t j = 0; j < N; ++j) {
    int64_t lo;
    const int64_t c = slice_range(t[j], tau_f, hd_f, delta_f, S, &lo);
    for (int64_t q = 0; q < c; ++q) {
      const int64_t s = lo + q;
      float yx, yy;
      const int64_t key = source_key(x[2 * j], x[2 * j + 1], v[2 * j], v[2 * j + 1], t[j], slice_c[s], b[j], s, S,
                                     ox_f, oy_f, cell_f, GW, GH, &yx, &yy);
      if (key < 0) continue;
      const int64_t p = cur[key]++;
      src_y[2 * p] = yx; src_y[2 * p + 1] = yy;
      src_v[2 * p] = v[2 * j]; src_v[2 * p + 1] = v[2 * j + 1];
      src_t[p] = t[j]; src_id[p] = j;
    }
  }
  free(cur);
  /* anchors, functional.py:170-175 */
  for (int64_t i = 0; i < M; ++i) {
    const int64_t a = anchors[i];
    const float ta = t[a];
    const float xx = anchor_xy ? anchor_xy[2 * i] : x[2 * a];
    const float yy = anchor_xy ? anchor_xy[2 * i + 1] : x[2 * a + 1];
    const int64_t sa = (int64_t)fclampf(floorf(ta / delta_f), 0.f, (float)(S - 1));
    const int64_t acx = imin64(imax64((int64_t)floorf((xx - ox_f) / cell_f), 0), GW - 1);
    const int64_t acy = imin64(imax64((int64_t)floorf((yy - oy_f) / cell_f), 0), GH - 1);
    anc_x[2 * i] = xx; anc_x[2 * i + 1] = yy; anc_t[i] = ta;
    anc_cell[3 * i] = b[a] * S + sa; anc_cell[3 * i + 1] = acx; anc_cell[3 * i + 2] = acy;
    anc_id[i] = a;
  }
}

/* ------------------------------------------------------------------------------------------------
 * Anchored pair sums over the plan.  csrc/atl_cpu.cpp:176-253 (for_each_pair, ats_pair_fwd/bwd).
 * ---------------------------------------------------------------------------------------------- */
typedef struct {
  const float *SY, *SV, *ST, *AX, *AT, *SC;
  const int64_t *SID, *CS, *AC, *AID;
  int64_t S, GH, GW;
  float h, tau, cut;
} pair_args;

#define FOR_EACH_PAIR(A, i, BODY)                                                                             \
  do {                                                                                                        \
    const float xi = (A).AX[2 * (i)], yi = (A).AX[2 * (i) + 1], ti = (A).AT[(i)];                             \
    const int64_t g = (A).AC[3 * (i)], cx = (A).AC[3 * (i) + 1], cy = (A).AC[3 * (i) + 2], id = (A).AID[(i)]; \
    const float cs = (A).SC[g % (A).S];                                                                      \
    const float r2max = (A).cut * (A).cut * (A).h * (A).h, inv2h2 = 1.f / (2.f * (A).h * (A).h);             \
    for (int64_t yy = imax64(cy - 1, 0); yy <= imin64(cy + 1, (A).GH - 1); ++yy) {                            \
      for (int64_t xx = imax64(cx - 1, 0); xx <= imin64(cx + 1, (A).GW - 1); ++xx) {                          \
        const int64_t cell = (g * (A).GH + yy) * (A).GW + xx;                                                 \
        for (int64_t k = (A).CS[cell]; k < (A).CS[cell + 1]; ++k) {                                           \
          if ((A).SID[k] == id) continue;                                                                     \
          const float dt = ti - (A).ST[k];                                                                    \
          if (fabsf(dt) > (A).tau) continue;                                                                  \
          const float rx = xi - ((A).SY[2 * k] + (A).SV[2 * k] * (ti - cs));                                  \
          const float ry = yi - ((A).SY[2 * k + 1] + (A).SV[2 * k + 1] * (ti - cs));                          \
          const float d2 = rx * rx + ry * ry;                                                                 \
          if (d2 > r2max) continue;                                                                           \
          const float kern = expf(-d2 * inv2h2);                                                              \
          BODY                                                                                                \
        }                                                                                                     \
      }                                                                                                       \
    }                                                                                                         \
  } while (0)

static pair_args make_pair_args(const float* SY, const float* SV, const float* ST, const int64_t* SID,
                                const int64_t* CS, const float* AX, const float* AT, const int64_t* AC,
                                const int64_t* AID, const float* SC, int64_t S, int64_t GH, int64_t GW, double h,
                                double tau, double cut) {
  pair_args a;
  a.SY = SY; a.SV = SV; a.ST = ST; a.SID = SID; a.CS = CS; a.AX = AX; a.AT = AT; a.AC = AC; a.AID = AID;
  a.SC = SC; a.S = S; a.GH = GH; a.GW = GW; a.h = (float)h; a.tau = (float)tau; a.cut = (float)cut;
  return a;
}

/* ats_pair_fwd, csrc/atl_cpu.cpp:203-222: double accumulator per anchor.  Also reports the number
 * of contributing pairs (the roofline's work count) when hits != NULL. */
ORACLE_API void oracle_pair_fwd(const float* SY, const float* SV, const float* ST, const int64_t* SID,
                                const int64_t* CS, const float* AX, const float* AT, const int64_t* AC,
                                const int64_t* AID, const float* SC, int64_t M, int64_t S, int64_t GH, int64_t GW,
                                double h, double tau, double cut, float* out, int64_t* hits) {
  const pair_args A = make_pair_args(SY, SV, ST, SID, CS, AX, AT, AC, AID, SC, S, GH, GW, h, tau, cut);
  int64_t nh = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : nh)
  for (int64_t i = 0; i < M; ++i) {
    double acc = 0.0;
    FOR_EACH_PAIR(A, i, { acc += kern; ++nh; (void)rx; (void)ry; });
    out[i] = (float)acc;
  }
  if (hits) *hits = nh;
}

/* ats_pair_bwd, csrc/atl_cpu.cpp:224-253: gv[j] += gS_i * k * r * (t_i - t_j) / h^2.
 * Sequential over anchors (the reference uses omp atomics; the order only changes rounding). */
ORACLE_API void oracle_pair_bwd(const float* G, const float* SY, const float* SV, const float* ST,
                                const int64_t* SID, const int64_t* CS, const float* AX, const float* AT,
                                const int64_t* AC, const int64_t* AID, const float* SC, int64_t M, int64_t S,
                                int64_t GH, int64_t GW, double h, double tau, double cut, int64_t N, float* gv) {
  const pair_args A = make_pair_args(SY, SV, ST, SID, CS, AX, AT, AC, AID, SC, S, GH, GW, h, tau, cut);
  const float invh2 = 1.f / (float)(h * h);
  memset(gv, 0, sizeof(float) * (size_t)(2 * N));
  for (int64_t i = 0; i < M; ++i) {
    const float gi = G[i];
    if (gi == 0.f) continue;
    FOR_EACH_PAIR(A, i, {
      const float f = gi * kern * dt * invh2;
      const int64_t j = A.SID[k];
      gv[2 * j] += f * rx;
      gv[2 * j + 1] += f * ry;
    });
  }
}

/* The same gradient as oracle_pair_bwd with every contribution f*r (rounded as the reference rounds it)
 * summed in double: the accurate value that fp32 results of any summation order are compared against.
 * Also returns, per event component, the sum of |contribution| (gabs) and the number of contributions
 * (cnt): the ingredients of the fp32 summation bound |err| <= (cnt - 1) u sum|x| + per-term rounding. */
ORACLE_API void oracle_pair_bwd_f64(const float* G, const float* SY, const float* SV, const float* ST,
                                    const int64_t* SID, const int64_t* CS, const float* AX, const float* AT,
                                    const int64_t* AC, const int64_t* AID, const float* SC, int64_t M, int64_t S,
                                    int64_t GH, int64_t GW, double h, double tau, double cut, int64_t N, double* gv,
                                    double* gabs, int64_t* cnt) {
  const pair_args A = make_pair_args(SY, SV, ST, SID, CS, AX, AT, AC, AID, SC, S, GH, GW, h, tau, cut);
  const float invh2 = 1.f / (float)(h * h);
  memset(gv, 0, sizeof(double) * (size_t)(2 * N));
  memset(gabs, 0, sizeof(double) * (size_t)(2 * N));
  memset(cnt, 0, sizeof(int64_t) * (size_t)N);
  for (int64_t i = 0; i < M; ++i) {
    const float gi = G[i];
    if (gi == 0.f) continue;
    FOR_EACH_PAIR(A, i, {
      const float f = gi * kern * dt * invh2;
      const int64_t j = A.SID[k];
      const float cx = f * rx;
      const float cy = f * ry;
      gv[2 * j] += (double)cx;
      gv[2 * j + 1] += (double)cy;
      gabs[2 * j] += fabs((double)cx);
      gabs[2 * j + 1] += fabs((double)cy);
      cnt[j] += 1;
    });
  }
}

/* ------------------------------------------------------------------------------------------------
 * Splat / gather / voxel.  csrc/atl_cpu.cpp:17-33 (bilinear_corners), :38-131, :134-172, :256-286.
 * ---------------------------------------------------------------------------------------------- */
#define BILINEAR_CORNERS(x, y, H, W, BODY)                                          \
  do {                                                                              \
    const float fx0 = floorf(x), fy0 = floorf(y);                                   \
    const int64_t x0 = (int64_t)fx0, y0 = (int64_t)fy0;                             \
    const float ax = (x) - fx0, ay = (y) - fy0;                                     \
    const float wx[2] = {1.f - ax, ax}, wy[2] = {1.f - ay, ay};                     \
    const float dwx[2] = {-1.f, 1.f}, dwy[2] = {-1.f, 1.f};                         \
    for (int jj = 0; jj < 2; ++jj) {                                                \
      const int64_t yy = y0 + jj;                                                   \
      if (yy < 0 || yy >= (H)) continue;                                            \
      for (int ii = 0; ii < 2; ++ii) {                                              \
        const int64_t xx = x0 + ii;                                                 \
        if (xx < 0 || xx >= (W)) continue;                                          \
        const float c = wx[ii] * wy[jj], dcx = dwx[ii] * wy[jj], dcy = wx[ii] * dwy[jj]; \
        (void)dcx; (void)dcy;                                                       \
        BODY                                                                        \
      }                                                                             \
    }                                                                               \
  } while (0)

ORACLE_API void oracle_splat_bilinear_fwd(const float* P, const float* Wt, const int64_t* Bi, int64_t N, int64_t B,
                                          int64_t H, int64_t W, float* img) {
  memset(img, 0, sizeof(float) * (size_t)(B * H * W));
  for (int64_t n = 0; n < N; ++n) {
    const float wn = Wt[n];
    if (wn == 0.f) continue;
    float* base = img + Bi[n] * H * W;
    BILINEAR_CORNERS(P[2 * n], P[2 * n + 1], H, W, { base[yy * W + xx] += wn * c; });
  }
}

ORACLE_API void oracle_splat_bilinear_bwd(const float* G, const float* P, const float* Wt, const int64_t* Bi,
                                          int64_t N, int64_t H, int64_t W, float* gpos, float* gw) {
  for (int64_t n = 0; n < N; ++n) {
    const float* base = G + Bi[n] * H * W;
    float sx = 0.f, sy = 0.f, sw = 0.f;
    BILINEAR_CORNERS(P[2 * n], P[2 * n + 1], H, W, {
      const float g = base[yy * W + xx];
      sw += g * c; sx += g * dcx; sy += g * dcy;
    });
    gw[n] = sw; gpos[2 * n] = Wt[n] * sx; gpos[2 * n + 1] = Wt[n] * sy;
  }
}

ORACLE_API void oracle_splat_gauss_fwd(const float* P, const float* Wt, const int64_t* Bi, int64_t N, int64_t B,
                                       int64_t H, int64_t W, double sigma, int64_t R, float* img) {
  const float inv2s2 = 1.f / (2.f * (float)(sigma * sigma));
  const float norm = 1.f / (2.f * (float)M_PI * (float)(sigma * sigma));
  memset(img, 0, sizeof(float) * (size_t)(B * H * W));
  for (int64_t n = 0; n < N; ++n) {
    const float wn = Wt[n] * norm;
    if (wn == 0.f) continue;
    const float x = P[2 * n], y = P[2 * n + 1];
    const int64_t cx = (int64_t)lroundf(x), cy = (int64_t)lroundf(y);
    float* base = img + Bi[n] * H * W;
    for (int64_t yy = imax64(cy - R, 0); yy <= imin64(cy + R, H - 1); ++yy) {
      const float dy = (float)yy - y;
      for (int64_t xx = imax64(cx - R, 0); xx <= imin64(cx + R, W - 1); ++xx) {
        const float dx = (float)xx - x;
        base[yy * W + xx] += wn * expf(-(dx * dx + dy * dy) * inv2s2);
      }
    }
  }
}

ORACLE_API void oracle_splat_gauss_bwd(const float* G, const float* P, const float* Wt, const int64_t* Bi,
                                       int64_t N, int64_t H, int64_t W, double sigma, int64_t R, float* gpos,
                                       float* gw) {
  const float s2 = (float)(sigma * sigma), inv2s2 = 1.f / (2.f * s2), norm = 1.f / (2.f * (float)M_PI * s2);
  for (int64_t n = 0; n < N; ++n) {
    const float x = P[2 * n], y = P[2 * n + 1];
    const int64_t cx = (int64_t)lroundf(x), cy = (int64_t)lroundf(y);
    const float* base = G + Bi[n] * H * W;
    float sw = 0.f, sx = 0.f, sy = 0.f;
    for (int64_t yy = imax64(cy - R, 0); yy <= imin64(cy + R, H - 1); ++yy) {
      const float dy = (float)yy - y;
      for (int64_t xx = imax64(cx - R, 0); xx <= imin64(cx + R, W - 1); ++xx) {
        const float dx = (float)xx - x;
        const float gk = norm * expf(-(dx * dx + dy * dy) * inv2s2) * base[yy * W + xx];
        sw += gk; sx += gk * dx / s2; sy += gk * dy / s2;
      }
    }
    gw[n] = sw; gpos[2 * n] = Wt[n] * sx; gpos[2 * n + 1] = Wt[n] * sy;
  }
}

ORACLE_API void oracle_gather_fwd(const float* I, const float* P, const int64_t* Bi, int64_t N, int64_t H, int64_t W,
                                  float* out) {
  for (int64_t n = 0; n < N; ++n) {
    const float* base = I + Bi[n] * H * W;
    float s = 0.f;
    BILINEAR_CORNERS(P[2 * n], P[2 * n + 1], H, W, { s += c * base[yy * W + xx]; });
    out[n] = s;
  }
}

ORACLE_API void oracle_gather_bwd(const float* GV, const float* I, const float* P, const int64_t* Bi, int64_t N,
                                  int64_t B, int64_t H, int64_t W, float* gimg, float* gpos) {
  memset(gimg, 0, sizeof(float) * (size_t)(B * H * W));
  for (int64_t n = 0; n < N; ++n) {
    const float g = GV[n];
    const float* base = I + Bi[n] * H * W;
    float* gbase = gimg + Bi[n] * H * W;
    float sx = 0.f, sy = 0.f;
    BILINEAR_CORNERS(P[2 * n], P[2 * n + 1], H, W, {
      const float vv = base[yy * W + xx];
      sx += dcx * vv; sy += dcy * vv;
      gbase[yy * W + xx] += g * c;
    });
    gpos[2 * n] = g * sx; gpos[2 * n + 1] = g * sy;
  }
}

ORACLE_API void oracle_voxel_grid(const float* P, const float* T, const float* Pol, const int64_t* Bi, int64_t N,
                                  int64_t B, int64_t C, int64_t H, int64_t W, float* vox) {
  memset(vox, 0, sizeof(float) * (size_t)(B * C * H * W));
  for (int64_t n = 0; n < N; ++n) {
    const float x = P[2 * n], y = P[2 * n + 1], tn = T[n] * (float)(C - 1);
    const int64_t x0 = (int64_t)floorf(x), y0 = (int64_t)floorf(y), t0 = (int64_t)floorf(tn);
    for (int dt = 0; dt < 2; ++dt) {
      const int64_t tt = t0 + dt;
      if (tt < 0 || tt >= C) continue;
      const float wt = 1.f - fabsf((float)tt - tn);
      for (int dy = 0; dy < 2; ++dy) {
        const int64_t yy = y0 + dy;
        if (yy < 0 || yy >= H) continue;
        const float wy = 1.f - fabsf((float)yy - y);
        for (int dx = 0; dx < 2; ++dx) {
          const int64_t xx = x0 + dx;
          if (xx < 0 || xx >= W) continue;
          const float wx = 1.f - fabsf((float)xx - x);
          vox[((Bi[n] * C + tt) * H + yy) * W + xx] += Pol[n] * wt * wy * wx;
        }
      }
    }
  }
}

/* ------------------------------------------------------------------------------------------------
 * window_counts, atl/ops/functional.py:210-217: #{j != i, same batch, |t_j - t_i| <= tau} through
 * float64 keys b*4 + t, a sort and two binary searches.  Keys need not be sorted on entry.
 * ---------------------------------------------------------------------------------------------- */
static int cmp_double(const void* a, const void* b) {
  const double x = *(const double*)a, y = *(const double*)b;
  return (x > y) - (x < y);
}

ORACLE_API void oracle_window_counts(const float* t, const int64_t* b, int64_t N, const int64_t* idx, int64_t M,
                                     double tau, float* out) {
  double* ks = (double*)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
  for (int64_t j = 0; j < N; ++j) ks[j] = (double)b[j] * 4.0 + (double)t[j];
  qsort(ks, (size_t)N, sizeof(double), cmp_double);
  for (int64_t q = 0; q < M; ++q) {
    const int64_t i = idx[q];
    const double ki = (double)b[i] * 4.0 + (double)t[i];
    const double lo_key = ki - tau, hi_key = ki + tau;
    int64_t lo = 0, hi = N; /* left: first ks >= lo_key */
    while (lo < hi) { const int64_t m = (lo + hi) / 2; if (ks[m] < lo_key) lo = m + 1; else hi = m; }
    const int64_t L = lo;
    lo = 0; hi = N; /* right: first ks > hi_key */
    while (lo < hi) { const int64_t m = (lo + hi) / 2; if (ks[m] <= hi_key) lo = m + 1; else hi = m; }
    const int64_t c = lo - L - 1;
    out[q] = (float)(c > 0 ? c : 0);
  }
  free(ks);
}

/* ------------------------------------------------------------------------------------------------
 * Motion fields on the path (velocity of stage 1), evaluated as torch's eager CPU ops round them.
 *   DenseLinearFlow.field + sample_grid : atl/motion/parametric.py:273-277, :296-312
 *   Translation.field                   : parametric.py:152-153
 *   Affine.field                        : parametric.py:211-217 (bmm = a0*d0 then + a1*d1, no FMA)
 * ---------------------------------------------------------------------------------------------- */
static inline void sample_grid_one(const float* field, int64_t C, int64_t Hg, int64_t Wg, float gx, float gy,
                                   int64_t bb, float* out) {
  gx = fclampf(gx, 0.f, (float)(Wg - 1));
  gy = fclampf(gy, 0.f, (float)(Hg - 1));
  float x0 = floorf(gx), y0 = floorf(gy);
  const float mx = (float)(Wg - 2 > 0 ? Wg - 2 : 0), my = (float)(Hg - 2 > 0 ? Hg - 2 : 0);
  x0 = x0 > mx ? mx : x0; y0 = y0 > my ? my : y0;
  const float ax = gx - x0, ay = gy - y0;
  const int64_t ix0 = (int64_t)x0, iy0 = (int64_t)y0;
  const int64_t ix1 = imin64(ix0 + 1, Wg - 1), iy1 = imin64(iy0 + 1, Hg - 1);
  const float w00 = (1.f - ax) * (1.f - ay), w01 = ax * (1.f - ay), w10 = (1.f - ax) * ay, w11 = ax * ay;
  const float* F = field + bb * C * Hg * Wg;
  for (int64_t c = 0; c < C; ++c) {
    const float* Fc = F + c * Hg * Wg;
    const float f00 = Fc[iy0 * Wg + ix0], f01 = Fc[iy0 * Wg + ix1], f10 = Fc[iy1 * Wg + ix0], f11 = Fc[iy1 * Wg + ix1];
    out[c] = f00 * w00 + f01 * w01 + f10 * w10 + f11 * w11;
  }
}

/* kind: 0 translation (theta (B,2)), 1 affine (theta (B,6)), 2 dense (grid (B,2,Hg,Wg)). */
ORACLE_API void oracle_velocity(int kind, const float* theta, int64_t Hg, int64_t Wg, int64_t H, int64_t W,
                                const float* xy, const int64_t* b, int64_t N, float* v) {
  const float cxf = (float)((W - 1) / 2.0), cyf = (float)((H - 1) / 2.0);
  for (int64_t j = 0; j < N; ++j) {
    const int64_t bb = b[j];
    if (kind == 0) {
      v[2 * j] = theta[2 * bb]; v[2 * j + 1] = theta[2 * bb + 1];
    } else if (kind == 1) {
      const float* th = theta + 6 * bb;
      const float d0 = xy[2 * j] - cxf, d1 = xy[2 * j + 1] - cyf;
      const float p0 = th[2] * d0 + th[3] * d1, p1 = th[4] * d0 + th[5] * d1;
      v[2 * j] = th[0] + p0; v[2 * j + 1] = th[1] + p1;
    } else {
      const float gx = xy[2 * j] / (float)(W - 1 > 1 ? W - 1 : 1) * (float)(Wg - 1);
      const float gy = xy[2 * j + 1] / (float)(H - 1 > 1 ? H - 1 : 1) * (float)(Hg - 1);
      sample_grid_one(theta, 2, Hg, Wg, gx, gy, bb, v + 2 * j);
    }
  }
}

/* ------------------------------------------------------------------------------------------------
 * visible_fraction (exposure correction), atl/objectives/ats.py:31-50, for motions linear at the
 * event (transport = x + v(x) (c - t), parametric.py:114-117).  n_check slice centres.
 * ---------------------------------------------------------------------------------------------- */
ORACLE_API void oracle_visible_fraction(int kind, const float* theta, int64_t Hg, int64_t Wg, const float* xa,
                                        const float* ta, const int64_t* ba, int64_t M, const float* t,
                                        const int64_t* b, int64_t N, int64_t B, int64_t H, int64_t W, double tau,
                                        int64_t n_check, float* out) {
  float* counts = (float*)calloc((size_t)(B * n_check), sizeof(float));
  float* centres = (float*)malloc(sizeof(float) * (size_t)n_check);
  /* torch.linspace(0, 1, n+1) on CPU: step = 1/n, values i*step for i < half, 1 - (n-i)*step after */
  float* edges = (float*)malloc(sizeof(float) * (size_t)(n_check + 1));
  const float step = (float)(1.0 / (double)n_check);
  const int64_t halfway = (n_check + 1) / 2;
  for (int64_t i = 0; i <= n_check; ++i)
    edges[i] = i < halfway ? 0.f + step * (float)i : 1.f - step * (float)(n_check - i);
  for (int64_t k = 0; k < n_check; ++k) centres[k] = 0.5f * (edges[k] + edges[k + 1]);
  for (int64_t j = 0; j < N; ++j) {
    int64_t s = (int64_t)(t[j] * (float)n_check);
    s = imin64(imax64(s, 0), n_check - 1);
    counts[b[j] * n_check + s] += 1.f;
  }
  const float tau_f = (float)tau, wmax = (float)(W - 1), hmax = (float)(H - 1);
  for (int64_t i = 0; i < M; ++i) {
    float v[2];
    oracle_velocity(kind, theta, Hg, Wg, H, W, xa + 2 * i, ba + i, 1, v);
    float vis = 0.f, tot = 0.f;
    for (int64_t k = 0; k < n_check; ++k) {
      const float c = centres[k];
      const float near = fabsf(ta[i] - c) <= tau_f ? 1.f : 0.f;
      const float dt = c - ta[i];
      const float yx = xa[2 * i] + v[0] * dt, yy = xa[2 * i + 1] + v[1] * dt;
      const float inside = (yx >= 0.f && yx <= wmax && yy >= 0.f && yy <= hmax) ? 1.f : 0.f;
      const float w = counts[ba[i] * n_check + k] * near;
      vis += w * inside;
      tot += w;
    }
    const float r = vis / (tot < 1.f ? 1.f : tot);
    out[i] = r < 1e-3f ? 1e-3f : r;
  }
  free(counts); free(centres); free(edges);
}

/* ------------------------------------------------------------------------------------------------
 * Opt-in device draws (no counterpart in the reference, which draws with torch's CPU generator):
 * Philox4x32-10 as published by Salmon, Moraes, Dror and Shaw (SC'11), restated in plain C, and the
 * library's stream layout: item i of call c uses counter (i, (i >> 32) << 1 | stream, c, c >> 32) and
 * key (seed, seed >> 32); stream 0 = two uniforms (w >> 8) 2^-24, stream 1 = two Box-Muller normals
 * (computed here in double: the GPU's fp32 log / sincospi differ by a few ulp).
 * ---------------------------------------------------------------------------------------------- */
ORACLE_API void oracle_philox4x32_10(const uint32_t* ctr, const uint32_t* key, uint32_t* out) {
  uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3], k0 = key[0], k1 = key[1];
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0, hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    c0 = hi1 ^ c1 ^ k0;
    c1 = lo1;
    c2 = hi0 ^ c3 ^ k1;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

ORACLE_API void oracle_rng_draw2(int normal, uint64_t seed, uint64_t call, int64_t n, double* out) {
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t iu = (uint64_t)i;
    const uint32_t ctr[4] = {(uint32_t)iu, ((uint32_t)(iu >> 32) << 1) | (uint32_t)(normal ? 1 : 0), (uint32_t)call,
                             (uint32_t)(call >> 32)};
    uint32_t o[4];
    oracle_philox4x32_10(ctr, key, o);
    if (!normal) {
      out[2 * i] = (double)(o[0] >> 8) * 0x1p-24;
      out[2 * i + 1] = (double)(o[1] >> 8) * 0x1p-24;
    } else {
      const double u1 = (double)((o[0] >> 8) + 1u) * 0x1p-24, u2 = (double)(o[1] >> 8) * 0x1p-24;
      const double r = sqrt(-2.0 * log(u1));
      out[2 * i] = r * cos(2.0 * M_PI * u2);
      out[2 * i + 1] = r * sin(2.0 * M_PI * u2);
    }
  }
}

