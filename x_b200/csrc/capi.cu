// extern "C" boundary of libatlb200.so (declarations and reference citations in include/atl_b200.h).
// Validates arguments, forwards to the kernels' launchers and turns CUDA errors into status codes.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"
#include "motion_math.cuh"
#include "plan_math.cuh"
#include "traj.cuh"

namespace atlb {

static thread_local char g_err[512] = "";
std::atomic<unsigned long long> g_launches{0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return ATLB_ERR_CUDA;
  }
  return ATLB_OK;
}

// launchers (plan.cu, pair.cu, splat.cu, motion.cu)
int plan_geometry(const float*, const float*, long long, const long long*, const float*, long long, long long,
                  long long, double, double, long long, void*, atlb_plan_geom*, cudaStream_t);
size_t plan_workspace_bytes(long long ncell);
int plan_count(const float*, const float*, const float*, const long long*, long long, long long, double,
               const atlb_plan_geom*, long long*, void*, long long*, cudaStream_t);
int plan_fill(const float*, const float*, const float*, const long long*, long long, long long, double,
              const atlb_plan_geom*, const long long*, const float*, long long, const long long*, void*, float*,
              float*, float*, long long*, float*, float*, long long*, long long*, float*, cudaStream_t);
size_t pair_workspace_bytes(long long M, long long ncell);
size_t unit_rates_scratch_bytes();
int measure_unit_rates(atlb_unit_rates*, void*, cudaStream_t);
int pair_fwd(const float*, const float*, const float*, const long long*, const long long*, const float*, const float*,
             const long long*, const long long*, const float*, long long, long long, long long, long long, long long,
             long long, double, double, double, float*, void*, cudaStream_t);
int pair_bwd(const float*, const float*, const float*, const float*, const long long*, const long long*, const float*,
             const float*, const long long*, const long long*, const float*, long long, long long, long long, long long,
             long long, long long, double, double, double, long long, float*, void*, cudaStream_t);
int flow_exact(int kind, const float* theta, long long B, long long H, long long W, const float* xy, const float* t,
               const float* t_dst, double t_dst_s, const long long* b, long long N, float* out, cudaStream_t s);
int flow_exact_bwd(int kind, const float* gy, const float* theta, long long B, long long H, long long W,
                   const float* xy, const float* t, const float* t_dst, double t_dst_s, const long long* b, long long N,
                   float* gtheta, float* gxy, cudaStream_t s);
int flow_rk4_steps_max();
int flow_rk4(const MotionView&, const float*, const float*, const float*, float, const long long*, long long, int,
             float*, cudaStream_t);
int flow_rk4_bwd(const MotionView&, const float*, const float*, const float*, const float*, float, const long long*,
                 long long, int, float*, cudaStream_t);
int rng_draw2(bool normal, unsigned long long seed, unsigned long long call, long long n, float* out,
              cudaStream_t s);
int pair_fwd_noalloc(const float*, const float*, const float*, const long long*, const long long*, const float*,
                     const float*, const long long*, const long long*, const float*, long long, long long, long long,
                     long long, long long, long long, double, double, double, float*, cudaStream_t);
size_t tile_ops_workspace_bytes(long long N, long long B, long long H, long long W);
int splat_bilinear_fwd(const float*, const float*, const long long*, long long, long long, long long, long long,
                       float*, void*, cudaStream_t);
int splat_bilinear_bwd(const float*, const float*, const float*, const long long*, long long, long long, long long,
                       long long, float*, float*, void*, cudaStream_t);
int blur(const float*, long long, long long, long long, double, float*, cudaStream_t);
int count_keys(const long long*, long long, long long, const float*, long long, long long*, cudaStream_t);
int sliced_score(long long, int, int, int, int, const float*, const float*, const float*, const float*, const float*,
                 double, double, double, long long, long long, float*, cudaStream_t);
int sliced_score_bwd(long long, int, int, int, int, const float*, const float*, const float*, const float*,
                     const float*, const float*, double, double, double, long long, long long, float*, float*,
                     cudaStream_t);
size_t splat_gauss_workspace_bytes(long long N, long long B, long long H, long long W);
int splat_gauss_fwd(const float*, const float*, const long long*, long long, long long, long long, long long, double,
                    long long, float*, void*, cudaStream_t);
int splat_gauss_bwd(const float*, const float*, const float*, const long long*, long long, long long, long long,
                    long long, double, long long, float*, float*, void*, cudaStream_t);
int splat_gauss_bwd_pos(const float*, const float*, long long, long long, long long, long long, double, long long,
                        float*, void*, cudaStream_t);
int gather_fwd(const float*, const float*, const long long*, long long, long long, long long, long long, float*, void*,
               cudaStream_t);
int gather_bwd(const float*, const float*, const float*, const long long*, long long, long long, long long, long long,
               float*, float*, void*, cudaStream_t);
int voxel_grid(const float*, const float*, const float*, const long long*, long long, long long, long long, long long,
               long long, float*, void*, cudaStream_t);
int velocity(const MotionView&, const float*, const long long*, long long, float*, cudaStream_t);
int velocity_bwd(const MotionView&, const float*, const float*, const long long*, long long, float*, cudaStream_t);
int visible_fraction(const MotionView&, const float*, const float*, const long long*, long long, const float*,
                     const long long*, long long, double, long long, float*, void*, cudaStream_t);
int window_counts(const float*, const long long*, long long, const long long*, long long, double, float*, void*,
                  cudaStream_t);
int window_counts_keys(const double*, long long, const float*, const long long*, const long long*, long long, double,
                       float*, cudaStream_t);

int traj_transport(const TrajView&, int, const float*, const float*, const float*, float, const long long*,
                   long long, float*, cudaStream_t);
int traj_transport_bwd(const TrajView&, int, const float*, const float*, const float*, const float*, float,
                       const long long*, long long, float*, float*, cudaStream_t);
int traj_records(const TrajView&, int, const float*, const float*, const float*, float, const long long*, long long,
                 float*, float*, cudaStream_t);
int traj_records_bwd(const TrajView&, int, const float*, const float*, const float*, const float*, float,
                     const long long*, long long, const float*, float*, cudaStream_t);
int traj_targets(const TrajView&, const float*, const float*, const long long*, long long, const float*, int, float*,
                 cudaStream_t);
int traj_targets_bwd(const TrajView&, const float*, const float*, const float*, const long long*, long long,
                     const float*, int, float*, cudaStream_t);
int traj_targets_max();
int traj_visible_fraction(const TrajView&, const float*, const float*, const long long*, long long, const float*,
                          const float*, int, float, float, float, float*, cudaStream_t);

size_t exact_workspace_bytes(const atlb_exact_cfg&, long long, long long, const atlb_plan_geom&);
int exact_prepare(const atlb_exact_cfg&, const float*, const float*, const float*, const long long*, long long,
                  const long long*, const float*, long long, float*, float*, long long*, void*, atlb_plan_geom*,
                  cudaStream_t);
int exact_forward(const atlb_exact_cfg&, const float*, const long long*, long long, long long, const float*,
                  const float*, const long long*, const atlb_plan_geom&, void*, float*, float*, float*, cudaStream_t);
int exact_backward(const atlb_exact_cfg&, const float*, const long long*, long long, long long, const float*,
                   const atlb_plan_geom&, void*, const float*, const float*, float*, float*, cudaStream_t);

}  // namespace atlb

using namespace atlb;

#define LL(p) reinterpret_cast<const long long*>(p)
#define LLW(p) reinterpret_cast<long long*>(p)
#define STREAM(s) reinterpret_cast<cudaStream_t>(s)

// A pointer may only be NULL when the array it stands for is empty.
#define NEED(ptr, n)                                                        \
  do {                                                                      \
    if ((n) > 0 && (ptr) == nullptr) {                                      \
      set_error("%s: %s is NULL for a non-empty array", __func__, #ptr);    \
      return ATLB_ERR_ARG;                                                  \
    }                                                                       \
  } while (0)
#define NONNEG(x)                                                           \
  do {                                                                      \
    if ((x) < 0) {                                                          \
      set_error("%s: %s = %lld is negative", __func__, #x, (long long)(x)); \
      return ATLB_ERR_ARG;                                                  \
    }                                                                       \
  } while (0)

static int clear() {
  g_err[0] = 0;
  return ATLB_OK;
}

static int check_kind(int kind, const char* fn) {
  if (kind != ATLB_MOTION_TRANSLATION && kind != ATLB_MOTION_AFFINE && kind != ATLB_MOTION_DENSE) {
    set_error("%s: unknown motion kind %d", fn, kind);
    return ATLB_ERR_ARG;
  }
  return ATLB_OK;
}

extern "C" {

const char* atlb_last_error(void) { return g_err; }
int atlb_abi_version(void) { return ATLB_ABI_VERSION; }

static int check_flow(int kind, const float* theta, int64_t B, int64_t H, int64_t W, int64_t N, const char* fn) {
  if (kind != ATLB_MOTION_TRANSLATION && kind != ATLB_MOTION_AFFINE) {
    set_error("%s: kind %d has no closed-form flow (translation or affine only)", fn, kind);
    return ATLB_ERR_ARG;
  }
  if (N < 0 || B < 1 || H < 1 || W < 1 || !theta) { set_error("%s: invalid sizes", fn); return ATLB_ERR_ARG; }
  return ATLB_OK;
}

int atlb_flow_exact(int kind, const float* theta, int64_t B, int64_t H, int64_t W, const float* xy, const float* t,
                    const float* t_dst, double t_dst_s, const int64_t* b, int64_t N, float* out, atlb_stream_t stream) {
  clear();
  if (int st = check_flow(kind, theta, B, H, W, N, __func__)) return st;
  NEED(xy, N); NEED(t, N); NEED(b, N); NEED(out, N);
  return flow_exact(kind, theta, B, H, W, xy, t, t_dst, t_dst_s, LL(b), N, out, STREAM(stream));
}

int atlb_flow_exact_bwd(int kind, const float* gy, const float* theta, int64_t B, int64_t H, int64_t W,
                        const float* xy, const float* t, const float* t_dst, double t_dst_s, const int64_t* b,
                        int64_t N, float* gtheta, float* gxy, atlb_stream_t stream) {
  clear();
  if (int st = check_flow(kind, theta, B, H, W, N, __func__)) return st;
  NEED(gy, N); NEED(xy, N); NEED(t, N); NEED(b, N);
  if (!gtheta) { set_error("%s: gtheta NULL", __func__); return ATLB_ERR_ARG; }
  return flow_exact_bwd(kind, gy, theta, B, H, W, xy, t, t_dst, t_dst_s, LL(b), N, gtheta, gxy, STREAM(stream));
}

int atlb_rng_uniform2(uint64_t seed, uint64_t call, int64_t n, float* out, atlb_stream_t stream) {
  clear();
  if (n < 0) { set_error("%s: negative size", __func__); return ATLB_ERR_ARG; }
  NEED(out, n);
  return rng_draw2(false, seed, call, n, out, STREAM(stream));
}

int atlb_rng_normal2(uint64_t seed, uint64_t call, int64_t n, float* out, atlb_stream_t stream) {
  clear();
  if (n < 0) { set_error("%s: negative size", __func__); return ATLB_ERR_ARG; }
  NEED(out, n);
  return rng_draw2(true, seed, call, n, out, STREAM(stream));
}
uint64_t atlb_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

size_t atlb_unit_rates_scratch_bytes(void) { return unit_rates_scratch_bytes(); }

int atlb_measure_unit_rates(atlb_unit_rates* out, void* scratch, size_t scratch_bytes, atlb_stream_t stream) {
  clear();
  if (!out) { set_error("atlb_measure_unit_rates: NULL out"); return ATLB_ERR_ARG; }
  if (!scratch || scratch_bytes < unit_rates_scratch_bytes()) {
    set_error("atlb_measure_unit_rates: scratch %zu < %zu bytes", scratch_bytes, unit_rates_scratch_bytes());
    return ATLB_ERR_WORKSPACE;
  }
  return measure_unit_rates(out, scratch, STREAM(stream));
}

size_t atlb_tile_ops_workspace_bytes(int64_t N, int64_t B, int64_t H, int64_t W) {
  return tile_ops_workspace_bytes(N < 0 ? 0 : N, B < 0 ? 0 : B, H < 0 ? 0 : H, W < 0 ? 0 : W);
}

// Sizes the tiled bilinear ops index with 32-bit integers, and their workspace.
static int check_tiles(int64_t N, int64_t B, int64_t H, int64_t W, void* ws, size_t ws_bytes, const char* fn) {
  if (N > (1LL << 31) - 1 || H > (1LL << 30) || W > (1LL << 30) || B * ((H + 31) / 32) * ((W + 31) / 32) > (1LL << 31) - 2) {
    set_error("%s: sizes exceed the int32 point / tile indices", fn);
    return ATLB_ERR_OVERFLOW;
  }
  if (!ws || ws_bytes < tile_ops_workspace_bytes(N, B, H, W)) {
    set_error("%s: workspace %zu < %zu bytes", fn, ws_bytes, tile_ops_workspace_bytes(N, B, H, W));
    return ATLB_ERR_WORKSPACE;
  }
  return ATLB_OK;
}

int atlb_splat_bilinear_fwd(const float* pos, const float* w, const int64_t* bidx, int64_t N, int64_t B, int64_t H,
                            int64_t W, float* img, void* workspace, size_t workspace_bytes, atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(B); NONNEG(H); NONNEG(W);
  NEED(pos, N); NEED(w, N); NEED(bidx, N); NEED(img, B * H * W);
  if (int st = check_tiles(N, B, H, W, workspace, workspace_bytes, __func__)) return st;
  return splat_bilinear_fwd(pos, w, LL(bidx), N, B, H, W, img, workspace, STREAM(stream));
}

int atlb_splat_bilinear_bwd(const float* gimg, const float* pos, const float* w, const int64_t* bidx, int64_t N,
                            int64_t B, int64_t H, int64_t W, float* gpos, float* gw, void* workspace,
                            size_t workspace_bytes, atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(B); NONNEG(H); NONNEG(W);
  NEED(gimg, B * H * W); NEED(pos, N); NEED(w, N); NEED(bidx, N); NEED(gpos, N); NEED(gw, N);
  if (int st = check_tiles(N, B, H, W, workspace, workspace_bytes, __func__)) return st;
  return splat_bilinear_bwd(gimg, pos, w, LL(bidx), N, B, H, W, gpos, gw, workspace, STREAM(stream));
}

int atlb_blur(const float* img, int64_t P, int64_t H, int64_t W, double sigma, float* out, atlb_stream_t stream) {
  clear();
  NONNEG(P); NONNEG(H); NONNEG(W);
  NEED(img, P * H * W); NEED(out, P * H * W);
  if (!(sigma > 0)) { set_error("%s: sigma must be positive", __func__); return ATLB_ERR_ARG; }
  if (img == out) { set_error("%s: out must not alias img", __func__); return ATLB_ERR_ARG; }
  return blur(img, P, H, W, sigma, out, STREAM(stream));
}

size_t atlb_splat_gauss_workspace_bytes(int64_t N, int64_t B, int64_t H, int64_t W) {
  return splat_gauss_workspace_bytes(N < 0 ? 0 : N, B < 0 ? 0 : B, H < 0 ? 0 : H, W < 0 ? 0 : W);
}

static int check_gauss(int64_t N, int64_t B, int64_t H, int64_t W, int64_t radius, void* ws, size_t ws_bytes,
                       const char* fn) {
  if (radius > ATLB_SPLAT_GAUSS_MAX_RADIUS) {
    set_error("%s: radius %lld above the tiled splat's limit of %d", fn, (long long)radius,
              ATLB_SPLAT_GAUSS_MAX_RADIUS);
    return ATLB_ERR_ARG;
  }
  if (N > (1LL << 31) - 1 || H > (1LL << 30) || W > (1LL << 30) || B * ((H + 31) / 32) * ((W + 31) / 32) > (1LL << 31) - 2) {
    set_error("%s: sizes exceed the int32 event / tile indices", fn);
    return ATLB_ERR_OVERFLOW;
  }
  if (!ws || ws_bytes < splat_gauss_workspace_bytes(N, B, H, W)) {
    set_error("%s: workspace %zu < %zu bytes", fn, ws_bytes, splat_gauss_workspace_bytes(N, B, H, W));
    return ATLB_ERR_WORKSPACE;
  }
  return ATLB_OK;
}

int atlb_splat_gauss_fwd(const float* pos, const float* w, const int64_t* bidx, int64_t N, int64_t B, int64_t H,
                         int64_t W, double sigma, int64_t radius, float* img, void* workspace, size_t workspace_bytes,
                         atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(B); NONNEG(H); NONNEG(W); NONNEG(radius);
  NEED(pos, N); NEED(w, N); NEED(bidx, N); NEED(img, B * H * W);
  if (int st = check_gauss(N, B, H, W, radius, workspace, workspace_bytes, __func__)) return st;
  return splat_gauss_fwd(pos, w, LL(bidx), N, B, H, W, sigma, radius, img, workspace, STREAM(stream));
}

int atlb_splat_gauss_bwd(const float* gimg, const float* pos, const float* w, const int64_t* bidx, int64_t N,
                         int64_t B, int64_t H, int64_t W, double sigma, int64_t radius, float* gpos, float* gw,
                         void* workspace, size_t workspace_bytes, atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(B); NONNEG(H); NONNEG(W); NONNEG(radius);
  NEED(gimg, B * H * W); NEED(pos, N); NEED(w, N); NEED(bidx, N); NEED(gpos, N); NEED(gw, N);
  if (int st = check_gauss(N, B, H, W, radius, workspace, workspace_bytes, __func__)) return st;
  return splat_gauss_bwd(gimg, pos, w, LL(bidx), N, B, H, W, sigma, radius, gpos, gw, workspace, STREAM(stream));
}

int atlb_splat_gauss_bwd_pos(const float* gimg, const float* w, int64_t N, int64_t B, int64_t H, int64_t W,
                             double sigma, int64_t R, float* gpos, void* workspace, size_t workspace_bytes,
                             atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(B); NONNEG(H); NONNEG(W); NONNEG(R);
  NEED(gimg, B * H * W); NEED(w, N); NEED(gpos, N);
  if (int st = check_gauss(N, B, H, W, R, workspace, workspace_bytes, __func__)) return st;
  return splat_gauss_bwd_pos(gimg, w, N, B, H, W, sigma, R, gpos, workspace, STREAM(stream));
}

int atlb_gather_bilinear_fwd(const float* img, const float* pos, const int64_t* bidx, int64_t N, int64_t B, int64_t H,
                             int64_t W, float* out, void* workspace, size_t workspace_bytes, atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(B); NONNEG(H); NONNEG(W);
  NEED(img, B * H * W); NEED(pos, N); NEED(bidx, N); NEED(out, N);
  if (int st = check_tiles(N, B, H, W, workspace, workspace_bytes, __func__)) return st;
  return gather_fwd(img, pos, LL(bidx), N, B, H, W, out, workspace, STREAM(stream));
}

int atlb_gather_bilinear_bwd(const float* gval, const float* img, const float* pos, const int64_t* bidx, int64_t N,
                             int64_t B, int64_t H, int64_t W, float* gimg, float* gpos, void* workspace,
                             size_t workspace_bytes, atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(B); NONNEG(H); NONNEG(W);
  NEED(gval, N); NEED(img, B * H * W); NEED(pos, N); NEED(bidx, N); NEED(gimg, B * H * W); NEED(gpos, N);
  if (int st = check_tiles(N, B, H, W, workspace, workspace_bytes, __func__)) return st;
  return gather_bwd(gval, img, pos, LL(bidx), N, B, H, W, gimg, gpos, workspace, STREAM(stream));
}

int atlb_voxel_grid(const float* pos, const float* t, const float* p, const int64_t* bidx, int64_t N, int64_t B,
                    int64_t C, int64_t H, int64_t W, float* vox, void* workspace, size_t workspace_bytes,
                    atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(B); NONNEG(C); NONNEG(H); NONNEG(W);
  NEED(pos, N); NEED(t, N); NEED(p, N); NEED(bidx, N); NEED(vox, B * C * H * W);
  if (int st = check_tiles(N, B, H, W, workspace, workspace_bytes, __func__)) return st;
  return voxel_grid(pos, t, p, LL(bidx), N, B, C, H, W, vox, workspace, STREAM(stream));
}

int atlb_plan_geometry(const float* x, const float* v, int64_t N, const int64_t* anchors, const float* anchor_xy,
                       int64_t M, int64_t H, int64_t W, double h, double cut, int64_t S, void* scratch,
                       atlb_plan_geom* geom_out, atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(M); NONNEG(H); NONNEG(W);
  NEED(x, N); NEED(v, N); NEED(anchors, M);
  if (S < 1 || S > (1 << 20)) { set_error("atlb_plan_geometry: n_slices = %lld", (long long)S); return ATLB_ERR_ARG; }
  if (!scratch || !geom_out) { set_error("atlb_plan_geometry: scratch / geom_out is NULL"); return ATLB_ERR_ARG; }
  const int st = plan_geometry(x, v, N, LL(anchors), anchor_xy, M, H, W, h, cut, S, scratch, geom_out, STREAM(stream));
  if (st) return st;
  if (!(geom_out->cell > 0) || geom_out->GW <= 0 || geom_out->GH <= 0 || geom_out->GW > (1LL << 31) ||
      geom_out->GH > (1LL << 31)) {
    set_error("atlb_plan_geometry: degenerate grid (cell %g, %lld x %lld cells); non-finite inputs?", geom_out->cell,
              (long long)geom_out->GW, (long long)geom_out->GH);
    return ATLB_ERR_OVERFLOW;
  }
  return ATLB_OK;
}

size_t atlb_plan_workspace_bytes(int64_t ncell) { return plan_workspace_bytes(ncell < 0 ? 0 : ncell); }

static int check_geom(const atlb_plan_geom* g, int64_t B, const char* fn) {
  if (!g || g->S < 1 || g->GW <= 0 || g->GH <= 0) { set_error("%s: invalid geometry", fn); return ATLB_ERR_ARG; }
  const double ncell = (double)B * g->S * (double)g->GH * (double)g->GW;
  if (ncell > 2.0e9) {
    set_error("%s: %.3g cells exceed the int32 cursor range", fn, ncell);
    return ATLB_ERR_OVERFLOW;
  }
  return ATLB_OK;
}

int atlb_plan_count(const float* x, const float* t, const float* v, const int64_t* b, int64_t N, int64_t B, double tau,
                    const atlb_plan_geom* geom, int64_t* cell_start, void* workspace, size_t workspace_bytes,
                    int64_t* n_entries_out, atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(B);
  NEED(x, N); NEED(t, N); NEED(v, N); NEED(b, N);
  if (int st = check_geom(geom, B, __func__)) return st;
  const long long ncell = B * (long long)geom->S * geom->GH * geom->GW;
  if (!cell_start || !n_entries_out) { set_error("atlb_plan_count: NULL output"); return ATLB_ERR_ARG; }
  if (!workspace || workspace_bytes < plan_workspace_bytes(ncell)) {
    set_error("atlb_plan_count: workspace %zu < %zu bytes", workspace_bytes, plan_workspace_bytes(ncell));
    return ATLB_ERR_WORKSPACE;
  }
  return plan_count(x, t, v, LL(b), N, B, tau, geom, LLW(cell_start), workspace, LLW(n_entries_out), STREAM(stream));
}

int atlb_plan_fill(const float* x, const float* t, const float* v, const int64_t* b, int64_t N, int64_t B, double tau,
                   const atlb_plan_geom* geom, const int64_t* anchors, const float* anchor_xy, int64_t M,
                   const int64_t* cell_start, void* workspace, size_t workspace_bytes, float* src_y, float* src_v,
                   float* src_t, int64_t* src_id, float* anc_x, float* anc_t, int64_t* anc_cell, int64_t* anc_id,
                   float* slice_c, atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(B); NONNEG(M);
  NEED(x, N); NEED(t, N); NEED(v, N); NEED(b, N); NEED(anchors, M);
  NEED(anc_x, M); NEED(anc_t, M); NEED(anc_cell, M); NEED(anc_id, M);
  if (int st = check_geom(geom, B, __func__)) return st;
  const long long ncell = B * (long long)geom->S * geom->GH * geom->GW;
  if (!cell_start || !slice_c) { set_error("atlb_plan_fill: NULL cell_start / slice_c"); return ATLB_ERR_ARG; }
  if (N > 0 && (!src_y || !src_v || !src_t || !src_id)) { set_error("atlb_plan_fill: NULL entry array"); return ATLB_ERR_ARG; }
  if (!workspace || workspace_bytes < plan_workspace_bytes(ncell)) {
    set_error("atlb_plan_fill: workspace %zu < %zu bytes", workspace_bytes, plan_workspace_bytes(ncell));
    return ATLB_ERR_WORKSPACE;
  }
  return plan_fill(x, t, v, LL(b), N, B, tau, geom, LL(anchors), anchor_xy, M, LL(cell_start), workspace, src_y,
                   src_v, src_t, LLW(src_id), anc_x, anc_t, LLW(anc_cell), LLW(anc_id), slice_c, STREAM(stream));
}

size_t atlb_pair_workspace_bytes(int64_t M, int64_t ncell) {
  return pair_workspace_bytes(M < 0 ? 0 : M, ncell < 0 ? 0 : ncell);
}

static int check_pair(const int64_t* cell_start, const float* slice_c, int64_t Ns, int64_t M, int64_t ncell, int64_t S,
                      int64_t GH, int64_t GW, void* ws, size_t ws_bytes, const char* fn) {
  if (Ns < 0 || M < 0 || ncell < 0 || S < 1 || GH < 0 || GW < 0) { set_error("%s: negative size", fn); return ATLB_ERR_ARG; }
  if (!cell_start || !slice_c) { set_error("%s: NULL cell_start / slice_c", fn); return ATLB_ERR_ARG; }
  if (M > (1LL << 31) - 1 || ncell > (1LL << 31) - 2) { set_error("%s: too many anchors / cells", fn); return ATLB_ERR_OVERFLOW; }
  if (!ws || ws_bytes < pair_workspace_bytes(M, ncell)) {
    set_error("%s: workspace %zu < %zu bytes", fn, ws_bytes, pair_workspace_bytes(M, ncell));
    return ATLB_ERR_WORKSPACE;
  }
  return ATLB_OK;
}

int atlb_ats_pair_fwd(const float* src_y, const float* src_v, const float* src_t, const int64_t* src_id,
                      const int64_t* cell_start, const float* anc_x, const float* anc_t, const int64_t* anc_cell,
                      const int64_t* anc_id, const float* slice_c, int64_t Ns, int64_t M, int64_t ncell, int64_t S,
                      int64_t GH, int64_t GW, double h, double tau, double cut, float* out, void* workspace,
                      size_t workspace_bytes, atlb_stream_t stream) {
  clear();
  if (int st = check_pair(cell_start, slice_c, Ns, M, ncell, S, GH, GW, workspace, workspace_bytes, __func__)) return st;
  NEED(src_y, Ns); NEED(src_v, Ns); NEED(src_t, Ns); NEED(src_id, Ns);
  NEED(anc_x, M); NEED(anc_t, M); NEED(anc_cell, M); NEED(anc_id, M); NEED(out, M);
  return pair_fwd(src_y, src_v, src_t, LL(src_id), LL(cell_start), anc_x, anc_t, LL(anc_cell), LL(anc_id), slice_c, Ns,
                  M, ncell, S, GH, GW, h, tau, cut, out, workspace, STREAM(stream));
}

int atlb_ats_pair_fwd_noalloc(const float* src_y, const float* src_v, const float* src_t, const int64_t* src_id,
                              const int64_t* cell_start, const float* anc_x, const float* anc_t,
                              const int64_t* anc_cell, const int64_t* anc_id, const float* slice_c, int64_t Ns,
                              int64_t M, int64_t ncell, int64_t S, int64_t GH, int64_t GW, double h, double tau,
                              double cut, float* out, atlb_stream_t stream) {
  clear();
  if (Ns < 0 || M < 0 || ncell < 0 || S < 1 || GH < 0 || GW < 0) { set_error("%s: negative size", __func__); return ATLB_ERR_ARG; }
  if (!cell_start || !slice_c) { set_error("%s: NULL cell_start / slice_c", __func__); return ATLB_ERR_ARG; }
  if (M > (1LL << 31) - 1 || ncell > (1LL << 31) - 2) { set_error("%s: too many anchors / cells", __func__); return ATLB_ERR_OVERFLOW; }
  NEED(src_y, Ns); NEED(src_v, Ns); NEED(src_t, Ns); NEED(src_id, Ns);
  NEED(anc_x, M); NEED(anc_t, M); NEED(anc_cell, M); NEED(anc_id, M); NEED(out, M);
  return pair_fwd_noalloc(src_y, src_v, src_t, LL(src_id), LL(cell_start), anc_x, anc_t, LL(anc_cell), LL(anc_id),
                          slice_c, Ns, M, ncell, S, GH, GW, h, tau, cut, out, STREAM(stream));
}

int atlb_ats_pair_bwd(const float* gS, const float* src_y, const float* src_v, const float* src_t,
                      const int64_t* src_id, const int64_t* cell_start, const float* anc_x, const float* anc_t,
                      const int64_t* anc_cell, const int64_t* anc_id, const float* slice_c, int64_t Ns, int64_t M,
                      int64_t ncell, int64_t S, int64_t GH, int64_t GW, double h, double tau, double cut, int64_t N,
                      float* gv, void* workspace, size_t workspace_bytes, atlb_stream_t stream) {
  clear();
  if (int st = check_pair(cell_start, slice_c, Ns, M, ncell, S, GH, GW, workspace, workspace_bytes, __func__)) return st;
  NONNEG(N);
  NEED(gS, M); NEED(src_y, Ns); NEED(src_v, Ns); NEED(src_t, Ns); NEED(src_id, Ns);
  NEED(anc_x, M); NEED(anc_t, M); NEED(anc_cell, M); NEED(anc_id, M); NEED(gv, N);
  return pair_bwd(gS, src_y, src_v, src_t, LL(src_id), LL(cell_start), anc_x, anc_t, LL(anc_cell), LL(anc_id), slice_c,
                  Ns, M, ncell, S, GH, GW, h, tau, cut, N, gv, workspace, STREAM(stream));
}

int atlb_window_counts(const float* t, const int64_t* b, int64_t N, const int64_t* idx, int64_t M, double tau,
                       float* out, void* scratch, atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(M);
  NEED(t, N); NEED(b, N); NEED(idx, M); NEED(out, M);
  if (!scratch) { set_error("atlb_window_counts: scratch is NULL"); return ATLB_ERR_ARG; }
  return window_counts(t, LL(b), N, LL(idx), M, tau, out, scratch, STREAM(stream));
}

int atlb_window_counts_keys(const double* sorted_keys, int64_t N, const float* t, const int64_t* b,
                            const int64_t* idx, int64_t M, double tau, float* out, atlb_stream_t stream) {
  clear();
  NONNEG(N); NONNEG(M);
  NEED(sorted_keys, N); NEED(t, N); NEED(b, N); NEED(idx, M); NEED(out, M);
  return window_counts_keys(sorted_keys, N, t, LL(b), LL(idx), M, tau, out, STREAM(stream));
}

int atlb_velocity(int kind, const float* theta, int64_t B, int64_t Hg, int64_t Wg, int64_t H, int64_t W,
                  const float* xy, const int64_t* b, int64_t N, float* v, atlb_stream_t stream) {
  clear();
  if (int st = check_kind(kind, __func__)) return st;
  NONNEG(B); NONNEG(N);
  if (kind == ATLB_MOTION_DENSE && (Hg < 1 || Wg < 1)) { set_error("atlb_velocity: empty grid"); return ATLB_ERR_ARG; }
  NEED(theta, B); NEED(xy, N); NEED(b, N); NEED(v, N);
  return velocity(make_motion_view(kind, theta, B, Hg, Wg, H, W), xy, LL(b), N, v, STREAM(stream));
}

int atlb_velocity_bwd(int kind, const float* gv, int64_t B, int64_t Hg, int64_t Wg, int64_t H, int64_t W,
                      const float* xy, const int64_t* b, int64_t N, float* gtheta, atlb_stream_t stream) {
  clear();
  if (int st = check_kind(kind, __func__)) return st;
  NONNEG(B); NONNEG(N);
  if (kind == ATLB_MOTION_DENSE && (Hg < 1 || Wg < 1)) { set_error("atlb_velocity_bwd: empty grid"); return ATLB_ERR_ARG; }
  NEED(gv, N); NEED(xy, N); NEED(b, N); NEED(gtheta, B);
  return velocity_bwd(make_motion_view(kind, nullptr, B, Hg, Wg, H, W), gv, xy, LL(b), N, gtheta, STREAM(stream));
}

int atlb_visible_fraction(int kind, const float* theta, int64_t B, int64_t Hg, int64_t Wg, int64_t H, int64_t W,
                          const float* xa, const float* ta, const int64_t* ba, int64_t M, const float* t,
                          const int64_t* b, int64_t N, double tau, int64_t n_check, float* out, void* scratch,
                          atlb_stream_t stream) {
  clear();
  if (int st = check_kind(kind, __func__)) return st;
  NONNEG(B); NONNEG(M); NONNEG(N);
  if (n_check < 1 || n_check > 4096) { set_error("atlb_visible_fraction: n_check = %lld", (long long)n_check); return ATLB_ERR_ARG; }
  NEED(theta, B); NEED(xa, M); NEED(ta, M); NEED(ba, M); NEED(t, N); NEED(b, N); NEED(out, M);
  if (!scratch) { set_error("atlb_visible_fraction: scratch is NULL"); return ATLB_ERR_ARG; }
  return visible_fraction(make_motion_view(kind, theta, B, Hg, Wg, H, W), xa, ta, LL(ba), M, t, LL(b), N, tau, n_check,
                          out, scratch, STREAM(stream));
}

static int check_exact_cfg(const atlb_exact_cfg* c, const char* fn) {
  if (!c) { set_error("%s: cfg is NULL", fn); return ATLB_ERR_ARG; }
  if (int st = check_kind(c->kind, fn)) return st;
  if (!c->theta || c->Bt < 1 || c->B < 1 || c->H < 1 || c->W < 1 || c->S < 1 || c->S > 65535 || c->n_check < 1 ||
      c->n_check > 4096 || (c->kind == ATLB_MOTION_DENSE && (c->Hg < 1 || c->Wg < 1))) {
    set_error("%s: invalid configuration", fn);
    return ATLB_ERR_ARG;
  }
  return ATLB_OK;
}

static int check_exact_sizes(const atlb_exact_cfg* c, int64_t N, int64_t M, const atlb_plan_geom* g, const char* fn) {
  if (N < 0 || M < 0) { set_error("%s: negative size", fn); return ATLB_ERR_ARG; }
  if (N * c->S > (1LL << 31) - 1 || M > (1LL << 31) - 1) {
    set_error("%s: N * n_slices = %lld entries exceed the int32 plan index", fn, (long long)(N * c->S));
    return ATLB_ERR_OVERFLOW;
  }
  if (c->src_end > 0 && (c->src_begin < 0 || c->src_begin > c->src_end || c->src_end > N)) {
    set_error("%s: source range [%lld, %lld) outside [0, %lld]", fn, (long long)c->src_begin, (long long)c->src_end,
              (long long)N);
    return ATLB_ERR_ARG;
  }
  // the fused plan indexes its sub-cells (kFine x kFine per plan cell) with 32-bit integers
  if (g && (g->S != c->S || g->GW < 1 || g->GH < 1 || (double)c->B * g->S * (double)g->GH * g->GW * 9.0 > 2.0e9)) {
    set_error("%s: invalid geometry", fn);
    return ATLB_ERR_OVERFLOW;
  }
  return ATLB_OK;
}

int atlb_exact_prepare(const atlb_exact_cfg* cfg, const float* xy, const float* u, const float* t, const int64_t* b,
                       int64_t N, const int64_t* anchors, const float* z, int64_t M, float* ev4, float* anc4,
                       int64_t* anc_b, void* scratch, atlb_plan_geom* geom_out, atlb_stream_t stream) {
  clear();
  if (int st = check_exact_cfg(cfg, __func__)) return st;
  if (int st = check_exact_sizes(cfg, N, M, nullptr, __func__)) return st;
  NEED(xy, N); NEED(t, N); NEED(b, N); NEED(ev4, N); NEED(anc4, M); NEED(anc_b, M);
  if (!anchors && M != N) { set_error("atlb_exact_prepare: anchors NULL needs M == N"); return ATLB_ERR_ARG; }
  if (!scratch || !geom_out) { set_error("atlb_exact_prepare: scratch / geom_out NULL"); return ATLB_ERR_ARG; }
  const int st = exact_prepare(*cfg, xy, u, t, LL(b), N, LL(anchors), z, M, ev4, anc4, LLW(anc_b), scratch, geom_out,
                               STREAM(stream));
  if (st) return st;
  return check_exact_sizes(cfg, N, M, geom_out, __func__);
}

size_t atlb_exact_workspace_bytes(const atlb_exact_cfg* cfg, int64_t N, int64_t M, const atlb_plan_geom* geom) {
  if (!cfg || !geom || N < 0 || M < 0) return 0;
  return exact_workspace_bytes(*cfg, N, M, *geom);
}

int atlb_exact_forward(const atlb_exact_cfg* cfg, const float* t, const int64_t* b, int64_t N, int64_t M,
                       const float* ev4, const float* anc4, const int64_t* anc_b, const atlb_plan_geom* geom,
                       void* workspace, size_t workspace_bytes, float* S_out, float* den_out, float* ls_out,
                       atlb_stream_t stream) {
  clear();
  if (int st = check_exact_cfg(cfg, __func__)) return st;
  if (!geom) { set_error("atlb_exact_forward: geom NULL"); return ATLB_ERR_ARG; }
  if (int st = check_exact_sizes(cfg, N, M, geom, __func__)) return st;
  NEED(t, N); NEED(b, N); NEED(ev4, N); NEED(anc4, M); NEED(anc_b, M); NEED(S_out, M); NEED(den_out, M);
  NEED(ls_out, M);
  if (!workspace || workspace_bytes < exact_workspace_bytes(*cfg, N, M, *geom)) {
    set_error("atlb_exact_forward: workspace too small");
    return ATLB_ERR_WORKSPACE;
  }
  return exact_forward(*cfg, t, LL(b), N, M, ev4, anc4, LL(anc_b), *geom, workspace, S_out, den_out, ls_out,
                       STREAM(stream));
}

int atlb_exact_prepare_forward(const atlb_exact_cfg* cfg, const float* xy, const float* u, const float* t,
                               const int64_t* b, int64_t N, const int64_t* anchors, const float* z, int64_t M,
                               float* ev4, float* anc4, int64_t* anc_b, void* scratch, atlb_plan_geom* geom_out,
                               void* workspace, size_t workspace_bytes, float* S_out, float* den_out, float* ls_out,
                               atlb_stream_t stream) {
  if (int st = atlb_exact_prepare(cfg, xy, u, t, b, N, anchors, z, M, ev4, anc4, anc_b, scratch, geom_out, stream))
    return st;
  // the forward's kernels are launched right after the geometry read-back, with no return to the caller between
  if (!workspace || workspace_bytes < exact_workspace_bytes(*cfg, N, M, *geom_out)) {
    set_error("atlb_exact_prepare_forward: workspace too small for this window's plan (prepared; size it with "
              "atlb_exact_workspace_bytes and call atlb_exact_forward)");
    return ATLB_ERR_WORKSPACE;
  }
  return atlb_exact_forward(cfg, t, b, N, M, ev4, anc4, anc_b, geom_out, workspace, workspace_bytes, S_out, den_out,
                            ls_out, stream);
}

int atlb_exact_backward(const atlb_exact_cfg* cfg, const float* grad_ls, const int64_t* b, int64_t N, int64_t M,
                        const float* ev4, const atlb_plan_geom* geom, void* workspace, size_t workspace_bytes,
                        const float* S, const float* den, float* gv, float* gtheta, atlb_stream_t stream) {
  clear();
  if (int st = check_exact_cfg(cfg, __func__)) return st;
  if (!geom) { set_error("atlb_exact_backward: geom NULL"); return ATLB_ERR_ARG; }
  if (int st = check_exact_sizes(cfg, N, M, geom, __func__)) return st;
  NEED(grad_ls, M); NEED(b, N); NEED(ev4, N); NEED(S, M); NEED(den, M); NEED(gv, N);
  if (!gtheta) { set_error("atlb_exact_backward: gtheta NULL"); return ATLB_ERR_ARG; }
  if (!workspace || workspace_bytes < exact_workspace_bytes(*cfg, N, M, *geom)) {
    set_error("atlb_exact_backward: workspace too small");
    return ATLB_ERR_WORKSPACE;
  }
  return exact_backward(*cfg, grad_ls, LL(b), N, M, ev4, *geom, workspace, S, den, gv, gtheta, STREAM(stream));
}

}  // extern "C"

static int make_traj(const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K, int basis, const float* bc,
                     double offset, double tile, int64_t n_fp, TrajView* V, const char* fn) {
  if (!coeff || B < 1 || Hq < 1 || Wq < 1 || K < 1 || K > kTrajKMax || n_fp < 0 || n_fp > kTrajKMax ||
      !(tile > 0) || (basis != 0 && basis != 1) || (basis == 1 && !bc) || B * Hq * Wq * 2 * K >= (1LL << 31)) {
    set_error("%s: invalid trajectory grid (B %lld, %lld x %lld, K %lld, basis %d, n_fp %lld, tile %g)", fn,
              (long long)B, (long long)Hq, (long long)Wq, (long long)K, basis, (long long)n_fp, tile);
    return ATLB_ERR_ARG;
  }
  V->C = coeff;
  V->B = (int)B;
  V->Hq = (int)Hq;
  V->Wq = (int)Wq;
  V->K = (int)K;
  V->n_fp = (int)n_fp;
  V->basis = basis;
  V->offset = (float)offset;
  V->tile = (float)tile;
  volatile float one = 1.f;  // an fp32 division on the host: RN(1 / tile), the device's 1.f / tile
  V->rtile = one / V->tile;
  int e2 = 0;
  V->tile_pow2 = std::frexp(V->tile, &e2) == 0.5f ? 1 : 0;
  for (int k = 0; k < kTrajKMax; ++k) V->bc[k] = (basis == 1 && k < K) ? bc[k] : 0.f;
  return ATLB_OK;
}

int atlb_traj_transport(int mode, const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K, int basis,
                        const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xy,
                        const float* t, const float* t_dst, double t_dst_s, const int64_t* b, int64_t N, float* out,
                        atlb_stream_t stream) {
  clear();
  NONNEG(N);
  NEED(xy, N); NEED(t, N); NEED(b, N); NEED(out, N);
  if (mode < 0 || mode > 3) { set_error("%s: mode %d", __func__, mode); return ATLB_ERR_ARG; }
  TrajView V;
  if (int st = make_traj(coeff, B, Hq, Wq, K, basis, bezier_c, offset, tile, n_fp, &V, __func__)) return st;
  return traj_transport(V, mode, xy, t, t_dst, (float)t_dst_s, LL(b), N, out, STREAM(stream));
}

int atlb_traj_transport_bwd(int mode, const float* gy, const float* coeff, int64_t B, int64_t Hq, int64_t Wq,
                            int64_t K, int basis, const float* bezier_c, double offset, double tile, int64_t n_fp,
                            const float* xy, const float* t, const float* t_dst, double t_dst_s, const int64_t* b,
                            int64_t N, float* gcoeff, float* gp, atlb_stream_t stream) {
  clear();
  NONNEG(N);
  NEED(gy, N); NEED(xy, N); NEED(t, N); NEED(b, N);
  if (mode < 0 || mode > 3) { set_error("%s: mode %d", __func__, mode); return ATLB_ERR_ARG; }
  if (mode == 2) NEED(gp, N);
  if (!gcoeff) { set_error("%s: gcoeff is NULL", __func__); return ATLB_ERR_ARG; }
  TrajView V;
  if (int st = make_traj(coeff, B, Hq, Wq, K, basis, bezier_c, offset, tile, n_fp, &V, __func__)) return st;
  return traj_transport_bwd(V, mode, gy, xy, t, t_dst, (float)t_dst_s, LL(b), N, gcoeff, gp, STREAM(stream));
}

int atlb_traj_visible_fraction(const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K, int basis,
                               const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xa,
                               const float* ta, const int64_t* ba, int64_t M, const float* counts,
                               const float* centres, int64_t n_check, double tau, int64_t H, int64_t W, float* out,
                               atlb_stream_t stream) {
  clear();
  NONNEG(M); NONNEG(H); NONNEG(W);
  NEED(xa, M); NEED(ta, M); NEED(ba, M); NEED(out, M);
  if (n_check < 1 || n_check > 4096 || !counts || !centres) {
    set_error("%s: n_check = %lld, counts / centres %s", __func__, (long long)n_check,
              (!counts || !centres) ? "NULL" : "set");
    return ATLB_ERR_ARG;
  }
  TrajView V;
  if (int st = make_traj(coeff, B, Hq, Wq, K, basis, bezier_c, offset, tile, n_fp, &V, __func__)) return st;
  return traj_visible_fraction(V, xa, ta, LL(ba), M, counts, centres, (int)n_check, (float)tau, (float)(W - 1),
                               (float)(H - 1), out, STREAM(stream));
}

static int check_score(int64_t N, int P, int ia, int io, int ip, double sigma, double delta, int64_t H, int64_t W,
                       const char* fn) {
  const bool slot_ok = P >= 1 && P <= 16 && ia >= 0 && ia < P && io < P && (ip < 0 || ip + 4 <= P);
  if (!slot_ok || !(sigma > 0) || !(delta > 0) || H < 1 || W < 1 || N > (1LL << 40)) {
    set_error("%s: P %d, slots a %d own %d probes %d, sigma %g, delta %g, image %lld x %lld", fn, P, ia, io, ip,
              sigma, delta, (long long)W, (long long)H);
    return ATLB_ERR_ARG;
  }
  return ATLB_OK;
}

int atlb_sliced_score(int64_t N, int P, int ia, int io, int ip, const float* pos, const float* val, const float* cnt,
                      const float* vis, const float* src, double sigma, double delta, double eps, int64_t H,
                      int64_t W, float* ls, atlb_stream_t stream) {
  clear();
  NONNEG(N);
  if (int st = check_score(N, P, ia, io, ip, sigma, delta, H, W, __func__)) return st;
  NEED(pos, N); NEED(val, N); NEED(cnt, N); NEED(src, N); NEED(ls, N);
  return sliced_score(N, P, ia, io, ip, pos, val, cnt, vis, src, sigma, delta, eps, H, W, ls, STREAM(stream));
}

int atlb_sliced_score_bwd(int64_t N, int P, int ia, int io, int ip, const float* gls, const float* pos,
                          const float* val, const float* cnt, const float* vis, const float* src, double sigma,
                          double delta, double eps, int64_t H, int64_t W, float* gval, float* gpos,
                          atlb_stream_t stream) {
  clear();
  NONNEG(N);
  if (int st = check_score(N, P, ia, io, ip, sigma, delta, H, W, __func__)) return st;
  NEED(gls, N); NEED(pos, N); NEED(val, N); NEED(cnt, N); NEED(src, N); NEED(gval, N); NEED(gpos, N);
  return sliced_score_bwd(N, P, ia, io, ip, gls, pos, val, cnt, vis, src, sigma, delta, eps, H, W, gval, gpos,
                          STREAM(stream));
}

int atlb_traj_records(const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K, int basis,
                      const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xy, int64_t R,
                      const float* t, const float* t_dst, double t_dst_s, const int64_t* b, int64_t N, float* out,
                      float* iterates, atlb_stream_t stream) {
  clear();
  NONNEG(N);
  if (R < 1 || R > 64) { set_error("%s: R = %lld records per event", __func__, (long long)R); return ATLB_ERR_ARG; }
  NEED(xy, N * R); NEED(t, N); NEED(b, N); NEED(out, N * R);
  TrajView V;
  if (int st = make_traj(coeff, B, Hq, Wq, K, basis, bezier_c, offset, tile, n_fp, &V, __func__)) return st;
  return traj_records(V, (int)R, xy, t, t_dst, (float)t_dst_s, LL(b), N, out, iterates, STREAM(stream));
}

int atlb_traj_records_bwd(const float* gy, const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K,
                          int basis, const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xy,
                          int64_t R, const float* t, const float* t_dst, double t_dst_s, const int64_t* b, int64_t N,
                          const float* iterates, float* gcoeff, atlb_stream_t stream) {
  clear();
  NONNEG(N);
  if (R < 1 || R > 64) { set_error("%s: R = %lld records per event", __func__, (long long)R); return ATLB_ERR_ARG; }
  NEED(gy, N * R); NEED(xy, N * R); NEED(t, N); NEED(b, N);
  if (!gcoeff) { set_error("%s: gcoeff is NULL", __func__); return ATLB_ERR_ARG; }
  TrajView V;
  if (int st = make_traj(coeff, B, Hq, Wq, K, basis, bezier_c, offset, tile, n_fp, &V, __func__)) return st;
  return traj_records_bwd(V, (int)R, gy, xy, t, t_dst, (float)t_dst_s, LL(b), N, iterates, gcoeff, STREAM(stream));
}

int atlb_traj_targets(const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K, int basis,
                      const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xy, const float* t,
                      const int64_t* b, int64_t N, const float* targets, int64_t T, float* out, atlb_stream_t stream) {
  clear();
  NONNEG(N);
  if (T < 1 || T > traj_targets_max() || !targets) {
    set_error("%s: T = %lld targets (1..%d), targets %s", __func__, (long long)T, traj_targets_max(),
              targets ? "set" : "NULL");
    return ATLB_ERR_ARG;
  }
  NEED(xy, N); NEED(t, N); NEED(b, N); NEED(out, N * T);
  TrajView V;
  if (int st = make_traj(coeff, B, Hq, Wq, K, basis, bezier_c, offset, tile, n_fp, &V, __func__)) return st;
  return traj_targets(V, xy, t, LL(b), N, targets, (int)T, out, STREAM(stream));
}

int atlb_traj_targets_bwd(const float* gy, const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K,
                          int basis, const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xy,
                          const float* t, const int64_t* b, int64_t N, const float* targets, int64_t T, float* gcoeff,
                          atlb_stream_t stream) {
  clear();
  NONNEG(N);
  if (T < 1 || T > traj_targets_max() || !targets) {
    set_error("%s: T = %lld targets (1..%d), targets %s", __func__, (long long)T, traj_targets_max(),
              targets ? "set" : "NULL");
    return ATLB_ERR_ARG;
  }
  NEED(gy, N * T); NEED(xy, N); NEED(t, N); NEED(b, N);
  if (!gcoeff) { set_error("%s: gcoeff is NULL", __func__); return ATLB_ERR_ARG; }
  TrajView V;
  if (int st = make_traj(coeff, B, Hq, Wq, K, basis, bezier_c, offset, tile, n_fp, &V, __func__)) return st;
  return traj_targets_bwd(V, gy, xy, t, LL(b), N, targets, (int)T, gcoeff, STREAM(stream));
}

int atlb_count_keys(const int64_t* key, int64_t N, int64_t nbins, const float* mask, int64_t R, int64_t* out,
                    atlb_stream_t stream) {
  clear();
  NONNEG(N);
  if (nbins < 1 || R < 1 || nbins * R > (1LL << 24)) {
    set_error("%s: nbins %lld x R %lld", __func__, (long long)nbins, (long long)R);
    return ATLB_ERR_ARG;
  }
  NEED(key, N); NEED(out, nbins * R);
  return count_keys(LL(key), N, nbins, mask, R, LLW(out), STREAM(stream));
}

static int check_rk4(int64_t B, int64_t Hg, int64_t Wg, int64_t H, int64_t W, int steps, const char* fn) {
  if (B < 1 || Hg < 1 || Wg < 1 || H < 1 || W < 1 || steps < 1 || steps > flow_rk4_steps_max()) {
    set_error("%s: grid %lld x %lld x %lld, image %lld x %lld, steps %d (1..%d)", fn, (long long)B, (long long)Hg,
              (long long)Wg, (long long)H, (long long)W, steps, flow_rk4_steps_max());
    return ATLB_ERR_ARG;
  }
  return ATLB_OK;
}

int atlb_flow_rk4(const float* theta, int64_t B, int64_t Hg, int64_t Wg, int64_t H, int64_t W, const float* xy,
                  const float* t, const float* t_dst, double t_dst_s, const int64_t* b, int64_t N, int steps,
                  float* out, atlb_stream_t stream) {
  clear();
  NONNEG(N);
  if (int st = check_rk4(B, Hg, Wg, H, W, steps, __func__)) return st;
  NEED(theta, B); NEED(xy, N); NEED(t, N); NEED(b, N); NEED(out, N);
  return flow_rk4(make_motion_view(ATLB_MOTION_DENSE, theta, B, Hg, Wg, H, W), xy, t, t_dst, (float)t_dst_s, LL(b), N,
                  steps, out, STREAM(stream));
}

int atlb_flow_rk4_bwd(const float* gy, const float* theta, int64_t B, int64_t Hg, int64_t Wg, int64_t H, int64_t W,
                      const float* xy, const float* t, const float* t_dst, double t_dst_s, const int64_t* b,
                      int64_t N, int steps, float* gtheta, atlb_stream_t stream) {
  clear();
  NONNEG(N);
  if (int st = check_rk4(B, Hg, Wg, H, W, steps, __func__)) return st;
  NEED(gy, N); NEED(theta, B); NEED(xy, N); NEED(t, N); NEED(b, N);
  if (!gtheta) { set_error("%s: gtheta is NULL", __func__); return ATLB_ERR_ARG; }
  return flow_rk4_bwd(make_motion_view(ATLB_MOTION_DENSE, theta, B, Hg, Wg, H, W), gy, xy, t, t_dst, (float)t_dst_s,
                      LL(b), N, steps, gtheta, STREAM(stream));
}

