/*
 * atl_b200.h -- C ABI of libatlb200.so, the B200 (sm_100a) implementation of the anchored transport
 * score path of KAVYANSHTYAGI/x (package `atl`).
 *
 * Conventions (the layout contract of the reference, csrc/atl_ops.h:3-8):
 *   pos  (N,2) float32 [x, y], pixel centres at integers;  w (N) float32;  bidx (N) int64 in [0, B);
 *   img  (B,H,W) float32.  All arrays are contiguous DEVICE pointers.  Events whose batch index lies
 *   outside [0, B) or whose position is not finite touch no pixel (the reference read out of bounds).  Outputs are caller-allocated
 *   and fully overwritten (the reference returned torch::zeros-initialised tensors).
 * Every entry point returns 0 (ATLB_OK) or an error code; atlb_last_error() gives the message of the
 * calling thread's last failure.  Work is enqueued on `stream`; an entry point documented as
 * "synchronous" waits for `stream` because it must read a device result on the host (as the
 * reference's torch code does with .item()-style reads).
 * There is no CPU path: every entry point needs a CUDA device of compute capability 10.0.
 */
#ifndef ATL_B200_H
#define ATL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* atlb_stream_t; /* a cudaStream_t; NULL = legacy default stream */

enum {
  ATLB_OK = 0,
  ATLB_ERR_ARG = 1,       /* invalid argument (null pointer, negative size, bad enum) */
  ATLB_ERR_CUDA = 2,      /* a CUDA launch or runtime call failed */
  ATLB_ERR_WORKSPACE = 3, /* workspace smaller than the matching *_workspace_bytes() */
  ATLB_ERR_UNSORTED = 4,  /* events not sorted by (b, t); see atlb_window_counts */
  ATLB_ERR_OVERFLOW = 5   /* a size does not fit the index types of the kernels */
};

/* Message of the calling thread's last non-zero status ("" if none). */
const char* atlb_last_error(void);
/* ABI version of this header (bumped on incompatible changes). */
int atlb_abi_version(void);
#define ATLB_ABI_VERSION 12
/* Number of kernels this library has launched in the calling process (instrumentation; no reference
 * counterpart). */
uint64_t atlb_kernel_launches(void);
/* Opt-in CUDA-event timing of the main kernels (instrumentation; no reference counterpart).  While
 * enabled, each launch of a timed kernel ("k_pair_fwd", "k_pair_bwd", ...) is bracketed by events on
 * its stream; atlb_timing_read waits for them and returns the summed milliseconds and launch count
 * for `name` (reset != 0 forgets them). */
int atlb_timing_enable(int on);
int atlb_timing_read(const char* name, double* total_ms, int64_t* count, int reset);

/* Execution-unit rates of the current device (instrumentation; no reference counterpart): the
 * denominators of the compute roofline of the pair and splat kernels.  Each figure is whole-device
 * operations per second, from a CUDA-event-timed kernel that runs independent chains of that one
 * operation on every SM, after an identical warm-up launch.  Blocking: returns when the measurement
 * kernels (about 10 ms) have finished on `stream`.  scratch: atlb_unit_rates_scratch_bytes() bytes of
 * device memory, overwritten. */
typedef struct {
  double fp32_lane_ops;   /* fma.rn.f32: lane operations per second */
  double fp32x2_lane_ops; /* fma.rn.f32x2: lane operations per second (two per instruction and lane) */
  double ex2;             /* ex2.approx.ftz.f32 per second */
  double red_f32;         /* red.global.add.f32 at scattered words of an L2-resident 32 MB buffer */
  double red_v4;          /* red.global.add.v4.f32 at scattered 16-byte quads of the same buffer */
  double smem_atomic;     /* atomicAdd on scattered shared-memory floats */
} atlb_unit_rates;
size_t atlb_unit_rates_scratch_bytes(void);
int atlb_measure_unit_rates(atlb_unit_rates* out, void* scratch, size_t scratch_bytes, atlb_stream_t stream);

/* ----------------------------------------------------------------------------------------------
 * Splat / gather / voxel.  Replace the reference's bound kernels
 *   splat_bilinear_fwd/bwd  csrc/atl_cpu.cpp:38-76   (decl. csrc/atl_ops.h:20-21)
 *   splat_gauss_fwd/bwd     csrc/atl_cpu.cpp:79-131  (decl. csrc/atl_ops.h:23-26)
 *   gather_bilinear_fwd/bwd csrc/atl_cpu.cpp:134-172 (decl. csrc/atl_ops.h:28-29)
 *   voxel_grid              csrc/atl_cpu.cpp:256-286 (decl. csrc/atl_ops.h:48-49)
 * and the separable blur of atl/ops/functional.py:99-110 (torch conv2d in the reference).
 * The bilinear splat, the gather and the voxel grid bucket their points by 32x32-pixel image tile in the
 * workspace (atlb_tile_ops_workspace_bytes) and work on shared-memory tiles; per point, corners are taken
 * in the reference's order and rounding (the gather and both backward passes are bit-identical to it).
 * ---------------------------------------------------------------------------------------------- */
size_t atlb_tile_ops_workspace_bytes(int64_t N, int64_t B, int64_t H, int64_t W);
int atlb_splat_bilinear_fwd(const float* pos, const float* w, const int64_t* bidx, int64_t N, int64_t B, int64_t H,
                            int64_t W, float* img, void* workspace, size_t workspace_bytes, atlb_stream_t stream);
int atlb_splat_bilinear_bwd(const float* gimg, const float* pos, const float* w, const int64_t* bidx, int64_t N,
                            int64_t B, int64_t H, int64_t W, float* gpos, float* gw, void* workspace,
                            size_t workspace_bytes, atlb_stream_t stream);
/* Gaussian splat: events are bucketed by 32x32-pixel image tile in the workspace
 * (atlb_splat_gauss_workspace_bytes), one shared-memory tile per CTA.  radius <= ATLB_SPLAT_GAUSS_MAX_RADIUS
 * (the tile and its halo live in shared memory). */
#define ATLB_SPLAT_GAUSS_MAX_RADIUS 96
size_t atlb_splat_gauss_workspace_bytes(int64_t N, int64_t B, int64_t H, int64_t W);
int atlb_splat_gauss_fwd(const float* pos, const float* w, const int64_t* bidx, int64_t N, int64_t B, int64_t H,
                         int64_t W, double sigma, int64_t radius, float* img, void* workspace, size_t workspace_bytes,
                         atlb_stream_t stream);
int atlb_splat_gauss_bwd(const float* gimg, const float* pos, const float* w, const int64_t* bidx, int64_t N,
                         int64_t B, int64_t H, int64_t W, double sigma, int64_t radius, float* gpos, float* gw,
                         void* workspace, size_t workspace_bytes, atlb_stream_t stream);
/* Backward w.r.t. the positions only (gpos (N,2)), over the buckets that the preceding atlb_splat_gauss_fwd
 * of the same (pos, w, bidx, B, H, W, R) left in `workspace`, which the caller keeps unchanged in between:
 * the forward's bucketing is reused instead of redone.  Events the forward skipped (zero weight) get 0. */
int atlb_splat_gauss_bwd_pos(const float* gimg, const float* w, int64_t N, int64_t B, int64_t H, int64_t W,
                             double sigma, int64_t R, float* gpos, void* workspace, size_t workspace_bytes,
                             atlb_stream_t stream);
int atlb_gather_bilinear_fwd(const float* img, const float* pos, const int64_t* bidx, int64_t N, int64_t B, int64_t H,
                             int64_t W, float* out, void* workspace, size_t workspace_bytes, atlb_stream_t stream);
int atlb_gather_bilinear_bwd(const float* gval, const float* img, const float* pos, const int64_t* bidx, int64_t N,
                             int64_t B, int64_t H, int64_t W, float* gimg, float* gpos, void* workspace,
                             size_t workspace_bytes, atlb_stream_t stream);
int atlb_voxel_grid(const float* pos, const float* t, const float* p, const int64_t* bidx, int64_t N, int64_t B,
                    int64_t C, int64_t H, int64_t W, float* vox, void* workspace, size_t workspace_bytes,
                    atlb_stream_t stream);
/* Separable Gaussian blur with zero padding of P planes of H x W: the normalised kernel of radius
 * max(ceil(3 sigma), 1) <= 32 along rows, then along columns.  The blur is its own adjoint (symmetric kernel,
 * zero padding), so the same call gives the backward.  out must not alias img. */
int atlb_blur(const float* img, int64_t P, int64_t H, int64_t W, double sigma, float* out, atlb_stream_t stream);

/* ----------------------------------------------------------------------------------------------
 * Pair plan: the device replacement of build_pair_plan (atl/ops/functional.py:132-178), in three
 * calls because two sizes are only known on the device:
 *   1. atlb_plan_geometry   vmax, anchor bounding box -> cell, origin, GW, GH    (synchronous)
 *   2. atlb_plan_count      per-cell counts -> cell_start (B*S*GH*GW + 1), #entries (synchronous)
 *   3. atlb_plan_fill       the sorted entries and the anchor cells               (asynchronous)
 * Cell keys, CSR offsets, slice ranges and anchor cells are bit-identical to the reference's CPU
 * path; entries inside one cell come in an unspecified order (the reference's argsort is unstable).
 * ---------------------------------------------------------------------------------------------- */
typedef struct {
  double cell, ox, oy; /* cell size and grid origin (double, as the reference's Python computes them) */
  int64_t GW, GH;      /* grid width / height in cells */
  float vmax;          /* max_j |v_j| (torch's row norm) */
  int32_t S;           /* number of slices */
  float t_lo, t_hi;    /* event time range (atlb_exact_prepare; NaN when not computed) */
} atlb_plan_geom;

/* x (N,2) positions, v (N,2) velocities, anchors (M) event indices, anchor_xy (M,2) the positions the
 * anchors are evaluated at, or NULL for x[anchors].  scratch: device buffer of >= 32 bytes.  Fails with
 * ATLB_ERR_ARG if an anchor index lies outside [0, N).  Replaces functional.py:136-149. */
int atlb_plan_geometry(const float* x, const float* v, int64_t N, const int64_t* anchors, const float* anchor_xy,
                       int64_t M, int64_t H, int64_t W, double h, double cut, int64_t S, void* scratch,
                       atlb_plan_geom* geom_out, atlb_stream_t stream);
size_t atlb_plan_workspace_bytes(int64_t ncell);
/* cell_start: int64[ncell + 1] with ncell = B*S*GH*GW.  *n_entries_out receives cell_start[ncell].
 * workspace must stay untouched until atlb_plan_fill.  Replaces functional.py:150-168. */
int atlb_plan_count(const float* x, const float* t, const float* v, const int64_t* b, int64_t N, int64_t B, double tau,
                    const atlb_plan_geom* geom, int64_t* cell_start, void* workspace, size_t workspace_bytes,
                    int64_t* n_entries_out, atlb_stream_t stream);
/* anchors (M) event indices; anchor_xy (M,2) or NULL (= x[anchors]).  Outputs as PairPlan
 * (functional.py:114-129): src_y/src_v (Ns,2), src_t (Ns), src_id (Ns) int64, anc_x (M,2), anc_t (M),
 * anc_cell (M,3) int64, anc_id (M) int64, slice_c (S).  Replaces functional.py:150-178. */
int atlb_plan_fill(const float* x, const float* t, const float* v, const int64_t* b, int64_t N, int64_t B, double tau,
                   const atlb_plan_geom* geom, const int64_t* anchors, const float* anchor_xy, int64_t M,
                   const int64_t* cell_start, void* workspace, size_t workspace_bytes, float* src_y, float* src_v,
                   float* src_t, int64_t* src_id, float* anc_x, float* anc_t, int64_t* anc_cell, int64_t* anc_id,
                   float* slice_c, atlb_stream_t stream);

/* ----------------------------------------------------------------------------------------------
 * Anchored pair sums over a plan.  Replace ats_pair_fwd / ats_pair_bwd
 *   csrc/atl_cpu.cpp:203-253 (decl. csrc/atl_ops.h:35-46; bound at csrc/atl_cpu.cpp:312-320).
 * Arguments are the plan arrays in the reference's layout; ncell = length(cell_start) - 1 and
 * Ns = cell_start[ncell].  The workspace holds the anchors bucketed by cell.
 * ---------------------------------------------------------------------------------------------- */
size_t atlb_pair_workspace_bytes(int64_t M, int64_t ncell);
int atlb_ats_pair_fwd(const float* src_y, const float* src_v, const float* src_t, const int64_t* src_id,
                      const int64_t* cell_start, const float* anc_x, const float* anc_t, const int64_t* anc_cell,
                      const int64_t* anc_id, const float* slice_c, int64_t Ns, int64_t M, int64_t ncell, int64_t S,
                      int64_t GH, int64_t GW, double h, double tau, double cut, float* out, void* workspace,
                      size_t workspace_bytes, atlb_stream_t stream);
/* atlb_ats_pair_fwd without a workspace argument: the same sums, for callers that cannot allocate
 * device memory when they need them -- hosts that give the library a fixed device-memory budget (a
 * custom allocator, an embedded runtime), loops that forbid cudaMalloc after start-up because it can
 * synchronise the device, and FFI layers that have no device allocator of their own.  No counterpart in
 * the reference: it is an addition of this library.  The anchor buckets live in one file-scope device
 * array of ATLB_PAIR_NOALLOC_SCRATCH_BYTES, which every device that loads the library holds until the
 * process exits; the call allocates nothing.  A call needs atlb_pair_workspace_bytes(M, ncell) - 256
 * bytes of it (the array is 256-byte aligned, so the workspace's alignment slack is not needed); larger
 * sizes fail with ATLB_ERR_WORKSPACE before any device work.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress, with that device current) and keeps it for the process,
 * so make that first call before any stream capture; the kept address belongs to the device's primary
 * context and does not survive cudaDeviceReset or a switch to another context on that device.  All
 * calls share the array: calls whose work overlaps on the GPU (other streams or host threads) race;
 * calls ordered on one stream do not.  Not covered by atlb_timing_*. */
#define ATLB_PAIR_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
int atlb_ats_pair_fwd_noalloc(const float* src_y, const float* src_v, const float* src_t, const int64_t* src_id,
                              const int64_t* cell_start, const float* anc_x, const float* anc_t,
                              const int64_t* anc_cell, const int64_t* anc_id, const float* slice_c, int64_t Ns,
                              int64_t M, int64_t ncell, int64_t S, int64_t GH, int64_t GW, double h, double tau,
                              double cut, float* out, atlb_stream_t stream);
/* gv (N,2): gradient of sum_i gS_i S_i w.r.t. the per-event velocities. */
int atlb_ats_pair_bwd(const float* gS, const float* src_y, const float* src_v, const float* src_t,
                      const int64_t* src_id, const int64_t* cell_start, const float* anc_x, const float* anc_t,
                      const int64_t* anc_cell, const int64_t* anc_id, const float* slice_c, int64_t Ns, int64_t M,
                      int64_t ncell, int64_t S, int64_t GH, int64_t GW, double h, double tau, double cut, int64_t N,
                      float* gv, void* workspace, size_t workspace_bytes, atlb_stream_t stream);

/* ----------------------------------------------------------------------------------------------
 * window_counts (atl/ops/functional.py:210-217): out[q] = #{j != idx[q], same batch,
 * |t_j - t_idx[q]| <= tau} through float64 keys b*4 + t.  Events must be sorted by (b, t) (the
 * EventPacket invariant, atl/core/events.py:12); the call checks it on the device and returns
 * ATLB_ERR_UNSORTED without a result otherwise (synchronous).  For unsorted events pass the sorted
 * float64 keys instead to atlb_window_counts_keys.
 * ---------------------------------------------------------------------------------------------- */
int atlb_window_counts(const float* t, const int64_t* b, int64_t N, const int64_t* idx, int64_t M, double tau,
                       float* out, void* scratch, atlb_stream_t stream);
int atlb_window_counts_keys(const double* sorted_keys, int64_t N, const float* t, const int64_t* b,
                            const int64_t* idx, int64_t M, double tau, float* out, atlb_stream_t stream);

/* ----------------------------------------------------------------------------------------------
 * Motion fields of stage 1 (velocity linear at the event) and the exposure correction.
 *   kind 0 Translation  theta (B,2)        atl/motion/parametric.py:148-157
 *   kind 1 Affine       theta (B,6)        atl/motion/parametric.py:207-217
 *   kind 2 DenseLinearFlow grid (B,2,Hg,Wg) atl/motion/parametric.py:257-312 (sample_grid)
 * ---------------------------------------------------------------------------------------------- */
enum { ATLB_MOTION_TRANSLATION = 0, ATLB_MOTION_AFFINE = 1, ATLB_MOTION_DENSE = 2 };
int atlb_velocity(int kind, const float* theta, int64_t B, int64_t Hg, int64_t Wg, int64_t H, int64_t W,
                  const float* xy, const int64_t* b, int64_t N, float* v, atlb_stream_t stream);
/* gtheta (same shape as theta) = d(sum_j gv_j . v_j)/d theta; overwritten. */
int atlb_velocity_bwd(int kind, const float* gv, int64_t B, int64_t Hg, int64_t Wg, int64_t H, int64_t W,
                      const float* xy, const int64_t* b, int64_t N, float* gtheta, atlb_stream_t stream);
/* visible_fraction (atl/objectives/ats.py:31-50) for linear transport; scratch >= B*n_check*4 bytes. */
int atlb_visible_fraction(int kind, const float* theta, int64_t B, int64_t Hg, int64_t Wg, int64_t H, int64_t W,
                          const float* xa, const float* ta, const int64_t* ba, int64_t M, const float* t,
                          const int64_t* b, int64_t N, double tau, int64_t n_check, float* out, void* scratch,
                          atlb_stream_t stream);

/* ----------------------------------------------------------------------------------------------
 * Continuous-time pixel trajectories (atl/motion/trajectories.py:40-90), the motion of the sliced
 * path: transport of events x at times t to t_dst and its backward to the tile coefficients.
 *   coeff  (B, Hq, Wq, 2K) channels-last tile coefficients, channels [y_1..y_K, x_1..x_K]
 *   basis  0: g_k(t) = t^k;  1: Bezier, g_k(t) = bezier_c[k] t^k (1 - t)^(K - k)  (bezier_c: K floats,
 *          exp(lgamma(K+1) - lgamma(k+1) - lgamma(K-k+1)) as the reference computes them in fp32)
 *   the coefficients at p are the bilinear (border-clamped) sample at (p - offset) / tile; the origin is
 *   the fixed point of p = x - d(p, t) after n_fp iterations; t_dst (N) per event, or NULL for t_dst_s.
 * K <= 16, n_fp <= 16 and B Hq Wq 2K < 2^31 floats.  Events with b outside [0, B) get NaN.  The
 * backward ADDS dL/dcoeff (same layout) for gy = dL/dout into gcoeff.
 * ---------------------------------------------------------------------------------------------- */
/* mode 0: out = transport(xy, t -> t_dst); 1: out = the origin p (the fixed point; t_dst unused);
 * 2: xy holds origins, out = p + d(p, t_dst) (t unused); 3: out = the first coefficient pair (c_x1, c_y1)
 * sampled at the origin, PixelTrajectories.velocity (atl/motion/trajectories.py:79-83) of the degree-1
 * polynomial trajectories (t_dst unused).  Modes 1 then 2 reproduce mode 0 exactly, so a caller moving
 * the same events to several times solves each origin once. */
int atlb_traj_transport(int mode, const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K, int basis,
                        const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xy,
                        const float* t, const float* t_dst, double t_dst_s, const int64_t* b, int64_t N, float* out,
                        atlb_stream_t stream);
/* Exposure correction (atl/objectives/ats.py:31-50) of M anchors (xa, ta, ba) under these trajectories:
 * counts (B, n_check) per-batch event counts of the n_check time slices, centres (n_check) the slice
 * centres (device arrays), sensor W x H; out (M).  The trajectory's origin is solved once per anchor. */
int atlb_traj_visible_fraction(const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K, int basis,
                               const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xa,
                               const float* ta, const int64_t* ba, int64_t M, const float* counts,
                               const float* centres, int64_t n_check, double tau, int64_t H, int64_t W, float* out,
                               atlb_stream_t stream);
/* Backward of the same mode (0..3) for gy = dL/dout: adds dL/dcoeff into gcoeff; mode 2 also writes
 * gp (N,2) = dL/d(its input origins). */
int atlb_traj_transport_bwd(int mode, const float* gy, const float* coeff, int64_t B, int64_t Hq, int64_t Wq,
                            int64_t K, int basis, const float* bezier_c, double offset, double tile, int64_t n_fp,
                            const float* xy, const float* t, const float* t_dst, double t_dst_s, const int64_t* b,
                            int64_t N, float* gcoeff, float* gp, atlb_stream_t stream);
/* Records: xy (N, R, 2) holds R positions per event, all at the event's time t; each is moved to the event's
 * target time (t_dst (N), or t_dst_s when t_dst is NULL) exactly as mode 0 moves it: out (N, R, 2).  The
 * transports of an anchor and of its finite-difference probes (atl/motion/base.py:43-50) in one call.
 * iterates (optional, NULL: none) receives the fixed-point iterates, (n_fp, N, R, 2).  The backward ADDS
 * dL/dcoeff for gy (N, R, 2) into gcoeff; given the forward's iterates it reads them instead of solving
 * the fixed points again. */
int atlb_traj_records(const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K, int basis,
                      const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xy, int64_t R,
                      const float* t, const float* t_dst, double t_dst_s, const int64_t* b, int64_t N, float* out,
                      float* iterates, atlb_stream_t stream);
int atlb_traj_records_bwd(const float* gy, const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K,
                          int basis, const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xy,
                          int64_t R, const float* t, const float* t_dst, double t_dst_s, const int64_t* b, int64_t N,
                          const float* iterates, float* gcoeff, atlb_stream_t stream);
/* Targets: every event (xy (N,2), t) moved to each of T target times (targets, a device array, T <= 64):
 * out (T, N, 2), entry (j, n) exactly as mode 0 moves event n to targets[j] (the transports of every source
 * to every slice centre, atl/objectives/ats.py:141-147, with one origin solve per event).  The backward ADDS
 * dL/dcoeff for gy (T, N, 2) into gcoeff. */
int atlb_traj_targets(const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K, int basis,
                      const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xy, const float* t,
                      const int64_t* b, int64_t N, const float* targets, int64_t T, float* out, atlb_stream_t stream);
int atlb_traj_targets_bwd(const float* gy, const float* coeff, int64_t B, int64_t Hq, int64_t Wq, int64_t K,
                          int basis, const float* bezier_c, double offset, double tile, int64_t n_fp, const float* xy,
                          const float* t, const int64_t* b, int64_t N, const float* targets, int64_t T, float* gcoeff,
                          atlb_stream_t stream);

/* ----------------------------------------------------------------------------------------------
 * AnchoredSliced per-anchor score (atl/objectives/ats.py:154-169; the leave-one-out terms of
 * ats.py:186-200 and atl/objectives/cmax.py:125-137), all anchors of all slices in one call.
 * pos (N, P, 2): per anchor P transported positions at its slice centre; slot ia = the smoothed anchor
 * position a, slot io = the unsmoothed (source) position (io < 0: self term at a), slots ip..ip+3 = the
 * transports of x +- delta e_x, x +- delta e_y (ip < 0: no log-determinant).  val (N) density gathered at a,
 * cnt (N) sources of the anchor's slice and batch minus src, vis (N) exposure correction (NULL: none),
 * src (N) 1 / 0 = the anchor is / is not a source of its slice.  Image W x H, Gaussian sigma, eps.
 *   ls = log(eps + max(val - src loo, 0) / max(cnt vis, 1)) + log(max(|det J|, 1e-12))
 * The backward writes gval (N) = dL/dval and gpos (N, P, 2) = dL/dpos for gls = dL/dls.
 * ---------------------------------------------------------------------------------------------- */
/* Key counts: out (R, nbins) int64, out[r][k] = #{n < N : key[n] == k and (mask == NULL or
 * mask[r * N + n] != 0)}; keys outside [0, nbins) are not counted; nbins * R <= 2^24.  The histograms of
 * AnchoredSliced: anchors per slice, sources per slice and batch (R = slices, mask = source masks),
 * events per exposure-check slice (ats.py:39-41). */
int atlb_count_keys(const int64_t* key, int64_t N, int64_t nbins, const float* mask, int64_t R, int64_t* out,
                    atlb_stream_t stream);
int atlb_sliced_score(int64_t N, int P, int ia, int io, int ip, const float* pos, const float* val, const float* cnt,
                      const float* vis, const float* src, double sigma, double delta, double eps, int64_t H,
                      int64_t W, float* ls, atlb_stream_t stream);
int atlb_sliced_score_bwd(int64_t N, int P, int ia, int io, int ip, const float* gls, const float* pos,
                          const float* val, const float* cnt, const float* vis, const float* src, double sigma,
                          double delta, double eps, int64_t H, int64_t W, float* gval, float* gpos,
                          atlb_stream_t stream);

/* ----------------------------------------------------------------------------------------------
 * Fused anchored score: AnchoredExact.log_scores (atl/objectives/ats.py:75-96) for the motion kinds
 * above, with its backward.  Three calls:
 *   atlb_exact_prepare   dequantised positions xs = xy + (u - 1/2) (u NULL: none), velocities v(xs),
 *                        anchor positions xa = xs[a] + h z (z NULL: none; anchors NULL: all events),
 *                        grid geometry.  Writes ev4 (N,4) = (xs, v) and anc4 (M,4) = (xa, t_a, a bits),
 *                        anc_b (M).  Synchronous.  ATLB_ERR_UNSORTED if events are not (b, t) sorted.
 *   atlb_exact_forward   plan, window counts (ats.py:92), exposure correction (ats.py:93-94), pair
 *                        sums; S (M), den (M) = W * vis * 2 pi h^2 and ls (M) = log(eps + S / den).
 *   atlb_exact_backward  from dL/dls (M): gv (N,2) = dL/dv and gtheta = dL/dtheta (overwritten).
 * The workspace (atlb_exact_workspace_bytes) carries the plan from forward to backward.
 * ---------------------------------------------------------------------------------------------- */
typedef struct {
  int32_t kind;          /* ATLB_MOTION_* */
  const float* theta;    /* motion parameters / flow grid */
  int64_t Bt, Hg, Wg;    /* parameter batch; flow grid height / width (dense) */
  int64_t B, H, W;       /* event batch size; sensor height / width */
  double h, tau, cut, eps_frac;
  int64_t S;             /* n_slices */
  int32_t visibility;    /* exposure correction on (1) / off (0) */
  int64_t n_check;       /* slices of the exposure check (16 in the reference) */
  int64_t src_begin, src_end; /* sources of the pair sums: events [src_begin, src_end); src_end <= 0: all.
                              * With a sub-range, S_out holds the partial sums over those sources (sum
                              * them across the ranges, then ls = log(eps + S / den)), and the backward
                              * returns gv and gtheta of those sources only (sum gtheta across ranges). */
  int32_t rng;           /* bit 0 (u) / bit 1 (z): atlb_exact_prepare draws that noise on the device when it
                          * is given as NULL (atlb_rng_uniform2 / atlb_rng_normal2 of rng_seed, call
                          * rng_call) instead of leaving it out; 0: NULL means "none", as in the reference */
  uint64_t rng_seed, rng_call;
} atlb_exact_cfg;

int atlb_exact_prepare(const atlb_exact_cfg* cfg, const float* xy, const float* u, const float* t, const int64_t* b,
                       int64_t N, const int64_t* anchors, const float* z, int64_t M, float* ev4, float* anc4,
                       int64_t* anc_b, void* scratch, atlb_plan_geom* geom_out, atlb_stream_t stream);
size_t atlb_exact_workspace_bytes(const atlb_exact_cfg* cfg, int64_t N, int64_t M, const atlb_plan_geom* geom);
int atlb_exact_forward(const atlb_exact_cfg* cfg, const float* t, const int64_t* b, int64_t N, int64_t M,
                       const float* ev4, const float* anc4, const int64_t* anc_b, const atlb_plan_geom* geom,
                       void* workspace, size_t workspace_bytes, float* S_out, float* den_out, float* ls_out,
                       atlb_stream_t stream);
/* atlb_exact_prepare then atlb_exact_forward in one call, for a caller that sized the workspace ahead (for
 * instance from the previous window's atlb_exact_workspace_bytes): the forward's kernels follow the geometry
 * read-back with no return to the caller in between, so the device does not wait on the caller's code there.
 * If the workspace is smaller than this window's plan needs, the prepare outputs (ev4, anc4, anc_b, geom_out)
 * are written and ATLB_ERR_WORKSPACE is returned: size the workspace from geom_out and call
 * atlb_exact_forward.  Replaces the same steps of AnchoredExact.log_scores (atl/objectives/ats.py:75-96). */
int atlb_exact_prepare_forward(const atlb_exact_cfg* cfg, const float* xy, const float* u, const float* t,
                               const int64_t* b, int64_t N, const int64_t* anchors, const float* z, int64_t M,
                               float* ev4, float* anc4, int64_t* anc_b, void* scratch, atlb_plan_geom* geom_out,
                               void* workspace, size_t workspace_bytes, float* S_out, float* den_out, float* ls_out,
                               atlb_stream_t stream);
int atlb_exact_backward(const atlb_exact_cfg* cfg, const float* grad_ls, const int64_t* b, int64_t N, int64_t M,
                        const float* ev4, const atlb_plan_geom* geom, void* workspace, size_t workspace_bytes,
                        const float* S, const float* den, float* gv, float* gtheta, atlb_stream_t stream);

/* ----------------------------------------------------------------------------------------------
 * Exact transport of the affine velocity fields (Translation, Affine), VectorFieldMotion.transport with
 * mode="exact" (atl/motion/parametric.py:60-71): y = c + E[:2,:2] (x - c) + E[:2,2] with
 * E = exp(dt [[A, t], [0, 0]]), dt = t_dst - t (t_dst per event, or the scalar t_dst_s when NULL),
 * c = ((W - 1) / 2, (H - 1) / 2).  kind: ATLB_MOTION_TRANSLATION or ATLB_MOTION_AFFINE.
 * The backward overwrites gtheta (B, 2|6) with dL/dtheta and, when gxy is not NULL, writes dL/dxy.
 * ---------------------------------------------------------------------------------------------- */
int atlb_flow_exact(int kind, const float* theta, int64_t B, int64_t H, int64_t W, const float* xy, const float* t,
                    const float* t_dst, double t_dst_s, const int64_t* b, int64_t N, float* out, atlb_stream_t stream);
int atlb_flow_exact_bwd(int kind, const float* gy, const float* theta, int64_t B, int64_t H, int64_t W,
                        const float* xy, const float* t, const float* t_dst, double t_dst_s, const int64_t* b,
                        int64_t N, float* gtheta, float* gxy, atlb_stream_t stream);
/* Exact transport of the dense velocity grid, DenseLinearFlow.transport with mode="exact"
 * (atl/motion/parametric.py:72-80): `steps` classic RK4 steps (1..64) of the grid's bilinear field
 * (theta (B, 2, Hg, Wg), the field of atlb_velocity) over dt = t_dst - t, rounded as the reference's torch
 * ops.  The backward overwrites gtheta (B, 2, Hg, Wg) with dL/dtheta for gy = dL/dout. */
int atlb_flow_rk4(const float* theta, int64_t B, int64_t Hg, int64_t Wg, int64_t H, int64_t W, const float* xy,
                  const float* t, const float* t_dst, double t_dst_s, const int64_t* b, int64_t N, int steps,
                  float* out, atlb_stream_t stream);
int atlb_flow_rk4_bwd(const float* gy, const float* theta, int64_t B, int64_t Hg, int64_t Wg, int64_t H, int64_t W,
                      const float* xy, const float* t, const float* t_dst, double t_dst_s, const int64_t* b,
                      int64_t N, int steps, float* gtheta, atlb_stream_t stream);

/* ----------------------------------------------------------------------------------------------
 * Opt-in device draws of the objective's noise.  No counterpart in the reference, which draws the
 * dequantisation jitter u ~ U[0,1)^2 (atl/objectives/ats.py:84-85, 133-134) and the anchor smoothing
 * noise z ~ N(0, I) (ats.py:87-88, 135) on the host with torch's CPU generator; these streams differ
 * from torch's, so callers use them only when they ask for device draws.  Philox4x32-10 (Salmon et
 * al., SC'11) with counter (i, stream, call, call >> 32) and key seed: out (n,2) float32.
 * ---------------------------------------------------------------------------------------------- */
int atlb_rng_uniform2(uint64_t seed, uint64_t call, int64_t n, float* out, atlb_stream_t stream);
int atlb_rng_normal2(uint64_t seed, uint64_t call, int64_t n, float* out, atlb_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* ATL_B200_H */
