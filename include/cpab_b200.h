/*
 * cpab_b200.h -- C ABI of the sm_100a implementation of the FG-CPAB hot path.
 *
 * The library (libcpab_b200.so) integrates points through continuous
 * piecewise-affine (CPA) velocity fields in 1D/2D/3D, runs the factorized
 * adjoint sweep that produces per-cell moments, projects the moments onto the
 * CPA basis (dtheta = B^T vec(M)) and resamples images/volumes on warped grids.
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers to contiguous fp32 / int32 arrays; the
 *     caller owns every buffer.  Nothing here allocates device memory.
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *     stream) and is asynchronous with respect to the host.
 *   - The return value is CPAB_OK (0) or a negative cpab_status.  Argument
 *     errors are detected on the host before anything is launched; the message
 *     is available from cpab_b200_last_error() (per host thread).  No entry
 *     point ever terminates the process.
 *   - Layouts follow the reference extension: points are [ndim, nP] (shared by
 *     all transformations) or [n_theta, ndim, nP]; affine cell matrices are
 *     [n_theta, nC, ndim, ndim+1] row-major; moments are [n_theta, nC, ppc]
 *     with ppc = ndim*(ndim+1).
 *   - Cell-matrix tables (As, trels) must be 16-byte aligned (they are read
 *     with vector loads); every other array only needs its natural alignment.
 *   - Tessellation: nc[0..ndim-1] cells per axis (1 <= nc[k] <= 2^20) on
 *     [0,1]^ndim; nC = nc[0]
 *     (1D), 4*nc[0]*nc[1] (2D, four triangles per square), 5*nc[0]*nc[1]*nc[2]
 *     (3D, five tetrahedra per cube).
 *
 * Reference interfaces replaced (paths inside the FG-CPAB project):
 *   cpab/pytorch/transformer_cuda.cpp:32-61   forward               -> cpab_b200_forward
 *   cpab/pytorch/transformer_cuda.cpp:66-85   forward_1d_closed_form -> cpab_b200_forward_1d_closed_form
 *   cpab/pytorch/transformer_cuda.cpp:92-116  backward_moments      -> cpab_b200_backward (grad_points = NULL)
 *   cpab/pytorch/transformer_cuda.cpp:122-153 backward_moments_and_points -> cpab_b200_backward
 *   cpab/pytorch/transformer_cuda.cpp:159-170 expm                  -> cpab_b200_expm
 *   cpab/pytorch/transformer.py:84-88         A = B theta^T (torch.sparse.mm) -> cpab_b200_build_A
 *   cpab/pytorch/transformer.py:165-166       dtheta = B^T m (torch.sparse.mm) -> cpab_b200_project
 *   cpab/pytorch/interpolation.py:8-160       interpolate{1,2,3}D (+autograd) -> cpab_b200_interpolate{,_backward}
 */
#ifndef CPAB_B200_H
#define CPAB_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *cpab_stream_t; /* identical to cudaStream_t */

typedef enum {
  CPAB_OK = 0,
  CPAB_ERR_ARG = -1,    /* invalid shape / pointer / flag                 */
  CPAB_ERR_STEPS = -2,  /* nstepsolver outside [1, cpab_b200_max_steps()] */
  CPAB_ERR_CUDA = -3,   /* a CUDA launch or runtime call failed           */
  CPAB_ERR_SIZE = -4    /* a size exceeds a documented limit              */
} cpab_status;

/* Library version (major*10000 + minor*100 + patch). */
int cpab_b200_version(void);

/* Largest nstepsolver accepted by forward/backward (the reference allows 100). */
int cpab_b200_max_steps(void);

/* Message of the last failed call on this host thread ("" if none). */
const char *cpab_b200_last_error(void);

/*
 * Trels[i] = expm(dT * [A_i; 0 ... 0 1]) restricted to its top ndim rows, for
 * n affine matrices A_i of shape [ndim, ndim+1].  Scaling-and-squaring with
 * the (2,2) Pade approximant in 2D/3D; closed form [e^a, b*(e^a-1)/a] in 1D.
 * Replaces cpab/pytorch/transformer_cuda.cpp:159-170 (cpab_expm).
 */
int cpab_b200_expm(int ndim, const float *As, int64_t n_matrices, float dT,
                   float *trels, cpab_stream_t stream);

/*
 * A = reshape((B theta^T)^T): As[t, r] = sum_k B[r, k] * theta[t, k] for the
 * D x d CSR basis B (D = nC*ppc rows).  When trels != NULL also writes
 * trels = expm(dT * A) per cell (same rule as cpab_b200_expm), fused.
 * Replaces cpab/pytorch/transformer.py:84-88 and :104-106.
 */
int cpab_b200_build_A(int ndim, int64_t nC, int64_t d, int n_theta,
                      const int32_t *B_rowptr, const int32_t *B_colidx,
                      const float *B_vals, const float *theta, float dT,
                      float *As, float *trels, cpab_stream_t stream);

/*
 * Forward integration to t = 1 in 2D/3D: nstepsolver exact per-cell steps
 * p <- trels[cell(p)] [p; 1]; with adaptive = 1 a step that changes cell is
 * replaced by one Heun step on the velocity fields As.  `points_batched` = 1
 * when points is [n_theta, ndim, nP], 0 when it is [ndim, nP].  out is
 * [n_theta, ndim, nP].  nc has ndim entries.  `order` (may be NULL) is a
 * processing order from cpab_b200_order_points: [1, nP] for shared points,
 * [n_theta, nP] for batched ones; it changes only which thread handles which
 * point, never a result.  For ndim == 1 this forwards to
 * cpab_b200_forward_1d_closed_form (trels and nstepsolver are then unused),
 * like the reference's dispatch.
 * Replaces cpab/pytorch/transformer_cuda.cpp:32-61 (cpab_forward).
 */
int cpab_b200_forward(int ndim, const int32_t *nc, const float *points,
                      int64_t nP, int points_batched, const int32_t *order,
                      const float *trels,
                      const float *As, int n_theta, int nstepsolver,
                      int adaptive, float *out, cpab_stream_t stream);

/*
 * Exact 1D CPA integration to t = 1 (analytic cell walk, no time stepping).
 * Replaces cpab/pytorch/transformer_cuda.cpp:66-85.
 */
int cpab_b200_forward_1d_closed_form(const float *points, int64_t nP,
                                     int points_batched, const int32_t *order,
                                     const float *As,
                                     int n_theta, int ncx, float *out,
                                     cpab_stream_t stream);

/*
 * Factorized adjoint sweep.  Replays every trajectory with the midpoint rule
 * (nstepsolver steps, Heun on crossings when adaptive = 1), walks it backwards
 * from lambda(1) = grad_out and accumulates the per-cell moments
 *   M_c += h lam p_mid^T + (h^2/2) (A_c^T lam) p^T    (as [n_theta, nC, ppc]).
 * moments (16-byte aligned) is overwritten (zeroed here first); its sums are
 * fp32 reductions in L2, so their last bits vary from run to run.  When
 * grad_points != NULL it
 * receives lambda(0) as [n_theta, ndim, nP] (the reference's grad_points
 * before its optional batch sum).
 * Replaces cpab/pytorch/transformer_cuda.cpp:92-116 and :122-153.
 */
int cpab_b200_backward(int ndim, const int32_t *nc, const float *points,
                       int64_t nP, int points_batched, const int32_t *order,
                       const float *As,
                       int n_theta, const float *grad_out, int nstepsolver,
                       int adaptive, float *moments, float *grad_points,
                       cpab_stream_t stream);

/*
 * cpab_b200_build_A with theta given transposed, theta_t [d, n_theta]
 * (theta_t[k * n_theta + t] = theta[t, k]); same results.  For bases with
 * many nonzeros per row (zero_boundary=False), where the row entries of all
 * transformations are then one contiguous load each.  Replaces the same
 * reference lines as cpab_b200_build_A (cpab/pytorch/transformer.py:84-88,
 * :104-106); the transposed operand has no counterpart there.
 */
int cpab_b200_build_A_tt(int ndim, int64_t nC, int64_t d, int n_theta,
                         const int32_t *B_rowptr, const int32_t *B_colidx,
                         const float *B_vals, const float *theta_t, float dT,
                         float *As, float *trels, cpab_stream_t stream);

/*
 * order[s, :] = the points of set s (s < n_sets; points [n_sets, ndim, nP],
 * or [ndim, nP] with n_sets = 1) sorted by the cell that contains them
 * (counting sort; ties in arbitrary order).  Passing it to forward/backward
 * makes the threads of a warp start in the same or adjacent cells.
 * counts_scratch is caller-provided scratch of n_sets * nC int32; order is
 * [n_sets, nP] int32.  No counterpart in the reference (its kernels take the
 * points in storage order).
 */
int cpab_b200_order_points(int ndim, const int32_t *nc, const float *points,
                           int64_t nP, int n_sets, int32_t *counts_scratch,
                           int32_t *order, cpab_stream_t stream);

/*
 * cpab_b200_order_points without the counts_scratch argument, for callers that
 * cannot allocate device memory (a host that only hands over the buffers it
 * owns, code that must not risk the device-wide synchronization of
 * cudaMalloc/cudaFree, a fixed memory budget).  The counters live in a 4 MiB
 * array built into the library, present on every GPU that loads it; n_sets * nC
 * may not exceed 2^20 (CPAB_ERR_SIZE otherwise).  All calls on a device share
 * that array: calls whose GPU work overlaps race.  The first call on a device
 * looks up the array's device address, so make it before any stream capture;
 * the address is kept for the life of the process, so after cudaDeviceReset
 * (a new primary context) this entry point must not be used on that device.
 * No counterpart in the reference.
 */
int cpab_b200_order_points_static(int ndim, const int32_t *nc,
                                  const float *points, int64_t nP, int n_sets,
                                  int32_t *order, cpab_stream_t stream);

/*
 * cells[i] = index of the tessellation cell containing points[:, i]
 * (points [ndim, n]); outside the domain, the cell the integrators use there.
 * Replaces the device lookups cuda_findcellidx_{1D,2D,3D}_fast of
 * cpab/core/cpab_ops_1d.cu:90-97, cpab/core/cpab_ops_2d.cu:119-176 and
 * cpab/core/cpab_ops_3d.cu:67-131 (same rule, bit for bit).
 */
int cpab_b200_cell_index(int ndim, const int32_t *nc, const float *points,
                         int64_t n, int32_t *cells, cpab_stream_t stream);

/*
 * dtheta[t, j] = sum_i Bt[j, i] * moments[t, i] for the d x D CSR matrix
 * Bt = B^T.  dtheta is [n_theta, d] and is overwritten.
 * Replaces cpab/pytorch/transformer.py:165-166.
 */
int cpab_b200_project(int64_t d, int64_t D, int n_theta,
                      const int32_t *Bt_rowptr, const int32_t *Bt_colidx,
                      const float *Bt_vals, const float *moments,
                      float *dtheta, cpab_stream_t stream);

/*
 * cpab_b200_project with the moments given transposed, moments_t [D, n_theta]
 * (moments_t[i * n_theta + t] = moments[t, i]); same results.  For general
 * (dense) bases, whose columns spread over the whole domain.  Replaces
 * cpab/pytorch/transformer.py:165-166 like cpab_b200_project.
 */
int cpab_b200_project_tt(int64_t d, int64_t D, int n_theta,
                         const int32_t *Bt_rowptr, const int32_t *Bt_colidx,
                         const float *Bt_vals, const float *moments_t,
                         float *dtheta, cpab_stream_t stream);

/*
 * Linear / bilinear / trilinear resampling of data [n_batch, C, *in_size] at
 * grid [n_batch, ndim, P] (P = prod(out_size), coordinate 0 fastest; grid
 * coordinate k indexes data axis 2+k after scaling by in_size[k]-1, border
 * clamped).  out is [n_batch, C, *out_size].
 * Replaces cpab/pytorch/interpolation.py:8-160 (forward).
 */
int cpab_b200_interpolate(int ndim, const float *data, int n_batch,
                          int n_channels, const int64_t *in_size,
                          const float *grid, const int64_t *out_size,
                          float *out, cpab_stream_t stream);

/*
 * Backward of cpab_b200_interpolate.  grad_grid ([n_batch, ndim, P], may be
 * NULL) is overwritten; grad_data ([n_batch, C, *in_size], may be NULL) is
 * zeroed and then receives the scatter-add of the interpolation weights.
 * Replaces the torch autograd graph of cpab/pytorch/interpolation.py:8-160.
 */
int cpab_b200_interpolate_backward(int ndim, const float *data, int n_batch,
                                   int n_channels, const int64_t *in_size,
                                   const float *grid, const int64_t *out_size,
                                   const float *grad_out, float *grad_grid,
                                   float *grad_data, cpab_stream_t stream);

/*
 * Fused chain (2D/3D): n_stages transformations applied in sequence to every
 * point in one kernel -- transform_grid_chain (cpab/cpab.py:269-278) without
 * the per-stage launches and intermediate tensors.  trels and As are
 * [n_stages, n_theta, nC, ndim, ndim+1] (stage-major; cpab_b200_build_A over
 * n_stages * n_theta rows of theta produces this layout).  points as for
 * cpab_b200_forward (stage 0 input); out [n_theta, ndim, nP] is the last
 * stage's output.  stage_points ([n_stages-1, n_theta, ndim, nP], may be NULL
 * when n_stages = 1) receives the inputs of stages 1.. indexed by processing
 * slot (order[s] when order != NULL); the backward needs them and the same
 * order.  Each stage's arithmetic is exactly cpab_b200_forward's.
 */
int cpab_b200_forward_chain(int ndim, const int32_t *nc, const float *points,
                            int64_t nP, int points_batched, const int32_t *order,
                            const float *trels, const float *As, int n_stages,
                            int n_theta, int nstepsolver, int adaptive,
                            float *stage_points, float *out, cpab_stream_t stream);

/*
 * Backward of cpab_b200_forward_chain: the adjoint sweeps of all stages, last
 * to first, lambda flowing from each stage into the previous one (the
 * gradient the reference's autograd passes between its per-stage
 * backward_moments_and_points calls).  moments (16-byte aligned, zeroed
 * here) is [n_stages, n_theta, nC, ppc]; grad_points as for
 * cpab_b200_backward (lambda at the chain input), may be NULL.
 */
int cpab_b200_backward_chain(int ndim, const int32_t *nc, const float *points,
                             int64_t nP, int points_batched, const int32_t *order,
                             const float *As, int n_stages, int n_theta,
                             const float *grad_out, const float *stage_points,
                             int nstepsolver, int adaptive, float *moments,
                             float *grad_points, cpab_stream_t stream);

/*
 * Fused transform_data (2D/3D):
 *   out = interpolate(data, transform_grid(meshgrid, theta), out_size)
 * in one kernel, for n_theta transformations given by As/trels (as for
 * cpab_b200_forward).  The meshgrid is the uniform grid of out_size whose
 * axis values are mesh_axes (out_size[0] values of axis 0, then out_size[1]
 * of axis 1 [, then axis 2]: the linspace vectors uniform_meshgrid meshes).
 * data is [n_theta, n_channels, *in_size], out [n_theta, n_channels,
 * *out_size] (P = prod(out_size) points, last axis fastest).  order (may be
 * NULL): a permutation of the P output indices giving the processing order,
 * e.g. cpab_b200_order_points applied to the meshgrid's points listed in
 * output order (the cell-sorted order the Python package passes); the kernel's
 * thread slot s handles output point order[s].  grid_t receives the
 * integrated grid as [n_theta, ndim, P] indexed by slot, which the backward
 * (given the same order) needs.  Results equal the unfused composition of
 * cpab_b200_forward and cpab_b200_interpolate bit for bit, whatever the order.
 * Replaces cpab/cpab.py:306-308 (transform_grid of uniform_meshgrid, then
 * interpolate, cpab/pytorch/interpolation.py:47-160); the reference has no
 * single native counterpart.
 */
int cpab_b200_transform_data(int ndim, const int32_t *nc, const int64_t *out_size,
                             const float *mesh_axes, const int32_t *order,
                             const float *trels, const float *As,
                             int n_theta, int nstepsolver, int adaptive,
                             const float *data, int n_channels, const int64_t *in_size,
                             float *grid_t, float *out, cpab_stream_t stream);

/*
 * Backward of cpab_b200_transform_data: forms the gradient of the resample
 * with respect to the grid at grid_t (as cpab_b200_interpolate_backward) and
 * runs the adjoint sweep of cpab_b200_backward from it, in one kernel.
 * moments (16-byte aligned, zeroed here) as for cpab_b200_backward;
 * grad_data ([n_theta, n_channels, *in_size], may be NULL) is zeroed and
 * receives the resample's data gradient.
 */
int cpab_b200_transform_data_backward(int ndim, const int32_t *nc, const int64_t *out_size,
                                      const float *mesh_axes, const int32_t *order,
                                      const float *As, int n_theta,
                                      int nstepsolver, int adaptive,
                                      const float *data, int n_channels,
                                      const int64_t *in_size, const float *grid_t,
                                      const float *grad_out, float *moments,
                                      float *grad_data, cpab_stream_t stream);

/*
 * Fused spatial-transformer warp (2D/3D): the CpabWarp layer of the
 * reference's stn/stn.py:58-86,
 *   out = F.grid_sample(data, T_1 o ... o T_K(pixel grid),
 *                       align_corners=True, padding_mode),
 * in one kernel.  K = n_stages transformations act on every output pixel,
 * stage 0 first (the STN's T_K: its thetas reversed); As/trels are
 * [n_stages, n_theta, nC, ppc] as for cpab_b200_forward_chain.  The pixel
 * grid is the meshgrid of out_size whose axis values are mesh_axes, in CPAB
 * coordinates: (linspace(-1, 1, n) + 1) / 2 per axis (0.5 for a one-pixel
 * axis), the points stn/stn.py:43-46,80-82 build; CPAB coordinate k runs
 * along image axis k.  data is [n_theta, n_channels, *in_size]
 * (data_batched = 1) or one [n_channels, *in_size] image for all
 * transformations (data_batched = 0); out is [n_theta, n_channels,
 * *out_size].  padding_mode: 0 zeros, 1 border, 2 reflection (F.grid_sample's
 * modes).  order (may be NULL): processing order of the output pixels, as
 * for cpab_b200_transform_data.  stage_points ([n_stages-1, n_theta, ndim,
 * P], may be NULL when n_stages == 1) and grid_t ([n_theta, ndim, P], the
 * sampled positions) are written for the backward, both indexed by slot.
 * The reference has no single native counterpart: it calls
 * cpab/pytorch/transformer.py:28 once per transformation, then grid_sample.
 */
int cpab_b200_warp(int ndim, const int32_t *nc, const int64_t *out_size,
                   const float *mesh_axes, const int32_t *order, const float *trels,
                   const float *As, int n_stages, int n_theta, int nstepsolver,
                   int adaptive, const float *data, int data_batched, int n_channels,
                   const int64_t *in_size, int padding_mode, float *stage_points,
                   float *grid_t, float *out, cpab_stream_t stream);

/*
 * Backward of cpab_b200_warp: grid_sample's gradient with respect to the
 * sampled positions (and, when grad_data is non-NULL, the image), then the
 * adjoint sweeps of all stages, last to first, in one kernel.  moments
 * ([n_stages, n_theta, nC, ppc], 16-byte aligned) and grad_data (shaped like
 * data) are zeroed here; the same order, stage_points and grid_t as the
 * forward.
 */
int cpab_b200_warp_backward(int ndim, const int32_t *nc, const int64_t *out_size,
                            const float *mesh_axes, const int32_t *order, const float *As,
                            int n_stages, int n_theta, int nstepsolver, int adaptive,
                            const float *data, int data_batched, int n_channels,
                            const int64_t *in_size, int padding_mode,
                            const float *stage_points, const float *grid_t,
                            const float *grad_out, float *moments, float *grad_data,
                            cpab_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CPAB_B200_H */
