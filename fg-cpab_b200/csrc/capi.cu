// extern "C" entry points of libcpab_b200.so (declared in include/cpab_b200.h).
//
// Every entry point validates its arguments on the host, enqueues its kernels
// on the caller's stream and reports failures as a negative status plus a
// per-thread message -- it never exits the process (the reference's launchers
// call exit() on a CUDA error, cpab/pytorch/transformer_cuda.cu:12-18).
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdint>
#include <cstring>

#include "../../include/cpab_b200.h"
#include "launch.h"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = '\0';
  return CPAB_OK;
}

int cuda_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return ok();
  return fail(CPAB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Number of cells of an ndim tessellation; 0 when invalid.  Each axis is
// limited to 2^20 cells (the lookup's floor is exact below 2^22).
int64_t cell_count(int ndim, const int32_t *nc) {
  if (nc == nullptr) return 0;
  int64_t n = 1;
  for (int k = 0; k < ndim; ++k) {
    if (nc[k] < 1 || nc[k] > (1 << 20)) return 0;
    n *= nc[k];
  }
  return ndim == 1 ? n : (ndim == 2 ? 4 * n : 5 * n);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Checks shared by forward and backward; fills the geometry part of `a`.
int check_integrate(const char *fn, int ndim, const int32_t *nc, const float *points, int64_t nP,
                    int points_batched, const float *As, int n_theta, int nstepsolver,
                    int adaptive, cpab::IntegrateArgs &a) {
  if (ndim < 1 || ndim > 3) return fail(CPAB_ERR_ARG, "%s: ndim must be 1, 2 or 3, got %d", fn, ndim);
  const int64_t nC = cell_count(ndim, nc);
  if (nC <= 0) return fail(CPAB_ERR_ARG, "%s: tessellation sizes must be in [1, 2^20]", fn);
  if (nC > (1 << 26)) return fail(CPAB_ERR_SIZE, "%s: too many cells (%lld)", fn, (long long)nC);
  if (nP < 0) return fail(CPAB_ERR_ARG, "%s: negative number of points", fn);
  if (n_theta < 0 || n_theta > 65535)
    return fail(CPAB_ERR_SIZE, "%s: n_theta must be in [0, 65535], got %d", fn, n_theta);
  if (points_batched != 0 && points_batched != 1)
    return fail(CPAB_ERR_ARG, "%s: points_batched must be 0 or 1", fn);
  if (adaptive != 0 && adaptive != 1)
    return fail(CPAB_ERR_ARG, "%s: adaptive_substeps must be 0 or 1", fn);
  if (nstepsolver < 1)
    return fail(CPAB_ERR_STEPS, "%s: invalid nstepsolver=%d, expected nstepsolver > 0", fn,
                nstepsolver);
  if (nstepsolver > cpab::kMaxSteps)
    return fail(CPAB_ERR_STEPS, "%s: invalid nstepsolver=%d, at most %d steps are supported", fn,
                nstepsolver, cpab::kMaxSteps);
  if (nP > 0 && n_theta > 0 && (points == nullptr || As == nullptr))
    return fail(CPAB_ERR_ARG, "%s: null input pointer", fn);
  if (!aligned16(As)) return fail(CPAB_ERR_ARG, "%s: As must be 16-byte aligned", fn);
  a = cpab::IntegrateArgs{};
  a.ndim = ndim;
  a.tess = cpab::make_tess(ndim, nc);
  a.nC = (int)nC;
  a.points = points;
  a.nP = nP;
  a.batched = points_batched;
  a.As = As;
  a.n_theta = n_theta;
  a.T = nstepsolver;
  a.adaptive = adaptive;
  return CPAB_OK;
}

}  // namespace

int cpab::report_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

extern "C" {

int cpab_b200_version(void) { return 10000; }

int cpab_b200_max_steps(void) { return cpab::kMaxSteps; }

const char *cpab_b200_last_error(void) { return g_err; }

int cpab_b200_expm(int ndim, const float *As, int64_t n_matrices, float dT, float *trels,
                   cpab_stream_t stream) {
  if (ndim < 1 || ndim > 3) return fail(CPAB_ERR_ARG, "expm: ndim must be 1, 2 or 3, got %d", ndim);
  if (n_matrices < 0) return fail(CPAB_ERR_ARG, "expm: negative matrix count");
  if (n_matrices > 0 && (As == nullptr || trels == nullptr))
    return fail(CPAB_ERR_ARG, "expm: null pointer");
  return cuda_status(cpab::launch_expm(ndim, As, n_matrices, dT, trels, stream), "expm");
}

int cpab_b200_build_A(int ndim, int64_t nC, int64_t d, int n_theta, const int32_t *B_rowptr,
                      const int32_t *B_colidx, const float *B_vals, const float *theta, float dT,
                      float *As, float *trels, cpab_stream_t stream) {
  if (ndim < 1 || ndim > 3) return fail(CPAB_ERR_ARG, "build_A: ndim must be 1, 2 or 3");
  if (nC < 0 || d < 0 || n_theta < 0) return fail(CPAB_ERR_ARG, "build_A: negative size");
  if (nC * n_theta > 0 &&
      (B_rowptr == nullptr || As == nullptr || (d > 0 && (theta == nullptr || B_colidx == nullptr ||
                                                           B_vals == nullptr))))
    return fail(CPAB_ERR_ARG, "build_A: null pointer");
  return cuda_status(cpab::launch_build_A(ndim, nC, d, n_theta, B_rowptr, B_colidx, B_vals, theta,
                                          dT, As, trels, stream),
                     "build_A");
}

int cpab_b200_build_A_tt(int ndim, int64_t nC, int64_t d, int n_theta, const int32_t *B_rowptr,
                         const int32_t *B_colidx, const float *B_vals, const float *theta_t,
                         float dT, float *As, float *trels, cpab_stream_t stream) {
  if (ndim < 1 || ndim > 3) return fail(CPAB_ERR_ARG, "build_A_tt: ndim must be 1, 2 or 3");
  if (nC < 0 || d < 0 || n_theta < 0) return fail(CPAB_ERR_ARG, "build_A_tt: negative size");
  if (nC * n_theta > 0 &&
      (B_rowptr == nullptr || As == nullptr || (d > 0 && (theta_t == nullptr || B_colidx == nullptr ||
                                                           B_vals == nullptr))))
    return fail(CPAB_ERR_ARG, "build_A_tt: null pointer");
  return cuda_status(cpab::launch_build_A_tt(ndim, nC, n_theta, B_rowptr, B_colidx, B_vals,
                                             theta_t, dT, As, trels, stream),
                     "build_A_tt");
}

int cpab_b200_forward_1d_closed_form(const float *points, int64_t nP, int points_batched,
                                     const int32_t *order, const float *As, int n_theta, int ncx,
                                     float *out, cpab_stream_t stream) {
  cpab::IntegrateArgs a;
  const int32_t nc[1] = {ncx};
  int st = check_integrate("forward_1d_closed_form", 1, nc, points, nP, points_batched, As, n_theta,
                           1, 0, a);
  if (st != CPAB_OK) return st;
  if (nP == 0 || n_theta == 0) return ok();
  if (out == nullptr) return fail(CPAB_ERR_ARG, "forward_1d_closed_form: null output");
  a.out = out;
  a.order = order;
  return cuda_status(cpab::launch_forward_1d(a, stream), "forward_1d_closed_form");
}

int cpab_b200_forward(int ndim, const int32_t *nc, const float *points, int64_t nP,
                      int points_batched, const int32_t *order, const float *trels,
                      const float *As, int n_theta,
                      int nstepsolver, int adaptive, float *out, cpab_stream_t stream) {
  cpab::IntegrateArgs a;
  int st = check_integrate("forward", ndim, nc, points, nP, points_batched, As, n_theta,
                           nstepsolver, adaptive, a);
  if (st != CPAB_OK) return st;
  if (nP == 0 || n_theta == 0) return ok();
  if (out == nullptr) return fail(CPAB_ERR_ARG, "forward: null output");
  if (ndim > 1 && trels == nullptr) return fail(CPAB_ERR_ARG, "forward: null trels");
  if (!aligned16(trels)) return fail(CPAB_ERR_ARG, "forward: trels must be 16-byte aligned");
  a.trels = trels;
  a.out = out;
  a.order = order;
  return cuda_status(cpab::launch_forward(a, stream), "forward");
}

int cpab_b200_backward(int ndim, const int32_t *nc, const float *points, int64_t nP,
                       int points_batched, const int32_t *order, const float *As, int n_theta,
                       const float *grad_out,
                       int nstepsolver, int adaptive, float *moments, float *grad_points,
                       cpab_stream_t stream) {
  cpab::IntegrateArgs a;
  int st = check_integrate("backward", ndim, nc, points, nP, points_batched, As, n_theta,
                           nstepsolver, adaptive, a);
  if (st != CPAB_OK) return st;
  if (n_theta == 0) return ok();
  if (moments == nullptr) return fail(CPAB_ERR_ARG, "backward: null moments");
  if (!aligned16(moments)) return fail(CPAB_ERR_ARG, "backward: moments must be 16-byte aligned");
  if (nP > 0 && grad_out == nullptr) return fail(CPAB_ERR_ARG, "backward: null grad_out");
  const size_t mbytes = (size_t)n_theta * a.nC * ndim * (ndim + 1) * sizeof(float);
  cudaError_t e = cudaMemsetAsync(moments, 0, mbytes, stream);
  if (e != cudaSuccess) return cuda_status(e, "backward: clearing moments");
  if (nP == 0) return ok();
  a.grad_out = grad_out;
  a.moments = moments;
  a.grad_points = grad_points;
  a.order = order;
  return cuda_status(cpab::launch_backward(a, stream), "backward");
}

int cpab_b200_forward_chain(int ndim, const int32_t *nc, const float *points, int64_t nP,
                            int points_batched, const int32_t *order, const float *trels,
                            const float *As, int n_stages, int n_theta, int nstepsolver,
                            int adaptive, float *stage_points, float *out, cpab_stream_t stream) {
  cpab::IntegrateArgs a;
  int st = check_integrate("forward_chain", ndim, nc, points, nP, points_batched, As, n_theta,
                           nstepsolver, adaptive, a);
  if (st != CPAB_OK) return st;
  if (ndim == 1) return fail(CPAB_ERR_ARG, "forward_chain: ndim must be 2 or 3");
  if (n_stages < 1 || n_stages > 4096)
    return fail(CPAB_ERR_ARG, "forward_chain: n_stages must be in [1, 4096], got %d", n_stages);
  if (nP == 0 || n_theta == 0) return ok();
  if (trels == nullptr || !aligned16(trels))
    return fail(CPAB_ERR_ARG, "forward_chain: trels must be non-null and 16-byte aligned");
  if (out == nullptr || (n_stages > 1 && stage_points == nullptr))
    return fail(CPAB_ERR_ARG, "forward_chain: null output");
  a.trels = trels;
  a.out = out;
  a.order = order;
  a.n_stages = n_stages;
  a.stage_points = stage_points;
  return cuda_status(cpab::launch_forward(a, stream), "forward_chain");
}

int cpab_b200_backward_chain(int ndim, const int32_t *nc, const float *points, int64_t nP,
                             int points_batched, const int32_t *order, const float *As,
                             int n_stages, int n_theta, const float *grad_out,
                             const float *stage_points, int nstepsolver, int adaptive,
                             float *moments, float *grad_points, cpab_stream_t stream) {
  cpab::IntegrateArgs a;
  int st = check_integrate("backward_chain", ndim, nc, points, nP, points_batched, As, n_theta,
                           nstepsolver, adaptive, a);
  if (st != CPAB_OK) return st;
  if (ndim == 1) return fail(CPAB_ERR_ARG, "backward_chain: ndim must be 2 or 3");
  if (n_stages < 1 || n_stages > 4096)
    return fail(CPAB_ERR_ARG, "backward_chain: n_stages must be in [1, 4096], got %d", n_stages);
  if (n_theta == 0) return ok();
  if (moments == nullptr || !aligned16(moments))
    return fail(CPAB_ERR_ARG, "backward_chain: moments must be non-null and 16-byte aligned");
  if (nP > 0 && (grad_out == nullptr || (n_stages > 1 && stage_points == nullptr)))
    return fail(CPAB_ERR_ARG, "backward_chain: null grad_out or stage_points");
  const size_t mbytes =
      (size_t)n_stages * n_theta * a.nC * ndim * (ndim + 1) * sizeof(float);
  cudaError_t e = cudaMemsetAsync(moments, 0, mbytes, stream);
  if (e != cudaSuccess) return cuda_status(e, "backward_chain: clearing moments");
  if (nP == 0) return ok();
  a.grad_out = grad_out;
  a.moments = moments;
  a.grad_points = grad_points;
  a.order = order;
  a.n_stages = n_stages;
  a.stage_points = const_cast<float *>(stage_points);
  return cuda_status(cpab::launch_backward(a, stream), "backward_chain");
}

int cpab_b200_order_points(int ndim, const int32_t *nc, const float *points, int64_t nP,
                           int n_sets, int32_t *counts_scratch, int32_t *order,
                           cpab_stream_t stream) {
  if (ndim < 1 || ndim > 3) return fail(CPAB_ERR_ARG, "order_points: ndim must be 1, 2 or 3");
  const int64_t nC = cell_count(ndim, nc);
  if (nC <= 0) return fail(CPAB_ERR_ARG, "order_points: tessellation sizes must be in [1, 2^20]");
  // Same cell limit as the integrators; the kernels index cells with int.
  if (nC > (1 << 26))
    return fail(CPAB_ERR_SIZE, "order_points: too many cells (%lld)", (long long)nC);
  if (nP < 0 || n_sets < 0) return fail(CPAB_ERR_ARG, "order_points: negative size");
  if (n_sets > 65535) return fail(CPAB_ERR_SIZE, "order_points: more than 65535 point sets");
  if (nP > INT32_MAX) return fail(CPAB_ERR_SIZE, "order_points: more than 2^31-1 points");
  if (nP > 0 && n_sets > 0 && (points == nullptr || counts_scratch == nullptr || order == nullptr))
    return fail(CPAB_ERR_ARG, "order_points: null pointer");
  return cuda_status(cpab::launch_order_points(ndim, cpab::make_tess(ndim, nc), points, nP, n_sets,
                                               (int)nC, counts_scratch, order, stream),
                     "order_points");
}

int cpab_b200_cell_index(int ndim, const int32_t *nc, const float *points, int64_t n,
                         int32_t *cells, cpab_stream_t stream) {
  if (ndim < 1 || ndim > 3) return fail(CPAB_ERR_ARG, "cell_index: ndim must be 1, 2 or 3");
  if (cell_count(ndim, nc) <= 0) return fail(CPAB_ERR_ARG, "cell_index: tessellation sizes must be in [1, 2^20]");
  if (n < 0) return fail(CPAB_ERR_ARG, "cell_index: negative number of points");
  if (n > 0 && (points == nullptr || cells == nullptr)) return fail(CPAB_ERR_ARG, "cell_index: null pointer");
  return cuda_status(cpab::launch_cell_index(ndim, cpab::make_tess(ndim, nc), points, n, cells, stream),
                     "cell_index");
}

int cpab_b200_project(int64_t d, int64_t D, int n_theta, const int32_t *Bt_rowptr,
                      const int32_t *Bt_colidx, const float *Bt_vals, const float *moments,
                      float *dtheta, cpab_stream_t stream) {
  if (d < 0 || D < 0 || n_theta < 0) return fail(CPAB_ERR_ARG, "project: negative size");
  if (d * n_theta > 0 && (Bt_rowptr == nullptr || dtheta == nullptr ||
                          (D > 0 && (moments == nullptr || Bt_colidx == nullptr ||
                                     Bt_vals == nullptr))))
    return fail(CPAB_ERR_ARG, "project: null pointer");
  return cuda_status(
      cpab::launch_project(d, D, n_theta, Bt_rowptr, Bt_colidx, Bt_vals, moments, dtheta, stream),
      "project");
}

int cpab_b200_project_tt(int64_t d, int64_t D, int n_theta, const int32_t *Bt_rowptr,
                         const int32_t *Bt_colidx, const float *Bt_vals, const float *moments_t,
                         float *dtheta, cpab_stream_t stream) {
  if (d < 0 || D < 0 || n_theta < 0) return fail(CPAB_ERR_ARG, "project_tt: negative size");
  if (d * n_theta > 0 && (Bt_rowptr == nullptr || dtheta == nullptr ||
                          (D > 0 && (moments_t == nullptr || Bt_colidx == nullptr ||
                                     Bt_vals == nullptr))))
    return fail(CPAB_ERR_ARG, "project_tt: null pointer");
  return cuda_status(cpab::launch_project_tt(d, n_theta, Bt_rowptr, Bt_colidx, Bt_vals, moments_t,
                                             dtheta, stream),
                     "project_tt");
}

}  // extern "C"

namespace {

int check_resample(const char *fn, int ndim, const float *data, int n_batch, int n_channels,
                   const int64_t *in_size, const float *grid, const int64_t *out_size,
                   cpab::ResampleArgs &a) {
  if (ndim < 1 || ndim > 3) return fail(CPAB_ERR_ARG, "%s: ndim must be 1, 2 or 3, got %d", fn, ndim);
  if (n_batch < 0 || n_channels < 0) return fail(CPAB_ERR_ARG, "%s: negative batch/channels", fn);
  if (in_size == nullptr || out_size == nullptr) return fail(CPAB_ERR_ARG, "%s: null sizes", fn);
  int64_t P = 1;
  for (int k = 0; k < ndim; ++k) {
    if (in_size[k] < 1) return fail(CPAB_ERR_ARG, "%s: input sizes must be positive", fn);
    if (in_size[k] > (1 << 24))
      return fail(CPAB_ERR_SIZE, "%s: input axis %d longer than 2^24", fn, k);
    if (out_size[k] < 0) return fail(CPAB_ERR_ARG, "%s: negative output size", fn);
    P *= out_size[k];
  }
  if (n_batch > 65535) return fail(CPAB_ERR_SIZE, "%s: batch larger than 65535", fn);
  int64_t plane = 1;
  for (int k = 0; k < ndim; ++k) plane *= in_size[k];
  if (plane >= ((int64_t)1 << 31))
    return fail(CPAB_ERR_SIZE, "%s: one input channel has 2^31 or more elements", fn);
  if (ndim >= 2 && (out_size[0] + 31) / 32 > 65535)
    return fail(CPAB_ERR_SIZE, "%s: output axis 0 too long", fn);
  if (ndim == 3 && (int64_t)n_batch * out_size[1] > 65535)
    return fail(CPAB_ERR_SIZE, "%s: batch * out_size[1] larger than 65535", fn);
  if (P > 0 && n_batch > 0 && n_channels > 0 && (data == nullptr || grid == nullptr))
    return fail(CPAB_ERR_ARG, "%s: null input pointer", fn);
  a = cpab::ResampleArgs{};
  a.ndim = ndim;
  a.data = data;
  a.n_batch = n_batch;
  a.n_channels = n_channels;
  a.grid = grid;
  for (int k = 0; k < 3; ++k) {
    a.in_size[k] = k < ndim ? in_size[k] : 1;
    a.out_size[k] = k < ndim ? out_size[k] : 1;
  }
  return CPAB_OK;
}

// Checks of the fused transform_data calls; fills `a` (integration over the
// meshgrid) and `m`.
int check_mesh(const char *fn, int ndim, const int32_t *nc, const int64_t *out_size,
               const float *mesh_axes, const int32_t *order, const float *As, int n_theta,
               int nstepsolver,
               int adaptive, const float *data, int n_channels, const int64_t *in_size,
               const float *grid_t, cpab::IntegrateArgs &a, cpab::MeshArgs &m) {
  if (ndim != 2 && ndim != 3)
    return fail(CPAB_ERR_ARG, "%s: ndim must be 2 or 3, got %d", fn, ndim);
  if (out_size == nullptr || in_size == nullptr) return fail(CPAB_ERR_ARG, "%s: null sizes", fn);
  int64_t P = 1, plane = 1;
  for (int k = 0; k < ndim; ++k) {
    if (out_size[k] < 0) return fail(CPAB_ERR_ARG, "%s: negative output size", fn);
    if (in_size[k] < 1) return fail(CPAB_ERR_ARG, "%s: input sizes must be positive", fn);
    if (in_size[k] > (1 << 24))
      return fail(CPAB_ERR_SIZE, "%s: input axis %d longer than 2^24", fn, k);
    P *= out_size[k];
    plane *= in_size[k];
  }
  if (P >= ((int64_t)1 << 31))
    return fail(CPAB_ERR_SIZE, "%s: 2^31 or more output points", fn);
  if (plane >= ((int64_t)1 << 31))
    return fail(CPAB_ERR_SIZE, "%s: one input channel has 2^31 or more elements", fn);
  if (n_channels < 0) return fail(CPAB_ERR_ARG, "%s: negative channel count", fn);
  // The meshgrid is shared by all transformations: not batched.
  int st = check_integrate(fn, ndim, nc, mesh_axes, P, 0, As, n_theta, nstepsolver, adaptive, a);
  if (st != CPAB_OK) return st;
  if (P > 0 && n_theta > 0 && (grid_t == nullptr || (n_channels > 0 && data == nullptr)))
    return fail(CPAB_ERR_ARG, "%s: null grid_t or data", fn);
  a.points = nullptr;
  m = cpab::MeshArgs{};
  for (int k = 0; k < 3; ++k) {
    m.out_size[k] = k < ndim ? out_size[k] : 1;
    m.in_size[k] = k < ndim ? (int)in_size[k] : 1;
  }
  m.axes = mesh_axes;
  m.order = order;
  m.data = data;
  m.C = n_channels;
  m.grid_t = const_cast<float *>(grid_t);
  return CPAB_OK;
}

}  // namespace

extern "C" {

int cpab_b200_transform_data(int ndim, const int32_t *nc, const int64_t *out_size,
                             const float *mesh_axes, const int32_t *order,
                             const float *trels, const float *As,
                             int n_theta, int nstepsolver, int adaptive, const float *data,
                             int n_channels, const int64_t *in_size, float *grid_t, float *out,
                             cpab_stream_t stream) {
  cpab::IntegrateArgs a;
  cpab::MeshArgs m;
  int st = check_mesh("transform_data", ndim, nc, out_size, mesh_axes, order, As, n_theta,
                      nstepsolver,
                      adaptive, data, n_channels, in_size, grid_t, a, m);
  if (st != CPAB_OK) return st;
  if (n_theta == 0 || a.nP == 0) return ok();
  if (trels == nullptr || !aligned16(trels))
    return fail(CPAB_ERR_ARG, "transform_data: trels must be non-null and 16-byte aligned");
  if (out == nullptr && n_channels > 0) return fail(CPAB_ERR_ARG, "transform_data: null output");
  a.trels = trels;
  m.out = out;
  return cuda_status(cpab::launch_transform_data(a, m, stream), "transform_data");
}

int cpab_b200_transform_data_backward(int ndim, const int32_t *nc, const int64_t *out_size,
                                      const float *mesh_axes, const int32_t *order,
                                      const float *As, int n_theta,
                                      int nstepsolver, int adaptive, const float *data,
                                      int n_channels, const int64_t *in_size,
                                      const float *grid_t, const float *grad_out,
                                      float *moments, float *grad_data, cpab_stream_t stream) {
  cpab::IntegrateArgs a;
  cpab::MeshArgs m;
  int st = check_mesh("transform_data_backward", ndim, nc, out_size, mesh_axes, order, As,
                      n_theta,
                      nstepsolver, adaptive, data, n_channels, in_size, grid_t, a, m);
  if (st != CPAB_OK) return st;
  if (n_theta == 0) return ok();
  if (moments == nullptr || !aligned16(moments))
    return fail(CPAB_ERR_ARG, "transform_data_backward: moments must be non-null and 16-byte aligned");
  if (grad_out == nullptr && a.nP > 0 && n_channels > 0)
    return fail(CPAB_ERR_ARG, "transform_data_backward: null grad_out");
  const size_t mbytes = (size_t)n_theta * a.nC * ndim * (ndim + 1) * sizeof(float);
  cudaError_t e = cudaMemsetAsync(moments, 0, mbytes, stream);
  if (e != cudaSuccess) return cuda_status(e, "transform_data_backward: clearing moments");
  if (grad_data != nullptr) {
    int64_t vol = 1;
    for (int k = 0; k < ndim; ++k) vol *= in_size[k];
    e = cudaMemsetAsync(grad_data, 0, (size_t)n_theta * n_channels * vol * sizeof(float), stream);
    if (e != cudaSuccess) return cuda_status(e, "transform_data_backward: clearing grad_data");
  }
  if (a.nP == 0 || n_channels == 0) return ok();  // zero upstream gradient
  m.grad_out = grad_out;
  m.grad_data = grad_data;
  a.moments = moments;
  return cuda_status(cpab::launch_transform_data_backward(a, m, stream), "transform_data_backward");
}

namespace {

// Arguments shared by cpab_b200_warp and cpab_b200_warp_backward, on top of
// check_mesh's: the chain length, the stage buffer, the padding mode and
// whether every transformation has its own image.
int check_warp(const char *fn, int n_stages, const float *stage_points, int data_batched,
               int padding_mode, cpab::IntegrateArgs &a, cpab::MeshArgs &m) {
  if (n_stages < 1 || n_stages > 4096)
    return fail(CPAB_ERR_ARG, "%s: n_stages must be in [1, 4096], got %d", fn, n_stages);
  if (data_batched != 0 && data_batched != 1)
    return fail(CPAB_ERR_ARG, "%s: data_batched must be 0 or 1", fn);
  if (padding_mode != cpab::kPadZeros && padding_mode != cpab::kPadBorder &&
      padding_mode != cpab::kPadReflection)
    return fail(CPAB_ERR_ARG, "%s: padding_mode must be 0 (zeros), 1 (border) or 2 (reflection)",
                fn);
  if (n_stages > 1 && a.nP > 0 && a.n_theta > 0 && stage_points == nullptr)
    return fail(CPAB_ERR_ARG, "%s: null stage_points with %d stages", fn, n_stages);
  const int64_t plane = (int64_t)m.in_size[0] * m.in_size[1] * m.in_size[2];
  a.n_stages = n_stages;
  a.stage_points = const_cast<float *>(stage_points);
  m.data_bstride = data_batched ? (int64_t)m.C * plane : 0;
  m.padding = padding_mode;
  return CPAB_OK;
}

}  // namespace

int cpab_b200_warp(int ndim, const int32_t *nc, const int64_t *out_size, const float *mesh_axes,
                   const int32_t *order, const float *trels, const float *As, int n_stages,
                   int n_theta, int nstepsolver, int adaptive, const float *data,
                   int data_batched, int n_channels, const int64_t *in_size, int padding_mode,
                   float *stage_points, float *grid_t, float *out, cpab_stream_t stream) {
  cpab::IntegrateArgs a;
  cpab::MeshArgs m;
  int st = check_mesh("warp", ndim, nc, out_size, mesh_axes, order, As, n_theta, nstepsolver,
                      adaptive, data, n_channels, in_size, grid_t, a, m);
  if (st != CPAB_OK) return st;
  st = check_warp("warp", n_stages, stage_points, data_batched, padding_mode, a, m);
  if (st != CPAB_OK) return st;
  if (n_theta == 0 || a.nP == 0) return ok();
  if (trels == nullptr || !aligned16(trels))
    return fail(CPAB_ERR_ARG, "warp: trels must be non-null and 16-byte aligned");
  if (out == nullptr && n_channels > 0) return fail(CPAB_ERR_ARG, "warp: null output");
  a.trels = trels;
  m.out = out;
  return cuda_status(cpab::launch_warp(a, m, stream), "warp");
}

int cpab_b200_warp_backward(int ndim, const int32_t *nc, const int64_t *out_size,
                            const float *mesh_axes, const int32_t *order, const float *As,
                            int n_stages, int n_theta, int nstepsolver, int adaptive,
                            const float *data, int data_batched, int n_channels,
                            const int64_t *in_size, int padding_mode, const float *stage_points,
                            const float *grid_t, const float *grad_out, float *moments,
                            float *grad_data, cpab_stream_t stream) {
  cpab::IntegrateArgs a;
  cpab::MeshArgs m;
  int st = check_mesh("warp_backward", ndim, nc, out_size, mesh_axes, order, As, n_theta,
                      nstepsolver, adaptive, data, n_channels, in_size, grid_t, a, m);
  if (st != CPAB_OK) return st;
  st = check_warp("warp_backward", n_stages, stage_points, data_batched, padding_mode, a, m);
  if (st != CPAB_OK) return st;
  if (n_theta == 0) return ok();
  if (moments == nullptr || !aligned16(moments))
    return fail(CPAB_ERR_ARG, "warp_backward: moments must be non-null and 16-byte aligned");
  if (grad_out == nullptr && a.nP > 0 && n_channels > 0)
    return fail(CPAB_ERR_ARG, "warp_backward: null grad_out");
  const size_t mbytes = (size_t)n_stages * n_theta * a.nC * ndim * (ndim + 1) * sizeof(float);
  cudaError_t e = cudaMemsetAsync(moments, 0, mbytes, stream);
  if (e != cudaSuccess) return cuda_status(e, "warp_backward: clearing moments");
  if (grad_data != nullptr) {
    const int64_t images = data_batched ? n_theta : 1;
    const int64_t plane = (int64_t)m.in_size[0] * m.in_size[1] * m.in_size[2];
    e = cudaMemsetAsync(grad_data, 0, (size_t)(images * n_channels * plane) * sizeof(float),
                        stream);
    if (e != cudaSuccess) return cuda_status(e, "warp_backward: clearing grad_data");
  }
  if (a.nP == 0 || n_channels == 0) return ok();  // zero upstream gradient
  m.grad_out = grad_out;
  m.grad_data = grad_data;
  a.moments = moments;
  return cuda_status(cpab::launch_warp_backward(a, m, stream), "warp_backward");
}

int cpab_b200_interpolate(int ndim, const float *data, int n_batch, int n_channels,
                          const int64_t *in_size, const float *grid, const int64_t *out_size,
                          float *out, cpab_stream_t stream) {
  cpab::ResampleArgs a;
  int st = check_resample("interpolate", ndim, data, n_batch, n_channels, in_size, grid, out_size, a);
  if (st != CPAB_OK) return st;
  a.out = out;
  if (out == nullptr && n_batch > 0 && n_channels > 0)
    return fail(CPAB_ERR_ARG, "interpolate: null output");
  return cuda_status(cpab::launch_interpolate(a, stream), "interpolate");
}

int cpab_b200_interpolate_backward(int ndim, const float *data, int n_batch, int n_channels,
                                   const int64_t *in_size, const float *grid,
                                   const int64_t *out_size, const float *grad_out,
                                   float *grad_grid, float *grad_data, cpab_stream_t stream) {
  cpab::ResampleArgs a;
  int st = check_resample("interpolate_backward", ndim, data, n_batch, n_channels, in_size, grid,
                          out_size, a);
  if (st != CPAB_OK) return st;
  if (grad_out == nullptr && n_batch > 0 && n_channels > 0)
    return fail(CPAB_ERR_ARG, "interpolate_backward: null grad_out");
  a.grad_out = grad_out;
  a.grad_grid = grad_grid;
  a.grad_data = grad_data;
  if (grad_data != nullptr) {
    int64_t vol = 1;
    for (int k = 0; k < ndim; ++k) vol *= in_size[k];
    const size_t bytes = (size_t)n_batch * n_channels * vol * sizeof(float);
    cudaError_t e = cudaMemsetAsync(grad_data, 0, bytes, stream);
    if (e != cudaSuccess) return cuda_status(e, "interpolate_backward: clearing grad_data");
  }
  if (grad_grid != nullptr && n_channels == 0) {
    int64_t P = 1;
    for (int k = 0; k < ndim; ++k) P *= out_size[k];
    cudaError_t e =
        cudaMemsetAsync(grad_grid, 0, (size_t)n_batch * ndim * P * sizeof(float), stream);
    if (e != cudaSuccess) return cuda_status(e, "interpolate_backward: clearing grad_grid");
    return ok();
  }
  return cuda_status(cpab::launch_interpolate_backward(a, stream), "interpolate_backward");
}

}  // extern "C"
