// Internal launch interface between the C ABI layer (capi.cu) and the kernel
// translation units.  Arguments here are already validated.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cpab_device.cuh"

namespace cpab {

struct IntegrateArgs {
  int ndim;
  Tess tess;
  int nC;
  const float *points;  // [ndim, nP] or [n_theta, ndim, nP]
  int64_t nP;
  int batched;
  const float *trels;   // [n_theta, nC, ppc] (forward 2D/3D)
  const float *As;      // [n_theta, nC, ppc]
  int n_theta;
  int T;                // nstepsolver
  int adaptive;
  const float *grad_out;  // backward: [n_theta, ndim, nP]
  float *out;             // forward: [n_theta, ndim, nP]
  float *moments;         // backward: [n_theta, nC, ppc]
  float *grad_points;     // backward: [n_theta, ndim, nP] or nullptr
  const int32_t *order;   // processing order [1 or n_theta, nP] or nullptr
  // Fused chains (2D/3D): n_stages transformations applied in sequence to
  // every point.  trels, As and moments are then [n_stages, n_theta, nC, ppc];
  // stage_points holds the inputs of stages 1..n_stages-1 as
  // [n_stages-1, n_theta, ndim, nP] indexed by processing slot (written by the
  // forward, read by the backward with the same order).
  int n_stages = 1;
  float *stage_points = nullptr;
};

// Fused transform_data: the points are the uniform meshgrid of out_size (axis
// values given), processed in output order o = i0*n1 + i1 (+ i2 fastest in
// 3D); the integrated grid is resampled into data's shape in the same kernel.
struct MeshArgs {
  int64_t out_size[3];
  const float *axes;       // meshgrid values: axis 0, then axis 1 (, axis 2)
  const float *data;       // [n_theta, C, *in_size]
  int C;
  int in_size[3];
  const int32_t *order;    // processing order of the output points [P], or nullptr
  float *grid_t;           // [n_theta, ndim, P] in processing order (forward out, backward in)
  float *out;              // forward: [n_theta, C, P]
  const float *grad_out;   // backward: [n_theta, C, P]
  float *grad_data;        // backward, may be null (zeroed by the caller)
  // Spatial-transformer warp (warp.cu) only: elements between the images of
  // consecutive transformations in data / grad_data (0: one image shared by
  // all), and F.grid_sample's padding mode (kPadZeros, kPadBorder,
  // kPadReflection).
  int64_t data_bstride;
  int padding;
};

enum : int { kPadZeros = 0, kPadBorder = 1, kPadReflection = 2 };

// Each returns cudaSuccess or the launch error.
cudaError_t launch_transform_data(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s);
cudaError_t launch_transform_data_backward(const IntegrateArgs &a, const MeshArgs &m,
                                           cudaStream_t s);
// Spatial-transformer warp: chains of a.n_stages stages over the meshgrid,
// sampled as F.grid_sample(align_corners=True) samples (warp.cu).
cudaError_t launch_warp(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s);
cudaError_t launch_warp_backward(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s);
cudaError_t launch_forward(const IntegrateArgs &a, cudaStream_t s);
cudaError_t launch_forward_1d(const IntegrateArgs &a, cudaStream_t s);
cudaError_t launch_backward(const IntegrateArgs &a, cudaStream_t s);

cudaError_t launch_order_points(int ndim, Tess t, const float *points, int64_t nP, int n_sets,
                                int nC, int32_t *counts, int32_t *order, cudaStream_t s);
cudaError_t launch_cell_index(int ndim, Tess t, const float *points, int64_t n, int32_t *cells,
                              cudaStream_t s);
cudaError_t launch_expm(int ndim, const float *As, int64_t n, float dT, float *trels,
                        cudaStream_t s);
cudaError_t launch_build_A(int ndim, int64_t nC, int64_t d, int n_theta, const int32_t *rowptr,
                           const int32_t *colidx, const float *vals, const float *theta,
                           float dT, float *As, float *trels, cudaStream_t s);
cudaError_t launch_build_A_tt(int ndim, int64_t nC, int n_theta, const int32_t *rowptr,
                              const int32_t *colidx, const float *vals, const float *theta_t,
                              float dT, float *As, float *trels, cudaStream_t s);
cudaError_t launch_project_tt(int64_t d, int n_theta, const int32_t *rowptr,
                              const int32_t *colidx, const float *vals, const float *moments_t,
                              float *dtheta, cudaStream_t s);
cudaError_t launch_project(int64_t d, int64_t D, int n_theta, const int32_t *rowptr,
                           const int32_t *colidx, const float *vals, const float *moments,
                           float *dtheta, cudaStream_t s);

struct ResampleArgs {
  int ndim;
  const float *data;
  int n_batch, n_channels;
  int64_t in_size[3];
  const float *grid;
  int64_t out_size[3];
  float *out;              // forward
  const float *grad_out;   // backward
  float *grad_grid;        // backward, may be null
  float *grad_data;        // backward, may be null (zeroed by the caller)
};

cudaError_t launch_interpolate(const ResampleArgs &a, cudaStream_t s);
cudaError_t launch_interpolate_backward(const ResampleArgs &a, cudaStream_t s);

// Record an error for cpab_b200_last_error() (this host thread) and return code.
int report_error(int code, const char *fmt, ...);

// Device properties cached per device (SM count, opt-in shared memory).
struct DeviceInfo {
  int sm_count;
  int max_smem_optin;
};
const DeviceInfo &device_info();

}  // namespace cpab
