// ref_shim.cu -- C ABI over the reference's CUDA kernels (TEST INFRASTRUCTURE).
//
// Built by oracle/build_oracle.py together with the reference's unmodified
// cpab/core/cpab_ops_{1,2,3}d.cu into oracle/_ref/libcpab_ref.so.  Each entry
// point launches the reference kernel with the reference launcher's geometry
// (cpab/pytorch/transformer_cuda.cu:50-51, 107-108, 135-136, 199-200, 295-296:
// grid (ceil(nP/256), batch), 256 threads, legacy default stream) and returns
// the cudaError_t of the launch.  Outputs are caller-allocated; moments must be
// zeroed by the caller (the reference allocates them with torch::zeros).
#include <cuda_runtime.h>

#include "cpab_ops_1d.cuh"
#include "cpab_ops_2d.cuh"
#include "cpab_ops_3d.cuh"

namespace {
inline unsigned tiles(int n) { return (unsigned)((n + 255) / 256); }
}  // namespace

extern "C" {

int ref_max_steps(void) { return CPAB_MAX_STEPS; }

int ref_expm(int ndim, const float *As, int n, float dT, float *out) {
  if (n <= 0) return 0;
  if (ndim == 1) cpab_cuda_kernel_expm2x2<<<tiles(n), 256>>>(n, dT, out, As);
  else if (ndim == 2) cpab_cuda_kernel_expm3x3<<<tiles(n), 256>>>(n, dT, out, As);
  else cpab_cuda_kernel_expm4x4<<<tiles(n), 256>>>(n, dT, out, As);
  return (int)cudaGetLastError();
}

int ref_forward(int ndim, int nx, int ny, int nz, const float *pts, int nP, int broadcast,
                const float *trels, const float *As, int batch, int T, int adaptive, float *out) {
  if (nP <= 0 || batch <= 0) return 0;
  const dim3 grid(tiles(nP), batch), block(256, 1);
  if (ndim == 1)
    cpab_cuda_kernel_forward_1D_closed_form<<<grid, block>>>(nP, batch, out, pts, As, nx, broadcast);
  else if (ndim == 2)
    cpab_cuda_kernel_forward_2D_optimized<<<grid, block>>>(nP, batch, out, pts, trels, As, T, nx, ny,
                                                           adaptive, broadcast);
  else
    cpab_cuda_kernel_forward_3D_optimized<<<grid, block>>>(nP, batch, out, pts, trels, As, T, nx, ny,
                                                           nz, adaptive, broadcast);
  return (int)cudaGetLastError();
}

int ref_backward(int ndim, int nx, int ny, int nz, int nC, const float *pts, int nP, int broadcast,
                 const float *As, int n_theta, const float *grad, int T, int adaptive,
                 float *moments, float *grad_points) {
  if (nP <= 0 || n_theta <= 0) return 0;
  const dim3 grid(tiles(nP), n_theta), block(256, 1);
  if (ndim == 1)
    cpab_cuda_kernel_fused_backward_1D<<<grid, block>>>(nP, n_theta, nC, T, moments, grad_points,
                                                        grad, pts, As, nx, adaptive, broadcast);
  else if (ndim == 2)
    cpab_cuda_kernel_fused_backward<<<grid, block>>>(nP, n_theta, nC, T, moments, grad_points, grad,
                                                     pts, As, nx, ny, adaptive, broadcast);
  else
    cpab_cuda_kernel_fused_backward_3D<<<grid, block>>>(nP, n_theta, nC, T, moments, grad_points,
                                                        grad, pts, As, nx, ny, nz, adaptive,
                                                        broadcast);
  return (int)cudaGetLastError();
}

int ref_synchronize(void) { return (int)cudaDeviceSynchronize(); }

}  // extern "C"
