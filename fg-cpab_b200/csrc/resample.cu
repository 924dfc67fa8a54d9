// Linear / bilinear / trilinear resampling on a warped grid, forward and
// backward, replacing the ~20 unfused torch ops (and int64 index tensors) of
// cpab/pytorch/interpolation.py:8-160 with one kernel each way.
//
// Semantics kept from the reference: grid coordinate k is scaled by
// (in_size[k]-1), the lower corner is floor() clamped to [0, in_size[k]-1],
// the upper corner floor()+1 clamped likewise, and the weight is measured from
// the clamped lower corner.  The interpolation arithmetic is evaluated with
// explicitly rounded mul/add in the reference's order, so forward values are
// bit-identical to the torch expression.
//
// Layout: grid points are ordered with coordinate 0 fastest
// (p = i0 + n0*i1 [+ n0*n1*i2]) while the output is [B, C, n0, n1(, n2)] with
// the LAST axis fastest.  Each block therefore handles a 32x32 tile of
// (i0, i_last) and transposes through shared memory so that both the grid
// reads and the output writes are coalesced.
#include <cuda_runtime.h>

#include "launch.h"
#include "resample_device.cuh"

namespace cpab {

namespace {

using namespace rs;

constexpr int kTile = 32;
constexpr int kRows = 8;

// ----------------------------------------------------------------------------
// Kernels.  Output index space: [B, C, n0, ..., n_last] with the last axis
// fastest; grid points: p = i0 + n0*(i1 + n1*i2), coordinate 0 fastest.  A
// block handles a 32x32 tile of (i0, i_last) at fixed middle index i1 (3D)
// and transposes the grid (forward) or d grid (backward) through shared
// memory; ND == 1 needs no transpose (n_last == n0).
// ----------------------------------------------------------------------------

// MODE 0: forward; 1: backward to the grid only; 2: backward to grid and data
// (a separate instantiation, so the common grid-only backward carries no
// scatter code).
template <int ND, int MODE>
__device__ __forceinline__ void interp_body(const ResampleArgs &a) {
  __shared__ float sg[ND][kTile][kTile + 1];  // [i_last local][i0 local]
  const int C = a.n_channels;
  const int in[3] = {(int)a.in_size[0], (int)a.in_size[1], (int)a.in_size[2]};
  const int64_t plane = a.in_size[0] * a.in_size[1] * a.in_size[2];
  const int64_t n0 = a.out_size[0];
  const int64_t nl = ND == 1 ? 1 : a.out_size[ND - 1];          // last axis
  const int64_t n1 = ND == 3 ? a.out_size[1] : 1;               // middle axis (3D)
  const int64_t P = n0 * n1 * (ND == 1 ? 1 : nl);
  const int b = (int)(blockIdx.z / n1);
  const int64_t i1 = blockIdx.z - (int64_t)b * n1;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const float *gx = a.grid + (int64_t)b * ND * P;
  if constexpr (ND == 1) {
    // One row of 32 x kRows points; grid and output are both contiguous in i0.
    const int64_t i0 = ((int64_t)blockIdx.x * kRows + ty) * kTile + tx;
    if (i0 >= n0) return;
    float g[1] = {__ldg(gx + i0)};
    const Corners<1> cr = corners<1>(g, in);
    if constexpr (MODE == 0) {
      point_fwd<1>(a.data, a.out, C, (int64_t)b * C, plane, n0, i0, cr);
    } else {
      float gw[1];
      point_bwd<1, MODE == 2>(a.data, a.grad_out, a.grad_data, C, (int64_t)b * C, plane, n0, i0, cr, gw);
      if (a.grad_grid) a.grad_grid[(int64_t)b * P + i0] = __fmul_rn(gw[0], (float)(in[0] - 1));
    }
    return;
  } else {
    const int64_t I0 = (int64_t)blockIdx.y * kTile, IL = (int64_t)blockIdx.x * kTile;
    const int64_t mid = ND == 3 ? n0 * i1 : 0;                 // i1 contribution to p
    const int64_t lstride = ND == 3 ? n0 * n1 : n0;            // p stride of the last axis
    for (int r = ty; r < kTile; r += kRows) {
      const int64_t i0 = I0 + tx, il = IL + r;
      if (i0 < n0 && il < nl) {
        const int64_t p = i0 + mid + lstride * il;
#pragma unroll
        for (int k = 0; k < ND; ++k) sg[k][r][tx] = __ldg(gx + k * P + p);
      }
    }
    __syncthreads();
    for (int r = ty; r < kTile; r += kRows) {
      const int64_t i0 = I0 + r, il = IL + tx;
      if (i0 < n0 && il < nl) {
        float g[ND];
#pragma unroll
        for (int k = 0; k < ND; ++k) g[k] = sg[k][tx][r];
        const Corners<ND> cr = corners<ND>(g, in);
        const int64_t o = (i0 * n1 + i1) * nl + il;  // offset inside one output plane
        const int64_t oplane = n0 * n1 * nl;
        if constexpr (MODE == 0) {
          point_fwd<ND>(a.data, a.out, C, (int64_t)b * C, plane, oplane, o, cr);
        } else {
          float gw[ND];
          point_bwd<ND, MODE == 2>(a.data, a.grad_out, a.grad_data, C, (int64_t)b * C, plane, oplane, o, cr, gw);
          // Each tile entry is read only by the thread that wrote it above.
#pragma unroll
          for (int k = 0; k < ND; ++k) sg[k][tx][r] = __fmul_rn(gw[k], (float)(in[k] - 1));
        }
      }
    }
    if constexpr (MODE != 0) {
      if (a.grad_grid == nullptr) return;
      __syncthreads();
      float *gg = a.grad_grid + (int64_t)b * ND * P;
      for (int r = ty; r < kTile; r += kRows) {
        const int64_t i0 = I0 + tx, il = IL + r;
        if (i0 < n0 && il < nl) {
          const int64_t p = i0 + mid + lstride * il;
#pragma unroll
          for (int k = 0; k < ND; ++k) gg[k * P + p] = sg[k][r][tx];
        }
      }
    }
  }
}

template <int ND, int MODE>
__global__ void __launch_bounds__(kTile *kRows) k_interp(ResampleArgs a) {
  interp_body<ND, MODE>(a);
}

// 2D forward and grid-only backward, compiled for 8 and 6 resident blocks per
// SM (32 and 40 registers): their gathers are latency-bound, and the extra
// resident warps hide more of it than the few spilled values cost.  Measured
// at the dense 2D shape (32 x 3 x 512^2, CUDA events): forward 141 -> 115 us,
// backward 199 -> 145 us (at 6 and 4 blocks: 120 and 167 us).  3D, whose
// per-point state is larger, spills heavily under such caps and ran slower
// (forward 113 -> 123 us at 4 blocks); it keeps the compiler's choice.
template <int MODE> struct Interp2dBlocks { static constexpr int v = MODE == 0 ? 8 : 6; };

template <int MODE>
__global__ void __launch_bounds__(kTile *kRows, Interp2dBlocks<MODE>::v)
    k_interp_2d(ResampleArgs a) {
  interp_body<2, MODE>(a);
}

cudaError_t launch(const ResampleArgs &a, cudaStream_t s, bool bwd) {
  if (a.n_batch == 0 || a.n_channels == 0) return cudaSuccess;
  const dim3 block(kTile, kRows);
  const int64_t n0 = a.out_size[0];
  if (a.ndim == 1) {
    if (n0 == 0) return cudaSuccess;
    const dim3 grid((unsigned)((n0 + kTile * kRows - 1) / (kTile * kRows)), 1, (unsigned)a.n_batch);
    if (!bwd) k_interp<1, 0><<<grid, block, 0, s>>>(a);
    else if (a.grad_data == nullptr) k_interp<1, 1><<<grid, block, 0, s>>>(a);
    else k_interp<1, 2><<<grid, block, 0, s>>>(a);
  } else if (a.ndim == 2) {
    const int64_t nl = a.out_size[1];
    if (n0 == 0 || nl == 0) return cudaSuccess;
    const dim3 grid((unsigned)((nl + kTile - 1) / kTile), (unsigned)((n0 + kTile - 1) / kTile),
                    (unsigned)a.n_batch);
    if (!bwd) k_interp_2d<0><<<grid, block, 0, s>>>(a);
    else if (a.grad_data == nullptr) k_interp_2d<1><<<grid, block, 0, s>>>(a);
    else k_interp<2, 2><<<grid, block, 0, s>>>(a);
  } else {
    const int64_t n1 = a.out_size[1], nl = a.out_size[2];
    if (n0 == 0 || n1 == 0 || nl == 0) return cudaSuccess;
    const dim3 grid((unsigned)((nl + kTile - 1) / kTile), (unsigned)((n0 + kTile - 1) / kTile),
                    (unsigned)(a.n_batch * n1));
    if (!bwd) k_interp<3, 0><<<grid, block, 0, s>>>(a);
    else if (a.grad_data == nullptr) k_interp<3, 1><<<grid, block, 0, s>>>(a);
    else k_interp<3, 2><<<grid, block, 0, s>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_interpolate(const ResampleArgs &a, cudaStream_t s) { return launch(a, s, false); }

cudaError_t launch_interpolate_backward(const ResampleArgs &a, cudaStream_t s) {
  return launch(a, s, true);
}

}  // namespace cpab
