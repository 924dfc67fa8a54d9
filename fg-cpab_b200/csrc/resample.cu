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

namespace cpab {

namespace {

constexpr int kTile = 32;
constexpr int kRows = 8;

struct Axis {
  int64_t lo, hi;  // clamped corner indices
  float w;         // weight of the upper corner, measured from lo
};

__device__ __forceinline__ Axis axis_of(float g, int64_t n) {
  const float top = (float)(n - 1);
  const float x = __fmul_rn(g, top);
  const float f = floorf(x);
  const float lo = fminf(fmaxf(f, 0.0f), top);
  const float hi = fminf(fmaxf(__fadd_rn(f, 1.0f), 0.0f), top);
  Axis a;
  a.lo = (int64_t)lo;
  a.hi = (int64_t)hi;
  a.w = __fsub_rn(x, lo);
  return a;
}

// (1 - w) * lo + w * hi with the reference's rounding of each operation.
__device__ __forceinline__ float lerp_ref(float lo, float hi, float w, float wc) {
  return __fadd_rn(__fmul_rn(lo, wc), __fmul_rn(hi, w));
}

// ----------------------------------------------------------------------------
// Per-location sample and its backward, for every channel.
// ----------------------------------------------------------------------------

struct Loc1 { Axis x; };
struct Loc2 { Axis x, y; };
struct Loc3 { Axis x, y, z; };

__device__ __forceinline__ float sample(const float *__restrict__ d, const Loc1 &l, int64_t) {
  const float wc = __fsub_rn(1.0f, l.x.w);
  return lerp_ref(__ldg(d + l.x.lo), __ldg(d + l.x.hi), l.x.w, wc);
}

// d points at data[b, ch] with axis strides (s1 = S1).
__device__ __forceinline__ float sample2(const float *__restrict__ d, const Loc2 &l, int64_t s1) {
  const float c00 = __ldg(d + l.x.lo * s1 + l.y.lo), c01 = __ldg(d + l.x.lo * s1 + l.y.hi);
  const float c10 = __ldg(d + l.x.hi * s1 + l.y.lo), c11 = __ldg(d + l.x.hi * s1 + l.y.hi);
  const float xc = __fsub_rn(1.0f, l.x.w), yc = __fsub_rn(1.0f, l.y.w);
  const float c0 = lerp_ref(c00, c10, l.x.w, xc);
  const float c1 = lerp_ref(c01, c11, l.x.w, xc);
  return lerp_ref(c0, c1, l.y.w, yc);
}

__device__ __forceinline__ float sample3(const float *__restrict__ d, const Loc3 &l, int64_t s1,
                                         int64_t s2) {
  const int64_t x0 = l.x.lo * s1 * s2, x1 = l.x.hi * s1 * s2;
  const int64_t y0 = l.y.lo * s2, y1 = l.y.hi * s2;
  const float c000 = __ldg(d + x0 + y0 + l.z.lo), c001 = __ldg(d + x0 + y0 + l.z.hi);
  const float c010 = __ldg(d + x0 + y1 + l.z.lo), c011 = __ldg(d + x0 + y1 + l.z.hi);
  const float c100 = __ldg(d + x1 + y0 + l.z.lo), c101 = __ldg(d + x1 + y0 + l.z.hi);
  const float c110 = __ldg(d + x1 + y1 + l.z.lo), c111 = __ldg(d + x1 + y1 + l.z.hi);
  const float xc = __fsub_rn(1.0f, l.x.w), yc = __fsub_rn(1.0f, l.y.w),
              zc = __fsub_rn(1.0f, l.z.w);
  const float c00 = lerp_ref(c000, c100, l.x.w, xc);
  const float c01 = lerp_ref(c001, c101, l.x.w, xc);
  const float c10 = lerp_ref(c010, c110, l.x.w, xc);
  const float c11 = lerp_ref(c011, c111, l.x.w, xc);
  const float c0 = lerp_ref(c00, c10, l.y.w, yc);
  const float c1 = lerp_ref(c01, c11, l.y.w, yc);
  return lerp_ref(c0, c1, l.z.w, zc);
}

// Backward at one location for one channel: accumulates d(out)/d(weights)
// times g into gw[] and scatters g * weights into gd (when non-null).  Each
// product is rounded on its own, as torch's autograd evaluates them, so that
// g*hi - g*lo is exactly 0 when a coordinate is clamped (hi == lo).
__device__ __forceinline__ float gdiff(float g, float hi, float lo) {
  return __fsub_rn(__fmul_rn(g, hi), __fmul_rn(g, lo));
}

__device__ __forceinline__ void sample_bwd(const float *__restrict__ d, float *__restrict__ gd,
                                           const Loc1 &l, int64_t, float g, float (&gw)[1]) {
  const float c0 = __ldg(d + l.x.lo), c1 = __ldg(d + l.x.hi);
  gw[0] = __fadd_rn(gw[0], gdiff(g, c1, c0));
  if (gd) {
    atomicAdd(gd + l.x.lo, __fmul_rn(g, __fsub_rn(1.0f, l.x.w)));
    atomicAdd(gd + l.x.hi, __fmul_rn(g, l.x.w));
  }
}

__device__ __forceinline__ void sample2_bwd(const float *__restrict__ d, float *__restrict__ gd,
                                            const Loc2 &l, int64_t s1, float g, float (&gw)[2]) {
  const int64_t a00 = l.x.lo * s1 + l.y.lo, a01 = l.x.lo * s1 + l.y.hi;
  const int64_t a10 = l.x.hi * s1 + l.y.lo, a11 = l.x.hi * s1 + l.y.hi;
  const float c00 = __ldg(d + a00), c01 = __ldg(d + a01), c10 = __ldg(d + a10), c11 = __ldg(d + a11);
  const float xw = l.x.w, xc = __fsub_rn(1.0f, xw), yw = l.y.w, yc = __fsub_rn(1.0f, yw);
  const float g0 = __fmul_rn(g, yc), g1 = __fmul_rn(g, yw);  // gradients of the two x-lerps
  const float c0 = lerp_ref(c00, c10, xw, xc), c1 = lerp_ref(c01, c11, xw, xc);
  gw[0] = __fadd_rn(gw[0], __fadd_rn(gdiff(g0, c10, c00), gdiff(g1, c11, c01)));
  gw[1] = __fadd_rn(gw[1], gdiff(g, c1, c0));
  if (gd) {
    atomicAdd(gd + a00, __fmul_rn(g0, xc));
    atomicAdd(gd + a10, __fmul_rn(g0, xw));
    atomicAdd(gd + a01, __fmul_rn(g1, xc));
    atomicAdd(gd + a11, __fmul_rn(g1, xw));
  }
}

__device__ __forceinline__ void sample3_bwd(const float *__restrict__ d, float *__restrict__ gd,
                                            const Loc3 &l, int64_t s1, int64_t s2, float g,
                                            float (&gw)[3]) {
  const int64_t x0 = l.x.lo * s1 * s2, x1 = l.x.hi * s1 * s2;
  const int64_t y0 = l.y.lo * s2, y1 = l.y.hi * s2;
  const int64_t z0 = l.z.lo, z1 = l.z.hi;
  const int64_t a[8] = {x0 + y0 + z0, x0 + y0 + z1, x0 + y1 + z0, x0 + y1 + z1,
                        x1 + y0 + z0, x1 + y0 + z1, x1 + y1 + z0, x1 + y1 + z1};
  float c[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) c[k] = __ldg(d + a[k]);
  // c[k] for k = 4*X + 2*Y + Z.
  const float xw = l.x.w, xc = __fsub_rn(1.0f, xw), yw = l.y.w, yc = __fsub_rn(1.0f, yw);
  const float zw = l.z.w, zc = __fsub_rn(1.0f, zw);
  const float c00 = lerp_ref(c[0], c[4], xw, xc);  // (y0, z0)
  const float c01 = lerp_ref(c[1], c[5], xw, xc);  // (y0, z1)
  const float c10 = lerp_ref(c[2], c[6], xw, xc);  // (y1, z0)
  const float c11 = lerp_ref(c[3], c[7], xw, xc);  // (y1, z1)
  const float c0 = lerp_ref(c00, c10, yw, yc), c1 = lerp_ref(c01, c11, yw, yc);
  const float gc0 = __fmul_rn(g, zc), gc1 = __fmul_rn(g, zw);
  const float g00 = __fmul_rn(gc0, yc), g10 = __fmul_rn(gc0, yw);
  const float g01 = __fmul_rn(gc1, yc), g11 = __fmul_rn(gc1, yw);
  gw[2] = __fadd_rn(gw[2], gdiff(g, c1, c0));
  gw[1] = __fadd_rn(gw[1], __fadd_rn(gdiff(gc0, c10, c00), gdiff(gc1, c11, c01)));
  gw[0] = __fadd_rn(gw[0], __fadd_rn(__fadd_rn(gdiff(g00, c[4], c[0]), gdiff(g01, c[5], c[1])),
                                     __fadd_rn(gdiff(g10, c[6], c[2]), gdiff(g11, c[7], c[3]))));
  if (gd) {
    atomicAdd(gd + a[0], __fmul_rn(g00, xc)); atomicAdd(gd + a[4], __fmul_rn(g00, xw));
    atomicAdd(gd + a[1], __fmul_rn(g01, xc)); atomicAdd(gd + a[5], __fmul_rn(g01, xw));
    atomicAdd(gd + a[2], __fmul_rn(g10, xc)); atomicAdd(gd + a[6], __fmul_rn(g10, xw));
    atomicAdd(gd + a[3], __fmul_rn(g11, xc)); atomicAdd(gd + a[7], __fmul_rn(g11, xw));
  }
}

// ----------------------------------------------------------------------------
// 1D: out[b, ch, i0], grid point p = i0 -- already aligned, no transpose.
// ----------------------------------------------------------------------------

__global__ void k_interp1d(ResampleArgs a) {
  const int b = blockIdx.y;
  const int64_t n0 = a.out_size[0], S0 = a.in_size[0];
  const int C = a.n_channels;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n0;
       i += (int64_t)gridDim.x * blockDim.x) {
    Loc1 l;
    l.x = axis_of(__ldg(a.grid + (int64_t)b * n0 + i), S0);
    for (int ch = 0; ch < C; ++ch) {
      const float *d = a.data + ((int64_t)b * C + ch) * S0;
      a.out[((int64_t)b * C + ch) * n0 + i] = sample(d, l, 0);
    }
  }
}

__global__ void k_interp1d_bwd(ResampleArgs a) {
  const int b = blockIdx.y;
  const int64_t n0 = a.out_size[0], S0 = a.in_size[0];
  const int C = a.n_channels;
  const float top = (float)(S0 - 1);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n0;
       i += (int64_t)gridDim.x * blockDim.x) {
    Loc1 l;
    l.x = axis_of(__ldg(a.grid + (int64_t)b * n0 + i), S0);
    float gw[1] = {0.0f};
    for (int ch = 0; ch < C; ++ch) {
      const int64_t base = ((int64_t)b * C + ch) * S0;
      const float g = __ldg(a.grad_out + ((int64_t)b * C + ch) * n0 + i);
      sample_bwd(a.data + base, a.grad_data ? a.grad_data + base : nullptr, l, 0, g, gw);
    }
    if (a.grad_grid) a.grad_grid[(int64_t)b * n0 + i] = __fmul_rn(gw[0], top);
  }
}

// ----------------------------------------------------------------------------
// 2D: tile (i0, i1); blockIdx.x -> i1 tile, blockIdx.y -> i0 tile, z -> batch.
// ----------------------------------------------------------------------------

template <bool BWD>
__global__ void __launch_bounds__(kTile *kRows) k_interp2d(ResampleArgs a) {
  __shared__ float sg[2][kTile][kTile + 1];  // grid tile, [i1 local][i0 local]
  __shared__ float sd[2][kTile][kTile + 1];  // backward: d grid, [i1 local][i0 local]
  const int b = blockIdx.z;
  const int64_t n0 = a.out_size[0], n1 = a.out_size[1];
  const int64_t P = n0 * n1;
  const int64_t S0 = a.in_size[0], S1 = a.in_size[1];
  const int C = a.n_channels;
  const int64_t I0 = (int64_t)blockIdx.y * kTile, I1 = (int64_t)blockIdx.x * kTile;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const float *gx = a.grid + (int64_t)b * 2 * P;
  for (int r = ty; r < kTile; r += kRows) {
    const int64_t i0 = I0 + tx, i1 = I1 + r;
    if (i0 < n0 && i1 < n1) {
      const int64_t p = i0 + n0 * i1;
      sg[0][r][tx] = __ldg(gx + p);
      sg[1][r][tx] = __ldg(gx + P + p);
    }
  }
  __syncthreads();
  for (int r = ty; r < kTile; r += kRows) {
    const int64_t i0 = I0 + r, i1 = I1 + tx;
    if (i0 < n0 && i1 < n1) {
      Loc2 l;
      l.x = axis_of(sg[0][tx][r], S0);
      l.y = axis_of(sg[1][tx][r], S1);
      if constexpr (!BWD) {
        for (int ch = 0; ch < C; ++ch) {
          const int64_t bc = (int64_t)b * C + ch;
          a.out[(bc * n0 + i0) * n1 + i1] = sample2(a.data + bc * S0 * S1, l, S1);
        }
      } else {
        float gw[2] = {0.0f, 0.0f};
        for (int ch = 0; ch < C; ++ch) {
          const int64_t bc = (int64_t)b * C + ch;
          const float g = __ldg(a.grad_out + (bc * n0 + i0) * n1 + i1);
          sample2_bwd(a.data + bc * S0 * S1, a.grad_data ? a.grad_data + bc * S0 * S1 : nullptr,
                      l, S1, g, gw);
        }
        sd[0][tx][r] = __fmul_rn(gw[0], (float)(S0 - 1));
        sd[1][tx][r] = __fmul_rn(gw[1], (float)(S1 - 1));
      }
    }
  }
  if constexpr (BWD) {
    if (a.grad_grid == nullptr) return;
    __syncthreads();
    float *gg = a.grad_grid + (int64_t)b * 2 * P;
    for (int r = ty; r < kTile; r += kRows) {
      const int64_t i0 = I0 + tx, i1 = I1 + r;
      if (i0 < n0 && i1 < n1) {
        const int64_t p = i0 + n0 * i1;
        gg[p] = sd[0][r][tx];
        gg[P + p] = sd[1][r][tx];
      }
    }
  }
}

// ----------------------------------------------------------------------------
// 3D: tile (i0, i2) at fixed i1; blockIdx.x -> i2 tile, y -> i0 tile,
// z -> b * n1 + i1.
// ----------------------------------------------------------------------------

template <bool BWD>
__global__ void __launch_bounds__(kTile *kRows) k_interp3d(ResampleArgs a) {
  __shared__ float sg[3][kTile][kTile + 1];  // [i2 local][i0 local]
  const int64_t n0 = a.out_size[0], n1 = a.out_size[1], n2 = a.out_size[2];
  const int64_t P = n0 * n1 * n2;
  const int b = (int)(blockIdx.z / n1);
  const int64_t i1 = blockIdx.z - (int64_t)b * n1;
  const int64_t S0 = a.in_size[0], S1 = a.in_size[1], S2 = a.in_size[2];
  const int C = a.n_channels;
  const int64_t I0 = (int64_t)blockIdx.y * kTile, I2 = (int64_t)blockIdx.x * kTile;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const float *gx = a.grid + (int64_t)b * 3 * P;
  for (int r = ty; r < kTile; r += kRows) {
    const int64_t i0 = I0 + tx, i2 = I2 + r;
    if (i0 < n0 && i2 < n2) {
      const int64_t p = i0 + n0 * (i1 + n1 * i2);
      sg[0][r][tx] = __ldg(gx + p);
      sg[1][r][tx] = __ldg(gx + P + p);
      sg[2][r][tx] = __ldg(gx + 2 * P + p);
    }
  }
  __syncthreads();
  const int64_t vol = S0 * S1 * S2;
  for (int r = ty; r < kTile; r += kRows) {
    const int64_t i0 = I0 + r, i2 = I2 + tx;
    if (i0 < n0 && i2 < n2) {
      Loc3 l;
      l.x = axis_of(sg[0][tx][r], S0);
      l.y = axis_of(sg[1][tx][r], S1);
      l.z = axis_of(sg[2][tx][r], S2);
      if constexpr (!BWD) {
        for (int ch = 0; ch < C; ++ch) {
          const int64_t bc = (int64_t)b * C + ch;
          a.out[((bc * n0 + i0) * n1 + i1) * n2 + i2] = sample3(a.data + bc * vol, l, S1, S2);
        }
      } else {
        float gw[3] = {0.0f, 0.0f, 0.0f};
        for (int ch = 0; ch < C; ++ch) {
          const int64_t bc = (int64_t)b * C + ch;
          const float g = __ldg(a.grad_out + ((bc * n0 + i0) * n1 + i1) * n2 + i2);
          sample3_bwd(a.data + bc * vol, a.grad_data ? a.grad_data + bc * vol : nullptr, l, S1,
                      S2, g, gw);
        }
        // Reuse the grid tile for d grid (each entry is read only by its owner).
        sg[0][tx][r] = __fmul_rn(gw[0], (float)(S0 - 1));
        sg[1][tx][r] = __fmul_rn(gw[1], (float)(S1 - 1));
        sg[2][tx][r] = __fmul_rn(gw[2], (float)(S2 - 1));
      }
    }
  }
  if constexpr (BWD) {
    if (a.grad_grid == nullptr) return;
    __syncthreads();
    float *gg = a.grad_grid + (int64_t)b * 3 * P;
    for (int r = ty; r < kTile; r += kRows) {
      const int64_t i0 = I0 + tx, i2 = I2 + r;
      if (i0 < n0 && i2 < n2) {
        const int64_t p = i0 + n0 * (i1 + n1 * i2);
        gg[p] = sg[0][r][tx];
        gg[P + p] = sg[1][r][tx];
        gg[2 * P + p] = sg[2][r][tx];
      }
    }
  }
}

cudaError_t launch(const ResampleArgs &a, cudaStream_t s, bool bwd) {
  if (a.n_batch == 0 || a.n_channels == 0) return cudaSuccess;
  const dim3 block2(kTile, kRows);
  if (a.ndim == 1) {
    const int64_t n0 = a.out_size[0];
    if (n0 == 0) return cudaSuccess;
    int64_t bx = (n0 + 255) / 256;
    if (bx > 4096) bx = 4096;
    const dim3 grid((unsigned)bx, (unsigned)a.n_batch);
    if (bwd) k_interp1d_bwd<<<grid, 256, 0, s>>>(a);
    else k_interp1d<<<grid, 256, 0, s>>>(a);
  } else if (a.ndim == 2) {
    const int64_t n0 = a.out_size[0], n1 = a.out_size[1];
    if (n0 == 0 || n1 == 0) return cudaSuccess;
    const dim3 grid((unsigned)((n1 + kTile - 1) / kTile), (unsigned)((n0 + kTile - 1) / kTile),
                    (unsigned)a.n_batch);
    if (bwd) k_interp2d<true><<<grid, block2, 0, s>>>(a);
    else k_interp2d<false><<<grid, block2, 0, s>>>(a);
  } else {
    const int64_t n0 = a.out_size[0], n1 = a.out_size[1], n2 = a.out_size[2];
    if (n0 == 0 || n1 == 0 || n2 == 0) return cudaSuccess;
    const dim3 grid((unsigned)((n2 + kTile - 1) / kTile), (unsigned)((n0 + kTile - 1) / kTile),
                    (unsigned)(a.n_batch * n1));
    if (bwd) k_interp3d<true><<<grid, block2, 0, s>>>(a);
    else k_interp3d<false><<<grid, block2, 0, s>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_interpolate(const ResampleArgs &a, cudaStream_t s) { return launch(a, s, false); }

cudaError_t launch_interpolate_backward(const ResampleArgs &a, cudaStream_t s) {
  return launch(a, s, true);
}

}  // namespace cpab
