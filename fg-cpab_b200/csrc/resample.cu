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
  int lo, hi;  // clamped corner indices (in-plane offsets are 32-bit: the
               // caller guarantees one (batch, channel) plane < 2^31 elements)
  float w;     // weight of the upper corner, measured from lo
};

__device__ __forceinline__ Axis axis_of(float g, int n) {
  const float top = (float)(n - 1);
  const float x = __fmul_rn(g, top);
  const float f = floorf(x);
  const float lo = fminf(fmaxf(f, 0.0f), top);
  const float hi = fminf(fmaxf(__fadd_rn(f, 1.0f), 0.0f), top);
  Axis a;
  a.lo = (int)lo;
  a.hi = (int)hi;
  a.w = __fsub_rn(x, lo);
  return a;
}

// (1 - w) * lo + w * hi with the reference's rounding of each operation.
__device__ __forceinline__ float lerp_ref(float lo, float hi, float w, float wc) {
  return __fadd_rn(__fmul_rn(lo, wc), __fmul_rn(hi, w));
}

// g*hi - g*lo with each product rounded on its own, as torch's autograd
// evaluates them, so that it is exactly 0 when a coordinate is clamped.
__device__ __forceinline__ float gdiff(float g, float hi, float lo) {
  return __fsub_rn(__fmul_rn(g, hi), __fmul_rn(g, lo));
}

// Corner offsets inside one channel plane, kept per axis (lo and hi already
// multiplied by the axis stride); corner m = sum_k bit_k(m) << (ND-1-k), axis
// 0 the most significant bit (c000, c001, c010, ... as in the reference's
// interpolate3D), sits at ax[0][bit_0] + ax[1][bit_1] (+ ax[2][bit_2]).
template <int ND> struct Corners {
  int ax[ND][2];
  float w[ND], wc[ND];
  __device__ __forceinline__ int off(int m) const {
    int o = 0;
#pragma unroll
    for (int k = 0; k < ND; ++k) o += ax[k][(m >> (ND - 1 - k)) & 1];
    return o;
  }
};

template <int ND>
__device__ __forceinline__ Corners<ND> corners(const float (&g)[ND], const int (&in)[3]) {
  Corners<ND> c;
  int stride = 1;
#pragma unroll
  for (int k = ND - 1; k >= 0; --k) {
    const Axis a = axis_of(g[k], in[k]);
    c.w[k] = a.w;
    c.wc[k] = __fsub_rn(1.0f, a.w);
    c.ax[k][0] = a.lo * stride;
    c.ax[k][1] = a.hi * stride;
    stride *= in[k];
  }
  return c;
}

// Channels gathered together: all their corner loads are issued before any
// of them is used, so a thread keeps Chunk<ND>::k * 2^ND independent loads in flight
// (the output stores of one channel cannot be ordered before the next
// channel's loads otherwise, since the compiler cannot rule out aliasing).
template <int ND> struct Chunk { static constexpr int k = ND == 3 ? 1 : 2; };

template <int ND>
__device__ __forceinline__ void gather(const float *__restrict__ d, const Corners<ND> &c,
                                       float (&v)[1 << ND]) {
#pragma unroll
  for (int m = 0; m < (1 << ND); ++m) v[m] = __ldg(d + c.off(m));
}

// Interpolated value from the corner values v (reference order: lerp along
// axis 0 first, then 1, then 2; v[4X + 2Y + Z] in 3D).
template <int ND>
__device__ __forceinline__ float combine(const float (&v)[1 << ND], const Corners<ND> &c) {
  if constexpr (ND == 1) {
    return lerp_ref(v[0], v[1], c.w[0], c.wc[0]);
  } else if constexpr (ND == 2) {
    const float c0 = lerp_ref(v[0], v[2], c.w[0], c.wc[0]);
    const float c1 = lerp_ref(v[1], v[3], c.w[0], c.wc[0]);
    return lerp_ref(c0, c1, c.w[1], c.wc[1]);
  } else {
    const float c00 = lerp_ref(v[0], v[4], c.w[0], c.wc[0]);  // (y0, z0)
    const float c01 = lerp_ref(v[1], v[5], c.w[0], c.wc[0]);  // (y0, z1)
    const float c10 = lerp_ref(v[2], v[6], c.w[0], c.wc[0]);  // (y1, z0)
    const float c11 = lerp_ref(v[3], v[7], c.w[0], c.wc[0]);  // (y1, z1)
    const float c0 = lerp_ref(c00, c10, c.w[1], c.wc[1]);
    const float c1 = lerp_ref(c01, c11, c.w[1], c.wc[1]);
    return lerp_ref(c0, c1, c.w[2], c.wc[2]);
  }
}

// Backward of one channel from its corner values v and output gradient g:
// adds d(out)/d(weights) * g to gw and scatters g * weights into gd (when
// non-null).  Each partial product is rounded as torch's autograd of the
// reference expression rounds it.
template <int ND>
__device__ __forceinline__ void combine_bwd(const float (&v)[1 << ND], const Corners<ND> &c,
                                            float g, float (&gw)[ND], float *__restrict__ gd) {
  if constexpr (ND == 1) {
    gw[0] = __fadd_rn(gw[0], gdiff(g, v[1], v[0]));
    if (gd) {
      atomicAdd(gd + c.off(0), __fmul_rn(g, c.wc[0]));
      atomicAdd(gd + c.off(1), __fmul_rn(g, c.w[0]));
    }
  } else if constexpr (ND == 2) {
    const float c00 = v[0], c01 = v[1], c10 = v[2], c11 = v[3];
    const float g0 = __fmul_rn(g, c.wc[1]), g1 = __fmul_rn(g, c.w[1]);  // the two x-lerps
    const float c0 = lerp_ref(c00, c10, c.w[0], c.wc[0]), c1 = lerp_ref(c01, c11, c.w[0], c.wc[0]);
    gw[0] = __fadd_rn(gw[0], __fadd_rn(gdiff(g0, c10, c00), gdiff(g1, c11, c01)));
    gw[1] = __fadd_rn(gw[1], gdiff(g, c1, c0));
    if (gd) {
      atomicAdd(gd + c.off(0), __fmul_rn(g0, c.wc[0]));
      atomicAdd(gd + c.off(2), __fmul_rn(g0, c.w[0]));
      atomicAdd(gd + c.off(1), __fmul_rn(g1, c.wc[0]));
      atomicAdd(gd + c.off(3), __fmul_rn(g1, c.w[0]));
    }
  } else {
    const float xw = c.w[0], xc = c.wc[0], yw = c.w[1], yc = c.wc[1], zw = c.w[2], zc = c.wc[2];
    const float c00 = lerp_ref(v[0], v[4], xw, xc), c01 = lerp_ref(v[1], v[5], xw, xc);
    const float c10 = lerp_ref(v[2], v[6], xw, xc), c11 = lerp_ref(v[3], v[7], xw, xc);
    const float c0 = lerp_ref(c00, c10, yw, yc), c1 = lerp_ref(c01, c11, yw, yc);
    const float gc0 = __fmul_rn(g, zc), gc1 = __fmul_rn(g, zw);
    const float g00 = __fmul_rn(gc0, yc), g10 = __fmul_rn(gc0, yw);
    const float g01 = __fmul_rn(gc1, yc), g11 = __fmul_rn(gc1, yw);
    gw[2] = __fadd_rn(gw[2], gdiff(g, c1, c0));
    gw[1] = __fadd_rn(gw[1], __fadd_rn(gdiff(gc0, c10, c00), gdiff(gc1, c11, c01)));
    gw[0] = __fadd_rn(gw[0], __fadd_rn(__fadd_rn(gdiff(g00, v[4], v[0]), gdiff(g01, v[5], v[1])),
                                       __fadd_rn(gdiff(g10, v[6], v[2]), gdiff(g11, v[7], v[3]))));
    if (gd) {
      const float gs[4] = {g00, g01, g10, g11};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        atomicAdd(gd + c.off(m), __fmul_rn(gs[m], xc));
        atomicAdd(gd + c.off(m + 4), __fmul_rn(gs[m], xw));
      }
    }
  }
}

// All channels of one output point: plane(ch) is channel ch's input plane,
// o_at(ch) the offset of the point in channel ch's output (or d out) plane.
template <int ND>
__device__ __forceinline__ void point_fwd(const ResampleArgs &a, int64_t bc0, int64_t plane,
                                          int64_t oplane, int64_t o, const Corners<ND> &cr) {
  constexpr int K = Chunk<ND>::k;
  const int C = a.n_channels;
  for (int c0 = 0; c0 < C; c0 += K) {
    float v[K][1 << ND];
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (c0 + j < C) gather<ND>(a.data + (bc0 + c0 + j) * plane, cr, v[j]);
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (c0 + j < C) a.out[(bc0 + c0 + j) * oplane + o] = combine<ND>(v[j], cr);
  }
}

template <int ND, bool GD>
__device__ __forceinline__ void point_bwd(const ResampleArgs &a, int64_t bc0, int64_t plane,
                                          int64_t oplane, int64_t o, const Corners<ND> &cr,
                                          float (&gw)[ND]) {
  constexpr int K = Chunk<ND>::k;
  const int C = a.n_channels;
#pragma unroll
  for (int k = 0; k < ND; ++k) gw[k] = 0.0f;
  for (int c0 = 0; c0 < C; c0 += K) {
    float v[K][1 << ND], g[K];
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (c0 + j < C) {
        gather<ND>(a.data + (bc0 + c0 + j) * plane, cr, v[j]);
        g[j] = __ldg(a.grad_out + (bc0 + c0 + j) * oplane + o);
      }
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (c0 + j < C)
        combine_bwd<ND>(v[j], cr, g[j], gw, GD ? a.grad_data + (bc0 + c0 + j) * plane : nullptr);
  }
}

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
__global__ void __launch_bounds__(kTile *kRows) k_interp(ResampleArgs a) {
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
      point_fwd<1>(a, (int64_t)b * C, plane, n0, i0, cr);
    } else {
      float gw[1];
      point_bwd<1, MODE == 2>(a, (int64_t)b * C, plane, n0, i0, cr, gw);
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
          point_fwd<ND>(a, (int64_t)b * C, plane, oplane, o, cr);
        } else {
          float gw[ND];
          point_bwd<ND, MODE == 2>(a, (int64_t)b * C, plane, oplane, o, cr, gw);
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
    if (!bwd) k_interp<2, 0><<<grid, block, 0, s>>>(a);
    else if (a.grad_data == nullptr) k_interp<2, 1><<<grid, block, 0, s>>>(a);
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
