// Resampling arithmetic shared by the resample kernels (resample.cu) and the
// fused transform_data kernels (integrate.cu): the reference's corner and
// weight rules (cpab/pytorch/interpolation.py:8-160) with every product and
// sum explicitly rounded in its order, so that results are bit-identical
// wherever they are evaluated.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace cpab {
namespace rs {

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

// All channels of one output point o: channel ch of batch entry b reads the
// input plane data + (bc0 + ch) * plane and writes out + (bc0 + ch) * oplane.
template <int ND>
__device__ __forceinline__ void point_fwd(const float *__restrict__ data, float *__restrict__ out,
                                          int C, int64_t bc0, int64_t plane, int64_t oplane,
                                          int64_t o, const Corners<ND> &cr) {
  constexpr int K = Chunk<ND>::k;
  for (int c0 = 0; c0 < C; c0 += K) {
    float v[K][1 << ND];
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (c0 + j < C) gather<ND>(data + (bc0 + c0 + j) * plane, cr, v[j]);
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (c0 + j < C) out[(bc0 + c0 + j) * oplane + o] = combine<ND>(v[j], cr);
  }
}

// Backward of point_fwd: gw = sum over channels of d(out)/d(weights) * g
// (g = grad_out at o), and, with GD, the weight scatter into grad_data.
template <int ND, bool GD>
__device__ __forceinline__ void point_bwd(const float *__restrict__ data,
                                          const float *__restrict__ grad_out,
                                          float *__restrict__ grad_data, int C, int64_t bc0,
                                          int64_t plane, int64_t oplane, int64_t o,
                                          const Corners<ND> &cr, float (&gw)[ND]) {
  constexpr int K = Chunk<ND>::k;
#pragma unroll
  for (int k = 0; k < ND; ++k) gw[k] = 0.0f;
  for (int c0 = 0; c0 < C; c0 += K) {
    float v[K][1 << ND], g[K];
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (c0 + j < C) {
        gather<ND>(data + (bc0 + c0 + j) * plane, cr, v[j]);
        g[j] = __ldg(grad_out + (bc0 + c0 + j) * oplane + o);
      }
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (c0 + j < C)
        combine_bwd<ND>(v[j], cr, g[j], gw, GD ? grad_data + (bc0 + c0 + j) * plane : nullptr);
  }
}

}  // namespace rs
}  // namespace cpab
