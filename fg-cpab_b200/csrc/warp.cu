// Fused spatial-transformer warp (2D/3D): the CpabWarp layer of the
// reference's stn/stn.py:58-86 in one kernel each way.  The reference maps
// its pixel grid through T_1 o ... o T_K with one CPAB_transformer call per
// transformation (stn/stn.py:79-86), writes the grid, and samples the image
// with F.grid_sample(x, grid, align_corners=True, padding_mode)
// (stn/stn.py:48-54); its backward runs grid_sample's backward, which writes
// the grid gradient, and then one adjoint sweep per transformation.  Here the
// K transformations run as a fused chain per pixel (the chain kernels of
// integrate_body.cuh), the last position is sampled in the same thread, and
// the backward forms the grid gradient in registers and starts the adjoint
// from it.
//
// The sampling restates F.grid_sample's bilinear (2D) / trilinear (3D) rule
// with align_corners=True as PyTorch (2.11) evaluates it on the GPU
// (aten/src/ATen/native/cuda/GridSampler.cuh and GridSampler.cu): the grid
// coordinate g = 2p - 1 of a CPAB coordinate p (stn/stn.py:86) is mapped to
// the source index x = ((g + 1) / 2) * (n - 1), folded into the image by the
// padding mode (border: clamped to [0, n-1]; reflection: reflected about 0
// and n-1, then clamped), and the 2^ND neighbours floor(x) and floor(x) + 1
// of each axis are weighted by products of their distances; neighbours
// outside the image are skipped (zeros padding).  The grid gradient is the
// sum over channels and in-image neighbours of value * d(weight)/dx * grad,
// times (n - 1)/2 (and the clamp's 0 or reflection's sign), and the STN's
// `points * 2 - 1` doubles it into the CPAB coordinate's gradient.
//
// Layout: CPAB coordinate k runs along image axis k (data [.., C, *in_size],
// axis 0 outermost); corner m of a point takes the upper neighbour on axis k
// when bit ND-1-k of m is set, so m counts with the LAST axis fastest, which
// is grid_sample's order (x = W fastest: nw, ne, sw, se; 3D t/b then n/s
// then w/e), and every sum runs in that order.
#include <cuda_runtime.h>

#include "integrate_body.cuh"
#include "launch.h"

namespace cpab {

namespace {

// Source index along an axis of n pixels for CPAB coordinate p; mult
// receives d(index)/d(g).  GRAD selects the backward's evaluation of the
// padding, which differs from the forward's only where PyTorch's two
// differ (a NaN clamps to 0 in the forward; -0 is not reflected in the
// backward), so that each matches its counterpart.
template <bool GRAD>
__device__ __forceinline__ float source_index(float p, int n, int pad, float &mult) {
  const float g = __fsub_rn(__fmul_rn(p, 2.0f), 1.0f);  // stn.py: points * 2 - 1
  const float top = (float)(n - 1);
  float x = __fmul_rn(__fmul_rn(__fadd_rn(g, 1.0f), 0.5f), top);
  mult = __fmul_rn(top, 0.5f);
  if (pad == kPadReflection) {
    if (n == 1) {
      x = 0.0f;
      mult = 0.0f;
    } else {
      float sgn = 1.0f;
      if constexpr (GRAD) {
        if (x < 0.0f) {
          sgn = -1.0f;
          x = -x;
        }
      } else {
        x = fabsf(x);
      }
      const float extra = fmodf(x, top);
      const int flips = (int)floorf(__fdiv_rn(x, top));
      if (flips % 2 == 0) {
        x = __fadd_rn(extra, 0.0f);
      } else {
        x = __fadd_rn(__fsub_rn(top, extra), 0.0f);
        sgn = -sgn;
      }
      mult = __fmul_rn(mult, sgn);
    }
  }
  if (pad != kPadZeros) {
    if constexpr (GRAD) {
      if (x <= 0.0f) {
        x = 0.0f;
        mult = 0.0f;
      } else if (x >= top) {
        x = top;
        mult = 0.0f;
      }
    } else {
      x = fminf(top, fmaxf(x, 0.0f));
    }
  }
  // Outside the int range (or not finite): a value no neighbour of which is
  // inside the image, as PyTorch substitutes.
  if (!(x <= 2147483648.0f && x >= -2147483648.0f)) x = -100.0f;
  return x;
}

// The 2^ND neighbours of one sampling point.
template <int ND> struct Taps {
  int off[1 << ND];     // offsets inside one channel plane (in-image corners)
  float w[1 << ND];     // weights
  unsigned in;          // bit m: corner m inside the image
  float fl[ND], fh[ND]; // per axis: weight factor of the lower / upper neighbour
  float mult[ND];       // per axis: d(index)/d(grid coordinate)
};

template <int ND, bool GRAD>
__device__ __forceinline__ Taps<ND> make_taps(const float (&p)[ND], const int (&n)[3], int pad) {
  Taps<ND> t;
  int lo[ND];
  bool il[ND], ih[ND];
#pragma unroll
  for (int k = 0; k < ND; ++k) {
    const float x = source_index<GRAD>(p[k], n[k], pad, t.mult[k]);
    lo[k] = (int)floorf(x);
    t.fl[k] = __fsub_rn(__fadd_rn((float)lo[k], 1.0f), x);
    t.fh[k] = __fsub_rn(x, (float)lo[k]);
    il[k] = lo[k] >= 0 && lo[k] < n[k];
    ih[k] = lo[k] >= -1 && lo[k] < n[k] - 1;
  }
  t.in = 0u;
#pragma unroll
  for (int m = 0; m < (1 << ND); ++m) {
    bool inside = true;
    unsigned o = 0u;  // wraps only for corners outside the image, never used
#pragma unroll
    for (int k = 0; k < ND; ++k) {
      const bool hi = (m >> (ND - 1 - k)) & 1;
      inside = inside && (hi ? ih[k] : il[k]);
      o = o * (unsigned)n[k] + (unsigned)lo[k] + (hi ? 1u : 0u);
    }
    // Product of the axes' factors, last axis first (grid_sample's order).
    float w = 0.0f;
#pragma unroll
    for (int k = ND - 1; k >= 0; --k) {
      const bool hi = (m >> (ND - 1 - k)) & 1;
      const float f = hi ? t.fh[k] : t.fl[k];
      w = k == ND - 1 ? f : __fmul_rn(w, f);
    }
    t.off[m] = inside ? (int)o : 0;
    t.w[m] = w;
    if (inside) t.in |= 1u << m;
  }
  return t;
}

// out[c] = sum over in-image corners of value * weight, for every channel.
template <int ND>
__device__ __forceinline__ void sample_fwd(const float *__restrict__ img, float *__restrict__ out,
                                           int C, int64_t plane, int64_t oplane, int64_t o,
                                           const Taps<ND> &t) {
  for (int c = 0; c < C; ++c) {
    const float *d = img + (int64_t)c * plane;
    float v[1 << ND];
#pragma unroll
    for (int m = 0; m < (1 << ND); ++m) v[m] = (t.in >> m & 1u) ? __ldg(d + t.off[m]) : 0.0f;
    float acc = 0.0f;
#pragma unroll
    for (int m = 0; m < (1 << ND); ++m)
      if (t.in >> m & 1u) acc = __fmaf_rn(v[m], t.w[m], acc);
    out[(int64_t)c * oplane + o] = acc;
  }
}

// Gradient of the sample with respect to the CPAB coordinates (lam) and,
// with GD, the image (scattered into gimg).
template <int ND, bool GD>
__device__ __forceinline__ void sample_bwd(const float *__restrict__ img,
                                           const float *__restrict__ gout,
                                           float *__restrict__ gimg, int C, int64_t plane,
                                           int64_t oplane, int64_t o, const Taps<ND> &t,
                                           float (&lam)[ND]) {
  float gk[ND];
#pragma unroll
  for (int k = 0; k < ND; ++k) gk[k] = 0.0f;
  for (int c = 0; c < C; ++c) {
    const float *d = img + (int64_t)c * plane;
    const float g = __ldg(gout + (int64_t)c * oplane + o);
    float v[1 << ND];
#pragma unroll
    for (int m = 0; m < (1 << ND); ++m) v[m] = (t.in >> m & 1u) ? __ldg(d + t.off[m]) : 0.0f;
#pragma unroll
    for (int m = 0; m < (1 << ND); ++m) {
      if (!(t.in >> m & 1u)) continue;
      if constexpr (GD) atomicAdd(gimg + (int64_t)c * plane + t.off[m], __fmul_rn(t.w[m], g));
      // d(weight)/d(index_k): +/- the product of the other axes' factors, in
      // grid_sample's order (last axis first), starting from the value.
#pragma unroll
      for (int kk = ND - 1; kk >= 0; --kk) {  // grid axes x, y(, z): gix, giy(, giz)
        float a = v[m];
#pragma unroll
        for (int j = ND - 1; j >= 0; --j) {
          if (j == kk) continue;
          const bool hj = (m >> (ND - 1 - j)) & 1;
          a = __fmul_rn(a, hj ? t.fh[j] : t.fl[j]);
        }
        const bool hk = (m >> (ND - 1 - kk)) & 1;
        gk[kk] = __fmaf_rn(hk ? a : -a, g, gk[kk]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < ND; ++k) lam[k] = __fmul_rn(2.0f, __fmul_rn(t.mult[k], gk[k]));
}

// Points: the meshgrid of out_size (axis values m.axes, the STN's pixel
// centres in CPAB coordinates), processed in the order m.order; K stages
// (a.n_stages) with stage inputs kept by slot; the result sampled from
// transformation b's image (or the shared one).
template <int ND, bool GD> struct WarpSrc {
  const MeshArgs &m;
  int64_t P, plane, sp_stride;
  const float *img;
  float *gimg;
  float *gt;
  float *sp;
  float *out;
  const float *gout;
  int n[3];
  __device__ WarpSrc(const IntegrateArgs &a, const MeshArgs &m_, int b) : m(m_) {
    P = m.out_size[0] * m.out_size[1] * (ND == 3 ? m.out_size[2] : 1);
    plane = (int64_t)m.in_size[0] * m.in_size[1] * (ND == 3 ? m.in_size[2] : 1);
    img = m.data + (int64_t)b * m.data_bstride;
    gimg = GD ? m.grad_data + (int64_t)b * m.data_bstride : nullptr;
    gt = m.grid_t + (int64_t)b * ND * P;
    sp = a.stage_points ? a.stage_points + (int64_t)b * ND * P : nullptr;
    sp_stride = (int64_t)a.n_theta * ND * P;
    out = m.out ? m.out + (int64_t)b * m.C * P : nullptr;
    gout = m.grad_out ? m.grad_out + (int64_t)b * m.C * P : nullptr;
    n[0] = m.in_size[0];
    n[1] = m.in_size[1];
    n[2] = m.in_size[2];
  }
  __device__ int64_t count() const { return P; }
  __device__ int64_t item(int64_t slot) const { return point_of(m.order, slot); }
  __device__ void start(int64_t, int64_t o, float (&p)[ND]) const { mesh_point<ND>(m, o, p); }
  __device__ void start_stage(int st, int64_t slot, int64_t o, float (&p)[ND]) const {
    if (st == 0) return start(slot, o, p);
    const float *q = sp + (st - 1) * sp_stride + slot;
#pragma unroll
    for (int k = 0; k < ND; ++k) p[k] = q[k * P];
  }
  __device__ void save_stage(int st, int64_t slot, const float (&p)[ND]) const {
    float *q = sp + st * sp_stride + slot;
#pragma unroll
    for (int k = 0; k < ND; ++k) q[k * P] = p[k];
  }
  __device__ void finish(int64_t slot, int64_t o, const float (&p)[ND]) const {
#pragma unroll
    for (int k = 0; k < ND; ++k) gt[k * P + slot] = p[k];
    const Taps<ND> t = make_taps<ND, false>(p, n, m.padding);
    sample_fwd<ND>(img, out, m.C, plane, P, o, t);
  }
  __device__ void lambda(int64_t slot, int64_t o, float (&lam)[ND]) const {
    float g[ND];
#pragma unroll
    for (int k = 0; k < ND; ++k) g[k] = __ldg(gt + k * P + slot);
    const Taps<ND> t = make_taps<ND, true>(g, n, m.padding);
    sample_bwd<ND, GD>(img, gout, gimg, m.C, plane, P, o, t, lam);
  }
  __device__ void grad(int64_t, int64_t, const float (&)[ND]) const {}
};

// 2D forward blocks of 1024 threads: measured at the STN 2D layer's shape (32 x 3 x 128^2,
// CUDA events) 84 -> 73 us for one transformation, 156 -> 140 us for two; 3D keeps 512.
template <int ND> struct WarpFwd { static constexpr int kThreads = ND == 2 ? 1024 : kFwdThreads; };

template <int ND, bool ADAPT, bool SMEM, bool CHAIN>
__global__ void __launch_bounds__(WarpFwd<ND>::kThreads) k_forward_warp(IntegrateArgs a, MeshArgs m) {
  forward_body<ND, ADAPT, SMEM, CHAIN>(a, WarpSrc<ND, false>(a, m, blockIdx.y));
}

template <int ND, bool ADAPT, bool A_SMEM, bool CL_SMEM, typename CellT, bool GD, bool CHAIN,
          bool WIDE = false>
__global__ void __launch_bounds__(BwdShape<ND, WIDE>::kThreads, BwdShape<ND, WIDE>::kMinBlocks)
    k_backward_warp(IntegrateArgs a, MeshArgs m) {
  backward_body<ND, ADAPT, A_SMEM, false, CL_SMEM, CellT, CHAIN, BwdShape<ND, WIDE>::kThreads,
                false>(a, WarpSrc<ND, GD>(a, m, blockIdx.y));
}

template <typename K>
cudaError_t launch_warp_kernel(K kernel, int threads, size_t smem, const IntegrateArgs &a,
                               const MeshArgs &m, cudaStream_t s) {
  const void *kp = reinterpret_cast<const void *>(kernel);
  const dim3 grid = wave_grid(kp, threads, smem, a.nP, a.n_theta, a.n_stages);
  kernel<<<grid, threads, smem, s>>>(a, m);
  return cudaGetLastError();
}

// Shared-memory choices as for the fused transform_data kernels; chains hold
// all their stages' tables in shared memory when they fit (the STN's small
// tessellations), else read them through L1/L2.
template <int ND, bool ADAPT>
cudaError_t warp_forward_nd(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s) {
  const size_t tab = (size_t)a.nC * Dim<ND>::kPpc * sizeof(float);
  if (a.n_stages > 1) {
    const size_t tabs = tab * (size_t)a.n_stages;
    if (tabs <= kFwdSmemBudget)
      return launch_warp_kernel(k_forward_warp<ND, ADAPT, true, true>, WarpFwd<ND>::kThreads, tabs, a, m, s);
    return launch_warp_kernel(k_forward_warp<ND, ADAPT, false, true>, WarpFwd<ND>::kThreads, 0, a, m, s);
  }
  if (tab <= kFwdSmemBudget)
    return launch_warp_kernel(k_forward_warp<ND, ADAPT, true, false>, WarpFwd<ND>::kThreads, tab, a, m, s);
  return launch_warp_kernel(k_forward_warp<ND, ADAPT, false, false>, WarpFwd<ND>::kThreads, 0, a, m, s);
}

template <int ND, bool ADAPT, typename CellT, bool GD>
cudaError_t warp_backward_cells(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s) {
  const size_t tab = (size_t)a.nC * Dim<ND>::kPpc * sizeof(float);
  constexpr int kT = BwdShape<ND>::kThreads;
  constexpr bool kCl = !ADAPT && sizeof(CellT) == 2;
  const size_t cl = kCl ? cell_record_bytes<ND, CellT>(kT, a.T) : 0;
  if (a.n_stages > 1) {
    const size_t tabs = tab * (size_t)a.n_stages;
    if constexpr (ND == 2 && kCl) {
      constexpr int kW = BwdShape<ND, true>::kThreads;
      const size_t cl_wide = (size_t)kW * a.T * sizeof(CellT);
      if (tabs + cl_wide <= kBwdWideSmemBudget)
        return launch_warp_kernel(k_backward_warp<ND, ADAPT, true, true, CellT, GD, true, true>,
                                  kW, tabs + cl_wide, a, m, s);
    }
    if (tabs <= kBwdSmemBudget) {
      if constexpr (kCl) {
        if (tabs + cl <= kBwdSmemBudget)
          return launch_warp_kernel(k_backward_warp<ND, ADAPT, true, true, CellT, GD, true>, kT,
                                    tabs + cl, a, m, s);
      }
      return launch_warp_kernel(k_backward_warp<ND, ADAPT, true, false, CellT, GD, true>, kT,
                                tabs, a, m, s);
    }
    if constexpr (kCl) {
      if (cl <= kBwdSmemBudget)
        return launch_warp_kernel(k_backward_warp<ND, ADAPT, false, true, CellT, GD, true>, kT,
                                  cl, a, m, s);
    }
    return launch_warp_kernel(k_backward_warp<ND, ADAPT, false, false, CellT, GD, true>, kT, 0,
                              a, m, s);
  }
  if constexpr (ND == 2 && kCl) {
    constexpr int kW = BwdShape<ND, true>::kThreads;
    const size_t cl_wide = (size_t)kW * a.T * sizeof(CellT);
    if (tab + cl > kBwdSmemBudget && tab + cl_wide <= kBwdWideSmemBudget)
      return launch_warp_kernel(k_backward_warp<ND, ADAPT, true, true, CellT, GD, false, true>,
                                kW, tab + cl_wide, a, m, s);
  }
  if (tab <= kBwdSmemBudget) {
    if constexpr (kCl) {
      if (tab + cl <= kBwdSmemBudget)
        return launch_warp_kernel(k_backward_warp<ND, ADAPT, true, true, CellT, GD, false>, kT,
                                  tab + cl, a, m, s);
    }
    return launch_warp_kernel(k_backward_warp<ND, ADAPT, true, false, CellT, GD, false>, kT, tab,
                              a, m, s);
  }
  if constexpr (kCl) {
    if (cl <= kBwdSmemBudget)
      return launch_warp_kernel(k_backward_warp<ND, ADAPT, false, true, CellT, GD, false>, kT, cl,
                                a, m, s);
  }
  return launch_warp_kernel(k_backward_warp<ND, ADAPT, false, false, CellT, GD, false>, kT, 0, a,
                            m, s);
}

template <int ND, bool ADAPT, bool GD>
cudaError_t warp_backward_nd(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s) {
  if (ADAPT || a.nC <= 65535) return warp_backward_cells<ND, ADAPT, uint16_t, GD>(a, m, s);
  return warp_backward_cells<ND, ADAPT, int32_t, GD>(a, m, s);
}

}  // namespace

cudaError_t launch_warp(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s) {
  if (a.ndim == 2) return a.adaptive ? warp_forward_nd<2, true>(a, m, s)
                                     : warp_forward_nd<2, false>(a, m, s);
  return a.adaptive ? warp_forward_nd<3, true>(a, m, s) : warp_forward_nd<3, false>(a, m, s);
}

cudaError_t launch_warp_backward(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s) {
  const bool gd = m.grad_data != nullptr;
  if (a.ndim == 2) {
    if (a.adaptive) return gd ? warp_backward_nd<2, true, true>(a, m, s)
                              : warp_backward_nd<2, true, false>(a, m, s);
    return gd ? warp_backward_nd<2, false, true>(a, m, s) : warp_backward_nd<2, false, false>(a, m, s);
  }
  if (a.adaptive) return gd ? warp_backward_nd<3, true, true>(a, m, s)
                            : warp_backward_nd<3, true, false>(a, m, s);
  return gd ? warp_backward_nd<3, false, true>(a, m, s) : warp_backward_nd<3, false, false>(a, m, s);
}

}  // namespace cpab
