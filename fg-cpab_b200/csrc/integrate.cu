// CPA trajectory integration on sm_100a: forward (1D closed form, 2D/3D
// exact per-cell steps) and the fused factorized-adjoint backward.
//
// Design (one CUDA thread per (point, transformation) pair, as in the
// reference, but):
//   * grids are sized to one resident wave (occupancy x SM count); blocks
//     stride over the points of one transformation, so the per-transformation
//     cell tables are staged into shared memory once per block, not per 256
//     points;
//   * cell tables live in shared memory when they fit (padded to 128-bit
//     rows), else they are read through the read-only cache with vector loads;
//   * the adjoint checkpoints every kSegSteps steps and records each step's
//     cell, replays one segment at a time into registers, and flushes a
//     thread's per-cell moments with vector L2 reductions only when its cell
//     changes.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "integrate_body.cuh"
#include "launch.h"
#include "resample_device.cuh"

namespace cpab {

namespace {

// transform_grid: points [ndim, nP] (or batched), results [n_theta, ndim, nP].
template <int ND> struct PointSrc {
  const float *pin;
  float *pout;
  const int32_t *ord;
  int64_t nP;
  const float *gin;
  float *gp;
  float *sp;          // stage inputs of this transformation, stage 1
  int64_t sp_stride;  // between stages
  __device__ PointSrc(const IntegrateArgs &a, int b)
      : pin(a.points + (a.batched ? (int64_t)b * ND * a.nP : 0)),
        pout(a.out ? a.out + (int64_t)b * ND * a.nP : nullptr),
        ord(a.order ? a.order + (a.batched ? (int64_t)b * a.nP : 0) : nullptr),
        nP(a.nP),
        gin(a.grad_out ? a.grad_out + (int64_t)b * ND * a.nP : nullptr),
        gp(a.grad_points ? a.grad_points + (int64_t)b * ND * a.nP : nullptr),
        sp(a.stage_points ? a.stage_points + (int64_t)b * ND * a.nP : nullptr),
        sp_stride((int64_t)a.n_theta * ND * a.nP) {}
  __device__ int64_t count() const { return nP; }
  __device__ int64_t item(int64_t slot) const { return point_of(ord, slot); }
  __device__ void start(int64_t, int64_t i, float (&p)[ND]) const {
#pragma unroll
    for (int k = 0; k < ND; ++k) p[k] = __ldg(pin + k * nP + i);
  }
  __device__ void start_stage(int st, int64_t slot, int64_t i, float (&p)[ND]) const {
    if (st == 0) return start(slot, i, p);
    const float *q = sp + (st - 1) * sp_stride + slot;
#pragma unroll
    for (int k = 0; k < ND; ++k) p[k] = q[k * nP];
  }
  __device__ void save_stage(int st, int64_t slot, const float (&p)[ND]) const {
    float *q = sp + st * sp_stride + slot;
#pragma unroll
    for (int k = 0; k < ND; ++k) q[k * nP] = p[k];
  }
  __device__ void finish(int64_t, int64_t i, const float (&p)[ND]) const {
#pragma unroll
    for (int k = 0; k < ND; ++k) pout[k * nP + i] = p[k];
  }
  __device__ void lambda(int64_t, int64_t i, float (&lam)[ND]) const {
#pragma unroll
    for (int k = 0; k < ND; ++k) lam[k] = __ldg(gin + k * nP + i);
  }
  __device__ void grad(int64_t, int64_t i, const float (&lam)[ND]) const {
    if (gp) {
#pragma unroll
      for (int k = 0; k < ND; ++k) gp[k * nP + i] = lam[k];
    }
  }
};

// transform_data (2D/3D): the uniform meshgrid of out_size, output point o =
// order[slot] (the library passes the meshgrid sorted by initial cell; NULL:
// output order); forward writes the integrated grid (at the slot: coalesced)
// and resamples every channel of data at it
// (cpab/cpab.py:306-308 = transform_grid then interpolate); backward forms the
// upstream gradient from the resample gradient at the saved grid, as the
// unfused autograd graph does (GD: also scatter grad_data).
template <int ND, bool GD> struct MeshSrc {
  const MeshArgs &m;
  int64_t P, bc0, plane;
  float *gt;
  int in[3];
  __device__ MeshSrc(const IntegrateArgs &a, const MeshArgs &m_, int b) : m(m_) {
    P = m.out_size[0] * m.out_size[1] * (ND == 3 ? m.out_size[2] : 1);
    bc0 = (int64_t)b * m.C;
    plane = (int64_t)m.in_size[0] * m.in_size[1] * (ND == 3 ? m.in_size[2] : 1);
    gt = m.grid_t + (int64_t)b * ND * P;
    in[0] = m.in_size[0];
    in[1] = m.in_size[1];
    in[2] = m.in_size[2];
  }
  __device__ int64_t count() const { return P; }
  __device__ int64_t item(int64_t slot) const { return point_of(m.order, slot); }
  __device__ void start(int64_t, int64_t o, float (&p)[ND]) const { mesh_point<ND>(m, o, p); }
  __device__ void start_stage(int, int64_t slot, int64_t o, float (&p)[ND]) const {
    start(slot, o, p);
  }
  __device__ void save_stage(int, int64_t, const float (&)[ND]) const {}
  __device__ void finish(int64_t slot, int64_t o, const float (&p)[ND]) const {
#pragma unroll
    for (int k = 0; k < ND; ++k) gt[k * P + slot] = p[k];
    const rs::Corners<ND> cr = rs::corners<ND>(p, in);
    rs::point_fwd<ND>(m.data, m.out, m.C, bc0, plane, P, o, cr);
  }
  __device__ void lambda(int64_t slot, int64_t o, float (&lam)[ND]) const {
    float g[ND];
#pragma unroll
    for (int k = 0; k < ND; ++k) g[k] = __ldg(gt + k * P + slot);
    const rs::Corners<ND> cr = rs::corners<ND>(g, in);
    float gw[ND];
    rs::point_bwd<ND, GD>(m.data, m.grad_out, m.grad_data, m.C, bc0, plane, P, o, cr, gw);
#pragma unroll
    for (int k = 0; k < ND; ++k) lam[k] = __fmul_rn(gw[k], (float)(in[k] - 1));
  }
  __device__ void grad(int64_t, int64_t, const float (&)[ND]) const {}
};

// ---------------------------------------------------------------------------
// 1D closed form.  cpab/core/cpab_ops_1d.cu:103-205.
// ---------------------------------------------------------------------------

__device__ __forceinline__ int sgn(float x) { return (x > 0.0f) - (x < 0.0f); }
__device__ __forceinline__ bool near0(float x) { return fabsf(x) < 1e-7f; }

// Time for the flow x' = a x + b started at x in cell c to reach the facet it
// moves towards (shifted 1e-7 past it); +-inf when it never does.  Writes the
// hit position and the next cell.
__device__ __forceinline__ float hit_time_1d(float x, float t, int c, float a, float b, int nx,
                                             float fnx, float &xc, int &cc) {
  const int s = sgn(t);
  const float never = INFINITY * (float)s;
  const float v = __fmaf_rn(a, x, b);
  if (near0(v)) return never;
  cc = c + sgn(v) * s;
  if (cc < 0 || cc >= nx) return never;
  // Moving right in time-forward direction exits through the right facet.
  if ((v > 0.0f) == (t > 0.0f)) xc = ((float)(c + 1) / fnx) + 1e-7f;
  else xc = ((float)c / fnx) - 1e-7f;
  const float vc = __fmaf_rn(a, xc, b);
  if (near0(vc)) return never;
  if (sgn(v) != sgn(vc)) return never;
  if (xc <= 0.0f || xc >= 1.0f) return never;
  if (near0(a)) return (xc - x) / b;
  return logf(vc / v) / a;
}

// psi(x, t) = e^{ta} (x + b/a) - b/a  (x + t b when a ~ 0).
__device__ __forceinline__ float flow_1d(float x, float t, float a, float b) {
  if (near0(a)) return __fmaf_rn(t, b, x);
  const float ba = b / a;
  return __fmaf_rn(expf(t * a), x + ba, -ba);
}

template <bool SMEM>
__global__ void __launch_bounds__(kFwdThreads) k_forward_1d(IntegrateArgs a) {
  extern __shared__ float4 smem4[];
  float *s_tab = reinterpret_cast<float *>(smem4);
  const int b = blockIdx.y;
  const float *ag = a.As + (int64_t)b * a.nC * 2;
  if constexpr (SMEM) {
    for (int i = threadIdx.x; i < a.nC * 2; i += blockDim.x) s_tab[i] = __ldg(ag + i);
    __syncthreads();
  }
  const float2 *tab = reinterpret_cast<const float2 *>(SMEM ? s_tab : ag);
  const float *pin = a.points + (a.batched ? (int64_t)b * a.nP : 0);
  float *pout = a.out + (int64_t)b * a.nP;
  const int32_t *ord = a.order ? a.order + (a.batched ? (int64_t)b * a.nP : 0) : nullptr;
  const Tess t = a.tess;
  const int nx = t.nx;
  for (int64_t slot = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; slot < a.nP;
       slot += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = point_of(ord, slot);
    float x = __ldg(pin + i);
    float tr = 1.0f;
    int c = cell_of(t, x);
    const int max_hops = max(c, nx - 1 - c) + 1;
    int hops = 0;
    float res;
    while (true) {
      const float2 ab = SMEM ? tab[c] : __ldg(tab + c);
      float xc = x;
      int cc = c;
      const float th = hit_time_1d(x, tr, c, ab.x, ab.y, nx, t.fx, xc, cc);
      const float sf = (float)sgn(tr);
      if (sf * th > sf * tr) {
        res = flow_1d(x, tr, ab.x, ab.y);
        break;
      }
      x = xc;
      c = cc;
      tr -= th;
      if (++hops > max_hops) {
        res = x;
        break;
      }
    }
    pout[i] = res;
  }
}

template <int ND, bool ADAPT, bool SMEM, bool CHAIN = false>
__global__ void __launch_bounds__(FwdShape<ND, ADAPT, SMEM, CHAIN>::kThreads)
    k_forward(IntegrateArgs a) {
  forward_body<ND, ADAPT, SMEM, CHAIN>(a, PointSrc<ND>(a, blockIdx.y));
}

template <int ND, bool ADAPT, bool SMEM>
__global__ void __launch_bounds__(kFwdThreads) k_forward_mesh(IntegrateArgs a, MeshArgs m) {
  forward_body<ND, ADAPT, SMEM, false>(a, MeshSrc<ND, false>(a, m, blockIdx.y));
}

// 2D: two resident 1024-thread blocks per SM (32 registers, a few spilled
// values, in the once-per-point resample), twice the 1024 threads that 46
// registers allow.  Measured at the dense 2D shape (32 x 3 x 512^2, 30 x 30,
// CUDA events): forward 0.605 -> 0.568 ms.  3D keeps the compiler's choice
// (the same target slowed it, 0.96 -> 1.18 ms).
template <bool ADAPT, bool SMEM>
__global__ void __launch_bounds__(1024, 2) k_forward_mesh_2d(IntegrateArgs a, MeshArgs m) {
  forward_body<2, ADAPT, SMEM, false>(a, MeshSrc<2, false>(a, m, blockIdx.y));
}

template <int ND, bool ADAPT, bool A_SMEM, bool M_SMEM, bool CL_SMEM, typename CellT,
          bool CHAIN = false, bool WIDE = false>
__global__ void __launch_bounds__(BwdShape<ND, WIDE>::kThreads, BwdShape<ND, WIDE>::kMinBlocks)
    k_backward(IntegrateArgs a) {
  backward_body<ND, ADAPT, A_SMEM, M_SMEM, CL_SMEM, CellT, CHAIN, BwdShape<ND, WIDE>::kThreads,
                ND == 2>(a, PointSrc<ND>(a, blockIdx.y));
}

// Fused transform_data backward; GD: also the data gradient.  WIDE as for
// k_backward: one 1024-thread block per SM holding one copy of the table.
template <int ND, bool ADAPT, bool A_SMEM, bool CL_SMEM, typename CellT, bool GD, bool WIDE = false>
__global__ void __launch_bounds__(BwdShape<ND, WIDE>::kThreads, BwdShape<ND, WIDE>::kMinBlocks)
    k_backward_mesh(IntegrateArgs a, MeshArgs m) {
  backward_body<ND, ADAPT, A_SMEM, false, CL_SMEM, CellT, false, BwdShape<ND, WIDE>::kThreads,
                false>(a, MeshSrc<ND, GD>(a, m, blockIdx.y));
}

// ---------------------------------------------------------------------------
// Cell lookup of a point set (the lookup the integrators use, exposed).
// ---------------------------------------------------------------------------

template <int ND>
__global__ void k_cell_index(Tess t, const float *__restrict__ pts, int64_t n,
                             int32_t *__restrict__ cells) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float p[ND];
#pragma unroll
    for (int k = 0; k < ND; ++k) p[k] = __ldg(pts + k * n + i);
    cells[i] = lookup<ND>(t, p);
  }
}

// ---------------------------------------------------------------------------
// Spatial ordering: a counting sort of the points of every set by initial
// cell, so that the threads of a warp start in the same or neighbouring cells
// (shared-memory broadcasts instead of bank conflicts, warp-aggregated moment
// flushes).  counts is [n_sets, nC] int32 scratch.
// ---------------------------------------------------------------------------

// Histogram of initial cells.  With SMEM, each block counts its contiguous
// chunk of points in shared memory and adds its non-zero bins to the global
// counts (one atomic per block and non-empty cell instead of one per point).
template <int ND, bool SMEM>
__global__ void k_cell_histogram(Tess t, const float *__restrict__ pts, int64_t nP, int nC,
                                 int32_t *__restrict__ counts) {
  extern __shared__ int32_t s_cnt[];
  const int set = blockIdx.y;
  const float *p0 = pts + (int64_t)set * ND * nP;
  int32_t *cnt = counts + (int64_t)set * nC;
  const int64_t chunk = (nP + gridDim.x - 1) / gridDim.x;
  const int64_t lo = blockIdx.x * chunk, hi = min(nP, lo + chunk);
  if constexpr (SMEM) {
    for (int c = threadIdx.x; c < nC; c += blockDim.x) s_cnt[c] = 0;
    __syncthreads();
  }
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    float p[ND];
#pragma unroll
    for (int k = 0; k < ND; ++k) p[k] = __ldg(p0 + k * nP + i);
    atomicAdd((SMEM ? s_cnt : cnt) + lookup<ND>(t, p), 1);
  }
  if constexpr (SMEM) {
    __syncthreads();
    for (int c = threadIdx.x; c < nC; c += blockDim.x)
      if (s_cnt[c]) atomicAdd(cnt + c, s_cnt[c]);
  }
}

// Exclusive prefix sum of each set's nC counts, in place; one block per set.
__global__ void __launch_bounds__(1024) k_exclusive_scan(int32_t *__restrict__ counts, int nC) {
  __shared__ int32_t part[1024];
  int32_t *cnt = counts + (int64_t)blockIdx.x * nC;
  const int per = (nC + blockDim.x - 1) / blockDim.x;
  const int lo = min(nC, (int)threadIdx.x * per), hi = min(nC, lo + per);
  int32_t sum = 0;
  for (int c = lo; c < hi; ++c) sum += cnt[c];
  part[threadIdx.x] = sum;
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {  // Hillis-Steele inclusive scan
    const int32_t v = threadIdx.x >= (unsigned)off ? part[threadIdx.x - off] : 0;
    __syncthreads();
    part[threadIdx.x] += v;
    __syncthreads();
  }
  int32_t run = part[threadIdx.x] - sum;
  for (int c = lo; c < hi; ++c) {
    const int32_t v = cnt[c];
    cnt[c] = run;
    run += v;
  }
}

// Scatter the points to their sorted positions.  With SMEM, each block counts
// its chunk per cell in shared memory, reserves one range per non-empty cell
// with a single global atomic, then places its points inside those ranges.
template <int ND, bool SMEM>
__global__ void k_cell_scatter(Tess t, const float *__restrict__ pts, int64_t nP, int nC,
                               int32_t *__restrict__ offsets, int32_t *__restrict__ order) {
  extern __shared__ int32_t s_cnt[];
  const int set = blockIdx.y;
  const float *p0 = pts + (int64_t)set * ND * nP;
  int32_t *off = offsets + (int64_t)set * nC;
  int32_t *ord = order + (int64_t)set * nP;
  const int64_t chunk = (nP + gridDim.x - 1) / gridDim.x;
  const int64_t lo = blockIdx.x * chunk, hi = min(nP, lo + chunk);
  if constexpr (SMEM) {
    for (int c = threadIdx.x; c < nC; c += blockDim.x) s_cnt[c] = 0;
    __syncthreads();
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      float p[ND];
#pragma unroll
      for (int k = 0; k < ND; ++k) p[k] = __ldg(p0 + k * nP + i);
      atomicAdd(s_cnt + lookup<ND>(t, p), 1);
    }
    __syncthreads();
    for (int c = threadIdx.x; c < nC; c += blockDim.x) {
      const int32_t n = s_cnt[c];
      s_cnt[c] = n ? atomicAdd(off + c, n) : 0;  // this block's first slot in cell c
    }
    __syncthreads();
  }
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    float p[ND];
#pragma unroll
    for (int k = 0; k < ND; ++k) p[k] = __ldg(p0 + k * nP + i);
    ord[atomicAdd((SMEM ? s_cnt : off) + lookup<ND>(t, p), 1)] = (int32_t)i;
  }
}

template <int ND>
cudaError_t forward_nd(const IntegrateArgs &a, cudaStream_t s) {
  const size_t tab = (size_t)a.nC * Dim<ND>::kPpc * sizeof(float);
  if constexpr (ND > 1) {
    if (a.n_stages > 1) {  // fused chain: all stages' tables in shared memory when they fit
      const size_t tabs = tab * (size_t)a.n_stages;
      if (tabs <= kFwdSmemBudget)
        return a.adaptive ? launch_wave(k_forward<ND, true, true, true>, kFwdThreads, tabs, a, s)
                          : launch_wave(k_forward<ND, false, true, true>, kFwdThreads, tabs, a, s);
      return a.adaptive ? launch_wave(k_forward<ND, true, false, true>, kFwdThreads, 0, a, s)
                        : launch_wave(k_forward<ND, false, false, true>, kFwdThreads, 0, a, s);
    }
  }
  const bool smem = tab <= kFwdSmemBudget;
  if (a.adaptive) {
    return smem ? launch_wave(k_forward<ND, true, true>, kFwdThreads, tab, a, s)
                : launch_wave(k_forward<ND, true, false>, kFwdThreads, 0, a, s);
  }
  return smem ? launch_wave(k_forward<ND, false, true>, FwdShape<ND, false, true, false>::kThreads,
                            tab, a, s)
              : launch_wave(k_forward<ND, false, false>, kFwdThreads, 0, a, s);
}

template <int ND, bool ADAPT, bool A_SMEM, bool M_SMEM, typename CellT>
cudaError_t backward_launch(const IntegrateArgs &a, size_t smem, size_t cl, cudaStream_t s) {
  constexpr int kT = BwdShape<ND>::kThreads;
  if constexpr (!ADAPT && sizeof(CellT) == 2) {
    if (cl > 0)
      return launch_wave(k_backward<ND, ADAPT, A_SMEM, M_SMEM, true, CellT>, kT, smem + cl, a, s);
  }
  return launch_wave(k_backward<ND, ADAPT, A_SMEM, M_SMEM, false, CellT>, kT, smem, a, s);
}

// Fused chains (stage after stage per thread): all stages' tables (tabs
// bytes) in shared memory when they fit beside the cell record -- in 2D one
// 1024-thread block per SM, as for single transformations -- else in global
// memory.
template <int ND, bool ADAPT, typename CellT>
cudaError_t backward_chain_launch(const IntegrateArgs &a, size_t tabs, size_t cl,
                                  cudaStream_t s) {
  constexpr int kT = BwdShape<ND>::kThreads;
  if constexpr (ND == 2 && !ADAPT && sizeof(CellT) == 2) {
    constexpr int kW = BwdShape<ND, true>::kThreads;
    const size_t cl_wide = (size_t)kW * a.T * sizeof(CellT);
    if (tabs + cl_wide <= kBwdWideSmemBudget)
      return launch_wave(k_backward<ND, false, true, false, true, CellT, true, true>, kW,
                         tabs + cl_wide, a, s);
  }
  if (tabs <= kBwdSmemBudget) {
    if constexpr (!ADAPT && sizeof(CellT) == 2) {
      if (cl > 0 && tabs + cl <= kBwdSmemBudget)
        return launch_wave(k_backward<ND, ADAPT, true, false, true, CellT, true>, kT, tabs + cl,
                           a, s);
    }
    return launch_wave(k_backward<ND, ADAPT, true, false, false, CellT, true>, kT, tabs, a, s);
  }
  if constexpr (!ADAPT && sizeof(CellT) == 2) {
    if (cl > 0)
      return launch_wave(k_backward<ND, ADAPT, false, false, true, CellT, true>, kT, cl, a, s);
  }
  return launch_wave(k_backward<ND, ADAPT, false, false, false, CellT, true>, kT, 0, a, s);
}

template <int ND, bool ADAPT, typename CellT>
cudaError_t backward_cells(const IntegrateArgs &a, cudaStream_t s) {
  const size_t tab = (size_t)a.nC * Dim<ND>::kPpc * sizeof(float);
  if constexpr (ND == 2 && !ADAPT && sizeof(CellT) == 2) {
    constexpr int kW = BwdShape<ND, true>::kThreads;
    const size_t cl_wide = (size_t)kW * a.T * sizeof(CellT);
    if (a.n_stages == 1 && tab + cl_wide <= kBwdWideSmemBudget)
      return launch_wave(k_backward<ND, false, true, false, true, CellT, false, true>, kW,
                         tab + cl_wide, a, s);
  }
  constexpr int kT = BwdShape<ND>::kThreads;
  // Shared memory, in order of preference: the cell table, the 1D moment
  // table, the 16-bit cell record (when all of it fits the budget).
  const size_t cl_bytes = (ADAPT || sizeof(CellT) != 2) ? 0 : cell_record_bytes<ND, CellT>(kT, a.T);
  auto cl_fits = [&](size_t used) { return used + cl_bytes <= kBwdSmemBudget ? cl_bytes : 0; };
  if constexpr (ND == 1) {
    if (2 * tab <= kBwdSmemBudget)
      return backward_launch<ND, ADAPT, true, true, CellT>(a, 2 * tab, cl_fits(2 * tab), s);
  }
  if constexpr (ND > 1) {
    if (a.n_stages > 1)
      return backward_chain_launch<ND, ADAPT, CellT>(a, tab * (size_t)a.n_stages, cl_fits(0), s);
  }
  if (tab <= kBwdSmemBudget)
    return backward_launch<ND, ADAPT, true, false, CellT>(a, tab, cl_fits(tab), s);
  return backward_launch<ND, ADAPT, false, false, CellT>(a, 0, cl_fits(0), s);
}

// Fused transform_data launches (2D/3D): same shared-memory choices as the
// transform_grid kernels.
template <int ND, bool ADAPT>
cudaError_t mesh_forward_nd(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s) {
  const size_t tab = (size_t)a.nC * Dim<ND>::kPpc * sizeof(float);
  if constexpr (ND == 2) {
    if (tab <= kFwdSmemBudget)
      return launch_wave_args(k_forward_mesh_2d<ADAPT, true>, 1024, tab, a, m, s);
    return launch_wave_args(k_forward_mesh_2d<ADAPT, false>, 1024, 0, a, m, s);
  }
  if (tab <= kFwdSmemBudget)
    return launch_wave_args(k_forward_mesh<ND, ADAPT, true>, kFwdThreads, tab, a, m, s);
  return launch_wave_args(k_forward_mesh<ND, ADAPT, false>, kFwdThreads, 0, a, m, s);
}

template <int ND, bool ADAPT, typename CellT, bool GD>
cudaError_t mesh_backward_cells(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s) {
  const size_t tab = (size_t)a.nC * Dim<ND>::kPpc * sizeof(float);
  constexpr int kT = BwdShape<ND>::kThreads;
  constexpr bool kCl = !ADAPT && sizeof(CellT) == 2;
  const size_t cl = kCl ? cell_record_bytes<ND, CellT>(kT, a.T) : 0;
  if constexpr (ND == 2 && kCl) {
    // 2D: the table and the cell record of 1024 threads in one block when
    // they fit (the 30 x 30 table beside a 512-thread record does not fit
    // two blocks' budget, and the record would go to local memory).
    constexpr int kW = BwdShape<ND, true>::kThreads;
    const size_t cl_wide = (size_t)kW * a.T * sizeof(CellT);
    if (tab + cl > kBwdSmemBudget && tab + cl_wide <= kBwdWideSmemBudget)
      return launch_wave_args(k_backward_mesh<ND, ADAPT, true, true, CellT, GD, true>, kW,
                              tab + cl_wide, a, m, s);
  }
  if (tab <= kBwdSmemBudget) {
    if constexpr (kCl) {
      if (tab + cl <= kBwdSmemBudget)
        return launch_wave_args(k_backward_mesh<ND, ADAPT, true, true, CellT, GD>, kT, tab + cl,
                                a, m, s);
    }
    return launch_wave_args(k_backward_mesh<ND, ADAPT, true, false, CellT, GD>, kT, tab, a, m, s);
  }
  if constexpr (kCl) {
    if (cl <= kBwdSmemBudget)
      return launch_wave_args(k_backward_mesh<ND, ADAPT, false, true, CellT, GD>, kT, cl, a, m, s);
  }
  return launch_wave_args(k_backward_mesh<ND, ADAPT, false, false, CellT, GD>, kT, 0, a, m, s);
}

template <int ND, bool ADAPT, bool GD>
cudaError_t mesh_backward_nd(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s) {
  if (ADAPT || a.nC <= 65535) return mesh_backward_cells<ND, ADAPT, uint16_t, GD>(a, m, s);
  return mesh_backward_cells<ND, ADAPT, int32_t, GD>(a, m, s);
}

template <int ND, bool ADAPT>
cudaError_t backward_nd(const IntegrateArgs &a, cudaStream_t s) {
  if (ADAPT || a.nC <= 65535) return backward_cells<ND, ADAPT, uint16_t>(a, s);
  return backward_cells<ND, ADAPT, int32_t>(a, s);
}

}  // namespace

const DeviceInfo &device_info() {
  static DeviceInfo info[64];
  static bool init[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  std::lock_guard<std::mutex> lock(mu);
  if (!init[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    info[dev].sm_count = v > 0 ? v : 1;
    v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    info[dev].max_smem_optin = v > 0 ? v : 48 * 1024;
    init[dev] = true;
  }
  return info[dev];
}

cudaError_t launch_cell_index(int ndim, Tess t, const float *points, int64_t n, int32_t *cells,
                              cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = (int64_t)device_info().sm_count * 8;
  if (blocks > cap) blocks = cap;
  switch (ndim) {
    case 1: k_cell_index<1><<<(unsigned)blocks, 256, 0, s>>>(t, points, n, cells); break;
    case 2: k_cell_index<2><<<(unsigned)blocks, 256, 0, s>>>(t, points, n, cells); break;
    default: k_cell_index<3><<<(unsigned)blocks, 256, 0, s>>>(t, points, n, cells); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_order_points(int ndim, Tess t, const float *points, int64_t nP, int n_sets,
                                int nC, int32_t *counts, int32_t *order, cudaStream_t s) {
  if (nP == 0 || n_sets == 0) return cudaSuccess;
  cudaError_t e = cudaMemsetAsync(counts, 0, (size_t)n_sets * nC * sizeof(int32_t), s);
  if (e != cudaSuccess) return e;
  // Shared-memory counts when the cell table fits.
  const size_t smem = (size_t)nC * sizeof(int32_t);
  const bool use_smem = smem <= 128 * 1024;
  int64_t bx;
  if (use_smem) {
    // 1024 points per block, at most two blocks per SM.  (Sizing blocks by the
    // cell count instead, to keep each block's flush of nC bins small, starved
    // the GPU: 7 blocks for 614k points over 20,480 cells took 263 us, 1024
    // points per block 53 us; 125k points over 1,600 cells 31 -> 24 us.)
    bx = nP / 1024;
    const int64_t cap = (int64_t)device_info().sm_count * 2 / n_sets;
    bx = bx > cap ? cap : bx;
  } else {
    bx = (nP + 255) / 256;
    const int64_t cap = (int64_t)device_info().sm_count * 8;
    bx = bx > cap ? cap : bx;
  }
  if (bx < 1) bx = 1;
  const dim3 grid((unsigned)bx, (unsigned)n_sets);
  const int thr = use_smem ? 512 : 256;
  const size_t sm = use_smem ? smem : 0;
#define CPAB_ORDER_LAUNCH(KERNEL, ...)                                                     \
  do {                                                                                     \
    if (use_smem) {                                                                        \
      switch (ndim) {                                                                      \
        case 1: KERNEL<1, true><<<grid, thr, sm, s>>>(__VA_ARGS__); break;                 \
        case 2: KERNEL<2, true><<<grid, thr, sm, s>>>(__VA_ARGS__); break;                 \
        default: KERNEL<3, true><<<grid, thr, sm, s>>>(__VA_ARGS__); break;                \
      }                                                                                    \
    } else {                                                                               \
      switch (ndim) {                                                                      \
        case 1: KERNEL<1, false><<<grid, thr, 0, s>>>(__VA_ARGS__); break;                 \
        case 2: KERNEL<2, false><<<grid, thr, 0, s>>>(__VA_ARGS__); break;                 \
        default: KERNEL<3, false><<<grid, thr, 0, s>>>(__VA_ARGS__); break;                \
      }                                                                                    \
    }                                                                                      \
  } while (0)
  if (use_smem && smem > 48 * 1024) {
    for (auto k : {(const void *)k_cell_histogram<1, true>, (const void *)k_cell_histogram<2, true>,
                   (const void *)k_cell_histogram<3, true>, (const void *)k_cell_scatter<1, true>,
                   (const void *)k_cell_scatter<2, true>, (const void *)k_cell_scatter<3, true>})
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 1024);
  }
  CPAB_ORDER_LAUNCH(k_cell_histogram, t, points, nP, nC, counts);
  k_exclusive_scan<<<n_sets, 1024, 0, s>>>(counts, nC);
  CPAB_ORDER_LAUNCH(k_cell_scatter, t, points, nP, nC, counts, order);
#undef CPAB_ORDER_LAUNCH
  return cudaGetLastError();
}

cudaError_t launch_forward_1d(const IntegrateArgs &a, cudaStream_t s) {
  const size_t tab = (size_t)a.nC * 2 * sizeof(float);
  if (tab <= kFwdSmemBudget) return launch_wave(k_forward_1d<true>, kFwdThreads, tab, a, s);
  return launch_wave(k_forward_1d<false>, kFwdThreads, 0, a, s);
}

cudaError_t launch_forward(const IntegrateArgs &a, cudaStream_t s) {
  switch (a.ndim) {
    case 1: return launch_forward_1d(a, s);
    case 2: return forward_nd<2>(a, s);
    default: return forward_nd<3>(a, s);
  }
}

cudaError_t launch_transform_data(const IntegrateArgs &a, const MeshArgs &m, cudaStream_t s) {
  if (a.ndim == 2) return a.adaptive ? mesh_forward_nd<2, true>(a, m, s)
                                     : mesh_forward_nd<2, false>(a, m, s);
  return a.adaptive ? mesh_forward_nd<3, true>(a, m, s) : mesh_forward_nd<3, false>(a, m, s);
}

cudaError_t launch_transform_data_backward(const IntegrateArgs &a, const MeshArgs &m,
                                           cudaStream_t s) {
  const bool gd = m.grad_data != nullptr;
  if (a.ndim == 2) {
    if (a.adaptive) return gd ? mesh_backward_nd<2, true, true>(a, m, s)
                              : mesh_backward_nd<2, true, false>(a, m, s);
    return gd ? mesh_backward_nd<2, false, true>(a, m, s) : mesh_backward_nd<2, false, false>(a, m, s);
  }
  if (a.adaptive) return gd ? mesh_backward_nd<3, true, true>(a, m, s)
                            : mesh_backward_nd<3, true, false>(a, m, s);
  return gd ? mesh_backward_nd<3, false, true>(a, m, s) : mesh_backward_nd<3, false, false>(a, m, s);
}

cudaError_t launch_backward(const IntegrateArgs &a, cudaStream_t s) {
  switch (a.ndim) {
    case 1: return a.adaptive ? backward_nd<1, true>(a, s) : backward_nd<1, false>(a, s);
    case 2: return a.adaptive ? backward_nd<2, true>(a, s) : backward_nd<2, false>(a, s);
    default: return a.adaptive ? backward_nd<3, true>(a, s) : backward_nd<3, false>(a, s);
  }
}

}  // namespace cpab
