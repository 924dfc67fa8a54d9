// Device bodies shared by the integration kernels (integrate.cu) and the
// fused spatial-transformer warp (warp.cu): launch shapes, the point-source
// interface, the forward and adjoint-backward loops, and the wave-sized grid
// helpers.  Everything here has internal linkage: each translation unit
// instantiates the kernels it launches.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "launch.h"

namespace cpab {

namespace {


constexpr int kFwdThreads = 512;
// Forward launch shape.  The plain 2D forward with its table in shared memory
// runs 1024-thread blocks: half as many table copies per SM (the 30x30 table,
// 86 KB, then serves 2048 resident threads instead of 1024).  Measured on the
// bench shapes: 2D 20x20 136 -> 131 us, 30x30 532 -> 488 us; the fused
// transform_data and chain forwards were slower at 1024, 3D unchanged.
template <int ND, bool ADAPT, bool SMEM, bool CHAIN> struct FwdShape {
  static constexpr int kThreads = (ND == 2 && !ADAPT && SMEM && !CHAIN) ? 1024 : kFwdThreads;
};
// Backward launch shape: 2 resident blocks per SM; 3D keeps 256 threads per
// block so that its larger per-thread state fits without spilling.
// WIDE (2D, not adaptive, not chained, table and cell record both in shared
// memory): one 1024-thread block per SM instead, so the SM holds one copy of
// the cell table and leaves more of its 256 KB to L1, where the adjoint's
// checkpoints live (measured: 2D 20x20 390 -> 380 us, 30x30 1467 -> 1420 us;
// the fused transform_data backward did not change and keeps 2 x 512).
template <int ND, bool WIDE = false> struct BwdShape {
  static constexpr bool kWide = WIDE && ND == 2;
  static constexpr int kThreads = ND == 3 ? 256 : (kWide ? 1024 : 512);
  static constexpr int kMinBlocks = kWide ? 1 : 2;
};
constexpr size_t kBwdWideSmemBudget = 200 * 1024;
// Shared-memory budget per block for the cell table (two resident blocks per
// SM at the largest table).
constexpr size_t kFwdSmemBudget = 100 * 1024;
constexpr size_t kBwdSmemBudget = 110 * 1024;

// Point processed by thread slot i: order[set][i] when an order is given.
__device__ __forceinline__ int64_t point_of(const int32_t *__restrict__ order, int64_t i) {
  return order ? (int64_t)__ldg(order + i) : i;
}

// Output point o of the uniform meshgrid whose axis values are m.axes (axis 0,
// then axis 1 [, then axis 2]), o counted with the last axis fastest.
template <int ND>
__device__ __forceinline__ void mesh_point(const MeshArgs &m, int64_t o, float (&p)[ND]) {
  const int n1 = (int)m.out_size[1];
  const float *ax = m.axes;
  if constexpr (ND == 2) {
    const int i0 = (int)(o / n1), i1 = (int)(o - (int64_t)i0 * n1);
    p[0] = __ldg(ax + i0);
    p[1] = __ldg(ax + m.out_size[0] + i1);
  } else {
    const int n2 = (int)m.out_size[2];
    const int64_t r = o / n2;
    const int i2 = (int)(o - r * n2), i0 = (int)(r / n1), i1 = (int)(r - (int64_t)i0 * n1);
    p[0] = __ldg(ax + i0);
    p[1] = __ldg(ax + m.out_size[0] + i1);
    p[2] = __ldg(ax + m.out_size[0] + m.out_size[1] + i2);
  }
}

// Where the integration kernels' points come from and where results go.
//   count()               points per transformation
//   item(slot)            point handled by thread slot `slot`
//   start(slot, i, p)     initial position
//   start_stage(st, ...)  input of chain stage st (stage 0: start)
//   save_stage(st, ...)   forward: keep the input of chain stage st + 1
//   finish(slot, i, p)    forward: consume the integrated position
//   lambda(slot, i, lam)  backward: adjoint at t = 1 (the upstream gradient)
//   grad(slot, i, lam)    backward: consume lambda(0)

// ---------------------------------------------------------------------------
// 2D/3D forward: T exact steps p <- Trels[cell(p)] [p;1].
// cpab/core/cpab_ops_2d.cu:212-278, cpab/core/cpab_ops_3d.cu:169-241.
// ---------------------------------------------------------------------------

// CHAIN: a.n_stages transformations per point (fused chains; with SMEM all
// stages' tables are staged, one after another).  Without it the stage loop
// compiles away.
template <int ND, bool ADAPT, bool SMEM, bool CHAIN, class Src>
__device__ __forceinline__ void forward_body(const IntegrateArgs &a, const Src &src) {
  constexpr int P = Dim<ND>::kPpc;
  extern __shared__ float4 smem4[];
  float *s_tab = reinterpret_cast<float *>(smem4);
  const int b = blockIdx.y;
  if constexpr (SMEM) {  // a fused chain stages every stage's table, one after another
    if constexpr (CHAIN) {
      for (int st = 0; st < a.n_stages; ++st)
        stage_table<ND>(s_tab + (size_t)st * a.nC * P,
                        a.trels + ((int64_t)st * a.n_theta + b) * a.nC * P, a.nC);
    } else {
      stage_table<ND>(s_tab, a.trels + (int64_t)b * a.nC * P, a.nC);
    }
    __syncthreads();
  }
  const Tess t = a.tess;
  const int T = a.T;
  const float h_half = 0.5f * (1.0f / (float)T);
  const int64_t nP = src.count();
  const int nst = CHAIN ? a.n_stages : 1;
  for (int64_t slot = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; slot < nP;
       slot += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = src.item(slot);
    float p[ND];
    src.start(slot, i, p);
    for (int st = 0; st < nst; ++st) {
    const int64_t off = ((int64_t)st * a.n_theta + b) * a.nC * P;
    const float *tab = SMEM ? (CHAIN ? s_tab + (size_t)st * a.nC * P : s_tab) : a.trels + off;
    const float *ag = a.As + off;
    // Unrolled by a divisor of the usual T = 50 (loop control is ~4% of a step);
    // measured: 2D 139 -> 136 us, 3D 971 -> 940 us on the bench shapes.
#pragma unroll(ND == 3 ? 10 : 5)
    for (int n = 0; n < T; ++n) {
      const int c = lookup<ND>(t, p);
      float m[P];
      load_cell<ND, SMEM>(tab, c, m);
      float q[ND];
      affine<ND>(m, p, q);
      if constexpr (ADAPT) {
        const int ce = lookup<ND>(t, q);
        if (ce != c) {  // Heun step across the facet
          float m0[P], m1[P], v0[ND], v1[ND];
          load_cell<ND, false>(ag, c, m0);
          load_cell<ND, false>(ag, ce, m1);
          affine<ND>(m0, p, v0);
          affine<ND>(m1, q, v1);
#pragma unroll
          for (int k = 0; k < ND; ++k) p[k] = __fmaf_rn(h_half, v0[k] + v1[k], p[k]);
          continue;
        }
      }
#pragma unroll
      for (int k = 0; k < ND; ++k) p[k] = q[k];
    }
    if (st + 1 < nst) src.save_stage(st, slot, p);
    }
    src.finish(slot, i, p);
  }
}

// ---------------------------------------------------------------------------
// Fused adjoint backward.  cpab/core/cpab_ops_2d.cu:432-561 (2D),
// cpab/core/cpab_ops_3d.cu:405-532 (3D), cpab/core/cpab_ops_1d.cu:331-422 (1D).
// ---------------------------------------------------------------------------

// CellT: type of the per-step cell record (uint16_t when nC <= 65535).
// M_SMEM (1D only): moments are summed in a per-block shared-memory table and
// added to global memory once per block.  With a handful of cells the lanes of
// a warp flush into the same few addresses, where L2 would serialize their
// reductions (measured: 1D backward 195 us with L2 reductions, 160 us with the
// shared table); with many cells the shared table's compare-and-swap loops
// cost more, so 2D/3D reduce in L2.
// CL_SMEM: the per-step cell record lives in shared memory, [T][blockDim]
// (a warp's 32 entries of one step are 64 contiguous bytes), instead of in
// each thread's local memory, whose ~200 bytes per thread across ~150k
// resident threads overflow L1 into L2 and DRAM.
// NT: the block size the kernel is launched with (a compile-time constant, so
// that the per-thread slots of the shared-memory record are addressed with
// immediate offsets).  AGG_FINAL: aggregate each point's last moment flush
// over the warp (flush_moments_final).  Measured on one B200 (backward, CUDA
// events): 2D bench workload 370 -> 362 us; the fused transform_data
// backwards got slower (3D 2796 -> 2874 us, where a flush is a small share of
// the much longer steps; dense 2D 1484 -> 1519 us), as did the 3D chain
// (6373 -> 6423 us), so only the 2D transform_grid kernels aggregate.
template <int ND, bool ADAPT, bool A_SMEM, bool M_SMEM, bool CL_SMEM, typename CellT, bool CHAIN,
          int NT, bool AGG_FINAL, class Src>
__device__ __forceinline__ void backward_body(const IntegrateArgs &a, const Src &src) {
  constexpr int P = Dim<ND>::kPpc;
  constexpr int S = kSegSteps;
  extern __shared__ float4 smem4[];
  float *s_tab = reinterpret_cast<float *>(smem4);
  // With A_SMEM the table (a fused chain: every stage's table) comes first.
  float *s_mom = s_tab + (A_SMEM ? (CHAIN ? a.n_stages * a.nC * P : a.nC * P) : 0);
  CellT *s_cl = reinterpret_cast<CellT *>(s_mom + (M_SMEM ? a.nC * P : 0)) + threadIdx.x;
  const int b = blockIdx.y;
  const int nC = a.nC;
  const float *ag = a.As + (int64_t)b * nC * P;
  float *gm = a.moments + (int64_t)b * nC * P;
  if constexpr (A_SMEM) {
    if constexpr (CHAIN) {
      for (int st = 0; st < a.n_stages; ++st)
        stage_table<ND>(s_tab + (size_t)st * nC * P,
                        a.As + ((int64_t)st * a.n_theta + b) * nC * P, nC);
    } else {
      stage_table<ND>(s_tab, ag, nC);
    }
  }
  if constexpr (M_SMEM) {
    for (int i = threadIdx.x; i < nC * P; i += blockDim.x) s_mom[i] = 0.0f;
  }
  if constexpr (A_SMEM || M_SMEM) __syncthreads();
  const float *tab = A_SMEM ? s_tab : ag;  // per stage in fused chains
  auto flush = [&](int c, float (&mo)[P]) {
    if constexpr (M_SMEM) flush_smem<P>(s_mom, c, mo);
    else flush_moments<P>(gm, c, mo);
  };

  const Tess t = a.tess;
  const int T = a.T;
  const float h = 1.0f / (float)T;
  const float h_half = h * 0.5f;
  const float hh = h_half * h;
  const int nfull = T / S;         // full segments of S steps
  const int rem = T - nfull * S;   // steps in the tail segment (0 = none)
  const int64_t nP = src.count();

  for (int64_t slot = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; slot < nP;
       slot += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = src.item(slot);
    float lam[ND];
    // Fused chains walk the stages backwards, lambda flowing from each stage
    // into the one before; a single transformation is one stage.
    const int nst = CHAIN ? a.n_stages : 1;
    for (int st = nst - 1; st >= 0; --st) {
    if constexpr (CHAIN) {
      tab = A_SMEM ? s_tab + (size_t)st * nC * P : a.As + ((int64_t)st * a.n_theta + b) * nC * P;
      gm = a.moments + ((int64_t)st * a.n_theta + b) * nC * P;
    }
    float p[ND];
    src.start_stage(st, slot, i, p);

    // Phase 1: midpoint replay, keeping the start of every segment and (for
    // the plain midpoint rule) every step's cell, so that phase 2 replays a
    // segment without cell lookups.  The record is 2 bytes per step for up to
    // 65535 cells, so a thread's record stays mostly in L1.  Full segments run
    // with compile-time trip counts; only the tail segment (T % S steps) is
    // guarded.
    // 3D: with the cell record in shared memory, the segment checkpoints sit
    // behind it ([seg][k][threads]); otherwise in local memory.
    constexpr bool kCkSmem = ND == 3 && CL_SMEM;
    float ck_local[kCkSmem ? 1 : kMaxSegs][ND];
    float *s_ck = reinterpret_cast<float *>(
                      reinterpret_cast<char *>(s_cl - threadIdx.x) +
                      (((size_t)a.T * NT * sizeof(CellT) + 15) & ~(size_t)15)) +
                  threadIdx.x;
    auto ck = [&](int seg, int k) -> float & {
      if constexpr (kCkSmem) return s_ck[(seg * ND + k) * NT];
      else return ck_local[seg][k];
    };
    CellT cl_local[(ADAPT || CL_SMEM) ? 1 : kMaxSteps];
    auto cl = [&](int step) -> CellT & {
      if constexpr (CL_SMEM) return s_cl[step * NT];
      else return cl_local[step];
    };
    auto phase1 = [&](int seg, auto tail) {
      constexpr bool kTail = decltype(tail)::value;
#pragma unroll
      for (int k = 0; k < ND; ++k) ck(seg, k) = p[k];
#pragma unroll
      for (int s = 0; s < S; ++s) {
        if (kTail && s >= rem) break;
        if constexpr (ADAPT) {
          replay_step<ND, true, A_SMEM>(t, tab, p, h, h_half);
        } else {
          const int c = lookup<ND>(t, p);
          cl(seg * S + s) = (CellT)c;
          float m[P];
          load_cell<ND, A_SMEM>(tab, c, m);
          midpoint_step<ND>(m, p, h, h_half);
        }
      }
    };
    for (int seg = 0; seg < nfull; ++seg) phase1(seg, std::false_type{});
    if (rem) phase1(nfull, std::true_type{});

    // Phase 2: segments last to first; replay into registers, then walk back.
    if (st == nst - 1) src.lambda(slot, i, lam);
    float mo[P];
#pragma unroll
    for (int k = 0; k < P; ++k) mo[k] = 0.0f;
    int prev = -1;
    auto phase2 = [&](int seg, auto tail) {
      constexpr bool kTail = decltype(tail)::value;
      float xs[S][ND];
      int cs[S];
#pragma unroll
      for (int k = 0; k < ND; ++k) p[k] = ck(seg, k);
#pragma unroll
      for (int s = 0; s < S; ++s) {
        if (kTail && s >= rem) break;
#pragma unroll
        for (int k = 0; k < ND; ++k) xs[s][k] = p[k];
        if constexpr (ADAPT) {
          cs[s] = replay_step<ND, true, A_SMEM>(t, tab, p, h, h_half);
        } else {
          cs[s] = (int)cl(seg * S + s);
          // The segment's end point is not needed.
          if (kTail ? s + 1 < rem : s + 1 < S) {
            float m[P];
            load_cell<ND, A_SMEM>(tab, cs[s], m);
            midpoint_step<ND>(m, p, h, h_half);
          }
        }
      }
#pragma unroll
      for (int s = S - 1; s >= 0; --s) {
        if (kTail && s >= rem) continue;
        const int c = cs[s];
        if (c != prev) {
          if (prev >= 0) flush(prev, mo);
          prev = c;
        }
        float m[P];
        load_cell<ND, A_SMEM>(tab, c, m);
        adjoint_step<ND>(m, xs[s], lam, mo, h, h_half, hh);
      }
    };
    if (rem) phase2(nfull, std::true_type{});
    for (int seg = nfull - 1; seg >= 0; --seg) phase2(seg, std::false_type{});
    // The last run ends at the point's initial cell, which the warp's lanes
    // (sorted by initial cell) reach together and usually share.
    if (prev >= 0) {
      if constexpr (M_SMEM) flush_smem<P>(s_mom, prev, mo);
      else if constexpr (AGG_FINAL) flush_moments_final<P>(gm, prev, mo);
      else flush_moments<P>(gm, prev, mo);
    }
    }
    src.grad(slot, i, lam);
  }

  if constexpr (M_SMEM) {
    __syncthreads();
    for (int i = threadIdx.x; i < nC * P; i += blockDim.x) {
      const float v = s_mom[i];
      if (v != 0.0f) atomicAdd(gm + i, v);
    }
  }
}

// ---------------------------------------------------------------------------
// Launch helpers.
// ---------------------------------------------------------------------------

// Resident blocks per SM for (kernel, threads, smem), cached per device.  The
// first query of a kernel on a device also raises its dynamic shared-memory
// limit to the device maximum.
int blocks_per_sm(const void *kernel, int threads, size_t smem) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> cache;
  static std::unordered_map<uint64_t, bool> raised;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t kkey = (reinterpret_cast<uint64_t>(kernel) << 6) ^ (uint64_t)dev;
  const uint64_t key = kkey * 1000003ull ^ (smem << 10) ^ (uint64_t)threads;
  std::lock_guard<std::mutex> lock(mu);
  if (!raised[kkey]) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         device_info().max_smem_optin);
    raised[kkey] = true;
  }
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess ||
      n < 1) {
    cudaGetLastError();
    n = 1;
  }
  cache[key] = n;
  return n;
}

// Blocks along x stride over the points of one transformation (blockIdx.y).
// The grid is 1 to 4 resident waves: about 6 points per thread per wave.
// One wave leaves the whole tail to the slowest blocks; more waves let early
// finishers take new blocks, at the cost of restaging the cell table.
// Measured (B200, backward): 2d bench 394 -> 387 us at 2 waves; 3D 10^3
// 3.15 -> 3.09 ms and dense 2D 1.54 -> 1.45 ms at 4 waves; a block per 512
// points was slower in both.
dim3 wave_grid(const void *kernel, int threads, size_t smem, int64_t nP, int n_theta,
               int n_stages = 1) {
  const int64_t wave = (int64_t)blocks_per_sm(kernel, threads, smem) * device_info().sm_count;
  const int64_t per_thread = nP * n_theta * n_stages / (wave * threads);
  const int64_t cap = wave * std::min<int64_t>(4, std::max<int64_t>(1, per_thread / 6));
  const int64_t need = (nP + threads - 1) / threads;
  int64_t nbx = cap / n_theta;
  if (nbx < 1) nbx = 1;
  if (nbx > need) nbx = need;
  return dim3((unsigned)nbx, (unsigned)n_theta);
}

template <typename K>
cudaError_t launch_wave_args(K kernel, int threads, size_t smem, const IntegrateArgs &a,
                             const MeshArgs &m, cudaStream_t s) {
  const void *kp = reinterpret_cast<const void *>(kernel);
  const dim3 grid = wave_grid(kp, threads, smem, a.nP, a.n_theta);
  kernel<<<grid, threads, smem, s>>>(a, m);
  return cudaGetLastError();
}

template <typename K>
cudaError_t launch_wave(K kernel, int threads, size_t smem, const IntegrateArgs &a,
                        cudaStream_t s) {
  const void *kp = reinterpret_cast<const void *>(kernel);
  const dim3 grid = wave_grid(kp, threads, smem, a.nP, a.n_theta, a.n_stages);
  kernel<<<grid, threads, smem, s>>>(a);
  return cudaGetLastError();
}

// Shared memory of the per-step cell record, plus in 3D the segment
// checkpoints that the backward keeps beside it (3D tables stay in global
// memory, so shared memory has room; in local memory the checkpoints competed
// with the table rows for L1).
template <int ND, typename CellT>
size_t cell_record_bytes(int threads, int T) {
  size_t b = (size_t)threads * T * sizeof(CellT);
  b = (b + 15) & ~(size_t)15;
  if constexpr (ND == 3) b += (size_t)((T + kSegSteps - 1) / kSegSteps) * ND * sizeof(float) * threads;
  return b;
}

}  // namespace

}  // namespace cpab
