// Device building blocks shared by the CPA kernels: tessellation cell lookup,
// per-cell affine steps, cell-table staging and moment flushes.
//
// The cell rules and the step arithmetic are the reference's numerical
// definitions (cpab/core/cpab_ops_{1,2,3}d.cu) restated with the same
// floating-point operation sequence, so that trajectories and cell indices
// agree bit for bit.  Only the way they are evaluated differs: floor() is done
// with one round-down add on the FMA pipe instead of F2I/I2F conversions, and
// cell tables are read from shared memory when they fit.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace cpab {

// Steps between adjoint checkpoints; each segment is replayed into registers
// (its last step is never needed, so shorter segments also replay fewer steps).
constexpr int kSegSteps = 4;
// Largest nstepsolver (reference: CPAB_MAX_STEPS = 100 in cpab_ops_2d.cuh:8).
constexpr int kMaxSteps = 256;
constexpr int kMaxSegs = kMaxSteps / kSegSteps;

// Clamp bound of the 1D/2D lookups: 1 - 1e-7 rounded to float (= 1 - 2^-23).
// cpab/core/cpab_ops_2d.cu:127-129, cpab/core/cpab_ops_1d.cu:92-93.
constexpr float kOneMinusEps = 1.0f - 1e-7f;

template <int ND> struct Dim {
  static constexpr int kPpc = ND * (ND + 1);  // params per cell (= row length of a cell table)
};

// Tessellation geometry passed by value to kernels.
struct Tess {
  int nx, ny, nz;
  float fx, fy, fz;    // (float)n*
};

// floor(v) for 0 <= v < 2^22, as float and int, without conversion units:
// v + 2^23 rounded toward -inf is 2^23 + floor(v) exactly.
__device__ __forceinline__ float floor_nonneg(float v, int &i) {
  const float r = __fadd_rd(v, 8388608.0f);
  i = __float_as_int(r) - 0x4B000000;
  return r - 8388608.0f;
}

// ---------------------------------------------------------------------------
// Cell lookup.  Return the cell (interval / triangle / tetrahedron) index.
// ---------------------------------------------------------------------------

// 1D: interval index; cpab/core/cpab_ops_1d.cu:52-59.
__device__ __forceinline__ int cell_of(const Tess &t, float x) {
  const float xc = fminf(fmaxf(x, 0.0f), kOneMinusEps);
  int i;
  floor_nonneg(xc * t.fx, i);
  return min(i, t.nx - 1);
}

// 2D: four triangles per square numbered bottom(0) right(1) top(2) left(3);
// outside the unit square the triangle facing the nearest boundary part is
// used.  cpab/core/cpab_ops_2d.cu:119-176 (the reference's `a*b - c`
// comparisons are contracted to fma by nvcc; they are written as fmaf here).
// Points strictly inside the square take a short path: there the reference's
// lower clamp is the identity and none of its boundary branches is taken.
// (Out-of-line and given scalars, so that the caller's Tess stays in registers.)
static __device__ __noinline__ int cell_of_2d_outside(int nx, float fnx, float fny, float px,
                                                      float py) {
  const float xc = fminf(fmaxf(px, 0.0f), kOneMinusEps);
  const float yc = fminf(fmaxf(py, 0.0f), kOneMinusEps);
  int ix, iy;
  const float fx0 = floor_nonneg(xc * fnx, ix);
  const float fy0 = floor_nonneg(yc * fny, iy);
  const int base = (ix + iy * nx) << 2;
  if (px <= 0.0f) {
    if (py <= 0.0f && py * fny < px * fnx) return base;
    if (py >= 1.0f && fmaf(py, fny, -fny) > -px * fnx) return base + 2;
    return base + 3;
  }
  if (px >= 1.0f) {
    if (py <= 0.0f && -py * fny > fmaf(px, fnx, -fnx)) return base;
    if (py >= 1.0f && fmaf(py, fny, -fny) > fmaf(px, fnx, -fnx)) return base + 2;
    return base + 1;
  }
  if (py <= 0.0f) return base;
  if (py >= 1.0f) return base + 2;
  // Unreachable for finite inputs (handled by the caller's inside path) but
  // kept for NaN coordinates, which fail every comparison above.
  const float lx = fmaf(xc, fnx, -fx0);
  const float ly = fmaf(yc, fny, -fy0);
  return base + (((lx < ly) * 3) ^ ((1.0f - lx) < ly));
}

__device__ __forceinline__ int cell_of(const Tess &t, float px, float py) {
  if (!(px > 0.0f && px < 1.0f && py > 0.0f && py < 1.0f))
    return cell_of_2d_outside(t.nx, t.fx, t.fy, px, py);
  const float xc = fminf(px, kOneMinusEps);
  const float yc = fminf(py, kOneMinusEps);
  int ix, iy;
  // xc * n < n for every n < 2^24 because xc <= 1 - 2^-23: no upper clamp.
  const float fx0 = floor_nonneg(xc * t.fx, ix);
  const float fy0 = floor_nonneg(yc * t.fy, iy);
  const float lx = fmaf(xc, t.fx, -fx0);
  const float ly = fmaf(yc, t.fy, -fy0);
  const int upper_left = lx < ly;           // above the main diagonal
  const int upper_right = (1.0f - lx) < ly;  // above the anti-diagonal
  return ((ix + iy * t.nx) << 2) + ((upper_left * 3) ^ upper_right);
}

// 3D: five tetrahedra per cube (central one = 0), cube parity flips the
// split; beyond a corner the coordinate with the smallest overshoot is moved
// half a cell inside.  cpab/core/cpab_ops_3d.cu:67-131.
__device__ __forceinline__ int tet_in_cube(int nx, int ny, int nz, float sx, float sy, float sz) {
  int i, j, k;
  float fi = floor_nonneg(sx, i);
  float fj = floor_nonneg(sy, j);
  float fk = floor_nonneg(sz, k);
  // A coordinate exactly on the upper face belongs to the last cube.
  if (i > nx - 1) { i = nx - 1; fi = (float)i; }
  if (j > ny - 1) { j = ny - 1; fj = (float)j; }
  if (k > nz - 1) { k = nz - 1; fk = (float)k; }
  float x = sx - fi;
  float y = sy - fj;
  const float z = sz - fk;
  const int c = 5 * (i + nx * (j + ny * k));
  if ((i ^ j ^ k) & 1) {  // odd cubes: rotate the local frame by 90 degrees
    const float x0 = x;
    x = y;
    y = 1.0f - x0;
  }
  if (-x - y + z >= 0.0f) return c + 1;
  if (x + y + z - 2.0f >= 0.0f) return c + 2;
  if (-x + y - z >= 0.0f) return c + 3;
  if (x - y - z >= 0.0f) return c + 4;
  return c;
}

static __device__ __noinline__ int cell_of_3d_outside(int nx, int ny, int nz, float px, float py,
                                                      float pz) {
  const float fx = (float)nx, fy = (float)ny, fz = (float)nz;
  const float ox = (fabsf(px - 0.5f) - 0.5f) * fx;
  const float oy = (fabsf(py - 0.5f) - 0.5f) * fy;
  const float oz = (fabsf(pz - 0.5f) - 0.5f) * fz;
  if (ox > 0.0f && oy > 0.0f && oz > 0.0f) {
    if (ox <= oy && ox <= oz) {
      px = (px < 0.5f) ? 0.5f / fx : 1.0f - 0.5f / fx;
    } else if (oy <= oz) {
      py = (py < 0.5f) ? 0.5f / fy : 1.0f - 0.5f / fy;
    } else {
      pz = (pz < 0.5f) ? 0.5f / fz : 1.0f - 0.5f / fz;
    }
  }
  return tet_in_cube(nx, ny, nz, fminf(fmaxf(px, 0.0f), 1.0f) * fx,
                     fminf(fmaxf(py, 0.0f), 1.0f) * fy, fminf(fmaxf(pz, 0.0f), 1.0f) * fz);
}

__device__ __forceinline__ int cell_of(const Tess &t, float px, float py, float pz) {
  // Inside the closed unit cube the clamps are identities and the corner rule
  // does not apply.
  if (px >= 0.0f && px <= 1.0f && py >= 0.0f && py <= 1.0f && pz >= 0.0f && pz <= 1.0f)
    return tet_in_cube(t.nx, t.ny, t.nz, px * t.fx, py * t.fy, pz * t.fz);
  return cell_of_3d_outside(t.nx, t.ny, t.nz, px, py, pz);
}

// ---------------------------------------------------------------------------
// Cell tables: kPpc floats per cell, rows packed back to back (the layout of
// the reference's As/Trels).  A 2D row is 24 bytes and loads as three 64-bit
// words; a 3D row is 48 bytes, three 128-bit words.  Packed rows spread
// neighbouring cells over distinct shared-memory banks.
// ---------------------------------------------------------------------------

template <int ND, bool SMEM>
__device__ __forceinline__ void load_cell(const float *__restrict__ tab, int c,
                                          float (&m)[Dim<ND>::kPpc]) {
  if constexpr (ND == 1) {
    const float2 v = SMEM ? reinterpret_cast<const float2 *>(tab)[c]
                          : __ldg(reinterpret_cast<const float2 *>(tab) + c);
    m[0] = v.x; m[1] = v.y;
  } else if constexpr (ND == 2) {
    const float2 *p = reinterpret_cast<const float2 *>(tab) + 3 * c;
    const float2 u = SMEM ? p[0] : __ldg(p), v = SMEM ? p[1] : __ldg(p + 1),
                 w = SMEM ? p[2] : __ldg(p + 2);
    m[0] = u.x; m[1] = u.y; m[2] = v.x; m[3] = v.y; m[4] = w.x; m[5] = w.y;
  } else {
    const float4 *p = reinterpret_cast<const float4 *>(tab) + 3 * c;
    const float4 u = SMEM ? p[0] : __ldg(p);
    const float4 v = SMEM ? p[1] : __ldg(p + 1);
    const float4 w = SMEM ? p[2] : __ldg(p + 2);
    m[0] = u.x; m[1] = u.y; m[2] = u.z; m[3] = u.w;
    m[4] = v.x; m[5] = v.y; m[6] = v.z; m[7] = v.w;
    m[8] = w.x; m[9] = w.y; m[10] = w.z; m[11] = w.w;
  }
}

// Copy n floats (a multiple of 2, 8-byte aligned) from global to shared memory.
__device__ __forceinline__ void stage_table(float *__restrict__ s, const float *__restrict__ g,
                                            int n) {
  const float2 *g2 = reinterpret_cast<const float2 *>(g);
  float2 *s2 = reinterpret_cast<float2 *>(s);
  for (int i = threadIdx.x; i < n / 2; i += blockDim.x) s2[i] = __ldg(g2 + i);
}

// ---------------------------------------------------------------------------
// Affine algebra on [ND] points with a row-major ND x (ND+1) matrix m.
// v = m [p; 1] evaluated as the reference does: nested fmaf from the last
// column inwards.
// ---------------------------------------------------------------------------

template <int ND>
__device__ __forceinline__ void affine(const float (&m)[Dim<ND>::kPpc], const float (&p)[ND],
                                       float (&v)[ND]) {
#pragma unroll
  for (int r = 0; r < ND; ++r) {
    const float *row = m + r * (ND + 1);
    float acc = row[ND];
#pragma unroll
    for (int k = ND - 1; k >= 0; --k) acc = __fmaf_rn(row[k], p[k], acc);
    v[r] = acc;
  }
}

template <int ND>
__device__ __forceinline__ int lookup(const Tess &t, const float (&p)[ND]) {
  if constexpr (ND == 1) return cell_of(t, p[0]);
  else if constexpr (ND == 2) return cell_of(t, p[0], p[1]);
  else return cell_of(t, p[0], p[1], p[2]);
}

// One midpoint (RK2) step inside cell matrix m:
// p <- p + h v(p + h/2 v(p)).  cpab/core/cpab_ops_2d.cu:317-340.
template <int ND>
__device__ __forceinline__ void midpoint_step(const float (&m)[Dim<ND>::kPpc], float (&p)[ND],
                                              float h, float h_half) {
  float v[ND], q[ND], w[ND];
  affine<ND>(m, p, v);
#pragma unroll
  for (int k = 0; k < ND; ++k) q[k] = __fmaf_rn(h_half, v[k], p[k]);
  affine<ND>(m, q, w);
#pragma unroll
  for (int k = 0; k < ND; ++k) p[k] = __fmaf_rn(h, w[k], p[k]);
}

// Replay step of the adjoint: midpoint step in the start cell; when adaptive
// and the step leaves the cell, a Heun step averaging the start and end cell
// velocities replaces it.  Returns the start cell.
// cpab/core/cpab_ops_2d.cu:342-380, cpab/core/cpab_ops_3d.cu:284-329.
template <int ND, bool ADAPT, bool SMEM>
__device__ __forceinline__ int replay_step(const Tess &t, const float *__restrict__ atab,
                                           float (&p)[ND], float h, float h_half) {
  const int c = lookup<ND>(t, p);
  float m[Dim<ND>::kPpc];
  load_cell<ND, SMEM>(atab, c, m);
  if constexpr (!ADAPT) {
    midpoint_step<ND>(m, p, h, h_half);
  } else {
    float q[ND];
#pragma unroll
    for (int k = 0; k < ND; ++k) q[k] = p[k];
    midpoint_step<ND>(m, q, h, h_half);
    const int ce = lookup<ND>(t, q);
    if (ce == c) {
#pragma unroll
      for (int k = 0; k < ND; ++k) p[k] = q[k];
    } else {
      float v0[ND], v1[ND], me[Dim<ND>::kPpc];
      affine<ND>(m, p, v0);
      load_cell<ND, SMEM>(atab, ce, me);
      affine<ND>(me, q, v1);
#pragma unroll
      for (int k = 0; k < ND; ++k) p[k] = __fmaf_rn(h_half, v0[k] + v1[k], p[k]);
    }
  }
  return c;
}

// One reverse step of the adjoint of the midpoint rule in cell matrix m at
// step start p: adds the step's contribution to the cell moments mo and moves
// lam from t_{n+1} to t_n.  cpab/core/cpab_ops_2d.cu:382-430 (2D),
// cpab/core/cpab_ops_3d.cu:331-403 (3D), cpab/core/cpab_ops_1d.cu:301-329 (1D).
template <int ND>
__device__ __forceinline__ void adjoint_step(const float (&m)[Dim<ND>::kPpc], const float (&p)[ND],
                                             float (&lam)[ND], float (&mo)[Dim<ND>::kPpc],
                                             float h, float h_half, float hh) {
  constexpr int C = ND + 1;
  float v[ND], q[ND], at[ND];
  affine<ND>(m, p, v);
#pragma unroll
  for (int k = 0; k < ND; ++k) q[k] = __fmaf_rn(h_half, v[k], p[k]);
  // at = A^T lam (linear part only)
#pragma unroll
  for (int k = 0; k < ND; ++k) {
    float s = m[k] * lam[0];
#pragma unroll
    for (int r = 1; r < ND; ++r) s = s + m[r * C + k] * lam[r];
    at[k] = s;
  }
  float wq[ND], wp[ND];
#pragma unroll
  for (int r = 0; r < ND; ++r) { wq[r] = h * lam[r]; wp[r] = hh * at[r]; }
#pragma unroll
  for (int r = 0; r < ND; ++r) {
#pragma unroll
    for (int k = 0; k < ND; ++k) mo[r * C + k] += wq[r] * q[k];
    mo[r * C + ND] += wq[r];
  }
#pragma unroll
  for (int r = 0; r < ND; ++r) {
#pragma unroll
    for (int k = 0; k < ND; ++k) mo[r * C + k] += wp[r] * p[k];
    mo[r * C + ND] += wp[r];
  }
  float lm[ND];
#pragma unroll
  for (int k = 0; k < ND; ++k) lm[k] = lam[k] + h_half * at[k];
#pragma unroll
  for (int k = 0; k < ND; ++k) {
    float s = m[k] * lm[0];
#pragma unroll
    for (int r = 1; r < ND; ++r) s = s + m[r * C + k] * lm[r];
    lam[k] += h * s;
  }
}

// Flush one cell's partial moments into a shared-memory table.
template <int P>
__device__ __forceinline__ void flush_smem(float *__restrict__ s_mom, int c, float (&mo)[P]) {
  float *dst = s_mom + c * P;
#pragma unroll
  for (int k = 0; k < P; ++k) {
    atomicAdd(dst + k, mo[k]);
    mo[k] = 0.0f;
  }
}

// Flush one cell's partial moments straight to global memory.  Lanes of the
// warp that flush the same cell are summed first, so each cell costs one
// atomic per moment per warp.
template <int P>
__device__ __forceinline__ void flush_global(float *__restrict__ g_mom, int c, float (&mo)[P]) {
  const unsigned active = __activemask();
  const unsigned same = __match_any_sync(active, c);
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(same) - 1;
  if (same != (1u << lane)) {
    // Sum the group's values into the leader, one peer at a time.
    unsigned rest = same & ~(1u << leader);
    float acc[P];
#pragma unroll
    for (int k = 0; k < P; ++k) acc[k] = mo[k];
    while (rest) {
      const int src = __ffs(rest) - 1;
      rest &= rest - 1;
#pragma unroll
      for (int k = 0; k < P; ++k) {
        const float v = __shfl_sync(same, mo[k], src);
        acc[k] += v;
      }
    }
    if (lane == leader) {
      float *dst = g_mom + (int64_t)c * P;
#pragma unroll
      for (int k = 0; k < P; ++k) atomicAdd(dst + k, acc[k]);
    }
  } else {
    float *dst = g_mom + (int64_t)c * P;
#pragma unroll
    for (int k = 0; k < P; ++k) atomicAdd(dst + k, mo[k]);
  }
#pragma unroll
  for (int k = 0; k < P; ++k) mo[k] = 0.0f;
}

}  // namespace cpab
