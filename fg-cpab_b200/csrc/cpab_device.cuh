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
  // Cell-index offsets that undo the 0x4B000000 bias of floor results read
  // from float bit patterns (floor_nonneg): 2D -4 * 0x4B000000 * (1 + nx),
  // 3D -5 * 0x4B000000 * (1 + nx + nx * ny), both modulo 2^32.
  unsigned c2, c3;
};

// Tessellation geometry of an ndim tessellation with nc[k] cells per axis.
inline Tess make_tess(int ndim, const int *nc) {
  Tess t;
  t.nx = nc[0];
  t.ny = ndim > 1 ? nc[1] : 1;
  t.nz = ndim > 2 ? nc[2] : 1;
  t.fx = (float)t.nx;
  t.fy = (float)t.ny;
  t.fz = (float)t.nz;
  const unsigned k = 0x4B000000u, nx = (unsigned)t.nx, ny = (unsigned)t.ny;
  t.c2 = 0u - 4u * k * (1u + nx);
  t.c3 = 0u - 5u * k * (1u + nx + nx * ny);
  return t;
}

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
  // Inside the square: points within 1e-7 of the upper faces (the caller's
  // short path excludes them) and NaN coordinates, which fail every
  // comparison above.
  const float lx = fmaf(xc, fnx, -fx0);
  const float ly = fmaf(yc, fny, -fy0);
  return base + (((lx < ly) * 3) ^ ((1.0f - lx) < ly));
}

__device__ __forceinline__ int cell_of(const Tess &t, float px, float py) {
  // Inside (0, 1 - 1e-7) the reference's clamp is the identity; the few
  // points in [1 - 1e-7, 1) take the general path, which clamps them.
  if (!(px > 0.0f && px < kOneMinusEps && py > 0.0f && py < kOneMinusEps))
    return cell_of_2d_outside(t.nx, t.fx, t.fy, px, py);
  // px * n < n for every n < 2^24 because px < 1 - 2^-23: no upper clamp.
  // floor_nonneg on both coordinates at once (paired fp32 instructions):
  // r = 2^23 + floor(p * n), -floor = 2^23 - r (exact), l = fma(p, n, -floor).
  const float2 p = make_float2(px, py), n = make_float2(t.fx, t.fy);
  const float2 k23 = make_float2(8388608.0f, 8388608.0f);
  const float2 r = __fadd2_rd(__fmul2_rn(p, n), k23);
  const float2 l = __ffma2_rn(p, n, __ffma2_rn(r, make_float2(-1.0f, -1.0f), k23));
  // r's bit patterns are 0x4B000000 + floor; t.c2 folds the bias out of the index
  const int upper_left = l.x < l.y;            // above the main diagonal
  const int upper_right = (1.0f - l.x) < l.y;  // above the anti-diagonal
  const unsigned sq = __float_as_uint(r.x) + __float_as_uint(r.y) * (unsigned)t.nx;
  return (int)((sq << 2) + t.c2) + ((upper_left * 3) ^ upper_right);
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
  // In [+0, 1) the reference's clamps are identities, the corner rule does not
  // apply, and p * n rounds below n, so floor(p * n) <= n - 1 needs no clamp;
  // everything else (including coordinates exactly 1, and -0, which the
  // general path places identically) takes the general path.  As unsigned
  // integers, the bit patterns of exactly the floats in [+0, 1) lie below
  // that of 1.0f (negatives and NaN have larger patterns).
  const unsigned hi = max(max(__float_as_uint(px), __float_as_uint(py)), __float_as_uint(pz));
  if (hi < 0x3F800000u) {
    // floor_nonneg of x and y together (paired instructions, same roundings):
    // r = 2^23 + floor(s), floor = r - 2^23, and s - floor is exact.
    const float2 sxy = __fmul2_rn(make_float2(px, py), make_float2(t.fx, t.fy));
    const float2 r = __fadd2_rd(sxy, make_float2(8388608.0f, 8388608.0f));
    const float2 fxy = __fadd2_rn(r, make_float2(-8388608.0f, -8388608.0f));
    const float2 lxy = __ffma2_rn(fxy, make_float2(-1.0f, -1.0f), sxy);
    const float sz = pz * t.fz;
    const float rz = __fadd_rd(sz, 8388608.0f);
    const float z = sz - (rz - 8388608.0f);
    // The bit patterns of r are 0x4B000000 + floor: the cube index comes from
    // them directly (t.c3 folds the offsets), and so does its parity
    // (0x4B000000 is even).
    // (Unsigned: the intermediate products wrap modulo 2^32, the sum does not.)
    const unsigned bx = __float_as_uint(r.x), by = __float_as_uint(r.y), bz = __float_as_uint(rz);
    const int c = (int)(5u * (bx + (unsigned)t.nx * (by + (unsigned)t.ny * bz)) + t.c3);
    float x = lxy.x, y = lxy.y;
    if ((bx ^ by ^ bz) & 1) {  // odd cubes: rotate the local frame by 90 degrees
      const float x0 = x;
      x = y;
      y = 1.0f - x0;
    }
    // The reference's four plane sums, from shared partial sums with the same
    // roundings: -x - y = -(x + y) and x - y = -(-x + y) exactly, so
    // x - y - z >= 0  <=>  (-x + y) + z <= 0.
    const float a = x + y, b = -x + y;
    int tet = (b + z <= 0.0f) ? 4 : 0;
    tet = (b - z >= 0.0f) ? 3 : tet;
    tet = ((a + z) - 2.0f >= 0.0f) ? 2 : tet;
    tet = (-a + z >= 0.0f) ? 1 : tet;
    return c + tet;
  }
  return cell_of_3d_outside(t.nx, t.ny, t.nz, px, py, pz);
}

// ---------------------------------------------------------------------------
// Cell tables: kPpc floats per cell, rows packed back to back.  In global
// memory this is the reference's As/Trels layout (row-major ND x (ND+1)).  A
// 2D table staged in shared memory is stored by column pairs instead --
// (m00, m10), (m01, m11), (m02, m12) -- so that both rows of a step are
// evaluated with paired fp32 instructions; it is still 24 bytes a cell, three
// 64-bit words.  A 3D row is 48 bytes, three 128-bit words, in the reference
// layout everywhere (3D tables rarely fit shared memory, and the 3D adjoint
// pairs neighbours within a row).  Packed rows spread neighbouring cells over
// distinct shared-memory banks.
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
    if constexpr (SMEM) {  // column pairs
      const float2 c0 = p[0], c1 = p[1], c2 = p[2];
      m[0] = c0.x; m[1] = c1.x; m[2] = c2.x; m[3] = c0.y; m[4] = c1.y; m[5] = c2.y;
    } else {
      const float2 u = __ldg(p), v = __ldg(p + 1), w = __ldg(p + 2);
      m[0] = u.x; m[1] = u.y; m[2] = v.x; m[3] = v.y; m[4] = w.x; m[5] = w.y;
    }
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

// Stage the nC-cell table g (global, reference layout, 8-byte aligned) into
// shared memory s; 2D tables are transposed into column pairs on the way.
template <int ND>
__device__ __forceinline__ void stage_table(float *__restrict__ s, const float *__restrict__ g,
                                            int nC) {
  const float2 *g2 = reinterpret_cast<const float2 *>(g);
  float2 *s2 = reinterpret_cast<float2 *>(s);
  if constexpr (ND == 2) {
    for (int c = threadIdx.x; c < nC; c += blockDim.x) {
      const float2 u = __ldg(g2 + 3 * c), v = __ldg(g2 + 3 * c + 1), w = __ldg(g2 + 3 * c + 2);
      s2[3 * c] = make_float2(u.x, v.y);
      s2[3 * c + 1] = make_float2(u.y, w.x);
      s2[3 * c + 2] = make_float2(v.x, w.y);
    }
  } else {
    const int n = nC * Dim<ND>::kPpc / 2;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s2[i] = __ldg(g2 + i);
  }
}

// ---------------------------------------------------------------------------
// Affine algebra on [ND] points with a row-major ND x (ND+1) matrix m.
// v = m [p; 1] evaluated as the reference does: nested fmaf from the last
// column inwards.
// ---------------------------------------------------------------------------

// Two fp32 lanes x, y -> one float2 (and back): the paired instructions of
// sm_100 (FFMA2/FMUL2/FADD2) round every component exactly as their scalar
// counterparts, so the 2D steps below are bit-identical to the scalar
// sequence while issuing half as many floating-point instructions.
__device__ __forceinline__ float2 bc(float x) { return make_float2(x, x); }

template <int ND>
__device__ __forceinline__ void affine(const float (&m)[Dim<ND>::kPpc], const float (&p)[ND],
                                       float (&v)[ND]) {
  if constexpr (ND == 2) {
    const float2 c0 = make_float2(m[0], m[3]), c1 = make_float2(m[1], m[4]),
                 c2 = make_float2(m[2], m[5]);
    const float2 r = __ffma2_rn(c0, bc(p[0]), __ffma2_rn(c1, bc(p[1]), c2));
    v[0] = r.x;
    v[1] = r.y;
  } else {
#pragma unroll
    for (int r = 0; r < ND; ++r) {
      const float *row = m + r * (ND + 1);
      float acc = row[ND];
#pragma unroll
      for (int k = ND - 1; k >= 0; --k) acc = __fmaf_rn(row[k], p[k], acc);
      v[r] = acc;
    }
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
  if constexpr (ND == 2) {
    const float2 c0 = make_float2(m[0], m[3]), c1 = make_float2(m[1], m[4]),
                 c2 = make_float2(m[2], m[5]);
    const float2 x = make_float2(p[0], p[1]);
    const float2 v = __ffma2_rn(c0, bc(x.x), __ffma2_rn(c1, bc(x.y), c2));
    const float2 q = __ffma2_rn(bc(h_half), v, x);
    const float2 w = __ffma2_rn(c0, bc(q.x), __ffma2_rn(c1, bc(q.y), c2));
    const float2 y = __ffma2_rn(bc(h), w, x);
    p[0] = y.x;
    p[1] = y.y;
    return;
  } else if constexpr (ND == 3) {
    float v[3], q[3], w[3];
    affine<3>(m, p, v);
    const float2 x = make_float2(p[0], p[1]);
    const float2 q01 = __ffma2_rn(bc(h_half), make_float2(v[0], v[1]), x);
    q[0] = q01.x; q[1] = q01.y; q[2] = __fmaf_rn(h_half, v[2], p[2]);
    affine<3>(m, q, w);
    const float2 y = __ffma2_rn(bc(h), make_float2(w[0], w[1]), x);
    p[0] = y.x; p[1] = y.y; p[2] = __fmaf_rn(h, w[2], p[2]);
    return;
  }
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
  if constexpr (ND == 2) {
    // Moment pairs run over the two rows: (mo[k], mo[C + k]).
    const float2 c0 = make_float2(m[0], m[3]), c1 = make_float2(m[1], m[4]),
                 c2 = make_float2(m[2], m[5]);
    const float2 x = make_float2(p[0], p[1]), l = make_float2(lam[0], lam[1]);
    const float2 v = __ffma2_rn(c0, bc(x.x), __ffma2_rn(c1, bc(x.y), c2));
    const float2 q = __ffma2_rn(bc(h_half), v, x);
    // at = A^T lam (linear part): at_k = m[C+k] lam1 + m[k] lam0.
    const float2 at = make_float2(__fmaf_rn(m[3], l.y, __fmul_rn(m[0], l.x)),
                                  __fmaf_rn(m[4], l.y, __fmul_rn(m[1], l.x)));
    const float2 wq = __fmul2_rn(bc(h), l), wp = __fmul2_rn(bc(hh), at);
    float2 m0 = make_float2(mo[0], mo[C]), m1 = make_float2(mo[1], mo[C + 1]),
           m2 = make_float2(mo[2], mo[C + 2]);
    m0 = __ffma2_rn(wq, bc(q.x), m0);
    m1 = __ffma2_rn(wq, bc(q.y), m1);
    m2 = __fadd2_rn(m2, wq);
    m0 = __ffma2_rn(wp, bc(x.x), m0);
    m1 = __ffma2_rn(wp, bc(x.y), m1);
    m2 = __fadd2_rn(m2, wp);
    mo[0] = m0.x; mo[1] = m1.x; mo[2] = m2.x;
    mo[C] = m0.y; mo[C + 1] = m1.y; mo[C + 2] = m2.y;
    const float2 lm = __ffma2_rn(bc(h_half), at, l);
    const float2 sv = make_float2(__fmaf_rn(m[3], lm.y, __fmul_rn(m[0], lm.x)),
                                  __fmaf_rn(m[4], lm.y, __fmul_rn(m[1], lm.x)));
    const float2 ln = __ffma2_rn(bc(h), sv, l);
    lam[0] = ln.x;
    lam[1] = ln.y;
    return;
  } else if constexpr (ND == 3) {
    // Row layout: the A^T products pair entries k = 0, 1 of each row, the
    // moment updates pair (mo[r][0], mo[r][1]) and (mo[r][2], mo[r][3]); the
    // constant column's update mo += w is written fma(w, 1, mo), which rounds
    // identically.
    float v[3];
    affine<3>(m, p, v);
    const float2 p01 = make_float2(p[0], p[1]), l01 = make_float2(lam[0], lam[1]);
    const float2 q01 = __ffma2_rn(bc(h_half), make_float2(v[0], v[1]), p01);
    const float q2 = __fmaf_rn(h_half, v[2], p[2]);
    const float2 r0 = make_float2(m[0], m[1]), r1 = make_float2(m[C], m[C + 1]),
                 r2 = make_float2(m[2 * C], m[2 * C + 1]);
    const float2 at01 = __ffma2_rn(r2, bc(lam[2]), __ffma2_rn(r1, bc(lam[1]), __fmul2_rn(r0, bc(lam[0]))));
    const float at2 = __fmaf_rn(m[2 * C + 2], lam[2], __fmaf_rn(m[C + 2], lam[1], __fmul_rn(m[2], lam[0])));
    const float2 wq01 = __fmul2_rn(bc(h), l01), wp01 = __fmul2_rn(bc(hh), at01);
    const float wq[3] = {wq01.x, wq01.y, __fmul_rn(h, lam[2])};
    const float wp[3] = {wp01.x, wp01.y, __fmul_rn(hh, at2)};
    const float2 q2one = make_float2(q2, 1.0f), p2one = make_float2(p[2], 1.0f);
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      float2 a = make_float2(mo[r * C], mo[r * C + 1]), b = make_float2(mo[r * C + 2], mo[r * C + 3]);
      a = __ffma2_rn(bc(wq[r]), q01, a);
      b = __ffma2_rn(bc(wq[r]), q2one, b);
      a = __ffma2_rn(bc(wp[r]), p01, a);
      b = __ffma2_rn(bc(wp[r]), p2one, b);
      mo[r * C] = a.x; mo[r * C + 1] = a.y; mo[r * C + 2] = b.x; mo[r * C + 3] = b.y;
    }
    const float2 lm01 = __ffma2_rn(bc(h_half), at01, l01);
    const float lm2 = __fmaf_rn(h_half, at2, lam[2]);
    const float2 s01 = __ffma2_rn(r2, bc(lm2), __ffma2_rn(r1, bc(lm01.y), __fmul2_rn(r0, bc(lm01.x))));
    const float s2 = __fmaf_rn(m[2 * C + 2], lm2, __fmaf_rn(m[C + 2], lm01.y, __fmul_rn(m[2], lm01.x)));
    const float2 ln = __ffma2_rn(bc(h), s01, l01);
    lam[2] = __fmaf_rn(h, s2, lam[2]);
    lam[0] = ln.x;
    lam[1] = ln.y;
    return;
  }
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

// Flush one cell's partial moments into a shared-memory table (fp32 atomics on
// shared memory: a compare-and-swap loop each).
template <int P>
__device__ __forceinline__ void flush_smem(float *__restrict__ s_mom, int c, float (&mo)[P]) {
  float *dst = s_mom + c * P;
#pragma unroll
  for (int k = 0; k < P; ++k) {
    atomicAdd(dst + k, mo[k]);
    mo[k] = 0.0f;
  }
}

// Moment flush scheme, fixed at compile time (-DCPAB_MOMENT_FLUSH=n):
//   0  every flushing lane adds its run straight into the global table with
//      vector reductions (red.global.add.v4/v2.f32, resolved in L2; fire and
//      forget): P/4 or P/2 instructions per flush;
//   1  warp-aggregated: the flushing lanes are grouped by cell
//      (__match_any_sync); a group that occupies a contiguous run of lanes is
//      summed into its first lane by a segmented shuffle reduction (log2 of
//      the longest run levels), which alone issues the reductions; lanes of
//      scattered groups reduce on their own;
//   2  warp-aggregated as the reference does it (cpab/core/cpab_ops_2d.cu:6-59):
//      the lowest lane of each cell group gathers the others' moments one lane
//      at a time by shuffles, then issues the reductions.
// 0 is the default: aggregation trades a few L2 reductions for tens of
// shuffle instructions per flush in a kernel bound by instruction issue.
#ifndef CPAB_MOMENT_FLUSH
#define CPAB_MOMENT_FLUSH 0
#endif

// Add one cell's moments v into the global table row c (vector reductions).
// g_mom must be 16-byte aligned when P % 4 == 0 (3D rows of 12 floats), else
// 8-byte aligned.
template <int P>
__device__ __forceinline__ void red_row(float *__restrict__ g_mom, int c, const float (&v)[P]) {
  if constexpr (P % 4 == 0) {
    float4 *dst = reinterpret_cast<float4 *>(g_mom + (int64_t)c * P);
#pragma unroll
    for (int k = 0; k < P / 4; ++k)
      atomicAdd(dst + k, make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]));
  } else {
    float2 *dst = reinterpret_cast<float2 *>(g_mom + (int64_t)c * P);
#pragma unroll
    for (int k = 0; k < P / 2; ++k) atomicAdd(dst + k, make_float2(v[2 * k], v[2 * k + 1]));
  }
}

// Warp-aggregated red_row over the active lanes: lanes adding to the same cell
// (__match_any_sync) that occupy a contiguous run of lanes are summed into the
// run's first lane by a segmented shuffle reduction (log2 of the longest run
// levels), which alone issues the reductions; lanes of scattered groups add
// their own rows.  The summation order of a cell's contributions changes, not
// the set.
template <int P>
__device__ __forceinline__ void red_row_warp(float *__restrict__ g_mom, int c,
                                             const float (&mo)[P]) {
  const unsigned act = __activemask();
  const unsigned grp = __match_any_sync(act, c);
  const int lane = threadIdx.x & 31;
  const int lo = __ffs(grp) - 1, hi = 31 - __clz(grp);
  // the group is the lanes lo..hi exactly (2u << 31 wraps to 0: all 32 lanes)
  const bool run = (grp >> lo) == (2u << (hi - lo)) - 1u;
  const int len = run ? hi - lo + 1 : 1;
  const int longest = __reduce_max_sync(act, len);
  if (longest == 1) {
    red_row<P>(g_mom, c, mo);
    return;
  }
  // Segmented suffix sums: after the level of offset `off`, lane i holds the
  // sum over lanes i..min(i + 2 off - 1, hi) of its run.  Source lanes past
  // the run's end (possibly inactive) are read but not used.
  float v[P];
#pragma unroll
  for (int k = 0; k < P; ++k) v[k] = mo[k];
  for (int off = 1; off < longest; off <<= 1) {
    const bool take = run && lane + off <= hi;
#pragma unroll
    for (int k = 0; k < P; ++k) {
      const float o = __shfl_down_sync(act, v[k], off);
      if (take) v[k] += o;
    }
  }
  if (!run) red_row<P>(g_mom, c, mo);
  else if (lane == lo) red_row<P>(g_mom, c, v);
}

// Flush one cell's partial moments mo into the global moment table and clear
// them.  A shared-memory table would cost more than any scheme below: fp32
// atomics on shared memory are compare-and-swap loops, and the lanes of a warp
// (processing points sorted by cell) usually hit the same cell, so those loops
// retry once per lane.  Called by the lanes whose cell changed (a divergent
// branch): the warp-aggregated schemes group whichever lanes are active.
template <int P>
__device__ __forceinline__ void flush_moments(float *__restrict__ g_mom, int c, float (&mo)[P]) {
#if CPAB_MOMENT_FLUSH == 0
  red_row<P>(g_mom, c, mo);
#elif CPAB_MOMENT_FLUSH == 1
  red_row_warp<P>(g_mom, c, mo);
#else
  const unsigned act = __activemask();
  const unsigned grp = __match_any_sync(act, c);
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(grp) - 1;
  if (grp == (1u << lane)) {
    red_row<P>(g_mom, c, mo);
  } else {
    float s[P];
#pragma unroll
    for (int k = 0; k < P; ++k) s[k] = 0.0f;
    for (unsigned peers = grp; peers != 0u; peers &= peers - 1u) {
      const int src = __ffs(peers) - 1;
#pragma unroll
      for (int k = 0; k < P; ++k) {
        const float o = __shfl_sync(grp, mo[k], src);
        if (lane == leader) s[k] += o;
      }
    }
    if (lane == leader) red_row<P>(g_mom, c, s);
  }
#endif
#pragma unroll
  for (int k = 0; k < P; ++k) mo[k] = 0.0f;
}

// The last flush of a point's moments, at its initial cell.  The lanes of a
// warp arrive together (converged, after the same number of steps) and, with
// the points sorted by initial cell, mostly share that cell: their reductions
// would all hit one address and serialize in L2, so they are aggregated over
// the warp first.  Mid-trajectory flushes are rare (about one lane in a
// hundred per step), divergent and spread over cells, so they stay per lane.
// CPAB_FINAL_FLUSH_WARP=0 turns the aggregation off (for measurements).
#ifndef CPAB_FINAL_FLUSH_WARP
#define CPAB_FINAL_FLUSH_WARP 1
#endif
template <int P>
__device__ __forceinline__ void flush_moments_final(float *__restrict__ g_mom, int c,
                                                    float (&mo)[P]) {
#if CPAB_FINAL_FLUSH_WARP && CPAB_MOMENT_FLUSH == 0
  red_row_warp<P>(g_mom, c, mo);
#pragma unroll
  for (int k = 0; k < P; ++k) mo[k] = 0.0f;
#else
  flush_moments<P>(g_mom, c, mo);
#endif
}

}  // namespace cpab
