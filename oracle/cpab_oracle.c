/*
 * cpab_oracle.c -- CPU restatement of the FG-CPAB reference kernels.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle and the timed CPU
 * baseline; the product (fg-cpab_b200/) never links or calls it.
 *
 * It restates, operation for operation, the per-point arithmetic of the
 * reference CUDA kernels in plain C (OpenMP over points):
 *   cell lookup        cpab/core/cpab_ops_1d.cu:90-97, cpab_ops_2d.cu:119-176,
 *                      cpab_ops_3d.cu:67-131
 *   1D closed form     cpab/core/cpab_ops_1d.cu:103-243
 *   2D/3D forward      cpab/core/cpab_ops_2d.cu:212-278, cpab_ops_3d.cu:169-241
 *   adjoint backward   cpab/core/cpab_ops_1d.cu:249-422, cpab_ops_2d.cu:317-561,
 *                      cpab_ops_3d.cu:247-532
 *   expm               cpab/core/cpab_ops_1d.cu:442-467, cpab_ops_2d.cu:585-701,
 *                      cpab_ops_3d.cu:538-674
 * __fmaf_rn maps to fmaf (compiled with -mfma -ffp-contract=off, so fmaf is
 * one fused instruction and nothing else is contracted), __float2int_rd to
 * floorf.  The adjoint stores the whole midpoint trajectory instead of
 * checkpoints; the reference's segment recompute repeats identical
 * operations, so the values are the same.  Moments are summed per thread and
 * then reduced in thread order (the reference sums with unordered atomics).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_MAX_STEPS 4096

typedef struct {
  int nx, ny, nz;
} tess_t;

static const float kOneMinusEps = 1.0f - 1e-7f;

/* ---------------------------------------------------------------- lookup */

static int cell1(float px, tess_t t) {
  float xc = fminf(fmaxf(px, 0.0f), kOneMinusEps);
  int c = (int)floorf(xc * (float)t.nx);
  return c < t.nx - 1 ? c : t.nx - 1;
}

static int cell2(float px, float py, tess_t t) {
  const float fx = (float)t.nx, fy = (float)t.ny;
  float xc = fminf(fmaxf(px, 0.0f), kOneMinusEps);
  float yc = fminf(fmaxf(py, 0.0f), kOneMinusEps);
  int cx = (int)floorf(xc * fx);
  int cy = (int)floorf(yc * fy);
  if (cx > t.nx - 1) cx = t.nx - 1;
  if (cy > t.ny - 1) cy = t.ny - 1;
  float lx = fmaf(xc, fx, -(float)cx);
  float ly = fmaf(yc, fy, -(float)cy);
  int base = (cx + cy * t.nx) * 4;
  if (px <= 0.0f) {
    if (py <= 0.0f && py * fy < px * fx) return base;
    if (py >= 1.0f && fmaf(py, fy, -fy) > -px * fx) return base + 2;
    return base + 3;
  }
  if (px >= 1.0f) {
    if (py <= 0.0f && -py * fy > fmaf(px, fx, -fx)) return base;
    if (py >= 1.0f && fmaf(py, fy, -fy) > fmaf(px, fx, -fx)) return base + 2;
    return base + 1;
  }
  if (py <= 0.0f) return base;
  if (py >= 1.0f) return base + 2;
  {
    int above_diag = lx < ly;
    int above_anti = (1.0f - lx) < ly;
    if (!above_diag) return base + (above_anti ? 1 : 0);
    return base + (above_anti ? 2 : 3);
  }
}

static int cell3(float px, float py, float pz, tess_t t) {
  const float fx = (float)t.nx, fy = (float)t.ny, fz = (float)t.nz;
  float ox = (fabsf(px - 0.5f) - 0.5f) * fx;
  float oy = (fabsf(py - 0.5f) - 0.5f) * fy;
  float oz = (fabsf(pz - 0.5f) - 0.5f) * fz;
  if (ox > 0.0f && oy > 0.0f && oz > 0.0f) {
    if (ox <= oy && ox <= oz)
      px = (px < 0.5f) ? 0.5f / fx : 1.0f - 0.5f / fx;
    else if (oy <= oz)
      py = (py < 0.5f) ? 0.5f / fy : 1.0f - 0.5f / fy;
    else
      pz = (pz < 0.5f) ? 0.5f / fz : 1.0f - 0.5f / fz;
  }
  float sx = fminf(fmaxf(px, 0.0f), 1.0f) * fx;
  float sy = fminf(fmaxf(py, 0.0f), 1.0f) * fy;
  float sz = fminf(fmaxf(pz, 0.0f), 1.0f) * fz;
  int i = (int)floorf(sx), j = (int)floorf(sy), k = (int)floorf(sz);
  if (i > t.nx - 1) i = t.nx - 1;
  if (j > t.ny - 1) j = t.ny - 1;
  if (k > t.nz - 1) k = t.nz - 1;
  float x = sx - (float)i, y = sy - (float)j, z = sz - (float)k;
  int c = 5 * (i + j * t.nx + k * t.nx * t.ny);
  if ((i ^ j ^ k) & 1) {
    float tmp = x;
    x = y;
    y = 1.0f - tmp;
  }
  if (-x - y + z >= 0.0f) return c + 1;
  if (x + y + z - 2.0f >= 0.0f) return c + 2;
  if (-x + y - z >= 0.0f) return c + 3;
  if (x - y - z >= 0.0f) return c + 4;
  return c;
}

static int cell_nd(int nd, const float *p, tess_t t) {
  if (nd == 1) return cell1(p[0], t);
  if (nd == 2) return cell2(p[0], p[1], t);
  return cell3(p[0], p[1], p[2], t);
}

/* v = m [p; 1] with nested fmaf from the last column. */
static void affine(int nd, const float *m, const float *p, float *v) {
  for (int r = 0; r < nd; ++r) {
    const float *row = m + r * (nd + 1);
    float acc = row[nd];
    for (int k = nd - 1; k >= 0; --k) acc = fmaf(row[k], p[k], acc);
    v[r] = acc;
  }
}

static tess_t make_tess(int nd, const int32_t *nc) {
  tess_t t;
  t.nx = nc[0];
  t.ny = nd > 1 ? nc[1] : 1;
  t.nz = nd > 2 ? nc[2] : 1;
  return t;
}

static int64_t n_cells(int nd, tess_t t) {
  int64_t n = (int64_t)t.nx * t.ny * t.nz;
  return nd == 1 ? n : (nd == 2 ? 4 * n : 5 * n);
}

void oracle_cells(int nd, const int32_t *nc, const float *pts, int64_t n, int32_t *cells) {
  tess_t t = make_tess(nd, nc);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    float p[3];
    for (int k = 0; k < nd; ++k) p[k] = pts[k * n + i];
    cells[i] = cell_nd(nd, p, t);
  }
}

/* ------------------------------------------------------------------ expm */
/* Sums of products are evaluated left to right, the first two products fused
 * as fmaf(a, b, c*d) and every further product fused onto the running sum:
 * the rounding of the reference's compiled expm kernels (verified bit for bit
 * against Trels they produced on a B200, tests/golden/kernel_golden.npz). */

static float dot2(float a, float b, float c, float d) { return fmaf(a, b, c * d); }
static float dot3(float a, float b, float c, float d, float e, float f) {
  return fmaf(e, f, fmaf(a, b, c * d));
}
static float diff2(float a, float b, float c, float d) { return fmaf(a, b, -(c * d)); }
static float pdiag(float h, float m, float s, float q) { return fmaf(s, q, fmaf(h, m, 1.0f)); }
static float poff(float h, float m, float s, float q) { return fmaf(h, m, s * q); }

static void expm1d(const float *A, float dT, float *out) {
  float m00 = dT * A[0], m01 = dT * A[1];
  float rel;
  if (fabsf(m00) > 1e-6f) {
    rel = expm1f(m00) / m00;
  } else {
    float q = m00 * m00;
    rel = fmaf((1.0f / 24.0f) * q, m00, fmaf(1.0f / 6.0f, q, fmaf(0.5f, m00, 1.0f)));
  }
  out[0] = expf(m00);
  out[1] = m01 * rel;
}

static int n_squarings(float norm) { return norm > 0.5f ? (int)ceilf(log2f(norm * 2.0f)) : 0; }

static void expm2d(const float *A, float dT, float *out) {
  float a[6];
  for (int k = 0; k < 6; ++k) a[k] = dT * A[k];
  float sq = dot2(a[0], a[0], a[1], a[1]);
  for (int k = 2; k < 6; ++k) sq = fmaf(a[k], a[k], sq);
  int ns = n_squarings(sqrtf(sq));
  float sc = 1.0f;
  for (int i = 0; i < ns; ++i) sc *= 0.5f;
  float m00 = a[0] * sc, m01 = a[1] * sc, m02 = a[2] * sc;
  float m10 = a[3] * sc, m11 = a[4] * sc, m12 = a[5] * sc;
  float q00 = dot2(m00, m00, m01, m10), q01 = dot2(m00, m01, m01, m11), q02 = dot2(m00, m02, m01, m12);
  float q10 = dot2(m10, m00, m11, m10), q11 = dot2(m10, m01, m11, m11), q12 = dot2(m10, m02, m11, m12);
  const float t = 1.0f / 12.0f;
  float P00 = pdiag(0.5f, m00, t, q00), P01 = poff(0.5f, m01, t, q01), P02 = poff(0.5f, m02, t, q02);
  float P10 = poff(0.5f, m10, t, q10), P11 = pdiag(0.5f, m11, t, q11), P12 = poff(0.5f, m12, t, q12);
  float Q00 = pdiag(-0.5f, m00, t, q00), Q01 = poff(-0.5f, m01, t, q01), Q02 = poff(-0.5f, m02, t, q02);
  float Q10 = poff(-0.5f, m10, t, q10), Q11 = pdiag(-0.5f, m11, t, q11), Q12 = poff(-0.5f, m12, t, q12);
  float inv = 1.0f / diff2(Q00, Q11, Q01, Q10);
  float i00 = Q11 * inv, i01 = -Q01 * inv, i10 = -Q10 * inv, i11 = Q00 * inv;
  float i02 = -dot2(i00, Q02, i01, Q12), i12 = -dot2(i10, Q02, i11, Q12);
  float r00 = dot2(i00, P00, i01, P10), r01 = dot2(i00, P01, i01, P11), r02 = dot2(i00, P02, i01, P12) + i02;
  float r10 = dot2(i10, P00, i11, P10), r11 = dot2(i10, P01, i11, P11), r12 = dot2(i10, P02, i11, P12) + i12;
  for (int s = 0; s < ns; ++s) {
    float n00 = dot2(r00, r00, r01, r10), n01 = dot2(r00, r01, r01, r11), n02 = dot2(r00, r02, r01, r12) + r02;
    float n10 = dot2(r10, r00, r11, r10), n11 = dot2(r10, r01, r11, r11), n12 = dot2(r10, r02, r11, r12) + r12;
    r00 = n00; r01 = n01; r02 = n02; r10 = n10; r11 = n11; r12 = n12;
  }
  out[0] = r00; out[1] = r01; out[2] = r02; out[3] = r10; out[4] = r11; out[5] = r12;
}

static void expm3d(const float *A, float dT, float *out) {
  float m[3][4];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 4; ++j) m[i][j] = dT * A[i * 4 + j];
  float sq = dot2(m[0][0], m[0][0], m[0][1], m[0][1]);
  for (int k = 2; k < 12; ++k) sq = fmaf(m[k / 4][k % 4], m[k / 4][k % 4], sq);
  int ns = n_squarings(sqrtf(sq));
  float sc = 1.0f;
  for (int i = 0; i < ns; ++i) sc *= 0.5f;
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 4; ++j) m[i][j] *= sc;
  float q[3][3], qt[3];
  for (int i = 0; i < 3; ++i) {
    for (int j = 0; j < 3; ++j) q[i][j] = dot3(m[i][0], m[0][j], m[i][1], m[1][j], m[i][2], m[2][j]);
    qt[i] = dot3(m[i][0], m[0][3], m[i][1], m[1][3], m[i][2], m[2][3]);
  }
  const float t12 = 1.0f / 12.0f;
  float P[3][3], Q[3][3], pt[3], qtt[3];
  for (int i = 0; i < 3; ++i) {
    for (int j = 0; j < 3; ++j) {
      P[i][j] = i == j ? pdiag(0.5f, m[i][j], t12, q[i][j]) : poff(0.5f, m[i][j], t12, q[i][j]);
      Q[i][j] = i == j ? pdiag(-0.5f, m[i][j], t12, q[i][j]) : poff(-0.5f, m[i][j], t12, q[i][j]);
    }
    pt[i] = poff(0.5f, m[i][3], t12, qt[i]);
    qtt[i] = poff(-0.5f, m[i][3], t12, qt[i]);
  }
  float c0 = diff2(Q[1][1], Q[2][2], Q[1][2], Q[2][1]);
  float c1 = diff2(Q[1][0], Q[2][2], Q[1][2], Q[2][0]);
  float c2 = diff2(Q[1][0], Q[2][1], Q[1][1], Q[2][0]);
  float id = 1.0f / fmaf(Q[0][2], c2, fmaf(Q[0][0], c0, -(Q[0][1] * c1)));
  float I[3][3];
  I[0][0] = c0 * id;
  I[0][1] = diff2(Q[0][2], Q[2][1], Q[0][1], Q[2][2]) * id;
  I[0][2] = diff2(Q[0][1], Q[1][2], Q[0][2], Q[1][1]) * id;
  I[1][0] = diff2(Q[1][2], Q[2][0], Q[1][0], Q[2][2]) * id;
  I[1][1] = diff2(Q[0][0], Q[2][2], Q[0][2], Q[2][0]) * id;
  I[1][2] = diff2(Q[0][2], Q[1][0], Q[0][0], Q[1][2]) * id;
  I[2][0] = c2 * id;
  I[2][1] = diff2(Q[0][1], Q[2][0], Q[0][0], Q[2][1]) * id;
  I[2][2] = diff2(Q[0][0], Q[1][1], Q[0][1], Q[1][0]) * id;
  float R[3][3], rt[3];
  for (int i = 0; i < 3; ++i) {
    float it = -dot3(I[i][0], qtt[0], I[i][1], qtt[1], I[i][2], qtt[2]);
    for (int j = 0; j < 3; ++j) R[i][j] = dot3(I[i][0], P[0][j], I[i][1], P[1][j], I[i][2], P[2][j]);
    rt[i] = dot3(I[i][0], pt[0], I[i][1], pt[1], I[i][2], pt[2]) + it;
  }
  for (int s = 0; s < ns; ++s) {
    float N[3][3], nt[3];
    for (int i = 0; i < 3; ++i) {
      for (int j = 0; j < 3; ++j) N[i][j] = dot3(R[i][0], R[0][j], R[i][1], R[1][j], R[i][2], R[2][j]);
      nt[i] = dot3(R[i][0], rt[0], R[i][1], rt[1], R[i][2], rt[2]) + rt[i];
    }
    memcpy(R, N, sizeof(R));
    memcpy(rt, nt, sizeof(rt));
  }
  for (int i = 0; i < 3; ++i) {
    for (int j = 0; j < 3; ++j) out[i * 4 + j] = R[i][j];
    out[i * 4 + 3] = rt[i];
  }
}

void oracle_expm(int nd, const float *As, int64_t n, float dT, float *out) {
  const int P = nd * (nd + 1);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    if (nd == 1) expm1d(As + i * P, dT, out + i * P);
    else if (nd == 2) expm2d(As + i * P, dT, out + i * P);
    else expm3d(As + i * P, dT, out + i * P);
  }
}

/* ----------------------------------------------------------- 1D closed form */

static int sgnf(float x) { return (x > 0.0f) - (x < 0.0f); }
static int near0(float x) { return fabsf(x) < 1e-7f; }

static float hit_time(float x, float t, int c, float a, float b, int nx, float *xc, int *cc) {
  int s = sgnf(t);
  float never = INFINITY * (float)s;
  float v = fmaf(a, x, b);
  if (near0(v)) return never;
  *cc = c + sgnf(v) * s;
  if (*cc < 0 || *cc >= nx) return never;
  float right = ((float)(c + 1) / (float)nx) + 1e-7f;
  float left = ((float)c / (float)nx) - 1e-7f;
  if (t > 0.0f)
    *xc = (v > 0.0f) ? right : left;
  else
    *xc = (v > 0.0f) ? left : right;
  float vc = fmaf(a, *xc, b);
  if (near0(vc)) return never;
  if (sgnf(v) != sgnf(vc)) return never;
  if (*xc <= 0.0f || *xc >= 1.0f) return never;
  if (near0(a)) return (*xc - x) / b;
  return logf(vc / v) / a;
}

static float closed_form_1d(float x, float t, const float *A, tess_t ts) {
  int c = cell1(x, ts);
  int hops = 0;
  int hopmax = (c > ts.nx - 1 - c ? c : ts.nx - 1 - c) + 1;
  int s = sgnf(t);
  for (;;) {
    float a = A[2 * c], b = A[2 * c + 1];
    float xc = x;
    int cc = c;
    float th = hit_time(x, t, c, a, b, ts.nx, &xc, &cc);
    if ((float)s * th > (float)s * t) {
      if (near0(a)) return fmaf(t, b, x);
      float ba = b / a;
      return fmaf(expf(t * a), x + ba, -ba);
    }
    x = xc;
    c = cc;
    t -= th;
    if (++hops > hopmax) break;
  }
  return x;
}

/* --------------------------------------------------------------- forward */

void oracle_forward(int nd, const int32_t *nc, const float *pts, int64_t nP, int batched,
                    const float *trels, const float *As, int n_theta, int T, int adaptive,
                    float *out) {
  tess_t ts = make_tess(nd, nc);
  const int P = nd * (nd + 1);
  const int64_t nC = n_cells(nd, ts);
  const float h = 1.0f / (float)T;
  const float hh = 0.5f * h;
#pragma omp parallel for collapse(2) schedule(static)
  for (int b = 0; b < n_theta; ++b) {
    for (int64_t i = 0; i < nP; ++i) {
      const float *src = pts + (batched ? (int64_t)b * nd * nP : 0);
      const float *Ab = As + (int64_t)b * nC * P;
      float *dst = out + (int64_t)b * nd * nP;
      if (nd == 1) {
        dst[i] = closed_form_1d(src[i], 1.0f, Ab, ts);
        continue;
      }
      const float *Tb = trels + (int64_t)b * nC * P;
      float p[3], q[3];
      for (int k = 0; k < nd; ++k) p[k] = src[k * nP + i];
      for (int n = 0; n < T; ++n) {
        int c = cell_nd(nd, p, ts);
        affine(nd, Tb + (int64_t)c * P, p, q);
        if (adaptive) {
          int ce = cell_nd(nd, q, ts);
          if (ce != c) {
            float v0[3], v1[3];
            affine(nd, Ab + (int64_t)c * P, p, v0);
            affine(nd, Ab + (int64_t)ce * P, q, v1);
            for (int k = 0; k < nd; ++k) p[k] = fmaf(hh, v0[k] + v1[k], p[k]);
            continue;
          }
        }
        for (int k = 0; k < nd; ++k) p[k] = q[k];
      }
      for (int k = 0; k < nd; ++k) dst[k * nP + i] = p[k];
    }
  }
}

/* -------------------------------------------------------------- backward */

/* Midpoint step in cell c's matrix; Heun across a facet when adaptive. */
static int replay(int nd, tess_t ts, const float *Ab, float *p, float h, float hh, int adaptive) {
  const int P = nd * (nd + 1);
  int c = cell_nd(nd, p, ts);
  const float *m = Ab + (int64_t)c * P;
  float v[3], q[3], w[3], e[3];
  affine(nd, m, p, v);
  for (int k = 0; k < nd; ++k) q[k] = fmaf(hh, v[k], p[k]);
  affine(nd, m, q, w);
  for (int k = 0; k < nd; ++k) e[k] = fmaf(h, w[k], p[k]);
  if (adaptive) {
    int ce = cell_nd(nd, e, ts);
    if (ce != c) {
      float v1[3];
      affine(nd, Ab + (int64_t)ce * P, e, v1);
      for (int k = 0; k < nd; ++k) p[k] = fmaf(hh, v[k] + v1[k], p[k]);
      return c;
    }
  }
  for (int k = 0; k < nd; ++k) p[k] = e[k];
  return c;
}

/* Reverse step of the midpoint adjoint in matrix m at step start p. */
static void adjoint(int nd, const float *m, const float *p, float *lam, float *mo, float h, float hh) {
  const int C = nd + 1;
  float v[3], q[3], at[3], lm[3];
  affine(nd, m, p, v);
  for (int k = 0; k < nd; ++k) q[k] = fmaf(hh, v[k], p[k]);
  for (int k = 0; k < nd; ++k) {
    float s = m[k] * lam[0];
    for (int r = 1; r < nd; ++r) s = s + m[r * C + k] * lam[r];
    at[k] = s;
  }
  for (int r = 0; r < nd; ++r) {
    float wq = h * lam[r];
    for (int k = 0; k < nd; ++k) mo[r * C + k] += wq * q[k];
    mo[r * C + nd] += wq;
  }
  for (int r = 0; r < nd; ++r) {
    float wp = hh * h * at[r];
    for (int k = 0; k < nd; ++k) mo[r * C + k] += wp * p[k];
    mo[r * C + nd] += wp;
  }
  for (int k = 0; k < nd; ++k) lm[k] = lam[k] + hh * at[k];
  for (int k = 0; k < nd; ++k) {
    float s = m[k] * lm[0];
    for (int r = 1; r < nd; ++r) s = s + m[r * C + k] * lm[r];
    lam[k] += h * s;
  }
}

void oracle_backward(int nd, const int32_t *nc, const float *pts, int64_t nP, int batched,
                     const float *As, int n_theta, const float *grad_out, int T, int adaptive,
                     float *moments, float *grad_points) {
  tess_t ts = make_tess(nd, nc);
  const int P = nd * (nd + 1);
  const int64_t nC = n_cells(nd, ts);
  const int64_t msize = (int64_t)n_theta * nC * P;
  const float h = 1.0f / (float)T;
  const float hh = h * 0.5f;
  int nthr = 1;
#ifdef _OPENMP
  nthr = omp_get_max_threads();
#endif
  float *part = (float *)calloc((size_t)nthr * msize, sizeof(float));
  if (T > ORACLE_MAX_STEPS) T = ORACLE_MAX_STEPS;
#pragma omp parallel
  {
    int tid = 0;
#ifdef _OPENMP
    tid = omp_get_thread_num();
#endif
    float *mine = part + (int64_t)tid * msize;
    float traj[(ORACLE_MAX_STEPS + 1) * 3];
    int cells[ORACLE_MAX_STEPS];
#pragma omp for collapse(2) schedule(static)
    for (int b = 0; b < n_theta; ++b) {
      for (int64_t i = 0; i < nP; ++i) {
        const float *src = pts + (batched ? (int64_t)b * nd * nP : 0);
        const float *Ab = As + (int64_t)b * nC * P;
        float *mb = mine + (int64_t)b * nC * P;
        float p[3];
        for (int k = 0; k < nd; ++k) p[k] = src[k * nP + i];
        for (int n = 0; n < T; ++n) {
          for (int k = 0; k < nd; ++k) traj[n * 3 + k] = p[k];
          cells[n] = replay(nd, ts, Ab, p, h, hh, adaptive);
        }
        float lam[3], mo[12] = {0};
        const float *g = grad_out + (int64_t)b * nd * nP;
        for (int k = 0; k < nd; ++k) lam[k] = g[k * nP + i];
        int prev = -1;
        for (int n = T - 1; n >= 0; --n) {
          int c = cells[n];
          if (c != prev && prev >= 0) {
            for (int k = 0; k < P; ++k) {
              mb[(int64_t)prev * P + k] += mo[k];
              mo[k] = 0.0f;
            }
          }
          prev = c;
          adjoint(nd, Ab + (int64_t)c * P, traj + n * 3, lam, mo, h, hh);
        }
        if (prev >= 0)
          for (int k = 0; k < P; ++k) mb[(int64_t)prev * P + k] += mo[k];
        if (grad_points) {
          float *gp = grad_points + (int64_t)b * nd * nP;
          for (int k = 0; k < nd; ++k) gp[k * nP + i] = lam[k];
        }
      }
    }
  }
  memset(moments, 0, (size_t)msize * sizeof(float));
  for (int t = 0; t < nthr; ++t) {
    const float *src = part + (int64_t)t * msize;
    for (int64_t k = 0; k < msize; ++k) moments[k] += src[k];
  }
  free(part);
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* The trajectory the adjoint differentiates: T midpoint steps (Heun across a
 * facet when adaptive), i.e. the replay of the backward kernels.  Used to
 * check the adjoint against finite differences. */
void oracle_midpoint_forward(int nd, const int32_t *nc, const float *pts, int64_t nP, int batched,
                             const float *As, int n_theta, int T, int adaptive, float *out) {
  tess_t ts = make_tess(nd, nc);
  const int P = nd * (nd + 1);
  const int64_t nC = n_cells(nd, ts);
  const float h = 1.0f / (float)T;
  const float hh = h * 0.5f;
#pragma omp parallel for collapse(2) schedule(static)
  for (int b = 0; b < n_theta; ++b) {
    for (int64_t i = 0; i < nP; ++i) {
      const float *src = pts + (batched ? (int64_t)b * nd * nP : 0);
      float p[3];
      for (int k = 0; k < nd; ++k) p[k] = src[k * nP + i];
      for (int n = 0; n < T; ++n) replay(nd, ts, As + (int64_t)b * nC * P, p, h, hh, adaptive);
      for (int k = 0; k < nd; ++k) out[(int64_t)b * nd * nP + k * nP + i] = p[k];
    }
  }
}

/* out[t, r] = sum over row r of a CSR matrix of vals * x[t, col] in float32,
 * in the order the GPU kernels use (the reference computes these products with
 * torch.sparse.mm, cpab/pytorch/transformer.py:84 and :166, whose fp32 order
 * is the library's).  chunk = 0: one fmaf chain over the row (k_build_A);
 * chunk = K: an fmaf chain over every K consecutive nonzeros, and the chunk
 * sums added left to right (k_project, whose chunks are summed by different
 * warps).  A row of at most K nonzeros gets the single chain either way. */
static float chunked_dot(const int32_t *colidx, const float *vals, int32_t k0, int32_t k1,
                         const float *x, int K) {
  if (K <= 0) K = k1 - k0 > 0 ? k1 - k0 : 1;
  float total = 0.0f;
  for (int32_t kc = k0; kc < k1; kc += K) {
    const int32_t ke = kc + K < k1 ? kc + K : k1;
    float s = 0.0f;
    for (int32_t k = kc; k < ke; ++k) s = fmaf(vals[k], x[colidx[k]], s);
    total = kc == k0 ? s : total + s;
  }
  return total;
}

void oracle_csr_matmul(int64_t rows, const int32_t *rowptr, const int32_t *colidx,
                       const float *vals, int n_rhs, const float *x, int64_t x_stride,
                       float *out, int64_t out_stride, int chunk) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int t = 0; t < n_rhs; ++t) {
    for (int64_t r = 0; r < rows; ++r) {
      out[(int64_t)t * out_stride + r] = chunked_dot(colidx, vals, rowptr[r], rowptr[r + 1],
                                                     x + (int64_t)t * x_stride, chunk);
    }
  }
}
