// Parameter-space kernels: A = B theta (fused with the per-cell matrix
// exponential Trels = expm(dT A)), the stand-alone expm, and the projection
// dtheta = B^T vec(M).
//
// These are small sparse contractions (a handful of nonzeros per row for
// zero-boundary bases, dozens for general ones) -- gathers, not GEMMs -- so
// they run on the SIMT pipes, one warp per cell (A-build) or per basis column
// (projection) with the nonzeros split over the lanes.
#include <cuda_runtime.h>

#include "launch.h"

namespace cpab {

namespace {

// ---------------------------------------------------------------------------
// Matrix exponential of the affine matrix dT*[A; 0 .. 0] (top rows only).
// Scaling and squaring with the (2,2) Pade approximant
//   R = (I - M/2 + M^2/12)^-1 (I + M/2 + M^2/12),
// the scheme of cpab/core/cpab_ops_2d.cu:585-701 (2D) and
// cpab/core/cpab_ops_3d.cu:538-674 (3D); the 1D case is the closed form of
// cpab/core/cpab_ops_1d.cu:442-467.
//
// Every sum of products is evaluated left to right with the first two
// products fused as fma(a, b, c*d) and each further product fused onto the
// running sum -- the rounding the reference's kernels get from the compiler,
// written out explicitly so that the result does not depend on contraction
// heuristics.  (Checked bit for bit against Trels computed by the
// reference's own kernels on a B200.)
// ---------------------------------------------------------------------------

__device__ __forceinline__ float dot2(float a, float b, float c, float d) {
  return __fmaf_rn(a, b, __fmul_rn(c, d));
}
__device__ __forceinline__ float dot3(float a, float b, float c, float d, float e, float f) {
  return __fmaf_rn(e, f, __fmaf_rn(a, b, __fmul_rn(c, d)));
}
__device__ __forceinline__ float diff2(float a, float b, float c, float d) {
  return __fmaf_rn(a, b, -__fmul_rn(c, d));
}
// 1 + h m + s q, h m + s q  (Pade numerator/denominator entries)
__device__ __forceinline__ float pade_diag(float h, float m, float s, float q) {
  return __fmaf_rn(s, q, __fmaf_rn(h, m, 1.0f));
}
__device__ __forceinline__ float pade_off(float h, float m, float s, float q) {
  return __fmaf_rn(h, m, __fmul_rn(s, q));
}

__device__ __forceinline__ int squarings(float norm) {
  return norm > 0.5f ? (int)ceilf(log2f(norm * 2.0f)) : 0;
}

__device__ __forceinline__ void expm1d(const float (&a)[2], float dT, float (&r)[2]) {
  const float m0 = __fmul_rn(dT, a[0]);
  const float m1 = __fmul_rn(dT, a[1]);
  float rel;  // (e^m0 - 1) / m0
  if (fabsf(m0) > 1e-6f) {
    rel = expm1f(m0) / m0;
  } else {
    const float sq = __fmul_rn(m0, m0);
    rel = __fmaf_rn(__fmul_rn(1.0f / 24.0f, sq), m0,
                    __fmaf_rn(1.0f / 6.0f, sq, __fmaf_rn(0.5f, m0, 1.0f)));
  }
  r[0] = expf(m0);
  r[1] = __fmul_rn(m1, rel);
}

__device__ __forceinline__ void expm2d(const float (&a)[6], float dT, float (&r)[6]) {
  float m[6];
#pragma unroll
  for (int k = 0; k < 6; ++k) m[k] = __fmul_rn(dT, a[k]);
  float sq = dot2(m[0], m[0], m[1], m[1]);
#pragma unroll
  for (int k = 2; k < 6; ++k) sq = __fmaf_rn(m[k], m[k], sq);
  const int ns = squarings(sqrtf(sq));
  float sc = 1.0f;
  for (int i = 0; i < ns; ++i) sc *= 0.5f;
#pragma unroll
  for (int k = 0; k < 6; ++k) m[k] = __fmul_rn(m[k], sc);
  // Rows of M^2 (the third row of M is zero).
  const float s00 = dot2(m[0], m[0], m[1], m[3]), s01 = dot2(m[0], m[1], m[1], m[4]);
  const float s02 = dot2(m[0], m[2], m[1], m[5]), s10 = dot2(m[3], m[0], m[4], m[3]);
  const float s11 = dot2(m[3], m[1], m[4], m[4]), s12 = dot2(m[3], m[2], m[4], m[5]);
  const float c12 = 1.0f / 12.0f;
  // Numerator N = I + M/2 + M^2/12, denominator D = I - M/2 + M^2/12.
  const float n00 = pade_diag(0.5f, m[0], c12, s00), d00 = pade_diag(-0.5f, m[0], c12, s00);
  const float n01 = pade_off(0.5f, m[1], c12, s01), d01 = pade_off(-0.5f, m[1], c12, s01);
  const float n02 = pade_off(0.5f, m[2], c12, s02), d02 = pade_off(-0.5f, m[2], c12, s02);
  const float n10 = pade_off(0.5f, m[3], c12, s10), d10 = pade_off(-0.5f, m[3], c12, s10);
  const float n11 = pade_diag(0.5f, m[4], c12, s11), d11 = pade_diag(-0.5f, m[4], c12, s11);
  const float n12 = pade_off(0.5f, m[5], c12, s12), d12 = pade_off(-0.5f, m[5], c12, s12);
  // D^-1 = [Di, -Di d_t; 0 1] with Di the inverse of D's 2x2 linear block.
  const float idet = 1.0f / diff2(d00, d11, d01, d10);
  const float i00 = __fmul_rn(d11, idet), i01 = __fmul_rn(-d01, idet);
  const float i10 = __fmul_rn(-d10, idet), i11 = __fmul_rn(d00, idet);
  const float i02 = -dot2(i00, d02, i01, d12);
  const float i12 = -dot2(i10, d02, i11, d12);
  float r00 = dot2(i00, n00, i01, n10), r01 = dot2(i00, n01, i01, n11);
  float r02 = __fadd_rn(dot2(i00, n02, i01, n12), i02);
  float r10 = dot2(i10, n00, i11, n10), r11 = dot2(i10, n01, i11, n11);
  float r12 = __fadd_rn(dot2(i10, n02, i11, n12), i12);
  for (int i = 0; i < ns; ++i) {
    const float t00 = dot2(r00, r00, r01, r10), t01 = dot2(r00, r01, r01, r11);
    const float t02 = __fadd_rn(dot2(r00, r02, r01, r12), r02);
    const float t10 = dot2(r10, r00, r11, r10), t11 = dot2(r10, r01, r11, r11);
    const float t12 = __fadd_rn(dot2(r10, r02, r11, r12), r12);
    r00 = t00; r01 = t01; r02 = t02; r10 = t10; r11 = t11; r12 = t12;
  }
  r[0] = r00; r[1] = r01; r[2] = r02; r[3] = r10; r[4] = r11; r[5] = r12;
}

__device__ __forceinline__ void expm3d(const float (&a)[12], float dT, float (&r)[12]) {
  // L = linear 3x3 block, u = translation column, both scaled by dT.
  float L[3][3], u[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) L[i][j] = __fmul_rn(dT, a[i * 4 + j]);
    u[i] = __fmul_rn(dT, a[i * 4 + 3]);
  }
  // Squared Frobenius norm in row-major order (translation last in each row).
  float sq = dot2(L[0][0], L[0][0], L[0][1], L[0][1]);
  sq = __fmaf_rn(L[0][2], L[0][2], sq);
  sq = __fmaf_rn(u[0], u[0], sq);
#pragma unroll
  for (int i = 1; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) sq = __fmaf_rn(L[i][j], L[i][j], sq);
    sq = __fmaf_rn(u[i], u[i], sq);
  }
  const int ns = squarings(sqrtf(sq));
  float sc = 1.0f;
  for (int i = 0; i < ns; ++i) sc *= 0.5f;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) L[i][j] = __fmul_rn(L[i][j], sc);
    u[i] = __fmul_rn(u[i], sc);
  }
  float S[3][3], su[3];  // M^2: linear block L*L and translation L*u
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j)
      S[i][j] = dot3(L[i][0], L[0][j], L[i][1], L[1][j], L[i][2], L[2][j]);
    su[i] = dot3(L[i][0], u[0], L[i][1], u[1], L[i][2], u[2]);
  }
  const float c12 = 1.0f / 12.0f;
  float N[3][3], D[3][3], nu[3], du[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      N[i][j] = i == j ? pade_diag(0.5f, L[i][j], c12, S[i][j]) : pade_off(0.5f, L[i][j], c12, S[i][j]);
      D[i][j] = i == j ? pade_diag(-0.5f, L[i][j], c12, S[i][j]) : pade_off(-0.5f, L[i][j], c12, S[i][j]);
    }
    nu[i] = pade_off(0.5f, u[i], c12, su[i]);
    du[i] = pade_off(-0.5f, u[i], c12, su[i]);
  }
  // Inverse of D's linear block by cofactors.
  const float c0 = diff2(D[1][1], D[2][2], D[1][2], D[2][1]);
  const float c1 = diff2(D[1][0], D[2][2], D[1][2], D[2][0]);
  const float c2 = diff2(D[1][0], D[2][1], D[1][1], D[2][0]);
  const float id = 1.0f / __fmaf_rn(D[0][2], c2, __fmaf_rn(D[0][0], c0, -__fmul_rn(D[0][1], c1)));
  float I[3][3];
  I[0][0] = __fmul_rn(c0, id);
  I[0][1] = __fmul_rn(diff2(D[0][2], D[2][1], D[0][1], D[2][2]), id);
  I[0][2] = __fmul_rn(diff2(D[0][1], D[1][2], D[0][2], D[1][1]), id);
  I[1][0] = __fmul_rn(diff2(D[1][2], D[2][0], D[1][0], D[2][2]), id);
  I[1][1] = __fmul_rn(diff2(D[0][0], D[2][2], D[0][2], D[2][0]), id);
  I[1][2] = __fmul_rn(diff2(D[0][2], D[1][0], D[0][0], D[1][2]), id);
  I[2][0] = __fmul_rn(c2, id);
  I[2][1] = __fmul_rn(diff2(D[0][1], D[2][0], D[0][0], D[2][1]), id);
  I[2][2] = __fmul_rn(diff2(D[0][0], D[1][1], D[0][1], D[1][0]), id);
  float R[3][3], ru[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const float it = -dot3(I[i][0], du[0], I[i][1], du[1], I[i][2], du[2]);
#pragma unroll
    for (int j = 0; j < 3; ++j)
      R[i][j] = dot3(I[i][0], N[0][j], I[i][1], N[1][j], I[i][2], N[2][j]);
    ru[i] = __fadd_rn(dot3(I[i][0], nu[0], I[i][1], nu[1], I[i][2], nu[2]), it);
  }
  for (int s = 0; s < ns; ++s) {
    float Q[3][3], qu[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
#pragma unroll
      for (int j = 0; j < 3; ++j)
        Q[i][j] = dot3(R[i][0], R[0][j], R[i][1], R[1][j], R[i][2], R[2][j]);
      qu[i] = __fadd_rn(dot3(R[i][0], ru[0], R[i][1], ru[1], R[i][2], ru[2]), ru[i]);
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) {
#pragma unroll
      for (int j = 0; j < 3; ++j) R[i][j] = Q[i][j];
      ru[i] = qu[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) r[i * 4 + j] = R[i][j];
    r[i * 4 + 3] = ru[i];
  }
}

template <int ND>
__device__ __forceinline__ void expm_cell(const float (&a)[Dim<ND>::kPpc], float dT,
                                          float (&r)[Dim<ND>::kPpc]) {
  if constexpr (ND == 1) expm1d(a, dT, r);
  else if constexpr (ND == 2) expm2d(a, dT, r);
  else expm3d(a, dT, r);
}

template <int ND>
__global__ void k_expm(const float *__restrict__ As, int64_t n, float dT, float *__restrict__ trels) {
  constexpr int P = Dim<ND>::kPpc;
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  float a[P], r[P];
#pragma unroll
  for (int k = 0; k < P; ++k) a[k] = __ldg(As + i * P + k);
  expm_cell<ND>(a, dT, r);
#pragma unroll
  for (int k = 0; k < P; ++k) trels[i * P + k] = r[k];
}

// Dot products of CSR row [k0, k1) with up to TC vectors x + u * stride
// (u < nt), split over the 32 lanes of a warp: lane l sums products k0 + l,
// k0 + l + 32, ... of every vector with an fmaf chain, and an xor butterfly
// adds the lane partials; every lane returns all sums.  The index and value
// of a nonzero are loaded once for the TC vectors, and the TC gathers and
// chains are independent, so a warp keeps TC loads in flight instead of one.
// (The per-vector order is fixed; the CPU oracle restates it.)
constexpr int kDotChunk = 8;

template <int TC>
__device__ __forceinline__ void warp_dots(const int32_t *__restrict__ colidx,
                                          const float *__restrict__ vals, int k0, int k1,
                                          const float *__restrict__ x, int64_t stride, int nt,
                                          float (&out)[TC]) {
#pragma unroll
  for (int u = 0; u < TC; ++u) out[u] = 0.0f;
  for (int k = k0 + (threadIdx.x & 31); k < k1; k += 32) {
    const float v = __ldg(vals + k);
    const float *xc = x + __ldg(colidx + k);
#pragma unroll
    for (int u = 0; u < TC; ++u)
      if (u < nt) out[u] = fmaf(v, __ldg(xc + u * stride), out[u]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
    for (int u = 0; u < TC; ++u) out[u] += __shfl_xor_sync(0xffffffffu, out[u], off);
  }
}

// A = B theta (and Trels = expm(A dT) when trels != NULL), in one of two
// mappings chosen on the device from B's nonzeros (rowptr[nC * P], one
// broadcast load, so the host needs no copy and the call stays asynchronous):
//   * sparse B (at most 4 nonzeros per row on average; zero-boundary bases
//     have <= 4 in every row): one thread per (transformation, cell), each row
//     summed with a sequential fmaf chain;
//   * otherwise one warp per cell: each row's nonzeros split over the lanes
//     (warp_dots), lane j keeping transformation t0 + j's entries, then each
//     lane computes the exponential, 32 transformations wide.
// The grid covers nC warps; the sparse mapping strides over nC * n_theta.
template <int ND>
__global__ void __launch_bounds__(256) k_build_A(int64_t nC, int64_t d, int n_theta,
                                                 const int32_t *__restrict__ rowptr,
                                                 const int32_t *__restrict__ colidx,
                                                 const float *__restrict__ vals,
                                                 const float *__restrict__ theta, float dT,
                                                 float *__restrict__ As,
                                                 float *__restrict__ trels) {
  constexpr int P = Dim<ND>::kPpc;
  const int64_t gtid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const bool sparse = __ldg(rowptr + nC * P) <= 4 * nC * P;
  if (sparse) {
    const int64_t n = nC * n_theta;
    for (int64_t i = gtid; i < n; i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t t = i / nC;
      const int64_t c = i - t * nC;
      const float *th = theta + t * d;
      float a[P];
#pragma unroll
      for (int r = 0; r < P; ++r) {
        const int k0 = __ldg(rowptr + c * P + r), k1 = __ldg(rowptr + c * P + r + 1);
        float sum = 0.0f;
        for (int k = k0; k < k1; ++k) sum = fmaf(__ldg(vals + k), __ldg(th + __ldg(colidx + k)), sum);
        a[r] = sum;
      }
#pragma unroll
      for (int r = 0; r < P; ++r) As[i * P + r] = a[r];
      if (trels != nullptr) {
        float e[P];
        expm_cell<ND>(a, dT, e);
#pragma unroll
        for (int r = 0; r < P; ++r) trels[i * P + r] = e[r];
      }
    }
    return;
  }
  const int64_t c = gtid >> 5;
  const int lane = threadIdx.x & 31;
  if (c >= nC) return;  // whole warps exit together
  int k0[P], k1[P];
#pragma unroll
  for (int r = 0; r < P; ++r) {
    k0[r] = __ldg(rowptr + c * P + r);
    k1[r] = __ldg(rowptr + c * P + r + 1);
  }
  for (int t0 = 0; t0 < n_theta; t0 += 32) {
    float mine[P];  // entries of transformation t0 + lane
#pragma unroll
    for (int r = 0; r < P; ++r) mine[r] = 0.0f;
    const int tn = min(32, n_theta - t0);
    for (int j0 = 0; j0 < tn; j0 += kDotChunk) {
      const float *th = theta + (int64_t)(t0 + j0) * d;
#pragma unroll
      for (int r = 0; r < P; ++r) {
        float sums[kDotChunk];
        warp_dots<kDotChunk>(colidx, vals, k0[r], k1[r], th, d, tn - j0, sums);
#pragma unroll
        for (int u = 0; u < kDotChunk; ++u)
          if (lane == j0 + u) mine[r] = sums[u];
      }
    }
    if (lane < tn) {
      const int64_t base = ((int64_t)(t0 + lane) * nC + c) * P;
#pragma unroll
      for (int r = 0; r < P; ++r) As[base + r] = mine[r];
      if (trels != nullptr) {
        float e[P];
        expm_cell<ND>(mine, dT, e);
#pragma unroll
        for (int r = 0; r < P; ++r) trels[base + r] = e[r];
      }
    }
  }
}

// dtheta[t, j] = sum over row j of B^T of vals * moments[t, col].  One warp
// per basis column j (warp_dots; clustered column indices let the moment
// gathers share sectors).  Columns have 16 to 80 nonzeros for zero-boundary
// bases and up to ~1,700 for general ones.
__global__ void __launch_bounds__(256) k_project(int64_t d, int64_t D, int n_theta,
                                                 const int32_t *__restrict__ rowptr,
                                                 const int32_t *__restrict__ colidx,
                                                 const float *__restrict__ vals,
                                                 const float *__restrict__ moments,
                                                 float *__restrict__ dtheta) {
  const int64_t j = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (j >= d) return;
  const int k0 = __ldg(rowptr + j), k1 = __ldg(rowptr + j + 1);
  const int lane = threadIdx.x & 31;
  for (int t0 = 0; t0 < n_theta; t0 += kDotChunk) {
    float sums[kDotChunk];
    warp_dots<kDotChunk>(colidx, vals, k0, k1, moments + (int64_t)t0 * D, D, n_theta - t0, sums);
#pragma unroll
    for (int u = 0; u < kDotChunk; ++u)
      if (lane == u && t0 + u < n_theta) dtheta[(int64_t)(t0 + u) * d + j] = sums[u];
  }
}

constexpr int kThreads = 256;

inline unsigned blocks_for(int64_t n) { return (unsigned)((n + kThreads - 1) / kThreads); }

}  // namespace

cudaError_t launch_expm(int ndim, const float *As, int64_t n, float dT, float *trels,
                        cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  switch (ndim) {
    case 1: k_expm<1><<<blocks_for(n), kThreads, 0, s>>>(As, n, dT, trels); break;
    case 2: k_expm<2><<<blocks_for(n), kThreads, 0, s>>>(As, n, dT, trels); break;
    default: k_expm<3><<<blocks_for(n), kThreads, 0, s>>>(As, n, dT, trels); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_build_A(int ndim, int64_t nC, int64_t d, int n_theta, const int32_t *rowptr,
                           const int32_t *colidx, const float *vals, const float *theta,
                           float dT, float *As, float *trels, cudaStream_t s) {
  if (nC * n_theta == 0) return cudaSuccess;
  const int64_t n = nC * 32;  // one warp per cell
  switch (ndim) {
    case 1:
      k_build_A<1><<<blocks_for(n), kThreads, 0, s>>>(nC, d, n_theta, rowptr, colidx, vals, theta,
                                                      dT, As, trels);
      break;
    case 2:
      k_build_A<2><<<blocks_for(n), kThreads, 0, s>>>(nC, d, n_theta, rowptr, colidx, vals, theta,
                                                      dT, As, trels);
      break;
    default:
      k_build_A<3><<<blocks_for(n), kThreads, 0, s>>>(nC, d, n_theta, rowptr, colidx, vals, theta,
                                                      dT, As, trels);
      break;
  }
  return cudaGetLastError();
}

cudaError_t launch_project(int64_t d, int64_t D, int n_theta, const int32_t *rowptr,
                           const int32_t *colidx, const float *vals, const float *moments,
                           float *dtheta, cudaStream_t s) {
  if (d * n_theta == 0) return cudaSuccess;
  const int64_t n = d * 32;  // one warp per basis column
  k_project<<<blocks_for(n), kThreads, 0, s>>>(d, D, n_theta, rowptr, colidx, vals, moments,
                                               dtheta);
  return cudaGetLastError();
}

}  // namespace cpab
