// Parameter-space kernels: A = B theta (fused with the per-cell matrix
// exponential Trels = expm(dT A)), the stand-alone expm, and the projection
// dtheta = B^T vec(M).
//
// These are small sparse contractions (a handful of nonzeros per row for
// zero-boundary bases, dozens for general ones) -- gathers, not GEMMs -- so
// they run on the SIMT pipes, one warp per cell (A-build) or per basis column
// (projection) with the lanes over the transformations.
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

// Rows of a CSR matrix times up to 32 vectors at once, lanes over the vectors:
// lane u of a warp sums row r of M times x[t0 + u] (x + (t0 + u) * stride)
// with one sequential fmaf chain over the row's nonzeros -- the summation
// order the CPU oracle restates.  The gathers x[t][col] of a row are staged
// through shared memory 32 nonzeros at a time: lanes over nonzeros load a
// vector's entries (the column indices of a row are sorted and clustered, so
// these loads coalesce), store them transposed with a padded stride (33:
// conflict-free both ways), then each lane reads its own vector's column.
// A nonzero's value and column are loaded once for all vectors.
constexpr int kStage = 32;
constexpr int kStagePad = 33;
constexpr int kWarpsPerBlock = 8;  // kThreads / 32

struct WarpStage {
  float x[kStage * kStagePad];
  float v[kStage];
};

__device__ __forceinline__ float row_times_lane_vector(const int32_t *__restrict__ colidx,
                                                       const float *__restrict__ vals, int k0,
                                                       int k1, const float *__restrict__ x,
                                                       int64_t stride, int nt,
                                                       WarpStage &st) {
  const int lane = threadIdx.x & 31;
  float acc = 0.0f;
  for (int kc = k0; kc < k1; kc += kStage) {
    const int n = min(kStage, k1 - kc);
    __syncwarp();
    if (lane < n) {
      const int col = __ldg(colidx + kc + lane);
      st.v[lane] = __ldg(vals + kc + lane);
      const float *xc = x + col;
      for (int u = 0; u < nt; ++u) st.x[lane * kStagePad + u] = __ldg(xc + u * stride);
    }
    __syncwarp();
    for (int k = 0; k < n; ++k) acc = fmaf(st.v[k], st.x[k * kStagePad + lane], acc);
  }
  return acc;
}

// A = B theta (and Trels = expm(A dT) when trels != NULL), in one of two
// mappings chosen on the device from B's nonzeros (rowptr[nC * P], one
// broadcast load, so the host needs no copy and the call stays asynchronous):
//   * sparse B (at most 4 nonzeros per row on average; zero-boundary bases
//     have <= 4 in every row): one thread per (transformation, cell), each row
//     summed with a sequential fmaf chain;
//   * otherwise one warp per cell, lanes over transformations (32 at a time),
//     each row through row_times_lane_vector; lane u then computes
//     transformation t0 + u's exponential.
// Both sum every entry with the same sequential chain.  The grid covers nC
// warps; the sparse mapping strides over nC * n_theta.
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
  __shared__ WarpStage stage[kWarpsPerBlock];
  WarpStage &st = stage[threadIdx.x >> 5];
  const int64_t c = gtid >> 5;
  const int lane = threadIdx.x & 31;
  if (c >= nC) return;  // whole warps exit together
  for (int t0 = 0; t0 < n_theta; t0 += 32) {
    const int tn = min(32, n_theta - t0);
    const float *th = theta + (int64_t)t0 * d;
    float a[P];
#pragma unroll
    for (int r = 0; r < P; ++r)
      a[r] = row_times_lane_vector(colidx, vals, __ldg(rowptr + c * P + r),
                                   __ldg(rowptr + c * P + r + 1), th, d, tn, st);
    if (lane < tn) {
      const int64_t base = ((int64_t)(t0 + lane) * nC + c) * P;
#pragma unroll
      for (int r = 0; r < P; ++r) As[base + r] = a[r];
      if (trels != nullptr) {
        float e[P];
        expm_cell<ND>(a, dT, e);
#pragma unroll
        for (int r = 0; r < P; ++r) trels[base + r] = e[r];
      }
    }
  }
}

// The same products with the vectors given transposed, xt[col * nt + t]
// (theta^T [d, n_theta] or moments^T [D, n_theta]): a nonzero's entries of
// all vectors are then one contiguous row, so lanes over the vectors read it
// as one coalesced load instead of n_theta scattered ones.  This is what
// makes general (dense) bases cheap: their rows and columns spread over the
// whole domain, so the untransposed gathers hit a different sector for every
// vector.  Sequential fmaf chain per row (the oracle's order).
// xl points at this lane's vector in column 0 (xt + t); nt is the row length.
__device__ __forceinline__ float row_times_lane_vector_t(const int32_t *__restrict__ colidx,
                                                         const float *__restrict__ vals, int k0,
                                                         int k1, const float *__restrict__ xl,
                                                         int nt) {
  float acc = 0.0f;
  int k = k0;
  // eight nonzeros' loads in flight ahead of the (sequential) chain: the
  // chain's length is what bounds these kernels, through load latency
  for (; k + 8 <= k1; k += 8) {
    int c[8];
    float v[8], x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) c[u] = __ldg(colidx + k + u);
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = __ldg(vals + k + u);
#pragma unroll
    for (int u = 0; u < 8; ++u) x[u] = __ldg(xl + (int64_t)c[u] * nt);
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = fmaf(v[u], x[u], acc);
  }
  for (; k < k1; ++k) acc = fmaf(__ldg(vals + k), __ldg(xl + (int64_t)__ldg(colidx + k) * nt), acc);
  return acc;
}

// k_build_A with theta given transposed (theta_t [d, n_theta]): one block per
// cell, one warp per row of the cell (so the longest dependent chain is one
// row, not the cell's ppc rows in turn), lanes over the transformations, 32
// at a time (in the last group, lanes past n_theta repeat the last
// transformation, in bounds, and store nothing).  Warp 0 then takes the
// cell's entries from shared memory and computes the exponentials.
template <int ND>
__global__ void __launch_bounds__(32 * Dim<ND>::kPpc) k_build_A_tt(
    int64_t nC, int n_theta, const int32_t *__restrict__ rowptr,
    const int32_t *__restrict__ colidx, const float *__restrict__ vals,
    const float *__restrict__ theta_t, float dT, float *__restrict__ As,
    float *__restrict__ trels) {
  constexpr int P = Dim<ND>::kPpc;
  __shared__ float s_a[P][32];
  const int64_t c = blockIdx.x;
  const int r = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = __ldg(rowptr + c * P + r), k1 = __ldg(rowptr + c * P + r + 1);
  for (int t0 = 0; t0 < n_theta; t0 += 32) {
    const int t = min(t0 + lane, n_theta - 1);
    s_a[r][lane] = row_times_lane_vector_t(colidx, vals, k0, k1, theta_t + t, n_theta);
    __syncthreads();
    if (r == 0 && t0 + lane < n_theta) {
      float a[P];
#pragma unroll
      for (int q = 0; q < P; ++q) a[q] = s_a[q][lane];
      const int64_t base = ((int64_t)t * nC + c) * P;
#pragma unroll
      for (int q = 0; q < P; ++q) As[base + q] = a[q];
      if (trels != nullptr) {
        float e[P];
        expm_cell<ND>(a, dT, e);
#pragma unroll
        for (int q = 0; q < P; ++q) trels[base + q] = e[q];
      }
    }
    __syncthreads();
  }
}

// dtheta[t, j] = sum over row j of B^T (basis column j) of vals * moments[t,
// col].  One block per basis column, lanes over the transformations.  Columns
// have 16 to 80 nonzeros for zero-boundary bases and up to ~1,700 for general
// ones, so a column is cut into chunks of kProjChunk nonzeros that the
// block's warps sum concurrently (an fmaf chain each); warp 0 then adds the
// chunk sums left to right -- the order the CPU oracle restates.  Chunk sums
// pass through shared memory kProjGroup chunks at a time.  TT: moments given
// transposed ([D, n_theta], one coalesced load per nonzero; for general
// bases, whose columns spread over the whole domain); otherwise [n_theta, D],
// gathered through row_times_lane_vector's staging.
constexpr int kProjWarps = 8;
constexpr int kProjChunk = 32;  // = kStage
constexpr int kProjGroup = 64;

template <bool TT>
__global__ void __launch_bounds__(32 * kProjWarps) k_project(int64_t d, int64_t D, int n_theta,
                                                             const int32_t *__restrict__ rowptr,
                                                             const int32_t *__restrict__ colidx,
                                                             const float *__restrict__ vals,
                                                             const float *__restrict__ m,
                                                             float *__restrict__ dtheta) {
  __shared__ float s_part[kProjGroup][32];
  const int64_t j = blockIdx.x;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = __ldg(rowptr + j), k1 = __ldg(rowptr + j + 1);
  const int nch = (k1 - k0 + kProjChunk - 1) / kProjChunk;
  for (int t0 = 0; t0 < n_theta; t0 += 32) {
    const int tn = min(32, n_theta - t0);
    const int t = min(t0 + lane, n_theta - 1);
    float total = 0.0f;  // warp 0: the column's running sum for transformation t
    for (int g0 = 0; g0 < nch; g0 += kProjGroup) {
      const int gn = min(kProjGroup, nch - g0);
      for (int i = w; i < gn; i += kProjWarps) {
        const int kc = k0 + (g0 + i) * kProjChunk, ke = min(kc + kProjChunk, k1);
        float sum;
        if constexpr (TT) {
          sum = row_times_lane_vector_t(colidx, vals, kc, ke, m + t, n_theta);
        } else {
          __shared__ WarpStage stage[kProjWarps];
          sum = row_times_lane_vector(colidx, vals, kc, ke, m + (int64_t)t0 * D, D, tn, stage[w]);
        }
        s_part[i][lane] = sum;
      }
      __syncthreads();
      if (w == 0) {
        for (int i = 0; i < gn; ++i) {
          const float part = s_part[i][lane];
          total = g0 + i == 0 ? part : total + part;
        }
      }
      __syncthreads();
    }
    if (w == 0 && lane < tn) dtheta[(int64_t)(t0 + lane) * d + j] = total;
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

cudaError_t launch_build_A_tt(int ndim, int64_t nC, int n_theta, const int32_t *rowptr,
                              const int32_t *colidx, const float *vals, const float *theta_t,
                              float dT, float *As, float *trels, cudaStream_t s) {
  if (nC * n_theta == 0) return cudaSuccess;
  if (nC > 0x7FFFFFFF) return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)nC;  // one block per cell, one warp per row
  switch (ndim) {
    case 1:
      k_build_A_tt<1><<<grid, 32 * Dim<1>::kPpc, 0, s>>>(nC, n_theta, rowptr, colidx, vals,
                                                         theta_t, dT, As, trels);
      break;
    case 2:
      k_build_A_tt<2><<<grid, 32 * Dim<2>::kPpc, 0, s>>>(nC, n_theta, rowptr, colidx, vals,
                                                         theta_t, dT, As, trels);
      break;
    default:
      k_build_A_tt<3><<<grid, 32 * Dim<3>::kPpc, 0, s>>>(nC, n_theta, rowptr, colidx, vals,
                                                         theta_t, dT, As, trels);
      break;
  }
  return cudaGetLastError();
}

cudaError_t launch_project_tt(int64_t d, int n_theta, const int32_t *rowptr,
                              const int32_t *colidx, const float *vals, const float *moments_t,
                              float *dtheta, cudaStream_t s) {
  if (d * n_theta == 0) return cudaSuccess;
  if (d > 0x7FFFFFFF) return cudaErrorInvalidValue;
  k_project<true><<<(unsigned)d, 32 * kProjWarps, 0, s>>>(d, 0, n_theta, rowptr, colidx, vals,
                                                          moments_t, dtheta);
  return cudaGetLastError();
}

cudaError_t launch_project(int64_t d, int64_t D, int n_theta, const int32_t *rowptr,
                           const int32_t *colidx, const float *vals, const float *moments,
                           float *dtheta, cudaStream_t s) {
  if (d * n_theta == 0) return cudaSuccess;
  if (d > 0x7FFFFFFF) return cudaErrorInvalidValue;
  k_project<false><<<(unsigned)d, 32 * kProjWarps, 0, s>>>(d, D, n_theta, rowptr, colidx, vals,
                                                           moments, dtheta);
  return cudaGetLastError();
}

}  // namespace cpab
