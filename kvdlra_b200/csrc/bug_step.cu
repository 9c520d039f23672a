// Batched augmented rank-adaptive BUG step and the coordinate carry (sm_100a).
//
// Restates src/kvdlra/integrators/streaming_torch.py:82-189 for a batch of
// independent problems (one CTA per problem x stream):
//   a = U^T X ; R = X - U a ; a2 = U^T R ; R -= U a2 ; a += a2   (fp32 FFMA)
//   one-sided Jacobi on R (n x b): R V = [s_j q_j]  -> singular values s,
//     orthonormal left vectors q_j, right vectors V; admit s > 100 eps |X|_F,
//     at most n - r of them
//   one-sided Jacobi on B^T, B = [[diag(sigma), a], [0, diag(s_m) V_m^T]]
//     ((r+m) x (r+b)):  B^T W = [sigma'_c w_c]  -> W = left singular vectors
//     of B (u_loc), sigma' its singular values
//   U_new = [U | Q] W[:, top keep], rot = W[:r, top keep]^T, coords = U_new^T X.
// One-sided (Hestenes) Jacobi never forms a Gram matrix, so it keeps the
// relative accuracy of a direct SVD; all rotations of a round touch disjoint
// columns, so a round costs one barrier.
#include <stdio.h>

#include <cfloat>

#include "kernels.cuh"

namespace kvd {

struct StepWs {
  float* a;      // [ld][b]   coordinates of the block in the old basis
  float* R;      // [b][n]    residual, then sigma-scaled left vectors
  float* Q;      // [b][n]    admitted orthonormal residual directions
  float* VH;     // [b][b]    right singular vectors of R (column-major)
  float* BT;     // [N][N+b]  B^T (column-major, ld = ld + b)   (global fallback)
  float* W;      // [N][N]    rotations of B^T (column-major)    (global fallback)
  double* nrm;   // [N]
  int* ord;      // [N]
  int* ordh;     // [b]
  double* sv;    // [b]
  float* WU;     // [N][ld]   top left singular vectors of B (row-major)
};

__host__ __device__ inline long align16(long x) { return (x + 15) & ~15L; }

__host__ __device__ inline long step_ws_bytes(int n, int b, int ld) {
  const long N = ld + b, LB = ld + b;
  long o = 0;
  o += align16(4L * ld * b);
  o += align16(4L * b * n) * 2;
  o += align16(4L * b * b);
  o += align16(4L * N * LB);
  o += align16(4L * N * N);
  o += align16(8L * N);
  o += align16(4L * N);
  o += align16(4L * b);
  o += align16(8L * b);
  o += align16(4L * N * ld);
  return o;
}

__device__ StepWs carve(char* base, int n, int b, int ld) {
  const long N = ld + b, LB = ld + b;
  StepWs w;
  long o = 0;
  auto take = [&](long bytes) { char* p = base + o; o += align16(bytes); return p; };
  w.a = (float*)take(4L * ld * b);
  w.R = (float*)take(4L * b * n);
  w.Q = (float*)take(4L * b * n);
  w.VH = (float*)take(4L * b * b);
  w.BT = (float*)take(4L * N * LB);
  w.W = (float*)take(4L * N * N);
  w.nrm = (double*)take(8L * N);
  w.ord = (int*)take(4L * N);
  w.ordh = (int*)take(4L * b);
  w.sv = (double*)take(8L * b);
  w.WU = (float*)take(4L * N * ld);
  return w;
}

constexpr int kGemmSmemFloats = 2 * 16 * 64;
constexpr int kStepThreads = 512;
constexpr int kStepMiscBytes = 4096;

// One-sided (Hestenes) Jacobi: orthogonalise the `cols` columns of X (column
// c at X + c*ldx, `len` rows) by plane rotations, accumulated into V
// (cols x cols, column-major, ldv; initialised to I here).  Round-robin
// ordering; each column pair is handled by a group of G lanes (all pairs of a
// round run concurrently), one barrier per round.  The rotation zeroes the
// pair's inner product (Golub & Van Loan sec. 8.6.3).  ACC is the type the
// 2x2 Gram of a pair is accumulated in.  Returns the sweeps taken
// (max_sweeps + 1 when not converged).
template <int G, typename ACC>
static __device__ int cta_hestenes(float* X, int len, int cols, int ldx, float* V, int ldv,
                                   float tol, int max_sweeps) {
  __shared__ int s_rot;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int groups = nthr / G, gid = tid / G, gl = tid % G;
  for (int e = tid; e < cols * cols; e += nthr) {
    const int c = e / cols, k = e % cols;
    V[c * ldv + k] = (c == k) ? 1.f : 0.f;
  }
  __syncthreads();
  if (cols <= 1) return 0;
  const int np = cols + (cols & 1);
  const int half = np / 2;
  int sweep = 0;
  for (; sweep < max_sweeps; ++sweep) {
    if (tid == 0) s_rot = 0;
    __syncthreads();
    for (int k = 0; k < np - 1; ++k) {
      for (int base = 0; base < half; base += groups) {
        const int i = base + gid;
        int p = 0, q = -1;
        if (i < half) {
          int a, b;
          rr_pair(i, k, np, &a, &b);
          p = a < b ? a : b;
          q = a < b ? b : a;
          if (q >= cols) q = -1;
        }
        const bool active = q >= 0;
        float* xp = X + (long)p * ldx;
        float* xq = X + (long)(active ? q : p) * ldx;
        ACC al = 0, be = 0, ga = 0;
        if (active) {
          for (int e = gl; e < len; e += G) {
            const ACC u = xp[e], v = xq[e];
            al += u * u;
            be += v * v;
            ga += u * v;
          }
        }
#pragma unroll
        for (int o = G / 2; o > 0; o >>= 1) {
          al += __shfl_xor_sync(0xffffffffu, al, o);
          be += __shfl_xor_sync(0xffffffffu, be, o);
          ga += __shfl_xor_sync(0xffffffffu, ga, o);
        }
        if (!active || ga == (ACC)0 || fabsf((float)ga) <= tol * sqrtf((float)al * (float)be))
          continue;
        // rotation angle in fp32: its rounding only perturbs the convergence
        // rate, the applied rotation stays orthogonal (c^2 + s^2 = 1)
        const float zeta = ((float)be - (float)al) / (2.f * (float)ga);
        const float az = fabsf(zeta);
        const float t = (az > 1e18f) ? 0.5f / zeta
                                     : copysignf(1.f, zeta) / (az + sqrtf(fmaf(zeta, zeta, 1.f)));
        const double cd = 1.0 / sqrt(1.0 + (double)t * (double)t);
        const float c = (float)cd, s = (float)(cd * (double)t);
        for (int e = gl; e < len; e += G) {
          const float u = xp[e], v = xq[e];
          xp[e] = c * u - s * v;
          xq[e] = s * u + c * v;
        }
        float* vp = V + (long)p * ldv;
        float* vq = V + (long)q * ldv;
        for (int e = gl; e < cols; e += G) {
          const float u = vp[e], v = vq[e];
          vp[e] = c * u - s * v;
          vq[e] = s * u + c * v;
        }
        if (gl == 0) s_rot = 1;
      }
      __syncthreads();
    }
    const int any = s_rot;
    __syncthreads();
    if (!any) break;
  }
  return sweep;
}

// out[k][j] = sum_i U[i][k] X[j][i]   (k < M, j < b; U row-major ld, X [b][n])
static __device__ void cta_proj_t(int M, int b, int n, const float* U, int ld, const float* X,
                                  float* out, int ldo) {
  for (int e = threadIdx.x; e < M * b; e += blockDim.x) {
    const int k = e % M, j = e / M;
    const float* x = X + (long)j * n;
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
    int i = 0;
    for (; i + 3 < n; i += 4) {
      acc0 = fmaf(U[(long)i * ld + k], x[i], acc0);
      acc1 = fmaf(U[(long)(i + 1) * ld + k], x[i + 1], acc1);
      acc2 = fmaf(U[(long)(i + 2) * ld + k], x[i + 2], acc2);
      acc3 = fmaf(U[(long)(i + 3) * ld + k], x[i + 3], acc3);
    }
    for (; i < n; ++i) acc0 = fmaf(U[(long)i * ld + k], x[i], acc0);
    out[k * ldo + j] = (acc0 + acc1) + (acc2 + acc3);
  }
  __syncthreads();
}

// Y[j][i] (=|+=) alpha * sum_k A[i][k] C[k][j]  for i < n, j < b; A row-major
// (lda), C row-major (ldc, in shared memory), Y [b][n].  One thread per row i.
template <bool ACCUM>
static __device__ void cta_rows_times(int n, int b, int K, const float* A, int lda, const float* C,
                                      int ldc, float* Y, float alpha) {
  constexpr int JB = 16;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float* ar = A + (long)i * lda;
    for (int j0 = 0; j0 < b; j0 += JB) {
      float acc[JB];
#pragma unroll
      for (int jj = 0; jj < JB; ++jj) acc[jj] = 0.f;
      const int jn = min(JB, b - j0);
      for (int k = 0; k < K; ++k) {
        const float av = ar[k];
        const float* cr = C + (long)k * ldc + j0;
#pragma unroll
        for (int jj = 0; jj < JB; ++jj)
          if (jj < jn) acc[jj] = fmaf(av, cr[jj], acc[jj]);
      }
#pragma unroll
      for (int jj = 0; jj < JB; ++jj) {
        if (jj >= jn) break;
        float* y = Y + (long)(j0 + jj) * n + i;
        *y = ACCUM ? fmaf(alpha, acc[jj], *y) : alpha * acc[jj];
      }
    }
  }
  __syncthreads();
}

// Column norms (fp64) of X[:, 0..cols) into nrm, then order = descending.
static __device__ void cta_colnorm_order(const float* X, int len, int cols, int ldx, double* nrm,
                                         int* order) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, nw = blockDim.x / 32;
  for (int c = warp; c < cols; c += nw) {
    const float* x = X + (long)c * ldx;
    double acc = 0.0;
    for (int e = lane; e < len; e += 32) acc += (double)x[e] * x[e];
    acc = warp_sum(acc);
    if (lane == 0) nrm[c] = sqrt(acc);
  }
  __syncthreads();
  cta_argsort_desc(nrm, cols, order);
}

// Orthonormalise the rows of Q[0..m) (length n) in order by classical
// Gram-Schmidt applied twice; a row that collapses (numerically dependent or
// null) is replaced by the first canonical vector e_i that survives the same
// orthogonalisation.  Used only when some admitted direction is (near) null.
static __device__ void cta_cgs2_rows(float* Q, int m, int n, double* dots /*>= m*/,
                                     double* red /*>=32*/) {
  __shared__ double s_norm, s_norm0;
  __shared__ int s_next_e;
  const int tid = threadIdx.x, nthr = blockDim.x, lane = tid % 32, warp = tid / 32,
            nw = nthr / 32;
  if (tid == 0) s_next_e = 0;
  __syncthreads();
  for (int j = 0; j < m; ++j) {
    float* qj = Q + (long)j * n;
    double acc = 0.0;
    for (int i = tid; i < n; i += nthr) acc += (double)qj[i] * qj[i];
    acc = warp_sum(acc);
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (tid == 0) { double t = 0; for (int w = 0; w < nw; ++w) t += red[w]; s_norm0 = sqrt(t); }
    __syncthreads();
    for (int attempt = 0; attempt < n + 1; ++attempt) {
      for (int pass = 0; pass < 2; ++pass) {
        for (int l = warp; l < j; l += nw) {
          const float* ql = Q + (long)l * n;
          double d = 0.0;
          for (int i = lane; i < n; i += 32) d += (double)ql[i] * qj[i];
          d = warp_sum(d);
          if (lane == 0) dots[l] = d;
        }
        __syncthreads();
        for (int i = tid; i < n; i += nthr) {
          double v = qj[i];
          for (int l = 0; l < j; ++l) v -= dots[l] * (double)Q[(long)l * n + i];
          qj[i] = (float)v;
        }
        __syncthreads();
      }
      acc = 0.0;
      for (int i = tid; i < n; i += nthr) acc += (double)qj[i] * qj[i];
      acc = warp_sum(acc);
      if (lane == 0) red[warp] = acc;
      __syncthreads();
      if (tid == 0) { double t = 0; for (int w = 0; w < nw; ++w) t += red[w]; s_norm = sqrt(t); }
      __syncthreads();
      const double nrm = s_norm, nrm0 = s_norm0;
      if (nrm > 1e-3 * nrm0 && nrm > 1e-30) break;
      const int e = s_next_e;
      __syncthreads();
      if (e >= n) break;
      for (int i = tid; i < n; i += nthr) qj[i] = (i == e) ? 1.f : 0.f;
      if (tid == 0) { s_next_e = e + 1; s_norm0 = 1.0; }
      __syncthreads();
    }
    const float inv = (float)(1.0 / s_norm);
    for (int i = tid; i < n; i += nthr) qj[i] *= inv;
    __syncthreads();
  }
}

// Two-sided cyclic Jacobi on a symmetric N x N fp64 matrix A (leading
// dimension lda, odd so column accesses are bank-conflict free), eigenvectors
// accumulated in V (N x N fp64, ldv).  N'/2 disjoint rotations per round
// (circle ordering), rows then columns.  Rotation: Golub & Van Loan
// Alg. 8.4.2 (sym.schur2), angle in fp32 (only the convergence rate depends
// on it), applied in fp64.  `cs` is shared scratch of 2*(N/2+1) doubles and
// 2*(N/2+1) ints (8-byte aligned).  Entries below 1e-17 of the largest diagonal are rounding
// noise and are left alone, so rank-deficient PSD matrices converge.
static __device__ int cta_jacobi_sym(double* A, int N, int lda, double* V, int ldv, float* cs,
                                     int max_sweeps) {
  __shared__ int s_rot;
  __shared__ double s_scale;
  const int tid = threadIdx.x, nthr = blockDim.x;
  for (int e = tid; e < N * N; e += nthr) {
    const int i = e / N, j = e % N;
    V[i * ldv + j] = (i == j) ? 1.0 : 0.0;
  }
  if (tid == 0) {
    double mx = 0.0;
    for (int i = 0; i < N; ++i) mx = fmax(mx, fabs(A[i * lda + i]));
    s_scale = mx;
  }
  __syncthreads();
  if (N <= 1) return 0;
  const double floor_rot = 1e-17 * s_scale, floor_flag = 1e-14 * s_scale;
  const int np = N + (N & 1), half = np / 2;
  double* pc = reinterpret_cast<double*>(cs);
  double* ps = pc + half;
  int* pp = reinterpret_cast<int*>(ps + half);
  int* pq = pp + half;
  int sweep = 0;
  for (; sweep < max_sweeps; ++sweep) {
    if (tid == 0) s_rot = 0;
    __syncthreads();
    for (int k = 0; k < np - 1; ++k) {
      for (int i = tid; i < half; i += nthr) {
        int a, b;
        rr_pair(i, k, np, &a, &b);
        int p = a < b ? a : b, q = a < b ? b : a;
        double pcd = 1.0, psd = 0.0;
        if (q < N) {
          const double apq = A[p * lda + q], app = A[p * lda + p], aqq = A[q * lda + q];
          const double thr = fmax(1e-15 * sqrt(fabs(app * aqq)), floor_rot);
          if (apq != 0.0 && fabs(apq) > thr) {
            const float tau = (float)((aqq - app) / (2.0 * apq));
            const float at = fabsf(tau);
            const float t = (at > 1e18f) ? 0.5f / tau
                                         : copysignf(1.f, tau) / (at + sqrtf(fmaf(tau, tau, 1.f)));
            // the angle is approximate (fp32 t) but (c, s) is an exact fp64
            // rotation, so applying it never changes norms
            const double cd = 1.0 / sqrt(1.0 + (double)t * (double)t);
            pcd = cd;
            psd = cd * (double)t;
            if (fabs(apq) > fmax(4e-15 * sqrt(fabs(app * aqq)), floor_flag)) s_rot = 1;
          }
        } else {
          q = -1;
        }
        pc[i] = pcd; ps[i] = psd; pp[i] = p; pq[i] = q;
      }
      __syncthreads();
      for (int e = tid; e < half * N; e += nthr) {   // rows: A <- J^T A
        const int i = e / N, j = e % N;
        const double s = ps[i];
        if (s == 0.0) continue;
        const int p = pp[i], q = pq[i];
        const double c = pc[i];
        const double x = A[p * lda + j], y = A[q * lda + j];
        A[p * lda + j] = c * x - s * y;
        A[q * lda + j] = s * x + c * y;
      }
      __syncthreads();
      for (int e = tid; e < half * N; e += nthr) {   // columns: A <- A J, V <- V J
        const int i = e / N, j = e % N;
        const double s = ps[i];
        if (s == 0.0) continue;
        const int p = pp[i], q = pq[i];
        const double c = pc[i];
        const double x = A[j * lda + p], y = A[j * lda + q];
        A[j * lda + p] = c * x - s * y;
        A[j * lda + q] = s * x + c * y;
        const double vx = V[j * ldv + p], vy = V[j * ldv + q];
        V[j * ldv + p] = c * vx - s * vy;
        V[j * ldv + q] = s * vx + c * vy;
      }
      __syncthreads();
    }
    const int any = s_rot;
    __syncthreads();
    if (!any) break;
  }
  return sweep;
}

// H = X^T X in fp64 for the `cols` columns of X (column c at X + c*ldx, len
// rows); one warp per (c1 <= c2) pair.
static __device__ void cta_gram_cols(const float* X, int len, int cols, int ldx, double* H, int ldh) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  const int pairs = cols * (cols + 1) / 2;
  for (int e = warp; e < pairs; e += nw) {
    int c1 = 0, rem = e;
    while (rem >= cols - c1) { rem -= cols - c1; ++c1; }
    const int c2 = c1 + rem;
    const float* x1 = X + (long)c1 * ldx;
    const float* x2 = X + (long)c2 * ldx;
    double acc = 0.0;
    for (int i = lane; i < len; i += 32) acc += (double)x1[i] * (double)x2[i];
    acc = warp_sum(acc);
    if (lane == 0) { H[c1 * ldh + c2] = acc; H[c2 * ldh + c1] = acc; }
  }
  __syncthreads();
}

// Make the rows of Q (m x n) orthonormal by one Cholesky-QR pass in fp64:
// G = Q Q^T = L L^T, Q <- L^{-1} Q.  `Gs` is shared scratch of m*(m+1)
// doubles.  Returns false (Q untouched) when a pivot is not safely positive,
// i.e. the rows are (numerically) dependent.
static __device__ bool cta_cholqr_rows(float* Q, int m, int n, double* Gs) {
  __shared__ int s_ok;
  const int ldg = m + 1;
  cta_gram_cols(Q, n, m, n, Gs, ldg);  // rows of Q are the "columns" here
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int j = 0; j < m && ok; ++j) {  // in-place Cholesky, lower triangle
      double d = Gs[j * ldg + j];
      for (int k = 0; k < j; ++k) d -= Gs[j * ldg + k] * Gs[j * ldg + k];
      if (!(d > 0.25)) { ok = 0; break; }  // rows are near-unit: pivots ~1
      d = sqrt(d);
      Gs[j * ldg + j] = d;
      for (int i = j + 1; i < m; ++i) {
        double v = Gs[i * ldg + j];
        for (int k = 0; k < j; ++k) v -= Gs[i * ldg + k] * Gs[j * ldg + k];
        Gs[i * ldg + j] = v / d;
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return false;
  // forward substitution per column i of Q, in place: Q[:, i] <- L^{-1} Q[:, i]
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    for (int j = 0; j < m; ++j) {
      double v = Q[(long)j * n + i];
      for (int k = 0; k < j; ++k) v -= Gs[j * ldg + k] * (double)Q[(long)k * n + i];
      Q[(long)j * n + i] = (float)(v / Gs[j * ldg + j]);
    }
  }
  __syncthreads();
  return true;
}

__global__ void __launch_bounds__(kStepThreads) bug_step_kernel(BugStepBatch batch, int smem_budget) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int p = blockIdx.x;
  const BugStepArgs& A = batch.s[blockIdx.y];
  const int n = A.n, b = A.b, cap = A.rank_cap, ld = A.ld;
  const float* U = A.u + p * A.u_sp;
  float* Uo = A.u_out + p * A.u_sp;
  float* sig = A.sigma + p * A.sig_sp;
  const float* X = A.x + p * A.x_sp;
  const int r = A.r[p];
  StepWs w = carve(A.ws + p * A.ws_sp, n, b, ld);
  float* gsm = reinterpret_cast<float*>(smem_raw);
  double* red = reinterpret_cast<double*>(smem_raw + 4 * kGemmSmemFloats);  // 64 doubles
  float* pool = reinterpret_cast<float*>(smem_raw + 4 * kGemmSmemFloats + kStepMiscBytes);
  const long pool_floats = (smem_budget - 4L * kGemmSmemFloats - kStepMiscBytes) / 4;
  __shared__ double s_xnorm2;
  __shared__ int s_m, s_keep, s_degenerate;
  const int tid = threadIdx.x, nthr = blockDim.x, lane = tid % 32, warp = tid / 32;

  // ||X||_F^2 (fp64 accumulation of fp32 squares)
  {
    double acc = 0.0;
    for (long e = tid; e < (long)b * n; e += nthr) acc += (double)X[e] * X[e];
    acc = warp_sum(acc);
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (tid == 0) { double t = 0; for (int i = 0; i < nthr / 32; ++i) t += red[i]; s_xnorm2 = t; }
    __syncthreads();
  }
  // ----- residual R = (I - U U^T)^2 X (the reference's re-orthogonalised residual)
  const bool r_in_smem = (long)b * n + (long)b * b <= pool_floats;
  float* Rm = r_in_smem ? pool : w.R;
  float* Vh = r_in_smem ? pool + (long)b * n : w.VH;
  // U staged in shared memory (at the end of the pool) when it fits beside the
  // residual phase; it is read by four projections and the basis update
  const long u_floats = (long)n * r;
  const long p1_floats = (long)b * n + (long)b * b + 2L * r * b;
  const bool u_smem = r > 0 && r_in_smem && p1_floats + u_floats <= pool_floats;
  const float* Us = U;
  int uld = ld;
  if (u_smem) {
    float* dst = pool + (pool_floats - u_floats);
    for (long e = tid; e < u_floats; e += nthr) {
      const long i = e / r, k = e % r;
      dst[e] = U[i * ld + k];
    }
    Us = dst;
    uld = r;
  }
  for (long e = tid; e < (long)b * n; e += nthr) Rm[e] = X[e];
  __syncthreads();
  if (r > 0) {
    // a and a2 live in shared memory when they fit beside R (small in steady state)
    const bool a_smem = r_in_smem && (long)b * n + (long)b * b + 2L * r * b <= pool_floats;
    float* as = a_smem ? pool + (long)b * n + (long)b * b : w.a;
    float* a2 = a_smem ? as + (long)r * b : w.Q;
    __syncthreads();
    cta_proj_t(r, b, n, Us, uld, Rm, as, b);                      // a = U^T X
    cta_rows_times<true>(n, b, r, Us, uld, as, b, Rm, -1.f);      // R -= U a
    cta_proj_t(r, b, n, Us, uld, Rm, a2, b);                      // a2 = U^T R
    cta_rows_times<true>(n, b, r, Us, uld, a2, b, Rm, -1.f);      // R -= U a2
    for (int e = tid; e < r * b; e += nthr) w.a[e] = as[e] + a2[e];
    __syncthreads();
  }
  // ----- SVD of R.  Small blocks: fp64 Gram + two-sided Jacobi, then
  // Q = R V S^-1 made orthonormal by Cholesky-QR.  Large blocks: one-sided
  // Jacobi directly on R (columns come out orthogonal).
  float* cs = reinterpret_cast<float*>(smem_raw + 4 * kGemmSmemFloats + 512);
  const int ldh = b | 1;
  const long p1_end = (long)b * n + (long)b * b + 2L * r * b;
  const long h_off = (p1_end + 1) & ~1L;  // 8-byte aligned for fp64
  const bool gram_r = r_in_smem && h_off + 4L * b * ldh <= pool_floats;
  int sw = 0;
  if (gram_r) {
    double* Hm = reinterpret_cast<double*>(pool + h_off);
    double* Vd = Hm + (long)b * ldh;
    cta_gram_cols(Rm, n, b, n, Hm, ldh);
    sw = cta_jacobi_sym(Hm, b, ldh, Vd, ldh, cs, 40);
    for (int j = tid; j < b; j += nthr) w.sv[j] = sqrt(fmax(Hm[j * ldh + j], 0.0));
    for (int e = tid; e < b * b; e += nthr) {  // fp32 column-major copy of V
      const int c = e / b, row = e % b;
      Vh[e] = (float)Vd[row * ldh + c];
    }
    __syncthreads();
    cta_argsort_desc(w.sv, b, w.ordh);
  } else {
    sw = cta_hestenes<32, double>(Rm, n, b, n, Vh, b, 1.2e-7f * sqrtf((float)n) + 2.4e-7f, 30);
    cta_colnorm_order(Rm, n, b, n, w.sv, w.ordh);
  }
  if (sw > 30 && tid == 0) atomicOr(&A.status[kStatusNumeric], 1);
  if (tid == 0) {
    const float xnorm = (float)sqrt(s_xnorm2);
    const double tol = 100.0 * (double)FLT_EPSILON * (double)xnorm;
    int m;
    if (r == 0) {
      m = min(n, b);
    } else {
      m = 0;
      for (int j = 0; j < b; ++j)
        if ((double)(float)w.sv[w.ordh[j]] > tol) ++m;
      m = min(m, max(0, n - r));
    }
    s_m = m;
    // a kept direction far below the largest is numerically null: its column
    // is rounding noise and must be completed to an orthonormal direction
    const double s0 = w.sv[w.ordh[0]];
    int deg = 0;
    for (int j = 0; j < m; ++j)
      if (!(w.sv[w.ordh[j]] > 1e-6 * s0) || s0 == 0.0) deg = 1;
    s_degenerate = deg;
  }
  __syncthreads();
  const int m = s_m;
  if (gram_r) {
    // Q_j = R V[:, ord_j] / s_j
    for (long e = tid; e < (long)m * n; e += nthr) {
      const int j = (int)(e / n), i = (int)(e % n);
      const int oj = w.ordh[j];
      const double sj = w.sv[oj];
      const float* vc = Vh + (long)oj * b;
      float acc = 0.f;
      for (int l = 0; l < b; ++l) acc = fmaf(Rm[(long)l * n + i], vc[l], acc);
      w.Q[e] = sj > 0.0 ? (float)(acc / sj) : 0.f;
    }
    __syncthreads();
    bool ok = !s_degenerate && m > 0;
    if (ok) ok = cta_cholqr_rows(w.Q, m, n, reinterpret_cast<double*>(pool + h_off));
    if (!ok && m > 0) cta_cgs2_rows(w.Q, m, n, w.nrm, red);
  } else {
    for (long e = tid; e < (long)m * n; e += nthr) {
      const int j = (int)(e / n), i = (int)(e % n);
      const int oj = w.ordh[j];
      const double sj = w.sv[oj];
      w.Q[e] = sj > 0.0 ? (float)(Rm[(long)oj * n + i] / sj) : 0.f;
    }
    __syncthreads();
    if (s_degenerate) cta_cgs2_rows(w.Q, m, n, w.nrm, red);
  }
  // ----- the core B = [[diag(sigma), a], [0, diag(s_m) V_m^T]] ((r+m) x (r+b)):
  // its left singular vectors W and values.  N <= 112: fp64 Gram B B^T +
  // two-sided Jacobi; larger: one-sided Jacobi on B^T.
  const int N = r + m, LB = r + b;
  if (Vh != w.VH) {  // V must survive while the pool is reused
    for (int e = tid; e < b * b; e += nthr) w.VH[e] = Vh[e];
    __syncthreads();
    Vh = w.VH;
  }
  const int ldg = N | 1;
  const bool gram_b = N <= 112 && 4L * N * ldg <= pool_floats;
  float* Wm = nullptr;   // one-sided path: W column-major [c*N + k]
  double* Wd = nullptr;  // two-sided path: W row-major [k*ldg + c]
  if (gram_b) {
    double* Gm = reinterpret_cast<double*>(pool);
    Wd = Gm + (long)N * ldg;
    for (int e = tid; e < N * N; e += nthr) {
      const int i = e / N, j = e % N;
      if (j < i) continue;
      double g = 0.0;
      if (i < r && j < r) {
        for (int l = 0; l < b; ++l) g += (double)w.a[i * b + l] * (double)w.a[j * b + l];
        if (i == j) g += (double)sig[i] * (double)sig[i];
      } else if (i < r) {
        const int jj = j - r, oj = w.ordh[jj];
        double t = 0.0;
        for (int l = 0; l < b; ++l) t += (double)w.a[i * b + l] * (double)Vh[(long)oj * b + l];
        g = t * (double)(float)w.sv[oj];
      } else {
        const int oi = w.ordh[i - r], oj = w.ordh[j - r];
        double t = 0.0;
        for (int l = 0; l < b; ++l) t += (double)Vh[(long)oi * b + l] * (double)Vh[(long)oj * b + l];
        g = t * (double)(float)w.sv[oi] * (double)(float)w.sv[oj];
      }
      Gm[i * ldg + j] = g;
      Gm[j * ldg + i] = g;
    }
    __syncthreads();
    sw = cta_jacobi_sym(Gm, N, ldg, Wd, ldg, cs, 40);
    for (int c = tid; c < N; c += nthr) w.nrm[c] = sqrt(fmax(Gm[c * ldg + c], 0.0));
    __syncthreads();
    cta_argsort_desc(w.nrm, N, w.ord);
  } else {
    const long bt_need = (long)N * LB + (long)N * N;
    float* BT = bt_need <= pool_floats ? pool : w.BT;
    Wm = bt_need <= pool_floats ? pool + (long)N * LB : w.W;
    for (long e = tid; e < (long)N * LB; e += nthr) {
      const int c = (int)(e / LB), row = (int)(e % LB);
      float v = 0.f;
      if (c < r) {
        if (row < r) v = (row == c) ? sig[c] : 0.f;
        else v = w.a[c * b + (row - r)];
      } else if (row >= r) {
        const int j = c - r;
        v = (float)w.sv[w.ordh[j]] * Vh[(long)w.ordh[j] * b + (row - r)];
      }
      BT[e] = v;
    }
    __syncthreads();
    const float btol = 1.2e-7f * sqrtf((float)LB) + 2.4e-7f;
    if (LB <= 64) sw = cta_hestenes<8, float>(BT, LB, N, LB, Wm, N, btol, 30);
    else if (LB <= 256) sw = cta_hestenes<16, float>(BT, LB, N, LB, Wm, N, btol, 30);
    else sw = cta_hestenes<32, double>(BT, LB, N, LB, Wm, N, btol, 30);
    cta_colnorm_order(BT, LB, N, LB, w.nrm, w.ord);
  }
  if (sw > 30 && tid == 0) atomicOr(&A.status[kStatusNumeric], 2);
  if (tid == 0) {
    int keep = min(cap, N);
    if (A.has_theta && N > 0) {
      // smallest k with sqrt(sum_{j>=k} sigma_j^2) <= theta (fp32, as the reference)
      const float th2 = A.theta * A.theta;
      int first_ok = -1;
      float tail = 0.f;
      for (int k = N - 1; k >= 0; --k) {
        const float sk = (float)w.nrm[w.ord[k]];
        tail += sk * sk;
        if (tail <= th2) first_ok = k;
      }
      const int tr = (first_ok < 0) ? N : max(1, first_ok);
      keep = max(1, min(keep, tr));
    }
    s_keep = keep;
  }
  __syncthreads();
  const int keep = s_keep;
  // WU[k][c] = W[k][ord_c]
  auto wget = [&](int k, int c) -> float {
    return Wd ? (float)Wd[(long)k * ldg + c] : Wm[(long)c * N + k];
  };
  for (int e = tid; e < N * keep; e += nthr) {
    const int k = e / keep, c = e % keep;
    w.WU[k * ld + c] = wget(k, w.ord[c]);
  }
  for (int c = tid; c < keep; c += nthr) sig[c] = (float)w.nrm[w.ord[c]];
  float* rot = A.rot + p * A.rot_sp;
  for (int e = tid; e < keep * r; e += nthr) {
    const int c = e / r, k = e % r;
    rot[c * ld + k] = wget(k, w.ord[c]);
  }
  __syncthreads();
  // U_new = U W[:r] + Q^T W[r:]  (one thread per basis row)
  {
    constexpr int CB = 16;
    for (int i = tid; i < n; i += nthr) {
      const float* ur = U + (long)i * ld;
      for (int c0 = 0; c0 < keep; c0 += CB) {
        float acc[CB];
#pragma unroll
        for (int cc = 0; cc < CB; ++cc) acc[cc] = 0.f;
        const int cn = min(CB, keep - c0);
        for (int k = 0; k < r; ++k) {
          const float uv = ur[k];
          const float* wr = w.WU + (long)k * ld + c0;
#pragma unroll
          for (int cc = 0; cc < CB; ++cc)
            if (cc < cn) acc[cc] = fmaf(uv, wr[cc], acc[cc]);
        }
        for (int j = 0; j < m; ++j) {
          const float qv = w.Q[(long)j * n + i];
          const float* wr = w.WU + (long)(r + j) * ld + c0;
#pragma unroll
          for (int cc = 0; cc < CB; ++cc)
            if (cc < cn) acc[cc] = fmaf(qv, wr[cc], acc[cc]);
        }
        float* uo = Uo + (long)i * ld + c0;
#pragma unroll
        for (int cc = 0; cc < CB; ++cc)
          if (c0 + cc < keep) uo[cc] = acc[cc];
      }
    }
    __syncthreads();
  }
  // coords[j][c] = sum_i U_new[i][c] X[j][i]
  float* co = A.coords + p * A.coords_sp;
  {
    float* ct = (r_in_smem && (long)keep * b <= pool_floats) ? pool : w.a;
    cta_proj_t(keep, b, n, Uo, ld, X, ct, b);
    for (int e = tid; e < keep * b; e += nthr) {
      const int c = e / b, j = e % b;
      co[(long)j * A.coords_ld + c] = ct[e];
    }
  }
  if (tid == 0) {
    int* d = A.dims + 4 * p;
    d[0] = r; d[1] = keep; d[2] = m; d[3] = sw;
    A.r[p] = keep;
  }
}

// C[p][t][0..keep) = rot[p] (keep x r_old) C[p][t][0..r_old), t < W.  rot is
// staged transposed in shared memory; one warp per token row.

__global__ void __launch_bounds__(256) carry_kernel(CarryBatch batch, int tokens_per_cta) {
  extern __shared__ __align__(16) float csm[];
  const CarryArgs& A = batch.s[blockIdx.z];
  const int p = blockIdx.y;
  const int r_old = A.dims[4 * p], keep = A.dims[4 * p + 1];
  const int ld = A.ld;
  if (r_old == 0) return;
  float* rotT = csm;                       // [r_old][keep]
  float* rows = csm + r_old * keep;        // [8 warps][r_old]
  const float* rot = A.rot + p * A.rot_sp;
  for (int e = threadIdx.x; e < r_old * keep; e += blockDim.x) {
    const int k = e / keep, c = e % keep;
    rotT[e] = rot[c * ld + k];
  }
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* row = rows + warp * r_old;
  const int t0 = blockIdx.x * tokens_per_cta;
  const int t1 = min(batch.W, t0 + tokens_per_cta);
  for (int t = t0 + warp; t < t1; t += 8) {
    float* ct = A.c + p * A.c_sp + (long)t * ld;
    for (int k = lane; k < r_old; k += 32) row[k] = ct[k];
    __syncwarp();
    for (int c = lane; c < keep; c += 32) {
      float acc = 0.f;
      for (int k = 0; k < r_old; ++k) acc = fmaf(rotT[k * keep + c], row[k], acc);
      ct[c] = acc;
    }
    __syncwarp();
  }
}

// Low-rank surprise of fp32 token-major columns (bug_cache.py:906-921).
__global__ void __launch_bounds__(256) surprise_f32_kernel(int n, int m, int ld, const float* u,
                                                            long u_sp, const int* rr,
                                                            const float* x, long x_sp,
                                                            float* out, long out_sp) {
  const int p = blockIdx.y;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int j = blockIdx.x * 8 + warp;
  if (j >= m) return;
  const int r = rr[p];
  const float* xj = x + p * x_sp + (long)j * n;
  const float* U = u + p * u_sp;
  float kk = 0.f;
  for (int i = lane; i < n; i += 32) kk = fmaf(xj[i], xj[i], kk);
  kk = warp_sum(kk);
  const float kn = sqrtf(kk);
  float res;
  if (r == 0) {
    res = 1.f;
  } else {
    float cc = 0.f;
    for (int k = lane; k < r; k += 32) {
      float c = 0.f;
      for (int i = 0; i < n; ++i) c = fmaf(U[(long)i * ld + k], xj[i], c);
      cc = fmaf(c, c, cc);
    }
    cc = warp_sum(cc);
    const float cn = sqrtf(cc);
    res = sqrtf(fmaxf(kn * kn - cn * cn, 0.f)) / fmaxf(kn, 1e-12f);
  }
  if (lane == 0) out[p * out_sp + j] = res;
}

// Stable descending top-k (bug_cache.py:810-812): one CTA per problem.
__global__ void __launch_bounds__(1024) select_topk_kernel(int m, int k, const float* scores,
                                                           int* keep_idx, int* demote_idx) {
  extern __shared__ float ssc[];
  __shared__ int scan_scratch[32];
  const int p = blockIdx.x;
  const float* s = scores + (long)p * m;
  for (int i = threadIdx.x; i < m; i += blockDim.x) ssc[i] = s[i];
  __syncthreads();
  int keep_base = 0, dem_base = 0;
  for (int i0 = 0; i0 < m; i0 += blockDim.x) {
    const int i = i0 + threadIdx.x;
    int kept = 0;
    if (i < m) {
      const float v = ssc[i];
      int rank = 0;
      for (int j = 0; j < m; ++j) {
        const float w = ssc[j];
        rank += (w > v) || (w == v && j < i);
      }
      kept = rank < k;
    }
    int tot;
    const int pre = cta_exclusive_scan(kept, scan_scratch, &tot);
    if (i < m) {
      if (kept) keep_idx[(long)p * k + keep_base + pre] = i;
      else demote_idx[(long)p * (m - k) + dem_base + (i - i0 - pre)] = i;
    }
    const int cnt = min(blockDim.x, m - i0);
    keep_base += tot;
    dem_base += cnt - tot;
    __syncthreads();
  }
}

// recon[p][t][i] = sum_c U[i][c] (sum_j U[j][c] x[t][j]) for c < r[p].
__global__ void __launch_bounds__(512) project_kernel(int n, int t, int ld, const float* u,
                                                      long u_sp, const int* rr, const float* x,
                                                      long x_sp, float* recon, long r_sp,
                                                      float* coef_ws, long cw_sp) {
  extern __shared__ __align__(16) float psm[];
  const int p = blockIdx.x;
  const int r = rr[p];
  const float* U = u + p * u_sp;
  const float* X = x + p * x_sp;
  float* Rc = recon + p * r_sp;
  float* Cf = coef_ws + p * cw_sp;  // [t][ld]
  // coef[t][c] = sum_i X[t][i] U[i][c]
  cta_gemm(t, r, n, X, n, 1, U, ld, 1, Cf, ld, 1, 1.f, 0.f, psm);
  // recon[t][i] = sum_c coef[t][c] U[i][c]
  cta_gemm(t, n, r, Cf, ld, 1, U, 1, ld, Rc, n, 1, 1.f, 0.f, psm);
}

}  // namespace kvd

// ---------------------------------------------------------------- host glue

namespace kvd_host {

using namespace kvd;

long bug_step_ws_per_problem(int n, int b, int ld) { return align16(step_ws_bytes(n, b, ld)); }

// Shared memory a step would like: gemm scratch + misc + the larger of the
// residual phase (R and V_h) and the core phase (V_h, B^T and W).
static long step_smem_want(int n, int b, int ld) {
  const long N = ld + b, LB = ld + b;
  const long phase1 = (long)b * n + (long)b * b;
  const long phase2 = (long)b * b + N * LB + N * N;
  return 4L * kGemmSmemFloats + kStepMiscBytes + 4L * (phase1 > phase2 ? phase1 : phase2);
}

int launch_bug_step(const BugStepBatch& batch, int n_problems, int n_streams, cudaStream_t stream) {
  const BugStepArgs& a0 = batch.s[0];
  static int max_dyn = 0;
  if (!max_dyn) {
    cudaFuncAttributes attr;
    int dev = 0, optin = 0;
    cudaFuncGetAttributes(&attr, (const void*)bug_step_kernel);
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    max_dyn = optin - (int)attr.sharedSizeBytes;
  }
  long want = step_smem_want(a0.n, a0.b, a0.ld);
  const int smem = (int)(want < max_dyn ? want : max_dyn);
  if (int rc = ensure_smem((const void*)bug_step_kernel, smem, "bug_step_kernel")) return rc;
  dim3 grid(n_problems, n_streams);
  {
    KTimerScope kts_("bug_step_kernel", stream);
    bug_step_kernel<<<grid, kStepThreads, smem, stream>>>(batch, smem);
  }
  return check_launch("bug_step_kernel");
}

int launch_carry(const CarryBatch& batch, int n_problems, int n_streams, int ld, cudaStream_t stream) {
  if (batch.W <= 0) return KVD_OK;
  const int tok = 128;
  dim3 grid((batch.W + tok - 1) / tok, n_problems, n_streams);
  const int smem = 4 * (ld * ld + 8 * ld);
  if (int rc = ensure_smem((const void*)carry_kernel, smem, "carry_kernel")) return rc;
  {
    KTimerScope kts_("carry_kernel", stream);
    carry_kernel<<<grid, 256, smem, stream>>>(batch, tok);
  }
  return check_launch("carry_kernel");
}

int launch_surprise_f32(int nb, int n, int m, int ld, const float* u, long u_sp, const int* r,
                        const float* x, long x_sp, float* out, long out_sp, cudaStream_t stream) {
  if (m <= 0 || nb <= 0) return KVD_OK;
  dim3 grid((m + 7) / 8, nb);
  surprise_f32_kernel<<<grid, 256, 0, stream>>>(n, m, ld, u, u_sp, r, x, x_sp, out, out_sp);
  return check_launch("surprise_f32_kernel");
}

}  // namespace kvd_host

// ---------------------------------------------------------------- C ABI

using namespace kvd;
using namespace kvd_host;

extern "C" size_t kvd_bug_step_workspace_bytes(int32_t n_batch, int32_t n, int32_t b, int32_t ld_u) {
  return (size_t)n_batch * (size_t)bug_step_ws_per_problem(n, b, ld_u) + 16;
}

extern "C" int kvd_bug_step(int32_t n_batch, int32_t n, int32_t b, int32_t rank_cap, int32_t ld_u,
                            const float* u, float* u_out, float* sigma, int32_t* r,
                            const float* block, float* rot_out, int32_t* m_out, float* coords_out,
                            int32_t has_theta, float theta, int32_t* status, void* workspace,
                            size_t ws_bytes, kvd_stream_t stream) {
  if (n_batch <= 0 || n <= 0 || b <= 0 || rank_cap < 1 || rank_cap > ld_u) {
    set_error("kvd_bug_step: bad sizes (n_batch=%d n=%d b=%d rank_cap=%d ld=%d)", n_batch, n, b,
              rank_cap, ld_u);
    return KVD_ERR_ARG;
  }
  if (u == u_out) {
    set_error("kvd_bug_step: u_out must not alias u");
    return KVD_ERR_ARG;
  }
  const long per = bug_step_ws_per_problem(n, b, ld_u);
  // dims live at the front of the workspace
  const size_t need = (size_t)n_batch * per + align16(16L * n_batch) + 16;
  if (ws_bytes < need) {
    set_error("kvd_bug_step: workspace %zu < %zu bytes", ws_bytes, need);
    return KVD_ERR_WORKSPACE;
  }
  char* base = (char*)(((uintptr_t)workspace + 15) & ~(uintptr_t)15);
  int* dims = (int*)base;
  char* ws = base + align16(16L * n_batch);
  BugStepBatch batch;
  BugStepArgs& a = batch.s[0];
  a.n = n; a.b = b; a.rank_cap = rank_cap; a.ld = ld_u;
  a.u = u; a.u_out = u_out; a.u_sp = (long)n * ld_u;
  a.sigma = sigma; a.sig_sp = ld_u; a.r = r;
  a.x = block; a.x_sp = (long)b * n;
  a.rot = rot_out; a.rot_sp = (long)ld_u * ld_u;
  a.dims = dims;
  a.coords = coords_out; a.coords_sp = (long)b * ld_u; a.coords_ld = ld_u;
  a.has_theta = has_theta; a.theta = theta; a.status = status;
  a.ws = ws; a.ws_sp = per;
  batch.s[1] = a;
  int rc = launch_bug_step(batch, n_batch, 1, (cudaStream_t)stream);
  if (rc) return rc;
  if (m_out) {
    // m is dims[p][2]: gather with a strided 2-D copy
    cudaMemcpy2DAsync(m_out, sizeof(int32_t), dims + 2, 4 * sizeof(int), sizeof(int32_t), n_batch,
                      cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
  }
  return check_launch("kvd_bug_step");
}

extern "C" int kvd_surprise(int32_t n_batch, int32_t n, int32_t m, int32_t ld_u, const float* u,
                            const int32_t* r, const float* x, float* out, kvd_stream_t stream) {
  if (n_batch < 0 || n <= 0 || m < 0 || ld_u < 1) {
    set_error("kvd_surprise: bad sizes");
    return KVD_ERR_ARG;
  }
  return launch_surprise_f32(n_batch, n, m, ld_u, u, (long)n * ld_u, r, x, (long)m * n, out, m,
                             (cudaStream_t)stream);
}

extern "C" int kvd_select_topk(int32_t n_batch, int32_t m, int32_t k, const float* scores,
                               int32_t* keep_idx, int32_t* demote_idx, kvd_stream_t stream) {
  if (n_batch < 0 || m < 0 || k < 0 || k > m || m > 16384) {
    set_error("kvd_select_topk: bad sizes (m=%d k=%d)", m, k);
    return KVD_ERR_ARG;
  }
  if (n_batch == 0 || m == 0) return KVD_OK;
  if (int rc = ensure_smem((const void*)select_topk_kernel, 4 * m, "select_topk_kernel")) return rc;
  {
    KTimerScope kts_("select_topk_kernel", (cudaStream_t)stream);
    select_topk_kernel<<<n_batch, 1024, 4 * m, (cudaStream_t)stream>>>(m, k, scores, keep_idx,
                                                                     demote_idx);
  }
  return check_launch("select_topk_kernel");
}
