// Batched augmented rank-adaptive BUG step and the coordinate carry (sm_100a).
//
// Restates src/kvdlra/integrators/streaming_torch.py:82-189 for a batch of
// independent problems (one CTA per problem x stream):
//   a = U^T X ; R = X - U a ; a2 = U^T R ; R -= U a2 ; a += a2     (fp32 FFMA)
//   eig(R^T R) in fp64 (two-sided Jacobi)  -> s, V ; admit s > 100 eps |X|_F
//   Q = R V_m / s, made orthonormal by CGS2 (completion for null directions)
//   eig(B B^T), B = [[diag(sigma), a], [0, diag(s_m) V_m^T]]  (fp64 Jacobi)
//   U_new = [U | Q] W[:, :keep], sigma_new, rot = W[:r, :keep]^T,
//   coords = U_new^T X.
// The left singular vectors/values of B are the eigenpairs of B B^T; forming
// the Gram in fp64 from fp32 inputs keeps the fp32-level accuracy of the
// reference's SVD for every singular value above ~1e-8 of the largest.
#include <stdio.h>

#include <cfloat>

#include "kernels.cuh"

namespace kvd {


struct StepWs {
  float* a;      // [ld][b]
  float* R;      // [b][n]
  float* Q;      // [b][n]
  double* H;     // [b][b]
  double* VH;    // [b][b]
  double* G;     // [N][N]
  double* VG;    // [N][N]
  double* lam;   // [N]
  int* ord;      // [N]
  int* ordh;     // [b]
  double* sv;    // [b]
  float* WU;     // [N][ld]  top eigenvectors of G (fp32)
  float* VQ;     // [b][b]   V_h[:, j] / s_j  (fp32)
  double* VS;    // [b][b]   V_h columns in descending-s order
};

__host__ __device__ inline long align16(long x) { return (x + 15) & ~15L; }

__host__ __device__ inline long step_ws_bytes(int n, int b, int ld) {
  const long N = ld + b;
  long o = 0;
  o += align16(4L * ld * b);
  o += align16(4L * b * n) * 2;
  o += align16(8L * b * b) * 2;
  o += align16(8L * N * N) * 2;
  o += align16(8L * N);
  o += align16(4L * N);
  o += align16(4L * b);
  o += align16(8L * b);
  o += align16(4L * N * ld);
  o += align16(4L * b * b);
  o += align16(8L * b * b);
  return o;
}

__device__ StepWs carve(char* base, int n, int b, int ld) {
  const long N = ld + b;
  StepWs w;
  long o = 0;
  auto take = [&](long bytes) { char* p = base + o; o += align16(bytes); return p; };
  w.a = (float*)take(4L * ld * b);
  w.R = (float*)take(4L * b * n);
  w.Q = (float*)take(4L * b * n);
  w.H = (double*)take(8L * b * b);
  w.VH = (double*)take(8L * b * b);
  w.G = (double*)take(8L * N * N);
  w.VG = (double*)take(8L * N * N);
  w.lam = (double*)take(8L * N);
  w.ord = (int*)take(4L * N);
  w.ordh = (int*)take(4L * b);
  w.sv = (double*)take(8L * b);
  w.WU = (float*)take(4L * N * ld);
  w.VQ = (float*)take(4L * b * b);
  w.VS = (double*)take(8L * b * b);
  return w;
}

// Shared-memory plan: gemm scratch (8 KB) + Jacobi pair table + optionally the
// Jacobi matrices when they fit.
constexpr int kGemmSmemFloats = 2 * 16 * 64;
constexpr int kStepThreads = 512;

__device__ void cta_copy_d(double* dst, const double* src, int count) {
  for (int e = threadIdx.x; e < count; e += blockDim.x) dst[e] = src[e];
  __syncthreads();
}

// Orthonormalise the rows of Q[0..m) (length n) in order by classical
// Gram-Schmidt applied twice; a row that collapses (numerically dependent or
// null) is replaced by the first canonical vector e_i that survives the same
// orthogonalisation.  Returns nothing; Q is updated in place.
__device__ void cta_cgs2_rows(float* Q, int m, int n, double* dots /*>= m*/, double* red /*>=33*/) {
  __shared__ double s_norm, s_norm0;
  __shared__ int s_next_e;
  const int tid = threadIdx.x, nthr = blockDim.x, lane = tid % 32, warp = tid / 32,
            nw = nthr / 32;
  if (tid == 0) s_next_e = 0;
  __syncthreads();
  for (int j = 0; j < m; ++j) {
    float* qj = Q + (long)j * n;
    // norm before
    double acc = 0.0;
    for (int i = tid; i < n; i += nthr) acc += (double)qj[i] * qj[i];
    acc = warp_sum(acc);
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (tid == 0) { double t = 0; for (int w = 0; w < nw; ++w) t += red[w]; s_norm0 = sqrt(t); }
    __syncthreads();
    bool replaced = false;
    for (int attempt = 0; attempt < n + 1; ++attempt) {
      for (int pass = 0; pass < 2; ++pass) {
        // dots with previous rows, one warp per previous row
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
      // collapsed: restart from the next canonical vector
      const int e = s_next_e;
      __syncthreads();
      if (e >= n) break;  // cannot happen while m <= n
      for (int i = tid; i < n; i += nthr) qj[i] = (i == e) ? 1.f : 0.f;
      if (tid == 0) { s_next_e = e + 1; s_norm0 = 1.0; }
      replaced = true;
      __syncthreads();
    }
    (void)replaced;
    const float inv = (float)(1.0 / s_norm);
    for (int i = tid; i < n; i += nthr) qj[i] *= inv;
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kStepThreads) bug_step_kernel(BugStepBatch batch, int smem_mat_ok) {
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
  double* jac_cs = reinterpret_cast<double*>(smem_raw + 4 * kGemmSmemFloats);  // 4*(N/2+1)
  const int Nmax = ld + b;
  double* red = jac_cs + 4 * (Nmax / 2 + 2);                                     // 64 doubles
  double* smat = red + 64;                                                       // optional
  __shared__ double s_xnorm2;
  __shared__ int s_m, s_keep;
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
  // ----- projections and residual
  for (long e = tid; e < (long)b * n; e += nthr) w.R[e] = X[e];
  __syncthreads();
  if (r > 0) {
    // a = U^T X : (r x b)
    cta_gemm(r, b, n, U, 1, ld, X, 1, n, w.a, b, 1, 1.f, 0.f, gsm);
    // R -= U a   (R stored [j][i])
    cta_gemm(n, b, r, U, ld, 1, w.a, b, 1, w.R, 1, n, -1.f, 1.f, gsm);
    // a2 = U^T R -> Q scratch [r][b]
    float* a2 = w.Q;
    cta_gemm(r, b, n, U, 1, ld, w.R, 1, n, a2, b, 1, 1.f, 0.f, gsm);
    cta_gemm(n, b, r, U, ld, 1, a2, b, 1, w.R, 1, n, -1.f, 1.f, gsm);
    for (int e = tid; e < r * b; e += nthr) w.a[e] += a2[e];
    __syncthreads();
  }
  // ----- H = R^T R (fp64), eig
  const bool h_in_smem = smem_mat_ok && (2L * b * b <= 2L * Nmax * Nmax);
  double* Hm = h_in_smem ? smat : w.H;
  double* Vm = h_in_smem ? smat + b * b : w.VH;
  cta_gram_rows(b, n, w.R, n, Hm, b);
  int sw = cta_jacobi_eig(Hm, Vm, b, b, jac_cs, 40);
  if (sw >= 40 && tid == 0) atomicOr(&A.status[kStatusNumeric], 1);
  for (int j = tid; j < b; j += nthr) w.sv[j] = Hm[j * b + j];
  __syncthreads();
  cta_argsort_desc(w.sv, b, w.ordh);
  // singular values in descending order; admission
  if (tid == 0) {
    const float xnorm = (float)sqrt(s_xnorm2);
    const double tol = 100.0 * (double)FLT_EPSILON * (double)xnorm;
    int m;
    if (r == 0) {
      m = min(n, b);
    } else {
      m = 0;
      for (int j = 0; j < b; ++j) {
        const double lamj = w.sv[w.ordh[j]];
        const float sj = (float)sqrt(fmax(lamj, 0.0));
        if ((double)sj > tol) ++m;
      }
      m = min(m, max(0, n - r));
    }
    s_m = m;
  }
  __syncthreads();
  const int m = s_m;
  // VQ[l][j] = V[l][ord_j] / s_j (fp32), j < m
  for (int e = tid; e < b * m; e += nthr) {
    const int l = e / m, j = e % m;
    const int oj = w.ordh[j];
    const double sj = sqrt(fmax(w.sv[oj], 0.0));
    const double s0 = sqrt(fmax(w.sv[w.ordh[0]], 0.0));
    // a direction below 1e-12 of the largest is numerically null: leave it to
    // the orthonormal completion in cta_cgs2_rows
    w.VQ[l * m + j] = (sj > 1e-12 * s0 && sj > 0.0) ? (float)(Vm[l * b + oj] / sj) : 0.f;
  }
  // V columns in sorted order for the core build (kept outside the Jacobi storage)
  double* Vs = w.VS;
  for (int e = tid; e < b * m; e += nthr) {
    const int l = e / m, j = e % m;
    Vs[l * b + j] = Vm[l * b + w.ordh[j]];
  }
  for (int j = tid; j < m; j += nthr) w.lam[j] = sqrt(fmax(w.sv[w.ordh[j]], 0.0));  // s_j sorted
  __syncthreads();
  for (int j = tid; j < m; j += nthr) w.sv[j] = w.lam[j];
  __syncthreads();
  // Q[j][i] = sum_l R[l][i] VQ[l][j]
  if (m > 0) {
    cta_gemm(m, n, b, w.VQ, 1, m, w.R, n, 1, w.Q, n, 1, 1.f, 0.f, gsm);
    cta_cgs2_rows(w.Q, m, n, w.lam, red);
  }
  // ----- core Gram G = B B^T, N = r + m
  const int N = r + m;
  const bool g_in_smem = smem_mat_ok != 0;
  double* Gm = g_in_smem ? smat : w.G;
  double* VGm = g_in_smem ? smat + N * N : w.VG;
  for (int e = tid; e < N * N; e += nthr) {
    const int i = e / N, j = e % N;
    if (j < i) continue;
    double g = 0.0;
    if (i < r && j < r) {
      for (int l = 0; l < b; ++l) g += (double)w.a[i * b + l] * (double)w.a[j * b + l];
      if (i == j) g += (double)sig[i] * (double)sig[i];
    } else if (i < r) {  // j >= r
      const int jj = j - r;
      double t = 0.0;
      for (int l = 0; l < b; ++l) t += (double)w.a[i * b + l] * Vs[l * b + jj];
      g = t * (double)(float)w.sv[jj];
    } else {
      const int ii = i - r, jj = j - r;
      double t = 0.0;
      for (int l = 0; l < b; ++l) t += Vs[l * b + ii] * Vs[l * b + jj];
      g = t * (double)(float)w.sv[ii] * (double)(float)w.sv[jj];
    }
    Gm[i * N + j] = g;
    Gm[j * N + i] = g;
  }
  __syncthreads();
  sw = cta_jacobi_eig(Gm, VGm, N, N, jac_cs, 40);
  if (sw >= 40 && tid == 0) atomicOr(&A.status[kStatusNumeric], 2);
  for (int j = tid; j < N; j += nthr) w.lam[j] = Gm[j * N + j];
  __syncthreads();
  cta_argsort_desc(w.lam, N, w.ord);
  if (tid == 0) {
    int keep = min(cap, N);
    if (A.has_theta && N > 0) {
      // smallest k with sqrt(sum_{j>=k} sigma_j^2) <= theta (fp32, as the reference)
      const float th2 = A.theta * A.theta;
      int first_ok = -1;
      float tail = 0.f;
      // tail_sq[k] for k = N-1 .. 0
      for (int k = N - 1; k >= 0; --k) {
        const float sk = (float)sqrt(fmax(w.lam[w.ord[k]], 0.0));
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
  // WU[k][c] = VG[k][ord_c] (fp32)
  for (int e = tid; e < N * keep; e += nthr) {
    const int k = e / keep, c = e % keep;
    w.WU[k * ld + c] = (float)VGm[k * N + w.ord[c]];
  }
  for (int c = tid; c < keep; c += nthr) sig[c] = (float)sqrt(fmax(w.lam[w.ord[c]], 0.0));
  float* rot = A.rot + p * A.rot_sp;
  for (int e = tid; e < keep * r; e += nthr) {
    const int c = e / r, k = e % r;
    rot[c * ld + k] = (float)VGm[k * N + w.ord[c]];
  }
  __syncthreads();
  // U_new = U W[:r] + Q^T W[r:]
  if (r > 0) {
    cta_gemm(n, keep, r, U, ld, 1, w.WU, ld, 1, Uo, ld, 1, 1.f, 0.f, gsm);
    if (m > 0) cta_gemm(n, keep, m, w.Q, 1, n, w.WU + r * ld, ld, 1, Uo, ld, 1, 1.f, 1.f, gsm);
  } else {
    cta_gemm(n, keep, m, w.Q, 1, n, w.WU, ld, 1, Uo, ld, 1, 1.f, 0.f, gsm);
  }
  // coords[j][c] = sum_i X[j][i] U_new[i][c]
  float* co = A.coords + p * A.coords_sp;
  cta_gemm(b, keep, n, X, n, 1, Uo, ld, 1, co, A.coords_ld, 1, 1.f, 0.f, gsm);
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

int step_smem_bytes(int b, int ld, bool with_mats) {
  const int Nmax = ld + b;
  long bytes = 4L * kGemmSmemFloats + 8L * 4 * (Nmax / 2 + 2) + 8L * 64;
  if (with_mats) bytes += 16L * Nmax * Nmax;
  return (int)bytes;
}

long bug_step_ws_per_problem(int n, int b, int ld) { return align16(step_ws_bytes(n, b, ld)); }

int launch_bug_step(const BugStepBatch& batch, int n_problems, int n_streams, cudaStream_t stream) {
  const BugStepArgs& a0 = batch.s[0];
  int smem = step_smem_bytes(a0.b, a0.ld, true);
  int ok = 1;
  if (smem > 200 * 1024) {  // Jacobi matrices stay in global workspace
    smem = step_smem_bytes(a0.b, a0.ld, false);
    ok = 0;
  }
  if (int rc = ensure_smem((const void*)bug_step_kernel, smem, "bug_step_kernel")) return rc;
  dim3 grid(n_problems, n_streams);
  {
    KTimerScope kts_("bug_step_kernel", stream);
    bug_step_kernel<<<grid, kStepThreads, smem, stream>>>(batch, ok);
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
