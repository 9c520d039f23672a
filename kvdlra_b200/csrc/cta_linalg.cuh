// CTA-wide dense linear algebra building blocks used by the BUG-step kernels.
//
// Everything here is executed cooperatively by all threads of one CTA and
// ends with __syncthreads(); matrices may live in shared or global memory
// (generic pointers).  Sizes are small (n <= a few thousand rows, ranks and
// blocks <= a few hundred), so these are latency-oriented, not peak-FLOP,
// routines.
#pragma once

#include "common.cuh"

namespace kvd {

// C(m,n) = alpha * sum_k A(m,k) B(k,n) + beta * C(m,n), fp32 FFMA.
// A(m,k) = A[m*sam + k*sak], B(k,n) = B[k*sbk + n*sbn], C(m,n) = C[m*scm + n*scn].
// 64x64 output tiles, K in steps of 16, 2x4 outputs per thread (512 threads).
// `sm` needs 2*16*64 floats.  beta == 0 never reads C.
static __device__ void cta_gemm(int M, int N, int K, const float* A, long sam, long sak, const float* B,
                         long sbk, long sbn, float* C, long scm, long scn, float alpha, float beta,
                         float* sm) {
  constexpr int BM = 64, BN = 64, BK = 16;
  float* As = sm;            // [BK][BM]
  float* Bs = sm + BK * BM;  // [BK][BN]
  const int tid = threadIdx.x;
  const int nthr = blockDim.x;
  const int tr = tid / 16, tc = tid % 16;  // 32 x 16 thread grid -> rows 2*tr.., cols 4*tc..
  const bool active = tid < 512;
  for (int m0 = 0; m0 < M; m0 += BM) {
    for (int n0 = 0; n0 < N; n0 += BN) {
      float acc[2][4];
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
      for (int k0 = 0; k0 < K; k0 += BK) {
        for (int e = tid; e < BK * BM; e += nthr) {
          const int kk = e / BM, mm = e % BM;
          const int gm = m0 + mm, gk = k0 + kk;
          As[kk * BM + mm] = (gm < M && gk < K) ? A[gm * sam + gk * sak] : 0.f;
        }
        for (int e = tid; e < BK * BN; e += nthr) {
          const int kk = e / BN, nn = e % BN;
          const int gn = n0 + nn, gk = k0 + kk;
          Bs[kk * BN + nn] = (gn < N && gk < K) ? B[gk * sbk + gn * sbn] : 0.f;
        }
        __syncthreads();
        if (active) {
#pragma unroll
          for (int kk = 0; kk < BK; ++kk) {
            const float a0 = As[kk * BM + 2 * tr], a1 = As[kk * BM + 2 * tr + 1];
            const float4 bv = *reinterpret_cast<const float4*>(&Bs[kk * BN + 4 * tc]);
            acc[0][0] = fmaf(a0, bv.x, acc[0][0]); acc[0][1] = fmaf(a0, bv.y, acc[0][1]);
            acc[0][2] = fmaf(a0, bv.z, acc[0][2]); acc[0][3] = fmaf(a0, bv.w, acc[0][3]);
            acc[1][0] = fmaf(a1, bv.x, acc[1][0]); acc[1][1] = fmaf(a1, bv.y, acc[1][1]);
            acc[1][2] = fmaf(a1, bv.z, acc[1][2]); acc[1][3] = fmaf(a1, bv.w, acc[1][3]);
          }
        }
        __syncthreads();
      }
      if (active) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int gm = m0 + 2 * tr + i;
          if (gm >= M) continue;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int gn = n0 + 4 * tc + j;
            if (gn >= N) continue;
            float* cp = C + gm * scm + gn * scn;
            *cp = (beta == 0.f) ? alpha * acc[i][j] : fmaf(alpha, acc[i][j], beta * (*cp));
          }
        }
      }
      __syncthreads();
    }
  }
}

// G = X X^T in fp64 for the `rows` row vectors X[j][0..len) (row stride ldx),
// G row-major with leading dimension ldg; one warp per (j1 <= j2) pair.
static __device__ void cta_gram_rows(int rows, int len, const float* X, long ldx, double* G, int ldg) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  const int pairs = rows * (rows + 1) / 2;
  for (int e = warp; e < pairs; e += nw) {
    // unrank e -> (j1, j2), j1 <= j2, row-major over the upper triangle
    int j1 = 0, rem = e;
    while (rem >= rows - j1) { rem -= rows - j1; ++j1; }
    const int j2 = j1 + rem;
    const float* x1 = X + j1 * ldx;
    const float* x2 = X + j2 * ldx;
    double acc = 0.0;
    for (int i = lane; i < len; i += 32) acc += (double)x1[i] * (double)x2[i];
    acc = warp_sum(acc);
    if (lane == 0) { G[j1 * ldg + j2] = acc; G[j2 * ldg + j1] = acc; }
  }
  __syncthreads();
}

// Round-robin (circle method) partner of slot i in round k for N' players.
KVD_DEVICE void rr_pair(int i, int k, int np, int* a, int* b) {
  auto idx = [&](int j) { return j == 0 ? 0 : ((j - 1 + k) % (np - 1)) + 1; };
  *a = idx(i);
  *b = idx(np - 1 - i);
}

// Cyclic two-sided Jacobi eigensolver for a symmetric N x N fp64 matrix A
// (leading dimension ld).  On exit A is (numerically) diagonal, V holds the
// eigenvectors (columns), and the function returns the number of sweeps it
// took (> max_sweeps when it did not converge).  `cs` needs 4*(N/2+1) doubles
// of shared memory.  Rotations follow Golub & Van Loan, Alg. 8.4.2 (sym.schur2),
// applied to N'/2 disjoint pairs per round in parallel.
static __device__ int cta_jacobi_eig(double* A, double* V, int N, int ld, double* cs, int max_sweeps) {
  __shared__ int s_rotated;
  const int tid = threadIdx.x, nthr = blockDim.x;
  for (int e = tid; e < N * N; e += nthr) {
    const int i = e / N, j = e % N;
    V[i * ld + j] = (i == j) ? 1.0 : 0.0;
  }
  __syncthreads();
  if (N <= 1) return 0;
  // Scale of the matrix (largest diagonal magnitude): entries below ~1e-17 of
  // it are rounding noise and never rotated, so rank-deficient PSD matrices
  // (null blocks full of noise) converge too.
  __shared__ double s_scale;
  if (tid == 0) {
    double m = 0.0;
    for (int i = 0; i < N; ++i) m = fmax(m, fabs(A[i * ld + i]));
    s_scale = m;
  }
  __syncthreads();
  const double floor_rot = 1e-17 * s_scale, floor_flag = 1e-14 * s_scale;
  const int np = N + (N & 1);
  const int half = np / 2;
  double* pc = cs;            // cos
  double* ps = cs + half;     // sin
  int* pidx = reinterpret_cast<int*>(cs + 2 * half);  // p, q per pair (2*half ints)
  int sweep = 0;
  for (; sweep < max_sweeps; ++sweep) {
    if (tid == 0) s_rotated = 0;
    __syncthreads();
    for (int k = 0; k < np - 1; ++k) {
      for (int i = tid; i < half; i += nthr) {
        int a, b;
        rr_pair(i, k, np, &a, &b);
        int p = a < b ? a : b, q = a < b ? b : a;
        double c = 1.0, s = 0.0;
        if (q < N) {
          const double apq = A[p * ld + q];
          const double app = A[p * ld + p], aqq = A[q * ld + q];
          const double thr = fmax(1e-15 * sqrt(fabs(app * aqq)), floor_rot);
          if (apq != 0.0 && fabs(apq) > thr) {
            const double tau = (aqq - app) / (2.0 * apq);
            const double t = (tau >= 0.0) ? 1.0 / (tau + sqrt(1.0 + tau * tau))
                                          : -1.0 / (-tau + sqrt(1.0 + tau * tau));
            c = 1.0 / sqrt(1.0 + t * t);
            s = t * c;
            if (fabs(apq) > fmax(4e-15 * sqrt(fabs(app * aqq)), floor_flag)) s_rotated = 1;
          }
        } else {
          q = -1;
        }
        pc[i] = c; ps[i] = s; pidx[2 * i] = p; pidx[2 * i + 1] = q;
      }
      __syncthreads();
      // rows: A <- J^T A
      for (int e = tid; e < half * N; e += nthr) {
        const int i = e / N, j = e % N;
        const int q = pidx[2 * i + 1];
        const double s = ps[i];
        if (q < 0 || s == 0.0) continue;
        const int p = pidx[2 * i];
        const double c = pc[i];
        const double x = A[p * ld + j], y = A[q * ld + j];
        A[p * ld + j] = c * x - s * y;
        A[q * ld + j] = s * x + c * y;
      }
      __syncthreads();
      // columns: A <- A J, V <- V J
      for (int e = tid; e < half * N; e += nthr) {
        const int i = e / N, j = e % N;
        const int q = pidx[2 * i + 1];
        const double s = ps[i];
        if (q < 0 || s == 0.0) continue;
        const int p = pidx[2 * i];
        const double c = pc[i];
        const double x = A[j * ld + p], y = A[j * ld + q];
        A[j * ld + p] = c * x - s * y;
        A[j * ld + q] = s * x + c * y;
        const double vx = V[j * ld + p], vy = V[j * ld + q];
        V[j * ld + p] = c * vx - s * vy;
        V[j * ld + q] = s * vx + c * vy;
      }
      __syncthreads();
    }
    const int rot = s_rotated;
    __syncthreads();
    if (!rot) break;
  }
  return sweep;
}

// order[0..N) = indices of vals sorted descending, ties by lower index.
static __device__ void cta_argsort_desc(const double* vals, int N, int* order) {
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const double v = vals[i];
    int rank = 0;
    for (int j = 0; j < N; ++j) {
      const double w = vals[j];
      rank += (w > v) || (w == v && j < i);
    }
    order[rank] = i;
  }
  __syncthreads();
}

// Block-wide exclusive prefix sum of one int per thread (blockDim <= 1024).
// `scratch` >= 32 ints of shared memory.  Returns the exclusive prefix; *total
// receives the block sum.
static __device__ int cta_exclusive_scan(int v, int* scratch, int* total) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, nw = (blockDim.x + 31) / 32;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) scratch[lane] = w;
  }
  __syncthreads();
  const int base = warp > 0 ? scratch[warp - 1] : 0;
  *total = scratch[nw - 1];
  __syncthreads();
  return base + x - v;
}

}  // namespace kvd
