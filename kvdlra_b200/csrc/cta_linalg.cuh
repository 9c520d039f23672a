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

// Round-robin (circle method) partner of slot i in round k for N' players
// (player 0 fixed, the others rotate by k; 0 <= k < np - 1).
KVD_DEVICE void rr_pair(int i, int k, int np, int* a, int* b) {
  const int m = np - 1;
  auto idx = [&](int j) {
    if (j == 0) return 0;
    int t = j - 1 + k;
    if (t >= m) t -= m;
    return t + 1;
  };
  *a = idx(i);
  *b = idx(np - 1 - i);
}

// order[0..N) = indices of vals sorted descending, ties by lower index.  NaN
// sorts below every number, so order is always a permutation.
static __device__ void cta_argsort_desc(const double* vals, int N, int* order) {
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const double v = vals[i] == vals[i] ? vals[i] : -INFINITY;
    int rank = 0;
    for (int j = 0; j < N; ++j) {
      const double w = vals[j] == vals[j] ? vals[j] : -INFINITY;
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
