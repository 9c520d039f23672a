// Exact-tier ("SLASH") selection kernels (sm_100a).
//
//  * slash_score_kernel   -- un-rotate every candidate of the pool [hh | grad]
//    (post-RoPE, model dtype) and score its low-rank surprise against the
//    pre-step basis: bug_cache.py:803-804 + 906-921.  fp64 accumulation of the
//    fp32 projection so the score is as exact as the basis allows.
//  * slash_rank_kernel    -- optional span boost (923-950), stable descending
//    top-h (810-812): the slot order of kept and demoted candidates, their
//    positions and graduation surprise, and the gather of the demoted ones
//    (un-rotated K, fp32 V) into the BUG-step block (813-825 + 871-888).
//    The same ranking runs inside slash_score_dmma_kernel's launch (the
//    last scoring CTA of each problem) where that kernel applies.
//  * slash_keep_kernel    -- compaction of the kept tokens into the other
//    exact-tier buffer, one warp per row over the whole GPU.
//  * gather_block_kernel  -- the no-tier absorb path (743-750).
//  * evict_kernel         -- coordinate-budget eviction (954-1067).
#include <cfloat>

#include "kernels.cuh"

namespace kvd {


constexpr int kScoreTile = 32;   // candidates per CTA
constexpr int kScoreMaxQ = 24;   // rank <= 8 * 24 = 192

template <typename T, int QN>
__global__ void __launch_bounds__(256) slash_score_kernel(CandSrc<T> src, int m, int H, int D,
                                                          RopeArgs rope, const float* u, long u_sp,
                                                          int ld, const int* rr, float* scores,
                                                          long sc_sp) {
  extern __shared__ __align__(16) float ssm[];
  const int p = blockIdx.y;
  const int j0 = blockIdx.x * kScoreTile;
  const int half = D / 2;
  const int r = rr[p];
  float* cs = ssm;                                   // [tile][half][2]
  float* kt = cs + kScoreTile * half * 2;            // [tile][D]
  float* us = kt + kScoreTile * D;                   // [D][r]
  const int tid = threadIdx.x;
  const int jl = tid / 8, sub = tid % 8;
  const int j = j0 + jl;
  for (int e = tid; e < kScoreTile * half; e += blockDim.x) {
    const int a = e / half, f = e % half;
    const int jj = j0 + a;
    float c = 1.f, s = 0.f;
    if (jj < m) rope_cs(src.pos(p, jj), rope.inv_freq[f], rope.scale, &c, &s);
    cs[2 * e] = c;
    cs[2 * e + 1] = s;
  }
  double acc[QN];
#pragma unroll
  for (int q = 0; q < QN; ++q) acc[q] = 0.0;
  double kk = 0.0;
  const float* U = u + p * u_sp;
  for (int h = 0; h < H; ++h) {
    __syncthreads();
    for (int e = tid; e < kScoreTile * half; e += blockDim.x) {
      const int a = e / half, f = e % half;
      const int jj = j0 + a;
      float y1 = 0.f, y2 = 0.f;
      if (jj < m) {
        const T* kr = src.krow(p, jj) + h * D;
        const float x1 = load_f<T>(kr + f), x2 = load_f<T>(kr + f + half);
        const float c = cs[2 * e], s = cs[2 * e + 1];
        y1 = (x1 * c + x2 * s) / rope.scale_sq;
        y2 = (x2 * c - x1 * s) / rope.scale_sq;
      }
      kt[a * D + f] = y1;
      kt[a * D + f + half] = y2;
    }
    if (r > 0) {
      for (int e = tid; e < D * r; e += blockDim.x) {
        const int d = e / r, k = e % r;
        us[e] = U[(long)(h * D + d) * ld + k];
      }
    }
    __syncthreads();
    const float* krow = kt + jl * D;
    for (int d = sub; d < D; d += 8) kk += (double)krow[d] * (double)krow[d];
    if (r > 0) {
      for (int d = 0; d < D; ++d) {
        const double kv = (double)krow[d];
        const float* ur = us + d * r;
#pragma unroll
        for (int q = 0; q < QN; ++q) {
          const int k = sub + 8 * q;
          if (k < r) acc[q] += (double)ur[k] * kv;
        }
      }
    }
  }
  double cc = 0.0;
#pragma unroll
  for (int q = 0; q < QN; ++q) cc += acc[q] * acc[q];
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) {
    cc += __shfl_xor_sync(0xffffffffu, cc, o);
    kk += __shfl_xor_sync(0xffffffffu, kk, o);
  }
  if (sub == 0 && j < m) {
    float out;
    if (r == 0) {
      out = 1.f;
    } else {
      const double kn = sqrt(kk);
      out = (float)(sqrt(fmax(kk - cc, 0.0)) / fmax(kn, 1e-12));
    }
    scores[p * sc_sp + j] = out;
  }
}


// The same scores with the projection on the fp64 tensor cores
// (mma.m8n8k4.f64: exact products of the fp32 values, fp64 sums), for
// rank <= 32 and head_dim a multiple of 8.  A CTA takes kScT candidates: their
// un-rotated rows (all heads) and the basis are staged once, in fp32 at padded
// pitches (conflict-free fragment loads), then the K = n product runs in one
// pass; warp w owns the candidate tile w % 2 and the coordinate tiles
// 2 (w / 2) + {0, 1}.
constexpr int kScT = 32;
constexpr int kScThreads = 4 * kScT * 4;  // (kScT / 8) candidate tiles x 2 coordinate-tile pairs x 2 k halves


__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

template <typename T>
__device__ __noinline__ void rank_problem(const CandSrc<T>& src, int p, int m, int keep_n, int H, int D,
                                          const RopeArgs& rope, const float* scores, long sc_sp,
                                          int hh_neighbor, const SelectOut& out, float* sel_sm);

// Requires rows of n*sizeof(T) and of ld floats in 16-byte multiples, 16-byte
// aligned (checked by the launcher): the basis and the candidates' raw rows
// are copied with cp.async, all in flight at once, then un-rotated in place.
// With rk.done, the CTA that completes a problem's scores also ranks it.
template <typename T>
__global__ void __launch_bounds__(kScThreads) slash_score_dmma_kernel(CandSrc<T> src, int m, int H, int D,
                                                               RopeArgs rope, const float* u,
                                                               long u_sp, int ld, const int* rr,
                                                               float* scores, long sc_sp, RankArgs rk) {
  extern __shared__ __align__(16) double dsm[];
  const int p = blockIdx.y;
  const int j0 = blockIdx.x * kScT;
  const int half = D / 2, n = H * D;
  const int r = rr[p];
  const int ldx = n + 4, ldu = 40;                 // floats: 4 / 8 mod 32 (conflict-free fragments)
  double* kk = dsm;                                // [kScT]     |k|^2
  double* ccp = kk + kScT;                         // [2][kScT]  |c|^2 halves
  double* pcb = ccp + 2 * kScT;                    // [8 warps][32][4] second k half's tiles
  float* xs = reinterpret_cast<float*>(pcb + 8 * 32 * 4);  // [kScT][ldx] un-rotated rows
  float* us = xs + kScT * ldx;                     // [n][ldu]   basis, zero past r
  float* cs = us + (long)n * ldu;                  // [kScT][half][2] RoPE
  T* kraw = reinterpret_cast<T*>(cs + kScT * half * 2);  // [kScT][n] raw candidate rows
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int mt = warp % (kScT / 8), ntp = (warp / (kScT / 8)) % 2, nt0 = 2 * ntp;
  const int ks = warp / (kScT / 4);  // half of the k range (n % 16 == 0)
  const int grp = lane >> 2, tig = lane & 3;
  const float* U = u + p * u_sp;
  const int nu = r < 32 ? r : 32;
  // asynchronous copies: the basis rows (first 32 columns) and the raw candidate rows
  {
    const int q4 = (nu + 3) / 4;  // 16-byte chunks per basis row actually needed
    for (int e = tid; e < n * q4; e += blockDim.x) {
      const int f = e / q4, q = e % q4;
      cp_async16(us + (long)f * ldu + 4 * q, U + (long)f * ld + 4 * q);
    }
    constexpr int per = 16 / sizeof(T);
    const int rq = n / per;
    for (int e = tid; e < kScT * rq; e += blockDim.x) {
      const int a = e / rq, q = e % rq;
      const int jj = j0 + a;
      if (jj < m) cp_async16(kraw + (long)a * n + q * per, src.krow(p, jj) + q * per);
    }
  }
  for (int e = tid; e < kScT * half; e += blockDim.x) {
    const int a = e / half, f = e % half;
    const int jj = j0 + a;
    float c = 1.f, s = 0.f;
    if (jj < m) rope_cs(src.pos(p, jj), rope.inv_freq[f], rope.scale, &c, &s);
    cs[2 * e] = c;
    cs[2 * e + 1] = s;
  }
  cp_async_wait_all();
  __syncthreads();
  if (nu < 32) {  // columns past the rank are zero
    for (int e = tid; e < n * 32; e += blockDim.x) {
      const int f = e / 32, k = e % 32;
      if (k >= 4 * ((nu + 3) / 4) || k >= nu) us[(long)f * ldu + k] = 0.f;
    }
  }
  for (int e = tid; e < kScT * H * half; e += blockDim.x) {  // (candidate, head, pair)
    const int a = e / (H * half), hf = e % (H * half), h = hf / half, f = hf % half;
    const int jj = j0 + a;
    float y1 = 0.f, y2 = 0.f;
    if (jj < m) {
      const T* kr = kraw + (long)a * n + h * D;
      const float x1 = load_f<T>(kr + f), x2 = load_f<T>(kr + f + half);
      const float c = cs[2 * (a * half + f)], s = cs[2 * (a * half + f) + 1];
      y1 = (x1 * c + x2 * s) / rope.scale_sq;
      y2 = (x2 * c - x1 * s) / rope.scale_sq;
    }
    xs[a * ldx + h * D + f] = y1;
    xs[a * ldx + h * D + f + half] = y2;
  }
  __syncthreads();
  {  // |k|^2: 16 threads per candidate, fp64
    const int a = tid / 16, sub = tid % 16;
    double sq = 0.0;
    for (int d = sub; d < n; d += 16) {
      const double v = xs[a * ldx + d];
      sq = fma(v, v, sq);
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (sub == 0) kk[a] = sq;
  }
  // tiles nt0, nt0 + 1, each as two chains over alternate k-steps (n % 8 == 0)
  double c00 = 0.0, c01 = 0.0, c10 = 0.0, c11 = 0.0, e00 = 0.0, e01 = 0.0, e10 = 0.0, e11 = 0.0;
  const float* xa = xs + (mt * 8 + grp) * ldx + tig;
  const float* ub = us + tig * ldu + nt0 * 8 + grp;
  const int kh = n / 2;
#pragma unroll 2
  for (int k0 = ks * kh; k0 < (ks + 1) * kh; k0 += 8) {
    const double av = xa[k0], bv = xa[k0 + 4];
    dmma_8x8x4(c00, c01, av, (double)ub[k0 * ldu]);
    dmma_8x8x4(c10, c11, av, (double)ub[k0 * ldu + 8]);
    dmma_8x8x4(e00, e01, bv, (double)ub[(k0 + 4) * ldu]);
    dmma_8x8x4(e10, e11, bv, (double)ub[(k0 + 4) * ldu + 8]);
  }
  c00 += e00; c01 += e01; c10 += e10; c11 += e11;
  double* pw = pcb + ((warp % (kScT / 4)) * 32 + lane) * 4;
  if (ks == 1) { pw[0] = c00; pw[1] = c01; pw[2] = c10; pw[3] = c11; }
  __syncthreads();
  if (ks == 0) {  // the full projection (both k halves), then |c|^2 of each candidate row:
    c00 += pw[0]; c01 += pw[1]; c10 += pw[2]; c11 += pw[3];  // the lane's four values, the
    double cc = c00 * c00 + c01 * c01 + c10 * c10 + c11 * c11;  // row's four lanes, two warps
    cc += __shfl_xor_sync(0xffffffffu, cc, 1);
    cc += __shfl_xor_sync(0xffffffffu, cc, 2);
    if (tig == 0) ccp[ntp * kScT + mt * 8 + grp] = cc;
  }
  __syncthreads();
  if (tid < kScT) {
    const int j = j0 + tid;
    if (j < m) {
      float out;
      if (r == 0) {
        out = 1.f;
      } else {
        const double k2 = kk[tid], c2 = ccp[tid] + ccp[kScT + tid];
        out = (float)(sqrt(fmax(k2 - c2, 0.0)) / fmax(sqrt(k2), 1e-12));
      }
      scores[p * sc_sp + j] = out;
    }
  }
  if (rk.done) {
    __shared__ int s_last;
    __threadfence();  // this CTA's scores are visible before it counts itself done
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(rk.done + p, 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (s_last) {
      __threadfence();
      if (tid == 0) rk.done[p] = 0;  // ready for the next launch
      rank_problem<T>(src, p, m, rk.keep_n, H, D, rope, scores, sc_sp, rk.hh_neighbor, rk.out,
                      reinterpret_cast<float*>(dsm));
    }
  }
}

// The scores for ranks past 32 or feature counts whose basis does not fit
// shared memory whole (head_dim 128: n = 1024), on the fp64 tensor cores.  A
// CTA takes kSwT candidates: their un-rotated rows (all heads, fp32) stay in
// shared memory while the basis streams through in chunks of kSwF feature
// rows (all rank columns, cp.async double buffer, columns past the rank
// zero-filled by the copy).  Warp w owns candidate tile w % 2 and the column
// tiles w / 2 + 4 i: every 8 x 8 x 4 step reuses one A fragment for up to
// six column tiles.  The projection is summed in fp64 (exact products of the
// fp32 values); |k|^2 in fp64; the score as in slash_score_dmma_kernel.
constexpr int kSwT = 16;                    // candidates per CTA
constexpr int kSwF = 64;                    // basis feature rows per chunk
constexpr int kSwThreads = 256;
constexpr int kSwMaxCT = 6;                 // column tiles per warp: rank <= 4 * 6 * 8 = 192

__host__ __device__ inline int sw_ldb(int ld) { return 32 * ((ld + 31) / 32) + 8; }  // = 8 mod 32
__host__ __device__ inline long sw_smem_bytes(int n, int D, int ld) {
  return 8L * (kSwT + 4 * kSwT) + 4L * (kSwT * (long)(n + 4) + 2L * kSwF * sw_ldb(ld) + kSwT * (D / 2) * 2);
}

template <typename T>
__global__ void __launch_bounds__(kSwThreads) slash_score_dmma_wide_kernel(CandSrc<T> src, int m, int H, int D,
                                                                          RopeArgs rope, const float* u,
                                                                          long u_sp, int ld, const int* rr,
                                                                          float* scores, long sc_sp,
                                                                          RankArgs rk) {
  extern __shared__ __align__(16) double wsm[];
  const int p = blockIdx.y;
  const int j0 = blockIdx.x * kSwT;
  const int half = D / 2, n = H * D;
  const int r = rr[p];
  const int ldx = n + 4, ldb = sw_ldb(ld);
  double* kk = wsm;                                   // [kSwT] |k|^2
  double* ccw = kk + kSwT;                            // [4][kSwT] |c|^2 per column-tile set
  float* xs = reinterpret_cast<float*>(ccw + 4 * kSwT);  // [kSwT][ldx] un-rotated rows
  float* bs = xs + kSwT * ldx;                        // 2 x [kSwF][ldb] basis chunks
  float* cs = bs + 2 * kSwF * ldb;                    // [kSwT][half][2] RoPE
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int mt = warp & 1, wc = warp >> 1;
  const int grp = lane >> 2, tig = lane & 3;
  const float* U = u + p * u_sp;
  const int q4 = (r + 3) / 4;          // 16-byte chunks of a basis row that hold rank columns
  const int nct = (r + 7) / 8;         // column tiles
  const int nchunks = n / kSwF;
  auto stage = [&](int c, int buf) {   // basis rows [c kSwF, +kSwF), columns [0, 8 nct)
    float* dst = bs + buf * kSwF * ldb;
    const int q8 = 2 * nct;            // 16-byte chunks per row to fill (zeros past the rank)
    for (int e = tid; e < kSwF * q8; e += kSwThreads) {
      const int f = e / q8, q = e % q8;
      const int bytes = q < q4 ? 4 * min(4, r - 4 * q) : 0;
      const float* srcp = U + (long)(c * kSwF + f) * ld + (q < q4 ? 4 * q : 0);
      const unsigned sa = (unsigned)__cvta_generic_to_shared(dst + f * ldb + 4 * q);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(srcp), "r"(bytes)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  if (r > 0) stage(0, 0);
  for (int e = tid; e < kSwT * half; e += kSwThreads) {
    const int a = e / half, f = e % half;
    const int jj = j0 + a;
    float c = 1.f, s = 0.f;
    if (jj < m) rope_cs(src.pos(p, jj), rope.inv_freq[f], rope.scale, &c, &s);
    cs[2 * e] = c;
    cs[2 * e + 1] = s;
  }
  __syncthreads();
  for (int e = tid; e < kSwT * H * half; e += kSwThreads) {  // (candidate, head, pair), pairs fastest
    const int a = e / (H * half), hf = e % (H * half), h = hf / half, f = hf % half;
    const int jj = j0 + a;
    float y1 = 0.f, y2 = 0.f;
    if (jj < m) {
      const T* kr = src.krow(p, jj) + h * D;
      const float x1 = load_f<T>(kr + f), x2 = load_f<T>(kr + f + half);
      const float c = cs[2 * (a * half + f)], s = cs[2 * (a * half + f) + 1];
      y1 = (x1 * c + x2 * s) / rope.scale_sq;
      y2 = (x2 * c - x1 * s) / rope.scale_sq;
    }
    xs[a * ldx + h * D + f] = y1;
    xs[a * ldx + h * D + f + half] = y2;
  }
  __syncthreads();
  {  // |k|^2: 16 threads per candidate, fp64
    const int a = tid / 16, sub = tid % 16;
    double sq = 0.0;
    for (int d = sub; d < n; d += 16) {
      const double v = xs[a * ldx + d];
      sq = fma(v, v, sq);
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (sub == 0) kk[a] = sq;
  }
  double acc[kSwMaxCT][2];
#pragma unroll
  for (int i = 0; i < kSwMaxCT; ++i) { acc[i][0] = 0.0; acc[i][1] = 0.0; }
  if (r > 0) {
    const float* xa = xs + (mt * 8 + grp) * ldx + tig;
    for (int c = 0; c < nchunks; ++c) {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      __syncthreads();  // chunk c landed for every thread; chunk c - 1's buffer is free
      if (c + 1 < nchunks) stage(c + 1, (c + 1) & 1);
      const float* bb = bs + (c & 1) * kSwF * ldb + tig * ldb + grp;
      const float* xc = xa + c * kSwF;
#pragma unroll 4
      for (int k0 = 0; k0 < kSwF; k0 += 4) {
        const double av = xc[k0];
#pragma unroll
        for (int i = 0; i < kSwMaxCT; ++i) {
          const int ct = wc + 4 * i;
          if (ct < nct) dmma_8x8x4(acc[i][0], acc[i][1], av, (double)bb[k0 * ldb + ct * 8]);
        }
      }
    }
  }
  {  // |c|^2 of each candidate row: the lane's values, the row's four lanes, then the four warps
    double cc = 0.0;
#pragma unroll
    for (int i = 0; i < kSwMaxCT; ++i) cc += acc[i][0] * acc[i][0] + acc[i][1] * acc[i][1];
    cc += __shfl_xor_sync(0xffffffffu, cc, 1);
    cc += __shfl_xor_sync(0xffffffffu, cc, 2);
    if (tig == 0) ccw[wc * kSwT + mt * 8 + grp] = cc;
  }
  __syncthreads();
  if (tid < kSwT) {
    const int j = j0 + tid;
    if (j < m) {
      float out;
      if (r == 0) {
        out = 1.f;
      } else {
        const double k2 = kk[tid];
        const double c2 = (ccw[tid] + ccw[kSwT + tid]) + (ccw[2 * kSwT + tid] + ccw[3 * kSwT + tid]);
        out = (float)(sqrt(fmax(k2 - c2, 0.0)) / fmax(sqrt(k2), 1e-12));
      }
      scores[p * sc_sp + j] = out;
    }
  }
  if (rk.done) {  // the CTA that completes a problem's scores also ranks it
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(rk.done + p, 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (s_last) {
      __threadfence();
      if (tid == 0) rk.done[p] = 0;
      rank_problem<T>(src, p, m, rk.keep_n, H, D, rope, scores, sc_sp, rk.hh_neighbor, rk.out,
                      reinterpret_cast<float*>(wsm));
    }
  }
}

// The 16/sizeof(T) elements of one 16-byte chunk, widened to fp32 (dst 16-byte aligned).
template <typename T> __device__ __forceinline__ void widen16(uint4 r, float* dst);
template <> __device__ __forceinline__ void widen16<float>(uint4 r, float* dst) {
  *reinterpret_cast<float4*>(dst) =
      make_float4(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z), __uint_as_float(r.w));
}
template <> __device__ __forceinline__ void widen16<__nv_bfloat16>(uint4 r, float* dst) {
  const unsigned w[4] = {r.x, r.y, r.z, r.w};
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // bf16 -> fp32 is the 16 bits shifted up
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
  *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// Ranking half of the tier update, one CTA per problem: span boost, stable
// descending rank, and the slot order [kept sources (chronological) |
// demoted sources (chronological)] written to out.order; positions and
// graduation surprise go straight to their buffers, and the demoted rows --
// all the BUG step needs -- are gathered here (one warp per row: key
// un-rotated into the fp32 block with cos/sin once per frequency, value
// widened).  The kept rows move in slash_keep_kernel, off the critical path.
// The ranking of problem p by the whole CTA (any block size), in `sel_sm`
// (16 m bytes of shared memory).  Scores are read from L2: another CTA of
// the same launch may have written them (slash_score_dmma_kernel's fused
// form).
template <typename T>
__device__ __noinline__ void rank_problem(const CandSrc<T>& src, int p, int m, int keep_n, int H, int D,
                                          const RopeArgs& rope, const float* scores, long sc_sp,
                                          int hh_neighbor, const SelectOut& out, float* sel_sm) {
  __shared__ int scan_scratch[32];
  float* raw = sel_sm;            // [m]
  float* sel = raw + m;           // [m]
  int* pos = reinterpret_cast<int*>(sel + m);  // [m]
  int* ords = pos + m;                         // [m] the slot order, shared copy
  int* order = out.order + p * out.order_sp;
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    raw[i] = __ldcg(scores + p * sc_sp + i);
    pos[i] = src.pos(p, i);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    float v = raw[i];
    if (hh_neighbor > 0) {
      const int pi = pos[i];
      const int lo = max(0, i - hh_neighbor), hi = min(m - 1, i + hh_neighbor);
      for (int j = lo; j <= hi; ++j) {
        if (j == i) continue;
        if (abs(pos[j] - pi) <= hh_neighbor) v = fmaxf(v, raw[j]);
      }
    }
    sel[i] = v;
  }
  __syncthreads();
  // the boosted scores become total-order keys in place (NaN-proof ranks)
  unsigned* skey = reinterpret_cast<unsigned*>(sel);
  for (int i = threadIdx.x; i < m; i += blockDim.x) skey[i] = order_key(sel[i]);
  __syncthreads();
  const int d = m - keep_n;
  int kbase = 0, dbase = 0;
  for (int i0 = 0; i0 < m; i0 += blockDim.x) {
    const int i = i0 + threadIdx.x;
    int kept = 0;
    if (i < m) {
      const unsigned v = skey[i];
      int rank = 0;
      for (int j = 0; j < m; ++j) {
        const unsigned w = skey[j];
        rank += (w > v) || (w == v && j < i);
      }
      kept = rank < keep_n;
    }
    int tot;
    const int pre = cta_exclusive_scan(kept, scan_scratch, &tot);
    if (i < m) {
      if (kept) {
        const int slot = kbase + pre;
        order[slot] = i;
        ords[slot] = i;
        out.hh_pos[p * out.hh_pos_sp + slot] = pos[i];
      } else {
        const int slot = dbase + (i - i0 - pre);
        order[keep_n + slot] = i;
        ords[keep_n + slot] = i;
        out.mid_pos[p * out.mid_sp + out.w_off + slot] = pos[i];
        if (out.mid_surprise) out.mid_surprise[p * out.mid_sp + out.w_off + slot] = raw[i];
      }
    }
    kbase += tot;
    dbase += min((int)blockDim.x, m - i0) - tot;
  }
  if (threadIdx.x == 0 && out.dem_count) out.dem_count[p] = d;
  __syncthreads();
  // loads are batched ahead of the stores (which the compiler cannot move
  // past: the rows and the block could alias as far as it knows)
  const int lane = threadIdx.x % 32, n = H * D, half = D / 2;
  constexpr int kHB = 8;               // heads per batch of key loads
  constexpr int kPer = 16 / sizeof(T);  // elements per 16-byte chunk
  for (int ds = threadIdx.x / 32; ds < d; ds += blockDim.x / 32) {
    const int jsrc = ords[keep_n + ds];
    const T* kss = src.krow(p, jsrc);
    const T* vss = src.vrow(p, jsrc);
    float* xk = out.xk + p * out.x_sp + (long)ds * n;
    float* xv = out.xv + p * out.x_sp + (long)ds * n;
    const int ps = pos[jsrc];
    for (int f = lane; f < half; f += 32) {
      float c, sn;
      rope_cs(ps, rope.inv_freq[f], rope.scale, &c, &sn);
      for (int h0 = 0; h0 < H; h0 += kHB) {
        float x1[kHB], x2[kHB];
#pragma unroll
        for (int hh = 0; hh < kHB; ++hh)
          if (h0 + hh < H) {
            x1[hh] = load_f<T>(kss + (h0 + hh) * D + f);
            x2[hh] = load_f<T>(kss + (h0 + hh) * D + f + half);
          }
#pragma unroll
        for (int hh = 0; hh < kHB; ++hh)
          if (h0 + hh < H) {
            xk[(h0 + hh) * D + f] = (x1[hh] * c + x2[hh] * sn) / rope.scale_sq;
            xk[(h0 + hh) * D + f + half] = (x2[hh] * c - x1[hh] * sn) / rope.scale_sq;
          }
      }
    }
    const bool vec = (n % (32 * kPer)) == 0 && ((reinterpret_cast<uintptr_t>(vss) |
                                                 reinterpret_cast<uintptr_t>(xv)) & 15) == 0;
    if (vec) {  // 16-byte chunks, two per lane in flight
      const int nch = n / kPer;
      for (int e0 = lane; e0 < nch; e0 += 64) {
        uint4 r0 = make_uint4(0, 0, 0, 0), r1 = r0;
        const bool two = e0 + 32 < nch;
        r0 = reinterpret_cast<const uint4*>(vss)[e0];
        if (two) r1 = reinterpret_cast<const uint4*>(vss)[e0 + 32];
        widen16<T>(r0, xv + e0 * kPer);
        if (two) widen16<T>(r1, xv + (e0 + 32) * kPer);
      }
    } else {
      for (int i = lane; i < n; i += 32) xv[i] = load_f<T>(vss + i);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(512) slash_rank_kernel(CandSrc<T> src, int m, int keep_n, int H,
                                                         int D, RopeArgs rope,
                                                         const float* scores, long sc_sp,
                                                         int hh_neighbor, SelectOut out) {
  extern __shared__ __align__(16) float sel_sm[];
  rank_problem<T>(src, blockIdx.x, m, keep_n, H, D, rope, scores, sc_sp, hh_neighbor, out, sel_sm);
}

constexpr int kMoveWarps = 8;   // rows per CTA of slash_keep_kernel (one warp each)

// Row half of the tier update: slot s < keep_n copies candidate order[s]
// verbatim into the new exact tier.  Grid (ceil(keep_n / 8), P), one warp per
// slot, 16-byte copies.
template <typename T>
__global__ void __launch_bounds__(32 * kMoveWarps) slash_keep_kernel(CandSrc<T> src, int keep_n,
                                                                     int n, SelectOut out) {
  const int p = blockIdx.y;
  const int lane = threadIdx.x % 32;
  const int slot = blockIdx.x * kMoveWarps + threadIdx.x / 32;
  if (slot >= keep_n) return;
  const int jsrc = out.order[p * out.order_sp + slot];
  const T* kss = src.krow(p, jsrc);
  const T* vss = src.vrow(p, jsrc);
  T* ok = reinterpret_cast<T*>(out.hh_k) + p * out.hh_sp + (long)slot * n;
  T* ov = reinterpret_cast<T*>(out.hh_v) + p * out.hh_sp + (long)slot * n;
  const bool aligned = ((reinterpret_cast<uintptr_t>(kss) | reinterpret_cast<uintptr_t>(vss) |
                         reinterpret_cast<uintptr_t>(ok) | reinterpret_cast<uintptr_t>(ov)) &
                        15) == 0;
  const int vec = aligned ? (int)((n * sizeof(T)) / 16) : 0;
  const uint4* ks = reinterpret_cast<const uint4*>(kss);
  const uint4* vs = reinterpret_cast<const uint4*>(vss);
  uint4* kd = reinterpret_cast<uint4*>(ok);
  uint4* vd = reinterpret_cast<uint4*>(ov);
  for (int e = lane; e < vec; e += 32) {
    const uint4 a = ks[e], b = vs[e];
    kd[e] = a;
    vd[e] = b;
  }
  for (int i = vec * (int)(16 / sizeof(T)) + lane; i < n; i += 32) {
    ok[i] = kss[i];
    ov[i] = vss[i];
  }
}

// No-tier absorb: rows [0, b) of `g_k`/`g_v` graduate at positions start + j.
template <typename T>
__global__ void __launch_bounds__(256) gather_block_kernel(const T* g_k, const T* g_v, long g_sp,
                                                           int b, int H, int D, int start,
                                                           RopeArgs rope, float* xk, float* xv,
                                                           long x_sp, int* mid_pos, long mid_sp,
                                                           int w_off) {
  const int p = blockIdx.y;
  const int n = H * D, half = D / 2;
  const long tot = (long)b * (n / 2);
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < tot; e += (long)gridDim.x * blockDim.x) {
    const int slot = (int)(e / (n / 2));
    const int rem = (int)(e % (n / 2));
    const int h = rem / half, f = rem % half;
    const T* kr = g_k + p * g_sp + (long)slot * n + h * D;
    const T* vr = g_v + p * g_sp + (long)slot * n + h * D;
    float c, s;
    rope_cs(start + slot, rope.inv_freq[f], rope.scale, &c, &s);
    const float x1 = load_f<T>(kr + f), x2 = load_f<T>(kr + f + half);
    float* xo = xk + p * x_sp + (long)slot * n + h * D;
    xo[f] = (x1 * c + x2 * s) / rope.scale_sq;
    xo[f + half] = (x2 * c - x1 * s) / rope.scale_sq;
    float* vo = xv + p * x_sp + (long)slot * n + h * D;
    vo[f] = load_f<T>(vr + f);
    vo[f + half] = load_f<T>(vr + f + half);
    if (h == 0 && f == 0) mid_pos[p * mid_sp + w_off + slot] = start + slot;
  }
}

// Evict `f_over` coordinate columns of each problem (ascending surprise with
// ties to the older column under lowrank_surprise; the oldest under fifo),
// then compact C_k, C_v, positions and surprise in place, keeping order.
__global__ void __launch_bounds__(1024) evict_kernel(int W, int f_over, int retention, float* c_k,
                                                     float* c_v, long c_sp, int ld, const int* rk,
                                                     const int* rv, int* mid_pos, float* mid_sur,
                                                     long mid_sp, int* keep_ws, long kw_sp) {
  extern __shared__ __align__(16) unsigned int ev_bits[];  // W bits
  __shared__ float s_bv[32];
  __shared__ int s_bi[32];
  __shared__ int scan_scratch[32];
  const int p = blockIdx.x;
  const int nwords = (W + 31) / 32;
  for (int i = threadIdx.x; i < nwords; i += blockDim.x) ev_bits[i] = 0u;
  __syncthreads();
  const float* sur = mid_sur + p * mid_sp;
  if (retention == KVD_RETENTION_FIFO) {
    for (int i = threadIdx.x; i < f_over; i += blockDim.x) atomicOr(&ev_bits[i / 32], 1u << (i % 32));
    __syncthreads();
  } else {
    const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, nw = blockDim.x / 32;
    for (int it = 0; it < f_over; ++it) {
      float bv = FLT_MAX;
      int bi = 0x7fffffff;
      for (int i = threadIdx.x; i < W; i += blockDim.x) {
        if (ev_bits[i / 32] & (1u << (i % 32))) continue;
        const float v = sur[i];
        if (v < bv || (v == bv && i < bi)) { bv = v; bi = i; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov < bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) { s_bv[warp] = bv; s_bi[warp] = bi; }
      __syncthreads();
      if (threadIdx.x == 0) {
        float v = s_bv[0];
        int ix = s_bi[0];
        for (int w2 = 1; w2 < nw; ++w2)
          if (s_bv[w2] < v || (s_bv[w2] == v && s_bi[w2] < ix)) { v = s_bv[w2]; ix = s_bi[w2]; }
        if (ix < W) ev_bits[ix / 32] |= 1u << (ix % 32);
      }
      __syncthreads();
    }
  }
  // kept index list
  int* keep = keep_ws + p * kw_sp;
  int base = 0;
  for (int i0 = 0; i0 < W; i0 += blockDim.x) {
    const int i = i0 + threadIdx.x;
    const int kept = (i < W) && !(ev_bits[i / 32] & (1u << (i % 32)));
    int tot;
    const int pre = cta_exclusive_scan(kept, scan_scratch, &tot);
    if (kept) keep[base + pre] = i;
    base += tot;
    __syncthreads();
  }
  const int Wk = W - f_over;
  // in-place compaction, chunk by chunk in increasing destination order
  const int r = max(rk[p], rv[p]);
  constexpr int kChunk = 4;  // token rows per chunk per pass (x r floats x 2 streams)
  float* ck = c_k + p * c_sp;
  float* cv = c_v + p * c_sp;
  int* pos = mid_pos + p * mid_sp;
  float* su = mid_sur ? mid_sur + p * mid_sp : nullptr;
  float* stage = reinterpret_cast<float*>(ev_bits + nwords + 1);  // [kChunk*? ] reuse smem tail
  const int rows_per = max(1, (int)(blockDim.x / max(r, 1)));
  const int chunk = min(1024, kChunk * rows_per);
  for (int d0 = 0; d0 < Wk; d0 += chunk) {
    const int cnt = min(chunk, Wk - d0);
    // stage k, v rows, position, surprise
    for (int e = threadIdx.x; e < cnt * r; e += blockDim.x) {
      const int t = e / r, c = e % r;
      const int s = keep[d0 + t];
      stage[e] = ck[(long)s * ld + c];
      stage[cnt * r + e] = cv[(long)s * ld + c];
    }
    int spos = 0;
    float ssur = 0.f;
    const bool own = threadIdx.x < cnt;
    if (own) {
      const int s = keep[d0 + threadIdx.x];
      spos = pos[s];
      if (su) ssur = su[s];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < cnt * r; e += blockDim.x) {
      const int t = e / r, c = e % r;
      ck[(long)(d0 + t) * ld + c] = stage[e];
      cv[(long)(d0 + t) * ld + c] = stage[cnt * r + e];
    }
    if (own) {
      pos[d0 + threadIdx.x] = spos;
      if (su) su[d0 + threadIdx.x] = ssur;
    }
    __syncthreads();
  }
}

}  // namespace kvd

// ---------------------------------------------------------------- host glue
namespace kvd_host {
using namespace kvd;

template <typename T>
int launch_slash_score(const CandSrc<T>& src, int P, int m, int H, int D, RopeArgs rope,
                       const float* u, long u_sp, int ld, const int* rr, float* scores, long sc_sp,
                       cudaStream_t stream, const RankArgs* fuse, bool* fused) {
  if (fused) *fused = false;
  if (m <= 0) return KVD_OK;
  if (ld > 8 * kScoreMaxQ) {
    set_error("slash score: rank %d exceeds %d", ld, 8 * kScoreMaxQ);
    return KVD_ERR_ARG;
  }
  const int half = D / 2;
  const long n = (long)H * D;
  const long dsmem_l = 8L * (3 * kScT + 8 * 32 * 4) + 4L * (kScT * (n + 4) + n * 40 + kScT * half * 2) +
                       (long)sizeof(T) * kScT * n;
  // cp.async staging: 16-byte rows and bases
  const bool al = (n * (long)sizeof(T)) % 16 == 0 && ld % 4 == 0 && u_sp % 4 == 0 &&
                  reinterpret_cast<uintptr_t>(u) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(src.g_k) % 16 == 0 &&
                  (src.hh_len == 0 || reinterpret_cast<uintptr_t>(src.hh_k) % 16 == 0) &&
                  (src.hh_sp * (long)sizeof(T)) % 16 == 0 && (src.g_sp * (long)sizeof(T)) % 16 == 0;
  if (ld <= 32 && D % 8 == 0 && n % 16 == 0 && al && dsmem_l <= 200 * 1024) {
    // the fused ranking reuses the kernel's shared memory (16 m bytes)
    const bool fuse_ok = fuse && fuse->done && 16L * m <= dsmem_l && fuse->out.order_sp >= m;
    RankArgs rk{};
    if (fuse_ok) rk = *fuse;
    const int dsmem = (int)dsmem_l;
    if (int rc = ensure_smem((const void*)slash_score_dmma_kernel<T>, dsmem, "slash_score_kernel")) return rc;
    {
      KTimerScope kts_("slash_score_kernel", stream);
      slash_score_dmma_kernel<T><<<dim3((m + kScT - 1) / kScT, P), kScThreads, dsmem, stream>>>(
          src, m, H, D, rope, u, u_sp, ld, rr, scores, sc_sp, rk);
    }
    if (fused) *fused = fuse_ok;
    return check_launch("slash_score_kernel");
  }
  // ranks past 32, or a basis too large for shared memory whole: the basis
  // streams through in feature chunks (slash_score_dmma_wide_kernel)
  const long wsm = sw_smem_bytes((int)n, D, ld);
  const bool wal = ld % 4 == 0 && u_sp % 4 == 0 && reinterpret_cast<uintptr_t>(u) % 16 == 0;
  if (ld <= 32 * kSwMaxCT && n % kSwF == 0 && D % 2 == 0 && wal && wsm <= device_smem_optin()) {
    const bool fuse_ok = fuse && fuse->done && 16L * m <= wsm && fuse->out.order_sp >= m;
    RankArgs rk{};
    if (fuse_ok) rk = *fuse;
    if (int rc = ensure_smem((const void*)slash_score_dmma_wide_kernel<T>, (int)wsm, "slash_score_kernel"))
      return rc;
    {
      KTimerScope kts_("slash_score_kernel", stream);
      slash_score_dmma_wide_kernel<T><<<dim3((m + kSwT - 1) / kSwT, P), kSwThreads, (int)wsm, stream>>>(
          src, m, H, D, rope, u, u_sp, ld, rr, scores, sc_sp, rk);
    }
    if (fused) *fused = fuse_ok;
    return check_launch("slash_score_kernel");
  }
  const int smem = 4 * (kScoreTile * half * 2 + kScoreTile * D + D * ld);
  dim3 grid((m + kScoreTile - 1) / kScoreTile, P);
  auto go = [&](auto kern) -> int {
    if (int rc = ensure_smem((const void*)kern, smem, "slash_score_kernel")) return rc;
    KTimerScope kts_("slash_score_kernel", stream);
    kern<<<grid, 256, smem, stream>>>(src, m, H, D, rope, u, u_sp, ld, rr, scores, sc_sp);
    return KVD_OK;
  };
  int rc;
  if (ld <= 32) rc = go(slash_score_kernel<T, 4>);
  else if (ld <= 64) rc = go(slash_score_kernel<T, 8>);
  else if (ld <= 128) rc = go(slash_score_kernel<T, 16>);
  else rc = go(slash_score_kernel<T, 24>);
  if (rc) return rc;
  return check_launch("slash_score_kernel");
}

template <typename T>
int launch_slash_select(const CandSrc<T>& src, int P, int m, int keep_n, int H, int D,
                        RopeArgs rope, const float* scores, long sc_sp, int hh_neighbor,
                        const SelectOut& out, cudaStream_t stream) {
  if (m <= 0) return KVD_OK;
  if (out.order_sp < m) {
    set_error("slash select: order stride %ld < pool %d", out.order_sp, m);
    return KVD_ERR_ARG;
  }
  const int smem = 4 * 4 * m;
  if (int rc = ensure_smem((const void*)slash_rank_kernel<T>, smem, "slash_rank_kernel")) return rc;
  {
    KTimerScope kts_("slash_rank_kernel", stream);
    slash_rank_kernel<T><<<P, 512, smem, stream>>>(src, m, keep_n, H, D, rope, scores, sc_sp,
                                                   hh_neighbor, out);
  }
  return check_launch("slash_rank_kernel");
}

template <typename T>
int launch_slash_keep(const CandSrc<T>& src, int P, int keep_n, int n, const SelectOut& out,
                      cudaStream_t stream) {
  if (keep_n <= 0) return KVD_OK;
  {
    KTimerScope kts_("slash_keep_kernel", stream);
    dim3 grid((keep_n + kMoveWarps - 1) / kMoveWarps, P);
    slash_keep_kernel<T><<<grid, 32 * kMoveWarps, 0, stream>>>(src, keep_n, n, out);
  }
  return check_launch("slash_keep_kernel");
}

template <typename T>
int launch_gather_block(const T* g_k, const T* g_v, long g_sp, int P, int b, int H, int D,
                        int start, RopeArgs rope, float* xk, float* xv, long x_sp, int* mid_pos,
                        long mid_sp, int w_off, cudaStream_t stream) {
  if (b <= 0) return KVD_OK;
  const long tot = (long)b * H * D / 2;
  const long nblk = (tot + 255) / 256;
  const int blocks = (int)(nblk < 1024 ? nblk : 1024);
  dim3 grid(blocks, P);
  {
    KTimerScope kts_("gather_block_kernel", stream);
    gather_block_kernel<T><<<grid, 256, 0, stream>>>(g_k, g_v, g_sp, b, H, D, start, rope, xk, xv,
                                                   x_sp, mid_pos, mid_sp, w_off);
  }
  return check_launch("gather_block_kernel");
}

int launch_evict(int P, int W, int f_over, int retention, float* c_k, float* c_v, long c_sp, int ld,
                 const int* rk, const int* rv, int* mid_pos, float* mid_sur, long mid_sp,
                 int* keep_ws, long kw_sp, cudaStream_t stream) {
  if (f_over <= 0) return KVD_OK;
  const int nwords = (W + 31) / 32;
  const int rows_per = 1024 / 1;  // upper bound for staging (r >= 1)
  (void)rows_per;
  // stage needs cnt * r * 2 floats with cnt*r <= 4*1024 -> 32 KB
  const int smem = 4 * (nwords + 1) + 4 * 2 * 4 * 1024 + 64;
  if (smem > 227 * 1024) {
    set_error("evict: coordinate count %d too large for the in-block bitmap", W);
    return KVD_ERR_ARG;
  }
  if (int rc = ensure_smem((const void*)evict_kernel, smem, "evict_kernel")) return rc;
  {
    KTimerScope kts_("evict_kernel", stream);
    evict_kernel<<<P, 1024, smem, stream>>>(W, f_over, retention, c_k, c_v, c_sp, ld, rk, rv, mid_pos,
                                          mid_sur, mid_sp, keep_ws, kw_sp);
  }
  return check_launch("evict_kernel");
}

#define KVD_INST(T)                                                                              \
  template int launch_slash_score<T>(const CandSrc<T>&, int, int, int, int, RopeArgs,            \
                                     const float*, long, int, const int*, float*, long,          \
                                     cudaStream_t, const RankArgs*, bool*);                      \
  template int launch_slash_select<T>(const CandSrc<T>&, int, int, int, int, int, RopeArgs,      \
                                      const float*, long, int, const SelectOut&, cudaStream_t);  \
  template int launch_slash_keep<T>(const CandSrc<T>&, int, int, int, const SelectOut&,          \
                                    cudaStream_t);                                               \
  template int launch_gather_block<T>(const T*, const T*, long, int, int, int, int, int,         \
                                      RopeArgs, float*, float*, long, int*, long, int,           \
                                      cudaStream_t);
KVD_INST(float)
KVD_INST(__nv_bfloat16)
#undef KVD_INST

}  // namespace kvd_host
