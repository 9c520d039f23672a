// Batched augmented rank-adaptive BUG step and the coordinate carry (sm_100a).
//
// Restates src/kvdlra/integrators/streaming_torch.py:82-189 for a batch of
// independent problems (one CTA per problem x stream):
//   a = U^T X ; R = X - U a ; a2 = U^T R ; R -= U a2 ; a += a2   (fp32 FFMA,
//     K-split with fp64 sums of the split partials)
//   SVD of R (n x b) -> singular values s, left vectors q_j, right vectors
//     V: up to 128 columns from the fp64 Gram R^T R = T^T T (Cholesky) and a
//     one-sided Jacobi on T's rows (rotated rows V S, q_j = R v_j / s_j; the
//     pre-fill blocks refine with a seeded Jacobi on R V), wider blocks by a
//     one-sided Jacobi on R itself; admit s > 100 eps |X|_F, at most n - r
//   one-sided Jacobi on B^T, B = [[diag(sigma), a], [0, diag(s_m) V_m^T]]
//     ((r+m) x (r+b)):  B^T W = [sigma'_c z_c]  -> W = left singular vectors
//     of B (u_loc), sigma' its singular values
//   U_new = [U | Q] W[:, top keep], rot = W[:r, top keep]^T, and the block's
//     coordinates U_new^T X = W^T B[:, r:], read off the rotated B^T.
// U_new is then brought back to orthonormal columns by one Newton-Schulz
// step U <- U (I - (U^T U - I)/2) with an fp64-summed Gram, so rounding and
// the Jacobi stopping tolerance cannot accumulate over a long stream.
// One-sided (Hestenes) Jacobi never forms a Gram matrix, so it keeps the
// relative accuracy of a direct SVD; all rotations of a round touch disjoint
// columns, so a round costs one barrier.
#include <stdio.h>

#include <cfloat>
#include <mutex>

#include "kernels.cuh"

namespace kvd {

__host__ __device__ inline long align16(long x) { return (x + 15) & ~15L; }

constexpr int kStepThreads = 512;
constexpr int kStepMiscBytes = 1024;   // fp64 reduction scratch
constexpr int kPartFloats = 8192;      // K-split partials: 16 warps x 32 lanes x 16
constexpr int kMaxGramB = 128;         // widest block the Gram + Cholesky residual SVD takes

// One-sided (Hestenes) Jacobi on augmented columns.  Column c of X (at
// X + c*ldx) holds the data in rows [0, len), zeros in [len, voff) and, from
// row voff (a multiple of 4), the accumulated rotations V[:, c] (cols rows,
// initialised to e_c here), so one pass rotates data and V together:
// X[:, :len] V = orthogonal columns, V = X[voff:voff+cols, :].
// Round-robin ordering; each column pair is handled by a group of G lanes
// that keeps the pair in registers as 4-float units: lane gl holds units
// gl, gl + G, ..., NU of them, so a group reads and writes contiguous
// 16-byte runs.  The column pitch covers the whole tile (ldx >= 4 G NU, rows
// past the rotations zeroed), so the tile needs no bounds tests; shapes that
// do not fit a tile stream the columns from shared memory (NU = 0).  Only
// the warps that own pairs take part: they leave every round on a named
// barrier of their own, while the other warps return at once and wait at
// the caller's next __syncthreads.  The rotation zeroes the pair's inner
// product (Golub & Van Loan sec. 8.6.3); its parameters come from the fast
// reciprocal square root and are renormalised by one Newton step so
// c^2 + s^2 = 1 to rounding (an inexact angle only slows convergence).  A
// lane sums its data values in fp32 and the group reduces in ACC.
// inv_scale2 is 1 / (squared Frobenius scale of the problem).  Returns the
// sweeps taken (max_sweeps when not converged) in the participating
// threads.  Callers must __syncthreads() before reading X.
constexpr double kJacobiFloor = 1e-30;
constexpr int kJacobiBarrier = 1;  // named barrier id (0 is __syncthreads)
// A sweep that rotated no pair whose cosine exceeded this ends the iteration:
// Jacobi converges quadratically, so the next sweep's cosines would be
// ~1e-6, at the stopping tolerance, and the confirming sweep is skipped.
constexpr float kJacobiQuadStop = 1e-3f;

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// The same barrier, returning whether `pred` held on any participating thread.
__device__ __forceinline__ bool named_barrier_or(int id, int nthreads, bool pred) {
  int any;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n"
      " selp.s32 %0, 1, 0, q;\n}"
      : "=r"(any)
      : "r"((int)pred), "r"(id), "r"(nthreads)
      : "memory");
  return any != 0;
}

// The rotation that zeroes a pair's inner product g (d = beta - alpha, g2 =
// 2 g), the smaller of the two angles (|theta| <= pi/4): with rho = 1 /
// sqrt(d^2 + g2^2), cos 2theta = |d| rho and sin 2theta = sgn(d) g2 rho, so
// c = sqrt(x) and s = sin 2theta / (2 c) with x = (1 + cos 2theta) / 2, both
// from one reciprocal square root of x.  A pair whose d and g2 are both
// tiny is rescaled first (the angle depends only on their ratio) so the
// squares cannot underflow.  One Newton step renormalises c^2 + s^2 to 1.
__device__ __forceinline__ void jacobi_rotation(float d, float g2, float& c, float& s) {
  const float sc = fmaxf(fabsf(d), fabsf(g2)) < 1e-15f ? 1e20f : 1.f;
  d *= sc;
  g2 *= sc;
  const float rho = rsqrtf(fmaf(d, d, g2 * g2));
  const float x = fmaf(0.5f * fabsf(d), rho, 0.5f);
  const float ic = rsqrtf(x);
  c = x * ic;
  s = copysignf(0.5f, d) * g2 * rho * ic;
  const float f = fmaf(-0.5f, fmaf(c, c, s * s), 1.5f);
  c *= f;
  s *= f;
}

// Register tile of the one-sided Jacobi for `cols` columns of `nut` 4-float
// units: lanes per pair G (about eight warps' worth of pairs, at most 9 units
// per lane) and units per lane NU (0 = stream from shared memory).  The
// same choice sizes the column pitch on the host.
// The instantiated tiles: fp64 sums (long residual columns) G in {16, 32}
// with NU in {2, 3, 5, 9}; fp32 sums (the core) G in {4, 8, 16}, NU in
// {2, 3, 4, 5, 6, 9}.  0 = none fits.
__host__ __device__ inline int jacobi_nu(int g, int need, bool dbl) {
  if (!(dbl ? (g == 16 || g == 32) : (g == 4 || g == 8 || g == 16))) return 0;
  if (need <= 2) return 2;
  if (need <= 3) return 3;
  if (!dbl && need <= 4) return 4;
  if (need <= 5) return 5;
  if (!dbl && need <= 6) return 6;
  if (need <= 9) return 9;
  return 0;
}

__host__ __device__ inline void jacobi_tile(int nut, int cols, bool dbl, int* G, int* NU,
                                            int gcap = 32) {
  const int half = (cols + 1) / 2;
  int g0 = gcap;
  while (g0 > 4 && half * g0 > 256) g0 >>= 1;
  while (g0 < 32 && g0 * 9 < nut) g0 <<= 1;
  if (dbl && g0 < 16) g0 = 16;  // fp64 tiles are instantiated for groups of 16 and 32
  // the widest instantiated group up to g0 whose tile is not padded far past
  // the column (small problems would waste shared memory), else the least
  // padded instantiated one, else streaming
  int gbest = 0, nubest = 0, gany = 0, nuany = 0;
  for (int g = g0; g >= 4; g >>= 1) {
    const int nu = jacobi_nu(g, (nut + g - 1) / g, dbl);
    if (!nu) continue;
    if (!gany || g * nu < gany * nuany) { gany = g; nuany = nu; }  // least padding
    if (4 * g * nu <= 5 * nut + 8) { gbest = g; nubest = nu; break; }
  }
  if (!gbest) { gbest = gany; nubest = nuany; }
  *G = nubest ? gbest : 32;
  *NU = nubest;
}
// Column pitch (floats) a Jacobi on `rows` augmented rows x `cols` columns needs.
__host__ __device__ inline int jacobi_pitch(int rows, int cols, bool dbl, int gcap = 32) {
  int g, nu;
  jacobi_tile((rows + 3) / 4, cols, dbl, &g, &nu, gcap);
  const int r4 = (rows + 3) & ~3;
  return nu ? (r4 > 4 * g * nu ? r4 : 4 * g * nu) : r4;
}

template <int G, int NU, typename ACC>
static __device__ __forceinline__ int cta_hestenes(float* X, int len, int voff, int cols, int ldx,
                                                   float tol, int max_sweeps, double inv_scale2,
                                                   bool accum, bool seeded) {
  const int tid = threadIdx.x, nthr = blockDim.x, warp = tid / 32, lane = tid % 32;
  const int gid = tid / G, gl = tid % G;
  const int vend = voff + (accum ? ((cols + 3) & ~3) : 0);
  const int rows = NU > 0 ? 4 * G * NU : vend;  // rows the tile touches; [len, rows) zeroed
  for (long e = tid; e < (long)cols * (rows - len); e += nthr) {
    const int c = (int)(e / (rows - len)), k = len + (int)(e % (rows - len));
    if (seeded && k >= voff && k < voff + cols) continue;  // the caller's starting rotations
    X[(long)c * ldx + k] = (accum && k - voff == c) ? 1.f : 0.f;
  }
  __syncthreads();
  if (cols <= 1) return 0;
  const int np = cols + (cols & 1);
  const int half = np / 2;
  const int groups = nthr / G;
  const int aw = min(nthr / 32, (half * G + 31) / 32);  // warps that own pairs
  if (warp >= aw) return 0;
  const int nbar = aw * 32;
  const int nud = voff / 4;  // data units
  const ACC tol2 = (ACC)tol * (ACC)tol;
  const ACC is2 = (ACC)inv_scale2;
  int sweep = 0;
  for (; sweep < max_sweeps; ++sweep) {
    // a pair rotated this sweep with a cosine above kJacobiQuadStop (which
    // also means some pair rotated at all); OR-reduced by the sweep's last barrier
    bool big = false;
    bool again = false;
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
        float4 up[NU > 0 ? NU : 1], uq[NU > 0 ? NU : 1];
        ACC al, be, ga;
        if constexpr (NU > 0) {
          float fal = 0.f, fbe = 0.f, fga = 0.f;
#pragma unroll
          for (int t = 0; t < NU; ++t) {
            const int u = gl + t * G;
            up[t] = reinterpret_cast<const float4*>(xp)[u];
            uq[t] = reinterpret_cast<const float4*>(xq)[u];
            if (u < nud) {
              fal = fmaf(up[t].x, up[t].x, fal); fal = fmaf(up[t].y, up[t].y, fal);
              fal = fmaf(up[t].z, up[t].z, fal); fal = fmaf(up[t].w, up[t].w, fal);
              fbe = fmaf(uq[t].x, uq[t].x, fbe); fbe = fmaf(uq[t].y, uq[t].y, fbe);
              fbe = fmaf(uq[t].z, uq[t].z, fbe); fbe = fmaf(uq[t].w, uq[t].w, fbe);
              fga = fmaf(up[t].x, uq[t].x, fga); fga = fmaf(up[t].y, uq[t].y, fga);
              fga = fmaf(up[t].z, uq[t].z, fga); fga = fmaf(up[t].w, uq[t].w, fga);
            }
          }
          al = fal; be = fbe; ga = fga;
        } else {  // stream the columns from shared memory twice
          al = 0; be = 0; ga = 0;
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
        // the pair's Gram relative to the problem's scale: a column below
        // kJacobiFloor of it is numerically null and is left alone, which
        // also keeps the fp32 rotation parameters clear of underflow
        al *= is2;
        be *= is2;
        ga *= is2;
        const bool live = active && al > (ACC)kJacobiFloor && be > (ACC)kJacobiFloor;
        if (!live || ga * ga <= tol2 * al * be) continue;
        float c, s;
        jacobi_rotation((float)be - (float)al, 2.f * (float)ga, c, s);
        if constexpr (NU > 0) {
#pragma unroll
          for (int t2 = 0; t2 < NU; ++t2) {
            const int u = gl + t2 * G;
            const float4 a = up[t2], bq = uq[t2];
            reinterpret_cast<float4*>(xp)[u] = make_float4(c * a.x - s * bq.x, c * a.y - s * bq.y,
                                                           c * a.z - s * bq.z, c * a.w - s * bq.w);
            reinterpret_cast<float4*>(xq)[u] = make_float4(s * a.x + c * bq.x, s * a.y + c * bq.y,
                                                           s * a.z + c * bq.z, s * a.w + c * bq.w);
          }
        } else {
          for (int e = gl; e < vend; e += G) {
            const float u = xp[e], v = xq[e];
            xp[e] = c * u - s * v;
            xq[e] = s * u + c * v;
          }
        }
        big = big || ga * ga > (ACC)(kJacobiQuadStop * kJacobiQuadStop) * al * be;
      }
      if (k < np - 2) named_barrier(kJacobiBarrier, nbar);
      else again = named_barrier_or(kJacobiBarrier, nbar, big);
    }
    if (!again) break;
  }
  return sweep;
}

// Warp w's k slice [w n/8, (w+1) n/8) of the fp64 Gram R^T R of the b <= 16
// columns of R (pitch n, n % 32 == 0) as 2 x 2 tiles of m8n8k4 products; the
// A (= R^T) and B (= R) fragments of a k-step are the same two values per
// lane.  Writes gpart[(w * 4 + tile) * 64 + row * 8 + col].
static __device__ __forceinline__ void warp_gram16_slice(const float* Rm, int n, int b, int w,
                                                      double* gpart) {
  const int lane = threadIdx.x & 31, grp = lane >> 2, tig = lane & 3;
  double c00 = 0.0, c01 = 0.0, c10 = 0.0, c11 = 0.0, c20 = 0.0, c21 = 0.0, c30 = 0.0, c31 = 0.0;
  const int kw = n / 8, k_begin = w * kw;
  const float* r0 = Rm + (long)grp * n + tig;
  const float* r1 = Rm + (long)(8 + grp) * n + tig;
  const bool h0 = grp < b, h1 = 8 + grp < b;
#pragma unroll 4
  for (int k0 = k_begin; k0 < k_begin + kw; k0 += 4) {
    const double x0 = h0 ? (double)r0[k0] : 0.0, x1 = h1 ? (double)r1[k0] : 0.0;
    dmma_8x8x4(c00, c01, x0, x0);
    dmma_8x8x4(c10, c11, x0, x1);
    dmma_8x8x4(c20, c21, x1, x0);
    dmma_8x8x4(c30, c31, x1, x1);
  }
  double* o = gpart + (long)w * 256 + grp * 8 + 2 * tig;
  o[0] = c00; o[1] = c01;
  o[64] = c10; o[65] = c11;
  o[128] = c20; o[129] = c21;
  o[192] = c30; o[193] = c31;
}

// Right-looking Cholesky of the b x b (b <= 16) fp64 Gram G (pitch ldg) by
// one warp in registers: lane j holds column j; each step broadcasts the
// pivot column by shuffles (a pivot at or below 1e-14 of the trace is taken
// as null: its column of the factor is zero).  Writes L's columns (the rows
// of T = L^T) into the columns of Tm (column c, rows k >= c; zero above).
// Call from warp 0 only.
static __device__ __noinline__ void warp_cholesky16(const double* G, int ldg, int b, float* Tm,
                                                    int ldr) {
  constexpr unsigned kAll = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  double a[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = (lane < b && i < b) ? G[i * ldg + lane] : 0.0;
  const double trace = warp_sum(lane < b ? G[lane * ldg + lane] : 0.0);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (j < b) {  // (no early exit: the loop must unroll for a[] to stay in registers)
    const double piv = __shfl_sync(kAll, a[j], j);
    const double t = piv > 1e-14 * trace ? sqrt(piv) : 0.0;
    const double rt = t > 0.0 ? 1.0 / t : 0.0;
    if (lane == j) {
#pragma unroll
      for (int i = j + 1; i < 16; ++i) a[i] *= rt;
      a[j] = t;
    }
    double l[16];
    double lk = 0.0;  // l[lane]: this lane's entry of the pivot column
#pragma unroll
    for (int i = j + 1; i < 16; ++i) {
      l[i] = __shfl_sync(kAll, a[i], j);
      if (i == lane) lk = l[i];
    }
    if (lane > j) {
#pragma unroll
      for (int i = j + 1; i < 16; ++i) a[i] = fma(-l[i], lk, a[i]);
    }
    }
  }
  if (lane < b) {  // lane c holds column c of L: L[k][c] for k >= c
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (k < b) Tm[lane * ldr + k] = k >= lane ? (float)a[k] : 0.f;
  }
  __syncwarp();
}

// One-sided Jacobi for up to 16 columns of at most 4 RK augmented rows (data
// rows [0, len), zero to voff, rotations accumulated in rows [voff,
// voff + cols)), run by one warp entirely in registers.  Slot i (lanes
// 4i .. 4i+3) holds the pair (top, bottom); lane 4i + g holds rows g + 4k
// (k < RK) of both.  Rounds follow the circle method (position 0 fixed, the others
// advancing one position per round, so np - 1 rounds meet every pair), the
// columns moving between slots by warp shuffles instead of through shared
// memory.  Rotation, tolerance, null floor and early stop are cta_hestenes's.
// Call from warp 0 only; writes the columns back to X and returns the sweeps.
template <int RK>
static __device__ __noinline__ int warp_hestenes16(float* X, int len, int voff, int cols, int ldx,
                                                   float tol, int max_sweeps, double inv_scale2) {
  constexpr unsigned kAll = 0xffffffffu;
  const int lane = threadIdx.x & 31, g = lane & 3, slot = lane >> 2;
  if (cols <= 1) {  // nothing to rotate: the identity below the data
    for (int c = 0; c < cols; ++c)
      for (int row = len + lane; row < voff + cols; row += 32)
        X[(long)c * ldx + row] = (row - voff == c) ? 1.f : 0.f;
    __syncwarp();
    return 0;
  }
  const int np = cols + (cols & 1), half = np / 2;
  int ti = slot < half ? slot : np, bi = slot < half ? np - 1 - slot : np;  // column indices
  float tp[RK], bt[RK];
  auto value = [&](int c, int row) -> float {
    if (c >= cols) return 0.f;
    if (row < len) return X[(long)c * ldx + row];
    return (row - voff == c) ? 1.f : 0.f;
  };
#pragma unroll
  for (int k = 0; k < RK; ++k) {
    tp[k] = value(ti, g + 4 * k);
    bt[k] = value(bi, g + 4 * k);
  }
  __syncwarp();
  const float tol2 = tol * tol, is2 = (float)inv_scale2;
  int sweep = 0;
  for (; sweep < max_sweeps; ++sweep) {
    bool big = false;
    for (int rd = 0; rd < np - 1; ++rd) {
      float al = 0.f, be = 0.f, ga = 0.f;
#pragma unroll
      for (int k = 0; k < RK; ++k)
        if (g + 4 * k < voff) {
          al = fmaf(tp[k], tp[k], al);
          be = fmaf(bt[k], bt[k], be);
          ga = fmaf(tp[k], bt[k], ga);
        }
      al += __shfl_xor_sync(kAll, al, 1); be += __shfl_xor_sync(kAll, be, 1); ga += __shfl_xor_sync(kAll, ga, 1);
      al += __shfl_xor_sync(kAll, al, 2); be += __shfl_xor_sync(kAll, be, 2); ga += __shfl_xor_sync(kAll, ga, 2);
      al *= is2;
      be *= is2;
      ga *= is2;
      const bool live = slot < half && al > kJacobiFloor && be > kJacobiFloor;
      if (live && ga * ga > tol2 * al * be) {
        float c, sn;
        jacobi_rotation(be - al, 2.f * ga, c, sn);
#pragma unroll
        for (int k = 0; k < RK; ++k) {
          const float a = tp[k], bq = bt[k];
          tp[k] = c * a - sn * bq;
          bt[k] = sn * a + c * bq;
        }
        big = big || ga * ga > kJacobiQuadStop * kJacobiQuadStop * al * be;
      }
      // advance: top of slot i <- top of i-1 (slot 1 <- bottom of 0, slot 0 fixed);
      // bottom of slot i <- bottom of i+1 (the last slot's bottom <- its own top);
      // a single pair never moves
      const bool first = slot == 0, second = slot == 1, last = slot == half - 1;
      if (half > 1) {
#pragma unroll
      for (int k = 0; k < RK; ++k) {
        const float t_prev = __shfl_up_sync(kAll, tp[k], 4);
        const float b_prev = __shfl_up_sync(kAll, bt[k], 4);
        const float b_next = __shfl_down_sync(kAll, bt[k], 4);
        const float nt = first ? tp[k] : (second ? b_prev : t_prev);
        bt[k] = last ? tp[k] : b_next;
        tp[k] = nt;
      }
      {
        const int t_prev = __shfl_up_sync(kAll, ti, 4), b_prev = __shfl_up_sync(kAll, bi, 4);
        const int b_next = __shfl_down_sync(kAll, bi, 4);
        const int nt = first ? ti : (second ? b_prev : t_prev);
        bi = last ? ti : b_next;
        ti = nt;
      }
      }
    }
    if (!__any_sync(kAll, big)) break;
  }
  if (slot < half) {
#pragma unroll
    for (int k = 0; k < RK; ++k) {
      const int row = g + 4 * k;
      if (row < voff + cols) {
        if (ti < cols) X[(long)ti * ldx + row] = tp[k];
        if (bi < cols) X[(long)bi * ldx + row] = bt[k];
      }
    }
  }
  __syncwarp();
  return sweep;
}

// Dispatch to the register tile jacobi_tile picks (groups of at most `gcap`
// lanes) when X is 16-byte aligned and the pitch covers it, else stream.
// accum = false: no rotations are accumulated (rows [len, voff) are padding);
// seeded = true: rows [voff, voff + cols) already hold starting rotations.
template <typename ACC>
static __device__ __forceinline__ int cta_hestenes_any(float* X, int len, int voff, int cols,
                                                       int ldx, float tol, int max_sweeps,
                                                       double inv_scale2, bool accum = true,
                                                       int gcap = 32, bool seeded = false) {
  const int nut = (voff + (accum ? ((cols + 3) & ~3) : 0)) / 4;
  int G, NU;
  jacobi_tile(nut, cols, sizeof(ACC) == 8, &G, &NU, gcap);
  const bool fits = NU > 0 && (reinterpret_cast<unsigned long>(X) & 15) == 0 && ldx % 4 == 0 &&
                    ldx >= 4 * G * NU;
  if (fits) {
#define KVD_HJ(GG, UU)                                                                       \
    if (G == GG && NU == UU)                                                                 \
      return cta_hestenes<GG, UU, ACC>(X, len, voff, cols, ldx, tol, max_sweeps, inv_scale2, accum, seeded);
    if constexpr (sizeof(ACC) == 8) {
      KVD_HJ(16, 2) KVD_HJ(16, 3) KVD_HJ(16, 5) KVD_HJ(16, 9)
      KVD_HJ(32, 2) KVD_HJ(32, 3) KVD_HJ(32, 5) KVD_HJ(32, 9)
    } else {
      KVD_HJ(4, 2) KVD_HJ(4, 3) KVD_HJ(4, 4) KVD_HJ(4, 5) KVD_HJ(4, 6) KVD_HJ(4, 9)
      KVD_HJ(8, 2) KVD_HJ(8, 3) KVD_HJ(8, 4) KVD_HJ(8, 5) KVD_HJ(8, 6) KVD_HJ(8, 9)
      KVD_HJ(16, 2) KVD_HJ(16, 3) KVD_HJ(16, 4) KVD_HJ(16, 5) KVD_HJ(16, 6) KVD_HJ(16, 9)
    }
#undef KVD_HJ
  }
  return cta_hestenes<32, 0, ACC>(X, len, voff, cols, ldx, tol, max_sweeps, inv_scale2, accum, seeded);
}

// Block-ordered one-sided Jacobi for the core (fp32 sums, rotations
// accumulated from row voff as in cta_hestenes), with the columns held in
// registers between barriers.  Columns form blocks of four; a block round
// gives warp w two blocks A, B (the circle method over blocks) and group j
// of eight lanes the column pair (A_j on top, B_j below), lane gl holding the
// 16-byte units gl + 8 t (t < NU) of both, of which the first NUD per lane
// can hold data rows.  The warp then runs, without leaving registers: in
// the first block round of a sweep the full circle over its eight columns
// (seven rounds, every pair inside A, inside B and across), in the others
// the four cross rounds (A_j against B_(j+t), the bottoms passed on by warp
// shuffles).  A sweep therefore meets every pair once in the same 47 rounds
// (48 columns) as the cyclic order, but the columns cross shared memory and
// a named barrier only once per block round (11 times a sweep instead of
// 47).  The rotation, the tolerance, the null floor and the quadratic stop
// are cta_hestenes's; the stop slides: the iteration ends once nbp - 1
// consecutive block rounds (each pair once) rotated no pair with a cosine
// above kJacobiQuadStop, wherever in the sweep that window starts.  Needs X
// 16-byte aligned and ldx % 4 == 0; with more block pairs than warps, warp w
// takes pairs w, w + warps, ... of each block round (they are disjoint);
// returns the sweeps taken less one (max_sweeps when not converged).
constexpr int kBlkLanes = 8;
// ACCUM = false: nothing accumulated (rows [len, voff) are padding, zeroed).
template <int NU, int NUD, bool ACCUM = true>
static __device__ __noinline__ int cta_block_hestenes(float* X, int len, int voff, int cols, int ldx,
                                                      float tol, int max_sweeps, double inv_scale2) {
  constexpr int G = kBlkLanes, P = 32 / G;
  constexpr unsigned kAll = 0xffffffffu;
  const int tid = threadIdx.x, nthr = blockDim.x, warp = tid / 32, lane = tid % 32;
  const int slot = lane / G, gl = lane % G;
  const int vend = voff + (ACCUM ? ((cols + 3) & ~3) : 0);
  for (long e = tid; e < (long)cols * (vend - len); e += nthr) {
    const int c = (int)(e / (vend - len)), k = len + (int)(e % (vend - len));
    X[(long)c * ldx + k] = (ACCUM && k - voff == c) ? 1.f : 0.f;
  }
  __syncthreads();
  if (cols <= 1) return 0;
  const int nut = vend / 4, nud = voff / 4;
  const int nb = (cols + P - 1) / P, nbp = nb + (nb & 1), npairs = nbp / 2;
  const int aw = min(npairs, nthr / 32);  // warps; warp w takes block pairs w, w + aw, ...
  if (warp >= aw) return 0;
  const int nbar = aw * 32;
  const float tol2 = tol * tol, is2 = (float)inv_scale2;
  const int max_br = max_sweeps * (nbp - 1);
  int br = 0, quiet = 0;
  for (; br < max_br; ++br) {
    const int k = br % (nbp - 1);
    bool big = false;
    for (int bp = warp; bp < npairs; bp += aw) {  // the block pairs are disjoint within a round
    int ba, bb;
    rr_pair(bp, k, nbp, &ba, &bb);
    int ti = ba * P + slot, bi = bb * P + slot;  // column ids; >= cols: padding
    float4 tp[NU], bt[NU];
#pragma unroll
    for (int t = 0; t < NU; ++t) {
      const int u = gl + G * t;
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      tp[t] = (ti < cols && u < nut) ? reinterpret_cast<const float4*>(X + (long)ti * ldx)[u] : z;
      bt[t] = (bi < cols && u < nut) ? reinterpret_cast<const float4*>(X + (long)bi * ldx)[u] : z;
    }
    const int nr = k == 0 ? 2 * P - 1 : P;
    for (int rd = 0; rd < nr; ++rd) {
      // the pair's Gram over the data rows, as packed fp32 pairs (sm_100
      // FFMA2): (x, y) and (z, w) of every unit in two accumulator pairs
      float2 al2 = make_float2(0.f, 0.f), be2 = al2, ga2 = al2;
#pragma unroll
      for (int t = 0; t < NUD; ++t) {
        const bool d = gl + G * t < nud;
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 a = d ? tp[t] : z, b = d ? bt[t] : z;
        const float2 a01 = make_float2(a.x, a.y), a23 = make_float2(a.z, a.w);
        const float2 b01 = make_float2(b.x, b.y), b23 = make_float2(b.z, b.w);
        al2 = __ffma2_rn(a01, a01, al2); al2 = __ffma2_rn(a23, a23, al2);
        be2 = __ffma2_rn(b01, b01, be2); be2 = __ffma2_rn(b23, b23, be2);
        ga2 = __ffma2_rn(a01, b01, ga2); ga2 = __ffma2_rn(a23, b23, ga2);
      }
      float al = al2.x + al2.y, be = be2.x + be2.y, ga = ga2.x + ga2.y;
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) {
        al += __shfl_xor_sync(kAll, al, o);
        be += __shfl_xor_sync(kAll, be, o);
        ga += __shfl_xor_sync(kAll, ga, o);
      }
      al *= is2;
      be *= is2;
      ga *= is2;
      const bool live = ti < cols && bi < cols && al > (float)kJacobiFloor && be > (float)kJacobiFloor;
      if (live && ga * ga > tol2 * al * be) {
        // the lower column index is the rotation's first column, as in cta_hestenes
        const bool swp = ti > bi;
        float c, s;
        jacobi_rotation(swp ? al - be : be - al, 2.f * ga, c, s);
        if (swp) s = -s;
        // top' = c a - s b, bottom' = s a + c b, on packed pairs
        const float2 c2 = make_float2(c, c), s2 = make_float2(s, s), ns2 = make_float2(-s, -s);
#pragma unroll
        for (int t = 0; t < NU; ++t) {
          const float4 a = tp[t], b = bt[t];
          const float2 a01 = make_float2(a.x, a.y), a23 = make_float2(a.z, a.w);
          const float2 b01 = make_float2(b.x, b.y), b23 = make_float2(b.z, b.w);
          const float2 t01 = __ffma2_rn(c2, a01, __fmul2_rn(ns2, b01));
          const float2 t23 = __ffma2_rn(c2, a23, __fmul2_rn(ns2, b23));
          const float2 u01 = __ffma2_rn(s2, a01, __fmul2_rn(c2, b01));
          const float2 u23 = __ffma2_rn(s2, a23, __fmul2_rn(c2, b23));
          tp[t] = make_float4(t01.x, t01.y, t23.x, t23.y);
          bt[t] = make_float4(u01.x, u01.y, u23.x, u23.y);
        }
        big = big || ga * ga > kJacobiQuadStop * kJacobiQuadStop * al * be;
      }
      if (k == 0) {
        // circle method over the P slots: slot 0's top stays; slot 1's top <-
        // slot 0's bottom, other tops <- the previous slot's top; bottoms <-
        // the next slot's bottom, the last slot's bottom <- its own top
        const bool first = slot == 0, last = slot == P - 1;
#pragma unroll
        for (int t = 0; t < NU; ++t) {
          float* tv = reinterpret_cast<float*>(&tp[t]);
          float* bv = reinterpret_cast<float*>(&bt[t]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float up = __shfl_up_sync(kAll, first ? bv[q] : tv[q], G);
            const float dn = __shfl_down_sync(kAll, bv[q], G);
            const float nt = first ? tv[q] : up;
            bv[q] = last ? tv[q] : dn;
            tv[q] = nt;
          }
        }
        const int up = __shfl_up_sync(kAll, first ? bi : ti, G);
        const int dn = __shfl_down_sync(kAll, bi, G);
        const int nt = first ? ti : up;
        bi = last ? ti : dn;
        ti = nt;
      } else if (rd < nr - 1) {  // cross rounds: the bottoms move on one group
        const int src = (lane + G) & 31;
#pragma unroll
        for (int t = 0; t < NU; ++t) {
          bt[t].x = __shfl_sync(kAll, bt[t].x, src);
          bt[t].y = __shfl_sync(kAll, bt[t].y, src);
          bt[t].z = __shfl_sync(kAll, bt[t].z, src);
          bt[t].w = __shfl_sync(kAll, bt[t].w, src);
        }
        bi = __shfl_sync(kAll, bi, src);
      }
    }
#pragma unroll
    for (int t = 0; t < NU; ++t) {
      const int u = gl + G * t;
      if (u < nut) {
        if (ti < cols) reinterpret_cast<float4*>(X + (long)ti * ldx)[u] = tp[t];
        if (bi < cols) reinterpret_cast<float4*>(X + (long)bi * ldx)[u] = bt[t];
      }
    }
    }
    quiet = named_barrier_or(kJacobiBarrier, nbar, big) ? 0 : quiet + 1;
    if (quiet >= nbp - 1) {
      ++br;
      break;
    }
  }
  if (quiet < nbp - 1) return max_sweeps;
  return (br + nbp - 2) / (nbp - 1) - 1;
}

// The core's Jacobi: the block-ordered register form when the shape fits
// it (up to two block pairs per warp, at most ten units per lane), else the
// cyclic form.  Same contract as cta_hestenes_any with accum = true.
static __device__ int core_hestenes(float* X, int len, int voff, int cols, int ldx, float tol,
                                    int max_sweeps, double inv_scale2) {
  const int nut = (voff + ((cols + 3) & ~3)) / 4, nud = voff / 4;
  const int nu = (nut + kBlkLanes - 1) / kBlkLanes, nud_l = (nud + kBlkLanes - 1) / kBlkLanes;
  const int nb = (cols + 3) / 4, npairs = (nb + (nb & 1)) / 2;
  // up to two block pairs per warp (the wider cores: r = 128, 128-column
  // pre-fill blocks), at most ten units per lane
  const bool fits = (reinterpret_cast<unsigned long>(X) & 15) == 0 && ldx % 4 == 0 &&
                    npairs <= 2 * (int)(blockDim.x / 32);
#define KVD_BJ(UU, DD)                                                                    \
  if (fits && nu == UU && nud_l == DD)                                                    \
    return cta_block_hestenes<UU, DD>(X, len, voff, cols, ldx, tol, max_sweeps, inv_scale2);
  KVD_BJ(2, 1) KVD_BJ(3, 2) KVD_BJ(4, 2) KVD_BJ(5, 3) KVD_BJ(6, 3) KVD_BJ(7, 4) KVD_BJ(8, 4)
  KVD_BJ(9, 5) KVD_BJ(10, 5)
#undef KVD_BJ
  return cta_hestenes_any<float>(X, len, voff, cols, ldx, tol, max_sweeps, inv_scale2);
}

// The same for a Jacobi with nothing accumulated (the pre-fill blocks'
// preconditioner on the Gram factor's rows): the block form when it fits,
// else cta_hestenes_any with accum = false.
static __device__ int plain_hestenes(float* X, int len, int voff, int cols, int ldx, float tol,
                                     int max_sweeps, double inv_scale2) {
  const int nu = (voff / 4 + kBlkLanes - 1) / kBlkLanes;
  const int nb = (cols + 3) / 4, npairs = (nb + (nb & 1)) / 2;
  const bool fits = (reinterpret_cast<unsigned long>(X) & 15) == 0 && ldx % 4 == 0 &&
                    npairs <= 2 * (int)(blockDim.x / 32);
#define KVD_BJ(UU)                                                                         \
  if (fits && nu == UU)                                                                    \
    return cta_block_hestenes<UU, UU, false>(X, len, voff, cols, ldx, tol, max_sweeps, inv_scale2);
  KVD_BJ(1) KVD_BJ(2) KVD_BJ(3) KVD_BJ(4)
#undef KVD_BJ
  return cta_hestenes_any<float>(X, len, voff, cols, ldx, tol, max_sweeps, inv_scale2, false);
}

// 16 consecutive floats p[j0 .. j0+16) of a row, zero past `nb`; `vec` =
// the row start and j0 are 16-byte aligned.
static __device__ __forceinline__ void load16(const float* p, int j0, int nb, bool vec,
                                              float (&v)[16]) {
  if (vec && j0 + 16 <= nb) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 t = *reinterpret_cast<const float4*>(p + j0 + 4 * q);
      v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) v[jj] = (j0 + jj < nb) ? p[j0 + jj] : 0.f;
  }
}

static __device__ __forceinline__ void store16(float* p, int j0, int nb, bool vec,
                                               const float (&v)[16]) {
  if (vec && j0 + 16 <= nb) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<float4*>(p + j0 + 4 * q) =
          make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
#pragma unroll
    for (int jj = 0; jj < 16; ++jj)
      if (j0 + jj < nb) p[j0 + jj] = v[jj];
  }
}

// out[k*ldo + j] = sum_{i<K} A[i*lda + k] B[i*ldb + j] - diag*[k == j]
// for k < M (<= kMaxStepLd), j < NB.  The warps split into ceil(M/32)
// k-chunks x ks K-slices; a lane owns one k and 16 j sums in fp32 over its
// slice, and the slices' partials are added in fp64.  A row of B is read as
// a broadcast, so B[i] rows are 16-byte vectors when `bvec`.
static __device__ __forceinline__ void cta_tn(int M, int NB, int K, const float* A, int lda, const float* B,
                              int ldb, bool bvec, float* out, int ldo, float diag, float* part) {
  const int tid = threadIdx.x, nthr = blockDim.x, lane = tid % 32, warp = tid / 32;
  const int nw = nthr / 32;
  const int kc = (M + 31) / 32;
  const int ks = max(1, nw / kc);
  const int slice = (K + ks - 1) / ks;
  for (int j0 = 0; j0 < NB; j0 += 16) {
    for (int wi = warp; wi < kc * ks; wi += nw) {
      const int kch = wi % kc, ksl = wi / kc;
      const int k = kch * 32 + lane;
      const int i0 = ksl * slice, i1 = min(K, i0 + slice);
      float acc[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) acc[jj] = 0.f;
#pragma unroll 2
      for (int i = i0; i < i1; ++i) {
        const float a = k < M ? A[(long)i * lda + k] : 0.f;
        float bv[16];
        load16(B + (long)i * ldb, j0, NB, bvec, bv);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) acc[jj] = fmaf(a, bv[jj], acc[jj]);
      }
      if (k < M) {
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) part[((long)ksl * 16 + jj) * M + k] = acc[jj];
      }
    }
    __syncthreads();
    for (int e = tid; e < 16 * M; e += nthr) {
      const int jj = e / M, k = e % M, j = j0 + jj;
      if (j >= NB) continue;
      double sum = 0.0;
      for (int sl = 0; sl < ks; ++sl) sum += (double)part[((long)sl * 16 + jj) * M + k];
      if (k == j) sum -= (double)diag;
      out[(long)k * ldo + j] = (float)sum;
    }
    __syncthreads();
  }
}

// Rows of the residual, one thread per row i, 16 tokens at a time:
//   v = (from_xr ? XR[i][j] : Rm[j][i]) - sum_{k<K} A[i*lda + k] C[k*ldc + j]
// written to Rm[j*ldr + i] (j < b) and, when to_xr, to XR[i*ldb + j].  C rows
// and XR rows are 16-byte aligned (ldc, ldb multiples of 4).
static __device__ __forceinline__ void cta_rows_sub(int n, int b, int b16, int K, const float* A, int lda,
                                    const float* C, int ldc, float* XR, int ldb, float* Rm,
                                    int ldr, bool from_xr, bool to_xr) {
  const bool avec = ((reinterpret_cast<unsigned long>(A) & 15) == 0) && (lda % 4 == 0);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float* ar = A + (long)i * lda;
    float* xr = XR + (long)i * ldb;
    for (int j0 = 0; j0 < b16; j0 += 16) {
      float acc[16];
      if (from_xr) {
        load16(xr, j0, b16, true, acc);
      } else {
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) acc[jj] = (j0 + jj < b) ? Rm[(long)(j0 + jj) * ldr + i] : 0.f;
      }
      int k = 0;
      if (avec) {
        for (; k + 4 <= K; k += 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(ar + k);
          const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            float cv[16];
            load16(C + (long)(k + kk) * ldc, j0, b16, true, cv);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) acc[jj] = fmaf(-av[kk], cv[jj], acc[jj]);
          }
        }
      }
      for (; k < K; ++k) {
        const float av = ar[k];
        float cv[16];
        load16(C + (long)k * ldc, j0, b16, true, cv);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) acc[jj] = fmaf(-av, cv[jj], acc[jj]);
      }
#pragma unroll
      for (int jj = 0; jj < 16; ++jj)
        if (j0 + jj < b) Rm[(long)(j0 + jj) * ldr + i] = acc[jj];
      if (to_xr) store16(xr, j0, b16, true, acc);
    }
  }
  __syncthreads();
}

// Uo[i*ld + c] = sum_{k<r} A[i*lda + k] WU[k*ldw + c] + sum_{j<m} Q[j*n + i] WU[(r+j)*ldw + c]
// for c < keep; one thread per row, 16 columns at a time (WU rows 16-byte
// aligned and zero-padded to ldw).
static __device__ __forceinline__ void cta_basis_rows(int n, int keep, int r, int m, const float* A, int lda,
                                      const float* Q, const float* WU, int ldw, float* Uo, int ld,
                                      bool uvec) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float* ar = A + (long)i * lda;
    for (int c0 = 0; c0 < keep; c0 += 16) {
      float acc[16];
#pragma unroll
      for (int cc = 0; cc < 16; ++cc) acc[cc] = 0.f;
      for (int k = 0; k < r; ++k) {
        const float av = ar[k];
        float wv[16];
        load16(WU + (long)k * ldw, c0, ldw, true, wv);
#pragma unroll
        for (int cc = 0; cc < 16; ++cc) acc[cc] = fmaf(av, wv[cc], acc[cc]);
      }
      for (int j = 0; j < m; ++j) {
        const float qv = Q[(long)j * n + i];
        float wv[16];
        load16(WU + (long)(r + j) * ldw, c0, ldw, true, wv);
#pragma unroll
        for (int cc = 0; cc < 16; ++cc) acc[cc] = fmaf(qv, wv[cc], acc[cc]);
      }
      store16(Uo + (long)i * ld, c0, keep, uvec, acc);
    }
  }
  __syncthreads();
}

// Uo[i][c] = S[i][c] - 1/2 sum_k S[i][k] E[k][c] for c < keep <= 32, one
// thread per row holding it in registers (E zero-padded to 32 x 32, row
// stride lde).  S may be Uo itself.
static __device__ __forceinline__ void cta_polish_rows(int n, int keep, const float* S, int lds,
                                                       bool svec, float* Uo, int ld, bool uvec,
                                                       const float* E, int lde) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float* sr = S + (long)i * lds;
    float row[32];
    {
      float t[16];
      load16(sr, 0, keep, svec, t);
#pragma unroll
      for (int c = 0; c < 16; ++c) row[c] = t[c];
      load16(sr, 16, keep, svec, t);
#pragma unroll
      for (int c = 0; c < 16; ++c) row[16 + c] = t[c];
    }
#pragma unroll
    for (int c0 = 0; c0 < 32; c0 += 16) {
      if (c0 >= keep) break;
      float acc[16];
#pragma unroll
      for (int cc = 0; cc < 16; ++cc) acc[cc] = row[c0 + cc];
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        if (k < keep) {
          const float h = -0.5f * row[k];
          float ev[16];
          load16(E + (long)k * lde, c0, 32, true, ev);
#pragma unroll
          for (int cc = 0; cc < 16; ++cc) acc[cc] = fmaf(h, ev[cc], acc[cc]);
        }
      }
      store16(Uo + (long)i * ld, c0, keep, uvec, acc);
    }
  }
  __syncthreads();
}

// Un[i*ldn + c] = sum_{k<r} Un[i*ldn + k] WU[k*ldw + c] + sum_{j<m} Q[j*n + i] WU[(r+j)*ldw + c]
// for c < keep <= 32, in place: a thread reads its whole row of U before it
// writes the row of U_new.  WU and Un rows are 16-byte aligned (ldw, ldn
// multiples of 4), WU zero past keep.
static __device__ __forceinline__ void cta_basis_rows32(int n, int keep, int r, int m, float* Un,
                                                        int ldn, const float* Q, const float* WU,
                                                        int ldw) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float* ur = Un + (long)i * ldn;
    float acc[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) acc[c] = 0.f;
    float u4[4];
    for (int k = 0; k < r + m; ++k) {
      float av;
      if (k < r) {
        if ((k & 3) == 0) {
          if (k + 4 <= r) {
            const float4 t = *reinterpret_cast<const float4*>(ur + k);
            u4[0] = t.x; u4[1] = t.y; u4[2] = t.z; u4[3] = t.w;
          } else {
            for (int kk = 0; kk < 4; ++kk) u4[kk] = k + kk < r ? ur[k + kk] : 0.f;
          }
        }
        av = u4[k & 3];
      } else {
        av = Q[(long)(k - r) * n + i];
      }
      float w[16];
      load16(WU + (long)k * ldw, 0, ldw, true, w);
#pragma unroll
      for (int c = 0; c < 16; ++c) acc[c] = fmaf(av, w[c], acc[c]);
      if (keep > 16) {
        load16(WU + (long)k * ldw, 16, ldw, true, w);
#pragma unroll
        for (int c = 0; c < 16; ++c) acc[16 + c] = fmaf(av, w[c], acc[16 + c]);
      }
    }
#pragma unroll
    for (int c = 0; c < 32; ++c)
      if (c < keep) ur[c] = acc[c];
  }
  __syncthreads();
}

// Register-blocked forms of the three products that turn the staged basis
// into the polished U_new (keep <= 32 columns, n % 4 == 0, every pointer and
// pitch 16-byte aligned): a thread owns a 4-row x 8-column tile, so one
// 16-byte load of a coefficient row serves four rows instead of one.  Each
// output keeps the operation order of the row-per-thread forms above (the
// same fmaf chains over k), so the results are the same bit for bit; the
// fmas of two adjacent columns issue as one packed pair (sm_100 FFMA2, each
// lane a round-to-nearest fma).

// Un[i][c] = sum_{k<r} Un[i][k] WU[k][c] + sum_{j<m} Q[j][i] WU[r+j][c], c < keep,
// in place: a row's old values are read only by the four lanes that own its
// tiles, all reads before the warp's writes.
static __device__ __forceinline__ void cta_basis_tiles(int n, int keep, int r, int m, float* Un,
                                                       int ldn, const float* Q, const float* WU,
                                                       int ldw) {
  const int tid = threadIdx.x, nthr = blockDim.x, cg = tid & 3;
  const int ngr = n / 4;
  for (int rg0 = 0; rg0 < ngr; rg0 += nthr / 4) {  // (uniform trip count: __syncwarp below)
    const int rg = rg0 + tid / 4;
    const bool live = rg < ngr;
    const int i0 = live ? 4 * rg : 0;
    float2 acc[4][4];  // columns (2c, 2c + 1) as packed pairs
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[q][c] = make_float2(0.f, 0.f);
    auto step = [&](int k, const float (&av)[4]) {  // acc += av (x) WU[k][8cg..8cg+8)
      const float4 w0 = *reinterpret_cast<const float4*>(WU + k * ldw + 8 * cg);
      const float4 w1 = *reinterpret_cast<const float4*>(WU + k * ldw + 8 * cg + 4);
      const float2 w[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                           make_float2(w1.z, w1.w)};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 a2 = make_float2(av[q], av[q]);
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[q][c] = __ffma2_rn(a2, w[c], acc[q][c]);
      }
    };
    int k = 0;
    for (; k + 4 <= r; k += 4) {  // U's columns four at a time
      float u4[4][4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 t = *reinterpret_cast<const float4*>(Un + (i0 + q) * ldn + k);
        u4[q][0] = t.x; u4[q][1] = t.y; u4[q][2] = t.z; u4[q][3] = t.w;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float av[4] = {u4[0][kk], u4[1][kk], u4[2][kk], u4[3][kk]};
        step(k + kk, av);
      }
    }
    for (; k < r; ++k) {
      float av[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) av[q] = Un[(i0 + q) * ldn + k];
      step(k, av);
    }
    for (int j = 0; j < m; ++j) {  // then Q's rows
      const float4 t = *reinterpret_cast<const float4*>(Q + j * n + i0);
      const float av[4] = {t.x, t.y, t.z, t.w};
      step(r + j, av);
    }
    __syncwarp();
    if (live) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int c = 0; c < 8; ++c)
          if (8 * cg + c < keep) Un[(i0 + q) * ldn + 8 * cg + c] = (c & 1) ? acc[q][c >> 1].y : acc[q][c >> 1].x;
    }
    __syncwarp();
  }
  __syncthreads();
}

// out[k][j] = sum_{i<K} A[i][k] B[i][j] - diag [k == j] for k < M <= 32, j < NB
// (cta_tn's result bit for bit with 512 threads): the rows are split into
// 16 slices (fp32 sums of a slice, in row order; fp64 sum of the slices), a
// thread owns a 4 x 4 tile of one slice -- eight row tiles by four column
// tiles per pass of 16 columns (part holds 16 x 16 x 32 partials).
static __device__ __forceinline__ void cta_tn_tiles(int M, int NB, int K, const float* A, int lda,
                                                    const float* B, int ldb, float* out, int ldo,
                                                    float diag, float* part) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  constexpr int ks = 16;
  const int slice = (K + ks - 1) / ks;
  for (int j0 = 0; j0 < NB; j0 += 16) {
    for (int it = tid; it < ks * 8 * 4; it += nthr) {  // (slice, row tile a, column tile c)
      const int c = it & 3, a = (it >> 2) & 7, sl = it >> 5;
      if (4 * a >= M || j0 + 4 * c >= NB) continue;
      const int i0 = sl * slice, i1 = min(K, i0 + slice);
      float2 acc[4][2];  // columns (2y, 2y + 1) as packed pairs
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 2; ++y) acc[x][y] = make_float2(0.f, 0.f);
      for (int i = i0; i < i1; ++i) {
        const float4 ua = *reinterpret_cast<const float4*>(A + i * lda + 4 * a);
        const float4 uc = *reinterpret_cast<const float4*>(B + i * ldb + j0 + 4 * c);
        const float va[4] = {ua.x, ua.y, ua.z, ua.w};
        const float2 vc[2] = {make_float2(uc.x, uc.y), make_float2(uc.z, uc.w)};
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const float2 a2 = make_float2(va[x], va[x]);
#pragma unroll
          for (int y = 0; y < 2; ++y) acc[x][y] = __ffma2_rn(a2, vc[y], acc[x][y]);
        }
      }
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y)
          part[(sl * 16 + 4 * c + y) * 32 + 4 * a + x] = (y & 1) ? acc[x][y >> 1].y : acc[x][y >> 1].x;
    }
    __syncthreads();
    for (int e = tid; e < 16 * 32; e += nthr) {
      const int jj = e / 32, k = e % 32, j = j0 + jj;
      if (j >= NB || k >= M) continue;
      double sum = 0.0;
      for (int sl = 0; sl < ks; ++sl) sum += (double)part[(sl * 16 + jj) * 32 + k];
      if (k == j) sum -= (double)diag;
      out[k * ldo + j] = (float)sum;
    }
    __syncthreads();
  }
}

// cta_rows_sub on tiles, for 16-column blocks (b16 == 16): a thread owns
// four rows n/4 apart (so the column-major stores of R are conflict-free)
// by four columns; the same fmaf chain over k per output.
static __device__ __forceinline__ void cta_rows_sub_tiles(int n, int b, int K, const float* A,
                                                          int lda, const float* C, int ldc,
                                                          float* XR, int ldb, float* Rm, int ldr,
                                                          bool from_xr, bool to_xr) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int ngr = n / 4;
  for (int it = tid; it < ngr * 4; it += nthr) {
    const int j0 = 4 * (it / ngr), rb = it % ngr;
    float2 acc[4][2];  // columns (2y, 2y + 1) as packed pairs
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = rb + q * ngr;
      if (from_xr) {
        const float4 t = *reinterpret_cast<const float4*>(XR + i * ldb + j0);
        acc[q][0] = make_float2(t.x, t.y); acc[q][1] = make_float2(t.z, t.w);
      } else {
        float v[4];
#pragma unroll
        for (int y = 0; y < 4; ++y) v[y] = j0 + y < b ? Rm[(j0 + y) * ldr + i] : 0.f;
        acc[q][0] = make_float2(v[0], v[1]); acc[q][1] = make_float2(v[2], v[3]);
      }
    }
    auto step = [&](int k, const float (&av)[4]) {  // packed pairs of columns (sm_100 FFMA2)
      const float4 c4 = *reinterpret_cast<const float4*>(C + k * ldc + j0);
      const float2 cv[2] = {make_float2(c4.x, c4.y), make_float2(c4.z, c4.w)};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 a2 = make_float2(-av[q], -av[q]);
#pragma unroll
        for (int y = 0; y < 2; ++y) acc[q][y] = __ffma2_rn(a2, cv[y], acc[q][y]);
      }
    };
    int k = 0;
    for (; k + 4 <= K; k += 4) {
      float a4[4][4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 t = *reinterpret_cast<const float4*>(A + (rb + q * ngr) * lda + k);
        a4[q][0] = t.x; a4[q][1] = t.y; a4[q][2] = t.z; a4[q][3] = t.w;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float av[4] = {a4[0][kk], a4[1][kk], a4[2][kk], a4[3][kk]};
        step(k + kk, av);
      }
    }
    for (; k < K; ++k) {
      float av[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) av[q] = A[(rb + q * ngr) * lda + k];
      step(k, av);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = rb + q * ngr;
      const float v[4] = {acc[q][0].x, acc[q][0].y, acc[q][1].x, acc[q][1].y};
#pragma unroll
      for (int y = 0; y < 4; ++y)
        if (j0 + y < b) Rm[(j0 + y) * ldr + i] = v[y];
      if (to_xr) *reinterpret_cast<float4*>(XR + i * ldb + j0) = make_float4(v[0], v[1], v[2], v[3]);
    }
  }
  __syncthreads();
}

// Uo[i][c] = S[i][c] - 1/2 sum_k S[i][k] E[k][c] for c < keep (E zero-padded
// to 32 x 32, row pitch lde), S in shared memory, Uo global.
static __device__ __forceinline__ void cta_polish_tiles(int n, int keep, const float* S, int lds,
                                                        float* Uo, int ld, bool uvec,
                                                        const float* E, int lde) {
  const int tid = threadIdx.x, nthr = blockDim.x, cg = tid & 3;
  const int ngr = n / 4;
  for (int rg = tid / 4; rg < ngr; rg += nthr / 4) {
    const int i0 = 4 * rg;
    float2 acc[4][4];  // columns (2c, 2c + 1) as packed pairs
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 t0 = *reinterpret_cast<const float4*>(S + (i0 + q) * lds + 8 * cg);
      const float4 t1 = *reinterpret_cast<const float4*>(S + (i0 + q) * lds + 8 * cg + 4);
      const float t[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
      float v[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) v[c] = 8 * cg + c < keep ? t[c] : 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[q][c] = make_float2(v[2 * c], v[2 * c + 1]);
    }
    for (int k0 = 0; k0 < keep; k0 += 4) {  // (columns past keep are read, not used)
      float h4[4][4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 t = *reinterpret_cast<const float4*>(S + (i0 + q) * lds + k0);
        h4[q][0] = t.x; h4[q][1] = t.y; h4[q][2] = t.z; h4[q][3] = t.w;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        if (k0 + kk < keep) {
          const int k = k0 + kk;
          const float4 e0 = *reinterpret_cast<const float4*>(E + k * lde + 8 * cg);
          const float4 e1 = *reinterpret_cast<const float4*>(E + k * lde + 8 * cg + 4);
          const float ev[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float h = -0.5f * h4[q][kk];
            const float2 h2 = make_float2(h, h);
#pragma unroll
            for (int c = 0; c < 4; ++c)  // packed pairs of columns (sm_100 FFMA2)
              acc[q][c] = __ffma2_rn(h2, make_float2(ev[2 * c], ev[2 * c + 1]), acc[q][c]);
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float* dst = Uo + (long)(i0 + q) * ld + 8 * cg;
      if (uvec && 8 * cg + 8 <= keep) {
        *reinterpret_cast<float4*>(dst) = make_float4(acc[q][0].x, acc[q][0].y, acc[q][1].x, acc[q][1].y);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(acc[q][2].x, acc[q][2].y, acc[q][3].x, acc[q][3].y);
      } else {
#pragma unroll
        for (int c = 0; c < 8; ++c)
          if (8 * cg + c < keep) dst[c] = (c & 1) ? acc[q][c >> 1].y : acc[q][c >> 1].x;
      }
    }
  }
  __syncthreads();
}

// Column norms (fp64) of X[:, 0..cols) into nrm, then order = descending.
static __device__ __forceinline__ void cta_colnorm_order(const float* X, int len, int cols, int ldx, double* nrm,
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
static __device__ __forceinline__ void cta_cgs2_rows(float* Q, int m, int n, double* dots /*>= m*/,
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

// kSmem: every buffer of the plan is staged in shared memory, so all of them
// are addressed from the shared pool and compile to shared-memory loads and
// stores; otherwise each region may live in the global workspace.
template <bool kSmem>
__global__ void __launch_bounds__(kStepThreads) bug_step_kernel(BugStepBatch batch) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const StepPlan& P = batch.plan;
  const int p = blockIdx.x;
  const BugStepArgs& A = batch.s[blockIdx.y];
  const int n = A.n, b = A.b, cap = A.rank_cap, ld = A.ld;
  const float* U = A.u + p * A.u_sp;
  float* Uo = A.u_out + p * A.u_sp;
  float* sig = A.sigma + p * A.sig_sp;
  const float* X = A.x + p * A.x_sp;
  const int r = A.r[p];
  char* wsb = A.ws + p * A.ws_sp;
  double* red = reinterpret_cast<double*>(smem_raw);  // 64 doubles
  float* pool = reinterpret_cast<float*>(smem_raw + kStepMiscBytes);
  auto region = [&](int g) -> float* {
    if constexpr (kSmem) return pool + P.smem[g];
    return P.smem[g] >= 0 ? pool + P.smem[g] : reinterpret_cast<float*>(wsb + P.ws[g]);
  };
  float* Rm = region(kRgRm);      // residual columns (pitch n, then ldr with V below)
  float* XR = region(kRgXr);      // [n][ldb] block rows, then residual rows, then Q [m][n]
  float* part = region(kRgPart);  // K-split partials
  float* AS = region(kRgAs);      // [ld][b16] a = U^T X
  float* A2 = region(kRgA2);      // [ld][b16] re-orthogonalisation correction
  float* BT = region(kRgCore);    // [N][ldbt] B^T columns with W below them
  float* Pol = region(kRgPol);    // [ldp][ldp] U_new^T U_new - I
  float* WU = region(kRgWu);      // [N][ldw] top left vectors of B, ordered
  double* nrm = reinterpret_cast<double*>(region(kRgSmall));  // [ld+b]
  double* sv = nrm + (ld + b);                                // [b]
  int* ord = reinterpret_cast<int*>(sv + b);                  // [ld+b]
  int* ordh = ord + (ld + b);                                 // [b]
  const bool us = P.smem[kRgUs] >= 0 && r > 0;
  const float* Uc;
  if constexpr (kSmem) Uc = pool + P.smem[kRgUs];  // read only when r > 0
  else Uc = us ? pool + P.smem[kRgUs] : U;
  const int lda = us ? P.ldu : ld;
  const int b16 = P.b16, ldb = P.ldb, ldbt = P.ldbt, ldw = P.ldw, ldp = P.ldp;
  const bool uvec = ((reinterpret_cast<unsigned long>(Uo) & 15) == 0) && (ld % 4 == 0);
  __shared__ double s_xnorm2;
  __shared__ int s_m, s_keep, s_degenerate;
  const int tid = threadIdx.x, nthr = blockDim.x, lane = tid % 32, warp = tid / 32;

  // ----- stage the block token-transposed (XR[i][j] = X[j][i], zero past b) and U,
  // and ||X||_F^2 (fp64 sums of fp32 squares).  The absorb block's shapes
  // (b n <= 16 threads' worth, n r <= 32) issue every 16-byte load -- four of
  // the block and eight of U per thread -- before the first store and square
  // the block from the same registers; other shapes take the loops below.
  double xacc = 0.0;
  const bool xvec = (n & 3) == 0 && (reinterpret_cast<unsigned long>(X) & 15) == 0;
  const bool uvec4 = (r & 3) == 0 && (ld & 3) == 0 && (reinterpret_cast<unsigned long>(U) & 15) == 0;
  if (us && xvec && uvec4 && b * n <= 16 * nthr && n * r <= 32 * nthr) {
    const int nx4 = b * n / 4, r4 = r / 4, nu4 = n * r4;
    const float4* X4 = reinterpret_cast<const float4*>(X);
    float4 xv[4], uv[8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = tid + u * nthr;
      if (e < nx4) xv[u] = X4[e];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = tid + u * nthr;
      if (e < nu4) uv[u] = *reinterpret_cast<const float4*>(U + (long)(e / r4) * ld + 4 * (e % r4));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = tid + u * nthr;
      if (e < nx4) {
        const float4 v = xv[u];
        xacc += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
        const int j = 4 * e / n, i = 4 * e % n;
        float* d = XR + i * ldb + j;
        d[0] = v.x; d[ldb] = v.y; d[2 * ldb] = v.z; d[3 * ldb] = v.w;
      }
    }
    float* dst = pool + P.smem[kRgUs];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = tid + u * nthr;
      if (e < nu4) *reinterpret_cast<float4*>(dst + (e / r4) * lda + 4 * (e % r4)) = uv[u];
    }
    if (b16 > b) {
      const int pad = b16 - b;
      for (int e = tid; e < n * pad; e += nthr) XR[(e / pad) * ldb + b + e % pad] = 0.f;
    }
  } else {
  for (long e = tid; e < (long)b * n; e += nthr) xacc += (double)X[e] * X[e];
  if ((n & 3) == 0 && (reinterpret_cast<unsigned long>(X) & 15) == 0) {
    const float4* X4 = reinterpret_cast<const float4*>(X);
    const long n4 = (long)b * n / 4;
    for (long e0 = tid; e0 < n4; e0 += 4L * nthr) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long e = e0 + (long)u * nthr;
        if (e < n4) v[u] = X4[e];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long e = e0 + (long)u * nthr;
        if (e < n4) {
          const int j = (int)(4 * e / n), i = (int)(4 * e % n);
          float* d = XR + (long)i * ldb + j;
          d[0] = v[u].x; d[ldb] = v[u].y; d[2 * ldb] = v[u].z; d[3 * ldb] = v[u].w;
        }
      }
    }
  } else {
    for (long e = tid; e < (long)b * n; e += nthr) {
      const int j = (int)(e / n), i = (int)(e % n);
      XR[(long)i * ldb + j] = X[e];
    }
  }
  if (b16 > b) {
    const int pad = b16 - b;
    for (long e = tid; e < (long)n * pad; e += nthr)
      XR[(e / pad) * ldb + b + (int)(e % pad)] = 0.f;
  }
  if (us) {
    float* dst = pool + P.smem[kRgUs];
    if ((r & 3) == 0 && (ld & 3) == 0 && (reinterpret_cast<unsigned long>(U) & 15) == 0) {
      const int r4 = r / 4;
      const long n4 = (long)n * r4;
      for (long e0 = tid; e0 < n4; e0 += 4L * nthr) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const long e = e0 + (long)u * nthr;
          if (e < n4) v[u] = *reinterpret_cast<const float4*>(U + (e / r4) * ld + 4 * (e % r4));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const long e = e0 + (long)u * nthr;
          if (e < n4) {
            float* d = dst + (e / r4) * lda + 4 * (e % r4);
            d[0] = v[u].x; d[1] = v[u].y; d[2] = v[u].z; d[3] = v[u].w;
          }
        }
      }
    } else {
      for (long e = tid; e < (long)n * r; e += nthr) {
        const long i = e / r, k = e % r;
        dst[i * lda + k] = U[i * ld + k];
      }
    }
  }
  }
  xacc = warp_sum(xacc);
  if (lane == 0) red[warp] = xacc;
  for (int e = tid; e < r * b16; e += nthr) { AS[e] = 0.f; A2[e] = 0.f; }
  __syncthreads();
  if (tid == 0) { double t = 0; for (int i = 0; i < nthr / 32; ++i) t += red[i]; s_xnorm2 = t; }
  // SVD geometry.  b <= n: one-sided Jacobi on R's b columns, R V = [s_j q_j].
  // b > n (more columns than rows cannot all be made orthogonal): on the n
  // columns of R^T, R^T J = [s_j v_j], so J holds the left vectors q_j.
  // The rotations accumulate below the data in each column (rows voff..).
  // Blocks of up to 16 tokens (the absorb block): the fp64 Gram R^T R
  // (tensor-core products) is factored T^T T (Cholesky, pivots below 1e-14
  // of the trace taken as null) and the one-sided Jacobi runs on T's b
  // rows (the columns of L = T^T) -- T has R's singular values and right
  // vectors, and the rotated rows are V S -- in one warp's registers.  17..kMaxGramB tokens (the
  // pre-fill blocks): the same factorisation by the CTA, whose Jacobi (on the
  // factor's rows) gives R's right vectors to within the factor's rounding; they
  // seed the one-sided Jacobi (fp64 sums) on R V itself, whose columns are then nearly
  // orthogonal, so it converges in about one sweep to the accuracy of the
  // Jacobi on R (the factor alone loses relative accuracy in the smallest
  // singular directions, and a noisy spectrum at the truncation amplifies it).
  const bool chol = b <= 16 && b <= n;
  // 17..kMaxGramB columns: the Gram's Cholesky factor preconditions the Jacobi on R
  const bool bigg = b > 16 && b <= kMaxGramB && b <= n;
  const bool tr = !chol && b > n;
  const int nsv = tr ? n : b;
  const int rlen = tr ? b : n;
  const int voff = chol ? ((b + 3) & ~3) : (rlen + 3) & ~3;
  const int ldr = chol ? jacobi_pitch(voff + b, b, false) : jacobi_pitch(voff + nsv, nsv, true);
  const int ldr0 = (tr || chol || bigg) ? n : ldr;  // pitch the residual is formed with
  float* Tm = chol ? part + 2 * (16 * 17 + 8) : Rm;  // the factor, augmented columns (after the Gram)
  const int voffT = (b + 3) & ~3, ldrT = jacobi_pitch(voffT, b, false);  // bigg: T^T's column pitch
  // ----- residual R = (I - U U^T)^2 X (the reference's re-orthogonalised residual)
  // the tiled forms when U is staged (16-byte rows of at least 32 floats), the
  // block has 16 columns and the rank is at most 32
  const bool ptiles = us && r <= 32 && lda >= 32 && lda % 4 == 0 && b16 == 16 && n % 4 == 0 &&
                      ldb % 4 == 0 && nthr == kStepThreads;
  if (r > 0) {  // a = U^T X
    if (ptiles) cta_tn_tiles(r, b, n, Uc, lda, XR, ldb, AS, b16, 0.f, part);
    else cta_tn(r, b, n, Uc, lda, XR, ldb, true, AS, b16, 0.f, part);
  }
  if (ptiles) cta_rows_sub_tiles(n, b, r, Uc, lda, AS, b16, XR, ldb, Rm, ldr0, true, r > 0);
  else cta_rows_sub(n, b, b16, r, Uc, lda, AS, b16, XR, ldb, Rm, ldr0, true, r > 0);  // R = X - U a
  if (r > 0) {
    if (ptiles) {  // a2 = U^T R, R -= U a2
      cta_tn_tiles(r, b, n, Uc, lda, XR, ldb, A2, b16, 0.f, part);
      cta_rows_sub_tiles(n, b, r, Uc, lda, A2, b16, XR, ldb, Rm, ldr0, false, false);
    } else {
      cta_tn(r, b, n, Uc, lda, XR, ldb, true, A2, b16, 0.f, part);
      cta_rows_sub(n, b, b16, r, Uc, lda, A2, b16, XR, ldb, Rm, ldr0, false, false);
    }
    for (int e = tid; e < r * b16; e += nthr) AS[e] += A2[e];
    __syncthreads();
  }
  // ----- SVD of R
  const double inv_x2 = s_xnorm2 > 0.0 ? 1.0 / s_xnorm2 : 1.0;
  if (chol) {
    constexpr int ldg = 17;
    double* GR = reinterpret_cast<double*>(part);  // [16][17] the Gram
    if (n % 32 == 0) {
      // fp64 tensor products, G = R^T R as 2 x 2 tiles of 8 x 8 with the
      // k range split over 8 warps; the A (= R^T) and B (= R) fragments of
      // a k-step are the same two values per lane
      double* gpart = reinterpret_cast<double*>(part + 4096);  // [8 warps][4 tiles][64]
      if (warp < 8) warp_gram16_slice(Rm, n, b, warp, gpart);
      __syncthreads();
      for (int e = tid; e < 256; e += nthr) {  // sum the k slices
        const int i = e / 16, j = e % 16, t = (i / 8) * 2 + j / 8, w = (i % 8) * 8 + j % 8;
        double sum = 0.0;
        for (int wv = 0; wv < 8; ++wv) sum += gpart[(wv * 4 + t) * 64 + w];
        GR[i * ldg + j] = sum;
      }
    } else {
      for (int pp = warp; pp < b * b; pp += nthr / 32) {  // fp64 Gram, one warp per pair
        const int pi = pp / b, qi = pp % b;
        if (pi > qi) continue;
        const float* xp = Rm + (long)pi * n;
        const float* xq = Rm + (long)qi * n;
        double acc = 0.0;
        for (int e = lane; e < n; e += 32) acc = fma((double)xp[e], (double)xq[e], acc);
        acc = warp_sum(acc);
        if (lane == 0) { GR[pi * ldg + qi] = acc; GR[qi * ldg + pi] = acc; }
      }
    }
    __syncthreads();
    if (warp == 0) warp_cholesky16(GR, ldg, b, Tm, ldr);
    __syncthreads();
  } else if (bigg) {
    // 17..128 columns: the same factorisation by the whole CTA
    double* G = reinterpret_cast<double*>(region(kRgGram));  // [b][b+1]
    const int ldgb = b + 1, nt = (b + 7) / 8, ntiles = nt * (nt + 1) / 2;
    if (n % 4 == 0) {
      // fp64 tensor products over the 8 x 8 tiles (ti <= tj) of the upper
      // triangle, mirrored below; one tile per warp at a time
      const int grp = lane >> 2, tig = lane & 3;
      for (int t = warp; t < ntiles; t += nthr / 32) {
        int ti = 0, rem = t;
        while (rem >= nt - ti) { rem -= nt - ti; ++ti; }
        const int tj = ti + rem;
        const int ra = ti * 8 + grp, rb = tj * 8 + grp;
        const float* pa = Rm + (long)(ra < b ? ra : 0) * n + tig;
        const float* pb = Rm + (long)(rb < b ? rb : 0) * n + tig;
        double c0 = 0.0, c1 = 0.0, e0 = 0.0, e1 = 0.0;
#pragma unroll 2
        for (int k0 = 0; k0 < n; k0 += 8) {  // two chains over alternate k-steps
          const double a0 = ra < b ? (double)pa[k0] : 0.0, b0 = rb < b ? (double)pb[k0] : 0.0;
          const bool more = k0 + 4 < n;
          const double a1 = (ra < b && more) ? (double)pa[k0 + 4] : 0.0;
          const double b1 = (rb < b && more) ? (double)pb[k0 + 4] : 0.0;
          dmma_8x8x4(c0, c1, a0, b0);
          dmma_8x8x4(e0, e1, a1, b1);
        }
        c0 += e0;
        c1 += e1;
        const int col = tj * 8 + 2 * tig;
        const double cv[2] = {c0, c1};
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          if (ra < b && col + q < b) {
            G[ra * ldgb + col + q] = cv[q];
            if (ti != tj) G[(col + q) * ldgb + ra] = cv[q];
          }
        }
      }
    } else {
      for (int pp = warp; pp < b * b; pp += nthr / 32) {  // fp64 Gram, one warp per pair
        const int pi = pp / b, qi = pp % b;
        if (pi > qi) continue;
        const float* xp = Rm + (long)pi * n;
        const float* xq = Rm + (long)qi * n;
        double acc = 0.0;
        for (int e = lane; e < n; e += 32) acc = fma((double)xp[e], (double)xq[e], acc);
        acc = warp_sum(acc);
        if (lane == 0) { G[pi * ldgb + qi] = acc; G[qi * ldgb + pi] = acc; }
      }
    }
    __syncthreads();
    if (warp == 0) {
      double trc = 0.0;
      for (int j = lane; j < b; j += 32) trc += G[j * ldgb + j];
      trc = warp_sum(trc);
      if (lane == 0) red[0] = trc;
    }
    __syncthreads();
    const double trace = red[0];
    // right-looking Cholesky on the lower triangle (pivots at or below 1e-14
    // of the trace taken as null, as for the small blocks); the scaled column
    // j of the factor goes to row j of the (unused) upper triangle in the same
    // pass as the update, which scales its products by 1/pivot^2 itself
    for (int j = 0; j < b; ++j) {
      if (tid == 0) {
        const double piv = G[j * ldgb + j];
        const double t = piv > 1e-14 * trace ? sqrt(piv) : 0.0;
        G[j * ldgb + j] = t;
        red[1] = t > 0.0 ? 1.0 / t : 0.0;
      }
      __syncthreads();
      const double rt = red[1], rt2 = rt * rt;
      for (int i = j + 1 + tid; i < b; i += nthr) G[j * ldgb + i] = G[i * ldgb + j] * rt;
      // the trailing lower triangle: a warp per row, lanes over its columns
      for (int i = j + 1 + warp; i < b; i += nthr / 32) {
        const double gi = -G[i * ldgb + j] * rt2;
        for (int k = j + 1 + lane; k <= i; k += 32) G[i * ldgb + k] = fma(gi, G[k * ldgb + j], G[i * ldgb + k]);
      }
      __syncthreads();
    }
    float* Tf = region(kRgTf);
    for (int e = tid; e < b * b; e += nthr) {  // column c of T^T = L: L[k][c], k >= c
      const int c = e / b, k = e % b;
      Tf[(long)c * ldrT + k] = k > c ? (float)G[c * ldgb + k] : (k == c ? (float)G[c * ldgb + c] : 0.f);
    }
    __syncthreads();
  } else if (tr) {
    for (long e = tid; e < (long)b * n; e += nthr) XR[e] = Rm[e];
    __syncthreads();
    for (long e = tid; e < (long)b * n; e += nthr) {  // column i of R^T: R[i][0..b)
      const int i = (int)(e / b), j = (int)(e % b);
      Rm[(long)i * ldr + j] = XR[(long)j * n + i];
    }
    __syncthreads();
  }
  int sw;
  if (chol) {
    if (voff + b <= 32) {  // the whole factor fits one warp's registers
      if (warp == 0) {
        // on L's columns (T's rows, 16 rows held as 4 per lane), nothing
        // accumulated: with T = U_T S V^T the rotated columns are V S
        const int w = warp_hestenes16<4>(Tm, b, 16, b, ldr, 1.2e-7f * sqrtf((float)b) + 2.4e-7f,
                                         30, inv_x2);
        if (lane == 0) s_m = w;
      }
      __syncthreads();
      sw = s_m;
    } else {  // (not reached for b <= 16) the same, by the CTA
      sw = cta_hestenes_any<float>(Tm, b, voff, b, ldr, 1.2e-7f * sqrtf((float)b) + 2.4e-7f, 30,
                                   inv_x2, false);
    }
    __syncthreads();
    cta_colnorm_order(Tm, b, b, ldr, sv, ordh);
  } else {
    if (bigg) {
      float* Tf = region(kRgTf);
      // a preconditioner only (the Jacobi on R V below sets the accuracy), fp32
      // sums: one-sided Jacobi on T^T (T's rows), nothing accumulated -- with
      // T = U_T S V_T^T the rotated columns are V_T S, so V_T = the columns over
      // their norms.  A numerically null column leaves V_T = I (no preconditioning).
      plain_hestenes(Tf, b, voffT, b, ldrT, 1.2e-7f * sqrtf((float)b) + 2.4e-7f, 30, inv_x2);
      __syncthreads();
      cta_colnorm_order(Tf, b, b, ldrT, sv, ordh);  // sv = the column norms (order unused)
      if (tid == 0) {
        double smax = 0.0;
        for (int j = 0; j < b; ++j) smax = fmax(smax, sv[j]);
        int deg = !(smax > 0.0);
        for (int j = 0; j < b; ++j) deg |= !(sv[j] > 1e-6 * smax);
        s_degenerate = deg;
      }
      __syncthreads();
      if (s_degenerate) {
        for (int e = tid; e < b * ldrT; e += nthr) Tf[e] = (e / ldrT == e % ldrT) ? 1.f : 0.f;
      } else {
        for (int e = tid; e < b * b; e += nthr) {
          const int j = e / b, l = e % b;
          Tf[(long)j * ldrT + l] = (float)((double)Tf[(long)j * ldrT + l] / sv[j]);
        }
      }
      __syncthreads();
      for (long e = tid; e < (long)b * n; e += nthr) XR[e] = Rm[e];  // R, contiguous columns
      __syncthreads();
      const int bq = (b + 3) / 4;
      if (n % 4 == 0 && ldr % 4 == 0) {
        // 4 rows x 4 columns per thread: one 16-byte load of R's column l
        // feeds 16 products (same summation order per element as below)
        const int nq = n / 4;
        for (long e = tid; e < (long)bq * nq; e += nthr) {
          const int jq = (int)(e / nq), i0 = 4 * (int)(e % nq);
          const int j0 = 4 * jq;
          const float* vc[4];
          bool hv[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            hv[c] = j0 + c < b;
            vc[c] = Tf + (long)(hv[c] ? j0 + c : j0) * ldrT;
          }
          float acc[4][4] = {};
#pragma unroll 2
          for (int l = 0; l < b; ++l) {
            const float4 x = *reinterpret_cast<const float4*>(XR + (long)l * n + i0);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const float v = vc[c][l];
              acc[c][0] = fmaf(x.x, v, acc[c][0]);
              acc[c][1] = fmaf(x.y, v, acc[c][1]);
              acc[c][2] = fmaf(x.z, v, acc[c][2]);
              acc[c][3] = fmaf(x.w, v, acc[c][3]);
            }
          }
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (hv[c])
              *reinterpret_cast<float4*>(Rm + (long)(j0 + c) * ldr + i0) =
                  make_float4(acc[c][0], acc[c][1], acc[c][2], acc[c][3]);
        }
      } else {
      for (long e = tid; e < (long)bq * n; e += nthr) {  // R V into the augmented columns,
        const int jq = (int)(e / n), i = (int)(e % n);   // four columns per thread
        const int j0 = 4 * jq;
        const float* v0 = Tf + (long)j0 * ldrT;
        const bool h1 = j0 + 1 < b, h2 = j0 + 2 < b, h3 = j0 + 3 < b;
        const float* v1 = h1 ? v0 + ldrT : v0;
        const float* v2 = h2 ? v0 + 2 * ldrT : v0;
        const float* v3 = h3 ? v0 + 3 * ldrT : v0;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 4
        for (int l = 0; l < b; ++l) {
          const float x = XR[(long)l * n + i];
          a0 = fmaf(x, v0[l], a0);
          a1 = fmaf(x, v1[l], a1);
          a2 = fmaf(x, v2[l], a2);
          a3 = fmaf(x, v3[l], a3);
        }
        Rm[(long)j0 * ldr + i] = a0;
        if (h1) Rm[(long)(j0 + 1) * ldr + i] = a1;
        if (h2) Rm[(long)(j0 + 2) * ldr + i] = a2;
        if (h3) Rm[(long)(j0 + 3) * ldr + i] = a3;
      }
      }
      for (int e = tid; e < b * b; e += nthr) {  // and V below them, the Jacobi's start
        const int j = e / b, l = e % b;
        Rm[(long)j * ldr + voff + l] = Tf[(long)j * ldrT + l];
      }
      __syncthreads();
    }
    sw = cta_hestenes_any<double>(Rm, rlen, voff, nsv, ldr,
                                  1.2e-7f * sqrtf((float)rlen) + 2.4e-7f, 30, inv_x2, true, 32, bigg);
    __syncthreads();
    cta_colnorm_order(Rm, rlen, nsv, ldr, sv, ordh);
  }
  if (sw >= 30 && tid == 0) atomicOr(&A.status[kStatusNumeric], 1);
  if (tid == 0) {
    const float xnorm = (float)sqrt(s_xnorm2);
    const double tol = 100.0 * (double)FLT_EPSILON * (double)xnorm;
    int m;
    if (r == 0) {
      m = nsv;
    } else {
      m = 0;
      for (int j = 0; j < nsv; ++j)
        if ((double)(float)sv[ordh[j]] > tol) ++m;
      m = min(m, max(0, n - r));
    }
    s_m = m;
    // a kept direction far below the largest is numerically null: its column
    // is rounding noise and must be completed to an orthonormal direction
    const double s0 = sv[ordh[0]];
    if (!isfinite(s0)) atomicOr(&A.status[kStatusNumeric], 4);
    int deg = 0;
    for (int j = 0; j < m; ++j)
      if (!(sv[ordh[j]] > 1e-6 * s0) || s0 == 0.0) deg = 1;
    s_degenerate = deg;
  }
  __syncthreads();
  const int m = s_m;
  float* Q = XR;  // [m][n]
  if (chol) {
    // q_j = R v_j / s_j = R x_j / s_j^2, x_j = s_j v_j the rotated column
    // (rows b..15 of the factor's columns are zero): 1/s_j^2 in fp64 first,
    // then a thread per row i holds R's row and runs over the columns
    if (tid < m) {
      const double sj = sv[ordh[tid]];
      nrm[tid] = sj > 0.0 ? 1.0 / (sj * sj) : 0.0;
    }
    __syncthreads();
    for (int i = tid; i < n; i += nthr) {
      float rrow[16];
#pragma unroll
      for (int l = 0; l < 16; ++l) rrow[l] = l < b ? Rm[l * n + i] : 0.f;
      for (int j = 0; j < m; ++j) {
        const float4* xj = reinterpret_cast<const float4*>(Tm + ordh[j] * ldr);
        float acc = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 x4 = xj[q];
          acc = fmaf(rrow[4 * q], x4.x, acc);
          acc = fmaf(rrow[4 * q + 1], x4.y, acc);
          acc = fmaf(rrow[4 * q + 2], x4.z, acc);
          acc = fmaf(rrow[4 * q + 3], x4.w, acc);
        }
        Q[j * n + i] = (float)((double)acc * nrm[j]);
      }
    }
  } else {
    for (long e = tid; e < (long)m * n; e += nthr) {
      const int j = (int)(e / n), i = (int)(e % n);
      const int oj = ordh[j];
      if (!tr) {  // q_j = (R V)[:, o_j] / s_j
        const double sj = sv[oj];
        Q[e] = sj > 0.0 ? (float)(Rm[(long)oj * ldr + i] / sj) : 0.f;
      } else {    // q_j = J[:, o_j]
        Q[e] = Rm[(long)oj * ldr + voff + i];
      }
    }
  }
  __syncthreads();
  if (s_degenerate) cta_cgs2_rows(Q, m, n, nrm, red);
  // ----- the core B = [[diag(sigma), a], [0, diag(s_m) V_m^T]] ((r+m) x (r+b)):
  // its left singular vectors W and values by one-sided Jacobi on B^T, with
  // W accumulated below each column.
  const int N = r + m, LB = r + b;
  const int woff = (LB + 3) & ~3;
  for (long e = tid; e < (long)N * LB; e += nthr) {
    const int c = (int)(e / LB), row = (int)(e % LB);
    float v = 0.f;
    if (c < r) {
      if (row < r) v = (row == c) ? sig[c] : 0.f;
      else v = AS[c * b16 + (row - r)];
    } else if (row >= r) {  // s_j v_j^T, the residual's right part
      const int oj = ordh[c - r], l = row - r;
      v = tr ? Rm[(long)oj * ldr + l]
             : (chol ? Tm[(long)oj * ldr + l] : (float)sv[oj] * Rm[(long)oj * ldr + voff + l]);
    }
    BT[(long)c * ldbt + row] = v;
  }
  __syncthreads();
  double b2 = s_xnorm2;  // ||B||_F^2 <= ||sigma||^2 + ||X||_F^2 sets the core's scale
  for (int c = 0; c < r; ++c) b2 += (double)sig[c] * sig[c];
  sw = core_hestenes(BT, LB, woff, N, ldbt, 1.2e-7f * sqrtf((float)LB) + 2.4e-7f, 30,
                     b2 > 0.0 ? 1.0 / b2 : 1.0);
  __syncthreads();
  cta_colnorm_order(BT, LB, N, ldbt, nrm, ord);
  if (sw >= 30 && tid == 0) atomicOr(&A.status[kStatusNumeric], 2);
  if (tid == 0) {
    int keep = min(cap, N);
    if (A.has_theta && N > 0) {
      // smallest k with sqrt(sum_{j>=k} sigma_j^2) <= theta (fp32, as the reference)
      const float th2 = A.theta * A.theta;
      int first_ok = -1;
      float tail = 0.f;
      for (int k = N - 1; k >= 0; --k) {
        const float sk = (float)nrm[ord[k]];
        tail += sk * sk;
        if (tail <= th2) first_ok = k;
      }
      const int tr_ = (first_ok < 0) ? N : max(1, first_ok);
      keep = max(1, min(keep, tr_));
    }
    s_keep = keep;
  }
  __syncthreads();
  const int keep = s_keep;
  for (int c = tid; c < keep; c += nthr) sig[c] = (float)nrm[ord[c]];
  float* CB = A2;  // [keep][b16] the block's coordinates W^T B[:, r:], ordered
  for (int e = tid; e < N * ldw; e += nthr) {  // WU[k][c] = W[k][ord_c], zero past keep
    const int k = e / ldw, c = e % ldw;
    WU[e] = c < keep ? BT[(long)ord[c] * ldbt + woff + k] : 0.f;
  }
  for (int e = tid; e < keep * b; e += nthr) {  // the rotated B^T column holds (B^T w_c)[r + j]
    const int c = e / b, j = e % b;
    CB[c * b16 + j] = BT[(long)ord[c] * ldbt + r + j];
  }
  __syncthreads();
  // ----- U_new = U W[:r] + Q^T W[r:], then one Newton-Schulz step to orthonormal.
  // Up to 32 columns with everything staged: U_new is formed in place of the
  // staged U (each thread owns its rows) and polished from there.
  const bool un_smem = kSmem && keep <= 32;
  const bool tiles = un_smem && n % 4 == 0 && ldp % 4 == 0 && ldw % 4 == 0 && nthr == kStepThreads;
  if (tiles) {
    float* Un = pool + P.smem[kRgUs];
    cta_basis_tiles(n, keep, r, m, Un, P.ldu, Q, WU, ldw);
    cta_tn_tiles(keep, keep, n, Un, P.ldu, Un, P.ldu, Pol, ldp, 1.f, part);  // E = U^T U - I
  } else if (un_smem) {
    float* Un = pool + P.smem[kRgUs];
    cta_basis_rows32(n, keep, r, m, Un, P.ldu, Q, WU, ldw);
    cta_tn(keep, keep, n, Un, P.ldu, Un, P.ldu, true, Pol, ldp, 1.f, part);  // E = U^T U - I
  } else {
    cta_basis_rows(n, keep, r, m, Uc, lda, Q, WU, ldw, Uo, ld, uvec);
    cta_tn(keep, keep, n, Uo, ld, Uo, ld, uvec, Pol, ldp, 1.f, part);
  }
  for (int e = tid; e < ldp * ldp; e += nthr) {
    const int k = e / ldp, c = e % ldp;
    if (k >= keep || c >= keep) Pol[e] = 0.f;
  }
  __syncthreads();
  // The carry map and the block's coordinates refer to the polished basis
  // U' = U (I - E/2):  rot' = U'^T U_old = (I - E/2) W[:r]^T and
  // c' = U'^T x = (I - E/2) W^T B[:, r:], where the rotated B^T column of
  // ordered value c holds W^T B's row c (its rows r.. are (B^T w_c)[r + j]).
  float* rot = A.rot + p * A.rot_sp;
  for (int e = tid; e < keep * r; e += nthr) {  // rot'[c][k] = W[k][c] - 1/2 sum_d W[k][d] E[d][c]
    const int k = e / keep, c = e % keep;
    const float* wr = WU + (long)k * ldw;
    float corr = 0.f;
    for (int d = 0; d < keep; ++d) corr = fmaf(wr[d], Pol[(long)d * ldp + c], corr);
    rot[c * ld + k] = fmaf(-0.5f, corr, wr[c]);
  }
  float* co = A.coords + p * A.coords_sp;
  for (int e = tid; e < keep * b; e += nthr) {  // c'[j][c] = CB[c][j] - 1/2 sum_d E[d][c] CB[d][j]
    const int j = e / keep, c = e % keep;   // (E is exactly symmetric: both halves sum alike)
    float corr = 0.f;
    for (int d = 0; d < keep; ++d) corr = fmaf(Pol[(long)d * ldp + c], CB[d * b16 + j], corr);
    co[(long)j * A.coords_ld + c] = fmaf(-0.5f, corr, CB[c * b16 + j]);
  }
  if (tiles) {
    cta_polish_tiles(n, keep, pool + P.smem[kRgUs], P.ldu, Uo, ld, uvec, Pol, ldp);
  } else if (un_smem) {
    cta_polish_rows(n, keep, pool + P.smem[kRgUs], P.ldu, true, Uo, ld, uvec, Pol, ldp);
  } else if (keep <= 32) {
    cta_polish_rows(n, keep, Uo, ld, uvec, Uo, ld, uvec, Pol, ldp);
  } else {
    float* WU2 = region(kRgWu2);  // W (I - E/2), then the basis is formed again
    for (int e = tid; e < N * ldw; e += nthr) {
      const int k = e / ldw, c = e % ldw;
      float v = 0.f;
      if (c < keep) {
        v = WU[e];
        for (int d = 0; d < keep; ++d) v = fmaf(-0.5f * WU[(long)k * ldw + d], Pol[(long)d * ldp + c], v);
      }
      WU2[e] = v;
    }
    __syncthreads();
    cta_basis_rows(n, keep, r, m, Uc, lda, Q, WU2, ldw, Uo, ld, uvec);
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

// The same carry with each thread owning two token rows (t, t + W/2 of the
// CTA's range): the rows (R >= r_old floats, read as 16-byte vectors) and
// their R outputs stay in registers, and every rot^T vector broadcast from
// shared memory feeds both rows.  Needs ld % 4 == 0 and ld <= R.
template <int R>
__global__ void __launch_bounds__(256) carry_reg_kernel(CarryBatch batch) {
  extern __shared__ __align__(16) float rsm[];  // rotT [R][R]
  const CarryArgs A = blockIdx.z ? batch.s[1] : batch.s[0];  // no dynamic indexing of the parameter
  const int p = blockIdx.y;
  const int r_old = A.dims[4 * p], keep = A.dims[4 * p + 1];
  const int ld = A.ld;
  if (r_old == 0) return;
  const float* rot = A.rot + p * A.rot_sp;
  for (int e = threadIdx.x; e < R * R; e += blockDim.x) {
    const int k = e / R, c = e % R;
    rsm[e] = (k < r_old && c < keep) ? rot[c * ld + k] : 0.f;
  }
  __syncthreads();
  const int t0 = blockIdx.x * 2 * blockDim.x + threadIdx.x;
  const int t1 = t0 + blockDim.x;
  if (t0 >= batch.W) return;
  const bool two = t1 < batch.W;
  float* c0 = A.c + p * A.c_sp + (long)t0 * ld;
  float* c1 = A.c + p * A.c_sp + (long)(two ? t1 : t0) * ld;
  float row0[R], row1[R];
#pragma unroll
  for (int q = 0; q < R / 4; ++q) {
    float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
    if (4 * q < ld) {
      v0 = reinterpret_cast<const float4*>(c0)[q];
      v1 = reinterpret_cast<const float4*>(c1)[q];
    }
    const float a0[4] = {v0.x, v0.y, v0.z, v0.w}, a1[4] = {v1.x, v1.y, v1.z, v1.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      row0[4 * q + i] = 4 * q + i < r_old ? a0[i] : 0.f;
      row1[4 * q + i] = 4 * q + i < r_old ? a1[i] : 0.f;
    }
  }
  float acc0[R], acc1[R];
#pragma unroll
  for (int c = 0; c < R; ++c) { acc0[c] = 0.f; acc1[c] = 0.f; }
  const float4* rt4 = reinterpret_cast<const float4*>(rsm);
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const float x0 = row0[k], x1 = row1[k];
#pragma unroll
    for (int q = 0; q < R / 4; ++q) {
      const float4 w = rt4[k * (R / 4) + q];
      acc0[4 * q] = fmaf(w.x, x0, acc0[4 * q]);
      acc0[4 * q + 1] = fmaf(w.y, x0, acc0[4 * q + 1]);
      acc0[4 * q + 2] = fmaf(w.z, x0, acc0[4 * q + 2]);
      acc0[4 * q + 3] = fmaf(w.w, x0, acc0[4 * q + 3]);
      acc1[4 * q] = fmaf(w.x, x1, acc1[4 * q]);
      acc1[4 * q + 1] = fmaf(w.y, x1, acc1[4 * q + 1]);
      acc1[4 * q + 2] = fmaf(w.z, x1, acc1[4 * q + 2]);
      acc1[4 * q + 3] = fmaf(w.w, x1, acc1[4 * q + 3]);
    }
  }
#pragma unroll
  for (int q = 0; q < R / 4; ++q) {
    if (4 * q + 3 < keep) {
      reinterpret_cast<float4*>(c0)[q] = make_float4(acc0[4 * q], acc0[4 * q + 1], acc0[4 * q + 2], acc0[4 * q + 3]);
      if (two) reinterpret_cast<float4*>(c1)[q] = make_float4(acc1[4 * q], acc1[4 * q + 1], acc1[4 * q + 2], acc1[4 * q + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (4 * q + i < keep) {
          c0[4 * q + i] = acc0[4 * q + i];
          if (two) c1[4 * q + i] = acc1[4 * q + i];
        }
    }
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
  extern __shared__ unsigned skey[];
  __shared__ int scan_scratch[32];
  const int p = blockIdx.x;
  const float* s = scores + (long)p * m;
  for (int i = threadIdx.x; i < m; i += blockDim.x) skey[i] = order_key(s[i]);
  __syncthreads();
  int keep_base = 0, dem_base = 0;
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
}  // namespace kvd

// ---------------------------------------------------------------- host glue

namespace kvd_host {

using namespace kvd;

// Buffer placement for one launch.  Every region gets a workspace slot; the
// regions that fit (in priority order) are staged in shared memory.
static StepPlan plan_bug_step(int n, int b, int ld, long pool_max_floats) {
  StepPlan P;
  const long N = (long)ld + b;
  P.b16 = (b + 15) & ~15;
  P.ldb = P.b16 + 4;  // = 4 mod 8: a quarter-warp reading 8 rows as float4 is conflict-free
  // = 4 mod 8: one thread per row reading its row as float4 (a quarter-warp
  // covers 8 rows) and a warp reading a row as a broadcast are conflict-free
  P.ldu = (ld + 3) & ~3;
  if (P.ldu % 8 == 0) P.ldu += 4;
  // B^T rows (<= ld + b) then W rows (<= ld + b), padded for the largest tile
  P.ldbt = 0;
  for (int nn = 1; nn <= N; ++nn) {
    const int pb = jacobi_pitch((int)((N + 3) & ~3L) + nn, nn, false);
    if (pb > P.ldbt) P.ldbt = pb;
  }
  P.ldbt = (P.ldbt + 3) & ~3;
  P.ldw = (ld + 15) & ~15;
  P.ldp = P.ldw > 32 ? P.ldw : 32;
  long fl[kRgCount];
  // residual columns with their rotations below: min(n, b) columns of
  // round4(n) + round4(b) rows (b > n transposes R first)
  {
    const int nsv = n < b ? n : b, rlen = n < b ? b : n;
    fl[kRgRm] = (long)nsv * jacobi_pitch(((rlen + 3) & ~3) + nsv, nsv, true);
  }
  if (fl[kRgRm] < (long)b * n) fl[kRgRm] = (long)b * n;
  fl[kRgXr] = (long)n * P.ldb;
  fl[kRgPart] = kPartFloats;
  fl[kRgAs] = (long)ld * P.b16;
  fl[kRgA2] = (long)ld * P.b16;
  fl[kRgSmall] = 3 * (N + b) + 8;
  fl[kRgCore] = N * P.ldbt;
  fl[kRgPol] = (long)P.ldp * P.ldp;
  fl[kRgWu] = N * P.ldw;
  fl[kRgWu2] = N * P.ldw;
  fl[kRgUs] = (long)n * P.ldu;
  // blocks of 17..kMaxGramB columns factor the Gram (b x (b+1) doubles) and
  // run the Jacobi (fp64 accumulation) on the b x b factor's columns with
  // their rotations below
  const bool big_chol = b > 16 && b <= kMaxGramB && b <= n;
  fl[kRgGram] = big_chol ? 2L * b * (b + 1) : 0;
  fl[kRgTf] = big_chol ? (long)b * jacobi_pitch((b + 3) & ~3, b, false) : 0;
  long wo = 0;
  for (int g = 0; g < kRgCount; ++g) {
    P.ws[g] = g == kRgUs ? -1 : wo;
    if (g != kRgUs) wo += align16(4 * fl[g]) + 128;
  }
  P.ws_bytes = align16(wo);
  const int prio[] = {kRgRm, kRgXr, kRgPart, kRgTf, kRgAs, kRgA2, kRgSmall,
                      kRgCore, kRgPol, kRgWu, kRgUs, kRgWu2, kRgGram};
  long used = 0;
  for (int g = 0; g < kRgCount; ++g) P.smem[g] = -1;
  for (int g : prio) {
    const long sz = (fl[g] + 31) & ~31L;  // 128-byte aligned slots
    if (used + sz <= pool_max_floats) {
      P.smem[g] = used;
      used += sz;
    }
  }
  // Wide blocks (the pre-fill blocks): the core would not fit beside the
  // residual's regions, and its Jacobi is the longest phase.  The core then
  // takes the shared memory from offset 0, overlapping the K-split partials
  // and the factor's columns: both are dead from the core's build on (the
  // build reads a, the residual's right factor and the small scalars), and
  // the partials serve again only as scratch for U_new's Gram, after the
  // core has been read out.  a and the small scalars sit after the core.
  const long sz_core = (fl[kRgCore] + 31) & ~31L, sz_as = (fl[kRgAs] + 31) & ~31L;
  const long sz_small = (fl[kRgSmall] + 31) & ~31L;
  const long sz_part = (fl[kRgPart] + 31) & ~31L, sz_tf = (fl[kRgTf] + 31) & ~31L;
  if (b > 16 && P.smem[kRgCore] < 0 && sz_core + sz_as + sz_small <= pool_max_floats &&
      sz_part + sz_tf <= sz_core) {
    for (int g = 0; g < kRgCount; ++g) P.smem[g] = -1;
    P.smem[kRgCore] = 0;
    P.smem[kRgPart] = 0;
    P.smem[kRgTf] = fl[kRgTf] ? sz_part : -1;
    P.smem[kRgAs] = sz_core;
    P.smem[kRgSmall] = sz_core + sz_as;
    used = sz_core + sz_as + sz_small;
    for (int g : prio) {  // what else fits goes after them (never over the core)
      if (P.smem[g] >= 0 || g == kRgPart || g == kRgTf) continue;
      const long sz = (fl[g] + 31) & ~31L;
      if (used + sz <= pool_max_floats) {
        P.smem[g] = used;
        used += sz;
      }
    }
  }
  P.smem_bytes = (int)(kStepMiscBytes + 4 * used);
  return P;
}

long bug_step_ws_per_problem(int n, int b, int ld) { return plan_bug_step(n, b, ld, 0).ws_bytes; }

// Dynamic shared memory a BUG-step launch may plan with on the current
// device: the opt-in limit less the kernels' static shared memory, looked up
// once per device under a lock (0 on error, with the message set).
static int step_max_dyn_smem() {
  static std::mutex mu;
  static int per_dev[kMaxDevices] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("bug step: no usable current device (%s)", cudaGetErrorString(e));
    return 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!per_dev[dev]) {
    cudaFuncAttributes a1, a2;
    int optin = 0;
    e = cudaFuncGetAttributes(&a1, (const void*)bug_step_kernel<true>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a2, (const void*)bug_step_kernel<false>);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) {
      set_error("bug step: %s", cudaGetErrorString(e));
      return 0;
    }
    const int st = (int)(a1.sharedSizeBytes > a2.sharedSizeBytes ? a1.sharedSizeBytes : a2.sharedSizeBytes);
    per_dev[dev] = optin - st;
  }
  return per_dev[dev];
}

int launch_bug_step(const BugStepBatch& batch_in, int n_problems, int n_streams, cudaStream_t stream) {
  const int max_dyn = step_max_dyn_smem();
  if (max_dyn <= kStepMiscBytes) return KVD_ERR_CUDA;
  BugStepBatch batch = batch_in;
  const BugStepArgs& a0 = batch.s[0];
  if (a0.ld > kMaxStepLd) {
    set_error("bug step: basis width %d exceeds %d", a0.ld, kMaxStepLd);
    return KVD_ERR_ARG;
  }
  batch.plan = plan_bug_step(a0.n, a0.b, a0.ld, (max_dyn - kStepMiscBytes) / 4);
  if (a0.ws_sp < batch.plan.ws_bytes) {
    set_error("bug step: workspace stride %ld < %ld bytes", a0.ws_sp, batch.plan.ws_bytes);
    return KVD_ERR_WORKSPACE;
  }
  bool all_smem = true;
  for (int g = 0; g < kRgCount; ++g) all_smem = all_smem && batch.plan.smem[g] >= 0;
  const int smem = batch.plan.smem_bytes;
  const void* fn = all_smem ? (const void*)bug_step_kernel<true> : (const void*)bug_step_kernel<false>;
  if (int rc = ensure_smem(fn, smem, "bug_step_kernel")) return rc;
  dim3 grid(n_problems, n_streams);
  {
    KTimerScope kts_("bug_step_kernel", stream);
    if (all_smem) bug_step_kernel<true><<<grid, kStepThreads, smem, stream>>>(batch);
    else bug_step_kernel<false><<<grid, kStepThreads, smem, stream>>>(batch);
  }
  return check_launch("bug_step_kernel");
}

int launch_carry(const CarryBatch& batch, int n_problems, int n_streams, int ld, cudaStream_t stream) {
  if (batch.W <= 0) return KVD_OK;
  bool aligned = ld % 4 == 0;
  for (int i = 0; i < n_streams; ++i)
    aligned = aligned && (reinterpret_cast<uintptr_t>(batch.s[i].c) % 16 == 0) && batch.s[i].c_sp % 4 == 0;
  if (aligned && ld <= 64) {
    if (ld > 32)
      if (int rc = ensure_smem((const void*)carry_reg_kernel<64>, 4 * 64 * 64, "carry_kernel")) return rc;
    KTimerScope kts_("carry_kernel", stream);
    if (ld <= 32) {  // 128 threads x 2 rows: ~170 registers each, several CTAs per SM
      dim3 grid((batch.W + 255) / 256, n_problems, n_streams);
      carry_reg_kernel<32><<<grid, 128, 4 * 32 * 32, stream>>>(batch);
    } else {
      dim3 grid((batch.W + 511) / 512, n_problems, n_streams);
      carry_reg_kernel<64><<<grid, 256, 4 * 64 * 64, stream>>>(batch);
    }
    return check_launch("carry_kernel");
  }
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
    const cudaError_t e = cudaMemcpy2DAsync(m_out, sizeof(int32_t), dims + 2, 4 * sizeof(int),
                                            sizeof(int32_t), n_batch, cudaMemcpyDeviceToDevice,
                                            (cudaStream_t)stream);
    if (e != cudaSuccess) {
      set_error("kvd_bug_step: copying m: %s", cudaGetErrorString(e));
      return KVD_ERR_CUDA;
    }
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
