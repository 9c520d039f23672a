// Verbatim-tier kernels (sm_100a): HF (B,H,T,D) <-> token-major rows, ring
// compaction, and the dense peek [sinks | exact tier | RoPE(U_k C_k) | ring |
// tail] that the reference returns from update() (bug_cache.py:1496-1575,
// 1390-1402).  The reconstructed middle is computed in fp32 and cast to the
// model dtype, as the reference's _ensure_mid_cache does.
#include "kernels.cuh"

namespace kvd {

// rows[p][slot0 + t][h*D + d] = src[b][h][t][d]   (p = b)
// One side (keys or values) of an HF-layout to ring-rows copy.
template <typename T>
struct HfRowsSide { const T* src; long sb, sh, st; T* dst; };
template <typename T>
struct HfRowsPair { HfRowsSide<T> s[2]; };

template <typename T>
__global__ void hf_to_rows_kernel(HfRowsPair<T> pr, int H, int D, int q, long dst_sp, int slot0) {
  const int p = blockIdx.y;
  const HfRowsSide<T> sd = blockIdx.z ? pr.s[1] : pr.s[0];  // keys, values
  const T* src = sd.src;
  const long sb = sd.sb, sh = sd.sh, st = sd.st;
  T* dst = sd.dst;
  const int n = H * D;
  const long tot = (long)q * n;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < tot; e += (long)gridDim.x * blockDim.x) {
    const int t = (int)(e / n), i = (int)(e % n);
    const int h = i / D, d = i % D;
    dst[p * dst_sp + (long)(slot0 + t) * n + i] = src[p * sb + h * sh + (long)t * st + d];
  }
}

// The same copy in 16-byte pieces (8 bf16 or 4 fp32 of one head's row), for
// views whose pointers, strides and head size are whole pieces.
template <typename T>
__global__ void hf_to_rows_vec_kernel(HfRowsPair<T> pr, int H, int D, int q, long dst_sp, int slot0) {
  constexpr int kPer = 16 / sizeof(T);
  const int p = blockIdx.y;
  const HfRowsSide<T> sd = blockIdx.z ? pr.s[1] : pr.s[0];  // keys, values
  const int dc = D / kPer, per_t = H * dc, n = H * D;
  const int tot = q * per_t;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < tot; e += gridDim.x * blockDim.x) {
    const int t = e / per_t, rem = e % per_t, h = rem / dc, d = (rem % dc) * kPer;
    const uint4 v = *reinterpret_cast<const uint4*>(sd.src + p * sd.sb + h * sd.sh + (long)t * sd.st + d);
    *reinterpret_cast<uint4*>(sd.dst + p * dst_sp + (long)(slot0 + t) * n + h * D + d) = v;
  }
}

// dst rows [0, count) <- src rows [0, count) of the same problem (copy).
template <typename T>
__global__ void rows_copy_kernel(const T* src, long src_sp, T* dst, long dst_sp, int count, int n) {
  const int p = blockIdx.y;
  const long tot = (long)count * n;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < tot; e += (long)gridDim.x * blockDim.x)
    dst[p * dst_sp + e] = src[p * src_sp + e];
}

// In-place move of rows [head, head+len) to [0, len): one CTA per problem,
// staged through shared memory chunk by chunk (destination < source).
template <typename T>
__global__ void __launch_bounds__(1024) ring_compact_kernel(T* ring, long sp, int head, int len, int n) {
  extern __shared__ __align__(16) unsigned char rsm[];
  T* stage = reinterpret_cast<T*>(rsm);
  const int p = blockIdx.x;
  T* base = ring + p * sp;
  const int chunk_elems = 8192;
  const long tot = (long)len * n;
  for (long c0 = 0; c0 < tot; c0 += chunk_elems) {
    const int cnt = (int)((tot - c0) < chunk_elems ? (tot - c0) : chunk_elems);
    for (int e = threadIdx.x; e < cnt; e += blockDim.x) stage[e] = base[(long)head * n + c0 + e];
    __syncthreads();
    for (int e = threadIdx.x; e < cnt; e += blockDim.x) base[c0 + e] = stage[e];
    __syncthreads();
  }
}

struct PeekSeg {
  const void* k; const void* v; long sp;  // token-major rows [p][slot][n]
  int len;
};

// Verbatim segments -> HF output rows [l0, l0 + len).
template <typename T>
__global__ void rows_to_hf_kernel(const T* k, const T* v, long sp, int len, int H, int D, T* ok,
                                  T* ov, long ob, long oh, long ot, int l0) {
  const int p = blockIdx.y;
  const int n = H * D;
  const long tot = (long)len * n;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < tot; e += (long)gridDim.x * blockDim.x) {
    const int t = (int)(e / n), i = (int)(e % n);
    const int h = i / D, d = i % D;
    const long o = p * ob + h * oh + (long)(l0 + t) * ot + d;
    ok[o] = k[p * sp + e];
    ov[o] = v[p * sp + e];
  }
}

// The same in 16-byte pieces (8 bf16 or 4 fp32 of one head's row), for
// outputs whose pointers, strides and head size are whole pieces.
template <typename T>
__global__ void rows_to_hf_vec_kernel(const T* k, const T* v, long sp, int len, int H, int D, T* ok,
                                      T* ov, long ob, long oh, long ot, int l0) {
  constexpr int kPer = 16 / sizeof(T);
  const int p = blockIdx.y;
  const int dc = D / kPer, per_t = H * dc, n = H * D;
  const int tot = len * per_t;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < tot; e += gridDim.x * blockDim.x) {
    const int t = e / per_t, rem = e % per_t, h = rem / dc, d = (rem % dc) * kPer;
    const long src = p * sp + (long)t * n + h * D + d;
    const long o = p * ob + h * oh + (long)(l0 + t) * ot + d;
    *reinterpret_cast<uint4*>(ok + o) = *reinterpret_cast<const uint4*>(k + src);
    *reinterpret_cast<uint4*>(ov + o) = *reinterpret_cast<const uint4*>(v + src);
  }
}

// HF tail (B,H,q,D) -> HF output rows [l0, l0+q).
template <typename T>
__global__ void hf_to_hf_kernel(const T* k, const T* v, long sb, long sh, long st, int q, int H,
                                int D, T* ok, T* ov, long ob, long oh, long ot, int l0) {
  const int p = blockIdx.y;
  const long tot = (long)q * H * D;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < tot; e += (long)gridDim.x * blockDim.x) {
    const int t = (int)(e / (H * D));
    const int i = (int)(e % (H * D));
    const int h = i / D, d = i % D;
    const long o = p * ob + h * oh + (long)(l0 + t) * ot + d;
    const long s = p * sb + h * sh + (long)t * st + d;
    ok[o] = k[s];
    ov[o] = v[s];
  }
}

// Middle reconstruction: K = RoPE(U_k c_t) at pos_t, V = U_v c_v,t for 32
// coordinate columns per CTA, written to HF rows [l0, l0+W).  The basis rows of
// one head are staged transposed ([c][d]) so a warp reads 32 consecutive d.
constexpr int kMidTile = 32;

template <typename T>
__global__ void __launch_bounds__(256) mid_hat_kernel(const float* uk, const float* uv, long u_sp,
                                                      int ld, const int* rk, const int* rv,
                                                      const float* ck, const float* cv, long c_sp,
                                                      const int* mid_pos, long mid_sp,
                                                      int pos_base, int W, int H, int D,
                                                      const float* inv_freq, float scale, T* ok,
                                                      T* ov, long ob, long oh, long ot, int l0) {
  extern __shared__ __align__(16) float msm[];
  const int p = blockIdx.y;
  const int t0 = blockIdx.x * kMidTile;
  const int cnt = min(kMidTile, W - t0);
  const int r_k = rk[p], r_v = rv[p];
  const int half = D / 2;
  float* ctk = msm;                        // [tile][ld]
  float* ctv = ctk + kMidTile * ld;        // [tile][ld]
  float* ukT = ctv + kMidTile * ld;        // [ld][D]
  float* uvT = ukT + D * ld;               // [ld][D]
  float* cs = uvT + D * ld;                // [tile][half][2]
  for (int e = threadIdx.x; e < cnt * ld; e += blockDim.x) {
    const int t = e / ld, c = e % ld;
    ctk[e] = c < r_k ? ck[p * c_sp + (long)(t0 + t) * ld + c] : 0.f;
    ctv[e] = c < r_v ? cv[p * c_sp + (long)(t0 + t) * ld + c] : 0.f;
  }
  for (int e = threadIdx.x; e < cnt * half; e += blockDim.x) {
    const int t = e / half, f = e % half;
    const int pos = mid_pos ? mid_pos[p * mid_sp + t0 + t] : pos_base + t0 + t;
    float c, s;
    rope_cs(pos, inv_freq[f], scale, &c, &s);
    cs[2 * e] = c;
    cs[2 * e + 1] = s;
  }
  const float* Uk = uk + p * u_sp;
  const float* Uv = uv + p * u_sp;
  const int rmax = max(r_k, r_v);
  for (int h = 0; h < H; ++h) {
    __syncthreads();
    for (int e = threadIdx.x; e < D * ld; e += blockDim.x) {
      const int d = e / ld, c = e % ld;  // coalesced global read along c
      ukT[c * D + d] = c < r_k ? Uk[(long)(h * D + d) * ld + c] : 0.f;
      uvT[c * D + d] = c < r_v ? Uv[(long)(h * D + d) * ld + c] : 0.f;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < cnt * half; e += blockDim.x) {
      const int t = e / half, f = e % half;
      const float* ckt = ctk + t * ld;
      const float* cvt = ctv + t * ld;
      float k1 = 0.f, k2 = 0.f, v1 = 0.f, v2 = 0.f;
      for (int c = 0; c < rmax; ++c) {
        const float a = ckt[c], bv = cvt[c];
        const float* uk_c = ukT + c * D;
        const float* uv_c = uvT + c * D;
        k1 = fmaf(uk_c[f], a, k1);
        k2 = fmaf(uk_c[f + half], a, k2);
        v1 = fmaf(uv_c[f], bv, v1);
        v2 = fmaf(uv_c[f + half], bv, v2);
      }
      float y1, y2;
      rope_apply_pair(k1, k2, cs[2 * e], cs[2 * e + 1], &y1, &y2);
      const long o = p * ob + h * oh + (long)(l0 + t0 + t) * ot;
      store_f<T>(ok + o + f, y1);
      store_f<T>(ok + o + f + half, y2);
      store_f<T>(ov + o + f, v1);
      store_f<T>(ov + o + f + half, v2);
    }
  }
}

// Packed store of N consecutive outputs (N = 2 or 4).
template <typename T, int N> KVD_DEVICE void store_n(T* p, const float* v);
template <> KVD_DEVICE void store_n<float, 2>(float* p, const float* v) {
  *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
}
template <> KVD_DEVICE void store_n<float, 4>(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
template <> KVD_DEVICE void store_n<__nv_bfloat16, 2>(__nv_bfloat16* p, const float* v) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v[0], v[1]);
}
template <> KVD_DEVICE void store_n<__nv_bfloat16, 4>(__nv_bfloat16* p, const float* v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// Register-tiled middle reconstruction (same arithmetic, same order as
// mid_hat_kernel, so the outputs are bit-identical): 64 tokens per CTA, each
// thread owns 4 tokens x FP frequency pairs of one head for K and V, so every
// coordinate / basis vector read from shared memory (16-byte loads) feeds
// 4 x 2*FP FMAs.  Thread tx owns frequencies tx*FP .. tx*FP+FP-1 and their
// partners + D/2, so the outputs leave as packed FP-element stores.
constexpr int kMhTok = 64;
constexpr int kMhCtPitch = kMhTok + 4;   // coordinate tile pitch (bank spread)

template <typename T, int D>
__global__ void __launch_bounds__(256) mid_hat_tiled_kernel(
    const float* uk, const float* uv, long u_sp, int ld, const int* rk, const int* rv,
    const float* ck, const float* cv, long c_sp, const int* mid_pos, long mid_sp, int pos_base,
    int W, int H, const float* inv_freq, float scale, T* ok, T* ov, long ob, long oh, long ot,
    int l0, int rc_cols) {
  constexpr int HALF = D / 2, FP = HALF / 16, NQ = 2 * FP;
  extern __shared__ __align__(16) float msm[];
  const int p = blockIdx.y;
  const int t0 = blockIdx.x * kMhTok;
  const int cnt = min(kMhTok, W - t0);
  const int r_k = rk[p], r_v = rv[p];
  const int rmax = max(r_k, r_v);
  float* ctk = msm;                          // [ld][kMhCtPitch], token-contiguous
  float* ctv = ctk + ld * kMhCtPitch;
  float* usk = ctv + ld * kMhCtPitch;        // [rc_cols][16][NQ]: a chunk of the head's basis
  float* usv = usk + rc_cols * D;
  float* cs = usv + rc_cols * D;             // [kMhTok][HALF][2]
  const int tid = threadIdx.x;
  for (int e = tid; e < kMhTok * ld; e += blockDim.x) {
    const int t = e / ld, c = e % ld;
    const bool in = t < cnt;
    const long g = p * c_sp + (long)(t0 + t) * ld + c;
    ctk[c * kMhCtPitch + t] = in && c < r_k ? ck[g] : 0.f;
    ctv[c * kMhCtPitch + t] = in && c < r_v ? cv[g] : 0.f;
  }
  for (int e = tid; e < cnt * HALF; e += blockDim.x) {
    const int t = e / HALF, f = e % HALF;
    const int pos = mid_pos ? mid_pos[p * mid_sp + t0 + t] : pos_base + t0 + t;
    float c, s;
    rope_cs(pos, inv_freq[f], scale, &c, &s);
    cs[2 * e] = c;
    cs[2 * e + 1] = s;
  }
  const int ty = tid / 16, tx = tid % 16;
  const float* Uk = uk + p * u_sp;
  const float* Uv = uv + p * u_sp;
  for (int h = 0; h < H; ++h) {
    float ak[4][NQ], av[4][NQ];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int q = 0; q < NQ; ++q) { ak[i][q] = 0.f; av[i][q] = 0.f; }
    // the head's basis rows are staged rc_cols rank columns at a time (the
    // whole rank when it fits); the sum over c keeps its order across chunks
    for (int c0 = 0; c0 < rmax; c0 += rc_cols) {
      const int cn = min(rc_cols, rmax - c0);
      __syncthreads();
      for (int e = tid; e < D * cn; e += blockDim.x) {
        const int d = e / cn, cl = e % cn, c = c0 + cl;
        const int hi = d >= HALF, f = hi ? d - HALF : d;
        const int q = (cl * 16 + f / FP) * NQ + hi * FP + f % FP;
        usk[q] = c < r_k ? Uk[(long)(h * D + d) * ld + c] : 0.f;
        usv[q] = c < r_v ? Uv[(long)(h * D + d) * ld + c] : 0.f;
      }
      __syncthreads();
#pragma unroll 4
      for (int cl = 0; cl < cn; ++cl) {
        const int c = c0 + cl;
        const float4 a4 = *reinterpret_cast<const float4*>(ctk + c * kMhCtPitch + 4 * ty);
        const float4 b4 = *reinterpret_cast<const float4*>(ctv + c * kMhCtPitch + 4 * ty);
        const float a[4] = {a4.x, a4.y, a4.z, a4.w}, b[4] = {b4.x, b4.y, b4.z, b4.w};
        float wk[NQ], wv[NQ];
#pragma unroll
        for (int q = 0; q < NQ; q += 4) {
          const float4 x = *reinterpret_cast<const float4*>(usk + (cl * 16 + tx) * NQ + q);
          const float4 y = *reinterpret_cast<const float4*>(usv + (cl * 16 + tx) * NQ + q);
          wk[q] = x.x; wk[q + 1] = x.y; wk[q + 2] = x.z; wk[q + 3] = x.w;
          wv[q] = y.x; wv[q + 1] = y.y; wv[q + 2] = y.z; wv[q + 3] = y.w;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int q = 0; q < NQ; ++q) {
            ak[i][q] = fmaf(wk[q], a[i], ak[i][q]);
            av[i][q] = fmaf(wv[q], b[i], av[i][q]);
          }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = 4 * ty + i;
      if (t >= cnt) continue;
      float y1[FP], y2[FP];
#pragma unroll
      for (int j = 0; j < FP; ++j) {
        const int f = tx * FP + j;
        const float c = cs[2 * (t * HALF + f)], s = cs[2 * (t * HALF + f) + 1];
        rope_apply_pair(ak[i][j], ak[i][FP + j], c, s, &y1[j], &y2[j]);
      }
      const long o = p * ob + h * oh + (long)(l0 + t0 + t) * ot + tx * FP;
      store_n<T, FP>(ok + o, y1);
      store_n<T, FP>(ok + o + HALF, y2);
      store_n<T, FP>(ov + o, &av[i][0]);
      store_n<T, FP>(ov + o + HALF, &av[i][FP]);
    }
  }
}

// Pair store of two consecutive outputs (the accumulator fragment's columns 2t, 2t+1).
template <typename T> KVD_DEVICE void store_pair(T* p, float a, float b);
template <> KVD_DEVICE void store_pair<float>(float* p, float a, float b) {
  *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
template <> KVD_DEVICE void store_pair<__nv_bfloat16>(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}

// The middle reconstruction on warp-level TF32 MMA (SPLIT = 3xTF32 products
// for fp32 models): K = RoPE(C_k U_k,g^T), V = C_v U_v,g^T for 64-token
// tiles of one problem, every group's basis rows staged once per CTA (the
// CTA walks `tpc` tiles).  Warps take (group, 16-token row block, K or V)
// tasks: the product in accumulator fragments (a lane holds columns 2t, 2t+1
// of each 8-column block, so the rotate-half partners d, d + D/2 are its
// own), RoPE on the key fragments, paired stores.
constexpr int kMhmThreads = 256;

struct MhmSmem { int ldc, cp, uk, uv, ck, cv, cosb, sinb, posb, total; };
__host__ __device__ inline MhmSmem mhm_smem(int n, int D, int ld) {
  MhmSmem m;
  m.ldc = ld + 4;  // fragment reads (4g + t) conflict-free
  m.cp = D / 2 + 4;
  m.uk = 0;
  m.uv = m.uk + n * m.ldc;
  m.ck = m.uv + n * m.ldc;
  m.cv = m.ck + kMhTok * m.ldc;
  m.cosb = m.cv + kMhTok * m.ldc;
  m.sinb = m.cosb + kMhTok * m.cp;
  m.posb = m.sinb + kMhTok * m.cp;
  m.total = m.posb + kMhTok;
  return m;
}

template <typename T, int D, bool SPLIT>
__global__ void __launch_bounds__(kMhmThreads) mid_hat_mma_kernel(
    const float* uk, const float* uv, long u_sp, int ld, const int* rk, const int* rv,
    const float* ck, const float* cv, long c_sp, const int* mid_pos, long mid_sp, int pos_base,
    int W, int H, const float* inv_freq, float scale, T* ok, T* ov, long ob, long oh, long ot,
    int l0, int tpc) {
  constexpr int half = D / 2, NT = D / 8, HT = D / 16;
  extern __shared__ __align__(16) float hsm[];
  const int p = blockIdx.y;
  const int n = H * D;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int r_k = rk[p], r_v = rv[p];
  const MhmSmem L = mhm_smem(n, D, ld);
  const int ldc = L.ldc, cp = L.cp;
  float* usk = hsm + L.uk;
  float* usv = hsm + L.uv;
  float* ckb = hsm + L.ck;
  float* cvb = hsm + L.cv;
  float* cosb = hsm + L.cosb;
  float* sinb = hsm + L.sinb;
  int* posb = reinterpret_cast<int*>(hsm + L.posb);
  const float* Uk = uk + p * u_sp;
  const float* Uv = uv + p * u_sp;
  for (int e = tid; e < n * ld; e += kMhmThreads) {  // basis rows, columns past the rank zero
    const int row = e / ld, c = e % ld;
    const float xk = Uk[(long)row * ld + c], xv = Uv[(long)row * ld + c];
    usk[row * ldc + c] = c < r_k ? (SPLIT ? xk : __uint_as_float(tf32_bits(xk))) : 0.f;
    usv[row * ldc + c] = c < r_v ? (SPLIT ? xv : __uint_as_float(tf32_bits(xv))) : 0.f;
  }
  const int nm = (W + kMhTok - 1) / kMhTok;
  const int t_begin = blockIdx.x * tpc, t_end = min(nm, t_begin + tpc);
  for (int tile = t_begin; tile < t_end; ++tile) {
    const int j0 = tile * kMhTok, ntok = min(kMhTok, W - j0);
    __syncthreads();  // the previous tile is written out
    for (int e = tid; e < kMhTok * ld; e += kMhmThreads) {
      const int tt = e / ld, c = e % ld;
      float xk = 0.f, xv = 0.f;
      if (tt < ntok) {
        const long gidx = p * c_sp + (long)(j0 + tt) * ld + c;
        if (c < r_k) xk = ck[gidx];
        if (c < r_v) xv = cv[gidx];
      }
      ckb[tt * ldc + c] = SPLIT ? xk : __uint_as_float(tf32_bits(xk));
      cvb[tt * ldc + c] = SPLIT ? xv : __uint_as_float(tf32_bits(xv));
    }
    for (int tt = tid; tt < kMhTok; tt += kMhmThreads)
      posb[tt] = tt < ntok ? (mid_pos ? mid_pos[p * mid_sp + j0 + tt] : pos_base + j0 + tt) : 0;
    __syncthreads();
    for (int e = tid; e < kMhTok * half; e += kMhmThreads) {
      const int tt = e / half, f = e % half;
      float c = 1.f, sn = 0.f;
      rope_cs(posb[tt], inv_freq[f], scale, &c, &sn);
      cosb[tt * cp + f] = c;
      sinb[tt * cp + f] = sn;
    }
    __syncthreads();
    // tasks: (group, row block, keys / values)
    for (int task = warp; task < H * 4 * 2; task += kMhmThreads / 32) {
      const int kv = task & 1, rb = (task >> 1) & 3, g = task >> 3;
      const float* cb = kv ? cvb : ckb;
      const float* ub = kv ? usv : usk;
      const int rr = kv ? r_v : r_k;
      const int tt0 = rb * 16 + gq, tt1 = tt0 + 8;
      float acc[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[j][q] = 0.f;
      const int nkk = (rr + 7) / 8;
      for (int kk = 0; kk < nkk; ++kk) {
        const int c0 = kk * 8 + tq;
        const float af[4] = {cb[tt0 * ldc + c0], cb[tt1 * ldc + c0], cb[tt0 * ldc + c0 + 4],
                             cb[tt1 * ldc + c0 + 4]};
        if constexpr (SPLIT) {
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const float* ur = ub + (g * D + j * 8 + gq) * ldc + c0;
            mma_f32<true>(acc[j], af, ur[0], ur[4]);
          }
        } else {
          const uint32_t ah[4] = {__float_as_uint(af[0]), __float_as_uint(af[1]),
                                  __float_as_uint(af[2]), __float_as_uint(af[3])};
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const float* ur = ub + (g * D + j * 8 + gq) * ldc + c0;
            mma_tf32(acc[j], ah, __float_as_uint(ur[0]), __float_as_uint(ur[4]));
          }
        }
      }
      if (!kv) {  // RoPE at each row's true position on the pairs (8j + 2t + e, + D/2)
#pragma unroll
        for (int j = 0; j < HT; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int f = 8 * j + 2 * tq + e;
            float y1, y2;
            rope_apply_pair(acc[j][e], acc[j + HT][e], cosb[tt0 * cp + f], sinb[tt0 * cp + f], &y1, &y2);
            acc[j][e] = y1; acc[j + HT][e] = y2;
            rope_apply_pair(acc[j][2 + e], acc[j + HT][2 + e], cosb[tt1 * cp + f], sinb[tt1 * cp + f], &y1, &y2);
            acc[j][2 + e] = y1; acc[j + HT][2 + e] = y2;
          }
        }
      }
      T* o = (kv ? ov : ok) + p * ob + g * oh;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int d = 8 * j + 2 * tq;
        if (tt0 < ntok) store_pair<T>(o + (long)(l0 + j0 + tt0) * ot + d, acc[j][0], acc[j][1]);
        if (tt1 < ntok) store_pair<T>(o + (long)(l0 + j0 + tt1) * ot + d, acc[j][2], acc[j][3]);
      }
    }
  }
}

}  // namespace kvd

namespace kvd_host {
using namespace kvd;

static inline int grid_for(long tot) {
  const long b = (tot + 255) / 256;
  return (int)(b < 2048 ? b : 2048);
}

template <typename T>
int launch_hf_to_rows(const kvd_hf_view& kv, const kvd_hf_view& vv, int P, int H, int D, T* dst_k,
                      T* dst_v, long dst_sp, int slot0, cudaStream_t s) {
  if (kv.tokens <= 0 || P <= 0) return KVD_OK;
  if (vv.tokens != kv.tokens) {
    set_error("keys and values carry %d and %d tokens", kv.tokens, vv.tokens);
    return KVD_ERR_ARG;
  }
  HfRowsPair<T> pr;
  pr.s[0] = {(const T*)kv.ptr, kv.stride_b, kv.stride_h, kv.stride_t, dst_k};
  pr.s[1] = {(const T*)vv.ptr, vv.stride_b, vv.stride_h, vv.stride_t, dst_v};
  constexpr int kPer = 16 / sizeof(T);
  auto whole = [&](const void* ptr, long a, long b, long c) {
    return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && a % kPer == 0 && b % kPer == 0 && c % kPer == 0;
  };
  const bool vec = D % kPer == 0 && dst_sp % kPer == 0 && whole(dst_k, 0, 0, 0) && whole(dst_v, 0, 0, 0) &&
                   whole(kv.ptr, kv.stride_b, kv.stride_h, kv.stride_t) &&
                   whole(vv.ptr, vv.stride_b, vv.stride_h, vv.stride_t);
  {
    KTimerScope kts_("hf_to_rows_kernel", s);
    if (vec) {
      dim3 grid(grid_for((long)kv.tokens * H * (D / kPer)), P, 2);  // keys and values in one launch
      hf_to_rows_vec_kernel<T><<<grid, 256, 0, s>>>(pr, H, D, kv.tokens, dst_sp, slot0);
    } else {
      dim3 grid(grid_for((long)kv.tokens * H * D), P, 2);
      hf_to_rows_kernel<T><<<grid, 256, 0, s>>>(pr, H, D, kv.tokens, dst_sp, slot0);
    }
  }
  return check_launch("hf_to_rows_kernel");
}

template <typename T>
int launch_rows_copy(const T* src, long src_sp, T* dst, long dst_sp, int count, int n, int P,
                     cudaStream_t s) {
  if (count <= 0 || P <= 0) return KVD_OK;
  dim3 grid(grid_for((long)count * n), P);
  {
    KTimerScope kts_("rows_copy_kernel", s);
    rows_copy_kernel<T><<<grid, 256, 0, s>>>(src, src_sp, dst, dst_sp, count, n);
  }
  return check_launch("rows_copy_kernel");
}

template <typename T>
int launch_ring_compact(T* ring, long sp, int head, int len, int n, int P, cudaStream_t s) {
  if (head == 0 || len <= 0 || P <= 0) return KVD_OK;
  if ((len + head - 1) / head <= 8) {
    // rows [head + d, head + d + head) -> [d, d + head): each round's source
    // starts where its destination ends, so a round is a plain parallel copy
    for (int d = 0; d < len; d += head) {
      const int cnt = len - d < head ? len - d : head;
      if (int rc = launch_rows_copy<T>(ring + (long)(head + d) * n, sp, ring + (long)d * n, sp, cnt, n, P, s))
        return rc;
    }
    return KVD_OK;
  }
  {  // a short offset under a long ring: one CTA per problem, staged through shared memory
    KTimerScope kts_("ring_compact_kernel", s);
    ring_compact_kernel<T><<<P, 1024, 8192 * sizeof(T), s>>>(ring, sp, head, len, n);
  }
  return check_launch("ring_compact_kernel");
}

template <typename T>
int launch_peek(const kvd_config& c, const kvd_buffers& b, const kvd_counters& k, int p0, int count,
                const kvd_hf_view& ok_, const kvd_hf_view& ov_, const kvd_hf_view& tk,
                const kvd_hf_view& tv, cudaStream_t s) {
  const int H = c.num_heads, D = c.head_dim, n = H * D;
  const long ob = ok_.stride_b, oh = ok_.stride_h, ot = ok_.stride_t;
  if (ov_.stride_b != ob || ov_.stride_h != oh || ov_.stride_t != ot) {
    set_error("kvd_peek: K and V outputs must share strides");
    return KVD_ERR_ARG;
  }
  T* okp = (T*)ok_.ptr;
  T* ovp = (T*)ov_.ptr;
  int l0 = 0;
  constexpr int kPer = 16 / sizeof(T);
  const bool out_vec = D % kPer == 0 && ob % kPer == 0 && oh % kPer == 0 && ot % kPer == 0 &&
                       ((reinterpret_cast<uintptr_t>(okp) | reinterpret_cast<uintptr_t>(ovp)) & 15) == 0;
  auto seg = [&](const void* kk, const void* vv, long sp, int len) -> int {
    if (len <= 0) return KVD_OK;
    const T* ks = (const T*)kk + p0 * sp;
    const T* vs = (const T*)vv + p0 * sp;
    const bool vec = out_vec && sp % kPer == 0 &&
                     ((reinterpret_cast<uintptr_t>(ks) | reinterpret_cast<uintptr_t>(vs)) & 15) == 0;
    {
      KTimerScope kts_("rows_to_hf_kernel", s);
      if (vec) {
        dim3 grid(grid_for((long)len * H * (D / kPer)), count);
        rows_to_hf_vec_kernel<T><<<grid, 256, 0, s>>>(ks, vs, sp, len, H, D, okp, ovp, ob, oh, ot, l0);
      } else {
        dim3 grid(grid_for((long)len * n), count);
        rows_to_hf_kernel<T><<<grid, 256, 0, s>>>(ks, vs, sp, len, H, D, okp, ovp, ob, oh, ot, l0);
      }
    }
    l0 += len;
    return check_launch("rows_to_hf_kernel");
  };
  int rc;
  if ((rc = seg(b.sink_k, b.sink_v, (long)c.n_sink * n, k.sink_len))) return rc;
  if (k.hh_len > 0) {
    if ((rc = seg(b.hh_k[k.hh_sel], b.hh_v[k.hh_sel], (long)c.hh_budget * n, k.hh_len))) return rc;
  }
  if (k.w_len > 0) {
    const int ld = c.rank;
    const long u_sp = (long)n * ld, c_sp = (long)c.w_cap * ld;
    const int track_pos = c.retention != KVD_RETENTION_FIFO;
    const int mid_len = k.hh_len + k.w_len;
    const int pos_base = (int)(k.cumulative_length - k.ring_len - mid_len);
    const int half = D / 2;
    const int fp = half / 16;
    const bool tiled = (D == 64 || D == 128) && ob % fp == 0 && oh % fp == 0 && ot % fp == 0 &&
                       reinterpret_cast<uintptr_t>(okp) % (fp * sizeof(T)) == 0 &&
                       reinterpret_cast<uintptr_t>(ovp) % (fp * sizeof(T)) == 0;
    int umma_rc = -1;  // bf16: the middle on the 5th-generation tensor cores when the shape allows
    if (sizeof(T) == 2) {
      umma_rc = launch_mid_hat_umma(c, b, k, p0, count, okp, ovp, ob, oh, ot, l0, s);
      if (umma_rc > 0) return umma_rc;
    }
    const MhmSmem hm = mhm_smem(n, D, ld);
    const bool mma = umma_rc < 0 && tiled && ld % 8 == 0 && 4L * hm.total <= 200 * 1024 &&
                     reinterpret_cast<uintptr_t>(okp) % (2 * sizeof(T)) == 0 &&
                     reinterpret_cast<uintptr_t>(ovp) % (2 * sizeof(T)) == 0 && ob % 2 == 0 &&
                     oh % 2 == 0 && ot % 2 == 0;
    if (mma) {
      constexpr bool kSplit = sizeof(T) == 4;
      auto fn = D == 64 ? mid_hat_mma_kernel<T, 64, kSplit> : mid_hat_mma_kernel<T, 128, kSplit>;
      if (int rc2 = ensure_smem((const void*)fn, 4 * hm.total, "mid_hat_kernel")) return rc2;
      const int nm = (k.w_len + kMhTok - 1) / kMhTok;
      int tpc = (int)(((long)nm * count + 2 * 148 - 1) / (2 * 148));  // about two waves of CTAs
      tpc = tpc < 1 ? 1 : (tpc > 8 ? 8 : tpc);
      dim3 grid((nm + tpc - 1) / tpc, count);
      {
        KTimerScope kts_("mid_hat_kernel", s);
        fn<<<grid, kMhmThreads, 4 * hm.total, s>>>(
          b.u_k[k.u_sel] + p0 * u_sp, b.u_v[k.u_sel] + p0 * u_sp, u_sp, ld, b.r_k + p0,
          b.r_v + p0, b.c_k + p0 * c_sp, b.c_v + p0 * c_sp, c_sp,
          track_pos ? b.mid_pos + (long)p0 * c.w_cap : nullptr, c.w_cap, pos_base, k.w_len, H,
          c.inv_freq, c.rope_scaling, okp, ovp, ob, oh, ot, l0, tpc);
      }
    } else if (umma_rc == 0) {
      // done on the tensor cores
    } else if (tiled) {
      // the coordinate tile stays whole; the basis is staged in rank chunks
      // sized to the device's shared-memory limit
      auto smem_for = [&](int rcc) { return 4 * (2 * ld * kMhCtPitch + 2 * rcc * D + kMhTok * half * 2); };
      const int limit = device_smem_optin();
      int rcc = ld;
      while (rcc > 4 && smem_for(rcc) > limit) rcc = ((rcc + 1) / 2 + 3) & ~3;
      const int smem = smem_for(rcc);
      auto fn = D == 64 ? mid_hat_tiled_kernel<T, 64> : mid_hat_tiled_kernel<T, 128>;
      if (int rc2 = ensure_smem((const void*)fn, smem, "mid_hat_kernel")) return rc2;
      dim3 grid((k.w_len + kMhTok - 1) / kMhTok, count);
      {
        KTimerScope kts_("mid_hat_kernel", s);
        fn<<<grid, 256, smem, s>>>(
          b.u_k[k.u_sel] + p0 * u_sp, b.u_v[k.u_sel] + p0 * u_sp, u_sp, ld, b.r_k + p0,
          b.r_v + p0, b.c_k + p0 * c_sp, b.c_v + p0 * c_sp, c_sp,
          track_pos ? b.mid_pos + (long)p0 * c.w_cap : nullptr, c.w_cap, pos_base, k.w_len, H,
          c.inv_freq, c.rope_scaling, okp, ovp, ob, oh, ot, l0, rcc);
      }
    } else {
      const int smem = 4 * (2 * kMidTile * ld + 2 * D * ld + kMidTile * half * 2);
      if (int rc2 = ensure_smem((const void*)mid_hat_kernel<T>, smem, "mid_hat_kernel")) return rc2;
      dim3 grid((k.w_len + kMidTile - 1) / kMidTile, count);
      {
        KTimerScope kts_("mid_hat_kernel", s);
        mid_hat_kernel<T><<<grid, 256, smem, s>>>(
          b.u_k[k.u_sel] + p0 * u_sp, b.u_v[k.u_sel] + p0 * u_sp, u_sp, ld, b.r_k + p0, b.r_v + p0,
          b.c_k + p0 * c_sp, b.c_v + p0 * c_sp, c_sp,
          track_pos ? b.mid_pos + (long)p0 * c.w_cap : nullptr, c.w_cap, pos_base, k.w_len, H, D,
          c.inv_freq, c.rope_scaling, okp, ovp, ob, oh, ot, l0);
      }
    }
    if ((rc = check_launch("mid_hat_kernel"))) return rc;
    l0 += k.w_len;
  }
  const long ring_sp = (long)c.ring_cap * n;
  if (k.ring_len > 0) {
    const T* rk = (const T*)b.ring_k + (long)k.ring_head * n;
    const T* rv = (const T*)b.ring_v + (long)k.ring_head * n;
    if ((rc = seg(rk, rv, ring_sp, k.ring_len))) return rc;
  }
  if (tk.tokens > 0) {
    dim3 grid(grid_for((long)tk.tokens * n), count);
    {
      KTimerScope kts_("hf_to_hf_kernel", s);
      hf_to_hf_kernel<T><<<grid, 256, 0, s>>>((const T*)tk.ptr, (const T*)tv.ptr, tk.stride_b,
                                            tk.stride_h, tk.stride_t, tk.tokens, H, D, okp, ovp,
                                            ob, oh, ot, l0);
    }
    if ((rc = check_launch("hf_to_hf_kernel"))) return rc;
  }
  return KVD_OK;
}

#define KVD_INST(T)                                                                             \
  template int launch_hf_to_rows<T>(const kvd_hf_view&, const kvd_hf_view&, int, int, int, T*,  \
                                    T*, long, int, cudaStream_t);                               \
  template int launch_rows_copy<T>(const T*, long, T*, long, int, int, int, cudaStream_t);      \
  template int launch_ring_compact<T>(T*, long, int, int, int, int, cudaStream_t);              \
  template int launch_peek<T>(const kvd_config&, const kvd_buffers&, const kvd_counters&, int,  \
                              int, const kvd_hf_view&, const kvd_hf_view&, const kvd_hf_view&, \
                              const kvd_hf_view&, cudaStream_t);
KVD_INST(float)
KVD_INST(__nv_bfloat16)
#undef KVD_INST

}  // namespace kvd_host

namespace kvd {
__global__ void rope_table_kernel(int n, const int* pos, int nf, const float* inv_freq, float scale,
                                  int fast, float* co, float* so) {
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < (long)n * nf;
       e += (long)gridDim.x * blockDim.x) {
    const int i = (int)(e / nf), f = (int)(e % nf);
    float c, s;
    if (fast) rope_cs_fast(pos[i], inv_freq[f], scale, &c, &s);
    else rope_cs(pos[i], inv_freq[f], scale, &c, &s);
    co[e] = c;
    so[e] = s;
  }
}
}  // namespace kvd

extern "C" int kvd_rope_table(int32_t n, const int32_t* pos, int32_t nf, const float* inv_freq,
                              float scale, int32_t fast, float* cos_out, float* sin_out,
                              kvd_stream_t stream) {
  using namespace kvd_host;
  if (n < 0 || nf < 0) { set_error("kvd_rope_table: negative size"); return KVD_ERR_ARG; }
  if ((long)n * nf == 0) return KVD_OK;
  if (!pos || !inv_freq || !cos_out || !sin_out) {
    set_error("kvd_rope_table: null pointer");
    return KVD_ERR_ARG;
  }
  const long tot = (long)n * nf;
  const int grid = (int)((tot + 255) / 256 < 4096 ? (tot + 255) / 256 : 4096);
  kvd::rope_table_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(n, pos, nf, inv_freq, scale, fast,
                                                                 cos_out, sin_out);
  return check_launch("rope_table_kernel");
}
