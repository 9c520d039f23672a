// Factored chunk attention (sm_100a, tcgen05): every query of an ingest chunk
// (or of a frozen-scoring window) against the retained cache
// [sinks | exact tier | RoPE(U_k C_k) | ring (| tail)], causal over the chunk,
// without materialising the middle tier in HBM.  It answers the transformers
// attention over the dense value bug_cache.py:1404-1423 (ingest) and
// 1390-1402 (scoring) return, whose middle is _ensure_mid_cache's
// reconstruction (1540-1575).
//
// One CTA of four warps per (128 query rows, KV group, sequence).  A query row
// is (token, head of the group), row = token * G + head; thread t owns row t,
// which is also TMEM lane t of every accumulator.  Key tiles of 128 run in
// order through the segments; per tile:
//   keys    verbatim tiers: the group's bf16 rows copied into the B operand of
//           the score MMA; middle: C_k U_k,g^T on the tensor core (kind::tf32,
//           TMEM), each row read back by its thread, rotated (RoPE at the
//           token's true position) and rounded to bf16 into the same operand;
//   scores  S = Q K^T with kind::f16 (bf16 operands, fp32 in TMEM), M = N = 128,
//           read back a row per thread, scaled, masked past the segment and
//           by causality, online softmax (running max and sum per row);
//   values  P (bf16) times the tile's values, the tile transposed in shared
//           memory as the B operand: verbatim rows add to acc_d (D columns),
//           the middle to acc_c (coordinate space, rank columns; U_v,g is
//           applied once at the end).  The product lands in TMEM and is added
//           to the row's register accumulators after the softmax correction.
// Operands sit in shared memory in the no-swizzle K-major core-matrix layout
// (8 rows x 16 bytes per core matrix).  Every MMA is issued by one thread and
// completes on an mbarrier whose wait is bounded: on time-out the status word
// is set, the outstanding MMA is waited for (bounded), TMEM is freed and the
// rows are written as zeros.
#include <stdio.h>

#include "kernels.cuh"
#include "umma.cuh"

namespace kvd {

constexpr int kCaRows = 128;     // query rows per CTA
constexpr int kCaKeys = 128;     // keys per tile
constexpr int kCaThreads = 128;  // one thread per row
constexpr int kCaR = 32;         // staged rank columns (rank <= 32)
constexpr int kCaD = 64;         // head dim
constexpr long kCaWaitPolls = 1L << 22;
constexpr int kCaSegs = 5;       // sinks, exact tier, middle, ring, tail

struct CaArgs {
  int H, G, ld, Hq, q_len, rows;
  long total;                          // keys in the concatenation of all segments
  int seg_len[kCaSegs];
  const __nv_bfloat16* seg_k[kCaSegs];
  const __nv_bfloat16* seg_v[kCaSegs];
  long seg_sp[kCaSegs], seg_tok[kCaSegs], seg_head[kCaSegs];  // element strides: problem, token, head
  const float* uk; const float* uv; long u_sp;
  const int* rk; const int* rv;
  const float* ck; const float* cv; long c_sp;
  const int* mid_pos; long mid_sp; long pos_base;
  const float* inv_freq; float rope_scale;
  const __nv_bfloat16* q; long q_sb, q_sh, q_st;
  __nv_bfloat16* out;                  // (count, q_len, Hq, D)
  float scaling;
  int* status;
  // split of the key tiles over CTAs: split z of nsplit takes tiles
  // [z * ntiles / nsplit, (z + 1) * ntiles / nsplit) of the concatenation and,
  // when nsplit > 1, writes a record per row instead of the output:
  // m, l, O[D] (O unnormalised, U_v,g already applied)
  int nsplit, ntiles;
  float* part;
};
constexpr int kCaRec = kCaD + 2;  // floats per partial record

struct CaSmem { int qs, ks, ps, vs, ck, uk, uv, pos, bar, total; };  // bytes
__host__ __device__ inline CaSmem ca_smem() {
  CaSmem m;
  m.qs = 0;                                 // [128 rows][64] bf16, A of S
  m.ks = m.qs + kCaRows * kCaD * 2;         // [128 keys][64] bf16, B of S
  m.ps = m.ks + kCaKeys * kCaD * 2;         // [128 rows][128 keys] bf16, A of P V
  m.vs = m.ps + kCaRows * kCaKeys * 2;      // [64 columns][128 keys] bf16, B of P V
  m.ck = m.vs + kCaD * kCaKeys * 2;         // [128 keys][32] tf32, A of the key rebuild
  m.uk = m.ck + kCaKeys * kCaR * 4;         // [64][32] tf32, B of the key rebuild
  m.uv = m.uk + kCaD * kCaR * 4;            // [64][32] fp32, U_v,g for the final expansion
  m.pos = m.uv + kCaD * kCaR * 4;           // [128] positions of the middle tile
  m.bar = m.pos + kCaKeys * 4;              // mbarrier, TMEM base
  m.total = m.bar + 16;
  return m;
}

// byte offset of element (row, k) in a K-major core-matrix tile of K extent kx
__device__ __forceinline__ int bf_off(int row, int k, int kx) {  // bf16
  return (row >> 3) * (kx * 16) + (k >> 3) * 128 + (row & 7) * 16 + (k & 7) * 2;
}
__device__ __forceinline__ int tf_off(int row, int k, int kx) {  // tf32
  return (row >> 3) * (kx * 32) + (k >> 2) * 128 + (row & 7) * 16 + (k & 3) * 4;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 8 rows of 8 bf16 (one 16-byte load each) transposed into 8 columns of 8
__device__ __forceinline__ void transpose8(const uint4 (&in)[8], uint4 (&out)[8]) {
  unsigned short e[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t w[4] = {in[i].x, in[i].y, in[i].z, in[i].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      e[i][2 * j] = (unsigned short)(w[j] & 0xffffu);
      e[i][2 * j + 1] = (unsigned short)(w[j] >> 16);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    out[j].x = (uint32_t)e[0][j] | ((uint32_t)e[1][j] << 16);
    out[j].y = (uint32_t)e[2][j] | ((uint32_t)e[3][j] << 16);
    out[j].z = (uint32_t)e[4][j] | ((uint32_t)e[5][j] << 16);
    out[j].w = (uint32_t)e[6][j] | ((uint32_t)e[7][j] << 16);
  }
}

__global__ void __launch_bounds__(kCaThreads) chunk_attn_kernel(CaArgs a) {
  constexpr int D = kCaD, HALF = kCaD / 2;
  extern __shared__ __align__(1024) unsigned char csm[];
  const CaSmem L = ca_smem();
  const int qt = blockIdx.x, g = blockIdx.y, b = blockIdx.z / a.nsplit, split = blockIdx.z % a.nsplit;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int tile_lo = (int)((long)split * a.ntiles / a.nsplit);
  const int tile_hi = (int)((long)(split + 1) * a.ntiles / a.nsplit);
  const int G = a.G, ld = a.ld;
  const int r_k = a.rk[b], r_v = a.rv[b];
  unsigned char* qs = csm + L.qs;
  unsigned char* ks = csm + L.ks;
  unsigned char* ps = csm + L.ps;
  unsigned char* vs = csm + L.vs;
  unsigned char* cks = csm + L.ck;
  unsigned char* uks = csm + L.uk;
  float* uvs = reinterpret_cast<float*>(csm + L.uv);
  int* posb = reinterpret_cast<int*>(csm + L.pos);
  uint64_t* bar = reinterpret_cast<uint64_t*>(csm + L.bar);
  uint32_t* tbase = reinterpret_cast<uint32_t*>(csm + L.bar + 8);
  if (warp == 0) {
    umma::tmem_alloc(tbase, 256);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    umma::mbar_init(bar, 1);
    umma::mbar_fence_init();
  }
  // this thread's query row
  const int R = qt * kCaRows + tid;
  const bool row_ok = R < a.rows;
  const int qi = row_ok ? R / G : 0, qh = g * G + (row_ok ? R % G : 0);
  {
    const __nv_bfloat16* src = a.q + (long)b * a.q_sb + (long)qh * a.q_sh + (long)qi * a.q_st;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      const uint4 v = row_ok ? *reinterpret_cast<const uint4*>(src + 8 * c) : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(qs + bf_off(tid, 8 * c, D)) = v;
    }
  }
  {  // U_k,g (tf32, columns past the rank zero) and U_v,g (fp32, plain [d][j])
    const float* Uk = a.uk + (long)b * a.u_sp + (long)g * D * ld;
    const float* Uv = a.uv + (long)b * a.u_sp + (long)g * D * ld;
    for (int e = tid; e < D * (kCaR / 4); e += kCaThreads) {
      const int d = e / (kCaR / 4), k = 4 * (e % (kCaR / 4));
      float4 u = make_float4(0.f, 0.f, 0.f, 0.f), w = u;
      if (k < ld) {
        u = *reinterpret_cast<const float4*>(Uk + (long)d * ld + k);
        w = *reinterpret_cast<const float4*>(Uv + (long)d * ld + k);
      }
      u.x = k < r_k ? u.x : 0.f; u.y = k + 1 < r_k ? u.y : 0.f;
      u.z = k + 2 < r_k ? u.z : 0.f; u.w = k + 3 < r_k ? u.w : 0.f;
      w.x = k < r_v ? w.x : 0.f; w.y = k + 1 < r_v ? w.y : 0.f;
      w.z = k + 2 < r_v ? w.z : 0.f; w.w = k + 3 < r_v ? w.w : 0.f;
      *reinterpret_cast<float4*>(uks + tf_off(d, k, kCaR)) =
          make_float4(umma::to_tf32(u.x), umma::to_tf32(u.y), umma::to_tf32(u.z), umma::to_tf32(u.w));
      *reinterpret_cast<float4*>(uvs + d * kCaR + k) = w;
    }
  }
  umma::fence_proxy_async_smem();
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tbase;
  const uint32_t t_s = tmem, t_pv = tmem + 128, t_k = tmem + 192;
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
  const uint32_t qs_a = (uint32_t)__cvta_generic_to_shared(qs);
  const uint32_t ks_a = (uint32_t)__cvta_generic_to_shared(ks);
  const uint32_t ps_a = (uint32_t)__cvta_generic_to_shared(ps);
  const uint32_t vs_a = (uint32_t)__cvta_generic_to_shared(vs);
  const uint32_t ck_a = (uint32_t)__cvta_generic_to_shared(cks);
  const uint32_t uk_a = (uint32_t)__cvta_generic_to_shared(uks);
  float acc_d[D], acc_c[kCaR];
#pragma unroll
  for (int d = 0; d < D; ++d) acc_d[d] = 0.f;
#pragma unroll
  for (int j = 0; j < kCaR; ++j) acc_c[j] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  uint32_t phase = 0;
  bool ok = true;
  // the MMAs issued so far complete; a time-out anywhere makes every thread stop
  auto wait_mma = [&]() {
    const bool mine = umma::mbar_wait_bounded(bar, phase, kCaWaitPolls);
    phase ^= 1;
    ok = __syncthreads_and(mine) != 0;
    umma::fence_after_sync();
  };
  // causal: row token i sees keys x <= total - q_len + i of the concatenation;
  // the CTA's last token bounds the keys any of its rows sees
  const int i_last = min(a.q_len - 1, (qt * kCaRows + kCaRows - 1) / G);
  const long vis_cta = a.total - a.q_len + i_last;
  const long vis_row = a.total - a.q_len + qi;
  long x0 = 0;
  int tile = 0;  // index of the tile in the concatenation
  for (int s = 0; s < kCaSegs && ok; ++s) {
    const int len = a.seg_len[s];
    for (int t0 = 0; t0 < len && ok; t0 += kCaKeys, ++tile) {
      if (tile < tile_lo || tile >= tile_hi || x0 + t0 > vis_cta) continue;
      const int nk = min(kCaKeys, len - t0);
      if (s == 2) {
        // ----- middle tile: stage C_k (tf32) and C_v^T (bf16), rebuild keys on the tensor core
        {
          const int kk = tid;
          const float* crow = a.ck + (long)b * a.c_sp + (long)(t0 + kk) * ld;
#pragma unroll
          for (int c = 0; c < kCaR / 4; ++c) {
            const int k = 4 * c;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (kk < nk && k < ld) v = *reinterpret_cast<const float4*>(crow + k);
            v.x = k < r_k ? v.x : 0.f; v.y = k + 1 < r_k ? v.y : 0.f;
            v.z = k + 2 < r_k ? v.z : 0.f; v.w = k + 3 < r_k ? v.w : 0.f;
            *reinterpret_cast<float4*>(cks + tf_off(kk, k, kCaR)) =
                make_float4(umma::to_tf32(v.x), umma::to_tf32(v.y), umma::to_tf32(v.z), umma::to_tf32(v.w));
          }
          posb[kk] = kk < nk ? (a.mid_pos ? a.mid_pos[(long)b * a.mid_sp + t0 + kk] : (int)(a.pos_base + t0 + kk)) : 0;
        }
        if (tid < (kCaKeys / 8) * (kCaR / 8)) {  // C_v^T: unit (key block, coordinate block)
          const int kb = tid / (kCaR / 8), jb = tid % (kCaR / 8);
          uint4 rows[8], cols[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int key = kb * 8 + i, j = jb * 8;
            float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
            if (key < nk && j < ld) {
              const float* cr = a.cv + (long)b * a.c_sp + (long)(t0 + key) * ld + j;
              lo = *reinterpret_cast<const float4*>(cr);
              if (j + 4 < ld) hi = *reinterpret_cast<const float4*>(cr + 4);
            }
            const float f[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            float z[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) z[e] = j + e < r_v ? f[e] : 0.f;
            rows[i] = make_uint4(pack_bf16(z[0], z[1]), pack_bf16(z[2], z[3]), pack_bf16(z[4], z[5]),
                                 pack_bf16(z[6], z[7]));
          }
          transpose8(rows, cols);
#pragma unroll
          for (int e = 0; e < 8; ++e) *reinterpret_cast<uint4*>(vs + bf_off(jb * 8 + e, kb * 8, kCaKeys)) = cols[e];
        }
        umma::fence_proxy_async_smem();
        umma::fence_before_sync();
        __syncthreads();
        if (tid == 0) {
          umma::fence_after_sync();
          const uint32_t idk = umma::idesc_tf32(kCaKeys, D);
#pragma unroll
          for (int j = 0; j < kCaR / 8; ++j)
            umma::mma_tf32(t_k, umma::smem_desc(ck_a + 256 * j, 128, 32 * kCaR),
                           umma::smem_desc(uk_a + 256 * j, 128, 32 * kCaR), idk, j > 0);
          umma::commit(bar);
        }
        wait_mma();
        if (!ok) break;
        {  // this thread's key row: RoPE at its position, bf16 into the score operand
          const int kk = tid;
          const int pos = posb[kk];
#pragma unroll
          for (int f0 = 0; f0 < HALF; f0 += 16) {
            float x1[16], x2[16];
            umma::tmem_ld16(t_k + lane_base + f0, x1);
            umma::tmem_ld16(t_k + lane_base + HALF + f0, x2);
            umma::tmem_wait_ld();
            float y1[16], y2[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float c, sn;
              rope_cs_fast(pos, a.inv_freq[f0 + i], a.rope_scale, &c, &sn);
              rope_apply_pair(x1[i], x2[i], c, sn, &y1[i], &y2[i]);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              *reinterpret_cast<uint4*>(ks + bf_off(kk, f0 + 8 * h, D)) =
                  make_uint4(pack_bf16(y1[8 * h], y1[8 * h + 1]), pack_bf16(y1[8 * h + 2], y1[8 * h + 3]),
                             pack_bf16(y1[8 * h + 4], y1[8 * h + 5]), pack_bf16(y1[8 * h + 6], y1[8 * h + 7]));
              *reinterpret_cast<uint4*>(ks + bf_off(kk, HALF + f0 + 8 * h, D)) =
                  make_uint4(pack_bf16(y2[8 * h], y2[8 * h + 1]), pack_bf16(y2[8 * h + 2], y2[8 * h + 3]),
                             pack_bf16(y2[8 * h + 4], y2[8 * h + 5]), pack_bf16(y2[8 * h + 6], y2[8 * h + 7]));
            }
          }
        }
      } else {
        // ----- verbatim tile: the group's key rows and the value rows transposed
        const __nv_bfloat16* kb0 = a.seg_k[s] + (long)b * a.seg_sp[s] + (long)g * a.seg_head[s];
        const __nv_bfloat16* vb0 = a.seg_v[s] + (long)b * a.seg_sp[s] + (long)g * a.seg_head[s];
        {
          const int kk = tid;
          const __nv_bfloat16* kr = kb0 + (long)(t0 + kk) * a.seg_tok[s];
#pragma unroll
          for (int c = 0; c < D / 8; ++c) {
            const uint4 v = kk < nk ? *reinterpret_cast<const uint4*>(kr + 8 * c) : make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(ks + bf_off(kk, 8 * c, D)) = v;
          }
        }
        {  // unit (key block of 8, column block of 8): 16 x 8 units over 128 threads
          const int kb = tid / (D / 8), db = tid % (D / 8);
          uint4 rows[8], cols[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int key = kb * 8 + i;
            rows[i] = key < nk ? *reinterpret_cast<const uint4*>(vb0 + (long)(t0 + key) * a.seg_tok[s] + 8 * db)
                               : make_uint4(0, 0, 0, 0);
          }
          transpose8(rows, cols);
#pragma unroll
          for (int e = 0; e < 8; ++e) *reinterpret_cast<uint4*>(vs + bf_off(db * 8 + e, kb * 8, kCaKeys)) = cols[e];
        }
      }
      // ----- scores S = Q K^T
      umma::fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      if (tid == 0) {
        umma::fence_after_sync();
        const uint32_t ids = umma::idesc_bf16(kCaRows, kCaKeys);
#pragma unroll
        for (int j = 0; j < D / 16; ++j)
          umma::mma_bf16(t_s, umma::smem_desc(qs_a + 256 * j, 128, 16 * D),
                         umma::smem_desc(ks_a + 256 * j, 128, 16 * D), ids, j > 0);
        umma::commit(bar);
      }
      wait_mma();
      if (!ok) break;
      // ----- online softmax of this row over the tile (keys [0, kvis) visible)
      const long lim = vis_row - (x0 + t0);
      const int kvis = row_ok ? (int)max(0L, min((long)nk, lim + 1)) : nk;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < kCaKeys / 16; ++c) {
        float v[16];
        umma::tmem_ld16(t_s + lane_base + 16 * c, v);
        umma::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (16 * c + e < kvis) mt = fmaxf(mt, v[e] * a.scaling);
      }
      const float m_new = fmaxf(m_run, mt);
      const float alpha = m_run == -INFINITY ? 0.f : __expf(m_run - m_new);
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < kCaKeys / 16; ++c) {
        float v[16];
        umma::tmem_ld16(t_s + lane_base + 16 * c, v);
        umma::tmem_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          float p0 = 16 * c + e < kvis ? __expf(v[e] * a.scaling - m_new) : 0.f;
          float p1 = 16 * c + e + 1 < kvis ? __expf(v[e + 1] * a.scaling - m_new) : 0.f;
          pk[e / 2] = pack_bf16(p0, p1);
          const __nv_bfloat162 r = *reinterpret_cast<const __nv_bfloat162*>(&pk[e / 2]);
          lsum += __low2float(r) + __high2float(r);  // the rounded weights the MMA sees
        }
        *reinterpret_cast<uint4*>(ps + bf_off(tid, 16 * c, kCaKeys)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(ps + bf_off(tid, 16 * c + 8, kCaKeys)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
      l_run = l_run * alpha + lsum;
      m_run = m_new;
#pragma unroll
      for (int d = 0; d < D; ++d) acc_d[d] *= alpha;
#pragma unroll
      for (int j = 0; j < kCaR; ++j) acc_c[j] *= alpha;
      // ----- values: P V (verbatim) or P C_v (middle, coordinate space)
      const int nv = s == 2 ? kCaR : D;
      umma::fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      if (tid == 0) {
        umma::fence_after_sync();
        const uint32_t idv = umma::idesc_bf16(kCaRows, nv);
#pragma unroll
        for (int j = 0; j < kCaKeys / 16; ++j)
          umma::mma_bf16(t_pv, umma::smem_desc(ps_a + 256 * j, 128, 16 * kCaKeys),
                         umma::smem_desc(vs_a + 256 * j, 128, 16 * kCaKeys), idv, j > 0);
        umma::commit(bar);
      }
      wait_mma();
      if (!ok) break;
      if (s == 2) {
#pragma unroll
        for (int c = 0; c < kCaR / 16; ++c) {
          float v[16];
          umma::tmem_ld16(t_pv + lane_base + 16 * c, v);
          umma::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) acc_c[16 * c + e] += v[e];
        }
      } else {
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          float v[16];
          umma::tmem_ld16(t_pv + lane_base + 16 * c, v);
          umma::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) acc_d[16 * c + e] += v[e];
        }
      }
      umma::fence_before_sync();
      __syncthreads();  // every read of this tile's operands and accumulators is done
      umma::fence_after_sync();
    }
    x0 += len;
  }
  if (!ok) {  // the MMA whose wait gave up (phase already advanced past it)
    if (tid == 0) atomicOr(&a.status[kStatusTimeout], 32);
    umma::mbar_wait_bounded(bar, phase ^ 1, kCaWaitPolls);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, 256);
  if (!row_ok) return;
  // O = acc_d + U_v,g acc_c; the output row O / l, or this split's record
  const bool rec = a.nsplit > 1;
  const float inv_l = rec ? 1.f : ((ok && l_run > 0.f) ? 1.f / l_run : 0.f);
  __nv_bfloat16* dst = a.out + (((long)b * a.q_len + qi) * a.Hq + qh) * D;
  float* pr = a.part + ((((long)b * a.H + g) * a.rows + R) * a.nsplit + split) * kCaRec;
  if (rec) {
    pr[0] = ok ? m_run : -INFINITY;
    pr[1] = ok ? l_run : 0.f;
  }
#pragma unroll
  for (int d0 = 0; d0 < D; d0 += 8) {
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float* ur = uvs + (d0 + e) * kCaR;
      float v = acc_d[d0 + e];
#pragma unroll
      for (int j = 0; j < kCaR; ++j) v = fmaf(acc_c[j], ur[j], v);
      o[e] = ok ? v * inv_l : 0.f;
    }
    if (rec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) pr[2 + d0 + e] = o[e];
    } else {
      *reinterpret_cast<uint4*>(dst + d0) =
          make_uint4(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]), pack_bf16(o[4], o[5]), pack_bf16(o[6], o[7]));
    }
  }
}

// Combine the splits' records of a row: M = max m_s, out = sum e^(m_s - M) O_s /
// sum e^(m_s - M) l_s.  One thread per (row, column), rows of every group and
// sequence.
__global__ void __launch_bounds__(256) chunk_merge_kernel(CaArgs a) {
  constexpr int D = kCaD;
  const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long nrows = (long)gridDim.y * a.H * a.rows;  // gridDim.y = sequences
  (void)nrows;
  const int d = (int)(e % D);
  const long rr = e / D;  // row within (group, row)
  if (rr >= (long)a.H * a.rows) return;
  const int b = blockIdx.y;
  const int g = (int)(rr / a.rows), R = (int)(rr % a.rows);
  const float* pr = a.part + (((long)b * a.H + g) * a.rows + R) * a.nsplit * kCaRec;
  float M = -INFINITY;
  for (int z = 0; z < a.nsplit; ++z) M = fmaxf(M, pr[z * kCaRec]);
  float num = 0.f, den = 0.f;
  if (M != -INFINITY) {
    for (int z = 0; z < a.nsplit; ++z) {
      const float mz = pr[z * kCaRec];
      if (mz == -INFINITY) continue;
      const float w = __expf(mz - M);
      den = fmaf(w, pr[z * kCaRec + 1], den);
      num = fmaf(w, pr[z * kCaRec + 2 + d], num);
    }
  }
  const int qi = R / a.G, qh = g * a.G + R % a.G;
  a.out[(((long)b * a.q_len + qi) * a.Hq + qh) * D + d] = __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
}

}  // namespace kvd

namespace kvd_host {
using namespace kvd;

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

bool chunk_attention_applicable(const kvd_config& c, int num_q_heads, int n_heads) {
  return c.dtype == KVD_DTYPE_BF16 && c.head_dim == kCaD && c.rank <= kCaR && c.rank % 4 == 0 &&
         n_heads >= 1 && n_heads <= c.num_heads && num_q_heads % n_heads == 0 && num_q_heads >= n_heads &&
         (c.num_heads * c.head_dim) % 8 == 0;
}

constexpr int kCaMaxSplit = 8;

size_t chunk_attention_ws_bytes(const kvd_config& c, int count, int num_q_heads, int q_len, int n_heads) {
  const long rows = (long)q_len * (num_q_heads / (n_heads > 0 ? n_heads : 1));
  return (size_t)count * n_heads * rows * kCaMaxSplit * kCaRec * sizeof(float);
}

int launch_chunk_attention(const kvd_config& c, const kvd_buffers& bu, const kvd_counters& k, int p0,
                           int count, int h0, int hc, const void* q, int64_t q_sb, int64_t q_sh,
                           int64_t q_st, int Hq, int q_len, float scaling, const kvd_hf_view& tail_k,
                           const kvd_hf_view& tail_v, void* out, void* ws, size_t ws_bytes,
                           cudaStream_t s) {
  if (h0 < 0 || hc < 1 || h0 + hc > c.num_heads) {
    set_error("factored chunk attention: bad KV head range [%d, %d) of %d", h0, h0 + hc, c.num_heads);
    return KVD_ERR_ARG;
  }
  if (!chunk_attention_applicable(c, Hq, hc)) {
    set_error("factored chunk attention: unsupported shape (bf16, head_dim %d, rank <= %d, rank %% 4 == 0)",
              kCaD, kCaR);
    return KVD_ERR_ARG;
  }
  const int n = c.num_heads * c.head_dim;
  CaArgs a;
  // KV heads [h0, h0 + hc): hc groups whose tier rows start h0 * D features
  // into each token row and whose basis rows start at row h0 * D; the query
  // and output hold only their heads
  a.H = hc; a.G = Hq / hc; a.ld = c.rank; a.Hq = Hq; a.q_len = q_len;
  a.rows = q_len * a.G;
  const int tail_len = tail_k.ptr ? tail_k.tokens : 0;
  const int lens[kCaSegs] = {k.sink_len, k.hh_len, k.w_len, k.ring_len, tail_len};
  long total = 0;
  for (int i = 0; i < kCaSegs; ++i) { a.seg_len[i] = lens[i]; total += lens[i]; }
  a.total = total;
  if (q_len < 1 || q_len > total) { set_error("factored chunk attention: %d queries over %ld keys", q_len, total); return KVD_ERR_ARG; }
  const long sink_sp = (long)c.n_sink * n, hh_sp = (long)c.hh_budget * n, ring_sp = (long)c.ring_cap * n;
  using bf = __nv_bfloat16;
  const long hoff = (long)h0 * c.head_dim;
  a.seg_k[0] = (const bf*)bu.sink_k + p0 * sink_sp + hoff; a.seg_v[0] = (const bf*)bu.sink_v + p0 * sink_sp + hoff; a.seg_sp[0] = sink_sp;
  a.seg_k[1] = (const bf*)bu.hh_k[k.hh_sel] + p0 * hh_sp + hoff; a.seg_v[1] = (const bf*)bu.hh_v[k.hh_sel] + p0 * hh_sp + hoff; a.seg_sp[1] = hh_sp;
  a.seg_k[2] = nullptr; a.seg_v[2] = nullptr; a.seg_sp[2] = 0;
  a.seg_k[3] = (const bf*)bu.ring_k + p0 * ring_sp + (long)k.ring_head * n + hoff;
  a.seg_v[3] = (const bf*)bu.ring_v + p0 * ring_sp + (long)k.ring_head * n + hoff; a.seg_sp[3] = ring_sp;
  for (int i = 0; i < 4; ++i) { a.seg_tok[i] = n; a.seg_head[i] = c.head_dim; }
  a.seg_k[4] = tail_k.ptr ? (const bf*)tail_k.ptr + (long)h0 * tail_k.stride_h : nullptr;
  a.seg_v[4] = tail_v.ptr ? (const bf*)tail_v.ptr + (long)h0 * tail_v.stride_h : nullptr;
  a.seg_sp[4] = tail_k.stride_b; a.seg_tok[4] = tail_k.stride_t; a.seg_head[4] = tail_k.stride_h;
  if (tail_len > 0) {
    const bool same = tail_v.ptr && tail_v.stride_b == tail_k.stride_b && tail_v.stride_h == tail_k.stride_h &&
                      tail_v.stride_t == tail_k.stride_t && tail_v.tokens == tail_k.tokens;
    const bool aligned = al16(tail_k.ptr) && al16(tail_v.ptr) && tail_k.stride_b % 8 == 0 &&
                         tail_k.stride_h % 8 == 0 && tail_k.stride_t % 8 == 0;
    if (!same || !aligned) { set_error("factored chunk attention: tail views must match and be 16-byte aligned"); return KVD_ERR_ARG; }
  }
  a.u_sp = (long)n * c.rank;
  a.uk = bu.u_k[k.u_sel] + p0 * a.u_sp + hoff * c.rank; a.uv = bu.u_v[k.u_sel] + p0 * a.u_sp + hoff * c.rank;
  a.rk = bu.r_k + p0; a.rv = bu.r_v + p0;
  a.c_sp = (long)c.w_cap * c.rank;
  a.ck = bu.c_k + p0 * a.c_sp; a.cv = bu.c_v + p0 * a.c_sp;
  const bool track = c.retention != KVD_RETENTION_FIFO;
  a.mid_pos = track ? bu.mid_pos + (long)p0 * c.w_cap : nullptr; a.mid_sp = c.w_cap;
  // positions of a FIFO middle are consecutive after the sinks (the exact tier holds none)
  a.pos_base = (long)(k.cumulative_length - k.ring_len - (k.hh_len + k.w_len));
  a.inv_freq = c.inv_freq; a.rope_scale = c.rope_scaling;
  a.q = (const bf*)q; a.q_sb = q_sb; a.q_sh = q_sh; a.q_st = q_st;
  a.out = (bf*)out; a.scaling = scaling; a.status = bu.status;
  const bool aligned = al16(q) && al16(out) && q_sb % 8 == 0 && q_sh % 8 == 0 && q_st % 8 == 0 &&
                       al16(a.uk) && al16(a.uv) && al16(a.ck) && al16(a.cv) && a.c_sp % 4 == 0 &&
                       al16(a.seg_k[0]) && al16(a.seg_k[1]) && al16(a.seg_k[3]) && al16(a.seg_v[3]);
  if (!aligned) { set_error("factored chunk attention: operands must be 16-byte aligned"); return KVD_ERR_ARG; }
  const CaSmem L = ca_smem();
  if (int rc = ensure_smem((const void*)chunk_attn_kernel, L.total, "chunk_attn_kernel")) return rc;
  // split the key tiles so about two CTAs per SM run (each fits two to an
  // SM); splits write records that chunk_merge_kernel combines
  a.ntiles = 0;
  for (int i = 0; i < kCaSegs; ++i) a.ntiles += (a.seg_len[i] + kCaKeys - 1) / kCaKeys;
  const int qtiles = (a.rows + kCaRows - 1) / kCaRows;
  const long ctas = (long)qtiles * a.H * count;
  static int sm_count[kMaxDevices] = {0};
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
    if (sm_count[dev] == 0) cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    if (sm_count[dev] > 0) sms = sm_count[dev];
  }
  int nsplit = (int)((2L * sms + ctas - 1) / ctas);
  nsplit = max(1, min(nsplit, min(kCaMaxSplit, a.ntiles / 4)));
  const size_t need = (size_t)count * a.H * a.rows * nsplit * kCaRec * sizeof(float);
  if (nsplit > 1 && (!ws || ws_bytes < need || !al16(ws))) nsplit = 1;
  a.nsplit = nsplit;
  a.part = (float*)ws;
  dim3 grid(qtiles, a.H, count * nsplit);
  {
    KTimerScope kts_("chunk_attn_kernel", s);
    chunk_attn_kernel<<<grid, kCaThreads, L.total, s>>>(a);
  }
  if (int rc = check_launch("chunk_attn_kernel")) return rc;
  if (nsplit > 1) {
    const long per = (long)a.H * a.rows * kCaD;
    dim3 mg((unsigned)((per + 255) / 256), count);
    KTimerScope kts_("chunk_merge_kernel", s);
    chunk_merge_kernel<<<mg, 256, 0, s>>>(a);
  }
  return check_launch("chunk_merge_kernel");
}

}  // namespace kvd_host
