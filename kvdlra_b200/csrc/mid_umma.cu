// The dense middle reconstruction on the 5th-generation tensor cores
// (tcgen05, sm_100a): K = RoPE(C_k U_k^T) and V = C_v U_v^T for 128-token
// tiles of one problem, bf16 outputs -- the middle of the peek the
// reference materialises (bug_cache.py:1540-1575).
//
// A CTA of four warps owns one tile of 128 coordinate rows.  Per stream (K,
// then V) it stages the tile's coordinates once and the basis rows of a group
// of heads at a time (N <= 256 features) in shared memory, both K-major in the
// no-swizzle core-matrix layout the tensor core reads (8 rows x 16 bytes per
// core matrix), rounded to TF32; one thread issues ceil(r / 8) kind::tf32
// MMAs of 128 x N x 8 into tensor memory and commits them to an mbarrier; then
// every warp reads its 32 accumulator rows (one token per thread, the head's
// rotate-half partners d and d + D/2 in the same thread), applies RoPE at the
// token's position (keys) and stores bf16.  Waits are bounded: a wait that
// gives up sets the timeout status word and the CTA still frees its TMEM.
#include "kernels.cuh"
#include "umma.cuh"

namespace kvd {

constexpr int kMuTok = 128;      // tokens per CTA: the MMA's M
constexpr int kMuThreads = 128;  // warp w reads TMEM lanes (tokens) [32 w, 32 w + 32)
constexpr long kMuWaitPolls = 1L << 22;

struct MuPlan { int K, NG, a, b, cs, bar, total; };  // byte offsets into shared memory

__host__ __device__ inline MuPlan mu_plan(int D, int ld, int n, int ng) {
  MuPlan m;
  m.K = (ld + 7) & ~7;
  m.NG = ng;
  m.a = 0;                                // [128 rows][K] coordinates
  m.b = m.a + kMuTok * m.K * 4;           // [NG rows][K] basis rows of a head group
  m.cs = m.b + ng * m.K * 4;              // [128][D/2] (cos, sin)
  m.bar = m.cs + kMuTok * (D / 2) * 8;    // mbarrier + TMEM base
  m.total = m.bar + 16;
  return m;
}

// Byte offset of element (row, k) of a K-major operand with K columns in the
// core-matrix layout: core matrices along K are 128 bytes apart (LBO), row
// groups of 8 are K * 32 bytes apart (SBO).
__device__ __forceinline__ int cm_off(int row, int k, int K) {
  return (row >> 3) * (K * 32) + (k >> 2) * 128 + (row & 7) * 16 + (k & 3) * 4;
}

// rows [0, nrows) x columns [0, K) of a row-major fp32 source (pitch `ld`),
// columns >= `rank` and rows >= `valid` as zeros, rounded to TF32
__device__ __forceinline__ void mu_stage(unsigned char* dst, const float* src, long pitch, int nrows,
                                         int valid, int K, int rank) {
  const int q4 = K / 4;
  for (int e = threadIdx.x; e < nrows * q4; e += blockDim.x) {
    const int row = e / q4, k = 4 * (e % q4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < valid && k < rank) {
      v = *reinterpret_cast<const float4*>(src + row * pitch + k);
      if (k + 1 >= rank) v.y = 0.f;
      if (k + 2 >= rank) v.z = 0.f;
      if (k + 3 >= rank) v.w = 0.f;
    }
    v = make_float4(umma::to_tf32(v.x), umma::to_tf32(v.y), umma::to_tf32(v.z), umma::to_tf32(v.w));
    *reinterpret_cast<float4*>(dst + cm_off(row, k, K)) = v;
  }
}

template <int D>
__global__ void __launch_bounds__(kMuThreads) mid_hat_umma_kernel(
    const float* uk, const float* uv, long u_sp, int ld, const int* rk, const int* rv,
    const float* ck, const float* cv, long c_sp, const int* mid_pos, long mid_sp, int pos_base,
    int W, int H, const float* inv_freq, float scale, __nv_bfloat16* ok, __nv_bfloat16* ov, long ob,
    long oh, long ot, int l0, int ng, int* status) {
  constexpr int HALF = D / 2;
  extern __shared__ __align__(1024) unsigned char msm[];
  const int p = blockIdx.y;
  const int j0 = blockIdx.x * kMuTok;
  const int ntok = min(kMuTok, W - j0);
  const int n = H * D;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const MuPlan L = mu_plan(D, ld, n, ng);
  const int K = L.K;
  unsigned char* sa = msm + L.a;
  unsigned char* sb = msm + L.b;
  float2* cs = reinterpret_cast<float2*>(msm + L.cs);
  uint64_t* bar = reinterpret_cast<uint64_t*>(msm + L.bar);
  uint32_t* tbase = reinterpret_cast<uint32_t*>(msm + L.bar + 8);
  const uint32_t sa_addr = (uint32_t)__cvta_generic_to_shared(sa);
  const uint32_t sb_addr = (uint32_t)__cvta_generic_to_shared(sb);
  const int tcols = ng <= 32 ? 32 : (ng <= 64 ? 64 : (ng <= 128 ? 128 : 256));
  if (warp == 0) {
    umma::tmem_alloc(tbase, tcols);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    umma::mbar_init(bar, 1);
    umma::mbar_fence_init();
  }
  // rotary cos/sin of every (token, frequency) of the tile
  for (int e = tid; e < kMuTok * HALF; e += kMuThreads) {
    const int t = e / HALF, f = e % HALF;
    float c = 1.f, s = 0.f;
    if (t < ntok) {
      const int pos = mid_pos ? mid_pos[p * mid_sp + j0 + t] : pos_base + j0 + t;
      rope_cs(pos, inv_freq[f], scale, &c, &s);
    }
    cs[e] = make_float2(c, s);
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tbase;
  const uint32_t idesc = umma::idesc_tf32(kMuTok, ng);
  uint32_t phase = 0;
  bool ok_wait = true;
  const int row = 32 * warp + lane;  // this thread's token within the tile
  for (int s = 0; s < 2 && ok_wait; ++s) {
    const float* U = (s == 0 ? uk : uv) + p * u_sp;
    const float* Cc = (s == 0 ? ck : cv) + p * c_sp + (long)j0 * ld;
    const int rank = s == 0 ? rk[p] : rv[p];
    __nv_bfloat16* out = (s == 0 ? ok : ov) + p * ob;
    mu_stage(sa, Cc, ld, kMuTok, ntok, K, rank);
    for (int g0 = 0; g0 < n && ok_wait; g0 += ng) {
      mu_stage(sb, U + (long)g0 * ld, ld, ng, ng, K, rank);
      umma::fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) {
        umma::fence_after_sync();
        for (int j = 0; j < K / 8; ++j)
          umma::mma_tf32(tmem, umma::smem_desc(sa_addr + 256 * j, 128, 32 * K),
                         umma::smem_desc(sb_addr + 256 * j, 128, 32 * K), idesc, j > 0);
        umma::commit(bar);
      }
      ok_wait = umma::mbar_wait_bounded(bar, phase, kMuWaitPolls);
      phase ^= 1;
      umma::fence_after_sync();
      if (ok_wait) {
        const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
        for (int h0 = 0; h0 < ng; h0 += D) {  // each head of the group
          const int h = (g0 + h0) / D;
          __nv_bfloat16* orow = out + h * oh + (long)(l0 + j0 + row) * ot;
#pragma unroll
          for (int f0 = 0; f0 < HALF; f0 += 16) {
            float x1[16], x2[16];
            umma::tmem_ld16(trow + h0 + f0, x1);
            umma::tmem_ld16(trow + h0 + HALF + f0, x2);
            umma::tmem_wait_ld();
            if (row < ntok) {
              __align__(16) __nv_bfloat162 y1[8], y2[8];
#pragma unroll
              for (int i = 0; i < 16; i += 2) {
                float a0 = x1[i], a1 = x1[i + 1], b0 = x2[i], b1 = x2[i + 1];
                if (s == 0) {
                  const float2 c0 = cs[row * HALF + f0 + i], c1 = cs[row * HALF + f0 + i + 1];
                  float r0, r1, q0, q1;
                  rope_apply_pair(x1[i], x2[i], c0.x, c0.y, &r0, &q0);
                  rope_apply_pair(x1[i + 1], x2[i + 1], c1.x, c1.y, &r1, &q1);
                  a0 = r0; a1 = r1; b0 = q0; b1 = q1;
                }
                y1[i / 2] = __floats2bfloat162_rn(a0, a1);
                y2[i / 2] = __floats2bfloat162_rn(b0, b1);
              }
              uint4* d1 = reinterpret_cast<uint4*>(orow + f0);
              uint4* d2 = reinterpret_cast<uint4*>(orow + HALF + f0);
              d1[0] = reinterpret_cast<const uint4*>(y1)[0];
              d1[1] = reinterpret_cast<const uint4*>(y1)[1];
              d2[0] = reinterpret_cast<const uint4*>(y2)[0];
              d2[1] = reinterpret_cast<const uint4*>(y2)[1];
            }
          }
        }
      }
      umma::fence_before_sync();
      __syncthreads();  // accumulators read and staging free before the next group
    }
  }
  if (!ok_wait) {
    if (tid == 0) atomicOr(&status[kStatusTimeout], 8);
    // the MMAs committed last may still run: give them a second bounded wait
    umma::mbar_wait_bounded(bar, phase ^ 1, kMuWaitPolls);
    __syncthreads();
  }
  if (warp == 0) umma::tmem_dealloc(tmem, tcols);
}

}  // namespace kvd

namespace kvd_host {
using namespace kvd;

// Group of heads (multiple of D features, at most 256) whose staged operands
// fit the shared-memory budget; 0 = this path does not apply.
static int mu_group(int D, int ld, int n, int limit) {
  for (int ng = 256; ng >= D; ng -= D) {
    if (ng > n || n % ng) continue;
    if (mu_plan(D, ld, n, ng).total <= limit) return ng;
  }
  return 0;
}

int launch_mid_hat_umma(const kvd_config& c, const kvd_buffers& b, const kvd_counters& k, int p0,
                        int count, void* okp, void* ovp, long ob, long oh, long ot, int l0,
                        cudaStream_t s) {
  const int H = c.num_heads, D = c.head_dim, n = H * D, ld = c.rank;
  if (c.dtype != KVD_DTYPE_BF16 || (D != 64 && D != 128) || ld > 128 || ld % 4) return -1;
  if (ob % 8 || oh % 8 || ot % 8 || (reinterpret_cast<uintptr_t>(okp) & 15) ||
      (reinterpret_cast<uintptr_t>(ovp) & 15))
    return -1;
  const long u_sp = (long)n * ld, c_sp = (long)c.w_cap * ld;
  const float* uk = b.u_k[k.u_sel] + p0 * u_sp;
  const float* uv = b.u_v[k.u_sel] + p0 * u_sp;
  const float* ckp = b.c_k + p0 * c_sp;
  const float* cvp = b.c_v + p0 * c_sp;
  if ((reinterpret_cast<uintptr_t>(uk) | reinterpret_cast<uintptr_t>(uv) | reinterpret_cast<uintptr_t>(ckp) |
       reinterpret_cast<uintptr_t>(cvp)) & 15)
    return -1;
  const int ng = mu_group(D, ld, n, device_smem_optin());
  if (!ng) return -1;
  const int smem = mu_plan(D, ld, n, ng).total;
  auto fn = D == 64 ? mid_hat_umma_kernel<64> : mid_hat_umma_kernel<128>;
  if (int rc = ensure_smem((const void*)fn, smem, "mid_hat_kernel")) return rc;
  const int track_pos = c.retention != KVD_RETENTION_FIFO;
  const int mid_len = k.hh_len + k.w_len;
  const int pos_base = (int)(k.cumulative_length - k.ring_len - mid_len);
  dim3 grid((k.w_len + kMuTok - 1) / kMuTok, count);
  {
    KTimerScope kts_("mid_hat_kernel", s);
    fn<<<grid, kMuThreads, smem, s>>>(uk, uv, u_sp, ld, b.r_k + p0, b.r_v + p0, ckp, cvp, c_sp,
                                      track_pos ? b.mid_pos + (long)p0 * c.w_cap : nullptr, c.w_cap,
                                      pos_base, k.w_len, H, c.inv_freq, c.rope_scaling,
                                      (__nv_bfloat16*)okp, (__nv_bfloat16*)ovp, ob, oh, ot, l0, ng,
                                      b.status);
  }
  return check_launch("mid_hat_kernel");
}

}  // namespace kvd_host
