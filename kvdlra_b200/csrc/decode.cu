// Factored decode attention (sm_100a).
//
// One query token per problem attends to [sinks | exact tier | middle | ring]
// without materialising the middle (the reference materialises RoPE(U_k C_k)
// and U_v C_v in bug_cache.py:1540-1575 and runs dense attention over the
// peek of 1496-1519):
//   * middle keys   k_t = RoPE_{pos_t}(U_k,g c_k,t)   per KV group g, built in
//     registers from the coordinate row and the group's basis rows;
//   * middle values accumulate in coordinate space, acc_c += p_t c_v,t, and
//     are expanded once per split by U_v,g in the merge;
//   * verbatim tiers read K/V rows directly.
// Split-K over the token axis: each CTA handles `kChunk` tokens of one
// (problem, KV group) for all G = Hq/Hkv query heads of the group and writes
// (max, sum, acc_d, acc_c) partials; decode_merge_kernel combines them.
#include "kernels.cuh"
#include "umma.cuh"

namespace kvd {

constexpr int kDecThreads = 128;  // 4 warps
constexpr int kChunk = 256;       // tokens per CTA
constexpr int kMaxG = 8;          // query heads per KV group
constexpr int kMaxNV = 4;         // head_dim <= 128 -> 4 values per lane
constexpr int kMaxNC = 6;         // rank <= 192 -> 6 coordinates per lane

struct DecArgs {
  int H, D, G, ld, Hq;  // the KV heads (groups) and query heads this launch answers
  int nrow;             // features per token row of the tier buffers (every KV head of the cache)
  int sink_len, hh_len, W, ring_len, L;
  const void* sink_k; const void* sink_v; long sink_sp;
  const void* hh_k; const void* hh_v; long hh_sp;
  const void* ring_k; const void* ring_v; long ring_sp;  // offset to the first live slot
  const float* uk; const float* uv; long u_sp;
  const int* rk; const int* rv;
  const float* ck; const float* cv; long c_sp;
  const int* mid_pos; long mid_sp; int pos_base;
  const float* inv_freq; float rope_scale;
  const void* q; void* out;
  float scaling;
  float* part; long part_sp_chunk;  // partial record per (problem, group, chunk)
  int n_chunks;
  int* status;                      // device status words (bounded waits report here)
};

// Partial record layout (floats): m[G], l[G], acc_d[G][D], acc_c[G][ld]
__host__ __device__ inline long part_floats(int G, int D, int ld) { return 2L * G + (long)G * D + (long)G * ld; }

template <typename T, int NV, int NC>
__global__ void __launch_bounds__(kDecThreads) decode_split_kernel(DecArgs a) {
  extern __shared__ __align__(16) float dsm[];
  const int chunk = blockIdx.x, g = blockIdx.y, p = blockIdx.z;
  const int D = a.D, G = a.G, ld = a.ld, n = a.nrow, half = D / 2;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int r_k = a.rk[p], r_v = a.rv[p];
  float* qs = dsm;                       // [G][D]
  float* ukT = qs + G * D;               // [ld][D]   U_k,g transposed
  float* crow = ukT + ld * D;            // [4 warps][ld]
  float* red = crow + 4 * ld;            // merge scratch
  const T* qp = reinterpret_cast<const T*>(a.q) + (long)p * a.Hq * D;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int qh = e / D, d = e % D;
    qs[e] = load_f<T>(qp + (long)(g * G + qh) * D + d);
  }
  const int t0 = chunk * kChunk;
  const int t1 = min(a.L, t0 + kChunk);
  const int mid0 = a.sink_len + a.hh_len, mid1 = mid0 + a.W;
  const bool has_mid = (t0 < mid1) && (t1 > mid0);
  if (has_mid) {
    const float* U = a.uk + p * a.u_sp;
    for (int e = threadIdx.x; e < ld * D; e += blockDim.x) {
      const int c = e / D, d = e % D;
      ukT[e] = c < r_k ? U[(long)(g * D + d) * ld + c] : 0.f;
    }
  }
  __syncthreads();
  float mrun[kMaxG], lrun[kMaxG], accd[kMaxG][NV], accc[kMaxG][NC];
#pragma unroll
  for (int qh = 0; qh < kMaxG; ++qh) {
    mrun[qh] = -INFINITY; lrun[qh] = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) accd[qh][i] = 0.f;
#pragma unroll
    for (int i = 0; i < NC; ++i) accc[qh][i] = 0.f;
  }
  float* myrow = crow + warp * ld;
  for (int t = t0 + warp; t < t1; t += 4) {
    float kv[NV], vv[NV];
    bool is_mid = false;
    if (t < a.sink_len || t >= mid1 || t < mid0) {
      const T* kr; const T* vr;
      if (t < a.sink_len) {
        kr = reinterpret_cast<const T*>(a.sink_k) + p * a.sink_sp + (long)t * n;
        vr = reinterpret_cast<const T*>(a.sink_v) + p * a.sink_sp + (long)t * n;
      } else if (t < mid0) {
        const int j = t - a.sink_len;
        kr = reinterpret_cast<const T*>(a.hh_k) + p * a.hh_sp + (long)j * n;
        vr = reinterpret_cast<const T*>(a.hh_v) + p * a.hh_sp + (long)j * n;
      } else {
        const int j = t - mid1;
        kr = reinterpret_cast<const T*>(a.ring_k) + p * a.ring_sp + (long)j * n;
        vr = reinterpret_cast<const T*>(a.ring_v) + p * a.ring_sp + (long)j * n;
      }
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int d = lane + 32 * i;
        kv[i] = d < D ? load_f<T>(kr + g * D + d) : 0.f;
        vv[i] = d < D ? load_f<T>(vr + g * D + d) : 0.f;
      }
    } else {
      is_mid = true;
      const int j = t - mid0;
      const float* ct = a.ck + p * a.c_sp + (long)j * ld;
      for (int c = lane; c < r_k; c += 32) myrow[c] = ct[c];
      __syncwarp();
      float kp[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) kp[i] = 0.f;
      for (int c = 0; c < r_k; ++c) {
        const float cc = myrow[c];
        const float* ur = ukT + c * D;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int d = lane + 32 * i;
          if (d < D) kp[i] = fmaf(ur[d], cc, kp[i]);
        }
      }
      __syncwarp();
      // RoPE at the column's true position on rotate-half pairs (d, d + D/2)
      const int pos = a.mid_pos ? a.mid_pos[p * a.mid_sp + j] : a.pos_base + j;
      if (half % 32 == 0) {
        // both members of a pair sit in this lane: value i pairs with i + half/32
        const int off = half / 32;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          if (i % (2 * off) >= off) continue;
          const int f = lane + 32 * (i % off) + 64 * off * (i / (2 * off));
          float c = 1.f, s = 0.f;
          if (f < half) rope_cs(pos, a.inv_freq[f], a.rope_scale, &c, &s);
          float y1, y2;
          rope_apply_pair(kp[i], kp[i + off], c, s, &y1, &y2);
          kv[i] = y1;
          kv[i + off] = y2;
        }
      } else {
        // D <= 32: one value per lane, the partner lives in lane d +- D/2
        const int d = lane;
        const int partner = d < half ? d + half : d - half;
        const float other = __shfl_sync(0xffffffffu, kp[0], partner < 32 ? partner : lane);
        const int f = d < half ? d : d - half;
        float c = 1.f, s = 0.f;
        if (d < D) rope_cs(pos, a.inv_freq[f], a.rope_scale, &c, &s);
        kv[0] = d < half ? kp[0] * c - other * s : kp[0] * c + other * s;
#pragma unroll
        for (int i = 1; i < NV; ++i) kv[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < NV; ++i) vv[i] = 0.f;
    }
    // scores for the group's query heads
    float cvals[NC];
    if (is_mid) {
      const float* cvt = a.cv + p * a.c_sp + (long)(t - mid0) * ld;
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        const int c = lane + 32 * i;
        cvals[i] = c < r_v ? cvt[c] : 0.f;
      }
    }
#pragma unroll
    for (int qh = 0; qh < kMaxG; ++qh) {
      if (qh >= G) break;
      float sdot = 0.f;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int d = lane + 32 * i;
        if (d < D) sdot = fmaf(qs[qh * D + d], kv[i], sdot);
      }
      sdot = warp_sum(sdot) * a.scaling;
      const float mnew = fmaxf(mrun[qh], sdot);
      const float corr = expf(mrun[qh] - mnew);
      const float pw = expf(sdot - mnew);
      lrun[qh] = lrun[qh] * corr + pw;
      mrun[qh] = mnew;
#pragma unroll
      for (int i = 0; i < NV; ++i) accd[qh][i] = accd[qh][i] * corr + pw * vv[i];
#pragma unroll
      for (int i = 0; i < NC; ++i) accc[qh][i] = accc[qh][i] * corr + (is_mid ? pw * cvals[i] : 0.f);
    }
  }
  // combine the 4 warps of the CTA through shared memory
  __syncthreads();
  const long rec = part_floats(G, D, ld);
  float* wrec = red + warp * rec;  // per-warp record
  for (int qh = 0; qh < G; ++qh) {
    if (lane == 0) { wrec[qh] = mrun[qh]; wrec[G + qh] = lrun[qh]; }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int d = lane + 32 * i;
      if (d < D) wrec[2 * G + qh * D + d] = accd[qh][i];
    }
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      if (c < ld) wrec[2 * G + G * D + qh * ld + c] = accc[qh][i];
    }
  }
  __syncthreads();
  float* out = a.part + ((long)(p * a.H + g) * a.n_chunks + chunk) * a.part_sp_chunk;
  for (int e = threadIdx.x; e < rec; e += blockDim.x) {
    // e indexes the record; find its query head
    int qh;
    if (e < 2 * G) qh = e % G;
    else if (e < 2 * G + G * D) qh = (e - 2 * G) / D;
    else qh = (e - 2 * G - G * D) / ld;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, red[w * rec + qh]);
    float v;
    if (e < G) {
      v = M;
    } else {
      v = 0.f;
      for (int w = 0; w < 4; ++w) {
        const float mw = red[w * rec + qh];
        const float sc = (mw == -INFINITY) ? 0.f : expf(mw - M);
        v += sc * red[w * rec + e];
      }
    }
    out[e] = v;
  }
}

// ---------------------------------------------------------------- tiled decode
// Tokens in tiles of kTT, a CTA walking kTilesPerCta consecutive tiles of one
// (problem, KV group) with the online-softmax state in registers.  A tile is
// either verbatim (sinks + exact tier, or the ring: K/V rows read directly)
// or middle: its keys are rebuilt as the register-tiled product
// C_k (kTT x r) U_k,g^T (r x D) -- a thread owns 4 tokens x 2*DPT dims that
// form DPT rotate-half pairs, so RoPE is applied in registers -- and its
// values accumulate in coordinate space.  One partial record per CTA.
constexpr int kTT = 64;
constexpr int kTileThreads = 128;
constexpr int kTilesPerCta = 8;

template <typename T, int D>
__global__ void __launch_bounds__(kTileThreads) decode_tile_kernel(DecArgs a, int nv0, int nm,
                                                                   int n_tiles) {
  constexpr int half = D / 2, DPT = half / 8;  // pairs per thread
  constexpr int ldk = D + 4;                   // = 4 mod 8: row-per-lane float4 reads conflict-free
  extern __shared__ __align__(16) float tsm[];
  const int chunk = blockIdx.x, g = blockIdx.y, p = blockIdx.z;
  const int G = a.G, ld = a.ld, n = a.nrow;
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int r_k = a.rk[p], r_v = a.rv[p];
  const int ldc = ld + 4;
  float* qs = tsm;                    // [G][D]
  float* ks = qs + G * D;             // [kTT][ldk] keys of the tile
  float* vs = ks + kTT * ldk;         // [kTT][ldk] values, or [kTT][ldc] value coordinates
  float* ps = vs + kTT * ldk;         // [G][kTT] scores, then probabilities
  float* ut = ps + G * kTT;           // [ld][D] U_k,g^T
  constexpr int kTTp = kTT + 4;       // = 4 mod 8: transposing writes spread over banks
  float* ct = ut + ld * D;            // [ld][kTTp] key coordinates, transposed
  float* st = ct + ld * kTTp;         // [G][4] -, -, running max, rescale of the tile
  const T* qp = reinterpret_cast<const T*>(a.q) + (long)p * a.Hq * D;
  for (int e = tid; e < G * D; e += kTileThreads) qs[e] = load_f<T>(qp + (long)(g * G + e / D) * D + e % D);
  const int mid0 = a.sink_len + a.hh_len;
  // running state: outputs o = tid + kTileThreads * k over [acc_d (G x D) | acc_c (G x ld)]
  const int n_out = G * (D + ld);
  constexpr int kMaxOut = 12;  // (G <= 8) x (D + ld <= 192) / 128
  float acc[kMaxOut];
#pragma unroll
  for (int k = 0; k < kMaxOut; ++k) acc[k] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // of head `warp`-strided: kept in st for all threads
  if (tid < G) { st[4 * tid + 2] = -INFINITY; }
  float lsum[2] = {0.f, 0.f};  // l_run of heads warp, warp + 4 (owned by lane 0 of each warp)
  (void)m_run; (void)l_run;
  // the thread's inverse frequencies (middle tiles)
  const int dg = tid % 8, tg = tid / 8;
  float invf[DPT];
#pragma unroll
  for (int j = 0; j < DPT; ++j) invf[j] = a.inv_freq[dg * DPT + j];
  const int t_begin = chunk * kTilesPerCta, t_end = min(n_tiles, t_begin + kTilesPerCta);
  if (t_end > nv0 && t_begin < nv0 + nm) {  // U_k,g^T, once for the CTA's middle tiles
    const float* U = a.uk + p * a.u_sp;
    for (int e = tid; e < ld * D; e += kTileThreads) {
      const int d = e / ld, c = e % ld;
      ut[c * D + d] = c < r_k ? U[(long)(g * D + d) * ld + c] : 0.f;
    }
  }
  for (int tile = t_begin; tile < t_end; ++tile) {
    __syncthreads();  // previous tile's buffers are free
    int kind, j0, ntok;
    if (tile < nv0) { kind = 0; j0 = tile * kTT; ntok = min(kTT, mid0 - j0); }
    else if (tile < nv0 + nm) { kind = 1; j0 = (tile - nv0) * kTT; ntok = min(kTT, a.W - j0); }
    else { kind = 2; j0 = (tile - nv0 - nm) * kTT; ntok = min(kTT, a.ring_len - j0); }
    if (kind != 1) {
      for (int e = tid; e < kTT * D; e += kTileThreads) {
        const int tt = e / D, d = e % D;
        float kv = 0.f, vv = 0.f;
        if (tt < ntok) {
          const int t = j0 + tt;
          const T* kr; const T* vr;
          if (kind == 2) {
            kr = reinterpret_cast<const T*>(a.ring_k) + p * a.ring_sp + (long)t * n;
            vr = reinterpret_cast<const T*>(a.ring_v) + p * a.ring_sp + (long)t * n;
          } else if (t < a.sink_len) {
            kr = reinterpret_cast<const T*>(a.sink_k) + p * a.sink_sp + (long)t * n;
            vr = reinterpret_cast<const T*>(a.sink_v) + p * a.sink_sp + (long)t * n;
          } else {
            kr = reinterpret_cast<const T*>(a.hh_k) + p * a.hh_sp + (long)(t - a.sink_len) * n;
            vr = reinterpret_cast<const T*>(a.hh_v) + p * a.hh_sp + (long)(t - a.sink_len) * n;
          }
          kv = load_f<T>(kr + g * D + d);
          vv = load_f<T>(vr + g * D + d);
        }
        ks[tt * ldk + d] = kv;
        vs[tt * ldk + d] = vv;
      }
    } else {
      const float* Ck = a.ck + p * a.c_sp + (long)j0 * ld;
      const float* Cv = a.cv + p * a.c_sp + (long)j0 * ld;
      for (int e = tid; e < kTT * ld; e += kTileThreads) {
        const int tt = e / ld, c = e % ld;
        const bool in = tt < ntok;
        ct[c * kTTp + tt] = (in && c < r_k) ? Ck[(long)tt * ld + c] : 0.f;
        vs[tt * ldc + c] = (in && c < r_v) ? Cv[(long)tt * ld + c] : 0.f;
      }
      __syncthreads();
      float kacc[4][2 * DPT];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 2 * DPT; ++j) kacc[i][j] = 0.f;
      for (int c = 0; c < r_k; ++c) {
        const float4 cv4 = *reinterpret_cast<const float4*>(ct + c * kTTp + 4 * tg);
        const float cc[4] = {cv4.x, cv4.y, cv4.z, cv4.w};
        float uu[2 * DPT];
#pragma unroll
        for (int j = 0; j < DPT; j += 4) {
          const float4 lo = *reinterpret_cast<const float4*>(ut + c * D + dg * DPT + j);
          const float4 hi = *reinterpret_cast<const float4*>(ut + c * D + half + dg * DPT + j);
          uu[j] = lo.x; uu[j + 1] = lo.y; uu[j + 2] = lo.z; uu[j + 3] = lo.w;
          uu[DPT + j] = hi.x; uu[DPT + j + 1] = hi.y; uu[DPT + j + 2] = hi.z; uu[DPT + j + 3] = hi.w;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 2 * DPT; ++j) kacc[i][j] = fmaf(cc[i], uu[j], kacc[i][j]);
      }
      // RoPE at each column's true position on the pairs (f, f + D/2)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tt = 4 * tg + i;
        const int jj = j0 + tt;
        const int pos = tt < ntok ? (a.mid_pos ? a.mid_pos[p * a.mid_sp + jj] : a.pos_base + jj) : 0;
#pragma unroll
        for (int j = 0; j < DPT; ++j) {
          float cs, sn;
          rope_cs(pos, invf[j], a.rope_scale, &cs, &sn);
          float y1, y2;
          rope_apply_pair(kacc[i][j], kacc[i][DPT + j], cs, sn, &y1, &y2);
          ks[tt * ldk + dg * DPT + j] = y1;
          ks[tt * ldk + half + dg * DPT + j] = y2;
        }
      }
    }
    __syncthreads();
    // scores of the group's query heads: thread -> token tt, heads hs, hs + 2, ...
    {
      const int tt = tid % kTT, hs = tid / kTT;
      const float* kr = ks + tt * ldk;
      for (int h = hs; h < G; h += kTileThreads / kTT) {
        const float* qr = qs + h * D;
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int d = 0; d < D; d += 8) {
          const float4 k0 = *reinterpret_cast<const float4*>(kr + d);
          const float4 k1 = *reinterpret_cast<const float4*>(kr + d + 4);
          const float4 q0 = *reinterpret_cast<const float4*>(qr + d);
          const float4 q1 = *reinterpret_cast<const float4*>(qr + d + 4);
          s0 = fmaf(q0.x, k0.x, s0); s0 = fmaf(q0.y, k0.y, s0); s0 = fmaf(q0.z, k0.z, s0); s0 = fmaf(q0.w, k0.w, s0);
          s1 = fmaf(q1.x, k1.x, s1); s1 = fmaf(q1.y, k1.y, s1); s1 = fmaf(q1.z, k1.z, s1); s1 = fmaf(q1.w, k1.w, s1);
        }
        ps[h * kTT + tt] = tt < ntok ? (s0 + s1) * a.scaling : -INFINITY;
      }
    }
    __syncthreads();
    // per head: tile max and probabilities relative to the new running max
    for (int h = warp; h < G; h += kTileThreads / 32) {
      float* pr = ps + h * kTT;
      const float x0 = pr[lane], x1 = pr[lane + 32];
      float mt = fmaxf(x0, x1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
      const float mold = st[4 * h + 2];
      const float mnew = fmaxf(mold, mt);
      const float e0 = mnew == -INFINITY ? 0.f : expf(x0 - mnew);
      const float e1 = mnew == -INFINITY ? 0.f : expf(x1 - mnew);
      pr[lane] = e0;
      pr[lane + 32] = e1;
      float ls = e0 + e1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
      const float corr = (mold == -INFINITY) ? 0.f : expf(mold - mnew);
      if (lane == 0) {
        const int slot = h / (kTileThreads / 32);
        lsum[slot] = lsum[slot] * corr + ls;
        st[4 * h + 2] = mnew;
        st[4 * h + 3] = corr;
      }
    }
    __syncthreads();
    // accumulate: acc_d over verbatim tokens, acc_c over middle tokens
#pragma unroll
    for (int k = 0; k < kMaxOut; ++k) {
      const int o = tid + kTileThreads * k;
      if (o >= n_out) break;
      int h;
      float add = 0.f;
      if (o < G * D) {
        h = o / D;
        if (kind != 1) {
          const int d = o % D;
          const float* pr = ps + h * kTT;
          for (int tt = 0; tt < ntok; ++tt) add = fmaf(pr[tt], vs[tt * ldk + d], add);
        }
      } else {
        const int oc = o - G * D;
        h = oc / ld;
        if (kind == 1) {
          const int c = oc % ld;
          const float* pr = ps + h * kTT;
          for (int tt = 0; tt < ntok; ++tt) add = fmaf(pr[tt], vs[tt * ldc + c], add);
        }
      }
      acc[k] = fmaf(acc[k], st[4 * h + 3], add);
    }
  }
  __syncthreads();
  // the CTA's partial record: m[G], l[G], acc_d[G][D], acc_c[G][ld]
  float* out = a.part + ((long)(p * a.H + g) * a.n_chunks + chunk) * a.part_sp_chunk;
  for (int h = warp; h < G; h += kTileThreads / 32)
    if (lane == 0) {
      out[h] = t_begin < t_end ? st[4 * h + 2] : -INFINITY;
      out[G + h] = lsum[h / (kTileThreads / 32)];
    }
#pragma unroll
  for (int k = 0; k < kMaxOut; ++k) {
    const int o = tid + kTileThreads * k;
    if (o >= n_out) break;
    out[2 * G + o] = acc[k];
  }
}

// The 16 / sizeof(T) elements of one 16-byte chunk, widened to fp32.
template <typename T> __device__ __forceinline__ void widen_chunk(uint4 r, float* v);
template <> __device__ __forceinline__ void widen_chunk<float>(uint4 r, float* v) {
  v[0] = __uint_as_float(r.x); v[1] = __uint_as_float(r.y);
  v[2] = __uint_as_float(r.z); v[3] = __uint_as_float(r.w);
}
template <> __device__ __forceinline__ void widen_chunk<__nv_bfloat16>(uint4 r, float* v) {
  const unsigned w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // bf16 -> fp32 is the 16 bits shifted up
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// ------------------------------------------------------- tensor-core decode
// decode_tile_kernel's tiling with the three products of a middle tile on
// the tensor cores (warp-level TF32 m16n8k8, fp32 accumulation; SPLIT =
// 3xTF32 products, ~fp32 accuracy, for fp32 models).  Warp w owns tokens
// 16w .. 16w+15 of the tile:
//   * keys     K = C_k (16 x r) U_k,g^T (r x D) in accumulator fragments; a
//     thread holds columns 8j + 2t, 8j + 2t + 1 of every n-tile j, so the
//     rotate-half partners (d, d + D/2) sit in its registers and RoPE is
//     applied there, one angle per (token, frequency);
//   * scores   S = K q^T: the key fragments are the A operand directly, with
//     the k index of each 8-column block permuted (accumulator column 2t
//     and 2t+1 as A columns t and t+4) and q's B fragment permuted alike;
//   * values   acc_c (heads x r) += P (heads x tokens) C_v (tokens x r), warp
//     w owning the coordinate n-tiles w, w + 4, ..; kept in fragments across
//     tiles with the online-softmax rescale.
// Verbatim tiles (sinks, exact tier, ring) are handled as in decode_tile_kernel.
constexpr int kMaxCT = 4;  // coordinate n-tiles per warp: rank <= 4 * 4 * 8 = 128

template <typename T, int D, bool SPLIT>
__global__ void __launch_bounds__(kTileThreads) decode_mma_kernel(DecArgs a, int nv0, int nm,
                                                                  int n_tiles, int tpc) {
  constexpr int half = D / 2, NT = D / 8, HT = D / 16;
  constexpr int ldk = D + 4;
  constexpr int ldps = kTT + 4;  // = 4 mod 32: P fragment reads (4g + t) conflict-free
  extern __shared__ __align__(16) float tsm[];
  const int chunk = blockIdx.x, g = blockIdx.y, p = blockIdx.z;
  const int G = a.G, ld = a.ld, n = a.nrow;
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int gq = lane >> 2, tq = lane & 3;
  const int r_k = a.rk[p], r_v = a.rv[p];
  const int ldc = ld + 4;  // key coordinates / basis rows: fragment reads (4g + t) conflict-free
  const int ldv = ld + 8;  // value coordinates: fragment reads (8t + g) conflict-free
  // a launch without middle tiles (nm == 0) holds no coordinates or basis
  const int vsz = kTT * (nm > 0 && ldv > ldk ? ldv : ldk);
  float* qs = tsm;              // [G][D]
  float* ks = qs + G * D;       // [kTT][ldk] keys | [kTT][ldc] key coordinates
  float* vs = ks + kTT * ldk;   // [kTT][ldk] values | [kTT][ldv] value coordinates
  float* ps = vs + vsz;         // [G][ldps] scores, then probabilities
  float* us = ps + G * ldps;    // [D][ldc] U_k,g rows (middle tiles only)
  float* st = us + (nm > 0 ? D * ldc : 0);  // [G][4] -, -, running max, rescale of the tile
  const T* qp = reinterpret_cast<const T*>(a.q) + (long)p * a.Hq * D;
  for (int e = tid; e < G * D; e += kTileThreads) qs[e] = load_f<T>(qp + (long)(g * G + e / D) * D + e % D);
  if (tid < G) st[4 * tid + 2] = -INFINITY;
  const int mid0 = a.sink_len + a.hh_len;
  const int t_begin = chunk * tpc, t_end = min(n_tiles, t_begin + tpc);
  if (t_end > nv0 && t_begin < nv0 + nm) {  // U_k,g rows, once for the CTA's middle tiles
    const float* U = a.uk + p * a.u_sp;
    for (int e = tid; e < D * ld; e += kTileThreads) {
      const int d = e / ld, c = e % ld;
      us[d * ldc + c] = c < r_k ? U[(long)(g * D + d) * ld + c] : 0.f;
    }
  }
  __syncthreads();
  // q's B fragments for the scores product (heads >= G are zero)
  float qf[NT][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    qf[j][0] = gq < G ? qs[gq * D + 8 * j + 2 * tq] : 0.f;
    qf[j][1] = gq < G ? qs[gq * D + 8 * j + 2 * tq + 1] : 0.f;
  }
  // verbatim outputs acc_d (G x D) strided over the threads; acc_c in fragments
  const int n_outd = G * D;
  constexpr int kMaxOutD = 8;  // (G <= 8) x (D <= 128) / 128
  float acc[kMaxOutD];
#pragma unroll
  for (int k = 0; k < kMaxOutD; ++k) acc[k] = 0.f;
  float cacc[kMaxCT][4];
#pragma unroll
  for (int i = 0; i < kMaxCT; ++i)
#pragma unroll
    for (int q = 0; q < 4; ++q) cacc[i][q] = 0.f;
  const int nct = ld / 8;
  float lsum[2] = {0.f, 0.f};  // running sums of heads warp, warp + 4 (lane 0 of each warp)
  for (int tile = t_begin; tile < t_end; ++tile) {
    __syncthreads();  // previous tile's buffers are free
    int kind, j0, ntok;
    if (tile < nv0) { kind = 0; j0 = tile * kTT; ntok = min(kTT, mid0 - j0); }
    else if (tile < nv0 + nm) { kind = 1; j0 = (tile - nv0) * kTT; ntok = min(kTT, a.W - j0); }
    else { kind = 2; j0 = (tile - nv0 - nm) * kTT; ntok = min(kTT, a.ring_len - j0); }
    if (kind != 1) {
      // the group's rows of the tile as 16-byte chunks (all in flight), widened to fp32
      constexpr int kPer = 16 / sizeof(T), kQ = D / kPer;
      for (int e = tid; e < kTT * kQ; e += kTileThreads) {
        const int tt = e / kQ, c = (e % kQ) * kPer;
        float kv[kPer], vv[kPer];
#pragma unroll
        for (int q = 0; q < kPer; ++q) { kv[q] = 0.f; vv[q] = 0.f; }
        if (tt < ntok) {
          const int t = j0 + tt;
          const T* kr; const T* vr;
          if (kind == 2) {
            kr = reinterpret_cast<const T*>(a.ring_k) + p * a.ring_sp + (long)t * n;
            vr = reinterpret_cast<const T*>(a.ring_v) + p * a.ring_sp + (long)t * n;
          } else if (t < a.sink_len) {
            kr = reinterpret_cast<const T*>(a.sink_k) + p * a.sink_sp + (long)t * n;
            vr = reinterpret_cast<const T*>(a.sink_v) + p * a.sink_sp + (long)t * n;
          } else {
            kr = reinterpret_cast<const T*>(a.hh_k) + p * a.hh_sp + (long)(t - a.sink_len) * n;
            vr = reinterpret_cast<const T*>(a.hh_v) + p * a.hh_sp + (long)(t - a.sink_len) * n;
          }
          kr += g * D + c;
          vr += g * D + c;
          if (((reinterpret_cast<uintptr_t>(kr) | reinterpret_cast<uintptr_t>(vr)) & 15) == 0) {
            widen_chunk<T>(*reinterpret_cast<const uint4*>(kr), kv);
            widen_chunk<T>(*reinterpret_cast<const uint4*>(vr), vv);
          } else {
#pragma unroll
            for (int q = 0; q < kPer; ++q) { kv[q] = load_f<T>(kr + q); vv[q] = load_f<T>(vr + q); }
          }
        }
#pragma unroll
        for (int q = 0; q < kPer; q += 4) {
          *reinterpret_cast<float4*>(ks + tt * ldk + c + q) = make_float4(kv[q], kv[q + 1], kv[q + 2], kv[q + 3]);
          *reinterpret_cast<float4*>(vs + tt * ldk + c + q) = make_float4(vv[q], vv[q + 1], vv[q + 2], vv[q + 3]);
        }
      }
      __syncthreads();
      const int tt = tid % kTT, hs = tid / kTT;  // thread -> token tt, heads hs, hs + 2, ...
      const float* kr = ks + tt * ldk;
      for (int h = hs; h < G; h += kTileThreads / kTT) {
        const float* qr = qs + h * D;
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int d = 0; d < D; d += 8) {
          const float4 k0 = *reinterpret_cast<const float4*>(kr + d);
          const float4 k1 = *reinterpret_cast<const float4*>(kr + d + 4);
          const float4 q0 = *reinterpret_cast<const float4*>(qr + d);
          const float4 q1 = *reinterpret_cast<const float4*>(qr + d + 4);
          s0 = fmaf(q0.x, k0.x, s0); s0 = fmaf(q0.y, k0.y, s0); s0 = fmaf(q0.z, k0.z, s0); s0 = fmaf(q0.w, k0.w, s0);
          s1 = fmaf(q1.x, k1.x, s1); s1 = fmaf(q1.y, k1.y, s1); s1 = fmaf(q1.z, k1.z, s1); s1 = fmaf(q1.w, k1.w, s1);
        }
        ps[h * ldps + tt] = tt < ntok ? (s0 + s1) * a.scaling : -INFINITY;
      }
    } else {
      const float* Ck = a.ck + p * a.c_sp + (long)j0 * ld;
      const float* Cv = a.cv + p * a.c_sp + (long)j0 * ld;
      const int l4 = ld / 4;
      for (int e = tid; e < kTT * l4; e += kTileThreads) {
        const int tt = e / l4, c = 4 * (e % l4);
        float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
        if (tt < ntok) {
          kv = *reinterpret_cast<const float4*>(Ck + (long)tt * ld + c);
          vv = *reinterpret_cast<const float4*>(Cv + (long)tt * ld + c);
          if (c + 4 > r_k) { if (c >= r_k) kv.x = 0.f; if (c + 1 >= r_k) kv.y = 0.f; if (c + 2 >= r_k) kv.z = 0.f; kv.w = 0.f; }
          if (c + 4 > r_v) { if (c >= r_v) vv.x = 0.f; if (c + 1 >= r_v) vv.y = 0.f; if (c + 2 >= r_v) vv.z = 0.f; vv.w = 0.f; }
        }
        *reinterpret_cast<float4*>(ks + tt * ldc + c) = kv;
        *reinterpret_cast<float4*>(vs + tt * ldv + c) = vv;
      }
      __syncthreads();
      // keys of rows tt0 = 16w + g and tt1 = tt0 + 8
      const int tt0 = warp * 16 + gq, tt1 = tt0 + 8;
      float kacc[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) kacc[j][q] = 0.f;
      const int nkk = (r_k + 7) / 8;
      for (int kk = 0; kk < nkk; ++kk) {
        const int c0 = kk * 8 + tq;
        const float af[4] = {ks[tt0 * ldc + c0], ks[tt1 * ldc + c0], ks[tt0 * ldc + c0 + 4],
                             ks[tt1 * ldc + c0 + 4]};
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const float* ur = us + (j * 8 + gq) * ldc + c0;
          mma_f32<SPLIT>(kacc[j], af, ur[0], ur[4]);
        }
      }
      // RoPE on the pairs (8j + 2t + e, + D/2) at each row's true position
      const int pos0 = tt0 < ntok ? (a.mid_pos ? a.mid_pos[p * a.mid_sp + j0 + tt0] : a.pos_base + j0 + tt0) : 0;
      const int pos1 = tt1 < ntok ? (a.mid_pos ? a.mid_pos[p * a.mid_sp + j0 + tt1] : a.pos_base + j0 + tt1) : 0;
#pragma unroll
      for (int j = 0; j < HT; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float w = a.inv_freq[8 * j + 2 * tq + e];
          float c0, s0, c1, s1, y1, y2;
          rope_cs_fast(pos0, w, a.rope_scale, &c0, &s0);
          rope_cs_fast(pos1, w, a.rope_scale, &c1, &s1);
          rope_apply_pair(kacc[j][e], kacc[j + HT][e], c0, s0, &y1, &y2);
          kacc[j][e] = y1; kacc[j + HT][e] = y2;
          rope_apply_pair(kacc[j][2 + e], kacc[j + HT][2 + e], c1, s1, &y1, &y2);
          kacc[j][2 + e] = y1; kacc[j + HT][2 + e] = y2;
        }
      // scores of the group's heads (n = head, heads >= G zero)
      float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const float af[4] = {kacc[j][0], kacc[j][2], kacc[j][1], kacc[j][3]};
        mma_f32<SPLIT>(sacc, af, qf[j][0], qf[j][1]);
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int h = 2 * tq + e;
        if (h < G) {
          ps[h * ldps + tt0] = tt0 < ntok ? sacc[e] * a.scaling : -INFINITY;
          ps[h * ldps + tt1] = tt1 < ntok ? sacc[2 + e] * a.scaling : -INFINITY;
        }
      }
    }
    __syncthreads();
    // per head: tile max and probabilities relative to the new running max
    for (int h = warp; h < G; h += kTileThreads / 32) {
      float* pr = ps + h * ldps;
      const float x0 = pr[lane], x1 = pr[lane + 32];
      float mt = fmaxf(x0, x1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
      const float mold = st[4 * h + 2];
      const float mnew = fmaxf(mold, mt);
      const float e0 = mnew == -INFINITY ? 0.f : expf(x0 - mnew);
      const float e1 = mnew == -INFINITY ? 0.f : expf(x1 - mnew);
      pr[lane] = e0;
      pr[lane + 32] = e1;
      float ls = e0 + e1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
      const float corr = (mold == -INFINITY) ? 0.f : expf(mold - mnew);
      if (lane == 0) {
        const int slot = h / (kTileThreads / 32);
        lsum[slot] = lsum[slot] * corr + ls;
        st[4 * h + 2] = mnew;
        st[4 * h + 3] = corr;
      }
    }
    __syncthreads();
    // acc_d over verbatim tokens
#pragma unroll
    for (int k = 0; k < kMaxOutD; ++k) {
      const int o = tid + kTileThreads * k;
      if (o >= n_outd) break;
      const int h = o / D;
      float add = 0.f;
      if (kind != 1) {
        const int d = o % D;
        const float* pr = ps + h * ldps;
        for (int tt = 0; tt < ntok; ++tt) add = fmaf(pr[tt], vs[tt * ldk + d], add);
      }
      acc[k] = fmaf(acc[k], st[4 * h + 3], add);
    }
    // acc_c = corr * acc_c (+ P C_v on middle tiles); fragment rows are heads
    const float corr_g = gq < G ? st[4 * gq + 3] : 0.f;
#pragma unroll
    for (int i = 0; i < kMaxCT; ++i) {
      const int ct = warp + 4 * i;
      if (ct >= nct) break;
      cacc[i][0] *= corr_g;
      cacc[i][1] *= corr_g;
      if (kind == 1) {
#pragma unroll 2
        for (int kk = 0; kk < kTT / 8; ++kk) {
          const int t0 = kk * 8 + tq;
          const float af[4] = {gq < G ? ps[gq * ldps + t0] : 0.f, 0.f,
                               gq < G ? ps[gq * ldps + t0 + 4] : 0.f, 0.f};
          mma_f32<SPLIT>(cacc[i], af, vs[t0 * ldv + ct * 8 + gq], vs[(t0 + 4) * ldv + ct * 8 + gq]);
        }
      }
    }
  }
  __syncthreads();
  // the CTA's partial record: m[G], l[G], acc_d[G][D], acc_c[G][ld]
  float* out = a.part + ((long)(p * a.H + g) * a.n_chunks + chunk) * a.part_sp_chunk;
  for (int h = warp; h < G; h += kTileThreads / 32)
    if (lane == 0) {
      out[h] = t_begin < t_end ? st[4 * h + 2] : -INFINITY;
      out[G + h] = lsum[h / (kTileThreads / 32)];
    }
#pragma unroll
  for (int k = 0; k < kMaxOutD; ++k) {
    const int o = tid + kTileThreads * k;
    if (o >= n_outd) break;
    out[2 * G + o] = acc[k];
  }
  if (nm == 0) {  // no middle tiles: acc_c is zero (at any rank)
    for (int e = tid; e < G * ld; e += kTileThreads) out[2 * G + G * D + e] = 0.f;
  } else if (gq < G) {
#pragma unroll
    for (int i = 0; i < kMaxCT; ++i) {
      const int ct = warp + 4 * i;
      if (ct >= nct) break;
      float* oc = out + 2 * G + G * D + gq * ld + ct * 8 + 2 * tq;
      oc[0] = cacc[i][0];
      oc[1] = cacc[i][1];
    }
  }
}

// ------------------------------------------------ middle tier, all groups
// One CTA per (chunk of middle tiles, problem) for every KV group at once,
// so a tile's coordinates are staged once (cp.async, the next tile's copy
// in flight during this tile's work) and its rotary angles computed once per
// (token, frequency).  Warps take (16-token row block, group) tasks: key
// rebuild C_k U_k,g^T, RoPE in the accumulator fragments, scores against the
// group's heads (as decode_mma_kernel).  The value product runs over all
// Hq = H*G query heads at once, acc_c (Hq x r) += P (Hq x tokens) C_v, in
// (16-head m-tile, 8-coordinate n-tile) fragments spread over the warps.
// Staged operands are masked (tokens past the tile, coordinates past the
// rank) and, without SPLIT, rounded to TF32 once in shared memory, so the
// fragment loads feed the MMAs directly.  Each CTA writes one partial record
// per group (acc_d zero).
constexpr int kMidThreads = 512;
constexpr int kMidWarps = kMidThreads / 32;
constexpr int kMaxPW = 2;   // value-product fragments per warp: ceil(Hq/16) * r/8 <= 32
constexpr int kMaxRW = 4;   // softmax rows per warp: Hq <= 64

__device__ __forceinline__ void cp_async16_dec(void* smem_dst, const void* gsrc) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async4_dec(void* smem_dst, const void* gsrc) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(sa), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait0() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

// Shared-memory layout of decode_mid_kernel (floats), host and device alike.
struct MidSmem {
  int ldc, ldv, cpitch, us, qs, cbuf, cbsz, cosb, sinb, ps, st, posb, invs, total;
};
__host__ __device__ inline MidSmem mid_smem(int n, int Hq, int D, int ld) {
  MidSmem m;
  m.ldc = ld + 4;        // key coordinates / basis rows: A and B fragment reads conflict-free
  m.ldv = ld + 8;        // value coordinates: B fragment reads conflict-free
  m.cpitch = D / 2 + 4;  // cos / sin rows
  m.us = 0;                                     // [n][ldc]
  m.qs = m.us + n * m.ldc;                      // [Hq][D]
  m.cbuf = m.qs + Hq * D;                       // 2 x ([kTT][ldc] + [kTT][ldv])
  m.cbsz = kTT * (m.ldc + m.ldv);
  m.cosb = m.cbuf + 2 * m.cbsz;                 // [kTT][cpitch]
  m.sinb = m.cosb + kTT * m.cpitch;             // [kTT][cpitch]
  m.ps = m.sinb + kTT * m.cpitch;               // [Hq + 1][kTT + 4], the last row zero
  m.st = m.ps + (Hq + 1) * (kTT + 4);           // [Hq][4]
  m.posb = m.st + 4 * Hq;                       // int [2][kTT]
  m.invs = m.posb + 2 * kTT;                    // [D/2]
  m.total = m.invs + D / 2;
  return m;
}

template <typename T, int D, bool SPLIT>
__global__ void __launch_bounds__(kMidThreads) decode_mid_kernel(DecArgs a, int tpc, int chunk0) {
  constexpr int half = D / 2, NT = D / 8, HT = D / 16;
  constexpr int ldps = kTT + 4;
  extern __shared__ __align__(16) float msm3[];
  const int p = blockIdx.y;
  const int H = a.H, G = a.G, Hq = a.H * a.G, ld = a.ld, n = a.H * D;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int r_k = a.rk[p], r_v = a.rv[p];
  const MidSmem L = mid_smem(n, Hq, D, ld);
  const int ldc = L.ldc, ldv = L.ldv, cp = L.cpitch;
  float* us = msm3 + L.us;
  float* qs = msm3 + L.qs;
  float* cbuf = msm3 + L.cbuf;
  float* cosb = msm3 + L.cosb;
  float* sinb = msm3 + L.sinb;
  float* ps = msm3 + L.ps;
  float* st = msm3 + L.st;
  int* posb = reinterpret_cast<int*>(msm3 + L.posb);
  float* invs = msm3 + L.invs;
  const int nm = (a.W + kTT - 1) / kTT;
  const int t_begin = blockIdx.x * tpc, t_end = min(nm, t_begin + tpc);
  const int l4 = ld / 4;
  auto prefetch = [&](int tile, int slot) {
    const int j0 = tile * kTT, ntok = min(kTT, a.W - j0);
    float* kb = cbuf + slot * L.cbsz;
    float* vb = kb + kTT * ldc;
    const float* Ck = a.ck + p * a.c_sp + (long)j0 * ld;
    const float* Cv = a.cv + p * a.c_sp + (long)j0 * ld;
    for (int e = tid; e < ntok * l4; e += kMidThreads) {
      const int tt = e / l4, c = 4 * (e % l4);
      cp_async16_dec(kb + tt * ldc + c, Ck + (long)tt * ld + c);
      cp_async16_dec(vb + tt * ldv + c, Cv + (long)tt * ld + c);
    }
    if (tid < ntok) {
      int* pb = posb + slot * kTT;
      if (a.mid_pos) cp_async4_dec(pb + tid, a.mid_pos + p * a.mid_sp + j0 + tid);
      else pb[tid] = a.pos_base + j0 + tid;
    }
  };
  // prologue: every group's basis rows, the queries, the first tile
  {
    const float* U = a.uk + p * a.u_sp;
    for (int e = tid; e < n * l4; e += kMidThreads) {
      const int row = e / l4, c = 4 * (e % l4);
      cp_async16_dec(us + row * ldc + c, U + (long)row * ld + c);
    }
  }
  prefetch(t_begin, 0);
  const T* qp = reinterpret_cast<const T*>(a.q) + (long)p * a.Hq * D;
  for (int e = tid; e < Hq * D; e += kMidThreads) qs[e] = load_f<T>(qp + e);
  for (int f = tid; f < half; f += kMidThreads) invs[f] = a.inv_freq[f];
  for (int h = tid; h < Hq; h += kMidThreads) st[4 * h + 2] = -INFINITY;
  for (int e = tid; e < ldps; e += kMidThreads) ps[Hq * ldps + e] = 0.f;
  cp_async_commit_wait0();
  __syncthreads();
  for (int e = tid; e < n * ld; e += kMidThreads) {  // columns past the rank are not basis
    const int row = e / ld, c = e % ld;
    const float x = us[row * ldc + c];
    us[row * ldc + c] = c < r_k ? (SPLIT ? x : __uint_as_float(tf32_bits(x))) : 0.f;
  }
  const int nct = ld / 8, nmt = (Hq + 15) / 16, npairs = nmt * nct;
  float cacc[kMaxPW][4];
#pragma unroll
  for (int i = 0; i < kMaxPW; ++i)
#pragma unroll
    for (int q = 0; q < 4; ++q) cacc[i][q] = 0.f;
  float lsum[kMaxRW];
#pragma unroll
  for (int i = 0; i < kMaxRW; ++i) lsum[i] = 0.f;
  for (int tile = t_begin; tile < t_end; ++tile) {
    const int slot = (tile - t_begin) & 1;
    __syncthreads();  // the other slot's previous tile is done; U zeroing visible
    if (tile + 1 < t_end) prefetch(tile + 1, slot ^ 1);
    cp_async_commit();
    const int j0 = tile * kTT, ntok = min(kTT, a.W - j0);
    const float* kb = cbuf + slot * L.cbsz;
    const float* vb = kb + kTT * ldc;
    const int* pb = posb + slot * kTT;
    for (int e = tid; e < kTT * half; e += kMidThreads) {  // the tile's rotary angles
      const int tt = e / half, f = e % half;
      float c = 1.f, sn = 0.f;
      if (tt < ntok) rope_cs_fast(pb[tt], invs[f], a.rope_scale, &c, &sn);
      cosb[tt * cp + f] = c;
      sinb[tt * cp + f] = sn;
    }
    {  // mask (and round) the staged coordinates in place
      float* kw = cbuf + slot * L.cbsz;
      float* vw = kw + kTT * ldc;
      for (int e = tid; e < kTT * ld; e += kMidThreads) {
        const int tt = e / ld, c = e % ld;
        const float xk = kw[tt * ldc + c], xv = vw[tt * ldv + c];
        kw[tt * ldc + c] = (tt < ntok && c < r_k) ? (SPLIT ? xk : __uint_as_float(tf32_bits(xk))) : 0.f;
        vw[tt * ldv + c] = (tt < ntok && c < r_v) ? (SPLIT ? xv : __uint_as_float(tf32_bits(xv))) : 0.f;
      }
    }
    __syncthreads();
    // task = (group, RB consecutive 16-token row blocks); each basis fragment
    // loaded from shared memory feeds RB products
    constexpr int RB = (!SPLIT && D == 64) ? 2 : 1;
    constexpr int kBlocks = 4 / RB;
    for (int task = warp; task < kBlocks * H; task += kMidWarps) {
      const int g = task / kBlocks, rb0 = (task % kBlocks) * RB;
      float kacc[RB][NT][4];
#pragma unroll
      for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int q = 0; q < 4; ++q) kacc[r][j][q] = 0.f;
      const int nkk = (r_k + 7) / 8;
      for (int kk = 0; kk < nkk; ++kk) {
        const int c0 = kk * 8 + tq;
        float af[RB][4];
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          const int t0 = (rb0 + r) * 16 + gq;
          af[r][0] = kb[t0 * ldc + c0];
          af[r][1] = kb[(t0 + 8) * ldc + c0];
          af[r][2] = kb[t0 * ldc + c0 + 4];
          af[r][3] = kb[(t0 + 8) * ldc + c0 + 4];
        }
        if constexpr (SPLIT) {
          uint32_t ah[4], al[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) tf32_split(af[0][q], &ah[q], &al[q]);
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const float* ur = us + (g * D + j * 8 + gq) * ldc + c0;
            uint32_t bh0, bl0, bh1, bl1;
            tf32_split(ur[0], &bh0, &bl0);
            tf32_split(ur[4], &bh1, &bl1);
            mma_tf32(kacc[0][j], al, bh0, bh1);
            mma_tf32(kacc[0][j], ah, bl0, bl1);
            mma_tf32(kacc[0][j], ah, bh0, bh1);
          }
        } else {
          uint32_t ah[RB][4];
#pragma unroll
          for (int r = 0; r < RB; ++r)
#pragma unroll
            for (int q = 0; q < 4; ++q) ah[r][q] = __float_as_uint(af[r][q]);
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const float* ur = us + (g * D + j * 8 + gq) * ldc + c0;
            const uint32_t b0 = __float_as_uint(ur[0]), b1 = __float_as_uint(ur[4]);
#pragma unroll
            for (int r = 0; r < RB; ++r) mma_tf32(kacc[r][j], ah[r], b0, b1);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const int tt0 = (rb0 + r) * 16 + gq, tt1 = tt0 + 8;
#pragma unroll
        for (int j = 0; j < HT; ++j) {
          const int f = 8 * j + 2 * tq;
          const float2 ca = *reinterpret_cast<const float2*>(cosb + tt0 * cp + f);
          const float2 sa = *reinterpret_cast<const float2*>(sinb + tt0 * cp + f);
          const float2 cb = *reinterpret_cast<const float2*>(cosb + tt1 * cp + f);
          const float2 sb = *reinterpret_cast<const float2*>(sinb + tt1 * cp + f);
          const float c0s[2] = {ca.x, ca.y}, s0s[2] = {sa.x, sa.y}, c1s[2] = {cb.x, cb.y}, s1s[2] = {sb.x, sb.y};
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float y1, y2;
            rope_apply_pair(kacc[r][j][e], kacc[r][j + HT][e], c0s[e], s0s[e], &y1, &y2);
            kacc[r][j][e] = y1; kacc[r][j + HT][e] = y2;
            rope_apply_pair(kacc[r][j][2 + e], kacc[r][j + HT][2 + e], c1s[e], s1s[e], &y1, &y2);
            kacc[r][j][2 + e] = y1; kacc[r][j + HT][2 + e] = y2;
          }
        }
        float sacc[4] = {0.f, 0.f, 0.f, 0.f};
        const float* qr = qs + (g * G + gq) * D + 2 * tq;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const float kf[4] = {kacc[r][j][0], kacc[r][j][2], kacc[r][j][1], kacc[r][j][3]};
          mma_f32<SPLIT>(sacc, kf, gq < G ? qr[8 * j] : 0.f, gq < G ? qr[8 * j + 1] : 0.f);
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int h = 2 * tq + e;
          if (h < G) {
            float* pr = ps + (g * G + h) * ldps;
            pr[tt0] = tt0 < ntok ? sacc[e] * a.scaling : -INFINITY;
            pr[tt1] = tt1 < ntok ? sacc[2 + e] * a.scaling : -INFINITY;
          }
        }
      }
    }
    __syncthreads();
    // softmax per query head over the tile, online across tiles
#pragma unroll
    for (int i = 0; i < kMaxRW; ++i) {
      const int row = warp + kMidWarps * i;
      if (row >= Hq) break;
      float* pr = ps + row * ldps;
      const float x0 = pr[lane], x1 = pr[lane + 32];
      float mt = fmaxf(x0, x1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
      const float mold = st[4 * row + 2];
      const float mnew = fmaxf(mold, mt);
      const float e0 = mnew == -INFINITY ? 0.f : expf(x0 - mnew);
      const float e1 = mnew == -INFINITY ? 0.f : expf(x1 - mnew);
      pr[lane] = SPLIT ? e0 : __uint_as_float(tf32_bits(e0));  // the value product's A operand
      pr[lane + 32] = SPLIT ? e1 : __uint_as_float(tf32_bits(e1));
      float ls = e0 + e1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
      const float corr = (mold == -INFINITY) ? 0.f : expf(mold - mnew);
      lsum[i] = lsum[i] * corr + ls;
      __syncwarp();
      if (lane == 0) {
        st[4 * row + 2] = mnew;
        st[4 * row + 3] = corr;
      }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxPW; ++i) {
      const int pair = warp + kMidWarps * i;
      if (pair >= npairs) break;
      const int mt = pair / nct, ct = pair % nct;
      const int ra = mt * 16 + gq, rb = ra + 8;
      const float ca = ra < Hq ? st[4 * ra + 3] : 0.f, cb = rb < Hq ? st[4 * rb + 3] : 0.f;
      cacc[i][0] *= ca; cacc[i][1] *= ca; cacc[i][2] *= cb; cacc[i][3] *= cb;
      // rows past Hq read the padding rows of ps (zero), columns are in range
      const float* pa = ps + (ra < Hq ? ra : Hq) * ldps;
      const float* pb2 = ps + (rb < Hq ? rb : Hq) * ldps;
      const float* vc = vb + ct * 8 + gq;
#pragma unroll 4
      for (int kk = 0; kk < kTT / 8; ++kk) {
        const int t0 = kk * 8 + tq;
        const float af[4] = {pa[t0], pb2[t0], pa[t0 + 4], pb2[t0 + 4]};
        if constexpr (SPLIT) {
          mma_f32<true>(cacc[i], af, vc[t0 * ldv], vc[(t0 + 4) * ldv]);
        } else {
          const uint32_t ah[4] = {__float_as_uint(af[0]), __float_as_uint(af[1]),
                                  __float_as_uint(af[2]), __float_as_uint(af[3])};
          mma_tf32(cacc[i], ah, __float_as_uint(vc[t0 * ldv]), __float_as_uint(vc[(t0 + 4) * ldv]));
        }
      }
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  }
  __syncthreads();
  // one partial record per group: m[G], l[G], acc_d[G][D] = 0, acc_c[G][ld]
  const int chunk = chunk0 + blockIdx.x;
  auto rec = [&](int g) { return a.part + ((long)(p * H + g) * a.n_chunks + chunk) * a.part_sp_chunk; };
#pragma unroll
  for (int i = 0; i < kMaxRW; ++i) {
    const int row = warp + kMidWarps * i;
    if (row >= Hq) break;
    if (lane == 0) {
      float* o = rec(row / G);
      o[row % G] = t_begin < t_end ? st[4 * row + 2] : -INFINITY;
      o[G + row % G] = lsum[i];
    }
  }
  for (int e = tid; e < H * G * D; e += kMidThreads) rec(e / (G * D))[2 * G + e % (G * D)] = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPW; ++i) {
    const int pair = warp + kMidWarps * i;
    if (pair >= npairs) break;
    const int mt = pair / nct, ct = pair % nct;
    const int cc = ct * 8 + 2 * tq;
#pragma unroll
    for (int half_ = 0; half_ < 2; ++half_) {
      const int row = mt * 16 + gq + 8 * half_;
      if (row < Hq) {
        float* o = rec(row / G) + 2 * G + G * D + (row % G) * ld + cc;
        o[0] = cacc[i][2 * half_];
        o[1] = cacc[i][2 * half_ + 1];
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(512) decode_merge_kernel(DecArgs a) {
  extern __shared__ __align__(16) float msm2[];
  const int g = blockIdx.x, p = blockIdx.y;
  const int D = a.D, G = a.G, ld = a.ld;
  const long rec = part_floats(G, D, ld);
  const float* parts = a.part + (long)(p * a.H + g) * a.n_chunks * a.part_sp_chunk;
  float* accc = msm2;        // [G][ld]
  float* accd = accc + G * ld;  // [G][D]
  float* ml = accd + G * D;     // [G][2]: M, Lsum
  float* sc = ml + 2 * G;       // [n_chunks][G]: exp(m_c - M) per chunk and head
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, nw = blockDim.x / 32;
  const int nch = a.n_chunks;
  const long sp = a.part_sp_chunk;
  for (int qh = warp; qh < G; qh += nw) {  // a warp per head, lanes over the chunks
    float M = -INFINITY;
    for (int c = lane; c < nch; c += 32) M = fmaxf(M, parts[c * sp + qh]);
    M = warp_max(M);
    float Ls = 0.f;
    for (int c = lane; c < nch; c += 32) {
      const float mc = parts[c * sp + qh];
      const float f = mc == -INFINITY ? 0.f : expf(mc - M);
      sc[c * G + qh] = f;
      Ls = fmaf(f, parts[c * sp + G + qh], Ls);
    }
    Ls = warp_sum(Ls);
    if (lane == 0) {
      ml[2 * qh] = M;
      ml[2 * qh + 1] = Ls;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * (D + ld); e += blockDim.x) {
    int qh; long off;
    if (e < G * D) { qh = e / D; off = 2 * G + e; }
    else { qh = (e - G * D) / ld; off = 2 * G + G * D + (e - G * D); }
    float v0 = 0.f, v1 = 0.f, v2 = 0.f, v3 = 0.f;  // four chains, their loads in flight together
    int c = 0;
    for (; c + 4 <= nch; c += 4) {
      const float x0 = parts[c * sp + off], x1 = parts[(c + 1) * sp + off];
      const float x2 = parts[(c + 2) * sp + off], x3 = parts[(c + 3) * sp + off];
      v0 = fmaf(sc[c * G + qh], x0, v0);
      v1 = fmaf(sc[(c + 1) * G + qh], x1, v1);
      v2 = fmaf(sc[(c + 2) * G + qh], x2, v2);
      v3 = fmaf(sc[(c + 3) * G + qh], x3, v3);
    }
    for (; c < nch; ++c) v0 = fmaf(sc[c * G + qh], parts[c * sp + off], v0);
    const float v = (v0 + v1) + (v2 + v3);
    if (e < G * D) accd[e] = v;
    else accc[e - G * D] = v;
  }
  __syncthreads();
  const float* Uv = a.uv + p * a.u_sp;
  const int r_v = a.rv[p];
  T* out = reinterpret_cast<T*>(a.out) + (long)p * a.Hq * D;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int qh = e / D, d = e % D;
    float v = accd[e];
    const float* ur = Uv + (long)(g * D + d) * ld;
#pragma unroll 8
    for (int c = 0; c < r_v; ++c) v = fmaf(ur[c], accc[qh * ld + c], v);
    store_f<T>(out + (long)(g * G + qh) * D + d, v / ml[2 * qh + 1]);
  }
}

}  // namespace kvd

namespace kvd_host {
using namespace kvd;

static int dec_chunks(int L) { return (L + kChunk - 1) / kChunk; }

size_t decode_ws_bytes(const kvd_config& c, int count, int num_q_heads, int n_heads) {
  const int G = num_q_heads / n_heads;
  const int L_max = c.n_sink + c.hh_budget + c.w_cap + c.ring_cap;
  const long rec = part_floats(G, c.head_dim, c.rank);
  // tiled paths: one chunk per verbatim tile plus middle chunks of >= 2 tiles
  const int nvt = (c.n_sink + c.hh_budget + kTT - 1) / kTT + (c.ring_cap + kTT - 1) / kTT;
  const int ch_tiled = nvt + ((c.w_cap + kTT - 1) / kTT + 1) / 2;
  const int ch = dec_chunks(L_max) > ch_tiled ? dec_chunks(L_max) : ch_tiled;
  return (size_t)count * n_heads * ch * rec * 4 + 256;
}

// ------------------------------------------------------------------
// The middle tier on the 5th-generation tensor cores (bf16 caches,
// head_dim 64, n <= 512, rank <= 32).  A CTA of eight warps walks `tpc`
// tiles of 128 middle tokens of one problem for every KV group: the key
// rebuild C_k U_k^T of a tile (128 tokens x all n features) is 2 x ceil(r/8)
// kind::tf32 MMAs of 128 x 256 x 8 into tensor memory (512 columns), issued
// by one thread from the tile's coordinates and the basis rows staged once
// per CTA (both K-major, no-swizzle core-matrix layout, TF32-rounded, columns
// past the rank zero).  Warp w then reads accumulator lanes (tokens)
// [32 (w % 4), +32) for half of the groups: one token per thread, the
// rotate-half partners d and d + 32 in the same thread, RoPE at the token's
// position, the scores against the group's query heads into shared memory;
// the softmax runs per query head online across tiles, and the value product
// P C_v accumulates in coordinate space in registers (U_v is applied once in
// the merge).  Partial records as decode_mid_kernel writes them.
constexpr int kDuTok = 128;
constexpr int kDuThreads = 512;
constexpr int kDuK = 32;  // staged rank columns (rank <= 32)
// score-row pitch = 4 mod 32 and value-coordinate pitch = 8 mod 32: the
// value product's TF32 fragment loads (rows g, columns t of the
// probabilities; rows t, columns g of the coordinates) hit distinct banks
constexpr int kDuPs = kDuTok + 4;
constexpr long kDuWaitPolls = 1L << 22;

struct DuSmem { int us, ck, cv, ldv, qs, cs, ps, st, posb, invf, bar, total; };  // bytes
// n = this CTA's features (its KV groups x D), Hq = its query heads
__host__ __device__ inline DuSmem du_smem(int n, int Hq, int D) {
  DuSmem m;
  m.ldv = kDuK + 8;
  m.us = 0;                                   // [n][32] basis, core-matrix layout
  m.ck = m.us + n * kDuK * 4;                 // 2 x [128][32] key coordinates, core-matrix layout
  m.cv = m.ck + 2 * kDuTok * kDuK * 4;        // 2 x [128][ldv] value coordinates
  m.qs = m.cv + 2 * kDuTok * m.ldv * 4;       // [Hq][D] queries
  m.cs = m.qs + Hq * D * 4;                   // [128 tokens][D/2 + 4] cos, then the same for sin
  m.ps = m.cs + 2 * kDuTok * (D / 2 + 4) * 4; // [Hq][kDuPs] scores, then probabilities
  m.st = m.ps + Hq * kDuPs * 4;               // [Hq][4]: running max, correction
  m.posb = m.st + Hq * 16;                    // 2 x [128] positions
  m.invf = m.posb + 2 * kDuTok * 4;           // [D/2] inverse frequencies
  m.bar = m.invf + (D / 2) * 4;               // mbarrier, TMEM base
  m.total = m.bar + 16;
  return m;
}

__device__ __forceinline__ int du_off(int row, int k) {  // core-matrix byte offset, K = 32
  return (row >> 3) * (kDuK * 32) + (k >> 2) * 128 + (row & 7) * 16 + (k & 3) * 4;
}

// 16-byte cp.async, zero-filled (nothing read) when `valid` is false
__device__ __forceinline__ void cp16_zfill(void* dst, const void* src, bool valid) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}

// KV groups one CTA covers: as many as fill the 512 TMEM columns (all of
// them at head_dim 64 with n <= 512; four of eight at head_dim 128)
__host__ __device__ inline int du_groups(int H, int D) { return H * D <= 512 ? H : 512 / D; }

template <int D>
__global__ void __launch_bounds__(kDuThreads) decode_mid_umma_kernel(DecArgs a, int tpc, int chunk0,
                                                                     int* status) {
  constexpr int HALF = D / 2;
  extern __shared__ __align__(1024) unsigned char dsm4[];
  const int hb = du_groups(a.H, D), nsg = a.H / hb;
  // group ranges fastest: the CTAs that read one coordinate tile run together
  // and share it through L2
  const int cx = blockIdx.x / nsg;                         // tile range
  const int p = blockIdx.y, g0 = (blockIdx.x % nsg) * hb;  // this CTA's groups [g0, g0 + hb)
  const int H = hb, G = a.G, Hq = hb * a.G, ld = a.ld, n = hb * D;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r_k = a.rk[p];
  const DuSmem L = du_smem(n, Hq, D);
  unsigned char* us = dsm4 + L.us;
  float* qs = reinterpret_cast<float*>(dsm4 + L.qs);
  // rotary tables, a row of HALF + 4 floats per token (16-byte rows, the
  // 16-byte loads of eight consecutive tokens on distinct banks)
  constexpr int CSP = HALF + 4;
  float* cos_t = reinterpret_cast<float*>(dsm4 + L.cs);
  float* sin_t = cos_t + kDuTok * CSP;
  float* ps = reinterpret_cast<float*>(dsm4 + L.ps);
  float* st = reinterpret_cast<float*>(dsm4 + L.st);
  int* posb = reinterpret_cast<int*>(dsm4 + L.posb);
  float* invf = reinterpret_cast<float*>(dsm4 + L.invf);
  uint64_t* bar = reinterpret_cast<uint64_t*>(dsm4 + L.bar);
  uint32_t* tbase = reinterpret_cast<uint32_t*>(dsm4 + L.bar + 8);
  const int ldv = L.ldv;
  const int nm = (a.W + kDuTok - 1) / kDuTok;
  const int t_begin = cx * tpc, t_end = min(nm, t_begin + tpc);
  if (warp == 0) {
    umma::tmem_alloc(tbase, 512);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    umma::mbar_init(bar, 1);
    umma::mbar_fence_init();
  }
  {  // the basis rows of every group (K-major core matrices, TF32, columns past the rank zero)
    const float* U = a.uk + p * a.u_sp + (long)g0 * D * ld;
    for (int e = tid; e < n * (kDuK / 4); e += kDuThreads) {
      const int row = e / (kDuK / 4), k = 4 * (e % (kDuK / 4));
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k < r_k) {
        v = *reinterpret_cast<const float4*>(U + (long)row * ld + k);
        if (k + 1 >= r_k) v.y = 0.f;
        if (k + 2 >= r_k) v.z = 0.f;
        if (k + 3 >= r_k) v.w = 0.f;
      }
      *reinterpret_cast<float4*>(us + du_off(row, k)) =
          make_float4(umma::to_tf32(v.x), umma::to_tf32(v.y), umma::to_tf32(v.z), umma::to_tf32(v.w));
    }
  }
  const __nv_bfloat16* qp = reinterpret_cast<const __nv_bfloat16*>(a.q) + ((long)p * a.Hq + g0 * G) * D;
  for (int e = tid; e < Hq * D; e += kDuThreads) qs[e] = __bfloat162float(qp[e]);
  for (int h = tid; h < Hq; h += kDuThreads) st[4 * h] = -INFINITY;
  if (tid < HALF) invf[tid] = a.inv_freq[tid];
  // a tile's coordinates land by cp.async straight into the MMA's layout (keys;
  // rank columns past the basis rank meet zero basis columns) and into a plain
  // pitch (values); rows past the middle are zero-filled without a read
  auto prefetch = [&](int tile, int buf) {
    const int j0 = tile * kDuTok, ntok = min(kDuTok, a.W - j0);
    const float* Ck = a.ck + p * a.c_sp + (long)j0 * ld;
    const float* Cv = a.cv + p * a.c_sp + (long)j0 * ld;
    unsigned char* ckb = dsm4 + L.ck + buf * kDuTok * kDuK * 4;
    float* cvb = reinterpret_cast<float*>(dsm4 + L.cv) + buf * kDuTok * ldv;
    for (int e = tid; e < kDuTok * (kDuK / 4); e += kDuThreads) {
      const int row = e / (kDuK / 4), k = 4 * (e % (kDuK / 4));
      const bool ok = row < ntok && k < ld;
      const long off = ok ? (long)row * ld + k : 0;
      cp16_zfill(ckb + du_off(row, k), Ck + off, ok);
      cp16_zfill(cvb + row * ldv + k, Cv + off, ok);
    }
    if (tid < kDuTok) {  // positions copied asynchronously too: the issuing warps do not wait on them
      int* pd = posb + buf * kDuTok + tid;
      if (tid < ntok && a.mid_pos) cp_async4_dec(pd, a.mid_pos + p * a.mid_sp + j0 + tid);
      else *pd = tid < ntok ? a.pos_base + j0 + tid : 0;
    }
    cp_async_commit();
  };
  if (t_begin < t_end) prefetch(t_begin, 0);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tbase;
  const uint32_t us_addr = (uint32_t)__cvta_generic_to_shared(us);
  const uint32_t idesc = umma::idesc_tf32(kDuTok, 256);
  // value product acc_c (Hq x ld) += P (Hq x tokens) C_v (tokens x ld) on
  // warp-level TF32 MMAs (m16n8k8): a task is a 16-head m-tile, an 8-column
  // n-tile and a 64-token half of the tile; warp w takes tasks w and w + 16
  const int n_nt = (ld + 7) / 8, n_task = 2 * ((Hq + 15) / 16) * n_nt;
  const int fg = lane >> 2, ft = lane & 3;
  float vfr[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  float lrow[4] = {0.f, 0.f, 0.f, 0.f};  // sums of the rows warp + 16 i
  uint32_t phase = 0;
  bool ok_wait = true;
  const int tok = 32 * (warp & 3) + lane;  // this thread's TMEM lane (token of the tile)
  const int gq = warp >> 2;                // which quarter of the groups this warp scores
  const int gper = (H + 3) / 4;
  const float4* qs4 = reinterpret_cast<const float4*>(qs);
  for (int tile = t_begin; tile < t_end && ok_wait; ++tile) {
    const int buf = (tile - t_begin) & 1;
    const int j0 = tile * kDuTok, ntok = min(kDuTok, a.W - j0);
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    umma::fence_proxy_async_smem();
    __syncthreads();  // the tile is in shared memory for every thread and the tensor core
    if (tid == 0) {
      umma::fence_after_sync();
      const uint32_t ck_addr = (uint32_t)__cvta_generic_to_shared(dsm4 + L.ck + buf * kDuTok * kDuK * 4);
      for (int nb = 0; nb < n; nb += 256)
        for (int j = 0; j < kDuK / 8; ++j)
          umma::mma_tf32(tmem + nb, umma::smem_desc(ck_addr + 256 * j, 128, 32 * kDuK),
                         umma::smem_desc(us_addr + nb * kDuK * 4 + 256 * j, 128, 32 * kDuK), idesc,
                         j > 0);
      umma::commit(bar);
    }
    if (tile + 1 < t_end) prefetch(tile + 1, buf ^ 1);  // lands while this tile is processed
    {  // [frequency][token] rotary table: a thread per token and every fourth frequency
      const int t = tid & (kDuTok - 1);
      const bool live = t < ntok;
      const int pos = posb[buf * kDuTok + t];
      for (int f = tid / kDuTok; f < HALF; f += kDuThreads / kDuTok) {
        float c = 1.f, sn = 0.f;
        if (live) rope_cs_fast(pos, invf[f], a.rope_scale, &c, &sn);
        cos_t[t * CSP + f] = c;
        sin_t[t * CSP + f] = sn;
      }
    }
    __syncthreads();
    ok_wait = umma::mbar_wait_bounded(bar, phase, kDuWaitPolls);
    phase ^= 1;
    umma::fence_after_sync();
    if (ok_wait) {
      const uint32_t trow = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
      const int g_lo = gq * gper, g_hi = min(H, g_lo + gper);
      const float4* cos4 = reinterpret_cast<const float4*>(cos_t + tok * CSP);
      const float4* sin4 = reinterpret_cast<const float4*>(sin_t + tok * CSP);
      for (int g = g_lo; g < g_hi; ++g) {
        // packed fp32 pairs over consecutive frequencies (sm_100 FFMA2): per
        // head the score's two halves, each as an (even, odd) frequency pair
        float2 s1[kMaxG], s2[kMaxG];
#pragma unroll
        for (int qh = 0; qh < kMaxG; ++qh) { s1[qh] = make_float2(0.f, 0.f); s2[qh] = s1[qh]; }
#pragma unroll
        for (int f0 = 0; f0 < HALF; f0 += 16) {
          float x1[16], x2[16];
          umma::tmem_ld16(trow + g * D + f0, x1);
          umma::tmem_ld16(trow + g * D + HALF + f0, x2);
          umma::tmem_wait_ld();
          float2 y1[8], y2[8];
#pragma unroll
          for (int i4 = 0; i4 < 4; ++i4) {  // RoPE: y1 = x1 c - x2 s, y2 = x2 c + x1 s
            const float4 c4 = cos4[(f0 >> 2) + i4], s4 = sin4[(f0 >> 2) + i4];
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              const int i = 4 * i4 + 2 * h2;
              const float2 X1 = make_float2(x1[i], x1[i + 1]), X2 = make_float2(x2[i], x2[i + 1]);
              const float2 C = h2 ? make_float2(c4.z, c4.w) : make_float2(c4.x, c4.y);
              const float2 S = h2 ? make_float2(s4.z, s4.w) : make_float2(s4.x, s4.y);
              const float2 t1 = __fmul2_rn(X2, S), t2 = __fmul2_rn(X1, S);
              y1[2 * i4 + h2] = __ffma2_rn(X1, C, make_float2(-t1.x, -t1.y));
              y2[2 * i4 + h2] = __ffma2_rn(X2, C, t2);
            }
          }
#pragma unroll
          for (int qh = 0; qh < kMaxG; ++qh) {
            if (qh < G) {
              const float4* qa = qs4 + (g * G + qh) * (D / 4) + f0 / 4;
              const float4* qb = qa + HALF / 4;
              float2 u1 = s1[qh], u2 = s2[qh];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 u = qa[i], w = qb[i];
                u1 = __ffma2_rn(y1[2 * i], make_float2(u.x, u.y), u1);
                u2 = __ffma2_rn(y2[2 * i], make_float2(w.x, w.y), u2);
                u1 = __ffma2_rn(y1[2 * i + 1], make_float2(u.z, u.w), u1);
                u2 = __ffma2_rn(y2[2 * i + 1], make_float2(w.z, w.w), u2);
              }
              s1[qh] = u1;
              s2[qh] = u2;
            }
          }
        }
#pragma unroll
        for (int qh = 0; qh < kMaxG; ++qh)
          if (qh < G)
            ps[(g * G + qh) * kDuPs + tok] =
                tok < ntok ? ((s1[qh].x + s1[qh].y) + (s2[qh].x + s2[qh].y)) * a.scaling : -INFINITY;
      }
    }
    umma::fence_before_sync();
    __syncthreads();
    if (!ok_wait) break;
    // softmax per query head over the tile, online across tiles (warp owns rows warp + 16 i)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = warp + 16 * i;
      if (row >= Hq) continue;
      float* pr = ps + row * kDuPs;
      const float x0 = pr[lane], x1 = pr[lane + 32], x2 = pr[lane + 64], x3 = pr[lane + 96];
      float mt = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
      mt = warp_max(mt);
      const float mold = st[4 * row];
      const float mnew = fmaxf(mold, mt);
      const float e0 = mnew == -INFINITY ? 0.f : expf(x0 - mnew);
      const float e1 = mnew == -INFINITY ? 0.f : expf(x1 - mnew);
      const float e2 = mnew == -INFINITY ? 0.f : expf(x2 - mnew);
      const float e3 = mnew == -INFINITY ? 0.f : expf(x3 - mnew);
      pr[lane] = e0; pr[lane + 32] = e1; pr[lane + 64] = e2; pr[lane + 96] = e3;
      const float ls = warp_sum((e0 + e1) + (e2 + e3));
      const float corr = mold == -INFINITY ? 0.f : expf(mold - mnew);
      lrow[i] = lrow[i] * corr + ls;
      __syncwarp();
      if (lane == 0) {
        st[4 * row] = mnew;
        st[4 * row + 1] = corr;
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 2; ++k) {  // acc = corr * acc + P C_v over the task's token half
      const int task = warp + 16 * k;
      if (task < n_task) {
        const int kh = task & 1, ot = task >> 1, mt = ot / n_nt, nt = ot % n_nt;
        const int r0 = 16 * mt + fg, r1 = r0 + 8;
        // rows past Hq read row Hq - 1 (inside the buffer) and use zero
        const bool v0 = r0 < Hq, v1 = r1 < Hq;
        const int q0 = v0 ? r0 : Hq - 1, q1 = v1 ? r1 : Hq - 1;
        const float c0 = v0 ? st[4 * q0 + 1] : 0.f, c1 = v1 ? st[4 * q1 + 1] : 0.f;
        vfr[k][0] *= c0; vfr[k][1] *= c0; vfr[k][2] *= c1; vfr[k][3] *= c1;
        const float* p0 = ps + q0 * kDuPs + 64 * kh + ft;
        const float* p1 = ps + q1 * kDuPs + 64 * kh + ft;
        const float* cb = reinterpret_cast<const float*>(dsm4 + L.cv) + buf * kDuTok * ldv +
                          (64 * kh + ft) * ldv + 8 * nt + fg;
#pragma unroll 4
        for (int k0 = 0; k0 < 64; k0 += 8) {
          const float x0 = p0[k0], x1 = p1[k0], x2 = p0[k0 + 4], x3 = p1[k0 + 4];
          const uint32_t af[4] = {v0 ? tf32_bits(x0) : 0u, v1 ? tf32_bits(x1) : 0u,
                                  v0 ? tf32_bits(x2) : 0u, v1 ? tf32_bits(x3) : 0u};
          mma_tf32(vfr[k], af, tf32_bits(cb[k0 * ldv]), tf32_bits(cb[(k0 + 4) * ldv]));
        }
      }
    }
    __syncthreads();  // this tile's buffers free for the prefetch after next
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  if (!ok_wait) {
    if (tid == 0) atomicOr(&status[kStatusTimeout], 16);
    umma::mbar_wait_bounded(bar, phase ^ 1, kDuWaitPolls);
  }
  __syncthreads();  // every product has read the probabilities before their rows take the halves
  float* hsum = ps;  // [Hq][32] the second token half's products
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int task = warp + 16 * k;
    if (task < n_task && (task & 1)) {
      const int ot = task >> 1, r0 = 16 * (ot / n_nt) + fg, r1 = r0 + 8, cc = 8 * (ot % n_nt) + 2 * ft;
      if (r0 < Hq) { hsum[r0 * 32 + cc] = vfr[k][0]; hsum[r0 * 32 + cc + 1] = vfr[k][1]; }
      if (r1 < Hq) { hsum[r1 * 32 + cc] = vfr[k][2]; hsum[r1 * 32 + cc + 1] = vfr[k][3]; }
    }
  }
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, 512);
  // one partial record per group: m[G], l[G], acc_d[G][D] = 0, acc_c[G][ld]
  const int chunk = chunk0 + cx;
  auto rec = [&](int g) {  // g: this CTA's group index
    return a.part + ((long)(p * a.H + g0 + g) * a.n_chunks + chunk) * a.part_sp_chunk;
  };
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = warp + 16 * i;
    if (row < Hq && lane == 0) {
      float* o = rec(row / G);
      o[row % G] = (t_begin < t_end && ok_wait) ? st[4 * row] : -INFINITY;
      o[G + row % G] = ok_wait ? lrow[i] : 0.f;
    }
  }
  for (int e = tid; e < H * G * D; e += kDuThreads) rec(e / (G * D))[2 * G + e % (G * D)] = 0.f;
#pragma unroll
  for (int k = 0; k < 2; ++k) {  // acc_c[G][ld] of each group: the two token halves
    const int task = warp + 16 * k;
    if (task < n_task && !(task & 1)) {
      const int ot = task >> 1, r0 = 16 * (ot / n_nt) + fg, cc = 8 * (ot % n_nt) + 2 * ft;
      if (cc < ld) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = r0 + 8 * h;
          if (row < Hq) {
            float* o = rec(row / G) + 2 * G + G * D + (row % G) * ld + cc;
            o[0] = ok_wait ? vfr[k][2 * h] + hsum[row * 32 + cc] : 0.f;
            o[1] = ok_wait ? vfr[k][2 * h + 1] + hsum[row * 32 + cc + 1] : 0.f;
          }
        }
      }
    }
  }
}

// ------------------------------------------------------------------
// The middle tier on the 5th-generation tensor cores for ranks 33..192
// (bf16 caches, head_dim 64 or 128).  The basis of every KV group no longer
// fits shared memory beside a tile's coordinates, so a CTA takes 128 features
// (one group at head_dim 128, two at 64) and K = 64, 128 or 192 staged rank
// columns: the key rebuild of a 128-token tile is K/8 kind::tf32 MMAs of
// 128 x 128 x 8 into 128 TMEM columns.  Up to K = 128 one buffer each holds
// a tile's key and value coordinates: the next tile's keys land while this
// tile's scores are formed (issued once its MMA has read the keys), its
// values while the next tile's MMA and scores run.  At K = 192 one buffer
// holds both in turn: the values land while the scores are formed, the next
// tile's keys after the value product.  The CTA's (group, 16-frequency block)
// units are four at both head dims: quarter q of the warps (warps 4q..4q+3
// cover the 128 TMEM lanes, one token per thread) takes unit q, forms the
// rotary angles of its token in registers while the MMA runs, rotates its
// 16 frequency pairs and writes partial scores for the group's query heads;
// the partials of a head are summed in a fixed order.  Softmax, value product
// and partial records as in decode_mid_umma_kernel.
constexpr int kDwN = 128;     // features per CTA
constexpr int kDwMaxHq = 16;  // query heads per CTA

struct DwSmem { int us, ck, cv, ldv, qs, pp, st, posb, invf, bar, total; };  // bytes
__host__ __device__ constexpr bool dw_one_buffer(int K) { return K > 128; }
__host__ __device__ inline DwSmem dw_smem(int K, int Hq, int D) {
  DwSmem m;
  m.ldv = K + 4;
  m.us = 0;                                  // [128 features][K] basis, core-matrix layout
  m.ck = m.us + kDwN * K * 4;                // [128 tokens][K] key coordinates, core-matrix layout
  // [128 tokens][ldv] value coordinates (in the key buffer at K > 128)
  m.cv = dw_one_buffer(K) ? m.ck : m.ck + kDuTok * K * 4;
  m.qs = m.cv + kDuTok * m.ldv * 4;          // [Hq][D] queries
  m.pp = m.qs + Hq * D * 4;                  // [4 quarters][Hq][128] partial scores; quarter 0's
                                             // slots then hold the scores and probabilities; at
                                             // the end the value-product halves [256][4]
  const int pp_bytes = 4 * Hq * kDuTok * 4;
  m.st = m.pp + (pp_bytes > 256 * 16 ? pp_bytes : 256 * 16);  // [Hq][4]: running max, correction
  m.posb = m.st + Hq * 16;                   // 2 x [128] positions
  m.invf = m.posb + 2 * kDuTok * 4;          // [D/2] inverse frequencies
  m.bar = m.invf + (D / 2) * 4;              // mbarrier, TMEM base
  m.total = m.bar + 16;
  return m;
}

template <int K>
__device__ __forceinline__ int dw_off(int row, int k) {  // core-matrix byte offset, K columns
  return (row >> 3) * (K * 32) + (k >> 2) * 128 + (row & 7) * 16 + (k & 3) * 4;
}

template <int D, int K>
__global__ void __launch_bounds__(kDuThreads) decode_mid_wide_kernel(DecArgs a, int tpc, int chunk0,
                                                                     int* status) {
  constexpr int HALF = D / 2, HB = kDwN / D, FB = HALF / 16;
  constexpr bool kOne = dw_one_buffer(K);
  static_assert(HB * FB == 4, "one (group, frequency block) unit per quarter of the warps");
  extern __shared__ __align__(1024) unsigned char dsm5[];
  const int nsg = a.H / HB;
  // group ranges fastest: the CTAs that read one coordinate tile run together
  // and share it through L2
  const int cx = blockIdx.x / nsg;                         // tile range
  const int p = blockIdx.y, g0 = (blockIdx.x % nsg) * HB;  // this CTA's groups [g0, g0 + HB)
  const int G = a.G, Hq = HB * a.G, ld = a.ld;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r_k = a.rk[p];
  const DwSmem L = dw_smem(K, Hq, D);
  unsigned char* us = dsm5 + L.us;
  unsigned char* ckb = dsm5 + L.ck;
  float* cvb = reinterpret_cast<float*>(dsm5 + L.cv);
  float* qs = reinterpret_cast<float*>(dsm5 + L.qs);
  float* pp = reinterpret_cast<float*>(dsm5 + L.pp);
  float* ps = pp;  // the scores overwrite quarter 0's partials in place
  float* st = reinterpret_cast<float*>(dsm5 + L.st);
  int* posb = reinterpret_cast<int*>(dsm5 + L.posb);
  float* invf = reinterpret_cast<float*>(dsm5 + L.invf);
  uint64_t* bar = reinterpret_cast<uint64_t*>(dsm5 + L.bar);
  uint32_t* tbase = reinterpret_cast<uint32_t*>(dsm5 + L.bar + 8);
  const int ldv = L.ldv;
  const int nm = (a.W + kDuTok - 1) / kDuTok;
  const int t_begin = cx * tpc, t_end = min(nm, t_begin + tpc);
  if (warp == 0) {
    umma::tmem_alloc(tbase, kDwN);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    umma::mbar_init(bar, 1);
    umma::mbar_fence_init();
  }
  {  // the basis rows of the CTA's groups (K-major core matrices, TF32, columns past the rank zero)
    const float* U = a.uk + p * a.u_sp + (long)g0 * D * ld;
    for (int e = tid; e < kDwN * (K / 4); e += kDuThreads) {
      const int row = e / (K / 4), k = 4 * (e % (K / 4));
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k < r_k) {  // r_k <= ld and ld % 4 == 0: the vector stays inside the row
        v = *reinterpret_cast<const float4*>(U + (long)row * ld + k);
        if (k + 1 >= r_k) v.y = 0.f;
        if (k + 2 >= r_k) v.z = 0.f;
        if (k + 3 >= r_k) v.w = 0.f;
      }
      *reinterpret_cast<float4*>(us + dw_off<K>(row, k)) =
          make_float4(umma::to_tf32(v.x), umma::to_tf32(v.y), umma::to_tf32(v.z), umma::to_tf32(v.w));
    }
  }
  const __nv_bfloat16* qp = reinterpret_cast<const __nv_bfloat16*>(a.q) + ((long)p * a.Hq + g0 * G) * D;
  for (int e = tid; e < Hq * D; e += kDuThreads) qs[e] = __bfloat162float(qp[e]);
  for (int h = tid; h < Hq; h += kDuThreads) st[4 * h] = -INFINITY;
  if (tid < HALF) invf[tid] = a.inv_freq[tid];
  // key coordinates straight into the MMA's layout (columns past ld zero-filled
  // without a read, as are rows past the middle) and the tile's positions
  auto prefetch_k = [&](int tile, int pb) {
    const int j0 = tile * kDuTok, ntok = min(kDuTok, a.W - j0);
    const float* Ck = a.ck + p * a.c_sp + (long)j0 * ld;
    for (int e = tid; e < kDuTok * (K / 4); e += kDuThreads) {
      const int row = e / (K / 4), k = 4 * (e % (K / 4));
      const bool ok = row < ntok && k < ld;
      cp16_zfill(ckb + dw_off<K>(row, k), Ck + (ok ? (long)row * ld + k : 0), ok);
    }
    if (tid < kDuTok) {  // positions copied asynchronously too: the issuing warps do not wait on them
      int* pd = posb + pb * kDuTok + tid;
      if (tid < ntok && a.mid_pos) cp_async4_dec(pd, a.mid_pos + p * a.mid_sp + j0 + tid);
      else *pd = tid < ntok ? a.pos_base + j0 + tid : 0;
    }
    cp_async_commit();
  };
  auto prefetch_v = [&](int tile) {
    const int j0 = tile * kDuTok, ntok = min(kDuTok, a.W - j0);
    const float* Cv = a.cv + p * a.c_sp + (long)j0 * ld;
    const int l4 = ld / 4;
    for (int e = tid; e < kDuTok * l4; e += kDuThreads) {
      const int row = e / l4, k = 4 * (e % l4);
      const bool ok = row < ntok;
      cp16_zfill(cvb + row * ldv + k, Cv + (ok ? (long)row * ld + k : 0), ok);
    }
    cp_async_commit();
  };
  if (t_begin < t_end) {
    prefetch_k(t_begin, 0);
    if (!kOne) prefetch_v(t_begin);
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tbase;
  const uint32_t us_addr = (uint32_t)__cvta_generic_to_shared(us);
  const uint32_t ck_addr = (uint32_t)__cvta_generic_to_shared(ckb);
  constexpr uint32_t idesc = umma::idesc_tf32(kDuTok, kDwN);
  // value product: thread (vh, vc) of token half th accumulates acc_c[vh][vc..vc+4)
  const int nvq = ld / 4;
  const int th = tid >> 8, vt = tid & 255;
  const int vh = vt / nvq, vc = 4 * (vt % nvq);
  const bool vown = vh < Hq;
  float vacc[4] = {0.f, 0.f, 0.f, 0.f};
  float lrow = 0.f;  // running sum of row `warp` (rows < Hq <= 16)
  uint32_t phase = 0;
  bool ok_wait = true;
  const int tok = 32 * (warp & 3) + lane;  // this thread's TMEM lane (token of the tile)
  const int unit = warp >> 2;              // this quarter's (group, frequency block)
  const int ug = unit / FB, f0 = 16 * (unit % FB);
  const float4* qs4 = reinterpret_cast<const float4*>(qs);
  for (int tile = t_begin; tile < t_end; ++tile) {
    const int pb = (tile - t_begin) & 1;
    const int j0 = tile * kDuTok, ntok = min(kDuTok, a.W - j0);
    const bool more = tile + 1 < t_end;
    if (kOne) asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    else asm volatile("cp.async.wait_group 1;\n" ::: "memory");  // the keys (the values may still land)
    umma::fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      umma::fence_after_sync();
#pragma unroll
      for (int j = 0; j < K / 8; ++j)
        umma::mma_tf32(tmem, umma::smem_desc(ck_addr + 256 * j, 128, 32 * K),
                       umma::smem_desc(us_addr + 256 * j, 128, 32 * K), idesc, j > 0);
      umma::commit(bar);
    }
    // this thread's rotary angles while the MMA runs
    float cs[16], sn[16];
    {
      const int pos = posb[pb * kDuTok + tok];
#pragma unroll
      for (int i = 0; i < 16; ++i) rope_cs_fast(pos, invf[f0 + i], a.rope_scale, &cs[i], &sn[i]);
    }
    ok_wait = umma::mbar_wait_bounded(bar, phase, kDuWaitPolls);
    phase ^= 1;
    ok_wait = __syncthreads_and(ok_wait);
    umma::fence_after_sync();
    if (!ok_wait) break;
    if (kOne) prefetch_v(tile);                   // the MMA has read the keys: the values in their place
    else if (more) prefetch_k(tile + 1, pb ^ 1);
    {
      const uint32_t trow = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
      float x1[16], x2[16];
      umma::tmem_ld16(trow + ug * D + f0, x1);
      umma::tmem_ld16(trow + ug * D + HALF + f0, x2);
      umma::tmem_wait_ld();
      float2 y1[8], y2[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {  // RoPE on frequency pairs: y1 = x1 c - x2 s, y2 = x2 c + x1 s
        const float2 X1 = make_float2(x1[2 * i], x1[2 * i + 1]), X2 = make_float2(x2[2 * i], x2[2 * i + 1]);
        const float2 C = make_float2(cs[2 * i], cs[2 * i + 1]), S = make_float2(sn[2 * i], sn[2 * i + 1]);
        const float2 t1 = __fmul2_rn(X2, S), t2 = __fmul2_rn(X1, S);
        y1[i] = __ffma2_rn(X1, C, make_float2(-t1.x, -t1.y));
        y2[i] = __ffma2_rn(X2, C, t2);
      }
#pragma unroll
      for (int qh = 0; qh < kMaxG; ++qh) {
        if (qh < G) {
          const int h = ug * G + qh;
          const float4* qa = qs4 + h * (D / 4) + f0 / 4;
          const float4* qb = qa + HALF / 4;
          float2 u1 = make_float2(0.f, 0.f), u2 = u1;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 u = qa[i], w = qb[i];
            u1 = __ffma2_rn(y1[2 * i], make_float2(u.x, u.y), u1);
            u2 = __ffma2_rn(y2[2 * i], make_float2(w.x, w.y), u2);
            u1 = __ffma2_rn(y1[2 * i + 1], make_float2(u.z, u.w), u1);
            u2 = __ffma2_rn(y2[2 * i + 1], make_float2(w.z, w.w), u2);
          }
          pp[(unit * Hq + h) * kDuTok + tok] = (u1.x + u1.y) + (u2.x + u2.y);
        }
      }
    }
    umma::fence_before_sync();
    __syncthreads();
    // a head's score: its group's FB partials in block order, scaled
    for (int e = tid; e < Hq * kDuTok; e += kDuThreads) {
      const int h = e / kDuTok, t = e % kDuTok, u0 = (h / G) * FB;
      float sc = pp[(u0 * Hq + h) * kDuTok + t];
#pragma unroll
      for (int b = 1; b < FB; ++b) sc += pp[((u0 + b) * Hq + h) * kDuTok + t];
      ps[h * kDuTok + t] = t < ntok ? sc * a.scaling : -INFINITY;
    }
    __syncthreads();
    // softmax per query head over the tile, online across tiles (warp owns row `warp`)
    if (warp < Hq) {
      float* pr = ps + warp * kDuTok;
      const float x0 = pr[lane], x1 = pr[lane + 32], x2 = pr[lane + 64], x3 = pr[lane + 96];
      float mt = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
      mt = warp_max(mt);
      const float mold = st[4 * warp];
      const float mnew = fmaxf(mold, mt);
      const float e0 = mnew == -INFINITY ? 0.f : expf(x0 - mnew);
      const float e1 = mnew == -INFINITY ? 0.f : expf(x1 - mnew);
      const float e2 = mnew == -INFINITY ? 0.f : expf(x2 - mnew);
      const float e3 = mnew == -INFINITY ? 0.f : expf(x3 - mnew);
      pr[lane] = e0; pr[lane + 32] = e1; pr[lane + 64] = e2; pr[lane + 96] = e3;
      const float ls = warp_sum((e0 + e1) + (e2 + e3));
      const float corr = mold == -INFINITY ? 0.f : expf(mold - mnew);
      lrow = lrow * corr + ls;
      __syncwarp();
      if (lane == 0) {
        st[4 * warp] = mnew;
        st[4 * warp + 1] = corr;
      }
    }
    // the values of this tile (the next tile's keys may still land)
    if (more && !kOne) asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    else asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncthreads();
    if (vown) {  // acc_c[vh][vc..vc+4) = corr * acc + sum_t p[vh][t] c_v[t][vc..] over this half
      const float corr = st[4 * vh + 1];
#pragma unroll
      for (int j = 0; j < 4; ++j) vacc[j] *= corr;
      const float* pr = ps + vh * kDuTok + 64 * th;
      const float* cvh = cvb + 64 * th * ldv;
#pragma unroll 2
      for (int t = 0; t < 64; t += 4) {  // four tokens' probabilities in one 16-byte read
        const float4 p4 = *reinterpret_cast<const float4*>(pr + t);
        const float pt[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float4 cvv = *reinterpret_cast<const float4*>(cvh + (t + u) * ldv + vc);
          vacc[0] = fmaf(pt[u], cvv.x, vacc[0]);
          vacc[1] = fmaf(pt[u], cvv.y, vacc[1]);
          vacc[2] = fmaf(pt[u], cvv.z, vacc[2]);
          vacc[3] = fmaf(pt[u], cvv.w, vacc[3]);
        }
      }
    }
    __syncthreads();  // the value buffer is free
    if (more) {
      if (kOne) prefetch_k(tile + 1, pb ^ 1);
      else prefetch_v(tile + 1);
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  if (!ok_wait) {
    if (tid == 0) atomicOr(&status[kStatusTimeout], 16);
    umma::mbar_wait_bounded(bar, phase ^ 1, kDuWaitPolls);
  }
  __syncthreads();  // every product has read the probabilities before their slots take the halves
  float* vred = pp;
  if (th == 1 && vown)
#pragma unroll
    for (int j = 0; j < 4; ++j) vred[vt * 4 + j] = vacc[j];
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, kDwN);
  // one partial record per group: m[G], l[G], acc_d[G][D] = 0, acc_c[G][ld]
  const int chunk = chunk0 + cx;
  auto rec = [&](int g) {  // g: this CTA's group index
    return a.part + ((long)(p * a.H + g0 + g) * a.n_chunks + chunk) * a.part_sp_chunk;
  };
  if (warp < Hq && lane == 0) {
    float* o = rec(warp / G);
    o[warp % G] = (t_begin < t_end && ok_wait) ? st[4 * warp] : -INFINITY;
    o[G + warp % G] = ok_wait ? lrow : 0.f;
  }
  for (int e = tid; e < HB * G * D; e += kDuThreads) rec(e / (G * D))[2 * G + e % (G * D)] = 0.f;
  if (th == 0 && vown) {
    float* o = rec(vh / G) + 2 * G + G * D + (vh % G) * ld + vc;
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = ok_wait ? vacc[j] + vred[vt * 4 + j] : 0.f;
  }
}

template <typename T>
int launch_factored_decode(const kvd_config& c, const kvd_buffers& b, const kvd_counters& k, int p0,
                           int count, int h0, int hc, const void* q, int Hq, float scaling, void* out,
                           char* ws, size_t ws_bytes, cudaStream_t s, cudaStream_t side,
                           cudaEvent_t ev_fork, cudaEvent_t ev_join) {
  DecArgs a;
  const int n = c.num_heads * c.head_dim;
  if (h0 < 0 || hc < 1 || h0 + hc > c.num_heads || Hq % hc) {
    set_error("factored decode: bad KV head range [%d, %d) of %d for %d query heads", h0, h0 + hc,
              c.num_heads, Hq);
    return KVD_ERR_ARG;
  }
  // KV heads [h0, h0 + hc): the kernels see hc groups whose tier rows start
  // h0 * D features into each token row (stride nrow) and whose basis rows
  // start at row h0 * D; the query and output hold only their heads
  a.H = hc; a.D = c.head_dim; a.G = Hq / hc; a.ld = c.rank; a.Hq = Hq; a.nrow = n;
  const bool d_ok = (c.head_dim <= 32) || ((c.head_dim / 2) % 32 == 0);
  if (a.G > kMaxG || c.head_dim > 32 * kMaxNV || c.rank > 32 * kMaxNC || !d_ok) {
    set_error("factored decode: unsupported shape (G=%d D=%d r=%d)", a.G, c.head_dim, c.rank);
    return KVD_ERR_ARG;
  }
  a.sink_len = k.sink_len; a.hh_len = k.hh_len; a.W = k.w_len; a.ring_len = k.ring_len;
  a.L = a.sink_len + a.hh_len + a.W + a.ring_len;
  if (a.L <= 0) { set_error("factored decode on an empty cache"); return KVD_ERR_ARG; }
  const long sink_sp = (long)c.n_sink * n, hh_sp = (long)c.hh_budget * n, ring_sp = (long)c.ring_cap * n;
  const size_t es = sizeof(T);
  const long hoff = (long)h0 * c.head_dim;  // first feature of the range in a token row
  a.sink_k = (const char*)b.sink_k + es * (p0 * sink_sp + hoff); a.sink_v = (const char*)b.sink_v + es * (p0 * sink_sp + hoff); a.sink_sp = sink_sp;
  a.hh_k = (const char*)b.hh_k[k.hh_sel] + es * (p0 * hh_sp + hoff); a.hh_v = (const char*)b.hh_v[k.hh_sel] + es * (p0 * hh_sp + hoff); a.hh_sp = hh_sp;
  a.ring_k = (const char*)b.ring_k + es * (p0 * ring_sp + (long)k.ring_head * n + hoff);
  a.ring_v = (const char*)b.ring_v + es * (p0 * ring_sp + (long)k.ring_head * n + hoff);
  a.ring_sp = ring_sp;
  a.u_sp = (long)n * c.rank;
  a.uk = b.u_k[k.u_sel] + p0 * a.u_sp + hoff * c.rank; a.uv = b.u_v[k.u_sel] + p0 * a.u_sp + hoff * c.rank;
  a.rk = b.r_k + p0; a.rv = b.r_v + p0;
  a.c_sp = (long)c.w_cap * c.rank;
  a.ck = b.c_k + p0 * a.c_sp; a.cv = b.c_v + p0 * a.c_sp;
  const bool track = c.retention != KVD_RETENTION_FIFO;
  a.mid_pos = track ? b.mid_pos + (long)p0 * c.w_cap : nullptr; a.mid_sp = c.w_cap;
  a.pos_base = (int)(k.cumulative_length - k.ring_len - (k.hh_len + k.w_len));
  a.inv_freq = c.inv_freq; a.rope_scale = c.rope_scaling;
  a.q = q; a.out = out; a.scaling = scaling;
  a.status = b.status;
  a.part_sp_chunk = part_floats(a.G, a.D, a.ld);
  // tiled kernel: head_dim 64 or 128, rank <= head_dim, G <= 8
  const bool tiled = (a.D == 64 || a.D == 128) && a.ld <= a.D && a.G <= 8 &&
                     a.G * (a.D + a.ld) <= 12 * kTileThreads;
  const int mid0 = a.sink_len + a.hh_len;
  const int nv0 = (mid0 + kTT - 1) / kTT, nm = (a.W + kTT - 1) / kTT,
            nr = (a.ring_len + kTT - 1) / kTT;
  const int n_tiles = nv0 + nm + nr;
  a.n_chunks = tiled ? (n_tiles + kTilesPerCta - 1) / kTilesPerCta : dec_chunks(a.L);
  const size_t need = (size_t)count * a.H * a.n_chunks * a.part_sp_chunk * 4;
  if (need > ws_bytes) { set_error("factored decode: workspace too small"); return KVD_ERR_WORKSPACE; }
  a.part = (float*)ws;
  const bool mma = tiled && a.ld % 8 == 0 && a.ld <= 32 * kMaxCT &&
                   (reinterpret_cast<uintptr_t>(a.ck) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.cv) & 15) == 0 && a.c_sp % 4 == 0;
  // middle tier by decode_mid_kernel (every group per CTA) when the basis of
  // all groups fits in shared memory; verbatim tiles by decode_mma_kernel
  const int Hq_all = a.H * a.G;
  const MidSmem ms = mid_smem(a.H * a.D, Hq_all, a.D, a.ld);
  const bool mid_all = mma && a.W > 0 && Hq_all <= kMidWarps * kMaxRW && a.ld <= 64 &&
                       ((Hq_all + 15) / 16) * (a.ld / 8) <= kMidWarps * kMaxPW &&
                       4L * ms.total <= 200 * 1024 &&
                       (reinterpret_cast<uintptr_t>(a.uk) & 15) == 0 && a.u_sp % 4 == 0;
  // bf16, head_dim 64 or 128, rank <= 32: the middle tier on the
  // 5th-generation tensor cores (128-token tiles; a CTA takes as many KV
  // groups as fill TMEM, a multiple of 256 features), else decode_mid_kernel
  const int du_hb = du_groups(a.H, a.D), du_n = du_hb * a.D, du_hq = du_hb * a.G;
  const bool umma_mid = sizeof(T) == 2 && (a.D == 64 || a.D == 128) && mma && a.W > 0 &&
                        a.H % du_hb == 0 && du_n % 256 == 0 && a.ld <= kDuK &&
                        a.ld % 4 == 0 && du_hq <= 64 &&
                        a.c_sp % 4 == 0 && (reinterpret_cast<uintptr_t>(a.ck) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(a.cv) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(a.uk) & 15) == 0 &&
                        du_smem(du_n, du_hq, a.D).total <= device_smem_optin();
  // bf16, head_dim 64 or 128, rank 33..128: the middle tier on tcgen05 with
  // 128 features per CTA (decode_mid_wide_kernel)
  // (the verbatim tiles then go to decode_mma_kernel alone, at any rank)
  const int dw_K = a.ld <= 64 ? 64 : (a.ld <= 128 ? 128 : 192);
  const int dw_hb = (a.D == 64 || a.D == 128) ? kDwN / a.D : 1;
  const int dw_hq = dw_hb * a.G;
  const bool umma_wide = !umma_mid && sizeof(T) == 2 && (a.D == 64 || a.D == 128) && a.G <= 8 && a.W > 0 &&
                         a.ld > 32 && a.ld <= 192 && a.ld % 4 == 0 && a.H % dw_hb == 0 &&
                         dw_hq <= kDwMaxHq && dw_hq * (a.ld / 4) <= 256 && a.c_sp % 4 == 0 &&
                         (reinterpret_cast<uintptr_t>(a.ck) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(a.cv) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(a.uk) & 15) == 0 &&
                         dw_smem(dw_K, dw_hq, a.D).total <= device_smem_optin();
  if (mid_all || umma_mid || umma_wide) {
    const int nvt = nv0 + nr;
    const int n_vch = nvt;  // one verbatim tile per CTA
    // tiles per CTA: one CTA fills an SM, so the launch takes
    // ceil(chunks / SMs) waves of about (tpc + 1/2) tile times each (the
    // half: staging the bases); the tpc in [2, 8] with the fewest such times
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) {
      static int sm_count[64] = {0};
      if (dev >= 0 && dev < 64) {
        if (sm_count[dev] == 0) cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
        if (sm_count[dev] > 0) sms = sm_count[dev];
      }
    }
    const bool umma = umma_mid || umma_wide;
    const int ttok = umma ? kDuTok : kTT;
    const int nmt = (a.W + ttok - 1) / ttok;
    int tpc = umma ? 1 : 2;
    long best = -1;
    const int nsg = umma_mid ? a.H / du_hb : umma_wide ? a.H / dw_hb : 1;  // CTAs per tile (group ranges)
    for (int t = tpc; t <= 8; ++t) {
      const long waves = ((long)((nmt + t - 1) / t) * count * nsg + sms - 1) / sms;
      const long cost = waves * (2 * t + 1);
      if (best < 0 || cost < best) { best = cost; tpc = t; }
    }
    const int n_mch = (nmt + tpc - 1) / tpc;
    a.n_chunks = n_vch + n_mch;
    const size_t need2 = (size_t)count * a.H * a.n_chunks * a.part_sp_chunk * 4;
    if (need2 > ws_bytes) { set_error("factored decode: workspace too small"); return KVD_ERR_WORKSPACE; }
    constexpr bool kSplit = sizeof(T) == 4;
    auto mid_fn = a.D == 64 ? decode_mid_kernel<T, 64, kSplit> : decode_mid_kernel<T, 128, kSplit>;
    if (!umma)
      if (int rc0 = ensure_smem((const void*)mid_fn, 4 * ms.total, "decode_mid_kernel")) return rc0;
    // the verbatim tiles run beside the middle tier (disjoint partial records)
    const bool fork = side && ev_fork && ev_join && n_vch > 0;
    if (n_vch > 0) {
      // no middle tiles in this launch: keys and values of a tile, no coordinates or basis
      const int ldk = a.D + 4;
      const int tsmem = 4 * (a.G * a.D + 2 * kTT * ldk + a.G * (kTT + 4) + 4 * a.G);
      auto fn = a.D == 64 ? decode_mma_kernel<T, 64, kSplit> : decode_mma_kernel<T, 128, kSplit>;
      if (int rc0 = ensure_smem((const void*)fn, tsmem, "decode_mma_kernel")) return rc0;
      cudaStream_t vs = s;
      if (fork) {
        cudaEventRecord(ev_fork, s);
        cudaStreamWaitEvent(side, ev_fork, 0);
        vs = side;
      }
      {
        KTimerScope kts_("decode_mma_kernel", vs);
        fn<<<dim3(n_vch, a.H, count), kTileThreads, tsmem, vs>>>(a, nv0, 0, nvt, 1);
      }
      if (fork) cudaEventRecord(ev_join, side);
    }
    if (int rc1 = check_launch("decode_mma_kernel")) {
      if (fork) cudaStreamWaitEvent(s, ev_join, 0);
      return rc1;
    }
    if (umma_mid) {
      const int dsm = du_smem(du_n, du_hq, a.D).total;
      auto ufn = a.D == 64 ? decode_mid_umma_kernel<64> : decode_mid_umma_kernel<128>;
      if (int rc0 = ensure_smem((const void*)ufn, dsm, "decode_mid_kernel")) {
        if (fork) cudaStreamWaitEvent(s, ev_join, 0);
        return rc0;
      }
      KTimerScope kts_("decode_mid_kernel", s);
      ufn<<<dim3(n_mch * nsg, count), kDuThreads, dsm, s>>>(a, tpc, n_vch, a.status);
    } else if (umma_wide) {
      const int dsm = dw_smem(dw_K, dw_hq, a.D).total;
      auto wfn = a.D == 64
          ? (dw_K == 64 ? decode_mid_wide_kernel<64, 64>
                        : dw_K == 128 ? decode_mid_wide_kernel<64, 128> : decode_mid_wide_kernel<64, 192>)
          : (dw_K == 64 ? decode_mid_wide_kernel<128, 64>
                        : dw_K == 128 ? decode_mid_wide_kernel<128, 128> : decode_mid_wide_kernel<128, 192>);
      if (int rc0 = ensure_smem((const void*)wfn, dsm, "decode_mid_kernel")) {
        if (fork) cudaStreamWaitEvent(s, ev_join, 0);
        return rc0;
      }
      KTimerScope kts_("decode_mid_kernel", s);
      wfn<<<dim3(n_mch * nsg, count), kDuThreads, dsm, s>>>(a, tpc, n_vch, a.status);
    } else {
      KTimerScope kts_("decode_mid_kernel", s);
      mid_fn<<<dim3(n_mch, count), kMidThreads, 4 * ms.total, s>>>(a, tpc, n_vch);
    }
    if (fork) cudaStreamWaitEvent(s, ev_join, 0);  // the merge reads both kernels' records
    if (int rc1 = check_launch("decode_mid_kernel")) return rc1;
  } else if (mma) {
    const int ldk = a.D + 4, ldv = a.ld + 8, ldc = a.ld + 4;
    const int tsmem = 4 * (a.G * a.D + kTT * ldk + kTT * (ldk > ldv ? ldk : ldv) +
                           a.G * (kTT + 4) + a.D * ldc + 4 * a.G);
    dim3 tgrid(a.n_chunks, a.H, count);
    constexpr bool kSplit = sizeof(T) == 4;
    auto fn = a.D == 64 ? decode_mma_kernel<T, 64, kSplit> : decode_mma_kernel<T, 128, kSplit>;
    if (int rc0 = ensure_smem((const void*)fn, tsmem, "decode_mma_kernel")) return rc0;
    KTimerScope kts_("decode_mma_kernel", s);
    fn<<<tgrid, kTileThreads, tsmem, s>>>(a, nv0, nm, n_tiles, kTilesPerCta);
  } else if (tiled) {
    const int tsmem = 4 * (a.G * a.D + 2 * kTT * (a.D + 4) + a.G * kTT + a.ld * a.D +
                           a.ld * (kTT + 4) + 4 * a.G);
    dim3 tgrid(a.n_chunks, a.H, count);
#define KVD_TDEC(DD)                                                                                {                                                                                                 if (int rc0 = ensure_smem((const void*)decode_tile_kernel<T, DD>, tsmem,                                                  "decode_tile_kernel")) return rc0;                                    KTimerScope kts_("decode_tile_kernel", s);                                                      decode_tile_kernel<T, DD><<<tgrid, kTileThreads, tsmem, s>>>(a, nv0, nm, n_tiles);            }
    if (a.D == 64) KVD_TDEC(64)
    else KVD_TDEC(128)
#undef KVD_TDEC
  } else {
  const int smem = 4 * (a.G * a.D + a.ld * a.D + 4 * a.ld + 4 * (int)a.part_sp_chunk);
  dim3 grid(a.n_chunks, a.H, count);
  const int nv = (a.D + 31) / 32, nc = (a.ld + 31) / 32;
#define KVD_DEC(NV, NC)                                                                         \
  {                                                                                             \
    if (int rc0 = ensure_smem((const void*)decode_split_kernel<T, NV, NC>, smem,                \
                              "decode_split_kernel")) return rc0;                               \
    { KTimerScope kts_("decode_split_kernel", s); decode_split_kernel<T, NV, NC><<<grid, kDecThreads, smem, s>>>(a); }                          \
  }
  if (nv <= 2 && nc <= 1) KVD_DEC(2, 1)
  else if (nv <= 2 && nc <= 2) KVD_DEC(2, 2)
  else if (nv <= 2 && nc <= 4) KVD_DEC(2, 4)
  else if (nv <= 2) KVD_DEC(2, 6)
  else if (nc <= 1) KVD_DEC(4, 1)
  else if (nc <= 2) KVD_DEC(4, 2)
  else if (nc <= 4) KVD_DEC(4, 4)
  else KVD_DEC(4, 6)
#undef KVD_DEC
  }
  int rc = check_launch("decode_split_kernel");
  if (rc) return rc;
  const int msmem = 4 * (a.G * a.ld + a.G * a.D + 2 * a.G + a.n_chunks * a.G);
  if (int rc0 = ensure_smem((const void*)decode_merge_kernel<T>, msmem, "decode_merge_kernel")) return rc0;
  {
    // a thread per combined value (G (D + ld) of them) where that fits 512
    int mthr = ((a.G * (a.D + a.ld) + 31) / 32) * 32;
    mthr = mthr < 128 ? 128 : (mthr > 512 ? 512 : mthr);
    KTimerScope kts_("decode_merge_kernel", s);
    decode_merge_kernel<T><<<dim3(a.H, count), mthr, msmem, s>>>(a);
  }
  return check_launch("decode_merge_kernel");
}

template int launch_factored_decode<float>(const kvd_config&, const kvd_buffers&, const kvd_counters&, int, int, int, int,
                                           const void*, int, float, void*, char*, size_t, cudaStream_t,
                                           cudaStream_t, cudaEvent_t, cudaEvent_t);
template int launch_factored_decode<__nv_bfloat16>(const kvd_config&, const kvd_buffers&, const kvd_counters&, int,
                                                   int, int, int, const void*, int, float, void*, char*, size_t,
                                                   cudaStream_t, cudaStream_t, cudaEvent_t, cudaEvent_t);

}  // namespace kvd_host
