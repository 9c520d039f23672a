// Blocked BUG projection behind the prefill press (sm_100a).
//
// Restates, for one feature-by-token matrix held token-major (x [t][n] fp32):
//   bug_press.py:231-247    _exact_mask: the n_sink leading columns plus the
//                           n_exact largest-norm columns after them are kept
//   bug_press.py:264-304    _lowrank_reconstruct: the other columns are
//                           replaced by U U^T x
//   streaming_torch.py:192-258  blocked_bug_subspace / blocked_bug_project:
//                           U from augmented BUG steps over blocks of
//                           block_size of those columns, in order
// The exact set is chosen by a radix select on the norms' bit patterns (norms
// are non-negative, so bits order like values; ties go to the lower index),
// the BUG steps run through the batched step kernel with one problem, and one
// tiled kernel writes every output column.
#include "kernels.cuh"

namespace kvd {

constexpr int kPressThreads = 1024;

// norms[j] = |x_{n_sink + j}| (fp32), one warp per column.
__global__ void __launch_bounds__(256) press_norms_kernel(int n, int t, int n_sink, const float* x,
                                                         float* norms) {
  const int lane = threadIdx.x % 32;
  const int col = blockIdx.x * 8 + threadIdx.x / 32;
  if (col >= t - n_sink) return;
  const float* xr = x + (long)(n_sink + col) * n;
  float acc = 0.f;
  for (int f = lane; f < n; f += 32) acc = fmaf(xr[f], xr[f], acc);
  acc = warp_sum(acc);
  if (lane == 0) norms[col] = sqrtf(acc);
}

// One CTA: mask[c] = 1 for c < n_sink and for the k largest norms among the
// rest (ties to the lower index); idx[0..t') lists the other columns in order.
__global__ void __launch_bounds__(kPressThreads) press_select_kernel(int t, int n_sink, int k,
                                                                     const float* norms,
                                                                     unsigned char* mask, int* idx) {
  __shared__ int hist[256];
  __shared__ unsigned s_prefix;
  __shared__ int s_need, s_run, s_total;
  __shared__ int scan_scratch[32];
  const int tid = threadIdx.x;
  const int m = t - n_sink;
  unsigned thr = 0xffffffffu;  // keys > thr are taken; keys == thr while need lasts
  int need_eq = 0;
  if (k > 0 && m > 0) {
    if (tid == 0) { s_prefix = 0u; s_need = k < m ? k : m; }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
      __syncthreads();
      const unsigned pre = s_prefix;
      for (int j = tid; j < m; j += blockDim.x) {
        const unsigned key = __float_as_uint(norms[j]);
        const bool match = shift == 24 || (key >> (shift + 8)) == (pre >> (shift + 8));
        if (match) atomicAdd(&hist[(key >> shift) & 255u], 1);
      }
      __syncthreads();
      if (tid == 0) {
        int need = s_need, bucket = 0;
        for (int bkt = 255; bkt >= 0; --bkt) {
          if (hist[bkt] >= need) { bucket = bkt; break; }
          need -= hist[bkt];
        }
        s_need = need;
        s_prefix = pre | ((unsigned)bucket << shift);
      }
      __syncthreads();
    }
    thr = s_prefix;
    need_eq = s_need;
  }
  // mask and the ordered list of the remaining columns (block-wide scans)
  if (tid == 0) { s_run = 0; s_total = 0; }
  __syncthreads();
  for (int c0 = 0; c0 < t; c0 += blockDim.x) {
    const int c = c0 + tid;
    bool eq = false;
    unsigned key = 0u;
    if (c < t && c >= n_sink && k > 0) {
      key = __float_as_uint(norms[c - n_sink]);
      eq = key == thr;
    }
    int tot_eq;
    const int before_eq = cta_exclusive_scan(eq ? 1 : 0, scan_scratch, &tot_eq);
    bool keep = false;
    if (c < t) {
      if (c < n_sink) keep = true;
      else if (k > 0) keep = key > thr || (eq && s_run + before_eq < need_eq);
    }
    int tot_low;
    const int before_low = cta_exclusive_scan((c < t && !keep) ? 1 : 0, scan_scratch, &tot_low);
    if (c < t) {
      mask[c] = keep ? 1 : 0;
      if (!keep) idx[s_total + before_low] = c;
    }
    __syncthreads();
    if (tid == 0) { s_run += tot_eq; s_total += tot_low; }
    __syncthreads();
  }
}

// xc[j] = x[idx[j]] (rows of n floats)
__global__ void __launch_bounds__(256) press_gather_kernel(int n, int tl, const int* idx,
                                                          const float* x, float* xc) {
  const int row = blockIdx.x * 8 + threadIdx.x / 32;
  if (row >= tl) return;
  const float* src = x + (long)idx[row] * n;
  float* dst = xc + (long)row * n;
  for (int f = threadIdx.x % 32; f < n; f += 32) dst[f] = src[f];
}

// out[c] = U (U^T x_c) for the columns with mask[c] == 0 (U [n][ld], rank
// *r); masked columns are copied.  A CTA takes kProjTok columns: coordinates
// by threads over (column, coordinate), then the reconstruction by threads
// over (column, feature) with U staged at an odd pitch.
constexpr int kProjTok = 16;
__global__ void __launch_bounds__(256) press_project_kernel(int n, int t, int ld, const int* rr,
                                                           const float* u, const float* x,
                                                           const unsigned char* mask, float* out,
                                                           int stage_u) {
  extern __shared__ __align__(16) float psm[];
  const int r = *rr;
  // U staged at an odd pitch when it fits the launch's shared memory, else read in place
  const int ldu = stage_u ? (ld | 1) : ld;
  float* xs = psm;                                       // [kProjTok][n]
  float* cs = xs + kProjTok * n;                         // [kProjTok][ld]
  float* ust = cs + kProjTok * ld;                       // [n][ldu] when staged
  const float* us = stage_u ? ust : u;
  const int c0 = blockIdx.x * kProjTok;
  const int nt = min(kProjTok, t - c0);
  if (stage_u) {
    for (long e = threadIdx.x; e < (long)n * r; e += blockDim.x) {
      const long f = e / r, k = e % r;
      ust[f * ldu + k] = u[f * ld + k];
    }
  }
  for (long e = threadIdx.x; e < (long)nt * n; e += blockDim.x) xs[e] = x[(long)c0 * n + e];
  __syncthreads();
  for (int e = threadIdx.x; e < nt * r; e += blockDim.x) {
    const int i = e / r, k = e % r;
    const float* xr = xs + (long)i * n;
    float a0 = 0.f, a1 = 0.f;
    int f = 0;
    for (; f + 1 < n; f += 2) {
      a0 = fmaf(xr[f], us[(long)f * ldu + k], a0);
      a1 = fmaf(xr[f + 1], us[(long)(f + 1) * ldu + k], a1);
    }
    if (f < n) a0 = fmaf(xr[f], us[(long)f * ldu + k], a0);
    cs[e] = a0 + a1;
  }
  __syncthreads();
  for (long e = threadIdx.x; e < (long)nt * n; e += blockDim.x) {
    const int i = (int)(e / n), f = (int)(e % n);
    float v;
    if (mask && mask[c0 + i]) {
      v = xs[e];
    } else {
      const float* cr = cs + i * r;
      const float* ur = us + (long)f * ldu;
      v = 0.f;
      for (int k = 0; k < r; ++k) v = fmaf(cr[k], ur[k], v);
    }
    out[(long)c0 * n + e] = v;
  }
}

}  // namespace kvd

namespace {

using namespace kvd;

struct PressWs {
  unsigned char* mask;
  float* norms;
  int* idx;
  float* xc;
  float* u[2];
  float* sigma;
  int* r;
  float* rot;
  float* coords;
  int* dims;
  int* status;
  char* step;
  size_t step_bytes;
  size_t total;
};

PressWs press_ws(char* base, int n, int t, int ld, int block) {
  PressWs w{};
  size_t o = 0;
  auto take = [&](size_t bytes) { char* p = base ? base + o : nullptr; o += (bytes + 255) & ~size_t(255); return p; };
  w.mask = (unsigned char*)take((size_t)t);
  w.norms = (float*)take(4ul * t);
  w.idx = (int*)take(4ul * t);
  w.xc = (float*)take(4ul * t * n);
  w.u[0] = (float*)take(4ul * n * ld);
  w.u[1] = (float*)take(4ul * n * ld);
  w.sigma = (float*)take(4ul * ld);
  w.r = (int*)take(16);
  w.rot = (float*)take(4ul * ld * ld);
  w.coords = (float*)take(4ul * block * ld);
  w.dims = (int*)take(16);
  w.status = (int*)take(16);
  w.step_bytes = (size_t)kvd_host::bug_step_ws_per_problem(n, block, ld);
  w.step = take(w.step_bytes);
  w.total = o + 256;
  return w;
}

}  // namespace

extern "C" size_t kvd_blocked_project_workspace_bytes(int32_t n, int32_t t, int32_t rank_cap,
                                                      int32_t block_size) {
  if (n <= 0 || t < 0 || rank_cap < 1 || block_size < 1) return 0;
  const int b = block_size < t ? block_size : (t > 0 ? t : 1);
  return press_ws(nullptr, n, t, rank_cap, b).total;
}

extern "C" int kvd_blocked_project(int32_t n, int32_t t, int32_t rank_cap, int32_t block_size,
                                   int32_t n_sink, int32_t n_exact, int32_t has_theta, float theta,
                                   const float* x, float* out, uint8_t* mask_out, void* workspace,
                                   size_t ws_bytes, kvd_stream_t stream) {
  using namespace kvd_host;
  if (n <= 0 || t < 0 || rank_cap < 1 || block_size < 1 || n_sink < 0 || n_exact < 0) {
    set_error("kvd_blocked_project: bad sizes (n=%d t=%d rank=%d block=%d n_sink=%d n_exact=%d)",
              n, t, rank_cap, block_size, n_sink, n_exact);
    return KVD_ERR_ARG;
  }
  if (rank_cap > kMaxStepLd) {
    set_error("kvd_blocked_project: rank %d > %d", rank_cap, kMaxStepLd);
    return KVD_ERR_ARG;
  }
  if (t == 0) return KVD_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int b = block_size < t ? block_size : t;
  const int ld = rank_cap;
  char* base = (char*)(((uintptr_t)workspace + 255) & ~(uintptr_t)255);
  PressWs w = press_ws(base, n, t, ld, b);
  if (!workspace || ws_bytes < w.total) {
    set_error("kvd_blocked_project: workspace %zu < %zu bytes", ws_bytes, w.total);
    return KVD_ERR_WORKSPACE;
  }
  // the exact set and the ordered list of the low-rank columns
  const int m = t > n_sink ? t - n_sink : 0;
  const int kx = n_exact < m ? n_exact : m;
  if (kx > 0 && m > 0) {
    KTimerScope kts_("press_norms_kernel", s);
    press_norms_kernel<<<(m + 7) / 8, 256, 0, s>>>(n, t, n_sink, x, w.norms);
  }
  if (int rc = check_launch("press_norms_kernel")) return rc;
  {
    KTimerScope kts_("press_select_kernel", s);
    press_select_kernel<<<1, kPressThreads, 0, s>>>(t, n_sink < t ? n_sink : t, kx, w.norms, w.mask, w.idx);
  }
  if (int rc = check_launch("press_select_kernel")) return rc;
  if (mask_out) {
    cudaMemcpyAsync(mask_out, w.mask, (size_t)t, cudaMemcpyDeviceToDevice, s);
    if (int rc = check_launch("kvd_blocked_project mask")) return rc;
  }
  if (!out) return KVD_OK;  // exact set only
  const int tl = m - kx;    // low-rank columns, in order
  if (tl == 0) {
    cudaMemcpyAsync(out, x, 4ul * t * n, cudaMemcpyDeviceToDevice, s);
    return check_launch("kvd_blocked_project copy");
  }
  {
    KTimerScope kts_("press_gather_kernel", s);
    press_gather_kernel<<<(tl + 7) / 8, 256, 0, s>>>(n, tl, w.idx, x, w.xc);
  }
  if (int rc = check_launch("press_gather_kernel")) return rc;
  // blocked BUG sweep over the low-rank columns (streaming_torch.py:192-238)
  cudaMemsetAsync(w.r, 0, sizeof(int), s);
  cudaMemsetAsync(w.sigma, 0, 4ul * ld, s);
  cudaMemsetAsync(w.u[0], 0, 4ul * n * ld, s);
  cudaMemsetAsync(w.status, 0, 16, s);
  int cur = 0;
  for (int start = 0; start < tl; start += b) {
    const int bb = tl - start < b ? tl - start : b;
    BugStepBatch batch;
    BugStepArgs& a = batch.s[0];
    a.n = n; a.b = bb; a.rank_cap = rank_cap; a.ld = ld;
    a.u = w.u[cur]; a.u_out = w.u[cur ^ 1]; a.u_sp = (long)n * ld;
    a.sigma = w.sigma; a.sig_sp = ld; a.r = w.r;
    a.x = w.xc + (long)start * n; a.x_sp = (long)bb * n;
    a.rot = w.rot; a.rot_sp = (long)ld * ld;
    a.dims = w.dims;
    a.coords = w.coords; a.coords_sp = (long)bb * ld; a.coords_ld = ld;
    a.has_theta = has_theta; a.theta = theta; a.status = w.status;
    a.ws = w.step; a.ws_sp = (long)w.step_bytes;
    batch.s[1] = a;
    if (int rc = launch_bug_step(batch, 1, 1, s)) return rc;
    cur ^= 1;
  }
  const long small = 4L * (kProjTok * n + kProjTok * ld);
  const long big = small + 4L * n * (ld | 1);
  const int stage = big <= 200 * 1024;
  const int smem = (int)(stage ? big : small);
  if (int rc = ensure_smem((const void*)press_project_kernel, smem, "press_project_kernel")) return rc;
  {
    KTimerScope kts_("press_project_kernel", s);
    press_project_kernel<<<(t + kProjTok - 1) / kProjTok, 256, smem, s>>>(n, t, ld, w.r, w.u[cur], x,
                                                                          w.mask, out, stage);
  }
  if (int rc = check_launch("press_project_kernel")) return rc;
  // numerical status of the sweep (the press runs once per prefill)
  int h[4] = {0, 0, 0, 0};
  cudaMemcpyAsync(h, w.status, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (cudaStreamSynchronize(s) != cudaSuccess) return check_launch("kvd_blocked_project sync");
  if (h[kStatusNumeric]) {
    set_error("kvd_blocked_project: BUG step numerics failed (flags %d)", h[kStatusNumeric]);
    return KVD_ERR_NUMERIC;
  }
  return KVD_OK;
}
