// Kernel argument structs and host launcher declarations shared by the
// translation units of the library.
#pragma once

#include "cta_linalg.cuh"

namespace kvd {

// Devices a process may drive through this library (per-device tables).
constexpr int kMaxDevices = 64;

struct BugStepArgs {
  int n, b, rank_cap, ld;
  const float* u; float* u_out; long u_sp;   // [P][n][ld]
  float* sigma; long sig_sp;                 // [P][ld]
  int* r;                                     // [P]
  const float* x; long x_sp;                  // [P][b][n]
  float* rot; long rot_sp;                    // [P][ld][ld]  rot[c*ld + k]
  int* dims;                                  // [P][4]  r_old, keep, m, sweeps
  float* coords; long coords_sp; int coords_ld;  // coords[p*sp + j*ld + c]
  int has_theta; float theta;
  int* status;
  char* ws; long ws_sp;                       // per-problem workspace bytes
};
// Placement of the BUG step's buffers.  Every region has a slot in the
// problem's global workspace (ws[g], bytes); the ones that fit are staged in
// the dynamic shared-memory pool instead (smem[g] >= 0, floats).  U is staged
// (kRgUs) only in shared memory; otherwise it is read in place.
enum StepRegion {
  kRgRm, kRgXr, kRgPart, kRgAs, kRgA2, kRgSmall, kRgCore, kRgPol, kRgWu, kRgWu2, kRgUs,
  kRgGram, kRgTf,  // blocks of 17..128 columns: the fp64 Gram and the factor's columns
  kRgCount
};
struct StepPlan {
  long smem[kRgCount];  // float offset in the pool, -1 = in the workspace
  long ws[kRgCount];    // byte offset in the per-problem workspace
  long ws_bytes;        // per-problem workspace bytes
  int b16, ldb, ldu, ldbt, ldw, ldp;
  int smem_bytes;       // dynamic shared memory of the launch
};
struct BugStepBatch { BugStepArgs s[2]; StepPlan plan; };

struct CarryArgs {
  float* c; long c_sp; int ld;     // [P][w_cap][ld]
  const float* rot; long rot_sp;   // [P][ld][ld]
  const int* dims;                 // [P][4]
};
struct CarryBatch { CarryArgs s[2]; int W; };

// Candidate pool of one problem: j < hh_len comes from the exact tier, the
// rest from `grad` (token-major rows, already offset to the first graduating
// token) at positions grad_start + (j - hh_len).
template <typename T>
struct CandSrc {
  const T* hh_k; const T* hh_v; const int* hh_pos; long hh_sp; long hh_pos_sp;
  const T* g_k; const T* g_v; long g_sp;
  int hh_len, grad_start, n;
  KVD_DEVICE const T* krow(int p, int j) const {
    return j < hh_len ? hh_k + p * hh_sp + (long)j * n : g_k + p * g_sp + (long)(j - hh_len) * n;
  }
  KVD_DEVICE const T* vrow(int p, int j) const {
    return j < hh_len ? hh_v + p * hh_sp + (long)j * n : g_v + p * g_sp + (long)(j - hh_len) * n;
  }
  KVD_DEVICE int pos(int p, int j) const {
    return j < hh_len ? hh_pos[p * hh_pos_sp + j] : grad_start + (j - hh_len);
  }
};

struct RopeArgs {
  const float* inv_freq;
  float scale;      // attention_scaling
  float scale_sq;   // scale * scale (the inverse divides by it)
};

struct SelectOut {
  void* hh_k; void* hh_v; int* hh_pos; long hh_sp; long hh_pos_sp;  // destination tier buffer
  float* xk; float* xv; long x_sp;        // demoted block [P][dmax][n]
  int* mid_pos; float* mid_surprise; long mid_sp; int w_off;  // written at [w_off + slot]
  int* dem_count;                          // [P] demoted count (diagnostic)
  int* order; long order_sp;               // [P][>= m] slot -> candidate (workspace)
};

// The ranking fused into the scoring launch: every CTA counts itself done
// on done[p] (zero before the launch); the CTA that completes problem p's
// scores ranks it and sets done[p] back to zero.  done == nullptr: scores
// only.
struct RankArgs {
  int* done;
  int keep_n, hh_neighbor;
  SelectOut out;
};

}  // namespace kvd

namespace kvd_host {
// Optional per-kernel CUDA-event timing (off unless kvd_profile(1) was called):
// brackets one launch with events on its stream; kvd_profile_read sums them.
struct KTimerScope {
  int slot;
  cudaStream_t s;
  KTimerScope(const char* name, cudaStream_t stream);
  ~KTimerScope();
};
// Allow `func` to use `bytes` of dynamic shared memory (checked against the
// device opt-in limit minus the kernel's static shared memory).
int ensure_smem(const void* func, size_t bytes, const char* name);
// The peek's middle on tcgen05 (bf16 caches, head_dim 64/128, rank <= 128);
// returns -1 when the shape or alignment does not apply (nothing launched).
int launch_mid_hat_umma(const kvd_config& c, const kvd_buffers& b, const kvd_counters& k, int p0,
                        int count, void* okp, void* ovp, long ob, long oh, long ot, int l0,
                        cudaStream_t s);
int device_smem_optin();
using kvd::BugStepBatch; using kvd::CarryBatch; using kvd::CandSrc; using kvd::RopeArgs; using kvd::SelectOut;
long bug_step_ws_per_problem(int n, int b, int ld);
constexpr int kMaxStepLd = 512;  // widest basis the BUG step supports
int launch_bug_step(const BugStepBatch& batch, int n_problems, int n_streams, cudaStream_t stream);
int launch_carry(const CarryBatch& batch, int n_problems, int n_streams, int ld, cudaStream_t stream);
int launch_surprise_f32(int nb, int n, int m, int ld, const float* u, long u_sp, const int* r,
                        const float* x, long x_sp, float* out, long out_sp, cudaStream_t stream);
int launch_evict(int P, int W, int f_over, int retention, float* c_k, float* c_v, long c_sp, int ld,
                 const int* rk, const int* rv, int* mid_pos, float* mid_sur, long mid_sp,
                 int* keep_ws, long kw_sp, cudaStream_t stream);
// `fuse` (optional): rank in the same launch where the fp64 scoring kernel
// runs; *fused tells whether it did (the caller then skips launch_slash_select)
template <typename T>
int launch_slash_score(const CandSrc<T>& src, int P, int m, int H, int D, RopeArgs rope,
                       const float* u, long u_sp, int ld, const int* rr, float* scores, long sc_sp,
                       cudaStream_t stream, const kvd::RankArgs* fuse = nullptr, bool* fused = nullptr);
template <typename T>
int launch_slash_select(const CandSrc<T>& src, int P, int m, int keep_n, int H, int D,
                        RopeArgs rope, const float* scores, long sc_sp, int hh_neighbor,
                        const SelectOut& out, cudaStream_t stream);
template <typename T>
int launch_slash_keep(const CandSrc<T>& src, int P, int keep_n, int n, const SelectOut& out,
                      cudaStream_t stream);
template <typename T>
int launch_gather_block(const T* g_k, const T* g_v, long g_sp, int P, int b, int H, int D,
                        int start, RopeArgs rope, float* xk, float* xv, long x_sp, int* mid_pos,
                        long mid_sp, int w_off, cudaStream_t stream);
template <typename T>
int launch_hf_to_rows(const kvd_hf_view& kv, const kvd_hf_view& vv, int P, int H, int D, T* dst_k,
                      T* dst_v, long dst_sp, int slot0, cudaStream_t s);
template <typename T>
int launch_rows_copy(const T* src, long src_sp, T* dst, long dst_sp, int count, int n, int P,
                     cudaStream_t s);
template <typename T>
int launch_ring_compact(T* ring, long sp, int head, int len, int n, int P, cudaStream_t s);
template <typename T>
int launch_peek(const kvd_config& c, const kvd_buffers& b, const kvd_counters& k, int p0, int count,
                const kvd_hf_view& ok_, const kvd_hf_view& ov_, const kvd_hf_view& tk,
                const kvd_hf_view& tv, cudaStream_t s);
// workspace of a decode over `n_heads` KV heads answering num_q_heads query heads
size_t decode_ws_bytes(const kvd_config& c, int count, int num_q_heads, int n_heads);
template <typename T>
// `side` (with two events), when given, runs the verbatim tiles concurrently
// with the middle tier; the merge waits for both on `s`.
// KV heads [h0, h0 + hc) of the cache; q and out hold their Hq query heads.
int launch_factored_decode(const kvd_config& c, const kvd_buffers& b, const kvd_counters& k, int p0,
                           int count, int h0, int hc, const void* q, int Hq, float scaling, void* out, char* ws,
                           size_t ws_bytes, cudaStream_t s, cudaStream_t side = nullptr,
                           cudaEvent_t ev_fork = nullptr, cudaEvent_t ev_join = nullptr);
// Factored chunk attention (chunk_attn.cu): bf16, head_dim 64, rank <= 32.
// KV heads [h0, h0 + hc) of the cache (n_heads = hc); q and out hold their
// Hq query heads, the tail views every KV head.
bool chunk_attention_applicable(const kvd_config& c, int num_q_heads, int n_heads);
int launch_chunk_attention(const kvd_config& c, const kvd_buffers& bu, const kvd_counters& k, int p0,
                           int count, int h0, int hc, const void* q, int64_t q_sb, int64_t q_sh,
                           int64_t q_st, int Hq, int q_len, float scaling, const kvd_hf_view& tail_k,
                           const kvd_hf_view& tail_v, void* out, void* ws, size_t ws_bytes,
                           cudaStream_t s);
size_t chunk_attention_ws_bytes(const kvd_config& c, int count, int num_q_heads, int q_len, int n_heads);
}  // namespace kvd_host
