// Host runtime of the streaming compressed-KV cache (C ABI).
//
// Owns the absorb schedule of one cache group and launches the kernels of one
// absorb step back to back on the caller's stream -- no host synchronisation
// inside a step.  The schedule mirrors the reference exactly:
//   consolidate                 bug_cache.py:1425-1429
//   _absorb_block_into_stream   bug_cache.py:725-750
//   _absorb_block_slash         bug_cache.py:752-825
//   _absorb_columns             bug_cache.py:827-904
//   _enforce_budgets            bug_cache.py:1010-1067
//   _prefill                    bug_cache.py:1431-1481
// Every lengths decision (ring, exact tier, coordinate count) depends only on
// token counts and so is taken here on the host; the data-dependent basis
// rank lives on the device (r_k/r_v) and is read by the kernels.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <cstdint>

#include <mutex>
#include <string>
#include <vector>
#include <type_traits>
#include <unordered_map>

#include "kernels.cuh"


namespace kvd_host {
using namespace kvd;

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return KVD_ERR_CUDA;
  }
  return KVD_OK;
}

// ------------------------------------------------------------ kernel timer

namespace {
struct TimerState {
  std::mutex mu;
  bool on = false;
  struct Rec { std::string name; cudaEvent_t a, b; };
  std::vector<Rec> pending;
  std::vector<cudaEvent_t> pool;
  std::unordered_map<std::string, std::pair<double, long>> acc;
  cudaEvent_t get() {
    if (!pool.empty()) { cudaEvent_t e = pool.back(); pool.pop_back(); return e; }
    cudaEvent_t e;
    cudaEventCreate(&e);
    return e;
  }
  void drain() {
    for (auto& r : pending) {
      float ms = 0.f;
      if (cudaEventSynchronize(r.b) == cudaSuccess && cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
        auto& v = acc[r.name];
        v.first += ms;
        v.second += 1;
      }
      pool.push_back(r.a);
      pool.push_back(r.b);
    }
    pending.clear();
  }
};
TimerState& timer() { static TimerState t; return t; }
}  // namespace

KTimerScope::KTimerScope(const char* name, cudaStream_t stream) : slot(-1), s(stream) {
  TimerState& t = timer();
  if (!t.on) return;
  std::lock_guard<std::mutex> lock(t.mu);
  if (t.pending.size() > 100000) t.drain();
  TimerState::Rec r{name, t.get(), t.get()};
  cudaEventRecord(r.a, stream);
  t.pending.push_back(r);
  slot = (int)t.pending.size() - 1;
}

KTimerScope::~KTimerScope() {
  if (slot < 0) return;
  TimerState& t = timer();
  std::lock_guard<std::mutex> lock(t.mu);
  if (slot < (int)t.pending.size()) cudaEventRecord(t.pending[slot].b, s);
}

// Largest dynamic shared memory a block may opt in to on the current device
// (cached per device; 0 when it cannot be read).
int device_smem_optin() {
  static std::mutex mu;
  static int per_dev[kvd::kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kvd::kMaxDevices) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (!per_dev[dev] &&
      cudaDeviceGetAttribute(&per_dev[dev], cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    per_dev[dev] = 0;
  return per_dev[dev];
}

// The dynamic shared-memory opt-in is an attribute of the function in the
// current device's context, so grants are remembered per (device, function):
// a process driving several GPUs opts in on each of them.
int ensure_smem(const void* func, size_t bytes, const char* name) {
  static std::mutex mu;
  static std::unordered_map<const void*, size_t> granted[kvd::kMaxDevices];
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) { set_error("%s: %s", name, cudaGetErrorString(e)); return KVD_ERR_CUDA; }
  if (dev < 0 || dev >= kvd::kMaxDevices) { set_error("%s: device %d beyond %d", name, dev, kvd::kMaxDevices); return KVD_ERR_ARG; }
  std::lock_guard<std::mutex> lock(mu);
  auto it = granted[dev].find(func);
  if (it != granted[dev].end() && it->second >= bytes) return KVD_OK;
  cudaFuncAttributes attr;
  e = cudaFuncGetAttributes(&attr, func);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) { set_error("%s: %s", name, cudaGetErrorString(e)); return KVD_ERR_CUDA; }
  if (bytes + attr.sharedSizeBytes > (size_t)optin) {
    set_error("%s needs %zu bytes of shared memory (+%zu static) > device limit %d", name, bytes,
              (size_t)attr.sharedSizeBytes, optin);
    return KVD_ERR_ARG;
  }
  const size_t want = (size_t)optin - attr.sharedSizeBytes;  // grant the maximum once
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)want);
  if (e != cudaSuccess) { set_error("%s: %s", name, cudaGetErrorString(e)); return KVD_ERR_CUDA; }
  granted[dev][func] = want;
  return KVD_OK;
}

// ------------------------------------------------------------ workspace

struct Ws {
  float* scores; long sc_sp;     // [P][hh_budget + max_block]
  float* xk; float* xv; long x_sp;  // [P][max_block][n]
  float* rot[4]; long rot_sp;    // [absorb parity][stream] -> [P][ld][ld]
  int* dims[4];                  // [absorb parity][stream] -> [P][4]
  int* dem;                      // [P]
  int* keep; long keep_sp;       // [P][w_cap]
  int* order;                    // [P][hh_budget + max_block] tier slot order
  int* done;                     // [P] scoring CTAs finished (fused ranking), zero between launches
  char* step[2]; long step_sp;   // per problem
  size_t total;
};

static inline size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

static Ws plan_ws(const kvd_config& c, char* base) {
  Ws w{};
  const int P = c.n_problems, n = c.num_heads * c.head_dim, ld = c.rank, mb = c.max_block;
  size_t o = 0;
  auto take = [&](size_t bytes) { char* p = base ? base + o : nullptr; o += a256(bytes); return p; };
  w.sc_sp = c.hh_budget + mb;
  w.scores = (float*)take(4ul * P * w.sc_sp);
  w.x_sp = (long)mb * n;
  w.xk = (float*)take(4ul * P * w.x_sp);
  w.xv = (float*)take(4ul * P * w.x_sp);
  w.rot_sp = (long)ld * ld;
  for (int i = 0; i < 4; ++i) w.rot[i] = (float*)take(4ul * P * w.rot_sp);
  for (int i = 0; i < 4; ++i) w.dims[i] = (int*)take(16ul * P);
  w.dem = (int*)take(4ul * P);
  w.keep_sp = c.w_cap;
  w.keep = (int*)take(4ul * P * w.keep_sp);
  w.order = (int*)take(4ul * P * w.sc_sp);
  w.done = (int*)take(4ul * P);
  w.step_sp = bug_step_ws_per_problem(n, mb, ld);
  w.step[0] = take((size_t)P * w.step_sp);
  w.step[1] = take((size_t)P * w.step_sp);
  w.total = o + 256;
  return w;
}

static int validate(const kvd_config* c) {
  if (!c) { set_error("null config"); return KVD_ERR_ARG; }
  if (c->n_problems < 1 || c->num_heads < 1 || c->head_dim < 2 || (c->head_dim & 1) ||
      c->rank < 1 || c->recent_window < 1 || c->absorb_block < 1 || c->n_sink < 0 ||
      c->prefill_block_size < 1 || c->hh_budget < 0 || c->ring_cap < 1 || c->w_cap < 1 ||
      c->max_block < c->absorb_block || c->max_block < c->prefill_block_size) {
    set_error("invalid kvd_config");
    return KVD_ERR_ARG;
  }
  if (c->dtype != KVD_DTYPE_F32 && c->dtype != KVD_DTYPE_BF16) {
    set_error("unsupported dtype %d", c->dtype);
    return KVD_ERR_DTYPE;
  }
  if (c->rank > 192) { set_error("rank %d > 192 is not supported", c->rank); return KVD_ERR_ARG; }
  if (c->w_cap < c->coord_budget + c->max_block && c->coord_budget < (1 << 30)) {
    // allowed: the host grows w_cap before it is needed; checked per step
  }
  return KVD_OK;
}

// ------------------------------------------------------------ carry stream
// The coordinate carry of absorb i (rotating every stored coordinate row into
// the new basis) is read by nothing the next absorb's scoring, selection and
// BUG step touch, so it is launched on a per-device side stream just before
// BUG step i+1 and runs beside it (the BUG step occupies one SM per problem
// and stream, the carry the rest): carry i waits for everything issued before
// BUG step i+1; BUG step i+2, which overwrites the rotation carry i reads
// (double-buffered by absorb parity), waits for carry i; eviction, which moves
// coordinate rows, flushes and waits for every carry; and each entry point
// joins the side stream back into the caller's stream before it returns, so
// callers see plain stream order.
struct CarryStream {
  cudaStream_t side = nullptr;
  cudaEvent_t bug[2] = {nullptr, nullptr}, carry[2] = {nullptr, nullptr}, join = nullptr;
  cudaEvent_t ranked = nullptr, kept = nullptr;  // the tier copy: after ranking, then done
  cudaEvent_t dfork = nullptr, djoin = nullptr;  // factored decode: verbatim tiles beside the middle
};

static CarryStream* carry_stream() {
  static std::mutex mu;
  static std::unordered_map<int, CarryStream> per_dev;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  auto it = per_dev.find(dev);
  if (it != per_dev.end()) return it->second.side ? &it->second : nullptr;
  CarryStream cs;
  bool ok = cudaStreamCreateWithFlags(&cs.side, cudaStreamNonBlocking) == cudaSuccess;
  for (int i = 0; ok && i < 2; ++i)
    ok = cudaEventCreateWithFlags(&cs.bug[i], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&cs.carry[i], cudaEventDisableTiming) == cudaSuccess;
  ok = ok && cudaEventCreateWithFlags(&cs.join, cudaEventDisableTiming) == cudaSuccess &&
       cudaEventCreateWithFlags(&cs.ranked, cudaEventDisableTiming) == cudaSuccess &&
       cudaEventCreateWithFlags(&cs.kept, cudaEventDisableTiming) == cudaSuccess &&
       cudaEventCreateWithFlags(&cs.dfork, cudaEventDisableTiming) == cudaSuccess &&
       cudaEventCreateWithFlags(&cs.djoin, cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    cs = CarryStream{};  // carries then run on the caller's stream
  }
  return (per_dev[dev] = cs).side ? &per_dev[dev] : nullptr;
}

// ------------------------------------------------------------ one group

template <typename T>
struct Group {
  const kvd_config& c;
  const kvd_buffers& b;
  kvd_counters& k;
  Ws w;
  cudaStream_t s;
  int n, P, ld;
  long row_sp_ring, row_sp_hh, u_sp, c_sp;
  RopeArgs rope;

  CarryStream* cs = nullptr;
  bool carry_pending = false;  // a carry on the side stream not yet joined
  CarryBatch pend_cb;          // the last absorb's carry, not yet launched
  int pend_par = -1;
  bool keep_pending = false;   // a tier copy on the side stream the next scoring must wait for
  bool done_zeroed = false;    // w.done cleared for this call (the fused ranking keeps it zero)

  Group(const kvd_config& c_, const kvd_buffers& b_, kvd_counters& k_, char* ws, cudaStream_t s_)
      : c(c_), b(b_), k(k_), w(plan_ws(c_, ws)), s(s_) {
    cs = carry_stream();
    n = c.num_heads * c.head_dim;
    P = c.n_problems;
    ld = c.rank;
    row_sp_ring = (long)c.ring_cap * n;
    row_sp_hh = (long)c.hh_budget * n;
    u_sp = (long)n * ld;
    c_sp = (long)c.w_cap * ld;
    rope.inv_freq = c.inv_freq;
    rope.scale = c.rope_scaling;
    rope.scale_sq = c.rope_scaling * c.rope_scaling;
  }

  ~Group() {
    flush_carry();
    join_carry();
  }

  // launch the deferred carry: on the side stream after everything issued so
  // far on the caller's stream, else on the caller's stream
  int flush_carry() {
    if (pend_par < 0) return KVD_OK;
    const int par = pend_par;
    pend_par = -1;
    if (!cs) return launch_carry(pend_cb, P, 2, ld, s);
    cudaEventRecord(cs->bug[par], s);
    cudaStreamWaitEvent(cs->side, cs->bug[par], 0);
    const int rc = launch_carry(pend_cb, P, 2, ld, cs->side);
    cudaEventRecord(cs->carry[par], cs->side);
    carry_pending = true;
    return rc;
  }

  // the caller's stream waits for every carry launched so far
  void join_carry() {
    if (!carry_pending) return;
    cudaEventRecord(cs->join, cs->side);
    cudaStreamWaitEvent(s, cs->join, 0);
    carry_pending = false;
  }

  bool lowrank() const { return c.rank >= 1 && c.coord_budget >= 1; }
  bool hh_enabled() const { return c.hh_budget >= 1 && lowrank(); }
  bool track_surprise() const { return lowrank() && c.retention == KVD_RETENTION_LOWRANK_SURPRISE; }

  // BUG step on the demoted / graduating block held in w.xk / w.xv (d columns,
  // positions and surprise already written at coordinate slots [w_len, w_len+d)).
  int absorb_columns(int d) {
    if (d <= 0) return KVD_OK;
    if (k.w_len + d > c.w_cap) {
      set_error("coordinate capacity %d too small (need %d)", c.w_cap, k.w_len + d);
      return KVD_ERR_ARG;
    }
    const int par = (int)(k.n_absorbs & 1);
    // the previous absorb's carry runs beside this step
    if (int rc0 = flush_carry()) return rc0;
    // this step overwrites rot/dims of parity `par`, last read by the carry two absorbs ago
    if (carry_pending) cudaStreamWaitEvent(s, cs->carry[par], 0);
    BugStepBatch bb;
    for (int sidx = 0; sidx < 2; ++sidx) {
      BugStepArgs& a = bb.s[sidx];
      a.n = n; a.b = d; a.rank_cap = c.rank; a.ld = ld;
      a.u = sidx == 0 ? b.u_k[k.u_sel] : b.u_v[k.u_sel];
      a.u_out = sidx == 0 ? b.u_k[k.u_sel ^ 1] : b.u_v[k.u_sel ^ 1];
      a.u_sp = u_sp;
      a.sigma = sidx == 0 ? b.sig_k : b.sig_v; a.sig_sp = ld;
      a.r = sidx == 0 ? b.r_k : b.r_v;
      a.x = sidx == 0 ? w.xk : w.xv; a.x_sp = w.x_sp;
      a.rot = w.rot[2 * par + sidx]; a.rot_sp = w.rot_sp;
      a.dims = w.dims[2 * par + sidx];
      a.coords = (sidx == 0 ? b.c_k : b.c_v) + (long)k.w_len * ld;
      a.coords_sp = c_sp; a.coords_ld = ld;
      a.has_theta = c.has_theta; a.theta = c.theta;
      a.status = b.status;
      a.ws = w.step[sidx]; a.ws_sp = w.step_sp;
    }
    int rc = launch_bug_step(bb, P, 2, s);
    if (rc) return rc;
    if (k.seeded && k.w_len > 0) {
      CarryBatch cb;
      for (int sidx = 0; sidx < 2; ++sidx) {
        CarryArgs& a = cb.s[sidx];
        a.c = sidx == 0 ? b.c_k : b.c_v; a.c_sp = c_sp; a.ld = ld;
        a.rot = w.rot[2 * par + sidx]; a.rot_sp = w.rot_sp; a.dims = w.dims[2 * par + sidx];
      }
      cb.W = k.w_len;
      pend_cb = cb;
      pend_par = par;
    }
    k.u_sel ^= 1;
    k.seeded = 1;
    k.w_len += d;
    k.n_absorbs += 1;
    return enforce_budgets();
  }

  int enforce_budgets() {
    const int f_over = k.w_len - c.coord_budget;
    if (f_over <= 0) return KVD_OK;
    if (int rc0 = flush_carry()) return rc0;
    join_carry();  // eviction moves coordinate rows
    int rc = launch_evict(P, k.w_len, f_over, c.retention, b.c_k, b.c_v, c_sp, ld, b.r_k, b.r_v,
                          b.mid_pos, track_surprise() ? b.mid_surprise : nullptr, c.w_cap, w.keep,
                          w.keep_sp, s);
    if (rc) return rc;
    k.w_len -= f_over;
    return KVD_OK;
  }

  // SLASH on a graduating block of `gb` tokens at ring slot `gslot`, true
  // positions grad_start.. (bug_cache.py:752-825).
  int absorb_slash(int gslot, int gb, int grad_start) {
    const int m = k.hh_len + gb;
    const int keep_n = m < c.hh_budget ? m : c.hh_budget;
    const int d = m - keep_n;
    if (keep_pending) {  // the exact tier this scoring reads was written on the side stream
      cudaStreamWaitEvent(s, cs->kept, 0);
      keep_pending = false;
    }
    if (gb > c.max_block) { set_error("graduating block %d > max_block", gb); return KVD_ERR_ARG; }
    CandSrc<T> src;
    src.hh_k = (const T*)b.hh_k[k.hh_sel]; src.hh_v = (const T*)b.hh_v[k.hh_sel];
    src.hh_pos = b.hh_pos[k.hh_sel]; src.hh_sp = row_sp_hh; src.hh_pos_sp = c.hh_budget;
    src.g_k = (const T*)b.ring_k + (long)gslot * n; src.g_v = (const T*)b.ring_v + (long)gslot * n;
    src.g_sp = row_sp_ring;
    src.hh_len = k.hh_len; src.grad_start = grad_start; src.n = n;
    if (d > 0 && k.w_len + d > c.w_cap) {
      set_error("coordinate capacity %d too small (need %d)", c.w_cap, k.w_len + d);
      return KVD_ERR_ARG;
    }
    SelectOut so;
    so.hh_k = b.hh_k[k.hh_sel ^ 1]; so.hh_v = b.hh_v[k.hh_sel ^ 1]; so.hh_pos = b.hh_pos[k.hh_sel ^ 1];
    so.hh_sp = row_sp_hh; so.hh_pos_sp = c.hh_budget;
    so.xk = w.xk; so.xv = w.xv; so.x_sp = w.x_sp;
    so.mid_pos = b.mid_pos; so.mid_surprise = track_surprise() ? b.mid_surprise : nullptr;
    so.mid_sp = c.w_cap; so.w_off = k.w_len; so.dem_count = w.dem;
    so.order = w.order; so.order_sp = w.sc_sp;
    // scoring and ranking in one launch where the fp64 scoring kernel runs
    if (!done_zeroed) {
      if (cudaMemsetAsync(w.done, 0, 4ul * P, s) != cudaSuccess) {
        set_error("clearing the ranking counters failed");
        return KVD_ERR_CUDA;
      }
      done_zeroed = true;
    }
    RankArgs ra{w.done, keep_n, c.hh_neighbor, so};
    bool fused = false;
    int rc = launch_slash_score<T>(src, P, m, c.num_heads, c.head_dim, rope, b.u_k[k.u_sel], u_sp,
                                   ld, b.r_k, w.scores, w.sc_sp, s, &ra, &fused);
    if (rc) return rc;
    if (!fused) {
      rc = launch_slash_select<T>(src, P, m, keep_n, c.num_heads, c.head_dim, rope, w.scores, w.sc_sp,
                                  c.hh_neighbor, so, s);
      if (rc) return rc;
    }
    // the kept tokens move into the other tier buffer beside the BUG step
    if (cs) {
      cudaEventRecord(cs->ranked, s);
      cudaStreamWaitEvent(cs->side, cs->ranked, 0);
      rc = launch_slash_keep<T>(src, P, keep_n, n, so, cs->side);
      cudaEventRecord(cs->kept, cs->side);
      keep_pending = true;
      carry_pending = true;
    } else {
      rc = launch_slash_keep<T>(src, P, keep_n, n, so, s);
    }
    if (rc) return rc;
    k.hh_sel ^= 1;
    k.hh_len = keep_n;
    return absorb_columns(d);
  }

  // Plain absorb of `gb` ring tokens at slot `gslot`, positions start.. .
  int absorb_plain(int gslot, int gb, int start) {
    if (k.w_len + gb > c.w_cap) {
      set_error("coordinate capacity %d too small (need %d)", c.w_cap, k.w_len + gb);
      return KVD_ERR_ARG;
    }
    const T* gk = (const T*)b.ring_k + (long)gslot * n;
    const T* gv = (const T*)b.ring_v + (long)gslot * n;
    int rc = launch_gather_block<T>(gk, gv, row_sp_ring, P, gb, c.num_heads, c.head_dim, start, rope,
                                    w.xk, w.xv, w.x_sp, b.mid_pos, c.w_cap, k.w_len, s);
    if (rc) return rc;
    if (track_surprise()) {
      rc = launch_surprise_f32(P, n, gb, ld, b.u_k[k.u_sel], u_sp, b.r_k, w.xk, w.x_sp,
                               b.mid_surprise + k.w_len, c.w_cap, s);
      if (rc) return rc;
    }
    return absorb_columns(gb);
  }

  int absorb_block_into_stream(int m) {
    const int gslot = k.ring_head;
    k.ring_head += m;
    k.ring_len -= m;
    if (!lowrank()) return KVD_OK;
    const int grad_start = (int)(k.cumulative_length - k.ring_len - m);
    if (hh_enabled()) return absorb_slash(gslot, m, grad_start);
    return absorb_plain(gslot, m, grad_start);
  }

  int consolidate() {
    while (k.ring_len >= c.recent_window + c.absorb_block) {
      const int rc = absorb_block_into_stream(c.absorb_block);
      if (rc) return rc;
    }
    return KVD_OK;
  }

  int ensure_ring_room(int q) {
    if (k.ring_head + k.ring_len + q <= c.ring_cap) return KVD_OK;
    if (k.ring_len + q > c.ring_cap) {
      set_error("ring capacity %d too small for %d + %d tokens", c.ring_cap, k.ring_len, q);
      return KVD_ERR_ARG;
    }
    int rc = launch_ring_compact<T>((T*)b.ring_k, row_sp_ring, k.ring_head, k.ring_len, n, P, s);
    if (rc) return rc;
    rc = launch_ring_compact<T>((T*)b.ring_v, row_sp_ring, k.ring_head, k.ring_len, n, P, s);
    if (rc) return rc;
    k.ring_head = 0;
    return KVD_OK;
  }

  int append(const kvd_hf_view& kv, const kvd_hf_view& vv) {
    const int q = kv.tokens;
    int rc = ensure_ring_room(q);
    if (rc) return rc;
    const int slot0 = k.ring_head + k.ring_len;
    if ((rc = launch_hf_to_rows<T>(kv, vv, P, c.num_heads, c.head_dim, (T*)b.ring_k, (T*)b.ring_v,
                                   row_sp_ring, slot0, s)))
      return rc;
    k.ring_len += q;
    k.cumulative_length += q;
    return KVD_OK;
  }

  int prefill(const kvd_hf_view& kv, const kvd_hf_view& vv) {
    const int t = kv.tokens;
    if (t > c.ring_cap) {
      set_error("prefill of %d tokens exceeds ring capacity %d", t, c.ring_cap);
      return KVD_ERR_ARG;
    }
    const int n_sink = t < c.n_sink ? t : c.n_sink;
    const int recent = (t - n_sink) < c.recent_window ? (t - n_sink) : c.recent_window;
    const int mid = t - n_sink - recent;
    int rc;
    if ((rc = launch_hf_to_rows<T>(kv, vv, P, c.num_heads, c.head_dim, (T*)b.ring_k, (T*)b.ring_v,
                                   row_sp_ring, 0, s)))
      return rc;
    const long sink_sp = (long)c.n_sink * n;
    if ((rc = launch_rows_copy<T>((const T*)b.ring_k, row_sp_ring, (T*)b.sink_k, sink_sp, n_sink, n, P, s))) return rc;
    if ((rc = launch_rows_copy<T>((const T*)b.ring_v, row_sp_ring, (T*)b.sink_v, sink_sp, n_sink, n, P, s))) return rc;
    k.sink_len = n_sink;
    // The ring holds the whole input while the middle is absorbed from it.
    k.ring_head = 0;
    k.ring_len = t;
    if (mid > 0 && lowrank()) {
      const bool seed = c.seed_hh_warmup && hh_enabled() && k.ingest_mode;
      for (int start = 0; start < mid; start += c.prefill_block_size) {
        const int stop = (start + c.prefill_block_size) < mid ? start + c.prefill_block_size : mid;
        const int slot = n_sink + start;
        rc = seed ? absorb_slash(slot, stop - start, slot) : absorb_plain(slot, stop - start, slot);
        if (rc) return rc;
      }
    }
    k.ring_head = n_sink + mid;
    k.ring_len = recent;
    k.cumulative_length = t;
    return KVD_OK;
  }
};

template <typename F>
static int dispatch(const kvd_config* c, F&& f) {
  if (c->dtype == KVD_DTYPE_F32) return f((float*)nullptr);
  return f((__nv_bfloat16*)nullptr);
}

}  // namespace kvd_host

using namespace kvd_host;

extern "C" const char* kvd_last_error(void) { return g_err; }

extern "C" int kvd_profile(int32_t enable) {
  TimerState& t = timer();
  std::lock_guard<std::mutex> lock(t.mu);
  t.drain();
  t.acc.clear();
  t.on = enable != 0;
  return KVD_OK;
}

extern "C" int kvd_profile_read(char* out, size_t cap) {
  TimerState& t = timer();
  std::lock_guard<std::mutex> lock(t.mu);
  t.drain();
  std::string js = "{";
  bool first = true;
  for (auto& kv : t.acc) {
    char buf[256];
    snprintf(buf, sizeof(buf), "%s\"%s\": [%.6f, %ld]", first ? "" : ", ", kv.first.c_str(),
             kv.second.first, kv.second.second);
    js += buf;
    first = false;
  }
  js += "}";
  if (!out || cap <= js.size()) { set_error("kvd_profile_read: buffer too small (%zu)", js.size() + 1); return KVD_ERR_ARG; }
  memcpy(out, js.c_str(), js.size() + 1);
  return KVD_OK;
}
extern "C" int kvd_version(void) { return 1; }

extern "C" size_t kvd_workspace_bytes(const kvd_config* cfg) {
  if (validate(cfg)) return 0;
  const Ws w = plan_ws(*cfg, nullptr);
  return w.total;
}

extern "C" int kvd_check_status(const kvd_buffers* buf, kvd_stream_t stream) {
  int32_t h[4] = {0, 0, 0, 0};
  cudaError_t e = cudaMemcpyAsync(h, buf->status, sizeof(h), cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) { set_error("status read: %s", cudaGetErrorString(e)); return KVD_ERR_CUDA; }
  cudaMemsetAsync(buf->status, 0, sizeof(h), (cudaStream_t)stream);
  if (h[kvd::kStatusTimeout]) { set_error("device wait timed out (code %d)", h[2]); return KVD_ERR_TIMEOUT; }
  if (h[kvd::kStatusBounds]) { set_error("device bounds check failed (code %d)", h[1]); return KVD_ERR_ARG; }
  if (h[kvd::kStatusNumeric]) { set_error("BUG step numerics failed (flags %d: 1 residual SVD or 2 core SVD not converged, 4 non-finite)", h[0]); return KVD_ERR_NUMERIC; }
  return KVD_OK;
}

#define KVD_WS_CHECK(cfg, ws, bytes)                                                    \
  do {                                                                                  \
    const size_t need_ = kvd_workspace_bytes(cfg);                                      \
    if ((bytes) < need_ || !(ws)) {                                                     \
      set_error("workspace %zu bytes < required %zu", (size_t)(bytes), need_);          \
      return KVD_ERR_WORKSPACE;                                                         \
    }                                                                                   \
  } while (0)

static char* align_ws(void* ws) { return (char*)(((uintptr_t)ws + 255) & ~(uintptr_t)255); }

extern "C" int kvd_prefill(const kvd_config* cfg, const kvd_buffers* buf, kvd_counters* ctr,
                           kvd_hf_view k, kvd_hf_view v, void* workspace, size_t ws_bytes,
                           kvd_stream_t stream) {
  int rc = validate(cfg);
  if (rc) return rc;
  KVD_WS_CHECK(cfg, workspace, ws_bytes);
  if (ctr->cumulative_length != 0) { set_error("kvd_prefill on a non-empty cache"); return KVD_ERR_ARG; }
  return dispatch(cfg, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    Group<T> g(*cfg, *buf, *ctr, align_ws(workspace), (cudaStream_t)stream);
    return g.prefill(k, v);
  });
}

extern "C" int kvd_append(const kvd_config* cfg, const kvd_buffers* buf, kvd_counters* ctr,
                          kvd_hf_view k, kvd_hf_view v, kvd_stream_t stream) {
  int rc = validate(cfg);
  if (rc) return rc;
  if (k.tokens != v.tokens || k.tokens < 0) { set_error("kvd_append: K/V token mismatch"); return KVD_ERR_ARG; }
  return dispatch(cfg, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    Group<T> g(*cfg, *buf, *ctr, nullptr, (cudaStream_t)stream);
    return g.append(k, v);
  });
}

extern "C" int kvd_consolidate(const kvd_config* cfg, const kvd_buffers* buf, kvd_counters* ctr,
                               void* workspace, size_t ws_bytes, kvd_stream_t stream) {
  int rc = validate(cfg);
  if (rc) return rc;
  KVD_WS_CHECK(cfg, workspace, ws_bytes);
  return dispatch(cfg, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    Group<T> g(*cfg, *buf, *ctr, align_ws(workspace), (cudaStream_t)stream);
    return g.consolidate();
  });
}

extern "C" int kvd_absorb_block(const kvd_config* cfg, const kvd_buffers* buf, kvd_counters* ctr,
                                void* workspace, size_t ws_bytes, kvd_stream_t stream) {
  int rc = validate(cfg);
  if (rc) return rc;
  KVD_WS_CHECK(cfg, workspace, ws_bytes);
  if (ctr->ring_len < cfg->recent_window + cfg->absorb_block) return KVD_OK;
  return dispatch(cfg, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    Group<T> g(*cfg, *buf, *ctr, align_ws(workspace), (cudaStream_t)stream);
    return g.absorb_block_into_stream(cfg->absorb_block);
  });
}

extern "C" int kvd_peek(const kvd_config* cfg, const kvd_buffers* buf, const kvd_counters* ctr,
                        int32_t p0, int32_t count, kvd_hf_view out_k, kvd_hf_view out_v,
                        kvd_hf_view tail_k, kvd_hf_view tail_v, kvd_stream_t stream) {
  int rc = validate(cfg);
  if (rc) return rc;
  if (p0 < 0 || count < 1 || p0 + count > cfg->n_problems) { set_error("kvd_peek: bad problem range"); return KVD_ERR_ARG; }
  const int L = ctr->sink_len + ctr->hh_len + ctr->w_len + ctr->ring_len + tail_k.tokens;
  if (out_k.tokens < L) { set_error("kvd_peek: output holds %d < %d tokens", out_k.tokens, L); return KVD_ERR_ARG; }
  return dispatch(cfg, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    return launch_peek<T>(*cfg, *buf, *ctr, p0, count, out_k, out_v, tail_k, tail_v, (cudaStream_t)stream);
  });
}

static int factored_decode(const kvd_config* cfg, const kvd_buffers* buf, const kvd_counters* ctr,
                           int32_t p0, int32_t count, int32_t head0, int32_t n_heads, const void* q,
                           int32_t num_q_heads, float scaling, void* out, void* workspace,
                           size_t ws_bytes, kvd_stream_t stream) {
  int rc = validate(cfg);
  if (rc) return rc;
  if (p0 < 0 || count < 1 || p0 + count > cfg->n_problems) { set_error("kvd_factored_decode: bad problem range"); return KVD_ERR_ARG; }
  if (head0 < 0 || n_heads < 1 || head0 + n_heads > cfg->num_heads) { set_error("kvd_factored_decode: bad KV head range [%d, %d) of %d", head0, head0 + n_heads, cfg->num_heads); return KVD_ERR_ARG; }
  if (num_q_heads < n_heads || num_q_heads % n_heads) { set_error("kvd_factored_decode: %d query heads do not group over %d KV heads", num_q_heads, n_heads); return KVD_ERR_ARG; }
  if (!q || !out) { set_error("kvd_factored_decode: null query or output"); return KVD_ERR_ARG; }
  const size_t need = decode_ws_bytes(*cfg, count, num_q_heads, n_heads);
  if (ws_bytes < need || !workspace) { set_error("kvd_factored_decode: workspace %zu < %zu", ws_bytes, need); return KVD_ERR_WORKSPACE; }
  return dispatch(cfg, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    CarryStream* cs = carry_stream();
    return launch_factored_decode<T>(*cfg, *buf, *ctr, p0, count, head0, n_heads, q, num_q_heads, scaling,
                                     out, align_ws(workspace), ws_bytes - 256, (cudaStream_t)stream,
                                     cs ? cs->side : nullptr, cs ? cs->dfork : nullptr,
                                     cs ? cs->djoin : nullptr);
  });
}

extern "C" int kvd_factored_decode(const kvd_config* cfg, const kvd_buffers* buf,
                                   const kvd_counters* ctr, int32_t p0, int32_t count,
                                   const void* q, int32_t num_q_heads, float scaling, void* out,
                                   void* workspace, size_t ws_bytes, kvd_stream_t stream) {
  if (int rc = validate(cfg)) return rc;
  return factored_decode(cfg, buf, ctr, p0, count, 0, cfg->num_heads, q, num_q_heads, scaling, out,
                         workspace, ws_bytes, stream);
}

extern "C" int kvd_factored_decode_heads(const kvd_config* cfg, const kvd_buffers* buf,
                                         const kvd_counters* ctr, int32_t p0, int32_t count,
                                         int32_t head0, int32_t n_heads, const void* q,
                                         int32_t num_q_heads, float scaling, void* out,
                                         void* workspace, size_t ws_bytes, kvd_stream_t stream) {
  return factored_decode(cfg, buf, ctr, p0, count, head0, n_heads, q, num_q_heads, scaling, out,
                         workspace, ws_bytes, stream);
}

static int factored_chunk_attention(const kvd_config* cfg, const kvd_buffers* buf,
                                    const kvd_counters* ctr, int32_t p0, int32_t count, int32_t head0,
                                    int32_t n_heads, const void* q, int64_t q_sb, int64_t q_sh,
                                    int64_t q_st, int32_t num_q_heads, int32_t q_len, float scaling,
                                    kvd_hf_view tail_k, kvd_hf_view tail_v, void* out,
                                    void* workspace, size_t ws_bytes, kvd_stream_t stream) {
  int rc = validate(cfg);
  if (rc) return rc;
  if (p0 < 0 || count < 1 || p0 + count > cfg->n_problems) { set_error("kvd_factored_chunk_attention: bad problem range"); return KVD_ERR_ARG; }
  if (!q || !out) { set_error("kvd_factored_chunk_attention: null query or output"); return KVD_ERR_ARG; }
  return launch_chunk_attention(*cfg, *buf, *ctr, p0, count, head0, n_heads, q, q_sb, q_sh, q_st,
                                num_q_heads, q_len, scaling, tail_k, tail_v, out, workspace, ws_bytes,
                                (cudaStream_t)stream);
}

extern "C" int kvd_factored_chunk_attention(const kvd_config* cfg, const kvd_buffers* buf,
                                            const kvd_counters* ctr, int32_t p0, int32_t count,
                                            const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                                            int32_t num_q_heads, int32_t q_len, float scaling,
                                            kvd_hf_view tail_k, kvd_hf_view tail_v, void* out,
                                            void* workspace, size_t ws_bytes, kvd_stream_t stream) {
  if (int rc = validate(cfg)) return rc;
  return factored_chunk_attention(cfg, buf, ctr, p0, count, 0, cfg->num_heads, q, q_sb, q_sh, q_st,
                                  num_q_heads, q_len, scaling, tail_k, tail_v, out, workspace, ws_bytes,
                                  stream);
}

extern "C" int kvd_factored_chunk_attention_heads(const kvd_config* cfg, const kvd_buffers* buf,
                                                  const kvd_counters* ctr, int32_t p0, int32_t count,
                                                  int32_t head0, int32_t n_heads, const void* q,
                                                  int64_t q_sb, int64_t q_sh, int64_t q_st,
                                                  int32_t num_q_heads, int32_t q_len, float scaling,
                                                  kvd_hf_view tail_k, kvd_hf_view tail_v, void* out,
                                                  void* workspace, size_t ws_bytes, kvd_stream_t stream) {
  return factored_chunk_attention(cfg, buf, ctr, p0, count, head0, n_heads, q, q_sb, q_sh, q_st,
                                  num_q_heads, q_len, scaling, tail_k, tail_v, out, workspace, ws_bytes,
                                  stream);
}

extern "C" size_t kvd_chunk_attention_workspace_bytes(const kvd_config* cfg, int32_t count,
                                                      int32_t num_q_heads, int32_t q_len) {
  if (!cfg || count < 1 || q_len < 1 || num_q_heads < 1) return 0;
  return chunk_attention_ws_bytes(*cfg, count, num_q_heads, q_len, cfg->num_heads);
}

extern "C" int kvd_chunk_attention_supported(const kvd_config* cfg, int32_t num_q_heads) {
  return cfg && chunk_attention_applicable(*cfg, num_q_heads, cfg->num_heads) ? 1 : 0;
}

extern "C" size_t kvd_decode_workspace_bytes(const kvd_config* cfg, int32_t count, int32_t num_q_heads) {
  if (!cfg || cfg->num_heads < 1) return 0;
  return decode_ws_bytes(*cfg, count, num_q_heads, cfg->num_heads) + 256;
}
