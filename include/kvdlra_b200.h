/*
 * kvdlra_b200 -- C ABI of the B200 (sm_100a) streaming compressed-KV path.
 *
 * The library implements, on device, one streaming-BUG KV cache "group":
 * P independent problems (sequence x layer) that share one configuration and
 * one absorb schedule.  Every buffer is owned by the caller (the Python host
 * allocates them with PyTorch); the library never allocates device memory,
 * except where an entry point says otherwise.  All pointers are device
 * pointers unless noted; every call is asynchronous on the given stream and
 * returns an int status (KVD_OK or a KVD_ERR_* code, with a message from
 * kvd_last_error()).
 *
 * Reference interfaces replaced (kvdlra, Python):
 *   src/kvdlra/cache/bug_cache.py         BugStreamingLayer / BugStreamingCache
 *   src/kvdlra/integrators/streaming_torch.py  augmented_bug_step, blocked_bug_*
 * Each entry point cites the reference function whose behaviour it provides.
 *
 * Layouts (P problems, n = num_heads * head_dim, feature index = head*D + d):
 *   verbatim tiers  token-major  [P][slots][n]   model dtype
 *   basis U         row-major    [P][n][rank]    fp32 (columns beyond r unused)
 *   coordinates C   token-major  [P][w_cap][rank] fp32
 *   HF tensors      (B, H, T, D) with explicit strides, model dtype
 */
#ifndef KVDLRA_B200_H
#define KVDLRA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* kvd_stream_t; /* == cudaStream_t */

enum {
  KVD_OK = 0,
  KVD_ERR_ARG = 1,       /* bad shape / argument / capacity */
  KVD_ERR_DTYPE = 2,     /* unsupported dtype */
  KVD_ERR_WORKSPACE = 3, /* workspace too small */
  KVD_ERR_CUDA = 4,      /* CUDA launch or runtime error */
  KVD_ERR_TIMEOUT = 5,   /* a bounded device-side wait gave up */
  KVD_ERR_NUMERIC = 6    /* device reported a numerical failure */
};

enum { KVD_DTYPE_F32 = 0, KVD_DTYPE_BF16 = 1 };
enum { KVD_RETENTION_FIFO = 0, KVD_RETENTION_LOWRANK_SURPRISE = 1 };

/* Configuration of one cache group (bug_cache.py:313-540 constructor knobs). */
typedef struct kvd_config {
  int32_t n_problems;         /* P */
  int32_t num_heads;          /* KV heads H */
  int32_t head_dim;           /* D (even) */
  int32_t dtype;              /* KVD_DTYPE_* of the verbatim tiers / HF tensors */
  int32_t rank;               /* rank cap r (>= 1) */
  int32_t coord_budget;       /* max coordinate columns per problem */
  int32_t recent_window;
  int32_t absorb_block;
  int32_t n_sink;
  int32_t prefill_block_size;
  int32_t retention;          /* KVD_RETENTION_* */
  int32_t hh_budget;          /* exact-tier size h (0 = no tier) */
  int32_t hh_neighbor;        /* span-boost half width (0 = off) */
  int32_t seed_hh_warmup;     /* route the first ingest chunk's middle through SLASH */
  int32_t has_theta;          /* Frobenius-tail truncation on/off */
  float theta;
  float rope_scaling;         /* rotary attention_scaling (cos/sin multiplier) */
  const float* inv_freq;      /* device, head_dim/2 fp32 rotary inverse frequencies */
  int32_t ring_cap;           /* recent-ring slots per problem */
  int32_t w_cap;              /* coordinate slots per problem (>= coord_budget + max block) */
  int32_t max_block;          /* largest BUG block (max(absorb_block, prefill_block_size)) */
} kvd_config;

/* Device buffers of one group (all caller-owned). */
typedef struct kvd_buffers {
  void* sink_k; void* sink_v;           /* [P][n_sink][n] */
  void* ring_k; void* ring_v;           /* [P][ring_cap][n] */
  void* hh_k[2]; void* hh_v[2];         /* [P][hh_budget][n]  ping-pong */
  int32_t* hh_pos[2];                   /* [P][hh_budget] */
  float* u_k[2]; float* u_v[2];         /* [P][n][rank]  ping-pong */
  float* sig_k; float* sig_v;           /* [P][rank]  diagonal square-root core */
  int32_t* r_k; int32_t* r_v;           /* [P] current basis rank */
  float* c_k; float* c_v;               /* [P][w_cap][rank] */
  int32_t* mid_pos;                     /* [P][w_cap] true positions of coordinates */
  float* mid_surprise;                  /* [P][w_cap] graduation-time surprise */
  int32_t* status;                      /* [4] device status words (0 = ok) */
} kvd_buffers;

/* Host-side schedule counters of one group, updated by the calls below. */
typedef struct kvd_counters {
  int64_t cumulative_length;  /* tokens seen (true positions advance with it) */
  int32_t sink_len;
  int32_t ring_head;          /* first live ring slot */
  int32_t ring_len;
  int32_t hh_len;             /* exact-tier tokens held */
  int32_t hh_sel;             /* live exact-tier buffer (0/1) */
  int32_t u_sel;              /* live basis buffer (0/1) */
  int32_t w_len;              /* coordinate columns held */
  int32_t seeded;             /* a basis exists (first BUG step done) */
  int32_t n_absorbs;          /* BUG steps taken */
  int32_t ingest_mode;        /* 1 while inside BugStreamingCache.ingesting() */
} kvd_counters;

/* HF-layout tensor view (B, H, T, D): element (b,h,t,d) at
 * ptr + b*stride_b + h*stride_h + t*stride_t + d  (element strides). */
typedef struct kvd_hf_view {
  void* ptr;
  int64_t stride_b, stride_h, stride_t;
  int32_t tokens;
} kvd_hf_view;

/* ------------------------------------------------------------------ meta */

const char* kvd_last_error(void);
int kvd_version(void);
/* Bytes of scratch workspace the calls below need for this configuration. */
size_t kvd_workspace_bytes(const kvd_config* cfg);
/* Read and clear the device status words (synchronises the stream). */
int kvd_check_status(const kvd_buffers* buf, kvd_stream_t stream);

/* ------------------------------------------------------------ cache ops */

/* First update of a group: sinks, ring and the middle absorbed in
 * prefill_block_size sub-blocks (through the exact-tier selection when
 * seed_hh_warmup and counters->ingest_mode).  bug_cache.py:1431-1481. */
int kvd_prefill(const kvd_config* cfg, const kvd_buffers* buf, kvd_counters* ctr,
                kvd_hf_view k, kvd_hf_view v, void* workspace, size_t ws_bytes,
                kvd_stream_t stream);

/* Append a chunk (ingest) or one token (decode) to the recent ring and advance
 * cumulative_length.  bug_cache.py:1404-1423 (ingest), 1483-1491 (decode). */
int kvd_append(const kvd_config* cfg, const kvd_buffers* buf, kvd_counters* ctr,
               kvd_hf_view k, kvd_hf_view v, kvd_stream_t stream);

/* Absorb while ring_len >= recent_window + absorb_block: per block the
 * exact-tier selection (surprise scores, stable top-h, tier compaction), the
 * augmented BUG step on K and V, the coordinate carry, the append of the new
 * coordinates and the budget eviction.  bug_cache.py:1425-1429, 725-1067. */
int kvd_consolidate(const kvd_config* cfg, const kvd_buffers* buf, kvd_counters* ctr,
                    void* workspace, size_t ws_bytes, kvd_stream_t stream);

/* One iteration of the loop above: graduate the oldest absorb_block ring
 * tokens if the ring holds at least recent_window + absorb_block of them
 * (bug_cache.py:725-750); a no-op otherwise. */
int kvd_absorb_block(const kvd_config* cfg, const kvd_buffers* buf, kvd_counters* ctr,
                     void* workspace, size_t ws_bytes, kvd_stream_t stream);

/* Dense [sinks | exact tier | RoPE(U_k C_k) | ring (| tail)] K and V in HF layout
 * for problems [p0, p0+count) -- the reference's _decode_peek / _score_forward
 * return value (bug_cache.py:1496-1575, 1390-1402).  `tail` (tokens may be 0)
 * is appended after the ring (frozen scoring's window). */
int kvd_peek(const kvd_config* cfg, const kvd_buffers* buf, const kvd_counters* ctr,
             int32_t p0, int32_t count, kvd_hf_view out_k, kvd_hf_view out_v,
             kvd_hf_view tail_k, kvd_hf_view tail_v, kvd_stream_t stream);

/* Factored decode attention for problems [p0, p0+count): one query token per
 * problem, q (count, Hq, D) post-RoPE, against the retained cache without
 * materialising the middle: keys RoPE(U_k,g c_t) per KV group g, values
 * U_v,g (sum_t p_t c_v,t); exact tiers read verbatim.  Replaces HF attention
 * over bug_cache.py:1496-1519's dense peek.  out (count, Hq, D) in the model
 * dtype.  q/out are contiguous. */
int kvd_factored_decode(const kvd_config* cfg, const kvd_buffers* buf, const kvd_counters* ctr,
                        int32_t p0, int32_t count, const void* q, int32_t num_q_heads,
                        float scaling, void* out, void* workspace, size_t ws_bytes,
                        kvd_stream_t stream);

/* Factored chunk attention for problems [p0, p0+count): every query of a
 * chunk, q (count, Hq, q_len, D) post-RoPE with element strides (q_sb, q_sh,
 * q_st) and unit stride over D, against [sinks | exact tier | RoPE(U_k C_k) |
 * ring (| tail)] with the causal mask over the last q_len keys, without
 * materialising the middle: keys rebuilt per 128-token tile on the tensor
 * cores, values accumulated in coordinate space.  Replaces HF attention over
 * bug_cache.py:1404-1423's (ingest: the chunk is the end of the ring, tail
 * empty) and 1390-1402's (frozen scoring: the chunk is `tail`) dense return
 * value.  out (count, q_len, Hq, D) contiguous.  bf16, head_dim 64, rank <=
 * 32 with rank % 4 == 0 (kvd_chunk_attention_supported); KVD_ERR_ARG
 * otherwise. */
int kvd_factored_chunk_attention(const kvd_config* cfg, const kvd_buffers* buf, const kvd_counters* ctr,
                                 int32_t p0, int32_t count, const void* q, int64_t q_sb, int64_t q_sh,
                                 int64_t q_st, int32_t num_q_heads, int32_t q_len, float scaling,
                                 kvd_hf_view tail_k, kvd_hf_view tail_v, void* out, void* workspace,
                                 size_t ws_bytes, kvd_stream_t stream);
/* Workspace bytes that let kvd_factored_chunk_attention split the keys over
 * several CTAs per query tile (a smaller or null workspace runs unsplit). */
size_t kvd_chunk_attention_workspace_bytes(const kvd_config* cfg, int32_t count, int32_t num_q_heads,
                                           int32_t q_len);
/* 1 when kvd_factored_chunk_attention takes this configuration. */
int kvd_chunk_attention_supported(const kvd_config* cfg, int32_t num_q_heads);

/* Head-sharded attention (no counterpart in the reference, which runs on one
 * device): the two calls above restricted to KV heads [head0, head0 +
 * n_heads) of the cache, for a single sequence whose attention is split over
 * GPUs by KV head while every GPU keeps the whole cache (the basis is joint
 * over heads, bug_cache.py:605-607, so each absorb needs every head's keys).
 * q and out hold only the query heads of those KV heads, grouped as in the
 * model (num_q_heads a multiple of n_heads); the tail views hold every KV
 * head.  Concatenating the outputs of a partition of the heads gives the
 * full call's output.  Workspace: the full call's size covers any range. */
int kvd_factored_decode_heads(const kvd_config* cfg, const kvd_buffers* buf, const kvd_counters* ctr,
                              int32_t p0, int32_t count, int32_t head0, int32_t n_heads,
                              const void* q, int32_t num_q_heads, float scaling, void* out,
                              void* workspace, size_t ws_bytes, kvd_stream_t stream);
int kvd_factored_chunk_attention_heads(const kvd_config* cfg, const kvd_buffers* buf,
                                       const kvd_counters* ctr, int32_t p0, int32_t count,
                                       int32_t head0, int32_t n_heads, const void* q, int64_t q_sb,
                                       int64_t q_sh, int64_t q_st, int32_t num_q_heads, int32_t q_len,
                                       float scaling, kvd_hf_view tail_k, kvd_hf_view tail_v,
                                       void* out, void* workspace, size_t ws_bytes,
                                       kvd_stream_t stream);

/* ------------------------------------------------ integrator primitives */

/* Batched augmented rank-adaptive BUG step on `n_batch` independent problems
 * (streaming_torch.py:82-189).  u/u_out [nb][n][ld_u] fp32 (u_out may not
 * alias u), sigma [nb][ld_u], r [nb] (0 = seeding step; updated in place),
 * block [nb][b][n] token-major fp32, rot_out [nb][ld_u][ld_u] (rot[k][j] =
 * u_new^T u_old), m_out [nb] admitted directions, coords_out [nb][b][ld_u]
 * (u_new^T block).  rank_cap <= ld_u. */
int kvd_bug_step(int32_t n_batch, int32_t n, int32_t b, int32_t rank_cap, int32_t ld_u,
                 const float* u, float* u_out, float* sigma, int32_t* r, const float* block,
                 float* rot_out, int32_t* m_out, float* coords_out, int32_t has_theta,
                 float theta, int32_t* status, void* workspace, size_t ws_bytes,
                 kvd_stream_t stream);
size_t kvd_bug_step_workspace_bytes(int32_t n_batch, int32_t n, int32_t b, int32_t ld_u);

/* kvd_bug_step for callers that cannot allocate device memory (no
 * counterpart in the reference, which has no compiled code): the same step
 * with no workspace argument.  Its scratch is a fixed 16 MiB array inside the
 * library (kvd_bug_step_noalloc_max_scratch()), held on every GPU that loads
 * the library; requests that need more return KVD_ERR_WORKSPACE.  The first
 * call on a device looks up the array's device address, so make it before any
 * stream capture.  The scratch used is the current device's: `stream` must
 * belong to the device current on the calling thread.  Calls share the array:
 * calls that overlap on the GPU race and must be serialised by the caller.
 * Allocates nothing. */
int kvd_bug_step_noalloc(int32_t n_batch, int32_t n, int32_t b, int32_t rank_cap, int32_t ld_u,
                         const float* u, float* u_out, float* sigma, int32_t* r,
                         const float* block, float* rot_out, int32_t* m_out, float* coords_out,
                         int32_t has_theta, float theta, int32_t* status, kvd_stream_t stream);
size_t kvd_bug_step_noalloc_max_scratch(void);

/* Low-rank surprise of token-major fp32 columns x [nb][m][n] against bases
 * u [nb][n][ld_u] of rank r[nb]: sqrt(max(|k|^2-|U^T k|^2,0))/max(|k|,1e-12),
 * 1.0 where r == 0.  bug_cache.py:906-921. */
int kvd_surprise(int32_t n_batch, int32_t n, int32_t m, int32_t ld_u, const float* u,
                 const int32_t* r, const float* x, float* out, kvd_stream_t stream);

/* Stable descending top-k over scores [nb][m]: keep_idx [nb][k] and
 * demote_idx [nb][m-k], each ascending.  bug_cache.py:810-812. */
int kvd_select_topk(int32_t n_batch, int32_t m, int32_t k, const float* scores,
                    int32_t* keep_idx, int32_t* demote_idx, kvd_stream_t stream);

/* ------------------------------------------------------- prefill press */

/* Blocked BUG projection of one feature-by-token matrix, held token-major as
 * x [t][n] fp32 (replaces bug_press.py:231-304 _exact_mask /
 * _lowrank_reconstruct on top of streaming_torch.py:192-258
 * blocked_bug_subspace / blocked_bug_project).  Columns c < n_sink and the
 * n_exact largest-norm columns after them (ties to the lower index) form the
 * exact set; the rest, in order, drive augmented BUG steps over blocks of
 * block_size columns (rank_cap <= 512, theta if has_theta) and are written as
 * U U^T x_c to out [t][n]; exact columns are copied.  mask_out [t] (may be
 * NULL) receives 1 for exact columns.  out == NULL computes the exact set
 * only.  Synchronises the stream once to read the sweep's numerical status. */
int kvd_blocked_project(int32_t n, int32_t t, int32_t rank_cap, int32_t block_size,
                        int32_t n_sink, int32_t n_exact, int32_t has_theta, float theta,
                        const float* x, float* out, uint8_t* mask_out, void* workspace,
                        size_t ws_bytes, kvd_stream_t stream);
size_t kvd_blocked_project_workspace_bytes(int32_t n, int32_t t, int32_t rank_cap,
                                           int32_t block_size);

/* Workspace bytes kvd_factored_decode needs for `count` problems. */
size_t kvd_decode_workspace_bytes(const kvd_config* cfg, int32_t count, int32_t num_q_heads);

/* ------------------------------------------------------------ RoPE angles */

/* cos/sin tables of the rotary angles, out[i][f] for i < n positions and
 * f < nf frequencies (fp32, row-major), each scaled by `scale`: fast = 0 is
 * the full-precision path the cache uses for un-rotation and peeks
 * (sincosf of the fp32 product pos * inv_freq, as the model's rotary module
 * forms it), fast = 1 the reduced-instruction path the factored decode
 * uses inside its tiles (Cody-Waite reduction by 2*pi, hardware sin/cos on
 * the reduced angle).  Device pointers; asynchronous on `stream`. */
int kvd_rope_table(int32_t n, const int32_t* pos, int32_t nf, const float* inv_freq, float scale,
                   int32_t fast, float* cos_out, float* sin_out, kvd_stream_t stream);

/* ------------------------------------------------------------- profiling */

/* Per-kernel CUDA-event timing: kvd_profile(1) brackets every kernel launch of
 * this library with an event pair on its stream (kvd_profile(0) stops and
 * clears); kvd_profile_read synchronises and writes
 * {"kernel_name": [total_ms, launches], ...} as a JSON string. */
int kvd_profile(int32_t enable);
int kvd_profile_read(char* out, size_t cap);

#ifdef __cplusplus
}
#endif

#endif /* KVDLRA_B200_H */
