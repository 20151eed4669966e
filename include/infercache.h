/*
 * infercache.h -- C ABI of the B200 (sm_100a) KV-cache decode hot path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as void*.  Nothing here allocates or frees memory and no pointer is
 * kept beyond a call: the caller owns every buffer.  Calls are asynchronous on
 * the given stream.  Every entry point returns IC_OK (0) or a negative
 * ic_status; ic_status_str() names it.
 *
 * Storage model (one PagePool shared by many sessions):
 *   pool K / V        [num_layers, num_kv_heads, pool_tokens, head_dim]
 *                     (the PagePool layout of paged_cache.py:103-123; a token
 *                     row is page_id * 16 + slot_in_page, paged_cache.py:156)
 *   slot_table        int32 [S, budget + 1]: pool row of each logical slot of
 *                     session s.  Entry `budget` is the session's staging row,
 *                     where the token being decoded is appended.
 *   positions         int64 [S, budget]  (-1 = empty)   hierarchical_cache.py:133
 *   importance        float [S, budget]                  hierarchical_cache.py:135
 *   occupied          uint8 [S, budget]                  hierarchical_cache.py:137
 *   ctrl              int32 [S, IC_CTRL_WORDS]  fill pointers, :140-143
 *   counters          int64 [S, IC_COUNTER_WORDS]  CacheStats, :98-105
 *
 * Logical slots follow CacheConfig (hierarchical_cache.py:67-93):
 * [0, sink) sinks, [sink, sink+recent) the recent ring, [sink+recent, budget)
 * the scored L2 pool.  A promotion moves a token between logical slots by
 * swapping slot_table entries; K/V rows are never copied after the append.
 */
#ifndef INFERCACHE_H_
#define INFERCACHE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IC_ABI_VERSION 3

/* Status codes.  The Python layer maps them to the reference's exception
 * types: RuntimeError for exhaustion / cap (paged_cache.py:229, 244),
 * ValueError for bad arguments (kll_sketch.py:49-50). */
enum ic_status {
  IC_OK = 0,
  IC_ERR_INVALID_ARG = -1,     /* null pointer, bad size, bad dtype      */
  IC_ERR_UNSUPPORTED = -2,     /* shape not compiled (head_dim, group)   */
  IC_ERR_OUT_OF_PAGES = -3,    /* page pool exhausted                    */
  IC_ERR_SESSION_CAP = -4,     /* per-session page cap exceeded          */
  IC_ERR_CORRUPT_TABLE = -5,   /* slot / page table entry out of range   */
  IC_ERR_LAUNCH = -6,          /* kernel launch failed                   */
  IC_ERR_DEVICE_TIMEOUT = -7,  /* a bounded device-side wait gave up     */
  IC_ERR_CUDA = -8,            /* other CUDA runtime error               */
  IC_ERR_NO_DEVICE = -9        /* no sm_100 device current               */
};

enum ic_dtype { IC_F32 = 0, IC_F16 = 1, IC_BF16 = 2 };

/* ctrl words per session */
enum ic_ctrl {
  IC_CTRL_SINK_FILL = 0,
  IC_CTRL_RECENT_FILL = 1,
  IC_CTRL_RECENT_PTR = 2,
  IC_CTRL_IMPORTANT_FILL = 3,
  IC_CTRL_WORDS = 8
};

/* counter words per session */
enum ic_counter {
  IC_CNT_TOKENS_SEEN = 0,
  IC_CNT_EVICTIONS = 1,
  IC_CNT_STEPS = 2,
  IC_CNT_PROMOTIONS = 3,
  IC_CNT_NEAR_TIES = 4,    /* eviction decisions whose two smallest L2 scores
                              were within 1e-6 relative (words 5-7 reserved) */
  IC_COUNTER_WORDS = 8
};

/* kinds in an event record {kind, displaced_pos, target_slot, evicted_pos} */
enum ic_event_kind {
  IC_EV_NONE = 0,    /* ring slot was empty                               */
  IC_EV_DROP = 1,    /* displaced token scored <= 0: dropped              */
  IC_EV_FILL = 2,    /* displaced token moved into a free L2 slot         */
  IC_EV_EVICT = 3,   /* displaced token replaced the L2 minimum           */
  IC_EV_REJECT = 4   /* displaced token scored <= the L2 minimum: dropped */
};

/* device status word bits (written by kernels with bounded waits) */
#define IC_DEVFLAG_TIMEOUT 1
#define IC_DEVFLAG_BAD_ROW 2

typedef struct ic_pool {
  void* k;                 /* [L, Hkv, pool_tokens, D] */
  void* v;
  int64_t pool_tokens;     /* n_pages * 16 */
  int32_t num_layers;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t dtype;           /* ic_dtype */
} ic_pool;

typedef struct ic_tiers {
  int32_t sink_size;
  int32_t recent_size;
  int32_t important_size;
  int32_t budget;          /* sink + recent + important */
} ic_tiers;

typedef struct ic_sessions {
  int32_t num_sessions;
  int32_t _pad;
  int32_t* slot_table;     /* [S, budget + 1] */
  int64_t* positions;      /* [S, budget] */
  float* importance;       /* [S, budget] */
  uint8_t* occupied;       /* [S, budget] */
  int32_t* ctrl;           /* [S, IC_CTRL_WORDS] */
  int64_t* counters;       /* [S, IC_COUNTER_WORDS] */
  int32_t* dev_status;     /* one int32, OR-ed with IC_DEVFLAG_*; may be NULL */
} ic_sessions;

/* ---- Kernel A: fused decode step for one layer over all sessions --------
 * For every session s and KV head h: appends k_new/v_new[s, h] into the
 * staging row of layer `layer`, attends the Hq/Hkv query heads of the group
 * over every occupied logical slot plus the new token (scale * q.k, softmax,
 * P.V), writes out[s, h*G + g], and folds the received mass of each slot
 * summed over the group's query heads into mass[s, h, slot] (index `budget`
 * is the new token): layer 0 stores it, every later layer adds its own after
 * the previous layer's kernel has completed, so the per-head sum runs in
 * layer order whatever the launches' overlap.  The first layer of a step must
 * be layer 0.
 * Replaces: compact_sdp_attention (triton_ops.py:251-287), gather_cache_kv
 * (:107-135), scatter_importance (:148-175), the model attention fed by
 * to_hf_past_key_values (hierarchical_cache.py:297-351, two_pass.py:312-321)
 * and the per-layer K/V writes of push (hierarchical_cache.py:271-275). */
typedef struct ic_decode_args {
  ic_pool pool;
  ic_tiers tiers;
  ic_sessions sess;
  int32_t layer;
  int32_t num_q_heads;
  const void* q;           /* [S, Hq, D]  pool dtype */
  const void* k_new;       /* [S, Hkv, D] pool dtype */
  const void* v_new;       /* [S, Hkv, D] pool dtype */
  void* out;               /* [S, Hq, D]  out_dtype */
  int32_t out_dtype;       /* ic_dtype: pool dtype or IC_F32 */
  int32_t inputs_ready;    /* 1: q, k_new and v_new of every layer of this
                              step were complete before the step's first
                              launch (ic_decode_step), so a layer may read them
                              before the previous layer finishes; 0: they may
                              come from the immediately preceding kernel */
  float* mass;             /* [S, Hkv, budget + 1] running sum over layers */
  float scale;             /* softmax scale, normally head_dim ** -0.5 */
  int32_t cluster_size;    /* cluster variants: 0 = choose; TENSOR_CORES 8 or
                              16, TENSOR_SPLIT 1..16 */
  int32_t kernel_variant;  /* ic_decode_variant */
  int32_t pdl;             /* 1: launch with programmatic dependent launch */
} ic_decode_args;

/* Kernel A implementations.  AUTO picks CUDA cores for fp32 pools; for fp16 /
 * bf16 pools the lean kernel when inputs_ready and pdl are set (the layers of
 * one ic_decode_step overlap) and the slot-split kernel otherwise (one layer at
 * a time, as a decoder forward calls it). */
enum ic_decode_variant {
  IC_DECODE_AUTO = 0,
  IC_DECODE_CUDA_CORES = 1,      /* fp32 / fp16 / bf16, one cluster per group   */
  IC_DECODE_TENSOR_CORES = 2,    /* fp16 / bf16, one cluster per group          */
  IC_DECODE_TENSOR_STREAM = 3,   /* fp16 / bf16, one CTA streams a whole group  */
  IC_DECODE_TENSOR_LEAN = 4,     /* fp16 / bf16, one CTA, four warp pipelines   */
  IC_DECODE_TENSOR_SPLIT = 5     /* fp16 / bf16, a cluster of CTAs over chunks of
                                    the group's slots, merged through distributed
                                    shared memory; cluster_size = CTAs per group
                                    (0 = choose: the fewest per group, up to 8,
                                    that fit and give 64 CTAs; at most 16)      */
};
int ic_decode_layer(const ic_decode_args* a, void* stream);

/* ---- Kernel B: importance update, promotion / eviction, ring advance -----
 * Once per session-step after the last layer.  For every occupied slot j:
 *   importance[j] = importance[j] * decay + (sum_h sum_l mass[s, h, j, l]) / mass_div
 * (sums in index order, heads outer; decay == 1 leaves the product exact;
 * mass == NULL adds nothing).  Then the
 * token in ring slot recent_ptr, if any, is promoted to L2 or dropped exactly
 * as _maybe_promote_to_l2 (hierarchical_cache.py:448-477) with the
 * first-index argmin of _l2_min_slot (:420-425), and the staging row becomes
 * ring slot recent_ptr holding position new_pos[s] (push, :264-288).
 * Replaces topk_min_slot (triton_ops.py:207-235), GPUImportanceTracker
 * (:299-346) and the KLL sketch path (kll_sketch.py, never read). */
typedef struct ic_evict_args {
  ic_tiers tiers;
  ic_sessions sess;
  const float* mass;       /* [S, mass_heads, budget + 1, mass_layers] or NULL */
  int32_t mass_heads;
  int32_t mass_layers;
  float mass_div;
  float decay;
  int32_t pdl;             /* 1: launch with programmatic dependent launch; 2: the
                              same, and the kernel before it on the stream writes
                              none of the session state but the mass (a kernel-A
                              layer): that state is staged before the wait */
  int32_t advance_pos;     /* 1: new_pos[s] += 1 once read (the next step's position) */
  int64_t* new_pos;        /* [S] */
  int64_t* events;         /* [S, 4] record of this step, or NULL */
} ic_evict_args;
int ic_evict_update(const ic_evict_args* a, void* stream);

/* ---- One whole decode step: kernel A for layers 0 .. L-1, then kernel B ---
 * `layer0` describes layer 0 (its `layer` and `inputs_ready` fields are
 * ignored); layer l reads q + l * q_layer_stride, k_new / v_new +
 * l * kv_layer_stride and writes out + l * out_layer_stride (strides in
 * elements of the respective dtype).  `evict` is then applied with its own
 * fields (normally the decode mass buffer with mass_heads = Hkv,
 * mass_layers = 1, mass_div = L * Hkv).
 * Layers are launched with inputs_ready = 1.  The decode loop of
 * _generate_two_pass (two_pass.py:302-336) with the model's per-layer
 * attention and the cache push of one token per session. */
typedef struct ic_step_args {
  ic_decode_args layer0;
  int64_t q_layer_stride;
  int64_t kv_layer_stride;
  int64_t out_layer_stride;
  ic_evict_args evict;
} ic_step_args;
int ic_decode_step(const ic_step_args* a, void* stream);

/* ---- Append the K/V of the token being pushed into the staging row ------
 * k, v: [S, L, Hkv, D] in the pool dtype with the given element strides
 * (D contiguous).  Used by the reference-compatible push path
 * (hierarchical_cache.py:271-275). */
typedef struct ic_append_args {
  ic_pool pool;
  ic_tiers tiers;
  ic_sessions sess;
  const void* k;
  const void* v;
  int64_t stride_s, stride_l, stride_h;
} ic_append_args;
int ic_append_staging(const ic_append_args* a, void* stream);

/* ---- Position order of the occupied slots --------------------------------
 * sorted_slots[s, r] = the occupied slot of rank r by (position, slot index),
 * -1 past the fill; fill[s] = number of occupied slots.  Rank order is the
 * order of to_hf_past_key_values / _boost_importance
 * (hierarchical_cache.py:320-323, 441-443). */
typedef struct ic_sort_args {
  ic_tiers tiers;
  ic_sessions sess;
  int32_t* sorted_slots;   /* [S, budget] */
  int32_t* fill;           /* [S] */
} ic_sort_args;
int ic_sort_slots(const ic_sort_args* a, void* stream);

/* ---- Reference push boost: mean attention weight by position rank --------
 * weights: float [S, L, H, Q, width] (the attn_weights of push, per
 * session).  agg[r] = (sum_h sum_l sum_q w[l, h, q, r]) / (L * H * Q);
 * mass_out[s, sorted_slots[s, r]] = agg[r] for r < min(width, fill), 0 for
 * every other slot (_boost_importance, hierarchical_cache.py:427-446); use it
 * as kernel B's mass with one head and one layer. */
typedef struct ic_boost_args {
  ic_tiers tiers;
  int32_t num_sessions;
  int32_t L, H, Q, width;
  const float* weights;
  const int32_t* sorted_slots;  /* from ic_sort_slots */
  const int32_t* fill;
  float* mass_out;              /* [S, budget + 1] */
} ic_boost_args;
int ic_boost_sorted(const ic_boost_args* a, void* stream);

/* ---- Gather pool rows through the slot table ------------------------------
 * out[l - layer_begin, h, r, :] = pool[l, h, slot_table[s, slots[r]], :] for
 * r < n (slots[r] < 0 gives zeros).  With slots = sorted_slots this is
 * to_hf_past_key_values (hierarchical_cache.py:297-351) and gather_cache_kv
 * (triton_ops.py:107-135). */
typedef struct ic_gather_args {
  ic_pool pool;
  ic_tiers tiers;
  ic_sessions sess;
  int32_t session;
  int32_t n;
  const int32_t* slots;     /* [n] logical slots (device) */
  int32_t layer_begin, layer_end;
  void* k_out;              /* [layer_end - layer_begin, Hkv, n, D] */
  void* v_out;
} ic_gather_args;
int ic_gather_slots(const ic_gather_args* a, void* stream);

/* ---- Kernel D: tier fill of one prompt (load_from_hf_output) -------------
 * For sessions [session0, session0 + n): classifies the T prompt tokens into
 * sinks / recent tail / L2 candidates and streams the candidates through the
 * "replace the first-index minimum iff strictly greater" rule
 * (hierarchical_cache.py:179-237, 390-418).  Writes slot_token[i, slot] (the
 * prompt token each slot holds, -1 = empty) and resets and fills the
 * session's metadata, ctrl and counters. */
typedef struct ic_tier_fill_args {
  ic_tiers tiers;
  ic_sessions sess;
  int32_t session0;
  int32_t n;
  int32_t T;
  int32_t _pad;
  const float* scores;       /* [n, T] */
  const int64_t* positions;  /* [n, T] or NULL for arange(T) */
  int32_t* slot_token;       /* [n, budget] */
} ic_tier_fill_args;
int ic_tier_fill(const ic_tier_fill_args* a, void* stream);

/* ---- Copy prompt K/V of one layer into the slots chosen by ic_tier_fill ---
 * k_src, v_src: [Hkv, T, D] (batch row of the HF past_key_values layer) with
 * element strides (stride_h, stride_t; D contiguous), in src_dtype. */
typedef struct ic_load_layer_args {
  ic_pool pool;
  ic_tiers tiers;
  ic_sessions sess;
  int32_t session;
  int32_t layer;
  const int32_t* slot_token; /* [budget] */
  const void* k_src;
  const void* v_src;
  int64_t stride_h, stride_t;
  int32_t src_dtype;
  int32_t T;
} ic_load_layer_args;
int ic_load_layer(const ic_load_layer_args* a, void* stream);

/* ---- Reset sessions [session0, session0 + n) ------------------------------
 * positions = -1, importance = 0, occupied = 0, ctrl = {0, 0, sink, 0},
 * counters = 0; when zero_kv != 0 the session's pool rows are zeroed in all
 * layers (reset, hierarchical_cache.py:362-378). */
typedef struct ic_reset_args {
  ic_pool pool;
  ic_tiers tiers;
  ic_sessions sess;
  int32_t session0;
  int32_t n;
  int32_t zero_kv;
} ic_reset_args;
int ic_reset_sessions(const ic_reset_args* a, void* stream);

/* ---- PagePool rows by page list (PagedSessionView) ------------------------
 * gather: out[l - layer_begin, h, t, :] = pool[l, h, page_ids[t / 16] * 16 +
 * t % 16, :] for t < n_tokens (gather_session, paged_cache.py:172-200).
 * write:  pool[l, h, page_ids[(start + t) / 16] * 16 + (start + t) % 16, :] =
 * src[l, h, t, :] for t < n_tokens (write_token, :159-170, looped by
 * PagedSessionView.push, :330-363).  src strides are in elements. */
typedef struct ic_page_rows_args {
  ic_pool pool;
  const int32_t* page_ids;
  int32_t n_page_ids;
  int32_t layer_begin, layer_end;
  int32_t _pad;
  int64_t start_token;
  int64_t n_tokens;
  void* k_buf;             /* gather: out [L', H, n, D]; write: src */
  void* v_buf;
  int64_t stride_l, stride_h, stride_t;   /* of k_buf / v_buf, elements */
} ic_page_rows_args;
int ic_page_gather(const ic_page_rows_args* a, void* stream);
int ic_page_write(const ic_page_rows_args* a, void* stream);

/* The same for `count` page lists (1 <= count <= IC_PAGE_BATCH_MAX) in one
 * launch: a[i] is one session's gather or write as above.  Every descriptor
 * names the same pool and layer range; each has its own page list, token
 * range and buffers.  Replaces a host loop of gather_session /
 * to_hf_past_key_values (paged_cache.py:172-200, 365-378) or of one-token
 * pushes (:330-363) over the sessions served in one decode tick.  Writes of
 * two descriptors to the same pool row race (the caller keeps page lists
 * disjoint, as the allocator does). */
#define IC_PAGE_BATCH_MAX 32
int ic_page_gather_batch(const ic_page_rows_args* a, int32_t count, void* stream);
int ic_page_write_batch(const ic_page_rows_args* a, int32_t count, void* stream);

/* ---- Kernel C: summary-pass scorer (tcgen05 / TMEM) -----------------------
 * Causal GQA attention over a prompt, P = softmax(scale * Q K^T) with query
 * head h reading KV head h / (Hq / Hkv):
 *   out[b, h, i, :]    = sum_j P[b, h, i, j] V[b, h / G, j, :]   (if out != NULL)
 *   lse[b, h, i]       = natural-log log-sum-exp of row i
 *   head_mass[b, h, j] = sum_i P[b, h, i, j]
 *   colsum[b, j]       = sum_h head_mass[b, h, j]  (+= when accumulate != 0,
 *                        summing layers as all_layers does)
 *   importance[b, j]   = colsum[b, j] / sum_j colsum[b, j] when that total
 *                        exceeds 1e-9, else colsum (if importance != NULL)
 * the received attention mass of _attention_mass (two_pass.py:104-137),
 * computed without materialising P.  q [B, Hq, T, D], k / v [B, Hkv, T, D]
 * contiguous, fp16 or bf16 (dtype), D = 128, any T >= 1; base pointers
 * 16-byte aligned.  Float outputs are caller-allocated.  With head_mass NULL
 * only out and lse are computed (a causal prefill attention; colsum and
 * importance are then ignored). */
typedef struct ic_summary_args {
  const void* q;
  const void* k;
  const void* v;            /* may be NULL when out is NULL */
  void* out;                /* [B, Hq, T, D] (q's dtype) or NULL */
  float* lse;               /* [B, Hq, T] */
  float* head_mass;         /* [B, Hq, T] or NULL */
  float* colsum;            /* [B, T] (required with head_mass) */
  float* importance;        /* [B, T] or NULL */
  int32_t batch, num_q_heads, num_kv_heads, seq_len, head_dim;
  int32_t dtype;            /* IC_F16 or IC_BF16 */
  int32_t accumulate;
  float scale;
  int32_t* dev_status;
} ic_summary_args;
int ic_summary_score(const ic_summary_args* a, void* stream);

/* ic_summary_score without a caller-provided head_mass buffer (no
 * counterpart in the reference: an addition of this library).  For callers
 * that cannot allocate device memory -- code running while another allocator
 * holds all of the GPU's free memory, or a binding with no CUDA allocator --
 * the per-head received mass [B, Hq, T] lives in a static device array of
 * IC_SUMMARY_STATIC_MASS_MAX floats (16 MiB) that the library owns; every GPU
 * that loads the library holds it until the process exits.  The call
 * allocates nothing.  Arguments as for ic_summary_score, except: head_mass
 * must be NULL, colsum is required, and batch * num_q_heads * seq_len must
 * not exceed IC_SUMMARY_STATIC_MASS_MAX (else IC_ERR_INVALID_ARG).  The first
 * call on a device looks up the array's device address on the current device
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * All calls share the one array: calls that overlap on the GPU (other
 * streams, other host threads) race and corrupt each other's results; order
 * them on one stream.  No element needs clearing between calls: each call
 * writes every element it reads.  The outputs are undefined when dev_status
 * reports an error, and calls after a cudaDeviceReset are not supported (the
 * array's address is looked up once per device). */
#define IC_SUMMARY_STATIC_MASS_MAX 4194304
int ic_summary_score_static(const ic_summary_args* a, void* stream);

/* ---- tensor-level helpers with the triton_ops names ---------------------------
 * For callers holding plain K / V buffers and an importance vector (the fused
 * path does not use them). */

/* gather_cache_kv (triton_ops.py:107-135): out[h, f, :] = src[h, idx[f], :]
 * (zeros for an index outside [0, N)).  src strides in elements, rows
 * contiguous; rows and bases 16-byte aligned. */
typedef struct ic_index_rows_args {
  const void* src;
  void* out;                /* [H, F, D] contiguous */
  const int64_t* idx;       /* [F] */
  int64_t stride_h, stride_n;
  int32_t H, N, F, D;
  int32_t dtype;
  int32_t _pad;
} ic_index_rows_args;
int ic_index_rows(const ic_index_rows_args* a, void* stream);

/* scatter_importance (triton_ops.py:148-175): for f < min(width, n_slots),
 * importance[slots[f]] += (sum over the `rows` rows of weights[r, f]) / rows,
 * weights float [rows, width] (rows = L * H * Q). */
typedef struct ic_scatter_mass_args {
  const float* weights;
  const int64_t* slots;
  float* importance;        /* [budget] */
  int32_t rows, width, n_slots, budget;
} ic_scatter_mass_args;
int ic_scatter_mass(const ic_scatter_mass_args* a, void* stream);

/* topk_min_slot (triton_ops.py:207-235): *out_idx = start + first index of the
 * minimum of x[start, start + n) (NaN counts as smallest); *out_val its
 * value (out_val may be NULL). */
typedef struct ic_argmin_args {
  const float* x;
  int32_t start, n;
  int64_t* out_idx;
  float* out_val;
} ic_argmin_args;
int ic_argmin_range(const ic_argmin_args* a, void* stream);

/* compact_sdp_attention (triton_ops.py:251-287): out[b, h, :] =
 * softmax(scale * q[b, h, :] . K[h, slots[f], :]) V[h, slots[f], :] over f.
 * q / out [B, H, D] contiguous; K / V buffers [H, budget, D] with the given
 * element strides; D a multiple of 32 up to 256. */
typedef struct ic_compact_attn_args {
  const void* q;
  const void* k_buf;
  const void* v_buf;
  const int64_t* slots;     /* [F] */
  void* out;
  int64_t k_stride_h, k_stride_n, v_stride_h, v_stride_n;
  int32_t B, H, F, D, budget;
  int32_t dtype;
  float scale;
  int32_t _pad;
} ic_compact_attn_args;
int ic_compact_attention(const ic_compact_attn_args* a, void* stream);

/* ---- Graph (cluster-routed) cache: GraphKVCache (graph_cache.py:218-495) --
 * One slot store K/V [L, H, NS, D], NS = sink + recent + n_clusters *
 * cluster_capacity, slots ordered sinks, ring, cluster 0, cluster 1, ...;
 * head_dim 128. */
typedef struct ic_graph_state {
  void* k;
  void* v;
  int64_t* positions;       /* [NS], -1 empty */
  float* scores;            /* [n_clusters * cluster_capacity] */
  float* centroid;          /* [n_clusters, head_dim] */
  int32_t* cl_fill;         /* [n_clusters] */
  int32_t* c_count;         /* [n_clusters] tokens in each centroid */
  int32_t* ctrl;            /* [3]: sink fill, ring pointer, ring fill */
  int32_t num_layers, num_kv_heads, head_dim, dtype;
  int32_t sink_size, recent_size, n_clusters, cluster_capacity;
  float sim_threshold;
  int32_t _pad;
} ic_graph_state;

/* push (graph_cache.py:287-361) of T tokens in order, or, with reset, the
 * bulk load_from_summary (:442-467) into a cleared cache.  k_src / v_src:
 * the tokens' K/V in the cache dtype, element offsets l * stride_l +
 * h * stride_h + t * stride_t, D contiguous, rows 16-byte aligned;
 * positions int64 [T] and scores float [T] (scores may be NULL: 0) on the
 * device; slot_src int32 [NS] scratch. */
typedef struct ic_graph_push_args {
  ic_graph_state g;
  const void* k_src;
  const void* v_src;
  int64_t stride_l, stride_h, stride_t;
  const int64_t* positions;
  const float* scores;
  int32_t* slot_src;
  int32_t T;
  int32_t reset;
} ic_graph_push_args;
int ic_graph_push(const ic_graph_push_args* a, void* stream);

/* retrieve's cluster choice and token order (graph_cache.py:363-440): query
 * float [H, head_dim]; top_n > 0 selects the top_n clusters by centroid
 * similarity of the head-mean query, else those with similarity >= threshold
 * (at least the best); selected uint8 [n_clusters]; slots int32 [NS] gets
 * the retrieve order (sinks, ring by position, selected clusters by
 * position) and *count its length. */
typedef struct ic_graph_select_args {
  ic_graph_state g;
  const float* query;
  float threshold;
  int32_t top_n;
  uint8_t* selected;
  int32_t* slots;
  int32_t* count;
} ic_graph_select_args;
int ic_graph_select(const ic_graph_select_args* a, void* stream);

/* ---- mapped host buffers ------------------------------------------------------
 * The device address of page-locked host memory (cudaHostGetDevicePointer),
 * so a decode step can read q / k_new / v_new from, and write `out` to, the
 * caller's pinned host buffers directly over PCIe, with no staging copies.
 * No reference counterpart (the reference moves tensors with .to(device)).
 * IC_ERR_INVALID_ARG when `host` is not page-locked mapped memory. */
int ic_host_device_pointer(const void* host, void** device);

/* ---- bounded-wait check ------------------------------------------------------
 * Launches one thread that waits, through the same bounded mbarrier wait every
 * kernel here uses, for a barrier phase that nothing completes.  After
 * limit_ns of %globaltimer (at most 2 s) the wait gives up, ORs
 * IC_DEVFLAG_TIMEOUT into *dev_status and the kernel returns normally, so the
 * context stays usable.  Lets a caller test its handling of a device-side
 * timeout (IC_ERR_DEVICE_TIMEOUT) without a real hang.  No reference
 * counterpart (the reference has no device-side waits). */
int ic_wait_probe(int32_t* dev_status, int64_t limit_ns, void* stream);

/* ---- graph replay loop -----------------------------------------------------
 * `rounds` times, for i < n: cudaGraphLaunch(execs[i], streams[i]) (execs are
 * cudaGraphExec_t, streams cudaStream_t, as void*).  A host loop of many small
 * graph launches -- one per session range and step in a grouped host stepper
 * -- then costs no interpreter call per launch.  No reference counterpart (the
 * reference launches every kernel from Python). */
int ic_graph_replay(void* const* execs, void* const* streams, int32_t n, int32_t rounds);

/* ---- library information --------------------------------------------------*/
const char* ic_status_str(int status);
int ic_abi_version(void);
/* IC_OK when the current device is sm_100 (B200); IC_ERR_NO_DEVICE else. */
int ic_device_check(void);
/* last CUDA error string seen by the library (thread-local) */
const char* ic_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* INFERCACHE_H_ */
