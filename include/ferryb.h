/*
 * ferryb.h -- C ABI of libferryb, the B200 (sm_100a) implementation of
 * FERRY's per-MoE-layer hot path.
 *
 * Conventions
 *  - Every function returns FERRYB_OK (0) or a FERRYB_E* code; the message of
 *    the last failure on the calling thread is ferryb_last_error().
 *  - Pointers named d_* or documented as "device" are CUDA device pointers of
 *    the current device; "host" arrays are plain CPU memory.
 *  - Work is enqueued on the cudaStream_t passed in (the caller's current
 *    stream, as the reference's ATen ops use the current stream,
 *    ferry/csrc/expert_ops.cpp:126).  No entry point allocates device memory
 *    unless documented; scratch comes from a caller-provided workspace whose
 *    size a *_workspace() query returns.
 *  - bf16 means IEEE bfloat16 stored as uint16; int64 tensors are int64_t.
 *
 * Reference interfaces replaced (paths within the FERRY repository):
 *  ferry/csrc/expert_ops.cpp:144-157  pybind module ferry_expert_ops
 *  ferry/policy.py, ferry/quota.py, ferry/layout.py, ferry/metadata.py
 *  ferry/transport.py, ferry/runtime.py
 */
#ifndef FERRYB_H_
#define FERRYB_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FERRYB_VERSION 1

enum {
  FERRYB_OK = 0,
  FERRYB_EINVAL = 1,    /* bad argument (the reference's TORCH_CHECK / ValueError) */
  FERRYB_ECUDA = 2,     /* a CUDA runtime/driver call failed */
  FERRYB_EDEVICE = 3,   /* a kernel reported an error word (see ferryb_last_error) */
  FERRYB_ECAPACITY = 4, /* missing experts exceed the admission capacity
                           (the reference's assert, ferry/quota.py:63) */
  FERRYB_ETIMEOUT = 5,  /* a bounded device or host wait gave up */
  FERRYB_ESTATE = 6     /* call out of order (e.g. use after close) */
};

typedef struct CUstream_st* ferryb_stream_t; /* == cudaStream_t */

#if defined(__GNUC__)
#define FERRYB_API __attribute__((visibility("default")))
#else
#define FERRYB_API
#endif

/* Message of the last failure on this thread ("" if none). */
FERRYB_API const char* ferryb_last_error(void);
FERRYB_API int ferryb_version(void);
FERRYB_API int ferryb_device_sm_count(int device);
/* 1 if the device supports stream memory operations (cuStreamWriteValue32),
 * which the H2D engine uses to raise per-copy readiness flags. */
FERRYB_API int ferryb_stream_mem_ops_supported(int device);

/* ------------------------------------------------------------------------
 * Kernel 5: routed-expert SwiGLU grouped GEMM (tcgen05 / TMEM / TMA).
 * Replaces execute_experts, ferry/csrc/expert_ops.cpp:16-45 (and silu_mul,
 * ferry/csrc/expert_ops.cu:6-25).
 *
 * cache:           device bf16 [cache_slots, 3*hidden*intermediate], rows
 *                  [gate I x H | up I x H | down H x I] (ferry/model.py:86-88)
 * input:           device bf16 [n_input, hidden]
 * routing_weights: device bf16 [n_input, topk]
 * slots, group_sizes: host int64 [n_groups]: cache slot and route count of
 *                  each group (the reference's `slots` and len(rows[i]))
 * rows, cols:      device int64 [sum(group_sizes)], the groups' rows/cols
 *                  concatenated in group order
 * out:             device bf16 [sum(group_sizes), hidden]; group i's outputs
 *                  are rows [offset_i, offset_i + group_sizes[i]), each
 *                  (silu(x Wg^T) * (x Wu^T)) Wd^T * w[row, col]
 * workspace:       device, >= ferryb_execute_experts_workspace(...) bytes
 * Synchronises `stream` before returning to report device-side errors.
 */
FERRYB_API int64_t ferryb_execute_experts_workspace(int64_t total_routes, int64_t n_groups, int64_t hidden,
                                         int64_t intermediate);
FERRYB_API int ferryb_execute_experts(const void* cache, int64_t cache_slots, const void* input,
                           int64_t n_input, const void* routing_weights, int64_t topk,
                           const int64_t* slots, const int64_t* group_sizes, int64_t n_groups,
                           const int64_t* rows, const int64_t* cols, int64_t hidden,
                           int64_t intermediate, void* out, void* workspace,
                           int64_t workspace_bytes, ferryb_stream_t stream);


/* The same computation as ferryb_execute_experts for callers that cannot
 * allocate device memory (a host that has already given the whole GPU to its
 * own memory pool, or a plugin reached through a C binding with no device
 * allocator).  No counterpart in the reference.  Its scratch is a fixed
 * 4 MiB array inside this library (ferryb_execute_experts_noalloc_limit()
 * bytes), which every process that loads the library holds on each GPU it
 * uses until exit; calls whose rows, activations and tables need more
 * return FERRYB_EINVAL.  Nothing is allocated: no cudaMalloc/cudaFree.
 * All calls share that array: calls that overlap on the GPU (other streams
 * or threads) race.  The first call on a device looks the array up
 * (cudaGetSymbolAddress) and should come before any stream capture.
 * Synchronises `stream` before returning, like ferryb_execute_experts. */
FERRYB_API int64_t ferryb_execute_experts_noalloc_limit(void);
FERRYB_API int ferryb_execute_experts_noalloc(const void* cache, int64_t cache_slots,
                                              const void* input, int64_t n_input,
                                              const void* routing_weights, int64_t topk,
                                              const int64_t* slots, const int64_t* group_sizes,
                                              int64_t n_groups, const int64_t* rows,
                                              const int64_t* cols, int64_t hidden,
                                              int64_t intermediate, void* out,
                                              ferryb_stream_t stream);

/* ------------------------------------------------------------------------
 * Kernel 2: placement planner (one CTA, bit-exact with the reference).
 * Replaces Controller.plan -> plan_layer (ferry/policy.py:130-194, :208-228)
 * with _demand (:25-33), _admission_capacity (:36-46), the quota LUT and
 * greedy_quota (ferry/quota.py:25-67), load_balanced_assignment
 * (ferry/policy.py:49-106), the RANDOM draw (:160-170) and _choose_slot
 * (:109-127); optionally GateHistory.update/scores (ferry/metadata.py:24-38)
 * on device state.
 *
 * All pointers are device pointers owned by the caller.  State arrays persist
 * across calls (the reference's Controller.slots/owner/last/scores and the
 * GateHistory ring); reset = fill slots/owner with -1, last/scores/ring and
 * hist_count/hist_head with 0.
 */
typedef struct ferryb_planner {
  int32_t world, experts, layers, topk, window, policy; /* policy 0 = FERRY, 1 = RANDOM */
  int64_t balance_tol_bps, salt;
  int32_t maxcap, total_slots, n_domains, lut_rows;
  const int32_t* capacities; /* [world] cache slots per rank */
  const int32_t* slot_rank;  /* [total_slots] rank of each flattened slot */
  const int32_t* slot_index; /* [total_slots] rank * maxcap + i */
  const int64_t* lut;        /* [lut_rows, world] quota lookup table */
  const int64_t* masks;      /* [n_domains] bandwidth-domain rank masks */
  const double* seconds;     /* [n_domains] 1 / bandwidth */
  int32_t* slots;            /* [world, maxcap] cached key per slot, -1 empty */
  int32_t* owner;            /* [layers * experts] rank caching each key, -1 none */
  int64_t* last;             /* [layers * experts] last-use tick */
  float* scores;             /* [layers, experts] eviction scores */
  uint8_t* ring;             /* [layers, window, topk] frequency history ids */
  float* ring_p;             /* [layers, window, experts] probability history, or NULL */
  int32_t* hist_count;       /* [layers] */
  int32_t* hist_head;        /* [layers] */
  /* The saved victim order (slot records sorted by eviction key as of the
   * last planned layer), updated incrementally from one layer to the next.
   * NULL = always sort every slot.  order_meta [1 + ceil(layers / 64)] int64:
   * a valid flag, then a bitmask of the layers whose records changed since
   * the order was saved; zero it whenever the state above is changed by
   * anything but ferryb_plan_layer (a reset), which makes the next call sort
   * every slot again.  order_rec: order_cap * 20 bytes, order_cap >= the
   * power of two >= max(64, total_slots). */
  int64_t* order_meta;
  uint8_t* order_rec;
  int32_t order_cap;
} ferryb_planner;

/* ids: [n_tokens, topk] uint8 gathered expert ids (rank-major when origins is
 * NULL, tokens_per_rank tokens per rank).  gate_scores: [experts] float32, or
 * NULL to update and read the device GateHistory (frequency rows from ids, or
 * prob_rows [n_prob_rows, experts] in probability mode).
 * Outputs: fetches [experts, 3] (rank, key, slot) in miss order, n_fetches
 * [1], dest [n_tokens, topk] owner rank of every route, counts [world].
 * err [1] receives a FERRYB device code (4 = capacity exceeded, the
 * reference's assert).  Asynchronous on `stream`. */
FERRYB_API int ferryb_plan_layer(const ferryb_planner* planner, int64_t event, int32_t layer,
                                 const uint8_t* ids, int32_t n_tokens, int32_t tokens_per_rank,
                                 const int64_t* origins, const float* gate_scores,
                                 const float* prob_rows, int32_t n_prob_rows, int32_t* fetches,
                                 int32_t* n_fetches, int32_t* dest, int32_t* counts, int32_t* err,
                                 ferryb_stream_t stream);

/* ---- the planner's steps one by one (device pointers) ------------------ */

/* greedy_quota (ferry/quota.py:25-67) for every m in [m_begin, m_end):
 * quota_out[m - m_begin, world].  capacity [world] or NULL for unlimited,
 * which makes the rows build_lut's table (ferry/quota.py:70-74).  err gets 4
 * where the reference asserts (missing experts exceed the capacity). */
FERRYB_API int ferryb_greedy_quota_rows(int32_t world, const int64_t* masks, const double* seconds,
                                        int32_t n_domains, const int32_t* capacity,
                                        int32_t m_begin, int32_t m_end, int64_t* quota_out,
                                        int32_t* err, ferryb_stream_t stream);

/* _demand (ferry/policy.py:25-33): demand [experts, world] int64. */
FERRYB_API int ferryb_demand(const int64_t* selected, const int64_t* origins, int32_t n_tokens,
                             int32_t topk, int32_t experts, int32_t world, int64_t* demand,
                             int32_t* err, ferryb_stream_t stream);

/* _admission_capacity (ferry/policy.py:36-46): u [world] int64. */
FERRYB_API int ferryb_admission_capacity(const int32_t* slots, int32_t maxcap,
                                         const int32_t* capacities, int32_t world, int32_t layer,
                                         const uint8_t* active, int32_t experts, int64_t* u,
                                         ferryb_stream_t stream);

/* load_balanced_assignment (ferry/policy.py:49-106): answer [m] int64. */
FERRYB_API int ferryb_load_balanced_assignment(const int64_t* demand, int32_t experts,
                                               int32_t world, const int64_t* misses, int32_t m,
                                               const int32_t* owner, int32_t layer,
                                               const int64_t* quota, int64_t balance_tol_bps,
                                               int64_t* answer, ferryb_stream_t stream);

/* _choose_slot (ferry/policy.py:109-127): result [1] slot index or -1. */
FERRYB_API int ferryb_choose_slot(int32_t rank, int32_t layer, const uint8_t* active,
                                  const int32_t* slots, int32_t maxcap, const int32_t* capacities,
                                  const int64_t* last, const float* scores, int32_t experts,
                                  int64_t* result, ferryb_stream_t stream);

/* Profiling aid: when dev_ptr (device, 16 x uint64) is not NULL the planner
 * writes %globaltimer stamps of its phases there (0 start, 1 gate scores,
 * 2 demand/misses/capacity, 3 quota + assignment, 4 victim records, 5 sort,
 * 6 commit, 7 end; in the incremental victim order 8 saved entries read and
 * classified, 9 clean/dirty split, 10 dirty records sorted, 11 merged) and
 * at 12 the number of dirty records.  NULL turns it off. */
FERRYB_API int ferryb_debug_plan_timestamps(void* dev_ptr);

/* Profiling aid: the same for the layout kernel of ferryb_layer_forward and
 * ferryb_build_layout (7 x uint64: 0 start, 1 fetched experts, 2 send side,
 * 3 receive pass 1 + expert starts, 4 receive pass 2, 5 GEMM groups and the
 * summary, 6 end after the host mirror's release).  NULL turns it off. */
FERRYB_API int ferryb_debug_layout_timestamps(void* dev_ptr);

/* Profiling aid: the router kernel of ferryb_layer_forward over all its CTAs
 * (4 x uint64, set to {UINT64_MAX, 0, 0, 0} before the launch): 0 earliest
 * start, 1 latest end of the logits, 2 latest end of the softmax and top-k,
 * 3 latest end.  NULL turns it off. */
FERRYB_API int ferryb_debug_router_timestamps(void* dev_ptr);

/* ------------------------------------------------------------------------
 * EP layout of one layer for one rank.  Replaces build_layout and
 * device_layout (ferry/layout.py:12-94; no blocking H2D) and layer_slots
 * (ferry/policy.py:197-205).  Device pointers; NULL skips an optional output.
 */
typedef struct ferryb_layout_summary {
  int32_t n_fetch_mine, n_hit, n_groups, n_recv, n_send, n_routes, err, reserved;
  int32_t fetch_keys[256];  /* this rank's fetches, in fetch order */
  int32_t fetch_slots[256];
  int32_t send_counts[32];  /* packets this rank sends to each peer */
  int32_t recv_counts[32];  /* packets this rank receives from each peer */
  int32_t fetch_counts[32]; /* fetches of every rank this layer (the planner's counts) */
} ferryb_layout_summary;

typedef struct ferryb_layout_args {
  const uint8_t* ids;        /* [world*T, topk] */
  const int32_t* dest;       /* [world*T, topk] */
  int32_t world, tokens_per_rank, topk, experts, rank;
  const int32_t* fetches;    /* planner output or NULL */
  const int32_t* n_fetches;  /* planner output or NULL */
  const int32_t* layer_slot; /* [experts] slot of each expert on this rank, or NULL */
  const int32_t* slots_row;  /* this rank's cache slots (computes layer_slot in-kernel), or NULL */
  int32_t slots_count, layer;
  int64_t* send_idx;         /* [T*world] */
  int64_t* send_ids;         /* [T*world, topk], -1 padded */
  int64_t* send_counts;      /* [world] */
  int64_t* recv_counts;      /* [world] */
  int64_t* starts;           /* [experts+1] */
  int64_t* rows;             /* [world*T*topk] */
  int64_t* cols;             /* [world*T*topk] */
  int32_t* n_send;           /* [1] */
  int32_t* n_recv;           /* [1] */
  int32_t* recv_token;       /* [world*T] global token of each receive row (optional) */
  int32_t* csr_pos;          /* [world*T, topk] route position of (row, col) (optional) */
  int32_t* peer_row;         /* [T, world] receive row of local token t at peer p (optional) */
  void* groups;              /* [experts] x 16-byte GEMM groups (optional) */
  ferryb_layout_summary* summary; /* optional */
  int32_t* err;              /* [1] */
} ferryb_layout_args;

FERRYB_API int ferryb_build_layout(const ferryb_layout_args* args, ferryb_stream_t stream);

/* layer_slots (ferry/policy.py:197-205): lookup[e] = slot of expert e of
 * `layer` in slots_row[0:capacity], else -1.  Device pointers. */
FERRYB_API int ferryb_layer_slots(const int32_t* slots_row, int32_t capacity, int32_t layer,
                                  int32_t experts, int32_t* lookup, ferryb_stream_t stream);

/* ------------------------------------------------------------------------
 * Kernel 3: expert fetch from pinned host memory into HBM cache slots on
 * copy-engine streams.  Replaces H2DEngine (ferry/csrc/expert_ops.cpp:97-142):
 * fetch (:107-117), wait_host (:119-122), mark_used (:124-128),
 * synchronize (:130-133), copies (:135).  Adds wait_device (a compute stream
 * waits for given slots' copies without blocking the host).  Slot and key
 * arrays are host arrays.  A pool with fewer rows than keys is read
 * cyclically (row = key mod pool_rows).
 */
typedef struct ferryb_h2d ferryb_h2d;
FERRYB_API int ferryb_h2d_create(void* cache, int64_t cache_slots, int64_t row_bytes,
                                 const void* pool, int64_t pool_rows, int32_t n_streams,
                                 ferryb_h2d** out);
FERRYB_API int ferryb_h2d_fetch(ferryb_h2d* h2d, const int64_t* slots, const int64_t* keys,
                                int64_t n);
/* Fetch with device-side readiness flags (flags: device uint32, one per
 * fetch): once fetch i's copy has landed, flags[i] = value is stored by the
 * engine's flag stream (stream memory operation).  Needs
 * ferryb_stream_mem_ops_supported. */
FERRYB_API int ferryb_h2d_fetch_flagged(ferryb_h2d* h2d, const int64_t* slots, const int64_t* keys,
                                        int64_t n, uint32_t* flags, uint32_t value);
FERRYB_API int ferryb_h2d_wait_host(ferryb_h2d* h2d, const int64_t* slots, int64_t n);
FERRYB_API int ferryb_h2d_wait_device(ferryb_h2d* h2d, const int64_t* slots, int64_t n,
                                      ferryb_stream_t stream);
FERRYB_API int ferryb_h2d_mark_used(ferryb_h2d* h2d, const int64_t* slots, int64_t n,
                                    ferryb_stream_t stream);
FERRYB_API int ferryb_h2d_synchronize(ferryb_h2d* h2d);
FERRYB_API int64_t ferryb_h2d_copies(const ferryb_h2d* h2d);
FERRYB_API int ferryb_h2d_destroy(ferryb_h2d* h2d);

/* ------------------------------------------------------------------------
 * Kernel 4 (reference-compatible ops): packets and partial sums.
 * pack_dispatch (ferry/csrc/expert_ops.cpp:50-66): payload [n_packets,
 *   2*hidden + 3*topk] bytes = hidden bf16 | routing weights bf16 (one per
 *   packet id, 0 for -1 padding) | ids u8.
 * unpack_dispatch (:68-73): x [m, hidden] bf16, w [m, topk] bf16.
 * reduce_partials (:76-83): partial[r] = bf16(sum over parts rows with
 *   rows[p] == r, in part order, in float32).
 * scatter_returned (:86-92): out[t] = bf16(sum of returned rows with
 *   send_idx[p] == t, in packet order, in float32).
 * The two sums synchronise `stream` to report out-of-range indices.
 */
FERRYB_API int ferryb_pack_dispatch(const void* hidden, int64_t tokens, int64_t hidden_dim,
                                    const int64_t* selected, const void* weights, int64_t topk,
                                    const int64_t* send_idx, const int64_t* send_ids,
                                    int64_t n_packets, int64_t experts, void* payload,
                                    int32_t* err, ferryb_stream_t stream);
FERRYB_API int ferryb_unpack_dispatch(const void* raw, int64_t m, int64_t hidden_dim,
                                      int64_t topk, void* x, void* w, ferryb_stream_t stream);
FERRYB_API int64_t ferryb_segment_sum_workspace(int64_t n, int64_t n_keys);
FERRYB_API int ferryb_reduce_partials(const void* parts, const int64_t* rows, int64_t total,
                                      int64_t received, int64_t hidden_dim, void* partial,
                                      void* workspace, int64_t workspace_bytes,
                                      ferryb_stream_t stream);
FERRYB_API int ferryb_scatter_returned(const void* returned, const int64_t* send_idx, int64_t n,
                                       int64_t tokens, int64_t hidden_dim, void* out,
                                       void* workspace, int64_t workspace_bytes,
                                       ferryb_stream_t stream);

/* ------------------------------------------------------------------------
 * Symmetric device buffers for the P2P transport: ferryb_symm_alloc
 * allocates (cudaMalloc, zeroed) and exports a 64-byte CUDA IPC handle
 * (handle_out NULL: no export, single rank); peers map it with ferryb_symm_open.  Replaces the process-group plumbing of the
 * reference's all-to-all (ferry/transport.py:17-20).
 */
FERRYB_API int ferryb_symm_alloc(int64_t bytes, void** ptr, void* handle_out);
FERRYB_API int ferryb_symm_open(const void* handle, void** ptr);
FERRYB_API int ferryb_symm_close(void* peer_ptr);
FERRYB_API int ferryb_symm_free(void* ptr);

/* ------------------------------------------------------------------------
 * Routing metadata for callers composing their own layer flow (the fused
 * executor does this inside kernels 1-2).
 *
 * GateHistory.update / .scores (ferry/metadata.py:15-38) on device state:
 * rows [layers, window, experts] float64, count/head [layers] int64, all
 * zero initially.  update: probs [n_rows, experts] float64 (device). */
FERRYB_API int ferryb_history_update(double* rows, int64_t* count, int64_t* head, int32_t layers,
                                     int32_t window, int32_t experts, int32_t layer,
                                     const double* probs, int64_t n_rows, ferryb_stream_t stream);
/* out [experts] float32 = float32(sum of the layer's ring rows / max(1, count)) */
FERRYB_API int ferryb_history_scores(const double* rows, const int64_t* count, int32_t layers,
                                     int32_t window, int32_t experts, int32_t layer, float* out,
                                     ferryb_stream_t stream);
/* RouteGather.collect's all-gather (ferry/metadata.py:67-76) over symmetric
 * buffers: copies `bytes` of src (device) into every rank's buffer at
 * offset + rank * bytes, then stores `seq` into every rank's flag word
 * flag_offset + 8 * rank (system-scope release).  peer_bases: DEVICE array
 * [world] of the buffers' addresses as mapped in this process. */
FERRYB_API int ferryb_symm_allgather(const uint64_t* peer_bases, int32_t world, int32_t rank,
                                     int64_t offset, const void* src, int64_t bytes,
                                     int64_t flag_offset, uint64_t seq, ferryb_stream_t stream);
/* Waits (on the GPU, at most 2 s) until all `world` flag words at
 * local_base + flag_offset reach seq; on time-out sets *err (device int32) to
 * a non-zero code instead. */
FERRYB_API int ferryb_symm_wait(const void* local_base, int64_t flag_offset, int32_t world,
                                uint64_t seq, int32_t* err, ferryb_stream_t stream);

/* ------------------------------------------------------------------------
 * The fused per-layer executor.  Replaces OffloadRuntime.execute
 * (ferry/runtime.py:64-89) together with the MoE hook's router
 * (ferry/model.py:137-148).  One call runs, on this rank: router + all-gather
 * (kernel 1), planner (kernel 2, which publishes this rank's fetch list to the
 * host), this rank's fetches (kernel 3, the first issued while the layout
 * runs), layout (whose ~2 KB plan summary the host polls before the
 * dispatch), P2P dispatch (kernel 4), the
 * grouped SwiGLU (kernel 5, cached experts first, then each fetched expert as
 * soon as its copy lands) and the combine (kernel 4).  The workspace and the
 * symmetric buffer are caller-allocated (sizes from the *_bytes queries); the
 * executor allocates only a pinned host summary and CUDA events.
 */
typedef struct ferryb_layer_config {
  int32_t world, rank, tokens_per_rank, topk, experts, hidden, intermediate;
  int32_t router_mode;       /* 0: Qwen3 (bf16 logits), 1: DeepSeek-V2 (float32 logits) */
  int32_t norm_topk;         /* Qwen3 norm_topk_prob */
  float scaling;             /* DeepSeek-V2 routed_scaling_factor */
  int32_t probability_score; /* eviction score 'probability' (ferry/metadata.py:59-60) */
  int32_t timing;            /* record per-phase CUDA-event times (collected by
                                ferryb_layer_collect_timing) */
  int32_t sync_fetch;        /* 1: issue all of a layer's copies first and make the compute
                                stream wait for them before the fetched-expert GEMM (for
                                profilers that serialise GPU work, e.g. ncu); 0: the GEMM
                                waits on the device for each copy's readiness flag */
  int32_t shared_intermediate; /* > 0: dense shared-expert SwiGLU of this intermediate size
                                added to every token's output (DeepSeek-V2 shared experts,
                                transformers DeepseekV2MLP outside ferry/model.py:151-158);
                                weights per MoE layer via ferryb_layer_set_shared */
} ferryb_layer_config;

/* Counters of the executor.  `fetches` and host_wait_us take the place of
 * OffloadRuntime.fetches_per_rank (this rank's entry) and serial_wait_ns
 * (ferry/runtime.py:60-62, updated at :70 and :79-81); the per-rank and
 * decode-only splits come from ferryb_layer_last_summary's counts. */
typedef struct ferryb_layer_stats {
  int64_t layers, fetches, routes, recv_rows, dispatch_bytes, combine_bytes;
  int64_t launches;          /* kernels launched by the executor */
  int64_t hit_experts;       /* experts served from the cache without a fetch */
  int64_t hit_weight_bytes;  /* their weight bytes (algorithmic GEMM traffic) */
  int64_t timed_layers;      /* layers whose phase times are in phase_us */
  double host_wait_us;       /* host time blocked on the plan summary */
  double phase_us[5];        /* timing mode (CUDA events, collected by
                                ferryb_layer_collect_timing): route+plan,
                                layout+summary+dispatch+permute, cached-expert
                                GEMM, fetched-expert GEMMs (incl. copy waits),
                                combine */
  double host_us[6];         /* host time spent issuing each stage (steady
                                clock, every call): router+planner+layout,
                                first fetch after the summary arrives,
                                dispatch+permute, cached-expert GEMM,
                                fetched-expert GEMM + remaining fetches,
                                combine + counters */
  double copy_us[3];         /* timing mode, layers with fetches: planner end ->
                                first copy start (the fetch list's release and
                                the host round trip), first copy start -> last
                                copy end, last copy end -> combine end (the
                                compute tail) */
  double hit_gemm_kernel_us; /* timing mode: cached-expert GEMM launches timed on the device
                                clock (earliest CTA start to latest CTA end), summed */
  int64_t hit_gemm_kernel_launches;
  double dispatch_permute_us; /* timing mode: dispatch (+ peer signal) and permute, from
                                 after the host wait to the permute's end (waits for the
                                 peers' packets included) */
  double combine_store_us;    /* timing mode: the combine kernel alone (this rank's partials
                                 reduced and stored to their source ranks) */
  double kernel_us[9];        /* timing mode, device clock (earliest CTA start to latest CTA
                                 end), summed: router, planner, layout, dispatch, permute,
                                 cached-expert GEMM, fetched-expert GEMM, combine, final
                                 scatter (more than one rank); spans are recorded for the
                                 first 4096 layers after each collect, kernel_launches
                                 counts the launches summed */
  int64_t kernel_launches[9];
  int64_t hit_gemm_kernel_bytes; /* timing mode: cached-expert weight bytes of exactly the
                                    launches in hit_gemm_kernel_us (the device-clock
                                    roofline's numerator) */
} ferryb_layer_stats;

typedef struct ferryb_layer ferryb_layer;
FERRYB_API int64_t ferryb_layer_workspace_bytes(const ferryb_layer_config* cfg);
FERRYB_API int64_t ferryb_layer_symm_bytes(const ferryb_layer_config* cfg, int32_t window);
/* peer_bases: host [world] device addresses of every rank's symmetric buffer
 * as mapped in this process (its own at index rank). */
FERRYB_API int ferryb_layer_create(const ferryb_layer_config* cfg, const ferryb_planner* planner,
                                   void* cache, int64_t cache_slots, ferryb_h2d* h2d,
                                   void* symm_local, const uint64_t* peer_bases, void* workspace,
                                   int64_t workspace_bytes, ferryb_layer** out);
/* Router in the loop: hidden [T, H] bf16, gate_weight [E, H] bf16, gate_bias
 * [E] float32 or NULL; out [T, H] bf16; optional selected_out [T, K] int64
 * and weights_out [T, K] bf16. `event` counts layer invocations from 0 and
 * must advance identically on every rank. */
FERRYB_API int ferryb_layer_forward(ferryb_layer* layer, int64_t event, int32_t moe_layer,
                                    const void* hidden, const void* gate_weight,
                                    const float* gate_bias, void* out, int64_t* selected_out,
                                    void* weights_out, ferryb_stream_t stream);
/* Reference signature (ferry/runtime.py:64): routing given by the caller:
 * selected [T, K] int64, weights [T, K] bf16, probs_tail [n, E] float32
 * (probability score only, else NULL). */
FERRYB_API int ferryb_layer_execute(ferryb_layer* layer, int64_t event, int32_t moe_layer,
                                    const void* hidden, const int64_t* selected,
                                    const void* weights, const float* probs_tail,
                                    int32_t n_probs_tail, void* out, ferryb_stream_t stream);
/* Errors of the layers already enqueued.  forward/execute return after
 * enqueueing the layer, so a device error of its expert GEMM or transport
 * (a bounded wait that ran out: FERRYB_ETIMEOUT; another device error word:
 * FERRYB_EDEVICE) is reported by the next forward/execute of this executor or
 * by this call, which waits for `stream` and names the failing MoE layer.
 * The output rows of a failed layer are NaN, never a partial sum.  Errors are
 * sticky: every later call reports them until the executor is destroyed.
 * Replaces the reference's raise at the call itself (TORCH_CHECK,
 * ferry/csrc/expert_ops.cpp:20-34), which needs a host sync per op. */
FERRYB_API int ferryb_layer_status(ferryb_layer* layer, ferryb_stream_t stream);
/* Failure injection for the failure-detection tests: host-side omissions
 * only (a flag store that is never issued), so every wait that depends on it
 * runs out after wait_ns (0 = the default 2 s) and reports FERRYB_ETIMEOUT;
 * no kernel is made to fault.  No counterpart in the reference. */
#define FERRYB_HOOK_NO_READY_FLAGS 1u     /* copies raise no readiness flags: the
                                             fetched-expert GEMM's wait runs out */
#define FERRYB_HOOK_NO_DISPATCH_SIGNAL 2u /* this rank raises no dispatch flags: the
                                             owners' permute waits run out */
#define FERRYB_HOOK_NO_COMBINE_SIGNAL 4u  /* this rank raises no combine flags: the
                                             sources' final-scatter waits run out */
FERRYB_API int ferryb_layer_set_fault_hooks(ferryb_layer* layer, uint32_t hooks, uint64_t wait_ns);
FERRYB_API int ferryb_layer_get_stats(const ferryb_layer* layer, ferryb_layer_stats* out);
/* Timing mode: wait for the recorded phase events and add them to the stats. */
FERRYB_API int ferryb_layer_collect_timing(ferryb_layer* layer);
/* The plan summary of the last layer run (fetch list, per-rank counts). */
FERRYB_API int ferryb_layer_last_summary(const ferryb_layer* layer, ferryb_layout_summary* out);
FERRYB_API int ferryb_layer_reset_stats(ferryb_layer* layer);
/* Shared-expert weights of one MoE layer: device bf16 [3 * hidden *
 * shared_intermediate] laid out [gate I x H | up I x H | down H x I] (row-
 * major nn.Linear weights), or NULL to clear.  Borrowed: the caller keeps
 * them alive while the layer runs.  ferryb_layer_forward (the whole MoE
 * block) runs them on every local token while the layer's expert copies
 * stream and adds bf16(routed) + bf16(shared) into the output (a torch bf16
 * add); ferryb_layer_execute (the reference's execute, whose caller adds the
 * shared expert itself) does not. */
FERRYB_API int ferryb_layer_set_shared(ferryb_layer* layer, int32_t moe_layer, const void* weights);
FERRYB_API int ferryb_layer_destroy(ferryb_layer* layer);

#ifdef __cplusplus
}
#endif

#endif /* FERRYB_H_ */
