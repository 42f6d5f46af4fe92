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

/* ------------------------------------------------------------------------
 * EP layout of one layer for one rank.  Replaces build_layout and
 * device_layout (ferry/layout.py:12-94; no blocking H2D) and layer_slots
 * (ferry/policy.py:197-205).  Device pointers; NULL skips an optional output.
 */
typedef struct ferryb_layout_summary {
  int32_t n_fetch_mine, n_hit, n_groups, n_recv, n_send, n_routes, err, reserved;
  int32_t fetch_keys[256];  /* this rank's fetches, in fetch order */
  int32_t fetch_slots[256];
} ferryb_layout_summary;

typedef struct ferryb_layout_args {
  const uint8_t* ids;        /* [world*T, topk] */
  const int32_t* dest;       /* [world*T, topk] */
  int32_t world, tokens_per_rank, topk, experts, rank;
  const int32_t* fetches;    /* planner output or NULL */
  const int32_t* n_fetches;  /* planner output or NULL */
  const int32_t* layer_slot; /* [experts] slot of each expert on this rank, or NULL */
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

#ifdef __cplusplus
}
#endif

#endif /* FERRYB_H_ */
