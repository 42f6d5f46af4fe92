// planner.cuh -- kernel-side view of the planner's configuration and state.
#pragma once
#include <stdint.h>

#include "../../include/ferryb.h"

namespace ferryb {

constexpr int kMaxExperts = 256;  // ids travel as uint8 (ferry/metadata.py:70)
constexpr int kMaxWorld = 32;     // ranks handled by one warp's lanes

struct PlanConfig {
  int world, experts, layers, topk, window, policy;
  int64_t bps, salt;
  int maxcap, total_slots, n_domains, lut_rows;
  const int32_t* capacities;  // [world]
  const int32_t* slot_rank;   // [total_slots]
  const int32_t* slot_index;  // [total_slots] = rank * maxcap + i
  const int64_t* lut;         // [lut_rows, world]
  const int64_t* masks;       // [n_domains]
  const double* seconds;      // [n_domains]
  // derived launch geometry
  size_t dyn_smem, sort_offset, greedy_offset, dirty_offset;  // dirty_offset 0: no room
  int sort_n;
};

struct PlanState {
  int32_t* slots;   // [world, maxcap]
  int32_t* owner;   // [layers * experts]
  int64_t* last;    // [layers * experts]
  float* scores;    // [layers, experts]
  uint8_t* ring;    // [layers, window, topk]
  float* ring_p;    // [layers, window, experts] (probability score) or null
  int32_t* hist_count;
  int32_t* hist_head;
  // saved victim order (null = off): meta [1 + ceil(layers / 64)], records SoA
  int64_t* order_meta;
  uint64_t *ord_k0, *ord_k1;
  uint32_t* ord_sl;
  int order_cap;
};

// PlanState of a planner (the saved order's SoA views of order_rec).
inline PlanState plan_state(const ferryb_planner* p) {
  PlanState s{p->slots, p->owner, p->last, p->scores, p->ring, p->ring_p, p->hist_count,
              p->hist_head, nullptr, nullptr, nullptr, nullptr, 0};
  if (p->order_meta && p->order_rec && p->order_cap >= 64) {
    s.order_meta = p->order_meta;
    s.ord_k0 = reinterpret_cast<uint64_t*>(p->order_rec);
    s.ord_k1 = s.ord_k0 + p->order_cap;
    s.ord_sl = reinterpret_cast<uint32_t*>(s.ord_k1 + p->order_cap);
    s.order_cap = p->order_cap;
  }
  return s;
}

struct PlanInputs {
  const uint8_t* ids;  // [n_tokens, topk] gathered expert ids
  int n_tokens, tokens_per_rank;
  const int64_t* origins;     // [n_tokens] or null (rank-major)
  const float* gate_scores;   // [experts] or null (use the device history)
  const float* prob_rows;     // [n_prob_rows, experts] or null
  int n_prob_rows;
  int64_t event;
  int layer;
  // fused path: gathered metadata from the router kernel (optional)
  const uint64_t* gflags;  // [world] gather flags to wait for (>= seq)
  uint64_t seq;
  const int* hist;         // [world, experts] per-rank demand histograms
  int* hist_clear;         // non-null (one rank): the router's own histogram, read from
                           // `hist` and zeroed here for the next layer
  unsigned long long* ts;  // device-clock span (timing mode) or null
};

// Optional early release of one rank's fetch list into pinned, mapped host
// memory: written by the planner's last step (error paths included), so that
// the host can start that rank's copies while the layout kernel still runs.
struct PlanMirror {
  int32_t* n_fetch;         // [1] this rank's fetches
  int32_t* keys;            // [experts] their keys, in fetch order
  int32_t* slots;           // [experts] their slots (rank-relative)
  int32_t* errs;            // [8] copy of the error words errs_dev[0..7]
  const int32_t* errs_dev;  // the executor's device error words
  uint64_t* seq;            // released to `value` last (null: no release)
  uint64_t value;
  int rank;
};

struct PlanOutputs {
  int32_t* fetches;    // [experts, 3] (rank, key, slot)
  int32_t* n_fetches;  // [1]
  int32_t* dest;       // [n_tokens, topk]
  int32_t* counts;     // [world]
  int* err;            // [1]
  PlanMirror mirror;   // optional (mirror.seq null: off)
};

int plan_launch(const PlanConfig& c, const PlanState& s, const PlanInputs& in,
                const PlanOutputs& out, cudaStream_t stream, bool after_router = false);
// Dynamic shared memory of the planner: demand, the slot records, greedy
// loads and (room permitting) the dirty-record buffer of the incremental
// victim order (*dirty_off = 0 when there is no room).
size_t plan_dyn_smem(int experts, int world, int total_slots, int n_domains, size_t* sort_off,
                     size_t* greedy_off, int* sort_n, size_t* dirty_off);
size_t plan_static_smem();

}  // namespace ferryb
