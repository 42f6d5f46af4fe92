// layer.cu -- the per-MoE-layer executor: one call runs FERRY's whole layer
// hot path on this rank (replaces OffloadRuntime.execute, ferry/runtime.py:64-89).
//
// Per layer, on the compute stream:
//   1  router (kernel 1): top-k, ids + histogram into every rank's gather buffer
//   2  planner (kernel 2): waits for all ranks' metadata, plans (replicated,
//      bit-exact), updates the device GateHistory and cache state
//   3  layer_slots + layout: this rank's packets, receive rows, expert CSR,
//      GEMM groups and a ~2 KB summary (fetch list, counts)
//   4  summary -> pinned host memory; the host waits for it (the only host
//      synchronisation of the layer; the reference has three)
//   5  this rank's fetches on the copy-engine streams (kernel 3)
//   6  dispatch (kernel 4): packets into the owners' receive buffers, flags
//   7  permute: routed rows into expert order (after all sources' flags)
//   8  grouped SwiGLU (kernel 5) over the experts cached before the layer,
//      then one launch per fetched expert gated by that slot's copy event
//      (the GEMM of an expert starts when its own bytes have landed)
//   9  combine + final scatter (kernel 4), output [T, H]
// The host returns after enqueueing step 9; the next layer's steps 1-3 queue
// behind it.  A layer's copies start only after its summary is on the host,
// which follows every earlier compute on the stream, so a cache slot is never
// overwritten while an earlier layer still reads it.
#include <atomic>
#include <chrono>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "experts.cuh"
#include "layout.cuh"
#include "planner.cuh"
#include "router.cuh"
#include "transport.cuh"

using namespace ferryb;

// The plan summary as the host sees it: pinned, mapped host memory filled by
// the planner (PlanMirror: this rank's fetch list, released by `plan_seq`)
// and then by the layout kernel (SummaryMirror, released by `seq`); both
// release words take the call's own value (ferryb_layer::releases).
struct HostMirror {
  ferryb_layout_summary sum;
  int32_t errs[8];
  uint64_t seq;
  // released earlier, by the planner (PlanMirror): this rank's fetch list and
  // the error words as the planner finished
  int32_t plan_n_fetch;
  int32_t plan_errs[8];
  int32_t plan_keys[256];
  int32_t plan_slots[256];
  uint64_t plan_seq;
};

struct ferryb_layer {
  ferryb_layer_config cfg{};
  ferryb_planner planner{};
  PlanConfig pc{};
  PlanState ps{};
  void* cache = nullptr;
  int64_t cache_slots = 0;
  ferryb_h2d* h2d = nullptr;
  uint8_t* symm = nullptr;
  uintptr_t* peer_base_dev = nullptr;  // inside the workspace
  SymLayout sl{};
  int prob_tail = 0;
  // workspace carve-up
  int32_t *dest, *fetches, *n_fetches, *counts, *errs, *layer_slot;
  int64_t *send_idx, *send_ids, *send_counts, *recv_counts, *starts, *rows, *cols;
  int32_t *n_send, *n_recv, *recv_token, *csr_pos, *peer_row;
  GemmGroup* groups;
  ferryb_layout_summary* summary_dev;
  __nv_bfloat16 *x_sorted, *act, *expert_out, *route_w, *weights;
  int64_t* selected;
  int* hist_local;
  unsigned* done;
  uint32_t* ready;  // [experts] copy readiness flags (monotonic sequence numbers)
  int* queue_dep;   // [2 + experts] GEMM work counter, done counter, phase-1 completions
  // shared experts (shared_intermediate > 0)
  std::vector<const void*> shared_w;  // per MoE layer, borrowed
  __nv_bfloat16 *shared_act = nullptr, *shared_out = nullptr, *shared_ones = nullptr;
  GemmGroup* shared_group = nullptr;
  // host side
  HostMirror* mirror_host = nullptr;  // pinned + mapped: the host's view of the plan summary
  HostMirror* mirror_dev = nullptr;   // the same memory as the device addresses it
  int32_t* errs_host = nullptr;  // pinned copy of the device error words (ferryb_layer_status)
  cudaEvent_t summary_ev = nullptr;  // after the layout kernel: tells a late mirror from a lost one
  // timing mode: 10 events per layer (8 on the compute stream, 2 on the copy
  // lane), recorded without host syncs and collected by
  // ferryb_layer_collect_timing
  std::vector<cudaEvent_t> tev_pool;
  std::vector<char> tev_fetched;  // per timed layer: copy-lane events recorded
  // device-clock spans of each timed layer's kernels, [kTs][kSpans][2]
  // (start initially ~0, end initially 0), in the workspace; kernel order:
  // router, planner, layout, dispatch, permute, cached GEMM, fetched GEMM,
  // combine, final scatter (more than one rank)
  static constexpr int kTs = 4096, kSpans = 9;
  unsigned long long* spans = nullptr;
  std::vector<char> ts_used;  // per timed layer: has a span slot
  std::vector<int64_t> ts_hit_bytes;  // per timed layer: its cached experts' weight bytes
  size_t tev_used = 0;
  cudaEvent_t* tev = nullptr;
  GemmMaps maps{};
  ferryb_layer_stats stats{};
  // error attribution: the last layer enqueued, and the last event whose GEMM
  // and transport error words were read back clean
  int64_t last_event = -1, clean_event = -1;
  uint64_t releases = 0;  // release values of the host mirror, one per call, never reused
  int32_t last_layer = -1;
  // failure injection (ferryb_layer_set_fault_hooks)
  uint32_t hooks = 0;
  uint64_t hook_wait_ns = 0;
};

namespace {

int64_t a256(int64_t b) { return (b + 255) & ~int64_t(255); }

struct Carve {
  int64_t off = 0;
  uint8_t* base = nullptr;
  template <class T>
  T* take(int64_t count) {
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += a256(count * (int64_t)sizeof(T));
    return p;
  }
};

int prob_tail_rows(const ferryb_layer_config& c, int window) {
  if (!c.probability_score) return 0;
  const int tail = (window + c.world - 1) / c.world;
  return tail < c.tokens_per_rank ? tail : c.tokens_per_rank;
}

SymLayout layout_of(const ferryb_layer_config& c, int window) {
  SymLayout l = sym_layout(c.world, c.tokens_per_rank, c.topk, c.hidden, c.experts);
  // probability-score tails follow the base layout
  const int tail = prob_tail_rows(c, window);
  l.half = a256(l.half) + a256((int64_t)c.world * tail * c.experts * 4);
  return l;
}

size_t prob_offset(const ferryb_layer_config& c) {
  return a256(sym_layout(c.world, c.tokens_per_rank, c.topk, c.hidden, c.experts).half);
}

template <class F>
int64_t carve_all(const ferryb_layer_config& c, uint8_t* base, F&& assign) {
  Carve cv;
  cv.base = base;
  const int64_t R = c.world, T = c.tokens_per_rank, K = c.topk, E = c.experts, H = c.hidden,
                I = c.intermediate;
  const int64_t n_tok = R * T, routes = n_tok * K;
  assign(cv, R, T, K, E, H, I, n_tok, routes);
  return cv.off;
}

}  // namespace

static int check_config(const ferryb_layer_config* c) {
  FB_CHECK_ARG(c && c->world >= 1 && c->world <= 32 && c->rank >= 0 && c->rank < c->world,
               "layer: bad world/rank");
  FB_CHECK_ARG(c->tokens_per_rank >= 1 && c->topk >= 1 && c->topk <= 16 && c->experts >= c->topk &&
                   c->experts <= 256,
               "layer: bad tokens/topk/experts");
  FB_CHECK_ARG(c->hidden % 256 == 0 && c->intermediate % 128 == 0,
               "layer: hidden must be a multiple of 256 and intermediate of 128");
  FB_CHECK_ARG(c->router_mode >= 0 && c->router_mode <= 1, "layer: router_mode must be 0 or 1");
  FB_CHECK_ARG(c->shared_intermediate >= 0 && c->shared_intermediate % 128 == 0,
               "layer: shared_intermediate must be a non-negative multiple of 128");
  return FERRYB_OK;
}

static int64_t workspace_bytes(const ferryb_layer_config& c, uint8_t* base, ferryb_layer* L) {
  return carve_all(c, base, [&](Carve& cv, int64_t R, int64_t T, int64_t K, int64_t E, int64_t H,
                                int64_t I, int64_t n_tok, int64_t routes) {
    auto dest = cv.take<int32_t>(n_tok * K);
    auto fetches = cv.take<int32_t>(E * 3);
    auto n_fetches = cv.take<int32_t>(1);
    auto counts = cv.take<int32_t>(R);
    auto errs = cv.take<int32_t>(8);
    auto layer_slot = cv.take<int32_t>(E);
    auto send_idx = cv.take<int64_t>(T * R);
    auto send_ids = cv.take<int64_t>(T * R * K);
    auto send_counts = cv.take<int64_t>(R);
    auto recv_counts = cv.take<int64_t>(R);
    auto starts = cv.take<int64_t>(E + 1);
    auto rows = cv.take<int64_t>(routes);
    auto cols = cv.take<int64_t>(routes);
    auto n_send = cv.take<int32_t>(1);
    auto n_recv = cv.take<int32_t>(1);
    auto recv_token = cv.take<int32_t>(n_tok);
    auto csr_pos = cv.take<int32_t>(n_tok * K);
    auto peer_row = cv.take<int32_t>(T * R);
    auto groups = cv.take<GemmGroup>(E);
    auto summary = cv.take<ferryb_layout_summary>(1);
    auto x_sorted = cv.take<__nv_bfloat16>(routes * H);
    auto act = cv.take<__nv_bfloat16>(routes * I);
    auto expert_out = cv.take<__nv_bfloat16>(routes * H);
    auto route_w = cv.take<__nv_bfloat16>(routes);
    auto weights = cv.take<__nv_bfloat16>(T * K);
    auto selected = cv.take<int64_t>(T * K);
    auto hist_local = cv.take<int>(E);
    auto done = cv.take<unsigned>(1);
    auto peer_base = cv.take<uintptr_t>(R);
    auto ready = cv.take<uint32_t>(2 * E);
    auto queue_dep = cv.take<int>(2 + E);
    auto spans = cv.take<unsigned long long>(2 * ferryb_layer::kTs * ferryb_layer::kSpans);
    const int64_t Is = c.shared_intermediate;
    auto shared_act = cv.take<__nv_bfloat16>(Is > 0 ? T * Is : 0);
    auto shared_out = cv.take<__nv_bfloat16>(Is > 0 ? T * H : 0);
    auto shared_ones = cv.take<__nv_bfloat16>(Is > 0 ? T : 0);
    auto shared_group = cv.take<GemmGroup>(Is > 0 ? 1 : 0);
    if (L) {
      L->dest = dest; L->fetches = fetches; L->n_fetches = n_fetches; L->counts = counts;
      L->errs = errs; L->layer_slot = layer_slot; L->send_idx = send_idx; L->send_ids = send_ids;
      L->send_counts = send_counts; L->recv_counts = recv_counts; L->starts = starts;
      L->rows = rows; L->cols = cols; L->n_send = n_send; L->n_recv = n_recv;
      L->recv_token = recv_token; L->csr_pos = csr_pos; L->peer_row = peer_row;
      L->groups = groups; L->summary_dev = summary; L->x_sorted = x_sorted; L->act = act;
      L->expert_out = expert_out; L->route_w = route_w; L->weights = weights;
      L->selected = selected; L->hist_local = hist_local; L->done = done;
      L->peer_base_dev = peer_base;
      L->ready = ready;
      L->queue_dep = queue_dep;
      L->spans = spans;
      if (Is > 0) {
        L->shared_act = shared_act; L->shared_out = shared_out; L->shared_ones = shared_ones;
        L->shared_group = shared_group;
      }
    }
  });
}

extern "C" int64_t ferryb_layer_workspace_bytes(const ferryb_layer_config* cfg) {
  if (check_config(cfg)) return -1;
  return workspace_bytes(*cfg, nullptr, nullptr);
}

extern "C" int64_t ferryb_layer_symm_bytes(const ferryb_layer_config* cfg, int32_t window) {
  if (check_config(cfg)) return -1;
  return (int64_t)layout_of(*cfg, window).half * 2;
}

static int init_layer(ferryb_layer* L, const ferryb_layer_config* cfg,
                      const ferryb_planner* planner, void* cache, int64_t cache_slots,
                      ferryb_h2d* h2d, void* symm_local, const uint64_t* peer_bases,
                      void* workspace, int64_t workspace_size);

extern "C" int ferryb_layer_create(const ferryb_layer_config* cfg, const ferryb_planner* planner,
                                   void* cache, int64_t cache_slots, ferryb_h2d* h2d,
                                   void* symm_local, const uint64_t* peer_bases, void* workspace,
                                   int64_t workspace_size, ferryb_layer** out) {
  int s = check_config(cfg);
  if (s) return s;
  FB_CHECK_ARG(planner && cache && h2d && symm_local && peer_bases && workspace && out,
               "layer_create: null argument");
  FB_CHECK_ARG(planner->world == cfg->world && planner->experts == cfg->experts &&
                   planner->topk == cfg->topk,
               "layer_create: planner and layer disagree on world/experts/topk");
  FB_CHECK_ARG(planner->capacities != nullptr, "planner not initialised");
  FB_CHECK_ARG(workspace_size >= workspace_bytes(*cfg, nullptr, nullptr),
               "layer_create: workspace too small");
  FB_CHECK_ARG((cfg->probability_score != 0) == (planner->ring_p != nullptr),
               "layer_create: probability score needs the planner's probability ring");
  {
    int device = 0;
    FB_CUDA(cudaGetDevice(&device));
    FB_CHECK_ARG(stream_mem_ops_supported(device),
                 "layer_create: the device lacks stream memory operations (cuStreamWriteValue32), "
                 "which the per-copy readiness flags need");
  }
  auto* L = new ferryb_layer();
  s = init_layer(L, cfg, planner, cache, cache_slots, h2d, symm_local, peer_bases, workspace,
                 workspace_size);
  if (s) {
    ferryb_layer_destroy(L);  // frees whatever init_layer got to
    return s;
  }
  *out = L;
  return FERRYB_OK;
}

static int init_layer(ferryb_layer* L, const ferryb_layer_config* cfg,
                      const ferryb_planner* planner, void* cache, int64_t cache_slots,
                      ferryb_h2d* h2d, void* symm_local, const uint64_t* peer_bases,
                      void* workspace, int64_t workspace_size) {
  L->cfg = *cfg;
  L->planner = *planner;
  L->cache = cache;
  L->cache_slots = cache_slots;
  L->h2d = h2d;
  L->symm = static_cast<uint8_t*>(symm_local);
  L->sl = layout_of(*cfg, planner->window);
  L->prob_tail = prob_tail_rows(*cfg, planner->window);
  workspace_bytes(*cfg, static_cast<uint8_t*>(workspace), L);
  // planner config (same derivation as ferryb_plan_layer)
  PlanConfig& c = L->pc;
  c.world = planner->world; c.experts = planner->experts; c.layers = planner->layers;
  c.topk = planner->topk; c.window = planner->window; c.policy = planner->policy;
  c.bps = planner->balance_tol_bps; c.salt = planner->salt; c.maxcap = planner->maxcap;
  c.total_slots = planner->total_slots; c.n_domains = planner->n_domains;
  c.lut_rows = planner->lut_rows; c.capacities = planner->capacities;
  c.slot_rank = planner->slot_rank; c.slot_index = planner->slot_index; c.lut = planner->lut;
  c.masks = planner->masks; c.seconds = planner->seconds;
  c.dyn_smem = plan_dyn_smem(c.experts, c.world, c.total_slots, c.n_domains, &c.sort_offset,
                             &c.greedy_offset, &c.sort_n, &c.dirty_offset);
  L->ps = plan_state(planner);
  FB_CUDA(cudaMemset(workspace, 0, (size_t)workspace_size));
  FB_CUDA(cudaMemcpy(L->peer_base_dev, peer_bases, sizeof(uint64_t) * cfg->world,
                     cudaMemcpyHostToDevice));
  {
    std::vector<unsigned long long> ts(2 * ferryb_layer::kTs * ferryb_layer::kSpans);
    for (size_t i = 0; i < ts.size() / 2; ++i) { ts[2 * i] = ~0ull; ts[2 * i + 1] = 0; }
    FB_CUDA(cudaMemcpy(L->spans, ts.data(), ts.size() * sizeof(unsigned long long),
                       cudaMemcpyHostToDevice));
  }
  L->shared_w.assign((size_t)planner->layers, nullptr);
  if (cfg->shared_intermediate > 0) {
    // one group over every local token, routing weight 1 (exact in bf16)
    std::vector<__nv_bfloat16> ones((size_t)cfg->tokens_per_rank, __float2bfloat16(1.0f));
    FB_CUDA(cudaMemcpy(L->shared_ones, ones.data(), ones.size() * sizeof(__nv_bfloat16),
                       cudaMemcpyHostToDevice));
    const GemmGroup g{0, 0, cfg->tokens_per_rank, 0};
    FB_CUDA(cudaMemcpy(L->shared_group, &g, sizeof(g), cudaMemcpyHostToDevice));
  }
  FB_CUDA(cudaHostAlloc(&L->mirror_host, sizeof(HostMirror), cudaHostAllocMapped));
  std::memset(L->mirror_host, 0, sizeof(HostMirror));
  FB_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&L->mirror_dev), L->mirror_host, 0));
  FB_CUDA(cudaHostAlloc(&L->errs_host, 8 * sizeof(int32_t), cudaHostAllocDefault));
  FB_CUDA(cudaEventCreateWithFlags(&L->summary_ev, cudaEventDisableTiming));
  const int64_t routes = (int64_t)cfg->world * cfg->tokens_per_rank * cfg->topk;
  return make_gemm_maps(&L->maps, cache, cache_slots, L->x_sorted, L->act, routes, cfg->hidden,
                        cfg->intermediate);
}

static FusedArgs fused_args(ferryb_layer* L, int parity, const __nv_bfloat16* hidden,
                            __nv_bfloat16* out) {
  const ferryb_layer_config& c = L->cfg;
  FusedArgs a{};
  a.world = c.world; a.rank = c.rank; a.tokens_per_rank = c.tokens_per_rank; a.topk = c.topk;
  a.hdim = c.hidden; a.experts = c.experts; a.parity = parity;
  a.peer_base = L->peer_base_dev;
  a.local_base = L->symm;
  a.buf_stride = L->sl.half;
  a.off_recv_x = L->sl.recv_x; a.off_recv_w = L->sl.recv_w; a.off_recv_ids = L->sl.recv_ids;
  a.off_ret = L->sl.ret; a.off_dflag = L->sl.dflag; a.off_cflag = L->sl.cflag;
  a.hidden = hidden;
  a.weights = L->weights;
  a.ids = L->symm + parity * L->sl.half + L->sl.gather_ids;
  a.dest = L->dest;
  a.peer_row = L->peer_row;
  a.rows = L->rows;
  a.cols = L->cols;
  a.n_routes_dev = &L->summary_dev->n_routes;
  a.n_recv_dev = L->n_recv;
  a.recv_token = L->recv_token;
  a.csr_pos = L->csr_pos;
  a.x_sorted = L->x_sorted;
  a.route_w = L->route_w;
  a.expert_out = L->expert_out;
  a.out = out;
  a.err = L->errs + 3;
  a.poison = L->errs + 2;
  a.wait_ns = L->hook_wait_ns;
  a.skip_signals = (int)((L->hooks >> 1) & 3u);
  return a;
}

// GEMM / transport error words ([2], [3]) as read back in `e`, for every layer
// enqueued up to L->last_event: FERRYB_OK, or FERRYB_ETIMEOUT / FERRYB_EDEVICE
// naming the layer whose kernels set them.  The words are sticky, so once a
// layer has failed every later call reports it until the runtime is reset.
static int exec_errors(ferryb_layer* L, const int32_t* e) {
  const int w = e[2] ? e[2] : e[3];
  if (!w) {
    L->clean_event = L->last_event;
    return FERRYB_OK;
  }
  const char* what =
      e[2] ? (w == DEV_WAIT_TIMEOUT ? "the expert GEMM gave up waiting for a fetched expert's copy"
                                    : "the expert GEMM reported a device error")
           : (w == DEV_WAIT_TIMEOUT ? "dispatch/combine gave up waiting for a peer rank's flags"
                                    : "dispatch/combine reported a device error");
  const int code = w == DEV_WAIT_TIMEOUT ? FERRYB_ETIMEOUT : FERRYB_EDEVICE;
  if (L->last_event == L->clean_event + 1)
    return fail(code, "MoE layer %d (event %lld): %s (device code %d); its output rows are NaN",
                L->last_layer, (long long)L->last_event, what, w);
  return fail(code, "a MoE layer between events %lld and %lld: %s (device code %d); its output "
              "rows are NaN", (long long)(L->clean_event + 1), (long long)L->last_event, what, w);
}

static int layer_forward(ferryb_layer* L, int64_t event, int32_t layer, const void* hidden,
                         const void* gate_weight, const float* gate_bias,
                         const int64_t* given_selected, const void* given_weights,
                         const float* given_probs, int32_t n_given_probs, void* out,
                         int64_t* selected_out, void* weights_out, cudaStream_t stream) {
  const ferryb_layer_config& c = L->cfg;
  FB_CHECK_ARG(layer >= 0 && layer < L->planner.layers, "layer %d out of range", layer);
  FB_CHECK_ARG(event >= 0 && event < ((int64_t)1 << 39), "event out of range");
  const int parity = (int)(event & 1);
  const uint64_t seq = (uint64_t)event + 1;
  const bool timing = c.timing != 0;
  // the shared expert belongs to the whole MoE block (forward), not to the
  // reference's execute, whose caller adds it
  const void* shared = (c.shared_intermediate > 0 && !given_selected) ? L->shared_w[layer] : nullptr;
  FB_CHECK_ARG(!shared || reinterpret_cast<uintptr_t>(hidden) % 16 == 0,
               "layer_forward: hidden must be 16-byte aligned with shared experts");
  uint8_t* half = L->symm + parity * L->sl.half;
  int64_t launches = 0;
  // the mirror's release words get a value no earlier call used: a planner
  // or layout kernel of a call that failed before observing its release may
  // still write one, and stream order puts those writes before this call's
  const uint64_t rel = ++L->releases;
  using clk = std::chrono::steady_clock;
  auto h_prev = clk::now();
  auto host_mark = [&](int stage) {
    const auto now = clk::now();
    L->stats.host_us[stage] += std::chrono::duration<double, std::micro>(now - h_prev).count();
    h_prev = now;
  };
  if (timing) {
    if (L->tev_used + 10 > L->tev_pool.size()) {
      for (int i = 0; i < 10 * 64; ++i) {
        cudaEvent_t e;
        FB_CUDA(cudaEventCreate(&e));
        L->tev_pool.push_back(e);
      }
    }
    L->tev = L->tev_pool.data() + L->tev_used;
    L->tev_used += 10;
    L->tev_fetched.push_back(0);
    L->ts_used.push_back(L->ts_used.size() < (size_t)ferryb_layer::kTs ? 1 : 0);
    L->ts_hit_bytes.push_back(0);
    FB_CUDA(cudaEventRecord(L->tev[0], stream));
  }
  // device-clock span slot k of this layer (timing mode), or null
  unsigned long long* const span_base =
      (timing && !L->ts_used.empty() && L->ts_used.back()) ? L->spans + 2 * ferryb_layer::kSpans * (L->ts_used.size() - 1) : nullptr;
  auto span_of = [&](int k) { return span_base ? span_base + 2 * k : nullptr; };

  // 1 router + all-gather
  RouterArgs ra{};
  ra.world = c.world; ra.rank = c.rank; ra.tokens_per_rank = c.tokens_per_rank; ra.topk = c.topk;
  ra.hdim = c.hidden; ra.experts = c.experts; ra.parity = parity;
  ra.mode = given_selected ? 2 : c.router_mode;
  ra.norm_topk = c.norm_topk; ra.scaling = c.scaling;
  ra.hidden = static_cast<const __nv_bfloat16*>(hidden);
  ra.gate = static_cast<const __nv_bfloat16*>(gate_weight);
  ra.bias = gate_bias;
  ra.weights = L->weights;
  ra.selected = L->selected;
  ra.hist_local = L->hist_local;
  ra.done = L->done;
  ra.given_selected = given_selected;
  ra.given_weights = static_cast<const __nv_bfloat16*>(given_weights);
  ra.given_probs = given_probs;
  ra.n_given_probs = n_given_probs;
  ra.prob_tail = L->prob_tail;
  ra.peer_base = L->peer_base_dev;
  ra.buf_stride = L->sl.half;
  ra.off_ids = L->sl.gather_ids;
  ra.off_hist = L->sl.gather_hist;
  ra.off_flag = L->sl.gflag;
  ra.off_prob = prob_offset(c);
  ra.ts = span_of(0);
  int s = router_launch(ra, seq, stream);
  if (s) return s;
  launches += 1;

  // 2 planner
  PlanInputs in{};
  in.ids = half + L->sl.gather_ids;
  in.n_tokens = c.world * c.tokens_per_rank;
  in.tokens_per_rank = c.tokens_per_rank;
  in.prob_rows = L->prob_tail ? reinterpret_cast<const float*>(half + prob_offset(c)) : nullptr;
  in.n_prob_rows = c.world * L->prob_tail;
  in.event = event;
  in.layer = layer;
  in.gflags = c.world > 1 ? reinterpret_cast<const uint64_t*>(half + L->sl.gflag) : nullptr;
  in.seq = seq;
  // one rank: the router's own histogram, which the planner also clears
  in.hist = c.world > 1 ? reinterpret_cast<const int*>(half + L->sl.gather_hist) : L->hist_local;
  in.hist_clear = c.world > 1 ? nullptr : L->hist_local;
  in.ts = span_of(1);
  PlanOutputs po{L->fetches, L->n_fetches, L->dest, L->counts, L->errs + 0};
  po.mirror = PlanMirror{&L->mirror_dev->plan_n_fetch, L->mirror_dev->plan_keys,
                         L->mirror_dev->plan_slots, L->mirror_dev->plan_errs, L->errs,
                         &L->mirror_dev->plan_seq, rel, c.rank};
  if ((s = plan_launch(L->pc, L->ps, in, po, stream, /*after_router=*/true))) return s;
  launches += 1;
  if (timing) FB_CUDA(cudaEventRecord(L->tev[1], stream));  // the critical path ends here

  // 3 layer slots + layout
  ferryb_layout_args la{};
  la.ids = in.ids; la.dest = L->dest;
  la.world = c.world; la.tokens_per_rank = c.tokens_per_rank; la.topk = c.topk;
  la.experts = c.experts; la.rank = c.rank;
  la.fetches = L->fetches; la.n_fetches = L->n_fetches; la.layer_slot = nullptr;
  // layer_slots in-kernel; slots past a rank's capacity are never filled, so
  // scanning maxcap slots is exact
  la.slots_row = L->planner.slots + (size_t)c.rank * L->planner.maxcap;
  la.slots_count = L->planner.maxcap;
  la.layer = layer;
  la.send_idx = L->send_idx; la.send_ids = L->send_ids; la.send_counts = L->send_counts;
  la.recv_counts = L->recv_counts; la.starts = L->starts; la.rows = L->rows; la.cols = L->cols;
  la.n_send = L->n_send; la.n_recv = L->n_recv; la.recv_token = L->recv_token;
  la.csr_pos = L->csr_pos; la.peer_row = L->peer_row; la.groups = L->groups;
  la.summary = L->summary_dev; la.err = L->errs + 1;
  const SummaryMirror mirror{&L->mirror_dev->sum, L->mirror_dev->errs, &L->mirror_dev->seq, L->errs,
                             rel};
  if ((s = layout_launch(la, stream, span_of(2), &mirror))) return s;
  launches += 1;  // layout

  // 4 the fetch list, then the layout summary, reach the host through the
  //   mapped mirror: the host polls each release word, checking the event
  //   behind the layout kernel now and then so that a launch that failed is
  //   reported instead of waited for (the planner runs before the layout, so
  //   a completed event with no release means the word was never written)
  FB_CUDA(cudaEventRecord(L->summary_ev, stream));
  host_mark(0);
  auto wait_release = [&](const uint64_t* word, const char* what) -> int {
    const volatile uint64_t* flag = word;
    for (uint32_t spins = 1; *flag != rel; ++spins) {
      if ((spins & 255) != 0) continue;
      const cudaError_t q = cudaEventQuery(L->summary_ev);
      if (q == cudaErrorNotReady) continue;
      if (q != cudaSuccess) return fail(FERRYB_ECUDA, "layer %d: %s", layer, cudaGetErrorString(q));
      if (*flag != rel)
        return fail(FERRYB_EDEVICE, "layer %d (event %lld): the %s was not written", layer,
                    (long long)event, what);
    }
    std::atomic_thread_fence(std::memory_order_acquire);
    const auto now = clk::now();
    L->stats.host_wait_us += std::chrono::duration<double, std::micro>(now - h_prev).count();
    h_prev = now;
    return FERRYB_OK;
  };
  // error words: [0] planner, [1] layout (this layer), [2] GEMM, [3] transport
  // (the layers enqueued before this one)
  auto plan_errors = [&](const int32_t* e, int layout_err) -> int {
    int st = exec_errors(L, e);
    if (st) return st;
    const int plan_err = e[0];
    if (layout_err || plan_err) {
      if (plan_err == DEV_CAPACITY || layout_err == DEV_CAPACITY)
        return fail(FERRYB_ECAPACITY, "missing experts exceed the total admission capacity");
      if (plan_err == DEV_WAIT_TIMEOUT)
        return fail(FERRYB_ETIMEOUT, "timed out waiting for the routing metadata of a peer rank");
      return fail(FERRYB_EDEVICE, "planner/layout device error %d/%d", plan_err, layout_err);
    }
    return FERRYB_OK;
  };
  if ((s = wait_release(&L->mirror_host->plan_seq, "fetch list"))) return s;
  int32_t errs_now[8];
  std::memcpy(errs_now, L->mirror_host->plan_errs, sizeof(errs_now));
  if ((s = plan_errors(errs_now, 0))) return s;
  const int n_fetch = L->mirror_host->plan_n_fetch;
  if (n_fetch < 0 || n_fetch > c.experts)
    return fail(FERRYB_EDEVICE, "layer %d: the planner reported %d fetches", layer, n_fetch);
  // 5 fetches on the copy engine, each raising a readiness flag when it has
  //   landed; the first goes out before the compute-stream launches
  std::vector<int64_t> fslots(n_fetch), fkeys(n_fetch);
  for (int i = 0; i < n_fetch; ++i) {
    fslots[i] = L->mirror_host->plan_slots[i];
    fkeys[i] = L->mirror_host->plan_keys[i];
  }
  const uint32_t ready_value = (uint32_t)seq;
  // failure injection: copies that never raise their readiness flags
  const bool no_flags = (L->hooks & FERRYB_HOOK_NO_READY_FLAGS) != 0;
  // readiness per fetch: ready[j] once the gate + up rows (the phase-1 tiles'
  // operand) have landed, ready[E + j] once the whole row has; the layer's
  // last fetch is copied in two parts so that its phase-1 tiles overlap the
  // copy of its down rows
  const int64_t split = 2 * (int64_t)c.hidden * c.intermediate * 2;
  auto fetch = [&](int first, int n) {
    if (no_flags) return ferryb_h2d_fetch(L->h2d, fslots.data() + first, fkeys.data() + first, n);
    return h2d_fetch_split_flagged(L->h2d, fslots.data() + first, fkeys.data() + first, n,
                                   L->ready + first, L->ready + c.experts + first, ready_value, split,
                                   first + n == n_fetch);
  };
  if (n_fetch > 0) {
    if (timing && (s = h2d_record_event(L->h2d, L->tev[6], 0))) return s;
    if ((s = fetch(0, 1))) return s;
  }
  host_mark(1);
  // the layout has run meanwhile (the first copy is already on its way)
  if ((s = wait_release(&L->mirror_host->seq, "plan summary"))) return s;
  const ferryb_layout_summary sum = L->mirror_host->sum;
  std::memcpy(errs_now, L->mirror_host->errs, sizeof(errs_now));
  if ((s = plan_errors(errs_now, sum.err))) return s;
  if (sum.n_fetch_mine != n_fetch)
    return fail(FERRYB_EDEVICE, "layer %d: the planner listed %d fetches, the layout %d", layer,
                n_fetch, sum.n_fetch_mine);

  // 6-7 dispatch + permute
  FusedArgs fa = fused_args(L, parity, static_cast<const __nv_bfloat16*>(hidden),
                            static_cast<__nv_bfloat16*>(out));
  if (shared) fa.addend = L->shared_out;
  fa.ts_dispatch = span_of(3);
  fa.ts_permute = span_of(4);
  fa.ts_combine = span_of(7);
  fa.ts_final = span_of(8);
  if (timing) FB_CUDA(cudaEventRecord(L->tev[8], stream));
  if ((s = fused_dispatch(fa, seq, stream))) return s;
  if ((s = fused_permute(fa, seq, sum.n_routes, stream))) return s;
  launches += 2 + (c.world > 1 ? 1 : 0);  // dispatch (+ signal) + permute
  if (timing) FB_CUDA(cudaEventRecord(L->tev[2], stream));
  host_mark(2);

  // 8 grouped SwiGLU (kernel 5), both phases per launch: the experts cached
  //   before this layer (no waits), then the fetched experts, whose tiles
  //   start as their readiness flags arrive
  if ((s = swiglu_fused_launch(L->maps, L->groups, sum.n_hit, sum.n_hit, nullptr, nullptr, 0,
                               L->queue_dep,
                               L->route_w, L->act, L->expert_out, L->errs + 2, stream,
                               span_of(5), L->hook_wait_ns)))
    return s;
  if (sum.n_hit) launches += 1;
  if (shared) {  // dense shared expert on every local token, in the copies' shadow
    if ((s = swiglu_grouped(shared, 1, L->shared_group, 1, c.tokens_per_rank,
                            static_cast<const __nv_bfloat16*>(hidden), L->shared_ones,
                            L->shared_act, L->shared_out, c.hidden, c.shared_intermediate,
                            L->errs + 2, stream)))
      return s;
    launches += 2;
  }
  if (timing) FB_CUDA(cudaEventRecord(L->tev[3], stream));
  host_mark(3);
  if (c.sync_fetch) {
    // profiler-safe order: every copy is issued (and its flag raised) before
    // the fetched-expert GEMM, which the compute stream makes wait for them
    if (sum.n_fetch_mine > 1 && (s = fetch(1, sum.n_fetch_mine - 1))) return s;
    if (sum.n_fetch_mine > 0) {
      if ((s = ferryb_h2d_wait_device(L->h2d, fslots.data(), sum.n_fetch_mine, stream))) return s;
    }
  }
  // with sync_fetch the stream has already waited for every copy: no flag waits
  if ((s = swiglu_fused_launch(L->maps, L->groups + sum.n_hit, sum.n_fetch_mine, 0,
                               c.sync_fetch ? nullptr : L->ready,
                               c.sync_fetch ? nullptr : L->ready + c.experts, ready_value,
                               L->queue_dep,
                               L->route_w, L->act, L->expert_out, L->errs + 2, stream, span_of(6),
                               L->hook_wait_ns)))
    return s;
  if (sum.n_fetch_mine) launches += 1;
  if (!c.sync_fetch && sum.n_fetch_mine > 1 && (s = fetch(1, sum.n_fetch_mine - 1))) return s;
  if (timing && sum.n_fetch_mine > 0) {
    if ((s = h2d_record_event(L->h2d, L->tev[7], 1))) return s;
    L->tev_fetched.back() = 1;
  }
  if (timing) FB_CUDA(cudaEventRecord(L->tev[4], stream));
  host_mark(4);

  // 9 combine
  if ((s = fused_combine(fa, seq, sum.n_recv, stream, timing ? L->tev[9] : nullptr))) return s;
  launches += (sum.n_recv > 0 ? 1 : 0) + (c.world > 1 ? 2 : 0);  // combine (+ signal + final)
  if (timing) FB_CUDA(cudaEventRecord(L->tev[5], stream));

  if (selected_out)
    FB_CUDA(cudaMemcpyAsync(selected_out, L->selected, sizeof(int64_t) * c.tokens_per_rank * c.topk,
                            cudaMemcpyDeviceToDevice, stream));
  if (weights_out)
    FB_CUDA(cudaMemcpyAsync(weights_out, L->weights, 2 * (size_t)c.tokens_per_rank * c.topk,
                            cudaMemcpyDeviceToDevice, stream));

  L->last_event = event;
  L->last_layer = layer;
  if (timing && !L->ts_hit_bytes.empty())
    L->ts_hit_bytes.back() = (int64_t)sum.n_hit * 3 * (int64_t)c.hidden * c.intermediate * 2;
  // counters (the reference's fetches_per_rank, copies, dispatch/combine bytes)
  L->stats.layers += 1;
  L->stats.launches += launches;
  L->stats.hit_experts += sum.n_hit;
  L->stats.hit_weight_bytes += (int64_t)sum.n_hit * 3 * (int64_t)c.hidden * c.intermediate * 2;
  L->stats.fetches += sum.n_fetch_mine;
  L->stats.routes += sum.n_routes;
  L->stats.recv_rows += sum.n_recv;
  int64_t sent_remote = 0, recv_remote = 0;
  for (int p = 0; p < c.world && p < 32; ++p) {
    if (p == c.rank) continue;
    sent_remote += sum.send_counts[p];
    recv_remote += sum.recv_counts[p];
  }
  L->stats.dispatch_bytes += sent_remote * (2 * (int64_t)c.hidden + 3 * c.topk);
  L->stats.combine_bytes += recv_remote * 2 * (int64_t)c.hidden;
  host_mark(5);
  return FERRYB_OK;
}

extern "C" int ferryb_layer_collect_timing(ferryb_layer* L) {
  FB_CHECK_ARG(L, "layer_collect_timing: null argument");
  for (size_t b = 0; b + 10 <= L->tev_used; b += 10) {
    cudaEvent_t* e = L->tev_pool.data() + b;
    FB_CUDA(cudaEventSynchronize(e[5]));
    for (int i = 0; i < 5; ++i) {
      float ms = 0.0f;
      FB_CUDA(cudaEventElapsedTime(&ms, e[i], e[i + 1]));
      L->stats.phase_us[i] += ms * 1000.0;
    }
    {
      float ms = 0.0f;
      FB_CUDA(cudaEventElapsedTime(&ms, e[8], e[2]));
      L->stats.dispatch_permute_us += ms * 1000.0;
    }
    {
      float ms = 0.0f;
      FB_CUDA(cudaEventElapsedTime(&ms, e[4], e[9]));
      L->stats.combine_store_us += ms * 1000.0;
    }
    if (L->tev_fetched[b / 10]) {
      const int pairs[3][2] = {{1, 6}, {6, 7}, {7, 5}};
      for (int i = 0; i < 3; ++i) {
        float ms = 0.0f;
        FB_CUDA(cudaEventSynchronize(e[pairs[i][1]]));
        FB_CUDA(cudaEventElapsedTime(&ms, e[pairs[i][0]], e[pairs[i][1]]));
        L->stats.copy_us[i] += ms * 1000.0;
      }
    }
    L->stats.timed_layers += 1;
  }
  L->tev_fetched.clear();
  if (!L->ts_used.empty()) {
    constexpr int S = ferryb_layer::kSpans;
    std::vector<unsigned long long> ts(2 * ferryb_layer::kTs * S);
    FB_CUDA(cudaMemcpy(ts.data(), L->spans, ts.size() * sizeof(unsigned long long),
                       cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < L->ts_used.size() && i < (size_t)ferryb_layer::kTs; ++i) {
      if (!L->ts_used[i]) continue;
      for (int k = 0; k < S; ++k) {
        const unsigned long long t0 = ts[2 * (i * S + k)], t1 = ts[2 * (i * S + k) + 1];
        if (t1 < t0) continue;  // the kernel did not run in this layer
        L->stats.kernel_us[k] += (double)(t1 - t0) / 1000.0;
        L->stats.kernel_launches[k] += 1;
        if (k == 5) {
          L->stats.hit_gemm_kernel_us += (double)(t1 - t0) / 1000.0;
          L->stats.hit_gemm_kernel_launches += 1;
          L->stats.hit_gemm_kernel_bytes += L->ts_hit_bytes[i];
        }
      }
    }
    for (size_t i = 0; i < ts.size() / 2; ++i) { ts[2 * i] = ~0ull; ts[2 * i + 1] = 0; }
    FB_CUDA(cudaMemcpy(L->spans, ts.data(), ts.size() * sizeof(unsigned long long),
                       cudaMemcpyHostToDevice));
    L->ts_used.clear();
    L->ts_hit_bytes.clear();
  }
  L->tev_used = 0;
  return FERRYB_OK;
}

extern "C" int ferryb_layer_forward(ferryb_layer* L, int64_t event, int32_t layer,
                                    const void* hidden, const void* gate_weight,
                                    const float* gate_bias, void* out, int64_t* selected_out,
                                    void* weights_out, cudaStream_t stream) {
  FB_CHECK_ARG(L && hidden && gate_weight && out, "layer_forward: null argument");
  return layer_forward(L, event, layer, hidden, gate_weight, gate_bias, nullptr, nullptr, nullptr,
                       0, out, selected_out, weights_out, stream);
}

extern "C" int ferryb_layer_execute(ferryb_layer* L, int64_t event, int32_t layer,
                                    const void* hidden, const int64_t* selected,
                                    const void* weights, const float* probs_tail,
                                    int32_t n_probs_tail, void* out, cudaStream_t stream) {
  FB_CHECK_ARG(L && hidden && selected && weights && out, "layer_execute: null argument");
  FB_CHECK_ARG(!L->prob_tail || (probs_tail && n_probs_tail >= L->prob_tail),
               "layer_execute: probability score needs probs_tail rows");
  return layer_forward(L, event, layer, hidden, nullptr, nullptr, selected, weights, probs_tail,
                       n_probs_tail, out, nullptr, nullptr, stream);
}

extern "C" int ferryb_layer_set_shared(ferryb_layer* L, int32_t moe_layer, const void* weights) {
  FB_CHECK_ARG(L, "layer_set_shared: null layer");
  FB_CHECK_ARG(L->cfg.shared_intermediate > 0, "layer_set_shared: the layer was created without "
               "shared experts (shared_intermediate = 0)");
  FB_CHECK_ARG(moe_layer >= 0 && moe_layer < (int32_t)L->shared_w.size(),
               "layer_set_shared: layer %d out of range", moe_layer);
  FB_CHECK_ARG(reinterpret_cast<uintptr_t>(weights) % 16 == 0,
               "layer_set_shared: weights must be 16-byte aligned");
  L->shared_w[moe_layer] = weights;
  return FERRYB_OK;
}

extern "C" int ferryb_layer_status(ferryb_layer* L, cudaStream_t stream) {
  FB_CHECK_ARG(L, "layer_status: null argument");
  FB_CUDA(cudaMemcpyAsync(L->errs_host, L->errs, 8 * sizeof(int32_t), cudaMemcpyDeviceToHost,
                          stream));
  FB_CUDA(cudaStreamSynchronize(stream));
  return exec_errors(L, L->errs_host);
}

extern "C" int ferryb_layer_set_fault_hooks(ferryb_layer* L, uint32_t hooks, uint64_t wait_ns) {
  FB_CHECK_ARG(L, "layer_set_fault_hooks: null argument");
  FB_CHECK_ARG((hooks & ~7u) == 0, "layer_set_fault_hooks: unknown hook bits 0x%x", hooks);
  FB_CHECK_ARG(wait_ns <= 10000000000ull, "layer_set_fault_hooks: wait limit above 10 s");
  L->hooks = hooks;
  L->hook_wait_ns = wait_ns;
  return FERRYB_OK;
}

extern "C" int ferryb_layer_get_stats(const ferryb_layer* L, ferryb_layer_stats* out) {
  FB_CHECK_ARG(L && out, "layer_get_stats: null argument");
  *out = L->stats;
  return FERRYB_OK;
}

extern "C" int ferryb_layer_last_summary(const ferryb_layer* L, ferryb_layout_summary* out) {
  FB_CHECK_ARG(L && out && L->mirror_host, "layer_last_summary: null argument");
  *out = L->mirror_host->sum;
  return FERRYB_OK;
}

extern "C" int ferryb_layer_reset_stats(ferryb_layer* L) {
  FB_CHECK_ARG(L, "layer_reset_stats: null argument");
  L->stats = ferryb_layer_stats{};
  return FERRYB_OK;
}

extern "C" int ferryb_layer_destroy(ferryb_layer* L) {
  if (!L) return FERRYB_OK;
  if (L->mirror_host) cudaFreeHost(L->mirror_host);
  if (L->errs_host) cudaFreeHost(L->errs_host);
  if (L->summary_ev) cudaEventDestroy(L->summary_ev);
  for (auto e : L->tev_pool) cudaEventDestroy(e);
  delete L;
  return FERRYB_OK;
}
