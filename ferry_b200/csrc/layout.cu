// layout.cu -- the expert-parallel layout of one MoE layer for one rank,
// computed on the GPU from the planner's destinations (no host round trip).
//
// Replaces ferry/layout.py:12-75 (build_layout) and :78-94 (device_layout,
// whose blocking H2D upload disappears) plus ferry/policy.py:197-205
// (layer_slots).  Orders are the reference's:
//   send packets by (peer, local token), ids ascending inside a packet;
//   receive packets by (source peer, token) = global token order;
//   per-expert CSR of (row, col) with rows ascending inside an expert.
// The CSR position of a route is a stable counting sort by expert; inside a
// chunk of 1024 tokens it is found with per-expert token bitmasks and popc.
//
// Extra outputs drive the fused dispatch / GEMM / combine:
//   recv_token[row]  global token of receive row `row`
//   csr_pos[row, j]  route position of column j of receive row `row`
//   peer_row[t, p]   receive row of local token t at peer p (-1: no packet)
//   groups           GEMM groups: experts cached before this layer (ascending),
//                    then the experts this rank fetched (in fetch order)
//   summary          counts and this rank's fetch list, copied to the host.
#include "common.cuh"
#include "layout.cuh"

namespace ferryb {

constexpr int kLayThreads = 1024;
constexpr int kChunk = 1024;  // tokens per pass

struct LaySmem {
  uint32_t mask[kMaxExpertsL][kChunk / 32];  // expert -> token bitmask of the chunk
  int expert_count[kMaxExpertsL];            // running per-expert route count
  int starts[kMaxExpertsL + 1];
  int warp_sum[32];
  int run;                                   // running scan carry
  int fetched_rank[kMaxExpertsL];            // fetch order of expert on this rank, or -1
  int lslot[kMaxExpertsL];                   // slot of each expert of the layer on this rank
  int fetch_key[kMaxExpertsL], fetch_slot[kMaxExpertsL];
  int recv_cnt[kMaxWorldL];
  int lower_cnt[kMaxWorldL];                 // tokens of lower ranks that send to each peer
  int n_groups, n_hit, n_fetch_mine;
};

// Exclusive block scan of one int per thread (1024 threads); returns the
// exclusive prefix and writes the total to *total.
__device__ int block_scan(int v, int* warp_sum, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sum[lane];
    int wx = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wx, o);
      if (lane >= o) wx += y;
    }
    warp_sum[lane] = wx - w;  // exclusive per warp
    if (lane == 31) *total = wx;
  }
  __syncthreads();
  const int res = warp_sum[warp] + x - v;
  __syncthreads();
  return res;
}

// One token's routes, loaded with all of its loads in flight at once:
// v[j] = (destination rank + 1) << 8 | expert id.
struct TokenRoutes {
  int v[16];
};

__device__ __forceinline__ void load_routes(const uint8_t* ids, const int32_t* dest, int g, int K,
                                            TokenRoutes& r) {
#pragma unroll
  for (int j = 0; j < 16; ++j)
    if (j < K) r.v[j] = ((dest[(size_t)g * K + j] + 1) << 8) | ids[(size_t)g * K + j];
}

// Sorted ids of the token's routes that go to `peer` (ascending, insertion
// sort as in ferry/layout.py:27-33).  Returns the count.
__device__ __forceinline__ int packet_ids(const TokenRoutes& r, int K, int peer, int* out, int E,
                                          int* err) {
  int size = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (j < K && (r.v[j] >> 8) - 1 == peer) {
      const int e = r.v[j] & 0xff;
      if (e >= E) {  // never index per-expert tables with an invalid id
        atomicCAS(err, 0, DEV_BAD_INPUT);
        continue;
      }
      int pos = size;
      while (pos > 0 && out[pos - 1] > e) { out[pos] = out[pos - 1]; --pos; }
      out[pos] = e;
      ++size;
    }
  }
  return size;
}

// Optional phase timestamps of the layout (profiling aid; NULL = off).
__device__ unsigned long long* g_layout_ts = nullptr;
#define LAY_TS(k)                                                           \
  do {                                                                      \
    if (threadIdx.x == 0 && g_layout_ts) g_layout_ts[k] = globaltimer_ns(); \
  } while (0)

__global__ void __launch_bounds__(kLayThreads, 1)
    layout_kernel(const LayoutArgs a, unsigned long long* ts, const SummaryMirror mirror) {
  __shared__ LaySmem sm;
  __shared__ int total_sh;
  const int tid = threadIdx.x;
  const int R = a.world, T = a.tokens_per_rank, K = a.topk, E = a.experts, rank = a.rank;
  const int n_tok = R * T;
  LAY_TS(0);
  span_begin(ts);
  int ids_buf[16];

  // ---- fetched experts of this rank, in fetch order -----------------------
  for (int e = tid; e < E; e += blockDim.x) {
    sm.fetched_rank[e] = -1;
    sm.expert_count[e] = 0;
    sm.lslot[e] = a.layer_slot ? a.layer_slot[e] : -1;
  }
  if (tid < R) sm.recv_cnt[tid] = 0;
  __syncthreads();
  if (a.slots_row) {  // layer_slots (ferry/policy.py:197-205) from this rank's slots row
    for (int i = tid; i < a.slots_count; i += blockDim.x) {
      const int key = a.slots_row[i];
      if (key >= 0 && key / E == a.layer) sm.lslot[key % E] = i;
    }
  }
  {
    const int nf = a.n_fetches ? *a.n_fetches : 0;  // <= experts <= 1024 threads
    int mine = 0, key = 0, slot = 0;
    if (tid < nf) {
      mine = a.fetches[tid * 3 + 0] == rank;
      key = a.fetches[tid * 3 + 1];
      slot = a.fetches[tid * 3 + 2];
    }
    const int j = block_scan(mine, sm.warp_sum, &total_sh);
    if (mine) {
      sm.fetched_rank[key % E] = j;
      sm.fetch_key[j] = key;
      sm.fetch_slot[j] = slot;
      if (a.summary) {
        a.summary->fetch_keys[j] = key;
        a.summary->fetch_slots[j] = slot;
      }
    }
    if (tid == 0) {
      sm.n_fetch_mine = total_sh;
      if (a.summary) a.summary->n_fetch_mine = total_sh;
      sm.run = 0;
    }
  }
  __syncthreads();
  if (a.layer_slot == nullptr && a.slots_row == nullptr) {
    // without a slot table, fetched experts still know their slots
    for (int j = tid; j < sm.n_fetch_mine; j += blockDim.x) sm.lslot[sm.fetch_key[j] % E] = sm.fetch_slot[j];
  }
  __syncthreads();
  LAY_TS(1);

  // ---- receive rows at every peer, part 1 ---------------------------------
  // The receive row of local token t at peer p is #{g' < g : g' sends to p}
  // (g = rank * T + t): the tokens of lower ranks that send to p (counted
  // here, order-free) plus this rank's earlier tokens that send to p (their
  // packet positions, from the send side below).
  if (a.peer_row) {
    if (tid < R) sm.lower_cnt[tid] = 0;
    __syncthreads();
    for (int g0 = 0; g0 < rank * T; g0 += kChunk) {
      const int g = g0 + tid;
      unsigned peers = 0;  // bit p: token g sends to p
      if (g < rank * T) {
        TokenRoutes tr;
        load_routes(a.ids, a.dest, g, K, tr);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int d = (tr.v[j] >> 8) - 1;
          if (j < K && d >= 0 && d < R) peers |= 1u << d;
        }
      }
      for (int p = 0; p < R; ++p) {  // warp-aggregated: one shared atomic per warp and peer
        const unsigned bal = __ballot_sync(0xffffffffu, (peers >> p) & 1u);
        if ((tid & 31) == 0 && bal) atomicAdd(&sm.lower_cnt[p], __popc(bal));
      }
    }
    __syncthreads();
  }

  // ---- send side: packets by (peer, token) --------------------------------
  int sent = 0;
  for (int peer = 0; peer < R; ++peer) {
    int peer_sent = 0;
    for (int t0 = 0; t0 < T; t0 += kChunk) {
      const int t = t0 + tid;
      const int g = rank * T + t;
      int size = 0;
      if (t < T) {
        TokenRoutes tr;
        load_routes(a.ids, a.dest, g, K, tr);
        size = packet_ids(tr, K, peer, ids_buf, E, a.err);
      }
      const int has = size > 0;
      const int before = block_scan(has, sm.warp_sum, &total_sh);  // this rank's earlier packets to peer
      const int pos = sent + before;
      if (has) {
        a.send_idx[pos] = t;
        for (int j = 0; j < K; ++j) a.send_ids[(size_t)pos * K + j] = j < size ? ids_buf[j] : -1;
      }
      if (a.peer_row && t < T)
        a.peer_row[(size_t)t * R + peer] = has ? sm.lower_cnt[peer] + peer_sent + before : -1;
      sent += total_sh;
      peer_sent += total_sh;
      __syncthreads();
    }
    if (tid == 0) a.send_counts[peer] = peer_sent;
  }
  if (tid == 0) *a.n_send = sent;
  LAY_TS(2);

  // ---- receive side pass 1: receive rows, per-expert counts --------------
  int received = 0;
  for (int g0 = 0; g0 < n_tok; g0 += kChunk) {
    const int g = g0 + tid;
    int size = 0;
    if (g < n_tok) {
      TokenRoutes tr;
      load_routes(a.ids, a.dest, g, K, tr);
      size = packet_ids(tr, K, rank, ids_buf, E, a.err);
    }
    const int has = size > 0;
    const int row = received + block_scan(has, sm.warp_sum, &total_sh);
    if (has) {
      if (a.recv_token) a.recv_token[row] = g;
      for (int j = 0; j < size; ++j) atomicAdd(&sm.expert_count[ids_buf[j]], 1);
      atomicAdd(&sm.recv_cnt[g / T], 1);
    }
    received += total_sh;
    __syncthreads();
  }
  __syncthreads();
  if (tid < R) a.recv_counts[tid] = sm.recv_cnt[tid];
  // starts = exclusive scan of expert counts (E <= 256 < 1024 threads)
  {
    const int v = tid < E ? sm.expert_count[tid] : 0;
    const int ex = block_scan(v, sm.warp_sum, &total_sh);
    if (tid < E) sm.starts[tid] = ex;
    if (tid == 0) sm.starts[E] = total_sh;
  }
  __syncthreads();
  for (int e = tid; e <= E; e += blockDim.x) a.starts[e] = sm.starts[e];
  for (int e = tid; e < E; e += blockDim.x) sm.expert_count[e] = 0;  // becomes the running cursor
  __syncthreads();
  LAY_TS(3);

  // ---- receive side pass 2: CSR positions ---------------------------------
  int row_base = 0;
  for (int g0 = 0; g0 < n_tok; g0 += kChunk) {
    for (int i = tid; i < E * (kChunk / 32); i += blockDim.x) (&sm.mask[0][0])[i] = 0;
    __syncthreads();
    const int g = g0 + tid;
    int size = 0;
    if (g < n_tok) {
      TokenRoutes tr;
      load_routes(a.ids, a.dest, g, K, tr);
      size = packet_ids(tr, K, rank, ids_buf, E, a.err);
    }
    for (int j = 0; j < size; ++j) atomicOr(&sm.mask[ids_buf[j]][tid >> 5], 1u << (tid & 31));
    const int has = size > 0;
    const int row = row_base + block_scan(has, sm.warp_sum, &total_sh);
    __syncthreads();
    if (has) {
      for (int j = 0; j < K; ++j) {
        int pos = -1;
        if (j < size) {
          const int e = ids_buf[j];
          int before = __popc(sm.mask[e][tid >> 5] & ((1u << (tid & 31)) - 1u));
          for (int w = 0; w < (tid >> 5); ++w) before += __popc(sm.mask[e][w]);
          pos = sm.starts[e] + sm.expert_count[e] + before;
          a.rows[pos] = row;
          a.cols[pos] = j;
        }
        if (a.csr_pos) a.csr_pos[(size_t)row * K + j] = pos;
      }
    }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) {
      int tot = 0;
      for (int w = 0; w < kChunk / 32; ++w) tot += __popc(sm.mask[e][w]);
      sm.expert_count[e] += tot;
    }
    row_base += total_sh;
    __syncthreads();
  }
  if (tid == 0) *a.n_recv = received;
  LAY_TS(4);

  // ---- GEMM groups: cached experts (ascending), then fetched (fetch order) --
  if (a.groups && a.summary) {
    GemmGroup* groups = reinterpret_cast<GemmGroup*>(a.groups);
    const int e = tid;
    int cnt = 0, hit = 0;
    if (e < E) {
      cnt = sm.starts[e + 1] - sm.starts[e];
      hit = cnt > 0 && sm.fetched_rank[e] < 0;
      if (cnt > 0 && sm.lslot[e] < 0)
        atomicCAS(a.err, 0, DEV_NO_SLOT);  // scheduled here but not cached (ferry/layout.py:91)
    }
    const int pos = block_scan(hit, sm.warp_sum, &total_sh);
    const int n_hit = total_sh;
    if (hit) groups[pos] = GemmGroup{sm.lslot[e], sm.starts[e], cnt, e};
    if (e < E && cnt > 0 && sm.fetched_rank[e] >= 0)
      groups[n_hit + sm.fetched_rank[e]] = GemmGroup{sm.lslot[e], sm.starts[e], cnt, e};
    if (tid < 32) {
      const int p = tid;
      a.summary->send_counts[p] = p < R ? (int)a.send_counts[p] : 0;
      a.summary->recv_counts[p] = p < R ? sm.recv_cnt[p] : 0;
      a.summary->fetch_counts[p] = 0;
    }
    __syncthreads();
    const int nf_all = a.n_fetches ? *a.n_fetches : 0;
    if (tid < nf_all) {
      const int r = a.fetches[tid * 3 + 0];
      if (r >= 0 && r < 32) atomicAdd(&a.summary->fetch_counts[r], 1);
    }
    if (tid == 0) {
      a.summary->n_groups = n_hit + sm.n_fetch_mine;
      a.summary->n_hit = n_hit;
      a.summary->n_recv = received;
      a.summary->n_send = sent;
      a.summary->n_routes = sm.starts[E];
    }
    __syncthreads();
    if (tid == 0) a.summary->err = atomicAdd(a.err, 0);
  }
  __syncthreads();
  LAY_TS(5);
  if (mirror.sum && a.summary) {
    // the finished summary and the error words straight into the host's
    // mapped mirror (no copy command, no event), then the release of `seq`
    // after one system-scope fence behind a CTA barrier
    static_assert(sizeof(ferryb_layout_summary) % 16 == 0, "summary copied in 16-byte pieces");
    const uint4* src = reinterpret_cast<const uint4*>(a.summary);
    uint4* dst = reinterpret_cast<uint4*>(mirror.sum);
    for (int i = tid; i < (int)(sizeof(ferryb_layout_summary) / 16); i += blockDim.x) dst[i] = src[i];
    if (tid < 8) mirror.errs[tid] = atomicAdd(const_cast<int32_t*>(mirror.errs_dev) + tid, 0);
    __syncthreads();
    if (tid == 0) {
      __threadfence_system();
      st_release_sys(reinterpret_cast<uint64_t*>(mirror.seq), mirror.value);
    }
  }
  LAY_TS(6);
  span_end(ts);
}

// layer_slots (ferry/policy.py:197-205) for one rank's slots row.
__global__ void layer_slots_kernel(const int32_t* slots_row, int capacity, int layer, int experts,
                                   int32_t* lookup) {
  for (int e = threadIdx.x; e < experts; e += blockDim.x) lookup[e] = -1;
  __syncthreads();
  for (int i = threadIdx.x; i < capacity; i += blockDim.x) {
    const int key = slots_row[i];
    if (key >= 0 && key / experts == layer) lookup[key % experts] = i;
  }
}

int layout_launch(const LayoutArgs& a, cudaStream_t stream, unsigned long long* ts,
                  const SummaryMirror* mirror) {
  FB_CHECK_ARG(a.experts <= kMaxExpertsL && a.topk <= 16 && a.world >= 1,
               "layout: experts <= %d and topk <= 16 required", kMaxExpertsL);
  layout_kernel<<<1, kLayThreads, 0, stream>>>(a, ts, mirror ? *mirror : SummaryMirror{});
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

int layer_slots_launch(const int32_t* slots_row, int capacity, int layer, int experts,
                       int32_t* lookup, cudaStream_t stream) {
  layer_slots_kernel<<<1, 1024, 0, stream>>>(slots_row, capacity, layer, experts, lookup);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

}  // namespace ferryb

using namespace ferryb;

extern "C" int ferryb_debug_layout_timestamps(void* dev_ptr) {
  FB_CUDA(cudaMemcpyToSymbol(g_layout_ts, &dev_ptr, sizeof(void*)));
  return FERRYB_OK;
}

extern "C" int ferryb_build_layout(const ferryb_layout_args* args, cudaStream_t stream) {
  FB_CHECK_ARG(args && args->ids && args->dest && args->err, "layout: null arguments");
  FB_CHECK_ARG(args->world >= 1 && args->world <= kMaxWorldL && args->tokens_per_rank >= 0 &&
                   args->rank >= 0 && args->rank < args->world,
               "layout: bad world/rank");
  FB_CHECK_ARG(args->send_idx && args->send_ids && args->send_counts && args->recv_counts &&
                   args->starts && args->rows && args->cols && args->n_send && args->n_recv,
               "layout: build_layout outputs are required");
  return layout_launch(*args, stream);
}

extern "C" int ferryb_layer_slots(const int32_t* slots_row, int32_t capacity, int32_t layer,
                                  int32_t experts, int32_t* lookup, cudaStream_t stream) {
  FB_CHECK_ARG(slots_row && lookup && capacity >= 0 && experts > 0, "layer_slots: bad arguments");
  return layer_slots_launch(slots_row, capacity, layer, experts, lookup, stream);
}
