// planner.cu -- kernel 2: the per-layer placement planner as one CTA on the
// GPU, bit-exact with the reference's decisions.
//
// Replaces, per MoE layer invocation (ferry/runtime.py:281-284):
//   GateHistory.update / scores        ferry/metadata.py:24-38
//   _demand                            ferry/policy.py:25-33
//   _admission_capacity                ferry/policy.py:36-46
//   quota LUT lookup + greedy_quota    ferry/policy.py:155-158, ferry/quota.py:25-67
//   load_balanced_assignment           ferry/policy.py:49-106
//   RANDOM branch (MT19937 randint)    ferry/policy.py:160-170
//   _choose_slot + commit loop         ferry/policy.py:109-127, :171-193
//
// Exactness notes.
//  * greedy_quota compares float64 makespans with 1e-12 relative tie rules;
//    products and sums use __dmul_rn/__dadd_rn (no FMA contraction) and the
//    per-rank domain sum runs g = 0..G-1 in order, as the reference does.
//  * The eviction of _choose_slot, applied once per miss in miss order, takes
//    on each rank first the empty slots in index order, then the eligible
//    slots (not holding an expert active in this layer) by ascending
//    (score, last use, key); scores and last uses do not change during the
//    commit loop and an installed slot becomes ineligible.  The planner
//    therefore sorts all slots once by (rank, class, score, last, key) and
//    hands the j-th victim of rank r to the j-th miss assigned to r.
//  * Step 3 picks, among ranks with quota left inside the tolerance window,
//    the lexicographic maximum of (d_{r,e}, -P_r, -N_r) with the lowest rank
//    winning ties -- the same rank the reference's sequential scan keeps.
//  * Gate scores are float32(float64 count / max(1, n)) (frequency) or the
//    float64 sum of the ring slots 0..W-1 in order (probability).
#include <math_constants.h>

#include <cstring>

#include "common.cuh"
#include "planner.cuh"

namespace ferryb {

constexpr int kPlanThreads = 1024;
// The incremental victim order keeps each thread's entries in registers:
// up to kMaxIncremental / kPlanThreads of them.
constexpr int kMaxIncremental = 4096;
constexpr int kIncPer = kMaxIncremental / kPlanThreads;
constexpr int kRankSort = kPlanThreads;  // dirty records sorted by counting below this

struct SlotRec {
  uint64_t k0;  // rank << 56 | class << 48 | score bits (eligible) / 0
  uint64_t k1;  // last use << 24 | key (eligible), slot index (empty)
  uint32_t slot;  // index into slots[] (rank * maxcap + i)
  uint32_t pad;
};

__device__ __forceinline__ bool rec_less(const SlotRec& a, const SlotRec& b) {
  return a.k0 < b.k0 || (a.k0 == b.k0 && a.k1 < b.k1);
}

// MT19937 as seeded by numba's np.random.seed (init_genrand) and drawn by
// np.random.randint(0, n) (masked rejection on the low bits; n == 1 draws
// nothing).  Published algorithm: Matsumoto & Nishimura (1998).
struct MT {
  uint32_t mt[624];
  int index;
  __device__ void seed(uint32_t s) {
    mt[0] = s;
    for (int i = 1; i < 624; ++i) mt[i] = 1812433253u * (mt[i - 1] ^ (mt[i - 1] >> 30)) + (uint32_t)i;
    index = 624;
  }
  __device__ uint32_t next() {
    if (index >= 624) {
      for (int i = 0; i < 624; ++i) {
        uint32_t y = (mt[i] & 0x80000000u) | (mt[(i + 1) % 624] & 0x7fffffffu);
        mt[i] = mt[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
      }
      index = 0;
    }
    uint32_t y = mt[index++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
  }
  __device__ int randint(int n) {
    if (n == 1) return 0;
    int bits = 32 - __clz(n - 1);
    uint32_t mask = bits >= 32 ? 0xffffffffu : ((1u << bits) - 1u);
    for (;;) {
      uint32_t r = next() & mask;
      if (r < (uint32_t)n) return (int)r;
    }
  }
};

struct PlanSmem {
  int demand_total[kMaxExperts];
  int active[kMaxExperts];
  int misses[kMaxExperts];
  int64_t totals[kMaxExperts];
  int order[kMaxExperts];
  int assignment[kMaxExperts];
  int victim_pos[kMaxExperts];
  int m;
  int capacity[kMaxWorld];
  int64_t quota[kMaxWorld];
  int64_t loads[kMaxWorld];
  int n_assigned[kMaxWorld];
  int seg_start[kMaxWorld + 1];
  int warp_sum[32];
  int scan_total;
  float gate[kMaxExperts];
  int owner_layer[kMaxExperts];
  int status;
  int n_mine;  // misses assigned to the mirror's rank
  MT rng;
};

__device__ __forceinline__ void set_err(int* err, int code) { atomicCAS(err, 0, code); }

// The planner's last step when a host mirror is given (every thread, on
// every exit path): this rank's fetch count and the error words next to the
// fetch list written at the commit, then the release of `seq` after one
// system-scope fence behind a CTA barrier.
__device__ void plan_release(const PlanMirror& pm, int n_mine) {
  if (pm.seq == nullptr) return;
  __syncthreads();
  if (threadIdx.x < 8) pm.errs[threadIdx.x] = atomicAdd(const_cast<int32_t*>(pm.errs_dev) + threadIdx.x, 0);
  if (threadIdx.x == 0) *pm.n_fetch = n_mine;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(pm.seq, pm.value);
  }
}

// Optional phase timestamps of the planner (profiling aid; NULL = off).
__device__ unsigned long long* g_plan_ts = nullptr;
#define PLAN_TS(k)                                              \
  do {                                                          \
    if (threadIdx.x == 0 && g_plan_ts) g_plan_ts[k] = globaltimer_ns(); \
  } while (0)

// ---------------------------------------------------------------------------
// GateHistory.update + scores for `layer` (ferry/metadata.py:24-38).
// Frequency rows come from the gathered ids: the last `tail` tokens of every
// rank, rank-major (ferry/metadata.py:57, :80-82).  Probability rows come in
// prob_rows [n_rows, E] (float32).
__device__ void history_step(const PlanConfig& c, const PlanState& s, const PlanInputs& in,
                             float* gate_out, int* cnt_scratch) {
  const int W = c.window, E = c.experts, K = c.topk;
  const int L = in.layer;
  const int T = in.tokens_per_rank;
  const int tail = min(T, (W + c.world - 1) / c.world);
  const int n_rows = in.prob_rows ? in.n_prob_rows : c.world * tail;
  int* count = s.hist_count + L;
  int* head = s.hist_head + L;
  uint8_t* ring = s.ring + (size_t)L * W * K;
  float* ring_p = s.ring_p ? s.ring_p + (size_t)L * W * E : nullptr;
  // The ring positions written by this update: replace (n >= W) or append.
  // Head and count are read once, before any thread writes them; after the
  // update the slots [0, filled) hold rows (the ring never has holes).
  const int h0 = *head, c0 = *count;
  const int filled = n_rows >= W ? W : min(W, c0 + n_rows);
  const int n = max(1, filled);
  __syncthreads();
  if (threadIdx.x == 0) {
    *head = n_rows >= W ? 0 : (h0 + n_rows) % W;
    *count = filled;
  }
  if (ring_p) {
    if (n_rows >= W) {
      // rows[-W:] -> slots 0..W-1
      for (int i = threadIdx.x; i < W * E; i += blockDim.x)
        ring_p[i] = in.prob_rows[(size_t)(n_rows - W + i / E) * E + i % E];
    } else {
      for (int i = threadIdx.x; i < n_rows * E; i += blockDim.x)
        ring_p[(size_t)((h0 + i / E) % W) * E + i % E] = in.prob_rows[i];
    }
    __syncthreads();
    // float64 sum over slots in slot order; loads batched 8 ahead
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      double acc = 0.0;
      int slot = 0;
      for (; slot + 8 <= filled; slot += 8) {
        float v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = ring_p[(size_t)(slot + q) * E + e];
#pragma unroll
        for (int q = 0; q < 8; ++q) acc = __dadd_rn(acc, (double)v[q]);
      }
      for (; slot < filled; ++slot) acc = __dadd_rn(acc, (double)ring_p[(size_t)slot * E + e]);
      gate_out[e] = __double2float_rn(__ddiv_rn(acc, (double)n));
    }
  } else {
    // frequency rows, one thread per ring slot: the slot's row is this
    // update's (copied in here) or the one it held; a row counts once for
    // each distinct id it holds (rows are 0/1 indicators)
    constexpr int kRowMax = 16;  // rows up to this long are held in registers
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt_scratch[e] = 0;
    __syncthreads();
    for (int slot = threadIdx.x; slot < W; slot += blockDim.x) {
      int row = -1;  // the row of this update that lands in `slot`
      if (n_rows >= W) {
        row = n_rows - W + slot;
      } else if ((slot - h0 + W) % W < n_rows) {
        row = (slot - h0 + W) % W;
      }
      uint8_t* dst = ring + (size_t)slot * K;
      const uint8_t* src = dst;
      if (row >= 0) src = in.ids + ((size_t)(row / tail) * T + (T - tail + row % tail)) * K;
      if (K <= kRowMax) {
        int v[kRowMax];
#pragma unroll
        for (int k = 0; k < kRowMax; ++k) v[k] = k < K ? src[k] : 0;
        if (row >= 0) {
#pragma unroll
          for (int k = 0; k < kRowMax; ++k)
            if (k < K) dst[k] = (uint8_t)v[k];
        }
        if (slot < filled) {
#pragma unroll
          for (int k = 0; k < kRowMax; ++k) {
            if (k < K) {
              bool dup = v[k] >= E;
#pragma unroll
              for (int q = 0; q < kRowMax; ++q) dup |= q < k && v[q] == v[k];
              if (!dup) atomicAdd(&cnt_scratch[v[k]], 1);
            }
          }
        }
      } else {
        if (row >= 0)
          for (int k = 0; k < K; ++k) dst[k] = src[k];
        if (slot < filled) {
          for (int k = 0; k < K; ++k) {
            const int e = dst[k];
            bool dup = e >= E;
            for (int q = 0; q < k; ++q) dup |= dst[q] == e;
            if (!dup) atomicAdd(&cnt_scratch[e], 1);
          }
        }
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      gate_out[e] = __double2float_rn(__ddiv_rn((double)cnt_scratch[e], (double)n));
  }
  __syncthreads();
}

// greedy_quota (ferry/quota.py:25-67) on one warp; lane r owns rank r.
__device__ bool greedy_quota_warp(const PlanConfig& c, int m, const int* capacity,
                                  int64_t* quota, int64_t* load /*[G] scratch*/) {
  const int lane = threadIdx.x & 31;
  const int R = c.world, G = c.n_domains;
  for (int g = lane; g < G; g += 32) load[g] = 0;
  double single = 0.0;
  if (lane < R)
    for (int g = 0; g < G; ++g)
      if (c.masks[g] == ((int64_t)1 << lane)) single = c.seconds[g];
  int64_t q = 0;
  __syncwarp();
  for (int step = 0; step < m; ++step) {
    double t = 0.0, total = 0.0, own = 0.0;
    const bool can = lane < R && q < capacity[lane];
    if (can) {
      for (int g = 0; g < G; ++g) {
        const double v = __dmul_rn((double)(load[g] + ((c.masks[g] >> lane) & 1)), c.seconds[g]);
        total = __dadd_rn(total, v);
        if (v > t) t = v;
      }
      own = __dmul_rn((double)(q + 1), single);
    }
    // Sequential tie-break scan over ranks 0..R-1 (lane 0 holds the winner).
    int best = -1;
    double best_t = CUDART_INF, best_sum = CUDART_INF, best_own = CUDART_INF;
    for (int r = 0; r < R; ++r) {
      const int cr = __shfl_sync(0xffffffffu, (int)can, r);
      const double tr = __shfl_sync(0xffffffffu, t, r);
      const double sr = __shfl_sync(0xffffffffu, total, r);
      const double orr = __shfl_sync(0xffffffffu, own, r);
      if (!cr) continue;
      bool better = false;
      if (tr < __dmul_rn(best_t, 1 - 1e-12)) {
        better = true;
      } else if (tr <= __dmul_rn(best_t, 1 + 1e-12)) {
        if (sr < __dmul_rn(best_sum, 1 - 1e-12)) better = true;
        else if (sr <= __dmul_rn(best_sum, 1 + 1e-12) && orr < __dmul_rn(best_own, 1 - 1e-12))
          better = true;
      }
      if (better) { best = r; best_t = tr; best_sum = sr; best_own = orr; }
    }
    if (best < 0) return false;
    if (lane == best) q += 1;
    __syncwarp();
    for (int g = lane; g < G; g += 32) load[g] += (c.masks[g] >> best) & 1;
    __syncwarp();
  }
  if (lane < R) quota[lane] = q;
  __syncwarp();
  return true;
}

// load_balanced_assignment (ferry/policy.py:49-106) on one warp; lane r
// owns rank r.  Loads are token counts (< 2^31), so 32-bit arithmetic is
// exact; the peak load only grows at the chosen rank, so it is kept
// incrementally.  The per-miss choice -- the lexicographic maximum of
// (d_{r,e}, -P_r, -N_r) over eligible ranks, lowest rank on ties -- is three
// warp reductions (redux.sync) and a ballot; the next miss's inputs are
// loaded while the current one is decided.  With one rank every miss goes to
// rank 0 while its quota lasts.
__device__ void assignment_warp(const PlanConfig& c, PlanSmem& sm, const int* demand /*[E*R]*/,
                                const int* owner_layer /*[E]*/) {
  const int lane = threadIdx.x & 31;
  const int R = c.world, E = c.experts, m = sm.m;
  if (R == 1) {
    const int q = (int)sm.quota[0];
    for (int oi = lane; oi < m; oi += 32) sm.assignment[sm.order[oi]] = oi < q ? 0 : -1;
    __syncwarp();
    return;
  }
  // N_r: tokens routed to experts already cached on r (owner_layer in smem).
  int load = 0;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    const int o = e < E ? owner_layer[e] : -1;
    const int d = e < E ? sm.demand_total[e] : 0;
    for (int r = 0; r < R; ++r) {
      const int v = __reduce_add_sync(0xffffffffu, o == r ? d : 0);
      if (lane == r) load += v;
    }
  }
  int remaining = lane < R ? (int)sm.quota[lane] : 0;
  int peak = __reduce_max_sync(0xffffffffu, lane < R ? load : 0);
  const int kBig = 0x7fffffff;
  int nx_i = 0, nx_total = 0, nx_a = 0;
  if (m > 0) {
    nx_i = sm.order[0];
    nx_total = (int)sm.totals[nx_i];
    nx_a = lane < R ? demand[sm.misses[nx_i] * R + lane] : 0;
  }
  for (int oi = 0; oi < m; ++oi) {
    const int i = nx_i, total = nx_total, a = nx_a;
    if (oi + 1 < m) {  // next miss's inputs, off the dependency chain
      nx_i = sm.order[oi + 1];
      nx_total = (int)sm.totals[nx_i];
      nx_a = lane < R ? demand[sm.misses[nx_i] * R + lane] : 0;
    }
    const bool has = lane < R && remaining > 0;
    const int projected = has ? max(peak, load + total) : kBig;
    const int lowest = __reduce_min_sync(0xffffffffu, projected);
    int slack = 0;
    if (c.bps > 0) {
      const int64_t q = (int64_t)lowest * c.bps / 10000;  // lowest >= 0 here
      slack = q > 1 ? (int)q : 1;
    }
    const bool eligible = has && (int64_t)projected <= (int64_t)lowest + slack;
    const int amax = __reduce_max_sync(0xffffffffu, eligible ? a : -1);
    const bool c1 = eligible && a == amax;
    const int pmin = __reduce_min_sync(0xffffffffu, c1 ? projected : kBig);
    const bool c2 = c1 && projected == pmin;
    const int lmin = __reduce_min_sync(0xffffffffu, c2 ? load : kBig);
    const unsigned win = __ballot_sync(0xffffffffu, c2 && load == lmin);
    const int best = win ? __ffs(win) - 1 : -1;
    if (lane == 0) sm.assignment[i] = best;
    if (best >= 0) {
      if (lane == best) { remaining -= 1; load += total; }
      peak = max(peak, __shfl_sync(0xffffffffu, load, best));
    }
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------
// Ascending bitonic sort of n (power of two >= 64) records (k0, k1, sl) in
// shared memory by (k0, k1).  Compare-exchanges of stride >= 64 run in shared
// memory, one pair per thread and a block barrier per stage; every stride
// <= 32 stays inside one 64-record block, which a warp sorts in registers
// (lane holds records base+lane and base+lane+32: stride 32 within the lane,
// strides 16..1 by shuffles).  Equal keys never swap, so no record is lost
// or duplicated.
struct Rec {
  uint64_t k0, k1;
  uint32_t sl;
};

__device__ __forceinline__ bool rec_lt(const Rec& a, const Rec& b) {
  return a.k0 < b.k0 || (a.k0 == b.k0 && a.k1 < b.k1);
}

__device__ __forceinline__ Rec shfl_rec(const Rec& r, int mask) {
  Rec o;
  o.k0 = __shfl_xor_sync(0xffffffffu, r.k0, mask);
  o.k1 = __shfl_xor_sync(0xffffffffu, r.k1, mask);
  o.sl = __shfl_xor_sync(0xffffffffu, r.sl, mask);
  return o;
}

// stages (size, stride) for stride = first..1 on the two records of a lane;
// idx_a = index of record a (b = idx_a + 32)
__device__ __forceinline__ void warp_stages(Rec& a, Rec& b, int idx_a, int size, int first,
                                            int lane) {
  for (int stride = first; stride > 0; stride >>= 1) {
    const bool up_a = (idx_a & size) == 0;
    const bool up_b = ((idx_a + 32) & size) == 0;
    if (stride == 32) {
      // a and b are partners (size >= 64 here, so up_a == up_b)
      const bool swap = up_a ? rec_lt(b, a) : rec_lt(a, b);
      if (swap) { const Rec t = a; a = b; b = t; }
    } else {
      const bool lower = (lane & stride) == 0;
      const Rec oa = shfl_rec(a, stride), ob = shfl_rec(b, stride);
      // the lower record of an ascending pair keeps the minimum
      const bool want_min_a = lower == up_a, want_min_b = lower == up_b;
      if (want_min_a ? rec_lt(oa, a) : rec_lt(a, oa)) a = oa;
      if (want_min_b ? rec_lt(ob, b) : rec_lt(b, ob)) b = ob;
    }
  }
}

__device__ void sort_records(uint64_t* k0, uint64_t* k1, uint32_t* sl, int n) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_warps = blockDim.x >> 5;
  // sizes 2..64 entirely inside each 64-record block
  for (int blk = warp; blk < n / 64; blk += n_warps) {
    const int ia = blk * 64 + lane, ib = ia + 32;
    Rec a{k0[ia], k1[ia], sl[ia]}, b{k0[ib], k1[ib], sl[ib]};
    for (int size = 2; size <= 64; size <<= 1) warp_stages(a, b, ia, size, size >> 1, lane);
    k0[ia] = a.k0; k1[ia] = a.k1; sl[ia] = a.sl;
    k0[ib] = b.k0; k1[ib] = b.k1; sl[ib] = b.sl;
  }
  __syncthreads();
  for (int size = 128; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride >= 64; stride >>= 1) {
      for (int i = tid; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint64_t a0 = k0[lo], b0 = k0[hi], a1 = k1[lo], b1 = k1[hi];
        const bool b_less = b0 < a0 || (b0 == a0 && b1 < a1);
        const bool a_less = a0 < b0 || (a0 == b0 && a1 < b1);
        if (up ? b_less : a_less) {
          k0[lo] = b0; k0[hi] = a0; k1[lo] = b1; k1[hi] = a1;
          const uint32_t t = sl[lo]; sl[lo] = sl[hi]; sl[hi] = t;
        }
      }
      __syncthreads();
    }
    for (int blk = warp; blk < n / 64; blk += n_warps) {
      const int ia = blk * 64 + lane, ib = ia + 32;
      Rec a{k0[ia], k1[ia], sl[ia]}, b{k0[ib], k1[ib], sl[ib]};
      warp_stages(a, b, ia, size, 32, lane);
      k0[ia] = a.k0; k1[ia] = a.k1; sl[ia] = a.sl;
      k0[ib] = b.k0; k1[ib] = b.k1; sl[ib] = b.sl;
    }
    __syncthreads();
  }
}

// Exclusive block-wide prefix sum of one int per thread; *total (shared
// memory) gets the sum, visible to every thread on return.
__device__ int plan_block_scan(int v, int* warp_sum, int* total) {
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
    const int w = lane < (int)(blockDim.x >> 5) ? warp_sum[lane] : 0;
    int wx = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wx, o);
      if (lane >= o) wx += y;
    }
    warp_sum[lane] = wx - w;
    if (lane == 31) *total = wx;
  }
  __syncthreads();
  const int res = warp_sum[warp] + x - v;
  __syncthreads();
  return res;
}

// Number of records of (k0, k1)[0, len) (ascending) that are smaller than key.
__device__ __forceinline__ int count_less(const uint64_t* k0, const uint64_t* k1, int len, uint64_t a0,
                                          uint64_t a1) {
  int lo = 0, hi = len;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    const bool less = k0[mid] < a0 || (k0[mid] == a0 && k1[mid] < a1);
    if (less) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// The eviction record of slot `idx` (rank r) holding `key` in layer L's plan:
// k0 = rank << 56 | class << 48 | score bits, k1 = last use << 24 | key;
// class 0 empty (by slot index), 1 eligible, 2 holds an expert active in L.
__device__ __forceinline__ void slot_record(const PlanConfig& c, const PlanState& s, const int* active,
                                            int r, int idx, int key, int L, uint64_t& a0, uint64_t& a1) {
  const int E = c.experts;
  uint64_t cls, lo, hi;
  if (key < 0) {
    cls = 0; lo = 0; hi = (uint64_t)(idx - r * c.maxcap);
  } else if (key / E == L && active[key % E]) {
    cls = 2; lo = 0; hi = (uint64_t)key;
  } else {
    cls = 1;
    lo = __float_as_uint(s.scores[key]);
    hi = ((uint64_t)s.last[key] << 24) | (uint64_t)key;
  }
  a0 = ((uint64_t)r << 56) | (cls << 48) | lo;
  a1 = hi;
}

__global__ void __launch_bounds__(kPlanThreads, 1)
    plan_kernel(const PlanConfig c, const PlanState s, const PlanInputs in, const PlanOutputs out) {
  extern __shared__ uint8_t dsm[];
  __shared__ PlanSmem sm;
  const int E = c.experts, R = c.world, K = c.topk;
  const int L = in.layer;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_tok = in.n_tokens;
  int* demand = reinterpret_cast<int*>(dsm);                            // [E*R]
  SlotRec* recs = reinterpret_cast<SlotRec*>(dsm + c.sort_offset);       // [sort_n]
  int64_t* greedy_load = reinterpret_cast<int64_t*>(dsm + c.greedy_offset);  // [G]

  if (tid == 0) {
    sm.status = 0;
    sm.m = 0;
    sm.n_mine = 0;
  }
  for (int i = tid; i < E * R; i += blockDim.x) demand[i] = 0;
  // launched early behind the router (programmatic dependent launch): its
  // ids and histogram are read only after this
  pdl_wait();
  PLAN_TS(0);
  span_begin(in.ts);
  // fused path: wait (bounded) until every rank's routing metadata landed
  if (tid == 0 && in.gflags && !wait_flags_bounded(in.gflags, R, in.seq, out.err))
    sm.status = DEV_WAIT_TIMEOUT;
  __syncthreads();
  if (sm.status) {
    if (tid == 0) *out.n_fetches = 0;
    plan_release(out.mirror, 0);
    return;
  }

  // -- gate scores: given, or from the device GateHistory -------------------
  if (in.gate_scores) {
    for (int e = tid; e < E; e += blockDim.x) sm.gate[e] = in.gate_scores[e];
  } else {
    history_step(c, s, in, sm.gate, sm.demand_total);  // demand_total is free until step 1
  }
  __syncthreads();
  PLAN_TS(1);
  for (int e = tid; e < E; e += blockDim.x) s.scores[(size_t)L * E + e] = sm.gate[e];

  const int base = L * E;
  // -- Step 1: demand d[e, r] ----------------------------------------------
  if (in.hist) {
    for (int i = tid; i < E * R; i += blockDim.x) demand[(i % E) * R + i / E] = in.hist[i];
    if (in.hist_clear) {
      __syncthreads();
      for (int i = tid; i < E * R; i += blockDim.x) in.hist_clear[i] = 0;
    }
  } else for (int i = tid; i < n_tok * K; i += blockDim.x) {
    const int t = i / K;
    const int e = in.ids[i];
    const int r = in.origins ? (int)in.origins[t] : t / in.tokens_per_rank;
    if (e >= E || r < 0 || r >= R) { sm.status = DEV_BAD_INPUT; continue; }
    atomicAdd(&demand[e * R + r], 1);
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    int tot = 0;
    for (int r = 0; r < R; ++r) tot += demand[e * R + r];
    sm.demand_total[e] = tot;
    sm.active[e] = tot > 0;
    sm.owner_layer[e] = s.owner[base + e];
  }
  if (tid < R) { sm.capacity[tid] = 0; sm.n_assigned[tid] = 0; }
  __syncthreads();
  // misses in ascending expert order (warp 0 ballot compaction)
  if (warp == 0) {
    int m = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const bool miss = e < E && sm.active[e] && sm.owner_layer[e] < 0;
      const unsigned bal = __ballot_sync(0xffffffffu, miss);
      if (miss) sm.misses[m + __popc(bal & ((1u << lane) - 1))] = e;
      m += __popc(bal);
    }
    if (lane == 0) sm.m = m;
  }
  // admission capacity u_r (ferry/policy.py:36-46)
  for (int i0 = 0; i0 < c.total_slots; i0 += blockDim.x) {
    const int i = i0 + tid;
    int r = -1;
    bool free_ = false;
    if (i < c.total_slots) {
      r = c.slot_rank[i];
      const int key = s.slots[c.slot_index[i]];
      free_ = key < 0 || !(key / E == L && sm.active[key % E]);
    }
    // warp-aggregated: one shared atomic per (warp, rank)
    const unsigned act = __ballot_sync(0xffffffffu, free_);
    const unsigned same = __match_any_sync(0xffffffffu, r);
    const unsigned grp = act & same;
    if (free_ && (__ffs(grp) - 1) == lane) atomicAdd(&sm.capacity[r], __popc(grp));
  }
  __syncthreads();
  PLAN_TS(2);
  const int m = sm.m;

  // -- Steps 2-3 (FERRY) or the random draw (RANDOM) ----------------------
  if (c.policy == 0) {
    if (warp == 0) {
      bool over = false;
      if (m >= c.lut_rows) {
        if (lane == 0) sm.status = DEV_BAD_INPUT;
      } else if (lane < R) {
        sm.quota[lane] = c.lut[(size_t)m * R + lane];
        over = sm.quota[lane] > sm.capacity[lane];
      }
      over = __any_sync(0xffffffffu, over);
      __syncwarp();
      if (over && sm.status == 0) {
        if (!greedy_quota_warp(c, m, sm.capacity, sm.quota, greedy_load) && lane == 0)
          sm.status = DEV_CAPACITY;
      }
    }
    // totals and the stable descending order (np.argsort(-totals, 'mergesort'))
    for (int i = tid; i < m; i += blockDim.x) sm.totals[i] = sm.demand_total[sm.misses[i]];
    __syncthreads();
    for (int i = tid; i < m; i += blockDim.x) {
      int rank_i = 0;
      const int64_t ti = sm.totals[i];
      for (int j = 0; j < m; ++j) {
        const int64_t tj = sm.totals[j];
        rank_i += (tj > ti) || (tj == ti && j < i);
      }
      sm.order[rank_i] = i;
    }
    __syncthreads();
    if (warp == 0 && sm.status == 0) assignment_warp(c, sm, demand, sm.owner_layer);
  } else {
    if (tid == 0) {
      int room = 0, left[kMaxWorld];
      for (int r = 0; r < R; ++r) { left[r] = sm.capacity[r]; room += left[r]; }
      if (m > room) {
        sm.status = DEV_CAPACITY;  // the reference would retry forever here
      } else {
        sm.rng.seed((uint32_t)(uint64_t)(c.salt * 1000003 + in.event));
        for (int i = 0; i < m; ++i) {
          int r = sm.rng.randint(R);
          while (left[r] <= 0) r = sm.rng.randint(R);
          sm.assignment[i] = r;
          left[r] -= 1;
        }
      }
    }
  }
  __syncthreads();
  PLAN_TS(3);
  if (sm.status) {
    if (tid == 0) {
      set_err(out.err, sm.status);
      *out.n_fetches = 0;
      // this layer's scores changed above: the saved victim order is stale
      if (s.order_meta) s.order_meta[0] = 0;
    }
    plan_release(out.mirror, 0);
    return;
  }

  // -- Step 4: victims (one ordering of every slot) and the commit ---------
  // The j-th miss assigned to rank r takes the j-th record of rank r's
  // segment of the order of all slot records.  That order is saved between
  // layers: a record changes only when its slot's content changes or when
  // its key belongs to a layer planned since the order was saved (scores at
  // the start of a plan, last uses and installs at its end) or to this layer
  // (class 2), so only those records are re-keyed, sorted among themselves
  // and merged into the rest.  Without a valid saved order every record is
  // sorted.
  const int words = (c.layers + 63) / 64;
  const bool can_save = s.order_meta != nullptr && c.dirty_offset != 0 && s.order_cap >= c.sort_n;
  if (m > 0) {
    const int n = c.sort_n;  // power of two >= total_slots, >= 64
    uint64_t* k0 = reinterpret_cast<uint64_t*>(recs);
    uint64_t* k1 = k0 + n;
    uint32_t* sl = reinterpret_cast<uint32_t*>(k1 + n);
    if (tid == 0) {
      int pos = 0;
      for (int r = 0; r < R; ++r) { sm.seg_start[r] = pos; pos += c.capacities[r]; }
    }
    for (int i = tid; i < m; i += blockDim.x) {
      const int r = sm.assignment[i];
      int before = 0;  // earlier misses assigned to the same rank
      for (int j = 0; j < i; ++j) before += sm.assignment[j] == r;
      sm.victim_pos[i] = before;  // rank-relative
    }
    const bool incremental = can_save && s.order_meta[0] != 0;
    PLAN_TS(4);
    // the order the commit reads: the saved one, or the records in smem
    const uint64_t* o0 = k0;
    const uint32_t* osl = sl;
    if (!incremental) {
      for (int i = tid; i < n; i += blockDim.x) {
        uint64_t a0 = ~0ull, a1 = ~0ull;
        uint32_t ix = 0xffffffffu;
        if (i < c.total_slots) {
          const int r = c.slot_rank[i], idx = c.slot_index[i];
          slot_record(c, s, sm.active, r, idx, s.slots[idx], L, a0, a1);
          ix = (uint32_t)idx;
        }
        k0[i] = a0; k1[i] = a1; sl[i] = ix;
      }
      __syncthreads();
      sort_records(k0, k1, sl, n);
      if (can_save) {
        for (int i = tid; i < n; i += blockDim.x) {
          s.ord_k0[i] = k0[i]; s.ord_k1[i] = k1[i]; s.ord_sl[i] = sl[i];
        }
      }
    } else {
      uint64_t* dk0 = reinterpret_cast<uint64_t*>(dsm + c.dirty_offset);
      uint64_t* dk1 = dk0 + n;
      uint32_t* dsl = reinterpret_cast<uint32_t*>(dk1 + n);
      const int64_t* changed = s.order_meta + 1;  // layers planned since the order was saved
      // each thread's saved entries i = tid * nq + q (consecutive), in
      // registers; a dirty entry is re-keyed at once (its key is in hand)
      const int nq = (n + (int)blockDim.x - 1) / (int)blockDim.x;  // <= kIncPer
      uint64_t e0[kIncPer], e1[kIncPer];
      uint32_t es[kIncPer];
      bool dirty[kIncPer], live[kIncPer];
      int n_clean = 0;
#pragma unroll
      for (int q = 0; q < kIncPer; ++q) {
        const int i = tid * nq + q;
        dirty[q] = false;
        live[q] = q < nq && i < n;
        if (live[q]) {
          e0[q] = s.ord_k0[i]; e1[q] = s.ord_k1[i]; es[q] = s.ord_sl[i];
          if (es[q] != 0xffffffffu) {
            const int idx = (int)es[q];
            const int key = s.slots[idx];
            const int cls = (int)((e0[q] >> 48) & 0xff);
            const int saved_key = cls == 0 ? -1 : (int)(e1[q] & 0xffffff);
            const int kl = key >= 0 ? key / E : -1;
            dirty[q] = key != saved_key ||
                       (key >= 0 && (kl == L || ((changed[kl >> 6] >> (kl & 63)) & 1)));
            if (dirty[q]) slot_record(c, s, sm.active, idx / c.maxcap, idx, key, L, e0[q], e1[q]);
          }
          n_clean += !dirty[q];
        }
      }
      PLAN_TS(8);
      // stable compaction: the clean entries (saved order kept) into k0/k1/sl,
      // the dirty records into dk0/dk1/dsl (one block scan of the per-thread
      // clean counts; the entries before a thread's first are tid * nq)
      int cpos = plan_block_scan(n_clean, sm.warp_sum, &sm.scan_total);
      int dpos = tid * nq - cpos;
      const int nc = sm.scan_total, nd = n - nc;
#pragma unroll
      for (int q = 0; q < kIncPer; ++q) {
        if (!live[q]) continue;
        if (dirty[q]) {
          dk0[dpos] = e0[q]; dk1[dpos] = e1[q]; dsl[dpos] = es[q];
          ++dpos;
        } else {
          k0[cpos] = e0[q]; k1[cpos] = e1[q]; sl[cpos] = es[q];
          ++cpos;
        }
      }
      __syncthreads();
      PLAN_TS(9);
      if (threadIdx.x == 0 && g_plan_ts) g_plan_ts[12] = (unsigned long long)nd;
      if (nd <= kRankSort) {
        // each dirty record's place is the number of dirty records below it
        // (their keys are unique).  Lane l of warp w holds record w + 32 * l;
        // the warp's lanes split the comparisons of each of its records.  All
        // reads are done before the barrier, so the records move in place.
        const int nw = (int)(blockDim.x >> 5);
        const int own = warp + nw * lane;
        uint64_t a0 = 0, a1 = 0;
        uint32_t ax = 0;
        int place = 0;
        if (own < nd) { a0 = dk0[own]; a1 = dk1[own]; ax = dsl[own]; }
        for (int l = 0; warp + nw * l < nd; ++l) {
          const uint64_t b0 = __shfl_sync(0xffffffffu, a0, l);
          const uint64_t b1 = __shfl_sync(0xffffffffu, a1, l);
          int below = 0;
          for (int k = lane; k < nd; k += 32) {
            const uint64_t x0 = dk0[k], x1 = dk1[k];
            below += (int)((x0 < b0) | ((x0 == b0) & (x1 < b1)));
          }
          below = __reduce_add_sync(0xffffffffu, below);
          if (lane == l) place = below;
        }
        __syncthreads();
        if (own < nd) { dk0[place] = a0; dk1[place] = a1; dsl[place] = ax; }
        __syncthreads();
      } else {
        int dn = 64;
        while (dn < nd) dn <<= 1;
        for (int j = nd + tid; j < dn; j += blockDim.x) { dk0[j] = ~0ull; dk1[j] = ~0ull; dsl[j] = 0xffffffffu; }
        __syncthreads();
        sort_records(dk0, dk1, dsl, dn);
      }
      PLAN_TS(10);
      // merge: a clean record's position is its index plus the dirty records
      // below it, and the other way round (keys of real records are unique)
      for (int i = tid; i < nc; i += blockDim.x) {
        const int pos = i + count_less(dk0, dk1, nd, k0[i], k1[i]);
        s.ord_k0[pos] = k0[i]; s.ord_k1[pos] = k1[i]; s.ord_sl[pos] = sl[i];
      }
      for (int j = tid; j < nd; j += blockDim.x) {
        const int pos = j + count_less(k0, k1, nc, dk0[j], dk1[j]);
        s.ord_k0[pos] = dk0[j]; s.ord_k1[pos] = dk1[j]; s.ord_sl[pos] = dsl[j];
      }
      __syncthreads();
      PLAN_TS(11);
      o0 = s.ord_k0; osl = s.ord_sl;
    }
    __syncthreads();
    PLAN_TS(5);
    for (int i = tid; i < m; i += blockDim.x) {
      const int r = sm.assignment[i];
      const int j = sm.victim_pos[i];
      const int vp = (r >= 0 && r < R && j < c.capacities[r]) ? sm.seg_start[r] + j : -1;
      if (vp < 0 || vp >= n) { set_err(out.err, DEV_NO_SLOT); continue; }
      const uint64_t rk0 = o0[vp];
      const uint32_t rslot = osl[vp];
      const uint64_t cls = (rk0 >> 48) & 0xff;
      const bool ok = rslot != 0xffffffffu && (int)(rk0 >> 56) == r && cls < 2;
      if (!ok) { set_err(out.err, DEV_NO_SLOT); continue; }
      const int idx = (int)rslot;
      const int key = base + sm.misses[i];
      const int victim = s.slots[idx];
      if (victim >= 0) s.owner[victim] = -1;
      s.slots[idx] = key;
      s.owner[key] = r;
      out.fetches[i * 3 + 0] = r;
      out.fetches[i * 3 + 1] = key;
      out.fetches[i * 3 + 2] = idx - r * c.maxcap;
      if (out.mirror.seq && r == out.mirror.rank) {  // the j-th fetch of this rank
        out.mirror.keys[j] = key;
        out.mirror.slots[j] = idx - r * c.maxcap;
      }
    }
    // the saved order now holds every record as of this plan; this layer's
    // records change at its commit, so they are re-keyed next time
    __syncthreads();
    if (can_save && tid == 0) {
      s.order_meta[0] = 1;
      for (int w = 0; w < words; ++w) s.order_meta[1 + w] = 0;
      s.order_meta[1 + (L >> 6)] = (int64_t)(1ull << (L & 63));
    }
  } else if (can_save && tid == 0 && s.order_meta[0] != 0) {
    s.order_meta[1 + (L >> 6)] |= (int64_t)(1ull << (L & 63));  // no commit, but scores and last uses change
  }
  __syncthreads();
  PLAN_TS(6);
  const int64_t tick = in.event + 1;
  for (int e = tid; e < E; e += blockDim.x)
    if (sm.active[e]) s.last[base + e] = tick;
  if (tid < R) out.counts[tid] = 0;
  __syncthreads();
  if (tid == 0) *out.n_fetches = m;
  for (int i = tid; i < m; i += blockDim.x) {
    const int r = sm.assignment[i];
    if (r >= 0 && r < R) atomicAdd(&out.counts[r], 1);
    if (r == out.mirror.rank) atomicAdd(&sm.n_mine, 1);
  }
  for (int i = tid; i < n_tok * K; i += blockDim.x) {
    const int e = in.ids[i];
    out.dest[i] = e < E ? s.owner[base + e] : -1;
  }
  __syncthreads();
  PLAN_TS(7);
  plan_release(out.mirror, sm.n_mine);
  span_end(in.ts);
}

// ---------------------------------------------------------------------------
// Single-step kernels: the planner's device functions exposed one by one, for
// the reference's helper names (quota.py:25/70, policy.py:25/36/49/109).

// greedy_quota for m in [m_begin, m_end), one warp per m.  capacity NULL =
// unlimited (build_lut, ferry/quota.py:70-74).
__global__ void greedy_rows_kernel(const PlanConfig c, const int32_t* capacity, int m_begin,
                                   int m_end, int64_t* quota_out, int* err) {
  extern __shared__ uint8_t dsm[];
  __shared__ int cap[kMaxWorld];
  __shared__ int64_t qsm[32][kMaxWorld];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  int64_t* load = reinterpret_cast<int64_t*>(dsm) + (size_t)warp * (c.n_domains > 0 ? c.n_domains : 1);
  if (threadIdx.x < c.world) cap[threadIdx.x] = capacity ? capacity[threadIdx.x] : (1 << 30);
  __syncthreads();
  for (int m = m_begin + blockIdx.x * nw + warp; m < m_end; m += gridDim.x * nw) {
    const bool ok = greedy_quota_warp(c, m, cap, qsm[warp], load);
    if (!ok) {
      if (lane == 0) set_err(err, DEV_CAPACITY);
    } else if (lane < c.world) {
      quota_out[(size_t)(m - m_begin) * c.world + lane] = qsm[warp][lane];
    }
  }
}

__global__ void demand_kernel(const int64_t* selected, const int64_t* origins, int n_tokens,
                              int topk, int experts, int world, int64_t* d, int* err) {
  for (int i = threadIdx.x + blockIdx.x * blockDim.x; i < n_tokens * topk; i += blockDim.x * gridDim.x) {
    const int64_t e = selected[i], r = origins[i / topk];
    if (e < 0 || e >= experts || r < 0 || r >= world) { set_err(err, DEV_BAD_INPUT); continue; }
    atomicAdd(reinterpret_cast<unsigned long long*>(&d[e * world + r]), 1ull);
  }
}

__global__ void admission_kernel(const int32_t* slots, int maxcap, const int32_t* capacities,
                                 int world, int layer, const uint8_t* active, int experts,
                                 int64_t* u) {
  const int r = blockIdx.x;
  __shared__ int cnt;
  if (threadIdx.x == 0) cnt = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < capacities[r]; i += blockDim.x) {
    const int key = slots[r * maxcap + i];
    if (key < 0 || !(key / experts == layer && active[key % experts])) atomicAdd(&cnt, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) u[r] = cnt;
}

__global__ void assignment_kernel(const PlanConfig c, const int64_t* demand, const int64_t* misses,
                                  int m, const int32_t* owner, int layer, const int64_t* quota,
                                  int64_t* answer) {
  __shared__ PlanSmem sm;
  extern __shared__ uint8_t dsm[];
  int* dem = reinterpret_cast<int*>(dsm);
  const int E = c.experts, R = c.world, tid = threadIdx.x;
  for (int i = tid; i < E * R; i += blockDim.x) dem[i] = (int)demand[i];
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    int tot = 0;
    for (int r = 0; r < R; ++r) tot += dem[e * R + r];
    sm.demand_total[e] = tot;
  }
  if (tid < R) sm.quota[tid] = quota[tid];
  if (tid == 0) sm.m = m;
  for (int i = tid; i < m; i += blockDim.x) sm.misses[i] = (int)misses[i];
  __syncthreads();
  for (int i = tid; i < m; i += blockDim.x) sm.totals[i] = sm.demand_total[sm.misses[i]];
  __syncthreads();
  for (int i = tid; i < m; i += blockDim.x) {
    int rank_i = 0;
    const int64_t ti = sm.totals[i];
    for (int j = 0; j < m; ++j) rank_i += (sm.totals[j] > ti) || (sm.totals[j] == ti && j < i);
    sm.order[rank_i] = i;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) sm.owner_layer[e] = owner[(size_t)layer * E + e];
  __syncthreads();
  if ((tid >> 5) == 0) assignment_warp(c, sm, dem, sm.owner_layer);
  __syncthreads();
  for (int i = tid; i < m; i += blockDim.x) answer[i] = sm.assignment[i];
}

// _choose_slot for one rank: the minimum slot record of that rank (empty
// slots by index first, then eligible ones by (score, last use, key)).
__global__ void choose_slot_kernel(int rank, int layer, const uint8_t* active, const int32_t* slots,
                                   int maxcap, const int32_t* capacities, const int64_t* last,
                                   const float* scores, int experts, int64_t* result) {
  __shared__ SlotRec best[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  SlotRec mine;
  mine.k0 = ~0ull; mine.k1 = ~0ull; mine.slot = 0xffffffffu; mine.pad = 0;
  for (int i = threadIdx.x; i < capacities[rank]; i += blockDim.x) {
    const int key = slots[rank * maxcap + i];
    SlotRec r;
    r.slot = (uint32_t)i; r.pad = 0;
    if (key < 0) { r.k0 = 0; r.k1 = (uint64_t)i; }
    else if (key / experts == layer && active[key % experts]) { r.k0 = ~0ull; r.k1 = ~0ull; r.slot = 0xffffffffu; }
    else { r.k0 = (1ull << 48) | __float_as_uint(scores[key]); r.k1 = ((uint64_t)last[key] << 24) | (uint64_t)key; }
    if (rec_less(r, mine)) mine = r;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    SlotRec other;
    other.k0 = __shfl_xor_sync(0xffffffffu, mine.k0, o);
    other.k1 = __shfl_xor_sync(0xffffffffu, mine.k1, o);
    other.slot = __shfl_xor_sync(0xffffffffu, mine.slot, o);
    if (rec_less(other, mine)) mine = other;
  }
  if (lane == 0) best[warp] = mine;
  __syncthreads();
  if (threadIdx.x == 0) {
    SlotRec b = best[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) if (rec_less(best[w], b)) b = best[w];
    *result = b.slot == 0xffffffffu ? -1 : (int64_t)b.slot;
  }
}

// ---------------------------------------------------------------------------
int plan_launch(const PlanConfig& c, const PlanState& s, const PlanInputs& in,
                const PlanOutputs& out, cudaStream_t stream, bool after_router) {
  const size_t dyn = c.dyn_smem;
  static int configured_bytes = -1;
  if ((int)dyn > configured_bytes) {
    FB_CUDA(cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn));
    configured_bytes = (int)dyn;
  }
  // behind the router kernel: a programmatic dependent launch, so that the
  // planner's launch overlaps the router (the kernel waits for its outputs)
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kPlanThreads);
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = after_router ? 1 : 0;
  FB_CUDA(cudaLaunchKernelEx(&cfg, plan_kernel, c, s, in, out));
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

size_t plan_dyn_smem(int experts, int world, int total_slots, int n_domains, size_t* sort_off,
                     size_t* greedy_off, int* sort_n, size_t* dirty_off) {
  size_t off = (size_t)experts * world * sizeof(int);
  off = (off + 15) & ~size_t(15);
  int n = 64;  // the sort works on whole 64-record warp blocks
  while (n < total_slots) n <<= 1;
  *sort_n = n;
  *sort_off = off;
  off += (size_t)n * sizeof(SlotRec);
  *greedy_off = off;
  off += (size_t)(n_domains > 0 ? n_domains : 1) * sizeof(int64_t);
  off = (off + 15) & ~size_t(15);
  *dirty_off = 0;
  if (n <= kMaxIncremental) {  // the incremental order's dirty records: up to n of them
    *dirty_off = off;
    off += (size_t)n * sizeof(SlotRec);
  }
  return off;
}

size_t plan_static_smem() { return sizeof(PlanSmem); }

}  // namespace ferryb

using namespace ferryb;

extern "C" int ferryb_plan_layer(const ferryb_planner* p, int64_t event, int32_t layer,
                                 const uint8_t* ids, int32_t n_tokens, int32_t tokens_per_rank,
                                 const int64_t* origins, const float* gate_scores,
                                 const float* prob_rows, int32_t n_prob_rows, int32_t* fetches,
                                 int32_t* n_fetches, int32_t* dest, int32_t* counts, int32_t* err,
                                 cudaStream_t stream) {
  FB_CHECK_ARG(p != nullptr, "planner is NULL");
  FB_CHECK_ARG(p->world >= 1 && p->world <= kMaxWorld, "world must be in [1, %d]", kMaxWorld);
  FB_CHECK_ARG(p->experts >= 1 && p->experts <= kMaxExperts, "experts must be in [1, %d]",
               kMaxExperts);
  FB_CHECK_ARG(layer >= 0 && layer < p->layers, "layer %d out of range", layer);
  FB_CHECK_ARG((int64_t)p->layers * p->experts < (1 << 24), "layers * experts must be < 2^24");
  FB_CHECK_ARG(event >= 0 && event < ((int64_t)1 << 39), "event out of range");
  FB_CHECK_ARG(p->policy == 0 || p->policy == 1, "policy must be 0 (ferry) or 1 (random)");
  FB_CHECK_ARG(n_tokens >= 0 && p->topk >= 1 && p->window >= 1, "bad sizes");
  FB_CHECK_ARG(origins != nullptr || (tokens_per_rank > 0 && n_tokens == tokens_per_rank * p->world),
               "without origins, n_tokens must be world * tokens_per_rank");
  FB_CHECK_ARG(gate_scores != nullptr || origins == nullptr,
               "the device history needs rank-major tokens (origins NULL)");
  FB_CHECK_ARG(p->slots && p->owner && p->last && p->scores && p->capacities && p->slot_rank &&
                   p->slot_index && (p->policy == 1 || (p->lut && p->masks && p->seconds)),
               "planner state/config pointers missing");
  FB_CHECK_ARG(gate_scores || (p->ring && p->hist_count && p->hist_head),
               "history state missing");
  FB_CHECK_ARG(fetches && n_fetches && dest && counts && err, "output pointers missing");
  PlanConfig c{};
  c.world = p->world; c.experts = p->experts; c.layers = p->layers; c.topk = p->topk;
  c.window = p->window; c.policy = p->policy; c.bps = p->balance_tol_bps; c.salt = p->salt;
  c.maxcap = p->maxcap; c.total_slots = p->total_slots; c.n_domains = p->n_domains;
  c.lut_rows = p->lut_rows; c.capacities = p->capacities; c.slot_rank = p->slot_rank;
  c.slot_index = p->slot_index; c.lut = p->lut; c.masks = p->masks; c.seconds = p->seconds;
  c.dyn_smem = plan_dyn_smem(c.experts, c.world, c.total_slots, c.n_domains, &c.sort_offset,
                             &c.greedy_offset, &c.sort_n, &c.dirty_offset);
  FB_CHECK_ARG(c.dyn_smem + plan_static_smem() <= 225 * 1024,
               "cache too large for the one-CTA planner (%d slots)", c.total_slots);
  const PlanState s = plan_state(p);
  PlanInputs in{};
  in.ids = ids; in.n_tokens = n_tokens; in.tokens_per_rank = tokens_per_rank;
  in.origins = origins; in.gate_scores = gate_scores; in.prob_rows = prob_rows;
  in.n_prob_rows = n_prob_rows; in.event = event; in.layer = layer;
  PlanOutputs out{fetches, n_fetches, dest, counts, err};
  return plan_launch(c, s, in, out, stream);
}

static PlanConfig config_of(const ferryb_planner* p) {
  PlanConfig c{};
  c.world = p->world; c.experts = p->experts; c.layers = p->layers; c.topk = p->topk;
  c.window = p->window; c.policy = p->policy; c.bps = p->balance_tol_bps; c.salt = p->salt;
  c.maxcap = p->maxcap; c.total_slots = p->total_slots; c.n_domains = p->n_domains;
  c.lut_rows = p->lut_rows; c.capacities = p->capacities; c.slot_rank = p->slot_rank;
  c.slot_index = p->slot_index; c.lut = p->lut; c.masks = p->masks; c.seconds = p->seconds;
  return c;
}

extern "C" int ferryb_greedy_quota_rows(int32_t world, const int64_t* masks, const double* seconds,
                                        int32_t n_domains, const int32_t* capacity, int32_t m_begin,
                                        int32_t m_end, int64_t* quota_out, int32_t* err,
                                        cudaStream_t stream) {
  FB_CHECK_ARG(world >= 1 && world <= kMaxWorld && n_domains >= 0 && m_begin >= 0 && m_end >= m_begin,
               "greedy_quota: bad arguments");
  FB_CHECK_ARG(masks && seconds && quota_out && err, "greedy_quota: null pointer");
  if (m_end == m_begin) return FERRYB_OK;
  PlanConfig c{};
  c.world = world; c.masks = masks; c.seconds = seconds; c.n_domains = n_domains;
  const int warps = 8;
  const size_t dyn = (size_t)warps * (n_domains > 0 ? n_domains : 1) * sizeof(int64_t);
  int blocks = (m_end - m_begin + warps - 1) / warps;
  if (blocks > 148) blocks = 148;
  greedy_rows_kernel<<<blocks, warps * 32, dyn, stream>>>(c, capacity, m_begin, m_end, quota_out, err);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

extern "C" int ferryb_demand(const int64_t* selected, const int64_t* origins, int32_t n_tokens,
                             int32_t topk, int32_t experts, int32_t world, int64_t* demand,
                             int32_t* err, cudaStream_t stream) {
  FB_CHECK_ARG(selected && origins && demand && err && n_tokens >= 0 && topk > 0, "demand: bad arguments");
  FB_CUDA(cudaMemsetAsync(demand, 0, sizeof(int64_t) * experts * world, stream));
  if (n_tokens == 0) return FERRYB_OK;
  demand_kernel<<<(n_tokens * topk + 255) / 256, 256, 0, stream>>>(selected, origins, n_tokens, topk,
                                                                   experts, world, demand, err);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

extern "C" int ferryb_admission_capacity(const int32_t* slots, int32_t maxcap,
                                         const int32_t* capacities, int32_t world, int32_t layer,
                                         const uint8_t* active, int32_t experts, int64_t* u,
                                         cudaStream_t stream) {
  FB_CHECK_ARG(slots && capacities && active && u && world >= 1, "admission: bad arguments");
  admission_kernel<<<world, 256, 0, stream>>>(slots, maxcap, capacities, world, layer, active, experts, u);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

extern "C" int ferryb_load_balanced_assignment(const int64_t* demand, int32_t experts, int32_t world,
                                               const int64_t* misses, int32_t m,
                                               const int32_t* owner, int32_t layer,
                                               const int64_t* quota, int64_t balance_tol_bps,
                                               int64_t* answer, cudaStream_t stream) {
  FB_CHECK_ARG(world >= 1 && world <= kMaxWorld && experts >= 1 && experts <= kMaxExperts &&
                   m >= 0 && m <= experts,
               "assignment: bad sizes");
  if (m == 0) return FERRYB_OK;
  PlanConfig c{};
  c.world = world; c.experts = experts; c.bps = balance_tol_bps;
  assignment_kernel<<<1, 1024, (size_t)experts * world * sizeof(int), stream>>>(
      c, demand, misses, m, owner, layer, quota, answer);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

extern "C" int ferryb_choose_slot(int32_t rank, int32_t layer, const uint8_t* active,
                                  const int32_t* slots, int32_t maxcap, const int32_t* capacities,
                                  const int64_t* last, const float* scores, int32_t experts,
                                  int64_t* result, cudaStream_t stream) {
  FB_CHECK_ARG(active && slots && capacities && last && scores && result && rank >= 0,
               "choose_slot: bad arguments");
  choose_slot_kernel<<<1, 1024, 0, stream>>>(rank, layer, active, slots, maxcap, capacities, last,
                                             scores, experts, result);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

extern "C" int ferryb_debug_plan_timestamps(void* dev_ptr) {
  FB_CUDA(cudaMemcpyToSymbol(g_plan_ts, &dev_ptr, sizeof(void*)));
  return FERRYB_OK;
}
