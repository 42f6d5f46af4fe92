// experts.cu -- routed/shared-expert SwiGLU as a grouped bf16 GEMM on the
// 5th-generation tensor cores (tcgen05.mma, accumulators in TMEM, operands
// staged by TMA with the 128-byte swizzle).
//
// Replaces ferry/csrc/expert_ops.cpp:16-45 (execute_experts: per cached expert
// x = input[rows]; y = (silu(x Wg^T) * (x Wu^T)) Wd^T; y * w[rows, cols]) and
// the silu_mul kernel of ferry/csrc/expert_ops.cu:6-25.
//
// Data layout.  An expert row of the cache is [gate I x H | up I x H | down
// H x I] bf16 (ferry/model.py:86-88).  The kernel sees the cache through two
// 2D tensor maps: W1 = [slots*3I, H] (gate rows of slot s at s*3I, up rows at
// s*3I + I) and W2 = [slots*3H, I] (down rows of slot s at s*3H + 2H).  The
// routed tokens of all groups sit back to back in X = [routes, H] (one row per
// (token, expert) route, grouped by expert); the activations in A = [routes, I].
//
// Orientation ("swap AB").  The expert weight tile is the MMA's M = 128 side
// and the group's routes are the N side (16..128 columns), so a decode group
// with a handful of tokens costs one pass over its weights: the kernel is
// HBM-bound at decode and tensor-bound only for groups of hundreds of routes.
//
// Phase 1 (GATE_UP): per (group, 128-row tile of I): D_g = Wg_tile X^T and
// D_u = Wu_tile X^T over K = H; epilogue act = bf16(silu(bf16 D_g) * bf16 D_u)
// in float32, written to A.  Phase 2 (DOWN): per (group, 128-row tile of H):
// D = Wd_tile A^T over K = I; epilogue out = bf16(bf16(D) * w_route), written
// to OUT = [routes, H].  The bf16 rounding points are the reference's.
//
// CTA roles (192 threads): warp 0 issues TMA loads, warp 1 allocates TMEM and
// issues tcgen05.mma from one elected lane, warps 2-5 drain TMEM (warp w reads
// TMEM lanes 32*(w%4)..+31).  Shared-memory stages are a ring guarded by
// full/empty mbarriers; TMEM holds two accumulator buffers so the epilogue of
// one tile overlaps the MMAs of the next.  The grid is persistent (<= #SMs).
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "experts.cuh"

namespace ferryb {

constexpr int kThreads = 192;
constexpr int kBlockM = 128;   // weight rows per tile (MMA M)
constexpr int kBlockK = 64;    // bf16 elements per 128-byte swizzle row
constexpr int kMaxN = 128;     // routes per tile (MMA N)
constexpr uint32_t kTileBytesA = kBlockM * kBlockK * 2;  // 16 KB
constexpr uint32_t kTileBytesB = kMaxN * kBlockK * 2;    // 16 KB (max)
constexpr uint64_t kWaitNs = 2000000000ull;               // 2 s bound on any wait


__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for an mbarrier phase, bounded by time; on timeout raise the CTA's
// abort flag and the kernel's error word.
__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity,
                                             volatile int* abort_flag, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > kWaitNs) {
        *abort_flag = 1;
        atomicCAS(err, 0, DEV_WAIT_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ int box_index(int n) {
  return n <= 16 ? 0 : n <= 32 ? 1 : n <= 64 ? 2 : 3;
}

template <int PHASE>
struct PhaseCfg;
template <>
struct PhaseCfg<1> {
  static constexpr int kA = 2;  // gate and up tiles per stage
  static constexpr int kStages = 4;
};
template <>
struct PhaseCfg<2> {
  static constexpr int kA = 1;
  static constexpr int kStages = 6;
};

template <int PHASE>
constexpr uint32_t stage_bytes() {
  return PhaseCfg<PHASE>::kA * kTileBytesA + kTileBytesB;
}
template <int PHASE>
constexpr uint32_t smem_bytes() {
  return PhaseCfg<PHASE>::kStages * stage_bytes<PHASE>() + 1024 /*align*/ + 256 /*barriers*/;
}

struct GemmParams {
  const GemmGroup* groups;
  int n_groups;
  int m_tiles;       // I/128 (phase 1) or H/128 (phase 2)
  int k_blocks;      // H/64 (phase 1) or I/64 (phase 2)
  int rows_per_slot; // 3I (W1 view) or 3H (W2 view)
  int up_offset;     // I: rows from gate to up inside a slot (phase 1)
  int down_offset;   // 2H: rows from slot start to down (phase 2)
  int out_cols;      // I (phase 1, act width) or H (phase 2, out width)
  __nv_bfloat16* out;             // A (phase 1) or OUT (phase 2)
  const __nv_bfloat16* route_w;   // per-route routing weight (phase 2), may be null (=1)
  int* err;
};

template <int PHASE>
__global__ void __launch_bounds__(kThreads, 1)
    swiglu_gemm_kernel(const __grid_constant__ CUtensorMap wmap,
                       const __grid_constant__ BMaps bmaps, const GemmParams p) {
  using Cfg = PhaseCfg<PHASE>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes<PHASE>());
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;   // [2]
  uint64_t* tempty = tfull + 2;  // [2]
  uint64_t* drain = tempty + 2;  // [1] MMA drain on abort
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_smem + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_items = p.n_groups * p.m_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 4); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&wmap);
    for (int i = 0; i < 4; ++i) tma_prefetch_desc(&bmaps.m[i]);
  }
  if (warp == 1) { tmem_alloc(tmem_base_smem, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_smem;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t pending = 0, pend_parity = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const GemmGroup g = p.groups[item / p.m_tiles];
        const int mt = item % p.m_tiles;
        const int chunks = (g.count + kMaxN - 1) / kMaxN;
        for (int c = 0; c < chunks && ok; ++c) {
          const int n_valid = min(kMaxN, g.count - c * kMaxN);
          const int bi = box_index(n_valid);
          const uint32_t b_bytes = (16u << bi) * kBlockK * 2;
          const int row_b = g.start + c * kMaxN;
          int row_a;
          if (PHASE == 1) row_a = g.slot * p.rows_per_slot + mt * kBlockM;
          else row_a = g.slot * p.rows_per_slot + p.down_offset + mt * kBlockM;
          for (int kb = 0; kb < p.k_blocks; ++kb) {
            if (!wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.err)) { ok = false; break; }
            uint8_t* st = smem + stage * stage_bytes<PHASE>();
            mbar_expect_tx(&full[stage], Cfg::kA * kTileBytesA + b_bytes);
            tma_load_2d(st, &wmap, &full[stage], kb * kBlockK, row_a);
            if (PHASE == 1)
              tma_load_2d(st + kTileBytesA, &wmap, &full[stage], kb * kBlockK, row_a + p.up_offset);
            tma_load_2d(st + Cfg::kA * kTileBytesA, &bmaps.m[bi], &full[stage], kb * kBlockK, row_b);
            pending |= 1u << stage;
            pend_parity = (pend_parity & ~(1u << stage)) | (phase << stage);
            if (++stage == S) { stage = 0; phase ^= 1; }
          }
        }
      }
      if (!ok) {
        // Drain this CTA's TMA loads still in flight before the CTA exits.
        uint64_t t0 = global_ns();
        for (int s = 0; s < S; ++s)
          if (pending & (1u << s))
            while (!mbar_try_wait(&full[s], (pend_parity >> s) & 1) && global_ns() - t0 < kWaitNs) {}
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const GemmGroup g = p.groups[item / p.m_tiles];
        const int chunks = (g.count + kMaxN - 1) / kMaxN;
        for (int c = 0; c < chunks && ok; ++c) {
          const int n_valid = min(kMaxN, g.count - c * kMaxN);
          const uint32_t n_mma = 16u << box_index(n_valid);
          const uint32_t idesc = idesc_bf16_f32(kBlockM, n_mma);
          if (!wait_bounded(&tempty[acc], acc_phase ^ 1, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d0 = tmem_base + acc * 256;        // gate (phase 1) / out (phase 2)
          const uint32_t d1 = tmem_base + acc * 256 + 128;  // up (phase 1)
          for (int kb = 0; kb < p.k_blocks; ++kb) {
            if (!wait_bounded(&full[stage], phase, abort_flag, p.err)) { ok = false; break; }
            tc_fence_after();
            const uint32_t st = smem_u32(smem + stage * stage_bytes<PHASE>());
            const uint32_t sb = st + Cfg::kA * kTileBytesA;
#pragma unroll
            for (int k = 0; k < kBlockK / 16; ++k) {
              const uint64_t bdesc = smem_desc_sw128(sb + k * 32);
              const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
              umma_bf16(d0, smem_desc_sw128(st + k * 32), bdesc, idesc, accum);
              if (PHASE == 1) umma_bf16(d1, smem_desc_sw128(st + kTileBytesA + k * 32), bdesc, idesc, accum);
            }
            umma_commit(&empty[stage]);
            if (++stage == S) { stage = 0; phase ^= 1; }
          }
          if (!ok) break;
          umma_commit(&tfull[acc]);
          if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
      }
      // Make sure no MMA is still writing TMEM before the CTA frees it.
      umma_commit(drain);
      uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < kWaitNs) {}
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const GemmGroup g = p.groups[item / p.m_tiles];
      const int mt = item % p.m_tiles;
      const int chunks = (g.count + kMaxN - 1) / kMaxN;
      const int feature = mt * kBlockM + q * 32 + lane;
      for (int c = 0; c < chunks; ++c) {
        const int n_valid = min(kMaxN, g.count - c * kMaxN);
        if (!wait_bounded(&tfull[acc], acc_phase, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
        const uint32_t d0 = tmem_base + lane_addr + acc * 256;
        for (int c0 = 0; c0 < n_valid; c0 += 16) {
          float v0[16];
          tmem_ld16(d0 + c0, v0);
          if (PHASE == 1) {
            float v1[16];
            tmem_ld16(d0 + 128 + c0, v1);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (c0 + j < n_valid) {
                const float gt = bf16_round(v0[j]);
                const float up = bf16_round(v1[j]);
                const float a = (gt / (1.0f + expf(-gt))) * up;
                const size_t row = static_cast<size_t>(g.start + c * kMaxN + c0 + j);
                p.out[row * p.out_cols + feature] = __float2bfloat16_rn(a);
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (c0 + j < n_valid) {
                const size_t row = static_cast<size_t>(g.start + c * kMaxN + c0 + j);
                float y = bf16_round(v0[j]);
                if (p.route_w) y = y * __bfloat162float(p.route_w[row]);
                p.out[row * p.out_cols + feature] = __float2bfloat16_rn(y);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ---------------------------------------------------------------------------
// Persistent fused kernel: both phases of every group in one launch.
//
// Phase-1 items pack gate and up into one MMA: the A tile holds 64 gate rows
// (features f0..f0+63) above the 64 up rows of the same features, so one
// M = 128 tcgen05.mma per k-step yields both, in TMEM lanes 0-63 (gate) and
// 64-127 (up).  An item then moves 512 KB of weights instead of 1 MB, which
// halves the granularity of the work queue (the last wave's imbalance), and
// the epilogue pairs each feature's gate and up through shared memory: the
// warps that read TMEM lanes 64-127 hand the up values to the warps that read
// lanes 0-63, which apply silu(gate) * up.  Phase-2 items are 128 down rows.
//
// Work items are claimed in order from an atomic counter:
//   cached groups' phase-1 tiles, cached groups' phase-2 tiles, then for each
//   fetched group (in fetch order) its phase-1 tiles and its phase-2 tiles.
// A phase-2 tile of group g starts when g's phase-1 tiles have all been
// written (dep[g] counts epilogue warps), and a fetched group's tiles start
// when its readiness flag has been raised (cuStreamWriteValue32 on the H2D
// engine's flag stream once the group's copy has landed).  A
// producer only waits on an item's dependencies after it has issued every
// load of the items it claimed before, and every dependency belongs to an
// earlier-claimed item or to an already-enqueued copy, so the grid (<= one
// CTA per SM, all resident) always makes progress; each wait is bounded.
constexpr int kPackM = 64;  // features per phase-1 item (gate rows = up rows)

struct FusedParams {
  const GemmGroup* groups;
  int n_groups, n_hit;
  int mt1, mt2, kb1, kb2;  // mt1 = I / 64 phase-1 items, mt2 = H / 128 phase-2 items
  int rows1, up_off, rows2, down_off;
  int inter, hidden;
  __nv_bfloat16* act;
  __nv_bfloat16* out;
  const __nv_bfloat16* route_w;
  const uint32_t* ready;  // [fetched] readiness of the gate/up rows, fetch order; null: the
                          // stream already waited for the copies
  const uint32_t* ready_down;  // [fetched] readiness of the down rows (phase-2 items)
  uint32_t ready_value;
  uint64_t ready_wait_ns;  // bound on one readiness wait
  int* queue;  // [1] claim counter, zero at launch
  int* done;   // [1] CTAs finished; the last one zeroes queue/dep/done for the next launch
  int* dep;    // [n_groups] phase-1 epilogue-warp completions, zero at launch
  int* err;
  unsigned long long* ts;  // null, or [2]: earliest CTA start / latest CTA end (globaltimer ns)
};

struct FusedItem {
  int phase, group, tile, fetched;  // fetched: fetch index or -1
};

__device__ __forceinline__ FusedItem decode_item(const FusedParams& p, int item) {
  FusedItem it;
  const int per = p.mt1 + p.mt2;
  const int h1 = p.n_hit * p.mt1, h2 = p.n_hit * per;
  if (item < h1) {
    it.phase = 1; it.group = item / p.mt1; it.tile = item % p.mt1; it.fetched = -1;
  } else if (item < h2) {
    const int i = item - h1;
    it.phase = 2; it.group = i / p.mt2; it.tile = i % p.mt2; it.fetched = -1;
  } else {
    const int i = item - h2;
    const int j = i / per, r = i % per;
    it.group = p.n_hit + j;
    it.fetched = j;
    if (r < p.mt1) { it.phase = 1; it.tile = r; }
    else { it.phase = 2; it.tile = r - p.mt1; }
  }
  return it;
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire_s32_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded spin until *flag >= value (readiness, at most limit_ns) / *cnt >=
// target (deps).
__device__ bool spin_ready(const uint32_t* flag, uint32_t value, uint64_t limit_ns,
                           volatile int* abort_flag, int* err) {
  if (ld_acquire_u32(flag) >= value) return true;
  const uint64_t t0 = global_ns();
  while (ld_acquire_u32(flag) < value) {
    __nanosleep(128);
    if (*abort_flag) return false;
    if (global_ns() - t0 > limit_ns) { *abort_flag = 1; atomicCAS(err, 0, DEV_WAIT_TIMEOUT); return false; }
  }
  return true;
}
__device__ bool spin_count(const int* cnt, int target, volatile int* abort_flag, int* err) {
  if (ld_acquire_s32_gpu(cnt) >= target) return true;
  const uint64_t t0 = global_ns();
  while (ld_acquire_s32_gpu(cnt) < target) {
    __nanosleep(64);
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitNs) { *abort_flag = 1; atomicCAS(err, 0, DEV_WAIT_TIMEOUT); return false; }
  }
  return true;
}

// The four epilogue warps (threads 64..191) meet at named barrier 1 (barrier
// 0 is __syncthreads).  epilogue_all is a barrier that also ANDs a predicate
// over the 128 threads: every decision to leave the epilogue loop goes
// through it, so the four warps always leave together and none can be left
// waiting at a barrier.
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ bool epilogue_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}

constexpr int kSched = 4;           // claimed-item ring depth
constexpr int kFusedStages = 6;
constexpr uint32_t kFusedStageBytes = kTileBytesA + kTileBytesB;  // 32 KB
constexpr int kXchgStride = 17;     // floats per feature row of the gate/up exchange (padded)
constexpr uint32_t kFusedSmem =
    kFusedStages * kFusedStageBytes + 1024 + 512 + kPackM * kXchgStride * 4;

__global__ void __launch_bounds__(kThreads, 1)
    swiglu_fused_kernel(const __grid_constant__ CUtensorMap w1h, const __grid_constant__ CUtensorMap w2,
                        const __grid_constant__ BMaps bx, const __grid_constant__ BMaps ba,
                        const FusedParams p) {
  constexpr int S = kFusedStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * kFusedStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;     // [2]
  uint64_t* tempty = tfull + 2;    // [2]
  uint64_t* drain = tempty + 2;    // [1]
  uint64_t* sfull = drain + 1;     // [kSched]
  uint64_t* sempty = sfull + kSched;  // [kSched]
  int* sched = reinterpret_cast<int*>(sempty + kSched);  // [kSched]
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(sched + kSched);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_smem + 1);
  float* xchg = reinterpret_cast<float*>(smem + S * kFusedStageBytes + 512);  // [64][17]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_items = p.n_groups * (p.mt1 + p.mt2);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 4); }
    mbar_init(drain, 1);
    for (int q = 0; q < kSched; ++q) { mbar_init(&sfull[q], 1); mbar_init(&sempty[q], 5); }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&w1h);
    tma_prefetch_desc(&w2);
    for (int i = 0; i < 4; ++i) { tma_prefetch_desc(&bx.m[i]); tma_prefetch_desc(&ba.m[i]); }
  }
  if (warp == 1) { tmem_alloc(tmem_base_smem, 256); tmem_relinquish(); }
  if (p.ts && threadIdx.x == 0) atomicMin(&p.ts[0], (unsigned long long)globaltimer_ns());
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_smem;

  if (warp == 0) {
    // ---------------- scheduler + TMA producer ----------------
    if (elect_one()) {
      int stage = 0, q = 0;
      uint32_t phase = 0, qphase = 0;
      uint32_t pending = 0, pend_parity = 0;
      bool ok = true;
      for (;;) {
        if (!wait_bounded(&sempty[q], qphase ^ 1, abort_flag, p.err)) { ok = false; break; }
        int item = atomicAdd(p.queue, 1);
        if (item >= n_items || *abort_flag) item = -1;
        sched[q] = item;
        mbar_arrive(&sfull[q]);
        if (++q == kSched) { q = 0; qphase ^= 1; }
        if (item < 0) break;
        const FusedItem it = decode_item(p, item);
        const GemmGroup g = p.groups[it.group];
        // dependencies: copy readiness of the rows the item reads (gate/up for
        // phase 1, down for phase 2), then (phase 2) the group's phase-1 tiles
        if (it.fetched >= 0 && p.ready &&
            !spin_ready((it.phase == 1 ? p.ready : p.ready_down) + it.fetched, p.ready_value,
                        p.ready_wait_ns, abort_flag, p.err)) {
          ok = false; break;
        }
        if (it.phase == 2 && !spin_count(p.dep + it.group, 4 * p.mt1, abort_flag, p.err)) {
          ok = false; break;
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");
        const int kb_n = it.phase == 1 ? p.kb1 : p.kb2;
        const BMaps* bm = it.phase == 1 ? &bx : &ba;
        // phase 1: gate rows f0.. and up rows f0.. (64 each); phase 2: 128 down rows
        const int row_a = it.phase == 1 ? g.slot * p.rows1 + it.tile * kPackM
                                        : g.slot * p.rows2 + p.down_off + it.tile * kBlockM;
        const int chunks = (g.count + kMaxN - 1) / kMaxN;
        for (int c = 0; c < chunks && ok; ++c) {
          const int n_valid = min(kMaxN, g.count - c * kMaxN);
          const int bi = box_index(n_valid);
          const uint32_t b_bytes = (16u << bi) * kBlockK * 2;
          const int row_b = g.start + c * kMaxN;
          for (int kb = 0; kb < kb_n; ++kb) {
            if (!wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.err)) { ok = false; break; }
            uint8_t* st = smem + stage * kFusedStageBytes;
            mbar_expect_tx(&full[stage], kTileBytesA + b_bytes);
            if (it.phase == 1) {
              tma_load_2d(st, &w1h, &full[stage], kb * kBlockK, row_a);
              tma_load_2d(st + kTileBytesA / 2, &w1h, &full[stage], kb * kBlockK, row_a + p.up_off);
            } else {
              tma_load_2d(st, &w2, &full[stage], kb * kBlockK, row_a);
            }
            tma_load_2d(st + kTileBytesA, &bm->m[bi], &full[stage], kb * kBlockK, row_b);
            pending |= 1u << stage;
            pend_parity = (pend_parity & ~(1u << stage)) | (phase << stage);
            if (++stage == S) { stage = 0; phase ^= 1; }
          }
        }
        if (!ok) break;
      }
      if (!ok) {
        // consumers poll the abort flag in their bounded waits and stop
        *abort_flag = 1;
        const uint64_t t0 = global_ns();
        for (int s2 = 0; s2 < S; ++s2)
          if (pending & (1u << s2))
            while (!mbar_try_wait(&full[s2], (pend_parity >> s2) & 1) && global_ns() - t0 < kWaitNs) {}
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      int stage = 0, acc = 0, q = 0;
      uint32_t phase = 0, acc_phase = 0, qphase = 0;
      bool ok = true;
      for (;;) {
        if (!wait_bounded(&sfull[q], qphase, abort_flag, p.err)) break;
        const int item = sched[q];
        mbar_arrive(&sempty[q]);
        if (++q == kSched) { q = 0; qphase ^= 1; }
        if (item < 0) break;
        const FusedItem it = decode_item(p, item);
        const GemmGroup g = p.groups[it.group];
        const int kb_n = it.phase == 1 ? p.kb1 : p.kb2;
        const int chunks = (g.count + kMaxN - 1) / kMaxN;
        for (int c = 0; c < chunks && ok; ++c) {
          const int n_valid = min(kMaxN, g.count - c * kMaxN);
          const uint32_t n_mma = 16u << box_index(n_valid);
          const uint32_t idesc = idesc_bf16_f32(kBlockM, n_mma);
          if (!wait_bounded(&tempty[acc], acc_phase ^ 1, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d0 = tmem_base + acc * kMaxN;
          for (int kb = 0; kb < kb_n; ++kb) {
            if (!wait_bounded(&full[stage], phase, abort_flag, p.err)) { ok = false; break; }
            tc_fence_after();
            const uint32_t st = smem_u32(smem + stage * kFusedStageBytes);
            const uint32_t sb = st + kTileBytesA;
#pragma unroll
            for (int k = 0; k < kBlockK / 16; ++k) {
              const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
              umma_bf16(d0, smem_desc_sw128(st + k * 32), smem_desc_sw128(sb + k * 32), idesc, accum);
            }
            umma_commit(&empty[stage]);
            if (++stage == S) { stage = 0; phase ^= 1; }
          }
          if (!ok) break;
          umma_commit(&tfull[acc]);
          if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
        if (!ok) break;
      }
      umma_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < kWaitNs) {}
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    // warp w reads TMEM lanes 32*(w%4)..+31: qd 0,1 = gate rows of a phase-1
    // tile (features f0 + 32*qd + lane), qd 2,3 = the up rows of the same
    // features; in phase 2 all four hold down rows tile*128 + 32*qd + lane.
    const int qd = warp & 3;
    const bool up_rows = qd >= 2;
    const int f_local = (qd & 1) * 32 + lane;
    int acc = 0, q = 0;
    uint32_t acc_phase = 0, qphase = 0;
    bool ok = true;
    for (;;) {
      if (!epilogue_all(wait_bounded(&sfull[q], qphase, abort_flag, p.err))) break;
      const int item = sched[q];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[q]);
      if (++q == kSched) { q = 0; qphase ^= 1; }
      if (item < 0) break;  // the same entry for all four warps
      const FusedItem it = decode_item(p, item);
      const GemmGroup g = p.groups[it.group];
      const int chunks = (g.count + kMaxN - 1) / kMaxN;
      for (int c = 0; c < chunks; ++c) {
        const int n_valid = min(kMaxN, g.count - c * kMaxN);
        if (!epilogue_all(wait_bounded(&tfull[acc], acc_phase, abort_flag, p.err))) { ok = false; break; }
        tc_fence_after();
        const uint32_t d0 = tmem_base + (static_cast<uint32_t>(qd * 32) << 16) + acc * kMaxN;
        for (int c0 = 0; c0 < n_valid; c0 += 16) {
          float v0[16];
          tmem_ld16(d0 + c0, v0);
          if (it.phase == 1) {
            if (up_rows) {
#pragma unroll
              for (int j = 0; j < 16; ++j) xchg[f_local * kXchgStride + j] = bf16_round(v0[j]);
            }
            epilogue_sync();
            if (!up_rows) {
              const int feature = it.tile * kPackM + f_local;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                if (c0 + j < n_valid) {
                  const float gt = bf16_round(v0[j]);
                  const float up = xchg[f_local * kXchgStride + j];
                  const float a = (gt / (1.0f + expf(-gt))) * up;
                  const size_t row = static_cast<size_t>(g.start + c * kMaxN + c0 + j);
                  p.act[row * p.inter + feature] = __float2bfloat16_rn(a);
                }
              }
            }
            epilogue_sync();
          } else {
            const int feature = it.tile * kBlockM + qd * 32 + lane;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (c0 + j < n_valid) {
                const size_t row = static_cast<size_t>(g.start + c * kMaxN + c0 + j);
                float y = bf16_round(v0[j]);
                if (p.route_w) y = y * __bfloat162float(p.route_w[row]);
                p.out[row * p.hidden + feature] = __float2bfloat16_rn(y);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      if (!ok) break;
      if (it.phase == 1) {
        // publish this warp's activations to the group's phase-2 tiles
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(p.dep + it.group, 1);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
  // the last CTA to finish leaves the counters zeroed for the next launch on
  // this stream (every CTA is past its last claim and dependency read)
  if (threadIdx.x == 0) {
    if (p.ts) atomicMax(&p.ts[1], (unsigned long long)globaltimer_ns());
    __threadfence();
    if (atomicAdd(p.done, 1) == (int)gridDim.x - 1) {
      for (int g = 0; g < p.n_groups; ++g) p.dep[g] = 0;
      *p.queue = 0;
      __threadfence();
      *p.done = 0;
    }
  }
}

int swiglu_fused_launch(const GemmMaps& m, const GemmGroup* groups, int n_groups, int n_hit,
                        const uint32_t* ready, const uint32_t* ready_down, uint32_t ready_value,
                        int* queue_dep,
                        const __nv_bfloat16* route_w, __nv_bfloat16* act, __nv_bfloat16* out,
                        int* err, cudaStream_t stream, unsigned long long* ts,
                        uint64_t ready_wait_ns) {
  if (n_groups == 0) return FERRYB_OK;
  int device = 0;
  FB_CUDA(cudaGetDevice(&device));
  FusedParams p{};
  p.ready_wait_ns = ready_wait_ns ? ready_wait_ns : kWaitNs;
  p.ts = ts;
  p.groups = groups;
  p.n_groups = n_groups;
  p.n_hit = n_hit;
  p.mt1 = static_cast<int>(m.inter / kPackM);
  p.mt2 = static_cast<int>(m.hidden / kBlockM);
  p.kb1 = static_cast<int>(m.hidden / kBlockK);
  p.kb2 = static_cast<int>(m.inter / kBlockK);
  p.rows1 = static_cast<int>(3 * m.inter);
  p.up_off = static_cast<int>(m.inter);
  p.rows2 = static_cast<int>(3 * m.hidden);
  p.down_off = static_cast<int>(2 * m.hidden);
  p.inter = static_cast<int>(m.inter);
  p.hidden = static_cast<int>(m.hidden);
  p.act = act;
  p.out = out;
  p.route_w = route_w;
  p.ready = ready;
  p.ready_down = ready_down ? ready_down : ready;
  p.ready_value = ready_value;
  p.queue = queue_dep;
  p.done = queue_dep + 1;
  p.dep = queue_dep + 2;
  p.err = err;
  const int items = n_groups * (p.mt1 + p.mt2);
  const int grid = items < num_sms(device) ? items : num_sms(device);
  static bool attr_set[64] = {};
  if (device < 64 && !attr_set[device]) {
    FB_CUDA(cudaFuncSetAttribute(swiglu_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kFusedSmem));
    attr_set[device] = true;
  }
  swiglu_fused_kernel<<<grid, kThreads, kFusedSmem, stream>>>(m.w1h, m.w2, m.bx, m.ba, p);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

// ---------------------------------------------------------------------------
// Gather of the routed rows into X (one row per route, grouped) and of their
// routing weights: X[p] = input[rows[p]], W[p] = routing_weights[rows[p], cols[p]].
__global__ void gather_routes_kernel(const __nv_bfloat16* __restrict__ input, int64_t n_input,
                                     const __nv_bfloat16* __restrict__ weights, int64_t topk,
                                     const int64_t* __restrict__ rows,
                                     const int64_t* __restrict__ cols, int64_t total,
                                     int64_t hidden, __nv_bfloat16* __restrict__ x,
                                     __nv_bfloat16* __restrict__ w, int* err) {
  const int64_t vec_per_row = hidden / 8;  // 16-byte vectors
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total * vec_per_row;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pidx = i / vec_per_row, v = i % vec_per_row;
    const int64_t r = rows[pidx];
    if (r < 0 || r >= n_input) { atomicCAS(err, 0, DEV_BAD_INPUT); continue; }
    reinterpret_cast<uint4*>(x + pidx * hidden)[v] =
        reinterpret_cast<const uint4*>(input + r * hidden)[v];
    if (v == 0) {
      const int64_t c = cols[pidx];
      if (c < 0 || c >= topk) { atomicCAS(err, 0, DEV_BAD_INPUT); continue; }
      w[pidx] = weights[r * topk + c];
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
static int launch_phase(int phase, const CUtensorMap& wmap, const BMaps& bmaps,
                        const GemmParams& p, int device, cudaStream_t stream) {
  const int items = p.n_groups * p.m_tiles;
  if (items == 0) return FERRYB_OK;
  const int grid = items < num_sms(device) ? items : num_sms(device);
  if (phase == 1) {
    const int smem = smem_bytes<1>();
    FB_CUDA(cudaFuncSetAttribute(swiglu_gemm_kernel<1>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    swiglu_gemm_kernel<1><<<grid, kThreads, smem, stream>>>(wmap, bmaps, p);
  } else {
    const int smem = smem_bytes<2>();
    FB_CUDA(cudaFuncSetAttribute(swiglu_gemm_kernel<2>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    swiglu_gemm_kernel<2><<<grid, kThreads, smem, stream>>>(wmap, bmaps, p);
  }
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

static int make_bmaps(BMaps* maps, const void* base, int64_t rows, int64_t cols) {
  for (int i = 0; i < 4; ++i) {
    int s = make_map_2d_bf16(&maps->m[i], base, rows > 0 ? rows : 1, cols, cols * 2, 16u << i,
                             kBlockK);
    if (s) return s;
  }
  return FERRYB_OK;
}

int make_gemm_maps(GemmMaps* m, const void* cache, int64_t cache_slots, const void* x,
                   const void* act, int64_t rows_cap, int64_t hidden, int64_t inter) {
  FB_CHECK_ARG(hidden % kBlockM == 0 && inter % kBlockM == 0,
               "hidden (%lld) and intermediate (%lld) must be multiples of 128",
               (long long)hidden, (long long)inter);
  int s;
  if ((s = make_map_2d_bf16(&m->w1, cache, cache_slots * 3 * inter, hidden, hidden * 2, kBlockM,
                            kBlockK)))
    return s;
  if ((s = make_map_2d_bf16(&m->w1h, cache, cache_slots * 3 * inter, hidden, hidden * 2, kPackM,
                            kBlockK)))
    return s;
  if ((s = make_map_2d_bf16(&m->w2, cache, cache_slots * 3 * hidden, inter, inter * 2, kBlockM,
                            kBlockK)))
    return s;
  if ((s = make_bmaps(&m->bx, x, rows_cap, hidden))) return s;
  if ((s = make_bmaps(&m->ba, act, rows_cap, inter))) return s;
  m->hidden = hidden;
  m->inter = inter;
  return FERRYB_OK;
}

// Both phases over `groups` (device array of n_groups) with precomputed maps.
int swiglu_grouped_maps(const GemmMaps& m, const GemmGroup* groups, int n_groups,
                        const __nv_bfloat16* route_w, __nv_bfloat16* act, __nv_bfloat16* out,
                        int* err, cudaStream_t stream) {
  if (n_groups == 0) return FERRYB_OK;
  int device = 0;
  FB_CUDA(cudaGetDevice(&device));
  GemmParams p1{};
  p1.groups = groups;
  p1.n_groups = n_groups;
  p1.m_tiles = static_cast<int>(m.inter / kBlockM);
  p1.k_blocks = static_cast<int>(m.hidden / kBlockK);
  p1.rows_per_slot = static_cast<int>(3 * m.inter);
  p1.up_offset = static_cast<int>(m.inter);
  p1.out_cols = static_cast<int>(m.inter);
  p1.out = act;
  p1.err = err;
  int s;
  if ((s = launch_phase(1, m.w1, m.bx, p1, device, stream))) return s;
  GemmParams p2{};
  p2.groups = groups;
  p2.n_groups = n_groups;
  p2.m_tiles = static_cast<int>(m.hidden / kBlockM);
  p2.k_blocks = static_cast<int>(m.inter / kBlockK);
  p2.rows_per_slot = static_cast<int>(3 * m.hidden);
  p2.down_offset = static_cast<int>(2 * m.hidden);
  p2.out_cols = static_cast<int>(m.hidden);
  p2.out = out;
  p2.route_w = route_w;
  p2.err = err;
  return launch_phase(2, m.w2, m.ba, p2, device, stream);
}

// Shared by the public entry points: run both phases over `groups` (device),
// given X (routes already gathered), route weights, and scratch A.
int swiglu_grouped(const void* cache, int64_t cache_slots, const GemmGroup* groups,
                   int n_groups, int64_t total_routes, const __nv_bfloat16* x,
                   const __nv_bfloat16* route_w, __nv_bfloat16* act, __nv_bfloat16* out,
                   int64_t hidden, int64_t inter, int* err, cudaStream_t stream) {
  if (n_groups == 0 || total_routes == 0) return FERRYB_OK;
  GemmMaps m;
  int s = make_gemm_maps(&m, cache, cache_slots, x, act, total_routes, hidden, inter);
  if (s) return s;
  return swiglu_grouped_maps(m, groups, n_groups, route_w, act, out, err, stream);
}

static int64_t align256(int64_t b) { return (b + 255) & ~int64_t(255); }

// Workspace carve-up of ferryb_execute_experts (and of the no-allocation
// variant, which uses everything up to `err`).
struct ExecWs {
  int64_t x, act, w, groups, err, queue, total;
};
static ExecWs exec_ws(int64_t total, int64_t n_groups, int64_t hidden, int64_t inter) {
  ExecWs w{};
  w.x = 0;
  w.act = w.x + align256(total * hidden * 2);
  w.w = w.act + align256(total * inter * 2);
  w.groups = w.w + align256(total * 2);
  w.err = w.groups + align256(n_groups * (int64_t)sizeof(GemmGroup));
  w.queue = w.err + 256;  // the fused kernel's claim/done/dependency counters
  w.total = w.queue + align256((2 + n_groups) * 4);
  return w;
}

}  // namespace ferryb

using namespace ferryb;

extern "C" int64_t ferryb_execute_experts_workspace(int64_t total_routes, int64_t n_groups,
                                                    int64_t hidden, int64_t intermediate) {
  return exec_ws(total_routes, n_groups, hidden, intermediate).total;
}

extern "C" int ferryb_execute_experts(const void* cache, int64_t cache_slots, const void* input,
                                      int64_t n_input, const void* routing_weights, int64_t topk,
                                      const int64_t* slots, const int64_t* group_sizes,
                                      int64_t n_groups, const int64_t* rows, const int64_t* cols,
                                      int64_t hidden, int64_t intermediate, void* out,
                                      void* workspace, int64_t workspace_bytes,
                                      cudaStream_t stream) {
  FB_CHECK_ARG(n_groups >= 0 && hidden > 0 && intermediate > 0, "bad sizes");
  FB_CHECK_ARG(n_groups == 0 || (slots && group_sizes), "slots/group_sizes required");
  int64_t total = 0;
  std::vector<GemmGroup> host_groups(static_cast<size_t>(n_groups));
  for (int64_t i = 0; i < n_groups; ++i) {
    FB_CHECK_ARG(slots[i] >= 0 && slots[i] < cache_slots, "slot %lld out of range [0, %lld)",
                 (long long)slots[i], (long long)cache_slots);
    FB_CHECK_ARG(group_sizes[i] >= 0, "negative group size");
    host_groups[i] = GemmGroup{static_cast<int32_t>(slots[i]), static_cast<int32_t>(total),
                               static_cast<int32_t>(group_sizes[i]), static_cast<int32_t>(i)};
    total += group_sizes[i];
  }
  if (total == 0) return FERRYB_OK;
  FB_CHECK_ARG(cache && input && routing_weights && rows && cols && out, "null pointer");
  const ExecWs ws = exec_ws(total, n_groups, hidden, intermediate);
  FB_CHECK_ARG(workspace && workspace_bytes >= ws.total, "workspace too small (%lld < %lld)",
               (long long)workspace_bytes, (long long)ws.total);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  auto* x = reinterpret_cast<__nv_bfloat16*>(base + ws.x);
  auto* act = reinterpret_cast<__nv_bfloat16*>(base + ws.act);
  auto* w = reinterpret_cast<__nv_bfloat16*>(base + ws.w);
  auto* groups = reinterpret_cast<GemmGroup*>(base + ws.groups);
  int* err = reinterpret_cast<int*>(base + ws.err);
  FB_CUDA(cudaMemsetAsync(err, 0, sizeof(int), stream));
  FB_CUDA(cudaMemcpyAsync(groups, host_groups.data(), n_groups * sizeof(GemmGroup),
                          cudaMemcpyHostToDevice, stream));
  const int64_t work = total * (hidden / 8);
  int blocks = static_cast<int>((work + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  gather_routes_kernel<<<blocks, 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(input), n_input,
      static_cast<const __nv_bfloat16*>(routing_weights), topk, rows, cols, total, hidden, x, w,
      err);
  FB_LAUNCH_CHECK();
  // both phases of every group in one launch of the fused kernel (the layer
  // executor's kernel; all groups cached, no readiness waits)
  GemmMaps maps;
  int s = make_gemm_maps(&maps, cache, cache_slots, x, act, total, hidden, intermediate);
  if (s) return s;
  int* queue = reinterpret_cast<int*>(base + ws.queue);
  FB_CUDA(cudaMemsetAsync(queue, 0, (2 + n_groups) * sizeof(int), stream));
  s = swiglu_fused_launch(maps, groups, static_cast<int>(n_groups), static_cast<int>(n_groups),
                          nullptr, nullptr, 0, queue, w, act, static_cast<__nv_bfloat16*>(out), err,
                          stream);
  if (s) return s;
  // Synchronous status check of the device error word (compat API semantics:
  // errors surface at the call, like the reference's TORCH_CHECKs).
  int h_err = 0;
  FB_CUDA(cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, stream));
  FB_CUDA(cudaStreamSynchronize(stream));
  if (h_err) return fail(FERRYB_EDEVICE, "execute_experts: device error %d", h_err);
  return FERRYB_OK;
}

// ---------------------------------------------------------------------------
// execute_experts without any allocation: the scratch (gathered rows,
// activations, route weights, group table, error word) lives in a fixed
// array inside this library instead of a caller-provided workspace.  For
// callers that cannot allocate device memory at all -- for example a host
// application that has already handed the whole GPU to its own memory pool,
// or a plugin reached through a C binding (cgo, JNI) with no device
// allocator of its own.
namespace ferryb {

// 4 MiB per GPU, held for the life of the process by every process that loads
// the library (the cost of offering this entry point).
constexpr int64_t kNoAllocScratchBytes = int64_t(4) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// In host code `g_noalloc_scratch` only names the symbol; its device address
// is looked up once per device, with that device current.
static std::mutex g_noalloc_mu;
static void* g_noalloc_addr[64] = {};

static int noalloc_scratch(void** out) {
  int device = 0;
  FB_CUDA(cudaGetDevice(&device));
  FB_CHECK_ARG(device >= 0 && device < 64, "execute_experts_noalloc: device index %d", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[device]) {
    void* p = nullptr;
    FB_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_addr[device] = p;
  }
  *out = g_noalloc_addr[device];
  return FERRYB_OK;
}

}  // namespace ferryb

extern "C" int64_t ferryb_execute_experts_noalloc_limit(void) { return ferryb::kNoAllocScratchBytes; }

extern "C" int ferryb_execute_experts_noalloc(const void* cache, int64_t cache_slots,
                                              const void* input, int64_t n_input,
                                              const void* routing_weights, int64_t topk,
                                              const int64_t* slots, const int64_t* group_sizes,
                                              int64_t n_groups, const int64_t* rows,
                                              const int64_t* cols, int64_t hidden,
                                              int64_t intermediate, void* out,
                                              cudaStream_t stream) {
  constexpr int64_t kMaxGroups = 1024;
  FB_CHECK_ARG(n_groups >= 0 && n_groups <= kMaxGroups && hidden > 0 && intermediate > 0,
               "execute_experts_noalloc: bad sizes (at most %lld groups)", (long long)kMaxGroups);
  FB_CHECK_ARG(n_groups == 0 || (slots && group_sizes), "slots/group_sizes required");
  GemmGroup host_groups[kMaxGroups];  // on the stack: no heap allocation either
  int64_t total = 0;
  for (int64_t i = 0; i < n_groups; ++i) {
    FB_CHECK_ARG(slots[i] >= 0 && slots[i] < cache_slots, "slot %lld out of range [0, %lld)",
                 (long long)slots[i], (long long)cache_slots);
    FB_CHECK_ARG(group_sizes[i] >= 0, "negative group size");
    host_groups[i] = GemmGroup{static_cast<int32_t>(slots[i]), static_cast<int32_t>(total),
                               static_cast<int32_t>(group_sizes[i]), static_cast<int32_t>(i)};
    total += group_sizes[i];
  }
  if (total == 0) return FERRYB_OK;
  FB_CHECK_ARG(cache && input && routing_weights && rows && cols && out, "null pointer");
  const ExecWs ws = exec_ws(total, n_groups, hidden, intermediate);
  // the two-launch GEMM needs the carve-up up to the error word's 256 bytes
  const int64_t need = ws.queue;
  if (need > kNoAllocScratchBytes)
    return fail(FERRYB_EINVAL,
                "execute_experts_noalloc: %lld routes of hidden %lld / intermediate %lld need "
                "%lld bytes of scratch, above the fixed %lld; use ferryb_execute_experts with a "
                "workspace",
                (long long)total, (long long)hidden, (long long)intermediate, (long long)need,
                (long long)kNoAllocScratchBytes);
  void* scratch = nullptr;
  int s = noalloc_scratch(&scratch);
  if (s) return s;
  uint8_t* base = static_cast<uint8_t*>(scratch);
  auto* x = reinterpret_cast<__nv_bfloat16*>(base + ws.x);
  auto* act = reinterpret_cast<__nv_bfloat16*>(base + ws.act);
  auto* w = reinterpret_cast<__nv_bfloat16*>(base + ws.w);
  auto* groups = reinterpret_cast<GemmGroup*>(base + ws.groups);
  int* err = reinterpret_cast<int*>(base + ws.err);
  // the array keeps the previous call's contents: the error word starts at zero
  FB_CUDA(cudaMemsetAsync(err, 0, sizeof(int), stream));
  FB_CUDA(cudaMemcpyAsync(groups, host_groups, n_groups * sizeof(GemmGroup),
                          cudaMemcpyHostToDevice, stream));
  const int64_t work = total * (hidden / 8);
  int blocks = static_cast<int>((work + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  gather_routes_kernel<<<blocks, 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(input), n_input,
      static_cast<const __nv_bfloat16*>(routing_weights), topk, rows, cols, total, hidden, x, w,
      err);
  FB_LAUNCH_CHECK();
  s = swiglu_grouped(cache, cache_slots, groups, static_cast<int>(n_groups), total, x, w, act,
                     static_cast<__nv_bfloat16*>(out), hidden, intermediate, err, stream);
  if (s) return s;
  int h_err = 0;
  FB_CUDA(cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, stream));
  FB_CUDA(cudaStreamSynchronize(stream));
  if (h_err) return fail(FERRYB_EDEVICE, "execute_experts_noalloc: device error %d", h_err);
  return FERRYB_OK;
}
