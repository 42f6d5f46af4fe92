// router.cu -- kernel 1: top-k router fused with the all-gather of routing
// metadata and of the per-rank demand histogram.
//
// Replaces the router of the MoE hooks (ferry/model.py:137-148 for Qwen3:
// bf16 logits, float32 softmax, top-k, renormalisation, bf16 weights; the
// DeepSeek-V2 greedy gate consumed by ferry/model.py:151-158: float32 logits
// and softmax, top-k, routed_scaling_factor) and RouteGather.collect's
// all_gather_into_tensor + blocking D2H copy (ferry/metadata.py:67-83).
//
// One CTA per token.  Each warp forms dot products of the token with a
// stripe of gate rows (16-byte loads, float32 accumulation); the softmax and
// the top-k (ties to the lower expert id) run in shared memory / one warp.
// The token's k ids go straight into every rank's gather buffer (plain stores;
// over NVLink for peers), its expert counts into a per-layer histogram.  The
// last CTA to finish (threadfence + done counter, no spinning) writes this
// rank's histogram into every rank's buffer and raises this rank's gather
// flag there with a system-scope release.
#include <math_constants.h>

#include "common.cuh"
#include "router.cuh"

namespace ferryb {

constexpr int kRouterThreads = 1024;  // 32 warps: a few experts per warp

// Optional phase stamps of the router (profiling aid; NULL = off), over all
// CTAs: [0] earliest start, [1] latest end of the logits, [2] of the softmax
// and top-k, [3] latest end.
__device__ unsigned long long* g_router_ts = nullptr;
#define ROUTER_TS(k)                                                              \
  do {                                                                            \
    if (threadIdx.x == 0 && g_router_ts) {                                        \
      if ((k) == 0) atomicMin(g_router_ts, (unsigned long long)globaltimer_ns()); \
      else atomicMax(g_router_ts + (k), (unsigned long long)globaltimer_ns());    \
    }                                                                             \
  } while (0)

__global__ void __launch_bounds__(kRouterThreads)
    router_kernel(const RouterArgs a, uint64_t seq) {
  __shared__ float logit[kMaxRouterExperts];
  __shared__ __align__(16) __nv_bfloat16 xs[kMaxRouterHidden];
  __shared__ float red[kRouterThreads / 32];
  __shared__ int top_id[kMaxRouterK];
  __shared__ float top_p[kMaxRouterK];
  __shared__ int is_last;
  const int t = blockIdx.x;
  const int H = a.hdim, E = a.experts, K = a.topk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const __nv_bfloat16* x = a.hidden + (size_t)t * H;
  pdl_launch_dependents();  // the planner may take its SM and wait there
  ROUTER_TS(0);
  span_begin(a.ts);

  if (a.mode == 2) {
    // routing given by the caller: gather only
    if (threadIdx.x < K) {
      const int j = threadIdx.x;
      const int64_t e = a.given_selected[(size_t)t * K + j];
      top_id[j] = (e >= 0 && e < E) ? (int)e : 0;
      a.weights[(size_t)t * K + j] = a.given_weights[(size_t)t * K + j];
      if (a.selected) a.selected[(size_t)t * K + j] = e;
      atomicAdd(&a.hist_local[top_id[j]], 1);
    }
    if (a.prob_tail > 0 && t >= a.tokens_per_rank - a.prob_tail && a.given_probs) {
      const int i = t - (a.tokens_per_rank - a.prob_tail);
      const float* src = a.given_probs + (size_t)(a.n_given_probs - a.prob_tail + i) * E;
      for (int q = threadIdx.x; q < a.world * E; q += blockDim.x) {
        const int p = q / E, e = q % E;
        uint8_t* base = reinterpret_cast<uint8_t*>(a.peer_base[p]) + a.parity * a.buf_stride;
        reinterpret_cast<float*>(base + a.off_prob)[((size_t)a.rank * a.prob_tail + i) * E + e] = src[e];
      }
    }
    __syncthreads();
  } else {
  // ---- logits ----
  // the token row once into shared memory; then each warp takes experts
  // e = warp, warp + 32, ...; a lane issues all its 16-byte weight loads of
  // an expert (8 at a time) before the FMAs, so loads overlap.
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x)
    reinterpret_cast<uint4*>(xs)[v] = reinterpret_cast<const uint4*>(x)[v];
  __syncthreads();
  const int nch = H / 256;  // 16-byte chunks per lane
  for (int e = warp; e < E; e += nw) {
    const __nv_bfloat16* w = a.gate + (size_t)e * H;
    float acc = 0.0f;
    for (int c0 = 0; c0 < nch; c0 += 8) {
      uint4 wv[8];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (c0 + q < nch) wv[q] = *reinterpret_cast<const uint4*>(w + (c0 + q) * 256 + lane * 8);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (c0 + q < nch) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xs + (c0 + q) * 256 + lane * 8);
          const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv);
          const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wv[q]);
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float2 xf = __bfloat1622float2(xp[h]);
            const float2 wf = __bfloat1622float2(wp[h]);
            acc = fmaf(xf.x, wf.x, acc);
            acc = fmaf(xf.y, wf.y, acc);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      if (a.bias) acc += a.bias[e];
      // Qwen3: the gate Linear outputs bf16 logits; DeepSeek-V2: float32.
      logit[e] = a.mode == 0 ? bf16_round(acc) : acc;
    }
  }
  __syncthreads();

  ROUTER_TS(1);
  // ---- softmax (float32), top-k and weights: warp 0 alone --------------
  // lane l holds logits l, l + 32, ... (E <= kMaxRouterExperts)
  if (warp == 0) {
    constexpr int kPer = kMaxRouterExperts / 32;
    float v[kPer];
    float m = -CUDART_INF_F;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? logit[e] : -CUDART_INF_F;
      m = fmaxf(m, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? expf(v[i] - m) : 0.0f;
      s += v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      if (e < E) {
        v[i] = v[i] / s;  // probabilities
        logit[e] = v[i];
      } else {
        v[i] = -1.0f;
      }
    }
    // top-k: largest probability, ties to the lower id
    for (int j = 0; j < K; ++j) {
      float bv = -2.0f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int e = lane + 32 * i;
        if (v[i] > bv || (v[i] == bv && e < bi)) { bv = v[i]; bi = e; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) { top_id[j] = bi; top_p[j] = bv; }
      if ((bi & 31) == lane) v[bi >> 5] = -1.0f;
    }
    __syncwarp();
    if (lane == 0) {
      float norm = 1.0f;
      if (a.mode == 0 && a.norm_topk) {
        float sum = 0.0f;
        for (int j = 0; j < K; ++j) sum += top_p[j];
        norm = sum;
      }
      for (int j = 0; j < K; ++j) {
        float w = a.mode == 0 ? (a.norm_topk ? top_p[j] / norm : top_p[j]) : top_p[j] * a.scaling;
        a.weights[(size_t)t * K + j] = __float2bfloat16_rn(w);
        if (a.selected) a.selected[(size_t)t * K + j] = top_id[j];
        atomicAdd(&a.hist_local[top_id[j]], 1);
      }
    }
  }
  __syncthreads();  // probabilities in logit[], top_id[] complete
  if (a.probs_out)
    for (int e = threadIdx.x; e < E; e += blockDim.x) a.probs_out[(size_t)t * E + e] = logit[e];
  if (a.prob_tail > 0 && t >= a.tokens_per_rank - a.prob_tail) {
    const int i = t - (a.tokens_per_rank - a.prob_tail);
    for (int q = threadIdx.x; q < a.world * E; q += blockDim.x) {
      const int p = q / E, e = q % E;
      uint8_t* base = reinterpret_cast<uint8_t*>(a.peer_base[p]) + a.parity * a.buf_stride;
      reinterpret_cast<float*>(base + a.off_prob)[((size_t)a.rank * a.prob_tail + i) * E + e] = logit[e];
    }
  }
  __syncthreads();
  }  // mode 0 / 1

  ROUTER_TS(2);
  // ---- all-gather of the ids: this token's k bytes into every rank ----
  if (threadIdx.x < a.world * K) {
    const int p = threadIdx.x / K, j = threadIdx.x % K;
    uint8_t* base = reinterpret_cast<uint8_t*>(a.peer_base[p]) + a.parity * a.buf_stride;
    base[a.off_ids + ((size_t)a.rank * a.tokens_per_rank + t) * K + j] = (uint8_t)top_id[j];
  }
  // With one rank the planner, next on the stream, reads the histogram and
  // the ids this kernel wrote (the kernel boundary orders them): no flags.
  ROUTER_TS(3);
  span_end(a.ts);
  if (a.world == 1) return;
  // ---- last CTA: histogram + flags ----
  // One system-scope fence per CTA, by thread 0 after a CTA barrier (the
  // barrier orders the CTA's peer stores before it), then the done counter.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    is_last = atomicAdd(a.done, 1u) == (unsigned)gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  for (int i = threadIdx.x; i < a.world * E; i += blockDim.x) {
    const int p = i / E, e = i % E;
    uint8_t* base = reinterpret_cast<uint8_t*>(a.peer_base[p]) + a.parity * a.buf_stride;
    reinterpret_cast<int*>(base + a.off_hist)[(size_t)a.rank * E + e] =
        atomicAdd(&a.hist_local[e], 0);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) a.hist_local[e] = 0;  // next layer
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < a.world; ++p) {
      uint8_t* base = reinterpret_cast<uint8_t*>(a.peer_base[p]) + a.parity * a.buf_stride;
      st_release_sys(reinterpret_cast<uint64_t*>(base + a.off_flag) + a.rank, seq);
    }
    *a.done = 0;
  }
}

int router_launch(const RouterArgs& a, uint64_t seq, cudaStream_t stream) {
  FB_CHECK_ARG(a.experts >= 1 && a.experts <= kMaxRouterExperts, "router: experts must be <= %d",
               kMaxRouterExperts);
  FB_CHECK_ARG(a.topk >= 1 && a.topk <= kMaxRouterK && a.topk <= a.experts, "router: bad topk");
  FB_CHECK_ARG(a.hdim % 256 == 0 && a.hdim <= kMaxRouterHidden,
               "router: hidden must be a multiple of 256 and at most %d", kMaxRouterHidden);
  FB_CHECK_ARG(a.world * a.topk <= kRouterThreads, "router: world * topk too large");
  if (a.tokens_per_rank == 0) return FERRYB_OK;
  router_kernel<<<a.tokens_per_rank, kRouterThreads, 0, stream>>>(a, seq);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

}  // namespace ferryb

extern "C" int ferryb_debug_router_timestamps(void* dev_ptr) {
  FB_CUDA(cudaMemcpyToSymbol(ferryb::g_router_ts, &dev_ptr, sizeof(void*)));
  return FERRYB_OK;
}
