// router.cuh -- arguments of the fused router (see router.cu).
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace ferryb {

constexpr int kMaxRouterExperts = 256;
constexpr int kMaxRouterK = 16;
constexpr int kMaxRouterHidden = 8192;

struct RouterArgs {
  int world, rank, tokens_per_rank, topk, hdim, experts, parity;
  int mode;        // 0: Qwen3 (bf16 logits, optional renormalisation), 1: DeepSeek-V2 (f32),
                   // 2: ids/weights given by the caller (gather only)
  int norm_topk;   // Qwen3 norm_topk_prob
  float scaling;   // DeepSeek-V2 routed_scaling_factor
  const __nv_bfloat16* hidden;  // [T, H]
  const __nv_bfloat16* gate;    // [E, H]
  const float* bias;            // [E] or null (synthetic popularity bias)
  __nv_bfloat16* weights;       // [T, K] out
  int64_t* selected;            // [T, K] out, optional
  float* probs_out;             // [T, E] out, optional (probability score)
  int* hist_local;              // [E] scratch, zero between layers
  unsigned* done;               // [1] scratch, zero between layers
  const int64_t* given_selected;      // [T, K] (mode 2)
  const __nv_bfloat16* given_weights; // [T, K] (mode 2)
  const float* given_probs;           // [n_given_probs, E] router probabilities (mode 2, optional)
  int n_given_probs;
  int prob_tail;                      // rows per rank of the probability history, 0 = off
  const uintptr_t* peer_base;   // [world] symmetric buffer bases
  size_t buf_stride, off_ids, off_hist, off_flag, off_prob;
  unsigned long long* ts;       // device-clock span (timing mode) or null
};

int router_launch(const RouterArgs& a, uint64_t seq, cudaStream_t stream);

}  // namespace ferryb
