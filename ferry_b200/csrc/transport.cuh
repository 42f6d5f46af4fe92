// transport.cuh -- arguments of the fused dispatch / combine kernels.
#pragma once
#include <stdint.h>

#include <algorithm>

#include "common.cuh"

namespace ferryb {

constexpr int kMaxTopK = 16;

// Offsets (bytes) inside one parity half of a rank's symmetric buffer; every
// rank uses the same offsets, so peer addresses are peer_base[p] + offset.
struct SymLayout {
  size_t recv_x, recv_w, recv_ids, ret, dflag, cflag, gather_ids, gather_hist, gflag, half;
};

struct FusedArgs {
  int world, rank, tokens_per_rank, topk, hdim, experts, parity;
  const uintptr_t* peer_base;  // device [world]: base of each rank's symmetric buffer
  void* local_base;            // this rank's symmetric buffer
  size_t buf_stride;           // bytes of one parity half
  size_t off_recv_x, off_recv_w, off_recv_ids, off_ret, off_dflag, off_cflag;
  // this layer's local inputs
  const __nv_bfloat16* hidden;   // [T, H]
  const __nv_bfloat16* weights;  // [T, K] routing weights in the router's column order
  const uint8_t* ids;            // [world*T, K] gathered ids
  const int32_t* dest;           // [world*T, K]
  const int32_t* peer_row;       // [T, world]
  // receiver layout
  const int64_t* rows;
  const int64_t* cols;
  const int32_t* n_routes_dev;
  const int32_t* n_recv_dev;
  const int32_t* recv_token;
  const int32_t* csr_pos;
  // expert operands / results
  __nv_bfloat16* x_sorted;    // [routes, H]
  __nv_bfloat16* route_w;     // [routes]
  const __nv_bfloat16* expert_out;  // [routes, H]
  __nv_bfloat16* out;         // [T, H]
  const __nv_bfloat16* addend;  // [T, H] or null: out = bf16(bf16(routed) + addend)
  int* err;
  // error words of this rank's expert GEMM and transport (2 ints) or null: when
  // either is set the combine writes NaN rows instead of sums, so output that
  // misses an expert's contribution never passes for a valid layer
  const int* poison;
  uint64_t wait_ns;  // bound on one flag wait (0: 2 s)
  int skip_signals;  // failure injection: 1 = no dispatch flags, 2 = no combine flags
  // device-clock spans (timing mode) or null
  unsigned long long *ts_dispatch, *ts_permute, *ts_combine, *ts_final;
};

SymLayout sym_layout(int world, int tokens_per_rank, int topk, int hidden, int experts);
int fused_dispatch(const FusedArgs& a, uint64_t seq, cudaStream_t stream);
int fused_permute(const FusedArgs& a, uint64_t seq, int n_routes_hint, cudaStream_t stream);
// after_stores (may be null): recorded once this rank's partials are stored,
// before the wait for the peers' partials
int fused_combine(const FusedArgs& a, uint64_t seq, int n_recv_hint, cudaStream_t stream,
                  cudaEvent_t after_stores = nullptr);
int ordered_segment_sum(const __nv_bfloat16* src, const int64_t* keys, int64_t n, int64_t n_keys,
                        int64_t H, __nv_bfloat16* dst, void* ws, int64_t ws_bytes,
                        cudaStream_t stream);
int64_t seg_workspace(int64_t n, int64_t n_keys);

}  // namespace ferryb
