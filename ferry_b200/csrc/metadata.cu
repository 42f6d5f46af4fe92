// metadata.cu -- device forms of the reference's routing-metadata helpers for
// callers that compose their own layer flow (the fused executor does the same
// work inside kernels 1 and 2).
//
//   ferryb_history_update / ferryb_history_scores
//       GateHistory.update / .scores (ferry/metadata.py:15-38): a per-layer
//       ring of the W most recent history rows (float64), replaced by the
//       last W rows when at least W arrive, else appended at the head; scores
//       are float32(sum over the W ring slots, in slot order, / max(1, count)).
//   ferryb_symm_allgather / ferryb_symm_wait
//       the all_gather_into_tensor of RouteGather.collect (ferry/metadata.py:
//       67-76) as P2P stores into every rank's symmetric buffer plus a
//       per-rank sequence flag (system-scope release), and a bounded wait on
//       this rank's flags.
#include "common.cuh"

namespace ferryb {

constexpr int kMetaThreads = 1024;

__global__ void __launch_bounds__(kMetaThreads)
    history_update_kernel(double* rows, int64_t* count, int64_t* head, int W, int E, int layer,
                          const double* probs, int64_t n) {
  double* ring = rows + (size_t)layer * W * E;
  __shared__ int64_t h0;
  if (threadIdx.x == 0) h0 = head[layer];
  __syncthreads();
  if (n >= W) {
    const double* src = probs + (size_t)(n - W) * E;
    for (int64_t i = threadIdx.x; i < (int64_t)W * E; i += blockDim.x) ring[i] = src[i];
    if (threadIdx.x == 0) {
      count[layer] = W;
      head[layer] = 0;
    }
  } else {
    for (int64_t i = threadIdx.x; i < n * E; i += blockDim.x) {
      const int64_t r = i / E, e = i % E;
      ring[((h0 + r) % W) * E + e] = probs[i];
    }
    if (threadIdx.x == 0) {
      head[layer] = (h0 + n) % W;
      const int64_t c = count[layer] + n;
      count[layer] = c < W ? c : W;
    }
  }
}

__global__ void history_scores_kernel(const double* rows, const int64_t* count, int W, int E,
                                      int layer, float* out) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  const double* ring = rows + (size_t)layer * W * E;
  double s = 0.0;
  for (int slot = 0; slot < W; ++slot) s = __dadd_rn(s, ring[(size_t)slot * E + e]);
  const int64_t c = count[layer];
  out[e] = __double2float_rn(__ddiv_rn(s, (double)(c > 1 ? c : 1)));
}

// One CTA: copy `bytes` of src into every rank's buffer at offset + rank *
// bytes, then raise this rank's flag (flag_offset + rank * 8) at every rank.
__global__ void __launch_bounds__(kMetaThreads)
    symm_allgather_kernel(const uintptr_t* peers, int world, int rank, int64_t offset,
                          const uint8_t* src, int64_t bytes, int64_t flag_offset, uint64_t seq) {
  const bool vec = bytes % 16 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 && offset % 16 == 0;
  for (int p = 0; p < world; ++p) {
    uint8_t* dst = reinterpret_cast<uint8_t*>(peers[p]) + offset + (size_t)rank * bytes;
    if (vec) {
      for (int64_t i = threadIdx.x; i < bytes / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
    } else {
      for (int64_t i = threadIdx.x; i < bytes; i += blockDim.x) dst[i] = src[i];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < world; ++p) {
      uint8_t* base = reinterpret_cast<uint8_t*>(peers[p]);
      st_release_sys(reinterpret_cast<uint64_t*>(base + flag_offset) + rank, seq);
    }
  }
}

__global__ void symm_wait_kernel(const uint8_t* local, int64_t flag_offset, int world, uint64_t seq,
                                 int* err) {
  if (threadIdx.x == 0)
    wait_flags_bounded(reinterpret_cast<const uint64_t*>(local + flag_offset), world, seq, err);
}

}  // namespace ferryb

using namespace ferryb;

extern "C" int ferryb_history_update(double* rows, int64_t* count, int64_t* head, int32_t layers,
                                     int32_t window, int32_t experts, int32_t layer,
                                     const double* probs, int64_t n_rows, cudaStream_t stream) {
  FB_CHECK_ARG(rows && count && head && layers > 0 && window > 0 && experts > 0,
               "history_update: bad arguments");
  FB_CHECK_ARG(layer >= 0 && layer < layers, "history_update: layer %d out of range", layer);
  FB_CHECK_ARG(n_rows >= 0 && (n_rows == 0 || probs), "history_update: bad rows");
  if (n_rows == 0) return FERRYB_OK;
  history_update_kernel<<<1, kMetaThreads, 0, stream>>>(rows, count, head, window, experts, layer,
                                                        probs, n_rows);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

extern "C" int ferryb_history_scores(const double* rows, const int64_t* count, int32_t layers,
                                     int32_t window, int32_t experts, int32_t layer, float* out,
                                     cudaStream_t stream) {
  FB_CHECK_ARG(rows && count && out && layers > 0 && window > 0 && experts > 0,
               "history_scores: bad arguments");
  FB_CHECK_ARG(layer >= 0 && layer < layers, "history_scores: layer %d out of range", layer);
  history_scores_kernel<<<(experts + 127) / 128, 128, 0, stream>>>(rows, count, window, experts,
                                                                   layer, out);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

extern "C" int ferryb_symm_allgather(const uint64_t* peer_bases, int32_t world, int32_t rank,
                                     int64_t offset, const void* src, int64_t bytes,
                                     int64_t flag_offset, uint64_t seq, cudaStream_t stream) {
  FB_CHECK_ARG(peer_bases && src && world >= 1 && world <= 32 && rank >= 0 && rank < world,
               "symm_allgather: bad arguments");
  FB_CHECK_ARG(bytes >= 0 && offset >= 0 && flag_offset >= 0 && flag_offset % 8 == 0,
               "symm_allgather: bad offsets");
  symm_allgather_kernel<<<1, kMetaThreads, 0, stream>>>(
      reinterpret_cast<const uintptr_t*>(peer_bases), world, rank, offset,
      static_cast<const uint8_t*>(src), bytes, flag_offset, seq);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

extern "C" int ferryb_symm_wait(const void* local_base, int64_t flag_offset, int32_t world,
                                uint64_t seq, int32_t* err, cudaStream_t stream) {
  FB_CHECK_ARG(local_base && err && world >= 1 && world <= 32 && flag_offset % 8 == 0,
               "symm_wait: bad arguments");
  symm_wait_kernel<<<1, 32, 0, stream>>>(static_cast<const uint8_t*>(local_base), flag_offset,
                                         world, seq, err);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}
