// experts.cuh -- host interface of the grouped SwiGLU GEMM (see experts.cu).
#pragma once
#include "common.cuh"

namespace ferryb {

// Tensor maps of the B operand for box heights 16, 32, 64, 128.
struct BMaps {
  CUtensorMap m[4];
};

struct GemmMaps {
  CUtensorMap w1, w2;  // cache as [slots*3I, H] and [slots*3H, I] (128-row boxes)
  CUtensorMap w1h;     // [slots*3I, H] with 64-row boxes (the fused kernel's gate/up halves)
  BMaps bx, ba;        // X [rows_cap, H] and A [rows_cap, I]
  int64_t hidden, inter;
};

int make_gemm_maps(GemmMaps* m, const void* cache, int64_t cache_slots, const void* x,
                   const void* act, int64_t rows_cap, int64_t hidden, int64_t inter);
// Two-launch grouped SwiGLU with maps encoded for this call (cache = expert
// rows [slots, 3*H*I]); x [total_routes, H], route_w [total_routes].
int swiglu_grouped(const void* cache, int64_t cache_slots, const GemmGroup* groups, int n_groups,
                   int64_t total_routes, const __nv_bfloat16* x, const __nv_bfloat16* route_w,
                   __nv_bfloat16* act, __nv_bfloat16* out, int64_t hidden, int64_t inter,
                   int* err, cudaStream_t stream);
int swiglu_grouped_maps(const GemmMaps& m, const GemmGroup* groups, int n_groups,
                        const __nv_bfloat16* route_w, __nv_bfloat16* act, __nv_bfloat16* out,
                        int* err, cudaStream_t stream);

// Both phases of every group in one persistent launch; groups [n_hit,
// n_groups) are fetched experts whose phase-1 tiles wait for ready[j] >=
// ready_value (raised when fetch j's gate/up rows have landed) and phase-2
// tiles for ready_down[j] (its down rows; null = ready); ready null: no
// readiness wait, the stream already waited for the copies; each wait gives
// up after ready_wait_ns, 0 = the default 2 s, and reports DEV_WAIT_TIMEOUT
// in *err.  queue_dep: device
// scratch of 2 + n_groups ints, zero before the first launch; every launch
// leaves it zeroed again (its last CTA resets it).  ts: null, or device [2]
// that the launch lowers to its earliest CTA start and raises to its latest CTA
// end (globaltimer ns; start ~0 and end 0 beforehand).
int swiglu_fused_launch(const GemmMaps& m, const GemmGroup* groups, int n_groups, int n_hit,
                        const uint32_t* ready, const uint32_t* ready_down, uint32_t ready_value,
                        int* queue_dep,
                        const __nv_bfloat16* route_w, __nv_bfloat16* act, __nv_bfloat16* out,
                        int* err, cudaStream_t stream, unsigned long long* ts = nullptr,
                        uint64_t ready_wait_ns = 0);

}  // namespace ferryb
