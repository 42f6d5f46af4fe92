/*
 * ferryb.h -- C ABI of libferryb, the B200 (sm_100a) implementation of
 * FERRY's per-MoE-layer hot path.
 *
 * Conventions
 *  - Every function returns FERRYB_OK (0) or a FERRYB_E* code; the message of
 *    the last failure on the calling thread is ferryb_last_error().
 *  - Pointers named d_* or documented as "device" are CUDA device pointers of
 *    the current device; "host" arrays are plain CPU memory.
 *  - Work is enqueued on the cudaStream_t passed in (the caller's current
 *    stream, as the reference's ATen ops use the current stream,
 *    ferry/csrc/expert_ops.cpp:126).  No entry point allocates device memory
 *    unless documented; scratch comes from a caller-provided workspace whose
 *    size a *_workspace() query returns.
 *  - bf16 means IEEE bfloat16 stored as uint16; int64 tensors are int64_t.
 *
 * Reference interfaces replaced (paths within the FERRY repository):
 *  ferry/csrc/expert_ops.cpp:144-157  pybind module ferry_expert_ops
 *  ferry/policy.py, ferry/quota.py, ferry/layout.py, ferry/metadata.py
 *  ferry/transport.py, ferry/runtime.py
 */
#ifndef FERRYB_H_
#define FERRYB_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FERRYB_VERSION 1

enum {
  FERRYB_OK = 0,
  FERRYB_EINVAL = 1,    /* bad argument (the reference's TORCH_CHECK / ValueError) */
  FERRYB_ECUDA = 2,     /* a CUDA runtime/driver call failed */
  FERRYB_EDEVICE = 3,   /* a kernel reported an error word (see ferryb_last_error) */
  FERRYB_ECAPACITY = 4, /* missing experts exceed the admission capacity
                           (the reference's assert, ferry/quota.py:63) */
  FERRYB_ETIMEOUT = 5,  /* a bounded device or host wait gave up */
  FERRYB_ESTATE = 6     /* call out of order (e.g. use after close) */
};

typedef struct CUstream_st* ferryb_stream_t; /* == cudaStream_t */

#if defined(__GNUC__)
#define FERRYB_API __attribute__((visibility("default")))
#else
#define FERRYB_API
#endif

/* Message of the last failure on this thread ("" if none). */
FERRYB_API const char* ferryb_last_error(void);
FERRYB_API int ferryb_version(void);
FERRYB_API int ferryb_device_sm_count(int device);

/* ------------------------------------------------------------------------
 * Kernel 5: routed-expert SwiGLU grouped GEMM (tcgen05 / TMEM / TMA).
 * Replaces execute_experts, ferry/csrc/expert_ops.cpp:16-45 (and silu_mul,
 * ferry/csrc/expert_ops.cu:6-25).
 *
 * cache:           device bf16 [cache_slots, 3*hidden*intermediate], rows
 *                  [gate I x H | up I x H | down H x I] (ferry/model.py:86-88)
 * input:           device bf16 [n_input, hidden]
 * routing_weights: device bf16 [n_input, topk]
 * slots, group_sizes: host int64 [n_groups]: cache slot and route count of
 *                  each group (the reference's `slots` and len(rows[i]))
 * rows, cols:      device int64 [sum(group_sizes)], the groups' rows/cols
 *                  concatenated in group order
 * out:             device bf16 [sum(group_sizes), hidden]; group i's outputs
 *                  are rows [offset_i, offset_i + group_sizes[i]), each
 *                  (silu(x Wg^T) * (x Wu^T)) Wd^T * w[row, col]
 * workspace:       device, >= ferryb_execute_experts_workspace(...) bytes
 * Synchronises `stream` before returning to report device-side errors.
 */
FERRYB_API int64_t ferryb_execute_experts_workspace(int64_t total_routes, int64_t n_groups, int64_t hidden,
                                         int64_t intermediate);
FERRYB_API int ferryb_execute_experts(const void* cache, int64_t cache_slots, const void* input,
                           int64_t n_input, const void* routing_weights, int64_t topk,
                           const int64_t* slots, const int64_t* group_sizes, int64_t n_groups,
                           const int64_t* rows, const int64_t* cols, int64_t hidden,
                           int64_t intermediate, void* out, void* workspace,
                           int64_t workspace_bytes, ferryb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FERRYB_H_ */
