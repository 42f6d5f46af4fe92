// common.cuh -- shared helpers of libferryb (status codes, error text, bf16,
// PTX wrappers for mbarriers, TMA and tcgen05 on sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "../../include/ferryb.h"

namespace ferryb {

// ---------------------------------------------------------------------------
// Error reporting: every entry point returns a FERRYB_* status and leaves a
// human-readable message behind for ferryb_last_error() (thread-local).
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);

#define FB_CHECK_ARG(cond, ...)                                   \
  do {                                                            \
    if (!(cond)) return ::ferryb::fail(FERRYB_EINVAL, __VA_ARGS__); \
  } while (0)

#define FB_CUDA(call)                                                                     \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess)                                                                \
      return ::ferryb::fail(FERRYB_ECUDA, "%s:%d %s: %s", __FILE__, __LINE__, #call,      \
                            cudaGetErrorString(e_));                                      \
  } while (0)

#define FB_LAUNCH_CHECK() FB_CUDA(cudaGetLastError())

// Device-side error flags written by kernels (bounded waits that gave up,
// violated invariants).  The host reads them with ferryb_*_status calls.
enum DeviceError : int {
  DEV_OK = 0,
  DEV_WAIT_TIMEOUT = 1,     // a bounded spin on a flag ran out
  DEV_CAPACITY = 2,         // missing experts exceed the admission capacity
  DEV_NO_SLOT = 3,          // eviction found no slot
  DEV_BAD_INPUT = 4,        // an id or index out of range
  DEV_LAYOUT_OVERFLOW = 5,  // a layout buffer was too small
};

// One expert's work in the grouped GEMM: its routes are rows
// [start, start + count) of the route-ordered operands.
struct GemmGroup {
  int32_t slot;    // cache slot holding the expert's weights
  int32_t start;   // first route row
  int32_t count;   // number of routes
  int32_t expert;  // expert id (informational)
};

// ---------------------------------------------------------------------------
// Driver entry points fetched through the runtime (the library must load on a
// machine without the CUDA driver, so it does not link libcuda).
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
PFN_encodeTiled encode_tiled_fn();

// cuStreamWriteValue32 (a flag store executed by the stream's front end, no SM
// needed) and whether the device supports stream memory operations.
typedef CUresult (*PFN_writeValue32)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
PFN_writeValue32 write_value32_fn();
int stream_mem_ops_supported(int device);
// h2d.cu: record an event on the copy lane (0: before the next fetch, 1:
// after the last fetch issued)
int h2d_record_event(ferryb_h2d* h, cudaEvent_t ev, int which);
// h2d.cu: whole-row copies raising flags_a[i] = value once bytes [0, split)
// have landed and flags_b[i] once the whole row has (with split_last, the
// last fetch of the call as two copies; every other fetch as one)
int h2d_fetch_split_flagged(ferryb_h2d* h, const int64_t* slots, const int64_t* keys, int64_t n,
                            uint32_t* flags_a, uint32_t* flags_b, uint32_t value, int64_t split,
                            bool split_last);

// 2D bf16 tensor map over a row-major [rows, cols] matrix (cols contiguous),
// box = [box_cols, box_rows], 128-byte swizzle (box_cols * 2 must be 128).
int make_map_2d_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                     uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_cols);

inline int num_sms(int device) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  return n > 0 ? n : 148;
}

// ---------------------------------------------------------------------------
// Device helpers
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and the caller records
// an error) if the phase did not complete within ~2^26 polls, so that a
// mis-programmed pipeline ends instead of hanging the GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < (1u << 26); ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2D TMA tile load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---- tcgen05 (5th-generation tensor cores, accumulators in TMEM) ----------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] x B[smem]^T, bf16 inputs, f32 accumulate, cta_group::1.
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32-bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor of a K-major operand tile written by TMA
// with the 128-byte swizzle: rows of 64 bf16 (128 B), 8-row core groups
// 1024 B apart.  Fields: start address >> 4 (bits 0-13), leading byte offset
// >> 4 (bits 16-29, unused for swizzled K-major, set to 1), stride byte
// offset >> 4 (bits 32-45), descriptor version 1 (bits 46-47), swizzle mode
// 2 = 128B (bits 61-63).  The tile base must be 1024-byte aligned.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B, f32 D, both K-major:
// D format f32 (bits 4-5 = 1), A bf16 (bits 7-9 = 1), B bf16 (bits 10-12 = 1),
// N >> 3 (bits 17-22), M >> 4 (bits 24-28).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(uint32_t m, uint32_t n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ uint32_t elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred;
}

// Acquire/release accesses at system scope (flags shared with peer GPUs and
// the copy engines).
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait until flags[0..n) all reach `seq` (system-scope acquire), giving up
// after `limit_ns` with DEV_WAIT_TIMEOUT in *err.  Called by one thread.
__device__ __forceinline__ bool wait_flags_bounded(const uint64_t* flags, int n, uint64_t seq,
                                                   int* err, uint64_t limit_ns = 2000000000ull) {
  for (int i = 0; i < n; ++i) {
    if (ld_acquire_sys(flags + i) >= seq) continue;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(flags + i) < seq) {
      __nanosleep(64);
      if (globaltimer_ns() - t0 > limit_ns) {
        atomicCAS(err, 0, 1 /* DEV_WAIT_TIMEOUT */);
        return false;
      }
    }
  }
  return true;
}

// Device-clock span of a launch (timing mode): ts[0] is lowered to the
// earliest CTA start, ts[1] raised to the latest CTA end; null = off.
__device__ __forceinline__ void span_begin(unsigned long long* ts) {
  if (ts && threadIdx.x == 0) atomicMin(ts, (unsigned long long)globaltimer_ns());
}
__device__ __forceinline__ void span_end(unsigned long long* ts) {
  if (ts && threadIdx.x == 0) atomicMax(ts + 1, (unsigned long long)globaltimer_ns());
}

// Programmatic dependent launch: a primary kernel lets the next kernel of its
// stream (launched with programmatic stream serialisation) start early; that
// kernel waits for the primary's completion and memory before it reads the
// primary's outputs.  Both are no-ops when the launches are not paired so.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace ferryb
