// h2d.cu -- kernel 3: expert fetch from the pinned host pool into HBM cache
// slots on copy-engine streams.
//
// Replaces H2DEngine (ferry/csrc/expert_ops.cpp:97-142) and its use in
// ferry/runtime.py:73-81, :87.  Semantics kept: a copy into a slot waits for
// the last compute that read the slot (mark_used), each slot has a "copy
// done" event, wait_host blocks on events, copies counts the transfers.
// Added for B200: copies round-robin over n_streams copy-engine streams, and
// wait_device makes a compute stream wait for one slot's copy (so the expert
// GEMM of that slot starts as soon as its own bytes have landed, with no host
// blocking); a pool with fewer rows than keys is read cyclically (key modulo
// pool_rows).
#include <vector>

#include "common.cuh"

struct ferryb_h2d {
  int device = 0;
  uint8_t* cache = nullptr;
  int64_t cache_slots = 0, row_bytes = 0;
  const uint8_t* pool = nullptr;
  int64_t pool_rows = 0;
  std::vector<cudaStream_t> streams;
  cudaStream_t flag_stream = nullptr;  // raises readiness flags after copies
  std::vector<cudaEvent_t> copy_done, used;
  std::vector<char> used_valid;
  int64_t copies = 0;
  int64_t next_stream = 0;
};

using namespace ferryb;

namespace {
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};
}  // namespace

namespace ferryb {
// Records `ev` on the copy stream the next fetch will use (which = 0) or on
// the stream of the last fetch issued (which = 1): timing of the copy lane.
int h2d_record_event(ferryb_h2d* h, cudaEvent_t ev, int which) {
  const size_t ns = h->streams.size();
  const int64_t i = which == 0 ? h->next_stream : h->next_stream - 1;
  FB_CUDA(cudaEventRecord(ev, h->streams[(size_t)((i % (int64_t)ns + ns) % ns)]));
  return FERRYB_OK;
}
}  // namespace ferryb

extern "C" int ferryb_h2d_create(void* cache, int64_t cache_slots, int64_t row_bytes,
                                 const void* pool, int64_t pool_rows, int32_t n_streams,
                                 ferryb_h2d** out) {
  FB_CHECK_ARG(out && cache && pool && cache_slots > 0 && row_bytes > 0 && pool_rows > 0,
               "h2d_create: bad arguments");
  FB_CHECK_ARG(n_streams >= 1 && n_streams <= 8, "h2d_create: n_streams must be in [1, 8]");
  cudaPointerAttributes attr{};
  FB_CUDA(cudaPointerGetAttributes(&attr, pool));
  FB_CHECK_ARG(attr.type == cudaMemoryTypeHost,
               "h2d_create: the expert pool must be pinned host memory");
  cudaPointerAttributes cattr{};
  FB_CUDA(cudaPointerGetAttributes(&cattr, cache));
  FB_CHECK_ARG(cattr.type == cudaMemoryTypeDevice, "h2d_create: the cache must be device memory");
  auto* h = new ferryb_h2d();
  h->device = cattr.device;
  DeviceGuard g(h->device);
  h->cache = static_cast<uint8_t*>(cache);
  h->cache_slots = cache_slots;
  h->row_bytes = row_bytes;
  h->pool = static_cast<const uint8_t*>(pool);
  h->pool_rows = pool_rows;
  h->streams.resize(n_streams);
  h->copy_done.assign(cache_slots, nullptr);
  h->used.assign(cache_slots, nullptr);
  h->used_valid.assign(cache_slots, 0);
  bool ok = cudaStreamCreateWithFlags(&h->flag_stream, cudaStreamNonBlocking) == cudaSuccess;
  for (auto& s : h->streams)
    ok = ok && cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess;
  if (!ok) {
    ferryb_h2d_destroy(h);  // releases what was created
    return fail(FERRYB_ECUDA, "h2d_create: cudaStreamCreate failed");
  }
  for (int64_t i = 0; i < cache_slots; ++i) {
    if (cudaEventCreateWithFlags(&h->copy_done[i], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&h->used[i], cudaEventDisableTiming) != cudaSuccess) {
      ferryb_h2d_destroy(h);
      return fail(FERRYB_ECUDA, "h2d_create: cudaEventCreate failed");
    }
  }
  *out = h;
  return FERRYB_OK;
}

extern "C" int ferryb_h2d_fetch(ferryb_h2d* h, const int64_t* slots, const int64_t* keys,
                                int64_t n) {
  FB_CHECK_ARG(h && (n == 0 || (slots && keys)), "h2d_fetch: bad arguments");
  DeviceGuard g(h->device);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t slot = slots[i], key = keys[i];
    FB_CHECK_ARG(slot >= 0 && slot < h->cache_slots, "h2d_fetch: slot %lld out of range",
                 (long long)slot);
    FB_CHECK_ARG(key >= 0, "h2d_fetch: negative key");
    cudaStream_t s = h->streams[h->next_stream++ % h->streams.size()];
    if (h->used_valid[slot]) FB_CUDA(cudaStreamWaitEvent(s, h->used[slot], 0));
    FB_CUDA(cudaMemcpyAsync(h->cache + slot * h->row_bytes,
                            h->pool + (key % h->pool_rows) * h->row_bytes, h->row_bytes,
                            cudaMemcpyHostToDevice, s));
    FB_CUDA(cudaEventRecord(h->copy_done[slot], s));
    ++h->copies;
  }
  return FERRYB_OK;
}

extern "C" int ferryb_h2d_wait_host(ferryb_h2d* h, const int64_t* slots, int64_t n) {
  FB_CHECK_ARG(h && (n == 0 || slots), "h2d_wait_host: bad arguments");
  for (int64_t i = 0; i < n; ++i) {
    FB_CHECK_ARG(slots[i] >= 0 && slots[i] < h->cache_slots, "h2d_wait_host: bad slot");
    FB_CUDA(cudaEventSynchronize(h->copy_done[slots[i]]));
  }
  return FERRYB_OK;
}

extern "C" int ferryb_h2d_wait_device(ferryb_h2d* h, const int64_t* slots, int64_t n,
                                      cudaStream_t stream) {
  FB_CHECK_ARG(h && (n == 0 || slots), "h2d_wait_device: bad arguments");
  for (int64_t i = 0; i < n; ++i) {
    FB_CHECK_ARG(slots[i] >= 0 && slots[i] < h->cache_slots, "h2d_wait_device: bad slot");
    FB_CUDA(cudaStreamWaitEvent(stream, h->copy_done[slots[i]], 0));
  }
  return FERRYB_OK;
}

extern "C" int ferryb_h2d_mark_used(ferryb_h2d* h, const int64_t* slots, int64_t n,
                                    cudaStream_t stream) {
  FB_CHECK_ARG(h && (n == 0 || slots), "h2d_mark_used: bad arguments");
  DeviceGuard g(h->device);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t slot = slots[i];
    FB_CHECK_ARG(slot >= 0 && slot < h->cache_slots, "h2d_mark_used: bad slot");
    FB_CUDA(cudaEventRecord(h->used[slot], stream));
    h->used_valid[slot] = 1;
  }
  return FERRYB_OK;
}

extern "C" int ferryb_h2d_synchronize(ferryb_h2d* h) {
  FB_CHECK_ARG(h, "h2d_synchronize: NULL engine");
  for (auto s : h->streams) FB_CUDA(cudaStreamSynchronize(s));
  FB_CUDA(cudaStreamSynchronize(h->flag_stream));
  return FERRYB_OK;
}

extern "C" int64_t ferryb_h2d_copies(const ferryb_h2d* h) { return h ? h->copies : -1; }

extern "C" int ferryb_h2d_destroy(ferryb_h2d* h) {
  if (!h) return FERRYB_OK;
  DeviceGuard g(h->device);
  for (auto s : h->streams) {
    if (!s) continue;
    cudaStreamSynchronize(s);
    cudaStreamDestroy(s);
  }
  if (h->flag_stream) {
    cudaStreamSynchronize(h->flag_stream);
    cudaStreamDestroy(h->flag_stream);
  }
  for (auto e : h->copy_done)
    if (e) cudaEventDestroy(e);
  for (auto e : h->used)
    if (e) cudaEventDestroy(e);
  delete h;
  return FERRYB_OK;
}

// Copies with readiness flags for a kernel that waits on the device: fetch i
// copies its whole row on a copy stream and records the slot's copy event; a
// separate flag stream waits for that event and stores flags[i] = value with
// cuStreamWriteValue32 (a stream memory operation with a memory barrier, run
// by the stream's front end, so no SM is involved).  Keeping the flag stores
// off the copy stream leaves the copies back to back.
extern "C" int ferryb_h2d_fetch_flagged(ferryb_h2d* h, const int64_t* slots, const int64_t* keys,
                                        int64_t n, uint32_t* flags, uint32_t value) {
  FB_CHECK_ARG(h && (n == 0 || (slots && keys && flags)), "h2d_fetch_flagged: bad arguments");
  PFN_writeValue32 wv = write_value32_fn();
  if (!wv) return fail(FERRYB_ECUDA, "cuStreamWriteValue32 is unavailable");
  DeviceGuard g(h->device);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t slot = slots[i], key = keys[i];
    FB_CHECK_ARG(slot >= 0 && slot < h->cache_slots, "h2d_fetch_flagged: slot out of range");
    FB_CHECK_ARG(key >= 0, "h2d_fetch_flagged: negative key");
    cudaStream_t s = h->streams[h->next_stream++ % h->streams.size()];
    if (h->used_valid[slot]) FB_CUDA(cudaStreamWaitEvent(s, h->used[slot], 0));
    FB_CUDA(cudaMemcpyAsync(h->cache + slot * h->row_bytes,
                            h->pool + (key % h->pool_rows) * h->row_bytes, h->row_bytes,
                            cudaMemcpyHostToDevice, s));
    FB_CUDA(cudaEventRecord(h->copy_done[slot], s));
    FB_CUDA(cudaStreamWaitEvent(h->flag_stream, h->copy_done[slot], 0));
    if (wv((CUstream)h->flag_stream, (CUdeviceptr)(flags + i), value, 0) != CUDA_SUCCESS)
      return fail(FERRYB_ECUDA, "cuStreamWriteValue32 failed");
    ++h->copies;
  }
  return FERRYB_OK;
}

namespace ferryb {
// Copies of whole expert rows with two readiness flags each: flags_a[i] for
// bytes [0, split), flags_b[i] for the whole row.  The last fetch of the call
// is copied in two parts, so with split = the gate + up rows its expert GEMM
// starts the gate/up tiles while the down rows are still on the link; the
// others raise both flags after one copy.  The slot's copy event follows the
// whole row (wait_host / wait_device see it complete).
int h2d_fetch_split_flagged(ferryb_h2d* h, const int64_t* slots, const int64_t* keys, int64_t n,
                            uint32_t* flags_a, uint32_t* flags_b, uint32_t value, int64_t split,
                            bool split_last) {
  FB_CHECK_ARG(h && (n == 0 || (slots && keys && flags_a && flags_b)),
               "h2d_fetch_split_flagged: bad arguments");
  FB_CHECK_ARG(split > 0 && split < h->row_bytes && split % 16 == 0,
               "h2d_fetch_split_flagged: split must be inside the row and 16-byte aligned");
  PFN_writeValue32 wv = write_value32_fn();
  if (!wv) return fail(FERRYB_ECUDA, "cuStreamWriteValue32 is unavailable");
  DeviceGuard g(h->device);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t slot = slots[i], key = keys[i];
    FB_CHECK_ARG(slot >= 0 && slot < h->cache_slots, "h2d_fetch_split_flagged: slot out of range");
    FB_CHECK_ARG(key >= 0, "h2d_fetch_split_flagged: negative key");
    cudaStream_t s = h->streams[h->next_stream++ % h->streams.size()];
    if (h->used_valid[slot]) FB_CUDA(cudaStreamWaitEvent(s, h->used[slot], 0));
    uint8_t* dst = h->cache + slot * h->row_bytes;
    const uint8_t* src = h->pool + (key % h->pool_rows) * h->row_bytes;
    // only the last fetch is split: each extra copy command costs the link a
    // little, and only the last one decides when the layer's GEMMs can end
    const bool two = split_last && i == n - 1;
    const int64_t parts[2][2] = {{0, two ? split : h->row_bytes}, {split, h->row_bytes - split}};
    for (int q = 0; q < (two ? 2 : 1); ++q) {
      FB_CUDA(cudaMemcpyAsync(dst + parts[q][0], src + parts[q][0], parts[q][1],
                              cudaMemcpyHostToDevice, s));
      FB_CUDA(cudaEventRecord(h->copy_done[slot], s));
      FB_CUDA(cudaStreamWaitEvent(h->flag_stream, h->copy_done[slot], 0));
      const bool whole = !two || q == 1;
      if ((q == 0 && wv((CUstream)h->flag_stream, (CUdeviceptr)(flags_a + i), value, 0) != CUDA_SUCCESS) ||
          (whole && wv((CUstream)h->flag_stream, (CUdeviceptr)(flags_b + i), value, 0) != CUDA_SUCCESS))
        return fail(FERRYB_ECUDA, "cuStreamWriteValue32 failed");
    }
    ++h->copies;
  }
  return FERRYB_OK;
}
}  // namespace ferryb
