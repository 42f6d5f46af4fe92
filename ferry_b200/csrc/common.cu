// common.cu -- error text, driver entry points and tensor-map construction.
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace ferryb {

static thread_local char g_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

PFN_encodeTiled encode_tiled_fn() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

int make_map_2d_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                     uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_cols) {
  PFN_encodeTiled enc = encode_tiled_fn();
  if (!enc) return fail(FERRYB_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride_bytes & 15))
    return fail(FERRYB_EINVAL, "tensor map base/stride must be 16-byte aligned");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                   strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FERRYB_ECUDA, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu box=%ux%u",
                (int)r, (unsigned long long)rows, (unsigned long long)cols, box_rows, box_cols);
  return FERRYB_OK;
}


PFN_writeValue32 write_value32_fn() {
  static PFN_writeValue32 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_writeValue32>(p);
  });
  return fn;
}

// Functional probe, once per device: a flag write by cuStreamWriteValue32 into
// a 4-byte buffer of our own, read back after a stream synchronisation.  Any
// failing call returns a status (the probe only touches its own memory).
int stream_mem_ops_supported(int device) {
  static int cached[64];
  static bool done[64];
  static std::mutex mu;
  if (device < 0 || device >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (done[device]) return cached[device];
  done[device] = true;
  cached[device] = 0;
  PFN_writeValue32 wv = write_value32_fn();
  if (!wv) return 0;
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return 0;
  if (prev != device && cudaSetDevice(device) != cudaSuccess) return 0;
  uint32_t* buf = nullptr;
  cudaStream_t st = nullptr;
  uint32_t host = 0;
  int ok = 0;
  if (cudaMalloc(&buf, sizeof(uint32_t)) == cudaSuccess &&
      cudaMemset(buf, 0, sizeof(uint32_t)) == cudaSuccess &&
      cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess &&
      wv((CUstream)st, (CUdeviceptr)buf, 0x5a5a1234u, 0) == CUDA_SUCCESS &&
      cudaStreamSynchronize(st) == cudaSuccess &&
      cudaMemcpy(&host, buf, sizeof(uint32_t), cudaMemcpyDeviceToHost) == cudaSuccess)
    ok = host == 0x5a5a1234u;
  if (st) cudaStreamDestroy(st);
  if (buf) cudaFree(buf);
  if (prev != device) cudaSetDevice(prev);
  cudaGetLastError();
  cached[device] = ok;
  return ok;
}

}  // namespace ferryb

extern "C" int ferryb_stream_mem_ops_supported(int device) {
  return ferryb::stream_mem_ops_supported(device);
}

extern "C" const char* ferryb_last_error(void) { return ferryb::g_error; }

extern "C" int ferryb_version(void) { return FERRYB_VERSION; }

extern "C" int ferryb_device_sm_count(int device) { return ferryb::num_sms(device); }
