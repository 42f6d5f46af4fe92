// symm.cu -- symmetric device buffers shared by the ranks of one node.
//
// Each rank allocates one buffer of identical size with cudaMalloc and exports
// it with a CUDA IPC handle; the handles are exchanged on the host (by the
// caller, e.g. torch.distributed) and every rank opens its peers' buffers.
// Kernels then read and write peers' memory directly over NVLink/NVSwitch.
// Only plain loads and stores are used on peer memory (no TMA).
#include <cstring>

#include "common.cuh"

using namespace ferryb;

extern "C" int ferryb_symm_alloc(int64_t bytes, void** ptr, void* handle_out /*64 bytes*/) {
  FB_CHECK_ARG(bytes > 0 && ptr, "symm_alloc: bad arguments");
  void* p = nullptr;
  FB_CUDA(cudaMalloc(&p, (size_t)bytes));
  FB_CUDA(cudaMemset(p, 0, (size_t)bytes));
  if (!handle_out) {  // one rank: nothing to export
    *ptr = p;
    return FERRYB_OK;
  }
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(FERRYB_ECUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return FERRYB_OK;
}

extern "C" int ferryb_symm_open(const void* handle /*64 bytes*/, void** ptr) {
  FB_CHECK_ARG(handle && ptr, "symm_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  FB_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return FERRYB_OK;
}

extern "C" int ferryb_symm_close(void* peer_ptr) {
  FB_CHECK_ARG(peer_ptr, "symm_close: NULL");
  FB_CUDA(cudaIpcCloseMemHandle(peer_ptr));
  return FERRYB_OK;
}

extern "C" int ferryb_symm_free(void* ptr) {
  FB_CHECK_ARG(ptr, "symm_free: NULL");
  FB_CUDA(cudaFree(ptr));
  return FERRYB_OK;
}
