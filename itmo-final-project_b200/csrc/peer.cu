// Set-up of the peer exchange buffers used by i4b_w4a16_matmul_allreduce (declared in include/int4_b200.h).
//
// Each rank of a tensor-parallel group owns one zero-filled buffer (layout in kernels.h) and maps every
// other rank's buffer into its address space through CUDA IPC, so the matmul's epilogue can store to
// it directly over NVLink.  These are set-up calls: unlike the rest of the C ABI they allocate and
// synchronise.  No multicast object is created; the kernels use plain peer stores and flag loads.
#include <cstring>

#include "common.cuh"
#include "kernels.h"

using namespace i4b;

namespace {
int peer_fail(cudaError_t e) { return cuda_error_status(e); }
}  // namespace

static_assert(sizeof(cudaIpcMemHandle_t) == I4B_IPC_HANDLE_BYTES, "CUDA IPC handle size");
static_assert(kArMaxRanks == I4B_PEER_MAX_RANKS, "peer group size");

extern "C" {

size_t i4b_peer_buffer_bytes(int64_t capacity) { return capacity < 0 ? 0 : ar_buffer_bytes(capacity); }

int i4b_peer_buffer_alloc(int64_t capacity, void** buffer) {
  if (!buffer || capacity < 0) return I4B_ERR_INVALID_ARG;
  *buffer = nullptr;
  const size_t bytes = ar_buffer_bytes(capacity);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return peer_fail(e);
  if ((e = cudaMemset(p, 0, bytes)) != cudaSuccess || (e = cudaDeviceSynchronize()) != cudaSuccess) {
    cudaFree(p);
    return peer_fail(e);
  }
  *buffer = p;
  return I4B_OK;
}

int i4b_peer_buffer_free(void* buffer) {
  if (!buffer) return I4B_OK;
  const cudaError_t e = cudaFree(buffer);
  return e == cudaSuccess ? I4B_OK : peer_fail(e);
}

int i4b_ipc_get_handle(void* buffer, void* handle) {
  if (!buffer || !handle) return I4B_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, buffer);
  if (e != cudaSuccess) return peer_fail(e);
  std::memcpy(handle, &h, sizeof(h));
  return I4B_OK;
}

int i4b_ipc_open_handle(const void* handle, void** buffer) {
  if (!handle || !buffer) return I4B_ERR_INVALID_ARG;
  *buffer = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(buffer, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? I4B_OK : peer_fail(e);
}

int i4b_ipc_close_handle(void* buffer) {
  if (!buffer) return I4B_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(buffer);
  return e == cudaSuccess ? I4B_OK : peer_fail(e);
}

}  // extern "C"
