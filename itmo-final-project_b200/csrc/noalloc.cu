// i4b_w4a16_matmul_noalloc: the W4A16 matmul for callers that cannot allocate device memory.
//
// Some callers have no allocator to hand: a plugin loaded into a host program
// that owns every cudaMalloc (and forbids others), code running where an
// allocation could block or fail mid-step, or a C caller that has no torch
// caching allocator behind it.  They cannot provide the workspace that
// i4b_w4a16_matmul takes.  This entry point instead uses one scratch array
// compiled into the library, g_noalloc_scratch below, and otherwise runs the
// exact same dispatch and kernels as i4b_w4a16_matmul.
//
// The array lives in the module's global memory, so every GPU that loads the
// library holds its I4B_NOALLOC_SCRATCH_BYTES until the process exits.  Host
// code cannot pass the array's name to a kernel (on the host it is only a
// stand-in symbol); its device address is looked up once per device with
// cudaGetSymbolAddress, with that device current, on the first call made on
// that device.  Make that first call before any stream capture begins.
//
// The looked-up address is kept for the life of the process: cudaDeviceReset
// between calls is not supported (the module reloads, possibly elsewhere).
//
// All calls on a device share the one array and it keeps whatever the last
// call left in it.  The split-K tickets at its start must read zero when a
// kernel begins, so each call that uses scratch clears them first.  Two calls
// that overlap on the GPU (different streams, no ordering between them) race
// on the array.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[I4B_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return I4B_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return I4B_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return I4B_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return I4B_OK;
}

}  // namespace

extern "C" int i4b_w4a16_matmul_noalloc(const void* x, int x_dtype, int64_t M, int64_t K, int64_t stride_xm,
                                        int64_t stride_xk, const int32_t* qweight, int64_t N, int64_t stride_qk,
                                        const uint16_t* scales, const uint16_t* zeros, int64_t stride_sg,
                                        int group_size, void* y, int64_t stride_ym, void* stream) {
  // The argument checks of i4b_w4a16_matmul, in its order, come before the scratch limit, so a bad
  // argument is reported as such whatever the sizes.
  if (x_dtype != I4B_F16 && x_dtype != I4B_BF16) return I4B_ERR_INVALID_ARG;
  if (M < 0 || N < 0 || K < 0) return I4B_ERR_INVALID_ARG;
  if (K % 8 != 0) return I4B_ERR_SHAPE;
  if (group_size <= 0 || group_size % 32 != 0 || K % group_size != 0) return I4B_ERR_GROUP;
  if (M == 0 || N == 0) return I4B_OK;
  if (!x || !qweight || !scales || !zeros || !y) return I4B_ERR_INVALID_ARG;
  // Sizes the regular entry point would reject for other reasons are reported by it, unchanged.
  const size_t need = (M > 0 && N > 0 && K > 0) ? i4b_w4a16_workspace_size(M, N, K, group_size) : 0;
  if (need > I4B_NOALLOC_SCRATCH_BYTES) return I4B_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (int st = scratch_address(&scratch)) return st;  // every call: the first one on a device does the lookup
  if (need == 0)
    return i4b_w4a16_matmul(x, x_dtype, M, K, stride_xm, stride_xk, qweight, N, stride_qk, scales, zeros, stride_sg,
                            group_size, y, stride_ym, nullptr, 0, stream);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch, 0, i4b::kTicketBytes, s) != cudaSuccess) return I4B_ERR_CUDA;
  return i4b_w4a16_matmul(x, x_dtype, M, K, stride_xm, stride_xk, qweight, N, stride_qk, scales, zeros, stride_sg,
                          group_size, y, stride_ym, scratch, I4B_NOALLOC_SCRATCH_BYTES, stream);
}
