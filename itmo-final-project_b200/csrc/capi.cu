// extern "C" entry points of libint4_b200.so (declared in include/int4_b200.h).
//
// Validation mirrors the reference's preconditions (int4_triton/quantize.py:69-75,
// int4_triton/gemm.py:305-307) as status codes; dispatch mirrors gemm.py:234-300
// (small M -> one split-K launch, large M -> tcgen05 GEMM).  Nothing here
// allocates device memory or synchronises: scratch comes from the caller's
// workspace, whose layout is
//   [64 KB split-K tickets, always left zero]
//   small M (W4 <= 32, W16 <= 16): [fp32 partials S x M x N]
//   larger M: [x copy][weight copies][split-K fp32 partials]   (copies only when
//             an operand breaks the TMA rules: 16-byte base / row stride)
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "kernels.h"

using namespace i4b;

namespace {

thread_local int t_last_cuda_error = 0;
bool g_pdl = false;

int fail_cuda(cudaError_t e) {
  t_last_cuda_error = int(e);
  return I4B_ERR_CUDA;
}

struct DevInfo {
  int sms = 0;
  int major = 0, minor = 0;
  int smem_optin = 0;  // shared memory per block with the opt-in attribute
};

// Per-device properties, read once (the device of the calling thread).
int current_device_info(DevInfo* out) {
  static DevInfo cache[64];
  static bool filled[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e);
  if (dev < 0 || dev >= 64) return I4B_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(mu);
  if (!filled[dev]) {
    DevInfo d;
    if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return fail_cuda(e);
    if ((e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
      return fail_cuda(e);
    if ((e = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
      return fail_cuda(e);
    if ((e = cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
      return fail_cuda(e);
    cache[dev] = d;
    filled[dev] = true;
  }
  *out = cache[dev];
  if (out->major != 10 || out->minor != 0) return I4B_ERR_ARCH;
  return I4B_OK;
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }
bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }
int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// Workspace of the large-M INT4 path for the worst case the size query can see:
// [tickets][x copy][qweight / scales / zeros copies when N % 8 != 0][split-K fp32 partials].
size_t tc_w4_workspace(int64_t M, int64_t N, int64_t K, int G, int sms) {
  size_t b = kTicketBytes + align256(size_t(M) * size_t(K) * 2);
  if (N % 8 != 0) {
    const int64_t Np = round_up(N, 8);
    b += align256(size_t(K / 8) * Np * 4) + 2 * align256(size_t(K / G) * Np * 2);
  }
  return b + align256(tc_partial_bytes(tc_plan_w4(M, N, K, sms), M, N));
}

size_t tc_w16_workspace(int64_t M, int64_t N, int64_t K, int sms) {
  const int64_t Kp = round_up(K, 8);
  size_t b = kTicketBytes + align256(size_t(M) * size_t(Kp) * 2);
  if (K % 8 != 0) b += align256(size_t(N) * size_t(Kp) * 2);
  return b + align256(tc_partial_bytes(tc_plan(M, N, Kp, sms), M, N));
}

// The reference switches from its split-K small-M path to the tiled GEMM at SMALL_M = 64 (gemm.py:17).
// Here: W16 runs the register kernel up to kSkinnyMaxM = 16; INT4 up to kW4MaxM = 32 at most, by the rule of
// w4_register_path below.
constexpr int64_t kSmallM = kSkinnyMaxM;

// INT4 routing between the register-dequant kernels (M <= 32) and the tcgen05 GEMM.  Measured on B200 at
// M = 16..32 (Llama-3.2-1B block): the GEMM's fixed cost per launch (~10 us) loses to the register kernels on
// matrices under ~12 M weights (q|k|v 7.8 against 10.9 us, o), and wins on larger ones (gate|up 17.4 against
// 18.1 us, down_proj 14.9 against 18.1 us at M = 16; ~15 against 65 us at M = 32).  The tuning hook sets a
// plain M threshold (8..32) instead.
int64_t g_w4_small_max = 0;  // 0: the shape rule above
bool w4_register_path(int64_t M, int64_t N, int64_t K) {
  if (g_w4_small_max) return M <= g_w4_small_max;
  if (!I4B_W4T_DEFAULT) return M <= kW4MaxM;  // the shape rule needs the TMEM-weight GEMM as the default
  return M <= 8 || (M <= kW4MaxM && N * K < (int64_t(12) << 20));
}

}  // namespace

namespace i4b {
int cuda_error_status(cudaError_t e) { return fail_cuda(e); }

cudaError_t ensure_dynamic_smem(const void* func, size_t bytes) {
  struct Entry {
    const void* func;
    int dev;
    size_t bytes;
  };
  static std::mutex mu;
  static std::vector<Entry> set;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  bytes = std::max<size_t>(bytes, 48 * 1024);
  std::lock_guard<std::mutex> lock(mu);
  Entry* hit = nullptr;
  for (Entry& en : set)
    if (en.func == func && en.dev == dev) hit = &en;
  if (hit && hit->bytes >= bytes) return cudaSuccess;
  if ((e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes))) != cudaSuccess)
    return e;
  if ((e = cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared)) != cudaSuccess)
    return e;
  if (hit) hit->bytes = bytes;
  else set.push_back({func, dev, bytes});
  return cudaSuccess;
}
}  // namespace i4b

extern "C" {

const char* i4b_status_string(int status) {
  switch (status) {
    case I4B_OK: return "ok";
    case I4B_ERR_INVALID_ARG: return "invalid argument";
    case I4B_ERR_SHAPE: return "unsupported shape";
    case I4B_ERR_GROUP: return "unsupported group size";
    case I4B_ERR_LAYOUT: return "unsupported stride or alignment";
    case I4B_ERR_WORKSPACE: return "workspace too small";
    case I4B_ERR_CUDA: return "CUDA error";
    case I4B_ERR_ARCH: return "device is not sm_100 (B200)";
    case I4B_ERR_SCRATCH_LIMIT: return "sizes exceed the built-in scratch of i4b_w4a16_matmul_noalloc";
    default: return "unknown status";
  }
}

int i4b_abi_version(void) { return I4B_ABI_VERSION; }

int i4b_last_cuda_error(void) { return t_last_cuda_error; }

void i4b_set_skinny_override(int wn, int wk, int splits) {
  set_skinny_override(wn, wk, splits);
  set_w4_split_override(splits);
}

void i4b_set_pdl(int enable) { g_pdl = enable != 0; }

void i4b_set_w4_kernel_override(int kernel, int wk, int splits) { set_w4_kernel_override(kernel, wk, splits); }

void i4b_set_gemm_override(int tile, int splits) { set_tc_override(tile, splits); }

void i4b_set_w4_small_m_override(int max_m) { g_w4_small_max = (max_m >= 8 && max_m <= kW4MaxM) ? max_m : 0; }

int i4b_quantize_int4(const void* w, int w_dtype, int64_t N, int64_t K, int64_t stride_wn, int64_t stride_wk,
                      int group_size, int32_t* qweight, uint16_t* scales, uint16_t* zeros, void* stream) {
  if (w_dtype != I4B_F16 && w_dtype != I4B_BF16 && w_dtype != I4B_F32) return I4B_ERR_INVALID_ARG;
  if (N < 0 || K < 0) return I4B_ERR_INVALID_ARG;
  const int64_t G = group_size == -1 ? K : group_size;
  if (K % 8 != 0) return I4B_ERR_SHAPE;
  if (G <= 0 || G % 8 != 0 || K % G != 0) return I4B_ERR_GROUP;
  if (N == 0 || K == 0) return I4B_OK;
  if (!w || !qweight || !scales || !zeros) return I4B_ERR_INVALID_ARG;
  if (N > INT32_MAX || K > INT32_MAX) return I4B_ERR_SHAPE;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  cudaError_t e = launch_quantize(w, w_dtype, N, K, stride_wn, stride_wk, int(G), qweight, scales, zeros,
                                  static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

int i4b_dequantize_int4(const int32_t* qweight, const uint16_t* scales, const uint16_t* zeros, int64_t N, int64_t K,
                        int group_size, int out_dtype, void* out, void* stream) {
  if (out_dtype != I4B_F16 && out_dtype != I4B_BF16 && out_dtype != I4B_F32) return I4B_ERR_INVALID_ARG;
  if (N < 0 || K < 0 || K % 8 != 0) return I4B_ERR_SHAPE;
  const int64_t G = group_size == -1 ? K : group_size;
  if (G <= 0 || G % 8 != 0 || (K > 0 && K % G != 0)) return I4B_ERR_GROUP;
  if (N == 0 || K == 0) return I4B_OK;
  if (!qweight || !scales || !zeros || !out) return I4B_ERR_INVALID_ARG;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  cudaError_t e = launch_dequantize(qweight, scales, zeros, N, K, int(G), out_dtype, out,
                                    static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

size_t i4b_w4a16_workspace_size(int64_t M, int64_t N, int64_t K, int group_size) {
  if (M <= 0 || N <= 0 || K <= 0 || group_size <= 0 || group_size % 32 != 0 || K % group_size != 0) return 0;
  DevInfo d;
  if (current_device_info(&d) != I4B_OK) d.sms = 148;
  // Up to M = 32 the size covers the register-dequant plan as well, which the prologue and all-reduce entry
  // points (sized by this query) always run.
  const size_t small = M <= kW4MaxM ? w4_workspace_bytes(plan_w4(M, N, K, group_size, d.sms)) : 0;
  if (w4_register_path(M, N, K)) return small;
  return std::max(small, tc_w4_workspace(M, N, K, group_size, d.sms));
}

int i4b_w4a16_matmul(const void* x, int x_dtype, int64_t M, int64_t K, int64_t stride_xm, int64_t stride_xk,
                     const int32_t* qweight, int64_t N, int64_t stride_qk, const uint16_t* scales,
                     const uint16_t* zeros, int64_t stride_sg, int group_size, void* y, int64_t stride_ym,
                     void* workspace, size_t workspace_bytes, void* stream) {
  if (x_dtype != I4B_F16 && x_dtype != I4B_BF16) return I4B_ERR_INVALID_ARG;
  if (M < 0 || N < 0 || K < 0) return I4B_ERR_INVALID_ARG;
  if (K % 8 != 0) return I4B_ERR_SHAPE;
  const int G = group_size;
  if (G <= 0 || G % 32 != 0 || K % G != 0) return I4B_ERR_GROUP;
  if (M == 0 || N == 0) return I4B_OK;
  if (!x || !qweight || !scales || !zeros || !y) return I4B_ERR_INVALID_ARG;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return I4B_ERR_SHAPE;
  if (stride_qk < N || stride_sg < N || stride_ym < N) return I4B_ERR_LAYOUT;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool f16 = x_dtype == I4B_F16;

  if (w4_register_path(M, N, K)) {
    const W4Plan p = plan_w4(M, N, K, G, d.sms);
    if (p.mode == 3) return I4B_ERR_SHAPE;
    if (w4_workspace_bytes(p) > workspace_bytes || (p.mode == 2 && !workspace)) return I4B_ERR_WORKSPACE;
    cudaError_t e = launch_w4(f16, x, M, K, stride_xm, stride_xk, qweight, N, stride_qk, scales, zeros, stride_sg, G,
                              y, stride_ym, workspace, p, g_pdl, s);
    return e == cudaSuccess ? I4B_OK : fail_cuda(e);
  }

  // Large M: TMA needs 16-byte aligned bases and row strides; copy what does not comply.
  const bool x_ok = aligned16(x) && stride_xk == 1 && (stride_xm * 2) % 16 == 0;
  const bool w_ok = aligned16(qweight) && (stride_qk * 4) % 16 == 0 && aligned16(scales) && aligned16(zeros) &&
                    (stride_sg * 2) % 16 == 0;
  if (!w_ok && N % 8 == 0) return I4B_ERR_LAYOUT;  // no workspace reserved for this case
  if (tc_w4_workspace(M, N, K, G, d.sms) > workspace_bytes || !workspace) return I4B_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace) + kTicketBytes;
  TcOperands o{x, stride_xm, qweight, stride_qk, scales, zeros, stride_sg};
  cudaError_t e = cudaSuccess;
  uint8_t* xcopy = ws;
  ws += align256(size_t(M) * size_t(K) * 2);
  if (!x_ok) {
    if ((e = launch_repack(x, 2, M, K, stride_xm, stride_xk, xcopy, K, s)) != cudaSuccess) return fail_cuda(e);
    o.x = xcopy;
    o.sxm = K;
  }
  if (!w_ok) {
    const int64_t Np = round_up(N, 8);
    uint8_t* qc = ws;
    ws += align256(size_t(K / 8) * Np * 4);
    uint8_t* scc = ws;
    ws += align256(size_t(K / G) * Np * 2);
    uint8_t* zc = ws;
    if ((e = launch_repack(qweight, 4, K / 8, N, stride_qk, 1, qc, Np, s)) != cudaSuccess) return fail_cuda(e);
    if ((e = launch_repack(scales, 2, K / G, N, stride_sg, 1, scc, Np, s)) != cudaSuccess) return fail_cuda(e);
    if ((e = launch_repack(zeros, 2, K / G, N, stride_sg, 1, zc, Np, s)) != cudaSuccess) return fail_cuda(e);
    o.w = qc;
    o.sw = Np;
    o.sc = reinterpret_cast<const uint16_t*>(scc);
    o.zr = reinterpret_cast<const uint16_t*>(zc);
    o.ssg = Np;
  }
  const TcPlan plan = tc_plan_w4(M, N, K, d.sms);
  uint8_t* part = static_cast<uint8_t*>(workspace) + tc_w4_workspace(M, N, K, G, d.sms) -
                  align256(tc_partial_bytes(plan, M, N));
  e = launch_tc(true, f16, o, M, N, K, G, static_cast<uint16_t*>(y), stride_ym, plan, reinterpret_cast<float*>(part),
                static_cast<unsigned int*>(workspace), s);
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

size_t i4b_w4a16_argmax_workspace_size(int64_t M, int64_t N, int64_t K, int group_size) {
  if (M <= 0 || M > 8 || N <= 0 || K <= 0 || group_size <= 0 || group_size % 32 != 0 || K % group_size != 0)
    return 0;
  DevInfo d;
  if (current_device_info(&d) != I4B_OK) d.sms = 148;
  return w4_argmax_workspace_bytes(M, N, K, group_size, d.sms);
}

int i4b_w4a16_matmul_argmax(const void* x, int x_dtype, int64_t M, int64_t K, int64_t stride_xm,
                            const int32_t* qweight, int64_t N, int64_t stride_qk, const uint16_t* scales,
                            const uint16_t* zeros, int64_t stride_sg, int group_size, void* y, int64_t stride_ym,
                            int64_t* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (x_dtype != I4B_F16 && x_dtype != I4B_BF16) return I4B_ERR_INVALID_ARG;
  if (M < 0 || N < 0 || K < 0) return I4B_ERR_INVALID_ARG;
  if (M > 8 || K % 8 != 0) return I4B_ERR_SHAPE;
  const int G = group_size;
  if (G <= 0 || G % 32 != 0 || K % G != 0) return I4B_ERR_GROUP;
  if (M == 0) return I4B_OK;
  if (N == 0 || K == 0) return I4B_ERR_SHAPE;  // no column to choose
  if (!x || !qweight || !scales || !zeros || !out) return I4B_ERR_INVALID_ARG;
  if (N > INT32_MAX || K > INT32_MAX) return I4B_ERR_SHAPE;
  if (stride_qk < N || stride_sg < N || (y && stride_ym < N) || stride_xm < K) return I4B_ERR_LAYOUT;
  if (N % 8 != 0 || !aligned16(qweight) || stride_qk % 4 != 0 || !aligned16(scales) || !aligned16(zeros) ||
      stride_sg % 8 != 0)
    return I4B_ERR_LAYOUT;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  const size_t need = w4_argmax_workspace_bytes(M, N, K, G, d.sms);
  if (need == 0) return I4B_ERR_SHAPE;
  if (!workspace || workspace_bytes < need) return I4B_ERR_WORKSPACE;
  const cudaError_t e = launch_w4_argmax(x_dtype == I4B_F16, x, M, K, stride_xm, qweight, N, stride_qk, scales, zeros,
                                         stride_sg, G, y, stride_ym, out, workspace, g_pdl, d.sms,
                                         static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidConfiguration) return I4B_ERR_LAYOUT;
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

int i4b_w4a16_matmul_prologue(int prologue, const void* src, const void* delta, const void* norm_weight, float eps,
                              void* resid_out, int64_t M, int64_t K, int64_t stride_src, const int32_t* qweight,
                              int64_t N, int64_t stride_qk, const uint16_t* scales, const uint16_t* zeros,
                              int64_t stride_sg, int group_size, void* y, int64_t stride_ym, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (prologue != I4B_PROLOGUE_RMSNORM && prologue != I4B_PROLOGUE_SWIGLU) return I4B_ERR_INVALID_ARG;
  if (M < 0 || N < 0 || K < 0) return I4B_ERR_INVALID_ARG;
  if (M > kW4MaxM || K % 8 != 0) return I4B_ERR_SHAPE;
  const int G = group_size;
  if (G <= 0 || G % 32 != 0 || K % G != 0) return I4B_ERR_GROUP;
  if (M == 0 || N == 0) return I4B_OK;
  if (!src || !qweight || !scales || !zeros || !y) return I4B_ERR_INVALID_ARG;
  if (prologue == I4B_PROLOGUE_RMSNORM && !norm_weight) return I4B_ERR_INVALID_ARG;
  if (N > INT32_MAX || K > INT32_MAX) return I4B_ERR_SHAPE;
  if (stride_qk < N || stride_sg < N || stride_ym < N) return I4B_ERR_LAYOUT;
  const int64_t row = prologue == I4B_PROLOGUE_SWIGLU ? 2 * K : K;
  if (stride_src < row || stride_src % 8 != 0 || !aligned16(src) || (delta && !aligned16(delta)) ||
      (norm_weight && !aligned16(norm_weight)) || (resid_out && !aligned16(resid_out)))
    return I4B_ERR_LAYOUT;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  const W4Plan p = plan_w4(M, N, K, G, d.sms);
  if (p.mode == 3) return I4B_ERR_SHAPE;
  if (w4_workspace_bytes(p) > workspace_bytes || (p.mode == 2 && !workspace)) return I4B_ERR_WORKSPACE;
  const W4Prologue pro{prologue, delta, norm_weight, resid_out, eps};
  cudaError_t e = launch_w4(false, src, M, K, stride_src, 1, qweight, N, stride_qk, scales, zeros, stride_sg, G, y,
                            stride_ym, workspace, p, g_pdl, static_cast<cudaStream_t>(stream), &pro);
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

int i4b_w4a16_matmul_allreduce(const i4b_peer_group* group, int prologue, const void* x, int x_dtype,
                               const void* delta, const void* norm_weight, float eps, void* resid_out, int64_t M,
                               int64_t K, int64_t stride_xm, const int32_t* qweight, int64_t N, int64_t stride_qk,
                               const uint16_t* scales, const uint16_t* zeros, int64_t stride_sg, int group_size,
                               void* y, int64_t stride_ym, void* stream) {
  if (!group || group->world < 1 || group->world > I4B_PEER_MAX_RANKS || group->rank < 0 ||
      group->rank >= group->world || group->capacity < 0)
    return I4B_ERR_INVALID_ARG;
  // RMSNorm needs the statistics of the whole row, which a K shard does not hold: plain or SwiGLU only
  if (prologue != 0 && prologue != I4B_PROLOGUE_SWIGLU) return I4B_ERR_INVALID_ARG;
  if (x_dtype != I4B_BF16 && (x_dtype != I4B_F16 || prologue != 0)) return I4B_ERR_INVALID_ARG;
  if (M < 0 || N < 0 || K < 0) return I4B_ERR_INVALID_ARG;
  if (M > kW4MaxM || K % 8 != 0) return I4B_ERR_SHAPE;
  const int G = group_size;
  if (G <= 0 || G % 32 != 0 || K % G != 0) return I4B_ERR_GROUP;
  if (M == 0 || N == 0) return I4B_OK;
  if (!x || !qweight || !scales || !zeros || !y) return I4B_ERR_INVALID_ARG;
  if (prologue == I4B_PROLOGUE_RMSNORM && !norm_weight) return I4B_ERR_INVALID_ARG;
  if (N > INT32_MAX || K > INT32_MAX || M * N > group->capacity) return I4B_ERR_SHAPE;
  if (stride_qk < N || stride_sg < N || stride_ym < N) return I4B_ERR_LAYOUT;
  if (prologue != 0) {
    const int64_t row = prologue == I4B_PROLOGUE_SWIGLU ? 2 * K : K;
    if (stride_xm < row || stride_xm % 8 != 0 || !aligned16(x) || (delta && !aligned16(delta)) ||
        (norm_weight && !aligned16(norm_weight)) || (resid_out && !aligned16(resid_out)))
      return I4B_ERR_LAYOUT;
  } else if (stride_xm < K) {
    return I4B_ERR_LAYOUT;
  }
  for (int q = 0; q < group->world; ++q)
    if (!group->buffers[q] || reinterpret_cast<uintptr_t>(group->buffers[q]) % 256 != 0) return I4B_ERR_INVALID_ARG;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  const W4Plan p = plan_w4(M, N, K, G, d.sms);
  // every CTA waits for the same CTA of the other ranks, so the whole grid must be resident at once
  if (p.mode != 0 && p.mode != 1) return I4B_ERR_SHAPE;
  if (p.ntiles * p.S > std::min<int64_t>(d.sms, kArMaxCtas)) return I4B_ERR_SHAPE;
  W4AllReduce ar{};
  for (int q = 0; q < group->world; ++q) ar.buffers[q] = group->buffers[q];
  ar.capacity = group->capacity;
  ar.world = group->world;
  ar.rank = group->rank;
  const W4Prologue pro{prologue, delta, norm_weight, resid_out, eps};
  cudaError_t e = launch_w4(x_dtype == I4B_F16, x, M, K, stride_xm, 1, qweight, N, stride_qk, scales, zeros, stride_sg,
                            G, y, stride_ym, nullptr, p, g_pdl, static_cast<cudaStream_t>(stream),
                            prologue ? &pro : nullptr, &ar);
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

int i4b_argmax_allreduce(const i4b_peer_group* group, const void* x, int64_t rows, int64_t n, int64_t stride_x,
                         int64_t offset, int64_t* out, void* stream) {
  if (!group || group->world < 1 || group->world > I4B_PEER_MAX_RANKS || group->rank < 0 ||
      group->rank >= group->world)
    return I4B_ERR_INVALID_ARG;
  if (rows < 0 || n <= 0 || stride_x < n || offset < 0 || offset + n > INT32_MAX) return I4B_ERR_SHAPE;
  if (rows == 0) return I4B_OK;
  if (!x || !out) return I4B_ERR_INVALID_ARG;
  if (2 * rows > group->capacity || rows > kArMaxCtas) return I4B_ERR_SHAPE;
  for (int q = 0; q < group->world; ++q)
    if (!group->buffers[q] || reinterpret_cast<uintptr_t>(group->buffers[q]) % 256 != 0) return I4B_ERR_INVALID_ARG;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  if (rows > d.sms) return I4B_ERR_SHAPE;  // every CTA waits for another GPU: all must be resident
  W4AllReduce ar{};
  for (int q = 0; q < group->world; ++q) ar.buffers[q] = group->buffers[q];
  ar.capacity = group->capacity;
  ar.world = group->world;
  ar.rank = group->rank;
  const cudaError_t e = launch_argmax_allreduce(static_cast<const uint16_t*>(x), rows, n, stride_x, offset, out, ar,
                                                static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

size_t i4b_w16a16_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  DevInfo d;
  if (current_device_info(&d) != I4B_OK) d.sms = 148;
  if (M <= kSmallM) return skinny_workspace_bytes(plan_skinny(M, N, K, d.sms));
  return tc_w16_workspace(M, N, K, d.sms);
}

int i4b_w16a16_matmul(const void* x, int dtype, int64_t M, int64_t K, int64_t stride_xm, int64_t stride_xk,
                      const void* w, int64_t N, int64_t stride_wn, int64_t stride_wk, void* y, int64_t stride_ym,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != I4B_F16 && dtype != I4B_BF16) return I4B_ERR_INVALID_ARG;
  if (M < 0 || N < 0 || K < 0) return I4B_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return I4B_OK;
  if (!x || !w || !y) return I4B_ERR_INVALID_ARG;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return I4B_ERR_SHAPE;
  if (stride_ym < N) return I4B_ERR_LAYOUT;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool f16 = dtype == I4B_F16;
  if (K == 0) {
    // Empty reduction: y = 0.
    for (int64_t m = 0; m < M; ++m) {
      cudaError_t e = cudaMemsetAsync(static_cast<uint16_t*>(y) + m * stride_ym, 0, size_t(N) * 2, s);
      if (e != cudaSuccess) return fail_cuda(e);
    }
    return I4B_OK;
  }
  if (M <= kSmallM) {
    const SkinnyPlan p = plan_skinny(M, N, K, d.sms);
    if (p.mode == 3) return I4B_ERR_SHAPE;
    if (skinny_workspace_bytes(p) > workspace_bytes || (p.mode == 2 && !workspace)) return I4B_ERR_WORKSPACE;
    cudaError_t e = launch_skinny(f16, x, M, K, stride_xm, stride_xk, w, N, stride_wn, stride_wk, y, stride_ym,
                                  workspace, p, g_pdl, s);
    return e == cudaSuccess ? I4B_OK : fail_cuda(e);
  }
  const int64_t Kp = round_up(K, 8);
  const bool x_ok = K % 8 == 0 && aligned16(x) && stride_xk == 1 && (stride_xm * 2) % 16 == 0;
  const bool w_ok = K % 8 == 0 && aligned16(w) && stride_wk == 1 && (stride_wn * 2) % 16 == 0;
  if (!w_ok && K % 8 == 0) return I4B_ERR_LAYOUT;
  if (tc_w16_workspace(M, N, K, d.sms) > workspace_bytes || !workspace) return I4B_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace) + kTicketBytes;
  TcOperands o{x, stride_xm, w, stride_wn, nullptr, nullptr, 0};
  cudaError_t e = cudaSuccess;
  uint8_t* xcopy = ws;
  ws += align256(size_t(M) * size_t(Kp) * 2);
  if (!x_ok) {
    if ((e = launch_repack(x, 2, M, K, stride_xm, stride_xk, xcopy, Kp, s)) != cudaSuccess) return fail_cuda(e);
    o.x = xcopy;
    o.sxm = Kp;
  }
  if (!w_ok) {
    if ((e = launch_repack(w, 2, N, K, stride_wn, stride_wk, ws, Kp, s)) != cudaSuccess) return fail_cuda(e);
    o.w = ws;
    o.sw = Kp;
  }
  const TcPlan plan = tc_plan(M, N, Kp, d.sms);
  uint8_t* part = static_cast<uint8_t*>(workspace) + tc_w16_workspace(M, N, K, d.sms) -
                  align256(tc_partial_bytes(plan, M, N));
  e = launch_tc(false, f16, o, M, N, Kp, 0, static_cast<uint16_t*>(y), stride_ym, plan,
                reinterpret_cast<float*>(part), static_cast<unsigned int*>(workspace), s);
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

// ------------------------------------------------------------------ decode-step glue

int i4b_add_rmsnorm(void* h, const void* delta, const void* weight, void* out, int64_t rows, int64_t H, float eps,
                    void* stream) {
  if (rows < 0 || H <= 0 || H % 8 != 0 || rows > INT32_MAX || H > INT32_MAX) return I4B_ERR_SHAPE;
  if (rows == 0) return I4B_OK;
  if (!h || !weight || !out) return I4B_ERR_INVALID_ARG;
  if (!aligned16(h) || (delta && !aligned16(delta)) || !aligned16(weight) || !aligned16(out)) return I4B_ERR_LAYOUT;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  const cudaError_t e = launch_add_rmsnorm(static_cast<uint16_t*>(h), static_cast<const uint16_t*>(delta),
                                           static_cast<const uint16_t*>(weight), static_cast<uint16_t*>(out),
                                           int(rows), int(H), eps, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

int i4b_rope_kv_cache(const void* qkv, const void* cos_table, const void* sin_table, const int64_t* pos, void* q_out,
                      void* k_cache, void* v_cache, int64_t B, int64_t nq, int64_t nkv, int64_t head_dim,
                      int64_t max_seq, void* stream) {
  if (head_dim != 64) return I4B_ERR_SHAPE;
  if (B < 0 || nq <= 0 || nkv <= 0 || max_seq <= 0 || B * (nq + 2 * nkv) > INT32_MAX || max_seq > INT32_MAX)
    return I4B_ERR_SHAPE;
  if (B == 0) return I4B_OK;
  if (!qkv || !cos_table || !sin_table || !pos || !q_out || !k_cache || !v_cache) return I4B_ERR_INVALID_ARG;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  const cudaError_t e = launch_rope_kv(
      static_cast<const uint16_t*>(qkv), static_cast<const uint16_t*>(cos_table),
      static_cast<const uint16_t*>(sin_table), pos, static_cast<uint16_t*>(q_out), static_cast<uint16_t*>(k_cache),
      static_cast<uint16_t*>(v_cache), int(B), int(nq), int(nkv), int(max_seq), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

int i4b_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos, void* out,
                         int64_t B, int64_t nq, int64_t nkv, int64_t head_dim, int64_t max_seq, float scale,
                         void* stream) {
  if (head_dim != 64 || B < 0 || nq <= 0 || nkv <= 0 || nq % nkv != 0 || max_seq <= 0) return I4B_ERR_SHAPE;
  if (max_seq > 8 * 6144 || B > 65535 || nq * 8 > INT32_MAX) return I4B_ERR_SHAPE;  // scores live in shared memory
  if (B == 0) return I4B_OK;
  if (!q || !k_cache || !v_cache || !pos || !out) return I4B_ERR_INVALID_ARG;
  if (!aligned16(k_cache) || !aligned16(v_cache)) return I4B_ERR_LAYOUT;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  const cudaError_t e = launch_decode_attn(static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k_cache),
                                           static_cast<const uint16_t*>(v_cache), pos, static_cast<uint16_t*>(out),
                                           int(B), int(nq), int(nkv), int(max_seq), scale,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

int i4b_silu_mul(const void* gate_up, void* y, int64_t B, int64_t I, void* stream) {
  if (B < 0 || I <= 0 || I % 8 != 0 || B * I > INT32_MAX) return I4B_ERR_SHAPE;
  if (B == 0) return I4B_OK;
  if (!gate_up || !y) return I4B_ERR_INVALID_ARG;
  if (!aligned16(gate_up) || !aligned16(y)) return I4B_ERR_LAYOUT;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  const cudaError_t e = launch_silu_mul(static_cast<const uint16_t*>(gate_up), static_cast<uint16_t*>(y), int(B),
                                        int(I), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

int i4b_argmax_rows(const void* x, int64_t rows, int64_t n, int64_t* out, void* stream) {
  if (rows < 0 || n <= 0 || rows > INT32_MAX) return I4B_ERR_SHAPE;
  if (rows == 0) return I4B_OK;
  if (!x || !out) return I4B_ERR_INVALID_ARG;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  const cudaError_t e = launch_argmax(static_cast<const uint16_t*>(x), rows, n, out, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

size_t i4b_tile_w4_bytes(int64_t N, int64_t K, int group_size) { return tile_w4_bytes(N, K, group_size); }

int i4b_tile_w4(const int32_t* qweight, int64_t N, int64_t stride_qk, const uint16_t* scales, const uint16_t* zeros,
                int64_t stride_sg, int64_t K, int group_size, void* out, void* stream) {
  if (group_size != 32 && group_size != 64 && group_size != 128) return I4B_ERR_GROUP;
  if (tile_w4_bytes(N, K, group_size) == 0) return I4B_ERR_SHAPE;
  if (!qweight || !scales || !zeros || !out) return I4B_ERR_INVALID_ARG;
  if (stride_qk < N || stride_sg < N) return I4B_ERR_LAYOUT;
  if (!aligned16(out)) return I4B_ERR_LAYOUT;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  const cudaError_t e =
      launch_tile_w4(qweight, stride_qk, scales, zeros, stride_sg, N, K, group_size, out, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? I4B_OK : fail_cuda(e);
}

int i4b_decode_workspace_size(const i4b_decode_model* model, size_t* bytes) {
  if (!model || !bytes) return I4B_ERR_INVALID_ARG;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  return decode_layers_workspace(*model, d.sms, bytes);
}

int i4b_decode_layers(const i4b_decode_model* model, void* workspace, size_t workspace_bytes, void* stream) {
  if (!model || !workspace) return I4B_ERR_INVALID_ARG;
  const i4b_decode_model& m = *model;
  if (!m.tokens || !m.pos || !m.embed || !m.w_qkv || !m.w_o || !m.w_gu || !m.w_down || !m.ln1 || !m.ln2 ||
      !m.cos_table || !m.sin_table || !m.k_cache || !m.v_cache || !m.h_out)
    return I4B_ERR_INVALID_ARG;
  const void* vec[] = {m.embed, m.w_qkv, m.w_o, m.w_gu, m.w_down, m.ln1, m.ln2, m.k_cache, m.v_cache, m.h_out, workspace};
  for (const void* p : vec)
    if (!aligned16(p)) return I4B_ERR_LAYOUT;
  DevInfo d;
  if (int st = current_device_info(&d)) return st;
  cudaError_t e = cudaSuccess;
  const int st = launch_decode_layers(m, d.sms, d.smem_optin, workspace, workspace_bytes,
                                      static_cast<cudaStream_t>(stream), &e);
  return st == I4B_ERR_CUDA ? fail_cuda(e) : st;
}

void i4b_set_decode_trace(void* buffer, size_t bytes) { set_decode_trace(buffer, bytes); }

int64_t i4b_decode_peer_capacity(int32_t layers, int32_t world, int32_t hidden) {
  if (layers <= 0 || world <= 0 || hidden <= 0) return 0;
  return decode_peer_capacity(layers, world, hidden);
}

int i4b_device_error_flags(int device, int clear) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return -1;
  if (cudaSetDevice(device) != cudaSuccess) return -1;
  int flags = -1;
  if (cudaDeviceSynchronize() == cudaSuccess) {
    flags = int(read_quant_error(clear != 0) | read_tc_error(clear != 0) | read_w4t_error(clear != 0) | read_dk_error(clear != 0) |
                read_w4_error(clear != 0));
  }
  cudaSetDevice(prev);
  return flags;
}

}  // extern "C"
