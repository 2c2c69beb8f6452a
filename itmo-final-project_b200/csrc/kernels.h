// Host-side declarations of the kernel launchers shared between the .cu files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/int4_b200.h"

namespace i4b {

// quantize.cu
cudaError_t launch_quantize(const void* w, int dt, int64_t N, int64_t K, int64_t swn, int64_t swk, int G,
                            int32_t* qw, uint16_t* sc, uint16_t* zr, cudaStream_t stream);
cudaError_t launch_dequantize(const int32_t* qw, const uint16_t* sc, const uint16_t* zr, int64_t N, int64_t K, int G,
                              int odt, void* out, cudaStream_t stream);
unsigned int read_quant_error(bool clear);

// Every workspace starts with a ticket region that only the split-K kernels
// use and always leave zero; scratch of any other kind starts after it.
constexpr size_t kTicketBytes = 64 * 1024;
constexpr int64_t kMaxTickets = int64_t(kTicketBytes / 4);

// skinny.cu (W16 weights, M <= kSkinnyMaxM)
constexpr int64_t kSkinnyMaxM = 16;
struct SkinnyPlan {
  int MT, WN, WK, S, KC, KW, L, xstride;
  int mode;  // 0: one CTA per column tile; 1: cluster along K; 2: workspace split-K; 3: unsupported
  size_t smem_bytes;
  size_t partial_bytes;
  int64_t ntiles;
};
SkinnyPlan plan_skinny(int64_t M, int64_t N, int64_t K, int num_sms);
size_t skinny_workspace_bytes(const SkinnyPlan& p);
cudaError_t launch_skinny(bool f16, const void* x, int64_t M, int64_t K, int64_t sxm, int64_t sxk, const void* w,
                          int64_t N, int64_t sw0, int64_t sw1, void* y, int64_t sym, void* ws, const SkinnyPlan& p,
                          bool pdl, cudaStream_t stream);
// Tuning override of the automatic decomposition (0 = automatic).
void set_skinny_override(int wn, int wk, int splits);

// gemv_w4.cu (INT4, M <= kW4MaxM: 8, 16 or 32 tokens per CTA)
constexpr int64_t kW4MaxM = 32;
struct W4Plan {
  int MT, SPS, S, KC;
  int mode;  // 0: one CTA per column tile; 1: cluster along K; 2: workspace split-K; 3: unsupported
  int64_t ntiles;
  size_t partial_bytes;
};
W4Plan plan_w4(int64_t M, int64_t N, int64_t K, int G, int num_sms);
size_t w4_workspace_bytes(const W4Plan& p);
// Optional activation prologue of the small-M kernel (bf16): kind 1 = rmsnorm(x + delta) * norm_weight
// (resid_out, when set, receives x + delta), kind 2 = silu(g) * u with g | u = the two halves of an x row.
struct W4Prologue {
  int kind;
  const void* delta;
  const void* norm_weight;
  void* resid_out;
  float eps;
};
// Peer exchange buffer of the fused tensor-parallel all-reduce (i4b_peer_group), per rank:
//   [control: epoch u32, done-ticket u32 | 256 B][reserved | kArDataOff]
//   [data: tagged values u64 [2 slots][8 source ranks][capacity]]
// A call of epoch e uses slot e & 1; each value is stored with the tag e + 1 in its high word.
constexpr size_t kArCtlBytes = 256;
constexpr int kArMaxRanks = 8;
constexpr int kArMaxCtas = 1024;
constexpr size_t kArDataOff = kArCtlBytes + size_t(2) * kArMaxRanks * kArMaxCtas * 4;
inline size_t ar_buffer_bytes(int64_t capacity) {
  return kArDataOff + size_t(2) * kArMaxRanks * size_t(capacity) * 8;
}
struct W4AllReduce {
  void* buffers[kArMaxRanks];
  int64_t capacity;
  int world, rank;
};
cudaError_t launch_w4(bool f16, const void* x, int64_t M, int64_t K, int64_t sxm, int64_t sxk, const int32_t* qw,
                      int64_t N, int64_t sqk, const uint16_t* sc, const uint16_t* zr, int64_t ssg, int G, void* y,
                      int64_t sym, void* ws, const W4Plan& p, bool pdl, cudaStream_t stream,
                      const W4Prologue* pro = nullptr, const W4AllReduce* ar = nullptr);
void set_w4_split_override(int splits);
// Tuning override of the M <= 8 kernel choice: kernel 0 automatic, 1 register-streaming GEMV, 2 the staged
// small-M kernel, 3 the staged kernel or the streaming lm_head kernel, 4 / 5 the register-streaming GEMV with a
// ring of 4 / 8 steps, 6 the slab-streaming GEMV (wk = its K split P: 1, 2, 4 or 8; splits = 2: a balanced grid
// instead of every resident CTA); wk / splits otherwise: warps along K per CTA and cluster split of the
// register-streaming GEMV (0 automatic).
void set_w4_kernel_override(int kernel, int wk, int splits);
// Greedy choice fused into the M <= 8 GEMV: out[m] = first column of row m's maximum logit (as rounded to x's
// dtype); y (may be null) receives the logits.  Workspace: w4_argmax_workspace_bytes (0 = sizes not supported).
size_t w4_argmax_workspace_bytes(int64_t M, int64_t N, int64_t K, int G, int sms);
cudaError_t launch_w4_argmax(bool f16, const void* x, int64_t M, int64_t K, int64_t sxm, const int32_t* qw, int64_t N,
                             int64_t sqk, const uint16_t* sc, const uint16_t* zr, int64_t ssg, int G, void* y,
                             int64_t sym, int64_t* out, void* ws, bool pdl, int sms, cudaStream_t stream);
unsigned int read_w4_error(bool clear);
// Greedy token of rows split over the ranks of a peer group (columns [offset, offset + n) on this rank).
cudaError_t launch_argmax_allreduce(const uint16_t* x, int64_t rows, int64_t n, int64_t sx, int64_t offset,
                                    int64_t* out, const W4AllReduce& ar, cudaStream_t stream);
// capi.cu: records e for i4b_last_cuda_error and returns I4B_ERR_CUDA
int cuda_error_status(cudaError_t e);
// capi.cu: lets kernel `func` use `bytes` of dynamic shared memory on the CURRENT device (and prefer the
// maximum shared-memory carveout).  The attribute is per device, so the setting is remembered per
// (kernel, device) pair, under a lock; a later call asking for no more than was set is free.
cudaError_t ensure_dynamic_smem(const void* func, size_t bytes);

// gemm_tc.cu (W4 M > 32, W16 M > 16)
struct TcOperands {
  const void* x;
  int64_t sxm;
  const void* w;
  int64_t sw;
  const uint16_t* sc;
  const uint16_t* zr;
  int64_t ssg;
};
struct TcPlan {
  int tile;    // 1: 128 x 128, 2: 256 x 128, 3: 128 x 256, 4: 256 x 256 (shared-memory operands);
               // INT4 only, weights in TMEM: 5..8 = 128 weight rows x 256 / 128 / 64 / 32 tokens
  int splits;  // K splits (fp32 partials in the workspace when > 1)
};
TcPlan tc_plan(int64_t M, int64_t N, int64_t K, int num_sms);     // W16 (and INT4 tiles 1..4)
TcPlan tc_plan_w4(int64_t M, int64_t N, int64_t K, int num_sms);  // INT4
void set_tc_override(int tile, int splits);  // tuning: 0 keeps the automatic choice
bool make_tma_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz);
bool make_tma_map_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
                     uint64_t d2, uint64_t stride1, uint64_t stride2, uint32_t b0, uint32_t b1, uint32_t b2,
                     CUtensorMapSwizzle swz);
size_t tc_partial_bytes(const TcPlan& p, int64_t M, int64_t N);
cudaError_t launch_tc(bool int4, bool f16, const TcOperands& o, int64_t M, int64_t N, int64_t K, int G, uint16_t* y,
                      int64_t sym, const TcPlan& plan, float* partials, unsigned int* tickets, cudaStream_t stream);
cudaError_t launch_repack(const void* in, int esize, int64_t rows, int64_t cols_in, int64_t sr, int64_t sc, void* out,
                          int64_t cols_out, cudaStream_t stream);
unsigned int read_tc_error(bool clear);

// gemm_w4t.cu (INT4, weights dequantized into TMEM; tile codes 5..8 of TcPlan).  I4B_W4T_DEFAULT: whether the
// INT4 dispatch chooses it by default (capi.cu w4_register_path, gemm_tc.cu tc_plan_w4).
#ifndef I4B_W4T_DEFAULT
#define I4B_W4T_DEFAULT 0
#endif
int w4t_token_tile(int tile);
int w4t_ctas_per_sm(int tile);
cudaError_t launch_w4t(bool f16, const TcOperands& o, int64_t M, int64_t N, int64_t K, int G, uint16_t* y,
                       int64_t sym, int tile, int ksplit, float* partials, unsigned int* tickets, cudaStream_t stream);
unsigned int read_w4t_error(bool clear);

// decode_ops.cu (decode-step glue of a Llama layer)
cudaError_t launch_add_rmsnorm(uint16_t* h, const uint16_t* delta, const uint16_t* w, uint16_t* out, int rows, int H,
                               float eps, cudaStream_t s);
cudaError_t launch_rope_kv(const uint16_t* qkv, const uint16_t* cosT, const uint16_t* sinT, const int64_t* pos,
                           uint16_t* q_out, uint16_t* kc, uint16_t* vc, int B, int nq, int nkv, int max_seq,
                           cudaStream_t s);
cudaError_t launch_decode_attn(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int64_t* pos,
                               uint16_t* out, int B, int nq, int nkv, int max_seq, float scale, cudaStream_t s);
cudaError_t launch_silu_mul(const uint16_t* gu, uint16_t* y, int B, int I, cudaStream_t s);
cudaError_t launch_argmax(const uint16_t* x, int64_t rows, int64_t n, int64_t* out, cudaStream_t s);

// decode_persistent.cu (all decoder layers of a decode step in one cooperative launch)
size_t tile_w4_bytes(int64_t N, int64_t K, int G);
cudaError_t launch_tile_w4(const int32_t* qw, int64_t sqk, const uint16_t* sc, const uint16_t* zr, int64_t ssg,
                           int64_t N, int64_t K, int G, void* out, cudaStream_t stream);
int decode_layers_workspace(const i4b_decode_model& m, int num_sms, size_t* bytes);
int64_t decode_peer_capacity(int layers, int world, int hidden);
int launch_decode_layers(const i4b_decode_model& m, int num_sms, int smem_optin, void* ws, size_t ws_bytes,
                         cudaStream_t stream, cudaError_t* err);
unsigned int read_dk_error(bool clear);
void set_decode_trace(void* buf, size_t bytes);

}  // namespace i4b
