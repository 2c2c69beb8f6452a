/* int4_b200 -- C ABI of the B200-native (sm_100a) INT4 W4A16 path.
 *
 * Drop-in boundary for the hot path of homomorfism/itmo-final-project
 * (Python package `int4_triton`): group-wise asymmetric INT4 quantize/pack and
 * the W4A16 matmul that consumes the packed weights.  Plain pointers, sizes
 * and strides; no torch types.  Every entry point is asynchronous on the
 * given CUDA stream (cudaStream_t passed as void*, NULL = legacy default),
 * allocates nothing, never synchronises the device, and returns an
 * I4B_STATUS code (0 = success).
 *
 * Storage format (identical to the reference, int4_triton/quantize.py:1-13):
 *   W        [N, K]     weights of an nn.Linear (out_features N, in_features K)
 *   qweight  int32[K/8, N]   word [k8, n] holds W[n, 8*k8 + i] in bits 4i..4i+3
 *   scales   fp16 [K/G, N]   per-group scale
 *   zeros    fp16 [K/G, N]   per-group integer zero point 0..15
 *   W_hat[n, k] = (q - zero) * scale      (fp32, exact)
 *
 * Element-type codes: I4B_F16, I4B_BF16, I4B_F32.  fp16 / bf16 buffers are
 * passed as raw 16-bit patterns.
 */
#ifndef INT4_B200_H
#define INT4_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define I4B_ABI_VERSION 1

enum { I4B_F16 = 0, I4B_BF16 = 1, I4B_F32 = 2 };

enum {
  I4B_OK = 0,
  I4B_ERR_INVALID_ARG = 1, /* null pointer where data is required, unknown dtype, negative size */
  I4B_ERR_SHAPE = 2,       /* K not a multiple of 8 / of G, qweight rows != K/8, ... */
  I4B_ERR_GROUP = 3,       /* group size not supported by this entry point */
  I4B_ERR_LAYOUT = 4,      /* a stride or alignment the entry point does not accept */
  I4B_ERR_WORKSPACE = 5,   /* workspace smaller than the matching *_workspace_size() */
  I4B_ERR_CUDA = 6,        /* a CUDA runtime / driver call failed (see i4b_last_cuda_error) */
  I4B_ERR_ARCH = 7,        /* current device is not sm_100 */
  I4B_ERR_SCRATCH_LIMIT = 8 /* i4b_w4a16_matmul_noalloc: these sizes need more than its built-in scratch */
};

/* Human-readable name of a status code. */
const char* i4b_status_string(int status);
/* I4B_ABI_VERSION of the loaded library. */
int i4b_abi_version(void);
/* cudaError_t of the last call that returned I4B_ERR_CUDA on this host thread. */
int i4b_last_cuda_error(void);

/* Quantize W[N, K] group-wise to INT4.
 * Replaces int4_triton.quantize_int4 (int4_triton/quantize.py:67-96) and is bit
 * exact with its torch reference quantize_int4_ref (quantize.py:102-117),
 * including all-zero groups (scale 1) and non-finite inputs (x86 NaN rules).
 * w: element (n, k) at w + n*stride_wn + k*stride_wk (strides in elements),
 *    dtype I4B_F16, I4B_BF16 or I4B_F32.
 * group_size: G, or -1 for G = K.  Requires K % G == 0 and G % 8 == 0.
 * Outputs are contiguous: qweight int32[K/8, N], scales/zeros fp16[K/G, N]. */
int i4b_quantize_int4(const void* w, int w_dtype, int64_t N, int64_t K, int64_t stride_wn, int64_t stride_wk,
                      int group_size, int32_t* qweight, uint16_t* scales, uint16_t* zeros, void* stream);

/* W_hat[N, K] = (q - zero) * scale computed in fp32 and rounded once to out_dtype.
 * Replaces dequantize_int4_ref (int4_triton/quantize.py:128-135).  Inputs and
 * the output are contiguous; G = K / (rows of scales). */
int i4b_dequantize_int4(const int32_t* qweight, const uint16_t* scales, const uint16_t* zeros, int64_t N, int64_t K,
                        int group_size, int out_dtype, void* out, void* stream);

/* Bytes of workspace i4b_w4a16_matmul needs for these sizes (0 is possible); for M <= 32 also enough for
 * i4b_w4a16_matmul_prologue and i4b_w4a16_matmul_allreduce.
 * The workspace must be zero-filled before its first use; every call leaves
 * its counter area zero again, so a workspace kept per stream needs no
 * further clearing.  Calls that share a workspace must not overlap in time. */
size_t i4b_w4a16_workspace_size(int64_t M, int64_t N, int64_t K, int group_size);

/* y[M, N] = x[M, K] @ W_hat^T in x's dtype (fp32 accumulation).
 * Replaces int4_triton.w4a16_matmul (int4_triton/gemm.py:303-309, dispatch
 * gemm.py:234-300): M <= 32 runs the register-dequant kernels (M <= 8: the
 * decode GEMVs; 9..32: deterministic in-kernel split-K reduction), larger M the
 * TMA + tcgen05/TMEM GEMM (the reference switches at M = 64; on B200 the tcgen05
 * GEMM wins from 33 tokens on).  A library built with -DI4B_W4T_DEFAULT=1 routes
 * instead by shape to the GEMM that dequantizes the weights into TMEM (from 9
 * tokens on matrices of 12 Mi weights or more).
 * When the tcgen05 GEMM runs, qweight, scales and zeros must meet the TMA rules
 * (16-byte aligned bases and row strides) unless N % 8 != 0 (then they are
 * copied into the workspace); otherwise I4B_ERR_LAYOUT.
 * x: element (m, k) at x + m*stride_xm + k*stride_xk, dtype I4B_BF16 or I4B_F16.
 * qweight: row k8 at qweight + k8*stride_qk (unit stride along N).
 * scales/zeros: row g at base + g*stride_sg (unit stride along N).
 * y: element (m, n) at y + m*stride_ym + n.
 * group_size G = K / (rows of scales); G must be a multiple of 32. */
int i4b_w4a16_matmul(const void* x, int x_dtype, int64_t M, int64_t K, int64_t stride_xm, int64_t stride_xk,
                     const int32_t* qweight, int64_t N, int64_t stride_qk, const uint16_t* scales,
                     const uint16_t* zeros, int64_t stride_sg, int group_size, void* y, int64_t stride_ym,
                     void* workspace, size_t workspace_bytes, void* stream);

/* i4b_w4a16_matmul for 1 <= M <= 32 bf16 tokens whose activations are produced inside the kernel from
 * the previous step's tensors, saving the separate launch transformers' Llama runs for them:
 *   I4B_PROLOGUE_RMSNORM: x = bf16(w * bf16(h' * rsqrt(mean(h'^2) + eps))), h' = bf16(src + delta)
 *       (delta may be NULL).  When resid_out is not NULL, h' is also written there (rows of stride_src);
 *       resid_out must not overlap src or delta.  norm_weight: bf16 [K].  (input / post-attention
 *       LlamaRMSNorm after the residual add)
 *   I4B_PROLOGUE_SWIGLU: x = bf16(bf16(silu(g)) * u), g = src[m, 0:K], u = src[m, K:2K]  (LlamaMLP)
 * src rows are contiguous with stride_src % 8 == 0; all pointers 16-byte aligned.  Workspace as for
 * i4b_w4a16_matmul (i4b_w4a16_workspace_size).  No counterpart in the reference. */
enum { I4B_PROLOGUE_RMSNORM = 1, I4B_PROLOGUE_SWIGLU = 2 };
int i4b_w4a16_matmul_prologue(int prologue, const void* src, const void* delta, const void* norm_weight, float eps,
                              void* resid_out, int64_t M, int64_t K, int64_t stride_src, const int32_t* qweight,
                              int64_t N, int64_t stride_qk, const uint16_t* scales, const uint16_t* zeros,
                              int64_t stride_sg, int group_size, void* y, int64_t stride_ym, void* workspace,
                              size_t workspace_bytes, void* stream);

/* Greedy choice fused into the W4 lm_head GEMV, for 1 <= M <= 8 rows:
 * out[m] = index of the first maximum of row m of x @ W_hat^T, the logits compared as rounded to x's dtype
 * (what torch.argmax(-1) sees on the stored logits; NaN never compares greater).  y, when not NULL, also
 * receives the logits (y element (m, n) at y + m*stride_ym + n).  Replaces the lm_head matmul followed by the
 * greedy choice of the reference's decode loop (benchmarks/eval_llama.py:121-183, logits[:, -1:].argmax(-1))
 * with one launch: each CTA keeps its columns' candidate, the last CTA to finish (atomic ticket, no spinning)
 * compares them.  x rows contiguous (stride_xm >= K); N % 8 == 0; qweight, scales and zeros 16-byte aligned
 * with stride_qk % 4 == 0 and stride_sg % 8 == 0 (else I4B_ERR_LAYOUT).  Workspace: zero-filled before first
 * use, left zero by every call, i4b_w4a16_argmax_workspace_size bytes (0: sizes not supported); calls sharing
 * it must not overlap in time. */
size_t i4b_w4a16_argmax_workspace_size(int64_t M, int64_t N, int64_t K, int group_size);
int i4b_w4a16_matmul_argmax(const void* x, int x_dtype, int64_t M, int64_t K, int64_t stride_xm,
                            const int32_t* qweight, int64_t N, int64_t stride_qk, const uint16_t* scales,
                            const uint16_t* zeros, int64_t stride_sg, int group_size, void* y, int64_t stride_ym,
                            int64_t* out, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes for i4b_w16a16_matmul (same zero-fill rule as above). */
size_t i4b_w16a16_workspace_size(int64_t M, int64_t N, int64_t K);

/* y[M, N] = x[M, K] @ w[N, K]^T, x and w of the same dtype (bf16 or fp16).
 * Replaces int4_triton.w16a16_matmul (int4_triton/gemm.py:312-317), the
 * full-precision baseline with the same kernel structure as the W4 path.
 * w: element (n, k) at w + n*stride_wn + k*stride_wk.  M <= 16 accepts any
 * strides; for M > 16 (tcgen05 GEMM) w must have unit stride along k and a
 * 16-byte aligned base and row stride when K % 8 == 0 (otherwise it is copied
 * into the workspace), else I4B_ERR_LAYOUT. */
int i4b_w16a16_matmul(const void* x, int dtype, int64_t M, int64_t K, int64_t stride_xm, int64_t stride_xk,
                      const void* w, int64_t N, int64_t stride_wn, int64_t stride_wk, void* y, int64_t stride_ym,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Programmatic dependent launch for the small-M kernels (W4 M <= 32, W16 M <= 16; default off).
 * When on, those kernels are launched with programmatic stream
 * serialization: they start while the previous kernel of the stream drains
 * and read qweight / scales / zeros BEFORE waiting for it, x only after.
 * Enable it only where no kernel directly before a matmul writes that
 * matmul's weights (e.g. a decode loop over fixed weights).  No counterpart
 * in the reference (its launches are plain Triton launches). */
void i4b_set_pdl(int enable);

/* Tuning hook for the small-M decomposition: columns per CTA (32*wn, W16 only),
 * k-warps per CTA (wk) and K splits; 0 keeps the automatic choice, an
 * unusable value is ignored.  Process-wide.  No counterpart in the reference
 * (which autotunes, int4_triton/gemm.py:51-56). */
void i4b_set_skinny_override(int wn, int wk, int splits);

/* Tuning hook for W4 M <= 8: kernel 0 = automatic (the register-streaming GEMV where it applies), 1 = the
 * register-streaming GEMV, 2 = the shared-memory-staged small-M kernel, 3 = the staged kernel or, for very
 * wide N, the streaming lm_head kernel (the choice before the register-streaming GEMV existed), 4 / 5 = the
 * register-streaming GEMV with 4 / 8 steps of weights in flight per lane; wk and splits
 * set the register-streaming GEMV's warps along K per CTA and its cluster split (0 = automatic).
 * Process-wide.  No counterpart in the reference. */
void i4b_set_w4_kernel_override(int kernel, int wk, int splits);

/* Bytes of the scratch array built into the library for i4b_w4a16_matmul_noalloc. */
#define I4B_NOALLOC_SCRATCH_BYTES (16u << 20)

/* i4b_w4a16_matmul for callers that cannot allocate device memory.
 * No counterpart in the reference, which always allocates its outputs and
 * split-K scratch with torch (int4_triton/gemm.py:246,266-268).
 * Same arguments, result and status codes as i4b_w4a16_matmul, minus the
 * workspace: a plugin inside a host program that owns all device allocation,
 * or a caller on a path where cudaMalloc may not run, passes only its inputs
 * and output.  Scratch comes from one I4B_NOALLOC_SCRATCH_BYTES array compiled
 * into the library (held by every GPU that loads it, until exit).  Sizes whose
 * i4b_w4a16_workspace_size exceeds that return I4B_ERR_SCRATCH_LIMIT.  No
 * cudaMalloc / cudaFree is called.  The first call on a device looks up the
 * array's device address, so make it before any stream capture; the address is
 * kept until exit, so cudaDeviceReset between calls is not supported.  Argument
 * errors are reported before the scratch limit.  All calls on a device share
 * the array: calls that overlap on the GPU race. */
int i4b_w4a16_matmul_noalloc(const void* x, int x_dtype, int64_t M, int64_t K, int64_t stride_xm, int64_t stride_xk,
                             const int32_t* qweight, int64_t N, int64_t stride_qk, const uint16_t* scales,
                             const uint16_t* zeros, int64_t stride_sg, int group_size, void* y, int64_t stride_ym,
                             void* stream);

/* ---- Tensor-parallel all-reduce fused into the small-M W4 matmul (peer memory over NVLink) ----
 *
 * The reference runs on one GPU.  Its tensor-parallel form shards o_proj and down_proj along K
 * (row-parallel): every rank computes a partial product over its slice of K and the ranks' partials
 * are summed.  i4b_w4a16_matmul_allreduce does that sum inside the matmul's epilogue. Each CTA:
 *   - stores each fp32 partial output, with a tag naming the call, as one 64-bit word into every rank's
 *     exchange buffer (plain stores through CUDA-IPC mappings);
 *   - polls, bounded, the words of the same outputs from every other rank until their tags match (the data
 *     is its own flag: no fence, no separate flag);
 *   - adds the ranks' partials in rank order and writes y.
 * It replaces w4a16_matmul (int4_triton/gemm.py:303-309) followed by a separate all-reduce launch.
 * Every rank ends with bit-identical y.  All ranks must make the same sequence of calls on one
 * peer group; a group's calls must not overlap in time on a rank.  A wait that gives up after
 * I4B_WAIT_LIMIT_NS sets bit 1 of i4b_device_error_flags, and later waits on that device then
 * return at once. */
#define I4B_PEER_MAX_RANKS 8
#define I4B_IPC_HANDLE_BYTES 64
typedef struct i4b_peer_group {
  int32_t world;    /* ranks, 1..I4B_PEER_MAX_RANKS */
  int32_t rank;     /* this process's rank, 0..world-1 */
  int64_t capacity; /* outputs (M * N) one call may exchange: what the buffers were allocated for */
  void* buffers[I4B_PEER_MAX_RANKS]; /* rank p's exchange buffer as mapped in this process */
} i4b_peer_group;

/* Bytes of one exchange buffer holding `capacity` outputs per call. */
size_t i4b_peer_buffer_bytes(int64_t capacity);
/* Set-up calls (they allocate and synchronise, unlike the rest of the ABI): cudaMalloc a zero-filled
 * exchange buffer on the current device / free it. */
int i4b_peer_buffer_alloc(int64_t capacity, void** buffer);
int i4b_peer_buffer_free(void* buffer);
/* CUDA-IPC handle (I4B_IPC_HANDLE_BYTES opaque bytes) of an exchange buffer, for the other ranks; open a
 * handle received from another rank (peer access enabled); close a mapping opened that way. */
int i4b_ipc_get_handle(void* buffer, void* handle);
int i4b_ipc_open_handle(const void* handle, void** buffer);
int i4b_ipc_close_handle(void* buffer);

/* y[M, N] = sum over the group's ranks of (this rank's x @ W_hat^T), in x's dtype.  prologue 0: x[M, K]
 * rows of stride_xm, x_dtype I4B_BF16 or I4B_F16, unit stride along K; I4B_PROLOGUE_SWIGLU: x = silu(g) * u
 * of src = x = (g | u) rows [M, 2K], as i4b_w4a16_matmul_prologue does (bf16; delta, norm_weight and
 * resid_out unused).  I4B_PROLOGUE_RMSNORM is rejected: a K shard does not hold the whole row the norm
 * needs.  1 <= M <= 32 and M * N <= capacity.  Needs no
 * workspace; sizes that would need the workspace split-K (K > 8192) or more CTAs than the device has SMs
 * return I4B_ERR_SHAPE.  world == 1 skips the exchange. */
int i4b_w4a16_matmul_allreduce(const i4b_peer_group* group, int prologue, const void* x, int x_dtype,
                               const void* delta, const void* norm_weight, float eps, void* resid_out, int64_t M,
                               int64_t K, int64_t stride_xm, const int32_t* qweight, int64_t N, int64_t stride_qk,
                               const uint16_t* scales, const uint16_t* zeros, int64_t stride_sg, int group_size,
                               void* y, int64_t stride_ym, void* stream);

/* Greedy next token of rows whose vocabulary is split over the ranks of a peer group (vocab-parallel
 * lm_head): out[r] = index of the first maximum of the concatenated row, where this rank holds bf16 columns
 * [offset, offset + n) at x + r * stride_x.  Each rank finds its own first maximum; the candidates are
 * exchanged through the exchange buffers (two fp32 words per row) and compared in rank order, so every rank
 * gets torch.argmax of the full row without gathering the logits.  rows <= SMs and 2 * rows <= capacity.
 * Replaces, under tensor parallelism, the all-gather of the logits and the argmax of the reference's greedy
 * decode loop (benchmarks/eval_llama.py:121-183, logits[:, -1].argmax(-1)); same group rules as above. */
int i4b_argmax_allreduce(const i4b_peer_group* group, const void* x, int64_t rows, int64_t n, int64_t stride_x,
                         int64_t offset, int64_t* out, void* stream);

/* ---- Decode-step glue of a Llama layer (bf16, head_dim 64), for the model-level caller of the
 * matmuls.  No counterpart in the reference, which runs these steps as transformers' torch ops
 * (benchmarks/eval_llama.py:121-183); each reproduces transformers' bf16 rounding points.
 * `pos` is a device int64 holding the decode position, so the calls can be captured in a CUDA graph. */

/* h[rows, H] = bf16(h + delta) (delta may be NULL); out = bf16(w * bf16(h * rsqrt(mean(h^2) + eps))).
 * Rows contiguous, H % 8 == 0, 16-byte aligned (LlamaRMSNorm after the residual add). */
int i4b_add_rmsnorm(void* h, const void* delta, const void* weight, void* out, int64_t rows, int64_t H, float eps,
                    void* stream);

/* Rotary embedding of one token per sequence.  qkv[B, (nq + 2 nkv) * 64] holds q, k, v heads in that order;
 * cos/sin tables [max_seq, 64]; writes rotated q to q_out[B, nq, 64] and rotated k / raw v to
 * k_cache / v_cache[B, nkv, max_seq, 64] at position *pos (apply_rotary_pos_emb + cache update). */
int i4b_rope_kv_cache(const void* qkv, const void* cos_table, const void* sin_table, const int64_t* pos, void* q_out,
                      void* k_cache, void* v_cache, int64_t B, int64_t nq, int64_t nkv, int64_t head_dim,
                      int64_t max_seq, void* stream);

/* out[B, nq * 64] = softmax(q . K^T * scale) . V over cache positions 0..*pos, query head h reading kv head
 * h / (nq / nkv) (grouped-query attention); fp32 softmax.  max_seq <= 49152.  The positions of a head
 * are split over a cluster of up to 8 CTAs whose partial softmax sums combine in a fixed order. */
int i4b_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos, void* out,
                         int64_t B, int64_t nq, int64_t nkv, int64_t head_dim, int64_t max_seq, float scale,
                         void* stream);

/* y[B, I] = bf16(bf16(silu(g)) * u) with gate_up[B, 2I] = (g | u); I % 8 == 0, 16-byte aligned. */
int i4b_silu_mul(const void* gate_up, void* y, int64_t B, int64_t I, void* stream);

/* out[r] = index of the first maximum of bf16 row x[r, 0..n) (greedy decoding, as torch.argmax). */
int i4b_argmax_rows(const void* x, int64_t rows, int64_t n, int64_t* out, void* stream);

/* ---- Persistent decode of all decoder layers (one launch per token step) ----
 *
 * Replaces, for batch <= 8 single-token steps of a Llama-shaped W4A16 model on
 * one GPU, the reference's per-layer sequence inside transformers' Llama with
 * Int4Linear projections (int4_triton/qlinear.py:8-43 -> gemm.py:185-220 per
 * projection, benchmarks/eval_llama.py:121-183): RMSNorm, q/k/v, rotary
 * embedding, KV-cache write, attention, o_proj + residual, RMSNorm, gate/up,
 * SiLU * up, down_proj + residual, for every layer, in ONE cooperative kernel.
 * Weights are the quantize_int4 triples re-laid by i4b_tile_w4; the gate/up
 * projection has its rows interleaved (row 2j = gate row j, row 2j + 1 = up
 * row j).  Numerics follow transformers' bf16 rounding points; attention is
 * fp32 inside. */
typedef struct i4b_decode_model {
  int32_t layers, hidden, heads, kv_heads, head_dim, intermediate, vocab;
  int32_t group_size; /* 32, 64 or 128 */
  int32_t batch;      /* tokens this step, 1..8 (one per sequence, all at position *pos) */
  int32_t max_seq;    /* positions of the caches and the rotary tables */
  int32_t cache_batch; /* sequences the caches hold (>= batch) */
  float eps;          /* RMSNorm epsilon */
  float attn_scale;   /* softmax scale, normally head_dim^-0.5 */
  const int64_t* tokens; /* device [batch] token ids */
  const int64_t* pos;    /* device [1] position of this step */
  const void* embed;     /* bf16 [vocab, hidden] */
  const void* w_qkv;     /* tiled [layers] x i4b_tile_w4_bytes((heads + 2 kv_heads) * 64, hidden) */
  const void* w_o;       /* tiled [layers] x i4b_tile_w4_bytes(hidden, heads * 64) */
  const void* w_gu;      /* tiled [layers] x i4b_tile_w4_bytes(2 * intermediate, hidden), rows interleaved */
  const void* w_down;    /* tiled [layers] x i4b_tile_w4_bytes(hidden, intermediate) */
  const void* ln1;       /* bf16 [layers, hidden] input_layernorm weights */
  const void* ln2;       /* bf16 [layers, hidden] post_attention_layernorm weights */
  const void* cos_table; /* bf16 [max_seq, 64] */
  const void* sin_table; /* bf16 [max_seq, 64] */
  void* k_cache;         /* bf16 [layers, cache_batch, kv_heads, max_seq, 64] */
  void* v_cache;         /* bf16 [layers, cache_batch, kv_heads, max_seq, 64] */
  void* h_out;           /* bf16 [batch, hidden]: the residual stream after the last layer */
  /* Tensor parallelism: NULL (or world 1) for one rank.  Otherwise heads, kv_heads and intermediate are
   * this rank's shares, the weights its shards (q/k/v and gate/up split along N, o and down along K) and
   * the caches hold its kv heads.  The o / down epilogues store each fp32 partial output, together with a
   * tag naming the step and stage, as one 64-bit word into every rank's exchange buffer (each of at least
   * i4b_decode_peer_capacity outputs, used by no other call); the stages that consume the residual stream
   * poll those words until the tags match (bounded) and add the ranks' partials in rank order: every rank
   * ends with the same h_out, and no fence or flag is needed between ranks.  All ranks must make the same
   * sequence of calls on one group. */
  const i4b_peer_group* peers;
} i4b_decode_model;

/* Capacity (outputs) of each exchange buffer of a tensor-parallel i4b_decode_layers group. */
int64_t i4b_decode_peer_capacity(int32_t layers, int32_t world, int32_t hidden);

/* Bytes of the tiled form of a quantize_int4 triple; 0 when N % 16, K % 512 or G is unsupported. */
size_t i4b_tile_w4_bytes(int64_t N, int64_t K, int group_size);

/* Re-lay qweight[K/8, N] (+ scales / zeros [K/G, N]) into 16-column x 512-k pieces of packed words (4 KB)
 * followed by each group's dequantization constants (128 bytes per group: bf16 128 + zero, the scale's top
 * 8 bits, the scale's remainder), slab by slab, the order in which the persistent decode streams them. */
int i4b_tile_w4(const int32_t* qweight, int64_t N, int64_t stride_qk, const uint16_t* scales, const uint16_t* zeros,
                int64_t stride_sg, int64_t K, int group_size, void* out, void* stream);

/* Workspace of i4b_decode_layers.  It must be zero before its first use; every call leaves it zero again.
 * Calls that share a workspace must not overlap in time. */
int i4b_decode_workspace_size(const i4b_decode_model* model, size_t* bytes);

/* One decode step through every layer: h_out = residual stream after the last layer (the final norm and
 * the lm_head are separate calls).  Writes k and v of position *pos into the caches. */
int i4b_decode_layers(const i4b_decode_model* model, void* workspace, size_t workspace_bytes, void* stream);

/* Diagnostic hook: when buffer is not null (device memory of at least SMs x layers x 5 x 16 x 8 bytes),
 * later i4b_decode_layers launches record uint64 stamps per (CTA, layer, stage) as [CTA][layer][stage][16]:
 * slots 0-6 are SM clock cycles, slot 7 the %globaltimer (ns) at stage entry, slots 8-11 warp 0's
 * cycles waiting for weights, cycles in the piece MMAs, piece count, and the producer's lead in pieces.  Stages: qkv, attention,
 * o_proj, gate/up, down_proj.  Projection stages: entry, dependency met, activations staged, pieces done,
 * epilogue done, fence done, published.  Attention: entry, dependency met, queries ready, partial written,
 * fence done, ticket taken, combined and published.  Process-wide; null turns it off. */
void i4b_set_decode_trace(void* buffer, size_t bytes);

/* Tuning hook for the tcgen05 GEMMs (W4 above the register-dequant range, W16 M > 16): tile 1..4 = the
 * shared-memory-operand kernel (1: 128x128, 2: 256x128, 3: 128x256, 4: 256x256; K splits 1, 2 or 4), tile
 * 5..8 = INT4 only, the TMEM-weight kernel with 128 weight rows x 256 / 128 / 64 / 32 tokens per CTA (K
 * splits 1, 2, 4 or 8); 0 keeps the automatic choice.  Process-wide.  Changes the workspace size a later
 * i4b_w4a16_workspace_size / i4b_w16a16_workspace_size reports.  No counterpart in the reference. */
void i4b_set_gemm_override(int tile, int splits);

/* Tuning hook: the largest M (8..32) for which i4b_w4a16_matmul runs the register-dequant kernels rather
 * than the tcgen05 GEMM; any other value restores the default routing (see i4b_w4a16_matmul).
 * Process-wide; changes the workspace size a later i4b_w4a16_workspace_size reports.  No counterpart in
 * the reference. */
void i4b_set_w4_small_m_override(int max_m);

/* Device-side error flags raised by kernels of this library on `device`
 * (a bounded wait that expired sets bit 0; a wait for another rank of a peer
 * group that expired sets bit 1).  Synchronises that device;
 * clear != 0 resets the flags.  Returns -1 if the flags cannot be read. */
int i4b_device_error_flags(int device, int clear);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* INT4_B200_H */
