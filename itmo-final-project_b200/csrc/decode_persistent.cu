// Persistent decode step: every decoder layer of a Llama-shaped W4A16 model for one token per sequence
// (batch <= 8), in ONE cooperative launch with one CTA per SM.
//
// The reference decodes through transformers' Llama with Int4Linear projections
// (int4_triton/qlinear.py:8-43, benchmarks/eval_llama.py:121-183): per layer four
// W4A16 GEMV launches (gemm.py:185-220) plus some forty torch kernels, each a
// dependent launch whose fixed cost (launch, ramp-up, drain) is several times the
// ~0.3-1.4 us it takes to stream one projection's packed weights from HBM.  Here
// the whole stack of layers is one kernel, organised around the fact that the
// weights do not depend on the data:
//
// * Weight stream.  Each CTA owns a fixed list of 16-column slabs of the four
//   projections of every layer (the same list in every layer; every stage's
//   slabs spread evenly over all CTAs).  A producer warp streams those slabs, as
//   4 KB pieces of packed words plus their scales and zeros, from HBM into a
//   ring of shared-memory slots with bulk copies
//   (cp.async.bulk, completion on an mbarrier per slot), in the order the CTA
//   will use them, running ahead across stage and layer boundaries as far as the
//   ring allows.  The packed weights are pre-tiled once (i4b_tile_w4) so that
//   each piece is one contiguous copy.
// * Stages.  Per layer: (1) qkv GEMV with the RMSNorm prologue, (2) attention
//   with the rotary embedding and the KV-cache write, (3) o_proj GEMV with the
//   residual add, (4) gate/up GEMV (rows interleaved gate/up) with the RMSNorm
//   prologue and the SiLU*up epilogue, (5) down_proj GEMV with the residual add.
//   A stage needs every output of the previous one, so each stage ends with one
//   atomic increment per CTA of a counter in the workspace, and the next stage's
//   CTAs wait (thread 0, acquire loads, bounded) until it reaches its total.
//   While compute warps wait, the producer keeps streaming: the critical path of
//   a layer is five such hand-offs plus compute on weights already on chip.
// * GEMV arithmetic is the decode GEMV's (gemv_w4.cu): one lop3 turns a nibble
//   pair into the bf16 pair (128 + q_i, 128 + q_{i+4}), three bf16x2 operations
//   turn it into the reference's weights (q - z) * s rounded once to bf16
//   (dq_pair), which are the A fragment of an mma.m16n8k16 with a slab's 16
//   output columns as rows and tokens as the 8 columns.  The 8 compute warps
//   split a stage's pieces; fp32 partials of one slab are added in a fixed order.
// * Attention: items (token, kv head, sequence split), one per CTA; the last
//   split of a (token, kv head) to finish (atomic ticket) combines the fp32
//   partial softmax sums in split order.
//
// Every wait is bounded (I4B_WAIT_LIMIT_NS) and checks an abort word, so an error
// in one CTA ends all of them; the last CTA to leave resets the counters.  All
// sums are in a fixed order: results are identical from run to run.
#include <math.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace i4b {

namespace {

constexpr int kCW = 8;               // compute warps (two per SM sub-partition: 168 registers each)
constexpr int kCT = kCW * 32;        // compute threads
constexpr int kThreads = kCT + 32;   // + the producer warp
constexpr int kAW = 8;               // warps of an attention item (one per 8 of the 64 head dims)
constexpr int kAT = kAW * 32;
constexpr int kSlabW = 16;           // output columns of one slab (the rows of one m16n8k16 tile)
constexpr int kPieceK = 512;         // k of one weight piece
constexpr int kPieceW = 4096;        // packed-word bytes of one piece (16 columns x 512 k x 4 bit)
constexpr int kRecB = 128;           // bytes of one group's dequantization records in a piece (8 x 16 bytes)
constexpr int kMaxSlots = 48;
constexpr int kMaxCtas = 160;
constexpr int kMaxItems = 24;        // slabs per CTA per layer
constexpr int kMaxTok = 8;
constexpr int kHD = 64;
constexpr int kPartRow = 68;  // floats per attention partial: o[64], m, l, padding to 16 bytes
constexpr int kAttnMinSplit = 32;  // cached positions per attention split, at least (short contexts use fewer)

enum { G_QKV = 0, G_O = 1, G_GU = 2, G_DOWN = 3 };                       // GEMV stages
enum { C_QKV = 0, C_ATTN = 1, C_O = 2, C_GU = 3, C_DOWN = 4, C_LAYER = 5 };  // counters of a layer

// Scalars and pointers of one launch; the kernel copies them to shared memory once.
struct DkHot {
  i4b_decode_model m;
  int nslab[4], npiece[4];  // 16-column slabs and 512-k pieces per slab of qkv, o, gate/up, down
  int64_t layer_bytes[4];   // tiled bytes of one layer's projection
  int piece_bytes, nslot, nsplit, gqa, qkv_n, q_n;
  int xpitch, off_x, off_xs, off_part;
  unsigned int* ctr;  // [layers][5] stage counters | [B * kv_heads] attention tickets | done | abort
  int n_ctr, i_ticket, i_done, i_abort;
  float* apart;       // attention partials [B * kv_heads * nsplit][gqa][kPartRow]
  uint16_t* qkv;      // [B][qkv_n]
  uint16_t* att;      // [B][q_n]
  uint16_t* act;      // [B][intermediate]
  unsigned long long* trace;  // optional: [grid][layers][5 stages][8] %globaltimer stamps, or null
  // Tensor parallelism (tp_world > 1): every rank's exchange buffer as mapped here (layout below), this
  // rank, the CTA that stores the summed residual rows in stages G_QKV / G_GU, and the residual rows
  // [kMaxTok][hidden] after update u in hbuf[u & 1].  Update u = 2l adds layer l's o_proj outputs of all
  // ranks, u = 2l + 1 its down_proj outputs.
  uint8_t* xb[kArMaxRanks];
  int tp_world, tp_rank;
  int writer[4];
  uint16_t* hbuf[2];
};

struct DkParams {
  DkHot h;
  uint8_t nitems[kMaxCtas];
  uint16_t items[kMaxCtas][kMaxItems];  // (stage << 14) | slab, in stage order
};

// Trace stamps per (CTA, layer, stage), 8 slots of SM clock cycles (clock64): 0 entry, 1 dependency met,
// 2 activations staged, 3 pieces done, 4 epilogue done, 5 fence done, 6 published; slot 7 holds
// %globaltimer at entry, the time base shared by all SMs.
// Slots 8..15: warp 0's cycles waiting for weight pieces, its cycles in the piece MMAs, its piece count,
// the producer's issued-piece count relative to this stage's first piece, at stage entry; the clocks at
// which the first and the last compute warp ended their pieces, and the last warp's index.
constexpr int kTraceSlots = 16;
__device__ __forceinline__ void stamp(const DkHot& P, int l, int st, int k) {
  if (P.trace && threadIdx.x == 0) {
    unsigned long long* t = P.trace + ((int64_t(blockIdx.x) * P.m.layers + l) * 5 + st) * kTraceSlots;
    t[k] = clock64();
    if (k == 0) t[7] = globaltimer_ns();
  }
}
__device__ __forceinline__ void trace_put(const DkHot& P, int l, int st, int k, long long v) {
  if (P.trace) P.trace[((int64_t(blockIdx.x) * P.m.layers + l) * 5 + st) * kTraceSlots + k] = (unsigned long long)v;
}

__device__ unsigned int g_dk_err = 0;

__device__ __forceinline__ float bfv(uint32_t bits16) { return __uint_as_float(bits16 << 16); }
__device__ __forceinline__ uint32_t bfr(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory"); }
// attention items run on the first kAW compute warps only, with their own barrier
__device__ __forceinline__ void abar() { asm volatile("bar.sync 2, %0;" ::"n"(kAT) : "memory"); }

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned int ld_relaxed_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint16_t ldcg16(const uint16_t* p) {
  return __ldcg(reinterpret_cast<const unsigned short*>(p));
}
__device__ __forceinline__ uint4 ldcg128(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Wait until *c >= target (acquire).  False on the abort word or after I4B_WAIT_LIMIT_NS.
__device__ bool wait_counter(const unsigned int* c, unsigned int target, const unsigned int* abort_word) {
  if (ld_acquire_u32(c) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_u32(c) >= target) return true;
    if ((i & 31u) == 0) {
      if (ld_relaxed_u32(abort_word)) return false;
      if (globaltimer_ns() - t0 > I4B_WAIT_LIMIT_NS) return false;
    }
  }
}

// ---- tensor parallelism: exchange buffer of rank p (i4b_peer_group), as this launch uses it:
//   [epoch u32 | 256 B] ... [tagged partial outputs u64 [layers][2][world][kMaxTok][hidden], at kArDataOff]
// Each exchanged fp32 partial travels with its tag in ONE 64-bit store (value in the low word, tag in the
// high word), and the reader polls the words it needs until every tag is the one it expects: the data is its
// own flag, so neither a memory fence nor a counter sits between a producer and its readers (a system-scope
// fence would wait for everything the SM has in flight, the weight prefetch included).  The tag of
// (step e, layer l, o_proj / down_proj s) is e * 2L + 2l + s + 1: never 0 (the zero-filled buffer), and
// different from every earlier use of the same words.
__device__ __forceinline__ uint64_t* xword(const DkHot& P, int p, int l, int s, int src) {
  return reinterpret_cast<uint64_t*>(P.xb[p] + kArDataOff) +
         int64_t((l * 2 + s) * P.tp_world + src) * kMaxTok * P.m.hidden;
}
__device__ __forceinline__ unsigned int xtag(unsigned int ep, int l, int s, int layers) {
  return ep * unsigned(2 * layers) + unsigned(2 * l + s) + 1u;
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void ld_relaxed_sys_u64x2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// The 8 partials (token t, columns 8ch..8ch+7) of source rank `src` for update u, once all carry `tag`.
// Bounded: false after I4B_WAIT_LIMIT_NS or when another CTA aborted.
__device__ __forceinline__ bool poll_partials(const DkHot& P, int u, int src, int t, int ch, unsigned int tag,
                                              const unsigned int* abort_word, float (&v)[8]) {
  const uint64_t* d = xword(P, P.tp_rank, u >> 1, u & 1, src) + int64_t(t) * P.m.hidden + 8 * ch;
  uint64_t w[8];
  uint64_t t0 = 0;
  for (uint32_t i = 1;; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) ld_relaxed_sys_u64x2(d + 2 * j, w[2 * j], w[2 * j + 1]);
    bool ready = true;
#pragma unroll
    for (int j = 0; j < 8; ++j) ready = ready && unsigned(w[j] >> 32) == tag;
    if (ready) break;
    if (i == 1) t0 = globaltimer_ns();
    if ((i & 15u) == 0) {
      if (ld_relaxed_u32(abort_word)) return false;
      if (globaltimer_ns() - t0 > I4B_WAIT_LIMIT_NS) return false;
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(unsigned(w[j]));
  return true;
}
// Eight residual values (token t, columns 8ch..8ch+7) after update u: bf16(h_{u-1} + bf16(sum over ranks,
// in rank order, of their fp32 partials)) -- the one-rank epilogue's rounding, bf16(h + bf16(sum)).
// h_{-1} is the token's embedding row.  The partials are polled until they carry this step's tag; a wait
// that gives up clears *ok.
__device__ __forceinline__ uint4 residual_chunk(const DkHot& P, int u, int t, int ch, unsigned int ep,
                                                const unsigned int* abort_word, bool* ok) {
  const i4b_decode_model& m = P.m;
  const int H = m.hidden;
  uint4 hv;
  if (u == 0) {
    int64_t id = m.tokens[t];
    if (id < 0 || id >= m.vocab) id = 0;
    hv = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(m.embed) + id * H + 8 * ch));
  } else {
    hv = ldcg128(P.hbuf[(u - 1) & 1] + int64_t(t) * H + 8 * ch);
  }
  float sm[8];
  const unsigned int tag = xtag(ep, u >> 1, u & 1, m.layers);
#pragma unroll 1
  for (int r = 0; r < P.tp_world; ++r) {
    float v[8];
    if (!poll_partials(P, u, r, t, ch, tag, abort_word, v)) {
      *ok = false;
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) sm[i] = r == 0 ? v[i] : sm[i] + v[i];
  }
  const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    o[i] = bfr(bfv(hw[i] & 0xFFFFu) + bfv(bfr(sm[2 * i]))) | (bfr(bfv(hw[i] >> 16) + bfv(bfr(sm[2 * i + 1]))) << 16);
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// mbarrier phase wait, bounded, giving up early when another CTA aborted.  Each probe lets the thread
// sleep in hardware until the phase completes (or ~1 us), so that a waiting warp -- the producer whenever
// the ring is full -- takes no issue slots from the compute warps.
__device__ bool wait_slot(uint64_t* bar, uint32_t parity, const unsigned int* abort_word) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (ld_relaxed_u32(abort_word)) return false;
      if (globaltimer_ns() - t0 > I4B_WAIT_LIMIT_NS) return false;
    }
  }
}

__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int i) { return and_or(w >> (4 * i), 0x000F000Fu, 0x43004300u); }

// mma.m16n8k16 bf16 -> fp32 without `volatile`: a pure function of its operands, so the compiler may
// schedule the shared-memory loads of later steps ahead of it.
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16_first(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.0f));
}

// One 512-k piece of a 16-column slab, by one warp: acc[e] += the piece's contribution to slab column
// r (e = 0, 1) and r + 8 (e = 2, 3) for tokens 2c + (e & 1), r = lane / 4, c = lane % 4.  Step j (32 k)
// gives lane (r, c) the packed words of k-row 4j + c at columns r and r + 8: the rows r and r + 8 of the
// A fragment.  wb: the piece in shared memory; xb: this lane's activations at the piece's first k.
// Every weight is dequantized exactly as the reference does -- (q - z) * s rounded once to bf16
// (dq_pair) -- so y = sum_k x_k * bf16(w_k) with fp32 accumulation.  The two k16 halves of a step
// accumulate in separate registers, acc and a1 (two independent MMA chains), which the caller carries
// from piece to piece of a slab and adds only when it stores the slab's partial: no piece waits for the
// previous one's last MMA.
template <int SPS>
__device__ __forceinline__ void piece_mma(const uint8_t* wb, const uint8_t* xb, int lane, float (&acc)[4],
                                          float (&a1)[4]) {
  const int r = lane >> 2;
  DqParams dp[2];
  // four blocks of four 32-k steps: the loads of a block are scheduled together, the block loop is not
  // unrolled (instruction cache); SPS divides 4, so group boundaries fall inside blocks
#pragma unroll 1
  for (int j0 = 0; j0 < 16; j0 += 4)
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const int j = j0 + jj;
    if (jj % SPS == 0) {  // a new group: the dequantization constants of columns r (low halves), r + 8 (high)
      const uint4 rc = *reinterpret_cast<const uint4*>(wb + kPieceW + ((j / SPS) * 8 + r) * 16);
      dp[0].zz = __byte_perm(rc.x, 0u, 0x1010);
      dp[0].shi = __byte_perm(rc.y, 0u, 0x1010);
      dp[0].slo = __byte_perm(rc.z, 0u, 0x1010);
      dp[1].zz = __byte_perm(rc.x, 0u, 0x3232);
      dp[1].shi = __byte_perm(rc.y, 0u, 0x3232);
      dp[1].slo = __byte_perm(rc.z, 0u, 0x3232);
    }
    const uint2 w2 = *reinterpret_cast<const uint2*>(wb + (j * 32 + lane) * 8);
    uint32_t af[2][4];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      af[s][0] = dq_pair<false>(nib_pair(w2.x, 2 * s), dp[0]);
      af[s][1] = dq_pair<false>(nib_pair(w2.y, 2 * s), dp[1]);
      af[s][2] = dq_pair<false>(nib_pair(w2.x, 2 * s + 1), dp[0]);
      af[s][3] = dq_pair<false>(nib_pair(w2.y, 2 * s + 1), dp[1]);
    }
    const uint4 b = *reinterpret_cast<const uint4*>(xb + j * 64);
    mma_bf16(acc, af[0], b.x, b.y);
    mma_bf16(a1, af[1], b.z, b.w);
  }
}

struct Smem {
  uint64_t full[kMaxSlots];
  uint64_t empty[kMaxSlots];
  float inv[kMaxTok];
  float wss[kCW * kMaxTok];  // per-warp sums of squares of the RMSNorm rows
  uint16_t slab[kMaxItems];
  uint8_t stage[kMaxItems];
  uint16_t poff[kMaxItems];  // piece offset of each item inside the CTA's layer sequence
  int nit, ppl;
  int flag;   // 1 until a wait fails in this CTA (then 0 for the rest of the launch)
  unsigned int ep;  // tensor parallelism: this launch's epoch (steps this rank's group has completed)
  int tflag;  // the attention ticket said: this CTA combines
  volatile int prod_seq;  // pieces issued by the producer so far (diagnostics)
  long long wexit[kCW];   // each compute warp's clock at the end of its pieces (diagnostics)
};

// The launch's shared memory as file-scope symbols: device functions that name them directly (rather than
// through a pointer or reference parameter) compile every access to a shared-memory instruction instead of
// a generic one.
__shared__ Smem dk_S;
__shared__ DkHot dk_P;
extern __shared__ __align__(128) uint8_t dk_smem[];  // ring | activations / attention scratch | partials

constexpr int kResPerThread = 4;  // residual values per thread: o / down slabs x tokens x 16 <= kCT * 4

// Stage the activations of GEMV stage g into shared memory: x permuted to the nibble-pair order of the
// A fragments, [token][k / 8] x 16 bytes with row pitch xpitch.  Written as plain (not unrolled) loops:
// this code runs once per stage and must stay small in the instruction cache.  (1) every 16-byte chunk
// of every token row is put in flight with cp.async straight into its staging slot; (2) RMSNorm stages
// take per-token sums of squares over the staged rows (fixed order: lanes, then warps); (3) each thread
// rewrites its chunks in place: x = bf16(w * bf16(h * rsqrt(mean(h^2) + eps))) (LlamaRMSNorm) where
// needed, then the permutation.
template <bool TP>
__device__ __noinline__ void stage_x(int g, int l, int K) {
  const DkHot& P = dk_P;
  Smem& S = dk_S;
  uint8_t* const smem = dk_smem;
  const i4b_decode_model& m = P.m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = m.batch, H = m.hidden;
  const bool norm = g == G_QKV || g == G_GU;
  const bool emb = g == G_QKV && l == 0;
  const uint16_t* nw = static_cast<const uint16_t*>(g == G_QKV ? m.ln1 : m.ln2) + int64_t(l) * H;
  const uint16_t* src = g == G_O ? P.att : g == G_DOWN ? P.act : static_cast<const uint16_t*>(m.h_out);
  const int64_t stride = g == G_O ? P.q_n : g == G_DOWN ? m.intermediate : H;
  uint8_t* sx = smem + P.off_x;
  const int nch = K / 8, lg = 31 - __clz(nch), total = B << lg;  // chunks per row: a power of two
  if (TP && (g == G_GU || (g == G_QKV && l > 0))) {
    // tensor parallelism: the residual rows are the previous update's rows plus all ranks' partials;
    // one CTA also stores them for the next update
    const int u = g == G_GU ? 2 * l : 2 * l - 1;
    uint16_t* hout = int(blockIdx.x) == P.writer[g] ? P.hbuf[u & 1] : nullptr;
    const unsigned int* abort_word = P.ctr + P.i_abort;
    bool ok = true;
#pragma unroll 1
    for (int idx = tid; idx < total; idx += kCT) {
      const int t = idx >> lg, ch = idx & (nch - 1);
      const uint4 v = residual_chunk(P, u, t, ch, S.ep, abort_word, &ok);
      *reinterpret_cast<uint4*>(sx + t * P.xpitch + ch * 16) = v;
      if (hout) *reinterpret_cast<uint4*>(hout + int64_t(t) * H + 8 * ch) = v;
    }
    if (!ok) S.flag = 0;  // a partial that never arrived: the stage fails (checked after the barrier)
    cbar();
  } else {
#pragma unroll 1
    for (int idx = tid; idx < total; idx += kCT) {
      const int t = idx >> lg, ch = idx & (nch - 1);
      const uint16_t* row = src + t * stride;
      if (emb) {
        int64_t id = m.tokens[t];
        if (id < 0 || id >= m.vocab) id = 0;
        row = static_cast<const uint16_t*>(m.embed) + id * H;
      }
      cp_async_16(sx + t * P.xpitch + ch * 16, row + 8 * ch, 16);
    }
    cp_async_commit();
    cp_async_wait<0>();
    cbar();
  }
  if (norm) {
#pragma unroll 1
    for (int t = 0; t < B; ++t) {
      float ss = 0.0f;
#pragma unroll 1
      for (int ch = tid; ch < nch; ch += kCT) {
        const uint4 v = *reinterpret_cast<const uint4*>(sx + t * P.xpitch + ch * 16);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float lo = bfv(u[i] & 0xFFFFu), hi = bfv(u[i] >> 16);
          ss = fmaf(lo, lo, ss);
          ss = fmaf(hi, hi, ss);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
      if (lane == 0) S.wss[warp * kMaxTok + t] = ss;
    }
    cbar();
    if (tid < B) {
      float sum = 0.0f;
      for (int w = 0; w < kCW; ++w) sum += S.wss[w * kMaxTok + tid];
      S.inv[tid] = rsqrtf(sum / float(K) + m.eps);
    }
    cbar();
  }
#pragma unroll 1
  for (int idx = tid; idx < total; idx += kCT) {
    const int t = idx >> lg, ch = idx & (nch - 1);
    uint4* pchunk = reinterpret_cast<uint4*>(sx + t * P.xpitch + ch * 16);
    const uint4 v = *pchunk;
    uint32_t u[4] = {v.x, v.y, v.z, v.w};
    if (norm) {
      const float inv = S.inv[t];
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(nw + 8 * ch));
      const uint32_t wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        u[i] = bfr(bfv(wa[i] & 0xFFFFu) * bfv(bfr(bfv(u[i] & 0xFFFFu) * inv))) |
               (bfr(bfv(wa[i] >> 16) * bfv(bfr(bfv(u[i] >> 16) * inv))) << 16);
    }
    // (x0,x4) (x1,x5) (x2,x6) (x3,x7): the nibble-pair order of the A fragments
    *pchunk = make_uint4(__byte_perm(u[0], u[2], 0x5410), __byte_perm(u[0], u[2], 0x7632),
                         __byte_perm(u[1], u[3], 0x5410), __byte_perm(u[1], u[3], 0x7632));
  }
}

// One GEMV stage of layer l for this CTA's slabs of it.  False on a failed wait.
template <int SPS, bool TP>
__device__ __noinline__ bool gemv_stage(int g, int l) {
  const DkHot& P = dk_P;
  Smem& S = dk_S;
  uint8_t* const smem = dk_smem;
  const i4b_decode_model& m = P.m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int ib = 0, n = 0;
  for (int i = 0; i < S.nit; ++i) {
    if (S.stage[i] < g) ++ib;
    else if (S.stage[i] == g) ++n;
  }
  if (n == 0) return true;
  const int st_id = g == G_QKV ? C_QKV : g == G_O ? C_O : g == G_GU ? C_GU : C_DOWN;
  stamp(P, l, st_id, 0);
  const unsigned int* abort_word = P.ctr + P.i_abort;
  if (g == G_QKV || g == G_GU) {  // the RMSNorm weights do not depend on the previous stage: fetch them now
    const uint16_t* nw = static_cast<const uint16_t*>(g == G_QKV ? m.ln1 : m.ln2) + int64_t(l) * m.hidden;
#pragma unroll 1
    for (int ch = tid; ch < m.hidden / 8; ch += kCT) asm volatile("prefetch.global.L1 [%0];" ::"l"(nw + 8 * ch));
  }
  // ---- dependency: every output of the previous stage
  if (tid == 0) {
    const unsigned int* c = nullptr;
    unsigned int target = 0;
    if (g == G_QKV) {
      if (l > 0) c = P.ctr + (l - 1) * C_LAYER + C_DOWN, target = unsigned(P.nslab[G_DOWN]);
    } else if (g == G_O) {
      c = P.ctr + l * C_LAYER + C_ATTN, target = unsigned(m.batch * m.kv_heads);
    } else if (g == G_GU) {
      c = P.ctr + l * C_LAYER + C_O, target = unsigned(P.nslab[G_O]);
    } else {
      c = P.ctr + l * C_LAYER + C_GU, target = unsigned(P.nslab[G_GU]);
    }
    if (c != nullptr && !wait_counter(c, target, abort_word)) S.flag = 0;  // sticky: errors are never cleared
  }
  cbar();
  if (!S.flag) return false;
  stamp(P, l, st_id, 1);
  const int K = g == G_DOWN ? m.intermediate : (g == G_O ? P.q_n : m.hidden);
  stage_x<TP>(g, l, K);  // under tensor parallelism it also waits for the other ranks' partials
  cbar();
  if (!S.flag) return false;
  stamp(P, l, st_id, 2);
  // residual inputs of the o_proj / down_proj epilogue: loaded here, consumed after the pieces
  uint16_t* h = static_cast<uint16_t*>(m.h_out);
  const int H = m.hidden;
  const int B = m.batch;
  constexpr int kRes = kResPerThread;
  uint16_t res[kRes];
  const bool tp_out = TP && (g == G_O || g == G_DOWN);
  if ((g == G_O || g == G_DOWN) && !tp_out) {
#pragma unroll
    for (int k = 0; k < kRes; ++k) {
      const int idx = tid + k * kCT;
      if (idx < n * B * kSlabW) {
        const int i = idx / (B * kSlabW), rem = idx - i * B * kSlabW, b = rem / kSlabW, col = rem % kSlabW;
        const int64_t nn = int64_t(S.slab[ib + i]) * kSlabW + col;
        if (g == G_O && l == 0) {
          int64_t id = m.tokens[b];
          if (id < 0 || id >= m.vocab) id = 0;
          res[k] = __ldg(static_cast<const uint16_t*>(m.embed) + id * H + nn);
        } else {
          res[k] = ldcg16(h + int64_t(b) * H + nn);
        }
      }
    }
  }

  // ---- pieces: piece q = i * ppi + p (slab i, k-piece p) of this stage goes to warp q % kCW; warp w's
  // sum over its pieces of slab i is partial row (i, p % kCW) of J per slab
  const int ppi = P.npiece[g], J = ppi < kCW ? ppi : kCW;
  float* part = reinterpret_cast<float*>(smem + P.off_part);
  const int r = lane >> 2, c = lane & 3;
  const uint8_t* xl = smem + P.off_x + min(r, B - 1) * P.xpitch + 16 * c;
  const int total = n * ppi;
  bool ok = true;
  float acc[4], a1[4];
  int cur = -1, cur_j = 0;
  auto flush = [&](int i, int j) {
    float* pp = part + (i * J + j) * (B * kSlabW);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = r + 8 * (e >> 1), tok = 2 * c + (e & 1);
      if (tok < B) pp[tok * kSlabW + col] = acc[e] + a1[e];
    }
  };
  const int seq0 = l * S.ppl;
  if (tid == 0) trace_put(P, l, st_id, 11, S.prod_seq - (seq0 + S.poff[ib]));
  long long t_wait = 0, t_mma = 0;
  int npc = 0;
#pragma unroll 1
  for (int q = warp; q < total; q += kCW) {
    const int i = q / ppi, pl = q - i * ppi, p = pl;
    if (i != cur) {
      if (cur >= 0) flush(cur, cur_j);
      cur = i;
      cur_j = pl % kCW;
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] = a1[e] = 0.0f;
    }
    const int seq = seq0 + S.poff[ib + i] + pl;
    const int slot = seq % P.nslot;
    const long long c0 = clock64();
    if (!wait_slot(&S.full[slot], uint32_t(seq / P.nslot) & 1u, abort_word)) {
      ok = false;
      break;
    }
    const long long c1 = clock64();
    piece_mma<SPS>(smem + slot * P.piece_bytes, xl + p * (kPieceK / 32) * 64, lane, acc, a1);
    t_wait += c1 - c0;
    t_mma += clock64() - c1;
    ++npc;
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.empty[slot]);
  }
  if (ok && cur >= 0) flush(cur, cur_j);
  if (P.trace && lane == 0) S.wexit[warp] = clock64();
  if (tid == 0) {
    trace_put(P, l, st_id, 8, t_wait);
    trace_put(P, l, st_id, 9, t_mma);
    trace_put(P, l, st_id, 10, npc);
  }
  if (!ok && lane == 0) S.flag = 0;
  cbar();
  if (P.trace && tid == 0) {  // first and last warp to finish its pieces, and which warp was last
    long long lo = S.wexit[0], hi = S.wexit[0];
    int wl = 0;
    for (int w = 1; w < kCW; ++w) {
      lo = min(lo, S.wexit[w]);
      if (S.wexit[w] > hi) hi = S.wexit[w], wl = w;
    }
    trace_put(P, l, st_id, 12, lo);
    trace_put(P, l, st_id, 13, hi);
    trace_put(P, l, st_id, 14, wl);
  }
  if (!S.flag) return false;
  stamp(P, l, st_id, 3);

  // ---- epilogue: fixed-order sum of the partials of each slab, then the stage's output operation
  if (g == G_GU) {
#pragma unroll 1
    for (int idx = tid; idx < n * B * (kSlabW / 2); idx += kCT) {
      constexpr int kH = kSlabW / 2;  // gate / up column pairs of a slab
      const int i = idx / (B * kH), rem = idx - i * B * kH, b = rem / kH, pr = rem % kH;
      float gs = 0.0f, us = 0.0f;
      for (int j = 0; j < J; ++j) {
        const float* pp = part + (i * J + j) * (B * kSlabW) + b * kSlabW;
        gs += pp[2 * pr];
        us += pp[2 * pr + 1];
      }
      const float gt = bfv(bfr(gs)), up = bfv(bfr(us));
      const float sl = bfv(bfr(gt / (1.0f + expf(-gt))));
      P.act[int64_t(b) * m.intermediate + int64_t(S.slab[ib + i]) * kH + pr] = uint16_t(bfr(sl * up));
    }
  } else {
#pragma unroll
    for (int k = 0; k < kRes; ++k) {
      const int idx = tid + k * kCT;
      if (idx >= n * B * kSlabW) break;
      const int i = idx / (B * kSlabW), rem = idx - i * B * kSlabW, b = rem / kSlabW, col = rem % kSlabW;
      float sum = 0.0f;
      for (int j = 0; j < J; ++j) sum += part[(i * J + j) * (B * kSlabW) + b * kSlabW + col];
      const int64_t nn = int64_t(S.slab[ib + i]) * kSlabW + col;
      if (g == G_QKV) {
        P.qkv[int64_t(b) * P.qkv_n + nn] = uint16_t(bfr(sum));
      } else if (tp_out) {  // this rank's fp32 partial with its tag, into every rank's buffer: one 64-bit store
        const int s2 = g == G_O ? 0 : 1;
        const uint64_t word = (uint64_t(xtag(S.ep, l, s2, m.layers)) << 32) | __float_as_uint(sum);
        for (int p = 0; p < P.tp_world; ++p) st_relaxed_sys_u64(xword(P, p, l, s2, P.tp_rank) + int64_t(b) * H + nn, word);
      } else {
        h[int64_t(b) * H + nn] = uint16_t(bfr(bfv(res[k]) + bfv(bfr(sum))));
      }
    }
  }
  cbar();
  stamp(P, l, st_id, 4);
  if (tid == 0) {
    stamp(P, l, st_id, 5);
    // release: the CTA's output stores (ordered before by the barrier) are visible before the count
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(P.ctr + l * C_LAYER + st_id), "r"(unsigned(n))
                 : "memory");
    // (the partials sent to the other ranks carry their own tags: nothing to publish for them)
  }
  stamp(P, l, st_id, 6);
  return true;
}

// Attention item a = (token b, kv head, split j) of layer l: GS query heads over cache positions of split j.
// Run by the first kAW compute warps (barrier 2); a failure clears the CTA's sticky S.flag.
template <int GS>
__device__ __noinline__ bool attention_item(int l, int a) {
  const DkHot& P = dk_P;
  Smem& S = dk_S;
  uint8_t* const smem = dk_smem;
  const i4b_decode_model& m = P.m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nkv = m.kv_heads, nsplit = P.nsplit, nq = m.heads;
  const int b = a / (nkv * nsplit), kvh = (a / nsplit) % nkv, j = a % nsplit;
  const unsigned int* abort_word = P.ctr + P.i_abort;
  const int64_t pos = *m.pos;
  const bool pvalid = pos >= 0 && pos < m.max_seq;
  const int Lp = pvalid ? int(pos) + 1 : 0;
  // splits in use: at least kAttnMinSplit positions each, so that short contexts combine fewer partials
  const int ns = max(1, min(nsplit, (Lp + kAttnMinSplit - 1) / kAttnMinSplit));
  if (j >= ns) return true;
  stamp(P, l, C_ATTN, 0);
  // scratch (the activation staging area): rotated queries, this block's keys and values, probabilities,
  // running max / sum / rescale per head, the new position's key and value
  constexpr int KP = 33;  // words per staged key row: 32 bf16 pairs + 1, so that 32 positions hit 32 banks
  float* qs = reinterpret_cast<float*>(smem + P.off_x);   // [GS][64]
  uint32_t* ks = reinterpret_cast<uint32_t*>(qs + GS * kHD);  // [64][KP] bf16 pairs
  uint16_t* vs = reinterpret_cast<uint16_t*>(ks + 64 * KP);   // [64][64]
  float* pr = reinterpret_cast<float*>(vs + 64 * kHD);        // [GS][64]
  float* sm = pr + GS * kHD;                                  // [GS] running max
  float* sl = sm + GS;                                        // [GS] running sum
  float* scr = sl + GS;                                       // [GS] rescale of this block
  uint16_t* newkv = reinterpret_cast<uint16_t*>(scr + GS);    // [2][64] rotated key, value of position pos
  const int chunk = (Lp + ns - 1) / ns;
  const int i0 = j * chunk, i1 = min(Lp, i0 + chunk);
  const int64_t head_stride = int64_t(m.max_seq) * kHD;
  const int64_t cache_off = ((int64_t(l) * m.cache_batch + b) * nkv + kvh) * head_stride;
  uint16_t* kc = static_cast<uint16_t*>(m.k_cache) + cache_off;
  uint16_t* vc = static_cast<uint16_t*>(m.v_cache) + cache_off;
  // keys (4-byte copies into conflict-free rows) and values (16-byte copies) of cached positions
  // [blk, blk + nb), all in flight at once.  Every position but pos was written by an earlier step, so the
  // first block goes out before the wait for this layer's q / k / v; row pos comes from newkv.
  auto issue_block = [&](int blk, int nb) {
#pragma unroll 1
    for (int cc = tid; cc < nb * 32; cc += kAT)
      if (blk + (cc >> 5) != pos)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(ks + (cc >> 5) * KP + (cc & 31))),
                     "l"(kc + int64_t(blk) * kHD + 2 * cc)
                     : "memory");
#pragma unroll 1
    for (int cc = tid; cc < nb * 8; cc += kAT)
      if (blk + (cc >> 3) != pos) cp_async_16(vs + cc * 8, vc + int64_t(blk) * kHD + cc * 8, 16);
    cp_async_commit();
  };
  if (i1 > i0) issue_block(i0, min(64, i1 - i0));
  if (tid == 0 && !wait_counter(P.ctr + l * C_LAYER + C_QKV, unsigned(P.nslab[G_QKV]), abort_word)) S.flag = 0;
  abar();
  if (!S.flag) {
    cp_async_wait<0>();  // nothing may land in shared memory after the CTA has moved on
    return false;
  }
  stamp(P, l, C_ATTN, 1);
  const uint16_t* qrow = P.qkv + int64_t(b) * P.qkv_n;
  const uint16_t* cosT = static_cast<const uint16_t*>(m.cos_table);
  const uint16_t* sinT = static_cast<const uint16_t*>(m.sin_table);
  // rotary embedding, apply_rotary_pos_emb's rounding: bf16(bf16(t * cos) + bf16(rotate_half(t) * sin))
  float c0 = 0.f, c1 = 0.f, s0 = 0.f, s1 = 0.f;
  if (pvalid) {
    c0 = bfv(__ldg(cosT + pos * kHD + lane));
    c1 = bfv(__ldg(cosT + pos * kHD + lane + 32));
    s0 = bfv(__ldg(sinT + pos * kHD + lane));
    s1 = bfv(__ldg(sinT + pos * kHD + lane + 32));
  }
#pragma unroll 1
  for (int hh = warp; hh < GS; hh += kAW) {
    const uint16_t* src = qrow + (kvh * GS + hh) * kHD;
    const float x0 = bfv(ldcg16(src + lane)), x1 = bfv(ldcg16(src + lane + 32));
    qs[hh * kHD + lane] = bfv(bfr(bfv(bfr(x0 * c0)) + bfv(bfr(-x1 * s0))));
    qs[hh * kHD + lane + 32] = bfv(bfr(bfv(bfr(x1 * c1)) + bfv(bfr(x0 * s1))));
  }
  if (pvalid && pos >= i0 && pos < i1) {  // this split holds the new position: write k and v to the caches
    if (warp == kAW - 1) {
      const uint16_t* src = qrow + (nq + kvh) * kHD;
      const float x0 = bfv(ldcg16(src + lane)), x1 = bfv(ldcg16(src + lane + 32));
      const uint16_t k0 = uint16_t(bfr(bfv(bfr(x0 * c0)) + bfv(bfr(-x1 * s0))));
      const uint16_t k1 = uint16_t(bfr(bfv(bfr(x1 * c1)) + bfv(bfr(x0 * s1))));
      kc[pos * kHD + lane] = k0;
      kc[pos * kHD + lane + 32] = k1;
      newkv[lane] = k0;
      newkv[lane + 32] = k1;
    } else if (warp == kAW - 2) {
      const uint16_t* src = qrow + (nq + nkv + kvh) * kHD;
      const uint16_t v0 = ldcg16(src + lane), v1 = ldcg16(src + lane + 32);
      vc[pos * kHD + lane] = v0;
      vc[pos * kHD + lane + 32] = v1;
      newkv[kHD + lane] = v0;
      newkv[kHD + lane + 32] = v1;
    }
  }
  if (tid < GS) {
    sm[tid] = -INFINITY;
    sl[tid] = 0.0f;
  }
  abar();  // rotated queries ready, the new cache row visible to this CTA
  stamp(P, l, C_ATTN, 2);

  // thread (head hh = tid / 64 + 4 pass, index x = tid % 64): position x of the block for the scores,
  // dimension x for the output, whose sum over positions it owns outright
  const int x = tid & 63, hq = tid >> 6;
  float acc[(GS + 3) / 4];
#pragma unroll
  for (int u = 0; u < (GS + 3) / 4; ++u) acc[u] = 0.0f;
  const float scale = m.attn_scale;
#pragma unroll 1
  for (int blk = i0; blk < i1; blk += 64) {
    const int nb = min(64, i1 - blk);
    if (blk != i0) issue_block(blk, nb);
    if (pos >= blk && pos < blk + nb) {  // the new position's row, from newkv (written before the last barrier)
      const int t = int(pos - blk);
      if (tid < 32) ks[t * KP + tid] = reinterpret_cast<const uint32_t*>(newkv)[tid];
      else if (tid < 32 + kHD) vs[t * kHD + tid - 32] = newkv[kHD + tid - 32];
    }
    cp_async_wait<0>();
    abar();
    // scores s[hh][x] = q[hh] . k[x] * scale
#pragma unroll
    for (int u = 0; u < (GS + 3) / 4; ++u) {
      const int hh = hq + 4 * u;
      if (hh < GS) {
        float d = 0.0f;
        const uint32_t* kr = ks + x * KP;
        const float* q = qs + hh * kHD;
#pragma unroll 8
        for (int w = 0; w < 32; ++w) {
          const uint32_t kw = kr[w];
          d = fmaf(q[2 * w], bfv(kw & 0xFFFFu), d);
          d = fmaf(q[2 * w + 1], bfv(kw >> 16), d);
        }
        pr[hh * kHD + x] = x < nb ? d * scale : -INFINITY;
      }
    }
    abar();
    // online softmax per head (warp hh)
#pragma unroll 1
    for (int hh = warp; hh < GS; hh += kAW) {
      const float x0 = pr[hh * kHD + lane], x1 = pr[hh * kHD + lane + 32];
      float mb = fmaxf(x0, x1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, o));
      const float mo = sm[hh], mn = fmaxf(mo, mb);
      const float p0 = expf(x0 - mn), p1 = expf(x1 - mn);
      float su = p0 + p1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) su += __shfl_xor_sync(0xFFFFFFFFu, su, o);
      pr[hh * kHD + lane] = p0;
      pr[hh * kHD + lane + 32] = p1;
      __syncwarp();
      if (lane == 0) {
        const float corr = expf(mo - mn);  // 0 for the first block (mo = -inf)
        scr[hh] = corr;
        sl[hh] = sl[hh] * corr + su;
        sm[hh] = mn;
      }
    }
    abar();
    // o[hh][x] = o[hh][x] * rescale + sum over the block's positions of p * v[., x]
#pragma unroll
    for (int u = 0; u < (GS + 3) / 4; ++u) {
      const int hh = hq + 4 * u;
      if (hh < GS) {
        float o = acc[u] * scr[hh];
        const float* ph = pr + hh * kHD;
#pragma unroll 4
        for (int t = 0; t < nb; ++t) o = fmaf(ph[t], bfv(vs[t * kHD + x]), o);
        acc[u] = o;
      }
    }
    abar();  // the block's keys, values and probabilities are read before the next block overwrites them
  }
  float* mine = P.apart + int64_t(a) * GS * kPartRow;
#pragma unroll
  for (int u = 0; u < (GS + 3) / 4; ++u) {
    const int hh = hq + 4 * u;
    if (hh < GS) mine[hh * kPartRow + x] = acc[u];
  }
  if (tid < GS) {
    const bool any = i1 > i0;
    mine[tid * kPartRow + 64] = any ? sm[tid] : -INFINITY;
    mine[tid * kPartRow + 65] = any ? sl[tid] : 0.0f;
  }
  abar();
  stamp(P, l, C_ATTN, 3);
  unsigned int* ticket = P.ctr + P.i_ticket + b * nkv + kvh;
  if (tid == 0) {
    __threadfence();
    stamp(P, l, C_ATTN, 4);
    S.tflag = atomicAdd(ticket, 1u) == unsigned(ns - 1) ? 1 : 0;
  }
  abar();
  stamp(P, l, C_ATTN, 5);
  if (!S.tflag) return true;
  // last split of (b, kvh): out = sum_j o_j e^(m_j - M) / sum_j l_j e^(m_j - M), splits in order.  All
  // partials are copied to shared memory first, every load in flight at once.
  __threadfence();
  const float4* base = reinterpret_cast<const float4*>(P.apart + int64_t(a - j) * GS * kPartRow);  // split 0
  // [ns][GS][kPartRow] partials, over the (now dead) key / value staging rows
  float4* cm = reinterpret_cast<float4*>(ks);
  const int n4 = ns * GS * kPartRow / 4;
#pragma unroll 1
  for (int q0 = tid; q0 < n4; q0 += 4 * kAT) {
    float4 t4[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (q0 + u * kAT < n4) t4[u] = __ldcg(base + q0 + u * kAT);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (q0 + u * kAT < n4) cm[q0 + u * kAT] = t4[u];
  }
  abar();
  const float* cf = reinterpret_cast<const float*>(cm);
#pragma unroll 1
  for (int idx = tid; idx < GS * kHD; idx += kAT) {
    const int hh = idx / kHD, d = idx % kHD;
    float M = -INFINITY;
    for (int jj = 0; jj < ns; ++jj) M = fmaxf(M, cf[(jj * GS + hh) * kPartRow + 64]);
    float num = 0.0f, den = 0.0f;
    for (int jj = 0; jj < ns; ++jj) {
      const float* pj = cf + (jj * GS + hh) * kPartRow;
      const float lj = pj[65];
      const float w = lj > 0.0f ? expf(pj[64] - M) : 0.0f;
      num = fmaf(pj[d], w, num);
      den = fmaf(lj, w, den);
    }
    P.att[int64_t(b) * P.q_n + (kvh * GS + hh) * kHD + d] = Lp > 0 ? uint16_t(bfr(num / den)) : uint16_t(0);
  }
  abar();
  if (tid == 0) {
    *ticket = 0u;
    __threadfence();
    atomicAdd(P.ctr + l * C_LAYER + C_ATTN, 1u);
  }
  stamp(P, l, C_ATTN, 6);
  return true;
}

// Tensor parallelism, one CTA: h_out = the residual rows after the last update (layer L-1's down_proj
// outputs of all ranks added), once every rank's partials have arrived.
__device__ __noinline__ bool tp_finalize() {
  const DkHot& P = dk_P;
  Smem& S = dk_S;
  const i4b_decode_model& m = P.m;
  const int tid = threadIdx.x, L = m.layers, H = m.hidden;
  const unsigned int* abort_word = P.ctr + P.i_abort;
  if (tid == 0) {
    if (!wait_counter(P.ctr + (L - 1) * C_LAYER + C_DOWN, unsigned(P.nslab[G_DOWN]), abort_word)) S.flag = 0;
  }
  cbar();
  if (!S.flag) return false;
  uint16_t* out = static_cast<uint16_t*>(m.h_out);
  const int nch = H / 8;
  bool ok = true;
#pragma unroll 1
  for (int idx = tid; idx < m.batch * nch; idx += kCT) {
    const int t = idx / nch, ch = idx - t * nch;
    *reinterpret_cast<uint4*>(out + int64_t(t) * H + 8 * ch) = residual_chunk(P, 2 * L - 1, t, ch, S.ep, abort_word, &ok);
  }
  if (!ok) S.flag = 0;
  cbar();
  return S.flag != 0;
}

template <int SPS, int GS, bool TP>
__global__ void __launch_bounds__(kThreads, 1) decode_layers_kernel(const __grid_constant__ DkParams Pg) {
  uint8_t* const smem = dk_smem;
  Smem& S = dk_S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  static_assert(sizeof(DkHot) % 4 == 0, "word copy");
  for (int i = tid; i < int(sizeof(DkHot) / 4); i += kThreads)
    reinterpret_cast<uint32_t*>(&dk_P)[i] = reinterpret_cast<const uint32_t*>(&Pg.h)[i];
  __syncthreads();
  const DkHot& P = dk_P;
  const i4b_decode_model& m = P.m;
  const unsigned int* abort_word = P.ctr + P.i_abort;
  if (tid == 0) {
    const int cta = blockIdx.x;
    const int nit = Pg.nitems[cta];
    int off = 0;
    for (int i = 0; i < nit; ++i) {
      const uint16_t it = Pg.items[cta][i];
      S.stage[i] = uint8_t(it >> 14);
      S.slab[i] = uint16_t(it & 0x3FFFu);
      S.poff[i] = uint16_t(off);
      off += P.npiece[it >> 14];
    }
    S.nit = nit;
    S.ppl = off;
    S.flag = 1;
    S.ep = TP ? *reinterpret_cast<volatile unsigned int*>(P.xb[P.tp_rank]) : 0u;
    S.prod_seq = 0;
    for (int s = 0; s < P.nslot; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  bool ok = true;
  if (warp == kCW) {
    // ---- producer: stream this CTA's pieces, layer after layer, into the ring
    if (lane == 0) {
      uint64_t policy;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
      const uint32_t ring = smem_u32(smem);
      const uint8_t* wsrc[4] = {static_cast<const uint8_t*>(m.w_qkv), static_cast<const uint8_t*>(m.w_o),
                                static_cast<const uint8_t*>(m.w_gu), static_cast<const uint8_t*>(m.w_down)};
      int seq = 0;
      for (int l = 0; l < m.layers && ok; ++l) {
        for (int i = 0; i < S.nit && ok; ++i) {
          const int g = S.stage[i], ppi = P.npiece[g];
          const uint8_t* src = wsrc[g] + int64_t(l) * P.layer_bytes[g] + int64_t(S.slab[i]) * ppi * P.piece_bytes;
          for (int p = 0; p < ppi; ++p, ++seq) {
            const int slot = seq % P.nslot;
            if (seq >= P.nslot && !wait_slot(&S.empty[slot], uint32_t(seq / P.nslot - 1) & 1u, abort_word)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&S.full[slot], uint32_t(P.piece_bytes));
            bulk_g2s(ring + slot * P.piece_bytes, src + int64_t(p) * P.piece_bytes, uint32_t(P.piece_bytes),
                     &S.full[slot], policy);
            S.prod_seq = seq + 1;
          }
        }
      }
      // every copy issued has landed before the CTA may exit (normally all were consumed already)
      for (int s = max(0, seq - P.nslot); s < seq; ++s)
        if (!mbar_wait(&S.full[s % P.nslot], uint32_t(s / P.nslot) & 1u)) ok = false;
      if (!ok) {
        atomicOr(&g_dk_err, I4B_DEVERR_WAIT_TIMEOUT);
        atomicExch(P.ctr + P.i_abort, 1u);
      }
    }
  } else {
    // ---- compute warps: the stages of every layer in order
    const int nattn = m.batch * m.kv_heads * P.nsplit;
    for (int l = 0; l < m.layers && ok; ++l) {
      ok = gemv_stage<SPS, TP>(G_QKV, l);
      // attention runs on warps 0..kAW-1; the others go on to the o_proj stage, whose barrier they pass
      // only together with them.  A failed attention clears S.flag, which that stage checks.
      if (ok && int(blockIdx.x) < nattn && warp < kAW) attention_item<GS>(l, blockIdx.x);
      ok = ok && gemv_stage<SPS, TP>(G_O, l);
      ok = ok && gemv_stage<SPS, TP>(G_GU, l);
      ok = ok && gemv_stage<SPS, TP>(G_DOWN, l);
    }
    if (TP && ok && blockIdx.x == 0) ok = tp_finalize();
    if (!ok && tid == 0) {
      atomicOr(&g_dk_err, I4B_DEVERR_WAIT_TIMEOUT);
      atomicExch(P.ctr + P.i_abort, 1u);
    }
  }
  __syncthreads();
  if (tid == 0) {
    // token ids outside the vocabulary were read as row 0: reported, not silently used
    if (blockIdx.x == 0)
      for (int b = 0; b < m.batch; ++b)
        if (m.tokens[b] < 0 || m.tokens[b] >= m.vocab) atomicOr(&g_dk_err, 2u);
    __threadfence();
    if (atomicAdd(P.ctr + P.i_done, 1u) == gridDim.x - 1) {  // the last CTA out resets the workspace counters
      for (int i = 0; i < P.n_ctr; ++i) P.ctr[i] = 0u;
      // and, under tensor parallelism, advances this rank's epoch for the next launch
      if (TP) *reinterpret_cast<volatile unsigned int*>(P.xb[P.tp_rank]) = S.ep + 1u;
      __threadfence();
    }
  }
}

// Re-lay a quantize_int4 tensor triple into pieces: for slab s (columns 16s..16s+15) and piece p (k in
// [512p, 512p + 512)), 16 steps x 32 lanes x 2 words -- lane (r, c) of step j holds qweight row
// 64p + 4j + c at columns 16s + r and 16s + r + 8 -- then, per group of the piece, 8 records of 16 bytes:
// record r holds the dequantization constants (dq_params) of columns 16s + r (low halves) and 16s + r + 8
// (high halves) as bf16 pairs: 128 + zero, the scale's high part, the scale's remainder, and 4 zero bytes.
// One thread per 16-byte unit.
__global__ void tile_w4_kernel(const int32_t* __restrict__ qw, int64_t sqk, const uint16_t* __restrict__ sc,
                               const uint16_t* __restrict__ zr, int64_t ssg, int64_t N, int64_t K, int G,
                               uint8_t* __restrict__ out, int piece_bytes) {
  const int units_per_piece = piece_bytes / 16;
  const int64_t pk = K / kPieceK;
  const int64_t total = (N / kSlabW) * pk * units_per_piece;
  for (int64_t u = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; u < total; u += int64_t(gridDim.x) * blockDim.x) {
    const int64_t piece = u / units_per_piece;
    const int w = int(u - piece * units_per_piece);
    const int64_t s = piece / pk, p = piece - s * pk;
    uint4 v;
    if (w < kPieceW / 16) {  // lanes 2h and 2h + 1 of step j
      const int j = w / 16, h = w % 16;
      uint32_t t[4];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int lane = 2 * h + e, r = lane >> 2, c = lane & 3;
        const int32_t* src = qw + (64 * p + 4 * j + c) * sqk + kSlabW * s + r;
        t[2 * e] = uint32_t(src[0]);
        t[2 * e + 1] = uint32_t(src[8]);
      }
      v = make_uint4(t[0], t[1], t[2], t[3]);
    } else {
      const int rec = w - kPieceW / 16, gi = rec / 8, r = rec % 8;
      const int64_t g = p * (kPieceK / G) + gi;
      const uint16_t* s2 = sc + g * ssg + kSlabW * s + r;
      const uint16_t* z2 = zr + g * ssg + kSlabW * s + r;
      const DqParams a = dq_params<false>(s2[0], z2[0]), b = dq_params<false>(s2[8], z2[8]);
      v = make_uint4((a.zz & 0xFFFFu) | (b.zz << 16), (a.shi & 0xFFFFu) | (b.shi << 16),
                     (a.slo & 0xFFFFu) | (b.slo << 16), 0u);
    }
    reinterpret_cast<uint4*>(out)[u] = v;
  }
}

// ------------------------------------------------------------------ host side

int piece_bytes_for(int G) { return kPieceW + (kPieceK / G) * kRecB; }

struct Sched {
  int max_part = 0;
  int max_res = 0;  // most o_proj or down_proj slabs of one CTA
  bool ok = false;
  std::vector<uint8_t> nitems;
  std::vector<uint16_t> items;  // [grid][kMaxItems]
};

// Assignment of one layer's slabs to the CTAs, stage by stage: each stage is its own critical path, so
// each slab goes to the CTA with the fewest pieces of that stage so far, ties to the fewest pieces over
// all stages, then to the lowest index.  Each CTA's list is in stage order; the same lists serve every
// layer.
Sched build_sched(int grid, const int nslab[4], const int npiece[4]) {
  Sched sc;
  sc.nitems.assign(grid, 0);
  sc.items.assign(size_t(grid) * kMaxItems, 0);
  std::vector<int64_t> load(grid, 0);
  std::vector<std::vector<std::pair<int, int>>> lists(grid);
  for (int g = 0; g < 4; ++g) {
    std::vector<int> st(grid, 0);
    for (int s = 0; s < nslab[g]; ++s) {
      int best = 0;
      for (int c = 1; c < grid; ++c)
        if (st[c] < st[best] || (st[c] == st[best] && load[c] < load[best])) best = c;
      st[best] += npiece[g];
      load[best] += npiece[g];
      lists[best].emplace_back(g, s);
    }
  }
  for (int c = 0; c < grid; ++c) {
    auto& L = lists[c];
    if (L.size() > size_t(kMaxItems)) return sc;
    std::sort(L.begin(), L.end());
    sc.nitems[c] = uint8_t(L.size());
    int cnt[4] = {0, 0, 0, 0};
    for (size_t i = 0; i < L.size(); ++i) {
      sc.items[size_t(c) * kMaxItems + i] = uint16_t((L[i].first << 14) | L[i].second);
      ++cnt[L[i].first];
    }
    for (int g = 0; g < 4; ++g) sc.max_part = std::max(sc.max_part, cnt[g] * std::min(npiece[g], kCW));
    sc.max_res = std::max(sc.max_res, std::max(cnt[G_O], cnt[G_DOWN]));
  }
  sc.ok = true;
  return sc;
}

struct Layout {
  int nslab[4], npiece[4];
  int64_t layer_bytes[4];
  int piece_bytes, gqa, nsplit, qkv_n, q_n;
  int n_ctr, i_ticket, i_done, i_abort;
  size_t off_apart, off_qkv, off_att, off_act, off_hbuf, total;
};

int make_layout(const i4b_decode_model& m, int grid, Layout* L) {
  if (m.layers <= 0 || m.hidden <= 0 || m.heads <= 0 || m.kv_heads <= 0 || m.intermediate <= 0 || m.vocab <= 0 ||
      m.max_seq <= 0)
    return I4B_ERR_SHAPE;
  if (m.head_dim != kHD) return I4B_ERR_SHAPE;
  if (m.batch < 1 || m.batch > kMaxTok || m.cache_batch < m.batch) return I4B_ERR_SHAPE;
  if (m.group_size != 32 && m.group_size != 64 && m.group_size != 128) return I4B_ERR_GROUP;
  if (m.heads % m.kv_heads != 0) return I4B_ERR_SHAPE;
  const int gqa = m.heads / m.kv_heads;
  if (gqa != 1 && gqa != 2 && gqa != 4 && gqa != 8) return I4B_ERR_SHAPE;
  const int q_n = m.heads * kHD, qkv_n = (m.heads + 2 * m.kv_heads) * kHD;
  // every projection input width is a power-of-two number of 8-value chunks, at least one 512-k piece
  auto pow2_chunks = [](int k) { return k >= kPieceK && k % 8 == 0 && ((k / 8) & (k / 8 - 1)) == 0; };
  if (!pow2_chunks(m.hidden) || !pow2_chunks(m.intermediate) || !pow2_chunks(q_n)) return I4B_ERR_SHAPE;
  L->gqa = gqa;
  L->q_n = q_n;
  L->qkv_n = qkv_n;
  L->piece_bytes = piece_bytes_for(m.group_size);
  const int64_t N[4] = {qkv_n, m.hidden, 2 * int64_t(m.intermediate), m.hidden};
  const int64_t K[4] = {m.hidden, q_n, m.hidden, m.intermediate};
  for (int g = 0; g < 4; ++g) {
    if (N[g] / kSlabW >= (1 << 14)) return I4B_ERR_SHAPE;
    L->nslab[g] = int(N[g] / kSlabW);
    L->npiece[g] = int(K[g] / kPieceK);
    L->layer_bytes[g] = int64_t(L->nslab[g]) * L->npiece[g] * L->piece_bytes;
  }
  const int items = m.batch * m.kv_heads;
  L->nsplit = std::max(1, std::min(16, grid / items));
  if (items > grid) return I4B_ERR_SHAPE;
  // the counter region (zero between calls) has the same size for every batch, so one workspace serves all
  L->i_ticket = m.layers * C_LAYER;
  L->i_done = L->i_ticket + kMaxTok * m.kv_heads;
  L->i_abort = L->i_done + 1;
  L->n_ctr = L->i_abort + 1;
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  size_t off = al(size_t(L->n_ctr) * 4);
  L->off_apart = off;
  off = al(off + size_t(items) * L->nsplit * gqa * kPartRow * 4);
  L->off_qkv = off;
  off = al(off + size_t(m.batch) * qkv_n * 2);
  L->off_att = off;
  off = al(off + size_t(m.batch) * q_n * 2);
  L->off_act = off;
  off = al(off + size_t(m.batch) * m.intermediate * 2);
  L->off_hbuf = off;  // tensor parallelism: the residual rows of two consecutive updates
  off = al(off + size_t(2) * kMaxTok * m.hidden * 2);
  L->total = off;
  return I4B_OK;
}

template <int SPS, int GS>
cudaError_t launch_dk_t(const DkParams& p, int grid, size_t smem, cudaStream_t stream) {
  // the one-rank kernel is compiled without the tensor-parallel exchange
  auto kern = p.h.tp_world > 1 ? decode_layers_kernel<SPS, GS, true> : decode_layers_kernel<SPS, GS, false>;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int SPS>
cudaError_t launch_dk_s(const DkParams& p, int grid, size_t smem, cudaStream_t stream) {
  switch (p.h.gqa) {
    case 1: return launch_dk_t<SPS, 1>(p, grid, smem, stream);
    case 2: return launch_dk_t<SPS, 2>(p, grid, smem, stream);
    case 4: return launch_dk_t<SPS, 4>(p, grid, smem, stream);
    default: return launch_dk_t<SPS, 8>(p, grid, smem, stream);
  }
}

}  // namespace

int64_t decode_peer_capacity(int layers, int world, int hidden) {
  // tagged partials (8 bytes each) [layers][2][world][kMaxTok][hidden] in the 2 x kArMaxRanks x capacity data
  // area of 8-byte words
  const int64_t words = int64_t(layers) * 2 * world * kMaxTok * hidden;
  return (words + 2 * kArMaxRanks - 1) / (2 * kArMaxRanks);
}

size_t tile_w4_bytes(int64_t N, int64_t K, int G) {
  if (N <= 0 || K <= 0 || N % kSlabW || K % kPieceK || (G != 32 && G != 64 && G != 128)) return 0;
  return size_t(N / kSlabW) * size_t(K / kPieceK) * size_t(piece_bytes_for(G));
}

cudaError_t launch_tile_w4(const int32_t* qw, int64_t sqk, const uint16_t* sc, const uint16_t* zr, int64_t ssg,
                           int64_t N, int64_t K, int G, void* out, cudaStream_t stream) {
  const int64_t units = int64_t(tile_w4_bytes(N, K, G) / 16);
  const int blocks = int(std::min<int64_t>((units + 255) / 256, 148 * 16));
  tile_w4_kernel<<<blocks, 256, 0, stream>>>(qw, sqk, sc, zr, ssg, N, K, G, static_cast<uint8_t*>(out),
                                             piece_bytes_for(G));
  return cudaGetLastError();
}

int decode_layers_workspace(const i4b_decode_model& m, int num_sms, size_t* bytes) {
  Layout L;
  if (int st = make_layout(m, std::min(num_sms, kMaxCtas), &L)) return st;
  *bytes = L.total;
  return I4B_OK;
}

static unsigned long long* g_dk_trace = nullptr;
static size_t g_dk_trace_bytes = 0;

void set_decode_trace(void* buf, size_t bytes) {
  g_dk_trace = static_cast<unsigned long long*>(buf);
  g_dk_trace_bytes = bytes;
}

int launch_decode_layers(const i4b_decode_model& m, int num_sms, int smem_optin, void* ws, size_t ws_bytes,
                         cudaStream_t stream, cudaError_t* err) {
  *err = cudaSuccess;
  const int grid = std::min(num_sms, kMaxCtas);
  Layout L;
  if (int st = make_layout(m, grid, &L)) return st;
  if (ws_bytes < L.total) return I4B_ERR_WORKSPACE;
  // the schedule depends on the grid and the projection shapes only: built once per shape
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int, int, int, int>, Sched> cache;
  const Sched* sc;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_tuple(grid, L.nslab[0], L.nslab[1], L.nslab[2], L.nslab[3], L.npiece[0], L.npiece[1],
                               L.npiece[2], L.npiece[3]);
    auto it = cache.find(key);
    if (it == cache.end()) it = cache.emplace(key, build_sched(grid, L.nslab, L.npiece)).first;
    sc = &it->second;
  }
  if (!sc->ok) return I4B_ERR_SHAPE;
  if (sc->max_res * m.batch * kSlabW > kCT * kResPerThread) return I4B_ERR_SHAPE;

  DkParams p;
  memset(&p, 0, sizeof(p));
  p.h.m = m;
  for (int g = 0; g < 4; ++g) {
    p.h.nslab[g] = L.nslab[g];
    p.h.npiece[g] = L.npiece[g];
    p.h.layer_bytes[g] = L.layer_bytes[g];
  }
  p.h.piece_bytes = L.piece_bytes;
  p.h.nsplit = L.nsplit;
  p.h.gqa = L.gqa;
  p.h.qkv_n = L.qkv_n;
  p.h.q_n = L.q_n;
  uint8_t* w = static_cast<uint8_t*>(ws);
  p.h.ctr = reinterpret_cast<unsigned int*>(w);
  p.h.n_ctr = L.n_ctr;
  p.h.i_ticket = L.i_ticket;
  p.h.i_done = L.i_done;
  p.h.i_abort = L.i_abort;
  p.h.apart = reinterpret_cast<float*>(w + L.off_apart);
  p.h.qkv = reinterpret_cast<uint16_t*>(w + L.off_qkv);
  p.h.att = reinterpret_cast<uint16_t*>(w + L.off_att);
  p.h.act = reinterpret_cast<uint16_t*>(w + L.off_act);
  p.h.tp_world = 1;
  if (m.peers && m.peers->world > 1) {
    const i4b_peer_group& pg = *m.peers;
    if (pg.world > kArMaxRanks || pg.rank < 0 || pg.rank >= pg.world) return I4B_ERR_INVALID_ARG;
    if (pg.capacity < decode_peer_capacity(m.layers, pg.world, m.hidden)) return I4B_ERR_SHAPE;
    for (int q = 0; q < pg.world; ++q) {
      if (!pg.buffers[q] || reinterpret_cast<uintptr_t>(pg.buffers[q]) % 256 != 0) return I4B_ERR_INVALID_ARG;
      p.h.xb[q] = static_cast<uint8_t*>(pg.buffers[q]);
    }
    p.h.tp_world = pg.world;
    p.h.tp_rank = pg.rank;
    p.h.hbuf[0] = reinterpret_cast<uint16_t*>(w + L.off_hbuf);
    p.h.hbuf[1] = p.h.hbuf[0] + size_t(kMaxTok) * m.hidden;
    // the residual rows of an update are stored by a CTA that runs the stage consuming them
    for (int g = 0; g < 4; ++g) {
      p.h.writer[g] = -1;
      for (int c = 0; c < grid && p.h.writer[g] < 0; ++c)
        for (int i = 0; i < sc->nitems[c]; ++i)
          if ((sc->items[size_t(c) * kMaxItems + i] >> 14) == g) {
            p.h.writer[g] = c;
            break;
          }
    }
    if (p.h.writer[G_QKV] < 0 || p.h.writer[G_GU] < 0) return I4B_ERR_SHAPE;
  }
  if (g_dk_trace && g_dk_trace_bytes >= size_t(grid) * m.layers * 5 * kTraceSlots * 8) p.h.trace = g_dk_trace;
  for (int c = 0; c < grid; ++c) {
    p.nitems[c] = sc->nitems[c];
    for (int i = 0; i < kMaxItems; ++i) p.items[c][i] = sc->items[size_t(c) * kMaxItems + i];
  }
  // dynamic shared memory: ring | activations | group sums | partials; the attention scratch reuses the
  // activation region
  const int kmax = std::max(std::max(m.hidden, m.intermediate), L.q_n);
  p.h.xpitch = 2 * kmax + 16;
  auto al = [](int v) { return (v + 127) & ~127; };
  // attention: queries, keys, values, probabilities, running max / sum / rescale, the new key and value; then
  // the partials of all splits when combining
  const int attn_block = (2 * L.gqa * kHD + 3 * L.gqa) * 4 + 64 * 33 * 4 + 64 * kHD * 2 + 2 * kHD * 2;
  const int attn_bytes = std::max(attn_block, L.gqa * kHD * 4 + L.nsplit * L.gqa * kPartRow * 4);
  const int x_bytes = al(std::max(m.batch * p.h.xpitch, attn_bytes));
  const int xs_bytes = 0;
  const int part_bytes = al(sc->max_part * m.batch * kSlabW * 4);
  const int fixed = x_bytes + xs_bytes + part_bytes;
  const int avail = smem_optin - int(sizeof(Smem)) - 1024;
  const int nslot = std::min(kMaxSlots, (avail - fixed) / p.h.piece_bytes);
  if (nslot < 2) return I4B_ERR_SHAPE;
  p.h.nslot = nslot;
  p.h.off_x = nslot * p.h.piece_bytes;
  p.h.off_xs = p.h.off_x + x_bytes;
  p.h.off_part = p.h.off_xs + xs_bytes;
  const size_t smem = size_t(p.h.off_part + part_bytes);
  cudaError_t e;
  switch (m.group_size) {
    case 32: e = launch_dk_s<1>(p, grid, smem, stream); break;
    case 64: e = launch_dk_s<2>(p, grid, smem, stream); break;
    default: e = launch_dk_s<4>(p, grid, smem, stream); break;
  }
  if (e != cudaSuccess) {
    *err = e;
    return I4B_ERR_CUDA;
  }
  return I4B_OK;
}

unsigned int read_dk_error(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_dk_err, sizeof(v));
  if (clear && v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_dk_err, &z, sizeof(z));
  }
  return v;
}

}  // namespace i4b
