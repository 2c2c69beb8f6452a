// Small-M (M <= 32) W4A16 kernel: the M == 1 decode GEMV and the small-batch split-K path.
//
// Replaces the reference's _gemv_kernel (int4_triton/gemm.py:185-220) and its
// small-M split-K pair _matmul_kernel + _reduce_split_k (gemm.py:74-182,
// launched at gemm.py:265-299) with ONE launch per matmul.
//
// Work split.  grid = (ceil(N / 128), S), cluster (1, S, 1) when 1 < S <= 8.
// A CTA owns 128 output columns and the K range [y*KC, (y+1)*KC), KC <= 1024;
// warp w owns columns 32w..32w+31.  Every lane puts ALL of the packed words it
// will use in flight at once (cp.async, 16 bytes per 32-k step, one commit
// group per stage of 4 steps) into its own slots of shared memory, so no
// barrier orders copy and use: cp.async.wait_group does.  These copies do not
// depend on the previous kernel of the stream, so with programmatic dependent
// launch they are issued before griddepcontrol.wait and overlap that kernel's
// tail; only the activations, staged once per CTA in shared memory, wait for it.
//
// Dequant and MMA.  Per 32-k step, lane (r = lane/4, c = lane%4) holds the 4
// words of columns 4r..4r+3 at k8 row 4*step + c.  One lop3 turns a nibble
// pair into the bf16 (fp16) pair (bias + q_i, bias + q_{i+4}), bias = 128
// (1024), exactly; dq_pair then forms w = (q - z) * s rounded once to the
// activation type -- the reference's own weight, int4_triton/gemm.py:211 --
// with a subtract and a split-scale multiply-add.  These pairs ARE the A
// fragments of mma.m16n8k16 (rows = output columns); the activations, stored
// pre-permuted to the same k order, are the B fragments; fp32 accumulators
// (two chains, one per k16 half of a step).  y = sum_k x_k * bf16(w_k) as in the
// reference, up to fp32 summation order.

// Reduction.  K splits inside a cluster add through distributed shared memory
// in fixed rank order.  More than 8 splits (K > 8192) write fp32 partials to
// the caller's workspace; the last CTA of a column tile (atomic ticket, no
// spinning) adds them in split order and resets the ticket.  Every path is
// bit-identical from run to run.  The only waits are those of the tensor-parallel
// epilogue (i4b_w4a16_matmul_allreduce), for the other ranks' flags, each bounded.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace i4b {

namespace {

constexpr int kBN = 128;      // output columns per CTA (4 warps x 32)
constexpr int kMaxKCAll = 1024;  // k per CTA, at most
constexpr int kStageSteps = 4;

struct W4SArgs {
  const uint16_t* x;
  int64_t sxm, sxk;
  const uint32_t* qw;
  int64_t sqk;  // words between k8 rows
  const uint16_t* sc;
  const uint16_t* zr;
  int64_t ssg;  // elements between group rows of scales / zeros
  uint16_t* y;
  int64_t sym;
  float* partials;
  unsigned int* tickets;
  int M, N, K, G;
  int S, KC, mode;
  int nstages;     // stages per CTA (the last one padded with zeros)
  int gpl_shift;   // log2(segments per group), or -1 when that count is not a power of two
  int gpl;         // segments per group
  int vec_w, vec_s, vec_x, pdl;
  int xpitch;
  int off_sz, off_x, off_part;
  int pro;
  // activation prologue (bf16 only): 1 = x := rmsnorm(x + delta) * norm_w, 2 = x := silu(g) * u with g | u = x
  const uint16_t* delta;
  const uint16_t* norm_w;
  uint16_t* resid_out;
  float eps;
  // fused tensor-parallel all-reduce of y (ar_world > 1): every rank's exchange buffer, mapped here
  uint8_t* ar_buf[kArMaxRanks];
  int64_t ar_cap;
  int ar_world, ar_rank;
  // w4_gemv_kernel: WN x WK warps per CTA (columns x K), KW k per warp, scale / zero rows staged per CTA
  int WN, WK, KW;
  int sz_rows;
  // fused greedy choice (w4_gemv_kernel with ARG): candidates [tiles][M] of (value, column), out [M]
  float2* cand;
  int64_t* amax_out;
};

enum { kProPlain = 0, kProRmsNorm = 1, kProSwiGlu = 2 };

__device__ unsigned int g_w4_err = 0;

// ---- fused all-reduce over peer exchange buffers (layout in kernels.h).  The helpers take any argument
// struct with the fields ar_buf, ar_cap, ar_world and ar_rank.
//
// Each exchanged fp32 value travels with its tag -- the call's epoch + 1 -- in ONE 64-bit store (value in the
// low word, tag in the high word), and the reader polls the words it needs until their tags match: the data
// is its own flag, so no memory fence and no per-CTA flag sit between the ranks.  Two slots (epoch & 1)
// alternate: a rank starts call e + 2, which rewrites call e's slot, only after every rank's data of call
// e + 1 reached it, i.e. after every rank finished call e.

// tagged outputs of source rank `src` in rank p's buffer
template <class A>
__device__ __forceinline__ uint64_t* ar_data(const A& a, int p, uint32_t slot, int src) {
  return reinterpret_cast<uint64_t*>(a.ar_buf[p] + kArDataOff) + (int64_t(slot) * kArMaxRanks + src) * a.ar_cap;
}
// The call's epoch, read once per CTA (after the previous kernel of the stream has completed).
template <class A>
__device__ __forceinline__ uint32_t ar_epoch(const A& a, uint32_t* s_ep) {
  if (threadIdx.x == 0) *s_ep = *reinterpret_cast<volatile unsigned int*>(a.ar_buf[a.ar_rank]);
  __syncthreads();
  return *s_ep;
}
// Push one output (offset tok * N + n) with the call's tag to every rank's buffer, slot of this epoch, region
// of this rank.
template <class A>
__device__ __forceinline__ void ar_push(const A& a, uint32_t ep, int64_t off, float v) {
  const uint64_t word = (uint64_t(ep + 1u) << 32) | __float_as_uint(v);
  for (int p = 0; p < a.ar_world; ++p)
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(ar_data(a, p, ep & 1u, a.ar_rank) + off), "l"(word)
                 : "memory");
}
// One output of source rank q once it carries the call's tag.  Bounded: a wait that gives up sets
// I4B_DEVERR_PEER_TIMEOUT and yields 0; once that bit is set, later waits on this device return at once.
template <class A>
__device__ __forceinline__ float ar_take(const A& a, uint32_t ep, int q, int64_t off) {
  const uint64_t* w = ar_data(a, a.ar_rank, ep & 1u, q) + off;
  uint64_t v;
  uint64_t t0 = 0;
  for (uint32_t it = 1;; ++it) {
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(w) : "memory");
    if (uint32_t(v >> 32) == ep + 1u) return __uint_as_float(uint32_t(v));
    if (it == 1) t0 = globaltimer_ns();
    if ((it & 63u) == 0) {
      if (*reinterpret_cast<volatile unsigned int*>(&g_w4_err) & I4B_DEVERR_PEER_TIMEOUT) return 0.0f;
      if (globaltimer_ns() - t0 > I4B_WAIT_LIMIT_NS) {
        atomicOr(&g_w4_err, I4B_DEVERR_PEER_TIMEOUT);
        return 0.0f;
      }
    }
  }
}
// Sum over source ranks, in rank order, of one output in this rank's buffer (a value that has already arrived
// costs one load).
template <class A>
__device__ __forceinline__ float ar_sum(const A& a, uint32_t ep, int64_t off) {
  float v = 0.0f;
  for (int q = 0; q < a.ar_world; ++q) {
    const float t = ar_take(a, ep, q, off);
    v = q == 0 ? t : v + t;
  }
  return v;
}
// The last CTA of the call advances this rank's epoch (read by the next call on the group).
template <class A>
__device__ __forceinline__ void ar_finish(const A& a, uint32_t ep) {
  if (threadIdx.x == 0) {
    unsigned int* ctl = reinterpret_cast<unsigned int*>(a.ar_buf[a.ar_rank]);
    const unsigned int prev = atomicAdd(ctl + 1, 1u);
    if (prev == gridDim.x * gridDim.y - 1) {
      atomicExch(ctl + 1, 0u);
      __threadfence();
      atomicExch(ctl, ep + 1);
    }
  }
}

// The dequantization constants of columns 4r .. 4r + 3 from their 16-byte scale / zero record
// (s0 s1 | s2 s3 | z0 z1 | z2 z3): lane c (of the four lanes with the same r) converts column 4r + c only and
// the four lanes exchange the results by shuffle, instead of each lane converting all four.
template <bool F16>
__device__ __forceinline__ void dq_params_shared(const uint4& sz, int c, DqParams (&dp)[4]) {
  const uint32_t sw = c < 2 ? sz.x : sz.y, zw = c < 2 ? sz.z : sz.w;
  const int sh = (c & 1) * 16;
  const DqParams mine = dq_params<F16>(uint16_t(sw >> sh), uint16_t(zw >> sh));
  const int base = (threadIdx.x & 31) & ~3;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    dp[j].zz = __shfl_sync(0xFFFFFFFFu, mine.zz, base + j);
    dp[j].shi = __shfl_sync(0xFFFFFFFFu, mine.shi, base + j);
    if constexpr (!F16) dp[j].slo = __shfl_sync(0xFFFFFFFFu, mine.slo, base + j);
    else dp[j].slo = 0u;
  }
}

// First maximum among (value, column) candidates in increasing column order: a strictly greater value wins, an
// equal one only at a lower column (NaN never compares greater, as in block_row_argmax).
__device__ __forceinline__ void first_max(float& best, int64_t& bi, float v, int64_t i) {
  if (v > best || (v == best && i < bi)) {
    best = v;
    bi = i;
  }
}

__device__ __forceinline__ float bfv(uint32_t bits16) { return __uint_as_float(bits16 << 16); }
__device__ __forceinline__ uint32_t bfr(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }

__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int i, uint32_t magic) {
  return and_or(w >> (4 * i), 0x000F000Fu, magic);
}

template <bool F16>
__device__ __forceinline__ uint16_t f2h_bits(float v) {
  if constexpr (F16) return __half_as_ushort(__float2half_rn(v));
  else return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// Shared-memory accesses by 32-bit address; volatile keeps them ordered after cp.async.wait_group.
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
// Packed weights are read once per call: 128-bit loads that do not allocate in L1.
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp8(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp4(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}

// cp.async.wait_group with a run-time count (0..7).
__device__ __forceinline__ void cp_async_wait_upto(int pending) {
  switch (pending) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    case 4: cp_async_wait<4>(); break;
    case 5: cp_async_wait<5>(); break;
    case 6: cp_async_wait<6>(); break;
    default: cp_async_wait<7>(); break;
  }
}

}  // namespace

// Stages the activations of token rows 0..M-1, k in [k0, k0 + 8*nreal), in shared memory at s_x (row pitch
// a.xpitch), each 8-k chunk permuted to the k order of the A fragments; chunks nreal..nch-1 are zero (padding).
// With a prologue the activations are derived from the previous step's tensors (RMSNorm of x + delta, with
// the full-row statistics computed here; or SwiGLU of a gate | up row).  s_inv: shared [32] floats.  All
// threads of the CTA take part; the caller synchronises before reading.
template <bool F16, int PRO>
__device__ __forceinline__ void stage_activations(const W4SArgs& a, uint32_t s_x, int k0, int nch, int nreal,
                                                  float* s_inv) {
  constexpr int XB = 4;  // chunks per thread in flight
  const int M = a.M;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthr = blockDim.x, nwarps = nthr >> 5;
  const int total = M * nch;
  if constexpr (PRO == kProRmsNorm) {
    // Full-row statistics of h' = bf16(h + delta) for every token (warp t % warps owns token t); CTA (0, 0)
    // also writes h' to resid_out.  Rows are contiguous with K % 8 == 0 and 16-byte alignment.
    const bool writer = a.resid_out && blockIdx.x == 0 && blockIdx.y == 0;
    for (int t = warp; t < M; t += nwarps) {
      const uint16_t* hr = a.x + int64_t(t) * a.sxm;
      const uint16_t* dr = a.delta ? a.delta + int64_t(t) * a.sxm : nullptr;
      float ss = 0.0f;
      for (int c = lane * 8; c < a.K; c += 256) {
        uint4 hv = __ldg(reinterpret_cast<const uint4*>(hr + c));
        if (dr) {
          const uint4 dv = __ldg(reinterpret_cast<const uint4*>(dr + c));
          const uint32_t* ha = reinterpret_cast<const uint32_t*>(&hv);
          const uint32_t* da = reinterpret_cast<const uint32_t*>(&dv);
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o[i] = bfr(bfv(ha[i] & 0xFFFFu) + bfv(da[i] & 0xFFFFu)) |
                   (bfr(bfv(ha[i] >> 16) + bfv(da[i] >> 16)) << 16);
          hv = make_uint4(o[0], o[1], o[2], o[3]);
        }
        if (writer) *reinterpret_cast<uint4*>(a.resid_out + int64_t(t) * a.sxm + c) = hv;
        const uint32_t* ha = reinterpret_cast<const uint32_t*>(&hv);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float lo = bfv(ha[i] & 0xFFFFu), hi = bfv(ha[i] >> 16);
          ss = fmaf(lo, lo, ss);
          ss = fmaf(hi, hi, ss);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
      if (lane == 0) s_inv[t] = rsqrtf(ss / float(a.K) + a.eps);
    }
    __syncthreads();
  }
  for (int base = 0; base < total; base += XB * nthr) {
    uint4 v[XB];
#pragma unroll
    for (int j = 0; j < XB; ++j) {
      const int idx = base + j * nthr + tid;
      const int t = idx / nch, ch = idx - t * nch;
      v[j] = make_uint4(0u, 0u, 0u, 0u);
      if (idx < total && ch < nreal) {
        const uint16_t* p = a.x + int64_t(t) * a.sxm + int64_t(k0 + 8 * ch) * a.sxk;
        if constexpr (PRO == kProRmsNorm) {
          // x = bf16(w * bf16(h' * inv)),  h' = bf16(h + delta)        (LlamaRMSNorm after the residual add)
          const uint4 hv = __ldg(reinterpret_cast<const uint4*>(p));
          const uint4 wv = __ldg(reinterpret_cast<const uint4*>(a.norm_w + k0 + 8 * ch));
          uint4 dv = make_uint4(0u, 0u, 0u, 0u);
          if (a.delta) dv = __ldg(reinterpret_cast<const uint4*>(a.delta + int64_t(t) * a.sxm + k0 + 8 * ch));
          const float inv = s_inv[t];
          const uint32_t* ha = reinterpret_cast<const uint32_t*>(&hv);
          const uint32_t* da = reinterpret_cast<const uint32_t*>(&dv);
          const uint32_t* wa = reinterpret_cast<const uint32_t*>(&wv);
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t lo = ha[i] & 0xFFFFu, hi = ha[i] >> 16;
            if (a.delta) {
              lo = bfr(bfv(lo) + bfv(da[i] & 0xFFFFu));
              hi = bfr(bfv(hi) + bfv(da[i] >> 16));
            }
            o[i] = bfr(bfv(wa[i] & 0xFFFFu) * bfv(bfr(bfv(lo) * inv))) |
                   (bfr(bfv(wa[i] >> 16) * bfv(bfr(bfv(hi) * inv))) << 16);
          }
          v[j] = make_uint4(o[0], o[1], o[2], o[3]);
        } else if constexpr (PRO == kProSwiGlu) {
          // x = bf16(bf16(silu(g)) * u),  g = row[k], u = row[K + k]                       (LlamaMLP)
          const uint4 gv = __ldg(reinterpret_cast<const uint4*>(p));
          const uint4 uv = __ldg(reinterpret_cast<const uint4*>(p + a.K));
          const uint32_t* ga = reinterpret_cast<const uint32_t*>(&gv);
          const uint32_t* ua = reinterpret_cast<const uint32_t*>(&uv);
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float g0 = bfv(ga[i] & 0xFFFFu), g1 = bfv(ga[i] >> 16);
            const float s0 = bfv(bfr(g0 / (1.0f + expf(-g0)))), s1 = bfv(bfr(g1 / (1.0f + expf(-g1))));
            o[i] = bfr(s0 * bfv(ua[i] & 0xFFFFu)) | (bfr(s1 * bfv(ua[i] >> 16)) << 16);
          }
          v[j] = make_uint4(o[0], o[1], o[2], o[3]);
        } else if (a.vec_x) {
          v[j] = __ldg(reinterpret_cast<const uint4*>(p));
        } else {
          uint16_t e[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) e[q] = __ldg(p + q * a.sxk);
          v[j] = make_uint4(uint32_t(e[0]) | (uint32_t(e[1]) << 16), uint32_t(e[2]) | (uint32_t(e[3]) << 16),
                            uint32_t(e[4]) | (uint32_t(e[5]) << 16), uint32_t(e[6]) | (uint32_t(e[7]) << 16));
        }
      }
    }
#pragma unroll
    for (int j = 0; j < XB; ++j) {
      const int idx = base + j * nthr + tid;
      if (base + j * nthr >= total) break;  // uniform over the CTA
      const int t = idx / nch, ch = idx - t * nch;
      const uint32_t u[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
      if (idx < total) {
        // (x0,x4) (x1,x5) (x2,x6) (x3,x7): the nibble-pair order of the A fragments
        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(s_x + t * a.xpitch + ch * 16),
                     "r"(__byte_perm(u[0], u[2], 0x5410)), "r"(__byte_perm(u[0], u[2], 0x7632)),
                     "r"(__byte_perm(u[1], u[3], 0x5410)), "r"(__byte_perm(u[1], u[3], 0x7632))
                     : "memory");
      }
    }
  }
}

// Shared memory: weights [step][warp][lane] x 16 B | scales+zeros [segment][warp][r] x 16 B (s0..s3, z0..z3) |
// activations [token][k/8] x 16 B (pre-permuted) | partial sums [token][128] fp32.  The K range of a CTA is
// padded to whole stages with zero weights, zero activations and zero scales, which add nothing.
template <int MT, bool F16, int SPS, int PRO>
__global__ void __launch_bounds__(128) w4_skinny_kernel(const W4SArgs a) {
  constexpr int SPST = SPS > 4 ? SPS : 4;  // 32-k steps per stage (one cp.async group); whole segments
  constexpr int SEGST = SPST / SPS;        // segments per stage
  constexpr int L = 32 * SPS;              // k per segment
  constexpr int WSTEP = 4 * 32 * 16;       // shared bytes of one step of weights (4 warps x 32 lanes x 16 B)
  constexpr int SZSEG = 4 * 8 * 16;        // shared bytes of one segment of scales + zeros
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = lane >> 2, c = lane & 3;
  const int64_t n0 = int64_t(blockIdx.x) * kBN;
  const int k0 = int(blockIdx.y) * a.KC;
  const int nsteps = a.KC / 32;
  const int nstages = a.nstages;
  const int M = a.M;

  const uint32_t s_w = smem_u32(smem);
  const uint32_t s_sz = s_w + a.off_sz;
  const uint32_t s_x = s_w + a.off_x;
  float* sP = reinterpret_cast<float*>(smem + a.off_part);

  // ---- weights, scales, zeros: independent of the previous kernel, all put in flight first
  const int64_t n_lane = n0 + warp * 32 + 4 * r;
  const bool n_in = n_lane < a.N;
  {
    const uint32_t* src = a.qw + int64_t(k0 / 8 + c) * a.sqk + (n_in ? n_lane : 0);
    const int64_t wstep = 4 * a.sqk;
    uint32_t dst = s_w + (warp * 32 + lane) * 16;
    const int nfull = nsteps / SPST;  // stages whose steps all lie inside K
    // Scales and zeros: the 16-byte record (s0 s1 | s2 s3 | z0 z1 | z2 z3) of a segment is copied 4 bytes
    // per lane c; a group row advances every gpl segments.
    const uint16_t* szsrc = (c < 2 ? a.sc : a.zr) + 2 * (c & 1);
    const int seg0 = k0 / L;
    int64_t g = a.gpl_shift >= 0 ? (seg0 >> a.gpl_shift) : seg0 / a.gpl;
    int gcnt = seg0 - int(g) * a.gpl;
    const bool sz_in = n_in && a.vec_s;
    uint32_t dst_sz = s_sz + (warp * 8 + r) * 16 + 4 * c;
    for (int st = 0; st < nstages; ++st) {
      if (st < nfull && a.vec_w) {
        const uint32_t bytes = n_in ? 16u : 0u;
#pragma unroll
        for (int i = 0; i < SPST; ++i) {
          cp16(dst + i * WSTEP, src, bytes);
          src += wstep;
        }
      } else {
#pragma unroll
        for (int i = 0; i < SPST; ++i) {
          const bool real = st * SPST + i < nsteps;
          if (a.vec_w) {
            cp16(dst + i * WSTEP, real ? src : a.qw, real && n_in ? 16u : 0u);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const bool in = real && n_lane + j < a.N;
              cp4(dst + i * WSTEP + 4 * j, in ? src + j : a.qw, in ? 4u : 0u);
            }
          }
          if (real) src += wstep;
        }
      }
#pragma unroll
      for (int j = 0; j < SEGST; ++j) {
        const bool real = (st * SEGST + j) * SPS < nsteps;
        const uint32_t d = dst_sz + j * SZSEG;
        if (a.vec_s || !real) {
          cp4(d, real && sz_in ? szsrc + g * a.ssg + n_lane : a.sc, real && sz_in ? 4u : 0u);
        } else {
          // unaligned scales / zeros: two plain loads per lane
          const bool in0 = n_lane + 2 * (c & 1) < a.N, in1 = n_lane + 2 * (c & 1) + 1 < a.N;
          const uint16_t* p = szsrc + g * a.ssg + n_lane;
          const uint32_t v = (in0 ? uint32_t(__ldg(p)) : 0u) | ((in1 ? uint32_t(__ldg(p + 1)) : 0u) << 16);
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(d), "r"(v) : "memory");
        }
        if (++gcnt == a.gpl) {
          gcnt = 0;
          ++g;
        }
      }
      cp_async_commit();
      dst += SPST * WSTEP;
      dst_sz += SEGST * SZSEG;
    }
  }

  // ---- activations: produced by the previous kernel of the stream
  if (a.pdl) {
    pdl_launch_dependents();
    pdl_wait();
  }
  {
    // Stage x in shared memory, each 8-k chunk permuted to the k order of the A fragments.
    __shared__ float s_inv[32];
    stage_activations<F16, PRO>(a, s_x, k0, nstages * SPST * 4, a.KC / 8, s_inv);
  }
  __syncthreads();

  // acc: the k16 halves of each step accumulate separately (two MMA chains), added at the end
  float acc[2][MT][4], acc1[2][MT][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[t][mt][e] = acc1[t][mt][e] = 0.0f;

  const uint32_t magic = F16 ? 0x64006400u : 0x43004300u;
  uint32_t wl = s_w + (warp * 32 + lane) * 16;
  uint32_t szl = s_sz + (warp * 8 + r) * 16;
  // Token rows past M read a real row instead: their outputs are discarded, and no branch is needed.
  uint32_t xl[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) xl[mt] = s_x + min(mt * 8 + r, M - 1) * a.xpitch + 16 * c;

  DqParams dp[4];
  for (int st = 0; st < nstages; ++st) {
    cp_async_wait_upto(nstages - 1 - st);  // this lane's copies of stage st have landed
    __syncwarp();                           // and the scales / zeros copied by lanes c == 0
#pragma unroll
    for (int i = 0; i < SPST; ++i) {
      if (i % SPS == 0) {  // a new segment: scale and zero of columns 4r .. 4r + 3
        const uint4 sz = lds128(szl + (i / SPS) * SZSEG);
        dp[0] = dq_params<F16>(uint16_t(sz.x & 0xFFFFu), uint16_t(sz.z & 0xFFFFu));
        dp[1] = dq_params<F16>(uint16_t(sz.x >> 16), uint16_t(sz.z >> 16));
        dp[2] = dq_params<F16>(uint16_t(sz.y & 0xFFFFu), uint16_t(sz.w & 0xFFFFu));
        dp[3] = dq_params<F16>(uint16_t(sz.y >> 16), uint16_t(sz.w >> 16));
      }
      const uint4 w4 = lds128(wl + i * WSTEP);
      const uint32_t wd[4] = {w4.x, w4.y, w4.z, w4.w};
      uint32_t af[2][2][4];  // [row tile][k16 half][reg]: the dequantized weights, rounded as the reference does
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          af[t][s][0] = dq_pair<F16>(nib_pair(wd[2 * t], 2 * s, magic), dp[2 * t]);
          af[t][s][1] = dq_pair<F16>(nib_pair(wd[2 * t + 1], 2 * s, magic), dp[2 * t + 1]);
          af[t][s][2] = dq_pair<F16>(nib_pair(wd[2 * t], 2 * s + 1, magic), dp[2 * t]);
          af[t][s][3] = dq_pair<F16>(nib_pair(wd[2 * t + 1], 2 * s + 1, magic), dp[2 * t + 1]);
        }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint4 b = lds128(xl[mt] + i * 64);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          mma_16816<F16>(acc[t][mt], af[t][0], b.x, b.y);
          mma_16816<F16>(acc1[t][mt], af[t][1], b.z, b.w);
        }
      }
    }
    wl += SPST * WSTEP;
    szl += SEGST * SZSEG;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) xl[mt] += SPST * 64;
  }
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[t][mt][e] += acc1[t][mt][e];

  // ---- outputs: acc[t][mt][e] is (token mt*8 + 2c + (e & 1), column 32*warp + 4r + 2t + (e >> 1))
  uint16_t* y = a.y;
  __shared__ uint32_t s_ep;
  if (a.ar_world > 1 && a.mode == 0) {
    // Tensor-parallel sum of the ranks' outputs: push, publish, wait for the other ranks, add in rank order.
    const uint32_t ep = ar_epoch(a, &s_ep);
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = mt * 8 + 2 * c + (e & 1);
          const int64_t n = n_lane + 2 * t + (e >> 1);
          if (tok < M && n < a.N) ar_push(a, ep, int64_t(tok) * a.N + n, acc[t][mt][e]);
        }
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = mt * 8 + 2 * c + (e & 1);
          const int64_t n = n_lane + 2 * t + (e >> 1);
          if (tok < M && n < a.N) y[int64_t(tok) * a.sym + n] = f2h_bits<F16>(ar_sum(a, ep, int64_t(tok) * a.N + n));
        }
    ar_finish(a, ep);
    return;
  }
  if (a.mode == 0) {
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = mt * 8 + 2 * c + (e & 1);
          const int64_t n = n_lane + 2 * t + (e >> 1);
          if (tok < M && n < a.N) y[int64_t(tok) * a.sym + n] = f2h_bits<F16>(acc[t][mt][e]);
        }
    return;
  }
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = mt * 8 + 2 * c + (e & 1);
        if (tok < M) sP[tok * kBN + warp * 32 + 4 * r + 2 * t + (e >> 1)] = acc[t][mt][e];
      }
  if (a.mode == 1) {
    // Cluster of S CTAs along K: rank q adds outputs q*128 + tid, (q + S)*128 + tid, ... over all ranks in order.
    const uint32_t ep = a.ar_world > 1 ? ar_epoch(a, &s_ep) : 0u;
    cluster_sync();
    const uint32_t rank = cluster_ctarank();
    if (a.ar_world > 1) {
      // The cluster's sums are this rank's partials: push them, then the tensor-parallel sum as in mode 0.
      for (int idx = int(rank) * kBN + tid; idx < M * kBN; idx += a.S * kBN) {
        const uint32_t addr = smem_u32(sP + idx);
        float t[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) t[q] = q < a.S ? ld_shared_cluster_f32(mapa_shared(addr, uint32_t(q))) : 0.0f;
        float v = t[0];
#pragma unroll
        for (int q = 1; q < 8; ++q)
          if (q < a.S) v += t[q];
        const int tok = idx / kBN;
        const int64_t n = n0 + idx % kBN;
        if (n < a.N) ar_push(a, ep, int64_t(tok) * a.N + n, v);
      }
      cluster_sync();  // remote shared-memory reads done before any CTA of the cluster moves on
      for (int idx = int(rank) * kBN + tid; idx < M * kBN; idx += a.S * kBN) {
        const int tok = idx / kBN;
        const int64_t n = n0 + idx % kBN;
        if (n < a.N) y[int64_t(tok) * a.sym + n] = f2h_bits<F16>(ar_sum(a, ep, int64_t(tok) * a.N + n));
      }
      ar_finish(a, ep);
      return;
    }
    for (int idx = int(rank) * kBN + tid; idx < M * kBN; idx += a.S * kBN) {
      const uint32_t addr = smem_u32(sP + idx);
      float t[8];  // all S (<= 8) remote loads in flight, then added in rank order
#pragma unroll
      for (int q = 0; q < 8; ++q) t[q] = q < a.S ? ld_shared_cluster_f32(mapa_shared(addr, uint32_t(q))) : 0.0f;
      float v = t[0];
#pragma unroll
      for (int q = 1; q < 8; ++q)
        if (q < a.S) v += t[q];
      const int tok = idx / kBN;
      const int64_t n = n0 + idx % kBN;
      if (n < a.N) y[int64_t(tok) * a.sym + n] = f2h_bits<F16>(v);
    }
    cluster_sync();  // no CTA leaves while others may still read its shared memory
    return;
  }
  // mode 2: fp32 partials in the workspace; the last CTA of the column tile adds them in split order.
  __syncthreads();
  for (int idx = tid; idx < M * kBN; idx += blockDim.x) {
    const int tok = idx / kBN;
    const int64_t n = n0 + idx % kBN;
    if (n < a.N) a.partials[(int64_t(blockIdx.y) * M + tok) * a.N + n] = sP[idx];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(a.tickets + blockIdx.x, 1u);
    s_last = (prev == unsigned(a.S - 1));
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = tid; idx < M * kBN; idx += blockDim.x) {
    const int tok = idx / kBN;
    const int64_t n = n0 + idx % kBN;
    if (n >= a.N) continue;
    const float* src = a.partials + int64_t(tok) * a.N + n;
    const int64_t sstride = int64_t(M) * a.N;
    float v = 0.0f;
    for (int s0 = 0; s0 < a.S; s0 += 8) {  // eight partials in flight, added in split order
      float t[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) t[j] = s0 + j < a.S ? __ldcg(src + (s0 + j) * sstride) : 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (s0 + j < a.S) v = (s0 + j == 0) ? t[j] : v + t[j];
    }
    y[int64_t(tok) * a.sym + n] = f2h_bits<F16>(v);
  }
  if (tid == 0) atomicExch(a.tickets + blockIdx.x, 0u);
}

// ------------------------------------------------------------------ streaming variant (very wide N)

#ifndef I4B_STREAM_RING
#define I4B_STREAM_RING 3
#endif
#ifndef I4B_STREAM_STEPS
#define I4B_STREAM_STEPS 4
#endif
constexpr int kStreamRing = I4B_STREAM_RING;    // stages in flight per warp
constexpr int kStreamSteps = I4B_STREAM_STEPS;  // 32-k steps per stage (at least SPS)

// For matrices with many more 32-column slabs than warps (an lm_head: N = 128256), a persistent grid of
// warps streams slabs of 32 columns x the whole K: warp g takes slabs g, g + W, g + 2W, ... (W warps in
// the grid), keeping kStreamRing stages of 4 (or SPS) 32-k steps in flight through its own cp.async ring, so
// the weight stream never stops between slabs.  The activations (M <= 8 rows x K) are staged once per
// CTA.  No K split, hence no cross-CTA reduction; the dequant / MMA / segment
// arithmetic is that of w4_skinny_kernel.
template <bool F16, int SPS, bool ONE, bool ARG = false>
__global__ void __launch_bounds__(128) w4_stream_kernel(const W4SArgs a) {
  constexpr int SPST = SPS > kStreamSteps ? SPS : kStreamSteps;  // 32-k steps per ring stage
  constexpr int SEGST = SPST / SPS;
  constexpr int RING = kStreamRing;
  constexpr int WSTAGE = SPST * 512;       // weight bytes of a stage (32 lanes x 16 B per step)
  constexpr int SZSTAGE = SEGST * 128;     // scale / zero bytes of a stage (8 records of 16 B per segment)
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = lane >> 2, c = lane & 3;
  const int M = a.M;
  const int K = a.K;
  const int stages_slab = K / (32 * SPST);
  const int nslabs = (a.N + 31) / 32;
  const int W = int(gridDim.x) * 4;
  const int gw = int(blockIdx.x) * 4 + warp;
  const int my_slabs = gw < nslabs ? (nslabs - gw + W - 1) / W : 0;
  const int total = my_slabs * stages_slab;

  const uint32_t s_base = smem_u32(smem);
  const uint32_t s_x = s_base;                                   // [M][xpitch]
  const uint32_t s_w = s_base + a.off_sz + warp * RING * (WSTAGE + SZSTAGE);  // this warp's ring

  // Issue cursor: the next stage of this warp's stream (slab, stage in the slab, ring slot), kept as
  // running pointers so that no division is needed per stage.
  const int64_t row4 = 4 * a.sqk;  // words between the k8 rows of consecutive 32-k steps
  int is_left = total, is_st = 0, is_slot = 0;
  int64_t is_n = int64_t(gw) * 32 + 4 * r;
  const uint32_t* is_w = a.qw + int64_t(c) * a.sqk + is_n;
  const uint16_t* const sz0 = (c < 2 ? a.sc : a.zr) + 2 * (c & 1);
  const uint16_t* is_sz = sz0 + is_n;
  int is_gcnt = 0;  // segments issued in the current group
  auto issue_next = [&]() {
    if (is_left > 0) {
      const bool n_in = is_n < a.N;
      const uint32_t dst = s_w + is_slot * (WSTAGE + SZSTAGE);
      if (n_in) {
        const uint32_t* src = is_w;
#pragma unroll
        for (int i = 0; i < SPST; ++i) {
          cp16(dst + i * 512 + lane * 16, src, 16u);
          src += row4;
        }
      } else {
#pragma unroll
        for (int i = 0; i < SPST; ++i) cp16(dst + i * 512 + lane * 16, a.qw, 0u);  // columns past N: zeros
      }
#pragma unroll
      for (int j = 0; j < SEGST; ++j) {
        cp4(dst + WSTAGE + j * 128 + r * 16 + 4 * c, n_in ? is_sz : a.sc, n_in ? 4u : 0u);
        if (++is_gcnt == a.gpl) {
          is_gcnt = 0;
          is_sz += a.ssg;
        }
      }
      --is_left;
      is_slot = is_slot == RING - 1 ? 0 : is_slot + 1;
      if (++is_st == stages_slab) {  // next slab of this warp
        is_st = 0;
        is_n += int64_t(W) * 32;
        is_w = a.qw + int64_t(c) * a.sqk + is_n;
        is_sz = sz0 + is_n;
        is_gcnt = 0;
      } else {
        is_w += SPST * row4;
      }
    }
    cp_async_commit();
  };
#pragma unroll 1
  for (int g = 0; g < RING; ++g) issue_next();

  if (a.pdl) {
    pdl_launch_dependents();
    pdl_wait();
  }
  {
    // stage x in shared memory, each 8-k chunk permuted to the k order of the A fragments
    const int nch = K / 8;
    const int ntot = M * nch;
    for (int idx = tid; idx < ntot; idx += 128) {
      const int t = idx / nch, ch = idx - t * nch;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(a.x + int64_t(t) * a.sxm + 8 * ch));
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(s_x + t * a.xpitch + ch * 16),
                   "r"(__byte_perm(v.x, v.z, 0x5410)), "r"(__byte_perm(v.x, v.z, 0x7632)),
                   "r"(__byte_perm(v.y, v.w, 0x5410)), "r"(__byte_perm(v.y, v.w, 0x7632))
                   : "memory");
    }
  }
  __syncthreads();

  const uint32_t magic = F16 ? 0x64006400u : 0x43004300u;
  const uint32_t xl0 = s_x + min(r, M - 1) * a.xpitch + 16 * c;
  float acc[2][4], acc1[2][4];  // the k16 halves of each step accumulate separately (two MMA chains)
  int st = 0, slot = 0;
  int64_t n_base = int64_t(gw) * 32 + 4 * r;
  float gbest[2] = {-INFINITY, -INFINITY};  // fused greedy choice: this lane's first maxima of tokens 2c, 2c+1
  int64_t gidx[2] = {INT64_MAX, INT64_MAX};
  uint32_t xl = xl0;
  DqParams dp[4];
#pragma unroll 1
  for (int g = 0; g < total; ++g) {
    if (st == 0) {
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[t][e] = acc1[t][e] = 0.0f;
    }
    cp_async_wait<RING - 1>();
    __syncwarp();
    const uint32_t sl = s_w + slot * (WSTAGE + SZSTAGE);
#pragma unroll
    for (int i = 0; i < SPST; ++i) {
      if (i % SPS == 0) {  // a new segment: scale and zero of columns 4r .. 4r + 3
        const uint4 sz = lds128(sl + WSTAGE + (i / SPS) * 128 + r * 16);
        dp[0] = dq_params<F16>(uint16_t(sz.x & 0xFFFFu), uint16_t(sz.z & 0xFFFFu));
        dp[1] = dq_params<F16>(uint16_t(sz.x >> 16), uint16_t(sz.z >> 16));
        dp[2] = dq_params<F16>(uint16_t(sz.y & 0xFFFFu), uint16_t(sz.w & 0xFFFFu));
        dp[3] = dq_params<F16>(uint16_t(sz.y >> 16), uint16_t(sz.w >> 16));
      }
      const uint4 w4 = lds128(sl + i * 512 + lane * 16);
      const uint32_t wd[4] = {w4.x, w4.y, w4.z, w4.w};
      uint32_t af[2][2][4];  // the dequantized weights, rounded as the reference does
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          af[t][q][0] = dq_pair<F16>(nib_pair(wd[2 * t], 2 * q, magic), dp[2 * t]);
          af[t][q][1] = dq_pair<F16>(nib_pair(wd[2 * t + 1], 2 * q, magic), dp[2 * t + 1]);
          af[t][q][2] = dq_pair<F16>(nib_pair(wd[2 * t], 2 * q + 1, magic), dp[2 * t]);
          af[t][q][3] = dq_pair<F16>(nib_pair(wd[2 * t + 1], 2 * q + 1, magic), dp[2 * t + 1]);
        }
      const uint4 b = lds128(xl + i * 64);
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        mma_16816<F16>(acc[t], af[t][0], b.x, b.y);
        mma_16816<F16>(acc1[t], af[t][1], b.z, b.w);
      }
    }
    __syncwarp();  // every lane is done with the slot before it is refilled
    issue_next();
    slot = slot == RING - 1 ? 0 : slot + 1;
    xl += SPST * 64;
    if (++st == stages_slab) {  // slab complete: acc[t][e] is (token 2c + (e & 1), column 4r + 2t + (e >> 1))
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (ONE && (e & 1)) continue;
          const int tok = 2 * c + (e & 1);
          const int64_t n = n_base + 2 * t + (e >> 1);
          const uint16_t bits = f2h_bits<F16>(acc[t][e] + acc1[t][e]);
          if (tok < M && n < a.N) {
            if (!ARG || a.y) a.y[int64_t(tok) * a.sym + n] = bits;
            if constexpr (ARG) {
              const float v = F16 ? __half2float(__ushort_as_half(bits)) : __uint_as_float(uint32_t(bits) << 16);
              first_max(gbest[e & 1], gidx[e & 1], v, n);
            }
          }
        }
      st = 0;
      n_base += int64_t(W) * 32;
      xl = xl0;
    }
  }
  cp_async_wait<0>();
  if constexpr (ARG) {
    // lanes with the same c hold the same two tokens: reduce over r, then one candidate per warp and token
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        const float ob = __shfl_xor_sync(0xFFFFFFFFu, gbest[h], o);
        const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, gidx[h], o);
        first_max(gbest[h], gidx[h], ob, oi);
      }
    if (r == 0)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int tok = 2 * c + h;
        if (tok < M)
          a.cand[int64_t(gw) * M + tok] = make_float2(gbest[h], __int_as_float(gidx[h] == INT64_MAX ? -1 : int(gidx[h])));
      }
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.tickets, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int nwarps_total = int(gridDim.x) * 4;
    for (int t = warp; t < M; t += 4) {
      float best = -INFINITY;
      int64_t bi = INT64_MAX;
      for (int w = lane; w < nwarps_total; w += 32) {
        const float2 cnd = __ldcg(a.cand + int64_t(w) * M + t);
        const int i = __float_as_int(cnd.y);
        if (i >= 0) first_max(best, bi, cnd.x, i);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        first_max(best, bi, ob, oi);
      }
      if (lane == 0) a.amax_out[t] = bi == INT64_MAX ? 0 : bi;
    }
    if (tid == 0) atomicExch(a.tickets, 0u);
  }
}

// ------------------------------------------------------------------ greedy choice fused into the GEMV


// Greedy token of every row, fused after the logits of the tile are final (vals[tok * BN + col]: the logits as
// stored, -inf past N).  Warp t finds token t's first maximum in the tile and stores it as the tile's candidate;
// the last CTA to finish (atomic ticket, no spinning) compares the candidates of all tiles in tile order --
// i.e. column order -- and writes the index of the first maximum of the row (0 when no logit exceeds -inf),
// then resets the ticket.
__device__ __forceinline__ void greedy_epilogue(const W4SArgs& a, const float* vals, int nout, int BN, int64_t n0) {
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  __syncthreads();
  for (int t = warp; t < a.M; t += nwarps) {
    float best = -INFINITY;
    int64_t bi = INT64_MAX;
    for (int col = lane; col < BN; col += 32) first_max(best, bi, vals[t * BN + col], n0 + col);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      first_max(best, bi, ob, oi);
    }
    if (lane == 0)
      a.cand[int64_t(blockIdx.x) * a.M + t] = make_float2(best, __int_as_float(bi == INT64_MAX ? -1 : int(bi)));
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(a.tickets, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int t = warp; t < a.M; t += nwarps) {
    float best = -INFINITY;
    int64_t bi = INT64_MAX;
    for (int tile = lane; tile < int(gridDim.x); tile += 32) {
      const float2 c = __ldcg(a.cand + int64_t(tile) * a.M + t);
      const int i = __float_as_int(c.y);
      if (i >= 0) first_max(best, bi, c.x, i);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      first_max(best, bi, ob, oi);
    }
    if (lane == 0) a.amax_out[t] = bi == INT64_MAX ? 0 : bi;
  }
  if (tid == 0) atomicExch(a.tickets, 0u);
}

// ------------------------------------------------------------------ decode GEMV, M <= 8, weights in registers

// Register-streaming form of the M <= 8 path.  grid = (ceil(N / (32 WN)), S), cluster (1, S, 1) when S > 1;
// CTA = WN x WK warps.  Warp (wn, wk) owns columns n0 + 32 wn .. + 31 and the k range
// [k0 + wk KW, k0 + (wk + 1) KW) of its CTA's K slice [k0, k0 + KC), KC = K / S.  Each lane streams its packed
// words straight into a ring of D registers with 128-bit loads that bypass L1 (lane (r, c) reads the words
// of columns 4r..4r+3 at k8 row 4 step + c: 4 x 128 contiguous bytes per warp and step), so no copy through
// shared memory and no barrier sits between the weight stream and the math.  The ring's first D steps are
// requested before griddepcontrol.wait.  Scales / zeros of the CTA's columns and groups are staged once in
// shared memory (cp.async), the activations once per CTA (stage_activations).  Dequant and MMA are those of
// w4_skinny_kernel.  The WK warp partials of a column add in shared memory in warp order; the S CTAs of a
// cluster then add through distributed shared memory in rank order: results are identical from run to run.
template <bool F16, int SPS, int PRO, int D, bool ARG>
__global__ void __launch_bounds__(256) w4_gemv_kernel(const W4SArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float s_inv[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wn = warp % a.WN, wk = warp / a.WN;
  const int r = lane >> 2, c = lane & 3;
  const int BN = 32 * a.WN;
  const int M = a.M;
  const int64_t n0 = int64_t(blockIdx.x) * BN;
  const int k0 = int(blockIdx.y) * a.KC;
  const int kw0 = wk * a.KW;  // warp's first k inside the CTA slice
  const int nsteps = a.KW / 32;
  const int64_t n_lane = n0 + wn * 32 + 4 * r;
  const bool n_in = n_lane < a.N;  // N % 8 == 0: a lane's 4 columns are all in or all out

  const uint32_t s_base = smem_u32(smem);
  const uint32_t s_sz = s_base + a.off_sz;  // scales [rows][BN] fp16, then zeros [rows][BN] fp16
  const uint32_t s_x = s_base + a.off_x;
  float* red = reinterpret_cast<float*>(smem + a.off_part);  // [WK][M][BN]

  // ---- weights: the first D steps of this lane's stream, independent of the previous kernel
  const uint32_t* wsrc = a.qw + int64_t((k0 + kw0) / 8 + c) * a.sqk + (n_in ? n_lane : 0);
  const int64_t wstep = 4 * a.sqk;
  uint4 wr[D];
#pragma unroll
  for (int i = 0; i < D; ++i)
    wr[i] = (i < nsteps && n_in) ? ld_stream_u4(wsrc + i * wstep) : make_uint4(0u, 0u, 0u, 0u);
  const int g_first = k0 / a.G;
  // ---- scales / zeros of the CTA's groups and columns: 16-byte chunks of 8 columns
  {
    const int rows = min(a.sz_rows, a.K / a.G - g_first);  // group rows of this CTA's K slice
    const int cpr = BN / 8;                                  // chunks per row
    const int nchunk = 2 * a.sz_rows * cpr;
    for (int i = tid; i < nchunk; i += blockDim.x) {
      const int arr = i / (a.sz_rows * cpr), rem = i - arr * (a.sz_rows * cpr);
      const int row = rem / cpr, ch = rem - row * cpr;
      if (row >= rows) continue;
      const int64_t n = n0 + 8 * ch;
      const uint16_t* src = (arr ? a.zr : a.sc) + int64_t(g_first + row) * a.ssg + (n < a.N ? n : 0);
      cp16(s_sz + uint32_t(arr * a.sz_rows * BN * 2 + row * BN * 2 + ch * 16), src, n < a.N ? 16u : 0u);
    }
    cp_async_commit();
  }
  // ---- activations: produced by the previous kernel of the stream
  if (a.pdl) {
    pdl_launch_dependents();
    pdl_wait();
  }
  stage_activations<F16, PRO>(a, s_x, k0, a.KC / 8, a.KC / 8, s_inv);
  cp_async_wait<0>();
  __syncthreads();

  const uint32_t magic = F16 ? 0x64006400u : 0x43004300u;
  const uint32_t xl = s_x + min(r, M - 1) * a.xpitch + (kw0 / 8 + c) * 16;
  const int L = 32 * SPS;
  const uint32_t szl = s_sz + uint32_t((wn * 32 + 4 * r) * 2);
  float acc[2][4], acc1[2][4];  // the k16 halves of each step accumulate separately (two MMA chains)
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[t][e] = acc1[t][e] = 0.0f;
  DqParams dp[4];
#pragma unroll 1
  for (int base = 0; base < nsteps; base += D) {
#pragma unroll
    for (int i = 0; i < D; ++i) {
      const int step = base + i;
      if (step >= nsteps) break;  // uniform over the CTA
      if (step % SPS == 0) {      // a new segment: scale and zero of columns 4r .. 4r + 3
        const int seg = (k0 + kw0) / L + step / SPS;
        const int row = (a.gpl_shift >= 0 ? (seg >> a.gpl_shift) : seg / a.gpl) - g_first;
        uint32_t sv0, sv1, zv0, zv1;
        const uint32_t sa = szl + uint32_t(row * BN * 2), za = sa + uint32_t(a.sz_rows * BN * 2);
        asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(sv0), "=r"(sv1) : "r"(sa));
        asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(zv0), "=r"(zv1) : "r"(za));
        dq_params_shared<F16>(make_uint4(sv0, sv1, zv0, zv1), c, dp);
      }
      const uint32_t wd[4] = {wr[i].x, wr[i].y, wr[i].z, wr[i].w};
      if (step + D < nsteps && n_in) wr[i] = ld_stream_u4(wsrc + (step + D) * wstep);  // refill the slot
      uint32_t af[2][2][4];  // [row tile][k16 half][reg]: the dequantized weights, rounded as the reference does
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          af[t][h][0] = dq_pair<F16>(nib_pair(wd[2 * t], 2 * h, magic), dp[2 * t]);
          af[t][h][1] = dq_pair<F16>(nib_pair(wd[2 * t + 1], 2 * h, magic), dp[2 * t + 1]);
          af[t][h][2] = dq_pair<F16>(nib_pair(wd[2 * t], 2 * h + 1, magic), dp[2 * t]);
          af[t][h][3] = dq_pair<F16>(nib_pair(wd[2 * t + 1], 2 * h + 1, magic), dp[2 * t + 1]);
        }
      const uint4 b = lds128(xl + step * 64);
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        mma_16816<F16>(acc[t], af[t][0], b.x, b.y);
        mma_16816<F16>(acc1[t], af[t][1], b.z, b.w);
      }
    }
  }
  // ---- this warp's partials: acc[t][e] is (token 2c + (e & 1), column 32 wn + 4r + 2t + (e >> 1))
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int tok = 2 * c + (e & 1);
      if (tok < M) red[(wk * M + tok) * BN + wn * 32 + 4 * r + 2 * t + (e >> 1)] = acc[t][e] + acc1[t][e];
    }
  __syncthreads();
  const int nout = M * BN;
  for (int idx = tid; idx < nout; idx += blockDim.x) {  // sum over the K warps, in warp order
    float v = red[idx];
    for (int q = 1; q < a.WK; ++q) v += red[q * nout + idx];
    if (a.S == 1) {
      const int tok = idx / BN;
      const int64_t n = n0 + (idx - tok * BN);
      const uint16_t bits = f2h_bits<F16>(v);
      if (n < a.N && a.y) a.y[int64_t(tok) * a.sym + n] = bits;
      if constexpr (ARG) {  // the logit as stored, or -inf past N; the warp-order sum above has read red[idx]
        const float r = F16 ? __half2float(__ushort_as_half(bits)) : __uint_as_float(uint32_t(bits) << 16);
        red[idx] = n < a.N ? r : -INFINITY;
      }
    } else {
      red[idx] = v;
    }
  }
  if constexpr (ARG) {
    greedy_epilogue(a, red, nout, BN, n0);
    return;
  }
  if (a.S == 1) return;
  // Cluster of S CTAs along K: rank q adds outputs q*blockDim + tid, ... over all ranks, in rank order.
  cluster_sync();
  const uint32_t rank = cluster_ctarank();
  for (int idx = int(rank) * blockDim.x + tid; idx < nout; idx += a.S * blockDim.x) {
    const uint32_t addr = smem_u32(red + idx);
    float t[8];  // all S (<= 8) remote loads in flight, then added in rank order
#pragma unroll
    for (int q = 0; q < 8; ++q) t[q] = q < a.S ? ld_shared_cluster_f32(mapa_shared(addr, uint32_t(q))) : 0.0f;
    float v = t[0];
#pragma unroll
    for (int q = 1; q < 8; ++q)
      if (q < a.S) v += t[q];
    const int tok = idx / BN;
    const int64_t n = n0 + (idx - tok * BN);
    if (n < a.N) a.y[int64_t(tok) * a.sym + n] = f2h_bits<F16>(v);
  }
  cluster_sync();  // no CTA leaves while others may still read its shared memory
}

// ------------------------------------------------------------------ slab-streaming GEMV (M <= 8), K split over P warps

// The streaming kernel above, generalised to any width: a persistent grid of CTAs of 4 warps; the warps of a
// CTA form 4 / P groups of P warps, and a group takes the CTA's slabs (32 columns x all of K) one after the
// other, its P warps splitting each slab's K into P consecutive parts.  Each warp streams its part of slab
// after slab through its own cp.async ring (RING stages of SPST 32-k steps), so the weight stream does not
// stop between slabs and the per-warp fixed work (ring fill, activation staging) is paid once per launch.
// The activations (any prologue) are staged once per CTA.  For P > 1 the warps of a group write their
// partial sums of a slab into a double-buffered shared array, meet at a named barrier of the group, and
// warp 0 of the group adds the P partials in part order: results are identical from run to run.
template <bool F16, int SPS, int PRO, int P>
__global__ void __launch_bounds__(32 * (P > 4 ? P : 4)) w4_slab_kernel(const W4SArgs a) {
  constexpr int SPST = SPS > kStreamSteps ? SPS : kStreamSteps;  // 32-k steps per ring stage
  constexpr int SEGST = SPST / SPS;
  constexpr int RING = kStreamRing;
  constexpr int WSTAGE = SPST * 512;    // weight bytes of a stage (32 lanes x 16 B per step)
  constexpr int SZSTAGE = SEGST * 128;  // scale / zero bytes of a stage (8 records of 16 B per segment)
  constexpr int NW = P > 4 ? P : 4;     // warps per CTA
  constexpr int GPC = NW / P;           // slab groups per CTA
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float s_inv[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = lane >> 2, c = lane & 3;
  const int part = warp % P, grp = warp / P;
  const int M = a.M;
  const int KP = a.K / P;  // k per warp and slab
  const int kp0 = part * KP;
  const int L = 32 * SPS;
  const int stages_slab = KP / (32 * SPST);
  const int nslabs = (a.N + 31) / 32;
  const int G_total = int(gridDim.x) * GPC;
  const int gg = int(blockIdx.x) * GPC + grp;
  const int my_slabs = gg < nslabs ? (nslabs - gg + G_total - 1) / G_total : 0;  // same for the group's warps
  const int total = my_slabs * stages_slab;

  const uint32_t s_base = smem_u32(smem);
  const uint32_t s_x = s_base;                                            // [M][xpitch]
  float* partials = reinterpret_cast<float*>(smem + a.off_part);         // [2][GPC][P][8 tokens][32 columns]
  const uint32_t s_w = s_base + a.off_sz + warp * RING * (WSTAGE + SZSTAGE);  // this warp's ring

  // Issue cursor: the next stage of this warp's stream, as running pointers (no division per stage).
  const int64_t row4 = 4 * a.sqk;  // words between the k8 rows of consecutive 32-k steps
  const int g_row0 = kp0 / a.G;    // first scale row of this warp's part
  const int gcnt0 = (kp0 / L) % a.gpl;
  int is_left = total, is_st = 0, is_slot = 0;
  int64_t is_n = int64_t(gg) * 32 + 4 * r;
  const uint32_t* const w_part = a.qw + int64_t(kp0 / 8 + c) * a.sqk;
  const uint32_t* is_w = w_part + is_n;
  const uint16_t* const sz0 = (c < 2 ? a.sc : a.zr) + 2 * (c & 1) + int64_t(g_row0) * a.ssg;
  const uint16_t* is_sz = sz0 + is_n;
  int is_gcnt = gcnt0;
  auto issue_next = [&]() {
    if (is_left > 0) {
      const bool n_in = is_n < a.N;
      const uint32_t dst = s_w + is_slot * (WSTAGE + SZSTAGE);
      if (n_in) {
        const uint32_t* src = is_w;
#pragma unroll
        for (int i = 0; i < SPST; ++i) {
          cp16(dst + i * 512 + lane * 16, src, 16u);
          src += row4;
        }
      } else {
#pragma unroll
        for (int i = 0; i < SPST; ++i) cp16(dst + i * 512 + lane * 16, a.qw, 0u);  // columns past N: zeros
      }
#pragma unroll
      for (int j = 0; j < SEGST; ++j) {
        cp4(dst + WSTAGE + j * 128 + r * 16 + 4 * c, n_in ? is_sz : a.sc, n_in ? 4u : 0u);
        if (++is_gcnt == a.gpl) {
          is_gcnt = 0;
          is_sz += a.ssg;
        }
      }
      --is_left;
      is_slot = is_slot == RING - 1 ? 0 : is_slot + 1;
      if (++is_st == stages_slab) {  // next slab of this group
        is_st = 0;
        is_n += int64_t(G_total) * 32;
        is_w = w_part + is_n;
        is_sz = sz0 + is_n;
        is_gcnt = gcnt0;
      } else {
        is_w += SPST * row4;
      }
    }
    cp_async_commit();
  };
#pragma unroll 1
  for (int g = 0; g < RING; ++g) issue_next();

  if (a.pdl) {
    pdl_launch_dependents();
    pdl_wait();
  }
  stage_activations<F16, PRO>(a, s_x, 0, a.K / 8, a.K / 8, s_inv);
  __syncthreads();

  const uint32_t magic = F16 ? 0x64006400u : 0x43004300u;
  const uint32_t xl0 = s_x + min(r, M - 1) * a.xpitch + (kp0 / 8 + c) * 16;
  float acc[2][4], acc1[2][4];  // the k16 halves of each step accumulate separately (two MMA chains)
  int st = 0, slot = 0, sl = 0;
  int64_t n_slab = int64_t(gg) * 32;
  uint32_t xl = xl0;
  DqParams dp[4];
#pragma unroll 1
  for (int g = 0; g < total; ++g) {
    if (st == 0) {
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[t][e] = acc1[t][e] = 0.0f;
    }
    cp_async_wait<RING - 1>();
    __syncwarp();
    const uint32_t sb = s_w + slot * (WSTAGE + SZSTAGE);
#pragma unroll
    for (int i = 0; i < SPST; ++i) {
      if (i % SPS == 0) {  // a new segment: scale and zero of columns 4r .. 4r + 3
        dq_params_shared<F16>(lds128(sb + WSTAGE + (i / SPS) * 128 + r * 16), c, dp);
      }
      const uint4 w4 = lds128(sb + i * 512 + lane * 16);
      const uint32_t wd[4] = {w4.x, w4.y, w4.z, w4.w};
      uint32_t af[2][2][4];  // the dequantized weights, rounded as the reference does
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          af[t][h][0] = dq_pair<F16>(nib_pair(wd[2 * t], 2 * h, magic), dp[2 * t]);
          af[t][h][1] = dq_pair<F16>(nib_pair(wd[2 * t + 1], 2 * h, magic), dp[2 * t + 1]);
          af[t][h][2] = dq_pair<F16>(nib_pair(wd[2 * t], 2 * h + 1, magic), dp[2 * t]);
          af[t][h][3] = dq_pair<F16>(nib_pair(wd[2 * t + 1], 2 * h + 1, magic), dp[2 * t + 1]);
        }
      const uint4 b = lds128(xl + i * 64);
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        mma_16816<F16>(acc[t], af[t][0], b.x, b.y);
        mma_16816<F16>(acc1[t], af[t][1], b.z, b.w);
      }
    }
    __syncwarp();  // every lane is done with the slot before it is refilled
    issue_next();
    slot = slot == RING - 1 ? 0 : slot + 1;
    xl += SPST * 64;
    if (++st == stages_slab) {  // slab complete: acc[t][e] is (token 2c + (e & 1), column 4r + 2t + (e >> 1))
      if constexpr (P == 1) {
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int tok = 2 * c + (e & 1);
            const int64_t n = n_slab + 4 * r + 2 * t + (e >> 1);
            if (tok < M && n < a.N) a.y[int64_t(tok) * a.sym + n] = f2h_bits<F16>(acc[t][e] + acc1[t][e]);
          }
      } else {
        float* pb = partials + ((sl & 1) * GPC + grp) * (P * 256);
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int tok = 2 * c + (e & 1);
            if (tok < M) pb[part * 256 + tok * 32 + 4 * r + 2 * t + (e >> 1)] = acc[t][e] + acc1[t][e];
          }
        // the group's P warps meet; warp 0 of the group adds the parts in order (the next slab's barrier
        // keeps the other buffer from being rewritten before it has been read)
        asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(32 * P) : "memory");
        if (part == 0) {
          const int64_t n = n_slab + lane;
          for (int tok = 0; tok < M; ++tok) {
            float v = pb[tok * 32 + lane];
#pragma unroll
            for (int q = 1; q < P; ++q) v += pb[q * 256 + tok * 32 + lane];
            if (n < a.N) a.y[int64_t(tok) * a.sym + n] = f2h_bits<F16>(v);
          }
        }
      }
      st = 0;
      ++sl;
      n_slab += int64_t(G_total) * 32;
      xl = xl0;
    }
  }
  cp_async_wait<0>();
}

// ------------------------------------------------------------------ planning

static int g_w4_ovr_s = 0;
static int g_w4_ovr_kernel = 0, g_w4_ovr_wk = 0, g_w4_ovr_gs = 0;

void set_w4_split_override(int splits) { g_w4_ovr_s = splits; }
void set_w4_kernel_override(int kernel, int wk, int splits) {
  g_w4_ovr_kernel = kernel;
  g_w4_ovr_wk = wk;
  g_w4_ovr_gs = splits;
}

static int gcd_i(int a, int b) {
  while (b) {
    const int t = a % b;
    a = b;
    b = t;
  }
  return a;
}

// K is cut into units of L = 32 * gcd(G/32, 8) k (a segment: L divides G, so it lies in one group);
// a CTA owns KC = K / S consecutive k, a whole number of units, at most kMaxKC.
W4Plan plan_w4(int64_t M, int64_t N, int64_t K, int G, int num_sms) {
  W4Plan p{};
  p.MT = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
  p.SPS = gcd_i(G / 32, 8);
  p.ntiles = cdiv(N, kBN);
  const int64_t L = 32 * p.SPS;
  const int64_t units = K / L;
  // k per CTA is capped so that the staged activations (M rows) leave room for several CTAs per SM
  const int64_t kMaxKC = p.MT <= 2 ? int64_t(1024) : int64_t(512);
  // Split count S (a divisor of the units): within one cluster (S <= 8) the largest S giving two CTAs
  // per SM with at most kMaxKC / 2 k each (more CTAs resident per SM; on B200 the M = 1 gate|up
  // projection, 16384 x 2048, takes 11.6 us at S = 8 against 13.8 us at S = 4), else the largest S that
  // keeps >= 128 k per CTA, else the smallest that fits; only K > 8 * kMaxKC needs S > 8 (workspace
  // partials).
  int64_t S = 0;
  const int64_t smax = std::min<int64_t>(8, units);
  auto fits = [&](int64_t s) { return units % s == 0 && K / s <= kMaxKC; };
  for (int64_t s = smax; s >= 1 && !S; --s)
    if (fits(s) && K / s <= kMaxKC / 2 && p.ntiles * s >= 2 * num_sms) S = s;
  for (int64_t s = smax; s >= 1 && !S; --s)
    if (fits(s) && K / s >= 128) S = s;
  for (int64_t s = 1; s <= smax && !S; ++s)
    if (fits(s)) S = s;
  for (int64_t s = 9; s <= units && !S; ++s)
    if (fits(s)) S = s;
  if (g_w4_ovr_s > 0 && units % g_w4_ovr_s == 0 && K / g_w4_ovr_s <= kMaxKC) S = g_w4_ovr_s;
  p.S = int(S);
  p.KC = int(K / S);
  p.mode = S == 1 ? 0 : (S <= 8 ? 1 : 2);
  if (p.mode == 2 && p.ntiles > kMaxTickets) p.mode = 3;  // unsupported: reported as an error
  p.partial_bytes = p.mode == 2 ? size_t(S) * size_t(M) * size_t(N) * 4 : 0;
  return p;
}

size_t w4_workspace_bytes(const W4Plan& p) { return p.mode == 2 ? kTicketBytes + p.partial_bytes : 0; }

template <int MT, bool F16, int SPS, int PRO>
static cudaError_t launch_w4_impl(const W4SArgs& a, const W4Plan& p, size_t smem, cudaStream_t stream) {
  auto kern = w4_skinny_kernel<MT, F16, SPS, PRO>;
  if (cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(p.ntiles), unsigned(p.S));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (p.mode == 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = unsigned(p.S);
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (a.pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int MT, bool F16, int PRO>
static cudaError_t launch_w4_pro(const W4SArgs& a, const W4Plan& p, size_t smem, cudaStream_t stream) {
  switch (p.SPS) {
    case 1: return launch_w4_impl<MT, F16, 1, PRO>(a, p, smem, stream);
    case 2: return launch_w4_impl<MT, F16, 2, PRO>(a, p, smem, stream);
    case 4: return launch_w4_impl<MT, F16, 4, PRO>(a, p, smem, stream);
    default: return launch_w4_impl<MT, F16, 8, PRO>(a, p, smem, stream);
  }
}

template <int MT, bool F16>
static cudaError_t launch_w4_sps(const W4SArgs& a, const W4Plan& p, size_t smem, cudaStream_t stream) {
  if constexpr (!F16) {
    if (a.pro == kProRmsNorm) return launch_w4_pro<MT, false, kProRmsNorm>(a, p, smem, stream);
    if (a.pro == kProSwiGlu) return launch_w4_pro<MT, false, kProSwiGlu>(a, p, smem, stream);
  }
  return launch_w4_pro<MT, F16, kProPlain>(a, p, smem, stream);
}

// Streaming variant: M <= 8, plain activations (contiguous, 16-byte aligned rows), K a whole number of
// stages, the staged activations small, and far more 32-column slabs than the warps of a wave.
static bool stream_eligible(const W4SArgs& a, const W4Plan& p, int num_sms) {
  const int spst = p.SPS > kStreamSteps ? p.SPS : kStreamSteps;
  const int64_t slabs = (int64_t(a.N) + 31) / 32;
  return a.M <= 8 && a.pro == kProPlain && a.vec_x && a.vec_w && a.vec_s && a.K % (32 * spst) == 0 &&
         int64_t(a.M) * (2 * int64_t(a.K) + 64) <= 48 * 1024 && slabs >= int64_t(num_sms) * 12 * 2;
}

template <bool F16, int SPS, bool ONE, bool ARG = false>
static cudaError_t launch_stream_impl(W4SArgs a, int num_sms, cudaStream_t stream) {
  auto kern = w4_stream_kernel<F16, SPS, ONE, ARG>;
  constexpr int SPST = SPS > kStreamSteps ? SPS : kStreamSteps;
  constexpr int SEGST = SPST / SPS;
  a.xpitch = (a.K / 8) % 8 == 0 ? a.K * 2 + 64 : a.K * 2;
  a.off_sz = int((size_t(a.M) * a.xpitch + 127) / 128 * 128);  // start of the rings
  const size_t smem = size_t(a.off_sz) + 4 * kStreamRing * (SPST * 512 + SEGST * 128);
  if (cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem)) return e;
  // as many CTAs per SM as shared memory allows (at most 8), even where registers keep fewer resident: the
  // CTAs waiting for a slot take over the slabs of the first ones to finish (measured: lm_head 48.4 us with
  // 7 per SM against 53.7 us with the 6 that registers allow)
  int per_sm = int((227 * 1024) / (smem + 1024));
  per_sm = per_sm < 1 ? 1 : (per_sm > 8 ? 8 : per_sm);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(num_sms * per_sm));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (a.pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <bool ARG = false>
static cudaError_t launch_stream(bool f16, const W4SArgs& a, int sps, int num_sms, cudaStream_t stream) {
#define I4B_ST(F, O) \
  switch (sps) { \
    case 1: return launch_stream_impl<F, 1, O, ARG>(a, num_sms, stream); \
    case 2: return launch_stream_impl<F, 2, O, ARG>(a, num_sms, stream); \
    case 4: return launch_stream_impl<F, 4, O, ARG>(a, num_sms, stream); \
    default: return launch_stream_impl<F, 8, O, ARG>(a, num_sms, stream); \
  }
  const bool one = a.M == 1;
  if (f16) {
    if (one) I4B_ST(true, true);
    I4B_ST(true, false);
  }
  if (one) I4B_ST(false, true);
  I4B_ST(false, false);
#undef I4B_ST
}

// Upper bound of the stream kernel's warps (its grid is SMs x at most 8 CTAs of 4 warps).
static int64_t stream_max_warps(int sms) { return int64_t(sms) * 8 * 4; }

// ---- register-streaming GEMV (M <= 8): plan and launch

struct W4GPlan {
  int WN, WK, S, KC, KW, sz_rows, D;
  size_t smem;
  bool ok;
};

// Shared memory of one CTA: scales + zeros [2][rows][32 WN] fp16 | activations [M][pitch] | partials [WK][M][32 WN].
static size_t w4g_smem(int M, int WN, int WK, int KC, int sz_rows, int* xpitch, int* off_x, int* off_part) {
  const int BN = 32 * WN;
  const size_t sz = size_t(2) * sz_rows * BN * 2;
  *xpitch = (KC / 8) % 8 == 0 ? KC * 2 + 64 : KC * 2;  // token rows 4 mod 8 16-byte units apart
  *off_x = int((sz + 127) / 128 * 128);
  *off_part = int((size_t(*off_x) + size_t(M) * *xpitch + 15) / 16 * 16);
  return size_t(*off_part) + size_t(WK) * M * BN * 4;
}

// K is cut into segments of L = 32 * gcd(G / 32, 8) k; a warp owns KW = K / (S WK) consecutive k, a whole number
// of segments.  The CTA has WK = 8 warps along K (fewer when K holds fewer segments); the cluster split S is the
// smallest that gives every SM a CTA, as long as a warp keeps at least one segment.
static W4GPlan plan_w4_gemv(int64_t M, int64_t N, int64_t K, int G, int sms) {
  W4GPlan p{};
  const int SPS = gcd_i(G / 32, 8);
  const int64_t L = 32 * SPS;
  const int64_t units = K / L;
  const int64_t ncg = cdiv(N, 32);
  p.WN = 1;
  int WK = 8;
  while (WK > 1 && units % WK) WK >>= 1;
  if (g_w4_ovr_wk > 0 && g_w4_ovr_wk <= 8 && units % g_w4_ovr_wk == 0) WK = g_w4_ovr_wk;
  int S = 1;
  while (S < 8 && ncg * S < sms && units % (int64_t(2 * S) * WK) == 0) S *= 2;
  if (g_w4_ovr_gs > 0 && g_w4_ovr_gs <= 8 && units % (int64_t(g_w4_ovr_gs) * WK) == 0) S = g_w4_ovr_gs;
  p.WK = WK;
  p.S = S;
  p.KC = int(K / S);
  p.KW = p.KC / WK;
  p.sz_rows = p.KC >= G ? p.KC / G + 1 : 2;  // groups a K slice can touch
  p.D = p.KW / 32 >= 8 ? 8 : 4;
  if (g_w4_ovr_kernel == 4) p.D = 4;
  if (g_w4_ovr_kernel == 5) p.D = 8;
  int xp, ox, op;
  p.smem = w4g_smem(int(M), p.WN, p.WK, p.KC, p.sz_rows, &xp, &ox, &op);
  p.ok = M <= 8 && units % (int64_t(S) * WK) == 0 && p.smem <= 200 * 1024 && K <= INT32_MAX;
  return p;
}

template <bool F16, int SPS, int PRO, int D, bool ARG = false>
static cudaError_t launch_gemv_impl(const W4SArgs& a, const W4GPlan& p, cudaStream_t stream) {
  auto kern = w4_gemv_kernel<F16, SPS, PRO, D, ARG>;
  if (cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), p.smem)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(cdiv(a.N, 32 * p.WN)), unsigned(p.S));
  cfg.blockDim = dim3(unsigned(32 * p.WN * p.WK));
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (p.S > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = unsigned(p.S);
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (a.pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <bool F16, int PRO, int D, bool ARG = false>
static cudaError_t launch_gemv_sps(const W4SArgs& a, const W4GPlan& p, int sps, cudaStream_t stream) {
  switch (sps) {
    case 1: return launch_gemv_impl<F16, 1, PRO, D, ARG>(a, p, stream);
    case 2: return launch_gemv_impl<F16, 2, PRO, D, ARG>(a, p, stream);
    case 4: return launch_gemv_impl<F16, 4, PRO, D, ARG>(a, p, stream);
    default: return launch_gemv_impl<F16, 8, PRO, D, ARG>(a, p, stream);
  }
}

template <int D>
static cudaError_t launch_gemv_d(bool f16, const W4SArgs& a, const W4GPlan& p, int sps, cudaStream_t stream) {
  if (f16) return launch_gemv_sps<true, kProPlain, D>(a, p, sps, stream);
  if (a.pro == kProRmsNorm) return launch_gemv_sps<false, kProRmsNorm, D>(a, p, sps, stream);
  if (a.pro == kProSwiGlu) return launch_gemv_sps<false, kProSwiGlu, D>(a, p, sps, stream);
  return launch_gemv_sps<false, kProPlain, D>(a, p, sps, stream);
}

// The register-streaming kernel takes M <= 8 without the tensor-parallel epilogue, with 16-byte aligned packed
// words and scale / zero rows (N % 8 == 0).
static bool gemv_eligible(const W4SArgs& a, const W4GPlan& p) {
  const auto addr = [](const void* ptr) { return reinterpret_cast<uintptr_t>(ptr); };
  return p.ok && a.M <= 8 && a.ar_world <= 1 && a.N % 8 == 0 && a.vec_w && addr(a.sc) % 16 == 0 &&
         addr(a.zr) % 16 == 0 && a.ssg % 8 == 0;
}

// ---- slab-streaming GEMV (M <= 8): plan and launch

struct W4SlabPlan {
  int P, per_sm, grid, sms;
  size_t smem;
  bool ok;
};

// Wide matrices only (at least two slabs per SM; narrower ones go to the register-streaming GEMV, whose
// cluster split spreads few slabs over all SMs).  P: the smallest split (1, 2, 4 or 8) giving kSlabWarpsPerSm
// busy warps per SM; the grid covers the slab groups, at most as many CTAs as are resident at once.
constexpr int kSlabWarpsPerSm = 32;

static W4SlabPlan plan_w4_slab(const W4SArgs& a, int sps, int sms) {
  W4SlabPlan p{};
  const int spst = sps > kStreamSteps ? sps : kStreamSteps;
  const int64_t slabs = cdiv(a.N, 32);
  p.P = 8;
  for (int P : {1, 2, 4, 8})
    if (slabs * P >= int64_t(kSlabWarpsPerSm) * sms) {
      p.P = P;
      break;
    }
  if (g_w4_ovr_kernel == 6 && (g_w4_ovr_wk == 1 || g_w4_ovr_wk == 2 || g_w4_ovr_wk == 4 || g_w4_ovr_wk == 8))
    p.P = g_w4_ovr_wk;
  const int NW = p.P > 4 ? p.P : 4;
  const int xpitch = (a.K / 8) % 8 == 0 ? a.K * 2 + 64 : a.K * 2;
  const size_t x_bytes = (size_t(a.M) * xpitch + 127) / 128 * 128;
  const size_t part_bytes = p.P > 1 ? size_t(2) * NW * 256 * 4 : 0;
  p.smem = x_bytes + part_bytes + NW * kStreamRing * (size_t(spst) * 512 + (spst / sps) * 128);
  int per_sm = int((227 * 1024) / (p.smem + 1024));
  p.per_sm = per_sm < 1 ? 1 : (per_sm > 8 ? 8 : per_sm);
  const int64_t groups = cdiv(slabs, NW / p.P);
  p.grid = int(groups);  // slab groups; the launch caps the grid at what is resident and balances it
  p.sms = sms;
  // Wide matrices (two slabs per SM or more) stream best as slabs; so do short ones (K <= 2048: a warp's
  // share of a slab is at most 256 columns of K at P = 8) as long as there are slabs for half the SMs, or one
  // or two tokens.  Measured at M = 1 (us): qkv 3072x2048 4.1 against 5.2 for the register kernel, o
  // 2048x2048 3.8 against 4.2; at M = 8 the register kernel keeps o (4.8 against 5.7) and long K (down
  // 2048x8192: 7.5 against 11.2 at M = 1).
  const bool shape_ok = slabs >= 2 * int64_t(sms) || (a.K <= 2048 && (a.M <= 2 || 2 * slabs >= sms));
  p.ok = a.M <= 8 && a.ar_world <= 1 && a.vec_w && a.vec_s && a.K % (p.P * 32 * spst) == 0 &&
         p.smem <= 200 * 1024 && (shape_ok || g_w4_ovr_kernel == 6);
  return p;
}

template <bool F16, int SPS, int PRO, int P>
static cudaError_t launch_slab_impl(const W4SArgs& a, const W4SlabPlan& p, cudaStream_t stream) {
  auto kern = w4_slab_kernel<F16, SPS, PRO, P>;
  if (cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), p.smem)) return e;
  // a persistent grid: no more CTAs than can be resident at once (registers and shared memory)
  constexpr int NW = P > 4 ? P : 4;
  int per_sm = 0;
  if (cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32 * NW, p.smem)) return e;
  per_sm = std::max(1, std::min(per_sm, p.per_sm));
  // every resident CTA (an equal number of slab groups per CTA measured slower: gate|up 13.2 against 9.3 us),
  // unless the tuning hook asks for the balanced grid (splits == 2)
  const int64_t resident = int64_t(p.sms) * per_sm, groups = p.grid;
  int64_t grid = std::min(groups, resident);
  if (g_w4_ovr_kernel == 6 && g_w4_ovr_gs == 2) grid = cdiv(groups, cdiv(groups, resident));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(32 * NW);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (a.pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <bool F16, int PRO, int P>
static cudaError_t launch_slab_sps(const W4SArgs& a, const W4SlabPlan& p, int sps, cudaStream_t stream) {
  switch (sps) {
    case 1: return launch_slab_impl<F16, 1, PRO, P>(a, p, stream);
    case 2: return launch_slab_impl<F16, 2, PRO, P>(a, p, stream);
    case 4: return launch_slab_impl<F16, 4, PRO, P>(a, p, stream);
    default: return launch_slab_impl<F16, 8, PRO, P>(a, p, stream);
  }
}

template <int P>
static cudaError_t launch_slab_p(bool f16, const W4SArgs& a, const W4SlabPlan& p, int sps, cudaStream_t stream) {
  if (f16) return launch_slab_sps<true, kProPlain, P>(a, p, sps, stream);
  if (a.pro == kProRmsNorm) return launch_slab_sps<false, kProRmsNorm, P>(a, p, sps, stream);
  if (a.pro == kProSwiGlu) return launch_slab_sps<false, kProSwiGlu, P>(a, p, sps, stream);
  return launch_slab_sps<false, kProPlain, P>(a, p, sps, stream);
}

static cudaError_t launch_slab(bool f16, W4SArgs a, const W4SlabPlan& p, int sps, cudaStream_t stream) {
  a.xpitch = (a.K / 8) % 8 == 0 ? a.K * 2 + 64 : a.K * 2;
  a.off_part = int((size_t(a.M) * a.xpitch + 127) / 128 * 128);
  const int NW = p.P > 4 ? p.P : 4;
  a.off_sz = a.off_part + (p.P > 1 ? 2 * NW * 256 * 4 : 0);  // start of the rings
  switch (p.P) {
    case 1: return launch_slab_p<1>(f16, a, p, sps, stream);
    case 2: return launch_slab_p<2>(f16, a, p, sps, stream);
    case 4: return launch_slab_p<4>(f16, a, p, sps, stream);
    default: return launch_slab_p<8>(f16, a, p, sps, stream);
  }
}

cudaError_t launch_w4(bool f16, const void* x, int64_t M, int64_t K, int64_t sxm, int64_t sxk, const int32_t* qw,
                      int64_t N, int64_t sqk, const uint16_t* sc, const uint16_t* zr, int64_t ssg, int G, void* y,
                      int64_t sym, void* ws, const W4Plan& p, bool pdl, cudaStream_t stream, const W4Prologue* pro,
                      const W4AllReduce* ar) {
  if (p.mode == 3) return cudaErrorInvalidConfiguration;
  W4SArgs a{};
  if (pro) {
    a.pro = pro->kind;
    a.delta = static_cast<const uint16_t*>(pro->delta);
    a.norm_w = static_cast<const uint16_t*>(pro->norm_weight);
    a.resid_out = static_cast<uint16_t*>(pro->resid_out);
    a.eps = pro->eps;
  }
  a.x = static_cast<const uint16_t*>(x);
  a.sxm = sxm;
  a.sxk = sxk;
  a.qw = reinterpret_cast<const uint32_t*>(qw);
  a.sqk = sqk;
  a.sc = sc;
  a.zr = zr;
  a.ssg = ssg;
  a.y = static_cast<uint16_t*>(y);
  a.sym = sym;
  a.M = int(M);
  a.N = int(N);
  a.K = int(K);
  a.G = G;
  a.S = p.S;
  a.KC = p.KC;
  a.mode = p.mode;
  a.pdl = pdl ? 1 : 0;
  if (p.mode == 2) {
    a.tickets = static_cast<unsigned int*>(ws);
    a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kTicketBytes);
  }
  const auto addr = [](const void* ptr) { return reinterpret_cast<uintptr_t>(ptr); };
  a.vec_w = addr(qw) % 16 == 0 && sqk % 4 == 0 && N % 4 == 0;
  a.vec_s = addr(sc) % 4 == 0 && addr(zr) % 4 == 0 && ssg % 2 == 0 && N % 4 == 0;
  a.vec_x = addr(x) % 16 == 0 && sxk == 1 && (sxm % 8 == 0 || M == 1);
  const int L = 32 * p.SPS;
  a.gpl = G / L;  // L divides G
  a.gpl_shift = (a.gpl & (a.gpl - 1)) == 0 ? __builtin_ctz(unsigned(a.gpl)) : -1;
  if (ar && ar->world > 1) {
    if (p.mode != 0 && p.mode != 1) return cudaErrorInvalidConfiguration;
    for (int q = 0; q < kArMaxRanks; ++q) a.ar_buf[q] = static_cast<uint8_t*>(ar->buffers[q]);
    a.ar_cap = ar->capacity;
    a.ar_world = ar->world;
    a.ar_rank = ar->rank;
  }
  int sms = 0, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // kernel choice for M <= 8: the slab-streaming GEMV, else the register-streaming one, unless the tuning hook
  // asks for another
  const bool ovr_reg = g_w4_ovr_kernel == 1 || g_w4_ovr_kernel == 4 || g_w4_ovr_kernel == 5;
  // one token over a very wide matrix (an lm_head): the one-warp-per-slab stream measured fastest
  if (sms > 0 && g_w4_ovr_kernel == 0 && a.M == 1 && a.ar_world <= 1 && stream_eligible(a, p, sms))
    return launch_stream(f16, a, p.SPS, sms, stream);
  if (sms > 0 && (g_w4_ovr_kernel == 0 || g_w4_ovr_kernel == 6)) {
    const W4SlabPlan sp = plan_w4_slab(a, p.SPS, sms);
    if (sp.ok) return launch_slab(f16, a, sp, p.SPS, stream);
  }
  if (sms > 0 && (g_w4_ovr_kernel == 0 || ovr_reg)) {
    const W4GPlan gp = plan_w4_gemv(M, N, K, G, sms);
    if (gemv_eligible(a, gp)) {
      a.WN = gp.WN;
      a.WK = gp.WK;
      a.KW = gp.KW;
      a.KC = gp.KC;
      a.S = gp.S;
      a.sz_rows = gp.sz_rows;
      int xp, ox, op;
      w4g_smem(a.M, gp.WN, gp.WK, gp.KC, gp.sz_rows, &xp, &ox, &op);
      a.xpitch = xp;
      a.off_sz = 0;
      a.off_x = ox;
      a.off_part = op;
      return gp.D == 8 ? launch_gemv_d<8>(f16, a, gp, p.SPS, stream) : launch_gemv_d<4>(f16, a, gp, p.SPS, stream);
    }
  }
  if (sms > 0 && a.ar_world <= 1 && g_w4_ovr_kernel != 2 && stream_eligible(a, p, sms))
    return launch_stream(f16, a, p.SPS, sms, stream);
  const int spst = p.SPS > 4 ? p.SPS : 4;  // steps per stage, as in the kernel
  const int nsteps = p.KC / 32;
  a.nstages = (nsteps + spst - 1) / spst;
  // token rows of x in shared memory: 4 mod 8 16-byte units apart (conflict-free fragment reads)
  const int kcp = a.nstages * spst * 32;  // padded k per CTA
  a.xpitch = (kcp / 8) % 8 == 0 ? kcp * 2 + 64 : kcp * 2;
  size_t off = size_t(a.nstages) * spst * 4 * 32 * 16;
  a.off_sz = int(off);
  off += size_t(a.nstages) * (spst / p.SPS) * 4 * 8 * 16;
  a.off_x = int(off);
  off += size_t(M) * a.xpitch;
  a.off_part = int(off);
  off += size_t(M) * kBN * 4;
  const size_t smem = off;
  switch (p.MT) {
    case 1: return f16 ? launch_w4_sps<1, true>(a, p, smem, stream) : launch_w4_sps<1, false>(a, p, smem, stream);
    case 2: return f16 ? launch_w4_sps<2, true>(a, p, smem, stream) : launch_w4_sps<2, false>(a, p, smem, stream);
    default: return f16 ? launch_w4_sps<4, true>(a, p, smem, stream) : launch_w4_sps<4, false>(a, p, smem, stream);
  }
}

// ---- greedy choice fused into the M <= 8 GEMV (the lm_head of a greedy decode step)

static W4GPlan plan_w4_argmax(int64_t M, int64_t N, int64_t K, int G, int sms) {
  W4GPlan p = plan_w4_gemv(M, N, K, G, sms);
  if (p.S != 1) {  // one CTA owns all of K for its columns, so each tile's logits are final in that CTA
    p.S = 1;
    p.KC = int(K);
    p.KW = p.KC / p.WK;
    p.sz_rows = p.KC >= G ? p.KC / G + 1 : 2;
    p.D = p.KW / 32 >= 8 ? 8 : 4;
    int xp, ox, op;
    p.smem = w4g_smem(int(M), p.WN, p.WK, p.KC, p.sz_rows, &xp, &ox, &op);
    p.ok = p.ok && p.smem <= 200 * 1024;
  }
  return p;
}

size_t w4_argmax_workspace_bytes(int64_t M, int64_t N, int64_t K, int G, int sms) {
  const W4GPlan p = plan_w4_argmax(M, N, K, G, sms);
  if (!p.ok) return 0;
  // candidates: one per column tile (register-streaming form) or per warp (streaming form), whichever is more
  const int64_t cands = std::max<int64_t>(cdiv(N, 32 * p.WN), stream_max_warps(sms));
  return kTicketBytes + size_t(cands) * size_t(M) * sizeof(float2);
}

cudaError_t launch_w4_argmax(bool f16, const void* x, int64_t M, int64_t K, int64_t sxm, const int32_t* qw, int64_t N,
                             int64_t sqk, const uint16_t* sc, const uint16_t* zr, int64_t ssg, int G, void* y,
                             int64_t sym, int64_t* out, void* ws, bool pdl, int sms, cudaStream_t stream) {
  const W4GPlan p = plan_w4_argmax(M, N, K, G, sms);
  W4SArgs a{};
  a.x = static_cast<const uint16_t*>(x);
  a.sxm = sxm;
  a.sxk = 1;
  a.qw = reinterpret_cast<const uint32_t*>(qw);
  a.sqk = sqk;
  a.sc = sc;
  a.zr = zr;
  a.ssg = ssg;
  a.y = static_cast<uint16_t*>(y);
  a.sym = sym;
  a.M = int(M);
  a.N = int(N);
  a.K = int(K);
  a.G = G;
  a.pdl = pdl ? 1 : 0;
  const auto addr = [](const void* ptr) { return reinterpret_cast<uintptr_t>(ptr); };
  a.vec_w = addr(qw) % 16 == 0 && sqk % 4 == 0 && N % 4 == 0;
  a.vec_x = addr(x) % 16 == 0 && (sxm % 8 == 0 || M == 1);
  const int SPS = gcd_i(G / 32, 8);
  a.gpl = G / (32 * SPS);
  a.gpl_shift = (a.gpl & (a.gpl - 1)) == 0 ? __builtin_ctz(unsigned(a.gpl)) : -1;
  a.tickets = static_cast<unsigned int*>(ws);
  a.cand = reinterpret_cast<float2*>(static_cast<uint8_t*>(ws) + kTicketBytes);
  a.amax_out = out;
  {  // a very wide head: the streaming kernel (the fastest form there), greedy choice in its epilogue
    const auto addr = [](const void* ptr) { return reinterpret_cast<uintptr_t>(ptr); };
    a.vec_s = addr(sc) % 4 == 0 && addr(zr) % 4 == 0 && ssg % 2 == 0 && N % 4 == 0;
    W4Plan wp{};
    wp.SPS = SPS;
    if (g_w4_ovr_kernel != 1 && stream_eligible(a, wp, sms)) return launch_stream<true>(f16, a, SPS, sms, stream);
  }
  if (!gemv_eligible(a, p)) return cudaErrorInvalidConfiguration;
  a.WN = p.WN;
  a.WK = p.WK;
  a.KW = p.KW;
  a.KC = p.KC;
  a.S = 1;
  a.sz_rows = p.sz_rows;
  int xp, ox, op;
  w4g_smem(a.M, p.WN, p.WK, p.KC, p.sz_rows, &xp, &ox, &op);
  a.xpitch = xp;
  a.off_sz = 0;
  a.off_x = ox;
  a.off_part = op;
  if (p.D == 8)
    return f16 ? launch_gemv_sps<true, kProPlain, 8, true>(a, p, SPS, stream)
               : launch_gemv_sps<false, kProPlain, 8, true>(a, p, SPS, stream);
  return f16 ? launch_gemv_sps<true, kProPlain, 4, true>(a, p, SPS, stream)
             : launch_gemv_sps<false, kProPlain, 4, true>(a, p, SPS, stream);
}

// ------------------------------------------------------------------ greedy token over tensor-parallel ranks

namespace {
struct ArgmaxArArgs {
  const uint16_t* x;  // [rows] rows of this rank's logits, bf16, n columns, row stride sx
  int64_t sx, n, offset;
  int64_t* out;       // [rows] global index of the first maximum over all ranks
  uint8_t* ar_buf[kArMaxRanks];
  int64_t ar_cap;
  int ar_world, ar_rank;
};

// One CTA per row: this rank's first maximum (value, global index), exchanged through the peer buffers as
// two fp32 words; the ranks' candidates are compared in rank order with a strict '>', so equal maxima go
// to the lower rank, whose columns come first: the result is torch.argmax over the concatenated row.
__global__ void __launch_bounds__(1024) argmax_allreduce_kernel(const ArgmaxArArgs a) {
  __shared__ uint32_t s_ep;
  const int row = blockIdx.x;
  float best;
  int64_t bi;
  block_row_argmax(a.x + int64_t(row) * a.sx, a.n, &best, &bi);
  const uint32_t ep = ar_epoch(a, &s_ep);
  if (threadIdx.x == 0) {
    const int gi = bi < a.n ? int(a.offset + bi) : -1;  // -1: nothing above -inf on this rank
    ar_push(a, ep, 2 * int64_t(row), best);
    ar_push(a, ep, 2 * int64_t(row) + 1, __int_as_float(gi));
  }
  if (threadIdx.x == 0) {
    float bv = 0.0f;
    int gi = -1;
    for (int q = 0; q < a.ar_world; ++q) {
      const float v = ar_take(a, ep, q, 2 * int64_t(row));
      const int i = __float_as_int(ar_take(a, ep, q, 2 * int64_t(row) + 1));
      if (i >= 0 && (gi < 0 || v > bv)) {
        bv = v;
        gi = i;
      }
    }
    a.out[row] = gi < 0 ? 0 : gi;
  }
  ar_finish(a, ep);
}
}  // namespace

cudaError_t launch_argmax_allreduce(const uint16_t* x, int64_t rows, int64_t n, int64_t sx, int64_t offset,
                                    int64_t* out, const W4AllReduce& ar, cudaStream_t stream) {
  ArgmaxArArgs a{};
  a.x = x;
  a.sx = sx;
  a.n = n;
  a.offset = offset;
  a.out = out;
  for (int q = 0; q < kArMaxRanks; ++q) a.ar_buf[q] = static_cast<uint8_t*>(ar.buffers[q]);
  a.ar_cap = ar.capacity;
  a.ar_world = ar.world;
  a.ar_rank = ar.rank;
  argmax_allreduce_kernel<<<unsigned(rows), 1024, 0, stream>>>(a);
  return cudaGetLastError();
}

unsigned int read_w4_error(bool clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_w4_err, sizeof(v)) != cudaSuccess) return 0;
  if (clear && v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_w4_err, &z, sizeof(z));
  }
  return v;
}

}  // namespace i4b
