// W4A16 GEMM on the 5th-generation tensor cores with the dequantized weights held in TMEM.
//
// Replaces the reference's large-M Triton path _matmul_kernel (int4_triton/gemm.py:74-157, launched at
// gemm.py:270-296) and, from 9 tokens on, its split-K small-M path (gemm.py:160-260).
// y[M, N] = x[M, K] @ W_hat[N, K]^T with W_hat = bf16_rn((q - z) * s) (int4_triton/gemm.py:137-140).
//
// The MMA is computed transposed, y^T tile = W_hat tile (A) x x^T tile (B):
//   A  128 weight rows x 16 k per instruction, read from TMEM (tcgen05.mma ... [a-tmem]): the dequant
//      warps write each 128 x 64 k-block of W_hat straight into a 4-slot TMEM ring with tcgen05.st, so
//      dequantized weights never pass through shared memory;
//   B  NT tokens x 16 k from shared memory (the TMA-loaded activation tile, K-major, 128-byte swizzle);
//   D  128 x NT fp32 accumulator in TMEM (lane = weight row, column = token).
// Shared-memory traffic per k-block is the activation tile written by TMA and read once by the MMAs plus
// the 4 KB of packed weights; keeping the bf16 weight tile out of shared memory is what lets the tensor pipe
// run instead of waiting on shared-memory bandwidth (which an A/B-from-shared design saturates first).
//
// One CTA computes a 128-weight-row x NT-token tile over k-blocks [kb0, kb1) (a K split when ksplit > 1).
// 18 warps:
//   warp 0      TMA producer: per 64-wide k-block the activation tile (NT x 64), the packed words
//               (8 k8-rows x 128 int32) and two group rows of scales and zeros;
//   warp 1      allocates TMEM (accumulator + A ring) and, from one thread, issues four
//               tcgen05.mma.kind::f16 per k-block, then tcgen05.commit frees the stage and the A slot;
//   warps 2..    dequantize in groups of four (four groups for 256-token tiles, two otherwise): group
//               h = (w - 2) / 4 takes every GROUPS-th k-block, and warp w of it owns TMEM lane quarter w % 4
//               (weight rows 32 (w % 4) + lane); then all of them read the accumulator back with
//               tcgen05.ld and store y (or fp32 partials of the K split);
//   last warp   weight producer: per two k-blocks the packed words and one box of scales and zeros.
// Every wait is bounded; on expiry the kernel records I4B_DEVERR_WAIT_TIMEOUT, drains its own TMA copies,
// frees TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace i4b {

static __device__ unsigned int g_w4t_err = 0;

// Build-time tuning knobs: A slots in TMEM, and whether the dequant warps wait with a suspend hint.
#ifndef I4B_W4T_NA
#define I4B_W4T_NA 8
#endif
#ifndef I4B_W4T_SLEEP
#define I4B_W4T_SLEEP 1
#endif

template <int NT>
struct W4tCfg {
  static constexpr int BF = 128, BK = 64;  // weight rows (the MMA's M) and k per k-block
  // Token tiles up to 128 run two CTAs per SM (each with two dequant groups, 256 TMEM columns and at most
  // 113 KB of shared memory): a pipeline step of the control warps costs a few hundred cycles whatever its
  // size, so two independent pipelines per SM double the steps in flight.  256-token tiles need all of TMEM.
  static constexpr int CPS = NT <= 128 ? 2 : 1;        // CTAs per SM
  static constexpr int GROUPS = CPS == 2 ? 2 : 4;      // dequant groups of four warps
  static constexpr int DQ_WARPS = 4 * GROUPS;
  static constexpr int THREADS = 32 * (3 + DQ_WARPS);  // X producer, MMA, dequant warps, W producer
  static constexpr int X_BYTES = NT * BK * 2;          // activation tile: NT rows of 128 B
  // weight stage: two k-blocks (128 k) of packed words, and scales + zeros of up to 4 groups
  static constexpr int P_BYTES = 16 * BF * 4;
  static constexpr int SZ_ROWS = 4;
  static constexpr int SZ_BYTES = 2 * SZ_ROWS * BF * 2;
  static constexpr int W_BYTES = P_BYTES + SZ_BYTES;
  static constexpr int SX = NT >= 256 ? 4 : NT >= 128 ? 4 : NT >= 64 ? 6 : 8;  // activation stages
  static constexpr int SW = NT >= 256 ? 6 : NT >= 128 ? 4 : NT >= 64 ? 5 : 7;  // weight stages
  static constexpr int NA = CPS == 2 ? 4 : I4B_W4T_NA;  // A slots (k-blocks) in TMEM
  static constexpr int A_COL = NT < 32 ? 32 : NT;      // first TMEM column of the A ring
  static constexpr int A_SLOT_COLS = BK / 2;           // 64 16-bit values per row = 32 columns
  static constexpr int TMEM_COLS = (A_COL + NA * A_SLOT_COLS) <= 256 ? 256 : 512;
  static constexpr int BAR_BYTES = (2 * SX + 2 * SW + 2 * NA + 1) * 8 + 8;
  static constexpr size_t SMEM = 1024 + size_t(SX) * X_BYTES + size_t(SW) * W_BYTES + BAR_BYTES;
  static_assert(X_BYTES % 1024 == 0, "activation stages keep the 1024-byte swizzle alignment");
  static_assert(SMEM <= (CPS == 2 ? 113 * 1024 : 227 * 1024), "shared memory");
  static_assert(NA % GROUPS == 0, "each dequant group owns NA / GROUPS slots");
  static_assert(CPS == 1 || TMEM_COLS == 256, "two CTAs per SM share TMEM");
  static_assert(A_COL + NA * A_SLOT_COLS <= TMEM_COLS && TMEM_COLS <= 512, "TMEM budget");
  static_assert(NT % 16 == 0 && NT >= 16 && NT <= 256, "MMA N for M = 128");
};

// 8 nibbles of one packed word -> 8 dequantized 16-bit values in k order, packed two per 32 bits
// (low half = even k): exactly the TMEM layout of one A row over 8 k.
template <bool F16>
__device__ __forceinline__ uint4 w4t_dequant_word(uint32_t w, const DqParams& p) {
  uint32_t r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t q = and_or(w >> (4 * i), 0x000F000Fu, F16 ? 0x64006400u : 0x43004300u);  // (q_i, q_{i+4})
    uint32_t d;
    if constexpr (F16) {
      asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(q), "r"(p.zz));
      asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r[i]) : "r"(d), "r"(p.shi));
    } else {
      uint32_t pl;
      asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(q), "r"(p.zz));
      asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(pl) : "r"(d), "r"(p.slo));
      asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r[i]) : "r"(d), "r"(p.shi), "r"(pl));
    }
  }
  return make_uint4(__byte_perm(r[0], r[1], 0x5410), __byte_perm(r[2], r[3], 0x5410),
                    __byte_perm(r[0], r[1], 0x7632), __byte_perm(r[2], r[3], 0x7632));
}

// 32 lanes x 32 bit, 16 consecutive columns from this thread's registers (the warp's lane quarter).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint4& a, const uint4& b, const uint4& c,
                                                   const uint4& d) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w), "r"(c.x), "r"(c.y), "r"(c.z),
      "r"(c.w), "r"(d.x), "r"(d.y), "r"(d.z), "r"(d.w)
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (bf16 or fp16 operands, fp32 accumulator).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// One lane of a converged warp (elect.sync).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\telect.sync r|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}
// Bounded wait by a whole warp, with one verdict for all its lanes.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

template <bool F16, int NT>
__global__ void __launch_bounds__(W4tCfg<NT>::THREADS, W4tCfg<NT>::CPS)
    w4t_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_sz, int sz_swap, int M, int N, int K, int G,
                    uint16_t* __restrict__ y, int64_t sym, int ksplit, float* __restrict__ partials,
                    unsigned int* __restrict__ tickets) {
  using C = W4tCfg<NT>;
  constexpr int SX = C::SX, SW = C::SW, NA = C::NA;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  // [SX activation stages][SW weight stages: P | scales and zeros][barriers]
  uint8_t* xring = smem;
  uint8_t* wring = xring + SX * C::X_BYTES;
  uint64_t* xfull = reinterpret_cast<uint64_t*>(wring + SW * C::W_BYTES);
  uint64_t* xempty = xfull + SX;   // MMA commit: the activation stage is read
  uint64_t* wfull = xempty + SX;
  uint64_t* wempty = wfull + SW;   // dequant arrivals: the weight stage is read
  uint64_t* aready = wempty + SW;  // A slot dequantized into TMEM (the four warps of a group)
  uint64_t* afree = aready + NA;   // A slot no longer read by the MMAs
  uint64_t* tfull = afree + NA;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  auto sX = [&](int s) { return xring + s * C::X_BYTES; };
  auto sW = [&](int s) { return wring + s * C::W_BYTES; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * C::BF, m0 = blockIdx.y * NT;
  const int KBT = (K + C::BK - 1) / C::BK;
  const int kb0 = int((int64_t(blockIdx.z) * KBT) / ksplit), kb1 = int((int64_t(blockIdx.z + 1) * KBT) / ksplit);
  const int KB = kb1 - kb0;  // k-blocks of this CTA; weight stage j holds its k-blocks 2j and 2j + 1
  const int NWS = (KB + 1) / 2;
  __shared__ int s_last;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < SW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 8);  // the two dequant groups (four warps each) of its two k-blocks
    }
    for (int b = 0; b < NA; ++b) {
      mbar_init(&aready[b], 4);
      mbar_init(&afree[b], 1);
    }
    mbar_init(tfull, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm_x);
  if (warp == 2 + C::DQ_WARPS && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_sz);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  // The control warps (activation producer, weight producer, MMA) run their loops on all 32 lanes, so that
  // stage indices, coordinates and descriptors are warp-uniform values, and issue each TMA / tcgen05
  // instruction from one elected lane.
  if (warp == 0) {
    // activation producer: one 64-k tile per k-block
    int issued = 0;
    for (int kbl = 0; kbl < KB; ++kbl) {
      const int s = kbl % SX, u = kbl / SX;
      if (kbl >= SX && !warp_wait(&xempty[s], (u - 1) & 1)) { ok = false; break; }
      if (elect_one()) {
        mbar_arrive_expect_tx(&xfull[s], C::X_BYTES);
        tma_load_2d(sX(s), &tm_x, &xfull[s], (kb0 + kbl) * C::BK, m0);
      }
      __syncwarp();
      ++issued;
    }
    for (int s = 0; s < SX && s < issued; ++s) {  // never leave a bulk copy in flight
      const int last = ((issued - 1 - s) / SX) * SX + s;
      if (!warp_wait(&xfull[s], (last / SX) & 1)) ok = false;
    }
    // Nor an MMA-completion arrival: tcgen05.commit arrives on its barrier asynchronously, and one landing after
    // the CTA has exited would write into the shared memory of the next CTA on this SM.  So wait for the
    // release of every stage's last use.
    for (int s = 0; ok && s < SX && s < issued; ++s) {
      const int last = ((issued - 1 - s) / SX) * SX + s;
      if (!warp_wait(&xempty[s], (last / SX) & 1)) ok = false;
    }
  } else if (warp == 2 + C::DQ_WARPS) {
    // weight producer: per weight stage the packed words of 128 k (16 rows) and one 3-D box of scales and
    // zeros (SZ_ROWS group rows of both tensors)
    int issued = 0;
    for (int j = 0; j < NWS; ++j) {
      const int s = j % SW, u = j / SW;
      if (j >= SW && !warp_wait(&wempty[s], (u - 1) & 1)) { ok = false; break; }
      const int k_begin = (kb0 + 2 * j) * C::BK;
      if (elect_one()) {
        mbar_arrive_expect_tx(&wfull[s], C::W_BYTES);
        tma_load_2d(sW(s), &tm_w, &wfull[s], n0, k_begin / 8);
        tma_load_3d(sW(s) + C::P_BYTES, &tm_sz, &wfull[s], n0, k_begin / G, 0);
      }
      __syncwarp();
      ++issued;
    }
    for (int s = 0; s < SW && s < issued; ++s) {
      const int last = ((issued - 1 - s) / SW) * SW + s;
      if (!warp_wait(&wfull[s], (last / SW) & 1)) ok = false;
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = umma_idesc_f16(F16 ? 0 : 1, C::BF, NT);
    for (int kbl = 0; kbl < KB; ++kbl) {
      const int s = kbl % SX, u = kbl / SX, b = kbl % NA;
      if (!warp_wait(&xfull[s], u & 1)) { ok = false; break; }
      if (!warp_wait(&aready[b], (kbl / NA) & 1)) { ok = false; break; }
      tc_fence_after();
      const uint64_t bdesc = umma_desc_sw128(smem_u32(sX(s)));
      const uint32_t acol = tmem + uint32_t(C::A_COL + b * C::A_SLOT_COLS);
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < C::BK / 16; ++kk)
          umma_f16_ts(tmem, acol + uint32_t(8 * kk), bdesc + 2 * kk, idesc, (kbl | kk) != 0 ? 1u : 0u);
        umma_commit(&xempty[s]);
        umma_commit(&afree[b]);
      }
      __syncwarp();
    }
    if (elect_one()) umma_commit(tfull);  // also on the error path: completes once the issued MMAs are done
    __syncwarp();
  } else {
    // Dequant warps in GROUPS groups of four: group h takes k-blocks h, h + GROUPS, ... (several dequant
    // passes in flight: one warp's pass -- wait, dequantize, tcgen05.st, wait::st, arrive -- is a latency
    // chain longer than a k-block's MMAs); within a group, warp q owns TMEM lane quarter q (weight rows
    // 32 q + lane) and all eight packed words of the row.
    const int q = warp & 3, h = (warp - 2) >> 2;
    const int nl = 32 * q + lane;
    const uint32_t lane_base = uint32_t(32 * q) << 16;
    const int zoff = sz_swap ? 0 : C::SZ_ROWS * C::BF, soff = sz_swap ? C::SZ_ROWS * C::BF : 0;
    for (int kbl = h; kbl < KB && ok; kbl += C::GROUPS) {
      const int j = kbl >> 1, ws = j % SW, b = kbl % NA;
      const int k_begin = (kb0 + kbl) * C::BK;
      if (!(I4B_W4T_SLEEP ? mbar_wait_sleep(&wfull[ws], (j / SW) & 1) : mbar_wait(&wfull[ws], (j / SW) & 1))) {
        ok = false;
        break;
      }
      if (kbl >= NA) {
        const uint32_t par = ((kbl / NA) - 1) & 1;
        if (!(I4B_W4T_SLEEP ? mbar_wait_sleep(&afree[b], par) : mbar_wait(&afree[b], par))) { ok = false; break; }
        tc_fence_after();
      }
      const uint32_t* P = reinterpret_cast<const uint32_t*>(sW(ws)) + (kbl & 1) * 8 * C::BF;
      const uint16_t* SZ = reinterpret_cast<const uint16_t*>(sW(ws) + C::P_BYTES);
      uint32_t w[8];
#pragma unroll
      for (int jw = 0; jw < 8; ++jw) w[jw] = P[jw * C::BF + nl];
      // group rows of the stage's scale / zero box: the stage starts at group (k of its first k-block) / G
      const int g_stage = ((kb0 + 2 * j) * C::BK) / G;
      const int g_lo = k_begin / G, g_end = (g_lo + 1) * G;
      const int r_lo = g_lo - g_stage;
      const DqParams p0 = dq_params<F16>(SZ[soff + r_lo * C::BF + nl], SZ[zoff + r_lo * C::BF + nl]);
      const int jsplit = (g_end - k_begin) >> 3;  // words of this k-block inside group g_lo (>= 1)
      const DqParams p1 =
          jsplit < 8 ? dq_params<F16>(SZ[soff + (r_lo + 1) * C::BF + nl], SZ[zoff + (r_lo + 1) * C::BF + nl]) : p0;
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[ws]);  // the words and parameters are in registers
      uint4 v[8];
#pragma unroll
      for (int jw = 0; jw < 8; ++jw) v[jw] = w4t_dequant_word<F16>(w[jw], jw >= jsplit ? p1 : p0);
      const uint32_t col = tmem + lane_base + uint32_t(C::A_COL + b * C::A_SLOT_COLS);
      tmem_st_32x32b_x16(col, v[0], v[1], v[2], v[3]);
      tmem_st_32x32b_x16(col + 16u, v[4], v[5], v[6], v[7]);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&aready[b]);
    }
    // The same for the A slots this group dequantized into: wait for the MMA release of each slot's last use.
    for (int b = h; ok && b < NA && b < KB; b += C::GROUPS) {
      const int last = b + NA * ((KB - 1 - b) / NA);
      const uint32_t par = (last / NA) & 1;
      if (!(I4B_W4T_SLEEP ? mbar_wait_sleep(&afree[b], par) : mbar_wait(&afree[b], par))) ok = false;
    }
    // ---- epilogue: the dequant warps read the accumulator in 16-token chunks: warp (q, h) takes chunks
    // h, h + GROUPS, ... of lane quarter q.  Thread = weight row n; per token, a warp stores 32 consecutive
    // outputs (64 bytes of y, or 128 bytes of fp32 partials).
    if (!mbar_wait_sleep(tfull, 0)) ok = false;
    tc_fence_after();
    const int n = n0 + nl;
#pragma unroll 1
    for (int c0 = 16 * h; c0 < NT; c0 += 16 * C::GROUPS) {
      uint32_t v[16];
      tmem_ld_32x32b_x16(tmem + lane_base + uint32_t(c0), v);  // the whole warp, every iteration
      tmem_ld_wait();
      const int rows = min(16, M - (m0 + c0));
      if (n < N && ksplit > 1) {
        float* dst = partials + (int64_t(blockIdx.z) * M + m0 + c0) * N + n;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i < rows) dst[int64_t(i) * N] = __uint_as_float(v[i]);
      } else if (n < N) {
        uint16_t* dst = y + int64_t(m0 + c0) * sym + n;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float a = __uint_as_float(v[i]);
          if (i < rows)
            dst[int64_t(i) * sym] =
                F16 ? __half_as_ushort(__float2half_rn(a)) : __bfloat16_as_ushort(__float2bfloat16_rn(a));
        }
      }
      __syncwarp();
    }
  }
  if (!ok) atomicOr(&g_w4t_err, I4B_DEVERR_WAIT_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (ksplit > 1) {
    // The last CTA of this output tile (atomic ticket, no spinning) adds the ksplit fp32 partials in split
    // order and writes y; then it resets the ticket for the next call.
    const unsigned int tile = blockIdx.y * gridDim.x + blockIdx.x;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(tickets + tile, 1u) == unsigned(ksplit - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int64_t stride_z = int64_t(M) * N;
    // items of 4 consecutive outputs of one token (N % 8 == 0 on this path); 32 threads cover a token's 128
    constexpr int NQ = C::BF / 4;
    for (int idx = threadIdx.x; idx < NT * NQ; idx += blockDim.x) {
      const int m = m0 + idx / NQ, nn = n0 + 4 * (idx % NQ);
      if (m >= M || nn >= N) continue;
      const float* src = partials + int64_t(m) * N + nn;
      float4 a = __ldcg(reinterpret_cast<const float4*>(src));
      for (int z = 1; z < ksplit; ++z) {  // split order
        const float4 t = __ldcg(reinterpret_cast<const float4*>(src + z * stride_z));
        a.x += t.x;
        a.y += t.y;
        a.z += t.z;
        a.w += t.w;
      }
      uint16_t* dst = y + int64_t(m) * sym + nn;
      if constexpr (F16) {
        dst[0] = __half_as_ushort(__float2half_rn(a.x));
        dst[1] = __half_as_ushort(__float2half_rn(a.y));
        dst[2] = __half_as_ushort(__float2half_rn(a.z));
        dst[3] = __half_as_ushort(__float2half_rn(a.w));
      } else {
        dst[0] = __bfloat16_as_ushort(__float2bfloat16_rn(a.x));
        dst[1] = __bfloat16_as_ushort(__float2bfloat16_rn(a.y));
        dst[2] = __bfloat16_as_ushort(__float2bfloat16_rn(a.z));
        dst[3] = __bfloat16_as_ushort(__float2bfloat16_rn(a.w));
      }
    }
    if (threadIdx.x == 0) atomicExch(tickets + tile, 0u);
  }
}

// ------------------------------------------------------------------ launch

template <bool F16, int NT>
static cudaError_t launch_w4t_impl(const TcOperands& o, int64_t M, int64_t N, int64_t K, int G, uint16_t* y,
                                   int64_t sym, int ksplit, float* partials, unsigned int* tickets,
                                   cudaStream_t stream) {
  using C = W4tCfg<NT>;
  const CUtensorMapDataType act = F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap mx{}, mw{}, msz{};
  bool ok = make_tma_map_2d(&mx, act, o.x, uint64_t(K), uint64_t(M), uint64_t(o.sxm) * 2, 64, NT,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  ok = ok && make_tma_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_INT32, o.w, uint64_t(N), uint64_t(K / 8),
                             uint64_t(o.sw) * 4, C::BF, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
  // scales and zeros as the two planes of one 3-D tensor (the lower address first), so that one box brings
  // both; the planes are 16-byte aligned allocations, so their distance is a multiple of 16 bytes
  const uintptr_t ps = reinterpret_cast<uintptr_t>(o.sc), pz = reinterpret_cast<uintptr_t>(o.zr);
  const int swap = pz < ps ? 1 : 0;
  const uint16_t* lo = swap ? o.zr : o.sc;
  const uint64_t dist = swap ? uint64_t(ps - pz) : uint64_t(pz - ps);
  if (dist == 0 || dist % 16 != 0) return cudaErrorNotSupported;
  ok = ok && make_tma_map_3d(&msz, CU_TENSOR_MAP_DATA_TYPE_UINT16, lo, uint64_t(N), uint64_t(K / G), 2,
                             uint64_t(o.ssg) * 2, dist, C::BF, C::SZ_ROWS, 2, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!ok) return cudaErrorNotSupported;  // the caller falls back to the shared-memory-operand kernel
  auto kern = w4t_gemm_kernel<F16, NT>;
  if (cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), C::SMEM)) return e;
  dim3 grid(unsigned(cdiv(N, C::BF)), unsigned(cdiv(M, NT)), unsigned(ksplit));
  kern<<<grid, C::THREADS, C::SMEM, stream>>>(mx, mw, msz, swap, int(M), int(N), int(K), G, y, sym, ksplit,
                                               partials, tickets);
  return cudaGetLastError();
}

int w4t_ctas_per_sm(int tile) { return tile == 5 ? W4tCfg<256>::CPS : W4tCfg<128>::CPS; }

int w4t_token_tile(int tile) { return tile == 5 ? 256 : tile == 6 ? 128 : tile == 7 ? 64 : tile == 8 ? 32 : 0; }

cudaError_t launch_w4t(bool f16, const TcOperands& o, int64_t M, int64_t N, int64_t K, int G, uint16_t* y,
                       int64_t sym, int tile, int ksplit, float* partials, unsigned int* tickets,
                       cudaStream_t stream) {
#define I4B_W4T(F)                                                                                   \
  switch (w4t_token_tile(tile)) {                                                                    \
    case 256: return launch_w4t_impl<F, 256>(o, M, N, K, G, y, sym, ksplit, partials, tickets, stream); \
    case 128: return launch_w4t_impl<F, 128>(o, M, N, K, G, y, sym, ksplit, partials, tickets, stream); \
    case 64: return launch_w4t_impl<F, 64>(o, M, N, K, G, y, sym, ksplit, partials, tickets, stream);   \
    case 32: return launch_w4t_impl<F, 32>(o, M, N, K, G, y, sym, ksplit, partials, tickets, stream);   \
    default: return cudaErrorInvalidValue;                                                           \
  }
  if (f16) I4B_W4T(true);
  I4B_W4T(false);
#undef I4B_W4T
}

unsigned int read_w4t_error(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_w4t_err, sizeof(v));
  if (clear) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_w4t_err, &z, sizeof(z));
  }
  return v;
}

}  // namespace i4b
