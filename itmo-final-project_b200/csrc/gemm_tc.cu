// Large-M (M > 16) W4A16 / W16A16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces the reference's large-M Triton path _matmul_kernel (int4_triton/gemm.py:74-157,
// launched at gemm.py:270-296).  y[M, N] = x[M, K] @ W_hat[N, K]^T.
//
// One CTA computes a 256 x 128 output tile as two 128 x 128 tcgen05 MMAs per k16 step that share
// one B (weight) tile, so every dequantized weight feeds 256 rows (a 128 x 128 tile with one MMA when
// 256-row tiles would leave most SMs idle).  18 warps:
//   warp 0      TMA producer: per 64-wide k-block the activation tile (256 x 64 bf16, 128-byte
//               swizzle) and either the packed weight tile (8 k8-rows x 128 int32) plus two rows
//               of scales and zeros (INT4), or the bf16 weight tile 128 x 64 (W16);
//   warp 1      allocates 256 TMEM columns (two fp32 accumulators) and, from one thread, issues
//               eight tcgen05.mma.kind::f16 (two row halves x four K = 16 steps) per k-block,
//               then tcgen05.commit to free the stage;
//   warps 2..17 INT4 only: dequantize the packed tile into the K-major, 128-byte-swizzled B
//               operand in shared memory (thread = one weight row x two packed words),
//                 W_hat = bf16_rn((q - z) * s)   (exactly the reference's dequantize-then-round,
//                 int4_triton/gemm.py:137-140),
//               using bf16x2 arithmetic: (128+q) - (128+z) is exact, the fp16 scale is split
//               into s_hi (top 8 significant bits, a bf16) and s_lo (the remaining 3 bits, also
//               an exact bf16), q*s_lo is exact and fma(qz, s_hi, qz*s_lo) rounds once;
//               then all sixteen read the accumulators back with tcgen05.ld and store bf16 /
//               fp16 rows of y.
// Stages are handed over with mbarriers (TMA transaction bytes, dequant arrivals,
// tcgen05.commit).  Every wait is bounded; on expiry the kernel records
// I4B_DEVERR_WAIT_TIMEOUT, drains its own TMA copies, frees TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace i4b {

static __device__ unsigned int g_tc_err = 0;

template <bool INT4, int BN, int BMT>
struct TcCfg {
  static constexpr int BM = 128 * BMT, BK = 64;  // BMT row halves of 128 share each B tile
  static constexpr int DQ_WARPS = 16;
  static constexpr int THREADS = 64 + 32 * DQ_WARPS;
  static constexpr int A_BYTES = BM * BK * 2;                 // activation tile, 128-byte rows
  static constexpr int B_BYTES = BN * BK * 2;                 // weight tile (bf16 / fp16), BN rows of 128 B
  static constexpr int P_BYTES = INT4 ? 8 * BN * 4 : 0;       // packed words of one k-block
  static constexpr int SZ_BYTES = INT4 ? 2 * 2 * BN * 2 : 0;  // scales + zeros, two group rows
  // TMA stages carry A (+ packed weights, scales, zeros for INT4, or the B tile for W16).  INT4 B tiles
  // are written by the dequant warps into their own NB-deep ring, decoupled from the TMA stages.
  // Four slots for 128-column tiles (a k-block's dequant, MMA and slot hand-back overlap); two for 256.
  static constexpr int NB = INT4 ? (BN == 128 ? 4 : 2) : 0;
  static constexpr int STAGE_BYTES = INT4 ? (A_BYTES + P_BYTES + SZ_BYTES) : (A_BYTES + B_BYTES);
  static constexpr int BUDGET = 216 * 1024 - NB * B_BYTES;
  static constexpr int STAGES = BUDGET / STAGE_BYTES > 8 ? 8 : BUDGET / STAGE_BYTES;
  static constexpr int TX_BYTES = STAGE_BYTES;
  static constexpr int BAR_BYTES = (2 * STAGES + 2 * NB + 1) * 8 + 8;
  static constexpr size_t SMEM = 1024 + size_t(STAGES) * STAGE_BYTES + size_t(NB) * B_BYTES + BAR_BYTES;
  static constexpr int TMEM_COLS = BMT * BN;
  static_assert(STAGES >= 2, "at least two pipeline stages");
  static_assert(TMEM_COLS <= 512, "accumulators exceed TMEM");
};

// 8 nibbles of one packed word -> 8 dequantized 16-bit values in k order (one 16-byte chunk).
template <bool F16>
__device__ __forceinline__ uint4 dequant_word(uint32_t w, const DqParams& p) {
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
  // r[i] = (w_i, w_{i+4}); reorder to (w0,w1) (w2,w3) (w4,w5) (w6,w7)
  return make_uint4(__byte_perm(r[0], r[1], 0x5410), __byte_perm(r[2], r[3], 0x5410),
                    __byte_perm(r[0], r[1], 0x7632), __byte_perm(r[2], r[3], 0x7632));
}

template <bool INT4, bool F16, int BN, int BMT>
__global__ void __launch_bounds__(TcCfg<INT4, BN, BMT>::THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z, int M, int N,
                   int K, int G, uint16_t* __restrict__ y, int64_t sym, int ksplit, float* __restrict__ partials,
                   unsigned int* __restrict__ tickets) {
  using C = TcCfg<INT4, BN, BMT>;
  constexpr int S = C::STAGES;
  constexpr int NB = C::NB;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms, by offsetting the shared array itself (a round trip
  // through an integer would turn every shared access below into a generic one).
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  // [S stages: A | (P | SZ) or B] [NB dequantized B tiles] [barriers]
  uint8_t* stage0 = smem;
  uint8_t* bring = stage0 + S * C::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(bring + NB * C::B_BYTES);
  uint64_t* empty = full + S;
  uint64_t* bready = empty + S;  // INT4: B tile b dequantized
  uint64_t* bfree = bready + NB; // INT4: B tile b no longer read by the MMAs
  uint64_t* tfull = bfree + NB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  auto sA = [&](int s) { return stage0 + s * C::STAGE_BYTES; };
  auto sP = [&](int s) { return stage0 + s * C::STAGE_BYTES + C::A_BYTES; };             // INT4
  auto sSZ = [&](int s) { return stage0 + s * C::STAGE_BYTES + C::A_BYTES + C::P_BYTES; };  // INT4
  auto sB = [&](int kb) {
    if constexpr (INT4) return bring + (kb % NB) * C::B_BYTES;
    else return stage0 + (kb % S) * C::STAGE_BYTES + C::A_BYTES;
  };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * C::BM;
  // split-K: this CTA owns k-blocks [kb0, kb1); kbl = kb - kb0 indexes the pipeline stages
  const int KBT = (K + C::BK - 1) / C::BK;
  const int kb0 = int((int64_t(blockIdx.z) * KBT) / ksplit), kb1 = int((int64_t(blockIdx.z + 1) * KBT) / ksplit);
  const int KB = kb1 - kb0;
  __shared__ int s_last;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&bready[b], C::DQ_WARPS);
      mbar_init(&bfree[b], 1);
    }
    mbar_init(tfull, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
    if constexpr (INT4) {
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_z);
    }
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

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int kp = kb0 + S; kp < kb0 + 2 * S && kp < kb1; ++kp) {  // the first S k-blocks are loaded right away
        tma_prefetch_l2_2d(&tm_x, kp * C::BK, m0);
        if constexpr (INT4) {
          tma_prefetch_l2_2d(&tm_w, n0, kp * 8);
          tma_prefetch_l2_2d(&tm_s, n0, (kp * C::BK) / G);
          tma_prefetch_l2_2d(&tm_z, n0, (kp * C::BK) / G);
        } else {
          tma_prefetch_l2_2d(&tm_w, kp * C::BK, n0);
        }
      }
      for (int kbl = 0; kbl < KB; ++kbl) {
        const int kb = kb0 + kbl;
        const int s = kbl % S, u = kbl / S;
        if (kbl >= S && !mbar_wait(&empty[s], (u - 1) & 1)) { ok = false; break; }
        // Pull the tiles of k-block kb + 2S into L2 now, so that their TMA loads, issued S k-blocks
        // from now, do not wait for HBM.
        const int kp = kb + 2 * S;
        if (kp < kb1) {
          tma_prefetch_l2_2d(&tm_x, kp * C::BK, m0);
          if constexpr (INT4) {
            tma_prefetch_l2_2d(&tm_w, n0, kp * 8);
            tma_prefetch_l2_2d(&tm_s, n0, (kp * C::BK) / G);
            tma_prefetch_l2_2d(&tm_z, n0, (kp * C::BK) / G);
          } else {
            tma_prefetch_l2_2d(&tm_w, kp * C::BK, n0);
          }
        }
        mbar_arrive_expect_tx(&full[s], C::TX_BYTES);
        tma_load_2d(sA(s), &tm_x, &full[s], kb * C::BK, m0);
        if constexpr (INT4) {
          const int g_lo = (kb * C::BK) / G;
          tma_load_2d(sP(s), &tm_w, &full[s], n0, kb * 8);
          tma_load_2d(sSZ(s), &tm_s, &full[s], n0, g_lo);
          tma_load_2d(sSZ(s) + 2 * BN * 2, &tm_z, &full[s], n0, g_lo);
        } else {
          tma_load_2d(sB(kbl), &tm_w, &full[s], kb * C::BK, n0);
        }
        ++issued;
      }
      // Never leave a bulk copy in flight: wait for the last use of every stage.
      for (int s = 0; s < S && s < issued; ++s) {
        const int last = ((issued - 1 - s) / S) * S + s;
        if (!mbar_wait(&full[s], (last / S) & 1)) ok = false;
      }
      // Nor an MMA-completion arrival (tcgen05.commit arrives asynchronously; one landing after the CTA has
      // exited would write into the shared memory of the next CTA on this SM): wait for the release of every
      // stage's last use.
      for (int s = 0; ok && s < S && s < issued; ++s) {
        const int last = ((issued - 1 - s) / S) * S + s;
        if (!mbar_wait(&empty[s], (last / S) & 1)) ok = false;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(F16 ? 0 : 1, 128, BN);
      for (int kbl = 0; kbl < KB; ++kbl) {
        const int s = kbl % S, u = kbl / S;
        // The activation tile arrives on full[s]; INT4 weights come dequantized on bready[kbl % NB].
        if (!mbar_wait(&full[s], u & 1)) { ok = false; break; }
        if constexpr (INT4) {
          if (!mbar_wait(&bready[kbl % NB], (kbl / NB) & 1)) { ok = false; break; }
        }
        tc_fence_after();
        const uint64_t adesc0 = umma_desc_sw128(smem_u32(sA(s)));
        const uint64_t adesc1 = umma_desc_sw128(smem_u32(sA(s) + C::A_BYTES / 2));
        const uint64_t bdesc = umma_desc_sw128(smem_u32(sB(kbl)));
#pragma unroll
        for (int kk = 0; kk < C::BK / 16; ++kk) {
          const uint32_t acc = (kbl | kk) != 0 ? 1u : 0u;
          umma_f16_ss(tmem, adesc0 + 2 * kk, bdesc + 2 * kk, idesc, acc);
          if constexpr (BMT == 2) umma_f16_ss(tmem + uint32_t(BN), adesc1 + 2 * kk, bdesc + 2 * kk, idesc, acc);
        }
        umma_commit(&empty[s]);
        if constexpr (INT4) umma_commit(&bfree[kbl % NB]);
      }
      umma_commit(tfull);  // also on the error path: completes once issued MMAs are done
    }
  } else {
    if constexpr (INT4) {
      // thread dt: weight row nl = dt % BN, packed words WPT*h .. WPT*h + WPT - 1 of the k-block (h = dt / BN)
      constexpr int WPT = 8 * BN / (32 * C::DQ_WARPS);
      const int dt = threadIdx.x - 64;
      const int nl = dt % BN, h = dt / BN;
      // Group bookkeeping without divisions: k-block kb covers k in [64 kb, 64 kb + 64); g_lo is the group
      // of its first k and g_end the first k of the next group.  The scale / zero parameters of a group
      // are computed once and kept while the group lasts (G >= 32, so a k-block touches at most 2 groups).
      int g_lo = (kb0 * C::BK) / G, g_end = (g_lo + 1) * G;
      int g_cached = -1;
      DqParams pc{};
      for (int kbl = 0; kbl < KB && ok; ++kbl) {
        const int s = kbl % S, u = kbl / S;
        const int k_begin = (kb0 + kbl) * C::BK;
        while (k_begin >= g_end) {
          ++g_lo;
          g_end += G;
        }
        if (!mbar_wait_sleep(&full[s], u & 1)) { ok = false; break; }
        if (kbl >= NB && !mbar_wait_sleep(&bfree[kbl % NB], ((kbl / NB) - 1) & 1)) { ok = false; break; }
        const uint32_t* P = reinterpret_cast<const uint32_t*>(sP(s));
        const uint16_t* Ss = reinterpret_cast<const uint16_t*>(sSZ(s));
        const uint16_t* Zs = Ss + 2 * BN;
        uint8_t* Bs = sB(kbl);
        if (g_cached != g_lo) {
          pc = dq_params<F16>(Ss[nl], Zs[nl]);
          g_cached = g_lo;
        }
        const DqParams p0 = pc;
        const int jsplit = (g_end - k_begin) >> 3;  // words of this k-block inside group g_lo (>= 1)
        DqParams p1 = p0;
        if (jsplit < 8) {
          p1 = dq_params<F16>(Ss[BN + nl], Zs[BN + nl]);
          pc = p1;
          g_cached = g_lo + 1;
        }
#pragma unroll
        for (int jj = 0; jj < WPT; ++jj) {
          const int j = WPT * h + jj;
          const uint4 v = dequant_word<F16>(P[j * BN + nl], j >= jsplit ? p1 : p0);
          *reinterpret_cast<uint4*>(Bs + nl * 128 + ((j ^ (nl & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bready[kbl % NB]);
      }
    }
    if constexpr (INT4) {
      // the MMA release of each B slot's last use (see the producer)
      for (int b = 0; ok && b < NB && b < KB; ++b) {
        const int last = b + NB * ((KB - 1 - b) / NB);
        if (!mbar_wait_sleep(&bfree[b], (last / NB) & 1)) ok = false;
      }
    }
    // ---- epilogue: TMEM -> registers -> y.  The dequant warps form DQ_WARPS / 4 sets of four (one per
    // TMEM lane quarter); with two row halves set j reads accumulator j % 2, and the sets split the
    // columns of their accumulator evenly.
    if (!mbar_wait_sleep(tfull, 0)) ok = false;
    tc_fence_after();
    constexpr int SETS = C::DQ_WARPS / 4;
    constexpr int CSPLIT = BMT == 2 ? SETS / 2 : SETS;  // column slices per accumulator
    const int q = warp & 3, set = (warp - 2) >> 2;
    const int half = BMT == 2 ? (set & 1) : 0, cs = BMT == 2 ? (set >> 1) : set;
    const int m = m0 + 128 * half + 32 * q + lane;
    const int cbeg = cs * (BN / CSPLIT), cend = cbeg + BN / CSPLIT;
    const uint32_t acc_col = uint32_t(half * BN);
    const bool vec = (sym % 8 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0);
#pragma unroll 1
    for (int c0 = cbeg; c0 < cend; c0 += 16) {
      uint32_t v[16];
      tmem_ld_32x32b_x16(tmem + (uint32_t(32 * q) << 16) + acc_col + uint32_t(c0), v);
      tmem_ld_wait();
      if (ksplit > 1) {  // fp32 partial of this K split; the tile's last CTA adds the splits below
        const int n = n0 + c0;
        if (m < M) {
          float* dst = partials + (int64_t(blockIdx.z) * M + m) * N + n;
          if ((N % 4) == 0 && n + 16 <= N) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              reinterpret_cast<uint4*>(dst)[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (n + i < N) dst[i] = __uint_as_float(v[i]);
          }
        }
        continue;
      }
      if (m < M) {
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float a = __uint_as_float(v[2 * i]), b = __uint_as_float(v[2 * i + 1]);
          if constexpr (F16) {
            const __half2 hh = __floats2half2_rn(a, b);
            pk[i] = *reinterpret_cast<const uint32_t*>(&hh);
          } else {
            const __nv_bfloat162 hh = __floats2bfloat162_rn(a, b);
            pk[i] = *reinterpret_cast<const uint32_t*>(&hh);
          }
        }
        const int n = n0 + c0;
        uint16_t* dst = y + int64_t(m) * sym + n;
        if (vec && n + 16 <= N) {
          reinterpret_cast<uint4*>(dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          reinterpret_cast<uint4*>(dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (n + i < N) dst[i] = uint16_t(pk[i >> 1] >> (16 * (i & 1)));
        }
      }
    }
  }
  if (!ok) atomicOr(&g_tc_err, I4B_DEVERR_WAIT_TIMEOUT);
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
    if (N % 4 == 0) {
      // items of 4 consecutive columns; each thread keeps 4 items x ksplit (<= 4) float4 loads in flight
      constexpr int NQ = BN / 4;
      constexpr int ITEMS = C::BM * NQ;
      for (int base = threadIdx.x; base < ITEMS; base += 4 * blockDim.x) {
        float4 t[4][4];
        int64_t off[4];
        bool valid[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int idx = base + u * blockDim.x;
          const int m = m0 + idx / NQ, n = n0 + 4 * (idx % NQ);
          valid[u] = idx < ITEMS && m < M && n < N;
          off[u] = valid[u] ? int64_t(m) * N + n : 0;
        }
#pragma unroll
        for (int z = 0; z < 4; ++z)
#pragma unroll
          for (int u = 0; u < 4; ++u)
            t[z][u] = (z < ksplit && valid[u]) ? __ldcg(reinterpret_cast<const float4*>(partials + off[u] + z * stride_z))
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (!valid[u]) continue;
          float4 a = t[0][u];
#pragma unroll
          for (int z = 1; z < 4; ++z)
            if (z < ksplit) {  // split order
              a.x += t[z][u].x;
              a.y += t[z][u].y;
              a.z += t[z][u].z;
              a.w += t[z][u].w;
            }
          const int64_t m = off[u] / N, n = off[u] % N;
          uint16_t* dst = y + m * sym + n;
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
      }
    } else {
      for (int idx = threadIdx.x; idx < C::BM * BN; idx += blockDim.x) {
        const int m = m0 + idx / BN, n = n0 + idx % BN;
        if (m >= M || n >= N) continue;
        const float* src = partials + int64_t(m) * N + n;
        float t[4];
#pragma unroll
        for (int z = 0; z < 4; ++z) t[z] = z < ksplit ? __ldcg(src + z * stride_z) : 0.0f;
        float acc = t[0];
#pragma unroll
        for (int z = 1; z < 4; ++z)
          if (z < ksplit) acc += t[z];
        if constexpr (F16) y[int64_t(m) * sym + n] = __half_as_ushort(__float2half_rn(acc));
        else y[int64_t(m) * sym + n] = __bfloat16_as_ushort(__float2bfloat16_rn(acc));
      }
    }
    if (threadIdx.x == 0) atomicExch(tickets + tile, 0u);
  }
}

// ------------------------------------------------------------------ repack (misaligned operands)

// out[r, c] = c < cols_in ? in[r*sr + c*sc] : 0   (element size 2 or 4 bytes)
template <typename T>
__global__ void repack2d_kernel(const T* __restrict__ in, int64_t rows, int64_t cols_in, int64_t sr, int64_t sc,
                                T* __restrict__ out, int64_t cols_out) {
  const int64_t total = rows * cols_out;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols_out, c = i % cols_out;
    out[i] = c < cols_in ? in[r * sr + c * sc] : T(0);
  }
}

cudaError_t launch_repack(const void* in, int esize, int64_t rows, int64_t cols_in, int64_t sr, int64_t sc, void* out,
                          int64_t cols_out, cudaStream_t stream) {
  const int64_t total = rows * cols_out;
  if (total == 0) return cudaSuccess;
  const int blocks = int(std::min<int64_t>((total + 255) / 256, 148 * 16));
  if (esize == 2)
    repack2d_kernel<uint16_t><<<blocks, 256, 0, stream>>>(static_cast<const uint16_t*>(in), rows, cols_in, sr, sc,
                                                          static_cast<uint16_t*>(out), cols_out);
  else
    repack2d_kernel<uint32_t><<<blocks, 256, 0, stream>>>(static_cast<const uint32_t*>(in), rows, cols_in, sr, sc,
                                                          static_cast<uint32_t*>(out), cols_out);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ tensor maps + launch

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D row-major tensor: `inner` contiguous elements per row, `rows` rows `row_bytes` apart.
bool make_tma_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}



// 3-D tensor: `d0` contiguous elements, then `d1` rows `stride1` bytes apart, then `d2` planes `stride2`
// bytes apart.
bool make_tma_map_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
                     uint64_t d2, uint64_t stride1, uint64_t stride2, uint32_t b0, uint32_t b1, uint32_t b2,
                     CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1, stride2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool INT4, bool F16, int BN, int BMT>
static cudaError_t launch_tc_impl(const TcOperands& o, int64_t M, int64_t N, int64_t K, int G, uint16_t* y,
                                  int64_t sym, int ksplit, float* partials, unsigned int* tickets,
                                  cudaStream_t stream) {
  using C = TcCfg<INT4, BN, BMT>;
  const CUtensorMapDataType act = F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap mx{}, mw{}, ms{}, mz{};
  bool ok = make_tma_map_2d(&mx, act, o.x, uint64_t(K), uint64_t(M), uint64_t(o.sxm) * 2, 64, C::BM,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if constexpr (INT4) {
    ok = ok && make_tma_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_INT32, o.w, uint64_t(N), uint64_t(K / 8), uint64_t(o.sw) * 4, BN,
                        8, CU_TENSOR_MAP_SWIZZLE_NONE);
    ok = ok && make_tma_map_2d(&ms, CU_TENSOR_MAP_DATA_TYPE_UINT16, o.sc, uint64_t(N), uint64_t(K / G), uint64_t(o.ssg) * 2,
                        BN, 2, CU_TENSOR_MAP_SWIZZLE_NONE);
    ok = ok && make_tma_map_2d(&mz, CU_TENSOR_MAP_DATA_TYPE_UINT16, o.zr, uint64_t(N), uint64_t(K / G), uint64_t(o.ssg) * 2,
                        BN, 2, CU_TENSOR_MAP_SWIZZLE_NONE);
  } else {
    ok = ok && make_tma_map_2d(&mw, act, o.w, uint64_t(K), uint64_t(N), uint64_t(o.sw) * 2, 64, BN,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    ms = mw;
    mz = mw;
  }
  if (!ok) return cudaErrorInvalidValue;
  auto kern = tc_gemm_kernel<INT4, F16, BN, BMT>;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(unsigned(cdiv(N, BN)), unsigned(cdiv(M, C::BM)), unsigned(ksplit));
  kern<<<grid, C::THREADS, C::SMEM, stream>>>(mx, mw, ms, mz, int(M), int(N), int(K), G, y, sym, ksplit, partials,
                                               tickets);
  return cudaGetLastError();
}

// Rows per CTA: 256 (two accumulators share each dequantized weight tile) when that still fills half a
// wave of the GPU, else 128 (twice the CTAs).
#ifndef I4B_TC_FORCE
#define I4B_TC_FORCE 0
#endif
// Tile code: 1 -> 128 x 128, 2 -> 256 x 128 (two MMAs share a B tile), 3 -> 128 x 256, 4 -> 256 x 256.
// The plan minimises a cost model fitted to B200 measurements of this kernel (INT4, G = 128, 148 SMs):
// a wave of CTAs costs F + c * (k-blocks per CTA) microseconds, with (F, c) = (4.0, 0.72) for 128 x 128,
// (6.4, 0.74) for 256 x 128 and (7.5, 0.90) for 256 x 256 -- the small tiles are bound by per-CTA
// latency, the large one by the tensor pipe -- and a K split adds 5 us + 17 us per MiB of fp32 partials
// that the last CTA of a tile reads back.  Bigger tiles read fewer activation and weight bytes per flop;
// splits fill the machine when there are few output tiles.
static int g_tc_ovr_tile = 0, g_tc_ovr_splits = 0;

void set_tc_override(int tile, int splits) {
  g_tc_ovr_tile = tile >= 1 && tile <= 8 ? tile : 0;
  g_tc_ovr_splits = (splits == 1 || splits == 2 || splits == 4 || splits == 8) ? splits : 0;
}

static int64_t tc_tiles(int tile, int64_t M, int64_t N) {
  const int64_t bm = (tile == 2 || tile == 4) ? 256 : 128, bn = (tile == 3 || tile == 4) ? 256 : 128;
  return cdiv(M, bm) * cdiv(N, bn);
}

static double tc_cost(int tile, int splits, int64_t M, int64_t N, int64_t kb, int num_sms) {
  const double F = tile == 4 ? 7.5 : tile == 2 ? 6.4 : 4.0;
  const double c = tile == 4 ? 0.90 : tile == 2 ? 0.74 : 0.72;
  const int64_t tiles = tc_tiles(tile, M, N);
  const int64_t waves = cdiv(tiles * splits, int64_t(num_sms));
  double t = double(waves) * (F + c * double(cdiv(kb, int64_t(splits))));
  if (splits > 1) {
    const double bm = (tile == 2 || tile == 4) ? 256 : 128, bn = (tile == 3 || tile == 4) ? 256 : 128;
    t += 5.0 + 17.0 * double(splits) * bm * bn * 4.0 / double(1 << 20);
  }
  return t;
}

TcPlan tc_plan(int64_t M, int64_t N, int64_t K, int num_sms) {
  const int64_t kb = cdiv(K, 64);
  TcPlan best{1, 1};
  double best_t = 1e30;
  const int ovr_tile = g_tc_ovr_tile <= 4 ? g_tc_ovr_tile : 0, ovr_splits = g_tc_ovr_splits <= 4 ? g_tc_ovr_splits : 0;
  for (int tile : {4, 2, 1}) {
    if (I4B_TC_FORCE && tile != I4B_TC_FORCE) continue;
    if (ovr_tile && tile != ovr_tile) continue;
    if (tile != 1 && M <= 128) continue;  // a 256-row tile would be half empty
    for (int splits : {1, 2, 4}) {
      if (ovr_splits && splits != ovr_splits) continue;
      if (splits > 1 && (tc_tiles(tile, M, N) > kMaxTickets || kb < 4 * splits)) continue;
      const double t = tc_cost(tile, splits, M, N, kb, num_sms);
      if (t < best_t) {
        best_t = t;
        best = TcPlan{tile, splits};
      }
    }
  }
  if (I4B_TC_FORCE && best_t >= 1e30) best = TcPlan{I4B_TC_FORCE, 1};
  if (ovr_tile && best_t >= 1e30) best = TcPlan{ovr_tile, 1};
  return best;
}

// INT4: the TMEM-weight kernel (gemm_w4t.cu), tile code 5..8 = 256, 128, 64 or 32 tokens per CTA, unless the
// tuning hook asks for one of the shared-memory tiles above (codes 1..4).  Cost model (us) in the form of the
// one above, fitted to B200 sweeps of the Llama-3.2-1B block shapes at M = 16..1024: a wave of CTAs (one per
// SM for 256-token tiles, two per SM otherwise) costs F + c_NT * (k-blocks per CTA), where a k-block's cost is
// set by the fixed latency of a pipeline step more than by its MMA work; a K split adds its fp32 partials'
// round trip through L2.
static double w4t_cost(int nt, int splits, int64_t M, int64_t N, int64_t kb, int num_sms) {
  const double F = 3.0;
  const double c = nt == 256 ? 0.60 : 0.65;
  const int64_t tiles = cdiv(N, 128) * cdiv(M, int64_t(nt));
  const int64_t waves = cdiv(tiles * splits, int64_t(num_sms) * w4t_ctas_per_sm(nt == 256 ? 5 : 6));
  double t = double(waves) * (F + c * double(cdiv(kb, int64_t(splits))));
  if (splits > 1) t += 2.0 + double(splits) * double(M) * double(N) * 8.0 / 3.0e6;
  return t;
}

TcPlan tc_plan_w4(int64_t M, int64_t N, int64_t K, int num_sms) {
  // I4B_W4T_DEFAULT = 0 holds the TMEM-weight kernel back (it then runs only when the tuning hook asks for
  // tile 5..8) and keeps the shared-memory-operand kernel as the default.
  if (!I4B_W4T_DEFAULT && g_tc_ovr_tile < 5) return tc_plan(M, N, K, num_sms);
  if (g_tc_ovr_tile >= 1 && g_tc_ovr_tile <= 4) return tc_plan(M, N, K, num_sms);
  const int64_t kb = cdiv(K, 64);
  TcPlan best{6, 1};
  double best_t = 1e30;
  for (int tile : {5, 6, 7, 8}) {
    if (g_tc_ovr_tile && tile != g_tc_ovr_tile) continue;
    const int nt = w4t_token_tile(tile);
    if (nt > 32 && M <= nt / 2) continue;  // more than half of the tile would be padding
    for (int splits : {1, 2, 4, 8}) {
      if (g_tc_ovr_splits && splits != g_tc_ovr_splits) continue;
      if (splits > 1 && (cdiv(N, 128) * cdiv(M, int64_t(nt)) > kMaxTickets || kb < 2 * splits || N % 4 != 0))
        continue;
      const double t = w4t_cost(nt, splits, M, N, kb, num_sms);
      if (t < best_t) {
        best_t = t;
        best = TcPlan{tile, splits};
      }
    }
  }
  if (best_t >= 1e30 && g_tc_ovr_tile) best = TcPlan{g_tc_ovr_tile, 1};
  return best;
}

size_t tc_partial_bytes(const TcPlan& p, int64_t M, int64_t N) {
  return p.splits > 1 ? size_t(p.splits) * size_t(M) * size_t(N) * 4 : 0;
}

cudaError_t launch_tc(bool int4, bool f16, const TcOperands& o, int64_t M, int64_t N, int64_t K, int G, uint16_t* y,
                      int64_t sym, const TcPlan& plan, float* partials, unsigned int* tickets, cudaStream_t stream) {
  const int bn = plan.tile, ks = plan.splits;
  // bn: tile code, ks: K splits (from tc_plan / tc_plan_w4)
  if (bn >= 5) {
    if (!int4 || (ks > 1 && N % 4 != 0)) return cudaErrorInvalidValue;
    const cudaError_t e = launch_w4t(f16, o, M, N, K, G, y, sym, bn, ks, partials, tickets, stream);
    if (e != cudaErrorNotSupported) return e;
    // scales / zeros whose tensor maps cannot be encoded as one 3-D box (e.g. interleaved views): the
    // shared-memory-operand kernel, one 128 x 128 tile per CTA, no K split (no workspace needed)
    return f16 ? launch_tc_impl<true, true, 128, 1>(o, M, N, K, G, y, sym, 1, partials, tickets, stream)
               : launch_tc_impl<true, false, 128, 1>(o, M, N, K, G, y, sym, 1, partials, tickets, stream);
  }
#define I4B_TC(I, F) \
  return bn == 4   ? launch_tc_impl<I, F, 256, 2>(o, M, N, K, G, y, sym, ks, partials, tickets, stream) \
         : bn == 2 ? launch_tc_impl<I, F, 128, 2>(o, M, N, K, G, y, sym, ks, partials, tickets, stream) \
         : bn == 3 ? launch_tc_impl<I, F, 256, 1>(o, M, N, K, G, y, sym, ks, partials, tickets, stream) \
                   : launch_tc_impl<I, F, 128, 1>(o, M, N, K, G, y, sym, ks, partials, tickets, stream)
  if (int4) {
    if (f16) I4B_TC(true, true);
    I4B_TC(true, false);
  }
  if (f16) I4B_TC(false, true);
  I4B_TC(false, false);
#undef I4B_TC
}

unsigned int read_tc_error(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_err, sizeof(v));
  if (clear) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_tc_err, &z, sizeof(z));
  }
  return v;
}

}  // namespace i4b
