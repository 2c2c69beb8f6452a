// Small-M (M <= 16) W16A16 kernel (full-precision weights): the w16a16_matmul decode GEMV and small-batch
// split-K path.  Only its W16 instantiations are built; INT4 weights are served by gemv_w4.cu, and the
// INT4 branches below are what that kernel grew out of.
//
// Replaces the reference's _gemv_kernel (int4_triton/gemm.py:185-220) and its
// small-M split-K _matmul_kernel + _reduce_split_k pair (gemm.py:74-182,
// launched at gemm.py:265-299) with ONE launch per matmul.
//
// Work split.  grid = (ceil(N / BN), S), cluster (1, S, 1) when 1 < S <= 8.
// A CTA owns BN = 32*WN output columns and the K-range [y*KC, (y+1)*KC);
// warp (wn, wk) owns 32 columns and KW = KC/WK consecutive k.  Every operand
// is fetched by the warp that uses it -- no block barrier before the main loop:
//   * packed words stream through a per-warp ring of 4 stages in shared
//     memory (cp.async, 16 bytes per lane per 32-k step, 4 steps per stage);
//     in one step a warp reads 4 consecutive k8 rows x 32 consecutive columns
//     (4 x 128 B) and lane (r = lane/4, c = lane%4) copies, then reads back,
//     the words of columns 4r..4r+3 at k8 row step*4 + c -- its own bytes, so
//     cp.async.wait_group is the only ordering needed;
//   * scales / zeros: 4 consecutive fp16 each per segment, in the same ring;
//   * activations: 16 bytes (8 consecutive k) per lane and token row, from L1/L2.
// W16 weights use plain 128-bit register loads.
//
// Dequant and MMA.  A word splits into four bf16 (fp16) pairs (128 + q_i,
// 128 + q_{i+4}) with one lop3 each (exact; magic 0x4300 / 0x6400).  The pairs
// ARE the A fragments of mma.m16n8k16 (rows = output columns, k permuted
// consistently with the activation fragment, which is permuted the same way
// in registers), B = activations, fp32 accumulators.  Zero point and scale are
// applied once per segment of L = 32*SPS consecutive k inside one group:
//     sum_k x_k (q_k - z) s  =  s * (D - (128 + z) * X),   D = sum_k x_k (128 + q_k),
// where X = sum_k x_k over the segment comes from one more MMA with an all-ones
// A fragment (it lands in exactly the accumulator layout the update needs).
// This is the exact value of x . ((q - z) s) up to fp32 summation order; the
// reference kernels additionally round each dequantized weight to bf16.
//
// Reduction.  Warps sharing columns add through shared memory in fixed warp
// order.  K-splits inside a cluster add through distributed shared memory in
// fixed rank order.  More than 8 splits fall back to fp32 partials in the
// caller's workspace: the last CTA of a column tile (atomic ticket, no
// spinning) adds them in split order and resets the ticket.  Every path is
// bit-identical from run to run.
//
// Programmatic dependent launch (opt-in): weights and scales are loaded
// before griddepcontrol.wait, activations after it.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace i4b {

struct SkinnyArgs {
  const void* x;
  int64_t sxm, sxk;
  const void* w;   // INT4: uint32 qweight [K/8, N]; W16: weights [N, K]
  int64_t sw0;     // INT4: words per k8 row; W16: stride between rows n
  int64_t sw1;     // W16: stride along k
  const uint16_t* sc;
  const uint16_t* zr;
  int64_t ssg;     // scales/zeros row stride (elements)
  void* y;
  int64_t sym;
  float* partials;
  unsigned int* tickets;
  int M, N, K, G;
  int S, KC, KW, WN, WK;
  int mode;        // 0: S == 1; 1: cluster of S CTAs along K; 2: global tickets
  int vec_w, vec_x, vec_s;
  int pdl;
};

__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int i, uint32_t magic) {
  return and_or(w >> (4 * i), 0x000F000Fu, magic);
}

// Weights are read once: keep them out of L1.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::128B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <bool F16>
__device__ __forceinline__ uint16_t f2h_bits(float v) {
  if constexpr (F16) return __half_as_ushort(__float2half_rn(v));
  else return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

template <int MT, bool INT4, bool F16, int SPS>
__global__ void __launch_bounds__(INT4 ? 512 : 256) skinny_kernel(const SkinnyArgs a) {
  constexpr int MP = MT * 8;                        // padded token count
  constexpr int CH = INT4 ? 4 : (MT == 1 ? 8 : 4);  // 32-k steps per ring stage (INT4) / load batch (W16)
  constexpr int RING = 4;                           // INT4: stages in flight per warp
  constexpr int NSEG = (CH >= SPS) ? CH / SPS : 1;  // segments starting inside one stage
  constexpr int STAGE_W = CH * 512;                 // packed bytes of a stage (32 lanes x 16 B per step)
  constexpr int STAGE_B = STAGE_W + NSEG * 512;     // + scales/zeros (16 B per lane per segment)
  extern __shared__ __align__(16) uint8_t smem_b[];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int wn = warp % a.WN, wk = warp / a.WN;
  const int r = lane >> 2, c = lane & 3;
  const int BN = 32 * a.WN;
  const int64_t n_cta = int64_t(blockIdx.x) * BN;
  const int64_t nb = n_cta + wn * 32;
  const int64_t k0 = int64_t(blockIdx.y) * a.KC;
  const int kw_off = wk * a.KW;                 // warp's first k inside the CTA range
  const int64_t kw0 = k0 + kw_off;
  const int nsteps = a.KW / 32;
  const int M_eff = a.M < MP ? a.M : MP;
  const uint32_t magic = F16 ? 0x64006400u : 0x43004300u;
  const float bias = F16 ? 1024.0f : 128.0f;

  // shared memory: [INT4 rings, RING x STAGE_B per warp][reductions]
  uint8_t* ring = smem_b + size_t(warp) * (INT4 ? RING * STAGE_B : 0);
  float* smem_f = reinterpret_cast<float*>(smem_b + size_t(nwarps) * (INT4 ? RING * STAGE_B : 0));

  // INT4: each lane copies -- and later reads back -- only its own 16-byte chunks of a stage,
  // so cp.async.wait_group alone orders the copy before the read.
  const int64_t n_lane = nb + 4 * r;
  const bool n_in = n_lane < a.N;
  const uint32_t* wsrc = static_cast<const uint32_t*>(a.w) + (kw0 / 8 + c) * a.sw0 + (n_in ? n_lane : 0);
  const int64_t wstep = 4 * a.sw0;  // words between consecutive 32-k steps
  auto issue_stage = [&](int st) {
    if constexpr (INT4) {
      uint8_t* slot = ring + (st % RING) * STAGE_B;
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const int step = st * CH + i;
        if (step < nsteps) {
          const uint32_t* src = wsrc + int64_t(step) * wstep;
          uint8_t* dst = slot + i * 512 + lane * 16;
          if (a.vec_w) {
            cp_async_16(dst, src, n_in ? 16u : 0u);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const bool in = n_lane + j < a.N;
              cp_async_4(dst + 4 * j, in ? src + j : src, in ? 4u : 0u);
            }
          }
        }
      }
      if (a.vec_s) {
#pragma unroll
        for (int j = 0; j < NSEG; ++j) {
          const int step = st * CH + j * SPS;
          if (step < nsteps && (step % SPS) == 0) {
            const int64_t g = (kw0 + int64_t(step) * 32) / a.G;
            uint8_t* dst = slot + STAGE_W + j * 512 + lane * 16;
            const int64_t off = g * a.ssg + (n_in ? n_lane : 0);
            cp_async_8(dst, a.sc + off, n_in ? 8u : 0u);
            cp_async_8(dst + 8, a.zr + off, n_in ? 8u : 0u);
          }
        }
      }
      cp_async_commit();  // one group per stage, empty past the end: keeps the group count uniform
    }
  };

  // W16: register batches loaded straight from global memory.
  uint4 wv[INT4 ? 1 : CH][4];
  auto load_batch_w16 = [&](int cs) {
    if constexpr (!INT4) {
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        if (cs + i < nsteps) {
          const int64_t k = kw0 + int64_t(cs + i) * 32 + 8 * c;
#pragma unroll
          for (int h = 0; h < 4; ++h) {  // rows nb + 16t + r (h = 2t) and nb + 16t + 8 + r (h = 2t+1)
            const int64_t n = nb + 16 * (h >> 1) + 8 * (h & 1) + r;
            const uint16_t* p = static_cast<const uint16_t*>(a.w) + n * a.sw0 + k * a.sw1;
            if (a.vec_w && n < a.N && k + 8 <= a.K) {
              wv[i][h] = ld_stream_v4(p);
            } else {
              uint16_t e[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) e[j] = (n < a.N && k + j < a.K) ? __ldg(p + j * a.sw1) : uint16_t(0);
              wv[i][h] = make_uint4(uint32_t(e[0]) | (uint32_t(e[1]) << 16), uint32_t(e[2]) | (uint32_t(e[3]) << 16),
                                    uint32_t(e[4]) | (uint32_t(e[5]) << 16), uint32_t(e[6]) | (uint32_t(e[7]) << 16));
            }
          }
        }
      }
    }
  };

  // weights and scales do not depend on the previous kernel: start them first
  if constexpr (INT4) {
#pragma unroll
    for (int st = 0; st < RING; ++st) issue_stage(st);
  } else {
    load_batch_w16(0);
  }
  if (a.pdl) pdl_wait();  // activations are produced by the previous kernel

  float acc[2][MT][4];
  float dacc[INT4 ? 2 : 1][INT4 ? MT : 1][4];
  uint2 szv[2];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[t][mt][e] = 0.0f;
  float xsum[INT4 ? MT : 1][4];
  const uint32_t ones = F16 ? 0x3C003C00u : 0x3F803F80u;
  // lane's activation pointer: token mt*8 + r, k = kw0 + step*32 + 8c (+8 values)
  const uint16_t* xlane = static_cast<const uint16_t*>(a.x) + int64_t(r) * a.sxm + (kw0 + 8 * c) * a.sxk;
  const int64_t xstep = 32 * a.sxk;
  const bool x_fast = a.vec_x && (a.K % 32 == 0);

  for (int cs = 0, st = 0; cs < nsteps; cs += CH, ++st) {
    if (!INT4 && cs > 0) load_batch_w16(cs);
    // activation fragments of this stage, permuted like the A fragments (INT4)
    uint4 xv[CH][MT];
#pragma unroll
    for (int i = 0; i < CH; ++i)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t u[4] = {0, 0, 0, 0};
        const int tok = mt * 8 + r;
        if (cs + i < nsteps && tok < M_eff) {
          const uint16_t* p = xlane + int64_t(mt * 8) * a.sxm + int64_t(cs + i) * xstep;
          if (x_fast) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
            u[0] = v.x; u[1] = v.y; u[2] = v.z; u[3] = v.w;
          } else {
            const int64_t k = kw0 + int64_t(cs + i) * 32 + 8 * c;
            uint16_t e[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) e[j] = (k + j < a.K) ? __ldg(p + j * a.sxk) : uint16_t(0);
#pragma unroll
            for (int j = 0; j < 4; ++j) u[j] = uint32_t(e[2 * j]) | (uint32_t(e[2 * j + 1]) << 16);
          }
        }
        if constexpr (INT4) {  // (x0,x4) (x1,x5) (x2,x6) (x3,x7): the nibble-pair order of the A fragments
          xv[i][mt] = make_uint4(__byte_perm(u[0], u[2], 0x5410), __byte_perm(u[0], u[2], 0x7632),
                                 __byte_perm(u[1], u[3], 0x5410), __byte_perm(u[1], u[3], 0x7632));
        } else {
          xv[i][mt] = make_uint4(u[0], u[1], u[2], u[3]);
        }
      }
    const uint8_t* slot = ring + (st % RING) * STAGE_B;
    if constexpr (INT4) cp_async_wait<RING - 1>();  // this stage's group has landed

#pragma unroll
    for (int i = 0; i < CH; ++i) {
      if (cs + i >= nsteps) break;
      const int step = cs + i;
      uint32_t af[2][2][4];  // [row tile][k16 step][reg]
      if constexpr (INT4) {
        if ((step % SPS) == 0) {
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              dacc[0][mt][e] = 0.0f;
              dacc[1][mt][e] = 0.0f;
              xsum[mt][e] = 0.0f;
            }
          const int j = (CH >= SPS) ? (i / SPS) : 0;
          if (a.vec_s) {
            const uint4 v = *reinterpret_cast<const uint4*>(slot + STAGE_W + j * 512 + lane * 16);
            szv[0] = make_uint2(v.x, v.y);
            szv[1] = make_uint2(v.z, v.w);
          } else {
            const int64_t g = (kw0 + int64_t(step) * 32) / a.G;
            uint16_t sv[4], zv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              sv[q] = (n_lane + q < a.N) ? __ldg(a.sc + g * a.ssg + n_lane + q) : uint16_t(0);
              zv[q] = (n_lane + q < a.N) ? __ldg(a.zr + g * a.ssg + n_lane + q) : uint16_t(0);
            }
            szv[0] = make_uint2(uint32_t(sv[0]) | (uint32_t(sv[1]) << 16), uint32_t(sv[2]) | (uint32_t(sv[3]) << 16));
            szv[1] = make_uint2(uint32_t(zv[0]) | (uint32_t(zv[1]) << 16), uint32_t(zv[2]) | (uint32_t(zv[3]) << 16));
          }
        }
        const uint4 w4 = *reinterpret_cast<const uint4*>(slot + i * 512 + lane * 16);
        const uint32_t wd[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            af[t][s][0] = nib_pair(wd[2 * t], 2 * s, magic);
            af[t][s][1] = nib_pair(wd[2 * t + 1], 2 * s, magic);
            af[t][s][2] = nib_pair(wd[2 * t], 2 * s + 1, magic);
            af[t][s][3] = nib_pair(wd[2 * t + 1], 2 * s + 1, magic);
          }
      } else {
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const uint4 lo = wv[i][2 * t], hi = wv[i][2 * t + 1];
          af[t][0][0] = lo.x; af[t][0][1] = hi.x; af[t][0][2] = lo.y; af[t][0][3] = hi.y;
          af[t][1][0] = lo.z; af[t][1][1] = hi.z; af[t][1][2] = lo.w; af[t][1][3] = hi.w;
        }
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint4 b = xv[i][mt];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if constexpr (INT4) {
            mma_16816<F16>(dacc[t][mt], af[t][0], b.x, b.y);
            mma_16816<F16>(dacc[t][mt], af[t][1], b.z, b.w);
          } else {
            mma_16816<F16>(acc[t][mt], af[t][0], b.x, b.y);
            mma_16816<F16>(acc[t][mt], af[t][1], b.z, b.w);
          }
        }
        if constexpr (INT4) {  // X = sum of x over the segment, in the accumulator layout of D
          const uint32_t one4[4] = {ones, ones, ones, ones};
          mma_16816<F16>(xsum[mt], one4, b.x, b.y);
          mma_16816<F16>(xsum[mt], one4, b.z, b.w);
        }
      }
      if constexpr (INT4) {
        if (((step + 1) % SPS) == 0) {  // segment complete: acc += s * (D - (bias + z) * X)
          float sv[4], zv[4];
          const uint32_t s01 = szv[0].x, s23 = szv[0].y, z01 = szv[1].x, z23 = szv[1].y;
          sv[0] = __half2float(__ushort_as_half(uint16_t(s01 & 0xFFFFu)));
          sv[1] = __half2float(__ushort_as_half(uint16_t(s01 >> 16)));
          sv[2] = __half2float(__ushort_as_half(uint16_t(s23 & 0xFFFFu)));
          sv[3] = __half2float(__ushort_as_half(uint16_t(s23 >> 16)));
          zv[0] = bias + __half2float(__ushort_as_half(uint16_t(z01 & 0xFFFFu)));
          zv[1] = bias + __half2float(__ushort_as_half(uint16_t(z01 >> 16)));
          zv[2] = bias + __half2float(__ushort_as_half(uint16_t(z23 & 0xFFFFu)));
          zv[3] = bias + __half2float(__ushort_as_half(uint16_t(z23 >> 16)));
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const float X0 = xsum[mt][0], X1 = xsum[mt][1];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              acc[t][mt][0] = fmaf(sv[2 * t], fmaf(-zv[2 * t], X0, dacc[t][mt][0]), acc[t][mt][0]);
              acc[t][mt][1] = fmaf(sv[2 * t], fmaf(-zv[2 * t], X1, dacc[t][mt][1]), acc[t][mt][1]);
              acc[t][mt][2] = fmaf(sv[2 * t + 1], fmaf(-zv[2 * t + 1], X0, dacc[t][mt][2]), acc[t][mt][2]);
              acc[t][mt][3] = fmaf(sv[2 * t + 1], fmaf(-zv[2 * t + 1], X1, dacc[t][mt][3]), acc[t][mt][3]);
            }
          }
        }
      }
    }
    if constexpr (INT4) issue_stage(st + RING);  // refill the slot just consumed
  }
  if constexpr (INT4) cp_async_wait<0>();
  // ---- outputs: acc[t][mt][e] is (token mt*8 + 2c + (e & 1), local column col(t, e >> 1))
  auto col_of = [&](int t, int half) {
    return INT4 ? (wn * 32 + 4 * r + 2 * t + half) : (wn * 32 + 16 * t + 8 * half + r);
  };
  if (a.mode == 0 && a.WK == 1) {  // each warp owns its columns outright: store from registers
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = mt * 8 + 2 * c + (e & 1);
          const int64_t n = n_cta + col_of(t, e >> 1);
          if (tok < M_eff && n < a.N) static_cast<uint16_t*>(a.y)[int64_t(tok) * a.sym + n] = f2h_bits<F16>(acc[t][mt][e]);
        }
    return;
  }
  float* red = smem_f;                       // [WK][MP][BN]
  float* part = smem_f + a.WK * MP * BN;     // [MP][BN]: this CTA's sum over its warps
  if (a.WK > 1) {
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = mt * 8 + 2 * c + (e & 1);
          if (tok < M_eff) red[(wk * MP + tok) * BN + col_of(t, e >> 1)] = acc[t][mt][e];
        }
    __syncthreads();
    for (int idx = tid; idx < M_eff * BN; idx += blockDim.x) {
      float v = red[idx];
      for (int q = 1; q < a.WK; ++q) v += red[q * MP * BN + idx];
      part[idx] = v;
    }
  } else {
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = mt * 8 + 2 * c + (e & 1);
          if (tok < M_eff) part[tok * BN + col_of(t, e >> 1)] = acc[t][mt][e];
        }
  }
  uint16_t* y = static_cast<uint16_t*>(a.y);
  if (a.mode == 0) {
    __syncthreads();
    for (int idx = tid; idx < M_eff * BN; idx += blockDim.x) {
      const int tok = idx / BN;
      const int64_t n = n_cta + idx % BN;
      if (n < a.N) y[int64_t(tok) * a.sym + n] = f2h_bits<F16>(part[idx]);
    }
    return;
  }
  if (a.mode == 1) {
    // Cluster of S CTAs along K: rank q adds elements q*blockDim + tid (+ S*blockDim ...) over all
    // ranks, in rank order.
    cluster_sync();
    const uint32_t rank = cluster_ctarank();
    for (int idx = int(rank) * blockDim.x + tid; idx < M_eff * BN; idx += a.S * blockDim.x) {
      const uint32_t addr = smem_u32(part + idx);
      float t[8];  // all S (<= 8) remote loads in flight, then added in rank order
#pragma unroll
      for (int q = 0; q < 8; ++q) t[q] = q < a.S ? ld_shared_cluster_f32(mapa_shared(addr, uint32_t(q))) : 0.0f;
      float v = t[0];
#pragma unroll
      for (int q = 1; q < 8; ++q)
        if (q < a.S) v += t[q];
      const int tok = idx / BN;
      const int64_t n = n_cta + idx % BN;
      if (n < a.N) y[int64_t(tok) * a.sym + n] = f2h_bits<F16>(v);
    }
    cluster_sync();  // no CTA leaves while others may still read its shared memory
    return;
  }
  // mode 2: fp32 partials in the workspace, the last CTA of the column tile adds them in split order.
  __syncthreads();
  for (int idx = tid; idx < M_eff * BN; idx += blockDim.x) {
    const int tok = idx / BN;
    const int64_t n = n_cta + idx % BN;
    if (n < a.N) a.partials[(int64_t(blockIdx.y) * a.M + tok) * a.N + n] = part[idx];
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
  for (int idx = tid; idx < M_eff * BN; idx += blockDim.x) {
    const int tok = idx / BN;
    const int64_t n = n_cta + idx % BN;
    if (n >= a.N) continue;
    float v = __ldcg(a.partials + int64_t(tok) * a.N + n);
    for (int s = 1; s < a.S; ++s) v += __ldcg(a.partials + (int64_t(s) * a.M + tok) * a.N + n);
    y[int64_t(tok) * a.sym + n] = f2h_bits<F16>(v);
  }
  if (tid == 0) atomicExch(a.tickets + blockIdx.x, 0u);
}

// ------------------------------------------------------------------ planning

static int gcd_int(int a, int b) {
  while (b) {
    const int t = a % b;
    a = b;
    b = t;
  }
  return a;
}

static int g_ovr_wn = 0, g_ovr_wk = 0, g_ovr_s = 0;

void set_skinny_override(int wn, int wk, int splits) {
  g_ovr_wn = wn;
  g_ovr_wk = wk;
  g_ovr_s = splits;
}

// Chooses the decomposition; shared by the workspace-size query and the launch.
// K is cut into units of L = 32*SPS k-values (INT4) or 32 (W16); a warp owns
// u_w consecutive units, a CTA WK warps along K, a cluster S CTAs along K.
SkinnyPlan plan_skinny(int64_t M, int64_t N, int64_t K, int G, bool int4, int num_sms) {
  SkinnyPlan p{};
  p.MT = M <= 8 ? 1 : 2;
  p.L = int4 ? 32 * gcd_int(G / 32, 8) : 32;
  const int unit = p.L;
  const int64_t units = int4 ? K / unit : (K + 31) / 32;
  const int max_warps = int4 ? 16 : 8;
  p.WN = 1;
  if (g_ovr_wn == 1 || g_ovr_wn == 2 || g_ovr_wn == 4 || g_ovr_wn == 8 || g_ovr_wn == 16) p.WN = g_ovr_wn;
  if (p.WN > max_warps) p.WN = max_warps;
  const int64_t ncol = cdiv(N, 32);
  const int64_t want_warps = int64_t(num_sms) * 6;
  auto next_divisor_down = [&](int64_t v) {
    while (v > 1 && units % v) --v;
    return v < 1 ? int64_t(1) : v;
  };
  // ~512 k per warp, fewer while the grid has too few warps.
  int64_t u_w = next_divisor_down(std::max<int64_t>(1, 512 / unit));
  while (u_w > 1 && ncol * (units / u_w) < want_warps) u_w = next_divisor_down(u_w / 2);
  const int64_t chunks = units / u_w;
  int WK = 1;
  const int wk_max = std::min(8, max_warps / p.WN);
  while (2 * WK <= wk_max && chunks % (2 * WK) == 0) WK *= 2;
  if (g_ovr_wk > 0 && g_ovr_wk <= wk_max && chunks % g_ovr_wk == 0) WK = g_ovr_wk;
  int64_t S = chunks / WK;
  if (g_ovr_s > 0 && chunks % (int64_t(g_ovr_s) * WK) == 0) {
    // fewer splits than chunks/WK means longer warps
    const int64_t f = chunks / (int64_t(g_ovr_s) * WK);
    u_w *= f;
    S = g_ovr_s;
  }
  p.WK = WK;
  p.S = int(S);
  p.KW = int(u_w * unit);
  p.KC = p.KW * WK;
  p.ntiles = cdiv(N, 32 * p.WN);
  p.mode = S == 1 ? 0 : (S <= 8 ? 1 : 2);
  if (p.mode == 2 && p.ntiles > kMaxTickets) p.mode = 3;  // unsupported: reported as an error
  const int MP = p.MT * 8;
  const int BN = 32 * p.WN;
  const int sps = p.L / 32;
  const int nseg = 4 >= sps ? 4 / sps : 1;
  const size_t ring = int4 ? size_t(4) * (4 * 512 + nseg * 512) : 0;  // RING stages x STAGE_B per warp
  p.smem_bytes = size_t(p.WN) * WK * ring + size_t(WK * MP * BN + MP * BN) * 4;
  p.partial_bytes = p.mode == 2 ? size_t(S) * size_t(M) * size_t(N) * 4 : 0;
  p.xstride = 0;
  return p;
}

size_t skinny_workspace_bytes(const SkinnyPlan& p) {
  if (p.mode != 2) return 0;
  return kTicketBytes + p.partial_bytes;
}

template <int MT, bool INT4, bool F16, int SPS>
static cudaError_t launch_one(const SkinnyArgs& a, const SkinnyPlan& p, cudaStream_t stream) {
  auto kern = skinny_kernel<MT, INT4, F16, SPS>;
  static size_t configured = 48 * 1024;  // dynamic shared memory this instance may use
  if (p.smem_bytes > configured) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(p.smem_bytes));
    if (e != cudaSuccess) return e;
    configured = p.smem_bytes;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(p.ntiles), unsigned(p.S));
  cfg.blockDim = dim3(unsigned(32 * p.WN * p.WK));
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (a.mode == 1) {
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

template <int MT, bool INT4, bool F16>
static cudaError_t launch_sps(const SkinnyArgs& a, const SkinnyPlan& p, cudaStream_t stream) {
  if constexpr (!INT4) {
    return launch_one<MT, false, F16, 1>(a, p, stream);
  } else {
    switch (p.L / 32) {
      case 1: return launch_one<MT, true, F16, 1>(a, p, stream);
      case 2: return launch_one<MT, true, F16, 2>(a, p, stream);
      case 4: return launch_one<MT, true, F16, 4>(a, p, stream);
      default: return launch_one<MT, true, F16, 8>(a, p, stream);
    }
  }
}

template <bool INT4, bool F16>
static cudaError_t launch_mt(const SkinnyArgs& a, const SkinnyPlan& p, cudaStream_t stream) {
  return p.MT == 1 ? launch_sps<1, INT4, F16>(a, p, stream) : launch_sps<2, INT4, F16>(a, p, stream);
}

cudaError_t launch_skinny(bool int4, bool f16, const void* x, int64_t M, int64_t K, int64_t sxm, int64_t sxk,
                          const void* w, int64_t N, int64_t sw0, int64_t sw1, const uint16_t* sc,
                          const uint16_t* zr, int64_t ssg, int G, void* y, int64_t sym, void* ws,
                          const SkinnyPlan& p, bool pdl, cudaStream_t stream) {
  if (p.mode == 3) return cudaErrorInvalidConfiguration;
  SkinnyArgs a{};
  a.x = x; a.sxm = sxm; a.sxk = sxk;
  a.w = w; a.sw0 = sw0; a.sw1 = sw1;
  a.sc = sc; a.zr = zr; a.ssg = ssg;
  a.y = y; a.sym = sym;
  a.M = int(M); a.N = int(N); a.K = int(K); a.G = G;
  a.S = p.S; a.KC = p.KC; a.KW = p.KW; a.WN = p.WN; a.WK = p.WK;
  a.mode = p.mode;
  a.pdl = pdl ? 1 : 0;
  if (p.mode == 2) {
    a.tickets = static_cast<unsigned int*>(ws);
    a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kTicketBytes);
  }
  if (int4) {
    a.vec_w = (reinterpret_cast<uintptr_t>(w) % 16 == 0) && (sw0 % 4 == 0) && (N % 4 == 0);
    a.vec_s = (reinterpret_cast<uintptr_t>(sc) % 8 == 0) && (reinterpret_cast<uintptr_t>(zr) % 8 == 0) &&
              (ssg % 4 == 0) && (N % 4 == 0);
  } else {
    a.vec_w = (reinterpret_cast<uintptr_t>(w) % 16 == 0) && (sw1 == 1) && (sw0 % 8 == 0);
  }
  a.vec_x = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (sxk == 1) && (sxm % 8 == 0 || M == 1);
  if (int4) return cudaErrorInvalidValue;  // INT4 weights go through launch_w4 (gemv_w4.cu)
  return f16 ? launch_mt<false, true>(a, p, stream) : launch_mt<false, false>(a, p, stream);
}

}  // namespace i4b
