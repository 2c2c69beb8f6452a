// Small-M (M <= 16) W16A16 kernel (full-precision weights): the w16a16_matmul decode GEMV and small-batch
// split-K path.  INT4 weights are served by gemv_w4.cu.
//
// Replaces the reference's full-precision branch of _gemv_kernel (int4_triton/gemm.py:185-220, W_INT4 off)
// and of its small-M split-K pair _matmul_kernel + _reduce_split_k (gemm.py:74-182, launched at
// gemm.py:265-299) with ONE launch per matmul.
//
// Work split.  grid = (ceil(N / BN), S), cluster (1, S, 1) when 1 < S <= 8.
// A CTA owns BN = 32*WN output columns and the K-range [y*KC, (y+1)*KC);
// warp (wn, wk) owns 32 columns and KW = KC/WK consecutive k.  Every operand
// is fetched by the warp that uses it, with no block barrier before the main loop:
//   * weights: batches of 32-k steps loaded with 128-bit register loads that
//     bypass L1 (lane (r, c) loads 8 consecutive k of rows 16t + r and
//     16t + 8 + r: exactly its A fragments of mma.m16n8k16);
//   * activations: 16 bytes (8 consecutive k) per lane and token row, from L1/L2.
// B = activations, fp32 accumulators: y = sum_k x_k w_k, the reference's
// arithmetic up to fp32 summation order.
//
// Reduction.  Warps sharing columns add through shared memory in fixed warp
// order.  K-splits inside a cluster add through distributed shared memory in
// fixed rank order.  More than 8 splits fall back to fp32 partials in the
// caller's workspace: the last CTA of a column tile (atomic ticket, no
// spinning) adds them in split order and resets the ticket.  Every path is
// bit-identical from run to run.
//
// Programmatic dependent launch (opt-in): the first weight batch is loaded
// before griddepcontrol.wait, activations after it.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace i4b {

struct SkinnyArgs {
  const void* x;
  int64_t sxm, sxk;
  const void* w;   // weights [N, K]
  int64_t sw0;     // stride between rows n
  int64_t sw1;     // stride along k
  void* y;
  int64_t sym;
  float* partials;
  unsigned int* tickets;
  int M, N, K;
  int S, KC, KW, WN, WK;
  int mode;        // 0: S == 1; 1: cluster of S CTAs along K; 2: global tickets
  int vec_w, vec_x;
  int pdl;
};

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

template <int MT, bool F16>
__global__ void __launch_bounds__(256) skinny_kernel(const SkinnyArgs a) {
  constexpr int MP = MT * 8;             // padded token count
  constexpr int CH = MT == 1 ? 8 : 4;    // 32-k steps per weight batch
  extern __shared__ __align__(16) uint8_t smem_b[];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wn = warp % a.WN, wk = warp / a.WN;
  const int r = lane >> 2, c = lane & 3;
  const int BN = 32 * a.WN;
  const int64_t n_cta = int64_t(blockIdx.x) * BN;
  const int64_t nb = n_cta + wn * 32;
  const int64_t k0 = int64_t(blockIdx.y) * a.KC;
  const int64_t kw0 = k0 + wk * a.KW;  // warp's first k
  const int nsteps = a.KW / 32;
  const int M_eff = a.M < MP ? a.M : MP;
  float* smem_f = reinterpret_cast<float*>(smem_b);

  // register batches of weights loaded straight from global memory
  uint4 wv[CH][4];
  auto load_batch = [&](int cs) {
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
  };

  load_batch(0);          // weights do not depend on the previous kernel: start them first
  if (a.pdl) pdl_wait();  // activations are produced by the previous kernel

  float acc[2][MT][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[t][mt][e] = 0.0f;
  // lane's activation pointer: token mt*8 + r, k = kw0 + step*32 + 8c (+8 values)
  const uint16_t* xlane = static_cast<const uint16_t*>(a.x) + int64_t(r) * a.sxm + (kw0 + 8 * c) * a.sxk;
  const int64_t xstep = 32 * a.sxk;
  const bool x_fast = a.vec_x && (a.K % 32 == 0);

  for (int cs = 0; cs < nsteps; cs += CH) {
    if (cs > 0) load_batch(cs);
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
        xv[i][mt] = make_uint4(u[0], u[1], u[2], u[3]);
      }
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      if (cs + i >= nsteps) break;
      uint32_t af[2][2][4];  // [row tile][k16 step][reg]
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const uint4 lo = wv[i][2 * t], hi = wv[i][2 * t + 1];
        af[t][0][0] = lo.x; af[t][0][1] = hi.x; af[t][0][2] = lo.y; af[t][0][3] = hi.y;
        af[t][1][0] = lo.z; af[t][1][1] = hi.z; af[t][1][2] = lo.w; af[t][1][3] = hi.w;
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint4 b = xv[i][mt];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          mma_16816<F16>(acc[t][mt], af[t][0], b.x, b.y);
          mma_16816<F16>(acc[t][mt], af[t][1], b.z, b.w);
        }
      }
    }
  }
  // ---- outputs: acc[t][mt][e] is (token mt*8 + 2c + (e & 1), local column col(t, e >> 1))
  auto col_of = [&](int t, int half) { return wn * 32 + 16 * t + 8 * half + r; };
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

static int g_ovr_wn = 0, g_ovr_wk = 0, g_ovr_s = 0;

void set_skinny_override(int wn, int wk, int splits) {
  g_ovr_wn = wn;
  g_ovr_wk = wk;
  g_ovr_s = splits;
}

// Chooses the decomposition; shared by the workspace-size query and the launch.
// K is cut into units of 32; a warp owns u_w consecutive units, a CTA WK warps along K, a cluster S CTAs
// along K.
SkinnyPlan plan_skinny(int64_t M, int64_t N, int64_t K, int num_sms) {
  SkinnyPlan p{};
  p.MT = M <= 8 ? 1 : 2;
  p.L = 32;
  const int64_t units = (K + 31) / 32;
  const int max_warps = 8;
  p.WN = 1;
  if (g_ovr_wn == 1 || g_ovr_wn == 2 || g_ovr_wn == 4 || g_ovr_wn == 8) p.WN = g_ovr_wn;
  const int64_t ncol = cdiv(N, 32);
  const int64_t want_warps = int64_t(num_sms) * 6;
  auto next_divisor_down = [&](int64_t v) {
    while (v > 1 && units % v) --v;
    return v < 1 ? int64_t(1) : v;
  };
  // ~512 k per warp, fewer while the grid has too few warps.
  int64_t u_w = next_divisor_down(16);
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
  p.KW = int(u_w * 32);
  p.KC = p.KW * WK;
  p.ntiles = cdiv(N, 32 * p.WN);
  p.mode = S == 1 ? 0 : (S <= 8 ? 1 : 2);
  if (p.mode == 2 && p.ntiles > kMaxTickets) p.mode = 3;  // unsupported: reported as an error
  const int MP = p.MT * 8;
  const int BN = 32 * p.WN;
  p.smem_bytes = size_t(WK * MP * BN + MP * BN) * 4;
  p.partial_bytes = p.mode == 2 ? size_t(S) * size_t(M) * size_t(N) * 4 : 0;
  p.xstride = 0;
  return p;
}

size_t skinny_workspace_bytes(const SkinnyPlan& p) {
  if (p.mode != 2) return 0;
  return kTicketBytes + p.partial_bytes;
}

template <int MT, bool F16>
static cudaError_t launch_one(const SkinnyArgs& a, const SkinnyPlan& p, cudaStream_t stream) {
  auto kern = skinny_kernel<MT, F16>;
  if (p.smem_bytes > 48 * 1024) {
    const cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), p.smem_bytes);
    if (e != cudaSuccess) return e;
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

cudaError_t launch_skinny(bool f16, const void* x, int64_t M, int64_t K, int64_t sxm, int64_t sxk, const void* w,
                          int64_t N, int64_t sw0, int64_t sw1, void* y, int64_t sym, void* ws, const SkinnyPlan& p,
                          bool pdl, cudaStream_t stream) {
  if (p.mode == 3) return cudaErrorInvalidConfiguration;
  SkinnyArgs a{};
  a.x = x; a.sxm = sxm; a.sxk = sxk;
  a.w = w; a.sw0 = sw0; a.sw1 = sw1;
  a.y = y; a.sym = sym;
  a.M = int(M); a.N = int(N); a.K = int(K);
  a.S = p.S; a.KC = p.KC; a.KW = p.KW; a.WN = p.WN; a.WK = p.WK;
  a.mode = p.mode;
  a.pdl = pdl ? 1 : 0;
  if (p.mode == 2) {
    a.tickets = static_cast<unsigned int*>(ws);
    a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kTicketBytes);
  }
  a.vec_w = (reinterpret_cast<uintptr_t>(w) % 16 == 0) && (sw1 == 1) && (sw0 % 8 == 0);
  a.vec_x = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (sxk == 1) && (sxm % 8 == 0 || M == 1);
  if (p.MT == 1) return f16 ? launch_one<1, true>(a, p, stream) : launch_one<1, false>(a, p, stream);
  return f16 ? launch_one<2, true>(a, p, stream) : launch_one<2, false>(a, p, stream);
}

}  // namespace i4b
