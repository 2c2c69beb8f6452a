// Decode-step glue around the W4A16 projections of a Llama layer, one launch each.
//
// The reference runs these steps as transformers' torch ops (eager, or captured
// in a CUDA graph, benchmarks/eval_llama.py:121-183): about forty small kernels
// per layer between the four matmuls.  Here they are four kernels, each
// reproducing transformers' bf16 rounding points:
//   add_rmsnorm   h = bf16(h + delta);  x = bf16(w * bf16(h * rsqrt(mean(h^2) + eps)))   (LlamaRMSNorm)
//   rope_kv       q, k = bf16(bf16(t * cos) + bf16(rotate_half(t) * sin)); k, v -> cache[pos] (apply_rotary_pos_emb)
//   decode_attn   softmax(q . K^T * scale) . V over cache positions 0..pos, GQA, fp32 inside  (scaled_dot_product_attention)
//   silu_mul      y = bf16(bf16(silu(g)) * u)                                              (LlamaMLP)
//   argmax        greedy next token: first index of the row maximum                       (torch.argmax)
// All take device pointers and a device-side position, so a decode step that
// uses them can be captured in a CUDA graph and replayed for every position.
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace i4b {

namespace {

__device__ __forceinline__ float bf(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }
__device__ __forceinline__ uint16_t to_bf(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }

// Sum over the block (blockDim.x a multiple of 32, <= 1024); every thread gets the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.0f;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = red[0];
  for (int i = 1; i < nw; ++i) m = fmaxf(m, red[i]);
  return m;
}

// One CTA per row; H a multiple of 8; each thread owns 8-element chunks.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(uint16_t* __restrict__ h, const uint16_t* __restrict__ delta,
                                                          const uint16_t* __restrict__ w, uint16_t* __restrict__ out,
                                                          int H, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  uint16_t* hr = h + row * H;
  const uint16_t* dr = delta ? delta + row * H : nullptr;
  float ss = 0.0f;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    uint4 hv = *reinterpret_cast<const uint4*>(hr + c);
    if (dr) {
      const uint4 dv = *reinterpret_cast<const uint4*>(dr + c);
      const uint32_t* a = reinterpret_cast<const uint32_t*>(&hv);
      const uint32_t* b = reinterpret_cast<const uint32_t*>(&dv);
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint16_t lo = to_bf(bf(uint16_t(a[i])) + bf(uint16_t(b[i])));
        const uint16_t hi = to_bf(bf(uint16_t(a[i] >> 16)) + bf(uint16_t(b[i] >> 16)));
        o[i] = uint32_t(lo) | (uint32_t(hi) << 16);
      }
      hv = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(hr + c) = hv;
    }
    const uint32_t* a = reinterpret_cast<const uint32_t*>(&hv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = bf(uint16_t(a[i])), hi = bf(uint16_t(a[i] >> 16));
      ss = fmaf(lo, lo, ss);
      ss = fmaf(hi, hi, ss);
    }
  }
  const float inv = rsqrtf(block_sum(ss, red) / float(H) + eps);
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    const uint4 hv = *reinterpret_cast<const uint4*>(hr + c);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
    const uint32_t* a = reinterpret_cast<const uint32_t*>(&hv);
    const uint32_t* b = reinterpret_cast<const uint32_t*>(&wv);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint16_t lo = to_bf(bf(uint16_t(b[i])) * bf(to_bf(bf(uint16_t(a[i])) * inv)));
      const uint16_t hi = to_bf(bf(uint16_t(b[i] >> 16)) * bf(to_bf(bf(uint16_t(a[i] >> 16)) * inv)));
      o[i] = uint32_t(lo) | (uint32_t(hi) << 16);
    }
    *reinterpret_cast<uint4*>(out + row * H + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// One warp per (token, head) of the stacked qkv row; lane i owns dims i and i + 32 (head_dim 64).
__global__ void __launch_bounds__(128) rope_kv_kernel(const uint16_t* __restrict__ qkv, const uint16_t* __restrict__ cosT,
                                                      const uint16_t* __restrict__ sinT, const int64_t* __restrict__ pos,
                                                      uint16_t* __restrict__ q_out, uint16_t* __restrict__ kc,
                                                      uint16_t* __restrict__ vc, int B, int nq, int nkv, int max_seq) {
  constexpr int HD = 64;
  const int heads = nq + 2 * nkv;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= B * heads) return;
  const int b = gw / heads, hh = gw % heads, lane = threadIdx.x & 31;
  const int64_t p = *pos;
  if (p < 0 || p >= max_seq) return;  // outside the cache: nothing is written
  const uint16_t* src = qkv + int64_t(b) * heads * HD + int64_t(hh) * HD;
  const float x0 = bf(src[lane]), x1 = bf(src[lane + 32]);
  if (hh >= nq + nkv) {  // value head: straight into the cache
    uint16_t* dst = vc + ((int64_t(b) * nkv + (hh - nq - nkv)) * max_seq + p) * HD;
    dst[lane] = src[lane];
    dst[lane + 32] = src[lane + 32];
    return;
  }
  const float c0 = bf(cosT[p * HD + lane]), c1 = bf(cosT[p * HD + lane + 32]);
  const float s0 = bf(sinT[p * HD + lane]), s1 = bf(sinT[p * HD + lane + 32]);
  // rotate_half: (-x[32:], x[:32])
  const uint16_t y0 = to_bf(bf(to_bf(x0 * c0)) + bf(to_bf(-x1 * s0)));
  const uint16_t y1 = to_bf(bf(to_bf(x1 * c1)) + bf(to_bf(x0 * s1)));
  uint16_t* dst = hh < nq ? q_out + (int64_t(b) * nq + hh) * HD
                          : kc + ((int64_t(b) * nkv + (hh - nq)) * max_seq + p) * HD;
  dst[lane] = y0;
  dst[lane + 32] = y1;
}

// Split-sequence decode attention: the cached positions 0..pos of one (query head, token) are cut into NS
// consecutive chunks, one per CTA of a (NS, 1, 1) cluster.  Each CTA computes its chunk's scores
// (four threads per position, 16 dims each), its local max m_r, sum l_r = sum exp(s - m_r) and the
// unnormalised o_r = sum exp(s - m_r) v; rank 0 then combines the NS partials in rank order through
// distributed shared memory:  out = sum_r o_r e^(m_r - m) / sum_r l_r e^(m_r - m),  m = max_r m_r.
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxChunk = 6144;  // positions per CTA held as scores in shared memory

__global__ void __launch_bounds__(kAttnThreads) decode_attn_kernel(const uint16_t* __restrict__ q,
                                                                   const uint16_t* __restrict__ kc,
                                                                   const uint16_t* __restrict__ vc,
                                                                   const int64_t* __restrict__ pos,
                                                                   uint16_t* __restrict__ out, int nq, int nkv,
                                                                   int max_seq, float scale) {
  constexpr int HD = 64;
  extern __shared__ float sc[];  // [chunk] scores, then [16][64] partial sums of V
  __shared__ float red[32];
  __shared__ float qs[HD];
  __shared__ float part_o[HD];   // this CTA's unnormalised output, read by rank 0
  __shared__ float part_ml[2];   // this CTA's (m_r, l_r)
  const int NS = int(gridDim.x) / nq;
  const int rank = int(cluster_ctarank());
  const int head = int(blockIdx.x) / NS, b = blockIdx.y, tid = threadIdx.x;
  const int kvh = head / (nq / nkv);
  const int64_t p = *pos;
  const int L = p < 0 ? 0 : (p >= max_seq ? max_seq : int(p) + 1);  // never reads past the cache
  const int chunk = (L + NS - 1) / NS;
  const int i0 = rank * chunk, i1 = min(L, i0 + chunk);
  const int n = i1 > i0 ? i1 - i0 : 0;
  if (tid < HD) qs[tid] = bf(q[(int64_t(b) * nq + head) * HD + tid]);
  __syncthreads();
  const uint16_t* K = kc + ((int64_t(b) * nkv + kvh) * max_seq + i0) * HD;
  const uint16_t* V = vc + ((int64_t(b) * nkv + kvh) * max_seq + i0) * HD;

  // scores: thread (position i = t / 4, quarter qd = t % 4) dots 16 dims; quarters meet by shuffle
  float mx = -INFINITY;
  const int qd = tid & 3;
  for (int i = tid >> 2; i < ((n + 31) & ~31); i += kAttnThreads / 4) {  // whole warps stay in the loop
    float d = 0.0f;
    if (i < n) {
      const uint4* kr = reinterpret_cast<const uint4*>(K + int64_t(i) * HD + 16 * qd);
      const uint4 k0 = __ldg(kr), k1 = __ldg(kr + 1);
      const uint32_t u[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        d = fmaf(qs[16 * qd + 2 * e], bf(uint16_t(u[e])), d);
        d = fmaf(qs[16 * qd + 2 * e + 1], bf(uint16_t(u[e] >> 16)), d);
      }
    }
    d += __shfl_xor_sync(0xFFFFFFFFu, d, 1);
    d += __shfl_xor_sync(0xFFFFFFFFu, d, 2);
    if (i < n && qd == 0) {
      d *= scale;
      sc[i] = d;
      mx = fmaxf(mx, d);
    }
  }
  mx = block_max(mx, red);
  float sum = 0.0f;
  for (int i = tid; i < n; i += kAttnThreads) {
    const float e = expf(sc[i] - mx);
    sc[i] = e;
    sum += e;
  }
  sum = block_sum(sum, red);  // (synchronises: all probabilities written)
  // o_r: thread t owns dims 8*(t%8)..+7 of positions t/8, t/8 + 16, ... (16 position phases)
  const int dg = tid & 7, ph = tid >> 3;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
  const uint16_t* vp = V + 8 * dg;
  int i = ph;
  for (; i + 48 < n; i += 64) {  // four positions in flight
    uint4 v4[4];
    float pr[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v4[u] = __ldg(reinterpret_cast<const uint4*>(vp + int64_t(i + 16 * u) * HD));
      pr[u] = sc[i + 16 * u];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t w[4] = {v4[u].x, v4[u].y, v4[u].z, v4[u].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[2 * e] = fmaf(pr[u], bf(uint16_t(w[e])), acc[2 * e]);
        acc[2 * e + 1] = fmaf(pr[u], bf(uint16_t(w[e] >> 16)), acc[2 * e + 1]);
      }
    }
  }
  for (; i < n; i += 16) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(vp + int64_t(i) * HD));
    const float pr = sc[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[2 * e] = fmaf(pr, bf(uint16_t(w[e])), acc[2 * e]);
      acc[2 * e + 1] = fmaf(pr, bf(uint16_t(w[e] >> 16)), acc[2 * e + 1]);
    }
  }
  float* part = sc + kAttnMaxChunk;
#pragma unroll
  for (int e = 0; e < 8; ++e) part[ph * HD + 8 * dg + e] = acc[e];
  __syncthreads();
  if (tid < HD) {
    float v = 0.0f;
    for (int k = 0; k < 16; ++k) v += part[k * HD + tid];
    part_o[tid] = v;
  }
  if (tid == 0) {
    part_ml[0] = n > 0 ? mx : -INFINITY;
    part_ml[1] = n > 0 ? sum : 0.0f;
  }
  cluster_sync();
  if (rank == 0 && tid < HD) {
    float mr[8], lr[8], orr[8];  // all remote loads in flight first, then combined in rank order
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      mr[r] = r < NS ? ld_shared_cluster_f32(mapa_shared(smem_u32(&part_ml[0]), uint32_t(r))) : -INFINITY;
      lr[r] = r < NS ? ld_shared_cluster_f32(mapa_shared(smem_u32(&part_ml[1]), uint32_t(r))) : 0.0f;
      orr[r] = r < NS ? ld_shared_cluster_f32(mapa_shared(smem_u32(&part_o[tid]), uint32_t(r))) : 0.0f;
    }
    float m = -INFINITY;
#pragma unroll
    for (int r = 0; r < 8; ++r) m = fmaxf(m, mr[r]);
    float num = 0.0f, den = 0.0f;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const float w = lr[r] > 0.0f ? expf(mr[r] - m) : 0.0f;
      num = fmaf(orr[r], w, num);
      den = fmaf(lr[r], w, den);
    }
    out[(int64_t(b) * nq + head) * HD + tid] = L > 0 ? to_bf(num / den) : uint16_t(0);
  }
  cluster_sync();  // no CTA leaves while rank 0 may still read its shared memory
}

// Row-wise argmax of bf16 values (first index of the maximum, as torch.argmax): one CTA per row.
__global__ void __launch_bounds__(1024) argmax_kernel(const uint16_t* __restrict__ x, int64_t n, int64_t* __restrict__ out) {
  const int64_t row = blockIdx.x;
  float best;
  int64_t bi;
  block_row_argmax(x + row * n, n, &best, &bi);
  if (threadIdx.x == 0) out[row] = bi < n ? bi : 0;
}

__global__ void silu_mul_kernel(const uint16_t* __restrict__ gu, uint16_t* __restrict__ y, int B, int I) {
  const int64_t total = int64_t(B) * I;
  for (int64_t e = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8; e < total;
       e += int64_t(gridDim.x) * blockDim.x * 8) {
    const int64_t b = e / I, i = e % I;
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + b * 2 * I + i);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + b * 2 * I + I + i);
    const uint32_t* g = reinterpret_cast<const uint32_t*>(&gv);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&uv);
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g0 = bf(uint16_t(g[k])), g1 = bf(uint16_t(g[k] >> 16));
      const float s0 = bf(to_bf(g0 / (1.0f + expf(-g0)))), s1 = bf(to_bf(g1 / (1.0f + expf(-g1))));
      o[k] = uint32_t(to_bf(s0 * bf(uint16_t(u[k])))) | (uint32_t(to_bf(s1 * bf(uint16_t(u[k] >> 16)))) << 16);
    }
    *reinterpret_cast<uint4*>(y + e) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace

cudaError_t launch_add_rmsnorm(uint16_t* h, const uint16_t* delta, const uint16_t* w, uint16_t* out, int rows, int H,
                               float eps, cudaStream_t s) {
  add_rmsnorm_kernel<<<rows, 256, 0, s>>>(h, delta, w, out, H, eps);
  return cudaGetLastError();
}

cudaError_t launch_rope_kv(const uint16_t* qkv, const uint16_t* cosT, const uint16_t* sinT, const int64_t* pos,
                           uint16_t* q_out, uint16_t* kc, uint16_t* vc, int B, int nq, int nkv, int max_seq,
                           cudaStream_t s) {
  const int warps = B * (nq + 2 * nkv);
  rope_kv_kernel<<<(warps + 3) / 4, 128, 0, s>>>(qkv, cosT, sinT, pos, q_out, kc, vc, B, nq, nkv, max_seq);
  return cudaGetLastError();
}

cudaError_t launch_decode_attn(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int64_t* pos,
                               uint16_t* out, int B, int nq, int nkv, int max_seq, float scale, cudaStream_t s) {
  // sequence splits: one CTA per 64 cache positions, at most a portable cluster of 8
  int ns = (max_seq + 63) / 64;
  ns = ns < 1 ? 1 : (ns > 8 ? 8 : ns);
  const size_t smem = (size_t(kAttnMaxChunk) + 16 * 64) * sizeof(float);
  const cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(decode_attn_kernel), smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(nq * ns), unsigned(B));
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(ns);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_attn_kernel, q, kc, vc, pos, out, nq, nkv, max_seq, scale);
}

cudaError_t launch_argmax(const uint16_t* x, int64_t rows, int64_t n, int64_t* out, cudaStream_t s) {
  argmax_kernel<<<unsigned(rows), 1024, 0, s>>>(x, n, out);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const uint16_t* gu, uint16_t* y, int B, int I, cudaStream_t s) {
  const int64_t chunks = (int64_t(B) * I + 7) / 8;
  const int blocks = int(std::min<int64_t>((chunks + 255) / 256, 148 * 8));
  silu_mul_kernel<<<blocks, 256, 0, s>>>(gu, y, B, I);
  return cudaGetLastError();
}

}  // namespace i4b
