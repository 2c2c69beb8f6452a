// Group-wise asymmetric INT4 quantize/pack and dequantize kernels.
//
// Bit-exact restatement, on the GPU, of the reference's torch implementation
// quantize_int4_ref (int4_triton/quantize.py:102-117):
//   wmax = max(max(w_group), 0); wmin = min(min(w_group), 0)
//   scale = (wmax - wmin) / 15; scale = 1 if scale == 0 (before rounding)
//   scale = fp32(fp16_rne(scale))
//   zero  = clamp(floor(-wmin / scale + 0.5), 0, 15)
//   q     = clamp(floor(w / scale + 0.5) + zero, 0, 15)
//   word[k8, n] = sum_i q[n, 8*k8 + i] << 4i   (int32 wrap-around)
// Every division is the IEEE round-to-nearest __fdiv_rn and every add is a
// separate __fadd_rn, so no reciprocal or FMA changes a rounding.  Groups with
// a non-finite or underflowing scale (and non-finite weights) take a slow path
// that follows x86 NaN rules, which is what the reference produces.
//
// Layout: W[N, K] row n, column k at w + n*stride_wn + k*stride_wk.
// Fast kernel (G a power of two >= 32): a CTA of 256 threads owns 32 rows x
// max(G, 256) columns; thread (row = t/8, sub = t%8) owns 32 consecutive
// columns = 4 packed words, so a group spans G/32 aligned lanes (G <= 256) and
// its max/min is a segmented xor-shuffle reduction.  Words are transposed
// through shared memory so qweight rows (128 B per 32 n) are written coalesced.
// Generic kernel (any G multiple of 8): one warp per (row, group).
#include "common.cuh"

namespace i4b {

static __device__ unsigned int g_quant_err = 0;  // reserved (no waits in this file)

template <int DT>
struct Loader {
  // Loads 8 consecutive elements of row n starting at column k as fp32.
  template <bool VEC>
  __device__ __forceinline__ static void load8(const void* w, int64_t n, int64_t k, int64_t swn, int64_t swk,
                                               float (&v)[8]) {
    if constexpr (DT == I4B_F32) {
      const float* p = static_cast<const float*>(w) + n * swn + k * swk;
      if constexpr (VEC) {
        float4 a = __ldg(reinterpret_cast<const float4*>(p));
        float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __ldg(p + i * swk);
      }
    } else {
      const uint16_t* p = static_cast<const uint16_t*>(w) + n * swn + k * swk;
      if constexpr (VEC) {
        uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
        const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[2 * i] = Elem<DT>::to_f32(uint16_t(u[i] & 0xFFFFu));
          v[2 * i + 1] = Elem<DT>::to_f32(uint16_t(u[i] >> 16));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = Elem<DT>::to_f32(__ldg(p + i * swk));
      }
    }
  }
};

struct GroupParams {
  float scale;     // fp16-rounded scale as fp32
  float zero;      // zero point (may be NaN on degenerate groups)
  uint16_t s16, z16;
  bool fast;       // scale finite and non-zero, zero not NaN
};

__device__ __forceinline__ GroupParams group_params(float vmax, float vmin) {
  GroupParams gp;
  float scale = x86_div(x86_sub(vmax, vmin), 15.0f);
  if (scale == 0.0f) scale = 1.0f;
  gp.s16 = f32_to_f16_bits_x86(scale);
  gp.scale = f16_bits_to_f32_x86(gp.s16);
  gp.zero = clamp_nan(x86_floor(x86_add(x86_div(f_neg(vmin), gp.scale), 0.5f)), 0.0f, 15.0f);
  gp.z16 = f32_to_f16_bits_x86(gp.zero);
  gp.fast = isfinite(gp.scale) && gp.scale != 0.0f && !f_isnan(gp.zero);
  return gp;
}

// Nibble bits for one element (before the shift); INT_MIN for NaN, as the x86 cast gives.
__device__ __forceinline__ uint32_t quant_bits(float w, const GroupParams& gp) {
  if (gp.fast && isfinite(w)) {
    float q = __fadd_rn(floorf(__fadd_rn(__fdiv_rn(w, gp.scale), 0.5f)), gp.zero);
    q = q < 0.0f ? 0.0f : (q > 15.0f ? 15.0f : q);
    return static_cast<uint32_t>(static_cast<int32_t>(q));
  }
  float q = x86_add(x86_floor(x86_add(x86_div(w, gp.scale), 0.5f)), gp.zero);
  return x86_f2i_bits(clamp_nan(q, 0.0f, 15.0f));
}

__device__ __forceinline__ uint32_t pack8(const float (&v)[8], const GroupParams& gp) {
  uint32_t word = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) word += quant_bits(v[i], gp) << (4 * i);  // uint32 wrap == int32 wrap
  return word;
}

template <int DT, bool VEC>
__global__ void __launch_bounds__(256) quantize_pow2_kernel(const void* __restrict__ w, int64_t N, int64_t K,
                                                            int64_t swn, int64_t swk, int G,
                                                            uint32_t* __restrict__ qw, uint16_t* __restrict__ sc,
                                                            uint16_t* __restrict__ zr) {
  __shared__ uint32_t tile[32][33];  // [k8 within chunk][row]
  const int t = threadIdx.x;
  const int row = t >> 3, sub = t & 7;
  const int64_t n = int64_t(blockIdx.x) * 32 + row;
  const bool nvalid = n < N;
  const int64_t span = G > 256 ? G : 256;      // columns owned by this CTA
  const int64_t kbase = int64_t(blockIdx.y) * span;
  const int nchunks = int(span / 256);
  const int lanes_per_group = G >= 256 ? 8 : G / 32;

  float v[4][8];  // chunk kept in registers when nchunks == 1
  float vmax = 0.0f, vmin = 0.0f;
  for (int c = 0; c < nchunks; ++c) {
    const int64_t k0 = kbase + int64_t(c) * 256 + sub * 32;
    if (nvalid && k0 < K) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        Loader<DT>::template load8<VEC>(w, n, k0 + 8 * j, swn, swk, v[j]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          vmax = max_nan(vmax, v[j][i]);
          vmin = min_nan(vmin, v[j][i]);
        }
      }
    }
  }
  for (int o = 1; o < lanes_per_group; o <<= 1) {
    vmax = max_nan(vmax, __shfl_xor_sync(0xFFFFFFFFu, vmax, o));
    vmin = min_nan(vmin, __shfl_xor_sync(0xFFFFFFFFu, vmin, o));
  }
  const GroupParams gp = group_params(vmax, vmin);
  if (nvalid && (sub % lanes_per_group) == 0) {
    const int64_t k0 = kbase + sub * 32;
    if (k0 < K) {
      const int64_t g = k0 / G;
      sc[g * N + n] = gp.s16;
      zr[g * N + n] = gp.z16;
    }
  }
  for (int c = 0; c < nchunks; ++c) {
    const int64_t k0 = kbase + int64_t(c) * 256 + sub * 32;
    if (nvalid && k0 < K) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (nchunks > 1) Loader<DT>::template load8<VEC>(w, n, k0 + 8 * j, swn, swk, v[j]);
        tile[sub * 4 + j][row] = pack8(v[j], gp);
      }
    }
    __syncthreads();
    const int64_t k8base = (kbase + int64_t(c) * 256) / 8;
    const int64_t nn = int64_t(blockIdx.x) * 32 + (t & 31);
    for (int r = t >> 5; r < 32; r += 8) {
      const int64_t k8 = k8base + r;
      if (k8 * 8 < K && nn < N) qw[k8 * N + nn] = tile[r][t & 31];
    }
    __syncthreads();
  }
}

// Any G that is a multiple of 8: one warp per (row, group).
template <int DT>
__global__ void __launch_bounds__(256) quantize_generic_kernel(const void* __restrict__ w, int64_t N, int64_t K,
                                                               int64_t swn, int64_t swk, int G,
                                                               uint32_t* __restrict__ qw, uint16_t* __restrict__ sc,
                                                               uint16_t* __restrict__ zr) {
  const int lane = threadIdx.x & 31;
  const int64_t item = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int64_t ngroups = K / G;
  if (item >= N * ngroups) return;  // warp-uniform
  const int64_t n = item / ngroups, g = item % ngroups;
  const int words = G / 8;
  float vmax = 0.0f, vmin = 0.0f;
  float v[8];
  for (int wi = lane; wi < words; wi += 32) {
    Loader<DT>::template load8<false>(w, n, g * G + 8 * wi, swn, swk, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      vmax = max_nan(vmax, v[i]);
      vmin = min_nan(vmin, v[i]);
    }
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    vmax = max_nan(vmax, __shfl_xor_sync(0xFFFFFFFFu, vmax, o));
    vmin = min_nan(vmin, __shfl_xor_sync(0xFFFFFFFFu, vmin, o));
  }
  const GroupParams gp = group_params(vmax, vmin);
  if (lane == 0) {
    sc[g * N + n] = gp.s16;
    zr[g * N + n] = gp.z16;
  }
  for (int wi = lane; wi < words; wi += 32) {
    Loader<DT>::template load8<false>(w, n, g * G + 8 * wi, swn, swk, v);
    qw[(g * words + wi) * N + n] = pack8(v, gp);
  }
}

// W_hat[n, k] = out_dtype(fp32((q - z) * s)); 32 n x 32 k8 tile per CTA, transposed through smem.
template <int ODT>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t* __restrict__ qw,
                                                         const uint16_t* __restrict__ sc,
                                                         const uint16_t* __restrict__ zr, int64_t N, int64_t K,
                                                         int G, void* __restrict__ out) {
  __shared__ uint32_t tile[32][33];  // [k8][n]
  const int t = threadIdx.x;
  const int64_t n0 = int64_t(blockIdx.x) * 32, k80 = int64_t(blockIdx.y) * 32;
  const int64_t K8 = K / 8;
  for (int r = t >> 5; r < 32; r += 8) {
    const int64_t k8 = k80 + r, n = n0 + (t & 31);
    tile[r][t & 31] = (k8 < K8 && n < N) ? __ldg(qw + k8 * N + n) : 0u;
  }
  __syncthreads();
  // thread -> (n = n0 + t/8 .. in 4 passes, k8 = k80 + t%8*4 .. )
  for (int pass = 0; pass < 4; ++pass) {
    const int nl = pass * 8 + (t >> 5);
    const int k8l = t & 31;
    const int64_t n = n0 + nl, k8 = k80 + k8l;
    if (n >= N || k8 >= K8) continue;
    const uint32_t word = tile[k8l][nl];
    const int64_t g = (k8 * 8) / G;
    const float s = f16_bits_to_f32_x86(__ldg(sc + g * N + n));
    const float z = f16_bits_to_f32_x86(__ldg(zr + g * N + n));
    float r[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = __fmul_rn(__fsub_rn(float((word >> (4 * i)) & 0xFu), z), s);
    if constexpr (ODT == I4B_F32) {
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + n * K + k8 * 8);
      o[0] = make_float4(r[0], r[1], r[2], r[3]);
      o[1] = make_float4(r[4], r[5], r[6], r[7]);
    } else {
      uint32_t p[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint16_t lo, hi;
        if constexpr (ODT == I4B_BF16) {
          lo = f32_to_bf16_bits_torch(r[2 * i]);
          hi = f32_to_bf16_bits_torch(r[2 * i + 1]);
        } else {
          lo = f32_to_f16_bits_x86(r[2 * i]);
          hi = f32_to_f16_bits_x86(r[2 * i + 1]);
        }
        p[i] = uint32_t(lo) | (uint32_t(hi) << 16);
      }
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + n * K + k8 * 8) = make_uint4(p[0], p[1], p[2], p[3]);
    }
  }
}

// ------------------------------------------------------------------ host launchers

static bool is_pow2(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }

cudaError_t launch_quantize(const void* w, int dt, int64_t N, int64_t K, int64_t swn, int64_t swk, int G,
                            int32_t* qw, uint16_t* sc, uint16_t* zr, cudaStream_t stream) {
  const int esize = dt == I4B_F32 ? 4 : 2;
  if (is_pow2(G) && G >= 32) {
    const bool vec = swk == 1 && (reinterpret_cast<uintptr_t>(w) % 16 == 0) && ((swn * esize) % 16 == 0);
    const int64_t span = G > 256 ? G : 256;
    dim3 grid(unsigned(cdiv(N, 32)), unsigned(cdiv(K, span)));
    auto* q = reinterpret_cast<uint32_t*>(qw);
#define I4B_QLAUNCH(DT_, VEC_) \
  quantize_pow2_kernel<DT_, VEC_><<<grid, 256, 0, stream>>>(w, N, K, swn, swk, G, q, sc, zr)
    if (dt == I4B_BF16) { if (vec) I4B_QLAUNCH(I4B_BF16, true); else I4B_QLAUNCH(I4B_BF16, false); }
    else if (dt == I4B_F16) { if (vec) I4B_QLAUNCH(I4B_F16, true); else I4B_QLAUNCH(I4B_F16, false); }
    else { if (vec) I4B_QLAUNCH(I4B_F32, true); else I4B_QLAUNCH(I4B_F32, false); }
#undef I4B_QLAUNCH
  } else {
    const int64_t items = N * (K / G);
    dim3 grid(unsigned(cdiv(items, 8)));
    auto* q = reinterpret_cast<uint32_t*>(qw);
    if (dt == I4B_BF16) quantize_generic_kernel<I4B_BF16><<<grid, 256, 0, stream>>>(w, N, K, swn, swk, G, q, sc, zr);
    else if (dt == I4B_F16) quantize_generic_kernel<I4B_F16><<<grid, 256, 0, stream>>>(w, N, K, swn, swk, G, q, sc, zr);
    else quantize_generic_kernel<I4B_F32><<<grid, 256, 0, stream>>>(w, N, K, swn, swk, G, q, sc, zr);
  }
  return cudaGetLastError();
}

cudaError_t launch_dequantize(const int32_t* qw, const uint16_t* sc, const uint16_t* zr, int64_t N, int64_t K, int G,
                              int odt, void* out, cudaStream_t stream) {
  dim3 grid(unsigned(cdiv(N, 32)), unsigned(cdiv(K / 8, 32)));
  auto* q = reinterpret_cast<const uint32_t*>(qw);
  if (odt == I4B_BF16) dequantize_kernel<I4B_BF16><<<grid, 256, 0, stream>>>(q, sc, zr, N, K, G, out);
  else if (odt == I4B_F16) dequantize_kernel<I4B_F16><<<grid, 256, 0, stream>>>(q, sc, zr, N, K, G, out);
  else dequantize_kernel<I4B_F32><<<grid, 256, 0, stream>>>(q, sc, zr, N, K, G, out);
  return cudaGetLastError();
}

unsigned int read_quant_error(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_quant_err, sizeof(v));
  if (clear) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_quant_err, &z, sizeof(z));
  }
  return v;
}

}  // namespace i4b
