// Shared device helpers for the int4_b200 kernels (sm_100a only).
//
// * element-type codes shared with include/int4_b200.h;
// * x86-semantics float helpers: the reference's bit-exact target
//   (quantize_int4_ref, int4_triton/quantize.py:102-117) runs on x86 CPUs,
//   where 0/0 produces the negative default NaN 0xFFC00000, NaN operands
//   propagate (quieted), floor keeps NaN, and a NaN float -> int32 cast gives
//   INT_MIN.  CUDA canonicalises NaNs instead, so the quantize kernel spells
//   these rules out;
// * PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor), tcgen05 (TMEM
//   alloc, UMMA, commit, tcgen05.ld) and griddepcontrol;
// * bounded mbarrier waits: every spin gives up after I4B_WAIT_LIMIT_NS of
//   %globaltimer and reports through the caller's error word, so a broken
//   pipeline ends the kernel instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/int4_b200.h"

#ifndef I4B_WAIT_LIMIT_NS
#define I4B_WAIT_LIMIT_NS 2000000000ull  // 2 s of %globaltimer per wait
#endif

// Device-side error codes (bit flags OR-ed into a per-file __device__ word).
#define I4B_DEVERR_WAIT_TIMEOUT 1u
#define I4B_DEVERR_PEER_TIMEOUT 2u  // a wait for another rank of a peer group gave up

namespace i4b {

// ------------------------------------------------------------------ small utils

__host__ __device__ __forceinline__ int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------ x86-semantics float ops

__device__ __forceinline__ bool f_isnan(float a) { return a != a; }
__device__ __forceinline__ float f_quiet(float a) {
  uint32_t r;
  asm("or.b32 %0, %1, 0x00400000;" : "=r"(r) : "r"(__float_as_uint(a)));
  return __uint_as_float(r);
}
__device__ __forceinline__ float f_default_nan() { return __uint_as_float(0xFFC00000u); }
// Sign flip as an integer xor in PTX: written in C++ the compiler turns it into neg.f32,
// which does not keep a NaN's sign.
__device__ __forceinline__ float f_neg(float a) {
  uint32_t r;
  asm("xor.b32 %0, %1, 0x80000000;" : "=r"(r) : "r"(__float_as_uint(a)));
  return __uint_as_float(r);
}

// SSE divss: NaN operand -> that operand quieted (first operand wins); invalid -> default NaN.
__device__ __forceinline__ float x86_div(float a, float b) {
  if (f_isnan(a)) return f_quiet(a);
  if (f_isnan(b)) return f_quiet(b);
  float r = __fdiv_rn(a, b);
  return f_isnan(r) ? f_default_nan() : r;
}
__device__ __forceinline__ float x86_add(float a, float b) {
  if (f_isnan(a)) return f_quiet(a);
  if (f_isnan(b)) return f_quiet(b);
  float r = __fadd_rn(a, b);
  return f_isnan(r) ? f_default_nan() : r;
}
__device__ __forceinline__ float x86_sub(float a, float b) {
  if (f_isnan(a)) return f_quiet(a);
  if (f_isnan(b)) return f_quiet(b);
  float r = __fsub_rn(a, b);
  return f_isnan(r) ? f_default_nan() : r;
}
// torch.floor keeps a NaN unchanged.
__device__ __forceinline__ float x86_floor(float a) { return f_isnan(a) ? a : floorf(a); }
// torch.clamp(lo, hi) propagates NaN.
__device__ __forceinline__ float clamp_nan(float a, float lo, float hi) {
  if (f_isnan(a)) return a;
  return a < lo ? lo : (a > hi ? hi : a);
}
// NaN-propagating max / min as torch.amax / amin compute them: any NaN in the
// reduction yields the canonical quiet NaN 0x7FC00000, whatever its sign or payload.
__device__ __forceinline__ float max_nan(float a, float b) {
  if (f_isnan(a) || f_isnan(b)) return __uint_as_float(0x7FC00000u);
  return a > b ? a : b;
}
__device__ __forceinline__ float min_nan(float a, float b) {
  if (f_isnan(a) || f_isnan(b)) return __uint_as_float(0x7FC00000u);
  return a < b ? a : b;
}
// cvttss2si: NaN (and out-of-range) -> INT_MIN.
__device__ __forceinline__ uint32_t x86_f2i_bits(float a) {
  if (f_isnan(a)) return 0x80000000u;
  return static_cast<uint32_t>(static_cast<int32_t>(a));
}
// fp32 -> fp16 bits, RNE; NaN keeps its sign and becomes 0x7E00 (F16C / c10::Half).
__device__ __forceinline__ uint16_t f32_to_f16_bits_x86(float a) {
  if (f_isnan(a)) return (__float_as_uint(a) & 0x80000000u) ? 0xFE00u : 0x7E00u;
  return __half_as_ushort(__float2half_rn(a));
}
// fp16 bits -> fp32; NaN -> quiet fp32 NaN of the same sign.
__device__ __forceinline__ float f16_bits_to_f32_x86(uint16_t h) {
  if ((h & 0x7C00u) == 0x7C00u && (h & 0x03FFu)) return __uint_as_float(((h & 0x8000u) << 16) | 0x7FC00000u);
  return __half2float(__ushort_as_half(h));
}
// fp32 -> bf16 bits, RNE; NaN -> 0x7FC0 (c10::BFloat16).
__device__ __forceinline__ uint16_t f32_to_bf16_bits_torch(float a) {
  if (f_isnan(a)) return 0x7FC0u;
  return __bfloat16_as_ushort(__float2bfloat16_rn(a));
}

// ------------------------------------------------------------------ element loads

template <int DT> struct Elem;
template <> struct Elem<I4B_F16> {
  using T = __half;
  __device__ __forceinline__ static float to_f32(uint16_t b) { return __half2float(__ushort_as_half(b)); }
};
template <> struct Elem<I4B_BF16> {
  using T = __nv_bfloat16;
  __device__ __forceinline__ static float to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }
};

// ------------------------------------------------------------------ mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity; false once I4B_WAIT_LIMIT_NS have passed since the
// 256th probe.  The global timer is read only every 256 probes: a read costs hundreds of cycles, which a
// pipeline stage waiting a few hundred cycles for its data would otherwise pay on every wait.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      const uint64_t t = globaltimer_ns();
      if (i == 255u) t0 = t;
      else if (t - t0 > I4B_WAIT_LIMIT_NS) return false;
    }
  }
}

// Like mbar_wait, but each probe lets the thread sleep in hardware (up to ~1 us) until the phase completes:
// for warps that only consume, so that their waiting does not take issue slots from working warps.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, 1000;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if ((i & 15u) == 15u) {  // each probe may sleep up to ~1 us: the timer every 16 probes
      const uint64_t t = globaltimer_ns();
      if (i == 15u) t0 = t;
      else if (t - t0 > I4B_WAIT_LIMIT_NS) return false;
    }
  }
}

// ------------------------------------------------------------------ TMA

__device__ __forceinline__ void tma_prefetch_desc(const void* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
// 2-D tiled load global -> shared, completion counted in bytes on `bar`.
// c0 is the innermost coordinate; callers keep c0 * element size a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* map, uint64_t* bar, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// 3-D tiled load global -> shared (box stored densely, innermost dimension first), completion on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* map, uint64_t* bar, int32_t c0, int32_t c1,
                                            int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// Fire-and-forget prefetch of a 2-D tensor tile into L2 (no shared memory, no completion to wait for).
__device__ __forceinline__ void tma_prefetch_l2_2d(const void* map, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------ tcgen05 / TMEM

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 or fp16 operands, fp32 accumulator).
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// UMMA shared-memory descriptor, K-major operand in the 128-byte swizzle canonical layout:
// rows of 128 B, 8-row core-matrix groups 1024 B apart (SBO), LBO unused (1), version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  return uint64_t((smem_addr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// Instruction descriptor, kind::f16: fp32 D, A/B bf16 (fmt 1) or fp16 (fmt 0), both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int ab_fmt, int m, int n) {
  return (1u << 4) | (uint32_t(ab_fmt) << 7) | (uint32_t(ab_fmt) << 10) | (uint32_t(n >> 3) << 17) |
         (uint32_t(m >> 4) << 24);
}

// ------------------------------------------------------------------ thread-block clusters / DSMEM

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of all CTAs of the cluster; release/acquire orders shared-memory writes before remote reads.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(addr), "r"(rank));
  return d;
}
// Volatile: stays after the cluster barrier that publishes the data.  Independent loads written one after
// another are still in flight together; callers issue all of them before using any result.
__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// ------------------------------------------------------------------ programmatic dependent launch

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ per-thread async copies (cp.async)

// 16 bytes global -> shared, bypassing L1; src_bytes < 16 zero-fills the rest.
__device__ __forceinline__ void cp_async_16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
// 4 / 8 bytes global -> shared (through L1); src_bytes 0 zero-fills.
__device__ __forceinline__ void cp_async_4(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_8(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ------------------------------------------------------------------ legacy warp MMA (small-M path)

// D(16x8 fp32) += A(16x16) * B(16x8), bf16 or fp16 operands.
template <bool F16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (F16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// D(16x8 fp32) = A(16x16) * B(16x8): a fresh accumulation (C = 0).
template <bool F16>
__device__ __forceinline__ void mma_16816_first(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  const float z = 0.0f;
  if constexpr (F16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
  }
}

// lop3: (a & b) | c
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ------------------------------------------------------------------ exact INT4 dequantization
// w = (q - z) * s rounded once to the activation type, as the reference's kernels compute it
// (int4_triton/gemm.py:144 and :211: fp32 (q - z) * s, then .to(x.dtype)).  A nibble pair arrives as
// (bias + q_i, bias + q_j) from one lop3 (bias 128 for bf16, 1024 for fp16, exact); d = p - (bias + z) is
// an exact small integer.  fp16: s is an fp16 operand, so d * s rounds once.  bf16: s (fp16, 11 bits)
// splits into s_hi (its top 8 bits, a bf16) and s_lo = s - s_hi (at most 3 significant bits, exact in
// bf16); d * s_lo (<= 7 bits) is exact, and fma(d, s_hi, d * s_lo) = d * s rounded once.
struct DqParams {
  uint32_t zz;   // (bias + z) twice
  uint32_t shi;  // bf16: scale high part twice; fp16: scale twice
  uint32_t slo;  // bf16: scale low part twice
};

template <bool F16>
__device__ __forceinline__ DqParams dq_params(uint16_t s_bits, uint16_t z_bits) {
  const float s = __half2float(__ushort_as_half(s_bits));
  const float z = __half2float(__ushort_as_half(z_bits));
  DqParams p;
  if constexpr (F16) {
    const uint32_t zz = __half_as_ushort(__float2half_rn(1024.0f + z));
    p.zz = zz * 0x10001u;
    p.shi = uint32_t(s_bits) * 0x10001u;
    p.slo = 0;
  } else {
    const uint32_t hi = __float_as_uint(s) & 0xFFFF0000u;
    const float lo = isfinite(s) ? (s - __uint_as_float(hi)) : 0.0f;
    const uint32_t lo16 = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
    const uint32_t zz = __bfloat16_as_ushort(__float2bfloat16_rn(128.0f + z));
    p.zz = zz * 0x10001u;
    p.shi = (hi >> 16) * 0x10001u;
    p.slo = lo16 * 0x10001u;
  }
  return p;
}

template <bool F16>
__device__ __forceinline__ uint32_t dq_pair(uint32_t p, const DqParams& dp) {
  uint32_t d, w;
  if constexpr (F16) {
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(p), "r"(dp.zz));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(w) : "r"(d), "r"(dp.shi));
  } else {
    uint32_t pl;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(p), "r"(dp.zz));
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(pl) : "r"(d), "r"(dp.slo));
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(w) : "r"(d), "r"(dp.shi), "r"(pl));
  }
  return w;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

// First maximum of the bf16 row xr[0, n) over the CTA (blockDim.x a multiple of 32, <= 1024): on thread 0,
// *best_out = the maximum and *idx_out = its first index (n when no element compares above -inf, e.g. all
// NaN).  kU 16-byte chunks per thread are in flight before any is compared; each thread visits its chunks in
// increasing index order and ties go to the lower index at every step.
__device__ __forceinline__ void block_row_argmax(const uint16_t* __restrict__ xr, int64_t n, float* best_out,
                                                 int64_t* idx_out) {
  __shared__ float vmax[32];
  __shared__ int64_t vidx[32];
  float best = -INFINITY;
  int64_t bi = n;
  const bool vec = (reinterpret_cast<uintptr_t>(xr) % 16 == 0);
  const int64_t n8 = vec ? n / 8 * 8 : 0;
  const int64_t nch = n8 / 8;  // 16-byte chunks
  // kU chunks per thread in flight before any is compared (one memory round trip per kU chunks, not per
  // chunk); a thread visits its chunks in increasing index order
  constexpr int kU = 8;
  for (int64_t base = 0; base < nch; base += int64_t(blockDim.x) * kU) {
    uint4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t ch = base + int64_t(u) * blockDim.x + threadIdx.x;
      v[u] = ch < nch ? __ldg(reinterpret_cast<const uint4*>(xr) + ch) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t ch = base + int64_t(u) * blockDim.x + threadIdx.x;
      if (ch >= nch) break;
      const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = bf16_bits_to_f32(uint16_t(w[e >> 1] >> (16 * (e & 1))));
        if (f > best) {  // strictly greater: the first index wins within a thread
          best = f;
          bi = ch * 8 + e;
        }
      }
    }
  }
  for (int64_t c = n8 + threadIdx.x; c < n; c += blockDim.x) {
    const float f = bf16_bits_to_f32(xr[c]);
    if (f > best) {
      best = f;
      bi = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    vmax[warp] = best;
    vidx[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < int(blockDim.x >> 5); ++w)
      if (vmax[w] > best || (vmax[w] == best && vidx[w] < bi)) {
        best = vmax[w];
        bi = vidx[w];
      }
    *best_out = best;
    *idx_out = bi;
  }
}

}  // namespace i4b
