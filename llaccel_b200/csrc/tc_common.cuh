// Shared device helpers of the tensor-core GEMMs (gemm_tc.cu, gemm_sab.cu): mbarriers,
// TMA tile loads, UMMA shared-memory and instruction descriptors for kind::i8, tcgen05 MMA /
// commit / TMEM loads, cluster barriers and DSMEM loads, and the integer requant helpers of
// NUMERICS.md:62-86 (golden.py:92-107).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "numerics.cuh"

namespace llx {
namespace tc {

constexpr int BM = 128;         // MMA M: activation rows per tile
constexpr int BK = 128;         // bytes of K per stage (= the 128-byte swizzle span)
constexpr int kThreads = 320;   // 10 warps: TMA, MMA, 8 epilogue
constexpr uint32_t kSpinLimit = 1u << 26;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait: false on timeout
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023) == 1023 && *abort) return false;
  }
  return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;         // start address
  d |= (uint64_t)1 << 16;               // leading byte offset (16 B, unused with swizzle)
  d |= (uint64_t)(1024 >> 4) << 32;     // stride byte offset
  d |= (uint64_t)1 << 46;               // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;               // SWIZZLE_128B
  return d;
}

// instruction descriptor: kind::i8, D = s32, A = B = s8, both K-major, M = 128, N = nt
__host__ __device__ constexpr uint32_t idesc_i8(int nt) {
  return (2u << 4)                 // D format s32
         | (1u << 7)               // A signed 8-bit
         | (1u << 10)              // B signed 8-bit
         | ((uint32_t)(nt >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }


__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 16 bytes of a cluster peer's shared memory at the address of `local` in this CTA
__device__ __forceinline__ uint4 dsmem_ld4(const void* local, uint32_t rank) {
  uint32_t remote;
  uint4 v;
  asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(remote));
  return v;
}

__device__ __forceinline__ int64_t rshr64(int64_t v, int s) { return s == 0 ? v : (v >> s) + ((v >> (s - 1)) & 1); }
__device__ __forceinline__ int32_t sat16_32(int32_t v) { return v < -32768 ? -32768 : (v > 32767 ? 32767 : v); }
// rshr of a value with |v| < 2^31: 32-bit arithmetic for s < 31, 64-bit otherwise
__device__ __forceinline__ int32_t rshr_small(int32_t v, int s) {
  if (s == 0) return v;
  if (s < 31) return (v >> s) + ((v >> (s - 1)) & 1);
  return (int32_t)rshr64(v, s);
}

// Per-channel requant of an int32 accumulator (NUMERICS.md:69-71) saturated to [lo, hi]:
// v = acc + bias in 32 bits when the host proved |acc + bias| < 2^31 (narrow), else in 64;
// v * M (M < 2^32) in 64 bits, rshr S.  Straight-line code: the 16 channels of a chunk
// interleave freely.
// When the bias add is 32-bit (narrow), S >= 32 and M < 2^31 -- the usual case: M is
// normalised to [2^30, 2^31) -- the rounding shift comes from the product's high word
// (mulshift_hi32, exact), in a handful of 32-bit instructions instead of 64-bit shifts.
__device__ __forceinline__ int32_t requant_sat(int32_t acc, int64_t bias, uint32_t M, int S, bool narrow, int32_t lo,
                                               int32_t hi) {
  if (narrow && S >= 32 && M < 0x80000000u) {
    const int32_t t = mulshift_hi32(acc + (int32_t)bias, (int32_t)M, S);
    return t < lo ? lo : (t > hi ? hi : t);
  }
  const int64_t v = narrow ? (int64_t)(int32_t)(acc + (int32_t)bias) : (int64_t)acc + bias;
  const int64_t t = rshr64(narrow ? (int64_t)(int32_t)v * (int64_t)M : (int64_t)((uint64_t)v * (uint64_t)M), S);
  return (int32_t)(t < lo ? lo : (t > hi ? hi : t));
}
// sat(mulshift(v, M, S)) of an i16 value v (|v| <= 2^15).  For M < 2^31 the product is below
// 2^46: with S >= 32 the high word carries the shift (mulshift_hi32); with 16 <= S <= 31 the
// shifted product fits 31 bits, so a funnel shift of the two product words gives it and bit
// S - 1 of the low word is the rounding bit.  Otherwise the 64-bit form.
__device__ __forceinline__ int32_t mulshift_clamp(int32_t v, uint32_t M, int S, int32_t lo, int32_t hi) {
  int32_t t;
  if (M < 0x80000000u && S >= 32) {
    t = mulshift_hi32(v, (int32_t)M, S);
  } else if (M < 0x80000000u && S >= 16) {
    const int64_t p = (int64_t)v * (int64_t)M;
    const uint32_t plo = (uint32_t)p, phi = (uint32_t)(p >> 32);
    t = (int32_t)__funnelshift_r(plo, phi, S) + (int32_t)((plo >> (S - 1)) & 1u);
  } else {
    const int64_t t64 = rshr64((int64_t)v * (int64_t)M, S);
    return (int32_t)(t64 < lo ? lo : (t64 > hi ? hi : t64));
  }
  return t < lo ? lo : (t > hi ? hi : t);
}

// SiLU of an i16 value with the sigmoid table in shared memory (numerics.h:45-51).  Every
// intermediate after the input scaling fits 32 bits: |x * sg| <= 2^15 * 65514 < 2^31.
__device__ __forceinline__ int32_t silu_fast(int32_t x, uint32_t Mi, int Si, int sh_out, const uint16_t* sig) {
  const int32_t u = mulshift_clamp(x, Mi, Si, -32768, 32767);
  const int idx = (u >> 8) + 128;
  const int32_t f = u & 255;
  const int32_t lo = sig[idx];
  const int32_t sg = lo + (((int32_t)sig[idx + 1] - lo) * f >> 8);
  return sat16_32(rshr_small(x * sg, sh_out));
}


__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}


// TMEM loads whose completion is awaited once for several (tmem_wait_ld)
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, uint32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace tc
}  // namespace llx
