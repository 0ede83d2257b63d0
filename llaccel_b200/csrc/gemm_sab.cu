// Decode GEMM with the operands swapped: for a few activation rows (R <= 128, a decode batch)
// the tensor core's M side is 128 weight channels and its N side the NB activation rows, so
//   TMEM lane l = channel n0 + l, TMEM column j = row m0 + j,
// and each epilogue thread owns one channel: its bias and requant pair (NUMERICS.md:62-86)
// sit in registers, loaded before the grid dependency wait, and a warp's stores of one row
// are 32 consecutive channels (64 contiguous bytes of an i16 row).  The arithmetic is that
// of golden.py:316-342, exactly as in k_linear_tc: int32 accumulation (exact for
// K < 2^17), 64-bit or proven-32-bit bias add, per-channel requant, epilogue.
//
// CTA: warp 0 issues the TMA loads of each 128-byte K block -- the weight tile [128 x 128 B]
// (requested for the first stages before the dependency wait: model constants) and the
// activation tile [NB x 128 B] -- into an S-stage ring; warp 1 allocates NB TMEM columns and
// one thread issues tcgen05.mma kind::i8 (M = 128, N = NB, K = 32) four times per block;
// warps 2..9 run the epilogue, two warps per TMEM lane quarter splitting the rows.
//
// Split-K: the CTAs of a cluster (1 x ksplit) take disjoint K ranges.  Each stages its
// partial tile in its own shared memory as [NB / 4 row quads][128 channels][4 rows] int32,
// so that a warp's 16-byte accesses of one row quad are 512 contiguous bytes (one warp
// request, locally and over DSMEM); groups of 8 rows then go round-robin over the cluster's
// CTAs and warp halves, and the owner sums the partials of every CTA over DSMEM (integer
// addition: exact in any order).
//
// The epilogue loops over 8-row groups with a rolled loop: a decode-chain kernel executes
// each instruction about once, so compact code matters more than unrolling.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

#include "kernels.h"
#include "launch.cuh"
#include "numerics.cuh"
#include "tc_common.cuh"

namespace llx {
namespace sab {

using namespace tc;

constexpr int kThreadsSab = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kMaxStages = 4;

template <int NB>
struct Cfg {
  static constexpr int kW = 128 * BK;          // weight tile: 128 channels x 128 B of K
  static constexpr int kA = NB * BK;           // activation tile: NB rows x 128 B of K
  static constexpr int kStage = kW + kA;
  static constexpr int kPart = NB * 128 * 4;  // partial tile [NB / 4][128][4] int32
  static constexpr int kCols = NB < 32 ? 32 : NB;
  static int smem_bytes(int stages, int ksplit) {
    const int ring = stages * kStage;
    return (ksplit > 1 && kPart > ring ? kPart : ring) + 1024;
  }
};

// Requant of one accumulator with this thread's channel constants, saturated to [lo, hi].
// fast: the bias add is proven 32-bit (narrow), S >= 32 and 0 <= M < 2^31, so the product's
// high word carries the shift (mulshift_hi32); otherwise the 64-bit form.
__device__ __forceinline__ int32_t rq_chan(int32_t acc, int64_t bias, int32_t M, int S, bool fast, bool narrow,
                                           int32_t lo, int32_t hi) {
  if (fast) {
    const int32_t t = mulshift_hi32(acc + (int32_t)bias, M, S);
    return t < lo ? lo : (t > hi ? hi : t);
  }
  return requant_sat(acc, bias, (uint32_t)M, S, narrow, lo, hi);
}

template <int NB>
__global__ void __launch_bounds__(kThreadsSab, 2)
    k_linear_sab(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w, LinearArgs a,
                 int ksplit, int S, int32_t* err) {
  using L = Cfg<NB>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[kMaxStages], empty_bar[kMaxStages], acc_bar;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ int issued;
  __shared__ uint16_t s_sig[260];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 128;
  const int m0 = (blockIdx.y / ksplit) * NB;
  const uint32_t crank = ksplit > 1 ? cluster_rank() : 0;
  const int nkb_total = (a.K + BK - 1) / BK;
  const int per = (nkb_total + ksplit - 1) / ksplit;
  const int kb0 = (int)crank * per;
  const int kb1 = min(nkb_total, kb0 + per);
  const int nkb = kb1 > kb0 ? kb1 - kb0 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&acc_bar, 1);
    abort_flag = 0;
    issued = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(L::kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (a.epi == EPI_SILU || a.gated)
    for (int i = threadIdx.x; i < 257; i += blockDim.x) s_sig[i] = a.luts[kLutSig + i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  // dependents may launch once every CTA of this grid holds its TMEM columns
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer: weight tiles of the first stages before the dependency wait ----
      const int pre = nkb < S ? nkb : S;
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(&full_bar[i], L::kStage);
        tma_load_2d(ring + i * L::kStage, &map_w, &full_bar[i], (kb0 + i) * BK, n0);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        tma_load_2d(ring + i * L::kStage + L::kW, &map_a, &full_bar[i], (kb0 + i) * BK, m0);
        issued = i + 1;
      }
      for (int i = pre; i < nkb; ++i) {
        const int s = i % S;
        if (!mbar_wait(&empty_bar[s], ((i / S) + 1) & 1, &abort_flag)) {
          abort_flag = 1;
          atomicExch(err, 12);
          break;
        }
        uint8_t* st = ring + s * L::kStage;
        mbar_expect_tx(&full_bar[s], L::kStage);
        const int kx = (kb0 + i) * BK;
        tma_load_2d(st, &map_w, &full_bar[s], kx, n0);
        tma_load_2d(st + L::kW, &map_a, &full_bar[s], kx, m0);
        issued = i + 1;
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      // ---- MMA issuer: D[128 ch][NB rows] += W[128 x 32] . A[NB x 32]^T per instruction ----
      const uint32_t idesc = idesc_i8(NB);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        if (!mbar_wait(&full_bar[s], (i / S) & 1, &abort_flag)) {
          abort_flag = 1;
          atomicExch(err, 13);
          break;
        }
        tc_fence_after();
        const uint8_t* st = ring + s * L::kStage;
        const uint64_t dw = smem_desc(st), da = smem_desc(st + L::kW);
#pragma unroll
        for (int k = 0; k < BK / 32; ++k)
          mma_i8(tmem, dw + (uint64_t)(k * 2), da + (uint64_t)(k * 2), idesc, (i > 0 || k > 0) ? 1u : 0u);
        mma_commit(&empty_bar[s]);
      }
      mma_commit(&acc_bar);
    }
  }

  // ---- epilogue warps: channel constants (model data) before the dependency wait ----
  const int q = warp & 3;
  const int half = (warp - 2) >> 2;
  const int cl = 32 * q + lane;  // TMEM lane = channel within the tile
  const int c = n0 + cl;
  const bool live = c < a.N;
  int64_t bias = 0;
  int32_t Mc = 0;
  int Sc = 0;
  void* dst = a.out;
  int ld = a.N, col = c, i8 = a.out_i8;
  if (warp >= 2) {
    if (live && a.bias) bias = a.bias[c];
    if (live && a.rq) {
      Mc = a.rq[2 * c];
      Sc = a.rq[2 * c + 1];
    }
    if (a.nseg > 0) {
      int sgi = 0;
      while (sgi + 1 < a.nseg && c >= a.seg_start[sgi + 1]) ++sgi;
      dst = a.seg_out[sgi];
      ld = a.seg_start[sgi + 1] - a.seg_start[sgi];
      col = c - a.seg_start[sgi];
      i8 = a.seg_i8[sgi];
    }
    pdl_wait();  // activations, aux rows and output buffers belong to earlier kernels
    if (warp == 2 && lane == 0 && !mbar_wait(&acc_bar, 0, &abort_flag)) {
      abort_flag = 1;
      atomicExch(err, 14);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kThreadsSab - 64) : "memory");
    tc_fence_after();
    if (ksplit > 1 && abort_flag == 0) {
      // all MMAs are complete, so the ring is free: stage this half's columns of the partial,
      // up to 32 columns per TMEM round trip (several loads, one wait)
      constexpr int HC = NB / 2, STEP = HC < 32 ? HC : 32;
      uint4* part = reinterpret_cast<uint4*>(ring) + cl;  // row quad j4 at part[128 * j4]
#pragma unroll 1
      for (int cc = half * HC; cc < (half + 1) * HC; cc += STEP) {
        uint32_t v[STEP];
#pragma unroll
        for (int u = 0; u < STEP / 8; ++u) tmem_ld8_nowait(tmem + ((uint32_t)(32 * q) << 16) + cc + 8 * u, v + 8 * u);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < STEP / 4; ++u)
          part[128 * (cc / 4 + u)] =
              nkb > 0 ? make_uint4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]) : make_uint4(0, 0, 0, 0);
      }
    }
  }
  if (ksplit > 1) cluster_sync();  // every CTA's partial is visible cluster-wide
  if (warp >= 2 && abort_flag == 0) {
    const bool fast = a.narrow != 0 && Sc >= 32 && Mc >= 0;
    const bool narrow = a.narrow != 0;
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
    const uint4* part = reinterpret_cast<const uint4*>(ring) + cl;
    const bool has_aux = a.epi == EPI_RESADD || a.epi == EPI_MUL;
    const int lo = i8 ? -128 : -32768, hi = i8 ? 127 : 32767;
    // group gi of 8 rows -> cluster rank gi % ksplit, warp half (gi / ksplit) % 2
#pragma unroll 1
    for (int gi = (int)crank + ksplit * half; gi < NB / 8; gi += 2 * ksplit) {
      const int r0 = m0 + 8 * gi;
      int32_t aux[8];
      if (has_aux) {
#pragma unroll
        for (int j = 0; j < 8; ++j) aux[j] = (live && r0 + j < a.R) ? a.aux[(int64_t)(r0 + j) * a.N + c] : 0;
      }
      int32_t acc[8];
      if (ksplit == 1) {
        uint32_t v[8];
        tmem_ld8(trow + 8 * gi, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = nkb > 0 ? (int32_t)v[j] : 0;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0;
        // the peers' partials in batches of four: every load of a batch is in flight before
        // any is summed (a DSMEM round trip is long; one at a time would serialise them)
#pragma unroll 1
        for (int p0 = 0; p0 < ksplit; p0 += 4) {
          uint4 x[8];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const bool ok = p0 + u < ksplit;
            x[2 * u] = ok ? dsmem_ld4(part + 128 * (2 * gi), (uint32_t)(p0 + u)) : make_uint4(0, 0, 0, 0);
            x[2 * u + 1] = ok ? dsmem_ld4(part + 128 * (2 * gi + 1), (uint32_t)(p0 + u)) : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            acc[0] += (int32_t)x[2 * u].x, acc[1] += (int32_t)x[2 * u].y;
            acc[2] += (int32_t)x[2 * u].z, acc[3] += (int32_t)x[2 * u].w;
            acc[4] += (int32_t)x[2 * u + 1].x, acc[5] += (int32_t)x[2 * u + 1].y;
            acc[6] += (int32_t)x[2 * u + 1].z, acc[7] += (int32_t)x[2 * u + 1].w;
          }
        }
      }
      if (a.out_i32) {
        // tensor-parallel partial sums: raw accumulators
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (live && r0 + j < a.R) reinterpret_cast<int32_t*>(dst)[(int64_t)(r0 + j) * ld + col] = acc[j];
        continue;
      }
      if (a.gated) {
        // lanes 0-15 hold gate channels, lanes 16-31 the up channels of the same 16 outputs:
        // gate lanes finish rows 0-3 of the group, up lanes rows 4-7, after one exchange
        const bool isg = lane < 16;
        int32_t t[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) t[j] = rq_chan(acc[j], bias, Mc, Sc, fast, narrow, -32768, 32767);
        const int o = (n0 + 32 * q) / 2 + (lane & 15);
        const int rb = r0 + (isg ? 0 : 4);
        const uint32_t Mi = (uint32_t)a.silu_Mi;
        const bool fq = a.q_S >= 32 && a.q_M >= 0 && a.q_M < ((int64_t)1 << 31);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int32_t other = __shfl_xor_sync(0xffffffffu, isg ? t[4 + k] : t[k], 16);
          const int32_t tg = isg ? t[k] : other, tu = isg ? other : t[4 + k];
          const int r = rb + k;
          if (r >= a.R || o >= a.Nout) continue;
          const int32_t sg = silu_fast(tg, Mi, a.silu_Si, a.silu_sh, s_sig);
          const int32_t f = sat16_32(rshr_small(tu * sg, a.aux_shift));
          const int64_t off = (int64_t)r * a.Nout + o;
          if (a.g_out) a.g_out[off] = (int16_t)sg;
          if (a.f_out) a.f_out[off] = (int16_t)f;
          if (a.q_out) {
            const int32_t qv = fq ? mulshift_hi32(f, (int32_t)a.q_M, a.q_S)
                                  : (int32_t)mulshift((int64_t)f, a.q_M, a.q_S);
            a.q_out[off] = (int8_t)(qv < -128 ? -128 : (qv > 127 ? 127 : qv));
          }
        }
        continue;
      }
      int32_t o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        int32_t v = rq_chan(acc[j], bias, Mc, Sc, fast, narrow, lo, hi);
        if (a.epi == EPI_RESADD)
          v = sat16_32(v + aux[j]);
        else if (a.epi == EPI_MUL)
          v = sat16_32(rshr_small(v * aux[j], a.aux_shift));
        else if (a.epi == EPI_SILU)
          v = silu_fast(v, (uint32_t)a.silu_Mi, a.silu_Si, a.silu_sh, s_sig);
        o[j] = v;
      }
      if (dst && live) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (r0 + j >= a.R) break;
          if (i8)
            reinterpret_cast<int8_t*>(dst)[(int64_t)(r0 + j) * ld + col] = (int8_t)o[j];
          else
            reinterpret_cast<int16_t*>(dst)[(int64_t)(r0 + j) * ld + col] = (int16_t)o[j];
        }
      }
      if (a.amax_key) {
        // fused argmax: the row's best (logit, lowest index) key over this warp's 32 channels
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          unsigned long long key = 0ull;
          if (live && c < a.amax_vocab)
            key = ((unsigned long long)(uint32_t)(o[j] + 32768) << 32) | (0xFFFFFFFFu - (uint32_t)(c + a.amax_base));
#pragma unroll
          for (int s2 = 16; s2 > 0; s2 >>= 1) {
            const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, s2);
            key = k2 > key ? k2 : key;
          }
          if (lane == 0 && key && r0 + j < a.R) atomicMax(a.amax_key + r0 + j, key);
        }
      }
    }
  }
  if (ksplit > 1) cluster_sync();  // peers keep their shared memory until every CTA has read it
  // ---- teardown: drain copies issued but never consumed (abort path), free TMEM ----
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag) {
    for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i)
      for (uint32_t it = 0; it < (1u << 22); ++it)
        if (mbar_try_wait(&full_bar[i % S], (i / S) & 1)) break;
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::kCols));
  }
}

template <int NB>
static cudaError_t launch_sab_t(const CUtensorMap& ma, const CUtensorMap& mw, const LinearArgs& a, int ksplit,
                                int32_t* err, cudaStream_t st) {
  using L = Cfg<NB>;
  const int nkb = (a.K + BK - 1) / BK;
  const int per = (nkb + ksplit - 1) / ksplit;
  // ring stages: up to four, but at most ~100 KB of shared memory so that two CTAs share an
  // SM (the next kernel of the chain can then start while this one runs)
  const int smax = std::max(1, std::min(kMaxStages, (100 * 1024) / L::kStage));
  const int S = std::max(1, std::min(per, smax));
  const int smem = L::smem_bytes(S, ksplit);
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(k_linear_sab<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         L::smem_bytes(kMaxStages, 16));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_linear_sab<NB>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    attr_set[dev].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + 127) / 128, (a.R + NB - 1) / NB * ksplit, 1);
  cfg.blockDim = dim3(kThreadsSab, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = g_pdl ? 1 : 0;
  ++na;
  if (ksplit > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = ksplit;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, k_linear_sab<NB>, ma, mw, a, ksplit, S, err);
}

}  // namespace sab

int sab_rows_per_tile(int R) {
  if (R <= 16) return 16;
  if (R <= 32) return 32;
  if (R <= 64) return 64;
  return 128;
}

cudaError_t launch_linear_sab(const CUtensorMap& map_a, const CUtensorMap& map_w, const LinearArgs& a, int nb,
                              int ksplit, int32_t* err, cudaStream_t st) {
  if (a.R <= 0 || a.N <= 0) return cudaSuccess;
  if (ksplit < 1 || ksplit > 16) return cudaErrorInvalidValue;
  switch (nb) {
    case 16: return sab::launch_sab_t<16>(map_a, map_w, a, ksplit, err, st);
    case 32: return sab::launch_sab_t<32>(map_a, map_w, a, ksplit, err, st);
    case 64: return sab::launch_sab_t<64>(map_a, map_w, a, ksplit, err, st);
    case 128: return sab::launch_sab_t<128>(map_a, map_w, a, ksplit, err, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace llx
