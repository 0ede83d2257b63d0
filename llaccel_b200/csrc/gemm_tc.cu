// Matrix engine on the 5th-generation tensor cores: tcgen05.mma kind::i8 with TMEM
// accumulators fed by TMA, and the fused requant epilogue of NUMERICS.md:62-86.
//
// CTA tile: 128 activation rows (MMA M) x NT weight channels (MMA N), K streamed in
// 128-byte blocks through an S-stage shared-memory ring:
//   warp 0  one thread issues the TMA loads of the activation tile [128 x 128 B] and the
//           weight tile [NT x 128 B] (both K-major, 128-byte swizzle) into stage s;
//   warp 1  allocates NT TMEM columns, one thread issues 4 MMAs (K = 32 each) per block
//           and commits each stage back to the producer, then the accumulator;
//   warps 2-9 read the int32 accumulator rows from TMEM (one row per thread; two warps
//           per TMEM lane quarter split the channel chunks), add the bias, requantize per
//           channel, apply the epilogue and store 16 channels at a time (i16 or i8).
// The int32 accumulation is exact (|acc| <= K * 2^14 < 2^31 for K < 2^17), so the tensor
// core result equals the reference's int64 matmul.  Rows and K past the tensor extents
// are zero-filled by TMA.  Every mbarrier wait is bounded: on timeout the CTA records an
// error word, stops issuing work, drains the copies it started and frees its TMEM.
//
// Split-K: with ksplit > 1, the CTAs of a thread-block cluster (cluster dims 1 x ksplit)
// take disjoint K ranges; each writes its accumulator tile to its own shared memory, and
// each CTA then owns a share of the tile's 16-channel chunks, summing the partials of every
// CTA of the cluster over DSMEM before its epilogue (integer addition: exact in any order).
// Every TMA load here is a plain single-CTA load.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "kernels.h"
#include "launch.cuh"
#include "numerics.cuh"
#include "tc_common.cuh"

namespace llx {

namespace tc {

// UW accumulators of tile columns c0 .. c0+UW-1 for one row: from TMEM, or (split-K) the
// sum of every cluster CTA's staged partial (integer addition: exact in any order)
template <int UW>
__device__ __forceinline__ void epi_fetch(int32_t (&acc)[UW], uint32_t trow, const uint4* part4, int row, int c0,
                                          int ksplit, int nkb) {
  if (ksplit == 1) {
    uint32_t v[UW];
    if (UW == 8)
      tmem_ld8(trow + c0, v);
    else
      tmem_ld4(trow + c0, v);
#pragma unroll
    for (int j = 0; j < UW; ++j) acc[j] = nkb > 0 ? (int32_t)v[j] : 0;
    return;
  }
#pragma unroll
  for (int j = 0; j < UW; ++j) acc[j] = 0;
  for (uint32_t p = 0; p < (uint32_t)ksplit; ++p) {
#pragma unroll
    for (int k = 0; k < UW / 4; ++k) {
      const uint4 v = dsmem_ld4(part4 + (c0 / 4 + k) * BM + row, p);
      acc[4 * k] += (int32_t)v.x;
      acc[4 * k + 1] += (int32_t)v.y;
      acc[4 * k + 2] += (int32_t)v.z;
      acc[4 * k + 3] += (int32_t)v.w;
    }
  }
}

// UW consecutive outputs (UW = 4 or 8 bytes-aligned groups) of one row
template <int UW>
__device__ __forceinline__ void store_i16(int16_t* p, const int32_t* o) {
  uint32_t w[UW / 2];
#pragma unroll
  for (int k = 0; k < UW / 2; ++k) w[k] = (uint32_t)(uint16_t)o[2 * k] | (uint32_t)(uint16_t)o[2 * k + 1] << 16;
  if (UW == 8)
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  else
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
}
template <int UW>
__device__ __forceinline__ void store_i8(int8_t* p, const int32_t* o) {
  uint32_t w[UW / 4];
#pragma unroll
  for (int k = 0; k < UW / 4; ++k)
    w[k] = (uint32_t)(uint8_t)o[4 * k] | (uint32_t)(uint8_t)o[4 * k + 1] << 8 |
           (uint32_t)(uint8_t)o[4 * k + 2] << 16 | (uint32_t)(uint8_t)o[4 * k + 3] << 24;
  if (UW == 8)
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  else
    *reinterpret_cast<uint32_t*>(p) = w[0];
}
template <int UW>
__device__ __forceinline__ void load_i16(const int16_t* p, int32_t* v) {
  uint32_t w[UW / 2];
  if (UW == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    w[0] = u.x, w[1] = u.y, w[2] = u.z, w[3] = u.w;
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    w[0] = u.x, w[1] = u.y;
  }
#pragma unroll
  for (int k = 0; k < UW / 2; ++k) {
    v[2 * k] = (int16_t)(w[k] & 0xFFFF);
    v[2 * k + 1] = (int16_t)(w[k] >> 16);
  }
}

// Epilogue of UW columns (tile columns c0.., global n0 + c0..) of row r: requant + epilogue
// + store, or raw int32 partial sums; the fused argmax key of the output linear.  Channel
// groups never straddle an output segment (segments are 16-channel multiples).
// `best` collects the row's packed argmax key (output linear only); the caller folds it into
// amax_key with one atomicMax per thread and row, not one per unit.
template <int UW>
__device__ __forceinline__ void epi_unit(const LinearArgs& a, const int32_t (&acc)[UW], int c0, int n0, int r,
                                         const int64_t* s_bias, const uint32_t* s_M, const int* s_S,
                                         const uint16_t* s_sig, unsigned long long& best) {
  const int nb = n0 + c0;
  void* dst = a.out;
  int ld = a.N, col = nb, i8 = a.out_i8;
  if (a.nseg > 0) {
    int sgi = 0;
    while (sgi + 1 < a.nseg && nb >= a.seg_start[sgi + 1]) ++sgi;
    dst = a.seg_out[sgi];
    ld = a.seg_start[sgi + 1] - a.seg_start[sgi];
    col = nb - a.seg_start[sgi];
    i8 = a.seg_i8[sgi];
  }
  if (a.out_i32) {
    // tensor-parallel partial sums: raw accumulators
    uint4* p = reinterpret_cast<uint4*>(reinterpret_cast<int32_t*>(dst) + (int64_t)r * ld + col);
#pragma unroll
    for (int k = 0; k < UW / 4; ++k)
      p[k] = make_uint4((uint32_t)acc[4 * k], (uint32_t)acc[4 * k + 1], (uint32_t)acc[4 * k + 2],
                        (uint32_t)acc[4 * k + 3]);
    return;
  }
  const bool narrow = a.narrow != 0;
  int32_t o[UW];
  if (i8) {
#pragma unroll
    for (int j = 0; j < UW; ++j) o[j] = requant_sat(acc[j], s_bias[c0 + j], s_M[c0 + j], s_S[c0 + j], narrow, -128, 127);
    store_i8<UW>(reinterpret_cast<int8_t*>(dst) + (int64_t)r * ld + col, o);
    return;
  }
#pragma unroll
  for (int j = 0; j < UW; ++j) o[j] = requant_sat(acc[j], s_bias[c0 + j], s_M[c0 + j], s_S[c0 + j], narrow, -32768, 32767);
  if (a.epi == EPI_RESADD || a.epi == EPI_MUL) {
    int32_t aux[UW];
    load_i16<UW>(a.aux + (int64_t)r * a.N + nb, aux);
    if (a.epi == EPI_RESADD) {
#pragma unroll
      for (int j = 0; j < UW; ++j) o[j] = sat16_32(o[j] + aux[j]);
    } else {
#pragma unroll
      for (int j = 0; j < UW; ++j) o[j] = sat16_32(rshr_small(o[j] * aux[j], a.aux_shift));
    }
  } else if (a.epi == EPI_SILU) {
    const uint32_t Mi = (uint32_t)a.silu_Mi;
#pragma unroll
    for (int j = 0; j < UW; ++j) o[j] = silu_fast(o[j], Mi, a.silu_Si, a.silu_sh, s_sig);
  }
  if (dst) store_i16<UW>(reinterpret_cast<int16_t*>(dst) + (int64_t)r * ld + col, o);  // null: argmax only
  if (a.amax_key) {
#pragma unroll
    for (int j = 0; j < UW; ++j) {
      const int n = nb + j;
      if (n < a.amax_vocab) {
        const unsigned long long key =
            ((unsigned long long)(uint32_t)(o[j] + 32768) << 32) | (0xFFFFFFFFu - (uint32_t)(n + a.amax_base));
        best = key > best ? key : best;
      }
    }
  }
}

// Fused gate/up unit: 8 output channels ob.. of row r from gate columns cg.. and up columns cu..
//   sg = silu16(requant16(acc_g)); f = sat16(rshr(requant16(acc_u) * sg, aux_shift));
//   fq = sat8(mulshift(f, q_M, q_S))
// The column loop stays rolled: each SM runs this epilogue once per launch, so its cost is
// the first fetch of its instructions, and one column's body is an eighth of the unrolled
// code.  The inputs shift through registers (constant indices) and the outputs are packed by
// shifting in from the top, so nothing is indexed dynamically.
__device__ __forceinline__ void epi_gated_unit(const LinearArgs& a, int32_t (&ag)[8], int32_t (&au)[8], int cg,
                                               int cu, int r, int ob, const int64_t* s_bias, const uint32_t* s_M,
                                               const int* s_S, const uint16_t* s_sig) {
  const bool narrow = a.narrow != 0;
  const uint32_t Mi = (uint32_t)a.silu_Mi;
  uint64_t g_lo = 0, g_hi = 0, f_lo = 0, f_hi = 0, q8 = 0;
#pragma unroll 1
  for (int j = 0; j < 8; ++j) {
    const int32_t tg = requant_sat(ag[0], s_bias[cg + j], s_M[cg + j], s_S[cg + j], narrow, -32768, 32767);
    const int32_t tu = requant_sat(au[0], s_bias[cu + j], s_M[cu + j], s_S[cu + j], narrow, -32768, 32767);
#pragma unroll
    for (int k = 0; k < 7; ++k) {
      ag[k] = ag[k + 1];
      au[k] = au[k + 1];
    }
    const int32_t sg = silu_fast(tg, Mi, a.silu_Si, a.silu_sh, s_sig);
    const int32_t f = sat16_32(rshr_small(tu * sg, a.aux_shift));
    const int32_t fq = mulshift_clamp(f, (uint32_t)a.q_M, a.q_S, -128, 127);
    g_lo = (g_lo >> 16) | (g_hi << 48);
    g_hi = (g_hi >> 16) | ((uint64_t)(uint16_t)sg << 48);
    f_lo = (f_lo >> 16) | (f_hi << 48);
    f_hi = (f_hi >> 16) | ((uint64_t)(uint16_t)f << 48);
    q8 = (q8 >> 8) | ((uint64_t)(uint8_t)fq << 56);
  }
  const int64_t off = (int64_t)r * a.Nout + ob;
  if (a.g_out)
    *reinterpret_cast<uint4*>(a.g_out + off) = make_uint4((uint32_t)g_lo, (uint32_t)(g_lo >> 32), (uint32_t)g_hi,
                                                          (uint32_t)(g_hi >> 32));
  if (a.f_out)
    *reinterpret_cast<uint4*>(a.f_out + off) = make_uint4((uint32_t)f_lo, (uint32_t)(f_lo >> 32), (uint32_t)f_hi,
                                                          (uint32_t)(f_hi >> 32));
  if (a.q_out) *reinterpret_cast<uint2*>(a.q_out + off) = make_uint2((uint32_t)q8, (uint32_t)(q8 >> 32));
}

template <int NT, int S>
struct Smem {
  static constexpr int kA = BM * BK;  // 16 KB activation tile
  static constexpr int kB = NT * BK;  // weight tile
  static constexpr int kStage = kA + kB;
  static constexpr int kRing = S * kStage;
  // partial accumulators for split-K reduction reuse the ring: BM x NT int32
  static constexpr int kPart = BM * NT * 4;
  static constexpr int kBytes = (kRing > kPart ? kRing : kPart) + 1024 /* alignment slack */ + 256;
};

template <int NT, int S>
__global__ void __launch_bounds__(kThreads, 2)
    k_linear_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w, LinearArgs a,
                int ksplit, int32_t* err) {
  using L = Smem<NT, S>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[S], empty_bar[S], acc_bar;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ int issued;  // TMA stages issued by the producer
  __shared__ int64_t s_bias[NT];
  __shared__ uint32_t s_M[NT];
  __shared__ int s_S[NT];
  __shared__ uint16_t s_sig[260];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * NT;
  const int m0 = (blockIdx.y / ksplit) * BM;
  const uint32_t crank = ksplit > 1 ? cluster_rank() : 0;
  // this CTA's K range in 128-byte blocks
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
                 "r"(NT < 32 ? 32 : NT));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // per-channel requant parameters
  for (int i = threadIdx.x; i < NT; i += blockDim.x) {
    const int n = n0 + i;
    s_M[i] = (n < a.N && a.rq) ? (uint32_t)a.rq[2 * n] : 0u;
    s_S[i] = (n < a.N && a.rq) ? a.rq[2 * n + 1] : 0;
    s_bias[i] = (n < a.N && a.bias) ? (int64_t)a.bias[n] : 0;
  }
  if (a.epi == EPI_SILU || a.gated)
    for (int i = threadIdx.x; i < 257; i += blockDim.x) s_sig[i] = a.luts[kLutSig + i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  // dependents may launch only once every CTA of this grid holds its TMEM columns, so a
  // waiting dependent CTA can never keep a CTA of this grid from allocating
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      // weights are model constants: the first S stages' weight tiles are requested before
      // the grid dependency wait, overlapping the previous kernel; activations after it
      const int pre = nkb < S ? nkb : S;
      for (int i = 0; i < pre; ++i) {
        uint8_t* sb = ring + i * L::kStage + L::kA;
        mbar_expect_tx(&full_bar[i], L::kA + L::kB);
        tma_load_2d(sb, &map_w, &full_bar[i], (kb0 + i) * BK, n0);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        tma_load_2d(ring + i * L::kStage, &map_a, &full_bar[i], (kb0 + i) * BK, m0);
        issued = i + 1;
      }
      for (int i = pre; i < nkb; ++i) {
        const int s = i % S;
        if (!mbar_wait(&empty_bar[s], ((i / S) + 1) & 1, &abort_flag)) {
          abort_flag = 1;
          atomicExch(err, 2);
          break;
        }
        uint8_t* sa = ring + s * L::kStage;
        uint8_t* sb = sa + L::kA;
        mbar_expect_tx(&full_bar[s], L::kA + L::kB);
        const int kx = (kb0 + i) * BK;
        tma_load_2d(sa, &map_a, &full_bar[s], kx, m0);
        tma_load_2d(sb, &map_w, &full_bar[s], kx, n0);
        issued = i + 1;
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      // ---- MMA issuer ----
      const uint32_t idesc = idesc_i8(NT);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        if (!mbar_wait(&full_bar[s], (i / S) & 1, &abort_flag)) {
          abort_flag = 1;
          atomicExch(err, 3);
          break;
        }
        tc_fence_after();
        const uint8_t* sa = ring + s * L::kStage;
        const uint8_t* sb = sa + L::kA;
        const uint64_t da = smem_desc(sa), db = smem_desc(sb);
#pragma unroll
        for (int k = 0; k < BK / 32; ++k) {
          // advance both descriptors by 32 bytes of K inside the swizzle atom
          mma_i8(tmem, da + (uint64_t)(k * 2), db + (uint64_t)(k * 2), idesc, (i > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&empty_bar[s]);
      }
      mma_commit(&acc_bar);  // fires once every MMA issued above has completed (or at once if none)
    }
  } else {
    pdl_wait();  // aux rows and the output buffer belong to earlier kernels
    // ---- epilogue warps 2..9: TMEM lane quarter = warp % 4, half = (warp - 2) / 4 ----
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = q * 32 + lane;
    // one thread polls the accumulator barrier; the eight epilogue warps then meet at named
    // barrier 1, which issues nothing while the main loop runs
    if (warp == 2 && lane == 0 && !mbar_wait(&acc_bar, 0, &abort_flag)) {
      abort_flag = 1;
      atomicExch(err, 4);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kThreads - 64) : "memory");
    const bool ok = abort_flag == 0;
    tc_fence_after();
    uint4* part4 = reinterpret_cast<uint4*>(ring);  // [NT/4][BM] 4-column groups of the partial tile
    if (ok && ksplit > 1) {
      // all MMAs are complete, so the ring is free: stage this CTA's partial tile, one
      // 16-byte group per row and 4 columns (rows consecutive: no bank conflicts)
      for (int u8 = half; u8 < NT / 8; u8 += 2) {
        uint32_t v[8];
        tmem_ld8(tmem + ((uint32_t)(q * 32) << 16) + u8 * 8, v);
        if (nkb == 0) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = 0;
        }
        part4[(2 * u8) * BM + row_in_tile] = make_uint4(v[0], v[1], v[2], v[3]);
        part4[(2 * u8 + 1) * BM + row_in_tile] = make_uint4(v[4], v[5], v[6], v[7]);
      }
    }
  }
  if (ksplit > 1) {
    // all threads of every CTA in the cluster meet here (partials visible cluster-wide)
    cluster_sync();
  }
  if (warp >= 2 && !abort_flag) {
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = q * 32 + lane;
    const int r = m0 + row_in_tile;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    const uint4* part4 = reinterpret_cast<const uint4*>(ring);
    // work units of UW columns go round-robin over the cluster's CTAs, then the two warp
    // halves: unit u -> CTA u % ksplit, half (u / ksplit) % 2
    const int first = (int)crank + ksplit * half, stride = 2 * ksplit;
    if (a.gated) {
      // unit v = 8 outputs: gate columns 32 (v/2) + 8 (v%2) .. +7, up columns 16 further
#pragma unroll 1
      for (int v = first; v < NT / 16; v += stride) {
        const int cg = 32 * (v >> 1) + 8 * (v & 1), cu = cg + 16;
        int32_t ag[8], au[8];
        epi_fetch<8>(ag, trow, part4, row_in_tile, cg, ksplit, nkb);
        epi_fetch<8>(au, trow, part4, row_in_tile, cu, ksplit, nkb);
        if (r >= a.R) continue;
        const int ob = (n0 + 32 * (v >> 1)) / 2 + 8 * (v & 1);  // first output channel of this unit
        if (ob >= a.Nout) continue;
        epi_gated_unit(a, ag, au, cg, cu, r, ob, s_bias, s_M, s_S, s_sig);
      }
    } else {
      unsigned long long best = 0ull;
      if (ksplit > 1) {
#pragma unroll 1
        for (int u = first; u < NT / 4; u += stride) {
          int32_t acc[4];
          epi_fetch<4>(acc, trow, part4, row_in_tile, 4 * u, ksplit, nkb);
          if (r < a.R && n0 + 4 * u < a.N) epi_unit<4>(a, acc, 4 * u, n0, r, s_bias, s_M, s_S, s_sig, best);
        }
      } else {
#pragma unroll 1
        for (int u = first; u < NT / 8; u += stride) {
          int32_t acc[8];
          epi_fetch<8>(acc, trow, part4, row_in_tile, 8 * u, ksplit, nkb);
          if (r < a.R && n0 + 8 * u < a.N) epi_unit<8>(a, acc, 8 * u, n0, r, s_bias, s_M, s_S, s_sig, best);
        }
      }
      if (best) atomicMax(a.amax_key + r, best);
    }
  }
  if (ksplit > 1) cluster_sync();  // peers keep their shared memory until rank 0 has read it
  // ---- teardown: drain copies issued but never consumed (abort path), free TMEM ----
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag) {
    // wait (bounded) for the last load issued into each stage to land before the CTA exits
    for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i) {
      for (uint32_t it = 0; it < (1u << 22); ++it)
        if (mbar_try_wait(&full_bar[i % S], (i / S) & 1)) break;
    }
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(NT < 32 ? 32 : NT));
  }
}


// ---------------------------------------------------------------------------------------
// Persistent variant for GEMMs with many output tiles (prefill, the vocabulary projection):
// one CTA per SM walks tiles t = blockIdx.x + j * gridDim.x: with more rows than channels
// (prefill) channel tiles fastest, so consecutive CTAs share an activation row tile in L2;
// otherwise (decode batches against wide weights) row tiles fastest, so the row tiles of one
// weight tile run in the same wave and the weight tile crosses HBM once.  The accumulator is double-buffered
// in TMEM (2 x NT columns): the MMA warp fills buffer j & 1 while the EW epilogue warps drain
// the other, so the integer epilogue of tile j overlaps the main loop of tile j + 1.
// Barriers: full/empty per ring stage (TMA <-> MMA), acc_full/acc_empty per buffer
// (MMA <-> epilogue).  Every wait is bounded; on timeout the CTA records an error word and
// every role stops.  No split-K here (ksplit == 1).
// ---------------------------------------------------------------------------------------
template <int NT, int S, int EW>
__global__ void __launch_bounds__(64 + 32 * EW, 1)
    k_linear_tc_persistent(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                           LinearArgs a, int32_t* err) {
  using L = Smem<NT, S>;
  constexpr int kEpiThreads = 32 * EW;
  constexpr int kQuads = EW / 4;  // epilogue warps per TMEM lane quarter
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[S], empty_bar[S], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ int issued;  // TMA stages issued by the producer (all tiles)
  __shared__ int64_t s_bias[NT];
  __shared__ uint32_t s_M[NT];
  __shared__ int s_S[NT];
  __shared__ uint16_t s_sig[260];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntn = (a.N + NT - 1) / NT, ntm = (a.R + BM - 1) / BM;
  const int tiles = ntn * ntm;
  const int nkb = (a.K + BK - 1) / BK;
  const int my_tiles = blockIdx.x < tiles ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const bool rows_fast = a.N > a.R;
  auto tile_origin = [&](int t, int& n0, int& m0) {
    n0 = (rows_fast ? t / ntm : t % ntn) * NT;
    m0 = (rows_fast ? t % ntm : t / ntn) * BM;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 1);
    }
    abort_flag = 0;
    issued = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(2 * NT));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (a.epi == EPI_SILU || a.gated)
    for (int i = threadIdx.x; i < 257; i += blockDim.x) s_sig[i] = a.luts[kLutSig + i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer: every k-block of every tile of this CTA through the ring ----
      int it = 0;
      bool waited = false;
      for (int j = 0; j < my_tiles && !abort_flag; ++j) {
        int n0, m0;
        tile_origin(blockIdx.x + j * gridDim.x, n0, m0);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S;
          if (it >= S && !mbar_wait(&empty_bar[s], ((it / S) + 1) & 1, &abort_flag)) {
            abort_flag = 1;
            atomicExch(err, 2);
            break;
          }
          uint8_t* sa = ring + s * L::kStage;
          uint8_t* sb = sa + L::kA;
          mbar_expect_tx(&full_bar[s], L::kA + L::kB);
          tma_load_2d(sb, &map_w, &full_bar[s], kb * BK, n0);  // weights: model constants
          if (!waited) {
            pdl_wait();  // activations belong to the previous kernel
            waited = true;
          }
          tma_load_2d(sa, &map_a, &full_bar[s], kb * BK, m0);
          issued = it + 1;
        }
      }
      if (!waited) pdl_wait();
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      // ---- MMA issuer: tile j into TMEM buffer j & 1 ----
      const uint32_t idesc = idesc_i8(NT);
      int it = 0;
      for (int j = 0; j < my_tiles && !abort_flag; ++j) {
        const int b = j & 1, u = j >> 1;
        if (u > 0 && !mbar_wait(&acc_empty[b], (u - 1) & 1, &abort_flag)) {
          abort_flag = 1;
          atomicExch(err, 5);
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * NT);
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full_bar[s], (it / S) & 1, &abort_flag)) {
            abort_flag = 1;
            atomicExch(err, 3);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* sa = ring + s * L::kStage;
          const uint8_t* sb = sa + L::kA;
          const uint64_t da = smem_desc(sa), db = smem_desc(sb);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_i8(acc, da + (uint64_t)(k * 2), db + (uint64_t)(k * 2), idesc, (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit(&empty_bar[s]);
        }
        if (!ok) break;
        mma_commit(&acc_full[b]);  // fires when every MMA of this tile has completed
      }
    }
  } else {
    pdl_wait();  // aux rows and the output buffer belong to earlier kernels
    // ---- epilogue warps: TMEM lane quarter = warp % 4, quad = (warp - 2) / 4 ----
    const int q = warp & 3;
    const int quad = (warp - 2) >> 2;
    const int row_in_tile = q * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    unsigned long long best = 0ull;  // argmax key of row best_r, folded in when the row changes
    int best_r = -1;
    for (int j = 0; j < my_tiles; ++j) {
      const int b = j & 1, u = j >> 1;
      int n0, m0;
      tile_origin(blockIdx.x + j * gridDim.x, n0, m0);
      // this tile's requant parameters (the previous tile's epilogue is done with them)
      for (int i = threadIdx.x - 64; i < NT; i += kEpiThreads) {
        const int n = n0 + i;
        s_M[i] = (n < a.N && a.rq) ? (uint32_t)a.rq[2 * n] : 0u;
        s_S[i] = (n < a.N && a.rq) ? a.rq[2 * n + 1] : 0;
        s_bias[i] = (n < a.N && a.bias) ? (int64_t)a.bias[n] : 0;
      }
      if (warp == 2 && lane == 0 && !abort_flag && !mbar_wait(&acc_full[b], u & 1, &abort_flag)) {
        abort_flag = 1;
        atomicExch(err, 4);
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (abort_flag) break;
      tc_fence_after();
      const int r = m0 + row_in_tile;
      const uint32_t tacc = trow + (uint32_t)(b * NT);
      if (a.gated) {
#pragma unroll 1
        for (int v = quad; v < NT / 16; v += kQuads) {
          const int cg = 32 * (v >> 1) + 8 * (v & 1), cu = cg + 16;
          int32_t ag[8], au[8];
          epi_fetch<8>(ag, tacc, nullptr, row_in_tile, cg, 1, nkb);
          epi_fetch<8>(au, tacc, nullptr, row_in_tile, cu, 1, nkb);
          if (r >= a.R) continue;
          const int ob = (n0 + 32 * (v >> 1)) / 2 + 8 * (v & 1);
          if (ob >= a.Nout) continue;
          epi_gated_unit(a, ag, au, cg, cu, r, ob, s_bias, s_M, s_S, s_sig);
        }
      } else {
        if (r != best_r) {
          if (best) atomicMax(a.amax_key + best_r, best);
          best = 0ull;
          best_r = r;
        }
#pragma unroll 1
        for (int v = quad; v < NT / 8; v += kQuads) {
          int32_t acc[8];
          epi_fetch<8>(acc, tacc, nullptr, row_in_tile, 8 * v, 1, nkb);
          if (r < a.R && n0 + 8 * v < a.N) epi_unit<8>(a, acc, 8 * v, n0, r, s_bias, s_M, s_S, s_sig, best);
        }
      }
      // every epilogue warp is done reading buffer b (and with s_M etc.): release it
      tc_fence_before();
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (warp == 2 && lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_empty[b])) : "memory");
    }
    if (best) atomicMax(a.amax_key + best_r, best);
  }
  // ---- teardown: drain copies issued but never consumed (abort path), free TMEM ----
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag) {
    for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i) {
      for (uint32_t k = 0; k < (1u << 22); ++k)
        if (mbar_try_wait(&full_bar[i % S], (i / S) & 1)) break;
    }
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * NT));
  }
}

}  // namespace tc

// ---------------------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
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

// int8 row-major matrix [rows][K] -> 2-D tensor map with a (128 B x box_rows) box, 128-byte swizzle
cudaError_t make_tmap_i8(CUtensorMap* map, const void* base, int64_t rows, int64_t K, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (K & 15) || box_rows < 1 || box_rows > 256)
    return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K};
  const cuuint32_t box[2] = {(cuuint32_t)tc::BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int NT, int S>
static cudaError_t launch_tc_t(const CUtensorMap& ma, const CUtensorMap& mw, const LinearArgs& a, int ksplit,
                               int32_t* err, cudaStream_t st) {
  using L = tc::Smem<NT, S>;
  // per-device "attributes set" flags: host threads may launch concurrently (sessions on
  // several devices, the allocation-free entry point); setting an attribute twice is harmless
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(tc::k_linear_tc<NT, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(tc::k_linear_tc<NT, S>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    attr_set[dev].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + NT - 1) / NT, (a.R + tc::BM - 1) / tc::BM * ksplit, 1);
  cfg.blockDim = dim3(tc::kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = g_pdl ? 1 : 0;
  ++na;
  if (ksplit > 1) {
    // cluster spans ksplit CTAs along y; blockIdx.y / ksplit is the row tile
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = ksplit;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, tc::k_linear_tc<NT, S>, ma, mw, a, ksplit, err);
}

template <int NT, int S, int EW>
static cudaError_t launch_tc_persistent_t(const CUtensorMap& ma, const CUtensorMap& mw, const LinearArgs& a,
                                          int grid, int32_t* err, cudaStream_t st) {
  using L = tc::Smem<NT, S>;
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    const cudaError_t e = cudaFuncSetAttribute(tc::k_linear_tc_persistent<NT, S, EW>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    attr_set[dev].store(true, std::memory_order_release);
  }
  const cudaError_t e = launch_k(tc::k_linear_tc_persistent<NT, S, EW>, dim3(grid), dim3(64 + 32 * EW), L::kBytes,
                                 st, ma, mw, a, err);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_linear_tc_persistent(const CUtensorMap& map_a, const CUtensorMap& map_w, const LinearArgs& a,
                                        int nt, int sms, int32_t* err, cudaStream_t st) {
  if (a.R <= 0 || a.N <= 0) return cudaSuccess;
  const int tiles = (a.N + nt - 1) / nt * ((a.R + tc::BM - 1) / tc::BM);
  const int grid = tiles < sms ? tiles : sms;
  switch (nt) {
    case 128: return launch_tc_persistent_t<128, 6, 16>(map_a, map_w, a, grid, err, st);
    case 256: return launch_tc_persistent_t<256, 4, 16>(map_a, map_w, a, grid, err, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t prepare_linear_tc() { return encode_fn() ? cudaSuccess : cudaErrorNotSupported; }

cudaError_t launch_linear_tc(const CUtensorMap& map_a, const CUtensorMap& map_w, const LinearArgs& a, int nt,
                             int ksplit, int32_t* err, cudaStream_t st) {
  if (a.R <= 0 || a.N <= 0) return cudaSuccess;
  switch (nt) {
    case 16: return launch_tc_t<16, 4>(map_a, map_w, a, ksplit, err, st);
    case 32: return launch_tc_t<32, 4>(map_a, map_w, a, ksplit, err, st);
    case 64: return launch_tc_t<64, 4>(map_a, map_w, a, ksplit, err, st);
    case 128: return launch_tc_t<128, 4>(map_a, map_w, a, ksplit, err, st);
    case 256: return launch_tc_t<256, 3>(map_a, map_w, a, ksplit, err, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace llx
