// Matrix engine on CUDA cores: int8 x int8 -> int32 with the fused requant epilogue
// (NUMERICS.md:62-86; golden.py:316-342; funcsim.cpp:199-261).
//
//   acc = sum_k A[r][k] * W[n][k]            exact int32 (|acc| <= K * 2^14 < 2^31)
//   v   = acc + bias[n]                      int64 (33-bit, no wrap)
//   t   = sat16(mulshift(v, M_n, S_n))       or sat8(...) for i8 outputs
//   out = t | sat16(t + aux) | silu16(t) | sat16(rshr(t * aux, aux_shift))
//
// Two schedules: a GEMV for a few rows (weights streamed once with 16-byte loads, K split
// over 32 lanes x 8 warps), and a 64x64 smem-tiled dp4a GEMM for many rows.  The tensor-core
// path lives in gemm_tc.cu; these stay as the small-batch path and as its cross-check.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "kernels.h"
#include "launch.cuh"
#include "numerics.cuh"

namespace llx {

__device__ __forceinline__ int64_t linear_epilogue(int32_t acc, int r, int n, const LinearArgs& a) {
  if (a.out_i32) return acc;  // tensor-parallel partial sums
  int64_t v = acc;
  if (a.bias) v += a.bias[n];
  const int64_t M = a.rq[2 * n];
  const int S = a.rq[2 * n + 1];
  if (a.out_i8) return sat8(mulshift(v, M, S));
  const int64_t t = sat16(mulshift(v, M, S));
  switch (a.epi) {
    case EPI_RESADD: return sat16(t + (int64_t)a.aux[(int64_t)r * a.N + n]);
    case EPI_SILU: return silu16(t, a.silu_Mi, a.silu_Si, a.silu_sh, a.luts + kLutSig);
    case EPI_MUL: return sat16(rshr(t * (int64_t)a.aux[(int64_t)r * a.N + n], a.aux_shift));
    default: return t;
  }
}

__device__ __forceinline__ void store_out(const LinearArgs& a, int r, int n, int64_t v) {
  if (a.out_i32)
    reinterpret_cast<int32_t*>(a.out)[(int64_t)r * a.N + n] = (int32_t)v;
  else if (a.out_i8)
    reinterpret_cast<int8_t*>(a.out)[(int64_t)r * a.N + n] = (int8_t)v;
  else
    reinterpret_cast<int16_t*>(a.out)[(int64_t)r * a.N + n] = (int16_t)v;
}

__device__ __forceinline__ int dot16(const uint4& w, const uint4& x, int acc) {
  acc = __dp4a((int)w.x, (int)x.x, acc);
  acc = __dp4a((int)w.y, (int)x.y, acc);
  acc = __dp4a((int)w.z, (int)x.z, acc);
  acc = __dp4a((int)w.w, (int)x.w, acc);
  return acc;
}

// ---- GEMV: CPB output channels per 256-thread block, RB rows per block row -----------------
// Warp lanes split into CPB channels x LPC = 32 / CPB K slots; with 8 warps, K is cut into
// 8 * LPC slots of 16-byte chunks.  The weights are model constants: the first round of
// weight loads is issued before the grid dependency wait, so it streams while the previous
// kernel finishes, and from then on the next round is always in flight while the current one
// is consumed (two register buffers).  CPB = 4 (more blocks, half the serial rounds per
// thread) serves long rows (K >= 8192, e.g. a down projection); CPB = 8 the others.
// Fused forms (one launch instead of one per constituent linear):
//   multi-output (a.nseg > 0): q/k/v over row-concatenated weights, each channel stored to
//     its segment's output;
//   GATED: the gate/up pair over the interleaved weights (rows 32j..32j+15 gate, 32j+16..
//     32j+31 up of outputs 16j..16j+15): a thread accumulates the gate and the up row of its
//     output, and the epilogue applies silu16(gate) * up, the shift and the quant.
template <bool GATED>
__device__ __forceinline__ void gemv_finish(const LinearArgs& a, int r, int oo, int32_t s0, int32_t s1) {
  if (GATED) {
    const int ng = 32 * (oo >> 4) + (oo & 15), nu = ng + 16;
    const int64_t tg = sat16(mulshift((int64_t)s0 + (a.bias ? a.bias[ng] : 0), a.rq[2 * ng], a.rq[2 * ng + 1]));
    const int64_t tu = sat16(mulshift((int64_t)s1 + (a.bias ? a.bias[nu] : 0), a.rq[2 * nu], a.rq[2 * nu + 1]));
    const int64_t sg = silu16(tg, a.silu_Mi, a.silu_Si, a.silu_sh, a.luts + kLutSig);
    const int64_t f = sat16(rshr(tu * sg, a.aux_shift));
    const int64_t off = (int64_t)r * a.Nout + oo;
    if (a.g_out) a.g_out[off] = (int16_t)sg;
    if (a.f_out) a.f_out[off] = (int16_t)f;
    if (a.q_out) a.q_out[off] = (int8_t)sat8(mulshift(f, a.q_M, a.q_S));
  } else if (a.nseg > 0) {
    // multi-output linear (epilogue none): the channel's segment and its output
    int sgi = 0;
    while (sgi + 1 < a.nseg && oo >= a.seg_start[sgi + 1]) ++sgi;
    const int ld = a.seg_start[sgi + 1] - a.seg_start[sgi], col = oo - a.seg_start[sgi];
    const int64_t v = mulshift((int64_t)s0 + (a.bias ? a.bias[oo] : 0), a.rq[2 * oo], a.rq[2 * oo + 1]);
    if (a.seg_i8[sgi])
      reinterpret_cast<int8_t*>(a.seg_out[sgi])[(int64_t)r * ld + col] = (int8_t)sat8(v);
    else
      reinterpret_cast<int16_t*>(a.seg_out[sgi])[(int64_t)r * ld + col] = (int16_t)sat16(v);
  } else {
    store_out(a, r, oo, linear_epilogue(s0, r, oo, a));
  }
}

// The folded RMSNorm + quant of a one-row GEMV: the row nx [K] i16 -> xs [K] i8 in shared
// memory (every thread of the block takes part; ends with a block barrier).
__device__ __forceinline__ void gemv_norm_prologue(const LinearArgs& a, int8_t* xs) {
  __shared__ uint64_t nsum[8];
  __shared__ uint32_t ninv;
  const uint4* xr = reinterpret_cast<const uint4*>(a.nx);  // written by the previous kernel: coherent loads
  const uint4* gr = reinterpret_cast<const uint4*>(a.ngamma);
  const int chunks = a.K >> 3;
  uint64_t ss = 0;
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
    const uint4 v = xr[c];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int32_t lo = (int16_t)(w[e] & 0xFFFF), hi = (int16_t)(w[e] >> 16);
      ss += (uint32_t)(lo * lo) + (uint64_t)(uint32_t)(hi * hi);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) nsum[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t t = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += nsum[i];
    const uint32_t r = isqrt48_fast(t + (uint64_t)a.n_eps);
    const uint64_t inv = udiv_fast((uint64_t)a.n_C, r > 1 ? r : 1);
    ninv = (uint32_t)(inv > 65535 ? 65535 : inv);
  }
  __syncthreads();
  const int64_t inv = ninv;
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
    const uint4 v = xr[c], g = __ldg(gr + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w}, gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t q[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int32_t x = (int16_t)((w[e >> 1] >> (16 * (e & 1))) & 0xFFFF);
      const int32_t gg = (int16_t)((gw[e >> 1] >> (16 * (e & 1))) & 0xFFFF);
      const int64_t y = sat16(rshr((int64_t)(x * gg) * inv, a.n_sh));
      const int64_t qq = sat8(mulshift(y, a.n_Mq, a.n_Sq));
      q[e >> 2] |= (uint32_t)(uint8_t)qq << (8 * (e & 3));
    }
    reinterpret_cast<uint2*>(xs)[c] = make_uint2(q[0], q[1]);
  }
  __syncthreads();
}

// The block walks channel groups g = blockIdx.x, + gridDim.x, ... (one group per block unless
// the grid is smaller: the folded-norm launch caps it at 4 blocks per SM so that each block
// normalises the row once); the next group's first round of weights is requested while the
// current group's sums are reduced and stored.
template <int RB, bool GATED, int CPB, bool NORM = false>
__global__ void __launch_bounds__(256) k_gemv(LinearArgs a) {
  pdl_trigger();
  static_assert(!NORM || RB == 1, "the folded RMSNorm serves one row");
  extern __shared__ __align__(16) int8_t xs_norm[];  // NORM: the normalised, quantized row [K]
  constexpr int NW = GATED ? 2 : 1;        // weight rows per output channel
  constexpr int U = GATED ? 2 : 4;         // 16-byte loads per row and round
  constexpr int LPC = 32 / CPB;            // lanes per channel
  constexpr int SLOTS = 8 * LPC;           // K slots of the block
  constexpr int STEP = SLOTS * U;          // K chunks per round of the block
  __shared__ int32_t part[8][NW][CPB][RB];  // [warp][row kind][channel][row]
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = lane / LPC, sub = lane % LPC;
  const int slot = w * LPC + sub;
  const int r0 = blockIdx.y * RB;
  const int nout = GATED ? a.Nout : a.N;
  const int ngroups = (nout + CPB - 1) / CPB;
  const int nk = a.K >> 4;
  bool live = false;
  const uint4 *wr0 = nullptr, *wr1 = nullptr;
  auto set_group = [&](int g) {
    const int o = g * CPB + c;
    live = o < nout;
    const int wrow = GATED ? 32 * (o >> 4) + (o & 15) : o;  // gate row (the up row is 16 further)
    wr0 = reinterpret_cast<const uint4*>(a.W + (int64_t)(live ? wrow : 0) * a.K);
    wr1 = wr0 + (int64_t)16 * nk;
  };
  auto fetch = [&](int k0, uint4 (&wv)[NW][U]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = k0 + SLOTS * u;
      const bool ok = live && k < nk;
      wv[0][u] = ok ? __ldcs(wr0 + k) : make_uint4(0, 0, 0, 0);
      if (GATED) wv[NW - 1][u] = ok ? __ldcs(wr1 + k) : make_uint4(0, 0, 0, 0);
    }
  };
  int32_t acc[NW][RB];
  auto consume = [&](int k0, const uint4 (&wv)[NW][U]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = k0 + SLOTS * u;
      if (!live || k >= nk) break;
#pragma unroll
      for (int i = 0; i < RB; ++i) {
        const int r = r0 + i;
        if (r < a.R) {
          // written by the previous kernel: a coherent load (or the folded norm's row)
          const uint4 xv = NORM ? reinterpret_cast<const uint4*>(xs_norm)[k]
                                : reinterpret_cast<const uint4*>(a.A + (int64_t)r * a.K)[k];
#pragma unroll
          for (int h = 0; h < NW; ++h) acc[h][i] = dot16(wv[h][u], xv, acc[h][i]);
        }
      }
    }
  };
  uint4 b0[NW][U], b1[NW][U];
  int g = blockIdx.x;
  set_group(g);
  fetch(slot, b0);
  pdl_wait();  // the activation rows and the output buffers belong to earlier kernels
  if (NORM) gemv_norm_prologue(a, xs_norm);
  for (; g < ngroups; g += gridDim.x) {
#pragma unroll
    for (int h = 0; h < NW; ++h)
#pragma unroll
      for (int i = 0; i < RB; ++i) acc[h][i] = 0;
    for (int k0 = slot; k0 < nk; k0 += 2 * STEP) {
      fetch(k0 + STEP, b1);  // next round in flight while this one is consumed
      consume(k0, b0);
      if (k0 + STEP >= nk) break;
      fetch(k0 + 2 * STEP, b0);
      consume(k0 + STEP, b1);
    }
    const int o0 = g * CPB;
    // the next group's first round streams while this group's sums are reduced and stored
    if (g + (int)gridDim.x < ngroups) {
      set_group(g + gridDim.x);
      fetch(slot, b0);
    }
#pragma unroll
    for (int h = 0; h < NW; ++h)
#pragma unroll
      for (int i = 0; i < RB; ++i)
#pragma unroll
        for (int x = 1; x < LPC; x <<= 1) acc[h][i] += __shfl_xor_sync(0xffffffffu, acc[h][i], x);
    if (sub == 0) {
#pragma unroll
      for (int h = 0; h < NW; ++h)
#pragma unroll
        for (int i = 0; i < RB; ++i) part[w][h][c][i] = acc[h][i];
    }
    __syncthreads();
    for (int t = threadIdx.x; t < CPB * RB; t += blockDim.x) {
      const int cc = t / RB, i = t % RB;
      const int oo = o0 + cc, r = r0 + i;
      if (oo >= nout || r >= a.R) continue;
      int32_t sum[NW];
#pragma unroll
      for (int h = 0; h < NW; ++h) {
        sum[h] = 0;
#pragma unroll
        for (int ww = 0; ww < 8; ++ww) sum[h] += part[ww][h][cc][i];
      }
      gemv_finish<GATED>(a, r, oo, sum[0], sum[NW - 1]);
    }
    __syncthreads();  // part is reused by the next group
  }
}

template <int RB, bool GATED>
static cudaError_t launch_gemv_t(const LinearArgs& a, cudaStream_t st) {
  const int nout = GATED ? a.Nout : a.N;
  const bool narrow_blocks = a.K >= 8192;
  const int cpb = narrow_blocks ? 4 : 8;
  const dim3 grid((nout + cpb - 1) / cpb, (a.R + RB - 1) / RB);
  if constexpr (RB == 1) {
    if (a.nx) {  // the folded RMSNorm: K bytes of shared memory for the row
      if (a.K > 16384 || a.K % 16) return cudaErrorInvalidValue;
      // at most 4 blocks per SM, each normalising the row once and walking several groups
      static int sms[64] = {};
      int dev = 0;
      cudaGetDevice(&dev);
      if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
      if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
      const dim3 g1(std::min<unsigned>(grid.x, 4u * (unsigned)(sms[dev] > 0 ? sms[dev] : 148)), 1);
      return narrow_blocks ? launch_k(k_gemv<1, GATED, 4, true>, g1, dim3(256), (size_t)a.K, st, a)
                           : launch_k(k_gemv<1, GATED, 8, true>, g1, dim3(256), (size_t)a.K, st, a);
    }
  }
  if (a.nx) return cudaErrorInvalidValue;
  return narrow_blocks ? launch_k(k_gemv<RB, GATED, 4>, grid, dim3(256), 0, st, a)
                       : launch_k(k_gemv<RB, GATED, 8>, grid, dim3(256), 0, st, a);
}

// ---- tiled dp4a GEMM: 64 rows x 64 channels per block, 4x4 outputs per thread -----------
constexpr int TB = 64, TK = 64, TKW = TK / 4, PADW = TKW + 1;

__global__ void __launch_bounds__(256) k_gemm_tiled(LinearArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ uint32_t As[TB][PADW];
  __shared__ uint32_t Ws[TB][PADW];
  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;
  const int r0 = blockIdx.y * TB, n0 = blockIdx.x * TB;
  int32_t acc[4][4] = {};
  const int lrow = tid >> 2, lch = tid & 3;  // loader: row, 16-byte chunk
  for (int k0 = 0; k0 < a.K; k0 += TK) {
    const int kc = k0 + lch * 16;
    uint4 av = make_uint4(0, 0, 0, 0), wv = make_uint4(0, 0, 0, 0);
    if (r0 + lrow < a.R && kc < a.K) av = *reinterpret_cast<const uint4*>(a.A + (int64_t)(r0 + lrow) * a.K + kc);
    if (n0 + lrow < a.N && kc < a.K) wv = __ldg(reinterpret_cast<const uint4*>(a.W + (int64_t)(n0 + lrow) * a.K + kc));
    __syncthreads();
    As[lrow][lch * 4 + 0] = av.x;
    As[lrow][lch * 4 + 1] = av.y;
    As[lrow][lch * 4 + 2] = av.z;
    As[lrow][lch * 4 + 3] = av.w;
    Ws[lrow][lch * 4 + 0] = wv.x;
    Ws[lrow][lch * 4 + 1] = wv.y;
    Ws[lrow][lch * 4 + 2] = wv.z;
    Ws[lrow][lch * 4 + 3] = wv.w;
    __syncthreads();
#pragma unroll
    for (int kw = 0; kw < TKW; ++kw) {
      uint32_t ar[4], wr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) ar[i] = As[ty * 4 + i][kw];
#pragma unroll
      for (int j = 0; j < 4; ++j) wr[j] = Ws[tx * 4 + j][kw];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __dp4a((int)ar[i], (int)wr[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + ty * 4 + i;
    if (r >= a.R) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < a.N) store_out(a, r, n, linear_epilogue(acc[i][j], r, n, a));
    }
  }
}

cudaError_t launch_linear(const LinearArgs& a, int path, cudaStream_t st) {
  if (a.R <= 0 || a.N <= 0) return cudaSuccess;
  if (path == 0) path = a.R <= 16 ? 1 : 2;
  if (path == 1) {
    const cudaError_t e = a.R == 1 ? (a.gated ? launch_gemv_t<1, true>(a, st) : launch_gemv_t<1, false>(a, st))
                                   : (a.gated ? launch_gemv_t<4, true>(a, st) : launch_gemv_t<4, false>(a, st));
    if (e != cudaSuccess) return e;
  } else {
    dim3 grid((a.N + TB - 1) / TB, (a.R + TB - 1) / TB);
    { const cudaError_t e_ = launch_k(k_gemm_tiled, dim3(grid), dim3(256), 0, st, a); if (e_ != cudaSuccess) return e_; }
  }
  return cudaGetLastError();
}

}  // namespace llx
