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

template <int RB, bool GATED, int CPB>
__global__ void __launch_bounds__(256) k_gemv(LinearArgs a) {
  pdl_trigger();
  constexpr int NW = GATED ? 2 : 1;        // weight rows per output channel
  constexpr int U = GATED ? 2 : 4;         // 16-byte loads per row and round
  constexpr int LPC = 32 / CPB;            // lanes per channel
  constexpr int SLOTS = 8 * LPC;           // K slots of the block
  __shared__ int32_t part[8][NW][CPB][RB];  // [warp][row kind][channel][row]
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = lane / LPC, sub = lane % LPC;
  const int slot = w * LPC + sub;
  const int o0 = blockIdx.x * CPB, r0 = blockIdx.y * RB;
  const int o = o0 + c;
  const int nout = GATED ? a.Nout : a.N;
  const int nk = a.K >> 4;
  const bool live = o < nout;
  const int wrow = GATED ? 32 * (o >> 4) + (o & 15) : o;  // gate row (the up row is 16 further)
  const uint4* wr0 = reinterpret_cast<const uint4*>(a.W + (int64_t)(live ? wrow : 0) * a.K);
  const uint4* wr1 = wr0 + (int64_t)16 * nk;
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
#pragma unroll
  for (int h = 0; h < NW; ++h)
#pragma unroll
    for (int i = 0; i < RB; ++i) acc[h][i] = 0;
  auto consume = [&](int k0, const uint4 (&wv)[NW][U]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = k0 + SLOTS * u;
      if (!live || k >= nk) break;
#pragma unroll
      for (int i = 0; i < RB; ++i) {
        const int r = r0 + i;
        if (r < a.R) {
          // written by the previous kernel: a coherent load
          const uint4 xv = reinterpret_cast<const uint4*>(a.A + (int64_t)r * a.K)[k];
#pragma unroll
          for (int h = 0; h < NW; ++h) acc[h][i] = dot16(wv[h][u], xv, acc[h][i]);
        }
      }
    }
  };
  constexpr int STEP = SLOTS * U;  // K chunks per round of the block
  uint4 b0[NW][U], b1[NW][U];
  fetch(slot, b0);
  pdl_wait();  // the activation rows and the output buffers belong to earlier kernels
  for (int k0 = slot; k0 < nk; k0 += 2 * STEP) {
    fetch(k0 + STEP, b1);  // next round in flight while this one is consumed
    consume(k0, b0);
    if (k0 + STEP >= nk) break;
    fetch(k0 + 2 * STEP, b0);
    consume(k0 + STEP, b1);
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
}

template <int RB, bool GATED>
static cudaError_t launch_gemv_t(const LinearArgs& a, cudaStream_t st) {
  const int nout = GATED ? a.Nout : a.N;
  const bool narrow_blocks = a.K >= 8192;
  const int cpb = narrow_blocks ? 4 : 8;
  const dim3 grid((nout + cpb - 1) / cpb, (a.R + RB - 1) / RB);
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
