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

// ---- GEMV: 8 channels per 256-thread block, RB rows per block row ------------------------
// The weights are model constants: a thread's first four 16-byte weight loads are issued
// before the grid dependency wait, so they stream while the previous kernel finishes.  Each
// later round of four is requested together, before any of it is consumed (one buffer:
// 38 registers keep 6 blocks per SM resident).
template <int RB>
__global__ void __launch_bounds__(256) k_gemv(LinearArgs a) {
  pdl_trigger();
  __shared__ int32_t part[8][8][RB];  // [warp][channel][row]
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = lane >> 2, sub = lane & 3;
  const int slot = w * 4 + sub;  // 0..31 over K
  const int n0 = blockIdx.x * 8, r0 = blockIdx.y * RB;
  const int n = n0 + c;
  const int nk = a.K >> 4;
  const bool live = n < a.N;
  const uint4* wr = reinterpret_cast<const uint4*>(a.W + (int64_t)(live ? n : 0) * a.K);
  auto fetch = [&](int k0, uint4 (&wv)[4]) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = k0 + 32 * u;
      wv[u] = live && k < nk ? __ldcs(wr + k) : make_uint4(0, 0, 0, 0);
    }
  };
  uint4 cur[4];
  fetch(slot, cur);
  pdl_wait();  // the activation rows and the output buffer belong to earlier kernels
  int32_t acc[RB];
#pragma unroll
  for (int i = 0; i < RB; ++i) acc[i] = 0;
  for (int k0 = slot; k0 < nk; k0 += 4 * 32) {
    if (k0 != slot) fetch(k0, cur);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = k0 + 32 * u;
      if (!live || k >= nk) break;
#pragma unroll
      for (int i = 0; i < RB; ++i) {
        const int r = r0 + i;
        if (r < a.R) {
          const uint4 xv = reinterpret_cast<const uint4*>(a.A + (int64_t)r * a.K)[k];  // written by the previous kernel: coherent load
          acc[i] = dot16(cur[u], xv, acc[i]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < RB; ++i) {
    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 1);
    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 2);
  }
  if (sub == 0) {
#pragma unroll
    for (int i = 0; i < RB; ++i) part[w][c][i] = acc[i];
  }
  __syncthreads();
  for (int t = threadIdx.x; t < 8 * RB; t += blockDim.x) {
    const int cc = t / RB, i = t % RB;
    const int nn = n0 + cc, r = r0 + i;
    if (nn >= a.N || r >= a.R) continue;
    int32_t s = 0;
#pragma unroll
    for (int ww = 0; ww < 8; ++ww) s += part[ww][cc][i];
    store_out(a, r, nn, linear_epilogue(s, r, nn, a));
  }
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
  if (path == 1 && a.R == 1) {
    const dim3 grid((a.N + 7) / 8, 1);
    { const cudaError_t e_ = launch_k(k_gemv<1>, grid, dim3(256), 0, st, a); if (e_ != cudaSuccess) return e_; }
  } else if (path == 1) {
    constexpr int RB = 4;
    dim3 grid((a.N + 7) / 8, (a.R + RB - 1) / RB);
    { const cudaError_t e_ = launch_k(k_gemv<RB>, dim3(grid), dim3(256), 0, st, a); if (e_ != cudaSuccess) return e_; }
  } else {
    dim3 grid((a.N + TB - 1) / TB, (a.R + TB - 1) / TB);
    { const cudaError_t e_ = launch_k(k_gemm_tiled, dim3(grid), dim3(256), 0, st, a); if (e_ != cudaSuccess) return e_; }
  }
  return cudaGetLastError();
}

}  // namespace llx
