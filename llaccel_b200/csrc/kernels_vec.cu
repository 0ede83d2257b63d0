// Vector-engine kernels: embedding gather, RMSNorm(+QUANT), QUANT, RoPE(+QUANT+K write),
// KV write, ADD, MUL, SILU, argmax, row gather.  One warp per row for the row
// reductions; 16-byte loads and stores everywhere the row width allows (every width on
// this path is a multiple of 16 elements, NUMERICS.md "Counts are multiples of 16").
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "kernels.h"
#include "launch.cuh"
#include "numerics.cuh"

namespace llx {

int g_pdl = 1;


static inline unsigned grid1d(int64_t n, int per_block) { return (unsigned)((n + per_block - 1) / per_block); }

// ---- embedding gather (golden.py:369-373; host.cpp:108-113) ------------------------------
__global__ void k_embed(const int32_t* tokens, const int16_t* __restrict__ embed,
                        int16_t* out, int R, int dim, int vocab_rows, int32_t* err,
                        unsigned long long* amax_key) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  if (amax_key && threadIdx.x == 0) amax_key[r] = 0ull;
  const int tok = tokens[r];
  const int chunks = dim / 8;
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)r * dim);
  if (tok < 0 || tok >= vocab_rows) {
    if (tok >= vocab_rows && threadIdx.x == 0 && err) atomicExch(err, 1);
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) dst[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(embed + (int64_t)tok * dim);
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) dst[c] = src[c];
}

cudaError_t launch_embed(const int32_t* tokens, const int16_t* embed, int16_t* out, int R, int dim, int vocab_rows,
                         int32_t* err, unsigned long long* amax_key, cudaStream_t st) {
  if (R <= 0) return cudaSuccess;
  { const cudaError_t e_ = launch_k(k_embed, dim3(R), dim3(64), 0, st, tokens, embed, out, R, dim, vocab_rows, err,
                                    amax_key); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

__global__ void k_amax_finish(const unsigned long long* keys, int32_t* out, int R) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < R) out[r] = (int32_t)(0xFFFFFFFFu - (uint32_t)(keys[r] & 0xFFFFFFFFull));
}

cudaError_t launch_amax_finish(const unsigned long long* keys, int32_t* out, int R, cudaStream_t st) {
  if (R <= 0) return cudaSuccess;
  { const cudaError_t e_ = launch_k(k_amax_finish, dim3((R + 255) / 256), dim3(256), 0, st, keys, out, R);
    if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

// ---- RMSNorm (numerics.h:60-71; NUMERICS.md:88-111), optionally fused with QUANT -----------
__device__ __forceinline__ void unpack8(const uint4& v, int32_t* o) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = (int16_t)(w[i] & 0xFFFF);
    o[2 * i + 1] = (int16_t)(w[i] >> 16);
  }
}
__device__ __forceinline__ uint4 pack8(const int32_t* v) {
  uint4 r;
  r.x = (uint32_t)(uint16_t)v[0] | ((uint32_t)(uint16_t)v[1] << 16);
  r.y = (uint32_t)(uint16_t)v[2] | ((uint32_t)(uint16_t)v[3] << 16);
  r.z = (uint32_t)(uint16_t)v[4] | ((uint32_t)(uint16_t)v[5] << 16);
  r.w = (uint32_t)(uint16_t)v[6] | ((uint32_t)(uint16_t)v[7] << 16);
  return r;
}
__device__ __forceinline__ uint2 pack8_i8(const int32_t* v) {
  uint2 r;
  r.x = (uint32_t)(uint8_t)v[0] | ((uint32_t)(uint8_t)v[1] << 8) | ((uint32_t)(uint8_t)v[2] << 16) |
        ((uint32_t)(uint8_t)v[3] << 24);
  r.y = (uint32_t)(uint8_t)v[4] | ((uint32_t)(uint8_t)v[5] << 8) | ((uint32_t)(uint8_t)v[6] << 16) |
        ((uint32_t)(uint8_t)v[7] << 24);
  return r;
}

// The row is read into registers for the sum of squares: every 16-byte load of the row is
// issued before any is used.  The elementwise pass then re-reads the row's chunks (L1 hits)
// in a rolled loop: a kernel in the decode chain runs each instruction about once, so a
// short loop body fetched once beats unrolled straight-line code.
//   ss = sum x^2 (u64), r = isqrt48(ss + eps_t), inv = min(65535, C / max(r, 1)),
//   y = sat16(rshr(x * g * inv, sh_post)), y8 = sat8(mulshift(y, Mq, Sq))
// y (i16) is stored only when a later step reads it.  fastq: Sq >= 32 and Mq < 2^31, so the
// quant runs on the product's high word (mulshift_hi32).
__device__ __noinline__ void rms_finish(const uint4* xr, const uint4* __restrict__ gr, int c0, int cstep,
                                        int chunks, uint32_t inv, int sh_post, int64_t Mq, int Sq, bool fastq,
                                        uint4* yr, uint2* yq) {
#pragma unroll 1
  for (int c = c0; c < chunks; c += cstep) {
    int32_t v[8], g[8], o[8];
    unpack8(xr[c], v);
    unpack8(__ldg(gr + c), g);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = (int32_t)sat16(rshr((int64_t)(v[e] * g[e]) * (int64_t)inv, sh_post));
    if (yr) yr[c] = pack8(o);
    if (yq) {
      int32_t q[8];
      if (fastq) {
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = (int32_t)sat8(mulshift_hi32(o[e], (int32_t)Mq, Sq));
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = (int32_t)sat8(mulshift(o[e], Mq, Sq));
      }
      yq[c] = pack8_i8(q);
    }
  }
}

__device__ __forceinline__ uint64_t sumsq8(const uint4& x) {
  int32_t v[8];
  unpack8(x, v);
  uint64_t s = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) s += (uint32_t)(v[e] * v[e]);
  return s;
}

// one warp per row (K < 2048): CPL chunks of 8 values per lane
template <int CPL>
__global__ void __launch_bounds__(64) k_rmsnorm(const int16_t* x, const int16_t* __restrict__ gamma,
                                                int16_t* y, int8_t* y8, int nrows, int K,
                                                int64_t eps_t, int64_t C, int sh_post, int64_t Mq, int Sq, int fastq) {
  pdl_trigger();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int chunks = K / 8;
  const uint4* gr = reinterpret_cast<const uint4*>(gamma);
  uint4 xv[CPL];
  // gamma is a model constant: bring this lane's chunks into L1 before the dependency wait
#pragma unroll
  for (int i = 0; i < CPL; ++i)
    if (lane + 32 * i < chunks) asm volatile("prefetch.global.L1 [%0];" ::"l"(gr + lane + 32 * i));
  pdl_wait();
  if (row >= nrows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * K);
#pragma unroll
  for (int i = 0; i < CPL; ++i) xv[i] = lane + 32 * i < chunks ? xr[lane + 32 * i] : make_uint4(0, 0, 0, 0);
  uint64_t ss = 0;
#pragma unroll
  for (int i = 0; i < CPL; ++i) ss += sumsq8(xv[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  // ss + eps_t < 2^48 (K <= 65536 values of |x| <= 2^15, eps_t < 2^32) and C < 2^40
  const uint32_t r = isqrt48_fast(ss + (uint64_t)eps_t);
  uint64_t inv = udiv_fast((uint64_t)C, r > 1 ? r : 1);
  if (inv > 65535) inv = 65535;
  rms_finish(xr, gr, lane, 32, chunks, (uint32_t)inv, sh_post, Mq, Sq, fastq != 0,
             y ? reinterpret_cast<uint4*>(y + (int64_t)row * K) : nullptr,
             y8 ? reinterpret_cast<uint2*>(y8 + (int64_t)row * K) : nullptr);
}

// Wide rows (K >= 2048, e.g. Llama-3-8B's 4096), or few rows (at most two per SM, e.g. a
// 128-sequence decode step): one 256-thread block per row, CPT chunks per thread, so a small
// batch still spreads its rows over many SMs and each thread's elementwise chain is short.
// Same arithmetic.
template <int CPT>
__global__ void __launch_bounds__(256) k_rmsnorm_wide(const int16_t* x, const int16_t* __restrict__ gamma,
                                                      int16_t* y, int8_t* y8, int K,
                                                      int64_t eps_t, int64_t C, int sh_post, int64_t Mq, int Sq,
                                                      int fastq) {
  pdl_trigger();
  __shared__ uint64_t part[8];
  const int row = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int chunks = K / 8;
  const uint4* gr = reinterpret_cast<const uint4*>(gamma);
  uint4 xv[CPT];
#pragma unroll
  for (int i = 0; i < CPT; ++i)
    if ((int)threadIdx.x + 256 * i < chunks) asm volatile("prefetch.global.L1 [%0];" ::"l"(gr + threadIdx.x + 256 * i));
  pdl_wait();
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * K);
#pragma unroll
  for (int i = 0; i < CPT; ++i)
    xv[i] = (int)threadIdx.x + 256 * i < chunks ? xr[threadIdx.x + 256 * i] : make_uint4(0, 0, 0, 0);
  uint64_t ss = 0;
#pragma unroll
  for (int i = 0; i < CPT; ++i) ss += sumsq8(xv[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) part[w] = ss;
  __syncthreads();
  uint64_t t = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) t += part[i];
  const uint32_t r = isqrt48_fast(t + (uint64_t)eps_t);
  uint64_t inv = udiv_fast((uint64_t)C, r > 1 ? r : 1);
  if (inv > 65535) inv = 65535;
  rms_finish(xr, gr, threadIdx.x, 256, chunks, (uint32_t)inv, sh_post, Mq, Sq, fastq != 0,
             y ? reinterpret_cast<uint4*>(y + (int64_t)row * K) : nullptr,
             y8 ? reinterpret_cast<uint2*>(y8 + (int64_t)row * K) : nullptr);
}

cudaError_t launch_rmsnorm(const int16_t* x, const int16_t* gamma, int16_t* y, int8_t* y8, int nrows, int K,
                           int64_t eps_t, int64_t C, int sh_post, int64_t Mq, int Sq, cudaStream_t st) {
  if (nrows <= 0) return cudaSuccess;
  const int fastq = (Sq >= 32 && Mq >= 0 && Mq < (int64_t)1 << 31) ? 1 : 0;
  const int chunks = K / 8;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  cudaError_t e;
  if (K >= 2048 || nrows <= 2 * sms) {
    const int cpt = (chunks + 255) / 256;
    auto kern = cpt <= 1 ? k_rmsnorm_wide<1> : cpt <= 2 ? k_rmsnorm_wide<2> : cpt <= 4 ? k_rmsnorm_wide<4> : k_rmsnorm_wide<8>;
    if (cpt > 8) return cudaErrorInvalidValue;
    e = launch_k(kern, dim3(nrows), dim3(256), 0, st, x, gamma, y, y8, K, eps_t, C, sh_post, Mq, Sq, fastq);
  } else {
    const int cpl = (chunks + 31) / 32;
    auto kern = cpl <= 1 ? k_rmsnorm<1> : cpl <= 2 ? k_rmsnorm<2> : cpl <= 4 ? k_rmsnorm<4> : k_rmsnorm<8>;
    e = launch_k(kern, dim3(grid1d(nrows, 2)), dim3(64), 0, st, x, gamma, y, y8, nrows, K, eps_t, C, sh_post, Mq, Sq,
                 fastq);
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

// ---- QUANT i16 -> i8 (numerics.h:56) -------------------------------------------------------
__global__ void k_quant(const int16_t* x, int8_t* y, int64_t n8, int64_t M, int S) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  int32_t v[8], q[8];
  unpack8(reinterpret_cast<const uint4*>(x)[i], v);
#pragma unroll
  for (int k = 0; k < 8; ++k) q[k] = (int32_t)sat8(mulshift(v[k], M, S));
  reinterpret_cast<uint2*>(y)[i] = pack8_i8(q);
}

cudaError_t launch_quant(const int16_t* x, int8_t* y, int64_t n, int64_t M, int S, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int64_t n8 = n / 8;
  { const cudaError_t e_ = launch_k(k_quant, dim3(grid1d(n8, 256)), dim3(256), 0, st, x, y, n8, M, S); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

// ---- RoPE (numerics.h:75-84; NUMERICS.md:113-125) [+ QUANT] [+ K cache write] ------------
// thread per (row, head, i < D/2): rotates the (i, i + D/2) pair.
__global__ void k_rope(const int16_t* x, int16_t* y16, int8_t* y8,
                       int64_t Mq, int Sq, int8_t* kcache, int R, int M, int H, int D,
                       const int16_t* __restrict__ cos_tab, const int16_t* __restrict__ sin_tab,
                       const int* d_pos, int max_seq) {
  pdl_trigger();
  pdl_wait();
  const int half = D >> 1;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)R * H * half;
  if (idx >= total) return;
  const int i = (int)(idx % half);
  const int h = (int)((idx / half) % H);
  const int r = (int)(idx / ((int64_t)half * H));
  const int m = r % M;
  const int p = *d_pos + m;
  const int64_t base = (int64_t)r * H * D + (int64_t)h * D;
  const int64_t x1 = x[base + i], x2 = x[base + i + half];
  const int64_t c = cos_tab[(int64_t)p * half + i], s = sin_tab[(int64_t)p * half + i];
  const int64_t a = sat16(rshr(x1 * c - x2 * s, 14));
  const int64_t b = sat16(rshr(x2 * c + x1 * s, 14));
  if (y16) {
    y16[base + i] = (int16_t)a;
    y16[base + i + half] = (int16_t)b;
  }
  if (y8) {
    const int8_t qa = (int8_t)sat8(mulshift(a, Mq, Sq)), qb = (int8_t)sat8(mulshift(b, Mq, Sq));
    y8[base + i] = qa;
    y8[base + i + half] = qb;
    if (kcache) {
      const int bseq = r / M;
      int8_t* dst = kcache + (((int64_t)bseq * H + h) * max_seq + p) * D;
      dst[i] = qa;
      dst[i + half] = qb;
    }
  }
}

cudaError_t launch_rope(const int16_t* x, int16_t* y16, int8_t* y8, int64_t Mq, int Sq, int8_t* kcache, int R, int M,
                        int H, int D, const int16_t* cos_tab, const int16_t* sin_tab, const int* d_pos, int max_seq,
                        cudaStream_t st) {
  const int64_t total = (int64_t)R * H * (D / 2);
  if (total <= 0) return cudaSuccess;
  { const cudaError_t e_ = launch_k(k_rope, dim3(grid1d(total, 256)), dim3(256), 0, st, x, y16, y8, Mq, Sq, kcache, R, M, H, D, cos_tab, sin_tab, d_pos,
                                             max_seq); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

// ---- RoPE group: q and k rotations (+ QUANT, K cache) and the V cache copy, one launch --------
__device__ __forceinline__ void rope_pair(const RopeJob& j, int r, int h, int i, int M, int D, int p,
                                          const int16_t* __restrict__ cos_tab, const int16_t* __restrict__ sin_tab,
                                          int max_seq) {
  const int half = D >> 1;
  const int64_t base = (int64_t)r * j.H * D + (int64_t)h * D;
  const int64_t x1 = j.x[base + i], x2 = j.x[base + i + half];
  const int64_t c = cos_tab[(int64_t)p * half + i], s = sin_tab[(int64_t)p * half + i];
  const int64_t a = sat16(rshr(x1 * c - x2 * s, 14));
  const int64_t b = sat16(rshr(x2 * c + x1 * s, 14));
  if (j.y16) {
    j.y16[base + i] = (int16_t)a;
    j.y16[base + i + half] = (int16_t)b;
  }
  if (j.y8) {
    const int8_t qa = (int8_t)sat8(mulshift(a, j.Mq, j.Sq)), qb = (int8_t)sat8(mulshift(b, j.Mq, j.Sq));
    j.y8[base + i] = qa;
    j.y8[base + i + half] = qb;
    if (j.kcache) {
      int8_t* dst = j.kcache + (((int64_t)(r / M) * j.H + h) * max_seq + p) * D;
      dst[i] = qa;
      dst[i + half] = qb;
    }
  }
}

__global__ void k_rope_group(RopeJob q, RopeJob k, const int8_t* v, int8_t* vcache,
                             int Hkv, int R, int M, int D, const int16_t* __restrict__ cos_tab,
                             const int16_t* __restrict__ sin_tab, const int* d_pos, int max_seq) {
  pdl_trigger();
  pdl_wait();
  const int half = D >> 1;
  const int64_t nq = (int64_t)R * q.H * half, nk = (int64_t)R * k.H * half;
  const int cpr = D / 16;
  const int64_t nv = v ? (int64_t)R * Hkv * cpr : 0;
  const int pos = *d_pos;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < nq + nk + nv;
       idx += (int64_t)gridDim.x * blockDim.x) {
    if (idx < nq + nk) {
      const RopeJob& j = idx < nq ? q : k;
      const int64_t t = idx < nq ? idx : idx - nq;
      const int i = (int)(t % half);
      const int h = (int)((t / half) % j.H);
      const int r = (int)(t / ((int64_t)half * j.H));
      rope_pair(j, r, h, i, M, D, pos + r % M, cos_tab, sin_tab, max_seq);
    } else {
      const int64_t t = idx - nq - nk;
      const int c = (int)(t % cpr);
      const int h = (int)((t / cpr) % Hkv);
      const int r = (int)(t / ((int64_t)cpr * Hkv));
      const int64_t src = (int64_t)r * Hkv * D + (int64_t)h * D + c * 16;
      const int64_t dst = (((int64_t)(r / M) * Hkv + h) * max_seq + pos + r % M) * D + c * 16;
      *reinterpret_cast<uint4*>(vcache + dst) = *reinterpret_cast<const uint4*>(v + src);
    }
  }
}

cudaError_t launch_rope_group(const RopeJob& q, const RopeJob& k, const int8_t* v, int8_t* vcache, int Hkv, int R,
                              int M, int D, const int16_t* cos_tab, const int16_t* sin_tab, const int* d_pos,
                              int max_seq, cudaStream_t st) {
  const int64_t total = (int64_t)R * (q.H + k.H) * (D / 2) + (v ? (int64_t)R * Hkv * (D / 16) : 0);
  if (total <= 0) return cudaSuccess;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
  { const cudaError_t e_ = launch_k(k_rope_group, dim3((unsigned)blocks), dim3(256), 0, st, q, k, v, vcache, Hkv, R, M, D,
                                    cos_tab, sin_tab, d_pos, max_seq); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

// ---- KV write (golden.py:344-351; funcsim.cpp:377-396) ----------------------------------
// thread per 16-byte chunk of one (row, kv head) segment
__global__ void k_kv_write(const int8_t* k, const int8_t* v, int8_t* kc,
                           int8_t* vc, int R, int M, int Hkv, int D, const int* d_pos,
                           int max_seq) {
  pdl_trigger();
  pdl_wait();
  const int cpr = D / 16;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)R * Hkv * cpr;
  if (idx >= total) return;
  const int c = (int)(idx % cpr);
  const int h = (int)((idx / cpr) % Hkv);
  const int r = (int)(idx / ((int64_t)cpr * Hkv));
  const int bseq = r / M, m = r % M;
  const int p = *d_pos + m;
  const int64_t src = (int64_t)r * Hkv * D + (int64_t)h * D + c * 16;
  const int64_t dst = (((int64_t)bseq * Hkv + h) * max_seq + p) * D + c * 16;
  if (k) *reinterpret_cast<uint4*>(kc + dst) = *reinterpret_cast<const uint4*>(k + src);
  if (v) *reinterpret_cast<uint4*>(vc + dst) = *reinterpret_cast<const uint4*>(v + src);
}

cudaError_t launch_kv_write(const int8_t* k, const int8_t* v, int8_t* kc, int8_t* vc, int R, int M, int Hkv, int D,
                            const int* d_pos, int max_seq, cudaStream_t st) {
  const int64_t total = (int64_t)R * Hkv * (D / 16);
  if (total <= 0) return cudaSuccess;
  { const cudaError_t e_ = launch_k(k_kv_write, dim3(grid1d(total, 256)), dim3(256), 0, st, k, v, kc, vc, R, M, Hkv, D, d_pos, max_seq); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

// ---- elementwise ADD / MUL / SILU (numerics.h:45-55) ----------------------------------------
__global__ void k_add(const int16_t* a, const int16_t* b, int16_t* y,
                      int64_t n8, int sh_b) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  int32_t va[8], vb[8], o[8];
  unpack8(reinterpret_cast<const uint4*>(a)[i], va);
  unpack8(reinterpret_cast<const uint4*>(b)[i], vb);
#pragma unroll
  for (int k = 0; k < 8; ++k) o[k] = (int32_t)sat16((int64_t)va[k] + rshr(vb[k], sh_b));
  reinterpret_cast<uint4*>(y)[i] = pack8(o);
}

__global__ void k_mul(const int16_t* a, const int16_t* b, int16_t* y,
                      int64_t n8, int sh) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  int32_t va[8], vb[8], o[8];
  unpack8(reinterpret_cast<const uint4*>(a)[i], va);
  unpack8(reinterpret_cast<const uint4*>(b)[i], vb);
#pragma unroll
  for (int k = 0; k < 8; ++k) o[k] = (int32_t)sat16(rshr((int64_t)va[k] * vb[k], sh));
  reinterpret_cast<uint4*>(y)[i] = pack8(o);
}

__global__ void k_silu(const int16_t* x, int16_t* y, int64_t n8, int64_t Mi, int Si,
                       int sh_out, const uint16_t* __restrict__ sig) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  int32_t v[8], o[8];
  unpack8(reinterpret_cast<const uint4*>(x)[i], v);
#pragma unroll
  for (int k = 0; k < 8; ++k) o[k] = (int32_t)silu16(v[k], Mi, Si, sh_out, sig);
  reinterpret_cast<uint4*>(y)[i] = pack8(o);
}

cudaError_t launch_add(const int16_t* a, const int16_t* b, int16_t* y, int64_t n, int sh_b, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  { const cudaError_t e_ = launch_k(k_add, dim3(grid1d(n / 8, 256)), dim3(256), 0, st, a, b, y, n / 8, sh_b); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}
cudaError_t launch_mul(const int16_t* a, const int16_t* b, int16_t* y, int64_t n, int sh, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  { const cudaError_t e_ = launch_k(k_mul, dim3(grid1d(n / 8, 256)), dim3(256), 0, st, a, b, y, n / 8, sh); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}
cudaError_t launch_silu(const int16_t* x, int16_t* y, int64_t n, int64_t Mi, int Si, int sh_out,
                        const uint16_t* luts, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  { const cudaError_t e_ = launch_k(k_silu, dim3(grid1d(n / 8, 256)), dim3(256), 0, st, x, y, n / 8, Mi, Si, sh_out, luts + kLutSig); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

// ---- argmax over the first `vocab` logits, lowest index on ties (NUMERICS.md:207-208) --------
// Grid (rows, slices): each block takes one slice of a row's first `vocab` logits and folds
// its best packed key (logit + 32768) << 32 | (0xFFFFFFFF - (base + n)) into keys[r] with a
// 64-bit atomicMax (keys zeroed beforehand); the max key is the row's first maximum.
__global__ void k_argmax(const int16_t* logits, int ld, int vocab, int base, int slice,
                         unsigned long long* keys) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  const int16_t* row = logits + (int64_t)r * ld;
  const int n0 = blockIdx.y * slice, n1 = min(vocab, n0 + slice);
  unsigned long long best = 0;
  for (int i = n0 + threadIdx.x; i < n1; i += blockDim.x) {
    const unsigned long long key =
        ((unsigned long long)(uint32_t)((int32_t)row[i] + 32768) << 32) | (0xFFFFFFFFu - (uint32_t)(base + i));
    best = key > best ? key : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  __shared__ unsigned long long warp_best[32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_best[w] = best;
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? warp_best[lane] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0 && best) atomicMax(keys + r, best);
  }
}

cudaError_t launch_argmax(const int16_t* logits, int R, int ld, int vocab, int base, unsigned long long* keys,
                          cudaStream_t st) {
  if (R <= 0 || vocab <= 0) return cudaSuccess;
  const int slice = 8192;
  const dim3 grid(R, (vocab + slice - 1) / slice);
  { const cudaError_t e_ = launch_k(k_argmax, grid, dim3(256), 0, st, logits, ld, vocab, base, slice, keys); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

// ---- tensor-parallel requant of all-reduced partial sums -----------------------------------
// Eight channels per thread: one 32-byte load of accumulators, one 16-byte (i16) or 8-byte
// (i8) store.  N is a multiple of 8, so a group never straddles two rows.
__global__ void k_requant(const int32_t* acc, LinearArgs a) {
  pdl_trigger();
  pdl_wait();
  const int64_t groups = (int64_t)a.R * a.N / 8;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = g * 8;
    const int n0 = (int)(e0 % a.N);
    const uint4 u0 = reinterpret_cast<const uint4*>(acc + e0)[0];
    const uint4 u1 = reinterpret_cast<const uint4*>(acc + e0)[1];
    const int32_t v[8] = {(int32_t)u0.x, (int32_t)u0.y, (int32_t)u0.z, (int32_t)u0.w,
                          (int32_t)u1.x, (int32_t)u1.y, (int32_t)u1.z, (int32_t)u1.w};
    int32_t o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + j;
      int64_t t = (int64_t)v[j] + (a.bias ? (int64_t)a.bias[n] : 0);
      t = mulshift(t, (int64_t)(uint32_t)a.rq[2 * n], a.rq[2 * n + 1]);
      if (a.out_i8) {
        o[j] = (int32_t)sat8(t);
        continue;
      }
      t = sat16(t);
      switch (a.epi) {
        case EPI_RESADD: t = sat16(t + (int64_t)a.aux[e0 + j]); break;
        case EPI_SILU: t = silu16(t, a.silu_Mi, a.silu_Si, a.silu_sh, a.luts + kLutSig); break;
        case EPI_MUL: t = sat16(rshr(t * (int64_t)a.aux[e0 + j], a.aux_shift)); break;
        default: break;
      }
      o[j] = (int32_t)t;
    }
    if (a.out_i8) {
      uint2 w;
      w.x = (uint32_t)(uint8_t)o[0] | (uint32_t)(uint8_t)o[1] << 8 | (uint32_t)(uint8_t)o[2] << 16 |
            (uint32_t)(uint8_t)o[3] << 24;
      w.y = (uint32_t)(uint8_t)o[4] | (uint32_t)(uint8_t)o[5] << 8 | (uint32_t)(uint8_t)o[6] << 16 |
            (uint32_t)(uint8_t)o[7] << 24;
      *reinterpret_cast<uint2*>(reinterpret_cast<int8_t*>(a.out) + e0) = w;
    } else {
      uint4 w;
      w.x = (uint32_t)(uint16_t)o[0] | (uint32_t)(uint16_t)o[1] << 16;
      w.y = (uint32_t)(uint16_t)o[2] | (uint32_t)(uint16_t)o[3] << 16;
      w.z = (uint32_t)(uint16_t)o[4] | (uint32_t)(uint16_t)o[5] << 16;
      w.w = (uint32_t)(uint16_t)o[6] | (uint32_t)(uint16_t)o[7] << 16;
      *reinterpret_cast<uint4*>(reinterpret_cast<int16_t*>(a.out) + e0) = w;
    }
  }
}

cudaError_t launch_requant(const int32_t* acc, const LinearArgs& a, cudaStream_t st) {
  const int64_t groups = (int64_t)a.R * a.N / 8;
  if (groups <= 0) return cudaSuccess;
  const int blocks = (int)std::min<int64_t>((groups + 255) / 256, 148 * 8);
  { const cudaError_t e_ = launch_k(k_requant, dim3(blocks), dim3(256), 0, st, acc, a); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

// ---- row gather ----------------------------------------------------------------------------
__global__ void k_gather_rows(const uint4* src, uint4* dst, const int32_t* idx,
                              int chunks) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  const int64_t s = (int64_t)idx[i] * chunks, d = (int64_t)i * chunks;
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) dst[d + c] = src[s + c];
}

cudaError_t launch_gather_rows(const void* src, void* dst, const int32_t* idx, int n, int row_bytes,
                               cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  { const cudaError_t e_ = launch_k(k_gather_rows, dim3(n), dim3(128), 0, st, reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), idx,
                                   row_bytes / 16); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

}  // namespace llx
