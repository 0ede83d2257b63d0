// Attention engine: causal GQA integer-softmax attention over the int8 KV cache
// (NUMERICS.md:150-197; numerics.h:88-120; golden.py:353-366).
//
// One CTA per (query row, KV head) serves the H/Hkv query heads that share the KV head,
// so each key row is read once for all of them.  The score pass keeps every score of the
// row on chip; max, exp-sum and the value pass follow the reference's global order
// (max over all keys, then the sum, then normalised probabilities x V), so the result is
// the reference's bit for bit regardless of how keys are split among threads: all
// reductions are integer max / integer sums.
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>

#include "kernels.h"
#include "launch.cuh"
#include "numerics.cuh"

namespace llx {

size_t attention_smem_bytes(int H, int Hkv, int D, int T) {
  const int rep = H / Hkv;
  return (size_t)rep * D + (size_t)rep * T * 4 + 64 * sizeof(long long);
}

__device__ __forceinline__ int dot4(uint32_t a, uint32_t b, int acc) { return __dp4a((int)a, (int)b, acc); }

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T* scratch, Op op) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) scratch[w] = v;
  __syncthreads();
  T r = scratch[0];
  for (int i = 1; i < nw; ++i) r = op(r, scratch[i]);
  return r;
}

__global__ void k_attention(const int8_t* __restrict__ q, const int8_t* __restrict__ kc, const int8_t* __restrict__ vc,
                            int8_t* __restrict__ out, int M, int H, int Hkv, int D, int max_seq,
                            const int* __restrict__ d_pos, int64_t Ms, int Ss, int64_t Mo, int So, int prob_bits,
                            const uint16_t* __restrict__ luts) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint16_t s_expi[16], s_expf[256];
  for (int i = threadIdx.x; i < 16 + 256; i += blockDim.x) {
    if (i < 16)
      s_expi[i] = luts[kLutExpI + i];
    else
      s_expf[i - 16] = luts[kLutExpF + i - 16];
  }
  const int r = blockIdx.x, kvh = blockIdx.y;
  const int bseq = r / M, m = r % M;
  const int rep = H / Hkv;
  const int T = *d_pos + m + 1;
  int8_t* q_s = reinterpret_cast<int8_t*>(smem);
  int32_t* sc = reinterpret_cast<int32_t*>(smem + ((rep * D + 15) & ~15));
  long long* red = reinterpret_cast<long long*>(sc + (size_t)rep * max_seq);

  const int8_t* qrow = q + (int64_t)r * H * D + (int64_t)kvh * rep * D;
  for (int i = threadIdx.x; i < rep * D / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(q_s)[i] = reinterpret_cast<const uint4*>(qrow)[i];
  __syncthreads();

  const int8_t* kbase = kc + ((int64_t)bseq * Hkv + kvh) * max_seq * D;
  const int8_t* vbase = vc + ((int64_t)bseq * Hkv + kvh) * max_seq * D;

  // scores s[j][t] = q_j . k_t (i32)
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const uint4* kr = reinterpret_cast<const uint4*>(kbase + (int64_t)t * D);
    for (int j = 0; j < rep; ++j) {
      const uint4* qj = reinterpret_cast<const uint4*>(q_s + j * D);
      int acc = 0;
      for (int c = 0; c < D / 16; ++c) {
        const uint4 kv = kr[c], qv = qj[c];
        acc = dot4(kv.x, qv.x, acc);
        acc = dot4(kv.y, qv.y, acc);
        acc = dot4(kv.z, qv.z, acc);
        acc = dot4(kv.w, qv.w, acc);
      }
      sc[j * max_seq + t] = acc;
    }
  }
  __syncthreads();

  const int pmax = (1 << prob_bits) - 1;
  const int pshift = 31 - prob_bits;
  for (int j = 0; j < rep; ++j) {
    int32_t* s = sc + j * max_seq;
    long long mx = LLONG_MIN;
    for (int t = threadIdx.x; t < T; t += blockDim.x) mx = s[t] > mx ? s[t] : mx;
    mx = block_reduce<long long>(mx, red, [](long long a, long long b) { return a > b ? a : b; });
    long long sum = 0;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
      const uint32_t p = exp_prob(mulshift(mx - (long long)s[t], Ms, Ss), s_expi, s_expf);
      s[t] = (int32_t)p;
      sum += p;
    }
    sum = block_reduce<long long>(sum, red, [](long long a, long long b) { return a + b; });
    const int64_t inv = udiv((uint64_t)1 << 31, (uint64_t)(uint32_t)sum);
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
      const int64_t pn = rshr((int64_t)s[t] * inv, pshift);
      s[t] = (int32_t)(pn < pmax ? pn : pmax);
    }
  }
  __syncthreads();

  // o[j][d] = sum_t pn[j][t] * v[t][d]
  int8_t* orow = out + (int64_t)r * H * D + (int64_t)kvh * rep * D;
  for (int idx = threadIdx.x; idx < rep * D; idx += blockDim.x) {
    const int j = idx / D, d = idx % D;
    const int32_t* pn = sc + j * max_seq;
    int32_t acc = 0;
    for (int t = 0; t < T; ++t) acc += pn[t] * (int32_t)vbase[(int64_t)t * D + d];
    int64_t o = acc;
    if (prob_bits == 15) o = rshr(o, 7);
    orow[idx] = (int8_t)sat8(mulshift(o, Mo, So));
  }
}

// ---------------------------------------------------------------------------------------
// Decode attention (one query row per sequence): one CTA per (sequence, KV head) streams
// the key rows, then the value rows, with 16-byte loads.  LPK = D/16 lanes share one key
// row; the H/Hkv query heads of the KV head reuse every loaded row.  Per-head max / sum /
// normalisation run one warp per head over the scores kept in shared memory; the value
// pass accumulates RB heads at a time in registers, reduces across lanes with shuffles and
// across warps through shared memory.  All reductions are integer: exact in any order.
// ---------------------------------------------------------------------------------------
constexpr int kDecThreads = 256, kDecWarps = kDecThreads / 32;

size_t attention_decode_smem_bytes(int H, int Hkv, int D, int max_seq) {
  const int rep = H / Hkv;
  // scores / probabilities (i32), normalised probabilities (i16), per-warp partial sums of
  // the value pass, q rows, per-warp head maxima and sums
  return (size_t)rep * D + (size_t)rep * max_seq * 4 + (size_t)rep * (size_t)((max_seq + 3) & ~1) * 2 +
         (size_t)kDecWarps * rep * D * 4 + (size_t)kDecWarps * rep * 8 + 64;
}

__device__ __forceinline__ int dot16_i8(const uint4& a, const uint4& b, int acc) {
  acc = __dp4a((int)a.x, (int)b.x, acc);
  acc = __dp4a((int)a.y, (int)b.y, acc);
  acc = __dp4a((int)a.z, (int)b.z, acc);
  acc = __dp4a((int)a.w, (int)b.w, acc);
  return acc;
}

template <int LPK, int RB>
__global__ void __launch_bounds__(kDecThreads) k_attention_decode(
    const int8_t* __restrict__ q, const int8_t* __restrict__ kc, const int8_t* __restrict__ vc, int8_t* __restrict__ out,
    int H, int Hkv, int max_seq, const int* __restrict__ d_pos, int64_t Ms, int Ss, int64_t Mo, int So, int prob_bits,
    const uint16_t* __restrict__ luts) {
  constexpr int D = LPK * 16;
  constexpr int KPW = 32 / LPK;  // key rows per warp per step
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint16_t s_expi[16], s_expf[256];
  const int rep = H / Hkv;
  const int pstride = (max_seq + 3) & ~1;                                // i16 row stride (even, > max_seq)
  int8_t* q_s = reinterpret_cast<int8_t*>(smem);                         // [rep][D] (16-byte rows)
  int32_t* sc = reinterpret_cast<int32_t*>(q_s + rep * D);               // [rep][max_seq] scores, then p
  int16_t* pn16 = reinterpret_cast<int16_t*>(sc + (size_t)rep * max_seq);  // [rep][pstride] normalised p
  int32_t* red = reinterpret_cast<int32_t*>(pn16 + (size_t)rep * pstride);  // [warps][rep][D]
  int32_t* wmax = red + (size_t)kDecWarps * rep * D;                     // [warps][rep]
  uint32_t* wsum = reinterpret_cast<uint32_t*>(wmax + kDecWarps * rep);  // [warps][rep]
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane % LPK, kg = lane / LPK;
  pdl_trigger();
  for (int i = threadIdx.x; i < 16 + 256; i += blockDim.x) {
    if (i < 16)
      s_expi[i] = luts[kLutExpI + i];
    else
      s_expf[i - 16] = luts[kLutExpF + i - 16];
  }
  pdl_wait();  // POS, q and the KV cache come from earlier kernels
  const int T = *d_pos + 1;
  const int8_t* qrow = q + ((int64_t)b * H + (int64_t)kvh * rep) * D;
  for (int i = threadIdx.x; i < rep * D / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(q_s)[i] = reinterpret_cast<const uint4*>(qrow)[i];
  __syncthreads();

  const int8_t* kbase = kc + ((int64_t)b * Hkv + kvh) * max_seq * D;
  const int8_t* vbase = vc + ((int64_t)b * Hkv + kvh) * max_seq * D;
  const int stride = kDecWarps * KPW;

  // ---- scores, with each head's running maximum ----
  int32_t mxl[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) mxl[j] = INT_MIN;
  for (int t0 = warp * KPW; t0 < T; t0 += 2 * stride) {
    const int ta = t0 + kg, tb = t0 + stride + kg;
    uint4 ka = make_uint4(0, 0, 0, 0), kb = make_uint4(0, 0, 0, 0);
    if (ta < T) ka = __ldg(reinterpret_cast<const uint4*>(kbase + (int64_t)ta * D) + sub);
    if (tb < T) kb = __ldg(reinterpret_cast<const uint4*>(kbase + (int64_t)tb * D) + sub);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j >= rep) break;
      const uint4 qv = reinterpret_cast<const uint4*>(q_s + j * D)[sub];
      int sa = dot16_i8(ka, qv, 0), sb = dot16_i8(kb, qv, 0);
#pragma unroll
      for (int o = 1; o < LPK; o <<= 1) {
        sa += __shfl_xor_sync(0xffffffffu, sa, o);
        sb += __shfl_xor_sync(0xffffffffu, sb, o);
      }
      if (ta < T) {
        mxl[j] = max(mxl[j], sa);
        if (sub == 0) sc[j * max_seq + ta] = sa;
      }
      if (tb < T) {
        mxl[j] = max(mxl[j], sb);
        if (sub == 0) sc[j * max_seq + tb] = sb;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (j >= rep) break;
    int32_t v = mxl[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) wmax[warp * rep + j] = v;
  }
  __syncthreads();

  // ---- exp LUT probabilities and their sums (all threads, heads outer) ----
  const int pmax = (1 << prob_bits) - 1, pshift = 31 - prob_bits;
  for (int j = 0; j < rep; ++j) {
    int32_t mx = wmax[j];
    for (int w = 1; w < kDecWarps; ++w) mx = max(mx, wmax[w * rep + j]);
    int32_t* s = sc + j * max_seq;
    uint32_t sum = 0;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
      const uint32_t p = exp_prob(mulshift((int64_t)mx - s[t], Ms, Ss), s_expi, s_expf);
      s[t] = (int32_t)p;
      sum += p;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) wsum[warp * rep + j] = sum;
  }
  __syncthreads();
  // ---- normalised probabilities (Q0.15 or Q0.8) as i16, zero past the last key ----
  for (int j = 0; j < rep; ++j) {
    uint32_t sum = 0;
    for (int w = 0; w < kDecWarps; ++w) sum += wsum[w * rep + j];
    const int64_t inv = udiv((uint64_t)1 << 31, sum);
    const int32_t* s = sc + j * max_seq;
    int16_t* pj = pn16 + (size_t)j * pstride;
    for (int t = threadIdx.x; t < T + 2; t += blockDim.x) {
      int32_t v = 0;
      if (t < T) {
        const int64_t pn = rshr((int64_t)s[t] * inv, pshift);
        v = (int32_t)(pn < pmax ? pn : pmax);
      }
      if (t < pstride) pj[t] = (int16_t)v;
    }
  }
  __syncthreads();

  // ---- o[j][d] = sum_t pn[j][t] * v[t][d]: key pairs through dp2a, RB heads per pass ----
  int8_t* orow = out + ((int64_t)b * H + (int64_t)kvh * rep) * D;
  const int pair_stride = kDecWarps * KPW * 2;
  for (int j0 = 0; j0 < rep; j0 += RB) {
    int32_t acc[RB][16];
#pragma unroll
    for (int r = 0; r < RB; ++r)
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[r][i] = 0;
    for (int t = (warp * KPW + kg) * 2; t < T; t += pair_stride) {
      const uint4 va = __ldg(reinterpret_cast<const uint4*>(vbase + (int64_t)t * D) + sub);
      uint4 vb = make_uint4(0, 0, 0, 0);
      if (t + 1 < T) vb = __ldg(reinterpret_cast<const uint4*>(vbase + (int64_t)(t + 1) * D) + sub);
      // (v_t[d], v_t+1[d]) byte pairs: x[2k] holds d = 4k, 4k+1; x[2k+1] holds d = 4k+2, 4k+3
      const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
      uint32_t x[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        x[2 * k] = __byte_perm(wa[k], wb[k], 0x5140);
        x[2 * k + 1] = __byte_perm(wa[k], wb[k], 0x7362);
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const int j = j0 + r;
        if (j >= rep) break;
        // (pn[t], pn[t+1]) as two i16 halves; pn past T is zero
        const int pp = *reinterpret_cast<const int*>(pn16 + (size_t)j * pstride + t);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          acc[r][2 * k] = __dp2a_lo(pp, (int)x[k], acc[r][2 * k]);
          acc[r][2 * k + 1] = __dp2a_hi(pp, (int)x[k], acc[r][2 * k + 1]);
        }
      }
    }
    // lanes holding the same d chunk (same sub) but different keys
#pragma unroll
    for (int o = LPK; o < 32; o <<= 1)
#pragma unroll
      for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[r][i] += __shfl_xor_sync(0xffffffffu, acc[r][i], o);
    if (kg == 0) {
#pragma unroll
      for (int r = 0; r < RB; ++r)
        if (j0 + r < rep)
#pragma unroll
          for (int i = 0; i < 16; ++i) red[((size_t)warp * rep + j0 + r) * D + sub * 16 + i] = acc[r][i];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < RB * D; idx += blockDim.x) {
      const int j = j0 + idx / D, d = idx % D;
      if (j >= rep) continue;
      int32_t o = 0;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) o += red[((size_t)w * rep + j) * D + d];
      int64_t ov = o;
      if (prob_bits == 15) ov = rshr(ov, 7);
      orow[j * D + d] = (int8_t)sat8(mulshift(ov, Mo, So));
    }
    __syncthreads();
  }
}

template <int LPK, int RB>
static cudaError_t launch_dec_rb(const AttnArgs& a, size_t smem, cudaStream_t st) {
  const cudaError_t e = launch_k(k_attention_decode<LPK, RB>, dim3(a.B, a.Hkv), dim3(kDecThreads), smem, st, a.q, a.kc,
                                 a.vc, a.out, a.H, a.Hkv, a.max_seq, a.d_pos, a.Ms, a.Ss, a.Mo, a.So, a.prob_bits,
                                 a.luts);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// heads per value pass: up to 4 (register budget of the 16-wide accumulators)
template <int LPK>
static cudaError_t launch_dec_l(const AttnArgs& a, size_t smem, cudaStream_t st) {
  const int rep = a.H / a.Hkv;
  if (rep >= 4) return launch_dec_rb<LPK, 4>(a, smem, st);
  if (rep >= 2) return launch_dec_rb<LPK, 2>(a, smem, st);
  return launch_dec_rb<LPK, 1>(a, smem, st);
}
template <int LPK>
static cudaError_t prep_dec_l(size_t smem) {
  for (auto f : {k_attention_decode<LPK, 1>, k_attention_decode<LPK, 2>, k_attention_decode<LPK, 4>}) {
    const cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t prepare_attention(size_t smem) {
  cudaError_t e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  for (auto f : {prep_dec_l<1>, prep_dec_l<2>, prep_dec_l<4>, prep_dec_l<8>, prep_dec_l<16>}) {
    e = f(smem);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_attention_decode(const AttnArgs& a, cudaStream_t st) {
  if (a.B <= 0) return cudaSuccess;
  if (a.H / a.Hkv > 16) return cudaErrorInvalidValue;
  const size_t smem = attention_decode_smem_bytes(a.H, a.Hkv, a.D, a.max_seq);
  switch (a.D) {
    case 16: return launch_dec_l<1>(a, smem, st);
    case 32: return launch_dec_l<2>(a, smem, st);
    case 64: return launch_dec_l<4>(a, smem, st);
    case 128: return launch_dec_l<8>(a, smem, st);
    case 256: return launch_dec_l<16>(a, smem, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st) {
  const int R = a.B * a.M;
  if (R <= 0) return cudaSuccess;
  if (a.M == 1 && (a.D == 16 || a.D == 32 || a.D == 64 || a.D == 128 || a.D == 256) && a.H / a.Hkv <= 16)
    return launch_attention_decode(a, st);
  const size_t smem = attention_smem_bytes(a.H, a.Hkv, a.D, a.max_seq);
  dim3 grid(R, a.Hkv);
  { const cudaError_t e_ = launch_k(k_attention, dim3(grid), dim3(256), smem, st, a.q, a.kc, a.vc, a.out, a.M, a.H, a.Hkv, a.D, a.max_seq, a.d_pos, a.Ms, a.Ss,
                                        a.Mo, a.So, a.prob_bits, a.luts); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

}  // namespace llx
