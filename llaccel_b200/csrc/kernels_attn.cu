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

cudaError_t prepare_attention(size_t smem) {
  return cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st) {
  const int R = a.B * a.M;
  if (R <= 0) return cudaSuccess;
  const size_t smem = attention_smem_bytes(a.H, a.Hkv, a.D, a.max_seq);
  dim3 grid(R, a.Hkv);
  k_attention<<<grid, 256, smem, st>>>(a.q, a.kc, a.vc, a.out, a.M, a.H, a.Hkv, a.D, a.max_seq, a.d_pos, a.Ms, a.Ss,
                                        a.Mo, a.So, a.prob_bits, a.luts);
  return cudaGetLastError();
}

}  // namespace llx
