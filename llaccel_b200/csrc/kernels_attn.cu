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

// KV tiles stream through a ring of kRing shared-memory stages by 1-D bulk copies.
constexpr int kRing = 4;
__host__ __device__ constexpr int dec_tile_keys(int D) { return D <= 64 ? 256 : 16384 / D; }

// heads per CTA: a KV head's H/Hkv query heads are split into groups of at most 4
__host__ __device__ constexpr int dec_heads_per_cta(int rep) { return rep < 4 ? rep : 4; }

size_t attention_decode_smem_bytes(int H, int Hkv, int D, int max_seq) {
  const int rep = dec_heads_per_cta(H / Hkv);
  const size_t ring = (size_t)kRing * dec_tile_keys(D) * D;
  return ring + (size_t)rep * D + (size_t)rep * max_seq * 4 + (size_t)rep * (size_t)((max_seq + 3) & ~1) * 2 +
         (size_t)kDecWarps * rep * D * 4 + (size_t)kDecWarps * rep * 8 + 128;
}

__device__ __forceinline__ int dot16_i8(const uint4& a, const uint4& b, int acc) {
  acc = __dp4a((int)a.x, (int)b.x, acc);
  acc = __dp4a((int)a.y, (int)b.y, acc);
  acc = __dp4a((int)a.z, (int)b.z, acc);
  acc = __dp4a((int)a.w, (int)b.w, acc);
  return acc;
}

__device__ __forceinline__ uint32_t att_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// exp-LUT probability of a score gap d = mx - s >= 0 (numerics.h:104-107): z = rshr(d * Ms, Ss)
// with d < 2^31 and Ms < 2^32, so one u32 x u32 -> u64 product carries it exactly
__device__ __forceinline__ uint32_t gap_prob(uint32_t d, uint32_t Ms, int Ss, const uint16_t* expi, const uint16_t* expf) {
  const uint64_t prod = (uint64_t)d * Ms;
  const uint64_t z = Ss == 0 ? prod : (prod >> Ss) + ((prod >> (Ss - 1)) & 1ull);
  if (z >= 4096u) return 0;
  const uint32_t zi = (uint32_t)z;
  return ((uint32_t)expi[zi >> 8] * (uint32_t)expf[zi & 255] + (1u << 15)) >> 16;
}
__device__ __forceinline__ void att_mbar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(att_smem_u32(bar)));
}
__device__ __forceinline__ void att_bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(att_smem_u32(bar)), "r"(bytes) : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   att_smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(att_smem_u32(bar))
               : "memory");
}
// bounded wait on an mbarrier phase: false after ~2^26 polls
__device__ __forceinline__ bool att_mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < (1u << 26); ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(att_smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

template <int LPK, int RB>
__global__ void __launch_bounds__(kDecThreads) k_attention_decode(
    const int8_t* __restrict__ q, const int8_t* __restrict__ kc, const int8_t* __restrict__ vc, int8_t* __restrict__ out,
    int H, int Hkv, int max_seq, const int* __restrict__ d_pos, int64_t Ms, int Ss, int64_t Mo, int So, int prob_bits,
    const uint16_t* __restrict__ luts, int32_t* err) {
  constexpr int D = LPK * 16;
  constexpr int KPW = 32 / LPK;  // key rows per warp per step
  constexpr int TK = dec_tile_keys(D);
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint16_t s_expi[16], s_expf[256];
  __shared__ __align__(8) uint64_t full_bar[kRing];
  __shared__ int s_abort;
  __shared__ uint32_t s_inv[16];
  // this CTA serves query heads [h0, h0 + rep) of KV head blockIdx.y
  const int rep_all = H / Hkv;
  const int hg0 = blockIdx.z * RB;
  const int rep = min(RB, rep_all - hg0);
  const int pstride = (max_seq + 3) & ~1;
  int8_t* ring = reinterpret_cast<int8_t*>(smem);                        // [kRing][TK][D]
  int8_t* q_s = ring + (size_t)kRing * TK * D;                           // [rep][D]
  int32_t* sc = reinterpret_cast<int32_t*>(q_s + rep * D);               // [rep][max_seq] scores, then p
  int16_t* pn16 = reinterpret_cast<int16_t*>(sc + (size_t)rep * max_seq);  // [rep][pstride] normalised p
  int32_t* red = reinterpret_cast<int32_t*>(pn16 + (size_t)rep * pstride);  // [warps][rep][D]
  int32_t* wmax = red + (size_t)kDecWarps * rep * D;                     // [warps][rep]
  uint32_t* wsum = reinterpret_cast<uint32_t*>(wmax + kDecWarps * rep);  // [warps][rep]
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane % LPK, kg = lane / LPK;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kRing; ++i) att_mbar_init(&full_bar[i]);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  pdl_trigger();
  for (int i = threadIdx.x; i < 16 + 256; i += blockDim.x) {
    if (i < 16)
      s_expi[i] = luts[kLutExpI + i];
    else
      s_expf[i - 16] = luts[kLutExpF + i - 16];
  }
  pdl_wait();  // POS, q and the KV cache come from earlier kernels
  const int T = *d_pos + 1;
  const int ntile = (T + TK - 1) / TK;  // tiles of K, then as many of V
  const int8_t* kbase = kc + ((int64_t)b * Hkv + kvh) * max_seq * D;
  const int8_t* vbase = vc + ((int64_t)b * Hkv + kvh) * max_seq * D;
  auto issue = [&](int i) {  // tile i of the K-then-V sequence into stage i % kRing
    const int kv = i >= ntile, ti = kv ? i - ntile : i;
    const int t0 = ti * TK, nk = min(TK, T - t0);
    att_bulk_load(ring + (size_t)(i % kRing) * TK * D, (kv ? vbase : kbase) + (int64_t)t0 * D, (uint32_t)(nk * D),
                  &full_bar[i % kRing]);
  };
  __syncthreads();
  if (threadIdx.x == 0)
    for (int i = 0; i < min(kRing, 2 * ntile); ++i) issue(i);
  const int8_t* qrow = q + ((int64_t)b * H + (int64_t)kvh * rep_all + hg0) * D;
  for (int i = threadIdx.x; i < rep * D / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(q_s)[i] = reinterpret_cast<const uint4*>(qrow)[i];

  int32_t mxl[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) mxl[j] = INT_MIN;
  const int pmax = (1 << prob_bits) - 1, pshift = 31 - prob_bits;
  int32_t acc[RB][16];
  int8_t* orow = out + ((int64_t)b * H + (int64_t)kvh * rep_all + hg0) * D;
  {
    const int j0 = 0;  // rep <= RB: every head of this CTA in one pass over V
#pragma unroll
    for (int r = 0; r < RB; ++r)
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[r][i] = 0;
    for (int i = 0; i < 2 * ntile; ++i) {
      const int stage = i % kRing;
      const uint32_t parity = (uint32_t)((i / kRing) & 1);
      if (!att_mbar_wait(&full_bar[stage], parity)) {
        s_abort = 1;
        if (err) atomicExch(err, 5);
      }
      __syncthreads();
      if (s_abort) break;
      const int8_t* tile = ring + (size_t)stage * TK * D;
      const int kv = i >= ntile, ti = kv ? i - ntile : i;
      const int t0 = ti * TK, nk = min(TK, T - t0);
      if (!kv) {
        // ---- scores of this K tile (one key per lane), running per-head maxima ----
        // lane l reads its row's 16-byte chunks starting at chunk l % LPK, so the 32 rows of a
        // warp spread over all shared-memory banks
        for (int l = warp * 32 + lane; l < nk; l += 32 * kDecWarps) {
          const int8_t* krow = tile + (size_t)l * D;
          int sv[RB];
#pragma unroll
          for (int r = 0; r < RB; ++r) sv[r] = 0;
#pragma unroll
          for (int cc = 0; cc < LPK; ++cc) {
            const int c = (cc + l) % LPK;
            const uint4 kk = reinterpret_cast<const uint4*>(krow)[c];
#pragma unroll
            for (int r = 0; r < RB; ++r) {
              if (r < rep) sv[r] = dot16_i8(kk, reinterpret_cast<const uint4*>(q_s + r * D)[c], sv[r]);
            }
          }
#pragma unroll
          for (int r = 0; r < RB; ++r) {
            if (r < rep) {
              mxl[r] = max(mxl[r], sv[r]);
              sc[r * max_seq + t0 + l] = sv[r];
            }
          }
        }
        if (i == ntile - 1) {
          // ---- all scores are in: per-head max, exp LUT probabilities, sums, Q0.15 ----
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (j >= rep) break;
            int32_t v = mxl[j];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (lane == 0) wmax[warp * rep + j] = v;
          }
          __syncthreads();
          for (int j = 0; j < rep; ++j) {
            int32_t mx = wmax[j];
            for (int w = 1; w < kDecWarps; ++w) mx = max(mx, wmax[w * rep + j]);
            int32_t* sj = sc + j * max_seq;
            uint32_t sum = 0;
            for (int t = threadIdx.x; t < T; t += blockDim.x) {
              const uint32_t p = gap_prob((uint32_t)(mx - sj[t]), (uint32_t)Ms, Ss, s_expi, s_expf);
              sj[t] = (int32_t)p;
              sum += p;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) wsum[warp * rep + j] = sum;
          }
          __syncthreads();
          if (threadIdx.x < rep) {
            // inv = udiv(2^31, sum): 2^31 fits 32 bits, so a 32-bit divide is exact
            uint32_t sum = 0;
            for (int w = 0; w < kDecWarps; ++w) sum += wsum[w * rep + threadIdx.x];
            s_inv[threadIdx.x] = 0x80000000u / (sum ? sum : 1u);
          }
          __syncthreads();
          for (int j = 0; j < rep; ++j) {
            // p <= sum, so p * inv <= 2^31 - 1: the product and its rounding shift stay in 32 bits
            const uint32_t inv = s_inv[j];
            const int32_t* sj = sc + j * max_seq;
            int16_t* pj = pn16 + (size_t)j * pstride;
            for (int t = threadIdx.x; t < T + 2; t += blockDim.x) {
              int32_t v = 0;
              if (t < T) {
                const uint32_t x = (uint32_t)sj[t] * inv;
                const uint32_t pn = (x >> pshift) + ((x >> (pshift - 1)) & 1u);
                v = (int32_t)(pn < (uint32_t)pmax ? pn : (uint32_t)pmax);
              }
              if (t < pstride) pj[t] = (int16_t)v;
            }
          }
        }
      } else {
        // ---- values of this V tile: key pairs through dp2a ----
        for (int l = (warp * KPW + kg) * 2; l < nk; l += KPW * kDecWarps * 2) {
          const int t = t0 + l;
          const uint4 va = reinterpret_cast<const uint4*>(tile + (size_t)l * D)[sub];
          // the row after the last key is stale shared memory, weighted by pn = 0
          const uint4 vb = reinterpret_cast<const uint4*>(tile + (size_t)(l + 1) * D)[sub];
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
            const int pp = *reinterpret_cast<const int*>(pn16 + (size_t)j * pstride + t);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              acc[r][2 * k] = __dp2a_lo(pp, (int)x[k], acc[r][2 * k]);
              acc[r][2 * k + 1] = __dp2a_hi(pp, (int)x[k], acc[r][2 * k + 1]);
            }
          }
        }
      }
      __syncthreads();  // stage consumed by every thread
      if (threadIdx.x == 0 && i + kRing < 2 * ntile) issue(i + kRing);
    }
  }
  if (!s_abort) {
    const int j0 = 0;
    // ---- reduce the value sums: lanes with the same d chunk, then warps ----
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
  }
  // drain (bounded) the copies still in flight after an abort before the CTA exits
  __syncthreads();
  if (threadIdx.x == 0 && s_abort)
    for (int i = 0; i < kRing; ++i) {
      for (uint32_t it = 0; it < (1u << 20); ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(att_smem_u32(&full_bar[i])), "r"(0u)
            : "memory");
        if (ok) break;
      }
    }
}

template <int LPK, int RB>
static cudaError_t launch_dec_rb(const AttnArgs& a, size_t smem, cudaStream_t st) {
  const int groups = (a.H / a.Hkv + RB - 1) / RB;
  const cudaError_t e = launch_k(k_attention_decode<LPK, RB>, dim3(a.B, a.Hkv, groups), dim3(kDecThreads), smem, st, a.q, a.kc,
                                 a.vc, a.out, a.H, a.Hkv, a.max_seq, a.d_pos, a.Ms, a.Ss, a.Mo, a.So, a.prob_bits,
                                 a.luts, a.err);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// heads per CTA (and per value pass): dec_heads_per_cta
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
  if (a.M == 1 && (a.D == 16 || a.D == 32 || a.D == 64 || a.D == 128 || a.D == 256))
    return launch_attention_decode(a, st);
  const size_t smem = attention_smem_bytes(a.H, a.Hkv, a.D, a.max_seq);
  dim3 grid(R, a.Hkv);
  { const cudaError_t e_ = launch_k(k_attention, dim3(grid), dim3(256), smem, st, a.q, a.kc, a.vc, a.out, a.M, a.H, a.Hkv, a.D, a.max_seq, a.d_pos, a.Ms, a.Ss,
                                        a.Mo, a.So, a.prob_bits, a.luts); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

}  // namespace llx
