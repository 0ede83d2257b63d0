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
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

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

__global__ void k_attention(const int8_t* q, const int8_t* kc, const int8_t* vc,
                            int8_t* out, int M, int H, int Hkv, int D, int max_seq,
                            const int* d_pos, int64_t Ms, int Ss, int64_t Mo, int So, int prob_bits,
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
// Decode attention (one query row per sequence), split over a thread-block cluster.
//
// The C CTAs of a cluster share one (sequence, KV head, group of up to RB query heads) and
// take disjoint slices of the T = pos + 1 keys.  Each CTA streams its K slice, then its V
// slice, through a ring of shared-memory stages filled by 1-D bulk copies.  The reference's
// global order is kept exactly with three exchanges over distributed shared memory:
//   1. per-head score maxima of every slice -> the global max (integer max);
//   2. per-head exp-LUT sums of every slice -> the global sum -> inv = 2^31 / sum;
//   3. per-head partial value sums sum_t pn_t * v_t of every slice -> the total
//      (integer sums, exact in any order); each CTA finishes 1/C of the outputs.
// Splitting the keys shortens every CTA's serial chain (load -> scores -> max -> exp ->
// normalise -> values) by C and spreads a layer's KV stream over C times more CTAs.
// ---------------------------------------------------------------------------------------
constexpr int kDecThreads = 256, kDecWarps = kDecThreads / 32;

// KV tiles of 8 KB (D <= 64) or 16 KB (D >= 128) stream through a ring of dec_ring(D) stages;
// at D >= 128 a tile has kDecThreads / dec_tpk(D) keys and dec_tpk(D) threads share a key.
// At head dim 128 two stages of 16 KB measured best: shared memory then holds more CTAs per
// SM, which overlap one another's phases (C4 decode attention 128.7 -> 111.9 us per layer
// against three stages; C5 unchanged; four stages held only 2 CTAs per SM and lost).  Head
// dims up to 64 keep three stages of 8 KB.
constexpr int kRingMax = 3;
__host__ __device__ constexpr int dec_ring(int D) { return D >= 128 ? 2 : 3; }
__host__ __device__ constexpr int dec_tile_keys(int D) { return (D >= 128 ? 16384 : 8192) / D; }
__host__ __device__ constexpr int dec_tpk(int D) { return D >= 128 ? kDecThreads / dec_tile_keys(D) : 1; }

// query heads per CTA: a KV head's H/Hkv query heads in groups of at most 8
__host__ __device__ constexpr int dec_heads_per_cta(int rep) { return rep < 8 ? rep : 8; }

// keys per CTA slice (capacity) for cluster size C: ceil(max_seq / C) + a zero pad entry
__host__ __device__ constexpr int dec_slice_cap(int max_seq, int C) { return ((max_seq + C - 1) / C + 2) & ~1; }

// CTAs of RB query heads at head dim D run the score and value passes on int8 tensor-core
// tiles (mma m16n8k32, 8 head columns): with 4 or more heads per CTA; at 1 or 2 heads most
// of the tile is padding and the CUDA-core passes are faster (measured at head dim 128)
__host__ __device__ constexpr bool dec_tc(int D, int RB) { return (D == 64 || D == 128) && RB >= 4; }
// row stride (bytes) of the hi / lo probability planes of the tensor-core value pass: whole
// tiles of the largest slice plus 16 bytes, so the 8 head rows of a fragment load fall in
// different banks
__host__ __device__ constexpr int dec_prow(int max_seq, int C, int TK) {
  return ((max_seq + C - 1) / C + TK - 1) / TK * TK + 16;
}
// Head dim 128 with the tensor-core passes (the 64-register instantiation) packs its shared
// memory: the hi / lo probability bytes of each head go into that head's own score slots
// (16-key groups of 16 hi then 16 lo bytes: key t near byte 2t, so written after the chunk's
// scores are read they only cover slots already consumed), and the value pass's output
// partials reuse the ring once the last value tile is consumed.
__host__ __device__ constexpr bool dec_packed(int D, int RB) { return D == 128 && RB >= 4; }
// int32 slots per head of the score array: the slice capacity, or (packed) at least the
// probability bytes of the slice's whole tiles
__host__ __device__ constexpr int dec_sstride(int max_seq, int C, int D, int RB) {
  return dec_packed(D, RB) && ((max_seq + C - 1) / C + dec_tile_keys(D) - 1) / dec_tile_keys(D) * dec_tile_keys(D) / 2 >
                                  dec_slice_cap(max_seq, C)
             ? (((max_seq + C - 1) / C + dec_tile_keys(D) - 1) / dec_tile_keys(D) * dec_tile_keys(D) / 2 + 1) & ~1
             : dec_slice_cap(max_seq, C);
}

// bytes of the probability region: the hi / lo u8 planes of the tensor-core value pass (the
// CUDA-core value pass keeps normalised p in the score array, one int32 slot per key; the
// packed layout keeps the planes there too)
static size_t dec_p_bytes(int RB, int D, int max_seq, int C) {
  return dec_tc(D, RB) && !dec_packed(D, RB) ? (size_t)2 * RB * dec_prow(max_seq, C, dec_tile_keys(D)) : 0;
}

static size_t dec_smem_bytes(int RB, int D, int max_seq, int C) {
  const size_t ss = (size_t)dec_sstride(max_seq, C, D, RB);
  return (size_t)dec_ring(D) * dec_tile_keys(D) * D + (size_t)RB * D + (size_t)RB * ss * 4 + dec_p_bytes(RB, D, max_seq, C) +
         (dec_packed(D, RB) ? 0 : (size_t)RB * D * 4) + (size_t)kDecWarps * RB * 4 + (size_t)2 * RB * 4 + 128;
}

static int dec_rb(int rep) {
  const int h = dec_heads_per_cta(rep);
  return h <= 1 ? 1 : h <= 2 ? 2 : h <= 4 ? 4 : 8;
}


// one CTA per unit (cluster size 1) holds the scores of the whole context: allowed while its
// shared memory fits the per-CTA limit
constexpr size_t kDecSmemLimit = 227 * 1024;
static bool dec_c1_fits(int RB, int D, int max_seq) { return dec_smem_bytes(RB, D, max_seq, 1) <= kDecSmemLimit; }

// largest dynamic shared memory any decode launch of this geometry uses (cluster size 1 when
// it fits, else 2)
size_t attention_decode_smem_bytes(int H, int Hkv, int D, int max_seq) {
  const int RB = dec_rb(H / Hkv);
  return dec_c1_fits(RB, D, max_seq) ? dec_smem_bytes(RB, D, max_seq, 1) : dec_smem_bytes(RB, D, max_seq, 2);
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
// gap_prob for Ss >= 33: z = rshr(d * Ms, Ss) from the high word of the product alone,
// z = (hi + 2^(Ss-33)) >> (Ss-32): the rounding constant leaves the low word untouched and
// the low word adds a fraction below one, which cannot change the floor.  d < 2^23 and
// Ms < 2^32 keep hi below 2^23.  rnd = 2^(Ss-33), sh = Ss - 32.
__device__ __forceinline__ uint32_t gap_prob_hi(uint32_t d, uint32_t Ms, uint32_t rnd, int sh, const uint16_t* expi,
                                                const uint16_t* expf) {
  const uint32_t z = (__umulhi(d, Ms) + rnd) >> sh;
  if (z >= 4096u) return 0;
  return ((uint32_t)expi[z >> 8] * (uint32_t)expf[z & 255] + (1u << 15)) >> 16;
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

__device__ __forceinline__ uint32_t dec_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void dec_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 32-bit word of cluster peer `rank`'s shared memory at the address of `local` in this CTA
__device__ __forceinline__ uint32_t dec_peer_u32(const void* local, uint32_t rank) {
  uint32_t remote, v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(att_smem_u32(local)), "r"(rank));
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(remote) : "memory");
  return v;
}

// d += a (16x32, s8) x b (32x8, s8, or u8 when B_U8): one m16n8k32 integer tensor-core tile
template <bool B_U8>
__device__ __forceinline__ void dec_mma(int32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  if (B_U8)
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// 4 x 4 byte transpose: x_e holds channels 0..3 of key e; w[q] gets channel q of keys 0..3
__device__ __forceinline__ void dec_transpose4(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3, uint32_t* w) {
  const uint32_t t0 = __byte_perm(x0, x1, 0x5140), t1 = __byte_perm(x0, x1, 0x7362);
  const uint32_t t2 = __byte_perm(x2, x3, 0x5140), t3 = __byte_perm(x2, x3, 0x7362);
  w[0] = __byte_perm(t0, t2, 0x5410);
  w[1] = __byte_perm(t0, t2, 0x7632);
  w[2] = __byte_perm(t1, t3, 0x5410);
  w[3] = __byte_perm(t1, t3, 0x7632);
}

template <int LPK, int RB>
__device__ __forceinline__ void attention_decode_body(
    const int8_t* q, const int8_t* kc, const int8_t* vc, int8_t* out,
    int H, int Hkv, int max_seq, const int* d_pos, int64_t Ms, int Ss, int64_t Mo, int So, int prob_bits,
    const uint16_t* __restrict__ luts, int32_t* err, int C, const AttnArgs rope) {
  constexpr int D = LPK * 16;
  constexpr int TK = dec_tile_keys(D);
  constexpr int TPK = dec_tpk(D);
  static_assert(TPK == 1 || TK * TPK == kDecThreads, "one key per TPK threads");
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint16_t s_expi[16], s_expf[256];
  constexpr int kRing = dec_ring(D);
  __shared__ __align__(8) uint64_t full_bar[kRingMax];
  __shared__ int s_abort;
  __shared__ int32_t s_gmax[RB];
  __shared__ uint32_t s_inv[RB];
  __shared__ __align__(16) int8_t s_knew[D], s_vnew[D];  // the newest key / value row (folded RoPE)
  const int rep_all = H / Hkv;
  const int hg0 = blockIdx.z * RB;
  const int rep = min(RB, rep_all - hg0);
  const int cap = dec_slice_cap(max_seq, C);
  constexpr bool PACKED = dec_packed(D, RB);
  const int ss = dec_sstride(max_seq, C, D, RB);  // int32 slots per head of the score array
  int8_t* ring = reinterpret_cast<int8_t*>(smem);                        // [kRing][TK][D]
  int8_t* q_s = ring + (size_t)kRing * TK * D;                           // [RB][D]
  // [RB][ss] scores, then p, then normalised p: each key in its slot (CUDA-core value pass),
  // or as hi / lo bytes over the head's slots (packed)
  int32_t* sc = reinterpret_cast<int32_t*>(q_s + RB * D);
  // tensor-core value pass, unpacked: normalised p as hi / lo u8 planes [RB][prow]
  constexpr bool TC = dec_tc(D, RB);
  const int prow = dec_prow(max_seq, C, TK);
  uint8_t* p_hi = reinterpret_cast<uint8_t*>(sc + (size_t)RB * ss);
  uint8_t* p_lo = p_hi + (size_t)RB * prow;
  // [RB][D] value partials: in the ring once it is free (packed), else after the planes;
  // the exchange scratch below is live while value tiles land, so it never sits in the ring
  int32_t* tail = reinterpret_cast<int32_t*>(p_hi + (TC && !PACKED ? (size_t)2 * RB * prow : 0));
  int32_t* opart = PACKED ? reinterpret_cast<int32_t*>(ring) : tail;
  int32_t* wred = PACKED ? tail : tail + RB * D;                         // [warps][RB]
  int32_t* xmax = wred + kDecWarps * RB;                                 // [RB] slice maxima (read by peers)
  uint32_t* xsum = reinterpret_cast<uint32_t*>(xmax + RB);               // [RB] slice sums (read by peers)
  const uint32_t crank = dec_cluster_rank();
  const int b = blockIdx.x / C, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
  // POS is written before the launch's first kernel (host copy, or the previous replay's
  // finalize step), so it is stable here.  The cached keys and values below position pos
  // were written by earlier launches: their first tiles are requested before the grid
  // dependency wait, overlapping the previous kernel.  The tile holding position pos, which
  // this launch's RoPE step writes, is requested after the wait.
  const int T = *d_pos + 1;
  const int chunk = (T + C - 1) / C;
  const int k0 = min(T, (int)crank * chunk), k1 = min(T, k0 + chunk);
  const int nkeys = k1 - k0;
  const int ntile = (nkeys + TK - 1) / TK;  // tiles of K, then as many of V
  const int8_t* kbase = kc + ((int64_t)b * Hkv + kvh) * max_seq * D;
  const int8_t* vbase = vc + ((int64_t)b * Hkv + kvh) * max_seq * D;
  auto issue = [&](int i) {  // tile i of the K-then-V sequence into stage i % kRing
    const int kv = i >= ntile, ti = kv ? i - ntile : i;
    const int t0 = k0 + ti * TK, nk = min(TK, k1 - t0);
    att_bulk_load(ring + (size_t)(i % kRing) * TK * D, (kv ? vbase : kbase) + (int64_t)t0 * D, (uint32_t)(nk * D),
                  &full_bar[i % kRing]);
  };
  auto fresh = [&](int i) {  // tile i holds position pos = T - 1
    const int ti = i >= ntile ? i - ntile : i;
    return ti == ntile - 1 && k1 == T;
  };
  // with the RoPE group folded in, the tile holding pos is patched after it lands
  const bool folded = rope.rq16 != nullptr;
  const bool owner = folded && nkeys > 0 && k1 == T;  // this slice holds position pos
  __syncthreads();
  if (threadIdx.x == 0)
    for (int i = 0; i < min(kRing, 2 * ntile); ++i)
      if (folded || !fresh(i)) issue(i);
  pdl_wait();  // q and the newest K/V row come from earlier kernels
  if (threadIdx.x == 0 && !folded)
    for (int i = 0; i < min(kRing, 2 * ntile); ++i)
      if (fresh(i)) issue(i);
  if (folded) {
    // rotate + quantize this CTA's query heads; the slice owner also rotates the newest key
    // and writes the newest K / V rows to the caches (one head group writes them)
    const int half = D / 2, pos = T - 1;
    const int16_t* ct = rope.cos_tab + (int64_t)pos * half;
    const int16_t* stb = rope.sin_tab + (int64_t)pos * half;
    for (int idx = threadIdx.x; idx < (rep + 1) * half; idx += blockDim.x) {
      const int r = idx / half, i = idx % half;
      if (r == rep && !owner) break;
      const int16_t* x = r < rep ? rope.rq16 + ((int64_t)b * H + (int64_t)kvh * rep_all + hg0 + r) * D
                                 : rope.rk16 + ((int64_t)b * Hkv + kvh) * D;
      const int64_t x1 = x[i], x2 = x[i + half], c = ct[i], sn = stb[i];
      const int64_t ya = sat16(rshr(x1 * c - x2 * sn, 14));
      const int64_t yb = sat16(rshr(x2 * c + x1 * sn, 14));
      const int64_t M = r < rep ? rope.q_M : rope.k_M;
      const int S = r < rep ? rope.q_S : rope.k_S;
      int8_t* dst = r < rep ? q_s + r * D : s_knew;
      dst[i] = (int8_t)sat8(mulshift(ya, M, S));
      dst[i + half] = (int8_t)sat8(mulshift(yb, M, S));
    }
    if (owner)
      for (int i = threadIdx.x; i < D; i += blockDim.x) s_vnew[i] = rope.rv8[((int64_t)b * Hkv + kvh) * D + i];
    __syncthreads();
    if (owner && blockIdx.z == 0)
      for (int i = threadIdx.x; i < D; i += blockDim.x) {
        const int64_t o = (((int64_t)b * Hkv + kvh) * max_seq + pos) * D + i;
        rope.kc_out[o] = s_knew[i];
        rope.vc_out[o] = s_vnew[i];
      }
  } else {
    const int8_t* qrow = q + ((int64_t)b * H + (int64_t)kvh * rep_all + hg0) * D;
    for (int i = threadIdx.x; i < rep * D / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(q_s)[i] = reinterpret_cast<const uint4*>(qrow)[i];
  }
  // the newest row of a landed tile is stale cache content under the folded RoPE: replace it
  auto patch = [&](int i) {
    if (!owner || !fresh(i)) return;
    int8_t* tile = ring + (size_t)(i % kRing) * TK * D;
    const int ti = i >= ntile ? i - ntile : i;
    int8_t* row = tile + (size_t)(T - 1 - (k0 + ti * TK)) * D;
    const int8_t* src = i >= ntile ? s_vnew : s_knew;
    for (int c = threadIdx.x; c < D / 16; c += blockDim.x)
      reinterpret_cast<uint4*>(row)[c] = reinterpret_cast<const uint4*>(src)[c];
    __syncthreads();
  };
  // one thread polls the stage's barrier; the others wait at the CTA barrier, which issues
  // nothing (a CTA-wide poll would take issue slots from the CTAs sharing the SM)
  auto wait_stage = [&](int i) {
    if (threadIdx.x == 0 && s_abort == 0 && !att_mbar_wait(&full_bar[i % kRing], (uint32_t)((i / kRing) & 1))) {
      s_abort = 1;
      if (err) atomicExch(err, 5);
    }
    __syncthreads();
    return s_abort == 0;
  };

  // ---- K slice: one key per lane, scores of every head, running per-head maxima ----
  int32_t mxl[RB];
#pragma unroll
  for (int j = 0; j < RB; ++j) mxl[j] = INT_MIN;
  // tensor-core score pass: S^T (16 keys x 8 heads) = K (16 x 32 channels) Q^T per MMA.  The
  // MMA's k index 4 tig + e (e < 4) is channel 8 tig + e of the 32-channel block and k index
  // 16 + 4 tig + e is channel 8 tig + 4 + e, so a thread's A and B operands of one block are
  // one 8-byte load each.  Thread (g, tig) keeps Q^T columns of head g; its results are the
  // scores of heads 2 tig and 2 tig + 1 (running maxima mxa, mxb).
  const int g = lane >> 2, tig = lane & 3, h0 = 2 * tig, h1 = 2 * tig + 1;
  int32_t mxa = INT_MIN, mxb = INT_MIN;
  uint2 qf[TC ? D / 32 : 1];
  if constexpr (TC) {
    __syncthreads();  // q_s complete
#pragma unroll
    for (int kb = 0; kb < D / 32; ++kb)
      qf[kb] = g < rep ? *reinterpret_cast<const uint2*>(q_s + g * D + kb * 32 + 8 * tig) : make_uint2(0u, 0u);
  }
  for (int i = 0; i < ntile; ++i) {
    if (!wait_stage(i)) break;
    patch(i);
    const int8_t* tile = ring + (size_t)(i % kRing) * TK * D;
    const int lt0 = i * TK, nk = min(TK, nkeys - lt0);
    if constexpr (TC) {
      static_assert(TK / 16 == kDecWarps, "one 16-key block per warp and tile");
      const int r = warp * 16 + g;  // tile rows r and r + 8 (rows past nk are stale, never stored)
      if (warp * 16 < nk) {
        const int8_t* r0 = tile + (size_t)r * D + 8 * tig;
        const int8_t* r1 = r0 + 8 * D;
        int32_t c[4] = {0, 0, 0, 0};
#pragma unroll
        for (int kb = 0; kb < D / 32; ++kb) {
          const uint2 x0 = *reinterpret_cast<const uint2*>(r0 + kb * 32);
          const uint2 x1 = *reinterpret_cast<const uint2*>(r1 + kb * 32);
          dec_mma<false>(c, x0.x, x1.x, x0.y, x1.y, qf[kb].x, qf[kb].y);
        }
        if (r < nk) {
          if (h0 < rep) {
            sc[h0 * ss + lt0 + r] = c[0];
            mxa = max(mxa, c[0]);
          }
          if (h1 < rep) {
            sc[h1 * ss + lt0 + r] = c[1];
            mxb = max(mxb, c[1]);
          }
        }
        if (r + 8 < nk) {
          if (h0 < rep) {
            sc[h0 * ss + lt0 + r + 8] = c[2];
            mxa = max(mxa, c[2]);
          }
          if (h1 < rep) {
            sc[h1 * ss + lt0 + r + 8] = c[3];
            mxb = max(mxb, c[3]);
          }
        }
      }
    } else if (TPK == 1) {
      for (int l = threadIdx.x; l < nk; l += kDecThreads) {
        const int8_t* krow = tile + (size_t)l * D;
        int sv[RB];
#pragma unroll
        for (int r = 0; r < RB; ++r) sv[r] = 0;
#pragma unroll
        for (int cc = 0; cc < LPK; ++cc) {
          // rotate the starting chunk by key so a warp's 32 rows spread over the banks
          const int c = (cc + l) % LPK;
          const uint4 kk = reinterpret_cast<const uint4*>(krow)[c];
#pragma unroll
          for (int r = 0; r < RB; ++r)
            if (r < rep) sv[r] = dot16_i8(kk, reinterpret_cast<const uint4*>(q_s + r * D)[c], sv[r]);
        }
#pragma unroll
        for (int r = 0; r < RB; ++r)
          if (r < rep) {
            mxl[r] = max(mxl[r], sv[r]);
            sc[r * ss + lt0 + l] = sv[r];
          }
      }
    } else {
      // TPK threads per key, each LPK / TPK 16-byte chunks; the tile has exactly one key per
      // TPK threads, so every thread takes part in the pair / quad reduction
      constexpr int CPT = LPK / TPK;
      const int l = threadIdx.x / TPK, sub = threadIdx.x % TPK;
      const bool valid = l < nk;
      const int8_t* krow = tile + (size_t)l * D;
      int sv[RB];
#pragma unroll
      for (int r = 0; r < RB; ++r) sv[r] = 0;
      if (valid) {
#pragma unroll
        for (int cc = 0; cc < CPT; ++cc) {
          const int c = sub * CPT + (cc + l) % CPT;
          const uint4 kk = reinterpret_cast<const uint4*>(krow)[c];
#pragma unroll
          for (int r = 0; r < RB; ++r)
            if (r < rep) sv[r] = dot16_i8(kk, reinterpret_cast<const uint4*>(q_s + r * D)[c], sv[r]);
        }
      }
#pragma unroll
      for (int o = 1; o < TPK; o <<= 1)
#pragma unroll
        for (int r = 0; r < RB; ++r) sv[r] += __shfl_xor_sync(0xffffffffu, sv[r], o);
      if (valid && sub == 0) {
#pragma unroll
        for (int r = 0; r < RB; ++r)
          if (r < rep) {
            mxl[r] = max(mxl[r], sv[r]);
            sc[r * ss + lt0 + l] = sv[r];
          }
      }
    }
    __syncthreads();  // stage consumed by every thread
    if (threadIdx.x == 0 && i + kRing < 2 * ntile) issue(i + kRing);
  }
  // ---- exchange 1: slice maxima -> global per-head max ----
  if constexpr (TC) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mxa = max(mxa, __shfl_xor_sync(0xffffffffu, mxa, o));
      mxb = max(mxb, __shfl_xor_sync(0xffffffffu, mxb, o));
    }
    if (g == 0) {
      if (h0 < RB) wred[warp * RB + h0] = mxa;
      if (h1 < RB) wred[warp * RB + h1] = mxb;
    }
  } else {
#pragma unroll
    for (int j = 0; j < RB; ++j) {
      int32_t v = mxl[j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) wred[warp * RB + j] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x < RB) {
    int32_t v = INT_MIN;
    for (int w = 0; w < kDecWarps; ++w) v = max(v, wred[w * RB + threadIdx.x]);
    xmax[threadIdx.x] = v;
  }
  dec_cluster_sync();
  if (threadIdx.x < C * RB) {
    // thread r * RB + j reads peer r's maximum of head j; the C reads run concurrently
    const int j = threadIdx.x % RB, r = threadIdx.x / RB;
    wred[threadIdx.x] = (int32_t)dec_peer_u32(xmax + j, (uint32_t)r);
  }
  __syncthreads();
  if (threadIdx.x < rep) {
    int32_t v = INT_MIN;
    for (int r = 0; r < C; ++r) v = max(v, wred[r * RB + threadIdx.x]);
    s_gmax[threadIdx.x] = v;
  }
  __syncthreads();
  // ---- exp-LUT probabilities of the slice, slice sums ----
  const bool live = s_abort == 0;
  {
    int32_t mx[RB];
    uint32_t sum[RB];
#pragma unroll
    for (int j = 0; j < RB; ++j) {
      mx[j] = j < rep ? s_gmax[j] : 0;
      sum[j] = 0;
    }
    // the exp-LUT gap: for Ss >= 33 from the product's high word (gap_prob_hi), chosen once
    // for the whole pass so the unrolled loop stays branch-free
    auto exp_pass = [&](auto fast) {
      constexpr bool FAST = decltype(fast)::value;
      const uint32_t rnd = FAST ? 1u << (Ss - 33) : 0u;
      const int zsh = FAST ? Ss - 32 : 0;
      for (int t = threadIdx.x; t < nkeys; t += kDecThreads) {
#pragma unroll
        for (int j = 0; j < RB; ++j) {
          if (j < rep) {
            const uint32_t d = (uint32_t)(mx[j] - sc[j * ss + t]);
            const uint32_t pr = FAST ? gap_prob_hi(d, (uint32_t)Ms, rnd, zsh, s_expi, s_expf)
                                     : gap_prob(d, (uint32_t)Ms, Ss, s_expi, s_expf);
            sc[j * ss + t] = (int32_t)pr;
            sum[j] += pr;
          }
        }
      }
    };
    if (live) {
      if (Ss >= 33)
        exp_pass(std::true_type{});
      else
        exp_pass(std::false_type{});
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int j = 0; j < RB; ++j) sum[j] += __shfl_xor_sync(0xffffffffu, sum[j], o);
    if (lane == 0)
#pragma unroll
      for (int j = 0; j < RB; ++j) wred[warp * RB + j] = (int32_t)sum[j];
  }
  __syncthreads();
  if (threadIdx.x < RB) {
    uint32_t v = 0;
    if (threadIdx.x < rep)
      for (int w = 0; w < kDecWarps; ++w) v += (uint32_t)wred[w * RB + threadIdx.x];
    xsum[threadIdx.x] = v;
  }
  // ---- exchange 2: slice sums -> global sum -> inv = 2^31 / sum (32-bit divide, exact) ----
  dec_cluster_sync();
  if (threadIdx.x < C * RB) {
    const int j = threadIdx.x % RB, r = threadIdx.x / RB;
    wred[threadIdx.x] = (int32_t)dec_peer_u32(xsum + j, (uint32_t)r);
  }
  __syncthreads();
  if (threadIdx.x < rep) {
    uint32_t v = 0;
    for (int r = 0; r < C; ++r) v += (uint32_t)wred[r * RB + threadIdx.x];
    s_inv[threadIdx.x] = 0x80000000u / (v ? v : 1u);
  }
  __syncthreads();
  // ---- normalised probabilities: pn = min(pmax, rshr(p * inv, 31 - prob_bits)) ----
  // p <= sum, so p * inv <= 2^31: the product and its rounding shift stay in 32 bits
  const uint32_t pmax = (1u << prob_bits) - 1u;
  const int pshift = 31 - prob_bits;
  if constexpr (PACKED) {
    // hi / lo bytes of pn over whole tiles (0 past the slice), in the head's own score slots:
    // 16-key group G at bytes 32 G (hi) and 32 G + 16 (lo), key u of a group at 4 (u % 4) +
    // u / 4 as below.  Chunks of 512 keys: every thread reads its keys of the chunk, and after
    // the barrier writes bytes < 2 (chunk end), i.e. slots below chunk end / 2, which belong
    // to this chunk or earlier ones and have been read; later chunks' slots are untouched.
    const int nfill = ntile * TK;
    for (int c0 = 0; c0 < nfill; c0 += 2 * kDecThreads) {
      uint32_t v[RB][2];
#pragma unroll
      for (int j = 0; j < RB; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = c0 + threadIdx.x + e * kDecThreads;
          v[j][e] = 0;
          if (j < rep && t < nkeys && live) {
            const uint32_t x = (uint32_t)sc[j * ss + t] * s_inv[j];
            const uint32_t pn = (x >> pshift) + ((x >> (pshift - 1)) & 1u);
            v[j][e] = pn < pmax ? pn : pmax;
          }
        }
      __syncthreads();
#pragma unroll
      for (int j = 0; j < RB; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = c0 + threadIdx.x + e * kDecThreads;
          if (j < rep && t < nfill) {
            const int u = t & 15;
            uint8_t* at = reinterpret_cast<uint8_t*>(sc + (size_t)j * ss) + 32 * (t >> 4) + 4 * (u & 3) + (u >> 2);
            at[0] = (uint8_t)(v[j][e] >> 8);
            at[16] = (uint8_t)(v[j][e] & 255u);
          }
        }
    }
  } else if constexpr (TC) {
    // hi / lo bytes of pn (pn < 2^15) for the value MMAs, over whole tiles (0 past the
    // slice).  Within each 16-key half the value pass's MMA k index 4 tig + e stands for key
    // 4 e + tig, so key u of a half is stored at 4 (u % 4) + u / 4: a thread's 4 keys are
    // one 4-byte load.
    const int nfill = ntile * TK;
    for (int j = 0; j < rep; ++j) {
      const uint32_t inv = s_inv[j];
      const int32_t* sj = sc + j * ss;
      for (int t = threadIdx.x; t < nfill; t += kDecThreads) {
        uint32_t v = 0;
        if (t < nkeys && live) {
          const uint32_t x = (uint32_t)sj[t] * inv;
          const uint32_t pn = (x >> pshift) + ((x >> (pshift - 1)) & 1u);
          v = pn < pmax ? pn : pmax;
        }
        const int u = t & 15, at = j * prow + (t & ~15) + 4 * (u & 3) + (u >> 2);
        p_hi[at] = (uint8_t)(v >> 8);
        p_lo[at] = (uint8_t)(v & 255u);
      }
    }
  } else {
    // in place: each thread rewrites only the slots it reads
    for (int j = 0; j < rep; ++j) {
      const uint32_t inv = s_inv[j];
      int32_t* sj = sc + j * ss;
      for (int t = threadIdx.x; t < cap; t += kDecThreads) {
        uint32_t v = 0;
        if (t < nkeys && live) {
          const uint32_t x = (uint32_t)sj[t] * inv;
          const uint32_t pn = (x >> pshift) + ((x >> (pshift - 1)) & 1u);
          v = pn < pmax ? pn : pmax;
        }
        sj[t] = (int32_t)v;  // entries past the slice are 0: they weight the stale pair row
      }
    }
  }
  __syncthreads();
  if constexpr (TC) {
    // ---- tensor-core value pass: O^T (16 channels x 8 heads) += V^T (16 x 32 keys) P^T ----
    // Warp w takes the 32-key chunk w % 4 of every tile and half w / 4 of the channels.  In
    // its m-block m, row g stands for channel g D/8 + half D/16 + 2 m and row g + 8 for the
    // next channel, so thread (g, tig) reads D/16 contiguous bytes of each of its 8 key rows
    // (keys 4 e + tig and 16 + 4 e + tig of the chunk) and transposes them into the A
    // operand.  pn enters as two unsigned bytes, O = 256 (hi V) + (lo V), exact in int32;
    // the hi MMAs are skipped when pn has 8 bits.  The warps' sums meet in opart through
    // shared-memory atomic adds (integer: exact in any order).
    constexpr int CW = D / 16, MBH = D / 32;
    const int kc = warp & 3, half = warp >> 2;
    const bool wide = prob_bits > 8;
    if constexpr (!PACKED)
      for (int i = threadIdx.x; i < rep * D; i += kDecThreads) opart[i] = 0;
    int32_t ah[MBH][4], al[MBH][4];
#pragma unroll
    for (int m = 0; m < MBH; ++m)
#pragma unroll
      for (int k = 0; k < 4; ++k) ah[m][k] = al[m][k] = 0;
    for (int i = ntile; i < 2 * ntile; ++i) {
      if (!wait_stage(i)) break;
      patch(i);
      const int8_t* tile = ring + (size_t)(i % kRing) * TK * D;
      const int lt0 = (i - ntile) * TK, nk = min(TK, nkeys - lt0);
      if (kc * 32 < nk) {  // rows past nk are stale shared memory; their pn bytes are 0
        const int8_t* vrow = tile + (size_t)(kc * 32 + tig) * D + g * (D / 8) + half * CW;
        uint32_t wa[CW], wb[CW];
        if constexpr (CW == 8) {
          uint2 xa[4], xb[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            xa[e] = *reinterpret_cast<const uint2*>(vrow + (size_t)(4 * e) * D);
            xb[e] = *reinterpret_cast<const uint2*>(vrow + (size_t)(16 + 4 * e) * D);
          }
          dec_transpose4(xa[0].x, xa[1].x, xa[2].x, xa[3].x, wa);
          dec_transpose4(xa[0].y, xa[1].y, xa[2].y, xa[3].y, wa + 4);
          dec_transpose4(xb[0].x, xb[1].x, xb[2].x, xb[3].x, wb);
          dec_transpose4(xb[0].y, xb[1].y, xb[2].y, xb[3].y, wb + 4);
        } else {
          uint32_t xa[4], xb[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            xa[e] = *reinterpret_cast<const uint32_t*>(vrow + (size_t)(4 * e) * D);
            xb[e] = *reinterpret_cast<const uint32_t*>(vrow + (size_t)(16 + 4 * e) * D);
          }
          dec_transpose4(xa[0], xa[1], xa[2], xa[3], wa);
          dec_transpose4(xb[0], xb[1], xb[2], xb[3], wb);
        }
        uint32_t bl0 = 0, bl1 = 0, bh0 = 0, bh1 = 0;
        if (PACKED && g < rep) {
          // the chunk's two 16-key groups: hi, lo, hi, lo (16 bytes each)
          const uint8_t* pg = reinterpret_cast<const uint8_t*>(sc + (size_t)g * ss) + 2 * (lt0 + kc * 32) + 4 * tig;
          bl0 = *reinterpret_cast<const uint32_t*>(pg + 16);
          bl1 = *reinterpret_cast<const uint32_t*>(pg + 48);
          if (wide) {
            bh0 = *reinterpret_cast<const uint32_t*>(pg);
            bh1 = *reinterpret_cast<const uint32_t*>(pg + 32);
          }
        } else if (g < rep) {
          const int pb = g * prow + lt0 + kc * 32 + 4 * tig;
          bl0 = *reinterpret_cast<const uint32_t*>(p_lo + pb);
          bl1 = *reinterpret_cast<const uint32_t*>(p_lo + pb + 16);
          if (wide) {
            bh0 = *reinterpret_cast<const uint32_t*>(p_hi + pb);
            bh1 = *reinterpret_cast<const uint32_t*>(p_hi + pb + 16);
          }
        }
#pragma unroll
        for (int m = 0; m < MBH; ++m) {
          dec_mma<true>(al[m], wa[2 * m], wa[2 * m + 1], wb[2 * m], wb[2 * m + 1], bl0, bl1);
          if (wide) dec_mma<true>(ah[m], wa[2 * m], wa[2 * m + 1], wb[2 * m], wb[2 * m + 1], bh0, bh1);
        }
      }
      __syncthreads();  // stage consumed by every thread
      if (threadIdx.x == 0 && i + kRing < 2 * ntile) issue(i + kRing);
    }
    if constexpr (PACKED) {
      // the ring is free: every value tile has been consumed and none is in flight
      for (int i = threadIdx.x; i < rep * D; i += kDecThreads) opart[i] = 0;
    }
    __syncthreads();  // opart zeroed by every thread before any adds
#pragma unroll
    for (int m = 0; m < MBH; ++m) {
      const int ch = g * (D / 8) + half * CW + 2 * m;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int hd = 2 * tig + (k & 1), c = ch + (k >> 1);
        if (hd < rep) atomicAdd(&opart[hd * D + c], ah[m][k] * 256 + al[m][k]);
      }
    }
  } else {
    // ---- V slice: item = (key phase, unit u = (head j, 4 channels)) over key pairs ----
    // A long slice splits each unit's key pairs into KS phases (the phase is the slow index,
    // so a warp reads neighbouring channels of the same key rows); the phase sums meet in
    // opart through shared-memory atomic adds (integer: exact in any order).
    constexpr int D4 = D / 4;
    const int units = rep * D4;
    int KS = 1;
    if (nkeys > 512)
      while (KS < 8 && units * KS * 2 <= kDecThreads) KS *= 2;
    const int items = units * KS;
    if (KS > 1)
      for (int i = threadIdx.x; i < rep * D; i += kDecThreads) opart[i] = 0;
    int32_t acc[2][4];
  #pragma unroll
    for (int x = 0; x < 2; ++x)
  #pragma unroll
      for (int k = 0; k < 4; ++k) acc[x][k] = 0;
    for (int i = ntile; i < 2 * ntile; ++i) {
      if (!wait_stage(i)) break;
      patch(i);
      const int8_t* tile = ring + (size_t)(i % kRing) * TK * D;
      const int lt0 = (i - ntile) * TK, nk = min(TK, nkeys - lt0);
  #pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int it = threadIdx.x + x * kDecThreads;
        if (it >= items) break;
        const int ph = it / units, u = it % units;
        const int j = u / D4, c4 = (u % D4) * 4;
        const int32_t* pj = sc + (size_t)j * ss + lt0;  // normalised p (< 2^15) per key
        // key pairs l, l + 1 with a compile-time stride per phase count
        auto pairs = [&](auto ks) {
          constexpr int KSC = decltype(ks)::value;
          for (int l = 2 * ph; l < nk; l += 2 * KSC) {
            // the row after the last key may be stale shared memory: its pn is 0
            const uint32_t va = *reinterpret_cast<const uint32_t*>(tile + (size_t)l * D + c4);
            const uint32_t vb = *reinterpret_cast<const uint32_t*>(tile + (size_t)(l + 1) * D + c4);
            // pn of keys l, l + 1 as the two 16-bit halves (l even, cap even: 8-byte aligned)
            const uint2 p2 = *reinterpret_cast<const uint2*>(pj + l);
            const int pp = (int)__byte_perm(p2.x, p2.y, 0x5410);
            const uint32_t lo = __byte_perm(va, vb, 0x5140), hi = __byte_perm(va, vb, 0x7362);
            acc[x][0] = __dp2a_lo(pp, (int)lo, acc[x][0]);
            acc[x][1] = __dp2a_hi(pp, (int)lo, acc[x][1]);
            acc[x][2] = __dp2a_lo(pp, (int)hi, acc[x][2]);
            acc[x][3] = __dp2a_hi(pp, (int)hi, acc[x][3]);
          }
        };
        switch (KS) {
          case 1: pairs(std::integral_constant<int, 1>{}); break;
          case 2: pairs(std::integral_constant<int, 2>{}); break;
          case 4: pairs(std::integral_constant<int, 4>{}); break;
          default: pairs(std::integral_constant<int, 8>{}); break;
        }
      }
      __syncthreads();  // stage consumed by every thread
      if (threadIdx.x == 0 && i + kRing < 2 * ntile) issue(i + kRing);
    }
    if (KS > 1) __syncthreads();  // opart zeroed by every thread before any adds
  #pragma unroll
    for (int x = 0; x < 2; ++x) {
      const int it = threadIdx.x + x * kDecThreads;
      if (it < items) {
        const int u = it % units;
  #pragma unroll
        for (int k = 0; k < 4; ++k) {
          int32_t* dst = &opart[(u / D4) * D + (u % D4) * 4 + k];
          if (KS > 1)
            atomicAdd(dst, acc[x][k]);
          else
            *dst = acc[x][k];
        }
      }
    }
  }
  // ---- exchange 3: slice value sums -> outputs; CTA `crank` finishes outputs idx = crank mod C ----
  dec_cluster_sync();
  if (s_abort == 0) {
    int8_t* orow = out + ((int64_t)b * H + (int64_t)kvh * rep_all + hg0) * D;
    for (int idx = (int)crank + C * threadIdx.x; idx < rep * D; idx += C * kDecThreads) {
      int32_t o = 0;
      for (int r = 0; r < C; ++r) o += (int32_t)dec_peer_u32(opart + idx, (uint32_t)r);
      int64_t ov = o;
      if (prob_bits == 15) ov = rshr(ov, 7);
      orow[idx] = (int8_t)sat8(mulshift(ov, Mo, So));
    }
  }
  dec_cluster_sync();  // peers keep their shared memory until every CTA has read it
  // drain (bounded) the copies still in flight after an abort before the CTA exits
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

// The kernel, in two register budgets.  Head dim 128 with the tensor-core passes (4+ heads
// per CTA) is held to 64 registers, which its slice state fits without spilling: 4 CTAs of
// two 16 KB ring stages then share an SM instead of 3 (shared memory allows 4 up to max_seq
// ~1500 at 4 heads).  The others keep the compiler's own allocation (an explicit minimum of
// one CTA per SM would loosen it).
#define LLX_DEC_PARAMS                                                                                         \
  const int8_t *q, const int8_t *kc, const int8_t *vc, int8_t *out, int H, int Hkv, int max_seq, const int *d_pos, \
      int64_t Ms, int Ss, int64_t Mo, int So, int prob_bits, const uint16_t *__restrict__ luts, int32_t *err, int C, \
      const AttnArgs rope
#define LLX_DEC_ARGS q, kc, vc, out, H, Hkv, max_seq, d_pos, Ms, Ss, Mo, So, prob_bits, luts, err, C, rope
template <int LPK, int RB>
__global__ void __launch_bounds__(kDecThreads) k_attention_decode(LLX_DEC_PARAMS) {
  attention_decode_body<LPK, RB>(LLX_DEC_ARGS);
}
template <int LPK, int RB>
__global__ void __launch_bounds__(kDecThreads, 4) k_attention_decode_r64(LLX_DEC_PARAMS) {
  attention_decode_body<LPK, RB>(LLX_DEC_ARGS);
}
#undef LLX_DEC_PARAMS
#undef LLX_DEC_ARGS
using DecKernel = void (*)(const int8_t*, const int8_t*, const int8_t*, int8_t*, int, int, int, const int*, int64_t,
                           int, int64_t, int, int, const uint16_t*, int32_t*, int, const AttnArgs);
template <int LPK, int RB>
static DecKernel dec_kernel() {
  if constexpr (LPK == 8 && RB >= 4)
    return k_attention_decode_r64<LPK, RB>;
  else
    return k_attention_decode<LPK, RB>;
}

// Resident clusters per cluster size, measured with the occupancy API at model load
// (outside any stream capture) for each decode geometry: key (LPK, RB, max_seq, C).
static std::mutex g_occ_mu;
static std::map<std::tuple<int, int, int, int>, int> g_occ;

template <int LPK, int RB>
static cudaError_t measure_dec_occupancy(int max_seq) {
  for (int C = 1; C <= 8; C *= 2) {
    if (C == 1 && !dec_c1_fits(RB, LPK * 16, max_seq)) continue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C * 148, 1, 1);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = dec_smem_bytes(RB, LPK * 16, max_seq, C);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, dec_kernel<LPK, RB>(), &cfg);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_occ_mu);
    g_occ[std::make_tuple(LPK, RB, max_seq, C)] = clusters;
  }
  return cudaSuccess;
}

// Cluster size: the largest C in {8, 4, 2} whose B * Hkv * groups clusters are all resident
// at once (one wave: the slowest slice bounds the launch).  When no split fits in one wave
// but one CTA per unit does, C = 1: every max / sum / output exchange is then a CTA barrier
// instead of a cluster round trip.  Beyond one wave: C = 1 again once one CTA per unit needs
// 3 or more waves (the last wave's tail then costs less than the cluster exchanges: C5 at
// 256 sequences, 2048 units over 444 resident CTAs, 158.6 against 177.7 us per layer), else
// 2 (C4 at 64 sequences, 1.7 waves: 107.3 against 115.5 us with C = 1).
template <int LPK, int RB>
static int dec_cluster_size(int units, int max_seq) {
  std::lock_guard<std::mutex> lock(g_occ_mu);
  for (int C = 8; C >= 1; C /= 2) {
    auto it = g_occ.find(std::make_tuple(LPK, RB, max_seq, C));
    if (it != g_occ.end() && it->second >= units) return C;
  }
  auto c1 = g_occ.find(std::make_tuple(LPK, RB, max_seq, 1));
  if (c1 != g_occ.end() && c1->second > 0 && units >= 3 * c1->second) return 1;
  return 2;
}

template <int LPK, int RB>
static cudaError_t launch_dec_rb(const AttnArgs& a, cudaStream_t st) {
  const int groups = (a.H / a.Hkv + RB - 1) / RB;
  const int C = dec_cluster_size<LPK, RB>(a.B * a.Hkv * groups, a.max_seq);
  const size_t smem = dec_smem_bytes(RB, LPK * 16, a.max_seq, C);
  const cudaError_t e = launch_kc(dec_kernel<LPK, RB>(), dim3(a.B * C, a.Hkv, groups), dim3(kDecThreads), smem,
                                  st, dim3(C, 1, 1), a.q, a.kc, a.vc, a.out, a.H, a.Hkv, a.max_seq, a.d_pos, a.Ms, a.Ss,
                                  a.Mo, a.So, a.prob_bits, a.luts, a.err, C, a);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <int LPK>
static cudaError_t launch_dec_l(const AttnArgs& a, cudaStream_t st) {
  switch (dec_rb(a.H / a.Hkv)) {
    case 1: return launch_dec_rb<LPK, 1>(a, st);
    case 2: return launch_dec_rb<LPK, 2>(a, st);
    case 4: return launch_dec_rb<LPK, 4>(a, st);
    default: return launch_dec_rb<LPK, 8>(a, st);
  }
}
template <int LPK>
static cudaError_t prep_dec_l(size_t smem) {
  for (DecKernel f : {dec_kernel<LPK, 1>(), dec_kernel<LPK, 2>(), dec_kernel<LPK, 4>(), dec_kernel<LPK, 8>()}) {
    const cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}


template <int LPK>
static cudaError_t measure_dec_l(int rep, int max_seq) {
  switch (dec_rb(rep)) {
    case 1: return measure_dec_occupancy<LPK, 1>(max_seq);
    case 2: return measure_dec_occupancy<LPK, 2>(max_seq);
    case 4: return measure_dec_occupancy<LPK, 4>(max_seq);
    default: return measure_dec_occupancy<LPK, 8>(max_seq);
  }
}

cudaError_t prepare_attention_decode(int H, int Hkv, int D, int max_seq) {
  const int rep = H / Hkv;
  switch (D) {
    case 16: return measure_dec_l<1>(rep, max_seq);
    case 32: return measure_dec_l<2>(rep, max_seq);
    case 64: return measure_dec_l<4>(rep, max_seq);
    case 128: return measure_dec_l<8>(rep, max_seq);
    case 256: return measure_dec_l<16>(rep, max_seq);
    default: return cudaSuccess;
  }
}

cudaError_t launch_attention_decode(const AttnArgs& a, cudaStream_t st) {
  if (a.B <= 0) return cudaSuccess;
  switch (a.D) {
    case 16: return launch_dec_l<1>(a, st);
    case 32: return launch_dec_l<2>(a, st);
    case 64: return launch_dec_l<4>(a, st);
    case 128: return launch_dec_l<8>(a, st);
    case 256: return launch_dec_l<16>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------------------
// Prefill attention (M > 1 query rows per sequence): int8 MMA tiles.
//
// A CTA of 4 warps serves one (sequence, KV head) and 64 stacked (query row, query head)
// pairs of that KV head; each warp owns 16 of them as the M side of m16n8k32 integer MMAs.
// Key tiles of 64 rows stream through two shared-memory stages by cp.async.  The exact
// integer softmax keeps the reference's global order with three passes over the keys:
//   1. S = Q K^T (s8 x s8 -> s32), masked per-row max;
//   2. S again, p = exp-LUT(mulshift(max - s)), per-row sum -> inv = 2^31 / sum;
//   3. S again, pn = min(pmax, rshr(p * inv, 31 - prob_bits)), then O += pn V.
// pn (up to 15 bits) enters the MMA as two unsigned bytes, O = 256 * (hi V) + (lo V), exact
// in int32.  The value tile is transposed in shared memory with its keys permuted so that
// the P fragments the softmax produces in the accumulator layout are the MMA's A operand
// directly: PV operand k = 4 t + e of a 32-key chunk is key 16 h + [2t, 2t+1, 8+2t, 9+2t][e].
// The MMA only moves multiply-adds; the exp-LUT softmax on the CUDA cores is the cost.
// ---------------------------------------------------------------------------------------
constexpr int kPfThreads = 128;  // 4 warps x 16 stacked rows
constexpr int kPfKeys = 64;      // keys per tile
constexpr int kPfRows = 64;      // stacked (row, head) pairs per CTA

template <int D>
struct PfSmem {
  static constexpr int kKStride = D + 16;  // padded key rows: conflict-free operand loads
  static constexpr int kVtStride = 68;     // transposed value rows: 64 keys + 4 bytes
  static constexpr int kK = kPfKeys * kKStride;
  static constexpr int kV = kPfKeys * D;
  static constexpr int kVt = D * kVtStride;
  static constexpr int kBytes = 2 * kK + 2 * kV + kVt;
};

__device__ __forceinline__ void pf_cp16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(att_smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void pf_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void pf_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// d += a (16x32, s8 or u8 per A_U8) x b (32x8, s8)
template <bool A_U8>
__device__ __forceinline__ void pf_mma(int32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if (A_U8)
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int D, bool FAST>
__global__ void __launch_bounds__(kPfThreads) k_attention_prefill(
    const int8_t* q, const int8_t* kc, const int8_t* vc, int8_t* out,
    int M, int H, int Hkv, int max_seq, const int* d_pos, int64_t Ms, int Ss, int64_t Mo, int So,
    int prob_bits, const uint16_t* __restrict__ luts) {
  using L = PfSmem<D>;
  constexpr int KB = D / 32;  // k-blocks of Q K^T
  constexpr int NT = D / 8;   // 8-channel tiles of P V
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint16_t s_expi[16], s_expf[256];
  int8_t* Ks = reinterpret_cast<int8_t*>(smem);
  int8_t* Vs = Ks + 2 * L::kK;
  int8_t* Vt = Vs + 2 * L::kV;
  const int rep = H / Hkv;
  const int mq = kPfRows / rep;  // query rows per CTA
  const int b = blockIdx.z, kvh = blockIdx.y, m0 = blockIdx.x * mq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  pdl_trigger();
  for (int i = threadIdx.x; i < 16 + 256; i += kPfThreads) {
    if (i < 16)
      s_expi[i] = luts[kLutExpI + i];
    else
      s_expf[i - 16] = luts[kLutExpF + i - 16];
  }
  pdl_wait();  // POS, q and the KV cache come from earlier kernels
  const int pos = *d_pos;
  // this thread's stacked rows 16 warp + g (+ 8): query row, head, validity, last visible key
  int rm[2], rj[2], rlim[2];
  bool rv[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = 16 * warp + g + 8 * i;
    rm[i] = m0 + r / rep;
    rj[i] = r % rep;
    rv[i] = r < mq * rep && rm[i] < M;
    rlim[i] = rv[i] ? pos + rm[i] : -1;
  }
  const int Tc = pos + min(m0 + mq, M);  // keys 0..Tc-1 are visible to some row of the CTA
  // exp-LUT probability of a score gap (FAST: Ss >= 33, the product's high word decides z)
  const uint32_t rnd = FAST ? 1u << (Ss - 33) : 0u;
  const int zsh = FAST ? Ss - 32 : 0;
  auto prob = [&](uint32_t d) {
    return FAST ? gap_prob_hi(d, (uint32_t)Ms, rnd, zsh, s_expi, s_expf)
                : gap_prob(d, (uint32_t)Ms, Ss, s_expi, s_expf);
  };
  const int nkt = (Tc + kPfKeys - 1) / kPfKeys;
  const int8_t* kbase = kc + ((int64_t)b * Hkv + kvh) * max_seq * D;
  const int8_t* vbase = vc + ((int64_t)b * Hkv + kvh) * max_seq * D;

  // Q fragments (A of Q K^T): reg e of k-block kb is row g + 8 (e & 1), channels kb*32 + 16 (e >> 1) + 4 tig
  uint32_t qa[KB][4];
#pragma unroll
  for (int kb = 0; kb < KB; ++kb)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = e & 1;
      const int ch = kb * 32 + (e >> 1) * 16 + tig * 4;
      qa[kb][e] = rv[i] ? *reinterpret_cast<const uint32_t*>(
                              q + ((int64_t)(b * M + rm[i]) * H + kvh * rep + rj[i]) * D + ch)
                        : 0u;
    }

  auto load_tile = [&](int stage, int t0, bool with_v) {
    int8_t* kd = Ks + stage * L::kK;
    int8_t* vd = Vs + stage * L::kV;
    for (int i = threadIdx.x; i < kPfKeys * (D / 16); i += kPfThreads) {
      const int key = i / (D / 16), c = (i % (D / 16)) * 16;
      const bool ok = t0 + key < Tc;
      const int64_t off = ok ? (int64_t)(t0 + key) * D + c : 0;
      pf_cp16(kd + key * L::kKStride + c, kbase + off, ok);
      if (with_v) pf_cp16(vd + key * D + c, vbase + off, ok);
    }
  };
  // S for keys kc0 .. kc0 + 31 of a staged tile: s[j][e] is row g + 8 (e >> 1), key kc0 + 8 j + 2 tig + (e & 1)
  auto qk_chunk = [&](const int8_t* kst, int kc0, int32_t (&sv)[4][4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) sv[j][e] = 0;
      const int8_t* krow = kst + (kc0 + 8 * j + g) * L::kKStride + tig * 4;
#pragma unroll
      for (int kb = 0; kb < KB; ++kb)
        pf_mma<false>(sv[j], qa[kb], *reinterpret_cast<const uint32_t*>(krow + kb * 32),
                      *reinterpret_cast<const uint32_t*>(krow + kb * 32 + 16));
    }
  };

  // ---- pass 1: per-row max ----
  int32_t mx[2] = {INT_MIN, INT_MIN};
  load_tile(0, 0, false);
  pf_commit();
  for (int kt = 0; kt < nkt; ++kt) {
    if (kt + 1 < nkt) load_tile((kt + 1) & 1, (kt + 1) * kPfKeys, false);
    pf_commit();
    pf_wait<1>();
    __syncthreads();
    const int8_t* kst = Ks + (kt & 1) * L::kK;
    for (int c2 = 0; c2 < 2; ++c2) {
      const int kc0 = kt * kPfKeys + c2 * 32;
      if (kc0 >= Tc) break;
      int32_t sv[4][4];
      qk_chunk(kst, c2 * 32, sv);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = kc0 + 8 * j + 2 * tig + (e & 1);
          if (key <= rlim[e >> 1]) mx[e >> 1] = max(mx[e >> 1], sv[j][e]);
        }
    }
    __syncthreads();
  }
  pf_wait<0>();
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    mx[i] = max(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
    mx[i] = max(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
  }

  // ---- pass 2: exp-LUT probabilities, per-row sum -> inv ----
  uint32_t sum[2] = {0u, 0u};
  __syncthreads();
  load_tile(0, 0, false);
  pf_commit();
  for (int kt = 0; kt < nkt; ++kt) {
    if (kt + 1 < nkt) load_tile((kt + 1) & 1, (kt + 1) * kPfKeys, false);
    pf_commit();
    pf_wait<1>();
    __syncthreads();
    const int8_t* kst = Ks + (kt & 1) * L::kK;
    for (int c2 = 0; c2 < 2; ++c2) {
      const int kc0 = kt * kPfKeys + c2 * 32;
      if (kc0 >= Tc) break;
      int32_t sv[4][4];
      qk_chunk(kst, c2 * 32, sv);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = e >> 1;
          const int key = kc0 + 8 * j + 2 * tig + (e & 1);
          if (key <= rlim[i]) sum[i] += prob((uint32_t)(mx[i] - sv[j][e]));
        }
    }
    __syncthreads();
  }
  pf_wait<0>();
  uint32_t inv[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    sum[i] += __shfl_xor_sync(0xffffffffu, sum[i], 1);
    sum[i] += __shfl_xor_sync(0xffffffffu, sum[i], 2);
    inv[i] = 0x80000000u / (sum[i] ? sum[i] : 1u);
  }

  // ---- pass 3: normalised probabilities x V ----
  const uint32_t pmax = (1u << prob_bits) - 1u;
  const int pshift = 31 - prob_bits;
  const bool two = prob_bits > 8;  // pn needs its high byte
  int32_t o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0;
  __syncthreads();
  load_tile(0, 0, true);
  pf_commit();
  for (int kt = 0; kt < nkt; ++kt) {
    if (kt + 1 < nkt) load_tile((kt + 1) & 1, (kt + 1) * kPfKeys, true);
    pf_commit();
    pf_wait<1>();
    __syncthreads();
    // transpose the value tile into Vt[d][k] with the PV key order: keys {2t, 2t+1, 8+2t, 9+2t}
    // (+ 16 h + 32 c) -> k = 32 c + 16 h + 4 t + 0..3, in 4 x 4 byte blocks
    {
      const int8_t* vst = Vs + (kt & 1) * L::kV;
      for (int u = threadIdx.x; u < 16 * (D / 4); u += kPfThreads) {
        const int d0 = (u % (D / 4)) * 4, kg = u / (D / 4);  // kg = c * 8 + h * 4 + t
        const int t = kg & 3, base = (kg >> 2) * 16;       // base = 32 c + 16 h
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(vst + (base + 2 * t) * D + d0);
        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(vst + (base + 2 * t + 1) * D + d0);
        const uint32_t w2 = *reinterpret_cast<const uint32_t*>(vst + (base + 8 + 2 * t) * D + d0);
        const uint32_t w3 = *reinterpret_cast<const uint32_t*>(vst + (base + 9 + 2 * t) * D + d0);
        const uint32_t x0 = __byte_perm(w0, w1, 0x5140), x1 = __byte_perm(w2, w3, 0x5140);
        const uint32_t x2 = __byte_perm(w0, w1, 0x7362), x3 = __byte_perm(w2, w3, 0x7362);
        int8_t* dst = Vt + d0 * L::kVtStride + base + 4 * t;
        *reinterpret_cast<uint32_t*>(dst) = __byte_perm(x0, x1, 0x5410);
        *reinterpret_cast<uint32_t*>(dst + L::kVtStride) = __byte_perm(x0, x1, 0x7632);
        *reinterpret_cast<uint32_t*>(dst + 2 * L::kVtStride) = __byte_perm(x2, x3, 0x5410);
        *reinterpret_cast<uint32_t*>(dst + 3 * L::kVtStride) = __byte_perm(x2, x3, 0x7632);
      }
    }
    __syncthreads();
    const int8_t* kst = Ks + (kt & 1) * L::kK;
    for (int c2 = 0; c2 < 2; ++c2) {
      const int kc0 = kt * kPfKeys + c2 * 32;
      if (kc0 >= Tc) break;
      int32_t sv[4][4];
      qk_chunk(kst, c2 * 32, sv);
      // A fragments: reg e holds row g + 8 (e & 1), S tiles 2 (e >> 1) and 2 (e >> 1) + 1
      uint32_t plo[4], phi[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = e & 1, jb = (e >> 1) * 2;
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const int j = jb + (x >> 1), c = 2 * i + (x & 1);
          const int key = kc0 + 8 * j + 2 * tig + (x & 1);
          uint32_t pn = 0;
          if (key <= rlim[i]) {
            const uint32_t y = prob((uint32_t)(mx[i] - sv[j][c])) * inv[i];  // p <= sum: p * inv <= 2^31
            pn = (y >> pshift) + ((y >> (pshift - 1)) & 1u);
            pn = pn < pmax ? pn : pmax;
          }
          lo |= (pn & 255u) << (8 * x);
          hi |= (pn >> 8) << (8 * x);
        }
        plo[e] = lo;
        phi[e] = hi;
      }
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int8_t* vrow = Vt + (8 * n + g) * L::kVtStride + c2 * 32 + 4 * tig;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(vrow);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(vrow + 16);
        int32_t tl[4] = {0, 0, 0, 0};
        pf_mma<true>(tl, plo, b0, b1);
        if (two) {
          int32_t th[4] = {0, 0, 0, 0};
          pf_mma<true>(th, phi, b0, b1);
#pragma unroll
          for (int e = 0; e < 4; ++e) o[n][e] += th[e] * 256 + tl[e];
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) o[n][e] += tl[e];
        }
      }
    }
    __syncthreads();
  }
  pf_wait<0>();
  // ---- outputs: o = rshr(acc, 7) (Q0.15), sat8(mulshift(o, Mo, So)) ----
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    if (!rv[i]) continue;
    int8_t* orow = out + ((int64_t)(b * M + rm[i]) * H + kvh * rep + rj[i]) * D;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      int64_t v0 = o[n][2 * i], v1 = o[n][2 * i + 1];
      if (two) {
        v0 = rshr(v0, 7);
        v1 = rshr(v1, 7);
      }
      const uint32_t b0 = (uint8_t)(int8_t)sat8(mulshift(v0, Mo, So));
      const uint32_t b1 = (uint8_t)(int8_t)sat8(mulshift(v1, Mo, So));
      *reinterpret_cast<uint16_t*>(orow + 8 * n + 2 * tig) = (uint16_t)(b0 | (b1 << 8));
    }
  }
}

template <int D>
static cudaError_t launch_prefill_d(const AttnArgs& a, cudaStream_t st) {
  const int rep = a.H / a.Hkv;
  const int mq = kPfRows / rep;
  const dim3 grid((a.M + mq - 1) / mq, a.Hkv, a.B);
  auto kern = a.Ss >= 33 ? k_attention_prefill<D, true> : k_attention_prefill<D, false>;
  const cudaError_t e = launch_k(kern, grid, dim3(kPfThreads), (size_t)PfSmem<D>::kBytes, st, a.q,
                                 a.kc, a.vc, a.out, a.M, a.H, a.Hkv, a.max_seq, a.d_pos, a.Ms, a.Ss, a.Mo, a.So,
                                 a.prob_bits, a.luts);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t prepare_attention(size_t smem) {
  cudaError_t e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  for (auto f : {k_attention_prefill<64, false>, k_attention_prefill<64, true>}) {
    e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, PfSmem<64>::kBytes);
    if (e != cudaSuccess) return e;
  }
  for (auto f : {k_attention_prefill<128, false>, k_attention_prefill<128, true>}) {
    e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, PfSmem<128>::kBytes);
    if (e != cudaSuccess) return e;
  }
  for (auto f : {prep_dec_l<1>, prep_dec_l<2>, prep_dec_l<4>, prep_dec_l<8>, prep_dec_l<16>}) {
    e = f(smem);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st) {
  const int R = a.B * a.M;
  if (R <= 0) return cudaSuccess;
  if (a.M == 1 && (a.D == 16 || a.D == 32 || a.D == 64 || a.D == 128 || a.D == 256))
    return launch_attention_decode(a, st);
  if (a.H / a.Hkv <= kPfRows && (a.prob_bits == 8 || a.prob_bits == 15)) {
    if (a.D == 64) return launch_prefill_d<64>(a, st);
    if (a.D == 128) return launch_prefill_d<128>(a, st);
  }
  const size_t smem = attention_smem_bytes(a.H, a.Hkv, a.D, a.max_seq);
  dim3 grid(R, a.Hkv);
  { const cudaError_t e_ = launch_k(k_attention, dim3(grid), dim3(256), smem, st, a.q, a.kc, a.vc, a.out, a.M, a.H, a.Hkv, a.D, a.max_seq, a.d_pos, a.Ms, a.Ss,
                                        a.Mo, a.So, a.prob_bits, a.luts); if (e_ != cudaSuccess) return e_; }
  return cudaGetLastError();
}

}  // namespace llx
