// Device-side integer primitives of the llaccel numerics contract.
//
// Each function is the exact integer formula of docs/NUMERICS.md "Primitives"
// (reference: include/llaccel/numerics.h:15-56, python/llaccel/golden.py:35-120).
// All widening happens in 64-bit registers; products are formed in unsigned 64-bit
// arithmetic so that out-of-range parameters wrap exactly like the numpy int64 golden
// model instead of hitting C++ signed-overflow rules.
#pragma once
#include <cstdint>

namespace llx {

// Sigmoid / exp tables (python/llaccel/luts.py:18-29) live in device global memory, uploaded
// with the model: kLutSig (257 entries), kLutExpI (16) and kLutExpF (256) back to back.
// Lookups are data dependent per lane, so they go through L1 (or shared memory), not
// the constant cache, which would serialise divergent addresses.
constexpr int kLutSig = 0, kLutExpI = 257, kLutExpF = 273, kLutCount = 529;

__device__ __forceinline__ int64_t mul64(int64_t a, int64_t b) {
  return (int64_t)((uint64_t)a * (uint64_t)b);
}

// round-half-up arithmetic right shift, s in [0, 63]; s == 0 passes v (numerics.h:15-18)
__device__ __forceinline__ int64_t rshr(int64_t v, int s) {
  if (s == 0) return v;
  return (v >> s) + ((v >> (s - 1)) & 1);
}

__device__ __forceinline__ int64_t clampi(int64_t v, int64_t lo, int64_t hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}
__device__ __forceinline__ int64_t sat8(int64_t v) { return clampi(v, -128, 127); }
__device__ __forceinline__ int64_t sat16(int64_t v) { return clampi(v, -32768, 32767); }

__device__ __forceinline__ int64_t mulshift(int64_t v, int64_t M, int S) { return rshr(mul64(v, M), S); }

// mulshift of a 32-bit value for S >= 32 and 0 <= M < 2^31 from the 64-bit product's high
// word: p = v * M, hi = floor(p / 2^32).  Then p >> S = hi >> (S - 32) and the rounding bit
// (bit S - 1 of p) is bit S - 33 of hi, or for S = 32 the top bit of the low word.  Equal to
// mulshift(v, M, S) for every int32 v.
__device__ __forceinline__ int32_t mulshift_hi32(int32_t v, int32_t M, int S) {
  const int32_t hi = __mulhi(v, M);
  const uint32_t rbit = S >= 33 ? ((uint32_t)hi >> (S - 33)) & 1u : ((uint32_t)v * (uint32_t)M) >> 31;
  return (hi >> (S - 32)) + (int32_t)rbit;
}

// floor(sqrt(t)) for t < 2^48, bit-serial (numerics.h:26-35): 24 iterations, one digit each.
__device__ __forceinline__ uint32_t isqrt48(uint64_t t) {
  uint64_t rem = 0, root = 0;
#pragma unroll
  for (int i = 23; i >= 0; --i) {
    rem = (rem << 2) | ((t >> (2 * i)) & 3);
    root <<= 1;
    const uint64_t trial = (root << 1) | 1;
    if (trial <= rem) {
      rem -= trial;
      root |= 1;
    }
  }
  return (uint32_t)root;
}

// unsigned division with b == 0 read as 1, truncated to u32 (numerics.h:36)
__device__ __forceinline__ uint32_t udiv(uint64_t a, uint64_t b) { return (uint32_t)(a / (b ? b : 1)); }

// isqrt48 through the hardware double square root, then corrected to the exact floor with
// integer products: for t < 2^48 the double result is within one unit of floor(sqrt(t)),
// and each correction step runs at most once.
__device__ __forceinline__ uint32_t isqrt48_fast(uint64_t t) {
  uint64_t r = (uint64_t)sqrt((double)t);
  if (r * r > t) --r;
  if ((r + 1) * (r + 1) <= t) ++r;
  return (uint32_t)r;
}

// floor(a / b) for a < 2^53, 1 <= b < 2^32 through a double divide, corrected to the exact
// quotient with integer products (the double quotient is within one unit of it).
__device__ __forceinline__ uint64_t udiv_fast(uint64_t a, uint32_t b) {
  uint64_t q = (uint64_t)((double)a / (double)b);
  if (q * b > a) --q;
  if ((q + 1) * b <= a) ++q;
  return q;
}

// LUT SiLU with linear interpolation (numerics.h:45-51; NUMERICS.md:127-139)
__device__ __forceinline__ int64_t silu16(int64_t x, int64_t Mi, int Si, int sh_out, const uint16_t* __restrict__ sig) {
  const int64_t u = sat16(mulshift(x, Mi, Si));
  const int idx = (int)(u >> 8) + 128;  // u in [-32768, 32767] -> idx in [0, 255]
  const int64_t f = u & 255;
  const int64_t lo = __ldg(sig + idx);
  const int64_t sg = lo + (((int64_t)__ldg(sig + idx + 1) - lo) * f >> 8);
  return sat16(rshr(x * sg, sh_out));
}

// exp LUT probability of a score gap z = mulshift(mx - s, Ms, Ss) >= 0 (numerics.h:104-107)
// expi/expf may point to shared or global memory
__device__ __forceinline__ uint32_t exp_prob(int64_t z, const uint16_t* expi, const uint16_t* expf) {
  if ((uint64_t)z >= 4096u) return 0;
  const uint32_t zi = (uint32_t)z;
  return ((uint32_t)expi[zi >> 8] * (uint32_t)expf[zi & 255] + (1u << 15)) >> 16;
}

}  // namespace llx
