// C-ABI shim over the reference's header-only numerics contract
// (include/llaccel/numerics.h, compiled in place from the reference checkout by
// oracle/Makefile).  TEST INFRASTRUCTURE ONLY: tests use it to cross-check the numpy
// oracle against the reference's own C++ arithmetic.  Nothing in the product links it.
#include <cstdint>
#include <span>
#include <vector>

#include "llaccel/numerics.h"

namespace n = llaccel::num;

extern "C" {
int64_t ref_rshr(int64_t v, uint32_t s) { return n::rshr(v, s); }
int64_t ref_mulshift(int64_t v, uint32_t M, uint32_t S) { return n::mulshift(v, M, S); }
uint32_t ref_isqrt48(uint64_t t) { return n::isqrt48(t); }
int64_t ref_requant16(int32_t acc, int32_t M, int32_t S) { return n::requant16(acc, n::RqEntry{M, S}); }
int64_t ref_silu16(int64_t x, uint32_t Mi, uint32_t Si, uint32_t sh) { return n::silu16(x, Mi, Si, sh); }
int64_t ref_vmul(int64_t a, int64_t b, uint32_t sh) { return n::vmul(a, b, sh); }
int64_t ref_vadd(int64_t a, int64_t b, uint32_t sh) { return n::vadd(a, b, sh); }
int64_t ref_vquant(int64_t x, uint32_t M, uint32_t S) { return n::vquant(x, M, S); }

void ref_rmsnorm(const int16_t* x, const int16_t* g, int16_t* y, uint32_t K, uint32_t eps_t, uint32_t C,
                 uint32_t sh_post) {
  n::rmsnorm(std::span<const int16_t>(x, K), std::span<const int16_t>(g, K), std::span<int16_t>(y, K), eps_t, C,
             sh_post);
}

void ref_rope(const int16_t* x, int16_t* y, uint32_t H, uint32_t D, const int16_t* cosv, const int16_t* sinv) {
  n::rope(std::span<const int16_t>(x, H * D), std::span<int16_t>(y, H * D), H, D,
          std::span<const int16_t>(cosv, D / 2), std::span<const int16_t>(sinv, D / 2));
}

// keys/vals: [T][D] int8 row-major
void ref_attention_head(const int8_t* q, const int8_t* keys, const int8_t* vals, uint32_t D, uint32_t T, uint32_t Ms,
                        uint32_t Ss, uint32_t Mo, uint32_t So, int8_t* out, int wide) {
  std::vector<int32_t> scores;
  std::vector<uint16_t> probs;
  n::attention_head(
      std::span<const int8_t>(q, D), D, T, [&](uint32_t t) { return keys + size_t(t) * D; },
      [&](uint32_t t) { return vals + size_t(t) * D; }, Ms, Ss, Mo, So, std::span<int8_t>(out, D), scores, probs,
      wide != 0);
}
}
