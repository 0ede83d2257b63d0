// Host-only check of the decode attention's shared-memory layout, compiled together with the
// real kernels_attn.cu (its layout functions are the ones the kernels and launches use).  No
// kernel is launched and no GPU is needed.  Exit status 0 when every invariant holds:
//   * every key of a slice has an int32 score slot per head (stride >= capacity >= slice);
//   * packed layout (head dim 128, 4+ heads per CTA): the hi / lo probability bytes of the
//     slice's whole tiles fit the head's own slots, and the chunked in-place writes of a
//     512-key chunk land only on slots that chunk (or an earlier one) has already read;
//   * the value partials fit the ring they reuse;
//   * the C4 and C5 bench shapes fit 4 CTAs per SM (228 KB per SM, 1 KB reserved per CTA).
#include "../llaccel_b200/csrc/kernels_attn.cu"

#include <algorithm>
#include <cstdio>

namespace llx {
int g_pdl = 0;
}
using namespace llx;

static int fails = 0;
#define CHECK(cond, ...)                            \
  do {                                              \
    if (!(cond)) {                                  \
      if (++fails <= 20) {                          \
        std::printf("FAIL %s: ", #cond);            \
        std::printf(__VA_ARGS__);                   \
        std::printf("\n");                          \
      }                                             \
    }                                               \
  } while (0)

int main() {
  long shapes = 0, chunks = 0;
  for (int D : {16, 32, 64, 128, 256})
    for (int RB : {1, 2, 4, 8})
      for (int C : {1, 2, 4, 8})
        for (int max_seq = 16; max_seq <= 8192; max_seq += max_seq < 512 ? 16 : 112) {
          const int TK = dec_tile_keys(D);
          const int cap = dec_slice_cap(max_seq, C);
          const int ss = dec_sstride(max_seq, C, D, RB);
          const int slice = (max_seq + C - 1) / C;
          CHECK(ss >= cap && ss % 2 == 0 && cap >= slice, "D=%d RB=%d C=%d max_seq=%d ss=%d cap=%d", D, RB, C,
                max_seq, ss, cap);
          if (dec_packed(D, RB)) {
            const int nfill_max = (slice + TK - 1) / TK * TK;
            CHECK(2 * nfill_max <= 4 * ss, "D=%d RB=%d C=%d max_seq=%d nfill=%d ss=%d", D, RB, C, max_seq,
                  nfill_max, ss);
            const int step = slice > 64 ? slice / 64 : 1;
            for (int nkeys = 1; nkeys <= slice; nkeys += step) {
              const int nfill = (nkeys + TK - 1) / TK * TK;
              for (int c0 = 0; c0 < nfill; c0 += 2 * kDecThreads) {
                const int end = std::min(c0 + 2 * kDecThreads, nfill);
                for (int t = c0; t < end; ++t) {
                  const int u = t & 15;
                  const int hi = 32 * (t >> 4) + 4 * (u & 3) + (u >> 2), lo = hi + 16;
                  // both bytes inside the head's slots, on a slot below the chunk's end
                  CHECK(lo < 4 * ss && lo / 4 < c0 + 2 * kDecThreads && hi / 4 < c0 + 2 * kDecThreads,
                        "D=%d RB=%d C=%d max_seq=%d t=%d", D, RB, C, max_seq, t);
                }
                ++chunks;
              }
            }
            CHECK((size_t)dec_ring(D) * TK * D >= (size_t)RB * D * 4, "ring D=%d RB=%d", D, RB);
          }
          ++shapes;
        }
  // the bench shapes: C5 (4 heads per KV head, D 128, max_seq 1280) at cluster size 1 and C4
  // (2 heads, max_seq 4224) at cluster size 2, each CTA with at most 1 KB of static shared
  // memory and 1 KB reserved
  const size_t c5 = dec_smem_bytes(4, 128, 1280, 1), c4 = dec_smem_bytes(2, 128, 4224, 2);
  CHECK(c5 == 54080, "C5 %zu bytes", c5);
  CHECK(c4 == 51168, "C4 %zu bytes", c4);
  CHECK(4 * (c5 + 2048) <= 228 * 1024 && 4 * (c4 + 2048) <= 228 * 1024, "C5 %zu, C4 %zu bytes", c5, c4);
  std::printf("%ld shapes, %ld chunks checked, %d failures\n", shapes, chunks, fails);
  return fails ? 1 : 0;
}
