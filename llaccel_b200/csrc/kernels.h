// Launch wrappers for the sm_100a kernels of the integer datapath.
// Every wrapper enqueues on `st` and returns cudaGetLastError() of the launch.
// Position-dependent kernels read POS from device memory (`d_pos`) so that a captured
// CUDA graph replays for any position.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace llx {

// ---- vector engine ----------------------------------------------------------------------
// tokens [R] (< 0 = zero pad row) -> out [R][dim] i16 rows of `embed`
// also zeroes amax_key[0..R) when non-null (the fused argmax of the output linear)
cudaError_t launch_embed(const int32_t* tokens, const int16_t* embed, int16_t* out, int R, int dim, int vocab_rows,
                         int32_t* err, unsigned long long* amax_key, cudaStream_t st);
// argmax tokens from the fused argmax keys: out[r] = 0xFFFFFFFF - low32(key[r])
cudaError_t launch_amax_finish(const unsigned long long* keys, int32_t* out, int R, cudaStream_t st);

// rows x [nrows][K] -> y [nrows][K]; optional fused quant to y8 (M_q, S_q)
cudaError_t launch_rmsnorm(const int16_t* x, const int16_t* gamma, int16_t* y, int8_t* y8, int nrows, int K,
                           int64_t eps_t, int64_t C, int sh_post, int64_t Mq, int Sq, cudaStream_t st);

cudaError_t launch_quant(const int16_t* x, int8_t* y, int64_t n, int64_t M, int S, cudaStream_t st);

// RoPE over x [R][H*D] (row r at position pos + r % M); y16 gets the rotated i16 rows;
// optional fused quant into y8; with kcache also writes y8 rows into
// kcache[b][h][pos + m][:] (b = r / M, cache [B][H][max_seq][D]).
cudaError_t launch_rope(const int16_t* x, int16_t* y16, int8_t* y8, int64_t Mq, int Sq, int8_t* kcache, int R, int M,
                        int H, int D, const int16_t* cos_tab, const int16_t* sin_tab, const int* d_pos, int max_seq,
                        cudaStream_t st);

// Both RoPEs of a layer in one launch: job q (no cache) and job k (K cache write), each with
// fused QUANT, plus the V rows copied into vcache.  Row r is at position pos + r % M.
struct RopeJob {
  const int16_t* x;
  int16_t* y16;
  int8_t* y8;
  int64_t Mq;
  int Sq;
  int8_t* kcache;
  int H;
};
cudaError_t launch_rope_group(const RopeJob& q, const RopeJob& k, const int8_t* v, int8_t* vcache, int Hkv, int R,
                              int M, int D, const int16_t* cos_tab, const int16_t* sin_tab, const int* d_pos,
                              int max_seq, cudaStream_t st);

// k, v [R][Hkv*D] i8 -> caches [B][Hkv][max_seq][D] at positions pos + m
cudaError_t launch_kv_write(const int8_t* k, const int8_t* v, int8_t* kc, int8_t* vc, int R, int M, int Hkv, int D,
                            const int* d_pos, int max_seq, cudaStream_t st);

cudaError_t launch_add(const int16_t* a, const int16_t* b, int16_t* y, int64_t n, int sh_b, cudaStream_t st);
cudaError_t launch_mul(const int16_t* a, const int16_t* b, int16_t* y, int64_t n, int sh, cudaStream_t st);
// luts: device tables laid out as numerics.cuh kLut* (sigmoid, exp-int, exp-frac)
cudaError_t launch_silu(const int16_t* x, int16_t* y, int64_t n, int64_t Mi, int Si, int sh_out,
                        const uint16_t* luts, cudaStream_t st);

// Packed argmax keys of logits [R][ld] i16 over the first `vocab` entries: keys[r] =
// max(keys[r], max_n (logit + 32768) << 32 | (0xFFFFFFFF - (base + n))), keys zeroed by the
// caller beforehand (base: global index of channel 0 of a vocabulary shard).  The max key
// is the first maximum; launch_amax_finish decodes it.
cudaError_t launch_argmax(const int16_t* logits, int R, int ld, int vocab, int base, unsigned long long* keys,
                          cudaStream_t st);

// dst[i][:] = src[idx[i]][:] for i < n (row bytes multiple of 16)
cudaError_t launch_gather_rows(const void* src, void* dst, const int32_t* idx, int n, int row_bytes,
                               cudaStream_t st);

// ---- matrix engine ------------------------------------------------------------------------
enum Epilogue : int { EPI_NONE = 0, EPI_RESADD = 1, EPI_SILU = 2, EPI_MUL = 3 };

struct LinearArgs {
  const int8_t* A;      // [R][K] i8, row stride K
  const int8_t* W;      // [N][K] i8 row-major
  const int32_t* bias;  // [N] or null
  const int32_t* rq;    // [N][2] {M, S}
  const int16_t* aux;   // [R][N] i16 (RESADD / MUL) or null
  void* out;            // [R][N] i16, or i8 when out_i8, or raw i32 sums when out_i32; null for an
                        // i16 output with fused argmax: only the argmax keys are produced
  int R, N, K;
  int out_i8;
  int out_i32;          // tensor-parallel partial: store sum_k A*W as int32, no bias / requant
  int epi;
  int64_t silu_Mi;
  int silu_Si, silu_sh;
  int aux_shift;
  const uint16_t* luts;  // device tables (SILU epilogue)
  int narrow;            // 1: |acc + bias| < 2^31 for every channel (proved at load), 32-bit bias add
  // Fused multi-output linear (several linears sharing A, epilogue none): channel segments
  // [seg_start[i], seg_start[i+1]) of the concatenated W go to seg_out[i] (row stride =
  // segment width, i8 when seg_i8[i]).  nseg = 0: single output `out`.
  int nseg;
  int seg_start[5];
  void* seg_out[4];
  int seg_i8[4];
  // Fused gate/up pair: W rows interleave 16 gate rows and 16 up rows; channel block j of
  // 16 outputs is gate chunk 2j and up chunk 2j+1.  Per output channel:
  //   sg = silu16(requant16(acc_g)); f = sat16(rshr(requant16(acc_u) * sg, aux_shift));
  //   fq = sat8(mulshift(f, q_M, q_S)).  Outputs [R][Nout]; each may be null.
  int gated, Nout;
  int16_t* g_out;
  int16_t* f_out;
  int8_t* q_out;
  int64_t q_M;
  int q_S;
  // Fused argmax (model output linear): per row, the max over channels n < amax_vocab of
  // key = (logit + 32768) << 32 | (0xFFFFFFFF - n) is folded into amax_key[r] with a 64-bit
  // atomicMax (largest logit, lowest index on ties).  amax_key must be zero beforehand.
  // amax_base: global index of channel 0 (a vocabulary shard under tensor parallelism).
  unsigned long long* amax_key;
  int amax_vocab;
  int amax_base;
  // RMSNorm folded into a one-row GEMV (R == 1; nx non-null): A is not read; every block
  // computes it from the i16 row nx [K] into shared memory, exactly as the RMSNorm + quant
  // step would (numerics.h:60-71): inv = min(65535, n_C / max(isqrt48(sum x^2 + n_eps), 1)),
  // A = sat8(mulshift(sat16(rshr(x * g * inv, n_sh)), n_Mq, n_Sq)).
  const int16_t* nx;
  const int16_t* ngamma;
  int64_t n_eps, n_C, n_Mq;
  int n_sh, n_Sq;
};

// Tensor-parallel requant: acc [R][N] i32 (the all-reduced partial sums of a row-split
// linear) -> bias, per-channel requant and epilogue exactly as the linear epilogue does,
// into out [R][N] (i16, or i8 when a.out_i8).  Reads a.bias / a.rq / a.aux / a.epi /
// silu / aux_shift / luts / out_i8 / narrow; a.A, a.W and a.K are unused.
cudaError_t launch_requant(const int32_t* acc, const LinearArgs& a, cudaStream_t st);

// CUDA-core paths: 0 = auto, 1 = GEMV (small R), 2 = tiled dp4a
cudaError_t launch_linear(const LinearArgs& a, int path, cudaStream_t st);

// Tensor-core path (gemm_tc.cu).  map_a: activations [rows][K] with a 128-row box;
// map_w: weights [N][K] with an nt-row box; both from make_tmap_i8.  nt in
// {16, 32, 64, 128, 256}; ksplit CTAs per cluster split K (1 = none).  err receives a
// nonzero code if a pipeline wait timed out.
cudaError_t make_tmap_i8(CUtensorMap* map, const void* base, int64_t rows, int64_t K, int box_rows);
// Decode GEMM with swapped operands (gemm_sab.cu), R <= 128 rows: map_a with an nb-row box
// (nb = sab_rows_per_tile(R)), map_w with a 128-row box; ksplit (1..16) CTAs per cluster
// split K.  Same arguments and results as launch_linear_tc.
int sab_rows_per_tile(int R);
cudaError_t launch_linear_sab(const CUtensorMap& map_a, const CUtensorMap& map_w, const LinearArgs& a, int nb,
                              int ksplit, int32_t* err, cudaStream_t st);
cudaError_t prepare_linear_tc();
cudaError_t launch_linear_tc(const CUtensorMap& map_a, const CUtensorMap& map_w, const LinearArgs& a, int nt,
                             int ksplit, int32_t* err, cudaStream_t st);
// Persistent tensor-core GEMM for many output tiles (no split-K): min(tiles, sms) CTAs walk
// the tiles with a double-buffered TMEM accumulator, the epilogue of one tile overlapping the
// main loop of the next.  nt in {128, 256}; map_w with an nt-row box.
cudaError_t launch_linear_tc_persistent(const CUtensorMap& map_a, const CUtensorMap& map_w, const LinearArgs& a,
                                        int nt, int sms, int32_t* err, cudaStream_t st);

// ---- attention engine -------------------------------------------------------------------
struct AttnArgs {
  const int8_t* q;   // [R][H*D]
  const int8_t* kc;  // [B][Hkv][max_seq][D]
  const int8_t* vc;
  int8_t* out;       // [R][H*D]
  int B, M, H, Hkv, D, max_seq;
  const int* d_pos;
  int pos_hint;      // host copy of pos (sizes shared memory; must be >= the device value)
  int64_t Ms, Mo;
  int Ss, So;
  int prob_bits;
  const uint16_t* luts;  // device tables (exp LUTs)
  int32_t* err;          // device error word (a bounded wait timed out)
  // Decode (M = 1) with the layer's RoPE group folded in (rq16 non-null): rq16 / rk16 are
  // the unrotated i16 rows [B][H*D] / [B][Hkv*D], rv8 the quantized values [B][Hkv*D].  The
  // kernel rotates and quantizes q and the newest key, writes the newest K and V rows to the
  // caches and uses them directly (RoPE: numerics.h:75-84).
  const int16_t* rq16;
  const int16_t* rk16;
  const int8_t* rv8;
  int8_t* kc_out;  // the caches kc / vc, written at position pos
  int8_t* vc_out;
  const int16_t* cos_tab;
  const int16_t* sin_tab;
  int64_t q_M, k_M;
  int q_S, k_S;
};
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st);
// opt the attention kernel into `smem` bytes of dynamic shared memory (once per device, before capture)
cudaError_t prepare_attention(size_t smem);
size_t attention_smem_bytes(int H, int Hkv, int D, int T);
size_t attention_decode_smem_bytes(int H, int Hkv, int D, int max_seq);
// measures resident clusters of the decode kernel for this geometry (after prepare_attention;
// outside stream capture): the decode launch picks its cluster size from them
cudaError_t prepare_attention_decode(int H, int Hkv, int D, int max_seq);

}  // namespace llx
