/*
 * llx -- C ABI of the B200 (sm_100a) backend for llaccel's integer transformer datapath.
 *
 * The backend executes the quantized graph that llaccel's importer/quantizer write
 * (qgraph.json + qweights.bin, docs/DIALECT.md section 2) with the exact integer semantics
 * of docs/NUMERICS.md, bit for bit against python/llaccel/golden.py.
 *
 * Reference interfaces replaced (paths in the llaccel tree):
 *   llx_model_load / llx_session_create   GoldenModel.__init__ + QGraph
 *                                          (python/llaccel/golden.py:189-264);
 *                                          Host::Host image upload (runtime/src/host.cpp:47-101)
 *   llx_session_reset                      GoldenModel.reset (golden.py:266-272);
 *                                          KV clear in Host::generateTokens (host.cpp:145-158)
 *   llx_run                                Host::launch (host.cpp:121-130) = writeInputRow +
 *                                          Device::run(pc, pos) (runtime/include/llaccel/device.h:26)
 *                                          + readLogitsRow + argmax
 *   llx_run_rows                           GoldenModel.run_chunk (golden.py:275-314)
 *   llx_generate                           GoldenModel.generate (golden.py:399-440);
 *                                          Host::generateTokens (host.cpp:137-188)
 *   llx_read_activation                    run_chunk(acts=...) / --dump-acts (golden.py:312-313, 443-450)
 *   llx_last_error                         the ValueError / std::runtime_error messages
 *
 * Conventions: host pointers are caller-owned; device memory is owned by the model (weights,
 * tables) and the session (KV cache, activations).  Every call returns LLX_OK or an error
 * code; llx_last_error() returns the thread's last message.  A session is not thread-safe;
 * a model may be shared by sessions on its device.  No call falls back to the CPU.
 */
#ifndef LLX_H
#define LLX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  LLX_OK = 0,
  LLX_ERR_INVALID = 1,     /* malformed qgraph / argument (golden: ValueError) */
  LLX_ERR_IO = 2,          /* file missing or unreadable */
  LLX_ERR_CUDA = 3,        /* CUDA runtime error */
  LLX_ERR_OOM = 4,         /* device allocation failed */
  LLX_ERR_RANGE = 5,       /* positions / rows / token ids out of range */
  LLX_ERR_UNSUPPORTED = 6, /* a qgraph feature this backend does not execute */
  LLX_ERR_DEVICE = 7       /* a kernel reported a device-side error word */
} llx_status;

typedef struct llx_model llx_model;
typedef struct llx_session llx_session;

typedef struct {
  int device;    /* CUDA device ordinal */
  int fuse;      /* 1: fuse QUANT/KV_WRITE into their producers (default); 0: one kernel per op */
  int gemm_path; /* 0 auto, 1 CUDA-core GEMV, 2 CUDA-core tiled, 3 tensor-core tcgen05, 4 tensor-core without
                    the swapped-operand decode kernel (a cross-check of 3) */
  int pdl;       /* 1: programmatic dependent launch between the kernels of a launch (default) */
} llx_opts;

typedef struct {
  int dim, n_layers, n_heads, n_kv_heads, head_dim, ffn, vocab, vocab_padded, max_seq, prefill_m;
  int E_RES, E_LOGIT;
  int n_ops, n_steps, n_activations;
  size_t weight_bytes;
  /* tensor parallelism (1, 0, 0 on one GPU): this rank's graph outputs global vocabulary
   * channels [vocab_base, vocab_base + vocab_local); vocab_padded is the full width that
   * logits outputs carry.  n_heads / n_kv_heads are this rank's heads. */
  int tp_world, tp_rank, vocab_base, vocab_local;
} llx_model_info;

/* Load qgraph_dir/{qgraph.json, <weights_file>}, validate every op, upload weights,
 * requant tables, RoPE tables and LUTs to the device. opts may be NULL (defaults). */
llx_status llx_model_load(const char* qgraph_dir, const llx_opts* opts, llx_model** out);
void llx_model_destroy(llx_model* m);
llx_status llx_model_get_info(const llx_model* m, llx_model_info* out);

/* A session holds the KV cache of `batch` independent sequences and the activation
 * buffers for launches of up to `max_rows` rows per sequence. keep_acts=1 keeps every
 * named activation of the last launch readable (no buffer reuse). */
llx_status llx_session_create(llx_model* m, int batch, int max_rows, int keep_acts, llx_session** out);
void llx_session_destroy(llx_session* s);
llx_status llx_session_reset(llx_session* s);

/* One launch over all sequences: tokens [batch][M] (-1 = zero pad row) at positions
 * pos..pos+M-1. rec_rows [batch][n_rec] selects the rows whose logits are produced
 * (NULL: all M rows, n_rec = M). Outputs (each may be NULL): logits [batch][n_rec][vocab_padded]
 * i16 at E_LOGIT, argmax [batch][n_rec] over the first vocab logits (lowest index on ties). */
llx_status llx_run(llx_session* s, const int32_t* tokens, int M, int pos, const int32_t* rec_rows, int n_rec,
                   int16_t* logits, int32_t* argmax);

/* Like llx_run with all rows recorded, but the input rows are given: rows [batch][M][dim] i16. */
llx_status llx_run_rows(llx_session* s, const int16_t* rows, int M, int pos, int16_t* logits, int32_t* argmax);

/* Greedy generation with the reference runtime's launch sequence for each of the batch
 * sequences (equal prompt length L): prefill, then one decode launch per generated token
 * (skipped when the next position would not fit max_seq). prefill_rows = 0 mirrors the
 * golden chunking (prefill_m-row chunks, zero pad rows); > 0 runs prefill launches of up
 * to prefill_rows rows per sequence (a multiple of prefill_m), which yields identical
 * records. Outputs: generated [batch][n_tokens]; argmax [batch][n_launch];
 * logits [batch][n_launch][vocab] (NULL to skip); *n_launch_out = launches per sequence. */
llx_status llx_generate(llx_session* s, const int32_t* prompts, int L, int n_tokens, int prefill_rows,
                        int32_t* generated, int32_t* argmax, int16_t* logits, int* n_launch_out);

/* Device-resident greedy decode for benchmarking and serving: n_steps M=1 launches at
 * positions pos..pos+n_steps-1, each fed by the previous launch's argmax on the device
 * (the first by the argmax of the last launch, or by llx_set_tokens). Enqueues only
 * (no host synchronisation); history (may be NULL) receives [n_steps][batch] argmax after
 * llx_sync. */
llx_status llx_set_tokens(llx_session* s, const int32_t* tokens);
llx_status llx_decode_async(llx_session* s, int pos, int n_steps);
llx_status llx_read_history(llx_session* s, int n_steps, int32_t* history);
llx_status llx_sync(llx_session* s);
/* The session's CUDA stream (cudaStream_t), for event timing by the caller. */
void* llx_session_stream(llx_session* s);
/* Kernel launches per decode step (for launch accounting). */
int llx_decode_launches_per_step(llx_session* s);

/* Profiling. The plan's steps (one kernel each), and a per-step timing of the M=1 decode
 * plan at position pos: each step is launched alone `iters` times on the session stream,
 * each launch between two CUDA events after a 256 MB write that evicts the L2 (every step
 * is idempotent; the first 256 MB call allocates that buffer). Fills ms[i] (average per launch),
 * bytes[i] and ops[i] (algorithmic HBM bytes / integer ops of one launch) for up to n_max
 * steps plus the argmax kernel; *n_out = entries written. */
int llx_plan_steps(const llx_model* m);
const char* llx_step_label(const llx_model* m, int i);
llx_status llx_profile_decode(llx_session* s, int pos, int iters, float* ms, double* bytes, double* ops, int n_max,
                              int* n_out);

/* Named activations of the last launch (requires keep_acts=1 except for the output). */
int llx_activation_count(const llx_model* m);
const char* llx_activation_name(const llx_model* m, int i);
llx_status llx_activation_shape(const llx_model* m, const char* name, int* cols, int* elem_bytes);
llx_status llx_read_activation(llx_session* s, const char* name, void* dst, size_t bytes, int* rows_out);

const char* llx_last_error(void);
const char* llx_version(void);
/* Compute capability the library's kernels were compiled for, as loaded on `device`
 * (major * 10 + minor: 100 for sm_100a), from the CUDA runtime's function attributes.
 * No counterpart in the reference (it has no GPU code); lets a host check the build. */
llx_status llx_binary_version(int device, int* version);

/* Tensor parallelism over NCCL (NVLink / NVSwitch).  A tensor-parallel group is `world`
 * processes, one per GPU, each loading its rank graph (written by llaccel_b200.tp.shard:
 * column-split q/k/v/gate/up/lm_head, row-split o/down as int32 partial sums + all-reduce +
 * requant).  No counterpart in the reference, which runs one device; results stay bit for
 * bit those of the unsharded graph.  Rank 0 calls llx_tp_unique_id and shares the 128
 * bytes with the other ranks (e.g. over torch.distributed); then every rank calls
 * llx_tp_init on its loaded model (collective: blocks until all ranks joined) before it
 * creates its one session.  From then on every launch call (llx_run, llx_run_rows,
 * llx_generate, llx_decode_async, llx_profile_decode) is collective: all ranks make the
 * same calls with the same shapes, positions and output choices (logits outputs all-gather
 * the vocabulary shards).  Argmax outputs are global token ids on every rank.  The
 * communicator lives until llx_model_destroy; NCCL is loaded at run time (libnccl.so.2). */
#define LLX_TP_UNIQUE_ID_BYTES 128
llx_status llx_tp_unique_id(void* id);
llx_status llx_tp_init(llx_model* m, const void* id, int rank, int world);

/* Output projection with fused argmax that allocates no device memory.
 * No counterpart in the reference: it exists for callers that cannot call cudaMalloc --
 * code running inside another framework's memory pool, plugin hosts that only hand out
 * pre-sized buffers, processes that must not grow their device footprint after start-up.
 * The caller passes device buffers for everything: A [R][K] i8, W [N][K] i8, bias [N] i32
 * (may be NULL), rq [N][2] i32, logits [R][N] i16 (out), argmax [R] i32 (out, over the first
 * `vocab` channels, lowest index on ties).  Semantics are those of a qgraph linear with
 * epilogue none followed by the argmax of golden.py:376.  The per-row argmax keys use a
 * fixed file-scope device array of 4096 rows held by every GPU that loads the library until
 * exit: R > 4096 is rejected with LLX_ERR_RANGE, and so is K > 131056 (beyond it the int32
 * sums of K products of int8 values could wrap).  The call is synchronous on `stream`
 * (a cudaStream_t, NULL = default stream).  Its first call on a device looks up that
 * array's device address and sets kernel attributes, so make it before any stream capture.
 * All calls share the array: calls that overlap on the GPU race. */
llx_status llx_linear_argmax_noalloc(const int8_t* A, const int8_t* W, const int32_t* bias, const int32_t* rq, int R,
                                     int N, int K, int vocab, int16_t* logits, int32_t* argmax, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LLX_H */
