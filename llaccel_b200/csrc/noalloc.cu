// llx_linear_argmax_noalloc: the output projection with fused argmax, for callers that
// cannot allocate device memory.
//
// Some callers of this library run where cudaMalloc is not available to them: code that
// lives inside another framework's memory pool or allocator, plugin hosts that hand out
// only pre-sized buffers, and processes that must not grow their device footprint after
// start-up.  The session API allocates its scratch (KV cache, activation arena, argmax
// keys) in llx_session_create; this entry point needs none of that.  The caller passes its
// own device buffers for every input and output; the only scratch the kernel needs -- one
// 64-bit argmax key per row plus a pipeline error word -- lives in the file-scope array
// below, which every GPU that loads the library holds until the process exits.
//
// The array is shared by every call on a device and keeps the last call's contents; the
// call clears the keys it uses before the GEMM.  Calls whose work overlaps on the GPU (for
// example from two host threads, or on two streams) race on the array.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/llx.h"
#include "kernels.h"

namespace llx {

// Rows per call (one argmax key each), plus one slot for the pipeline error word.
constexpr int kNoAllocMaxRows = 4096;
// The int32 tensor-core accumulators are exact while K * 128 * 128 < 2^31: the largest K
// (a multiple of 16) below 2^17.  Beyond it a sum could wrap and the argmax would be wrong.
constexpr int kNoAllocMaxK = 131056;
static __device__ __align__(256) unsigned long long g_noalloc_scratch[kNoAllocMaxRows + 1];

extern int g_pdl;
void noalloc_set_error(const std::string& msg);

namespace {

struct DeviceScratch {
  bool ready = false;
  unsigned long long* ptr = nullptr;
};
std::mutex g_setup_mu;
DeviceScratch g_dev[64];

// Once per device, with that device current: the device address of the scratch array.
// (In host code the array's name is only a host-side stand-in, never a device address.)
cudaError_t scratch_for_current_device(unsigned long long** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_dev[dev].ready) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_dev[dev].ptr = static_cast<unsigned long long*>(p);
    g_dev[dev].ready = true;
  }
  *out = g_dev[dev].ptr;
  return cudaSuccess;
}

}  // namespace
}  // namespace llx

using namespace llx;

extern "C" llx_status llx_linear_argmax_noalloc(const int8_t* A, const int8_t* W, const int32_t* bias,
                                                const int32_t* rq, int R, int N, int K, int vocab,
                                                int16_t* logits, int32_t* argmax, void* stream) {
  if (!A || !W || !rq || !logits || !argmax) {
    noalloc_set_error("llx_linear_argmax_noalloc: null pointer");
    return LLX_ERR_INVALID;
  }
  if (R < 1 || R > kNoAllocMaxRows) {
    noalloc_set_error("llx_linear_argmax_noalloc: R = " + std::to_string(R) + " rows exceeds the fixed scratch of " +
                      std::to_string(kNoAllocMaxRows) + " rows (or is < 1)");
    return LLX_ERR_RANGE;
  }
  if (K < 16 || K % 16 || N < 8 || N % 8 || vocab < 1 || vocab > N) {
    noalloc_set_error("llx_linear_argmax_noalloc: K must be a multiple of 16, N of 8, and 1 <= vocab <= N");
    return LLX_ERR_INVALID;
  }
  if (K > kNoAllocMaxK) {
    noalloc_set_error("llx_linear_argmax_noalloc: K = " + std::to_string(K) + " exceeds " +
                      std::to_string(kNoAllocMaxK) + ", the largest K whose int32 sums cannot wrap");
    return LLX_ERR_RANGE;
  }
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(logits)) & 15) {
    noalloc_set_error("llx_linear_argmax_noalloc: A, W and logits must be 16-byte aligned");
    return LLX_ERR_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned long long* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e == cudaSuccess) e = prepare_linear_tc();
  CUtensorMap map_a, map_w;
  const int nt = (N + 127) / 128 >= 64 ? 128 : 16;
  if (e == cudaSuccess) e = make_tmap_i8(&map_a, A, R, K, 128);
  if (e == cudaSuccess) e = make_tmap_i8(&map_w, W, N, K, nt);
  int32_t* fault = reinterpret_cast<int32_t*>(scratch + kNoAllocMaxRows);
  // keys start at zero for this call's rows; the error word too
  if (e == cudaSuccess) e = cudaMemsetAsync(scratch, 0, sizeof(unsigned long long) * R, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(fault, 0, sizeof(int32_t), st);
  if (e == cudaSuccess) {
    LinearArgs a{};
    a.A = A;
    a.W = W;
    a.bias = bias;
    a.rq = rq;
    a.out = logits;
    a.R = R;
    a.N = N;
    a.K = K;
    a.epi = EPI_NONE;
    a.narrow = 0;  // the bias range is not inspected: 64-bit bias add, exact for any int32 bias
    a.amax_key = scratch;
    a.amax_vocab = vocab;
    e = launch_linear_tc(map_a, map_w, a, nt, 1, fault, st);
  }
  if (e == cudaSuccess) e = launch_amax_finish(scratch, argmax, R, st);
  // the error word is read on the caller's stream (never the legacy default stream, which
  // would wait for every other blocking stream of the device), then that stream is drained
  int32_t f = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&f, fault, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    noalloc_set_error(std::string("llx_linear_argmax_noalloc: ") + cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? LLX_ERR_OOM : LLX_ERR_CUDA;
  }
  if (f) {
    noalloc_set_error("llx_linear_argmax_noalloc: a tensor-core pipeline wait timed out (code " + std::to_string(f) +
                      ")");
    return LLX_ERR_DEVICE;
  }
  return LLX_OK;
}
