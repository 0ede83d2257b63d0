// Tensor-parallel communicator (NCCL, loaded at run time).  Each call returns false and
// fills *err on failure.  Collectives are enqueued on `st` and may be captured into a
// CUDA graph; every rank must issue the same collectives in the same order.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <string>

namespace llx {

constexpr int kTpUniqueIdBytes = 128;

struct TpComm;

bool tp_unique_id(void* out /* kTpUniqueIdBytes */, std::string* err);
TpComm* tp_comm_create(const void* id, int rank, int world, int device, std::string* err);
void tp_comm_destroy(TpComm* c);
int tp_world(const TpComm* c);
int tp_rank(const TpComm* c);

bool tp_allreduce_sum_i32(TpComm* c, int32_t* buf, size_t n, cudaStream_t st, std::string* err);
bool tp_allreduce_max_u64(TpComm* c, unsigned long long* buf, size_t n, cudaStream_t st, std::string* err);
bool tp_allgather_bytes(TpComm* c, const void* send, void* recv, size_t bytes, cudaStream_t st, std::string* err);
// true when the communicator holds an asynchronous error (message in *err)
bool tp_async_error(TpComm* c, std::string* err);

}  // namespace llx
