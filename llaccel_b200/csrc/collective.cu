// Tensor-parallel collectives over NCCL (NVLink / NVSwitch), loaded at run time.
//
// libnccl is opened with dlopen on first use, so the library carries no link-time NCCL
// dependency and a process that already loaded NCCL (a PyTorch process) shares that copy
// (dlopen by soname returns the loaded object).  Three collectives serve the integer
// datapath, all exact:
//   * int32 sum of the row-split linears' partial accumulators (integer addition is
//     associative, and |sum| < 2^31 for K * 128 * 128 < 2^31);
//   * uint64 max of the packed argmax keys (logit, inverted global index) of the
//     vocabulary shards -- the max key is the global first maximum;
//   * all-gather of the vocabulary shards of the logits, when the caller asks for logits.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>

#include "collective.h"

namespace llx {

namespace {

struct NcclApi {
  bool tried = false, ok = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

std::mutex g_mu;
NcclApi g_api;

template <class F>
bool sym(void* h, const char* name, F** out) {
  *out = reinterpret_cast<F*>(dlsym(h, name));
  return *out != nullptr;
}

const NcclApi* api(std::string* err) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_api.tried) {
    g_api.tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      const char* e = dlerror();
      g_api.why = std::string("cannot load libnccl.so.2: ") + (e ? e : "not found");
    } else if (!sym(h, "ncclGetUniqueId", &g_api.GetUniqueId) || !sym(h, "ncclCommInitRank", &g_api.CommInitRank) ||
               !sym(h, "ncclCommDestroy", &g_api.CommDestroy) ||
               !sym(h, "ncclCommGetAsyncError", &g_api.CommGetAsyncError) ||
               !sym(h, "ncclAllReduce", &g_api.AllReduce) || !sym(h, "ncclAllGather", &g_api.AllGather) ||
               !sym(h, "ncclGetErrorString", &g_api.GetErrorString)) {
      g_api.why = "libnccl.so.2 lacks an expected symbol";
    } else {
      g_api.ok = true;
    }
  }
  if (!g_api.ok) {
    *err = g_api.why;
    return nullptr;
  }
  return &g_api;
}

bool check(const NcclApi* a, ncclResult_t r, const char* what, std::string* err) {
  if (r == ncclSuccess) return true;
  *err = std::string(what) + ": " + a->GetErrorString(r);
  return false;
}

}  // namespace

struct TpComm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
};

bool tp_unique_id(void* out, std::string* err) {
  const NcclApi* a = api(err);
  if (!a) return false;
  ncclUniqueId id;
  if (!check(a, a->GetUniqueId(&id), "ncclGetUniqueId", err)) return false;
  static_assert(sizeof(id) == kTpUniqueIdBytes, "NCCL unique id size");
  memcpy(out, &id, sizeof(id));
  return true;
}

TpComm* tp_comm_create(const void* id, int rank, int world, int device, std::string* err) {
  const NcclApi* a = api(err);
  if (!a) return nullptr;
  if (cudaSetDevice(device) != cudaSuccess) {
    *err = "cudaSetDevice failed";
    return nullptr;
  }
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  TpComm* c = new TpComm;
  c->rank = rank;
  c->world = world;
  c->device = device;
  if (!check(a, a->CommInitRank(&c->comm, world, uid, rank), "ncclCommInitRank", err)) {
    delete c;
    return nullptr;
  }
  return c;
}

void tp_comm_destroy(TpComm* c) {
  if (!c) return;
  std::string err;
  const NcclApi* a = api(&err);
  if (a && c->comm) {
    cudaSetDevice(c->device);
    a->CommDestroy(c->comm);
  }
  delete c;
}

int tp_world(const TpComm* c) { return c ? c->world : 1; }
int tp_rank(const TpComm* c) { return c ? c->rank : 0; }

bool tp_allreduce_sum_i32(TpComm* c, int32_t* buf, size_t n, cudaStream_t st, std::string* err) {
  const NcclApi* a = api(err);
  return a && check(a, a->AllReduce(buf, buf, n, ncclInt32, ncclSum, c->comm, st), "ncclAllReduce(int32 sum)", err);
}

bool tp_allreduce_max_u64(TpComm* c, unsigned long long* buf, size_t n, cudaStream_t st, std::string* err) {
  const NcclApi* a = api(err);
  return a && check(a, a->AllReduce(buf, buf, n, ncclUint64, ncclMax, c->comm, st), "ncclAllReduce(uint64 max)", err);
}

bool tp_allgather_bytes(TpComm* c, const void* send, void* recv, size_t bytes, cudaStream_t st, std::string* err) {
  const NcclApi* a = api(err);
  return a && check(a, a->AllGather(send, recv, bytes, ncclUint8, c->comm, st), "ncclAllGather", err);
}

bool tp_async_error(TpComm* c, std::string* err) {
  const NcclApi* a = api(err);
  if (!a) return true;
  ncclResult_t r = ncclSuccess;
  if (a->CommGetAsyncError(c->comm, &r) != ncclSuccess) {
    *err = "ncclCommGetAsyncError failed";
    return true;
  }
  if (r != ncclSuccess && r != ncclInProgress) {
    *err = std::string("NCCL communicator error: ") + a->GetErrorString(r);
    return true;
  }
  return false;
}

}  // namespace llx
