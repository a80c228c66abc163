// comm.cu — the optional all-gather of sharded outputs over NVLink/NVSwitch.
//
// The units of this path are independent (GEMM output rows, attention (batch, KV head)
// groups), so every rank computes its shard with no collective; a caller that wants the
// whole output on every GPU gathers the shards afterwards. Python hosts have
// torch.distributed for that; this file gives the same step to hosts that only have the C
// ABI (the Julia package): an NCCL communicator over the ranks of one box and one
// all-gather of equal byte ranges.
//
// NCCL is opened at first use (dlopen of libnccl.so.2), so liblvb loads and runs its kernels
// on a machine without NCCL; a missing library or symbol is reported as LVB_ERR_NCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "lvb_internal.h"

struct lvb_comm {
  ncclComm_t comm;
  int nranks;
  int rank;
  int device;
};

namespace lvb {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
  std::string why;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    // A process that already loaded NCCL (torch does) gets that copy back from dlopen.
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      api.why = std::string("cannot open libnccl.so.2: ") + (e ? e : "unknown error");
      return;
    }
    auto get = [&](const char* name) -> void* {
      void* f = dlsym(h, name);
      if (!f && api.why.empty()) api.why = std::string("libnccl has no symbol ") + name;
      return f;
    };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(get("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(get("ncclCommInitRank"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(get("ncclAllGather"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(get("ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(get("ncclGetErrorString"));
    api.ok = api.why.empty();
  });
  return api;
}

int fail_nccl(const char* op, const char* call, ncclResult_t r) {
  const NcclApi& a = nccl();
  std::string msg = std::string(call) + " failed (" + std::to_string((int)r) + ")";
  if (a.error_string) msg += std::string(": ") + a.error_string(r);
  return fail(LVB_ERR_NCCL, op, msg);
}

int need_nccl(const char* op) {
  const NcclApi& a = nccl();
  if (a.ok) return LVB_OK;
  return fail(LVB_ERR_NCCL, op, a.why, "install NCCL 2.x (libnccl.so.2) on the library path");
}

}  // namespace
}  // namespace lvb

using namespace lvb;

static_assert(sizeof(lvb_comm_id) == sizeof(ncclUniqueId), "id size");

extern "C" int lvb_comm_unique_id(lvb_comm_id* id) {
  const char* op = "lvb_comm_unique_id";
  if (!id) return fail(LVB_ERR_INVALID_ARG, op, "id is null");
  if (int st = need_nccl(op)) return st;
  ncclUniqueId u;
  ncclResult_t r = nccl().get_unique_id(&u);
  if (r != ncclSuccess) return fail_nccl(op, "ncclGetUniqueId", r);
  std::memcpy(id->bytes, &u, sizeof u);
  return LVB_OK;
}

extern "C" int lvb_comm_init(lvb_comm** comm, const lvb_comm_id* id, int32_t nranks,
                             int32_t rank) {
  const char* op = "lvb_comm_init";
  if (!comm || !id) return fail(LVB_ERR_INVALID_ARG, op, "comm or id is null");
  *comm = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return fail(LVB_ERR_INVALID_ARG, op,
                "need 0 <= rank < nranks (rank " + std::to_string(rank) + ", nranks " +
                    std::to_string(nranks) + ")");
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return fail_cuda(e, op, "cudaGetDevice");
  if (int st = need_nccl(op)) return st;
  ncclUniqueId u;
  std::memcpy(&u, id->bytes, sizeof u);
  ncclComm_t c = nullptr;
  ncclResult_t r = nccl().comm_init_rank(&c, nranks, u, rank);
  if (r != ncclSuccess) return fail_nccl(op, "ncclCommInitRank", r);
  *comm = new lvb_comm{c, nranks, rank, device};
  return LVB_OK;
}

extern "C" int lvb_comm_destroy(lvb_comm* comm) {
  const char* op = "lvb_comm_destroy";
  if (!comm) return LVB_OK;
  if (int st = need_nccl(op)) return st;
  ncclResult_t r = nccl().comm_destroy(comm->comm);
  delete comm;
  if (r != ncclSuccess) return fail_nccl(op, "ncclCommDestroy", r);
  return LVB_OK;
}

extern "C" int lvb_comm_size(const lvb_comm* comm, int32_t* nranks, int32_t* rank) {
  if (!comm || !nranks || !rank) return fail(LVB_ERR_INVALID_ARG, "lvb_comm_size", "null argument");
  *nranks = comm->nranks;
  *rank = comm->rank;
  return LVB_OK;
}

extern "C" int lvb_allgather(lvb_comm* comm, const void* send, void* recv, size_t bytes,
                             void* stream) {
  const char* op = "lvb_allgather";
  if (!comm) return fail(LVB_ERR_INVALID_ARG, op, "comm is null");
  if (bytes == 0) return LVB_OK;
  if (!send || !recv) return fail(LVB_ERR_INVALID_ARG, op, "send or recv is null");
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return fail_cuda(e, op, "cudaGetDevice");
  if (device != comm->device)
    return fail(LVB_ERR_INVALID_ARG, op,
                "the current device (" + std::to_string(device) +
                    ") is not the communicator's (" + std::to_string(comm->device) + ")");
  // In place when send is recv's own slot: NCCL reads and writes the same bytes.
  ncclResult_t r = nccl().all_gather(send, recv, bytes, ncclUint8, comm->comm,
                                     static_cast<cudaStream_t>(stream));
  if (r != ncclSuccess) return fail_nccl(op, "ncclAllGather", r);
  return LVB_OK;
}
