// nccl_dyn.cpp — NCCL for tensor parallelism, loaded on first use (dlopen),
// so the library itself needs no NCCL unless a model is loaded with
// tp_size > 1. Inside one process that already has NCCL loaded (e.g. by
// torch) the same library is reused.
#include "nccl_dyn.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace armai {
namespace {

struct NcclFns {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
  std::string why;
};

NcclFns& fns() {
  static NcclFns f;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      f.why = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    f.get_unique_id = (decltype(f.get_unique_id))dlsym(h, "ncclGetUniqueId");
    f.comm_init_rank = (decltype(f.comm_init_rank))dlsym(h, "ncclCommInitRank");
    f.all_reduce = (decltype(f.all_reduce))dlsym(h, "ncclAllReduce");
    f.all_gather = (decltype(f.all_gather))dlsym(h, "ncclAllGather");
    f.comm_destroy = (decltype(f.comm_destroy))dlsym(h, "ncclCommDestroy");
    f.comm_abort = (decltype(f.comm_abort))dlsym(h, "ncclCommAbort");
    f.error_string = (decltype(f.error_string))dlsym(h, "ncclGetErrorString");
    f.ok = f.get_unique_id && f.comm_init_rank && f.all_reduce && f.all_gather && f.comm_destroy &&
           f.comm_abort && f.error_string;
    if (!f.ok) f.why = "libnccl.so.2 lacks a required symbol";
  });
  return f;
}

int nccl_fail(ncclResult_t r, const char* what) {
  return fail(ARMAI_E_CUDA, std::string(what) + ": " + fns().error_string(r));
}

}  // namespace

int nccl_unique_id(void* out128) {
  NcclFns& f = fns();
  if (!f.ok) return fail(ARMAI_E_INVALID, f.why);
  ncclUniqueId id;
  const ncclResult_t r = f.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(out128, &id, sizeof id);
  return ARMAI_OK;
}

int nccl_comm_init(void** comm, int nranks, const void* id128, int rank) {
  NcclFns& f = fns();
  if (!f.ok) return fail(ARMAI_E_INVALID, f.why);
  ncclUniqueId id;
  std::memcpy(&id, id128, sizeof id);
  ncclComm_t c = nullptr;
  const ncclResult_t r = f.comm_init_rank(&c, nranks, id, rank);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
  *comm = c;
  return ARMAI_OK;
}

int nccl_allreduce_sum_f32(const float* send, float* recv, size_t n, void* comm, cudaStream_t s) {
  const ncclResult_t r = fns().all_reduce(send, recv, n, ncclFloat32, ncclSum, (ncclComm_t)comm, s);
  return r == ncclSuccess ? ARMAI_OK : nccl_fail(r, "ncclAllReduce");
}

int nccl_allgather_b32(const void* send, void* recv, size_t n_per_rank, void* comm, cudaStream_t s) {
  const ncclResult_t r = fns().all_gather(send, recv, n_per_rank, ncclUint32, (ncclComm_t)comm, s);
  return r == ncclSuccess ? ARMAI_OK : nccl_fail(r, "ncclAllGather");
}

void nccl_comm_destroy(void* comm) {
  if (comm && fns().ok) fns().comm_destroy((ncclComm_t)comm);
}

void nccl_comm_abort(void* comm) {
  if (comm && fns().ok) fns().comm_abort((ncclComm_t)comm);
}

}  // namespace armai
