// Vocabulary-sharded sampling over NCCL, and the communicator helpers.
//
// The reference samples every row whole on one CPU thread
// (ContinuousBatchingEngine::step, src/inference.rs:112-138); for a
// vocabulary split across devices, each rank streams only its columns and
// the ranks exchange one packed record per row (the shard's sorted top list
// and its softmax summary, 1056 bytes) with a single ncclAllGather, after
// which every rank merges the same records and draws the same token.
//
// NCCL is loaded at run time (dlopen): the one already in the process when
// there is one (a framework's), else libnccl.so.2 from the library path, or
// the file named by RL_NCCL_LIBRARY. Without NCCL these entry points return
// RL_ERR_UNSUPPORTED; nothing else of the library needs it.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"

static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");

namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommCount)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*CommUserRank)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

template <typename F>
bool sym(void* lib, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(lib, name));
  return *out != nullptr;
}

void load_nccl() {
  const char* path = std::getenv("RL_NCCL_LIBRARY");
  void* lib = nullptr;
  if (path && *path) {
    lib = dlopen(path, RTLD_NOW | RTLD_LOCAL);
  } else {
    lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the process's own NCCL
    if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  }
  if (!lib) return;
  NcclApi a;
  a.ok = sym(lib, "ncclGetUniqueId", &a.GetUniqueId) && sym(lib, "ncclCommInitRank", &a.CommInitRank) &&
         sym(lib, "ncclCommDestroy", &a.CommDestroy) && sym(lib, "ncclCommCount", &a.CommCount) &&
         sym(lib, "ncclCommUserRank", &a.CommUserRank) && sym(lib, "ncclAllGather", &a.AllGather) &&
         sym(lib, "ncclGetErrorString", &a.GetErrorString);
  if (a.ok) g_nccl = a;
}

const NcclApi* nccl() {
  std::call_once(g_nccl_once, load_nccl);
  return g_nccl.ok ? &g_nccl : nullptr;
}

thread_local char g_nerr[256];

rl_status nccl_fail(const NcclApi* n, ncclResult_t r, const char* what) {
  std::snprintf(g_nerr, sizeof(g_nerr), "%s: %s", what, n->GetErrorString(r));
  return rl::set_error(RL_ERR_NCCL, g_nerr);
}

}  // namespace

namespace rl {

// The collective step of rl_sample_sharded: every rank's send records
// ([B, kRec] u64) gathered into recv ([G, B, kRec]) on `stream`.
rl_status nccl_gather_records(void* comm, const uint64_t* send, uint64_t* recv, int B, int* G, cudaStream_t stream) {
  const NcclApi* n = nccl();
  if (!n) return set_error(RL_ERR_UNSUPPORTED, "rl_sample_sharded: NCCL could not be loaded");
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  ncclResult_t r = n->CommCount(c, G);
  if (r != ncclSuccess) return nccl_fail(n, r, "rl_sample_sharded: ncclCommCount");
  if (*G < 1 || *G > kMergeMaxShards) return set_error(RL_ERR_SHAPE, "rl_sample_sharded: more than 16 ranks");
  const size_t bytes = static_cast<size_t>(B) * kRec * sizeof(uint64_t);
  r = n->AllGather(send, recv, bytes, ncclInt8, c, stream);
  if (r != ncclSuccess) return nccl_fail(n, r, "rl_sample_sharded: ncclAllGather");
  return RL_OK;
}

}  // namespace rl

extern "C" {
#pragma GCC visibility push(default)

rl_status rl_nccl_unique_id(void* id_out) {
  rl::clear_error();
  if (!id_out) return rl::set_error(RL_ERR_INVALID_ARG, "rl_nccl_unique_id: id_out is NULL");
  const NcclApi* n = nccl();
  if (!n) return rl::set_error(RL_ERR_UNSUPPORTED, "rl_nccl_unique_id: NCCL could not be loaded");
  ncclUniqueId id;
  const ncclResult_t r = n->GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(n, r, "rl_nccl_unique_id: ncclGetUniqueId");
  std::memcpy(id_out, &id, sizeof(id));
  return RL_OK;
}

rl_status rl_nccl_comm_init(void** comm_out, int nranks, const void* id, int rank) {
  rl::clear_error();
  if (!comm_out || !id) return rl::set_error(RL_ERR_INVALID_ARG, "rl_nccl_comm_init: NULL pointer");
  *comm_out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_nccl_comm_init: rank outside [0, nranks)");
  const NcclApi* n = nccl();
  if (!n) return rl::set_error(RL_ERR_UNSUPPORTED, "rl_nccl_comm_init: NCCL could not be loaded");
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  const ncclResult_t r = n->CommInitRank(&c, nranks, uid, rank);
  if (r != ncclSuccess) return nccl_fail(n, r, "rl_nccl_comm_init: ncclCommInitRank");
  *comm_out = c;
  return RL_OK;
}

rl_status rl_nccl_comm_destroy(void* comm) {
  rl::clear_error();
  if (!comm) return RL_OK;
  const NcclApi* n = nccl();
  if (!n) return rl::set_error(RL_ERR_UNSUPPORTED, "rl_nccl_comm_destroy: NCCL could not be loaded");
  const ncclResult_t r = n->CommDestroy(static_cast<ncclComm_t>(comm));
  if (r != ncclSuccess) return nccl_fail(n, r, "rl_nccl_comm_destroy: ncclCommDestroy");
  return RL_OK;
}

#pragma GCC visibility pop
}  // extern "C"
