// mtp_nccl.cuh -- NCCL opened at run time, for hosts that drive the
// vocab-parallel verify through the C ABI without torch.distributed.
//
// The reference exchanges shard results through a torch process group
// (ParallelPrimitives, mtp_parallel.py:12-66).  A C or FFI host has no such
// group; it creates one NCCL communicator per rank (mtp_nccl_comm_init) and
// hands it to mtp_vocab_parallel_multi_verify, whose only collective is an
// all-reduce(MAX) of B*S int64 argmax keys.
//
// The library does not link NCCL: the first call that needs it dlopen()s
// "libnccl.so.2" (or the file named by MTP_NCCL_LIBRARY).  A process that
// already holds NCCL -- torch loads one -- gets that same copy back, so one
// NCCL serves the whole process.  Only the types and enum values come from
// nccl.h.
#pragma once

#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <stdlib.h>

#include <mutex>

namespace mtp {
namespace nccl {

struct Api {
  bool ok = false;
  int version = 0;
  char why[384] = "";
  ncclResult_t (*GetVersion)(int*) = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

template <typename F>
static inline bool bind(void* h, F& fn, const char* sym, Api& a) {
  fn = reinterpret_cast<F>(dlsym(h, sym));
  if (!fn) snprintf(a.why, sizeof(a.why), "NCCL library lacks %s", sym);
  return fn != nullptr;
}

// Loaded once per process; a failure is remembered (a.ok false, a.why set).
// Internal linkage: this header belongs to the library's one translation unit.
static inline const Api& api() {
  static Api a;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* env = getenv("MTP_NCCL_LIBRARY");
    const char* names[3] = {env, "libnccl.so.2", "libnccl.so"};
    void* h = nullptr;
    for (const char* n : names) {
      if (!n || !*n) continue;
      if ((h = dlopen(n, RTLD_NOW | RTLD_GLOBAL)) != nullptr) break;
      if (n == env) break;  // an explicit choice that fails is not replaced by another NCCL
    }
    if (!h) {
      const char* e = dlerror();
      snprintf(a.why, sizeof(a.why), "cannot open NCCL (%s): %s", env && *env ? env : "libnccl.so.2",
               e ? e : "not found");
      return;
    }
    bool all = bind(h, a.GetVersion, "ncclGetVersion", a) && bind(h, a.GetUniqueId, "ncclGetUniqueId", a) &&
               bind(h, a.CommInitRank, "ncclCommInitRank", a) && bind(h, a.CommDestroy, "ncclCommDestroy", a) &&
               bind(h, a.CommAbort, "ncclCommAbort", a) &&
               bind(h, a.CommGetAsyncError, "ncclCommGetAsyncError", a) &&
               bind(h, a.AllReduce, "ncclAllReduce", a) && bind(h, a.GetErrorString, "ncclGetErrorString", a);
    if (!all) return;
    if (a.GetVersion(&a.version) != ncclSuccess) {
      snprintf(a.why, sizeof(a.why), "ncclGetVersion failed");
      return;
    }
    a.ok = true;
  });
  return a;
}

static inline const char* error_string(ncclResult_t r) {
  const Api& a = api();
  return a.ok ? a.GetErrorString(r) : "NCCL not loaded";
}

// What one mtp_nccl_comm_init hands out: the NCCL communicator plus the
// rank layout the verify call checks its arguments against.
struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0;
  int world = 1;
  int device = -1;
};

}  // namespace nccl
}  // namespace mtp
