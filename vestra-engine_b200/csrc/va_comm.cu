// NCCL plumbing for query-sharded global attention (one process per GPU).
//
// The reference has no multi-GPU code at all (one CudaRuntime per device,
// engine.rs:288); this is the new exchange step of the global blocks: every rank
// produces K'/V for its own contiguous slice of the view-major window in place
// inside a window-sized buffer, and one grouped in-place all-gather fills in the
// other ranks' slices before the fused attention reads the whole window.
//
// NCCL is opened with dlopen at communicator creation, so the library loads and
// runs single-GPU without it; in a PyTorch process the already loaded libnccl is
// reused.  VA_NCCL_LIB overrides the library name.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "va_comm.h"

namespace va {

namespace {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  std::string error;
};

NcclApi g_api;
std::once_flag g_once;

template <class F>
bool sym(void* h, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(h, name));
  return *out != nullptr;
}

const NcclApi* api() {
  std::call_once(g_once, [] {
    const char* env = std::getenv("VA_NCCL_LIB");
    const char* names[] = {env, "libnccl.so.2", "libnccl.so"};
    for (const char* n : names) {
      if (!n) continue;
      g_api.handle = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
      if (g_api.handle) break;
    }
    if (!g_api.handle) {
      g_api.error = "cannot dlopen libnccl.so.2 (set VA_NCCL_LIB)";
      return;
    }
    void* h = g_api.handle;
    const bool ok = sym(h, "ncclGetUniqueId", &g_api.GetUniqueId) &&
                    sym(h, "ncclCommInitRank", &g_api.CommInitRank) &&
                    sym(h, "ncclCommDestroy", &g_api.CommDestroy) &&
                    sym(h, "ncclCommAbort", &g_api.CommAbort) &&
                    sym(h, "ncclAllGather", &g_api.AllGather) &&
                    sym(h, "ncclGroupStart", &g_api.GroupStart) &&
                    sym(h, "ncclGroupEnd", &g_api.GroupEnd) &&
                    sym(h, "ncclCommGetAsyncError", &g_api.CommGetAsyncError) &&
                    sym(h, "ncclGetErrorString", &g_api.GetErrorString);
    if (!ok) g_api.error = "libnccl is missing an entry point";
  });
  return g_api.error.empty() ? &g_api : nullptr;
}

std::string nccl_msg(const NcclApi* a, ncclResult_t r, const char* what) {
  return std::string(what) + ": " + (a ? a->GetErrorString(r) : "nccl unavailable");
}

}  // namespace

struct Comm {
  ncclComm_t comm = nullptr;
  int nranks = 0;
  int rank = 0;
};

bool comm_unique_id(void* out128, std::string* err) {
  const NcclApi* a = api();
  if (!a) {
    *err = g_api.error;
    return false;
  }
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId must be 128 bytes");
  ncclUniqueId id;
  const ncclResult_t r = a->GetUniqueId(&id);
  if (r != ncclSuccess) {
    *err = nccl_msg(a, r, "ncclGetUniqueId");
    return false;
  }
  std::memcpy(out128, &id, sizeof(id));
  return true;
}

Comm* comm_init(const void* id128, int nranks, int rank, std::string* err) {
  const NcclApi* a = api();
  if (!a) {
    *err = g_api.error;
    return nullptr;
  }
  ncclUniqueId id;
  std::memcpy(&id, id128, sizeof(id));
  Comm* c = new Comm();
  const ncclResult_t r = a->CommInitRank(&c->comm, nranks, id, rank);
  if (r != ncclSuccess) {
    *err = nccl_msg(a, r, "ncclCommInitRank");
    delete c;
    return nullptr;
  }
  c->nranks = nranks;
  c->rank = rank;
  return c;
}

void comm_destroy(Comm* c, bool abort) {
  if (!c) return;
  const NcclApi* a = api();
  if (a && c->comm) (abort ? a->CommAbort : a->CommDestroy)(c->comm);
  delete c;
}

int comm_rank(const Comm* c) { return c->rank; }
int comm_size(const Comm* c) { return c->nranks; }

bool comm_allgather_inplace2(Comm* c, void* buf_a, void* buf_b, size_t count_per_rank,
                             cudaStream_t st, std::string* err) {
  const NcclApi* a = api();
  if (!a) {
    *err = g_api.error;
    return false;
  }
  const size_t bytes = count_per_rank * 2;  // bf16
  char* pa = static_cast<char*>(buf_a);
  char* pb = static_cast<char*>(buf_b);
  ncclResult_t r = a->GroupStart();
  if (r == ncclSuccess)
    r = a->AllGather(pa + c->rank * bytes, pa, count_per_rank, ncclBfloat16, c->comm, st);
  if (r == ncclSuccess)
    r = a->AllGather(pb + c->rank * bytes, pb, count_per_rank, ncclBfloat16, c->comm, st);
  const ncclResult_t r2 = a->GroupEnd();
  if (r == ncclSuccess) r = r2;
  if (r != ncclSuccess) {
    *err = nccl_msg(a, r, "ncclAllGather");
    return false;
  }
  return true;
}

bool comm_allgather_bytes(Comm* c, const void* send, void* recv, size_t bytes, cudaStream_t st,
                          std::string* err) {
  const NcclApi* a = api();
  if (!a) {
    *err = g_api.error;
    return false;
  }
  const ncclResult_t r = a->AllGather(send, recv, bytes, ncclUint8, c->comm, st);
  if (r != ncclSuccess) {
    *err = nccl_msg(a, r, "ncclAllGather");
    return false;
  }
  return true;
}

bool comm_async_error(Comm* c, std::string* err) {
  const NcclApi* a = api();
  if (!a || !c) return false;
  ncclResult_t st = ncclSuccess;
  if (a->CommGetAsyncError(c->comm, &st) != ncclSuccess || (st != ncclSuccess && st != ncclInProgress)) {
    *err = nccl_msg(a, st, "nccl async error");
    return true;
  }
  return false;
}

}  // namespace va
