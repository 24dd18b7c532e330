// pw_nccl.cu -- NCCL, loaded on first use.
//
// The library does not link NCCL: pw_ep_init dlopens libnccl.so.2 (inside a
// process that already loaded NCCL, e.g. through torch, the loaded copy is
// reused) so that single-GPU users need no NCCL at all.  Communicators are
// created non-blocking; every wait on them is bounded by the caller's
// deadline and ends in ncclCommAbort.
#include <dlfcn.h>

#include <chrono>
#include <mutex>
#include <string>
#include <thread>

#include "pw_internal.h"

namespace pw {
namespace nccl {
namespace {

struct Api {
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

Api g_api;
bool g_loaded = false;
std::mutex g_mu;

template <typename F>
bool sym(void *h, const char *name, F &out) {
  out = reinterpret_cast<F>(dlsym(h, name));
  return out != nullptr;
}

}  // namespace

bool load(std::string &err) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_loaded) return true;
  void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    err = std::string("cannot load NCCL: ") + dlerror();
    return false;
  }
  Api a;
  bool ok = sym(h, "ncclGetUniqueId", a.GetUniqueId) && sym(h, "ncclCommInitRankConfig", a.CommInitRankConfig) &&
            sym(h, "ncclCommGetAsyncError", a.CommGetAsyncError) && sym(h, "ncclCommAbort", a.CommAbort) &&
            sym(h, "ncclCommFinalize", a.CommFinalize) && sym(h, "ncclCommDestroy", a.CommDestroy) &&
            sym(h, "ncclAllGather", a.AllGather) && sym(h, "ncclSend", a.Send) && sym(h, "ncclRecv", a.Recv) &&
            sym(h, "ncclGroupStart", a.GroupStart) && sym(h, "ncclGroupEnd", a.GroupEnd) &&
            sym(h, "ncclGetErrorString", a.GetErrorString);
  if (!ok) {
    err = "NCCL is missing an entry point this build needs (ncclCommInitRankConfig, ncclSend, ...)";
    return false;
  }
  g_api = a;
  g_loaded = true;
  return true;
}

const char *error_string(ncclResult_t r) { return g_loaded ? g_api.GetErrorString(r) : "NCCL not loaded"; }

ncclResult_t unique_id(ncclUniqueId *id) { return g_api.GetUniqueId(id); }

// Waits until the communicator has no operation in progress (non-blocking
// mode), the deadline passes, or it reports an error.
static ncclResult_t settle(ncclComm_t comm, ncclResult_t first, double deadline_s) {
  if (first != ncclInProgress) return first;
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t q = g_api.CommGetAsyncError(comm, &st);
    if (q != ncclSuccess) return q;
    if (st != ncclInProgress) return st;
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > deadline_s) return ncclInProgress;  // caller aborts
    if (el > 2e-3) std::this_thread::sleep_for(std::chrono::microseconds(50));
    else std::this_thread::yield();
  }
}

ncclResult_t init_rank(ncclComm_t *comm, int world, const ncclUniqueId &id, int rank, double deadline_s) {
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  *comm = nullptr;
  ncclResult_t r = g_api.CommInitRankConfig(comm, world, id, rank, &cfg);
  if (*comm == nullptr) return r == ncclSuccess ? ncclInternalError : r;
  return settle(*comm, r, deadline_s);
}

ncclResult_t async_error(ncclComm_t comm) {
  ncclResult_t st = ncclSuccess;
  ncclResult_t q = g_api.CommGetAsyncError(comm, &st);
  return q != ncclSuccess ? q : st;
}

// Abort on a detached thread: ncclCommAbort waits for the communicator's
// background work, which may itself be waiting on a peer that is gone; the
// caller must get its error back within its deadline regardless.
void abort_comm(ncclComm_t comm) {
  if (!comm || !g_loaded) return;
  std::thread([comm]() { g_api.CommAbort(comm); }).detach();
}

ncclResult_t destroy(ncclComm_t comm, double deadline_s) {
  if (!comm) return ncclSuccess;
  ncclResult_t r = settle(comm, g_api.CommFinalize(comm), deadline_s);
  if (r != ncclSuccess) {
    abort_comm(comm);
    return r;
  }
  return g_api.CommDestroy(comm);
}

ncclResult_t all_gather(const void *send, void *recv, size_t count, ncclDataType_t t, ncclComm_t comm,
                        cudaStream_t s, double deadline_s) {
  return settle(comm, g_api.AllGather(send, recv, count, t, comm, s), deadline_s);
}

ncclResult_t exchange(const Transfer *sends, int n_sends, const Transfer *recvs, int n_recvs, ncclComm_t comm,
                      cudaStream_t s, double deadline_s) {
  ncclResult_t r = g_api.GroupStart();
  if (r != ncclSuccess) return r;
  for (int i = 0; i < n_sends && (r == ncclSuccess || r == ncclInProgress); ++i)
    if (sends[i].bytes) r = g_api.Send(sends[i].ptr, sends[i].bytes, ncclUint8, sends[i].peer, comm, s);
  for (int i = 0; i < n_recvs && (r == ncclSuccess || r == ncclInProgress); ++i)
    if (recvs[i].bytes)
      r = g_api.Recv(const_cast<void *>(recvs[i].ptr), recvs[i].bytes, ncclUint8, recvs[i].peer, comm, s);
  ncclResult_t e = g_api.GroupEnd();
  if (r != ncclSuccess && r != ncclInProgress) return r;
  return settle(comm, e, deadline_s);
}

}  // namespace nccl
}  // namespace pw
