// Cross-GPU block migration over NCCL (NVLink / NVSwitch).
//
// The reference has no multi-GPU KV path (its distributed crates are never
// enabled).  With the pool sharded by KV head the per-step append, gather,
// quantisation and copy-on-write need no collective; moving blocks between
// pools on different GPUs (rebalancing sequences between data-parallel
// groups, or re-sharding) is the one exchange.  It is done as
//   pack (copy_blocks_kernel, pool -> local staging)
//   -> grouped ncclSend / ncclRecv between the two ranks
//   -> unpack (staging -> pool)
// all on one stream.  No kernel reads a peer's memory, and nothing here uses
// TMA multicast.
//
// Communicators are created non-blocking, and every wait on NCCL is a
// bounded poll: when the deadline passes the communicator is aborted and the
// call returns RMLX_E_TIMEOUT, so a peer that never posts its half of the
// exchange surfaces as an error rather than a hang.
//
// NCCL is resolved at first use with dlopen("libnccl.so.2") instead of being
// linked: a process that already loaded an NCCL (PyTorch loads its own) gets
// that same copy, so loading this library first cannot pin a different NCCL
// under the shared soname.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>

#include "device_common.cuh"

using rmlx::cuda_check;
using rmlx::DeviceGuard;
using rmlx::fail;

struct rmlx_comm {
  ncclComm_t comm = nullptr;
  int device = 0;
  int nranks = 0, rank = 0;
  int timeout_ms = 0;
  bool aborted = false;
};

namespace {

using Clock = std::chrono::steady_clock;

// The NCCL entry points this file uses, resolved from the process's NCCL.
struct NcclApi {
  bool ok = false;
  char why[256] = {0};
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommFinalize)(ncclComm_t);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      snprintf(api.why, sizeof(api.why), "cannot load libnccl.so.2: %s", dlerror());
      return;
    }
    bool all = true;
    auto sym = [&](const char* name) {
      void* f = dlsym(h, name);
      if (!f) all = false;
      return f;
    };
    api.GetUniqueId = (decltype(api.GetUniqueId))sym("ncclGetUniqueId");
    api.CommInitRankConfig = (decltype(api.CommInitRankConfig))sym("ncclCommInitRankConfig");
    api.CommGetAsyncError = (decltype(api.CommGetAsyncError))sym("ncclCommGetAsyncError");
    api.CommAbort = (decltype(api.CommAbort))sym("ncclCommAbort");
    api.CommFinalize = (decltype(api.CommFinalize))sym("ncclCommFinalize");
    api.CommDestroy = (decltype(api.CommDestroy))sym("ncclCommDestroy");
    api.GroupStart = (decltype(api.GroupStart))sym("ncclGroupStart");
    api.GroupEnd = (decltype(api.GroupEnd))sym("ncclGroupEnd");
    api.Send = (decltype(api.Send))sym("ncclSend");
    api.Recv = (decltype(api.Recv))sym("ncclRecv");
    api.GetErrorString = (decltype(api.GetErrorString))sym("ncclGetErrorString");
    if (!all) {
      snprintf(api.why, sizeof(api.why), "libnccl.so.2 lacks an entry point this library needs");
      return;
    }
    api.ok = true;
  });
  return api;
}

rmlx_status nccl_fail(ncclResult_t r, const char* what) {
  return fail(RMLX_E_NCCL, "%s: %s", what, nccl().GetErrorString(r));
}

rmlx_status need_nccl() {
  return nccl().ok ? RMLX_OK : fail(RMLX_E_NCCL, "%s", nccl().why);
}

// Poll the communicator until it leaves ncclInProgress or the deadline
// passes (then abort it).
rmlx_status settle(rmlx_comm* c, ncclResult_t r, const char* what, int timeout_ms) {
  const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
  while (r == ncclInProgress) {
    if (Clock::now() > deadline) {
      nccl().CommAbort(c->comm);
      c->aborted = true;
      return fail(RMLX_E_TIMEOUT, "%s: no progress within %d ms (communicator aborted)", what, timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
    nccl().CommGetAsyncError(c->comm, &r);
  }
  return r == ncclSuccess ? RMLX_OK : nccl_fail(r, what);
}

}  // namespace

extern "C" {

rmlx_status rmlx_nccl_unique_id(uint8_t* out) {
  if (!out) return fail(RMLX_E_BAD_ARG, "NULL out");
  if (rmlx_status s = need_nccl()) return s;
  ncclUniqueId id;
  ncclResult_t r = nccl().GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
  return RMLX_OK;
}

rmlx_status rmlx_nccl_comm_new(int32_t nranks, const uint8_t* id, int32_t rank, int device, int32_t timeout_ms,
                               rmlx_comm** out) {
  if (!id || !out) return fail(RMLX_E_BAD_ARG, "NULL id or out");
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(RMLX_E_BAD_ARG, "rank %d outside [0, %d)", rank, nranks);
  if (timeout_ms <= 0) return fail(RMLX_E_BAD_ARG, "timeout_ms must be > 0");
  if (rmlx_status s = need_nccl()) return s;
  *out = nullptr;
  rmlx_comm* c = new (std::nothrow) rmlx_comm();
  if (!c) return fail(RMLX_E_EXHAUSTED, "host allocation failed");
  c->device = device;
  c->nranks = nranks;
  c->rank = rank;
  c->timeout_ms = timeout_ms;
  DeviceGuard dg(device);
  ncclUniqueId uid;
  memcpy(uid.internal, id, NCCL_UNIQUE_ID_BYTES);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = nccl().CommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete c;
    return nccl_fail(r, "ncclCommInitRankConfig");
  }
  rmlx_status s = settle(c, r, "ncclCommInitRankConfig", timeout_ms);
  if (s != RMLX_OK) {
    if (!c->aborted) nccl().CommAbort(c->comm);
    delete c;
    return s;
  }
  *out = c;
  return RMLX_OK;
}

void rmlx_nccl_comm_destroy(rmlx_comm* c) {
  if (!c) return;
  if (!c->aborted && c->comm) {
    DeviceGuard dg(c->device);
    nccl().CommFinalize(c->comm);
    ncclResult_t r = ncclInProgress;
    const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
    while (r == ncclInProgress && Clock::now() < deadline) {
      nccl().CommGetAsyncError(c->comm, &r);
      if (r == ncclInProgress) std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
    if (r == ncclSuccess) nccl().CommDestroy(c->comm);
    else nccl().CommAbort(c->comm);
  }
  delete c;
}

rmlx_status rmlx_kv_migrate(rmlx_kv_pool* p, rmlx_comm* c, int32_t peer, const int32_t* send_ids, int32_t n_send,
                            void* send_staging, const int32_t* recv_ids, int32_t n_recv, void* recv_staging,
                            void* stream) {
  if (!p || !c) return fail(RMLX_E_BAD_ARG, "NULL pool or communicator");
  if (c->aborted) return fail(RMLX_E_NCCL, "communicator was aborted");
  if (peer < 0 || peer >= c->nranks || peer == c->rank)
    return fail(RMLX_E_BAD_ARG, "peer %d is not another rank of %d", peer, c->nranks);
  if (n_send < 0 || n_recv < 0) return fail(RMLX_E_BAD_ARG, "negative block count");
  rmlx_pool_layout lay;
  rmlx_status s = rmlx_kv_pool_layout(p, &lay);
  if (s != RMLX_OK) return s;
  DeviceGuard dg(c->device);
  // pack
  if (n_send > 0 && (s = rmlx_kv_pack_blocks(p, send_ids, n_send, send_staging, stream)) != RMLX_OK) return s;
  // exchange
  ncclResult_t r = nccl().GroupStart();
  if (r != ncclSuccess) return nccl_fail(r, "ncclGroupStart");
  if (n_send > 0) {
    r = nccl().Send(send_staging, (size_t)n_send * lay.block_bytes, ncclUint8, peer, c->comm, (cudaStream_t)stream);
    if (r != ncclSuccess && r != ncclInProgress) {
      nccl().GroupEnd();
      return nccl_fail(r, "ncclSend");
    }
  }
  if (n_recv > 0) {
    r = nccl().Recv(recv_staging, (size_t)n_recv * lay.block_bytes, ncclUint8, peer, c->comm, (cudaStream_t)stream);
    if (r != ncclSuccess && r != ncclInProgress) {
      nccl().GroupEnd();
      return nccl_fail(r, "ncclRecv");
    }
  }
  r = nccl().GroupEnd();
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclGroupEnd");
  // The unpack must be enqueued after NCCL has enqueued the receive.
  if ((s = settle(c, r, "ncclGroupEnd", c->timeout_ms)) != RMLX_OK) return s;
  if (n_recv > 0 && (s = rmlx_kv_unpack_blocks(p, recv_ids, n_recv, recv_staging, stream)) != RMLX_OK) return s;
  return RMLX_OK;
}

rmlx_status rmlx_nccl_wait(rmlx_comm* c, void* stream, int32_t timeout_ms) {
  if (!c) return fail(RMLX_E_BAD_ARG, "NULL communicator");
  if (c->aborted) return fail(RMLX_E_NCCL, "communicator was aborted");
  DeviceGuard dg(c->device);
  const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : c->timeout_ms);
  for (;;) {
    cudaError_t e = cudaStreamQuery((cudaStream_t)stream);
    if (e == cudaSuccess) return RMLX_OK;
    if (e != cudaErrorNotReady) return cuda_check(e, "cudaStreamQuery");
    ncclResult_t r = ncclSuccess;
    nccl().CommGetAsyncError(c->comm, &r);
    if (r != ncclSuccess && r != ncclInProgress) {
      nccl().CommAbort(c->comm);
      c->aborted = true;
      return nccl_fail(r, "NCCL asynchronous error (communicator aborted)");
    }
    if (Clock::now() > deadline) {
      nccl().CommAbort(c->comm);
      c->aborted = true;
      return fail(RMLX_E_TIMEOUT, "stream not done within the deadline (communicator aborted)");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // extern "C"
