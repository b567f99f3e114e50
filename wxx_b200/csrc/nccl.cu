// NCCL plumbing for batch-sharded inference: one communicator per process
// (one process per GPU), an all-gather of per-rank outputs over NVLink /
// NVSwitch on the library stream.  The reference has no collectives; this is
// the only exchange step of the sharded path (every rank computes its own
// batch shard, then the logits are gathered).
//
// libnccl is opened lazily with dlopen so single-GPU use needs no NCCL.
#include "common.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>

namespace {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi g_api;
ncclComm_t g_comm = nullptr;

// Asynchronous gathers: a second stream carries the all-gathers so the
// library stream can go on computing (the next step's forward) while a
// step's outputs cross NVLink.  Each slot has a "gather done" event.
constexpr int kAsyncSlots = 4;
cudaStream_t g_comm_stream = nullptr;
cudaEvent_t g_ready = nullptr;             // library stream -> comm stream
cudaEvent_t g_done[kAsyncSlots] = {};      // comm stream -> library stream

int ensure_comm_stream() {
  if (g_comm_stream) return WXX_OK;
  WXX_CUDA_CHECK(cudaStreamCreateWithFlags(&g_comm_stream, cudaStreamNonBlocking));
  WXX_CUDA_CHECK(cudaEventCreateWithFlags(&g_ready, cudaEventDisableTiming));
  for (int i = 0; i < kAsyncSlots; ++i)
    WXX_CUDA_CHECK(cudaEventCreateWithFlags(&g_done[i], cudaEventDisableTiming));
  return WXX_OK;
}

int load_api() {
  if (g_api.handle) return WXX_OK;
  const char* names[] = {"libnccl.so.2", "libnccl.so"};
  for (const char* n : names) {
    g_api.handle = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (g_api.handle) break;
  }
  if (!g_api.handle) {
    wxx::set_error("NCCL library not found (dlopen libnccl.so.2 failed)");
    return WXX_E_UNSUPPORTED;
  }
#define WXX_SYM(field, name)                                                \
  g_api.field = reinterpret_cast<decltype(g_api.field)>(dlsym(g_api.handle, name)); \
  if (!g_api.field) {                                                       \
    wxx::set_error("NCCL symbol %s missing", name);                         \
    return WXX_E_UNSUPPORTED;                                               \
  }
  WXX_SYM(GetUniqueId, "ncclGetUniqueId");
  WXX_SYM(CommInitRank, "ncclCommInitRank");
  WXX_SYM(AllGather, "ncclAllGather");
  WXX_SYM(CommDestroy, "ncclCommDestroy");
  WXX_SYM(CommAbort, "ncclCommAbort");
  WXX_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
  WXX_SYM(GetErrorString, "ncclGetErrorString");
#undef WXX_SYM
  return WXX_OK;
}

int check(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return WXX_OK;
  wxx::set_error("%s failed: %s", what, g_api.GetErrorString ? g_api.GetErrorString(r) : "?");
  return WXX_E_CUDA;
}

}  // namespace

// Writes the 128-byte NCCL unique id (rank 0 creates it and shares it with the
// other ranks through the host-side rendezvous).
WXX_EXPORT int wxx_nccl_unique_id(uint8_t* out128) {
  int st = load_api();
  if (st) return st;
  ncclUniqueId id;
  st = check(g_api.GetUniqueId(&id), "ncclGetUniqueId");
  if (st) return st;
  static_assert(sizeof(ncclUniqueId) == 128, "unexpected ncclUniqueId size");
  memcpy(out128, &id, 128);
  return WXX_OK;
}

WXX_EXPORT int wxx_nccl_init(const uint8_t* id128, int nranks, int rank) {
  WXX_REQUIRE_INIT();
  int st = load_api();
  if (st) return st;
  WXX_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "wxx_nccl_init: bad rank %d of %d", rank,
              nranks);
  if (g_comm) {
    wxx::set_error("wxx_nccl_init: communicator already initialised");
    return WXX_E_STATE;
  }
  ncclUniqueId id;
  memcpy(&id, id128, 128);
  return check(g_api.CommInitRank(&g_comm, nranks, id, rank), "ncclCommInitRank");
}

// recv (nranks * nbytes) <- concat over ranks of send (nbytes), on the library stream.
WXX_EXPORT int wxx_nccl_allgather(void* recv, const void* send, uint64_t nbytes) {
  WXX_REQUIRE_INIT();
  if (!g_comm) {
    wxx::set_error("wxx_nccl_allgather: call wxx_nccl_init first");
    return WXX_E_STATE;
  }
  return check(g_api.AllGather(send, recv, (size_t)nbytes, ncclUint8, g_comm, wxx::stream()),
               "ncclAllGather");
}

// All-gather on the communication stream, ordered after everything enqueued
// on the library stream so far (send is complete when it starts).  The
// library stream does not wait for it: call wxx_nccl_wait(slot) before any
// library-stream work that reads recv or overwrites send.  The caller keeps
// both buffers allocated until that wait is enqueued (frees are ordered on
// the library stream only).  slot in [0, 4).
WXX_EXPORT int wxx_nccl_allgather_async(void* recv, const void* send, uint64_t nbytes, int slot) {
  WXX_REQUIRE_INIT();
  if (!g_comm) {
    wxx::set_error("wxx_nccl_allgather_async: call wxx_nccl_init first");
    return WXX_E_STATE;
  }
  WXX_REQUIRE(slot >= 0 && slot < kAsyncSlots, "wxx_nccl_allgather_async: slot %d not in [0, %d)",
              slot, kAsyncSlots);
  int st = ensure_comm_stream();
  if (st) return st;
  WXX_CUDA_CHECK(cudaEventRecord(g_ready, wxx::stream()));
  WXX_CUDA_CHECK(cudaStreamWaitEvent(g_comm_stream, g_ready, 0));
  st = check(g_api.AllGather(send, recv, (size_t)nbytes, ncclUint8, g_comm, g_comm_stream),
             "ncclAllGather");
  if (st) return st;
  WXX_CUDA_CHECK(cudaEventRecord(g_done[slot], g_comm_stream));
  return WXX_OK;
}

// Makes the library stream wait for the last asynchronous gather of `slot`
// (no host wait).  A slot never used is already complete.
WXX_EXPORT int wxx_nccl_wait(int slot) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(slot >= 0 && slot < kAsyncSlots, "wxx_nccl_wait: slot %d not in [0, %d)", slot,
              kAsyncSlots);
  if (!g_comm_stream) return WXX_OK;
  WXX_CUDA_CHECK(cudaStreamWaitEvent(wxx::stream(), g_done[slot], 0));
  return WXX_OK;
}

// Reads the communicator's asynchronous error state (0 = healthy).
WXX_EXPORT int wxx_nccl_async_error(int* code) {
  if (!g_comm) {
    *code = 0;
    return WXX_OK;
  }
  ncclResult_t r = ncclSuccess;
  int st = check(g_api.CommGetAsyncError(g_comm, &r), "ncclCommGetAsyncError");
  *code = (int)r;
  return st;
}

// abort = 1 tears the communicator down without waiting for peers (used when
// a peer is known to be gone); 0 is the orderly destroy.
WXX_EXPORT int wxx_nccl_destroy(int abort) {
  if (!g_comm) return WXX_OK;
  if (g_comm_stream && !abort) {
    // orderly: the last gathers finish before the communicator goes
    WXX_CUDA_CHECK(cudaStreamSynchronize(g_comm_stream));
  }
  ncclResult_t r = abort ? g_api.CommAbort(g_comm) : g_api.CommDestroy(g_comm);
  g_comm = nullptr;
  return check(r, abort ? "ncclCommAbort" : "ncclCommDestroy");
}
