// collective.cu -- the embedding gather of the image-sharded encoder as C
// entry points over NCCL, with a deadline on every wait.
//
// Images are independent, so the only exchange of a multi-GPU encoder run is
// one all-gather of every rank's [B/G, T/4, C_out] fp16 embeddings. These
// entries wrap it so that a peer that dies or hangs never blocks a caller
// for good:
//
//   * the communicator is created NON-BLOCKING (ncclConfig_t.blocking = 0):
//     every NCCL call returns at once, possibly with ncclInProgress, and the
//     host polls ncclCommGetAsyncError until the call has completed, the
//     communicator reports an error, or the caller's deadline passes;
//   * completion of the gather on the device is polled the same way
//     (cudaStreamQuery on the caller's stream, the communicator's async error
//     between polls);
//   * when a deadline passes, the communicator is aborted (ncclCommAbort:
//     NCCL's kernels observe the abort and return, freeing the stream) and
//     the call answers HEXLIB_B200_ERR_TIMEOUT; an error reported by NCCL
//     (a peer that closed its connections, say) aborts it too and answers
//     HEXLIB_B200_ERR_COMM. An aborted communicator refuses further work.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, which resolves to the
// copy a process has already loaded, e.g. torch's), so the library links
// against nothing but the CUDA runtime. No peer loads, no multicast: the
// transfer is NCCL's own over NVLink / NVSwitch.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdint.h>
#include <string.h>
#include <time.h>

#include <mutex>

#include "../../include/hexlib_b200.h"

struct hexlib_b200_comm {
  ncclComm_t comm = nullptr;
  int device = -1;
  int nranks = 0;
  int rank = -1;
  bool aborted = false;
};

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*finalize)(ncclComm_t) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.init_rank_config =
        reinterpret_cast<decltype(api.init_rank_config)>(dlsym(h, "ncclCommInitRankConfig"));
    api.async_error =
        reinterpret_cast<decltype(api.async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    api.abort = reinterpret_cast<decltype(api.abort)>(dlsym(h, "ncclCommAbort"));
    api.finalize = reinterpret_cast<decltype(api.finalize)>(dlsym(h, "ncclCommFinalize"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.ok = api.get_unique_id && api.init_rank_config && api.async_error && api.abort &&
             api.finalize && api.destroy && api.all_gather;
  });
  return api;
}

uint64_t now_ns() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
}

void pause_briefly() {
  timespec ts{0, 20000};   // 20 us between polls
  nanosleep(&ts, nullptr);
}

// Aborts the communicator once; returns `status` for the caller to answer.
int give_up(hexlib_b200_comm* c, int status) {
  if (!c->aborted && c->comm) {
    nccl().abort(c->comm);
    c->aborted = true;
  }
  return status;
}

// Polls until the communicator's last call has completed on the host.
int settle(hexlib_b200_comm* c, uint64_t deadline) {
  const NcclApi& A = nccl();
  for (;;) {
    ncclResult_t st = ncclInProgress;
    if (A.async_error(c->comm, &st) != ncclSuccess) return give_up(c, HEXLIB_B200_ERR_COMM);
    if (st == ncclSuccess) return HEXLIB_B200_OK;
    if (st != ncclInProgress) return give_up(c, HEXLIB_B200_ERR_COMM);
    if (now_ns() >= deadline) return give_up(c, HEXLIB_B200_ERR_TIMEOUT);
    pause_briefly();
  }
}

uint64_t deadline_after(uint32_t timeout_ms) {
  return now_ns() + (uint64_t)timeout_ms * 1000000ull;
}

}  // namespace

extern "C" {

int hexlib_b200_nccl_available(void) { return nccl().ok ? 1 : 0; }

int hexlib_b200_nccl_unique_id(uint8_t* id_out) {
  if (!id_out) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (!nccl().ok) return HEXLIB_B200_ERR_NO_KERNEL;
  ncclUniqueId id;
  if (nccl().get_unique_id(&id) != ncclSuccess) return HEXLIB_B200_ERR_COMM;
  static_assert(sizeof(id) == HEXLIB_B200_NCCL_ID_BYTES, "unique id size");
  memcpy(id_out, &id, sizeof(id));
  return HEXLIB_B200_OK;
}

int hexlib_b200_nccl_open(const uint8_t* id, int nranks, int rank, int device,
                          uint32_t timeout_ms, hexlib_b200_comm** out) {
  if (!out) return HEXLIB_B200_ERR_INVAL_PARAMS;
  *out = nullptr;
  if (!id || nranks < 1 || rank < 0 || rank >= nranks || device < 0 || timeout_ms == 0)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (!nccl().ok) return HEXLIB_B200_ERR_NO_KERNEL;
  if (cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  hexlib_b200_comm* c = new hexlib_b200_comm();
  c->device = device;
  c->nranks = nranks;
  c->rank = rank;
  const uint64_t deadline = deadline_after(timeout_ms);
  const ncclResult_t r = nccl().init_rank_config(&c->comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (c->comm) give_up(c, 0);
    delete c;
    return HEXLIB_B200_ERR_COMM;
  }
  const int rc = settle(c, deadline);
  if (rc != HEXLIB_B200_OK) {
    delete c;     // aborted by settle(): its resources are released
    return rc;
  }
  *out = c;
  return HEXLIB_B200_OK;
}

int hexlib_b200_nccl_allgather_f16(hexlib_b200_comm* c, const void* send, void* recv,
                                   uint64_t count, void* stream, uint32_t timeout_ms) {
  if (!c) return HEXLIB_B200_ERR_NOT_STARTED;
  if (c->aborted) return HEXLIB_B200_ERR_COMM;
  if (timeout_ms == 0 || (count > 0 && (!send || !recv))) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (count == 0) return HEXLIB_B200_OK;
  if (cudaSetDevice(c->device) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  const uint64_t deadline = deadline_after(timeout_ms);
  const ncclResult_t r = nccl().all_gather(send, recv, (size_t)count, ncclFloat16, c->comm,
                                           static_cast<cudaStream_t>(stream));
  if (r != ncclSuccess && r != ncclInProgress) return give_up(c, HEXLIB_B200_ERR_COMM);
  return settle(c, deadline);    // enqueued on the stream once this answers OK
}

int hexlib_b200_nccl_wait(hexlib_b200_comm* c, void* stream, uint32_t timeout_ms) {
  if (!c) return HEXLIB_B200_ERR_NOT_STARTED;
  if (c->aborted) return HEXLIB_B200_ERR_COMM;
  if (timeout_ms == 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (cudaSetDevice(c->device) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  const uint64_t deadline = deadline_after(timeout_ms);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (;;) {
    const cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) return HEXLIB_B200_OK;
    if (q != cudaErrorNotReady) {
      cudaGetLastError();
      return give_up(c, HEXLIB_B200_ERR_CUDA);
    }
    ncclResult_t st = ncclSuccess;
    if (nccl().async_error(c->comm, &st) != ncclSuccess ||
        (st != ncclSuccess && st != ncclInProgress))
      return give_up(c, HEXLIB_B200_ERR_COMM);
    if (now_ns() >= deadline) return give_up(c, HEXLIB_B200_ERR_TIMEOUT);
    pause_briefly();
  }
}

int hexlib_b200_nccl_abort(hexlib_b200_comm* c) {
  if (!c) return HEXLIB_B200_ERR_NOT_STARTED;
  give_up(c, 0);
  return HEXLIB_B200_OK;
}

int hexlib_b200_nccl_close(hexlib_b200_comm* c, uint32_t timeout_ms) {
  if (!c) return HEXLIB_B200_OK;
  int rc = HEXLIB_B200_OK;
  if (!c->aborted && c->comm) {
    cudaSetDevice(c->device);
    if (timeout_ms == 0) timeout_ms = 10000;
    const ncclResult_t r = nccl().finalize(c->comm);
    rc = (r == ncclSuccess || r == ncclInProgress) ? settle(c, deadline_after(timeout_ms))
                                                   : give_up(c, HEXLIB_B200_ERR_COMM);
    if (rc == HEXLIB_B200_OK) nccl().destroy(c->comm);
  }
  delete c;
  return rc;
}

}  // extern "C"
