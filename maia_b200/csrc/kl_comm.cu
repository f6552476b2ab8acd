// kl_comm: the collective of the N-sharded path (the all-gather of C's column blocks) on an NCCL
// communicator whose every wait is bounded. No counterpart in the reference, which has no
// multi-GPU code.
//
// The communicator is created non-blocking (ncclConfig_t.blocking = 0), so no NCCL call stalls the
// caller: initialisation, enqueueing and completion are all polled against a host deadline, with
// ncclCommGetAsyncError reporting errors the library found meanwhile (a peer gone, a broken
// connection). When the deadline passes or an error shows, the communicator is aborted
// (ncclCommAbort, which also makes its kernels still waiting on the GPU return) and the call
// returns KL_ERR_TIMEOUT or KL_ERR_NCCL; the caller's stream is left drained and usable.
//
// NCCL is loaded at run time: the libnccl.so.2 already in the process (e.g. torch's), else the
// system's. Only the few entry points below are used, through their stable C signatures.

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include <kl_gemm.h>

#include "kl_internal.cuh"

struct kl_comm {
  ncclComm_t comm = nullptr;
  int world = 0, rank = 0;
  bool aborted = false;
  std::string error;
};

namespace {

using kl::capi::cuda_fail;
using kl::capi::fail;

struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*finalize)(ncclComm_t) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string load_error;
};

Nccl const& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) {
      n.load_error = std::string("libnccl.so.2 not found: ") + dlerror();
      return;
    }
    auto sym = [&](auto& fn, char const* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (fn == nullptr && n.load_error.empty()) n.load_error = std::string("libnccl.so.2 lacks ") + name;
    };
    sym(n.get_unique_id, "ncclGetUniqueId");
    sym(n.init_rank_config, "ncclCommInitRankConfig");
    sym(n.get_async_error, "ncclCommGetAsyncError");
    sym(n.abort, "ncclCommAbort");
    sym(n.finalize, "ncclCommFinalize");
    sym(n.destroy, "ncclCommDestroy");
    sym(n.all_gather, "ncclAllGather");
    sym(n.error_string, "ncclGetErrorString");
  });
  return n;
}

kl_status nccl_ready() {
  Nccl const& n = nccl();
  if (!n.load_error.empty()) return fail(KL_ERR_NOT_SUPPORTED, "kl_comm: " + n.load_error);
  return KL_OK;
}

using Clock = std::chrono::steady_clock;

Clock::time_point deadline_after(int64_t timeout_ms) {
  return Clock::now() + std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : 1);
}

// Abort the communicator (its kernels still waiting on the GPU return), then let `stream` drain,
// itself bounded. Returns `s` with the message.
kl_status abort_comm(kl_comm* c, cudaStream_t stream, kl_status s, std::string const& why) {
  Nccl const& n = nccl();
  if (!c->aborted && c->comm != nullptr) {
    n.abort(c->comm);
    c->aborted = true;
    c->comm = nullptr;
  }
  const auto until = deadline_after(10000);
  while (cudaStreamQuery(stream) == cudaErrorNotReady && Clock::now() < until)
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  c->error = why;
  return fail(s, why);
}

// Poll until the communicator's pending operation is no longer in progress (non-blocking mode
// returns ncclInProgress from init and enqueue calls), or the deadline passes.
kl_status settle(kl_comm* c, ncclResult_t r, Clock::time_point until, cudaStream_t stream, char const* what) {
  Nccl const& n = nccl();
  while (r == ncclInProgress) {
    if (Clock::now() >= until)
      return abort_comm(c, stream, KL_ERR_TIMEOUT, std::string("kl_comm: ") + what + " did not complete in time");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    ncclResult_t st = ncclSuccess;
    r = n.get_async_error(c->comm, &st);
    if (r == ncclSuccess) r = st;
  }
  if (r != ncclSuccess)
    return abort_comm(c, stream, KL_ERR_NCCL, std::string("kl_comm: ") + what + ": " + n.error_string(r));
  return KL_OK;
}

}  // namespace

extern "C" {

kl_status kl_comm_get_unique_id(void* id) {
  if (id == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "kl_comm_get_unique_id: null id");
  kl_status s = nccl_ready();
  if (s != KL_OK) return s;
  ncclUniqueId u;
  ncclResult_t r = nccl().get_unique_id(&u);
  if (r != ncclSuccess) return fail(KL_ERR_NCCL, std::string("ncclGetUniqueId: ") + nccl().error_string(r));
  std::memcpy(id, u.internal, sizeof(u.internal));
  return KL_OK;
}

kl_status kl_comm_init(const void* id, int32_t world, int32_t rank, int64_t timeout_ms, kl_comm** out) {
  if (id == nullptr || out == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "kl_comm_init: null argument");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world) return fail(KL_ERR_INVALID_ARGUMENT, "kl_comm_init: rank outside the world");
  kl_status s = nccl_ready();
  if (s != KL_OK) return s;
  ncclUniqueId u;
  std::memcpy(u.internal, id, sizeof(u.internal));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  auto* c = new kl_comm;
  c->world = world;
  c->rank = rank;
  const auto until = deadline_after(timeout_ms);
  ncclResult_t r = nccl().init_rank_config(&c->comm, world, u, rank, &cfg);
  s = settle(c, r, until, nullptr, "communicator initialisation");
  if (s != KL_OK) {
    delete c;
    return s;
  }
  *out = c;
  return KL_OK;
}

kl_status kl_comm_all_gather(kl_comm* c, const void* send, void* recv, int64_t bytes, void* stream_ptr) {
  if (c == nullptr || send == nullptr || recv == nullptr || bytes < 0)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_comm_all_gather: null argument or negative size");
  if (c->aborted) return fail(KL_ERR_NCCL, "kl_comm_all_gather: the communicator was aborted (" + c->error + ")");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  ncclResult_t r = nccl().all_gather(send, recv, size_t(bytes), ncclUint8, c->comm, stream);
  // Enqueueing itself is quick; bound it anyway.
  return settle(c, r, deadline_after(10000), stream, "all-gather enqueue");
}

kl_status kl_comm_wait(kl_comm* c, void* stream_ptr, int64_t timeout_ms) {
  if (c == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "kl_comm_wait: null communicator");
  if (c->aborted) return fail(KL_ERR_NCCL, "kl_comm_wait: the communicator was aborted (" + c->error + ")");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const auto until = deadline_after(timeout_ms);
  for (;;) {
    cudaError_t q = cudaStreamQuery(stream);
    if (q == cudaSuccess) return KL_OK;
    if (q != cudaErrorNotReady) return cuda_fail(q, "kl_comm_wait: cudaStreamQuery");
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = nccl().get_async_error(c->comm, &st);
    if (r == ncclSuccess) r = st;
    if (r != ncclSuccess && r != ncclInProgress)
      return abort_comm(c, stream, KL_ERR_NCCL, std::string("kl_comm_wait: ") + nccl().error_string(r));
    if (Clock::now() >= until)
      return abort_comm(c, stream, KL_ERR_TIMEOUT,
                        "kl_comm_wait: the stream's collectives did not finish in " + std::to_string(timeout_ms) +
                            " ms (a rank may have left); communicator aborted");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int32_t kl_comm_is_aborted(const kl_comm* c) { return c != nullptr && c->aborted ? 1 : 0; }

kl_status kl_comm_destroy(kl_comm* c, int64_t timeout_ms) {
  if (c == nullptr) return KL_OK;
  kl_status s = KL_OK;
  if (!c->aborted && c->comm != nullptr) {
    // Finalize flushes what was issued and waits (non-blocking: polled) for the other ranks.
    ncclResult_t r = nccl().finalize(c->comm);
    s = settle(c, r, deadline_after(timeout_ms), nullptr, "communicator finalisation");
    if (s == KL_OK) nccl().destroy(c->comm);
  }
  delete c;
  return s;
}

}  // extern "C"
