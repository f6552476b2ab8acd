// Split-tail workspaces of the tile kernels: one fixed-size buffer per (device, stream), allocated on
// first use and never freed or moved while the process runs, so a CUDA graph that captured a launch
// keeps a valid pointer. Its ticket area is zeroed once and stays zero between launches (the last
// K-range of each split tile to arrive resets its ticket); after a timed-out launch it is re-zeroed on the
// stream before the next use.

#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

#include <kl/gemm/gemm.hpp>

#include "kl_internal.cuh"

namespace kl::capi {

namespace {

struct TileWorkspace {
  void* ptr = nullptr;
  bool dirty = false;
};
std::mutex g_tile_ws_mutex;
std::map<std::pair<int, cudaStream_t>, TileWorkspace> g_tile_ws;

}  // namespace

kl_status tile_stream_k_workspace(cudaStream_t stream, void** out) {
  *out = nullptr;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(stream, &cap);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  const bool capturing = cap != cudaStreamCaptureStatusNone;
  std::lock_guard<std::mutex> lock(g_tile_ws_mutex);
  TileWorkspace& w = g_tile_ws[{dev, stream}];
  if (w.ptr == nullptr) {
    if (capturing) return KL_OK;  // no allocation inside a capture: this launch deals whole tiles
    e = cudaMalloc(&w.ptr, kl::gemm::kTnStreamKWorkspaceBytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      w.ptr = nullptr;
      return KL_OK;  // out of memory: whole tiles
    }
    w.dirty = true;
  }
  if (w.dirty) {
    if (capturing) return KL_OK;
    e = cudaMemsetAsync(w.ptr, 0, kl::gemm::kTnStreamKTicketBytes, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(split-tail tickets)");
    w.dirty = false;
  }
  *out = w.ptr;
  return KL_OK;
}

kl_status release_tile_workspaces() {
  std::lock_guard<std::mutex> lock(g_tile_ws_mutex);
  if (g_tile_ws.empty()) return KL_OK;
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  while (e == cudaSuccess && !g_tile_ws.empty()) {
    auto it = g_tile_ws.begin();
    if (it->second.ptr != nullptr) {
      e = cudaSetDevice(it->first.first);
      if (e == cudaSuccess) e = cudaDeviceSynchronize();  // no launch may still use it
      if (e == cudaSuccess) e = cudaFree(it->second.ptr);
      if (e != cudaSuccess) break;
    }
    g_tile_ws.erase(it);
  }
  cudaSetDevice(prev);
  return e == cudaSuccess ? KL_OK : cuda_fail(e, "kl_release_workspaces (split tail)");
}

void tile_workspaces_mark_dirty(int device) {
  std::lock_guard<std::mutex> lock(g_tile_ws_mutex);
  for (auto& [key, w] : g_tile_ws)
    if (key.first == device) w.dirty = true;
}

}  // namespace kl::capi
