#pragma once

// Shared between the translation units of libkl_b200.so; not part of the public ABI.

#include <cuda_runtime.h>

#include <cstddef>
#include <string>

#include <kl_gemm.h>

namespace kl::capi {

// Record `msg` as this thread's last error and return `s`.
kl_status fail(kl_status s, std::string const& msg);
kl_status cuda_fail(cudaError_t e, char const* where);

// Bound for every device-side wait, and the device status word those waits report into.
unsigned long long wait_timeout_ns();
kl_status device_status_ptr(int** out);

// KL_ALGO_AUTO resolution.
int choose_algo(kl_gemm_desc const& d);

// Memory-bound small-M path (kl_skinny.cu).
kl_status skinny_workspace_size(kl_gemm_desc const& d, size_t* bytes);
kl_status run_skinny(kl_gemm_desc const& d, void* workspace, size_t workspace_bytes, cudaStream_t stream);
// After a timed-out kernel the library workspace's tickets may be mid-count: re-zero before reuse.
// (Marks the skinny workspace and every split-tail workspace of the device.)
void mark_workspace_dirty(int device);

// Split-tail workspace of the tile kernels for `stream` on the current device (kl_tile_ws.cu):
// kl::gemm::kTnStreamKWorkspaceBytes with zeroed tickets, or nullptr where none can be had without
// allocating inside a stream capture (the launch then deals whole tiles).
kl_status tile_stream_k_workspace(cudaStream_t stream, void** out);
void tile_workspaces_mark_dirty(int device);

// kl_release_workspaces' two halves: free every library-owned workspace (after synchronising its
// device) so the next call allocates afresh.
kl_status release_skinny_workspaces();
kl_status release_tile_workspaces();
// Drops the cached device addresses of kl_gemm_skinny_noalloc's scratch array (looked up again on
// the next call).
void forget_noalloc_scratch();

// Failure-path probe (kl_probe.cu).
kl_status launch_wait_probe(int* status, unsigned long long timeout_ns, cudaStream_t stream);

}  // namespace kl::capi
