// kl_gemm_host: a GEMM whose operands and result live in host memory. The library moves A to the
// device, then streams B in column blocks of C, so that the host-to-device copies of block j+1,
// the GEMM of block j and the device-to-host copy of block j-1 run at the same time on three
// streams (two copy engines and the SMs). Chained with events; ordered after and before the
// caller's stream. kl_gemm_host_b is the same with A already on the device (a sharded caller
// gathers it from the other GPUs over NVLink instead of copying all of it over PCIe on every GPU):
// the B copies start at once and the GEMMs also wait for the caller's "A ready" event. Block-scaled problems (block_scale 1 or 2) also stage the blocked scale arrays: A's whole,
// then B's row blocks along with each block of B.

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include <kl_gemm.h>

#include "kl_internal.cuh"

namespace {

struct HostPipe {
  cudaStream_t in = nullptr, mm = nullptr, out = nullptr;
  cudaEvent_t start = nullptr, done = nullptr;
  std::vector<cudaEvent_t> loaded, computed;
  void* scales = nullptr;  // device staging of block scales, grown on demand
  size_t scale_bytes = 0;
};

std::mutex g_pipe_mutex;
HostPipe g_pipes[64];

// Called with g_pipe_mutex held.
kl_status get_pipe(int dev, int chunks, HostPipe** out) {
  HostPipe& p = g_pipes[dev];
  cudaError_t e = cudaSuccess;
  if (p.in == nullptr) {
    if ((e = cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaStreamCreateWithFlags(&p.mm, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&p.done, cudaEventDisableTiming)) != cudaSuccess)
      return kl::capi::cuda_fail(e, "kl_gemm_host: stream/event creation");
  }
  while (int(p.loaded.size()) < chunks) {
    cudaEvent_t a = nullptr, b = nullptr;
    if ((e = cudaEventCreateWithFlags(&a, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&b, cudaEventDisableTiming)) != cudaSuccess)
      return kl::capi::cuda_fail(e, "kl_gemm_host: event creation");
    p.loaded.push_back(a);
    p.computed.push_back(b);
  }
  *out = &p;
  return KL_OK;
}

int elem_bytes(int32_t t) {
  return (t == KL_BF16 || t == KL_F16) ? 2 : (t == KL_E4M3 || t == KL_E5M2 || t == KL_I8 || t == KL_U8) ? 1 : 4;
}

// Both entry points. copy_a: A (and its scales) come from the host into dev_a; otherwise desc->a
// (and desc->sfa) are device pointers already, and the GEMMs also wait for `a_ready` (if given).
kl_status host_gemm(const kl_gemm_desc* h, void* dev_a, bool copy_a, cudaEvent_t a_ready, void* dev_b, void* dev_c,
                    int32_t chunks, void* stream_ptr) {
  using kl::capi::cuda_fail;
  using kl::capi::fail;
  if (h == nullptr || (copy_a && dev_a == nullptr) || dev_b == nullptr || dev_c == nullptr || (!copy_a && h->a == nullptr))
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_host: null argument");
  if (h->m <= 0 || h->n <= 0 || h->k <= 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_host: m, n and k must be positive");
  if (h->lda < h->k || h->ldb < h->k || h->ldc < h->n) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_host: leading dimension too small");
  if (h->batch > 1) return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm_host: one problem per call (batch must be 0 or 1)");
  if (h->c_reduce != 0) return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm_host: C is output only (c_reduce must be 0)");
  const bool mx = h->block_scale != 0;
  if (mx && (h->sfa == nullptr || h->sfb == nullptr))
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_host: block scaling needs host scales of A and B (desc->sfa, desc->sfb)");
  if (h->a_major != 0 || h->b_major != 0)
    return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm_host: K-major operands only (B is streamed by rows)");
  if (h->m_block_group != nullptr)
    return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm_host: m-grouped GEMMs take device buffers (kl_gemm)");
  cudaStream_t caller = static_cast<cudaStream_t>(stream_ptr);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(KL_ERR_NOT_SUPPORTED, "device index above 63");

  // Column blocks of C (rows of B): multiples of 256 so every block starts on a tile boundary and
  // a 16-byte-aligned column of C.
  if (chunks <= 0) chunks = int(std::min<int64_t>(8, std::max<int64_t>(1, h->n / 1024)));
  int64_t block = (h->n + chunks - 1) / chunks;
  block = (block + 255) / 256 * 256;
  chunks = int((h->n + block - 1) / block);

  // One pipeline per device: calls from several host threads take turns enqueueing.
  std::lock_guard<std::mutex> lock(g_pipe_mutex);
  HostPipe* p = nullptr;
  kl_status s = get_pipe(dev, chunks, &p);
  if (s != KL_OK) return s;

  const int ec = elem_bytes(h->c_type);
  // Bytes of `elems` operand elements.
  auto ab_bytes = [&](int64_t elems) {
    if (h->ab_type == KL_E2M1) return size_t(elems / 2);                           // packed fp4
    if (h->ab_type == KL_E3M2 || h->ab_type == KL_E2M3) return size_t(elems / 4 * 3);  // packed fp6
    return size_t(elems * elem_bytes(h->ab_type));
  };
  // Block scales: blocked arrays, A's then B's, in one staging buffer.
  const int32_t vec = h->block_scale == 2 ? 16 : 32;
  const int64_t sfa_bytes = (mx && copy_a) ? kl_block_scale_bytes(h->m, h->k, vec) : 0;
  const int64_t sfb_bytes = mx ? kl_block_scale_bytes(h->n, h->k, vec) : 0;
  const int64_t sf_row_block = ((h->k + 4 * vec - 1) / (4 * vec)) * 512;  // bytes per 128 rows
  if (mx && p->scale_bytes < size_t(sfa_bytes + sfb_bytes)) {
    if (p->scales != nullptr) {
      if ((e = cudaDeviceSynchronize()) != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
      cudaFree(p->scales);
      p->scales = nullptr;
      p->scale_bytes = 0;
    }
    if ((e = cudaMalloc(&p->scales, size_t(sfa_bytes + sfb_bytes))) != cudaSuccess)
      return cuda_fail(e, "kl_gemm_host: cudaMalloc(scale staging)");
    p->scale_bytes = size_t(sfa_bytes + sfb_bytes);
  }
  char* dsfa = static_cast<char*>(p->scales);
  char* dsfb = dsfa + sfa_bytes;
  const char* ha = static_cast<const char*>(h->a);
  const char* hb = static_cast<const char*>(h->b);
  char* hc = static_cast<char*>(h->c);
  char* da = static_cast<char*>(dev_a);
  char* db = static_cast<char*>(dev_b);
  char* dc = static_cast<char*>(dev_c);

  // Start after everything already queued on the caller's stream.
  if ((e = cudaEventRecord(p->start, caller)) != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  if ((e = cudaStreamWaitEvent(p->in, p->start, 0)) != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent");
  if (copy_a) {
    if ((e = cudaMemcpyAsync(da, ha, ab_bytes(h->m * h->lda), cudaMemcpyHostToDevice, p->in)) != cudaSuccess)
      return cuda_fail(e, "kl_gemm_host: copy of A");
    if (mx && (e = cudaMemcpyAsync(dsfa, h->sfa, size_t(sfa_bytes), cudaMemcpyHostToDevice, p->in)) != cudaSuccess)
      return cuda_fail(e, "kl_gemm_host: copy of A's scales");
  } else if (a_ready != nullptr) {
    if ((e = cudaStreamWaitEvent(p->mm, a_ready, 0)) != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent(A ready)");
  }
  for (int j = 0; j < chunks; ++j) {
    const int64_t n0 = int64_t(j) * block, nj = std::min<int64_t>(block, h->n - n0);
    e = cudaMemcpyAsync(db + ab_bytes(n0 * h->ldb), hb + ab_bytes(n0 * h->ldb), ab_bytes(nj * h->ldb),
                        cudaMemcpyHostToDevice, p->in);
    if (e != cudaSuccess) return cuda_fail(e, "kl_gemm_host: copy of B");
    // Block j starts on a 256-row boundary of B, so its scales are whole 128-row blocks.
    const int64_t sf_off = (n0 / 128) * sf_row_block, sf_len = ((nj + 127) / 128) * sf_row_block;
    if (mx) {
      e = cudaMemcpyAsync(dsfb + sf_off, static_cast<const char*>(h->sfb) + sf_off, size_t(sf_len),
                          cudaMemcpyHostToDevice, p->in);
      if (e != cudaSuccess) return cuda_fail(e, "kl_gemm_host: copy of B's scales");
    }
    if ((e = cudaEventRecord(p->loaded[j], p->in)) != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    if ((e = cudaStreamWaitEvent(p->mm, p->loaded[j], 0)) != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent");
    kl_gemm_desc d = *h;
    d.n = nj;
    d.a = copy_a ? da : h->a;
    d.b = db + ab_bytes(n0 * h->ldb);
    d.c = dc + size_t(n0) * ec;
    if (mx) {
      d.sfa = copy_a ? dsfa : h->sfa;
      d.sfb = dsfb + sf_off;
    }
    s = kl_gemm(&d, p->mm);
    if (s != KL_OK) return s;
    if ((e = cudaEventRecord(p->computed[j], p->mm)) != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    if ((e = cudaStreamWaitEvent(p->out, p->computed[j], 0)) != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent");
    e = cudaMemcpy2DAsync(hc + size_t(n0) * ec, size_t(h->ldc) * ec, dc + size_t(n0) * ec, size_t(h->ldc) * ec,
                          size_t(nj) * ec, size_t(h->m), cudaMemcpyDeviceToHost, p->out);
    if (e != cudaSuccess) return cuda_fail(e, "kl_gemm_host: copy of C");
  }
  // The caller's stream continues once C is back on the host.
  if ((e = cudaEventRecord(p->done, p->out)) != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  if ((e = cudaStreamWaitEvent(caller, p->done, 0)) != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent");
  return KL_OK;
}

}  // namespace

extern "C" kl_status kl_gemm_host(const kl_gemm_desc* h, void* dev_a, void* dev_b, void* dev_c, int32_t chunks,
                                  void* stream_ptr) {
  return host_gemm(h, dev_a, true, nullptr, dev_b, dev_c, chunks, stream_ptr);
}

extern "C" kl_status kl_gemm_host_b(const kl_gemm_desc* h, void* a_ready, void* dev_b, void* dev_c, int32_t chunks,
                                    void* stream_ptr) {
  return host_gemm(h, nullptr, false, static_cast<cudaEvent_t>(a_ready), dev_b, dev_c, chunks, stream_ptr);
}
