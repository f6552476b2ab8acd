#pragma once

// TMA copy wrappers (cp.async.bulk.tensor) for the maps built by kl::make_tma_desc.
// No counterpart in the reference: kernel_lib builds the maps (tma_desc.hpp) but issues no copies.
//
// There is deliberately no cluster-multicast load here. Loads only read this GPU's memory; a
// CTA pair shares an operand by each CTA loading its own half (the .cta_group::2 form below).

#include <cstdint>

#include <kl/config.hpp>

namespace kl {

#if defined(__CUDACC__)

KL_DEVICE void tma_prefetch_map(const void* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tile load into this CTA's shared memory; completes `tx` bytes on `bar` (this CTA's barrier).
KL_DEVICE void tma_load_2d(uint32_t dst, const void* map, uint32_t bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// Same with an L2 eviction-policy hint (a createpolicy value).
KL_DEVICE void tma_load_2d_hint(uint32_t dst, const void* map, uint32_t bar, int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// CTA-pair load: the tile lands in this CTA's shared memory, and the byte count completes on
// `bar_cluster`, a shared::cluster barrier address that may be in the peer CTA of the pair.
KL_DEVICE void tma_load_2d_pair(uint32_t dst, const void* map, uint32_t bar_cluster, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

// Ask the TMA unit to bring a 2-D tile into L2 (no shared memory, no barrier): lets a producer
// run further ahead of its shared-memory ring than the ring itself allows.
KL_DEVICE void tma_prefetch_l2_2d(const void* map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

// 3-D forms (batched tensors: the third coordinate is the batch index).
KL_DEVICE void tma_load_3d(uint32_t dst, const void* map, uint32_t bar, int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

KL_DEVICE void tma_load_3d_pair(uint32_t dst, const void* map, uint32_t bar_cluster, int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}

KL_DEVICE void tma_store_3d(const void* map, uint32_t src, int32_t x, int32_t y, int32_t z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}

KL_DEVICE uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
KL_DEVICE uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2-D tile store from this CTA's shared memory (bulk-group completion).
KL_DEVICE void tma_store_2d(const void* map, uint32_t src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}

// Reducing stores: global[box] += shared[box], element-wise in the tensor map's data type (the
// kernels here use them on fp32 tensors only), performed by the TMA unit. Same bulk-group
// completion as the plain stores.
KL_DEVICE void tma_reduce_add_2d(const void* map, uint32_t src, int32_t x, int32_t y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}

KL_DEVICE void tma_reduce_add_3d(const void* map, uint32_t src, int32_t x, int32_t y, int32_t z) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}

KL_DEVICE void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N committed store groups still read shared memory.
template <int N>
KL_DEVICE void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until at most N committed store groups are incomplete (writes done).
template <int N>
KL_DEVICE void tma_store_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Order this thread's generic-proxy shared-memory writes before later async-proxy (TMA) reads.
KL_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

#endif  // __CUDACC__

}  // namespace kl
