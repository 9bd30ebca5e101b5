// TMA, cluster and bounded-wait helpers shared by the TMA-fed kernels (sm_100a).
#pragma once
#include <cuda.h>

#include "lb_common.cuh"

namespace lb {

// 2-D tensor copy global -> this CTA's shared memory (coordinates: innermost first), completing on `bar`.
// No multicast: the destination is the issuing CTA's own shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// Bounded mbarrier wait: after kSpinLimit unsuccessful polls it records kErrBarrierTimeout in *status and gives up.
__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity, int* status) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicExch(status, kErrBarrierTimeout);
  return false;
}

// One loader thread streaming chunks 0..nc-1 through a stage ring: refills stage s once its consumers released it
// (empty[s]), then waits for its own last copies so that none is in flight when the CTA exits.
template <typename Issue>
__device__ __forceinline__ void run_loader(int nc, int stages, uint64_t* full, uint64_t* empty, uint32_t bytes,
                                           int* status, Issue issue) {
  int issued = 0;
  for (int i = 0; i < nc; ++i) {
    const int s = i % stages;
    if (i >= stages && !wait_bounded(&empty[s], ((i / stages) - 1) & 1, status)) break;
    mbar_arrive_expect_tx(&full[s], bytes);
    issue(i, s);
    issued = i + 1;
  }
  for (int i = issued > stages ? issued - stages : 0; i < issued; ++i)
    wait_bounded(&full[i % stages], (i / stages) & 1, status);
}

}  // namespace lb
