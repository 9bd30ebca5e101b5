// Shared device helpers for the W4A16 kernels (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lb {

// fp16 constants as packed f16x2 bit patterns
constexpr uint32_t kMagic = 0x64006400u;     // 1024.0 | 1024.0: OR-ing a nibble u into the mantissa gives 1024 + u
constexpr uint32_t kBias1032 = 0x64086408u;  // 1032.0 = 1024 + 8
constexpr uint32_t kSixteenth = 0x2C002C00u; // 1 / 16
constexpr uint32_t kMinus72 = 0xD480D480u;   // -72.0 = -(1024 / 16 + 8)

__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Signed values of nibble pair j = 0 and j = 1 of a word in the v3 slot order, as exact f16x2.
//   pair 0: slots 0 and 4 (bits 0-3, 16-19)      -> (1024 + u) - 1032
//   pair 1: slots 1 and 5 (bits 4-7, 20-23)      -> (1024 + 16u) / 16 - 72
// Both results are small integers, so every step is exact. Pairs 2 and 3 are the same on (word >> 8).
// (a & b) | c in one instruction (lop3 truth table 0xEA)
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t q_pair_lo(uint32_t word) {
  return hsub2_bits(and_or(word, 0x000F000Fu, kMagic), kBias1032);
}
__device__ __forceinline__ uint32_t q_pair_hi(uint32_t word) {
  return hfma2_bits(and_or(word, 0x00F000F0u, kMagic), kSixteenth, kMinus72);
}

// Pair j (0..3) of a v3-order word as exact f16x2 of (u - 8): (k0 + 2j, k0 + 2j + 1)
__device__ __forceinline__ uint32_t q_pair(uint32_t word, int j) {
  return hsub2_bits(((word >> (4 * j)) & 0x000F000Fu) | kMagic, kBias1032);
}

// Streaming 128-bit load of data read exactly once (weights): no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint16_t ldg_u16(const void* p) {
  uint16_t v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Load of data a previous kernel in the stream may have just written (activations): cached in L2 only, so no
// stale L1 line from before the programmatic-dependency wait can be hit.
__device__ __forceinline__ uint32_t ldg_cg_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Programmatic dependent launch: let the next kernel in the stream launch, and wait for the previous one.
// Both are no-ops when the launch carries no programmatic dependency.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// The wait behind a branch on a kernel argument that is always nonzero: the compiler may legally sink loads
// issued before an unconditional wait below it (which serializes them behind the previous kernel); it does
// not move them across the branch, so weight loads issued first really are in flight during the wait.
__device__ __forceinline__ void pdl_wait_after_loads(int guard) {
  if (guard) pdl_wait();
}

// D += A * B, m16n8k16, f16 inputs, f32 accumulators (PTX ISA fragment layout: lane = 4g + t;
// a0 = A[g][2t..2t+1], a1 = A[g+8][2t..], a2 = A[g][2t+8..], a3 = A[g+8][2t+8..]; b0 = B[2t..][g], b1 = B[2t+8..][g];
// d0,d1 = D[g][2t, 2t+1], d2,d3 = D[g+8][2t, 2t+1]).
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// four 8x8 b16 matrices from shared memory (lane L supplies the address of row L & 7 of matrix L >> 3);
// register j of lane (g, t) receives matrix j's elements (row g, columns 2t and 2t + 1)
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// the same four matrices transposed: register j of lane (g, t) receives matrix j's elements (rows 2t and 2t + 1,
// column g) -- the A fragment of a row-major [k][m] tile
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// two 8x8 b16 matrices (lanes 0-15 supply the row addresses): the B fragment of an [n][k] row-major tile
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}

// An output value as the reference's W4Linear produces it (lowbit/model.py:22-27): the product rounded to fp16, then,
// with a bias, the fp16 bias added and the sum rounded again (torch's fp16 add: computed in fp32, rounded once)
__device__ __forceinline__ __half out_half(float v, const __half* bias, int row) {
  const __half h = __float2half_rn(v);
  return bias ? __float2half_rn(__half2float(h) + __half2float(bias[row])) : h;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace lb

namespace lb {

// ---------------------------------------------------------------------------------------------- mbarriers
// Every wait in this library is bounded: after kSpinLimit unsuccessful polls the waiting thread records
// an error code in g_device_error (read by lb_device_error()) and gives up instead of hanging the GPU.
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr int kErrBarrierTimeout = 1;
constexpr int kErrPeerTimeout = 2;    // a peer rank did not publish its epoch in time (allreduce)
constexpr int kErrBadPosition = 3;   // a decode position outside the KV cache (nothing was read or written)

// ------------------------------------------------------------------------------------- peer-memory epochs
// Row-parallel sums over NVLink peer memory: every rank owns a peer-mapped buffer that starts with
// kPeerFlagBytes of per-rank epoch flags (flag r = the last epoch rank r has published into this buffer).
constexpr int kPeerFlagBytes = 256;
constexpr long long kPeerWaitCycles = 2000000000LL;   // ~1 s at B200 clocks, then kErrPeerTimeout

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Poll flag f until it reaches epoch e (wrap-around safe) for at most kPeerWaitCycles; false on timeout, after
// recording kErrPeerTimeout in *status
__device__ __forceinline__ bool wait_peer_epoch(const uint32_t* f, uint32_t e, int* status) {
  const long long t0 = clock64();
  while ((int)(ld_acquire_sys(f) - e) < 0) {
    if (clock64() - t0 > kPeerWaitCycles) {
      atomicExch(status, kErrPeerTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global -> shared copy through L2 only (no L1 allocation), completed by cp_async_wait<N>
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` transactions on `bar`
// (16-byte aligned addresses, size a multiple of 16)
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 16-byte asynchronous global -> shared copy cached in L2 only, committed and awaited in groups
__device__ __forceinline__ void cp_async_cg16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_group_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_group_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace lb
