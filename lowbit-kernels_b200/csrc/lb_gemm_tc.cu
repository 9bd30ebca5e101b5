// W4A16 skinny GEMM on the 5th-generation tensor cores: y[M, N] = x[M, K] * dequant(W)[N, K]^T, M <= 64.
//
// Role of the reference's gemm_v5 (csrc/w4_gemv.cu:209-294), which ran mma.sync on a T4. Swap-AB: the weights
// are the 128-row A operand, the activation rows the N side of the MMA (NB = M rounded up to 32, 48 or 64).
// Grid: one column of CTAs per 128-row tile of W; the S CTAs of a column form a thread-block cluster that splits
// K into S contiguous ranges and adds its fp32 partial tiles through distributed shared memory (no workspace).
//   * 8 producer warps: each owns a 16-row slice of the tile. Per 128-wide K chunk a lane takes the 16-byte
//     words t of rows g and g+8 (the mma layout is the m16n8k16 A fragment), turns them into fp16 weights
//     fp16_rn((u - 8) * scale) -- bit-identical to the dequantize kernel -- and writes them with stmatrix into
//     the canonical no-swizzle K-major layout (8x8 core matrices of 16-byte rows: the fragment registers of a
//     warp are exactly four core matrices). Each lane keeps 8 chunks of raw words in flight in a private
//     cp.async ring; the CTA's scales are staged once.
//   * one TMA warp: a single thread loads the activations of each chunk with two 2-D tensor copies (64 k x NB
//     rows, 128-byte swizzle; rows >= M read as zeros) into a 4-deep stage ring.
//   * one MMA warp: a single thread issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=NB, K=16) per k16
//     step with the fp32 accumulator in tensor memory; tcgen05.commit releases the stages.
//   * the producers read the accumulator with tcgen05.ld (each warp its 32-lane quarter of the tile) and store
//     fp16, or, split across a cluster, park fp32 partials in shared memory that every CTA of the cluster sums
//     for its share of the outputs in a fixed rank order (deterministic).
// Stages are handed over through mbarriers; every wait is bounded and records a status code instead of hanging,
// no copy is left in flight at exit, and tensor memory is released on every path.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>

#include "lb_common.cuh"
#include "lb_launch.h"

namespace lb {

// status word of this file's kernels (a bounded wait that gave up); read by gemm_tc_device_error()
__device__ int g_tc_status;

namespace {

constexpr int kProducerWarps = 8;
constexpr int kMmaWarp = 8;
constexpr int kTmaWarp = 9;
constexpr int kThreads = 10 * 32;
constexpr int kAStages = 2;          // dequantized weight tiles the tensor core reads
constexpr int kBStages = 4;          // activation tiles in flight
constexpr int kRing = 8;             // chunks of raw packed weights in flight per producer lane
constexpr int kRingLaneBytes = 32;   // per chunk: the lane's 16-byte words of rows g and g + 8
constexpr int kAStepBytes = 16 * 2 * 128;      // one k16 step of the 128-row A tile: 16 row groups x 2 k halves
constexpr int kAStageBytes = 8 * kAStepBytes;  // a 128-wide K chunk
constexpr int kMaxSplits = 8;        // portable cluster size
constexpr int kSmemLimit = 227 * 1024;

// an activation stage: two 64-wide k halves of NB rows x 128 bytes (each half a whole number of 1024-byte
// swizzle atoms)
__host__ __device__ inline int b_stage_bytes(int nb) { return nb * 256; }

struct TcLayout {
  int a, b, ring, scales, bars, tmem_slot, total;
};

// offsets from the 1024-byte aligned start of dynamic shared memory; `ngroups` = scale groups per CTA
__host__ __device__ inline TcLayout tc_layout(int nb, int ngroups) {
  TcLayout L;
  L.a = 0;
  L.b = kAStages * kAStageBytes;
  L.ring = L.b + kBStages * b_stage_bytes(nb);
  L.scales = L.ring + kRing * kProducerWarps * 32 * kRingLaneBytes;
  L.bars = L.scales + ((128 * ngroups * 2 + 15) & ~15);
  L.tmem_slot = L.bars + (2 * kAStages + 2 * kBStages + 1) * 8;
  L.total = L.tmem_slot + 16;
  return L;
}

__host__ __device__ inline int tc_nb(int m) { return m <= 32 ? 32 : m <= 48 ? 48 : 64; }

struct TcParams {
  const void* w;  // packed uint8 [N, K / 2], mma layout
  const void* s;  // fp16 [N, K / G]
  __half* y;      // fp16 [M, N]
  int M, N, K, KG, cpg;
  int flags;
  int wait_guard;  // always 1 (see pdl_wait_after_loads)
  int splits;      // CTAs per cluster splitting K (gridDim.y)
  int ngroups;     // scale groups staged per CTA (the largest K range's)
};

__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicExch(&g_tc_status, kErrBarrierTimeout);
  return false;
}

__device__ __forceinline__ void stsm_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.x4.m8n8.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor (sm_100 format: version 1 at bit 46, layout type at bits 61-63).
// No swizzle, K-major: core matrices of 8 rows x 16 bytes; LBO = byte distance between the two k halves of a
// k16 step, SBO = between consecutive 8-row groups.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}
// 128-byte swizzle, K-major: rows of 128 bytes (64 fp16 k), 8-row atoms of 1024 bytes (SBO); a k16 step inside
// the atom starts 32 bytes further (the swizzle is applied to the computed addresses, atoms 1024-byte aligned)
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return smem_desc(addr, 16, 1024) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// 2-D tensor copy global -> this CTA's shared memory (coordinates: innermost first), completing on `bar`
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
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

}  // namespace

template <int NB>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc05_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const TcLayout L = tc_layout(NB, p.ngroups);
  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty_a = full_a + kAStages;
  uint64_t* full_b = empty_a + kAStages;
  uint64_t* empty_b = full_b + kBStages;
  uint64_t* done = empty_b + kBStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem_slot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = p.N, M = p.M, cpg = p.cpg, S = p.splits;
  const int n0 = blockIdx.x * 128;
  const int KC = p.K >> 7;
  const int c_begin = (KC * (int)blockIdx.y) / S, nc = (KC * ((int)blockIdx.y + 1)) / S - c_begin;
  constexpr int kTmemCols = NB <= 32 ? 32 : 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&full_a[s], kProducerWarps * 32);
      mbar_init(&empty_a[s], 1);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&full_b[s], 1);
      mbar_init(&empty_b[s], 1);
    }
    mbar_init(done, 1);
    mbar_fence_init();
  }
  if (warp == kTmaWarp && lane == 0)
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
  if (warp == kMmaWarp) {   // the MMA warp owns the tensor-memory allocation
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    // instruction descriptor: fp32 accumulate, fp16 A and B, both K-major, N = NB, M = 128
    const uint32_t idesc = (1u << 4) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    bool ok = true;
    for (int i = 0; i < nc; ++i) {
      const int sa = i % kAStages, sb = i % kBStages;
      if (ok) ok = wait_bounded(&full_a[sa], (i / kAStages) & 1);
      if (ok) ok = wait_bounded(&full_b[sb], (i / kBStages) & 1);
      tc_fence_after();
      if (lane == 0 && ok) {
        const uint32_t a0 = smem_addr(smem + L.a + sa * kAStageBytes);
        const uint32_t b0 = smem_addr(smem + L.b + sb * b_stage_bytes(NB));
#pragma unroll
        for (int st = 0; st < 8; ++st)
          umma_f16(tmem, smem_desc(a0 + st * kAStepBytes, 128, 256),
                   smem_desc_sw128(b0 + (st >> 2) * (NB * 128) + (st & 3) * 32), idesc, (i > 0 || st > 0) ? 1u : 0u);
      }
      __syncwarp();
      if (lane == 0) {   // each arrives when this chunk's MMAs have read their stage
        umma_commit(&empty_a[sa]);
        umma_commit(&empty_b[sb]);
      }
    }
    __syncwarp();
    if (lane == 0) umma_commit(done);
    __syncwarp();
    if (ok) wait_bounded(done, 0);   // no MMA in flight past this point
  } else if (warp == kTmaWarp) {
    // ------------------------------------------------------------------ activation loads
    if (lane == 0) {
      if (p.wait_guard) pdl_wait();   // the activations come from the previous kernel in the stream
      bool ok = true;
      int issued = 0;
      for (int i = 0; i < nc && ok; ++i) {
        const int sb = i % kBStages;
        if (i >= kBStages) ok = wait_bounded(&empty_b[sb], ((i / kBStages) - 1) & 1);
        if (!ok) break;
        uint8_t* dst = smem + L.b + sb * b_stage_bytes(NB);
        const int kx = (c_begin + i) * 128;
        mbar_arrive_expect_tx(&full_b[sb], b_stage_bytes(NB));
        tma_load_2d(dst, &xmap, kx, 0, &full_b[sb]);
        tma_load_2d(dst + NB * 128, &xmap, kx + 64, 0, &full_b[sb]);
        issued = i + 1;
      }
      // no copy may outlive the CTA: wait for the last stages' transfers (already consumed phases pass at once)
      for (int i = issued > kBStages ? issued - kBStages : 0; i < issued; ++i)
        wait_bounded(&full_b[i % kBStages], (i / kBStages) & 1);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ weight producers
    const int g = lane >> 2, t = lane & 3;
    const int pt = threadIdx.x;   // producer thread 0..255
    const int ra = min(n0 + 16 * warp + g, N - 1), rb = min(n0 + 16 * warp + g + 8, N - 1);  // tail rows: N-1
    const uint4* wa = reinterpret_cast<const uint4*>(p.w) + (size_t)ra * (p.K >> 5) + t;
    const uint4* wb = reinterpret_cast<const uint4*>(p.w) + (size_t)rb * (p.K >> 5) + t;
    // this lane's private ring of raw packed words: slot i % kRing holds (row g, row g + 8) of chunk i
    const uint32_t ring = smem_addr(smem + L.ring) + (uint32_t)pt * (kRing * kRingLaneBytes);
    auto issue = [&](int i) {
      if (i < nc) {
        const int c = c_begin + i;
        cp_async_cg16(ring + (i % kRing) * kRingLaneBytes, wa + 4 * c);
        cp_async_cg16(ring + (i % kRing) * kRingLaneBytes + 16, wb + 4 * c);
      }
      cp_async_group_commit();
    };
    // weights and scales may be fetched before the stream dependency resolves only when the caller declared
    // them static (kFlagEarlyWeights); otherwise wait first
    if (!(p.flags & kFlagEarlyWeights) && p.wait_guard) pdl_wait();
#pragma unroll
    for (int i = 0; i < kRing - 1; ++i) issue(i);
    // scales of the CTA's groups, rows n0 .. n0 + 127 (tail rows repeat row N - 1): two threads per row
    const int g0 = c_begin / cpg, ng = (c_begin + nc - 1) / cpg - g0 + 1;
    uint16_t* sc = reinterpret_cast<uint16_t*>(smem + L.scales);
    {
      const int r = pt >> 1;
      const uint16_t* srow = reinterpret_cast<const uint16_t*>(p.s) + (size_t)min(n0 + r, N - 1) * p.KG + g0;
      for (int gi = pt & 1; gi < ng; gi += 2) sc[r * p.ngroups + gi] = ldg_u16(srow + gi);
    }
    named_barrier(1, kProducerWarps * 32);
    if (p.wait_guard) pdl_wait();   // the outputs are written in stream order
    // stmatrix row addresses: lane L writes row (L & 7) of core matrix j = L >> 3, which is row group
    // 2 * warp + (j & 1) and k half j >> 1 of every k16 step
    const int jm = lane >> 3;
    const uint32_t a_row = (uint32_t)((((2 * warp + (jm & 1)) * 2 + (jm >> 1)) * 128) + (lane & 7) * 16);
    const int sra = (16 * warp + g) * p.ngroups, srb = (16 * warp + g + 8) * p.ngroups;
    bool ok = true;
    for (int i = 0; i < nc; ++i) {
      const int sa = i % kAStages;
      issue(i + kRing - 1);
      cp_async_group_wait<kRing - 1>();   // this lane's copies of chunk i have landed (groups complete in order)
      const uint8_t* slot = smem + L.ring + pt * (kRing * kRingLaneBytes) + (i % kRing) * kRingLaneBytes;
      const uint4 qa = *reinterpret_cast<const uint4*>(slot);
      const uint4 qb = *reinterpret_cast<const uint4*>(slot + 16);
      const int grp = cpg == 1 ? i : (c_begin + i) / cpg - g0;
      const uint32_t s2a = (uint32_t)sc[sra + grp] * 0x10001u, s2b = (uint32_t)sc[srb + grp] * 0x10001u;
      if (i >= kAStages && ok) ok = wait_bounded(&empty_a[sa], ((i / kAStages) - 1) & 1);
      __syncwarp();   // stmatrix is warp-collective
      tc_fence_after();
      // fp16_rn((u - 8) * scale), four core matrices per k16 step
      const uint32_t abase = smem_addr(smem + L.a + sa * kAStageBytes) + a_row;
#pragma unroll
      for (int qd = 0; qd < 4; ++qd) {
        const uint32_t w0 = (&qa.x)[qd], w1 = (&qb.x)[qd];
        // k16 step 2qd: pairs 0 and 1; step 2qd + 1: pairs 2 and 3
        stsm_x4(abase + (2 * qd) * kAStepBytes, hmul2_bits(q_pair_lo(w0), s2a), hmul2_bits(q_pair_lo(w1), s2b),
                hmul2_bits(q_pair_hi(w0), s2a), hmul2_bits(q_pair_hi(w1), s2b));
        stsm_x4(abase + (2 * qd + 1) * kAStepBytes, hmul2_bits(q_pair_lo(w0 >> 8), s2a),
                hmul2_bits(q_pair_lo(w1 >> 8), s2b), hmul2_bits(q_pair_hi(w0 >> 8), s2a),
                hmul2_bits(q_pair_hi(w1 >> 8), s2b));
      }
      fence_async_smem();   // generic-proxy writes (stmatrix) become visible to the tensor core
      mbar_arrive(&full_a[sa]);
    }
    cp_async_group_wait<0>();   // no ring copy is left in flight
    // epilogue: wait for the last MMA, then each warp reads its 32 lanes (rows) of the accumulator; warps q and
    // q + 4 share lanes 32q.. and alternate 16-column blocks
    if (ok) ok = wait_bounded(done, 0);
    __syncwarp();   // tcgen05.ld is warp-collective
    tc_fence_after();
    const int quarter = warp & 3, half = warp >> 2;
    const int trow = 32 * quarter + lane;   // row within the tile
    float* red = reinterpret_cast<float*>(smem + L.a);   // [m][128] fp32 partials (the A stages are free now)
#pragma unroll
    for (int blk = half; blk < NB / 16; blk += 2) {
      const int col0 = blk * 16;
      uint32_t v[16];
      tmem_ld16(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)col0, v);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (S == 1) {
        if (n0 + trow < N) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (col0 + j < M) p.y[(size_t)(col0 + j) * N + n0 + trow] = __float2half_rn(__uint_as_float(v[j]));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (col0 + j < M) red[(col0 + j) * 128 + trow] = __uint_as_float(v[j]);
      }
    }
  }

  __syncwarp();
  if (S > 1) {
    // every CTA of the cluster sums its share of the M x 128 outputs over all ranks' partials, in rank order
    cluster_sync_all();
    const int e4 = 32 * M, r = (int)cluster_rank();
    const int e_begin = (e4 * r) / S, e_end = (e4 * (r + 1)) / S;
    const uint32_t red0 = smem_addr(smem + L.a);
    for (int e = e_begin + (int)threadIdx.x; e < e_end; e += kThreads) {
      const int m = e >> 5, row4 = (e & 31) * 4;
      const uint32_t off = red0 + (uint32_t)(m * 128 + row4) * 4u;
      float4 acc = ld_dsmem_f4(mapa_shared(off, 0));
      for (int q = 1; q < S; ++q) {
        const float4 v = ld_dsmem_f4(mapa_shared(off, (uint32_t)q));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      __half* yo = p.y + (size_t)m * N + n0 + row4;
      const float a[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (n0 + row4 + j < N) yo[j] = __float2half_rn(a[j]);
    }
    cluster_sync_all();   // no CTA leaves while another still reads its partials
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

constexpr int kMaxDevices = 64;
std::atomic<int> g_sms[kMaxDevices];                        // 0: not queried yet
std::atomic<int> g_clusters[kMaxDevices][3][kMaxSplits + 1];  // max active clusters + 1 (0: not queried)

int device_sms(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return 148;
  int v = g_sms[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    g_sms[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

template <int NB>
cudaLaunchConfig_t tc_config(int N, int splits, size_t smem, cudaStream_t st, cudaLaunchAttribute* attr, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N + 127) / 128, splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (splits > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = splits;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cfg;
}

// scale groups spanned by the largest of the S contiguous K ranges
int groups_per_cta(int KC, int cpg, int S) {
  int best = 0;
  for (int r = 0; r < S; ++r) {
    const int c0 = (KC * r) / S, c1 = (KC * (r + 1)) / S;
    if (c1 > c0) best = max(best, (c1 - 1) / cpg - c0 / cpg + 1);
  }
  return best;
}

size_t tc_smem(int nb, int KC, int cpg, int S) { return (size_t)tc_layout(nb, groups_per_cta(KC, cpg, S)).total + 1024; }

template <int NB>
int max_active_clusters(int dev, int S, size_t smem) {
  const int ib = NB == 32 ? 0 : NB == 48 ? 1 : 2;
  if (dev < 0 || dev >= kMaxDevices) return 1;
  int v = g_clusters[dev][ib][S].load(std::memory_order_relaxed);
  if (v == 0) {
    auto kern = gemm_tc05_kernel<NB>;
    int n = 0;
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = tc_config<NB>(128 * S, S, smem, nullptr, attr, false);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
      n = 0;
      cudaGetLastError();   // the failed query's own error
    }
    v = n + 1;
    g_clusters[dev][ib][S].store(v, std::memory_order_relaxed);
  }
  return v - 1;
}

template <int NB>
int pick_splits(int N, int K, int G, int forced, int dev) {
  const int KC = K / 128, cpg = G / 128, tiles = (N + 127) / 128;
  if (forced > 0) {
    const int S = min(min(forced, kMaxSplits), KC);
    return tc_smem(NB, KC, cpg, S) <= (size_t)kSmemLimit ? S : 0;
  }
  const int sms = device_sms(dev);
  int best = 0;
  for (int S = 1; S <= min(kMaxSplits, KC); ++S) {
    const size_t smem = tc_smem(NB, KC, cpg, S);
    if (smem > (size_t)kSmemLimit) continue;
    if (best == 0) best = S;   // the smallest split that fits at all
    if (S > 1 && (tiles * S > sms || max_active_clusters<NB>(dev, S, smem) < tiles)) break;   // keep one wave
    best = S;
  }
  return best;
}

template <int NB>
cudaError_t launch_tc_t(const GemvParams& g, int S, bool pdl, cudaStream_t st) {
  auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  const int KC = g.K / 128;
  TcParams p{g.w, g.s, g.y, g.M, g.N, g.K, g.KG, g.cpg, g.flags, g.wait_guard, S, groups_per_cta(KC, g.cpg, S)};
  // activations as a [M, K] fp16 tensor; boxes of 64 k x NB rows, rows past M are filled with zeros
  CUtensorMap xmap;
  const cuuint64_t dims[2] = {(cuuint64_t)g.K, (cuuint64_t)g.M};
  const cuuint64_t strides[1] = {(cuuint64_t)g.K * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)NB};
  const cuuint32_t estride[2] = {1, 1};
  if (encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(g.x), dims, strides, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  const size_t smem = (size_t)tc_layout(NB, p.ngroups).total + 1024;
  auto kern = gemm_tc05_kernel<NB>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = tc_config<NB>(g.N, S, smem, st, attr, pdl);
  return cudaLaunchKernelEx(&cfg, kern, xmap, p);
}

}  // namespace

int gemm_tc05_splits(int M, int N, int K, int G, int forced) {
  if (M < 1 || M > 64 || K % 128 || G % 128 || K % G) return 0;
  int dev = 0;
  cudaGetDevice(&dev);
  switch (tc_nb(M)) {
    case 32: return pick_splits<32>(N, K, G, forced, dev);
    case 48: return pick_splits<48>(N, K, G, forced, dev);
    default: return pick_splits<64>(N, K, G, forced, dev);
  }
}

cudaError_t launch_gemm_tc05(const GemvParams& p, int splits, bool pdl, cudaStream_t st) {
  switch (tc_nb(p.M)) {
    case 32: return launch_tc_t<32>(p, splits, pdl, st);
    case 48: return launch_tc_t<48>(p, splits, pdl, st);
    default: return launch_tc_t<64>(p, splits, pdl, st);
  }
}

int gemm_tc_device_error() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int));
  return v;
}

void gemm_tc_clear_device_error() {
  int z = 0;
  cudaMemcpyToSymbol(g_tc_status, &z, sizeof(int));
}

}  // namespace lb
