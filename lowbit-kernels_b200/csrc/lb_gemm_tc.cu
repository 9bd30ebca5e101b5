// W4A16 skinny GEMM on the 5th-generation tensor cores: y[M, N] = x[M, K] * dequant(W)[N, K]^T, 17 <= M <= 64.
//
// Role of the reference's gemm_v5 (csrc/w4_gemv.cu:209-294), which ran mma.sync on a T4. Swap-AB: the weights
// are the 128-row A operand, the activation rows the N side of the MMA (NB = M rounded up to 16).
//   * 8 producer warps: each owns a 16-row slice of the CTA's 128-row tile. Per 128-wide K chunk a lane loads
//     the 16-byte words t of rows g and g+8 (the mma layout is the m16n8k16 A fragment), turns them into fp16
//     weights fp16_rn((u - 8) * scale) -- bit-identical to the dequantize kernel -- and writes them with
//     stmatrix into the canonical no-swizzle K-major layout the tensor core reads (8x8 core matrices of 16-byte
//     rows: the fragment registers of a warp are exactly four core matrices). Each lane keeps 8 chunks of its raw
//     words in flight in a private cp.async ring; the activations of a chunk are loaded one chunk ahead and
//     stored into the same canonical layout; the tile's scales are staged once.
//   * one MMA warp: a single elected thread issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=NB, K=16) per
//     k16 step with the fp32 accumulator in tensor memory, and tcgen05.commit releases the stage.
//   * the producers then read the accumulator with tcgen05.ld (each warp its 32-lane quarter of the tile) and
//     store fp16.
// Stages are handed over through mbarriers; every wait is bounded and records a status code instead of hanging,
// and tensor memory is released on every path.
#include "lb_common.cuh"
#include "lb_launch.h"

namespace lb {

// status word of this file's kernels (a bounded wait that gave up); read by gemm_tc_device_error()
__device__ int g_tc_status;

namespace {

constexpr int kProducerWarps = 8;
constexpr int kThreads = (kProducerWarps + 1) * 32;
constexpr int kStages = 2;        // A/B stages the tensor core reads
constexpr int kRing = 8;          // chunks of raw packed weights in flight per producer lane
constexpr int kRingLaneBytes = 32;  // per chunk: the lane's 16-byte words of rows g and g + 8
constexpr int kAStepBytes = 16 * 2 * 128;    // one k16 step of the 128-row A tile: 16 row groups x 2 k halves
constexpr int kAStageBytes = 8 * kAStepBytes;  // a 128-wide K chunk

__host__ __device__ inline int b_step_bytes(int nb) { return nb / 8 * 2 * 128; }

struct TcLayout {
  int a, b, ring, scales, bars, tmem_slot, total;
};

__host__ __device__ inline TcLayout tc_layout(int nb, int kg) {
  TcLayout L;
  L.a = 0;
  L.b = kStages * kAStageBytes;
  L.ring = L.b + kStages * 8 * b_step_bytes(nb);
  L.scales = L.ring + kRing * kProducerWarps * 32 * kRingLaneBytes;
  L.bars = L.scales + ((128 * kg * 2 + 15) & ~15);
  L.tmem_slot = L.bars + (2 * kStages + 1) * 8;
  L.total = L.tmem_slot + 16;
  return L;
}

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

// UMMA shared-memory descriptor, canonical K-major layout without swizzle: core matrices of 8 rows x 16 bytes;
// LBO = byte distance between the two k halves of a k16 step, SBO = between consecutive 8-row groups
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;   // descriptor version (sm_100)
  return d;                 // base offset 0, layout type 0 = no swizzle
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

}  // namespace

template <int NB>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc05_kernel(GemvParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const TcLayout L = tc_layout(NB, p.KG);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem_slot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = p.K, N = p.N, M = p.M, KC = K >> 7, KG = p.KG, cpg = p.cpg;
  const int n0 = blockIdx.x * 128;
  constexpr int kTmemCols = NB <= 32 ? 32 : 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], kProducerWarps * 32);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_fence_init();
  }
  if (warp == kProducerWarps) {   // the MMA warp owns the tensor-memory allocation
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

  if (warp == kProducerWarps) {
    // ------------------------------------------------------------------ MMA issuer
    // instruction descriptor: fp32 accumulate, fp16 A and B, both K-major, N = NB, M = 128
    const uint32_t idesc = (1u << 4) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    bool ok = true;
    for (int c = 0; c < KC; ++c) {
      const int s = c % kStages;
      if (ok) ok = wait_bounded(&full[s], (c / kStages) & 1);
      tc_fence_after();
      if (lane == 0 && ok) {
        const uint32_t a0 = smem_addr(smem + L.a + s * kAStageBytes);
        const uint32_t b0 = smem_addr(smem + L.b + s * 8 * b_step_bytes(NB));
#pragma unroll
        for (int st = 0; st < 8; ++st)
          umma_f16(tmem, smem_desc(a0 + st * kAStepBytes, 128, 256), smem_desc(b0 + st * b_step_bytes(NB), 128, 256),
                   idesc, (c > 0 || st > 0) ? 1u : 0u);
      }
      __syncwarp();
      if (lane == 0) umma_commit(&empty[s]);   // arrives when this chunk's MMAs have read the stage
    }
    __syncwarp();
    if (lane == 0) umma_commit(done);
  } else {
    // ------------------------------------------------------------------ producers
    const int g = lane >> 2, t = lane & 3;
    const int pt = threadIdx.x;   // producer thread 0..255
    const int ra = min(n0 + 16 * warp + g, N - 1), rb = min(n0 + 16 * warp + g + 8, N - 1);  // tail rows: N-1
    const uint4* wa = reinterpret_cast<const uint4*>(p.w) + (size_t)ra * (K >> 5) + t;
    const uint4* wb = reinterpret_cast<const uint4*>(p.w) + (size_t)rb * (K >> 5) + t;
    // this lane's private ring of raw packed words: slot c % kRing holds (row g, row g + 8) of chunk c
    const uint32_t ring = smem_addr(smem + L.ring) + (uint32_t)pt * (kRing * kRingLaneBytes);
    auto issue = [&](int c) {
      if (c < KC) {
        cp_async_cg16(ring + (c % kRing) * kRingLaneBytes, wa + 4 * c);
        cp_async_cg16(ring + (c % kRing) * kRingLaneBytes + 16, wb + 4 * c);
      }
      cp_async_group_commit();
    };
    // weights and scales may be fetched before the stream dependency resolves only when the caller declared
    // them static (kFlagEarlyWeights); otherwise wait first
    if (!(p.flags & kFlagEarlyWeights) && p.wait_guard) pdl_wait();
#pragma unroll
    for (int c = 0; c < kRing - 1; ++c) issue(c);
    // the tile's scales, rows n0 .. n0 + 127 (tail rows repeat row N - 1)
    uint16_t* sc = reinterpret_cast<uint16_t*>(smem + L.scales);
    const uint16_t* sg = reinterpret_cast<const uint16_t*>(p.s);
    for (int i = pt; i < 128 * KG; i += kProducerWarps * 32) {
      const int r = i / KG, gidx = i - r * KG;
      sc[i] = ldg_u16(sg + (size_t)min(n0 + r, N - 1) * KG + gidx);
    }
    named_barrier(1, kProducerWarps * 32);
    if (p.wait_guard) pdl_wait();   // activations and outputs follow the stream order from here on
    // stmatrix row addresses: lane L writes row (L & 7) of core matrix j = L >> 3, which is row group
    // 2 * warp + (j & 1) and k half j >> 1 of every k16 step
    const int jm = lane >> 3;
    const uint32_t a_row = (uint32_t)((((2 * warp + (jm & 1)) * 2 + (jm >> 1)) * 128) + (lane & 7) * 16);
    const int sra = (16 * warp + g) * KG, srb = (16 * warp + g + 8) * KG;
    // activations: NB rows (row m >= M repeats row M - 1) x 16 pieces of 8 k per chunk, kXPer pieces per thread,
    // loaded into registers one chunk ahead and stored into the stage once the tensor core has released it
    constexpr int kXPer = NB * 16 / (kProducerWarps * 32);
    const uint8_t* xg = reinterpret_cast<const uint8_t*>(p.x);
    uint4 xv[kXPer];
    auto load_x = [&](int c) {
#pragma unroll
      for (int j = 0; j < kXPer; ++j) {
        const int it = pt + j * kProducerWarps * 32, m = it >> 4, piece = it & 15;
        const uint8_t* src = xg + (size_t)min(m, M - 1) * (K * 2) + (size_t)c * 256 + piece * 16;
        asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(xv[j].x), "=r"(xv[j].y), "=r"(xv[j].z), "=r"(xv[j].w)
                     : "l"(src));
      }
    };
    load_x(0);
    bool ok = true;
    for (int c = 0; c < KC; ++c) {
      const int s = c % kStages;
      issue(c + kRing - 1);
      cp_async_group_wait<kRing - 1>();   // this lane's copies of chunk c have landed (groups complete in order)
      const uint8_t* slot = smem + L.ring + pt * (kRing * kRingLaneBytes) + (c % kRing) * kRingLaneBytes;
      const uint4 qa = *reinterpret_cast<const uint4*>(slot);
      const uint4 qb = *reinterpret_cast<const uint4*>(slot + 16);
      const int grp = cpg == 1 ? c : c / cpg;
      const uint32_t s2a = (uint32_t)sc[sra + grp] * 0x10001u, s2b = (uint32_t)sc[srb + grp] * 0x10001u;
      if (c >= kStages && ok) ok = wait_bounded(&empty[s], ((c / kStages) - 1) & 1);
      tc_fence_after();
      // activations of chunk c into the canonical layout: piece (m, 8 k) -> k16 step, k half, core-matrix row
      uint8_t* bst = smem + L.b + s * 8 * b_step_bytes(NB);
#pragma unroll
      for (int j = 0; j < kXPer; ++j) {
        const int it = pt + j * kProducerWarps * 32, m = it >> 4, piece = it & 15;
        *reinterpret_cast<uint4*>(bst + (piece >> 1) * b_step_bytes(NB) + ((m >> 3) * 2 + (piece & 1)) * 128 +
                                  (m & 7) * 16) = xv[j];
      }
      if (c + 1 < KC) load_x(c + 1);
      // weights of chunk c: fp16_rn((u - 8) * scale), four core matrices per k16 step
      const uint32_t abase = smem_addr(smem + L.a + s * kAStageBytes) + a_row;
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
      fence_async_smem();   // generic-proxy writes (stmatrix, st.shared) become visible to the tensor core
      tc_fence_before();
      mbar_arrive(&full[s]);
    }
    cp_async_group_wait<0>();   // no ring copy is left in flight
    // epilogue: wait for the last MMA, then each warp reads its 32 lanes (rows) of the accumulator
    if (ok) ok = wait_bounded(done, 0);
    tc_fence_after();
    const int quarter = warp & 3, half = warp >> 2;   // warps q and q + 4 share lanes 32q..: blocks alternate
    const int row = n0 + 32 * quarter + lane;
#pragma unroll
    for (int blk = half; blk < NB / 16; blk += 2) {
      const int col0 = blk * 16;
      uint32_t v[16];
      tmem_ld16(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)col0, v);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (ok && row < N) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = col0 + j;
          if (m < M) p.y[(size_t)m * N + row] = __float2half_rn(__uint_as_float(v[j]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kProducerWarps) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

template <int NB>
static cudaError_t launch_tc_t(const GemvParams& p, bool pdl, cudaStream_t st) {
  const TcLayout L = tc_layout(NB, p.KG);
  auto kern = gemm_tc05_kernel<NB>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N + 127) / 128, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

size_t gemm_tc05_smem_bytes(int M, int K, int G) {
  const int nb = M <= 32 ? 32 : M <= 48 ? 48 : 64;
  return (size_t)tc_layout(nb, K / G).total;
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

cudaError_t launch_gemm_tc05(const GemvParams& p, bool pdl, cudaStream_t st) {
  if (p.M <= 32) return launch_tc_t<32>(p, pdl, st);
  if (p.M <= 48) return launch_tc_t<48>(p, pdl, st);
  return launch_tc_t<64>(p, pdl, st);
}

}  // namespace lb
