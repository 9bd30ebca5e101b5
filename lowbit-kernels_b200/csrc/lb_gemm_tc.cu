// W4A16 skinny GEMM on the 5th-generation tensor cores: y[M, N] = x[M, K] * dequant(W)[N, K]^T, M <= 64.
//
// Role of the reference's gemm_v5 (csrc/w4_gemv.cu:209-294), which ran mma.sync on a T4. Swap-AB: the weights
// are the 128-row A operand, the activation rows the N side of the MMA (NB = M rounded up to 32, 48 or 64).
// Grid: one column of CTAs per 128-row tile of W; the S CTAs of a column form a thread-block cluster that splits
// K into S contiguous ranges and adds its fp32 partial tiles through distributed shared memory (no workspace).
//   * weight loader warp: one thread copies each 128-wide K chunk of the tile's packed weights (128 rows x 64
//     bytes, mma layout) with a 2-D tensor copy (64-byte swizzle) into an 8-deep stage ring.
//   * activation loader warp: one thread copies the chunk's activations with two 2-D tensor copies (64 k x NB
//     rows, 128-byte swizzle; rows >= M read as zeros) into a 6-deep stage ring.
//   * 8 dequantizing warps, two per 32-lane quarter of tensor memory, each taking one 64-wide K half of every
//     chunk: a thread takes its row's 32 bytes of that half, turns them into fp16 weights
//     fp16_rn((u - 8) * scale) -- bit-identical to the dequantize kernel -- and stores the 32 packed columns
//     into tensor memory with tcgen05.st (3 stages): the A operand never passes through shared memory.
//   * MMA warp: a single thread issues tcgen05.mma.cta_group::1.kind::f16 with A in tensor memory (M=128, N=NB,
//     K=16 per instruction) and the fp32 accumulator in tensor memory. One tcgen05.commit per chunk (to a ring of
//     completion barriers) releases both the activation stage and the tensor-memory stage; the next chunk's
//     barriers are polled while this chunk's MMAs run, so the tensor core is fed back to back (one 128 x N x 16
//     MMA costs about 100 cycles for any N <= 128 on B200: this, not memory, bounds the kernel at small M).
//   * the dequantizing warps read the accumulator with tcgen05.ld and store fp16, or, split across a cluster,
//     park fp32 partials in shared memory that every CTA of the cluster sums for its share of the outputs in a
//     fixed rank order (deterministic).
// Stages are handed over through mbarriers; every wait is bounded and records a status code instead of hanging,
// no copy is left in flight at exit, and tensor memory is released on every path.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>

#include "lb_launch.h"
#include "lb_tma.cuh"

namespace lb {

// status word of this file's kernels (a bounded wait that gave up); read by gemm_tc_device_error()
__device__ int g_tc_status;

namespace {

constexpr int kDequantWarps = 8;
constexpr int kMmaWarp = 8;
constexpr int kWLoadWarp = 9;
constexpr int kXLoadWarp = 10;
constexpr int kThreads = 11 * 32;
constexpr int kWStages = 8;           // packed weight chunks in flight
constexpr int kWStageBytes = 128 * 64;
constexpr int kBStages = 6;           // activation chunks in flight
constexpr int kAStages = 3;           // dequantized chunks in tensor memory
constexpr int kTmemCols = 256;        // accumulator (<= 64 columns) + three A stages of 64 columns
constexpr int kTmemA = 64;            // first column of A stage 0
constexpr int kMaxSplits = 8;         // portable cluster size
constexpr int kSmemLimit = 227 * 1024;

// an activation stage: two 64-wide k halves of NB rows x 128 bytes (each half a whole number of 1024-byte
// swizzle atoms)
__host__ __device__ inline int b_stage_bytes(int nb) { return nb * 256; }

struct TcLayout {
  int w, b, scales, bars, tmem_slot, total;
};

// offsets from the 1024-byte aligned start of dynamic shared memory; `ngroups` = scale groups per CTA
__host__ __device__ inline TcLayout tc_layout(int nb, int ngroups) {
  TcLayout L;
  L.w = 0;
  L.b = kWStages * kWStageBytes;
  L.scales = L.b + kBStages * b_stage_bytes(nb);
  L.bars = L.scales + ((128 * ngroups * 2 + 15) & ~15);
  L.tmem_slot = L.bars + (2 * kWStages + 2 * kBStages + kAStages + 1) * 8;
  L.total = L.tmem_slot + 16;
  return L;
}

__host__ __device__ inline int tc_nb(int m) { return m <= 32 ? 32 : m <= 48 ? 48 : 64; }

struct TcParams {
  const void* s;  // fp16 [N, K / G]
  __half* y;      // fp16 [M, N]
  int M, N, K, KG, cpg;
  int flags;
  int wait_guard;  // always 1 (see pdl_wait_after_loads)
  int splits;      // CTAs per cluster splitting K (gridDim.y)
  int ngroups;     // scale groups staged per CTA (the largest K range's)
  const __half* bias;   // fp16 [N] added to every output row, or null
};

// both phases, polled together (each poll of a completed barrier still costs a full shared-memory round trip)
__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity) {
  return lb::wait_bounded(bar, parity, &g_tc_status);
}

__device__ __forceinline__ bool wait_pair(uint64_t* a, uint32_t pa, uint64_t* b, uint32_t pb) {
  bool da = false, db = false;
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (!da) da = mbar_try_wait(a, pa);
    if (!db) db = mbar_try_wait(b, pb);
    if (da && db) return true;
  }
  atomicExch(&g_tc_status, kErrBarrierTimeout);
  return false;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor (sm_100 format: version 1 at bit 46), 128-byte swizzle, K-major: rows of 128
// bytes (64 fp16 k), 8-row atoms of 1024 bytes (SBO); a k16 step inside the atom starts 32 bytes further (the
// swizzle is applied to the computed addresses, atoms 1024-byte aligned); layout type 2 at bits 61-63
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;                  // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;        // SBO
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// D[tmem] (+)= A[tmem] * B[smem]^T
__device__ __forceinline__ void umma_ts_f16(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
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

// 32 consecutive columns of this thread's tensor-memory lane
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]),
      "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]),
      "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

}  // namespace

template <int NB>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc05_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                     const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const TcLayout L = tc_layout(NB, p.ngroups);
  uint64_t* full_w = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty_w = full_w + kWStages;
  uint64_t* full_b = empty_w + kWStages;
  uint64_t* empty_b = full_b + kBStages;
  uint64_t* full_a = empty_b + kBStages;       // dequantized chunk in tensor memory
  uint64_t* done = full_a + kAStages;          // all MMAs complete
  uint64_t* mma_done = empty_b;                // chunk i's MMAs complete: ring of kBStages (= empty_b)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem_slot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = p.N, M = p.M, S = p.splits;
  const int n0 = blockIdx.x * 128;
  const int KC = p.K >> 7;
  const int c_begin = (KC * (int)blockIdx.y) / S, nc = (KC * ((int)blockIdx.y + 1)) / S - c_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&full_w[s], 1);
      mbar_init(&empty_w[s], kDequantWarps);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&full_b[s], 1);
      mbar_init(&empty_b[s], 1);
    }
    for (int s = 0; s < kAStages; ++s) mbar_init(&full_a[s], kDequantWarps * 32);
    mbar_init(done, 1);
    mbar_fence_init();
  }
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
    // ------------------------------------------------------------------ MMA issuer (one thread)
    if (lane == 0) {
      // instruction descriptor: fp32 accumulate, fp16 A and B, both K-major, N = NB, M = 128
      const uint32_t idesc = (1u << 4) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
      bool ok = nc == 0 || wait_pair(&full_a[0], 0, &full_b[0], 0);
      for (int i = 0; i < nc && ok; ++i) {
        const int sa = i % kAStages, sb = i % kBStages;
        tc_fence_after();
        const uint32_t a0 = tmem + kTmemA + 64 * sa;
        const uint32_t b0 = smem_addr(smem + L.b + sb * b_stage_bytes(NB));
#pragma unroll
        for (int st = 0; st < 8; ++st)
          umma_ts_f16(tmem, a0 + 8 * st, smem_desc_sw128(b0 + (st >> 2) * (NB * 128) + (st & 3) * 32), idesc,
                      (i > 0 || st > 0) ? 1u : 0u);
        // the next chunk's operands, polled while these MMAs run
        const int j = i + 1;
        if (j < nc) ok = wait_pair(&full_a[j % kAStages], (j / kAStages) & 1, &full_b[j % kBStages], (j / kBStages) & 1);
        umma_commit(&mma_done[sb]);   // arrives when chunk i's MMAs (and all earlier ones) have completed
      }
      umma_commit(done);
      wait_bounded(done, 0);   // no MMA in flight past this point
    }
    __syncwarp();
  } else if (warp == kWLoadWarp) {
    // ------------------------------------------------------------------ packed weights
    if (lane == 0) {
      tma_prefetch_map(&wmap);
      // static weights may be fetched before the stream dependency resolves (kFlagEarlyWeights)
      if (!(p.flags & kFlagEarlyWeights) && p.wait_guard) pdl_wait();
      run_loader(nc, kWStages, full_w, empty_w, kWStageBytes, &g_tc_status, [&](int i, int s) {
        tma_load_2d(smem + L.w + s * kWStageBytes, &wmap, (c_begin + i) * 64, n0, &full_w[s]);
      });
    }
    __syncwarp();
  } else if (warp == kXLoadWarp) {
    // ------------------------------------------------------------------ activations
    if (lane == 0) {
      tma_prefetch_map(&xmap);
      if (p.wait_guard) pdl_wait();   // the activations come from the previous kernel in the stream
      run_loader(nc, kBStages, full_b, empty_b, b_stage_bytes(NB), &g_tc_status, [&](int i, int s) {
        uint8_t* dst = smem + L.b + s * b_stage_bytes(NB);
        tma_load_2d(dst, &xmap, (c_begin + i) * 128, 0, &full_b[s]);
        tma_load_2d(dst + NB * 128, &xmap, (c_begin + i) * 128 + 64, 0, &full_b[s]);
      });
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ dequantizing warps
    const int quarter = warp & 3, hh = warp >> 2;   // TMEM lanes 32q.. ; K half hh of every chunk
    const int row = 32 * quarter + lane;             // row of the tile = TMEM lane
    const int cpg = p.cpg;
    if (!(p.flags & kFlagEarlyWeights) && p.wait_guard) pdl_wait();
    // scales of the CTA's groups, rows n0 .. n0 + 127 (tail rows repeat row N - 1)
    const int g0 = c_begin / cpg, ng = (c_begin + nc - 1) / cpg - g0 + 1;
    uint16_t* sc = reinterpret_cast<uint16_t*>(smem + L.scales);
    {
      // batches of 16 independent loads in flight (a load-store loop would pay one memory latency per scale)
      constexpr int kBatch = 16;
      const uint16_t* srow = reinterpret_cast<const uint16_t*>(p.s) + (size_t)min(n0 + row, N - 1) * p.KG + g0;
      for (int gb = hh; gb < ng; gb += 2 * kBatch) {
        uint16_t v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) v[j] = gb + 2 * j < ng ? ldg_u16(srow + gb + 2 * j) : (uint16_t)0;
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
          if (gb + 2 * j < ng) sc[row * p.ngroups + gb + 2 * j] = v[j];
      }
    }
    named_barrier(1, kDequantWarps * 32);
    if (p.wait_guard) pdl_wait();   // the outputs are written in stream order
    // the row's 64 bytes sit at row * 64 in a weight stage, 16-byte word t at slot t ^ ((row >> 1) & 3); u32 qd
    // of word t holds the pairs of columns 16qd + t (+4, +8, +12), column j = fp16 weights k 2j, 2j + 1: K half
    // hh (columns 32hh ..) is u32s 2hh and 2hh + 1 of every word
    const uint32_t wrow = smem_addr(smem + L.w) + (uint32_t)row * 64 + 8u * hh;
    const uint32_t wsw = (uint32_t)(row >> 1) & 3u;
    const uint32_t tlane = (uint32_t)(32 * quarter) << 16;
    // chunk i's words and scale are fetched during chunk i - 1; its fp16 values are computed before waiting for
    // the tensor-memory stage (chunk i - kAStages's MMAs) to free up
    uint2 q[4];
    uint32_t s2 = 0;
    auto fetch = [&](int i) -> bool {
      const int sw = i % kWStages;
      const bool got = wait_bounded(&full_w[sw], (i / kWStages) & 1);
#pragma unroll
      for (int t = 0; t < 4; ++t) q[t] = lds64(wrow + sw * kWStageBytes + ((t ^ wsw) << 4));
      const int grp = (cpg == 1 ? c_begin + i : (c_begin + i) / cpg) - g0;
      s2 = (uint32_t)sc[row * p.ngroups + grp] * 0x10001u;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_w[sw]);
      return got;
    };
    bool ok = nc == 0 || fetch(0);
    for (int i = 0; i < nc; ++i) {
      const int sa = i % kAStages;
      uint32_t v[32];
#pragma unroll
      for (int d = 0; d < 2; ++d) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint32_t w = d ? q[t].y : q[t].x;
          v[16 * d + t] = hmul2_bits(q_pair_lo(w), s2);
          v[16 * d + 4 + t] = hmul2_bits(q_pair_hi(w), s2);
          v[16 * d + 8 + t] = hmul2_bits(q_pair_lo(w >> 8), s2);
          v[16 * d + 12 + t] = hmul2_bits(q_pair_hi(w >> 8), s2);
        }
      }
      if (i + 1 < nc && ok) ok = fetch(i + 1);
      if (i >= kAStages && ok) {
        const int c = i - kAStages;   // the chunk whose MMAs last read this stage
        ok = wait_bounded(&mma_done[c % kBStages], (c / kBStages) & 1);
      }
      __syncwarp();   // tcgen05.st is warp-collective
      tc_fence_after();
      tmem_st32(tmem + tlane + kTmemA + 64 * sa + 32 * hh, v);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&full_a[sa]);
    }
    // epilogue: wait for the last MMA, then each warp reads its 32 lanes (rows) of the accumulator; warps q and
    // q + 4 share lanes 32q.. and alternate 16-column blocks
    if (ok) ok = wait_bounded(done, 0);
    __syncwarp();   // tcgen05.ld is warp-collective
    tc_fence_after();
    float* red = reinterpret_cast<float*>(smem + L.w);   // [m][128] fp32 partials (the weight ring is idle now)
#pragma unroll
    for (int blk = hh; blk < NB / 16; blk += 2) {
      const int col0 = blk * 16;
      uint32_t v[16];
      tmem_ld16(tmem + tlane + (uint32_t)col0, v);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (S == 1) {
        if (n0 + row < N) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (col0 + j < M) p.y[(size_t)(col0 + j) * N + n0 + row] = out_half(__uint_as_float(v[j]), p.bias, n0 + row);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (col0 + j < M) red[(col0 + j) * 128 + row] = __uint_as_float(v[j]);
      }
    }
  }

  __syncwarp();
  if (S > 1) {
    // every CTA of the cluster sums its share of the M x 128 outputs over all ranks' partials, in rank order
    cluster_sync_all();
    const int e4 = 32 * M, r = (int)cluster_rank();
    const int e_begin = (e4 * r) / S, e_end = (e4 * (r + 1)) / S;
    const uint32_t red0 = smem_addr(smem + L.w);
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
        if (n0 + row4 + j < N) yo[j] = out_half(a[j], p.bias, n0 + row4 + j);
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
    cudaLaunchConfig_t cfg = tc_config(128 * S, S, smem, nullptr, attr, false);
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
  TcParams p{g.s, g.y, g.M, g.N, g.K, g.KG, g.cpg, g.flags, g.wait_guard, S, groups_per_cta(KC, g.cpg, S), g.bias};
  const cuuint32_t estride[2] = {1, 1};
  // activations as a [M, K] fp16 tensor; boxes of 64 k x NB rows, rows past M are filled with zeros
  CUtensorMap xmap, wmap;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)g.K, (cuuint64_t)g.M};
    const cuuint64_t strides[1] = {(cuuint64_t)g.K * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)NB};
    if (encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(g.x), dims, strides, box, estride,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  // packed weights as a [N, K / 2] byte tensor; boxes of one 64-byte chunk x 128 rows, rows past N read as zeros
  {
    const cuuint64_t dims[2] = {(cuuint64_t)g.K / 2, (cuuint64_t)g.N};
    const cuuint64_t strides[1] = {(cuuint64_t)g.K / 2};
    const cuuint32_t box[2] = {64, 128};
    if (encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(g.w), dims, strides, box, estride,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  const size_t smem = (size_t)tc_layout(NB, p.ngroups).total + 1024;
  auto kern = gemm_tc05_kernel<NB>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = tc_config(g.N, S, smem, st, attr, pdl);
  return cudaLaunchKernelEx(&cfg, kern, xmap, wmap, p);
}

}  // namespace

bool encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  auto encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estride[2] = {1, 1};
  return encode(map, type, 2, const_cast<void*>(base), dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

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
