// W4A16 skinny GEMM, 9..64 activation rows: y[M, N] = x[M, K] * dequant(W)[N, K]^T on mma.sync tiles, every
// operand landed in shared memory by the tensor-memory accelerator.
//
// Role of the reference's gemm_v5 (csrc/w4_gemv.cu:209-294) for the row counts between the decode GEMV and the
// prefill path. At these sizes the work is a stream of 4-bit weights (N K / 2 bytes) against a few activation
// rows that every weight row needs, so the design keeps each weight byte read from HBM once and each activation
// byte read from L2 once per CTA:
//   * a CTA owns 64 RT weight rows (4 consumer warps x RT 16-row tiles) and a contiguous K range; the S CTAs of a
//     column of the grid form a thread-block cluster that splits K and adds its fp32 partial tiles through
//     distributed shared memory in a fixed rank order (deterministic, no workspace). (128-row CTAs of 8 warps
//     measured slower: narrow layers then need splits that leave each CTA one or two chunks);
//   * a producer thread streams the range through a ring of stages, one 128-wide K chunk each: the CTA's packed
//     weight rows (a 2-D tensor copy of 64-byte rows) and the chunk's activations (two 2-D tensor copies of 64 k x
//     8 MT rows, 128-byte swizzle, rows past M read as zeros), completing on the stage's mbarrier; the weights of
//     the first stages are requested before the wait on the previous kernel in the stream;
//   * every consumer warp reads the chunk's activation fragments once per 32 k (ldmatrix, conflict-free through
//     the swizzle) and uses each for its RT row tiles, so shared-memory traffic per weight is 2 M / (16 RT) bytes;
//     its weights come from the stage as one 16-byte read per row and chunk, are decoded with the lop3 / f16x2
//     sequence of the other kernels and scaled in f16x2 -- fp16_rn((u - 8) * scale), bit-identical to the
//     dequantize kernel -- then fed to m16n8k16 MMAs accumulating in fp32 over the whole range (the arithmetic of
//     dequantize + an fp16 GEMM with fp32 accumulation, as the reference's tensor-core kernel and cuBLAS do).
//     With EXACT (M <= 16), the products of a chunk are instead formed from the exact nibble values and scaled per
//     group in fp32, as the decode GEMV does;
//   * a warp releases a stage with one mbarrier arrive after its last MMA on it; the MMAs of a 32-k block run
//     k16-step-outer, so an accumulator's next MMA comes RT MT instructions after its previous one.
// Every wait is bounded and records a status code instead of hanging; the producer waits for its own last copies
// so that none is in flight when the CTA exits.
#include <cuda.h>

#include <atomic>

#include "lb_launch.h"
#include "lb_tma.cuh"

namespace lb {

__device__ int g_mma_status;   // a bounded wait in this file's kernel gave up; read by gemm_mma_device_error()

namespace {

constexpr int kConsumerWarps = 4;                        // each owns RT 16-row tiles
constexpr int kMmaThreads = (kConsumerWarps + 1) * 32;   // + the producer warp
constexpr int kRingBudget = 96 * 1024;                     // stage ring per CTA: two CTAs fit one SM (a 64 KB
                                                           // ring for three measured slower: too shallow)
constexpr int kMaxStages = 8;
constexpr int kMaxClusterSplits = 8;

__host__ __device__ constexpr int x_stage_bytes(int mt) { return mt * 8 * 256; }   // 2 halves x 8 MT rows x 128 B
__host__ __device__ constexpr int w_stage_bytes(int rt) { return kConsumerWarps * rt * 16 * 64; }
__host__ __device__ constexpr int stage_bytes(int mt, int rt) { return x_stage_bytes(mt) + w_stage_bytes(rt); }
__host__ __device__ constexpr int ring_stages(int mt, int rt) {
  return kRingBudget / stage_bytes(mt, rt) < kMaxStages ? kRingBudget / stage_bytes(mt, rt) : kMaxStages;
}
// partial tile [8 MT][rows + 4] fp32 (the pad keeps the parking stores on distinct banks)
__host__ __device__ constexpr int part_pitch(int rt) { return kConsumerWarps * rt * 16 + 4; }
__host__ __device__ constexpr int part_bytes(int mt, int rt) { return mt * 8 * part_pitch(rt) * 4; }
__host__ __device__ constexpr int ring_bytes(int mt, int rt) {
  return ring_stages(mt, rt) * stage_bytes(mt, rt) > part_bytes(mt, rt) ? ring_stages(mt, rt) * stage_bytes(mt, rt)
                                                                      : part_bytes(mt, rt);
}
// dynamic shared memory: 1024-byte alignment slack + the ring (or the partial tile) + the barriers + the CTA's
// scales ([rows][ngroups] fp16)
__host__ __device__ constexpr int scales_offset(int mt, int rt) { return ring_bytes(mt, rt) + 2 * kMaxStages * 8; }
__host__ __device__ constexpr int mma_smem_bytes(int mt, int rt, int ngroups) {
  return 1024 + scales_offset(mt, rt) + ((kConsumerWarps * rt * 16 * ngroups * 2 + 15) & ~15);
}

struct MmaParams {
  const void* s;   // fp16 [N, K / G]
  __half* y;       // fp16 [M, N]
  const __half* bias;
  int M, N, K, KG, cpg;
  int flags;
  int wait_guard;
  int splits;
  int ngroups;   // scale groups staged per CTA (the largest K range's)
};

__device__ __forceinline__ bool wait_full(uint64_t* bar, uint32_t parity) { return wait_bounded(bar, parity, &g_mma_status); }

}  // namespace

template <int MT, int RT, bool EXACT>
__global__ void __launch_bounds__(kMmaThreads, 2)
    gemm_mma_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                    const MmaParams p) {
  constexpr int D = ring_stages(MT, RT);
  constexpr int XB = x_stage_bytes(MT), SB = stage_bytes(MT, RT), ROWS = kConsumerWarps * RT * 16;
  constexpr int PP = part_pitch(RT);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring_bytes(MT, RT));
  uint64_t* empty = full + kMaxStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int N = p.N, M = p.M, S = p.splits;
  const int n0 = blockIdx.x * ROWS;
  const int KC = p.K >> 7;
  const int c_begin = (KC * (int)blockIdx.y) / S, nc = (KC * ((int)blockIdx.y + 1)) / S - c_begin;
  const bool producer = warp == kConsumerWarps;

  if (threadIdx.x == 0) {
    for (int s = 0; s < D; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // chunk i of the range into stage s: the weight rows, then the two 64-k halves of the activations
  auto load_weights = [&](int i, int s) {
    mbar_arrive_expect_tx(&full[s], SB);
    tma_load_2d(smem + s * SB + XB, &wmap, (c_begin + i) * 64, n0, &full[s]);
  };
  auto load_x = [&](int i, int s) {
    tma_load_2d(smem + s * SB, &xmap, (c_begin + i) * 128, 0, &full[s]);
    tma_load_2d(smem + s * SB + XB / 2, &xmap, (c_begin + i) * 128 + 64, 0, &full[s]);
  };
  if (producer) {
    // ------------------------------------------------------------------ producer (one thread)
    if (lane == 0) {
      tma_prefetch_map(&wmap);
      tma_prefetch_map(&xmap);
      const bool early = (p.flags & kFlagEarlyWeights) != 0;
      if (!early && p.wait_guard) pdl_wait();
      const int first = nc < D ? nc : D;
      // the weights of the first stages do not depend on the previous kernel: requested before its wait
      for (int i = 0; i < first; ++i) load_weights(i, i);
      if (early && p.wait_guard) pdl_wait();
      for (int i = 0; i < first; ++i) load_x(i, i);
      int issued = first;
      for (int i = D; i < nc; ++i) {
        const int s = i % D;
        if (!wait_bounded(&empty[s], ((i / D) - 1) & 1, &g_mma_status)) break;
        load_weights(i, s);
        load_x(i, s);
        issued = i + 1;
      }
      // none of this CTA's copies may still be in flight when it exits
      for (int i = issued > D ? issued - D : 0; i < issued; ++i) wait_full(&full[i % D], (i / D) & 1);
    }
    __syncwarp();
  }

  // the CTA's scales, [ROWS][ng] for groups g0 .. g0 + ng - 1, fetched once with every load of a batch in flight
  // (the tensor copies run meanwhile); tail rows repeat row N - 1
  const int KG = p.KG, cpg = p.cpg, NG = p.ngroups;
  const int g0 = c_begin / cpg, ng = nc > 0 ? (c_begin + nc - 1) / cpg - g0 + 1 : 0;
  uint16_t* sc = reinterpret_cast<uint16_t*>(smem + scales_offset(MT, RT));
  constexpr int kCT = kConsumerWarps * 32;
  if (!producer) {
    const uint16_t* sp = reinterpret_cast<const uint16_t*>(p.s);
    const int total = ROWS * ng;
    constexpr int kBatch = 8;
    for (int base = threadIdx.x; base < total; base += kCT * kBatch) {
      uint16_t v[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int idx = base + kCT * j, row = idx / ng;
        if (idx < total) v[j] = ldg_u16(sp + (size_t)min(n0 + row, N - 1) * KG + g0 + (idx - row * ng));
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int idx = base + kCT * j, row = idx / ng;
        if (idx < total) sc[row * NG + idx - row * ng] = v[j];
      }
    }
    named_barrier(1, kCT);
  }
  // this lane's scales: row g of tile r at sc_lane + 16 r NG, row g + 8 another 8 NG further
  const uint16_t* sc_lane = sc + (16 * RT * warp + g) * NG;
  // ldmatrix: lane L addresses row L & 7 of 8x8 matrix L >> 3 (k piece (L >> 3) of a 32-k block); in a swizzled
  // 128-byte row r, 16-byte piece j sits at slot j ^ (r & 7)
  const uint32_t xo0 = (uint32_t)(lane & 7) * 128u + ((uint32_t)((lane >> 3) ^ (lane & 7)) << 4);
  const uint32_t xo1 = (uint32_t)(lane & 7) * 128u + ((uint32_t)((4 + (lane >> 3)) ^ (lane & 7)) << 4);
  const uint32_t wo = (uint32_t)(16 * RT * warp + g) * 64u + (uint32_t)t * 16u;
  const uint32_t ring = smem_addr(smem);

  float acc[RT][MT][4];
#pragma unroll
  for (int r = 0; r < RT; ++r)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[r][mt][i] = 0.f;

  // Software-pipelined: the activation fragments of the next 32-k block (at a chunk's last block: the next
  // chunk's first block and weights, after waiting for its stage) are read before this block's MMAs are issued,
  // so a single warp per scheduler keeps the tensor pipe fed across the shared-memory latency.
  bool ok = true;
  const int my_nc = producer ? 0 : nc;
  uint4 qa[RT], qb[RT];
  uint32_t xb[2][MT][4];
  auto load_w = [&](int i, uint4 (&a)[RT], uint4 (&b)[RT]) {
    const uint32_t ws = ring + (i % D) * SB + XB + wo;
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      a[r] = lds128(ws + r * 1024);
      b[r] = lds128(ws + r * 1024 + 512);
    }
  };
  auto load_xb = [&](uint32_t (&dst)[MT][4], int i, int qd) {
    const uint32_t xq = ring + (i % D) * SB + (uint32_t)(qd >> 1) * (XB / 2) + ((qd & 1) ? xo1 : xo0);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) ldsm_x4(dst[mt], xq + mt * 1024);
  };
  if (my_nc > 0) {
    ok = wait_full(&full[0], 0);
    load_w(0, qa, qb);
    load_xb(xb[0], 0, 0);
  }
  for (int i = 0; i < my_nc; ++i) {
    const int s = i % D;
    const int gi = (cpg == 1 ? c_begin + i : (c_begin + i) / cpg) - g0;
    uint32_t s2a[RT], s2b[RT];
    float fa[RT], fb[RT];
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      const uint16_t sa = sc_lane[16 * r * NG + gi], sb = sc_lane[(16 * r + 8) * NG + gi];
      s2a[r] = (uint32_t)sa * 0x10001u;
      s2b[r] = (uint32_t)sb * 0x10001u;
      fa[r] = __half2float(__ushort_as_half(sa));
      fb[r] = __half2float(__ushort_as_half(sb));
    }
    float d[EXACT ? RT : 1][EXACT ? MT : 1][4];
    if constexpr (EXACT) {
#pragma unroll
      for (int r = 0; r < RT; ++r)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int j = 0; j < 4; ++j) d[r][mt][j] = 0.f;
    }
    uint4 qa_n[RT], qb_n[RT];
#pragma unroll
    for (int qd = 0; qd < 4; ++qd) {
      if (qd < 3) {
        load_xb(xb[(qd + 1) & 1], i, qd + 1);
      } else if (i + 1 < my_nc) {
        if (ok) ok = wait_full(&full[(i + 1) % D], ((i + 1) / D) & 1);
        load_w(i + 1, qa_n, qb_n);
        load_xb(xb[0], i + 1, 0);
      }
      uint32_t f[RT][8];
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        const uint32_t w0 = (&qa[r].x)[qd], w1 = (&qb[r].x)[qd];
        f[r][0] = q_pair_lo(w0); f[r][1] = q_pair_lo(w1); f[r][2] = q_pair_hi(w0); f[r][3] = q_pair_hi(w1);
        f[r][4] = q_pair_lo(w0 >> 8); f[r][5] = q_pair_lo(w1 >> 8);
        f[r][6] = q_pair_hi(w0 >> 8); f[r][7] = q_pair_hi(w1 >> 8);
        if constexpr (!EXACT) {
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            f[r][j] = hmul2_bits(f[r][j], s2a[r]);
            f[r][j + 1] = hmul2_bits(f[r][j + 1], s2b[r]);
          }
        }
      }
      // k16 step 2 qd (fragment words 0-3) over every accumulator, then step 2 qd + 1 (words 4-7): an
      // accumulator's next MMA is RT MT instructions after its previous one
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int r = 0; r < RT; ++r)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            float (&dd)[4] = EXACT ? d[EXACT ? r : 0][EXACT ? mt : 0] : acc[r][mt];
            mma16816(dd, f[r][4 * h], f[r][4 * h + 1], f[r][4 * h + 2], f[r][4 * h + 3], xb[qd & 1][mt][2 * h],
                     xb[qd & 1][mt][2 * h + 1]);
          }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);   // every read of stage s is done (the next stage's came after)
    if constexpr (EXACT) {
#pragma unroll
      for (int r = 0; r < RT; ++r)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          acc[r][mt][0] = fmaf(fa[r], d[r][mt][0], acc[r][mt][0]);
          acc[r][mt][1] = fmaf(fa[r], d[r][mt][1], acc[r][mt][1]);
          acc[r][mt][2] = fmaf(fb[r], d[r][mt][2], acc[r][mt][2]);
          acc[r][mt][3] = fmaf(fb[r], d[r][mt][3], acc[r][mt][3]);
        }
    }
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      qa[r] = qa_n[r];
      qb[r] = qb_n[r];
    }
  }
  // the outputs are written in stream order
  if (p.wait_guard) pdl_wait();
  __syncthreads();   // every stage consumed and every copy landed: the ring becomes the partial tile
  float* part = reinterpret_cast<float*>(smem);
  if (!producer) {
#pragma unroll
    for (int r = 0; r < RT; ++r)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = 16 * (RT * warp + r) + g + (i >= 2 ? 8 : 0), m = 8 * mt + 2 * t + (i & 1);
          part[m * PP + row] = acc[r][mt][i];
        }
  }
  if (S == 1) {
    __syncthreads();
    for (int e = threadIdx.x; e < M * ROWS; e += kMmaThreads) {
      const int m = e / ROWS, row = e - m * ROWS;
      if (n0 + row < N) p.y[(size_t)m * N + n0 + row] = out_half(part[m * PP + row], p.bias, n0 + row);
    }
    return;
  }
  // every CTA of the cluster sums its share of the M x ROWS outputs over all ranks' partials, in rank order
  cluster_sync_all();
  constexpr int Q = ROWS / 4;
  const int e4 = Q * M, rk = (int)cluster_rank();
  const int e_begin = (e4 * rk) / S, e_end = (e4 * (rk + 1)) / S;
  const uint32_t part0 = smem_addr(part);
  for (int e = e_begin + (int)threadIdx.x; e < e_end; e += kMmaThreads) {
    const int m = e / Q, row4 = (e - m * Q) * 4;
    const uint32_t off = part0 + (uint32_t)(m * PP + row4) * 4u;
    float4 a = ld_dsmem_f4(mapa_shared(off, 0));
    for (int q = 1; q < S; ++q) {
      const float4 v = ld_dsmem_f4(mapa_shared(off, (uint32_t)q));
      a.x += v.x;
      a.y += v.y;
      a.z += v.z;
      a.w += v.w;
    }
    __half* yo = p.y + (size_t)m * N + n0 + row4;
    const float o[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (n0 + row4 + j < N) yo[j] = out_half(o[j], p.bias, n0 + row4 + j);
  }
  cluster_sync_all();   // no CTA leaves while another still reads its partials
}

namespace {

constexpr int kMaxDev = 64;
std::atomic<int> g_dev_sms[kMaxDev];   // 0: not queried yet

int sm_count(int dev) {
  if (dev < 0 || dev >= kMaxDev) return 148;
  int v = g_dev_sms[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    g_dev_sms[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

template <int MT, int RT, bool EXACT>
cudaError_t launch_mma_t(const GemvParams& g, int S, bool pdl, cudaStream_t st) {
  constexpr int ROWS = kConsumerWarps * RT * 16;
  CUtensorMap xmap, wmap;
  // activations as a [M, K] fp16 tensor, boxes of 64 k x 8 MT rows (rows past M read as zeros); packed weights as
  // a [N, K / 2] byte tensor, boxes of one chunk's 64 bytes x the CTA's rows (rows past N read as zeros)
  if (!encode_tensor_map_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, g.x, (uint64_t)g.K, (uint64_t)g.M,
                            (uint64_t)g.K * 2, 64, MT * 8, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.w, (uint64_t)g.K / 2, (uint64_t)g.N,
                            (uint64_t)g.K / 2, 64, ROWS, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  const int KC = g.K / 128;
  int ngroups = 0;   // scale groups spanned by the largest of the S contiguous K ranges
  for (int r = 0; r < S; ++r) {
    const int c0 = (KC * r) / S, c1 = (KC * (r + 1)) / S;
    if (c1 > c0 && (c1 - 1) / g.cpg - c0 / g.cpg + 1 > ngroups) ngroups = (c1 - 1) / g.cpg - c0 / g.cpg + 1;
  }
  MmaParams p{g.s, g.y, g.bias, g.M, g.N, g.K, g.KG, g.cpg, g.flags, g.wait_guard, S, ngroups};
  auto kern = gemm_mma_kernel<MT, RT, EXACT>;
  const int smem = mma_smem_bytes(MT, RT, ngroups);
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((g.N + ROWS - 1) / ROWS, S, 1);
  cfg.blockDim = dim3(kMmaThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (S > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = S;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, xmap, wmap, p);
}

template <int RT>
cudaError_t launch_mma_rt(const GemvParams& g, int S, bool pdl, cudaStream_t st) {
  const int m = g.M;
  if (m <= 16) return launch_mma_t<2, RT, true>(g, S, pdl, st);
  if (m <= 32) return launch_mma_t<4, RT, false>(g, S, pdl, st);
  if (m <= 48) return launch_mma_t<6, RT, false>(g, S, pdl, st);
  return launch_mma_t<8, RT, false>(g, S, pdl, st);
}

// CTAs of one (MT, RT) instance resident per SM at its ring's shared memory (registers and warps included),
// queried once per device
std::atomic<int> g_resident[kMaxDev][4][2];   // value + 1 (0: not queried yet)

template <int MT, int RT>
int resident_base(int dev) {
  const int im = MT / 2 - 1, ir = RT - 1;
  if (dev < 0 || dev >= kMaxDev) return 1;
  int v = g_resident[dev][im][ir].load(std::memory_order_relaxed);
  if (v == 0) {
    auto kern = gemm_mma_kernel<MT, RT, MT == 2>;
    const int smem = mma_smem_bytes(MT, RT, 0);
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kMmaThreads, smem) != cudaSuccess || n < 1) {
      cudaGetLastError();   // the failed query's own error
      n = 1;
    }
    v = n + 1;
    g_resident[dev][im][ir].store(v, std::memory_order_relaxed);
  }
  return v - 1;
}

int resident_per_sm(int M, int rt, int dev) {
  const int mt = M <= 16 ? 2 : M <= 32 ? 4 : M <= 48 ? 6 : 8;
  switch (mt * 2 + rt - 1) {
    case 4: return resident_base<2, 1>(dev);
    case 5: return resident_base<2, 2>(dev);
    case 8: return resident_base<4, 1>(dev);
    case 9: return resident_base<4, 2>(dev);
    case 12: return resident_base<6, 1>(dev);
    case 13: return resident_base<6, 2>(dev);
    case 16: return resident_base<8, 1>(dev);
    default: return resident_base<8, 2>(dev);
  }
}

}  // namespace

// One 16-row tile per warp (measured on B200 faster than two at every config-2 shape but one); the largest split
// whose CTAs are all resident at once (tiles x S <= SMs x CTAs per SM), since a split CTA carries less of the
// weight stream and the clusters' partial sums cost little -- except for K of fewer than four chunks, where a
// split leaves each CTA too little to overlap (a sweep over splits 1..8 on the config-2 shapes picked these).
MmaConfig gemm_mma_config(int M, int N, int K, int G, int forced_splits, int forced_rt) {
  MmaConfig c{0, 0};
  if (M < 1 || M > 64 || N < 1 || K < 128 || K % 128 || G % 128 || K % G) return c;
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = sm_count(dev), KC = K / 128;
  const int rt = forced_rt == 1 || forced_rt == 2 ? forced_rt : 1;
  const int rows = kConsumerWarps * 16 * rt, tiles = (N + rows - 1) / rows;
  int S = 1;
  if (forced_splits > 0) {
    S = forced_splits < kMaxClusterSplits ? forced_splits : kMaxClusterSplits;
    if (S > KC) S = KC;
  } else if (KC >= 4) {
    const int slots = sms * resident_per_sm(M, rt, dev);
    S = slots / tiles;
    if (S > kMaxClusterSplits) S = kMaxClusterSplits;
    if (S > KC) S = KC;
    if (S < 1) S = 1;
  }
  c.splits = S;
  c.rt = rt;
  return c;
}

cudaError_t launch_gemm_mma(const GemvParams& p, const MmaConfig& c, bool pdl, cudaStream_t st) {
  if (p.M < 1 || p.M > 64 || c.splits < 1 || c.splits > kMaxClusterSplits) return cudaErrorInvalidConfiguration;
  if (c.rt == 2) return launch_mma_rt<2>(p, c.splits, pdl, st);
  if (c.rt == 1) return launch_mma_rt<1>(p, c.splits, pdl, st);
  return cudaErrorInvalidConfiguration;
}

int gemm_mma_device_error() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_mma_status, sizeof(int));
  return v;
}

void gemm_mma_clear_device_error() {
  int z = 0;
  cudaMemcpyToSymbol(g_mma_status, &z, sizeof(int));
}

}  // namespace lb
