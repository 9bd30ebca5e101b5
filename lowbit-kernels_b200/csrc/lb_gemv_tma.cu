// W4A16 decode GEMV, bulk-copy pipeline: y[M, N] = x[M, K] * dequant(W)[N, K]^T for M <= 16.
//
// The decode-step problem on B200 is small per SM (an 11.7 MB projection is ~80 KB per SM, about one
// latency x bandwidth product), so the kernel is built to put every byte an SM needs in flight at once and
// to serialize nothing while it lands:
//   * one CTA per SM owns a contiguous range of 16-row tiles (balanced to +-1 tile);
//   * a producer warp streams the range through a ring of R shared-memory stages with cp.async.bulk: a stage
//     is 16 rows x up to 8 chunks (128 k each), one bulk copy per row, completing on the stage's mbarrier
//     (transaction count) -- one thread-instruction per 0.5 KB;
//   * 8 consumer warps split each stage's chunks: lane (g, t) reads the 16-byte words t of rows g and g+8
//     (the mma layout is exactly the m16n8k16 A fragment), turns nibbles into exact fp16 integers q = u - 8
//     in registers and runs mma.sync with the staged activations as the B operand; each chunk's fp32 result
//     is scaled by its group scale in fp32 (scales prefetched into registers two stages ahead);
//   * a tile is reduced without a CTA barrier: each warp parks its partial sums in a slot and bumps a
//     shared counter; the last warp to arrive adds the slots in warp order (deterministic) and stores;
//   * every mbarrier wait is bounded and records an error code instead of hanging.
// The weights are static model state, so the producer may start before the previous kernel in the stream
// finishes (programmatic dependent launch); consumers wait for it before reading x or writing y.
#include "lb_common.cuh"
#include "lb_launch.h"

namespace lb {

__device__ int g_tma_error;   // set by a wait that gave up (bounded spin); read by tma_device_error()

namespace {

constexpr int kNC = 8;          // consumer warps
constexpr int kStages = 8;      // ring depth
constexpr int kCPS = 8;         // chunks (128 k) per stage
constexpr int kRowBytes = kCPS * 64 + 64;  // staged row stride: 512 B of data + 64 B so rows g, g+1 use other banks
constexpr int kStageBytes = 16 * kRowBytes;
constexpr int kSlots = kStages + 2;        // tile reduction slots: warps are at most kStages stages apart

__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicExch(&g_tma_error, kErrBarrierTimeout);
  return false;
}

struct TmaLayout {
  int x, ring, red, bars, cnt, total;
};

__host__ __device__ inline TmaLayout tma_layout(int M, int KC, int mt) {
  TmaLayout L;
  L.x = 0;
  L.ring = ((M * (KC * 64 + 16) * 4) + 127) & ~127;
  L.red = L.ring + kStages * kStageBytes;
  L.bars = L.red + kSlots * kNC * mt * 512;
  L.cnt = L.bars + 2 * kStages * 8;
  L.total = L.cnt + kSlots * 4;
  return L;
}

}  // namespace

template <int MT>
__global__ void __launch_bounds__((kNC + 1) * 32, 1) gemv_tma_kernel(GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = p.K, N = p.N, M = p.M;
  const int KC = K >> 7, KG = K / p.G, cpg = p.G >> 7;
  const TmaLayout L = tma_layout(M, KC, MT);
  uint32_t* xs = reinterpret_cast<uint32_t*>(smem + L.x);
  float* red = reinterpret_cast<float*>(smem + L.red);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + kStages;
  int* cnt = reinterpret_cast<int*>(smem + L.cnt);
  const int row_words = KC * 64 + 16;

  // this CTA's tiles [t0, t1); each tile is `pieces` stages of up to kCPS chunks
  const int NT = (N + 15) >> 4;
  const int t0 = (int)((int64_t)NT * blockIdx.x / gridDim.x);
  const int t1 = (int)((int64_t)NT * (blockIdx.x + 1) / gridDim.x);
  const int pieces = (KC + kCPS - 1) / kCPS;
  const int Q = (t1 - t0) * pieces;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kNC);
    }
    mbar_fence_init();
  }
  for (int i = threadIdx.x; i < kSlots; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kNC) {
    // ------------------------------------------------------------------ producer
    if (!(p.flags & kFlagEarlyWeights)) pdl_wait();
    const uint8_t* wbytes = reinterpret_cast<const uint8_t*>(p.w);
    int tile = t0, piece = 0;
    for (int q = 0; q < Q; ++q) {
      const int slot = q % kStages;
      if (q >= kStages && !wait_bounded(&empty[slot], ((q / kStages) - 1) & 1)) break;
      const int c0 = piece * kCPS;
      const int nch = min(kCPS, KC - c0);
      const uint32_t row_bytes = (uint32_t)nch * 64;
      if (lane == 0) mbar_arrive_expect_tx(&full[slot], 16 * row_bytes);
      __syncwarp();
      if (lane < 16) {
        const int row = min(tile * 16 + lane, N - 1);   // tail rows re-read row N-1, never stored
        bulk_copy_g2s(smem + L.ring + slot * kStageBytes + lane * kRowBytes,
                      wbytes + (size_t)row * (K >> 1) + (size_t)c0 * 64, row_bytes, &full[slot]);
      }
      if (++piece == pieces) { piece = 0; ++tile; }
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int g = lane >> 2, t = lane & 3;
  pdl_wait();
  {
    // activations in consumption order: word (m * row_words + c * 64 + qd * 16 + t * 4 + e) holds the pair
    // x[m][128 c + 8 s + 2 t .. +1] with s = 4 qd + e
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(p.x);
    const int pairs = KC * 64;
    for (int m = 0; m < M; ++m)
      for (int pi = threadIdx.x; pi < pairs; pi += kNC * 32) {
        const int c = pi >> 6, o = pi & 63, s = o >> 2, tt = o & 3;
        xs[m * row_words + c * 64 + (s >> 2) * 16 + tt * 4 + (s & 3)] = __ldg(xw + (size_t)m * (K >> 1) + pi);
      }
  }
  named_barrier(1, kNC * 32);

  int xoff[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) xoff[mt] = min(8 * mt + g, M - 1) * row_words + t * 4;
  const uint16_t* s16 = reinterpret_cast<const uint16_t*>(p.s);

  // scales of (stage q, this warp's chunk) for rows g and g + 8, loaded two stages ahead
  uint16_t sc_a[3], sc_b[3];
  auto load_scales = [&](int q, uint16_t& a, uint16_t& b) {
    if (q < Q) {
      const int tile = t0 + q / pieces, c = (q % pieces) * kCPS + warp;
      if (c < KC) {
        const int grp = cpg == 1 ? c : c / cpg;
        a = ldg_u16(s16 + (size_t)min(tile * 16 + g, N - 1) * KG + grp);
        b = ldg_u16(s16 + (size_t)min(tile * 16 + g + 8, N - 1) * KG + grp);
      }
    }
  };
  load_scales(0, sc_a[0], sc_b[0]);
  load_scales(1, sc_a[1], sc_b[1]);

  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mt][i] = 0.f;
  constexpr int kTile = MT * 128;
  bool ok = true;

  for (int q0 = 0; q0 < Q; q0 += 3) {
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      const int q = q0 + u;
      if (q >= Q) break;
      load_scales(q + 2, sc_a[(u + 2) % 3], sc_b[(u + 2) % 3]);
      const int slot = q % kStages;
      const int piece = q % pieces, tile = t0 + q / pieces;
      const int c = piece * kCPS + warp;
      if (ok) ok = wait_bounded(&full[slot], (q / kStages) & 1);
      if (ok && c < KC) {
        const uint8_t* st = smem + L.ring + slot * kStageBytes + warp * 64 + t * 16;
        const uint4 qa = *reinterpret_cast<const uint4*>(st + g * kRowBytes);
        const uint4 qb = *reinterpret_cast<const uint4*>(st + (g + 8) * kRowBytes);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);   // the stage's bytes for this warp are in registers
        float d[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) d[mt][i] = 0.f;
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          uint32_t w0 = (&qa.x)[qd], w1 = (&qb.x)[qd];
          uint4 xb[MT];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            xb[mt] = *reinterpret_cast<const uint4*>(xs + xoff[mt] + c * 64 + qd * 16);
          uint32_t f0 = q_pair_lo(w0), f1 = q_pair_lo(w1), f2 = q_pair_hi(w0), f3 = q_pair_hi(w1);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) mma16816(d[mt], f0, f1, f2, f3, xb[mt].x, xb[mt].y);
          w0 >>= 8;
          w1 >>= 8;
          f0 = q_pair_lo(w0); f1 = q_pair_lo(w1); f2 = q_pair_hi(w0); f3 = q_pair_hi(w1);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) mma16816(d[mt], f0, f1, f2, f3, xb[mt].z, xb[mt].w);
        }
        const float s0 = h2f_bits(sc_a[u]), s1 = h2f_bits(sc_b[u]);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          acc[mt][0] = fmaf(s0, d[mt][0], acc[mt][0]);
          acc[mt][1] = fmaf(s0, d[mt][1], acc[mt][1]);
          acc[mt][2] = fmaf(s1, d[mt][2], acc[mt][2]);
          acc[mt][3] = fmaf(s1, d[mt][3], acc[mt][3]);
        }
      } else {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }

      if (piece == pieces - 1) {
        // tile done: park this warp's partial tile, and let the last warp to arrive reduce and store
        const int ts = (tile - t0) % kSlots;
        float* rs = red + (ts * kNC + warp) * kTile;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            rs[mt * 128 + i * 32 + lane] = acc[mt][i];
            acc[mt][i] = 0.f;
          }
        __threadfence_block();
        __syncwarp();
        int prev = 0;
        if (lane == 0) prev = atomicAdd(&cnt[ts], 1);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == kNC - 1) {
          __threadfence_block();
          const float* rt = red + ts * kNC * kTile;
          const int n0 = tile * 16;
#pragma unroll
          for (int e = lane; e < kTile; e += 32) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kNC; ++w) v += rt[w * kTile + e];
            const int mt = e >> 7, i = (e >> 5) & 3, ln = e & 31;
            const int row = n0 + (ln >> 2) + (i >= 2 ? 8 : 0);
            const int m = 8 * mt + 2 * (ln & 3) + (i & 1);
            if (row < N && m < M) p.y[(size_t)m * N + row] = __float2half_rn(v);
          }
          __syncwarp();
          if (lane == 0) cnt[ts] = 0;
        }
      }
    }
  }
}

template <int MT>
static cudaError_t launch_tma_t(const GemvParams& p, int ctas, bool pdl, cudaStream_t st) {
  const TmaLayout L = tma_layout(p.M, p.K >> 7, MT);
  auto kern = gemv_tma_kernel<MT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3((kNC + 1) * 32, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

size_t gemv_tma_smem_bytes(int M, int K) {
  return (size_t)tma_layout(M, K >> 7, M <= 8 ? 1 : 2).total;
}

cudaError_t launch_gemv_tma(const GemvParams& p, int ctas, bool pdl, cudaStream_t st) {
  return p.M <= 8 ? launch_tma_t<1>(p, ctas, pdl, st) : launch_tma_t<2>(p, ctas, pdl, st);
}

int tma_device_error() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_tma_error, sizeof(int));
  return v;
}

void tma_clear_device_error() {
  int z = 0;
  cudaMemcpyToSymbol(g_tma_error, &z, sizeof(int));
}

}  // namespace lb
