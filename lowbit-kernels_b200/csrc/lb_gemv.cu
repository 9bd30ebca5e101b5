// W4A16 decode GEMV for sm_100a: y[M, N] = x[M, K] * dequant(W)[N, K]^T for M <= 16 rows.
//
// Role of the reference's gemv_v6 (csrc/w4_gemv.cu:327-391): reads the mma layout a model keeps
// (lowbit/quant.py:67-78). Design:
//   * a warp owns one 16-row tile of W and a strided set of its 128-wide K chunks; lane (g, t) streams
//     16-byte words t of rows g and g+8 with L1-bypassing 128-bit loads (4 lanes cover a row's 64-byte chunk);
//   * the nibbles become exact fp16 integers q = u - 8 in registers (mask-OR into the 1024.0 mantissa, one
//     f16x2 subtract or fma per pair, no integer conversion), and go straight into mma.sync m16n8k16 as the
//     A fragment -- the mma layout is exactly that fragment, so no shuffles are needed;
//   * activations are the B operand (up to 8 rows per n8 tile, MT tiles), staged once per CTA in shared
//     memory in the order each lane consumes them (one 128-bit shared load per two k16 steps);
//   * each chunk's fp32 accumulator is scaled by its group scale in fp32 and folded into the running sum,
//     so products q * x are exact and the group scale is applied without rounding the weight to fp16;
//   * warps of a CTA split K and reduce through shared memory; for narrow or long layers a thread-block
//     cluster splits K further and reduces through distributed shared memory (no global scratch);
//   * programmatic dependent launch: the kernel lets its successor launch at entry and waits for its
//     predecessor before reading activations (optionally after issuing its first weight loads).
#include <cooperative_groups.h>

#include "lb_common.cuh"
#include "lb_launch.h"

namespace cg = cooperative_groups;

namespace lb {

// shared-memory words of activations per CTA: M rows of (chunks * 64 + 16) words (the +16 words put
// consecutive activation rows 16 banks apart, so two rows read in one phase never collide)
__host__ __device__ inline int gemv_x_row_words(int nchunks) { return nchunks * 64 + 16; }

template <int MT, int NW, int U>
__global__ void __launch_bounds__(NW * 32) gemv_mma_kernel(GemvParams p) {
  extern __shared__ __align__(16) uint32_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int K = p.K, N = p.N, M = p.M;
  const int KC = K >> 7;
  const int split = blockIdx.y, nsplit = gridDim.y;
  const int c_begin = (int)((int64_t)KC * split / nsplit);
  const int c_end = (int)((int64_t)KC * (split + 1) / nsplit);
  const int nl = c_end - c_begin;
  const int row_words = gemv_x_row_words(nl);
  const int n0 = blockIdx.x * 16;
  const int ra = min(n0 + g, N - 1), rb = min(n0 + g + 8, N - 1);  // tail rows re-read row N-1, never stored
  const uint4* wa = reinterpret_cast<const uint4*>(p.w) + (size_t)ra * (K >> 5) + t;
  const uint4* wb = reinterpret_cast<const uint4*>(p.w) + (size_t)rb * (K >> 5) + t;
  const int KG = K / p.G, cpg = p.G >> 7;
  const uint16_t* sa = reinterpret_cast<const uint16_t*>(p.s) + (size_t)ra * KG;
  const uint16_t* sb = reinterpret_cast<const uint16_t*>(p.s) + (size_t)rb * KG;

  pdl_launch_dependents();

  // This warp's chunks are c_begin + warp + NW * i. Two register buffers of U chunks each alternate: the
  // loads of one are in flight while the other is consumed, and a buffer is refilled right after use, so
  // a warp never waits for one batch before requesting the next.
  const int first = c_begin + warp, stride = NW * U;
  uint4 a0[U], b0[U], a1[U], b1[U];      // buffer 0 / 1: rows g (a) and g + 8 (b)
  uint16_t sa0[U], sb0[U], sa1[U], sb1[U];
  auto load = [&](uint4 (&qa)[U], uint4 (&qb)[U], uint16_t (&ssa)[U], uint16_t (&ssb)[U], int c0) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + NW * u;
      if (c < c_end) {
        const int grp = cpg == 1 ? c : c / cpg;
        qa[u] = ldg_stream(wa + 4 * c);
        qb[u] = ldg_stream(wb + 4 * c);
        ssa[u] = ldg_u16(sa + grp);
        ssb[u] = ldg_u16(sb + grp);
      }
    }
  };

  if (p.flags & kFlagEarlyWeights) {
    // weights and scales are static model state: fetch them before the predecessor kernel finishes
    load(a0, b0, sa0, sb0, first);
    load(a1, b1, sa1, sb1, first + stride);
    pdl_wait();
  } else {
    pdl_wait();
    load(a0, b0, sa0, sb0, first);
    load(a1, b1, sa1, sb1, first + stride);
  }

  // stage x[:, chunks c_begin..c_end) in consumption order: word ((m * row_words) + lc * 64 + qd * 16 + t * 4 + e)
  // holds the pair x[m][128 c + 8 s + 2 t .. +1] with s = 4 qd + e
  {
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(p.x);
    const int pairs = nl * 64;
    for (int idx = threadIdx.x; idx < M * pairs; idx += NW * 32) {
      int m = idx / pairs, pi = idx - m * pairs;
      int lc = pi >> 6, o = pi & 63, s = o >> 2, tt = o & 3;
      smem[m * row_words + lc * 64 + (s >> 2) * 16 + tt * 4 + (s & 3)] =
          __ldg(xw + (size_t)m * (K >> 1) + (size_t)(c_begin + lc) * 64 + o);
    }
  }
  __syncthreads();

  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mt][i] = 0.f;

  int xoff[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) xoff[mt] = min(8 * mt + g, M - 1) * row_words + t * 4;

  auto compute = [&](const uint4 (&qa)[U], const uint4 (&qb)[U], const uint16_t (&ssa)[U],
                     const uint16_t (&ssb)[U], int c0) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + NW * u;
      if (c < c_end) {
        const int lc = c - c_begin;
        float d[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) d[mt][i] = 0.f;
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          uint32_t w0 = (&qa[u].x)[qd], w1 = (&qb[u].x)[qd];
          uint4 xb[MT];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            xb[mt] = *reinterpret_cast<const uint4*>(smem + xoff[mt] + lc * 64 + qd * 16);
          // k16 step 2qd: pairs 0 (k = .. + 2t) and 1 (k = .. + 8 + 2t)
          uint32_t f0 = q_pair_lo(w0), f1 = q_pair_lo(w1), f2 = q_pair_hi(w0), f3 = q_pair_hi(w1);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) mma16816(d[mt], f0, f1, f2, f3, xb[mt].x, xb[mt].y);
          // k16 step 2qd + 1: pairs 2 and 3, the same extraction on the word shifted by 8
          w0 >>= 8;
          w1 >>= 8;
          f0 = q_pair_lo(w0); f1 = q_pair_lo(w1); f2 = q_pair_hi(w0); f3 = q_pair_hi(w1);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) mma16816(d[mt], f0, f1, f2, f3, xb[mt].z, xb[mt].w);
        }
        const float s0 = h2f_bits(ssa[u]), s1 = h2f_bits(ssb[u]);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          acc[mt][0] = fmaf(s0, d[mt][0], acc[mt][0]);
          acc[mt][1] = fmaf(s0, d[mt][1], acc[mt][1]);
          acc[mt][2] = fmaf(s1, d[mt][2], acc[mt][2]);
          acc[mt][3] = fmaf(s1, d[mt][3], acc[mt][3]);
        }
      }
    }
  };

  for (int c0 = first; c0 < c_end; c0 += 2 * stride) {
    compute(a0, b0, sa0, sb0, c0);
    load(a0, b0, sa0, sb0, c0 + 2 * stride);
    compute(a1, b1, sa1, sb1, c0 + stride);
    load(a1, b1, sa1, sb1, c0 + 3 * stride);
  }

  // reduce the NW warps' partial tiles: red[warp][mt][i][lane]
  __syncthreads();  // the activation buffer is reused for the reduction
  float* red = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[((warp * MT + mt) * 4 + i) * 32 + lane] = acc[mt][i];
  __syncthreads();

  // element e of the tile is (mt = e / 128, i = e / 32 % 4, lane = e % 32); a CTA has fewer threads than
  // a multi-tile (MT > 1) tile has elements, so threads stride over them
  constexpr int kTile = MT * 128;
  auto store = [&](int e, float v) {
    const int mt = e >> 7, i = (e >> 5) & 3, ln = e & 31;
    const int row = n0 + (ln >> 2) + (i >= 2 ? 8 : 0);
    const int m = 8 * mt + 2 * (ln & 3) + (i & 1);
    if (row < N && m < M) p.y[(size_t)m * N + row] = __float2half_rn(v);
  };
  auto cta_sum = [&](int e) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) v += red[w * kTile + e];
    return v;
  };

  if (nsplit > 1) {
    // cluster split-K: every CTA writes its partial tile into its slot of rank 0's buffer; rank 0 sums the
    // slots in rank order. The first cluster barrier makes sure rank 0 is past its main loop (the buffer
    // overlaps its activation stage), the second that every slot has landed.
    cg::cluster_group cluster = cg::this_cluster();
    float* part = red + NW * kTile;  // [nsplit][kTile] in rank 0's shared memory
    float* dst = cluster.map_shared_rank(part, 0);
    cluster.sync();
    for (int e = threadIdx.x; e < kTile; e += NW * 32) dst[split * kTile + e] = cta_sum(e);
    cluster.sync();
    if (split != 0) return;
    for (int e = threadIdx.x; e < kTile; e += NW * 32) {
      float v = 0.f;
      for (int r = 0; r < nsplit; ++r) v += part[r * kTile + e];
      store(e, v);
    }
  } else {
    for (int e = threadIdx.x; e < kTile; e += NW * 32) store(e, cta_sum(e));
  }
}

// Compatibility GEMV for the canonical and v3 layouts (the reference's v1-v4 roles, csrc/w4_gemv.cu:38-207),
// any group size that is a multiple of 32, M <= 8: a warp owns R rows; lanes stride over 32-weight words;
// exact integer values times activations accumulate in fp32, scaled once per 32-weight piece.
template <int M, int R, bool V3>
__global__ void __launch_bounds__(128) gemv_compat_kernel(GemvParams p) {
  const int lane = threadIdx.x & 31;
  const int n0 = (blockIdx.x * 4 + (threadIdx.x >> 5)) * R;
  const int K = p.K, N = p.N, KG = K / p.G;
  pdl_launch_dependents();
  pdl_wait();
  if (n0 >= N) return;
  float acc[R][M];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
  const uint4* w = reinterpret_cast<const uint4*>(p.w);
  const uint16_t* s = reinterpret_cast<const uint16_t*>(p.s);
  const uint4* x4 = reinterpret_cast<const uint4*>(p.x);
  for (int c = lane; c < (K >> 5); c += 32) {  // piece c: k = 32c .. 32c + 31 (one scale: 32 | G)
    uint4 q[R];
    float sc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      int n = min(n0 + r, N - 1);
      q[r] = ldg_stream(w + (size_t)n * (K >> 5) + c);
      sc[r] = h2f_bits(ldg_u16(s + (size_t)n * KG + (32 * c) / p.G));
    }
    float part[R][M];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) part[r][m] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {       // word i: k = 32c + 8i .. + 7
      float wv[R][8];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        uint32_t word = (&q[r].x)[i];
#pragma unroll
        for (int j = 0; j < 4; ++j) {   // pair (8i + 2j, 8i + 2j + 1)
          uint32_t bits;
          if (V3) {
            bits = q_pair(word, j);
          } else {                      // canonical: byte j holds the pair, low nibble first
            uint32_t b = (word >> (8 * j)) & 0xFFu;
            bits = hsub2_bits((b & 0xFu) | ((b & 0xF0u) << 12) | kMagic, kBias1032);
          }
          float2 f = __half22float2(*reinterpret_cast<__half2*>(&bits));
          wv[r][2 * j] = f.x;
          wv[r][2 * j + 1] = f.y;
        }
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        uint4 xv = __ldg(x4 + (size_t)m * (K >> 3) + 4 * c + i);
        const __half2* xh = reinterpret_cast<const __half2*>(&xv);
        float xf[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = __half22float2(xh[j]);
          xf[2 * j] = f.x;
          xf[2 * j + 1] = f.y;
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int e = 0; e < 8; ++e) part[r][m] = fmaf(wv[r][e], xf[e], part[r][m]);
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] = fmaf(part[r][m], sc[r], acc[r][m]);
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float v = warp_sum(acc[r][m]);
      if (lane == 0 && n0 + r < N) p.y[(size_t)m * N + n0 + r] = __float2half_rn(v);
    }
}

// ------------------------------------------------------------------------------------------------ launchers

template <int MT, int NW, int U>
static cudaError_t launch_mma(const GemvParams& p, int nsplit, cudaStream_t st, bool pdl) {
  const int KC = p.K >> 7;
  const int max_nl = (KC + nsplit - 1) / nsplit;
  const int tile_elems = MT * 128;
  size_t x_bytes = (size_t)p.M * gemv_x_row_words(max_nl) * 4;
  size_t red_bytes = (size_t)(NW + nsplit) * tile_elems * 4;
  size_t smem = x_bytes > red_bytes ? x_bytes : red_bytes;
  auto kern = gemv_mma_kernel<MT, NW, U>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N + 15) / 16, nsplit, 1);
  cfg.blockDim = dim3(NW * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (nsplit > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = nsplit;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

size_t gemv_mma_smem_bytes(int M, int K, int nsplit, int mt, int nw) {
  const int KC = K >> 7, max_nl = (KC + nsplit - 1) / nsplit;
  size_t x_bytes = (size_t)M * gemv_x_row_words(max_nl) * 4;
  size_t red_bytes = (size_t)(nw + nsplit) * mt * 128 * 4;
  return x_bytes > red_bytes ? x_bytes : red_bytes;
}

cudaError_t launch_gemv_mma(const GemvParams& p, const GemvConfig& c, cudaStream_t st) {
  const bool pdl = c.pdl != 0;
#define LB_MMA(MT_, NW_)                                                 \
  if (c.mt == MT_ && c.warps == NW_) return launch_mma<MT_, NW_, 2>(p, c.ksplit, st, pdl);
  LB_MMA(1, 4) LB_MMA(1, 8) LB_MMA(2, 4) LB_MMA(2, 8) LB_MMA(4, 4) LB_MMA(8, 4)
#undef LB_MMA
  return cudaErrorInvalidConfiguration;
}

template <int M, int R, bool V3>
static cudaError_t launch_compat_t(const GemvParams& p, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N + 4 * R - 1) / (4 * R), 1, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_compat_kernel<M, R, V3>, p);
}

template <int M>
static cudaError_t launch_compat_m(const GemvParams& p, int R, bool v3, cudaStream_t st, bool pdl) {
  if (v3) {
    if (R == 4) return launch_compat_t<M, 4, true>(p, st, pdl);
    if (R == 2) return launch_compat_t<M, 2, true>(p, st, pdl);
    return launch_compat_t<M, 1, true>(p, st, pdl);
  }
  if (R == 4) return launch_compat_t<M, 4, false>(p, st, pdl);
  if (R == 2) return launch_compat_t<M, 2, false>(p, st, pdl);
  return launch_compat_t<M, 1, false>(p, st, pdl);
}

cudaError_t launch_gemv_compat(const GemvParams& p, int rows_per_warp, bool v3, bool pdl, cudaStream_t st) {
  switch (p.M) {
    case 1: return launch_compat_m<1>(p, rows_per_warp, v3, st, pdl);
    case 2: return launch_compat_m<2>(p, rows_per_warp, v3, st, pdl);
    case 3: return launch_compat_m<3>(p, rows_per_warp, v3, st, pdl);
    case 4: return launch_compat_m<4>(p, rows_per_warp, v3, st, pdl);
    case 5: return launch_compat_m<5>(p, rows_per_warp, v3, st, pdl);
    case 6: return launch_compat_m<6>(p, rows_per_warp, v3, st, pdl);
    case 7: return launch_compat_m<7>(p, rows_per_warp, v3, st, pdl);
    default: return launch_compat_m<8>(p, rows_per_warp, v3, st, pdl);
  }
}

}  // namespace lb
