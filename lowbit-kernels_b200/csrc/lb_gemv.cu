// W4A16 decode GEMV for sm_100a: y[M, N] = x[M, K] * dequant(W)[N, K]^T for small M.
//
// Role of the reference's gemv_v6 (csrc/w4_gemv.cu:327-391): reads the mma layout a model keeps
// (lowbit/quant.py:67-78). Design:
//   * persistent CTAs (grid sized to the SM count): a CTA stages its slice of the activations once, then
//     streams 16-row tiles of W; the warps of the CTA split each tile's 128-wide K chunks;
//   * each warp keeps a D-deep ring of cp.async (LDGSTS) copies in shared memory: lane (g, t) copies the
//     16-byte words t of rows g and g+8 of a chunk -- exactly the tensor-core fragment it will consume -- so
//     bytes in flight do not depend on registers, the ring runs on across tile boundaries, and no
//     cross-lane synchronization is needed (each lane reads back only what it copied);
//   * the nibbles become exact fp16 integers q = u - 8 in registers (mask-OR into the 1024.0 mantissa, one
//     f16x2 subtract or fma per pair, no integer conversion) and feed mma.sync m16n8k16 as the A fragment;
//     activations are the B operand (n8 tiles of up to 8 rows), staged in consumption order;
//   * each chunk's fp32 accumulator is scaled by its group scale in fp32 and folded into the running sum,
//     so products q * x are exact and the weight is never rounded to fp16;
//   * per tile, warps publish partial sums to shared memory (double-buffered) and one warp reduces and
//     stores; for narrow, long-K layers a thread-block cluster splits K and the reducing warp adds the
//     ranks' partials through distributed shared memory (no global scratch, no spin-waits);
//   * programmatic dependent launch: the kernel lets its successor launch at entry and waits for its
//     predecessor before touching activations or outputs (optionally after starting its weight copies).
#include <cooperative_groups.h>

#include "lb_common.cuh"
#include "lb_launch.h"

namespace cg = cooperative_groups;

namespace lb {

// shared-memory words of activations per row: (chunks * 64 + 16) -- the +16 words put consecutive activation
// rows 16 banks apart, so two rows read in one phase never collide
__host__ __device__ inline int gemv_x_row_words(int nchunks) { return nchunks * 64 + 16; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// One-shot GEMV (M <= 16), the decode path. One CTA owns RT 16-row tiles and a K range (a cluster of S
// CTAs splits long K); its warps split the range's chunks, at most CPW each. At entry every thread issues
// ALL of its weight and scale loads (register destinations, L1 bypassed) -- ahead of the wait on the previous
// kernel when the weights are known static -- so the whole share is in flight at once while the previous
// kernel finishes. The kernel is built to issue as few instructions as possible after that wait, because in
// a chain of decode kernels that post-wait work is what sets the pace:
//   * activations are staged with one 16-byte L2 load and four shared stores per eight values;
//   * each warp runs two row tiles against the same activation fragments;
//   * nibbles become exact fp16 integers q = u - 8 in registers (mask-OR into the 1024.0 mantissa, one f16x2
//     subtract or fma per pair) and feed mma.sync m16n8k16 as the A fragment: products q * x are exact, sums
//     fp32, and each chunk's result is scaled by its group scale in fp32 (the weight is never rounded);
//   * warps reduce through shared memory, cluster ranks through distributed shared memory, rank 0 stores.
// Status word: a kernel whose bounded wait gives up records an error code here instead of hanging the GPU;
// the host reads it with lb_device_error().
__device__ int g_device_status;

int device_error() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
  return v;
}

void clear_device_error() {
  int z = 0;
  cudaMemcpyToSymbol(g_device_status, &z, sizeof(int));
}

// fp32 sum over the CTA (every thread calls it; red: 32 floats of shared memory)
__device__ __forceinline__ float cta_sum_f32(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ void st_volatile_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_volatile_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// fetch-and-add with acquire-release semantics at GPU scope: publishes what this thread (and, after a bar.sync,
// its CTA) wrote before it and makes visible what the earlier adders published
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(int* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ uint4 ldg_cg_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

template <int MT, int RT, int CPW, bool EARLY, int PRO = 0, int EPI = 0>
__global__ void __launch_bounds__(512) gemv_oneshot_kernel(GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint32_t* const sw = reinterpret_cast<uint32_t*>(smem);
  const int NW = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int K = p.K, N = p.N, M = p.M;
  const int KC = K >> 7, KG = p.KG, cpg = p.cpg;
  const int split = blockIdx.y, nsplit = gridDim.y;
  // K range of this cluster rank; the divisions only run when K is split
  const int c_begin = nsplit == 1 ? 0 : KC * split / nsplit;
  const int c_end = nsplit == 1 ? KC : KC * (split + 1) / nsplit;
  const int nl = c_end - c_begin;
  const int row_words = gemv_x_row_words(nl);
  const int n0 = blockIdx.x * (16 * RT);
  const int c_warp = c_begin + warp;
  const size_t row_u4 = (size_t)(K >> 5);

  uint4 qa[RT][CPW], qb[RT][CPW];
  uint16_t ssa[RT][CPW], ssb[RT][CPW];
  pdl_launch_dependents();
  if (!EARLY) pdl_wait();
#pragma unroll
  for (int r = 0; r < RT; ++r) {
    const int ra = min(n0 + 16 * r + g, N - 1), rb = min(n0 + 16 * r + g + 8, N - 1);   // tail rows: row N-1
    const uint4* wa = reinterpret_cast<const uint4*>(p.w) + (size_t)ra * row_u4 + t;
    const uint4* wb = reinterpret_cast<const uint4*>(p.w) + (size_t)rb * row_u4 + t;
    const uint16_t* sa = reinterpret_cast<const uint16_t*>(p.s) + (size_t)ra * KG;
    const uint16_t* sb = reinterpret_cast<const uint16_t*>(p.s) + (size_t)rb * KG;
#pragma unroll
    for (int i = 0; i < CPW; ++i) {
      const int c = c_warp + NW * i;
      if (c < c_end) {
        const int grp = cpg == 1 ? c : c / cpg;
        qa[r][i] = ldg_stream(wa + 4 * c);
        qb[r][i] = ldg_stream(wb + 4 * c);
        ssa[r][i] = ldg_u16(sa + grp);
        ssb[r][i] = ldg_u16(sb + grp);
      }
    }
  }
  if (EARLY) pdl_wait_after_loads(p.wait_guard);

  // Activations of this K range, copied verbatim (cp.async, L2 only) into shared memory rows of
  // xrow_bytes = nl * 256 + 16 bytes (the 16-byte skew puts the 8 rows an ldmatrix reads on distinct banks).
  // Within a k16 step the mma layout already follows natural k order, so ldmatrix on these rows yields the B
  // fragments directly.
  const int xrow_bytes = nl * 256 + 16;
  {
    const uint8_t* xg = reinterpret_cast<const uint8_t*>(p.x) + (size_t)c_begin * 256;
    const int pieces = nl * 16;   // 16-byte pieces per row
    for (int m = 0; m < M; ++m)
      for (int it = threadIdx.x; it < pieces; it += blockDim.x)
        cp_async16(smem_u32(smem + m * xrow_bytes + it * 16), xg + (size_t)m * (K * 2) + it * 16);
    cp_async_commit();
  }

  // the first chunk's fragments are decoded while the activations are in flight
  uint32_t fr0[RT][4][8];
  {
    const int c = c_warp;
    if (c < c_end) {
#pragma unroll
      for (int r = 0; r < RT; ++r)
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          const uint32_t w0 = (&qa[r][0].x)[qd], w1 = (&qb[r][0].x)[qd];
          fr0[r][qd][0] = q_pair_lo(w0); fr0[r][qd][1] = q_pair_lo(w1);
          fr0[r][qd][2] = q_pair_hi(w0); fr0[r][qd][3] = q_pair_hi(w1);
          fr0[r][qd][4] = q_pair_lo(w0 >> 8); fr0[r][qd][5] = q_pair_lo(w1 >> 8);
          fr0[r][qd][6] = q_pair_hi(w0 >> 8); fr0[r][qd][7] = q_pair_hi(w1 >> 8);
        }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  if constexpr (PRO != 0) {
    // activation prologue (M = 1, the CTA holds the whole row): the decode step's RMSNorm (with the residual add)
    // or SwiGLU, applied to the staged row in place -- the same fp16 roundings as the standalone kernels
    __shared__ float pro_red[32];
    uint4* xs = reinterpret_cast<uint4*>(smem);
    const int n8 = K / 8;
    if constexpr (PRO == 1) {
      float ss = 0.f;
      for (int v = threadIdx.x; v < n8; v += blockDim.x) {
        uint4 xv = xs[v];
        __half2* xh = reinterpret_cast<__half2*>(&xv);
        if (p.pro_r) {
          const uint4 rv = ldg_cg_u4(p.pro_r + 8 * (size_t)v);
          const __half2* rh = reinterpret_cast<const __half2*>(&rv);
#pragma unroll
          for (int j = 0; j < 4; ++j) xh[j] = __hadd2(xh[j], rh[j]);
          xs[v] = xv;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(xh[j]);
          ss += f.x * f.x + f.y * f.y;
        }
      }
      const float inv = rsqrtf(cta_sum_f32(ss, pro_red) / (float)K + p.pro_eps);
      for (int v = threadIdx.x; v < n8; v += blockDim.x) {
        const uint4 xv = xs[v];
        const uint4 wv = ldg_stream(reinterpret_cast<const uint4*>(p.pro_w) + v);
        if (blockIdx.x == 0 && p.pro_out) reinterpret_cast<uint4*>(p.pro_out)[v] = xv;
        const __half2* xh = reinterpret_cast<const __half2*>(&xv);
        const __half2* wh = reinterpret_cast<const __half2*>(&wv);
        uint4 o;
        __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(xh[j]);
          oh[j] = __hmul2(wh[j], __floats2half2_rn(f.x * inv, f.y * inv));
        }
        xs[v] = o;
      }
    } else {
      const __half* up = reinterpret_cast<const __half*>(p.x) + K;
      for (int v = threadIdx.x; v < n8; v += blockDim.x) {
        const uint4 gv = xs[v];
        const uint4 uv = ldg_cg_u4(up + 8 * (size_t)v);
        const __half* gh = reinterpret_cast<const __half*>(&gv);
        const __half* uh = reinterpret_cast<const __half*>(&uv);
        uint4 o;
        __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float gf = __half2float(gh[j]);
          const __half sg = __float2half_rn(gf / (1.f + expf(-gf)));
          oh[j] = __float2half_rn(__half2float(sg) * __half2float(uh[j]));
        }
        xs[v] = o;
      }
    }
    __syncthreads();
  }

  float acc[RT][MT][4];
#pragma unroll
  for (int r = 0; r < RT; ++r)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[r][mt][i] = 0.f;
  // ldmatrix row addresses: lane L serves row (L & 7) of 8x8 matrix L >> 3 (k offset 8 * (L >> 3) in a 32-k
  // block); activation rows past M repeat row M - 1 (their outputs are dropped)
  uint32_t xaddr[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
    xaddr[mt] = smem_u32(smem + min(8 * mt + (lane & 7), M - 1) * xrow_bytes + (lane >> 3) * 16);

#pragma unroll
  for (int i = 0; i < CPW; ++i) {
    const int c = c_warp + NW * i;
    if (c < c_end) {
      const int lc = c - c_begin;
      float d[RT][MT][4];
#pragma unroll
      for (int r = 0; r < RT; ++r)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int j = 0; j < 4; ++j) d[r][mt][j] = 0.f;
#pragma unroll
      for (int qd = 0; qd < 4; ++qd) {
        uint32_t xb[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) ldsm_x4(xb[mt], xaddr[mt] + lc * 256 + qd * 64);
#pragma unroll
        for (int r = 0; r < RT; ++r) {
          uint32_t f[8];
          if (i == 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] = fr0[r][qd][j];
          } else {
            const uint32_t w0 = (&qa[r][i].x)[qd], w1 = (&qb[r][i].x)[qd];
            f[0] = q_pair_lo(w0); f[1] = q_pair_lo(w1); f[2] = q_pair_hi(w0); f[3] = q_pair_hi(w1);
            f[4] = q_pair_lo(w0 >> 8); f[5] = q_pair_lo(w1 >> 8); f[6] = q_pair_hi(w0 >> 8); f[7] = q_pair_hi(w1 >> 8);
          }
          // k16 step 2qd: pairs 0 (k = .. + 2t) and 1 (k = .. + 8 + 2t); step 2qd + 1: pairs 2 and 3
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            mma16816(d[r][mt], f[0], f[1], f[2], f[3], xb[mt][0], xb[mt][1]);
            mma16816(d[r][mt], f[4], f[5], f[6], f[7], xb[mt][2], xb[mt][3]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        const float s0 = h2f_bits(ssa[r][i]), s1 = h2f_bits(ssb[r][i]);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          acc[r][mt][0] = fmaf(s0, d[r][mt][0], acc[r][mt][0]);
          acc[r][mt][1] = fmaf(s0, d[r][mt][1], acc[r][mt][1]);
          acc[r][mt][2] = fmaf(s1, d[r][mt][2], acc[r][mt][2]);
          acc[r][mt][3] = fmaf(s1, d[r][mt][3], acc[r][mt][3]);
        }
      }
    }
  }

  // reduce the warps' partial tiles through shared memory: red[warp][r][mt][i][lane]
  constexpr int kTile = RT * MT * 128;
  __syncthreads();
  float* red = reinterpret_cast<float*>(sw);
#pragma unroll
  for (int r = 0; r < RT; ++r)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[warp * kTile + (r * MT + mt) * 128 + i * 32 + lane] = acc[r][mt][i];
  __syncthreads();
  auto store = [&](int e, float v) {
    const int rm = e >> 7, i = (e >> 5) & 3, ln = e & 31;
    const int r = rm / MT, mt = rm - r * MT;
    const int row = n0 + 16 * r + (ln >> 2) + (i >= 2 ? 8 : 0);
    const int m = 8 * mt + 2 * (ln & 3) + (i & 1);
    if (row < N && m < M) p.y[(size_t)m * N + row] = out_half(v, p.bias, row);
  };
  auto cta_sum = [&](int e) {
    float v = 0.f;
#pragma unroll 8
    for (int w = 0; w < NW; ++w) v += red[w * kTile + e];   // the loads issue together; the adds keep their order
    return v;
  };
  // the finished tile: one CTA's warps summed (nsplit == 1), or, with K split over a cluster, each rank's sum
  // written into its slot of rank 0's buffer (after a cluster barrier: the buffer follows rank 0's reduction area),
  // a second barrier publishing the slots, and rank 0 adding them in rank order
  float* part = red + NW * kTile;
  if (nsplit > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    float* dst = cluster.map_shared_rank(part, 0) + split * kTile;
    cluster.sync();
    for (int e = threadIdx.x; e < kTile; e += blockDim.x) dst[e] = cta_sum(e);
    cluster.sync();
    if (split != 0) return;
  }
  auto tile_sum = [&](int e) {
    if (nsplit == 1) return cta_sum(e);
    float v = 0.f;
    for (int r = 0; r < nsplit; ++r) v += part[r * kTile + e];
    return v;
  };
  if constexpr (EPI == 1) {
    // SwiGLU over interleaved rows (M = 1): the CTA's 16 RT row sums are formed in parallel (element (i, lane) of
    // row tile r holds row 16 r + lane / 4 for i = 0 and 16 r + 8 + lane / 4 for i = 2) and rounded to fp16 like
    // the GEMV's output; thread j < 8 RT then combines rows 2j (gate) and 2j + 1 (up) into output n0 / 2 + j, with
    // the roundings of the separate SiLU*up kernel
    __shared__ float rows_f[16 * RT];
    for (int e = threadIdx.x; e < kTile; e += blockDim.x) {
      const int rm = e >> 7, i = (e >> 5) & 3, ln = e & 31;
      const int r = rm / MT, mt = rm - r * MT;
      if (mt == 0 && (ln & 3) == 0 && (i & 1) == 0)
        rows_f[16 * r + (ln >> 2) + (i >= 2 ? 8 : 0)] = __half2float(__float2half_rn(tile_sum(e)));
    }
    __syncthreads();
    if (threadIdx.x < 8 * RT) {
      const int j = threadIdx.x;
      const float gf = rows_f[2 * j], uf = rows_f[2 * j + 1];
      const __half sg = __float2half_rn(gf / (1.f + expf(-gf)));
      if (n0 + 2 * j + 1 < N) p.y[n0 / 2 + j] = __float2half_rn(__half2float(sg) * uf);
    }
    return;
  }
  if constexpr (EPI != 3) {
    for (int e = threadIdx.x; e < kTile; e += blockDim.x) store(e, tile_sum(e));
  }
  if constexpr (EPI == 2 || EPI == 3) {
    // the last row tile to finish (the counter counts the tiles' finishing CTAs -- rank 0 of each cluster -- and
    // is left zero for the next call) adds the whole output row into the residual stream and normalizes it.
    // Every such CTA first loads its pieces of the residual row and the norm weights (neither is written by this
    // kernel before the count completes), so the last one starts with only y still to read.
    constexpr int kPre = 4;   // pieces held per thread: N <= 8 * kPre * blockDim covers N <= 8192 at 256 threads
    __shared__ int last, timed_out;
    __shared__ float epi_red[32];
    const int n8 = N / 8;
    uint4 xpre[kPre], wpre[kPre];
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
      const int v = threadIdx.x + j * blockDim.x;
      if (v < n8) {
        xpre[j] = ldg_cg_u4(p.epi_x + 8 * (size_t)v);
        wpre[j] = ldg_stream(reinterpret_cast<const uint4*>(p.epi_w) + v);
      }
    }
    uint32_t ep = 0;
    if constexpr (EPI == 3) {
      // this tile's fp16 partial, pushed over NVLink into region (ep & 1, rank) of every rank's buffer as
      // self-validating 8-byte words (epoch << 32 | two fp16 outputs): a reader polls each word until it carries
      // the epoch, so the pushes need no fence and no flag
      __shared__ __align__(16) __half tile_h[16 * RT];
      __shared__ uint32_t ep_s;
      if (threadIdx.x == 0) ep_s = *reinterpret_cast<volatile uint32_t*>(p.ar_epoch) + 1;
      for (int e = threadIdx.x; e < kTile; e += blockDim.x) {
        const int rm = e >> 7, i = (e >> 5) & 3, ln = e & 31;
        const int r = rm / MT, mt = rm - r * MT;
        if (mt == 0 && (ln & 3) == 0 && (i & 1) == 0)   // activation row 0
          tile_h[16 * r + (ln >> 2) + (i >= 2 ? 8 : 0)] = __float2half_rn(tile_sum(e));
      }
      __syncthreads();
      ep = ep_s;
      const int world = p.ar_world;
      for (int j = threadIdx.x; j < 8 * RT * world; j += blockDim.x) {
        const int dst = j / (8 * RT), wi = j - dst * (8 * RT);
        const int row = n0 + 2 * wi;
        if (row + 2 <= N) {
          uint64_t* region = reinterpret_cast<uint64_t*>(p.ar_bufs[dst] + kPeerFlagBytes) +
                             (size_t)((ep & 1) * world + p.ar_rank) * (p.ar_cap / 2);
          const uint32_t data = reinterpret_cast<const uint32_t*>(tile_h)[wi];
          st_volatile_u64(region + row / 2, ((uint64_t)ep << 32) | data);
        }
      }
    }
    __syncthreads();   // this CTA's stores precede thread 0's release (bar.sync, then a cumulative release)
    if (threadIdx.x == 0) {
      last = atom_add_acq_rel_gpu(p.epi_counter, 1) == gridDim.x - 1;
      timed_out = 0;
    }
    __syncthreads();
    if (!last) return;
    // piece v of the finished output row: y as stored above, or the rank-ordered fp32 sum of the ranks' words
    // (each polled, for at most ~1 s in all, until it carries this epoch)
    const long long t_wait = clock64();
    if constexpr (EPI == 3) {
      // every rank's words of this thread's pieces carry the epoch, or the wait ran out: then nothing is written
      // (y, x_res and h keep their values, the epoch does not advance) and the status word holds 2 for the host
      for (int v = threadIdx.x; v < N / 8 && !timed_out; v += blockDim.x) {
        const uint64_t* base = reinterpret_cast<const uint64_t*>(p.ar_bufs[p.ar_rank] + kPeerFlagBytes) +
                               (size_t)(ep & 1) * p.ar_world * (p.ar_cap / 2) + 4 * (size_t)v;
        for (int r = 0; r < p.ar_world && !timed_out; ++r)
          for (int k = 0; k < 4; ++k)
            while ((uint32_t)(ld_volatile_u64(base + (size_t)r * (p.ar_cap / 2) + k) >> 32) != ep) {
              if (clock64() - t_wait > kPeerWaitCycles) {
                atomicExch(&g_device_status, kErrPeerTimeout);
                timed_out = 1;
                break;
              }
            }
      }
      __syncthreads();
      if (timed_out) {
        if (threadIdx.x == 0) *p.epi_counter = 0;
        return;
      }
    }
    auto y_piece = [&](int v) -> uint4 {
      if constexpr (EPI == 2) {
        return ldg_cg_u4(p.y + 8 * (size_t)v);
      } else {
        const uint64_t* base = reinterpret_cast<const uint64_t*>(p.ar_bufs[p.ar_rank] + kPeerFlagBytes) +
                               (size_t)(ep & 1) * p.ar_world * (p.ar_cap / 2) + 4 * (size_t)v;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int r = 0; r < p.ar_world; ++r) {
          const uint64_t* src = base + (size_t)r * (p.ar_cap / 2);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint64_t wv = ld_volatile_u64(src + k);
            while ((uint32_t)(wv >> 32) != ep) {
              if (clock64() - t_wait > kPeerWaitCycles) {
                atomicExch(&g_device_status, kErrPeerTimeout);
                timed_out = 1;
                break;
              }
              wv = ld_volatile_u64(src + k);
            }
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv));
            acc[2 * k] += f.x;
            acc[2 * k + 1] += f.y;
          }
        }
        uint4 o;
        __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) oh[k] = __floats2half2_rn(acc[2 * k], acc[2 * k + 1]);
        if (p.y) reinterpret_cast<uint4*>(p.y)[v] = o;
        return o;
      }
    };
    float ss = 0.f;
    auto add_piece = [&](int v, uint4& xv) {
      const uint4 yv = y_piece(v);
      __half2* xh = reinterpret_cast<__half2*>(&xv);
      const __half2* yh = reinterpret_cast<const __half2*>(&yv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xh[j] = __hadd2(xh[j], yh[j]);
        const float2 f = __half22float2(xh[j]);
        ss += f.x * f.x + f.y * f.y;
      }
      reinterpret_cast<uint4*>(p.epi_x)[v] = xv;
    };
    auto norm_piece = [&](int v, const uint4& xv, const uint4& wv, float inv) {
      const __half2* xh = reinterpret_cast<const __half2*>(&xv);
      const __half2* wh = reinterpret_cast<const __half2*>(&wv);
      uint4 o;
      __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(xh[j]);
        oh[j] = __hmul2(wh[j], __floats2half2_rn(f.x * inv, f.y * inv));
      }
      reinterpret_cast<uint4*>(p.epi_h)[v] = o;
    };
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
      const int v = threadIdx.x + j * blockDim.x;
      if (v < n8) add_piece(v, xpre[j]);
    }
    for (int v = threadIdx.x + kPre * blockDim.x; v < n8; v += blockDim.x) {   // rows longer than the registers hold
      uint4 xv = ldg_cg_u4(p.epi_x + 8 * (size_t)v);
      add_piece(v, xv);
    }
    const float inv = rsqrtf(cta_sum_f32(ss, epi_red) / (float)N + p.epi_eps);
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
      const int v = threadIdx.x + j * blockDim.x;
      if (v < n8) norm_piece(v, xpre[j], wpre[j], inv);
    }
    for (int v = threadIdx.x + kPre * blockDim.x; v < n8; v += blockDim.x) {   // this thread's own writes above
      const uint4 xv = reinterpret_cast<const uint4*>(p.epi_x)[v];
      norm_piece(v, xv, ldg_stream(reinterpret_cast<const uint4*>(p.epi_w) + v), inv);
    }
    __syncthreads();   // timed_out is final
    if (threadIdx.x == 0) {
      *p.epi_counter = 0;
      if constexpr (EPI == 3) {
        if (!timed_out) *p.ar_epoch = ep;
      }
    }
  }
}

// Plain decode GEMV, M <= 8, one 16-row tile and the whole K range per CTA: the arithmetic of gemv_oneshot_kernel
// at its unsplit, one-row-tile configuration -- the same chunk-to-warp assignment (chunk c to warp c % NW, in
// order), the same mma.sync sequence per chunk, the same fp32 operations in the same order, so the outputs have
// its bits -- with less work around it:
//   * each warp stages only the activations of its own chunks (one 16-byte load and store per lane and 128 k of
//     a row), so no CTA barrier stands between the wait on the previous kernel and the first mma;
//   * the only barrier is the one before the cross-warp sum, which covers just the 16 M real outputs of the tile;
//   * the chunk count per warp and M == 1 are compile-time, so index math and the single-row epilogue fold away.
template <int CPW, bool EARLY, bool M1>
__global__ void __launch_bounds__(512) gemv_tile_kernel(GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int NW = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int K = p.K, N = p.N, M = M1 ? 1 : p.M, KC = K >> 7, KG = p.KG, cpg = p.cpg;
  const int n0 = blockIdx.x * 16;
  const int xrow = CPW * 256 + 16;             // bytes per activation row in a warp's region (16-byte skew)
  uint8_t* xw = smem + warp * M * xrow;        // this warp's activations: [M][CPW chunks of 256 bytes]
  float* red = reinterpret_cast<float*>(smem + NW * M * xrow);   // [NW][16 M] partial sums

  const size_t row_u4 = (size_t)(K >> 5);
  const int ra = min(n0 + g, N - 1), rb = min(n0 + g + 8, N - 1);   // tail rows re-read row N - 1
  const uint4* wa = reinterpret_cast<const uint4*>(p.w) + (size_t)ra * row_u4 + t;
  const uint4* wb = reinterpret_cast<const uint4*>(p.w) + (size_t)rb * row_u4 + t;
  const uint16_t* sa = reinterpret_cast<const uint16_t*>(p.s) + (size_t)ra * KG;
  const uint16_t* sb = reinterpret_cast<const uint16_t*>(p.s) + (size_t)rb * KG;

  uint4 qa[CPW], qb[CPW];
  uint16_t ssa[CPW], ssb[CPW];
  pdl_launch_dependents();
  if (!EARLY) pdl_wait();
#pragma unroll
  for (int i = 0; i < CPW; ++i) {
    const int c = warp + NW * i;
    if (c < KC) {
      const int grp = cpg == 1 ? c : c / cpg;
      qa[i] = ldg_stream(wa + 4 * c);
      qb[i] = ldg_stream(wb + 4 * c);
      ssa[i] = ldg_u16(sa + grp);
      ssb[i] = ldg_u16(sb + grp);
    }
  }
  if (EARLY) pdl_wait_after_loads(p.wait_guard);

  // this warp's activations: piece (m, i, j) = 16 bytes j of chunk warp + NW i of row m, loaded through L2 (the
  // previous kernel may just have written them) in rounds of PR pieces per lane -- every load of a round issued
  // before its first shared-memory store, so a round costs one L2 round trip
  constexpr int PR = M1 ? (CPW / 2 > 0 ? CPW / 2 : 1) : 4;
  {
    const uint8_t* xg = reinterpret_cast<const uint8_t*>(p.x);
    const int total = M * CPW * 16;
    for (int base = 0; base < total; base += 32 * PR) {
      uint4 v[PR];
      int off[PR];
#pragma unroll
      for (int r = 0; r < PR; ++r) {
        const int e = base + 32 * r + lane;
        const int m = M1 ? 0 : e / (CPW * 16), rr = M1 ? e : e - m * (CPW * 16), i = rr >> 4, j = rr & 15;
        const int c = warp + NW * i;
        off[r] = -1;
        if (e < total && c < KC) {
          v[r] = ldg_cg_u4(xg + (size_t)m * K * 2 + (size_t)c * 256 + j * 16);
          off[r] = m * xrow + i * 256 + j * 16;
        }
      }
#pragma unroll
      for (int r = 0; r < PR; ++r)
        if (off[r] >= 0) *reinterpret_cast<uint4*>(xw + off[r]) = v[r];
    }
  }
  // the first chunk's fragments are decoded while the activations are in flight
  uint32_t fr0[4][8];
#pragma unroll
  for (int qd = 0; qd < 4; ++qd) {
    const uint32_t w0 = (&qa[0].x)[qd], w1 = (&qb[0].x)[qd];
    fr0[qd][0] = q_pair_lo(w0); fr0[qd][1] = q_pair_lo(w1); fr0[qd][2] = q_pair_hi(w0); fr0[qd][3] = q_pair_hi(w1);
    fr0[qd][4] = q_pair_lo(w0 >> 8); fr0[qd][5] = q_pair_lo(w1 >> 8);
    fr0[qd][6] = q_pair_hi(w0 >> 8); fr0[qd][7] = q_pair_hi(w1 >> 8);
  }
  __syncwarp();

  // ldmatrix row addresses: lane L serves row (L & 7) of 8x8 matrix L >> 3; rows past M repeat row M - 1
  const uint32_t xaddr = smem_u32(xw + min(lane & 7, M - 1) * xrow + (lane >> 3) * 16);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < CPW; ++i) {
    if (warp + NW * i < KC) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int qd = 0; qd < 4; ++qd) {
        uint32_t xb[4];
        ldsm_x4(xb, xaddr + i * 256 + qd * 64);
        uint32_t f[8];
        if (i == 0) {
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] = fr0[qd][j];
        } else {
          const uint32_t w0 = (&qa[i].x)[qd], w1 = (&qb[i].x)[qd];
          f[0] = q_pair_lo(w0); f[1] = q_pair_lo(w1); f[2] = q_pair_hi(w0); f[3] = q_pair_hi(w1);
          f[4] = q_pair_lo(w0 >> 8); f[5] = q_pair_lo(w1 >> 8); f[6] = q_pair_hi(w0 >> 8); f[7] = q_pair_hi(w1 >> 8);
        }
        mma16816(d, f[0], f[1], f[2], f[3], xb[0], xb[1]);
        mma16816(d, f[4], f[5], f[6], f[7], xb[2], xb[3]);
      }
      const float s0 = h2f_bits(ssa[i]), s1 = h2f_bits(ssb[i]);
      acc[0] = fmaf(s0, d[0], acc[0]);
      acc[2] = fmaf(s1, d[2], acc[2]);
      if (!M1) {
        acc[1] = fmaf(s0, d[1], acc[1]);
        acc[3] = fmaf(s1, d[3], acc[3]);
      }
    }
  }
  // partial sums of the tile's 16 x M outputs: lane (g, t) holds rows g, g + 8 and activation rows 2t, 2t + 1
  const int MS = 16 * M;
  if (M1) {
    if (t == 0) {
      red[warp * 16 + g] = acc[0];
      red[warp * 16 + g + 8] = acc[2];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = 2 * t + (i & 1);
      if (m < M) red[warp * MS + (g + (i >= 2 ? 8 : 0)) * M + m] = acc[i];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < MS; e += blockDim.x) {   // 16 M outputs; a one-warp CTA loops at M > 2
    float v = 0.f;
#pragma unroll 8
    for (int w = 0; w < NW; ++w) v += red[w * MS + e];   // the loads issue together; the adds keep their order
    const int row = M1 ? e : e / M, m = M1 ? 0 : e - row * M;
    if (n0 + row < N) p.y[(size_t)m * N + n0 + row] = out_half(v, p.bias, n0 + row);
  }
}

size_t tile_smem_bytes(int M, int nw, int cpw) { return (size_t)nw * M * (cpw * 256 + 16) + (size_t)nw * 16 * M * 4; }

template <int CPW, bool M1>
static cudaError_t launch_tile_t(const GemvParams& p, int nw, bool pdl, cudaStream_t st) {
  auto kern = (p.flags & kFlagEarlyWeights) ? gemv_tile_kernel<CPW, true, M1> : gemv_tile_kernel<CPW, false, M1>;
  const size_t smem = tile_smem_bytes(p.M, nw, CPW);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N + 15) / 16, 1, 1);
  cfg.blockDim = dim3(nw * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

cudaError_t launch_gemv_tile(const GemvParams& p, const OneshotConfig& c, cudaStream_t st) {
  if (p.M < 1 || p.M > 8 || c.ksplit != 1 || c.rt != 1 || p.pro || p.epi) return cudaErrorInvalidConfiguration;
  const bool m1 = p.M == 1;
#define LB_TILE(CPW_) \
  if (c.cpw == CPW_) return m1 ? launch_tile_t<CPW_, true>(p, c.warps, c.pdl, st) : launch_tile_t<CPW_, false>(p, c.warps, c.pdl, st);
  LB_TILE(2) LB_TILE(4) LB_TILE(8)
#undef LB_TILE
  return cudaErrorInvalidConfiguration;
}

// Plain decode GEMV, M <= 8, the weights of the CTA's 16-row tile landed in shared memory by one bulk copy. The
// tile's rows are contiguous in the mma layout (16 x K/2 bytes), so one cp.async.bulk moves them -- issued by one
// thread before the wait on the previous kernel, completing on an mbarrier -- and no register holds a weight in
// flight: a CTA needs few registers, several CTAs share an SM, and the next kernel in the stream finds room to
// start its own copies while this one computes. Scales, activations, arithmetic and the reduction are those of
// gemv_tile_kernel (and so the bits of gemv_oneshot_kernel at the same tiling).
__host__ __device__ inline size_t bulk_w_bytes(int K) { return (size_t)16 * (K / 2); }
size_t bulk_smem_bytes(int M, int K, int nw, int cpw) {
  return bulk_w_bytes(K) + (size_t)nw * M * (cpw * 256 + 16) + (size_t)nw * 16 * M * 4 + 16;
}

template <int CPW, bool EARLY, bool M1>
__global__ void __launch_bounds__(512) gemv_bulk_kernel(GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int NW = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int K = p.K, N = p.N, M = M1 ? 1 : p.M, KC = K >> 7, KG = p.KG, cpg = p.cpg;
  const int n0 = blockIdx.x * 16, rows = min(16, N - n0);
  const int row_bytes = K >> 1;
  const int xrow = CPW * 256 + 16;
  uint8_t* ws = smem;                                             // [16][K/2] weights (rows past N: never read back)
  uint8_t* xw = smem + bulk_w_bytes(K) + warp * M * xrow;          // this warp's activations
  float* red = reinterpret_cast<float*>(smem + bulk_w_bytes(K) + NW * M * xrow);
  uint64_t* bar = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + NW * 16 * M * 4);

  pdl_launch_dependents();
  if (!EARLY) pdl_wait();
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
    const uint32_t bytes = (uint32_t)rows * (uint32_t)row_bytes;   // a multiple of 64
    mbar_arrive_expect_tx(bar, bytes);
    bulk_copy_g2s(ws, reinterpret_cast<const uint8_t*>(p.w) + (size_t)n0 * row_bytes, bytes, bar);
  }
  const int ra = min(n0 + g, N - 1), rb = min(n0 + g + 8, N - 1);
  const uint16_t* sa = reinterpret_cast<const uint16_t*>(p.s) + (size_t)ra * KG;
  const uint16_t* sb = reinterpret_cast<const uint16_t*>(p.s) + (size_t)rb * KG;
  uint16_t ssa[CPW], ssb[CPW];
#pragma unroll
  for (int i = 0; i < CPW; ++i) {
    const int c = warp + NW * i;
    if (c < KC) {
      const int grp = cpg == 1 ? c : c / cpg;
      ssa[i] = ldg_u16(sa + grp);
      ssb[i] = ldg_u16(sb + grp);
    }
  }
  __syncthreads();   // the barrier is initialized before anyone waits on it
  if (EARLY) pdl_wait_after_loads(p.wait_guard);

  constexpr int PR = M1 ? (CPW / 2 > 0 ? CPW / 2 : 1) : 4;
  {   // activations of this warp's chunks, as in gemv_tile_kernel
    const uint8_t* xg = reinterpret_cast<const uint8_t*>(p.x);
    const int total = M * CPW * 16;
    for (int base = 0; base < total; base += 32 * PR) {
      uint4 v[PR];
      int off[PR];
#pragma unroll
      for (int r = 0; r < PR; ++r) {
        const int e = base + 32 * r + lane;
        const int m = M1 ? 0 : e / (CPW * 16), rr = M1 ? e : e - m * (CPW * 16), i = rr >> 4, j = rr & 15;
        const int c = warp + NW * i;
        off[r] = -1;
        if (e < total && c < KC) {
          v[r] = ldg_cg_u4(xg + (size_t)m * K * 2 + (size_t)c * 256 + j * 16);
          off[r] = m * xrow + i * 256 + j * 16;
        }
      }
#pragma unroll
      for (int r = 0; r < PR; ++r)
        if (off[r] >= 0) *reinterpret_cast<uint4*>(xw + off[r]) = v[r];
    }
  }
  // the weights have landed (bounded wait: a copy that never completes records kErrBarrierTimeout and the outputs
  // are undefined, instead of a hang)
  {
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, 0)) {
      if (++spins > kSpinLimit) {
        if (lane == 0) atomicExch(&g_device_status, kErrBarrierTimeout);
        break;
      }
    }
  }
  __syncwarp();

  const uint32_t xaddr = smem_u32(xw + min(lane & 7, M - 1) * xrow + (lane >> 3) * 16);
  const uint8_t* wra = ws + g * row_bytes + t * 16;
  const uint8_t* wrb = ws + (g + 8) * row_bytes + t * 16;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < CPW; ++i) {
    const int c = warp + NW * i;
    if (c < KC) {
      const uint4 qa = *reinterpret_cast<const uint4*>(wra + c * 64);
      const uint4 qb = *reinterpret_cast<const uint4*>(wrb + c * 64);
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int qd = 0; qd < 4; ++qd) {
        uint32_t xb[4];
        ldsm_x4(xb, xaddr + i * 256 + qd * 64);
        const uint32_t w0 = (&qa.x)[qd], w1 = (&qb.x)[qd];
        uint32_t f[8];
        f[0] = q_pair_lo(w0); f[1] = q_pair_lo(w1); f[2] = q_pair_hi(w0); f[3] = q_pair_hi(w1);
        f[4] = q_pair_lo(w0 >> 8); f[5] = q_pair_lo(w1 >> 8); f[6] = q_pair_hi(w0 >> 8); f[7] = q_pair_hi(w1 >> 8);
        mma16816(d, f[0], f[1], f[2], f[3], xb[0], xb[1]);
        mma16816(d, f[4], f[5], f[6], f[7], xb[2], xb[3]);
      }
      const float s0 = h2f_bits(ssa[i]), s1 = h2f_bits(ssb[i]);
      acc[0] = fmaf(s0, d[0], acc[0]);
      acc[2] = fmaf(s1, d[2], acc[2]);
      if (!M1) {
        acc[1] = fmaf(s0, d[1], acc[1]);
        acc[3] = fmaf(s1, d[3], acc[3]);
      }
    }
  }
  const int MS = 16 * M;
  if (M1) {
    if (t == 0) {
      red[warp * 16 + g] = acc[0];
      red[warp * 16 + g + 8] = acc[2];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = 2 * t + (i & 1);
      if (m < M) red[warp * MS + (g + (i >= 2 ? 8 : 0)) * M + m] = acc[i];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < MS; e += blockDim.x) {
    float v = 0.f;
#pragma unroll 8
    for (int w = 0; w < NW; ++w) v += red[w * MS + e];   // the loads issue together; the adds keep their order
    const int row = M1 ? e : e / M, m = M1 ? 0 : e - row * M;
    if (row < rows) p.y[(size_t)m * N + n0 + row] = out_half(v, p.bias, n0 + row);
  }
}

template <int CPW, bool M1>
static cudaError_t launch_bulk_t(const GemvParams& p, int nw, bool pdl, cudaStream_t st) {
  auto kern = (p.flags & kFlagEarlyWeights) ? gemv_bulk_kernel<CPW, true, M1> : gemv_bulk_kernel<CPW, false, M1>;
  const size_t smem = bulk_smem_bytes(p.M, p.K, nw, CPW);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N + 15) / 16, 1, 1);
  cfg.blockDim = dim3(nw * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

cudaError_t launch_gemv_bulk(const GemvParams& p, const OneshotConfig& c, cudaStream_t st) {
  if (p.M < 1 || p.M > 8 || c.ksplit != 1 || c.rt != 1 || p.pro || p.epi) return cudaErrorInvalidConfiguration;
  const bool m1 = p.M == 1;
#define LB_BULK(CPW_) \
  if (c.cpw == CPW_) return m1 ? launch_bulk_t<CPW_, true>(p, c.warps, c.pdl, st) : launch_bulk_t<CPW_, false>(p, c.warps, c.pdl, st);
  LB_BULK(2) LB_BULK(4) LB_BULK(8)
#undef LB_BULK
  return cudaErrorInvalidConfiguration;
}

template <int MT, int RT, int CPW, int PRO = 0, int EPI = 0>
static cudaError_t launch_oneshot_t(const GemvParams& p, const OneshotConfig& c, cudaStream_t st) {
  auto kern = (p.flags & kFlagEarlyWeights) ? gemv_oneshot_kernel<MT, RT, CPW, true, PRO, EPI>
                                            : gemv_oneshot_kernel<MT, RT, CPW, false, PRO, EPI>;
  const size_t smem = oneshot_smem_bytes(p.M, p.K, c.ksplit, c.warps, RT);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N + 16 * RT - 1) / (16 * RT), c.ksplit, 1);
  cfg.blockDim = dim3(c.warps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (c.ksplit > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = c.ksplit;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (c.pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

size_t oneshot_smem_bytes(int M, int K, int nsplit, int nw, int rt) {
  const int KC = K >> 7, max_nl = (KC + nsplit - 1) / nsplit;
  const int mt = M <= 8 ? 1 : 2;
  const size_t x_bytes = (size_t)M * (max_nl * 256 + 16);
  const size_t red_bytes = (size_t)(nw + (nsplit > 1 ? nsplit : 0)) * rt * mt * 128 * 4;
  return x_bytes > red_bytes ? x_bytes : red_bytes;
}

cudaError_t launch_gemv_oneshot(const GemvParams& p, const OneshotConfig& c, cudaStream_t st) {
  const int mt = p.M <= 8 ? 1 : 2;
  if (p.epi != 0) {   // decode-step epilogues: M = 1, any K split and row tiling of the plain GEMV
    if (p.M != 1 || p.pro != 0) return cudaErrorInvalidConfiguration;
#define LB_ONESHOT_EPI(EPI_, RT_, CPW_) \
    if (p.epi == EPI_ && c.rt == RT_ && c.cpw == CPW_) return launch_oneshot_t<1, RT_, CPW_, 0, EPI_>(p, c, st);
    LB_ONESHOT_EPI(1, 1, 2) LB_ONESHOT_EPI(1, 1, 4) LB_ONESHOT_EPI(1, 1, 8) LB_ONESHOT_EPI(1, 2, 2)
    LB_ONESHOT_EPI(1, 2, 4) LB_ONESHOT_EPI(2, 1, 2) LB_ONESHOT_EPI(2, 1, 4) LB_ONESHOT_EPI(2, 1, 8)
    LB_ONESHOT_EPI(2, 2, 2) LB_ONESHOT_EPI(2, 2, 4) LB_ONESHOT_EPI(3, 1, 2) LB_ONESHOT_EPI(3, 1, 4)
    LB_ONESHOT_EPI(3, 1, 8) LB_ONESHOT_EPI(3, 2, 2) LB_ONESHOT_EPI(3, 2, 4)
#undef LB_ONESHOT_EPI
    return cudaErrorInvalidConfiguration;
  }
  if (p.pro != 0) {   // decode-step prologues: M = 1, the whole K range in one CTA, one row tile
    if (p.M != 1 || c.ksplit != 1 || c.rt != 1) return cudaErrorInvalidConfiguration;
#define LB_ONESHOT_PRO(PRO_, CPW_) \
    if (p.pro == PRO_ && c.cpw == CPW_) return launch_oneshot_t<1, 1, CPW_, PRO_>(p, c, st);
    LB_ONESHOT_PRO(1, 2) LB_ONESHOT_PRO(1, 4) LB_ONESHOT_PRO(1, 8)
    LB_ONESHOT_PRO(2, 2) LB_ONESHOT_PRO(2, 4) LB_ONESHOT_PRO(2, 8)
#undef LB_ONESHOT_PRO
    return cudaErrorInvalidConfiguration;
  }
#define LB_ONESHOT(MT_, RT_, CPW_) \
  if (mt == MT_ && c.rt == RT_ && c.cpw == CPW_) return launch_oneshot_t<MT_, RT_, CPW_>(p, c, st);
  LB_ONESHOT(1, 1, 2) LB_ONESHOT(1, 1, 4) LB_ONESHOT(1, 1, 8) LB_ONESHOT(1, 2, 2) LB_ONESHOT(1, 2, 4)
  LB_ONESHOT(2, 1, 2) LB_ONESHOT(2, 1, 4) LB_ONESHOT(2, 1, 8) LB_ONESHOT(2, 2, 2) LB_ONESHOT(2, 2, 4)
#undef LB_ONESHOT
  return cudaErrorInvalidConfiguration;
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
        uint4 xv;
        asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(xv.x), "=r"(xv.y), "=r"(xv.z), "=r"(xv.w)
                     : "l"(x4 + (size_t)m * (K >> 3) + 4 * c + i));
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
      if (lane == 0 && n0 + r < N) p.y[(size_t)m * N + n0 + r] = out_half(v, p.bias, n0 + r);
    }
}

// ------------------------------------------------------------------------------------------------ launchers

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
