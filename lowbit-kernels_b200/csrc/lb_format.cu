// Format kernels: dequantize (prefill path), quantize (model preparation) and layout repacking.
//
//   dequant   fp16 W[N, K] = fp16_rn((u - 8) * scale) from the canonical, v3 or mma layout, bit-identical to
//             the reference's dequant_kernel / dequant_mma_kernel (csrc/w4_gemv.cu:296-310, 393-408) and to
//             lowbit/ops.py:119-123. Every thread writes whole 16-byte runs of 8 consecutive k, so a warp's
//             store instruction covers 512 contiguous bytes (the reference's mma variant stores 4-byte pairs at
//             a 16-byte stride).
//   quantize  lowbit/quant.py:23-35 / lowbit/ops.py:81-116 on the GPU, with the optional clip grid.
//   repack    canonical -> v3 or mma order (lowbit/quant.py:55-78) on the GPU, so a model's weights never
//             travel back to the host to be interleaved.
#include "lb_common.cuh"
#include "lb_launch.h"

namespace lb {

// The exact fp16 value (u - 8) * scale for the pair j of a v3-order word: mul.rn.f16x2 of two fp16 values
// rounds the exact product once, the same rounding as fp32 (q * s exact) followed by a conversion to fp16.
__device__ __forceinline__ uint32_t deq_pair(uint32_t word, int j, uint32_t s2) {
  return hmul2_bits(q_pair(word, j), s2);
}

// canonical byte -> exact f16x2 (lo nibble, hi nibble) minus 8
__device__ __forceinline__ uint32_t deq_byte(uint32_t b, uint32_t s2) {
  return hmul2_bits(hsub2_bits((b & 0xFu) | ((b & 0xF0u) << 12) | kMagic, kBias1032), s2);
}

// layout 0 (canonical) and 1 (v3): thread = one 32-bit word = 8 consecutive k -> one 16-byte store; a warp's
// loads cover 128 contiguous bytes and its stores 512. Idx is 32-bit whenever the layer has fewer than 2^32 words.
template <bool V3, typename Idx>
__global__ void __launch_bounds__(256) dequant_linear_kernel(const uint32_t* __restrict__ w,
                                                             const uint16_t* __restrict__ s, uint4* __restrict__ out,
                                                             int N, int K, int G) {
  const Idx per_row = (Idx)(K >> 3), total = (Idx)N * per_row;
  const int KG = K / G;
  for (Idx idx = (Idx)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (Idx)gridDim.x * blockDim.x) {
    const Idx n = idx / per_row;
    const int k = (int)(idx - n * per_row) * 8;
    const uint16_t sb = __ldg(s + (size_t)n * KG + k / G);
    const uint32_t s2 = (uint32_t)sb | ((uint32_t)sb << 16);
    const uint32_t word = __ldg(w + idx);
    uint4 o;
    if (V3) {
      o.x = deq_pair(word, 0, s2); o.y = deq_pair(word, 1, s2); o.z = deq_pair(word, 2, s2); o.w = deq_pair(word, 3, s2);
    } else {
      o.x = deq_byte(word & 0xFFu, s2); o.y = deq_byte((word >> 8) & 0xFFu, s2);
      o.z = deq_byte((word >> 16) & 0xFFu, s2); o.w = deq_byte(word >> 24, s2);
    }
    out[idx] = o;
  }
}

// layout 2 (mma). Output octet o of a chunk (k = 8o .. 8o + 7, o = 4i + j) is pair j of word i of the chunk's four
// 16-byte words t = 0..3 (pair j of word i of word t holds k = 8o + 2t, + 1). Thread (chunk q, pair j) loads the
// chunk's 64 bytes as four 16-byte loads (the chunk's four threads share them through L1) and writes octets j,
// 4 + j, 8 + j, 12 + j, so the four threads of a chunk write 64 contiguous bytes per store instruction.
template <typename Idx>
__global__ void __launch_bounds__(256) dequant_mma_kernel(const uint4* __restrict__ w, const uint16_t* __restrict__ s,
                                                          uint4* __restrict__ out, int N, int K, int G) {
  const Idx KC = (Idx)(K >> 7), total = (Idx)N * KC * 4;
  const int KG = K / G, cpg = G >> 7;
  for (Idx idx = (Idx)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (Idx)gridDim.x * blockDim.x) {
    const Idx q = idx >> 2;        // chunk, row-major over (row, chunk)
    const int j = (int)(idx & 3);
    const Idx n = q / KC;
    const int c = (int)(q - n * KC);
    const uint16_t sb = __ldg(s + (size_t)n * KG + (cpg == 1 ? c : c / cpg));
    const uint32_t s2 = (uint32_t)sb | ((uint32_t)sb << 16);
    uint4 wt[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) wt[t] = __ldg(w + (size_t)q * 4 + t);
    uint4* dst = out + (size_t)q * 16 + j;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 r;
      r.x = deq_pair((&wt[0].x)[i], j, s2);
      r.y = deq_pair((&wt[1].x)[i], j, s2);
      r.z = deq_pair((&wt[2].x)[i], j, s2);
      r.w = deq_pair((&wt[3].x)[i], j, s2);
      dst[4 * i] = r;
    }
  }
}

static int grid_for(size_t work, int threads) {
  size_t blocks = (work + threads - 1) / threads;
  const size_t cap = 148 * 8;   // eight 256-thread blocks per SM are resident; larger problems loop
  return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

cudaError_t launch_dequant(const void* w, const void* s, __half* out, int N, int K, int G, int layout,
                           cudaStream_t st) {
  const int threads = 256;
  auto sp = reinterpret_cast<const uint16_t*>(s);
  auto op = reinterpret_cast<uint4*>(out);
  const bool small = (size_t)N * (size_t)(K >> 3) < (1ull << 31);   // every index fits 32 bits
  if (layout == 2) {
    auto wp = reinterpret_cast<const uint4*>(w);
    const int grid = grid_for((size_t)N * (K >> 7) * 4, threads);
    if (small) dequant_mma_kernel<uint32_t><<<grid, threads, 0, st>>>(wp, sp, op, N, K, G);
    else dequant_mma_kernel<uint64_t><<<grid, threads, 0, st>>>(wp, sp, op, N, K, G);
    return cudaGetLastError();
  }
  auto wp = reinterpret_cast<const uint32_t*>(w);
  const int grid = grid_for((size_t)N * (K >> 3), threads);
  if (layout == 1) {
    if (small) dequant_linear_kernel<true, uint32_t><<<grid, threads, 0, st>>>(wp, sp, op, N, K, G);
    else dequant_linear_kernel<true, uint64_t><<<grid, threads, 0, st>>>(wp, sp, op, N, K, G);
  } else {
    if (small) dequant_linear_kernel<false, uint32_t><<<grid, threads, 0, st>>>(wp, sp, op, N, K, G);
    else dequant_linear_kernel<false, uint64_t><<<grid, threads, 0, st>>>(wp, sp, op, N, K, G);
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ quantize

constexpr int kMaxClip = 32;
struct ClipGrid {
  float a[kMaxClip];
  int n;
};

template <typename T>
__device__ __forceinline__ float load_w(const T* p);
template <>
__device__ __forceinline__ float load_w<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float load_w<__half>(const __half* p) { return __half2float(__ldg(p)); }

__device__ __forceinline__ uint16_t scale_for(float amax, float a) {
  const float v = a == 1.0f ? amax : amax * a;
  uint16_t s = __half_as_ushort(__float2half_rn(__fdiv_rn(v, 7.0f)));
  return (s & 0x7FFFu) == 0 ? (uint16_t)0x3C00u : s;   // an all-zero group (or one that rounds to zero): 1.0
}

__device__ __forceinline__ int quant_value(float wv, float s) {
  float q = rintf(__fdiv_rn(wv, s));
  q = fminf(fmaxf(q, -8.f), 7.f);
  return (int)q;
}

// one warp per (row, group); lane handles pairs p = lane, lane + 32, ... (k = 2p, 2p + 1 -> packed byte p)
template <typename T>
__global__ void quantize_kernel(const T* __restrict__ w, uint8_t* __restrict__ packed, uint16_t* __restrict__ scales,
                                int N, int K, int G, ClipGrid clip) {
  const int lane = threadIdx.x & 31;
  const size_t warp_id = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int KG = K / G;
  if (warp_id >= (size_t)N * KG) return;
  const int n = (int)(warp_id / KG), grp = (int)(warp_id - (size_t)n * KG);
  const T* src = w + (size_t)n * K + (size_t)grp * G;
  float amax = 0.f;
  for (int i = lane; i < G; i += 32) amax = fmaxf(amax, fabsf(load_w(src + i)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));

  uint16_t best = scale_for(amax, clip.n > 0 ? clip.a[0] : 1.0f);
  if (clip.n > 1) {
    // try every clip factor; keep the first one with the smallest squared error (lowbit/ops.py:98-111)
    float best_err = 0.f;
    for (int ci = 0; ci < clip.n; ++ci) {
      const uint16_t sb = scale_for(amax, clip.a[ci]);
      const float s = h2f_bits(sb);
      float err = 0.f;
      for (int i = lane; i < G; i += 32) {
        const float wv = load_w(src + i);
        // (q * s - w)^2 with every operation rounded on its own, as lowbit/ops.py:101 computes it
        const float d = __fsub_rn(__fmul_rn((float)quant_value(wv, s), s), wv);
        err = __fadd_rn(err, __fmul_rn(d, d));
      }
      err = warp_sum(err);
      if (ci == 0 || err < best_err) { best = sb; best_err = err; }
    }
  }
  const float s = h2f_bits(best);
  for (int pi = lane; pi < G / 2; pi += 32) {
    const int u0 = quant_value(load_w(src + 2 * pi), s) + 8;
    const int u1 = quant_value(load_w(src + 2 * pi + 1), s) + 8;
    packed[(size_t)n * (K / 2) + (size_t)grp * (G / 2) + pi] = (uint8_t)(u0 | (u1 << 4));
  }
  if (lane == 0) scales[(size_t)n * KG + grp] = best;
}

cudaError_t launch_quantize(const void* w, int w_is_half, uint8_t* packed, __half* scales, int N, int K, int G,
                            const float* clip, int n_clip, cudaStream_t st) {
  ClipGrid cg_ = {};
  cg_.n = n_clip;
  for (int i = 0; i < n_clip && i < kMaxClip; ++i) cg_.a[i] = clip[i];
  const size_t warps = (size_t)N * (K / G);
  const int threads = 256;
  const size_t blocks = (warps * 32 + threads - 1) / threads;
  auto sp = reinterpret_cast<uint16_t*>(scales);
  if (w_is_half)
    quantize_kernel<__half><<<(unsigned)blocks, threads, 0, st>>>(reinterpret_cast<const __half*>(w), packed, sp, N, K, G, cg_);
  else
    quantize_kernel<float><<<(unsigned)blocks, threads, 0, st>>>(reinterpret_cast<const float*>(w), packed, sp, N, K, G, cg_);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ repack

__device__ __forceinline__ uint32_t ldg_u8(const uint8_t* p) { return (uint32_t)__ldg(p); }

// One thread per output 32-bit word. Canonical bytes b0..b3 (value order k0 + 2b, k0 + 2b + 1) go to v3 slots
// b (low nibble) and 4 + b (high nibble). For the mma order, output word 4t + i of a 64-byte chunk takes the
// canonical bytes 4s + t, s = 4i .. 4i + 3, of the same chunk (lowbit/quant.py:67-78).
__global__ void repack_kernel(const uint8_t* __restrict__ src, uint32_t* __restrict__ dst, int N, int K, int mma) {
  const size_t total = (size_t)N * (K >> 3);
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(idx / (K >> 3));
    const int q = (int)(idx - (size_t)n * (K >> 3));
    const uint8_t* row = src + (size_t)n * (K >> 1);
    uint32_t b[4];
    if (mma) {
      const int c = q >> 4, t = (q >> 2) & 3, i = q & 3;
#pragma unroll
      for (int e = 0; e < 4; ++e) b[e] = ldg_u8(row + 64 * c + 4 * (4 * i + e) + t);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) b[e] = ldg_u8(row + 4 * q + e);
    }
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) word |= ((b[e] & 0xFu) << (4 * e)) | ((b[e] >> 4) << (16 + 4 * e));
    dst[idx] = word;
  }
}

cudaError_t launch_repack(const uint8_t* canonical, uint8_t* out, int N, int K, int layout, cudaStream_t st) {
  const size_t work = (size_t)N * (K >> 3);
  const int threads = 256, grid = grid_for(work, threads);
  repack_kernel<<<grid, threads, 0, st>>>(canonical, reinterpret_cast<uint32_t*>(out), N, K, layout == 2);
  return cudaGetLastError();
}

}  // namespace lb
