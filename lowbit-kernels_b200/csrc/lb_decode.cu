// The small kernels of a batch-1 Qwen2 decode step around the INT4 projections (the decoder harness of the
// benchmark's end-to-end config; the reference drives a transformers model instead, bench/e2e.py:84-147).
//
// Every kernel reads the decode position from device memory, so one CUDA graph replays every step, and is
// launched with programmatic stream serialization: it lets its successor launch at entry and waits for its
// predecessor before touching activations. Arithmetic follows the transformers Qwen2 modules in fp32 with one
// rounding to fp16 per stored tensor.
#include <cuda_fp16.h>

#include <atomic>

#include "lb_common.cuh"
#include "lb_launch.h"

namespace lb {
namespace {

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

// x = fp16(x + r) when r is given (the residual add), then h = fp16(w * fp16(x * rsqrt(mean(x^2) + eps)))
// (Qwen2RMSNorm: the normalized value is rounded to fp16 before the weight multiply). One CTA; every thread
// loads its (up to kRmsVec) 8-wide pieces at once and keeps them in registers. H % 8 == 0.
constexpr int kRmsThreads = 256;
constexpr int kRmsVec = 4;   // H <= 8192

__global__ void __launch_bounds__(kRmsThreads) rmsnorm_kernel(__half* __restrict__ x, const __half* __restrict__ r,
                                                              const __half* __restrict__ w, __half* __restrict__ h,
                                                              int H, float eps) {
  __shared__ float red[32];
  pdl_launch_dependents();
  const int n8 = H / 8;
  uint4 xv[kRmsVec], rv[kRmsVec], wv[kRmsVec];
#pragma unroll
  for (int j = 0; j < kRmsVec; ++j) {   // the norm weights are model state: fetched before the dependency wait
    const int i = threadIdx.x + j * kRmsThreads;
    if (i < n8) wv[j] = reinterpret_cast<const uint4*>(w)[i];
  }
  pdl_wait();
#pragma unroll
  for (int j = 0; j < kRmsVec; ++j) {
    const int i = threadIdx.x + j * kRmsThreads;
    if (i < n8) {
      xv[j] = reinterpret_cast<const uint4*>(x)[i];
      if (r) rv[j] = reinterpret_cast<const uint4*>(r)[i];
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kRmsVec; ++j) {
    const int i = threadIdx.x + j * kRmsThreads;
    if (i < n8) {
      __half2* xh = reinterpret_cast<__half2*>(&xv[j]);
      if (r) {
        const __half2* rh = reinterpret_cast<const __half2*>(&rv[j]);
#pragma unroll
        for (int k = 0; k < 4; ++k) xh[k] = __hadd2(xh[k], rh[k]);
        reinterpret_cast<uint4*>(x)[i] = xv[j];
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(xh[k]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
  }
  const float inv = rsqrtf(block_sum(ss, red) / (float)H + eps);
#pragma unroll
  for (int j = 0; j < kRmsVec; ++j) {
    const int i = threadIdx.x + j * kRmsThreads;
    if (i < n8) {
      const __half2* xh = reinterpret_cast<const __half2*>(&xv[j]);
      const __half2* wh = reinterpret_cast<const __half2*>(&wv[j]);
      uint4 o;
      __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(xh[k]);
        const __half2 n = __floats2half2_rn(f.x * inv, f.y * inv);
        oh[k] = __hmul2(wh[k], n);
      }
      reinterpret_cast<uint4*>(h)[i] = o;
    }
  }
}

// Split attention for one query token, fused with the q|k|v epilogue. CTA (kv head, split) takes cache positions
// [64 s, 64 s + 64) that are <= pos:
//   * the range's cached K and V rows (< pos, written by earlier steps) are copied into shared memory with
//     cp.async before the kernel waits on its predecessor, so their HBM latency overlaps the q|k|v projection;
//   * q of the group's heads = RoPE(qkv + bias) (rotate-half pairing: dims j and j + hd/2, angle pos *
//     inv_freq[j]), in fp32 shared memory, pre-multiplied by the softmax scale;
//   * the CTA whose range holds pos also rotates k, and writes k and v (+ bias) into the caches at row pos;
//   * scores: one thread per (head, position), a full hd-long dot product (a warp = one head's 32 positions, so
//     q reads broadcast; K rows are padded by 16 bytes so the 32 rows a warp reads sit on distinct banks);
//   * writes the split's running max, sum of exponentials and unnormalized output (fp32) for attn_combine_kernel.
constexpr int kAttnChunk = 64;
constexpr int kAttnThreads = 256;

__host__ __device__ constexpr int attn_k_stride(int hd) { return hd + 8; }

// status word of the decode kernels (a position outside the cache); read by decode_device_error()
__device__ int g_decode_status;

__device__ __forceinline__ void rope_pair(float a, float b, float c, float s, float& ra, float& rb) {
  ra = a * c - b * s;
  rb = b * c + a * s;
}

// HD: the head dimension when it is a compile-time constant (64, 128: fully unrolled dot products), 0 for any
template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(const __half* __restrict__ qkv,
                                                                  const __half* __restrict__ bias,
                                                                  const float* __restrict__ inv_freq,
                                                                  const int64_t* __restrict__ pos_p, __half* kc,
                                                                  __half* vc, float* __restrict__ part_o,
                                                                  float* __restrict__ part_ml, int nh, int nkv, int hd_,
                                                                  int max_len_, float scale) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  pdl_launch_dependents();
  const int hd = HD ? HD : hd_, max_len = max_len_;
  const int kvh = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y;
  const int g = nh / nkv, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = kAttnThreads / 32, half = hd / 2;
  const int ks = attn_k_stride(hd);
  // the position and the cached rows below it were written by earlier steps, before this step's kernels
  const int64_t pos64 = *pos_p;
  if (pos64 < 0 || pos64 >= max_len) {   // nothing is read or written outside the caches
    if (threadIdx.x == 0) atomicExch(&g_decode_status, kErrBadPosition);
    pdl_wait();
    return;
  }
  const int pos = (int)pos64, L = pos + 1;
  const int p0 = split * kAttnChunk, np = min(kAttnChunk, L - p0);
  const size_t pbase = ((size_t)kvh * nsplit + split) * g;
  if (np <= 0) {   // nothing cached here yet: an empty partial
    pdl_wait();
    for (int i = threadIdx.x; i < g; i += blockDim.x) {
      part_ml[(pbase + i) * 2] = -INFINITY;
      part_ml[(pbase + i) * 2 + 1] = 0.f;
    }
    return;
  }
  __half* sk = reinterpret_cast<__half*>(sm_raw);               // [64][ks]
  __half* sv = sk + kAttnChunk * ks;                             // [64][ks]
  float* sq = reinterpret_cast<float*>(sv + kAttnChunk * ks);    // [g][hd]
  float* ss = sq + g * hd;                                       // [g][64]
  __half* q16 = reinterpret_cast<__half*>(ss + g * kAttnChunk);  // [8][ks]   tensor-core path: q in fp16
  __half* p16 = q16 + 8 * ks;                                    // [8][72]   tensor-core path: exp(s - m) in fp16
  // scores and P V on the tensor cores (mma.sync m16n8k16, the group's heads as the 8 columns) when the group
  // fits one n-tile and the head dim is a compile-time 64 or 128; the scalar loops otherwise
  const bool use_mma = HD != 0 && g <= 8;
  const int ncached = min(np, pos - p0), vec = hd / 8;
  const __half* kg = kc + ((size_t)kvh * max_len + p0) * hd;
  const __half* vg = vc + ((size_t)kvh * max_len + p0) * hd;
  for (int i = threadIdx.x; i < ncached * vec; i += blockDim.x) {
    const int r = i / vec, c8 = (i - r * vec) * 8;
    cp_async16(smem_addr(sk + r * ks + c8), kg + (size_t)r * hd + c8);
    cp_async16(smem_addr(sv + r * ks + c8), vg + (size_t)r * hd + c8);
  }
  cp_async_commit();
  // q of the group's heads, and (in the range holding pos) this token's k and v: thread (row, quad) takes dims
  // j..j+3 and their rotate-half partners j+hd/2..j+hd/2+3 with 8-byte loads, all issued in one round; the bias
  // and frequencies of the thread's first item are model state, fetched before the dependency wait
  const bool mine = pos < p0 + kAttnChunk;
  const int quads = half / 4, items = (g + (mine ? 2 : 0)) * quads;
  auto item_head = [&](int hh) { return hh < g ? kvh * g + hh : hh == g ? nh + kvh : nh + nkv + kvh; };
  uint2 ba0 = make_uint2(0, 0), bb0 = make_uint2(0, 0);
  float4 fr0 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (threadIdx.x < items) {
    const int hh = threadIdx.x / quads, j = (threadIdx.x - hh * quads) * 4;
    if (bias) {
      ba0 = *reinterpret_cast<const uint2*>(bias + (size_t)item_head(hh) * hd + j);
      bb0 = *reinterpret_cast<const uint2*>(bias + (size_t)item_head(hh) * hd + j + half);
    }
    fr0 = *reinterpret_cast<const float4*>(inv_freq + j);
  }
  pdl_wait();   // qkv comes from the previous kernel in the stream
  for (int i = threadIdx.x; i < items; i += blockDim.x) {
    const int hh = i / quads, j = (i - hh * quads) * 4;
    const int head = item_head(hh);   // q / k / v row of qkv
    const __half* src = qkv + (size_t)head * hd;
    uint2 ua = *reinterpret_cast<const uint2*>(src + j), ub = *reinterpret_cast<const uint2*>(src + j + half);
    const bool first = i == threadIdx.x;
    if (bias) {
      const uint2 ba = first ? ba0 : *reinterpret_cast<const uint2*>(bias + (size_t)head * hd + j);
      const uint2 bb = first ? bb0 : *reinterpret_cast<const uint2*>(bias + (size_t)head * hd + j + half);
      __half2* pa = reinterpret_cast<__half2*>(&ua);
      __half2* pb = reinterpret_cast<__half2*>(&ub);
      pa[0] = __hadd2(pa[0], *reinterpret_cast<const __half2*>(&ba.x));
      pa[1] = __hadd2(pa[1], *reinterpret_cast<const __half2*>(&ba.y));
      pb[0] = __hadd2(pb[0], *reinterpret_cast<const __half2*>(&bb.x));
      pb[1] = __hadd2(pb[1], *reinterpret_cast<const __half2*>(&bb.y));
    }
    const __half* ha4 = reinterpret_cast<const __half*>(&ua);
    const __half* hb4 = reinterpret_cast<const __half*>(&ub);
    if (hh == g + 1) {   // v: no rotation
      *reinterpret_cast<uint2*>(sv + (pos - p0) * ks + j) = ua;
      *reinterpret_cast<uint2*>(sv + (pos - p0) * ks + j + half) = ub;
      *reinterpret_cast<uint2*>(vc + ((size_t)kvh * max_len + pos) * hd + j) = ua;
      *reinterpret_cast<uint2*>(vc + ((size_t)kvh * max_len + pos) * hd + j + half) = ub;
      continue;
    }
    const float4 fr = first ? fr0 : *reinterpret_cast<const float4*>(inv_freq + j);
    const float frq[4] = {fr.x, fr.y, fr.z, fr.w};
    __half ra4[4], rb4[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float sn, cs;
      sincosf((float)pos * frq[c], &sn, &cs);
      float ra, rb;
      rope_pair(__half2float(ha4[c]), __half2float(hb4[c]), cs, sn, ra, rb);
      ra4[c] = __float2half_rn(ra);
      rb4[c] = __float2half_rn(rb);
    }
    if (hh < g) {   // q rounded to fp16 like the reference path, then scaled in fp32
      if (use_mma) {   // q16 holds 8 rows: only groups of up to 8 heads take the tensor-core path
        *reinterpret_cast<uint2*>(q16 + hh * ks + j) = *reinterpret_cast<const uint2*>(ra4);
        *reinterpret_cast<uint2*>(q16 + hh * ks + j + half) = *reinterpret_cast<const uint2*>(rb4);
      }
      *reinterpret_cast<float4*>(sq + hh * hd + j) =
          make_float4(__half2float(ra4[0]) * scale, __half2float(ra4[1]) * scale, __half2float(ra4[2]) * scale,
                      __half2float(ra4[3]) * scale);
      *reinterpret_cast<float4*>(sq + hh * hd + j + half) =
          make_float4(__half2float(rb4[0]) * scale, __half2float(rb4[1]) * scale, __half2float(rb4[2]) * scale,
                      __half2float(rb4[3]) * scale);
    } else {
      const uint2 ka = *reinterpret_cast<const uint2*>(ra4), kb = *reinterpret_cast<const uint2*>(rb4);
      *reinterpret_cast<uint2*>(sk + (pos - p0) * ks + j) = ka;
      *reinterpret_cast<uint2*>(sk + (pos - p0) * ks + j + half) = kb;
      *reinterpret_cast<uint2*>(kc + ((size_t)kvh * max_len + pos) * hd + j) = ka;
      *reinterpret_cast<uint2*>(kc + ((size_t)kvh * max_len + pos) * hd + j + half) = kb;
    }
  }
  if (use_mma) {   // V rows past the range enter the P V products (times P = 0): make them finite
    for (int i = threadIdx.x; i < (kAttnChunk - np) * (hd / 8); i += blockDim.x) {
      const int r = np + i / (hd / 8), c8 = (i % (hd / 8)) * 8;
      *reinterpret_cast<uint4*>(sv + r * ks + c8) = make_uint4(0, 0, 0, 0);
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  if (use_mma) {
    // S^T[16 positions][8 heads] per warp 0..3: A = K rows (ldmatrix), B = q16 rows; scaled in fp32 afterwards
    if (warp < 4 && warp * 16 < np) {
      float dd[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t a_base =
          smem_addr(sk + (warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * ks + (lane >> 4) * 8);
      const uint32_t b_base = smem_addr(q16 + (lane & 7) * ks + ((lane >> 3) & 1) * 8);
#pragma unroll
      for (int kk = 0; kk < (HD ? HD : 16) / 16; ++kk) {
        uint32_t a[4], b[2];
        ldsm_x4(a, a_base + kk * 32);
        ldsm_x2(b, b_base + kk * 32);
        mma16816(dd, a[0], a[1], a[2], a[3], b[0], b[1]);
      }
      const int gq = lane >> 2, tq = lane & 3;
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int p = warp * 16 + gq + 8 * r, h = 2 * tq + c;
          if (p < np && h < g) ss[h * kAttnChunk + p] = dd[2 * r + c] * scale;
        }
    }
  } else {
  // scores: thread (head h, position p), the whole dot product in fp32
  for (int i = threadIdx.x; i < g * kAttnChunk; i += blockDim.x) {
    const int h = i / kAttnChunk, p = i - h * kAttnChunk;
    if (p < np) {
      const float* q = sq + h * hd;
      const __half* k = sk + p * ks;
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int e = 0; e < (HD ? HD : hd); e += 8) {
        const uint4 kr = *reinterpret_cast<const uint4*>(k + e);
        const float4 qa = *reinterpret_cast<const float4*>(q + e);
        const float4 qb = *reinterpret_cast<const float4*>(q + e + 4);
        const __half2* kh = reinterpret_cast<const __half2*>(&kr);
        const float2 f0 = __half22float2(kh[0]), f1 = __half22float2(kh[1]);
        const float2 f2 = __half22float2(kh[2]), f3 = __half22float2(kh[3]);
        d0 = fmaf(qa.x, f0.x, d0);
        d1 = fmaf(qa.y, f0.y, d1);
        d0 = fmaf(qa.z, f1.x, d0);
        d1 = fmaf(qa.w, f1.y, d1);
        d0 = fmaf(qb.x, f2.x, d0);
        d1 = fmaf(qb.y, f2.y, d1);
        d0 = fmaf(qb.z, f3.x, d0);
        d1 = fmaf(qb.w, f3.y, d1);
      }
      ss[h * kAttnChunk + p] = d0 + d1;
    }
  }
  }
  __syncthreads();
  // per head: max and exponentials (warp h handles heads h, h + nw, ...)
  for (int h = warp; h < g; h += nw) {
    float m = -INFINITY;
    for (int p = lane; p < np; p += 32) m = fmaxf(m, ss[h * kAttnChunk + p]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    if (use_mma) {   // P in fp16 (zero past the range), and l summed from the rounded values P V uses
      for (int p = lane; p < kAttnChunk; p += 32) {
        const __half e = __float2half_rn(p < np ? expf(ss[h * kAttnChunk + p] - m) : 0.f);
        p16[h * 72 + p] = e;
        l += __half2float(e);
      }
    } else {
      for (int p = lane; p < np; p += 32) {
        const float e = expf(ss[h * kAttnChunk + p] - m);
        ss[h * kAttnChunk + p] = e;
        l += e;
      }
    }
    l = warp_sum(l);
    if (lane == 0) {
      part_ml[(pbase + h) * 2] = m;
      part_ml[(pbase + h) * 2 + 1] = l;
    }
  }
  __syncthreads();
  if (use_mma) {
    // O^T[16 dims][8 heads] per warp: A = V^T (ldmatrix.trans of V rows), B = P rows; 16 positions per step
    if (warp < (HD ? HD : 16) / 16) {
      float dd[4] = {0.f, 0.f, 0.f, 0.f};
      const int jm = lane >> 3, rm = lane & 7;
      const uint32_t a_base = smem_addr(sv + (rm + (jm >= 2 ? 8 : 0)) * ks + warp * 16 + (jm & 1) * 8);
      const uint32_t b_base = smem_addr(p16 + (lane & 7) * 72 + ((lane >> 3) & 1) * 8);
#pragma unroll
      for (int kb = 0; kb < kAttnChunk / 16; ++kb) {
        if (kb * 16 >= np) break;
        uint32_t a[4], b[2];
        ldsm_x4_trans(a, a_base + kb * 16 * ks * 2);
        ldsm_x2(b, b_base + kb * 32);
        mma16816(dd, a[0], a[1], a[2], a[3], b[0], b[1]);
      }
      const int gq = lane >> 2, tq = lane & 3;
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int e = warp * 16 + gq + 8 * r, h = 2 * tq + c;
          if (h < g) part_o[(pbase + h) * hd + e] = dd[2 * r + c];
        }
    }
    return;
  }
  // unnormalized outputs: thread (h, 4 dims) sums over the range's positions
  const int q4 = hd / 4;
  for (int i = threadIdx.x; i < g * q4; i += blockDim.x) {
    const int h = i / q4, e0 = (i - h * q4) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int p = 0; p < np; ++p) {
      const float w = ss[h * kAttnChunk + p];
      const uint2 vr = *reinterpret_cast<const uint2*>(sv + p * ks + e0);
      const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vr.x));
      const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vr.y));
      acc.x += w * v01.x;
      acc.y += w * v01.y;
      acc.z += w * v23.x;
      acc.w += w * v23.y;
    }
    *reinterpret_cast<float4*>(part_o + (pbase + h) * hd + e0) = acc;
  }
}

// out[head] = sum_s exp(m_s - M) o_s / sum_s exp(m_s - M) l_s over the splits that hold rows 0..pos (the others
// are empty); grid nh, block hd. The splits' (m, l) pairs are read once into shared memory (in parallel), warp 0
// turns them into weights exp(m_s - M) and their weighted sum, and the hd-long partial rows are read with
// independent loads.
constexpr int kCombineMaxSplits = 1024;
__global__ void attn_combine_kernel(const float* part_o, const float* part_ml, const int64_t* __restrict__ pos_p,
                                    __half* out, int nh, int nkv, int hd, int nsplit, int max_len) {
  __shared__ float sw[kCombineMaxSplits], sl[kCombineMaxSplits];
  __shared__ float s_den;
  pdl_launch_dependents();
  const int64_t pos = *pos_p;
  pdl_wait();
  if (pos < 0 || pos >= max_len) return;   // the split kernel has recorded the bad position
  const int nact = min(nsplit, (int)(pos / kAttnChunk) + 1);
  const int head = blockIdx.x, e = threadIdx.x, g = nh / nkv, kvh = head / g, h = head - kvh * g;
  for (int s = threadIdx.x; s < nact; s += blockDim.x) {
    const float2 v = *reinterpret_cast<const float2*>(part_ml + (((size_t)kvh * nsplit + s) * g + h) * 2);
    sw[s] = v.x;
    sl[s] = v.y;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float M = -INFINITY;
    for (int s = lane; s < nact; s += 32) M = fmaxf(M, sw[s]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float den = 0.f;
    for (int s = lane; s < nact; s += 32) {
      const float w = expf(sw[s] - M);
      sw[s] = w;
      den += w * sl[s];
    }
    den = warp_sum(den);
    if (lane == 0) s_den = den;
  }
  __syncthreads();
  float num = 0.f;
  const float* po = part_o + ((size_t)kvh * nsplit * g + h) * hd + e;
#pragma unroll 8
  for (int s = 0; s < nact; ++s) num += sw[s] * po[(size_t)s * g * hd];
  out[(size_t)head * hd + e] = __float2half_rn(num / s_den);
}

// a = fp16(fp16(silu(g)) * u) from the fused [gate | up] projection output (act_fn(gate) * up in fp16)
__global__ void silu_mul_kernel(const __half* gu, __half* a, int I) {
  pdl_launch_dependents();
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < I; i += gridDim.x * blockDim.x) {
    const float g = __half2float(gu[i]);
    const __half sg = __float2half_rn(g / (1.f + expf(-g)));
    a[i] = __float2half_rn(__half2float(sg) * __half2float(gu[I + i]));
  }
}

// x = embed[tok]
__global__ void embed_kernel(const __half* emb, const int64_t* tok, __half* x, int H) {
  pdl_launch_dependents();
  pdl_wait();
  const __half* row = emb + (size_t)*tok * H;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x) x[i] = row[i];
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace

cudaError_t launch_rmsnorm(__half* x, const __half* r, const __half* w, __half* h, int H, float eps, cudaStream_t st) {
  return launch_pdl(rmsnorm_kernel, dim3(1), dim3(kRmsThreads), 0, st, x, r, w, h, H, eps);
}

int rmsnorm_max_hidden() { return 8 * kRmsThreads * kRmsVec; }

int attn_splits(int max_len) { return (max_len + kAttnChunk - 1) / kAttnChunk; }

int attn_max_len() { return kAttnChunk * kCombineMaxSplits; }

int decode_device_error() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_decode_status, sizeof(int));
  return v;
}

void decode_clear_device_error() {
  int z = 0;
  cudaMemcpyToSymbol(g_decode_status, &z, sizeof(int));
}

size_t attn_smem_bytes(int nh, int nkv, int hd) {
  const int g = nh / nkv, ks = attn_k_stride(hd);
  return (size_t)(2 * kAttnChunk * ks + 8 * ks + 8 * 72) * sizeof(__half) +
         (size_t)(g * hd + g * kAttnChunk) * sizeof(float);
}

cudaError_t launch_attention(const __half* qkv, const __half* bias, const float* inv_freq, const int64_t* pos,
                             __half* kc, __half* vc, float* part_o, float* part_ml, __half* out, int nh, int nkv,
                             int hd, int max_len, cudaStream_t st) {
  const int nsplit = attn_splits(max_len);
  const size_t smem = attn_smem_bytes(nh, nkv, hd);
  auto kern = hd == 128 ? attn_split_kernel<128> : hd == 64 ? attn_split_kernel<64> : attn_split_kernel<0>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  e = launch_pdl(kern, dim3(nkv, nsplit), dim3(kAttnThreads), smem, st, qkv, bias, inv_freq, pos, kc, vc, part_o,
                 part_ml, nh, nkv, hd, max_len, 1.f / sqrtf((float)hd));
  if (e != cudaSuccess) return e;
  return launch_pdl(attn_combine_kernel, dim3(nh), dim3(hd), 0, st, (const float*)part_o, (const float*)part_ml, pos,
                    out, nh, nkv, hd, nsplit, max_len);
}

// Scratch of lb_decode_attention_noalloc: the split partials (part_o, then part_ml) of callers that cannot pass
// their own. Nothing in it needs to start at zero -- each call writes every partial its combine step reads.
static __device__ __align__(256) float g_attn_scratch[kNoAllocScratchFloats];

float* noalloc_attn_scratch() {
  static std::atomic<float*> addr[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  float* p = addr[dev].load(std::memory_order_acquire);
  if (!p) {
    void* sym = nullptr;
    if (cudaGetSymbolAddress(&sym, g_attn_scratch) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    p = static_cast<float*>(sym);
    addr[dev].store(p, std::memory_order_release);
  }
  return p;
}

cudaError_t launch_silu_mul(const __half* gu, __half* a, int I, cudaStream_t st) {
  return launch_pdl(silu_mul_kernel, dim3((I + 255) / 256), dim3(256), 0, st, gu, a, I);
}

cudaError_t launch_embed(const __half* emb, const int64_t* tok, __half* x, int H, cudaStream_t st) {
  return launch_pdl(embed_kernel, dim3((H + 255) / 256), dim3(256), 0, st, emb, tok, x, H);
}

}  // namespace lb
