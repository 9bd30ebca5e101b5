// The small kernels of a batch-1 Qwen2 decode step around the INT4 projections (the decoder harness of the
// benchmark's end-to-end config; the reference drives a transformers model instead, bench/e2e.py:84-147).
//
// Every kernel reads the decode position from device memory, so one CUDA graph replays every step, and is
// launched with programmatic stream serialization: it lets its successor launch at entry and waits for its
// predecessor before touching activations. Arithmetic follows the transformers Qwen2 modules in fp32 with one
// rounding to fp16 per stored tensor.
#include <cuda_fp16.h>

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
// (Qwen2RMSNorm: the normalized value is rounded to fp16 before the weight multiply)
__global__ void __launch_bounds__(256) rmsnorm_kernel(__half* x, const __half* r, const __half* w, __half* h, int H,
                                                      float eps) {
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = __half2float(x[i]);
    if (r) {
      const __half s = __hadd(x[i], r[i]);
      x[i] = s;
      v = __half2float(s);
    }
    ss += v * v;
  }
  const float inv = rsqrtf(block_sum(ss, red) / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const __half n = __float2half_rn(__half2float(x[i]) * inv);
    h[i] = __float2half_rn(__half2float(w[i]) * __half2float(n));
  }
}

// qkv = [q (nh heads) | k (nkv) | v (nkv)] from the fused projection: add the bias, rotate q and k by the
// position's angles (rotate-half pairing: dims j and j + hd/2), write q and append k, v to the cache at pos.
// Grid: nh + 2 * nkv heads; block: hd / 2 threads.
__global__ void qkv_rope_kernel(const __half* qkv, const __half* bias, const float* inv_freq, const int64_t* pos_p,
                                __half* q_out, __half* kc, __half* vc, int nh, int nkv, int hd, int max_len) {
  pdl_launch_dependents();
  pdl_wait();
  const int head = blockIdx.x, j = threadIdx.x, half = hd / 2;
  const int pos = (int)*pos_p;
  const __half* src = qkv + (size_t)head * hd;
  const __half* bsrc = bias ? bias + (size_t)head * hd : nullptr;
  __half a = src[j], b = src[j + half];
  if (bsrc) {
    a = __hadd(a, bsrc[j]);
    b = __hadd(b, bsrc[j + half]);
  }
  if (head >= nh + nkv) {   // v: straight into the cache
    __half* dst = vc + ((size_t)(head - nh - nkv) * max_len + pos) * hd;
    dst[j] = a;
    dst[j + half] = b;
    return;
  }
  float s, c;
  sincosf((float)pos * inv_freq[j], &s, &c);
  const float fa = __half2float(a), fb = __half2float(b);
  const __half ra = __float2half_rn(fa * c - fb * s), rb = __float2half_rn(fb * c + fa * s);
  __half* dst = head < nh ? q_out + (size_t)head * hd : kc + ((size_t)(head - nh) * max_len + pos) * hd;
  dst[j] = ra;
  dst[j + half] = rb;
}

// Split attention for one query token: CTA (kv head, split) scores positions [64 s, 64 s + 64) of the cache
// (those <= pos) for the group's query heads, and writes the split's running max, sum of exponentials and
// unnormalized output (fp32) for attn_combine_kernel.
constexpr int kAttnChunk = 64;
constexpr int kAttnThreads = 256;

__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(const __half* q, const __half* kc, const __half* vc,
                                                                  const int64_t* pos_p, float* part_o, float* part_ml,
                                                                  int nh, int nkv, int hd, int max_len, float scale) {
  extern __shared__ float sm[];   // q [g][hd] fp32, scores [g][chunk]
  pdl_launch_dependents();
  pdl_wait();
  const int kvh = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y;
  const int g = nh / nkv, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = kAttnThreads / 32;
  const int L = (int)*pos_p + 1;
  const int p0 = split * kAttnChunk, np = min(kAttnChunk, L - p0);
  float* sq = sm;
  float* ss = sm + g * hd;
  const size_t pbase = ((size_t)kvh * nsplit + split) * g;
  if (np <= 0) {   // nothing cached here yet: an empty partial
    for (int i = threadIdx.x; i < g; i += blockDim.x) {
      part_ml[(pbase + i) * 2] = -INFINITY;
      part_ml[(pbase + i) * 2 + 1] = 0.f;
    }
    return;
  }
  for (int i = threadIdx.x; i < g * hd; i += blockDim.x) sq[i] = __half2float(q[(size_t)kvh * g * hd + i]) * scale;
  __syncthreads();
  const __half* kb = kc + ((size_t)kvh * max_len + p0) * hd;
  const __half* vb = vc + ((size_t)kvh * max_len + p0) * hd;
  // scores: warp per position, lanes over the head dimension
  for (int p = warp; p < np; p += nw) {
    const __half* kr = kb + (size_t)p * hd;
    for (int h = 0; h < g; ++h) {
      float d = 0.f;
      for (int e = lane; e < hd; e += 32) d += sq[h * hd + e] * __half2float(kr[e]);
      d = warp_sum(d);
      if (lane == 0) ss[h * kAttnChunk + p] = d;
    }
  }
  __syncthreads();
  // per head: max and exponentials (warp h handles head h, h + nw, ...)
  for (int h = warp; h < g; h += nw) {
    float m = -INFINITY;
    for (int p = lane; p < np; p += 32) m = fmaxf(m, ss[h * kAttnChunk + p]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int p = lane; p < np; p += 32) {
      const float e = expf(ss[h * kAttnChunk + p] - m);
      ss[h * kAttnChunk + p] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      part_ml[(pbase + h) * 2] = m;
      part_ml[(pbase + h) * 2 + 1] = l;
    }
  }
  __syncthreads();
  // unnormalized outputs: thread (h, e) sums over the split's positions
  for (int i = threadIdx.x; i < g * hd; i += blockDim.x) {
    const int h = i / hd, e = i - h * hd;
    float acc = 0.f;
    for (int p = 0; p < np; ++p) acc += ss[h * kAttnChunk + p] * __half2float(vb[(size_t)p * hd + e]);
    part_o[(pbase + h) * hd + e] = acc;
  }
}

// out[head] = sum_s exp(m_s - M) o_s / sum_s exp(m_s - M) l_s; grid nh, block hd
__global__ void attn_combine_kernel(const float* part_o, const float* part_ml, __half* out, int nh, int nkv, int hd,
                                    int nsplit) {
  pdl_launch_dependents();
  pdl_wait();
  const int head = blockIdx.x, e = threadIdx.x, g = nh / nkv, kvh = head / g, h = head - kvh * g;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part_ml[(((size_t)kvh * nsplit + s) * g + h) * 2]);
  float num = 0.f, den = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const size_t b = ((size_t)kvh * nsplit + s) * g + h;
    const float m = part_ml[b * 2];
    if (m == -INFINITY) continue;
    const float w = expf(m - M);
    den += w * part_ml[b * 2 + 1];
    num += w * part_o[b * hd + e];
  }
  out[(size_t)head * hd + e] = __float2half_rn(num / den);
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
  return launch_pdl(rmsnorm_kernel, dim3(1), dim3(256), 0, st, x, r, w, h, H, eps);
}

cudaError_t launch_qkv_rope(const __half* qkv, const __half* bias, const float* inv_freq, const int64_t* pos,
                            __half* q, __half* kc, __half* vc, int nh, int nkv, int hd, int max_len, cudaStream_t st) {
  return launch_pdl(qkv_rope_kernel, dim3(nh + 2 * nkv), dim3(hd / 2), 0, st, qkv, bias, inv_freq, pos, q, kc, vc, nh,
                    nkv, hd, max_len);
}

int attn_splits(int max_len) { return (max_len + kAttnChunk - 1) / kAttnChunk; }

cudaError_t launch_attention(const __half* q, const __half* kc, const __half* vc, const int64_t* pos, float* part_o,
                             float* part_ml, __half* out, int nh, int nkv, int hd, int max_len, cudaStream_t st) {
  const int nsplit = attn_splits(max_len), g = nh / nkv;
  const size_t smem = (size_t)(g * hd + g * kAttnChunk) * sizeof(float);
  cudaError_t e = launch_pdl(attn_split_kernel, dim3(nkv, nsplit), dim3(kAttnThreads), smem, st, q, kc, vc, pos, part_o,
                             part_ml, nh, nkv, hd, max_len, 1.f / sqrtf((float)hd));
  if (e != cudaSuccess) return e;
  return launch_pdl(attn_combine_kernel, dim3(nh), dim3(hd), 0, st, (const float*)part_o, (const float*)part_ml, out, nh,
                    nkv, hd, nsplit);
}

cudaError_t launch_silu_mul(const __half* gu, __half* a, int I, cudaStream_t st) {
  return launch_pdl(silu_mul_kernel, dim3((I + 255) / 256), dim3(256), 0, st, gu, a, I);
}

cudaError_t launch_embed(const __half* emb, const int64_t* tok, __half* x, int H, cudaStream_t st) {
  return launch_pdl(embed_kernel, dim3((H + 255) / 256), dim3(256), 0, st, emb, tok, x, H);
}

}  // namespace lb
