// One-shot sum allreduce of a small fp16 vector over NVLink peer memory, one kernel per call on every rank -- the
// row-parallel step of tensor-parallel decode (after the o and down projections), in place of a library
// collective whose per-call latency dominates at batch 1.
//
// Each rank owns a peer-mapped buffer: a flag array of `world` epochs followed by two data slots of `cap` fp16.
// A call with epoch e (a device counter the kernel advances, so graph replays stay aligned across ranks):
//   1. copies this rank's partial into slot e & 1 of its own buffer;
//   2. publishes e into flags[rank] of every rank's buffer (release, system scope);
//   3. polls its own flags until every rank has published e (acquire, system scope), for at most ~1 s of SM
//      clock, after which it records kErrPeerTimeout in the status word and gives up instead of hanging;
//   4. reads every rank's slot e & 1 over NVLink and sums them in rank order (fp32, one rounding), so every rank
//      obtains the same bits.
// A slot is written again two epochs later, and only after this rank has seen every peer publish the epoch in
// between -- which each peer does only after its previous call, the last reader of that slot, has completed.
#include <atomic>

#include "lb_common.cuh"
#include "lb_launch.h"

namespace lb {

__device__ int g_ar_status;

namespace {

constexpr int kArThreads = 512;

__device__ __forceinline__ uint4 ld_u4_volatile(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// n % 8 == 0: every thread moves whole 16-byte pieces; the peers' pieces of a round are all requested before any
// is added, so a call pays about one NVLink round trip
// with x_res: the sum is also added into the residual stream x_res and the new row is normalized, h = norm_w *
// fp16(x * rsqrt(mean(x^2) + eps)) -- the decode step's residual add + RMSNorm after a row-parallel projection
__global__ void __launch_bounds__(kArThreads) allreduce_oneshot_kernel(const __half* in, __half* out, int n, int cap,
                                                                      uint8_t* const* bufs, uint32_t* epoch_p,
                                                                      int rank, int world, __half* x_res,
                                                                      const __half* norm_w, __half* h_out,
                                                                      float eps) {
  constexpr int kRanksPerRound = 8;
  __shared__ int timed_out;
  __shared__ const uint8_t* src[64];
  pdl_launch_dependents();
  pdl_wait();   // `in` comes from the previous kernel in the stream
  const uint32_t e = *epoch_p + 1;
  const int slot = e & 1, n8 = n / 8;
  const size_t flag_bytes = kPeerFlagBytes, slot_bytes = (size_t)cap * 2;
  uint8_t* mine = bufs[rank];
  uint4* my_slot = reinterpret_cast<uint4*>(mine + flag_bytes + slot * slot_bytes);
  for (int v = threadIdx.x; v < n8; v += blockDim.x) {   // L2-cached load: `in` was just written by another kernel
    uint4 x;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(x.x), "=r"(x.y), "=r"(x.z), "=r"(x.w)
                 : "l"(reinterpret_cast<const uint4*>(in) + v));
    my_slot[v] = x;
  }
  if (threadIdx.x == 0) timed_out = 0;
  if (threadIdx.x < world) src[threadIdx.x] = bufs[threadIdx.x] + flag_bytes + slot * slot_bytes;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < world; ++r) st_release_sys(reinterpret_cast<uint32_t*>(bufs[r]) + rank, e);
  }
  // wait for every rank's epoch (thread r polls rank r's flag in this rank's buffer)
  if (threadIdx.x < world &&
      !wait_peer_epoch(reinterpret_cast<const uint32_t*>(mine) + threadIdx.x, e, &g_ar_status))
    timed_out = 1;
  __syncthreads();
  // a peer that never published: write nothing (out, x_res and h_out keep their values, the epoch does not advance)
  // and leave the status word at 2 for the host
  if (timed_out) return;
  float ss_part = 0.f;
  for (int v = threadIdx.x; v < n8; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r0 = 0; r0 < world; r0 += kRanksPerRound) {
      uint4 q[kRanksPerRound];
#pragma unroll
      for (int j = 0; j < kRanksPerRound; ++j)
        if (r0 + j < world) q[j] = ld_u4_volatile(src[r0 + j] + (size_t)v * 16);
#pragma unroll
      for (int j = 0; j < kRanksPerRound; ++j) {
        if (r0 + j < world) {   // rank order
          const __half2* h = reinterpret_cast<const __half2*>(&q[j]);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = __half22float2(h[k]);
            acc[2 * k] += f.x;
            acc[2 * k + 1] += f.y;
          }
        }
      }
    }
    uint4 o;
    __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) oh[k] = __floats2half2_rn(acc[2 * k], acc[2 * k + 1]);
    if (out) reinterpret_cast<uint4*>(out)[v] = o;
    if (x_res) {
      uint4 xv = reinterpret_cast<const uint4*>(x_res)[v];
      __half2* xh = reinterpret_cast<__half2*>(&xv);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        xh[k] = __hadd2(xh[k], oh[k]);
        const float2 f = __half22float2(xh[k]);
        ss_part += f.x * f.x + f.y * f.y;
      }
      reinterpret_cast<uint4*>(x_res)[v] = xv;
    }
  }
  if (x_res) {
    __shared__ float red[32];
    float v = warp_sum(ss_part);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = (threadIdx.x & 31) < (int)(blockDim.x >> 5) ? red[threadIdx.x & 31] : 0.f;
    const float inv = rsqrtf(warp_sum(t) / (float)n + eps);
    for (int i = threadIdx.x; i < n8; i += blockDim.x) {   // the same pieces this thread wrote above
      const uint4 xv = reinterpret_cast<const uint4*>(x_res)[i];
      const uint4 wv = reinterpret_cast<const uint4*>(norm_w)[i];
      const __half2* xh = reinterpret_cast<const __half2*>(&xv);
      const __half2* wh = reinterpret_cast<const __half2*>(&wv);
      uint4 hv;
      __half2* hh = reinterpret_cast<__half2*>(&hv);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(xh[k]);
        hh[k] = __hmul2(wh[k], __floats2half2_rn(f.x * inv, f.y * inv));
      }
      reinterpret_cast<uint4*>(h_out)[i] = hv;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && !timed_out) *epoch_p = e;
}

}  // namespace

cudaError_t launch_allreduce_oneshot(const __half* in, __half* out, int n, int cap, uint8_t* const* bufs,
                                     uint32_t* epoch, int rank, int world, cudaStream_t st, __half* x_res,
                                     const __half* norm_w, __half* h_out, float eps) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kArThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, allreduce_oneshot_kernel, in, out, n, cap, bufs, epoch, rank, world, x_res, norm_w,
                            h_out, eps);
}

int allreduce_device_error() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_ar_status, sizeof(int));
  return v;
}

void allreduce_clear_device_error() {
  int z = 0;
  cudaMemcpyToSymbol(g_ar_status, &z, sizeof(int));
}

}  // namespace lb
