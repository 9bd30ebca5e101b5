// Host-side launch descriptors shared by the C-ABI layer and the kernel files.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace lb {

enum : int {
  kFlagEarlyWeights = 1,  // issue the first weight loads before waiting on the predecessor kernel
};

struct GemvParams {
  const void* x;  // fp16 [M, K]
  const void* w;  // packed uint8 [N, K / 2]
  const void* s;  // fp16 [N, K / G]
  __half* y;      // fp16 [M, N]
  int M, N, K, G;
  int flags;
  int wait_guard;  // always 1 (see pdl_wait_after_loads)
  int KG;          // K / G, groups per row
  int cpg;         // G / 128, 128-wide chunks per group (mma layout kernels)
  const __half* bias = nullptr;   // fp16 [N] added to every output row (plain GEMV / GEMM only), or null
  // activation prologue of the one-shot GEMV (M = 1, K unsplit): 0 none; 1 x <- w * fp16((x + r) *
  // rsqrt(mean((x + r)^2) + eps)) with x + r written to out by CTA 0 (r, out may be null); 2 x <- silu(x[0:K]) *
  // x[K:2K] (x is a [gate | up] row of 2K values)
  int pro = 0;
  const __half* pro_r = nullptr;
  const __half* pro_w = nullptr;
  __half* pro_out = nullptr;
  float pro_eps = 0.f;
  // output epilogue of the one-shot GEMV (M = 1, K unsplit, one row tile): 0 none; 1 SwiGLU over interleaved rows
  // (W rows 2i, 2i + 1 = gate_i, up_i): y[i] = fp16(fp16(silu(fp16(gate_i))) * fp16(up_i)), N / 2 outputs; 2 y is
  // stored, then the last CTA to finish (epi_counter, zero between calls) adds y into the residual stream epi_x
  // and writes epi_h = epi_w * fp16(x * rsqrt(mean(x^2) + eps)) for the next projection
  // 3 (row-parallel, tensor parallelism): each finished tile's fp16 partial is stored into region (e & 1, ar_rank)
  // of every rank's peer-mapped buffer (kPeerFlagBytes of header, then 2 x ar_world regions of ar_cap / 2 words
  // e << 32 | two fp16, region (parity, source rank)), e = *ar_epoch + 1; the last CTA polls its own buffer's
  // words until each carries e, sums the ranks in rank order (y, if not null, receives the sum), then continues
  // as 2
  int epi = 0;
  int* epi_counter = nullptr;
  __half* epi_x = nullptr;
  const __half* epi_w = nullptr;
  __half* epi_h = nullptr;
  float epi_eps = 0.f;
  uint8_t* const* ar_bufs = nullptr;
  uint32_t* ar_epoch = nullptr;
  int ar_rank = 0, ar_world = 1, ar_cap = 0;
};

// one-shot GEMV (M <= 16): one 16-row tile per CTA, all weight loads issued at entry
struct OneshotConfig {
  int warps;   // warps per CTA (1..16)
  int cpw;     // most chunks per warp: 2, 4 or 8 (8 only with one row tile)
  int ksplit;  // CTAs per cluster splitting K (1..8)
  int rt;      // 16-row tiles per CTA: 1 or 2
  int pdl;
};
cudaError_t launch_gemv_oneshot(const GemvParams& p, const OneshotConfig& c, cudaStream_t st);  // p.pro / p.epi: M = 1, ksplit 1, rt 1
size_t oneshot_smem_bytes(int M, int K, int nsplit, int nw, int rt);
// the plain M <= 8 GEMV at an unsplit, one-row-tile one-shot configuration: activations staged per warp, the
// one-shot kernel's bits (lb_gemv.cu gemv_tile_kernel)
cudaError_t launch_gemv_tile(const GemvParams& p, const OneshotConfig& c, cudaStream_t st);
size_t tile_smem_bytes(int M, int nw, int cpw);
// the same with the tile's weights landed in shared memory by one bulk copy (lb_gemv.cu gemv_bulk_kernel)
cudaError_t launch_gemv_bulk(const GemvParams& p, const OneshotConfig& c, cudaStream_t st);
size_t bulk_smem_bytes(int M, int K, int nw, int cpw);

// device status word (lb_gemv.cu): nonzero after a bounded wait in a kernel gave up
int device_error();   // synchronizes
void clear_device_error();
cudaError_t launch_gemv_compat(const GemvParams& p, int rows_per_warp, bool v3, bool pdl, cudaStream_t st);

// format kernels (lb_format.cu)
cudaError_t launch_dequant(const void* w, const void* s, __half* out, int N, int K, int G, int layout,
                           cudaStream_t st);
cudaError_t launch_quantize(const void* w, int w_is_half, uint8_t* packed, __half* scales, int N, int K, int G,
                            const float* clip, int n_clip, cudaStream_t st);
cudaError_t launch_repack(const uint8_t* canonical, uint8_t* out, int N, int K, int layout, cudaStream_t st);

// decode-step kernels (lb_decode.cu)
cudaError_t launch_embed(const __half* emb, const int64_t* tok, __half* x, int H, cudaStream_t st);
cudaError_t launch_rmsnorm(__half* x, const __half* r, const __half* w, __half* h, int H, float eps, cudaStream_t st);
int rmsnorm_max_hidden();
int attn_splits(int max_len);
int attn_max_len();   // longest cache the split attention and its combine step take
int decode_device_error();
void decode_clear_device_error();
size_t attn_smem_bytes(int nh, int nkv, int hd);
cudaError_t launch_attention(const __half* qkv, const __half* bias, const float* inv_freq, const int64_t* pos,
                             __half* kc, __half* vc, float* part_o, float* part_ml, __half* out, int nh, int nkv,
                             int hd, int max_len, cudaStream_t st);
cudaError_t launch_silu_mul(const __half* gu, __half* a, int I, cudaStream_t st);
// one-shot allreduce over peer memory (lb_allreduce.cu)
cudaError_t launch_allreduce_oneshot(const __half* in, __half* out, int n, int cap, uint8_t* const* bufs,
                                     uint32_t* epoch, int rank, int world, cudaStream_t st, __half* x_res = nullptr,
                                     const __half* norm_w = nullptr, __half* h_out = nullptr, float eps = 0.f);
int allreduce_device_error();   // synchronizes
void allreduce_clear_device_error();
// lb_decode_attention_noalloc: library-held scratch for the split partials (1 MiB per device)
constexpr size_t kNoAllocScratchFloats = 262144;
float* noalloc_attn_scratch();   // this device's scratch address (cudaGetSymbolAddress on first use), or null

// 2-D tiled tensor map (no interleave, L2 256-byte promotion, out-of-bound elements read as zero); false on failure
bool encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);

// tcgen05 skinny GEMM (lb_gemm_tc.cu), M <= 64: per 128-row tile a cluster of `splits` CTAs splitting K.
// gemm_tc05_splits picks the split for a shape on the current device (forced > 0: that split, capped by the
// cluster limit and the number of K chunks), 0 if the shape does not fit the kernel.
int gemm_tc05_splits(int M, int N, int K, int G, int forced);
cudaError_t launch_gemm_tc05(const GemvParams& p, int splits, bool pdl, cudaStream_t st);
int gemm_tc_device_error();   // synchronizes
void gemm_tc_clear_device_error();

// skinny GEMM on mma.sync tiles fed by tensor copies (lb_gemm_mma.cu), M <= 64 (exact per-group products up to 16
// rows, fp16-rounded weights above): CTAs of 64 rt weight rows, `splits` of them per cluster splitting K.
// gemm_mma_config picks both for a shape on the current device (forced > 0: that split / row-tile count), splits 0
// if the shape does not fit the kernel.
struct MmaConfig {
  int splits;
  int rt;
};
MmaConfig gemm_mma_config(int M, int N, int K, int G, int forced_splits, int forced_rt);
cudaError_t launch_gemm_mma(const GemvParams& p, const MmaConfig& c, bool pdl, cudaStream_t st);
int gemm_mma_device_error();   // synchronizes
void gemm_mma_clear_device_error();

}  // namespace lb
