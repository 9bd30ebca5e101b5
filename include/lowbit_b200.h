/*
 * lowbit_b200 -- C ABI of the B200 (sm_100a) W4A16 kernel library.
 *
 * Plain pointers, sizes and a CUDA stream; no framework types. Every entry point validates its arguments
 * before touching the GPU, launches asynchronously on `stream` (NULL = the legacy default stream) and never
 * synchronizes. Outputs are caller-allocated. Return value: LB_OK or an lb_status code; lb_last_error()
 * then holds a message for the calling host thread.
 *
 * Weight format (identical bytes to the reference's lowbit/quant.py): a weight W [N, K] is stored as
 * packed uint8 [N, K/2] (two 4-bit values u = q + 8 per byte, q in [-8, 7]) in one of three layouts --
 * canonical (lowbit/quant.py:23-35), v3 (lowbit/quant.py:55-64) or mma (lowbit/quant.py:67-78) -- plus
 * fp16 scales [N, K/G], one per group of G consecutive k (G a multiple of 32, K a multiple of G).
 * Activations x are fp16 [M, K] row-major, outputs fp16 [M, N] row-major.
 *
 * Each entry point replaces one binding of the reference's torch extension (csrc/w4_gemv.cu:542-550) or
 * one of its host-side helpers; the cited lines are the interface replaced.
 */
#ifndef LOWBIT_B200_H
#define LOWBIT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define LB_API __attribute__((visibility("default")))
#else
#define LB_API
#endif

/* the same handle type as cudaStream_t */
typedef struct CUstream_st* lb_stream_t;

typedef enum lb_status {
  LB_OK = 0,
  LB_ERR_ARGUMENT = 1,    /* sizes, group size, version or row count out of range (TORCH_CHECK in the reference) */
  LB_ERR_ALIGNMENT = 2,   /* a pointer is not aligned as the kernel's vector loads require */
  LB_ERR_UNSUPPORTED = 3, /* the current device is not sm_100, or the layout cannot serve this call */
  LB_ERR_CUDA = 4         /* the CUDA runtime reported an error at launch */
} lb_status;

typedef enum lb_layout { LB_LAYOUT_CANONICAL = 0, LB_LAYOUT_V3 = 1, LB_LAYOUT_MMA = 2 } lb_layout;

typedef enum lb_option {
  LB_OPT_PDL = 0,           /* 1 (default): launch with programmatic dependent launch enabled */
  LB_OPT_EARLY_WEIGHTS = 1, /* 1: GEMV kernels fetch their first weights before waiting on the previous kernel
                               in the stream (only for weights no in-flight kernel writes); default 0 */
  LB_OPT_GEMV_KSPLIT = 2,   /* 0 (default): automatic; 1..8 forces the GEMV's K-split cluster size */
  LB_OPT_GEMV_WARPS = 3,    /* 0 (default): automatic; 4, 8 or 16 forces the GEMV's warps per CTA */
  LB_OPT_GEMV_DEPTH = 4,    /* reserved: no effect (the copy-ring GEMV it tuned was removed) */
  LB_OPT_GEMV_KERNEL = 5,   /* 0 (default): automatic; 1 reserved (it forced a copy-ring GEMV, since removed),
                               2 the tcgen05 GEMM (any M <= 64), 3 the one-shot GEMV with activations staged per CTA (the
                               automatic choice at M <= 8 stages them per warp, with the same bits), 4 the
                               M <= 8 GEMV with each weight tile landed in shared memory by one bulk copy, 5 the
                               skinny GEMM on mma.sync tiles fed by tensor copies (any M <= 64; the automatic
                               choice above 16 rows) */
  LB_OPT_GEMV_ROWTILES = 6  /* 0 (default): automatic; 1 or 2 forces the one-shot GEMV's 16-row tiles per CTA, and
                               the skinny GEMM's 16-row tiles per warp */
} lb_option;

/* ABI version of this header; bumped on any signature change. */
#define LB_ABI_VERSION 1
LB_API int lb_abi_version(void);

LB_API const char* lb_status_string(int status);
/* message of the last failed call on this host thread ("" after a successful call) */
LB_API const char* lb_last_error(void);

/* Device-side status of the current device: nonzero when a kernel's bounded wait gave up (1: a pipeline barrier,
 * a kernel bug, never expected; 2: a peer rank's epoch, tensor parallelism) or a decode position read from device
 * memory lay outside the KV cache (3); that kernel's output is then undefined. Synchronizes the device. */
LB_API int lb_device_error(void);
LB_API void lb_clear_device_error(void);

/* process-wide launch options (lb_option); returns the previous value, or -1 for an unknown option */
LB_API int lb_set_option(int option, int value);
LB_API int lb_get_option(int option);

/*
 * y[M, N] = x[M, K] * dequant(W)^T for 1 <= M <= 8.
 * Replaces w4_gemv(x, w, s, group, version, rows_per_warp) (csrc/w4_gemv.cu:454-484).
 *   version 1, 2: w in the canonical layout;  3, 4: the v3 layout;  6: the mma layout (K and group % 128 == 0).
 *   rows_per_warp: 0 (auto), 1, 2 or 4; used by versions 1-4, accepted and ignored by version 6 (its warps
 *   always own 16-row tensor-core tiles).
 * x and w must be 16-byte aligned.
 */
LB_API int lb_w4_gemv(const void* x, const void* w, const void* scales, void* y, int64_t m, int64_t n, int64_t k,
               int64_t group, int version, int rows_per_warp, lb_stream_t stream);

/*
 * y[M, N] = x[M, K] * dequant(W)^T for 1 <= M <= 64 on the tensor cores, w in the mma layout
 * (K and group % 128 == 0).
 * Replaces w4_gemm_tc(x, w, s, group, row_tiles) (csrc/w4_gemv.cu:486-515).
 *   row_tiles: 0 (auto), 1, 2 or 4 -- accepted for compatibility; the kernel picks its own tiling.
 */
LB_API int lb_w4_gemm_tc(const void* x, const void* w, const void* scales, void* y, int64_t m, int64_t n, int64_t k,
                  int64_t group, int row_tiles, lb_stream_t stream);

/*
 * y[M, N] = x[M, K] * dequant(W)^T + bias, the bias added in the kernel's epilogue: each output is the product
 * rounded to fp16, plus bias[n] (fp16 [N], 2-byte aligned; NULL for none), rounded again -- the bits of the
 * reference's W4Linear.forward, which adds the bias to the kernel's fp16 output (lowbit/model.py:22-27).
 * version 1..4 or 6: the checks and kernels of lb_w4_gemv (M <= 8); version 5: those of lb_w4_gemm_tc (M <= 64).
 */
LB_API int lb_w4_linear(const void* x, const void* w, const void* scales, const void* bias, void* y, int64_t m,
                        int64_t n, int64_t k, int64_t group, int version, lb_stream_t stream);

/*
 * out[N, K] fp16 = fp16_rn((u - 8) * scale), bit-identical to the reference's dequantize kernels.
 * Replaces w4_dequant(w, s, group, mma_layout) (csrc/w4_gemv.cu:517-540); layout is an lb_layout
 * (the reference's mma_layout=False/True are LB_LAYOUT_CANONICAL / LB_LAYOUT_MMA).
 * w and out must be 16-byte aligned.
 */
LB_API int lb_w4_dequant(const void* w, const void* scales, void* out, int64_t n, int64_t k, int64_t group, int layout,
                  lb_stream_t stream);

/*
 * Quantize W [N, K] (fp32, or fp16 when w_is_half) into canonical packed [N, K/2] + fp16 scales [N, K/G].
 * With clip_grid == NULL (or n_clip == 0) the bits equal lowbit/quant.py:23-35. With a clip grid
 * (host array of n_clip <= 32 factors), each group keeps the first factor whose squared error is smallest.
 * Replaces quantize_w4_gpu(w, group, clip_grid) (lowbit/ops.py:81-116).
 */
LB_API int lb_w4_quantize(const void* w, int w_is_half, void* packed, void* scales, int64_t n, int64_t k, int64_t group,
                   const float* clip_grid, int n_clip, lb_stream_t stream);

/*
 * Reorder canonical packed bytes [N, K/2] into the v3 (layout 1) or mma (layout 2, K % 128 == 0) layout.
 * Replaces the host-side quant.interleave_for_gpu / interleave_for_mma calls of W4Weight
 * (lowbit/ops.py:43-44, lowbit/quant.py:55-78). src and dst must not overlap.
 */
LB_API int lb_w4_repack(const void* canonical, void* dst, int64_t n, int64_t k, int layout, lb_stream_t stream);

/*
 * Batch-1 decode-step kernels of the benchmark's end-to-end decoder (Qwen2 architecture) around the INT4
 * projections. No counterpart in the reference's extension: its end-to-end benchmark runs these steps as
 * transformers/torch modules (bench/e2e.py:84-147). Each reads the decode position `pos` (int64, device) at run
 * time, so a captured CUDA graph replays every step. All tensors are fp16 device arrays unless stated.
 *
 * lb_decode_embed:     x[H] = emb[*tok][:]                       (tok: int64 on the device)
 * lb_decode_rmsnorm:   if r: x = x + r; h = w * fp16(x * rsqrt(mean(x^2) + eps))   (Qwen2RMSNorm); H % 8 == 0,
 *                      all four arrays 16-byte aligned (r may be NULL); w (model state) is read before the kernel
 *                      waits on the previous kernel in the stream
 * lb_decode_attention: qkv = [q (nh x hd) | k (nkv x hd) | v (nkv x hd)] of the fused projection, + bias (may be
 *                      NULL); q and k rotated by the rotate-half RoPE at angle pos * inv_freq[j] (fp32 [hd/2]);
 *                      k, v appended to the caches [nkv, max_len, hd] at row pos; then one query token attends
 *                      to rows 0..pos (grouped heads, nh % nkv == 0, scale 1/sqrt(hd)) -> out [nh, hd].
 *                      part_o (fp32, nh * lb_decode_attention_splits(max_len) * hd) and part_ml (fp32, twice
 *                      nh * splits) are caller-owned scratch; qkv, bias, inv_freq, the caches and part_o 16-byte
 *                      aligned, part_ml 8-byte aligned; hd a multiple of
 *                      8 in 32..1024, max_len <= 65536; the cache rows below pos, bias and inv_freq are read before the
 *                      kernel waits on the previous kernel in the stream (they must not be its output); a pos outside
 *                      0..max_len-1 writes nothing and sets lb_device_error() to 3
 * lb_decode_silu_mul:  a[I] = fp16(silu(gu[i])) * gu[I + i]     (gu = [gate | up])
 */
LB_API int lb_decode_embed(const void* emb, const int64_t* tok, void* x, int64_t H, lb_stream_t stream);
LB_API int lb_decode_rmsnorm(void* x, const void* r, const void* w, void* h, int64_t H, float eps, lb_stream_t stream);
LB_API int lb_decode_attention_splits(int64_t max_len);
LB_API int lb_decode_attention(const void* qkv, const void* bias, const float* inv_freq, const int64_t* pos,
                        void* k_cache, void* v_cache, float* part_o, float* part_ml, void* out, int nh, int nkv,
                        int hd, int64_t max_len, lb_stream_t stream);
LB_API int lb_decode_silu_mul(const void* gu, void* a, int64_t I, lb_stream_t stream);

/*
 * The decode step's activation work folded into the INT4 GEMV that consumes it (M = 1, mma-layout W, K and the
 * group size multiples of 128, K <= 16384: one CTA holds the whole row; larger K -> LB_ERR_UNSUPPORTED, see
 * lb_decode_gemv_fusable). Same numerics as the separate kernels followed by lb_w4_gemv.
 * lb_decode_norm_gemv:   y[n] = W * (norm_w * fp16((x + r) * rsqrt(mean((x + r)^2) + eps))); x + r is also written
 *                        to x_out (r and x_out may be NULL; x_out must not alias x or r)
 * lb_decode_swiglu_gemv: y[n] = W * (fp16(silu(gu[0:k])) * gu[k:2k])
 * lb_decode_gemv_fusable: 1 when a [n, k] layer can take these entry points, else 0
 */
LB_API int lb_decode_gemv_fusable(int64_t n, int64_t k);

/*
 * Tensor-parallel decode: in-place-capable sum allreduce of n fp16 values over `world` ranks, one kernel per call
 * on each rank, through peer-mapped memory (NVLink). No counterpart in the reference (single GPU only).
 * bufs: device array of `world` pointers, bufs[r] = rank r's peer-mapped buffer: 256 bytes of epoch flags (zero
 * at setup) then two slots of `cap` fp16. epoch: this rank's uint32 device counter (zero at setup), advanced by
 * each call. Every rank must make the same sequence of calls. A rank waits about a second for its peers, then
 * records 2 in the device status word (lb_device_error) and gives up instead of hanging: it then writes none of its
 * outputs and does not advance its epoch, so the ranks no longer agree and the group must be set up again. A caller
 * that cannot rule out a missing peer checks lb_device_error() before using the outputs. out may alias in; n and
 * cap are multiples of 8, in and out 16-byte aligned.
 */
LB_API int lb_tp_allreduce(const void* in, void* out, int64_t n, int64_t cap, void* const* bufs, uint32_t* epoch,
                    int rank, int world, lb_stream_t stream);

/*
 * lb_tp_allreduce followed, in the same kernel, by the decode step's residual add and RMSNorm: x_res += sum of the
 * ranks' `in`; h_out = norm_w * fp16(x_res * rsqrt(mean(x_res^2) + eps)). The sum itself is not stored.
 */
LB_API int lb_tp_allreduce_norm(const void* in, int64_t n, int64_t cap, void* const* bufs, uint32_t* epoch, int rank,
                         int world, void* x_res, const void* norm_w, void* h_out, float eps, lb_stream_t stream);

/*
 * Row-parallel decode GEMV fused with the allreduce, residual add and RMSNorm of tensor-parallel decode (one kernel
 * per call on every rank): y_rank = W_rank x over this rank's K shard; x_res += sum over ranks of y_r (fp16
 * partials summed in rank order in fp32, one rounding -- the bits of lb_w4_gemv version 6 followed by
 * lb_tp_allreduce_norm); h_out = norm_w * fp16(x_res * rsqrt(mean(x_res^2) + eps)); y (may be null) receives the
 * sum. Each finished 16-row tile is stored over NVLink into every rank's buffer as it completes, as 8-byte words
 * (epoch << 32 | two fp16 outputs) that validate themselves; the last CTA polls only local memory until every
 * rank's words carry the epoch (at most ~1 s, then lb_device_error() = 2, and y, x_res and h_out are left as they
 * were, as in lb_tp_allreduce). bufs[r]: rank r's peer-mapped buffer
 * of 256 bytes of header + 2 * world * cap * 4 bytes (zeroed before first use, not shared with lb_tp_allreduce),
 * epoch: this rank's device counter (equal on every rank), counter: a device int, zero before the first call.
 */
LB_API int lb_tp_gemv_allreduce_norm(const void* x, const void* w, const void* scales, void* y, int64_t n, int64_t k,
                              int64_t group, int64_t cap, void* const* bufs, uint32_t* epoch, int rank, int world,
                              void* x_res, const void* norm_w, void* h_out, float eps, int* counter,
                              lb_stream_t stream);

/*
 * Decode GEMVs with the following step in their epilogue: M = 1, the kernel, K split and row tiling of lb_w4_gemv
 * version 6 at M = 1 (so y has its bits), K a multiple of 128:
 * lb_decode_gemv_swiglu:        W's rows interleave gate and up (row 2i = gate_i, row 2i + 1 = up_i, N % 16 == 0);
 *                               a[i] = fp16(fp16(silu(fp16(gate_i))) * fp16(up_i)), N / 2 outputs -- the bits of
 *                               lb_w4_gemv followed by lb_decode_silu_mul
 * lb_decode_gemv_residual_norm: y = W x is stored; the last CTA to finish then adds y into x_res and writes h_out =
 *                               norm_w * fp16(x_res * rsqrt(mean(x_res^2) + eps)). counter: a device int, zero before
 *                               the first call, left zero by every call; calls that can overlap need distinct ones
 */
LB_API int lb_decode_gemv_swiglu(const void* x, const void* w, const void* scales, void* a, int64_t n, int64_t k,
                          int64_t group, lb_stream_t stream);
LB_API int lb_decode_gemv_residual_norm(const void* x, const void* w, const void* scales, void* y, int64_t n, int64_t k,
                                 int64_t group, void* x_res, const void* norm_w, void* h_out, float eps, int* counter,
                                 lb_stream_t stream);
LB_API int lb_decode_norm_gemv(const void* x, const void* r, const void* norm_w, void* x_out, float eps, const void* w,
                        const void* scales, void* y, int64_t n, int64_t k, int64_t group, lb_stream_t stream);
LB_API int lb_decode_swiglu_gemv(const void* gu, const void* w, const void* scales, void* y, int64_t n, int64_t k,
                          int64_t group, lb_stream_t stream);

/*
 * lb_decode_attention without caller-owned scratch, for callers that cannot allocate device memory when they call
 * it -- a host loop in plain C, or another runtime's decode step that has no device allocator or memory pool of
 * its own to draw from -- and so cannot pass part_o / part_ml. No counterpart in the reference (its extension
 * returns torch-allocated tensors and has no scratch at all).
 *
 * Same arguments and results as lb_decode_attention minus part_o and part_ml. The partials live in a scratch
 * array inside the library: 262144 floats (1 MiB) per device. A call needs nh * lb_decode_attention_splits(max_len)
 * * (hd + 2) floats of it (Qwen2.5-3B at a 1024-token cache: 16 * 16 * 130 = 33280); larger calls fail with
 * LB_ERR_ARGUMENT and a message naming the sizes. Nothing in the scratch needs to start at zero: every partial the
 * combine step reads is written first by the same call. The scratch is one per device and shared by every call on
 * it: calls that can run at the same time (different streams, or host threads without ordering between them)
 * race on it, so the caller must serialize them. The first call on each device resolves the scratch address with
 * cudaGetSymbolAddress; make that first call outside any stream capture. The address is kept for the life of the
 * process: do not use this entry point on a device after cudaDeviceReset of that device.
 */
LB_API int lb_decode_attention_noalloc(const void* qkv, const void* bias, const float* inv_freq, const int64_t* pos,
                                void* k_cache, void* v_cache, void* out, int nh, int nkv, int hd, int64_t max_len,
                                lb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LOWBIT_B200_H */
