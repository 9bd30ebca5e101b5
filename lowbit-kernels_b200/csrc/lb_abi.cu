// The C ABI (include/lowbit_b200.h): argument validation with the reference's error contract
// (csrc/w4_gemv.cu:312-325 and the per-op checks at :454-540), tiling heuristics, kernel launches.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "../../include/lowbit_b200.h"
#include "lb_launch.h"

namespace {

thread_local char g_err[512];

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = 0;
  return LB_OK;
}

constexpr int kNumOptions = 7;
std::atomic<int> g_opt[kNumOptions] = {{1}, {0}, {0}, {0}, {0}, {0}, {0}};

int g_sm_count = 0;  // SMs of the current device (set by check_device)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned2(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 1u) == 0; }

// The library carries sm_100a code only: refuse other devices with a clear message instead of a launch error.
int check_device() {
  static thread_local int cached_dev = -1, cached_ok = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(LB_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev == cached_dev && cached_ok) return LB_OK;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return fail(LB_ERR_UNSUPPORTED, "lowbit_b200 is built for sm_100a (B200); device %d is sm_%d%d", dev, major, minor);
  cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
  cached_dev = dev;
  cached_ok = 1;
  return LB_OK;
}

int launched(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(LB_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return ok();
}

// csrc/w4_gemv.cu:312-325 for raw pointers: shapes, group size, 16-byte alignment of x and w
int check_common(const void* x, const void* w, const void* s, const void* y, int64_t m, int64_t n, int64_t k,
                 int64_t group) {
  if (!x || !w || !s || !y) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  if (group <= 0) return fail(LB_ERR_ARGUMENT, "group size must be positive");
  if (n <= 0 || k <= 0 || m < 0) return fail(LB_ERR_ARGUMENT, "shape mismatch: M=%lld N=%lld K=%lld",
                                             (long long)m, (long long)n, (long long)k);
  if (group % 32 || k % group)
    return fail(LB_ERR_ARGUMENT, "K must be a multiple of the group size, itself a multiple of 32");
  if (n > (1 << 30) || k > (1 << 28)) return fail(LB_ERR_ARGUMENT, "N or K too large");
  if (!aligned16(x) || !aligned16(w)) return fail(LB_ERR_ALIGNMENT, "x and w must be 16-byte aligned for the 128-bit loads");
  if (!aligned2(s) || !aligned2(y)) return fail(LB_ERR_ALIGNMENT, "scales and y must be 2-byte aligned");
  return LB_OK;
}

// One-shot GEMV tiling, from a B200 sweep of the Qwen2.5 projections at M = 1 (every K-split 1..8, row tiles
// 1..2, warps 2..16): splitting K across a cluster never paid (its two cluster barriers cost more than the
// extra parallelism), one 16-row tile per CTA was best or within noise, and the post-wait critical path is
// shortest with many warps per CTA -- 16 on layers up to 4096 rows, 8 on wider ones, never more than the
// number of 128-wide chunks. A K split remains only where the staged activations would not fit otherwise.
lb::OneshotConfig oneshot_config(int M, int N, int K) {
  lb::OneshotConfig c{0, 0, 0, 0, g_opt[LB_OPT_PDL].load()};
  const int kc = K >> 7;
  int rt = 1;
  const int forced_rt = g_opt[LB_OPT_GEMV_ROWTILES].load();
  if (forced_rt == 1 || forced_rt == 2) rt = forced_rt;
  int s = 1;
  const int forced = g_opt[LB_OPT_GEMV_KSPLIT].load();
  if (forced >= 1 && forced <= 8 && forced <= kc) s = forced;
  int nl = (kc + s - 1) / s;
  int nw = N >= 4096 ? 8 : 16;
  const int fw = g_opt[LB_OPT_GEMV_WARPS].load();
  if (fw >= 1 && fw <= 16) nw = fw;
  if (nw > nl) nw = nl;
  // grow the split until every warp's share fits the register budget and the activations fit
  while (!forced && s < 8 && s < kc &&
         ((nl + nw - 1) / nw > (rt == 1 ? 8 : 4) || lb::oneshot_smem_bytes(M, K, s, nw, rt) > 200 * 1024)) {
    ++s;
    nl = (kc + s - 1) / s;
    if (nw > nl) nw = nl;
  }
  const int per = (nl + nw - 1) / nw;
  const int cpw = per <= 2 ? 2 : per <= 4 ? 4 : (per <= 8 && rt == 1) ? 8 : 0;
  if (cpw == 0) return c;
  if (lb::oneshot_smem_bytes(M, K, s, nw, rt) > 200 * 1024) return c;
  c.warps = nw;
  c.cpw = cpw;
  c.ksplit = s;
  c.rt = rt;
  return c;
}

// One-shot configuration for M = 1 with the whole K range in one CTA (the decode prologues need the full row):
// warps as the sweep chose them, up to 16 when the row is long; invalid (warps = 0) beyond 16 warps x 8 chunks.
lb::OneshotConfig unsplit_config(int N, int K) {
  lb::OneshotConfig c{0, 0, 0, 0, g_opt[LB_OPT_PDL].load()};
  const int kc = K >> 7;
  int nw = N >= 4096 ? 8 : 16;
  const int fw = g_opt[LB_OPT_GEMV_WARPS].load();
  if (fw >= 1 && fw <= 16) nw = fw;
  if ((kc + nw - 1) / nw > 8) nw = 16;
  if (nw > kc) nw = kc;
  const int per = (kc + nw - 1) / nw;
  const int cpw = per <= 2 ? 2 : per <= 4 ? 4 : per <= 8 ? 8 : 0;
  if (cpw == 0 || lb::oneshot_smem_bytes(1, K, 1, nw, 1) > 200 * 1024) return c;
  c.warps = nw;
  c.cpw = cpw;
  c.ksplit = 1;
  c.rt = 1;
  return c;
}

int run_gemv_mma(const void* x, const void* w, const void* s, void* y, int64_t m, int64_t n, int64_t k,
                 int64_t group, cudaStream_t st, const void* bias = nullptr) {
  lb::GemvParams p{x, w, s, reinterpret_cast<__half*>(y), (int)m, (int)n, (int)k, (int)group,
                   g_opt[LB_OPT_EARLY_WEIGHTS].load() ? (int)lb::kFlagEarlyWeights : 0, 1, (int)(k / group),
                   (int)(group / 128)};
  p.bias = static_cast<const __half*>(bias);
  const int kernel = g_opt[LB_OPT_GEMV_KERNEL].load();
  // The skinny mma.sync GEMM from 17 rows; from 9 rows on layers of 8M+ weights or K < 512, and from 13 rows on
  // layers of 2048+ rows (there, measured on B200, 1.1-2.4x faster than the one-shot GEMV's 16-row CTAs, which
  // each re-read every activation row); the
  // tcgen05 GEMM above 48 rows on layers of more than 4.2M weights, where it measured up to 12 % faster (the
  // tensor-core pipe, not the weight stream, bounds the mma.sync kernel there).
  const bool tc_rows = m > 48 && n * k > 4200000;
  if (kernel == 2 || (kernel == 0 && tc_rows)) {
    // tcgen05: per 128-row tile a cluster of CTAs splitting K, tensor-memory accumulators
    const int splits = lb::gemm_tc05_splits((int)m, (int)n, (int)k, (int)group, g_opt[LB_OPT_GEMV_KSPLIT].load());
    if (splits > 0)
      return launched(lb::launch_gemm_tc05(p, splits, g_opt[LB_OPT_PDL].load() != 0, st), "w4_gemm_tc");
  }
  if (kernel == 5 ||
      (kernel == 0 && (m > 16 || (m > 8 && (n * k >= (int64_t)1 << 23 || k < 512 || (m > 12 && n >= 2048)))))) {
    // mma.sync tiles fed by tensor copies: CTAs of 64 weight rows sharing each activation chunk, clusters splitting K
    const lb::MmaConfig c = lb::gemm_mma_config((int)m, (int)n, (int)k, (int)group,
                                                g_opt[LB_OPT_GEMV_KSPLIT].load(), g_opt[LB_OPT_GEMV_ROWTILES].load());
    if (c.splits > 0) return launched(lb::launch_gemm_mma(p, c, g_opt[LB_OPT_PDL].load() != 0, st), "w4_gemm");
  }
  if (m <= 16) {
    const lb::OneshotConfig c = oneshot_config((int)m, (int)n, (int)k);
    if (c.warps > 0) {
      // the same tiling through the kernel that stages activations per warp (same bits) where it applies and, from
      // an interleaved B200 comparison over the config-1 shapes, is faster: always at M = 1 (1.0-1.3x), on layers of
      // 4096+ rows at M = 2..8 (up to 1.3x; narrower layers keep the CTA-wide asynchronous staging)
      if (kernel == 4 && m <= 8 && c.ksplit == 1 && c.rt == 1 &&
          lb::bulk_smem_bytes((int)m, (int)k, c.warps, c.cpw) <= 200 * 1024)
        return launched(lb::launch_gemv_bulk(p, c, st), "w4_gemv");
      if (kernel != 3 && m <= 8 && (m == 1 || n >= 4096) && c.ksplit == 1 && c.rt == 1 &&
          lb::tile_smem_bytes((int)m, c.warps, c.cpw) <= 200 * 1024)
        return launched(lb::launch_gemv_tile(p, c, st), "w4_gemv");
      return launched(lb::launch_gemv_oneshot(p, c, st), "w4_gemv");
    }
  }
  // what the kernels above do not take (the one-shot GEMV's staged activations would not fit shared memory at this
  // K, or kernel 3 / 4 forced past 8 rows): the skinny GEMM, whose shared memory does not grow with K
  const lb::MmaConfig c = lb::gemm_mma_config((int)m, (int)n, (int)k, (int)group, g_opt[LB_OPT_GEMV_KSPLIT].load(),
                                              g_opt[LB_OPT_GEMV_ROWTILES].load());
  if (c.splits == 0) return fail(LB_ERR_ARGUMENT, "no GEMV kernel takes M=%lld K=%lld", (long long)m, (long long)k);
  return launched(lb::launch_gemm_mma(p, c, g_opt[LB_OPT_PDL].load() != 0, st), "w4_gemm");
}

}  // namespace

extern "C" {

int lb_abi_version(void) { return LB_ABI_VERSION; }

const char* lb_status_string(int status) {
  switch (status) {
    case LB_OK: return "ok";
    case LB_ERR_ARGUMENT: return "invalid argument";
    case LB_ERR_ALIGNMENT: return "misaligned pointer";
    case LB_ERR_UNSUPPORTED: return "unsupported device or layout";
    case LB_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

const char* lb_last_error(void) { return g_err; }

int lb_device_error(void) {
  int a = lb::device_error();
  if (!a) a = lb::gemm_tc_device_error();
  if (!a) a = lb::gemm_mma_device_error();
  if (!a) a = lb::allreduce_device_error();
  return a ? a : lb::decode_device_error();
}

void lb_clear_device_error(void) {
  lb::clear_device_error();
  lb::gemm_tc_clear_device_error();
  lb::gemm_mma_clear_device_error();
  lb::allreduce_clear_device_error();
  lb::decode_clear_device_error();
}

int lb_set_option(int option, int value) {
  if (option < 0 || option >= kNumOptions) return -1;
  return g_opt[option].exchange(value);
}

int lb_get_option(int option) {
  if (option < 0 || option >= kNumOptions) return -1;
  return g_opt[option].load();
}

}  // extern "C"

// lb_w4_gemv's checks and dispatch (csrc/w4_gemv.cu:454-484), with an optional bias for lb_w4_linear
static int w4_gemv_impl(const void* x, const void* w, const void* scales, const void* bias, void* y, int64_t m,
                        int64_t n, int64_t k, int64_t group, int version, int rows_per_warp, lb_stream_t stream) {
  int rc = check_common(x, w, scales, y, m, n, k, group);
  if (rc) return rc;
  if (m < 1 || m > 8)
    return fail(LB_ERR_ARGUMENT, "the GEMV kernels take 1..8 rows; use the dequantize + matmul path above that");
  if (!((version >= 1 && version <= 4) || version == 6)) return fail(LB_ERR_ARGUMENT, "version is 1..4 or 6");
  if (version == 6 && (k % 128 || group % 128))
    return fail(LB_ERR_ARGUMENT, "v6 needs K and the group size to be multiples of 128");
  if (!(rows_per_warp == 0 || rows_per_warp == 1 || rows_per_warp == 2 || rows_per_warp == 4))
    return fail(LB_ERR_ARGUMENT, "rows_per_warp is 0 (auto), 1, 2 or 4");
  if (!aligned2(bias)) return fail(LB_ERR_ALIGNMENT, "bias must be 2-byte aligned");
  if ((rc = check_device())) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (version == 6) return run_gemv_mma(x, w, scales, y, m, n, k, group, st, bias);
  lb::GemvParams p{x, w, scales, reinterpret_cast<__half*>(y), (int)m, (int)n, (int)k, (int)group, 0, 1,
                   (int)(k / group), (int)(group / 128)};
  p.bias = static_cast<const __half*>(bias);
  int R = rows_per_warp ? rows_per_warp : (n >= 512 ? 4 : (m >= 4 ? 2 : 1));
  return launched(lb::launch_gemv_compat(p, R, version >= 3, g_opt[LB_OPT_PDL].load() != 0, st), "w4_gemv");
}

// lb_w4_gemm_tc's checks and dispatch (csrc/w4_gemv.cu:486-515), with an optional bias for lb_w4_linear
static int w4_gemm_impl(const void* x, const void* w, const void* scales, const void* bias, void* y, int64_t m,
                        int64_t n, int64_t k, int64_t group, int row_tiles, lb_stream_t stream) {
  int rc = check_common(x, w, scales, y, m, n, k, group);
  if (rc) return rc;
  if (m < 1 || m > 64) return fail(LB_ERR_ARGUMENT, "the tensor-core kernel takes 1..64 rows");
  if (k % 128 || group % 128) return fail(LB_ERR_ARGUMENT, "v5 needs K and the group size to be multiples of 128");
  if (!(row_tiles == 0 || row_tiles == 1 || row_tiles == 2 || row_tiles == 4))
    return fail(LB_ERR_ARGUMENT, "row_tiles must be 1, 2 or 4");
  if (!aligned2(bias)) return fail(LB_ERR_ALIGNMENT, "bias must be 2-byte aligned");
  if ((rc = check_device())) return rc;
  return run_gemv_mma(x, w, scales, y, m, n, k, group, reinterpret_cast<cudaStream_t>(stream), bias);
}

extern "C" {

int lb_w4_gemv(const void* x, const void* w, const void* scales, void* y, int64_t m, int64_t n, int64_t k,
               int64_t group, int version, int rows_per_warp, lb_stream_t stream) {
  return w4_gemv_impl(x, w, scales, nullptr, y, m, n, k, group, version, rows_per_warp, stream);
}

int lb_w4_gemm_tc(const void* x, const void* w, const void* scales, void* y, int64_t m, int64_t n, int64_t k,
                  int64_t group, int row_tiles, lb_stream_t stream) {
  return w4_gemm_impl(x, w, scales, nullptr, y, m, n, k, group, row_tiles, stream);
}

int lb_w4_linear(const void* x, const void* w, const void* scales, const void* bias, void* y, int64_t m, int64_t n,
                 int64_t k, int64_t group, int version, lb_stream_t stream) {
  if (version == 5) return w4_gemm_impl(x, w, scales, bias, y, m, n, k, group, 0, stream);
  return w4_gemv_impl(x, w, scales, bias, y, m, n, k, group, version, 0, stream);
}

int lb_w4_dequant(const void* w, const void* scales, void* out, int64_t n, int64_t k, int64_t group, int layout,
                  lb_stream_t stream) {
  if (!w || !scales || !out) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  if (group <= 0) return fail(LB_ERR_ARGUMENT, "w [N,K/2], scales [N,K/G], positive group size");
  if (n <= 0 || k <= 0 || group % 32 || k % group) return fail(LB_ERR_ARGUMENT, "shape mismatch");
  if (n > (1 << 30) || k > (1 << 28)) return fail(LB_ERR_ARGUMENT, "N or K too large");
  if (layout < 0 || layout > 2) return fail(LB_ERR_ARGUMENT, "layout is 0 (canonical), 1 (v3) or 2 (mma)");
  if (layout == 2 && (k % 128 || group % 128))
    return fail(LB_ERR_ARGUMENT, "the v5 layout needs K and group % 128 == 0");
  if (!aligned16(w) || !aligned16(out))
    return fail(LB_ERR_ALIGNMENT, "packed weights must be contiguous and 16-byte aligned");
  if (!aligned2(scales)) return fail(LB_ERR_ALIGNMENT, "scales must be 2-byte aligned");
  int rc = check_device();
  if (rc) return rc;
  return launched(lb::launch_dequant(w, scales, reinterpret_cast<__half*>(out), (int)n, (int)k, (int)group, layout,
                                     reinterpret_cast<cudaStream_t>(stream)),
                  "w4_dequant");
}

int lb_w4_quantize(const void* w, int w_is_half, void* packed, void* scales, int64_t n, int64_t k, int64_t group,
                   const float* clip_grid, int n_clip, lb_stream_t stream) {
  if (!w || !packed || !scales) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  if (group <= 0 || n <= 0 || k <= 0 || k % group || group % 32)
    return fail(LB_ERR_ARGUMENT, "K=%lld must be a multiple of the group size %lld, itself a multiple of 32",
                (long long)k, (long long)group);
  if (n > (1 << 30) || k > (1 << 28)) return fail(LB_ERR_ARGUMENT, "N or K too large");
  if (n_clip < 0 || n_clip > 32 || (n_clip > 0 && !clip_grid))
    return fail(LB_ERR_ARGUMENT, "clip grid holds 0..32 factors");
  for (int i = 0; i < n_clip; ++i)
    if (!(clip_grid[i] > 0.f)) return fail(LB_ERR_ARGUMENT, "clip factors must be positive");
  if (!aligned2(scales) || (w_is_half ? !aligned2(w) : (reinterpret_cast<uintptr_t>(w) & 3u) != 0))
    return fail(LB_ERR_ALIGNMENT, "misaligned weight or scale pointer");
  int rc = check_device();
  if (rc) return rc;
  return launched(lb::launch_quantize(w, w_is_half, reinterpret_cast<uint8_t*>(packed),
                                      reinterpret_cast<__half*>(scales), (int)n, (int)k, (int)group, clip_grid,
                                      n_clip, reinterpret_cast<cudaStream_t>(stream)),
                  "w4_quantize");
}

int lb_w4_repack(const void* canonical, void* dst, int64_t n, int64_t k, int layout, lb_stream_t stream) {
  if (!canonical || !dst) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  if (n <= 0 || k <= 0 || k % 8) return fail(LB_ERR_ARGUMENT, "K must be a positive multiple of 8");
  if (n > (1 << 30) || k > (1 << 28)) return fail(LB_ERR_ARGUMENT, "N or K too large");
  if (layout != 1 && layout != 2) return fail(LB_ERR_ARGUMENT, "repack layout is 1 (v3) or 2 (mma)");
  if (layout == 2 && k % 128)
    return fail(LB_ERR_ARGUMENT, "K=%lld must be a multiple of 128 for the tensor-core layout", (long long)k);
  if ((reinterpret_cast<uintptr_t>(dst) & 3u) != 0) return fail(LB_ERR_ALIGNMENT, "dst must be 4-byte aligned");
  const char* a = static_cast<const char*>(canonical);
  const char* b = static_cast<const char*>(dst);
  const size_t bytes = (size_t)n * (size_t)(k / 2);
  if (a < b + bytes && b < a + bytes) return fail(LB_ERR_ARGUMENT, "src and dst overlap");
  int rc = check_device();
  if (rc) return rc;
  return launched(lb::launch_repack(static_cast<const uint8_t*>(canonical), static_cast<uint8_t*>(dst), (int)n,
                                    (int)k, layout, reinterpret_cast<cudaStream_t>(stream)),
                  "w4_repack");
}

// ------------------------------------------------------------------------------------------ decode step
int lb_decode_embed(const void* emb, const int64_t* tok, void* x, int64_t H, lb_stream_t stream) {
  if (!emb || !tok || !x) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  if (H <= 0 || H > (1 << 20)) return fail(LB_ERR_ARGUMENT, "bad hidden size %lld", (long long)H);
  int rc = check_device();
  if (rc) return rc;
  return launched(lb::launch_embed(static_cast<const __half*>(emb), tok, static_cast<__half*>(x), (int)H,
                                   reinterpret_cast<cudaStream_t>(stream)),
                  "decode_embed");
}

int lb_decode_rmsnorm(void* x, const void* r, const void* w, void* h, int64_t H, float eps, lb_stream_t stream) {
  if (!x || !w || !h) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  if (H <= 0 || H % 8 || H > lb::rmsnorm_max_hidden())
    return fail(LB_ERR_ARGUMENT, "hidden size %lld must be a positive multiple of 8 up to %d", (long long)H,
                lb::rmsnorm_max_hidden());
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(r) | reinterpret_cast<uintptr_t>(w) |
        reinterpret_cast<uintptr_t>(h)) & 15u) != 0)
    return fail(LB_ERR_ALIGNMENT, "x, r, w and h must be 16-byte aligned");
  int rc = check_device();
  if (rc) return rc;
  return launched(lb::launch_rmsnorm(static_cast<__half*>(x), static_cast<const __half*>(r),
                                     static_cast<const __half*>(w), static_cast<__half*>(h), (int)H, eps,
                                     reinterpret_cast<cudaStream_t>(stream)),
                  "decode_rmsnorm");
}

static int check_heads(int nh, int nkv, int hd, int64_t max_len) {
  if (nh <= 0 || nkv <= 0 || nh % nkv) return fail(LB_ERR_ARGUMENT, "head counts %d / %d", nh, nkv);
  // the combine step runs one thread per head dimension and reduces with full-warp shuffles: at least one warp
  if (hd < 32 || hd % 8 || hd > 1024)
    return fail(LB_ERR_ARGUMENT, "head dim %d must be a multiple of 8 in 32..1024", hd);
  if (max_len <= 0 || max_len > lb::attn_max_len())
    return fail(LB_ERR_ARGUMENT, "cache length %lld must be in 1..%d", (long long)max_len, lb::attn_max_len());
  if (lb::attn_smem_bytes(nh, nkv, hd) > 227 * 1024)
    return fail(LB_ERR_UNSUPPORTED, "%d query heads per kv head at head dim %d need more shared memory than a CTA has",
                nh / nkv, hd);
  return 0;
}

// the attention kernels read qkv and bias with 8-byte vectors, inv_freq and the caches with 16-byte ones
static int check_attention_alignment(const void* qkv, const void* bias, const void* inv_freq, const void* kc,
                                     const void* vc) {
  if (((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(inv_freq) |
        reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15u) != 0)
    return fail(LB_ERR_ALIGNMENT, "qkv, bias, inv_freq and the caches must be 16-byte aligned");
  return 0;
}

int lb_decode_attention_splits(int64_t max_len) { return max_len > 0 ? lb::attn_splits((int)max_len) : 0; }

int lb_decode_attention(const void* qkv, const void* bias, const float* inv_freq, const int64_t* pos, void* k_cache,
                        void* v_cache, float* part_o, float* part_ml, void* out, int nh, int nkv, int hd,
                        int64_t max_len, lb_stream_t stream) {
  if (!qkv || !inv_freq || !pos || !k_cache || !v_cache || !part_o || !part_ml || !out)
    return fail(LB_ERR_ARGUMENT, "null pointer argument");
  int rc = check_heads(nh, nkv, hd, max_len);
  if (rc) return rc;
  if ((rc = check_attention_alignment(qkv, bias, inv_freq, k_cache, v_cache))) return rc;
  if (((reinterpret_cast<uintptr_t>(part_o) & 15u) | (reinterpret_cast<uintptr_t>(part_ml) & 7u)) != 0)
    return fail(LB_ERR_ALIGNMENT, "part_o must be 16-byte and part_ml 8-byte aligned");
  if ((rc = check_device())) return rc;
  return launched(lb::launch_attention(static_cast<const __half*>(qkv), static_cast<const __half*>(bias), inv_freq, pos,
                                       static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), part_o, part_ml,
                                       static_cast<__half*>(out), nh, nkv, hd, (int)max_len,
                                       reinterpret_cast<cudaStream_t>(stream)),
                  "decode_attention");
}

int lb_decode_attention_noalloc(const void* qkv, const void* bias, const float* inv_freq, const int64_t* pos,
                                void* k_cache, void* v_cache, void* out, int nh, int nkv, int hd, int64_t max_len,
                                lb_stream_t stream) {
  if (!qkv || !inv_freq || !pos || !k_cache || !v_cache || !out) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  int rc = check_heads(nh, nkv, hd, max_len);
  if (rc) return rc;
  const size_t splits = (size_t)lb::attn_splits((int)max_len);
  const size_t need = (size_t)nh * splits * (size_t)(hd + 2);
  if (need > lb::kNoAllocScratchFloats)
    return fail(LB_ERR_ARGUMENT,
                "lb_decode_attention_noalloc needs %zu floats of scratch (%d heads x %zu splits x (%d + 2)); the "
                "library holds %zu -- pass caller-owned scratch to lb_decode_attention instead",
                need, nh, splits, hd, lb::kNoAllocScratchFloats);
  if ((rc = check_attention_alignment(qkv, bias, inv_freq, k_cache, v_cache))) return rc;
  if ((rc = check_device())) return rc;
  float* scratch = lb::noalloc_attn_scratch();
  if (!scratch) return fail(LB_ERR_CUDA, "could not resolve the attention scratch on this device");
  float* part_o = scratch;
  float* part_ml = scratch + (size_t)nh * splits * hd;
  return launched(lb::launch_attention(static_cast<const __half*>(qkv), static_cast<const __half*>(bias), inv_freq, pos,
                                       static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), part_o, part_ml,
                                       static_cast<__half*>(out), nh, nkv, hd, (int)max_len,
                                       reinterpret_cast<cudaStream_t>(stream)),
                  "decode_attention_noalloc");
}

static int decode_gemv(int pro, const void* x, const void* r, const void* norm_w, void* x_out, float eps, const void* w,
                       const void* scales, void* y, int64_t n, int64_t k, int64_t group, lb_stream_t stream) {
  int rc = check_common(x, w, scales, y, 1, n, k, group);
  if (rc) return rc;
  if (k % 128 || group % 128) return fail(LB_ERR_ARGUMENT, "the fused decode GEMV needs K and the group size to be multiples of 128");
  if (pro == 1 && !norm_w) return fail(LB_ERR_ARGUMENT, "null norm weight");
  if (((reinterpret_cast<uintptr_t>(r) | reinterpret_cast<uintptr_t>(norm_w) | reinterpret_cast<uintptr_t>(x_out)) &
       15u) != 0)
    return fail(LB_ERR_ALIGNMENT, "r, norm weight and x_out must be 16-byte aligned");
  const lb::OneshotConfig c = unsplit_config((int)n, (int)k);
  if (c.warps == 0)
    return fail(LB_ERR_UNSUPPORTED, "K=%lld is too long for a fused decode GEMV (one CTA holds at most 16384)",
                (long long)k);
  lb::GemvParams p{x, w, scales, reinterpret_cast<__half*>(y), 1, (int)n, (int)k, (int)group,
                   g_opt[LB_OPT_EARLY_WEIGHTS].load() ? (int)lb::kFlagEarlyWeights : 0, 1, (int)(k / group),
                   (int)(group / 128)};
  p.pro = pro;
  p.pro_r = static_cast<const __half*>(r);
  p.pro_w = static_cast<const __half*>(norm_w);
  p.pro_out = static_cast<__half*>(x_out);
  p.pro_eps = eps;
  return launched(lb::launch_gemv_oneshot(p, c, reinterpret_cast<cudaStream_t>(stream)), "decode_gemv");
}

int lb_decode_gemv_fusable(int64_t n, int64_t k) {
  if (n <= 0 || k <= 0 || k % 128 || n > (1 << 30) || k > (1 << 28)) return 0;
  return unsplit_config((int)n, (int)k).warps > 0 ? 1 : 0;
}

int lb_decode_norm_gemv(const void* x, const void* r, const void* norm_w, void* x_out, float eps, const void* w,
                        const void* scales, void* y, int64_t n, int64_t k, int64_t group, lb_stream_t stream) {
  return decode_gemv(1, x, r, norm_w, x_out, eps, w, scales, y, n, k, group, stream);
}

int lb_decode_swiglu_gemv(const void* gu, const void* w, const void* scales, void* y, int64_t n, int64_t k, int64_t group,
                          lb_stream_t stream) {
  return decode_gemv(2, gu, nullptr, nullptr, nullptr, 0.f, w, scales, y, n, k, group, stream);
}

int lb_tp_allreduce(const void* in, void* out, int64_t n, int64_t cap, void* const* bufs, uint32_t* epoch, int rank,
                    int world, lb_stream_t stream) {
  if (!in || !out || !bufs || !epoch) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  if (world < 1 || world > 64 || rank < 0 || rank >= world)
    return fail(LB_ERR_ARGUMENT, "rank %d of world %d (at most 64 ranks)", rank, world);
  if (n <= 0 || cap < n || cap > (1 << 26)) return fail(LB_ERR_ARGUMENT, "n = %lld must fit the slot capacity %lld",
                                                        (long long)n, (long long)cap);
  if (n % 8 || cap % 8) return fail(LB_ERR_ARGUMENT, "n and the slot capacity must be multiples of 8");
  if (((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) != 0)
    return fail(LB_ERR_ALIGNMENT, "in and out must be 16-byte aligned");
  int rc = check_device();
  if (rc) return rc;
  return launched(lb::launch_allreduce_oneshot(static_cast<const __half*>(in), static_cast<__half*>(out), (int)n,
                                               (int)cap, reinterpret_cast<uint8_t* const*>(bufs), epoch, rank, world,
                                               reinterpret_cast<cudaStream_t>(stream)),
                  "tp_allreduce");
}

int lb_tp_allreduce_norm(const void* in, int64_t n, int64_t cap, void* const* bufs, uint32_t* epoch, int rank, int world,
                         void* x_res, const void* norm_w, void* h_out, float eps, lb_stream_t stream) {
  if (!in || !bufs || !epoch || !x_res || !norm_w || !h_out) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  if (world < 1 || world > 64 || rank < 0 || rank >= world)
    return fail(LB_ERR_ARGUMENT, "rank %d of world %d (at most 64 ranks)", rank, world);
  if (n <= 0 || cap < n || cap > (1 << 26) || n % 8 || cap % 8)
    return fail(LB_ERR_ARGUMENT, "n = %lld must be a multiple of 8 within the slot capacity %lld", (long long)n,
                (long long)cap);
  if (((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(x_res) | reinterpret_cast<uintptr_t>(norm_w) |
        reinterpret_cast<uintptr_t>(h_out)) & 15u) != 0)
    return fail(LB_ERR_ALIGNMENT, "in, x_res, norm_w and h_out must be 16-byte aligned");
  int rc = check_device();
  if (rc) return rc;
  return launched(lb::launch_allreduce_oneshot(static_cast<const __half*>(in), nullptr, (int)n, (int)cap,
                                               reinterpret_cast<uint8_t* const*>(bufs), epoch, rank, world,
                                               reinterpret_cast<cudaStream_t>(stream), static_cast<__half*>(x_res),
                                               static_cast<const __half*>(norm_w), static_cast<__half*>(h_out), eps),
                  "tp_allreduce_norm");
}

// the plain M = 1 GEMV's own configuration (the same kernel, split and tiling as lb_w4_gemv version 6), with an
// epilogue
static int epi_gemv(lb::GemvParams& p, int64_t n, int64_t k, int64_t group, lb_stream_t stream) {
  int rc = check_common(p.x, p.w, p.s, p.y, 1, n, k, group);
  if (rc) return rc;
  if (k % 128 || group % 128)
    return fail(LB_ERR_ARGUMENT, "the fused decode GEMV needs K and the group size to be multiples of 128");
  const lb::OneshotConfig c = oneshot_config(1, (int)n, (int)k);
  if (c.warps == 0)
    return fail(LB_ERR_UNSUPPORTED, "K=%lld is too long for the one-shot GEMV", (long long)k);
  return launched(lb::launch_gemv_oneshot(p, c, reinterpret_cast<cudaStream_t>(stream)), "decode_gemv");
}

int lb_decode_gemv_swiglu(const void* x, const void* w, const void* scales, void* a, int64_t n, int64_t k, int64_t group,
                          lb_stream_t stream) {
  if (n % 16) return fail(LB_ERR_ARGUMENT, "the interleaved gate|up layer needs N %% 16 == 0 (N = %lld)", (long long)n);
  lb::GemvParams p{x, w, scales, reinterpret_cast<__half*>(a), 1, (int)n, (int)k, (int)group,
                   g_opt[LB_OPT_EARLY_WEIGHTS].load() ? (int)lb::kFlagEarlyWeights : 0, 1, (int)(k / group),
                   (int)(group / 128)};
  p.epi = 1;
  return epi_gemv(p, n, k, group, stream);
}

int lb_decode_gemv_residual_norm(const void* x, const void* w, const void* scales, void* y, int64_t n, int64_t k,
                                 int64_t group, void* x_res, const void* norm_w, void* h_out, float eps, int* counter,
                                 lb_stream_t stream) {
  if (!x_res || !norm_w || !h_out || !counter) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  if (n % 8) return fail(LB_ERR_ARGUMENT, "N = %lld must be a multiple of 8", (long long)n);
  if (((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(x_res) | reinterpret_cast<uintptr_t>(norm_w) |
        reinterpret_cast<uintptr_t>(h_out)) & 15u) != 0)
    return fail(LB_ERR_ALIGNMENT, "y, x_res, norm_w and h_out must be 16-byte aligned");
  lb::GemvParams p{x, w, scales, reinterpret_cast<__half*>(y), 1, (int)n, (int)k, (int)group,
                   g_opt[LB_OPT_EARLY_WEIGHTS].load() ? (int)lb::kFlagEarlyWeights : 0, 1, (int)(k / group),
                   (int)(group / 128)};
  p.epi = 2;
  p.epi_counter = counter;
  p.epi_x = static_cast<__half*>(x_res);
  p.epi_w = static_cast<const __half*>(norm_w);
  p.epi_h = static_cast<__half*>(h_out);
  p.epi_eps = eps;
  return epi_gemv(p, n, k, group, stream);
}

int lb_tp_gemv_allreduce_norm(const void* x, const void* w, const void* scales, void* y, int64_t n, int64_t k,
                              int64_t group, int64_t cap, void* const* bufs, uint32_t* epoch, int rank, int world,
                              void* x_res, const void* norm_w, void* h_out, float eps, int* counter,
                              lb_stream_t stream) {
  if (!bufs || !epoch || !x_res || !norm_w || !h_out || !counter) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  if (world < 1 || world > 64 || rank < 0 || rank >= world)
    return fail(LB_ERR_ARGUMENT, "rank %d of world %d (at most 64 ranks)", rank, world);
  if (n % 8 || cap % 8 || cap < n || cap > (1 << 26))
    return fail(LB_ERR_ARGUMENT, "N = %lld must be a multiple of 8 within the slot capacity %lld (a multiple of 8)",
                (long long)n, (long long)cap);
  if (((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(x_res) | reinterpret_cast<uintptr_t>(norm_w) |
        reinterpret_cast<uintptr_t>(h_out)) & 15u) != 0)
    return fail(LB_ERR_ALIGNMENT, "y, x_res, norm_w and h_out must be 16-byte aligned");
  lb::GemvParams p{x, w, scales, reinterpret_cast<__half*>(y), 1, (int)n, (int)k, (int)group,
                   g_opt[LB_OPT_EARLY_WEIGHTS].load() ? (int)lb::kFlagEarlyWeights : 0, 1, (int)(k / group),
                   (int)(group / 128)};
  p.epi = 3;
  p.epi_counter = counter;
  p.epi_x = static_cast<__half*>(x_res);
  p.epi_w = static_cast<const __half*>(norm_w);
  p.epi_h = static_cast<__half*>(h_out);
  p.epi_eps = eps;
  p.ar_bufs = reinterpret_cast<uint8_t* const*>(bufs);
  p.ar_epoch = epoch;
  p.ar_rank = rank;
  p.ar_world = world;
  p.ar_cap = (int)cap;
  int rc = check_common(x, w, scales, y ? y : x_res, 1, n, k, group);
  if (rc) return rc;
  if (k % 128 || group % 128)
    return fail(LB_ERR_ARGUMENT, "the fused decode GEMV needs K and the group size to be multiples of 128");
  const lb::OneshotConfig c = oneshot_config(1, (int)n, (int)k);
  if (c.warps == 0) return fail(LB_ERR_UNSUPPORTED, "K=%lld is too long for the one-shot GEMV", (long long)k);
  return launched(lb::launch_gemv_oneshot(p, c, reinterpret_cast<cudaStream_t>(stream)), "tp_gemv_allreduce_norm");
}

int lb_decode_silu_mul(const void* gu, void* a, int64_t I, lb_stream_t stream) {
  if (!gu || !a) return fail(LB_ERR_ARGUMENT, "null pointer argument");
  if (I <= 0 || I > (1 << 28)) return fail(LB_ERR_ARGUMENT, "bad size %lld", (long long)I);
  int rc = check_device();
  if (rc) return rc;
  return launched(lb::launch_silu_mul(static_cast<const __half*>(gu), static_cast<__half*>(a), (int)I,
                                      reinterpret_cast<cudaStream_t>(stream)),
                  "decode_silu_mul");
}

}  // extern "C"
