/*
 * CPU oracle for the W4A16 path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's format and arithmetic, used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline / --impl reference leg as the checker. The
 * library under lowbit-kernels_b200/ never links, loads or calls this code.
 *
 * Every function cites the reference file:line it restates (paths inside YuchenHe985/lowbit-kernels).
 * Parity of this file is pinned against golden vectors produced by the reference's own Python
 * (tests/golden/make_golden.py) in tests/test_oracle.py.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define LBO_QMIN (-8)
#define LBO_QMAX 7
#define LBO_OFFSET 8

/* ---- IEEE binary16 <-> binary32, round to nearest even (written from the IEEE 754 definitions) ---- */

uint16_t lbo_f32_to_f16(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  uint32_t sign = (b >> 16) & 0x8000u;
  uint32_t exp = (b >> 23) & 0xFFu;
  uint32_t man = b & 0x7FFFFFu;
  if (exp == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u)); /* inf / nan */
  int e = (int)exp - 127 + 15;                                              /* rebias */
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);                           /* overflow -> inf */
  if (e <= 0) {                                                             /* subnormal or zero */
    if (e < -10) return (uint16_t)sign;
    uint32_t m = man | 0x800000u;                                           /* implicit one */
    int shift = 14 - e;                                                     /* 24-bit mantissa -> (10 + e) bits */
    uint32_t half = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1u))) half++;
    return (uint16_t)(sign | half);
  }
  uint32_t half = ((uint32_t)e << 10) | (man >> 13);
  uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half++;             /* may carry into the exponent */
  return (uint16_t)(sign | half);
}

float lbo_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t b;
  if (exp == 0) {
    if (man == 0) {
      b = sign;
    } else {                                                                /* normalise a subnormal */
      int e = -1;
      do { man <<= 1; e++; } while (!(man & 0x400u));
      b = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    b = sign | 0x7F800000u | (man << 13);
  } else {
    b = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &b, 4);
  return f;
}

static int bad_group(int64_t k, int64_t group) { return group <= 0 || k % group || group % 32; }

/* lowbit/quant.py:23-35 (quantize_w4): scale = fp16(amax / 7) (fp32 division), an all-zero group -> 1.0;
 * q = clip(rint(w / fp32(scale)), -8, 7); byte j = u[2j] | u[2j+1] << 4 with u = q + 8. rintf rounds half to
 * even under the default rounding mode, like numpy.rint. */
int lbo_quantize(const float* w, int64_t n, int64_t k, int64_t group, uint8_t* packed, uint16_t* scales) {
  if (bad_group(k, group)) return 1;
  int64_t ng = k / group;
  for (int64_t r = 0; r < n; ++r) {
    for (int64_t g = 0; g < ng; ++g) {
      const float* src = w + r * k + g * group;
      float amax = 0.f;
      for (int64_t i = 0; i < group; ++i) {
        float a = fabsf(src[i]);
        if (a > amax || isnan(a)) amax = a;
      }
      uint16_t s16 = lbo_f32_to_f16(amax / 7.0f);
      if ((s16 & 0x7FFFu) == 0) s16 = 0x3C00u;                                 /* 1.0 */
      scales[r * ng + g] = s16;
      float s = lbo_f16_to_f32(s16);
      for (int64_t i = 0; i < group; i += 2) {
        int u[2];
        for (int h = 0; h < 2; ++h) {
          float q = rintf(src[i + h] / s);
          if (q < LBO_QMIN) q = LBO_QMIN;
          if (q > LBO_QMAX) q = LBO_QMAX;
          u[h] = (int)q + LBO_OFFSET;
        }
        packed[r * (k / 2) + (g * group + i) / 2] = (uint8_t)(u[0] | (u[1] << 4));
      }
    }
  }
  return 0;
}

/* lowbit/quant.py:38-44 (unpack_w4): canonical nibble k of row r, as a signed value -8..7 */
static inline int canon_q(const uint8_t* packed, int64_t k, int64_t r, int64_t kk) {
  uint8_t b = packed[r * (k / 2) + kk / 2];
  return (int)((kk & 1) ? (b >> 4) : (b & 0xF)) - LBO_OFFSET;
}

/* lowbit/quant.py:47-51 (dequantize_w4): q * scale in fp32 (exact) */
int lbo_dequantize_f32(const uint8_t* packed, const uint16_t* scales, int64_t n, int64_t k, int64_t group,
                       float* out) {
  if (bad_group(k, group)) return 1;
  for (int64_t r = 0; r < n; ++r)
    for (int64_t kk = 0; kk < k; ++kk)
      out[r * k + kk] = (float)canon_q(packed, k, r, kk) * lbo_f16_to_f32(scales[r * (k / group) + kk / group]);
  return 0;
}

/* lowbit/ops.py:119-123 (dequantize_w4_gpu) and csrc/w4_gemv.cu:296-310 (dequant_kernel): fp16 bits of
 * (u - 8) * scale computed in fp32 and rounded once to fp16 */
int lbo_dequantize_f16(const uint8_t* packed, const uint16_t* scales, int64_t n, int64_t k, int64_t group,
                       uint16_t* out) {
  if (bad_group(k, group)) return 1;
  for (int64_t r = 0; r < n; ++r)
    for (int64_t kk = 0; kk < k; ++kk)
      out[r * k + kk] = lbo_f32_to_f16((float)canon_q(packed, k, r, kk) *
                                       lbo_f16_to_f32(scales[r * (k / group) + kk / group]));
  return 0;
}

/* lowbit/quant.py:53-64 (SLOT_TO_K, interleave_for_gpu): nibble slot s of every word holds k0 + SLOT_TO_K[s] */
static const int kSlotToK[8] = {0, 2, 4, 6, 1, 3, 5, 7};

int lbo_interleave_gpu(const uint8_t* packed, int64_t n, int64_t k, uint8_t* out) {
  if (k % 8) return 1;
  for (int64_t r = 0; r < n; ++r) {
    const uint8_t* src = packed + r * (k / 2);
    uint8_t* dst = out + r * (k / 2);
    for (int64_t wd = 0; wd < k / 8; ++wd) {
      uint32_t word = 0;
      for (int s = 0; s < 8; ++s) {
        int64_t kk = 8 * wd + kSlotToK[s];
        uint32_t u = (kk & 1) ? (src[kk / 2] >> 4) : (src[kk / 2] & 0xF);
        word |= u << (4 * s);
      }
      for (int b = 0; b < 4; ++b) dst[4 * wd + b] = (uint8_t)(word >> (8 * b));
    }
  }
  return 0;
}

/* lowbit/quant.py:66-78 (MMA_BYTE_ORDER, interleave_for_mma): inside each 64-byte chunk, byte 16t + s takes
 * canonical byte 4s + t, then the v3 slot order is applied to every word */
int lbo_interleave_mma(const uint8_t* packed, int64_t n, int64_t k, uint8_t* out) {
  if (k % 128) return 1;
  int64_t half = k / 2;
  uint8_t* tmp = (uint8_t*)malloc((size_t)(n * half));
  if (!tmp) return 2;
  for (int64_t r = 0; r < n; ++r)
    for (int64_t c = 0; c < half / 64; ++c)
      for (int t = 0; t < 4; ++t)
        for (int s = 0; s < 16; ++s)
          tmp[r * half + 64 * c + 16 * t + s] = packed[r * half + 64 * c + 4 * s + t];
  int rc = lbo_interleave_gpu(tmp, n, k, out);
  free(tmp);
  return rc;
}

/* The signed value the mma layout stores for (row r, k = kk): the inverse of lbo_interleave_mma, read the way
 * the reference's gemv_v6 reads it (csrc/w4_gemv.cu:327-391): chunk c = kk / 128, lane t, word i, pair j. */
static inline int mma_q(const uint8_t* w, int64_t k, int64_t r, int64_t kk) {
  int64_t c = kk / 128, o = kk % 128;           /* o = 32i + 8j + 2t + h */
  int i = (int)(o / 32), j = (int)((o % 32) / 8), t = (int)((o % 8) / 2), h = (int)(o % 2);
  const uint8_t* p = w + r * (k / 2) + 64 * c + 16 * t + 4 * i;
  uint32_t word = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
  return (int)((word >> (4 * j + 16 * h)) & 0xF) - LBO_OFFSET;
}

/* The same for the v3 layout: word k / 8, slot of k0 + d is (d even ? d / 2 : 4 + d / 2) */
static inline int v3_q(const uint8_t* w, int64_t k, int64_t r, int64_t kk) {
  const uint8_t* p = w + r * (k / 2) + 4 * (kk / 8);
  uint32_t word = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
  int d = (int)(kk % 8), slot = (d % 2) ? 4 + d / 2 : d / 2;
  return (int)((word >> (4 * slot)) & 0xF) - LBO_OFFSET;
}

/* layout: 0 canonical, 1 v3, 2 mma */
static inline int layout_q(const uint8_t* w, int layout, int64_t k, int64_t r, int64_t kk) {
  return layout == 2 ? mma_q(w, k, r, kk) : layout == 1 ? v3_q(w, k, r, kk) : canon_q(w, k, r, kk);
}

/* csrc/w4_gemv.cu:393-408 (dequant_mma_kernel) and :296-310: fp16 weights [N, K] from any layout */
int lbo_dequantize_layout_f16(const uint8_t* w, int layout, const uint16_t* scales, int64_t n, int64_t k,
                              int64_t group, uint16_t* out) {
  if (bad_group(k, group) || (layout == 2 && k % 128) || (layout == 1 && k % 8)) return 1;
  for (int64_t r = 0; r < n; ++r)
    for (int64_t kk = 0; kk < k; ++kk)
      out[r * k + kk] = lbo_f32_to_f16((float)layout_q(w, layout, k, r, kk) *
                                       lbo_f16_to_f32(scales[r * (k / group) + kk / group]));
  return 0;
}

/* lowbit/quant.py:81-84 (gemv_reference): y[m, n] = sum_k x[m, k] * (q * scale) in double, with x given as fp16
 * bits, for weights in any of the three layouts */
int lbo_gemv_ref(const uint16_t* x, int64_t m, const uint8_t* w, int layout, const uint16_t* scales, int64_t n,
                 int64_t k, int64_t group, double* y) {
  if (bad_group(k, group) || (layout == 2 && k % 128) || (layout == 1 && k % 8)) return 1;
  double* wrow = (double*)malloc(sizeof(double) * (size_t)k);
  if (!wrow) return 2;
  for (int64_t r = 0; r < n; ++r) {
    for (int64_t kk = 0; kk < k; ++kk)
      wrow[kk] = (double)layout_q(w, layout, k, r, kk) * (double)lbo_f16_to_f32(scales[r * (k / group) + kk / group]);
    for (int64_t i = 0; i < m; ++i) {
      double acc = 0.0;
      const uint16_t* xr = x + i * k;
      for (int64_t kk = 0; kk < k; ++kk) acc += (double)lbo_f16_to_f32(xr[kk]) * wrow[kk];
      y[i * n + r] = acc;
    }
  }
  free(wrow);
  return 0;
}
