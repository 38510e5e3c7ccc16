/*
 * oracle.c -- CPU restatement of Nimformer's quantised-weight matmul path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Every function follows the
 * reference procedure cited above it, in the same loop order and with the
 * same float32 rounding points.  Compile with -O2 -ffp-contract=off.
 */
#include "oracle.h"

#include <math.h>
#include <float.h>
#include <stdlib.h>
#include <string.h>

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline int64_t clampi(int64_t v, int64_t lo, int64_t hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

/* Nim's round(float32) is C roundf (half away from zero); int() truncates. */
static inline int64_t nim_round_to_int(float v) { return (int64_t)roundf(v); }

/* ------------------------------------------------------------------------ */
/* quant.nim:45-49 maxAbs */
static float max_abs(const float* a, int64_t n) {
  float r = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    float v = fabsf(a[i]);
    if (v > r) r = v;
  }
  return r;
}

/* quant.nim:51-61 */
void orc_quantize_int8(const float* arr, int64_t n, int8_t* q, float* scale) {
  float m = max_abs(arr, n);
  float sc = (m == 0.0f) ? 1.0f : m / 127.0f;
  *scale = sc;
  for (int64_t i = 0; i < n; ++i) {
    float t = arr[i] / sc;
    q[i] = (int8_t)clampi(nim_round_to_int(t), -127, 127);
  }
}

/* quant.nim:63-67 */
void orc_dequantize_int8(const int8_t* q, int64_t n, float scale, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = (float)q[i] * scale;
}

/* quant.nim:69-85 */
void orc_quantize_int4_sym(const float* arr, int64_t n, uint8_t* packed, float* scale) {
  float m = max_abs(arr, n);
  float sc = (m == 0.0f) ? 1.0f : m / 7.0f;
  *scale = sc;
  if (n > 0) memset(packed, 0, (size_t)((n + 1) / 2));
  for (int64_t i = 0; i < n; ++i) {
    float t = arr[i] / sc;
    int64_t qv = clampi(nim_round_to_int(t), -7, 7);
    uint8_t nib = (uint8_t)(qv & 0x0F);
    int64_t b = i / 2;
    if (i % 2 == 0) packed[b] = (uint8_t)((packed[b] & 0xF0u) | nib);
    else packed[b] = (uint8_t)((packed[b] & 0x0Fu) | (uint8_t)(nib << 4));
  }
}

/* quant.nim:87-98 */
void orc_dequantize_int4_sym(const uint8_t* packed, int64_t n, float scale, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    uint8_t b = packed[i / 2];
    int nib = (i % 2 == 0) ? (b & 0x0F) : ((b >> 4) & 0x0F);
    int s = nib >= 8 ? nib - 16 : nib;
    out[i] = (float)s * scale;
  }
}

/* quant.nim:104-129 */
void orc_quantize_int4_asym_tensor(const float* arr, int64_t n, uint8_t* packed,
                                   float* scale, float* zero) {
  float mn = FLT_MAX, mx = -FLT_MAX;
  for (int64_t i = 0; i < n; ++i) {
    if (arr[i] < mn) mn = arr[i];
    if (arr[i] > mx) mx = arr[i];
  }
  float range = mx - mn;
  float sc = (range < 1e-12f) ? 1.0f : range / 15.0f;
  float zp = (range < 1e-12f) ? 0.0f : -mn / sc;
  *scale = sc;
  *zero = zp;
  if (n > 0) memset(packed, 0, (size_t)((n + 1) / 2));
  for (int64_t i = 0; i < n; ++i) {
    float t = arr[i] / sc;
    t = t + zp;
    int64_t qv = clampi(nim_round_to_int(t), 0, 15);
    uint8_t nib = (uint8_t)(qv & 0x0F);
    int64_t b = i / 2;
    if (i % 2 == 0) packed[b] = (uint8_t)((packed[b] & 0xF0u) | nib);
    else packed[b] = (uint8_t)((packed[b] & 0x0Fu) | (uint8_t)(nib << 4));
  }
}

static inline int nibble_at(const uint8_t* data, int64_t byte_idx, int64_t c) {
  uint8_t b = data[byte_idx];
  return (c % 2 == 0) ? (b & 0x0F) : ((b >> 4) & 0x0F);
}

/* quant.nim:131-192 */
void orc_dequantize_int4_asym(const uint8_t* data, const float* scale, const float* zero,
                              int64_t n_scales, int64_t rows, int64_t cols,
                              int64_t group_size, float* out) {
  float lut[16];
  if (group_size > 0) {
    int64_t bpr = (cols + 1) / 2;
    int64_t ngr = (cols + group_size - 1) / group_size;
    for (int64_t r = 0; r < rows; ++r) {
      int64_t rbo = r * bpr, rgo = r * ngr, g = -1;
      for (int64_t c = 0; c < cols; ++c) {
        int64_t gn = c / group_size;
        if (gn != g) {
          g = gn;
          float sc = scale[rgo + g], zp = zero[rgo + g];
          for (int k = 0; k < 16; ++k) { float d = (float)k - zp; lut[k] = d * sc; }
        }
        out[r * cols + c] = lut[nibble_at(data, rbo + c / 2, c)];
      }
    }
  } else if (n_scales > 1) {
    int64_t bpr = (cols + 1) / 2;
    for (int64_t r = 0; r < rows; ++r) {
      float sc = scale[r], zp = zero[r];
      for (int k = 0; k < 16; ++k) { float d = (float)k - zp; lut[k] = d * sc; }
      int64_t rbo = r * bpr;
      for (int64_t c = 0; c < cols; ++c)
        out[r * cols + c] = lut[nibble_at(data, rbo + c / 2, c)];
    }
  } else {
    float sc = scale[0], zp = zero[0];
    int64_t n = rows * cols;
    for (int64_t i = 0; i < n; ++i) {
      float d = (float)nibble_at(data, i / 2, i) - zp;
      out[i] = d * sc;
    }
  }
}

/* quant.nim:256-345 (int kinds and raw; float kinds go through decode). */
int orc_dequantize_transposed(int kind, const uint8_t* data, const float* scale,
                              const float* zero, int64_t n_scales, int64_t rows,
                              int64_t cols, int64_t group_size, float* out) {
  float lut[16];
  if (kind == 3) {
    int64_t bpr = (cols + 1) / 2;
    if (group_size > 0) {
      int64_t ngr = (cols + group_size - 1) / group_size;
      for (int64_t r = 0; r < rows; ++r) {
        int64_t rbo = r * bpr, rgo = r * ngr, g = -1;
        for (int64_t c = 0; c < cols; ++c) {
          int64_t gn = c / group_size;
          if (gn != g) {
            g = gn;
            float sc = scale[rgo + g], zp = zero[rgo + g];
            for (int k = 0; k < 16; ++k) { float d = (float)k - zp; lut[k] = d * sc; }
          }
          out[c * rows + r] = lut[nibble_at(data, rbo + c / 2, c)];
        }
      }
    } else if (n_scales > 1) {
      for (int64_t r = 0; r < rows; ++r) {
        float sc = scale[r], zp = zero[r];
        for (int k = 0; k < 16; ++k) { float d = (float)k - zp; lut[k] = d * sc; }
        int64_t rbo = r * bpr;
        for (int64_t c = 0; c < cols; ++c)
          out[c * rows + r] = lut[nibble_at(data, rbo + c / 2, c)];
      }
    } else {
      float sc = scale[0], zp = zero[0];
      for (int k = 0; k < 16; ++k) { float d = (float)k - zp; lut[k] = d * sc; }
      for (int64_t r = 0; r < rows; ++r) {
        int64_t rbo = r * bpr;
        for (int64_t c = 0; c < cols; ++c)
          out[c * rows + r] = lut[nibble_at(data, rbo + c / 2, c)];
      }
    }
    return 0;
  }
  if (kind == 2) {
    float sc = scale[0];
    int64_t bpr = (cols + 1) / 2;
    for (int k = 0; k < 16; ++k) { int s = k >= 8 ? k - 16 : k; lut[k] = (float)s * sc; }
    for (int64_t r = 0; r < rows; ++r) {
      int64_t rbo = r * bpr;
      for (int64_t c = 0; c < cols; ++c)
        out[c * rows + r] = lut[nibble_at(data, rbo + c / 2, c)];
    }
    return 0;
  }
  if (kind == 1) {
    float sc = scale[0];
    for (int64_t r = 0; r < rows; ++r)
      for (int64_t c = 0; c < cols; ++c)
        out[c * rows + r] = (float)(int8_t)data[r * cols + c] * sc;
    return 0;
  }
  if (kind == 0) {
    for (int64_t r = 0; r < rows; ++r)
      for (int64_t c = 0; c < cols; ++c) {
        float v;
        memcpy(&v, data + 4 * (r * cols + c), 4);
        out[c * rows + r] = v;
      }
    return 0;
  }
  return -1;
}

/* ------------------------------------------------------------------------ */
/* customfloat.nim:15-31 */
orc_custom_float orc_cf_new(int e, int m) {
  orc_custom_float cf;
  cf.exponent_bits = e;
  cf.mantissa_bits = m;
  cf.total_bits = 1 + e + m;
  cf.item_size = (cf.total_bits + 7) / 8;
  if (e > 0) {
    cf.bias = (1 << (e - 1)) - 1;
    cf.max_exp = (1 << e) - 1;
  } else {
    cf.bias = 0;
    cf.max_exp = 0;
  }
  cf.uses_uint64 = cf.total_bits <= 64;
  return cf;
}

/* customfloat.nim:49-78 */
uint64_t orc_cf_fp32_to_packed(float x, int e, int m) {
  orc_custom_float cf = orc_cf_new(e, m);
  uint32_t b = f2u(x);
  uint64_t sign = (b >> 31) & 1u;
  uint64_t exp32 = (b >> 23) & 0xFFu;
  uint64_t mant32 = b & 0x7FFFFFu;
  int64_t real_exp = (int64_t)exp32 - 127;
  int is_zero = (exp32 == 0) && (mant32 == 0);
  int is_inf_nan = (exp32 == 255);
  int64_t new_exp = real_exp + cf.bias;
  int overflow = (new_exp >= cf.max_exp) && !is_zero;
  int underflow = (new_exp <= 0) && !is_zero;
  uint64_t mant = (m <= 23) ? (mant32 >> (23 - m)) : (mant32 << (m - 23));
  uint64_t new_exp_u = (uint64_t)clampi(new_exp, 0, cf.max_exp);
  uint64_t top = (uint64_t)(e + m);
  uint64_t packed = (sign << top) | (new_exp_u << m) | mant;
  uint64_t inf_pattern = (uint64_t)cf.max_exp << m;
  if (is_inf_nan || (overflow && !is_inf_nan)) packed = (sign << top) | inf_pattern;
  else if (underflow || is_zero) packed = sign << top;
  return packed;
}

/* customfloat.nim:80-102 */
float orc_cf_packed_to_fp32(uint64_t packed, int e, int m) {
  orc_custom_float cf = orc_cf_new(e, m);
  uint64_t mant_mask = (m == 0) ? 0 : ((1ull << m) - 1);
  uint64_t top = (uint64_t)(e + m);
  uint64_t sign = (packed >> top) & 1u;
  uint64_t ex = (packed >> m) & (uint64_t)cf.max_exp;
  uint64_t mant = packed & mant_mask;
  int is_zero = (ex == 0) && (mant == 0);
  int is_inf_nan = (ex == (uint64_t)cf.max_exp);
  int64_t real_exp = (int64_t)ex - cf.bias;
  uint32_t exp32 = (uint32_t)clampi(real_exp + 127, 0, 255);
  uint32_t mant32 = (m <= 23) ? (uint32_t)(mant << (23 - m)) : (uint32_t)(mant >> (m - 23));
  uint32_t bits = ((uint32_t)sign << 31) | (exp32 << 23) | mant32;
  if (is_zero) bits = (uint32_t)sign << 31;
  if (is_inf_nan) bits = ((uint32_t)sign << 31) | (0xFFu << 23);
  return u2f(bits);
}

/* customfloat.nim:108-113,125-129 */
int orc_cf_encode_array(const float* arr, int64_t n, int e, int m, uint8_t* out) {
  orc_custom_float cf = orc_cf_new(e, m);
  if (!cf.uses_uint64) return -1;
  for (int64_t i = 0; i < n; ++i) {
    uint64_t p = orc_cf_fp32_to_packed(arr[i], e, m);
    for (int b = 0; b < cf.item_size; ++b)
      out[i * cf.item_size + b] = (uint8_t)((p >> (8 * b)) & 0xFFu);
  }
  return 0;
}

/* customfloat.nim:115-123,131-136 */
int orc_cf_decode_array(const uint8_t* buf, int64_t nbytes, int e, int m, float* out) {
  orc_custom_float cf = orc_cf_new(e, m);
  if (!cf.uses_uint64) return -1;
  if (nbytes % cf.item_size != 0) return -1;
  int64_t n = nbytes / cf.item_size;
  for (int64_t i = 0; i < n; ++i) {
    uint64_t p = 0;
    for (int b = 0; b < cf.item_size; ++b)
      p |= (uint64_t)buf[i * cf.item_size + b] << (8 * b);
    out[i] = orc_cf_packed_to_fp32(p, e, m);
  }
  return 0;
}

/* Nim classify(v) notin {fcNan, fcInf, fcNegInf} and v != 0 */
static inline int finite_nonzero(float v) { return isfinite(v) && v != 0.0f; }

/* customfloat.nim:149-165 */
int orc_cf_required_exponent_bits(const float* arr, int64_t n, int exp_margin) {
  float mn = FLT_MAX, mx = 0.0f;
  int any = 0;
  for (int64_t i = 0; i < n; ++i) {
    float v = arr[i];
    if (finite_nonzero(v)) {
      any = 1;
      float a = fabsf(v);
      if (a < mn) mn = a;
      if (a > mx) mx = a;
    }
  }
  if (!any) return 1;
  int64_t max_e = (int64_t)floor(log2((double)mx));
  int64_t min_e = (int64_t)floor(log2((double)mn));
  int64_t span = (max_e - min_e) + 2 * (int64_t)exp_margin + 2;
  int64_t s2 = span > 2 ? span : 2;
  int64_t r = (int64_t)ceil(log2((double)s2));
  return (int)(r > 1 ? r : 1);
}

static int cmp_float(const void* a, const void* b) {
  float x = *(const float*)a, y = *(const float*)b;
  return (x > y) - (x < y);
}

/* customfloat.nim:167-198 */
int orc_cf_required_mantissa_bits(const float* arr, int64_t n, double tol,
                                  const float* grad, int64_t n_grad) {
  int64_t nv = 0;
  for (int64_t i = 0; i < n; ++i) nv += finite_nonzero(arr[i]);
  if (nv == 0) return 2;
  double t = tol > 1e-12 ? tol : 1e-12;
  int64_t base = (int64_t)ceil(log2(1.0 / t));
  int64_t extra = 0;
  if (grad != NULL && n_grad > 0) {
    int64_t ng = 0;
    for (int64_t i = 0; i < n_grad; ++i) ng += finite_nonzero(grad[i]);
    if (ng > 0) {
      float* vs = (float*)malloc((size_t)nv * sizeof(float));
      float* gs = (float*)malloc((size_t)ng * sizeof(float));
      int64_t j = 0;
      for (int64_t i = 0; i < n; ++i) if (finite_nonzero(arr[i])) vs[j++] = fabsf(arr[i]);
      j = 0;
      for (int64_t i = 0; i < n_grad; ++i) if (finite_nonzero(grad[i])) gs[j++] = fabsf(grad[i]);
      qsort(vs, (size_t)nv, sizeof(float), cmp_float);
      qsort(gs, (size_t)ng, sizeof(float), cmp_float);
      float wmed = vs[nv / 2];
      if (wmed < 1e-12f) wmed = 1e-12f;
      float gmed = gs[ng / 2];
      double ratio = (double)gmed / (double)wmed;
      if (ratio > 0 && ratio < 1) {
        int64_t need = (int64_t)ceil(-log2(ratio));
        extra = need - base > 0 ? need - base : 0;
      }
      free(vs);
      free(gs);
    }
  }
  return (int)clampi(base + extra, 2, 23);
}

/* ------------------------------------------------------------------------ */
/* gpubackend.nim:560-582 */
void orc_cpu_matmul(const float* a, const float* b, int64_t m, int64_t k, int64_t n,
                    float* c) {
  const int64_t bs = 64;
  if (m > 0 && n > 0) memset(c, 0, (size_t)(m * n) * sizeof(float));
  for (int64_t ii = 0; ii < m; ii += bs) {
    int64_t imax = ii + bs < m ? ii + bs : m;
    for (int64_t kk = 0; kk < k; kk += bs) {
      int64_t kmax = kk + bs < k ? kk + bs : k;
      for (int64_t jj = 0; jj < n; jj += bs) {
        int64_t jmax = jj + bs < n ? jj + bs : n;
        for (int64_t i = ii; i < imax; ++i) {
          float* crow = c + i * n;
          for (int64_t p = kk; p < kmax; ++p) {
            float av = a[i * k + p];
            if (av == 0.0f) continue;
            const float* brow = b + p * n;
            for (int64_t j = jj; j < jmax; ++j) {
              float prod = av * brow[j];
              crow[j] = crow[j] + prod;
            }
          }
        }
      }
    }
  }
}

/* gpubackend.nim:628-653 */
void orc_dequant_matmul_q4(const float* a, const uint8_t* wq, const float* scales,
                           const float* zeros, int64_t m, int64_t k, int64_t n,
                           int64_t group_size, int64_t n_groups_per_row,
                           float* wt, float* out) {
  int64_t bpr = (k + 1) / 2;
  float lut[16];
  for (int64_t row = 0; row < n; ++row) {
    int64_t rbo = row * bpr, rgo = row * n_groups_per_row, g = -1;
    for (int64_t c = 0; c < k; ++c) {
      int64_t gn = group_size > 0 ? c / group_size : 0;
      if (gn != g) {
        g = gn;
        float sc = scales[rgo + g], zp = zeros[rgo + g];
        for (int q = 0; q < 16; ++q) { float d = (float)q - zp; lut[q] = d * sc; }
      }
      wt[c * n + row] = lut[nibble_at(wq, rbo + c / 2, c)];
    }
  }
  orc_cpu_matmul(a, wt, m, k, n, out);
}

/* ------------------------------------------------------------------------ */
/* export_to_nimq.py:363-395 */
void orc_quantize_int4_asym_per_group(const float* arr, int64_t rows, int64_t cols,
                                      int64_t gs, uint8_t* packed, float* scales,
                                      float* zeros) {
  int64_t ngr = (cols + gs - 1) / gs;
  int64_t bpr = (cols + 1) / 2;
  if (rows > 0 && bpr > 0) memset(packed, 0, (size_t)(rows * bpr));
  for (int64_t r = 0; r < rows; ++r) {
    const float* row = arr + r * cols;
    for (int64_t g = 0; g < ngr; ++g) {
      int64_t c0 = g * gs, c1 = c0 + gs < cols ? c0 + gs : cols;
      float mnf = row[c0], mxf = row[c0];
      for (int64_t c = c0 + 1; c < c1; ++c) {
        if (row[c] < mnf) mnf = row[c];
        if (row[c] > mxf) mxf = row[c];
      }
      double mn = (double)mnf, mx = (double)mxf;
      double rng = mx - mn;
      double scale = rng > 1e-12 ? rng / 15.0 : 1.0;
      double zp = rng > 1e-12 ? (-mn / scale) : 0.0;
      float sf = (float)scale, zf = (float)zp;
      for (int64_t c = c0; c < c1; ++c) {
        float t = row[c] / sf;
        t = t + zf;
        float q = rintf(t);
        if (q < 0.0f) q = 0.0f;
        if (q > 15.0f) q = 15.0f;
        uint8_t nib = (uint8_t)q;
        uint8_t* p = packed + r * bpr + c / 2;
        if (c % 2 == 0) *p = (uint8_t)(*p | nib);
        else *p = (uint8_t)(*p | (uint8_t)(nib << 4));
      }
      scales[r * ngr + g] = (float)scale;
      zeros[r * ngr + g] = (float)zp;
    }
  }
}

/* export_to_nimq.py:353-360 */
void orc_quantize_int8_vectorized(const float* arr, int64_t n, int8_t* q, float* scale) {
  float mx = 0.0f;
  for (int64_t i = 0; i < n; ++i) { float a = fabsf(arr[i]); if (a > mx) mx = a; }
  if (mx < 1e-12f) {
    if (n > 0) memset(q, 0, (size_t)n);
    *scale = 1.0f;
    return;
  }
  float sc = mx / 127.0f;
  *scale = sc;
  for (int64_t i = 0; i < n; ++i) {
    float t = rintf(arr[i] / sc);
    if (t < -127.0f) t = -127.0f;
    if (t > 127.0f) t = 127.0f;
    q[i] = (int8_t)t;
  }
}

static float half_bits_to_float(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) << 31;
  uint32_t e = (h >> 10) & 0x1F, f = h & 0x3FF;
  if (e == 0) {
    if (f == 0) return u2f(s);
    float v = ldexpf((float)f, -24);
    return (h >> 15) ? -v : v;
  }
  if (e == 31) return u2f(s | 0x7F800000u | (f << 13));
  return u2f(s | ((e + 112) << 23) | (f << 13));
}

/* export_to_nimq.py:219-254 */
void orc_dequantize_gptq_linear(const int32_t* qweight, const int32_t* qzeros,
                                const uint16_t* scales_f16, const int32_t* g_idx,
                                int64_t in_features, int64_t out_features,
                                int64_t n_groups, float* out) {
  (void)n_groups;
  int64_t nzc = out_features / 8;
  for (int64_t k = 0; k < in_features; ++k) {
    int64_t g = g_idx[k];
    for (int64_t nn = 0; nn < out_features; ++nn) {
      uint32_t qw = (uint32_t)qweight[(k / 8) * out_features + nn];
      int w = (int)((qw >> (4 * (k % 8))) & 0xFu);
      uint32_t qz = (uint32_t)qzeros[g * nzc + nn / 8];
      int z = (int)(((qz >> (4 * (nn % 8))) & 0xFu) + 1) & 0xF;
      float sc = half_bits_to_float(scales_f16[g * out_features + nn]);
      float d = (float)w - (float)z;
      out[nn * in_features + k] = d * sc;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* OCP E4M3 (bias 7, subnormals, max 448, 0x7F/0xFF NaN). */
float orc_e4m3_ocp_to_float(uint8_t v) {
  int s = v >> 7, e = (v >> 3) & 0xF, m = v & 7;
  float r;
  if (e == 15 && m == 7) r = NAN;
  else if (e == 0) r = ldexpf((float)m, -9);
  else r = ldexpf((float)(8 + m), e - 10);
  return s ? -r : r;
}

/* Round-to-nearest-even into OCP E4M3, saturating at 448; NaN -> 0x7F. */
uint8_t orc_float_to_e4m3_ocp(float x) {
  if (isnan(x)) return 0x7F;
  uint8_t s = signbit(x) ? 0x80 : 0x00;
  double a = fabs((double)x);
  if (a >= 448.0) return s | 0x7E;
  if (a == 0.0) return s;
  int ex;
  frexp(a, &ex);          /* a = f * 2^ex, f in [0.5, 1) -> unbiased exponent ex-1 */
  int e = ex - 1;
  if (e < -6) {           /* subnormal grid step 2^-9 */
    double q = nearbyint(ldexp(a, 9));
    int qi = (int)q;      /* qi == 8 lands on the smallest normal 0x08 */
    return s | (uint8_t)qi;
  }
  double q = nearbyint(ldexp(a, 3 - e)); /* in [8, 16] */
  int qi = (int)q;
  if (qi == 16) { qi = 8; e += 1; }
  int be = e + 7;
  if (be > 15 || (be == 15 && qi - 8 == 7)) return s | 0x7E;
  return s | (uint8_t)((be << 3) | (qi - 8));
}

static const float kE2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

float orc_e2m1_to_float(uint8_t nib) {
  float v = kE2M1[nib & 7];
  return (nib & 8) ? -v : v;
}

/* RNE to E2M1, ties to the code with an even mantissa bit, saturating at 6. */
static uint8_t float_to_e2m1(float x) {
  if (isnan(x)) return 0;
  uint8_t s = signbit(x) ? 8 : 0;
  float a = fabsf(x);
  int best = 0;
  float bd = INFINITY;
  for (int c = 0; c < 8; ++c) {
    float d = fabsf(a - kE2M1[c]);
    if (d < bd || (d == bd && (c & 1) == 0)) { bd = d; best = c; }
  }
  if (a >= 6.0f) best = 7;
  return s | (uint8_t)best;
}

void orc_quantize_fp4_block16(const float* arr, int64_t rows, int64_t cols,
                              float tensor_scale, uint8_t* packed, uint8_t* block_scales) {
  int64_t bpr = (cols + 1) / 2, nb = (cols + 15) / 16;
  if (rows > 0 && bpr > 0) memset(packed, 0, (size_t)(rows * bpr));
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < nb; ++b) {
      int64_t c0 = b * 16, c1 = c0 + 16 < cols ? c0 + 16 : cols;
      float amax = 0.0f;
      for (int64_t c = c0; c < c1; ++c) { float a = fabsf(arr[r * cols + c]); if (a > amax) amax = a; }
      float want = amax / (6.0f * tensor_scale);
      uint8_t sc = orc_float_to_e4m3_ocp(want);
      block_scales[r * nb + b] = sc;
      float bs = orc_e4m3_ocp_to_float(sc) * tensor_scale;
      for (int64_t c = c0; c < c1; ++c) {
        uint8_t q = (bs == 0.0f) ? 0 : float_to_e2m1(arr[r * cols + c] / bs);
        uint8_t* p = packed + r * bpr + c / 2;
        if (c % 2 == 0) *p = (uint8_t)(*p | q);
        else *p = (uint8_t)(*p | (uint8_t)(q << 4));
      }
    }
  }
}

void orc_dequantize_fp4_block16(const uint8_t* packed, const uint8_t* block_scales,
                                float tensor_scale, int64_t rows, int64_t cols, float* out) {
  int64_t bpr = (cols + 1) / 2, nb = (cols + 15) / 16;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      float bs = orc_e4m3_ocp_to_float(block_scales[r * nb + c / 16]);
      float v = orc_e2m1_to_float((uint8_t)nibble_at(packed, r * bpr + c / 2, c));
      float t = bs * tensor_scale;
      out[r * cols + c] = v * t;
    }
}

void orc_gemv_f64(const float* x, const float* w, int64_t m, int64_t k, int64_t n,
                  float* y) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      double acc = 0.0;
      for (int64_t p = 0; p < k; ++p) acc += (double)x[i * k + p] * (double)w[j * k + p];
      y[i * n + j] = (float)acc;
    }
}

/* ------------------------------------------------------------------------ */
/* Decode glue of nim_inference.nim (Llama path).                            */

/* nim_inference.nim:143-200 RMSNorm.forward with rmsNormPrep :114-140:
 * x2 = x * x, sumSq = beMatmul(x2, ones) (orc_cpu_matmul order), invStd =
 * 1 / sqrt(sumSq / cols + eps), then (x * invStd) * w as two rounded muls. */
void orc_rmsnorm(const float* x, const float* w, int64_t rows, int64_t cols, float eps,
                 float* y) {
  float* x2 = (float*)malloc((size_t)cols * sizeof(float));
  float* ones = (float*)malloc((size_t)cols * sizeof(float));
  for (int64_t c = 0; c < cols; ++c) ones[c] = 1.0f;
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * cols;
    for (int64_t c = 0; c < cols; ++c) x2[c] = xr[c] * xr[c];
    float ss;
    orc_cpu_matmul(x2, ones, 1, cols, 1, &ss);
    float inv = 1.0f / sqrtf(ss / (float)cols + eps);
    for (int64_t c = 0; c < cols; ++c) {
      float t = xr[c] * inv;
      y[r * cols + c] = t * w[c];
    }
  }
  free(x2);
  free(ones);
}

/* LayerNorm.forward (nimformer.nim:188-197) through beLayernorm
 * (backend.nim:149-150) on the CPU path cpuLayernorm
 * (vendor/bybylang/gpubackend.nim:252-266): per row, mean = (sum x) / cols,
 * var = (sum (x - mean)^2) / cols, both sums sequential in c; invStd =
 * 1 / sqrt(var + eps); y = ((x - mean) * invStd) * gamma + beta. */
void orc_layernorm(const float* x, const float* gamma, const float* beta, int64_t rows,
                   int64_t cols, float eps, float* y) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * cols;
    float mean = 0.0f;
    for (int64_t c = 0; c < cols; ++c) mean += xr[c];
    mean /= (float)cols;
    float var = 0.0f;
    for (int64_t c = 0; c < cols; ++c) {
      float d = xr[c] - mean;
      var += d * d;
    }
    var /= (float)cols;
    float inv = 1.0f / sqrtf(var + eps);
    for (int64_t c = 0; c < cols; ++c) {
      float t = (xr[c] - mean) * inv;
      t = t * gamma[c];
      y[r * cols + c] = t + beta[c];
    }
  }
}

/* cpuEmbeddingLookup (vendor/bybylang/gpubackend.nim:268-278): row ids[i] of
 * table [vocab][dim], zeros for an id outside [0, vocab). */
void orc_embedding_lookup(const float* table, int64_t vocab, int64_t dim, const int32_t* ids,
                          int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    int64_t id = ids[i];
    for (int64_t j = 0; j < dim; ++j)
      out[i * dim + j] = (id >= 0 && id < vocab) ? table[id * dim + j] : 0.0f;
  }
}

/* sampleTopP (nim_inference.nim:1019-1036) with temperature <= 0, per row:
 * adjLogits = logits; for id in recentIds (in order, ids in range): divide by
 * repeatPenalty if adjLogits[id] > 0 else multiply (skipped when the penalty is
 * 1); best = 0; for i in 1 ..< vocab: if adj[i] > adj[best]: best = i. */
void orc_greedy_sample(const float* logits, int64_t rows, int64_t vocab, const int32_t* recent,
                       int64_t n_recent, float penalty, int32_t* out_ids) {
  float* adj = (float*)malloc((size_t)vocab * sizeof(float));
  for (int64_t r = 0; r < rows; ++r) {
    memcpy(adj, logits + r * vocab, (size_t)vocab * sizeof(float));
    if (penalty != 1.0f)
      for (int64_t q = 0; q < n_recent; ++q) {
        int64_t id = recent[r * n_recent + q];
        if (id >= 0 && id < vocab) {
          if (adj[id] > 0.0f) adj[id] = adj[id] / penalty;
          else adj[id] = adj[id] * penalty;
        }
      }
    int64_t best = 0;
    for (int64_t i = 1; i < vocab; ++i)
      if (adj[i] > adj[best]) best = i;
    out_ids[r] = (int32_t)best;
  }
  free(adj);
}

/* nim_inference.nim:336-356 SwiGLUL gating: sig = 1 / (1 + exp(-g))
 * (vendor/bybylang/gpubackend.nim:111-114 cpuSigmoid), out = (g * sig) * up. */
void orc_swiglu(const float* g, const float* u, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    float sig = 1.0f / (1.0f + expf(-g[i]));
    float t = g[i] * sig;
    out[i] = t * u[i];
  }
}

/* nim_inference.nim:261-330 applyRoPEInplace on [B][T][H][D]:
 * out = x * cosFull + rotHalf * sinFull, rotHalf = concat(-x2, x1), with the
 * newRoPEL tables cos_t / sin_t [max_seq][D/2] (:246-259). */
void orc_rope(float* data, int64_t B, int64_t T, int64_t H, int64_t D, int64_t pos_offset,
              const float* cos_t, const float* sin_t) {
  int64_t half = D / 2;
  for (int64_t b = 0; b < B; ++b)
    for (int64_t t = 0; t < T; ++t) {
      int64_t pos = pos_offset + t;
      for (int64_t h = 0; h < H; ++h) {
        float* d = data + ((b * T + t) * H + h) * D;
        for (int64_t i = 0; i < half; ++i) {
          float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
          float x1 = d[i], x2 = d[i + half];
          float a1 = x1 * c, b1 = (-x2) * s;
          float a2 = x2 * c, b2 = x1 * s;
          d[i] = a1 + b1;
          d[i + half] = a2 + b2;
        }
      }
    }
}

/* nim_inference.nim:404-426 appendKV (row pos of each KV head, cache layout
 * [HKV][max_seq][D]) then the attention core of forwardDecode :624-748: per
 * KV head, qGroup = q * scale, scores = qGroup . K^T (orc_cpu_matmul),
 * softmax as vendor/bybylang/gpubackend.nim:236-250 cpuSoftmax, out = P . V. */
void orc_attention_decode(const float* q, const float* k_new, const float* v_new,
                          float* k_cache, float* v_cache, int64_t H, int64_t HKV, int64_t D,
                          int64_t max_seq, int64_t pos, float scale, float* out) {
  int64_t nrep = H / HKV, S = pos + 1;
  for (int64_t h = 0; h < HKV; ++h)
    for (int64_t d = 0; d < D; ++d) {
      k_cache[(h * max_seq + pos) * D + d] = k_new[h * D + d];
      v_cache[(h * max_seq + pos) * D + d] = v_new[h * D + d];
    }
  float* kt = (float*)malloc((size_t)(D * S) * sizeof(float));
  float* vb = (float*)malloc((size_t)(S * D) * sizeof(float));
  float* qg = (float*)malloc((size_t)(nrep * D) * sizeof(float));
  float* sc = (float*)malloc((size_t)(nrep * S) * sizeof(float));
  float* og = (float*)malloc((size_t)(nrep * D) * sizeof(float));
  for (int64_t hk = 0; hk < HKV; ++hk) {
    for (int64_t s = 0; s < S; ++s)
      for (int64_t d = 0; d < D; ++d) {
        kt[d * S + s] = k_cache[(hk * max_seq + s) * D + d];
        vb[s * D + d] = v_cache[(hk * max_seq + s) * D + d];
      }
    for (int64_t r = 0; r < nrep; ++r)
      for (int64_t d = 0; d < D; ++d) qg[r * D + d] = q[(hk * nrep + r) * D + d] * scale;
    orc_cpu_matmul(qg, kt, nrep, D, S, sc);
    for (int64_t r = 0; r < nrep; ++r) {
      float* row = sc + r * S;
      float mx = row[0];
      for (int64_t s = 1; s < S; ++s)
        if (row[s] > mx) mx = row[s];
      float sum = 0.0f;
      for (int64_t s = 0; s < S; ++s) {
        float e = expf(row[s] - mx);
        row[s] = e;
        sum += e;
      }
      for (int64_t s = 0; s < S; ++s) row[s] /= sum;
    }
    orc_cpu_matmul(sc, vb, nrep, S, D, og);
    for (int64_t r = 0; r < nrep; ++r)
      for (int64_t d = 0; d < D; ++d) out[(hk * nrep + r) * D + d] = og[r * D + d];
  }
  free(kt);
  free(vb);
  free(qg);
  free(sc);
  free(og);
}

/* nim_inference.nim:574-620 forwardPrefill's attention core, generalised to a
 * chunk of T prompt tokens at positions pos0 .. pos0 + T - 1: appendKV
 * (:404-426) of the T new K / V rows [T][HKV][D] into the caches
 * [HKV][max_seq][D], then for each query head h (KV head h / (H / HKV), the
 * repeat_kv expansion of :596-606) and query t, the causal softmax attention
 * of vendor/bybylang/gpubackend.nim:171-201 cpuAttentionFused over cache rows
 * 0 .. pos0 + t: score = (q . k) * scale with the dot summed over d in order,
 * max, exp(score - max) summed in order, p = e / sum, out = sum_j p_j v_j in
 * order.  q and out are [T][H][D] (the projections' row layout). */
void orc_attention_prefill(const float* q, const float* k_new, const float* v_new,
                           float* k_cache, float* v_cache, int64_t T, int64_t H, int64_t HKV,
                           int64_t D, int64_t max_seq, int64_t pos0, float scale, float* out) {
  int64_t nrep = H / HKV;
  for (int64_t t = 0; t < T; ++t)
    for (int64_t h = 0; h < HKV; ++h)
      for (int64_t d = 0; d < D; ++d) {
        k_cache[(h * max_seq + pos0 + t) * D + d] = k_new[(t * HKV + h) * D + d];
        v_cache[(h * max_seq + pos0 + t) * D + d] = v_new[(t * HKV + h) * D + d];
      }
  float* sc = (float*)malloc((size_t)(pos0 + T) * sizeof(float));
  for (int64_t h = 0; h < H; ++h) {
    const int64_t hk = h / nrep;
    const float* K = k_cache + hk * max_seq * D;
    const float* V = v_cache + hk * max_seq * D;
    for (int64_t t = 0; t < T; ++t) {
      const float* qr = q + (t * H + h) * D;
      const int64_t S = pos0 + t + 1;
      float mx = -1e30f;
      for (int64_t j = 0; j < S; ++j) {
        float dot = 0.0f;
        for (int64_t d = 0; d < D; ++d) dot += qr[d] * K[j * D + d];
        sc[j] = dot * scale;
        if (sc[j] > mx) mx = sc[j];
      }
      float sum = 0.0f;
      for (int64_t j = 0; j < S; ++j) {
        sc[j] = expf(sc[j] - mx);
        sum += sc[j];
      }
      for (int64_t j = 0; j < S; ++j) sc[j] /= sum;
      for (int64_t d = 0; d < D; ++d) {
        float acc = 0.0f;
        for (int64_t j = 0; j < S; ++j) acc += sc[j] * V[j * D + d];
        out[(t * H + h) * D + d] = acc;
      }
    }
  }
  free(sc);
}
