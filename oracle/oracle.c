/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for the jax4j B200 engine. See oracle.h.
 *
 * Reference files are cited by their path inside the jax4j project:
 *   core/ = jax4j-core/src/main/java/com/nablatensor/jax4j/
 * Build: see oracle/Makefile (-O2 -ffp-contract=off, no fast-math: Java float semantics).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------------------------ */
/* PRNG                                                                                        */
/* ------------------------------------------------------------------------------------------ */

/* core/tensor/spi/ComputeBackend.java:290-295 (splitmix64 finaliser). */
uint64_t j4o_mix64(uint64_t v) {
  v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ULL;
  v = (v ^ (v >> 27)) * 0x94D049BB133111EBULL;
  return v ^ (v >> 31);
}

static const uint64_t kGolden = 0x9E3779B97F4A7C15ULL;

/* ComputeBackend.java:282-284: (mix64(seed + phi*counter) >>> 40) * 2^-24 */
static float uniform_at(int64_t seed, int64_t counter) {
  uint64_t m = j4o_mix64((uint64_t)seed + kGolden * (uint64_t)counter);
  return (float)(m >> 40) * 0x1.0p-24f;
}

/* ComputeBackend.java:286-288: ((mix >>> 40) + 1) * 2^-24, the open-at-zero variant. */
static float uniform_open_at(int64_t seed, int64_t counter) {
  uint64_t m = j4o_mix64((uint64_t)seed + kGolden * (uint64_t)counter);
  return (float)((m >> 40) + 1) * 0x1.0p-24f;
}

/* ComputeBackend.java:51-61 */
void j4o_random_uniform(int64_t seed, int64_t counter, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = uniform_at(seed, counter + i);
}

/* ComputeBackend.java:64-76: Box-Muller on counters 2i (open) and 2i+1, evaluated in double. */
void j4o_random_normal(int64_t seed, int64_t counter, int64_t n, float* out) {
  const double kPi = 3.141592653589793;
  for (int64_t i = 0; i < n; i++) {
    float u1 = uniform_open_at(seed, counter + 2 * i);
    float u2 = uniform_at(seed, counter + 2 * i + 1);
    out[i] = (float)(sqrt(-2.0 * log((double)u1)) * cos(2.0 * kPi * (double)u2));
  }
}

/* core/tensor/PrngKey.java:44-56 */
void j4o_prng_split(int64_t seed, int64_t counter, int count, int64_t* seeds_out) {
  for (int i = 0; i < count; i++)
    seeds_out[i] = (int64_t)j4o_mix64((uint64_t)seed + kGolden * (uint64_t)(counter + i + 1));
}

/* ------------------------------------------------------------------------------------------ */
/* half precision                                                                              */
/* ------------------------------------------------------------------------------------------ */

static float bits_to_float(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}

static uint32_t float_to_bits(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}

/* core/backend/cpu/CpuQ4Gemm.java:58-77 */
float j4o_half_to_float(uint32_t bits) {
  uint32_t sign = (bits & 0x8000u) << 16;
  int exponent = (int)((bits >> 10) & 0x1f);
  uint32_t fraction = bits & 0x3ff;
  if (exponent == 0) {
    if (fraction == 0) return bits_to_float(sign);
    exponent = 1;
    while ((fraction & 0x400) == 0) {
      fraction <<= 1;
      exponent--;
    }
    return bits_to_float(sign | ((uint32_t)(exponent + 112) << 23) | ((fraction & 0x3ff) << 13));
  }
  if (exponent == 31) return bits_to_float(sign | 0x7f800000u | (fraction << 13));
  return bits_to_float(sign | ((uint32_t)(exponent + 112) << 23) | (fraction << 13));
}

/* binary32 -> binary16, round to nearest even (IEEE 754 conversion; used by our encoders). */
uint16_t j4o_float_to_half(float f) {
  uint32_t x = float_to_bits(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t absx = x & 0x7fffffffu;
  if (absx > 0x7f800000u) return (uint16_t)(sign | 0x7e00u); /* NaN */
  if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
  int e = (int)(absx >> 23) - 127;
  uint32_t mant = (absx & 0x7fffffu) | 0x800000u;
  if (e < -25) return (uint16_t)sign; /* below half of the smallest subnormal */
  uint32_t shift;
  uint32_t base;
  if (e < -14) { /* subnormal half: value = m * 2^-24 */
    shift = (uint32_t)(-1 - e); /* mant has 23 fraction bits; target unit 2^-24 */
    base = 0;
    uint32_t q = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1))) q++;
    return (uint16_t)(sign | (base + q));
  }
  /* normal: 10 fraction bits kept out of 23 */
  uint32_t q = mant >> 13;
  uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
  uint32_t he = (uint32_t)(e + 15);
  uint32_t h = (he << 10) + (q - 0x400u); /* q may carry into the exponent: still correct */
  return (uint16_t)(sign | h);
}

/* ------------------------------------------------------------------------------------------ */
/* GGUF block codecs                                                                           */
/* ------------------------------------------------------------------------------------------ */

static int block_elems(int type) {
  switch (type) {
    case J4O_Q4_0: return 32;
    case J4O_Q8_0: return 32;
    case J4O_Q4_K: return 256;
    case J4O_Q6_K: return 256;
    case J4O_Q2_0: return 128;
    default: return -1;
  }
}

static int block_bytes(int type) {
  switch (type) {
    case J4O_Q4_0: return 18;
    case J4O_Q8_0: return 34;
    case J4O_Q4_K: return 144;
    case J4O_Q6_K: return 210;
    case J4O_Q2_0: return 34;
    default: return -1;
  }
}

/* QuantType.byteSizeFor (core/tensor/QuantType.java:46-53), per row. */
int64_t j4o_quant_row_bytes(int type, int64_t cols) {
  int be = block_elems(type);
  if (be <= 0 || cols <= 0 || cols % be) return -1;
  return cols / be * block_bytes(type);
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void wr16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xff);
  p[1] = (uint8_t)(v >> 8);
}

/* round half away from zero, as C roundf */
static int round_away(float v) { return (int)roundf(v); }

/* Q8_0 (GGUF type 8): f16 d = max|w|/127, 32 int8 codes, w = d*q.
 * Encoding: q = round-half-away-from-zero(w * (1/d)) clamped to [-127, 127], using the f32 d
 * (before its rounding to f16), as the GGUF reference encoder does. */
static void enc_q8_0(const float* w, uint8_t* blk) {
  float amax = 0.0f;
  for (int i = 0; i < 32; i++) {
    float a = fabsf(w[i]);
    if (a > amax) amax = a;
  }
  float d = amax / 127.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  wr16(blk, j4o_float_to_half(d));
  for (int i = 0; i < 32; i++) {
    int q = round_away(w[i] * id);
    if (q > 127) q = 127;
    if (q < -127) q = -127;
    blk[2 + i] = (uint8_t)(int8_t)q;
  }
}

static float dec_q8_0(const uint8_t* blk, int i) {
  float d = j4o_half_to_float(rd16(blk));
  return d * (float)(int8_t)blk[2 + i];
}

/* Q4_0 (GGUF type 2): CpuQ4Gemm.java:3-8 layout -- f16 d, byte j holds element j (low nibble)
 * and j+16 (high nibble), w = d*(q-8). Encoding (published GGUF method): m = the signed value
 * of largest magnitude, d = m / -8, q = min(15, (int)(w/d + 8.5)). */
static void enc_q4_0(const float* w, uint8_t* blk) {
  float amax = 0.0f, m = 0.0f;
  for (int i = 0; i < 32; i++) {
    if (fabsf(w[i]) > amax) {
      amax = fabsf(w[i]);
      m = w[i];
    }
  }
  float d = m / -8.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  wr16(blk, j4o_float_to_half(d));
  for (int j = 0; j < 16; j++) {
    int q0 = (int)(w[j] * id + 8.5f);
    int q1 = (int)(w[j + 16] * id + 8.5f);
    if (q0 > 15) q0 = 15;
    if (q1 > 15) q1 = 15;
    if (q0 < 0) q0 = 0;
    if (q1 < 0) q1 = 0;
    blk[2 + j] = (uint8_t)(q0 | (q1 << 4));
  }
}

/* CpuQ4Gemm.packedValue (CpuQ4Gemm.java:48-56) */
static float dec_q4_0(const uint8_t* blk, int within) {
  float scale = j4o_half_to_float(rd16(blk));
  int packed = blk[2 + (within % 16)];
  int nibble = within < 16 ? (packed & 0x0f) : ((packed >> 4) & 0x0f);
  return scale * (float)(nibble - 8);
}

/* Q2_0 (prism fork, id 42): CpuQ2Gemm.java:133-140 layout -- f16 d, 32 bytes of 2-bit codes,
 * element 4p+s in bits 2s of byte p, w = d*(code-1). Encoding (ours): d = max|w|,
 * code = clamp(round(w/d), -1, 1) + 1. */
static void enc_q2_0(const float* w, uint8_t* blk) {
  float amax = 0.0f;
  for (int i = 0; i < 128; i++)
    if (fabsf(w[i]) > amax) amax = fabsf(w[i]);
  float d = amax;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  wr16(blk, j4o_float_to_half(d));
  for (int p = 0; p < 32; p++) {
    int byte = 0;
    for (int s = 0; s < 4; s++) {
      int q = round_away(w[4 * p + s] * id);
      if (q > 1) q = 1;
      if (q < -1) q = -1;
      byte |= (q + 1) << (2 * s);
    }
    blk[2 + p] = (uint8_t)byte;
  }
}

/* CpuQ2Gemm.packedValue (CpuQ2Gemm.java:133-140) */
static float dec_q2_0(const uint8_t* blk, int within) {
  float scale = j4o_half_to_float(rd16(blk));
  int packed = blk[2 + within / 4];
  return scale * (float)(((packed >> ((within & 3) * 2)) & 3) - 1);
}

/* Q4_K (GGUF type 12): 256-element super-block = f16 d, f16 dmin, 12 bytes of packed 6-bit
 * (scale, min) pairs for 8 sub-blocks of 32, 128 bytes of 4-bit codes. Sub-block j of chunk
 * c = j/2 uses the low (j even) or high (j odd) nibble of bytes qs[32c .. 32c+31];
 * w = (d*sc_j)*q - dmin*m_j (public GGUF layout). */
static void q4k_get_scale_min(int j, const uint8_t* q, int* sc, int* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

/* Encoding (ours, single pass): per sub-block lo = min(0, min w), hi = max w;
 * scale_j = (hi - lo)/15, min_j = -lo; d = max scale_j / 63, dmin = max min_j / 63 (f16);
 * sc_j = round(scale_j / d), m_j = round(min_j / dmin) in [0, 63];
 * q = clamp(round((w + dmin*m_j) / (d*sc_j)), 0, 15). All arithmetic in float. */
static void enc_q4_k(const float* w, uint8_t* blk) {
  float scale[8], mins[8];
  float max_scale = 0.0f, max_min = 0.0f;
  for (int j = 0; j < 8; j++) {
    float lo = 0.0f, hi = w[32 * j];
    for (int i = 0; i < 32; i++) {
      float v = w[32 * j + i];
      if (v < lo) lo = v;
      if (v > hi) hi = v;
    }
    if (hi < 0.0f) hi = 0.0f;
    scale[j] = (hi - lo) / 15.0f;
    mins[j] = -lo;
    if (scale[j] > max_scale) max_scale = scale[j];
    if (mins[j] > max_min) max_min = mins[j];
  }
  uint16_t dh = j4o_float_to_half(max_scale / 63.0f);
  uint16_t mh = j4o_float_to_half(max_min / 63.0f);
  float d = j4o_half_to_float(dh);
  float dmin = j4o_half_to_float(mh);
  int sc[8], m[8];
  for (int j = 0; j < 8; j++) {
    int s = d > 0.0f ? round_away(scale[j] / d) : 0;
    int mm = dmin > 0.0f ? round_away(mins[j] / dmin) : 0;
    sc[j] = s < 0 ? 0 : (s > 63 ? 63 : s);
    m[j] = mm < 0 ? 0 : (mm > 63 ? 63 : mm);
  }
  wr16(blk, dh);
  wr16(blk + 2, mh);
  uint8_t* sb = blk + 4;
  for (int j = 0; j < 4; j++) {
    sb[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    sb[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
    sb[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
  }
  uint8_t* qs = blk + 16;
  for (int c = 0; c < 4; c++) {
    for (int l = 0; l < 32; l++) {
      int q[2];
      for (int h = 0; h < 2; h++) {
        int j = 2 * c + h;
        float ds = d * (float)sc[j];
        float v = w[64 * c + 32 * h + l] + dmin * (float)m[j];
        int qq = ds > 0.0f ? round_away(v / ds) : 0;
        q[h] = qq < 0 ? 0 : (qq > 15 ? 15 : qq);
      }
      qs[32 * c + l] = (uint8_t)(q[0] | (q[1] << 4));
    }
  }
}

/* Dequantisation of one Q4_K element, in the order d1 = d*sc, m1 = dmin*m, w = d1*q - m1. */
static float dec_q4_k(const uint8_t* blk, int within) {
  float d = j4o_half_to_float(rd16(blk));
  float dmin = j4o_half_to_float(rd16(blk + 2));
  int c = within / 64, h = (within % 64) / 32, l = within % 32;
  int j = 2 * c + h;
  int sc, m;
  q4k_get_scale_min(j, blk + 4, &sc, &m);
  float d1 = d * (float)sc;
  float m1 = dmin * (float)m;
  int byte = blk[16 + 32 * c + l];
  int q = h ? (byte >> 4) : (byte & 0xF);
  return d1 * (float)q - m1;
}

/* Q6_K (GGUF type 14, QuantType.java:10 geometry only): 256-element super-block = ql[128] low
 * nibbles, qh[64] high 2-bit pairs, scales[16] int8 (one per 16 elements), f16 d (public GGUF
 * layout). Element l + 32 s of half n (l < 32, s < 4): ql byte 64 n + l + 32 (s & 1), low
 * nibble for s < 2 and high for s >= 2; qh byte 32 n + l, bits 2 s .. 2 s + 1; scale 8 n + l/16
 * + 2 s; code q = nibble | high << 4 in [0, 63]; w = (d * sc) * (q - 32), in that order.
 * Encoding (ours, single pass): per 16 elements s_j = max|w| / 31 (signed by the largest
 * magnitude); d = max |s_j| / 127 (f16); sc_j = round(s_j / d) in [-127, 127];
 * q = clamp(round(w / (d sc_j)), -32, 31) + 32. All arithmetic in float. */
static void enc_q6_k(const float* w, uint8_t* blk) {
  float sub[16], max_abs = 0.0f;
  for (int j = 0; j < 16; j++) {
    float best = 0.0f;
    for (int i = 0; i < 16; i++) {
      float v = w[16 * j + i];
      if (fabsf(v) > fabsf(best)) best = v;
    }
    sub[j] = best / 31.0f;
    if (fabsf(sub[j]) > max_abs) max_abs = fabsf(sub[j]);
  }
  uint16_t dh = j4o_float_to_half(max_abs / 127.0f);
  float d = j4o_half_to_float(dh);
  int8_t sc[16];
  for (int j = 0; j < 16; j++) {
    int v = d > 0.0f ? round_away(sub[j] / d) : 0;
    sc[j] = (int8_t)(v < -127 ? -127 : (v > 127 ? 127 : v));
  }
  uint8_t* ql = blk;
  uint8_t* qh = blk + 128;
  int8_t* scales = (int8_t*)(blk + 192);
  memset(blk, 0, 192);
  for (int j = 0; j < 16; j++) scales[j] = sc[j];
  wr16(blk + 208, dh);
  for (int e = 0; e < 256; e++) {
    int n = e / 128, r = e % 128, s = r / 32, l = r % 32;
    float ds = d * (float)sc[16 * 0 + (e / 16)];
    int q = ds != 0.0f ? round_away(w[e] / ds) : 0;
    q = (q < -32 ? -32 : (q > 31 ? 31 : q)) + 32;
    int qlb = 64 * n + l + 32 * (s & 1);
    ql[qlb] |= (uint8_t)((q & 0xF) << (s >= 2 ? 4 : 0));
    qh[32 * n + l] |= (uint8_t)(((q >> 4) & 3) << (2 * s));
  }
}

static float dec_q6_k(const uint8_t* blk, int within) {
  float d = j4o_half_to_float(rd16(blk + 208));
  int n = within / 128, r = within % 128, s = r / 32, l = r % 32;
  int qlb = blk[64 * n + l + 32 * (s & 1)];
  int nib = s >= 2 ? (qlb >> 4) : (qlb & 0xF);
  int hi = (blk[128 + 32 * n + l] >> (2 * s)) & 3;
  int q = (nib | (hi << 4)) - 32;
  int sc = (int)((const int8_t*)(blk + 192))[8 * n + l / 16 + 2 * s];
  return (d * (float)sc) * (float)q;
}

int j4o_quantize(int type, const float* w, int64_t rows, int64_t cols, uint8_t* out) {
  int64_t rb = j4o_quant_row_bytes(type, cols);
  if (rb < 0 || rows <= 0) return -1;
  int be = block_elems(type), bb = block_bytes(type);
  for (int64_t r = 0; r < rows; r++) {
    for (int64_t b = 0; b < cols / be; b++) {
      const float* src = w + r * cols + b * be;
      uint8_t* dst = out + r * rb + b * bb;
      switch (type) {
        case J4O_Q8_0: enc_q8_0(src, dst); break;
        case J4O_Q4_0: enc_q4_0(src, dst); break;
        case J4O_Q4_K: enc_q4_k(src, dst); break;
        case J4O_Q6_K: enc_q6_k(src, dst); break;
        case J4O_Q2_0: enc_q2_0(src, dst); break;
        default: return -1;
      }
    }
  }
  return 0;
}

static float dec_elem(int type, const uint8_t* row, int64_t idx) {
  int be = block_elems(type), bb = block_bytes(type);
  const uint8_t* blk = row + (idx / be) * bb;
  int within = (int)(idx % be);
  switch (type) {
    case J4O_Q8_0: return dec_q8_0(blk, within);
    case J4O_Q4_0: return dec_q4_0(blk, within);
    case J4O_Q4_K: return dec_q4_k(blk, within);
    case J4O_Q6_K: return dec_q6_k(blk, within);
    case J4O_Q2_0: return dec_q2_0(blk, within);
  }
  return NAN;
}

/* quantGatherRow: CpuBackend.java:738-755 -> CpuQ4Gemm.gather (CpuQ4Gemm.java:17-24). */
int j4o_gather_row(int type, const uint8_t* blob, int64_t rows, int64_t cols, int64_t row,
                   float* out) {
  int64_t rb = j4o_quant_row_bytes(type, cols);
  if (rb < 0 || rows <= 0 || row < 0 || row >= rows) return -1;
  const uint8_t* r = blob + row * rb;
  for (int64_t i = 0; i < cols; i++) out[i] = dec_elem(type, r, i);
  return 0;
}

/* Q4_0 multiply: CpuQ4Gemm.java:26-46, accumulation order kept exactly:
 *   sum += scale*(low-8)*x[i]; sum += scale*(high-8)*x[i+16]; */
static void mv_q4_0(const uint8_t* w, const float* x, int64_t rows, int64_t cols, float* y) {
  int64_t blocks = cols / 32;
  for (int64_t row = 0; row < rows; row++) {
    float sum = 0.0f;
    const uint8_t* ro = w + row * blocks * 18;
    for (int64_t b = 0; b < blocks; b++) {
      const uint8_t* bo = ro + b * 18;
      float scale = j4o_half_to_float(rd16(bo));
      const float* xi = x + b * 32;
      for (int p = 0; p < 16; p++) {
        int packed = bo[2 + p];
        int low = packed & 0x0f, high = (packed >> 4) & 0x0f;
        sum += scale * (float)(low - 8) * xi[p];
        sum += scale * (float)(high - 8) * xi[p + 16];
      }
    }
    y[row] = sum;
  }
}

/* Q2_0 multiply: CpuQ2Gemm.java:26-47, order kept. */
static void mv_q2_0(const uint8_t* w, const float* x, int64_t rows, int64_t cols, float* y) {
  int64_t blocks = cols / 128;
  for (int64_t row = 0; row < rows; row++) {
    float sum = 0.0f;
    const uint8_t* ro = w + row * blocks * 34;
    for (int64_t b = 0; b < blocks; b++) {
      const uint8_t* bo = ro + b * 34;
      float scale = j4o_half_to_float(rd16(bo));
      const float* xi = x + b * 128;
      for (int p = 0; p < 32; p++) {
        int packed = bo[2 + p];
        int idx = p << 2;
        sum += scale * (float)((packed & 3) - 1) * xi[idx];
        sum += scale * (float)(((packed >> 2) & 3) - 1) * xi[idx + 1];
        sum += scale * (float)(((packed >> 4) & 3) - 1) * xi[idx + 2];
        sum += scale * (float)(((packed >> 6) & 3) - 1) * xi[idx + 3];
      }
    }
    y[row] = sum;
  }
}

/* Q8_0 / Q4_K / Q6_K multiply: no reference implementation exists. Same style as CpuQ4Gemm: one float
 * accumulator per row, elements in index order, sum += w_dequant * x. */
static void mv_generic(int type, const uint8_t* w, const float* x, int64_t rows, int64_t cols,
                       float* y) {
  int64_t rb = j4o_quant_row_bytes(type, cols);
  for (int64_t row = 0; row < rows; row++) {
    const uint8_t* ro = w + row * rb;
    float sum = 0.0f;
    for (int64_t i = 0; i < cols; i++) sum += dec_elem(type, ro, i) * x[i];
    y[row] = sum;
  }
}

int j4o_quant_matvec(int type, const uint8_t* blob, int64_t rows, int64_t cols,
                     const float* x, int64_t batch, float* y) {
  if (j4o_quant_row_bytes(type, cols) < 0 || rows <= 0 || batch <= 0) return -1;
  for (int64_t b = 0; b < batch; b++) {
    const float* xb = x + b * cols;
    float* yb = y + b * rows;
    switch (type) {
      case J4O_Q4_0: mv_q4_0(blob, xb, rows, cols, yb); break;
      case J4O_Q2_0: mv_q2_0(blob, xb, rows, cols, yb); break;
      case J4O_Q8_0:
      case J4O_Q4_K:
      case J4O_Q6_K: mv_generic(type, blob, xb, rows, cols, yb); break;
      default: return -1;
    }
  }
  return 0;
}

int j4o_quant_matvec_f64(int type, const uint8_t* blob, int64_t rows, int64_t cols,
                         const float* x, int64_t batch, double* y) {
  int64_t rb = j4o_quant_row_bytes(type, cols);
  if (rb < 0 || rows <= 0 || batch <= 0) return -1;
  float* wrow = (float*)malloc((size_t)cols * sizeof(float));
  if (!wrow) return -1;
  for (int64_t r = 0; r < rows; r++) {
    for (int64_t i = 0; i < cols; i++) wrow[i] = dec_elem(type, blob + r * rb, i);
    for (int64_t b = 0; b < batch; b++) {
      double acc = 0.0;
      const float* xb = x + b * cols;
      for (int64_t i = 0; i < cols; i++) acc += (double)wrow[i] * (double)xb[i];
      y[b * rows + r] = acc;
    }
  }
  free(wrow);
  return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* CpuBackend primitives                                                                       */
/* ------------------------------------------------------------------------------------------ */

/* java.lang.Math.max(float, float): NaN if either is NaN, +0.0 > -0.0. */
static float java_max(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == 0.0f && b == 0.0f) return signbit(a) ? b : a;
  return a >= b ? a : b;
}

/* java.lang.Math.min(float, float): NaN if either is NaN, -0.0 < +0.0. */
static float java_min(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == 0.0f && b == 0.0f) return signbit(a) ? a : b;
  return a <= b ? a : b;
}

/* CpuBackend.applyBinary (CpuBackend.java:657-667) */
float j4o_apply_binary(int op, float x, float y) {
  switch (op) {
    case J4O_ADD: return x + y;
    case J4O_SUB: return x - y;
    case J4O_MUL: return x * y;
    case J4O_DIV: return x / y;
    case J4O_MAX: return java_max(x, y);
    case J4O_MIN: return java_min(x, y);
  }
  return NAN;
}

/* CpuBackend.unary (CpuBackend.java:127-167): transcendental math in double, cast to float. */
float j4o_apply_unary(int op, float x) {
  switch (op) {
    case J4O_NEG: return -x;
    case J4O_EXP: return (float)exp((double)x);
    case J4O_LOG: return (float)log((double)x);
    case J4O_SQRT: return (float)sqrt((double)x);
    case J4O_RSQRT: return (float)(1.0 / sqrt((double)x));
    case J4O_TANH: return (float)tanh((double)x);
    case J4O_SIGMOID: return (float)(1.0 / (1.0 + exp(-(double)x)));
    case J4O_RELU: return java_max(0.0f, x);
    case J4O_ABS: return fabsf(x);
    case J4O_SIGN: return x > 0 ? 1.0f : (x < 0 ? -1.0f : 0.0f);
  }
  return NAN;
}

/* CpuBackend.binary (CpuBackend.java:61-94) */
void j4o_binary(int op, const float* a, const float* b, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = j4o_apply_binary(op, a[i], b[i]);
}

/* CpuBackend.scalar (CpuBackend.java:96-124): the double operand is cast to float first. */
void j4o_scalar(int op, const float* a, double value, int64_t n, float* out) {
  float s = (float)value;
  for (int64_t i = 0; i < n; i++) out[i] = j4o_apply_binary(op, a[i], s);
}

void j4o_unary(int op, const float* a, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = j4o_apply_unary(op, a[i]);
}

/* CpuBackend.transpose (CpuBackend.java:169-186) */
void j4o_transpose(const float* a, int64_t rows, int64_t cols, float* out) {
  for (int64_t r = 0; r < rows; r++)
    for (int64_t c = 0; c < cols; c++) out[c * rows + r] = a[r * cols + c];
}

/* CpuBackend.matmul (CpuBackend.java:188-216): i-p-j loop, float accumulation. */
void j4o_matmul(const float* a, const float* b, int64_t m, int64_t k, int64_t n, float* out) {
  memset(out, 0, (size_t)(m * n) * sizeof(float));
  for (int64_t i = 0; i < m; i++)
    for (int64_t p = 0; p < k; p++) {
      float xip = a[i * k + p];
      const float* yr = b + p * n;
      float* orow = out + i * n;
      for (int64_t j = 0; j < n; j++) orow[j] += xip * yr[j];
    }
}

/* CpuBackend.batchedMatmul (CpuBackend.java:218-248) */
void j4o_batched_matmul(const float* a, const float* b, int64_t batch, int64_t m, int64_t k,
                        int64_t n, float* out) {
  for (int64_t bi = 0; bi < batch; bi++)
    j4o_matmul(a + bi * m * k, b + bi * k * n, m, k, n, out + bi * m * n);
}

/* CpuBackend.reduceSum (CpuBackend.java:264-272): double accumulator. */
float j4o_reduce_sum(const float* a, int64_t n) {
  double acc = 0;
  for (int64_t i = 0; i < n; i++) acc += a[i];
  return (float)acc;
}

/* CpuBackend.reduceMax (CpuBackend.java:274-284): strict '>' -- NaN is skipped. */
float j4o_reduce_max(const float* a, int64_t n) {
  float m = -INFINITY;
  for (int64_t i = 0; i < n; i++)
    if (a[i] > m) m = a[i];
  return m;
}

/* CpuBackend.sumAxis (CpuBackend.java:295-311): double accumulator per output. */
void j4o_sum_axis(const float* a, int64_t outer, int64_t axis, int64_t inner, float* out) {
  for (int64_t o = 0; o < outer; o++)
    for (int64_t in = 0; in < inner; in++) {
      double total = 0;
      int64_t base = o * axis * inner + in;
      for (int64_t i = 0; i < axis; i++) total += a[base + i * inner];
      out[o * inner + in] = (float)total;
    }
}

/* CpuBackend.maxAxis (CpuBackend.java:313-329): Math.max, so NaN propagates. */
void j4o_max_axis(const float* a, int64_t outer, int64_t axis, int64_t inner, float* out) {
  for (int64_t o = 0; o < outer; o++)
    for (int64_t in = 0; in < inner; in++) {
      float best = -INFINITY;
      int64_t base = o * axis * inner + in;
      for (int64_t i = 0; i < axis; i++) best = java_max(best, a[base + i * inner]);
      out[o * inner + in] = best;
    }
}

/* CpuBackend.argMaxAxis (CpuBackend.java:331-355): first NaN wins, else first maximum. */
void j4o_argmax_axis(const float* a, int64_t outer, int64_t axis, int64_t inner, float* out) {
  for (int64_t o = 0; o < outer; o++)
    for (int64_t in = 0; in < inner; in++) {
      float best = -INFINITY;
      int64_t bi = 0;
      int64_t base = o * axis * inner + in;
      for (int64_t i = 0; i < axis; i++) {
        float v = a[base + i * inner];
        if (v != v) {
          bi = i;
          break;
        } else if (v > best) {
          best = v;
          bi = i;
        }
      }
      out[o * inner + in] = (float)bi;
    }
}

/* CpuBackend.maxAxisBackward (CpuBackend.java:357-391) */
void j4o_max_axis_backward(const float* up, const float* in, int64_t outer, int64_t axis,
                           int64_t inner, float* out) {
  memset(out, 0, (size_t)(outer * axis * inner) * sizeof(float));
  for (int64_t o = 0; o < outer; o++)
    for (int64_t n = 0; n < inner; n++) {
      int64_t base = o * axis * inner + n;
      int64_t bi = 0;
      float best = -INFINITY;
      for (int64_t i = 0; i < axis; i++) {
        float v = in[base + i * inner];
        if (v != v || v > best) {
          best = v;
          bi = i;
          if (v != v) break;
        }
      }
      out[base + bi * inner] = up[o * inner + n];
    }
}

/* CpuBackend.broadcastTo (CpuBackend.java:401-447) */
void j4o_broadcast_to(const float* a, const int64_t* src_dims, int src_rank,
                      const int64_t* dst_dims, int dst_rank, float* out) {
  int64_t sd[16], ss[16], ts[16];
  int pad = dst_rank - src_rank;
  for (int i = 0; i < dst_rank; i++) sd[i] = i < pad ? 1 : src_dims[i - pad];
  int64_t stride = 1;
  for (int i = dst_rank - 1; i >= 0; i--) {
    ss[i] = sd[i] == 1 ? 0 : stride;
    stride *= sd[i];
  }
  int64_t s = 1;
  for (int i = dst_rank - 1; i >= 0; i--) {
    ts[i] = s;
    s *= dst_dims[i];
  }
  for (int64_t lin = 0; lin < s; lin++) {
    int64_t rem = lin, off = 0;
    for (int d = 0; d < dst_rank; d++) {
      int64_t coord = rem / ts[d];
      rem = rem % ts[d];
      off += coord * ss[d];
    }
    out[lin] = a[off];
  }
}

/* ComputeBackend.reindex default (ComputeBackend.java:247-259) */
int j4o_reindex(const float* a, int64_t n_src, const int32_t* map, int64_t n_dst, float* out) {
  for (int64_t i = 0; i < n_dst; i++) {
    if (map[i] < -1 || map[i] >= n_src) return -1;
    out[i] = map[i] >= 0 ? a[map[i]] : 0.0f;
  }
  return 0;
}

/* ComputeBackend.scatterAdd default (ComputeBackend.java:261-274): float accumulation in
 * source order. */
int j4o_scatter_add(const float* a, int64_t n_src, const int32_t* map, int64_t n_dst,
                    float* out) {
  memset(out, 0, (size_t)n_dst * sizeof(float));
  for (int64_t i = 0; i < n_src; i++) {
    if (map[i] < -1 || map[i] >= n_dst) return -1;
    if (map[i] >= 0) out[map[i]] += a[i];
  }
  return 0;
}

/* CpuBackend.reluBackward (CpuBackend.java:608-619) */
void j4o_relu_backward(const float* up, const float* in, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = in[i] > 0.0f ? up[i] : 0.0f;
}

/* CpuBackend.fused / evalFused (CpuBackend.java:628-655), as a postfix program. The reference
 * CPU applyUnary omits SIGN (CpuBackend.java:669-682); the CUDA fused kernel and CpuBackend.unary
 * both define it, and the oracle uses that definition. */
int j4o_fused(const int32_t* prog, int prog_len, const float* const* inputs, int n_inputs,
              int64_t n, float* out) {
  float stack[256];
  for (int64_t e = 0; e < n; e++) {
    int sp = 0;
    for (int pc = 0; pc < prog_len;) {
      int kind = prog[pc];
      if (kind == 0) {
        int idx = prog[pc + 1];
        if (idx < 0 || idx >= n_inputs || sp >= 256) return -1;
        stack[sp++] = inputs[idx][e];
        pc += 2;
      } else if (kind == 1) {
        if (sp < 1) return -1;
        stack[sp - 1] = j4o_apply_unary(prog[pc + 1], stack[sp - 1]);
        pc += 2;
      } else if (kind == 2) {
        if (sp < 2) return -1;
        float r = stack[--sp];
        stack[sp - 1] = j4o_apply_binary(prog[pc + 1], stack[sp - 1], r);
        pc += 2;
      } else if (kind == 3) {
        if (sp < 1) return -1;
        uint64_t bits = (uint64_t)(uint32_t)prog[pc + 2] | ((uint64_t)(uint32_t)prog[pc + 3] << 32);
        double v;
        memcpy(&v, &bits, 8);
        stack[sp - 1] = j4o_apply_binary(prog[pc + 1], stack[sp - 1], (float)v);
        pc += 4;
      } else {
        return -1;
      }
    }
    if (sp != 1) return -1;
    out[e] = stack[0];
  }
  return 0;
}

/* ------------------------------------------------------------------------------------------
 * Scalar-AAD replay (test infrastructure): the CPU engine's Monte-Carlo replay of a recorded
 * scalar tape, one scenario at a time, forward then reverse, in double precision.
 *
 * Philox2x32-10 keyed on the scenario: core/engine/cpu/Philox.java:30-94. lo = (int) path ^
 * (int) seed, hi = (int) (path >>> 32) ^ (int) (seed >>> 32), stream s != 0 folds s *
 * 0x9E3779B1 into hi. normal(): Philox of (lo, hi ^ counter++) -> Box-Muller pair, cosine leg
 * returned first and the sine leg on the next call; uniform(): counter (ucounter++ | 0x40000000).
 * Replay: core/engine/cpu/ScalarReplay.java:145-232 (forward switch, adjoint switch with the
 * active-node skip, per-output value / value^2 / gradient sums); active flags as
 * core/engine/AadTape.java:61-74. Op codes are AadOp ordinals (core/engine/AadOp.java:22-37).
 * ------------------------------------------------------------------------------------------ */
enum { AAD_CONST, AAD_INPUT, AAD_RANDN, AAD_RANDU, AAD_ADD, AAD_SUB, AAD_MUL, AAD_DIV, AAD_NEG,
       AAD_EXP, AAD_LOG, AAD_SQRT, AAD_MAX, AAD_MIN, AAD_ABS };

typedef struct {
  uint32_t lo, hi, counter, ucounter;
  double spare;
  int has;
} philox_t;

static void philox_rounds_key(uint32_t* c0, uint32_t* c1, uint32_t key) {
  for (int i = 0; i < 10; i++) {
    uint64_t product = (uint64_t)0xD256D193u * (uint64_t)*c0;
    uint32_t high = (uint32_t)(product >> 32), low = (uint32_t)product;
    *c0 = high ^ key ^ *c1;
    *c1 = low;
    key += 0x9E3779B9u;
  }
}
/* The replay's generator always starts from key 0x1BD11BDA (Philox.java:56). */
static void philox_rounds(uint32_t* c0, uint32_t* c1) { philox_rounds_key(c0, c1, 0x1BD11BDAu); }

static void philox_init(philox_t* g, int64_t path, int64_t seed, int stream) {
  g->lo = (uint32_t)path ^ (uint32_t)seed;
  g->hi = (uint32_t)((uint64_t)path >> 32) ^ (uint32_t)((uint64_t)seed >> 32);
  if (stream != 0) g->hi ^= (uint32_t)stream * 0x9E3779B1u;
  g->counter = g->ucounter = 0;
  g->has = 0;
  g->spare = 0.0;
}

static const double kUintScale = 2.3283064365386963e-10;

static double philox_normal(philox_t* g) {
  if (g->has) {
    g->has = 0;
    return g->spare;
  }
  uint32_t c0 = g->lo, c1 = g->hi ^ g->counter++;
  philox_rounds(&c0, &c1);
  double u1 = ((double)c0 + 0.5) * kUintScale;
  double u2 = ((double)c1 + 0.5) * kUintScale;
  double radius = sqrt(-2.0 * log(u1));
  double angle = 6.283185307179586 * u2;
  g->spare = radius * sin(angle);
  g->has = 1;
  return radius * cos(angle);
}

static double philox_uniform(philox_t* g) {
  uint32_t c0 = g->lo, c1 = g->hi ^ (g->ucounter++ | 0x40000000u);
  philox_rounds(&c0, &c1);
  return ((double)c0 + 0.5) * kUintScale;
}

/* java.lang.Math.max / min on doubles: NaN if either is NaN; +0.0 above -0.0. */
static double java_max_d(double a, double b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == 0.0 && b == 0.0) return signbit(a) ? b : a;
  return a >= b ? a : b;
}
static double java_min_d(double a, double b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == 0.0 && b == 0.0) return signbit(a) ? a : b;
  return a <= b ? a : b;
}

int j4o_aad_replay(int n, const int32_t* op, const int32_t* arg_a, const int32_t* arg_b,
                   const double* constant, const double* inputs, int n_in, const int32_t* in_nodes,
                   int n_out, const int32_t* out_nodes, int n_streams, int adjoints, int64_t path_from,
                   int64_t count, int64_t seed, double* value, double* sumsq, double* grad) {
  if (n <= 0 || n_out <= 0 || n_streams <= 0) return -1;
  double* v = (double*)calloc((size_t)n, sizeof(double));
  double* d = (double*)calloc((size_t)n, sizeof(double));
  unsigned char* active = (unsigned char*)calloc((size_t)n, 1);
  philox_t* rng = (philox_t*)calloc((size_t)n_streams, sizeof(philox_t));
  if (!v || !d || !active || !rng) {
    free(v); free(d); free(active); free(rng);
    return -2;
  }
  for (int i = 0; i < n; i++) {
    switch (op[i]) {
      case AAD_INPUT: active[i] = 1; break;
      case AAD_CONST: case AAD_RANDN: case AAD_RANDU: active[i] = 0; break;
      case AAD_NEG: case AAD_EXP: case AAD_LOG: case AAD_SQRT: case AAD_ABS: active[i] = active[arg_a[i]]; break;
      default: active[i] = active[arg_a[i]] || active[arg_b[i]];
    }
  }
  for (int o = 0; o < n_out; o++) {
    value[o] = 0.0;
    sumsq[o] = 0.0;
    for (int j = 0; j < n_in; j++) grad[o * n_in + j] = 0.0;
  }
  for (int64_t path = path_from; path < path_from + count; path++) {
    for (int s = 0; s < n_streams; s++) philox_init(&rng[s], path, seed, s);
    for (int i = 0; i < n; i++) {
      const int a = arg_a[i], b = arg_b[i];
      double r = 0.0;
      switch (op[i]) {
        case AAD_CONST: r = constant[i]; break;
        case AAD_INPUT: r = inputs[a]; break;
        case AAD_RANDN: r = philox_normal(&rng[b]); break;
        case AAD_RANDU: r = philox_uniform(&rng[b]); break;
        case AAD_ADD: r = v[a] + v[b]; break;
        case AAD_SUB: r = v[a] - v[b]; break;
        case AAD_MUL: r = v[a] * v[b]; break;
        case AAD_DIV: r = v[a] / v[b]; break;
        case AAD_NEG: r = -v[a]; break;
        case AAD_EXP: r = exp(v[a]); break;
        case AAD_LOG: r = log(v[a]); break;
        case AAD_SQRT: r = sqrt(v[a]); break;
        case AAD_ABS: r = fabs(v[a]); break;
        case AAD_MAX: r = java_max_d(v[a], v[b]); break;
        case AAD_MIN: r = java_min_d(v[a], v[b]); break;
      }
      v[i] = r;
    }
    for (int o = 0; o < n_out; o++) {
      const double y = v[out_nodes[o]];
      value[o] += y;
      sumsq[o] += y * y;
    }
    if (!adjoints) continue;
    for (int o = 0; o < n_out; o++) {
      memset(d, 0, (size_t)n * sizeof(double));
      d[out_nodes[o]] = 1.0;
      for (int i = n - 1; i >= 0; i--) {
        const double adj = d[i];
        if (adj == 0.0 || !active[i]) continue;
        const int a = arg_a[i], b = arg_b[i];
        switch (op[i]) {
          case AAD_ADD: d[a] += adj; d[b] += adj; break;
          case AAD_SUB: d[a] += adj; d[b] -= adj; break;
          case AAD_MUL: d[a] += adj * v[b]; d[b] += adj * v[a]; break;
          case AAD_DIV: d[a] += adj / v[b]; d[b] -= adj * v[i] / v[b]; break;
          case AAD_NEG: d[a] -= adj; break;
          case AAD_EXP: d[a] += adj * v[i]; break;
          case AAD_LOG: d[a] += adj / v[a]; break;
          case AAD_SQRT: d[a] += adj * 0.5 / v[i]; break;
          case AAD_ABS: d[a] += v[a] < 0.0 ? -adj : adj; break;
          case AAD_MAX: if (v[a] >= v[b]) d[a] += adj; else d[b] += adj; break;
          case AAD_MIN: if (v[a] <= v[b]) d[a] += adj; else d[b] += adj; break;
          default: break;
        }
      }
      for (int j = 0; j < n_in; j++) grad[o * n_in + j] += d[in_nodes[j]];
    }
  }
  free(v); free(d); free(active); free(rng);
  return 0;
}

/* One Philox2x32-10 block (10 rounds on counter (c0, c1) from `key`), exposed for known-answer
 * checks against the published Random123 vectors. */
void j4o_philox2x32_10(uint32_t c0, uint32_t c1, uint32_t key, uint32_t* out0, uint32_t* out1) {
  philox_rounds_key(&c0, &c1, key);
  *out0 = c0;
  *out1 = c1;
}

/* ------------------------------------------------------------------------------------------
 * conv2d, conv2dGradInput, conv2dGradWeight: CpuBackend.java:479-609, float accumulation in the
 * same loop order (image, out channel, output row, output column, in channel, kernel row, kernel
 * column), taps in the zero padding skipped, zero upstream elements skipped in the gradients.
 * ------------------------------------------------------------------------------------------ */
typedef struct { int C, H, W, O, k, s, pad, OH, OW; } conv_geom;

static int conv_geometry(int in_c, int in_h, int in_w, int out_c, int kernel, int stride, int pad, conv_geom* g) {
  if (in_c < 1 || in_h < 1 || in_w < 1 || out_c < 1 || kernel < 1 || stride < 1 || pad < 0) return -1;
  if (in_h + 2 * pad < kernel || in_w + 2 * pad < kernel) return -1;
  g->C = in_c; g->H = in_h; g->W = in_w; g->O = out_c; g->k = kernel; g->s = stride; g->pad = pad;
  g->OH = (in_h + 2 * pad - kernel) / stride + 1;
  g->OW = (in_w + 2 * pad - kernel) / stride + 1;
  return 0;
}

int j4o_conv2d(const float* x, const float* w, int64_t batch, int in_c, int in_h, int in_w, int out_c, int kernel,
               int stride, int pad, float* out) {
  conv_geom g;
  if (conv_geometry(in_c, in_h, in_w, out_c, kernel, stride, pad, &g)) return -1;
  const int64_t isz = (int64_t)g.C * g.H * g.W, osz = (int64_t)g.O * g.OH * g.OW, wsz = (int64_t)g.C * g.k * g.k;
  for (int64_t b = 0; b < batch; b++)
    for (int oc = 0; oc < g.O; oc++)
      for (int oh = 0; oh < g.OH; oh++)
        for (int ow = 0; ow < g.OW; ow++) {
          float acc = 0.0f;
          for (int ic = 0; ic < g.C; ic++)
            for (int kh = 0; kh < g.k; kh++) {
              const int ih = oh * g.s - g.pad + kh;
              if (ih < 0 || ih >= g.H) continue;
              for (int kw = 0; kw < g.k; kw++) {
                const int iw = ow * g.s - g.pad + kw;
                if (iw < 0 || iw >= g.W) continue;
                acc += x[b * isz + ((int64_t)ic * g.H + ih) * g.W + iw] * w[oc * wsz + ((int64_t)ic * g.k + kh) * g.k + kw];
              }
            }
          out[b * osz + ((int64_t)oc * g.OH + oh) * g.OW + ow] = acc;
        }
  return 0;
}

int j4o_conv2d_grad_input(const float* up, const float* w, int64_t batch, int in_c, int in_h, int in_w, int out_c,
                          int kernel, int stride, int pad, float* dx) {
  conv_geom g;
  if (conv_geometry(in_c, in_h, in_w, out_c, kernel, stride, pad, &g)) return -1;
  const int64_t isz = (int64_t)g.C * g.H * g.W, osz = (int64_t)g.O * g.OH * g.OW, wsz = (int64_t)g.C * g.k * g.k;
  memset(dx, 0, (size_t)(batch * isz) * sizeof(float));
  for (int64_t b = 0; b < batch; b++)
    for (int oc = 0; oc < g.O; oc++)
      for (int oh = 0; oh < g.OH; oh++)
        for (int ow = 0; ow < g.OW; ow++) {
          const float gv = up[b * osz + ((int64_t)oc * g.OH + oh) * g.OW + ow];
          if (gv == 0.0f) continue;
          for (int ic = 0; ic < g.C; ic++)
            for (int kh = 0; kh < g.k; kh++) {
              const int ih = oh * g.s - g.pad + kh;
              if (ih < 0 || ih >= g.H) continue;
              for (int kw = 0; kw < g.k; kw++) {
                const int iw = ow * g.s - g.pad + kw;
                if (iw < 0 || iw >= g.W) continue;
                dx[b * isz + ((int64_t)ic * g.H + ih) * g.W + iw] += gv * w[oc * wsz + ((int64_t)ic * g.k + kh) * g.k + kw];
              }
            }
        }
  return 0;
}

int j4o_conv2d_grad_weight(const float* x, const float* up, int64_t batch, int in_c, int in_h, int in_w, int out_c,
                           int kernel, int stride, int pad, float* dw) {
  conv_geom g;
  if (conv_geometry(in_c, in_h, in_w, out_c, kernel, stride, pad, &g)) return -1;
  const int64_t isz = (int64_t)g.C * g.H * g.W, osz = (int64_t)g.O * g.OH * g.OW, wsz = (int64_t)g.C * g.k * g.k;
  memset(dw, 0, (size_t)(g.O * wsz) * sizeof(float));
  for (int64_t b = 0; b < batch; b++)
    for (int oc = 0; oc < g.O; oc++)
      for (int oh = 0; oh < g.OH; oh++)
        for (int ow = 0; ow < g.OW; ow++) {
          const float gv = up[b * osz + ((int64_t)oc * g.OH + oh) * g.OW + ow];
          if (gv == 0.0f) continue;
          for (int ic = 0; ic < g.C; ic++)
            for (int kh = 0; kh < g.k; kh++) {
              const int ih = oh * g.s - g.pad + kh;
              if (ih < 0 || ih >= g.H) continue;
              for (int kw = 0; kw < g.k; kw++) {
                const int iw = ow * g.s - g.pad + kw;
                if (iw < 0 || iw >= g.W) continue;
                dw[oc * wsz + ((int64_t)ic * g.k + kh) * g.k + kw] += gv * x[b * isz + ((int64_t)ic * g.H + ih) * g.W + iw];
              }
            }
        }
  return 0;
}
