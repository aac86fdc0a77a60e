/*
 * rv_oracle.c -- CPU restatement of ramvamp's routed-expert FFN path.
 *
 * TEST INFRASTRUCTURE ONLY (see rv_oracle.h).  Built with
 * -ffp-contract=off: Rust never fuses a*b+c, so neither may this file,
 * except where the reference itself calls _mm256_fmadd_ps.
 *
 * Reference paths below are relative to the ramvamp source tree
 * (crates/core/src/...).
 */
#include "rv_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#if defined(__x86_64__)
#include <immintrin.h>
#define OR_HAVE_X86 1
#else
#define OR_HAVE_X86 0
#endif

#ifdef _OPENMP
#include <omp.h>
#endif

#define QK_K 256

const char *or_version(void) { return "rv_oracle 1 (ramvamp kernels/quants + model MoE block)"; }

int or_has_avx2(void) {
#if OR_HAVE_X86
  __builtin_cpu_init();
  return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
#else
  return 0;
#endif
}

/* ------------------------------------------------------------------ f16 */
/* kernels/quants/f16.rs:17-32 */
float or_f16_to_f32(uint16_t bits) {
  uint32_t sign = (uint32_t)(bits >> 15) << 31;
  uint32_t exp = (bits >> 10) & 0x1F;
  uint32_t frac = bits & 0x03FF;
  uint32_t out;
  if (exp == 0) {
    float mag = (float)frac * 5.9604644775390625e-08f; /* 2^-24, exact */
    memcpy(&out, &mag, 4);
    out |= sign;
  } else if (exp == 0x1F) {
    out = sign | 0x7F800000u | (frac << 13);
  } else {
    out = sign | ((exp + 112) << 23) | (frac << 13);
  }
  float f;
  memcpy(&f, &out, 4);
  return f;
}

/* kernels/quants/f16.rs:39-91 */
uint16_t or_f32_to_f16(float x) {
  uint32_t bits;
  memcpy(&bits, &x, 4);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
  int32_t exp = (int32_t)((bits >> 23) & 0xFF);
  uint32_t frac = bits & 0x007FFFFF;
  if (exp == 0xFF) {
    if (frac == 0) return sign | 0x7C00;
    return sign | 0x7C00 | 0x0200 | ((uint16_t)(frac >> 13) & 0x03FF);
  }
  int32_t e16 = exp - 112;
  if (e16 >= 0x1F) return sign | 0x7C00;
  if (e16 <= 0) {
    if (e16 < -10) return sign;
    uint32_t mant = exp == 0 ? frac : (frac | 0x00800000u);
    uint32_t shift = (uint32_t)(14 - e16);
    uint32_t ulp = 1u << shift;
    uint32_t half = ulp >> 1;
    uint32_t v = mant >> shift;
    uint32_t rem = mant & (ulp - 1);
    if (rem > half || (rem == half && (v & 1))) v += 1;
    return sign | (uint16_t)v;
  }
  uint32_t v = ((uint32_t)e16 << 10) | (frac >> 13);
  uint32_t rem = frac & 0x1FFF;
  if (rem > 0x1000 || (rem == 0x1000 && (v & 1))) v += 1;
  return sign | (uint16_t)v;
}

static inline float f16_at(const uint8_t *b, size_t off) {
  return or_f16_to_f32((uint16_t)(b[off] | (b[off + 1] << 8)));
}

/* --------------------------------------------------------------- blocks */
/* kernels/quants/mod.rs:72-105 */
size_t or_block_bytes(int fmt) {
  switch (fmt) {
    case OR_Q4_K: return 144;
    case OR_Q5_K: return 176;
    case OR_Q6_K: return 210;
    case OR_Q8_0: return 34;
    case OR_Q8_K: return 292;
  }
  return 0;
}
size_t or_block_weights(int fmt) { return fmt == OR_Q8_0 ? 32 : 256; }

/* kernels/quants/blocks.rs:127-141 (get_scale_min_k4) */
void or_get_scale_min_k4(int j, const uint8_t *s, uint8_t *sc, uint8_t *m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
    *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

/* kernels/quants/avx2.rs:463-485 (three-word mask unpack) */
void or_unpack_scales_mins(const uint8_t *scales, uint8_t *sc8, uint8_t *m8) {
  const uint32_t k1 = 0x3f3f3f3fu, k2 = 0x0f0f0f0fu, k3 = 0x03030303u;
  uint32_t u[4];
  memcpy(u, scales, 12);
  u[3] = ((u[2] >> 4) & k2) | (((u[1] >> 6) & k3) << 4);
  uint32_t uaux = u[1] & k1;
  u[1] = (u[2] & k2) | (((u[0] >> 6) & k3) << 4);
  u[2] = uaux;
  u[0] &= k1;
  memcpy(sc8, &u[0], 4);
  memcpy(sc8 + 4, &u[1], 4);
  memcpy(m8, &u[2], 4);
  memcpy(m8 + 4, &u[3], 4);
}

/* ------------------------------------------------------- Q8_K quantizer */
/* kernels/quants/quantize.rs:68-103 */
static void quantize_q8k_scalar(const float *xs, or_block_q8k *b) {
  float amax = 0.0f, max = 0.0f;
  for (int j = 0; j < QK_K; j++) {
    float av = fabsf(xs[j]);
    if (av > amax) {
      amax = av;
      max = xs[j];
    }
  }
  if (amax == 0.0f) {
    memset(b, 0, sizeof(*b));
    return;
  }
  float iscale = -127.0f / max;
  for (int j = 0; j < QK_K; j++) {
    float p = iscale * xs[j];
    int n = (int)rintf(p); /* round_ties_even under the default mode */
    if (n < -128) n = -128;
    if (n > 127) n = 127;
    b->qs[j] = (int8_t)n;
  }
  for (int g = 0; g < 16; g++) {
    int s = 0;
    for (int l = 0; l < 16; l++) s += b->qs[16 * g + l];
    b->bsums[g] = (int16_t)s;
  }
  b->d = 1.0f / iscale;
}

#if OR_HAVE_X86
__attribute__((target("avx2,fma"))) static inline float hsum_ps_8(__m256 v) {
  __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  s = _mm_add_ps(s, _mm_movehl_ps(s, s));
  s = _mm_add_ss(s, _mm_movehdup_ps(s));
  return _mm_cvtss_f32(s);
}
__attribute__((target("avx2,fma"))) static inline float hsum_ps_4(__m128 v) {
  __m128 s = _mm_add_ps(v, _mm_movehl_ps(v, v));
  s = _mm_add_ss(s, _mm_movehdup_ps(s));
  return _mm_cvtss_f32(s);
}
__attribute__((target("avx2,fma"))) static inline float hmax_ps_8(__m256 v) {
  __m128 m = _mm_max_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  m = _mm_max_ps(m, _mm_movehl_ps(m, m));
  m = _mm_max_ss(m, _mm_movehdup_ps(m));
  return _mm_cvtss_f32(m);
}
__attribute__((target("avx2,fma"))) static inline int32_t hsum_epi32_8(__m256i v) {
  __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
  s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
  s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
  return _mm_cvtsi128_si32(s);
}
__attribute__((target("avx2,fma"))) static inline void pack_store_i8(int8_t *dst, __m256i i0,
                                                                     __m256i i1, __m256i i2,
                                                                     __m256i i3) {
  __m256i p01 = _mm256_packs_epi32(i0, i1);
  __m256i p23 = _mm256_packs_epi32(i2, i3);
  __m256i p = _mm256_packs_epi16(p01, p23);
  p = _mm256_permutevar8x32_epi32(p, _mm256_setr_epi32(0, 4, 1, 5, 2, 6, 3, 7));
  _mm256_storeu_si256((__m256i *)dst, p);
}

/* kernels/quants/avx2.rs:1070-1130 */
__attribute__((target("avx2,fma"))) static void quantize_q8k_avx2(const float *xs,
                                                                  or_block_q8k *b) {
  const __m256 sign_mask = _mm256_set1_ps(-0.0f);
  __m256 amax_v = _mm256_setzero_ps();
  for (int k = 0; k < QK_K / 8; k++)
    amax_v = _mm256_max_ps(amax_v, _mm256_andnot_ps(sign_mask, _mm256_loadu_ps(xs + 8 * k)));
  float amax = hmax_ps_8(amax_v);
  if (amax == 0.0f) {
    memset(b, 0, sizeof(*b));
    return;
  }
  __m256 target = _mm256_set1_ps(amax);
  float max = 0.0f;
  for (int k = 0; k < QK_K / 8; k++) {
    __m256 v = _mm256_loadu_ps(xs + 8 * k);
    int m = _mm256_movemask_ps(_mm256_cmp_ps(_mm256_andnot_ps(sign_mask, v), target, _CMP_EQ_OQ));
    if (m != 0) {
      max = xs[8 * k + __builtin_ctz((unsigned)m)];
      break;
    }
  }
  float iscale = -127.0f / max;
  __m256 iv = _mm256_set1_ps(iscale);
  for (int c = 0; c < QK_K / 32; c++) {
    int base = 32 * c;
    __m256i i0 = _mm256_cvtps_epi32(_mm256_mul_ps(_mm256_loadu_ps(xs + base), iv));
    __m256i i1 = _mm256_cvtps_epi32(_mm256_mul_ps(_mm256_loadu_ps(xs + base + 8), iv));
    __m256i i2 = _mm256_cvtps_epi32(_mm256_mul_ps(_mm256_loadu_ps(xs + base + 16), iv));
    __m256i i3 = _mm256_cvtps_epi32(_mm256_mul_ps(_mm256_loadu_ps(xs + base + 24), iv));
    b->bsums[2 * c] = (int16_t)hsum_epi32_8(_mm256_add_epi32(i0, i1));
    b->bsums[2 * c + 1] = (int16_t)hsum_epi32_8(_mm256_add_epi32(i2, i3));
    pack_store_i8(b->qs + base, i0, i1, i2, i3);
  }
  b->d = 1.0f / iscale;
}
#endif

int or_quantize_row_q8_k(const float *x, size_t n, or_block_q8k *out, size_t out_blocks,
                         int impl) {
  if (n != out_blocks * QK_K) return OR_ERR_QUANTIZE_LEN_MISMATCH;
  for (size_t b = 0; b < out_blocks; b++) {
#if OR_HAVE_X86
    if (impl == OR_IMPL_AVX2 && or_has_avx2()) {
      quantize_q8k_avx2(x + QK_K * b, out + b);
      continue;
    }
#endif
    quantize_q8k_scalar(x + QK_K * b, out + b);
  }
  return OR_OK;
}

/* ------------------------------------------------------ scalar k-dots */
/* dot.rs:59-90 (k_quant_affine_block) */
static float k_quant_affine_block(const int8_t *aux, const uint8_t *scales,
                                  const or_block_q8k *y, float d, float dmin) {
  uint8_t sc[8], mins[8];
  for (int j = 0; j < 8; j++) or_get_scale_min_k4(j, scales, &sc[j], &mins[j]);
  int32_t sumi_mins = 0;
  for (int g = 0; g < 16; g++) sumi_mins += (int32_t)y->bsums[g] * (int32_t)mins[g / 2];
  int32_t sumi = 0;
  for (int j = 0; j < 8; j++) {
    int32_t s = 0;
    for (int l = 0; l < 32; l++) s += (int32_t)aux[32 * j + l] * (int32_t)y->qs[32 * j + l];
    sumi += (int32_t)sc[j] * s;
  }
  return d * (float)sumi - dmin * (float)sumi_mins;
}

static void expand_q4k(const uint8_t *block, int8_t *aux) {
  const uint8_t *qs = block + 16;
  for (int span = 0; span < 4; span++)
    for (int l = 0; l < 32; l++) {
      aux[64 * span + l] = (int8_t)(qs[32 * span + l] & 0xF);
      aux[64 * span + 32 + l] = (int8_t)(qs[32 * span + l] >> 4);
    }
}
static void expand_q5k(const uint8_t *block, int8_t *aux) {
  const uint8_t *qh = block + 16, *qs = block + 48;
  for (int j = 0; j < 8; j++) {
    const uint8_t *q = qs + 32 * (j / 2);
    uint8_t mask = (uint8_t)(1u << j);
    for (int l = 0; l < 32; l++) {
      int low = (j % 2 == 0) ? (q[l] & 0xF) : (q[l] >> 4);
      int hi = (qh[l] & mask) ? 16 : 0;
      aux[32 * j + l] = (int8_t)(low + hi);
    }
  }
}
static void expand_q6k(const uint8_t *block, int8_t *aux) {
  for (int half = 0; half < 2; half++) {
    const uint8_t *ql = block + 64 * half;
    const uint8_t *qh = block + 128 + 32 * half;
    int8_t *a = aux + 128 * half;
    for (int l = 0; l < 32; l++) {
      int h = qh[l];
      a[l] = (int8_t)(((ql[l] & 0xF) | ((h & 3) << 4)) - 32);
      a[l + 32] = (int8_t)(((ql[l + 32] & 0xF) | (((h >> 2) & 3) << 4)) - 32);
      a[l + 64] = (int8_t)(((ql[l] >> 4) | (((h >> 4) & 3) << 4)) - 32);
      a[l + 96] = (int8_t)(((ql[l + 32] >> 4) | (((h >> 6) & 3) << 4)) - 32);
    }
  }
}

/* dot.rs:96-116, 122-145, 152-184 */
static float dot_scalar(int fmt, const uint8_t *w, const or_block_q8k *a, size_t nb) {
  float sumf = 0.0f;
  int8_t aux[QK_K];
  for (size_t b = 0; b < nb; b++) {
    const or_block_q8k *y = a + b;
    if (fmt == OR_Q4_K || fmt == OR_Q5_K) {
      const uint8_t *blk = w + b * or_block_bytes(fmt);
      float d = f16_at(blk, 0) * y->d;
      float dmin = f16_at(blk, 2) * y->d;
      if (fmt == OR_Q4_K) expand_q4k(blk, aux); else expand_q5k(blk, aux);
      sumf += k_quant_affine_block(aux, blk + 4, y, d, dmin);
    } else {
      const uint8_t *blk = w + b * 210;
      expand_q6k(blk, aux);
      int32_t sumi = 0;
      for (int g = 0; g < 16; g++) {
        int32_t scale = (int8_t)blk[192 + g];
        int32_t s = 0;
        for (int l = 0; l < 16; l++) s += (int32_t)aux[16 * g + l] * (int32_t)y->qs[16 * g + l];
        sumi += scale * s;
      }
      sumf += f16_at(blk, 208) * y->d * (float)sumi;
    }
  }
  return sumf;
}

/* ------------------------------------------------- lane model (portable)
 * The AVX2 arm (avx2.rs:554-600, 695-734, 744-838) keeps eight i32 lanes
 * per block: lane i sums the products of bytes 4i..4i+3 of every 32-byte
 * weight vector, each vector scaled by its sub-block scale (madd_epi16).
 * Per block: acc[i] = fma(d, (float)lane[i], acc[i]); Q4_K/Q5_K also keep
 * four min lanes (mins_dot, avx2.rs:536-548).  The result is the fixed
 * horizontal-sum tree of hsum_ps_8 / hsum_ps_4 (avx2.rs:494-510). */
static inline float lane_hsum8(const float *v) {
  float s0 = v[0] + v[4], s1 = v[1] + v[5], s2 = v[2] + v[6], s3 = v[3] + v[7];
  return (s0 + s2) + (s1 + s3);
}
static inline float lane_hsum4(const float *v) { return (v[0] + v[2]) + (v[1] + v[3]); }

/* Integer lanes of one block (the GPU reproduces exactly these). */
static void block_lanes(int fmt, const uint8_t *blk, const or_block_q8k *y, int32_t *lane,
                        int32_t *mlane) {
  if (fmt == OR_Q4_K || fmt == OR_Q5_K) {
    uint8_t sc[8], m[8];
    or_unpack_scales_mins(blk + 4, sc, m);
    const uint8_t *qh = blk + 16;
    const uint8_t *qs = blk + (fmt == OR_Q4_K ? 16 : 48);
    for (int i = 0; i < 8; i++) {
      int32_t s = 0;
      for (int j = 0; j < 4; j++) {
        int32_t lo = 0, hi = 0;
        for (int t = 0; t < 4; t++) {
          int bidx = 4 * i + t;
          int ql = qs[32 * j + bidx] & 0xF, qhh = qs[32 * j + bidx] >> 4;
          if (fmt == OR_Q5_K) {
            ql += ((qh[bidx] >> (2 * j)) & 1) << 4;
            qhh += ((qh[bidx] >> (2 * j + 1)) & 1) << 4;
          }
          lo += ql * y->qs[64 * j + bidx];
          hi += qhh * y->qs[64 * j + 32 + bidx];
        }
        s += (int32_t)sc[2 * j] * lo + (int32_t)sc[2 * j + 1] * hi;
      }
      lane[i] = s;
    }
    for (int l = 0; l < 4; l++) {
      int32_t p0 = y->bsums[4 * l] + y->bsums[4 * l + 1];
      int32_t p1 = y->bsums[4 * l + 2] + y->bsums[4 * l + 3];
      mlane[l] = (int32_t)m[2 * l] * p0 + (int32_t)m[2 * l + 1] * p1;
    }
  } else {
    const int8_t *scs = (const int8_t *)(blk + 192);
    for (int i = 0; i < 8; i++) {
      int32_t s = 0;
      for (int h = 0; h < 2; h++) {
        const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
        for (int k = 0; k < 4; k++) {
          int32_t part = 0;
          for (int t = 0; t < 4; t++) {
            int b = 4 * i + t, q;
            int hb = qh[b];
            switch (k) {
              case 0: q = (ql[b] & 0xF) | ((hb & 3) << 4); break;
              case 1: q = (ql[b + 32] & 0xF) | (((hb >> 2) & 3) << 4); break;
              case 2: q = (ql[b] >> 4) | (((hb >> 4) & 3) << 4); break;
              default: q = (ql[b + 32] >> 4) | (((hb >> 6) & 3) << 4); break;
            }
            part += (q - 32) * y->qs[128 * h + 32 * k + b];
          }
          s += (int32_t)scs[8 * h + 2 * k + (i >= 4)] * part;
        }
      }
      lane[i] = s;
    }
    if (mlane) memset(mlane, 0, 4 * sizeof(int32_t));
  }
}

static float dot_lanes(int fmt, const uint8_t *w, const or_block_q8k *a, size_t nb) {
  float acc[8] = {0}, accm[4] = {0};
  size_t bb = or_block_bytes(fmt);
  for (size_t b = 0; b < nb; b++) {
    const uint8_t *blk = w + b * bb;
    const or_block_q8k *y = a + b;
    int32_t lane[8], mlane[4];
    block_lanes(fmt, blk, y, lane, mlane);
    if (fmt == OR_Q6_K) {
      float d = f16_at(blk, 208) * y->d;
      for (int i = 0; i < 8; i++) acc[i] = fmaf(d, (float)lane[i], acc[i]);
    } else {
      float d = f16_at(blk, 0) * y->d;
      float dmin = f16_at(blk, 2) * y->d;
      for (int l = 0; l < 4; l++) accm[l] = fmaf(dmin, (float)mlane[l], accm[l]);
      for (int i = 0; i < 8; i++) acc[i] = fmaf(d, (float)lane[i], acc[i]);
    }
  }
  if (fmt == OR_Q6_K) return lane_hsum8(acc);
  return lane_hsum8(acc) - lane_hsum4(accm);
}

int or_block_int_sums(int fmt, const uint8_t *blk, const or_block_q8k *y, int32_t *lanes8,
                      int32_t *mins4, int32_t *sumi, int32_t *sumi_mins) {
  if (fmt != OR_Q4_K && fmt != OR_Q5_K && fmt != OR_Q6_K) return OR_ERR_UNSUPPORTED_FORMAT;
  int32_t mtmp[4];
  block_lanes(fmt, blk, y, lanes8, mins4 ? mins4 : mtmp);
  int32_t s = 0;
  for (int i = 0; i < 8; i++) s += lanes8[i];
  if (sumi) *sumi = s;
  if (sumi_mins) {
    int32_t sm = 0;
    if (fmt != OR_Q6_K) {
      uint8_t sc[8], m[8];
      for (int j = 0; j < 8; j++) or_get_scale_min_k4(j, blk + 4, &sc[j], &m[j]);
      for (int g = 0; g < 16; g++) sm += (int32_t)y->bsums[g] * (int32_t)m[g / 2];
    }
    *sumi_mins = sm;
  }
  return OR_OK;
}

/* --------------------------------------------------------- AVX2 k-dots */
#if OR_HAVE_X86
__attribute__((target("avx2,fma"))) static inline __m128i mins_dot(const or_block_q8k *y,
                                                                   const uint8_t *mins) {
  __m256i q8sums = _mm256_loadu_si256((const __m256i *)y->bsums);
  __m128i q8s = _mm_hadd_epi16(_mm256_castsi256_si128(q8sums), _mm256_extracti128_si256(q8sums, 1));
  __m128i minsv = _mm_cvtepu8_epi16(_mm_loadl_epi64((const __m128i *)mins));
  return _mm_madd_epi16(minsv, q8s);
}

/* avx2.rs:554-600 */
__attribute__((target("avx2,fma"))) static float dot_q4k_avx2(const uint8_t *w,
                                                              const or_block_q8k *a, size_t nb) {
  const __m256i m4 = _mm256_set1_epi8(0xF);
  __m256 acc = _mm256_setzero_ps();
  __m128 acc_m = _mm_setzero_ps();
  for (size_t b = 0; b < nb; b++) {
    const uint8_t *blk = w + 144 * b;
    const or_block_q8k *y = a + b;
    float d = f16_at(blk, 0) * y->d;
    float dmin = f16_at(blk, 2) * y->d;
    uint8_t sc[8], mins[8];
    or_unpack_scales_mins(blk + 4, sc, mins);
    __m128i prod = mins_dot(y, mins);
    acc_m = _mm_fmadd_ps(_mm_set1_ps(dmin), _mm_cvtepi32_ps(prod), acc_m);
    const uint8_t *qs = blk + 16;
    __m256i sumi = _mm256_setzero_si256();
    for (int j = 0; j < 4; j++) {
      __m256i q4bits = _mm256_loadu_si256((const __m256i *)(qs + 32 * j));
      __m256i q4l = _mm256_and_si256(q4bits, m4);
      __m256i q4h = _mm256_and_si256(_mm256_srli_epi16(q4bits, 4), m4);
      __m256i q8l = _mm256_loadu_si256((const __m256i *)(y->qs + 64 * j));
      __m256i q8h = _mm256_loadu_si256((const __m256i *)(y->qs + 64 * j + 32));
      __m256i p16l = _mm256_madd_epi16(_mm256_set1_epi16(sc[2 * j]), _mm256_maddubs_epi16(q4l, q8l));
      __m256i p16h = _mm256_madd_epi16(_mm256_set1_epi16(sc[2 * j + 1]), _mm256_maddubs_epi16(q4h, q8h));
      sumi = _mm256_add_epi32(sumi, _mm256_add_epi32(p16l, p16h));
    }
    acc = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi), acc);
  }
  return hsum_ps_8(acc) - hsum_ps_4(acc_m);
}

/* avx2.rs:615-662 */
__attribute__((target("avx2,fma"))) static void dot_q4k_avx2_x4(const uint8_t *w,
                                                                const or_block_q8k *const ya[4],
                                                                size_t nb, float *out) {
  const __m256i m4 = _mm256_set1_epi8(0xF);
  __m256 acc[4];
  __m128 acc_m[4];
  for (int r = 0; r < 4; r++) {
    acc[r] = _mm256_setzero_ps();
    acc_m[r] = _mm_setzero_ps();
  }
  for (size_t b = 0; b < nb; b++) {
    const uint8_t *blk = w + 144 * b;
    float dw = f16_at(blk, 0), dminw = f16_at(blk, 2);
    uint8_t sc[8], mins[8];
    or_unpack_scales_mins(blk + 4, sc, mins);
    for (int r = 0; r < 4; r++) {
      const or_block_q8k *y = ya[r] + b;
      float dmin = dminw * y->d;
      __m128i prod = mins_dot(y, mins);
      acc_m[r] = _mm_fmadd_ps(_mm_set1_ps(dmin), _mm_cvtepi32_ps(prod), acc_m[r]);
    }
    const uint8_t *qs = blk + 16;
    __m256i sumi[4];
    for (int r = 0; r < 4; r++) sumi[r] = _mm256_setzero_si256();
    for (int j = 0; j < 4; j++) {
      __m256i q4bits = _mm256_loadu_si256((const __m256i *)(qs + 32 * j));
      __m256i q4l = _mm256_and_si256(q4bits, m4);
      __m256i q4h = _mm256_and_si256(_mm256_srli_epi16(q4bits, 4), m4);
      __m256i scl = _mm256_set1_epi16(sc[2 * j]);
      __m256i sch = _mm256_set1_epi16(sc[2 * j + 1]);
      for (int r = 0; r < 4; r++) {
        const or_block_q8k *y = ya[r] + b;
        __m256i q8l = _mm256_loadu_si256((const __m256i *)(y->qs + 64 * j));
        __m256i q8h = _mm256_loadu_si256((const __m256i *)(y->qs + 64 * j + 32));
        __m256i p16l = _mm256_madd_epi16(scl, _mm256_maddubs_epi16(q4l, q8l));
        __m256i p16h = _mm256_madd_epi16(sch, _mm256_maddubs_epi16(q4h, q8h));
        sumi[r] = _mm256_add_epi32(sumi[r], _mm256_add_epi32(p16l, p16h));
      }
    }
    for (int r = 0; r < 4; r++) {
      float d = dw * ya[r][b].d;
      acc[r] = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi[r]), acc[r]);
    }
  }
  for (int r = 0; r < 4; r++) out[r] = hsum_ps_8(acc[r]) - hsum_ps_4(acc_m[r]);
}

/* avx2.rs:695-734 */
__attribute__((target("avx2,fma"))) static float dot_q5k_avx2(const uint8_t *w,
                                                              const or_block_q8k *a, size_t nb) {
  const __m256i m4 = _mm256_set1_epi8(0xF);
  __m256 acc = _mm256_setzero_ps();
  __m128 acc_m = _mm_setzero_ps();
  for (size_t b = 0; b < nb; b++) {
    const uint8_t *blk = w + 176 * b;
    const or_block_q8k *y = a + b;
    float d = f16_at(blk, 0) * y->d;
    float dmin = f16_at(blk, 2) * y->d;
    uint8_t sc[8], mins[8];
    or_unpack_scales_mins(blk + 4, sc, mins);
    __m128i prod = mins_dot(y, mins);
    acc_m = _mm_fmadd_ps(_mm_set1_ps(dmin), _mm_cvtepi32_ps(prod), acc_m);
    const uint8_t *qh = blk + 16, *qs = blk + 48;
    __m256i hbits = _mm256_loadu_si256((const __m256i *)qh);
    __m256i hmask = _mm256_set1_epi8(1);
    __m256i sumi = _mm256_setzero_si256();
    for (int j = 0; j < 4; j++) {
      __m256i q5bits = _mm256_loadu_si256((const __m256i *)(qs + 32 * j));
      __m256i h0 = _mm256_slli_epi16(
          _mm256_srl_epi16(_mm256_and_si256(hbits, hmask), _mm_cvtsi32_si128(2 * j)), 4);
      __m256i q5_0 = _mm256_add_epi8(_mm256_and_si256(q5bits, m4), h0);
      hmask = _mm256_slli_epi16(hmask, 1);
      __m256i h1 = _mm256_slli_epi16(
          _mm256_srl_epi16(_mm256_and_si256(hbits, hmask), _mm_cvtsi32_si128(2 * j + 1)), 4);
      __m256i q5_1 = _mm256_add_epi8(_mm256_and_si256(_mm256_srli_epi16(q5bits, 4), m4), h1);
      hmask = _mm256_slli_epi16(hmask, 1);
      __m256i q8l = _mm256_loadu_si256((const __m256i *)(y->qs + 64 * j));
      __m256i q8h = _mm256_loadu_si256((const __m256i *)(y->qs + 64 * j + 32));
      __m256i p16l = _mm256_madd_epi16(_mm256_set1_epi16(sc[2 * j]), _mm256_maddubs_epi16(q5_0, q8l));
      __m256i p16h = _mm256_madd_epi16(_mm256_set1_epi16(sc[2 * j + 1]), _mm256_maddubs_epi16(q5_1, q8h));
      sumi = _mm256_add_epi32(sumi, _mm256_add_epi32(p16l, p16h));
    }
    acc = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi), acc);
  }
  return hsum_ps_8(acc) - hsum_ps_4(acc_m);
}

__attribute__((target("avx2,fma"))) static inline __m256i scale_pair(int8_t lo, int8_t hi) {
  return _mm256_set_m128i(_mm_set1_epi16(hi), _mm_set1_epi16(lo));
}

/* The four 6-bit weight vectors of one half-block (avx2.rs:760-800). */
__attribute__((target("avx2,fma"))) static inline void q6_vectors(const uint8_t *blk, int half,
                                                                  __m256i q4[4]) {
  const __m256i m4 = _mm256_set1_epi8(0xF), m2 = _mm256_set1_epi8(3);
  __m256i q4bits1 = _mm256_loadu_si256((const __m256i *)(blk + 64 * half));
  __m256i q4bits2 = _mm256_loadu_si256((const __m256i *)(blk + 64 * half + 32));
  __m256i bits_h = _mm256_loadu_si256((const __m256i *)(blk + 128 + 32 * half));
  __m256i h0 = _mm256_slli_epi16(_mm256_and_si256(bits_h, m2), 4);
  __m256i h1 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(bits_h, 2), m2), 4);
  __m256i h2 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(bits_h, 4), m2), 4);
  __m256i h3 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(bits_h, 6), m2), 4);
  q4[0] = _mm256_or_si256(_mm256_and_si256(q4bits1, m4), h0);
  q4[1] = _mm256_or_si256(_mm256_and_si256(q4bits2, m4), h1);
  q4[2] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(q4bits1, 4), m4), h2);
  q4[3] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(q4bits2, 4), m4), h3);
}

/* avx2.rs:744-838 */
__attribute__((target("avx2,fma"))) static float dot_q6k_avx2(const uint8_t *w,
                                                              const or_block_q8k *a, size_t nb) {
  const __m256i m32s = _mm256_set1_epi8(32);
  __m256 acc = _mm256_setzero_ps();
  for (size_t b = 0; b < nb; b++) {
    const uint8_t *blk = w + 210 * b;
    const or_block_q8k *y = a + b;
    float d = f16_at(blk, 208) * y->d;
    const int8_t *scs = (const int8_t *)(blk + 192);
    __m256i sumi = _mm256_setzero_si256();
    for (int half = 0; half < 2; half++) {
      int base = 128 * half;
      __m256i q4[4];
      q6_vectors(blk, half, q4);
      __m256i p32[4];
      for (int k = 0; k < 4; k++) {
        __m256i q8 = _mm256_loadu_si256((const __m256i *)(y->qs + base + 32 * k));
        __m256i p16 = _mm256_sub_epi16(_mm256_maddubs_epi16(q4[k], q8), _mm256_maddubs_epi16(m32s, q8));
        int s = 8 * half + 2 * k;
        p32[k] = _mm256_madd_epi16(scale_pair(scs[s], scs[s + 1]), p16);
      }
      sumi = _mm256_add_epi32(sumi, _mm256_add_epi32(p32[0], p32[1]));
      sumi = _mm256_add_epi32(sumi, _mm256_add_epi32(p32[2], p32[3]));
    }
    acc = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi), acc);
  }
  return hsum_ps_8(acc);
}

/* avx2.rs:853-930 */
__attribute__((target("avx2,fma"))) static void dot_q6k_avx2_x4(const uint8_t *w,
                                                                const or_block_q8k *const ya[4],
                                                                size_t nb, float *out) {
  const __m256i m32s = _mm256_set1_epi8(32);
  __m256 acc[4];
  for (int r = 0; r < 4; r++) acc[r] = _mm256_setzero_ps();
  for (size_t b = 0; b < nb; b++) {
    const uint8_t *blk = w + 210 * b;
    float dw = f16_at(blk, 208);
    const int8_t *scs = (const int8_t *)(blk + 192);
    __m256i sumi[4];
    for (int r = 0; r < 4; r++) sumi[r] = _mm256_setzero_si256();
    for (int half = 0; half < 2; half++) {
      int base = 128 * half;
      __m256i q4[4], sc[4];
      q6_vectors(blk, half, q4);
      for (int k = 0; k < 4; k++) sc[k] = scale_pair(scs[8 * half + 2 * k], scs[8 * half + 2 * k + 1]);
      for (int r = 0; r < 4; r++) {
        const or_block_q8k *y = ya[r] + b;
        __m256i p32[4];
        for (int k = 0; k < 4; k++) {
          __m256i q8 = _mm256_loadu_si256((const __m256i *)(y->qs + base + 32 * k));
          __m256i p16 = _mm256_sub_epi16(_mm256_maddubs_epi16(q4[k], q8), _mm256_maddubs_epi16(m32s, q8));
          p32[k] = _mm256_madd_epi16(sc[k], p16);
        }
        sumi[r] = _mm256_add_epi32(sumi[r], _mm256_add_epi32(p32[0], p32[1]));
        sumi[r] = _mm256_add_epi32(sumi[r], _mm256_add_epi32(p32[2], p32[3]));
      }
    }
    for (int r = 0; r < 4; r++) {
      float d = dw * ya[r][b].d;
      acc[r] = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi[r]), acc[r]);
    }
  }
  for (int r = 0; r < 4; r++) out[r] = hsum_ps_8(acc[r]);
}
#endif

static int fmt_is_k(int fmt) { return fmt == OR_Q4_K || fmt == OR_Q5_K || fmt == OR_Q6_K; }

/* Unchecked single dot with the chosen arm. */
static float dot_one(int fmt, const uint8_t *w, const or_block_q8k *a, size_t nb, int impl) {
#if OR_HAVE_X86
  if (impl == OR_IMPL_AVX2 && or_has_avx2()) {
    if (fmt == OR_Q4_K) return dot_q4k_avx2(w, a, nb);
    if (fmt == OR_Q5_K) return dot_q5k_avx2(w, a, nb);
    return dot_q6k_avx2(w, a, nb);
  }
#endif
  if (impl == OR_IMPL_LANES) return dot_lanes(fmt, w, a, nb);
  return dot_scalar(fmt, w, a, nb);
}

/* dot.rs:30-51 (weight_blocks): same checks, same precedence. */
int or_vec_dot(int fmt, const uint8_t *w, size_t w_len, const or_block_q8k *a, size_t n_blocks,
               int impl, float *out) {
  if (!fmt_is_k(fmt)) return OR_ERR_UNSUPPORTED_FORMAT;
  size_t bb = or_block_bytes(fmt);
  if (w_len % bb != 0) return OR_ERR_ROW_BYTES_NOT_BLOCK_MULTIPLE;
  if (w_len / bb != n_blocks) return OR_ERR_BLOCK_COUNT_MISMATCH;
  *out = dot_one(fmt, w, a, n_blocks, impl);
  return OR_OK;
}

/* avx2.rs:267-329 (dot_rows): four activation rows per pass on AVX2 for
 * Q4_K/Q6_K, the single-row kernel for the remainder. */
static void dot_rows_unchecked(int fmt, const uint8_t *w, size_t nb, const or_block_q8k *a,
                               size_t n_acts, float *out, int impl) {
  size_t r = 0;
#if OR_HAVE_X86
  if (impl == OR_IMPL_AVX2 && or_has_avx2() && (fmt == OR_Q4_K || fmt == OR_Q6_K) && nb > 0) {
    for (; r + 4 <= n_acts; r += 4) {
      const or_block_q8k *ya[4] = {a + r * nb, a + (r + 1) * nb, a + (r + 2) * nb, a + (r + 3) * nb};
      if (fmt == OR_Q4_K) dot_q4k_avx2_x4(w, ya, nb, out + r);
      else dot_q6k_avx2_x4(w, ya, nb, out + r);
    }
  }
#endif
  for (; r < n_acts; r++) out[r] = dot_one(fmt, w, a + r * nb, nb, impl);
}

int or_vec_dot_rows(int fmt, const uint8_t *w, size_t w_len, const or_block_q8k *a, size_t n_acts,
                    float *out, int impl) {
  if (!fmt_is_k(fmt)) return OR_ERR_UNSUPPORTED_FORMAT;
  size_t bb = or_block_bytes(fmt);
  if (w_len % bb != 0) return OR_ERR_ROW_BYTES_NOT_BLOCK_MULTIPLE;
  dot_rows_unchecked(fmt, w, w_len / bb, a, n_acts, out, impl);
  return OR_OK;
}

/* gemv.rs:212-264 (validate) + :296-330 (gemv_impl). */
int or_gemv(int fmt, const uint8_t *w, size_t w_len, size_t in_dim, size_t out_dim,
            const or_block_q8k *acts, size_t n_acts, size_t r0, size_t r1, float *out,
            size_t out_len, int impl, int threads) {
  if (!fmt_is_k(fmt)) return OR_ERR_UNSUPPORTED_FORMAT;
  if (in_dim % QK_K != 0) return OR_ERR_INDIVISIBLE_ROW;
  size_t nb = in_dim / QK_K;
  size_t row_bytes = nb * or_block_bytes(fmt);
  if (row_bytes * out_dim != w_len) return OR_ERR_LENGTH_MISMATCH;
  if (r0 > r1 || r1 > out_dim) return OR_ERR_LENGTH_MISMATCH;
  if ((r1 - r0) * n_acts != out_len) return OR_ERR_LENGTH_MISMATCH;
  (void)acts;
  if (n_acts == 0) return OR_OK;
  long rows = (long)(r1 - r0);
#ifdef _OPENMP
  int nt = threads > 0 ? threads : 1;
#pragma omp parallel for num_threads(nt) schedule(static)
#endif
  for (long i = 0; i < rows; i++) {
    const uint8_t *row = w + (r0 + (size_t)i) * row_bytes;
    if (n_acts >= 4) dot_rows_unchecked(fmt, row, nb, acts, n_acts, out + (size_t)i * n_acts, impl);
    else
      for (size_t a = 0; a < n_acts; a++)
        out[(size_t)i * n_acts + a] = dot_one(fmt, row, acts + a * nb, nb, impl);
  }
  (void)threads;
  return OR_OK;
}

/* ------------------------------------------------------------------ Q8_0 */
/* Rust's saturating `f32 as i8`: NaN -> 0, out-of-range -> the nearest bound. */
static inline int8_t sat_i8(float r) {
  if (r != r) return 0;
  if (r >= 127.0f) return 127;
  if (r <= -128.0f) return -128;
  return (int8_t)r;
}

/* quantize.rs:37-54 (scalar).  amax starts at 0 and f32::max ignores NaN,
 * as fmaxf does. */
static void quantize_q8_0_scalar(const float *xs, or_block_q8_0 *b) {
  float amax = 0.0f;
  for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(xs[j]));
  float d = amax / 127.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  b->d = or_f16_to_f32(or_f32_to_f16(d));
  for (int j = 0; j < 32; j++) b->qs[j] = sat_i8(roundf(xs[j] * id));
}

#if OR_HAVE_X86
/* avx2.rs:997-1012 (round_away_ps): ties-to-even, then ties fixed away. */
__attribute__((target("avx2,fma"))) static inline __m256 round_away_ps(__m256 x) {
  __m256 t = _mm256_round_ps(x, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
  __m256 diff = _mm256_sub_ps(x, t);
  __m256 one = _mm256_set1_ps(1.0f), zero = _mm256_setzero_ps();
  __m256 tie_up = _mm256_and_ps(_mm256_cmp_ps(diff, _mm256_set1_ps(0.5f), _CMP_EQ_OQ),
                                _mm256_cmp_ps(x, zero, _CMP_GT_OQ));
  __m256 tie_dn = _mm256_and_ps(_mm256_cmp_ps(diff, _mm256_set1_ps(-0.5f), _CMP_EQ_OQ),
                                _mm256_cmp_ps(x, zero, _CMP_LT_OQ));
  t = _mm256_add_ps(t, _mm256_and_ps(tie_up, one));
  return _mm256_sub_ps(t, _mm256_and_ps(tie_dn, one));
}

/* avx2.rs:1022-1056 */
__attribute__((target("avx2,fma"))) static void quantize_q8_0_avx2(const float *xs, or_block_q8_0 *b) {
  const __m256 sm = _mm256_set1_ps(-0.0f);
  __m256 v0 = _mm256_loadu_ps(xs), v1 = _mm256_loadu_ps(xs + 8);
  __m256 v2 = _mm256_loadu_ps(xs + 16), v3 = _mm256_loadu_ps(xs + 24);
  __m256 a01 = _mm256_max_ps(_mm256_andnot_ps(sm, v0), _mm256_andnot_ps(sm, v1));
  __m256 a23 = _mm256_max_ps(_mm256_andnot_ps(sm, v2), _mm256_andnot_ps(sm, v3));
  float amax = hmax_ps_8(_mm256_max_ps(a01, a23));
  float d = amax / 127.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  b->d = or_f16_to_f32(or_f32_to_f16(d));
  __m256 iv = _mm256_set1_ps(id);
  __m256i i0 = _mm256_cvtps_epi32(round_away_ps(_mm256_mul_ps(v0, iv)));
  __m256i i1 = _mm256_cvtps_epi32(round_away_ps(_mm256_mul_ps(v1, iv)));
  __m256i i2 = _mm256_cvtps_epi32(round_away_ps(_mm256_mul_ps(v2, iv)));
  __m256i i3 = _mm256_cvtps_epi32(round_away_ps(_mm256_mul_ps(v3, iv)));
  pack_store_i8(b->qs, i0, i1, i2, i3);
}

/* avx2.rs:942-963: sign trick, maddubs + madd -> eight i32 lanes (lane i =
 * products 4i..4i+3), one FMA per lane per block, hsum_ps_8. */
__attribute__((target("avx2,fma"))) static float dot_q8_0_avx2(const uint8_t *w, const or_block_q8_0 *a,
                                                               size_t nb) {
  const __m256i ones = _mm256_set1_epi16(1);
  __m256 acc = _mm256_setzero_ps();
  for (size_t b = 0; b < nb; b++) {
    const uint8_t *blk = w + 34 * b;
    float d = f16_at(blk, 0) * a[b].d;
    __m256i qx = _mm256_loadu_si256((const __m256i *)(blk + 2));
    __m256i qy = _mm256_loadu_si256((const __m256i *)a[b].qs);
    __m256i dot16 = _mm256_maddubs_epi16(_mm256_sign_epi8(qx, qx), _mm256_sign_epi8(qy, qx));
    __m256i sum32 = _mm256_madd_epi16(ones, dot16);
    acc = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sum32), acc);
  }
  return hsum_ps_8(acc);
}
#endif

/* dot.rs:190-201 (scalar ground truth). */
static float dot_q8_0_scalar(const uint8_t *w, const or_block_q8_0 *a, size_t nb) {
  float sumf = 0.0f;
  for (size_t b = 0; b < nb; b++) {
    const uint8_t *blk = w + 34 * b;
    int32_t sumi = 0;
    for (int l = 0; l < 32; l++) sumi += (int32_t)(int8_t)blk[2 + l] * (int32_t)a[b].qs[l];
    sumf += (float)sumi * (f16_at(blk, 0) * a[b].d);
  }
  return sumf;
}

/* Lane model of avx2.rs:942-963: lane i of block b is the exact sum of
 * products 4i..4i+3; acc[i] = fma(d_b, lane, acc[i]); hsum_ps_8 order. */
static float dot_q8_0_lanes(const uint8_t *w, const or_block_q8_0 *a, size_t nb) {
  float acc[8] = {0};
  for (size_t b = 0; b < nb; b++) {
    const uint8_t *blk = w + 34 * b;
    float d = f16_at(blk, 0) * a[b].d;
    for (int i = 0; i < 8; i++) {
      int32_t s = 0;
      for (int t = 0; t < 4; t++) s += (int32_t)(int8_t)blk[2 + 4 * i + t] * (int32_t)a[b].qs[4 * i + t];
      acc[i] = fmaf(d, (float)s, acc[i]);
    }
  }
  return lane_hsum8(acc);
}

static float dot_q8_0_one(const uint8_t *w, const or_block_q8_0 *a, size_t nb, int impl) {
#if OR_HAVE_X86
  if (impl == OR_IMPL_AVX2 && or_has_avx2()) return dot_q8_0_avx2(w, a, nb);
#endif
  if (impl == OR_IMPL_LANES) return dot_q8_0_lanes(w, a, nb);
  return dot_q8_0_scalar(w, a, nb);
}

int or_quantize_row_q8_0(const float *x, size_t n, or_block_q8_0 *out, size_t out_blocks, int impl) {
  if (n != out_blocks * 32) return OR_ERR_QUANTIZE_LEN_MISMATCH;
  for (size_t b = 0; b < out_blocks; b++) {
#if OR_HAVE_X86
    if (impl == OR_IMPL_AVX2 && or_has_avx2()) {
      quantize_q8_0_avx2(x + 32 * b, out + b);
      continue;
    }
#endif
    quantize_q8_0_scalar(x + 32 * b, out + b);
  }
  return OR_OK;
}

/* dot.rs:30-51 (weight_blocks) + the arm chosen by impl. */
int or_vec_dot_q8_0(const uint8_t *w, size_t w_len, const or_block_q8_0 *a, size_t n_blocks, int impl,
                    float *out) {
  if (w_len % 34 != 0) return OR_ERR_ROW_BYTES_NOT_BLOCK_MULTIPLE;
  if (w_len / 34 != n_blocks) return OR_ERR_BLOCK_COUNT_MISMATCH;
  *out = dot_q8_0_one(w, a, n_blocks, impl);
  return OR_OK;
}

/* gemv.rs:544-640 (gemv_q8_0 / _rows / _batched through gemv_impl,
 * :212-264 validation): out[i*n_acts+a] = row(r0+i) . act_a. */
int or_gemv_q8_0(const uint8_t *w, size_t w_len, size_t in_dim, size_t out_dim, const or_block_q8_0 *acts,
                 size_t acts_len, size_t n_acts, size_t r0, size_t r1, float *out, size_t out_len, int impl,
                 int threads) {
  if (in_dim % 32 != 0) return OR_ERR_INDIVISIBLE_ROW;
  size_t nb = in_dim / 32, row_bytes = nb * 34;
  if (row_bytes * out_dim != w_len) return OR_ERR_LENGTH_MISMATCH;
  if (r0 > r1 || r1 > out_dim) return OR_ERR_LENGTH_MISMATCH;
  if ((r1 - r0) * n_acts != out_len) return OR_ERR_LENGTH_MISMATCH;
  if (nb * n_acts != acts_len) return OR_ERR_BLOCK_COUNT_MISMATCH;
  if (n_acts == 0) return OR_OK;
  long rows = (long)(r1 - r0);
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads > 0 ? threads : 1) schedule(static)
#endif
  for (long i = 0; i < rows; i++)
    for (size_t a = 0; a < n_acts; a++)
      out[(size_t)i * n_acts + a] = dot_q8_0_one(w + (r0 + (size_t)i) * row_bytes, acts + a * nb, nb, impl);
  (void)threads;
  return OR_OK;
}

/* test_support.rs:221-234: packed 34-byte blocks via the activation
 * quantizer (d is already f16-rounded, so the f16 store is exact). */
void or_quantize_row_q8_0_test(const float *x, size_t n, uint8_t *out) {
  for (size_t b = 0; b < n / 32; b++) {
    or_block_q8_0 blk;
    quantize_q8_0_scalar(x + 32 * b, &blk);
    uint16_t h = or_f32_to_f16(blk.d);
    out[34 * b] = (uint8_t)(h & 0xFF);
    out[34 * b + 1] = (uint8_t)(h >> 8);
    memcpy(out + 34 * b + 2, blk.qs, 32);
  }
}

/* ------------------------------------------------------------- attention */
/* rope.rs:30-45 (rotate_head): f64 inverse frequency and angle, libm sin and
 * cos, applied in f32 as separate multiplies. */
static void rope_rotate_head(float *head, size_t half, uint32_t position, float theta) {
  double pos = (double)position, base = (double)theta, dim = (double)(2 * half);
  for (size_t i = 0; i < half; i++) {
    double inv_freq = pow(base, -2.0 * (double)i / dim);
    double ang = pos * inv_freq;
    float sn = (float)sin(ang), cs = (float)cos(ang);
    float x0 = head[i], x1 = head[i + half];
    head[i] = x0 * cs - x1 * sn;
    head[i + half] = x0 * sn + x1 * cs;
  }
}

/* rope.rs:80-111 (rope_neox_heads) */
int or_rope_neox_heads(float *x, size_t n_heads, size_t head_dim, uint32_t position, float theta) {
  if (head_dim == 0 || head_dim % 2) return OR_ERR_INVALID_HEAD_DIM;
  for (size_t h = 0; h < n_heads; h++) rope_rotate_head(x + h * head_dim, head_dim / 2, position, theta);
  return OR_OK;
}

/* The f32 rotation factors rotate_head forms for one position. */
void or_rope_factors(size_t head_dim, uint32_t position, float theta, float *cos_out, float *sin_out) {
  double pos = (double)position, base = (double)theta, dim = (double)head_dim;
  for (size_t i = 0; i < head_dim / 2; i++) {
    double ang = pos * pow(base, -2.0 * (double)i / dim);
    cos_out[i] = (float)cos(ang);
    sin_out[i] = (float)sin(ang);
  }
}

/* attention.rs:1075-1303, the scalar arm (the AVX2 + F16C arm is pinned
 * bit-identical to it): per kv head, scores[g][t] = scale * (q_g . K[t])
 * with one f32 accumulator over i ascending (separate multiply and add),
 * softmax per query head, out[g][i] = sum over t ascending of w_t * V[t][i].
 * Caches are f16 bits, [positions][n_kv_heads * head_dim]. */
int or_attention(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, size_t positions,
                 size_t n_heads, size_t n_kv_heads, size_t head_dim, float scale, float *out) {
  if (positions == 0 || n_kv_heads == 0 || head_dim == 0) return OR_ERR_EMPTY;
  if (n_heads % n_kv_heads) return OR_ERR_LENGTH_MISMATCH;
  size_t group = n_heads / n_kv_heads, kv_dim = n_kv_heads * head_dim;
  float *scores = (float *)malloc(group * positions * sizeof(float));
  float *buf = (float *)malloc(head_dim * sizeof(float));
  if (!scores || !buf) { free(scores); free(buf); return OR_ERR_EMPTY; }
  for (size_t kvh = 0; kvh < n_kv_heads; kvh++) {
    const float *qg = q + kvh * group * head_dim;
    float *og = out + kvh * group * head_dim;
    size_t col = kvh * head_dim;
    for (size_t t = 0; t < positions; t++) {
      for (size_t i = 0; i < head_dim; i++) buf[i] = or_f16_to_f32(k_cache[t * kv_dim + col + i]);
      for (size_t g = 0; g < group; g++) {
        float acc = 0.0f;
        for (size_t i = 0; i < head_dim; i++) acc += qg[g * head_dim + i] * buf[i];
        scores[g * positions + t] = scale * acc;
      }
    }
    for (size_t g = 0; g < group; g++) or_softmax(scores + g * positions, positions);
    for (size_t k = 0; k < group * head_dim; k++) og[k] = 0.0f;
    for (size_t t = 0; t < positions; t++) {
      for (size_t i = 0; i < head_dim; i++) buf[i] = or_f16_to_f32(v_cache[t * kv_dim + col + i]);
      for (size_t g = 0; g < group; g++) {
        float w = scores[g * positions + t];
        for (size_t i = 0; i < head_dim; i++) og[g * head_dim + i] += w * buf[i];
      }
    }
  }
  free(scores);
  free(buf);
  return OR_OK;
}

/* The attention half of one decode step (model/forward.rs:2614-2631): per-head
 * QK-RMSNorm of q and k (norm.rs:72-90, shared [head_dim] weights), NeoX RoPE
 * of both at `position`, the f16 append of k and v at row `position`
 * (kv/mod.rs:336-373), then attention over positions 0..position.  q and k
 * are updated in place, as the reference does. */
int or_attn_decode_step(float *q, float *k, const float *v, const float *q_norm, const float *k_norm,
                        uint16_t *k_cache, uint16_t *v_cache, size_t position, size_t n_heads, size_t n_kv_heads,
                        size_t head_dim, float eps, float theta, float *out) {
  for (size_t h = 0; h < n_heads; h++) or_rmsnorm(q + h * head_dim, q_norm, head_dim, eps, q + h * head_dim);
  for (size_t h = 0; h < n_kv_heads; h++) or_rmsnorm(k + h * head_dim, k_norm, head_dim, eps, k + h * head_dim);
  int rc = or_rope_neox_heads(q, n_heads, head_dim, (uint32_t)position, theta);
  if (rc) return rc;
  or_rope_neox_heads(k, n_kv_heads, head_dim, (uint32_t)position, theta);
  size_t kv_dim = n_kv_heads * head_dim;
  for (size_t i = 0; i < kv_dim; i++) {
    k_cache[position * kv_dim + i] = or_f32_to_f16(k[i]);
    v_cache[position * kv_dim + i] = or_f32_to_f16(v[i]);
  }
  float scale = 1.0f / sqrtf((float)head_dim);
  return or_attention(q, k_cache, v_cache, position + 1, n_heads, n_kv_heads, head_dim, scale, out);
}

/* ------------------------------------------------------------------ Lcg */
/* test_support.rs:23-39 */
uint64_t or_lcg_next_u64(uint64_t *s) {
  *s = *s * 6364136223846793005ULL + 1442695040888963407ULL;
  return *s;
}
float or_lcg_next_f32(uint64_t *s) {
  return (float)(or_lcg_next_u64(s) >> 40) / (float)(1ULL << 24) * 2.0f - 1.0f;
}
void or_lcg_fill_f32(uint64_t *s, float *out, size_t n, float scale) {
  for (size_t i = 0; i < n; i++) out[i] = or_lcg_next_f32(s) * scale;
}

/* ------------------------------------------------- weight quantizers */
/* Rust's f32::clamp followed by `as u8`: NaN stays NaN, then saturates to 0. */
static inline uint8_t clamp_to_u8(float v, float lo, float hi) {
  if (v < lo) v = lo;
  else if (v > hi) v = hi;
  if (!(v == v)) return 0;
  return (uint8_t)v;
}

/* test_support.rs:45-58 */
static void pack_scales_k4(const uint8_t *ls, const uint8_t *lm, uint8_t *s) {
  memset(s, 0, 12);
  for (int j = 0; j < 8; j++) {
    if (j < 4) {
      s[j] = ls[j] & 63;
      s[j + 4] = lm[j] & 63;
    } else {
      s[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
      s[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
      s[j] |= (uint8_t)((lm[j] >> 4) << 6);
    }
  }
}

/* test_support.rs:66-95 (affine_scales) */
static void affine_scales(const float *x, float levels, uint8_t *packed, float *d_out,
                          float *dmin_out, float *step, float *minv) {
  float scale_f[8], min_f[8];
  for (int j = 0; j < 8; j++) {
    float vmin = INFINITY, vmax = -INFINITY;
    for (int l = 0; l < 32; l++) {
      float v = x[32 * j + l];
      vmin = fminf(vmin, v);
      vmax = fmaxf(vmax, v);
    }
    float nm = -vmin;
    min_f[j] = fmaxf(nm, 0.0f);
    float s = (vmax + min_f[j]) / levels;
    scale_f[j] = fmaxf(s, 0.0f);
  }
  float max_scale = 0.0f, max_min = 0.0f;
  for (int j = 0; j < 8; j++) {
    max_scale = fmaxf(max_scale, scale_f[j]);
    max_min = fmaxf(max_min, min_f[j]);
  }
  float d = or_f16_to_f32(or_f32_to_f16(max_scale / 63.0f));
  float dmin = or_f16_to_f32(or_f32_to_f16(max_min / 63.0f));
  uint8_t ls[8] = {0}, lm[8] = {0};
  for (int j = 0; j < 8; j++) {
    if (d > 0.0f) ls[j] = clamp_to_u8(ceilf(scale_f[j] / d), 0.0f, 63.0f);
    if (dmin > 0.0f) lm[j] = clamp_to_u8(roundf(min_f[j] / dmin), 0.0f, 63.0f);
  }
  for (int j = 0; j < 8; j++) {
    step[j] = d * (float)ls[j];
    minv[j] = dmin * (float)lm[j];
  }
  pack_scales_k4(ls, lm, packed);
  *d_out = d;
  *dmin_out = dmin;
}

/* test_support.rs:99-104 */
static inline uint8_t affine_q(float v, float step, float min, float levels) {
  if (step <= 0.0f) return 0;
  return clamp_to_u8(roundf((v + min) / step), 0.0f, levels);
}

static void put_f16(uint8_t *p, float v) {
  uint16_t h = or_f32_to_f16(v);
  p[0] = (uint8_t)(h & 0xFF);
  p[1] = (uint8_t)(h >> 8);
}

/* test_support.rs:106-128 */
void or_quantize_row_q4_k_test(const float *x, size_t n, uint8_t *out) {
  for (size_t b = 0; b < n / QK_K; b++) {
    const float *xs = x + b * QK_K;
    uint8_t *o = out + b * 144;
    uint8_t scales[12];
    float d, dmin, step[8], minv[8];
    affine_scales(xs, 15.0f, scales, &d, &dmin, step, minv);
    uint8_t q[QK_K];
    for (int j = 0; j < 8; j++)
      for (int l = 0; l < 32; l++) q[32 * j + l] = affine_q(xs[32 * j + l], step[j], minv[j], 15.0f);
    put_f16(o, d);
    put_f16(o + 2, dmin);
    memcpy(o + 4, scales, 12);
    for (int span = 0; span < 4; span++)
      for (int l = 0; l < 32; l++)
        o[16 + 32 * span + l] = (uint8_t)(q[64 * span + l] | (q[64 * span + 32 + l] << 4));
  }
}

/* test_support.rs:130-161 */
void or_quantize_row_q5_k_test(const float *x, size_t n, uint8_t *out) {
  for (size_t b = 0; b < n / QK_K; b++) {
    const float *xs = x + b * QK_K;
    uint8_t *o = out + b * 176;
    uint8_t scales[12];
    float d, dmin, step[8], minv[8];
    affine_scales(xs, 31.0f, scales, &d, &dmin, step, minv);
    uint8_t q[QK_K];
    for (int j = 0; j < 8; j++)
      for (int l = 0; l < 32; l++) q[32 * j + l] = affine_q(xs[32 * j + l], step[j], minv[j], 31.0f);
    uint8_t qh[32] = {0};
    for (int j = 0; j < 8; j++)
      for (int l = 0; l < 32; l++)
        if (q[32 * j + l] >= 16) qh[l] |= (uint8_t)(1u << j);
    put_f16(o, d);
    put_f16(o + 2, dmin);
    memcpy(o + 4, scales, 12);
    memcpy(o + 16, qh, 32);
    for (int span = 0; span < 4; span++)
      for (int l = 0; l < 32; l++)
        o[48 + 32 * span + l] =
            (uint8_t)((q[64 * span + l] & 0xF) | ((q[64 * span + 32 + l] & 0xF) << 4));
  }
}

/* test_support.rs:163-219 */
void or_quantize_row_q6_k_test(const float *x, size_t n, uint8_t *out) {
  for (size_t b = 0; b < n / QK_K; b++) {
    const float *xs = x + b * QK_K;
    uint8_t *o = out + b * 210;
    float scale_f[16];
    for (int g = 0; g < 16; g++) {
      float amax = 0.0f;
      for (int l = 0; l < 16; l++) amax = fmaxf(amax, fabsf(xs[16 * g + l]));
      scale_f[g] = amax / 31.0f;
    }
    float max_scale = 0.0f;
    for (int g = 0; g < 16; g++) max_scale = fmaxf(max_scale, scale_f[g]);
    float d = or_f16_to_f32(or_f32_to_f16(max_scale / 127.0f));
    uint8_t ls[16] = {0};
    for (int g = 0; g < 16; g++)
      if (d > 0.0f) ls[g] = clamp_to_u8(ceilf(scale_f[g] / d), 0.0f, 127.0f);
    uint8_t q[QK_K];
    for (int g = 0; g < 16; g++) {
      float step = d * (float)ls[g];
      for (int l = 0; l < 16; l++) {
        int v = 0;
        if (step > 0.0f) {
          float r = roundf(xs[16 * g + l] / step);
          if (r < -32.0f) r = -32.0f;
          else if (r > 31.0f) r = 31.0f;
          v = (int)r;
        }
        q[16 * g + l] = (uint8_t)(v + 32);
      }
    }
    uint8_t *ql = o, *qh = o + 128;
    for (int half = 0; half < 2; half++) {
      int base = 128 * half;
      for (int l = 0; l < 32; l++) {
        uint8_t v1 = q[base + l], v2 = q[base + l + 32], v3 = q[base + l + 64], v4 = q[base + l + 96];
        ql[64 * half + l] = (uint8_t)((v1 & 0xF) | ((v3 & 0xF) << 4));
        ql[64 * half + l + 32] = (uint8_t)((v2 & 0xF) | ((v4 & 0xF) << 4));
        qh[32 * half + l] = (uint8_t)((v1 >> 4) | ((v2 >> 4) << 2) | ((v3 >> 4) << 4) | ((v4 >> 4) << 6));
      }
    }
    for (int g = 0; g < 16; g++) o[192 + g] = ls[g];
    put_f16(o + 208, d);
  }
}

/* dequant.rs:28-132 */
int or_dequantize_row(int fmt, const uint8_t *bytes, size_t len, float *out) {
  if (fmt == OR_Q8_0) { /* dequant.rs:134-147 */
    if (len % 34 != 0) return OR_ERR_ROW_BYTES_NOT_BLOCK_MULTIPLE;
    for (size_t b = 0; b < len / 34; b++) {
      float d = f16_at(bytes + 34 * b, 0);
      for (int l = 0; l < 32; l++) out[32 * b + l] = d * (float)(int8_t)bytes[34 * b + 2 + l];
    }
    return OR_OK;
  }
  if (!fmt_is_k(fmt)) return OR_ERR_UNSUPPORTED_FORMAT;
  size_t bb = or_block_bytes(fmt);
  if (len % bb != 0) return OR_ERR_ROW_BYTES_NOT_BLOCK_MULTIPLE;
  for (size_t b = 0; b < len / bb; b++) {
    const uint8_t *blk = bytes + b * bb;
    float *y = out + b * QK_K;
    int8_t aux[QK_K];
    if (fmt == OR_Q6_K) {
      float d = f16_at(blk, 208);
      expand_q6k(blk, aux);
      for (int g = 0; g < 16; g++) {
        float s = d * (float)(int8_t)blk[192 + g];
        for (int l = 0; l < 16; l++) y[16 * g + l] = s * (float)aux[16 * g + l];
      }
    } else {
      float d = f16_at(blk, 0), dmin = f16_at(blk, 2);
      if (fmt == OR_Q4_K) expand_q4k(blk, aux); else expand_q5k(blk, aux);
      for (int j = 0; j < 8; j++) {
        uint8_t sc, m;
        or_get_scale_min_k4(j, blk + 4, &sc, &m);
        float d1 = d * (float)sc, m1 = dmin * (float)m;
        for (int l = 0; l < 32; l++) y[32 * j + l] = d1 * (float)aux[32 * j + l] - m1;
      }
    }
  }
  return OR_OK;
}

/* ------------------------------------------------------------ primitives */
/* norm.rs:17-60 */
int or_rmsnorm(const float *x, const float *w, size_t n, float eps, float *out) {
  if (n == 0) return OR_ERR_EMPTY;
  double sum = 0.0;
  for (size_t i = 0; i < n; i++) {
    double v = (double)x[i];
    sum += v * v;
  }
  double mean = sum / (double)n;
  float inv = (float)(1.0 / sqrt(mean + (double)eps));
  for (size_t i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
  return OR_OK;
}

/* softmax.rs:18-40 */
int or_softmax(float *x, size_t n) {
  if (n == 0) return OR_ERR_EMPTY;
  float maxf = -INFINITY;
  for (size_t i = 0; i < n; i++)
    if (x[i] > maxf) maxf = x[i];
  double max = (double)maxf, sum = 0.0;
  for (size_t i = 0; i < n; i++) {
    double e = exp((double)x[i] - max);
    x[i] = (float)e;
    sum += e;
  }
  float inv = (float)(1.0 / sum);
  for (size_t i = 0; i < n; i++) x[i] *= inv;
  return OR_OK;
}

/* activation.rs:14-42 */
static inline float silu_one(float v) { return v / (1.0f + expf(-v)); }
int or_swiglu_combine(float *gate, const float *up, size_t n) {
  for (size_t i = 0; i < n; i++) gate[i] = silu_one(gate[i]) * up[i];
  return OR_OK;
}

/* forward.rs:1231-1237 */
float or_dot_f32(const float *a, const float *b, size_t n) {
  float acc = 0.0f;
  for (size_t i = 0; i < n; i++) acc += a[i] * b[i];
  return acc;
}

/* forward.rs:2669-2705 */
int or_route(const float *normed, const float *router, uint32_t hidden, uint32_t n_experts,
             uint32_t top_k, int norm_topk_prob, float *logits, uint32_t *ids, float *weights) {
  float probs[1024];
  if (n_experts == 0 || n_experts > 1024 || top_k > n_experts) return OR_ERR_LENGTH_MISMATCH;
  for (uint32_t e = 0; e < n_experts; e++) {
    float l = or_dot_f32(router + (size_t)e * hidden, normed, hidden);
    if (logits) logits[e] = l;
    probs[e] = l;
  }
  or_softmax(probs, n_experts);
  for (uint32_t k = 0; k < top_k; k++) {
    uint32_t best_e = 0;
    float best_p = -INFINITY;
    for (uint32_t e = 0; e < n_experts; e++)
      if (probs[e] > best_p) {
        best_p = probs[e];
        best_e = e;
      }
    ids[k] = best_e;
    weights[k] = best_p;
    probs[best_e] = -INFINITY;
  }
  if (norm_topk_prob) {
    float sum = -0.0f;
    for (uint32_t k = 0; k < top_k; k++) sum += weights[k];
    for (uint32_t k = 0; k < top_k; k++) weights[k] /= sum;
  }
  return OR_OK;
}

/* ---------------------------------------------------------- MoE block */
static const uint8_t *slab(const or_moe_layer *L, uint32_t e, uint64_t off) {
  return L->blobs + (size_t)e * L->stride + off;
}

static int check_layer(const or_moe_layer *L) {
  if (L->hidden == 0 || L->hidden % QK_K || L->moe == 0 || L->moe % QK_K) return OR_ERR_INDIVISIBLE_ROW;
  if (L->top_k == 0 || L->top_k > L->n_experts || L->n_experts > 1024) return OR_ERR_LENGTH_MISMATCH;
  if (!fmt_is_k(L->gate_fmt) || !fmt_is_k(L->up_fmt) || !fmt_is_k(L->down_fmt))
    return OR_ERR_UNSUPPORTED_FORMAT;
  return OR_OK;
}

/* Per token: forward.rs:2654-2754 with run_expert_window (:2159-2261).
 * Output rows of gemv are independent, so threads split rows (bit-neutral,
 * gemv.rs:17-44). */
int or_moe_decode(const or_moe_layer *L, float *residual, size_t T, uint32_t *topk_ids,
                  float *topk_w, const or_moe_taps *taps, int impl, int threads) {
  int rc = check_layer(L);
  if (rc) return rc;
  const size_t H = L->hidden, M = L->moe, K = L->top_k;
  const size_t hb = H / QK_K, mb = M / QK_K;
  float *normed = malloc(H * sizeof(float));
  or_block_q8k *acts = malloc(hb * sizeof(or_block_q8k));
  or_block_q8k *acts_moe = malloc(K * mb * sizeof(or_block_q8k));
  float *gate_up = malloc(2 * K * M * sizeof(float));
  float *staged = malloc(K * H * sizeof(float));
  float *acc = malloc(H * sizeof(float));
  uint32_t ids[1024];
  float w[1024];
  for (size_t t = 0; t < T; t++) {
    float *res = residual + t * H;
    or_rmsnorm(res, L->ffn_norm, H, L->eps, normed);
    float *lg = taps && taps->logits ? taps->logits + t * L->n_experts : NULL;
    or_route(normed, L->router, (uint32_t)H, L->n_experts, (uint32_t)K, L->norm_topk_prob, lg, ids, w);
    or_quantize_row_q8_k(normed, H, acts, hb, impl);
    if (taps && taps->normed) memcpy(taps->normed + t * H, normed, H * sizeof(float));
    if (taps && taps->acts) memcpy(taps->acts + t * hb, acts, hb * sizeof(or_block_q8k));
    /* gate || up of every routed expert: one fused row space. */
    size_t gu_rows = 2 * K * M;
    size_t gbytes = hb * or_block_bytes(L->gate_fmt), ubytes = hb * or_block_bytes(L->up_fmt);
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads > 0 ? threads : 1) schedule(static)
#endif
    for (long r = 0; r < (long)gu_rows; r++) {
      size_t j = (size_t)r / (2 * M), part = ((size_t)r / M) % 2, row = (size_t)r % M;
      const uint8_t *wrow = part == 0 ? slab(L, ids[j], L->gate_off) + row * gbytes
                                      : slab(L, ids[j], L->up_off) + row * ubytes;
      int fmt = part == 0 ? L->gate_fmt : L->up_fmt;
      gate_up[r] = dot_one(fmt, wrow, acts, hb, impl);
    }
    if (taps && taps->gate_up) memcpy(taps->gate_up + t * 2 * K * M, gate_up, gu_rows * sizeof(float));
    for (size_t j = 0; j < K; j++) {
      float *g = gate_up + j * 2 * M;
      or_swiglu_combine(g, g + M, M);
      or_quantize_row_q8_k(g, M, acts_moe + j * mb, mb, impl);
    }
    if (taps && taps->acts_moe) memcpy(taps->acts_moe + t * K * mb, acts_moe, K * mb * sizeof(or_block_q8k));
    size_t dbytes = mb * or_block_bytes(L->down_fmt);
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads > 0 ? threads : 1) schedule(static)
#endif
    for (long r = 0; r < (long)(K * H); r++) {
      size_t j = (size_t)r / H, row = (size_t)r % H;
      staged[r] = dot_one(L->down_fmt, slab(L, ids[j], L->down_off) + row * dbytes,
                          acts_moe + j * mb, mb, impl);
    }
    if (taps && taps->staged) memcpy(taps->staged + t * K * H, staged, K * H * sizeof(float));
    /* Fixed-order reduction (forward.rs:2744-2753) and vec_add. */
    for (size_t h = 0; h < H; h++) acc[h] = 0.0f;
    for (size_t k = 0; k < K; k++)
      for (size_t h = 0; h < H; h++) acc[h] += w[k] * staged[k * H + h];
    for (size_t h = 0; h < H; h++) res[h] += acc[h];
    if (topk_ids) memcpy(topk_ids + t * K, ids, K * sizeof(uint32_t));
    if (topk_w) memcpy(topk_w + t * K, w, K * sizeof(float));
  }
  free(normed); free(acts); free(acts_moe); free(gate_up); free(staged); free(acc);
  return OR_OK;
}

/* prefill.rs:2536-2580 */
int or_build_index(const uint32_t *topk_ids, size_t T, uint32_t top_k, uint32_t n_experts,
                   uint32_t *index_start, uint32_t *index) {
  memset(index_start, 0, (n_experts + 1) * sizeof(uint32_t));
  for (size_t i = 0; i < T * top_k; i++) {
    if (topk_ids[i] >= n_experts) return OR_ERR_ROUTED_OUT_OF_RANGE;
    index_start[topk_ids[i] + 1]++;
  }
  for (uint32_t e = 0; e < n_experts; e++) {
    if (index_start[e + 1] > T) return OR_ERR_LENGTH_MISMATCH;
    index_start[e + 1] += index_start[e];
  }
  uint32_t *cursor = malloc(n_experts * sizeof(uint32_t));
  memcpy(cursor, index_start, n_experts * sizeof(uint32_t));
  for (size_t r = 0; r < T; r++)
    for (uint32_t s = 0; s < top_k; s++) {
      uint32_t e = topk_ids[r * top_k + s];
      index[cursor[e]++] = ((uint32_t)r << 16) | s;
    }
  free(cursor);
  return OR_OK;
}

/* prefill.rs:2136-2263 (run_chunk MoE half), run_expert :2585-2732,
 * reduce_experts :2749-2778. */
int or_moe_prefill(const or_moe_layer *L, float *residual, size_t T, uint32_t *topk_ids,
                   float *topk_w, int impl, int threads) {
  int rc = check_layer(L);
  if (rc) return rc;
  if (T >= 65536) return OR_ERR_LENGTH_MISMATCH;
  const size_t H = L->hidden, M = L->moe, K = L->top_k, E = L->n_experts;
  const size_t hb = H / QK_K, mb = M / QK_K;
  float *normed = malloc(T * H * sizeof(float));
  or_block_q8k *acts = malloc(T * hb * sizeof(or_block_q8k));
  uint32_t *ids = malloc(T * K * sizeof(uint32_t));
  float *w = malloc(T * K * sizeof(float));
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads > 0 ? threads : 1) schedule(static)
#endif
  for (long t = 0; t < (long)T; t++) {
    or_rmsnorm(residual + t * H, L->ffn_norm, H, L->eps, normed + t * H);
    or_quantize_row_q8_k(normed + t * H, H, acts + t * hb, hb, impl);
    or_route(normed + t * H, L->router, (uint32_t)H, (uint32_t)E, (uint32_t)K, L->norm_topk_prob,
             NULL, ids + t * K, w + t * K);
  }
  uint32_t *start = malloc((E + 1) * sizeof(uint32_t));
  uint32_t *index = malloc(T * K * sizeof(uint32_t));
  rc = or_build_index(ids, T, (uint32_t)K, (uint32_t)E, start, index);
  if (rc) goto out;
  float *staged = calloc(T * K * H, sizeof(float));
  or_block_q8k *gather = malloc(T * hb * sizeof(or_block_q8k));
  float *gate = malloc(M * T * sizeof(float)), *up = malloc(M * T * sizeof(float));
  float *moe_t = malloc(M * sizeof(float));
  or_block_q8k *acts_moe = malloc(T * mb * sizeof(or_block_q8k));
  float *tmat = malloc(H * T * sizeof(float));
  size_t gbytes = hb * or_block_bytes(L->gate_fmt), ubytes = hb * or_block_bytes(L->up_fmt);
  size_t dbytes = mb * or_block_bytes(L->down_fmt);
  for (size_t e = 0; e < E; e++) {
    size_t lo = start[e], hi = start[e + 1], count = hi - lo;
    if (count == 0) continue;
    for (size_t j = 0; j < count; j++)
      memcpy(gather + j * hb, acts + (index[lo + j] >> 16) * hb, hb * sizeof(or_block_q8k));
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads > 0 ? threads : 1) schedule(static)
#endif
    for (long r = 0; r < (long)M; r++) {
      dot_rows_unchecked(L->gate_fmt, slab(L, (uint32_t)e, L->gate_off) + r * gbytes, hb, gather,
                         count, gate + r * count, impl);
      dot_rows_unchecked(L->up_fmt, slab(L, (uint32_t)e, L->up_off) + r * ubytes, hb, gather,
                         count, up + r * count, impl);
    }
    or_swiglu_combine(gate, up, M * count);
    for (size_t j = 0; j < count; j++) {
      for (size_t i = 0; i < M; i++) moe_t[i] = gate[i * count + j];
      or_quantize_row_q8_k(moe_t, M, acts_moe + j * mb, mb, impl);
    }
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads > 0 ? threads : 1) schedule(static)
#endif
    for (long r = 0; r < (long)H; r++)
      dot_rows_unchecked(L->down_fmt, slab(L, (uint32_t)e, L->down_off) + r * dbytes, mb, acts_moe,
                         count, tmat + r * count, impl);
    for (size_t h = 0; h < H; h++)
      for (size_t j = 0; j < count; j++) {
        uint32_t rs = index[lo + j];
        size_t row = rs >> 16, s = rs & 0xFFFF;
        staged[(row * K + s) * H + h] = tmat[h * count + j];
      }
  }
  for (size_t t = 0; t < T; t++) {
    float *res = residual + t * H;
    for (size_t h = 0; h < H; h++) {
      float a = 0.0f;
      for (size_t s = 0; s < K; s++) a += w[t * K + s] * staged[(t * K + s) * H + h];
      res[h] += a;
    }
  }
  if (topk_ids) memcpy(topk_ids, ids, T * K * sizeof(uint32_t));
  if (topk_w) memcpy(topk_w, w, T * K * sizeof(float));
  free(staged); free(gather); free(gate); free(up); free(moe_t); free(acts_moe); free(tmat);
out:
  free(normed); free(acts); free(ids); free(w); free(start); free(index);
  return rc;
}

/* ------------------------------------------------- synthetic weights */
static inline uint64_t splitmix64_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

void or_synth_normal(uint64_t seed, uint64_t offset, float sigma, float *out, size_t n) {
  for (size_t i = 0; i < n; i++) {
    uint64_t j = offset + i;
    int64_t s = 0;
    for (int k = 0; k < 6; k++) {
      uint64_t z = splitmix64_mix(seed + (j * 6 + (uint64_t)k + 1) * 0x9E3779B97F4A7C15ULL);
      s += (int64_t)(z >> 40) + (int64_t)((z >> 16) & 0xFFFFFFULL);
    }
    s -= (int64_t)6 << 24;
    float v = (float)s * 5.9604644775390625e-08f;
    out[i] = v * sigma;
  }
}

static void quantize_any(int fmt, const float *x, size_t n, uint8_t *out) {
  if (fmt == OR_Q4_K) or_quantize_row_q4_k_test(x, n, out);
  else if (fmt == OR_Q5_K) or_quantize_row_q5_k_test(x, n, out);
  else or_quantize_row_q6_k_test(x, n, out);
}

void or_fill_layer_synthetic(uint32_t hidden, uint32_t moe, uint32_t n_experts, uint64_t stride,
                             uint64_t gate_off, uint64_t up_off, uint64_t down_off, int gate_fmt,
                             int up_fmt, int down_fmt, uint64_t seed, float sigma, uint8_t *blobs,
                             int threads) {
  const size_t mh = (size_t)moe * hidden;
#ifdef _OPENMP
#pragma omp parallel num_threads(threads > 0 ? threads : 1)
#endif
  {
    float *tmp = malloc(3 * mh * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
    for (long e = 0; e < (long)n_experts; e++) {
      uint8_t *blob = blobs + (size_t)e * stride;
      or_synth_normal(seed, (uint64_t)e * 3 * mh, sigma, tmp, 3 * mh);
      quantize_any(gate_fmt, tmp, mh, blob + gate_off);
      quantize_any(up_fmt, tmp + mh, mh, blob + up_off);
      quantize_any(down_fmt, tmp + 2 * mh, mh, blob + down_off);
    }
    free(tmp);
  }
  (void)threads;
}
