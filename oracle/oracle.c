/*
 * oracle.c — CPU restatement of the reference's quantized-Llama decode path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker + timed CPU baseline). The CUDA
 * product never links this file. Build: oracle/build.py (gcc, -O2,
 * -ffp-contract=off so every f32 multiply and add rounds separately, as the
 * Rust code does; -fopenmp for the rayon-style row/column parallelism, which
 * never changes a result because each output is computed by one thread).
 *
 * Sources restated (see oracle.h for the parity status of each):
 *   candle-core 0.8.4  src/quantized/k_quants.rs   (BlockQ8K/Q4K/Q6K)
 *   candle-core 0.8.4  src/quantized/k_quants.rs   matmul()
 *   candle-nn 0.8.4    src/ops.rs rms_norm, softmax_last_dim; src/rotary_emb.rs rope_i
 *   candle-transformers 0.8.4 src/models/quantized_llama.rs
 *   reference native/arm_ai_nif/src/llama_candle.rs:69-176
 *   reference native/arm_ai_nif/src/shape_ops.rs (primitives, lines cited below)
 */
#include "oracle.h"

#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

static __thread char g_err[512];
static void set_err(const char* msg) {
  strncpy(g_err, msg, sizeof(g_err) - 1);
  g_err[sizeof(g_err) - 1] = 0;
}
const char* orc_last_error(void) { return g_err; }
void orc_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}
int orc_get_threads(void) { return omp_get_max_threads(); }

/* IEEE binary16 -> binary32, exact (half::f16::to_f32). */
float orc_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t ex = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t bits;
  if (ex == 0) {
    if (mant == 0) {
      bits = sign;
    } else {
      int e = -1;
      do {
        e++;
        mant <<= 1;
      } while ((mant & 0x400u) == 0);
      mant &= 0x3ffu;
      bits = sign | ((uint32_t)(112 - e) << 23) | (mant << 13);
    }
  } else if (ex == 31) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else {
    bits = sign | ((ex + 112u) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* Rust `f32 as i8`: saturating, NaN -> 0. */
/* IEEE binary32 -> binary16, round to nearest even (half::f16::from_f32). */
uint16_t orc_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
  if (ax < 0x38800000u) {
    float a;
    memcpy(&a, &ax, 4);
    return (uint16_t)(sign | (uint32_t)nearbyintf(a * 16777216.0f));
  }
  uint32_t hh = (((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13);
  uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (hh & 1u))) hh++;
  return (uint16_t)(sign | hh);
}

static int8_t sat_i8(float v) {
  if (v != v) return 0;
  if (v >= 127.f) return 127;
  if (v <= -128.f) return -128;
  return (int8_t)v;
}
static int32_t sat_i32(float v) {
  if (v != v) return 0;
  if (v >= 2147483647.f) return 2147483647;
  if (v <= -2147483648.f) return (int32_t)0x80000000u;
  return (int32_t)v;
}

/* ------------------------------------------------------------------ */
/* candle-core 0.8.4 k_quants.rs: BlockQ8K::from_float                 */
/* ------------------------------------------------------------------ */
int orc_quantize_row_q8k(const float* x, int64_t k, orc_block_q8k* y) {
  if (k % ORC_QK_K != 0) {
    set_err("quantize_row_q8k: k is not divisible by 256");
    return -1;
  }
  for (int64_t i = 0; i < k / ORC_QK_K; i++) {
    const float* xs = x + i * ORC_QK_K;
    orc_block_q8k* b = &y[i];
    float max = 0.f, amax = 0.f;
    for (int j = 0; j < ORC_QK_K; j++) {
      float a = fabsf(xs[j]);
      if (amax < a) {
        amax = a;
        max = xs[j];
      }
    }
    if (amax == 0.f) {
      b->d = 0.f;
      memset(b->qs, 0, sizeof b->qs);
      memset(b->bsums, 0, sizeof b->bsums); /* candle's buffer is zero-initialised */
    } else {
      float iscale = -128.f / max;
      for (int j = 0; j < ORC_QK_K; j++) {
        float v = roundf(iscale * xs[j]); /* Rust f32::round: half away from zero */
        b->qs[j] = sat_i8(fminf(v, 127.f));
      }
      for (int j = 0; j < ORC_QK_K / 16; j++) {
        int32_t s = 0;
        for (int ii = 0; ii < 16; ii++) s += b->qs[j * 16 + ii];
        b->bsums[j] = (int16_t)s;
      }
      b->d = 1.0f / iscale;
    }
  }
  return 0;
}

/* Unpack the 12-byte 6-bit scale/min field the way the generic
 * vec_dot_q4k_q8k does (utmp/kmask shuffling). */
static void q4k_scales_mins(const uint8_t* s12, uint8_t scales[8], uint8_t mins[8]) {
  const uint32_t kmask1 = 0x3f3f3f3fu, kmask2 = 0x0f0f0f0fu, kmask3 = 0x03030303u;
  uint32_t utmp[4];
  memcpy(utmp, s12, 12);
  utmp[3] = ((utmp[2] >> 4) & kmask2) | (((utmp[1] >> 6) & kmask3) << 4);
  uint32_t uaux = utmp[1] & kmask1;
  utmp[1] = (utmp[2] & kmask2) | (((utmp[0] >> 6) & kmask3) << 4);
  utmp[2] = uaux;
  utmp[0] &= kmask1;
  memcpy(scales, &utmp[0], 8);
  memcpy(mins, &utmp[2], 8);
}

/* candle-core 0.8.4 k_quants.rs: BlockQ4K::vec_dot_unopt (the path an
 * x86_64 build without `avx` in target_feature runs). */
float orc_vec_dot_q4k_q8k(int64_t n, const orc_block_q4k* xs, const orc_block_q8k* ys) {
  uint8_t scales[8], mins[8];
  int8_t aux8[ORC_QK_K];
  int16_t aux16[8];
  float sums[8] = {0};
  int32_t aux32[8];
  float sumf = 0.f;
  for (int64_t b = 0; b < n / ORC_QK_K; b++) {
    const orc_block_q4k* x = &xs[b];
    const orc_block_q8k* y = &ys[b];
    memset(aux32, 0, sizeof aux32);
    int8_t* a = aux8;
    const uint8_t* q4 = x->qs;
    for (int j = 0; j < ORC_QK_K / 64; j++) {
      for (int l = 0; l < 32; l++) a[l] = (int8_t)(q4[l] & 0xF);
      a += 32;
      for (int l = 0; l < 32; l++) a[l] = (int8_t)(q4[l] >> 4);
      a += 32;
      q4 += 32;
    }
    q4k_scales_mins(x->scales, scales, mins);
    int32_t sumi = 0;
    for (int j = 0; j < ORC_QK_K / 16; j++) sumi += (int32_t)y->bsums[j] * (int32_t)mins[j / 2];
    a = aux8;
    const int8_t* q8 = y->qs;
    for (int is = 0; is < 8; is++) {
      int32_t scale = scales[is];
      for (int r = 0; r < 4; r++) {
        for (int l = 0; l < 8; l++) aux16[l] = (int16_t)(q8[l] * a[l]);
        for (int l = 0; l < 8; l++) aux32[l] += scale * (int32_t)aux16[l];
        q8 += 8;
        a += 8;
      }
    }
    float d = orc_f16_to_f32(x->d) * y->d;
    for (int l = 0; l < 8; l++) sums[l] += d * (float)aux32[l];
    float dmin = orc_f16_to_f32(x->dmin) * y->d;
    sumf -= dmin * (float)sumi;
  }
  float s = -0.0f;
  for (int l = 0; l < 8; l++) s += sums[l];
  return sumf + s;
}

static void q6k_unpack(const orc_block_q6k* x, int8_t aux8[ORC_QK_K]) {
  for (int j = 0; j < ORC_QK_K; j += 128) {
    int8_t* a8 = aux8 + j;
    const uint8_t* q4 = x->ql + j / 2;
    const uint8_t* qh = x->qh + j / 4;
    for (int l = 0; l < 32; l++) {
      a8[l] = (int8_t)((int32_t)((q4[l] & 0xF) | ((qh[l] & 3) << 4)) - 32);
      a8[l + 32] = (int8_t)((int32_t)((q4[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32);
      a8[l + 64] = (int8_t)((int32_t)((q4[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32);
      a8[l + 96] = (int8_t)((int32_t)((q4[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32);
    }
  }
}

/* candle-core 0.8.4 k_quants.rs: BlockQ6K::vec_dot_unopt. */
float orc_vec_dot_q6k_q8k(int64_t n, const orc_block_q6k* xs, const orc_block_q8k* ys) {
  int8_t aux8[ORC_QK_K];
  int16_t aux16[8];
  float sums[8] = {0};
  float aux32[8];
  for (int64_t b = 0; b < n / ORC_QK_K; b++) {
    const orc_block_q6k* x = &xs[b];
    const orc_block_q8k* y = &ys[b];
    for (int l = 0; l < 8; l++) aux32[l] = 0.f;
    q6k_unpack(x, aux8);
    for (int j = 0; j < 16; j++) {
      float scale = (float)x->scales[j];
      const int8_t* q8 = y->qs + 16 * j;
      const int8_t* a = aux8 + 16 * j;
      for (int l = 0; l < 8; l++) aux16[l] = (int16_t)(q8[l] * a[l]);
      for (int l = 0; l < 8; l++) aux32[l] += scale * (float)aux16[l];
      for (int l = 0; l < 8; l++) aux16[l] = (int16_t)(q8[8 + l] * a[8 + l]);
      for (int l = 0; l < 8; l++) aux32[l] += scale * (float)aux16[l];
    }
    float d = orc_f16_to_f32(x->d) * y->d;
    for (int l = 0; l < 8; l++) sums[l] += aux32[l] * d;
  }
  float s = -0.0f;
  for (int l = 0; l < 8; l++) s += sums[l];
  return s;
}

/* Integer halves of the two dot products above, one pair per super-block. */
/* candle-core 0.8.4 k_quants.rs: BlockQ5K::vec_dot_unopt — BlockQ4K's
 * structure with the fifth bit of each value from qh (bit 2j of qh[l] for
 * the low nibbles of the j-th 64-value group, bit 2j + 1 for the high). */
float orc_vec_dot_q5k_q8k(int64_t n, const orc_block_q5k* xs, const orc_block_q8k* ys) {
  uint8_t scales[8], mins[8];
  int8_t aux8[ORC_QK_K];
  int16_t aux16[8];
  float sums[8] = {0};
  int32_t aux32[8];
  float sumf = 0.f;
  for (int64_t b = 0; b < n / ORC_QK_K; b++) {
    const orc_block_q5k* x = &xs[b];
    const orc_block_q8k* y = &ys[b];
    memset(aux32, 0, sizeof aux32);
    int8_t* a = aux8;
    const uint8_t* q4 = x->qs;
    const uint8_t* hm = x->qh;
    uint8_t m = 1;
    for (int j = 0; j < ORC_QK_K / 64; j++) {
      for (int l = 0; l < 32; l++) a[l] = (int8_t)(q4[l] & 0xF);
      for (int l = 0; l < 32; l++) a[l] = (int8_t)(a[l] + ((hm[l] & m) ? 16 : 0));
      a += 32;
      m <<= 1;
      for (int l = 0; l < 32; l++) a[l] = (int8_t)(q4[l] >> 4);
      for (int l = 0; l < 32; l++) a[l] = (int8_t)(a[l] + ((hm[l] & m) ? 16 : 0));
      a += 32;
      m <<= 1;
      q4 += 32;
    }
    q4k_scales_mins(x->scales, scales, mins);
    int32_t sumi = 0;
    for (int j = 0; j < ORC_QK_K / 16; j++) sumi += (int32_t)y->bsums[j] * (int32_t)mins[j / 2];
    a = aux8;
    const int8_t* q8 = y->qs;
    for (int is = 0; is < 8; is++) {
      int32_t scale = scales[is];
      for (int r = 0; r < 4; r++) {
        for (int l = 0; l < 8; l++) aux16[l] = (int16_t)(q8[l] * a[l]);
        for (int l = 0; l < 8; l++) aux32[l] += scale * (int32_t)aux16[l];
        q8 += 8;
        a += 8;
      }
    }
    float d = orc_f16_to_f32(x->d) * y->d;
    for (int l = 0; l < 8; l++) sums[l] += d * (float)aux32[l];
    float dmin = orc_f16_to_f32(x->dmin) * y->d;
    sumf -= dmin * (float)sumi;
  }
  float s = -0.0f;
  for (int l = 0; l < 8; l++) s += sums[l];
  return sumf + s;
}

/* candle-core 0.8.4 k_quants.rs BlockQ8_0::from_float: per 32 values
 * d = amax / 127, id = 1/d (0 when d = 0), q = round-half-away(x * id),
 * d stored as f16. */
int orc_quantize_row_q8_0(const float* x, int64_t k, orc_block_q8_0* y) {
  if (k % ORC_QK8_0 != 0) {
    set_err("quantize_row_q8_0: k is not divisible by 32");
    return -1;
  }
  for (int64_t b = 0; b < k / ORC_QK8_0; b++) {
    const float* xs = x + b * ORC_QK8_0;
    float amax = 0.f;
    for (int j = 0; j < ORC_QK8_0; j++) amax = fmaxf(amax, fabsf(xs[j]));
    const float d = amax / 127.0f;
    const float id = d != 0.f ? 1.0f / d : 0.f;
    y[b].d = orc_f32_to_f16(d);
    for (int j = 0; j < ORC_QK8_0; j++) y[b].qs[j] = sat_i8(roundf(xs[j] * id));
  }
  return 0;
}

/* k_quants.rs BlockQ4_0::vec_dot (generic): per block the integer sum of
 * (nibble - 8) * q8 (low nibbles pair with q8[j], high with q8[j + 16]),
 * then sumf += sumi * d_x * d_y. */
float orc_vec_dot_q4_0_q8_0(int64_t n, const orc_block_q4_0* xs, const orc_block_q8_0* ys) {
  float sumf = 0.f;
  for (int64_t b = 0; b < n / ORC_QK8_0; b++) {
    int32_t sumi = 0;
    for (int j = 0; j < ORC_QK8_0 / 2; j++) {
      const int32_t v0 = (int32_t)(xs[b].qs[j] & 0x0F) - 8;
      const int32_t v1 = (int32_t)(xs[b].qs[j] >> 4) - 8;
      sumi += v0 * (int32_t)ys[b].qs[j] + v1 * (int32_t)ys[b].qs[j + ORC_QK8_0 / 2];
    }
    sumf += (float)sumi * orc_f16_to_f32(xs[b].d) * orc_f16_to_f32(ys[b].d);
  }
  return sumf;
}

/* k_quants.rs BlockQ5_0::vec_dot (generic): the fifth bit of value j from
 * bit j of qh (low nibbles) and bit j + 16 (high nibbles), values - 16. */
float orc_vec_dot_q5_0_q8_0(int64_t n, const orc_block_q5_0* xs, const orc_block_q8_0* ys) {
  float sumf = 0.f;
  for (int64_t b = 0; b < n / ORC_QK8_0; b++) {
    uint32_t qh;
    memcpy(&qh, xs[b].qh, 4);
    int32_t sumi = 0;
    for (int j = 0; j < ORC_QK8_0 / 2; j++) {
      const uint32_t xh0 = ((qh & (1u << j)) >> j) << 4;
      const uint32_t xh1 = (qh & (1u << (j + 16))) >> (j + 12);
      const int32_t x0 = (int32_t)((xs[b].qs[j] & 0x0Fu) | xh0) - 16;
      const int32_t x1 = (int32_t)(((uint32_t)xs[b].qs[j] >> 4) | xh1) - 16;
      sumi += x0 * (int32_t)ys[b].qs[j] + x1 * (int32_t)ys[b].qs[j + ORC_QK8_0 / 2];
    }
    sumf += (float)sumi * orc_f16_to_f32(xs[b].d) * orc_f16_to_f32(ys[b].d);
  }
  return sumf;
}

/* k_quants.rs BlockQ8_0::vec_dot (generic). */
float orc_vec_dot_q8_0_q8_0(int64_t n, const orc_block_q8_0* xs, const orc_block_q8_0* ys) {
  float sumf = 0.f;
  for (int64_t b = 0; b < n / ORC_QK8_0; b++) {
    int32_t sumi = 0;
    for (int j = 0; j < ORC_QK8_0; j++) sumi += (int32_t)xs[b].qs[j] * (int32_t)ys[b].qs[j];
    sumf += (float)sumi * orc_f16_to_f32(xs[b].d) * orc_f16_to_f32(ys[b].d);
  }
  return sumf;
}

void orc_q4k_block_ints(const orc_block_q4k* xs, const orc_block_q8k* ys, int64_t nb,
                        int32_t* isum, int32_t* msum) {
  uint8_t scales[8], mins[8];
  for (int64_t b = 0; b < nb; b++) {
    const orc_block_q4k* x = &xs[b];
    const orc_block_q8k* y = &ys[b];
    q4k_scales_mins(x->scales, scales, mins);
    int32_t sumi = 0, tot = 0;
    for (int j = 0; j < 16; j++) sumi += (int32_t)y->bsums[j] * (int32_t)mins[j / 2];
    for (int j = 0; j < 4; j++) {
      int32_t dlo = 0, dhi = 0;
      for (int l = 0; l < 32; l++) {
        dlo += (int32_t)(x->qs[32 * j + l] & 0xF) * y->qs[64 * j + l];
        dhi += (int32_t)(x->qs[32 * j + l] >> 4) * y->qs[64 * j + 32 + l];
      }
      tot += (int32_t)scales[2 * j] * dlo + (int32_t)scales[2 * j + 1] * dhi;
    }
    isum[b] = tot;
    msum[b] = sumi;
  }
}

void orc_q6k_block_ints(const orc_block_q6k* xs, const orc_block_q8k* ys, int64_t nb,
                        int32_t* isum) {
  int8_t aux8[ORC_QK_K];
  for (int64_t b = 0; b < nb; b++) {
    q6k_unpack(&xs[b], aux8);
    int32_t tot = 0;
    for (int j = 0; j < 16; j++) {
      int32_t s = 0;
      for (int l = 0; l < 16; l++) s += (int32_t)aux8[16 * j + l] * ys[b].qs[16 * j + l];
      tot += (int32_t)xs[b].scales[j] * s;
    }
    isum[b] = tot;
  }
}

/* candle-core 0.8.4 k_quants.rs: BlockQ4K::to_float (get_scale_min_k4). */
static void get_scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
  if (j < 4) {
    *d = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *d = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

void orc_dequant_row_q4k(const orc_block_q4k* xs, int64_t k, float* y) {
  for (int64_t b = 0; b < k / ORC_QK_K; b++) {
    const orc_block_q4k* x = &xs[b];
    float d = orc_f16_to_f32(x->d), min = orc_f16_to_f32(x->dmin);
    float* out = y + b * ORC_QK_K;
    int is = 0, yi = 0;
    for (int j = 0; j < ORC_QK_K; j += 64) {
      const uint8_t* q = x->qs + j / 2;
      uint8_t sc, m;
      get_scale_min_k4(is, x->scales, &sc, &m);
      float d1 = d * (float)sc, m1 = min * (float)m;
      get_scale_min_k4(is + 1, x->scales, &sc, &m);
      float d2 = d * (float)sc, m2 = min * (float)m;
      for (int l = 0; l < 32; l++) out[yi++] = d1 * (float)(q[l] & 0xF) - m1;
      for (int l = 0; l < 32; l++) out[yi++] = d2 * (float)(q[l] >> 4) - m2;
      is += 2;
    }
  }
}

/* candle-core 0.8.4 k_quants.rs: BlockQ6K::to_float. */
void orc_dequant_row_q6k(const orc_block_q6k* xs, int64_t k, float* y) {
  for (int64_t b = 0; b < k / ORC_QK_K; b++) {
    const orc_block_q6k* x = &xs[b];
    float d = orc_f16_to_f32(x->d);
    for (int n = 0; n < ORC_QK_K; n += 128) {
      int idx = n / 128;
      float* ys = y + b * ORC_QK_K + n;
      const int8_t* sc = x->scales + 8 * idx;
      const uint8_t* ql = x->ql + 64 * idx;
      const uint8_t* qh = x->qh + 32 * idx;
      for (int l = 0; l < 32; l++) {
        int is = l / 16;
        int8_t q1 = (int8_t)(((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32);
        int8_t q2 = (int8_t)(((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32);
        int8_t q3 = (int8_t)(((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32);
        int8_t q4 = (int8_t)(((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32);
        ys[l] = d * (float)sc[is] * (float)q1;
        ys[l + 32] = d * (float)sc[is + 2] * (float)q2;
        ys[l + 64] = d * (float)sc[is + 4] * (float)q3;
        ys[l + 96] = d * (float)sc[is + 6] * (float)q4;
      }
    }
  }
}

static int64_t row_bytes(int type, int64_t k) {
  switch (type) {
    case ORC_F32: return 4 * k;
    case ORC_F16: return 2 * k;
    case ORC_Q4_0: return (k / ORC_QK8_0) * (int64_t)sizeof(orc_block_q4_0);
    case ORC_Q5_0: return (k / ORC_QK8_0) * (int64_t)sizeof(orc_block_q5_0);
    case ORC_Q8_0: return (k / ORC_QK8_0) * (int64_t)sizeof(orc_block_q8_0);
    case ORC_Q4_K: return (k / ORC_QK_K) * (int64_t)sizeof(orc_block_q4k);
    case ORC_Q5_K: return (k / ORC_QK_K) * (int64_t)sizeof(orc_block_q5k);
    case ORC_Q6_K: return (k / ORC_QK_K) * (int64_t)sizeof(orc_block_q6k);
    default: return -1;
  }
}

/* to_float of one row (k_quants.rs Block*::to_float; f16 via half). */
int orc_dequant_row(int type, const void* row, int64_t k, float* y) {
  switch (type) {
    case ORC_F32:
      memcpy(y, row, sizeof(float) * (size_t)k);
      return 0;
    case ORC_F16:
      for (int64_t i = 0; i < k; i++) y[i] = orc_f16_to_f32(((const uint16_t*)row)[i]);
      return 0;
    case ORC_Q4_K:
      orc_dequant_row_q4k((const orc_block_q4k*)row, k, y);
      return 0;
    case ORC_Q6_K:
      orc_dequant_row_q6k((const orc_block_q6k*)row, k, y);
      return 0;
    case ORC_Q4_0:
      for (int64_t b = 0; b < k / ORC_QK8_0; b++) {
        const orc_block_q4_0* x = (const orc_block_q4_0*)row + b;
        const float d = orc_f16_to_f32(x->d);
        for (int j = 0; j < ORC_QK8_0 / 2; j++) {
          y[b * ORC_QK8_0 + j] = (float)((int)(x->qs[j] & 0x0F) - 8) * d;
          y[b * ORC_QK8_0 + j + ORC_QK8_0 / 2] = (float)((int)(x->qs[j] >> 4) - 8) * d;
        }
      }
      return 0;
    case ORC_Q5_0:
      for (int64_t b = 0; b < k / ORC_QK8_0; b++) {
        const orc_block_q5_0* x = (const orc_block_q5_0*)row + b;
        const float d = orc_f16_to_f32(x->d);
        uint32_t qh;
        memcpy(&qh, x->qh, 4);
        for (int j = 0; j < ORC_QK8_0 / 2; j++) {
          const uint32_t xh0 = ((qh >> j) << 4) & 0x10u;
          const uint32_t xh1 = (qh >> (j + 12)) & 0x10u;
          y[b * ORC_QK8_0 + j] = (float)((int)((x->qs[j] & 0x0Fu) | xh0) - 16) * d;
          y[b * ORC_QK8_0 + j + ORC_QK8_0 / 2] = (float)((int)(((uint32_t)x->qs[j] >> 4) | xh1) - 16) * d;
        }
      }
      return 0;
    case ORC_Q8_0:
      for (int64_t b = 0; b < k / ORC_QK8_0; b++) {
        const orc_block_q8_0* x = (const orc_block_q8_0*)row + b;
        const float d = orc_f16_to_f32(x->d);
        for (int j = 0; j < ORC_QK8_0; j++) y[b * ORC_QK8_0 + j] = (float)x->qs[j] * d;
      }
      return 0;
    case ORC_Q5_K:
      for (int64_t b = 0; b < k / ORC_QK_K; b++) {
        const orc_block_q5k* x = (const orc_block_q5k*)row + b;
        const float d = orc_f16_to_f32(x->d), mn = orc_f16_to_f32(x->dmin);
        const uint8_t* ql = x->qs;
        float* o = y + b * ORC_QK_K;
        uint8_t u1 = 1, u2 = 2;
        for (int j = 0, is = 0; j < ORC_QK_K; j += 64, is += 2) {
          uint8_t sc, m;
          get_scale_min_k4(is, x->scales, &sc, &m);
          const float d1 = d * (float)sc, m1 = mn * (float)m;
          get_scale_min_k4(is + 1, x->scales, &sc, &m);
          const float d2 = d * (float)sc, m2 = mn * (float)m;
          for (int l = 0; l < 32; l++) *o++ = d1 * (float)((ql[l] & 0xF) + ((x->qh[l] & u1) ? 16 : 0)) - m1;
          for (int l = 0; l < 32; l++) *o++ = d2 * (float)((ql[l] >> 4) + ((x->qh[l] & u2) ? 16 : 0)) - m2;
          ql += 32;
          u1 <<= 2;
          u2 <<= 2;
        }
      }
      return 0;
    default:
      set_err("dequant_row: unsupported type");
      return -1;
  }
}

/* candle-core 0.8.4 k_quants.rs matmul(): every lhs row is quantised to the
 * weight's VecDotType (Q8_K here), then each output column is one vec_dot. */
int orc_qmatmul(const void* w, int wtype, int64_t n, int64_t k, const float* x, int64_t m,
                float* out) {
  if (wtype == ORC_F32) {
    /* f32 weights (not used by Q4_K_M files) — plain dot products. */
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < n; c++) {
      const float* wr = (const float*)w + c * k;
      for (int64_t r = 0; r < m; r++) {
        float s = 0.f;
        for (int64_t i = 0; i < k; i++) s += x[r * k + i] * wr[i];
        out[r * n + c] = s;
      }
    }
    return 0;
  }
  if (wtype == ORC_Q4_0 || wtype == ORC_Q5_0 || wtype == ORC_Q8_0) {
    /* the legacy types' VecDotType is Q8_0 */
    if (k % ORC_QK8_0 != 0) {
      set_err("qmatmul: k is not divisible by 32");
      return -1;
    }
    const int64_t nb0 = k / ORC_QK8_0;
    orc_block_q8_0* l0 = (orc_block_q8_0*)calloc((size_t)(m * nb0), sizeof(orc_block_q8_0));
    if (!l0) {
      set_err("qmatmul: out of memory");
      return -1;
    }
    for (int64_t r = 0; r < m; r++) orc_quantize_row_q8_0(x + r * k, k, l0 + r * nb0);
    const int64_t rb0 = row_bytes(wtype, k);
    for (int64_t r = 0; r < m; r++) {
      const orc_block_q8_0* lr = l0 + r * nb0;
#pragma omp parallel for schedule(static)
      for (int64_t c = 0; c < n; c++) {
        const void* wr = (const uint8_t*)w + c * rb0;
        out[r * n + c] = wtype == ORC_Q4_0   ? orc_vec_dot_q4_0_q8_0(k, (const orc_block_q4_0*)wr, lr)
                         : wtype == ORC_Q5_0 ? orc_vec_dot_q5_0_q8_0(k, (const orc_block_q5_0*)wr, lr)
                                             : orc_vec_dot_q8_0_q8_0(k, (const orc_block_q8_0*)wr, lr);
      }
    }
    free(l0);
    return 0;
  }
  if (wtype != ORC_Q4_K && wtype != ORC_Q5_K && wtype != ORC_Q6_K) {
    set_err("qmatmul: unsupported weight type");
    return -1;
  }
  if (k % ORC_QK_K != 0) {
    set_err("qmatmul: k is not divisible by 256");
    return -1;
  }
  int64_t nb = k / ORC_QK_K;
  orc_block_q8k* lhs = (orc_block_q8k*)calloc((size_t)(m * nb), sizeof(orc_block_q8k));
  if (!lhs) {
    set_err("qmatmul: out of memory");
    return -1;
  }
  for (int64_t r = 0; r < m; r++) orc_quantize_row_q8k(x + r * k, k, lhs + r * nb);
  int64_t rb = row_bytes(wtype, k);
  for (int64_t r = 0; r < m; r++) {
    const orc_block_q8k* lr = lhs + r * nb;
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < n; c++) {
      const void* wr = (const uint8_t*)w + c * rb;
      out[r * n + c] = wtype == ORC_Q4_K   ? orc_vec_dot_q4k_q8k(k, (const orc_block_q4k*)wr, lr)
                       : wtype == ORC_Q5_K ? orc_vec_dot_q5k_q8k(k, (const orc_block_q5k*)wr, lr)
                                           : orc_vec_dot_q6k_q8k(k, (const orc_block_q6k*)wr, lr);
    }
  }
  free(lhs);
  return 0;
}

/* ------------------------------------------------------------------ */
/* candle-transformers 0.8.4 quantized_llama                            */
/* ------------------------------------------------------------------ */
typedef struct {
  const void* p;
  int type;
  int64_t rows, cols;
} orc_tensor;

typedef struct {
  orc_tensor attn_norm, ffn_norm, wq, wk, wv, wo, wg, wu, wd;
} orc_layer;

struct orc_llama {
  int n_layer, n_embd, n_head, n_head_kv, head_dim, rope_dim, n_vocab, n_ff, max_seq;
  float eps, rope_base;
  orc_tensor tok_embd, output_norm, output;
  orc_layer* layers;
  float *cos_t, *sin_t; /* [max_seq][rope_dim/2] */
  float *kc, *vc;       /* [L][n_head_kv][max_seq][head_dim] */
  int kv_len;
  int kv_f16;
};

/* f32 -> binary16 (round to nearest even) -> f32. */
static float round_f16(float f) { return orc_f16_to_f32(orc_f32_to_f16(f)); }

void orc_llama_set_kv_f16(orc_llama* m, int on) { m->kv_f16 = on ? 1 : 0; }

orc_llama* orc_llama_new(int n_layer, int n_embd, int n_head, int n_head_kv, int rope_dim,
                         int n_vocab, int n_ff, float eps, float rope_base, int max_seq) {
  orc_llama* m = (orc_llama*)calloc(1, sizeof(orc_llama));
  if (!m) return NULL;
  m->n_layer = n_layer;
  m->n_embd = n_embd;
  m->n_head = n_head;
  m->n_head_kv = n_head_kv;
  m->head_dim = n_embd / n_head; /* quantized_llama: embedding_length / head_count */
  m->rope_dim = rope_dim;
  m->n_vocab = n_vocab;
  m->n_ff = n_ff;
  m->eps = eps;
  m->rope_base = rope_base;
  m->max_seq = max_seq;
  m->layers = (orc_layer*)calloc((size_t)n_layer, sizeof(orc_layer));
  return m;
}

int orc_llama_set_tensor(orc_llama* m, const char* role, int layer, const void* data,
                         int ggml_type, int64_t rows, int64_t cols) {
  orc_tensor t = {data, ggml_type, rows, cols};
  if (!strcmp(role, "token_embd")) { m->tok_embd = t; return 0; }
  if (!strcmp(role, "output_norm")) { m->output_norm = t; return 0; }
  if (!strcmp(role, "output")) { m->output = t; return 0; }
  if (layer < 0 || layer >= m->n_layer) { set_err("set_tensor: bad layer"); return -1; }
  orc_layer* L = &m->layers[layer];
  if (!strcmp(role, "attn_norm")) L->attn_norm = t;
  else if (!strcmp(role, "ffn_norm")) L->ffn_norm = t;
  else if (!strcmp(role, "attn_q")) L->wq = t;
  else if (!strcmp(role, "attn_k")) L->wk = t;
  else if (!strcmp(role, "attn_v")) L->wv = t;
  else if (!strcmp(role, "attn_output")) L->wo = t;
  else if (!strcmp(role, "ffn_gate")) L->wg = t;
  else if (!strcmp(role, "ffn_up")) L->wu = t;
  else if (!strcmp(role, "ffn_down")) L->wd = t;
  else { set_err("set_tensor: unknown role"); return -1; }
  return 0;
}

/* precomput_freqs_cis(rope_dim, freq_base): theta_i = 1 / base^(i/d) for
 * even i, idx_theta = p * theta, then f32 cos / sin. */
int orc_llama_finalize(orc_llama* m) {
  int half = m->rope_dim / 2;
  m->cos_t = (float*)malloc(sizeof(float) * (size_t)m->max_seq * half);
  m->sin_t = (float*)malloc(sizeof(float) * (size_t)m->max_seq * half);
  float* theta = (float*)malloc(sizeof(float) * half);
  for (int i = 0; i < m->rope_dim; i += 2)
    theta[i / 2] = 1.0f / powf(m->rope_base, (float)i / (float)m->rope_dim);
  for (int p = 0; p < m->max_seq; p++)
    for (int j = 0; j < half; j++) {
      float a = (float)p * theta[j];
      m->cos_t[(size_t)p * half + j] = cosf(a);
      m->sin_t[(size_t)p * half + j] = sinf(a);
    }
  free(theta);
  size_t kvn = (size_t)m->n_layer * m->n_head_kv * m->max_seq * m->head_dim;
  m->kc = (float*)calloc(kvn, sizeof(float));
  m->vc = (float*)calloc(kvn, sizeof(float));
  if (!m->kc || !m->vc || !m->cos_t || !m->sin_t) {
    set_err("finalize: out of memory");
    return -1;
  }
  m->kv_len = 0;
  return 0;
}

void orc_llama_free(orc_llama* m) {
  if (!m) return;
  free(m->layers);
  free(m->cos_t);
  free(m->sin_t);
  free(m->kc);
  free(m->vc);
  free(m);
}

/* candle-nn 0.8.4 ops.rs RmsNorm::cpu_fwd: sum2 = sum(v*v) (sequential f32),
 * m = sqrt(sum2/dim + eps), y = x / m * alpha. */
/* Sensitivity probe (tests only, not candle's arithmetic): 1 = accumulate
 * the rmsnorm sum of squares in f64; 2 / 3 = move the rms scale m one ulp
 * up / down; 4 = sum the squares in reverse order.
 * Either moves the normalised values by about one ulp, which is what the
 * CUDA path's different f32 summation orders do; how far the logits then
 * move is the model's own sensitivity. */
static int g_norm_variant = 0;
void orc_set_norm_variant(int v) { g_norm_variant = v; }

static void rms_norm_row(const float* x, const float* alpha, int dim, float eps, float* y) {
  float sum2 = -0.0f;
  if (g_norm_variant == 1) {
    double s = 0.0;
    for (int i = 0; i < dim; i++) s += (double)x[i] * (double)x[i];
    sum2 = (float)s;
  } else if (g_norm_variant == 4) {
    for (int i = dim - 1; i >= 0; i--) sum2 += x[i] * x[i];
  } else {
    for (int i = 0; i < dim; i++) sum2 += x[i] * x[i];
  }
  float mm = sqrtf(sum2 / (float)dim + eps);
  if (g_norm_variant == 2) mm = nextafterf(mm, INFINITY);
  if (g_norm_variant == 3) mm = nextafterf(mm, 0.0f);
  for (int i = 0; i < dim; i++) y[i] = x[i] / mm * alpha[i];
}

/* candle-nn 0.8.4 rotary_emb.rs rope_i cpu kernel, one (head,pos) row. */
static void rope_i_row(float* x, int d, const float* cs, const float* sn) {
  for (int i2 = 0; i2 < d / 2; i2++) {
    float a = x[2 * i2], b = x[2 * i2 + 1];
    x[2 * i2] = a * cs[i2] - b * sn[i2];
    x[2 * i2 + 1] = a * sn[i2] + b * cs[i2];
  }
}

static void embed_row(const orc_llama* m, uint32_t tok, float* out) {
  const orc_tensor* t = &m->tok_embd;
  int64_t rb = row_bytes(t->type, t->cols);
  const uint8_t* row = (const uint8_t*)t->p + (int64_t)tok * rb;
  orc_dequant_row(t->type, row, t->cols, out);
}

static int qmm(const orc_tensor* t, const float* x, int64_t m, float* out) {
  return orc_qmatmul(t->p, t->type, t->rows, t->cols, x, m, out);
}

/* ModelWeights::forward(x, index_pos), returning last-position logits. */
int orc_llama_forward(orc_llama* m, const uint32_t* tokens, int S, int index_pos, float* logits) {
  const int E = m->n_embd, H = m->n_head, HKV = m->n_head_kv, D = m->head_dim, F = m->n_ff;
  const int QN = H * D, KN = HKV * D;
  if (S <= 0) { set_err("forward: empty input"); return -1; }
  if (index_pos + S > m->max_seq) {
    set_err("forward: position beyond the rotary table (MAX_SEQ_LEN)");
    return -1;
  }
  if (index_pos == 0) m->kv_len = 0; /* cache replaced when index_pos == 0 */
  if (S > 1 && m->kv_len != 0) {
    set_err("forward: mask shape does not broadcast to the attention shape");
    return -1;
  }
  for (int s = 0; s < S; s++)
    if (tokens[s] >= (uint32_t)m->n_vocab) { set_err("forward: token id out of range"); return -1; }
  const int T = m->kv_len + S;
  float* x = (float*)malloc(sizeof(float) * (size_t)S * E);
  float* xn = (float*)malloc(sizeof(float) * (size_t)S * E);
  float* q = (float*)malloc(sizeof(float) * (size_t)S * QN);
  float* kk = (float*)malloc(sizeof(float) * (size_t)S * KN);
  float* vv = (float*)malloc(sizeof(float) * (size_t)S * KN);
  float* y = (float*)malloc(sizeof(float) * (size_t)S * QN);
  float* ao = (float*)malloc(sizeof(float) * (size_t)S * E);
  float* g = (float*)malloc(sizeof(float) * (size_t)S * F);
  float* u = (float*)malloc(sizeof(float) * (size_t)S * F);
  int rc = 0;
  for (int s = 0; s < S; s++) embed_row(m, tokens[s], x + (size_t)s * E);
  const float scale = (float)(1.0 / sqrt((double)D));
  const int half = m->rope_dim / 2;
  for (int l = 0; l < m->n_layer && rc == 0; l++) {
    orc_layer* L = &m->layers[l];
    for (int s = 0; s < S; s++)
      rms_norm_row(x + (size_t)s * E, (const float*)L->attn_norm.p, E, m->eps, xn + (size_t)s * E);
    rc |= qmm(&L->wq, xn, S, q);
    rc |= qmm(&L->wk, xn, S, kk);
    rc |= qmm(&L->wv, xn, S, vv);
    for (int s = 0; s < S; s++) {
      const float* cs = m->cos_t + (size_t)(index_pos + s) * half;
      const float* sn = m->sin_t + (size_t)(index_pos + s) * half;
      for (int h = 0; h < H; h++) rope_i_row(q + (size_t)s * QN + h * D, D, cs, sn);
      for (int h = 0; h < HKV; h++) rope_i_row(kk + (size_t)s * KN + h * D, D, cs, sn);
    }
    size_t lbase = (size_t)l * HKV * m->max_seq * D;
    for (int s = 0; s < S; s++)
      for (int h = 0; h < HKV; h++) {
        size_t o = lbase + ((size_t)h * m->max_seq + (m->kv_len + s)) * D;
        memcpy(m->kc + o, kk + (size_t)s * KN + h * D, sizeof(float) * D);
        memcpy(m->vc + o, vv + (size_t)s * KN + h * D, sizeof(float) * D);
        if (m->kv_f16)
          for (int d = 0; d < D; d++) {
            m->kc[o + d] = round_f16(m->kc[o + d]);
            m->vc[o + d] = round_f16(m->vc[o + d]);
          }
      }
    const int nrep = H / HKV;
#pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; h++)
      for (int s = 0; s < S; s++) {
        const int kvh = h / nrep; /* repeat_kv */
        const float* K = m->kc + lbase + (size_t)kvh * m->max_seq * D;
        const float* V = m->vc + lbase + (size_t)kvh * m->max_seq * D;
        const float* qs = q + (size_t)s * QN + h * D;
        float* sc = (float*)malloc(sizeof(float) * (size_t)T);
        for (int t = 0; t < T; t++) {
          float acc = 0.f;
          for (int d = 0; d < D; d++) acc += qs[d] * K[(size_t)t * D + d];
          sc[t] = acc * scale;
          if (S > 1 && t > s) sc[t] = -INFINITY; /* masked_fill(j > i) */
        }
        float mx = sc[0];
        for (int t = 1; t < T; t++) mx = fmaxf(mx, sc[t]);
        float sum = 0.f;
        for (int t = 0; t < T; t++) {
          sc[t] = expf(sc[t] - mx);
          sum += sc[t];
        }
        for (int t = 0; t < T; t++) sc[t] /= sum;
        float* yo = y + (size_t)s * QN + h * D;
        for (int d = 0; d < D; d++) {
          float acc = 0.f;
          for (int t = 0; t < T; t++) acc += sc[t] * V[(size_t)t * D + d];
          yo[d] = acc;
        }
        free(sc);
      }
    rc |= qmm(&L->wo, y, S, ao);
    for (size_t i = 0; i < (size_t)S * E; i++) x[i] = ao[i] + x[i];
    for (int s = 0; s < S; s++)
      rms_norm_row(x + (size_t)s * E, (const float*)L->ffn_norm.p, E, m->eps, xn + (size_t)s * E);
    rc |= qmm(&L->wg, xn, S, g);
    rc |= qmm(&L->wu, xn, S, u);
    for (size_t i = 0; i < (size_t)S * F; i++) {
      float v = g[i];
      g[i] = (v / (1.0f + expf(-v))) * u[i]; /* silu(w1 x) * (w3 x) */
    }
    rc |= qmm(&L->wd, g, S, ao);
    for (size_t i = 0; i < (size_t)S * E; i++) x[i] = ao[i] + x[i];
  }
  if (rc == 0) {
    rms_norm_row(x + (size_t)(S - 1) * E, (const float*)m->output_norm.p, E, m->eps, xn);
    rc = qmm(&m->output, xn, 1, logits);
    m->kv_len = T;
  }
  free(x); free(xn); free(q); free(kk); free(vv); free(y); free(ao); free(g); free(u);
  return rc;
}

/* llama_candle.rs:145-176: first maximum, strict '>', NEG_INFINITY start. */
uint32_t orc_argmax(const float* v, int64_t n) {
  int64_t bi = 0;
  float bv = -INFINITY;
  for (int64_t i = 0; i < n; i++)
    if (v[i] > bv) { bi = i; bv = v[i]; }
  return (uint32_t)bi;
}

static uint64_t now_us(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (uint64_t)ts.tv_sec * 1000000ull + (uint64_t)ts.tv_nsec / 1000ull;
}

/* llama_candle.rs:69-137 generate_greedy_with. */
int orc_llama_generate(orc_llama* m, const uint32_t* prompt, int n_prompt, int max_new,
                       const uint32_t* stop, int n_stop, uint32_t* out, int* n_out,
                       uint64_t* prefill_us, uint64_t* decode_us) {
  *n_out = 0;
  *prefill_us = 0;
  *decode_us = 0;
  if (max_new == 0 || n_prompt == 0) return 0;
  float* logits = (float*)malloc(sizeof(float) * (size_t)m->n_vocab);
  uint64_t t0 = now_us();
  if (orc_llama_forward(m, prompt, n_prompt, 0, logits)) { free(logits); return -1; }
  *prefill_us = now_us() - t0;
  uint32_t next = orc_argmax(logits, m->n_vocab);
  out[(*n_out)++] = next;
  uint64_t t1 = now_us();
  int offset = n_prompt;
  for (int i = 1; i < max_new; i++) {
    int is_stop = 0;
    for (int j = 0; j < n_stop; j++) is_stop |= (stop[j] == next);
    if (is_stop) break;
    if (orc_llama_forward(m, &next, 1, offset, logits)) { free(logits); return -1; }
    next = orc_argmax(logits, m->n_vocab);
    out[(*n_out)++] = next;
    offset += 1;
  }
  *decode_us = now_us() - t1;
  free(logits);
  return 0;
}

/* ------------------------------------------------------------------ */
/* Reference primitives: native/arm_ai_nif/src/shape_ops.rs             */
/* ------------------------------------------------------------------ */

/* shape_ops.rs:1364-1370 int8_dot (non-aarch64 scalar). */
static int32_t int8_dot(const int8_t* a, const int8_t* w, int64_t k) {
  int32_t total = 0;
  for (int64_t i = 0; i < k; i++) total += (int32_t)a[i] * (int32_t)w[i];
  return total;
}

/* shape_ops.rs:1169-1211 int8_matmul_f32. */
int orc_int8_matmul_f32(const int8_t* a, const int8_t* w, float act_scale, const float* w_scales,
                        int64_t m, int64_t n, int64_t k, float* out) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t i = 0; i < m; i++)
    for (int64_t j = 0; j < n; j++)
      out[i * n + j] = ((float)int8_dot(a + i * k, w + j * k, k)) * act_scale * w_scales[j];
  return 0;
}

/* shape_ops.rs:1222-1264 int8_matmul_f32_per_token. */
int orc_int8_matmul_f32_per_token(const int8_t* a, const int8_t* w, const float* act_scales,
                                  const float* w_scales, int64_t m, int64_t n, int64_t k,
                                  float* out) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t i = 0; i < m; i++)
    for (int64_t j = 0; j < n; j++)
      out[i * n + j] = ((float)int8_dot(a + i * k, w + j * k, k)) * act_scales[i] * w_scales[j];
  return 0;
}

/* The s32 accumulators of the two functions above (s8 x s8 -> s32 GEMM). */
int orc_int8_matmul_s32(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                        int32_t* out) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t i = 0; i < m; i++)
    for (int64_t j = 0; j < n; j++) out[i * n + j] = int8_dot(a + i * k, w + j * k, k);
  return 0;
}

/* shape_ops.rs:1273-1292 quantize_int8_per_token. */
int orc_quantize_int8_per_token(const float* a, int64_t m, int64_t k, int8_t* q, float* scales) {
  for (int64_t mi = 0; mi < m; mi++) {
    const float* row = a + mi * k;
    float max_abs = 0.f;
    for (int64_t j = 0; j < k; j++) max_abs = fmaxf(max_abs, fabsf(row[j]));
    float scale = max_abs > 0.f ? max_abs / 127.0f : 1.0f;
    scales[mi] = scale;
    for (int64_t j = 0; j < k; j++) {
      int32_t v = sat_i32(roundf(row[j] / scale));
      q[mi * k + j] = (int8_t)(v < -127 ? -127 : (v > 127 ? 127 : v));
    }
  }
  return 0;
}

/* shape_ops.rs:3175-3236 int4_matmul_f32 (also the x86 body of
 * int4_matmul_gemv_neon, shape_ops.rs:3157-3166). */
int orc_int4_matmul_f32(const float* a, const uint8_t* w_packed, const float* w_scales, int64_t m,
                        int64_t n, int64_t k, float* out) {
  if (k % 32 != 0) { set_err("int4_matmul: K must be a multiple of 32"); return -1; }
  const int64_t ng = k / 32, bpr = k / 2;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t mi = 0; mi < m; mi++)
    for (int64_t ni = 0; ni < n; ni++) {
      const float* ar = a + mi * k;
      const uint8_t* wr = w_packed + ni * bpr;
      const float* sr = w_scales + ni * ng;
      float acc = 0.f;
      for (int64_t g = 0; g < ng; g++) {
        float scale = sr[g], gacc = 0.f;
        for (int j = 0; j < 16; j++) {
          uint8_t byte = wr[g * 16 + j];
          int32_t lo = (int32_t)(byte & 0x0F) - 8;
          int32_t hi = (int32_t)((byte >> 4) & 0x0F) - 8;
          float alo = ar[g * 32 + 2 * j], ahi = ar[g * 32 + 2 * j + 1];
          gacc += alo * (float)lo + ahi * (float)hi;
        }
        acc += gacc * scale;
      }
      out[mi * n + ni] = acc;
    }
  return 0;
}

/* shape_ops.rs:2923-3028 int4_matmul_gemv_q4_x_q8_neon (the aarch64
 * semantics: Q8_0-style activations, integer group dots). */
int orc_int4_matmul_q4_x_q8(const float* a, const uint8_t* w_packed, const float* w_scales,
                            int64_t n, int64_t k, float* out) {
  if (k % 32 != 0) { set_err("int4_matmul: K must be a multiple of 32"); return -1; }
  const int64_t ng = k / 32, bpr = k / 2;
  int8_t* ai = (int8_t*)malloc((size_t)k);
  float* as = (float*)malloc(sizeof(float) * (size_t)ng);
  for (int64_t g = 0; g < ng; g++) {
    const float* grp = a + g * 32;
    float max_abs = 0.f;
    for (int i = 0; i < 32; i++) {
      float av = fabsf(grp[i]);
      if (av > max_abs) max_abs = av;
    }
    float scale = max_abs > 0.f ? max_abs / 127.0f : 1.0f;
    as[g] = scale;
    float inv = 1.0f / scale;
    for (int i = 0; i < 32; i++) {
      float qv = roundf(grp[i] * inv);
      /* f32::clamp(-128, 127) keeps NaN; `as i8` maps NaN to 0 */
      ai[g * 32 + i] = (qv != qv) ? 0 : sat_i8(fmaxf(-128.f, fminf(qv, 127.f)));
    }
  }
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < n; j++) {
    const uint8_t* wr = w_packed + j * bpr;
    const float* sr = w_scales + j * ng;
    float total = 0.f;
    for (int64_t g = 0; g < ng; g++) {
      int32_t dot = 0;
      for (int i = 0; i < 16; i++) {
        uint8_t byte = wr[g * 16 + i];
        dot += ((int32_t)(byte & 0x0F) - 8) * ai[g * 32 + 2 * i];
        dot += ((int32_t)(byte >> 4) - 8) * ai[g * 32 + 2 * i + 1];
      }
      total += (float)dot * sr[g] * as[g];
    }
    out[j] = total;
  }
  free(ai);
  free(as);
  return 0;
}

/* shape_ops.rs:3242-3275 quantize_int4_q4_0. */
int orc_quantize_int4_q4_0(const float* w, int64_t n, int64_t k, uint8_t* packed, float* scales) {
  if (k % 32 != 0) { set_err("quantize_int4: K must be a multiple of 32"); return -1; }
  const int64_t ng = k / 32;
  for (int64_t ni = 0; ni < n; ni++)
    for (int64_t g = 0; g < ng; g++) {
      const float* grp = w + ni * k + g * 32;
      float max_abs = 0.f;
      for (int i = 0; i < 32; i++) max_abs = fmaxf(max_abs, fabsf(grp[i]));
      float scale = max_abs > 0.f ? max_abs / 7.0f : 1.0f;
      scales[ni * ng + g] = scale;
      for (int j = 0; j < 16; j++) {
        float xlo = grp[2 * j] / scale, xhi = grp[2 * j + 1] / scale;
        int32_t qlo = sat_i32(roundf(xlo)), qhi = sat_i32(roundf(xhi));
        qlo = (qlo < -8 ? -8 : (qlo > 7 ? 7 : qlo)) + 8;
        qhi = (qhi < -8 ? -8 : (qhi > 7 ? 7 : qhi)) + 8;
        packed[ni * (k / 2) + g * 16 + j] = (uint8_t)(((uint32_t)qhi << 4) | (uint32_t)qlo);
      }
    }
  return 0;
}

/* shape_ops.rs:976-1018 rmsnorm_f32. */
int orc_rmsnorm_f32(const float* x, const float* gamma, int64_t n_outer, int64_t inner, float eps,
                    float* out) {
  const float inv_n = 1.0f / (float)inner;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n_outer; i++) {
    const float* r = x + i * inner;
    float sumsq = 0.f;
    for (int64_t j = 0; j < inner; j++) sumsq += r[j] * r[j];
    float inv_rms = 1.0f / sqrtf(sumsq * inv_n + eps);
    for (int64_t j = 0; j < inner; j++) out[i * inner + j] = r[j] * inv_rms * gamma[j];
  }
  return 0;
}

/* shape_ops.rs:464-558 flash_attention_f32. */
int orc_flash_attention_f32(const float* q, const float* k, const float* v, float scale,
                            int64_t b, int64_t h, int64_t sq, int64_t sk, int64_t d, int causal,
                            float* out) {
#pragma omp parallel for schedule(dynamic)
  for (int64_t bh = 0; bh < b * h; bh++) {
    const float* qb = q + bh * sq * d;
    const float* kb = k + bh * sk * d;
    const float* vb = v + bh * sk * d;
    float* ob = out + bh * sq * d;
    float* o = (float*)malloc(sizeof(float) * (size_t)d);
    for (int64_t i = 0; i < sq; i++) {
      float mm = -INFINITY, l = 0.f;
      for (int64_t x = 0; x < d; x++) o[x] = 0.f;
      int64_t lim = causal ? i + 1 : sk;
      for (int64_t j = 0; j < lim; j++) {
        float s = 0.f;
        for (int64_t x = 0; x < d; x++) s += qb[i * d + x] * kb[j * d + x];
        s *= scale;
        if (s > mm) {
          float m_new = s;
          float factor = expf(mm - m_new);
          for (int64_t x = 0; x < d; x++) o[x] = o[x] * factor + 1.0f * vb[j * d + x];
          l = l * factor + 1.0f;
          mm = m_new;
        } else {
          float p = expf(s - mm);
          for (int64_t x = 0; x < d; x++) o[x] += p * vb[j * d + x];
          l += p;
        }
      }
      float inv_l = l > 0.f ? 1.0f / l : 0.f;
      for (int64_t x = 0; x < d; x++) ob[i * d + x] = o[x] * inv_l;
    }
    free(o);
  }
  return 0;
}

/* shape_ops.rs:1525-1582 dequant_matmul_int8_f32. */
int orc_dequant_matmul_int8_f32(const float* act, const int8_t* w, const float* scales, int64_t b,
                                int64_t m, int64_t n, int64_t k, float* out) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t r = 0; r < b * m; r++)
    for (int64_t j = 0; j < n; j++) {
      const float* ar = act + r * k;
      const int8_t* wr = w + j * k;
      float acc = 0.f;
      for (int64_t kk = 0; kk < k; kk++) acc += ar[kk] * (float)wr[kk];
      out[r * n + j] = acc * scales[j];
    }
  return 0;
}

/* shape_ops.rs:1040-1100 rope_f32: row r uses positions[r / heads_per_token];
 * pairs (2k, 2k+1) rotated by theta = (f32)pos * inv_freq[k]. */
int orc_rope_f32(const float* x, const int64_t* positions, const float* inv_freq, int64_t n_rows,
                 int64_t head_dim, int64_t heads_per_token, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t row = 0; row < n_rows; row++) {
    const float pos = (float)positions[row / heads_per_token];
    const float* in = x + row * head_dim;
    float* o = out + row * head_dim;
    for (int64_t k = 0; k < head_dim / 2; k++) {
      const float theta = pos * inv_freq[k];
      const float c = cosf(theta), s = sinf(theta);
      const float x0 = in[2 * k], x1 = in[2 * k + 1];
      o[2 * k] = x0 * c - x1 * s;
      o[2 * k + 1] = x0 * s + x1 * c;
    }
  }
  return 0;
}

/* shape_ops.rs:2719-2751 softmax_last_axis_f32: max scanned from src[0]
 * (replaced on v > max), e = exp(x - max) summed in order, then e * (1/sum). */
int orc_softmax_last_axis_f32(const float* x, int64_t outer, int64_t inner, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < outer; r++) {
    const float* src = x + r * inner;
    float* row = out + r * inner;
    float max = src[0];
    for (int64_t i = 1; i < inner; i++)
      if (src[i] > max) max = src[i];
    float sum = 0.f;
    for (int64_t i = 0; i < inner; i++) {
      const float e = expf(src[i] - max);
      row[i] = e;
      sum += e;
    }
    const float inv = 1.0f / sum;
    for (int64_t i = 0; i < inner; i++) row[i] *= inv;
  }
  return 0;
}

/* shape_ops.rs:2755-2770 silu_gate_mul_up_f32: g * (1 / (1 + exp(-g))) * u. */
int orc_silu_gate_mul_up_f32(const float* gate, const float* up, int64_t n, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) {
    const float g = gate[i];
    const float sig = 1.0f / (1.0f + expf(-g));
    out[i] = g * sig * up[i];
  }
  return 0;
}

/* shape_ops.rs:2848-2899 dequantize_q6_k, as the reference writes it: the
 * sub-scales of each 32-value group are scales[8n + {0, 2, 4, 6}] for every
 * l (ggml's dequantize_row_q6_K would add l / 16), and they are read from a
 * `&[u8]` slice and widened with `as i32` (shape_ops.rs:2860,2887-2890), so
 * they are UNSIGNED 0..255 (ggml's block_q6_K holds int8 scales). */
int orc_dequantize_q6_k(const uint8_t* in, int64_t n_blocks, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < n_blocks; b++) {
    const uint8_t* blk = in + b * 210;
    float* o = out + b * 256;
    const uint8_t* ql = blk;
    const uint8_t* qh = blk + 128;
    const uint8_t* sc = blk + 192; /* u8 -> i32: zero-extended */
    const float d = orc_f16_to_f32((uint16_t)(blk[208] | (blk[209] << 8)));
    for (int n = 0; n < 2; n++) {
      for (int l = 0; l < 32; l++) {
        const uint8_t qhi = qh[32 * n + l];
        const int q1 = ((ql[64 * n + l] & 0xF) | (((qhi >> 0) & 3) << 4)) - 32;
        const int q2 = ((ql[64 * n + l + 32] & 0xF) | (((qhi >> 2) & 3) << 4)) - 32;
        const int q3 = (((ql[64 * n + l] >> 4) & 0xF) | (((qhi >> 4) & 3) << 4)) - 32;
        const int q4 = (((ql[64 * n + l + 32] >> 4) & 0xF) | (((qhi >> 6) & 3) << 4)) - 32;
        o[128 * n + l] = d * (float)((int)sc[8 * n + 0] * q1);
        o[128 * n + l + 32] = d * (float)((int)sc[8 * n + 2] * q2);
        o[128 * n + l + 64] = d * (float)((int)sc[8 * n + 4] * q3);
        o[128 * n + l + 96] = d * (float)((int)sc[8 * n + 6] * q4);
      }
    }
  }
  return 0;
}

/* shape_ops.rs:1462-1490 dequant_matmul_f16_f32 (x86 path): out[r][j] = sum
 * over k in order of a[r][k] * f32(w[j][k]). */
int orc_dequant_matmul_f16_f32(const float* act, const uint16_t* w, int64_t b, int64_t m, int64_t n,
                               int64_t k, float* out) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t r = 0; r < b * m; r++)
    for (int64_t j = 0; j < n; j++) {
      const float* a = act + r * k;
      const uint16_t* wr = w + j * k;
      float total = 0.f;
      for (int64_t kk = 0; kk < k; kk++) total += a[kk] * orc_f16_to_f32(wr[kk]);
      out[r * n + j] = total;
    }
  return 0;
}
