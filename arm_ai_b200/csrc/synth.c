/*
 * synth.c — seeded random-init weights quantised to GGML Q4_K / Q6_K blocks.
 *
 * Builds the synthetic "Q4_K_M" models the benchmarks and parity tests run on
 * (the reference's real model files are not available here). Host-only
 * helper; not part of the CUDA path.
 *
 * Weights: w = std * N(0,1), where N(0,1) comes from a counter-based
 * generator (splitmix64 of seed + element pair index, Box-Muller in double),
 * so every element depends only on (seed, index) and the result does not
 * depend on the thread count.
 *
 * The quantisers are this project's own simple min/max fits. They produce
 * valid blocks of the public GGML layouts:
 *   Q4_K (144 B / 256 w): f16 d, f16 dmin, 12 B of packed 6-bit
 *         (scale, min) pairs for 8 sub-blocks of 32, 128 B of nibbles where
 *         byte 32c+l holds element 64c+l (low) and 64c+32+l (high).
 *   Q6_K (210 B / 256 w): 128 B low nibbles, 64 B high 2-bit pairs,
 *         16 signed 8-bit sub-block scales, f16 d.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

static inline double unit_open(uint64_t r) { /* (0, 1] */
  return ((double)(r >> 11) + 1.0) * (1.0 / 9007199254740992.0);
}

static inline float normal_at(uint64_t seed, uint64_t i) {
  uint64_t p = i >> 1;
  double u1 = unit_open(splitmix64(seed ^ (2 * p)));
  double u2 = unit_open(splitmix64(seed ^ (2 * p + 1) ^ 0x5851F42D4C957F2Dull));
  double r = sqrt(-2.0 * log(u1));
  double t = 6.283185307179586 * u2;
  return (float)((i & 1) ? r * sin(t) : r * cos(t));
}

void synth_fill_normal(float* out, int64_t n, uint64_t seed, float mean, float std) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) out[i] = mean + std * normal_at(seed, (uint64_t)i);
}

/* float -> IEEE binary16, round to nearest even. */
static uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* overflow -> inf */
  if (ax < 0x38800000u) {                                    /* subnormal / zero */
    float a;
    memcpy(&a, &ax, 4);
    float scaled = a * 16777216.0f; /* 2^24: units of the smallest subnormal */
    uint32_t m = (uint32_t)nearbyintf(scaled);
    return (uint16_t)(sign | m);
  }
  uint32_t e = ((ax >> 23) - 112u) << 10;
  uint32_t mant = ax & 0x7fffffu;
  uint32_t h = e | (mant >> 13);
  uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1fu, mant = h & 0x3ffu, bits;
  if (ex == 0) {
    if (!mant) bits = sign;
    else {
      int e = -1;
      do { e++; mant <<= 1; } while (!(mant & 0x400u));
      bits = sign | ((uint32_t)(112 - e) << 23) | ((mant & 0x3ffu) << 13);
    }
  } else if (ex == 31) bits = sign | 0x7f800000u | (mant << 13);
  else bits = sign | ((ex + 112u) << 23) | (mant << 13);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* One Q4_K super-block from 256 floats. */
static void quant_block_q4k(const float* x, uint8_t* out) {
  float scale[8], minv[8];
  float max_scale = 0.f, max_min = 0.f;
  for (int j = 0; j < 8; j++) {
    float lo = 0.f, hi = -INFINITY;
    for (int l = 0; l < 32; l++) {
      float v = x[32 * j + l];
      if (v < lo) lo = v;
      if (v > hi) hi = v;
    }
    if (hi < lo) hi = lo;
    scale[j] = (hi - lo) / 15.f;
    minv[j] = -lo;
    if (scale[j] > max_scale) max_scale = scale[j];
    if (minv[j] > max_min) max_min = minv[j];
  }
  uint16_t dh = f32_to_f16(max_scale / 63.f), mh = f32_to_f16(max_min / 63.f);
  float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
  int sc[8], mn[8];
  for (int j = 0; j < 8; j++) {
    sc[j] = d > 0.f ? clampi((int)nearbyintf(scale[j] / d), 0, 63) : 0;
    mn[j] = dmin > 0.f ? clampi((int)nearbyintf(minv[j] / dmin), 0, 63) : 0;
  }
  memcpy(out, &dh, 2);
  memcpy(out + 2, &mh, 2);
  uint8_t* s = out + 4;
  for (int j = 0; j < 4; j++) {
    s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
    s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
  }
  uint8_t q[256];
  for (int j = 0; j < 8; j++) {
    float ds = d * (float)sc[j], dm = dmin * (float)mn[j];
    for (int l = 0; l < 32; l++) {
      int v = ds > 0.f ? (int)nearbyintf((x[32 * j + l] + dm) / ds) : 0;
      q[32 * j + l] = (uint8_t)clampi(v, 0, 15);
    }
  }
  uint8_t* qs = out + 16;
  for (int c = 0; c < 4; c++)
    for (int l = 0; l < 32; l++) qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
}

/* One Q6_K super-block from 256 floats. Signed sub-scales, as llama.cpp's
 * quantiser makes them: each 16-value group's scale maps the group's value of
 * largest magnitude (the first one on ties) to -32, so a sub-scale's sign is
 * the opposite of that value's and about half of them are negative. */
static void quant_block_q6k(const float* x, uint8_t* out) {
  float scale[16], max_abs_scale = 0.f;
  for (int j = 0; j < 16; j++) {
    float amax = 0.f, mx = 0.f;
    for (int l = 0; l < 16; l++) {
      const float v = x[16 * j + l];
      if (fabsf(v) > amax) {
        amax = fabsf(v);
        mx = v;
      }
    }
    scale[j] = mx / -32.f;
    if (amax / 32.f > max_abs_scale) max_abs_scale = amax / 32.f;
  }
  uint16_t dh = f32_to_f16(max_abs_scale / 127.f);
  float d = f16_to_f32(dh);
  int8_t sc[16];
  int q[256];
  for (int j = 0; j < 16; j++) {
    sc[j] = (int8_t)(d > 0.f ? clampi((int)nearbyintf(scale[j] / d), -128, 127) : 0);
    float ds = d * (float)sc[j];
    for (int l = 0; l < 16; l++) {
      int v = ds != 0.f ? (int)nearbyintf(x[16 * j + l] / ds) : 0;
      q[16 * j + l] = clampi(v, -32, 31) + 32;
    }
  }
  uint8_t* ql = out;
  uint8_t* qh = out + 128;
  for (int n = 0; n < 2; n++)
    for (int l = 0; l < 32; l++) {
      int q1 = q[128 * n + l], q2 = q[128 * n + l + 32], q3 = q[128 * n + l + 64],
          q4 = q[128 * n + l + 96];
      ql[64 * n + l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
      ql[64 * n + l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
      qh[32 * n + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  memcpy(out + 192, sc, 16);
  memcpy(out + 208, &dh, 2);
}

int synth_quantize_q4k(const float* w, int64_t rows, int64_t k, uint8_t* out) {
  if (k % 256) return -1;
  int64_t nb = k / 256;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++)
    for (int64_t b = 0; b < nb; b++) quant_block_q4k(w + r * k + b * 256, out + (r * nb + b) * 144);
  return 0;
}

int synth_quantize_q6k(const float* w, int64_t rows, int64_t k, uint8_t* out) {
  if (k % 256) return -1;
  int64_t nb = k / 256;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++)
    for (int64_t b = 0; b < nb; b++) quant_block_q6k(w + r * k + b * 256, out + (r * nb + b) * 210);
  return 0;
}

/* Generate + quantise a [rows, k] weight tensor without an f32 copy of it.
 * qtype: 12 = Q4_K, 14 = Q6_K. */
int synth_tensor(uint64_t seed, int64_t rows, int64_t k, float std, int qtype, uint8_t* out) {
  if (k % 256) return -1;
  if (qtype != 12 && qtype != 14) return -2;
  int64_t nb = k / 256;
  int64_t bb = qtype == 12 ? 144 : 210;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) {
    float buf[256];
    for (int64_t b = 0; b < nb; b++) {
      for (int l = 0; l < 256; l++)
        buf[l] = std * normal_at(seed, (uint64_t)(r * k + b * 256 + l));
      if (qtype == 12) quant_block_q4k(buf, out + (r * nb + b) * bb);
      else quant_block_q6k(buf, out + (r * nb + b) * bb);
    }
  }
  return 0;
}
