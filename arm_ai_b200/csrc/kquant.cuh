// kquant.cuh — device-side GGML k-quant arithmetic for sm_100a.
//
// Restates, as warp-cooperative device code, the semantics of candle-core
// 0.8.4's k_quants.rs (the crate the reference calls from
// native/arm_ai_nif/src/llama_candle.rs:17-19):
//   * BlockQ8K::from_float  — q8k_quant_block_warp
//   * BlockQ4K / BlockQ6K vec_dot with a Q8_K lhs — q4k_row_dot / q6k_row_dot
//   * BlockQ4K::to_float     — q4k_dequant_row
// The integer parts (the Q8_K bytes, bsums and per-super-block integer sums)
// are bit-exact with candle; only the f32 combine order of the per-block
// partial sums differs.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"

namespace armai {

__device__ __forceinline__ float h2f(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// Q8_K activations, laid out for dp4a: qs[k] int8, d[k/256] f32, bs[k/16] i32.
// ---------------------------------------------------------------------------
struct ActQ8 {
  int8_t* qs;
  float* d;
  int32_t* bs;
};

// One 256-value Q8_K block, computed by one warp. Lane l owns values
// [8l, 8l+8). Matches BlockQ8K::from_float: the scale comes from the value of
// largest magnitude (first one on ties), iscale = -128/max, q =
// min(round_half_away(iscale*x), 127) saturated to i8, d = 1/iscale, bsums
// over 16-value groups; an all-zero block gives d = 0 and zero bytes.
__device__ __forceinline__ void q8k_quant_block_warp(const float (&v)[8], int lane, int8_t* qs,
                                                     float* d, int32_t* bs) {
  float amax = 0.f, mx = 0.f;
  int idx = 0x7fffffff;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    float a = fabsf(v[i]);
    if (amax < a) {
      amax = a;
      mx = v[i];
      idx = 8 * lane + i;
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    float oa = __shfl_xor_sync(0xffffffffu, amax, off);
    float om = __shfl_xor_sync(0xffffffffu, mx, off);
    int oi = __shfl_xor_sync(0xffffffffu, idx, off);
    if (oa > amax || (oa == amax && oi < idx)) {
      amax = oa;
      mx = om;
      idx = oi;
    }
  }
  uint32_t w0 = 0, w1 = 0;
  int32_t s = 0;
  if (amax != 0.f) {
    const float iscale = __fdiv_rn(-128.f, mx);
#pragma unroll
    for (int i = 0; i < 8; i++) {
      float r = fminf(roundf(__fmul_rn(iscale, v[i])), 127.f);
      r = fmaxf(r, -128.f);
      int q = (int)r;
      s += q;
      uint32_t b = (uint32_t)(q & 0xff);
      if (i < 4) w0 |= b << (8 * i);
      else w1 |= b << (8 * (i - 4));
    }
    if (lane == 0) *d = __fdiv_rn(1.0f, iscale);
  } else {
    if (lane == 0) *d = 0.f;
  }
  reinterpret_cast<uint2*>(qs)[lane] = make_uint2(w0, w1);
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  if ((lane & 1) == 0) bs[lane >> 1] = s;
}

// ---------------------------------------------------------------------------
// Q4_K: 144-byte super-block {f16 d, f16 dmin, u8 scales[12], u8 qs[128]}.
// Sub-block j (32 values) has 6-bit scale sc_j and min m_j; value =
// d*sc_j*q - dmin*m_j. qs byte 32c+l holds value 64c+l (low nibble) and
// 64c+32+l (high nibble).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int j, int& sc, int& m) {
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// Integer part of one lane's quarter of a Q4_K x Q8_K super-block dot.
// Lane t (0..3) covers sub-blocks 2t and 2t+1 (qs bytes [32t, 32t+32)).
// Returns isum = sc_2t*<q,q8> + sc_2t+1*<q,q8>, msum = m_2t*bs + m_2t+1*bs.
__device__ __forceinline__ void q4k_quarter_ints(const uint8_t* blk, int t, const int8_t* q8blk,
                                                 const int32_t* bsblk, int& isum, int& msum) {
  const int4 qa = *reinterpret_cast<const int4*>(blk + 16 + 32 * t);
  const int4 qb = *reinterpret_cast<const int4*>(blk + 16 + 32 * t + 16);
  const int4* q8v = reinterpret_cast<const int4*>(q8blk + 64 * t);
  const int4 y0 = q8v[0], y1 = q8v[1], y2 = q8v[2], y3 = q8v[3];
  const uint32_t w[8] = {(uint32_t)qa.x, (uint32_t)qa.y, (uint32_t)qa.z, (uint32_t)qa.w,
                         (uint32_t)qb.x, (uint32_t)qb.y, (uint32_t)qb.z, (uint32_t)qb.w};
  const int ylo[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
  const int yhi[8] = {y2.x, y2.y, y2.z, y2.w, y3.x, y3.y, y3.z, y3.w};
  int dlo = 0, dhi = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    dlo = __dp4a((int)(w[i] & 0x0F0F0F0Fu), ylo[i], dlo);
    dhi = __dp4a((int)((w[i] >> 4) & 0x0F0F0F0Fu), yhi[i], dhi);
  }
  int sa, ma, sb, mb;
  q4k_scale_min(blk + 4, 2 * t, sa, ma);
  q4k_scale_min(blk + 4, 2 * t + 1, sb, mb);
  isum = sa * dlo + sb * dhi;
  msum = ma * (bsblk[4 * t] + bsblk[4 * t + 1]) + mb * (bsblk[4 * t + 2] + bsblk[4 * t + 3]);
}

// Full-warp dot of one Q4_K row (nb super-blocks, 144 B each, at `row`)
// with a Q8_K vector. Four lanes per super-block, eight super-blocks per
// pass; the four lanes' integers are summed exactly before the f32 combine
// d*isum - dmin*msum. Result valid in every lane.
__device__ __forceinline__ float q4k_row_dot(const uint8_t* row, int nb, const ActQ8& a,
                                             int lane) {
  const int t = lane & 3;
  float acc = 0.f;
  for (int b0 = 0; b0 < nb; b0 += 8) {
    const int b = b0 + (lane >> 2);
    int isum = 0, msum = 0;
    float dx = 0.f, dmx = 0.f;
    if (b < nb) {
      const uint8_t* blk = row + (int64_t)b * Q4K_BLOCK_BYTES;
      q4k_quarter_ints(blk, t, a.qs + b * QK_K, a.bs + b * 16, isum, msum);
      const uint32_t hd = *reinterpret_cast<const uint32_t*>(blk);
      dx = h2f((uint16_t)(hd & 0xffffu));
      dmx = h2f((uint16_t)(hd >> 16));
    }
    isum += __shfl_xor_sync(0xffffffffu, isum, 1);
    isum += __shfl_xor_sync(0xffffffffu, isum, 2);
    msum += __shfl_xor_sync(0xffffffffu, msum, 1);
    msum += __shfl_xor_sync(0xffffffffu, msum, 2);
    if (t == 0 && b < nb) {
      const float dy = a.d[b];
      acc += __fmul_rn(dx, dy) * (float)isum - __fmul_rn(dmx, dy) * (float)msum;
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  return acc;
}

// ---------------------------------------------------------------------------
// Q6_K (device layout): per row nb bodies of 208 B {ql[128], qh[64],
// i8 scales[16]} then nb f16 d values. Lane unit u = 2n + lh (n = half of the
// block, lh = 16-value slice) covers values 128n + 16lh + 32g + [0,16) for
// g = 0..3, each with scale 8n + lh + 2g. Value = d*scale*(q6 - 32).
// ---------------------------------------------------------------------------
__device__ __forceinline__ int q6k_unit_ints(const uint8_t* body, int u, const int8_t* q8blk,
                                             const int32_t* bsblk) {
  const int n = u >> 1, lh = u & 1;
  const int4 L = *reinterpret_cast<const int4*>(body + 64 * n + 16 * lh);
  const int4 Hh = *reinterpret_cast<const int4*>(body + 64 * n + 32 + 16 * lh);
  const int4 Q = *reinterpret_cast<const int4*>(body + 128 + 32 * n + 16 * lh);
  const uint32_t lw[4] = {(uint32_t)L.x, (uint32_t)L.y, (uint32_t)L.z, (uint32_t)L.w};
  const uint32_t hw[4] = {(uint32_t)Hh.x, (uint32_t)Hh.y, (uint32_t)Hh.z, (uint32_t)Hh.w};
  const uint32_t qw[4] = {(uint32_t)Q.x, (uint32_t)Q.y, (uint32_t)Q.z, (uint32_t)Q.w};
  const int8_t* base = q8blk + 128 * n + 16 * lh;
  const int4 y1 = *reinterpret_cast<const int4*>(base);
  const int4 y2 = *reinterpret_cast<const int4*>(base + 32);
  const int4 y3 = *reinterpret_cast<const int4*>(base + 64);
  const int4 y4 = *reinterpret_cast<const int4*>(base + 96);
  const int a1[4] = {y1.x, y1.y, y1.z, y1.w}, a2[4] = {y2.x, y2.y, y2.z, y2.w};
  const int a3[4] = {y3.x, y3.y, y3.z, y3.w}, a4[4] = {y4.x, y4.y, y4.z, y4.w};
  int d1 = 0, d2 = 0, d3 = 0, d4 = 0;
#pragma unroll
  for (int w = 0; w < 4; w++) {
    const uint32_t q1 = (lw[w] & 0x0F0F0F0Fu) | ((qw[w] & 0x03030303u) << 4);
    const uint32_t q2 = (hw[w] & 0x0F0F0F0Fu) | (((qw[w] >> 2) & 0x03030303u) << 4);
    const uint32_t q3 = ((lw[w] >> 4) & 0x0F0F0F0Fu) | (((qw[w] >> 4) & 0x03030303u) << 4);
    const uint32_t q4 = ((hw[w] >> 4) & 0x0F0F0F0Fu) | (((qw[w] >> 6) & 0x03030303u) << 4);
    d1 = __dp4a((int)q1, a1[w], d1);
    d2 = __dp4a((int)q2, a2[w], d2);
    d3 = __dp4a((int)q3, a3[w], d3);
    d4 = __dp4a((int)q4, a4[w], d4);
  }
  const int8_t* sc = reinterpret_cast<const int8_t*>(body + 192);
  const int s0 = 8 * n + lh;
  // sum_g sc_g * (<q6u, q8> - 32 * bsum_g) == sum_g sc_g * <q6u - 32, q8>
  return (int)sc[s0] * (d1 - 32 * bsblk[s0]) + (int)sc[s0 + 2] * (d2 - 32 * bsblk[s0 + 2]) +
         (int)sc[s0 + 4] * (d3 - 32 * bsblk[s0 + 4]) + (int)sc[s0 + 6] * (d4 - 32 * bsblk[s0 + 6]);
}

__device__ __forceinline__ float q6k_row_dot(const uint8_t* row, int nb, const ActQ8& a,
                                             int lane) {
  const int u = lane & 3;
  const uint16_t* dv = reinterpret_cast<const uint16_t*>(row + (int64_t)nb * Q6K_BODY_BYTES);
  float acc = 0.f;
  for (int b0 = 0; b0 < nb; b0 += 8) {
    const int b = b0 + (lane >> 2);
    int isum = 0;
    if (b < nb)
      isum = q6k_unit_ints(row + (int64_t)b * Q6K_BODY_BYTES, u, a.qs + b * QK_K, a.bs + b * 16);
    isum += __shfl_xor_sync(0xffffffffu, isum, 1);
    isum += __shfl_xor_sync(0xffffffffu, isum, 2);
    if (u == 0 && b < nb) acc += __fmul_rn(h2f(dv[b]), a.d[b]) * (float)isum;
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  return acc;
}

__device__ __forceinline__ float row_dot(int type, const uint8_t* row, int nb, const ActQ8& a,
                                         int lane) {
  return type == GGML_Q4_K ? q4k_row_dot(row, nb, a, lane) : q6k_row_dot(row, nb, a, lane);
}

// ---------------------------------------------------------------------------
// Register-resident activation slices (the matvec kernels' inner loop).
//
// Lane l of a warp owns quarter t = l & 3 of super-block 8p + (l >> 2) in pass
// p: values [64t, 64t+64) of that block. Its slice of the Q8_K activation —
// 16 words of int8, the 4 bsums of those values and the block scale d — is
// loaded once per pass and reused for every weight row of the chunk. Both
// weight types are mapped onto the same slice:
//   Q4_K: qs bytes [32t, 32t+32): low nibbles = sub-block 2t (words 0..7),
//         high nibbles = sub-block 2t+1 (words 8..15); scales sc/m of 2t, 2t+1.
//   Q6_K: with t = 2n + h, value 64t + i (i < 64) takes ql[64n + i] nibble h
//         and qh[32n + (i & 31)] bits 4h + 2*(i >> 5); its 16-value scale is
//         sc[4t + i/16] — the same index as its Q8_K bsum.
// ---------------------------------------------------------------------------
struct ActSlice {
  uint32_t q[16];
  int bs[4];
  float dy;
};

__device__ __forceinline__ void load_slice(const ActQ8& a, int blk, int t, ActSlice& s) {
  const int4* qv = reinterpret_cast<const int4*>(a.qs + (size_t)blk * QK_K + 64 * t);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int4 v = qv[i];
    s.q[4 * i] = (uint32_t)v.x;
    s.q[4 * i + 1] = (uint32_t)v.y;
    s.q[4 * i + 2] = (uint32_t)v.z;
    s.q[4 * i + 3] = (uint32_t)v.w;
  }
  const int4 b = *reinterpret_cast<const int4*>(a.bs + (size_t)blk * 16 + 4 * t);
  s.bs[0] = b.x;
  s.bs[1] = b.y;
  s.bs[2] = b.z;
  s.bs[3] = b.w;
  s.dy = a.d[blk];
}

// Integers of one Q4_K quarter: isum = sc_2t*<q,q8> + sc_2t+1*<q,q8>,
// msum = m_2t*bs + m_2t+1*bs; also returns the block's f16 d and dmin.
__device__ __forceinline__ void q4k_quarter(const uint8_t* blk, int t, const ActSlice& A, int& isum,
                                            int& msum, float& dx, float& dmx) {
  const int4 hd = *reinterpret_cast<const int4*>(blk);
  const int4 qa = *reinterpret_cast<const int4*>(blk + 16 + 32 * t);
  const int4 qb = *reinterpret_cast<const int4*>(blk + 32 + 32 * t);
  const uint32_t w[8] = {(uint32_t)qa.x, (uint32_t)qa.y, (uint32_t)qa.z, (uint32_t)qa.w,
                         (uint32_t)qb.x, (uint32_t)qb.y, (uint32_t)qb.z, (uint32_t)qb.w};
  int dlo = 0, dhi = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    dlo = __dp4a((int)(w[i] & 0x0F0F0F0Fu), (int)A.q[i], dlo);
    dhi = __dp4a((int)((w[i] >> 4) & 0x0F0F0F0Fu), (int)A.q[8 + i], dhi);
  }
  // 12 scale bytes s[0..11] live in words hd.y (s0..3), hd.z (s4..7), hd.w (s8..11)
  const uint32_t s03 = (uint32_t)hd.y, s47 = (uint32_t)hd.z, s811 = (uint32_t)hd.w;
  int sa, ma, sb, mb;
  {
    const int j = 2 * t, j1 = 2 * t + 1;
    auto byte = [&](int i) -> uint32_t {
      const uint32_t wd = i < 4 ? s03 : (i < 8 ? s47 : s811);
      return (wd >> (8 * (i & 3))) & 0xffu;
    };
    if (t < 2) {
      sa = byte(j) & 63;  ma = byte(j + 4) & 63;
      sb = byte(j1) & 63; mb = byte(j1 + 4) & 63;
    } else {
      sa = (byte(j + 4) & 0xF) | ((byte(j - 4) >> 6) << 4);
      ma = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
      sb = (byte(j1 + 4) & 0xF) | ((byte(j1 - 4) >> 6) << 4);
      mb = (byte(j1 + 4) >> 4) | ((byte(j1) >> 6) << 4);
    }
  }
  isum = sa * dlo + sb * dhi;
  msum = ma * (A.bs[0] + A.bs[1]) + mb * (A.bs[2] + A.bs[3]);
  dx = h2f((uint16_t)((uint32_t)hd.x & 0xffffu));
  dmx = h2f((uint16_t)((uint32_t)hd.x >> 16));
}

// Integer of one Q6_K quarter: sum_g sc[4t+g] * <q6 - 32, q8> over the four
// 16-value groups of the slice. `body` is the block's 208-byte body.
__device__ __forceinline__ int q6k_quarter(const uint8_t* body, int t, const ActSlice& A) {
  const int n = t >> 1, h = t & 1;
  const int4* qlv = reinterpret_cast<const int4*>(body + 64 * n);
  const int4* qhv = reinterpret_cast<const int4*>(body + 128 + 32 * n);
  const int4 l0 = qlv[0], l1 = qlv[1], l2 = qlv[2], l3 = qlv[3];
  const int4 h0 = qhv[0], h1 = qhv[1];
  const uint32_t lw[16] = {(uint32_t)l0.x, (uint32_t)l0.y, (uint32_t)l0.z, (uint32_t)l0.w,
                           (uint32_t)l1.x, (uint32_t)l1.y, (uint32_t)l1.z, (uint32_t)l1.w,
                           (uint32_t)l2.x, (uint32_t)l2.y, (uint32_t)l2.z, (uint32_t)l2.w,
                           (uint32_t)l3.x, (uint32_t)l3.y, (uint32_t)l3.z, (uint32_t)l3.w};
  const uint32_t hw[8] = {(uint32_t)h0.x, (uint32_t)h0.y, (uint32_t)h0.z, (uint32_t)h0.w,
                          (uint32_t)h1.x, (uint32_t)h1.y, (uint32_t)h1.z, (uint32_t)h1.w};
  const uint32_t sc4 = *reinterpret_cast<const uint32_t*>(body + 192 + 4 * t);
  int tot = 0;
#pragma unroll
  for (int g = 0; g < 4; g++) {
    int dot = 0;
#pragma unroll
    for (int w4 = 0; w4 < 4; w4++) {
      const int w = 4 * g + w4;  // word w covers values 4w..4w+3 of the slice
      const uint32_t lo = (lw[w] >> (4 * h)) & 0x0F0F0F0Fu;
      const uint32_t hi = (hw[w & 7] >> (4 * h + 2 * (w >> 3))) & 0x03030303u;
      dot = __dp4a((int)(lo | (hi << 4)), (int)A.q[w], dot);
    }
    const int sc = (int)(int8_t)((sc4 >> (8 * g)) & 0xffu);
    tot += sc * (dot - 32 * A.bs[g]);
  }
  return tot;
}

// One lane's f32 share of <weight row, activation> over pass `pass`.
__device__ __forceinline__ float quarter_dot(int type, const uint8_t* row, int nb, int blk, int t,
                                             const ActSlice& A) {
  if (type == GGML_Q4_K) {
    int is, ms;
    float dx, dmx;
    q4k_quarter(row + (size_t)blk * Q4K_BLOCK_BYTES, t, A, is, ms, dx, dmx);
    return __fmul_rn(dx, A.dy) * (float)is - __fmul_rn(dmx, A.dy) * (float)ms;
  }
  const uint16_t dh = reinterpret_cast<const uint16_t*>(row + (size_t)nb * Q6K_BODY_BYTES)[blk];
  return __fmul_rn(h2f(dh), A.dy) * (float)q6k_quarter(row + (size_t)blk * Q6K_BODY_BYTES, t, A);
}

// BlockQ4K::to_float for one row, by one warp: y = (d*sc)*q - (dmin*m), with
// each product and the difference rounded separately.
__device__ __forceinline__ void q4k_dequant_row(const uint8_t* row, int nb, float* y, int lane) {
  for (int e = lane; e < nb * QK_K; e += 32) {
    const int b = e / QK_K, i = e % QK_K;
    const uint8_t* blk = row + (int64_t)b * Q4K_BLOCK_BYTES;
    const int c = i / 64, l = i % 64;
    const int j = 2 * c + (l >= 32 ? 1 : 0);
    const uint8_t byte = blk[16 + 32 * c + (l & 31)];
    const int q = l >= 32 ? (byte >> 4) : (byte & 0xF);
    int sc, m;
    q4k_scale_min(blk + 4, j, sc, m);
    const float d = h2f(*reinterpret_cast<const uint16_t*>(blk));
    const float dmin = h2f(*reinterpret_cast<const uint16_t*>(blk + 2));
    y[e] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
  }
}

// BlockQ6K::to_float for one row (device layout), by one warp:
// y = (d*sc)*(q-32).
__device__ __forceinline__ void q6k_dequant_row(const uint8_t* row, int nb, float* y, int lane) {
  const uint16_t* dv = reinterpret_cast<const uint16_t*>(row + (int64_t)nb * Q6K_BODY_BYTES);
  for (int e = lane; e < nb * QK_K; e += 32) {
    const int b = e / QK_K, i = e % QK_K;
    const uint8_t* body = row + (int64_t)b * Q6K_BODY_BYTES;
    const int n = i / 128, r = i % 128, g = r / 32, l = r % 32;
    const uint8_t qlb = body[64 * n + l + (g & 1) * 32];
    const int lo = (g < 2) ? (qlb & 0xF) : (qlb >> 4);
    const int hi = (body[128 + 32 * n + l] >> (2 * g)) & 3;
    const int q = (lo | (hi << 4)) - 32;
    const int8_t sc = reinterpret_cast<const int8_t*>(body + 192)[8 * n + l / 16 + 2 * g];
    y[e] = __fmul_rn(__fmul_rn(h2f(dv[b]), (float)sc), (float)q);
  }
}

}  // namespace armai
