// kquant.cuh — device-side GGML k-quant arithmetic for sm_100a.
//
// Restates, as warp-cooperative device code, the semantics of candle-core
// 0.8.4's k_quants.rs (the crate the reference calls from
// native/arm_ai_nif/src/llama_candle.rs:17-19):
//   * BlockQ8K::from_float  — q8k_quant_block_warp
//   * BlockQ4K / BlockQ6K vec_dot with a Q8_K lhs — load_slice + q4k_quarter /
//     q6k_quarter (integers) + quarter_dot (f32 combine)
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

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
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
  // The same values as candle's Q8_0 (the VecDotType of Q4_0 / Q5_0 /
  // Q8_0 weights): qs0[k] int8, d0[k/32] the f16 scale as f32, s0[k/32] the
  // block's sum of qs0. nullptr when no matrix of the phase needs them.
  int8_t* qs0;
  float* d0;
  int32_t* s0;
};

// One 256-value Q8_K block, computed by one warp. Lane l owns values
// [8l, 8l+8). Matches BlockQ8K::from_float: the scale comes from the value of
// largest magnitude (first one on ties), iscale = -128/max, q =
// min(round_half_away(iscale*x), 127) saturated to i8, d = 1/iscale, bsums
// over 16-value groups; an all-zero block gives d = 0 and zero bytes.
//
// `swz` XOR-swizzles the 16 sixteen-byte chunks of the block's qs (chunk c is
// stored at c ^ swz). Activation buffers read by load_slice use swz =
// block & 7, which spreads the 32 lanes of a slice load over all banks.
__device__ __forceinline__ void q8k_quant_block_warp(const float (&v)[8], int lane, int8_t* qs,
                                                     float* d, int32_t* bs, int swz = 0) {
  // The first value of largest magnitude: |x| compared through its bits
  // (non-negative floats order as unsigned integers), a NaN never chosen (as
  // candle's `amax < |x|` never takes one); the warp's largest key, then the
  // lowest index holding it, then that lane's signed value.
  uint32_t key = 0u;
  int ib = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float a = fabsf(v[i]);
    const uint32_t k = isnan(a) ? 0u : __float_as_uint(a);
    if (k > key) {
      key = k;
      ib = i;
    }
  }
  float mine = v[0];
#pragma unroll
  for (int i = 1; i < 8; i++)
    if (ib == i) mine = v[i];
  const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
  const uint32_t first = __reduce_min_sync(0xffffffffu, (kmax != 0u && key == kmax) ? (uint32_t)(8 * lane + ib) : 0xffffffffu);
  const float amax = __uint_as_float(kmax);
  const float mx = __shfl_sync(0xffffffffu, mine, (int)((first >> 3) & 31u));
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
  reinterpret_cast<uint2*>(qs)[(((lane >> 1) ^ swz) << 1) | (lane & 1)] = make_uint2(w0, w1);
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  if ((lane & 1) == 0) bs[lane >> 1] = s;
}

// The same 256 values as eight Q8_0 blocks of 32 (lanes 4b..4b+3 hold block
// b). Matches BlockQ8_0::from_float: d = amax / 127 (amax ignores NaN, as
// f32::max does), id = 1/d (0 when d is 0), q = round_half_away(x * id)
// saturated to i8 (NaN -> 0, as `as i8`), d kept as f16. Same chunk swizzle
// as the Q8_K bytes.
__device__ __forceinline__ void q80_quant_block_warp(const float (&v)[8], int lane, int8_t* qs, float* d,
                                                     int32_t* s, int swz = 0) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const float dd = __fdiv_rn(amax, 127.0f);
  const float id = dd != 0.f ? __fdiv_rn(1.0f, dd) : 0.f;
  uint32_t w0 = 0, w1 = 0;
  int32_t sum = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float r = roundf(__fmul_rn(v[i], id));
    const int q = isnan(r) ? 0 : (int)fmaxf(fminf(r, 127.f), -128.f);
    sum += q;
    const uint32_t b = (uint32_t)(q & 0xff);
    if (i < 4) w0 |= b << (8 * i);
    else w1 |= b << (8 * (i - 4));
  }
  reinterpret_cast<uint2*>(qs)[(((lane >> 1) ^ swz) << 1) | (lane & 1)] = make_uint2(w0, w1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  if ((lane & 3) == 0) {
    d[lane >> 2] = __half2float(__float2half_rn(dd));
    s[lane >> 2] = sum;
  }
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

// The activation's qs blocks are stored chunk-swizzled (chunk c of block b at
// c ^ (b & 7), see q8k_quant_block_warp).
__device__ __forceinline__ void load_slice(const ActQ8& a, int blk, int t, ActSlice& s) {
  const int4* qv = reinterpret_cast<const int4*>(a.qs + (size_t)blk * QK_K);
  const int swz = blk & 7;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int4 v = qv[(4 * t + i) ^ swz];
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
  // High nibbles stay in place (q << 4, u8) against signed activations:
  // the sum is exactly 16x the sub-block dot, one shift-free mask per word.
  int dlo = 0, dhi16 = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    dlo = __dp4a((int)(w[i] & 0x0F0F0F0Fu), (int)A.q[i], dlo);
    dhi16 = dp4a_us(w[i] & 0xF0F0F0F0u, A.q[8 + i], dhi16);
  }
  const int dhi = dhi16 >> 4;
  // 12 scale bytes s[0..11] live in words hd.y (s0..3), hd.z (s4..7), hd.w (s8..11).
  // All eight 6-bit scales / mins, one per byte (get_scale_min_k4 in word form):
  //   sc0..3 = s0..3 & 63            sc4..7 = (s8..11 & 15) | (s0..3 >> 6) << 4
  //   m0..3  = s4..7 & 63            m4..7  = (s8..11 >> 4) | (s4..7 >> 6) << 4
  const uint32_t s03 = (uint32_t)hd.y, s47 = (uint32_t)hd.z, s811 = (uint32_t)hd.w;
  const uint32_t scw = t < 2 ? (s03 & 0x3f3f3f3fu)
                             : ((s811 & 0x0f0f0f0fu) | ((s03 >> 2) & 0x30303030u));
  const uint32_t mw = t < 2 ? (s47 & 0x3f3f3f3fu)
                            : (((s811 >> 4) & 0x0f0f0f0fu) | ((s47 >> 2) & 0x30303030u));
  const int sh = 16 * (t & 1);  // lane t uses sub-blocks 2t, 2t+1 = bytes (2t, 2t+1) mod 4
  const int sa = (int)((scw >> sh) & 0xffu), sb = (int)((scw >> (sh + 8)) & 0xffu);
  const int ma = (int)((mw >> sh) & 0xffu), mb = (int)((mw >> (sh + 8)) & 0xffu);
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

// Integers of one Q5_K quarter: Q4_K's plus the fifth bit of each value
// (qh byte l, bit 2t for the low nibbles, 2t + 1 for the high), as
// BlockQ5K::vec_dot; the same scales / mins and combine as Q4_K.
__device__ __forceinline__ void q5k_quarter(const uint8_t* blk, int t, const ActSlice& A, int& isum, int& msum,
                                            float& dx, float& dmx) {
  const int4 hd = *reinterpret_cast<const int4*>(blk);
  const int4 h0 = *reinterpret_cast<const int4*>(blk + 16);
  const int4 h1 = *reinterpret_cast<const int4*>(blk + 32);
  const int4 qa = *reinterpret_cast<const int4*>(blk + 48 + 32 * t);
  const int4 qb = *reinterpret_cast<const int4*>(blk + 64 + 32 * t);
  const uint32_t w[8] = {(uint32_t)qa.x, (uint32_t)qa.y, (uint32_t)qa.z, (uint32_t)qa.w,
                         (uint32_t)qb.x, (uint32_t)qb.y, (uint32_t)qb.z, (uint32_t)qb.w};
  const uint32_t h[8] = {(uint32_t)h0.x, (uint32_t)h0.y, (uint32_t)h0.z, (uint32_t)h0.w,
                         (uint32_t)h1.x, (uint32_t)h1.y, (uint32_t)h1.z, (uint32_t)h1.w};
  int dlo = 0, dhi16 = 0, blo = 0, bhi = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    dlo = __dp4a((int)(w[i] & 0x0F0F0F0Fu), (int)A.q[i], dlo);
    dhi16 = dp4a_us(w[i] & 0xF0F0F0F0u, A.q[8 + i], dhi16);
    blo = __dp4a((int)((h[i] >> (2 * t)) & 0x01010101u), (int)A.q[i], blo);
    bhi = __dp4a((int)((h[i] >> (2 * t + 1)) & 0x01010101u), (int)A.q[8 + i], bhi);
  }
  const int vlo = dlo + 16 * blo, vhi = (dhi16 >> 4) + 16 * bhi;
  const uint32_t s03 = (uint32_t)hd.y, s47 = (uint32_t)hd.z, s811 = (uint32_t)hd.w;
  const uint32_t scw = t < 2 ? (s03 & 0x3f3f3f3fu) : ((s811 & 0x0f0f0f0fu) | ((s03 >> 2) & 0x30303030u));
  const uint32_t mw = t < 2 ? (s47 & 0x3f3f3f3fu) : (((s811 >> 4) & 0x0f0f0f0fu) | ((s47 >> 2) & 0x30303030u));
  const int sh = 16 * (t & 1);
  const int sa = (int)((scw >> sh) & 0xffu), sb = (int)((scw >> (sh + 8)) & 0xffu);
  const int ma = (int)((mw >> sh) & 0xffu), mb = (int)((mw >> (sh + 8)) & 0xffu);
  isum = sa * vlo + sb * vhi;
  msum = ma * (A.bs[0] + A.bs[1]) + mb * (A.bs[2] + A.bs[3]);
  dx = h2f((uint16_t)((uint32_t)hd.x & 0xffffu));
  dmx = h2f((uint16_t)((uint32_t)hd.x >> 16));
}

// Q8_0 activation slice of lane (super-block blk, quarter t): values
// [256 blk + 64 t, + 64) = legacy blocks 8 blk + 2t and 8 blk + 2t + 1.
struct ActSlice0 {
  uint32_t q[16];
  float d[2];
  int s[2];
};
__device__ __forceinline__ void load_slice0(const ActQ8& a, int blk, int t, ActSlice0& s) {
  const int4* qv = reinterpret_cast<const int4*>(a.qs0 + (size_t)blk * QK_K);
  const int swz = blk & 7;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int4 v = qv[(4 * t + i) ^ swz];
    s.q[4 * i] = (uint32_t)v.x;
    s.q[4 * i + 1] = (uint32_t)v.y;
    s.q[4 * i + 2] = (uint32_t)v.z;
    s.q[4 * i + 3] = (uint32_t)v.w;
  }
  const float2 dd = *reinterpret_cast<const float2*>(a.d0 + 8 * blk + 2 * t);
  const int2 ss = *reinterpret_cast<const int2*>(a.s0 + 8 * blk + 2 * t);
  s.d[0] = dd.x;
  s.d[1] = dd.y;
  s.s[0] = ss.x;
  s.s[1] = ss.y;
}

// Words [i0, i0 + n) of a byte sequence that starts 2 bytes past a 4-byte
// boundary (w = the aligned words covering it).
__device__ __forceinline__ uint32_t shr16(uint32_t lo, uint32_t hi) { return __funnelshift_r(lo, hi, 16); }

// One lane's share of a legacy-type row against the Q8_0 activation: two
// 32-value blocks, each sumf += (float)sumi * d_x * d_y in candle's order
// (k_quants.rs BlockQ4_0 / BlockQ5_0 / BlockQ8_0 ::vec_dot); the two blocks'
// terms are added here and across lanes afterwards. `row` is 4-byte aligned
// (rows start 16-byte aligned; two blocks span a multiple of 4 bytes).
__device__ __forceinline__ float legacy_pair_dot(int type, const uint8_t* row, int blk, int t, const ActSlice0& B) {
  const int bb = legacy_block_bytes(type);
  const uint32_t* wp = reinterpret_cast<const uint32_t*>(row + (size_t)(8 * blk + 2 * t) * bb);
  int sumi[2];
  float dx[2];
  if (type == GGML_Q4_0) {  // 36 bytes: d | 16 qs | d | 16 qs
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; i++) w[i] = wp[i];
    const uint32_t qa[4] = {shr16(w[0], w[1]), shr16(w[1], w[2]), shr16(w[2], w[3]), shr16(w[3], w[4])};
    const uint32_t qb[4] = {w[5], w[6], w[7], w[8]};
    dx[0] = h2f((uint16_t)(w[0] & 0xffffu));
    dx[1] = h2f((uint16_t)(w[4] >> 16));
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint32_t* q = h ? qb : qa;
      int acc = 0;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        acc = __dp4a((int)(q[i] & 0x0F0F0F0Fu), (int)B.q[8 * h + i], acc);
        acc = __dp4a((int)((q[i] >> 4) & 0x0F0F0F0Fu), (int)B.q[8 * h + 4 + i], acc);
      }
      sumi[h] = acc - 8 * B.s[h];
    }
  } else if (type == GGML_Q5_0) {  // 44 bytes: d | qh(4) | 16 qs | d | qh(4) | 16 qs
    uint32_t w[11];
#pragma unroll
    for (int i = 0; i < 11; i++) w[i] = wp[i];
    const uint32_t qha = shr16(w[0], w[1]);
    const uint32_t qa[4] = {shr16(w[1], w[2]), shr16(w[2], w[3]), shr16(w[3], w[4]), shr16(w[4], w[5])};
    const uint32_t qhb = w[6];
    const uint32_t qb[4] = {w[7], w[8], w[9], w[10]};
    dx[0] = h2f((uint16_t)(w[0] & 0xffffu));
    dx[1] = h2f((uint16_t)(w[5] >> 16));
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint32_t* q = h ? qb : qa;
      const uint32_t qh = h ? qhb : qha;
      int acc = 0;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        // bit j of qh -> bit 4 of value j's byte (values 4i..4i+3), and
        // bit j + 16 for the high nibbles
        const uint32_t lo = (q[i] & 0x0F0F0F0Fu) | ((((qh >> (4 * i)) & 0xFu) * 0x00204081u & 0x01010101u) << 4);
        const uint32_t hi = ((q[i] >> 4) & 0x0F0F0F0Fu) |
                            ((((qh >> (16 + 4 * i)) & 0xFu) * 0x00204081u & 0x01010101u) << 4);
        acc = __dp4a((int)lo, (int)B.q[8 * h + i], acc);
        acc = __dp4a((int)hi, (int)B.q[8 * h + 4 + i], acc);
      }
      sumi[h] = acc - 16 * B.s[h];
    }
  } else {  // Q8_0, 68 bytes: d | 32 qs | d | 32 qs
    uint32_t w[17];
#pragma unroll
    for (int i = 0; i < 17; i++) w[i] = wp[i];
    dx[0] = h2f((uint16_t)(w[0] & 0xffffu));
    dx[1] = h2f((uint16_t)(w[8] >> 16));
    int a = 0, b = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      a = __dp4a((int)shr16(w[i], w[i + 1]), (int)B.q[i], a);
      b = __dp4a((int)w[9 + i], (int)B.q[8 + i], b);
    }
    sumi[0] = a;
    sumi[1] = b;
  }
  return __fmul_rn(__fmul_rn((float)sumi[0], dx[0]), B.d[0]) + __fmul_rn(__fmul_rn((float)sumi[1], dx[1]), B.d[1]);
}

// Values [8 lane, 8 lane + 8) of 256-value group j of a device row (token
// embedding rows), each as the type's to_float computes it.
__device__ __forceinline__ void dequant8(int type, const uint8_t* row, int nb, int j, int lane, float (&out)[8]) {
  if (is_legacy(type)) {
    const int bb = legacy_block_bytes(type);
    const uint8_t* blk = row + (size_t)(8 * j + (lane >> 2)) * bb;
    const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
    uint32_t qh = 0;
    if (type == GGML_Q5_0) qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) | ((uint32_t)blk[5] << 24);
    const uint8_t* qs = blk + (type == GGML_Q5_0 ? 6 : 2);
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int v = 8 * (lane & 3) + k;  // value within the 32-block
      int q;
      if (type == GGML_Q8_0) {
        q = (int)(int8_t)qs[v];
      } else {
        const int nib = v < 16 ? (qs[v] & 0xF) : (qs[v - 16] >> 4);
        q = type == GGML_Q4_0 ? nib - 8 : (nib | (int)(((qh >> v) & 1u) << 4)) - 16;
      }
      out[k] = __fmul_rn((float)q, d);
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const int i = 8 * lane + k;
    if (type == GGML_Q4_K || type == GGML_Q5_K) {
      const int bb = type == GGML_Q4_K ? Q4K_BLOCK_BYTES : Q5K_BLOCK_BYTES, qo = type == GGML_Q4_K ? 16 : 48;
      const uint8_t* blk = row + (int64_t)j * bb;
      const int c = i / 64, l = i % 64, sj = 2 * c + (l >= 32);
      const uint8_t byte = blk[qo + 32 * c + (l & 31)];
      int q = l >= 32 ? (byte >> 4) : (byte & 0xF);
      if (type == GGML_Q5_K) q += ((blk[16 + (l & 31)] >> sj) & 1) << 4;
      int sc, m;
      q4k_scale_min(blk + 4, sj, sc, m);
      const float d = h2f(*reinterpret_cast<const uint16_t*>(blk));
      const float dmin = h2f(*reinterpret_cast<const uint16_t*>(blk + 2));
      out[k] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
    } else {
      const uint8_t* body = row + (int64_t)j * Q6K_BODY_BYTES;
      const uint16_t* dv = reinterpret_cast<const uint16_t*>(row + (int64_t)nb * Q6K_BODY_BYTES);
      const int n = i / 128, r = i % 128, g = r / 32, l = r % 32;
      const uint8_t qlb = body[64 * n + l + (g & 1) * 32];
      const int lo = (g < 2) ? (qlb & 0xF) : (qlb >> 4);
      const int hi = (body[128 + 32 * n + l] >> (2 * g)) & 3;
      const int8_t sc = reinterpret_cast<const int8_t*>(body + 192)[8 * n + l / 16 + 2 * g];
      out[k] = __fmul_rn(__fmul_rn(h2f(dv[j]), (float)sc), (float)((lo | (hi << 4)) - 32));
    }
  }
}

// One lane's f32 share of <weight row, activation> over pass `pass`.
__device__ __forceinline__ float quarter_dot(int type, const uint8_t* row, int nb, int blk, int t,
                                             const ActSlice& A) {
  if (type == GGML_Q4_K || type == GGML_Q5_K) {
    int is, ms;
    float dx, dmx;
    if (type == GGML_Q4_K) q4k_quarter(row + (size_t)blk * Q4K_BLOCK_BYTES, t, A, is, ms, dx, dmx);
    else q5k_quarter(row + (size_t)blk * Q5K_BLOCK_BYTES, t, A, is, ms, dx, dmx);
    return __fmul_rn(dx, A.dy) * (float)is - __fmul_rn(dmx, A.dy) * (float)ms;
  }
  const uint16_t dh = reinterpret_cast<const uint16_t*>(row + (size_t)nb * Q6K_BODY_BYTES)[blk];
  return __fmul_rn(h2f(dh), A.dy) * (float)q6k_quarter(row + (size_t)blk * Q6K_BODY_BYTES, t, A);
}

// Same, with the weight type fixed at compile time (no dual-path predication
// in the unrolled inner loops).
template <int TYPE>
__device__ __forceinline__ float quarter_dot_t(const uint8_t* row, int nb, int blk, int t,
                                               const ActSlice& A) {
  if constexpr (TYPE == GGML_Q4_K) {
    int is, ms;
    float dx, dmx;
    q4k_quarter(row + (size_t)blk * Q4K_BLOCK_BYTES, t, A, is, ms, dx, dmx);
    return __fmul_rn(dx, A.dy) * (float)is - __fmul_rn(dmx, A.dy) * (float)ms;
  } else {
    const uint16_t dh = reinterpret_cast<const uint16_t*>(row + (size_t)nb * Q6K_BODY_BYTES)[blk];
    return __fmul_rn(h2f(dh), A.dy) * (float)q6k_quarter(row + (size_t)blk * Q6K_BODY_BYTES, t, A);
  }
}

// Both dot products of a row pair of any supported types (each row's type
// is the same for the whole warp): k-quant rows against the Q8_K slice,
// legacy rows against the Q8_0 slice; the per-lane shares are then summed
// across the warp. Shared by the persistent kernel and the per-kernel chain's
// generic path.
__device__ __forceinline__ float2 row_pair_dots(int ty0, const uint8_t* p0, int ty1, const uint8_t* p1, bool has1,
                                                int nb, const ActQ8& act, int lane) {
  const int t = lane & 3, bl = lane >> 2;
  const bool k0 = is_kquant(ty0), k1 = has1 && is_kquant(ty1);
  const bool l0 = !k0, l1 = has1 && !k1;
  float a0 = 0.f, a1 = 0.f;
  const int npass = (nb + 7) >> 3;
  // one loop per activation type, so that only one slice is live at a time
  if (k0 || k1) {
    for (int ps = 0; ps < npass; ps++) {
      const int blk = ps * 8 + bl;
      if (blk < nb) {
        ActSlice A;
        load_slice(act, blk, t, A);
        if (k0) a0 += quarter_dot(ty0, p0, nb, blk, t, A);
        if (k1) a1 += quarter_dot(ty1, p1, nb, blk, t, A);
      }
    }
  }
  if (l0 || l1) {
    for (int ps = 0; ps < npass; ps++) {
      const int blk = ps * 8 + bl;
      if (blk < nb) {
        ActSlice0 B;
        load_slice0(act, blk, t, B);
        if (l0) a0 += legacy_pair_dot(ty0, p0, blk, t, B);
        if (l1) a1 += legacy_pair_dot(ty1, p1, blk, t, B);
      }
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    a0 += __shfl_xor_sync(0xffffffffu, a0, off);
    a1 += __shfl_xor_sync(0xffffffffu, a1, off);
  }
  return make_float2(a0, a1);
}

}  // namespace armai
