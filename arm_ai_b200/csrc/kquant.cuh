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

}  // namespace armai
