// llama_kernels.cuh — sm_100a kernels of the quantized-Llama forward pass.
//
// Decode (one token per sequence, NB sequences) is five kinds of kernel per
// layer, launched back to back with programmatic dependent launch (PDL):
//
//   k_matvec<MODE_QKV>    rmsnorm(x) -> Q8_K -> q|k|v rows -> RoPE -> KV append
//   k_attn_decode         split-K GQA flash-decode + last-CTA combine -> y
//   k_matvec<MODE_RESID>  Q8_K(y) -> attn_output rows -> x += .
//   k_matvec<MODE_GATEUP> rmsnorm(x) -> Q8_K -> gate,up rows -> h = silu(g)*u
//   k_matvec<MODE_RESID>  Q8_K(h) -> ffn_down rows -> x += .
//   ... and k_matvec<MODE_HEAD> (output_norm, output rows, argmax) at the end.
//
// Every k_matvec CTA owns a contiguous range of weight rows. One thread
// streams that range HBM -> shared memory with cp.async.bulk (TMA bulk
// copies, L2 evict-first, completion on an mbarrier) into a ring of stages;
// the copies are issued BEFORE griddepcontrol.wait, so a kernel's weight
// traffic overlaps the tail of the kernel it depends on. All 12 warps then
// compute warp-per-row integer dot products (dp4a) against the Q8_K
// activation held in shared memory.
#pragma once

#include <float.h>

#include "kquant.cuh"

namespace armai {

constexpr int MV_THREADS = 384;  // 12 warps; two CTAs (of consecutive kernels) fit one SM
constexpr int MV_WARPS = MV_THREADS / 32;
constexpr uint32_t WAIT_LIMIT = 1u << 18;  // with 256 ns sleeps: a stuck copy ends the CTA in well under a second or two

enum { MODE_QKV = 0, MODE_RESID = 1, MODE_GATEUP = 2, MODE_HEAD = 3, MODE_STORE = 4 };

// ---------------------------------------------------------------------------
// PTX helpers: PDL, mbarrier, bulk copies.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// Global -> shared bulk copy (no multicast); 16-B aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// Bounded wait on an mbarrier phase. On expiry sets the device error flag and
// returns false (the caller makes the whole CTA leave).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return true;
    if (i > 8) __nanosleep(256);
  }
  atomicOr(err, DEVERR_MBAR_TIMEOUT);
  return false;
}

// ---------------------------------------------------------------------------
// Parameters.
// ---------------------------------------------------------------------------
struct Seg {
  const uint8_t* w;  // device rows (device layout)
  int type;          // GGML_Q4_K / GGML_Q6_K
  int rows;
  int nb;            // super-blocks per row
  int row_bytes;
};

struct MvParams {
  const float* x;      // [NB][K] activation input (f32)
  const float* gamma;  // rmsnorm weight [K] or nullptr
  float eps;
  int K, nb;
  Seg seg[3];
  int nseg;
  int acts;            // activations the rows need: 1 Q8_K (k-quants), 2 Q8_0 (legacy types)
  int nrows;           // activation rows (tokens / sequences) of this launch, <= NB
  int total_rows;      // QKV: q+k+v rows; GATEUP: rows of one of the pair; else rows
  int rows_per_cta, chunk_rows, ns;
  uint32_t stage_bytes;
  float* out;          // RESID: x in/out; GATEUP: h; HEAD: logits; QKV: q; STORE: out
  int out_stride;      // elements between batch rows of `out`
  // QKV epilogue
  int qn, kn, hd, max_seq, kv_f16;
  void* kc;
  void* vc;
  int64_t kv_seq_stride;  // elements between sequences' KV caches
  const int* pos;         // [NB]
  const float* cos_t;
  const float* sin_t;
  // HEAD epilogue
  float* am_val;          // [NB][grid]
  int* am_idx;            // [NB][grid]
  unsigned* counter;
  uint32_t* token;        // [NB]
  int* pos_out;           // [NB] or nullptr: pos_out[b] = pos[b] + 1
  float* best_val;        // [NB] or nullptr: the winning logit (tensor-parallel merge)
  int* best_idx;          // [NB] or nullptr: its row, 0x7fffffff when nothing won
  uint32_t* err;
};

// Shared-memory layout of k_matvec (bytes), host and device agree on it.
struct MvSmem {
  size_t stages, act_qs, act_d, act_bs, gamma, bars, red, act0_qs, act0_d, act0_s, total;
};
__host__ __device__ inline size_t al16(size_t v) { return (v + 15) & ~size_t(15); }
// red: 64 floats of scratch, NB*(K/256) per-block partial sums of squares,
// NB rms values.
// The Q8_0 buffers exist only when a matrix of the launch needs them.
__host__ __device__ inline MvSmem mv_smem_layout(int ns, uint32_t stage_bytes, int K, int NB,
                                                 bool norm, bool q80 = false) {
  MvSmem L;
  size_t o = 0;
  L.stages = o;  o += al16((size_t)ns * stage_bytes);
  L.act_qs = o;  o += al16((size_t)NB * K);
  L.act_d = o;   o += al16((size_t)NB * (K / QK_K) * 4);
  L.act_bs = o;  o += al16((size_t)NB * (K / 16) * 4);
  L.gamma = o;   o += norm ? al16((size_t)K * 4) : 0;
  L.bars = o;    o += al16((size_t)(ns + 1) * 8);
  L.red = o;     o += al16((64 + (size_t)NB * (K / QK_K) + NB) * 4);
  L.act0_qs = o; o += q80 ? al16((size_t)NB * K) : 0;
  L.act0_d = o;  o += q80 ? al16((size_t)NB * (K / QK8_0) * 4) : 0;
  L.act0_s = o;  o += q80 ? al16((size_t)NB * (K / QK8_0) * 4) : 0;
  L.total = o;
  return L;
}

// ---------------------------------------------------------------------------
// Chunk geometry: which bytes of which segment land where in a stage.
// ---------------------------------------------------------------------------
// parts[s] covers segment s (rows [lo, hi), segment-local, possibly empty)
// at byte `off` of the stage. Fixed slots, so every index is a compile-time
// constant and the array stays in registers.
struct Part {
  int lo, hi;
  uint32_t off;
};

template <int MODE>
__device__ __forceinline__ void make_parts(const Seg* seg, int nseg, int c0, int c1, Part (&parts)[3]) {
  if (MODE == MODE_QKV) {
    int sb = 0;
    uint32_t off = 0;
#pragma unroll
    for (int s = 0; s < 3; s++) {
      const int rows = s < nseg ? seg[s].rows : 0;
      const int se = sb + rows;
      const int lo = min(max(c0, sb), se), hi = max(lo, min(c1, se));
      parts[s] = Part{lo - sb, hi - sb, off};
      off += (uint32_t)(hi - lo) * (s < nseg ? (uint32_t)seg[s].row_bytes : 0u);
      sb = se;
    }
  } else if (MODE == MODE_GATEUP) {
    parts[0] = Part{c0, c1, 0};
    parts[1] = Part{c0, c1, (uint32_t)(c1 - c0) * seg[0].row_bytes};
    parts[2] = Part{0, 0, 0};
  } else {
    parts[0] = Part{c0, c1, 0};
    parts[1] = Part{0, 0, 0};
    parts[2] = Part{0, 0, 0};
  }
}

// One bulk copy per non-empty part, all completing on `bar`.
__device__ __forceinline__ void issue_parts(const Seg* seg, const Part (&parts)[3], uint8_t* stage,
                                            uint64_t* bar, uint64_t pol) {
  uint32_t total = 0;
#pragma unroll
  for (int k = 0; k < 3; k++) total += (uint32_t)(parts[k].hi - parts[k].lo) * seg[k].row_bytes;
  mbar_expect_tx(bar, total);
#pragma unroll
  for (int k = 0; k < 3; k++)
    if (parts[k].hi > parts[k].lo)
      bulk_g2s(stage + parts[k].off, seg[k].w + (int64_t)parts[k].lo * seg[k].row_bytes,
               (uint32_t)(parts[k].hi - parts[k].lo) * seg[k].row_bytes, bar, pol);
}

template <int MODE>
__device__ __forceinline__ void issue_chunk(const MvParams& p, int c0, int c1, uint8_t* stage,
                                            uint64_t* bar, uint64_t pol) {
  Part parts[3];
  make_parts<MODE>(p.seg, p.nseg, c0, c1, parts);
  issue_parts(p.seg, parts, stage, bar, pol);
}

// ---------------------------------------------------------------------------
// Prologue: build the Q8_K activation(s) in shared memory.
// Warp w owns 256-value jobs (b, j) = w, w + nwarps, ...: it loads its x
// values, (norm) contributes its per-block sum of squares, and after one
// barrier quantises them (candle rms_norm: y = x / sqrt(sum(x^2)/K + eps) *
// gamma; then BlockQ8K::from_float). The per-block partial sums are added in
// block order by every thread, so the result does not depend on scheduling.
// gamma was brought into shared memory by the bulk-copy engine before the
// kernel waited on its producer.
// ---------------------------------------------------------------------------
template <int NB>
__device__ void build_act(const MvParams& p, uint8_t* smem, const MvSmem& L, ActQ8 (&act)[NB],
                          uint64_t* gamma_bar) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const int K = p.K, nb = p.nb;
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* part = red + 64;              // [NB][nb]
  float* rms = part + NB * nb;         // [NB]
  for (int b = 0; b < NB; b++) {
    act[b].qs = reinterpret_cast<int8_t*>(smem + L.act_qs) + (size_t)b * K;
    act[b].d = reinterpret_cast<float*>(smem + L.act_d) + (size_t)b * nb;
    act[b].bs = reinterpret_cast<int32_t*>(smem + L.act_bs) + (size_t)b * (K / 16);
    act[b].qs0 = reinterpret_cast<int8_t*>(smem + L.act0_qs) + (size_t)b * K;
    act[b].d0 = reinterpret_cast<float*>(smem + L.act0_d) + (size_t)b * (K / QK8_0);
    act[b].s0 = reinterpret_cast<int32_t*>(smem + L.act0_s) + (size_t)b * (K / QK8_0);
  }
  const float* src = p.x;
  const bool norm = p.gamma != nullptr;
  if (norm) {
    for (int job = warp; job < p.nrows * nb; job += nw) {
      const int b = job / nb, j = job % nb;
      const float4* xr = reinterpret_cast<const float4*>(src + (size_t)b * K + j * QK_K + 8 * lane);
      const float4 x0 = xr[0], x1 = xr[1];
      float ss = x0.x * x0.x + x0.y * x0.y + x0.z * x0.z + x0.w * x0.w +
                 x1.x * x1.x + x1.y * x1.y + x1.z * x1.z + x1.w * x1.w;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) part[b * nb + j] = ss;
    }
    __syncthreads();
    if (tid < p.nrows) {
      float sum2 = 0.f;
      for (int j = 0; j < nb; j++) sum2 += part[tid * nb + j];
      rms[tid] = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum2, (float)K), p.eps));
    }
    // gamma must have landed before anyone reads it
    if (!mbar_wait(gamma_bar, 0, p.err)) { /* error flagged; values unused */ }
    __syncthreads();
  }
  const float* gs = reinterpret_cast<const float*>(smem + L.gamma);
  for (int job = warp; job < p.nrows * nb; job += nw) {
    const int b = job / nb, j = job % nb;
    const float4* xr = reinterpret_cast<const float4*>(src + (size_t)b * K + j * QK_K + 8 * lane);
    const float4 x0 = xr[0], x1 = xr[1];
    float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    if (norm) {
      const float m = rms[b];
      const float4* gr = reinterpret_cast<const float4*>(gs + j * QK_K + 8 * lane);
      const float4 g0 = gr[0], g1 = gr[1];
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fdiv_rn(v[i], m), g[i]);
    }
    if (p.acts & 1) q8k_quant_block_warp(v, lane, act[b].qs + j * QK_K, act[b].d + j, act[b].bs + j * 16, j & 7);
    if (p.acts & 2)
      q80_quant_block_warp(v, lane, act[b].qs0 + j * QK_K, act[b].d0 + 8 * j, act[b].s0 + 8 * j, j & 7);
  }
  __syncthreads();
}

// Total order used by the argmax: larger value first, then smaller index.
// NaN never wins (every comparison with it is false), matching a strict-'>'
// first-max scan started at -inf.
__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void store_kv(void* base, int kv_f16, int64_t idx, float a, float b) {
  if (kv_f16) {
    *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(base) + idx) = __floats2half2_rn(a, b);
  } else {
    *reinterpret_cast<float2*>(reinterpret_cast<float*>(base) + idx) = make_float2(a, b);
  }
}

// ---------------------------------------------------------------------------
// The chunk routine shared by k_matvec and the persistent decode kernel.
// A warp takes one "unit" at a time: two dot products that share an epilogue
// — rows r, r+1 of one segment (QKV: the RoPE pair), gate row r and up row r
// (GATEUP), or rows r, r+1 (RESID / HEAD / STORE; the second may be absent).
// The weight types of the two rows are dispatched once per unit into
// compile-time-typed inner loops.
// ---------------------------------------------------------------------------
// Ctx supplies the segment table and the epilogue's parameters through
// accessors, so that what a kernel keeps in its constant bank (its own launch
// parameters) is read from there instead of occupying registers.
template <int T0, int T1>
__device__ __forceinline__ void unit_dots(const uint8_t* p0, const uint8_t* p1, bool has1, int nb,
                                          const ActQ8& act, int lane, float& d0, float& d1) {
  const int t = lane & 3, bl = lane >> 2;
  float a0 = 0.f, a1 = 0.f;
  const int npass = (nb + 7) >> 3;
  for (int ps = 0; ps < npass; ps++) {
    const int blk = ps * 8 + bl;
    if (blk < nb) {
      // the activation slice is re-read from shared memory per row pair:
      // keeping it in registers across rows spilled elsewhere
      ActSlice A;
      load_slice(act, blk, t, A);
      a0 += quarter_dot_t<T0>(p0, nb, blk, t, A);
      if (has1) a1 += quarter_dot_t<T1>(p1, nb, blk, t, A);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    a0 += __shfl_xor_sync(0xffffffffu, a0, off);
    a1 += __shfl_xor_sync(0xffffffffu, a1, off);
  }
  d0 = a0;
  d1 = a1;
}

// Two units at once (four rows, one activation slice per pass): independent
// dot chains that a warp interleaves. Unit a = rows a0 (type T0), a1 (T1);
// unit b likewise.
template <int T0, int T1>
__device__ __forceinline__ void unit_dots2(const uint8_t* a0p, const uint8_t* a1p, bool hasa1, const uint8_t* b0p,
                                           const uint8_t* b1p, bool hasb1, int nb, const ActQ8& act, int lane,
                                           float (&d)[4]) {
  const int t = lane & 3, bl = lane >> 2;
  float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
  const int npass = (nb + 7) >> 3;
  for (int ps = 0; ps < npass; ps++) {
    const int blk = ps * 8 + bl;
    if (blk < nb) {
      ActSlice A;
      load_slice(act, blk, t, A);
      a0 += quarter_dot_t<T0>(a0p, nb, blk, t, A);
      b0 += quarter_dot_t<T0>(b0p, nb, blk, t, A);
      if (hasa1) a1 += quarter_dot_t<T1>(a1p, nb, blk, t, A);
      if (hasb1) b1 += quarter_dot_t<T1>(b1p, nb, blk, t, A);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    a0 += __shfl_xor_sync(0xffffffffu, a0, off);
    a1 += __shfl_xor_sync(0xffffffffu, a1, off);
    b0 += __shfl_xor_sync(0xffffffffu, b0, off);
    b1 += __shfl_xor_sync(0xffffffffu, b1, off);
  }
  d[0] = a0; d[1] = a1; d[2] = b0; d[3] = b1;
}

// Unit u of a staged chunk [c0, c1): its two row pointers, their types, its
// first row r, the QKV segment si and whether the second row exists.
struct UnitRows {
  const uint8_t *p0, *p1;
  int ty0, ty1, r, si;
  bool has1;
};
template <int MODE, class Ctx>
__device__ __forceinline__ UnitRows unit_rows(const Ctx& cx, const uint8_t* stage, int c0, int c1,
                                              const Part (&parts)[3], int u) {
  UnitRows w;
  w.si = 0;
  w.has1 = true;
  if (MODE == MODE_QKV) {
    w.r = c0 + 2 * u;
    const int qn = cx.qn(), kn = cx.kn();
    w.si = w.r < qn ? 0 : (w.r < qn + kn ? 1 : 2);
    const int sb = w.si == 0 ? 0 : (w.si == 1 ? qn : qn + kn);
    const uint32_t off = w.si == 0 ? parts[0].off : (w.si == 1 ? parts[1].off : parts[2].off);
    const int lo = w.si == 0 ? parts[0].lo : (w.si == 1 ? parts[1].lo : parts[2].lo);
    const Seg& sg = cx.seg(w.si);
    w.p0 = stage + off + (size_t)(w.r - sb - lo) * sg.row_bytes;
    w.p1 = w.p0 + sg.row_bytes;
    w.ty0 = w.ty1 = sg.type;
  } else if (MODE == MODE_GATEUP) {
    w.r = c0 + u;
    w.p0 = stage + (size_t)u * cx.seg(0).row_bytes;
    w.p1 = stage + parts[1].off + (size_t)u * cx.seg(1).row_bytes;
    w.ty0 = cx.seg(0).type;
    w.ty1 = cx.seg(1).type;
  } else {
    w.r = c0 + 2 * u;
    w.p0 = stage + (size_t)(2 * u) * cx.seg(0).row_bytes;
    w.p1 = w.p0 + cx.seg(0).row_bytes;
    w.has1 = w.r + 1 < c1;
    w.ty0 = w.ty1 = cx.seg(0).type;
  }
  return w;
}

template <int MODE>
__device__ __forceinline__ int chunk_nunits(int c0, int c1) {
  return MODE == MODE_GATEUP ? c1 - c0 : (c1 - c0 + 1) >> 1;
}

// Both dot products of one unit, dispatched on the rows' types.
template <int MODE>
__device__ __forceinline__ void unit_dot_any(const UnitRows& w, int nb, const ActQ8& act, int lane, float& d0,
                                             float& d1) {
  if ((w.ty0 != GGML_Q4_K && w.ty0 != GGML_Q6_K) || (w.ty1 != GGML_Q4_K && w.ty1 != GGML_Q6_K)) {
    // Q5_K / legacy types: the generic runtime-typed path
    const float2 r = row_pair_dots(w.ty0, w.p0, w.ty1, w.p1, w.has1, nb, act, lane);
    d0 = r.x;
    d1 = r.y;
  } else if (MODE != MODE_GATEUP || w.ty0 == w.ty1) {  // both rows of one matrix
    if (w.ty0 == GGML_Q4_K) unit_dots<GGML_Q4_K, GGML_Q4_K>(w.p0, w.p1, w.has1, nb, act, lane, d0, d1);
    else unit_dots<GGML_Q6_K, GGML_Q6_K>(w.p0, w.p1, w.has1, nb, act, lane, d0, d1);
  } else if (w.ty0 == GGML_Q4_K) {
    unit_dots<GGML_Q4_K, GGML_Q6_K>(w.p0, w.p1, w.has1, nb, act, lane, d0, d1);
  } else {
    unit_dots<GGML_Q6_K, GGML_Q4_K>(w.p0, w.p1, w.has1, nb, act, lane, d0, d1);
  }
}

// RoPE factors of a q / k pair, loaded before the dots so that their latency
// overlaps them (same address for the whole warp).
template <int MODE, class Ctx>
__device__ __forceinline__ void unit_rope(const Ctx& cx, const UnitRows& w, float& cs, float& sn) {
  cs = 0.f;
  sn = 0.f;
  if (MODE == MODE_QKV && w.si < 2) {
    const int hd = cx.hd(), rr = w.si == 0 ? w.r : w.r - cx.qn();
    const size_t ti = (size_t)cx.pos() * (hd >> 1) + ((rr % hd) >> 1);
    cs = __ldg(cx.cos_t() + ti);
    sn = __ldg(cx.sin_t() + ti);
  }
}

// The unit's epilogue (one lane).
template <int MODE, class Ctx>
__device__ __forceinline__ void unit_epilogue(const Ctx& cx, const UnitRows& w, float d0, float d1, float cs,
                                              float sn, float& best_v, int& best_i) {
  const int r = w.r;
  if (MODE == MODE_QKV) {
    const int hd = cx.hd();
    const int qn = cx.qn(), kn = cx.kn();
    if (w.si < 2) {
      const int rr = w.si == 0 ? r : r - qn;
      // candle rope_i: (a*c - b*s, a*s + b*c), each op rounded
      const float o0 = __fsub_rn(__fmul_rn(d0, cs), __fmul_rn(d1, sn));
      const float o1 = __fadd_rn(__fmul_rn(d0, sn), __fmul_rn(d1, cs));
      if (w.si == 0) cx.put_q(r, o0, o1);
      else cx.put_kv(0, rr / hd, rr % hd, o0, o1);
    } else {
      const int rv = r - qn - kn;
      cx.put_kv(1, rv / hd, rv % hd, d0, d1);
    }
  } else if (MODE == MODE_GATEUP) {
    // candle: silu(v) = v / (1 + exp(-v)); then * up
    const float sl = __fdiv_rn(d0, __fadd_rn(1.0f, expf(-d0)));
    cx.put_h(r, __fmul_rn(sl, d1));
  } else {
    float* out = cx.out();
#pragma unroll
    for (int k = 0; k < 2; k++) {
      if (k == 1 && !w.has1) break;
      const float v = k == 0 ? d0 : d1;
      if (MODE == MODE_RESID) cx.resid_add(out + r + k, r + k, v);
      else if (out) out[r + k] = v;
      if (MODE == MODE_HEAD && am_better(v, r + k, best_v, best_i)) {
        best_v = v;
        best_i = r + k;
      }
    }
  }
}

template <int MODE, class Ctx>
__device__ __forceinline__ void chunk_units(const Ctx& cx, const uint8_t* stage, int c0, int c1,
                                            const Part (&parts)[3], const ActQ8& act, int warp,
                                            int nwarps, int lane, float& best_v, int& best_i) {
  const int nb = cx.nb();
  const int nunits = chunk_nunits<MODE>(c0, c1);
  for (int u = warp; u < nunits; u += nwarps) {
    const UnitRows w = unit_rows<MODE>(cx, stage, c0, c1, parts, u);
    float cs, sn;
    unit_rope<MODE>(cx, w, cs, sn);
    float d0, d1;
    unit_dot_any<MODE>(w, nb, act, lane, d0, d1);
    if (lane != 0) continue;
    if (u == 0) cx.stamp(8);
    unit_epilogue<MODE>(cx, w, d0, d1, cs, sn, best_v, best_i);
    if (u == 0) cx.stamp(9);
  }
}

// Context of k_matvec: its launch parameters and the sequence index.
struct MvCtx {
  const MvParams& p;
  int b;
  __device__ const Seg& seg(int i) const { return p.seg[i]; }
  __device__ int nb() const { return p.nb; }
  __device__ float* out() const { return p.out + (size_t)b * p.out_stride; }
  __device__ int qn() const { return p.qn; }
  __device__ int kn() const { return p.kn; }
  __device__ int hd() const { return p.hd; }
  __device__ int max_seq() const { return p.max_seq; }
  __device__ int kv_f16() const { return p.kv_f16; }
  __device__ void* kc() const { return p.kc; }
  __device__ void* vc() const { return p.vc; }
  __device__ int64_t kv_off() const { return (int64_t)b * p.kv_seq_stride; }
  __device__ int pos() const { return p.pos[b]; }
  __device__ const float* cos_t() const { return p.cos_t; }
  __device__ const float* sin_t() const { return p.sin_t; }
  __device__ void stamp(int) const {}
  // epilogue outputs: q rows, the K (which = 0) / V (1) cache row at pos, h
  __device__ void put_q(int r, float a, float b) const {
    *reinterpret_cast<float2*>(out() + r) = make_float2(a, b);
  }
  __device__ void put_kv(int which, int kvh, int dd, float a, float b) const {
    store_kv(which ? vc() : kc(), kv_f16(), kv_off() + ((int64_t)kvh * max_seq() + pos()) * hd() + dd, a, b);
  }
  __device__ void put_h(int r, float v) const { out()[r] = v; }
  // x[r] += v (the residual stream lives in global memory between kernels)
  __device__ void resid_add(float* o, int, float v) const { *o = __fadd_rn(v, __ldcg(o)); }
};

// ---------------------------------------------------------------------------
// The streaming matvec kernel.
// ---------------------------------------------------------------------------
template <int MODE, int NB>
__global__ void __launch_bounds__(MV_THREADS, 2) k_matvec(const MvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const MvSmem L = mv_smem_layout(p.ns, p.stage_bytes, p.K, NB, p.gamma != nullptr, (p.acts & 2) != 0);
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int r1 = min(r0 + p.rows_per_cta, p.total_rows);
  const int nchunks = r1 > r0 ? (r1 - r0 + p.chunk_rows - 1) / p.chunk_rows : 0;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint8_t* stages = smem + L.stages;

  if (tid == 0) {
    for (int s = 0; s <= p.ns; s++) mbar_init(&bars[s], 1);  // ns stages + gamma
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint64_t pol = l2_evict_first_policy();
    if (p.gamma) {
      mbar_expect_tx(&bars[p.ns], (uint32_t)p.K * 4u);
      bulk_g2s(smem + L.gamma, p.gamma, (uint32_t)p.K * 4u, &bars[p.ns], pol);
    }
    for (int c = 0; c < min(p.ns, nchunks); c++) {
      const int c0 = r0 + c * p.chunk_rows, c1 = min(c0 + p.chunk_rows, r1);
      issue_chunk<MODE>(p, c0, c1, stages + (size_t)c * p.stage_bytes, &bars[c], pol);
    }
  }
  // Weights are in flight; let the next kernel start its own prefetch, then
  // wait for the producer of our activations.
  pdl_launch();
  pdl_wait();

  ActQ8 act[NB];
  build_act<NB>(p, smem, L, act, &bars[p.ns]);

  float best_v[NB];
  int best_i[NB];
#pragma unroll
  for (int b = 0; b < NB; b++) { best_v[b] = -INFINITY; best_i[b] = 0x7fffffff; }

  for (int c = 0; c < nchunks; c++) {
    const int s = c % p.ns;
    const int c0 = r0 + c * p.chunk_rows, c1 = min(c0 + p.chunk_rows, r1);
    const bool ok = mbar_wait(&bars[s], (uint32_t)((c / p.ns) & 1), p.err);
    if (__syncthreads_or(!ok)) return;
    const uint8_t* stage = stages + (size_t)s * p.stage_bytes;
    Part parts[3];
    make_parts<MODE>(p.seg, p.nseg, c0, c1, parts);
#pragma unroll 1
    for (int b = 0; b < p.nrows; b++)
      chunk_units<MODE>(MvCtx{p, b}, stage, c0, c1, parts, act[b], warp, MV_WARPS, lane, best_v[b],
                        best_i[b]);
    __syncthreads();
    if (tid == 0 && c + p.ns < nchunks) {
      fence_proxy_async();
      const int n0 = r0 + (c + p.ns) * p.chunk_rows, n1 = min(n0 + p.chunk_rows, r1);
      issue_chunk<MODE>(p, n0, n1, stages + (size_t)s * p.stage_bytes, &bars[s],
                        l2_evict_first_policy());
    }
  }

  if (MODE == MODE_HEAD) {
    // CTA argmax -> partial; the last CTA to finish reduces all partials.
    float* rv = reinterpret_cast<float*>(smem + L.red);
    int* ri = reinterpret_cast<int*>(rv + 32);
    __shared__ int s_last;
    for (int b = 0; b < p.nrows; b++) {
      if (lane == 0) { rv[warp] = best_v[b]; ri[warp] = best_i[b]; }
      __syncthreads();
      if (tid == 0) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int w = 0; w < MV_WARPS; w++)
          if (am_better(rv[w], ri[w], bv, bi)) { bv = rv[w]; bi = ri[w]; }
        p.am_val[(size_t)b * gridDim.x + blockIdx.x] = bv;
        p.am_idx[(size_t)b * gridDim.x + blockIdx.x] = bi;
      }
      __syncthreads();
    }
    if (tid == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(p.counter, 1u);
      s_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      for (int b = warp; b < p.nrows; b += MV_WARPS) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = lane; i < (int)gridDim.x; i += 32) {
          const float v = __ldcg(p.am_val + (size_t)b * gridDim.x + i);
          const int ix = __ldcg(p.am_idx + (size_t)b * gridDim.x + i);
          if (am_better(v, ix, bv, bi)) { bv = v; bi = ix; }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
          if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
          // No finite winner (all NaN / -inf): the reference's fold keeps index 0.
          p.token[b] = (bi == 0x7fffffff) ? 0u : (uint32_t)bi;
          if (p.pos_out) p.pos_out[b] = p.pos[b] + 1;
          if (p.best_val) { p.best_val[b] = bv; p.best_idx[b] = bi; }
        }
      }
      if (tid == 0) *p.counter = 0u;
    }
  }
}

// ---------------------------------------------------------------------------
// Split-K GQA flash-decode. grid (n_kv, splits, NB), 128 threads.
// CTA (kvh, s, b) scores positions [t0, t1) of sequence b for the nrep query
// heads that share KV head kvh (repeat_kv: kvh = h / nrep), keeps an
// unnormalised partial (m, l, o), and the last CTA of (b, kvh) merges the
// splits in split order: y = sum_s o_s e^{m_s-M} / sum_s l_s e^{m_s-M}.
// ---------------------------------------------------------------------------
struct AttnParams {
  const float* q;      // [NB][n_head*hd]
  const void* kc;      // layer base, [seq][n_kv][max_seq][hd]
  const void* vc;
  int64_t kv_seq_stride;
  int kv_f16;
  const int* pos;      // [NB]
  int max_seq, hd, n_head, n_kv;
  float scale;
  float* part;         // [NB][n_kv][splits][nrep][hd+2]
  unsigned* counters;  // [NB][n_kv]
  float* y;            // [NB][n_head*hd]
  uint32_t* err;
};

constexpr int ATT_THREADS = 128;
constexpr int ATT_MAX_REP = 8;   // query heads per KV head
constexpr int ATT_SPLITS = 16;   // most context splits per (sequence, KV head): the partials' layout
// Positions per shared-memory tile: 64 at head_dim 64, 32 at 128 (the same
// 16 KB K tile either way).
template <int HD>
__host__ __device__ constexpr int att_tile() { return 4096 / HD; }

// Shared memory of k_attn_decode<HD> (floats): q[rep][HD], K[TILE][HD],
// V[TILE][HD], p[rep][TILE], corr/m/l[rep], combine weights[SPLITS][rep]
// (37.5 KB at either head_dim: six CTAs per SM).
__host__ __device__ inline size_t attn_smem_floats(int hd) {
  const size_t tile = (size_t)(4096 / hd);
  return (size_t)ATT_MAX_REP * hd + 2 * tile * hd + (size_t)ATT_MAX_REP * tile + 3 * ATT_MAX_REP +
         (size_t)ATT_SPLITS * ATT_MAX_REP + ATT_MAX_REP;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}

// n rows of HD values of K and V into shared memory. K row t keeps its
// 16-byte chunk c at c ^ (t & 7), so that float4 reads of one chunk by a lane
// per row hit distinct banks. f32 caches: asynchronous 16-byte copies, every
// copy of the tile in flight at once; f16 caches: loaded and widened by the
// threads.
template <int HD, typename KV>
__device__ __forceinline__ void load_kv_tile(const KV* base, int n, float* Ks, float* Vs, const KV* vbase) {
  constexpr int V4 = HD / 4;
  if constexpr (sizeof(KV) == 4) {
    for (int i = threadIdx.x; i < n * V4; i += blockDim.x) {
      const int t = i / V4, c = (i % V4) * 4;
      cp_async16(Ks + t * HD + ((c >> 2) ^ (t & 7)) * 4, reinterpret_cast<const float*>(base) + (size_t)t * HD + c);
      cp_async16(Vs + t * HD + c, reinterpret_cast<const float*>(vbase) + (size_t)t * HD + c);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  } else {
#pragma unroll 4
    for (int i = threadIdx.x; i < n * V4; i += blockDim.x) {
      const int t = i / V4, c = (i % V4) * 4;
      const uint2 kr = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(base) + (size_t)t * HD + c);
      const uint2 vr = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(vbase) + (size_t)t * HD + c);
      const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&kr.x));
      const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&kr.y));
      const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&vr.x));
      const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&vr.y));
      *reinterpret_cast<float4*>(Ks + t * HD + ((c >> 2) ^ (t & 7)) * 4) = make_float4(k0.x, k0.y, k1.x, k1.y);
      *reinterpret_cast<float4*>(Vs + t * HD + c) = make_float4(v0.x, v0.y, v1.x, v1.y);
    }
  }
}

// Split-K GQA flash-decode. grid (n_kv, ATT_SPLITS, NB), ATT_THREADS threads.
// Sequence b's T positions are split over the fewest CTAs that keep one tile
// (att_tile<HD>() positions) per CTA, at most ATT_SPLITS (longer contexts
// give a CTA several tiles); CTAs past that count return at once. CTA
// (kvh, s, b) covers positions [t0, t1) for the nrep query heads sharing KV
// head kvh (repeat_kv: kvh = h / nrep): scores s = (q . k) * scale with a
// lane per position (two heads per warp pass), an online softmax per head,
// o += p v with a thread per output dim. The last CTA of (b, kvh) merges the
// splits in split order: y = sum_s o_s e^{m_s-M} / sum_s l_s e^{m_s-M}.
// For prefill the batch index runs over the prompt's tokens with a shared
// cache (kv_seq_stride 0): token b attends positions 0..pos[b] (causal).
template <int HD, typename KV>
__global__ void __launch_bounds__(ATT_THREADS) k_attn_decode(const AttnParams p) {
  constexpr int TILE = att_tile<HD>();
  constexpr int PPL = TILE / 32;                    // positions per lane
  extern __shared__ __align__(16) float sm[];
  const int kvh = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nrep = p.n_head / p.n_kv;
  float* qs = sm;                                   // [ATT_MAX_REP][HD]
  float* Ks = qs + ATT_MAX_REP * HD;                // [TILE][HD], chunk-swizzled
  float* Vs = Ks + TILE * HD;                       // [TILE][HD]
  float* ps = Vs + TILE * HD;                       // [ATT_MAX_REP][TILE]
  float* corr = ps + ATT_MAX_REP * TILE;            // [rep]
  float* mrow = corr + ATT_MAX_REP;                 // [rep]
  float* lrow = mrow + ATT_MAX_REP;                 // [rep]
  float* wts = lrow + ATT_MAX_REP;                  // [SPLITS][rep]
  float* Ltot = wts + ATT_SPLITS * ATT_MAX_REP;     // [rep]
  __shared__ int s_last;
  pdl_launch();
  pdl_wait();
  const int T = p.pos[b] + 1;
  const int splits = min(ATT_SPLITS, (T + TILE - 1) / TILE);
  if (s >= splits) return;
  const int chunk = (T + splits - 1) / splits;
  const int t0 = min(T, s * chunk), t1 = min(T, t0 + chunk);
  const float* qb = p.q + (size_t)b * p.n_head * HD + (size_t)kvh * nrep * HD;
  for (int i = tid; i < nrep * HD / 4; i += blockDim.x)
    reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(qb)[i];
  if (tid < ATT_MAX_REP) { mrow[tid] = -INFINITY; lrow[tid] = 0.f; }
  const int64_t kvbase = (int64_t)b * p.kv_seq_stride + (int64_t)kvh * p.max_seq * HD;
  const KV* kc = reinterpret_cast<const KV*>(p.kc) + kvbase;
  const KV* vc = reinterpret_cast<const KV*>(p.vc) + kvbase;
  // PV ownership: thread -> (dim d, group of heads)
  constexpr int DGROUPS = ATT_THREADS / HD;          // 2 for HD=64, 1 for HD=128
  constexpr int RPG = ATT_MAX_REP / DGROUPS;         // heads per thread
  const int d = tid % HD, rg = tid / HD;
  const int nmine = min(RPG, nrep - rg * RPG);       // heads of this thread (may be <= 0)
  float o[RPG];
#pragma unroll
  for (int i = 0; i < RPG; i++) o[i] = 0.f;
  for (int tt0 = t0; tt0 < t1; tt0 += TILE) {
    const int n = min(TILE, t1 - tt0);
    __syncthreads();  // previous tile fully consumed (and q / m / l initialised)
    load_kv_tile<HD, KV>(kc + (size_t)tt0 * HD, n, Ks, Vs, vc + (size_t)tt0 * HD);
    __syncthreads();
    // scores and online softmax: warp per head pair (r, r + 4), lane per
    // position(s) lane + 32 j; the two heads share each K element load
    constexpr int NW = ATT_THREADS / 32;
    for (int r = warp; r < nrep; r += 2 * NW) {
      const int r2 = r + NW;
      const bool two = r2 < nrep;
      const float* qa = qs + r * HD;
      const float* qb2 = qs + (two ? r2 : r) * HD;
      float sc[PPL], sc2[PPL];
#pragma unroll
      for (int j = 0; j < PPL; j++) {
        sc[j] = -INFINITY;
        sc2[j] = -INFINITY;
        if (lane + 32 * j < n) {
          const float4* kr = reinterpret_cast<const float4*>(Ks + (lane + 32 * j) * HD);
          const int sw = lane & 7;  // the row's chunk swizzle
          const float4* q4a = reinterpret_cast<const float4*>(qa);
          const float4* q4b = reinterpret_cast<const float4*>(qb2);
          float acc = 0.f, acc2 = 0.f;
#pragma unroll 4
          for (int d4 = 0; d4 < HD / 4; d4++) {  // dims in order: each sum as the sequential dot
            const float4 kv = kr[d4 ^ sw], xa = q4a[d4], xb = q4b[d4];
            acc = fmaf(xa.x, kv.x, acc);
            acc = fmaf(xa.y, kv.y, acc);
            acc = fmaf(xa.z, kv.z, acc);
            acc = fmaf(xa.w, kv.w, acc);
            acc2 = fmaf(xb.x, kv.x, acc2);
            acc2 = fmaf(xb.y, kv.y, acc2);
            acc2 = fmaf(xb.z, kv.z, acc2);
            acc2 = fmaf(xb.w, kv.w, acc2);
          }
          sc[j] = acc * p.scale;
          sc2[j] = acc2 * p.scale;
        }
      }
      float mt = sc[0], mt2 = sc2[0];
#pragma unroll
      for (int j = 1; j < PPL; j++) {
        mt = fmaxf(mt, sc[j]);
        mt2 = fmaxf(mt2, sc2[j]);
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
        mt2 = fmaxf(mt2, __shfl_xor_sync(0xffffffffu, mt2, off));
      }
      const float mold = mrow[r], mold2 = mrow[two ? r2 : r];
      const float mnew = fmaxf(mold, mt), mnew2 = fmaxf(mold2, mt2);
      float ls = 0.f, ls2 = 0.f;
#pragma unroll
      for (int j = 0; j < PPL; j++) {
        const bool in = lane + 32 * j < n;
        const float pe = in ? expf(sc[j] - mnew) : 0.f;
        const float pe2 = in ? expf(sc2[j] - mnew2) : 0.f;
        ls += pe;
        ls2 += pe2;
        ps[r * TILE + lane + 32 * j] = pe;
        if (two) ps[r2 * TILE + lane + 32 * j] = pe2;
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        ls += __shfl_xor_sync(0xffffffffu, ls, off);
        ls2 += __shfl_xor_sync(0xffffffffu, ls2, off);
      }
      __syncwarp();
      if (lane == 0) {
        const float c = expf(mold - mnew);  // 0 on the first tile (mold = -inf)
        corr[r] = c;
        lrow[r] = lrow[r] * c + ls;
        mrow[r] = mnew;
        if (two) {
          const float c2 = expf(mold2 - mnew2);
          corr[r2] = c2;
          lrow[r2] = lrow[r2] * c2 + ls2;
          mrow[r2] = mnew2;
        }
      }
    }
    __syncthreads();
    // o += p v: position outer, the thread's heads inner (one V load per
    // position; each head's sum in position order)
    const float* pr = ps + rg * RPG * TILE;
#pragma unroll
    for (int i = 0; i < RPG; i++)
      if (i < nmine) o[i] *= corr[rg * RPG + i];
    for (int tt = 0; tt < n; tt++) {
      const float v = Vs[tt * HD + d];
#pragma unroll
      for (int i = 0; i < RPG; i++)
        if (i < nmine) o[i] += pr[i * TILE + tt] * v;
    }
  }
  if (splits == 1) {  // the whole context in this CTA: y directly
#pragma unroll
    for (int i = 0; i < RPG; i++)
      if (i < nmine) {
        const int r = rg * RPG + i;
        p.y[(size_t)b * p.n_head * HD + ((size_t)kvh * nrep + r) * HD + d] = o[i] / lrow[r];
      }
    return;
  }
  __syncthreads();
  // partial of this split: o[rep][HD], m[rep], l[rep]
  const size_t pbase = ((((size_t)b * p.n_kv + kvh) * ATT_SPLITS + s) * nrep) * (HD + 2);
#pragma unroll
  for (int i = 0; i < RPG; i++)
    if (i < nmine) p.part[pbase + (size_t)(rg * RPG + i) * (HD + 2) + d] = o[i];
  if (tid < nrep) {
    p.part[pbase + (size_t)tid * (HD + 2) + HD] = mrow[tid];
    p.part[pbase + (size_t)tid * (HD + 2) + HD + 1] = lrow[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&p.counters[b * p.n_kv + kvh], 1u);
    s_last = (prev == (unsigned)splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const size_t base0 = (((size_t)b * p.n_kv + kvh) * ATT_SPLITS) * nrep * (HD + 2);
  // 1) (m, l) of every (split, head) -> smem; per-head max and weights
  if (tid < splits * nrep) {
    const int s2 = tid / nrep, r = tid % nrep;
    const size_t o2 = base0 + ((size_t)s2 * nrep + r) * (HD + 2);
    wts[s2 * ATT_MAX_REP + r] = __ldcg(p.part + o2 + HD);        // m
    ps[s2 * ATT_MAX_REP + r] = __ldcg(p.part + o2 + HD + 1);     // l (ps reused)
  }
  __syncthreads();
  if (tid < nrep) {
    float M = -INFINITY;
    for (int s2 = 0; s2 < splits; s2++)
      if (ps[s2 * ATT_MAX_REP + tid] > 0.f) M = fmaxf(M, wts[s2 * ATT_MAX_REP + tid]);
    float Ls = 0.f;
    for (int s2 = 0; s2 < splits; s2++) {
      const float l = ps[s2 * ATT_MAX_REP + tid];
      const float w = l > 0.f ? expf(wts[s2 * ATT_MAX_REP + tid] - M) : 0.f;
      wts[s2 * ATT_MAX_REP + tid] = w;
      Ls += l * w;
    }
    Ltot[tid] = Ls;
  }
  __syncthreads();
  // 2) y[r][d] = sum_s w_s o_s[r][d] / L
  for (int i = tid; i < nrep * HD; i += blockDim.x) {
    const int r = i / HD, dd = i % HD;
    float ov[ATT_SPLITS];
#pragma unroll
    for (int s2 = 0; s2 < ATT_SPLITS; s2++)
      if (s2 < splits) ov[s2] = __ldcg(p.part + base0 + ((size_t)s2 * nrep + r) * (HD + 2) + dd);
    float O = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < ATT_SPLITS; s2++)
      if (s2 < splits) O += wts[s2 * ATT_MAX_REP + r] * ov[s2];
    p.y[(size_t)b * p.n_head * HD + ((size_t)kvh * nrep + r) * HD + dd] = O / Ltot[r];
  }
  if (tid == 0) p.counters[b * p.n_kv + kvh] = 0u;
}

// ---------------------------------------------------------------------------
// Embedding: x[b] = to_float(token_embd row token[b]).
// ---------------------------------------------------------------------------
static __global__ void __launch_bounds__(256) k_embed(const uint8_t* table, int type, int nb,
                                               int64_t row_bytes, const uint32_t* tokens,
                                               float* x, int K, int n_vocab, uint32_t* err) {
  pdl_launch();
  pdl_wait();
  const int b = blockIdx.x;
  uint32_t tok = tokens[b];
  if (tok >= (uint32_t)n_vocab) {
    if (threadIdx.x == 0) atomicOr(err, 4u);
    tok = 0;
  }
  const uint8_t* row = table + (int64_t)tok * row_bytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* y = x + (size_t)b * K;
  // one warp per 256-value block, 8 values per lane (each type's to_float)
  for (int j = warp; j < nb; j += blockDim.x >> 5) {
    float v[8];
    dequant8(type, row, nb, j, lane, v);
#pragma unroll
    for (int k = 0; k < 8; k++) y[j * QK_K + 8 * lane + k] = v[k];
  }
}

static __global__ void k_set_int(int* p, int v) { *p = v; }

}  // namespace armai
