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
constexpr uint32_t WAIT_LIMIT = 1u << 20;

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
  uint32_t* err;
};

// Shared-memory layout of k_matvec (bytes), host and device agree on it.
struct MvSmem {
  size_t stages, act_qs, act_d, act_bs, xbuf, bars, red, total;
};
__host__ __device__ inline size_t al16(size_t v) { return (v + 15) & ~size_t(15); }
__host__ __device__ inline MvSmem mv_smem_layout(int ns, uint32_t stage_bytes, int K, int NB,
                                                 bool norm) {
  MvSmem L;
  size_t o = 0;
  L.stages = o;  o += al16((size_t)ns * stage_bytes);
  L.act_qs = o;  o += al16((size_t)NB * K);
  L.act_d = o;   o += al16((size_t)NB * (K / QK_K) * 4);
  L.act_bs = o;  o += al16((size_t)NB * (K / 16) * 4);
  L.xbuf = o;    o += norm ? al16((size_t)NB * K * 4) : 0;
  L.bars = o;    o += al16((size_t)ns * 8);
  L.red = o;     o += al16(64 * 4 + NB * 8);
  L.total = o;
  return L;
}

// ---------------------------------------------------------------------------
// Chunk geometry: which bytes of which segment land where in a stage.
// ---------------------------------------------------------------------------
struct Part {
  int seg, lo, hi;   // rows [lo, hi) of segment `seg` (segment-local)
  uint32_t off;      // byte offset in the stage
};

template <int MODE>
__device__ __forceinline__ int chunk_parts(const MvParams& p, int c0, int c1, Part (&parts)[3]) {
  int n = 0;
  uint32_t off = 0;
  if (MODE == MODE_QKV) {
    int sb = 0;
    for (int s = 0; s < p.nseg; s++) {
      const int se = sb + p.seg[s].rows;
      const int lo = max(c0, sb), hi = min(c1, se);
      if (lo < hi) {
        parts[n++] = Part{s, lo - sb, hi - sb, off};
        off += (uint32_t)(hi - lo) * p.seg[s].row_bytes;
      }
      sb = se;
    }
  } else if (MODE == MODE_GATEUP) {
    parts[n++] = Part{0, c0, c1, 0};
    parts[n++] = Part{1, c0, c1, (uint32_t)(c1 - c0) * p.seg[0].row_bytes};
  } else {
    parts[n++] = Part{0, c0, c1, 0};
  }
  return n;
}

template <int MODE>
__device__ __forceinline__ void issue_chunk(const MvParams& p, int c0, int c1, uint8_t* stage,
                                            uint64_t* bar, uint64_t pol) {
  Part parts[3];
  const int n = chunk_parts<MODE>(p, c0, c1, parts);
  uint32_t total = 0;
  for (int i = 0; i < n; i++) total += (uint32_t)(parts[i].hi - parts[i].lo) * p.seg[parts[i].seg].row_bytes;
  mbar_expect_tx(bar, total);
  for (int i = 0; i < n; i++) {
    const Seg& s = p.seg[parts[i].seg];
    bulk_g2s(stage + parts[i].off, s.w + (int64_t)parts[i].lo * s.row_bytes,
             (uint32_t)(parts[i].hi - parts[i].lo) * s.row_bytes, bar, pol);
  }
}

// ---------------------------------------------------------------------------
// Prologues: build the Q8_K activation(s) in shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (warp == 0) {
    t = lane < nw ? red[lane] : 0.f;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

// Q8_K of NB rows of `src` (global), optionally rmsnorm'ed first (candle
// rms_norm: y = x / sqrt(sum(x^2)/K + eps) * gamma, then Q8_K).
template <int NB>
__device__ void build_act(const MvParams& p, uint8_t* smem, const MvSmem& L, ActQ8 (&act)[NB]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const int K = p.K, nb = p.nb;
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* rms = red + 64;
  for (int b = 0; b < NB; b++) {
    act[b].qs = reinterpret_cast<int8_t*>(smem + L.act_qs) + (size_t)b * K;
    act[b].d = reinterpret_cast<float*>(smem + L.act_d) + (size_t)b * nb;
    act[b].bs = reinterpret_cast<int32_t*>(smem + L.act_bs) + (size_t)b * (K / 16);
  }
  const float* src = p.x;
  if (p.gamma) {
    float* xs = reinterpret_cast<float*>(smem + L.xbuf);
    for (int b = 0; b < NB; b++) {
      float ss = 0.f;
      for (int i = tid * 4; i < K; i += blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4*>(src + (size_t)b * K + i);
        *reinterpret_cast<float4*>(xs + (size_t)b * K + i) = v;
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      const float sum2 = block_sum(ss, red);
      if (tid == 0) rms[b] = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum2, (float)K), p.eps));
    }
    __syncthreads();
    for (int job = warp; job < NB * nb; job += nw) {
      const int b = job / nb, j = job % nb;
      const float m = rms[b];
      const float* xr = xs + (size_t)b * K + j * QK_K + 8 * lane;
      const float* gr = p.gamma + j * QK_K + 8 * lane;
      const float4 x0 = *reinterpret_cast<const float4*>(xr);
      const float4 x1 = *reinterpret_cast<const float4*>(xr + 4);
      const float4 g0 = *reinterpret_cast<const float4*>(gr);
      const float4 g1 = *reinterpret_cast<const float4*>(gr + 4);
      float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fdiv_rn(v[i], m), g[i]);
      q8k_quant_block_warp(v, lane, act[b].qs + j * QK_K, act[b].d + j, act[b].bs + j * 16);
    }
  } else {
    for (int job = warp; job < NB * nb; job += nw) {
      const int b = job / nb, j = job % nb;
      const float* xr = src + (size_t)b * K + j * QK_K + 8 * lane;
      const float4 x0 = *reinterpret_cast<const float4*>(xr);
      const float4 x1 = *reinterpret_cast<const float4*>(xr + 4);
      float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      q8k_quant_block_warp(v, lane, act[b].qs + j * QK_K, act[b].d + j, act[b].bs + j * 16);
    }
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
// The streaming matvec kernel.
// ---------------------------------------------------------------------------
template <int MODE, int NB>
__global__ void __launch_bounds__(MV_THREADS, 2) k_matvec(const MvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const MvSmem L = mv_smem_layout(p.ns, p.stage_bytes, p.K, NB, p.gamma != nullptr);
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int r1 = min(r0 + p.rows_per_cta, p.total_rows);
  const int nchunks = r1 > r0 ? (r1 - r0 + p.chunk_rows - 1) / p.chunk_rows : 0;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint8_t* stages = smem + L.stages;

  if (tid == 0) {
    for (int s = 0; s < p.ns; s++) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint64_t pol = l2_evict_first_policy();
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
  build_act<NB>(p, smem, L, act);

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
    const int np = chunk_parts<MODE>(p, c0, c1, parts);
    (void)np;
    if (MODE == MODE_QKV) {
      const int npairs = (c1 - c0) >> 1;
      for (int pr = warp; pr < npairs; pr += MV_WARPS) {
        const int r = c0 + 2 * pr;
        // segment of virtual row r and its first virtual row
        const int si = r < p.qn ? 0 : (r < p.qn + p.kn ? 1 : 2);
        const int sb = si == 0 ? 0 : (si == 1 ? p.qn : p.qn + p.kn);
        int pi = 0;
        for (int i = 0; i < np; i++)
          if (parts[i].seg == si) pi = i;
        const Seg& sg = p.seg[parts[pi].seg];
        const uint8_t* row = stage + parts[pi].off + (size_t)(r - sb - parts[pi].lo) * sg.row_bytes;
#pragma unroll
        for (int b = 0; b < NB; b++) {
          const float d0 = row_dot(sg.type, row, sg.nb, act[b], lane);
          const float d1 = row_dot(sg.type, row + sg.row_bytes, sg.nb, act[b], lane);
          if (lane == 0) {
            const int pos = p.pos[b];
            const int half = p.hd >> 1;
            if (r < p.qn + p.kn) {
              const int rr = r < p.qn ? r : r - p.qn;
              const int i2 = (rr % p.hd) >> 1;
              const float cs = p.cos_t[(size_t)pos * half + i2];
              const float sn = p.sin_t[(size_t)pos * half + i2];
              // candle rope_i: (a*c - b*s, a*s + b*c), each op rounded
              const float o0 = __fsub_rn(__fmul_rn(d0, cs), __fmul_rn(d1, sn));
              const float o1 = __fadd_rn(__fmul_rn(d0, sn), __fmul_rn(d1, cs));
              if (r < p.qn) {
                p.out[(size_t)b * p.out_stride + r] = o0;
                p.out[(size_t)b * p.out_stride + r + 1] = o1;
              } else {
                const int kvh = rr / p.hd, dd = rr % p.hd;
                const int64_t idx = (int64_t)b * p.kv_seq_stride + ((int64_t)kvh * p.max_seq + pos) * p.hd + dd;
                store_kv(p.kc, p.kv_f16, idx, o0, o1);
              }
            } else {
              const int rv = r - p.qn - p.kn;
              const int kvh = rv / p.hd, dd = rv % p.hd;
              const int64_t idx = (int64_t)b * p.kv_seq_stride + ((int64_t)kvh * p.max_seq + pos) * p.hd + dd;
              store_kv(p.vc, p.kv_f16, idx, d0, d1);
            }
          }
        }
      }
    } else if (MODE == MODE_GATEUP) {
      const Seg& sg = p.seg[0];
      const Seg& su = p.seg[1];
      for (int r = c0 + warp; r < c1; r += MV_WARPS) {
        const uint8_t* rg = stage + (size_t)(r - c0) * sg.row_bytes;
        const uint8_t* ru = stage + parts[1].off + (size_t)(r - c0) * su.row_bytes;
#pragma unroll
        for (int b = 0; b < NB; b++) {
          const float g = row_dot(sg.type, rg, sg.nb, act[b], lane);
          const float u = row_dot(su.type, ru, su.nb, act[b], lane);
          if (lane == 0) {
            // candle: silu(v) = v / (1 + exp(-v)); then * up
            const float sl = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
            p.out[(size_t)b * p.out_stride + r] = __fmul_rn(sl, u);
          }
        }
      }
    } else {
      const Seg& sg = p.seg[0];
      for (int r = c0 + warp; r < c1; r += MV_WARPS) {
        const uint8_t* row = stage + (size_t)(r - c0) * sg.row_bytes;
#pragma unroll
        for (int b = 0; b < NB; b++) {
          const float v = row_dot(sg.type, row, sg.nb, act[b], lane);
          if (lane == 0) {
            float* o = p.out + (size_t)b * p.out_stride + r;
            if (MODE == MODE_RESID) *o = __fadd_rn(v, *o);
            else *o = v;
            if (MODE == MODE_HEAD && am_better(v, r, best_v[b], best_i[b])) {
              best_v[b] = v;
              best_i[b] = r;
            }
          }
        }
      }
    }
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
    for (int b = 0; b < NB; b++) {
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
      for (int b = warp; b < NB; b += MV_WARPS) {
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
  int max_seq, hd, n_head, n_kv, splits, max_chunk;
  float scale;
  float* part;         // [NB][n_kv][splits][nrep][hd+2]
  unsigned* counters;  // [NB][n_kv]
  float* y;            // [NB][n_head*hd]
  uint32_t* err;
};

__device__ __forceinline__ float kv_load(const void* base, int kv_f16, int64_t idx) {
  return kv_f16 ? __half2float(reinterpret_cast<const __half*>(base)[idx])
                : reinterpret_cast<const float*>(base)[idx];
}

static __global__ void __launch_bounds__(128) k_attn_decode(const AttnParams p) {
  extern __shared__ __align__(16) float sm[];
  const int kvh = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nrep = p.n_head / p.n_kv, hd = p.hd;
  float* qs = sm;                        // [nrep][hd]
  float* sc = qs + nrep * hd;            // [nrep][max_chunk]
  float* ml = sc + nrep * p.max_chunk;   // [nrep][2]
  __shared__ int s_last;
  pdl_launch();
  pdl_wait();
  const int T = p.pos[b] + 1;
  const int chunk = (T + p.splits - 1) / p.splits;
  const int t0 = min(T, s * chunk), t1 = min(T, t0 + chunk), n = t1 - t0;
  const float* qb = p.q + (size_t)b * p.n_head * hd + (size_t)kvh * nrep * hd;
  for (int i = tid; i < nrep * hd; i += blockDim.x) qs[i] = qb[i];
  __syncthreads();
  const int64_t kvbase = (int64_t)b * p.kv_seq_stride + (int64_t)kvh * p.max_seq * hd;
  // scores: one position per thread
  for (int t = tid; t < n; t += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; r++) acc[r] = 0.f;
    const int64_t kb = kvbase + (int64_t)(t0 + t) * hd;
    for (int d = 0; d < hd; d++) {
      const float kv = kv_load(p.kc, p.kv_f16, kb + d);
#pragma unroll
      for (int r = 0; r < 8; r++)
        if (r < nrep) acc[r] += qs[r * hd + d] * kv;
    }
    for (int r = 0; r < nrep; r++) sc[r * p.max_chunk + t] = acc[r] * p.scale;
  }
  __syncthreads();
  // per-head max / exp / sum over this split
  for (int r = warp; r < nrep; r += 4) {
    float m = -INFINITY;
    for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[r * p.max_chunk + t]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float l = 0.f;
    for (int t = lane; t < n; t += 32) {
      const float e = n > 0 ? expf(sc[r * p.max_chunk + t] - m) : 0.f;
      sc[r * p.max_chunk + t] = e;
      l += e;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (lane == 0) { ml[2 * r] = m; ml[2 * r + 1] = l; }
  }
  __syncthreads();
  // o[r][d] = sum_t p[r][t] * v[t][d]
  const size_t pbase = ((((size_t)b * p.n_kv + kvh) * p.splits + s) * nrep) * (hd + 2);
  for (int d = tid; d < hd; d += blockDim.x) {
    float o[8];
#pragma unroll
    for (int r = 0; r < 8; r++) o[r] = 0.f;
    for (int t = 0; t < n; t++) {
      const float v = kv_load(p.vc, p.kv_f16, kvbase + (int64_t)(t0 + t) * hd + d);
#pragma unroll
      for (int r = 0; r < 8; r++)
        if (r < nrep) o[r] += sc[r * p.max_chunk + t] * v;
    }
    for (int r = 0; r < nrep; r++) p.part[pbase + (size_t)r * (hd + 2) + d] = o[r];
  }
  if (tid < nrep) {
    p.part[pbase + (size_t)tid * (hd + 2) + hd] = ml[2 * tid];
    p.part[pbase + (size_t)tid * (hd + 2) + hd + 1] = ml[2 * tid + 1];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&p.counters[b * p.n_kv + kvh], 1u);
    s_last = (prev == (unsigned)p.splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const size_t base0 = (((size_t)b * p.n_kv + kvh) * p.splits) * nrep * (hd + 2);
  for (int i = tid; i < nrep * hd; i += blockDim.x) {
    const int r = i / hd, d = i % hd;
    float M = -INFINITY;
    for (int s2 = 0; s2 < p.splits; s2++) {
      const size_t o = base0 + ((size_t)s2 * nrep + r) * (hd + 2);
      if (__ldcg(p.part + o + hd + 1) > 0.f) M = fmaxf(M, __ldcg(p.part + o + hd));
    }
    float Lsum = 0.f, O = 0.f;
    for (int s2 = 0; s2 < p.splits; s2++) {
      const size_t o = base0 + ((size_t)s2 * nrep + r) * (hd + 2);
      const float l = __ldcg(p.part + o + hd + 1);
      if (l > 0.f) {
        const float w = expf(__ldcg(p.part + o + hd) - M);
        Lsum += l * w;
        O += __ldcg(p.part + o + d) * w;
      }
    }
    p.y[(size_t)b * p.n_head * hd + ((size_t)kvh * nrep + r) * hd + d] = O / Lsum;
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
  // one warp per 256-value block
  for (int j = warp; j < nb; j += blockDim.x >> 5) {
    if (type == GGML_Q4_K) {
      const uint8_t* blk = row + (int64_t)j * Q4K_BLOCK_BYTES;
      const float d = h2f(*reinterpret_cast<const uint16_t*>(blk));
      const float dmin = h2f(*reinterpret_cast<const uint16_t*>(blk + 2));
      for (int i = lane; i < QK_K; i += 32) {
        const int c = i / 64, l = i % 64, sj = 2 * c + (l >= 32);
        const uint8_t byte = blk[16 + 32 * c + (l & 31)];
        const int q = l >= 32 ? (byte >> 4) : (byte & 0xF);
        int sc, m;
        q4k_scale_min(blk + 4, sj, sc, m);
        y[j * QK_K + i] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q),
                                    __fmul_rn(dmin, (float)m));
      }
    } else {
      const uint8_t* body = row + (int64_t)j * Q6K_BODY_BYTES;
      const uint16_t* dv = reinterpret_cast<const uint16_t*>(row + (int64_t)nb * Q6K_BODY_BYTES);
      for (int i = lane; i < QK_K; i += 32) {
        const int n = i / 128, r = i % 128, g = r / 32, l = r % 32;
        const uint8_t qlb = body[64 * n + l + (g & 1) * 32];
        const int lo = (g < 2) ? (qlb & 0xF) : (qlb >> 4);
        const int hi = (body[128 + 32 * n + l] >> (2 * g)) & 3;
        const int8_t sc = reinterpret_cast<const int8_t*>(body + 192)[8 * n + l / 16 + 2 * g];
        y[j * QK_K + i] = __fmul_rn(__fmul_rn(h2f(dv[j]), (float)sc), (float)((lo | (hi << 4)) - 32));
      }
    }
  }
}

static __global__ void k_set_int(int* p, int v) { *p = v; }

}  // namespace armai
