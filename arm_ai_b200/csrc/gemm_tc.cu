// gemm_tc.cu — device code and launchers of the tensor-core prefill GEMM
// (interface and design notes in gemm_tc.cuh).
#include "gemm_tc.cuh"

#include "kquant.cuh"
#include "llama_kernels.cuh"

namespace armai {

// ---- tcgen05 / mbarrier helpers (PTX) --------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// K-major operand, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t qg_smem_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);          // start address
  d |= (uint64_t)1u << 16;                          // leading byte offset (unused for this layout)
  d |= (uint64_t)(1024u >> 4) << 32;                // stride byte offset: next 8-row group
  d |= (uint64_t)1u << 46;                          // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                          // layout: 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: f16 A and B (K-major), f32 D, M = 128, N = 128.
__host__ __device__ constexpr uint32_t qg_instr_desc() {
  return (1u << 4)                 // D format f32
         | (0u << 7) | (0u << 10)  // A, B format f16
         | ((uint32_t)(QG_N >> 3) << 17) | ((uint32_t)(QG_M >> 4) << 24);
}

__device__ __forceinline__ void qg_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void qg_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Bounded parity wait (true when the phase completed); sets DEVERR on timeout.
__device__ __forceinline__ bool qg_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
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
    if (i > 16) __nanosleep(64);
  }
  atomicOr(err, DEVERR_MBAR_TIMEOUT);
  return false;
}

// 16 consecutive accumulator columns of this warp's 32 lanes.
__device__ __forceinline__ void qg_tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// ---- W dequantisation: 64 values [k0, k0 + 64) of one row, as 8 x 8 f16 ----
__device__ __forceinline__ void qg_store_row(uint8_t* tile, int r, const float (&v)[64]) {
#pragma unroll
  for (int c = 0; c < 8; c++) {
    __half2 h[4];
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(v[8 * c + 2 * i], v[8 * c + 2 * i + 1]);
    *reinterpret_cast<uint4*>(tile + r * 128 + ((c ^ (r & 7)) << 4)) = *reinterpret_cast<uint4*>(h);
  }
}

// BlockQ4K::to_float of values [64c, 64c + 64) of one super-block: bytes
// qs[32c .. 32c + 32) hold them (low nibbles: sub-block 2c, high: 2c + 1).
__device__ __forceinline__ void qg_deq_q4k(const uint8_t* blk, int c, float (&v)[64]) {
  const uint4 hd = __ldg(reinterpret_cast<const uint4*>(blk));
  const uint4 q0 = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 32 * c));
  const uint4 q1 = __ldg(reinterpret_cast<const uint4*>(blk + 32 + 32 * c));
  uint8_t sc8[12];
  const uint32_t sw[3] = {hd.y, hd.z, hd.w};
#pragma unroll
  for (int i = 0; i < 12; i++) sc8[i] = (uint8_t)(sw[i >> 2] >> (8 * (i & 3)));
  int sc0, m0, sc1, m1;
  q4k_scale_min(sc8, 2 * c, sc0, m0);
  q4k_scale_min(sc8, 2 * c + 1, sc1, m1);
  const float d = h2f((uint16_t)(hd.x & 0xffffu)), dmin = h2f((uint16_t)(hd.x >> 16));
  const float d0 = __fmul_rn(d, (float)sc0), mm0 = __fmul_rn(dmin, (float)m0);
  const float d1 = __fmul_rn(d, (float)sc1), mm1 = __fmul_rn(dmin, (float)m1);
  const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int l = 0; l < 32; l++) {
    const uint32_t b = (qw[l >> 2] >> (8 * (l & 3))) & 0xffu;
    v[l] = __fsub_rn(__fmul_rn(d0, (float)(b & 0xF)), mm0);
    v[32 + l] = __fsub_rn(__fmul_rn(d1, (float)(b >> 4)), mm1);
  }
}

// BlockQ6K::to_float of values [64t, 64t + 64) of one super-block (device
// body: ql 128, qh 64, i8 scales 16; d from the row's f16 array). With
// t = 2n + h, value 64t + i takes ql[64n + i] nibble h and qh[32n + (i & 31)]
// bits 4h + 2 (i >> 5); its scale is sc[4t + i / 16].
__device__ __forceinline__ void qg_deq_q6k(const uint8_t* body, float d, int t, float (&v)[64]) {
  const int n = t >> 1, h = t & 1;
  uint32_t lw[16], hw[8];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(body + 64 * n) + i);
    lw[4 * i] = a.x; lw[4 * i + 1] = a.y; lw[4 * i + 2] = a.z; lw[4 * i + 3] = a.w;
  }
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(body + 128 + 32 * n) + i);
    hw[4 * i] = a.x; hw[4 * i + 1] = a.y; hw[4 * i + 2] = a.z; hw[4 * i + 3] = a.w;
  }
  const uint32_t sc4 = __ldg(reinterpret_cast<const uint32_t*>(body + 192 + 4 * t));
#pragma unroll
  for (int i = 0; i < 64; i++) {
    const uint32_t lo = (lw[i >> 2] >> (8 * (i & 3) + 4 * h)) & 0xFu;
    const uint32_t hi = (hw[(i & 31) >> 2] >> (8 * (i & 3) + 4 * h + 2 * (i >> 5))) & 0x3u;
    const int q = (int)(lo | (hi << 4)) - 32;
    const float sc = (float)(int8_t)((sc4 >> (8 * (i >> 4))) & 0xffu);
    v[i] = __fmul_rn(__fmul_rn(d, sc), (float)q);
  }
}

__global__ void __launch_bounds__(QG_THREADS, 1) k_qgemm(const QgParams p) {
  extern __shared__ uint8_t qg_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // 1024-byte aligned tiles (the swizzle pattern repeats every 1024 bytes)
  const uint32_t raw_addr = smem_u32(qg_raw);
  uint8_t* smem = qg_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* a_st = smem;
  uint8_t* b_st = smem + QG_STAGES * QG_TILE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * QG_STAGES * QG_TILE_BYTES);
  uint64_t* empty = full + QG_STAGES;
  uint64_t* accb = empty + QG_STAGES;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accb + 1);
  __shared__ int s_fail;

  const int n0 = blockIdx.x * QG_N, m0 = blockIdx.y * QG_M;
  const int nk = p.k / QG_K;
  if (tid == 0) {
    for (int s = 0; s < QG_STAGES; s++) {
      mbar_init(&full[s], 1 + 4);   // A copy (arrive + tx) and the 4 dequantising warps
      mbar_init(&empty[s], 1);      // tcgen05.commit after the stage's MMAs
    }
    mbar_init(accb, 1);
    fence_mbar_init();
    s_fail = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(QG_N)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      const uint8_t* asrc = p.a_tiles + (size_t)blockIdx.y * nk * QG_TILE_BYTES;
      const uint64_t pol = l2_evict_first_policy();
      int issued = 0;
      for (int kc = 0; kc < nk; kc++) {
        const int s = kc % QG_STAGES;
        if (kc >= QG_STAGES && !qg_wait(&empty[s], (uint32_t)((kc / QG_STAGES - 1) & 1), p.err)) break;
        mbar_arrive_tx(&full[s], QG_TILE_BYTES);
        bulk_g2s(a_st + s * QG_TILE_BYTES, asrc + (size_t)kc * QG_TILE_BYTES, QG_TILE_BYTES, &full[s], pol);
        issued = kc + 1;
      }
      // every copy this thread issued has landed before the CTA may exit
      for (int kc = issued > QG_STAGES ? issued - QG_STAGES : 0; kc < issued; kc++)
        qg_wait(&full[kc % QG_STAGES], (uint32_t)((kc / QG_STAGES) & 1), p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = qg_instr_desc();
      for (int kc = 0; kc < nk; kc++) {
        const int s = kc % QG_STAGES;
        if (!qg_wait(&full[s], (uint32_t)((kc / QG_STAGES) & 1), p.err)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(a_st + s * QG_TILE_BYTES), b0 = smem_u32(b_st + s * QG_TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < QG_K / 16; kk++)   // K = 16 per MMA: 32 bytes along the swizzled row
          qg_mma(taddr, qg_smem_desc(a0 + 32 * kk), qg_smem_desc(b0 + 32 * kk), idesc, (kc | kk) != 0);
        qg_commit(&empty[s]);
      }
      qg_commit(accb);  // also on an early exit: completes once the issued MMAs have
    }
    __syncwarp();
  } else {
    // ---- W producers: thread r owns weight row n0 + r of the tile ----
    const int r = tid - 64;
    const int n = n0 + r;
    int si = -1, nl = 0;
    {
      int base = 0;
      for (int s = 0; s < p.nseg; s++) {
        if (n >= base && n < base + p.seg[s].rows) { si = s; nl = n - base; }
        base += p.seg[s].rows;
      }
    }
    const uint8_t* wrow = si >= 0 ? p.seg[si].w + (size_t)nl * p.seg[si].row_bytes : nullptr;
    const int wtype = si >= 0 ? p.seg[si].type : 0;
    const int nb = p.k / QK_K;
    bool ok = true;
    for (int kc = 0; kc < nk; kc++) {
      const int s = kc % QG_STAGES;
      if (kc >= QG_STAGES && !qg_wait(&empty[s], (uint32_t)((kc / QG_STAGES - 1) & 1), p.err)) { ok = false; break; }
      float v[64];
      const int blk = kc >> 2, c = kc & 3;
      if (!wrow) {
#pragma unroll
        for (int i = 0; i < 64; i++) v[i] = 0.f;
      } else if (wtype == GGML_Q4_K) {
        qg_deq_q4k(wrow + (size_t)blk * Q4K_BLOCK_BYTES, c, v);
      } else {
        const float d = h2f(__ldg(reinterpret_cast<const uint16_t*>(wrow + (size_t)nb * Q6K_BODY_BYTES) + blk));
        qg_deq_q6k(wrow + (size_t)blk * Q6K_BODY_BYTES, d, c, v);
      }
      qg_store_row(b_st + s * QG_TILE_BYTES, r, v);
      fence_async_smem();  // generic-proxy writes -> visible to the tensor cores
      __syncwarp();
      if (lane == 0) mbar_arrive1(&full[s]);
    }
    if (!ok) atomicExch(&s_fail, 1);
    // ---- epilogue: this warp's 32 tokens x 128 columns ----
    const bool acc_ok = qg_wait(accb, 0, p.err);
    tc_fence_after();
    const int q = warp & 3;                 // tensor-memory lane quarter of this warp
    const int m = m0 + 32 * q + lane;
    if (acc_ok) {
#pragma unroll 1
      for (int c0 = 0; c0 < QG_N; c0 += 16) {
        float v[16];
        qg_tmem_ld16(taddr + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
        if (m < p.m) {
          float* o = p.out + (size_t)m * p.ldo + n0 + c0;
          if (n0 + c0 + 16 <= p.n) {
#pragma unroll
            for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          } else {
            for (int i = 0; i < 16; i++)
              if (n0 + c0 + i < p.n) o[i] = v[i];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(QG_N) : "memory");
  }
}

// ---- A operand: (rms-norm +) Q8_K + f16 expansion into swizzled tiles ------
// One CTA (256 threads) per token row; rows m..m_pad-1 are zero. The norm
// follows candle's rms_norm with per-block partial sums added in block order
// (as the decode kernels); Q8_K as BlockQ8K::from_float.
__global__ void __launch_bounds__(256) k_qgemm_act(const float* __restrict__ x, const float* __restrict__ gamma,
                                                   float eps, int m, int k, uint8_t* __restrict__ a_tiles) {
  __shared__ float part[64];  // K <= 16384
  __shared__ float s_rms;
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = k / QK_K, nkc = k / QG_K;
  uint8_t* tbase = a_tiles + (size_t)(row / QG_M) * nkc * QG_TILE_BYTES;
  const int r = row % QG_M;
  if (row >= m) {
    for (int c = tid; c < nkc * 8; c += blockDim.x)
      *reinterpret_cast<uint4*>(tbase + (size_t)(c >> 3) * QG_TILE_BYTES + r * 128 + (((c & 7) ^ (r & 7)) << 4)) =
          make_uint4(0, 0, 0, 0);
    return;
  }
  const float* xr = x + (size_t)row * k;
  float inv_m = 1.f;
  if (gamma) {
    for (int j = warp; j < nb; j += 8) {
      const float4 a = *reinterpret_cast<const float4*>(xr + j * QK_K + 8 * lane);
      const float4 b = *reinterpret_cast<const float4*>(xr + j * QK_K + 8 * lane + 4);
      float ss = a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) part[j] = ss;
    }
    __syncthreads();
    if (tid == 0) {
      float sum2 = 0.f;
      for (int j = 0; j < nb; j++) sum2 += part[j];
      s_rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum2, (float)k), eps));
    }
    __syncthreads();
    inv_m = s_rms;
  }
  for (int j = warp; j < nb; j += 8) {
    const float4 a = *reinterpret_cast<const float4*>(xr + j * QK_K + 8 * lane);
    const float4 b = *reinterpret_cast<const float4*>(xr + j * QK_K + 8 * lane + 4);
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if (gamma) {
      const float4 g0 = *reinterpret_cast<const float4*>(gamma + j * QK_K + 8 * lane);
      const float4 g1 = *reinterpret_cast<const float4*>(gamma + j * QK_K + 8 * lane + 4);
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fdiv_rn(v[i], inv_m), g[i]);
    }
    // BlockQ8K::from_float: first value of largest magnitude sets the scale
    float amax = 0.f, mx = 0.f;
    int idx = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float av = fabsf(v[i]);
      if (amax < av) { amax = av; mx = v[i]; idx = 8 * lane + i; }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
      const float om = __shfl_xor_sync(0xffffffffu, mx, off);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
      if (oa > amax || (oa == amax && oi < idx)) { amax = oa; mx = om; idx = oi; }
    }
    __half2 h[4];
    if (amax != 0.f) {
      const float iscale = __fdiv_rn(-128.f, mx);
      const float d = __fdiv_rn(1.0f, iscale);
      float q[8];
#pragma unroll
      for (int i = 0; i < 8; i++) q[i] = __fmul_rn(fmaxf(fminf(roundf(__fmul_rn(iscale, v[i])), 127.f), -128.f), d);
#pragma unroll
      for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(q[2 * i], q[2 * i + 1]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(0.f, 0.f);
    }
    // values [j*256 + 8 lane, +8): k-chunk 4j + lane/8, 16-byte chunk lane % 8
    const int kc = 4 * j + (lane >> 3), c = lane & 7;
    *reinterpret_cast<uint4*>(tbase + (size_t)kc * QG_TILE_BYTES + r * 128 + ((c ^ (r & 7)) << 4)) =
        *reinterpret_cast<uint4*>(h);
  }
}

// ---- prefill epilogues --------------------------------------------------
__global__ void k_qkv_post(const float* __restrict__ g, int ldg, int S, const int* __restrict__ pos, int qn,
                           int kn, int hd, int max_seq, const float* __restrict__ cos_t,
                           const float* __restrict__ sin_t, float* __restrict__ q_out, void* kc, void* vc,
                           int kv_f16) {
  const int t = blockIdx.y;
  const int pr = blockIdx.x * blockDim.x + threadIdx.x;  // row pair
  const int rows = ldg;
  if (t >= S || 2 * pr >= rows) return;
  const int r = 2 * pr;
  const float d0 = g[(size_t)t * ldg + r], d1 = g[(size_t)t * ldg + r + 1];
  const int p = pos[t], half = hd >> 1;
  if (r < qn + kn) {
    const int rr = r < qn ? r : r - qn;
    const int i2 = (rr % hd) >> 1;
    const float cs = cos_t[(size_t)p * half + i2], sn = sin_t[(size_t)p * half + i2];
    // candle rope_i: (a*c - b*s, a*s + b*c), each op rounded
    const float o0 = __fsub_rn(__fmul_rn(d0, cs), __fmul_rn(d1, sn));
    const float o1 = __fadd_rn(__fmul_rn(d0, sn), __fmul_rn(d1, cs));
    if (r < qn) {
      *reinterpret_cast<float2*>(q_out + (size_t)t * qn + r) = make_float2(o0, o1);
    } else {
      const int kvh = rr / hd, dd = rr % hd;
      store_kv(kc, kv_f16, ((int64_t)kvh * max_seq + p) * hd + dd, o0, o1);
    }
  } else {
    const int rv = r - qn - kn;
    const int kvh = rv / hd, dd = rv % hd;
    store_kv(vc, kv_f16, ((int64_t)kvh * max_seq + p) * hd + dd, d0, d1);
  }
}

__global__ void k_resid_add(float* __restrict__ x, const float* __restrict__ g, int S, int n, int ldg) {
  const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (t < S && i < n) x[(size_t)t * n + i] = __fadd_rn(g[(size_t)t * ldg + i], x[(size_t)t * n + i]);
}

__global__ void k_silu_mul(const float* __restrict__ g, int S, int n, float* __restrict__ h) {
  const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= S || i >= n) return;
  const float v = g[(size_t)t * 2 * n + i], u = g[(size_t)t * 2 * n + n + i];
  h[(size_t)t * n + i] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u);
}

int qkv_post_launch(const float* g, int ldg, int S, const int* pos, int qn, int kn, int hd, int max_seq,
                    const float* cos_t, const float* sin_t, float* q_out, void* kc, void* vc, int kv_f16,
                    cudaStream_t s) {
  const dim3 grid((unsigned)((ldg / 2 + 127) / 128), (unsigned)S);
  k_qkv_post<<<grid, 128, 0, s>>>(g, ldg, S, pos, qn, kn, hd, max_seq, cos_t, sin_t, q_out, kc, vc, kv_f16);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

int resid_add_launch(float* x, const float* g, int S, int n, int ldg, cudaStream_t s) {
  k_resid_add<<<dim3((unsigned)((n + 255) / 256), (unsigned)S), 256, 0, s>>>(x, g, S, n, ldg);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

int silu_mul_launch(const float* g, int S, int n, float* h, cudaStream_t s) {
  k_silu_mul<<<dim3((unsigned)((n + 255) / 256), (unsigned)S), 256, 0, s>>>(g, S, n, h);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

int qgemm_act_launch(const float* x, const float* gamma, float eps, int m, int k, uint8_t* a_tiles,
                     cudaStream_t s) {
  if (k % QK_K || k / QK_K > 64) return fail(ARMAI_E_INVALID, "qgemm: K must be a multiple of 256, at most 16384");
  const int m_pad = ((m + QG_M - 1) / QG_M) * QG_M;
  k_qgemm_act<<<m_pad, 256, 0, s>>>(x, gamma, eps, m, k, a_tiles);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

int qgemm_launch(const QgParams& p, cudaStream_t s) {
  static thread_local int attr_dev = -1;
  int dev = 0;
  ARMAI_CUDA(cudaGetDevice(&dev));
  if (attr_dev != dev) {
    ARMAI_CUDA(cudaFuncSetAttribute(k_qgemm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QG_SMEM));
    attr_dev = dev;
  }
  const dim3 grid((unsigned)((p.n + QG_N - 1) / QG_N), (unsigned)((p.m + QG_M - 1) / QG_M));
  k_qgemm<<<grid, QG_THREADS, QG_SMEM, s>>>(p);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

}  // namespace armai
