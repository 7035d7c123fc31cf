// gemm_tc.cu — device code and launchers of the tensor-core GEMM for
// prompts and batched decode (interface and design notes in gemm_tc.cuh).
#include "gemm_tc.cuh"

#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "kquant.cuh"
#include "llama_kernels.cuh"
#include "tcgen05.cuh"
#include "fa_tc.cuh"

namespace armai {

namespace {
template <typename... KArgs, typename... Args>
cudaError_t qg_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
}  // namespace

// kind::f16 instruction descriptor: f16 A (tensor memory) and B (shared
// memory, K-major), f32 D, M = 128 weight rows, N = ntok tokens.
__host__ __device__ constexpr uint32_t qg_instr_desc(int ntok) {
  return (1u << 4)                 // D format f32
         | (0u << 7) | (0u << 10)  // A, B format f16
         | ((uint32_t)(ntok >> 3) << 17) | ((uint32_t)(QG_W >> 4) << 24);
}

// ---- packed f32 pairs (sm_100 f32x2 arithmetic) ----------------------------
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint32_t f2_to_h2(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// 2^23 + byte i of x: an f32 whose value is exact (bytes are at most 255).
__device__ __forceinline__ float qg_byte_f(uint32_t x, int i) {
  return __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7440u | (uint32_t)i));
}

// ---- W dequantisation from raw super-blocks in shared memory --------------
// A stage of a super-block holds 64 values; DW / 4 dequantising warps share
// it per tensor-memory lane quarter, each taking VPT = 64 / (DW / 4)
// consecutive values (part kp: values kp VPT .. kp VPT + VPT - 1).

// Q4_K (BlockQ4K::to_float): stage c holds values [64c, 64c + 64):
// sub-block 2c (low nibbles of qs[32c .. 32c + 32)) and 2c + 1 (high
// nibbles). Value l of sub-block j is d * sc_j * q_l - dmin * m_j (the
// products d * sc and dmin * m rounded in f32 as candle does; the last step
// fused), rounded to f16 in pairs.
template <int QG_VPT>
__device__ __forceinline__ void qg_deq_q4k(const uint8_t* blk, uint4 hd, int c, int kp,
                                           uint32_t (&o)[QG_VPT / 2]) {
  const int off = kp * QG_VPT, nib = off >> 5, l0 = off & 31;
  // 6-bit scale and min of sub-block j = 2c + nib from the 12 scale bytes
  // (header words y, z, w), as get_scale_min_k4, in registers
  const int j = 2 * c + nib, j4 = (j & 3) * 8;
  int sc, mn;
  if (j < 4) {
    sc = (int)((hd.y >> j4) & 63u);
    mn = (int)((hd.z >> j4) & 63u);
  } else {
    const uint32_t s8 = (hd.w >> j4) & 0xffu, s0 = (hd.y >> j4) & 0xffu, s4 = (hd.z >> j4) & 0xffu;
    sc = (int)((s8 & 0xFu) | ((s0 >> 6) << 4));
    mn = (int)((s8 >> 4) | ((s4 >> 6) << 4));
  }
  const float d = h2f((uint16_t)(hd.x & 0xffffu)), dmin = h2f((uint16_t)(hd.x >> 16));
  const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
  const uint64_t dd = f2_pack(d1, d1), mm = f2_pack(-m1, -m1), bias = f2_pack(-8388608.f, -8388608.f);
  uint32_t qw[QG_VPT / 4];
#pragma unroll
  for (int i = 0; i < QG_VPT / 16; i++) {
    const uint4 q = *reinterpret_cast<const uint4*>(blk + 16 + 32 * c + l0 + 16 * i);
    qw[4 * i] = q.x; qw[4 * i + 1] = q.y; qw[4 * i + 2] = q.z; qw[4 * i + 3] = q.w;
  }
#pragma unroll
  for (int w = 0; w < QG_VPT / 4; w++) {
    const uint32_t x = (qw[w] >> (4 * nib)) & 0x0F0F0F0Fu;
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const uint64_t n = f2_add(f2_pack(qg_byte_f(x, 2 * i), qg_byte_f(x, 2 * i + 1)), bias);
      o[2 * w + i] = f2_to_h2(f2_fma(n, dd, mm));
    }
  }
}

// Q6_K (BlockQ6K::to_float; device body: ql 128, qh 64, i8 scales 16, d from
// the row's f16 array): stage t = 2n + hq holds values 128n + 64hq + [0, 64);
// value 32h + l of the stage takes ql[64n + 32h + l] nibble hq and
// qh[32n + l] bits 4hq + 2h, scale sc[4t + 2h + l / 16]; (d * sc) * (q - 32).
template <int QG_VPT>
__device__ __forceinline__ void qg_deq_q6k(const uint8_t* body, float d, int t, int kp,
                                           uint32_t (&o)[QG_VPT / 2]) {
  const int n = t >> 1, hq = t & 1, off = kp * QG_VPT, h = off >> 5, l0 = off & 31;
  uint32_t lw[QG_VPT / 4], hw[QG_VPT / 4];
#pragma unroll
  for (int i = 0; i < QG_VPT / 16; i++) {
    const uint4 a = *reinterpret_cast<const uint4*>(body + 64 * n + 32 * h + l0 + 16 * i);
    const uint4 b = *reinterpret_cast<const uint4*>(body + 128 + 32 * n + l0 + 16 * i);
    lw[4 * i] = a.x; lw[4 * i + 1] = a.y; lw[4 * i + 2] = a.z; lw[4 * i + 3] = a.w;
    hw[4 * i] = b.x; hw[4 * i + 1] = b.y; hw[4 * i + 2] = b.z; hw[4 * i + 3] = b.w;
  }
  const int8_t* sc = reinterpret_cast<const int8_t*>(body + 192 + 4 * t + 2 * h + (l0 >> 4));
  const uint64_t bias = f2_pack(-8388640.f, -8388640.f);  // -(2^23 + 32)
#pragma unroll
  for (int w = 0; w < QG_VPT / 4; w++) {
    const float s = __fmul_rn(d, (float)sc[w >> 2]);
    const uint64_t ss = f2_pack(s, s);
    const uint32_t x = ((lw[w] >> (4 * hq)) & 0x0F0F0F0Fu) | (((hw[w] >> (4 * hq + 2 * h)) & 0x03030303u) << 4);
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const uint64_t q = f2_add(f2_pack(qg_byte_f(x, 2 * i), qg_byte_f(x, 2 * i + 1)), bias);
      o[2 * w + i] = f2_to_h2(f2_mul(ss, q));
    }
  }
}

// 2-D TMA load (no multicast) of a box of raw weight rows into shared memory.
__device__ __forceinline__ void qg_tma_load(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Segment holding weight row n (its index and the row within it), -1 past the end.
__device__ __forceinline__ int qg_find_seg(const QgParams& p, int n, int& local) {
  int base = 0, si = -1;
  local = 0;
  for (int s2 = 0; s2 < p.nseg; s2++) {
    if (n >= base && n < base + p.seg[s2].rows) { si = s2; local = n - base; }
    base += p.seg[s2].rows;
  }
  return si;
}

// Grid: x = 128-row weight tiles, y = token tiles (p.ntok tokens), z = K
// splits (p.kb_split super-blocks each). DW dequantising warps.
template <int DW>
__global__ void __launch_bounds__(32 * (3 + DW), 1) k_qgemm(const __grid_constant__ QgMaps maps, const QgParams p) {
  constexpr int QG_KPARTS = DW / 4, QG_VPT = 64 / QG_KPARTS;
  extern __shared__ uint8_t qg_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // 1024-byte aligned tiles (the swizzle pattern repeats every 1024 bytes)
  const uint32_t raw_addr = smem_u32(qg_raw);
  uint8_t* smem = qg_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  const int ntok = p.ntok;
  const uint32_t b_bytes = (uint32_t)ntok * 128u;
  uint8_t* b_st = smem;                            // token tiles: QG_STAGES x ntok rows x 128 B
  uint8_t* rw = b_st + QG_STAGES * b_bytes;        // raw weight slots (128-byte aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(rw + QG_RAW_SLOTS * QG_RAW_SLOT_BYTES);
  uint64_t* empty = full + QG_STAGES;
  uint64_t* rfull = empty + QG_STAGES;
  uint64_t* rempty = rfull + QG_RAW_SLOTS;
  uint64_t* accb = rempty + QG_RAW_SLOTS;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accb + 1);

  const int n0 = blockIdx.x * QG_W, t0 = blockIdx.y * ntok;
  const int nb_all = p.k / QK_K;
  const int kb0 = blockIdx.z * p.kb_split, nblk = min(nb_all, kb0 + p.kb_split) - kb0;
  const int nk = 4 * nblk;
  if (tid == 0) {
    for (int s = 0; s < QG_STAGES; s++) {
      mbar_init(&full[s], 1 + DW);  // token copy (arrive + tx) and the dequantising warps
      mbar_init(&empty[s], 1);                // tcgen05.commit after the stage's MMAs
    }
    for (int r = 0; r < QG_RAW_SLOTS; r++) {
      mbar_init(&rfull[r], 1);                // the raw loader's arrival + tx
      mbar_init(&rempty[r], DW);    // every dequantising warp done with the slot
    }
    mbar_init(accb, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tslot;
  const uint32_t t_a = taddr + (uint32_t)p.acc_cols;  // A stages: 32 columns each

  if (warp == 0) {
    if (lane == 0) {
      // token rows [t0, t0 + ntok) of k-chunk kc: within one 128-token tile
      // (ntok <= 128, t0 = 0) or two whole tiles (ntok = 256)
      const int nkc_all = p.k / QG_K;
      const int parts = ntok > 128 ? 2 : 1;
      const uint32_t part_bytes = ntok > 128 ? QG_TILE_BYTES : b_bytes;
      // the activation tiles come from the previous kernel (programmatic
      // dependent launch: everything before this point overlaps it; the
      // epilogue's stores follow the MMAs, which follow these copies)
      pdl_wait();
      const uint64_t pol = l2_evict_last_policy();
      int issued = 0;
      for (int kc = 0; kc < nk; kc++) {
        const int s = kc % QG_STAGES;
        if (kc >= QG_STAGES && !qg_wait(&empty[s], (uint32_t)((kc / QG_STAGES - 1) & 1), p.err)) break;
        mbar_arrive_tx(&full[s], b_bytes);
        const int kcg = 4 * kb0 + kc;
        for (int part = 0; part < parts; part++) {
          const int mt = t0 / 128 + part;
          bulk_g2s(b_st + s * b_bytes + part * QG_TILE_BYTES,
                   p.a_tiles + ((size_t)mt * nkc_all + kcg) * QG_TILE_BYTES, part_bytes, &full[s], pol);
        }
        issued = kc + 1;
      }
      // every copy this thread issued has landed before the CTA may exit
      for (int kc = issued > QG_STAGES ? issued - QG_STAGES : 0; kc < issued; kc++)
        qg_wait(&full[kc % QG_STAGES], (uint32_t)((kc / QG_STAGES) & 1), p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = qg_instr_desc(ntok);
      for (int kc = 0; kc < nk; kc++) {
        const int s = kc % QG_STAGES;
        if (!qg_wait(&full[s], (uint32_t)((kc / QG_STAGES) & 1), p.err)) break;
        tc_fence_after();
        const uint32_t b0 = smem_u32(b_st + s * b_bytes);
#pragma unroll
        for (int kk = 0; kk < QG_K / 16; kk++)   // K = 16 per MMA: 8 columns of A, 32 bytes along B's rows
          qg_mma_ts(taddr, t_a + 32 * s + 8 * kk, qg_smem_desc(b0 + 32 * kk), idesc, (kc | kk) != 0);
        qg_commit(&empty[s]);
      }
      qg_commit(accb);  // also on an early exit: completes once the issued MMAs have
    }
    __syncwarp();
  } else if (warp == 2) {
    if (lane == 0) {
      // raw super-blocks: 32-row groups g of the tile, each from the segment
      // holding it (segments before the last hold multiples of 32 rows; rows
      // past a segment's end or the matrix are zero-filled by the TMA unit)
      int gseg[4], grow[4], gbb[4];
      uint32_t tx = 0;
#pragma unroll
      for (int g = 0; g < 4; g++) {
        int nl;
        int si = qg_find_seg(p, n0 + 32 * g, nl);
        if (si < 0) { si = p.nseg - 1; nl = p.seg[si].rows; }  // past the matrix: all fill
        gseg[g] = si;
        grow[g] = nl;
        gbb[g] = p.seg[si].type == GGML_Q4_K ? Q4K_BLOCK_BYTES : Q6K_BODY_BYTES;
        tx += 32u * (uint32_t)gbb[g];
      }
      int issued = 0;
      for (int b = 0; b < nblk; b++) {
        const int r = b % QG_RAW_SLOTS;
        if (b >= QG_RAW_SLOTS && !qg_wait(&rempty[r], (uint32_t)((b / QG_RAW_SLOTS - 1) & 1), p.err)) break;
        mbar_arrive_tx(&rfull[r], tx);
#pragma unroll
        for (int g = 0; g < 4; g++)
          qg_tma_load(rw + r * QG_RAW_SLOT_BYTES + g * QG_RAW_GROUP_BYTES, &maps.m[gseg[g]], (kb0 + b) * gbb[g],
                      grow[g], &rfull[r]);
        issued = b + 1;
      }
      for (int b = issued > QG_RAW_SLOTS ? issued - QG_RAW_SLOTS : 0; b < issued; b++)
        qg_wait(&rfull[b % QG_RAW_SLOTS], (uint32_t)((b / QG_RAW_SLOTS) & 1), p.err);
    }
  } else {
    // ---- W dequantisers: warp -> tensor-memory lane quarter q, K part kp ----
    const int q = warp & 3, kp = (warp - 3) >> 2;
    const int r = 32 * q + lane, n = n0 + r;
    int nl;
    const int si = qg_find_seg(p, n, nl);
    const int wtype = si >= 0 ? p.seg[si].type : 0;
    const int bb = wtype == GGML_Q4_K ? Q4K_BLOCK_BYTES : Q6K_BODY_BYTES;
    const uint16_t* q6d = (si >= 0 && wtype == GGML_Q6_K)
                              ? reinterpret_cast<const uint16_t*>(p.seg[si].w + (size_t)nl * p.seg[si].row_bytes +
                                                                  (size_t)nb_all * Q6K_BODY_BYTES)
                              : nullptr;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    uint4 hd = make_uint4(0, 0, 0, 0);
    float d6 = 0.f;
    for (int kc = 0; kc < nk; kc++) {
      const int s = kc % QG_STAGES, b = kc >> 2, c = kc & 3, rs = b % QG_RAW_SLOTS;
      const uint8_t* row = rw + rs * QG_RAW_SLOT_BYTES + q * QG_RAW_GROUP_BYTES + lane * bb;
      if (c == 0) {
        if (!qg_wait_warp(&rfull[rs], (uint32_t)((b / QG_RAW_SLOTS) & 1), p.err)) break;
        if (q6d) d6 = h2f(__ldg(q6d + kb0 + b));
        else hd = *reinterpret_cast<const uint4*>(row);
      }
      uint32_t o[QG_VPT / 2];
      if (si < 0) {
#pragma unroll
        for (int i = 0; i < QG_VPT / 2; i++) o[i] = 0u;
      } else if (wtype == GGML_Q4_K) {
        qg_deq_q4k<QG_VPT>(row, hd, c, kp, o);
      } else {
        qg_deq_q6k<QG_VPT>(row, d6, c, kp, o);
      }
      __syncwarp();
      if (lane == 0 && c == 3) mbar_arrive1(&rempty[rs]);  // the raw slot's last stage has been read
      // the MMAs of the stage that last used these columns have completed
      if (kc >= QG_STAGES && !qg_wait_warp(&empty[s], (uint32_t)((kc / QG_STAGES - 1) & 1), p.err)) break;
      tc_fence_after();
      const uint32_t ta = t_a + lane_base + 32 * s + (QG_VPT / 2) * kp;
      qg_tmem_st(ta, o);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive1(&full[s]);
    }
    // ---- epilogue: this warp's 32 weight rows x every QG_KPARTS-th group of 8 tokens ----
    const bool acc_ok = qg_wait_warp(accb, 0, p.err);
    tc_fence_after();
    if (acc_ok) {
      float* out = p.out + (size_t)blockIdx.z * p.split_stride;
#pragma unroll 1
      for (int c0 = 8 * kp; c0 < ntok; c0 += 8 * QG_KPARTS) {
        float v[8];
        qg_tmem_ld8(taddr + lane_base + (uint32_t)c0, v);
        if (n < p.n) {
#pragma unroll
          for (int j = 0; j < 8; j++) {
            const int t = t0 + c0 + j;
            if (t < p.m) {
              float* o2 = out + (size_t)t * p.ldo + n;
              *o2 = p.add ? __fadd_rn(v[j], *o2) : v[j];
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(p.tmem_cols) : "memory");
  }
}

// ---- B operand: (rms-norm +) Q8_K + f16 expansion into swizzled tiles ------
// Q8_K (BlockQ8K::from_float: the first value of largest magnitude sets the
// scale) of one 256-value block j held 8 per lane (values 8 lane .. + 7),
// expanded to f16 q * d, into token row r of the block's four k-chunk tiles.
__device__ __forceinline__ void qg_act_block(const float (&v)[8], int lane, int j, int r, uint8_t* tbase) {
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

__device__ __forceinline__ void qg_ld8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// The split sums of 8 consecutive columns of two column sets (offsets oa,
// ob; ob < 0: one set), each added in split order. All loads of a batch of
// splits are issued before the first add, so a row kernel waits for one
// memory round trip per batch rather than one per split (B splits per batch:
// 8 for one set, 4 for two).
template <int B>
__device__ __forceinline__ void qg_split_sum8x2(const QgSplit& g, size_t oa, long long ob, float (&va)[8],
                                                float (&vb)[8]) {
  for (int sp0 = 0; sp0 < g.splits; sp0 += B) {
    float wa[B][8], wb[B][8];
#pragma unroll
    for (int u = 0; u < B; u++)
      if (sp0 + u < g.splits) {
        qg_ld8(g.ws + (size_t)(sp0 + u) * g.stride + oa, wa[u]);
        if (ob >= 0) qg_ld8(g.ws + (size_t)(sp0 + u) * g.stride + (size_t)ob, wb[u]);
      }
#pragma unroll
    for (int u = 0; u < B; u++)
      if (sp0 + u < g.splits) {
#pragma unroll
        for (int i = 0; i < 8; i++) {
          va[i] = sp0 + u == 0 ? wa[u][i] : __fadd_rn(va[i], wa[u][i]);
          if (ob >= 0) vb[i] = sp0 + u == 0 ? wb[u][i] : __fadd_rn(vb[i], wb[u][i]);
        }
      }
  }
}
template <int B>
__device__ __forceinline__ void qg_split_sum8(const QgSplit& g, size_t off, float (&v)[8]) {
  float unused[8];
  qg_split_sum8x2<B>(g, off, -1, v, unused);
}

enum { ACT_X = 0, ACT_RESID = 1, ACT_SILU = 2 };
struct RowAct {
  const float* x;    // ACT_X: input rows [m][k]
  float* xo;         // ACT_RESID: residual rows [m][k], updated in place
  const float* gamma;
  float eps;
  int k;
  QgSplit g;         // ACT_RESID, ACT_SILU
  uint8_t* a_tiles;  // null: no tiles (ACT_RESID only)
};

// Token row blockIdx.x, one warp per 256-value block: the row's values
// (ACT_X: x; ACT_RESID: x + the split sums, stored back; ACT_SILU:
// silu(gate) * up from the split sums), optionally rms-normalised with gamma,
// as activation tiles. ACT_X / ACT_RESID: one CTA per row (the norm needs the
// whole row). ACT_SILU (no norm): blockIdx.y picks
// the row's blocks [y * warps, (y + 1) * warps). The norm follows candle's
// rms_norm with per-block partial sums added in block order (as the decode
// kernels). B: split partials loaded per round trip — 8 for few rows (a
// decode batch: latency; a warp's first block also stays in registers across
// the norm's barrier), 2 for many (a prompt: registers, occupancy; every
// block is read again after the barrier).
template <int KIND, int B>
__global__ void __launch_bounds__(512) k_row_act(const RowAct p) {
  pdl_launch();
  pdl_wait();
  __shared__ float part[64];  // K <= 16384
  __shared__ float s_rms;
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const int k = p.k, nb = k / QK_K, nkc = k / QG_K;
  uint8_t* tbase = p.a_tiles ? p.a_tiles + (size_t)(row / 128) * nkc * QG_TILE_BYTES : nullptr;
  const int r = row % 128;
  const float* xr = KIND == ACT_X ? p.x + (size_t)row * k : p.xo + (size_t)row * k;
  const bool norm = KIND != ACT_SILU && p.gamma != nullptr && tbase != nullptr;
  constexpr bool KEEP = B >= 8;
  const int j0 = KIND == ACT_SILU ? (int)blockIdx.y * nw : 0, j1 = KIND == ACT_SILU ? min(nb, j0 + nw) : nb;
  float keep[8], g0[8];
  for (int j = j0 + warp; j < j1; j += nw) {
    const int col = j * QK_K + 8 * lane;
    float v[8];
    if (KEEP && norm && j == warp) qg_ld8(p.gamma + col, g0);  // used after the barrier
    if (KIND == ACT_X) {
      qg_ld8(xr + col, v);
    } else if (KIND == ACT_RESID) {
      float x0[8];
      qg_ld8(xr + col, x0);
      qg_split_sum8<B>(p.g, (size_t)row * p.g.ld + col, v);
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = __fadd_rn(v[i], x0[i]);
      float* xw = p.xo + (size_t)row * k + col;
      *reinterpret_cast<float4*>(xw) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(xw + 4) = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      float u[8];
      qg_split_sum8x2<(B > 1 ? B / 2 : 1)>(p.g, (size_t)row * p.g.ld + col, (long long)((size_t)row * p.g.ld + k + col), v, u);
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fdiv_rn(v[i], __fadd_rn(1.0f, expf(-v[i]))), u[i]);
    }
    if (norm) {
      float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3] + v[4] * v[4] + v[5] * v[5] + v[6] * v[6] +
                 v[7] * v[7];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) part[j] = ss;
      if (KEEP && j == warp) {
#pragma unroll
        for (int i = 0; i < 8; i++) keep[i] = v[i];
      }
    } else if (tbase) {
      qg_act_block(v, lane, j, r, tbase);
    }
  }
  if (!norm) return;
  __syncthreads();
  if (tid == 0) {
    float sum2 = 0.f;
    for (int j = 0; j < nb; j++) sum2 += part[j];
    s_rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum2, (float)k), p.eps));
  }
  __syncthreads();
  const float rms = s_rms;
  for (int j = warp; j < nb; j += nw) {
    const int col = j * QK_K + 8 * lane;
    float v[8], g[8];
    if (KEEP && j == warp) {
#pragma unroll
      for (int i = 0; i < 8; i++) { v[i] = keep[i]; g[i] = g0[i]; }
    } else {
      qg_ld8(xr + col, v);  // ACT_RESID: this thread's own stores above
      qg_ld8(p.gamma + col, g);
    }
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fdiv_rn(v[i], rms), g[i]);
    qg_act_block(v, lane, j, r, tbase);
  }
}

// ---- q|k|v epilogue -------------------------------------------------------
template <int B>
__global__ void k_qkv_post(const QgSplit g, int S, const int* __restrict__ pos, int qn, int kn, int hd,
                           int max_seq, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                           float* __restrict__ q_out, void* kc, void* vc, int kv_f16, int64_t slot_stride,
                           const FaTilesOut tl) {
  pdl_launch();
  pdl_wait();
  const int t = blockIdx.y;
  const int pr = blockIdx.x * blockDim.x + threadIdx.x;  // row pair
  const int rows = g.ld;
  if (t >= S || 2 * pr >= rows) return;
  const int r = 2 * pr;
  const float* w = g.ws + (size_t)t * g.ld + r;
  // rows (q | k | v, multiples of head_dim) and the split stride are even,
  // so each row pair is one aligned float2; a batch's loads in flight together
  float d0 = 0.f, d1 = 0.f;
  for (int sp0 = 0; sp0 < g.splits; sp0 += B) {
    float2 pv[B];
#pragma unroll
    for (int u = 0; u < B; u++)
      if (sp0 + u < g.splits) pv[u] = *reinterpret_cast<const float2*>(w + (size_t)(sp0 + u) * g.stride);
#pragma unroll
    for (int u = 0; u < B; u++)
      if (sp0 + u < g.splits) {
        d0 = sp0 + u == 0 ? pv[u].x : __fadd_rn(d0, pv[u].x);
        d1 = sp0 + u == 0 ? pv[u].y : __fadd_rn(d1, pv[u].y);
      }
  }
  const int p = pos[t], half = hd >> 1;
  if (r < qn + kn) {
    const int rr = r < qn ? r : r - qn;
    const int i2 = (rr % hd) >> 1;
    const float cs = cos_t[(size_t)p * half + i2], sn = sin_t[(size_t)p * half + i2];
    // candle rope_i: (a*c - b*s, a*s + b*c), each op rounded
    const float o0 = __fsub_rn(__fmul_rn(d0, cs), __fmul_rn(d1, sn));
    const float o1 = __fadd_rn(__fmul_rn(d0, sn), __fmul_rn(d1, cs));
    const int dd = rr % hd;
    if (r < qn) {
      if (q_out) *reinterpret_cast<float2*>(q_out + (size_t)t * qn + r) = make_float2(o0, o1);
      if (tl.q)
        *reinterpret_cast<__half2*>(tl.q + ((size_t)(rr / hd) * tl.nqt + t / 128) * tl.tile + fa_qk_off(t & 127, dd)) =
            __floats2half2_rn(o0, o1);
    } else {
      const int kvh = rr / hd;
      store_kv(kc, kv_f16, t * slot_stride + ((int64_t)kvh * max_seq + p) * hd + dd, o0, o1);
      if (tl.k)
        *reinterpret_cast<__half2*>(tl.k + ((size_t)kvh * tl.nkt + p / 128) * tl.tile + fa_qk_off(p & 127, dd)) =
            __floats2half2_rn(o0, o1);
    }
  } else {
    const int rv = r - qn - kn;
    const int kvh = rv / hd, dd = rv % hd;
    store_kv(vc, kv_f16, t * slot_stride + ((int64_t)kvh * max_seq + p) * hd + dd, d0, d1);
    if (tl.v) {
      uint8_t* vt = tl.v + ((size_t)kvh * tl.nkt + p / 128) * tl.tile;
      *reinterpret_cast<__half*>(vt + fa_vt_off(hd, p & 127, dd)) = __float2half_rn(d0);
      *reinterpret_cast<__half*>(vt + fa_vt_off(hd, p & 127, dd + 1)) = __float2half_rn(d1);
    }
  }
}

__global__ void k_resid_add(float* __restrict__ x, const float* __restrict__ g, int S, int n, int ldg) {
  const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (t < S && i < n) x[(size_t)t * n + i] = __fadd_rn(g[(size_t)t * ldg + i], x[(size_t)t * n + i]);
}

// out[t][j] = sum over splits of ws (split order), then the job's consumer.
__global__ void k_qg_finish(const float* __restrict__ ws, int splits, size_t split_stride, int m, int ncols, int ldw,
                            int mode, float* __restrict__ dst, int ldd) {
  pdl_launch();
  pdl_wait();
  const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= m || i >= ncols) return;
  const float* w = ws + (size_t)t * ldw + i;
  const bool two = mode != QG_STORE && mode != QG_RESID;
  float a = 0.f, u = 0.f;
  for (int sp0 = 0; sp0 < splits; sp0 += 8) {  // a batch's loads in flight together
    float pa[8], pu[8];
#pragma unroll
    for (int k = 0; k < 8; k++)
      if (sp0 + k < splits) {
        pa[k] = w[(size_t)(sp0 + k) * split_stride];
        if (two) pu[k] = w[(size_t)(sp0 + k) * split_stride + ncols];
      }
#pragma unroll
    for (int k = 0; k < 8; k++)
      if (sp0 + k < splits) {
        a = sp0 + k == 0 ? pa[k] : __fadd_rn(a, pa[k]);
        if (two) u = sp0 + k == 0 ? pu[k] : __fadd_rn(u, pu[k]);
      }
  }
  float* o = dst + (size_t)t * ldd + i;
  if (mode == QG_STORE) {
    *o = a;
  } else if (mode == QG_RESID) {
    *o = __fadd_rn(a, *o);
  } else {
    *o = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), u);
  }
}

// token[t] = argmax of logits row t (am_better order), pos[t] += 1; the
// winner's value and index also into best_val / best_idx when given. Each
// thread scans a strided slice, 4 loads in flight.
__global__ void __launch_bounds__(1024) k_row_argmax(const float* __restrict__ logits, int n, int ld, uint32_t* token,
                                                     int* pos, float* best_val, int* best_idx) {
  pdl_launch();
  pdl_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = blockDim.x;
  const float* row = logits + (size_t)t * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  int i = tid;
  for (; i + 3 * nt < n; i += 4 * nt) {
    const float v0 = __ldg(row + i), v1 = __ldg(row + i + nt), v2 = __ldg(row + i + 2 * nt),
                v3 = __ldg(row + i + 3 * nt);
    if (am_better(v0, i, bv, bi)) { bv = v0; bi = i; }
    if (am_better(v1, i + nt, bv, bi)) { bv = v1; bi = i + nt; }
    if (am_better(v2, i + 2 * nt, bv, bi)) { bv = v2; bi = i + 2 * nt; }
    if (am_better(v3, i + 3 * nt, bv, bi)) { bv = v3; bi = i + 3 * nt; }
  }
  for (; i < n; i += nt) {
    const float v = __ldg(row + i);
    if (am_better(v, i, bv, bi)) { bv = v; bi = i; }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < (nt >> 5); w++)
      if (am_better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
    token[t] = (uint32_t)(bi == 0x7fffffff ? 0 : bi);
    pos[t] += 1;
    if (best_val) {
      best_val[t] = bv;
      best_idx[t] = bi;
    }
  }
}

// ---- launchers --------------------------------------------------------------
// Row counts up to this take the row kernels' many-loads-per-round-trip
// variants (a decode batch); longer inputs the lighter ones (prompts).
constexpr int QG_FEW_ROWS = 64;

int qkv_post_launch(const QgSplit& g, int S, const int* pos, int qn, int kn, int hd, int max_seq,
                    const float* cos_t, const float* sin_t, float* q_out, void* kc, void* vc, int kv_f16,
                    int64_t kv_seq_stride, int seq_step, cudaStream_t s, bool pdl, const FaTilesOut* tiles) {
  if (S <= 0) return ARMAI_OK;
  FaTilesOut tl{};
  if (tiles) tl = *tiles;
  const dim3 grid((unsigned)((g.ld / 2 + 127) / 128), (unsigned)S);
  ARMAI_CUDA(qg_launch(S <= QG_FEW_ROWS ? k_qkv_post<8> : k_qkv_post<2>, grid, dim3(128), 0, s, pdl, g, S, pos, qn,
                       kn, hd, max_seq, cos_t, sin_t,
                       q_out, kc, vc, kv_f16, (int64_t)(kv_seq_stride * seq_step), tl));
  return ARMAI_OK;
}

// One warp per 256-value block of a row (8 .. 16 warps; longer rows give a
// warp several blocks).
static unsigned row_threads(int k) { return 32u * (unsigned)std::min(16, std::max(8, k / QK_K)); }

int resid_act_launch(const QgSplit& g, float* x, int S, int n, const float* gamma, float eps, uint8_t* a_tiles,
                     cudaStream_t s, bool pdl) {
  if (n % QK_K || n / QK_K > 64) return fail(ARMAI_E_INVALID, "resid_act: n must be a multiple of 256, at most 16384");
  if (S <= 0) return ARMAI_OK;
  RowAct p{};
  p.xo = x;
  p.gamma = gamma;
  p.eps = eps;
  p.k = n;
  p.g = g;
  p.a_tiles = a_tiles;
  ARMAI_CUDA(qg_launch(S <= QG_FEW_ROWS ? k_row_act<ACT_RESID, 8> : k_row_act<ACT_RESID, 2>, dim3(S),
                       dim3(row_threads(n)), 0, s, pdl, p));
  return ARMAI_OK;
}

int silu_act_launch(const QgSplit& g, int S, int F, uint8_t* a_tiles, cudaStream_t s, bool pdl) {
  if (F % QK_K || F / QK_K > 64) return fail(ARMAI_E_INVALID, "silu_act: F must be a multiple of 256, at most 16384");
  if (S <= 0) return ARMAI_OK;
  RowAct p{};
  p.k = F;
  p.g = g;
  p.a_tiles = a_tiles;
  const int nb = F / QK_K, per = std::min(nb, 8);  // 8 blocks per CTA: no norm, so rows split freely
  ARMAI_CUDA(qg_launch(S <= QG_FEW_ROWS ? k_row_act<ACT_SILU, 8> : k_row_act<ACT_SILU, 2>, dim3(S, (unsigned)((nb + per - 1) / per)), dim3(32u * per), 0, s, pdl,
                       p));
  return ARMAI_OK;
}

int resid_add_launch(float* x, const float* g, int S, int n, int ldg, cudaStream_t s) {
  k_resid_add<<<dim3((unsigned)((n + 255) / 256), (unsigned)S), 256, 0, s>>>(x, g, S, n, ldg);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

int row_argmax_launch(const float* logits, int S, int n, int ld, uint32_t* token, int* pos, cudaStream_t s, bool pdl,
                      float* best_val, int* best_idx) {
  if (S <= 0) return ARMAI_OK;
  ARMAI_CUDA(qg_launch(k_row_argmax, dim3(S), dim3(1024), 0, s, pdl, logits, n, ld, token, pos, best_val, best_idx));
  return ARMAI_OK;
}

int qgemm_act_launch(const float* x, const float* gamma, float eps, int m, int k, uint8_t* a_tiles,
                     cudaStream_t s, bool pdl) {
  if (k % QK_K || k / QK_K > 64) return fail(ARMAI_E_INVALID, "qgemm: K must be a multiple of 256, at most 16384");
  if (m <= 0) return ARMAI_OK;
  RowAct p{};
  p.x = x;
  p.gamma = gamma;
  p.eps = eps;
  p.k = k;
  p.a_tiles = a_tiles;
  ARMAI_CUDA(qg_launch(m <= QG_FEW_ROWS ? k_row_act<ACT_X, 8> : k_row_act<ACT_X, 2>, dim3(m), dim3(row_threads(k)), 0, s, pdl, p));
  return ARMAI_OK;
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 qg_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// The tensor map of one weight segment, built once per (address, shape,
// type): weights do not move while a model is loaded, so the maps are reused
// by every later launch (and by captured graphs, which hold them by value).
int qg_weight_map(const QgSeg& sg, CUtensorMap* out) {
  struct Key {
    const void* w;
    int type, rows, row_bytes;
    bool operator==(const Key& o) const {
      return w == o.w && type == o.type && rows == o.rows && row_bytes == o.row_bytes;
    }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.w) ^ ((size_t)k.rows << 20) ^ ((size_t)k.row_bytes << 40) ^ (size_t)k.type;
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> cache;
  const Key key{sg.w, sg.type, sg.rows, sg.row_bytes};
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return ARMAI_OK;
  }
  auto enc = qg_encoder();
  if (!enc) return fail(ARMAI_E_CUDA, "qgemm: cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {(cuuint64_t)sg.row_bytes, (cuuint64_t)sg.rows};
  const cuuint64_t strides[1] = {(cuuint64_t)sg.row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)(sg.type == GGML_Q4_K ? Q4K_BLOCK_BYTES : Q6K_BODY_BYTES), 32u};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(sg.w), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ARMAI_E_CUDA, "qgemm: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  cache.emplace(key, m);
  *out = m;
  return ARMAI_OK;
}

}  // namespace

int qgemm_run(const QgJob& j, cudaStream_t s, QgSplit* split) {
  static thread_local int attr_dev = -1;
  static thread_local int n_sms = 148;
  int dev = 0;
  ARMAI_CUDA(cudaGetDevice(&dev));
  if (attr_dev != dev) {
    ARMAI_CUDA(cudaFuncSetAttribute(k_qgemm<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)qg_smem_bytes(QG_TOK_MAX)));
    ARMAI_CUDA(cudaFuncSetAttribute(k_qgemm<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)qg_smem_bytes(QG_TOK_MAX)));
    ARMAI_CUDA(cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, dev));
    attr_dev = dev;
  }
  if (j.k <= 0 || j.k % QK_K || j.k > 16384)
    return fail(ARMAI_E_INVALID, "qgemm: K must be a multiple of 256, at most 16384");
  if (j.nseg < 1 || j.nseg > 3) return fail(ARMAI_E_INVALID, "qgemm: 1 to 3 weight segments");
  if (j.mode == QG_SILU && (j.nseg != 2 || j.seg[0].rows != j.seg[1].rows))
    return fail(ARMAI_E_INVALID, "qgemm: SiLU jobs take gate and up segments of equal rows");
  if ((j.mode == QG_PARTIAL) != (split != nullptr))
    return fail(ARMAI_E_INVALID, "qgemm: a QgSplit goes with QG_PARTIAL jobs");
  QgParams p;
  std::memset(&p, 0, sizeof p);
  QgMaps maps;
  std::memset(&maps, 0, sizeof maps);
  for (int i = 0; i < j.nseg; i++) {
    const QgSeg& sg = j.seg[i];
    if (sg.type != GGML_Q4_K && sg.type != GGML_Q6_K)
      return fail(ARMAI_E_INVALID, "qgemm: Q4_K / Q6_K matrices only");
    // every segment but the last starts a 32-row group of its own
    if ((i + 1 < j.nseg && sg.rows % 32) || sg.row_bytes % 16 || (reinterpret_cast<uintptr_t>(sg.w) & 15))
      return fail(ARMAI_E_INVALID,
                  "qgemm: segments before the last need rows in multiples of 32; rows 16-byte aligned");
    ARMAI_TRY(qg_weight_map(sg, &maps.m[i]));
    p.seg[i] = sg;
    p.n += sg.rows;
  }
  if (j.m <= 0 || p.n == 0) return ARMAI_OK;
  p.a_tiles = j.a_tiles;
  p.m = j.m;
  p.k = j.k;
  p.nseg = j.nseg;
  p.err = j.err;
  p.ntok = j.m <= 128 ? ((j.m + 15) / 16) * 16 : QG_TOK_MAX;
  p.acc_cols = std::max(32, p.ntok);
  p.tmem_cols = 32;
  while (p.tmem_cols < p.acc_cols + 32 * QG_STAGES) p.tmem_cols <<= 1;
  const uint32_t smem = qg_smem_bytes(p.ntok);
  // few tokens: 8 dequantising warps, two CTAs per SM hide each other's
  // latency; wide token tiles: 16 warps, one CTA per SM (shared memory)
  const bool wide = p.ntok > 64;
  auto kern = wide ? k_qgemm<16> : k_qgemm<8>;
  const int threads = 32 * (3 + (wide ? 16 : 8));
  int occ = 1;
  ARMAI_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem));
  occ = std::max(1, std::min(occ, 512 / p.tmem_cols));
  const int tiles_n = (p.n + QG_W - 1) / QG_W, tiles_t = (j.m + p.ntok - 1) / p.ntok;
  const int ctas = tiles_n * tiles_t, slots = n_sms * occ, nb = j.k / QK_K;
  // K split: fewest (waves x (super-blocks per CTA + 1 for the CTA's fill
  // and drain)), within the workspace
  const size_t part = (size_t)j.m * p.n;
  int splits = 1;
  long best = -1;
  for (int sp = 1; sp <= std::min(nb, 32); sp++) {
    const int per = (nb + sp - 1) / sp, real = (nb + per - 1) / per;
    if (real != sp) continue;
    const bool need_ws = sp > 1 || j.mode == QG_SILU || j.mode == QG_PARTIAL;
    if (need_ws && (!j.ws || (size_t)sp * part > j.ws_floats)) continue;
    const long waves = ((long)ctas * sp + slots - 1) / slots;
    const long cost = waves * (per + 1);
    if (best < 0 || cost < best) { best = cost; splits = sp; }
  }
  if (best < 0) return fail(ARMAI_E_INVALID, "qgemm: workspace too small for this job");
  p.kb_split = (nb + splits - 1) / splits;
  const bool direct = splits == 1 && (j.mode == QG_STORE || j.mode == QG_RESID);
  if (direct) {
    p.out = j.dst;
    p.ldo = j.ldd;
    p.add = j.mode == QG_RESID;
  } else {
    p.out = j.ws;
    p.ldo = p.n;
    p.split_stride = part;
  }
  const dim3 grid((unsigned)tiles_n, (unsigned)tiles_t, (unsigned)splits);
  ARMAI_CUDA(qg_launch(kern, grid, dim3(threads), smem, s, j.pdl != 0, maps, p));
  if (split) {
    *split = QgSplit{j.ws, splits, part, p.n};
  } else if (!direct) {
    const int ncols = j.mode == QG_SILU ? p.n / 2 : p.n;
    ARMAI_CUDA(qg_launch(k_qg_finish, dim3((unsigned)((ncols + 255) / 256), (unsigned)j.m), dim3(256), 0, s,
                         j.pdl != 0, (const float*)j.ws, splits, part, j.m, ncols, p.n, j.mode, j.dst, j.ldd));
  }
  return ARMAI_OK;
}

}  // namespace armai
