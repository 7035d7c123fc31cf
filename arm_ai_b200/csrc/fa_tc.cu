// fa_tc.cu — tensor-core attention (interface and design notes in fa_tc.cuh).
#include "fa_tc.cuh"

#include "llama_kernels.cuh"
#include "tcgen05.cuh"

namespace armai {

constexpr int FA_Q = 128;       // queries per CTA (tensor-memory lanes, MMA M)
constexpr int FA_KT = 128;      // keys per tile (MMA N of Q K^T, K of P V)
// warps 0-7: softmax (warp w: query rows 32 (w % 4) .. + 31, key half w / 4);
// warp 8: one thread streams the operand tiles and issues the MMAs
constexpr int FA_SOFTMAX_THREADS = 256;
constexpr int FA_THREADS = FA_SOFTMAX_THREADS + 32;
// Two S buffers (columns 0-127 and 128-255; key half h of buffer b at
// 128b + 64h; P of key half h over the first 32 of those, S values its own
// warp has read) and the output in 256 .. 256 + hd: the whole tensor memory,
// so one CTA per SM.
constexpr uint32_t FA_TMEM_COLS = 512;

template <int HD>
struct FaLayout {
  static constexpr uint32_t QB = HD * 256u;  // Q: HD / 64 K-blocks x 128 rows x 128 B
  static constexpr uint32_t KB = HD * 256u;  // K tile: same, rows = keys
  static constexpr uint32_t VB = HD * 256u;  // V^T tile: 2 K-blocks of 64 keys x HD rows x 128 B
  static constexpr uint32_t XCH = QB + 2 * KB + 2 * VB;  // f32 [2 parity][2 half][128] maxima, [2][128] sums
  static constexpr uint32_t BAR = XCH + 6 * 128 * 4;
  // at least half the shared memory, so that a second CTA (which could not
  // get tensor memory) is never placed on the SM
  static constexpr uint32_t SMEM = (1024 + BAR + 256) > 116u * 1024 ? (1024 + BAR + 256) : 116u * 1024;
};

// 8 consecutive values as 4 f16 pairs.
__device__ __forceinline__ void fa_ld8h(const float* p, uint32_t (&h)[4]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  const __half2 r[4] = {__floats2half2_rn(a.x, a.y), __floats2half2_rn(a.z, a.w), __floats2half2_rn(b.x, b.y),
                        __floats2half2_rn(b.z, b.w)};
#pragma unroll
  for (int i = 0; i < 4; i++) h[i] = *reinterpret_cast<const uint32_t*>(&r[i]);
}
__device__ __forceinline__ void fa_ld8h(const __half* p, uint32_t (&h)[4]) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  h[0] = a.x; h[1] = a.y; h[2] = a.z; h[3] = a.w;
}

// 2^x by the special-function unit's approximation (ex2.approx, relative
// error about 2^-22; results below the normal range flush to 0): the
// probabilities are rounded to f16 next, and a flushed one is 0 in f16 too.
__device__ __forceinline__ float fa_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 16-byte chunk c of row r of a K-major, 128-byte-swizzled block.
__device__ __forceinline__ void fa_st16(uint8_t* blk, int r, int c, const uint32_t (&h)[4]) {
  *reinterpret_cast<uint4*>(blk + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
}

template <int HD>
__global__ void __launch_bounds__(FA_THREADS, 1) k_fa_tc(const FaParams p) {
  using L = FaLayout<HD>;
  extern __shared__ uint8_t fa_raw[];
  const uint32_t raw_addr = smem_u32(fa_raw);
  uint8_t* smem = fa_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* qs = smem;
  uint8_t* ks = smem + L::QB;       // 2 buffers
  uint8_t* vs = ks + 2 * L::KB;     // 2 buffers
  float* xmax = reinterpret_cast<float*>(smem + L::XCH);  // [parity][half][row]
  float* xsum = xmax + 4 * 128;                             // [half][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint64_t* qfull = bars;
  uint64_t* kfull = bars + 1;       // [2] bulk copies of K tiles
  uint64_t* kempty = bars + 3;      // [2] S MMA that read the K tile completed
  uint64_t* vfull = bars + 5;       // [2]
  uint64_t* vempty = bars + 7;      // [2] P V MMA that read the V^T tile completed
  uint64_t* sfull = bars + 9;       // [2] S of a tile in its buffer
  uint64_t* pready = bars + 11;     // softmax warps: P and the rescaled output in place
  uint64_t* pvdone = bars + 12;     // P V of a tile completed
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 13);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // the longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z, kvh = h / p.group, n_kv = p.n_head / p.group;
  const int q0 = qt * FA_Q;
  const int qlast = min(p.sq, q0 + FA_Q) - 1;
  const int kend = p.causal ? min(p.sk, qlast + 1) : p.sk;
  const int ntiles = (kend + FA_KT - 1) / FA_KT;

  if (tid == 0) {
    mbar_init(qfull, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(&kfull[i], 1);
      mbar_init(&kempty[i], 1);
      mbar_init(&vfull[i], 1);
      mbar_init(&vempty[i], 1);
      mbar_init(&sfull[i], 1);
    }
    mbar_init(pready, FA_SOFTMAX_THREADS / 32);
    mbar_init(pvdone, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, FA_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tslot;
  const uint32_t tO = taddr + 256;
  pdl_launch();
  pdl_wait();  // the operand tiles come from the previous kernel; the output may be read by it

  if (warp == FA_SOFTMAX_THREADS / 32) {
    // ---- issuer: operand tiles by bulk copy, S = Q K^T and O += P V ----
    if (lane == 0) {
      const uint64_t keep = l2_evict_last_policy();  // K / V tiles serve every query tile of the group
      const uint32_t idesc_s = (1u << 4) | ((uint32_t)(FA_KT >> 3) << 17) | ((uint32_t)(FA_Q >> 4) << 24);
      const uint32_t idesc_pv = (1u << 4) | ((uint32_t)(HD >> 3) << 17) | ((uint32_t)(FA_Q >> 4) << 24);
      const size_t kv0 = (size_t)(b * n_kv + kvh) * p.nkt;
      auto load_k = [&](int j) {
        const int bf = j & 1;
        if (j >= 2) qg_wait(&kempty[bf], (uint32_t)(((j >> 1) - 1) & 1), p.err);
        mbar_arrive_tx(&kfull[bf], L::KB);
        bulk_g2s(ks + bf * L::KB, p.kt + (kv0 + j) * L::KB, L::KB, &kfull[bf], keep);
      };
      auto load_v = [&](int j) {
        const int bf = j & 1;
        if (j >= 2) qg_wait(&vempty[bf], (uint32_t)(((j >> 1) - 1) & 1), p.err);
        mbar_arrive_tx(&vfull[bf], L::VB);
        bulk_g2s(vs + bf * L::VB, p.vt + (kv0 + j) * L::VB, L::VB, &vfull[bf], keep);
      };
      auto issue_s = [&](int j) {
        const int bf = j & 1;
        qg_wait(&kfull[bf], (uint32_t)((j >> 1) & 1), p.err);
        tc_fence_after();
        const uint32_t qa = smem_u32(qs), ka = smem_u32(ks + bf * L::KB);
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
          const uint32_t off = (uint32_t)(kk >> 2) * (128u * 128u) + 32u * (uint32_t)(kk & 3);
          tc_mma_ss(taddr + 128u * (uint32_t)bf, qg_smem_desc(qa + off), qg_smem_desc(ka + off), idesc_s, kk > 0);
        }
        qg_commit(&sfull[bf]);
        qg_commit(&kempty[bf]);
      };
      mbar_arrive_tx(qfull, L::QB);
      bulk_g2s(qs, p.qt + ((size_t)(b * p.n_head + h) * p.nqt + qt) * L::QB, L::QB, qfull, keep);
      for (int j = 0; j < min(ntiles, 2); j++) {
        load_k(j);
        load_v(j);
      }
      qg_wait(qfull, 0, p.err);
      if (ntiles > 0) issue_s(0);
      for (int j = 0; j < ntiles; j++) {
        if (j + 1 < ntiles) {
          // the next tile's scores run while the softmax warps work on this
          // one; its buffer held P of tile j - 1, which P V j - 1 has read
          if (j >= 1) qg_wait(pvdone, (uint32_t)((j - 1) & 1), p.err);
          issue_s(j + 1);
        }
        if (j + 2 < ntiles) load_k(j + 2);  // after S j (committed earlier) released the buffer
        qg_wait(pready, (uint32_t)(j & 1), p.err);
        qg_wait(&vfull[j & 1], (uint32_t)((j >> 1) & 1), p.err);
        tc_fence_after();
        const uint32_t va = smem_u32(vs + (j & 1) * L::VB), pa0 = taddr + 128u * (uint32_t)(j & 1);
#pragma unroll
        for (int kk = 0; kk < FA_KT / 16; kk++) {
          const uint32_t off = (uint32_t)(kk >> 2) * (uint32_t)(HD * 128) + 32u * (uint32_t)(kk & 3);
          const uint32_t pa = pa0 + 64u * (uint32_t)(kk >> 2) + 8u * (uint32_t)(kk & 3);
          qg_mma_ts(tO, pa, qg_smem_desc(va + off), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        qg_commit(pvdone);
        qg_commit(&vempty[j & 1]);
        if (j + 2 < ntiles) load_v(j + 2);
      }
    }
  } else {
    // ---- softmax warps: thread = (query row, key half) ----
    const int qr = warp & 3, hf = warp >> 2;
    const int row = 32 * qr + lane, qi = q0 + row;
    const int klim = p.causal ? min(p.sk, qi + 1) : p.sk;  // keys < klim take part
    const uint32_t lane_base = (uint32_t)(32 * qr) << 16;
    const uint32_t oh = tO + lane_base + (uint32_t)(hf * (HD / 2));
    // exp(scale s - m) as exp2(s * scale * log2(e) - m'): m' is the running
    // max in the same units
    const float sl2 = p.scale * 1.4426950408889634f;
    float m_run = -INFINITY, l_run = 0.f;  // l_run: this half's share of the row sum
    for (int j = 0; j < ntiles; j++) {
      const int k0 = j * FA_KT + 64 * hf;
      const uint32_t sh = taddr + 128u * (uint32_t)(j & 1) + lane_base + 64u * (uint32_t)hf;
      qg_wait_warp(&sfull[j & 1], (uint32_t)((j >> 1) & 1), p.err);
      tc_fence_after();
      // pass 1: the row max over this half's keys, then over both halves
      float mt = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 64; c += 16) {
        float v[16];
        qg_tmem_ld16(sh + (uint32_t)c, v);
#pragma unroll
        for (int e = 0; e < 16; e++)
          if (k0 + c + e < klim) mt = fmaxf(mt, __fmul_rn(v[e], sl2));
      }
      float* xm = xmax + (j & 1) * 256;  // by tile parity: a partner one tile behind still reads the other
      xm[hf * 128 + row] = mt;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      mt = fmaxf(mt, xm[(1 - hf) * 128 + row]);
      const float m_new = fmaxf(m_run, mt);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = m_run == -INFINITY ? 0.f : fa_exp2(m_run - m_use);
      // pass 2: P = exp2(s' - m') as f16 over the S columns this thread has
      // read (P column c of the half holds keys 2c, 2c + 1), and P's row sum
      // in f32 (of the values before their f16 rounding)
      float lsum = 0.f;
#pragma unroll 1
      for (int c = 0; c < 64; c += 16) {
        float v[16];
        qg_tmem_ld16(sh + (uint32_t)c, v);
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float p0 = k0 + c + e < klim ? fa_exp2(__fmul_rn(v[e], sl2) - m_use) : 0.f;
          const float p1 = k0 + c + e + 1 < klim ? fa_exp2(__fmul_rn(v[e + 1], sl2) - m_use) : 0.f;
          const __half2 hp = __floats2half2_rn(p0, p1);
          lsum += p0 + p1;
          pk[e >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
        }
        qg_tmem_st8(sh + (uint32_t)(c >> 1), pk);
      }
      l_run = l_run * alpha + lsum;
      m_run = m_new;
      if (j > 0) {
        // this half of the output row (tiles < j) scaled to the new max,
        // once P V j - 1 has completed
        qg_wait_warp(pvdone, (uint32_t)((j - 1) & 1), p.err);
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < HD / 2; c += 16) {
            float v[16];
            qg_tmem_ld16(oh + (uint32_t)c, v);
            uint32_t r[16];
#pragma unroll
            for (int e = 0; e < 16; e++) r[e] = __float_as_uint(v[e] * alpha);
            qg_tmem_st16(oh + (uint32_t)c, r);
          }
        }
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive1(pready);
    }
    // ---- output: O / l, l the sum of both halves' shares ----
    xsum[hf * 128 + row] = l_run;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float l = l_run + xsum[(1 - hf) * 128 + row];
    if (ntiles > 0) qg_wait_warp(pvdone, (uint32_t)((ntiles - 1) & 1), p.err);
    tc_fence_after();
    float* ob = p.o + b * p.o_bs + (int64_t)qi * p.o_ts + (int64_t)h * p.o_hs + hf * (HD / 2);
#pragma unroll 1
    for (int c = 0; c < HD / 2; c += 16) {
      float v[16];
      qg_tmem_ld16(oh + (uint32_t)c, v);
      if (qi < p.sq) {
#pragma unroll
        for (int e = 0; e < 16; e += 4) {
          const float4 w = l > 0.f ? make_float4(__fdiv_rn(v[e], l), __fdiv_rn(v[e + 1], l),
                                                 __fdiv_rn(v[e + 2], l), __fdiv_rn(v[e + 3], l))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(ob + c + e) = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(taddr, FA_TMEM_COLS);
  }
}

// One CTA per (tile, head, batch): 128 rows of one head into its tile.
template <typename T, int HD, bool TRANSPOSE>
__global__ void __launch_bounds__(256) k_fa_tiles(const T* __restrict__ src, int64_t bs, int64_t ts, int64_t hs,
                                                  int heads, int n_rows, uint8_t* __restrict__ dst) {
  const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z, ntiles = gridDim.x;
  const T* sb = src + b * bs + (int64_t)h * hs;
  uint8_t* out = dst + ((size_t)(b * heads + h) * ntiles + tile) * fa_tile_bytes(HD);
  const int r0 = tile * 128;
  if constexpr (!TRANSPOSE) {
    for (int task = threadIdx.x; task < 128 * (HD / 8); task += blockDim.x) {
      const int r = task / (HD / 8), c = task % (HD / 8);
      uint32_t hv[4] = {0u, 0u, 0u, 0u};
      if (r0 + r < n_rows) fa_ld8h(sb + (int64_t)(r0 + r) * ts + 8 * c, hv);
      fa_st16(out + (c >> 3) * (128 * 128), r, c & 7, hv);
    }
  } else {
  // V^T: the tile's rows staged as f16 [128][HD] (coalesced loads), then
  // 8 keys x 1 dim per 16-byte chunk
  __shared__ __align__(16) __half st[128 * HD];
  for (int task = threadIdx.x; task < 128 * (HD / 8); task += blockDim.x) {
    const int r = task / (HD / 8), c = task % (HD / 8);
    uint32_t hv[4] = {0u, 0u, 0u, 0u};
    if (r0 + r < n_rows) fa_ld8h(sb + (int64_t)(r0 + r) * ts + 8 * c, hv);
    *reinterpret_cast<uint4*>(st + r * HD + 8 * c) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
  }
  __syncthreads();
  for (int task = threadIdx.x; task < HD * 16; task += blockDim.x) {
    const int d = task % HD, g = task / HD;
    uint32_t hv[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const __half2 t2 = __halves2half2(st[(8 * g + 2 * i) * HD + d], st[(8 * g + 2 * i + 1) * HD + d]);
      hv[i] = *reinterpret_cast<const uint32_t*>(&t2);
    }
    fa_st16(out + (g >> 3) * (HD * 128), d, g & 7, hv);
  }
  }
}

int fa_tiles_launch(const void* src, bool f16, int64_t bs, int64_t ts, int64_t hs, int batch, int heads, int n_rows,
                    int hd, bool transpose, uint8_t* dst, cudaStream_t s) {
  if (n_rows <= 0 || batch <= 0 || heads <= 0) return ARMAI_OK;
  const int64_t es = f16 ? 2 : 4;
  if ((reinterpret_cast<uintptr_t>(src) % 16) || (ts * es) % 16 || (hs * es) % 16 || (bs * es) % 16)
    return fail(ARMAI_E_INVALID, "attention: rows must be 16-byte aligned");
  const dim3 grid((unsigned)((n_rows + 127) / 128), (unsigned)heads, (unsigned)batch);
#define FA_TILES(T, HDV)                                                                                        \
  (transpose ? (k_fa_tiles<T, HDV, true><<<grid, 256, 0, s>>>((const T*)src, bs, ts, hs, heads, n_rows, dst))  \
             : (k_fa_tiles<T, HDV, false><<<grid, 256, 0, s>>>((const T*)src, bs, ts, hs, heads, n_rows, dst)))
  if (hd == 64) {
    if (f16) FA_TILES(__half, 64); else FA_TILES(float, 64);
  } else if (hd == 128) {
    if (f16) FA_TILES(__half, 128); else FA_TILES(float, 128);
  } else {
    return fail(ARMAI_E_INVALID, "attention: tensor-core path needs head dim 64 or 128");
  }
#undef FA_TILES
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

namespace {
template <int HD>
int fa_launch_t(const FaParams& p, int batch, cudaStream_t s, bool pdl) {
  static thread_local int attr_dev = -1;
  int dev = 0;
  ARMAI_CUDA(cudaGetDevice(&dev));
  if (attr_dev != dev) {
    ARMAI_CUDA(cudaFuncSetAttribute(k_fa_tc<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)FaLayout<HD>::SMEM));
    attr_dev = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((p.sq + FA_Q - 1) / FA_Q), (unsigned)p.n_head, (unsigned)batch);
  cfg.blockDim = dim3(FA_THREADS);
  cfg.dynamicSmemBytes = FaLayout<HD>::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  ARMAI_CUDA(cudaLaunchKernelEx(&cfg, k_fa_tc<HD>, p));
  return ARMAI_OK;
}
}  // namespace

// Error word of launches given no flag of their own (lives as long as the
// module; the primitive entry points use it).
static __device__ uint32_t g_fa_err;

int fa_tc_launch(const FaParams& p_in, int hd, int batch, cudaStream_t s, bool pdl) {
  FaParams p = p_in;
  if (p.sq <= 0 || p.sk <= 0 || batch <= 0 || p.n_head <= 0) return ARMAI_OK;
  if (p.group <= 0 || p.n_head % p.group) return fail(ARMAI_E_INVALID, "attention: heads must split into groups");
  if (!p.qt || !p.kt || !p.vt) return fail(ARMAI_E_INVALID, "attention: operand tiles missing");
  if ((reinterpret_cast<uintptr_t>(p.qt) | reinterpret_cast<uintptr_t>(p.kt) | reinterpret_cast<uintptr_t>(p.vt)) % 16 ||
      reinterpret_cast<uintptr_t>(p.o) % 16 || (p.o_ts * 4) % 16 || (p.o_hs * 4) % 16 || (p.o_bs * 4) % 16)
    return fail(ARMAI_E_INVALID, "attention: tiles and output rows must be 16-byte aligned");
  if (!p.err) ARMAI_CUDA(cudaGetSymbolAddress((void**)&p.err, g_fa_err));
  if (hd == 64) return fa_launch_t<64>(p, batch, s, pdl);
  if (hd == 128) return fa_launch_t<128>(p, batch, s, pdl);
  return fail(ARMAI_E_INVALID, "attention: tensor-core path needs head dim 64 or 128");
}

}  // namespace armai
