// fa_tc.cu — tensor-core attention (interface and design notes in fa_tc.cuh).
#include "fa_tc.cuh"

#include "llama_kernels.cuh"
#include "tcgen05.cuh"

namespace armai {

constexpr int FA_Q = 128;       // queries per CTA (tensor-memory lanes, MMA M)
constexpr int FA_KT = 128;      // keys per tile (MMA N of Q K^T, K of P V)
// warps 0-7: softmax (warp w: query rows 32 (w % 4) .. + 31, key half w / 4);
// warps 8-11: loaders
constexpr int FA_THREADS = 384;
constexpr int FA_SOFTMAX_THREADS = 256;
// S in columns 0-127 (key half h: 64h .. 64h + 63), P of key half h in
// columns 64h .. 64h + 31 (over S values its own warp has read), the output
// in 128 .. 128 + hd
constexpr uint32_t FA_TMEM_COLS = 256;

template <int HD>
struct FaLayout {
  static constexpr uint32_t QB = HD * 256u;  // Q: HD / 64 K-blocks x 128 rows x 128 B
  static constexpr uint32_t KB = HD * 256u;  // K tile: same, rows = keys
  static constexpr uint32_t VB = HD * 256u;  // V^T tile: 2 K-blocks of 64 keys x HD rows x 128 B
  static constexpr uint32_t XCH = QB + 2 * KB + 2 * VB;       // [2][128] f32: row max / sum exchange
  static constexpr uint32_t BAR = XCH + 2 * 128 * 4;
  static constexpr uint32_t SMEM = 1024 + BAR + 128;
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
__device__ __forceinline__ float fa_ldf(const float* p) { return *p; }
__device__ __forceinline__ float fa_ldf(const __half* p) { return __half2float(*p); }

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

template <typename TQ, typename TKV, int HD>
__global__ void __launch_bounds__(FA_THREADS, HD == 64 ? 2 : 1) k_fa_tc(const FaParams p) {
  using L = FaLayout<HD>;
  extern __shared__ uint8_t fa_raw[];
  const uint32_t raw_addr = smem_u32(fa_raw);
  uint8_t* smem = fa_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* qs = smem;
  uint8_t* ks = smem + L::QB;       // 2 buffers
  uint8_t* vs = ks + 2 * L::KB;     // 2 buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint64_t* qfull = bars;
  uint64_t* kvfull = bars + 1;      // [2]
  uint64_t* kvempty = bars + 3;     // [2]
  uint64_t* sbar = bars + 5;
  uint64_t* pvbar = bars + 6;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 7);
  float* xch = reinterpret_cast<float*>(smem + L::XCH);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // the longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z, kvh = h / p.group;
  const int q0 = qt * FA_Q;
  const int qlast = min(p.sq, q0 + FA_Q) - 1;
  const int kend = p.causal ? min(p.sk, qlast + 1) : p.sk;
  const int ntiles = (kend + FA_KT - 1) / FA_KT;

  const bool tiled = p.qt != nullptr;
  if (tid == 0) {
    mbar_init(qfull, tiled ? 1 : 4);
    for (int i = 0; i < 2; i++) {
      mbar_init(&kvfull[i], tiled ? 1 : 4);   // the bulk copies, or one arrival per loader warp
      mbar_init(&kvempty[i], 1);  // tcgen05.commit after the tile's P V
    }
    mbar_init(sbar, 1);
    mbar_init(pvbar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, FA_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tslot;
  pdl_launch();
  pdl_wait();  // q / k / v come from the previous kernel; the output may be read by it

  if (warp >= 8 && tiled) {
    // ---- tiles already in the staged layout: one bulk copy each ----
    if (tid == FA_SOFTMAX_THREADS) {
      const uint64_t keep = l2_evict_last_policy();  // K / V tiles serve every query tile of the group
      const int n_kv = p.n_head / p.group;
      mbar_arrive_tx(qfull, L::QB);
      bulk_g2s(qs, p.qt + ((size_t)(b * p.n_head + h) * p.nqt + qt) * L::QB, L::QB, qfull, keep);
      for (int j = 0; j < ntiles; j++) {
        const int buf = j & 1;
        if (j >= 2) qg_wait(&kvempty[buf], (uint32_t)(((j >> 1) - 1) & 1), p.err);
        mbar_arrive_tx(&kvfull[buf], L::KB + L::VB);
        const size_t kv_tile = (size_t)(b * n_kv + kvh) * p.nkt + j;
        bulk_g2s(ks + buf * L::KB, p.kt + kv_tile * L::KB, L::KB, &kvfull[buf], keep);
        bulk_g2s(vs + buf * L::VB, p.vt + kv_tile * L::VB, L::VB, &kvfull[buf], keep);
      }
    }
  } else if (warp >= 8) {
    // ---- loaders: f16, K-major, swizzled ----
    const int lt = tid - FA_SOFTMAX_THREADS;
    const TQ* qb = reinterpret_cast<const TQ*>(p.q) + b * p.q_bs + (int64_t)h * p.q_hs;
#pragma unroll
    for (int u0 = 0; u0 < HD / 8; u0 += 4) {  // 128 loader threads, HD / 8 Q chunks each
      uint32_t hv[4][4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int task = lt + 128 * (u0 + u);
        const int row = task / (HD / 8), ch = task % (HD / 8), t = q0 + row;
        hv[u][0] = hv[u][1] = hv[u][2] = hv[u][3] = 0u;
        if (t < p.sq) fa_ld8h(qb + (int64_t)t * p.q_ts + ch * 8, hv[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int task = lt + 128 * (u0 + u);
        const int row = task / (HD / 8), ch = task % (HD / 8);
        fa_st16(qs + (ch >> 3) * (128 * 128), row, ch & 7, hv[u]);
      }
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive1(qfull);
    const TKV* kb = reinterpret_cast<const TKV*>(p.k) + b * p.kv_bs + (int64_t)kvh * p.kv_hs;
    const TKV* vb = reinterpret_cast<const TKV*>(p.v) + b * p.kv_bs + (int64_t)kvh * p.kv_hs;
    for (int j = 0; j < ntiles; j++) {
      const int buf = j & 1, k0 = j * FA_KT;
      if (j >= 2) qg_wait_warp(&kvempty[buf], (uint32_t)(((j >> 1) - 1) & 1), p.err);
      uint8_t* kt = ks + buf * L::KB;
      // each loader thread: HD / 8 K chunks and HD / 8 V^T chunks, loaded in
      // batches of 4 so that many loads are in flight
      constexpr int TASKS = HD / 8;
#pragma unroll
      for (int u0 = 0; u0 < TASKS; u0 += 4) {
        uint32_t hv[4][4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int task = lt + 128 * (u0 + u);
          const int row = task / (HD / 8), ch = task % (HD / 8), key = k0 + row;
          hv[u][0] = hv[u][1] = hv[u][2] = hv[u][3] = 0u;
          if (key < p.sk) fa_ld8h(kb + (int64_t)key * p.kv_ts + ch * 8, hv[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int task = lt + 128 * (u0 + u);
          const int row = task / (HD / 8), ch = task % (HD / 8);
          fa_st16(kt + (ch >> 3) * (128 * 128), row, ch & 7, hv[u]);
        }
      }
      // V^T: row d holds keys k0 .. k0 + 127 (two 64-key K-blocks); a warp's
      // lanes take consecutive d, so each of the 8 key loads is coalesced
      uint8_t* vt = vs + buf * L::VB;
#pragma unroll
      for (int u0 = 0; u0 < TASKS; u0 += 4) {
        float f[4][8];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int task = lt + 128 * (u0 + u);
          const int d = task % HD, g = task / HD;
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const int key = k0 + 8 * g + i;
            f[u][i] = key < p.sk ? fa_ldf(vb + (int64_t)key * p.kv_ts + d) : 0.f;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int task = lt + 128 * (u0 + u);
          const int d = task % HD, g = task / HD;
          uint32_t hv[4];
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const __half2 t2 = __floats2half2_rn(f[u][2 * i], f[u][2 * i + 1]);
            hv[i] = *reinterpret_cast<const uint32_t*>(&t2);
          }
          fa_st16(vt + (g >> 3) * (HD * 128), d, g & 7, hv);
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive1(&kvfull[buf]);
    }
  } else {
    // ---- softmax warps: thread = (query row, key half) ----
    const int qr = warp & 3, hf = warp >> 2;
    const int row = 32 * qr + lane, qi = q0 + row;
    const int klim = p.causal ? min(p.sk, qi + 1) : p.sk;  // keys < klim take part
    const uint32_t lane_base = (uint32_t)(32 * qr) << 16;
    const uint32_t tS = taddr, tO = taddr + 128;
    const uint32_t sh = tS + lane_base + 64u * (uint32_t)hf;  // this half's S / P columns
    const uint32_t oh = tO + lane_base + (uint32_t)(hf * (HD / 2));
    const uint32_t idesc_s = (1u << 4) | ((uint32_t)(FA_KT >> 3) << 17) | ((uint32_t)(FA_Q >> 4) << 24);
    const uint32_t idesc_pv = (1u << 4) | ((uint32_t)(HD >> 3) << 17) | ((uint32_t)(FA_Q >> 4) << 24);
    // exp(scale s - m) as exp2(s * scale * log2(e) - m'): m' is the running
    // max in the same units
    const float sl2 = p.scale * 1.4426950408889634f;
    float m_run = -INFINITY, l_run = 0.f;  // l_run: this half's share of the row sum
    if (tid == 0) qg_wait(qfull, 0, p.err);
    for (int j = 0; j < ntiles; j++) {
      const int buf = j & 1, k0 = j * FA_KT + 64 * hf;
      if (tid == 0) {
        qg_wait(&kvfull[buf], (uint32_t)((j >> 1) & 1), p.err);
        if (j > 0) qg_wait(pvbar, (uint32_t)((j - 1) & 1), p.err);  // P of tile j - 1 consumed
        tc_fence_after();
        const uint32_t qa = smem_u32(qs), ka = smem_u32(ks + buf * L::KB);
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
          const uint32_t off = (uint32_t)(kk >> 2) * (128u * 128u) + 32u * (uint32_t)(kk & 3);
          tc_mma_ss(tS, qg_smem_desc(qa + off), qg_smem_desc(ka + off), idesc_s, kk > 0);
        }
        qg_commit(sbar);
      }
      qg_wait_warp(sbar, (uint32_t)(j & 1), p.err);
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
      xch[hf * 128 + row] = mt;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      mt = fmaxf(mt, xch[(1 - hf) * 128 + row]);
      const float m_new = fmaxf(m_run, mt);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = m_run == -INFINITY ? 0.f : fa_exp2(m_run - m_use);
      // pass 2: P = exp2(s' - m') as f16 over the S columns this thread has
      // read (P column 64h + c holds keys 64h + 2c, + 1), and P's row sum in
      // f32 (of the values before their f16 rounding)
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
      // this half of the output row (tiles < j) scaled to the new max; tile
      // j - 1's P V has completed (sbar's commit followed it)
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
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
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      asm volatile("bar.sync 1, 256;" ::: "memory");  // every row's P and output are in place
      if (tid == 0) {
        tc_fence_after();
        const uint32_t va = smem_u32(vs + buf * L::VB);
#pragma unroll
        for (int kk = 0; kk < FA_KT / 16; kk++) {
          const uint32_t off = (uint32_t)(kk >> 2) * (uint32_t)(HD * 128) + 32u * (uint32_t)(kk & 3);
          const uint32_t pa = tS + 64u * (uint32_t)(kk >> 2) + 8u * (uint32_t)(kk & 3);
          qg_mma_ts(tO, pa, qg_smem_desc(va + off), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        qg_commit(pvbar);
        qg_commit(&kvempty[buf]);  // the tile's K and V buffers are free again
      }
    }
    // ---- output: O / l, l the sum of both halves' shares ----
    xch[hf * 128 + row] = l_run;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float l = l_run + xch[(1 - hf) * 128 + row];
    if (ntiles > 0) qg_wait_warp(pvbar, (uint32_t)((ntiles - 1) & 1), p.err);
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
template <typename TQ, typename TKV, int HD>
int fa_launch_t(const FaParams& p, int batch, cudaStream_t s, bool pdl) {
  static thread_local int attr_dev = -1;
  int dev = 0;
  ARMAI_CUDA(cudaGetDevice(&dev));
  if (attr_dev != dev) {
    ARMAI_CUDA(cudaFuncSetAttribute(k_fa_tc<TQ, TKV, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
  ARMAI_CUDA(cudaLaunchKernelEx(&cfg, k_fa_tc<TQ, TKV, HD>, p));
  return ARMAI_OK;
}
}  // namespace

// Error word of launches given no flag of their own (lives as long as the
// module; the primitive entry points use it).
static __device__ uint32_t g_fa_err;

int fa_tc_launch(const FaParams& p_in, int hd, int batch, bool q_f16, bool kv_f16, cudaStream_t s, bool pdl) {
  FaParams p = p_in;
  if (p.sq <= 0 || p.sk <= 0 || batch <= 0 || p.n_head <= 0) return ARMAI_OK;
  if (!p.err) ARMAI_CUDA(cudaGetSymbolAddress((void**)&p.err, g_fa_err));
  if (p.group <= 0 || p.n_head % p.group) return fail(ARMAI_E_INVALID, "attention: heads must split into groups");
  // every 8-value row chunk is read with 16-byte (f32: 2 x 16-byte) loads
  const int64_t es_q = q_f16 ? 2 : 4, es_kv = kv_f16 ? 2 : 4;
  const bool al = (reinterpret_cast<uintptr_t>(p.q) % 16 == 0) && (reinterpret_cast<uintptr_t>(p.k) % 16 == 0) &&
                  (p.q_ts * es_q) % 16 == 0 && (p.q_hs * es_q) % 16 == 0 && (p.q_bs * es_q) % 16 == 0 &&
                  (p.kv_ts * es_kv) % 16 == 0 && (p.kv_hs * es_kv) % 16 == 0 && (p.kv_bs * es_kv) % 16 == 0 &&
                  (reinterpret_cast<uintptr_t>(p.o) % 16 == 0) && (p.o_ts * 4) % 16 == 0 &&
                  (p.o_hs * 4) % 16 == 0 && (p.o_bs * 4) % 16 == 0;
  if (!al) return fail(ARMAI_E_INVALID, "attention: q / k / out rows must be 16-byte aligned");
#define FA_CASE(TQ, TKV)                                                               \
  if (hd == 64) return fa_launch_t<TQ, TKV, 64>(p, batch, s, pdl);                   \
  if (hd == 128) return fa_launch_t<TQ, TKV, 128>(p, batch, s, pdl);                 \
  return fail(ARMAI_E_INVALID, "attention: tensor-core path needs head dim 64 or 128");
  if (q_f16 && kv_f16) { FA_CASE(__half, __half) }
  if (!q_f16 && kv_f16) { FA_CASE(float, __half) }
  if (!q_f16 && !kv_f16) { FA_CASE(float, float) }
  return fail(ARMAI_E_INVALID, "attention: f16 queries need f16 keys and values");
#undef FA_CASE
}

}  // namespace armai
