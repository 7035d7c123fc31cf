// prims.cu — the int8 / int4 / rmsnorm / flash-attention primitive NIFs and
// the LLM helpers (rope, softmax, silu(gate) * up, Q6_K dequantisation,
// f16-weight matmul) on sm_100a (reference: native/arm_ai_nif/src/
// shape_ops.rs, x86 scalar paths).
//
// Exactness: every integer result is bit-exact. Where the reference's f32
// arithmetic is a short, fixed-order chain (int8 scale products, the int4
// group sums and their sequential fold over groups, the weight-only int8
// dot), the kernels reproduce that order with non-contracted __f*_rn ops, so
// those f32 outputs are bit-exact too (also the Q6_K dequantisation and the
// f16-weight matmul). rmsnorm (one 4096-long serial sum per row), softmax
// (parallel sum) and flash attention use parallel reductions, rope CUDA's
// cosf / sinf and silu(gate) * up CUDA's expf: those are checked to a
// tolerance.
#include <cuda_fp16.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "fa_tc.cuh"

using namespace armai;

namespace {

// ---------------------------------------------------------------------------
// Per-thread stream + stream-ordered allocations for the host-pointer API.
// ---------------------------------------------------------------------------
struct ThreadStream {
  int dev = -1;
  cudaStream_t s = nullptr;
};
thread_local ThreadStream g_ts;

int thread_stream(cudaStream_t* out) {
  int dev = 0;
  ARMAI_CUDA(cudaGetDevice(&dev));
  if (g_ts.s == nullptr || g_ts.dev != dev) {
    ARMAI_CUDA(cudaStreamCreateWithFlags(&g_ts.s, cudaStreamNonBlocking));
    g_ts.dev = dev;
  }
  *out = g_ts.s;
  return ARMAI_OK;
}

struct Scoped {
  cudaStream_t s;
  void* p = nullptr;
  explicit Scoped(cudaStream_t st) : s(st) {}
  ~Scoped() { if (p) cudaFreeAsync(p, s); }
};

// Stream-ordered allocations come from the library's own memory pool per
// device, which keeps freed memory for the next call (release threshold at
// its maximum): with a threshold of 0, as the default pool has, every call
// after a synchronisation paid for a fresh device allocation.
int lib_pool(cudaMemPool_t* out) {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  int dev = 0;
  ARMAI_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(ARMAI_E_INVALID, "device ordinal beyond 64");
  std::lock_guard<std::mutex> lk(mu);
  if (!pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    ARMAI_CUDA(cudaMemPoolCreate(&pool, &props));
    uint64_t keep = ~0ull;
    ARMAI_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
    pools[dev] = pool;
  }
  *out = pools[dev];
  return ARMAI_OK;
}

int dalloc(Scoped& b, size_t bytes) {
  cudaMemPool_t pool;
  ARMAI_TRY(lib_pool(&pool));
  ARMAI_CUDA(cudaMallocFromPoolAsync(&b.p, bytes ? bytes : 16, pool, b.s));
  return ARMAI_OK;
}
int h2d(Scoped& b, const void* src, size_t bytes) {
  ARMAI_TRY(dalloc(b, bytes));
  if (bytes) ARMAI_CUDA(cudaMemcpyAsync(b.p, src, bytes, cudaMemcpyHostToDevice, b.s));
  return ARMAI_OK;
}

std::string lenmsg(const char* what, size_t got, const char* expr, size_t want) {
  return std::string(what) + " len " + std::to_string(got) + " != " + expr + " = " + std::to_string(want);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_isum(int v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// P1/P2/P4: s8 x s8 -> s32 (dp4a), optional f32 scale epilogue
// (shape_ops.rs:1205: (acc as f32) * act_scale * w_scales[j]).
// CTA: 8 warps x RW weight rows, MT activation rows staged through smem in
// 2048-byte K chunks. Weight rows stream from HBM once per MT tile; two rows
// per warp give 2 x (number of SMs) CTAs on 4096-row matrices, and the K loop
// keeps two 16-byte loads per row in flight.
// ---------------------------------------------------------------------------
constexpr int I8_KC = 2048;
constexpr int I8_RW = 2;  // weight rows per warp

template <int MT>
__global__ void __launch_bounds__(256) k_int8_gemm(const int8_t* __restrict__ a,
                                                   const int8_t* __restrict__ w, int32_t* out_s32,
                                                   float* out_f32, const float* act_scales,
                                                   int per_token, float act_scale,
                                                   const float* w_scales, int m, int n, int k) {
  __shared__ __align__(16) int8_t As[MT][I8_KC];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row0 = blockIdx.x * (8 * I8_RW) + warp * I8_RW;
  const int m0 = blockIdx.y * MT;
  int acc[I8_RW][MT];
#pragma unroll
  for (int r = 0; r < I8_RW; r++)
#pragma unroll
    for (int t = 0; t < MT; t++) acc[r][t] = 0;
  for (int kc = 0; kc < k; kc += I8_KC) {
    const int klen = min(I8_KC, k - kc);
    __syncthreads();
    for (int i = threadIdx.x; i < MT * (I8_KC / 16); i += blockDim.x) {
      const int t = i / (I8_KC / 16), c = (i % (I8_KC / 16)) * 16;
      int4 v = make_int4(0, 0, 0, 0);
      if (m0 + t < m && c < klen) v = *reinterpret_cast<const int4*>(a + (size_t)(m0 + t) * k + kc + c);
      *reinterpret_cast<int4*>(&As[t][c]) = v;
    }
    __syncthreads();
#pragma unroll 2
    for (int c = lane * 16; c < klen; c += 512) {
      int4 wv[I8_RW];
#pragma unroll
      for (int r = 0; r < I8_RW; r++)
        wv[r] = (row0 + r < n) ? __ldg(reinterpret_cast<const int4*>(w + (size_t)(row0 + r) * k + kc + c))
                               : make_int4(0, 0, 0, 0);
#pragma unroll
      for (int t = 0; t < MT; t++) {
        const int4 av = *reinterpret_cast<const int4*>(&As[t][c]);
#pragma unroll
        for (int r = 0; r < I8_RW; r++) {
          int s = acc[r][t];
          s = __dp4a(wv[r].x, av.x, s);
          s = __dp4a(wv[r].y, av.y, s);
          s = __dp4a(wv[r].z, av.z, s);
          s = __dp4a(wv[r].w, av.w, s);
          acc[r][t] = s;
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < I8_RW; r++)
#pragma unroll
    for (int t = 0; t < MT; t++) {
      const int s = warp_isum(acc[r][t]);
      if (lane == 0 && row0 + r < n && m0 + t < m) {
        const size_t o = (size_t)(m0 + t) * n + row0 + r;
        if (out_s32) out_s32[o] = s;
        if (out_f32) {
          const float as = per_token ? act_scales[m0 + t] : act_scale;
          out_f32[o] = __fmul_rn(__fmul_rn((float)s, as), w_scales[row0 + r]);
        }
      }
    }
}

}  // namespace
namespace armai {
int launch_int8_gemm_tc(const int8_t* a, const int8_t* w, int32_t* o32, float* of32, const float* act_scales,
                        int per_token, float act_scale, const float* w_scales, int64_t m, int64_t n, int64_t k,
                        cudaStream_t s);
int int8_gemm_tc_check();
}  // namespace armai
namespace {

// M >= 64 (GEMM-shaped): the tcgen05 kind::i8 kernel (i8gemm_tc.cu); smaller
// M (matrix-vector shaped, bound by streaming W): the dp4a kernels below.
constexpr int64_t I8_TC_MIN_M = 64;

int launch_int8_gemm(const int8_t* a, const int8_t* w, int32_t* o32, float* of32, const float* act_scales,
                     int per_token, float act_scale, const float* w_scales, int64_t m, int64_t n,
                     int64_t k, cudaStream_t s) {
  if (k % 16) {
    // rows are read 16 bytes at a time
    return fail(ARMAI_E_INVALID, "int8_matmul: K must be a multiple of 16 on this path");
  }
  const bool aligned = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w)) & 15) == 0;
  if (m >= I8_TC_MIN_M && aligned && m <= INT32_MAX && n <= INT32_MAX && k <= INT32_MAX)
    return launch_int8_gemm_tc(a, w, o32, of32, act_scales, per_token, act_scale, w_scales, m, n, k, s);
  const unsigned rows_per_cta = 8 * I8_RW;
  if (m <= 4) {
    dim3 g((unsigned)((n + rows_per_cta - 1) / rows_per_cta), (unsigned)m);
    k_int8_gemm<1><<<g, 256, 0, s>>>(a, w, o32, of32, act_scales, per_token, act_scale, w_scales, (int)m, (int)n, (int)k);
  } else {
    dim3 g((unsigned)((n + rows_per_cta - 1) / rows_per_cta), (unsigned)((m + 15) / 16));
    k_int8_gemm<16><<<g, 256, 0, s>>>(a, w, o32, of32, act_scales, per_token, act_scale, w_scales, (int)m, (int)n, (int)k);
  }
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

// ---------------------------------------------------------------------------
// P3: quantize_int8_per_token (shape_ops.rs:1273-1292). One CTA per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_quant_int8_rows(const float* a, int k, int8_t* q, float* scales) {
  __shared__ float red[32];
  const float* row = a + (size_t)blockIdx.x * k;
  float mx = 0.f;
  for (int i = threadIdx.x; i < k; i += blockDim.x) mx = fmaxf(mx, fabsf(row[i]));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float max_abs = red[0];
  const float scale = max_abs > 0.f ? __fdiv_rn(max_abs, 127.0f) : 1.0f;
  if (threadIdx.x == 0) scales[blockIdx.x] = scale;
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const float r = roundf(__fdiv_rn(row[i], scale));
    // `as i32` saturates (NaN -> 0), then clamp(-127, 127)
    int v = (r != r) ? 0 : (int)fmaxf(-2147483648.f, fminf(r, 2147483520.f));
    v = max(-127, min(127, v));
    q[(size_t)blockIdx.x * k + i] = (int8_t)v;
  }
}

// ---------------------------------------------------------------------------
// P5/P6: int4_matmul_f32 (shape_ops.rs:3175-3236). Warp per output (m, n).
// Each lane owns groups g = lane + 32i and runs the reference's 16-step
// chain  gacc += a_lo*lo + a_hi*hi  for them; the products gacc*scale are
// then folded into acc in group order by lane 0 (acc += p_0; acc += p_1; ...).
// SCALE_T: float (the reference ABI) or __half (per-32-group f16 scales).
// ---------------------------------------------------------------------------
template <typename SCALE_T>
__device__ __forceinline__ float load_scale(const SCALE_T* s, size_t i);
template <>
__device__ __forceinline__ float load_scale<float>(const float* s, size_t i) { return s[i]; }
template <>
__device__ __forceinline__ float load_scale<__half>(const __half* s, size_t i) { return __half2float(s[i]); }

__device__ __forceinline__ float fold_in_order(float acc, const float* prod, int ng, int lane) {
  // prod[i] is group lane + 32 i; fold groups 0, 1, 2, ... in order.
  for (int base = 0; base < ng; base += 32) {
    const float mine = prod[base >> 5];
    const int cnt = min(32, ng - base);
    for (int j = 0; j < cnt; j++) {
      const float v = __shfl_sync(0xffffffffu, mine, j);
      acc = __fadd_rn(acc, v);
    }
  }
  return acc;
}

constexpr int MAX_GROUPS_PER_LANE = 16;  // K <= 16384

template <typename SCALE_T>
__global__ void __launch_bounds__(256) k_int4_f32(const float* __restrict__ a, const uint8_t* __restrict__ wp,
                                                  const SCALE_T* __restrict__ ws, float* out, int m, int n, int k) {
  const int lane = threadIdx.x & 31;
  const int ni = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int mi = blockIdx.y;
  if (ni >= n) return;
  const int ng = k / 32;
  const float* ar = a + (size_t)mi * k;
  const uint8_t* wr = wp + (size_t)ni * (k / 2);
  float prod[MAX_GROUPS_PER_LANE];
#pragma unroll
  for (int i = 0; i < MAX_GROUPS_PER_LANE; i++) {
    prod[i] = 0.f;
    const int g = lane + 32 * i;
    if (g < ng) {
      const uint4 pk = *reinterpret_cast<const uint4*>(wr + (size_t)g * 16);
      const uint32_t bw[4] = {pk.x, pk.y, pk.z, pk.w};
      const float4* af = reinterpret_cast<const float4*>(ar + (size_t)g * 32);
      float gacc = 0.f;
#pragma unroll
      for (int q4 = 0; q4 < 8; q4++) {
        const float4 av = af[q4];
        const uint32_t word = bw[q4 >> 1];
        const int sh = (q4 & 1) * 16;
        const uint32_t b0 = (word >> sh) & 0xff, b1 = (word >> (sh + 8)) & 0xff;
        gacc = __fadd_rn(gacc, __fadd_rn(__fmul_rn(av.x, (float)((int)(b0 & 15) - 8)),
                                         __fmul_rn(av.y, (float)((int)(b0 >> 4) - 8))));
        gacc = __fadd_rn(gacc, __fadd_rn(__fmul_rn(av.z, (float)((int)(b1 & 15) - 8)),
                                         __fmul_rn(av.w, (float)((int)(b1 >> 4) - 8))));
      }
      prod[i] = __fmul_rn(gacc, load_scale(ws, (size_t)ni * ng + g));
    }
  }
  const float acc = fold_in_order(0.f, prod, ng, lane);
  if (lane == 0) out[(size_t)mi * n + ni] = acc;
}

// ---------------------------------------------------------------------------
// P7: int4_matmul_gemv_q4_x_q8 (shape_ops.rs:2923-3028).
// Stage 1 (k_q8_0_acts): Q8_0-style activations into scratch: per 32 values
// scale = max|x|/127 (1.0 for an all-zero group), q = clamp(round(x*(1/scale)),
// -128, 127). Stage 2 (k_int4_q4q8): warp per output row, integer group
// dots, total += (dot * w_scale) * a_scale folded in group order.
// ---------------------------------------------------------------------------
__global__ void k_q8_0_acts(const float* __restrict__ a, int k, int8_t* q, float* sc) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= k / 32) return;
  const float* grp = a + (size_t)g * 32;
  float mx = 0.f;
  for (int i = 0; i < 32; i++) {
    const float av = fabsf(grp[i]);
    if (av > mx) mx = av;
  }
  const float scale = mx > 0.f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, scale);
  sc[g] = scale;
  for (int i = 0; i < 32; i++) {
    // Rust: (x * inv).round().clamp(-128.0, 127.0) as i8 -- clamp keeps NaN,
    // and `as i8` maps NaN to 0.
    const float r = roundf(__fmul_rn(grp[i], inv));
    q[(size_t)g * 32 + i] = (int8_t)(r != r ? 0 : (int)fmaxf(-128.f, fminf(r, 127.f)));
  }
}

template <typename SCALE_T>
__global__ void __launch_bounds__(256) k_int4_q4q8(const int8_t* __restrict__ aq, const float* __restrict__ as,
                                                   const uint8_t* __restrict__ wp,
                                                   const SCALE_T* __restrict__ ws, float* out, int n, int k) {
  const int lane = threadIdx.x & 31;
  const int ni = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (ni >= n) return;
  const int ng = k / 32;
  const uint8_t* wr = wp + (size_t)ni * (k / 2);
  float prod[MAX_GROUPS_PER_LANE];
#pragma unroll
  for (int i = 0; i < MAX_GROUPS_PER_LANE; i++) {
    prod[i] = 0.f;
    const int g = lane + 32 * i;
    if (g < ng) {
      const uint4 pk = *reinterpret_cast<const uint4*>(wr + (size_t)g * 16);
      const int4 a0 = *reinterpret_cast<const int4*>(aq + (size_t)g * 32);
      const int4 a1 = *reinterpret_cast<const int4*>(aq + (size_t)g * 32 + 16);
      const uint32_t bw[4] = {pk.x, pk.y, pk.z, pk.w};
      const uint32_t aw[8] = {(uint32_t)a0.x, (uint32_t)a0.y, (uint32_t)a0.z, (uint32_t)a0.w,
                              (uint32_t)a1.x, (uint32_t)a1.y, (uint32_t)a1.z, (uint32_t)a1.w};
      int dot = 0;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        // 4 packed bytes = 8 weights (k = 8j .. 8j+7); even k in the low nibble.
        const uint32_t lo = bw[j] & 0x0F0F0F0Fu, hi = (bw[j] >> 4) & 0x0F0F0F0Fu;
        // de-interleave the activations: even k -> lo lanes, odd k -> hi lanes
        const uint32_t x0 = aw[2 * j], x1 = aw[2 * j + 1];  // k = 8j..8j+3, 8j+4..8j+7
        const uint32_t ev = __byte_perm(x0, x1, 0x6420), od = __byte_perm(x0, x1, 0x7531);
        dot = __dp4a((int)lo, (int)ev, dot);
        dot = __dp4a((int)hi, (int)od, dot);
        // the -8 bias: sum_i -8 * a_i
        dot -= 8 * (__dp4a(0x01010101, (int)ev, 0) + __dp4a(0x01010101, (int)od, 0));
      }
      prod[i] = __fmul_rn(__fmul_rn((float)dot, load_scale(ws, (size_t)ni * ng + g)), as[g]);
    }
  }
  const float acc = fold_in_order(0.f, prod, ng, lane);
  if (lane == 0) out[ni] = acc;
}

// ---------------------------------------------------------------------------
// P8: quantize_int4_q4_0 (shape_ops.rs:3242-3275). Thread per group.
// ---------------------------------------------------------------------------
__global__ void k_quant_int4(const float* __restrict__ w, int64_t n, int k, uint8_t* packed, float* scales) {
  const int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int ng = k / 32;
  if (gi >= n * ng) return;
  const int64_t ni = gi / ng;
  const int g = (int)(gi % ng);
  const float* grp = w + ni * k + (int64_t)g * 32;
  float mx = 0.f;
  for (int i = 0; i < 32; i++) mx = fmaxf(mx, fabsf(grp[i]));
  const float scale = mx > 0.f ? __fdiv_rn(mx, 7.0f) : 1.0f;
  scales[gi] = scale;
  for (int j = 0; j < 16; j++) {
    const float xl = roundf(__fdiv_rn(grp[2 * j], scale)), xh = roundf(__fdiv_rn(grp[2 * j + 1], scale));
    int ql = (xl != xl) ? 0 : (int)fmaxf(-2147483648.f, fminf(xl, 2147483520.f));
    int qh = (xh != xh) ? 0 : (int)fmaxf(-2147483648.f, fminf(xh, 2147483520.f));
    ql = max(-8, min(7, ql)) + 8;
    qh = max(-8, min(7, qh)) + 8;
    packed[ni * (k / 2) + (int64_t)g * 16 + j] = (uint8_t)((qh << 4) | ql);
  }
}

// ---------------------------------------------------------------------------
// P9: rmsnorm_f32 (shape_ops.rs:976-1018), parallel sum of squares.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_rmsnorm(const float* __restrict__ x, const float* __restrict__ g,
                                                 float* out, int inner, float eps) {
  __shared__ float red[33];
  const float* r = x + (size_t)blockIdx.x * inner;
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < inner; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(r + i);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[32] = v;
  }
  __syncthreads();
  const float inv_n = __fdiv_rn(1.0f, (float)inner);
  const float inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(red[32], inv_n), eps)));
  float* o = out + (size_t)blockIdx.x * inner;
  for (int i = threadIdx.x * 4; i < inner; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(r + i);
    const float4 gg = *reinterpret_cast<const float4*>(g + i);
    float4 res;
    res.x = __fmul_rn(__fmul_rn(v.x, inv_rms), gg.x);
    res.y = __fmul_rn(__fmul_rn(v.y, inv_rms), gg.y);
    res.z = __fmul_rn(__fmul_rn(v.z, inv_rms), gg.z);
    res.w = __fmul_rn(__fmul_rn(v.w, inv_rms), gg.w);
    *reinterpret_cast<float4*>(o + i) = res;
  }
}

// ---------------------------------------------------------------------------
// P10: flash attention, online softmax (shape_ops.rs:464-558), f32 CUDA
// cores. CTA = 8 warps x 8 query rows; key/value tiles of 64 in shared
// memory; causal rows stop at their own index (Sq == Sk aligned at 0 in the
// reference). T = float or __half inputs; output f32.
// ---------------------------------------------------------------------------
constexpr int FA_KT = 64, FA_ROWS_PER_WARP = 8, FA_WARPS = 8;

template <typename T>
__device__ __forceinline__ float ldf(const T* p);
template <>
__device__ __forceinline__ float ldf<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldf<__half>(const __half* p) { return __half2float(*p); }

template <typename T, int D>
__global__ void __launch_bounds__(256) k_flash_attn(const T* __restrict__ q, const T* __restrict__ kk,
                                                    const T* __restrict__ vv, float* out, float scale,
                                                    int sq, int sk, int causal) {
  extern __shared__ float fsm[];
  constexpr int ROWS = FA_WARPS * FA_ROWS_PER_WARP;
  float* Ks = fsm;                    // [FA_KT][D+1] (padded: conflict-free column reads)
  float* Vs = Ks + FA_KT * (D + 1);   // [FA_KT][D]
  float* Qs = Vs + FA_KT * D;         // [ROWS][D]
  const int bh = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cta_row0 = blockIdx.x * ROWS;
  const int row0 = cta_row0 + warp * FA_ROWS_PER_WARP;
  const T* qb = q + (size_t)bh * sq * D;
  const T* kb = kk + (size_t)bh * sk * D;
  const T* vb = vv + (size_t)bh * sk * D;
  constexpr int DL = D / 32;  // output dims per lane
  for (int i = threadIdx.x; i < ROWS * D; i += blockDim.x) {
    const int r = i / D, d = i % D;
    Qs[i] = cta_row0 + r < sq ? ldf(qb + (size_t)(cta_row0 + r) * D + d) : 0.f;
  }
  float o[FA_ROWS_PER_WARP][DL];
  float mrow[FA_ROWS_PER_WARP], lrow[FA_ROWS_PER_WARP];
#pragma unroll
  for (int r = 0; r < FA_ROWS_PER_WARP; r++) {
#pragma unroll
    for (int j = 0; j < DL; j++) o[r][j] = 0.f;
    mrow[r] = -INFINITY;
    lrow[r] = 0.f;
  }
  const int cta_last_row = min(sq - 1, cta_row0 + ROWS - 1);
  const int kend = causal ? min(sk, cta_last_row + 1) : sk;
  const float* Qw = Qs + warp * FA_ROWS_PER_WARP * D;
  for (int t0 = 0; t0 < kend; t0 += FA_KT) {
    __syncthreads();
    for (int i = threadIdx.x; i < FA_KT * D; i += blockDim.x) {
      const int t = i / D, d = i % D;
      const bool ok = t0 + t < sk;
      Ks[t * (D + 1) + d] = ok ? ldf(kb + (size_t)(t0 + t) * D + d) : 0.f;
      Vs[t * D + d] = ok ? ldf(vb + (size_t)(t0 + t) * D + d) : 0.f;
    }
    __syncthreads();
    if (row0 >= sq || (causal && t0 > row0 + FA_ROWS_PER_WARP - 1)) continue;
    // scores: lane owns keys t0+lane and t0+lane+32 for the warp's rows
    float acc[FA_ROWS_PER_WARP][2];
#pragma unroll
    for (int r = 0; r < FA_ROWS_PER_WARP; r++) acc[r][0] = acc[r][1] = 0.f;
    for (int d = 0; d < D; d++) {
      const float k0 = Ks[lane * (D + 1) + d], k1 = Ks[(lane + 32) * (D + 1) + d];
#pragma unroll
      for (int r = 0; r < FA_ROWS_PER_WARP; r++) {
        const float qv = Qw[r * D + d];
        acc[r][0] += qv * k0;
        acc[r][1] += qv * k1;
      }
    }
#pragma unroll
    for (int r = 0; r < FA_ROWS_PER_WARP; r++) {
      const int i = row0 + r;
      const int lim = i >= sq ? 0 : (causal ? min(sk, i + 1) : sk);
      if (t0 >= lim) continue;  // warp-uniform
      const float s0 = (t0 + lane < lim) ? acc[r][0] * scale : -INFINITY;
      const float s1 = (t0 + lane + 32 < lim) ? acc[r][1] * scale : -INFINITY;
      float mt = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float mnew = fmaxf(mrow[r], mt);
      const float corr = expf(mrow[r] - mnew);
      const float p0 = expf(s0 - mnew), p1 = expf(s1 - mnew);
      lrow[r] = lrow[r] * corr + warp_sum(p0 + p1);
      mrow[r] = mnew;
#pragma unroll
      for (int j = 0; j < DL; j++) o[r][j] *= corr;
      for (int t = 0; t < FA_KT; t++) {
        const float p = __shfl_sync(0xffffffffu, t < 32 ? p0 : p1, t & 31);
#pragma unroll
        for (int j = 0; j < DL; j++) o[r][j] += p * Vs[t * D + lane + 32 * j];
      }
    }
  }
#pragma unroll
  for (int r = 0; r < FA_ROWS_PER_WARP; r++) {
    const int i = row0 + r;
    if (i >= sq) continue;
    const float inv = lrow[r] > 0.f ? 1.0f / lrow[r] : 0.f;
#pragma unroll
    for (int j = 0; j < DL; j++) out[((size_t)bh * sq + i) * D + lane + 32 * j] = o[r][j] * inv;
  }
}

template <typename T>
int launch_flash(const T* q, const T* k, const T* v, float* out, float scale, int64_t b, int64_t h,
                 int64_t sq, int64_t sk, int64_t d, int causal, cudaStream_t s) {
  const int rows = FA_WARPS * FA_ROWS_PER_WARP;
  dim3 grid((unsigned)((sq + rows - 1) / rows), (unsigned)(b * h));
  const size_t smem = ((size_t)FA_KT * ((d + 1) + d) + (size_t)rows * d) * 4;
#define FA_CASE(DD)                                                                                  \
  case DD:                                                                                           \
    ARMAI_CUDA(cudaFuncSetAttribute(k_flash_attn<T, DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    k_flash_attn<T, DD><<<grid, 256, smem, s>>>(q, k, v, out, scale, (int)sq, (int)sk, causal);     \
    break;
  switch (d) {
    FA_CASE(32)
    FA_CASE(64)
    FA_CASE(128)
    default:
      return fail(ARMAI_E_INVALID, "flash_attn: head dim must be 32, 64 or 128");
  }
#undef FA_CASE
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

// ---------------------------------------------------------------------------
// P11: dequant_matmul_int8_f32 (shape_ops.rs:1525-1582): acc += a*w in k
// order, row = acc * s. Thread per output (the serial chain IS the spec).
// ---------------------------------------------------------------------------
__global__ void k_dequant_i8(const float* __restrict__ act, const int8_t* __restrict__ w,
                             const float* __restrict__ sc, float* out, int64_t rows, int n, int k) {
  const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= rows * n) return;
  const int64_t r = o / n;
  const int j = (int)(o % n);
  const float* a = act + r * k;
  const int8_t* wr = w + (int64_t)j * k;
  float acc = 0.f;
  for (int i = 0; i < k; i++) acc = __fadd_rn(acc, __fmul_rn(a[i], (float)wr[i]));
  out[o] = __fmul_rn(acc, sc[j]);
}

// ---------------------------------------------------------------------------
// LLM helper primitives (lib.rs:147-354 -> shape_ops.rs).
// ---------------------------------------------------------------------------
// rope_f32 (shape_ops.rs:1040-1100): thread per (row, pair k). pos =
// positions[row / heads_per_token] as f32, theta = pos * inv_freq[k], then
// (x0 cos - x1 sin, x0 sin + x1 cos), each product and sum rounded on its own.
__global__ void k_rope(const float* __restrict__ x, const int64_t* __restrict__ pos,
                       const float* __restrict__ inv_freq, float* out, int64_t n_rows, int half,
                       int64_t heads_per_token) {
  const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= n_rows * half) return;
  const int64_t row = o / half;
  const int k = (int)(o % half);
  const float p = (float)pos[row / heads_per_token];
  const float theta = __fmul_rn(p, inv_freq[k]);
  const float c = cosf(theta), s = sinf(theta);
  const float2 v = reinterpret_cast<const float2*>(x)[o];
  reinterpret_cast<float2*>(out)[o] = make_float2(__fsub_rn(__fmul_rn(v.x, c), __fmul_rn(v.y, s)),
                                                  __fadd_rn(__fmul_rn(v.x, s), __fmul_rn(v.y, c)));
}

// softmax_last_axis_f32 (shape_ops.rs:2719-2751): block per row. max as the
// reference scans it (start at src[0], replace on v > max: a NaN at src[0]
// stays, later NaNs are skipped), e = exp(x - max), sum (parallel), then
// e * (1 / sum).
__global__ void k_softmax(const float* __restrict__ x, float* out, int inner) {
  __shared__ float red[32];
  __shared__ float bc;
  const float* src = x + (int64_t)blockIdx.x * inner;
  float* dst = out + (int64_t)blockIdx.x * inner;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  float m = -INFINITY;
  for (int i = tid; i < inner; i += blockDim.x) m = fmaxf(m, src[i]);  // fmaxf skips NaN
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[wid] = m;
  __syncthreads();
  if (tid == 0) {
    float mm = red[0];
    for (int w = 1; w < nw; w++) mm = fmaxf(mm, red[w]);
    const float s0 = src[0];
    bc = isnan(s0) ? s0 : fmaxf(s0, mm);
  }
  __syncthreads();
  const float mx = bc;
  float sum = 0.f;
  for (int i = tid; i < inner; i += blockDim.x) {
    const float e = expf(__fsub_rn(src[i], mx));
    dst[i] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = warp_sum(sum);
  __syncthreads();
  if (lane == 0) red[wid] = sum;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < nw; w++) t = __fadd_rn(t, red[w]);
    bc = __fdiv_rn(1.0f, t);
  }
  __syncthreads();
  const float inv = bc;
  for (int i = tid; i < inner; i += blockDim.x) dst[i] = __fmul_rn(dst[i], inv);
}

// silu_gate_mul_up_f32 (shape_ops.rs:2755-2770): g * (1 / (1 + exp(-g))) * u.
__global__ void k_silu_gate_mul_up(const float* __restrict__ g, const float* __restrict__ u, float* out,
                                   int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gv = g[i];
  const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
  out[i] = __fmul_rn(__fmul_rn(gv, sig), u[i]);
}

// dequantize_q6_k (shape_ops.rs:2848-2899): thread per (block, half n,
// l < 32), four outputs like the reference's inner loop. The reference takes
// the sub-scales scales[8n + {0, 2, 4, 6}] for all 32 values of each group
// (ggml's dequantize_row_q6_K uses 8n + l/16 + {0, 2, 4, 6}); this follows
// the reference. The reference reads the sub-scales from a `&[u8]` and
// widens them with `as i32` (shape_ops.rs:2860,2887-2890), so they are
// unsigned 0..255 here (ggml's Q6_K scales are int8).
// value = d * (float)(scale * q), one rounding.
__global__ void k_dequant_q6k(const uint8_t* __restrict__ in, float* out, int64_t n_blocks) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n_blocks * 64) return;
  const int64_t b = t >> 6;
  const int n = (int)(t >> 5) & 1, l = (int)t & 31;
  const uint8_t* blk = in + b * 210;
  const uint8_t* ql = blk + 64 * n;
  const uint8_t qh = blk[128 + 32 * n + l];
  const uint8_t* sc = blk + 192 + 8 * n;  // u8 -> i32: zero-extended
  const float d = __half2float(__ushort_as_half((uint16_t)(blk[208] | (blk[209] << 8))));
  const int q1 = ((ql[l] & 0xF) | (((qh >> 0) & 3) << 4)) - 32;
  const int q2 = ((ql[l + 32] & 0xF) | (((qh >> 2) & 3) << 4)) - 32;
  const int q3 = ((ql[l] >> 4) | (((qh >> 4) & 3) << 4)) - 32;
  const int q4 = ((ql[l + 32] >> 4) | (((qh >> 6) & 3) << 4)) - 32;
  float* o = out + b * 256 + 128 * n + l;
  o[0] = __fmul_rn(d, (float)((int)sc[0] * q1));
  o[32] = __fmul_rn(d, (float)((int)sc[2] * q2));
  o[64] = __fmul_rn(d, (float)((int)sc[4] * q3));
  o[96] = __fmul_rn(d, (float)((int)sc[6] * q4));
}

// dequant_matmul_f16_f32 (shape_ops.rs:1462-1490, the x86 path): out[r][j] =
// sum over k in order of a[r][k] * f32(w[j][k]), product and sum rounded
// separately (bit-exact with the reference's serial loop). A CTA of 8 warps
// covers JW * 32 weight rows (lane = row) and 4 * 8 / JW activation rows per
// thread group; weights and activations pass through shared memory in chunks
// of 32 along K, converted to f32 and padded so lanes read distinct banks.
constexpr int F16_KC = 32;
template <int JW>
__global__ void __launch_bounds__(256) k_dequant_f16(const float* __restrict__ act,
                                                     const uint16_t* __restrict__ w, float* out, int64_t rows,
                                                     int n, int k) {
  constexpr int RW = 8 / JW;          // warps along activation rows
  constexpr int JT = 32 * JW;         // weight rows per CTA
  constexpr int RT = 4 * RW;          // activation rows per CTA
  __shared__ float ws[JT][F16_KC + 1];
  __shared__ float as[RT][F16_KC];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int jw = wid % JW, rw = wid / JW;
  const int64_t j0 = (int64_t)blockIdx.x * JT, r0 = (int64_t)blockIdx.y * RT;
  const int64_t j = j0 + jw * 32 + lane;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int kc = 0; kc < k; kc += F16_KC) {
    const int kn = min(F16_KC, k - kc);
    for (int e = tid; e < JT * F16_KC; e += 256) {
      const int jr = e / F16_KC, kk = e % F16_KC;
      const int64_t jj = j0 + jr;
      ws[jr][kk] = (jj < n && kk < kn) ? __half2float(__ushort_as_half(w[jj * k + kc + kk])) : 0.f;
    }
    for (int e = tid; e < RT * F16_KC; e += 256) {
      const int rr = e / F16_KC, kk = e % F16_KC;
      const int64_t r = r0 + rr;
      as[rr][kk] = (r < rows && kk < kn) ? act[r * k + kc + kk] : 0.f;
    }
    __syncthreads();
    for (int kk = 0; kk < kn; kk++) {
      const float wv = ws[jw * 32 + lane][kk];
#pragma unroll
      for (int i = 0; i < 4; i++) acc[i] = __fadd_rn(acc[i], __fmul_rn(as[rw * 4 + i][kk], wv));
    }
    __syncthreads();
  }
  if (j < n) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int64_t r = r0 + rw * 4 + i;
      if (r < rows) out[r * n + j] = acc[i];
    }
  }
}

int finish(cudaStream_t s, void* dst, const void* src, size_t bytes) {
  ARMAI_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s));
  ARMAI_CUDA(cudaStreamSynchronize(s));
  return ARMAI_OK;
}

}  // namespace

// ===========================================================================
// Host-pointer entry points (NIF mirrors).
// ===========================================================================
extern "C" int armai_int8_matmul_s32(const int8_t* a, size_t a_len, const int8_t* w, size_t w_len,
                                     size_t m, size_t n, size_t k, int32_t* out) {
  if (a_len != m * k) return fail(ARMAI_E_INVALID, lenmsg("int8_matmul: a", a_len, "M*K", m * k));
  if (w_len != n * k) return fail(ARMAI_E_INVALID, lenmsg("int8_matmul: w", w_len, "N*K", n * k));
  if (!m || !n) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped da(s), dw(s), dout(s);
  ARMAI_TRY(h2d(da, a, a_len));
  ARMAI_TRY(h2d(dw, w, w_len));
  ARMAI_TRY(dalloc(dout, m * n * 4));
  ARMAI_TRY(launch_int8_gemm((int8_t*)da.p, (int8_t*)dw.p, (int32_t*)dout.p, nullptr, nullptr, 0, 0.f,
                             nullptr, (int64_t)m, (int64_t)n, (int64_t)k, s));
  ARMAI_TRY(finish(s, out, dout.p, m * n * 4));
  return int8_gemm_tc_check();
}

static int int8_f32_common(const int8_t* a, size_t a_len, const int8_t* w, size_t w_len,
                           const float* act_scales, size_t act_len, int per_token, float act_scale,
                           const float* w_scales, size_t ws_len, size_t m, size_t n, size_t k, float* out,
                           const char* name) {
  const std::string nm(name);
  if (a_len != m * k) return fail(ARMAI_E_INVALID, lenmsg((nm + ": a").c_str(), a_len, "M*K", m * k));
  if (w_len != n * k) return fail(ARMAI_E_INVALID, lenmsg((nm + ": w").c_str(), w_len, "N*K", n * k));
  if (ws_len != n) return fail(ARMAI_E_INVALID, lenmsg((nm + ": w_scales").c_str(), ws_len, "N", n));
  if (per_token && act_len != m)
    return fail(ARMAI_E_INVALID, lenmsg((nm + ": act_scales").c_str(), act_len, "M", m));
  if (!m || !n) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped da(s), dw(s), dws(s), das(s), dout(s);
  ARMAI_TRY(h2d(da, a, a_len));
  ARMAI_TRY(h2d(dw, w, w_len));
  ARMAI_TRY(h2d(dws, w_scales, n * 4));
  if (per_token) ARMAI_TRY(h2d(das, act_scales, m * 4));
  ARMAI_TRY(dalloc(dout, m * n * 4));
  ARMAI_TRY(launch_int8_gemm((int8_t*)da.p, (int8_t*)dw.p, nullptr, (float*)dout.p, (float*)das.p,
                             per_token, act_scale, (float*)dws.p, (int64_t)m, (int64_t)n, (int64_t)k, s));
  ARMAI_TRY(finish(s, out, dout.p, m * n * 4));
  return int8_gemm_tc_check();
}

extern "C" int armai_int8_matmul_f32(const int8_t* a, size_t a_len, const int8_t* w, size_t w_len,
                                     const float* w_scales, size_t w_scales_len, double act_scale,
                                     size_t m, size_t n, size_t k, float* out) {
  return int8_f32_common(a, a_len, w, w_len, nullptr, 0, 0, (float)act_scale, w_scales, w_scales_len, m,
                         n, k, out, "int8_matmul");
}

extern "C" int armai_int8_matmul_f32_per_token(const int8_t* a, size_t a_len, const int8_t* w,
                                               size_t w_len, const float* act_scales,
                                               size_t act_scales_len, const float* w_scales,
                                               size_t w_scales_len, size_t m, size_t n, size_t k,
                                               float* out) {
  return int8_f32_common(a, a_len, w, w_len, act_scales, act_scales_len, 1, 0.f, w_scales, w_scales_len,
                         m, n, k, out, "int8_matmul_per_token");
}

extern "C" int armai_quantize_int8_per_token(const float* a, size_t a_len, size_t m, size_t k, int8_t* q,
                                             float* scales) {
  if (a_len != m * k)
    return fail(ARMAI_E_INVALID, lenmsg("quantize_int8_per_token: a", a_len, "M*K", m * k));
  if (!m) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped da(s), dq(s), dsc(s);
  ARMAI_TRY(h2d(da, a, a_len * 4));
  ARMAI_TRY(dalloc(dq, m * k));
  ARMAI_TRY(dalloc(dsc, m * 4));
  k_quant_int8_rows<<<(unsigned)m, 256, 0, s>>>((float*)da.p, (int)k, (int8_t*)dq.p, (float*)dsc.p);
  ARMAI_CUDA(cudaGetLastError());
  ARMAI_CUDA(cudaMemcpyAsync(q, dq.p, m * k, cudaMemcpyDeviceToHost, s));
  return finish(s, scales, dsc.p, m * 4);
}

static int int4_checks(size_t a_len, size_t w_len, size_t s_len, size_t m, size_t n, size_t k) {
  if (k % 32) return fail(ARMAI_E_INVALID, "int4_matmul: K=" + std::to_string(k) + " must be multiple of 32");
  if (k / 32 > 32 * MAX_GROUPS_PER_LANE) return fail(ARMAI_E_INVALID, "int4_matmul: K above 16384 is not supported");
  if (a_len != m * k) return fail(ARMAI_E_INVALID, lenmsg("int4_matmul: a", a_len, "M*K", m * k));
  if (w_len != n * (k / 2)) return fail(ARMAI_E_INVALID, "int4_matmul: packed len " + std::to_string(w_len) + " != N*K/2 = " + std::to_string(n * (k / 2)));
  if (s_len != n * (k / 32)) return fail(ARMAI_E_INVALID, "int4_matmul: scales len " + std::to_string(s_len) + " != N*K/32 = " + std::to_string(n * (k / 32)));
  return ARMAI_OK;
}

extern "C" int armai_dev_int4_matmul_f32(const float* a, const uint8_t* w_packed, const float* w_scales,
                                         float* out, int64_t m, int64_t n, int64_t k, void* stream) {
  if (k % 32 || k / 32 > 32 * MAX_GROUPS_PER_LANE) return fail(ARMAI_E_INVALID, "int4_matmul: unsupported K");
  if (!m || !n) return ARMAI_OK;
  dim3 g((unsigned)((n + 7) / 8), (unsigned)m);
  k_int4_f32<float><<<g, 256, 0, (cudaStream_t)stream>>>(a, w_packed, w_scales, out, (int)m, (int)n, (int)k);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

extern "C" int armai_int4_matmul_f32(const float* a, size_t a_len, const uint8_t* w_packed,
                                     size_t w_packed_len, const float* w_scales, size_t w_scales_len,
                                     size_t m, size_t n, size_t k, float* out) {
  ARMAI_TRY(int4_checks(a_len, w_packed_len, w_scales_len, m, n, k));
  if (!m || !n) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped da(s), dw(s), dsc(s), dout(s);
  ARMAI_TRY(h2d(da, a, a_len * 4));
  ARMAI_TRY(h2d(dw, w_packed, w_packed_len));
  ARMAI_TRY(h2d(dsc, w_scales, w_scales_len * 4));
  ARMAI_TRY(dalloc(dout, m * n * 4));
  ARMAI_TRY(armai_dev_int4_matmul_f32((float*)da.p, (uint8_t*)dw.p, (float*)dsc.p, (float*)dout.p,
                                      (int64_t)m, (int64_t)n, (int64_t)k, s));
  return finish(s, out, dout.p, m * n * 4);
}

extern "C" int armai_int4_matmul_gemv(const float* a, size_t a_len, const uint8_t* w_packed,
                                      size_t w_packed_len, const float* w_scales, size_t w_scales_len,
                                      size_t n, size_t k, float* out) {
  // On x86 the reference's gemv NIF is int4_matmul_f32 with M = 1
  // (shape_ops.rs:3157-3166); the CUDA path computes the same thing.
  return armai_int4_matmul_f32(a, a_len, w_packed, w_packed_len, w_scales, w_scales_len, 1, n, k, out);
}

namespace {
template <typename SCALE_T>
int q4q8_dev(const float* a, const uint8_t* w_packed, const SCALE_T* w_scales, float* out, int64_t n,
             int64_t k, int8_t* aq, float* as, cudaStream_t s) {
  const int ng = (int)(k / 32);
  k_q8_0_acts<<<(ng + 127) / 128, 128, 0, s>>>(a, (int)k, aq, as);
  k_int4_q4q8<SCALE_T><<<(unsigned)((n + 7) / 8), 256, 0, s>>>(aq, as, w_packed, w_scales, out, (int)n, (int)k);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

template <typename SCALE_T>
int q4q8_dev_alloc(const float* a, const uint8_t* w_packed, const SCALE_T* w_scales, float* out, int64_t n,
                   int64_t k, cudaStream_t s) {
  if (k % 32 || k / 32 > 32 * MAX_GROUPS_PER_LANE) return fail(ARMAI_E_INVALID, "int4_matmul: unsupported K");
  if (!n) return ARMAI_OK;
  Scoped scratch(s);
  ARMAI_TRY(dalloc(scratch, (size_t)k + (size_t)(k / 32) * 4));
  int8_t* aq = (int8_t*)scratch.p;
  float* as = (float*)((uint8_t*)scratch.p + k);  // k % 32 == 0 keeps this 4-byte aligned
  return q4q8_dev<SCALE_T>(a, w_packed, w_scales, out, n, k, aq, as, s);
}
}  // namespace

extern "C" int armai_dev_int4_gemv_q4_x_q8(const float* a, const uint8_t* w_packed, const float* w_scales,
                                           float* out, int64_t n, int64_t k, void* stream) {
  return q4q8_dev_alloc<float>(a, w_packed, w_scales, out, n, k, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// No-allocation variant of armai_dev_int4_gemv_q4_x_q8: the stage-1 scratch
// (K int8 activations, then K/32 f32 group scales) is a file-scope device
// array sized for the kernel's largest K, so a call makes no allocation.
// Nothing in it needs to start at zero: stage 1 writes every byte stage 2
// reads. Calls on one device share it, so they must not overlap in time.
// ---------------------------------------------------------------------------
constexpr int64_t Q4Q8_NOALLOC_MAX_K = 32LL * 32 * MAX_GROUPS_PER_LANE;  // 16384
static __device__ __align__(256) uint8_t g_q4q8_scratch[Q4Q8_NOALLOC_MAX_K + Q4Q8_NOALLOC_MAX_K / 32 * 4];

namespace {
// Device address of the current device's copy of the scratch. Looked up on
// every call rather than cached: the lookup is cheap once the module is
// loaded, and an address cached per device number would go stale if the
// host program reset the device (cudaDeviceReset) and made a new context.
// The first call on a device may load the module.
int q4q8_scratch(uint8_t** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_q4q8_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_q4q8_scratch)", __FILE__, __LINE__);
  *out = static_cast<uint8_t*>(p);
  return ARMAI_OK;
}
}  // namespace

extern "C" int armai_dev_int4_gemv_q4_x_q8_noalloc(const float* a, const uint8_t* w_packed,
                                                   const float* w_scales, float* out, int64_t n, int64_t k,
                                                   void* stream) {
  if (k <= 0 || k % 32)
    return fail(ARMAI_E_INVALID, "int4_gemv_q4_x_q8_noalloc: K=" + std::to_string(k) +
                                     " must be a positive multiple of 32");
  if (k > Q4Q8_NOALLOC_MAX_K)
    return fail(ARMAI_E_RANGE, "int4_gemv_q4_x_q8_noalloc: K=" + std::to_string(k) +
                                   " exceeds the static scratch (K <= " + std::to_string(Q4Q8_NOALLOC_MAX_K) +
                                   "); use armai_dev_int4_gemv_q4_x_q8");
  if (n < 0) return fail(ARMAI_E_INVALID, "int4_gemv_q4_x_q8_noalloc: negative N");
  if (!n) return ARMAI_OK;
  uint8_t* scratch = nullptr;
  ARMAI_TRY(q4q8_scratch(&scratch));
  int8_t* aq = reinterpret_cast<int8_t*>(scratch);
  float* as = reinterpret_cast<float*>(scratch + k);  // k % 32 == 0 keeps this 4-byte aligned
  return q4q8_dev<float>(a, w_packed, w_scales, out, n, k, aq, as, (cudaStream_t)stream);
}

extern "C" int armai_dev_int4_gemv_f16s(const float* a, const uint8_t* w_packed, const uint16_t* w_scales,
                                        float* out, int64_t n, int64_t k, void* stream) {
  return q4q8_dev_alloc<__half>(a, w_packed, reinterpret_cast<const __half*>(w_scales), out, n, k,
                                (cudaStream_t)stream);
}

extern "C" int armai_int4_matmul_gemv_q4_x_q8(const float* a, size_t a_len, const uint8_t* w_packed,
                                              size_t w_packed_len, const float* w_scales,
                                              size_t w_scales_len, size_t n, size_t k, float* out) {
  ARMAI_TRY(int4_checks(a_len, w_packed_len, w_scales_len, 1, n, k));
  if (!n) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped da(s), dw(s), dsc(s), dout(s);
  ARMAI_TRY(h2d(da, a, a_len * 4));
  ARMAI_TRY(h2d(dw, w_packed, w_packed_len));
  ARMAI_TRY(h2d(dsc, w_scales, w_scales_len * 4));
  ARMAI_TRY(dalloc(dout, n * 4));
  ARMAI_TRY(armai_dev_int4_gemv_q4_x_q8((float*)da.p, (uint8_t*)dw.p, (float*)dsc.p, (float*)dout.p,
                                        (int64_t)n, (int64_t)k, s));
  return finish(s, out, dout.p, n * 4);
}

extern "C" int armai_quantize_int4_q4_0(const float* w, size_t w_len, size_t n, size_t k, uint8_t* packed,
                                        float* scales) {
  if (k % 32) return fail(ARMAI_E_INVALID, "quantize_int4: K=" + std::to_string(k) + " must be multiple of 32");
  if (w_len != n * k) return fail(ARMAI_E_INVALID, lenmsg("quantize_int4: w", w_len, "N*K", n * k));
  if (!n || !k) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped dwt(s), dp(s), dsc(s);
  ARMAI_TRY(h2d(dwt, w, w_len * 4));
  ARMAI_TRY(dalloc(dp, n * k / 2));
  ARMAI_TRY(dalloc(dsc, n * (k / 32) * 4));
  const int64_t groups = (int64_t)n * (k / 32);
  k_quant_int4<<<(unsigned)((groups + 255) / 256), 256, 0, s>>>((float*)dwt.p, (int64_t)n, (int)k,
                                                                 (uint8_t*)dp.p, (float*)dsc.p);
  ARMAI_CUDA(cudaGetLastError());
  ARMAI_CUDA(cudaMemcpyAsync(packed, dp.p, n * k / 2, cudaMemcpyDeviceToHost, s));
  return finish(s, scales, dsc.p, n * (k / 32) * 4);
}

extern "C" int armai_dev_rmsnorm_f32(const float* x, const float* gamma, float* out, int64_t n_outer,
                                     int64_t inner, float eps, void* stream) {
  if (inner % 4) return fail(ARMAI_E_INVALID, "rmsnorm: inner must be a multiple of 4 on this path");
  if (!n_outer) return ARMAI_OK;
  k_rmsnorm<<<(unsigned)n_outer, 256, 0, (cudaStream_t)stream>>>(x, gamma, out, (int)inner, eps);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

extern "C" int armai_rmsnorm_f32(const float* input, size_t input_len, const float* gamma, size_t gamma_len,
                                 size_t n_outer, size_t inner, double epsilon, float* out) {
  if (input_len != n_outer * inner)
    return fail(ARMAI_E_INVALID, lenmsg("rmsnorm: input", input_len, "n_outer*inner", n_outer * inner));
  if (gamma_len != inner)
    return fail(ARMAI_E_INVALID, "rmsnorm: gamma len " + std::to_string(gamma_len) + " != inner " + std::to_string(inner));
  if (!n_outer) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped dx(s), dg(s), dout(s);
  ARMAI_TRY(h2d(dx, input, input_len * 4));
  ARMAI_TRY(h2d(dg, gamma, gamma_len * 4));
  ARMAI_TRY(dalloc(dout, input_len * 4));
  ARMAI_TRY(armai_dev_rmsnorm_f32((float*)dx.p, (float*)dg.p, (float*)dout.p, (int64_t)n_outer,
                                  (int64_t)inner, (float)epsilon, s));
  return finish(s, out, dout.p, input_len * 4);
}

extern "C" int armai_dev_flash_attention_f32(const float* q, const float* k, const float* v, float* out,
                                             float scale, int64_t b, int64_t h, int64_t sq, int64_t sk,
                                             int64_t d, int causal, void* stream) {
  if (!b || !h || !sq) return ARMAI_OK;
  return launch_flash<float>(q, k, v, out, scale, b, h, sq, sk, d, causal, (cudaStream_t)stream);
}

extern "C" int armai_dev_flash_attention_f16(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                             float* out, float scale, int64_t b, int64_t h, int64_t sq,
                                             int64_t sk, int64_t d, int causal, void* stream) {
  if (!b || !h || !sq) return ARMAI_OK;
  if ((d == 64 || d == 128) && sk > 0) {
    // tensor cores (f16 operands are the inputs' own type): q, k and v^T
    // rearranged into the kernel's operand tiles first (stream-ordered
    // scratch from the library pool, freed after the launch)
    const cudaStream_t s = (cudaStream_t)stream;
    const size_t tb = fa_tile_bytes((int)d), nqt = (size_t)(sq + 127) / 128, nkt = (size_t)(sk + 127) / 128;
    Scoped tq(s), tk(s), tv(s);
    ARMAI_TRY(dalloc(tq, (size_t)b * h * nqt * tb));
    ARMAI_TRY(dalloc(tk, (size_t)b * h * nkt * tb));
    ARMAI_TRY(dalloc(tv, (size_t)b * h * nkt * tb));
    ARMAI_TRY(fa_tiles_launch(q, true, h * sq * d, d, sq * d, (int)b, (int)h, (int)sq, (int)d, false, (uint8_t*)tq.p, s));
    ARMAI_TRY(fa_tiles_launch(k, true, h * sk * d, d, sk * d, (int)b, (int)h, (int)sk, (int)d, false, (uint8_t*)tk.p, s));
    ARMAI_TRY(fa_tiles_launch(v, true, h * sk * d, d, sk * d, (int)b, (int)h, (int)sk, (int)d, true, (uint8_t*)tv.p, s));
    FaParams p{};
    p.qt = (const uint8_t*)tq.p;
    p.kt = (const uint8_t*)tk.p;
    p.vt = (const uint8_t*)tv.p;
    p.nqt = (int)nqt;
    p.nkt = (int)nkt;
    p.o = out;
    p.o_bs = h * sq * d;
    p.o_hs = sq * d;
    p.o_ts = d;
    p.sq = (int)sq;
    p.sk = (int)sk;
    p.n_head = (int)h;
    p.group = 1;
    p.scale = scale;
    p.causal = causal;
    return fa_tc_launch(p, (int)d, (int)b, s);
  }
  return launch_flash<__half>(reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(k),
                              reinterpret_cast<const __half*>(v), out, scale, b, h, sq, sk, d, causal,
                              (cudaStream_t)stream);
}

extern "C" int armai_flash_attention_f32(const float* q, size_t q_len, const float* k, size_t k_len,
                                         const float* v, size_t v_len, double scale, size_t b, size_t h,
                                         size_t sq, size_t sk, size_t d, int causal, float* out) {
  if (q_len != b * h * sq * d) return fail(ARMAI_E_INVALID, lenmsg("flash_attn: q", q_len, "B*H*Sq*D", b * h * sq * d));
  if (k_len != b * h * sk * d) return fail(ARMAI_E_INVALID, lenmsg("flash_attn: k", k_len, "B*H*Sk*D", b * h * sk * d));
  if (v_len != b * h * sk * d) return fail(ARMAI_E_INVALID, lenmsg("flash_attn: v", v_len, "B*H*Sk*D", b * h * sk * d));
  if (!q_len) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped dq(s), dk(s), dv(s), dout(s);
  ARMAI_TRY(h2d(dq, q, q_len * 4));
  ARMAI_TRY(h2d(dk, k, k_len * 4));
  ARMAI_TRY(h2d(dv, v, v_len * 4));
  ARMAI_TRY(dalloc(dout, q_len * 4));
  ARMAI_TRY(armai_dev_flash_attention_f32((float*)dq.p, (float*)dk.p, (float*)dv.p, (float*)dout.p,
                                          (float)scale, (int64_t)b, (int64_t)h, (int64_t)sq, (int64_t)sk,
                                          (int64_t)d, causal, s));
  return finish(s, out, dout.p, q_len * 4);
}

extern "C" int armai_dequant_matmul_int8_f32(const float* act, size_t act_len, const int8_t* w, size_t w_len,
                                             const float* scales, size_t scales_len, size_t b, size_t m,
                                             size_t n, size_t k, float* out) {
  if (act_len != b * m * k) return fail(ARMAI_E_INVALID, lenmsg("dequant_matmul_int8: act", act_len, "B*M*K", b * m * k));
  if (w_len != n * k) return fail(ARMAI_E_INVALID, lenmsg("dequant_matmul_int8: weights", w_len, "N*K", n * k));
  if (scales_len != n) return fail(ARMAI_E_INVALID, lenmsg("dequant_matmul_int8: scales", scales_len, "N", n));
  if (!b || !m || !n) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped da(s), dw(s), dsc(s), dout(s);
  ARMAI_TRY(h2d(da, act, act_len * 4));
  ARMAI_TRY(h2d(dw, w, w_len));
  ARMAI_TRY(h2d(dsc, scales, scales_len * 4));
  const int64_t total = (int64_t)(b * m) * (int64_t)n;
  ARMAI_TRY(dalloc(dout, (size_t)total * 4));
  k_dequant_i8<<<(unsigned)((total + 255) / 256), 256, 0, s>>>((float*)da.p, (int8_t*)dw.p, (float*)dsc.p,
                                                               (float*)dout.p, (int64_t)(b * m), (int)n, (int)k);
  ARMAI_CUDA(cudaGetLastError());
  return finish(s, out, dout.p, (size_t)total * 4);
}

extern "C" int armai_dev_int8_matmul_s32(const int8_t* a, const int8_t* w, int32_t* out, int64_t m, int64_t n,
                                         int64_t k, void* stream) {
  if (!m || !n) return ARMAI_OK;
  return launch_int8_gemm(a, w, out, nullptr, nullptr, 0, 0.f, nullptr, m, n, k, (cudaStream_t)stream);
}

extern "C" int armai_dev_int8_matmul_f32(const int8_t* a, const int8_t* w, const float* act_scales, int per_token,
                                         float act_scale, const float* w_scales, float* out, int64_t m, int64_t n,
                                         int64_t k, void* stream) {
  if (!m || !n) return ARMAI_OK;
  return launch_int8_gemm(a, w, nullptr, out, act_scales, per_token, act_scale, w_scales, m, n, k,
                          (cudaStream_t)stream);
}

// ===========================================================================
// LLM helper primitives: rope, softmax, silu(gate) * up, Q6_K dequantisation,
// f16-weight matmul.
// ===========================================================================
extern "C" int armai_dev_rope_f32(const float* x, const int64_t* positions, const float* inv_freq, float* out,
                                  int64_t n_rows, int64_t head_dim, int64_t heads_per_token, void* stream) {
  if (head_dim % 2) return fail(ARMAI_E_INVALID, "rope: head_dim " + std::to_string(head_dim) + " must be even");
  const int64_t pairs = n_rows * (head_dim / 2);
  if (!pairs) return ARMAI_OK;
  if (heads_per_token <= 0) return fail(ARMAI_E_INVALID, "rope: heads_per_token must be positive");
  k_rope<<<(unsigned)((pairs + 255) / 256), 256, 0, (cudaStream_t)stream>>>(x, positions, inv_freq, out, n_rows,
                                                                           (int)(head_dim / 2), heads_per_token);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

extern "C" int armai_rope_f32(const float* input, size_t input_len, const int64_t* positions, size_t n_positions,
                              const float* inv_freq, size_t inv_freq_len, size_t n_rows, size_t head_dim,
                              size_t heads_per_token, float* out) {
  if (input_len != n_rows * head_dim)
    return fail(ARMAI_E_INVALID, lenmsg("rope: input", input_len, "n_rows*head_dim", n_rows * head_dim));
  if (head_dim % 2) return fail(ARMAI_E_INVALID, "rope: head_dim " + std::to_string(head_dim) + " must be even");
  if (inv_freq_len != head_dim / 2)
    return fail(ARMAI_E_INVALID, lenmsg("rope: inv_freq", inv_freq_len, "head_dim/2", head_dim / 2));
  if (n_rows != n_positions * heads_per_token)
    return fail(ARMAI_E_INVALID, "rope: n_rows " + std::to_string(n_rows) + " != n_tokens * heads_per_token = " +
                                     std::to_string(n_positions * heads_per_token));
  if (!input_len) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped dx(s), dp(s), df(s), dout(s);
  ARMAI_TRY(h2d(dx, input, input_len * 4));
  ARMAI_TRY(h2d(dp, positions, n_positions * 8));
  ARMAI_TRY(h2d(df, inv_freq, inv_freq_len * 4));
  ARMAI_TRY(dalloc(dout, input_len * 4));
  ARMAI_TRY(armai_dev_rope_f32((float*)dx.p, (int64_t*)dp.p, (float*)df.p, (float*)dout.p, (int64_t)n_rows,
                               (int64_t)head_dim, (int64_t)heads_per_token, s));
  return finish(s, out, dout.p, input_len * 4);
}

extern "C" int armai_dev_softmax_last_axis_f32(const float* x, float* out, int64_t outer, int64_t inner,
                                               void* stream) {
  if (inner <= 0) return fail(ARMAI_E_INVALID, "softmax: inner must be positive");
  if (!outer) return ARMAI_OK;
  if (outer > 0x7fffffff) return fail(ARMAI_E_INVALID, "softmax: outer exceeds 2^31 - 1 rows");
  const int threads = inner >= 1024 ? 256 : 128;
  k_softmax<<<(unsigned)outer, threads, 0, (cudaStream_t)stream>>>(x, out, (int)inner);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

extern "C" int armai_softmax_last_axis_f32(const float* input, size_t input_len, size_t outer, size_t inner,
                                           float* out) {
  if (inner == 0) return fail(ARMAI_E_INVALID, "softmax: inner must be positive");
  if (input_len != outer * inner)
    return fail(ARMAI_E_INVALID, lenmsg("softmax: input", input_len, "outer*inner", outer * inner));
  if (!outer) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped dx(s), dout(s);
  ARMAI_TRY(h2d(dx, input, input_len * 4));
  ARMAI_TRY(dalloc(dout, input_len * 4));
  ARMAI_TRY(armai_dev_softmax_last_axis_f32((float*)dx.p, (float*)dout.p, (int64_t)outer, (int64_t)inner, s));
  return finish(s, out, dout.p, input_len * 4);
}

extern "C" int armai_dev_silu_gate_mul_up_f32(const float* gate, const float* up, float* out, int64_t n,
                                              void* stream) {
  if (n <= 0) return ARMAI_OK;
  k_silu_gate_mul_up<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(gate, up, out, n);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

extern "C" int armai_silu_gate_mul_up_f32(const float* gate, size_t gate_len, const float* up, size_t up_len,
                                          float* out) {
  if (up_len != gate_len)
    return fail(ARMAI_E_INVALID, "silu_gate_mul_up: up len " + std::to_string(up_len) + " != gate len " +
                                     std::to_string(gate_len));
  if (!gate_len) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped dg(s), du(s), dout(s);
  ARMAI_TRY(h2d(dg, gate, gate_len * 4));
  ARMAI_TRY(h2d(du, up, up_len * 4));
  ARMAI_TRY(dalloc(dout, gate_len * 4));
  ARMAI_TRY(armai_dev_silu_gate_mul_up_f32((float*)dg.p, (float*)du.p, (float*)dout.p, (int64_t)gate_len, s));
  return finish(s, out, dout.p, gate_len * 4);
}

extern "C" int armai_dev_dequantize_q6_k(const uint8_t* in, float* out, int64_t n_blocks, void* stream) {
  if (n_blocks <= 0) return ARMAI_OK;
  const int64_t threads = n_blocks * 64;
  k_dequant_q6k<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(in, out, n_blocks);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

extern "C" int armai_dequantize_q6_k(const uint8_t* input, size_t input_len, size_t n_elements, float* out) {
  const size_t n_blocks = input_len / 210;
  if (n_elements != n_blocks * 256)
    return fail(ARMAI_E_INVALID, "dequantize_q6_k: n_elements " + std::to_string(n_elements) +
                                     " != 256 * blocks = " + std::to_string(n_blocks * 256));
  if (!n_blocks) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped din(s), dout(s);
  ARMAI_TRY(h2d(din, input, n_blocks * 210));
  ARMAI_TRY(dalloc(dout, n_elements * 4));
  ARMAI_TRY(armai_dev_dequantize_q6_k((uint8_t*)din.p, (float*)dout.p, (int64_t)n_blocks, s));
  return finish(s, out, dout.p, n_elements * 4);
}

extern "C" int armai_dev_dequant_matmul_f16_f32(const float* act, const uint16_t* w, float* out, int64_t rows,
                                                int64_t n, int64_t k, void* stream) {
  if (rows <= 0 || n <= 0) return ARMAI_OK;
  if (n > 0x7fffffff || k > 0x7fffffff) return fail(ARMAI_E_INVALID, "dequant_matmul_f16: N or K too large");
  const cudaStream_t s = (cudaStream_t)stream;
  if (rows <= 4) {  // decode: one activation row group, 256 weight rows per CTA
    const dim3 grid((unsigned)((n + 255) / 256), 1);
    k_dequant_f16<8><<<grid, 256, 0, s>>>(act, w, out, rows, (int)n, (int)k);
  } else {
    const dim3 grid((unsigned)((n + 31) / 32), (unsigned)((rows + 31) / 32));
    k_dequant_f16<1><<<grid, 256, 0, s>>>(act, w, out, rows, (int)n, (int)k);
  }
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

extern "C" int armai_dequant_matmul_f16_f32(const float* act, size_t act_len, const uint16_t* weights,
                                            size_t weights_len, size_t b, size_t m, size_t n, size_t k,
                                            float* out) {
  if (act_len != b * m * k) return fail(ARMAI_E_INVALID, lenmsg("dequant_matmul_f16: act", act_len, "B*M*K", b * m * k));
  if (weights_len != n * k)
    return fail(ARMAI_E_INVALID, lenmsg("dequant_matmul_f16: weights", weights_len, "N*K", n * k));
  const size_t rows = b * m;
  if (!rows || !n) return ARMAI_OK;
  cudaStream_t s;
  ARMAI_TRY(thread_stream(&s));
  Scoped da(s), dw(s), dout(s);
  ARMAI_TRY(h2d(da, act, act_len * 4));
  ARMAI_TRY(h2d(dw, weights, weights_len * 2));
  ARMAI_TRY(dalloc(dout, rows * n * 4));
  ARMAI_TRY(armai_dev_dequant_matmul_f16_f32((float*)da.p, (uint16_t*)dw.p, (float*)dout.p, (int64_t)rows,
                                             (int64_t)n, (int64_t)k, s));
  return finish(s, out, dout.p, rows * n * 4);
}
