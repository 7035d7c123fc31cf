// i8gemm_tc.cu — s8 x s8 -> s32 GEMM on the 5th-generation tensor cores, for
// the int8 matmul primitives (reference native/arm_ai_nif/src/shape_ops.rs:
// int8_matmul_f32 :1169-1211, _per_token :1222-1264, int8_dot :1294-1370)
// at M >= 64:
//
//   acc[m][n] = sum_k a[m][k] * w[n][k]          (exact, s32 in tensor memory)
//   out_s32[m][n] = acc, or
//   out_f32[m][n] = ((float)acc * act_scale(m)) * w_scales[n]   (the
//                    reference's `(acc as f32) * act_scale * w_scales[j]`)
//
// A and W stay row-major (K-major) in global memory. Per 128 x 128 output
// tile and K stage of 128 bytes, one thread brings a 128 x 128-byte box of
// each with a TMA load (tensor maps with the 128-byte swizzle, boxes past
// the edges zero-filled, no multicast), one thread issues four
// tcgen05.mma.cta_group::1.kind::i8 (K = 32 each) into a 128-column s32
// accumulator in tensor memory, and four warps read it back with
// tcgen05.ld for the epilogue. 4-stage ring on full/empty mbarriers; every
// wait is bounded and sets the error word; tensor memory is always freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "common.cuh"
#include "kquant.cuh"
#include "llama_kernels.cuh"

namespace armai {

constexpr int IG_M = 128, IG_N = 128;
constexpr int IG_KB = 128;      // K bytes (= int8 values) per stage
constexpr int IG_STAGES = 4;
constexpr int IG_THREADS = 192;
constexpr uint32_t IG_TILE = 128u * 128u;  // one operand box (16 KB)
constexpr uint32_t IG_SMEM = 1024 + IG_STAGES * 2 * IG_TILE + 256;

struct IgParams {
  int m, n, k;
  int32_t* out_s32;
  float* out_f32;
  const float* act_scales;  // per_token: [m]
  int per_token;
  float act_scale;
  const float* w_scales;    // [n]
  uint32_t* err;
};

__device__ __forceinline__ void ig_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void ig_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand, 128-byte swizzle: 128-byte rows, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t ig_smem_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
  d |= (uint64_t)1u << 16;                  // leading byte offset (unused with this swizzle)
  d |= (uint64_t)(1024u >> 4) << 32;        // stride byte offset: next 8-row group
  d |= (uint64_t)1u << 46;                  // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                  // 128-byte swizzle
  return d;
}

// kind::i8 instruction descriptor: s8 A and B (K-major), s32 D, M = N = 128.
__host__ __device__ constexpr uint32_t ig_instr_desc() {
  return (2u << 4)                  // D format s32
         | (1u << 7) | (1u << 10)   // A, B signed 8-bit
         | ((uint32_t)(IG_N >> 3) << 17) | ((uint32_t)(IG_M >> 4) << 24);
}

__device__ __forceinline__ void ig_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void ig_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 2-D TMA load of box (x = K byte offset, y = row) into shared memory,
// completing on `bar` (no multicast).
__device__ __forceinline__ void ig_tma_load(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ bool ig_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
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

__device__ __forceinline__ void ig_tmem_ld16(uint32_t taddr, int32_t (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = (int32_t)r[i];
}

__global__ void __launch_bounds__(IG_THREADS, 1) k_i8gemm(const __grid_constant__ CUtensorMap ta,
                                                          const __grid_constant__ CUtensorMap tw, const IgParams p) {
  extern __shared__ uint8_t ig_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t raw_addr = smem_u32(ig_raw);
  uint8_t* smem = ig_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);  // swizzle atoms repeat every 1024 B
  uint8_t* a_st = smem;
  uint8_t* b_st = smem + IG_STAGES * IG_TILE;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * IG_STAGES * IG_TILE);
  uint64_t* empty = full + IG_STAGES;
  uint64_t* accb = empty + IG_STAGES;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accb + 1);

  const int n0 = blockIdx.x * IG_N, m0 = blockIdx.y * IG_M;
  const int nk = (p.k + IG_KB - 1) / IG_KB;
  if (tid == 0) {
    for (int s = 0; s < IG_STAGES; s++) {
      mbar_init(&full[s], 1);   // the TMA thread's expect_tx arrival + the boxes' bytes
      mbar_init(&empty[s], 1);  // tcgen05.commit after the stage's MMAs
    }
    mbar_init(accb, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(IG_N)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  ig_fence_before();
  __syncthreads();
  ig_fence_after();
  const uint32_t taddr = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int kc = 0; kc < nk; kc++) {
        const int s = kc % IG_STAGES;
        if (kc >= IG_STAGES && !ig_wait(&empty[s], (uint32_t)((kc / IG_STAGES - 1) & 1), p.err)) break;
        mbar_expect_tx(&full[s], 2 * IG_TILE);
        ig_tma_load(a_st + s * IG_TILE, &ta, kc * IG_KB, m0, &full[s]);
        ig_tma_load(b_st + s * IG_TILE, &tw, kc * IG_KB, n0, &full[s]);
        issued = kc + 1;
      }
      // every box this thread requested has landed before the CTA may exit
      for (int kc = issued > IG_STAGES ? issued - IG_STAGES : 0; kc < issued; kc++)
        ig_wait(&full[kc % IG_STAGES], (uint32_t)((kc / IG_STAGES) & 1), p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = ig_instr_desc();
      for (int kc = 0; kc < nk; kc++) {
        const int s = kc % IG_STAGES;
        if (!ig_wait(&full[s], (uint32_t)((kc / IG_STAGES) & 1), p.err)) break;
        ig_fence_after();
        const uint32_t a0 = smem_u32(a_st + s * IG_TILE), b0 = smem_u32(b_st + s * IG_TILE);
#pragma unroll
        for (int kk = 0; kk < IG_KB / 32; kk++)  // K = 32 int8 per MMA: 32 bytes along the swizzled row
          ig_mma(taddr, ig_smem_desc(a0 + 32 * kk), ig_smem_desc(b0 + 32 * kk), idesc, (kc | kk) != 0);
        ig_commit(&empty[s]);
      }
      ig_commit(accb);  // also after an early exit: completes once the issued MMAs have
    }
    __syncwarp();
  } else {
    // epilogue: warp w reads tensor-memory lanes 32 (w % 4) .. + 31 = rows
    const bool ok = ig_wait(accb, 0, p.err);
    ig_fence_after();
    const int q = warp & 3;
    const int m = m0 + 32 * q + lane;
    const float as = (m < p.m && p.out_f32) ? (p.per_token ? p.act_scales[m] : p.act_scale) : 0.f;
    if (ok) {
#pragma unroll 1
      for (int c0 = 0; c0 < IG_N; c0 += 16) {
        int32_t v[16];
        ig_tmem_ld16(taddr + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
        if (m >= p.m) continue;
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int n = n0 + c0 + i;
          if (n >= p.n) break;
          const size_t o = (size_t)m * p.n + n;
          if (p.out_s32) p.out_s32[o] = v[i];
          if (p.out_f32) p.out_f32[o] = __fmul_rn(__fmul_rn((float)v[i], as), p.w_scales[n]);
        }
      }
    }
  }
  ig_fence_before();
  __syncthreads();
  if (warp == 1) {
    ig_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(IG_N) : "memory");
  }
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// Row-major [rows][k] int8 matrix as a 2-D tensor map with 128 x 128-byte
// boxes and the 128-byte swizzle.
int make_map(CUtensorMap* map, const int8_t* base, int64_t rows, int64_t k) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(ARMAI_E_CUDA, "int8_matmul: cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)k};
  const cuuint32_t box[2] = {(cuuint32_t)IG_KB, (cuuint32_t)IG_M};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(ARMAI_E_CUDA, "int8_matmul: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return ARMAI_OK;
}

}  // namespace

// Device error word of this kernel's bounded waits (one per device that
// loads the library); read and cleared by int8_gemm_tc_check.
static __device__ uint32_t g_ig_err;

// The tensor-core path of launch_int8_gemm (prims.cu): K % 16 == 0 (TMA row
// strides are multiples of 16 bytes), a and w 16-byte aligned.
int launch_int8_gemm_tc(const int8_t* a, const int8_t* w, int32_t* o32, float* of32, const float* act_scales,
                        int per_token, float act_scale, const float* w_scales, int64_t m, int64_t n, int64_t k,
                        cudaStream_t s) {
  uint32_t* err = nullptr;
  ARMAI_CUDA(cudaGetSymbolAddress((void**)&err, g_ig_err));
  CUtensorMap ta, tw;
  ARMAI_TRY(make_map(&ta, a, m, k));
  ARMAI_TRY(make_map(&tw, w, n, k));
  static thread_local int attr_dev = -1;
  int dev = 0;
  ARMAI_CUDA(cudaGetDevice(&dev));
  if (attr_dev != dev) {
    ARMAI_CUDA(cudaFuncSetAttribute(k_i8gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)IG_SMEM));
    attr_dev = dev;
  }
  IgParams p{(int)m, (int)n, (int)k, o32, of32, act_scales, per_token, act_scale, w_scales, err};
  const dim3 grid((unsigned)((n + IG_N - 1) / IG_N), (unsigned)((m + IG_M - 1) / IG_M));
  k_i8gemm<<<grid, IG_THREADS, IG_SMEM, s>>>(ta, tw, p);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

// After the stream's work is done: ARMAI_E_DEVICE (and the word cleared) if a
// wait of the kernel gave up.
int int8_gemm_tc_check() {
  uint32_t e = 0;
  ARMAI_CUDA(cudaMemcpyFromSymbol(&e, g_ig_err, sizeof e));
  if (!e) return ARMAI_OK;
  const uint32_t zero = 0;
  ARMAI_CUDA(cudaMemcpyToSymbol(g_ig_err, &zero, sizeof zero));
  return fail(ARMAI_E_DEVICE, "int8_matmul: a wait of the tensor-core kernel gave up (error word " +
                                  std::to_string(e) + ")");
}

}  // namespace armai
