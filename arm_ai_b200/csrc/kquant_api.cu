// kquant_api.cu — C-ABI access to the k-quant device building blocks, for
// bit-exact parity tests: Q8_K quantisation, per-super-block integer dot
// products, and QMatMul through the decode / prefill matvec kernels.
#include <cstring>
#include <vector>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "llama_kernels.cuh"

using namespace armai;

namespace {

// One warp per (row, 256-block): Q8_K quantisation into BlockQ8K structs.
// The warp quantises into 8-byte-aligned scratch (the packed 292-byte
// structs only guarantee 4-byte alignment of `qs`), then copies out with
// 4-byte stores.
__global__ void k_quant_q8k(const float* x, int64_t m, int K, BlockQ8K* out, int8_t* scratch_qs,
                            int32_t* scratch_bs) {
  const int lane = threadIdx.x & 31;
  const int64_t job = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nb = K / QK_K;
  if (job >= m * nb) return;
  const int64_t row = job / nb;
  const int j = (int)(job % nb);
  const float* src = x + row * K + j * QK_K + 8 * lane;
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; i++) v[i] = src[i];
  BlockQ8K* b = out + job;
  int8_t* qs = scratch_qs + job * QK_K;
  int32_t* bs = scratch_bs + job * 16;
  q8k_quant_block_warp(v, lane, qs, &b->d, bs);
  __syncwarp();
  const uint32_t* qw = reinterpret_cast<const uint32_t*>(qs);
  uint32_t* dst = reinterpret_cast<uint32_t*>(b->qs);
  dst[2 * lane] = qw[2 * lane];
  dst[2 * lane + 1] = qw[2 * lane + 1];
  if (lane < 16) b->bsums[lane] = (int16_t)bs[lane];
}

// BlockQ8K structs -> the split ActQ8 layout the kernels read (qs chunks
// swizzled by block index, as load_slice expects). `nb` = blocks per row.
__global__ void k_q8k_split(const BlockQ8K* in, int64_t nblocks, int nb, int8_t* qs, float* d, int32_t* bs) {
  const int64_t b = blockIdx.x;
  if (b >= nblocks) return;
  const int swz = (int)(b % nb) & 7;
  for (int i = threadIdx.x; i < QK_K; i += blockDim.x)
    qs[b * QK_K + (((i >> 4) ^ swz) << 4) + (i & 15)] = in[b].qs[i];
  if (threadIdx.x < 16) bs[b * 16 + threadIdx.x] = in[b].bsums[threadIdx.x];
  if (threadIdx.x == 0) d[b] = in[b].d;
}

// Per-(token, row, super-block) integers through load_slice + q4k_quarter /
// q6k_quarter, the exact code of the matvec kernels' inner loop (four lanes
// per super-block, their quarter integers summed).
__global__ void k_block_dots(const uint8_t* w, int type, int rows, int nb, int row_bytes,
                             const int8_t* qs, const float* dq, const int32_t* bs, int m,
                             int32_t* isum, int32_t* msum) {
  const int lane = threadIdx.x & 31;
  const int64_t job = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t groups = (nb + 7) / 8;
  if (job >= (int64_t)m * rows * groups) return;
  const int t = (int)(job / ((int64_t)rows * groups));
  const int r = (int)((job / groups) % rows);
  const int b = (int)(job % groups) * 8 + (lane >> 2);
  const int u = lane & 3;
  int is = 0, ms = 0;
  if (b < nb) {
    const uint8_t* row = w + (int64_t)r * row_bytes;
    ActQ8 a;
    a.qs = const_cast<int8_t*>(qs) + (int64_t)t * nb * QK_K;
    a.d = const_cast<float*>(dq) + (int64_t)t * nb;
    a.bs = const_cast<int32_t*>(bs) + (int64_t)t * nb * 16;
    ActSlice A;
    load_slice(a, b, u, A);
    if (type == GGML_Q4_K) {
      float dx, dmx;
      q4k_quarter(row + (int64_t)b * Q4K_BLOCK_BYTES, u, A, is, ms, dx, dmx);
    } else {
      is = q6k_quarter(row + (int64_t)b * Q6K_BODY_BYTES, u, A);
    }
  }
  is += __shfl_xor_sync(0xffffffffu, is, 1);
  is += __shfl_xor_sync(0xffffffffu, is, 2);
  ms += __shfl_xor_sync(0xffffffffu, ms, 1);
  ms += __shfl_xor_sync(0xffffffffu, ms, 2);
  if (u == 0 && b < nb) {
    const int64_t o = ((int64_t)t * rows + r) * nb + b;
    isum[o] = is;
    if (msum) msum[o] = ms;
  }
}

struct DevBuf {
  void* p = nullptr;
  ~DevBuf() { if (p) cudaFree(p); }
};

int upload_weights(const void* w, int type, size_t n, size_t k, DevBuf& dw, int& row_bytes) {
  if (type != GGML_Q4_K && type != GGML_Q6_K) return fail(ARMAI_E_INVALID, "unsupported weight type");
  if (k % QK_K) return fail(ARMAI_E_INVALID, "k must be a multiple of 256");
  row_bytes = (int)dev_row_bytes(type, (int64_t)k);
  std::vector<uint8_t> host;
  const uint8_t* src = (const uint8_t*)w;
  if (type == GGML_Q6_K) {
    host.resize((size_t)row_bytes * n);
    repack_q6k_rows(src, (int64_t)n, (int64_t)k, host.data());
    src = host.data();
  }
  ARMAI_CUDA(cudaMalloc(&dw.p, (size_t)row_bytes * n));
  ARMAI_CUDA(cudaMemcpy(dw.p, src, (size_t)row_bytes * n, cudaMemcpyHostToDevice));
  return ARMAI_OK;
}

}  // namespace

extern "C" int armai_quantize_q8k(const float* x, size_t m, size_t k, void* out) {
  if (!x || !out) return fail(ARMAI_E_INVALID, "quantize_q8k: null argument");
  if (k % QK_K) return fail(ARMAI_E_INVALID, "quantize_row_q8k: k is not divisible by 256");
  if (m == 0) return ARMAI_OK;
  const int64_t nblk = (int64_t)m * (k / QK_K);
  DevBuf dx, dout, dbs, dqs;
  ARMAI_CUDA(cudaMalloc(&dx.p, m * k * 4));
  ARMAI_CUDA(cudaMalloc(&dout.p, nblk * sizeof(BlockQ8K)));
  ARMAI_CUDA(cudaMalloc(&dbs.p, nblk * 16 * 4));
  ARMAI_CUDA(cudaMalloc(&dqs.p, nblk * QK_K));
  ARMAI_CUDA(cudaMemcpy(dx.p, x, m * k * 4, cudaMemcpyHostToDevice));
  const int wpb = 8;
  k_quant_q8k<<<(unsigned)((nblk + wpb - 1) / wpb), wpb * 32>>>((const float*)dx.p, (int64_t)m, (int)k,
                                                                 (BlockQ8K*)dout.p, (int8_t*)dqs.p, (int32_t*)dbs.p);
  ARMAI_CUDA(cudaGetLastError());
  ARMAI_CUDA(cudaMemcpy(out, dout.p, nblk * sizeof(BlockQ8K), cudaMemcpyDeviceToHost));
  return ARMAI_OK;
}

extern "C" int armai_kquant_block_dots(const void* w, int type, size_t n, size_t k, const void* q8,
                                       size_t m, int32_t* isum, int32_t* msum) {
  if (!w || !q8 || !isum) return fail(ARMAI_E_INVALID, "kquant_block_dots: null argument");
  DevBuf dw, dq, dqs, dd, dbs, di, dm;
  int rb = 0;
  ARMAI_TRY(upload_weights(w, type, n, k, dw, rb));
  const int nb = (int)(k / QK_K);
  const int64_t nblk = (int64_t)m * nb;
  ARMAI_CUDA(cudaMalloc(&dq.p, nblk * sizeof(BlockQ8K)));
  ARMAI_CUDA(cudaMemcpy(dq.p, q8, nblk * sizeof(BlockQ8K), cudaMemcpyHostToDevice));
  ARMAI_CUDA(cudaMalloc(&dqs.p, nblk * QK_K));
  ARMAI_CUDA(cudaMalloc(&dd.p, nblk * 4));
  ARMAI_CUDA(cudaMalloc(&dbs.p, nblk * 16 * 4));
  k_q8k_split<<<(unsigned)nblk, 256>>>((const BlockQ8K*)dq.p, nblk, nb, (int8_t*)dqs.p, (float*)dd.p,
                                       (int32_t*)dbs.p);
  const size_t outn = (size_t)m * n * nb;
  ARMAI_CUDA(cudaMalloc(&di.p, outn * 4));
  ARMAI_CUDA(cudaMalloc(&dm.p, outn * 4));
  const int64_t jobs = (int64_t)m * n * ((nb + 7) / 8);
  k_block_dots<<<(unsigned)((jobs + 7) / 8), 256>>>((const uint8_t*)dw.p, type, (int)n, nb, rb,
                                                    (const int8_t*)dqs.p, (const float*)dd.p, (const int32_t*)dbs.p,
                                                    (int)m, (int32_t*)di.p,
                                                    type == GGML_Q4_K ? (int32_t*)dm.p : nullptr);
  ARMAI_CUDA(cudaGetLastError());
  ARMAI_CUDA(cudaMemcpy(isum, di.p, outn * 4, cudaMemcpyDeviceToHost));
  if (msum && type == GGML_Q4_K) ARMAI_CUDA(cudaMemcpy(msum, dm.p, outn * 4, cudaMemcpyDeviceToHost));
  return ARMAI_OK;
}

namespace {
template <int NB>
int qmm_launch(const uint8_t* w, int type, int n, int k, int rb, const float* x, float* out,
               uint32_t* err) {
  MvParams p;
  std::memset(&p, 0, sizeof p);
  const int nsm = sm_count();
  int per = (n + nsm - 1) / nsm;
  const size_t act = mv_smem_layout(0, 0, k, NB, false).total;
  int chunk = (int)std::min<size_t>((size_t)per, (size_t)(44 * 1024) / (size_t)rb);
  if (chunk < 1) chunk = 1;
  const uint32_t stage = (uint32_t)al16((size_t)chunk * rb);
  int ns = std::min(3, (per + chunk - 1) / chunk);
  while (ns > 1 && act + (size_t)ns * stage + 1024 > 227 * 1024) ns--;
  const size_t smem = mv_smem_layout(ns, stage, k, NB, false).total;
  if (smem > 227 * 1024) return fail(ARMAI_E_INVALID, "qmatmul: rows too wide for shared memory");
  p.x = x;
  p.K = k;
  p.nb = k / QK_K;
  p.seg[0] = Seg{w, type, n, k / QK_K, rb};
  p.nseg = 1;
  p.acts = is_legacy(type) ? 2 : 1;
  p.total_rows = n;
  p.nrows = NB;
  p.rows_per_cta = per;
  p.chunk_rows = chunk;
  p.ns = ns;
  p.stage_bytes = stage;
  p.out = out;
  p.out_stride = n;
  p.err = err;
  ARMAI_CUDA(cudaFuncSetAttribute(k_matvec<MODE_STORE, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_matvec<MODE_STORE, NB><<<(n + per - 1) / per, MV_THREADS, smem>>>(p);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}
}  // namespace

extern "C" int armai_qmatmul(const void* w, int type, size_t n, size_t k, const float* x, size_t m,
                             float* out) {
  if (!w || !x || !out) return fail(ARMAI_E_INVALID, "qmatmul: null argument");
  DevBuf dw, dx, dout, derr;
  int rb = 0;
  ARMAI_TRY(upload_weights(w, type, n, k, dw, rb));
  ARMAI_CUDA(cudaMalloc(&dx.p, m * k * 4));
  ARMAI_CUDA(cudaMalloc(&dout.p, m * n * 4));
  ARMAI_CUDA(cudaMalloc(&derr.p, 4));
  ARMAI_CUDA(cudaMemset(derr.p, 0, 4));
  ARMAI_CUDA(cudaMemcpy(dx.p, x, m * k * 4, cudaMemcpyHostToDevice));
  size_t t = 0;
  for (; t + 8 <= m; t += 8)
    ARMAI_TRY(qmm_launch<8>((const uint8_t*)dw.p, type, (int)n, (int)k, rb, (const float*)dx.p + t * k,
                            (float*)dout.p + t * n, (uint32_t*)derr.p));
  for (; t < m; t++)
    ARMAI_TRY(qmm_launch<1>((const uint8_t*)dw.p, type, (int)n, (int)k, rb, (const float*)dx.p + t * k,
                            (float*)dout.p + t * n, (uint32_t*)derr.p));
  uint32_t herr = 0;
  ARMAI_CUDA(cudaMemcpy(&herr, derr.p, 4, cudaMemcpyDeviceToHost));
  if (herr) return fail(ARMAI_E_DEVICE, "qmatmul: device error flag set");
  ARMAI_CUDA(cudaMemcpy(out, dout.p, m * n * 4, cudaMemcpyDeviceToHost));
  return ARMAI_OK;
}

extern "C" int armai_qgemm(const void* w, int type, size_t n, size_t k, const float* x, size_t m,
                           const float* gamma, float eps, float* out) {
  if (!w || !x || !out) return fail(ARMAI_E_INVALID, "qgemm: null argument");
  if (k % QK_K || k > 16384) return fail(ARMAI_E_INVALID, "qgemm: K must be a multiple of 256, at most 16384");
  if (!m || !n) return ARMAI_OK;
  DevBuf dw, dx, dg, da, dout, derr;
  int rb = 0;
  ARMAI_TRY(upload_weights(w, type, n, k, dw, rb));
  ARMAI_CUDA(cudaMalloc(&dx.p, m * k * 4));
  ARMAI_CUDA(cudaMemcpy(dx.p, x, m * k * 4, cudaMemcpyHostToDevice));
  if (gamma) {
    ARMAI_CUDA(cudaMalloc(&dg.p, k * 4));
    ARMAI_CUDA(cudaMemcpy(dg.p, gamma, k * 4, cudaMemcpyHostToDevice));
  }
  ARMAI_CUDA(cudaMalloc(&da.p, qgemm_a_bytes((int)m, (int)k)));
  ARMAI_CUDA(cudaMalloc(&dout.p, m * n * 4));
  ARMAI_CUDA(cudaMalloc(&derr.p, 4));
  ARMAI_CUDA(cudaMemset(derr.p, 0, 4));
  // split-K partials: up to 8 splits
  const size_t ws_floats = 8 * m * n;
  DevBuf dws;
  ARMAI_CUDA(cudaMalloc(&dws.p, ws_floats * 4));
  ARMAI_TRY(qgemm_act_launch((const float*)dx.p, (const float*)dg.p, eps, (int)m, (int)k, (uint8_t*)da.p, 0));
  QgJob j;
  std::memset(&j, 0, sizeof j);
  j.a_tiles = (const uint8_t*)da.p;
  j.m = (int)m;
  j.k = (int)k;
  j.seg[0] = QgSeg{(const uint8_t*)dw.p, type, (int)n, rb};
  j.nseg = 1;
  j.mode = QG_STORE;
  j.dst = (float*)dout.p;
  j.ldd = (int)n;
  j.ws = (float*)dws.p;
  j.ws_floats = ws_floats;
  j.err = (uint32_t*)derr.p;
  ARMAI_TRY(qgemm_run(j, 0));
  uint32_t herr = 0;
  ARMAI_CUDA(cudaMemcpy(&herr, derr.p, 4, cudaMemcpyDeviceToHost));
  if (herr) return fail(ARMAI_E_DEVICE, "qgemm: device error flag set");
  ARMAI_CUDA(cudaMemcpy(out, dout.p, m * n * 4, cudaMemcpyDeviceToHost));
  return ARMAI_OK;
}
