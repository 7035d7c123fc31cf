// gemm_tc.cuh — prefill GEMM on the 5th-generation tensor cores (sm_100a).
//
// out[m][n] = sum_k A[m][k] * W[n][k] for a block of prompt tokens (m) and
// the rows (n) of up to three GGUF weight matrices (Q4_K / Q6_K):
//   * A: each token's activation row, optionally rms-normalised, quantised to
//     Q8_K exactly as BlockQ8K::from_float (candle-core 0.8.4 k_quants.rs,
//     called from QMatMul for every forward, native/arm_ai_nif/src/
//     llama_candle.rs:92-94), then expanded to f16 q * d — written by
//     k_qgemm_act into 128 x 64 tiles in the tensor cores' 128-byte-swizzled
//     K-major layout, so one bulk copy brings a tile into shared memory.
//   * W: dequantised in shared memory by the CTA's own warps from the raw
//     super-blocks (BlockQ4K / BlockQ6K::to_float), rounded to f16, written
//     into the same swizzled layout.
//   * tcgen05.mma (kind::f16, f32 accumulate) issued by one thread, the
//     128 x 128 f32 accumulator in tensor memory, read back with tcgen05.ld.
// Relative to candle's integer Q8_K dots the only differences are the f16
// rounding of the dequantised weights and of q * d (2^-11 relative) and the
// f32 summation order.
//
// Roles (192 threads): warp 0 lane 0 streams A tiles (cp.async.bulk), warp 1
// allocates tensor memory and one lane issues the MMAs, warps 2-5 dequantise
// W (thread = weight row) and then run the epilogue (warp w reads tensor
// memory lanes 32 * (w % 4) .. + 31, i.e. tokens). Every wait is bounded and
// sets an error flag; tensor memory is always released.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include <cuda_runtime.h>

#include "common.cuh"

namespace armai {

constexpr int QG_M = 128;                 // tokens per tile (tensor-memory lanes)
constexpr int QG_N = 128;                 // weight rows per tile (accumulator columns)
constexpr int QG_K = 64;                  // K per stage: one 128-byte row of f16
constexpr int QG_STAGES = 4;
constexpr int QG_THREADS = 192;
constexpr uint32_t QG_TILE_BYTES = 128u * 128u;          // one operand tile (16 KB)
constexpr uint32_t QG_SMEM = 1024 + QG_STAGES * 2 * QG_TILE_BYTES + 256;

struct QgSeg {
  const uint8_t* w;
  int type, rows, row_bytes;
};

struct QgParams {
  const uint8_t* a_tiles;  // [m_tiles][k / 64][128 rows][128 B], swizzled
  int m, n, k;             // tokens, weight rows (all segments), K
  QgSeg seg[3];
  int nseg;
  float* out;              // out[m][ldo]; tile columns land at n0 ..
  int ldo;
  uint32_t* err;
};

// Bytes of the A-tile buffer for m tokens and K.
inline size_t qgemm_a_bytes(int m, int k) {
  return (size_t)((m + QG_M - 1) / QG_M) * (size_t)(k / QG_K) * QG_TILE_BYTES;
}
// A operand of m token rows x[m][k] (rms-normalised with gamma when gamma is
// not null) into a_tiles (qgemm_a_bytes(m, k) bytes). K % 256 == 0, K <= 16384.
int qgemm_act_launch(const float* x, const float* gamma, float eps, int m, int k, uint8_t* a_tiles,
                     cudaStream_t s);
// out[m][n] (row stride ldo) = A x W^T over the segments of p; p.a_tiles from
// qgemm_act_launch. Sets the kernel's shared-memory limit on first use.
int qgemm_launch(const QgParams& p, cudaStream_t s);

// Prefill epilogues on the GEMM output g (row stride ldg), t = 0..S-1:
// q|k|v rows -> RoPE'd q into q_out[t][QN], RoPE'd k and v into the KV cache
// of the sequence (positions pos[t]), as the matvec QKV epilogue does.
int qkv_post_launch(const float* g, int ldg, int S, const int* pos, int qn, int kn, int hd, int max_seq,
                    const float* cos_t, const float* sin_t, float* q_out, void* kc, void* vc, int kv_f16,
                    cudaStream_t s);
// x[t][i] += g[t][i] (residual), i < n.
int resid_add_launch(float* x, const float* g, int S, int n, int ldg, cudaStream_t s);
// h[t][i] = silu(g[t][i]) * g[t][n + i] (candle: v / (1 + exp(-v)), then * up).
int silu_mul_launch(const float* g, int S, int n, float* h, cudaStream_t s);

}  // namespace armai
