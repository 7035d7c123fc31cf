// gemm_tc.cuh — quantised-weight GEMM on the 5th-generation tensor cores
// (sm_100a), for prompts (prefill) and batched decode.
//
// out[t][n] = sum_k X[t][k] * W[n][k] for a block of tokens (t) and the rows
// (n) of up to three GGUF weight matrices (Q4_K / Q6_K), computed as
// D = W X^T: weights are the MMA's M side (128 rows per tile), tokens its N
// side (16 .. 256 per tile), so one dequantised weight tile serves up to 256
// tokens and a decode batch of 16 wastes no tensor-core rows.
//   * X: each token's activation row, optionally rms-normalised, quantised to
//     Q8_K exactly as BlockQ8K::from_float (candle-core 0.8.4 k_quants.rs,
//     called from QMatMul for every forward, native/arm_ai_nif/src/
//     llama_candle.rs:92-94), then expanded to f16 q * d — written by the row
//     kernels into 128-token x 64-K tiles in the tensor cores'
//     128-byte-swizzled K-major layout; a bulk copy brings the tile's first
//     16 .. 128 token rows (or two whole tiles) into shared memory as the MMA
//     B operand.
//   * W: raw super-blocks streamed into shared memory by TMA (32-row boxes of
//     one super-block per segment, a 2-slot ring), dequantised by 8 or 16
//     warps (BlockQ4K / BlockQ6K::to_float; one thread per weight row and 32
//     or 16 K values per stage) straight into tensor memory as f16 — the A
//     operand — so the weights never pass through shared memory as f16.
//   * tcgen05.mma (kind::f16, f32 accumulate) issued by one thread; the
//     128-row x tokens f32 accumulator in tensor memory, read back with
//     tcgen05.ld (lane = weight row, column = token).
//   * Split K: with few tiles (short prompts, decode batches) the super-blocks
//     are split over gridDim.z CTAs; partial sums go to a workspace and the
//     consumer adds them in split order (deterministic): k_qg_finish, or a
//     fused row kernel (residual add + norm + next activation tiles, SiLU +
//     activation tiles, or RoPE + KV-cache store).
// Relative to candle's integer Q8_K dots the only differences are the f16
// rounding of the dequantised weights and of q * d (2^-11 relative) and the
// f32 summation order.
//
// Roles (32 x (3 + DW) threads, DW = 8 dequantising warps for up to 64
// tokens per tile, 16 above): warp 0 lane 0 streams token tiles
// (cp.async.bulk), warp 1 allocates tensor memory and one lane issues the
// MMAs, warp 2 lane 0 streams raw weight super-blocks (TMA), warps 3 ..
// 2 + DW dequantise (warp w owns tensor-memory lanes 32 * (w % 4) .. + 31 and
// K part (w - 3) / 4 of each stage) and then run the epilogue (every
// (DW / 4)-th group of 8 tokens). Every wait is bounded and sets an error
// flag; tensor memory is always released.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace armai {

constexpr int QG_W = 128;                 // weight rows per tile (MMA M, tensor-memory lanes)
constexpr int QG_K = 64;                  // K per stage: one 128-byte row of f16
constexpr int QG_STAGES = 4;
constexpr int QG_TOK_MAX = 256;           // tokens per tile (MMA N; 16 .. 128 in steps of 16, or 256)
constexpr uint32_t QG_TILE_BYTES = 128u * 128u;          // one 128-token x 64-K activation tile (16 KB)
// Raw weight super-blocks in shared memory: per slot four 32-row groups of
// one super-block each (Q4_K 144 B, Q6_K body 208 B per row)
constexpr int QG_RAW_SLOTS = 2;
constexpr uint32_t QG_RAW_GROUP_BYTES = 32u * 208u;
constexpr uint32_t QG_RAW_SLOT_BYTES = 4u * QG_RAW_GROUP_BYTES;
inline uint32_t qg_smem_bytes(int ntok) {
  return 1024 + QG_STAGES * (uint32_t)ntok * 128u + QG_RAW_SLOTS * QG_RAW_SLOT_BYTES + 256;
}

struct QgSeg {
  const uint8_t* w;
  int type, rows, row_bytes;
};

// Tensor maps of the segments' raw weight rows ([rows][row_bytes] bytes,
// boxes of 32 rows x one super-block), built by qgemm_run.
struct alignas(64) QgMaps {
  CUtensorMap m[3];
};

// Kernel parameters (filled by qgemm_run).
struct QgParams {
  const uint8_t* a_tiles;  // [token tiles of 128][k / 64][128 rows][128 B], swizzled
  int m, n, k;             // tokens, weight rows (all segments), K
  QgSeg seg[3];
  int nseg;
  int ntok;                // tokens per CTA tile
  int kb_split;            // super-blocks per split (gridDim.z splits)
  int acc_cols, tmem_cols; // accumulator columns; tensor-memory allocation
  int add;                 // 1: out += result (one split only)
  float* out;              // out[t][ldo] (+ blockIdx.z * split_stride)
  int ldo;
  size_t split_stride;
  uint32_t* err;
};

enum QgMode { QG_STORE = 0, QG_RESID = 1, QG_SILU = 2, QG_PARTIAL = 3 };

// One weight GEMM and its consumer.
//   QG_STORE  : dst[t][j] = (X W^T)[t][j], j < n (row stride ldd)
//   QG_RESID  : dst[t][j] += (X W^T)[t][j]
//   QG_SILU   : segments gate | up of F rows each; dst[t][i] =
//               silu(gate_i) * up_i (candle: v / (1 + exp(-v)), then * up)
//   QG_PARTIAL: the split partial sums stay in ws (QgSplit says where) for a
//               fused consumer (qkv_post_launch, resid_act_launch,
//               silu_act_launch).
// ws (ws_floats) holds split-K partials; with ws null or too small the GEMM
// runs unsplit (QG_SILU and QG_PARTIAL always need ws for m x n floats).
struct QgJob {
  const uint8_t* a_tiles;  // from qgemm_act_launch or a fused row kernel
  int m, k;
  QgSeg seg[3];
  int nseg;
  int mode;
  float* dst;
  int ldd;
  float* ws;
  size_t ws_floats;
  uint32_t* err;
  int pdl;                 // launch with programmatic dependent launch: the
                           // weight stream starts before the previous kernel ends
};

// Where a QG_PARTIAL job left its result: element (t, j) is the sum over
// sp < splits of ws[sp * stride + t * ld + j], added in split order.
struct QgSplit {
  const float* ws;
  int splits;
  size_t stride;
  int ld;
};

// Tokens covered by the activation tile buffer for m tokens (a tile of 256
// tokens reads two 128-token tiles, so longer inputs round up to 256).
inline int qgemm_tok_pad(int m) { return m <= 128 ? 128 : ((m + 255) / 256) * 256; }
// Bytes of the activation tile buffer for m tokens and K.
inline size_t qgemm_a_bytes(int m, int k) {
  return (size_t)(qgemm_tok_pad(m) / 128) * (size_t)(k / QG_K) * QG_TILE_BYTES;
}

// The launchers below take pdl: launch with programmatic dependent launch
// (the kernels let their successor start early and wait for their
// predecessor before reading its output).
//
// Activation tiles of m token rows x[m][k] (rms-normalised with gamma when
// gamma is not null) into a_tiles (qgemm_a_bytes(m, k) bytes). K % 256 == 0,
// K <= 16384. Rows m .. qgemm_tok_pad(m) - 1 are left as they are: they only
// reach accumulator columns (tokens) that are never stored.
int qgemm_act_launch(const float* x, const float* gamma, float eps, int m, int k, uint8_t* a_tiles,
                     cudaStream_t s, bool pdl = false);
// Runs a job: picks the token tile and the K split, launches k_qgemm and,
// for QG_SILU and split QG_STORE / QG_RESID jobs, k_qg_finish. Sets the
// kernel's shared-memory limit on first use.
int qgemm_run(const QgJob& j, cudaStream_t s, QgSplit* split = nullptr);
// x[t][0, n) += the split sums (residual add, as candle's x + y), then, when
// a_tiles is not null, the activation tiles of the new rows normalised with
// gamma (as qgemm_act_launch). One CTA per token row.
int resid_act_launch(const QgSplit& g, float* x, int S, int n, const float* gamma, float eps, uint8_t* a_tiles,
                     cudaStream_t s, bool pdl = false);
// Activation tiles (no norm) of h[t][i] = silu(gate) * up from the split sums
// of a gate | up job (F columns each); h itself is not stored.
int silu_act_launch(const QgSplit& g, int S, int F, uint8_t* a_tiles, cudaStream_t s, bool pdl = false);
// Epilogue of the q|k|v GEMM split sums g (q | k | v columns), t = 0..S-1:
// RoPE'd q into q_out[t][QN], RoPE'd k and v into the KV cache at positions
// pos[t] of sequence slot t * seq_step (kv_seq_stride elements between
// slots; a prompt uses seq_step 0, a decode batch 1), as the matvec QKV
// epilogue does.
// With tiles, q, k and v are also written as the tensor-core attention's f16
// operand tiles (fa_tc.cuh; positions pos[t] must lie in the key tiles, rows
// of a tile that no token writes keep what they held); q_out may then be null.
struct FaTilesOut {
  uint8_t *q, *k, *v;
  int nqt, nkt;   // q tiles per head, key tiles per kv head
  int tile;       // bytes per tile
};
int qkv_post_launch(const QgSplit& g, int S, const int* pos, int qn, int kn, int hd, int max_seq,
                    const float* cos_t, const float* sin_t, float* q_out, void* kc, void* vc, int kv_f16,
                    int64_t kv_seq_stride, int seq_step, cudaStream_t s, bool pdl = false,
                    const FaTilesOut* tiles = nullptr);
// x[t][i] += g[t][i] (residual), i < n.
int resid_add_launch(float* x, const float* g, int S, int n, int ldg, cudaStream_t s);
// For each of the S rows of logits[t][0, n) (row stride ld): token[t] =
// first index of the largest value (the decode head's order), pos[t] += 1;
// with best_val / best_idx, also the winner's value and index (a tensor-
// parallel rank's candidate for the merge across ranks).
int row_argmax_launch(const float* logits, int S, int n, int ld, uint32_t* token, int* pos, cudaStream_t s,
                      bool pdl = false, float* best_val = nullptr, int* best_idx = nullptr);

}  // namespace armai
