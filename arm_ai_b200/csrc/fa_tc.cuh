// fa_tc.cuh — attention on the 5th-generation tensor cores (sm_100a):
// out = softmax(scale * Q K^T [causal]) V for a block of queries against a
// key/value sequence: the prompt attention of candle's quantized_llama
// (candle-transformers 0.8.4 ModelWeights::forward at offset 0, reached from
// native/arm_ai_nif/src/llama_candle.rs:69-137: q.matmul(k^T) / sqrt(d),
// masked_fill(-inf) above the diagonal, softmax, @ v) and the reference's
// flash_attention_f32_op (native/arm_ai_nif/src/shape_ops.rs:464-558),
// computed with an online softmax over key tiles.
//
// One CTA = 128 queries of one head (tensor-memory lanes), one CTA per SM.
// Per key tile of 128: S = Q K^T by tcgen05.mma (kind::f16, f32 into one of
// two S buffers in tensor memory); eight softmax warps (two per row: each
// half the keys) read S with tcgen05.ld, keep the running max / sum in f32,
// write P = exp(S - max) as f16 back into the same tensor-memory columns,
// rescale the f32 output accumulator in tensor memory when the max moves;
// O += P V is a second MMA with P as the A operand from tensor memory and
// V^T from shared memory. One thread streams the f16 operand tiles (already
// in the K-major, 128-byte-swizzled layout) by bulk copy, two K and two V^T
// tiles deep, and issues the MMAs: the next tile's S runs while the softmax
// warps work on this one.
//
// Precision: f16 operands (2^-11 relative) and f32 accumulation; the
// reference computes in f32. Every wait is bounded and sets an error flag.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include <cuda_runtime.h>

#include "common.cuh"

namespace armai {

struct FaParams {
  // Operand tiles, f16 in the layout the kernel stages, indexed over batch,
  // then head, then tile (fa_tiles_launch writes them from strided rows; the
  // prompt's q/k/v epilogue writes them directly).
  const uint8_t* qt;     // [batch][n_head][q tiles][hd / 64][128 rows][128 B]
  const uint8_t* kt;     // [batch][kv heads][key tiles][hd / 64][128 keys][128 B]
  const uint8_t* vt;     // [batch][kv heads][key tiles][2][hd rows][128 B]: V^T, 64 keys per 128-byte row
  int nqt, nkt;          // q tiles per head, key tiles per kv head
  float* o;              // f32 output: element (b, t, h, d) at b*o_bs + t*o_ts + h*o_hs + d
  int64_t o_bs, o_ts, o_hs;
  int sq, sk;            // queries, keys (causal: query i sees keys 0 .. i)
  int n_head, group;     // heads; query heads per key/value head
  float scale;
  int causal;
  uint32_t* err;         // device error word (null: the module's own)
};

// Bytes of one operand tile (128 rows or keys) of head dimension hd.
__host__ __device__ inline size_t fa_tile_bytes(int hd) { return (size_t)hd * 256; }

// Tiled operands: byte offset of element (row, d) of a Q or K tile (row =
// query or key within the tile, d < hd), and of element (key, d) of a V^T
// tile; 128-byte rows, 16-byte chunks XOR-swizzled by row & 7.
__host__ __device__ inline uint32_t fa_qk_off(int row, int d) {
  const int kb = d >> 6, c = (d & 63) >> 3;
  return (uint32_t)(kb * 128 * 128 + row * 128 + ((c ^ (row & 7)) << 4) + 2 * (d & 7));
}
__host__ __device__ inline uint32_t fa_vt_off(int hd, int key, int d) {
  const int kb = key >> 6, c = (key & 63) >> 3;
  return (uint32_t)(kb * hd * 128 + d * 128 + ((c ^ (d & 7)) << 4) + 2 * (key & 7));
}

// Operand tiles from strided rows: src element (b, row, h, d) at
// b*bs + row*ts + h*hs + d (f16 when f16, else f32), rows < n_rows (the
// rest of the last tile is zero), into dst as [batch][heads][tiles][...]:
// Q / K tiles, or V^T tiles when transpose. dst holds
// batch * heads * ceil(n_rows / 128) * fa_tile_bytes(hd) bytes.
int fa_tiles_launch(const void* src, bool f16, int64_t bs, int64_t ts, int64_t hs, int batch, int heads, int n_rows,
                    int hd, bool transpose, uint8_t* dst, cudaStream_t s);

// Launch for head dim 64 or 128 and batch b (gridDim.z). Returns
// ARMAI_E_INVALID for other head dims.
int fa_tc_launch(const FaParams& p, int hd, int batch, cudaStream_t s, bool pdl = false);

}  // namespace armai
