// common.cuh — shared host/device helpers for libarmai_cuda.so (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "armai.h"

namespace armai {

// ---------------------------------------------------------------------------
// Host-side error plumbing: every C-ABI entry point returns a status and leaves
// a message in a thread-local buffer (armai_last_error).
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what, const char* file, int line);

#define ARMAI_CUDA(call)                                                        \
  do {                                                                          \
    cudaError_t _e = (call);                                                    \
    if (_e != cudaSuccess) return ::armai::cuda_fail(_e, #call, __FILE__, __LINE__); \
  } while (0)

#define ARMAI_TRY(call)        \
  do {                         \
    int _rc = (call);          \
    if (_rc != ARMAI_OK) return _rc; \
  } while (0)

// Number of SMs of the current device (cached per device).
int sm_count();

// Device error flag: kernels whose bounded waits expire set a bit here and
// return; the host checks it after synchronising.
enum : uint32_t {
  DEVERR_MBAR_TIMEOUT = 1u,
  DEVERR_COUNTER_TIMEOUT = 2u,
};

// ---------------------------------------------------------------------------
// GGML block formats (public GGUF layouts).
// ---------------------------------------------------------------------------
constexpr int QK_K = 256;
constexpr int GGML_F32 = 0;
constexpr int GGML_F16 = 1;
constexpr int GGML_Q4_0 = 2;
constexpr int GGML_Q5_0 = 6;
constexpr int GGML_Q8_0 = 8;
constexpr int GGML_Q4_K = 12;
constexpr int GGML_Q5_K = 13;
constexpr int GGML_Q6_K = 14;
constexpr int QK8_0 = 32;              // values per legacy block (Q4_0 / Q5_0 / Q8_0)
constexpr int Q4_0_BLOCK_BYTES = 18;   // f16 d, 16 B nibbles
constexpr int Q5_0_BLOCK_BYTES = 22;   // f16 d, 4 B high bits, 16 B nibbles
constexpr int Q8_0_BLOCK_BYTES = 34;   // f16 d, 32 i8
constexpr int Q5K_BLOCK_BYTES = 176;   // f16 d, f16 dmin, 12 B scales, 32 B qh, 128 B qs
constexpr int Q4K_BLOCK_BYTES = 144;  // f16 d, f16 dmin, 12 B scales, 128 B qs
constexpr int Q6K_BLOCK_BYTES = 210;  // 128 B ql, 64 B qh, 16 i8 scales, f16 d
// Q6_K as laid out in HBM: per row, nb blocks of [ql|qh|scales] (208 B each)
// followed by the nb f16 d values padded to a 16-byte multiple. Every row is
// then a 16-byte-aligned unit for bulk (TMA) copies.
constexpr int Q6K_BODY_BYTES = 208;
inline int64_t q6k_dpad_bytes(int64_t nb) { return ((nb * 2 + 15) / 16) * 16; }
// The weight types whose dot products take a Q8_K activation (k-quants) or
// a Q8_0 activation (legacy 32-value blocks), as candle's VecDotType.
__host__ __device__ inline bool is_kquant(int type) {
  return type == GGML_Q4_K || type == GGML_Q5_K || type == GGML_Q6_K;
}
__host__ __device__ inline bool is_legacy(int type) {
  return type == GGML_Q4_0 || type == GGML_Q5_0 || type == GGML_Q8_0;
}
__host__ __device__ inline int legacy_block_bytes(int type) {
  return type == GGML_Q4_0 ? Q4_0_BLOCK_BYTES : type == GGML_Q5_0 ? Q5_0_BLOCK_BYTES : Q8_0_BLOCK_BYTES;
}
inline int64_t dev_row_bytes(int type, int64_t k) {
  const int64_t nb = k / QK_K;
  if (type == GGML_Q4_K) return nb * Q4K_BLOCK_BYTES;
  if (type == GGML_Q5_K) return nb * Q5K_BLOCK_BYTES;
  if (type == GGML_Q6_K) return nb * Q6K_BODY_BYTES + q6k_dpad_bytes(nb);
  if (is_legacy(type)) return (k / QK8_0) * legacy_block_bytes(type);
  if (type == GGML_F32) return 4 * k;
  return -1;
}
// Q8_K as the host-facing test API stores it (candle BlockQ8K, 292 B).
struct BlockQ8K {
  float d;
  int8_t qs[256];
  int16_t bsums[16];
};
static_assert(sizeof(BlockQ8K) == 292, "BlockQ8K layout");

// Repack raw GGUF Q6_K rows into the device layout above (host side).
void repack_q6k_rows(const uint8_t* raw, int64_t rows, int64_t k, uint8_t* dst);

}  // namespace armai
