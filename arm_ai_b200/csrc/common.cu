// common.cu — error plumbing and small host helpers for libarmai_cuda.so.
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace armai {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what, const char* file, int line) {
  const char* base = strrchr(file, '/');
  g_last_error = std::string("CUDA error: ") + cudaGetErrorString(e) + " (" + what + " at " +
                 (base ? base + 1 : file) + ":" + std::to_string(line) + ")";
  return e == cudaErrorMemoryAllocation ? ARMAI_E_NOMEM : ARMAI_E_CUDA;
}

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// Raw GGUF Q6_K rows -> device layout: nb bodies {ql, qh, scales} (208 B)
// then the nb f16 `d` values, zero-padded to a 16-byte multiple.
void repack_q6k_rows(const uint8_t* raw, int64_t rows, int64_t k, uint8_t* dst) {
  const int64_t nb = k / QK_K;
  const int64_t drow = dev_row_bytes(GGML_Q6_K, k);
  for (int64_t r = 0; r < rows; r++) {
    const uint8_t* src = raw + r * nb * Q6K_BLOCK_BYTES;
    uint8_t* out = dst + r * drow;
    uint8_t* dv = out + nb * Q6K_BODY_BYTES;
    std::memset(dv, 0, (size_t)q6k_dpad_bytes(nb));
    for (int64_t b = 0; b < nb; b++) {
      std::memcpy(out + b * Q6K_BODY_BYTES, src + b * Q6K_BLOCK_BYTES, Q6K_BODY_BYTES);
      std::memcpy(dv + 2 * b, src + b * Q6K_BLOCK_BYTES + Q6K_BODY_BYTES, 2);
    }
  }
}

}  // namespace armai

extern "C" const char* armai_last_error(void) { return armai::g_last_error.c_str(); }
extern "C" const char* armai_version(void) { return "armai-b200 0.1.0 (sm_100a)"; }
