// gguf.h — minimal GGUF (v1-v3) reader: metadata + tensor directory.
//
// Replaces the role of candle-core 0.8.4 `quantized::gguf_file::Content::read`
// (called at native/arm_ai_nif/src/llama_candle.rs:39-40): it reads the
// header, every key/value pair and the tensor infos, and records where the
// aligned tensor-data section starts. Tensor bytes are read later, straight
// into pinned staging buffers, by the model loader.
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace armai {

struct GgufValue {
  enum Kind { UINT, INT, FLOAT, BOOL, STRING, ARRAY } kind = UINT;
  uint32_t type = 0;  // GGUF value type id
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  std::string s;
  uint64_t array_len = 0;
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;  // GGUF order: dims[0] is the contiguous axis
  uint32_t type = 0;
  uint64_t offset = 0;         // relative to the data section
  uint64_t nbytes = 0;
  int64_t rows() const;        // product of dims[1..]
  int64_t cols() const { return dims.empty() ? 0 : (int64_t)dims[0]; }
};

struct GgufFile {
  uint32_t version = 0;
  uint64_t alignment = 32;
  uint64_t data_offset = 0;  // absolute file offset of the tensor data section
  uint64_t file_size = 0;
  std::map<std::string, GgufValue> kv;
  std::map<std::string, GgufTensor> tensors;
};

// Returns 0 or an ARMAI_E_* status with armai_last_error() set.
int gguf_read(const char* path, GgufFile& out);
// Bytes of one row of `cols` elements of GGML type `type` (raw GGUF layout);
// -1 for unsupported types.
int64_t ggml_row_bytes(uint32_t type, int64_t cols);
const char* ggml_type_name(uint32_t type);

}  // namespace armai
