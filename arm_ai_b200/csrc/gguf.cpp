// gguf.cpp — GGUF v1-v3 header / metadata / tensor-directory reader.
#include "gguf.h"

#include <cstdio>
#include <cerrno>
#include <cstring>

#include "armai.h"

namespace armai {
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

namespace {

struct Reader {
  FILE* f = nullptr;
  uint32_t version = 3;
  bool ok = true;
  bool read(void* p, size_t n) {
    if (!ok) return false;
    if (fread(p, 1, n, f) != n) ok = false;
    return ok;
  }
  template <class T>
  T get() {
    T v{};
    read(&v, sizeof v);
    return v;
  }
  uint64_t count() { return version == 1 ? (uint64_t)get<uint32_t>() : get<uint64_t>(); }
  bool str(std::string& s) {
    uint64_t n = count();
    if (!ok || n > (1ull << 30)) return ok = false;
    s.resize(n);
    return n == 0 || read(&s[0], n);
  }
};

// GGUF value type ids.
enum : uint32_t {
  T_U8 = 0, T_I8 = 1, T_U16 = 2, T_I16 = 3, T_U32 = 4, T_I32 = 5, T_F32 = 6, T_BOOL = 7,
  T_STR = 8, T_ARR = 9, T_U64 = 10, T_I64 = 11, T_F64 = 12
};

bool read_scalar(Reader& r, uint32_t t, GgufValue& v) {
  v.type = t;
  switch (t) {
    case T_U8: v.kind = GgufValue::UINT; v.u = r.get<uint8_t>(); break;
    case T_U16: v.kind = GgufValue::UINT; v.u = r.get<uint16_t>(); break;
    case T_U32: v.kind = GgufValue::UINT; v.u = r.get<uint32_t>(); break;
    case T_U64: v.kind = GgufValue::UINT; v.u = r.get<uint64_t>(); break;
    case T_I8: v.kind = GgufValue::INT; v.i = r.get<int8_t>(); break;
    case T_I16: v.kind = GgufValue::INT; v.i = r.get<int16_t>(); break;
    case T_I32: v.kind = GgufValue::INT; v.i = r.get<int32_t>(); break;
    case T_I64: v.kind = GgufValue::INT; v.i = r.get<int64_t>(); break;
    case T_F32: v.kind = GgufValue::FLOAT; v.f = r.get<float>(); break;
    case T_F64: v.kind = GgufValue::FLOAT; v.f = r.get<double>(); break;
    case T_BOOL: v.kind = GgufValue::BOOL; v.u = r.get<uint8_t>(); break;
    case T_STR: v.kind = GgufValue::STRING; r.str(v.s); break;
    default: return false;
  }
  if (v.kind == GgufValue::UINT) { v.i = (int64_t)v.u; v.f = (double)v.u; }
  if (v.kind == GgufValue::INT) { v.u = (uint64_t)v.i; v.f = (double)v.i; }
  return r.ok;
}

bool read_value(Reader& r, uint32_t t, GgufValue& v) {
  if (t != T_ARR) return read_scalar(r, t, v);
  v.kind = GgufValue::ARRAY;
  v.type = T_ARR;
  uint32_t et = r.get<uint32_t>();
  uint64_t n = r.count();
  if (!r.ok || n > (1ull << 32)) return false;
  v.array_len = n;
  GgufValue tmp;
  for (uint64_t i = 0; i < n && r.ok; i++) {
    if (et == T_ARR) return false;  // nested arrays are not used by llama files
    if (!read_scalar(r, et, tmp)) return false;
  }
  return r.ok;
}

}  // namespace

int64_t GgufTensor::rows() const {
  int64_t r = 1;
  for (size_t i = 1; i < dims.size(); i++) r *= (int64_t)dims[i];
  return r;
}

int64_t ggml_row_bytes(uint32_t type, int64_t cols) {
  struct TS { uint32_t t; int64_t blk, bytes; };
  static const TS table[] = {{0, 1, 4},     {1, 1, 2},     {2, 32, 18},   {3, 32, 20},
                             {6, 32, 22},   {7, 32, 24},   {8, 32, 34},   {9, 32, 36},
                             {10, 256, 84}, {11, 256, 110}, {12, 256, 144}, {13, 256, 176},
                             {14, 256, 210}, {15, 256, 292}, {30, 1, 2}};
  for (const TS& e : table)
    if (e.t == type) return cols % e.blk ? -1 : (cols / e.blk) * e.bytes;
  return -1;
}

const char* ggml_type_name(uint32_t type) {
  switch (type) {
    case 0: return "F32"; case 1: return "F16"; case 2: return "Q4_0"; case 3: return "Q4_1";
    case 6: return "Q5_0"; case 7: return "Q5_1"; case 8: return "Q8_0"; case 9: return "Q8_1";
    case 10: return "Q2_K"; case 11: return "Q3_K"; case 12: return "Q4_K"; case 13: return "Q5_K";
    case 14: return "Q6_K"; case 15: return "Q8_K"; case 30: return "BF16";
    default: return "unknown";
  }
}

int gguf_read(const char* path, GgufFile& out) {
  if (!path || !*path) return fail(ARMAI_E_IO, "open failed: empty path");
  FILE* f = fopen(path, "rb");
  if (!f) return fail(ARMAI_E_IO, std::string("open ") + path + " failed: " + strerror(errno));
  Reader r;
  r.f = f;
  fseek(f, 0, SEEK_END);
  out.file_size = (uint64_t)ftell(f);
  fseek(f, 0, SEEK_SET);
  uint32_t magic = r.get<uint32_t>();
  if (!r.ok || magic != 0x46554747u) {  // "GGUF" little-endian
    fclose(f);
    return fail(ARMAI_E_FORMAT, "gguf read failed: bad magic (not a GGUF file)");
  }
  out.version = r.get<uint32_t>();
  if (out.version < 1 || out.version > 3) {
    fclose(f);
    return fail(ARMAI_E_FORMAT, "gguf read failed: unsupported version " + std::to_string(out.version));
  }
  r.version = out.version;
  uint64_t n_tensors = r.count();
  uint64_t n_kv = r.count();
  if (!r.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) {
    fclose(f);
    return fail(ARMAI_E_FORMAT, "gguf read failed: truncated header");
  }
  for (uint64_t i = 0; i < n_kv; i++) {
    std::string key;
    if (!r.str(key)) break;
    uint32_t t = r.get<uint32_t>();
    GgufValue v;
    if (!read_value(r, t, v)) {
      fclose(f);
      return fail(ARMAI_E_FORMAT, "gguf read failed: bad metadata value for key '" + key + "'");
    }
    out.kv[key] = v;
  }
  if (!r.ok) {
    fclose(f);
    return fail(ARMAI_E_FORMAT, "gguf read failed: truncated metadata");
  }
  auto al = out.kv.find("general.alignment");
  if (al != out.kv.end() && al->second.kind == GgufValue::UINT && al->second.u > 0)
    out.alignment = al->second.u;
  for (uint64_t i = 0; i < n_tensors; i++) {
    GgufTensor t;
    if (!r.str(t.name)) break;
    uint32_t nd = r.get<uint32_t>();
    if (!r.ok || nd == 0 || nd > 4) {
      fclose(f);
      return fail(ARMAI_E_FORMAT, "gguf read failed: bad tensor rank for '" + t.name + "'");
    }
    for (uint32_t d = 0; d < nd; d++) t.dims.push_back(r.version == 1 ? r.get<uint32_t>() : r.get<uint64_t>());
    t.type = r.get<uint32_t>();
    t.offset = r.get<uint64_t>();
    if (!r.ok) break;
    int64_t rb = ggml_row_bytes(t.type, t.cols());
    t.nbytes = rb < 0 ? 0 : (uint64_t)(rb * t.rows());
    out.tensors[t.name] = t;
  }
  if (!r.ok) {
    fclose(f);
    return fail(ARMAI_E_FORMAT, "gguf read failed: truncated tensor directory");
  }
  uint64_t pos = (uint64_t)ftell(f);
  out.data_offset = (pos + out.alignment - 1) / out.alignment * out.alignment;
  fclose(f);
  for (auto& kvp : out.tensors) {
    const GgufTensor& t = kvp.second;
    if (t.nbytes && out.data_offset + t.offset + t.nbytes > out.file_size)
      return fail(ARMAI_E_FORMAT, "gguf read failed: tensor '" + t.name + "' extends past end of file");
  }
  return ARMAI_OK;
}

}  // namespace armai
