// Model export containers (native runtime): SafeTensors and GGUF v3.
//
// Reference: SafeTensorsExporter and GGUFExporter
// (include/dlvk/export/model_export.h:25-253, src/export/model_export.cpp:
// 150-366) write headers with no tensor payload (`extract_tensors` returns
// an empty list, model_export.cpp:17-48).  These write and read the full
// public formats:
//
//  SafeTensors: u64 little-endian header length N, N bytes of JSON
//    {"name": {"dtype": "F32"|"BF16"|..., "shape": [...],
//              "data_offsets": [begin, end]}, ..., "__metadata__": {str: str}}
//    (padded with spaces to a multiple of 8), then the tensor bytes.
//  GGUF v3: "GGUF", u32 version 3, u64 tensor count, u64 key/value count,
//    key/values (u64-length strings, u32 value type, value), tensor infos
//    (name, u32 n_dims, u64 dims innermost first, u32 ggml type, u64 offset
//    relative to the data section), padding to `general.alignment`
//    (default 32), tensor data (each tensor aligned).
#pragma once
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace dlvk {
namespace exportfmt {

struct Tensor {
  std::string name;
  std::string dtype;             // "F32", "F16", "BF16", "I32", "I8", "U8", "I64", "F64"
  std::vector<int64_t> shape;    // row-major, outermost first
  std::string data;              // raw little-endian bytes
};

// ---- SafeTensors -----------------------------------------------------------
std::string encode_safetensors(const std::vector<Tensor>& tensors,
                               const std::vector<std::pair<std::string, std::string>>& metadata);
void decode_safetensors(const std::string& blob, std::vector<Tensor>& tensors,
                        std::vector<std::pair<std::string, std::string>>& metadata);

// ---- GGUF v3 ---------------------------------------------------------------
// Key/value types written: string (8), u32 (4), i64 (11), f32 (6), bool (7),
// u64 (10).  Other types are read and skipped (their values kept as text).
struct KV {
  std::string key;
  uint32_t type = 8;
  std::string s;     // string value (or text of a value read but not typed here)
  uint64_t u = 0;    // u32 / u64 / bool
  int64_t i = 0;     // i64
  double f = 0.0;    // f32
};
std::string encode_gguf(const std::vector<Tensor>& tensors, const std::vector<KV>& kvs, uint32_t alignment);
void decode_gguf(const std::string& blob, std::vector<Tensor>& tensors, std::vector<KV>& kvs);

}  // namespace exportfmt
}  // namespace dlvk
