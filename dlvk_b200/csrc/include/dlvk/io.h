// `.dlvk` model file format (v2 writer, v1/v2 readers).  See dlvk_io.cpp.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace dlvk {
namespace io {

struct TensorRecord {
  std::string name;
  uint32_t dtype = 0;          // dlvk::DType value
  std::vector<uint64_t> dims;
  std::string data;            // raw little-endian bytes
};

struct DlvkFile {
  uint32_t version = 0;
  std::string variant = "v2";  // "v2", "v1-header", "v1-weights"
  std::string meta_json;
  std::vector<TensorRecord> tensors;
};

std::string encode_v2(const std::string& meta_json, const std::vector<TensorRecord>& tensors);
void save_v2(const std::string& path, const std::string& meta_json, const std::vector<TensorRecord>& tensors);
std::string encode_v1_header(const std::string& meta_json);
DlvkFile decode(const std::string& blob);
DlvkFile load(const std::string& path);

}  // namespace io
}  // namespace dlvk
