// `.dlvk` model file reader/writer.
//
// Framing kept from the reference (src/training/model_persistence.cpp:13-45,
// src/export/model_export.cpp:369-469): "DLVK" magic, u32 version, then a
// version-specific body, all little-endian.
//
//  v2 (written here):
//    "DLVK" | u32 2 | u32 meta_len | meta JSON (UTF-8) | u32 tensor_count |
//    tensor_count x { u32 name_len | name | u32 dtype | u32 ndim |
//                     u64 dims[ndim] | u64 nbytes | zero pad to a 64-byte file
//                     offset | nbytes raw bytes }
//    Files are written to "<path>.tmp" and renamed into place, so a crash
//    mid-write never leaves a truncated checkpoint under the final name.
//
//  v1, header-only variant (reference ModelSerializer::save_binary and
//    DLVKExporter): "DLVK" | u32 1 | u32 meta_len | meta JSON | u32 n=0.
//  v1, weight-bearing variant (the reference's linear_model.dlvk):
//    "DLVK" | u32 1 | u32 n_sizes | u32 sizes[n] | u32 n_w | f32 w[n_w] |
//    u32 n_b | f32 b[n_b] | u32 len | activation | f32 final_loss |
//    u32 epochs | u32 len | timestamp.
#include "dlvk/io.h"

#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>

namespace dlvk {
namespace io {

namespace {

void put_u32(std::string& b, uint32_t v) { b.append(reinterpret_cast<const char*>(&v), 4); }
void put_u64(std::string& b, uint64_t v) { b.append(reinterpret_cast<const char*>(&v), 8); }

struct Reader {
  const std::string& s;
  size_t off = 0;
  explicit Reader(const std::string& str) : s(str) {}
  void need(size_t n) const {
    if (off + n > s.size()) throw std::runtime_error("dlvk file truncated at byte " + std::to_string(off));
  }
  uint32_t u32() {
    need(4);
    uint32_t v;
    std::memcpy(&v, s.data() + off, 4);
    off += 4;
    return v;
  }
  uint64_t u64() {
    need(8);
    uint64_t v;
    std::memcpy(&v, s.data() + off, 8);
    off += 8;
    return v;
  }
  float f32() {
    need(4);
    float v;
    std::memcpy(&v, s.data() + off, 4);
    off += 4;
    return v;
  }
  std::string bytes(size_t n) {
    need(n);
    std::string r = s.substr(off, n);
    off += n;
    return r;
  }
};

std::string json_escape(const std::string& in) {
  std::string o;
  for (char c : in) {
    if (c == '"' || c == '\\') {
      o.push_back('\\');
      o.push_back(c);
    } else if (c == '\n') {
      o += "\\n";
    } else {
      o.push_back(c);
    }
  }
  return o;
}

TensorRecord f32_record(const std::string& name, const std::vector<float>& v) {
  TensorRecord r;
  r.name = name;
  r.dtype = 0;  // F32
  r.dims = {v.size()};
  r.data.assign(reinterpret_cast<const char*>(v.data()), v.size() * 4);
  return r;
}

}  // namespace

std::string encode_v2(const std::string& meta_json, const std::vector<TensorRecord>& tensors) {
  std::string b;
  b.reserve(64 + meta_json.size());
  b.append("DLVK", 4);
  put_u32(b, 2);
  put_u32(b, (uint32_t)meta_json.size());
  b += meta_json;
  put_u32(b, (uint32_t)tensors.size());
  for (const auto& t : tensors) {
    put_u32(b, (uint32_t)t.name.size());
    b += t.name;
    put_u32(b, t.dtype);
    put_u32(b, (uint32_t)t.dims.size());
    for (uint64_t d : t.dims) put_u64(b, d);
    put_u64(b, (uint64_t)t.data.size());
    const size_t pad = (64 - (b.size() % 64)) % 64;
    b.append(pad, '\0');
    b += t.data;
  }
  return b;
}

void save_v2(const std::string& path, const std::string& meta_json, const std::vector<TensorRecord>& tensors) {
  const std::string blob = encode_v2(meta_json, tensors);
  const std::string tmp = path + ".tmp";
  {
    std::ofstream f(tmp, std::ios::binary | std::ios::trunc);
    if (!f) throw std::runtime_error("dlvk: cannot open " + tmp + " for writing");
    f.write(blob.data(), (std::streamsize)blob.size());
    f.flush();
    if (!f) throw std::runtime_error("dlvk: write failed for " + tmp);
  }
  if (std::rename(tmp.c_str(), path.c_str()) != 0) throw std::runtime_error("dlvk: rename to " + path + " failed");
}

DlvkFile decode(const std::string& blob) {
  Reader r(blob);
  if (blob.size() < 8 || blob.compare(0, 4, "DLVK") != 0) throw std::runtime_error("dlvk: bad magic");
  r.off = 4;
  DlvkFile f;
  f.version = r.u32();
  if (f.version == 2) {
    const uint32_t ml = r.u32();
    f.meta_json = r.bytes(ml);
    const uint32_t n = r.u32();
    for (uint32_t i = 0; i < n; ++i) {
      TensorRecord t;
      const uint32_t nl = r.u32();
      t.name = r.bytes(nl);
      t.dtype = r.u32();
      const uint32_t nd = r.u32();
      for (uint32_t d = 0; d < nd; ++d) t.dims.push_back(r.u64());
      const uint64_t nb = r.u64();
      r.off += (64 - (r.off % 64)) % 64;
      t.data = r.bytes(nb);
      f.tensors.push_back(std::move(t));
    }
    return f;
  }
  if (f.version != 1) throw std::runtime_error("dlvk: unsupported version " + std::to_string(f.version));
  // v1: header-only variant has JSON right after the length word.
  if (blob.size() > 12 && blob[12] == '{') {
    f.variant = "v1-header";
    const uint32_t ml = r.u32();
    f.meta_json = r.bytes(ml);
    const uint32_t n = (r.off + 4 <= blob.size()) ? r.u32() : 0;
    if (n != 0) throw std::runtime_error("dlvk v1: header-only file with non-zero parameter count");
    return f;
  }
  f.variant = "v1-weights";
  const uint32_t ns = r.u32();
  std::vector<float> sizes_f;
  std::vector<uint32_t> sizes;
  for (uint32_t i = 0; i < ns; ++i) sizes.push_back(r.u32());
  const uint32_t nw = r.u32();
  std::vector<float> w(nw);
  for (auto& x : w) x = r.f32();
  const uint32_t nb = r.u32();
  std::vector<float> b(nb);
  for (auto& x : b) x = r.f32();
  const uint32_t al = r.u32();
  const std::string act = r.bytes(al);
  const float final_loss = r.f32();
  const uint32_t epochs = r.u32();
  const uint32_t tl = r.u32();
  const std::string ts = r.bytes(tl);
  TensorRecord ls;
  ls.name = "layer_sizes";
  ls.dtype = 3;  // I32
  ls.dims = {sizes.size()};
  ls.data.assign(reinterpret_cast<const char*>(sizes.data()), sizes.size() * 4);
  f.tensors.push_back(ls);
  f.tensors.push_back(f32_record("weights", w));
  f.tensors.push_back(f32_record("biases", b));
  std::ostringstream js;
  js.precision(9);
  js << "{\"framework\": \"DLVK\", \"version\": 1, \"activation\": \"" << json_escape(act)
     << "\", \"final_loss\": " << final_loss << ", \"epochs_trained\": " << epochs << ", \"timestamp\": \""
     << json_escape(ts) << "\"}";
  f.meta_json = js.str();
  return f;
}

DlvkFile load(const std::string& path) {
  std::ifstream in(path, std::ios::binary);
  if (!in) throw std::runtime_error("dlvk: cannot open " + path);
  std::stringstream ss;
  ss << in.rdbuf();
  return decode(ss.str());
}

std::string encode_v1_header(const std::string& meta_json) {
  std::string b;
  b.append("DLVK", 4);
  put_u32(b, 1);
  put_u32(b, (uint32_t)meta_json.size());
  b += meta_json;
  put_u32(b, 0);
  return b;
}

}  // namespace io
}  // namespace dlvk
