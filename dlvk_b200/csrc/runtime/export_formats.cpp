// SafeTensors and GGUF v3 encoders/decoders (see dlvk/export.h).
#include <cstring>
#include <map>
#include <sstream>
#include <stdexcept>

#include "dlvk/export.h"

namespace dlvk {
namespace exportfmt {

namespace {

int64_t dtype_size(const std::string& dt) {
  if (dt == "F32" || dt == "I32") return 4;
  if (dt == "F16" || dt == "BF16") return 2;
  if (dt == "I8" || dt == "U8" || dt == "BOOL") return 1;
  if (dt == "I64" || dt == "F64") return 8;
  throw std::runtime_error("dlvk.export: unknown dtype " + dt);
}

int64_t numel(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (auto d : s) n *= d;
  return n;
}

void check_size(const Tensor& t) {
  if ((int64_t)t.data.size() != numel(t.shape) * dtype_size(t.dtype))
    throw std::runtime_error("dlvk.export: tensor '" + t.name + "' byte size does not match its shape");
}

std::string json_escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if ((unsigned char)c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", (unsigned)(unsigned char)c);
          o += buf;
        } else {
          o += c;
        }
    }
  }
  return o;
}

// Minimal JSON reader for the safetensors header: objects, arrays, strings,
// integers; enough for {"name": {"dtype":..,"shape":[..],"data_offsets":[..]}}.
struct JsonReader {
  const std::string& s;
  size_t p = 0;
  explicit JsonReader(const std::string& str) : s(str) {}
  void ws() {
    while (p < s.size() && (s[p] == ' ' || s[p] == '\n' || s[p] == '\r' || s[p] == '\t')) ++p;
  }
  void expect(char c) {
    ws();
    if (p >= s.size() || s[p] != c) throw std::runtime_error(std::string("dlvk.export: bad JSON, expected ") + c);
    ++p;
  }
  bool peek(char c) {
    ws();
    return p < s.size() && s[p] == c;
  }
  std::string str() {
    expect('"');
    std::string o;
    while (p < s.size() && s[p] != '"') {
      if (s[p] == '\\') {
        ++p;
        if (p >= s.size()) break;
        char e = s[p];
        if (e == 'n') o += '\n';
        else if (e == 't') o += '\t';
        else if (e == 'r') o += '\r';
        else if (e == 'u' && p + 4 < s.size()) {
          o += (char)std::stoi(s.substr(p + 1, 4), nullptr, 16);
          p += 4;
        } else o += e;
        ++p;
      } else {
        o += s[p++];
      }
    }
    expect('"');
    return o;
  }
  int64_t integer() {
    ws();
    size_t q = p;
    if (p < s.size() && s[p] == '-') ++p;
    while (p < s.size() && s[p] >= '0' && s[p] <= '9') ++p;
    if (q == p) throw std::runtime_error("dlvk.export: bad JSON number");
    return std::stoll(s.substr(q, p - q));
  }
  std::vector<int64_t> int_array() {
    std::vector<int64_t> v;
    expect('[');
    if (peek(']')) {
      ++p;
      return v;
    }
    for (;;) {
      v.push_back(integer());
      if (peek(',')) {
        ++p;
        continue;
      }
      expect(']');
      return v;
    }
  }
};

void put_u32(std::string& o, uint32_t v) { o.append(reinterpret_cast<const char*>(&v), 4); }
void put_u64(std::string& o, uint64_t v) { o.append(reinterpret_cast<const char*>(&v), 8); }
void put_str(std::string& o, const std::string& s) {
  put_u64(o, s.size());
  o += s;
}

struct Cursor {
  const std::string& b;
  size_t p = 0;
  explicit Cursor(const std::string& blob) : b(blob) {}
  void need(size_t n) const {
    if (p + n > b.size()) throw std::runtime_error("dlvk.export: truncated file");
  }
  template <typename T>
  T get() {
    need(sizeof(T));
    T v;
    std::memcpy(&v, b.data() + p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    need(n);
    std::string s = b.substr(p, n);
    p += n;
    return s;
  }
};

// ggml tensor types for the dtypes exported here
uint32_t ggml_type(const std::string& dt) {
  if (dt == "F32") return 0;
  if (dt == "F16") return 1;
  if (dt == "I8") return 24;
  if (dt == "I32") return 26;
  if (dt == "I64") return 27;
  if (dt == "F64") return 28;
  if (dt == "BF16") return 30;
  throw std::runtime_error("dlvk.export: dtype " + dt + " has no GGUF tensor type");
}
std::string from_ggml(uint32_t t) {
  switch (t) {
    case 0: return "F32";
    case 1: return "F16";
    case 24: return "I8";
    case 26: return "I32";
    case 27: return "I64";
    case 28: return "F64";
    case 30: return "BF16";
    default: throw std::runtime_error("dlvk.export: GGUF tensor type " + std::to_string(t) + " not supported");
  }
}

uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

// size in bytes of a scalar GGUF value type (0 for string / array)
size_t gguf_scalar_size(uint32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
  }
}

void skip_gguf_value(Cursor& c, uint32_t t, KV* kv) {
  if (t == 8) {
    std::string s = c.str();
    if (kv) kv->s = s;
    return;
  }
  if (t == 9) {  // array: u32 element type, u64 count, elements
    const uint32_t et = c.get<uint32_t>();
    const uint64_t n = c.get<uint64_t>();
    for (uint64_t i = 0; i < n; ++i) skip_gguf_value(c, et, nullptr);
    if (kv) kv->s = "[array of " + std::to_string(n) + "]";
    return;
  }
  const size_t sz = gguf_scalar_size(t);
  if (!sz) throw std::runtime_error("dlvk.export: unknown GGUF value type " + std::to_string(t));
  c.need(sz);
  c.p += sz;
}

}  // namespace

std::string encode_safetensors(const std::vector<Tensor>& tensors,
                               const std::vector<std::pair<std::string, std::string>>& metadata) {
  std::ostringstream h;
  h << "{";
  bool first = true;
  if (!metadata.empty()) {
    h << "\"__metadata__\":{";
    for (size_t i = 0; i < metadata.size(); ++i) {
      if (i) h << ",";
      h << "\"" << json_escape(metadata[i].first) << "\":\"" << json_escape(metadata[i].second) << "\"";
    }
    h << "}";
    first = false;
  }
  uint64_t off = 0;
  for (const auto& t : tensors) {
    check_size(t);
    if (!first) h << ",";
    first = false;
    h << "\"" << json_escape(t.name) << "\":{\"dtype\":\"" << t.dtype << "\",\"shape\":[";
    for (size_t i = 0; i < t.shape.size(); ++i) h << (i ? "," : "") << t.shape[i];
    h << "],\"data_offsets\":[" << off << "," << off + t.data.size() << "]}";
    off += t.data.size();
  }
  h << "}";
  std::string header = h.str();
  while (header.size() % 8) header += ' ';
  std::string out;
  put_u64(out, header.size());
  out += header;
  for (const auto& t : tensors) out += t.data;
  return out;
}

void decode_safetensors(const std::string& blob, std::vector<Tensor>& tensors,
                        std::vector<std::pair<std::string, std::string>>& metadata) {
  Cursor c(blob);
  const uint64_t n = c.get<uint64_t>();
  c.need(n);
  const std::string header = blob.substr(8, n);
  const size_t base = 8 + n;
  JsonReader j(header);
  j.expect('{');
  if (j.peek('}')) return;
  for (;;) {
    const std::string key = j.str();
    j.expect(':');
    if (key == "__metadata__") {
      j.expect('{');
      if (!j.peek('}')) {
        for (;;) {
          std::string k = j.str();
          j.expect(':');
          metadata.emplace_back(k, j.str());
          if (j.peek(',')) {
            ++j.p;
            continue;
          }
          break;
        }
      }
      j.expect('}');
    } else {
      Tensor t;
      t.name = key;
      std::vector<int64_t> offs;
      j.expect('{');
      for (;;) {
        const std::string f = j.str();
        j.expect(':');
        if (f == "dtype") t.dtype = j.str();
        else if (f == "shape") t.shape = j.int_array();
        else if (f == "data_offsets") offs = j.int_array();
        else throw std::runtime_error("dlvk.export: unexpected safetensors field " + f);
        if (j.peek(',')) {
          ++j.p;
          continue;
        }
        break;
      }
      j.expect('}');
      if (offs.size() != 2 || offs[0] < 0 || offs[1] < offs[0] || base + (size_t)offs[1] > blob.size())
        throw std::runtime_error("dlvk.export: bad data_offsets for " + key);
      t.data = blob.substr(base + (size_t)offs[0], (size_t)(offs[1] - offs[0]));
      check_size(t);
      tensors.push_back(std::move(t));
    }
    if (j.peek(',')) {
      ++j.p;
      continue;
    }
    break;
  }
  j.expect('}');
}

std::string encode_gguf(const std::vector<Tensor>& tensors, const std::vector<KV>& kvs_in, uint32_t alignment) {
  if (alignment == 0 || (alignment & (alignment - 1))) throw std::runtime_error("dlvk.export: alignment");
  std::vector<KV> kvs = kvs_in;
  bool has_align = false;
  for (const auto& kv : kvs) has_align |= kv.key == "general.alignment";
  if (!has_align && alignment != 32) {
    KV a;
    a.key = "general.alignment";
    a.type = 4;
    a.u = alignment;
    kvs.push_back(a);
  }
  std::string o = "GGUF";
  put_u32(o, 3);
  put_u64(o, tensors.size());
  put_u64(o, kvs.size());
  for (const auto& kv : kvs) {
    put_str(o, kv.key);
    put_u32(o, kv.type);
    switch (kv.type) {
      case 8: put_str(o, kv.s); break;
      case 4: put_u32(o, (uint32_t)kv.u); break;
      case 10: put_u64(o, kv.u); break;
      case 11: put_u64(o, (uint64_t)kv.i); break;
      case 6: {
        const float f = (float)kv.f;
        o.append(reinterpret_cast<const char*>(&f), 4);
        break;
      }
      case 7: o += (char)(kv.u ? 1 : 0); break;
      default: throw std::runtime_error("dlvk.export: GGUF value type not writable: " + std::to_string(kv.type));
    }
  }
  uint64_t off = 0;
  for (const auto& t : tensors) {
    check_size(t);
    put_str(o, t.name);
    put_u32(o, (uint32_t)t.shape.size());
    for (auto it = t.shape.rbegin(); it != t.shape.rend(); ++it) put_u64(o, (uint64_t)*it);  // innermost first
    put_u32(o, ggml_type(t.dtype));
    put_u64(o, off);
    off = align_up(off + t.data.size(), alignment);
  }
  o.resize(align_up(o.size(), alignment), '\0');
  for (const auto& t : tensors) {
    o += t.data;
    o.resize(align_up(o.size(), alignment), '\0');
  }
  return o;
}

void decode_gguf(const std::string& blob, std::vector<Tensor>& tensors, std::vector<KV>& kvs) {
  Cursor c(blob);
  c.need(4);
  if (blob.compare(0, 4, "GGUF") != 0) throw std::runtime_error("dlvk.export: bad GGUF magic");
  c.p = 4;
  const uint32_t version = c.get<uint32_t>();
  if (version != 3 && version != 2) throw std::runtime_error("dlvk.export: GGUF version " + std::to_string(version));
  const uint64_t nt = c.get<uint64_t>();
  const uint64_t nkv = c.get<uint64_t>();
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < nkv; ++i) {
    KV kv;
    kv.key = c.str();
    kv.type = c.get<uint32_t>();
    switch (kv.type) {
      case 4: kv.u = c.get<uint32_t>(); break;
      case 10: kv.u = c.get<uint64_t>(); break;
      case 11: kv.i = c.get<int64_t>(); break;
      case 6: kv.f = c.get<float>(); break;
      case 7: kv.u = (uint8_t)c.get<uint8_t>(); break;
      default: skip_gguf_value(c, kv.type, &kv);
    }
    if (kv.key == "general.alignment" && (kv.type == 4 || kv.type == 10)) alignment = kv.u;
    kvs.push_back(std::move(kv));
  }
  struct Info {
    std::string name;
    std::vector<int64_t> shape;
    std::string dtype;
    uint64_t off;
  };
  std::vector<Info> infos;
  for (uint64_t i = 0; i < nt; ++i) {
    Info in;
    in.name = c.str();
    const uint32_t nd = c.get<uint32_t>();
    std::vector<int64_t> dims(nd);
    for (uint32_t d = 0; d < nd; ++d) dims[d] = (int64_t)c.get<uint64_t>();
    in.shape.assign(dims.rbegin(), dims.rend());
    in.dtype = from_ggml(c.get<uint32_t>());
    in.off = c.get<uint64_t>();
    infos.push_back(std::move(in));
  }
  const uint64_t data0 = align_up(c.p, alignment);
  for (auto& in : infos) {
    Tensor t;
    t.name = in.name;
    t.dtype = in.dtype;
    t.shape = in.shape;
    const uint64_t bytes = (uint64_t)(numel(t.shape) * dtype_size(t.dtype));
    if (data0 + in.off + bytes > blob.size()) throw std::runtime_error("dlvk.export: GGUF tensor out of range");
    t.data = blob.substr(data0 + in.off, bytes);
    tensors.push_back(std::move(t));
  }
}

}  // namespace exportfmt
}  // namespace dlvk
