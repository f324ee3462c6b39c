// Native batch assembly for the data loader (see dlvk/data.h).
#include <algorithm>
#include <cstring>
#include <fstream>
#include <functional>
#include <stdexcept>
#include <thread>

#include "dlvk/data.h"

namespace dlvk {
namespace data {

void parallel_for(int64_t n, int threads, int64_t min_chunk, const std::function<void(int64_t, int64_t)>& fn) {
  if (n <= 0) return;
  if (threads < 1) threads = 1;
  const int64_t chunks = std::max<int64_t>(1, std::min<int64_t>(threads, n / std::max<int64_t>(1, min_chunk)));
  if (chunks == 1) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve((size_t)chunks - 1);
  const int64_t per = (n + chunks - 1) / chunks;
  for (int64_t c = 1; c < chunks; ++c) {
    const int64_t b = c * per, e = std::min(n, b + per);
    if (b < e) pool.emplace_back(fn, b, e);
  }
  fn(0, std::min(n, per));
  for (auto& t : pool) t.join();
}

namespace {
void check_idx(const int64_t* idx, int64_t n, int64_t rows) {
  for (int64_t i = 0; i < n; ++i)
    if (idx[i] < 0 || idx[i] >= rows) throw std::out_of_range("dlvk.data: sample index out of range");
}
}  // namespace

void gather_rows(const uint8_t* src, int64_t src_rows, int64_t row_bytes, const int64_t* idx, int64_t n,
                 uint8_t* dst, int threads) {
  check_idx(idx, n, src_rows);
  // ~64 KB per task keeps thread start-up below the copy time
  const int64_t min_rows = std::max<int64_t>(1, (64 << 10) / std::max<int64_t>(1, row_bytes));
  parallel_for(n, threads, min_rows, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) std::memcpy(dst + i * row_bytes, src + idx[i] * row_bytes, (size_t)row_bytes);
  });
}

void gather_u8_to_f32(const uint8_t* src, int64_t src_rows, int64_t row_elems, const int64_t* idx, int64_t n,
                      float* dst, float scale, float shift, int threads) {
  check_idx(idx, n, src_rows);
  const int64_t min_rows = std::max<int64_t>(1, (32 << 10) / std::max<int64_t>(1, row_elems));
  parallel_for(n, threads, min_rows, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) {
      const uint8_t* s = src + idx[i] * row_elems;
      float* d = dst + i * row_elems;
      for (int64_t j = 0; j < row_elems; ++j) d[j] = (float)s[j] * scale + shift;
    }
  });
}

bool gather_labels(const int32_t* labels, int64_t src_rows, const int64_t* idx, int64_t n, int classes,
                   int32_t* ids_out, float* one_hot_out) {
  check_idx(idx, n, src_rows);
  bool ok = true;
  if (one_hot_out) std::memset(one_hot_out, 0, sizeof(float) * (size_t)n * (size_t)classes);
  for (int64_t i = 0; i < n; ++i) {
    const int32_t l = labels[idx[i]];
    if (ids_out) ids_out[i] = l;
    if (l < 0 || l >= classes) {
      ok = false;
      continue;
    }
    if (one_hot_out) one_hot_out[i * classes + l] = 1.f;
  }
  return ok;
}

namespace {
uint64_t splitmix64(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
}  // namespace

std::vector<int64_t> permutation(int64_t n, uint64_t seed, uint64_t epoch) {
  std::vector<int64_t> p((size_t)std::max<int64_t>(n, 0));
  for (int64_t i = 0; i < n; ++i) p[(size_t)i] = i;
  uint64_t s = seed * 0x2545F4914F6CDD1Dull + epoch;
  for (int64_t i = n - 1; i > 0; --i) {
    // unbiased bounded draw (Lemire's multiply-shift with rejection)
    const uint64_t range = (uint64_t)i + 1;
    uint64_t x = splitmix64(s);
    __uint128_t m = (__uint128_t)x * range;
    uint64_t lo = (uint64_t)m;
    if (lo < range) {
      const uint64_t t = (0 - range) % range;
      while (lo < t) {
        x = splitmix64(s);
        m = (__uint128_t)x * range;
        lo = (uint64_t)m;
      }
    }
    const int64_t j = (int64_t)(m >> 64);
    std::swap(p[(size_t)i], p[(size_t)j]);
  }
  return p;
}

namespace {
int elem_size(int code) {
  switch (code) {
    case 0x08: case 0x09: return 1;
    case 0x0B: return 2;
    case 0x0C: case 0x0D: return 4;
    case 0x0E: return 8;
    default: throw std::runtime_error("dlvk.data: unknown IDX element type");
  }
}
uint32_t be32(const unsigned char* b) {
  return ((uint32_t)b[0] << 24) | ((uint32_t)b[1] << 16) | ((uint32_t)b[2] << 8) | (uint32_t)b[3];
}
}  // namespace

IdxFile read_idx(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("dlvk.data: cannot open " + path);
  unsigned char hdr[4];
  if (!f.read(reinterpret_cast<char*>(hdr), 4)) throw std::runtime_error("dlvk.data: truncated IDX header");
  if (hdr[0] != 0 || hdr[1] != 0) throw std::runtime_error("dlvk.data: bad IDX magic in " + path);
  IdxFile out;
  out.type_code = hdr[2];
  const int nd = hdr[3];
  const int es = elem_size(out.type_code);
  int64_t total = 1;
  for (int d = 0; d < nd; ++d) {
    unsigned char b[4];
    if (!f.read(reinterpret_cast<char*>(b), 4)) throw std::runtime_error("dlvk.data: truncated IDX dims");
    out.dims.push_back((int64_t)be32(b));
    total *= (int64_t)be32(b);
  }
  out.data.resize((size_t)(total * es));
  if (total > 0 && !f.read(&out.data[0], (std::streamsize)out.data.size()))
    throw std::runtime_error("dlvk.data: truncated IDX data in " + path);
  if (es > 1) {  // big-endian -> host (little-endian)
    for (size_t i = 0; i < out.data.size(); i += (size_t)es) std::reverse(&out.data[i], &out.data[i] + es);
  }
  return out;
}

void write_idx(const std::string& path, int type_code, const std::vector<int64_t>& dims, const std::string& data) {
  const int es = elem_size(type_code);
  int64_t total = 1;
  for (auto d : dims) total *= d;
  if ((int64_t)data.size() != total * es) throw std::runtime_error("dlvk.data: IDX payload size mismatch");
  std::ofstream f(path, std::ios::binary | std::ios::trunc);
  if (!f) throw std::runtime_error("dlvk.data: cannot write " + path);
  const unsigned char hdr[4] = {0, 0, (unsigned char)type_code, (unsigned char)dims.size()};
  f.write(reinterpret_cast<const char*>(hdr), 4);
  for (auto d : dims) {
    const uint32_t v = (uint32_t)d;
    const unsigned char b[4] = {(unsigned char)(v >> 24), (unsigned char)(v >> 16), (unsigned char)(v >> 8),
                                (unsigned char)v};
    f.write(reinterpret_cast<const char*>(b), 4);
  }
  if (es == 1) {
    f.write(data.data(), (std::streamsize)data.size());
  } else {
    std::string be = data;
    for (size_t i = 0; i < be.size(); i += (size_t)es) std::reverse(&be[i], &be[i] + es);
    f.write(be.data(), (std::streamsize)be.size());
  }
  if (!f) throw std::runtime_error("dlvk.data: write failed for " + path);
}

}  // namespace data
}  // namespace dlvk
