// Host-side batch assembly for the data loader (native runtime).
//
// Reference: DataLoader::get_batch copies each sample of an MnistDataset
// into a std::vector, builds one-hot targets and uploads through a mapped
// host-visible buffer (src/data/dataloader.cpp:43-111); MnistDataset reads
// big-endian idx3/idx1 files (src/data/mnist.cpp:97-151).
//
// Here a batch is gathered by a small thread pool straight into a pinned
// host buffer that the H2D copy engine reads, optionally converting u8
// pixels to f32 with (x * scale + shift) on the way, and the shuffle is a
// deterministic function of (seed, epoch) so every data-parallel rank can
// derive its shard of the same permutation without communicating.
#pragma once
#include <cstdint>
#include <functional>
#include <string>
#include <vector>

namespace dlvk {
namespace data {

// Run fn(begin, end) over [0, n) on up to `threads` threads (inline for
// small n).
void parallel_for(int64_t n, int threads, int64_t min_chunk, const std::function<void(int64_t, int64_t)>& fn);

// dst[i, :] = src[idx[i], :] for rows of `row_bytes` bytes.
void gather_rows(const uint8_t* src, int64_t src_rows, int64_t row_bytes, const int64_t* idx, int64_t n,
                 uint8_t* dst, int threads);

// dst[i, j] = float(src[idx[i], j]) * scale + shift for u8 rows of `row_elems`.
void gather_u8_to_f32(const uint8_t* src, int64_t src_rows, int64_t row_elems, const int64_t* idx, int64_t n,
                      float* dst, float scale, float shift, int threads);

// Labels of the gathered rows: int32 ids (ids_out) and/or one-hot float
// rows of `classes` entries (one_hot_out).  Returns false if a label is
// outside [0, classes) (the one-hot row is then left all zero).
bool gather_labels(const int32_t* labels, int64_t src_rows, const int64_t* idx, int64_t n, int classes,
                   int32_t* ids_out, float* one_hot_out);

// Deterministic permutation of [0, n) for (seed, epoch): Fisher-Yates
// driven by splitmix64.
std::vector<int64_t> permutation(int64_t n, uint64_t seed, uint64_t epoch);

// IDX file (big-endian magic 0x0000 TT DD, TT = element type code, DD =
// number of dimensions, then DD big-endian u32 sizes, then the data).
struct IdxFile {
  int type_code = 0;  // 0x08 u8, 0x09 i8, 0x0B i16, 0x0C i32, 0x0D f32, 0x0E f64
  std::vector<int64_t> dims;
  std::string data;   // raw bytes, converted to host byte order for multi-byte types
};
IdxFile read_idx(const std::string& path);
void write_idx(const std::string& path, int type_code, const std::vector<int64_t>& dims, const std::string& data);

}  // namespace data
}  // namespace dlvk
