// Self-test of the host-side native runtime (.dlvk container, batch
// assembly, IDX files, SafeTensors / GGUF containers), built without CUDA so
// it can run under AddressSanitizer and UndefinedBehaviorSanitizer:
//
//   g++ -std=c++17 -O1 -g -fsanitize=address,undefined -fno-omit-frame-pointer \
//       -I dlvk_b200/csrc/include dlvk_b200/csrc/tests/runtime_selftest.cpp \
//       dlvk_b200/csrc/runtime/dlvk_io.cpp dlvk_b200/csrc/runtime/data_loader.cpp \
//       dlvk_b200/csrc/runtime/export_formats.cpp -o runtime_selftest -lpthread
//
// Exit code 0 and "ok" on success; any sanitizer report aborts.
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "dlvk/data.h"
#include "dlvk/export.h"
#include "dlvk/io.h"

#define CHECK(c)                                                   \
  do {                                                             \
    if (!(c)) {                                                    \
      std::fprintf(stderr, "CHECK failed: %s (%d)\n", #c, __LINE__); \
      return 1;                                                    \
    }                                                              \
  } while (0)

int main(int argc, char** argv) {
  const std::string dir = argc > 1 ? argv[1] : ".";
  // .dlvk v2 round trip (encode / decode / save / load)
  std::vector<dlvk::io::TensorRecord> recs(2);
  recs[0].name = "w";
  recs[0].dtype = 0;
  recs[0].dims = {3, 5};
  recs[0].data.assign(3 * 5 * 4, '\x01');
  recs[1].name = "empty";
  recs[1].dtype = 1;
  recs[1].dims = {0};
  const std::string blob = dlvk::io::encode_v2("{\"k\":1}", recs);
  auto f = dlvk::io::decode(blob);
  CHECK(f.version == 2 && f.tensors.size() == 2 && f.tensors[0].data == recs[0].data);
  CHECK(f.tensors[1].data.empty() && f.meta_json == "{\"k\":1}");
  dlvk::io::save_v2(dir + "/selftest.dlvk", "{}", recs);
  auto g = dlvk::io::load(dir + "/selftest.dlvk");
  CHECK(g.tensors.size() == 2 && g.tensors[0].dims == recs[0].dims);
  // truncated blobs are rejected, never read past the end
  for (size_t cut : {size_t(3), size_t(10), blob.size() / 2, blob.size() - 1}) {
    bool threw = false;
    try {
      dlvk::io::decode(blob.substr(0, cut));
    } catch (const std::exception&) {
      threw = true;
    }
    CHECK(threw);
  }
  // batch assembly
  std::vector<uint8_t> src(100 * 7);
  for (size_t i = 0; i < src.size(); ++i) src[i] = (uint8_t)(i * 31);
  auto perm = dlvk::data::permutation(100, 7, 3);
  CHECK(perm.size() == 100);
  std::vector<float> dst(100 * 7);
  dlvk::data::gather_u8_to_f32(src.data(), 100, 7, perm.data(), 100, dst.data(), 1.f / 255.f, 0.f, 4);
  CHECK(dst[7 * 5 + 2] == (float)src[perm[5] * 7 + 2] * (1.f / 255.f));
  std::vector<uint8_t> rows(100 * 7);
  dlvk::data::gather_rows(src.data(), 100, 7, perm.data(), 100, rows.data(), 3);
  CHECK(rows[7 * 9 + 6] == src[perm[9] * 7 + 6]);
  std::vector<int32_t> labels(100);
  for (int i = 0; i < 100; ++i) labels[i] = i % 10;
  std::vector<float> oh(100 * 10);
  std::vector<int32_t> ids(100);
  CHECK(dlvk::data::gather_labels(labels.data(), 100, perm.data(), 100, 10, ids.data(), oh.data()));
  CHECK(oh[10 * 3 + ids[3]] == 1.f);
  bool threw = false;
  std::vector<int64_t> bad = {5, 100};
  try {
    dlvk::data::gather_rows(src.data(), 100, 7, bad.data(), 2, rows.data(), 1);
  } catch (const std::out_of_range&) {
    threw = true;
  }
  CHECK(threw);
  // IDX
  std::string raw(2 * 3 * 4, '\0');
  for (int i = 0; i < 6; ++i) {
    int32_t v = i * 1000 - 2500;
    std::memcpy(&raw[i * 4], &v, 4);
  }
  dlvk::data::write_idx(dir + "/selftest.idx", 0x0C, {2, 3}, raw);
  auto idx = dlvk::data::read_idx(dir + "/selftest.idx");
  CHECK(idx.type_code == 0x0C && idx.dims.size() == 2 && idx.data == raw);
  // SafeTensors / GGUF
  std::vector<dlvk::exportfmt::Tensor> ts(1);
  ts[0].name = "layers.0.weight";
  ts[0].dtype = "F32";
  ts[0].shape = {2, 2};
  ts[0].data.assign(16, '\x02');
  const std::string st = dlvk::exportfmt::encode_safetensors(ts, {{"name", "a\"b"}});
  std::vector<dlvk::exportfmt::Tensor> back;
  std::vector<std::pair<std::string, std::string>> meta;
  dlvk::exportfmt::decode_safetensors(st, back, meta);
  CHECK(back.size() == 1 && back[0].data == ts[0].data && meta[0].second == "a\"b");
  dlvk::exportfmt::KV kv;
  kv.key = "general.name";
  kv.type = 8;
  kv.s = "m";
  const std::string gg = dlvk::exportfmt::encode_gguf(ts, {kv}, 32);
  std::vector<dlvk::exportfmt::Tensor> gb;
  std::vector<dlvk::exportfmt::KV> gk;
  dlvk::exportfmt::decode_gguf(gg, gb, gk);
  CHECK(gb.size() == 1 && gb[0].data == ts[0].data && gk[0].s == "m");
  for (size_t cut : {size_t(5), gg.size() / 2}) {
    bool t2 = false;
    try {
      std::vector<dlvk::exportfmt::Tensor> x;
      std::vector<dlvk::exportfmt::KV> y;
      dlvk::exportfmt::decode_gguf(gg.substr(0, cut), x, y);
    } catch (const std::exception&) {
      t2 = true;
    }
    CHECK(t2);
  }
  std::printf("ok\n");
  return 0;
}
