// Bindings of the host C++ runtime: `.dlvk` I/O and the CPU oracle.
#include "bind_common.h"
#include "dlvk/data.h"
#include "dlvk/export.h"
#include "dlvk/io.h"
#include "dlvk/oracle.h"

namespace dlvk {
namespace bind {

namespace {

float* fp(const at::Tensor& t) {
  TORCH_CHECK(!t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous(),
              "dlvk.ref: expected a contiguous CPU float32 tensor");
  return t.data_ptr<float>();
}
float* fpo(const c10::optional<at::Tensor>& t) { return t.has_value() ? fp(*t) : nullptr; }

py::tuple file_to_py(const io::DlvkFile& f) {
  py::list tens;
  for (const auto& t : f.tensors) {
    py::list dims;
    for (auto d : t.dims) dims.append(d);
    tens.append(py::make_tuple(t.name, t.dtype, dims, py::bytes(t.data)));
  }
  return py::make_tuple(f.version, f.variant, f.meta_json, tens);
}

std::vector<io::TensorRecord> py_to_records(const py::list& recs) {
  std::vector<io::TensorRecord> out;
  for (auto item : recs) {
    auto tup = item.cast<py::tuple>();
    io::TensorRecord r;
    r.name = tup[0].cast<std::string>();
    r.dtype = tup[1].cast<uint32_t>();
    r.dims = tup[2].cast<std::vector<uint64_t>>();
    r.data = tup[3].cast<std::string>();
    out.push_back(std::move(r));
  }
  return out;
}

}  // namespace

void cpu_contig(const at::Tensor& t, const char* what) {
  TORCH_CHECK(!t.is_cuda() && t.is_contiguous(), "dlvk.data: ", what, " must be a contiguous CPU tensor");
}

void register_data(py::module& m) {
  auto d = m.def_submodule("data", "native batch assembly (gather into pinned buffers, IDX files)");
  d.def("gather_rows", [](const at::Tensor& src, const at::Tensor& idx, at::Tensor& dst, int threads) {
    cpu_contig(src, "src");
    cpu_contig(idx, "idx");
    cpu_contig(dst, "dst");
    TORCH_CHECK(idx.scalar_type() == at::kLong, "dlvk.data: idx must be int64");
    TORCH_CHECK(src.dim() >= 1 && dst.size(0) >= idx.numel(), "dlvk.data: dst too small");
    const int64_t rows = src.size(0);
    const int64_t row_bytes = rows ? src.nbytes() / rows : 0;
    TORCH_CHECK(dst.nbytes() >= (size_t)(idx.numel() * row_bytes), "dlvk.data: dst bytes");
    py::gil_scoped_release nogil;
    data::gather_rows(static_cast<const uint8_t*>(src.data_ptr()), rows, row_bytes, idx.data_ptr<int64_t>(),
                      idx.numel(), static_cast<uint8_t*>(dst.data_ptr()), threads);
  }, py::arg("src"), py::arg("idx"), py::arg("dst"), py::arg("threads") = 4);
  d.def("gather_u8_to_f32", [](const at::Tensor& src, const at::Tensor& idx, at::Tensor& dst, double scale,
                               double shift, int threads) {
    cpu_contig(src, "src");
    cpu_contig(idx, "idx");
    cpu_contig(dst, "dst");
    TORCH_CHECK(src.scalar_type() == at::kByte && dst.scalar_type() == at::kFloat && idx.scalar_type() == at::kLong,
                "dlvk.data: gather_u8_to_f32 wants u8 src, f32 dst, int64 idx");
    const int64_t rows = src.size(0);
    const int64_t row = rows ? src.numel() / rows : 0;
    TORCH_CHECK(dst.numel() >= idx.numel() * row, "dlvk.data: dst too small");
    py::gil_scoped_release nogil;
    data::gather_u8_to_f32(src.data_ptr<uint8_t>(), rows, row, idx.data_ptr<int64_t>(), idx.numel(),
                           dst.data_ptr<float>(), (float)scale, (float)shift, threads);
  }, py::arg("src"), py::arg("idx"), py::arg("dst"), py::arg("scale") = 1.0, py::arg("shift") = 0.0,
     py::arg("threads") = 4);
  d.def("gather_labels", [](const at::Tensor& labels, const at::Tensor& idx, int classes,
                            c10::optional<at::Tensor> ids_out, c10::optional<at::Tensor> one_hot_out) {
    cpu_contig(labels, "labels");
    cpu_contig(idx, "idx");
    TORCH_CHECK(labels.scalar_type() == at::kInt && idx.scalar_type() == at::kLong, "dlvk.data: labels i32, idx i64");
    int32_t* ip = nullptr;
    float* op = nullptr;
    if (ids_out.has_value()) {
      cpu_contig(*ids_out, "ids_out");
      TORCH_CHECK(ids_out->scalar_type() == at::kInt && ids_out->numel() >= idx.numel(), "dlvk.data: ids_out");
      ip = ids_out->data_ptr<int32_t>();
    }
    if (one_hot_out.has_value()) {
      cpu_contig(*one_hot_out, "one_hot_out");
      TORCH_CHECK(one_hot_out->scalar_type() == at::kFloat && one_hot_out->numel() >= idx.numel() * classes,
                  "dlvk.data: one_hot_out");
      op = one_hot_out->data_ptr<float>();
    }
    return data::gather_labels(labels.data_ptr<int32_t>(), labels.numel(), idx.data_ptr<int64_t>(), idx.numel(),
                               classes, ip, op);
  }, py::arg("labels"), py::arg("idx"), py::arg("classes"), py::arg("ids_out") = py::none(),
     py::arg("one_hot_out") = py::none());
  d.def("permutation", [](int64_t n, uint64_t seed, uint64_t epoch) {
    auto p = data::permutation(n, seed, epoch);
    auto t = at::empty({n}, at::TensorOptions().dtype(at::kLong));
    if (n) std::memcpy(t.data_ptr<int64_t>(), p.data(), sizeof(int64_t) * (size_t)n);
    return t;
  });
  d.def("read_idx", [](const std::string& path) {
    auto f = data::read_idx(path);
    return py::make_tuple(f.type_code, f.dims, py::bytes(f.data));
  });
  d.def("write_idx", [](const std::string& path, int code, const std::vector<int64_t>& dims, const std::string& raw) {
    data::write_idx(path, code, dims, raw);
  });
}

std::vector<exportfmt::Tensor> py_to_ex(const py::list& recs) {
  std::vector<exportfmt::Tensor> out;
  for (auto item : recs) {
    auto tup = item.cast<py::tuple>();
    exportfmt::Tensor t;
    t.name = tup[0].cast<std::string>();
    t.dtype = tup[1].cast<std::string>();
    t.shape = tup[2].cast<std::vector<int64_t>>();
    t.data = tup[3].cast<std::string>();
    out.push_back(std::move(t));
  }
  return out;
}

py::list ex_to_py(const std::vector<exportfmt::Tensor>& ts) {
  py::list l;
  for (const auto& t : ts) l.append(py::make_tuple(t.name, t.dtype, t.shape, py::bytes(t.data)));
  return l;
}

void register_export(py::module& m) {
  auto e = m.def_submodule("export", "SafeTensors / GGUF v3 containers (C++)");
  e.def("encode_safetensors", [](const py::list& recs, const std::vector<std::pair<std::string, std::string>>& meta) {
    return py::bytes(exportfmt::encode_safetensors(py_to_ex(recs), meta));
  });
  e.def("decode_safetensors", [](const std::string& blob) {
    std::vector<exportfmt::Tensor> ts;
    std::vector<std::pair<std::string, std::string>> meta;
    exportfmt::decode_safetensors(blob, ts, meta);
    return py::make_tuple(ex_to_py(ts), meta);
  });
  // kvs: list of (key, type, value) with value str / int / float / bool
  e.def("encode_gguf", [](const py::list& recs, const py::list& kvs, uint32_t alignment) {
    std::vector<exportfmt::KV> kv;
    for (auto item : kvs) {
      auto tup = item.cast<py::tuple>();
      exportfmt::KV k;
      k.key = tup[0].cast<std::string>();
      k.type = tup[1].cast<uint32_t>();
      if (k.type == 8) k.s = tup[2].cast<std::string>();
      else if (k.type == 6) k.f = tup[2].cast<double>();
      else if (k.type == 11) k.i = tup[2].cast<int64_t>();
      else k.u = tup[2].cast<uint64_t>();
      kv.push_back(std::move(k));
    }
    return py::bytes(exportfmt::encode_gguf(py_to_ex(recs), kv, alignment));
  }, py::arg("recs"), py::arg("kvs"), py::arg("alignment") = 32);
  e.def("decode_gguf", [](const std::string& blob) {
    std::vector<exportfmt::Tensor> ts;
    std::vector<exportfmt::KV> kv;
    exportfmt::decode_gguf(blob, ts, kv);
    py::list kl;
    for (const auto& k : kv) {
      py::object v;
      if (k.type == 4 || k.type == 10) v = py::int_(k.u);
      else if (k.type == 7) v = py::bool_(k.u != 0);
      else if (k.type == 11) v = py::int_(k.i);
      else if (k.type == 6) v = py::float_(k.f);
      else v = py::str(k.s);
      kl.append(py::make_tuple(k.key, k.type, v));
    }
    return py::make_tuple(ex_to_py(ts), kl);
  });
}

void register_runtime(py::module& m) {
  register_data(m);
  register_export(m);
  auto io_m = m.def_submodule("io", ".dlvk file format (C++)");
  io_m.def("save_v2", [](const std::string& path, const std::string& meta, const py::list& recs) {
    io::save_v2(path, meta, py_to_records(recs));
  });
  io_m.def("encode_v2", [](const std::string& meta, const py::list& recs) {
    return py::bytes(io::encode_v2(meta, py_to_records(recs)));
  });
  io_m.def("encode_v1_header", [](const std::string& meta) { return py::bytes(io::encode_v1_header(meta)); });
  io_m.def("load", [](const std::string& path) { return file_to_py(io::load(path)); });
  io_m.def("decode", [](const std::string& blob) { return file_to_py(io::decode(blob)); });

  auto r = m.def_submodule("ref", "CPU oracle (plain C++ restatement of the reference op semantics)");
  r.def("dense_fwd", [](const at::Tensor& x, const at::Tensor& w, c10::optional<at::Tensor> b) {
    auto y = at::empty({x.size(0), w.size(1)}, x.options());
    ref::dense_fwd(fp(x), fp(w), fpo(b), fp(y), x.size(0), x.size(1), w.size(1));
    return y;
  });
  r.def("dense_bwd", [](const at::Tensor& x, const at::Tensor& w, const at::Tensor& g) {
    auto dx = at::empty_like(x), dw = at::empty_like(w), db = at::empty({w.size(1)}, w.options());
    ref::dense_bwd(fp(x), fp(w), fp(g), fp(dx), fp(dw), fp(db), x.size(0), x.size(1), w.size(1));
    return py::make_tuple(dx, dw, db);
  });
  r.def("relu", [](const at::Tensor& x) {
    auto y = at::empty_like(x);
    ref::relu(fp(x), fp(y), x.numel());
    return y;
  });
  r.def("relu_bwd", [](const at::Tensor& g, const at::Tensor& x) {
    auto d = at::empty_like(x);
    ref::relu_bwd(fp(g), fp(x), fp(d), x.numel());
    return d;
  });
  r.def("softmax", [](const at::Tensor& x) {
    auto y = at::empty_like(x);
    ref::softmax(fp(x), fp(y), x.size(0), x.size(1));
    return y;
  });
  r.def("cross_entropy", [](const at::Tensor& p, const at::Tensor& t) {
    return ref::cross_entropy(fp(p), fp(t), p.size(0), p.size(1));
  });
  r.def("cross_entropy_grad", [](const at::Tensor& p, const at::Tensor& t) {
    auto g = at::empty_like(p);
    ref::cross_entropy_grad(fp(p), fp(t), fp(g), p.size(0), p.size(1));
    return g;
  });
  r.def("mse", [](const at::Tensor& p, const at::Tensor& t) {
    auto g = at::empty_like(p);
    float l = ref::mse(fp(p), fp(t), fp(g), p.numel());
    return py::make_tuple(l, g);
  });
  r.def("bce", [](const at::Tensor& p, const at::Tensor& t) {
    auto g = at::empty_like(p);
    float l = ref::bce(fp(p), fp(t), fp(g), p.numel());
    return py::make_tuple(l, g);
  });
  r.def("adam", [](at::Tensor p, const at::Tensor& g, at::Tensor m_, at::Tensor v, double lr, double b1, double b2,
                   double eps, int step, bool bc) {
    ref::adam(fp(p), fp(g), fp(m_), fp(v), p.numel(), (float)lr, (float)b1, (float)b2, (float)eps, step, bc);
  });
  r.def("sgd", [](at::Tensor p, const at::Tensor& g, at::Tensor vel, double lr, double mom) {
    ref::sgd(fp(p), fp(g), fp(vel), p.numel(), (float)lr, (float)mom);
  });
  r.def("rmsprop", [](at::Tensor p, const at::Tensor& g, at::Tensor sq, double lr, double alpha, double eps) {
    ref::rmsprop(fp(p), fp(g), fp(sq), p.numel(), (float)lr, (float)alpha, (float)eps);
  });
  r.def("conv2d_fwd", [](const at::Tensor& x, const at::Tensor& w, c10::optional<at::Tensor> b, int stride, int pad) {
    ref::ConvShape s{(int)x.size(0), (int)x.size(1), (int)x.size(2), (int)x.size(3), (int)w.size(0),
                     (int)w.size(2), (int)w.size(3), stride, pad};
    auto y = at::empty({x.size(0), w.size(0), s.Ho(), s.Wo()}, x.options());
    ref::conv2d_fwd(fp(x), fp(w), fpo(b), fp(y), s);
    return y;
  });
  r.def("conv2d_bwd", [](const at::Tensor& x, const at::Tensor& w, const at::Tensor& g, int stride, int pad) {
    ref::ConvShape s{(int)x.size(0), (int)x.size(1), (int)x.size(2), (int)x.size(3), (int)w.size(0),
                     (int)w.size(2), (int)w.size(3), stride, pad};
    auto dx = at::empty_like(x), dw = at::empty_like(w), db = at::empty({w.size(0)}, w.options());
    ref::conv2d_bwd(fp(x), fp(w), fp(g), fp(dx), fp(dw), fp(db), s);
    return py::make_tuple(dx, dw, db);
  });
  r.def("maxpool_fwd", [](const at::Tensor& x, int k, int stride) {
    const int N = x.size(0), C = x.size(1), H = x.size(2), W = x.size(3);
    const int Ho = (H - k) / stride + 1, Wo = (W - k) / stride + 1;
    auto y = at::empty({N, C, Ho, Wo}, x.options());
    auto idx = at::empty({N, C, Ho, Wo}, x.options().dtype(at::kInt));
    ref::maxpool_fwd(fp(x), fp(y), idx.data_ptr<int32_t>(), N, C, H, W, k, stride);
    return py::make_tuple(y, idx);
  });
  r.def("maxpool_bwd", [](const at::Tensor& g, const at::Tensor& idx, int H, int W) {
    const int N = g.size(0), C = g.size(1), Ho = g.size(2), Wo = g.size(3);
    auto dx = at::empty({N, C, H, W}, g.options());
    ref::maxpool_bwd(fp(g), idx.data_ptr<int32_t>(), fp(dx), N, C, H, W, Ho, Wo);
    return dx;
  });
  r.def("avgpool_fwd", [](const at::Tensor& x, int k, int stride, int pad) {
    const int N = x.size(0), C = x.size(1), H = x.size(2), W = x.size(3);
    auto y = at::empty({N, C, (H + 2 * pad - k) / stride + 1, (W + 2 * pad - k) / stride + 1}, x.options());
    ref::avgpool_fwd(fp(x), fp(y), N, C, H, W, k, stride, pad);
    return y;
  });
  r.def("avgpool_bwd", [](const at::Tensor& g, int H, int W, int k, int stride, int pad) {
    const int N = g.size(0), C = g.size(1);
    auto dx = at::empty({N, C, H, W}, g.options());
    ref::avgpool_bwd(fp(g), fp(dx), N, C, H, W, k, stride, pad);
    return dx;
  });
  r.def("batchnorm_fwd", [](const at::Tensor& x, const at::Tensor& gamma, const at::Tensor& beta, at::Tensor rm,
                            at::Tensor rv, double momentum, double eps, bool training) {
    const int N = x.size(0), C = x.size(1);
    const int S = x.numel() / std::max<int64_t>(1, (int64_t)N * C);
    auto y = at::empty_like(x), mean = at::empty({C}, x.options()), rstd = at::empty({C}, x.options());
    ref::batchnorm_fwd(fp(x), fp(gamma), fp(beta), fp(y), fp(mean), fp(rstd), fp(rm), fp(rv), N, C, S,
                       (float)momentum, (float)eps, training);
    return py::make_tuple(y, mean, rstd);
  });
  r.def("batchnorm_bwd", [](const at::Tensor& x, const at::Tensor& gamma, const at::Tensor& mean,
                            const at::Tensor& rstd, const at::Tensor& g) {
    const int N = x.size(0), C = x.size(1);
    const int S = x.numel() / std::max<int64_t>(1, (int64_t)N * C);
    auto dx = at::empty_like(x), dg = at::empty({C}, x.options()), db = at::empty({C}, x.options());
    ref::batchnorm_bwd(fp(x), fp(gamma), fp(mean), fp(rstd), fp(g), fp(dx), fp(dg), fp(db), N, C, S);
    return py::make_tuple(dx, dg, db);
  });
  r.def("layernorm_fwd", [](const at::Tensor& x, const at::Tensor& gamma, const at::Tensor& beta, double eps) {
    const int64_t D = x.size(-1), R = x.numel() / D;
    auto y = at::empty_like(x), mean = at::empty({R}, x.options()), rstd = at::empty({R}, x.options());
    ref::layernorm_fwd(fp(x), fp(gamma), fp(beta), fp(y), fp(mean), fp(rstd), R, D, (float)eps);
    return py::make_tuple(y, mean, rstd);
  });
  r.def("layernorm_bwd", [](const at::Tensor& x, const at::Tensor& gamma, const at::Tensor& mean,
                            const at::Tensor& rstd, const at::Tensor& g) {
    const int64_t D = x.size(-1), R = x.numel() / D;
    auto dx = at::empty_like(x), dg = at::empty({D}, x.options()), db = at::empty({D}, x.options());
    ref::layernorm_bwd(fp(x), fp(gamma), fp(mean), fp(rstd), fp(g), fp(dx), fp(dg), fp(db), R, D);
    return py::make_tuple(dx, dg, db);
  });
  r.def("embedding_fwd", [](const at::Tensor& ids, const at::Tensor& table) {
    auto idc = ids.to(at::kInt).contiguous();
    auto out = at::empty({idc.numel(), table.size(1)}, table.options());
    ref::embedding_fwd(idc.data_ptr<int32_t>(), fp(table), fp(out), idc.numel(), table.size(0), table.size(1));
    return out;
  });
  r.def("embedding_bwd", [](const at::Tensor& ids, const at::Tensor& g, int64_t V) {
    auto idc = ids.to(at::kInt).contiguous();
    auto dt = at::empty({V, g.size(-1)}, g.options());
    ref::embedding_bwd(idc.data_ptr<int32_t>(), fp(g), fp(dt), idc.numel(), V, g.size(-1));
    return dt;
  });
  r.def("dropout_mask", [](int64_t n, double p, uint64_t seed, uint32_t stream, uint32_t step) {
    auto keep = at::empty({n}, at::TensorOptions().dtype(at::kByte));
    ref::dropout_mask(keep.data_ptr<uint8_t>(), n, (float)p, seed, stream, step);
    return keep;
  });
  r.def("attention", [](const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, bool causal) {
    auto o = at::empty_like(q);
    ref::attention(fp(q), fp(k), fp(v), fp(o), q.size(0), q.size(1), q.size(2), q.size(3), causal);
    return o;
  });
}

}  // namespace bind
}  // namespace dlvk
