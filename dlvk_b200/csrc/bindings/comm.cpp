// Bindings of the peer-memory communication layer.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "bind_common.h"
#include "dlvk/comm.h"

namespace dlvk {
namespace bind {
namespace {

at::ScalarType scalar_of(int code) {
  switch (code) {
    case 0: return at::kFloat;
    case 1: return at::kBFloat16;
    case 3: return at::kInt;
    case 6: return at::kLong;
    default: TORCH_CHECK(false, "SymmetricBuffer.tensor: unsupported dtype code ", code);
  }
}

struct PySym {
  std::shared_ptr<SymmetricBuffer> buf;
};

// Arguments of one fused launch, gathered from tensors on the Python side.
void fused_ar_op(std::shared_ptr<SymmetricBuffer> grads, std::shared_ptr<SymmetricBuffer> values,
                 std::shared_ptr<SymmetricBuffer> flags, const at::Tensor& counters, int64_t bucket, int64_t start,
                 int64_t end, const at::Tensor& master, c10::optional<at::Tensor> m, c10::optional<at::Tensor> v,
                 const at::Tensor& hyper, int64_t kind, const at::Tensor& epoch, int64_t world, int64_t rank,
                 bool one_shot, bool values_are_master, int64_t grad_code, int64_t value_code, int64_t ctas,
                 double budget_s) {
  c10::cuda::CUDAGuard g(master.device());
  FusedARArgs a;
  a.world = (int)world;
  a.rank = (int)rank;
  a.peer_grads = const_cast<const void* const*>(grads->device_ptrs());
  a.peer_values = values->device_ptrs();
  a.peer_flags = reinterpret_cast<uint32_t* const*>(flags->device_ptrs());
  a.my_flags = static_cast<uint32_t*>(flags->local());
  a.cta_counter = reinterpret_cast<unsigned int*>(counters.data_ptr<int>()) + bucket;
  a.start = start;
  a.end = end;
  a.bucket = (int)bucket;
  a.master = master.data_ptr<float>();
  a.m = m.has_value() ? m->data_ptr<float>() : nullptr;
  a.v = v.has_value() ? v->data_ptr<float>() : nullptr;
  a.hyper = reinterpret_cast<const OptimHyper*>(hyper.data_ptr());
  a.kind = (int)kind;
  a.scale = 1.f / (float)world;
  a.epoch_ptr = epoch.data_ptr<int64_t>();
  a.one_shot = one_shot ? 1 : 0;
  a.values_are_master = values_are_master ? 1 : 0;
  a.err = device_error_word();
  a.budget_ns = (uint64_t)(budget_s * 1e9);
  fused_allreduce_optimizer(a, grad_code == 0 ? DType::F32 : DType::BF16, value_code == 0 ? DType::F32 : DType::BF16,
                            (int)ctas, stream());
}

// NVLS two-shot variant: `grads` and `values` carry NVLink-multicast
// addresses (SymmetricBuffer views of multicast-bound memory).
void fused_ar_nvls_op(std::shared_ptr<SymmetricBuffer> grads, std::shared_ptr<SymmetricBuffer> values,
                      std::shared_ptr<SymmetricBuffer> flags, const at::Tensor& counters, int64_t bucket, int64_t start,
                      int64_t end, const at::Tensor& master, c10::optional<at::Tensor> m, c10::optional<at::Tensor> v,
                      const at::Tensor& hyper, int64_t kind, const at::Tensor& epoch, int64_t world, int64_t rank,
                      bool values_are_master, int64_t value_code, int64_t ctas, double budget_s) {
  c10::cuda::CUDAGuard g(master.device());
  TORCH_CHECK(grads->multicast() != nullptr && values->multicast() != nullptr,
              "NVLS all-reduce: the buffers have no multicast mapping");
  FusedARArgs a;
  a.world = (int)world;
  a.rank = (int)rank;
  a.peer_grads = const_cast<const void* const*>(grads->device_ptrs());
  a.peer_values = values->device_ptrs();
  a.peer_flags = reinterpret_cast<uint32_t* const*>(flags->device_ptrs());
  a.my_flags = static_cast<uint32_t*>(flags->local());
  a.cta_counter = reinterpret_cast<unsigned int*>(counters.data_ptr<int>()) + bucket;
  a.start = start;
  a.end = end;
  a.bucket = (int)bucket;
  a.master = master.data_ptr<float>();
  a.m = m.has_value() ? m->data_ptr<float>() : nullptr;
  a.v = v.has_value() ? v->data_ptr<float>() : nullptr;
  a.hyper = reinterpret_cast<const OptimHyper*>(hyper.data_ptr());
  a.kind = (int)kind;
  a.scale = 1.f / (float)world;
  a.epoch_ptr = epoch.data_ptr<int64_t>();
  a.values_are_master = values_are_master ? 1 : 0;
  a.err = device_error_word();
  a.budget_ns = (uint64_t)(budget_s * 1e9);
  a.mc_grads = grads->multicast();
  a.mc_values = values->multicast();
  fused_allreduce_optimizer_nvls(a, value_code == 0 ? DType::F32 : DType::BF16, (int)ctas, stream());
}

// Push two-shot variant: `recv` holds world-1 slots of recv_slot gradient
// elements; `cflags` is the [PUSH_MAX_BUCKETS][PUSH_MAX_CHUNKS][world] table.
void fused_ar_push_op(std::shared_ptr<SymmetricBuffer> grads, std::shared_ptr<SymmetricBuffer> values,
                      std::shared_ptr<SymmetricBuffer> flags, std::shared_ptr<SymmetricBuffer> recv,
                      std::shared_ptr<SymmetricBuffer> cflags, const at::Tensor& counters, int64_t bucket,
                      int64_t cbucket, int64_t start, int64_t end, int64_t recv_off, int64_t recv_slot,
                      const at::Tensor& master, c10::optional<at::Tensor> m, c10::optional<at::Tensor> v,
                      const at::Tensor& hyper, int64_t kind, const at::Tensor& epoch, int64_t world, int64_t rank,
                      bool values_are_master, int64_t grad_code, int64_t value_code, int64_t ctas,
                      double budget_s) {
  c10::cuda::CUDAGuard g(master.device());
  const int64_t gsz = grad_code == 0 ? 4 : 2;
  TORCH_CHECK((world - 1) * recv_slot * gsz <= recv->bytes(), "push all-reduce: receive buffer too small");
  TORCH_CHECK((int64_t)PUSH_MAX_BUCKETS * PUSH_MAX_CHUNKS * world * 4 <= cflags->bytes(),
              "push all-reduce: chunk-flag buffer too small");
  FusedARArgs a;
  a.world = (int)world;
  a.rank = (int)rank;
  a.peer_grads = const_cast<const void* const*>(grads->device_ptrs());
  a.peer_values = values->device_ptrs();
  a.peer_flags = reinterpret_cast<uint32_t* const*>(flags->device_ptrs());
  a.my_flags = static_cast<uint32_t*>(flags->local());
  a.cta_counter = reinterpret_cast<unsigned int*>(counters.data_ptr<int>()) + bucket;
  a.start = start;
  a.end = end;
  a.bucket = (int)bucket;
  a.master = master.data_ptr<float>();
  a.m = m.has_value() ? m->data_ptr<float>() : nullptr;
  a.v = v.has_value() ? v->data_ptr<float>() : nullptr;
  a.hyper = reinterpret_cast<const OptimHyper*>(hyper.data_ptr());
  a.kind = (int)kind;
  a.scale = 1.f / (float)world;
  a.epoch_ptr = epoch.data_ptr<int64_t>();
  a.values_are_master = values_are_master ? 1 : 0;
  a.err = device_error_word();
  a.budget_ns = (uint64_t)(budget_s * 1e9);
  a.peer_recv = recv->device_ptrs();
  a.my_recv = recv->local();
  a.recv_off = recv_off;
  a.recv_slot = recv_slot;
  a.peer_cflags = reinterpret_cast<uint32_t* const*>(cflags->device_ptrs());
  a.my_cflags = static_cast<uint32_t*>(cflags->local());
  a.cbucket = (int)cbucket;
  const int64_t n = end - start;
  a.chunk = push_chunk_elems(((n + world - 1) / world + 63) / 64 * 64, (int)ctas);
  fused_allreduce_optimizer_push(a, grad_code == 0 ? DType::F32 : DType::BF16,
                                 value_code == 0 ? DType::F32 : DType::BF16, stream());
}

// LL one-shot variant: `ll` holds [2][world-1][ll_cap] 8-byte words.
void fused_ar_ll_op(std::shared_ptr<SymmetricBuffer> grads, std::shared_ptr<SymmetricBuffer> values,
                    std::shared_ptr<SymmetricBuffer> ll, int64_t start, int64_t end, int64_t ll_off, int64_t ll_cap,
                    const at::Tensor& master, c10::optional<at::Tensor> m, c10::optional<at::Tensor> v,
                    const at::Tensor& hyper, int64_t kind, const at::Tensor& epoch, int64_t world, int64_t rank,
                    bool values_are_master, int64_t value_code, int64_t ctas, double budget_s) {
  c10::cuda::CUDAGuard g(master.device());
  TORCH_CHECK(2 * (world - 1) * ll_cap * 8 <= ll->bytes(), "LL all-reduce: buffer too small");
  FusedARArgs a;
  a.world = (int)world;
  a.rank = (int)rank;
  a.peer_grads = const_cast<const void* const*>(grads->device_ptrs());
  a.peer_values = values->device_ptrs();
  a.start = start;
  a.end = end;
  a.master = master.data_ptr<float>();
  a.m = m.has_value() ? m->data_ptr<float>() : nullptr;
  a.v = v.has_value() ? v->data_ptr<float>() : nullptr;
  a.hyper = reinterpret_cast<const OptimHyper*>(hyper.data_ptr());
  a.kind = (int)kind;
  a.scale = 1.f / (float)world;
  a.epoch_ptr = epoch.data_ptr<int64_t>();
  a.one_shot = 1;
  a.values_are_master = values_are_master ? 1 : 0;
  a.err = device_error_word();
  a.budget_ns = (uint64_t)(budget_s * 1e9);
  a.peer_ll = ll->device_ptrs();
  a.my_ll = ll->local();
  a.ll_off = ll_off;
  a.ll_cap = ll_cap;
  fused_allreduce_optimizer_ll(a, value_code == 0 ? DType::F32 : DType::BF16, (int)ctas, stream());
}

void p2p_allreduce_op(std::shared_ptr<SymmetricBuffer> data, std::shared_ptr<SymmetricBuffer> flags,
                      const at::Tensor& counters, int64_t slot, int64_t start, int64_t end, const at::Tensor& epoch,
                      int64_t world, int64_t rank, int64_t dtype_code, bool average, int64_t ctas, double budget_s) {
  c10::cuda::CUDAGuard g(epoch.device());
  FusedARArgs a;
  a.world = (int)world;
  a.rank = (int)rank;
  a.peer_grads = const_cast<const void* const*>(data->device_ptrs());
  a.peer_flags = reinterpret_cast<uint32_t* const*>(flags->device_ptrs());
  a.my_flags = static_cast<uint32_t*>(flags->local());
  a.cta_counter = reinterpret_cast<unsigned int*>(counters.data_ptr<int>()) + slot;
  a.start = start;
  a.end = end;
  a.bucket = (int)slot;
  a.epoch_ptr = epoch.data_ptr<int64_t>();
  a.err = device_error_word();
  a.budget_ns = (uint64_t)(budget_s * 1e9);
  p2p_allreduce(a, dtype_code == 0 ? DType::F32 : DType::BF16, average, (int)ctas, stream());
}

// Broadcast / all-gather / reduce-scatter of the staging buffer `data`
// into the local tensor `out` (mode 0 / 1 / 2; see p2p_collective).
void p2p_collective_op(std::shared_ptr<SymmetricBuffer> data, std::shared_ptr<SymmetricBuffer> flags,
                       const at::Tensor& counters, int64_t slot, const at::Tensor& out, int64_t numel, int64_t mode,
                       int64_t root, const at::Tensor& epoch, int64_t world, int64_t rank, int64_t dtype_code,
                       int64_t ctas, double budget_s) {
  c10::cuda::CUDAGuard g(epoch.device());
  const int64_t esz = dtype_code == 0 ? 4 : 2;
  TORCH_CHECK(numel * esz <= data->bytes(), "p2p collective: staging buffer too small");
  TORCH_CHECK(out.is_cuda() && out.is_contiguous(), "p2p collective: contiguous CUDA output");
  const int64_t need = mode == 1 ? numel * world : (mode == 2 ? (numel + world - 1) / world : numel);
  TORCH_CHECK(out.numel() >= need && out.element_size() == esz, "p2p collective: output too small or wrong dtype");
  FusedARArgs a;
  a.world = (int)world;
  a.rank = (int)rank;
  a.peer_grads = const_cast<const void* const*>(data->device_ptrs());
  a.peer_flags = reinterpret_cast<uint32_t* const*>(flags->device_ptrs());
  a.my_flags = static_cast<uint32_t*>(flags->local());
  a.cta_counter = reinterpret_cast<unsigned int*>(counters.data_ptr<int>()) + slot;
  a.bucket = (int)slot;
  a.epoch_ptr = epoch.data_ptr<int64_t>();
  a.err = device_error_word();
  a.budget_ns = (uint64_t)(budget_s * 1e9);
  p2p_collective(a, dtype_code == 0 ? DType::F32 : DType::BF16, (int)mode, (int)root, out.data_ptr(), numel,
                 (int)ctas, stream());
}

}  // namespace

void register_comm(py::module& m) {
  auto c = m.def_submodule("comm", "NVLink peer-memory communication");
  py::class_<SymmetricBuffer, std::shared_ptr<SymmetricBuffer>>(c, "SymmetricBuffer")
      .def(py::init<int64_t, int>(), py::arg("bytes"), py::arg("device"))
      .def(py::init<const std::vector<uint64_t>&, int, int64_t, int, uint64_t>(), py::arg("ptrs"), py::arg("rank"),
           py::arg("bytes"), py::arg("device"), py::arg("multicast") = 0)
      .def("multicast_ptr", [](const SymmetricBuffer& b) { return (int64_t)(uintptr_t)b.multicast(); })
      .def("handle", [](const SymmetricBuffer& b) { return py::bytes(b.handle()); })
      .def("open",
           [](SymmetricBuffer& b, const std::vector<py::bytes>& hs, int rank) {
             std::vector<std::string> v;
             for (auto& h : hs) v.push_back(std::string(h));
             b.open(v, rank);
           })
      .def("local_ptr", [](const SymmetricBuffer& b) { return (int64_t)(uintptr_t)b.local(); })
      .def("nbytes", &SymmetricBuffer::bytes)
      .def("tensor",
           [](std::shared_ptr<SymmetricBuffer> b, int code, int64_t numel, int64_t byte_offset) {
             auto st = scalar_of(code);
             const int64_t esz = c10::elementSize(st);
             TORCH_CHECK(byte_offset + numel * esz <= b->bytes(), "SymmetricBuffer.tensor: out of range");
             auto opts = at::TensorOptions().dtype(st).device(at::kCUDA, b->device());
             // The deleter keeps the buffer alive as long as any view exists.
             return torch::from_blob(static_cast<char*>(b->local()) + byte_offset, {numel},
                                     [b](void*) mutable { b.reset(); }, opts);
           },
           py::arg("dtype_code"), py::arg("numel"), py::arg("byte_offset") = 0);
  c.def("fused_allreduce_optimizer", &fused_ar_op);
  c.def("fused_allreduce_optimizer_push", &fused_ar_push_op);
  c.def("fused_allreduce_optimizer_ll", &fused_ar_ll_op);
  c.def("fused_allreduce_optimizer_nvls", &fused_ar_nvls_op);
  c.attr("PUSH_MAX_BUCKETS") = PUSH_MAX_BUCKETS;
  c.attr("PUSH_MAX_CHUNKS") = PUSH_MAX_CHUNKS;
  c.def("p2p_allreduce", &p2p_allreduce_op);
  c.def("p2p_collective", &p2p_collective_op);
  c.def("wait_flag_probe", [](const at::Tensor& flag, int64_t epoch, double budget_s) {
    TORCH_CHECK(flag.is_cuda() && flag.scalar_type() == at::kInt && flag.numel() >= 1, "wait_flag_probe: int32 flag");
    c10::cuda::CUDAGuard g(flag.device());
    auto res = at::zeros({1}, flag.options());
    wait_flag_probe(reinterpret_cast<const uint32_t*>(flag.data_ptr<int>()), (uint32_t)epoch,
                    (uint64_t)(budget_s * 1e9), device_error_word(), res.data_ptr<int>(), stream());
    return res;
  });
  c.def("can_access_peer", [](int a, int b) {
    int ok = 0;
    DLVK_CUDA_CHECK(cudaDeviceCanAccessPeer(&ok, a, b));
    return ok != 0;
  });
}

}  // namespace bind
}  // namespace dlvk
