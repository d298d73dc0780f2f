// Thin PyTorch binding over the C ABI (include/trring.h).  It owns the device buffers the C
// library never allocates (packed cores, workspace) as torch tensors, so PyTorch's allocation
// counters see them, and it launches on the caller's current CUDA stream.
//
// The bound object's __call__ is the callable that prepare_optimized returns
// (factorized_inference/submission.py:26-48): no Python frame runs per call.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/pybind11.h>
#include <torch/extension.h>

#include <memory>
#include <string>
#include <vector>

#include "trring.h"

namespace py = pybind11;

namespace {

[[noreturn]] void raise_status(int st, const char* what) {
  std::string msg = std::string(what) + ": " + tr_status_string(st) + " (" + tr_last_error() + ")";
  if (st == TR_ERR_INVALID) throw py::value_error(msg);
  throw std::runtime_error(msg);
}

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return TR_F32;
    case at::kHalf: return TR_F16;
    case at::kBFloat16: return TR_BF16;
    default: return -1;
  }
}

class RingOp {
 public:
  RingOp(std::vector<int64_t> in_modes, std::vector<int64_t> out_modes, int64_t rank,
         at::ScalarType dtype, int64_t device)
      : dtype_(dtype), device_((int)device) {
    if (in_modes.size() != 3 || out_modes.size() != 3)
      throw py::value_error("Exactly three input and output modes are required");
    tr_spec s;
    for (int k = 0; k < 3; ++k) {
      s.input_modes[k] = (int32_t)in_modes[k];
      s.output_modes[k] = (int32_t)out_modes[k];
    }
    s.rank = (int32_t)rank;
    const int code = dtype_code(dtype);
    if (code < 0) throw py::value_error("cores must be float32, float16 or bfloat16");
    tr_plan* p = nullptr;
    const int st = tr_plan_create(&s, code, device_, &p);
    if (st != TR_OK) raise_status(st, "tr_plan_create");
    plan_.reset(p);
    d_in_ = (int64_t)s.input_modes[0] * s.input_modes[1] * s.input_modes[2];
    d_out_ = (int64_t)s.output_modes[0] * s.output_modes[1] * s.output_modes[2];
    for (int k = 0; k < 3; ++k) {
      core_shapes_.push_back({rank, out_modes[k], in_modes[k], rank});
    }
  }

  // Pack the three cores; they are read, never modified or retained.
  void pack(const std::vector<at::Tensor>& cores) {
    if (cores.size() != 3) throw py::value_error("Expected three cores");
    const void* ptrs[3];
    for (int k = 0; k < 3; ++k) {
      const at::Tensor& c = cores[k];
      if (!c.is_cuda() || c.get_device() != device_)
        throw py::value_error("cores must be CUDA tensors on the plan's device");
      if (c.scalar_type() != dtype_) throw py::value_error("all cores must share one dtype");
      if (c.sizes().vec() != core_shapes_[k])
        throw py::value_error("Core " + std::to_string(k) + " has the wrong shape");
      if (!c.is_contiguous()) throw py::value_error("cores must be contiguous");
      ptrs[k] = c.data_ptr();
    }
    size_t bytes = 0;
    int st = tr_packed_bytes(plan_.get(), &bytes);
    if (st != TR_OK) raise_status(st, "tr_packed_bytes");
    c10::cuda::CUDAGuard guard((c10::DeviceIndex)device_);
    packed_ = at::empty({(int64_t)bytes}, at::TensorOptions().dtype(at::kByte).device(
                                              at::kCUDA, (c10::DeviceIndex)device_));
    st = tr_pack_cores(plan_.get(), ptrs, packed_.data_ptr(),
                       at::cuda::getCurrentCUDAStream((c10::DeviceIndex)device_).stream());
    if (st != TR_OK) raise_status(st, "tr_pack_cores");
  }

  at::Tensor forward_impl(const at::Tensor& xin, const tr_tiling* tiling) {
    if (xin.dim() != 2 || xin.size(1) != d_in_)
      throw py::value_error("Expected x with shape [tokens, " + std::to_string(d_in_) + "]");
    if (!xin.is_cuda() || xin.get_device() != device_)
      throw py::value_error("x must be a CUDA tensor on the plan's device");
    if (xin.scalar_type() != dtype_) throw py::value_error("x dtype must match the cores");
    if (!packed_.defined()) throw std::runtime_error("cores are not packed");
    const at::Tensor x = xin.is_contiguous() ? xin : xin.contiguous();
    const int64_t T = x.size(0);
    c10::cuda::OptionalCUDAGuard guard;
    if (c10::cuda::current_device() != device_) guard.set_index((c10::DeviceIndex)device_);
    at::Tensor y = at::empty({T, d_out_}, x.options());
    if (T == 0) return y;
    size_t need = 0;
    int st = tr_workspace_bytes_tiled(plan_.get(), T, tiling, &need);
    if (st != TR_OK) raise_status(st, "tr_workspace_bytes");
    if (need > ws_bytes_) {
      ws_ = at::zeros({(int64_t)need}, at::TensorOptions().dtype(at::kByte).device(x.device()));
      ws_bytes_ = need;
    }
    cudaStream_t stream = at::cuda::getCurrentCUDAStream((c10::DeviceIndex)device_).stream();
    st = tr_forward_tiled(plan_.get(), packed_.data_ptr(), x.data_ptr(), T, y.data_ptr(),
                          ws_bytes_ ? ws_.data_ptr() : nullptr, ws_bytes_, tiling, stream);
    if (st != TR_OK) raise_status(st, "tr_forward");
    return y;
  }

  at::Tensor call(const at::Tensor& x) { return forward_impl(x, nullptr); }

  at::Tensor call_tiled(const at::Tensor& x, int64_t kernel, int64_t tokens_per_tile,
                        int64_t cluster, int64_t clusters) {
    tr_tiling t;
    t.kernel = (int32_t)kernel;
    t.tokens_per_tile = (int32_t)tokens_per_tile;
    t.cluster = (int32_t)cluster;
    t.clusters = (int32_t)clusters;
    return forward_impl(x, &t);
  }

  py::dict tiling(int64_t T) const {
    tr_tiling t;
    const int st = tr_plan_tiling(plan_.get(), T, &t);
    if (st != TR_OK) raise_status(st, "tr_plan_tiling");
    py::dict d;
    d["kernel"] = t.kernel;
    d["tokens_per_tile"] = t.tokens_per_tile;
    d["cluster"] = t.cluster;
    d["clusters"] = t.clusters;
    return d;
  }

  std::string describe() const {
    char buf[1024];
    const int st = tr_plan_describe(plan_.get(), buf, sizeof(buf));
    if (st != TR_OK) raise_status(st, "tr_plan_describe");
    return std::string(buf);
  }

  double flops_per_token() const {
    double f = 0;
    const int st = tr_plan_flops_per_token(plan_.get(), &f);
    if (st != TR_OK) raise_status(st, "tr_plan_flops_per_token");
    return f;
  }

  int64_t workspace_bytes(int64_t T) const {
    size_t b = 0;
    const int st = tr_workspace_bytes(plan_.get(), T, &b);
    if (st != TR_OK) raise_status(st, "tr_workspace_bytes");
    return (int64_t)b;
  }

  at::Tensor packed() const { return packed_; }
  at::Tensor workspace() const { return ws_; }

 private:
  struct PlanDeleter {
    void operator()(tr_plan* p) const { tr_plan_destroy(p); }
  };
  std::unique_ptr<tr_plan, PlanDeleter> plan_;
  at::ScalarType dtype_;
  int device_;
  int64_t d_in_ = 0, d_out_ = 0;
  std::vector<std::vector<int64_t>> core_shapes_;
  at::Tensor packed_;
  at::Tensor ws_;
  size_t ws_bytes_ = 0;
};

void empty_launch() {
  const int st = tr_empty_launch(at::cuda::getCurrentCUDAStream().stream());
  if (st != TR_OK) raise_status(st, "tr_empty_launch");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "PyTorch binding of the trring C ABI (tensor-ring linear operator, sm_100a)";
  py::class_<RingOp>(m, "RingOp")
      .def(py::init<std::vector<int64_t>, std::vector<int64_t>, int64_t, at::ScalarType, int64_t>(),
           py::arg("input_modes"), py::arg("output_modes"), py::arg("rank"), py::arg("dtype"),
           py::arg("device"))
      .def("pack", &RingOp::pack)
      .def("__call__", &RingOp::call)
      .def("call_tiled", &RingOp::call_tiled, py::arg("x"), py::arg("kernel") = 0,
           py::arg("tokens_per_tile") = 0, py::arg("cluster") = 0, py::arg("clusters") = 0)
      .def("tiling", &RingOp::tiling)
      .def("describe", &RingOp::describe)
      .def("flops_per_token", &RingOp::flops_per_token)
      .def("workspace_bytes", &RingOp::workspace_bytes)
      .def_property_readonly("packed", &RingOp::packed)
      .def_property_readonly("workspace", &RingOp::workspace);
  m.def("empty_launch", &empty_launch, "launch an empty kernel on the current stream");
}
