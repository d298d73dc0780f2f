// Thin PyTorch binding over the C ABI (include/trring.h).  It owns the device buffers the C
// library never allocates (packed cores, workspace) as torch tensors, so PyTorch's allocation
// counters see them, and it launches on the caller's current CUDA stream.
//
// The bound object's __call__ is the callable that prepare_optimized returns
// (factorized_inference/submission.py:26-48): no Python frame runs per call.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <cstdlib>
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
    // TRR_CHECK_STATUS=1: after every call, read the workspace status word (a stream
    // synchronisation) and raise if a bounded device-side wait gave up.  Debugging aid.
    const char* chk = std::getenv("TRR_CHECK_STATUS");
    check_status_ = chk && chk[0] == '1';
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

  at::Tensor forward_impl(const at::Tensor& xin, const tr_tiling* tiling,
                          int kind = TR_EPI_NONE, const at::Tensor* auxin = nullptr,
                          bool out_f32 = false) {
    if (xin.dim() != 2 || xin.size(1) != d_in_)
      throw py::value_error("Expected x with shape [tokens, " + std::to_string(d_in_) + "]");
    if (!xin.is_cuda() || xin.get_device() != device_)
      throw py::value_error("x must be a CUDA tensor on the plan's device");
    if (xin.scalar_type() != dtype_) throw py::value_error("x dtype must match the cores");
    if (!packed_.defined()) throw std::runtime_error("cores are not packed");
    const at::Tensor x = xin.is_contiguous() ? xin : xin.contiguous();
    const int64_t T = x.size(0);
    at::Tensor aux;
    if (kind != TR_EPI_NONE) {
      if (!auxin) throw py::value_error("the epilogue needs a second operand");
      if (auxin->dim() != 2 || auxin->size(0) != T || auxin->size(1) != d_out_)
        throw py::value_error("Expected the epilogue operand with shape [" + std::to_string(T) +
                              ", " + std::to_string(d_out_) + "]");
      if (!auxin->is_cuda() || auxin->get_device() != device_)
        throw py::value_error("the epilogue operand must be a CUDA tensor on the plan's device");
      if (auxin->scalar_type() != dtype_ && auxin->scalar_type() != at::kFloat)
        throw py::value_error("the epilogue operand must be float32 or the cores' dtype");
      aux = auxin->is_contiguous() ? *auxin : auxin->contiguous();
    }
    c10::cuda::OptionalCUDAGuard guard;
    if (c10::cuda::current_device() != device_) guard.set_index((c10::DeviceIndex)device_);
    at::Tensor y = at::empty({T, d_out_}, x.options().dtype(out_f32 ? at::kFloat : dtype_));
    if (T == 0) return y;
    size_t need = 0;
    int st = tr_workspace_bytes_tiled(plan_.get(), T, tiling, &need);
    if (st != TR_OK) raise_status(st, "tr_workspace_bytes");
    if (need > ws_bytes_) {
      ws_ = at::zeros({(int64_t)need}, at::TensorOptions().dtype(at::kByte).device(x.device()));
      ws_bytes_ = need;
    }
    cudaStream_t stream = at::cuda::getCurrentCUDAStream((c10::DeviceIndex)device_).stream();
    if (kind == TR_EPI_NONE && !out_f32) {
      st = tr_forward_tiled(plan_.get(), packed_.data_ptr(), x.data_ptr(), T, y.data_ptr(),
                            ws_bytes_ ? ws_.data_ptr() : nullptr, ws_bytes_, tiling, stream);
      if (st != TR_OK) raise_status(st, "tr_forward");
      if (check_status_) check_device_status();
      return y;
    }
    tr_epilogue e;
    e.kind = kind;
    e.out_dtype = out_f32 ? TR_F32 : dtype_code(dtype_);
    e.aux = aux.defined() ? aux.data_ptr() : nullptr;
    e.aux_dtype = aux.defined() ? dtype_code(aux.scalar_type()) : TR_F32;
    st = tr_forward_epilogue(plan_.get(), packed_.data_ptr(), x.data_ptr(), T, y.data_ptr(), &e,
                             ws_bytes_ ? ws_.data_ptr() : nullptr, ws_bytes_, tiling, stream);
    if (st != TR_OK) raise_status(st, "tr_forward_epilogue");
    if (check_status_) check_device_status();
    return y;
  }

  // The workspace's device status word (TR_OK, or TR_ERR_TIMEOUT after a bounded wait gave
  // up); synchronises the current stream; `reset` clears the word.
  int64_t workspace_status(bool reset) {
    int32_t status = TR_OK;
    if (ws_bytes_ == 0) return TR_OK;
    c10::cuda::CUDAGuard guard((c10::DeviceIndex)device_);
    const int st = tr_workspace_status(
        ws_.data_ptr(), ws_bytes_, &status, reset ? 1 : 0,
        at::cuda::getCurrentCUDAStream((c10::DeviceIndex)device_).stream());
    if (st != TR_OK) raise_status(st, "tr_workspace_status");
    return status;
  }

  void check_device_status() {
    const int64_t status = workspace_status(true);
    if (status != TR_OK)
      throw std::runtime_error(std::string("tensor-ring kernel: ") +
                               tr_status_string((int)status) + " (the call's output is not valid)");
  }

  // Polls of a bounded device-side wait before it gives up (0 = built-in limit).
  void set_wait_limit(int64_t polls) {
    const int st = tr_plan_set_wait_limit(plan_.get(), (uint32_t)polls);
    if (st != TR_OK) raise_status(st, "tr_plan_set_wait_limit");
  }

  at::Tensor call(const at::Tensor& x) { return forward_impl(x, nullptr); }

  // y = TR(x) for a host-resident x (tr_forward_host): one call issues the copy of x to the
  // device, the forward and the copy of y back, on the current stream, and returns `out` (or a
  // new page-locked tensor) before they finish: synchronise the stream before reading it.  The
  // device staging buffers belong to this object and are reused by its next call.
  at::Tensor forward_host(const at::Tensor& x, c10::optional<at::Tensor> out) {
    if (x.dim() != 2 || x.size(1) != d_in_)
      throw py::value_error("Expected x with shape [tokens, " + std::to_string(d_in_) + "]");
    if (x.is_cuda()) throw py::value_error("forward_host takes x in host memory");
    if (x.scalar_type() != dtype_) throw py::value_error("x dtype must match the cores");
    if (!x.is_contiguous()) throw py::value_error("x must be contiguous");
    if (!packed_.defined()) throw std::runtime_error("cores are not packed");
    const int64_t T = x.size(0);
    at::Tensor y;
    if (out.has_value()) {
      y = *out;
      if (y.is_cuda() || y.dim() != 2 || y.size(0) != T || y.size(1) != d_out_ ||
          y.scalar_type() != dtype_ || !y.is_contiguous())
        throw py::value_error("out must be a contiguous host tensor [tokens, " +
                              std::to_string(d_out_) + "] of the cores' dtype");
    } else {
      y = at::empty({T, d_out_}, x.options().pinned_memory(true));
    }
    if (T == 0) return y;
    c10::cuda::OptionalCUDAGuard guard;
    if (c10::cuda::current_device() != device_) guard.set_index((c10::DeviceIndex)device_);
    const auto dev = at::TensorOptions().dtype(at::kByte).device(at::kCUDA,
                                                                  (c10::DeviceIndex)device_);
    const size_t es = x.element_size();
    const size_t xb = (size_t)T * d_in_ * es, yb = (size_t)T * d_out_ * es;
    if (xb > xs_bytes_) {
      xs_ = at::empty({(int64_t)xb}, dev);
      xs_bytes_ = xb;
    }
    if (yb > ys_bytes_) {
      ys_ = at::empty({(int64_t)yb}, dev);
      ys_bytes_ = yb;
    }
    size_t need = 0;
    int st = tr_workspace_bytes(plan_.get(), T, &need);
    if (st != TR_OK) raise_status(st, "tr_workspace_bytes");
    if (need > ws_bytes_) {
      ws_ = at::zeros({(int64_t)need}, dev);
      ws_bytes_ = need;
    }
    cudaStream_t stream = at::cuda::getCurrentCUDAStream((c10::DeviceIndex)device_).stream();
    st = tr_forward_host(plan_.get(), packed_.data_ptr(), x.data_ptr(), T, y.data_ptr(),
                         xs_.data_ptr(), ys_.data_ptr(), ws_bytes_ ? ws_.data_ptr() : nullptr,
                         ws_bytes_, stream);
    if (st != TR_OK) raise_status(st, "tr_forward_host");
    if (check_status_) check_device_status();
    return y;
  }

  // y in fp32, no rounding to the cores' dtype (the reference's accumulate / forward_fp32)
  at::Tensor accumulate(const at::Tensor& x) {
    return forward_impl(x, nullptr, TR_EPI_NONE, nullptr, true);
  }
  // h + TR(x) in the cores' dtype (residual add fused into the forward kernel)
  at::Tensor forward_add(const at::Tensor& x, const at::Tensor& h) {
    return forward_impl(x, nullptr, TR_EPI_ADD, &h, false);
  }
  // silu(g) * TR(x) in the cores' dtype (gated MLP fused into the up projection)
  at::Tensor forward_silu_mul(const at::Tensor& x, const at::Tensor& g) {
    return forward_impl(x, nullptr, TR_EPI_SILU_MUL, &g, false);
  }
  // any epilogue with an explicit geometry (kernel 0 = planner's choice)
  at::Tensor call_epilogue(const at::Tensor& x, int64_t kind, c10::optional<at::Tensor> aux,
                           bool out_fp32, int64_t kernel, int64_t tokens_per_tile,
                           int64_t cluster, int64_t clusters) {
    tr_tiling t;
    t.kernel = (int32_t)kernel;
    t.tokens_per_tile = (int32_t)tokens_per_tile;
    t.cluster = (int32_t)cluster;
    t.clusters = (int32_t)clusters;
    const at::Tensor* a = aux.has_value() ? &aux.value() : nullptr;
    return forward_impl(x, kernel ? &t : nullptr, (int)kind, a, out_fp32);
  }

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
  at::Tensor xs_, ys_;  // device staging of forward_host
  size_t xs_bytes_ = 0, ys_bytes_ = 0;
  bool check_status_ = false;
};

void check_consume_f32(const at::Tensor& t, const at::Tensor& like, const char* what) {
  if (!t.is_cuda() || t.scalar_type() != at::kFloat || !t.is_contiguous() ||
      t.sizes() != like.sizes() || t.get_device() != like.get_device())
    throw py::value_error(std::string(what) + ": FP32 contiguous CUDA tensors of one shape");
}

// silu(g) * u in `dtype` (bf16 like the reference by default); g and u are cleared
at::Tensor consume_silu_mul(at::Tensor g, at::Tensor u, at::ScalarType dtype) {
  check_consume_f32(g, g, "consume_silu_mul");
  check_consume_f32(u, g, "consume_silu_mul");
  const int code = dtype_code(dtype);
  if (code != TR_F16 && code != TR_BF16)
    throw py::value_error("consume_silu_mul: output dtype float16 or bfloat16");
  c10::cuda::CUDAGuard guard(g.device());
  at::Tensor out = at::empty(g.sizes(), g.options().dtype(dtype));
  const int st = tr_consume_silu_mul(g.data_ptr<float>(), u.data_ptr<float>(), out.data_ptr(),
                                     code, g.numel(), at::cuda::getCurrentCUDAStream().stream());
  if (st != TR_OK) raise_status(st, "tr_consume_silu_mul");
  return out;
}

// h + y in h's dtype; y (fp32) is cleared
at::Tensor consume_add(at::Tensor h, at::Tensor y) {
  check_consume_f32(y, h, "consume_add");
  const int code = dtype_code(h.scalar_type());
  if (code != TR_F16 && code != TR_BF16)
    throw py::value_error("consume_add: h must be float16 or bfloat16");
  if (!h.is_contiguous()) throw py::value_error("consume_add: h must be contiguous");
  c10::cuda::CUDAGuard guard(h.device());
  at::Tensor out = at::empty_like(h);
  const int st = tr_consume_add(h.data_ptr(), y.data_ptr<float>(), out.data_ptr(), code,
                                h.numel(), at::cuda::getCurrentCUDAStream().stream());
  if (st != TR_OK) raise_status(st, "tr_consume_add");
  return out;
}

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
      .def("forward_host", &RingOp::forward_host, py::arg("x"), py::arg("out") = py::none())
      .def("accumulate", &RingOp::accumulate)
      .def("forward_add", &RingOp::forward_add, py::arg("x"), py::arg("h"))
      .def("forward_silu_mul", &RingOp::forward_silu_mul, py::arg("x"), py::arg("g"))
      .def("call_epilogue", &RingOp::call_epilogue, py::arg("x"), py::arg("kind"),
           py::arg("aux") = py::none(), py::arg("out_fp32") = false, py::arg("kernel") = 0,
           py::arg("tokens_per_tile") = 0, py::arg("cluster") = 0, py::arg("clusters") = 0)
      .def("call_tiled", &RingOp::call_tiled, py::arg("x"), py::arg("kernel") = 0,
           py::arg("tokens_per_tile") = 0, py::arg("cluster") = 0, py::arg("clusters") = 0)
      .def("tiling", &RingOp::tiling)
      .def("describe", &RingOp::describe)
      .def("flops_per_token", &RingOp::flops_per_token)
      .def("workspace_bytes", &RingOp::workspace_bytes)
      .def("workspace_status", &RingOp::workspace_status, py::arg("reset") = true)
      .def("set_wait_limit", &RingOp::set_wait_limit, py::arg("polls"))
      .def_property_readonly("packed", &RingOp::packed)
      .def_property_readonly("workspace", &RingOp::workspace);
  m.def("empty_launch", &empty_launch, "launch an empty kernel on the current stream");
  m.def("consume_silu_mul", &consume_silu_mul, py::arg("g"), py::arg("u"),
        py::arg("dtype") = at::kBFloat16, "silu(g) * u (fp32 inputs, cleared) -> dtype");
  m.def("consume_add", &consume_add, py::arg("h"), py::arg("y"),
        "h + y (y fp32, cleared) -> h's dtype");
}
