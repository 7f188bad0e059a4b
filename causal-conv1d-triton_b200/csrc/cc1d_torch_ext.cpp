// Torch-side launchers of the forward and backward (the reference's `_fwd` and `_bwd`,
// causal_conv1d_triton/causal_conv1d.py:433-541): output and workspace allocation through
// torch's caching allocator, the device guard, torch's current stream, then the C ABI of
// include/causal_conv1d_b200.h. Host C++ only (no device code); the C ABI stays free of torch
// types, and this module is the package's layer above it.
//
// Written in C++ because the launchers run once per call: at small shapes (
// kernels of a few microseconds) three Python-level allocations and the argument handling of the
// backward cost more host time than the library call itself.
//
// Each function returns the C ABI's result code first; the Python caller turns a non-zero code
// into its error (the same messages as the library's cc1d_error_string).
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <tuple>

#include "causal_conv1d_b200.h"

namespace {

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return CC1D_F32;
    case at::kHalf: return CC1D_F16;
    case at::kBFloat16: return CC1D_BF16;
    default: return -1;
  }
}

// Parameters in a float type the kernels do not read (e.g. float64) are passed as fp32.
at::Tensor as_float(const at::Tensor& t) { return dtype_code(t.scalar_type()) < 0 ? t.to(at::kFloat) : t; }

c10::optional<at::Tensor> as_float(const c10::optional<at::Tensor>& t) {
  if (!t.has_value()) return t;
  return as_float(*t);
}

const void* ptr(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }
void* mptr(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }
int code(const c10::optional<at::Tensor>& t) { return t.has_value() ? dtype_code(t->scalar_type()) : 0; }

// (rc, out)
std::tuple<int, at::Tensor> fwd(const at::Tensor& x, const at::Tensor& weight, const c10::optional<at::Tensor>& bias,
                                const c10::optional<at::Tensor>& seq_idx,
                                const c10::optional<at::Tensor>& initial_states,
                                const c10::optional<at::Tensor>& final_states, bool silu) {
  const int64_t B = x.size(0), T = x.size(1), D = x.size(2), W = weight.size(1);
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor out = at::empty({B, T, D}, x.options());
  const at::Tensor w = as_float(weight);
  const c10::optional<at::Tensor> b = as_float(bias), init = as_float(initial_states);
  const int rc = cc1d_fwd(x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), ptr(b), ptr(init),
                          static_cast<const int32_t*>(ptr(seq_idx)), out.data_ptr(), mptr(final_states), B, T, D, W,
                          dtype_code(x.scalar_type()), dtype_code(w.scalar_type()), code(b), code(init), silu ? 1 : 0,
                          c10::cuda::getCurrentCUDAStream(x.device().index()).stream());
  return {rc, out};
}

// (rc, dx, dweight, dbias, dinit). With grad_f32 the weight/bias gradients go there as
// [dweight (D, W), dbias (D)] and dweight/dbias are None. With fp32 weight and bias and
// fuse_param_grads, dweight and dbias are views of one fp32 buffer written the same way.
std::tuple<int, at::Tensor, c10::optional<at::Tensor>, c10::optional<at::Tensor>, c10::optional<at::Tensor>> bwd(
    const at::Tensor& x, const at::Tensor& weight, const c10::optional<at::Tensor>& bias,
    const c10::optional<at::Tensor>& seq_idx, const c10::optional<at::Tensor>& initial_states, const at::Tensor& dout,
    const c10::optional<at::Tensor>& dfinal_states, bool need_dinit, bool silu,
    const c10::optional<at::Tensor>& grad_f32, bool fuse_param_grads) {
  const int64_t B = x.size(0), T = x.size(1), D = x.size(2), W = weight.size(1);
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor dx = at::empty({B, T, D}, x.options());
  if (need_dinit && !initial_states.has_value()) return {CC1D_ERR_INVALID, dx, c10::nullopt, c10::nullopt, c10::nullopt};
  c10::optional<at::Tensor> dinit;
  if (need_dinit) dinit = at::empty_like(*initial_states);
  const at::Tensor w = as_float(weight);
  const c10::optional<at::Tensor> b = as_float(bias), init = as_float(initial_states), dinit_k = as_float(dinit);
  c10::optional<at::Tensor> flat, dweight, dbias;
  if (!grad_f32.has_value()) {
    if (fuse_param_grads && weight.scalar_type() == at::kFloat &&
        (!bias.has_value() || bias->scalar_type() == at::kFloat)) {
      flat = at::empty({D * (W + 1)}, x.options().dtype(at::kFloat));
    } else {
      dweight = at::empty_like(w);
      if (b.has_value()) dbias = at::empty_like(*b);
    }
  }
  c10::optional<at::Tensor> dfinal = dfinal_states;
  if (dfinal.has_value() && dfinal->scalar_type() != x.scalar_type()) dfinal = dfinal->to(x.scalar_type());
  const int xdt = dtype_code(x.scalar_type());
  const int64_t ws_bytes = cc1d_bwd_workspace_bytes(x.data_ptr(), x.stride(0), x.stride(1), dout.data_ptr(),
                                                    dout.stride(0), dout.stride(1), B, T, D, W, xdt);
  if (ws_bytes < 0) return {CC1D_ERR_INVALID, dx, c10::nullopt, c10::nullopt, c10::nullopt};
  const at::Tensor workspace = at::empty({std::max<int64_t>(1, ws_bytes / 4)}, x.options().dtype(at::kFloat));
  float* g32 = grad_f32.has_value() ? grad_f32->data_ptr<float>() : (flat.has_value() ? flat->data_ptr<float>() : nullptr);
  const int rc = cc1d_bwd(x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), ptr(b), ptr(init),
                          static_cast<const int32_t*>(ptr(seq_idx)), dout.data_ptr(), dout.stride(0), dout.stride(1),
                          ptr(dfinal), dx.data_ptr(), mptr(dweight), mptr(dbias), mptr(dinit_k), g32,
                          workspace.data_ptr(), ws_bytes, B, T, D, W, xdt, dtype_code(w.scalar_type()), code(b),
                          code(init), silu ? 1 : 0, c10::cuda::getCurrentCUDAStream(x.device().index()).stream());
  if (rc != CC1D_OK) return {rc, dx, c10::nullopt, c10::nullopt, c10::nullopt};
  if (dinit.has_value() && !dinit_k->is_same(*dinit)) dinit->copy_(*dinit_k);
  if (flat.has_value()) {
    dweight = flat->narrow(0, 0, D * W).view({D, W});
    if (bias.has_value()) dbias = flat->narrow(0, D * W, D);
  } else if (!grad_f32.has_value()) {
    if (dweight->scalar_type() != weight.scalar_type()) dweight = dweight->to(weight.scalar_type());
    if (dbias.has_value() && dbias->scalar_type() != bias->scalar_type()) dbias = dbias->to(bias->scalar_type());
  }
  return {rc, dx, dweight, dbias, dinit};
}

// Throws the library's error for a non-zero result code (inside the autograd Function, where the
// code cannot be handed back to Python).
void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == CC1D_OK, what, ": ", cc1d_error_string(rc), rc == CC1D_ERR_CUDA ? " (cudaError " : "",
              rc == CC1D_ERR_CUDA ? std::to_string(cc1d_last_cuda_error()) + ")" : std::string());
}

// `t` itself, or a contiguous copy when its channel stride is not 1 or when its rows could feed the
// TMA kernels (width <= 16, channels x element size a multiple of 16 bytes) but its base or
// batch/time strides are not 16-byte multiples (the rule of the package's _tma_layout).
at::Tensor tma_layout(const at::Tensor& t0, int64_t width) {
  const at::Tensor t = t0.stride(-1) == 1 ? t0 : t0.contiguous();
  const int64_t B = t.size(0), D = t.size(2), es = t.element_size();
  if (width > 16 || (D * es) % 16 != 0 || t.numel() == 0) return t;
  const bool aligned = reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0 && (t.stride(1) * es) % 16 == 0 &&
                       (B == 1 || (t.stride(0) * es) % 16 == 0);
  return aligned ? t : t.clone(at::MemoryFormat::Contiguous);
}

// The reference's `_CausalConv1dFn` (causal_conv1d.py:544-576) as a C++ autograd Function: the same
// saved tensors, the same need_dinit rule and the same gradients, without the Python-level
// Function machinery on every call. Absent tensors come in as empty optionals, which the autograd
// machinery treats as non-tensor arguments (no edge), so needs_input_grad counts only the tensors
// given.
struct ConvFn : public torch::autograd::Function<ConvFn> {
  static torch::autograd::variable_list forward(torch::autograd::AutogradContext* ctx, const at::Tensor& x,
                                                const at::Tensor& weight, const c10::optional<at::Tensor>& bias,
                                                const c10::optional<at::Tensor>& seq_idx,
                                                const c10::optional<at::Tensor>& initial_states,
                                                bool return_final_states, bool silu) {
    c10::optional<at::Tensor> final_states;
    if (return_final_states) final_states = at::empty({x.size(0), weight.size(1) - 1, x.size(2)}, x.options());
    auto [rc, out] = fwd(x, weight, bias, seq_idx, initial_states, final_states, silu);
    check_rc(rc, "causal_conv1d forward");
    ctx->save_for_backward({x, weight, bias.value_or(at::Tensor()), seq_idx.value_or(at::Tensor()),
                            initial_states.value_or(at::Tensor())});
    ctx->saved_data["silu"] = silu;
    ctx->saved_data["final"] = return_final_states;
    // Edge index of initial_states among the tensor inputs given (x, weight, [bias], [seq_idx]).
    ctx->saved_data["init_edge"] =
        static_cast<int64_t>(2 + (bias.has_value() ? 1 : 0) + (seq_idx.has_value() ? 1 : 0));
    if (return_final_states) return {out, *final_states};
    return {out};
  }

  static torch::autograd::variable_list backward(torch::autograd::AutogradContext* ctx,
                                                 torch::autograd::variable_list grads) {
    const auto saved = ctx->get_saved_variables();
    const at::Tensor &x = saved[0], &weight = saved[1], &bias = saved[2], &seq_idx = saved[3], &init = saved[4];
    auto opt = [](const at::Tensor& t) { return t.defined() ? c10::optional<at::Tensor>(t) : c10::nullopt; };
    const bool silu = ctx->saved_data["silu"].toBool(), ret_final = ctx->saved_data["final"].toBool();
    c10::optional<at::Tensor> dfinal;
    if (ret_final && grads.size() > 1 && grads[1].defined()) dfinal = grads[1].contiguous();
    const bool need_dinit =
        init.defined() && ctx->needs_input_grad(static_cast<size_t>(ctx->saved_data["init_edge"].toInt()));
    at::Tensor dout = grads[0];
    if (!dout.defined()) dout = at::zeros_like(x);
    dout = tma_layout(dout, weight.size(1));
    auto [rc, dx, dweight, dbias, dinit] =
        bwd(x, weight, opt(bias), opt(seq_idx), opt(init), dout, dfinal, need_dinit, silu, c10::nullopt, true);
    check_rc(rc, "causal_conv1d backward");
    return {dx, dweight.value_or(at::Tensor()), dbias.value_or(at::Tensor()), at::Tensor(),
            dinit.value_or(at::Tensor()), at::Tensor(), at::Tensor()};
  }
};

torch::autograd::variable_list conv_fn(const at::Tensor& x, const at::Tensor& weight,
                                       const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& seq_idx,
                                       const c10::optional<at::Tensor>& initial_states, bool return_final_states,
                                       bool silu) {
  return ConvFn::apply(x, weight, bias, seq_idx, initial_states, return_final_states, silu);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "torch-side launchers of libcausal_conv1d_b200 (forward and backward)";
  m.def("fwd", &fwd, "(rc, out) = fwd(x, weight, bias, seq_idx, initial_states, final_states, silu)");
  m.def("conv_fn", &conv_fn,
        "[out] or [out, final_states] = conv_fn(x, weight, bias, seq_idx, initial_states, return_final_states, "
        "silu): forward with autograd");
  m.def("bwd", &bwd,
        "(rc, dx, dweight, dbias, dinit) = bwd(x, weight, bias, seq_idx, initial_states, dout, dfinal_states, "
        "need_dinit, silu, grad_f32, fuse_param_grads)");
}
