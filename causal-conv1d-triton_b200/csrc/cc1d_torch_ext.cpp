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

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "torch-side launchers of libcausal_conv1d_b200 (forward and backward)";
  m.def("fwd", &fwd, "(rc, out) = fwd(x, weight, bias, seq_idx, initial_states, final_states, silu)");
  m.def("bwd", &bwd,
        "(rc, dx, dweight, dbias, dinit) = bwd(x, weight, bias, seq_idx, initial_states, dout, dfinal_states, "
        "need_dinit, silu, grad_f32, fuse_param_grads)");
}
