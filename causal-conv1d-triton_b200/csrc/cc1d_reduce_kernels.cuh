// The deterministic second-stage reduction of the backward's per-CTA partial sums (both kernel
// paths) and the fill kernel for T == 0. Non-template kernels: included by cc1d_api.cu only.
//
// Reference: jxiong21029/causal-conv1d-triton, causal_conv1d_triton/causal_conv1d.py
// (`_reduce_partials_kernel` :344-374, empty-input handling in `_fwd` :437-444, `_bwd` :480-489).
#pragma once

#include "cc1d_device.cuh"

namespace cc1d {

// Second stage of the dweight/dbias reduction (causal_conv1d.py:344-374): column n = k * D + d of
// the (P, W+1, D) partials is summed over P in increasing P order, so the result does not depend
// on scheduling. Writes dweight[d, k] (k < W) and dbias[d] (k == W) in their own dtypes, or, when
// grad_f32 is given, the fp32 vector [dweight (D, W) row-major, dbias (D)] instead (its dbias
// part zero when there is no bias).
__global__ void __launch_bounds__(256) cc1d_reduce_partials_kernel(const float* __restrict__ partials, int P, int D, int W,
                                                                   void* dweight, int w_dtype, void* dbias, int b_dtype,
                                                                   float* grad_f32, int has_bias) {
  const int64_t N = static_cast<int64_t>(W + 1) * D;
  for (int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; n < N;
       n += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.0f;
    int q = 0;
    for (; q + 8 <= P; q += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(partials + (q + u) * N + n);
#pragma unroll
      for (int u = 0; u < 8; ++u) s += v[u];
    }
    for (; q < P; ++q) s += __ldg(partials + q * N + n);
    const int k = static_cast<int>(n / D), d = static_cast<int>(n - static_cast<int64_t>(k) * D);
    if (grad_f32 != nullptr) {
      if (k < W)
        grad_f32[static_cast<int64_t>(d) * W + k] = s;
      else
        grad_f32[static_cast<int64_t>(D) * W + d] = has_bias ? s : 0.0f;
    } else if (k < W) {
      st_any(dweight, static_cast<int64_t>(d) * W + k, w_dtype, s);
    } else if (dbias != nullptr) {
      st_any(dbias, d, b_dtype, s);
    }
  }
}

// dst[i] = src[i] converted (or 0 when src is null), i < n.
__global__ void cc1d_fill_kernel(void* dst, int dst_dtype, const void* src, int src_dtype, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    st_any(dst, i, dst_dtype, src != nullptr ? ld_any(src, i, src_dtype) : 0.0f);
}

}  // namespace cc1d
