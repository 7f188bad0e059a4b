// The deterministic second-stage reduction of the backward's per-CTA partial sums (both kernel
// paths) and the fill kernel for T == 0. Non-template kernels: included by cc1d_api.cu only.
//
// Reference: jxiong21029/causal-conv1d-triton, causal_conv1d_triton/causal_conv1d.py
// (`_reduce_partials_kernel` :344-374, empty-input handling in `_fwd` :437-444, `_bwd` :480-489).
#pragma once

#include "cc1d_device.cuh"

namespace cc1d {

// Second stage of the dweight/dbias reduction (causal_conv1d.py:344-374): column n = k * D + d of
// the (P, W+1, D) partials is summed over P in a fixed order, so the result does not depend on
// scheduling. One warp per group of VEC adjacent columns: lane l sums rows l, l + 32, l + 64, ...
// in increasing order (its loads are independent, so all of them are in flight at once), then
// the 32 lane sums are combined by a fixed butterfly of shuffles. Eight warps per block, so that
// even the headline shape's 1280 column groups spread over every SM. Writes dweight[d, k] (k < W)
// and dbias[d] (k == W) in their own dtypes, or, when grad_f32 is given, the fp32 vector
// [dweight (D, W) row-major, dbias (D)] instead (its dbias part zero when there is no bias).
constexpr int kReduceWarps = 8;  // column groups per block, one warp each

__device__ __forceinline__ void reduce_store(int64_t n, float t, int D, int W, void* dweight, int w_dtype,
                                             void* dbias, int b_dtype, float* grad_f32, int has_bias) {
  const int k = static_cast<int>(n / D), d = static_cast<int>(n - static_cast<int64_t>(k) * D);
  if (grad_f32 != nullptr) {
    if (k < W)
      grad_f32[static_cast<int64_t>(d) * W + k] = t;
    else
      grad_f32[static_cast<int64_t>(D) * W + d] = has_bias ? t : 0.0f;
  } else if (k < W) {
    st_any(dweight, static_cast<int64_t>(d) * W + k, w_dtype, t);
  } else if (dbias != nullptr) {
    st_any(dbias, d, b_dtype, t);
  }
}

// VEC = 4: each warp sums 4 adjacent columns with 16-byte loads (requires N % 4 == 0 and a
// 16-byte aligned buffer); VEC = 1: one column per warp.
template <int VEC>
__global__ void __launch_bounds__(kReduceWarps * 32)
    cc1d_reduce_partials_kernel(const float* __restrict__ partials, int P, int D, int W, void* dweight, int w_dtype,
                                void* dbias, int b_dtype, float* grad_f32, int has_bias) {
  const int64_t N = static_cast<int64_t>(W + 1) * D;
  const int64_t NG = N / VEC;  // column groups
  const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
  for (int64_t gi = static_cast<int64_t>(blockIdx.x) * kReduceWarps + wi; gi < NG;
       gi += static_cast<int64_t>(gridDim.x) * kReduceWarps) {
    float s[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) s[v] = 0.0f;
    const float* col = partials + gi * VEC;
#pragma unroll 4
    for (int q = lane; q < P; q += 32) {
      if constexpr (VEC == 4) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(col + static_cast<int64_t>(q) * N));
        s[0] += x.x, s[1] += x.y, s[2] += x.z, s[3] += x.w;
      } else {
        s[0] += __ldg(col + static_cast<int64_t>(q) * N);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int v = 0; v < VEC; ++v) s[v] += __shfl_down_sync(0xffffffffu, s[v], off);
    if (lane == 0) {
#pragma unroll
      for (int v = 0; v < VEC; ++v)
        reduce_store(gi * VEC + v, s[v], D, W, dweight, w_dtype, dbias, b_dtype, grad_f32, has_bias);
    }
  }
}

// Waits on a shared-memory mbarrier that nothing completes: the bounded wait gives up after
// kWaitLimitNs and records kStatusWaitTimeout (the failure-detection self-test).
__global__ void cc1d_wait_timeout_probe_kernel(unsigned* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  mbar_wait(&bar, 0, status);  // phase 0 never completes: no thread arrives
}

// dst[i] = src[i] converted (or 0 when src is null), i < n.
__global__ void cc1d_fill_kernel(void* dst, int dst_dtype, const void* src, int src_dtype, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    st_any(dst, i, dst_dtype, src != nullptr ? ld_any(src, i, src_dtype) : 0.0f);
}

}  // namespace cc1d
