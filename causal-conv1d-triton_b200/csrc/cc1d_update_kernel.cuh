// Decode-time state update: L new rows per batch row through the conv, with the streaming state in
// the reference's layout (B, W-1, D), the inputs preceding the new rows (causal_conv1d.py:597-599).
// The reference has no decode kernel; this is the single-step companion of its forward.
//
// For each batch row b (state row s = state_indices ? state_indices[b] : b) and channel d:
//   window = concat(state[s, :, d], x[b, :, d])                     (W-1 + L values)
//   out[b, l, d] = act(bias[d] + sum_k w[d, k] window[l + k])       in the forward's order
//   state[s, p, d] = window[L + p]                                  (p < W-1), in place
// One thread per (b, d), so a warp reads and writes 32 consecutive channels. Element types are
// run-time values: decode is latency-bound, not arithmetic-bound.
#pragma once

#include "cc1d_device.cuh"

namespace cc1d {

struct UpdateParams {
  const void* x;             // (B, L, D) at strides (sxb, sxt, 1)
  void* state;               // (n_slots, W-1, D) contiguous
  const int32_t* indices;    // (B) state slot per batch row, or null
  const void* weight;        // (D, W)
  const void* bias;          // (D) or null
  void* out;                 // (B, L, D) contiguous, dtype of x
  int64_t sxb, sxt;
  int B, L, D, W;
  int x_dtype, s_dtype, w_dtype, b_dtype;
  int silu;
};

__global__ void __launch_bounds__(256) cc1d_update_kernel(const UpdateParams p) {
  const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<int64_t>(p.B) * p.D) return;
  const int b = static_cast<int>(idx / p.D), d = static_cast<int>(idx - static_cast<int64_t>(b) * p.D);
  const int PAD = p.W - 1;
  const int64_t srow = p.indices != nullptr ? p.indices[b] : b;
  if (srow < 0) return;  // a negative slot marks a padded batch entry: nothing to do
  const int64_t sbase = srow * PAD * p.D + d;
  const int64_t xbase = b * p.sxb + d;
  // window[j]: j < PAD from the state, else x row j - PAD.
  auto window = [&](int j) -> float {
    return j < PAD ? ld_any(p.state, sbase + static_cast<int64_t>(j) * p.D, p.s_dtype)
                   : ld_any(p.x, xbase + static_cast<int64_t>(j - PAD) * p.sxt, p.x_dtype);
  };
  const float bias = p.bias != nullptr ? ld_any(p.bias, d, p.b_dtype) : 0.0f;
  const int64_t wb = static_cast<int64_t>(d) * p.W;
  const bool fast = p.x_dtype != kF32;
  for (int l = 0; l < p.L; ++l) {
    float z = ld_any(p.weight, wb + PAD, p.w_dtype) * window(l + PAD);
    for (int k = 0; k < PAD; ++k) z = fmaf(ld_any(p.weight, wb + k, p.w_dtype), window(l + k), z);
    z += bias;
    if (p.silu) z = fast ? silu2<true>(make_float2(z, z)).x : silu2<false>(make_float2(z, z)).x;
    st_any(p.out, (static_cast<int64_t>(b) * p.L + l) * p.D + d, p.x_dtype, z);
  }
  // New state: entry q takes window[L + q]. Walking q upwards, entry q is written only after the
  // entry it may still need (old entry q + L > q) has been read.
  for (int q = 0; q < PAD; ++q) st_any(p.state, sbase + static_cast<int64_t>(q) * p.D, p.s_dtype, window(p.L + q));
}

}  // namespace cc1d
