// Decode-time state update: L new rows per batch row through the conv, with the streaming state in
// the reference's layout (B, W-1, D), the inputs preceding the new rows (causal_conv1d.py:597-599).
// The reference has no decode kernel; this is the single-step companion of its forward.
//
// For each batch row b (state row s = state_indices ? state_indices[b] : b) and channel d:
//   window = concat(state[s, :, d], x[b, :, d])                     (W-1 + L values)
//   out[b, l, d] = act(bias[d] + sum_k w[d, k] window[l + k])       in the forward's order
//   state[s, p, d] = window[L + p]                                  (p < W-1), in place
// Two kernels. cc1d_update_vec_kernel<T, W> (widths 2..8, x and state of one type T, D a multiple
// of the vector's channels, 8-byte aligned rows) gives each thread one 8-byte vector of channels
// (4 bf16/fp16, 2 fp32): it loads its W-1 state rows and each new x row as one vector each, keeps
// the window in registers, and writes the outputs and the new state rows once, so a thread makes
// one round trip to memory and a 256-sequence batch of a Mamba-2 layer fits in one resident wave.
// cc1d_update_kernel covers every other case (run-time width and element types, one thread per
// (b, d)).
#pragma once

#include "cc1d_device.cuh"
#include "cc1d_tma_kernels.cuh"  // load_taps_fast

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

template <typename T, int W>
__global__ void __launch_bounds__(256) cc1d_update_vec_kernel(const UpdateParams p) {
  constexpr int CPT = 8 / static_cast<int>(sizeof(T));  // one 8-byte vector: 4 bf16/fp16 or 2 fp32
  constexpr int NP = CPT / 2, PAD = W - 1;
  constexpr bool FAST = sizeof(T) == 2;
  const int DV = p.D / CPT;
  const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<int64_t>(p.B) * DV) return;
  const int b = static_cast<int>(idx / DV), d = CPT * static_cast<int>(idx - static_cast<int64_t>(b) * DV);
  const int64_t srow = p.indices != nullptr ? p.indices[b] : b;
  if (srow < 0) return;  // a padded batch entry
  T* st = static_cast<T*>(p.state) + srow * PAD * p.D + d;
  const T* xb = static_cast<const T*>(p.x) + b * p.sxb + d;
  T* ob = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.L * p.D + d;

  float2 win[PAD][NP];  // win[k] = the input PAD - k rows before the next one
#pragma unroll
  for (int q = 0; q < PAD; ++q) load_vec<T, CPT>(st + static_cast<int64_t>(q) * p.D, win[q]);
  float2 w[W][NP], bv[NP];
  load_taps_fast<W, NP>(p.weight, p.w_dtype, p.bias, p.b_dtype, d, true, w, bv);
  for (int l = 0; l < p.L; ++l) {
    float2 xr[NP], z[NP];
    load_vec<T, CPT>(xb + static_cast<int64_t>(l) * p.sxt, xr);
    // The forward's per-element order (causal_conv1d.py:129-143).
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      z[i] = fmul2(w[PAD][i], xr[i]);
#pragma unroll
      for (int k = 0; k < PAD; ++k) z[i] = ffma2(w[k][i], win[k][i], z[i]);
      z[i] = fadd2(z[i], bv[i]);
      if (p.silu) z[i] = silu2<FAST>(z[i]);
    }
    store_vec<T, CPT>(ob + static_cast<int64_t>(l) * p.D, z);
#pragma unroll
    for (int i = 0; i < NP; ++i) {
#pragma unroll
      for (int k = 0; k + 1 < PAD; ++k) win[k][i] = win[k + 1][i];
      win[PAD - 1][i] = xr[i];
    }
  }
#pragma unroll
  for (int q = 0; q < PAD; ++q) store_vec<T, CPT>(st + static_cast<int64_t>(q) * p.D, win[q]);
}

}  // namespace cc1d
