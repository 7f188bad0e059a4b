// Kernels for the inputs the TMA path cannot take: widths above 8 (up to kGenericMaxWidth), and
// x / dout whose base address or batch/time strides are not multiples of 16 bytes. A CTA stages a
// GT-row x GC-channel tile (plus halo) of fp32 in shared memory with plain loads, the width is a
// run-time value, and taps, bias and sequence ids come from shared memory.
//
// Reference: jxiong21029/causal-conv1d-triton, causal_conv1d_triton/causal_conv1d.py
// (`_fwd_kernel` :44-164, `_bwd_kernel` :167-341).
#pragma once

#include "cc1d_device.cuh"

namespace cc1d {

constexpr int kGenericMaxWidth = 256;
constexpr int GT = 64;        // rows per tile
constexpr int GC = 32;        // channels per tile (one warp across)
constexpr int GTHREADS = 256; // 8 warps: warp = row lane, lane = channel

struct GenericParams {
  const void* x;
  const void* weight;
  const void* bias;
  const void* init;
  const int32_t* seq;
  const void* dy;
  const void* dfinal;
  void* out;           // forward output (B, T, D) contiguous
  void* final_states;  // (B, W-1, D) contiguous, may be null
  void* dx;            // (B, T, D) contiguous
  void* dinit;         // (B, W-1, D) contiguous, may be null
  float* partials;     // (P, W+1, D)
  unsigned* status;
  int64_t sxb, sxt, syb, syt;
  int B, T, D, W;
  int n_tt, n_dc;      // time tiles, channel tiles
  int w_dtype, b_dtype, init_dtype;
  int silu;
};

__device__ __forceinline__ float sigmoid_generic(float z, bool fast) {
  if (fast) return fmaf(0.5f, tanh_approx(0.5f * z), 0.5f);
  return __fdividef(1.0f, 1.0f + __expf(-z));
}

// SiLU with the same per-element operations as the TMA forward's silu2.
__device__ __forceinline__ float silu_generic(float z, bool fast) {
  return fast ? silu2<true>(make_float2(z, z)).x : silu2<false>(make_float2(z, z)).x;
}

// Row t of concat(initial_states, x) at channel d in fp32 (causal_conv1d.py:28-41).
template <typename T>
__device__ __forceinline__ float x_at(const GenericParams& p, int b, int t, int d) {
  if (t >= 0 && t < p.T) return to_f(static_cast<const T*>(p.x)[b * p.sxb + t * p.sxt + d]);
  const int PAD = p.W - 1;
  if (p.init != nullptr && t < 0 && t >= -PAD)
    return ld_any(p.init, (static_cast<int64_t>(b) * PAD + t + PAD) * p.D + d, p.init_dtype);
  return 0.0f;
}

__device__ __forceinline__ int seq_generic(const GenericParams& p, int b, int t) {
  if (t >= p.T) return -1;
  const int32_t* srow = p.seq + static_cast<int64_t>(b) * p.T;
  if (t >= 0) return srow[t];
  return p.init != nullptr ? srow[0] : -1;
}

// Forward: one CTA per (batch, time tile, channel tile), flattened with the channel tile fastest.
template <typename T>
__global__ void __launch_bounds__(GTHREADS) cc1d_fwd_generic_kernel(const GenericParams p) {
  constexpr bool FAST = sizeof(T) == 2;
  const int W = p.W, PAD = W - 1;
  const int dcb = blockIdx.x % p.n_dc;
  const int rest = blockIdx.x / p.n_dc;
  const int t0 = (rest % p.n_tt) * GT, d0 = dcb * GC, b = rest / p.n_tt;
  extern __shared__ float gsm[];
  float* xs = gsm;                       // [GT + PAD][GC], row of t: t - t0 + PAD
  float* ws = xs + (GT + PAD) * GC;      // [W][GC]
  int* sq = reinterpret_cast<int*>(ws + W * GC);  // [GT + PAD]
  const int tid = threadIdx.x;

  for (int i = tid; i < (GT + PAD) * GC; i += GTHREADS) {
    const int r = i / GC, c = i - r * GC, d = d0 + c;
    xs[i] = d < p.D ? x_at<T>(p, b, t0 - PAD + r, d) : 0.0f;
  }
  for (int i = tid; i < W * GC; i += GTHREADS) {
    const int k = i / GC, c = i - k * GC, d = d0 + c;
    ws[i] = d < p.D ? ld_any(p.weight, static_cast<int64_t>(d) * W + k, p.w_dtype) : 0.0f;
  }
  if (p.seq != nullptr)
    for (int r = tid; r < GT + PAD; r += GTHREADS) sq[r] = seq_generic(p, b, t0 - PAD + r);
  __syncthreads();

  // Thread (row group rg, channel c) computes the GRB = 8 consecutive rows r0 .. r0 + 7 of its
  // channel, taps outer: one shared-memory load of a tap and one of a new input row feed 8 FMAs.
  // acc[j] takes z = w[PAD] x[t] then taps k = 0..PAD-1 in order, the reference's order per element.
  // The 8-row input window is a ring indexed by compile-time slots (tap loop unrolled by 8).
  constexpr int GRB = GT / (GTHREADS / GC);
  static_assert(GRB == 8, "8 rows per thread");
  const int c = tid % GC, r0 = (tid / GC) * GRB, d = d0 + c;
  const float bias = (p.bias != nullptr && d < p.D) ? ld_any(p.bias, d, p.b_dtype) : 0.0f;
  const bool seq = p.seq != nullptr;
  float acc[GRB], xr[GRB];
  int st[GRB], sr[GRB];  // seq id of each output row; ring of the input rows' seq ids
  const float wl = ws[PAD * GC + c];
#pragma unroll
  for (int j = 0; j < GRB; ++j) {
    acc[j] = wl * xs[(r0 + j + PAD) * GC + c];
    xr[j] = xs[(r0 + j) * GC + c];  // window of tap 0: rows r0 .. r0 + 7 (local x rows)
    st[j] = seq ? sq[r0 + j + PAD] : 0;
    sr[j] = seq ? sq[r0 + j] : 0;
  }
  for (int k0 = 0; k0 < PAD; k0 += GRB) {
#pragma unroll
    for (int kk = 0; kk < GRB; ++kk) {
      const int k = k0 + kk;
      if (k < PAD) {
        const float wk = ws[k * GC + c];
#pragma unroll
        for (int j = 0; j < GRB; ++j)
          if (!seq || sr[(j + kk) % GRB] == st[j]) acc[j] = fmaf(wk, xr[(j + kk) % GRB], acc[j]);
        // Slide: slot kk held row r0 + k; it takes row r0 + k + 8 (read up to row GT + PAD - 1).
        if (k + GRB < GT + PAD - r0) {
          xr[kk] = xs[(r0 + k + GRB) * GC + c];
          if (seq) sr[kk] = sq[r0 + k + GRB];
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < GRB; ++j) {
    const int r = r0 + j;
    if (t0 + r >= p.T) break;
    float z = acc[j] + bias;
    if (seq && st[j] < 0) z = 0.0f;
    if (p.silu) z = silu_generic(z, FAST);
    if (d < p.D) static_cast<T*>(p.out)[(static_cast<int64_t>(b) * p.T + t0 + r) * p.D + d] = from_f<T>(z);
  }

  if (p.final_states != nullptr && t0 + GT >= p.T) {
    for (int i = tid; i < PAD * GC; i += GTHREADS) {
      const int q = i / GC, cc = i - q * GC, dd = d0 + cc;
      if (dd < p.D)
        static_cast<T*>(p.final_states)[(static_cast<int64_t>(b) * PAD + q) * p.D + dd] =
            from_f<T>(x_at<T>(p, b, p.T - PAD + q, dd));
    }
  }
}

// Backward: grid P * n_dc CTAs; CTA (part, dc) walks the (batch, time-tile) items
// part, part + P, ... for channel tile dc and keeps its dweight/dbias sums in shared memory.
template <typename T>
__global__ void __launch_bounds__(GTHREADS) cc1d_bwd_generic_kernel(const GenericParams p) {
  constexpr bool FAST = sizeof(T) == 2;
  const int W = p.W, PAD = W - 1;
  const int n_dc = p.n_dc;
  const int P = gridDim.x / n_dc;
  const int dc = blockIdx.x % n_dc, part = blockIdx.x / n_dc;
  const int d0 = dc * GC;
  const int M = p.B * p.n_tt;
  extern __shared__ float gsm[];
  float* xs = gsm;                          // [GT + 2 PAD][GC], row of t: t - t0 + PAD
  float* dzs = xs + (GT + 2 * PAD) * GC;    // [GT + PAD][GC],   row of t: t - t0
  float* ws = dzs + (GT + PAD) * GC;        // [W][GC]
  float* acc = ws + W * GC;                 // [W + 1][GC]
  int* sq = reinterpret_cast<int*>(acc + (W + 1) * GC);  // [GT + 2 PAD], row of t: t - t0 + PAD
  const int tid = threadIdx.x;
  const int c = tid % GC, rl = tid / GC, d = d0 + c;
  const bool dvalid = d < p.D;

  for (int i = tid; i < W * GC; i += GTHREADS) {
    const int k = i / GC, cc = i - k * GC, dd = d0 + cc;
    ws[i] = dd < p.D ? ld_any(p.weight, static_cast<int64_t>(dd) * W + k, p.w_dtype) : 0.0f;
  }
  for (int i = tid; i < (W + 1) * GC; i += GTHREADS) acc[i] = 0.0f;

  for (int m = part; m < M; m += P) {
    const int b = m / p.n_tt;
    const int t0 = (m - b * p.n_tt) * GT;
    __syncthreads();  // previous item fully consumed (and ws/acc initialised)
    for (int i = tid; i < (GT + 2 * PAD) * GC; i += GTHREADS) {
      const int r = i / GC, cc = i - r * GC, dd = d0 + cc;
      xs[i] = dd < p.D ? x_at<T>(p, b, t0 - PAD + r, dd) : 0.0f;
    }
    for (int i = tid; i < (GT + PAD) * GC; i += GTHREADS) {
      const int r = i / GC, cc = i - r * GC, dd = d0 + cc, t = t0 + r;
      dzs[i] = (dd < p.D && t < p.T) ? to_f(static_cast<const T*>(p.dy)[b * p.syb + t * p.syt + dd]) : 0.0f;
    }
    if (p.seq != nullptr)
      for (int r = tid; r < GT + 2 * PAD; r += GTHREADS) sq[r] = seq_generic(p, b, t0 - PAD + r);
    __syncthreads();

    // dz = dy * SiLU'(z) in place, rows [t0, t0 + GT + PAD).
    for (int i = tid; i < (GT + PAD) * GC; i += GTHREADS) {
      const int r = i / GC, cc = i - r * GC, t = t0 + r;
      const int seq_t = p.seq ? sq[r + PAD] : 0;
      float g = dzs[i];
      if (p.silu) {
        float z = ws[PAD * GC + cc] * xs[(r + PAD) * GC + cc];
        for (int k = 0; k < PAD; ++k)
          if (!p.seq || sq[r + k] == seq_t) z = fmaf(ws[k * GC + cc], xs[(r + k) * GC + cc], z);
        const int dd = d0 + cc;
        z += (p.bias != nullptr && dd < p.D) ? ld_any(p.bias, dd, p.b_dtype) : 0.0f;
        const float s = sigmoid_generic(z, FAST);
        g = g * s * fmaf(z, 1.0f - s, 1.0f);
      }
      if ((p.seq && seq_t < 0) || t >= p.T) g = 0.0f;
      dzs[i] = g;
    }
    __syncthreads();

    // dx for the tile's own rows.
    for (int r = rl; r < GT && t0 + r < p.T; r += GTHREADS / GC) {
      const int t = t0 + r;
      const int seq_t = p.seq ? sq[r + PAD] : 0;
      float g = ws[PAD * GC + c] * dzs[r * GC + c];
      for (int j = 1; j <= PAD; ++j)
        if (!p.seq || sq[r + PAD + j] == seq_t) g = fmaf(ws[(PAD - j) * GC + c], dzs[(r + j) * GC + c], g);
      if (p.dfinal != nullptr && dvalid) {
        const int f = t - (p.T - PAD);
        if (f >= 0 && f < PAD) g += to_f(static_cast<const T*>(p.dfinal)[(static_cast<int64_t>(b) * PAD + f) * p.D + d]);
      }
      if (dvalid) static_cast<T*>(p.dx)[(static_cast<int64_t>(b) * p.T + t) * p.D + d] = from_f<T>(g);
    }
    // dinitial_states: rows t = -1 .. -PAD of the first tile, where dz = 0.
    if (p.dinit != nullptr && t0 == 0 && dvalid) {
      for (int q = rl + 1; q <= PAD; q += GTHREADS / GC) {
        const int t = -q;
        const int seq_t = p.seq ? sq[t + PAD] : 0;
        float g = 0.0f;
        for (int j = 1; j <= PAD; ++j) {
          const int u = t + j;
          if (u >= 0 && (!p.seq || sq[u + PAD] == seq_t)) g = fmaf(ws[(PAD - j) * GC + c], dzs[u * GC + c], g);
        }
        if (p.dfinal != nullptr) {
          const int f = t - (p.T - PAD);
          if (f >= 0 && f < PAD) g += to_f(static_cast<const T*>(p.dfinal)[(static_cast<int64_t>(b) * PAD + f) * p.D + d]);
        }
        st_any(p.dinit, (static_cast<int64_t>(b) * PAD + t + PAD) * p.D + d, p.init_dtype, g);
      }
    }
    // dweight[k] and dbias (k == W) partial sums over the tile's own rows.
    for (int k = rl; k <= W; k += GTHREADS / GC) {
      float s = 0.0f;
      for (int r = 0; r < GT && t0 + r < p.T; ++r) {
        const float g = dzs[r * GC + c];
        if (k == W) {
          s += g;
        } else if (!p.seq || k == PAD || sq[r + k] == sq[r + PAD]) {
          s = fmaf(g, xs[(r + k) * GC + c], s);
        }
      }
      acc[k * GC + c] += s;
    }
  }
  __syncthreads();
  for (int i = tid; i < (W + 1) * GC; i += GTHREADS) {
    const int k = i / GC, cc = i - k * GC, dd = d0 + cc;
    if (dd < p.D) p.partials[(static_cast<int64_t>(part) * (W + 1) + k) * p.D + dd] = acc[i];
  }
}

inline int generic_fwd_smem(int W) { return ((GT + W - 1) * GC + W * GC) * 4 + (GT + W - 1) * 4; }
inline int generic_bwd_smem(int W) {
  return ((GT + 2 * (W - 1)) * GC + (GT + W - 1) * GC + W * GC + (W + 1) * GC) * 4 + (GT + 2 * (W - 1)) * 4;
}

}  // namespace cc1d
