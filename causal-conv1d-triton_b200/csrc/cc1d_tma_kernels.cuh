// TMA-staged sm_100a forward of the causal depthwise conv1d over channels-last inputs:
//
//   out[b,t,d] = act(bias[d] + sum_k weight[d,k] * x[b, t-(W-1)+k, d])
//
// Work decomposition. The (B, T, D) input is cut into tiles of T_TILE = 64 time rows by D_TILE
// channels (one 256-byte row segment: 128 channels of bf16/fp16, 64 of fp32), one tile per CTA,
// the grid covering every tile with the channel block fastest, so that the CTAs resident at any
// moment sweep the tensor front to back together (each tile's W-1 halo rows were fetched by the
// neighbouring tile moments earlier and come from L2).
//
// A CTA's thread 0 issues one 3-D TMA bulk tensor load of the tile and its halo into shared memory
// (rows outside [0, T) zero-filled by the TMA unit), completion counted on an mbarrier; the
// threads load the taps and the tile's seq_idx window meanwhile. The 128 threads form RG row
// groups of LANES_D threads; row group rg owns the R = 64 / RG consecutive rows [t0 + R rg,
// t0 + R rg + R), and each of its threads owns CPT consecutive channels of one vector. Up to W = 4
// (and for fp32) a vector is 8 bytes: 4 channels of bf16/fp16 (2 of fp32), a warp per row, R = 16.
// Wider 16-bit windows use 4-byte vectors (2 channels, two warps per row, R = 32): with 4 channels a
// thread's W x 4 fp32 taps and (W-1) x 4 window values alone fill the 80 registers that 6 CTAs per
// SM allow, and occupancy, not arithmetic, sets this kernel's speed. Each thread reads its rows
// from shared memory, computes in fp32 pairs with the sm_100 f32x2 instructions and stores its
// vector straight to global memory (a warp writes a contiguous 256- or 128-byte row segment).
//
// The backward is in cc1d_bwd_kernel.cuh; TileCfg's constants, the tap loaders and the seq_idx
// convention here are shared with it.
//
// Reference: jxiong21029/causal-conv1d-triton, causal_conv1d_triton/causal_conv1d.py
// (`_fwd_kernel` :44-164). The per-element arithmetic and its order follow the reference; the
// tiling, staging and scheduling are this file's own.
#pragma once

#include "cc1d_device.cuh"

namespace cc1d {

template <typename T, int W>
struct TileCfg {
  static constexpr int ES = static_cast<int>(sizeof(T));
  static constexpr int ROW_BYTES = 256;               // bytes of one tile row (TMA box inner extent)
  static constexpr int D_TILE = ROW_BYTES / ES;       // channels per tile
  static constexpr int VEC_BYTES = (ES == 2 && W > 4) ? 4 : 8;  // one vector per thread per row
  static constexpr int CPT = VEC_BYTES / ES;          // channels per thread (4 or 2)
  static constexpr int NP = CPT / 2;                  // fp32 pairs per thread
  static constexpr int LANES_D = D_TILE / CPT;        // threads across one tile row: 32 or 64
  static constexpr int CONSUMERS = 128;               // threads per CTA
  static constexpr int RG = CONSUMERS / LANES_D;      // row groups per tile
  static constexpr int T_TILE = 64;
  static constexpr int R = T_TILE / RG;               // rows per thread per tile: 16 or 32
  static constexpr int PAD = W - 1;
  static_assert(LANES_D % 32 == 0 && RG * LANES_D == CONSUMERS, "row groups are whole warps");
  static_assert(W >= 2 && W <= 16, "TMA path covers template widths 2..16");
  static_assert(R >= PAD, "only row group 0 of the first tile reads rows t < 0");
};

constexpr int kSmemAlign = 128;
constexpr int kBarBytes = 128;  // full[] and empty[] barriers, at most 8 stages each

template <typename T, int W, bool SEQ>
struct FwdLayout {
  using C = TileCfg<T, W>;
  static constexpr int XROWS = C::T_TILE + C::PAD;    // rows [t0 - PAD, t0 + T_TILE)
  static constexpr int XBYTES = XROWS * C::ROW_BYTES;
  static constexpr int SEQ_BYTES = SEQ ? (XROWS * 4 + 127) / 128 * 128 : 0;
  // Registers are bounded for 6 CTAs (24 warps) per SM with 8-byte vectors, 8 CTAs with 4-byte
  // vectors; 17-19 KB of shared memory each.
  // Template widths 12 and 16 (taps and window of 2 x W fp32 values per channel pair) get 5.
  static constexpr int MIN_CTAS = W > 8 ? 5 : (C::VEC_BYTES == 4 ? 8 : 6);
  static constexpr int SMEM_BYTES = kSmemAlign + kBarBytes + XBYTES + SEQ_BYTES;
};

struct alignas(64) FwdParams {
  CUtensorMap tmap_x;  // x viewed as (D, T, B), box (D_TILE, T_TILE + PAD, 1)
  const void* x;
  const void* weight;
  const void* bias;    // may be null
  const void* init;    // initial_states (B, W-1, D), may be null
  const int32_t* seq;  // seq_idx (B, T), null unless the SEQ variant runs
  void* out;           // (B, T, D) contiguous, dtype of x
  void* final_states;  // (B, W-1, D) contiguous, dtype of x, may be null
  unsigned* status;
  int64_t sxb, sxt;    // x strides in elements (channel stride 1)
  int B, T, D;
  int W;               // true width: the template width less any leading zero taps
  int n_tt, n_db;      // time tiles per row, channel blocks
  int w_dtype, b_dtype, init_dtype;
};

// Sequence id of row t of batch row `srow` with the reference's conventions (causal_conv1d.py:
// 17-25): rows t < 0 belong to seq_idx[b, 0]'s sequence when initial states are given, every
// other row outside [0, T) gets -1.
__device__ __forceinline__ int seq_at(const int32_t* srow, int t, int T, bool has_init) {
  if (t >= T) return -1;
  if (t >= 0) return srow[t];
  return has_init ? srow[0] : -1;
}

// Loads the CPT weights of each of the W taps and the bias for channels [d, d + CPT) as fp32
// pairs (zeros for an out-of-range channel group). weight is (D, W) row-major in any float type.
template <int W, int NP>
__device__ __forceinline__ void load_taps(const void* weight, int w_dtype, const void* bias, int b_dtype,
                                          int d, bool dvalid, float2 (&w)[W][NP], float2 (&bv)[NP]) {
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int64_t d0 = d + 2 * i;
#pragma unroll
    for (int k = 0; k < W; ++k)
      w[k][i] = dvalid ? make_float2(ld_any(weight, d0 * W + k, w_dtype), ld_any(weight, (d0 + 1) * W + k, w_dtype))
                       : make_float2(0.f, 0.f);
    bv[i] = (dvalid && bias) ? make_float2(ld_any(bias, d0, b_dtype), ld_any(bias, d0 + 1, b_dtype))
                             : make_float2(0.f, 0.f);
  }
}

// load_taps for fp32 weights and bias with vector loads: a thread's CPT channels x W taps are
// CPT * W consecutive floats of the (D, W) weight, read as float4s when their count and address
// allow, else as float2s; the bias likewise. Falls back to load_taps for other dtypes or
// misaligned addresses. Requires an even CPT.
template <int W, int NP>
__device__ __forceinline__ void load_taps_fast(const void* weight, int w_dtype, const void* bias, int b_dtype, int d,
                                               bool dvalid, float2 (&w)[W][NP], float2 (&bv)[NP]) {
  constexpr int CPT = 2 * NP;
  constexpr int WV = (CPT * W) % 4 == 0 ? 4 : 2;  // floats per weight load
  constexpr int BV = CPT % 4 == 0 ? 4 : 2;        // floats per bias load
  const float* wf = static_cast<const float*>(weight) + static_cast<int64_t>(d) * W;
  const float* bf = bias != nullptr ? static_cast<const float*>(bias) + d : nullptr;
  const bool vec_w = w_dtype == kF32 && (reinterpret_cast<uintptr_t>(wf) & (4 * WV - 1)) == 0;
  const bool vec_b = bias == nullptr || (b_dtype == kF32 && (reinterpret_cast<uintptr_t>(bf) & (4 * BV - 1)) == 0);
  if (!dvalid || !vec_w || !vec_b) {
    load_taps<W, NP>(weight, w_dtype, bias, b_dtype, d, dvalid, w, bv);
    return;
  }
  float wv[CPT * W];
#pragma unroll
  for (int q = 0; q < CPT * W / WV; ++q) {
    if constexpr (WV == 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(wf) + q);
      wv[4 * q] = v.x, wv[4 * q + 1] = v.y, wv[4 * q + 2] = v.z, wv[4 * q + 3] = v.w;
    } else {
      const float2 v = __ldg(reinterpret_cast<const float2*>(wf) + q);
      wv[2 * q] = v.x, wv[2 * q + 1] = v.y;
    }
  }
#pragma unroll
  for (int i = 0; i < NP; ++i)
#pragma unroll
    for (int k = 0; k < W; ++k) w[k][i] = make_float2(wv[(2 * i) * W + k], wv[(2 * i + 1) * W + k]);
  if (bias == nullptr) {
#pragma unroll
    for (int i = 0; i < NP; ++i) bv[i] = make_float2(0.f, 0.f);
  } else if constexpr (BV == 4) {
#pragma unroll
    for (int q = 0; q < CPT / 4; ++q) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(bf) + q);
      bv[2 * q] = make_float2(v.x, v.y);
      bv[2 * q + 1] = make_float2(v.z, v.w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < NP; ++i) bv[i] = __ldg(reinterpret_cast<const float2*>(bf) + i);
  }
}

// Multiplies the taps and the bias by 0.5 (exact), for the kernels that compute h = z / 2.
template <int W, int NP>
__device__ __forceinline__ void halve_taps(float2 (&w)[W][NP], float2 (&bv)[NP]) {
  const float2 half = make_float2(0.5f, 0.5f);
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    bv[i] = fmul2(bv[i], half);
#pragma unroll
    for (int k = 0; k < W; ++k) w[k][i] = fmul2(w[k][i], half);
  }
}

// load_taps for a true width Wt below the template width W: the (D, Wt) weight rows fill taps
// W-Wt .. W-1 and the leading W-Wt taps are zero. A causal conv of width Wt equals the width-W conv
// with those zero taps bit for bit on finite inputs (each zero product adds an exact zero).
template <int W, int NP>
__device__ __forceinline__ void load_taps_off(const void* weight, int w_dtype, const void* bias, int b_dtype, int d,
                                              bool dvalid, int Wt, float2 (&w)[W][NP], float2 (&bv)[NP]) {
  const int off = W - Wt;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int64_t d0 = d + 2 * i;
#pragma unroll
    for (int k = 0; k < W; ++k) {
      const int kk = k - off;
      w[k][i] = (dvalid && kk >= 0)
                    ? make_float2(ld_any(weight, d0 * Wt + kk, w_dtype), ld_any(weight, (d0 + 1) * Wt + kk, w_dtype))
                    : make_float2(0.f, 0.f);
    }
    bv[i] = (dvalid && bias) ? make_float2(ld_any(bias, d0, b_dtype), ld_any(bias, d0 + 1, b_dtype))
                             : make_float2(0.f, 0.f);
  }
}

// Loads CPT channels of a row of a contiguous (B, W-1, D) state tensor (run-time dtype).
template <int NP>
__device__ __forceinline__ void load_state_row(const void* base, int dtype, int64_t row, int D, int d,
                                               float2 (&v)[NP]) {
  const int64_t o = row * D + d;
#pragma unroll
  for (int i = 0; i < NP; ++i) v[i] = make_float2(ld_any(base, o + 2 * i, dtype), ld_any(base, o + 2 * i + 1, dtype));
}

// =============================================================================================
// Forward
// =============================================================================================
// One tile per CTA: thread 0 issues the TMA load of rows t0-PAD .. t0+63 (zero-filled outside
// [0, T)), every thread loads its taps while the copy is in flight, waits once on the mbarrier,
// computes its 16 rows from shared memory and stores them. The grid holds every tile of the
// tensor: on B200 a streaming copy through one TMA box per CTA over such a grid reaches ~6.7 TB/s,
// while persistent CTAs looping over a multi-stage ring of the same boxes stay near 5.9 TB/s.
// PLAIN: x's base or strides rule out a tensor map; the threads fill the same tile with plain loads
// (separate instantiations, so the TMA variants keep their registers).
template <typename T, int W, bool SEQ, bool SILU, bool PLAIN>
__global__ void __launch_bounds__(TileCfg<T, W>::CONSUMERS, FwdLayout<T, W, SEQ>::MIN_CTAS)
    cc1d_fwd_tma_kernel(const __grid_constant__ FwdParams p) {
  using C = TileCfg<T, W>;
  using L = FwdLayout<T, W, SEQ>;
  constexpr int PAD = C::PAD, R = C::R, CPT = C::CPT, NP = C::NP;
  constexpr int DT = C::D_TILE;
  constexpr bool FAST = sizeof(T) == 2;

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = aligned_smem<kSmemAlign>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  unsigned char* tile = smem + kBarBytes;

  // (channel block fastest, then time tile, then batch row): the block's (x, y, z) index when the
  // grid is 3-D, else its x index decomposed (grids beyond 65535 time tiles or batch rows).
  int db = blockIdx.x, tt = blockIdx.y, b = blockIdx.z;
  if (gridDim.y == 1 && gridDim.z == 1 && (p.n_tt > 1 || p.B > 1)) {
    db = blockIdx.x % p.n_db;
    const int rest = blockIdx.x / p.n_db;
    tt = rest % p.n_tt;
    b = rest / p.n_tt;
  }
  const int t0 = tt * C::T_TILE;
  const int rg = threadIdx.x / C::LANES_D, lane = threadIdx.x % C::LANES_D;

  if constexpr (PLAIN) {
    // Layouts a tensor map cannot describe (base or batch/time strides not 16-byte multiples): the
    // threads fill the same tile with element loads, 8 rows in flight per thread, rows outside
    // [0, T) and channels outside [0, D) as zeros, as the TMA unit would.
    constexpr int ROWS_PER_PASS = C::CONSUMERS / DT > 0 ? C::CONSUMERS / DT : 1;
    const int c = threadIdx.x % DT, r_first = threadIdx.x / DT;
    const int dd = db * DT + c;
    const T* xrow = static_cast<const T*>(p.x) + static_cast<int64_t>(b) * p.sxb + dd;
    T* trow = reinterpret_cast<T*>(tile) + c;
    const T zero = from_f<T>(0.0f);
    for (int r0 = r_first; r0 < L::XROWS; r0 += 8 * ROWS_PER_PASS) {
      T v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int r = r0 + u * ROWS_PER_PASS, t = t0 - PAD + r;
        v[u] = (r < L::XROWS && t >= 0 && t < p.T && dd < p.D) ? xrow[static_cast<int64_t>(t) * p.sxt] : zero;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int r = r0 + u * ROWS_PER_PASS;
        if (r < L::XROWS) trow[r * DT] = v[u];
      }
    }
  } else if (threadIdx.x == 0) {
    mbar_init(full, 1);
    fence_mbar_init();
    mbar_expect_tx(full, L::XBYTES);
    mbar_arrive(full);
    tma_load_3d(tile, &p.tmap_x, full, db * DT, t0 - PAD, b);
  }
  // seq_idx window of the tile: rows t0 - PAD .. t0 + T_TILE - 1
  int* sq = reinterpret_cast<int*>(tile + L::XBYTES);
  bool one_seq = false;  // the whole window is one sequence (ids equal and >= 0): every mask passes
  if constexpr (SEQ) {
    const int32_t* srow = p.seq + static_cast<int64_t>(b) * p.T;
    const int first = seq_at(srow, t0 - PAD, p.T, p.init != nullptr);
    one_seq = first >= 0;
    for (int r = threadIdx.x; r < L::XROWS; r += C::CONSUMERS) {
      const int v = seq_at(srow, t0 - PAD + r, p.T, p.init != nullptr);
      sq[r] = v;
      one_seq = one_seq && v == first;
    }
  }

  const int d = db * DT + lane * CPT;
  const bool dvalid = d < p.D;  // D is a multiple of CPT on this path
  const int64_t D = p.D;
  float2 w[W][NP], bv[NP];
  if (p.W == W) {
    load_taps_fast<W, NP>(p.weight, p.w_dtype, p.bias, p.b_dtype, d, dvalid, w, bv);
  } else {
    load_taps_off<W, NP>(p.weight, p.w_dtype, p.bias, p.b_dtype, d, dvalid, p.W, w, bv);
  }
  if constexpr (SILU && FAST) halve_taps<W, NP>(w, bv);  // z below is h = z / 2
  const int pw = p.W - 1, off = W - p.W;  // true state rows; leading zero taps
  // barrier initialised (or tile filled), seq window written; with seq_idx, the tile-wide vote
  if constexpr (SEQ)
    one_seq = __syncthreads_and(one_seq) != 0;
  else
    __syncthreads();
  if (!PLAIN && !mbar_wait(full, 0, p.status)) {
    // Gave up (status recorded). The tile copy may still be landing in this CTA's shared memory:
    // wait for it once more, again bounded, before the CTA exits.
    mbar_wait(full, 0, p.status);
    return;
  }

  const T* xt = reinterpret_cast<const T*>(tile) + lane * CPT;  // local row r <-> global row t0 - PAD + r
  const int rb = rg * R;  // local row of global row ts - PAD
  const int ts = t0 + rb;

  // Ring of the last PAD + 1 input rows: local row j (global row ts - PAD + j) sits in slot
  // j % NW. Every index below is a compile-time constant, so the ring never moves a value.
  constexpr int NW = PAD + 1;
  float2 xw[NW][NP];
  if (p.init != nullptr && ts == 0) {
#pragma unroll
    for (int k = 0; k < PAD; ++k) {  // row t = k - PAD is initial_states row k - off
      if (dvalid && k >= off) {
        load_state_row<NP>(p.init, p.init_dtype, static_cast<int64_t>(b) * pw + (k - off), p.D, d, xw[k]);
      } else {
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) xw[k][i2] = make_float2(0.f, 0.f);
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < PAD; ++k) load_vec<T, CPT>(xt + (rb + k) * DT, xw[k]);
  }

  T* orow = static_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.T + ts) * D + d;  // advanced one row per step
  const bool full_rows = dvalid && ts + R <= p.T;
  // masked: apply the seq_idx masks (false for a tile whose window is one sequence, where every
  // mask passes; the results are the same bits).
  auto rows = [&](auto masked) {
  constexpr bool SQ = SEQ && decltype(masked)::value;
  static_for<0, R>([&](auto rc) {
    constexpr int r = decltype(rc)::value;
    constexpr int cur = (r + PAD) % NW;
    load_vec<T, CPT>(xt + (rb + PAD + r) * DT, xw[cur]);
    const int seq_t = SQ ? sq[rb + PAD + r] : 0;
    // z = w[PAD] x[t], then taps k = 0..PAD-1 oldest first, then bias (causal_conv1d.py:129-136).
    float2 z[NP];
#pragma unroll
    for (int i2 = 0; i2 < NP; ++i2) z[i2] = fmul2(w[PAD][i2], xw[cur][i2]);
#pragma unroll
    for (int k = 0; k < PAD; ++k) {
      if (!SQ || sq[rb + r + k] == seq_t) {
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) z[i2] = ffma2(w[k][i2], xw[(r + k) % NW][i2], z[i2]);
      }
    }
#pragma unroll
    for (int i2 = 0; i2 < NP; ++i2) z[i2] = fadd2(z[i2], bv[i2]);
    if (SQ && seq_t < 0) {
#pragma unroll
      for (int i2 = 0; i2 < NP; ++i2) z[i2] = make_float2(0.f, 0.f);
    }
    if constexpr (SILU) {
#pragma unroll
      for (int i2 = 0; i2 < NP; ++i2) z[i2] = FAST ? silu2_of_half(z[i2]) : silu2<false>(z[i2]);
    }
    if (full_rows || (dvalid && ts + r < p.T)) store_vec<T, CPT>(orow, z);
    orow += D;
  });
  };
  if (SEQ && one_seq)
    rows(std::false_type{});
  else
    rows(std::true_type{});

  // final_states = last W-1 rows (true width) of concat(initial_states, x) (causal_conv1d.py:153-164).
  if (p.final_states != nullptr && tt == p.n_tt - 1 && rg == 0 && dvalid) {
#pragma unroll
    for (int q = 0; q < PAD; ++q) {
      if (q >= pw) break;
      const int src = p.T - pw + q;
      float2 v[NP];
      if (src >= 0) {
        const T* xs = static_cast<const T*>(p.x) + b * p.sxb + src * p.sxt + d;
        if constexpr (PLAIN) {  // x may be only element-aligned here
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) v[i2] = make_float2(to_f(xs[2 * i2]), to_f(xs[2 * i2 + 1]));
        } else {
          load_vec<T, CPT>(xs, v);
        }
      } else if (p.init != nullptr) {
        load_state_row<NP>(p.init, p.init_dtype, static_cast<int64_t>(b) * pw + src + pw, p.D, d, v);
      } else {
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) v[i2] = make_float2(0.f, 0.f);
      }
      store_vec<T, CPT>(static_cast<T*>(p.final_states) + (static_cast<int64_t>(b) * pw + q) * D + d, v);
    }
  }
}

}  // namespace cc1d
