// TMA-pipelined sm_100a forward of the causal depthwise conv1d over channels-last inputs:
//
//   out[b,t,d] = act(bias[d] + sum_k weight[d,k] * x[b, t-(W-1)+k, d])
//
// Work decomposition. The (B, T, D) input is cut into tiles of T_TILE = 64 time
// rows by D_TILE channels (one 256-byte row segment: 128 channels of bf16/fp16, 64 of fp32).
// A CTA owns one channel block `db` for its whole life and walks the time tiles
// m = part, part + P, part + 2P, ... of the flattened (batch, time-tile) index, so that the CTAs of
// one wave sweep the tensor front to back together (each tile's W-1 halo rows were fetched by the
// neighbouring tile moments earlier and come from L2) and the taps stay in registers.
//
// Each CTA runs 4 consumer warps and 1 producer warp. The producer issues one 3-D TMA bulk tensor
// load per tile into a ring of shared-memory stages guarded by
// full/empty mbarriers; rows outside [0, T) are zero-filled by the TMA unit. It also writes the
// tile's seq_idx window into the stage. Consumer warp rg owns the R = 16 consecutive rows
// [t0 + 16 rg, t0 + 16 rg + 16) of the tile; its lane owns CPT consecutive channels (one 8-byte
// vector: 4 channels of bf16/fp16, 2 of fp32). Each thread reads its rows from shared memory,
// computes in fp32 pairs with the sm_100 f32x2 instructions and stores 8-byte vectors straight to
// global memory (a warp writes one contiguous 256-byte row segment per store).
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
  static constexpr int VEC_BYTES = 8;                 // one 8-byte vector per thread per row
  static constexpr int CPT = VEC_BYTES / ES;          // channels per thread (4, or 2 for fp32)
  static constexpr int NP = CPT / 2;                  // fp32 pairs per thread
  static constexpr int LANES_D = D_TILE / CPT;        // threads across one tile row: a whole warp
  static constexpr int CONSUMERS = 128;
  static constexpr int THREADS = CONSUMERS + 32;      // + producer warp
  static constexpr int RG = CONSUMERS / LANES_D;      // row groups per tile: one per warp
  static constexpr int T_TILE = 64;
  static constexpr int R = T_TILE / RG;               // rows per thread per tile
  static constexpr int PAD = W - 1;
  static_assert(LANES_D == 32, "a warp spans one tile row");
  static_assert(W >= 2 && W <= 8, "TMA path covers widths 2..8");
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
  static constexpr int STAGE_BYTES = XBYTES + SEQ_BYTES;
  // CTAs per SM the stages and registers are sized for: 4 x 3 stages up to W = 4, 3 x 4 stages
  // for wider windows (which need more registers per thread).
  static constexpr int STAGES = W <= 4 ? 3 : 4;
  static constexpr int MIN_CTAS = W <= 4 ? 4 : 3;
  static constexpr int SMEM_BYTES = kSmemAlign + kBarBytes + STAGES * STAGE_BYTES;
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
template <typename T, int W, bool SEQ, bool SILU>
__global__ void __launch_bounds__(TileCfg<T, W>::THREADS, FwdLayout<T, W, SEQ>::MIN_CTAS)
    cc1d_fwd_tma_kernel(const __grid_constant__ FwdParams p) {
  using C = TileCfg<T, W>;
  using L = FwdLayout<T, W, SEQ>;
  constexpr int PAD = C::PAD, R = C::R, CPT = C::CPT, NP = C::NP, S = L::STAGES;
  constexpr int DT = C::D_TILE;
  constexpr bool FAST = sizeof(T) == 2;

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + (kSmemAlign - 1)) & ~uintptr_t(kSmemAlign - 1));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  unsigned char* stage0 = smem + kBarBytes;

  const int n_db = p.n_db;
  const int P = gridDim.x / n_db;
  const int db = blockIdx.x % n_db;
  const int part = blockIdx.x / n_db;
  const int M = p.B * p.n_tt;
  const int n_my = part < M ? (M - 1 - part) / P + 1 : 0;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 32);  // the 32 producer lanes
      mbar_init(&empty[s], 4);  // one arrival per consumer warp
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 4) {
    // ---------------- producer warp ----------------
    if (lane == 0) prefetch_tensormap(&p.tmap_x);
    int issued = 0;
    for (int i = 0; i < n_my; ++i) {
      const int s = i % S;
      if (i >= S && !mbar_wait(&empty[s], ((i / S) - 1) & 1, p.status)) break;
      const int m = part + i * P;
      const int b = m / p.n_tt;
      const int t0 = (m - b * p.n_tt) * C::T_TILE;
      unsigned char* st = stage0 + s * L::STAGE_BYTES;
      if (lane == 0) {
        mbar_expect_tx(&full[s], L::XBYTES);
        tma_load_3d(st, &p.tmap_x, &full[s], db * DT, t0 - PAD, b);
      }
      if constexpr (SEQ) {
        int* sq = reinterpret_cast<int*>(st + L::XBYTES);
        const int32_t* srow = p.seq + static_cast<int64_t>(b) * p.T;
        for (int r = lane; r < L::XROWS; r += 32) sq[r] = seq_at(srow, t0 - PAD + r, p.T, p.init != nullptr);
      }
      mbar_arrive(&full[s]);
      issued = i + 1;
    }
    // Every copy this CTA issued must have landed before the CTA may exit.
    if (lane == 0)
      for (int j = issued > S ? issued - S : 0; j < issued; ++j) mbar_wait(&full[j % S], (j / S) & 1, p.status);
    return;
  }

  // ---------------- consumer warps ----------------
  const int ct = threadIdx.x;
  const int lane_d = ct % C::LANES_D;
  const int rg = ct / C::LANES_D;
  const int d = db * DT + lane_d * CPT;
  const bool dvalid = d < p.D;  // D is a multiple of CPT on this path
  const int64_t D = p.D;

  float2 w[W][NP], bv[NP];
  load_taps<W, NP>(p.weight, p.w_dtype, p.bias, p.b_dtype, d, dvalid, w, bv);

  for (int i = 0; i < n_my; ++i) {
    const int s = i % S;
    const int m = part + i * P;
    const int b = m / p.n_tt;
    const int tt = m - b * p.n_tt;
    const int t0 = tt * C::T_TILE;
    if (!mbar_wait(&full[s], (i / S) & 1, p.status)) break;

    const unsigned char* st = stage0 + s * L::STAGE_BYTES;
    const T* xt = reinterpret_cast<const T*>(st) + lane_d * CPT;  // local row r at xt + r * DT
    const int* sq = reinterpret_cast<const int*>(st + L::XBYTES);
    const int rb = rg * R;  // local row of global row ts - PAD
    const int ts = t0 + rb;

    // Before the step at row t: xw[k] = x[t - PAD + k], k < PAD.
    float2 xw[PAD][NP];
    if (p.init != nullptr && ts == 0) {
#pragma unroll
      for (int k = 0; k < PAD; ++k) {
        if (dvalid) {
          load_state_row<NP>(p.init, p.init_dtype, static_cast<int64_t>(b) * PAD + k, p.D, d, xw[k]);
        } else {
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) xw[k][i2] = make_float2(0.f, 0.f);
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < PAD; ++k) load_vec<T, CPT>(xt + (rb + k) * DT, xw[k]);
    }

    T* orow = static_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.T + ts) * D + d;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float2 xr[NP];
      load_vec<T, CPT>(xt + (rb + PAD + r) * DT, xr);
      const int seq_t = SEQ ? sq[rb + PAD + r] : 0;
      // z = w[PAD] x[t], then taps k = 0..PAD-1 oldest first, then bias (causal_conv1d.py:129-136).
      float2 z[NP];
#pragma unroll
      for (int i2 = 0; i2 < NP; ++i2) z[i2] = fmul2(w[PAD][i2], xr[i2]);
#pragma unroll
      for (int k = 0; k < PAD; ++k) {
        if (!SEQ || sq[rb + r + k] == seq_t) {
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) z[i2] = ffma2(w[k][i2], xw[k][i2], z[i2]);
        }
      }
#pragma unroll
      for (int i2 = 0; i2 < NP; ++i2) z[i2] = fadd2(z[i2], bv[i2]);
      if (SEQ && seq_t < 0) {
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) z[i2] = make_float2(0.f, 0.f);
      }
      if constexpr (SILU) {
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) z[i2] = silu2<FAST>(z[i2]);
      }
      if (dvalid && ts + r < p.T) store_vec<T, CPT>(orow + r * D, z);
#pragma unroll
      for (int k = 0; k + 1 < PAD; ++k)
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) xw[k][i2] = xw[k + 1][i2];
#pragma unroll
      for (int i2 = 0; i2 < NP; ++i2) xw[PAD - 1][i2] = xr[i2];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the stage

    // final_states = last PAD rows of concat(initial_states, x) (causal_conv1d.py:153-164).
    if (p.final_states != nullptr && tt == p.n_tt - 1 && rg == 0 && dvalid) {
#pragma unroll
      for (int q = 0; q < PAD; ++q) {
        const int src = p.T - PAD + q;
        float2 v[NP];
        if (src >= 0) {
          load_vec<T, CPT>(static_cast<const T*>(p.x) + b * p.sxb + src * p.sxt + d, v);
        } else if (p.init != nullptr) {
          load_state_row<NP>(p.init, p.init_dtype, static_cast<int64_t>(b) * PAD + src + PAD, p.D, d, v);
        } else {
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) v[i2] = make_float2(0.f, 0.f);
        }
        store_vec<T, CPT>(static_cast<T*>(p.final_states) + (static_cast<int64_t>(b) * PAD + q) * D + d, v);
      }
    }
  }
}

}  // namespace cc1d
