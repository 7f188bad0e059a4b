// TMA-pipelined sm_100a kernels for the causal depthwise conv1d over channels-last inputs:
//
//   out[b,t,d] = act(bias[d] + sum_k weight[d,k] * x[b, t-(W-1)+k, d])
//
// Work decomposition (both kernels). The (B, T, D) input is cut into tiles of T_TILE = 64 time
// rows by D_TILE channels (one 256-byte row segment: 128 channels of bf16/fp16, 64 of fp32).
// A CTA owns one channel block `db` for its whole life and walks the time tiles
// m = part, part + P, part + 2P, ... of the flattened (batch, time-tile) index, so that the CTAs of
// one wave sweep the tensor front to back together (each tile's W-1 halo rows were fetched by the
// neighbouring tile moments earlier and come from L2), and so that the backward can keep its
// dweight/dbias partial sums in registers for the whole run.
//
// Each CTA runs 4 consumer warps and 1 producer warp. The producer issues one 3-D TMA bulk tensor
// load per tile (two in the backward: x and dy) into a ring of shared-memory stages guarded by
// full/empty mbarriers; rows outside [0, T) are zero-filled by the TMA unit. It also writes the
// tile's seq_idx window into the stage. Consumer warp rg owns the R = 16 consecutive rows
// [t0 + 16 rg, t0 + 16 rg + 16) of the tile; its lane owns CPT consecutive channels (one 8-byte
// vector: 4 channels of bf16/fp16, 2 of fp32). Each thread reads its rows from shared memory,
// computes in fp32 pairs with the sm_100 f32x2 instructions and stores 8-byte vectors straight to
// global memory (a warp writes one contiguous 256-byte row segment per store).
//
// Reference: jxiong21029/causal-conv1d-triton, causal_conv1d_triton/causal_conv1d.py
// (`_fwd_kernel` :44-164, `_bwd_kernel` :167-341). The per-element arithmetic and its order
// follow the reference; the tiling, staging and scheduling are this file's own.
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

// Backward schedule knobs (see the step loop of cc1d_bwd_tma_kernel).
#ifndef CC1D_BWD_LAG
#define CC1D_BWD_LAG 0
#endif
#ifndef CC1D_BWD_DX_FAR_FIRST
#define CC1D_BWD_DX_FAR_FIRST 0
#endif
#ifndef CC1D_BWD_BIAS_FIRST
#define CC1D_BWD_BIAS_FIRST 0
#endif

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

template <typename T, int W, bool SEQ>
struct BwdLayout {
  using C = TileCfg<T, W>;
  static constexpr int XROWS = C::T_TILE + 2 * C::PAD;  // rows [t0 - PAD, t0 + T_TILE + PAD)
  static constexpr int YROWS = C::T_TILE + C::PAD;      // rows [t0, t0 + T_TILE + PAD)
  static constexpr int XBYTES = XROWS * C::ROW_BYTES;
  static constexpr int YBYTES = YROWS * C::ROW_BYTES;
  static constexpr int SEQ_BYTES = SEQ ? (XROWS * 4 + 127) / 128 * 128 : 0;
  static constexpr int STAGE_BYTES = XBYTES + YBYTES + SEQ_BYTES;
  // Two stages per CTA: up to W = 4 three CTAs (12 consumer warps) per SM fit in its 228 KB
  // (each CTA also reserves 1 KB), which hides more latency than a third stage would; wider
  // windows need more registers per thread and run two CTAs per SM.
  static constexpr int STAGES = 2;
  static constexpr int MIN_CTAS = W <= 4 ? 3 : 2;
  static constexpr int SMEM_BYTES = kSmemAlign + kBarBytes + STAGES * STAGE_BYTES;
  static constexpr int RED_BYTES = 4 * (W + 1) * C::D_TILE * 4;  // CTA-level dweight/dbias sum
  static_assert(RED_BYTES <= STAGES * STAGE_BYTES, "reduction buffer reuses the stages");
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

struct alignas(64) BwdParams {
  CUtensorMap tmap_x;   // x as (D, T, B), box (D_TILE, T_TILE + 2 PAD, 1)
  CUtensorMap tmap_dy;  // dout as (D, T, B), box (D_TILE, T_TILE + PAD, 1)
  const void* x;
  const void* weight;
  const void* bias;
  const void* init;
  const int32_t* seq;
  const void* dfinal;   // (B, W-1, D) contiguous, dtype of x, may be null
  void* dx;             // (B, T, D) contiguous, dtype of x
  void* dinit;          // (B, W-1, D) contiguous, dtype of init, may be null
  float* partials;      // (P, W+1, D) fp32, P = gridDim.x / n_db
  unsigned* status;
  int64_t sxb, sxt;
  int B, T, D;
  int n_tt, n_db;
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

// =============================================================================================
// Backward
// =============================================================================================
// Per tile, thread (lane_d, rg) walks its rows backwards in time from ts + R + PAD - 1 down to ts:
// the first PAD steps only recompute dz on the halo rows that follow its own rows; the next R
// steps produce dx, dweight and dbias for its own rows. Row group 0 of the first tile then
// continues to t = -PAD for dinitial_states. dz = dy * SiLU'(z) with z recomputed in the
// forward's order (causal_conv1d.py:274-288); dx[t] = sum_j w[PAD-j] dz[t+j] masked to the same
// sequence (:290-296) plus dfinal_states (:297-302).
template <typename T, int W, bool SEQ, bool SILU>
__global__ void __launch_bounds__(TileCfg<T, W>::THREADS, BwdLayout<T, W, SEQ>::MIN_CTAS)
    cc1d_bwd_tma_kernel(const __grid_constant__ BwdParams p) {
  using C = TileCfg<T, W>;
  using L = BwdLayout<T, W, SEQ>;
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
      mbar_init(&full[s], 32);
      mbar_init(&empty[s], 4);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 4) {
    // ---------------- producer warp ----------------
    if (lane == 0) {
      prefetch_tensormap(&p.tmap_x);
      prefetch_tensormap(&p.tmap_dy);
    }
    int issued = 0;
    for (int i = 0; i < n_my; ++i) {
      const int s = i % S;
      if (i >= S && !mbar_wait(&empty[s], ((i / S) - 1) & 1, p.status)) break;
      const int m = part + i * P;
      const int b = m / p.n_tt;
      const int t0 = (m - b * p.n_tt) * C::T_TILE;
      unsigned char* st = stage0 + s * L::STAGE_BYTES;
      if (lane == 0) {
        mbar_expect_tx(&full[s], L::XBYTES + L::YBYTES);
        tma_load_3d(st, &p.tmap_x, &full[s], db * DT, t0 - PAD, b);
        tma_load_3d(st + L::XBYTES, &p.tmap_dy, &full[s], db * DT, t0, b);
      }
      if constexpr (SEQ) {
        int* sq = reinterpret_cast<int*>(st + L::XBYTES + L::YBYTES);
        const int32_t* srow = p.seq + static_cast<int64_t>(b) * p.T;
        for (int r = lane; r < L::XROWS; r += 32) sq[r] = seq_at(srow, t0 - PAD + r, p.T, p.init != nullptr);
      }
      mbar_arrive(&full[s]);
      issued = i + 1;
    }
    if (lane == 0)
      for (int j = issued > S ? issued - S : 0; j < issued; ++j) mbar_wait(&full[j % S], (j / S) & 1, p.status);
    return;
  }

  // ---------------- consumer warps ----------------
  const int ct = threadIdx.x;
  const int lane_d = ct % C::LANES_D;
  const int rg = ct / C::LANES_D;
  const int d = db * DT + lane_d * CPT;
  const bool dvalid = d < p.D;
  const int64_t D = p.D;
  const int T_ = p.T;

  float2 w[W][NP], bv[NP];
  load_taps<W, NP>(p.weight, p.w_dtype, p.bias, p.b_dtype, d, dvalid, w, bv);
  float2 dw[W][NP], dbs[NP];
#pragma unroll
  for (int i2 = 0; i2 < NP; ++i2) {
    dbs[i2] = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < W; ++k) dw[k][i2] = make_float2(0.f, 0.f);
  }

  for (int i = 0; i < n_my; ++i) {
    const int s = i % S;
    const int m = part + i * P;
    const int b = m / p.n_tt;
    const int t0 = (m - b * p.n_tt) * C::T_TILE;
    if (!mbar_wait(&full[s], (i / S) & 1, p.status)) break;

    const unsigned char* st = stage0 + s * L::STAGE_BYTES;
    const T* xt = reinterpret_cast<const T*>(st) + lane_d * CPT;             // row of t: t - t0 + PAD
    const T* yt = reinterpret_cast<const T*>(st + L::XBYTES) + lane_d * CPT;  // row of t: t - t0
    const int* sq = reinterpret_cast<const int*>(st + L::XBYTES + L::YBYTES);  // row of t: t - t0 + PAD
    const int rb = rg * R;
    const int ts = t0 + rb;
    const bool init_rows = p.init != nullptr && ts == 0;

    // Step s (0 <= s < NS) handles row t = top - s, walking backwards in time; steps s < PAD are
    // the halo rows after this thread's own rows, which only provide dz. x rows are indexed from
    // the top as xr[i] = x[top - i]; the window of step s is x[t - PAD + k] = xr[s + PAD - k].
    // Each step is split into part A (load x and dy, recompute z, form dz) and part B (dx,
    // dweight, dbias of an own row), and part B of step s is issued after part A of step s + LAG
    // so that the independent A chains of later rows overlap the B chains of earlier ones.
    constexpr int NS = R + PAD;
    constexpr int NX = R + 2 * PAD;
    constexpr int LAG = CC1D_BWD_LAG;
    const int top_lt = rb + R + PAD - 1;  // t - t0 of step 0
    float2 xr[NX][NP];
    float2 dzr[NS][NP];

    auto load_x = [&](int i) {
      // global row top - i; local smem row rb + R + 2 PAD - 1 - i; init row R + 2 PAD - 1 - i
      if (i >= R + PAD && init_rows) {
        if (dvalid) {
          load_state_row<NP>(p.init, p.init_dtype, static_cast<int64_t>(b) * PAD + (R + 2 * PAD - 1 - i), p.D, d, xr[i]);
        } else {
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) xr[i][i2] = make_float2(0.f, 0.f);
        }
      } else {
        load_vec<T, CPT>(xt + (rb + R + 2 * PAD - 1 - i) * DT, xr[i]);
      }
    };

    auto part_a = [&](int s_, auto tail) {
      constexpr bool TAIL = decltype(tail)::value;
      const int lt = top_lt - s_;
      const int t = t0 + lt;
      if (s_ == 0) {
#pragma unroll
        for (int i = 0; i < PAD; ++i) load_x(i);
      }
      load_x(s_ + PAD);
      float2 dz[NP];
      load_vec<T, CPT>(yt + lt * DT, dz);
      const int seq_t = SEQ ? sq[lt + PAD] : 0;
      if constexpr (SILU) {
        float2 z[NP];
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2)
          z[i2] = CC1D_BWD_BIAS_FIRST ? ffma2(w[PAD][i2], xr[s_][i2], bv[i2]) : fmul2(w[PAD][i2], xr[s_][i2]);
#pragma unroll
        for (int k = 0; k < PAD; ++k) {
          if (!SEQ || sq[lt + k] == seq_t) {
#pragma unroll
            for (int i2 = 0; i2 < NP; ++i2) z[i2] = ffma2(w[k][i2], xr[s_ + PAD - k][i2], z[i2]);
          }
        }
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) {
          if (!CC1D_BWD_BIAS_FIRST) z[i2] = fadd2(z[i2], bv[i2]);
          const float2 sg = sigmoid2<FAST>(z[i2]);
          const float2 one = make_float2(1.f, 1.f);
          const float2 oms = fadd2(one, make_float2(-sg.x, -sg.y));
          // dz = dy * sig * (1 + z * (1 - sig))   (causal_conv1d.py:285-286)
          dz[i2] = fmul2(fmul2(dz[i2], sg), ffma2(z[i2], oms, one));
        }
      }
      if ((SEQ && seq_t < 0) || (TAIL && t >= T_)) {
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) dz[i2] = make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int i2 = 0; i2 < NP; ++i2) dzr[s_][i2] = dz[i2];
    };

    auto part_b = [&](int s_, auto tail) {
      constexpr bool TAIL = decltype(tail)::value;
      const int lt = top_lt - s_;
      const int t = t0 + lt;
      const int seq_t = SEQ ? sq[lt + PAD] : 0;
      // dx[t] = w[PAD] dz[t] + sum_j w[PAD - j] dz[t + j] (dz[t + j] is step s - j), masked to the
      // same sequence (causal_conv1d.py:290-296).
      float2 g[NP];
      if (CC1D_BWD_DX_FAR_FIRST) {
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) g[i2] = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = PAD; j >= 1; --j) {
          if (!SEQ || sq[lt + PAD + j] == seq_t) {
#pragma unroll
            for (int i2 = 0; i2 < NP; ++i2) g[i2] = ffma2(w[PAD - j][i2], dzr[s_ - j][i2], g[i2]);
          }
        }
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) g[i2] = ffma2(w[PAD][i2], dzr[s_][i2], g[i2]);
      } else {
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) g[i2] = fmul2(w[PAD][i2], dzr[s_][i2]);
#pragma unroll
        for (int j = 1; j <= PAD; ++j) {
          if (!SEQ || sq[lt + PAD + j] == seq_t) {
#pragma unroll
            for (int i2 = 0; i2 < NP; ++i2) g[i2] = ffma2(w[PAD - j][i2], dzr[s_ - j][i2], g[i2]);
          }
        }
      }
      if (TAIL && p.dfinal != nullptr && dvalid) {
        const int f = t - (T_ - PAD);
        if (f >= 0 && f < PAD) {
          float2 v[NP];
          load_state_row<NP>(p.dfinal, sizeof(T) == 4 ? kF32 : (std::is_same_v<T, __nv_bfloat16> ? kBF16 : kF16),
                             static_cast<int64_t>(b) * PAD + f, p.D, d, v);
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) g[i2] = fadd2(g[i2], v[i2]);
        }
      }
      if (!TAIL || (dvalid && t < T_))
        store_vec<T, CPT>(static_cast<T*>(p.dx) + (static_cast<int64_t>(b) * T_ + t) * D + d, g);
      // dweight / dbias partial sums (causal_conv1d.py:313-321).
#pragma unroll
      for (int k = 0; k < PAD; ++k) {
        if (!SEQ || sq[lt + k] == seq_t) {
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) dw[k][i2] = ffma2(dzr[s_][i2], xr[s_ + PAD - k][i2], dw[k][i2]);
        }
      }
#pragma unroll
      for (int i2 = 0; i2 < NP; ++i2) {
        dw[PAD][i2] = ffma2(dzr[s_][i2], xr[s_][i2], dw[PAD][i2]);
        dbs[i2] = fadd2(dbs[i2], dzr[s_][i2]);
      }
    };

    // With SiLU (compute-bound), interior tiles (every row of the window inside [0, T), no
    // final-state rows, every channel in range) run a copy of the loop without any per-row bounds
    // or final-state checks. Without it the kernel is bandwidth-bound and one general copy of the
    // loop is faster.
    const bool tail = !SILU || !dvalid || t0 + C::T_TILE + PAD > T_ || (p.dfinal != nullptr && t0 + C::T_TILE > T_ - PAD);
    if (SILU && !tail) {
#pragma unroll
      for (int u = 0; u < NS + LAG; ++u) {
        if (u < NS) part_a(u, std::false_type{});
        if (u - LAG >= PAD && u - LAG < NS) part_b(u - LAG, std::false_type{});
      }
    } else {
#pragma unroll
      for (int u = 0; u < NS + LAG; ++u) {
        if (u < NS) part_a(u, std::true_type{});
        if (u - LAG >= PAD && u - LAG < NS) part_b(u - LAG, std::true_type{});
      }
    }
    // dz of rows ts .. ts + PAD - 1, for the dinitial_states rows below.
    float2 dzs[PAD][NP];
#pragma unroll
    for (int j = 0; j < PAD; ++j)
#pragma unroll
      for (int i2 = 0; i2 < NP; ++i2) dzs[j][i2] = dzr[NS - 1 - j][i2];
    // dinitial_states: rows t = -1 .. -PAD, where dz = 0 (causal_conv1d.py:224-225, 306-311).
    if (p.dinit != nullptr && ts == 0 && dvalid) {
      const int seq0 = SEQ ? sq[PAD - 1] : 0;  // rows t < 0 carry seq_idx[b, 0]
#pragma unroll
      for (int q = 1; q <= PAD; ++q) {
        const int t = -q;
        float2 g[NP];
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) g[i2] = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 1; j <= PAD; ++j) {
          if (t + j >= 0 && (!SEQ || sq[t + j + PAD] == seq0)) {
#pragma unroll
            for (int i2 = 0; i2 < NP; ++i2) g[i2] = ffma2(w[PAD - j][i2], dzs[j - 1][i2], g[i2]);
          }
        }
        if (p.dfinal != nullptr) {
          const int f = t - (T_ - PAD);
          if (f >= 0 && f < PAD) {
            float2 v[NP];
            load_state_row<NP>(p.dfinal, sizeof(T) == 4 ? kF32 : (std::is_same_v<T, __nv_bfloat16> ? kBF16 : kF16),
                               static_cast<int64_t>(b) * PAD + f, p.D, d, v);
#pragma unroll
            for (int i2 = 0; i2 < NP; ++i2) g[i2] = fadd2(g[i2], v[i2]);
          }
        }
        const int64_t o = (static_cast<int64_t>(b) * PAD + t + PAD) * D + d;
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) {
          st_any(p.dinit, o + 2 * i2, p.init_dtype, g[i2].x);
          st_any(p.dinit, o + 2 * i2 + 1, p.init_dtype, g[i2].y);
        }
#pragma unroll
        for (int j = PAD - 1; j > 0; --j)
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) dzs[j][i2] = dzs[j - 1][i2];
#pragma unroll
        for (int i2 = 0; i2 < NP; ++i2) dzs[0][i2] = make_float2(0.f, 0.f);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // the stage (including its seq window) is free
  }

  // CTA-level sum of the dweight/dbias partials over the row groups that share a channel group:
  // a warp shuffle when a warp holds two row groups, then a fixed-order sum over the 4 warps in
  // shared memory. One (W+1) x D_TILE partial per CTA goes to global memory.
  if constexpr (C::LANES_D == 16) {
#pragma unroll
    for (int i2 = 0; i2 < NP; ++i2) {
#pragma unroll
      for (int k = 0; k < W; ++k) {
        dw[k][i2].x += __shfl_xor_sync(0xffffffffu, dw[k][i2].x, 16);
        dw[k][i2].y += __shfl_xor_sync(0xffffffffu, dw[k][i2].y, 16);
      }
      dbs[i2].x += __shfl_xor_sync(0xffffffffu, dbs[i2].x, 16);
      dbs[i2].y += __shfl_xor_sync(0xffffffffu, dbs[i2].y, 16);
    }
  }
  named_sync(1, C::CONSUMERS);  // all consumers are done with the stages
  float* red = reinterpret_cast<float*>(stage0);  // [4 warps][W + 1][D_TILE]
  if (lane < C::LANES_D) {
    float* rw = red + warp * (W + 1) * DT + lane_d * CPT;
#pragma unroll
    for (int i2 = 0; i2 < NP; ++i2) {
#pragma unroll
      for (int k = 0; k < W; ++k) *reinterpret_cast<float2*>(rw + k * DT + 2 * i2) = dw[k][i2];
      *reinterpret_cast<float2*>(rw + W * DT + 2 * i2) = dbs[i2];
    }
  }
  named_sync(1, C::CONSUMERS);
  for (int idx = ct; idx < (W + 1) * DT; idx += C::CONSUMERS) {
    const int k = idx / DT, c = idx - k * DT;
    const float v = ((red[idx] + red[(W + 1) * DT + idx]) + red[2 * (W + 1) * DT + idx]) + red[3 * (W + 1) * DT + idx];
    const int dc = db * DT + c;
    if (dc < p.D) p.partials[(static_cast<int64_t>(part) * (W + 1) + k) * D + dc] = v;
  }
}

}  // namespace cc1d
