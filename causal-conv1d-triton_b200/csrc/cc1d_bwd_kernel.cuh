// TMA-pipelined sm_100a backward of the causal depthwise conv1d (template widths 2..8, 12, 16):
//
//   dz[t]  = dout[t] * act'(z[t]),   z[t] = bias + sum_k w[k] x[t-(W-1)+k]    (recomputed)
//   dx[t]  = sum_{j=0..W-1} w[W-1-j] dz[t+j]                                  (+ dfinal_states)
//   dw[k] += dz[t] x[t-(W-1)+k],  db += dz[t]                                 (over all b, t)
//
// Work decomposition. A CTA owns a channel group of WARPS x D_TILE channels (one channel block per
// consumer warp: 128 channels of bf16/fp16 with SiLU, 64 without, 64 of fp32) and one contiguous
// stretch of L rows of the
// flattened (batch, time) index, i.e. one or two contiguous time segments of batch rows. It walks
// each segment backwards in time, RS rows per pipeline stage (16, or 24 in the warp-specialized
// layout), from W-1 rows past the segment's end
// (the halo whose dz the segment's last dx rows need) down to the segment's first row, and then,
// for the segment that starts at t = 0 when initial states need a gradient, to t = -(W-1). Because
// the walk is continuous, every row's dz is computed once; only the W-1 halo rows per segment are
// computed twice. The dz of the W-1 most recent rows, and all partial sums, stay in registers.
//
// Each CTA runs one producer warp, which issues per stage one TMA load of x (rows a_lo-(W-1) ..
// a_lo+RS-1) and one of dout (rows a_lo .. a_lo+RS-1) per channel block into a 2-stage mbarrier ring
// and writes the stage's seq_idx window, and the consumer warps. With SiLU at template widths
// 5..8 the CTA is warp-specialized: warpgroup 0 (whose warp 0 is the producer) gives up its
// registers with setmaxnreg and two consumer warpgroups (8 channel blocks) take them, 232 per
// thread instead of 168, one CTA per SM. Stages are aligned to the bottom of each segment, so the
// last stage of a segment starts exactly at its first row; only the segment's top stage can be
// partial. Consumer lanes own CPT consecutive channels (a 4- or 8-byte vector) and compute in fp32 pairs
// with the sm_100 f32x2 instructions. A stage whose rows all belong to the segment (no halo, no
// initial-state rows, no final-state rows, channels in range) runs a copy of the step loop without
// any per-row checks.
//
// Each warp owns distinct channels, so at the end each thread writes its dweight/dbias partials
// for its channels straight to the (P, W+1, D) workspace (P = CTAs per channel group); a
// fixed-order reduction over P follows (cc1d_reduce_kernels.cuh).
//
// Reference: jxiong21029/causal-conv1d-triton, causal_conv1d_triton/causal_conv1d.py,
// `_bwd_kernel` :167-341 (per-element arithmetic and its order, except that the recomputed z takes
// the bias with its first tap; seq_idx conventions, dinit rows).
#pragma once

#include "cc1d_tma_kernels.cuh"

namespace cc1d {

// Most channel pieces dout may be split into (cc1d_bwd_split).
constexpr int kMaxDoutPieces = 4;

// Per-lane vector width and consumer warps per CTA. With SiLU the kernel is bound by arithmetic
// latency and runs best with 8-byte lanes (4 channels of bf16) and 4 warps per CTA; without it the
// kernel is bandwidth-bound and 4-byte lanes with 8 warps per CTA keep more rows in flight (both
// measured on B200 at BASELINE config 2).
// Warp-specialized walk for SiLU at template widths 5..8 on the TMA path: 1 (the default): one
// CTA per SM of a producer warpgroup and two consumer warpgroups; 2: two CTAs per SM of a
// producer warpgroup and one consumer warpgroup; 0: the 5-warp walk. The producer warpgroup gives
// its registers to the consumers with setmaxnreg (see BwdCfg). Measured on B200 at B=16 T=8192
// D=8192 W=8 bf16 with SiLU: 1530 / 1635 / 1866 us for 1 / 2 / 0 (without SiLU, where the walk is
// bound by its data movement, layout 1 is 5 % slower and 2 equal to 0). Four consumer warpgroups
// of 2-channel lanes (104 registers each) measured 1758 us against 1479 us for layout 1: at W = 8
// the per-row loads, conversions and loop work per channel count more than the extra warps.
#ifndef CC1D_BWD_WS
#define CC1D_BWD_WS 1
#endif

template <typename T, int W, bool SILU, bool PLAIN = false, bool LONG = false>
struct BwdCfg {
  static constexpr int ES = static_cast<int>(sizeof(T));
  // bytes per lane: 8 with SiLU, above W = 4 and for fp32; 4 without SiLU up to W = 4 and for
  // 16-bit template widths above 8 (whose 4-channel taps, sums and windows would not fit).
  static constexpr int VEC = ES == 4 ? 8 : (W > 8 ? 4 : ((SILU || W > 4) ? 8 : 4));
  static constexpr int ROW_BYTES = 32 * VEC;     // one channel block's row segment
  static constexpr int D_TILE = ROW_BYTES / ES;  // channels per warp
  static constexpr int CPT = VEC / ES;           // channels per lane
  static constexpr int NP = CPT / 2;             // fp32 pairs per lane
  // Warp specialization: a warp's registers come from one SM sub-partition (16K registers), so a
  // producer warp holding the consumers' register count wastes a consumer's share. In the
  // warp-specialized layout warps 0-3 (one warpgroup; warp 0 produces, 1-3 exit) drop to
  // REGS_PRODUCER registers and the consumer warpgroups rise to REGS_CONSUMER, which fills each
  // sub-partition exactly: 40 + 2 x 232 (one CTA per SM) or 2 x (40 + 216) (two CTAs).
  static constexpr int WS = (!PLAIN && SILU && W > 4 && W <= 8 && VEC == 8) ? CC1D_BWD_WS : 0;
  static constexpr int WARPS = WS == 1 ? 8 : ((VEC == 8 || W > 8) ? 4 : 8);  // consumer warps = channel blocks per CTA
  static constexpr int THREADS = WS ? 128 + WARPS * 32 : WARPS * 32 + 32;
  static constexpr int PRODUCER_WARP = WS ? 0 : WARPS;
  static constexpr int CONSUMER_WARP0 = WS ? 4 : 0;
  static constexpr int REGS_PRODUCER = 40;
  static constexpr int REGS_CONSUMER = WS == 1 ? 232 : 216;
  // Registers per thread the launch must hold for the split (setmaxnreg.inc waits for them).
  static constexpr int REGS_LAUNCH_MIN = WS ? (4 * REGS_PRODUCER + WARPS * REGS_CONSUMER + THREADS / 32 - 1) / (THREADS / 32) : 0;
  static constexpr int DG = WARPS * D_TILE;      // channels per CTA
  // Rows per stage: 16, or with LONG in the one-CTA warp-specialized layout 24, whose 2-stage ring
  // still fits in shared memory (226 KB at W = 8). Longer stages spread the per-stage work (barrier
  // waits, the W-1 halo rows of x loaded and converted again, the carried dz) over more rows, but
  // take longer to fill and drain the ring: the host picks LONG for long walks only (B200, SiLU,
  // bf16: 1476 -> 1430 us at B=16 T=8192 D=8192 W=8, 7282 rows per CTA; 477 -> 475 us at B=4
  // T=16384 D=4352 W=8, 2260 rows; 191 -> 204 us at B=8 T=8192 D=2048 W=7, 886 rows).
  static constexpr bool LONG_STAGES = LONG && WS == 1;
  static constexpr int RS = LONG_STAGES ? 24 : 16;
  static constexpr int PAD = W - 1;
  static constexpr int XROWS = RS + PAD;         // x rows a_lo - PAD .. a_lo + RS - 1
  static constexpr int SROWS = RS + 2 * PAD;     // seq rows a_lo - PAD .. a_lo + RS + PAD - 1
  static constexpr int XBYTES = WARPS * XROWS * ROW_BYTES;
  static constexpr int YBYTES = WARPS * RS * ROW_BYTES;
  // seq_idx window of a stage, then one int: non-zero when the whole window is one sequence
  // (ids equal and >= 0), where every mask of the stage passes.
  static constexpr int SEQ_BYTES = ((SROWS + 1) * 4 + 127) / 128 * 128;
  static constexpr int STAGE_BYTES = XBYTES + YBYTES + SEQ_BYTES;
  static constexpr int STAGES = 2;
  // CTAs per SM the registers are bounded for: three up to W = 4, two for wider windows (one or
  // two in the warp-specialized layouts).
  static constexpr int MIN_CTAS = WS == 1 ? 1 : (WS == 2 ? 2 : (W <= 4 ? 3 : 2));
  static constexpr int SMEM_BYTES = kSmemAlign + kBarBytes + STAGES * STAGE_BYTES;
  static_assert(RS >= PAD, "dinit rows come from the last stage of a segment");
  static_assert(!WS || REGS_LAUNCH_MIN * (THREADS / 32) <= 65536 / 32 / MIN_CTAS, "register split exceeds the SM");
};

struct alignas(64) BwdWalkParams {
  CUtensorMap tmap_x;   // x as (D, T, B), box (D_TILE, RS + PAD, 1)
  // dout as up to kMaxDoutPieces channel ranges, each its own (channels, T, B) tensor map with box
  // (D_TILE, RS, 1); piece i holds channels [dy_end[i-1], dy_end[i]) (dy_end[-1] = 0), and every
  // piece boundary is a multiple of D_TILE, so each channel block reads from one piece.
  CUtensorMap tmap_dy[kMaxDoutPieces];
  const void* weight;
  const void* bias;
  const void* init;     // (B, W-1, D) contiguous or null
  const int32_t* seq;   // (B, T) or null (the SEQ variant only)
  const void* dfinal;   // (B, W-1, D) contiguous, dtype of x, or null
  void* dx;             // (B, T, D) at strides (sdxb, sdxt, 1)
  void* dinit;          // (B, W-1, D) contiguous, dtype of init, or null
  float* partials;      // (P, W+1, D) fp32, P = gridDim.x / n_groups
  int64_t sdxb, sdxt;   // dx strides in elements (channel stride 1)
  // PLAIN variant (x or dout not addressable by a tensor map, rows a multiple of 8 bytes): the
  // producer copies the stage with 8-byte cp.async chunks from these, one dout piece only.
  const void* x;
  const void* dy;
  int64_t sxb, sxt, syb, syt;
  int dy_end[kMaxDoutPieces];
  int n_dy;
  unsigned* status;
  int64_t rows_per_part;  // L, a multiple of RS
  int B, T, D;
  int W;                  // true width: the template width less any leading zero taps
  int n_groups;           // channel groups of DG channels
  int w_dtype, b_dtype, init_dtype;
};

// The stages a CTA walks, in order: for each segment [s_lo, s_hi) of each batch row its stretch of
// rows touches, the stages from the top (partial) one down to the one starting at s_lo. The
// producer and the consumers run the same enumeration.
template <int RS, int PAD>
struct SegmentWalk {
  int64_t r0, r1;  // flattened rows [r0, r1) of this CTA
  int T;

  template <typename F>
  __device__ __forceinline__ void for_each_segment(F&& f) const {
    if (r0 >= r1) return;
    const int b_first = static_cast<int>(r0 / T), b_last = static_cast<int>((r1 - 1) / T);
    for (int b = b_first; b <= b_last; ++b) {
      const int64_t base = static_cast<int64_t>(b) * T;
      const int s_lo = static_cast<int>(r0 > base ? r0 - base : 0);
      const int s_hi = static_cast<int>(r1 - base < T ? r1 - base : T);
      const int t_top = (s_hi + PAD < T ? s_hi + PAD : T) - 1;
      const int n_st = (t_top - s_lo + RS) / RS;  // ceil((t_top - s_lo + 1) / RS)
      f(b, s_lo, s_hi, t_top, n_st);
    }
  }
};

template <typename T, int W, bool SEQ, bool SILU, bool PLAIN, bool LONG = false>
__global__ void __launch_bounds__(BwdCfg<T, W, SILU, PLAIN, LONG>::THREADS, BwdCfg<T, W, SILU, PLAIN, LONG>::MIN_CTAS)
    cc1d_bwd_walk_kernel(const __grid_constant__ BwdWalkParams p) {
  using C = BwdCfg<T, W, SILU, PLAIN, LONG>;
  constexpr int PAD = C::PAD, RS = C::RS, CPT = C::CPT, NP = C::NP, S = C::STAGES;
  constexpr int DT = C::D_TILE;
  constexpr bool FAST = sizeof(T) == 2;
  constexpr int XDT = sizeof(T) == 4 ? kF32 : (std::is_same_v<T, __nv_bfloat16> ? kBF16 : kF16);

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = aligned_smem<kSmemAlign>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  unsigned char* stage0 = smem + kBarBytes;

  const int ng = p.n_groups;
  const int g = blockIdx.x % ng;
  const int part = blockIdx.x / ng;
  const int T_ = p.T;
  const int64_t D = p.D;
  const int64_t total = static_cast<int64_t>(p.B) * T_;
  SegmentWalk<RS, PAD> walk;
  walk.r0 = static_cast<int64_t>(part) * p.rows_per_part;
  walk.r1 = walk.r0 + p.rows_per_part < total ? walk.r0 + p.rows_per_part : total;
  walk.T = T_;
  // Channel blocks of this group that hold any channel < D.
  const int nvb = min(C::WARPS, static_cast<int>((D - static_cast<int64_t>(g) * C::DG + DT - 1) / DT));

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], PLAIN ? 64 : 32);  // producer lanes (+ their cp.async completions)
      mbar_init(&empty[s], C::WARPS);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if constexpr (C::WS != 0) {
    // Every warp of a warpgroup takes part in its register change.
    if (warp < 4) {
      setmaxnreg_dec<C::REGS_PRODUCER>();
      if (warp != C::PRODUCER_WARP) return;
    } else {
      setmaxnreg_inc<C::REGS_CONSUMER>();
    }
  }
  if (warp == C::PRODUCER_WARP) {
    // ---------------- producer warp ----------------
    if (lane == 0 && !PLAIN) {
      prefetch_tensormap(&p.tmap_x);
      for (int i = 0; i < p.n_dy; ++i) prefetch_tensormap(&p.tmap_dy[i]);
    }
    int i = 0;
    bool ok = true;
    walk.for_each_segment([&](int b, int s_lo, int, int, int n_st) {
      for (int j = n_st - 1; j >= 0 && ok; --j, ++i) {
        const int a_lo = s_lo + RS * j;  // processed top stage first: j = n_st - 1 .. 0
        const int s = i % S;
        // The lanes leave together on a timeout (the seq_idx vote below is warp-wide).
        const bool got = i < S || mbar_wait(&empty[s], ((i / S) - 1) & 1, p.status);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        unsigned char* st = stage0 + s * C::STAGE_BYTES;
        if constexpr (PLAIN) {
          // The same stage layout from 8-byte chunks; chunks outside [0, T) or [0, D) are zeros.
          // Lane = chunk column (RPI rows per pass when a row segment has fewer chunks than lanes).
          constexpr int CPR = C::ROW_BYTES / 8, EPC = 8 / static_cast<int>(sizeof(T)), RPI = 32 / CPR;
          constexpr int64_t ES = sizeof(T);
          const int jc = lane % CPR, qo = lane / CPR;
          const unsigned char* xg = static_cast<const unsigned char*>(p.x);
          const unsigned char* yg = static_cast<const unsigned char*>(p.dy);
          for (int k = 0; k < nvb; ++k) {
            const int c = (g * C::WARPS + k) * DT + jc * EPC;
            const bool cv = c < p.D;
            const unsigned char* xcol = xg + (b * p.sxb + c) * ES;
            const unsigned char* ycol = yg + (b * p.syb + c) * ES;
            unsigned char* xdst = st + k * C::XROWS * C::ROW_BYTES + jc * 8;
            unsigned char* ydst = st + C::XBYTES + k * RS * C::ROW_BYTES + jc * 8;
#pragma unroll 4
            for (int q = qo; q < C::XROWS; q += RPI) {
              const int t = a_lo - PAD + q;
              const bool v = cv && t >= 0 && t < T_;
              cp_async_8(xdst + q * C::ROW_BYTES, v ? xcol + t * p.sxt * ES : xg, v ? 8 : 0);
            }
#pragma unroll 4
            for (int q = qo; q < RS; q += RPI) {
              const int t = a_lo + q;
              const bool v = cv && t < T_;
              cp_async_8(ydst + q * C::ROW_BYTES, v ? ycol + t * p.syt * ES : yg, v ? 8 : 0);
            }
          }
        } else if (lane == 0) {
          mbar_expect_tx(&full[s], static_cast<uint32_t>(nvb) * (C::XROWS + RS) * C::ROW_BYTES);
          for (int k = 0; k < nvb; ++k) {
            const int c0 = (g * C::WARPS + k) * DT;
            tma_load_3d(st + k * C::XROWS * C::ROW_BYTES, &p.tmap_x, &full[s], c0, a_lo - PAD, b);
            int pc = 0;
            while (pc + 1 < p.n_dy && c0 >= p.dy_end[pc]) ++pc;
            tma_load_3d(st + C::XBYTES + k * RS * C::ROW_BYTES, &p.tmap_dy[pc], &full[s],
                        c0 - (pc > 0 ? p.dy_end[pc - 1] : 0), a_lo, b);
          }
        }
        if constexpr (SEQ) {
          int* sq = reinterpret_cast<int*>(st + C::XBYTES + C::YBYTES);
          const int32_t* srow = p.seq + static_cast<int64_t>(b) * T_;
          const int first = seq_at(srow, a_lo - PAD, T_, p.init != nullptr);
          bool one = first >= 0;
          for (int r = lane; r < C::SROWS; r += 32) {
            const int v = seq_at(srow, a_lo - PAD + r, T_, p.init != nullptr);
            sq[r] = v;
            one = one && v == first;
          }
          one = __all_sync(0xffffffffu, one);
          if (lane == 0) sq[C::SROWS] = one ? 1 : 0;
        }
        mbar_arrive(&full[s]);
        if constexpr (PLAIN) cp_async_mbar_arrive_noinc(&full[s]);
      }
    });
    // Every copy this CTA issued must have landed before the CTA may exit.
    if (lane == 0)
      for (int j = i > S ? i - S : 0; j < i; ++j) mbar_wait(&full[j % S], (j / S) & 1, p.status);
    return;
  }

  // ---------------- consumer warps: warp = channel block ----------------
  const int blk = warp - C::CONSUMER_WARP0;
  const bool blk_valid = blk < nvb;
  const int d = (g * C::WARPS + blk) * DT + lane * CPT;
  const bool dvalid = d < p.D;
  const bool has_init = p.init != nullptr;

  // With SiLU on 16-bit data the taps are halved: the step below computes h = z / 2 and carries
  // dz2 = 2 dz, so w dz2 products equal the reference's w dz and dweight / dbias are halved once
  // at the end (all exact power-of-two scalings).
  constexpr bool HALF = SILU && FAST;
  float2 w[W][NP], bv[NP];
  if (p.W == W) {
    load_taps<W, NP>(p.weight, p.w_dtype, p.bias, p.b_dtype, d, dvalid, w, bv);
  } else {
    load_taps_off<W, NP>(p.weight, p.w_dtype, p.bias, p.b_dtype, d, dvalid, p.W, w, bv);
  }
  if constexpr (HALF) halve_taps<W, NP>(w, bv);
  const int pw = p.W - 1, off = W - p.W;  // true state rows; leading zero taps
  float2 dw[W][NP], dbs[NP];
#pragma unroll
  for (int i2 = 0; i2 < NP; ++i2) {
    dbs[i2] = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < W; ++k) dw[k][i2] = make_float2(0.f, 0.f);
  }

  int i = 0;
  bool ok = true;
  walk.for_each_segment([&](int b, int s_lo, int s_hi, int t_top, int n_st) {
    // dzs[j] = dz[a_hi + 1 + j]: the dz of the PAD rows above the current stage.
    float2 dzs[PAD][NP];
#pragma unroll
    for (int j = 0; j < PAD; ++j)
#pragma unroll
      for (int i2 = 0; i2 < NP; ++i2) dzs[j][i2] = make_float2(0.f, 0.f);

    for (int jst = n_st - 1; jst >= 0 && ok; --jst, ++i) {
      const int s = i % S;
      const int a_lo = s_lo + RS * jst;
      const int a_hi = a_lo + RS - 1;
      if (!mbar_wait(&full[s], (i / S) & 1, p.status)) {
        ok = false;
        break;
      }
      const unsigned char* st = stage0 + s * C::STAGE_BYTES;
      // x row q <-> global row a_lo - PAD + q; dy row q <-> a_lo + q; seq row q <-> a_lo - PAD + q.
      const T* xt = reinterpret_cast<const T*>(st + blk * C::XROWS * C::ROW_BYTES) + lane * CPT;
      const T* yt = reinterpret_cast<const T*>(st + C::XBYTES + blk * RS * C::ROW_BYTES) + lane * CPT;
      const int* sq = reinterpret_cast<const int*>(st + C::XBYTES + C::YBYTES);

      if (blk_valid) {
        // Step s handles row t = a_hi - s. xr[i] = x[a_hi - i] (x row RS - 1 + PAD - i); the window
        // of step s is x[t - PAD + k] = xr[s + PAD - k]. dzall[PAD + s] = dz of step s and
        // dzall[PAD - 1 - j] = dzs[j], so dz[t + j] = dzall[PAD + s - j].
        float2 xr[RS + PAD][NP];
        float2 dzall[PAD + RS][NP];
#pragma unroll
        for (int j = 0; j < PAD; ++j)
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) dzall[PAD - 1 - j][i2] = dzs[j][i2];

        auto load_x = [&](int ix, auto general) {
          constexpr bool GEN = decltype(general)::value;
          const int q = RS - 1 + PAD - ix;
          if (GEN && has_init && a_lo - PAD + q < 0) {
            const int ir = a_lo - PAD + q + pw;  // initial_states row of t = a_lo - PAD + q
            if (dvalid && ir >= 0) {
              load_state_row<NP>(p.init, p.init_dtype, static_cast<int64_t>(b) * pw + ir, p.D, d, xr[ix]);
            } else {
#pragma unroll
              for (int i2 = 0; i2 < NP; ++i2) xr[ix][i2] = make_float2(0.f, 0.f);
            }
          } else {
            load_vec<T, CPT>(xt + q * DT, xr[ix]);
          }
        };

        // dx row of step s_ (row a_hi - s_), moved down one row per step.
        T* dxrow = static_cast<T*>(p.dx) + b * p.sdxb + static_cast<int64_t>(a_hi) * p.sdxt + d;
        // masked: apply the seq_idx masks (false for stages whose window is one sequence, where
        // every mask passes; the results are the same bits).
        auto step = [&](int s_, auto general, auto masked) {
          constexpr bool GEN = decltype(general)::value;
          constexpr bool SQ = SEQ && decltype(masked)::value;
          const int t = a_hi - s_;
          if (s_ > 0) dxrow -= p.sdxt;
          const int qs = RS - 1 - s_ + PAD;  // seq row of t
          if (s_ == 0) {
#pragma unroll
            for (int ix = 0; ix < PAD; ++ix) load_x(ix, general);
          }
          load_x(s_ + PAD, general);
          // Row classes (general stages only): above the walk (t > t_top: dz = 0), halo rows
          // (s_hi <= t <= t_top: dz only), own rows.
          const bool above = GEN && t > t_top;
          const bool own = !GEN || t < s_hi;
          float2 dz[NP];
          load_vec<T, CPT>(yt + (RS - 1 - s_) * DT, dz);
          const int seq_t = SQ ? sq[qs] : 0;
          if constexpr (SILU) {
            float2 z[NP];
#pragma unroll
            for (int i2 = 0; i2 < NP; ++i2) z[i2] = ffma2(w[PAD][i2], xr[s_][i2], bv[i2]);
#pragma unroll
            for (int k = 0; k < PAD; ++k) {
              if (!SQ || sq[qs - PAD + k] == seq_t) {
#pragma unroll
                for (int i2 = 0; i2 < NP; ++i2) z[i2] = ffma2(w[k][i2], xr[s_ + PAD - k][i2], z[i2]);
              }
            }
#pragma unroll
            for (int i2 = 0; i2 < NP; ++i2) {
              // dz = dy * sig * (1 + z * (1 - sig))   (causal_conv1d.py:285-286)
              if constexpr (HALF) {
                dz[i2] = dsilu2_of_half(z[i2], dz[i2]);  // z holds h = z / 2; this is 2 dz
              } else {
                const float2 sg = sigmoid2<FAST>(z[i2]);
                const float2 one = make_float2(1.f, 1.f);
                const float2 oms = ffma2(sg, make_float2(-1.f, -1.f), one);
                dz[i2] = fmul2(fmul2(dz[i2], sg), ffma2(z[i2], oms, one));
              }
            }
          }
          if ((SQ && seq_t < 0) || above) {
#pragma unroll
            for (int i2 = 0; i2 < NP; ++i2) dz[i2] = make_float2(0.f, 0.f);
          }
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) dzall[PAD + s_][i2] = dz[i2];
          if (!own) return;

          // dx[t] = w[PAD] dz[t] + sum_j w[PAD - j] dz[t + j], masked to the same sequence
          // (causal_conv1d.py:290-296), + dfinal_states (:297-302).
          float2 gx[NP];
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) gx[i2] = fmul2(w[PAD][i2], dz[i2]);
#pragma unroll
          for (int j = 1; j <= PAD; ++j) {
            if (!SQ || sq[qs + j] == seq_t) {
#pragma unroll
              for (int i2 = 0; i2 < NP; ++i2) gx[i2] = ffma2(w[PAD - j][i2], dzall[PAD + s_ - j][i2], gx[i2]);
            }
          }
          if (GEN && p.dfinal != nullptr && dvalid) {
            const int f = t - (T_ - pw);
            if (f >= 0) {
              float2 v[NP];
              load_state_row<NP>(p.dfinal, XDT, static_cast<int64_t>(b) * pw + f, p.D, d, v);
#pragma unroll
              for (int i2 = 0; i2 < NP; ++i2) gx[i2] = fadd2(gx[i2], v[i2]);
            }
          }
          if (!GEN || dvalid) store_vec<T, CPT>(dxrow, gx);
          // dweight / dbias partial sums (causal_conv1d.py:313-321).
#pragma unroll
          for (int k = 0; k < PAD; ++k) {
            if (!SQ || sq[qs - PAD + k] == seq_t) {
#pragma unroll
              for (int i2 = 0; i2 < NP; ++i2) dw[k][i2] = ffma2(dz[i2], xr[s_ + PAD - k][i2], dw[k][i2]);
            }
          }
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) {
            dw[PAD][i2] = ffma2(dz[i2], xr[s_][i2], dw[PAD][i2]);
            dbs[i2] = fadd2(dbs[i2], dz[i2]);
          }
        };

        const bool interior = a_hi < s_hi && a_lo - PAD >= 0 && dvalid &&
                              !(p.dfinal != nullptr && a_hi >= T_ - PAD);
        if (interior && SEQ && sq[C::SROWS] != 0) {
#pragma unroll
          for (int s_ = 0; s_ < RS; ++s_) step(s_, std::false_type{}, std::false_type{});
        } else if (interior) {
#pragma unroll
          for (int s_ = 0; s_ < RS; ++s_) step(s_, std::false_type{}, std::true_type{});
        } else {
#pragma unroll
          for (int s_ = 0; s_ < RS; ++s_) step(s_, std::true_type{}, std::true_type{});
        }
        // Carry the dz of this stage's lowest PAD rows into the next stage.
#pragma unroll
        for (int j = 0; j < PAD; ++j)
#pragma unroll
          for (int i2 = 0; i2 < NP; ++i2) dzs[j][i2] = dzall[PAD + RS - 1 - j][i2];

        // dinitial_states: rows t = -1 .. -PAD after the stage that starts at t = 0, where dz = 0
        // (causal_conv1d.py:224-225, 306-311). dzs[j] = dz[j] here.
        if (jst == 0 && s_lo == 0 && p.dinit != nullptr && dvalid) {
          const int seq0 = SEQ ? sq[PAD - 1] : 0;  // rows t < 0 carry seq_idx[b, 0]
#pragma unroll
          for (int q = 1; q <= PAD; ++q) {
            if (q > pw) break;  // rows t < -(W-1) have no initial state (their taps are zero)
            const int t = -q;
            float2 gx[NP];
#pragma unroll
            for (int i2 = 0; i2 < NP; ++i2) gx[i2] = make_float2(0.f, 0.f);
#pragma unroll
            for (int j = q; j <= PAD; ++j) {  // dz[t + j] with t + j >= 0
              if (!SEQ || sq[t + j + PAD] == seq0) {
#pragma unroll
                for (int i2 = 0; i2 < NP; ++i2) gx[i2] = ffma2(w[PAD - j][i2], dzs[j - q][i2], gx[i2]);
              }
            }
            if (p.dfinal != nullptr) {
              const int f = t - (T_ - pw);
              if (f >= 0) {
                float2 v[NP];
                load_state_row<NP>(p.dfinal, XDT, static_cast<int64_t>(b) * pw + f, p.D, d, v);
#pragma unroll
                for (int i2 = 0; i2 < NP; ++i2) gx[i2] = fadd2(gx[i2], v[i2]);
              }
            }
            const int64_t o = (static_cast<int64_t>(b) * pw + t + pw) * D + d;
#pragma unroll
            for (int i2 = 0; i2 < NP; ++i2) {
              st_any(p.dinit, o + 2 * i2, p.init_dtype, gx[i2].x);
              st_any(p.dinit, o + 2 * i2 + 1, p.init_dtype, gx[i2].y);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  });

  if constexpr (HALF) {
    const float2 half = make_float2(0.5f, 0.5f);
#pragma unroll
    for (int i2 = 0; i2 < NP; ++i2) {
      dbs[i2] = fmul2(dbs[i2], half);
#pragma unroll
      for (int k = 0; k < W; ++k) dw[k][i2] = fmul2(dw[k][i2], half);
    }
  }
  // This thread's channels belong to this warp alone: write the partial sums directly.
  if (dvalid) {
    // Partial row layout (W+1, D) with the true width; the leading zero taps are not stored.
    float* pp = p.partials + static_cast<int64_t>(part) * (p.W + 1) * D + d;
#pragma unroll
    for (int k = 0; k < W; ++k) {
      if (k < off) continue;
#pragma unroll
      for (int i2 = 0; i2 < NP; ++i2) *reinterpret_cast<float2*>(pp + (k - off) * D + 2 * i2) = dw[k][i2];
    }
#pragma unroll
    for (int i2 = 0; i2 < NP; ++i2) *reinterpret_cast<float2*>(pp + p.W * D + 2 * i2) = dbs[i2];
  }
}

}  // namespace cc1d
