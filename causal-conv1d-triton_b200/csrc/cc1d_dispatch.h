// Internal: tables of the compiled kernel variants, one translation unit per element type.
#pragma once

#include "cc1d_bwd_kernel.cuh"
#include "cc1d_generic_kernels.cuh"
#include "cc1d_tma_kernels.cuh"

namespace cc1d {

struct KernelInfo {
  const void* fn = nullptr;  // __global__ function
  int smem = 0;              // dynamic shared memory bytes
  int threads = 0;           // block size
  int d_tile = 0;            // channels per CTA tile (per CTA channel group for the TMA backward)
  int t_tile = 0;            // time rows per CTA tile (per pipeline stage for the TMA backward)
  int box_d = 0;             // channels per TMA box (TMA backward: per consumer warp)
  int min_regs = 0;          // registers per thread the launch must hold (warp-specialized backward)
};

// TMA path, template widths 2..8, 12 and 16; fn is null for other widths.
// `plain`: the variant that copies its tiles with plain loads / cp.async chunks instead of TMA.
template <typename T> KernelInfo fwd_tma_info(int W, bool seq, bool silu, bool plain);
// `long_stages`: the 24-row-stage kernel where the layout has one (see BwdCfg::LONG_STAGES).
template <typename T> KernelInfo bwd_tma_info(int W, bool seq, bool silu, bool plain, bool long_stages);
// Generic path, any width up to kGenericMaxWidth.
template <typename T> KernelInfo fwd_generic_info(int W);
template <typename T> KernelInfo bwd_generic_info(int W);

}  // namespace cc1d
