// Internal: definitions of the variant tables declared in cc1d_dispatch.h. Included by one
// translation unit per element type, which instantiates them explicitly.
#pragma once

#include "cc1d_dispatch.h"

namespace cc1d {
namespace detail {

template <typename T, int W, bool SEQ, bool SILU, bool PLAIN>
KernelInfo fwd_tma_one() {
  using C = TileCfg<T, W>;
  return {reinterpret_cast<const void*>(&cc1d_fwd_tma_kernel<T, W, SEQ, SILU, PLAIN>), FwdLayout<T, W, SEQ>::SMEM_BYTES,
          C::CONSUMERS, C::D_TILE, C::T_TILE, C::D_TILE};
}
template <typename T, int W, bool SEQ, bool SILU, bool PLAIN, bool LONG = false>
KernelInfo bwd_tma_one() {
  using C = BwdCfg<T, W, SILU, PLAIN, LONG>;
  return {reinterpret_cast<const void*>(&cc1d_bwd_walk_kernel<T, W, SEQ, SILU, PLAIN, LONG>), C::SMEM_BYTES, C::THREADS,
          C::DG, C::RS, C::D_TILE, C::REGS_LAUNCH_MIN};
}
template <typename T, int W, bool PLAIN>
KernelInfo fwd_tma_p(bool seq, bool silu) {
  if (seq) return silu ? fwd_tma_one<T, W, true, true, PLAIN>() : fwd_tma_one<T, W, true, false, PLAIN>();
  return silu ? fwd_tma_one<T, W, false, true, PLAIN>() : fwd_tma_one<T, W, false, false, PLAIN>();
}
template <typename T, int W>
KernelInfo fwd_tma_w(bool seq, bool silu, bool plain) {
  return plain ? fwd_tma_p<T, W, true>(seq, silu) : fwd_tma_p<T, W, false>(seq, silu);
}
template <typename T, int W, bool PLAIN>
KernelInfo bwd_tma_p(bool seq, bool silu, bool long_stages) {
  // Long stages exist only for the layouts that have them (BwdCfg::LONG_STAGES); elsewhere the
  // request falls back to the 16-row kernel (t_tile tells the caller which it got).
  if constexpr (BwdCfg<T, W, true, PLAIN, true>::LONG_STAGES) {
    if (silu && long_stages)
      return seq ? bwd_tma_one<T, W, true, true, PLAIN, true>() : bwd_tma_one<T, W, false, true, PLAIN, true>();
  }
  if (seq) return silu ? bwd_tma_one<T, W, true, true, PLAIN>() : bwd_tma_one<T, W, true, false, PLAIN>();
  return silu ? bwd_tma_one<T, W, false, true, PLAIN>() : bwd_tma_one<T, W, false, false, PLAIN>();
}
template <typename T, int W>
KernelInfo bwd_tma_w(bool seq, bool silu, bool plain, bool long_stages) {
  return plain ? bwd_tma_p<T, W, true>(seq, silu, long_stages) : bwd_tma_p<T, W, false>(seq, silu, long_stages);
}

}  // namespace detail

template <typename T>
KernelInfo fwd_tma_info(int W, bool seq, bool silu, bool plain) {
  switch (W) {
    case 2: return detail::fwd_tma_w<T, 2>(seq, silu, plain);
    case 3: return detail::fwd_tma_w<T, 3>(seq, silu, plain);
    case 4: return detail::fwd_tma_w<T, 4>(seq, silu, plain);
    case 5: return detail::fwd_tma_w<T, 5>(seq, silu, plain);
    case 6: return detail::fwd_tma_w<T, 6>(seq, silu, plain);
    case 7: return detail::fwd_tma_w<T, 7>(seq, silu, plain);
    case 8: return detail::fwd_tma_w<T, 8>(seq, silu, plain);
    case 12: return detail::fwd_tma_w<T, 12>(seq, silu, plain);
    case 16: return detail::fwd_tma_w<T, 16>(seq, silu, plain);
    default: return {};
  }
}

template <typename T>
KernelInfo bwd_tma_info(int W, bool seq, bool silu, bool plain, bool long_stages) {
  switch (W) {
    case 2: return detail::bwd_tma_w<T, 2>(seq, silu, plain, long_stages);
    case 3: return detail::bwd_tma_w<T, 3>(seq, silu, plain, long_stages);
    case 4: return detail::bwd_tma_w<T, 4>(seq, silu, plain, long_stages);
    case 5: return detail::bwd_tma_w<T, 5>(seq, silu, plain, long_stages);
    case 6: return detail::bwd_tma_w<T, 6>(seq, silu, plain, long_stages);
    case 7: return detail::bwd_tma_w<T, 7>(seq, silu, plain, long_stages);
    case 8: return detail::bwd_tma_w<T, 8>(seq, silu, plain, long_stages);
    case 12: return detail::bwd_tma_w<T, 12>(seq, silu, plain, long_stages);
    case 16: return detail::bwd_tma_w<T, 16>(seq, silu, plain, long_stages);
    default: return {};
  }
}

template <typename T>
KernelInfo fwd_generic_info(int W) {
  return {reinterpret_cast<const void*>(&cc1d_fwd_generic_kernel<T>), generic_fwd_smem(W), GTHREADS, GC, GT};
}

template <typename T>
KernelInfo bwd_generic_info(int W) {
  return {reinterpret_cast<const void*>(&cc1d_bwd_generic_kernel<T>), generic_bwd_smem(W), GTHREADS, GC, GT};
}

}  // namespace cc1d
