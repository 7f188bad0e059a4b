// Internal: definitions of the variant tables declared in cc1d_dispatch.h. Included by one
// translation unit per element type, which instantiates them explicitly.
#pragma once

#include "cc1d_dispatch.h"

namespace cc1d {
namespace detail {

template <typename T, int W, bool SEQ, bool SILU>
KernelInfo fwd_tma_one() {
  using C = TileCfg<T, W>;
  return {reinterpret_cast<const void*>(&cc1d_fwd_tma_kernel<T, W, SEQ, SILU>), FwdLayout<T, W, SEQ>::SMEM_BYTES,
          C::CONSUMERS, C::D_TILE, C::T_TILE, C::D_TILE};
}
template <typename T, int W, bool SEQ, bool SILU>
KernelInfo bwd_tma_one() {
  using C = BwdCfg<T, W, SILU>;
  return {reinterpret_cast<const void*>(&cc1d_bwd_walk_kernel<T, W, SEQ, SILU>), C::SMEM_BYTES, C::THREADS, C::DG,
          C::RS, C::D_TILE};
}
template <typename T, int W>
KernelInfo fwd_tma_w(bool seq, bool silu) {
  if (seq) return silu ? fwd_tma_one<T, W, true, true>() : fwd_tma_one<T, W, true, false>();
  return silu ? fwd_tma_one<T, W, false, true>() : fwd_tma_one<T, W, false, false>();
}
template <typename T, int W>
KernelInfo bwd_tma_w(bool seq, bool silu) {
  if (seq) return silu ? bwd_tma_one<T, W, true, true>() : bwd_tma_one<T, W, true, false>();
  return silu ? bwd_tma_one<T, W, false, true>() : bwd_tma_one<T, W, false, false>();
}

}  // namespace detail

template <typename T>
KernelInfo fwd_tma_info(int W, bool seq, bool silu) {
  switch (W) {
    case 2: return detail::fwd_tma_w<T, 2>(seq, silu);
    case 3: return detail::fwd_tma_w<T, 3>(seq, silu);
    case 4: return detail::fwd_tma_w<T, 4>(seq, silu);
    case 5: return detail::fwd_tma_w<T, 5>(seq, silu);
    case 6: return detail::fwd_tma_w<T, 6>(seq, silu);
    case 7: return detail::fwd_tma_w<T, 7>(seq, silu);
    case 8: return detail::fwd_tma_w<T, 8>(seq, silu);
    case 12: return detail::fwd_tma_w<T, 12>(seq, silu);
    case 16: return detail::fwd_tma_w<T, 16>(seq, silu);
    default: return {};
  }
}

template <typename T>
KernelInfo bwd_tma_info(int W, bool seq, bool silu) {
  switch (W) {
    case 2: return detail::bwd_tma_w<T, 2>(seq, silu);
    case 3: return detail::bwd_tma_w<T, 3>(seq, silu);
    case 4: return detail::bwd_tma_w<T, 4>(seq, silu);
    case 5: return detail::bwd_tma_w<T, 5>(seq, silu);
    case 6: return detail::bwd_tma_w<T, 6>(seq, silu);
    case 7: return detail::bwd_tma_w<T, 7>(seq, silu);
    case 8: return detail::bwd_tma_w<T, 8>(seq, silu);
    case 12: return detail::bwd_tma_w<T, 12>(seq, silu);
    case 16: return detail::bwd_tma_w<T, 16>(seq, silu);
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
