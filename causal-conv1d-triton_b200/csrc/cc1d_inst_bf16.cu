// Kernel variants for __nv_bfloat16 inputs (see cc1d_inst_impl.cuh).
#include "cc1d_inst_impl.cuh"

namespace cc1d {
template KernelInfo fwd_tma_info<__nv_bfloat16>(int, bool, bool, bool);
template KernelInfo bwd_tma_info<__nv_bfloat16>(int, bool, bool, bool, bool);
template KernelInfo fwd_generic_info<__nv_bfloat16>(int);
template KernelInfo bwd_generic_info<__nv_bfloat16>(int);
}  // namespace cc1d
