// Kernel variants for float inputs (see cc1d_inst_impl.cuh).
#include "cc1d_inst_impl.cuh"

namespace cc1d {
template KernelInfo fwd_tma_info<float>(int, bool, bool, bool);
template KernelInfo bwd_tma_info<float>(int, bool, bool, bool, bool);
template KernelInfo fwd_generic_info<float>(int);
template KernelInfo bwd_generic_info<float>(int);
}  // namespace cc1d
