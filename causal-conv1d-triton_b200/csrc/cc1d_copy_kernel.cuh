// Copy of a (B, T, C) channel block between two channels-last tensors with their own batch/time
// strides (channel stride 1 on both sides): the glue that assembles d(zxbcdt) around the split
// backward (cc1d_bwd_split writes the xBC slice; this kernel places dz and ddt). Each thread moves
// one VB-byte vector; VB is the widest of 16/8/4/2 bytes that divides both bases, both strides and
// the row length, so a 4096-channel bf16 row moves as 512 16-byte vectors.
#pragma once

#include "cc1d_device.cuh"

namespace cc1d {

struct CopyParams {
  const unsigned char* src;
  unsigned char* dst;
  int64_t src_sb, src_st, dst_sb, dst_st;  // strides in bytes
  int64_t T, rows;                         // rows = B * T
  int64_t vpr;                             // vectors per row
};

template <int VB>
__global__ void __launch_bounds__(256) cc1d_copy_channels_kernel(const CopyParams p) {
  using V = std::conditional_t<VB == 16, uint4, std::conditional_t<VB == 8, uint2, std::conditional_t<VB == 4, uint32_t, uint16_t>>>;
  const int64_t n = p.rows * p.vpr;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / p.vpr, v = i - r * p.vpr;
    const int64_t b = r / p.T, t = r - b * p.T;
    const V val = *reinterpret_cast<const V*>(p.src + b * p.src_sb + t * p.src_st + v * VB);
    *reinterpret_cast<V*>(p.dst + b * p.dst_sb + t * p.dst_st + v * VB) = val;
  }
}

}  // namespace cc1d
