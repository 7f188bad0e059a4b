// seq_idx from cumulative sequence boundaries, for packed variable-length batches.
//
// Row b of the batch holds sequences [cu[b][i], cu[b][i+1]) for i < n_seqs (cu is (B, n_seqs + 1),
// non-decreasing, cu[b][0] = 0). Position t gets the id of the sequence containing it, and -1 (the
// reference's padding id, README.md:44-46, causal_conv1d.py:17-25) at or past cu[b][n_seqs]. One
// thread per (b, t): a binary search over the row's boundaries, so a warp writes 32 consecutive
// positions.
#pragma once

#include "cc1d_device.cuh"

namespace cc1d {

__global__ void __launch_bounds__(256) cc1d_seq_idx_kernel(const int32_t* __restrict__ cu, int n_seqs,
                                                           int32_t* __restrict__ seq_idx, int B, int T) {
  const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<int64_t>(B) * T) return;
  const int b = static_cast<int>(idx / T), t = static_cast<int>(idx - static_cast<int64_t>(b) * T);
  const int32_t* row = cu + static_cast<int64_t>(b) * (n_seqs + 1);
  int id = -1;
  if (t < row[n_seqs]) {
    // largest i with row[i] <= t, i in [0, n_seqs)
    int lo = 0, hi = n_seqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (row[mid] <= t)
        lo = mid;
      else
        hi = mid - 1;
    }
    id = lo;
  }
  seq_idx[idx] = id;
}

}  // namespace cc1d
