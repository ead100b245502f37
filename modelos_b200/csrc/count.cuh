// Per-slot occurrence counts (a bincount of int64 slot indices into int32
// bins), shared by the fast-weight update and the addressing statistics.
#pragma once

#include "common.cuh"

namespace pkm {

// counts[k] += 1 for every index k in [0, rows); the caller zeroes counts.
// Indices outside [0, rows) set PKM_DEVERR_INDEX and are not counted.
// Internal linkage: every translation unit that launches it has its own copy.
static __global__ void slot_count_kernel(const int64_t* __restrict__ idx, int64_t n, int64_t rows,
                                         int32_t* __restrict__ counts, uint32_t* err) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = idx[i];
    if (k < 0 || k >= rows) {
      raise_err(err, PKM_DEVERR_INDEX);
      continue;
    }
    atomicAdd(&counts[k], 1);
  }
}

}  // namespace pkm
