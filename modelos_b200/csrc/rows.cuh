// Row-streaming helpers shared by the column-wise kernels (batch norm,
// SwiGLU, column sums) over row-major [n, c] activations: a thread owns 8
// consecutive channels (one 16-byte vector of bf16), a warp 256 channels, the
// rows of a column tile are split over the grid's second dimension, and
// per-channel reductions go through per-row-block partials summed in a fixed
// order (deterministic).
#pragma once

#include <algorithm>

#include "common.cuh"

namespace pkm {

constexpr int kNormThreads = 256;  // 8 warps
constexpr int kNormChan = 8;       // channels per thread (one 16-byte vector of bf16)

template <typename T>
struct RowIO;
template <>
struct RowIO<float> {
  __device__ static __forceinline__ void load(const float* p, float (&v)[kNormChan]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
  __device__ static __forceinline__ void store(float* p, const float (&v)[kNormChan]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
};
template <>
struct RowIO<__nv_bfloat16> {
  __device__ static __forceinline__ void load(const __nv_bfloat16* p, float (&v)[kNormChan]) {
    VecTraits<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(p), v);
  }
  __device__ static __forceinline__ void store(__nv_bfloat16* p, const float (&v)[kNormChan]) {
    st_run(p, PKM_DT_BF16, 0, v, kNormChan);
  }
};

// Row range of row block rb of nb over n rows.
__device__ __forceinline__ void row_range(int64_t n, int rb, int nb, int64_t& r0, int64_t& r1) {
  r0 = n * rb / nb;
  r1 = n * (rb + 1) / nb;
}


// Row blocks of the grid's second dimension: about 4 blocks per SM over the
// whole grid, at least 64 rows per block.
inline int row_blocks(int64_t n, int64_t c) {
  const int64_t tiles = (c + 32 * kNormChan - 1) / (32 * kNormChan);
  int64_t nb = std::max<int64_t>(1, (int64_t)num_sms() * 4 / std::max<int64_t>(tiles, 1));
  nb = std::min<int64_t>(nb, std::max<int64_t>(1, n / 64));
  return (int)std::min<int64_t>(nb, 4096);
}

// Fixed-order sum of the per-row-block partials part[rb][ch] (rb < nb) for
// the 32 channels of this block (blockDim 256, grid ceil(c / 32)): warp w
// adds blocks w, w+8, w+16, ... in order (fp64), then warp 0 adds the eight
// warp sums in warp order.  Valid in warp 0 (lane = channel in the group);
// every thread of the block must call it.
struct Sum2 {
  double a, b;
};
__device__ __forceinline__ Sum2 colsum_fixed(const float* part, const float2* part2, int nb, int64_t c) {
  __shared__ double sa[8][32], sb[8][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ch = (int64_t)blockIdx.x * 32 + lane;
  double a = 0.0, b = 0.0;
  if (ch < c) {
    for (int rb = warp; rb < nb; rb += 8) {
      if (part2) {
        const float2 v = part2[(int64_t)rb * c + ch];
        a += v.x;
        b += v.y;
      } else {
        a += part[(int64_t)rb * c + ch];
      }
    }
  }
  sa[warp][lane] = a;
  sb[warp][lane] = b;
  __syncthreads();
  Sum2 r{0.0, 0.0};
  if (warp == 0) {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      r.a += sa[w][lane];
      r.b += sb[w][lane];
    }
  }
  return r;
}

inline dim3 row_grid(int64_t n, int64_t c) {
  return dim3((unsigned)((c + 32 * kNormChan - 1) / (32 * kNormChan)), (unsigned)row_blocks(n, c));
}

}  // namespace pkm
