// Device-wide exclusive scan and a stable LSD radix sort of (key, occurrence)
// pairs.  Both are written for the bag backward (K4): the scan turns per-row
// occurrence counts into segment offsets, and the sort orders occurrence ids
// by row with ties kept in ascending occurrence order, which is what makes
// the segment sums of K4 deterministic.  The row-sharded routing uses one
// pass of the same sort (the owner rank as the digit) and the scan.  The
// non-template kernels have internal linkage so that several translation
// units can include this header.
#pragma once

#include "common.cuh"

namespace pkm {

struct I4 {
  int x, y, z, w;
};
__device__ __forceinline__ I4 operator+(const I4& a, const I4& b) {
  return I4{a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w};
}

template <typename T>
__device__ __forceinline__ T zero_of();
template <>
__device__ __forceinline__ int zero_of<int>() {
  return 0;
}
template <>
__device__ __forceinline__ I4 zero_of<I4>() {
  return I4{0, 0, 0, 0};
}

template <typename T>
__device__ __forceinline__ T shfl_up_t(T v, int d);
template <>
__device__ __forceinline__ int shfl_up_t<int>(int v, int d) {
  return __shfl_up_sync(0xffffffffu, v, d);
}
template <>
__device__ __forceinline__ I4 shfl_up_t<I4>(I4 v, int d) {
  return I4{__shfl_up_sync(0xffffffffu, v.x, d), __shfl_up_sync(0xffffffffu, v.y, d),
            __shfl_up_sync(0xffffffffu, v.z, d), __shfl_up_sync(0xffffffffu, v.w, d)};
}

constexpr int kScanThreads = 512;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

// Exclusive block-wide scan of one value per thread; returns the block total.
template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T& total, T* sm /*[32]*/) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T inc = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    T o = shfl_up_t(inc, d);
    if (lane >= d) inc = inc + o;
  }
  if (lane == 31) sm[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    T s = lane < nw ? sm[lane] : zero_of<T>();
    T si = s;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      T o = shfl_up_t(si, d);
      if (lane >= d) si = si + o;
    }
    if (lane < nw) sm[lane] = si;  // inclusive warp prefix
  }
  __syncthreads();
  total = sm[(blockDim.x >> 5) - 1];
  T warp_off = warp > 0 ? sm[warp - 1] : zero_of<T>();
  T excl = shfl_up_t(inc, 1);
  if (lane == 0) excl = zero_of<T>();
  T res = warp_off + excl;
  __syncthreads();
  return res;
}

// Loader for the K4 row scan: (count, items, partial rows, 0) per row, where
// items = max(1, ceil(count/chunk)) for real rows and 0 for the sentinel row.
struct RowScanLoad {
  const int32_t* counts;
  int64_t K;
  int chunk;
  __device__ __forceinline__ I4 operator()(int64_t i) const {
    const int c = counts[i];
    if (i >= K) return I4{c, 0, 0, 0};
    const int items = c == 0 ? 1 : (c + chunk - 1) / chunk;
    return I4{c, items, items > 1 ? items : 0, 0};
  }
};
struct IntLoad {
  const int* p;
  __device__ __forceinline__ int operator()(int64_t i) const { return p[i]; }
};

template <typename T, typename Load>
__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(Load ld, int64_t n, T* block_sums) {
  __shared__ T sm[32];
  const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
  T s = zero_of<T>();
#pragma unroll
  for (int j = 0; j < kScanItems; ++j)
    if (base + j < n) s = s + ld(base + j);
  T total;
  block_exclusive_scan<T>(s, total, sm);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

// In-place exclusive scan of the block sums (one block, any count).
template <typename T>
__global__ void __launch_bounds__(kScanThreads) scan_sums_kernel(T* sums, int64_t nb) {
  __shared__ T sm[32];
  T carry = zero_of<T>();
  for (int64_t b0 = 0; b0 < nb; b0 += kScanThreads) {
    const int64_t i = b0 + threadIdx.x;
    T v = i < nb ? sums[i] : zero_of<T>();
    T total;
    T ex = block_exclusive_scan<T>(v, total, sm);
    if (i < nb) sums[i] = carry + ex;
    carry = carry + total;
  }
  if (threadIdx.x == 0) sums[nb] = carry;
}

// out[i] = exclusive prefix of ld(i); out[n] = total.  out may alias the
// loader's source.
template <typename T, typename Load>
__global__ void __launch_bounds__(kScanThreads) scan_down_kernel(Load ld, int64_t n, const T* block_sums,
                                                                 T* out) {
  __shared__ T sm[32];
  const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
  T v[kScanItems];
  T s = zero_of<T>();
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) {
    v[j] = (base + j < n) ? ld(base + j) : zero_of<T>();
    s = s + v[j];
  }
  T total;
  T ex = block_exclusive_scan<T>(s, total, sm);
  T run = block_sums[blockIdx.x] + ex;
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) {
    if (base + j < n) out[base + j] = run;
    run = run + v[j];
  }
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) out[n] = block_sums[gridDim.x];
}

inline int64_t scan_blocks(int64_t n) { return (n + kScanTile - 1) / kScanTile; }

// Enqueue an exclusive scan of n elements; block_sums needs scan_blocks(n)+1.
template <typename T, typename Load>
void scan_exclusive(Load ld, int64_t n, T* out, T* block_sums, cudaStream_t st) {
  const int64_t nb = scan_blocks(n);
  scan_reduce_kernel<T, Load><<<(unsigned)nb, kScanThreads, 0, st>>>(ld, n, block_sums);
  scan_sums_kernel<T><<<1, kScanThreads, 0, st>>>(block_sums, nb);
  scan_down_kernel<T, Load><<<(unsigned)nb, kScanThreads, 0, st>>>(ld, n, block_sums, out);
}

// ---------------------------------------------------------------------------
// Stable LSD radix sort, RB-bit digits (8, or 9 or 10 where that saves a
// pass: the row keys of a 2^18-row table, its sentinel row included, have
// 19 bits and sort in two 10-bit passes instead of three 8-bit ones).
// A tile of kSortTile items is ranked by one block: warp w owns items
// [w*32*kSortIpt, (w+1)*32*kSortIpt) in rounds of 32, so (warp, round, lane)
// order is item order, and equal digits keep their order through
// __match_any_sync ranks.
// ---------------------------------------------------------------------------
#ifndef PKM_SORT_THREADS
#define PKM_SORT_THREADS 256
#endif
#ifndef PKM_SORT_IPT
#define PKM_SORT_IPT 8  // items per thread: 2048-item tiles (measured 50 us faster per c2 backward than 4096)
#endif
constexpr int kSortThreads = PKM_SORT_THREADS;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortIpt = PKM_SORT_IPT;
constexpr int kSortTile = kSortThreads * kSortIpt;
constexpr int kRadix = 256;     // 8-bit digits
constexpr int kRadixMax = 1024;  // the widest digit (10 bits)

template <int RB = 8>
static __global__ void __launch_bounds__(kSortThreads) radix_upsweep_kernel(const uint32_t* keys, int64_t n, int shift,
                                                                     int* hist, int64_t tiles) {
  constexpr int kRadix = 1 << RB;
  __shared__ int cnt[kRadix];
  for (int i = threadIdx.x; i < kRadix; i += kSortThreads) cnt[i] = 0;
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * kSortTile;
  for (int j = threadIdx.x; j < kSortTile; j += kSortThreads) {
    const int64_t i = base + j;
    if (i < n) atomicAdd(&cnt[(keys[i] >> shift) & (kRadix - 1)], 1);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < kRadix; d += kSortThreads) hist[(int64_t)d * tiles + blockIdx.x] = cnt[d];
}

// vals_in == nullptr: the values are the item positions (first pass).
// keys_out == nullptr: keys are not written (last pass).
// w != nullptr: also writes w_out[pos] = float(w[value]) (last pass).
template <int RB = 8>
static __global__ void __launch_bounds__(kSortThreads) radix_downsweep_kernel(
    const uint32_t* keys_in, const int32_t* vals_in, int64_t n, int shift, const int* hist_scan,
    int64_t tiles, uint32_t* keys_out, int32_t* vals_out, const void* w, int w_dtype, float* w_out) {
  constexpr int kRadix = 1 << RB;
  __shared__ int wcnt[kSortWarps][kRadix];
  __shared__ int tbase[kRadix];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kSortWarps * kRadix; i += kSortThreads) (&wcnt[0][0])[i] = 0;
  for (int d = threadIdx.x; d < kRadix; d += kSortThreads) tbase[d] = hist_scan[(int64_t)d * tiles + blockIdx.x];
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * kSortTile + (int64_t)warp * 32 * kSortIpt;
  const unsigned lt = (1u << lane) - 1u;
  uint32_t key[kSortIpt];
  int32_t rank[kSortIpt];
#pragma unroll
  for (int r = 0; r < kSortIpt; ++r) {
    const int64_t i = base + r * 32 + lane;
    const bool valid = i < n;
    key[r] = valid ? keys_in[i] : 0u;
    const int d = valid ? (int)((key[r] >> shift) & (kRadix - 1)) : kRadix;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    int before = 0;
    if (valid) before = wcnt[warp][d];
    rank[r] = before + __popc(peers & lt);
    __syncwarp();
    if (valid && lane == __ffs(peers) - 1) wcnt[warp][d] = before + __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  for (int d = threadIdx.x; d < kRadix; d += kSortThreads) {
    int run = 0;
#pragma unroll
    for (int q = 0; q < kSortWarps; ++q) {
      const int c = wcnt[q][d];
      wcnt[q][d] = run;
      run += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kSortIpt; ++r) {
    const int64_t i = base + r * 32 + lane;
    if (i < n) {
      const int d = (int)((key[r] >> shift) & (kRadix - 1));
      const int64_t pos = (int64_t)tbase[d] + wcnt[warp][d] + rank[r];
      const int32_t val = vals_in ? vals_in[i] : (int32_t)i;
      if (keys_out) keys_out[pos] = key[r];
      vals_out[pos] = val;
      if (w_out) w_out[pos] = w ? ld_f(w, w_dtype, val) : 1.0f;
    }
  }
}

inline int64_t sort_tiles(int64_t n) { return (n + kSortTile - 1) / kSortTile; }

// Digit width and pass count for keys of `bits` bits: the fewest passes of
// at most 10-bit digits, each as narrow as that allows.
inline void sort_plan(int bits, int& rb, int& passes) {
  passes = (bits + 9) / 10;
  rb = (bits + passes - 1) / passes;
  if (rb < 8) rb = 8;
}

}  // namespace pkm
