// Routing of embedding-bag occurrences for a value table split by rows over
// the ranks of a group (the row-sharded bag): the pack before the first
// all-to-all, the segment lists on both sides of it, and the combine of the
// partial sums that come back.  Around the collective's all-to-all these
// replace a host sequence of sort / bincount / unique / index_add with a few
// stream-ordered kernels.
//
// Reference: the bag reads table rows by global index
// (pkm/xformer_embeddingbag.py:97-138) and scatters the table gradient by
// row (:331-386).  With the table split by rows, each occurrence is served by
// the rank that owns its row; these kernels move the occurrences there and
// put the results back together in a fixed order.
//
// pack      owner = index / shard_rows.  A stable partition of the n =
//           bags * L occurrences by owner (one pass of the LSD radix sort
//           with the owner as the digit), so each owner's part keeps
//           occurrence order and hence bag order; per packed entry its local
//           row, fp32 weight and bag; send_counts[o] = entries for owner o.
//           Indices outside [0, world * shard_rows) set PKM_DEVERR_INDEX, are
//           left out of send_counts and sort after the last owner.
// segments  Over entries grouped by counts (owner groups on the sending
//           side, source-rank groups on the receiving side) with bags
//           ascending inside a group: one segment per run of equal bag
//           inside a group.  seg_of[e], seg_start[s] (seg_start[n_seg] = n),
//           seg_bag[s], seg_counts[g].
// combine   out[b] = the partial rows of bag b's segments summed in group
//           order (fp32 accumulation from zero, rounded once to the output
//           dtype): the order the host framework's index_add per owner gives.
#include <algorithm>

#include "common.cuh"
#include "sort.cuh"

namespace pkm {

namespace {

constexpr int kRouteThreads = 256;
constexpr int kRouteMaxGroups = kRadix - 1;  // owners fit one digit, with a discard bucket after them

size_t r256(size_t b) { return (b + 255) & ~size_t(255); }

unsigned route_blocks(int64_t n) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + kRouteThreads - 1) / kRouteThreads,
                                                          (int64_t)num_sms() * 8));
}

// Group prefix sums in shared memory: pre[g] = first entry of group g,
// pre[groups] = total.  One thread computes them (groups <= 255).
__device__ __forceinline__ void load_prefix(const int64_t* counts, int groups, int64_t* pre) {
  if (threadIdx.x == 0) {
    int64_t run = 0;
    pre[0] = 0;
    for (int g = 0; g < groups; ++g) {
      run += counts[g];
      pre[g + 1] = run;
    }
  }
  __syncthreads();
}

// Group of entry i: the largest g with pre[g] <= i (empty groups skipped);
// entries at or past the total belong to no group (returns groups).
__device__ __forceinline__ int group_of(const int64_t* pre, int groups, int64_t i) {
  if (i >= pre[groups]) return groups;
  int lo = 0, hi = groups;  // pre[lo] <= i < pre[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (pre[mid] <= i) lo = mid;
    else hi = mid;
  }
  return lo;
}

__global__ void route_keys_kernel(const int64_t* __restrict__ idx, int64_t n, int64_t shard_rows, int world,
                                  uint32_t* __restrict__ keys, uint32_t* err) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = idx[i];
    const int64_t o = k >= 0 ? k / shard_rows : -1;
    const bool ok = k >= 0 && o < world;
    if (!ok) raise_err(err, PKM_DEVERR_INDEX);
    keys[i] = ok ? (uint32_t)o : (uint32_t)world;
  }
}

__global__ void route_pack_kernel(const int64_t* __restrict__ idx, const int32_t* __restrict__ order, int64_t n,
                                  int64_t shard_rows, int64_t bag_size, int world, int32_t* __restrict__ local_row,
                                  int32_t* __restrict__ bag) {
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += (int64_t)gridDim.x * blockDim.x) {
    const int32_t i = order[p];
    const int64_t k = idx[i];
    const int64_t o = k >= 0 ? k / shard_rows : -1;
    const bool ok = k >= 0 && o < world;
    local_row[p] = ok ? (int32_t)(k - o * shard_rows) : 0;
    bag[p] = (int32_t)(i / bag_size);
  }
}

// send_counts[d] = items with digit d, from the digit-major scanned histogram
__global__ void route_counts_kernel(const int* __restrict__ hist_scan, int64_t tiles, int world,
                                    int64_t* __restrict__ send_counts) {
  for (int d = threadIdx.x; d < world; d += blockDim.x)
    send_counts[d] = (int64_t)hist_scan[(int64_t)(d + 1) * tiles] - hist_scan[(int64_t)d * tiles];
}

__global__ void __launch_bounds__(kRouteThreads) route_flags_kernel(const int32_t* __restrict__ bag, int64_t n,
                                                                   const int64_t* __restrict__ group_counts,
                                                                   int groups, int* __restrict__ flags) {
  __shared__ int64_t pre[kRouteMaxGroups + 1];
  load_prefix(group_counts, groups, pre);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int start = 1;
    if (i > 0) start = bag[i] != bag[i - 1] || group_of(pre, groups, i) != group_of(pre, groups, i - 1);
    flags[i] = start;
  }
}

// ex = exclusive scan of the start flags (ex[n] = segment count)
__global__ void __launch_bounds__(kRouteThreads) route_scatter_kernel(
    const int32_t* __restrict__ bag, int64_t n, const int* __restrict__ ex, const int64_t* __restrict__ group_counts,
    int groups, int32_t* __restrict__ seg_of, int64_t* __restrict__ seg_start, int32_t* __restrict__ seg_bag,
    unsigned long long* __restrict__ seg_counts) {
  __shared__ int64_t pre[kRouteMaxGroups + 1];
  __shared__ int cnt[kRouteMaxGroups + 1];
  for (int g = threadIdx.x; g <= kRouteMaxGroups; g += blockDim.x) cnt[g] = 0;
  load_prefix(group_counts, groups, pre);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int after = ex[i + 1];
    const int s = after - 1;
    seg_of[i] = s;
    if (after != ex[i]) {
      seg_start[s] = i;
      seg_bag[s] = bag[i];
      const int g = group_of(pre, groups, i);
      if (g < groups) atomicAdd(&cnt[g], 1);
    }
    if (i == n - 1) seg_start[after] = n;
  }
  __syncthreads();
  for (int g = threadIdx.x; g < groups; g += blockDim.x)
    if (cnt[g]) atomicAdd(&seg_counts[g], (unsigned long long)cnt[g]);
}

__global__ void __launch_bounds__(kRouteThreads) route_map_kernel(const int32_t* __restrict__ seg_bag, int64_t n_seg,
                                                                 const int64_t* __restrict__ seg_counts, int groups,
                                                                 int64_t n_bags, int32_t* __restrict__ map,
                                                                 uint32_t* err) {
  __shared__ int64_t pre[kRouteMaxGroups + 1];
  load_prefix(seg_counts, groups, pre);
  for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < n_seg;
       s += (int64_t)gridDim.x * blockDim.x) {
    const int g = group_of(pre, groups, s);
    const int32_t b = seg_bag[s];
    if (g < groups && b >= 0 && b < n_bags) map[(int64_t)g * n_bags + b] = (int32_t)s;
    else raise_err(err, PKM_DEVERR_INDEX);
  }
}

// one warp per bag; lanes over the columns; groups in order
__global__ void __launch_bounds__(kRouteThreads) route_combine_kernel(const void* __restrict__ partial, int dtype,
                                                                     int64_t dim, const int32_t* __restrict__ map,
                                                                     int groups, int64_t n_bags, void* __restrict__ out,
                                                                     int out_dtype) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_bags; b += warps) {
    for (int64_t c = lane; c < dim; c += 32) {
      float acc = 0.f;
      for (int g = 0; g < groups; ++g) {
        const int32_t s = map[(int64_t)g * n_bags + b];
        if (s >= 0) acc += ld_f(partial, dtype, (int64_t)s * dim + c);
      }
      st_f(out, out_dtype, b * dim + c, acc);
    }
  }
}

size_t pack_bytes(int64_t n) {
  const int64_t tiles = std::max<int64_t>(1, sort_tiles(n));
  const int64_t hn = (int64_t)kRadix * tiles;
  return r256(sizeof(uint32_t) * (size_t)std::max<int64_t>(n, 1)) + r256(sizeof(int) * (size_t)(hn + 1)) +
         r256(sizeof(int) * (size_t)(scan_blocks(hn) + 1));
}

size_t segments_bytes(int64_t n) {
  return r256(sizeof(int) * (size_t)(n + 1)) + r256(sizeof(int) * (size_t)(scan_blocks(std::max<int64_t>(n, 1)) + 1));
}

}  // namespace

}  // namespace pkm

using namespace pkm;

extern "C" int pkm_route_pack_workspace(int64_t n, size_t* bytes) {
  if (!bytes) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  if (n < 0 || n >= (int64_t)INT32_MAX) return fail(PKM_ERR_INVALID_ARG, "occurrence count must be in [0, 2^31 - 1)");
  *bytes = pack_bytes(n);
  return PKM_OK;
}

extern "C" int pkm_route_pack(const int64_t* indices, const void* psw, int psw_dtype, int64_t n_bags,
                              int64_t bag_size, int64_t shard_rows, int world, int64_t* send_counts, int32_t* order,
                              int32_t* local_row, float* weight, int32_t* bag, void* workspace,
                              size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  if (n_bags < 0 || bag_size < 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  const int64_t n = n_bags * bag_size;
  size_t need = 0;
  int rc = pkm_route_pack_workspace(n, &need);
  if (rc) return rc;
  if (world < 1 || world > kRouteMaxGroups) return fail(PKM_ERR_INVALID_ARG, "world must be in [1, 255]");
  if (shard_rows < 1 || shard_rows > (int64_t)INT32_MAX) return fail(PKM_ERR_INVALID_ARG, "shard_rows must be in [1, 2^31)");
  if (psw && !valid_dtype(psw_dtype)) return fail(PKM_ERR_UNSUPPORTED, "bad weight dtype");
  if (!send_counts) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    cudaMemsetAsync(send_counts, 0, sizeof(int64_t) * (size_t)world, st);
    return check_cuda("pkm_route_pack");
  }
  if (!indices || !order || !local_row || !weight || !bag || !workspace)
    return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  if (workspace_bytes < need) return fail(PKM_ERR_INVALID_ARG, "workspace too small");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(PKM_ERR_INVALID_ARG, "workspace must be 256-byte aligned");
  const int64_t tiles = sort_tiles(n);
  const int64_t hn = (int64_t)kRadix * tiles;
  char* w = static_cast<char*>(workspace);
  uint32_t* keys = reinterpret_cast<uint32_t*>(w);
  w += r256(sizeof(uint32_t) * (size_t)n);
  int* hist = reinterpret_cast<int*>(w);
  w += r256(sizeof(int) * (size_t)(hn + 1));
  int* sums = reinterpret_cast<int*>(w);
  route_keys_kernel<<<route_blocks(n), kRouteThreads, 0, st>>>(indices, n, shard_rows, world, keys, dev_err);
  radix_upsweep_kernel<<<(unsigned)tiles, kSortThreads, 0, st>>>(keys, n, 0, hist, tiles);
  scan_exclusive<int>(IntLoad{hist}, hn, hist, sums, st);
  radix_downsweep_kernel<<<(unsigned)tiles, kSortThreads, 0, st>>>(keys, nullptr, n, 0, hist, tiles, nullptr, order,
                                                                    psw, psw_dtype, weight);
  route_pack_kernel<<<route_blocks(n), kRouteThreads, 0, st>>>(indices, order, n, shard_rows, bag_size, world,
                                                               local_row, bag);
  route_counts_kernel<<<1, 256, 0, st>>>(hist, tiles, world, send_counts);
  return check_cuda("pkm_route_pack");
}

extern "C" int pkm_route_segments_workspace(int64_t n, size_t* bytes) {
  if (!bytes) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  if (n < 0 || n >= (int64_t)INT32_MAX) return fail(PKM_ERR_INVALID_ARG, "entry count must be in [0, 2^31 - 1)");
  *bytes = segments_bytes(n);
  return PKM_OK;
}

extern "C" int pkm_route_segments(const int32_t* bag, int64_t n, const int64_t* group_counts, int groups,
                                  int32_t* seg_of, int64_t* seg_start, int32_t* seg_bag, int64_t* seg_counts,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  size_t need = 0;
  int rc = pkm_route_segments_workspace(n, &need);
  if (rc) return rc;
  if (groups < 1 || groups > kRouteMaxGroups) return fail(PKM_ERR_INVALID_ARG, "groups must be in [1, 255]");
  if (!group_counts || !seg_start || !seg_counts) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaMemsetAsync(seg_counts, 0, sizeof(int64_t) * (size_t)groups, st);
  if (n == 0) {
    cudaMemsetAsync(seg_start, 0, sizeof(int64_t), st);
    return check_cuda("pkm_route_segments");
  }
  if (!bag || !seg_of || !seg_bag || !workspace) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  if (workspace_bytes < need) return fail(PKM_ERR_INVALID_ARG, "workspace too small");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(PKM_ERR_INVALID_ARG, "workspace must be 256-byte aligned");
  int* flags = static_cast<int*>(workspace);
  int* sums = reinterpret_cast<int*>(static_cast<char*>(workspace) + r256(sizeof(int) * (size_t)(n + 1)));
  route_flags_kernel<<<route_blocks(n), kRouteThreads, 0, st>>>(bag, n, group_counts, groups, flags);
  scan_exclusive<int>(IntLoad{flags}, n, flags, sums, st);
  route_scatter_kernel<<<route_blocks(n), kRouteThreads, 0, st>>>(bag, n, flags, group_counts, groups, seg_of,
                                                                  seg_start, seg_bag,
                                                                  reinterpret_cast<unsigned long long*>(seg_counts));
  return check_cuda("pkm_route_segments");
}

extern "C" int pkm_route_combine_workspace(int groups, int64_t n_bags, size_t* bytes) {
  if (!bytes) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  if (groups < 1 || groups > kRouteMaxGroups || n_bags < 0 || n_bags >= (int64_t)INT32_MAX)
    return fail(PKM_ERR_INVALID_ARG, "bad size");
  *bytes = r256(sizeof(int32_t) * (size_t)groups * (size_t)std::max<int64_t>(n_bags, 1));
  return PKM_OK;
}

extern "C" int pkm_route_combine(const void* partial, int dtype, int64_t n_seg, int64_t dim, const int32_t* seg_bag,
                                 const int64_t* seg_counts, int groups, int64_t n_bags, void* out, int out_dtype,
                                 void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  size_t need = 0;
  int rc = pkm_route_combine_workspace(groups, n_bags, &need);
  if (rc) return rc;
  if (n_seg < 0 || n_seg >= (int64_t)INT32_MAX || dim < 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  if (!valid_dtype(dtype) || !valid_dtype(out_dtype)) return fail(PKM_ERR_UNSUPPORTED, "bad dtype");
  if (n_bags == 0 || dim == 0) return PKM_OK;
  if (!out || !seg_counts || !workspace || (n_seg > 0 && (!partial || !seg_bag)))
    return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  if (workspace_bytes < need) return fail(PKM_ERR_INVALID_ARG, "workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* map = static_cast<int32_t*>(workspace);
  cudaMemsetAsync(map, 0xff, sizeof(int32_t) * (size_t)groups * (size_t)n_bags, st);  // -1: no segment
  if (n_seg > 0)
    route_map_kernel<<<route_blocks(n_seg), kRouteThreads, 0, st>>>(seg_bag, n_seg, seg_counts, groups, n_bags, map,
                                                                    dev_err);
  const int64_t warps_per_block = kRouteThreads / 32;
  const unsigned blocks = (unsigned)std::max<int64_t>(
      1, std::min<int64_t>((n_bags + warps_per_block - 1) / warps_per_block, (int64_t)num_sms() * 8));
  route_combine_kernel<<<blocks, kRouteThreads, 0, st>>>(partial, dtype, dim, map, groups, n_bags, out, out_dtype);
  return check_cuda("pkm_route_combine");
}
