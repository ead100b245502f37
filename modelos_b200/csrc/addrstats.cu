// Addressing statistics of one batch of memory-slot indices, computed on the
// device: the per-slot histogram and three reductions over it, with no host
// round trip until the caller reads the result.
//
// Reference: Qwen3PKMDecoderLayer.compute_addr_stats
// (modeling_qwen3pkm.py:447-471), which runs
//   counts   = bincount(idcs, minlength=K)
//   collision_ratio = sum(counts[counts > 1]) / (numel + 1e-6)
//   coverage_ratio  = count(counts > 0) / K
//   kld = KL(Categorical(counts / sum(counts)) || Categorical(uniform over K))
// with three .item() synchronisations.  torch.distributions evaluates the KL
// as sum_i p_i * (log c(p_i) - log c(q_i)), c(x) = clamp(x, eps, 1 - eps)
// with eps the fp32 machine epsilon, and drops the terms with p_i = 0; the
// reduction here evaluates that expression in fp64.
//
// Kernels: slot_count_kernel (int32 atomics into the caller's bins), then
// addr_reduce_kernel (grid-stride over the bins, per-block partials reduced
// in a fixed tree order) and addr_finalize_kernel (one warp over the
// partials, fixed order).  The block count depends only on the bin count,
// so results are bit-reproducible on any device.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "count.cuh"

namespace pkm {

namespace {

constexpr int kAddrThreads = 256;
constexpr int64_t kAddrBinsPerBlock = 2048;
constexpr int64_t kAddrMaxBlocks = 1024;

struct AddrPartial {
  unsigned long long collided, covered, total;
  double kl;
};

int64_t addr_blocks(int64_t rows) {
  return std::max<int64_t>(1, std::min<int64_t>((rows + kAddrBinsPerBlock - 1) / kAddrBinsPerBlock, kAddrMaxBlocks));
}

size_t round_up256(size_t b) { return (b + 255) & ~size_t(255); }

__device__ __forceinline__ double clamp_prob(double p) {
  const double eps = 1.1920928955078125e-07;  // 2^-23, the fp32 machine epsilon
  return fmin(fmax(p, eps), 1.0 - eps);
}

__device__ __forceinline__ void warp_sum(AddrPartial& a) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    a.collided += __shfl_xor_sync(0xffffffffu, a.collided, o);
    a.covered += __shfl_xor_sync(0xffffffffu, a.covered, o);
    a.total += __shfl_xor_sync(0xffffffffu, a.total, o);
    a.kl += __shfl_xor_sync(0xffffffffu, a.kl, o);
  }
}

__global__ void __launch_bounds__(kAddrThreads) addr_reduce_kernel(const int32_t* __restrict__ counts, int64_t rows,
                                                                  double inv_total, double log_q,
                                                                  AddrPartial* __restrict__ partial) {
  AddrPartial a{0ull, 0ull, 0ull, 0.0};
  for (int64_t k = (int64_t)blockIdx.x * kAddrThreads + threadIdx.x; k < rows;
       k += (int64_t)gridDim.x * kAddrThreads) {
    const int c = counts[k];
    if (c > 0) {
      const double p = (double)c * inv_total;
      a.covered += 1ull;
      a.total += (unsigned long long)c;
      if (c > 1) a.collided += (unsigned long long)c;
      a.kl += p * (log(clamp_prob(p)) - log_q);
    }
  }
  warp_sum(a);
  __shared__ AddrPartial warps[kAddrThreads / 32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warps[w] = a;
  __syncthreads();
  if (w == 0) {
    AddrPartial b = lane < kAddrThreads / 32 ? warps[lane] : AddrPartial{0ull, 0ull, 0ull, 0.0};
    warp_sum(b);
    if (lane == 0) partial[blockIdx.x] = b;
  }
}

__global__ void addr_finalize_kernel(const AddrPartial* __restrict__ partial, int nb, double* __restrict__ out) {
  AddrPartial a{0ull, 0ull, 0ull, 0.0};
  for (int i = threadIdx.x; i < nb; i += 32) {
    const AddrPartial p = partial[i];
    a.collided += p.collided;
    a.covered += p.covered;
    a.total += p.total;
    a.kl += p.kl;
  }
  warp_sum(a);
  if (threadIdx.x == 0) {
    out[0] = (double)a.collided;
    out[1] = (double)a.covered;
    out[2] = a.kl;
    out[3] = (double)a.total;
  }
}

}  // namespace

}  // namespace pkm

using namespace pkm;

extern "C" int pkm_addr_stats_workspace(int64_t rows, size_t* bytes) {
  if (!bytes) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  if (rows <= 0 || rows > (int64_t)INT32_MAX) return fail(PKM_ERR_INVALID_ARG, "rows must be in [1, 2^31)");
  *bytes = round_up256(sizeof(int32_t) * (size_t)rows) + sizeof(AddrPartial) * (size_t)addr_blocks(rows);
  return PKM_OK;
}

extern "C" int pkm_addr_stats(const int64_t* indices, int64_t n_indices, int64_t rows, double* out,
                              void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  size_t need = 0;
  int rc = pkm_addr_stats_workspace(rows, &need);
  if (rc) return rc;
  if (n_indices <= 0) return fail(PKM_ERR_INVALID_ARG, "no indices (the distribution is undefined)");
  if (!indices || !out || !workspace) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  if (workspace_bytes < need) return fail(PKM_ERR_INVALID_ARG, "workspace too small");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return fail(PKM_ERR_INVALID_ARG, "workspace must be 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* counts = static_cast<int32_t*>(workspace);
  AddrPartial* partial =
      reinterpret_cast<AddrPartial*>(static_cast<char*>(workspace) + round_up256(sizeof(int32_t) * (size_t)rows));
  const int64_t nb = addr_blocks(rows);
  cudaMemsetAsync(counts, 0, sizeof(int32_t) * (size_t)rows, st);
  const unsigned cblocks =
      (unsigned)std::max<int64_t>(1, std::min<int64_t>((n_indices + 255) / 256, (int64_t)num_sms() * 16));
  slot_count_kernel<<<cblocks, 256, 0, st>>>(indices, n_indices, rows, counts, dev_err);
  // the reference's uniform distribution: q = 1/K, its log clamped like p's
  const double eps = 1.1920928955078125e-07;
  const double log_q = std::log(std::min(std::max(1.0 / (double)rows, eps), 1.0 - eps));
  addr_reduce_kernel<<<(unsigned)nb, kAddrThreads, 0, st>>>(counts, rows, 1.0 / (double)n_indices, log_q, partial);
  addr_finalize_kernel<<<1, 32, 0, st>>>(partial, (int)nb, out);
  return check_cuda("pkm_addr_stats");
}
