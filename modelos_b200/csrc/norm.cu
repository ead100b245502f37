// Batch normalisation of the query projection (rows = tokens, columns =
// channels), training and evaluation forward and the training backward.
//
// Replaces `nn.BatchNorm1d(heads * k_dim, eps=1e-6, momentum=0.1)` of the
// query network (pkm/memory.py:308-309), i.e. ATen's native_batch_norm and
// native_batch_norm_backward on a [N, C] row-major activation.
//
// Every pass streams the activation with 16-byte vectors: a thread owns 8
// consecutive channels, a warp 256, and the rows of a column tile are split
// over the blocks of the grid's second dimension.  Column statistics are
// reduced per block in a fixed order into fp32 partials, and a small
// finalise kernel sums the partials in row-block order in fp64, so results
// are deterministic.  The forward statistics use the first row as a shift
// (sums of x - x[0] and its square), which keeps the one-pass variance
// accurate when the mean is large against the spread.
#include <algorithm>

#include "rows.cuh"

namespace pkm {

// Column partial sums of two per-element quantities over a row block:
//   mode 0 (forward statistics):  a = x - x[0], b = a * a
//   mode 1 (backward reduction):  a = dy,       b = dy * (x - mean)
// written to part[rb][c] as float2 {a, b}.
template <typename T, int MODE>
__global__ void __launch_bounds__(kNormThreads) norm_reduce_kernel(const T* __restrict__ x, const T* __restrict__ dy,
                                                                  const float* __restrict__ mean, int64_t n,
                                                                  int64_t c, float2* __restrict__ part) {
  __shared__ float2 red[kNormThreads / 32][32 * kNormChan];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c0 = ((int64_t)blockIdx.x * 32 + lane) * kNormChan;
  const bool live = c0 < c;
  int64_t r0, r1;
  row_range(n, blockIdx.y, gridDim.y, r0, r1);
  float sa[kNormChan], sb[kNormChan], ref[kNormChan];
#pragma unroll
  for (int i = 0; i < kNormChan; ++i) sa[i] = sb[i] = ref[i] = 0.f;
  if (live) {
    if (MODE == 0) {
      RowIO<T>::load(x + c0, ref);  // shift: row 0
    } else {
#pragma unroll
      for (int i = 0; i < kNormChan; ++i) ref[i] = mean[c0 + i];
    }
  #pragma unroll 4
  for (int64_t r = r0 + warp; r < r1; r += kNormThreads / 32) {
      float v[kNormChan];
      RowIO<T>::load(x + r * c + c0, v);
      if (MODE == 0) {
#pragma unroll
        for (int i = 0; i < kNormChan; ++i) {
          const float d = v[i] - ref[i];
          sa[i] += d;
          sb[i] = fmaf(d, d, sb[i]);
        }
      } else {
        float g[kNormChan];
        RowIO<T>::load(dy + r * c + c0, g);
#pragma unroll
        for (int i = 0; i < kNormChan; ++i) {
          sa[i] += g[i];
          sb[i] = fmaf(g[i], v[i] - ref[i], sb[i]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kNormChan; ++i) red[warp][lane * kNormChan + i] = make_float2(sa[i], sb[i]);
  __syncthreads();
  // warp w sums the 8 warps' partials of channels w*32 .. w*32+31 of the tile
  const int t = warp * 32 + lane;
  const int64_t ch = (int64_t)blockIdx.x * 32 * kNormChan + t;
  if (ch < c) {
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) {
      a += red[w][t].x;
      b += red[w][t].y;
    }
    part[(int64_t)blockIdx.y * c + ch] = make_float2(a, b);
  }
}

// Forward finalise: mean, 1/sqrt(var + eps) (biased variance), the running
// statistics update (unbiased variance), per channel.
__global__ void __launch_bounds__(256) norm_fwd_finalize_kernel(const float2* __restrict__ part, int nb, const void* x,
                                                                int x_dtype, int64_t n, int64_t c, double eps,
                                                                double momentum, void* running_mean,
                                                                void* running_var, int r_dtype,
                                                                float* __restrict__ save_mean,
                                                                float* __restrict__ save_rstd) {
  const Sum2 r = colsum_fixed(nullptr, part, nb, c);
  const int64_t ch = (int64_t)blockIdx.x * 32 + (threadIdx.x & 31);
  if (threadIdx.x >= 32 || ch >= c) return;
  const double sa = r.a, sb = r.b;
  const double shift = ld_f(x, x_dtype, ch);
  const double dm = sa / (double)n;
  const double var = std::max(0.0, sb / (double)n - dm * dm);
  const double mean = shift + dm;
  save_mean[ch] = (float)mean;
  save_rstd[ch] = (float)(1.0 / sqrt(var + eps));
  if (running_mean) {
    const double rm = ld_f(running_mean, r_dtype, ch);
    st_f(running_mean, r_dtype, ch, (float)((1.0 - momentum) * rm + momentum * mean));
  }
  if (running_var) {
    const double unb = n > 1 ? var * (double)n / (double)(n - 1) : var;
    const double rv = ld_f(running_var, r_dtype, ch);
    st_f(running_var, r_dtype, ch, (float)((1.0 - momentum) * rv + momentum * unb));
  }
}

// Evaluation: the running statistics as (mean, 1/sqrt(var + eps)).
__global__ void norm_eval_stats_kernel(const void* running_mean, const void* running_var, int r_dtype, int64_t c,
                                       double eps, float* __restrict__ save_mean, float* __restrict__ save_rstd) {
  const int64_t ch = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= c) return;
  save_mean[ch] = ld_f(running_mean, r_dtype, ch);
  save_rstd[ch] = (float)(1.0 / sqrt((double)ld_f(running_var, r_dtype, ch) + eps));
}

// out = (x - mean) * (rstd * w) + b.  Same tiling as the reduction: a
// thread keeps its 8 channels' coefficients in registers over its rows.
template <typename T>
__global__ void __launch_bounds__(kNormThreads) norm_apply_kernel(const T* __restrict__ x, const float* __restrict__ mean,
                                                                 const float* __restrict__ rstd, const void* weight,
                                                                 const void* bias, int p_dtype, int64_t n, int64_t c,
                                                                 T* __restrict__ out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c0 = ((int64_t)blockIdx.x * 32 + lane) * kNormChan;
  if (c0 >= c) return;
  int64_t r0, r1;
  row_range(n, blockIdx.y, gridDim.y, r0, r1);
  float mu[kNormChan], sc[kNormChan], bi[kNormChan];
#pragma unroll
  for (int k = 0; k < kNormChan; ++k) {
    mu[k] = mean[c0 + k];
    sc[k] = rstd[c0 + k] * (weight ? ld_f(weight, p_dtype, c0 + k) : 1.f);
    bi[k] = bias ? ld_f(bias, p_dtype, c0 + k) : 0.f;
  }
  constexpr int64_t kStep = kNormThreads / 32;
  for (int64_t r = r0 + warp; r < r1; r += 4 * kStep) {
    float v[4][kNormChan];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (r + u * kStep < r1) RowIO<T>::load(x + (r + u * kStep) * c + c0, v[u]);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (r + u * kStep < r1) {
#pragma unroll
        for (int k = 0; k < kNormChan; ++k) v[u][k] = fmaf(v[u][k] - mu[k], sc[k], bi[k]);
        RowIO<T>::store(out + (r + u * kStep) * c + c0, v[u]);
      }
    }
  }
}

// Backward finalise: dbias = sum dy, dweight = rstd * sum dy (x - mean), and
// the coefficients of dx = a (dy - m) - b (x - mean):
//   a = w rstd, m = sum dy / n, b = a rstd^2 sum dy (x - mean) / n.
__global__ void __launch_bounds__(256) norm_bwd_finalize_kernel(const float2* __restrict__ part, int nb, int64_t n,
                                                                int64_t c, const float* __restrict__ rstd,
                                                                const void* weight, int p_dtype, void* dweight,
                                                                void* dbias, float4* __restrict__ coef) {
  const Sum2 r = colsum_fixed(nullptr, part, nb, c);
  const int64_t ch = (int64_t)blockIdx.x * 32 + (threadIdx.x & 31);
  if (threadIdx.x >= 32 || ch >= c) return;
  const double sa = r.a, sb = r.b;
  const double rs = rstd[ch];
  const double w = weight ? ld_f(weight, p_dtype, ch) : 1.0;
  if (dbias) st_f(dbias, p_dtype, ch, (float)sa);
  if (dweight) st_f(dweight, p_dtype, ch, (float)(sb * rs));
  const double a = w * rs;
  coef[ch] = make_float4((float)a, (float)(sa / (double)n), (float)(a * rs * rs * sb / (double)n), 0.f);
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads) norm_bwd_apply_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                                     const float* __restrict__ mean,
                                                                     const float4* __restrict__ coef, int64_t n,
                                                                     int64_t c, T* __restrict__ dx) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c0 = ((int64_t)blockIdx.x * 32 + lane) * kNormChan;
  if (c0 >= c) return;
  int64_t r0, r1;
  row_range(n, blockIdx.y, gridDim.y, r0, r1);
  float mu[kNormChan], ka[kNormChan], km[kNormChan], kb[kNormChan];
#pragma unroll
  for (int k = 0; k < kNormChan; ++k) {
    const float4 q = coef[c0 + k];
    mu[k] = mean[c0 + k];
    ka[k] = q.x;
    km[k] = q.y;
    kb[k] = q.z;
  }
#pragma unroll 4
  for (int64_t r = r0 + warp; r < r1; r += kNormThreads / 32) {
    float g[kNormChan], v[kNormChan];
    RowIO<T>::load(dy + r * c + c0, g);
    RowIO<T>::load(x + r * c + c0, v);
#pragma unroll
    for (int k = 0; k < kNormChan; ++k) v[k] = ka[k] * (g[k] - km[k]) - kb[k] * (v[k] - mu[k]);
    RowIO<T>::store(dx + r * c + c0, v);
  }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
static int norm_check(const void* x, int x_dtype, int64_t n, int64_t c) {
  if (x_dtype != PKM_DT_F32 && x_dtype != PKM_DT_BF16) return fail(PKM_ERR_UNSUPPORTED, "x must be f32 or bf16");
  if (n <= 0 || c <= 0) return fail(PKM_ERR_INVALID_ARG, "need n > 0 and c > 0");
  if (c % kNormChan != 0) return fail(PKM_ERR_UNSUPPORTED, "channels must be a multiple of 8");
  if (!aligned16(x)) return fail(PKM_ERR_UNSUPPORTED, "x must be 16-byte aligned");
  return PKM_OK;
}

template <typename T>
static void launch_apply(const void* x, const float* mean, const float* rstd, const void* w, const void* b, int p_dtype,
                         int64_t n, int64_t c, void* out, cudaStream_t st) {
  const dim3 grid((unsigned)((c + 32 * kNormChan - 1) / (32 * kNormChan)), (unsigned)row_blocks(n, c));
  norm_apply_kernel<T><<<grid, kNormThreads, 0, st>>>(static_cast<const T*>(x), mean, rstd, w, b, p_dtype, n, c,
                                                      static_cast<T*>(out));
}

}  // namespace pkm

using namespace pkm;

extern "C" int pkm_batchnorm_workspace(int64_t n, int64_t c, size_t* bytes) {
  if (!bytes || n <= 0 || c <= 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  const int nb = row_blocks(n, c);
  *bytes = (((size_t)nb * (size_t)c * sizeof(float2) + 255) & ~(size_t)255) + (size_t)c * sizeof(float4);
  return PKM_OK;
}

extern "C" int pkm_batchnorm_fwd(const void* x, int x_dtype, int64_t n, int64_t c, const void* weight,
                                 const void* bias, int p_dtype, void* running_mean, void* running_var, int r_dtype,
                                 int training, double momentum, double eps, void* out, float* save_mean,
                                 float* save_rstd, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = norm_check(x, x_dtype, n, c);
  if (rc) return rc;
  if (!out || !aligned16(out) || !save_mean || !save_rstd)
    return fail(PKM_ERR_INVALID_ARG, "out (16-byte aligned), save_mean and save_rstd are required");
  if ((weight || bias) && !valid_dtype(p_dtype)) return fail(PKM_ERR_INVALID_ARG, "bad parameter dtype");
  if ((running_mean || running_var) && !valid_dtype(r_dtype)) return fail(PKM_ERR_INVALID_ARG, "bad statistics dtype");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!training && (!running_mean || !running_var))
    return fail(PKM_ERR_INVALID_ARG, "evaluation needs the running statistics");
  size_t need = 0;
  pkm_batchnorm_workspace(n, c, &need);
  if (training && (!workspace || workspace_bytes < need)) return fail(PKM_ERR_WORKSPACE, "batchnorm workspace too small");
  const int nb = row_blocks(n, c);
  const unsigned fin_blocks = (unsigned)((c + 255) / 256);
  if (training) {
    float2* part = static_cast<float2*>(workspace);
    const dim3 grid((unsigned)((c + 32 * kNormChan - 1) / (32 * kNormChan)), (unsigned)nb);
    if (x_dtype == PKM_DT_F32)
      norm_reduce_kernel<float, 0><<<grid, kNormThreads, 0, st>>>(static_cast<const float*>(x), nullptr, nullptr, n,
                                                                  c, part);
    else
      norm_reduce_kernel<__nv_bfloat16, 0><<<grid, kNormThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(x), nullptr,
                                                                          nullptr, n, c, part);
    norm_fwd_finalize_kernel<<<(unsigned)((c + 31) / 32), 256, 0, st>>>(part, nb, x, x_dtype, n, c, eps, momentum, running_mean,
                                                         running_var, r_dtype, save_mean, save_rstd);
  } else {
    norm_eval_stats_kernel<<<fin_blocks, 256, 0, st>>>(running_mean, running_var, r_dtype, c, eps, save_mean,
                                                       save_rstd);
  }
  if (x_dtype == PKM_DT_F32)
    launch_apply<float>(x, save_mean, save_rstd, weight, bias, p_dtype, n, c, out, st);
  else
    launch_apply<__nv_bfloat16>(x, save_mean, save_rstd, weight, bias, p_dtype, n, c, out, st);
  return check_cuda("pkm_batchnorm_fwd");
}

extern "C" int pkm_batchnorm_bwd(const void* dy, const void* x, int x_dtype, int64_t n, int64_t c,
                                 const float* save_mean, const float* save_rstd, const void* weight, int p_dtype,
                                 void* dx, void* dweight, void* dbias, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  int rc = norm_check(x, x_dtype, n, c);
  if (rc) return rc;
  if (!dy || !aligned16(dy) || !save_mean || !save_rstd) return fail(PKM_ERR_INVALID_ARG, "NULL or unaligned input");
  if (dx && !aligned16(dx)) return fail(PKM_ERR_INVALID_ARG, "dx must be 16-byte aligned");
  if ((weight || dweight || dbias) && !valid_dtype(p_dtype)) return fail(PKM_ERR_INVALID_ARG, "bad parameter dtype");
  size_t need = 0;
  pkm_batchnorm_workspace(n, c, &need);
  if (!workspace || workspace_bytes < need) return fail(PKM_ERR_WORKSPACE, "batchnorm workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nb = row_blocks(n, c);
  float2* part = static_cast<float2*>(workspace);
  float4* coef = reinterpret_cast<float4*>(static_cast<char*>(workspace) + (((size_t)nb * c * sizeof(float2) + 255) & ~(size_t)255));
  const dim3 grid((unsigned)((c + 32 * kNormChan - 1) / (32 * kNormChan)), (unsigned)nb);
  if (x_dtype == PKM_DT_F32)
    norm_reduce_kernel<float, 1><<<grid, kNormThreads, 0, st>>>(static_cast<const float*>(x),
                                                                static_cast<const float*>(dy), save_mean, n, c, part);
  else
    norm_reduce_kernel<__nv_bfloat16, 1><<<grid, kNormThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(dy), save_mean, n, c, part);
  norm_bwd_finalize_kernel<<<(unsigned)((c + 31) / 32), 256, 0, st>>>(part, nb, n, c, save_rstd, weight, p_dtype,
                                                                        dweight, dbias, coef);
  if (dx) {
    if (x_dtype == PKM_DT_F32)
      norm_bwd_apply_kernel<float><<<grid, kNormThreads, 0, st>>>(
          static_cast<const float*>(dy), static_cast<const float*>(x), save_mean, coef, n, c, static_cast<float*>(dx));
    else
      norm_bwd_apply_kernel<__nv_bfloat16><<<grid, kNormThreads, 0, st>>>(
          static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x), save_mean, coef, n, c,
          static_cast<__nv_bfloat16*>(dx));
  }
  return check_cuda("pkm_batchnorm_bwd");
}
