// Score transform of the fast-weight memory: the normalisation of each
// token's H*knn top-k scores, jointly over all heads (fwpkm/fwpkm.py:105-115,
// called at :179).
//
//   x = scores / temperature
//   softmax: y = exp(x - max x) / sum exp(x - max x)   over the row
//   silu:    y = x * sigmoid(x)
//   relu:    y = max(x, 0)
//
// One warp per row (a row is one token's H*knn scores, 128 at config 4),
// persistent grid; arithmetic in fp32, results rounded to the score dtype as
// the reference's `.type_as(scores)`.  The backward is the exact derivative:
//   softmax: dx = y * (dy - sum(dy * y)),  silu: dx = dy * s * (1 + x (1 - s)),
//   relu: dx = dy * [x > 0];  d scores = dx / temperature.
#include <algorithm>

#include "common.cuh"

namespace pkm {

constexpr int kSmWarps = 8;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}
__device__ __forceinline__ float sigmoidf(float x) { return 1.f / (1.f + expf(-x)); }

// Row elements held per lane (widths up to 32 * kMaxPerLane)
constexpr int kMaxPerLane = 16;

__global__ void __launch_bounds__(kSmWarps * 32) score_transform_fwd_kernel(const void* __restrict__ s, int dt,
                                                                            int64_t rows, int width, float temp,
                                                                            int mode, void* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * kSmWarps;
  for (int64_t r = (int64_t)blockIdx.x * kSmWarps + (threadIdx.x >> 5); r < rows; r += nw) {
    const int64_t base = r * width;
    float x[kMaxPerLane];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < kMaxPerLane; ++k) {
      const int c = lane + 32 * k;
      x[k] = c < width ? __fdiv_rn(ld_f(s, dt, base + c), temp) : -INFINITY;
      mx = fmaxf(mx, x[k]);
    }
    if (mode == 0) {
      mx = warp_max(mx);
      float sum = 0.f;
#pragma unroll
      for (int k = 0; k < kMaxPerLane; ++k) {
        x[k] = (lane + 32 * k) < width ? expf(x[k] - mx) : 0.f;
        sum += x[k];
      }
      sum = warp_sum(sum);
#pragma unroll
      for (int k = 0; k < kMaxPerLane; ++k) {
        const int c = lane + 32 * k;
        if (c < width) st_f(y, dt, base + c, __fdiv_rn(x[k], sum));
      }
    } else {
#pragma unroll
      for (int k = 0; k < kMaxPerLane; ++k) {
        const int c = lane + 32 * k;
        if (c < width) st_f(y, dt, base + c, mode == 1 ? __fdiv_rn(x[k], 1.f + expf(-x[k])) : fmaxf(x[k], 0.f));
      }
    }
  }
}

__global__ void __launch_bounds__(kSmWarps * 32) score_transform_bwd_kernel(
    const void* __restrict__ s, const void* __restrict__ y, const void* __restrict__ dy, int dt, int64_t rows,
    int width, float temp, int mode, void* __restrict__ ds) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * kSmWarps;
  for (int64_t r = (int64_t)blockIdx.x * kSmWarps + (threadIdx.x >> 5); r < rows; r += nw) {
    const int64_t base = r * width;
    if (mode == 0) {
      float yv[kMaxPerLane], g[kMaxPerLane];
      float dot = 0.f;
#pragma unroll
      for (int k = 0; k < kMaxPerLane; ++k) {
        const int c = lane + 32 * k;
        yv[k] = c < width ? ld_f(y, dt, base + c) : 0.f;
        g[k] = c < width ? ld_f(dy, dt, base + c) : 0.f;
        dot += g[k] * yv[k];
      }
      dot = warp_sum(dot);
#pragma unroll
      for (int k = 0; k < kMaxPerLane; ++k) {
        const int c = lane + 32 * k;
        if (c < width) st_f(ds, dt, base + c, __fdiv_rn(yv[k] * (g[k] - dot), temp));
      }
    } else {
#pragma unroll
      for (int k = 0; k < kMaxPerLane; ++k) {
        const int c = lane + 32 * k;
        if (c >= width) continue;
        const float x = __fdiv_rn(ld_f(s, dt, base + c), temp);
        const float g = ld_f(dy, dt, base + c);
        float d;
        if (mode == 1) {
          const float sg = sigmoidf(x);
          d = g * sg * (1.f + x * (1.f - sg));
        } else {
          d = x > 0.f ? g : 0.f;
        }
        st_f(ds, dt, base + c, __fdiv_rn(d, temp));
      }
    }
  }
}

static int transform_checks(const void* a, int dt, int64_t rows, int64_t width, double temp, int mode) {
  if (rows < 0 || width < 0) return fail(PKM_ERR_INVALID_ARG, "negative size");
  if (width > 32 * kMaxPerLane) return fail(PKM_ERR_UNSUPPORTED, "score rows wider than 512");
  if (!valid_dtype(dt)) return fail(PKM_ERR_INVALID_ARG, "bad dtype");
  if (mode < 0 || mode > 2) return fail(PKM_ERR_INVALID_ARG, "mode must be 0 (softmax), 1 (silu) or 2 (relu)");
  if (!(temp > 0.0)) return fail(PKM_ERR_INVALID_ARG, "temperature must be positive");
  if (rows > 0 && width > 0 && !a) return fail(PKM_ERR_INVALID_ARG, "null pointer");
  return PKM_OK;
}

static unsigned transform_grid(int64_t rows) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((rows + kSmWarps - 1) / kSmWarps, (int64_t)num_sms() * 8));
}

}  // namespace pkm

using namespace pkm;

extern "C" int pkm_score_transform_fwd(const void* scores, int dtype, int64_t rows, int64_t width,
                                       double temperature, int mode, void* out, void* stream) {
  int rc = transform_checks(scores, dtype, rows, width, temperature, mode);
  if (rc) return rc;
  if (rows == 0 || width == 0) return PKM_OK;
  if (!out) return fail(PKM_ERR_INVALID_ARG, "null pointer");
  score_transform_fwd_kernel<<<transform_grid(rows), kSmWarps * 32, 0, (cudaStream_t)stream>>>(
      scores, dtype, rows, (int)width, (float)temperature, mode, out);
  return check_cuda("score_transform_fwd_kernel");
}

extern "C" int pkm_score_transform_bwd(const void* scores, const void* out, const void* grad_out, int dtype,
                                       int64_t rows, int64_t width, double temperature, int mode, void* grad_scores,
                                       void* stream) {
  int rc = transform_checks(grad_out, dtype, rows, width, temperature, mode);
  if (rc) return rc;
  if (rows == 0 || width == 0) return PKM_OK;
  if (!grad_scores || (mode == 0 && !out) || (mode != 0 && !scores))
    return fail(PKM_ERR_INVALID_ARG, "null pointer");
  score_transform_bwd_kernel<<<transform_grid(rows), kSmWarps * 32, 0, (cudaStream_t)stream>>>(
      scores, out, grad_out, dtype, rows, (int)width, (float)temperature, mode, grad_scores);
  return check_cuda("score_transform_bwd_kernel");
}
