// Sub-key scores (K1), SIMT path.
//
// scores[r, p, m] = <query[r, p*half : (p+1)*half], keys[(h*2+p)*n + m]>,
// r = token*heads + h, for the dot and idw score types (and the plain
// Euclidean distance the idw score is built from).  Every score is a
// sequential fp32 sum over the half dimension in ascending order; for fp32
// inputs products and sums are rounded separately (no fused multiply-add),
// which is the oracle's definition and makes top-k indices bit-exact.
//
// One block computes a 64 (query rows of one head) x 64 (sub-keys) tile of
// one (head, half), staging 32-wide slices of both operands in shared memory;
// each thread owns a 4 x 4 micro-tile.
#include "common.cuh"

namespace pkm {

bool subkey_scores_tc_eligible(int64_t heads, int64_t k_dim, int64_t n_keys, const void* query, const void* keys,
                               const void* scores);
int subkey_scores_tc(const void* query, const void* keys, int64_t n_tokens, int64_t heads, int64_t k_dim,
                     int64_t n_keys, void* scores, uint32_t* err, cudaStream_t st);

constexpr int kTR = 64, kTM = 64, kKC = 32;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T, int MODE>
__global__ void __launch_bounds__(256) subkey_scores_kernel(const T* __restrict__ q, const T* __restrict__ keys,
                                                            int64_t n_tokens, int heads, int kd, int n,
                                                            T* __restrict__ scores) {
  __shared__ float sq[kKC][kTR + 1];
  __shared__ float sk[kKC][kTM + 1];
  const int half = kd >> 1;
  const int hp = blockIdx.z;  // head*2 + half
  const int h = hp >> 1, p = hp & 1;
  const int64_t t0 = (int64_t)blockIdx.x * kTR;
  const int m0 = blockIdx.y * kTM;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
  float qq[4], kk[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    qq[i] = 0.f;
    kk[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  }
  for (int c0 = 0; c0 < half; c0 += kKC) {
    // stage q rows (tokens t0.., head h, half p) and key rows
    for (int e = threadIdx.x; e < kKC * kTR; e += 256) {
      const int rr = e / kKC, cc = e % kKC;
      const int64_t t = t0 + rr;
      float v = 0.f;
      if (t < n_tokens && c0 + cc < half) v = to_f(q[(t * heads + h) * (int64_t)kd + p * half + c0 + cc]);
      sq[cc][rr] = v;
    }
    for (int e = threadIdx.x; e < kKC * kTM; e += 256) {
      const int rr = e / kKC, cc = e % kKC;
      const int m = m0 + rr;
      float v = 0.f;
      if (m < n && c0 + cc < half) v = to_f(keys[((int64_t)hp * n + m) * half + c0 + cc]);
      sk[cc][rr] = v;
    }
    __syncthreads();
    const int cmax = min(kKC, half - c0);
    for (int c = 0; c < cmax; ++c) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sq[c][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sk[c][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
      if (MODE >= 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) qq[i] = __fadd_rn(qq[i], __fmul_rn(a[i], a[i]));
#pragma unroll
        for (int j = 0; j < 4; ++j) kk[j] = __fadd_rn(kk[j], __fmul_rn(b[j], b[j]));
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t t = t0 + ty * 4 + i;
    if (t >= n_tokens) continue;
    const int64_t r = t * heads + h;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + tx * 4 + j;
      if (m >= n) continue;
      float s = acc[i][j];
      if (MODE >= 1) {
        float rr = __fadd_rn(__fsub_rn(qq[i], __fmul_rn(2.f, s)), kk[j]);
        rr = fmaxf(rr, 1e-30f);
        const float d = __fsqrt_rn(rr);
        if (MODE == 1) {
          const float t2 = __fadd_rn(1e-3f, __fmul_rn(d, d));
          s = -(float)log((double)t2);
        } else {
          s = d;  // the Euclidean distance itself
        }
      }
      const int64_t o = (r * 2 + p) * (int64_t)n + m;
      if (sizeof(T) == 4)
        reinterpret_cast<float*>(scores)[o] = s;
      else
        reinterpret_cast<__nv_bfloat16*>(scores)[o] = __float2bfloat16_rn(s);
    }
  }
}

}  // namespace pkm

using namespace pkm;

extern "C" int pkm_subkey_scores(const void* query, const void* keys, int dtype, int64_t n_tokens, int64_t heads,
                                 int64_t k_dim, int64_t n_keys, int mode, void* scores, uint32_t* dev_err,
                                 void* stream) {
  if (dtype != PKM_DT_F32 && dtype != PKM_DT_BF16) return fail(PKM_ERR_UNSUPPORTED, "dtype must be f32 or bf16");
  if (n_tokens < 0 || heads <= 0 || k_dim < 2 || (k_dim & 1) || n_keys <= 0)
    return fail(PKM_ERR_INVALID_ARG, "bad size (k_dim must be even)");
  if (mode < 0 || mode > 3)
    return fail(PKM_ERR_INVALID_ARG, "mode must be 0 (dot), 1 (idw), 2 (distance) or 3 (dot, sequential sum)");
  if (heads * 2 > 65535) return fail(PKM_ERR_UNSUPPORTED, "too many heads");
  if (n_tokens == 0) return PKM_OK;
  if (!query || !keys || !scores) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (mode == 0 && dtype == PKM_DT_BF16 && subkey_scores_tc_eligible(heads, k_dim, n_keys, query, keys, scores))
    return subkey_scores_tc(query, keys, n_tokens, heads, k_dim, n_keys, scores, dev_err, st);
  if (mode == 3) mode = 0;
  dim3 grid((unsigned)((n_tokens + kTR - 1) / kTR), (unsigned)((n_keys + kTM - 1) / kTM), (unsigned)(heads * 2));
  if (grid.y > 65535) return fail(PKM_ERR_UNSUPPORTED, "n_keys too large");
#define PKM_SC(T, M)                                                                                              \
  subkey_scores_kernel<T, M><<<grid, 256, 0, st>>>(static_cast<const T*>(query), static_cast<const T*>(keys),    \
                                                   n_tokens, (int)heads, (int)k_dim, (int)n_keys,                 \
                                                   static_cast<T*>(scores))
  if (dtype == PKM_DT_F32) {
    if (mode == 0)
      PKM_SC(float, 0);
    else if (mode == 1)
      PKM_SC(float, 1);
    else
      PKM_SC(float, 2);
  } else {
    if (mode == 0)
      PKM_SC(__nv_bfloat16, 0);
    else if (mode == 1)
      PKM_SC(__nv_bfloat16, 1);
    else
      PKM_SC(__nv_bfloat16, 2);
  }
#undef PKM_SC
  return check_cuda("subkey_scores_kernel");
}
