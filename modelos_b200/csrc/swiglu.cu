// SwiGLU gate of the memory output and column sums (bias gradients).
//
// Reference: HashingMemory.forward (pkm/memory.py:226-229),
//   output = value_proj(output * F.silu(swilu_projection(input)))
// whose elementwise part torch runs as silu and mul passes forward and as
// mul, mul and silu_backward passes plus two column reductions (the bias
// gradients of the two nn.Linear layers) backward.  Here the gate is one
// pass each way, the bias gradient of the gate's projection is reduced in
// the same backward pass, and the other bias gradient is one column-sum
// pass.  Each intermediate is rounded to the activation dtype where torch's
// eager ops round it:
//   s = silu(h); z = a * s                             (forward)
//   da = dz * s; ds = dz * a; dh = silu_backward(ds, h)  (backward)
// with silu(h) = h / (1 + exp(-h)) and silu_backward(g, h) =
// g * sig * (1 + h * (1 - sig)), sig = 1 / (1 + exp(-h)), in fp32.
#include "rows.cuh"

namespace pkm {

template <typename T>
__device__ __forceinline__ float rnd_t(float x) {
  return sizeof(T) == 4 ? x : __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float silu_f(float h) { return h / (1.f + expf(-h)); }

template <typename T>
__global__ void __launch_bounds__(kNormThreads) swiglu_fwd_kernel(const T* __restrict__ a, const T* __restrict__ h,
                                                                 int64_t n, int64_t c, T* __restrict__ z) {
  const int64_t total = n * (c / kNormChan);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t off = i * kNormChan;
    float av[kNormChan], hv[kNormChan];
    RowIO<T>::load(a + off, av);
    RowIO<T>::load(h + off, hv);
#pragma unroll
    for (int k = 0; k < kNormChan; ++k) av[k] = rnd_t<T>(av[k] * rnd_t<T>(silu_f(hv[k])));
    RowIO<T>::store(z + off, av);
  }
}

// Backward of the gate, and the partial column sums of dh per row block
// (part[rb][c], fp32) when dbias is wanted.
template <typename T>
__global__ void __launch_bounds__(kNormThreads) swiglu_bwd_kernel(const T* __restrict__ dz, const T* __restrict__ a,
                                                                 const T* __restrict__ h, int64_t n, int64_t c,
                                                                 T* __restrict__ da, T* __restrict__ dh,
                                                                 float* __restrict__ part) {
  __shared__ float red[kNormThreads / 32][32 * kNormChan];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c0 = ((int64_t)blockIdx.x * 32 + lane) * kNormChan;
  float sum[kNormChan];
#pragma unroll
  for (int k = 0; k < kNormChan; ++k) sum[k] = 0.f;
  if (c0 < c) {
    int64_t r0, r1;
    row_range(n, blockIdx.y, gridDim.y, r0, r1);
#pragma unroll 2
    for (int64_t r = r0 + warp; r < r1; r += kNormThreads / 32) {
      const int64_t off = r * c + c0;
      float g[kNormChan], av[kNormChan], hv[kNormChan];
      RowIO<T>::load(dz + off, g);
      RowIO<T>::load(a + off, av);
      RowIO<T>::load(h + off, hv);
      float o1[kNormChan], o2[kNormChan];
#pragma unroll
      for (int k = 0; k < kNormChan; ++k) {
        const float sig = 1.f / (1.f + expf(-hv[k]));
        const float s = rnd_t<T>(silu_f(hv[k]));  // silu(h) as the forward rounded it
        const float ds = rnd_t<T>(g[k] * av[k]);
        o1[k] = rnd_t<T>(g[k] * s);
        o2[k] = rnd_t<T>(ds * sig * (1.f + hv[k] * (1.f - sig)));
        sum[k] += o2[k];
      }
      if (da) RowIO<T>::store(da + off, o1);
      RowIO<T>::store(dh + off, o2);
    }
  }
  if (part == nullptr) return;  // grid-uniform
#pragma unroll
  for (int k = 0; k < kNormChan; ++k) red[warp][lane * kNormChan + k] = sum[k];
  __syncthreads();
  const int t = warp * 32 + lane;
  const int64_t ch = (int64_t)blockIdx.x * 32 * kNormChan + t;
  if (ch < c) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) s += red[w][t];
    part[(int64_t)blockIdx.y * c + ch] = s;
  }
}

// Column sums of x over a row block: part[rb][c].
template <typename T>
__global__ void __launch_bounds__(kNormThreads) colsum_kernel(const T* __restrict__ x, int64_t n, int64_t c,
                                                             float* __restrict__ part) {
  __shared__ float red[kNormThreads / 32][32 * kNormChan];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c0 = ((int64_t)blockIdx.x * 32 + lane) * kNormChan;
  float sum[kNormChan];
#pragma unroll
  for (int k = 0; k < kNormChan; ++k) sum[k] = 0.f;
  if (c0 < c) {
    int64_t r0, r1;
    row_range(n, blockIdx.y, gridDim.y, r0, r1);
#pragma unroll 4
    for (int64_t r = r0 + warp; r < r1; r += kNormThreads / 32) {
      float v[kNormChan];
      RowIO<T>::load(x + r * c + c0, v);
#pragma unroll
      for (int k = 0; k < kNormChan; ++k) sum[k] += v[k];
    }
  }
#pragma unroll
  for (int k = 0; k < kNormChan; ++k) red[warp][lane * kNormChan + k] = sum[k];
  __syncthreads();
  const int t = warp * 32 + lane;
  const int64_t ch = (int64_t)blockIdx.x * 32 * kNormChan + t;
  if (ch < c) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) s += red[w][t];
    part[(int64_t)blockIdx.y * c + ch] = s;
  }
}

// out[c] = sum over row blocks of part (fixed order, fp64), as dtype.
__global__ void __launch_bounds__(256) colsum_finalize_kernel(const float* __restrict__ part, int nb, int64_t c,
                                                              void* out, int out_dtype) {
  const Sum2 r = colsum_fixed(part, nullptr, nb, c);
  const int64_t ch = (int64_t)blockIdx.x * 32 + (threadIdx.x & 31);
  if (threadIdx.x < 32 && ch < c) st_f(out, out_dtype, ch, (float)r.a);
}

static int rows_check(int dtype, int64_t n, int64_t c, std::initializer_list<const void*> ptrs) {
  if (dtype != PKM_DT_F32 && dtype != PKM_DT_BF16) return fail(PKM_ERR_UNSUPPORTED, "dtype must be f32 or bf16");
  if (n < 0 || c <= 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  if (c % kNormChan != 0) return fail(PKM_ERR_UNSUPPORTED, "columns must be a multiple of 8");
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return fail(PKM_ERR_INVALID_ARG, "tensors must be 16-byte aligned");
  return PKM_OK;
}

static unsigned flat_blocks(int64_t total) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + kNormThreads - 1) / kNormThreads,
                                                          (int64_t)num_sms() * 8));
}

}  // namespace pkm

using namespace pkm;

extern "C" int pkm_colsum_workspace(int64_t n, int64_t c, size_t* bytes) {
  if (!bytes || n < 0 || c <= 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  *bytes = (size_t)row_blocks(std::max<int64_t>(n, 1), c) * (size_t)c * sizeof(float);
  return PKM_OK;
}

extern "C" int pkm_swiglu_fwd(const void* a, const void* h, int dtype, int64_t n, int64_t c, void* z, void* stream) {
  int rc = rows_check(dtype, n, c, {a, h, z});
  if (rc) return rc;
  if (n == 0) return PKM_OK;
  if (!a || !h || !z) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = flat_blocks(n * (c / kNormChan));
  if (dtype == PKM_DT_F32)
    swiglu_fwd_kernel<float><<<blocks, kNormThreads, 0, st>>>(static_cast<const float*>(a),
                                                               static_cast<const float*>(h), n, c,
                                                               static_cast<float*>(z));
  else
    swiglu_fwd_kernel<__nv_bfloat16><<<blocks, kNormThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(h), n, c,
        static_cast<__nv_bfloat16*>(z));
  return check_cuda("pkm_swiglu_fwd");
}

extern "C" int pkm_swiglu_bwd(const void* dz, const void* a, const void* h, int dtype, int64_t n, int64_t c, void* da,
                              void* dh, void* dbias, int bias_dtype, void* workspace, size_t workspace_bytes,
                              void* stream) {
  int rc = rows_check(dtype, n, c, {dz, a, h, da, dh});
  if (rc) return rc;
  if (!dh) return fail(PKM_ERR_INVALID_ARG, "dh is NULL");
  if (dbias && !valid_dtype(bias_dtype)) return fail(PKM_ERR_INVALID_ARG, "bad bias dtype");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    if (dbias) cudaMemsetAsync(dbias, 0, (size_t)c * dtype_size(bias_dtype), st);
    return check_cuda("pkm_swiglu_bwd");
  }
  if (!dz || !a || !h) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  size_t need = 0;
  pkm_colsum_workspace(n, c, &need);
  if (dbias && (!workspace || workspace_bytes < need)) return fail(PKM_ERR_WORKSPACE, "workspace too small");
  const dim3 grid = row_grid(n, c);
  float* part = dbias ? static_cast<float*>(workspace) : nullptr;
  if (dtype == PKM_DT_F32)
    swiglu_bwd_kernel<float><<<grid, kNormThreads, 0, st>>>(
        static_cast<const float*>(dz), static_cast<const float*>(a), static_cast<const float*>(h), n, c,
        static_cast<float*>(da), static_cast<float*>(dh), part);
  else
    swiglu_bwd_kernel<__nv_bfloat16><<<grid, kNormThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(dz), static_cast<const __nv_bfloat16*>(a),
        static_cast<const __nv_bfloat16*>(h), n, c, static_cast<__nv_bfloat16*>(da), static_cast<__nv_bfloat16*>(dh),
        part);
  if (dbias) colsum_finalize_kernel<<<(unsigned)((c + 31) / 32), 256, 0, st>>>(part, (int)grid.y, c, dbias, bias_dtype);
  return check_cuda("pkm_swiglu_bwd");
}

extern "C" int pkm_colsum(const void* x, int dtype, int64_t n, int64_t c, void* out, int out_dtype, void* workspace,
                          size_t workspace_bytes, void* stream) {
  int rc = rows_check(dtype, n, c, {x});
  if (rc) return rc;
  if (!out || !valid_dtype(out_dtype)) return fail(PKM_ERR_INVALID_ARG, "bad output");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    cudaMemsetAsync(out, 0, (size_t)c * dtype_size(out_dtype), st);
    return check_cuda("pkm_colsum");
  }
  size_t need = 0;
  pkm_colsum_workspace(n, c, &need);
  if (!x) return fail(PKM_ERR_INVALID_ARG, "x is NULL");
  if (!workspace || workspace_bytes < need) return fail(PKM_ERR_WORKSPACE, "workspace too small");
  const dim3 grid = row_grid(n, c);
  float* part = static_cast<float*>(workspace);
  if (dtype == PKM_DT_F32)
    colsum_kernel<float><<<grid, kNormThreads, 0, st>>>(static_cast<const float*>(x), n, c, part);
  else
    colsum_kernel<__nv_bfloat16><<<grid, kNormThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(x), n, c, part);
  colsum_finalize_kernel<<<(unsigned)((c + 31) / 32), 256, 0, st>>>(part, (int)grid.y, c, out, out_dtype);
  return check_cuda("pkm_colsum");
}
