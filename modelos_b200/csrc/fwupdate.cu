// Fused fast-weight update of the FwPKM value table (one SGD step of the
// inner loop) and its backward.
//
// Reference: FastWeightProductKeyMemory.update_fw (fwpkm/fwpkm.py:274-367)
// with update_fw_param (:266-272), value branch:
//   g_s  = g * scale / max(bincount(indices), 1)     (per row)
//   u    = clamp(g_s, -1, 1) if grad_clip else g_s
//   p'   = p - lr * (u + wd * p)
// which torch runs as six elementwise passes over the [K, D] table (plus the
// bincount).  Here: one counting kernel and one pass that reads p and g and
// writes p' and g_s (the reference returns g_s for its gradient norms).
// The arithmetic is the reference's operation by operation, each rounded to
// the table dtype as torch's eager ops round their results (no contraction
// into fused multiply-adds), so fp32 results are bit-identical.
//
// Backward (the outer loss differentiates through the inner update when the
// inner gradients were taken with create_graph):
//   dp = dp' * (1 - lr * wd)
//   dg = (scale / count) * (dg_s - lr * dp' * [|g_s| <= 1 when clipping])
#include <algorithm>

#include "common.cuh"
#include "count.cuh"

namespace pkm {

template <typename T>
struct FwIO;
template <>
struct FwIO<float> {
  static constexpr int EPV = 4;
  __device__ static __forceinline__ float rnd(float x) { return x; }
  __device__ static __forceinline__ void load(const float* p, float (&v)[4]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
  }
  __device__ static __forceinline__ void store(float* p, const float (&v)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <>
struct FwIO<__nv_bfloat16> {
  static constexpr int EPV = 8;
  __device__ static __forceinline__ float rnd(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
  __device__ static __forceinline__ void load(const __nv_bfloat16* p, float (&v)[8]) {
    VecTraits<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(p), v);
  }
  __device__ static __forceinline__ void store(__nv_bfloat16* p, const float (&v)[8]) {
    st_run(p, PKM_DT_BF16, 0, v, 8);
  }
};

struct FwScalars {
  float scale, lr, wd, one_minus;
  int clip;
};

template <typename T>
__global__ void __launch_bounds__(256) fw_update_kernel(const T* __restrict__ p, const T* __restrict__ g,
                                                       const int32_t* __restrict__ counts, int64_t rows, int64_t dim,
                                                       FwScalars s, T* __restrict__ out_p, T* __restrict__ out_gs) {
  using IO = FwIO<T>;
  constexpr int E = IO::EPV;
  const int64_t vec = dim / E;
  const int64_t total = rows * vec;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec;
    const int64_t off = i * E;
    const int c = counts[r];
    const float cnt = IO::rnd((float)(c == 0 ? 1 : c));  // the counts are cast to the table dtype
    float pv[E], gv[E];
    IO::load(p + off, pv);
    IO::load(g + off, gv);
#pragma unroll
    for (int k = 0; k < E; ++k) {
      const float gs = IO::rnd(__fdiv_rn(IO::rnd(__fmul_rn(gv[k], s.scale)), cnt));
      const float u = s.clip ? fminf(fmaxf(gs, -1.f), 1.f) : gs;
      const float decay = IO::rnd(__fmul_rn(s.wd, pv[k]));
      const float step = IO::rnd(__fmul_rn(s.lr, IO::rnd(__fadd_rn(u, decay))));
      gv[k] = gs;
      pv[k] = IO::rnd(__fsub_rn(pv[k], step));
    }
    IO::store(out_p + off, pv);
    if (out_gs) IO::store(out_gs + off, gv);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) fw_update_bwd_kernel(const T* __restrict__ d_new, const T* __restrict__ d_gs,
                                                           const T* __restrict__ gs, const int32_t* __restrict__ counts,
                                                           int64_t rows, int64_t dim, FwScalars s,
                                                           T* __restrict__ d_p, T* __restrict__ d_g) {
  using IO = FwIO<T>;
  constexpr int E = IO::EPV;
  const int64_t vec = dim / E;
  const int64_t total = rows * vec;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec;
    const int64_t off = i * E;
    const int c = counts[r];
    const float f = s.scale / (float)(c == 0 ? 1 : c);
    float dn[E], dg[E], gv[E];
    IO::load(d_new + off, dn);
    if (d_gs) {
      IO::load(d_gs + off, dg);
    } else {
#pragma unroll
      for (int k = 0; k < E; ++k) dg[k] = 0.f;
    }
    if (s.clip) IO::load(gs + off, gv);
#pragma unroll
    for (int k = 0; k < E; ++k) {
      const bool pass = !s.clip || (gv[k] >= -1.f && gv[k] <= 1.f);
      const float du = pass ? -s.lr * dn[k] : 0.f;
      dg[k] = f * (dg[k] + du);
      dn[k] = dn[k] * s.one_minus;
    }
    if (d_p) IO::store(d_p + off, dn);
    if (d_g) IO::store(d_g + off, dg);
  }
}

static unsigned fw_blocks(int64_t total) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16));
}

static int fw_check(int dtype, int64_t rows, int64_t dim, std::initializer_list<const void*> vec_ptrs) {
  if (dtype != PKM_DT_F32 && dtype != PKM_DT_BF16) return fail(PKM_ERR_UNSUPPORTED, "dtype must be f32 or bf16");
  if (rows < 0 || dim <= 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  if ((dim * dtype_size(dtype)) % 16 != 0) return fail(PKM_ERR_UNSUPPORTED, "row bytes must be a multiple of 16");
  for (const void* q : vec_ptrs)
    if (q && !aligned16(q)) return fail(PKM_ERR_INVALID_ARG, "tensors must be 16-byte aligned");
  return PKM_OK;
}

static FwScalars fw_scalars(int dtype, double scale, double lr, double wd, int clip) {
  // torch's elementwise ops on f32 / bf16 tensors compute in fp32 with the
  // Python scalar cast to fp32, and round each result to the tensor dtype
  (void)dtype;
  FwScalars s;
  s.scale = (float)scale;
  s.lr = (float)lr;
  s.wd = (float)wd;
  s.one_minus = (float)(1.0 - lr * wd);
  s.clip = clip;
  return s;
}

}  // namespace pkm

using namespace pkm;

extern "C" int pkm_fw_update(const void* values, const void* grad, int dtype, int64_t rows, int64_t dim,
                             const int64_t* indices, int64_t n_indices, double scale, double lr, double weight_decay,
                             int grad_clip, void* new_values, void* scaled_grad, int32_t* counts, uint32_t* dev_err,
                             void* stream) {
  int rc = fw_check(dtype, rows, dim, {values, grad, new_values, scaled_grad});
  if (rc) return rc;
  if (rows == 0) return PKM_OK;
  if (!values || !grad || !new_values || !counts || (n_indices > 0 && !indices))
    return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaMemsetAsync(counts, 0, sizeof(int32_t) * rows, st);
  if (n_indices > 0)
    slot_count_kernel<<<fw_blocks(n_indices), 256, 0, st>>>(indices, n_indices, rows, counts, dev_err);
  const FwScalars s = fw_scalars(dtype, scale, lr, weight_decay, grad_clip);
  const int64_t total = rows * dim * dtype_size(dtype) / 16;
  if (dtype == PKM_DT_F32)
    fw_update_kernel<float><<<fw_blocks(total), 256, 0, st>>>(
        static_cast<const float*>(values), static_cast<const float*>(grad), counts, rows, dim, s,
        static_cast<float*>(new_values), static_cast<float*>(scaled_grad));
  else
    fw_update_kernel<__nv_bfloat16><<<fw_blocks(total), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(values), static_cast<const __nv_bfloat16*>(grad), counts, rows, dim, s,
        static_cast<__nv_bfloat16*>(new_values), static_cast<__nv_bfloat16*>(scaled_grad));
  return check_cuda("pkm_fw_update");
}

extern "C" int pkm_fw_update_bwd(const void* d_new_values, const void* d_scaled_grad, const void* scaled_grad,
                                 const int32_t* counts, int dtype, int64_t rows, int64_t dim, double scale, double lr,
                                 double weight_decay, int grad_clip, void* d_values, void* d_grad, void* stream) {
  int rc = fw_check(dtype, rows, dim, {d_new_values, d_scaled_grad, scaled_grad, d_values, d_grad});
  if (rc) return rc;
  if (rows == 0) return PKM_OK;
  if (!d_new_values || !counts || (grad_clip && !scaled_grad)) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const FwScalars s = fw_scalars(dtype, scale, lr, weight_decay, grad_clip);
  const int64_t total = rows * dim * dtype_size(dtype) / 16;
  if (dtype == PKM_DT_F32)
    fw_update_bwd_kernel<float><<<fw_blocks(total), 256, 0, st>>>(
        static_cast<const float*>(d_new_values), static_cast<const float*>(d_scaled_grad),
        static_cast<const float*>(scaled_grad), counts, rows, dim, s, static_cast<float*>(d_values),
        static_cast<float*>(d_grad));
  else
    fw_update_bwd_kernel<__nv_bfloat16><<<fw_blocks(total), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(d_new_values), static_cast<const __nv_bfloat16*>(d_scaled_grad),
        static_cast<const __nv_bfloat16*>(scaled_grad), counts, rows, dim, s, static_cast<__nv_bfloat16*>(d_values),
        static_cast<__nv_bfloat16*>(d_grad));
  return check_cuda("pkm_fw_update_bwd");
}
