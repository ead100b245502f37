// Shared helpers for the sm_100a product-key-memory kernels: dtype codes,
// vector conversions, the PTX wrappers for mbarriers and bulk copies, the
// device error word, and host-side argument checking.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/pkm_b200.h"

namespace pkm {

// ---------------------------------------------------------------------------
// host side: error reporting
// ---------------------------------------------------------------------------
void set_last_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_cuda(const char* what);
int num_sms();
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool valid_dtype(int dt) { return dt == PKM_DT_F32 || dt == PKM_DT_BF16 || dt == PKM_DT_F16; }
inline int dtype_size(int dt) { return dt == PKM_DT_F32 ? 4 : 2; }
__host__ __device__ inline int dtype_size_dev(int dt) { return dt == PKM_DT_F32 ? 4 : 2; }

// ---------------------------------------------------------------------------
// device side: scalar conversions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ld_f(const void* p, int dt, int64_t i) {
  if (dt == PKM_DT_F32) return static_cast<const float*>(p)[i];
  if (dt == PKM_DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void st_f(void* p, int dt, int64_t i, float v) {
  if (dt == PKM_DT_F32) {
    static_cast<float*>(p)[i] = v;
  } else if (dt == PKM_DT_BF16) {
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half*>(p)[i] = __float2half_rn(v);
  }
}

template <typename T>
struct DtOf;
template <>
struct DtOf<float> {
  static constexpr int value = PKM_DT_F32;
};
template <>
struct DtOf<__nv_bfloat16> {
  static constexpr int value = PKM_DT_BF16;
};
template <>
struct DtOf<__half> {
  static constexpr int value = PKM_DT_F16;
};

template <typename T>
struct VecTraits;
template <>
struct VecTraits<float> {
  static constexpr int EPV = 4;  // elements per 16-byte vector
  __device__ static __forceinline__ void unpack(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
};
template <>
struct VecTraits<__nv_bfloat16> {
  static constexpr int EPV = 8;
  __device__ static __forceinline__ void unpack(const uint4& v, float* f) {
    // bf16 -> fp32 is a 16-bit left shift of the bit pattern
    f[0] = __uint_as_float(v.x << 16);
    f[1] = __uint_as_float(v.x & 0xffff0000u);
    f[2] = __uint_as_float(v.y << 16);
    f[3] = __uint_as_float(v.y & 0xffff0000u);
    f[4] = __uint_as_float(v.z << 16);
    f[5] = __uint_as_float(v.z & 0xffff0000u);
    f[6] = __uint_as_float(v.w << 16);
    f[7] = __uint_as_float(v.w & 0xffff0000u);
  }
};
template <>
struct VecTraits<__half> {
  static constexpr int EPV = 8;
  __device__ static __forceinline__ void unpack(const uint4& v, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};

// Store n (<= 8) consecutive floats as dtype dt starting at element e0 of p,
// using 16-byte stores where the run is 16-byte aligned.
__device__ __forceinline__ void st_run(void* p, int dt, int64_t e0, const float* f, int n) {
  if (dt == PKM_DT_F32) {
    float* q = static_cast<float*>(p) + e0;
    if (n == 4 && ((reinterpret_cast<uintptr_t>(q) & 15u) == 0)) {
      *reinterpret_cast<float4*>(q) = make_float4(f[0], f[1], f[2], f[3]);
      return;
    }
    if (n == 8 && ((reinterpret_cast<uintptr_t>(q) & 15u) == 0)) {
      reinterpret_cast<float4*>(q)[0] = make_float4(f[0], f[1], f[2], f[3]);
      reinterpret_cast<float4*>(q)[1] = make_float4(f[4], f[5], f[6], f[7]);
      return;
    }
    for (int i = 0; i < n; ++i) q[i] = f[i];
  } else if (dt == PKM_DT_BF16) {
    __nv_bfloat16* q = static_cast<__nv_bfloat16*>(p) + e0;
    if (n == 8 && ((reinterpret_cast<uintptr_t>(q) & 15u) == 0)) {
      uint4 v;
      __nv_bfloat162 t;
      t = __floats2bfloat162_rn(f[0], f[1]);
      v.x = *reinterpret_cast<uint32_t*>(&t);
      t = __floats2bfloat162_rn(f[2], f[3]);
      v.y = *reinterpret_cast<uint32_t*>(&t);
      t = __floats2bfloat162_rn(f[4], f[5]);
      v.z = *reinterpret_cast<uint32_t*>(&t);
      t = __floats2bfloat162_rn(f[6], f[7]);
      v.w = *reinterpret_cast<uint32_t*>(&t);
      *reinterpret_cast<uint4*>(q) = v;
      return;
    }
    for (int i = 0; i < n; ++i) q[i] = __float2bfloat16_rn(f[i]);
  } else {
    __half* q = static_cast<__half*>(p) + e0;
    for (int i = 0; i < n; ++i) q[i] = __float2half_rn(f[i]);
  }
}

// ---------------------------------------------------------------------------
// device side: error word
// ---------------------------------------------------------------------------
__device__ __forceinline__ void raise_err(uint32_t* err, uint32_t bits) {
  if (err) atomicOr(err, bits);
}

// ---------------------------------------------------------------------------
// device side: warp helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// device side: mbarrier + bulk async copy (PTX ISA 8.x, sm_90+)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit` polls (each poll may suspend the
// thread for a hardware-chosen interval) and reports PKM_DEVERR_TIMEOUT.
constexpr uint32_t kWaitLimit = 1u << 24;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  raise_err(err, PKM_DEVERR_TIMEOUT);
  return false;
}

// One contiguous global -> shared copy completing on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace pkm
