// Product-key top-k (K2) and the softmax / sub-key-bag preparation for the
// scoring backward.
//
// One warp owns one (token, head) row.  Stage 1 selects the knn best
// sub-keys of each half with a bitwise radix select on order-preserving
// integer keys (ties to the lowest sub-key index), sorts them with a warp
// bitonic network, and stage 2 merges the knn sorted candidate lists
// s1[i] + s2[.] (one list per lane) with warp max/min reductions, taking
// equal sums in ascending slot order.  Nothing of the knn*knn product is
// materialised.
#include <algorithm>

#include "common.cuh"

namespace pkm {

// Order-preserving integer key of a score (larger score -> larger key).
__device__ __forceinline__ uint32_t key32(float x) {
  if (x == 0.f) x = 0.f;  // -0 and +0 compare equal
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ uint32_t key16(uint16_t b) {
  if (b == 0x8000u) b = 0;
  return (b & 0x8000u) ? (uint32_t)(~b & 0xffffu) : (uint32_t)(b | 0x8000u);
}

template <typename T>
struct ScoreT;
template <>
struct ScoreT<float> {
  static constexpr int KEYBITS = 32;
  __device__ static __forceinline__ void load(const float* p, int64_t i, float& v, uint32_t& k) {
    v = p[i];
    k = key32(v);
  }
  __device__ static __forceinline__ float round(float x) { return x; }
  __device__ static __forceinline__ void store(float* p, int64_t i, float v) { p[i] = v; }
};
template <>
struct ScoreT<__nv_bfloat16> {
  static constexpr int KEYBITS = 16;
  __device__ static __forceinline__ void load(const __nv_bfloat16* p, int64_t i, float& v, uint32_t& k) {
    const uint16_t b = reinterpret_cast<const uint16_t*>(p)[i];
    v = __uint_as_float((uint32_t)b << 16);
    k = key16(b);
  }
  __device__ static __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
  __device__ static __forceinline__ void store(__nv_bfloat16* p, int64_t i, float v) {
    p[i] = __float2bfloat16_rn(v);
  }
};

// Warp bitonic sort of one (key, idx, val) per lane: key descending, idx
// ascending.
__device__ __forceinline__ void warp_sort_desc(uint32_t& key, uint32_t& idx, float& val) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const uint32_t ok = __shfl_xor_sync(0xffffffffu, key, stride);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, stride);
      const float ov = __shfl_xor_sync(0xffffffffu, val, stride);
      const bool lower = (lane & stride) == 0;
      // final order is "descending"; in each bitonic merge of `size`, the
      // direction alternates with bit `size` of the lane index
      const bool desc = ((lane & size) == 0) || size == 32;
      const bool other_first = (ok > key) || (ok == key && oi < idx);  // other precedes mine
      const bool take = (lower == desc) ? other_first : !other_first;
      if (take && !(ok == key && oi == idx)) {
        key = ok;
        idx = oi;
        val = ov;
      }
    }
  }
}

// Stage 1 on one half: lane l holds elements l*EPL .. l*EPL+EPL-1.  Returns,
// in lane j < knn, the j-th best (key, index, value), sorted.
template <int EPL, int KEYBITS>
__device__ __forceinline__ void stage1_select(const uint32_t (&key)[EPL], const float (&val)[EPL], int n, int knn,
                                              uint32_t* s_key, uint32_t* s_idx, float* s_val, uint32_t& okey,
                                              uint32_t& oidx, float& oval) {
  const int lane = threadIdx.x & 31;
  uint32_t T = 0;
#pragma unroll 1
  for (int bit = KEYBITS - 1; bit >= 0; --bit) {
    const uint32_t cand = T | (1u << bit);
    int c = 0;
#pragma unroll
    for (int e = 0; e < EPL; ++e) c += key[e] >= cand;
    c = __reduce_add_sync(0xffffffffu, c);
    if (c >= knn) T = cand;
  }
  int gt = 0, eq = 0;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    gt += key[e] > T;
    eq += key[e] == T;
  }
  const int n_gt = __reduce_add_sync(0xffffffffu, gt);
  const int need_eq = knn - n_gt;
  // exclusive prefix of equal counts over lanes (lower lanes hold lower indices)
  int eq_pre = eq;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, eq_pre, d);
    if (lane >= d) eq_pre += o;
  }
  eq_pre -= eq;
  // selection flags and compaction
  int sel = 0;
  uint32_t selmask = 0;
  int eqr = eq_pre;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    bool s = key[e] > T;
    if (key[e] == T) {
      s = eqr < need_eq;
      ++eqr;
    }
    if (lane * EPL + e >= n) s = false;
    if (s) {
      selmask |= 1u << e;
      ++sel;
    }
  }
  int sel_pre = sel;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, sel_pre, d);
    if (lane >= d) sel_pre += o;
  }
  sel_pre -= sel;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    if (selmask & (1u << e)) {
      s_key[sel_pre] = key[e];
      s_idx[sel_pre] = lane * EPL + e;
      s_val[sel_pre] = val[e];
      ++sel_pre;
    }
  }
  __syncwarp();
  if (lane < knn) {
    okey = s_key[lane];
    oidx = s_idx[lane];
    oval = s_val[lane];
  } else {
    okey = 0;
    oidx = 0xffffffffu;
    oval = -INFINITY;
  }
  __syncwarp();
  warp_sort_desc(okey, oidx, oval);
}

template <typename T, int EPL>
__global__ void __launch_bounds__(256) product_topk_kernel(const T* __restrict__ scores, int64_t rows, int n, int knn,
                                                           int64_t* __restrict__ out_idx, T* __restrict__ out_scores,
                                                           T* __restrict__ out_psw, int64_t* __restrict__ sub1,
                                                           int64_t* __restrict__ sub2) {
  __shared__ uint32_t sh_key[8][32];
  __shared__ uint32_t sh_idx[8][32];
  __shared__ float sh_val[8][32];
  __shared__ uint32_t sh_idx2[8][32];
  __shared__ float sh_val2[8][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= rows) return;
  constexpr int KB = ScoreT<T>::KEYBITS;

  uint32_t k1, i1, k2, i2;
  float v1, v2;
  for (int p = 0; p < 2; ++p) {
    const T* row = scores + (r * 2 + p) * (int64_t)n;
    uint32_t key[EPL];
    float val[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int m = lane * EPL + e;
      if (m < n) {
        ScoreT<T>::load(row, m, val[e], key[e]);
      } else {
        val[e] = -INFINITY;
        key[e] = 0;
      }
    }
    uint32_t ok, oi;
    float ov;
    stage1_select<EPL, KB>(key, val, n, knn, sh_key[warp], sh_idx[warp], sh_val[warp], ok, oi, ov);
    if (p == 0) {
      k1 = ok;
      i1 = oi;
      v1 = ov;
    } else {
      k2 = ok;
      i2 = oi;
      v2 = ov;
    }
  }
  (void)k1;
  (void)k2;
  if (sub1 && lane < knn) {
    sub1[r * knn + lane] = i1;
    sub2[r * knn + lane] = i2;
  }
  // stage 2: lane i owns candidates (i, j), j < knn, non-increasing in j
  sh_idx2[warp][lane] = i2;
  sh_val2[warp][lane] = v2;
  __syncwarp();
  const uint32_t* idx2 = sh_idx2[warp];
  const float* val2 = sh_val2[warp];
  const bool live = lane < knn;
  uint32_t done = 0;
  const uint32_t all = knn == 32 ? 0xffffffffu : ((1u << knn) - 1u);
  auto head = [&](uint32_t& hkey, uint32_t& hslot, int& hj, float& hval) {
    hkey = 0;
    hslot = 0xffffffffu;
    hj = -1;
    hval = -INFINITY;
    if (!live) return;
    const uint32_t left = all & ~done;
    if (left == 0) return;
    const int j0 = __ffs(left) - 1;
    const float s0 = ScoreT<T>::round(v1 + val2[j0]);
    hkey = key32(s0);
    hval = s0;
    hj = j0;
    hslot = i1 * (uint32_t)n + idx2[j0];
    for (int j = j0 + 1; j < knn; ++j) {
      const float s = ScoreT<T>::round(v1 + val2[j]);
      if (key32(s) != hkey) break;
      if (done & (1u << j)) continue;
      const uint32_t sl = i1 * (uint32_t)n + idx2[j];
      if (sl < hslot) {
        hslot = sl;
        hj = j;
      }
    }
  };
  uint32_t hkey, hslot;
  int hj;
  float hval;
  head(hkey, hslot, hj, hval);
  uint32_t my_slot = 0;
  float my_val = -INFINITY;
  for (int t = 0; t < knn; ++t) {
    const uint32_t best = __reduce_max_sync(0xffffffffu, hkey);
    const uint32_t cslot = (hkey == best) ? hslot : 0xffffffffu;
    const uint32_t bslot = __reduce_min_sync(0xffffffffu, cslot);
    const bool win = live && hkey == best && hslot == bslot;
    const float wval = __shfl_sync(0xffffffffu, hval, __ffs(__ballot_sync(0xffffffffu, win)) - 1);
    if (lane == t) {
      my_slot = bslot;
      my_val = wval;
    }
    if (win) {
      done |= 1u << hj;
      head(hkey, hslot, hj, hval);
    }
  }
  // outputs + per-row softmax (fp32, stored in the score dtype)
  if (live) {
    out_idx[r * knn + lane] = my_slot;
    ScoreT<T>::store(out_scores, r * knn + lane, my_val);
  }
  if (out_psw) {
    const float mx = __shfl_sync(0xffffffffu, my_val, 0);
    const float ex = live ? expf(my_val - mx) : 0.f;
    const float sum = warp_sum(ex);
    if (live) ScoreT<T>::store(out_psw, r * knn + lane, ex / sum);
  }
}

template <typename T>
static int launch_topk(const void* scores, int64_t rows, int64_t n, int64_t knn, int64_t* idx, void* ts, void* psw,
                       int64_t* s1, int64_t* s2, cudaStream_t st) {
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  const T* sc = static_cast<const T*>(scores);
  T* o = static_cast<T*>(ts);
  T* pw = static_cast<T*>(psw);
  const int ni = (int)n, ki = (int)knn;
#define PKM_TOPK_CASE(E)                                                                      \
  if (n <= 32 * (E)) {                                                                        \
    product_topk_kernel<T, E><<<blocks, 256, 0, st>>>(sc, rows, ni, ki, idx, o, pw, s1, s2); \
    return check_cuda("product_topk_kernel");                                                 \
  }
  PKM_TOPK_CASE(1)
  PKM_TOPK_CASE(2)
  PKM_TOPK_CASE(4)
  PKM_TOPK_CASE(8)
  PKM_TOPK_CASE(16)
  PKM_TOPK_CASE(32)
#undef PKM_TOPK_CASE
  return fail(PKM_ERR_UNSUPPORTED, "n_keys above 1024");
}

// ---------------------------------------------------------------------------
// softmax backward + sub-key bags
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) score_bwd_prep_kernel(const int64_t* __restrict__ indices,
                                                             const T* __restrict__ psw, const T* __restrict__ dpsw,
                                                             int64_t rows, int knn, int heads, int64_t n,
                                                             int64_t* __restrict__ sub_idx, T* __restrict__ sub_w) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= rows) return;
  const bool live = lane < knn;
  float g = 0.f, p = 0.f;
  if (live) {
    g = ld_f(dpsw, sizeof(T) == 4 ? PKM_DT_F32 : PKM_DT_BF16, r * knn + lane);
    if (psw) p = ld_f(psw, sizeof(T) == 4 ? PKM_DT_F32 : PKM_DT_BF16, r * knn + lane);
  }
  float ds = g;
  if (psw) {
    const float dot = warp_sum(p * g);
    ds = p * (g - dot);
  }
  if (!live) return;
  const int64_t slot = indices[r * knn + lane];
  const int64_t h = r % heads;
  const int64_t a = slot / n, b = slot % n;
  const int64_t base = r * 2 * knn;
  sub_idx[base + lane] = (h * 2 + 0) * n + a;
  sub_idx[base + knn + lane] = (h * 2 + 1) * n + b;
  ScoreT<T>::store(sub_w, base + lane, ds);
  ScoreT<T>::store(sub_w, base + knn + lane, ds);
}

// ---------------------------------------------------------------------------
// dense sub-score gradient
// ---------------------------------------------------------------------------
// dS[r, p, m] = sum of ds[r, j] over the selected slots j whose half-p sub-key
// is m, where ds is the softmax backward of the row (or dpsw itself when psw
// is NULL), rounded to the score dtype as the reference's autograd does.
// Entries sharing a sub-key are summed in slot-rank order, so the result is
// deterministic; the whole [2, n] row is written (zeros included).
template <typename T>
__global__ void __launch_bounds__(256) score_grad_dense_kernel(const int64_t* __restrict__ indices,
                                                               const T* __restrict__ psw, const T* __restrict__ dpsw,
                                                               int64_t rows, int knn, int n, T* __restrict__ dS) {
  __shared__ float sh_ds[8][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= rows) return;
  const bool live = lane < knn;
  const int dt = sizeof(T) == 4 ? PKM_DT_F32 : PKM_DT_BF16;
  float g = 0.f, p = 0.f;
  int64_t slot = 0;
  if (live) {
    g = ld_f(dpsw, dt, r * knn + lane);
    if (psw) p = ld_f(psw, dt, r * knn + lane);
    slot = indices[r * knn + lane];
  }
  float ds = g;
  if (psw) {
    const float dot = warp_sum(p * g);
    ds = p * (g - dot);
  }
  sh_ds[warp][lane] = live ? ScoreT<T>::round(ds) : 0.f;
  T* row = dS + r * 2 * (int64_t)n;
  for (int m = lane; m < 2 * n; m += 32) ScoreT<T>::store(row, m, 0.f);
  __syncwarp();
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int key = live ? (int)(half ? slot % n : slot / n) : n + lane;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    if (live && lane == __ffs(peers) - 1) {
      float s = 0.f;
      unsigned mrem = peers;
      while (mrem) {
        const int b = __ffs(mrem) - 1;
        s += sh_ds[warp][b];
        mrem &= mrem - 1;
      }
      ScoreT<T>::store(row, (int64_t)half * n + key, s);
    }
  }
}

}  // namespace pkm

using namespace pkm;

extern "C" int pkm_product_topk(const void* scores, int dtype, int64_t rows, int64_t n_keys, int64_t knn,
                                int64_t* indices, void* top_scores, void* psw, int64_t* sub_indices1,
                                int64_t* sub_indices2, void* stream) {
  if (dtype != PKM_DT_F32 && dtype != PKM_DT_BF16) return fail(PKM_ERR_UNSUPPORTED, "scores must be f32 or bf16");
  if (rows < 0 || knn <= 0 || knn > 32 || n_keys < knn) return fail(PKM_ERR_INVALID_ARG, "need 0 < knn <= 32, knn <= n_keys");
  if (n_keys > 1024) return fail(PKM_ERR_UNSUPPORTED, "n_keys above 1024");
  if ((sub_indices1 == nullptr) != (sub_indices2 == nullptr))
    return fail(PKM_ERR_INVALID_ARG, "sub_indices1/2 must both be given or both NULL");
  if (rows == 0) return PKM_OK;
  if (!scores || !indices || !top_scores) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == PKM_DT_F32)
    return launch_topk<float>(scores, rows, n_keys, knn, indices, top_scores, psw, sub_indices1, sub_indices2, st);
  return launch_topk<__nv_bfloat16>(scores, rows, n_keys, knn, indices, top_scores, psw, sub_indices1, sub_indices2,
                                    st);
}

extern "C" int pkm_score_bwd_prep(const int64_t* indices, const void* psw, const void* dpsw, int dtype, int64_t rows,
                                  int64_t knn, int64_t heads, int64_t n_keys, int64_t* sub_idx, void* sub_w,
                                  void* stream) {
  if (dtype != PKM_DT_F32 && dtype != PKM_DT_BF16) return fail(PKM_ERR_UNSUPPORTED, "dtype must be f32 or bf16");
  if (rows < 0 || knn <= 0 || knn > 32 || heads <= 0 || n_keys <= 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  if (rows == 0) return PKM_OK;
  if (!indices || !dpsw || !sub_idx || !sub_w) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (dtype == PKM_DT_F32)
    score_bwd_prep_kernel<float><<<blocks, 256, 0, st>>>(indices, static_cast<const float*>(psw),
                                                         static_cast<const float*>(dpsw), rows, (int)knn, (int)heads,
                                                         n_keys, sub_idx, static_cast<float*>(sub_w));
  else
    score_bwd_prep_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        indices, static_cast<const __nv_bfloat16*>(psw), static_cast<const __nv_bfloat16*>(dpsw), rows, (int)knn,
        (int)heads, n_keys, sub_idx, static_cast<__nv_bfloat16*>(sub_w));
  return check_cuda("score_bwd_prep_kernel");
}

extern "C" int pkm_score_grad_dense(const int64_t* indices, const void* psw, const void* dpsw, int dtype,
                                    int64_t rows, int64_t knn, int64_t n_keys, void* d_scores, void* stream) {
  if (dtype != PKM_DT_F32 && dtype != PKM_DT_BF16) return fail(PKM_ERR_UNSUPPORTED, "dtype must be f32 or bf16");
  if (rows < 0 || knn <= 0 || knn > 32 || n_keys <= 0 || n_keys > (1 << 30))
    return fail(PKM_ERR_INVALID_ARG, "bad size");
  if (rows == 0) return PKM_OK;
  if (!indices || !dpsw || !d_scores) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (dtype == PKM_DT_F32)
    score_grad_dense_kernel<float><<<blocks, 256, 0, st>>>(indices, static_cast<const float*>(psw),
                                                           static_cast<const float*>(dpsw), rows, (int)knn,
                                                           (int)n_keys, static_cast<float*>(d_scores));
  else
    score_grad_dense_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        indices, static_cast<const __nv_bfloat16*>(psw), static_cast<const __nv_bfloat16*>(dpsw), rows, (int)knn,
        (int)n_keys, static_cast<__nv_bfloat16*>(d_scores));
  return check_cuda("score_grad_dense_kernel");
}
