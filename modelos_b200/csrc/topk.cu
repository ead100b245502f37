// Product-key top-k (K2) and the softmax / sub-key-bag preparation for the
// scoring backward.
//
// One warp owns one (token, head) row at a time (a persistent grid walks the
// rows).  Stage 1 selects the knn best sub-keys of each half: a bitwise radix
// select on order-preserving integer keys finds the knn-th largest key T,
// the keys above T and the lowest-index keys equal to T are compacted, and a
// warp bitonic network sorts them (score descending, index ascending).  Full
// bf16 rows first try a shorter route (a bound from each lane's best two, a
// few dozen candidates placed by their ranks; stage1_select_bf16).
//
// Stage 2 needs the knn best sums s1[i] + s2[j] (rounded to the score dtype)
// of the knn x knn product.  With both lists sorted, the pair (i, j) is
// preceded by the (i+1)(j+1)-1 pairs (i', j') with i' <= i, j' <= j, whose
// sums are no smaller, so every pair of the top knn in the order
// (sum descending, (i, j) ascending) has (i+1)(j+1) <= knn: at most 119
// candidates for knn = 32 instead of 1024.  The knn-th largest sum T of the
// candidates is therefore the knn-th largest of all pairs, every pair with a
// larger sum is a candidate, and only pairs equal to T can lie outside the
// candidate set.  Row i's sums fall with j, so pair (i, knn/(i+1)) tells
// whether row i has such a pair; if any row has one (rare), the row is
// finished by an exact k-way merge of the knn sorted rows instead.  Pairs
// equal to T are taken in ascending slot order (slot = i1 * n + i2), as
// many as the top knn has room for; the knn selected pairs are placed in
// the output by their ranks.  Nothing of the product is materialised.
//
// Non-finite scores (a diverged model) keep every index a valid slot: NaN
// ranks above +inf, as in torch.topk, in both stages.
#include <algorithm>

#include "common.cuh"

namespace pkm {

// Order-preserving integer key of a score (larger score -> larger key).
// Every NaN takes the largest key (torch.topk ranks NaN above +inf), so a
// present element never has key 0, the mark of an absent one.
__device__ __forceinline__ uint32_t key32(float x) {
  if (x == 0.f) x = 0.f;  // -0 and +0 compare equal
  const uint32_t u = __float_as_uint(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unkey32(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
__device__ __forceinline__ uint32_t key16(uint32_t b) {
  if (b == 0x8000u) b = 0;
  if ((b & 0x7fffu) > 0x7f80u) return 0xffffu;  // NaN
  return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}
// When a row's stage-1 values hold both +inf and -inf, its pair sums are
// formed with +-inf taken as +-FLT_MAX, so that no sum is inf - inf: the
// sum's key then never increases along a sorted row or column (NaN operands
// give NaN sums, the largest key), which the candidate pruning and the
// bounded selection rely on.  Rows without that mix keep exact sums.
__device__ __forceinline__ float sat_inf(float x) {
  return fabsf(x) == INFINITY ? copysignf(3.402823466e38f, x) : x;
}
__device__ __forceinline__ float unkey16(uint32_t k) {
  const uint32_t b = (k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu);
  return __uint_as_float(b << 16);
}

template <typename T>
struct ScoreT;
template <>
struct ScoreT<float> {
  static constexpr int KEYBITS = 32;
  static constexpr int PER_VEC = 4;  // scores per 16-byte load
  __device__ static __forceinline__ uint32_t key_at(const float* p, int64_t i) { return key32(p[i]); }
  __device__ static __forceinline__ void keys_of(const uint4& v, uint32_t* k) {
    k[0] = key32(__uint_as_float(v.x));
    k[1] = key32(__uint_as_float(v.y));
    k[2] = key32(__uint_as_float(v.z));
    k[3] = key32(__uint_as_float(v.w));
  }
  __device__ static __forceinline__ float value(uint32_t k) { return unkey32(k); }
  __device__ static __forceinline__ float round(float x) { return x; }
  // key of a value already representable in the score dtype
  __device__ static __forceinline__ uint32_t key_of(float x) { return key32(x); }
  __device__ static __forceinline__ void store(float* p, int64_t i, float v) { p[i] = v; }
};
template <>
struct ScoreT<__nv_bfloat16> {
  static constexpr int KEYBITS = 16;
  static constexpr int PER_VEC = 8;
  __device__ static __forceinline__ uint32_t key_at(const __nv_bfloat16* p, int64_t i) {
    return key16(reinterpret_cast<const uint16_t*>(p)[i]);
  }
  __device__ static __forceinline__ void keys_of(const uint4& v, uint32_t* k) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      k[2 * i] = key16(w[i] & 0xffffu);
      k[2 * i + 1] = key16(w[i] >> 16);
    }
  }
  __device__ static __forceinline__ float value(uint32_t k) { return unkey16(k); }
  __device__ static __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
  __device__ static __forceinline__ uint32_t key_of(float x) { return key16(__float_as_uint(x) >> 16); }
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

// The k-th largest key (counting repeats) over the whole warp: bitwise
// radix select.  Absent elements carry key 0, which no finite score has, so
// they are never counted.  The caller passes keys lo <= T <= hi that bound
// the answer: T shares their common high bits, and the search starts below
// them.
template <int NE>
__device__ __forceinline__ uint32_t warp_kth_key(const uint32_t (&key)[NE], int k, uint32_t lo, uint32_t hi) {
  const uint32_t diff = lo ^ hi;
  if (diff == 0) return lo;
  const int top = 31 - __clz(diff);  // highest bit where lo and hi differ
  uint32_t T = lo & ~((2u << top) - 1u);
#pragma unroll 1
  for (int bit = top; bit >= 0; --bit) {
    const uint32_t cand = T | (1u << bit);
    int c = 0;
#pragma unroll
    for (int e = 0; e < NE; ++e) c += key[e] >= cand;
    if (__reduce_add_sync(0xffffffffu, c) >= k) T = cand;
  }
  return T;
}

__device__ __forceinline__ int warp_excl_prefix(int v) {
  const int lane = threadIdx.x & 31;
  int p = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, p, d);
    if (lane >= d) p += o;
  }
  return p - v;
}

// Stage 1 on one half: lane l holds the keys of elements l*EPL ..
// l*EPL+EPL-1 (key 0 where the element does not exist).  Returns, in lane
// j < knn, the j-th best (key, index), sorted.
template <typename T, int EPL>
__device__ __forceinline__ void stage1_select(const uint32_t (&key)[EPL], int knn, uint32_t* s_key,
                                              uint32_t* s_idx, uint32_t& okey, uint32_t& oidx) {
  const int lane = threadIdx.x & 31;
  // bounds: the largest key, and the smallest lane maximum (every lane's
  // maximum is at least that, so at least 32 >= knn keys are)
  uint32_t lmax = key[0];
#pragma unroll
  for (int e = 1; e < EPL; ++e) lmax = max(lmax, key[e]);
  const uint32_t Tk = warp_kth_key<EPL>(key, knn, __reduce_min_sync(0xffffffffu, lmax),
                                        __reduce_max_sync(0xffffffffu, lmax));
  int gt = 0, eq = 0;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    gt += key[e] > Tk;
    eq += key[e] == Tk;
  }
  const int need_eq = knn - __reduce_add_sync(0xffffffffu, gt);
  // lower lanes hold lower indices: equal keys are taken in lane order
  int eqr = warp_excl_prefix(eq);
  uint32_t selmask = 0;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    bool s = key[e] > Tk;
    if (key[e] == Tk) {
      s = eqr < need_eq;
      ++eqr;
    }
    if (s) selmask |= 1u << e;
  }
  int pos = warp_excl_prefix(__popc(selmask));
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    if (selmask & (1u << e)) {
      s_key[pos] = key[e];
      s_idx[pos] = lane * EPL + e;
      ++pos;
    }
  }
  __syncwarp();
  okey = lane < knn ? s_key[lane] : 0u;
  oidx = lane < knn ? s_idx[lane] : 0xffffffffu;
  __syncwarp();
  float dummy = 0.f;
  warp_sort_desc(okey, oidx, dummy);
}

// Number of true halves in the sum (mod 2^32) of at most 8 bf16x2 compare
// masks (0xffff per true half): the low half holds -lo mod 2^16, the high
// half -hi mod 2^16 after the low half's borrow is removed.
__device__ __forceinline__ int mask_count(uint32_t s) {
  const uint32_t lo = (0u - s) & 0xffffu;
  const uint32_t rest = s - lo * 0xffffu;
  return (int)(lo + (((0u - rest) >> 16) & 0xffffu));
}
__device__ __forceinline__ __nv_bfloat162 bf2(uint32_t w) { return *reinterpret_cast<__nv_bfloat162*>(&w); }
__device__ __forceinline__ uint32_t unkey16_bits(uint32_t k) { return (k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu); }

// Stage 1 for bf16 rows held as raw pairs (lane l: elements l*EPL ..
// l*EPL+EPL-1, word k = elements 2k and 2k+1): the same selection as
// stage1_select, with every count taken by packed bf16x2 comparisons
// (two elements per instruction, -0 equal to +0 as in the key order).
//
// Most rows take a shorter route first.  The knn-th largest L of the 64
// values {best two of each lane} is a lower bound of the knn-th largest
// score T (at least knn distinct elements are >= L), and on scores of
// trained or random layers only ~36 of 512 elements reach it.  Those are
// compacted as 32-bit composites (key << 16 | 0xffff - index: larger is
// better, all distinct), each one's rank among them is counted, and the
// knn of rank < knn land in rank order: sorted, ties at T taken by lowest
// index, exactly the selection below.  Rows with more than 64 elements at
// or above L (wide ties) take the radix select.
constexpr int kCandCap = 64;

template <int EPL>
__device__ __forceinline__ void stage1_select_bf16(const uint32_t (&w)[EPL / 2], int knn, uint32_t* s_key,
                                                   uint32_t* s_idx, uint32_t* s_comp, uint32_t& okey,
                                                   uint32_t& oidx) {
  constexpr int NW = EPL / 2;
  static_assert(NW <= 8, "mask_count takes at most 8 masks");
  const int lane = threadIdx.x & 31;
  __nv_bfloat162 m2 = bf2(w[0]);
#pragma unroll
  for (int k = 1; k < NW; ++k) m2 = __hmax2_nan(m2, bf2(w[k]));  // a NaN anywhere reaches the lane maximum
  const uint32_t mw = *reinterpret_cast<uint32_t*>(&m2);
  if (__any_sync(0xffffffffu, (mw & 0x7fffu) > 0x7f80u || ((mw >> 16) & 0x7fffu) > 0x7f80u)) {
    // packed comparisons never count a NaN: select on integer keys instead
    uint32_t key[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) key[e] = key16((e & 1) ? (w[e >> 1] >> 16) : (w[e >> 1] & 0xffffu));
    stage1_select<__nv_bfloat16, EPL>(key, knn, s_key, s_idx, okey, oidx);
    return;
  }
  const uint32_t lmax = max(key16(mw & 0xffffu), key16(mw >> 16));
  const uint32_t lo = __reduce_min_sync(0xffffffffu, lmax), hi = __reduce_max_sync(0xffffffffu, lmax);
  {
    // the lane's best two (even and odd elements apart, then merged)
    __nv_bfloat162 t1 = bf2(w[0]), t2 = bf2(0xff80ff80u);
#pragma unroll
    for (int k = 1; k < NW; ++k) {
      const __nv_bfloat162 x = bf2(w[k]);
      t2 = __hmax2(t2, __hmin2(t1, x));
      t1 = __hmax2(t1, x);
    }
    const uint32_t t1w = *reinterpret_cast<uint32_t*>(&t1), t2w = *reinterpret_cast<uint32_t*>(&t2);
    const uint32_t ka = key16(t1w & 0xffffu), kb = key16(t1w >> 16);
    const uint32_t two[2] = {max(ka, kb), max(min(ka, kb), max(key16(t2w & 0xffffu), key16(t2w >> 16)))};
    const uint32_t L = warp_kth_key<2>(two, knn, lo, hi);
    const uint32_t lb = unkey16_bits(L);
    const __nv_bfloat162 l2 = bf2(lb | (lb << 16));
    uint32_t gem[NW];
    uint32_t gacc = 0;
#pragma unroll
    for (int k = 0; k < NW; ++k) {
      gem[k] = __hge2_mask(bf2(w[k]), l2);
      gacc += gem[k];
    }
    const int cnt = mask_count(gacc);
    const int total = __reduce_add_sync(0xffffffffu, cnt);
    if (total <= kCandCap) {
      int pos = warp_excl_prefix(cnt);
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        if ((gem[e >> 1] >> ((e & 1) ? 31 : 15)) & 1u) {
          const uint32_t kk = key16((e & 1) ? (w[e >> 1] >> 16) : (w[e >> 1] & 0xffffu));
          s_comp[pos++] = (kk << 16) | (0xffffu - (uint32_t)(lane * EPL + e));
        }
      }
      if (lane < 4) s_comp[total + lane] = 0u;  // pads the last 16-byte group; no element's composite is 0
      __syncwarp();
      const uint32_t c0 = lane < total ? s_comp[lane] : 0u;
      const uint32_t c1 = lane + 32 < total ? s_comp[lane + 32] : 0u;
      int r0 = 0, r1 = 0;
      for (int i = 0; i < total; i += 4) {
        const uint4 x = *reinterpret_cast<const uint4*>(s_comp + i);
        r0 += (x.x > c0) + (x.y > c0) + (x.z > c0) + (x.w > c0);
        r1 += (x.x > c1) + (x.y > c1) + (x.z > c1) + (x.w > c1);
      }
      if (lane < total && r0 < knn) {
        s_key[r0] = c0 >> 16;
        s_idx[r0] = 0xffffu - (c0 & 0xffffu);
      }
      if (lane + 32 < total && r1 < knn) {
        s_key[r1] = c1 >> 16;
        s_idx[r1] = 0xffffu - (c1 & 0xffffu);
      }
      __syncwarp();
      okey = lane < knn ? s_key[lane] : 0u;
      oidx = lane < knn ? s_idx[lane] : 0xffffffffu;
      __syncwarp();
      return;
    }
  }
  uint32_t T = lo;
  if (lo != hi) {
    const int top = 31 - __clz(lo ^ hi);
    T = lo & ~((2u << top) - 1u);
#pragma unroll 1
    for (int bit = top; bit >= 0; --bit) {
      const uint32_t cand = T | (1u << bit);
      const uint32_t cb = unkey16_bits(cand);
      const __nv_bfloat162 c2 = bf2(cb | (cb << 16));
      uint32_t acc = 0;
#pragma unroll
      for (int k = 0; k < NW; ++k) acc += __hge2_mask(bf2(w[k]), c2);
      if (__reduce_add_sync(0xffffffffu, mask_count(acc)) >= knn) T = cand;
    }
  }
  const uint32_t tb = unkey16_bits(T);
  const __nv_bfloat162 t2 = bf2(tb | (tb << 16));
  uint32_t gtm[NW], eqm[NW];
  uint32_t gacc = 0, eacc = 0;
#pragma unroll
  for (int k = 0; k < NW; ++k) {
    gtm[k] = __hgt2_mask(bf2(w[k]), t2);
    eqm[k] = __heq2_mask(bf2(w[k]), t2);
    gacc += gtm[k];
    eacc += eqm[k];
  }
  const int need_eq = knn - __reduce_add_sync(0xffffffffu, mask_count(gacc));
  // lower lanes hold lower indices: equal keys are taken in lane order
  int eqr = warp_excl_prefix(mask_count(eacc));
  uint32_t selmask = 0;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const uint32_t sh = (e & 1) ? 31 : 15;
    bool sel = (gtm[e >> 1] >> sh) & 1u;
    if ((eqm[e >> 1] >> sh) & 1u) {
      sel = eqr < need_eq;
      ++eqr;
    }
    if (sel) selmask |= 1u << e;
  }
  int pos = warp_excl_prefix(__popc(selmask));
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    if (selmask & (1u << e)) {
      s_key[pos] = key16((e & 1) ? (w[e >> 1] >> 16) : (w[e >> 1] & 0xffffu));
      s_idx[pos] = lane * EPL + e;
      ++pos;
    }
  }
  __syncwarp();
  okey = lane < knn ? s_key[lane] : 0u;
  oidx = lane < knn ? s_idx[lane] : 0xffffffffu;
  __syncwarp();
  float dummy = 0.f;
  warp_sort_desc(okey, oidx, dummy);
}

// Exact stage 2 by a k-way merge of the knn sorted rows s1[i] + s2[.] (one
// row per lane, equal sums in ascending slot order).  Used for rows where
// pairs equal to the knn-th sum lie outside the candidate set.
template <typename T>
__device__ void stage2_merge(float v1, uint32_t i1, const uint32_t* idx2, const float* val2, int knn, int n,
                             uint32_t& my_slot, float& my_val) {
  const int lane = threadIdx.x & 31;
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
  my_slot = 0;
  my_val = -INFINITY;
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
}

constexpr int kTopkWarps = 8;
#ifndef PKM_TOPK_MINB
#define PKM_TOPK_MINB 3  // resident blocks per SM the register budget is sized for
#endif
constexpr int kPairCap = 128;  // candidate pairs for knn <= 32 (119 at knn = 32)

template <typename T, int EPL>
__global__ void __launch_bounds__(kTopkWarps * 32, PKM_TOPK_MINB) product_topk_kernel(const T* __restrict__ scores, int64_t rows,
                                                                        int n, int knn,
                                                                        int64_t* __restrict__ out_idx,
                                                                        T* __restrict__ out_scores,
                                                                        T* __restrict__ out_psw,
                                                                        int64_t* __restrict__ sub1,
                                                                        int64_t* __restrict__ sub2, bool vec_ok) {
  __shared__ __align__(16) uint32_t sh_key[kTopkWarps][32];
  __shared__ __align__(16) uint32_t sh_idx[kTopkWarps][32];
  __shared__ float sh_v1[kTopkWarps][32];
  __shared__ uint32_t sh_i1[kTopkWarps][32];
  __shared__ float sh_v2[kTopkWarps][32];
  __shared__ uint32_t sh_i2[kTopkWarps][32];
  __shared__ uint16_t sh_pair[kTopkWarps][kPairCap];
  __shared__ __align__(16) uint32_t sh_comp[kTopkWarps][kCandCap + 4];
  __shared__ __align__(16) unsigned long long sh_comp64[kTopkWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int KB = ScoreT<T>::KEYBITS;
  constexpr int PV = ScoreT<T>::PER_VEC;
  constexpr int NV = (EPL % PV == 0) ? EPL / PV : 0;  // 16-byte loads per lane and half
  // bf16 rows of 8 or 16 scores per lane take the packed-pair stage 1
  constexpr bool kPackedBf16 = sizeof(T) == 2 && (EPL == 8 || EPL == 16);
  const bool full = n == 32 * EPL;

  // candidate pairs (i, j) with (i+1)(j+1) <= knn, packed i | j << 8
  int n_pairs;
  {
    const int cnt = lane < knn ? knn / (lane + 1) : 0;
    const int off = warp_excl_prefix(cnt);
    for (int j = 0; j < cnt; ++j) sh_pair[warp][off + j] = (uint16_t)(lane | (j << 8));
    n_pairs = __shfl_sync(0xffffffffu, off + cnt, 31);
    __syncwarp();
  }
  uint32_t* s_key = sh_key[warp];
  uint32_t* s_idx = sh_idx[warp];
  unsigned long long* s_comp64 = sh_comp64[warp];

  const int64_t warps_total = (int64_t)gridDim.x * kTopkWarps;
  for (int64_t r = (int64_t)blockIdx.x * kTopkWarps + warp; r < rows; r += warps_total) {
    uint32_t k1, i1, k2, i2;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const T* row = scores + (r * 2 + p) * (int64_t)n;
      uint32_t key[EPL];
      uint32_t ok, oi;
      if constexpr (kPackedBf16) {
        if (full && vec_ok) {
        // bf16 rows compared as packed pairs
        uint32_t w[EPL / 2];
        const uint4* vp = reinterpret_cast<const uint4*>(row + (int64_t)lane * EPL);
#pragma unroll
        for (int v = 0; v < EPL / 8; ++v) {
          const uint4 q = __ldg(vp + v);
          w[4 * v] = q.x;
          w[4 * v + 1] = q.y;
          w[4 * v + 2] = q.z;
          w[4 * v + 3] = q.w;
        }
        stage1_select_bf16<EPL>(w, knn, s_key, s_idx, sh_comp[warp], ok, oi);
        if (p == 0) {
          k1 = ok;
          i1 = oi;
        } else {
          k2 = ok;
          i2 = oi;
        }
        continue;
        }
      }
      if (NV > 0 && full && vec_ok) {
        const uint4* vp = reinterpret_cast<const uint4*>(row + (int64_t)lane * EPL);
#pragma unroll
        for (int v = 0; v < (NV > 0 ? NV : 1); ++v) ScoreT<T>::keys_of(__ldg(vp + v), key + v * PV);
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const int m = lane * EPL + e;
          key[e] = m < n ? ScoreT<T>::key_at(row, m) : 0u;
        }
      }
      stage1_select<T, EPL>(key, knn, s_key, s_idx, ok, oi);
      if (p == 0) {
        k1 = ok;
        i1 = oi;
      } else {
        k2 = ok;
        i2 = oi;
      }
    }
    const bool live = lane < knn;
    float v1 = live ? ScoreT<T>::value(k1) : -INFINITY;
    float v2 = live ? ScoreT<T>::value(k2) : -INFINITY;
    if (__any_sync(0xffffffffu, live && (v1 == INFINITY || v2 == INFINITY)) &&
        __any_sync(0xffffffffu, live && (v1 == -INFINITY || v2 == -INFINITY)) && live) {
      v1 = sat_inf(v1);  // +inf and -inf both present: keep every sum free of inf - inf
      v2 = sat_inf(v2);
    }
    if (sub1 && live) {
      sub1[r * knn + lane] = i1;
      sub2[r * knn + lane] = i2;
    }
    sh_v1[warp][lane] = v1;
    sh_i1[warp][lane] = i1;
    sh_v2[warp][lane] = v2;
    sh_i2[warp][lane] = i2;
    __syncwarp();

    // stage 2 over the candidate pairs, four per lane
    uint32_t ck[4], cs[4];
    float cv[4];
    uint32_t cvalid = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int c = lane + 32 * t;
      ck[t] = 0;
      cs[t] = 0xffffffffu;
      cv[t] = -INFINITY;
      if (c < n_pairs) {
        const uint32_t pr = sh_pair[warp][c];
        const int pi = pr & 0xff, pj = pr >> 8;
        cv[t] = ScoreT<T>::round(sh_v1[warp][pi] + sh_v2[warp][pj]);
        ck[t] = ScoreT<T>::key_of(cv[t]);
        cs[t] = sh_i1[warp][pi] * (uint32_t)n + sh_i2[warp][pj];
        cvalid |= 1u << t;
      }
    }
    // bounds: the best pair (0, 0), and the knn pairs (i, 0) or (0, j)
    const float b0 = sh_v2[warp][0], a0 = sh_v1[warp][0];
    const uint32_t hi_k = ScoreT<T>::key_of(ScoreT<T>::round(a0 + b0));
    const uint32_t lo_k = max(ScoreT<T>::key_of(ScoreT<T>::round(sh_v1[warp][knn - 1] + b0)),
                              ScoreT<T>::key_of(ScoreT<T>::round(a0 + sh_v2[warp][knn - 1])));
    const uint32_t Tk = warp_kth_key<4>(ck, knn, lo_k, hi_k);
    // a row with a pair equal to Tk outside the candidates?
    bool outside = false;
    if (live) {
      const int jb = knn / (lane + 1);
      if (jb < knn) outside = ScoreT<T>::key_of(ScoreT<T>::round(v1 + sh_v2[warp][jb])) == Tk;
    }
    uint32_t my_slot;
    float my_val;
    if (__any_sync(0xffffffffu, outside)) {
      stage2_merge<T>(v1, i1, sh_i2[warp], sh_v2[warp], knn, n, my_slot, my_val);
    } else {
      int gt = 0, eq = 0;
      uint32_t sel = 0, tie = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const bool v = (cvalid >> t) & 1u;
        if (v && ck[t] > Tk) {
          sel |= 1u << t;
          ++gt;
        }
        if (v && ck[t] == Tk) {
          tie |= 1u << t;
          ++eq;
        }
      }
      const int need = knn - __reduce_add_sync(0xffffffffu, gt);
      if (__reduce_add_sync(0xffffffffu, eq) == need) {
        sel |= tie;
      } else {
        // the `need` lowest slots among the tied pairs
        for (int q = 0; q < need; ++q) {
          uint32_t mine = 0xffffffffu;
#pragma unroll
          for (int t = 0; t < 4; ++t)
            if ((tie >> t) & 1u) mine = min(mine, cs[t]);
          const uint32_t m = __reduce_min_sync(0xffffffffu, mine);
#pragma unroll
          for (int t = 0; t < 4; ++t)
            if (((tie >> t) & 1u) && cs[t] == m) {
              tie &= ~(1u << t);
              sel |= 1u << t;
            }
        }
      }
      int pos = warp_excl_prefix(__popc(sel));
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        if ((sel >> t) & 1u) {
          s_key[pos] = ck[t];
          s_idx[pos] = cs[t];
          sh_v1[warp][pos] = cv[t];  // the stage-1 values are no longer needed
          ++pos;
        }
      }
      // each pair's rank among the knn (sum descending, slot ascending; the
      // slots are distinct) is its place in the output: one 64-bit compare
      // per pair of composites key << 32 | ~slot (padding 0 ranks last)
      __syncwarp();  // the compacted pairs are visible to every lane
      const uint32_t ok = live ? s_key[lane] : 0u, os = live ? s_idx[lane] : 0xffffffffu;
      const float ov = live ? sh_v1[warp][lane] : -INFINITY;
      const unsigned long long mine = ((unsigned long long)ok << 32) | (uint32_t)~os;
      __syncwarp();
      s_comp64[lane] = live ? mine : 0ull;
      __syncwarp();
      int rk = 0;
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const ulonglong2 cq = *reinterpret_cast<const ulonglong2*>(s_comp64 + i);
        rk += (cq.x > mine) + (cq.y > mine);
      }
      if (live) {
        s_idx[rk] = os;
        sh_v1[warp][rk] = ov;
      }
      __syncwarp();
      my_slot = live ? s_idx[lane] : 0xffffffffu;
      my_val = live ? sh_v1[warp][lane] : -INFINITY;
      __syncwarp();
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
    __syncwarp();
  }
}

template <typename T>
static int launch_topk(const void* scores, int64_t rows, int64_t n, int64_t knn, int64_t* idx, void* ts, void* psw,
                       int64_t* s1, int64_t* s2, cudaStream_t st) {
  const int64_t want = (rows + kTopkWarps - 1) / kTopkWarps;
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)num_sms() * 8));
  const T* sc = static_cast<const T*>(scores);
  T* o = static_cast<T*>(ts);
  T* pw = static_cast<T*>(psw);
  const int ni = (int)n, ki = (int)knn;
  const bool vec_ok = aligned16(scores);  // 16-byte loads of whole rows
#define PKM_TOPK_CASE(E)                                                                                          \
  if (n <= 32 * (E)) {                                                                                            \
    product_topk_kernel<T, E><<<blocks, kTopkWarps * 32, 0, st>>>(sc, rows, ni, ki, idx, o, pw, s1, s2, vec_ok); \
    return check_cuda("product_topk_kernel");                                                                     \
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
  // a slot outside [0, n^2) has no sub-keys to credit
  const bool in_range = slot >= 0 && slot < (int64_t)n * n;
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
    const bool use = live && in_range;
    const int key = use ? (int)(half ? slot % n : slot / n) : n + lane;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    if (use && lane == __ffs(peers) - 1) {
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
