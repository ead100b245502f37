// Row-gather engine shared by the embedding-bag forward (K3), its
// double-backward (K5) and the sorted-segment backward (K4).
//
// One warp owns a contiguous range of "items" (bags, or chunks of a row's
// sorted occurrence list).  The items' entries form one contiguous stream;
// each entry names a source row, a weight and a position for an optional
// per-entry dot product.  Source rows stream through a per-warp ring of
// shared-memory slots: lane 0 issues one cp.async.bulk per row, `slots`
// entries ahead of the consumer, and each slot's mbarrier flips when the
// bytes land.  The whole warp then accumulates weight * row into fp32
// registers (lane l owns 16-byte vectors l, l+32, ...) in entry order, so
// every output row is summed in a fixed, deterministic order, and reduces
// <row, dot_vector> across the warp when a dot output is requested.
//
// Entry metadata (row id, weight, dot position) is staged through a 64-entry
// shared ring, filled one 32-entry page ahead from registers that were loaded
// another page earlier, so neither the copy issue nor the consumer waits on
// a metadata load.
#pragma once

#include "common.cuh"

namespace pkm {

enum { G_BAG = 0, G_SEG = 1 };
constexpr int kGatherWarps = 8;
constexpr int kMetaRing = 64;

struct GatherArgs {
  const char* rows;  // gathered table
  int64_t row_bytes;
  int64_t dim;
  int64_t num_rows;  // bag mode: index bound
  // entry stream
  const int64_t* idx;   // bag mode: [n_items * L]
  const void* w;        // bag mode: per-sample weights, nullable (= 1)
  int w_dtype;
  const int32_t* occ;   // seg mode: occurrence ids sorted by row
  const float* occ_w;   // seg mode: their weights (fp32)
  int64_t L;            // bag size
  // items
  int64_t n_items;             // bag mode
  const int32_t* n_items_dev;  // seg mode: item count written by an earlier kernel
  const int4* item_desc;       // seg mode: {row, entry_begin, entry_end, partial_slot or -1}
  // optional per-item dot vector and per-entry dot output
  const char* dotvec;  // bag mode: [n_items, dim]; seg mode: [num_rows, dim]
  void* dotout;
  int dotout_dtype;
  // outputs
  void* out;
  int out_dtype;
  float* partials;  // seg mode: rows of multi-chunk segments
  uint32_t* err;
  int slots;
  int64_t warp_smem;
};

struct GatherPrefetch {
  int64_t a;   // bag: index; seg: occurrence id
  uint32_t b;  // weight bits (bag: raw dtype bits; seg: fp32 bits)
};

template <int MODE>
__device__ __forceinline__ GatherPrefetch gather_prefetch(const GatherArgs& a, int64_t e, int64_t E1) {
  GatherPrefetch p{-1, 0u};
  if (e < E1) {
    if (MODE == G_BAG) {
      p.a = a.idx[e];
      if (a.w) {
        if (a.w_dtype == PKM_DT_F32)
          p.b = __float_as_uint(static_cast<const float*>(a.w)[e]);
        else
          p.b = static_cast<const uint16_t*>(a.w)[e];
      } else {
        p.b = __float_as_uint(1.0f);
      }
    } else {
      p.a = a.occ[e];
      p.b = __float_as_uint(a.occ_w[e]);
    }
  }
  return p;
}

template <int MODE>
__device__ __forceinline__ void gather_commit(const GatherArgs& a, const GatherPrefetch& p, int64_t e,
                                              int64_t E1, int32_t* m_src, float* m_w, int32_t* m_pos,
                                              int mi) {
  int32_t src = -1, pos = -1;
  float w = 0.f;
  if (e < E1) {
    if (MODE == G_BAG) {
      if (p.a < 0 || p.a >= a.num_rows) {
        raise_err(a.err, PKM_DEVERR_INDEX);
      } else {
        src = static_cast<int32_t>(p.a);
      }
      if (a.w_dtype == PKM_DT_F32 || a.w == nullptr)
        w = __uint_as_float(p.b);
      else if (a.w_dtype == PKM_DT_BF16)
        w = __uint_as_float(p.b << 16);
      else
        w = __half2float(__ushort_as_half(static_cast<unsigned short>(p.b)));
      pos = static_cast<int32_t>(e);
    } else {
      src = static_cast<int32_t>(p.a / a.L);
      w = __uint_as_float(p.b);
      pos = static_cast<int32_t>(p.a);
    }
  }
  m_src[mi] = src;
  m_w[mi] = w;
  m_pos[mi] = pos;
}

template <typename RowT, int VPL>
__device__ __forceinline__ void load_row_f(const char* row, int64_t row_bytes, int lane,
                                           float (&f)[VPL][VecTraits<RowT>::EPV]) {
  constexpr int EPV = VecTraits<RowT>::EPV;
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    const int64_t off = (int64_t)(v * 32 + lane) * 16;
    if (off < row_bytes) {
      uint4 raw = *reinterpret_cast<const uint4*>(row + off);
      VecTraits<RowT>::unpack(raw, f[v]);
    } else {
#pragma unroll
      for (int t = 0; t < EPV; ++t) f[v][t] = 0.f;
    }
  }
}

template <typename RowT, int VPL, int MODE, bool DOT>
__global__ void __launch_bounds__(kGatherWarps * 32, 1) gather_kernel(const GatherArgs a) {
  constexpr int EPV = VecTraits<RowT>::EPV;
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int P = a.slots;
  const int64_t RB = a.row_bytes;

  unsigned char* wbase = smem + warp * a.warp_smem;
  unsigned char* ring = wbase;
  const int64_t ring_bytes = ((int64_t)P * RB + 127) & ~(int64_t)127;
  int32_t* m_src = reinterpret_cast<int32_t*>(wbase + ring_bytes);
  float* m_w = reinterpret_cast<float*>(m_src + kMetaRing);
  int32_t* m_pos = reinterpret_cast<int32_t*>(m_w + kMetaRing);
  uint64_t* bars = reinterpret_cast<uint64_t*>(m_pos + kMetaRing);

  const int64_t nw = (int64_t)gridDim.x * kGatherWarps;
  const int64_t gw = (int64_t)blockIdx.x * kGatherWarps + warp;
  const int64_t n_items = (MODE == G_BAG) ? a.n_items : (int64_t)(*a.n_items_dev);
  const int64_t i0 = n_items * gw / nw;
  const int64_t i1 = n_items * (gw + 1) / nw;
  if (i0 >= i1) return;  // warp-uniform; no block-wide barrier follows

  int64_t E0, E1;
  if (MODE == G_BAG) {
    E0 = i0 * a.L;
    E1 = i1 * a.L;
  } else {
    E0 = a.item_desc[i0].y;
    E1 = a.item_desc[i1 - 1].z;
  }

  if (lane == 0) {
    for (int s = 0; s < P; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  // metadata pages 0 and 1, registers hold page 2
  {
    GatherPrefetch p0 = gather_prefetch<MODE>(a, E0 + lane, E1);
    GatherPrefetch p1 = gather_prefetch<MODE>(a, E0 + 32 + lane, E1);
    gather_commit<MODE>(a, p0, E0 + lane, E1, m_src, m_w, m_pos, lane);
    gather_commit<MODE>(a, p1, E0 + 32 + lane, E1, m_src, m_w, m_pos, 32 + lane);
  }
  GatherPrefetch pf = gather_prefetch<MODE>(a, E0 + 64 + lane, E1);
  __syncwarp();

  // issue entry `e` (metadata at ring index mi) into slot `s`
  auto issue = [&](int s, int mi, int64_t e) {
    const int32_t src = m_src[mi];
    if (src >= 0) {
      mbar_arrive_expect_tx(&bars[s], (uint32_t)RB);
      bulk_g2s(ring + (int64_t)s * RB, a.rows + (int64_t)src * RB, (uint32_t)RB, &bars[s]);
    } else {
      mbar_arrive(&bars[s]);
    }
    (void)e;
  };
  if (lane == 0) {
    for (int r = 0; r < P && E0 + r < E1; ++r) issue(r, r & (kMetaRing - 1), E0 + r);
  }

  // seg mode: item descriptors and dot vectors run ahead of the consumer
  int4 desc_cur = make_int4(0, 0, 0, -1), desc_nxt = make_int4(0, 0, 0, -1);
  if (MODE == G_SEG) {
    desc_cur = a.item_desc[i0];
    if (i0 + 1 < i1) desc_nxt = a.item_desc[i0 + 1];
  }
  uint4 dv_raw_nxt[VPL];
  auto dot_row_ptr = [&](int64_t item, const int4& d) -> const char* {
    const int64_t r = (MODE == G_BAG) ? item : (int64_t)d.x;
    return a.dotvec + r * RB;
  };
  auto fetch_dv = [&](int64_t item, const int4& d, uint4 (&raw)[VPL]) {
    const char* row = dot_row_ptr(item, d);
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int64_t off = (int64_t)(v * 32 + lane) * 16;
      raw[v] = (off < RB) ? *reinterpret_cast<const uint4*>(row + off) : make_uint4(0, 0, 0, 0);
    }
  };
  if (DOT) fetch_dv(i0, desc_cur, dv_raw_nxt);

  int64_t e = E0;
  int32_t rel = 0;  // consumer position relative to E0
  int cs = 0;       // consumer slot
  uint32_t cpar = 0;
  bool failed = false;
  for (int64_t it = i0; it < i1 && !failed; ++it) {
    int64_t ee, out_row;
    int pslot = -1;
    int4 d_this = desc_cur;
    if (MODE == G_BAG) {
      ee = (it + 1) * a.L;
      out_row = it;
    } else {
      ee = d_this.z;
      out_row = d_this.x;
      pslot = d_this.w;
      // advance the descriptor window: next item, and load the one after
      desc_cur = desc_nxt;
      if (it + 2 < i1) desc_nxt = a.item_desc[it + 2];
    }
    float dv[VPL][EPV];
    if (DOT) {
#pragma unroll
      for (int v = 0; v < VPL; ++v) VecTraits<RowT>::unpack(dv_raw_nxt[v], dv[v]);
      if (it + 1 < i1) fetch_dv(it + 1, desc_cur, dv_raw_nxt);
    }
    float acc[VPL][EPV];
#pragma unroll
    for (int v = 0; v < VPL; ++v)
#pragma unroll
      for (int t = 0; t < EPV; ++t) acc[v][t] = 0.f;

    for (; e < ee; ++e, ++rel) {
      const int mi = rel & (kMetaRing - 1);
      const int32_t src = m_src[mi];
      const float w = m_w[mi];
      const int32_t pos = m_pos[mi];
      if (!mbar_wait(&bars[cs], cpar, a.err)) {
        failed = true;
        break;
      }
      float dsum = 0.f;
      if (src >= 0) {
        const unsigned char* slot = ring + (int64_t)cs * RB;
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
          const int64_t off = (int64_t)(v * 32 + lane) * 16;
          if (off < RB) {
            uint4 raw = *reinterpret_cast<const uint4*>(slot + off);
            float f[EPV];
            VecTraits<RowT>::unpack(raw, f);
#pragma unroll
            for (int t = 0; t < EPV; ++t) {
              acc[v][t] = fmaf(w, f[t], acc[v][t]);
              if (DOT) dsum = fmaf(dv[v][t], f[t], dsum);
            }
          }
        }
      }
      if (DOT && a.dotout != nullptr) {
        dsum = warp_sum(dsum);
        if (lane == 0) st_f(a.dotout, a.dotout_dtype, pos, src >= 0 ? dsum : 0.f);
      }
      // every lane has read the slot (the values are in registers) before
      // lane 0 reuses it for the row P entries ahead
      __syncwarp();
      if (lane == 0 && e + P < E1) issue(cs, (rel + P) & (kMetaRing - 1), e + P);
      if ((rel & 31) == 31) {
        // page rel/32 is consumed: its ring half now receives page rel/32 + 2
        const int64_t page = rel >> 5;
        const int64_t e2 = E0 + (page + 2) * 32 + lane;
        gather_commit<MODE>(a, pf, e2, E1, m_src, m_w, m_pos, (int)((e2 - E0) & (kMetaRing - 1)));
        pf = gather_prefetch<MODE>(a, E0 + (page + 3) * 32 + lane, E1);
        __syncwarp();
      }
      if (++cs == P) {
        cs = 0;
        cpar ^= 1u;
      }
    }
    if (failed) break;

    // write the item's row
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int64_t c = (int64_t)(v * 32 + lane);
      if (c * 16 < RB) {
        const int64_t e0 = c * EPV;
        if (MODE == G_SEG && pslot >= 0) {
          st_run(a.partials, PKM_DT_F32, (int64_t)pslot * a.dim + e0, acc[v], EPV);
        } else {
          st_run(a.out, a.out_dtype, out_row * a.dim + e0, acc[v], EPV);
        }
      }
    }
  }

  if (failed) {
    // drain copies that may still be in flight before the warp exits
    int ds = cs;
    uint32_t dp = cpar;
    for (int64_t r = e; r < E1 && r < e + P; ++r) {
      if (!mbar_wait(&bars[ds], dp, nullptr)) break;
      if (++ds == P) {
        ds = 0;
        dp ^= 1u;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host launcher
// ---------------------------------------------------------------------------
int gather_launch(int row_dtype, bool seg, bool dot, GatherArgs a, int64_t items_upper,
                  cudaStream_t stream);

}  // namespace pkm
