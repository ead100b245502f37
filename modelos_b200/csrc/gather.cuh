// Row-gather engine of the embedding-bag forward (K3) and its
// double-backward (K5); the backward's segment pass (K4) is in seg.cuh.
//
// One warp owns a contiguous range of bags.  The bags' entries form one
// contiguous stream; each entry names a source row, a weight and a position
// for an optional per-entry dot product.  Source rows stream through a
// per-warp ring of shared-memory slots: lane 0 issues one cp.async.bulk per
// row, `slots` entries ahead of the consumer, and each slot's mbarrier flips
// when the bytes land.  The whole warp then accumulates weight * row into
// fp32 registers (lane l owns 16-byte vectors l, l+32, ...; pairs of
// elements are accumulated with the packed fma.rn.f32x2) in entry order, so
// every output row is summed in a fixed, deterministic order, and reduces
// <row, dot_vector> across the warp when a dot output is requested.
//
// Entry metadata (row id, weight, dot position) is staged through a 64-entry
// shared ring filled one 32-entry page ahead from registers loaded another
// page earlier; the per-bag dot vector is loaded into registers one bag
// ahead.
#pragma once

#include "common.cuh"

namespace pkm {

enum { G_BAG = 0, G_SEG = 1 };
constexpr int kMaxShards = 8;  // ranks of one NVLink domain
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
  const int32_t* src_of;  // seg mode, optional: source row of each occurrence (else occurrence / L)
  int64_t n_src;          // with src_of: number of source rows
  int64_t row_lo, row_hi;  // seg mode: only the items of table rows [row_lo, row_hi) (row_hi <= row_lo: all)
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
  // segment mode, data-parallel: row r's gradient goes to rank r / shard_rows,
  // at row (shard_rank * shard_rows + r % shard_rows) of that rank's receive
  // buffer shard_base[r / shard_rows] (peer memory); shard_rows == 0: `out`
  int64_t shard_rows;
  int shard_rank;
  char* shard_base[kMaxShards];
};

// ---------------------------------------------------------------------------
// packed fp32 pairs
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t pack2(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t r, float& lo, float& hi) {
  uint32_t a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(a), "=r"(b) : "l"(r));
  lo = __uint_as_float(a);
  hi = __uint_as_float(b);
}
// acc = a * b + acc on both halves, each rounded like fmaf
__device__ __forceinline__ void ffma2(uint64_t& acc, uint64_t a, uint64_t b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}

template <typename T>
struct Pairs;
template <>
struct Pairs<float> {
  static constexpr int NP = 2;  // fp32 pairs per 16-byte vector
  __device__ static __forceinline__ void unpack(const uint4& v, uint64_t* p) {
    p[0] = pack2(v.x, v.y);
    p[1] = pack2(v.z, v.w);
  }
};
template <>
struct Pairs<__nv_bfloat16> {
  static constexpr int NP = 4;
  __device__ static __forceinline__ void unpack(const uint4& v, uint64_t* p) {
    p[0] = pack2(v.x << 16, v.x & 0xffff0000u);
    p[1] = pack2(v.y << 16, v.y & 0xffff0000u);
    p[2] = pack2(v.z << 16, v.z & 0xffff0000u);
    p[3] = pack2(v.w << 16, v.w & 0xffff0000u);
  }
};
template <>
struct Pairs<__half> {
  static constexpr int NP = 4;
  __device__ static __forceinline__ void unpack(const uint4& v, uint64_t* p) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __half22float2(h[i]);
      p[i] = pack2(__float_as_uint(t.x), __float_as_uint(t.y));
    }
  }
};

// ---------------------------------------------------------------------------
// metadata pages
// ---------------------------------------------------------------------------
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
                                              int64_t E1, int2* m_sp, float* m_w, int mi) {
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
  m_sp[mi] = make_int2(src, pos);
  m_w[mi] = w;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <typename RowT, int VPL, int MODE, bool DOT, int NW, bool FULL>
__global__ void __launch_bounds__(NW * 32, 1) gather_kernel(const GatherArgs a) {
  constexpr int NP = Pairs<RowT>::NP;
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int P = a.slots;
  const int64_t RB = a.row_bytes;

  // per-warp shared layout: ring | meta | item descs | barriers
  unsigned char* wbase = smem + warp * a.warp_smem;
  unsigned char* ring = wbase;
  const int64_t ring_bytes = ((int64_t)P * RB + 127) & ~(int64_t)127;
  int2* m_sp = reinterpret_cast<int2*>(wbase + ring_bytes);
  float* m_w = reinterpret_cast<float*>(m_sp + kMetaRing);
  int4* m_items = reinterpret_cast<int4*>(m_w + kMetaRing);
  uint64_t* bars = reinterpret_cast<uint64_t*>(m_items + (MODE == G_SEG ? kMetaRing : 0));

  const int64_t nw = (int64_t)gridDim.x * NW;
  const int64_t gw = (int64_t)blockIdx.x * NW + warp;
  const int64_t n_items = (MODE == G_BAG) ? a.n_items : (int64_t)(*a.n_items_dev);
  const int64_t i0 = n_items * gw / nw;
  const int64_t i1 = n_items * (gw + 1) / nw;
  if (i0 >= i1) return;  // warp-uniform; no block-wide barrier follows
  const int64_t ni = i1 - i0;

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
  // entry metadata pages 0 and 1; registers hold page 2
  {
    GatherPrefetch p0 = gather_prefetch<MODE>(a, E0 + lane, E1);
    GatherPrefetch p1 = gather_prefetch<MODE>(a, E0 + 32 + lane, E1);
    gather_commit<MODE>(a, p0, E0 + lane, E1, m_sp, m_w, lane);
    gather_commit<MODE>(a, p1, E0 + 32 + lane, E1, m_sp, m_w, 32 + lane);
  }
  GatherPrefetch pf = gather_prefetch<MODE>(a, E0 + 64 + lane, E1);
  // item descriptor pages (segment mode)
  int4 ipf = make_int4(0, 0, 0, -1);
  if (MODE == G_SEG) {
    m_items[lane] = lane < ni ? a.item_desc[i0 + lane] : make_int4(0, 0, 0, -1);
    m_items[32 + lane] = 32 + lane < ni ? a.item_desc[i0 + 32 + lane] : make_int4(0, 0, 0, -1);
    if (64 + lane < ni) ipf = a.item_desc[i0 + 64 + lane];
  }
  __syncwarp();

  // issue the entry whose metadata sits at ring index mi into slot s
  auto issue = [&](int s, int mi) {
    const int32_t src = m_sp[mi].x;
    if (src >= 0) {
      mbar_arrive_expect_tx(&bars[s], (uint32_t)RB);
      bulk_g2s(ring + (int64_t)s * RB, a.rows + (int64_t)src * RB, (uint32_t)RB, &bars[s]);
    } else {
      mbar_arrive(&bars[s]);
    }
  };
  if (lane == 0) {
    for (int r = 0; r < P && E0 + r < E1; ++r) issue(r, r & (kMetaRing - 1));
  }

  // the dot vector of the next item is prefetched into registers (bag mode:
  // the bag's upstream-gradient row; segment mode: the item's table row)
  uint4 dv_raw_nxt[VPL];
  auto fetch_dv = [&](int64_t j, uint4 (&raw)[VPL]) {
    const int64_t r = (MODE == G_BAG) ? i0 + j : (int64_t)m_items[j & (kMetaRing - 1)].x;
    const char* row = a.dotvec + r * RB;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int64_t off = (int64_t)(v * 32 + lane) * 16;
      raw[v] = (FULL || off < RB) ? *reinterpret_cast<const uint4*>(row + off) : make_uint4(0, 0, 0, 0);
    }
  };
  if (DOT) fetch_dv(0, dv_raw_nxt);

  int64_t e = E0;
  int32_t rel = 0;  // consumer position relative to E0
  int cs = 0;       // consumer slot
  uint32_t cpar = 0;
  bool failed = false;
  for (int64_t j = 0; j < ni && !failed; ++j) {
    const int64_t it = i0 + j;
    int64_t ee, out_row;
    int pslot = -1;
    if (MODE == G_BAG) {
      ee = (it + 1) * a.L;
      out_row = it;
    } else {
      const int4 d = m_items[j & (kMetaRing - 1)];
      ee = d.z;
      out_row = d.x;
      pslot = d.w;
    }
    uint64_t dv[VPL][NP];
    if (DOT) {
#pragma unroll
      for (int v = 0; v < VPL; ++v) Pairs<RowT>::unpack(dv_raw_nxt[v], dv[v]);
      if (j + 1 < ni) fetch_dv(j + 1, dv_raw_nxt);
    }
    uint64_t acc[VPL][NP];
#pragma unroll
    for (int v = 0; v < VPL; ++v)
#pragma unroll
      for (int t = 0; t < NP; ++t) acc[v][t] = 0ull;

    // entries are consumed two at a time where the item allows: the two rows'
    // loads and FMAs interleave, and their two dot products share one
    // butterfly reduction
    while (e < ee) {
      const bool two = e + 1 < ee;
      const int cs1 = (cs + 1 == P) ? 0 : cs + 1;
      const uint32_t cpar1 = (cs + 1 == P) ? (cpar ^ 1u) : cpar;
      const int mi0 = rel & (kMetaRing - 1);
      const int mi1 = (rel + 1) & (kMetaRing - 1);
      const int2 sp0 = m_sp[mi0];
      const float w0 = m_w[mi0];
      int2 sp1 = make_int2(-1, -1);
      float w1 = 0.f;
      if (two) {
        sp1 = m_sp[mi1];
        w1 = m_w[mi1];
      }
      if (!mbar_wait(&bars[cs], cpar, a.err) || (two && !mbar_wait(&bars[cs1], cpar1, a.err))) {
        failed = true;
        break;
      }
      uint64_t ds0[VPL], ds1[VPL];  // per-vector partial dots: short dependency chains
      const unsigned char* slot0 = ring + (int64_t)cs * RB;
      const unsigned char* slot1 = ring + (int64_t)cs1 * RB;
      const uint64_t w20 = pack2(__float_as_uint(w0), __float_as_uint(w0));
      const uint64_t w21 = pack2(__float_as_uint(w1), __float_as_uint(w1));
#pragma unroll
      for (int v = 0; v < VPL; ++v) {
        ds0[v] = 0ull;
        ds1[v] = 0ull;
        const int64_t off = (int64_t)(v * 32 + lane) * 16;
        if (FULL || off < RB) {
          uint64_t f0[NP], f1[NP];
          if (sp0.x >= 0) Pairs<RowT>::unpack(*reinterpret_cast<const uint4*>(slot0 + off), f0);
          if (sp1.x >= 0) Pairs<RowT>::unpack(*reinterpret_cast<const uint4*>(slot1 + off), f1);
          if (sp0.x >= 0) {
#pragma unroll
            for (int t = 0; t < NP; ++t) {
              ffma2(acc[v][t], w20, f0[t]);
              if (DOT) ffma2(ds0[v], dv[v][t], f0[t]);
            }
          }
          if (sp1.x >= 0) {
#pragma unroll
            for (int t = 0; t < NP; ++t) {
              ffma2(acc[v][t], w21, f1[t]);
              if (DOT) ffma2(ds1[v], dv[v][t], f1[t]);
            }
          }
        }
      }
      if (DOT && a.dotout != nullptr) {
        float d0 = 0.f, d1 = 0.f;
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
          float a0, a1, b0, b1;
          unpack2(ds0[v], a0, a1);
          unpack2(ds1[v], b0, b1);
          d0 += a0 + a1;
          d1 += b0 + b1;
        }
        if (two) {
          // lanes 0-15 reduce entry e, lanes 16-31 entry e+1
          const bool hi = (lane & 16) != 0;
          float keep = hi ? d1 : d0;
          keep += __shfl_xor_sync(0xffffffffu, hi ? d0 : d1, 16);
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
          if (lane == 0) st_f(a.dotout, a.dotout_dtype, sp0.y, sp0.x >= 0 ? keep : 0.f);
          if (lane == 16) st_f(a.dotout, a.dotout_dtype, sp1.y, sp1.x >= 0 ? keep : 0.f);
        } else {
          const float dt = warp_sum(d0);
          if (lane == 0) st_f(a.dotout, a.dotout_dtype, sp0.y, sp0.x >= 0 ? dt : 0.f);
        }
      }
      // every lane has read the slots (the values are in registers) before
      // they are refilled
      __syncwarp();
      int64_t done_page = -1;  // a metadata page whose last entry was just consumed
      if ((rel & 31) == 31)
        done_page = rel >> 5;
      else if (two && ((rel + 1) & 31) == 31)
        done_page = (rel + 1) >> 5;
      if (done_page >= 0) {
        // its ring half now receives page done_page + 2
        const int64_t e2 = E0 + (done_page + 2) * 32 + lane;
        gather_commit<MODE>(a, pf, e2, E1, m_sp, m_w, (int)((e2 - E0) & (kMetaRing - 1)));
        pf = gather_prefetch<MODE>(a, E0 + (done_page + 3) * 32 + lane, E1);
        __syncwarp();
      }
      if (lane == 0) {
        if (e + P < E1) issue(cs, (rel + P) & (kMetaRing - 1));
        if (two && e + 1 + P < E1) issue(cs1, (rel + 1 + P) & (kMetaRing - 1));
      }
      const int adv = two ? 2 : 1;
      e += adv;
      rel += adv;
      cs += adv;
      if (cs >= P) {
        cs -= P;
        cpar ^= 1u;
      }
    }
    if (failed) break;

    // write the item's row
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int64_t c = (int64_t)(v * 32 + lane);
      if (FULL || c * 16 < RB) {
        float o[2 * NP];
#pragma unroll
        for (int t = 0; t < NP; ++t) unpack2(acc[v][t], o[2 * t], o[2 * t + 1]);
        const int64_t e0 = c * (2 * NP);
        if (MODE == G_SEG && pslot >= 0) {
          st_run(a.partials, PKM_DT_F32, (int64_t)pslot * a.dim + e0, o, 2 * NP);
        } else {
          st_run(a.out, a.out_dtype, out_row * a.dim + e0, o, 2 * NP);
        }
      }
    }
    if (MODE == G_SEG && (j & 31) == 31) {
      // item page j/32 is done: its half receives page j/32 + 2
      const int64_t ip = j >> 5;
      m_items[((ip + 2) * 32 + lane) & (kMetaRing - 1)] = ipf;
      ipf = make_int4(0, 0, 0, -1);
      if ((ip + 3) * 32 + lane < ni) ipf = a.item_desc[i0 + (ip + 3) * 32 + lane];
      __syncwarp();
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
int gather_launch(int row_dtype, bool seg, bool dot, GatherArgs a, int64_t items_upper, cudaStream_t stream);

}  // namespace pkm
