// Segment pass of the embedding-bag backward (K4), direct-load form.
//
// After the radix sort, the occurrences of every table row are contiguous
// and split into items of at most 256 occurrences (one row, a range of the
// sorted list, and a partial-row slot when the row spans several items).
// One warp owns a contiguous range of items and walks their occurrences in
// order.  Each lane copies its own 16-byte vectors (lane l owns vectors l,
// l+32, ...) of the bag's upstream-gradient row into a per-warp shared ring
// with cp.async, DEPTH occurrences ahead of the one it accumulates, and reads
// back only what it copied, so completion is a per-thread wait_group and
// the loop needs no barrier and no producer lane.  The upstream-gradient rows
// are small ([n_bags, D], tens of MiB) and re-read about L times from L2,
// where they stay: everything else the pass touches is read or written with
// an L2 evict-first policy.  The table row of
// the item (the vector of the per-sample-weight dot products) is loaded into
// registers once per item, one item ahead, with evict-first, and the gradient
// row written at the item's end is stored evict-first: the table and its
// gradient stream through HBM once each.
//
// Per occurrence: dW_row += w * g_bag with packed fma.rn.f32x2 (fp32, in
// occurrence order: deterministic), and the lane's share of <g_bag, W_row>.
// The 32 dots of a metadata page are reduced together through a shared
// 32x33 transpose (one row per occurrence, summed in lane order), so each
// occurrence costs one shared store instead of a butterfly.
//
// Reference: the segment loop of `embedding_bag_bw_rev_indices`
// (pkm/xformer_embeddingbag.py:293-329), which sums a row's occurrences with
// one program per row and an fp32 accumulator.
#pragma once

#include "gather.cuh"

namespace pkm {

// L2 cache policy (createpolicy, sm_80+): lines loaded or stored with it are
// the first to be evicted, so streamed data does not displace reused data.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint4 ld_nc_hint(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ void st_hint(void* p, const uint4& v, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.v4.u32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w), "l"(pol)
               : "memory");
}

// Store 2*NP fp32 values (NP packed pairs) as dtype dt at element e0 of p.
// The vectors here are 16-byte aligned (whole rows of 16-byte multiples).
template <int NP>
__device__ __forceinline__ void seg_store_vec(void* p, int dt, int64_t e0, const uint64_t (&acc)[NP],
                                              uint64_t pol) {
  float o[2 * NP];
#pragma unroll
  for (int t = 0; t < NP; ++t) unpack2(acc[t], o[2 * t], o[2 * t + 1]);
  if (dt == PKM_DT_BF16 && NP == 4) {
    uint4 v;
    __nv_bfloat162 h;
    h = __floats2bfloat162_rn(o[0], o[1]);
    v.x = *reinterpret_cast<uint32_t*>(&h);
    h = __floats2bfloat162_rn(o[2], o[3]);
    v.y = *reinterpret_cast<uint32_t*>(&h);
    h = __floats2bfloat162_rn(o[4], o[5]);
    v.z = *reinterpret_cast<uint32_t*>(&h);
    h = __floats2bfloat162_rn(o[6], o[7]);
    v.w = *reinterpret_cast<uint32_t*>(&h);
    st_hint(static_cast<__nv_bfloat16*>(p) + e0, v, pol);
  } else if (dt == PKM_DT_F32 && NP == 2) {
    st_hint(static_cast<float*>(p) + e0,
            make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]), __float_as_uint(o[3])),
            pol);
  } else {
    st_run(p, dt, e0, o, 2 * NP);
  }
}

// Per-lane asynchronous 16-byte copies global -> shared (L2 only), grouped
// per occurrence; each lane later reads back exactly the vectors it copied,
// so completion is tracked per thread with wait_group and no warp barrier.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Shared-memory bytes of one warp of the segment pass.
__host__ __device__ constexpr int64_t seg_warp_smem(int64_t rb, int depth, bool dot) {
  return ((depth * rb + 127) & ~(int64_t)127) + kMetaRing * (8 + 4 + 16) + (dot ? 32 * 33 * 4 : 0);
}

template <typename RowT, int VPL, bool DOT, int NW, bool FULL, int DEPTH>
__global__ void __launch_bounds__(NW * 32, 1) seg_direct_kernel(const GatherArgs a) {
  static_assert(DEPTH >= 2 && DEPTH <= 8, "at most 8 copy groups in flight per thread");
  constexpr int NP = Pairs<RowT>::NP;
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t RB = a.row_bytes;
  unsigned char* wbase = smem + warp * a.warp_smem;
  unsigned char* ring = wbase;
  int2* m_sp = reinterpret_cast<int2*>(wbase + ((DEPTH * RB + 127) & ~(int64_t)127));  // {bag, occurrence}
  float* m_w = reinterpret_cast<float*>(m_sp + kMetaRing);
  int4* m_items = reinterpret_cast<int4*>(m_w + kMetaRing);
  float(*m_dot)[33] = reinterpret_cast<float(*)[33]>(m_items + kMetaRing);

  const int64_t nw = (int64_t)gridDim.x * NW;
  const int64_t gw = (int64_t)blockIdx.x * NW + warp;
  const int64_t n_items = (int64_t)(*a.n_items_dev);
  const int64_t i0 = n_items * gw / nw;
  const int64_t i1 = n_items * (gw + 1) / nw;
  if (i0 >= i1) return;  // warp-uniform; the block has no barrier
  const int64_t ni = i1 - i0;
  const int64_t E0 = a.item_desc[i0].y;
  const int64_t NE = (int64_t)a.item_desc[i1 - 1].z - E0;

  const uint64_t stream = l2_policy_evict_first();

  // metadata pages 0 and 1 in shared memory, page 2 in registers
  {
    GatherPrefetch p0 = gather_prefetch<G_SEG>(a, E0 + lane, E0 + NE);
    GatherPrefetch p1 = gather_prefetch<G_SEG>(a, E0 + 32 + lane, E0 + NE);
    gather_commit<G_SEG>(a, p0, E0 + lane, E0 + NE, m_sp, m_w, lane);
    gather_commit<G_SEG>(a, p1, E0 + 32 + lane, E0 + NE, m_sp, m_w, 32 + lane);
  }
  GatherPrefetch pf = gather_prefetch<G_SEG>(a, E0 + 64 + lane, E0 + NE);
  m_items[lane] = lane < ni ? a.item_desc[i0 + lane] : make_int4(0, 0, 0, -1);
  m_items[32 + lane] = 32 + lane < ni ? a.item_desc[i0 + 32 + lane] : make_int4(0, 0, 0, -1);
  int4 ipf = (64 + lane < ni) ? a.item_desc[i0 + 64 + lane] : make_int4(0, 0, 0, -1);
  __syncwarp();

  // copy this lane's vectors of entry `rel` into ring slot `slot` (= rel mod
  // DEPTH); one group per entry (empty past the end) keeps the group count
  // uniform
  const int rb = (int)RB;
  auto issue = [&](int64_t rel, int slot) {
    if (rel < NE) {
      const int32_t bag = m_sp[rel & (kMetaRing - 1)].x;
      if (bag >= 0 && bag < a.num_rows) {
        const char* src = a.rows + (int64_t)bag * RB;
        unsigned char* dst = ring + slot * rb;
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
          const int off = (v * 32 + lane) * 16;
          if (FULL || off < RB) cp_async16(dst + off, src + off);
        }
      } else {
        raise_err(a.err, PKM_DEVERR_INDEX);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int k = 0; k < DEPTH; ++k) issue(k, k);

  auto load_row = [&](const char* base, uint4 (&r)[VPL], uint64_t pol) {
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int off = (v * 32 + lane) * 16;
      r[v] = (FULL || off < RB) ? ld_nc_hint(base + off, pol) : make_uint4(0, 0, 0, 0);
    }
  };

  // item state
  int64_t j = 0;         // current item (relative)
  int64_t item_end = 0;  // its end (relative entry index)
  int4 cur = make_int4(0, 0, 0, -1);
  uint64_t acc[VPL][NP];
  uint64_t dv[VPL][NP];
  uint4 dv_raw[VPL];
  int64_t dv_item = -1;  // item whose table row sits in dv_raw
  if (DOT) {
    load_row(a.dotvec + (int64_t)m_items[0].x * RB, dv_raw, stream);
    dv_item = 0;
  }

  auto write_row = [&](const int4& d, const uint64_t (&row)[VPL][NP]) {
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int64_t c = (int64_t)(v * 32 + lane);
      if (FULL || c * 16 < RB) {
        const int64_t e0 = c * (2 * NP);
        if (d.w >= 0)
          seg_store_vec<NP>(a.partials, PKM_DT_F32, (int64_t)d.w * a.dim + e0, row[v], stream);
        else
          seg_store_vec<NP>(a.out, a.out_dtype, (int64_t)d.x * a.dim + e0, row[v], stream);
      }
    }
  };
  // item page bookkeeping after item j is finished
  auto item_done = [&]() {
    if ((j & 31) == 31) {
      const int64_t ip = j >> 5;
      __syncwarp();
      m_items[((ip + 2) * 32 + lane) & (kMetaRing - 1)] = ipf;
      ipf = make_int4(0, 0, 0, -1);
      if ((ip + 3) * 32 + lane < ni) ipf = a.item_desc[i0 + (ip + 3) * 32 + lane];
      __syncwarp();
    }
    ++j;
  };
  // open the next item that has entries, writing zero rows for empty ones
  auto open_item = [&]() {
#pragma unroll
    for (int v = 0; v < VPL; ++v)
#pragma unroll
      for (int t = 0; t < NP; ++t) acc[v][t] = 0ull;
    while (j < ni) {
      cur = m_items[j & (kMetaRing - 1)];
      if (cur.z > cur.y) break;
      write_row(cur, acc);
      item_done();
    }
    if (j >= ni) return;
    item_end = (int64_t)cur.z - E0;
    if (DOT) {
      if (dv_item != j) load_row(a.dotvec + (int64_t)cur.x * RB, dv_raw, stream);
#pragma unroll
      for (int v = 0; v < VPL; ++v) Pairs<RowT>::unpack(dv_raw[v], dv[v]);
      // the next item's table row, one item ahead
      if (j + 1 < ni) {
        load_row(a.dotvec + (int64_t)m_items[(j + 1) & (kMetaRing - 1)].x * RB, dv_raw, stream);
        dv_item = j + 1;
      }
    }
  };

  open_item();
  int cslot = 0;  // ring slot of entry rel
#pragma unroll 1
  for (int64_t rel = 0; rel < NE; ++rel) {
    if (rel == item_end) {
      write_row(cur, acc);
      item_done();
      open_item();
    }
    cp_async_wait<DEPTH - 1>();  // this lane's copies of entry rel have landed
    const unsigned char* slot = ring + cslot * rb;
    const float w = m_w[rel & (kMetaRing - 1)];
    const uint64_t w2 = pack2(__float_as_uint(w), __float_as_uint(w));
    uint64_t ds[VPL];
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      ds[v] = 0ull;
      const int off = (v * 32 + lane) * 16;
      if (FULL || off < RB) {
        uint64_t f[NP];
        Pairs<RowT>::unpack(*reinterpret_cast<const uint4*>(slot + off), f);
#pragma unroll
        for (int t = 0; t < NP; ++t) {
          ffma2(acc[v][t], w2, f[t]);
          if (DOT) ffma2(ds[v], dv[v][t], f[t]);
        }
      }
    }
    issue(rel + DEPTH, cslot);  // the slot's values are in registers now
    cslot = cslot + 1 == DEPTH ? 0 : cslot + 1;
    if (DOT) {
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int v = 0; v < VPL; ++v) {
        float x0, x1;
        unpack2(ds[v], x0, x1);
        d0 += x0;
        d1 += x1;
      }
      m_dot[rel & 31][lane] = d0 + d1;
    }
    if ((rel & 31) == 31 || rel + 1 == NE) {
      __syncwarp();
      if (DOT) {
        // the page's dots: row r of the transpose is entry r's lane partials
        const int64_t first = rel & ~(int64_t)31;
        if (lane <= (int)(rel - first)) {
          float s = 0.f;
#pragma unroll 8
          for (int l = 0; l < 32; ++l) s += m_dot[lane][l];
          st_f(a.dotout, a.dotout_dtype, m_sp[(first + lane) & (kMetaRing - 1)].y, s);
        }
        __syncwarp();
      }
      if ((rel & 31) == 31) {
        // metadata page rel/32 is consumed: its half receives page rel/32 + 2
        const int64_t page = rel >> 5;
        const int64_t e2 = E0 + (page + 2) * 32 + lane;
        gather_commit<G_SEG>(a, pf, e2, E0 + NE, m_sp, m_w, (int)((e2 - E0) & (kMetaRing - 1)));
        pf = gather_prefetch<G_SEG>(a, E0 + (page + 3) * 32 + lane, E0 + NE);
        __syncwarp();
      }
    }
  }
  cp_async_wait<0>();
  // the last item with entries, then any empty items after it
  if (j < ni) {
    write_row(cur, acc);
    item_done();
  }
  open_item();
}

}  // namespace pkm
