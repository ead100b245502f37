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

#include <type_traits>

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

__device__ __forceinline__ void st_plain(void* p, const uint4& v) { *reinterpret_cast<uint4*>(p) = v; }

// Store 2*NP fp32 values (NP packed pairs) as dtype dt at element e0 of p,
// with the L2 evict-first policy `pol` (local memory) or a plain store
// (peer memory, pol == 0).  The vectors here are 16-byte aligned.
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
    if (pol)
      st_hint(static_cast<__nv_bfloat16*>(p) + e0, v, pol);
    else
      st_plain(static_cast<__nv_bfloat16*>(p) + e0, v);
  } else if (dt == PKM_DT_F32 && NP == 2) {
    const uint4 v =
        make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]), __float_as_uint(o[3]));
    if (pol)
      st_hint(static_cast<float*>(p) + e0, v, pol);
    else
      st_plain(static_cast<float*>(p) + e0, v);
  } else {
    st_run(p, dt, e0, o, 2 * NP);
  }
}

// Per-lane asynchronous 16-byte copies global -> shared (L2 only), grouped
// per occurrence; each lane later reads back exactly the vectors it copied,
// so completion is tracked per thread with wait_group and no warp barrier.
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// f(std::integral_constant<int, i>{}) for i = 0 .. N-1, unrolled at compile
// time (immediate address offsets in inline PTX need constants).
template <int I, int N>
struct StaticFor {
  template <class F>
  __device__ __forceinline__ static void run(F&& f) {
    f(std::integral_constant<int, I>{});
    StaticFor<I + 1, N>::run(f);
  }
};
template <int N>
struct StaticFor<N, N> {
  template <class F>
  __device__ __forceinline__ static void run(F&&) {}
};

// Shared-memory bytes of one warp of the segment pass.
__host__ __device__ constexpr int64_t seg_warp_smem(int64_t rb, int depth, bool dot) {
  return ((depth * rb + 127) & ~(int64_t)127) + kMetaRing * (8 + 4 + 16) + (dot ? 32 * 33 * 4 : 0);
}

template <typename RowT, int VPL, bool DOT, int NW, bool FULL, int DEPTH>
__global__ void __launch_bounds__(NW * 32, 1) seg_direct_kernel(const __grid_constant__ GatherArgs a) {
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
  int64_t it_lo = 0, it_hi = (int64_t)(*a.n_items_dev);
  if (a.row_hi > a.row_lo) {
    // the items (sorted by row) of rows [row_lo, row_hi): two lower bounds
    auto lower = [&](int64_t row) {
      int64_t lo = 0, hi = it_hi;
      while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if ((int64_t)a.item_desc[mid].x < row)
          lo = mid + 1;
        else
          hi = mid;
      }
      return lo;
    };
    const int64_t b = lower(a.row_lo), e = lower(a.row_hi);
    it_lo = b;
    it_hi = e;
  }
  const int64_t n_items = it_hi - it_lo;
  const int64_t i0 = it_lo + n_items * gw / nw;
  const int64_t i1 = it_lo + n_items * (gw + 1) / nw;
  if (i0 >= i1) return;  // warp-uniform; the block has no barrier
  const int ni = (int)(i1 - i0);
  const int64_t E0 = a.item_desc[i0].y;
  const int NE = (int)((int64_t)a.item_desc[i1 - 1].z - E0);  // < 2^31: checked on the host
  const uint32_t L = (uint32_t)a.L;
  const uint32_t n_occ = (uint32_t)(a.num_rows * a.L);

  const uint64_t stream = l2_policy_evict_first();

  // entry metadata: {bag, occurrence} and weight; an occurrence id outside
  // [0, n_bags * L) is reported and read as bag 0 (never out of bounds)
  auto fetch_meta = [&](int e, int32_t& occ, float& w) {
    occ = -1;
    w = 0.f;
    if (e < NE) {
      occ = a.occ[E0 + e];
      w = a.occ_w[E0 + e];
    }
  };
  auto commit_meta = [&](int e, int32_t occ, float w) {
    int32_t bag = 0;
    if (e < NE) {
      if ((uint32_t)occ < n_occ) {
        if (a.src_of) {
          bag = a.src_of[occ];
          if ((uint64_t)(uint32_t)bag >= (uint64_t)a.n_src) {
            raise_err(a.err, PKM_DEVERR_INDEX);
            bag = 0;
            w = 0.f;
          }
        } else {
          bag = (int32_t)((uint32_t)occ / L);
        }
      } else {
        raise_err(a.err, PKM_DEVERR_INDEX);
        occ = 0;
        w = 0.f;
      }
    }
    m_sp[e & (kMetaRing - 1)] = make_int2(bag, occ);
    m_w[e & (kMetaRing - 1)] = w;
  };
  // metadata pages 0 and 1 in shared memory, page 2 in registers
  {
    int32_t o0, o1;
    float w0, w1;
    fetch_meta(lane, o0, w0);
    fetch_meta(32 + lane, o1, w1);
    commit_meta(lane, o0, w0);
    commit_meta(32 + lane, o1, w1);
  }
  int32_t pf_occ;
  float pf_w;
  fetch_meta(64 + lane, pf_occ, pf_w);
  m_items[lane] = lane < ni ? a.item_desc[i0 + lane] : make_int4(0, 0, 0, -1);
  m_items[32 + lane] = 32 + lane < ni ? a.item_desc[i0 + 32 + lane] : make_int4(0, 0, 0, -1);
  int4 ipf = (64 + lane < ni) ? a.item_desc[i0 + 64 + lane] : make_int4(0, 0, 0, -1);
  __syncwarp();

  // this lane's 16-byte vectors: global row offset lane*16 + v*512, ring
  // offset slot*RB + lane*16 + v*512
  const int rb = (int)RB;
  const char* src_lane = a.rows + lane * 16;
  const uint32_t ring_lane = smem_u32(ring) + lane * 16;
  // copy entry e's vectors into ring slot `slot` (= e mod DEPTH); one group
  // per entry, empty past the end, keeps the group count uniform
  auto issue = [&](int e, int slot) {
    if (e < NE) {
      const char* src = src_lane + (int64_t)m_sp[e & (kMetaRing - 1)].x * RB;
      const uint32_t dst = ring_lane + slot * rb;
#pragma unroll
      for (int v = 0; v < VPL; ++v) {
        if (FULL || (v * 32 + lane) * 16 < rb)
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst + v * 512), "l"(src + v * 512)
                       : "memory");
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
      r[v] = (FULL || off < rb) ? ld_nc_hint(base + off, pol) : make_uint4(0, 0, 0, 0);
    }
  };

  // item state
  int j = 0;         // current item (relative)
  int item_end = 0;  // its end (relative entry index)
  int4 cur = make_int4(0, 0, 0, -1);
  uint64_t acc[VPL][NP];
  uint64_t dv[VPL][NP];
  uint4 dv_raw[VPL];
  int dv_item = -1;  // item whose table row sits in dv_raw
  if (DOT) {
    load_row(a.dotvec + (int64_t)m_items[0].x * RB, dv_raw, stream);
    dv_item = 0;
  }

  auto write_row = [&](const int4& d, const uint64_t (&row)[VPL][NP]) {
    // destination of a finished row: the local gradient, or the owner rank's
    // receive buffer in data-parallel mode
    void* dst = a.out;
    int64_t drow = d.x;
    uint64_t pol = stream;
    if (a.shard_rows > 0) {
      const int64_t o = d.x / a.shard_rows;
      dst = a.shard_base[o];
      drow = a.shard_rank * a.shard_rows + (d.x - o * a.shard_rows);
      pol = 0;
    }
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int64_t c = (int64_t)(v * 32 + lane);
      if (FULL || c * 16 < RB) {
        const int64_t e0 = c * (2 * NP);
        if (d.w >= 0)
          seg_store_vec<NP>(a.partials, PKM_DT_F32, (int64_t)d.w * a.dim + e0, row[v], stream);
        else
          seg_store_vec<NP>(dst, a.out_dtype, drow * a.dim + e0, row[v], pol);
      }
    }
  };
  // item page bookkeeping after item j is finished
  auto item_done = [&]() {
    if ((j & 31) == 31) {
      const int ip = j >> 5;
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
    item_end = (int)((int64_t)cur.z - E0);
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
  int cslot = 0;  // ring slot of entry e
  int e = 0;
  while (e < NE) {
    if (e == item_end) {
      write_row(cur, acc);
      item_done();
      open_item();
    }
    // a run of entries with no item or page boundary inside
    const int stop = min(min(item_end, NE), (e | 31) + 1);
    const bool all_issue = stop + DEPTH <= NE;
#pragma unroll 1
    for (; e < stop; ++e) {
      cp_async_wait<DEPTH - 1>();  // this lane's copies of entry e have landed
      const uint32_t slot = ring_lane + cslot * rb;
      const float w = m_w[e & (kMetaRing - 1)];
      const uint64_t w2 = pack2(__float_as_uint(w), __float_as_uint(w));
      uint64_t ds[VPL];  // dot accumulators, one per vector (short dependency chains)
      // the entry's vectors, at immediate offsets from the slot
      uint4 raw[VPL];
      StaticFor<0, VPL>::run([&](auto vc) {
        constexpr int v = decltype(vc)::value;
        if (FULL || (v * 32 + lane) * 16 < rb)
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4+%5];"
                       : "=r"(raw[v].x), "=r"(raw[v].y), "=r"(raw[v].z), "=r"(raw[v].w)
                       : "r"(slot), "n"(v * 512));
      });
#pragma unroll
      for (int v = 0; v < VPL; ++v) {
        ds[v] = 0ull;
        if (FULL || (v * 32 + lane) * 16 < rb) {
          uint64_t f[NP];
          Pairs<RowT>::unpack(raw[v], f);
#pragma unroll
          for (int t = 0; t < NP; ++t) {
            ffma2(acc[v][t], w2, f[t]);
            if (DOT) ffma2(ds[v], dv[v][t], f[t]);
          }
        }
      }
      // the slot's values are in registers: refill it with entry e + DEPTH
      if (all_issue) {
        const char* src = src_lane + (int64_t)m_sp[(e + DEPTH) & (kMetaRing - 1)].x * RB;
        StaticFor<0, VPL>::run([&](auto vc) {
          constexpr int v = decltype(vc)::value;
          if (FULL || (v * 32 + lane) * 16 < rb)
            asm volatile("cp.async.cg.shared.global [%0+%2], [%1+%2], 16;" ::"r"(slot), "l"(src), "n"(v * 512)
                         : "memory");
        });
        cp_async_commit();
      } else {
        issue(e + DEPTH, cslot);
      }
      cslot = cslot + 1 == DEPTH ? 0 : cslot + 1;
      if (DOT) {
        // pairwise over the vectors, then the two halves of the pair
#pragma unroll
        for (int h = 1; h < VPL; h <<= 1)
#pragma unroll
          for (int v = 0; v + h < VPL; v += 2 * h) asm("add.rn.f32x2 %0, %0, %1;" : "+l"(ds[v]) : "l"(ds[v + h]));
        float x0, x1;
        unpack2(ds[0], x0, x1);
        m_dot[e & 31][lane] = x0 + x1;
      }
    }
    if ((e & 31) == 0 || e == NE) {
      // the page of entries (e - 1) / 32 is consumed (or the stream ended)
      const int last = e - 1;
      const int first = last & ~31;
      __syncwarp();
      if (DOT) {
        // row r of the transpose holds entry r's lane partials
        if (lane <= last - first) {
          float sum = 0.f;
#pragma unroll 8
          for (int l = 0; l < 32; ++l) sum += m_dot[lane][l];
          st_f(a.dotout, a.dotout_dtype, m_sp[(first + lane) & (kMetaRing - 1)].y, sum);
        }
        __syncwarp();
      }
      if ((e & 31) == 0) {
        // its half of the metadata ring receives page last/32 + 2
        const int page = last >> 5;
        commit_meta((page + 2) * 32 + lane, pf_occ, pf_w);
        fetch_meta((page + 3) * 32 + lane, pf_occ, pf_w);
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
  // peer stores are ordered before whatever this GPU signals to its peers next
  if (a.shard_rows > 0) __threadfence_system();
}

}  // namespace pkm
