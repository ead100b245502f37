// Dense bf16 GEMMs of the product-key layer on the 5th-generation tensor
// cores: the query projection, the SwiLU and value projections and their
// gradients (pkm/memory.py:143-149, 226-229, 317-349), and the dense part of
// the scoring backward (pkm/memory.py:267-268).
//
//   C[b][m, n] = sum_k A[b][m, k] * B[b][n, k]  (+ bias[n])    fp32 accumulate
//
// A and B are bf16 row-major matrices read through TMA.  Either operand may
// be stored K-major ([M, K] / [N, K], the forward projections) or MN-major
// ([K, M] / [K, N], the data and weight gradients), which the tcgen05
// instruction descriptor's transpose bits and the shared-memory descriptor's
// layout take care of, so no operand is ever transposed in memory.  A batch
// of GEMMs (the (head, half) groups of the scoring backward) is expressed as
// per-batch offsets of the TMA coordinates and of C.
//
// One persistent, warp-specialised CTA per SM computes 128 x 256 tiles:
//   warp 0    TMA producer into a 4-stage ring of 128-byte-swizzled tiles;
//   warp 1    MMA issuer: tcgen05.mma kind::f16 128x256x16 into one of two
//             256-column TMEM accumulators; tcgen05.commit frees each stage
//             and hands a finished accumulator to the epilogue;
//   warps 2-9 epilogue: two warps per TMEM lane quarter, 128 of the 256
//             columns each; tcgen05.ld of the next 32 columns in flight
//             while the current ones get their bias, rounding and 16-byte
//             stores (or fp32 partials), one output row per thread.
// GEMMs of more than 128 rows run as CTA pairs (clusters of two,
// tcgen05.mma.cta_group::2): a pair computes 256 x 256 tiles, each CTA
// stages its 128 rows of A and half of the tile's 256 rows of B (6 stages
// of 32 KiB) and holds 128 accumulator rows; rank 0's warp 1 issues the
// 256x256x16 MMAs, its commits reach the mbarriers of both CTAs, both CTAs'
// copies complete on rank 0's stage barriers, and the epilogue warps of both
// CTAs release an accumulator on rank 0's barrier.  Per output element a
// pair stages a third less operand data than two single CTAs, which is what
// bounds the single form (its operand copies, not the tensor pipe).
// When the tiles alone cannot fill the SMs (weight gradients, K = tokens),
// the K range is split over several CTAs that write fp32 partials; a second
// kernel sums them in split order (deterministic) and applies the epilogue.
// Every wait is bounded; a timeout raises PKM_DEVERR_TIMEOUT and each role
// drains its own outstanding copies / MMAs before TMEM is released.
#include <algorithm>
#include <atomic>
#include <cstring>

#include "umma.cuh"

namespace pkm {

constexpr int GM_BM = 128, GM_BN = 256, GM_BK = 64;
constexpr int GM_EPI_WARPS = 8;  // two per TMEM lane quarter, 128 columns each
constexpr int GM_THREADS = 64 + GM_EPI_WARPS * 32;
constexpr int GM_MN_BOX = 64;                   // MN-major tiles arrive as 64-wide boxes
constexpr int GM_MN_BOX_BYTES = GM_MN_BOX * GM_BK * 2;  // 8 KiB

// Tile geometry of the single-CTA form and of the CTA-pair form.  Every CTA
// holds 128 accumulator rows x 256 columns; a pair's tile is 256 x 256, each
// CTA staging its 128 rows of A and 128 of the 256 rows of B, so a pair
// stages a third less operand data per output element than two single CTAs.
template <bool PAIR>
struct GmTile {
  static constexpr int TM = PAIR ? 2 * GM_BM : GM_BM;  // tile rows
  static constexpr int BROWS = PAIR ? GM_BN / 2 : GM_BN;  // B rows staged per CTA
  static constexpr int STAGES = PAIR ? 6 : 4;
  static constexpr int A_BYTES = GM_BM * GM_BK * 2;  // 16 KiB
  static constexpr int B_BYTES = BROWS * GM_BK * 2;  // 16 or 32 KiB
  static constexpr int STAGE = A_BYTES + B_BYTES;
  // per epilogue warp, one 32-row x 128-byte box of output staged for a
  // TMA store (128-byte swizzle)
  static constexpr int STAGING = GM_EPI_WARPS * 4096;
  static constexpr int SMEM = STAGES * STAGE + STAGING + 1024 + 256;
};

struct GemmArgs {
  int M, N, K, batch;
  int a_mn, b_mn;
  int a_bx, a_by, b_bx, b_by;  // per-batch offsets of the TMA coordinates (x: columns, y: rows)
  int64_t c_bs;                // per-batch element offset of C
  int m_tiles, n_tiles, k_blocks, splits;
  int64_t units;
  void* c;
  int c_dtype;
  int64_t ldc;
  const void* bias;
  int bias_dtype;
  float* ws;  // split partials [splits][batch][M][N]
  uint32_t* err;
  uint32_t wait_limit;
  // fused SwiGLU gate (batch 1, no split, bf16): epi 1 forward, 2 backward
  int epi;
  const __nv_bfloat16* aux_a;  // the gate's other input a  [M, N], pitch ld_aux
  const __nv_bfloat16* aux_h;  // the gate projection's output h (backward)
  __nv_bfloat16* aux_out;      // z (forward) or da (backward, may be NULL)
  int64_t ld_aux;
  // st_tma: the epilogue writes whole 32-row boxes of C (or of the split
  // partials) through TMA stores, the box of split s, batch b, rows m.., and
  // columns n.. at x = b * st_bx + n, y = s * st_sy + b * st_by + m; boxes
  // that cross the edge of M or N are stored directly
  int st_tma;
  int st_bx, st_by, st_sy;
  // gt_tma: the gate epilogue moves whole 32 x 32 boxes through TMA: a (and
  // h) loaded, h / dh and z / da stored (64-byte swizzle, two 2 KiB boxes
  // per warp); boxes crossing the edge of M or N use direct accesses
  int gt_tma;
};

// Rounding to bf16 and back (each step of the gate is rounded where torch's
// eager ops round it, as the standalone gate kernels do).
__device__ __forceinline__ float rb16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// The gate on 8 consecutive columns.  Forward: h = acc + bias (the
// projection's output), s = silu(h), z = a * s.  Backward: g = acc (the
// gradient of z), da = g * s, ds = g * a, dh = ds * sig * (1 + h (1 - sig)).
// `o` receives h (forward) or dh (backward), `o2` z or da.
__device__ __forceinline__ void gate8(int epi, const float* av, const float* hv, const float* acc, float* o,
                                      float* o2) {
  if (epi == 1) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float h = rb16(acc[k]);
      o[k] = h;
      o2[k] = rb16(av[k] * rb16(h / (1.f + expf(-h))));
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float g = rb16(acc[k]);
      const float sig = 1.f / (1.f + expf(-hv[k]));
      const float sl = rb16(hv[k] / (1.f + expf(-hv[k])));
      o2[k] = rb16(g * sl);
      o[k] = rb16(rb16(g * av[k]) * sig * (1.f + hv[k] * (1.f - sig)));
    }
  }
}

// The same with a and h read from global memory.
__device__ __forceinline__ void gm_gate8(const GemmArgs& a, int64_t x0, const float* acc, float* o, float* o2) {
  float av[8], hv[8];
  VecTraits<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(a.aux_a + x0), av);
  if (a.epi == 2) VecTraits<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(a.aux_h + x0), hv);
  gate8(a.epi, av, hv, acc, o, o2);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Bounded wait; CL: an acquire at cluster scope (arrivals from the other
// CTA of a pair).
template <bool CL = false>
__device__ __forceinline__ bool gm_wait(uint64_t* bar, uint32_t parity, const GemmArgs& a, volatile int* abort_flag) {
  for (uint32_t i = 0; i < a.wait_limit; ++i) {
    if (CL ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
    if ((i & 1023) == 1023 && *abort_flag) return false;
  }
  raise_err(a.err, PKM_DEVERR_TIMEOUT);
  *abort_flag = 1;
  return false;
}

// Shared-memory descriptor of an MN-major tile stored as 64-element-wide
// boxes of GM_BK rows (128-byte swizzle): 8-row groups 1024 bytes apart
// (stride byte offset), 64-element MN blocks one box apart (leading byte
// offset).
__device__ __forceinline__ uint64_t umma_desc_mn_sw128(const void* smem) {
  const uint64_t addr = smem_u32(smem);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3fffull;
  d |= (uint64_t)(GM_MN_BOX_BYTES >> 4) << 16;  // leading byte offset
  d |= (uint64_t)(1024 >> 4) << 32;             // stride byte offset
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void gm_decode(const GemmArgs& a, int64_t u, int& b, int& mt, int& nt, int& s) {
  s = (int)(u % a.splits);
  int64_t r = u / a.splits;
  nt = (int)(r % a.n_tiles);
  r /= a.n_tiles;
  mt = (int)(r % a.m_tiles);
  b = (int)(r / a.m_tiles);
}

__device__ __forceinline__ void gm_krange(const GemmArgs& a, int s, int& kb0, int& kb1) {
  kb0 = (int)((int64_t)a.k_blocks * s / a.splits);
  kb1 = (int)((int64_t)a.k_blocks * (s + 1) / a.splits);
}

__device__ __forceinline__ float gm_bias(const GemmArgs& a, int n) {
  if (!a.bias) return 0.f;
  return ld_f(a.bias, a.bias_dtype, n);
}

// bias[n0 .. n0+31] (0 past N or without a bias), 16-byte loads where whole
__device__ __forceinline__ void gm_bias32(const GemmArgs& a, int n0, float* f) {
  if (!a.bias) {
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = 0.f;
    return;
  }
  const bool whole = n0 + 32 <= a.N;
  if (whole && a.bias_dtype == PKM_DT_BF16 && (reinterpret_cast<uintptr_t>(a.bias) & 15u) == 0) {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.bias) + n0);
#pragma unroll
    for (int v = 0; v < 4; ++v) VecTraits<__nv_bfloat16>::unpack(__ldg(p + v), f + 8 * v);
  } else if (whole && a.bias_dtype == PKM_DT_F32 && (reinterpret_cast<uintptr_t>(a.bias) & 15u) == 0) {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const float*>(a.bias) + n0);
#pragma unroll
    for (int v = 0; v < 8; ++v) VecTraits<float>::unpack(__ldg(p + v), f + 4 * v);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = n0 + j < a.N ? ld_f(a.bias, a.bias_dtype, n0 + j) : 0.f;
  }
}

// PAIR: launched as clusters of two CTAs; rank 0 of each pair issues the
// pair's MMAs (M = 256), both CTAs load their halves of the operands and run
// the epilogue on their own 128 accumulator rows.
template <bool PAIR>
__global__ void __launch_bounds__(GM_THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                     const __grid_constant__ CUtensorMap tc, const __grid_constant__ CUtensorMap tx_a,
                     const __grid_constant__ CUtensorMap tx_h, const __grid_constant__ CUtensorMap tx_o,
                     const GemmArgs a) {
  using G = GmTile<PAIR>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::STAGES * G::STAGE + G::STAGING);
  uint64_t* empty = full + G::STAGES;
  uint64_t* tfull = empty + G::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* ebar = drain + 1;  // one per epilogue warp: its gate-input boxes
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar + GM_EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int64_t cta0 = PAIR ? (int64_t)(blockIdx.x >> 1) : (int64_t)blockIdx.x;  // first unit
  const int64_t ctas = PAIR ? (int64_t)(gridDim.x >> 1) : (int64_t)gridDim.x;    // unit stride
  if (threadIdx.x == 0) {
    for (int s = 0; s < G::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      // pair: one arrival per epilogue warp of both CTAs (rank 0's barrier)
      mbar_init(&tempty[i], PAIR ? 2 * GM_EPI_WARPS : GM_EPI_WARPS * 32);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < GM_EPI_WARPS; ++i) mbar_init(&ebar[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 512);
      tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&ta);
    prefetch_tmap(&tb);
    if (a.st_tma || a.gt_tma) prefetch_tmap(&tc);
    if (a.gt_tma) {
      prefetch_tmap(&tx_a);
      if (a.epi == 2) prefetch_tmap(&tx_h);
      if (a.aux_out) prefetch_tmap(&tx_o);
    }
  }
  tc_fence_before();
  __syncwarp();  // barrier.cluster is warp-aligned
  if constexpr (PAIR)
    cluster_sync_all();  // both CTAs' barriers are initialised before any copy or arrival reaches them
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // rank 0's full barriers count the copies of both CTAs of a pair
      const uint32_t full0 = PAIR ? mapa_shared(smem_u32(full), 0) : smem_u32(full);
      uint32_t u = 0;
      for (int64_t unit = cta0; unit < a.units && !*abort_flag; unit += ctas) {
        int b, mt, nt, s, kb0, kb1;
        gm_decode(a, unit, b, mt, nt, s);
        gm_krange(a, s, kb0, kb1);
        const int m0 = mt * G::TM + (int)rank * GM_BM;   // this CTA's A rows
        const int n0 = nt * GM_BN + (int)rank * G::BROWS;  // this CTA's B rows
        for (int kb = kb0; kb < kb1; ++kb, ++u) {
          const int st = (int)(u % G::STAGES);
          if (!gm_wait(&empty[st], ((u / G::STAGES) & 1) ^ 1, a, abort_flag)) break;
          unsigned char* sa = smem + st * G::STAGE;
          unsigned char* sb = sa + G::A_BYTES;
          if (rank == 0) mbar_arrive_expect_tx(&full[st], PAIR ? 2 * G::STAGE : G::STAGE);
          const uint32_t fb = full0 + (uint32_t)st * 8u;
          auto load = [&](void* dst, const CUtensorMap* map, int x, int y) {
            if constexpr (PAIR)
              tma_load_2d_pair(dst, map, x, y, fb);
            else
              tma_load_2d(dst, map, x, y, &full[st]);
          };
          const int k0 = kb * GM_BK;
          if (a.a_mn) {
#pragma unroll
            for (int i = 0; i < GM_BM / GM_MN_BOX; ++i)
              load(sa + i * GM_MN_BOX_BYTES, &ta, m0 + i * GM_MN_BOX + b * a.a_bx, k0 + b * a.a_by);
          } else {
            load(sa, &ta, k0 + b * a.a_bx, m0 + b * a.a_by);
          }
          if (a.b_mn) {
#pragma unroll
            for (int i = 0; i < G::BROWS / GM_MN_BOX; ++i)
              load(sb + i * GM_MN_BOX_BYTES, &tb, n0 + i * GM_MN_BOX + b * a.b_bx, k0 + b * a.b_by);
          } else {
            load(sb, &tb, k0 + b * a.b_bx, n0 + b * a.b_by);
          }
        }
      }
      // the copies in flight must land before the block exits (full wait
      // limit); in a pair, rank 0's barriers count both CTAs' copies and the
      // final cluster barrier holds rank 1 until rank 0 has seen them land
      if (rank == 0)
        for (uint32_t j = (u > (uint32_t)G::STAGES ? u - G::STAGES : 0u); j < u; ++j)
          if (!mbar_wait(&full[j % G::STAGES], (j / G::STAGES) & 1, nullptr)) break;
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc =
          umma_idesc_bf16(G::TM, GM_BN) | ((uint32_t)a.a_mn << 15) | ((uint32_t)a.b_mn << 16);
      // descriptor step per 16-element K slice: 32 bytes along a K-major row,
      // 16 rows of 128 bytes in an MN-major box
      const uint64_t a_step = a.a_mn ? (16 * 128) >> 4 : 32 >> 4;
      const uint64_t b_step = a.b_mn ? (16 * 128) >> 4 : 32 >> 4;
      uint32_t u = 0;
      int li = 0;
      bool ok = true;
      for (int64_t unit = cta0; unit < a.units && ok && !*abort_flag; unit += ctas, ++li) {
        int b, mt, nt, s, kb0, kb1;
        gm_decode(a, unit, b, mt, nt, s);
        gm_krange(a, s, kb0, kb1);
        const int acc = li & 1;
        if (!gm_wait<PAIR>(&tempty[acc], ((li >> 1) & 1) ^ 1, a, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * GM_BN);
        for (int kb = kb0; kb < kb1; ++kb, ++u) {
          const int st = (int)(u % G::STAGES);
          if (!gm_wait(&full[st], (u / G::STAGES) & 1, a, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const unsigned char* sa = smem + st * G::STAGE;
          const uint64_t ad = a.a_mn ? umma_desc_mn_sw128(sa) : umma_desc_k_sw128(sa);
          const uint64_t bd =
              a.b_mn ? umma_desc_mn_sw128(sa + G::A_BYTES) : umma_desc_k_sw128(sa + G::A_BYTES);
#pragma unroll
          for (int k = 0; k < GM_BK / 16; ++k) {
            const uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
            if constexpr (PAIR)
              umma_bf16_pair(d_tmem, ad + a_step * k, bd + b_step * k, idesc, accum);
            else
              umma_bf16(d_tmem, ad + a_step * k, bd + b_step * k, idesc, accum);
          }
          // the stage is free in both CTAs once these MMAs have read it
          if constexpr (PAIR)
            umma_commit_pair(&empty[st], 3);
          else
            umma_commit(&empty[st]);
        }
        if (ok) {
          if constexpr (PAIR)
            umma_commit_pair(&tfull[acc], 3);
          else
            umma_commit(&tfull[acc]);
        }
      }
      // every MMA issued here completes before TMEM is released
      if constexpr (PAIR)
        umma_commit_pair(drain, 1);
      else
        umma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  } else {
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;       // which 128 of the tile's 256 columns
    constexpr int HC = GM_BN / 2 / 32;      // 32-column chunks per warp
    // pair: the accumulator-empty barriers of rank 0
    const uint32_t tempty0 = PAIR ? mapa_shared(smem_u32(tempty), 0) : 0u;
    // TMA store boxes are 32 rows x 128 bytes: 32 fp32 columns (one chunk)
    // or 64 bf16 columns (two chunks)
    const bool f32box = a.splits > 1 || a.c_dtype == PKM_DT_F32;
    unsigned char* stg = smem + G::STAGES * G::STAGE + (warp - 2) * 4096;
    unsigned char* stg_row = stg + lane * 128;
    // gate boxes: 32 rows x 64 bytes each, 16-byte chunk j of row r at
    // j ^ ((r >> 1) & 3) (64-byte swizzle); box A holds a, then z / da;
    // box H holds h (backward), then h / dh
    unsigned char* gbox_a = stg;
    unsigned char* gbox_h = stg + 2048;
    const uint32_t g_sw = (uint32_t)((lane >> 1) & 3);
    uint64_t* my_ebar = &ebar[warp - 2];
    uint32_t eph = 0;  // loads completed on my_ebar
    int li = 0;
    for (int64_t unit = cta0; unit < a.units; unit += ctas, ++li) {
      const int acc = li & 1;
      // the warp leaves together (tcgen05.ld is warp-collective)
      const bool got = gm_wait(&tfull[acc], (li >> 1) & 1, a, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      int b, mt, nt, s;
      gm_decode(a, unit, b, mt, nt, s);
      const int mw = mt * G::TM + (int)rank * GM_BM + q * 32;  // the warp's first row
      const int m = mw + lane;
      const bool rows_in = mw + 32 <= a.M;
      const uint32_t tbase =
          tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * GM_BN + half * (GM_BN / 2));
      // two register buffers: the load of chunk c + 1 is in flight while
      // chunk c is converted and stored (tcgen05.wait::ld waits for all)
      uint32_t r[2][32];
      tmem_ld_32x32b_x32(tbase, r[0]);
      tmem_ld_wait();
      bool gate_fail = false;  // a gate box never arrived: the warp leaves (the error is raised)
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        if (c + 1 < HC) tmem_ld_32x32b_x32(tbase + (uint32_t)((c + 1) * 32), r[(c + 1) & 1]);
        const uint32_t* rc = r[c & 1];
        const int n0 = nt * GM_BN + half * (GM_BN / 2) + c * 32;
        const int nb = f32box ? n0 : n0 - (c & 1) * 32;  // the box's first column
        if (a.gt_tma && rows_in && n0 + 32 <= a.N) {
          // the gate through TMA boxes
          if (lane == 0) {
            bulk_wait_read_all();  // the previous boxes have left shared memory
            mbar_arrive_expect_tx(my_ebar, a.epi == 2 ? 4096u : 2048u);
            tma_load_2d(gbox_a, &tx_a, n0, mw, my_ebar);
            if (a.epi == 2) tma_load_2d(gbox_h, &tx_h, n0, mw, my_ebar);
          }
          const bool got_box = gm_wait(my_ebar, eph & 1u, a, abort_flag);
          ++eph;
          if (!__all_sync(0xffffffffu, got_box)) {
            tmem_ld_wait();
            gate_fail = true;
            break;
          }
          float f[32];
          gm_bias32(a, n0, f);
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] += __uint_as_float(rc[j]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t off = (uint32_t)lane * 64u + ((((uint32_t)j) ^ g_sw) << 4);
            float av[8], hv[8], o[8], o2[8];
            VecTraits<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(gbox_a + off), av);
            if (a.epi == 2) VecTraits<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(gbox_h + off), hv);
            gate8(a.epi, av, hv, f + 8 * j, o, o2);
            *reinterpret_cast<uint4*>(gbox_h + off) =
                make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                           pack_bf16x2(o[6], o[7]));
            *reinterpret_cast<uint4*>(gbox_a + off) =
                make_uint4(pack_bf16x2(o2[0], o2[1]), pack_bf16x2(o2[2], o2[3]), pack_bf16x2(o2[4], o2[5]),
                           pack_bf16x2(o2[6], o2[7]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tc, gbox_h, n0, mw);
            if (a.aux_out) tma_store_2d(&tx_o, gbox_a, n0, mw);
            bulk_commit_group();
          }
        } else if (a.st_tma && rows_in && nb + (f32box ? 32 : 64) <= a.N) {
          // into the staging box (row = lane, 16-byte chunk j at j ^ (row & 7))
          if (f32box || (c & 1) == 0) {
            if (lane == 0) bulk_wait_read_all();  // the previous box has left shared memory
            __syncwarp();
          }
          if (a.splits > 1) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<uint4*>(stg_row + ((j ^ (lane & 7)) << 4)) =
                  make_uint4(rc[4 * j], rc[4 * j + 1], rc[4 * j + 2], rc[4 * j + 3]);
          } else {
            float f[32];
            gm_bias32(a, n0, f);
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] += __uint_as_float(rc[j]);
            if (f32box) {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                *reinterpret_cast<uint4*>(stg_row + ((j ^ (lane & 7)) << 4)) =
                    make_uint4(__float_as_uint(f[4 * j]), __float_as_uint(f[4 * j + 1]),
                               __float_as_uint(f[4 * j + 2]), __float_as_uint(f[4 * j + 3]));
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint4 v;
                __nv_bfloat162 h;
                h = __floats2bfloat162_rn(f[8 * j], f[8 * j + 1]);
                v.x = *reinterpret_cast<uint32_t*>(&h);
                h = __floats2bfloat162_rn(f[8 * j + 2], f[8 * j + 3]);
                v.y = *reinterpret_cast<uint32_t*>(&h);
                h = __floats2bfloat162_rn(f[8 * j + 4], f[8 * j + 5]);
                v.z = *reinterpret_cast<uint32_t*>(&h);
                h = __floats2bfloat162_rn(f[8 * j + 6], f[8 * j + 7]);
                v.w = *reinterpret_cast<uint32_t*>(&h);
                *reinterpret_cast<uint4*>(stg_row + ((((c & 1) * 4 + j) ^ (lane & 7)) << 4)) = v;
              }
            }
          }
          if (f32box || (c & 1) == 1) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tc, stg, b * a.st_bx + nb, s * a.st_sy + b * a.st_by + mw);
              bulk_commit_group();
            }
          }
        } else if (m < a.M && n0 < a.N) {
          if (a.splits > 1) {
            float* dst = a.ws + (((int64_t)s * a.batch + b) * a.M + m) * (int64_t)a.N + n0;
#pragma unroll
            for (int v = 0; v < 8; ++v)
              if (n0 + v * 4 + 4 <= a.N)
                reinterpret_cast<float4*>(dst)[v] =
                    make_float4(__uint_as_float(rc[4 * v]), __uint_as_float(rc[4 * v + 1]),
                                __uint_as_float(rc[4 * v + 2]), __uint_as_float(rc[4 * v + 3]));
          } else {
            float f[32];
            gm_bias32(a, n0, f);
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] += __uint_as_float(rc[j]);
            const int64_t e0 = b * a.c_bs + (int64_t)m * a.ldc + n0;
            if (a.epi) {
              const int64_t x0 = (int64_t)m * a.ld_aux + n0;
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                if (n0 + v * 8 + 8 > a.N) continue;
                float o[8], o2[8];
                gm_gate8(a, x0 + v * 8, f + v * 8, o, o2);
                st_run(a.c, PKM_DT_BF16, e0 + v * 8, o, 8);
                if (a.aux_out) st_run(a.aux_out, PKM_DT_BF16, x0 + v * 8, o2, 8);
              }
            } else {
#pragma unroll
              for (int v = 0; v < 4; ++v)
                if (n0 + v * 8 + 8 <= a.N) st_run(a.c, a.c_dtype, e0 + v * 8, f + v * 8, 8);
            }
          }
        }
        tmem_ld_wait();
      }
      if (gate_fail) break;
      tc_fence_before();
      if constexpr (PAIR) {
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(tempty0 + (uint32_t)acc * 8u);
      } else {
        mbar_arrive(&tempty[acc]);
      }
    }
    if (lane == 0) bulk_wait_all();  // this warp's boxes are written
  }
  tc_fence_before();
  __syncwarp();
  if constexpr (PAIR)
    cluster_sync_all();  // no copy, MMA or arrival of either CTA is still aimed at the other
  else
    __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, 512);
    else
      tmem_dealloc(tmem_base, 512);
  }
}

// out[b][m][n] = sum_s ws[s][b][m][n] + bias[n], summed in split order.
__global__ void gemm_split_reduce_kernel(const GemmArgs a) {
  const int64_t per = (int64_t)a.batch * a.M * (a.N / 4);
  const int64_t plane = (int64_t)a.batch * a.M * a.N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / (a.N / 4);
    const int n = (int)(i % (a.N / 4)) * 4;
    const int b = (int)(row / a.M);
    const int m = (int)(row % a.M);
    float4 acc = reinterpret_cast<const float4*>(a.ws + row * a.N + n)[0];
    for (int s = 1; s < a.splits; ++s) {
      const float4 v = reinterpret_cast<const float4*>(a.ws + s * plane + row * a.N + n)[0];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    float f[4] = {acc.x + gm_bias(a, n), acc.y + gm_bias(a, n + 1), acc.z + gm_bias(a, n + 2),
                  acc.w + gm_bias(a, n + 3)};
    st_run(a.c, a.c_dtype, b * a.c_bs + (int64_t)m * a.ldc + n, f, 4);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static std::atomic<int64_t> g_gemm_wait_limit{-1};

int make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t row_stride_bytes,
                      uint32_t box_cols, uint32_t box_rows);

// -1: CTA pairs whenever the tile has more than 128 rows; 0: never; 1:
// always (a test hook: both forms run every shape).
static std::atomic<int> g_gemm_pair{-1};

static bool gemm_use_pair(int64_t M) {
  const int mode = g_gemm_pair.load();
  return mode == 1 || (mode < 0 && M > GM_BM);
}

// Clusters of two CTAs resident at once (the pair kernel's persistent grid),
// cached per device ordinal.
static int gemm_pair_slots() {
  static std::atomic<int> cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    v = num_sms() / 2;
    if (cudaFuncSetAttribute(gemm_bf16_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GmTile<true>::SMEM) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(2 * std::max(1, num_sms() / 2)));
      cfg.blockDim = dim3(GM_THREADS);
      cfg.dynamicSmemBytes = GmTile<true>::SMEM;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, gemm_bf16_kernel<true>, &cfg) == cudaSuccess && n > 0) v = n;
    }
    cudaGetLastError();  // a failed query leaves the fallback and no sticky error
    v = std::max(v, 1);
    cache[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

// Split count: the K range is divided while the tiles alone would leave
// CTAs (or CTA pairs) idle and every split keeps at least four 64-deep K
// blocks.
static int gemm_splits(int64_t tiles, int64_t k_blocks, int64_t slots) {
  int s = 1;
  while (tiles * s * 2 <= slots && k_blocks / (s * 2) >= 4 && s < 16) s *= 2;
  return s;
}

static void gemm_shape(int64_t batch, int64_t M, int64_t N, int64_t K, bool pair, int64_t& mt, int64_t& nt,
                       int64_t& kb, int& splits) {
  const int64_t tm = pair ? 2 * GM_BM : GM_BM;
  mt = (M + tm - 1) / tm;
  nt = (N + GM_BN - 1) / GM_BN;
  kb = (K + GM_BK - 1) / GM_BK;
  splits = gemm_splits(batch * mt * nt, kb, pair ? gemm_pair_slots() : num_sms());
}

struct GateArgs {
  int epi;
  const void* a;
  const void* h;
  void* out;
  int64_t ld;
};

int gemm_launch(const void* A, int a_mn_major, int64_t a_rows, int64_t a_cols, int64_t lda, const void* B,
                int b_mn_major, int64_t b_rows, int64_t b_cols, int64_t ldb, int64_t batch, int64_t M, int64_t N,
                int64_t K, int64_t a_batch_x, int64_t a_batch_y, int64_t b_batch_x, int64_t b_batch_y,
                const void* bias, int bias_dtype, void* C, int c_dtype, int64_t ldc, int64_t c_batch_stride,
                void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream, const GateArgs& gate);

}  // namespace pkm

using namespace pkm;

extern "C" int pkm_gemm_workspace(int64_t batch, int64_t M, int64_t N, int64_t K, size_t* bytes) {
  if (!bytes) return fail(PKM_ERR_INVALID_ARG, "null bytes");
  if (batch < 0 || M < 0 || N < 0 || K < 0) return fail(PKM_ERR_INVALID_ARG, "negative size");
  int64_t mt, nt, kb;
  int s;
  gemm_shape(batch, M, N, K, gemm_use_pair(M), mt, nt, kb, s);
  *bytes = s > 1 ? (size_t)s * batch * M * N * sizeof(float) : 0;
  return PKM_OK;
}

extern "C" int pkm_debug_gemm_pair(int mode) {
  if (mode < -1 || mode > 1) return fail(PKM_ERR_INVALID_ARG, "mode must be -1, 0 or 1");
  g_gemm_pair.store(mode);
  return PKM_OK;
}

extern "C" int pkm_debug_set_wait_limit(int64_t polls) {
  g_gemm_wait_limit.store(polls < 0 ? -1 : std::min<int64_t>(polls, kWaitLimit));
  return PKM_OK;
}

extern "C" int pkm_gemm_bf16(const void* A, int a_mn_major, int64_t a_rows, int64_t a_cols, int64_t lda,
                             const void* B, int b_mn_major, int64_t b_rows, int64_t b_cols, int64_t ldb,
                             int64_t batch, int64_t M, int64_t N, int64_t K, int64_t a_batch_x, int64_t a_batch_y,
                             int64_t b_batch_x, int64_t b_batch_y, const void* bias, int bias_dtype, void* C,
                             int c_dtype, int64_t ldc, int64_t c_batch_stride, void* workspace,
                             size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  return gemm_launch(A, a_mn_major, a_rows, a_cols, lda, B, b_mn_major, b_rows, b_cols, ldb, batch, M, N, K,
                     a_batch_x, a_batch_y, b_batch_x, b_batch_y, bias, bias_dtype, C, c_dtype, ldc, c_batch_stride,
                     workspace, workspace_bytes, dev_err, stream, GateArgs{0, nullptr, nullptr, nullptr, 0});
}

static int gate_checks(const void* a, const void* h, const void* out, int64_t ld, int64_t N, bool need_h) {
  if (!a || (need_h && !h)) return fail(PKM_ERR_INVALID_ARG, "null gate input");
  if (ld < N || (ld * 2) % 16 || !aligned16(a) || (h && !aligned16(h)) || (out && !aligned16(out)))
    return fail(PKM_ERR_INVALID_ARG, "gate operands need 16-byte aligned bases and row pitches");
  return PKM_OK;
}

extern "C" int pkm_gemm_swiglu_fwd(const void* x, int64_t ldx, const void* ws, const void* bs, int bias_dtype,
                                   const void* a, int64_t M, int64_t N, int64_t K, void* h, void* z, int64_t ld,
                                   uint32_t* dev_err, void* stream) {
  int rc = gate_checks(a, nullptr, z, ld, N, false);
  if (rc) return rc;
  if (!z) return fail(PKM_ERR_INVALID_ARG, "null z");
  return gemm_launch(x, 0, M, K, ldx, ws, 0, N, K, K, 1, M, N, K, 0, 0, 0, 0, bs, bias_dtype, h, PKM_DT_BF16, ld,
                     0, nullptr, 0, dev_err, stream, GateArgs{1, a, nullptr, z, ld});
}

extern "C" int pkm_gemm_swiglu_bwd(const void* dy, int64_t ldy, const void* wv, int64_t ldw, const void* a,
                                   const void* h, int64_t M, int64_t N, int64_t K, void* dh, void* da, int64_t ld,
                                   uint32_t* dev_err, void* stream) {
  int rc = gate_checks(a, h, da, ld, N, true);
  if (rc) return rc;
  // dz = dy @ wv: wv is [K, N] (the value projection's weight [out, in]), read MN-major
  return gemm_launch(dy, 0, M, K, ldy, wv, 1, K, N, ldw, 1, M, N, K, 0, 0, 0, 0, nullptr, 0, dh, PKM_DT_BF16, ld,
                     0, nullptr, 0, dev_err, stream, GateArgs{2, a, h, da, ld});
}

int pkm::gemm_launch(const void* A, int a_mn_major, int64_t a_rows, int64_t a_cols, int64_t lda, const void* B,
                     int b_mn_major, int64_t b_rows, int64_t b_cols, int64_t ldb, int64_t batch, int64_t M, int64_t N,
                     int64_t K, int64_t a_batch_x, int64_t a_batch_y, int64_t b_batch_x, int64_t b_batch_y,
                     const void* bias, int bias_dtype, void* C, int c_dtype, int64_t ldc, int64_t c_batch_stride,
                     void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream,
                     const GateArgs& gate) {
  if (batch < 0 || M < 0 || N < 0 || K < 0) return fail(PKM_ERR_INVALID_ARG, "negative size");
  if (batch == 0 || M == 0 || N == 0) return PKM_OK;
  if (!A || !B || !C) return fail(PKM_ERR_INVALID_ARG, "null operand");
  if (c_dtype != PKM_DT_BF16 && c_dtype != PKM_DT_F32) return fail(PKM_ERR_INVALID_ARG, "C must be bf16 or fp32");
  if (bias && !valid_dtype(bias_dtype)) return fail(PKM_ERR_INVALID_ARG, "bad bias dtype");
  if (K <= 0) return fail(PKM_ERR_UNSUPPORTED, "K must be positive");
  if (K % GM_BK != 0) {
    // the last K block runs past K: TMA fills zeros there only where K ends
    // at the operand's edge, so the K extent must be exactly K
    const int64_t a_k_extent = a_mn_major ? a_rows : a_cols, b_k_extent = b_mn_major ? b_rows : b_cols;
    const int64_t a_k_off = a_mn_major ? a_batch_y : a_batch_x, b_k_off = b_mn_major ? b_batch_y : b_batch_x;
    if ((batch > 1 && (a_k_off || b_k_off)) || a_k_extent != K || b_k_extent != K)
      return fail(PKM_ERR_UNSUPPORTED, "K must be a multiple of 64 unless it spans the operands' whole K extent");
  }
  if (N % 8 != 0) return fail(PKM_ERR_UNSUPPORTED, "N must be a multiple of 8");
  if (ldc < N) return fail(PKM_ERR_INVALID_ARG, "ldc < N");
  if ((lda * 2) % 16 || (ldb * 2) % 16 || !aligned16(A) || !aligned16(B) || !aligned16(C) ||
      (ldc * dtype_size(c_dtype)) % 16 || (c_batch_stride * dtype_size(c_dtype)) % 16)
    return fail(PKM_ERR_INVALID_ARG, "operands need 16-byte aligned bases and row pitches");
  if (a_rows <= 0 || a_cols <= 0 || b_rows <= 0 || b_cols <= 0 || a_cols > lda || b_cols > ldb)
    return fail(PKM_ERR_INVALID_ARG, "bad operand extents");
  // A tile that overhangs a batch's M or N range reads the next batch's rows
  // into accumulator rows / columns the epilogue discards; along K no tile
  // overhangs (K is a multiple of the 64-deep K block).  A TMA copy's
  // innermost coordinate must be a multiple of 16 bytes: every column offset
  // here is a multiple of 8 elements.
  if (a_batch_x % 8 || b_batch_x % 8) return fail(PKM_ERR_INVALID_ARG, "column batch offsets must be multiples of 8");
  // operand extents cover every batch's region
  const int64_t a_need_x = (a_mn_major ? M : K) + (batch - 1) * a_batch_x;
  const int64_t a_need_y = (a_mn_major ? K : M) + (batch - 1) * a_batch_y;
  const int64_t b_need_x = (b_mn_major ? N : K) + (batch - 1) * b_batch_x;
  const int64_t b_need_y = (b_mn_major ? K : N) + (batch - 1) * b_batch_y;
  if (a_need_x > a_cols || a_need_y > a_rows || b_need_x > b_cols || b_need_y > b_rows)
    return fail(PKM_ERR_INVALID_ARG, "operand extents smaller than the GEMM");
  if (a_batch_x < 0 || a_batch_y < 0 || b_batch_x < 0 || b_batch_y < 0 || c_batch_stride < 0)
    return fail(PKM_ERR_INVALID_ARG, "negative batch offset");
  if (a_rows > INT32_MAX || a_cols > INT32_MAX || b_rows > INT32_MAX || b_cols > INT32_MAX)
    return fail(PKM_ERR_UNSUPPORTED, "operand extent above 2^31");

  const bool pair = gemm_use_pair(M);
  int64_t mt, nt, kb;
  int splits;
  gemm_shape(batch, M, N, K, pair, mt, nt, kb, splits);
  if (gate.epi) {
    if (batch != 1) return fail(PKM_ERR_INVALID_ARG, "the fused gate takes one GEMM");
    splits = 1;
  }
  const size_t need = splits > 1 ? (size_t)splits * batch * M * N * sizeof(float) : 0;
  if (need > workspace_bytes || (need && !workspace))
    return fail(PKM_ERR_WORKSPACE, "pkm_gemm_bf16: workspace smaller than pkm_gemm_workspace()");
  if (need && !aligned16(workspace)) return fail(PKM_ERR_INVALID_ARG, "workspace must be 16-byte aligned");

  CUtensorMap ta, tb;
  int rc = make_tmap_bf16_2d(&ta, A, (uint64_t)a_cols, (uint64_t)a_rows, (uint64_t)(lda * 2),
                             a_mn_major ? GM_MN_BOX : GM_BK, a_mn_major ? GM_BK : GM_BM);
  if (rc) return rc;
  rc = make_tmap_bf16_2d(&tb, B, (uint64_t)b_cols, (uint64_t)b_rows, (uint64_t)(ldb * 2),
                         b_mn_major ? GM_MN_BOX : GM_BK, b_mn_major ? GM_BK : (pair ? GM_BN / 2 : GM_BN));
  if (rc) return rc;
  GemmArgs a{};
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.batch = (int)batch;
  a.a_mn = a_mn_major ? 1 : 0;
  a.b_mn = b_mn_major ? 1 : 0;
  a.a_bx = (int)a_batch_x;
  a.a_by = (int)a_batch_y;
  a.b_bx = (int)b_batch_x;
  a.b_by = (int)b_batch_y;
  a.c_bs = c_batch_stride;
  a.m_tiles = (int)mt;
  a.n_tiles = (int)nt;
  a.k_blocks = (int)kb;
  a.splits = splits;
  a.units = batch * mt * nt * splits;
  a.c = C;
  a.c_dtype = c_dtype;
  a.ldc = ldc;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.ws = static_cast<float*>(workspace);
  a.err = dev_err;
  a.epi = gate.epi;
  a.aux_a = static_cast<const __nv_bfloat16*>(gate.a);
  a.aux_h = static_cast<const __nv_bfloat16*>(gate.h);
  a.aux_out = static_cast<__nv_bfloat16*>(gate.out);
  a.ld_aux = gate.ld;
  // the epilogue's TMA store map: the split partials [splits * batch * M, N]
  // fp32, or C viewed as one matrix holding every batch (batches offset by
  // whole rows or by columns within a row); anything else stores directly
  CUtensorMap tcm, txa, txh, txo;
  memset(&tcm, 0, sizeof(tcm));
  memset(&txa, 0, sizeof(txa));
  memset(&txh, 0, sizeof(txh));
  memset(&txo, 0, sizeof(txo));
  a.st_tma = 0;
  a.gt_tma = 0;
  if (gate.epi && M < INT32_MAX) {
    // the gate's operands are [M, N] bf16: C at pitch ldc, a / h / aux_out at
    // the gate pitch; boxes of 32 columns x 32 rows, 64-byte swizzle
    const int64_t lg = gate.ld * 2;
    bool ok = make_tmap_2d(&tcm, C, PKM_DT_BF16, (uint64_t)N, (uint64_t)M, (uint64_t)(ldc * 2), 32, 32, 64) ==
                  PKM_OK &&
              make_tmap_2d(&txa, gate.a, PKM_DT_BF16, (uint64_t)N, (uint64_t)M, (uint64_t)lg, 32, 32, 64) == PKM_OK;
    if (ok && gate.epi == 2)
      ok = make_tmap_2d(&txh, gate.h, PKM_DT_BF16, (uint64_t)N, (uint64_t)M, (uint64_t)lg, 32, 32, 64) == PKM_OK;
    if (ok && gate.out)
      ok = make_tmap_2d(&txo, gate.out, PKM_DT_BF16, (uint64_t)N, (uint64_t)M, (uint64_t)lg, 32, 32, 64) == PKM_OK;
    a.gt_tma = ok ? 1 : 0;
  }
  if (!gate.epi) {
    int64_t rows = 0, cols = 0, bx = 0, by = 0, sy = 0;
    if (splits > 1) {
      rows = (int64_t)splits * batch * M;
      cols = N;
      by = M;
      sy = batch * M;
    } else if (batch == 1) {
      rows = M;
      cols = N;
    } else if (c_batch_stride % ldc == 0) {
      by = c_batch_stride / ldc;
      rows = (batch - 1) * by + M;
      cols = N;
    } else if ((batch - 1) * c_batch_stride + N <= ldc) {
      bx = c_batch_stride;
      rows = M;
      cols = (batch - 1) * c_batch_stride + N;
    }
    if (rows > 0 && rows < INT32_MAX && cols < INT32_MAX) {
      const bool ws32 = splits > 1;
      const int dt = ws32 ? PKM_DT_F32 : c_dtype;
      const int64_t pitch = ws32 ? N * 4 : ldc * dtype_size(c_dtype);
      if (make_tmap_2d(&tcm, ws32 ? workspace : C, dt, (uint64_t)cols, (uint64_t)rows, (uint64_t)pitch,
                       dt == PKM_DT_F32 ? 32 : 64, 32, 128) == PKM_OK) {
        a.st_tma = 1;
        a.st_bx = (int)bx;
        a.st_by = (int)by;
        a.st_sy = (int)sy;
      }
    }
  }
  const int64_t wl = g_gemm_wait_limit.load();
  a.wait_limit = wl < 0 ? kWaitLimit : (uint32_t)wl;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pair) {
    if (cudaFuncSetAttribute(gemm_bf16_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GmTile<true>::SMEM) != cudaSuccess)
      return check_cuda("cudaFuncSetAttribute(gemm_bf16 pair)");
    const int64_t clusters = std::max<int64_t>(1, std::min<int64_t>(a.units, gemm_pair_slots()));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * clusters));
    cfg.blockDim = dim3(GM_THREADS);
    cfg.dynamicSmemBytes = GmTile<true>::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<true>, ta, tb, tcm, txa, txh, txo, a);
    if (le != cudaSuccess) {
      cudaGetLastError();
      return fail(PKM_ERR_CUDA, std::string("gemm_bf16_kernel (pair) launch: ") + cudaGetErrorString(le));
    }
  } else {
    if (cudaFuncSetAttribute(gemm_bf16_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GmTile<false>::SMEM) != cudaSuccess)
      return check_cuda("cudaFuncSetAttribute(gemm_bf16)");
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(a.units, num_sms()));
    gemm_bf16_kernel<false><<<(unsigned)grid, GM_THREADS, GmTile<false>::SMEM, st>>>(ta, tb, tcm, txa, txh, txo,
                                                                                       a);
  }
  rc = check_cuda("gemm_bf16_kernel");
  if (rc || splits == 1) return rc;
  const int64_t per = batch * M * (N / 4);
  const int64_t rgrid = std::max<int64_t>(1, std::min<int64_t>((per + 255) / 256, (int64_t)num_sms() * 8));
  gemm_split_reduce_kernel<<<(unsigned)rgrid, 256, 0, st>>>(a);
  return check_cuda("gemm_split_reduce_kernel");
}
