// Sub-key scores (K1) on the 5th-generation tensor cores.
//
// For every (head, half) group hp the scores are the GEMM
//   S_hp[t, m] = Q_hp[t, :] . K_hp[m, :]      (t: token, m: sub-key)
// with Q_hp the hp-th half-query slice of every token (row pitch H*k_dim) and
// K_hp the hp-th block of the key table.  A persistent, warp-specialised
// kernel computes 128 x 256 output tiles:
//   warp 0    TMA producer: 64-wide K slices of Q and K into a 4-stage ring
//             of 128-byte-swizzled shared tiles;
//   warp 1    MMA issuer: tcgen05.mma kind::f16 (bf16 x bf16 -> fp32) into
//             one of two 256-column TMEM accumulators, tcgen05.commit frees
//             each stage and hands finished accumulators to the epilogue;
//   warps 2-5 epilogue: tcgen05.ld of the accumulator rows (one token row
//             per thread, the next 32 columns in flight), round to bf16
//             into a swizzled 32-token x 64-key staging box per warp, one
//             TMA store per box into [N, H, 2, n] (viewed as [N, H*2*n]);
//             boxes at a ragged edge are stored directly.
// Two accumulators let the epilogue of one tile overlap the MMAs of the next.
// Every wait is bounded; a timeout raises PKM_DEVERR_TIMEOUT and each role
// drains its own outstanding work before TMEM is released.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "umma.cuh"

namespace pkm {

constexpr int TC_BM = 128, TC_BN = 256, TC_BK = 64, TC_STAGES = 4;
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;
constexpr int TC_B_BYTES = TC_BN * TC_BK * 2;
constexpr int TC_STAGE = TC_A_BYTES + TC_B_BYTES;
constexpr int TC_THREADS = 192;
constexpr int TC_STAGING = 4 * 4096;  // per epilogue warp: 32 rows x 128 bytes
constexpr int TC_SMEM = TC_STAGES * TC_STAGE + TC_STAGING + 1024 + 256;

struct TcScoreArgs {
  int64_t n_tokens;
  int heads;
  int half;
  int n_keys;
  int m_tiles;
  int n_tiles;
  int k_blocks;
  int64_t n_tile_total;
  __nv_bfloat16* out;
  uint32_t* err;
  int st_tma;  // the output map is valid: whole boxes leave by TMA stores
};

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, uint32_t* err, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023) == 1023 && *abort_flag) return false;
  }
  raise_err(err, PKM_DEVERR_TIMEOUT);
  *abort_flag = 1;
  return false;
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    subkey_scores_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                            const __grid_constant__ CUtensorMap to, const TcScoreArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_STAGES * TC_STAGE + TC_STAGING);
  uint64_t* empty = full + TC_STAGES;
  uint64_t* tfull = empty + TC_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    if (a.st_tma) prefetch_tmap(&to);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int64_t ntiles = a.n_tile_total;
  const int KB = a.k_blocks;

  auto decode = [&](int64_t tile, int& hp, int& mt, int& nt) {
    nt = (int)(tile % a.n_tiles);
    const int64_t r = tile / a.n_tiles;
    mt = (int)(r % a.m_tiles);
    hp = (int)(r / a.m_tiles);
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t u = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles && !*abort_flag; tile += gridDim.x) {
        int hp, mt, nt;
        decode(tile, hp, mt, nt);
        for (int kb = 0; kb < KB; ++kb, ++u) {
          const int s = (int)(u % TC_STAGES);
          if (!tc_wait(&empty[s], ((u / TC_STAGES) & 1) ^ 1, a.err, abort_flag)) break;
          unsigned char* st = smem + s * TC_STAGE;
          mbar_arrive_expect_tx(&full[s], TC_STAGE);
          tma_load_2d(st, &tq, hp * a.half + kb * TC_BK, mt * TC_BM, &full[s]);
          tma_load_2d(st + TC_A_BYTES, &tk, kb * TC_BK, hp * a.n_keys + nt * TC_BN, &full[s]);
        }
      }
      // the last stages' copies must have landed before the block exits
      for (uint32_t j = (u > (uint32_t)TC_STAGES ? u - TC_STAGES : 0u); j < u; ++j)
        if (!mbar_wait(&full[j % TC_STAGES], (j / TC_STAGES) & 1, nullptr)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(TC_BM, TC_BN);
      uint32_t u = 0;
      int li = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < ntiles && ok && !*abort_flag; tile += gridDim.x, ++li) {
        const int acc = li & 1;
        if (!tc_wait(&tempty[acc], ((li >> 1) & 1) ^ 1, a.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * TC_BN);
        for (int kb = 0; kb < KB; ++kb, ++u) {
          const int s = (int)(u % TC_STAGES);
          if (!tc_wait(&full[s], (u / TC_STAGES) & 1, a.err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const unsigned char* st = smem + s * TC_STAGE;
          const uint64_t ad = umma_desc_k_sw128(st);
          const uint64_t bd = umma_desc_k_sw128(st + TC_A_BYTES);
#pragma unroll
          for (int k = 0; k < TC_BK / 16; ++k)  // 16 bf16 = 32 bytes = 2 descriptor units per step
            umma_bf16(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tfull[acc]);
      }
      // every MMA issued here completes before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int64_t H2 = (int64_t)a.heads * 2;
    // staging box: row = lane, 16-byte chunk j at j ^ (lane & 7) (128-byte swizzle)
    unsigned char* stg = smem + TC_STAGES * TC_STAGE + (warp - 2) * 4096;
    unsigned char* stg_row = stg + lane * 128;
    int li = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++li) {
      const int acc = li & 1;
      // the warp leaves together (tcgen05.ld is warp-collective)
      const bool got = tc_wait(&tfull[acc], (li >> 1) & 1, a.err, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      int hp, mt, nt;
      decode(tile, hp, mt, nt);
      const int64_t mw = (int64_t)mt * TC_BM + q * 32;  // the warp's first token
      const int64_t t = mw + lane;
      const bool rows_in = mw + 32 <= a.n_tokens;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * TC_BN);
      __nv_bfloat16* orow = a.out + (t * H2 + hp) * (int64_t)a.n_keys;
      uint32_t r[2][32];
      tmem_ld_32x32b_x32(tbase, r[0]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < TC_BN / 32; ++c) {
        if (c + 1 < TC_BN / 32) tmem_ld_32x32b_x32(tbase + (uint32_t)((c + 1) * 32), r[(c + 1) & 1]);
        const uint32_t* rc = r[c & 1];
        const int col0 = nt * TC_BN + c * 32;
        const int nb = col0 - (c & 1) * 32;  // the 64-key box's first key
        if (a.st_tma && rows_in && nb + 64 <= a.n_keys) {
          if ((c & 1) == 0) {
            if (lane == 0) bulk_wait_read_all();  // the previous box has left shared memory
            __syncwarp();
          }
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 o;
            __nv_bfloat162 h;
            h = __floats2bfloat162_rn(__uint_as_float(rc[v * 8 + 0]), __uint_as_float(rc[v * 8 + 1]));
            o.x = *reinterpret_cast<uint32_t*>(&h);
            h = __floats2bfloat162_rn(__uint_as_float(rc[v * 8 + 2]), __uint_as_float(rc[v * 8 + 3]));
            o.y = *reinterpret_cast<uint32_t*>(&h);
            h = __floats2bfloat162_rn(__uint_as_float(rc[v * 8 + 4]), __uint_as_float(rc[v * 8 + 5]));
            o.z = *reinterpret_cast<uint32_t*>(&h);
            h = __floats2bfloat162_rn(__uint_as_float(rc[v * 8 + 6]), __uint_as_float(rc[v * 8 + 7]));
            o.w = *reinterpret_cast<uint32_t*>(&h);
            *reinterpret_cast<uint4*>(stg_row + ((((c & 1) * 4 + v) ^ (lane & 7)) << 4)) = o;
          }
          if ((c & 1) == 1) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&to, stg, (int32_t)(hp * a.n_keys + nb), (int32_t)mw);
              bulk_commit_group();
            }
          }
        } else if (t < a.n_tokens) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const int col = col0 + v * 8;
            if (col + 8 <= a.n_keys) {
              uint4 o;
              __nv_bfloat162 h;
              h = __floats2bfloat162_rn(__uint_as_float(rc[v * 8 + 0]), __uint_as_float(rc[v * 8 + 1]));
              o.x = *reinterpret_cast<uint32_t*>(&h);
              h = __floats2bfloat162_rn(__uint_as_float(rc[v * 8 + 2]), __uint_as_float(rc[v * 8 + 3]));
              o.y = *reinterpret_cast<uint32_t*>(&h);
              h = __floats2bfloat162_rn(__uint_as_float(rc[v * 8 + 4]), __uint_as_float(rc[v * 8 + 5]));
              o.z = *reinterpret_cast<uint32_t*>(&h);
              h = __floats2bfloat162_rn(__uint_as_float(rc[v * 8 + 6]), __uint_as_float(rc[v * 8 + 7]));
              o.w = *reinterpret_cast<uint32_t*>(&h);
              *reinterpret_cast<uint4*>(orow + col) = o;
            }
          }
        }
        tmem_ld_wait();
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
    if (lane == 0) bulk_wait_all();  // this warp's boxes are written
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 512);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, int dtype, uint64_t cols, uint64_t rows,
                 uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows, int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(PKM_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  if (dtype != PKM_DT_BF16 && dtype != PKM_DT_F32) return fail(PKM_ERR_INVALID_ARG, "tensor map dtype");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      fn(map, dtype == PKM_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PKM_ERR_INVALID_ARG, "cuTensorMapEncodeTiled rejected the operand");
  return PKM_OK;
}

int make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t row_stride_bytes,
                      uint32_t box_cols, uint32_t box_rows) {
  return make_tmap_2d(map, base, PKM_DT_BF16, cols, rows, row_stride_bytes, box_cols, box_rows, 128);
}

bool subkey_scores_tc_eligible(int64_t heads, int64_t k_dim, int64_t n_keys, const void* query, const void* keys,
                               const void* scores) {
  const int64_t half = k_dim / 2;
  return half % TC_BK == 0 && n_keys % 8 == 0 && aligned16(query) && aligned16(keys) && aligned16(scores) &&
         heads * k_dim * 2 % 16 == 0;
}

int subkey_scores_tc(const void* query, const void* keys, int64_t n_tokens, int64_t heads, int64_t k_dim,
                     int64_t n_keys, void* scores, uint32_t* err, cudaStream_t st) {
  const int64_t half = k_dim / 2;
  CUtensorMap tq, tk;
  // Q viewed as [N, H*k_dim]: box 64 columns x 128 tokens
  int rc = make_tmap_bf16_2d(&tq, query, (uint64_t)(heads * k_dim), (uint64_t)n_tokens,
                             (uint64_t)(heads * k_dim * 2), TC_BK, TC_BM);
  if (rc) return rc;
  // keys [2*H*n, half]: box 64 columns x 256 keys
  rc = make_tmap_bf16_2d(&tk, keys, (uint64_t)half, (uint64_t)(2 * heads * n_keys), (uint64_t)(half * 2), TC_BK,
                         TC_BN);
  if (rc) return rc;
  TcScoreArgs a{};
  a.n_tokens = n_tokens;
  a.heads = (int)heads;
  a.half = (int)half;
  a.n_keys = (int)n_keys;
  a.m_tiles = (int)((n_tokens + TC_BM - 1) / TC_BM);
  a.n_tiles = (int)((n_keys + TC_BN - 1) / TC_BN);
  a.k_blocks = (int)(half / TC_BK);
  a.n_tile_total = (int64_t)a.m_tiles * a.n_tiles * heads * 2;
  a.out = static_cast<__nv_bfloat16*>(scores);
  a.err = err;
  // the scores [N, H*2*n] for the epilogue's TMA stores: boxes of 64 keys x
  // 32 tokens (a failed encode leaves the direct stores)
  CUtensorMap to;
  memset(&to, 0, sizeof(to));
  a.st_tma = n_tokens < INT32_MAX && 2 * heads * n_keys < INT32_MAX &&
             make_tmap_2d(&to, scores, PKM_DT_BF16, (uint64_t)(2 * heads * n_keys), (uint64_t)n_tokens,
                          (uint64_t)(2 * heads * n_keys * 2), 64, 32, 128) == PKM_OK;
  if (cudaFuncSetAttribute(subkey_scores_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM) !=
      cudaSuccess)
    return check_cuda("cudaFuncSetAttribute(subkey_scores_tc)");
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(a.n_tile_total, num_sms()));
  subkey_scores_tc_kernel<<<(unsigned)grid, TC_THREADS, TC_SMEM, st>>>(tq, tk, to, a);
  return check_cuda("subkey_scores_tc_kernel");
}

}  // namespace pkm
