// Embedding-bag kernels: forward gather-sum (K3), sorted-segment backward
// (K4) and the double-backward of the weight gradient (K5), with their C ABI
// entry points.
#include <algorithm>
#include <type_traits>
#include <string>

#include "gather.cuh"
#include "seg.cuh"
#include "sort.cuh"

namespace pkm {

// ---------------------------------------------------------------------------
// gather launch
// ---------------------------------------------------------------------------
static int max_dyn_smem() {
  int dev = 0, v = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return v;
}

// Ring depth and per-warp shared-memory stride for rows of rb bytes with nw
// warps per block (segment mode adds the item-descriptor ring).
static bool gather_geometry(int64_t rb, int nw, bool seg, bool dot, int* slots, int64_t* warp_smem) {
  const int64_t budget = (int64_t)(max_dyn_smem() - 1024) / nw;
  (void)dot;
  const int64_t fixed = kMetaRing * 12 + (seg ? kMetaRing * 16 : 0);
  for (int p = 32; p >= 2; --p) {
    int64_t ring = ((int64_t)p * rb + 127) & ~(int64_t)127;
    int64_t tot = ring + fixed + (int64_t)p * 8;
    tot = (tot + 127) & ~(int64_t)127;
    if (tot <= budget) {
      *slots = p;
      *warp_smem = tot;
      return true;
    }
  }
  return false;
}

// Segment pass: one block per SM, 12 warps (the register limit: the fp32
// accumulator, the unpacked table row and the next one), each with about
// 12 KiB of upstream-gradient rows in flight in its shared ring.
#ifndef PKM_SEG_WARPS
#define PKM_SEG_WARPS 12
#endif
#ifndef PKM_SEG_BYTES
#define PKM_SEG_BYTES 12288
#endif
template <typename RowT, int VPL, bool DOT, bool FULL>
static int launch_seg(GatherArgs a, int64_t items_upper, cudaStream_t st) {
  // 4 KiB rows (VPL 8) need more registers: 8 warps with 16 KiB rings
  constexpr int NW = VPL >= 8 ? 8 : PKM_SEG_WARPS;
  constexpr int RING = (VPL >= 8 ? 16384 : PKM_SEG_BYTES) / (VPL * 512);
  constexpr int DEPTH = RING < 2 ? 2 : (RING > 8 ? 8 : RING);
  auto kern = seg_direct_kernel<RowT, VPL, DOT, NW, FULL, DEPTH>;
  a.warp_smem = seg_warp_smem(a.row_bytes, DEPTH, DOT);
  const int smem = (int)(a.warp_smem * NW);
  if (smem > max_dyn_smem()) return fail(PKM_ERR_UNSUPPORTED, "row too large for the segment ring");
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return check_cuda("cudaFuncSetAttribute(seg)");
  int64_t blocks = (items_upper + NW - 1) / NW;
  blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, num_sms()));
  kern<<<(unsigned)blocks, NW * 32, smem, st>>>(a);
  return check_cuda("seg_direct_kernel");
}

template <typename RowT, int VPL, int MODE, bool DOT, bool FULL>
static int launch_one(GatherArgs a, int64_t items_upper, cudaStream_t st) {
  if (MODE == G_SEG) return launch_seg<RowT, VPL, DOT, FULL>(a, items_upper, st);
  // warps per block: as many as the registers allow, fewer for 4 KB rows so
  // that every warp still keeps a few rows in flight
  constexpr int NW = VPL >= 8 ? 8 : (DOT ? 12 : 16);
  int slots;
  int64_t ws;
  if (!gather_geometry(a.row_bytes, NW, MODE == G_SEG, DOT, &slots, &ws))
    return fail(PKM_ERR_UNSUPPORTED, "row too large for the gather ring");
  a.slots = slots;
  a.warp_smem = ws;
  const int smem = (int)(ws * NW);
  auto kern = gather_kernel<RowT, VPL, MODE, DOT, NW, FULL>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return check_cuda("cudaFuncSetAttribute(gather)");
  int64_t blocks = (items_upper + NW - 1) / NW;
  blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, num_sms()));
  kern<<<(unsigned)blocks, NW * 32, smem, st>>>(a);
  return check_cuda("gather_kernel");
}

template <typename RowT, int VPL, int MODE, bool DOT>
static int launch_full(GatherArgs a, int64_t items_upper, cudaStream_t st) {
  if (a.row_bytes == (int64_t)VPL * 512) return launch_one<RowT, VPL, MODE, DOT, true>(a, items_upper, st);
  return launch_one<RowT, VPL, MODE, DOT, false>(a, items_upper, st);
}

template <typename RowT, int MODE, bool DOT>
static int launch_vpl(GatherArgs a, int64_t items_upper, cudaStream_t st) {
  const int64_t v = (a.row_bytes + 511) / 512;
  if (v <= 1) return launch_full<RowT, 1, MODE, DOT>(a, items_upper, st);
  if (v <= 2) return launch_full<RowT, 2, MODE, DOT>(a, items_upper, st);
  if (v <= 4) return launch_full<RowT, 4, MODE, DOT>(a, items_upper, st);
  if (v <= 8) return launch_full<RowT, 8, MODE, DOT>(a, items_upper, st);
  return fail(PKM_ERR_UNSUPPORTED, "rows above 4096 bytes are not supported");
}

template <typename RowT>
static int launch_mode(bool seg, bool dot, GatherArgs a, int64_t items_upper, cudaStream_t st) {
  if (!seg) {
    return dot ? launch_vpl<RowT, G_BAG, true>(a, items_upper, st)
               : launch_vpl<RowT, G_BAG, false>(a, items_upper, st);
  }
  return dot ? launch_vpl<RowT, G_SEG, true>(a, items_upper, st)
             : launch_vpl<RowT, G_SEG, false>(a, items_upper, st);
}

int gather_launch(int row_dtype, bool seg, bool dot, GatherArgs a, int64_t items_upper, cudaStream_t st) {
  if (row_dtype == PKM_DT_F32) return launch_mode<float>(seg, dot, a, items_upper, st);
  if (row_dtype == PKM_DT_BF16) return launch_mode<__nv_bfloat16>(seg, dot, a, items_upper, st);
  return launch_mode<__half>(seg, dot, a, items_upper, st);
}

// ---------------------------------------------------------------------------
// K4 helper kernels
// ---------------------------------------------------------------------------
// Row key of every occurrence (invalid indices map to the sentinel row K)
// and the per-row occurrence counts.
__global__ void bwd_keys_kernel(const int64_t* __restrict__ idx, int64_t M, int64_t K,
                                uint32_t* __restrict__ keys, int32_t* __restrict__ counts, void* grad_psw,
                                int grad_psw_dtype, uint32_t* err) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < M; o += stride) {
    const int64_t k = idx[o];
    uint32_t key;
    if (k < 0 || k >= K) {
      key = (uint32_t)K;  // sentinel row: never aggregated, its per-sample gradient is 0
      raise_err(err, PKM_DEVERR_INDEX);
      if (grad_psw) st_f(grad_psw, grad_psw_dtype, o, 0.f);
    } else {
      key = (uint32_t)k;
    }
    keys[o] = key;
    atomicAdd(&counts[key], 1);
  }
}

// One descriptor per chunk of at most `chunk` occurrences of a row (one for an
// empty row, so that its zero gradient row is written too).
__global__ void items_fill_kernel(const int32_t* __restrict__ counts, const I4* __restrict__ offs, int64_t K,
                                  int chunk, int4* __restrict__ desc, int32_t* n_items,
                                  int32_t* __restrict__ row_counts) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < K; k += stride) {
    const int c = counts[k];
    const I4 o = offs[k];
    const int items = offs[k + 1].y - o.y;
    for (int j = 0; j < items; ++j) {
      const int b = o.x + j * chunk;
      const int e = min(o.x + c, b + chunk);
      desc[o.y + j] = make_int4((int)k, b, e, items > 1 ? o.z + j : -1);
    }
    if (row_counts) row_counts[k] = c;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *n_items = offs[K].y;
}

// Destination rows of the bag backward's weight gradient: the local gradient,
// or (data-parallel) row r of the table goes to rank r / shard_rows, row
// rank * shard_rows + r % shard_rows of that rank's receive buffer.
struct GradDest {
  void* out;
  int64_t shard_rows;  // 0: local
  int rank;
  char* base[kMaxShards];
  __device__ __forceinline__ void* row(int64_t r, int64_t D, int dt) const {
    if (shard_rows == 0) return static_cast<char*>(out) + r * D * dtype_size_dev(dt);
    const int64_t o = r / shard_rows;
    return base[o] + (rank * shard_rows + (r - o * shard_rows)) * D * dtype_size_dev(dt);
  }
};

// Rows split over several chunks: sum the chunk partials in chunk order.
// A warp checks 32 rows at once and sums only the split ones (rare: a row
// needs more than one chunk of occurrences).
__global__ void reduce_partials_kernel(const I4* __restrict__ offs, int64_t k0, int64_t k1,
                                       const float* __restrict__ partials, int64_t D,
                                       const __grid_constant__ GradDest dest, int out_dtype) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t g = k0 + ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 32; g < k1;
       g += warps * 32) {
    const int64_t mine = g + lane;
    bool split = false;
    if (mine < k1) split = offs[mine + 1].y - offs[mine].y > 1;
    unsigned todo = __ballot_sync(0xffffffffu, split);
    while (todo) {
      const int64_t k = g + __ffs(todo) - 1;
      todo &= todo - 1;
      const I4 o = offs[k];
      const int items = offs[k + 1].y - o.y;
      const float* base = partials + (int64_t)o.z * D;
      void* row = dest.row(k, D, out_dtype);
      for (int64_t e = lane; e < D; e += 32) {
        float s = 0.f;
        for (int j = 0; j < items; ++j) s += base[(int64_t)j * D + e];
        st_f(row, out_dtype, e, s);
      }
    }
  }
  if (dest.shard_rows > 0) __threadfence_system();
}

// Zero rows for every table row (data-parallel backward of an empty bag set:
// this rank's slots of all owners' receive buffers).
__global__ void zero_rows_kernel(int64_t K, int64_t D, const __grid_constant__ GradDest dest, int out_dtype) {
  const int64_t vec = D * dtype_size_dev(out_dtype) / 16;
  const int64_t total = K * vec;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec;
    reinterpret_cast<uint4*>(dest.row(r, D, out_dtype))[i - r * vec] = make_uint4(0, 0, 0, 0);
  }
  if (dest.shard_rows > 0) __threadfence_system();
}

// Owner side of the data-parallel exchange: sum the world partial copies of
// this rank's shard rows in source order 0..world-1, scale, and store the
// result into row (rank * shard_rows + r) of every rank's gradient.  bf16
// copies are added as packed pairs (each addition rounded to bf16, as a
// bf16 all-reduce does; with two ranks that is the single rounding of the
// exact sum), fp32 in fp32.  Each thread handles kShardVec 16-byte vectors
// with all their loads in flight before the additions.
constexpr int kShardVec = 4;
__device__ __forceinline__ uint32_t add_pair(uint32_t a, uint32_t b, bool bf16) {
  if (bf16) {
    __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&a), y = *reinterpret_cast<__nv_bfloat162*>(&b);
    __nv_bfloat162 r = __hadd2(x, y);
    return *reinterpret_cast<uint32_t*>(&r);
  }
  return __float_as_uint(__uint_as_float(a) + __uint_as_float(b));
}
__device__ __forceinline__ uint4 add_vec(const uint4& a, const uint4& b, bool bf16) {
  return make_uint4(add_pair(a.x, b.x, bf16), add_pair(a.y, b.y, bf16), add_pair(a.z, b.z, bf16),
                    add_pair(a.w, b.w, bf16));
}
__device__ __forceinline__ uint4 scale_vec(const uint4& a, float s, bool bf16) {
  if (bf16) {
    float f[8];
    VecTraits<__nv_bfloat16>::unpack(a, f);
    uint4 r;
    uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i] * s, f[2 * i + 1] * s);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return r;
  }
  return make_uint4(__float_as_uint(__uint_as_float(a.x) * s), __float_as_uint(__uint_as_float(a.y) * s),
                    __float_as_uint(__uint_as_float(a.z) * s), __float_as_uint(__uint_as_float(a.w) * s));
}

__global__ void __launch_bounds__(256) shard_reduce_kernel(const uint4* __restrict__ recv, int64_t shard_vecs,
                                                           int64_t n_vecs, int64_t row_vecs, int world, int rank,
                                                           bool bf16, float scale,
                                                           const __grid_constant__ GradDest dest) {
  const int64_t n_chunks = (n_vecs + (int64_t)blockDim.x * kShardVec - 1) / ((int64_t)blockDim.x * kShardVec);
  for (int64_t chunk = blockIdx.x; chunk < n_chunks; chunk += gridDim.x) {
  const int64_t v0 = (chunk * blockDim.x) * kShardVec + threadIdx.x;
  uint4 acc[kShardVec];
  bool live[kShardVec];
#pragma unroll
  for (int u = 0; u < kShardVec; ++u) {
    const int64_t v = v0 + (int64_t)u * blockDim.x;
    live[u] = v < n_vecs;
    acc[u] = live[u] ? recv[v] : make_uint4(0, 0, 0, 0);
  }
  for (int s = 1; s < world; ++s) {
    uint4 x[kShardVec];
#pragma unroll
    for (int u = 0; u < kShardVec; ++u) {
      const int64_t v = v0 + (int64_t)u * blockDim.x;
      x[u] = live[u] ? recv[(int64_t)s * shard_vecs + v] : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kShardVec; ++u) acc[u] = add_vec(acc[u], x[u], bf16);
  }
  if (scale != 1.f) {
#pragma unroll
    for (int u = 0; u < kShardVec; ++u) acc[u] = scale_vec(acc[u], scale, bf16);
  }
  const int64_t base = (int64_t)rank * shard_vecs;  // this shard's first vector in a full gradient
  for (int d = 0; d < world; ++d) {
    uint4* dst = reinterpret_cast<uint4*>(dest.base[d]) + base;
#pragma unroll
    for (int u = 0; u < kShardVec; ++u) {
      const int64_t v = v0 + (int64_t)u * blockDim.x;
      if (live[u]) dst[v] = acc[u];
    }
  }
  }
  (void)row_vecs;
  __threadfence_system();
}

// In-switch variant (NVLS): every rank's gradient sits in one symmetric
// buffer with a multicast mapping.  The owner of a shard reads each 16-byte
// vector of its rows through the multicast address with
// multimem.ld_reduce, which returns the sum over all ranks' copies (bf16
// accumulated in fp32 in the switch), and stores it with multimem.st to the
// multicast address of the gradient buffer, which writes every rank's copy.
// Each rank's NVLink carries its own rows out once for the reduction and the
// reduced shard out once for the broadcast.
constexpr int kMmVec = 8;
__global__ void __launch_bounds__(256) multimem_allreduce_kernel(const char* mc_src, char* mc_dst, int64_t v_begin,
                                                                 int64_t n_vecs, bool bf16, float scale) {
  const int64_t n_chunks = (n_vecs + (int64_t)blockDim.x * kMmVec - 1) / ((int64_t)blockDim.x * kMmVec);
  for (int64_t chunk = blockIdx.x; chunk < n_chunks; chunk += gridDim.x) {
    const int64_t v0 = chunk * blockDim.x * kMmVec + threadIdx.x;
    uint4 r[kMmVec];
#pragma unroll
    for (int u = 0; u < kMmVec; ++u) {
      const int64_t v = v0 + (int64_t)u * blockDim.x;
      r[u] = make_uint4(0, 0, 0, 0);
      if (v < n_vecs) {
        const char* a = mc_src + (v_begin + v) * 16;
        if (bf16)
          asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                       : "=r"(r[u].x), "=r"(r[u].y), "=r"(r[u].z), "=r"(r[u].w)
                       : "l"(a)
                       : "memory");
        else
          asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(r[u].x), "=r"(r[u].y), "=r"(r[u].z), "=r"(r[u].w)
                       : "l"(a)
                       : "memory");
      }
    }
#pragma unroll
    for (int u = 0; u < kMmVec; ++u) {
      const int64_t v = v0 + (int64_t)u * blockDim.x;
      if (v < n_vecs) {
        uint4 x = scale != 1.f ? scale_vec(r[u], scale, bf16) : r[u];
        char* d = mc_dst + (v_begin + v) * 16;
        asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(d), "r"(x.x), "r"(x.y),
                     "r"(x.z), "r"(x.w)
                     : "memory");
      }
    }
  }
  __threadfence_system();
}

// Row-owner optimizer step (reduce-scatter -> owner update -> all-gather):
// the owner sums the world copies of its shard's gradient rows exactly as
// shard_reduce_kernel does, applies plain SGD to its rows of the table,
//   d  = g + weight_decay * p        (rounded to the table dtype; skipped when 0)
//   p' = p - lr * d                  (one fused multiply-add, rounded once)
// which is torch.optim.SGD's foreach update without momentum, and stores the
// new rows into row (rank * shard_rows + r) of every rank's table.
__device__ __forceinline__ void unpack_vec(const uint4& a, float (&f)[8], bool bf16) {
  if (bf16) {
    VecTraits<__nv_bfloat16>::unpack(a, f);
  } else {
    f[0] = __uint_as_float(a.x), f[1] = __uint_as_float(a.y), f[2] = __uint_as_float(a.z),
    f[3] = __uint_as_float(a.w);
    f[4] = f[5] = f[6] = f[7] = 0.f;
  }
}
__device__ __forceinline__ uint4 pack_vec(const float (&f)[8], bool bf16) {
  if (bf16) {
    uint4 r;
    uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return r;
  }
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
}

__global__ void __launch_bounds__(256) shard_sgd_kernel(const uint4* __restrict__ recv, int64_t shard_vecs,
                                                       int64_t n_vecs, int world, int rank, bool bf16, float scale,
                                                       float lr, float wd, const __grid_constant__ GradDest dest) {
  const int64_t n_chunks = (n_vecs + (int64_t)blockDim.x * kShardVec - 1) / ((int64_t)blockDim.x * kShardVec);
  const int64_t base = (int64_t)rank * shard_vecs;  // this shard's first vector in a full table
  const uint4* own = reinterpret_cast<const uint4*>(dest.base[rank]) + base;
  const int n = bf16 ? 8 : 4;
  for (int64_t chunk = blockIdx.x; chunk < n_chunks; chunk += gridDim.x) {
    const int64_t v0 = (chunk * blockDim.x) * kShardVec + threadIdx.x;
    uint4 acc[kShardVec], par[kShardVec];
    bool live[kShardVec];
#pragma unroll
    for (int u = 0; u < kShardVec; ++u) {
      const int64_t v = v0 + (int64_t)u * blockDim.x;
      live[u] = v < n_vecs;
      acc[u] = live[u] ? recv[v] : make_uint4(0, 0, 0, 0);
      par[u] = live[u] ? own[v] : make_uint4(0, 0, 0, 0);
    }
    for (int s = 1; s < world; ++s) {
      uint4 x[kShardVec];
#pragma unroll
      for (int u = 0; u < kShardVec; ++u) {
        const int64_t v = v0 + (int64_t)u * blockDim.x;
        x[u] = live[u] ? recv[(int64_t)s * shard_vecs + v] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kShardVec; ++u) acc[u] = add_vec(acc[u], x[u], bf16);
    }
#pragma unroll
    for (int u = 0; u < kShardVec; ++u) {
      if (scale != 1.f) acc[u] = scale_vec(acc[u], scale, bf16);
      float g[8], p[8];
      unpack_vec(acc[u], g, bf16);
      unpack_vec(par[u], p, bf16);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i >= n) break;
        float d = g[i];
        if (wd != 0.f) {
          d = __fmaf_rn(wd, p[i], d);
          if (bf16) d = __bfloat162float(__float2bfloat16_rn(d));
        }
        p[i] = __fmaf_rn(-lr, d, p[i]);
      }
      par[u] = pack_vec(p, bf16);
    }
    for (int d = 0; d < world; ++d) {
      uint4* dst = reinterpret_cast<uint4*>(dest.base[d]) + base;
#pragma unroll
      for (int u = 0; u < kShardVec; ++u) {
        const int64_t v = v0 + (int64_t)u * blockDim.x;
        if (live[u]) dst[v] = par[u];
      }
    }
  }
  __threadfence_system();
}

constexpr int kChunk = 256;

struct BwdLayout {
  size_t counts, offs, keys_a, keys_b, vals_a, vals_b, w_sorted, hist, sums_i, sums_4, desc, n_items,
      partials, total;
};

static size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }

static BwdLayout bwd_layout(int64_t M, int64_t K, int64_t D) {
  BwdLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off += up256(bytes);
    return at;
  };
  const int64_t tiles = sort_tiles(M);
  const int64_t nh = (int64_t)kRadixMax * tiles;
  const int64_t max_items = K + (M + kChunk - 1) / kChunk + 1;
  const int64_t max_partial = 2 * ((M + kChunk - 1) / kChunk) + 2;
  L.counts = take(sizeof(int32_t) * (K + 1));
  L.offs = take(sizeof(I4) * (K + 2));
  L.keys_a = take(sizeof(uint32_t) * M);
  L.keys_b = take(sizeof(uint32_t) * M);
  L.vals_a = take(sizeof(int32_t) * M);
  L.vals_b = take(sizeof(int32_t) * M);
  L.w_sorted = take(sizeof(float) * M);
  L.hist = take(sizeof(int) * (nh + 1));
  L.sums_i = take(sizeof(int) * (scan_blocks(nh) + 1));
  L.sums_4 = take(sizeof(I4) * (scan_blocks(K + 1) + 1));
  L.desc = take(sizeof(int4) * max_items);
  L.n_items = take(sizeof(int32_t));
  L.partials = take(sizeof(float) * max_partial * D);
  L.total = off;
  return L;
}

static int bits_for(int64_t v) {
  int b = 0;
  while (b < 63 && (int64_t(1) << b) <= v) ++b;
  return std::max(b, 1);
}

}  // namespace pkm

using namespace pkm;

// ---------------------------------------------------------------------------
// argument checks shared by the entry points
// ---------------------------------------------------------------------------
static int check_bag_common(const int64_t* indices, int64_t n_bags, int64_t bag_size, int64_t num_rows,
                            int64_t dim, int row_dtype) {
  if (n_bags < 0 || bag_size < 0 || num_rows < 0 || dim <= 0)
    return fail(PKM_ERR_INVALID_ARG, "negative size or dim <= 0");
  if (!valid_dtype(row_dtype)) return fail(PKM_ERR_INVALID_ARG, "bad table dtype");
  if (n_bags * bag_size > 0 && indices == nullptr) return fail(PKM_ERR_INVALID_ARG, "indices is NULL");
  if (n_bags * bag_size >= (int64_t(1) << 31))
    return fail(PKM_ERR_UNSUPPORTED, "n_bags * bag_size must stay below 2^31");
  if (num_rows >= (int64_t(1) << 31) - 1) return fail(PKM_ERR_UNSUPPORTED, "num_rows must stay below 2^31-1");
  const int64_t rb = dim * dtype_size(row_dtype);
  if (rb % 16 != 0) return fail(PKM_ERR_UNSUPPORTED, "row bytes (dim * element size) must be a multiple of 16");
  if (rb > 4096) return fail(PKM_ERR_UNSUPPORTED, "row bytes above 4096 are not supported");
  return PKM_OK;
}

extern "C" int pkm_bag_fwd(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                           int weight_dtype, int64_t n_bags, int64_t bag_size, int64_t num_rows, int64_t dim,
                           void* out, int out_dtype, uint32_t* dev_err, void* stream) {
  int rc = check_bag_common(indices, n_bags, bag_size, num_rows, dim, weight_dtype);
  if (rc) return rc;
  if (!valid_dtype(out_dtype) || (psw && !valid_dtype(psw_dtype)))
    return fail(PKM_ERR_INVALID_ARG, "bad dtype");
  if (n_bags == 0) return PKM_OK;
  if (out == nullptr) return fail(PKM_ERR_INVALID_ARG, "out is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bag_size == 0 || num_rows == 0) {
    cudaMemsetAsync(out, 0, (size_t)(n_bags * dim * dtype_size(out_dtype)), st);
    if (bag_size > 0 && dev_err)  // every index is out of range of an empty table
      cudaMemsetAsync(dev_err, PKM_DEVERR_INDEX, 1, st);
    return check_cuda("pkm_bag_fwd memset");
  }
  if (weight == nullptr || !aligned16(weight)) return fail(PKM_ERR_INVALID_ARG, "weight NULL or not 16-byte aligned");
  GatherArgs a{};
  a.rows = static_cast<const char*>(weight);
  a.row_bytes = dim * dtype_size(weight_dtype);
  a.dim = dim;
  a.num_rows = num_rows;
  a.idx = indices;
  a.w = psw;
  a.w_dtype = psw ? psw_dtype : PKM_DT_F32;
  a.L = bag_size;
  a.n_items = n_bags;
  a.out = out;
  a.out_dtype = out_dtype;
  a.err = dev_err;
  return gather_launch(weight_dtype, false, false, a, n_bags, st);
}

extern "C" int pkm_bag_bwd2(const int64_t* indices, const void* a_w, int a_dtype, const void* gbar,
                            int gbar_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size,
                            int64_t num_rows, int64_t dim, void* d_grad_out, int d_grad_out_dtype, void* d_a,
                            int d_a_dtype, uint32_t* dev_err, void* stream) {
  int rc = check_bag_common(indices, n_bags, bag_size, num_rows, dim, gbar_dtype);
  if (rc) return rc;
  if (!valid_dtype(d_grad_out_dtype) || (a_w && !valid_dtype(a_dtype)) || (d_a && !valid_dtype(d_a_dtype)))
    return fail(PKM_ERR_INVALID_ARG, "bad dtype");
  if (d_a && !a_w) return fail(PKM_ERR_INVALID_ARG, "d_a requested without per-sample weights");
  if (n_bags == 0) return PKM_OK;
  if (d_grad_out == nullptr) return fail(PKM_ERR_INVALID_ARG, "d_grad_out is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bag_size == 0 || num_rows == 0) {
    cudaMemsetAsync(d_grad_out, 0, (size_t)(n_bags * dim * dtype_size(d_grad_out_dtype)), st);
    if (d_a && bag_size > 0) cudaMemsetAsync(d_a, 0, (size_t)(n_bags * bag_size * dtype_size(d_a_dtype)), st);
    if (bag_size > 0 && dev_err) cudaMemsetAsync(dev_err, PKM_DEVERR_INDEX, 1, st);
    return check_cuda("pkm_bag_bwd2 memset");
  }
  if (gbar == nullptr || !aligned16(gbar)) return fail(PKM_ERR_INVALID_ARG, "gbar NULL or not 16-byte aligned");
  if (d_a && (grad_out == nullptr || !aligned16(grad_out)))
    return fail(PKM_ERR_INVALID_ARG, "grad_out NULL or not 16-byte aligned");
  GatherArgs a{};
  a.rows = static_cast<const char*>(gbar);
  a.row_bytes = dim * dtype_size(gbar_dtype);
  a.dim = dim;
  a.num_rows = num_rows;
  a.idx = indices;
  a.w = a_w;
  a.w_dtype = a_w ? a_dtype : PKM_DT_F32;
  a.L = bag_size;
  a.n_items = n_bags;
  a.out = d_grad_out;
  a.out_dtype = d_grad_out_dtype;
  a.dotvec = static_cast<const char*>(grad_out);
  a.dotout = d_a;
  a.dotout_dtype = d_a_dtype;
  a.err = dev_err;
  return gather_launch(gbar_dtype, false, d_a != nullptr, a, n_bags, st);
}

extern "C" int pkm_bag_bwd_workspace(int64_t n_bags, int64_t bag_size, int64_t num_rows, int64_t dim,
                                     size_t* bytes) {
  if (!bytes) return fail(PKM_ERR_INVALID_ARG, "bytes is NULL");
  if (n_bags < 0 || bag_size < 0 || num_rows < 0 || dim <= 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  *bytes = bwd_layout(n_bags * bag_size, num_rows, dim).total;
  return PKM_OK;
}

// Segment pass (+ per-sample dots) and the partial-row sums for the table
// rows [row_begin, row_end) of a sorted workspace.
static int bag_bwd_rows(const void* grad_out, const void* weight, int weight_dtype, int64_t n_bags,
                        int64_t bag_size, int64_t K, int64_t D, const GradDest& dest, int grad_weight_dtype,
                        void* grad_psw, int grad_psw_dtype, const int32_t* sorted, const float* w_sorted,
                        const int4* desc, const int32_t* n_items, const I4* offs, float* partials, uint32_t* dev_err,
                        const int32_t* src_of, int64_t n_src, int64_t row_begin, int64_t row_end, cudaStream_t st) {
  if (row_end <= row_begin) return PKM_OK;
  const int64_t M = n_bags * bag_size;
  GatherArgs a{};
  a.rows = static_cast<const char*>(grad_out);
  a.row_bytes = D * dtype_size(weight_dtype);
  a.dim = D;
  a.num_rows = n_bags;
  a.occ = sorted;
  a.occ_w = w_sorted;
  a.L = bag_size;
  a.n_items_dev = n_items;
  a.item_desc = desc;
  a.dotvec = static_cast<const char*>(weight);
  a.dotout = grad_psw;
  a.dotout_dtype = grad_psw_dtype;
  a.out = dest.out;
  a.out_dtype = grad_weight_dtype;
  a.partials = partials;
  a.err = dev_err;
  a.src_of = src_of;
  a.n_src = n_src;
  a.row_lo = row_begin;
  a.row_hi = row_end;
  a.shard_rows = dest.shard_rows;
  a.shard_rank = dest.rank;
  for (int i = 0; i < kMaxShards; ++i) a.shard_base[i] = dest.base[i];
  const int64_t items_upper = K + (M + kChunk - 1) / kChunk + 1;
  int rc = gather_launch(weight_dtype, true, grad_psw != nullptr, a, items_upper, st);
  if (rc) return rc;
  // rows that were split over several chunks
  const int64_t nk = row_end - row_begin;
  int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((nk + 255) / 256, (int64_t)num_sms() * 8));
  reduce_partials_kernel<<<(unsigned)blocks, 256, 0, st>>>(offs, row_begin, row_end, partials, D, dest,
                                                           grad_weight_dtype);
  return check_cuda("pkm_bag_bwd");
}

// Phases of the bag backward: the sort (keys, scan, radix sort, chunk
// descriptors) and the segment pass over a range of table rows, which can be
// run as separate calls on the same workspace (the rows in any number of
// ranges, each once, after the sort).
enum { kBwdAll = 0, kBwdSort = 1, kBwdRows = 2 };

static int bag_bwd_impl(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                        int weight_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size, int64_t num_rows,
                        int64_t dim, const GradDest& dest, int grad_weight_dtype, void* grad_psw,
                        int grad_psw_dtype, int32_t* row_counts, void* workspace, size_t workspace_bytes,
                        uint32_t* dev_err, void* stream, const int32_t* src_of = nullptr, int64_t n_src = 0,
                        int phase = kBwdAll, int64_t row_begin = 0, int64_t row_end = -1) {
  int rc = check_bag_common(indices, n_bags, bag_size, num_rows, dim, weight_dtype);
  if (rc) return rc;
  if (!valid_dtype(grad_weight_dtype) || (psw && !valid_dtype(psw_dtype)) ||
      (grad_psw && !valid_dtype(grad_psw_dtype)))
    return fail(PKM_ERR_INVALID_ARG, "bad dtype");
  if (grad_psw && !psw) return fail(PKM_ERR_INVALID_ARG, "grad_psw requested without per-sample weights");
  if (num_rows > 0 && dest.shard_rows == 0 && dest.out == nullptr)
    return fail(PKM_ERR_INVALID_ARG, "grad_weight is NULL");
  const int64_t M = n_bags * bag_size;
  const int64_t K = num_rows;
  const int64_t D = dim;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M > 0 && (grad_out == nullptr || !aligned16(grad_out)))
    return fail(PKM_ERR_INVALID_ARG, "grad_out NULL or not 16-byte aligned");
  if (grad_psw && (weight == nullptr || !aligned16(weight)))
    return fail(PKM_ERR_INVALID_ARG, "weight NULL or not 16-byte aligned");
  const BwdLayout L = bwd_layout(M, K, D);
  if (row_end < 0) row_end = K;
  if (row_begin < 0 || row_begin > row_end || row_end > K) return fail(PKM_ERR_INVALID_ARG, "bad row range");
  if (phase != kBwdAll && dest.shard_rows > 0) return fail(PKM_ERR_UNSUPPORTED, "phased backward writes locally");
  if ((M == 0 || K == 0) && phase != kBwdAll) {
    if (phase == kBwdRows && row_end > row_begin)
      cudaMemsetAsync(static_cast<char*>(dest.out) + row_begin * D * dtype_size(grad_weight_dtype), 0,
                      (size_t)((row_end - row_begin) * D * dtype_size(grad_weight_dtype)), st);
    if (phase == kBwdSort) {
      if (row_counts && K > 0) cudaMemsetAsync(row_counts, 0, sizeof(int32_t) * K, st);
      if (grad_psw && M > 0) cudaMemsetAsync(grad_psw, 0, (size_t)(M * dtype_size(grad_psw_dtype)), st);
      if (M > 0 && dev_err) cudaMemsetAsync(dev_err, PKM_DEVERR_INDEX, 1, st);
    }
    return check_cuda("pkm_bag_bwd memset");
  }
  if (M == 0 || K == 0) {
    if (K > 0 && dest.shard_rows > 0) {
      const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((K * D / 8 + 255) / 256, (int64_t)num_sms() * 8));
      zero_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(K, D, dest, grad_weight_dtype);
    } else if (K > 0) {
      cudaMemsetAsync(dest.out, 0, (size_t)(K * D * dtype_size(grad_weight_dtype)), st);
    }
    if (row_counts && K > 0) cudaMemsetAsync(row_counts, 0, sizeof(int32_t) * K, st);
    if (grad_psw && M > 0) cudaMemsetAsync(grad_psw, 0, (size_t)(M * dtype_size(grad_psw_dtype)), st);
    if (M > 0 && dev_err) cudaMemsetAsync(dev_err, PKM_DEVERR_INDEX, 1, st);
    return check_cuda("pkm_bag_bwd memset");
  }
  if (workspace == nullptr || workspace_bytes < L.total)
    return fail(PKM_ERR_WORKSPACE, "workspace smaller than pkm_bag_bwd_workspace()");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(PKM_ERR_INVALID_ARG, "workspace must be 256-byte aligned");
  char* ws = static_cast<char*>(workspace);
  int32_t* counts = reinterpret_cast<int32_t*>(ws + L.counts);
  I4* offs = reinterpret_cast<I4*>(ws + L.offs);
  uint32_t* keys_a = reinterpret_cast<uint32_t*>(ws + L.keys_a);
  uint32_t* keys_b = reinterpret_cast<uint32_t*>(ws + L.keys_b);
  int32_t* vals_a = reinterpret_cast<int32_t*>(ws + L.vals_a);
  int32_t* vals_b = reinterpret_cast<int32_t*>(ws + L.vals_b);
  float* w_sorted = reinterpret_cast<float*>(ws + L.w_sorted);
  int* hist = reinterpret_cast<int*>(ws + L.hist);
  int* sums_i = reinterpret_cast<int*>(ws + L.sums_i);
  I4* sums_4 = reinterpret_cast<I4*>(ws + L.sums_4);
  int4* desc = reinterpret_cast<int4*>(ws + L.desc);
  int32_t* n_items = reinterpret_cast<int32_t*>(ws + L.n_items);
  float* partials = reinterpret_cast<float*>(ws + L.partials);

  const int nsm = num_sms();
  int sort_rb, sort_passes;
  sort_plan(bits_for(K), sort_rb, sort_passes);
  if (phase == kBwdRows) {
    int32_t* sorted = sort_passes & 1 ? vals_a : vals_b;  // where the last radix pass wrote the values
    return bag_bwd_rows(grad_out, weight, weight_dtype, n_bags, bag_size, K, D, dest, grad_weight_dtype, grad_psw,
                        grad_psw_dtype, sorted, w_sorted, desc, n_items, offs, partials, dev_err, src_of, n_src,
                        row_begin, row_end, st);
  }
  // 1. row keys + counts
  cudaMemsetAsync(counts, 0, sizeof(int32_t) * (K + 1), st);
  {
    int64_t blocks = std::min<int64_t>((M + 255) / 256, (int64_t)nsm * 16);
    bwd_keys_kernel<<<(unsigned)blocks, 256, 0, st>>>(indices, M, K, keys_a, counts, grad_psw, grad_psw_dtype,
                                                      dev_err);
  }
  // 2. segment offsets, chunk counts and partial-row offsets per row
  scan_exclusive<I4>(RowScanLoad{counts, K, kChunk}, K + 1, offs, sums_4, st);
  // 3. stable radix sort of occurrence ids by row (sentinel row K included)
  {
    const int passes = sort_passes;
    const int rb = sort_rb;
    const int64_t tiles = sort_tiles(M);
    const uint32_t* kin = keys_a;
    const int32_t* vin = nullptr;
    uint32_t* kbuf[2] = {keys_b, keys_a};
    int32_t* vbuf[2] = {vals_a, vals_b};
    for (int p = 0; p < passes; ++p) {
      const bool last = p == passes - 1;
      uint32_t* kout = last ? nullptr : kbuf[p & 1];
      int32_t* vout = vbuf[p & 1];
      const int shift = rb * p;
      auto pass = [&](auto rbc) {
        constexpr int RB = decltype(rbc)::value;
        radix_upsweep_kernel<RB><<<(unsigned)tiles, kSortThreads, 0, st>>>(kin, M, shift, hist, tiles);
        scan_exclusive<int>(IntLoad{hist}, (int64_t)(1 << RB) * tiles, hist, sums_i, st);
        radix_downsweep_kernel<RB><<<(unsigned)tiles, kSortThreads, 0, st>>>(
            kin, vin, M, shift, hist, tiles, kout, vout, last ? psw : nullptr, psw_dtype,
            last ? w_sorted : nullptr);
      };
      if (rb == 10)
        pass(std::integral_constant<int, 10>{});
      else if (rb == 9)
        pass(std::integral_constant<int, 9>{});
      else
        pass(std::integral_constant<int, 8>{});
      kin = kout;
      vin = vout;
    }
    // vin now holds the sorted occurrence ids
    // 4. chunk descriptors
    {
      int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((K + 255) / 256, (int64_t)nsm * 8));
      items_fill_kernel<<<(unsigned)blocks, 256, 0, st>>>(counts, offs, K, kChunk, desc, n_items, row_counts);
    }
    rc = check_cuda("pkm_bag_bwd prologue");
    if (rc) return rc;
    if (phase == kBwdSort) return PKM_OK;
    return bag_bwd_rows(grad_out, weight, weight_dtype, n_bags, bag_size, K, D, dest, grad_weight_dtype, grad_psw,
                        grad_psw_dtype, vin, w_sorted, desc, n_items, offs, partials, dev_err, src_of, n_src,
                        row_begin, row_end, st);
  }
  return check_cuda("pkm_bag_bwd");
}

extern "C" int pkm_bag_bwd(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                           int weight_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size,
                           int64_t num_rows, int64_t dim, void* grad_weight, int grad_weight_dtype,
                           void* grad_psw, int grad_psw_dtype, int32_t* row_counts, void* workspace,
                           size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  GradDest dest{};
  dest.out = grad_weight;
  return bag_bwd_impl(indices, psw, psw_dtype, weight, weight_dtype, grad_out, n_bags, bag_size, num_rows, dim, dest,
                      grad_weight_dtype, grad_psw, grad_psw_dtype, row_counts, workspace, workspace_bytes, dev_err,
                      stream);
}

static int shard_dest(GradDest& dest, void* const* bases, int world, int rank, int64_t shard_rows, int64_t num_rows,
                      int64_t dim, int dtype) {
  if (world < 1 || world > kMaxShards || rank < 0 || rank >= world)
    return fail(PKM_ERR_INVALID_ARG, "need 1 <= world <= 8 and 0 <= rank < world");
  if (!bases) return fail(PKM_ERR_INVALID_ARG, "shard base pointers are NULL");
  if (shard_rows <= 0 || shard_rows * world < num_rows)
    return fail(PKM_ERR_INVALID_ARG, "shard_rows * world must cover num_rows");
  if ((dim * dtype_size(dtype)) % 16 != 0) return fail(PKM_ERR_UNSUPPORTED, "row bytes must be a multiple of 16");
  dest.out = nullptr;
  dest.shard_rows = shard_rows;
  dest.rank = rank;
  for (int i = 0; i < kMaxShards; ++i) dest.base[i] = nullptr;
  for (int i = 0; i < world; ++i) {
    if (!bases[i] || !aligned16(bases[i])) return fail(PKM_ERR_INVALID_ARG, "shard base NULL or not 16-byte aligned");
    dest.base[i] = static_cast<char*>(bases[i]);
  }
  return PKM_OK;
}

extern "C" int pkm_bag_bwd_sharded(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                                   int weight_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size,
                                   int64_t num_rows, int64_t dim, void* const* recv_bases, int world, int rank,
                                   int64_t shard_rows, int grad_weight_dtype, void* grad_psw, int grad_psw_dtype,
                                   int32_t* row_counts, void* workspace, size_t workspace_bytes, uint32_t* dev_err,
                                   void* stream) {
  GradDest dest{};
  int rc = shard_dest(dest, recv_bases, world, rank, shard_rows, num_rows, dim, grad_weight_dtype);
  if (rc) return rc;
  return bag_bwd_impl(indices, psw, psw_dtype, weight, weight_dtype, grad_out, n_bags, bag_size, num_rows, dim, dest,
                      grad_weight_dtype, grad_psw, grad_psw_dtype, row_counts, workspace, workspace_bytes, dev_err,
                      stream);
}

extern "C" int pkm_grad_shard_reduce(const void* recv, int dtype, int64_t num_rows, int64_t dim, int world, int rank,
                                     int64_t shard_rows, void* const* grad_bases, float scale, int max_blocks,
                                     void* stream) {
  if (dtype != PKM_DT_F32 && dtype != PKM_DT_BF16) return fail(PKM_ERR_UNSUPPORTED, "dtype must be f32 or bf16");
  GradDest dest{};
  int rc = shard_dest(dest, grad_bases, world, rank, shard_rows, num_rows, dim, dtype);
  if (rc) return rc;
  if (!recv || !aligned16(recv)) return fail(PKM_ERR_INVALID_ARG, "recv NULL or not 16-byte aligned");
  const int64_t rows = std::min<int64_t>(shard_rows, num_rows - (int64_t)rank * shard_rows);
  if (rows <= 0) return PKM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t row_vecs = dim * dtype_size(dtype) / 16;
  const int64_t n_vecs = rows * row_vecs;
  const int64_t per_block = 256 * kShardVec;
  int64_t blocks = (n_vecs + per_block - 1) / per_block;
  if (max_blocks > 0) blocks = std::min<int64_t>(blocks, max_blocks);
  shard_reduce_kernel<<<(unsigned)blocks, 256, 0, st>>>(static_cast<const uint4*>(recv), shard_rows * row_vecs,
                                                        n_vecs, row_vecs, world, rank, dtype == PKM_DT_BF16, scale,
                                                        dest);
  return check_cuda("pkm_grad_shard_reduce");
}

extern "C" int pkm_grad_shard_sgd(const void* recv, int dtype, int64_t num_rows, int64_t dim, int world, int rank,
                                  int64_t shard_rows, void* const* table_bases, float lr, float weight_decay,
                                  float scale, int max_blocks, void* stream) {
  if (dtype != PKM_DT_F32 && dtype != PKM_DT_BF16) return fail(PKM_ERR_UNSUPPORTED, "dtype must be f32 or bf16");
  GradDest dest{};
  int rc = shard_dest(dest, table_bases, world, rank, shard_rows, num_rows, dim, dtype);
  if (rc) return rc;
  if (!recv || !aligned16(recv)) return fail(PKM_ERR_INVALID_ARG, "recv NULL or not 16-byte aligned");
  const int64_t rows = std::min<int64_t>(shard_rows, num_rows - (int64_t)rank * shard_rows);
  if (rows <= 0) return PKM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t row_vecs = dim * dtype_size(dtype) / 16;
  const int64_t n_vecs = rows * row_vecs;
  const int64_t per_block = 256 * kShardVec;
  int64_t blocks = (n_vecs + per_block - 1) / per_block;
  if (max_blocks > 0) blocks = std::min<int64_t>(blocks, max_blocks);
  shard_sgd_kernel<<<(unsigned)blocks, 256, 0, st>>>(static_cast<const uint4*>(recv), shard_rows * row_vecs, n_vecs,
                                                     world, rank, dtype == PKM_DT_BF16, scale, lr, weight_decay,
                                                     dest);
  return check_cuda("pkm_grad_shard_sgd");
}

// ---------------------------------------------------------------------------
// allocation-free variant of the backward
// ---------------------------------------------------------------------------
// Some callers cannot allocate device memory at all: an FFI binding that has
// no device allocator of its own, or a latency-critical serving loop where a
// cudaMalloc (which may synchronise the device) is not allowed.  For them the
// backward's scratch lives in this file-scope device array, which every GPU
// that loads the library holds until the process exits.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
// Device address of the scratch array on the current device (the host-side
// symbol is only a stand-in, never a device address).  It is looked up on
// every call, with the caller's device current: after the first call on a
// device (which loads the library's device code there) the lookup is cheap,
// and an address cached across calls would go stale if the caller reset the
// device or its primary context in between.
int noalloc_scratch(void** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess)
    return check_cuda("cudaGetSymbolAddress(g_noalloc_scratch)");
  *out = p;
  return PKM_OK;
}
}  // namespace

extern "C" int pkm_bag_bwd_noalloc(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                                   int weight_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size,
                                   int64_t num_rows, int64_t dim, void* grad_weight, int grad_weight_dtype,
                                   void* grad_psw, int grad_psw_dtype, int32_t* row_counts, uint32_t* dev_err,
                                   void* stream) {
  size_t need = 0;
  int rc = pkm_bag_bwd_workspace(n_bags, bag_size, num_rows, dim, &need);
  if (rc) return rc;
  if (need > kNoAllocScratchBytes)
    return fail(PKM_ERR_UNSUPPORTED, "pkm_bag_bwd_noalloc: this size needs " + std::to_string(need) +
                                         " bytes of scratch; the static scratch holds " +
                                         std::to_string(kNoAllocScratchBytes) + " (use pkm_bag_bwd with a workspace)");
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return pkm_bag_bwd(indices, psw, psw_dtype, weight, weight_dtype, grad_out, n_bags, bag_size, num_rows, dim,
                     grad_weight, grad_weight_dtype, grad_psw, grad_psw_dtype, row_counts, scratch,
                     kNoAllocScratchBytes, dev_err, stream);
}

extern "C" int pkm_grad_multimem_allreduce(const void* mc_src, void* mc_dst, int dtype, int64_t num_rows, int64_t dim,
                                           int world, int rank, int64_t shard_rows, int64_t row_begin,
                                           int64_t row_end, float scale, int max_blocks, void* stream) {
  if (dtype != PKM_DT_F32 && dtype != PKM_DT_BF16) return fail(PKM_ERR_UNSUPPORTED, "dtype must be f32 or bf16");
  if (world < 1 || rank < 0 || rank >= world) return fail(PKM_ERR_INVALID_ARG, "bad world / rank");
  if (shard_rows <= 0 || shard_rows * world < num_rows || dim <= 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  if ((dim * dtype_size(dtype)) % 16 != 0) return fail(PKM_ERR_UNSUPPORTED, "row bytes must be a multiple of 16");
  if (!mc_src || !mc_dst || !aligned16(mc_src) || !aligned16(mc_dst))
    return fail(PKM_ERR_INVALID_ARG, "multicast addresses NULL or not 16-byte aligned");
  if (row_end < 0) row_end = num_rows;
  const int64_t r0 = std::max<int64_t>((int64_t)rank * shard_rows, row_begin);
  const int64_t r1 = std::min<int64_t>(std::min<int64_t>((int64_t)(rank + 1) * shard_rows, num_rows), row_end);
  const int64_t rows = r1 - r0;
  if (rows <= 0) return PKM_OK;
  const int64_t row_vecs = dim * dtype_size(dtype) / 16;
  const int64_t n_vecs = rows * row_vecs;
  int64_t blocks = (n_vecs + 256 * kMmVec - 1) / (256 * kMmVec);
  if (max_blocks > 0) blocks = std::min<int64_t>(blocks, max_blocks);
  multimem_allreduce_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char*>(mc_src), static_cast<char*>(mc_dst), r0 * row_vecs, n_vecs, dtype == PKM_DT_BF16,
      scale);
  return check_cuda("pkm_grad_multimem_allreduce");
}

// ---------------------------------------------------------------------------
// ragged entry lists (row-sharded tables)
// ---------------------------------------------------------------------------
__global__ void seg_items_kernel(const int64_t* __restrict__ offs, int64_t n_segs, int4* __restrict__ desc,
                                 int32_t* n_items, uint32_t* err) {
  for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < n_segs; s += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = offs[s], e = offs[s + 1];
    if (b < 0 || e < b) {  // malformed offsets: an empty segment, reported
      raise_err(err, PKM_DEVERR_INDEX);
      b = e = 0;
    }
    desc[s] = make_int4((int)s, (int)b, (int)e, -1);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *n_items = (int32_t)n_segs;
}

extern "C" int pkm_segment_sum_workspace(int64_t n_segs, size_t* bytes) {
  if (!bytes || n_segs < 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  *bytes = (size_t)n_segs * sizeof(int4) + 256;
  return PKM_OK;
}

extern "C" int pkm_segment_sum(const void* rows, int row_dtype, int64_t num_rows, int64_t dim, const int32_t* entry_row,
                               const float* entry_w, int64_t n_entries, const int64_t* seg_offsets, int64_t n_segs,
                               void* out, int out_dtype, void* workspace, size_t workspace_bytes, uint32_t* dev_err,
                               void* stream) {
  if (!valid_dtype(row_dtype) || !valid_dtype(out_dtype)) return fail(PKM_ERR_INVALID_ARG, "bad dtype");
  if (num_rows < 0 || dim <= 0 || n_entries < 0 || n_segs < 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  if (n_entries >= (int64_t(1) << 31) || num_rows >= (int64_t(1) << 31) || n_segs >= (int64_t(1) << 31))
    return fail(PKM_ERR_UNSUPPORTED, "sizes must stay below 2^31");
  const int64_t rb = dim * dtype_size(row_dtype);
  if (rb % 16 != 0 || rb > 4096) return fail(PKM_ERR_UNSUPPORTED, "row bytes must be a multiple of 16, at most 4096");
  if (n_segs == 0) return PKM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!out || !seg_offsets) return fail(PKM_ERR_INVALID_ARG, "NULL pointer");
  if (n_entries == 0 || num_rows == 0) {
    cudaMemsetAsync(out, 0, (size_t)(n_segs * dim * dtype_size(out_dtype)), st);
    return check_cuda("pkm_segment_sum memset");
  }
  if (!rows || !aligned16(rows) || !entry_row || !entry_w) return fail(PKM_ERR_INVALID_ARG, "NULL or unaligned input");
  size_t need = 0;
  pkm_segment_sum_workspace(n_segs, &need);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(PKM_ERR_WORKSPACE, "workspace too small or not 256-byte aligned");
  int4* desc = static_cast<int4*>(workspace);
  int32_t* n_items = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + (size_t)n_segs * sizeof(int4));
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((n_segs + 255) / 256, (int64_t)num_sms() * 8));
  seg_items_kernel<<<(unsigned)blocks, 256, 0, st>>>(seg_offsets, n_segs, desc, n_items, dev_err);
  GatherArgs a{};
  a.rows = static_cast<const char*>(rows);
  a.row_bytes = rb;
  a.dim = dim;
  a.num_rows = num_rows;  // entry rows are checked against the table
  a.occ = entry_row;
  a.occ_w = entry_w;
  a.L = 1;
  a.n_items_dev = n_items;
  a.item_desc = desc;
  a.out = out;
  a.out_dtype = out_dtype;
  a.err = dev_err;
  return gather_launch(row_dtype, true, false, a, n_segs, st);
}

extern "C" int pkm_bag_bwd_ragged(const int64_t* row_idx, const int32_t* src_of, const void* psw, int psw_dtype,
                                  const void* weight, int weight_dtype, const void* grad_rows, int64_t n_entries,
                                  int64_t n_src, int64_t num_rows, int64_t dim, void* grad_weight,
                                  int grad_weight_dtype, void* grad_psw, int grad_psw_dtype, int32_t* row_counts,
                                  void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  if (n_entries > 0 && !src_of) return fail(PKM_ERR_INVALID_ARG, "src_of is NULL");
  if (n_src < 0) return fail(PKM_ERR_INVALID_ARG, "bad size");
  GradDest dest{};
  dest.out = grad_weight;
  return bag_bwd_impl(row_idx, psw, psw_dtype, weight, weight_dtype, grad_rows, n_entries, 1, num_rows, dim, dest,
                      grad_weight_dtype, grad_psw, grad_psw_dtype, row_counts, workspace, workspace_bytes, dev_err,
                      stream, src_of, n_src);
}

extern "C" int pkm_bag_bwd_sort(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                                int weight_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size,
                                int64_t num_rows, int64_t dim, void* grad_psw, int grad_psw_dtype,
                                int32_t* row_counts, void* workspace, size_t workspace_bytes, uint32_t* dev_err,
                                void* stream) {
  GradDest dest{};
  dest.out = reinterpret_cast<void*>(uintptr_t(1));  // not written by this phase
  return bag_bwd_impl(indices, psw, psw_dtype, weight, weight_dtype, grad_out, n_bags, bag_size, num_rows, dim, dest,
                      weight_dtype, grad_psw, grad_psw_dtype, row_counts, workspace, workspace_bytes, dev_err, stream,
                      nullptr, 0, kBwdSort);
}

extern "C" int pkm_bag_bwd_rows(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                                int weight_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size,
                                int64_t num_rows, int64_t dim, int64_t row_begin, int64_t row_end, void* grad_weight,
                                int grad_weight_dtype, void* grad_psw, int grad_psw_dtype, void* workspace,
                                size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  GradDest dest{};
  dest.out = grad_weight;
  return bag_bwd_impl(indices, psw, psw_dtype, weight, weight_dtype, grad_out, n_bags, bag_size, num_rows, dim, dest,
                      grad_weight_dtype, grad_psw, grad_psw_dtype, nullptr, workspace, workspace_bytes, dev_err,
                      stream, nullptr, 0, kBwdRows, row_begin, row_end);
}
