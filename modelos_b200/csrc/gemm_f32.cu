// fp32 GEMM on the CUDA cores for the fast-weight memory's scoring backward
// (fwpkm/fwpkm.py:853-869: the einsum and cdist of compute_qk_scores, whose
// gradients are dense GEMMs per (head, half) group in fp32; the fast weights
// are fp32 by default, fwpkm/fwpkm.py:47, so the tensor cores' bf16 path
// does not apply).
//
//   C[b][m, n] = sum_k A[b][m, k] * B[b][n, k]
//
// with A and B row-major fp32 matrices read K-major or MN-major and batch b
// shifting the operands by (column, row) offsets, the same views as the
// tensor-core GEMM.  128 x 128 output tiles, 256 threads, 8 x 8 outputs per
// thread in two 4-wide groups 64 apart (conflict-free 16-byte shared loads),
// K in slices of 8 through a double-buffered shared tile: the next slice is
// fetched into registers (16-byte loads where its four elements are inside
// and aligned) while the current one is multiplied, then stored; fp32 FMAs,
// ascending k within a thread.  Grids the tiles alone cannot fill split K
// (with a workspace): fp32 partials per split, summed in split order by a
// second kernel (deterministic).
#include <algorithm>

#include "common.cuh"

namespace pkm {

constexpr int F_BM = 128, F_BN = 128, F_BK = 8, F_THREADS = 256;

struct GemmF32Args {
  const float* A;
  const float* B;
  float* C;
  int64_t lda, ldb, ldc;
  int a_mn, b_mn;
  int vec_a, vec_b;  // 16-byte loads allowed (aligned base, pitch and batch offsets)
  int M, N, K;
  int64_t a_rows, a_cols, b_rows, b_cols;
  int64_t a_bx, a_by, b_bx, b_by, c_bs;
  int m_tiles, n_tiles, batch, splits;
  float* ws;  // split partials [splits][batch][M][N]
};

// Element (i along M or N, k) of an operand view, 0 outside the matrix.
__device__ __forceinline__ float f_at(const float* P, int64_t ld, int mn_major, int64_t rows, int64_t cols,
                                      int64_t bx, int64_t by, int64_t i, int64_t k) {
  const int64_t r = (mn_major ? k : i) + by, c = (mn_major ? i : k) + bx;
  return (r < rows && c < cols) ? __ldg(P + r * ld + c) : 0.f;
}

// This thread's 4 elements of one operand's 8 x 128 slice, into registers:
// MN-major: (k = t / 32, i = (t % 32) * 4 .. +3); K-major: (i = t / 2,
// k = (t % 2) * 4 .. +3); both runs are contiguous in memory.
__device__ __forceinline__ void f_fetch(const float* P, int64_t ld, int mn_major, int vec, int64_t rows, int64_t cols,
                                        int64_t bx, int64_t by, int64_t i0, int64_t k0, int lim_i, int lim_k,
                                        float (&r)[4]) {
  const int t = threadIdx.x;
  if (mn_major) {
    const int64_t k = k0 + (t >> 5), i = i0 + (t & 31) * 4;
    if (vec && k < lim_k && i + 3 < lim_i) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(P + (k + by) * ld + i + bx));
      r[0] = v.x;
      r[1] = v.y;
      r[2] = v.z;
      r[3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = (k < lim_k && i + j < lim_i) ? f_at(P, ld, 1, rows, cols, bx, by, i + j, k) : 0.f;
    }
  } else {
    const int64_t i = i0 + (t >> 1), k = k0 + (t & 1) * 4;
    if (vec && i < lim_i && k + 3 < lim_k) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(P + (i + by) * ld + k + bx));
      r[0] = v.x;
      r[1] = v.y;
      r[2] = v.z;
      r[3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = (i < lim_i && k + j < lim_k) ? f_at(P, ld, 0, rows, cols, bx, by, i, k + j) : 0.f;
    }
  }
}

__device__ __forceinline__ void f_store(int mn_major, const float (&r)[4], float (*S)[F_BM + 4]) {
  const int t = threadIdx.x;
  if (mn_major) {
    *reinterpret_cast<float4*>(&S[t >> 5][(t & 31) * 4]) = make_float4(r[0], r[1], r[2], r[3]);
  } else {
    const int i = t >> 1, k = (t & 1) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) S[k + j][i] = r[j];
  }
}

__global__ void __launch_bounds__(F_THREADS) gemm_f32_kernel(const GemmF32Args a) {
  __shared__ __align__(16) float As[2][F_BK][F_BM + 4];
  __shared__ __align__(16) float Bs[2][F_BK][F_BN + 4];
  const int s = (int)(blockIdx.x % a.splits);
  const int64_t tile = blockIdx.x / a.splits;
  const int nt = (int)(tile % a.n_tiles);
  const int mt = (int)((tile / a.n_tiles) % a.m_tiles);
  const int b = (int)(tile / ((int64_t)a.n_tiles * a.m_tiles));
  const int64_t m0 = (int64_t)mt * F_BM, n0 = (int64_t)nt * F_BN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t abx = b * a.a_bx, aby = b * a.a_by, bbx = b * a.b_bx, bby = b * a.b_by;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int nk = (a.K + F_BK - 1) / F_BK;
  const int kt0 = (int)((int64_t)nk * s / a.splits), kt1 = (int)((int64_t)nk * (s + 1) / a.splits);
  float ra[4], rb[4];
  if (kt0 < kt1) {
    f_fetch(a.A, a.lda, a.a_mn, a.vec_a, a.a_rows, a.a_cols, abx, aby, m0, (int64_t)kt0 * F_BK, a.M, a.K, ra);
    f_fetch(a.B, a.ldb, a.b_mn, a.vec_b, a.b_rows, a.b_cols, bbx, bby, n0, (int64_t)kt0 * F_BK, a.N, a.K, rb);
    f_store(a.a_mn, ra, As[0]);
    f_store(a.b_mn, rb, Bs[0]);
  }
  __syncthreads();
  for (int kt = kt0; kt < kt1; ++kt) {
    const int cur = (kt - kt0) & 1;
    const bool more = kt + 1 < kt1;
    if (more) {
      // in flight while this slice is multiplied
      f_fetch(a.A, a.lda, a.a_mn, a.vec_a, a.a_rows, a.a_cols, abx, aby, m0, (int64_t)(kt + 1) * F_BK, a.M, a.K,
              ra);
      f_fetch(a.B, a.ldb, a.b_mn, a.vec_b, a.b_rows, a.b_cols, bbx, bby, n0, (int64_t)(kt + 1) * F_BK, a.N, a.K,
              rb);
    }
#pragma unroll
    for (int k = 0; k < F_BK; ++k) {
      float av[8], bv[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][k][64 + tx * 4]);
      av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
      av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
      bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
      bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) {
      // the other buffer was last read before the previous barrier
      f_store(a.a_mn, ra, As[cur ^ 1]);
      f_store(a.b_mn, rb, Bs[cur ^ 1]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= a.M) continue;
    float* crow = a.splits > 1 ? a.ws + (((int64_t)s * a.batch + b) * a.M + m) * a.N
                               : a.C + b * a.c_bs + m * a.ldc;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (n < a.N) crow[n] = acc[i][j];
    }
  }
}

// C[b][m][n] = sum over s of the split partials, in split order.
__global__ void gemm_f32_reduce_kernel(const GemmF32Args a) {
  const int64_t per = (int64_t)a.batch * a.M * a.N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per; i += (int64_t)gridDim.x * blockDim.x) {
    float acc = a.ws[i];
    for (int s = 1; s < a.splits; ++s) acc += a.ws[s * per + i];
    const int64_t n = i % a.N, r = i / a.N;
    const int64_t m = r % a.M, b = r / a.M;
    a.C[b * a.c_bs + m * a.ldc + n] = acc;
  }
}

// Splits of K: while the tiles would leave SMs idle (two blocks each) and
// every split keeps at least 32 slices of 8.
static int gemm_f32_splits(int64_t tiles, int64_t K) {
  const int64_t nk = (K + F_BK - 1) / F_BK, target = 2 * (int64_t)num_sms();
  int s = 1;
  while (tiles * s * 2 <= target && nk / (s * 2) >= 32 && s < 16) s *= 2;
  return s;
}

}  // namespace pkm

using namespace pkm;

extern "C" int pkm_gemm_f32_workspace(int64_t batch, int64_t M, int64_t N, int64_t K, size_t* bytes) {
  if (!bytes) return fail(PKM_ERR_INVALID_ARG, "null bytes");
  if (batch < 0 || M < 0 || N < 0 || K < 0) return fail(PKM_ERR_INVALID_ARG, "negative size");
  const int64_t tiles = batch * ((M + F_BM - 1) / F_BM) * ((N + F_BN - 1) / F_BN);
  const int s = gemm_f32_splits(tiles, K);
  *bytes = s > 1 ? (size_t)s * batch * M * N * sizeof(float) : 0;
  return PKM_OK;
}

extern "C" int pkm_gemm_f32_ws(const float* A, int a_mn_major, int64_t a_rows, int64_t a_cols, int64_t lda,
                               const float* B, int b_mn_major, int64_t b_rows, int64_t b_cols, int64_t ldb,
                               int64_t batch, int64_t M, int64_t N, int64_t K, int64_t a_batch_x,
                               int64_t a_batch_y, int64_t b_batch_x, int64_t b_batch_y, float* C, int64_t ldc,
                               int64_t c_batch_stride, void* workspace, size_t workspace_bytes, void* stream) {
  if (batch < 0 || M < 0 || N < 0 || K < 0) return fail(PKM_ERR_INVALID_ARG, "negative size");
  if (batch == 0 || M == 0 || N == 0) return PKM_OK;
  if (!A || !B || !C) return fail(PKM_ERR_INVALID_ARG, "null operand");
  if (ldc < N || a_cols > lda || b_cols > ldb || a_rows < 0 || b_rows < 0)
    return fail(PKM_ERR_INVALID_ARG, "bad row pitch");
  if (a_batch_x < 0 || a_batch_y < 0 || b_batch_x < 0 || b_batch_y < 0 || c_batch_stride < 0)
    return fail(PKM_ERR_INVALID_ARG, "negative batch offset");
  const int64_t a_need_x = (a_mn_major ? M : K) + (batch - 1) * a_batch_x;
  const int64_t a_need_y = (a_mn_major ? K : M) + (batch - 1) * a_batch_y;
  const int64_t b_need_x = (b_mn_major ? N : K) + (batch - 1) * b_batch_x;
  const int64_t b_need_y = (b_mn_major ? K : N) + (batch - 1) * b_batch_y;
  if (a_need_x > a_cols || a_need_y > a_rows || b_need_x > b_cols || b_need_y > b_rows)
    return fail(PKM_ERR_INVALID_ARG, "operand extents smaller than the GEMM");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail(PKM_ERR_UNSUPPORTED, "dimension above 2^31");
  GemmF32Args a{};
  a.A = A;
  a.B = B;
  a.C = C;
  a.lda = lda;
  a.ldb = ldb;
  a.ldc = ldc;
  a.a_mn = a_mn_major ? 1 : 0;
  a.b_mn = b_mn_major ? 1 : 0;
  a.vec_a = aligned16(A) && lda % 4 == 0 && a_batch_x % 4 == 0;
  a.vec_b = aligned16(B) && ldb % 4 == 0 && b_batch_x % 4 == 0;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.a_rows = a_rows;
  a.a_cols = a_cols;
  a.b_rows = b_rows;
  a.b_cols = b_cols;
  a.a_bx = a_batch_x;
  a.a_by = a_batch_y;
  a.b_bx = b_batch_x;
  a.b_by = b_batch_y;
  a.c_bs = c_batch_stride;
  a.m_tiles = (int)((M + F_BM - 1) / F_BM);
  a.n_tiles = (int)((N + F_BN - 1) / F_BN);
  a.batch = (int)batch;
  const int64_t tiles = batch * a.m_tiles * a.n_tiles;
  int splits = gemm_f32_splits(tiles, K);
  const size_t need = splits > 1 ? (size_t)splits * batch * M * N * sizeof(float) : 0;
  if (splits > 1 && (!workspace || workspace_bytes < need || !aligned16(workspace))) splits = 1;
  a.splits = splits;
  a.ws = static_cast<float*>(workspace);
  if (tiles * splits > INT32_MAX) return fail(PKM_ERR_UNSUPPORTED, "too many tiles");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  gemm_f32_kernel<<<(unsigned)(tiles * splits), F_THREADS, 0, st>>>(a);
  int rc = check_cuda("gemm_f32_kernel");
  if (rc || splits == 1) return rc;
  const int64_t per = batch * M * N;
  const int64_t rgrid = std::max<int64_t>(1, std::min<int64_t>((per + 255) / 256, (int64_t)num_sms() * 8));
  gemm_f32_reduce_kernel<<<(unsigned)rgrid, 256, 0, st>>>(a);
  return check_cuda("gemm_f32_reduce_kernel");
}

extern "C" int pkm_gemm_f32(const float* A, int a_mn_major, int64_t a_rows, int64_t a_cols, int64_t lda,
                            const float* B, int b_mn_major, int64_t b_rows, int64_t b_cols, int64_t ldb,
                            int64_t batch, int64_t M, int64_t N, int64_t K, int64_t a_batch_x, int64_t a_batch_y,
                            int64_t b_batch_x, int64_t b_batch_y, float* C, int64_t ldc, int64_t c_batch_stride,
                            void* stream) {
  return pkm_gemm_f32_ws(A, a_mn_major, a_rows, a_cols, lda, B, b_mn_major, b_rows, b_cols, ldb, batch, M, N, K,
                         a_batch_x, a_batch_y, b_batch_x, b_batch_y, C, ldc, c_batch_stride, nullptr, 0, stream);
}
