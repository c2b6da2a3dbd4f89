// CUDA-core fp32 gather-GEMM: 128x128 tile per CTA, 8x8 outputs per thread,
// BK = 8 with register prefetch and double-buffered shared memory.  Used for
// shapes the tensor-core kernel does not take, and as the cross-check of it.
// Optional split-K writes per-split partial tiles to a workspace that
// k_splitk_reduce sums in split order (deterministic).
#pragma once

#include "tp_core.h"
#include "tp_gemm.cuh"

namespace tp {

constexpr int SG_BM = 128, SG_BN = 128, SG_BK = 8, SG_PAD = 4;

template <class LD, int ROWS>
__device__ __forceinline__ void sg_fetch(const LD& ld, int b, int64_t r0, int64_t rows, int64_t k0, int64_t kend,
                                         float (&reg)[4]) {
  int tid = threadIdx.x;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int rr, kk;
    if (LD::kContigK) {
      kk = tid % SG_BK;
      rr = tid / SG_BK + 32 * j;
    } else {
      rr = tid % ROWS;
      kk = tid / ROWS + 2 * j;
    }
    int64_t r = r0 + rr, k = k0 + kk;
    reg[j] = (r < rows && k < kend) ? ld(b, r, k) : 0.0f;
  }
}

template <class LD, int ROWS>
__device__ __forceinline__ void sg_stash(float (*S)[ROWS + SG_PAD], const float (&reg)[4]) {
  int tid = threadIdx.x;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int rr, kk;
    if (LD::kContigK) {
      kk = tid % SG_BK;
      rr = tid / SG_BK + 32 * j;
    } else {
      rr = tid % ROWS;
      kk = tid / ROWS + 2 * j;
    }
    S[kk][rr] = reg[j];
  }
}

template <class LA, class LB, class EP>
__global__ void __launch_bounds__(256) k_gemm_simt(LA la, LB lb, EP ep, int64_t M, int64_t N, int64_t K,
                                                   int64_t k_per_split, int splitk, float* __restrict__ ws) {
  ::tp::pdl_enter();
  __shared__ __align__(16) float As[2][SG_BK][SG_BM + SG_PAD];
  __shared__ __align__(16) float Bs[2][SG_BK][SG_BN + SG_PAD];
  int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  int64_t m0 = (int64_t)blockIdx.x * SG_BM, n0 = (int64_t)blockIdx.y * SG_BN;
  int z = blockIdx.z;
  int b = splitk ? 0 : z;
  int64_t kb = splitk ? (int64_t)z * k_per_split : 0;
  int64_t ke = splitk ? (kb + k_per_split < K ? kb + k_per_split : K) : K;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  float ra[4], rb[4];
  sg_fetch<LA, SG_BM>(la, b, m0, M, kb, ke, ra);
  sg_fetch<LB, SG_BN>(lb, b, n0, N, kb, ke, rb);
  sg_stash<LA, SG_BM>(As[0], ra);
  sg_stash<LB, SG_BN>(Bs[0], rb);
  __syncthreads();
  int buf = 0;
  for (int64_t k0 = kb; k0 < ke; k0 += SG_BK) {
    bool more = k0 + SG_BK < ke;
    if (more) {
      sg_fetch<LA, SG_BM>(la, b, m0, M, k0 + SG_BK, ke, ra);
      sg_fetch<LB, SG_BN>(lb, b, n0, N, k0 + SG_BK, ke, rb);
    }
#pragma unroll
    for (int kk = 0; kk < SG_BK; ++kk) {
      float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) {
      sg_stash<LA, SG_BM>(As[buf ^ 1], ra);
      sg_stash<LB, SG_BN>(Bs[buf ^ 1], rb);
      __syncthreads();
      buf ^= 1;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int64_t n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (n >= N) continue;
      if (splitk) ws[((int64_t)z * M + m) * N + n] = acc[i][j];
      else ep(b, m, n, acc[i][j]);
    }
  }
}

template <class EP>
__global__ void k_splitk_reduce(const float* __restrict__ ws, int splits, int64_t M, int64_t N, int b, EP ep) {
  ::tp::pdl_enter();
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < M * N; i += stride) {
    // eight splits' loads in flight at a time, added in split order
    float s = 0.0f;
    int z = 0;
    for (; z + 8 <= splits; z += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = ws[(int64_t)(z + u) * M * N + i];
#pragma unroll
      for (int u = 0; u < 8; ++u) s += v[u];
    }
    for (; z < splits; ++z) s += ws[(int64_t)z * M * N + i];
    ep(b, i / N, i % N, s);
  }
}

// C(b, m, n) = sum_k A(b, m, k) B(b, n, k) for b < batch.  split-K only when
// batch == 1 and the tile grid cannot fill the GPU.
template <class LA, class LB, class EP>
void gemm_simt(const LA& la, const LB& lb, const EP& ep, int64_t M, int64_t N, int64_t K, int batch) {
  if (M == 0 || N == 0 || batch == 0) return;
  int64_t gm = (M + SG_BM - 1) / SG_BM, gn = (N + SG_BN - 1) / SG_BN;
  TP_REQUIRE(gn <= 65535, "gemm: N tiles exceed the grid limit");
  int splits = 1;
  int64_t tiles = gm * gn * batch;
  if (batch == 1 && K > 0) {
    int64_t want = (2 * (int64_t)sm_count() + tiles - 1) / tiles;
    int64_t maxs = K / 256;
    splits = (int)(want < maxs ? want : maxs);
    if (splits > 64) splits = 64;
    if (splits < 1) splits = 1;
  }
  int64_t kps = (K + splits - 1) / splits;
  kps = (kps + SG_BK - 1) / SG_BK * SG_BK;
  if (splits > 1) splits = (int)((K + kps - 1) / kps);
  if (splits > 1) {
    float* ws = (float*)scratch((size_t)splits * M * N * sizeof(float));
    auto kfn = k_gemm_simt<LA, LB, EP>;
    TP_LAUNCH(kfn, dim3((unsigned)gm, (unsigned)gn, (unsigned)splits), 256, 0, la, lb, ep, M, N, K, kps, 1, ws);
    auto rfn = k_splitk_reduce<EP>;
    TP_LAUNCH(rfn, grid_for(M * N, 256), 256, 0, ws, splits, M, N, 0, ep);
  } else {
    if (K == 0) {  // no terms: every output is the epilogue of 0
      auto rfn = k_splitk_reduce<EP>;
      for (int bb = 0; bb < batch; ++bb) TP_LAUNCH(rfn, grid_for(M * N, 256), 256, 0, (const float*)nullptr, 0, M, N, bb, ep);
      return;
    }
    auto kfn = k_gemm_simt<LA, LB, EP>;
    TP_LAUNCH(kfn, dim3((unsigned)gm, (unsigned)gn, (unsigned)batch), 256, 0, la, lb, ep, M, N, K, K, 0,
              (float*)nullptr);
  }
}

// ---- skinny products: one side of at most 16 rows ---------------------------------------------
// C(m, n) = sum_k A(m, k) B(n, k) with M <= 16 (SMALL_IS_M) or N <= 16.  A
// 128-thread CTA takes 128 rows l of the large side and a k range; per chunk
// of 32 k the small side's values are staged in shared memory (read back as
// broadcasts) and each thread first loads its 32 large-side values, then does
// the S x 32 multiply-adds with its S sums in registers, so 32 loads are in
// flight per thread instead of one at a time.  A 128 x 128 tensor-core or
// CUDA-core tile would be more than 87% padding here (the 512 -> 10
// classifier of a CNN, its weight gradient).  Partial sums of a k split go to
// ws[split][M][N], which k_splitk_reduce adds in split order.
constexpr int SK_S = 16, SK_KC = 32, SK_THREADS = 128;

template <class LS, class LL, class EP, bool SMALL_IS_M>
__global__ void __launch_bounds__(SK_THREADS) k_gemm_skinny(LS ls, LL ll, EP ep, int64_t M, int64_t N, int64_t K,
                                                            int64_t k_per_split, int splitk, float* __restrict__ ws) {
  ::tp::pdl_enter();
  __shared__ float sm[SK_KC][SK_S];
  const int64_t S = SMALL_IS_M ? M : N, L = SMALL_IS_M ? N : M;
  const int64_t l = (int64_t)blockIdx.x * SK_THREADS + threadIdx.x;
  const int z = blockIdx.y;
  const int64_t kb = (int64_t)z * k_per_split;
  const int64_t ke = kb + k_per_split < K ? kb + k_per_split : K;
  float acc[SK_S];
#pragma unroll
  for (int j = 0; j < SK_S; ++j) acc[j] = 0.0f;
  for (int64_t k0 = kb; k0 < ke; k0 += SK_KC) {
    __syncthreads();
    for (int i = threadIdx.x; i < SK_KC * SK_S; i += SK_THREADS) {
      const int kk = i / SK_S, j = i % SK_S;
      sm[kk][j] = (j < S && k0 + kk < ke) ? ls(0, j, k0 + kk) : 0.0f;
    }
    float v[SK_KC];
#pragma unroll
    for (int kk = 0; kk < SK_KC; ++kk) v[kk] = (l < L && k0 + kk < ke) ? ll(0, l, k0 + kk) : 0.0f;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SK_KC; ++kk)
#pragma unroll
      for (int j = 0; j < SK_S; ++j) acc[j] = fmaf(sm[kk][j], v[kk], acc[j]);
  }
  if (l >= L) return;
#pragma unroll
  for (int j = 0; j < SK_S; ++j) {
    if (j >= S) break;
    const int64_t m = SMALL_IS_M ? j : l, n = SMALL_IS_M ? l : j;
    if (splitk) ws[((int64_t)z * M + m) * N + n] = acc[j];
    else ep(0, m, n, acc[j]);
  }
}

inline bool gemm_skinny_ok(int64_t M, int64_t N, int batch) { return batch == 1 && (M <= SK_S || N <= SK_S); }

template <class LA, class LB, class EP>
void gemm_skinny(const LA& la, const LB& lb, const EP& ep, int64_t M, int64_t N, int64_t K) {
  if (M == 0 || N == 0) return;
  const bool small_m = M <= SK_S;
  const int64_t L = small_m ? N : M;
  const int64_t lblocks = (L + SK_THREADS - 1) / SK_THREADS;
  int splits = 1;
  if (K > 0) {
    // about 4 CTAs per SM, at least one 32-wide chunk of k each
    int64_t want = (4 * (int64_t)sm_count() + lblocks - 1) / lblocks;
    int64_t maxs = (K + SK_KC - 1) / SK_KC;
    splits = (int)(want < maxs ? want : maxs);
    if (splits > 256) splits = 256;
    if (splits < 1) splits = 1;
  }
  int64_t kps = (K + splits - 1) / splits;
  kps = (kps + SK_KC - 1) / SK_KC * SK_KC;
  if (K > 0) splits = (int)((K + kps - 1) / kps);
  TP_REQUIRE(lblocks <= 0x7fffffff, "gemm: too many rows");
  float* ws = splits > 1 ? (float*)scratch((size_t)splits * M * N * sizeof(float)) : nullptr;
  const dim3 grid((unsigned)lblocks, (unsigned)splits);
  if (small_m)
    TP_LAUNCH((k_gemm_skinny<LA, LB, EP, true>), grid, SK_THREADS, 0, la, lb, ep, M, N, K, kps, splits > 1, ws);
  else
    TP_LAUNCH((k_gemm_skinny<LB, LA, EP, false>), grid, SK_THREADS, 0, lb, la, ep, M, N, K, kps, splits > 1, ws);
  if (splits > 1) {
    auto rfn = k_splitk_reduce<EP>;
    TP_LAUNCH(rfn, grid_for(M * N, 256), 256, 0, ws, splits, M, N, 0, ep);
  }
}

}  // namespace tp
