// GEMM kernel selection shared by the contraction translation units.
//
//   gemm_path() == 0   TMA-fed tensor-core kernel where both operands can be
//                      described by tensor maps, else the gather tensor-core
//                      kernel (M >= 64, K > 0), else the CUDA-core kernel
//   gemm_path() == 1   CUDA-core kernel only
//   gemm_path() == 2   gather tensor-core kernel where it applies, no TMA
//   gemm_path() == 3   as 0, but the TMA kernel on single CTAs only (no CTA pairs)
//   gemm_path() == 4   as 0, with CTA pairs wherever they fit (N > 32, two row
//                      tiles; cross-check of the pair kernel on small shapes)
#pragma once

#include "tp_gemm.cuh"
#include "tp_gemm_simt.cuh"
#include "tp_gemm_tc.cuh"
#include "tp_gemm_tma.cuh"
#include "tp_gemm_tma2.cuh"
#include "tp_tma.h"

namespace tp {

int gemm_path();
// 128-wide single-CTA tiles: 0 = 4 stages, one CTA per SM; 1 = 2 stages, two
// CTAs per SM when there are more CTAs than SMs; 2 = two per SM always
// (tp_set_gemm_twocta)
int gemm_twocta();
// paths 0 and 3 use the TMA kernels
inline bool tma_enabled() { return gemm_path() == 0 || gemm_path() == 3 || gemm_path() == 4; }

// Gather tensor-core kernel with the N tile following N (K > 0).
template <class LA, class LB, class EP>
void gemm_tc(const LA& la, const LB& lb, const EP& ep, int64_t M, int64_t N, int64_t K, int batch) {
  if (M == 0 || N == 0 || batch == 0) return;
  if (N <= 32) gemm_tc_launch<LA, LB, EP, 32, 4>(la, lb, ep, M, N, K, batch);
  else if (N <= 64) gemm_tc_launch<LA, LB, EP, 64, 4>(la, lb, ep, M, N, K, batch);
  else gemm_tc_launch<LA, LB, EP, 128, 3>(la, lb, ep, M, N, K, batch);
}

// Products with a side of at most 16 rows: the skinny CUDA-core kernel.  Else
// the gather tensor-core path for M >= 64 and K > 16, else the CUDA-core kernel.
template <class LA, class LB, class EP>
void gemm_auto(const LA& la, const LB& lb, const EP& ep, int64_t M, int64_t N, int64_t K, int batch) {
  if (M == 0 || N == 0 || batch == 0) return;
  if (gemm_skinny_ok(M, N, batch)) gemm_skinny(la, lb, ep, M, N, K);
  else if (gemm_path() == 1 || K <= 16 || M < 64) gemm_simt(la, lb, ep, M, N, K, batch);
  else gemm_tc(la, lb, ep, M, N, K, batch);
}

inline uint32_t tma_bn(int64_t N) { return N <= 32 ? 32u : (N <= 64 ? 64u : 128u); }

// The CTA-pair kernel (tp_gemm_tma2.cuh): 256 x 256 tiles, each CTA holding
// 128 columns of B.  Its main loop does twice the work per k-block in ~1.55x
// the time of the single-CTA kernel's, but a tile is 4x larger and its
// epilogue 2x longer, so it is taken for N >= 256 with at least 8192 pair-tile
// k-blocks of work (measured on the VGG convolutions: 256 -> 512 channels at
// 4x4 1.7x faster, 512 -> 512 at 2x2 (4608 pair-tile k-blocks) 1.15x slower);
// not yet for the wide dense products (N > 1024), whose L2 reuse it lowers.
inline bool tma_pair(int64_t M, int64_t N, int64_t K, int batch) {
  if (gemm_path() == 4) return M > tc::BM && N > 32;
  if (gemm_path() != 0 || N < 256 || N > 1024 || M <= tc::BM) return false;
  const int64_t work = ((M + 255) / 256) * ((N + 255) / 256) * batch * ((K + tc::BK - 1) / tc::BK);
  return work >= 8192;
}

// Pair tile width: 256, or 64 / 128 for narrow N under path 4.
inline uint32_t tma_bnp(int64_t N) { return N <= 64 ? 64u : (N <= 128 ? 128u : 256u); }

// Rows of B's tensor-map box for the kernel gemm_tma_bn picks.
inline uint32_t tma_b_rows(int64_t M, int64_t N, int64_t K, int batch) {
  return tma_pair(M, N, K, batch) ? tma_bnp(N) / 2 : tma_bn(N);
}

// Single-CTA TMA kernel with 128-column tiles: when there are more CTAs (tiles x
// split-K splits, the split gemm_tma_launch computes) than SMs, two per SM on a
// 2-stage ring, each one's prologue and epilogue under the other's main loop; a
// single wave keeps the deeper 4-stage ring (measured on the VGG convolutions:
// 64 -> 128 channels at batch 1024, 2048 CTAs, 220 -> 178 us with two per SM;
// 512 -> 512 at 2x2, 128 CTAs, 97 -> 122 us).
template <class SA, class SB, class EP>
void gemm_tma_128(const CUtensorMap& ma, const CUtensorMap& mb, const SA& sa, const SB& sb, const EP& ep, int64_t M,
                  int64_t N, int64_t K, int batch, const CUtensorMap* mbl = nullptr) {
  const int two = gemm_twocta();
  const int64_t tiles = ((M + tc::BM - 1) / tc::BM) * ((N + 127) / 128) * batch;
  const int64_t ctas = tiles * gemm_splits(tiles, K, sm_count(), M * N * batch);
  if (two == 2 || (two == 1 && ctas > sm_count()))
    gemm_tma_launch<SA, SB, EP, 128, 2>(ma, mb, sa, sb, ep, M, N, K, batch, mbl);
  else
    gemm_tma_launch<SA, SB, EP, 128, 4>(ma, mb, sa, sb, ep, M, N, K, batch, mbl);
}

// TMA kernel with the N tile following N; the maps' B box must be tma_b_rows(M, N, K, batch).
template <class SA, class SB, class EP>
void gemm_tma_bn(const CUtensorMap& ma, const CUtensorMap& mb, const SA& sa, const SB& sb, const EP& ep, int64_t M,
                 int64_t N, int64_t K, int batch, const CUtensorMap* mbl = nullptr) {
  if (tma_pair(M, N, K, batch)) {
    if (N <= 64) gemm_tma2_launch<SA, SB, EP, 32, 4>(ma, mb, sa, sb, ep, M, N, K, batch, mbl);
    else if (N <= 128) gemm_tma2_launch<SA, SB, EP, 64, 4>(ma, mb, sa, sb, ep, M, N, K, batch, mbl);
    else gemm_tma2_launch<SA, SB, EP, 128, 4>(ma, mb, sa, sb, ep, M, N, K, batch, mbl);
    return;
  }
  // N <= 64: 3-stage tiles, two CTAs per SM (one's epilogue under the other's main loop)
  if (N <= 32) {
    gemm_tma_launch<SA, SB, EP, 32, 3>(ma, mb, sa, sb, ep, M, N, K, batch, mbl);
  } else if (N <= 64) {
    gemm_tma_launch<SA, SB, EP, 64, 3>(ma, mb, sa, sb, ep, M, N, K, batch, mbl);
  } else {
    gemm_tma_128(ma, mb, sa, sb, ep, M, N, K, batch, mbl);
  }
}

// A dense operand: element (r, k) of batch b at p[b*bs + r*ld + k] (K-major)
// or p[b*bs + k*ld + r] (mn: MN-major); batched = false shares it across the
// batch.
struct MatOp {
  const float* p;
  bool mn;
  int64_t ld, bs;
  bool batched;
};

// An MN-major operand is addressed in 32-row groups (an outer map dimension
// of stride 128 B), so its rows must be a multiple of 32.
inline bool mat_tma_ok(const MatOp& o, int64_t rows) {
  if (o.ld <= 0 || o.ld % 4 || (o.batched && o.bs % 4)) return false;
  if (o.mn && rows % 32) return false;
  uint64_t st[2] = {(uint64_t)o.ld * 4, (uint64_t)(o.batched ? o.bs : o.ld) * 4};
  return tma_aligned(o.p, st, 2);
}

// Map over the operand (rows x K per batch).  K-major: dims (K, rows, batch),
// box (32, box_rows, 1).  MN-major: dims (32, K, rows/32, batch), box
// (32, 32, box_rows/32, 1).
inline void mat_map(CUtensorMap* m, const MatOp& o, int64_t rows, int64_t K, int batch, uint32_t box_rows) {
  const uint64_t bst = (uint64_t)(o.batched ? o.bs : o.ld * (o.mn ? K : rows)) * 4;
  if (!o.mn) {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)rows, (uint64_t)(o.batched ? batch : 1)};
    uint64_t st[2] = {(uint64_t)o.ld * 4, bst};
    uint32_t box[3] = {32, box_rows, 1};
    make_map_f32(m, o.p, 3, dims, st, box, false);
  } else {
    uint64_t dims[4] = {32, (uint64_t)K, (uint64_t)(rows / 32), (uint64_t)(o.batched ? batch : 1)};
    uint64_t st[3] = {(uint64_t)o.ld * 4, 128, bst};
    uint32_t box[4] = {32, 32, box_rows / 32, 1};
    make_map_f32(m, o.p, 4, dims, st, box, true);
  }
}

template <class SA, class SB, class EP>
void gemm_tma_mat(const MatOp& a, const MatOp& b, const EP& ep, int64_t M, int64_t N, int64_t K, int batch) {
  CUtensorMap ma, mb, mbl;
  mat_map(&ma, a, M, K, batch, (uint32_t)tc::BM);
  mat_map(&mb, b, N, K, batch, tma_b_rows(M, N, K, batch));
  // a dense B shared by at least 16 row tiles: split its tf32 low parts once
  const bool pre = !b.batched && M * batch >= 16 * tc::BM && b.ld == (b.mn ? N : K);
  if (pre) {
    MatOp lo = b;
    lo.p = (const float*)scratch3((size_t)N * K * sizeof(float));
    tf32_lo_plane(b.p, (float*)lo.p, N * K);
    mat_map(&mbl, lo, N, K, batch, tma_b_rows(M, N, K, batch));
  }
  gemm_tma_bn(ma, mb, SA{a.batched ? 1 : 0}, SB{b.batched ? 1 : 0}, ep, M, N, K, batch, pre ? &mbl : nullptr);
}

// C = A . B^T through the TMA kernel when the path and the operands allow;
// returns false (nothing launched) otherwise.
template <class EP>
bool gemm_tma(const MatOp& a, const MatOp& b, const EP& ep, int64_t M, int64_t N, int64_t K, int batch) {
  if (!tma_enabled() || K <= 16 || M < 64 || N <= 0 || batch <= 0) return false;
  if (gemm_skinny_ok(M, N, batch)) return false;
  if (K > 0x7fffffff || M > 0x7fffffff || N > 0x7fffffff) return false;
  if (!mat_tma_ok(a, M) || !mat_tma_ok(b, N)) return false;
  if (a.mn) {
    if (b.mn) gemm_tma_mat<tma::SrcMN, tma::SrcMN>(a, b, ep, M, N, K, batch);
    else gemm_tma_mat<tma::SrcMN, tma::SrcK>(a, b, ep, M, N, K, batch);
  } else {
    if (b.mn) gemm_tma_mat<tma::SrcK, tma::SrcMN>(a, b, ep, M, N, K, batch);
    else gemm_tma_mat<tma::SrcK, tma::SrcK>(a, b, ep, M, N, K, batch);
  }
  return true;
}

}  // namespace tp
