// The TMA-fed 3xTF32 GEMM on CTA pairs: tcgen05.mma.cta_group::2.
//
// Two CTAs of a cluster (ranks 0 and 1, on two SMs) compute a 256 x BNP tile
// with M = 256 MMAs issued by one thread of rank 0.  Each CTA holds its own
// 128 rows of A (hi / lo in its own TMEM, split by its own splitter warps,
// exactly as in tp_gemm_tma.cuh) and HALF of B: the BNH = BNP / 2 columns
// [n0 + rank * BNH, n0 + (rank + 1) * BNH) in its own shared memory, raw tile
// and tf32 low parts.  The tensor cores of the pair read both halves, so per
// SM and per k-block the shared-memory traffic is that of a 128 x BNH tile
// while the MMA work is that of a 128 x BNP one -- half the bytes per flop of
// the single-CTA kernel, whose main loop is bound by shared-memory bandwidth.
//
// Pipeline per stage s (each CTA has its own ring; the MMA lane of rank 0 is
// the only consumer):
//   full[s]   own TMA boxes landed (A rows, B half; tx count)
//   ready[s]  on rank 0 only: one arrival per splitter warp of BOTH CTAs (16),
//             the peer's by remote arrive (mapa + mbarrier.arrive.shared::cluster)
//   empty[s]  the MMAs that read stage s are done: rank 0's tcgen05.commit
//             multicast to the barrier at the same offset in both CTAs
//   done      all MMAs done (same multicast commit); each CTA then reads its own
//             128 TMEM lanes x BNP columns and stores its rows
// TMEM (512 columns, allocated by one warp of each CTA together): the
// accumulator at [0, BNP), A stage s at 256 + 64 s (hi) / + 32 (lo).
//
// TMA loads carry no multicast: each CTA loads its own boxes from this GPU's
// memory.  Every wait is bounded (tc::WAIT_NS) and records a code in
// tc::g_status when it expires.  The MMA sequence per output element (k order,
// the three products per 8-wide k-step) is that of the single-CTA kernel.
#pragma once

#include "tp_gemm_tma.cuh"

namespace tp {

namespace tma2 {

using tc::BK;
using tc::BM;
constexpr int NTHREADS = 320;
constexpr int NSPLIT = 256;
constexpr int MMA_WARP = 8;
constexpr int TMA_WARP = 9;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t A_TMEM0 = 256;
constexpr uint32_t READY_COUNT = 2 * NSPLIT / 32;  // splitter warps of both CTAs

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Arrive on a barrier of either CTA of the pair (default .release.cta
// semantics, as the remote arrivals of CUTLASS's cluster pipelines): the
// splitters' TMEM stores are ordered before it by tcgen05.wait::st and
// tcgen05.fence::before_thread_sync, and their TMA data by the tx count of
// their own full barrier.  A .release.cluster arrive would order every prior
// memory access of the thread at cluster scope, which costs ~1000 cycles per
// k-block on the splitters' critical path.
__device__ __forceinline__ void arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool try_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, "
      "0, p;\n}"
      : "=r"(ok)
      : "r"(tc::smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// bounded wait, acquire at cluster scope (the arrivals come from the peer CTA)
__device__ __forceinline__ bool wait_cluster(uint64_t* bar, uint32_t parity, int code) {
  if (try_cluster(bar, parity)) return true;
  const unsigned long long t0 = tc::globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (try_cluster(bar, parity)) return true;
    if ((i & 255) == 0 && tc::globaltimer() - t0 > tc::WAIT_NS) {
      atomicCAS(&tc::g_status, 0, code);
      return false;
    }
  }
}

// kind::tf32, D f32, M = 256 (the pair), N = BNP; bits 15 / 16 (operand majors) set by the caller
template <int BNP>
__device__ __forceinline__ uint32_t idesc_tf32_m256() {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BNP >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

__device__ __forceinline__ void mma2_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                             uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
}

// arrive on the barrier at this offset in both CTAs once the MMAs issued so far are done
__device__ __forceinline__ void commit2(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          tc::smem_u32(bar)),
      "h"((unsigned short)3)
      : "memory");
}

template <class SA, class SB, class EP, int BNH, int STAGES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTHREADS, 1)
    k_gemm_tma2(const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mb,
                const __grid_constant__ CUtensorMap mbl, SA sa, SB sb, EP ep, int64_t M, int64_t N, int64_t K,
                int64_t k_per_split, int splits, float* __restrict__ ws, int b_lo) {
  using S = tma::Smem<BNH, STAGES>;
  constexpr int BNP = 2 * BNH;
  static_assert(BNP <= 256, "the accumulator takes columns [0, 256)");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::TILES);
  uint64_t* ready = full + STAGES;
  uint64_t* empty = ready + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // the tensor maps are kernel parameters, not data of the predecessor kernel: fetch them
  // while it drains
  if (warp == TMA_WARP && lane == 0) {
    tma::prefetch_map(&ma);
    tma::prefetch_map(&mb);
    if (b_lo) tma::prefetch_map(&mbl);
  }
  const uint32_t rank = cluster_rank();
  const int64_t m0 = (int64_t)blockIdx.x * BM;  // this CTA's rows
  const int64_t n0p = (int64_t)blockIdx.y * BNP;  // the pair's columns
  const int64_t n0 = n0p + (int64_t)rank * BNH;  // this CTA's half of B
  const int batch = (int)(gridDim.z / splits);
  const int b = (int)(blockIdx.z % batch), split = (int)(blockIdx.z / batch);
  const int64_t kb0 = (int64_t)split * k_per_split;
  const int64_t kend = kb0 + k_per_split < K ? kb0 + k_per_split : K;
  const int nk = kend > kb0 ? (int)((kend - kb0 + BK - 1) / BK) : 0;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&ready[s], READY_COUNT);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(done, 1);
    tc::fence_barrier_init();
  }
  // the predecessor kernel has finished before this CTA allocates tensor memory
  // or touches global memory; dependents may launch once all CTAs hold theirs
  ::tp::pdl_wait();
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     tc::smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc::tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised before any remote arrive
  ::tp::pdl_trigger();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == TMA_WARP) {
    if (lane == 0) {
      int last[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last[s] = -1;
      auto ca = sa.template begin<BM>(b, m0, kb0);
      auto cb = sb.template begin<BNH>(b, n0, kb0);
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % STAGES;
        ok = wait_cluster(&empty[s], (uint32_t)((kb / STAGES) & 1) ^ 1u, 31);
        if (!ok) break;
        const uint32_t st = tc::smem_u32(smem + s * S::STAGE);
        tma::expect_tx(&full[s], S::A_BYTES + (b_lo ? 2u : 1u) * S::B_BYTES);
        sa.issue(&ma, st, &full[s], ca);
        sb.issue(&mb, st + S::A_BYTES, &full[s], cb);
        if (b_lo) sb.issue(&mbl, st + S::A_BYTES + S::B_BYTES, &full[s], cb);
        sa.next(ca);
        sb.next(cb);
        last[s] = kb;
      }
#pragma unroll
      for (int s = 0; s < STAGES; ++s)
        if (last[s] >= 0) tc::mbar_wait(&full[s], (uint32_t)((last[s] / STAGES) & 1), 32);
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = idesc_tf32_m256<BNP>() | ((uint32_t)SB::kMN << 16);
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % STAGES;
        ok = wait_cluster(&ready[s], (uint32_t)((kb / STAGES) & 1), 33);
        if (!ok) break;
        tc::tc_fence_after();
        const uint32_t base = tc::smem_u32(smem + s * S::STAGE);
        const uint32_t b_hi = base + S::A_BYTES, b_lo_addr = base + S::A_BYTES + S::B_BYTES;
        const uint32_t a_hi = tmem + A_TMEM0 + 64 * s, a_lo = a_hi + 32;
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint32_t db = SB::kMN ? kk * 1024 : kk * 32;
          const uint64_t bh = SB::kMN ? tma::mn_desc(b_hi + db) : tc::sw128_desc(b_hi + db);
          const uint64_t bl = SB::kMN ? tma::mn_desc(b_lo_addr + db) : tc::sw128_desc(b_lo_addr + db);
          mma2_tf32_ts(tmem, a_hi + 8 * kk, bh, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          mma2_tf32_ts(tmem, a_hi + 8 * kk, bl, idesc, 1u);
          mma2_tf32_ts(tmem, a_lo + 8 * kk, bh, idesc, 1u);
        }
        commit2(&empty[s]);
      }
      commit2(done);
    }
  } else {
    // ---- splitters (both CTAs): own A rows -> own TMEM hi/lo; own B half's lo ----
    const int r = 32 * (warp & 3) + lane, kh = (warp >> 2) * 16;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int s = kb % STAGES;
      ok = tc::mbar_wait(&full[s], (uint32_t)((kb / STAGES) & 1), 34);
      if (!ok) break;
      uint8_t* st = smem + s * S::STAGE;
      {
        float v[16];
        uint32_t h[16], l[16];
        tma::read_a16<SA::kMN>(st, r, kh, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float hf, lf;
          tc::split_tf32(v[i], hf, lf);
          h[i] = __float_as_uint(hf);
          l[i] = __float_as_uint(lf);
        }
        const uint32_t col = tmem + lane_base + A_TMEM0 + 64 * s + kh;
        tma::tmem_st16(col, h);
        tma::tmem_st16(col + 32, l);
      }
      if (!b_lo) {
        const float4* hi = reinterpret_cast<const float4*>(st + S::A_BYTES);
        float4* lo = reinterpret_cast<float4*>(st + S::A_BYTES + S::B_BYTES);
#pragma unroll
        for (int i = tid; i < (int)(S::B_BYTES / 16); i += NSPLIT) {
          float4 v = hi[i], h, l;
          tc::split_tf32(v.x, h.x, l.x);
          tc::split_tf32(v.y, h.y, l.y);
          tc::split_tf32(v.z, h.z, l.z);
          tc::split_tf32(v.w, h.w, l.w);
          lo[i] = l;
        }
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc::fence_proxy_async();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_cluster(mapa(tc::smem_u32(&ready[s]), 0));
    }
  }
  __syncwarp();

  // ---- epilogue: warps 0-7 of each CTA; its TMEM lanes = its 128 rows, all BNP columns ----
  if (warp < 8) {
    const bool fin = nk > 0 && wait_cluster(done, 0, 35);
    const bool have = __all_sync(0xffffffffu, ok && fin);
    tc::tc_fence_after();
    const int q = warp & 3, h = warp >> 2;
    const int64_t m = m0 + q * 32 + lane;
    constexpr int HALF = BNP / 2;
    static_assert(128u * (BNP + 4) * 4 <= S::TILES, "the staged epilogue tile must fit in the operand ring");
    if (HasRow4<EP>::value || splits > 1) {
      if (have || nk == 0)
        tma::staged_rows<BNP>(reinterpret_cast<float*>(smem), q, h, lane, tmem, have, m0, n0p, M, N, b, split,
                              splits, ws, ep);
    } else {
#pragma unroll 1
    for (int c0 = h * HALF; c0 < (h + 1) * HALF; c0 += 16) {
      float v[16];
      if (have) {
        tc::tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.0f;
      }
      if (m < M && (have || nk == 0)) {
        if (splits > 1) {
          float* w = ws + (((int64_t)b * splits + split) * M + m) * N;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (n0p + c0 + i < N) w[n0p + c0 + i] = v[i];
        } else {
          ep.row16(b, m, n0p + c0, N, v);
        }
      }
    }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA frees TMEM or leaves while the pair's MMAs may read it
  if (warp == MMA_WARP) {
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

}  // namespace tma2

// CTA pairs: grid.x = the row tiles rounded up to even (a pair's second CTA
// past M loads zeros and stores nothing).  B's tensor map box is BNH rows.
template <class SA, class SB, class EP, int BNH, int STAGES>
void gemm_tma2_launch(const CUtensorMap& ma, const CUtensorMap& mb, const SA& sa, const SB& sb, const EP& ep,
                      int64_t M, int64_t N, int64_t K, int batch, const CUtensorMap* mbl = nullptr) {
  using S = tma::Smem<BNH, STAGES>;
  constexpr int BNP = 2 * BNH;
  int64_t gm = (M + tma::BM - 1) / tma::BM, gn = (N + BNP - 1) / BNP;
  gm = (gm + 1) & ~(int64_t)1;
  TP_REQUIRE(gn <= 65535 && gm <= 0x7fffffff, "gemm: tile grid exceeds the launch limits");
  auto kfn = tma2::k_gemm_tma2<SA, SB, EP, BNH, STAGES>;
  static bool attr = false;
  if (!attr) {
    TP_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::BYTES));
    attr = true;
  }
  int splits = gemm_splits(gm * gn * batch, K, sm_count(), M * N * batch);
  int64_t kps = (K + splits - 1) / splits;
  kps = (kps + tma::BK - 1) / tma::BK * tma::BK;
  splits = K > 0 ? (int)((K + kps - 1) / kps) : 1;
  TP_REQUIRE((int64_t)batch * splits <= 65535, "gemm: batch x splits exceeds the grid limit");
  float* ws = nullptr;
  if (splits > 1) ws = (float*)scratch((size_t)batch * splits * M * N * sizeof(float));
  TP_LAUNCH(kfn, dim3((unsigned)gm, (unsigned)gn, (unsigned)(batch * splits)), tma2::NTHREADS, S::BYTES, ma, mb,
            mbl ? *mbl : mb, sa, sb, ep, M, N, K, kps, splits, ws, mbl ? 1 : 0);
  if (splits > 1) {
    auto rfn = tc::k_splitk_reduce_b<EP>;
    unsigned gx = (unsigned)((M * N / 4 + 255) / 256 + 1);
    if (gx > (unsigned)sm_count() * 8) gx = (unsigned)sm_count() * 8;
    TP_LAUNCH(rfn, dim3(gx, (unsigned)batch), 256, 0, ws, splits, M, N, ep);
  }
}

}  // namespace tp
