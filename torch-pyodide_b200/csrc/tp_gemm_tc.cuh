// Tensor-core gather-GEMM for sm_100a: tcgen05.mma (kind::tf32) with the
// accumulator in TMEM and the 3xTF32 split for fp32 accuracy.
//
//   C(m, n) = sum_k A(m, k) B(n, k)
//   x = hi + lo, hi = x truncated to tf32 (10-bit mantissa), lo = x - hi (exact);
//   a*b ~= ah*bh + ah*bl + al*bh  (the dropped al*bl is ~2^-20 relative)
//
// CTA = 288 threads.  Warps 0-7 are producers in two groups of four; group g
// fills the k-blocks kb with kb % 2 == g, so two k-blocks are gathered at once.
// A producer gathers A and B through the loader functors (tp_gemm.cuh), splits
// each value into hi/lo with integer ops and stores both into 128-byte
// swizzled K-major shared-memory tiles (the canonical SWIZZLE_128B UMMA
// layout: 8-row x 128-byte atoms, 16-byte chunk c of row r stored at c ^ r).
// Warp 8 allocates TMEM and one lane issues the MMAs.  A ring of STAGES
// k-blocks (32 fp32 of K each) is guarded by mbarriers: a group arrives on
// full[s] after a proxy fence; the issuer's tcgen05.commit arrives on empty[s]
// when the tensor core has read the stage.  After the last k-block warps 0-7
// read the 128 x BN accumulator from TMEM (warp w: lanes 32*(w%4).., column half
// w/4) and run the epilogue functor.  grid.z = batch x split-K.
//
// Every mbarrier wait is bounded by %globaltimer; on expiry the kernel records
// an error code, skips the rest of its work, waits (bounded) for its last MMA
// commit and still frees its TMEM, so a scheduling bug surfaces as an error
// status instead of a hung GPU.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "tp_core.h"
#include "tp_gemm.cuh"

namespace tp {

namespace tc {

constexpr int BM = 128;
constexpr int BK = GB_K;                          // fp32 per k-block: one 128-byte swizzle row
constexpr int NTHREADS = 288;
constexpr int MMA_WARP = 8;
constexpr unsigned long long WAIT_NS = 2000000000ull;  // 2 s bound on any single wait

__device__ int g_status;  // 0 ok; nonzero: code of the first wait that timed out

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n.reg .b64 st;\nmbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; returns false (and records `code`) if the phase never
// completed within limit_ns.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int code,
                                              unsigned long long limit_ns) {
  if (mbar_try(bar, parity)) return true;
  unsigned long long t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255) == 0 && globaltimer() - t0 > limit_ns) {
      atomicCAS(&g_status, 0, code);
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  return mbar_wait_for(bar, parity, code, WAIT_NS);
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// hi = x with the 13 low mantissa bits cleared, which is the tf32 value the
// tensor core takes from an fp32 pattern, so an unconverted fp32 operand tile
// already is its own hi; lo = x - hi, exact in fp32 (|lo| < 2^-10 |x|; the
// tensor core reads it to 10 bits, so a*b is kept to ~2^-20 relative).
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = x - hi;
}

// Byte offset of fp32 element (row r, k) inside a K-major SWIZZLE_128B tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int k) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((((k >> 2) ^ (r & 7)) & 7) << 4) + (k & 3) * 4);
}

// UMMA shared-memory descriptor: K-major, SWIZZLE_128B, SBO = 1024 B (8-row
// atoms stacked along M/N), LBO unused (1), version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::tf32: D f32, A/B tf32, both K-major, M = 128.
template <int BN>
__device__ __forceinline__ uint32_t idesc_tf32() {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 consecutive columns of 32-bit TMEM cells into registers.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN, int STAGES>
struct Smem {
  static constexpr uint32_t A_BYTES = BM * BK * 4;               // 16 KB per A tile
  static constexpr uint32_t B_BYTES = BN * BK * 4;               // BN x 128 B per B tile
  static constexpr uint32_t STAGE = 2 * A_BYTES + 2 * B_BYTES;   // hi and lo of each
  static constexpr uint32_t TILES = STAGES * STAGE;
  static constexpr uint32_t BYTES = TILES + 256 + 1024;          // barriers, TMEM slot, alignment slack
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
};

// A producer group (128 threads, gtid 0..127) fills one operand tile of a
// stage in two halves, load (global -> registers) and store (split into hi/lo
// -> swizzled shared memory), so the next k-block's loads can be in flight
// while the current one is stored.  REGS values per thread.
//
// Loader contiguous along the row index: thread = tile row, 32 values of k.
template <class LD>
__device__ __forceinline__ void load_rows(const LD& ld, const typename LD::Row& rw, bool mine, int64_t k0,
                                          int64_t kend, float (&v)[BK]) {
  if (mine) ld.fill(rw, k0, kend, v);
}

__device__ __forceinline__ void store_rows(const float (&v)[BK], bool mine, int gtid, uint8_t* hi, uint8_t* lo) {
  if (!mine) return;
#pragma unroll
  for (int c = 0; c < BK / 4; ++c) {
    float4 h, l;
    split_tf32(v[4 * c], h.x, l.x);
    split_tf32(v[4 * c + 1], h.y, l.y);
    split_tf32(v[4 * c + 2], h.z, l.z);
    split_tf32(v[4 * c + 3], h.w, l.w);
    uint32_t off = sw128_off(gtid, 4 * c);
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) = l;
  }
}

// Loader contiguous along k: lane = k, the group's 4 warps take rows
// round-robin (ROWS/4 values per thread).
template <class LD, int ROWS>
__device__ __forceinline__ void load_kcontig(const LD& ld, int b, int64_t r0, int64_t rows_total, int gwarp,
                                             int lane, int64_t k0, int64_t kend, float (&v)[ROWS / 4]) {
  typename LD::Kc kc = ld.kctx(b, k0 + lane, kend);
#pragma unroll
  for (int i = 0; i < ROWS / 4; ++i) {
    int r = gwarp + 4 * i;
    v[i] = (r0 + r < rows_total) ? ld.at(b, r0 + r, kc) : 0.0f;
  }
}

template <int ROWS>
__device__ __forceinline__ void store_kcontig(const float (&v)[ROWS / 4], int gwarp, int lane, uint8_t* hi,
                                              uint8_t* lo) {
#pragma unroll
  for (int i = 0; i < ROWS / 4; ++i) {
    int r = gwarp + 4 * i;
    float h, l;
    split_tf32(v[i], h, l);
    uint32_t off = sw128_off(r, lane);
    *reinterpret_cast<float*>(hi + off) = h;
    *reinterpret_cast<float*>(lo + off) = l;
  }
}

// Registers per thread for one operand tile of ROWS rows.
template <class LD, int ROWS>
struct TileRegs {
  static constexpr int N = LD::kContigK ? ROWS / 4 : BK;
};

// Per-thread row context of a loader contiguous along the row index (none for
// loaders contiguous along k).
struct NoRow {};
template <class LD, bool KC = LD::kContigK>
struct RowOf {
  using type = typename LD::Row;
};
template <class LD>
struct RowOf<LD, true> {
  using type = NoRow;
};

template <class LA, class LB, class EP, int BN, int STAGES>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_gemm_tc(LA la, LB lb, EP ep, int64_t M, int64_t N, int64_t K, int64_t k_per_split, int splits,
              float* __restrict__ ws) {
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  // 1 KB aligned; derived from smem_raw by an offset so accesses stay shared-space loads/stores
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::TILES);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;
  // z = split * batch + b: the batches (filter taps) of one k range run side by side and share L2
  const int batch = (int)(gridDim.z / splits);
  const int b = (int)(blockIdx.z % batch), split = (int)(blockIdx.z / batch);
  const int64_t kb0 = (int64_t)split * k_per_split;
  const int64_t kend = kb0 + k_per_split < K ? kb0 + k_per_split : K;
  const int nk = kend > kb0 ? (int)((kend - kb0 + BK - 1) / BK) : 0;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  // the predecessor kernel has finished before this CTA allocates tensor memory
  // or touches global memory; dependents may launch once all CTAs hold theirs
  ::tp::pdl_wait();
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)S::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  ::tp::pdl_trigger();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp < 8) {
    // ---- producers: group = warp / 4 takes every other k-block ----
    const int group = warp >> 2, gtid = tid & 127, gwarp = warp & 3;
    typename RowOf<LA>::type ra{};
    typename RowOf<LB>::type rb{};
    if constexpr (!LA::kContigK) ra = la.row(b, m0 + gtid, M);
    if constexpr (!LB::kContigK) rb = lb.row(b, n0 + (gtid < BN ? gtid : 0), N);
    const bool bmine = gtid < BN;
    float va[1][TileRegs<LA, BM>::N], vb[1][TileRegs<LB, BN>::N];
    auto load = [&](int kb, int slot) {
      int64_t k0 = kb0 + (int64_t)kb * BK;
      if constexpr (LA::kContigK) load_kcontig<LA, BM>(la, b, m0, M, gwarp, lane, k0, kend, va[slot]);
      else load_rows(la, ra, true, k0, kend, va[slot]);
      if constexpr (LB::kContigK) load_kcontig<LB, BN>(lb, b, n0, N, gwarp, lane, k0, kend, vb[slot]);
      else load_rows(lb, rb, bmine, k0, kend, vb[slot]);
    };
    auto store = [&](int kb, int slot) {
      int s = kb % STAGES;
      ok = mbar_wait(&empty[s], (uint32_t)((kb / STAGES) & 1) ^ 1u, 1);
      if (!ok) return;
      uint8_t* st = smem + s * S::STAGE;
      uint8_t* bh = st + 2 * S::A_BYTES;
      if constexpr (LA::kContigK) store_kcontig<BM>(va[slot], gwarp, lane, st, st + S::A_BYTES);
      else store_rows(va[slot], true, gtid, st, st + S::A_BYTES);
      if constexpr (LB::kContigK) store_kcontig<BN>(vb[slot], gwarp, lane, bh, bh + S::B_BYTES);
      else store_rows(vb[slot], bmine, gtid, bh, bh + S::B_BYTES);
      fence_proxy_async();
      mbar_arrive(&full[s]);
    };
    // the loads of a k-block are issued before its stage is waited for, so
    // their latency overlaps the wait
    for (int kb = group; kb < nk && ok; kb += 2) {
      load(kb, 0);
      store(kb, 0);
    }
  } else if (lane == 0) {
    // ---- MMA issuer ----
    const uint32_t idesc = idesc_tf32<BN>();
    for (int kb = 0; kb < nk && ok; ++kb) {
      int s = kb % STAGES;
      ok = mbar_wait(&full[s], (uint32_t)((kb / STAGES) & 1), 2);
      if (!ok) break;
      tc_fence_after();
      uint32_t base = smem_u32(smem + s * S::STAGE);
      uint64_t ahi = sw128_desc(base), alo = sw128_desc(base + S::A_BYTES);
      uint64_t bhi = sw128_desc(base + 2 * S::A_BYTES), blo = sw128_desc(base + 2 * S::A_BYTES + S::B_BYTES);
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        uint64_t adv = (uint64_t)(kk * 32) >> 4;  // 8 tf32 = 32 bytes along K inside the swizzle atom
        mma_tf32(tmem, ahi + adv, bhi + adv, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        mma_tf32(tmem, ahi + adv, blo + adv, idesc, 1u);
        mma_tf32(tmem, alo + adv, bhi + adv, idesc, 1u);
      }
      mma_commit(&empty[s]);
    }
    mma_commit(done);
  }
  __syncwarp();

  // ---- epilogue: warps 0-7; TMEM lane quadrant warp%4 = tile rows, column half warp/4 ----
  if (warp < 8) {
    // always wait for the final commit (bounded) so no MMA is in flight when
    // TMEM is freed; keep tcgen05.ld warp-uniform
    bool fin = nk > 0 && mbar_wait(done, 0, 3);
    bool have = __all_sync(0xffffffffu, ok && fin);
    tc_fence_after();
    const int q = warp & 3, h = warp >> 2;
    const int64_t m = m0 + q * 32 + lane;
    constexpr int HALF = BN / 2;
#pragma unroll 1
    for (int c0 = h * HALF; c0 < (h + 1) * HALF; c0 += 16) {
      float v[16];
      if (have) {
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.0f;
      }
      if (m < M && (have || nk == 0)) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          int64_t n = n0 + c0 + i;
          if (n < N) {
            if (splits > 1) ws[(((int64_t)b * splits + split) * M + m) * N + n] = v[i];
            else ep(b, m, n, v[i]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)S::TMEM_COLS));
  }
}

// Sum the split-K partials of batch b in split order and apply the epilogue
// (16-byte partial loads when N % 4 == 0).
template <class EP>
__global__ void k_splitk_reduce_b(const float* __restrict__ ws, int splits, int64_t M, int64_t N, EP ep) {
  ::tp::pdl_enter();
  const int b = blockIdx.y;
  const int64_t MN = M * N;
  const float* base = ws + (int64_t)b * splits * MN;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if ((N & 3) == 0) {
    const int64_t n4 = MN >> 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
      // four splits' loads in flight at a time, added in split order
      float4 s = reinterpret_cast<const float4*>(base)[i];
      int z = 1;
      for (; z + 4 <= splits; z += 4) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = reinterpret_cast<const float4*>(base + (int64_t)(z + u) * MN)[i];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          s.x += v[u].x;
          s.y += v[u].y;
          s.z += v[u].z;
          s.w += v[u].w;
        }
      }
      for (; z < splits; ++z) {
        float4 v = reinterpret_cast<const float4*>(base + (int64_t)z * MN)[i];
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      const int64_t e = i * 4, m = e / N, n = e - m * N;
      ep(b, m, n, s.x);
      ep(b, m, n + 1, s.y);
      ep(b, m, n + 2, s.z);
      ep(b, m, n + 3, s.w);
    }
    return;
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < MN; i += stride) {
    float s = 0.0f;
    int z = 0;
    for (; z + 8 <= splits; z += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = base[(int64_t)(z + u) * MN + i];
#pragma unroll
      for (int u = 0; u < 8; ++u) s += v[u];
    }
    for (; z < splits; ++z) s += base[(int64_t)z * MN + i];
    ep(b, i / N, i % N, s);
  }
}

}  // namespace tc

// Host side: read (and optionally clear) the device status word.
int tc_status(bool reset);
int tc_status_nhwc(bool reset);  // the channels-last conv module's status word

// Split-K factor shared by the tensor-core launchers: minimise the k-blocks
// one SM runs (waves x k-blocks per split) plus the split-K partial traffic
// (each split writes and the reduce reads out_elems floats; one unit ~ one
// k-block of time per ~0.7 M floats of the whole GPU's traffic), keeping
// >= 8 k-blocks per split.
int gemm_kmax();

inline int gemm_splits(int64_t tiles, int64_t K, int sms, int64_t out_elems) {
  if (K <= 0 || tiles <= 0) return 1;
  const int64_t nk = (K + 31) / 32;
  // Accuracy floor for long reductions (weight gradients over many pixels): the
  // tensor core's fp32 accumulation drifts over thousands of MMAs into one
  // accumulator, so no split of such a GEMM accumulates more than kmax k-blocks.
  // Forward / data-gradient K (<= 4 kmax k-blocks) keeps the cost-model split;
  // longer reductions take at least ceil(nk / kmax) splits, more where the
  // cost model wants more CTAs than that (few output tiles).
  const int kmax = gemm_kmax();
  int64_t need = 1;
  if (kmax > 0 && nk > 4 * (int64_t)kmax) need = (nk + kmax - 1) / kmax;
  if (need > 2048) need = 2048;
  int64_t maxs = nk / 8;
  if (maxs > 64) maxs = 64;
  if (maxs <= 1) return (int)need;
  int best = 1;
  double best_t = 1e300;
  for (int s = 1; s <= maxs; ++s) {
    const int64_t waves = (tiles * s + sms - 1) / sms;
    const double t = (double)waves * (double)((nk + s - 1) / s) + (s > 1 ? 1.4e-6 * (double)out_elems * s : 0.0);
    if (t < best_t * (1.0 - 1e-9)) {
      best_t = t;
      best = s;
    }
  }
  return best > need ? best : (int)need;
}

template <class LA, class LB, class EP, int BN, int STAGES>
void gemm_tc_launch(const LA& la, const LB& lb, const EP& ep, int64_t M, int64_t N, int64_t K, int batch) {
  using S = tc::Smem<BN, STAGES>;
  int64_t gm = (M + tc::BM - 1) / tc::BM, gn = (N + BN - 1) / BN;
  TP_REQUIRE(gn <= 65535 && gm <= 0x7fffffff, "gemm: tile grid exceeds the launch limits");
  auto kfn = tc::k_gemm_tc<LA, LB, EP, BN, STAGES>;
  static bool attr = false;
  if (!attr) {
    TP_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::BYTES));
    attr = true;
  }
  // split K when the tile grid cannot fill the SMs
  int splits = gemm_splits(gm * gn * batch, K, sm_count(), M * N * batch);
  int64_t kps = (K + splits - 1) / splits;
  kps = (kps + tc::BK - 1) / tc::BK * tc::BK;
  splits = K > 0 ? (int)((K + kps - 1) / kps) : 1;
  TP_REQUIRE((int64_t)batch * splits <= 65535, "gemm: batch x splits exceeds the grid limit");
  float* ws = nullptr;
  if (splits > 1) ws = (float*)scratch((size_t)batch * splits * M * N * sizeof(float));
  TP_LAUNCH(kfn, dim3((unsigned)gm, (unsigned)gn, (unsigned)(batch * splits)), tc::NTHREADS, S::BYTES, la, lb, ep,
            M, N, K, kps, splits, ws);
  if (splits > 1) {
    auto rfn = tc::k_splitk_reduce_b<EP>;
    unsigned gx = (unsigned)((M * N / 4 + 255) / 256 + 1);
    if (gx > (unsigned)sm_count() * 8) gx = (unsigned)sm_count() * 8;
    TP_LAUNCH(rfn, dim3(gx, (unsigned)batch), 256, 0, ws, splits, M, N, ep);
  }
}

}  // namespace tp
