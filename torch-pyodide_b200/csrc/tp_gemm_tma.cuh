// TMA-fed tensor-core GEMM for sm_100a: tcgen05.mma (kind::tf32), accumulator
// in TMEM, 3xTF32 split for fp32 accuracy.
//
//   C(m, n) = sum_k A(m, k) B(n, k),   a*b ~= ah*bh + ah*bl + al*bh
//
// Operand tiles arrive by TMA (cp.async.bulk.tensor, no multicast) straight
// into 128-byte-swizzled shared memory, so no thread computes a gather
// address.  Each operand is either K-major (a tile row = 32 consecutive k of
// one m/n, the same canonical layout as the gather kernel) or MN-major (32
// consecutive m/n per 128-byte row, one row per k, 32-byte-atom swizzle;
// 32-wide column groups LBO = 4 KB apart, 4-row k groups SBO = 512 B apart),
// chosen by the source
// functor, so transposed operands and channels-last convolution operands are
// read in place.
//
// CTA = 320 threads, one CTA per SM (it allocates all 512 TMEM columns):
//   warp 9, one lane   TMA producer: waits empty[s], arms full[s] with the
//                      stage's byte count, issues the A and B boxes
//   warps 0-7          splitters: wait full[s]; split each A value into its
//                      tf32 hi and lo = x - hi and store both into TMEM
//                      (tcgen05.st; thread = tile row, 16 k each); write B's
//                      lo beside the raw B tile, which is its own hi (the
//                      tensor core reads fp32 as tf32 by dropping the 13 low
//                      mantissa bits); fence, arrive on ready[s]; after the
//                      last k-block they run the epilogue
//   warp 8             allocates TMEM; one lane issues 3 MMAs per 8-wide
//                      k-step, A read from TMEM and B from shared memory, once
//                      ready[s] completes, and commits to empty[s]
// When B is reused by many tiles (conv filters) its tf32 low parts can be
// computed once into memory (tf32_lo_plane) and loaded by TMA beside the raw
// tile, which takes the splitters' B pass (16 + 16 KB of shared memory
// traffic per k-block at BN = 128) off the critical path.
// With A in TMEM the tensor core reads only B from shared memory, which is
// what bounds this kernel: per k-block and 128-wide N tile, 128 KB of shared
// memory traffic (TMA writes 32, splitter reads 32 and writes 16, MMA reads
// 48) instead of 224 KB with both operands and both halves there.
// The split is the same as the gather kernel's (tp_gemm_tc.cuh) and the MMA
// sequence is the same, so both kernels produce identical bits for the same
// tile shape and split-K.
//
// Every wait is bounded (2 s by %globaltimer): on expiry the kernel records a
// code in tc::g_status, stops issuing, waits (bounded) for the boxes and MMAs
// it already issued and frees its TMEM.
#pragma once

#include <cuda.h>

#include "tp_gemm_tc.cuh"

namespace tp {

namespace tma {

using tc::BK;
using tc::BM;
constexpr int NTHREADS = 320;
constexpr int NSPLIT = 256;  // splitter threads (warps 0-7)
constexpr int MMA_WARP = 8;
constexpr int TMA_WARP = 9;

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void load3(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(tc::smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void load4(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w,
                                      uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(tc::smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void load5(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, int c4,
                                      uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5, %6}], [%7];" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(tc::smem_u32(bar))
      : "memory");
}

// MN-major descriptor for tf32: layout SWIZZLE_128B_BASE32B (32-byte chunks
// of each 128-byte row permuted over 4-row periods), column groups of 32 fp32
// LBO = 4 KB apart, 4-row k groups SBO = 512 B apart.
__device__ __forceinline__ uint64_t mn_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(4096 >> 4) << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)1 << 61;
  return d;
}

// ---- operand sources: issue the boxes of one ROWS x 32 tile --------------------------------------

// Every source hands the producer lane a cursor: begin() places it at the
// tile's first k-block (the only place that divides), issue() copies the
// k-block it points at, next() moves it on by 32 k with additions only.

// K-major rows of a row-major [batch][rows][K] tensor; map dims (K, rows, batch), box (32, ROWS, 1).
// bmul = 0 when every batch shares the matrix.
struct SrcK {
  static constexpr bool kMN = false;
  int bmul;
  struct Cur {
    int k, r, z;
  };
  template <int ROWS>
  __device__ __forceinline__ Cur begin(int b, int64_t r0, int64_t k0) const {
    return {(int)k0, (int)r0, b * bmul};
  }
  __device__ __forceinline__ void issue(const CUtensorMap* map, uint32_t dst, uint64_t* bar, const Cur& c) const {
    load3(dst, map, c.k, c.r, c.z, bar);
  }
  __device__ __forceinline__ void next(Cur& c) const { c.k += 32; }
};

// MN-major: a row-major [batch][K][rows] tensor (rows contiguous).  Map dims
// (32, K, rows/32, batch) with the 32-wide row groups as an outer dimension
// (stride 128 B), box (32, 32, ROWS/32, 1): one box lands the tile as 32-row
// groups 4 KB apart, each 32 k-rows of 128 B.
struct SrcMN {
  static constexpr bool kMN = true;
  int bmul;
  struct Cur {
    int k, rg, z;
  };
  template <int ROWS>
  __device__ __forceinline__ Cur begin(int b, int64_t r0, int64_t k0) const {
    return {(int)k0, (int)(r0 >> 5), b * bmul};
  }
  __device__ __forceinline__ void issue(const CUtensorMap* map, uint32_t dst, uint64_t* bar, const Cur& c) const {
    load4(dst, map, 0, c.k, c.rg, c.z, bar);
  }
  __device__ __forceinline__ void next(Cur& c) const { c.k += 32; }
};

// Pixel tiles of an OH x OW output grid (N images): a tile is a TW x TH
// rectangle of one image (TN == 1, tiles_w x tiles_h tiles per image, the
// last row / column of tiles may reach past the grid) or TN whole images.
// Tile t covers GEMM rows (or k) [t*rows, (t+1)*rows) in the order w fastest,
// then h, then image, which is the order a TMA box of extents (TW, TH, TN)
// lands in shared memory.  With tiles_w == 1 and TW == OW the order is the
// plain pixel order n*OH*OW + oh*OW + ow.
struct PixTile {
  int OH, OW, TW, TH, TN, tiles_w, tiles_h;
  __device__ __forceinline__ void origin(int64_t t, int& n0, int& oh0, int& ow0) const {
    if (TN > 1) {
      n0 = (int)(t * TN);
      oh0 = 0;
      ow0 = 0;
      return;
    }
    const int per = tiles_w * tiles_h;
    n0 = (int)(t / per);
    const int r = (int)(t - (int64_t)n0 * per);
    oh0 = (r / tiles_w) * TH;
    ow0 = (r - (r / tiles_w) * tiles_w) * TW;
  }
  // GEMM row m (tile = m / rows) -> pixel; false when it falls outside the grid
  __device__ __forceinline__ bool pixel(int64_t m, int rows, int64_t N, int& n, int& oh, int& ow) const {
    const int64_t t = m / rows;
    const int r = (int)(m - t * rows);
    int n0, oh0, ow0;
    origin(t, n0, oh0, ow0);
    const int twh = TW * TH;
    n = n0 + r / twh;
    const int rr = r - (r / twh) * twh;
    oh = oh0 + rr / TW;
    ow = ow0 + (rr - (rr / TW) * TW);
    return n < N && oh < OH && ow < OW;
  }
};

// K-major implicit-GEMM operand of a stride-1 convolution over a channels-last
// [N][H][W][C] input: tile rows = the 128 output pixels of one pixel tile,
// k-block = (tap, 32 channels) with taps outermost.  Map dims (C, W, H, N),
// box (32, TW, TH, TN); the tap shift moves the box origin and the zero fill
// outside the input is the padding.
struct SrcConvK {
  static constexpr bool kMN = false;
  PixTile pt;
  int cblocks, KW, PH, PW;
  int DW = 1;  // spacing of the taps along W (2: the paired space-to-depth stem)
  struct Cur {
    int c0, kh, kw, n0, oh0, ow0;
  };
  template <int ROWS>
  __device__ __forceinline__ Cur begin(int, int64_t r0, int64_t k0) const {
    Cur c;
    pt.origin(r0 / ROWS, c.n0, c.oh0, c.ow0);
    const int kb = (int)(k0 >> 5), tap = kb / cblocks;
    c.c0 = (kb - tap * cblocks) * 32;
    c.kh = tap / KW;
    c.kw = tap - c.kh * KW;
    return c;
  }
  __device__ __forceinline__ void issue(const CUtensorMap* map, uint32_t dst, uint64_t* bar, const Cur& c) const {
    load4(dst, map, c.c0, c.ow0 + c.kw * DW - PW, c.oh0 + c.kh - PH, c.n0, bar);
  }
  __device__ __forceinline__ void next(Cur& c) const {
    c.c0 += 32;
    if (c.c0 == cblocks * 32) {
      c.c0 = 0;
      if (++c.kw == KW) {
        c.kw = 0;
        ++c.kh;
      }
    }
  }
};

// MN-major operand of the per-tap weight gradient over a channels-last tensor:
// tile rows = channels, k = output pixels in pixel-tile order, one 32-pixel
// tile per k-block.  Batch index b = tap; with `shift` the pixel reads move by
// the tap offset (the input x), without it they do not (the output gradient
// dy); pixels outside the grid read zeros in dy, so they add nothing.  Map
// dims (32, W, H, N, C/32): channel groups of 32 as the outermost dimension
// (stride 128 B), box (32, TW, TH, TN, ROWS/32) covering every group of the
// tile in one copy.
struct SrcPixMN {
  static constexpr bool kMN = true;
  PixTile pt;
  int KW, PH, PW, shift;
  int DW = 1;  // tap spacing along W
  // k-block = one 32-pixel tile (n0, tile row th, tile column tw)
  struct Cur {
    int n0, th, tw, dh, dw, cg;
  };
  template <int ROWS>
  __device__ __forceinline__ Cur begin(int b, int64_t r0, int64_t k0) const {
    Cur c;
    int oh0, ow0;
    pt.origin(k0 >> 5, c.n0, oh0, ow0);
    c.th = pt.TN > 1 ? 0 : oh0 / pt.TH;
    c.tw = pt.TN > 1 ? 0 : ow0 / pt.TW;
    c.dh = shift ? b / KW - PH : 0;
    c.dw = shift ? (b - (b / KW) * KW) * DW - PW : 0;
    c.cg = (int)(r0 >> 5);
    return c;
  }
  __device__ __forceinline__ void issue(const CUtensorMap* map, uint32_t dst, uint64_t* bar, const Cur& c) const {
    load5(dst, map, 0, c.tw * pt.TW + c.dw, c.th * pt.TH + c.dh, c.n0, c.cg, bar);
  }
  __device__ __forceinline__ void next(Cur& c) const {
    if (pt.TN > 1) {
      c.n0 += pt.TN;
    } else if (++c.tw == pt.tiles_w) {
      c.tw = 0;
      if (++c.th == pt.tiles_h) {
        c.th = 0;
        ++c.n0;
      }
    }
  }
};

// SrcPixMN for the input operand of a several-tap weight gradient: batch b =
// taps (TAPS*b .. TAPS*b + TAPS - 1), the B tile's 128 rows are the 128/TAPS
// input channels shifted by each tap in turn (Cin = 64: 2 taps; Cin = 32: 4),
// one box of 128/TAPS channels per tap, 4 KB x 32/TAPS... apart.  Taps past KHW
// repeat the last one (their columns are dropped by the epilogue).
template <int TAPS>
struct SrcPixMNT {
  static constexpr bool kMN = true;
  static constexpr uint32_t kTapBytes = 16384 / TAPS;  // (128 / TAPS) rows of the MN-major tile
  PixTile pt;
  int KW, PH, PW, KHW;
  int DW = 1;  // tap spacing along W
  struct Cur {
    int n0, th, tw;
    int dh[TAPS], dw[TAPS];
  };
  template <int ROWS>
  __device__ __forceinline__ Cur begin(int b, int64_t, int64_t k0) const {
    static_assert(ROWS == 128, "128-row B tiles");
    Cur c;
    int oh0, ow0;
    pt.origin(k0 >> 5, c.n0, oh0, ow0);
    c.th = pt.TN > 1 ? 0 : oh0 / pt.TH;
    c.tw = pt.TN > 1 ? 0 : ow0 / pt.TW;
#pragma unroll
    for (int j = 0; j < TAPS; ++j) {
      const int t = TAPS * b + j < KHW ? TAPS * b + j : KHW - 1;
      c.dh[j] = t / KW - PH;
      c.dw[j] = (t - (t / KW) * KW) * DW - PW;
    }
    return c;
  }
  __device__ __forceinline__ void issue(const CUtensorMap* map, uint32_t dst, uint64_t* bar, const Cur& c) const {
    const int ow = c.tw * pt.TW, oh = c.th * pt.TH;
#pragma unroll
    for (int j = 0; j < TAPS; ++j) load5(dst + j * kTapBytes, map, 0, ow + c.dw[j], oh + c.dh[j], c.n0, 0, bar);
  }
  __device__ __forceinline__ void next(Cur& c) const {
    if (pt.TN > 1) {
      c.n0 += pt.TN;
    } else if (++c.tw == pt.tiles_w) {
      c.tw = 0;
      if (++c.th == pt.tiles_h) {
        c.th = 0;
        ++c.n0;
      }
    }
  }
};

// MN-major B of the flipped-filter data gradient, read from filters stored
// [Cout][KH*KW][Cin]: rows = input channels, k = (flipped tap, output channel)
// with taps outermost, 32 output channels per k-block.  Map dims
// (32, KH*KW, Cout, Cin/32), box (32, 1, 32, ROWS/32).
struct SrcFilterMN {
  static constexpr bool kMN = true;
  int cblocks, KHW;
  struct Cur {
    int tf, co0, cg;
  };
  template <int ROWS>
  __device__ __forceinline__ Cur begin(int, int64_t r0, int64_t k0) const {
    const int kb = (int)(k0 >> 5), tf = kb / cblocks;
    return {tf, (kb - tf * cblocks) * 32, (int)(r0 >> 5)};
  }
  __device__ __forceinline__ void issue(const CUtensorMap* map, uint32_t dst, uint64_t* bar, const Cur& c) const {
    load4(dst, map, 0, KHW - 1 - c.tf, c.co0, c.cg, bar);
  }
  __device__ __forceinline__ void next(Cur& c) const {
    c.co0 += 32;
    if (c.co0 == cblocks * 32) {
      c.co0 = 0;
      ++c.tf;
    }
  }
};

// TMEM columns: the accumulator at [0, BN); stage s of A at A_TMEM0 + 64 s
// (hi: +0..31, lo: +32..63).  Tiles of N <= 64 with 3 stages run two CTAs per
// SM (97 KB of shared memory and 256 TMEM columns each: the accumulator at
// [0, 64), A stages at 64, 128, 192), so one CTA's epilogue and prologue overlap
// the other's main loop; so do 128-wide tiles with 2 stages (97 KB, the
// accumulator at [0, 128), A stages at 128 and 192); otherwise a CTA holds the
// SM (120 KB floor, all 512 columns: the accumulator in [0, 256), 4 A stages
// from 256).
template <int BN, int STAGES>
struct Smem {
  static constexpr bool TWO = (STAGES <= 3 && BN <= 64) || (STAGES == 2 && BN == 128);
  static constexpr uint32_t A_BYTES = BM * BK * 4;  // raw A (TMA); its hi/lo go to TMEM
  static constexpr uint32_t B_BYTES = BN * BK * 4;
  static constexpr uint32_t STAGE = A_BYTES + 2 * B_BYTES;  // raw A | B raw -> hi | B lo
  static constexpr uint32_t TILES = STAGES * STAGE;
  static constexpr uint32_t BYTES = TWO || TILES + 1280 > 122880u ? TILES + 1280 : 122880u;
  static constexpr uint32_t TMEM_COLS = TWO ? 256 : 512;
  static constexpr uint32_t A_TMEM0 = TWO ? (BN > 64 ? BN : 64) : 256;
  static constexpr int MIN_BLOCKS = TWO ? 2 : 1;
  static_assert(STAGE % 1024 == 0, "stages must keep 1 KB swizzle alignment");
  static_assert(STAGES <= 4 && BN <= 256, "TMEM holds the accumulator (256 columns) and 4 A stages");
  static_assert(A_TMEM0 + 64 * STAGES <= TMEM_COLS && BN <= (int)A_TMEM0, "TMEM regions overlap");
  static_assert(128u * (BN + 4) * 4 <= TILES, "the staged epilogue tile must fit in the operand ring");
};

__device__ __forceinline__ void mma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

// 32 lanes x 16 consecutive 32-bit TMEM columns from registers.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Values k = k0..k0+15 of tile row r of a raw A tile: K-major 128-byte swizzle
// (row r: 8 chunks of 16 B at chunk ^ (r & 7)) or MN-major 32-byte-atom
// swizzle (32-row groups 4 KB apart, one 128-byte row per k, 32-byte chunk
// ^ (k & 3)).
template <bool MN>
__device__ __forceinline__ void read_a16(const uint8_t* tile, int r, int k0, float (&v)[16]) {
  if constexpr (!MN) {
    const uint8_t* row = tile + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int chunk = (k0 >> 2) + c;
      float4 q = *reinterpret_cast<const float4*>(row + ((chunk ^ (r & 7)) << 4));
      v[4 * c] = q.x;
      v[4 * c + 1] = q.y;
      v[4 * c + 2] = q.z;
      v[4 * c + 3] = q.w;
    }
  } else {
    const uint8_t* grp = tile + (r >> 5) * 4096;
    const int rr = r & 31;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int k = k0 + i;
      v[i] = *reinterpret_cast<const float*>(grp + k * 128 + ((((rr >> 3) ^ (k & 3)) << 5) | ((rr & 7) << 2)));
    }
  }
}

// Epilogue through shared memory for warp (quadrant q, column half h) of a
// 128 x BN accumulator at TMEM column 0: tcgen05.ld 16 columns at a time into
// the warp's 32 staged rows (pitch BN + 4 floats: the float4 stores of 8 lanes
// hit distinct banks), then each pass stores RPI whole row segments of HALF
// columns with float4 per lane -- split-K partials into ws[b][split], else
// through ep.row4.  Only this warp's rows and columns are touched, so a
// __syncwarp orders the two phases.
template <int BN, class EP>
__device__ __forceinline__ void staged_rows(float* stage, int q, int h, int lane, uint32_t tmem, bool have,
                                            int64_t m0, int64_t n0, int64_t M, int64_t N, int b, int split,
                                            int splits, float* __restrict__ ws, const EP& ep) {
  constexpr int HALF = BN / 2, PITCH = BN + 4, LPR = HALF / 4, RPI = 32 / LPR;
  static_assert(HALF % 16 == 0 && 32 % LPR == 0, "column half must be 16..128 columns");
  float* st = stage + (size_t)(q * 32) * PITCH;
#pragma unroll 1
  for (int c0 = h * HALF; c0 < (h + 1) * HALF; c0 += 16) {
    float v[16];
    if (have) {
      tc::tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = 0.0f;
    }
    float4* d = reinterpret_cast<float4*>(st + lane * PITCH + c0);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
  __syncwarp();
  const int cl = h * HALF + (lane % LPR) * 4;
  if (n0 + cl >= N) return;
#pragma unroll 4
  for (int rr = lane / LPR; rr < 32; rr += RPI) {
    const int64_t mm = m0 + q * 32 + rr;
    if (mm >= M) break;
    const float4 v4 = *reinterpret_cast<const float4*>(st + rr * PITCH + cl);
    if (splits > 1) {
      float* w = ws + (((int64_t)b * splits + split) * M + mm) * N + n0 + cl;
      if (n0 + cl + 4 <= N && ((uintptr_t)w & 15) == 0) {
        *reinterpret_cast<float4*>(w) = v4;
      } else {
        const float o[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (n0 + cl + i < N) w[i] = o[i];
      }
    } else if constexpr (HasRow4<EP>::value) {
      ep.row4(b, mm, n0 + cl, N, v4);
    }
  }
}

template <class SA, class SB, class EP, int BN, int STAGES>
__global__ void __launch_bounds__(NTHREADS, (Smem<BN, STAGES>::MIN_BLOCKS))
    k_gemm_tma(const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mb,
               const __grid_constant__ CUtensorMap mbl, SA sa, SB sb, EP ep, int64_t M, int64_t N, int64_t K,
               int64_t k_per_split, int splits, float* __restrict__ ws, int b_lo) {
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  // 1 KB aligned; derived from smem_raw by an offset so accesses stay shared-space loads/stores
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
  const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;
  // z = split * batch + b: the batches (filter taps) of one k range run side by side and share L2
  const int batch = (int)(gridDim.z / splits);
  const int b = (int)(blockIdx.z % batch), split = (int)(blockIdx.z / batch);
  const int64_t kb0 = (int64_t)split * k_per_split;
  const int64_t kend = kb0 + k_per_split < K ? kb0 + k_per_split : K;
  const int nk = kend > kb0 ? (int)((kend - kb0 + BK - 1) / BK) : 0;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&ready[s], NSPLIT);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(done, 1);
    tc::fence_barrier_init();
  }
  // the predecessor kernel has finished before this CTA allocates tensor memory
  // or touches global memory; dependents may launch once all CTAs hold theirs
  ::tp::pdl_wait();
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     tc::smem_u32(tmem_slot)),
                 "r"(S::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc::tc_fence_before();
  __syncthreads();
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
      auto cb = sb.template begin<BN>(b, n0, kb0);
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % STAGES;
        ok = tc::mbar_wait(&empty[s], (uint32_t)((kb / STAGES) & 1) ^ 1u, 11);
        if (!ok) break;
        const uint32_t st = tc::smem_u32(smem + s * S::STAGE);
        expect_tx(&full[s], S::A_BYTES + (b_lo ? 2u : 1u) * S::B_BYTES);
        sa.issue(&ma, st, &full[s], ca);
        sb.issue(&mb, st + S::A_BYTES, &full[s], cb);
        if (b_lo) sb.issue(&mbl, st + S::A_BYTES + S::B_BYTES, &full[s], cb);
        sa.next(ca);
        sb.next(cb);
        last[s] = kb;
      }
      // no box may still be landing when the CTA exits
#pragma unroll
      for (int s = 0; s < STAGES; ++s)
        if (last[s] >= 0) tc::mbar_wait(&full[s], (uint32_t)((last[s] / STAGES) & 1), 12);
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_tf32<BN>() | ((uint32_t)SB::kMN << 16);
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % STAGES;
        ok = tc::mbar_wait(&ready[s], (uint32_t)((kb / STAGES) & 1), 13);
        if (!ok) break;
        tc::tc_fence_after();
        const uint32_t base = tc::smem_u32(smem + s * S::STAGE);
        const uint32_t b_hi = base + S::A_BYTES, b_lo = base + S::A_BYTES + S::B_BYTES;
        const uint32_t a_hi = tmem + S::A_TMEM0 + 64 * s, a_lo = a_hi + 32;
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          // k-step of 8: 8 TMEM columns of A; +32 B inside a K-major B row, +1 KB (8 rows) when MN-major
          const uint32_t db = SB::kMN ? kk * 1024 : kk * 32;
          const uint64_t bh = SB::kMN ? mn_desc(b_hi + db) : tc::sw128_desc(b_hi + db);
          const uint64_t bl = SB::kMN ? mn_desc(b_lo + db) : tc::sw128_desc(b_lo + db);
          mma_tf32_ts(tmem, a_hi + 8 * kk, bh, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_tf32_ts(tmem, a_hi + 8 * kk, bl, idesc, 1u);
          mma_tf32_ts(tmem, a_lo + 8 * kk, bh, idesc, 1u);
        }
        tc::mma_commit(&empty[s]);
      }
      tc::mma_commit(done);
    }
  } else {
    // ---- splitters: A row r = 32*(warp%4) + lane, k half warp/4 -> TMEM hi/lo;
    //      B lo beside the raw B tile ----
    const int r = 32 * (warp & 3) + lane, kh = (warp >> 2) * 16;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int s = kb % STAGES;
      ok = tc::mbar_wait(&full[s], (uint32_t)((kb / STAGES) & 1), 14);
      if (!ok) break;
      uint8_t* st = smem + s * S::STAGE;
      {
        float v[16];
        uint32_t h[16], l[16];
        read_a16<SA::kMN>(st, r, kh, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float hf, lf;
          tc::split_tf32(v[i], hf, lf);
          h[i] = __float_as_uint(hf);
          l[i] = __float_as_uint(lf);
        }
        const uint32_t col = tmem + lane_base + S::A_TMEM0 + 64 * s + kh;
        tmem_st16(col, h);
        tmem_st16(col + 32, l);
      }
      // B: the raw tile is its own hi (the tensor core truncates fp32 to tf32); only lo is
      // written, unless the lo tile came from memory with the raw one (b_lo)
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
      tc::mbar_arrive(&ready[s]);
    }
  }
  __syncwarp();

  // ---- epilogue: warps 0-7; TMEM lane quadrant warp%4 = tile rows, column half warp/4 ----
  if (warp < 8) {
    bool fin = nk > 0 && tc::mbar_wait(done, 0, 15);
    bool have = __all_sync(0xffffffffu, ok && fin);
    tc::tc_fence_after();
    const int q = warp & 3, h = warp >> 2;
    const int64_t m = m0 + q * 32 + lane;
    constexpr int HALF = BN / 2;
    if (HasRow4<EP>::value || splits > 1) {
      // through shared memory (the operand ring is idle once `done` completed): the
      // warp stages its 32 rows x HALF columns, then stores them a row at a time
      if (have || nk == 0)
        staged_rows<BN>(reinterpret_cast<float*>(smem), q, h, lane, tmem, have, m0, n0, M, N, b, split, splits, ws,
                        ep);
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
            if (n0 + c0 + i < N) w[n0 + c0 + i] = v[i];
        } else {
          ep.row16(b, m, n0 + c0, N, v);
        }
      }
    }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::TMEM_COLS));
  }
}

}  // namespace tma

// mbl (optional): a map of B's tf32 low parts (tf32_lo_plane), with mb's
// geometry; the kernel then loads them instead of computing them per tile.
template <class SA, class SB, class EP, int BN, int STAGES>
void gemm_tma_launch(const CUtensorMap& ma, const CUtensorMap& mb, const SA& sa, const SB& sb, const EP& ep,
                     int64_t M, int64_t N, int64_t K, int batch, const CUtensorMap* mbl = nullptr) {
  using S = tma::Smem<BN, STAGES>;
  int64_t gm = (M + tma::BM - 1) / tma::BM, gn = (N + BN - 1) / BN;
  TP_REQUIRE(gn <= 65535 && gm <= 0x7fffffff, "gemm: tile grid exceeds the launch limits");
  auto kfn = tma::k_gemm_tma<SA, SB, EP, BN, STAGES>;
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
  TP_LAUNCH(kfn, dim3((unsigned)gm, (unsigned)gn, (unsigned)(batch * splits)), tma::NTHREADS, S::BYTES, ma, mb,
            mbl ? *mbl : mb, sa, sb, ep, M, N, K, kps, splits, ws, mbl ? 1 : 0);
  if (splits > 1) {
    auto rfn = tc::k_splitk_reduce_b<EP>;
    unsigned gx = (unsigned)((M * N / 4 + 255) / 256 + 1);
    if (gx > (unsigned)sm_count() * 8) gx = (unsigned)sm_count() * 8;
    TP_LAUNCH(rfn, dim3(gx, (unsigned)batch), 256, 0, ws, splits, M, N, ep);
  }
}

}  // namespace tp
