// Channels-last ([N][H][W][C]) stride-1 convolution: forward, data gradient
// and per-tap weight gradient on the TMA-fed tensor-core kernel.
//
// The reference's conv shaders work on NCHW (conv.wgsl:25-60,
// conv_backward.wgsl:24-101) and the per-op C ABI keeps that layout
// (tp_conv.cu).  A training step that owns its activations (tpcuda.vgg) keeps
// them channels-last instead: every im2col tile of 128 output pixels x 32
// channels of one tap is then one TMA box whose origin carries the tap shift
// and whose zero fill is the padding, and the weight gradient reads dy and
// the shifted x as MN-major boxes.  Filters and filter gradients stay in the
// reference layout [Cout][Cin][KH][KW]; filters are repacked per call.
//
// A 4-channel input (an RGB first layer padded to 4) runs on the CUDA-core
// kernels of tp_conv_small.cu.  Other shapes the TMA tiling cannot express
// (channels not a multiple of 32, pixel grids that 128 / 32 pixel boxes do
// not tile) run on gather loaders over the same layout.
#include <cuda_runtime.h>

#include "tp_core.h"
#include "tp_fastdiv.cuh"
#include "tp_gemm_dispatch.cuh"
#include "tp_launch.h"

namespace tp {

// ---- gather loaders over channels-last tensors (fallback) ---------------------------------

// Forward im2col: m = (n, oh, ow), k = (kh, kw, c) -> x[n, oh+kh-PH, ow+kw-PW, c].
struct LdNhwcIm2col {
  const float* x;
  int64_t H, W, C, OH, OW;
  int KW, PH, PW;
  static constexpr bool kContigK = true;
  __device__ __forceinline__ float load(int64_t m, int c, int kh, int kw) const {
    int64_t ow = m % OW, t = m / OW, oh = t % OH, n = t / OH;
    int64_t ih = oh + kh - PH, iw = ow + kw - PW;
    if (ih < 0 || ih >= H || iw < 0 || iw >= W) return 0.0f;
    return x[((n * H + ih) * W + iw) * C + c];
  }
  __device__ __forceinline__ float operator()(int, int64_t m, int64_t k) const {
    int c = (int)(k % C), tap = (int)(k / C);
    return load(m, c, tap / KW, tap % KW);
  }
  struct Kc {
    int c, kh, kw;
    bool ok;
  };
  __device__ __forceinline__ Kc kctx(int, int64_t k, int64_t kend) const {
    Kc r;
    r.ok = k < kend;
    int64_t kk = r.ok ? k : 0;
    r.c = (int)(kk % C);
    int tap = (int)(kk / C);
    r.kh = tap / KW;
    r.kw = tap % KW;
    return r;
  }
  __device__ __forceinline__ float at(int, int64_t m, const Kc& c) const {
    return c.ok && m < rows ? load(m, c.c, c.kh, c.kw) : 0.0f;
  }
  int64_t rows;  // N * OH * OW
};

// Weight gradient B operand: row r = (ci, kh, kw) (reference filter order) or
// (kh, kw, ci), k = output pixel (n, oh, ow) -> x[n, oh+kh-PH, ow+kw-PW, ci].
struct LdNhwcWgradB {
  const float* x;
  int64_t H, W, C, OH, OW, P;
  int KH, KW, PH, PW;
  int khwc;  // rows r = (kh, kw, ci) (filters stored [Cout][KH][KW][Cin]) instead of (ci, kh, kw)
  static constexpr bool kContigK = true;
  struct Kc {
    int64_t n;
    int oh, ow;
    bool ok;
  };
  __device__ __forceinline__ Kc kctx(int, int64_t k, int64_t kend) const {
    Kc r;
    r.ok = k < kend && k < P;
    int64_t kk = r.ok ? k : 0;
    r.ow = (int)(kk % OW);
    int64_t t = kk / OW;
    r.oh = (int)(t % OH);
    r.n = t / OH;
    return r;
  }
  __device__ __forceinline__ float at(int, int64_t r, const Kc& c) const {
    if (!c.ok || r >= C * KH * KW) return 0.0f;
    int kw, kh;
    int64_t ci;
    if (khwc) {
      ci = r % C;
      const int tap = (int)(r / C);
      kh = tap / KW;
      kw = tap - kh * KW;
    } else {
      kw = (int)(r % KW);
      int64_t t = r / KW;
      kh = (int)(t % KH);
      ci = t / KH;
    }
    int64_t ih = c.oh + kh - PH, iw = c.ow + kw - PW;
    if (ih < 0 || ih >= H || iw < 0 || iw >= W) return 0.0f;
    return x[((c.n * H + ih) * W + iw) * C + ci];
  }
  __device__ __forceinline__ float operator()(int b, int64_t r, int64_t k) const { return at(b, r, kctx(b, k, P)); }
};

// ---- TMA maps over channels-last tensors ---------------------------------------------------

// Pixel tiles of `rows` output pixels over an N x OH x OW grid, with the
// number of GEMM rows (or k) they span.  Whole rows of the grid when OW
// divides `rows` and `rows` divides OH*OW (or whole images when OH*OW
// divides `rows`): then tile order is plain pixel order and no row is padding.
// Otherwise TW x TH rectangles (TW a power of two) with the least padding.
struct Tiling {
  tma::PixTile pt;
  int64_t span;   // tiles x rows
  bool linear;    // tile order == pixel order, span == N*OH*OW rounded up to `rows`
};

static bool pixel_tiling(int64_t N, int64_t OH, int64_t OW, int rows, Tiling& t) {
  if (OH <= 0 || OW <= 0 || N <= 0) return false;
  const int64_t hw = OH * OW;
  tma::PixTile& p = t.pt;
  p.OH = (int)OH;
  p.OW = (int)OW;
  if (OW <= rows && rows % OW == 0 && hw >= rows && hw % rows == 0 && rows / OW <= 256) {
    p.TW = (int)OW, p.TH = (int)(rows / OW), p.TN = 1, p.tiles_w = 1, p.tiles_h = (int)(OH / p.TH);
    t.span = N * hw;
    t.linear = true;
    return true;
  }
  if (hw < rows && rows % hw == 0 && OW <= 256 && OH <= 256) {
    p.TW = (int)OW, p.TH = (int)OH, p.TN = (int)(rows / hw), p.tiles_w = 1, p.tiles_h = 1;
    t.span = (N + p.TN - 1) / p.TN * rows;
    t.linear = true;
    return true;
  }
  int64_t best = -1;
  for (int tw = 4; tw <= rows && tw <= 256; tw *= 2) {
    const int th = rows / tw;
    if (th < 1 || th > 256 || tw * th != rows) continue;
    const int64_t cw = (OW + tw - 1) / tw, ch = (OH + th - 1) / th;
    const int64_t area = cw * ch * rows;
    if (best < 0 || area < best) {
      best = area;
      p.TW = tw, p.TH = th, p.TN = 1, p.tiles_w = (int)cw, p.tiles_h = (int)ch;
    }
  }
  if (best < 0) return false;
  t.span = N * best;
  t.linear = false;
  return t.span < ((int64_t)1 << 31);
}

// Row-major [pixel][C] output through pixel tiles: GEMM row m -> pixel, rows
// outside the grid are skipped.
struct EpPixTile {
  float* c;
  int64_t ldc, N;
  const float* bias;
  tma::PixTile pt;
  __device__ __forceinline__ bool at(int64_t m, int64_t& row) const {
    int n, oh, ow;
    if (!pt.pixel(m, 128, N, n, oh, ow)) return false;
    row = ((int64_t)n * pt.OH + oh) * pt.OW + ow;
    return true;
  }
  __device__ __forceinline__ void operator()(int, int64_t m, int64_t n, float v) const {
    int64_t row;
    if (!at(m, row)) return;
    c[row * ldc + n] = bias ? v + bias[n] : v;
  }
  __device__ __forceinline__ void row16(int b, int64_t m, int64_t n0, int64_t Nn, const float (&v)[16]) const {
    int64_t row;
    if (!at(m, row)) return;
    EpRowMajor{c, ldc, 0, bias, 0}.row16(b, row, n0, Nn, v);
  }
  __device__ __forceinline__ void row4(int b, int64_t m, int64_t n0, int64_t Nn, float4 v) const {
    int64_t row;
    if (!at(m, row)) return;
    EpRowMajor{c, ldc, 0, bias, 0}.row4(b, row, n0, Nn, v);
  }
};

// NCHW output [N][C][HW] of a channels-last GEMM (row m = pixel, linear or
// through pixel tiles): writes the per-op NCHW tensor directly, so no
// channels-last copy is transposed back.  For a fixed column a warp's lanes
// hold consecutive pixels, so each store instruction covers a contiguous run.
struct EpNchwOut {
  float* y;
  const float* bias;
  int64_t C, HW, N;
  tma::PixTile pt;
  int linear;
  __device__ __forceinline__ bool pix(int64_t m, int64_t& img, int64_t& p) const {
    if (linear) {
      img = m / HW;
      p = m - img * HW;
      return img < N;
    }
    int n, oh, ow;
    if (!pt.pixel(m, 128, N, n, oh, ow)) return false;
    img = n;
    p = (int64_t)oh * pt.OW + ow;
    return true;
  }
  __device__ __forceinline__ void operator()(int, int64_t m, int64_t c, float v) const {
    int64_t img, p;
    if (pix(m, img, p)) y[(img * C + c) * HW + p] = bias ? v + bias[c] : v;
  }
  __device__ __forceinline__ void row16(int, int64_t m, int64_t n0, int64_t Nn, const float (&v)[16]) const {
    int64_t img, p;
    if (!pix(m, img, p)) return;
    float* dst = y + (img * C + n0) * HW + p;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (n0 + i < Nn) dst[(int64_t)i * HW] = bias ? v[i] + bias[n0 + i] : v[i];
  }
};

// K-major (im2col) map: dims (C, W, H, N), box (32, TW, TH, TN).
static bool nhwc_map(CUtensorMap* m, const float* t, int64_t N, int64_t H, int64_t W, int64_t C,
                     const tma::PixTile& pt, bool make) {
  uint64_t dims[4] = {(uint64_t)C, (uint64_t)W, (uint64_t)H, (uint64_t)N};
  uint64_t st[3] = {(uint64_t)C * 4, (uint64_t)(W * C) * 4, (uint64_t)(H * W * C) * 4};
  if (!tma_aligned(t, st, 3)) return false;
  if (N > 0x7fffffff || H * W > 0x7fffffff) return false;
  if (make) {
    uint32_t box[4] = {32, (uint32_t)pt.TW, (uint32_t)pt.TH, (uint32_t)pt.TN};
    make_map_f32(m, t, 4, dims, st, box, false);
  }
  return true;
}

// MN-major map for the weight gradient: dims (32, W, H, N, C/32) with the
// 32-channel groups outermost (stride 128 B), box (32, pixel box, rows/32);
// C % 32 == 0.
static bool nhwc_mn_map(CUtensorMap* m, const float* t, int64_t N, int64_t H, int64_t W, int64_t C,
                        const tma::PixTile& pt, uint32_t rows, bool make) {
  if (C % 32) return false;
  uint64_t dims[5] = {32, (uint64_t)W, (uint64_t)H, (uint64_t)N, (uint64_t)(C / 32)};
  uint64_t st[4] = {(uint64_t)C * 4, (uint64_t)(W * C) * 4, (uint64_t)(H * W * C) * 4, 128};
  if (!tma_aligned(t, st, 4)) return false;
  if (N > 0x7fffffff || H * W > 0x7fffffff) return false;
  if (make) {
    uint32_t box[5] = {32, (uint32_t)pt.TW, (uint32_t)pt.TH, (uint32_t)pt.TN, rows / 32};
    make_map_f32(m, t, 5, dims, st, box, true);
  }
  return true;
}

static bool nhwc_tma_ok() { return tma_enabled(); }

// ---- launchers -------------------------------------------------------------------------------

struct NhwcShape {
  int64_t N, Cin, H, W, Cout, OH, OW;
  int KH, KW, PH, PW;
  bool khwc;  // filters stored [Cout][KH][KW][Cin] (else the reference's [Cout][Cin][KH][KW])
  int DW = 1;  // tap spacing along W (the TMA paths only; the paired space-to-depth stem uses 2)
};

static NhwcShape nhwc_shape(int64_t N, int64_t Cin, int64_t H, int64_t W, int64_t Cout, int KH, int KW, int PH,
                            int PW, int filter_layout) {
  TP_REQUIRE(N >= 0 && Cin > 0 && H > 0 && W > 0 && Cout > 0, "conv2d (channels-last): bad shape");
  TP_REQUIRE(KH > 0 && KW > 0 && PH >= 0 && PW >= 0, "conv2d (channels-last): bad kernel or padding");
  TP_REQUIRE(filter_layout == 0 || filter_layout == 1,
             "conv2d (channels-last): filter layout must be 0 ([Cout][Cin][KH][KW]) or 1 ([Cout][KH][KW][Cin])");
  NhwcShape s{N,  Cin, H,  W,  Cout, H + 2 * PH - KH + 1, W + 2 * PW - KW + 1, KH, KW,
              PH, PW,  filter_layout == 1};
  TP_REQUIRE(s.OH > 0 && s.OW > 0, "conv2d (channels-last): output would be empty");
  return s;
}

__global__ void k_pack_filters(const float* __restrict__ w, float* __restrict__ wp, int64_t Cout, int64_t Cin_pg,
                               int khw, int mode);

// tp_conv_small.cu: 4-channel first-layer kernels on the CUDA cores
bool conv_c4_ok(int64_t N, int64_t H, int64_t W, int64_t Cin, int KH, int KW, int64_t Cout, const void* a,
                const void* b);
void conv_c4_fwd(const float* x, const float* w, const float* bias, float* y, int64_t N, int64_t H, int64_t W,
                 int64_t Cout, int PH, int PW);
void conv_c4_wgrad(const float* dy, const float* x, float* dw, int64_t N, int64_t H, int64_t W, int64_t Cout, int PH,
                   int PW);

// y[N][OH][OW][Cout] = conv(x[N][H][W][Cin], w) + bias
// w_lo (optional): the tf32 low parts of w (tf32_lo_plane), kept by the caller
// beside w; used when the filters are read in place (filter layout 1).
// y_nchw (optional): when the TMA path runs, the output goes straight to this
// NCHW tensor instead of y (returns true); otherwise y gets it (false).
static bool conv_fwd_nhwc(const NhwcShape& s, const float* x, const float* w, const float* bias, float* y,
                          const float* w_lo = nullptr, float* y_nchw = nullptr) {
  const int khw = s.KH * s.KW;
  const int64_t M = s.N * s.OH * s.OW, K = s.Cin * khw;
  if (M == 0) return false;
  if (!s.khwc && conv_c4_ok(s.N, s.H, s.W, s.Cin, s.KH, s.KW, s.Cout, x, y) &&
      (bias == nullptr || ((uintptr_t)bias & 15) == 0)) {
    conv_c4_fwd(x, w, bias, y, s.N, s.H, s.W, s.Cout, s.PH, s.PW);
    return false;
  }
  // K order (kh, kw, c): filters stored that way are used as they are
  const float* wp = w;
  if (!s.khwc) {
    float* t = (float*)scratch2((size_t)s.Cout * K * sizeof(float));
    TP_LAUNCH(k_pack_filters, grid_for(s.Cout * K, 256), 256, 0, w, t, s.Cout, s.Cin, khw, 0);
    wp = t;
  }
  EpRowMajor ep{y, s.Cout, 0, bias, 0};
  Tiling tl;
  MatOp b{wp, false, K, 0, false};
  if (nhwc_tma_ok() && M >= 64 && s.Cin % 32 == 0 && pixel_tiling(s.N, s.OH, s.OW, tc::BM, tl) &&
      nhwc_map(nullptr, x, s.N, s.H, s.W, s.Cin, tl.pt, false) && mat_tma_ok(b, s.Cout)) {
    CUtensorMap ma, mb, mbl;
    const uint32_t brows = tma_b_rows(tl.linear ? M : tl.span, s.Cout, K, 1);
    nhwc_map(&ma, x, s.N, s.H, s.W, s.Cin, tl.pt, true);
    mat_map(&mb, b, s.Cout, K, 1, brows);
    // every pixel tile reads all filters: their tf32 low parts are split once
    const float* wlo = (w_lo && wp == w) ? w_lo : nullptr;
    if (!wlo) {
      float* t = (float*)scratch3((size_t)s.Cout * K * sizeof(float));
      tf32_lo_plane(wp, t, s.Cout * K);
      wlo = t;
    }
    mat_map(&mbl, MatOp{wlo, false, K, 0, false}, s.Cout, K, 1, brows);
    tma::SrcConvK sa{tl.pt, (int)(s.Cin / 32), s.KW, s.PH, s.PW, s.DW};
    if (y_nchw) {
      EpNchwOut eo{y_nchw, bias, s.Cout, s.OH * s.OW, s.N, tl.pt, tl.linear ? 1 : 0};
      gemm_tma_bn(ma, mb, sa, tma::SrcK{0}, eo, tl.linear ? M : tl.span, s.Cout, K, 1, &mbl);
      return true;
    }
    if (tl.linear) gemm_tma_bn(ma, mb, sa, tma::SrcK{0}, ep, M, s.Cout, K, 1, &mbl);
    else gemm_tma_bn(ma, mb, sa, tma::SrcK{0}, EpPixTile{y, s.Cout, s.N, bias, tl.pt}, tl.span, s.Cout, K, 1, &mbl);
    return false;
  }
  TP_REQUIRE(s.DW == 1, "conv2d (channels-last): spaced taps need the TMA path");
  LdNhwcIm2col la{x, s.H, s.W, s.Cin, s.OH, s.OW, s.KW, s.PH, s.PW, M};
  gemm_auto(la, LdRowMajor{wp, K, 0}, ep, M, s.Cout, K, 1);
  return false;
}

// dx[N][H][W][Cin] from dy[N][OH][OW][Cout]: the forward convolution of dy
// with the flipped, transposed filters and padding K-1-P.
static bool conv_dgrad_nhwc(const NhwcShape& s, const float* dy, const float* w, float* dx,
                            const float* w_lo = nullptr, float* dx_nchw = nullptr) {
  const int khw = s.KH * s.KW;
  const int64_t M = s.N * s.H * s.W, K = s.Cout * khw;
  if (M == 0) return false;
  TP_REQUIRE(s.PH <= s.KH - 1 && s.PW <= (s.KW - 1) * s.DW,
             "conv2d data gradient (channels-last): padding exceeds the kernel's extent - 1");
  EpRowMajor ep{dx, s.Cin, 0, nullptr, 0};
  const int qh = s.KH - 1 - s.PH, qw = (s.KW - 1) * s.DW - s.PW;
  Tiling tl;
  const bool tma_a = nhwc_tma_ok() && M >= 64 && s.Cout % 32 == 0 && pixel_tiling(s.N, s.H, s.W, tc::BM, tl) &&
                     nhwc_map(nullptr, dy, s.N, s.OH, s.OW, s.Cout, tl.pt, false);
  if (tma_a && s.khwc && s.Cin % 32 == 0 && ((uintptr_t)w & 15) == 0) {
    // filters stored [Cout][tap][Cin] are read in place as the MN-major B
    CUtensorMap ma, mb, mbl;
    nhwc_map(&ma, dy, s.N, s.OH, s.OW, s.Cout, tl.pt, true);
    uint64_t dims[4] = {32, (uint64_t)khw, (uint64_t)s.Cout, (uint64_t)(s.Cin / 32)};
    uint64_t st[3] = {(uint64_t)s.Cin * 4, (uint64_t)(khw * s.Cin) * 4, 128};
    uint32_t box[4] = {32, 1, 32, tma_b_rows(tl.linear ? M : tl.span, s.Cin, K, 1) / 32};
    make_map_f32(&mb, w, 4, dims, st, box, true);
    const float* wlo = w_lo;
    if (!wlo) {
      float* t = (float*)scratch3((size_t)s.Cin * K * sizeof(float));
      tf32_lo_plane(w, t, s.Cin * K);
      wlo = t;
    }
    TP_REQUIRE(((uintptr_t)wlo & 15) == 0, "conv2d data gradient (channels-last): w_lo must be 16-byte aligned");
    make_map_f32(&mbl, wlo, 4, dims, st, box, true);
    tma::SrcConvK sa{tl.pt, (int)(s.Cout / 32), s.KW, qh, qw, s.DW};
    tma::SrcFilterMN sb{(int)(s.Cout / 32), khw};
    if (dx_nchw) {
      EpNchwOut eo{dx_nchw, nullptr, s.Cin, s.H * s.W, s.N, tl.pt, tl.linear ? 1 : 0};
      gemm_tma_bn(ma, mb, sa, sb, eo, tl.linear ? M : tl.span, s.Cin, K, 1, &mbl);
      return true;
    }
    if (tl.linear) gemm_tma_bn(ma, mb, sa, sb, ep, M, s.Cin, K, 1, &mbl);
    else gemm_tma_bn(ma, mb, sa, sb, EpPixTile{dx, s.Cin, s.N, nullptr, tl.pt}, tl.span, s.Cin, K, 1, &mbl);
    return false;
  }
  float* wp = (float*)scratch2((size_t)s.Cin * K * sizeof(float));
  TP_LAUNCH(k_pack_filters, grid_for(s.Cout * s.Cin * khw, 256), 256, 0, w, wp, s.Cout, s.Cin, khw, s.khwc ? 2 : 1);
  MatOp b{wp, false, K, 0, false};
  if (tma_a && mat_tma_ok(b, s.Cin)) {
    CUtensorMap ma, mb, mbl;
    const uint32_t brows = tma_b_rows(tl.linear ? M : tl.span, s.Cin, K, 1);
    nhwc_map(&ma, dy, s.N, s.OH, s.OW, s.Cout, tl.pt, true);
    mat_map(&mb, b, s.Cin, K, 1, brows);
    float* wlo = (float*)scratch3((size_t)s.Cin * K * sizeof(float));
    tf32_lo_plane(wp, wlo, s.Cin * K);
    mat_map(&mbl, MatOp{wlo, false, K, 0, false}, s.Cin, K, 1, brows);
    tma::SrcConvK sa{tl.pt, (int)(s.Cout / 32), s.KW, qh, qw, s.DW};
    if (dx_nchw) {
      EpNchwOut eo{dx_nchw, nullptr, s.Cin, s.H * s.W, s.N, tl.pt, tl.linear ? 1 : 0};
      gemm_tma_bn(ma, mb, sa, tma::SrcK{0}, eo, tl.linear ? M : tl.span, s.Cin, K, 1, &mbl);
      return true;
    }
    if (tl.linear) gemm_tma_bn(ma, mb, sa, tma::SrcK{0}, ep, M, s.Cin, K, 1, &mbl);
    else gemm_tma_bn(ma, mb, sa, tma::SrcK{0}, EpPixTile{dx, s.Cin, s.N, nullptr, tl.pt}, tl.span, s.Cin, K, 1,
                     &mbl);
    return false;
  }
  TP_REQUIRE(s.DW == 1, "conv2d data gradient (channels-last): spaced taps need the TMA path");
  LdNhwcIm2col la{dy, s.OH, s.OW, s.Cout, s.H, s.W, s.KW, qh, qw, M};
  gemm_auto(la, LdRowMajor{wp, K, 0}, ep, M, s.Cin, K, 1);
  return false;
}

// dw[Cout][Cin][KH][KW] = sum over output pixels of dy x (x shifted by the tap)
static void conv_wgrad_nhwc(const NhwcShape& s, const float* dy, const float* x, float* dw) {
  const int khw = s.KH * s.KW;
  const int64_t P = s.N * s.OH * s.OW;
  if (!s.khwc && conv_c4_ok(s.N, s.H, s.W, s.Cin, s.KH, s.KW, s.Cout, x, dy)) {
    conv_c4_wgrad(dy, x, dw, s.N, s.H, s.W, s.Cout, s.PH, s.PW);
    return;
  }
  Tiling tl;
  if (nhwc_tma_ok() && s.Cout >= 64 && P > 0 && pixel_tiling(s.N, s.OH, s.OW, 32, tl) &&
      nhwc_mn_map(nullptr, dy, s.N, s.OH, s.OW, s.Cout, tl.pt, tc::BM, false) &&
      nhwc_mn_map(nullptr, x, s.N, s.H, s.W, s.Cin, tl.pt, 32, false)) {
    // 64 / 32 input channels: 2 / 4 taps per GEMM (N = 128), the dy tile shared by them
    if (s.khwc && (s.Cin == 64 || s.Cin == 32) && khw > 1) {
      CUtensorMap ma, mb;
      nhwc_mn_map(&ma, dy, s.N, s.OH, s.OW, s.Cout, tl.pt, tc::BM, true);
      nhwc_mn_map(&mb, x, s.N, s.H, s.W, s.Cin, tl.pt, (uint32_t)s.Cin, true);
      tma::SrcPixMN sa{tl.pt, s.KW, s.PH, s.PW, 0, s.DW};
      if (s.Cin == 64) {
        tma::SrcPixMNT<2> sb{tl.pt, s.KW, s.PH, s.PW, khw, s.DW};
        gemm_tma_launch<tma::SrcPixMN, tma::SrcPixMNT<2>, EpWgradTapsKhwc<2>, 128, 4>(
            ma, mb, sa, sb, EpWgradTapsKhwc<2>{dw, s.Cin, khw}, s.Cout, 128, tl.span, (khw + 1) / 2);
      } else {
        tma::SrcPixMNT<4> sb{tl.pt, s.KW, s.PH, s.PW, khw, s.DW};
        gemm_tma_launch<tma::SrcPixMN, tma::SrcPixMNT<4>, EpWgradTapsKhwc<4>, 128, 4>(
            ma, mb, sa, sb, EpWgradTapsKhwc<4>{dw, s.Cin, khw}, s.Cout, 128, tl.span, (khw + 3) / 4);
      }
      return;
    }
    const uint32_t bn = tma_b_rows(s.Cout, s.Cin, tl.span, khw);
    CUtensorMap ma, mb;
    nhwc_mn_map(&ma, dy, s.N, s.OH, s.OW, s.Cout, tl.pt, tc::BM, true);
    nhwc_mn_map(&mb, x, s.N, s.H, s.W, s.Cin, tl.pt, bn, true);
    tma::SrcPixMN sa{tl.pt, s.KW, s.PH, s.PW, 0, s.DW};
    tma::SrcPixMN sb{tl.pt, s.KW, s.PH, s.PW, 1, s.DW};
    if (s.khwc) gemm_tma_bn(ma, mb, sa, sb, EpWgradTapKhwc{dw, s.Cin, khw}, s.Cout, s.Cin, tl.span, khw);
    else gemm_tma_bn(ma, mb, sa, sb, EpWgradTap{dw, s.Cin, khw}, s.Cout, s.Cin, tl.span, khw);
    return;
  }
  TP_REQUIRE(s.DW == 1, "conv2d weight gradient (channels-last): spaced taps need the TMA path");
  const int64_t R = s.Cin * khw;
  EpRowMajor ep{dw, R, 0, nullptr, 0};
  if (P == 0) {
    launch_fill(dw, s.Cout * R, 0.0f);
    return;
  }
  LdNhwcWgradB lb{x, s.H, s.W, s.Cin, s.OH, s.OW, P, s.KH, s.KW, s.PH, s.PW, s.khwc ? 1 : 0};
  gemm_auto(LdColMajor{dy, s.Cout, 0}, lb, ep, s.Cout, R, P, 1);
}

// ---- NCHW convolutions through channels-last copies ----------------------------------------
// The per-op API's tensors are NCHW (the reference's layout).  For shapes the
// TMA-fed kernel takes, transposing the operands into channels-last scratch
// copies (one coalesced pass each way) and back costs far less than the
// gather kernel's per-element index work.

static bool via_ok(const ConvShape& s) {
  return tma_enabled() && s.SH == 1 && s.SW == 1 && s.icpg == s.Cin && s.KH <= 7 && s.KW <= 7 &&
         s.OH == s.H + 2 * s.PH - s.KH + 1 && s.OW == s.W + 2 * s.PW - s.KW + 1 && s.N * s.OH * s.OW >= 128;
}

static NhwcShape nhwc_of(const ConvShape& s) {
  return NhwcShape{s.N, s.Cin, s.H, s.W, s.Cout, s.OH, s.OW, s.KH, s.KW, s.PH, s.PW, false};
}

bool conv_fwd_via_nhwc(const ConvShape& s, const float* x, const float* w, const float* bias, float* y) {
  if (!via_ok(s) || s.Cin % 32 || s.Cout % 4 || (bias && ((uintptr_t)bias & 15))) return false;
  float* xn = (float*)dalloc((size_t)s.N * s.H * s.W * s.Cin * 4);
  float* yn = (float*)dalloc((size_t)s.N * s.OH * s.OW * s.Cout * 4);
  transpose_nchw_nhwc(x, xn, s.N, s.Cin, s.H * s.W, true);
  if (!conv_fwd_nhwc(nhwc_of(s), xn, w, bias, yn, nullptr, y)) transpose_nchw_nhwc(yn, y, s.N, s.Cout, s.OH * s.OW, false);
  dfree(xn);
  dfree(yn);
  return true;
}

bool conv_dgrad_via_nhwc(const ConvShape& s, const float* dy, const float* w, float* dx) {
  if (!via_ok(s) || s.Cout % 32 || s.Cin % 4 || s.PH > s.KH - 1 || s.PW > s.KW - 1) return false;
  float* dyn = (float*)dalloc((size_t)s.N * s.OH * s.OW * s.Cout * 4);
  float* dxn = (float*)dalloc((size_t)s.N * s.H * s.W * s.Cin * 4);
  transpose_nchw_nhwc(dy, dyn, s.N, s.Cout, s.OH * s.OW, true);
  if (!conv_dgrad_nhwc(nhwc_of(s), dyn, w, dxn, nullptr, dx)) transpose_nchw_nhwc(dxn, dx, s.N, s.Cin, s.H * s.W, false);
  dfree(dyn);
  dfree(dxn);
  return true;
}

bool conv_wgrad_via_nhwc(const ConvShape& s, const float* dy, const float* x, float* dw) {
  if (!via_ok(s) || s.Cout % 32 || s.Cin % 32 || s.Cout < 64) return false;
  float* dyn = (float*)dalloc((size_t)s.N * s.OH * s.OW * s.Cout * 4);
  float* xn = (float*)dalloc((size_t)s.N * s.H * s.W * s.Cin * 4);
  transpose_nchw_nhwc(dy, dyn, s.N, s.Cout, s.OH * s.OW, true);
  transpose_nchw_nhwc(x, xn, s.N, s.Cin, s.H * s.W, true);
  conv_wgrad_nhwc(nhwc_of(s), dyn, xn, dw);
  dfree(dyn);
  dfree(xn);
  return true;
}

// ---- stride-2 convolutions of few channels through space-to-depth ------------------------------
// A stride-2 KxK convolution of C <= 8 channels equals a stride-1 AxA
// convolution (A = ((K - 1 + (P & 1)) >> 1) + 1) over the space-to-depth image
// x'[n][Y][X][(dy*2 + dx)*C + ci] = x[n][ci][2Y + dy - O][2X + dx - O] (O = P
// rounded up to even, zeros outside), with filters w'[co][a][b][(dy*2+dx)*C+ci]
// = w[co][ci][2a + dy + P - O][2b + dx + P - O] (zero where that tap does not
// exist).  x' is padded to 32 channels, so all three passes run on the TMA
// tensor-core kernels (the 7x7 / 3-channel network stem: K = 16 taps x 32
// instead of 147 gathered values) and the results map back exactly.
struct S2d {
  int C, K, P, O, A;
  int64_t N, H, W, OH, OW, HY, WX;
};

static bool s2d_plan(const ConvShape& s, S2d& d) {
  if (!tma_enabled() || s.SH != 2 || s.SW != 2 || s.KH != s.KW || s.PH != s.PW || s.icpg != s.Cin) return false;
  if (s.Cin > 8 || s.KH > 8 || s.Cout % 4) return false;
  d.C = (int)s.Cin;
  d.K = s.KH;
  d.P = s.PH;
  d.O = s.PH + (s.PH & 1);
  d.A = ((s.KH - 1 + (s.PH & 1)) >> 1) + 1;
  d.N = s.N;
  d.H = s.H;
  d.W = s.W;
  d.OH = s.OH;
  d.OW = s.OW;
  d.HY = s.OH + d.A - 1;
  d.WX = s.OW + d.A - 1;
  return d.N * d.HY * d.WX >= 128 && d.N * d.HY * d.WX * 32 < ((int64_t)1 << 31);
}

// x (NCHW, C channels) -> x' [N][HY][WX][32]; one thread per x' pixel, 8 16-byte stores
template <int C>
__global__ void k_s2d_in(const float* __restrict__ x, float* __restrict__ xs, S2d d, FastDiv fwx, FastDiv fhy) {
  ::tp::pdl_enter();
  const uint32_t total = (uint32_t)(d.N * d.HY * d.WX);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t t = fwx.div(i), X = i - t * (uint32_t)d.WX;
    const uint32_t n = fhy.div(t), Y = t - n * (uint32_t)d.HY;
    float v[32];
#pragma unroll
    for (int q = 0; q < 32; ++q) v[q] = 0.0f;
#pragma unroll
    for (int ph = 0; ph < 4; ++ph) {
      const int64_t ih = 2 * (int64_t)Y + (ph >> 1) - d.O, iw = 2 * (int64_t)X + (ph & 1) - d.O;
      if (ih < 0 || ih >= d.H || iw < 0 || iw >= d.W) continue;
      const float* src = x + ((int64_t)n * C * d.H + ih) * d.W + iw;
#pragma unroll
      for (int ci = 0; ci < C; ++ci) v[ph * C + ci] = src[(int64_t)ci * d.H * d.W];
    }
    float4* dst = reinterpret_cast<float4*>(xs + (int64_t)i * 32);
#pragma unroll
    for (int k = 0; k < 8; ++k) dst[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
  }
}

static void s2d_in(const float* x, float* xs, const S2d& d) {
  const int g = grid_for(d.N * d.HY * d.WX, 256);
  const FastDiv fwx = fast_div((uint32_t)d.WX), fhy = fast_div((uint32_t)d.HY);
  switch (d.C) {
#define TP_S2D_IN(c) \
  case c: TP_LAUNCH(k_s2d_in<c>, g, 256, 0, x, xs, d, fwx, fhy); break;
    TP_S2D_IN(1) TP_S2D_IN(2) TP_S2D_IN(3) TP_S2D_IN(4) TP_S2D_IN(5) TP_S2D_IN(6) TP_S2D_IN(7) TP_S2D_IN(8)
#undef TP_S2D_IN
    default: TP_REQUIRE(false, "space-to-depth: 1 to 8 channels");
  }
}
// dx' [N][HY][WX][32] -> dx (NCHW): every input pixel has exactly one (Y, dy) / (X, dx)
__global__ void k_s2d_out(const float* __restrict__ dxs, float* __restrict__ dx, S2d d) {
  ::tp::pdl_enter();
  const int64_t total = d.N * d.C * d.H * d.W;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t iw = i % d.W;
    int64_t t = i / d.W;
    const int64_t ih = t % d.H;
    t /= d.H;
    const int ci = (int)(t % d.C);
    const int64_t n = t / d.C;
    const int64_t ry = ih + d.O, rx = iw + d.O;
    const int64_t Y = ry >> 1, X = rx >> 1;
    const int q = (int)(((ry & 1) * 2 + (rx & 1)) * d.C + ci);
    dx[i] = (Y < d.HY && X < d.WX) ? dxs[((n * d.HY + Y) * d.WX + X) * 32 + q] : 0.0f;
  }
}

// w [Cout][C][K][K] <-> w' [Cout][A][A][32]; to_s2d = 1 builds w' (zeros where no
// tap), 0 maps a w'-shaped gradient back onto w's taps.
__global__ void k_s2d_filters(const float* __restrict__ src, float* __restrict__ dst, int64_t Cout, S2d d,
                              int to_s2d) {
  ::tp::pdl_enter();
  const int64_t total = Cout * d.A * d.A * 32;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int q = (int)(i & 31);
    int64_t t = i >> 5;
    const int b = (int)(t % d.A);
    t /= d.A;
    const int a = (int)(t % d.A);
    const int64_t co = t / d.A;
    int kh = -1, kw = -1, ci = 0;
    if (q < 4 * d.C) {
      const int ph = q / d.C;
      ci = q - ph * d.C;
      kh = 2 * a + (ph >> 1) + d.P - d.O;
      kw = 2 * b + (ph & 1) + d.P - d.O;
    }
    const bool tap = kh >= 0 && kh < d.K && kw >= 0 && kw < d.K;
    const int64_t wi = ((co * d.C + ci) * d.K + kh) * d.K + kw;
    if (to_s2d) dst[i] = tap ? src[wi] : 0.0f;
    else if (tap) dst[wi] = src[i];
  }
}

// ---- paired space-to-depth (C <= 4): two x' pixels per 32-channel vector ---------------------
// x''[n][Y][X][q*4C + ph*C + ci] = x'[n][Y][X + q][ph*C + ci] (q = 0, 1; zeros past WX): the
// AxA convolution over x' becomes an A x ceil(A/2) one over x'' whose column taps are 2
// pixels apart (tap (a, p) reads x'' at (Y + a, X + 2p), i.e. x' at X + 2p + q), so a
// 32-wide k-block carries 8C real values instead of 4C and K halves (7x7 / 3-channel stem:
// 8 taps x 32 = 256 instead of 16 x 32 = 512 for 147 real products).
template <int C>
__global__ void k_s2d_pair_in(const float* __restrict__ x, float* __restrict__ xs, S2d d, FastDiv fwx,
                              FastDiv fhy) {
  ::tp::pdl_enter();
  const uint32_t total = (uint32_t)(d.N * d.HY * d.WX);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t t = fwx.div(i), X = i - t * (uint32_t)d.WX;
    const uint32_t n = fhy.div(t), Y = t - n * (uint32_t)d.HY;
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = 0.0f;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (X + q >= (uint32_t)d.WX) continue;
#pragma unroll
      for (int ph = 0; ph < 4; ++ph) {
        const int64_t ih = 2 * (int64_t)Y + (ph >> 1) - d.O, iw = 2 * (int64_t)(X + q) + (ph & 1) - d.O;
        if (ih < 0 || ih >= d.H || iw < 0 || iw >= d.W) continue;
        const float* src = x + ((int64_t)n * C * d.H + ih) * d.W + iw;
#pragma unroll
        for (int ci = 0; ci < C; ++ci) v[q * 4 * C + ph * C + ci] = src[(int64_t)ci * d.H * d.W];
      }
    }
    float4* dst = reinterpret_cast<float4*>(xs + (int64_t)i * 32);
#pragma unroll
    for (int k = 0; k < 8; ++k) dst[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
  }
}

static void s2d_pair_in(const float* x, float* xs, const S2d& d) {
  const int g = grid_for(d.N * d.HY * d.WX, 256);
  const FastDiv fwx = fast_div((uint32_t)d.WX), fhy = fast_div((uint32_t)d.HY);
  switch (d.C) {
    case 1: TP_LAUNCH(k_s2d_pair_in<1>, g, 256, 0, x, xs, d, fwx, fhy); break;
    case 2: TP_LAUNCH(k_s2d_pair_in<2>, g, 256, 0, x, xs, d, fwx, fhy); break;
    case 3: TP_LAUNCH(k_s2d_pair_in<3>, g, 256, 0, x, xs, d, fwx, fhy); break;
    case 4: TP_LAUNCH(k_s2d_pair_in<4>, g, 256, 0, x, xs, d, fwx, fhy); break;
    default: TP_REQUIRE(false, "paired space-to-depth: 1 to 4 channels");
  }
}

// w [Cout][C][K][K] <-> w'' [Cout][A][AP][32], AP = (A + 1) / 2: slot q*4C + ph*C + ci of
// tap (a, p) is w' tap (a, 2p + q), phase ph, channel ci (zero where that tap does not exist);
// to_s2d = 0 maps a w''-shaped gradient back (each w tap has exactly one slot).
__global__ void k_s2d_pair_filters(const float* __restrict__ src, float* __restrict__ dst, int64_t Cout, S2d d,
                                   int to_s2d) {
  ::tp::pdl_enter();
  const int AP = (d.A + 1) / 2;
  const int64_t total = Cout * d.A * AP * 32;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int sl = (int)(i & 31);
    int64_t t = i >> 5;
    const int p = (int)(t % AP);
    t /= AP;
    const int a = (int)(t % d.A);
    const int64_t co = t / d.A;
    int kh = -1, kw = -1, ci = 0;
    if (sl < 8 * d.C) {
      const int q = sl / (4 * d.C), r = sl - q * 4 * d.C, ph = r / d.C;
      ci = r - ph * d.C;
      const int b = 2 * p + q;
      if (b < d.A) {
        kh = 2 * a + (ph >> 1) + d.P - d.O;
        kw = 2 * b + (ph & 1) + d.P - d.O;
      }
    }
    const bool tap = kh >= 0 && kh < d.K && kw >= 0 && kw < d.K;
    const int64_t wi = ((co * d.C + ci) * d.K + kh) * d.K + kw;
    if (to_s2d) dst[i] = tap ? src[wi] : 0.0f;
    else if (tap) dst[wi] = src[i];
  }
}

// dx'' [N][HY][WX][32] -> dx (NCHW): x' pixel (Y, X) was copied to x'' (Y, X) slot q = 0 and
// (Y, X - 1) slot q = 1, so its gradient is the sum of those two.
__global__ void k_s2d_pair_out(const float* __restrict__ dxs, float* __restrict__ dx, S2d d) {
  ::tp::pdl_enter();
  const int64_t total = d.N * d.C * d.H * d.W;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t iw = i % d.W;
    int64_t t = i / d.W;
    const int64_t ih = t % d.H;
    t /= d.H;
    const int ci = (int)(t % d.C);
    const int64_t n = t / d.C;
    const int64_t ry = ih + d.O, rx = iw + d.O;
    const int64_t Y = ry >> 1, X = rx >> 1;
    const int r = (int)(((ry & 1) * 2 + (rx & 1)) * d.C + ci);
    float v = 0.0f;
    if (Y < d.HY && X < d.WX) {
      const float* row = dxs + (n * d.HY + Y) * d.WX * 32;
      v = row[X * 32 + r];
      if (X >= 1) v += row[(X - 1) * 32 + 4 * d.C + r];
    }
    dx[i] = v;
  }
}

static NhwcShape pair_shape(const S2d& d, int64_t Cout) {
  NhwcShape t = nhwc_shape(d.N, 32, d.HY, d.WX, Cout, d.A, (d.A + 1) / 2, 0, 0, 1);
  t.DW = 2;
  t.OH = d.OH;  // the paired taps reach past the last output column; the grid is the s2d one
  t.OW = d.OW;
  return t;
}

// the paired taps exist only on the TMA paths: every pass's pixel tiling must be possible
static bool pair_ok(const S2d& d) {
  Tiling tl;
  return d.C <= 4 && nhwc_tma_ok() && pixel_tiling(d.N, d.OH, d.OW, tc::BM, tl) &&
         pixel_tiling(d.N, d.HY, d.WX, tc::BM, tl) && pixel_tiling(d.N, d.OH, d.OW, 32, tl);
}

bool conv_fwd_s2d(const ConvShape& s, const float* x, const float* w, const float* bias, float* y) {
  S2d d;
  if (!s2d_plan(s, d) || (bias && ((uintptr_t)bias & 15))) return false;
  if (pair_ok(d) && s.Cout % 4 == 0) {
    const NhwcShape t = pair_shape(d, s.Cout);
    const int AP = (d.A + 1) / 2;
    float* xs = (float*)dalloc((size_t)d.N * d.HY * d.WX * 32 * 4);
    float* ws = (float*)dalloc((size_t)s.Cout * d.A * AP * 32 * 4);
    float* yn = (float*)dalloc((size_t)d.N * d.OH * d.OW * s.Cout * 4);
    s2d_pair_in(x, xs, d);
    TP_LAUNCH(k_s2d_pair_filters, grid_for(s.Cout * d.A * AP * 32, 256), 256, 0, w, ws, s.Cout, d, 1);
    if (!conv_fwd_nhwc(t, xs, ws, bias, yn, nullptr, y)) transpose_nchw_nhwc(yn, y, d.N, s.Cout, d.OH * d.OW, false);
    dfree(xs);
    dfree(ws);
    dfree(yn);
    return true;
  }
  const NhwcShape t = nhwc_shape(d.N, 32, d.HY, d.WX, s.Cout, d.A, d.A, 0, 0, 1);
  float* xs = (float*)dalloc((size_t)d.N * d.HY * d.WX * 32 * 4);
  float* ws = (float*)dalloc((size_t)s.Cout * d.A * d.A * 32 * 4);
  float* yn = (float*)dalloc((size_t)d.N * d.OH * d.OW * s.Cout * 4);
  s2d_in(x, xs, d);
  TP_LAUNCH(k_s2d_filters, grid_for(s.Cout * d.A * d.A * 32, 256), 256, 0, w, ws, s.Cout, d, 1);
  if (!conv_fwd_nhwc(t, xs, ws, bias, yn, nullptr, y)) transpose_nchw_nhwc(yn, y, d.N, s.Cout, d.OH * d.OW, false);
  dfree(xs);
  dfree(ws);
  dfree(yn);
  return true;
}

bool conv_dgrad_s2d(const ConvShape& s, const float* dy, const float* w, float* dx) {
  S2d d;
  if (!s2d_plan(s, d) || s.Cout % 32) return false;
  if (pair_ok(d)) {
    const NhwcShape t = pair_shape(d, s.Cout);
    const int AP = (d.A + 1) / 2;
    float* dyn = (float*)dalloc((size_t)d.N * d.OH * d.OW * s.Cout * 4);
    float* ws = (float*)dalloc((size_t)s.Cout * d.A * AP * 32 * 4);
    float* dxs = (float*)dalloc((size_t)d.N * d.HY * d.WX * 32 * 4);
    transpose_nchw_nhwc(dy, dyn, d.N, s.Cout, d.OH * d.OW, true);
    TP_LAUNCH(k_s2d_pair_filters, grid_for(s.Cout * d.A * AP * 32, 256), 256, 0, w, ws, s.Cout, d, 1);
    conv_dgrad_nhwc(t, dyn, ws, dxs);
    TP_LAUNCH(k_s2d_pair_out, grid_for(d.N * d.C * d.H * d.W, 256), 256, 0, dxs, dx, d);
    dfree(dyn);
    dfree(ws);
    dfree(dxs);
    return true;
  }
  const NhwcShape t = nhwc_shape(d.N, 32, d.HY, d.WX, s.Cout, d.A, d.A, 0, 0, 1);
  float* dyn = (float*)dalloc((size_t)d.N * d.OH * d.OW * s.Cout * 4);
  float* ws = (float*)dalloc((size_t)s.Cout * d.A * d.A * 32 * 4);
  float* dxs = (float*)dalloc((size_t)d.N * d.HY * d.WX * 32 * 4);
  transpose_nchw_nhwc(dy, dyn, d.N, s.Cout, d.OH * d.OW, true);
  TP_LAUNCH(k_s2d_filters, grid_for(s.Cout * d.A * d.A * 32, 256), 256, 0, w, ws, s.Cout, d, 1);
  conv_dgrad_nhwc(t, dyn, ws, dxs);
  TP_LAUNCH(k_s2d_out, grid_for(d.N * d.C * d.H * d.W, 256), 256, 0, dxs, dx, d);
  dfree(dyn);
  dfree(ws);
  dfree(dxs);
  return true;
}

bool conv_wgrad_s2d(const ConvShape& s, const float* dy, const float* x, float* dw) {
  S2d d;
  if (!s2d_plan(s, d) || s.Cout % 32 || s.Cout < 64) return false;
  if (pair_ok(d)) {
    const NhwcShape t = pair_shape(d, s.Cout);
    const int AP = (d.A + 1) / 2;
    float* dyn = (float*)dalloc((size_t)d.N * d.OH * d.OW * s.Cout * 4);
    float* xs = (float*)dalloc((size_t)d.N * d.HY * d.WX * 32 * 4);
    float* dws = (float*)dalloc((size_t)s.Cout * d.A * AP * 32 * 4);
    transpose_nchw_nhwc(dy, dyn, d.N, s.Cout, d.OH * d.OW, true);
    s2d_pair_in(x, xs, d);
    conv_wgrad_nhwc(t, dyn, xs, dws);
    TP_LAUNCH(k_s2d_pair_filters, grid_for(s.Cout * d.A * AP * 32, 256), 256, 0, dws, dw, s.Cout, d, 0);
    dfree(dyn);
    dfree(xs);
    dfree(dws);
    return true;
  }
  const NhwcShape t = nhwc_shape(d.N, 32, d.HY, d.WX, s.Cout, d.A, d.A, 0, 0, 1);
  float* dyn = (float*)dalloc((size_t)d.N * d.OH * d.OW * s.Cout * 4);
  float* xs = (float*)dalloc((size_t)d.N * d.HY * d.WX * 32 * 4);
  float* dws = (float*)dalloc((size_t)s.Cout * d.A * d.A * 32 * 4);
  transpose_nchw_nhwc(dy, dyn, d.N, s.Cout, d.OH * d.OW, true);
  s2d_in(x, xs, d);
  conv_wgrad_nhwc(t, dyn, xs, dws);
  TP_LAUNCH(k_s2d_filters, grid_for(s.Cout * d.A * d.A * 32, 256), 256, 0, dws, dw, s.Cout, d, 0);
  dfree(dyn);
  dfree(xs);
  dfree(dws);
  return true;
}

int tc_status_nhwc(bool reset) {
  int v = 0;
  TP_CUDA(cudaMemcpyFromSymbol(&v, tc::g_status, sizeof(int)));
  if (reset && v) {
    int z = 0;
    TP_CUDA(cudaMemcpyToSymbol(tc::g_status, &z, sizeof(int)));
  }
  return v;
}

}  // namespace tp

using namespace tp;

extern "C" {

TP_API int tpk_conv2d_fwd_nhwc(const float* x, const float* w, const float* bias, float* y, int64_t N, int64_t Cin,
                               int64_t H, int64_t W, int64_t Cout, int KH, int KW, int PH, int PW,
                               int filter_layout) {
  return guard(
      [&] { conv_fwd_nhwc(nhwc_shape(N, Cin, H, W, Cout, KH, KW, PH, PW, filter_layout), x, w, bias, y); });
}

TP_API int tpk_conv2d_dgrad_nhwc(const float* dy, const float* w, float* dx, int64_t N, int64_t Cin, int64_t H,
                                 int64_t W, int64_t Cout, int KH, int KW, int PH, int PW, int filter_layout) {
  return guard([&] { conv_dgrad_nhwc(nhwc_shape(N, Cin, H, W, Cout, KH, KW, PH, PW, filter_layout), dy, w, dx); });
}

TP_API int tpk_conv2d_wgrad_nhwc(const float* dy, const float* x, float* dw, int64_t N, int64_t Cin, int64_t H,
                                 int64_t W, int64_t Cout, int KH, int KW, int PH, int PW, int filter_layout) {
  return guard([&] { conv_wgrad_nhwc(nhwc_shape(N, Cin, H, W, Cout, KH, KW, PH, PW, filter_layout), dy, x, dw); });
}

TP_API int tpk_conv2d_fwd_nhwc_lo(const float* x, const float* w, const float* w_lo, const float* bias, float* y,
                                  int64_t N, int64_t Cin, int64_t H, int64_t W, int64_t Cout, int KH, int KW, int PH,
                                  int PW, int filter_layout) {
  return guard([&] {
    conv_fwd_nhwc(nhwc_shape(N, Cin, H, W, Cout, KH, KW, PH, PW, filter_layout), x, w, bias, y, w_lo);
  });
}

TP_API int tpk_conv2d_dgrad_nhwc_lo(const float* dy, const float* w, const float* w_lo, float* dx, int64_t N,
                                    int64_t Cin, int64_t H, int64_t W, int64_t Cout, int KH, int KW, int PH, int PW,
                                    int filter_layout) {
  return guard([&] {
    conv_dgrad_nhwc(nhwc_shape(N, Cin, H, W, Cout, KH, KW, PH, PW, filter_layout), dy, w, dx, w_lo);
  });
}

TP_API int tpk_tf32_lo(const float* x, float* lo, int64_t n) {
  return guard([&] {
    if (n > 0) tf32_lo_plane(x, lo, n);
  });
}

}  // extern "C"
