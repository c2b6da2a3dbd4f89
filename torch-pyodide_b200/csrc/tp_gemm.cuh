// Generic "gather GEMM" building blocks shared by matmul, linear and the
// implicit-GEMM convolutions.
//
// Every contraction on the hot path is C[m, n] = sum_k A(m, k) * B(n, k) where
// A and B are *gathered* from a tensor: a dense matrix in either layout, or an
// im2col view of an NCHW activation (forward and data-gradient) or of the
// (activation, output-gradient) pair (weight-gradient).  Nothing is
// materialised: im2col, transposes and flipped filters exist only as index
// maps.  b = batch index (matmul batch, conv group, or filter tap).
//
// A loader gives element access three ways:
//   operator()(b, r, k)            any element (CUDA-core kernel);
//   row(b, r, rows) + fill(row, k0, kend, v[32])
//                                  for loaders contiguous along r: one thread
//                                  per tile row gathers 32 consecutive k with
//                                  the row's index math hoisted (kContigK false);
//   kctx(b, k, kend) + at(b, r, kctx)
//                                  for loaders contiguous along k: lane = k,
//                                  the k decomposition is done once per lane
//                                  and each row costs one load (kContigK true).
// Epilogue functors place C(b, m, n).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace tp {

constexpr int GB_K = 32;  // k values per producer block

// ---- dense matrices ----------------------------------------------------------------------
// Row-major [rows, K] (leading dim ld, batch stride bs): contiguous along k.
struct LdRowMajor {
  const float* p;
  int64_t ld, bs;
  static constexpr bool kContigK = true;
  __device__ __forceinline__ float operator()(int b, int64_t r, int64_t k) const { return p[b * bs + r * ld + k]; }
  struct Kc {
    int64_t off;
    bool ok;
  };
  __device__ __forceinline__ Kc kctx(int b, int64_t k, int64_t kend) const { return Kc{b * bs + k, k < kend}; }
  __device__ __forceinline__ float at(int, int64_t r, const Kc& c) const { return c.ok ? p[c.off + r * ld] : 0.0f; }
};

// Column-major view: element (r, k) at p[k*ld + r]: contiguous along r.
struct LdColMajor {
  const float* p;
  int64_t ld, bs;
  static constexpr bool kContigK = false;
  __device__ __forceinline__ float operator()(int b, int64_t r, int64_t k) const { return p[b * bs + k * ld + r]; }
  struct Row {
    const float* q;
    bool ok;
  };
  __device__ __forceinline__ Row row(int b, int64_t r, int64_t rows) const { return Row{p + b * bs + r, r < rows}; }
  __device__ __forceinline__ void fill(const Row& w, int64_t k0, int64_t kend, float (&v)[GB_K]) const {
    const float* q = w.q + k0 * ld;
#pragma unroll
    for (int j = 0; j < GB_K; ++j) v[j] = (w.ok && k0 + j < kend) ? q[j * ld] : 0.0f;
  }
};

struct ConvShape {
  int64_t N, Cin, H, W, Cout, OH, OW;
  int KH, KW, SH, SW, PH, PW;
  int icpg, ocpg;  // channels per group
};

// ---- convolution, reference K order k = (ic, kh, kw) (any shape) ---------------------------
// Forward A: m = (n, oh, ow), k = (ic_in_group, kh, kw) -> x[n, g*icpg+ic, ih, iw]
// (conv.wgsl:35-54 taps, zero outside the image).  Contiguous along m.
struct LdConvIm2col {
  const float* x;
  ConvShape s;
  static constexpr bool kContigK = false;
  __device__ __forceinline__ float operator()(int g, int64_t m, int64_t k) const {
    int64_t ow = m % s.OW, t = m / s.OW, oh = t % s.OH, n = t / s.OH;
    int kw = (int)(k % s.KW);
    int64_t t2 = k / s.KW;
    int kh = (int)(t2 % s.KH);
    int64_t ic = t2 / s.KH + (int64_t)g * s.icpg;
    int64_t ih = oh * s.SH + kh - s.PH, iw = ow * s.SW + kw - s.PW;
    if (ih < 0 || ih >= s.H || iw < 0 || iw >= s.W) return 0.0f;
    return x[((n * s.Cin + ic) * s.H + ih) * s.W + iw];
  }
  struct Row {
    const float* q;  // x at (n, group channel 0, 0, 0)
    int ih0, iw0;
    bool ok;
  };
  __device__ __forceinline__ Row row(int g, int64_t m, int64_t rows) const {
    Row w;
    w.ok = m < rows;
    int64_t mm = w.ok ? m : 0;
    int ow = (int)(mm % s.OW);
    int64_t t = mm / s.OW;
    int oh = (int)(t % s.OH);
    int64_t n = t / s.OH;
    w.q = x + (n * s.Cin + (int64_t)g * s.icpg) * s.H * s.W;
    w.ih0 = oh * s.SH - s.PH;
    w.iw0 = ow * s.SW - s.PW;
    return w;
  }
  __device__ __forceinline__ void fill(const Row& w, int64_t k0, int64_t kend, float (&v)[GB_K]) const {
    int khw = s.KH * s.KW;
    int ic = (int)(k0 / khw), tap = (int)(k0 - (int64_t)ic * khw);
    int kh = tap / s.KW, kw = tap - kh * s.KW;
#pragma unroll
    for (int j = 0; j < GB_K; ++j) {
      int ih = w.ih0 + kh, iw = w.iw0 + kw;
      bool in = w.ok && k0 + j < kend && ih >= 0 && ih < s.H && iw >= 0 && iw < s.W;
      v[j] = in ? w.q[((int64_t)ic * s.H + ih) * s.W + iw] : 0.0f;
      if (++kw == s.KW) {
        kw = 0;
        if (++kh == s.KH) {
          kh = 0;
          ++ic;
        }
      }
    }
  }
};

// Forward B: weights [Cout, icpg*KH*KW], row n = output channel (of group g).
struct LdConvWeight {
  const float* w;
  int64_t K;  // icpg*KH*KW
  int ocpg;
  static constexpr bool kContigK = true;
  __device__ __forceinline__ float operator()(int g, int64_t n, int64_t k) const {
    return w[((int64_t)g * ocpg + n) * K + k];
  }
  struct Kc {
    int64_t off;
    bool ok;
  };
  __device__ __forceinline__ Kc kctx(int g, int64_t k, int64_t kend) const {
    return Kc{(int64_t)g * ocpg * K + k, k < kend};
  }
  __device__ __forceinline__ float at(int, int64_t n, const Kc& c) const { return c.ok ? w[c.off + n * K] : 0.0f; }
};

// ---- convolution, filter-major K order k = (kh, kw, c) with C % 32 == 0 ---------------------
// A 32-wide k-block then covers one tap and 32 consecutive channels: one
// bounds check per row per block and a strided load per element.  Used for
// the forward (input x, channels icpg) and for the stride-1 data gradient
// written as a forward convolution of dy with flipped, transposed filters
// (input dy, channels Cout, padding K-1-P).  B is the filter repacked to
// [out][kh][kw][c] (k_pack_filters).
struct LdConvFM {
  const float* x;
  int64_t Ctot;      // channels of the input tensor
  int C;             // channels per group (multiple of 32)
  int64_t H, W, OH, OW;
  int KW, SH, SW, PH, PW;
  static constexpr bool kContigK = false;
  struct Row {
    const float* q;
    int ih0, iw0;
    bool ok;
  };
  __device__ __forceinline__ Row row(int g, int64_t m, int64_t rows) const {
    Row w;
    w.ok = m < rows;
    int64_t mm = w.ok ? m : 0;
    int ow = (int)(mm % OW);
    int64_t t = mm / OW;
    int oh = (int)(t % OH);
    int64_t n = t / OH;
    w.q = x + (n * Ctot + (int64_t)g * C) * H * W;
    w.ih0 = oh * SH - PH;
    w.iw0 = ow * SW - PW;
    return w;
  }
  __device__ __forceinline__ void fill(const Row& w, int64_t k0, int64_t kend, float (&v)[GB_K]) const {
    int tap = (int)(k0 / C), c0 = (int)(k0 - (int64_t)tap * C);
    int kh = tap / KW, kw = tap - kh * KW;
    int ih = w.ih0 + kh, iw = w.iw0 + kw;
    bool in = w.ok && k0 < kend && ih >= 0 && ih < H && iw >= 0 && iw < W;
    const int64_t hw = H * W;
    const float* q = w.q + (int64_t)c0 * hw + (int64_t)ih * W + iw;
#pragma unroll
    for (int j = 0; j < GB_K; ++j) v[j] = in ? q[j * hw] : 0.0f;
  }
};

// ---- data gradient, general stride --------------------------------------------------------
// A: m = (n, ih, iw), k = (oc, kh, kw) -> dy[n, oc, oh, ow] where
// ih + PH - kh = oh*SH and iw + PW - kw = ow*SW (conv_backward.wgsl:24-61).
struct LdConvDgradA {
  const float* dy;
  ConvShape s;
  static constexpr bool kContigK = false;
  __device__ __forceinline__ float operator()(int, int64_t m, int64_t k) const {
    int64_t iw = m % s.W, t = m / s.W, ih = t % s.H, n = t / s.H;
    int kw = (int)(k % s.KW);
    int64_t t2 = k / s.KW;
    int kh = (int)(t2 % s.KH);
    int64_t oc = t2 / s.KH;
    int64_t ohb = ih + s.PH - kh, owb = iw + s.PW - kw;
    if (ohb < 0 || owb < 0 || ohb % s.SH || owb % s.SW) return 0.0f;
    int64_t oh = ohb / s.SH, ow = owb / s.SW;
    if (oh >= s.OH || ow >= s.OW) return 0.0f;
    return dy[((n * s.Cout + oc) * s.OH + oh) * s.OW + ow];
  }
  struct Row {
    int64_t m;
    bool ok;
  };
  __device__ __forceinline__ Row row(int, int64_t m, int64_t rows) const { return Row{m, m < rows}; }
  __device__ __forceinline__ void fill(const Row& w, int64_t k0, int64_t kend, float (&v)[GB_K]) const {
#pragma unroll 4
    for (int j = 0; j < GB_K; ++j) v[j] = (w.ok && k0 + j < kend) ? (*this)(0, w.m, k0 + j) : 0.0f;
  }
};

// B: row n = input channel ic, k = (oc, kh, kw) -> w[oc, ic, kh, kw].
struct LdConvDgradB {
  const float* w;
  ConvShape s;
  static constexpr bool kContigK = true;
  __device__ __forceinline__ float operator()(int, int64_t ic, int64_t k) const {
    int64_t khw = k % ((int64_t)s.KH * s.KW), oc = k / ((int64_t)s.KH * s.KW);
    return w[(oc * s.Cin + ic) * s.KH * s.KW + khw];
  }
  struct Kc {
    int64_t off;
    bool ok;
  };
  __device__ __forceinline__ Kc kctx(int, int64_t k, int64_t kend) const {
    int64_t kk = (int64_t)s.KH * s.KW;
    int64_t oc = k / kk;
    return Kc{oc * s.Cin * kk + (k - oc * kk), k < kend};
  }
  __device__ __forceinline__ float at(int, int64_t ic, const Kc& c) const {
    return c.ok ? w[c.off + ic * s.KH * s.KW] : 0.0f;
  }
};

// ---- weight gradient ------------------------------------------------------------------------
// Reference K order (CUDA-core path): row m = oc, k = (n, oh, ow) -> dy[n, oc, oh, ow];
// row n = (ic, kh, kw), k = (n, oh, ow) -> x[n, ic, ih, iw] (conv_backward.wgsl:66-101).
struct LdConvWgradA {
  const float* dy;
  ConvShape s;
  static constexpr bool kContigK = true;
  __device__ __forceinline__ float operator()(int, int64_t oc, int64_t k) const {
    int64_t p = k % (s.OH * s.OW), n = k / (s.OH * s.OW);
    return dy[(n * s.Cout + oc) * s.OH * s.OW + p];
  }
  struct Kc {
    int64_t off;
    bool ok;
  };
  __device__ __forceinline__ Kc kctx(int, int64_t k, int64_t kend) const {
    int64_t P = s.OH * s.OW;
    int64_t n = k / P;
    return Kc{n * s.Cout * P + (k - n * P), k < kend};
  }
  __device__ __forceinline__ float at(int, int64_t oc, const Kc& c) const {
    return c.ok ? dy[c.off + oc * s.OH * s.OW] : 0.0f;
  }
};

struct LdConvWgradB {
  const float* x;
  ConvShape s;
  static constexpr bool kContigK = true;
  __device__ __forceinline__ float operator()(int, int64_t r, int64_t k) const {
    int kw = (int)(r % s.KW);
    int64_t t = r / s.KW;
    int kh = (int)(t % s.KH);
    int64_t ic = t / s.KH;
    int64_t ow = k % s.OW, t2 = k / s.OW, oh = t2 % s.OH, n = t2 / s.OH;
    int64_t ih = oh * s.SH + kh - s.PH, iw = ow * s.SW + kw - s.PW;
    if (ih < 0 || ih >= s.H || iw < 0 || iw >= s.W) return 0.0f;
    return x[((n * s.Cin + ic) * s.H + ih) * s.W + iw];
  }
  // per lane: the image and output position of k; per row: the tap and channel
  struct Kc {
    const float* xn;
    int ih0, iw0;
    bool ok;
  };
  __device__ __forceinline__ Kc kctx(int, int64_t k, int64_t kend) const {
    Kc c;
    c.ok = k < kend;
    int64_t kk = c.ok ? k : 0;
    int64_t P = s.OH * s.OW;
    int64_t n = kk / P;
    int p = (int)(kk - n * P);
    int oh = p / (int)s.OW, ow = p - oh * (int)s.OW;
    c.xn = x + n * s.Cin * s.H * s.W;
    c.ih0 = oh * s.SH - s.PH;
    c.iw0 = ow * s.SW - s.PW;
    return c;
  }
  __device__ __forceinline__ float at(int, int64_t r, const Kc& c) const {
    int ri = (int)r;
    int t = ri / s.KW, kw = ri - t * s.KW;
    int ic = t / s.KH, kh = t - ic * s.KH;
    int ih = c.ih0 + kh, iw = c.iw0 + kw;
    bool in = c.ok && ih >= 0 && ih < s.H && iw >= 0 && iw < s.W;
    return in ? c.xn[((int64_t)ic * s.H + ih) * s.W + iw] : 0.0f;
  }
};

// Per-tap weight gradient for the tensor-core path: batch index = tap (kh, kw).
// A(oc, k = (n, p)) = dy[n, oc, p];  B(ic, k = (n, oh, ow)) = x[n, ic, oh*SH+kh-PH, ow*SW+kw-PW].
struct LdWgradTapDy {
  const float* dy;
  int64_t Cout, P;
  static constexpr bool kContigK = true;
  struct Kc {
    int64_t off;
    bool ok;
  };
  __device__ __forceinline__ Kc kctx(int, int64_t k, int64_t kend) const {
    int64_t n = k / P;
    return Kc{n * Cout * P + (k - n * P), k < kend};
  }
  __device__ __forceinline__ float at(int, int64_t oc, const Kc& c) const { return c.ok ? dy[c.off + oc * P] : 0.0f; }
};

struct LdWgradTapX {
  const float* x;
  int64_t Cin, H, W, OH, OW;
  int KW, SH, SW, PH, PW;
  static constexpr bool kContigK = true;
  struct Kc {
    int64_t off;
    bool ok;
  };
  __device__ __forceinline__ Kc kctx(int tap, int64_t k, int64_t kend) const {
    int kh = tap / KW, kw = tap - kh * KW;
    int64_t P = OH * OW;
    int64_t n = k / P, p = k - n * P;
    int oh = (int)(p / OW), ow = (int)(p - (int64_t)oh * OW);
    int ih = oh * SH + kh - PH, iw = ow * SW + kw - PW;
    bool ok = k < kend && ih >= 0 && ih < H && iw >= 0 && iw < W;
    return Kc{ok ? (n * Cin * H + ih) * W + iw : 0, ok};
  }
  __device__ __forceinline__ float at(int, int64_t ic, const Kc& c) const {
    return c.ok ? x[c.off + ic * H * W] : 0.0f;
  }
};

// ---- epilogues ------------------------------------------------------------------------------
// Row-major C[b][m][n] (+ bias[n]) (+ ReLU).
struct EpRowMajor {
  float* c;
  int64_t ldc, bs;
  const float* bias;
  int relu;
  __device__ __forceinline__ void operator()(int b, int64_t m, int64_t n, float v) const {
    if (bias) v += bias[n];
    if (relu) v = fmaxf(v, 0.0f);
    c[b * bs + m * ldc + n] = v;
  }
  // 4 consecutive columns of row m (columns >= N skipped), one 128-bit store
  // when whole and 16-byte aligned
  __device__ __forceinline__ void row4(int b, int64_t m, int64_t n0, int64_t N, float4 v) const {
    if (n0 >= N) return;
    float* dst = c + b * bs + m * ldc + n0;
    if (bias) {
      const float4 z = n0 + 4 <= N ? make_float4(bias[n0], bias[n0 + 1], bias[n0 + 2], bias[n0 + 3])
                                   : make_float4(bias[n0], n0 + 1 < N ? bias[n0 + 1] : 0.0f,
                                                 n0 + 2 < N ? bias[n0 + 2] : 0.0f, n0 + 3 < N ? bias[n0 + 3] : 0.0f);
      v.x += z.x;
      v.y += z.y;
      v.z += z.z;
      v.w += z.w;
    }
    if (relu) {
      v.x = fmaxf(v.x, 0.0f);
      v.y = fmaxf(v.y, 0.0f);
      v.z = fmaxf(v.z, 0.0f);
      v.w = fmaxf(v.w, 0.0f);
    }
    if (n0 + 4 <= N && ((uintptr_t)dst & 15) == 0) {
      *reinterpret_cast<float4*>(dst) = v;
      return;
    }
    const float o[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (n0 + i < N) dst[i] = o[i];
  }
  // 16 consecutive columns of row m (columns >= N skipped); 128-bit stores
  // when the row segment is whole and 16-byte aligned
  __device__ __forceinline__ void row16(int b, int64_t m, int64_t n0, int64_t N, const float (&v)[16]) const {
    float* dst = c + b * bs + m * ldc + n0;
    if (n0 + 16 <= N && ((uintptr_t)dst & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        float4 o;
        o.x = bias ? v[i] + bias[n0 + i] : v[i];
        o.y = bias ? v[i + 1] + bias[n0 + i + 1] : v[i + 1];
        o.z = bias ? v[i + 2] + bias[n0 + i + 2] : v[i + 2];
        o.w = bias ? v[i + 3] + bias[n0 + i + 3] : v[i + 3];
        if (relu) {
          o.x = fmaxf(o.x, 0.0f);
          o.y = fmaxf(o.y, 0.0f);
          o.z = fmaxf(o.z, 0.0f);
          o.w = fmaxf(o.w, 0.0f);
        }
        *reinterpret_cast<float4*>(dst + i) = o;
      }
      return;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (n0 + i < N) (*this)(b, m, n0 + i, v[i]);
  }
};

// NCHW output plane: m = (img, p), n = channel within group b -> out[img, b*ocpg+n, p] (+ bias).
struct EpNCHW {
  float* out;
  const float* bias;
  int64_t C, P;  // total channels, spatial size
  int ocpg;
  __device__ __forceinline__ void operator()(int b, int64_t m, int64_t n, float v) const {
    int64_t c = (int64_t)b * ocpg + n;
    if (bias) v += bias[c];
    int64_t img = m / P, p = m % P;
    out[(img * C + c) * P + p] = v;
  }
  __device__ __forceinline__ void row16(int b, int64_t m, int64_t n0, int64_t N, const float (&v)[16]) const {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (n0 + i < N) (*this)(b, m, n0 + i, v[i]);
  }
};

// Per-tap weight gradient: C_tap[oc][ic] -> dW[oc, ic, tap].
struct EpWgradTap {
  float* dw;
  int64_t Cin;
  int KHW;
  __device__ __forceinline__ void operator()(int tap, int64_t oc, int64_t ic, float v) const {
    dw[(oc * Cin + ic) * KHW + tap] = v;
  }
  __device__ __forceinline__ void row16(int b, int64_t m, int64_t n0, int64_t N, const float (&v)[16]) const {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (n0 + i < N) (*this)(b, m, n0 + i, v[i]);
  }
};

// Per-tap weight gradient into filters stored [Cout][KHW][Cin]:
// C_tap[oc][ic] -> dw[oc, tap, ic] (16 consecutive ic are one contiguous run).
struct EpWgradTapKhwc {
  float* dw;
  int64_t Cin;
  int KHW;
  __device__ __forceinline__ void operator()(int tap, int64_t oc, int64_t ic, float v) const {
    dw[(oc * KHW + tap) * Cin + ic] = v;
  }
  __device__ __forceinline__ void row16(int b, int64_t m, int64_t n0, int64_t N, const float (&v)[16]) const {
    EpRowMajor{dw + (m * KHW + b) * Cin, 0, 0, nullptr, 0}.row16(0, 0, n0, N, v);
  }
  __device__ __forceinline__ void row4(int b, int64_t m, int64_t n0, int64_t N, float4 v) const {
    EpRowMajor{dw + (m * KHW + b) * Cin, 0, 0, nullptr, 0}.row4(0, 0, n0, N, v);
  }
};

// Per-tap weight gradient of TAPS taps at once (Cin = 128 / TAPS): batch b
// covers taps TAPS*b .., GEMM column n = (n / Cin)-th tap of the group, channel
// n % Cin; columns of a tap past KHW are dropped.
template <int TAPS>
struct EpWgradTapsKhwc {
  float* dw;
  int64_t Cin;
  int KHW;
  __device__ __forceinline__ void operator()(int b, int64_t oc, int64_t n, float v) const {
    const int tap = TAPS * b + (int)(n / Cin);
    if (tap < KHW) dw[(oc * KHW + tap) * Cin + n % Cin] = v;
  }
  __device__ __forceinline__ void row16(int b, int64_t m, int64_t n0, int64_t, const float (&v)[16]) const {
    const int tap = TAPS * b + (int)(n0 / Cin);  // Cin % 16 == 0: the 16 columns share a tap
    if (tap >= KHW) return;
    EpRowMajor{dw + (m * KHW + tap) * Cin, 0, 0, nullptr, 0}.row16(0, 0, n0 % Cin, Cin, v);
  }
  __device__ __forceinline__ void row4(int b, int64_t m, int64_t n0, int64_t, float4 v) const {
    const int tap = TAPS * b + (int)(n0 / Cin);
    if (tap >= KHW) return;
    EpRowMajor{dw + (m * KHW + tap) * Cin, 0, 0, nullptr, 0}.row4(0, 0, n0 % Cin, Cin, v);
  }
};

// Epilogues whose row m is one contiguous run of columns provide row4(b, m, n,
// N, float4); the TMA kernels then stage the accumulator tile in shared memory
// and store whole rows (each warp instruction a contiguous 256-512 B run)
// instead of 16 columns per thread (a row per lane: 32 rows per instruction).
template <class E, class = void>
struct HasRow4 : std::false_type {};
template <class E>
struct HasRow4<E, std::void_t<decltype(&E::row4)>> : std::true_type {};

}  // namespace tp
