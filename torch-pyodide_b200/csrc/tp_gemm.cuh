// Generic "gather GEMM" building blocks shared by matmul, linear and the
// implicit-GEMM convolutions.
//
// Every contraction on the hot path is C[m, n] = sum_k A(m, k) * B(n, k) where
// A and B are *gathered* from a tensor: a dense matrix in either layout, or an
// im2col view of an NCHW activation (forward and data-gradient) or of the
// (activation, output-gradient) pair (weight-gradient).  Loader functors give
// A(b, m, k) / B(b, n, k) (b = batch or conv group) and report which index is
// contiguous in memory; epilogue functors place C(b, m, n) (row-major matrix,
// NCHW plane with bias, ...).  The tcgen05 kernel and the CUDA-core kernel use
// the same functors.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tp {

// ---- loaders -------------------------------------------------------------------------------
// Dense row-major [rows, K] (leading dim ld): contiguous along k.
struct LdRowMajor {
  const float* p;
  int64_t ld, bs;
  static constexpr bool kContigK = true;
  __device__ __forceinline__ float operator()(int b, int64_t r, int64_t k) const { return p[b * bs + r * ld + k]; }
};

// Dense column-major view: element (r, k) at p[k*ld + r]: contiguous along r.
struct LdColMajor {
  const float* p;
  int64_t ld, bs;
  static constexpr bool kContigK = false;
  __device__ __forceinline__ float operator()(int b, int64_t r, int64_t k) const { return p[b * bs + k * ld + r]; }
};

struct ConvShape {
  int64_t N, Cin, H, W, Cout, OH, OW;
  int KH, KW, SH, SW, PH, PW;
  int icpg, ocpg;  // channels per group
};

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
};

// Data-gradient A: m = (n, ih, iw), k = (oc, kh, kw) -> dy[n, oc, oh, ow] where
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
};

// Data-gradient B: row n = input channel ic, k = (oc, kh, kw) -> w[oc, ic, kh, kw].
struct LdConvDgradB {
  const float* w;
  ConvShape s;
  static constexpr bool kContigK = true;
  __device__ __forceinline__ float operator()(int, int64_t ic, int64_t k) const {
    int64_t khw = k % ((int64_t)s.KH * s.KW), oc = k / ((int64_t)s.KH * s.KW);
    return w[(oc * s.Cin + ic) * s.KH * s.KW + khw];
  }
};

// Weight-gradient A: row m = oc, k = (n, oh, ow) -> dy[n, oc, oh, ow].
struct LdConvWgradA {
  const float* dy;
  ConvShape s;
  static constexpr bool kContigK = true;
  __device__ __forceinline__ float operator()(int, int64_t oc, int64_t k) const {
    int64_t p = k % (s.OH * s.OW), n = k / (s.OH * s.OW);
    return dy[(n * s.Cout + oc) * s.OH * s.OW + p];
  }
};

// Weight-gradient B: row n = (ic, kh, kw), k = (n, oh, ow) -> x[n, ic, ih, iw]
// (conv_backward.wgsl:66-101 taps).
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
};

}  // namespace tp
