// First-layer convolution with 4 input channels (an RGB batch padded to 4 so
// every pixel is one 16-byte vector), channels-last, 3x3, stride 1: forward
// and weight gradient on the CUDA cores.
//
// Such a layer does only K = 36 multiply-adds per output (VGG-11-BN's first
// conv: 3.6 GFLOP each way at batch 1024).  The tensor-core kernel needs 32
// channels per k-block, so it would run this shape padded 8x with half-empty
// 128-row tiles; a register-tiled CUDA-core kernel that reads each pixel's 4
// channels as one vector does the real work instead.
//
// Forward:  thread = (pixel lane, 4 output channels); filters in shared memory
//           as float4 over output channels; y = bias + sum_(kh,kw,c) x w.
// Gradient: thread = (pixel lane, input channel, 4 output channels) with the
//           9 taps x 4 outputs in registers; per-CTA sums over pixel lanes in
//           shared memory (fixed order), per-split partials summed in f64 in
//           split order by a second kernel.
#include <cuda_runtime.h>

#include "tp_core.h"

namespace tp {

constexpr int SC_THREADS = 256;

template <int KH, int KW>
__global__ void __launch_bounds__(SC_THREADS)
    k_conv_c4_fwd(const float4* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias,
                  float4* __restrict__ y, int64_t P, int H, int W, int OH, int OW, int PH, int PW, int Cout) {
  extern __shared__ float4 wsm[];  // [tap][ci][G]: (w[4g..4g+3][ci][tap])
  const int G = Cout >> 2, R = SC_THREADS / G;
  constexpr int T = KH * KW;
  for (int i = threadIdx.x; i < T * 4 * G; i += blockDim.x) {
    const int g = i % G, ci = (i / G) & 3, tap = i / (4 * G);
    float4 v;
    v.x = w[((4 * g + 0) * 4 + ci) * T + tap];
    v.y = w[((4 * g + 1) * 4 + ci) * T + tap];
    v.z = w[((4 * g + 2) * 4 + ci) * T + tap];
    v.w = w[((4 * g + 3) * 4 + ci) * T + tap];
    wsm[i] = v;
  }
  __syncthreads();
  const int g = threadIdx.x % G, r = threadIdx.x / G;
  if (r >= R) return;
  const float4 b4 = bias ? reinterpret_cast<const float4*>(bias)[g] : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t p = (int64_t)blockIdx.x * R + r; p < P; p += (int64_t)gridDim.x * R) {
    const int ow = (int)(p % OW);
    const int64_t t = p / OW;
    const int oh = (int)(t % OH);
    const int64_t n = t / OH;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh + kh - PH;
      if (ih < 0 || ih >= H) continue;
#pragma unroll
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow + kw - PW;
        if (iw < 0 || iw >= W) continue;
        const float4 xv = x[(n * H + ih) * W + iw];
        const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int ci = 0; ci < 4; ++ci) {
          const float4 wv = wsm[((kh * KW + kw) * 4 + ci) * G + g];
          acc.x = fmaf(xs[ci], wv.x, acc.x);
          acc.y = fmaf(xs[ci], wv.y, acc.y);
          acc.z = fmaf(xs[ci], wv.z, acc.z);
          acc.w = fmaf(xs[ci], wv.w, acc.w);
        }
      }
    }
    y[p * G + g] = make_float4(acc.x + b4.x, acc.y + b4.y, acc.z + b4.z, acc.w + b4.w);
  }
}

template <int KH, int KW>
__global__ void __launch_bounds__(SC_THREADS)
    k_conv_c4_wgrad(const float4* __restrict__ dy, const float* __restrict__ x, float* __restrict__ part, int64_t P,
                    int H, int W, int OH, int OW, int PH, int PW, int Cout, int64_t rows_per_split) {
  extern __shared__ float sh[];  // [R][Cout][4][T]
  constexpr int T = KH * KW;
  const int G = Cout >> 2, R = SC_THREADS / (4 * G);
  const int g = threadIdx.x % G, ci = (threadIdx.x / G) & 3, r = threadIdx.x / (4 * G);
  const int64_t p0 = (int64_t)blockIdx.x * rows_per_split;
  const int64_t p1 = p0 + rows_per_split < P ? p0 + rows_per_split : P;
  float acc[T][4];
#pragma unroll
  for (int t = 0; t < T; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
  if (r < R) {
    for (int64_t p = p0 + r; p < p1; p += R) {
      const int ow = (int)(p % OW);
      const int64_t q = p / OW;
      const int oh = (int)(q % OH);
      const int64_t n = q / OH;
      const float4 d = dy[p * G + g];
#pragma unroll
      for (int kh = 0; kh < KH; ++kh) {
        const int ih = oh + kh - PH;
#pragma unroll
        for (int kw = 0; kw < KW; ++kw) {
          const int iw = ow + kw - PW;
          const float v = (ih >= 0 && ih < H && iw >= 0 && iw < W) ? x[((n * H + ih) * W + iw) * 4 + ci] : 0.0f;
          const int t = kh * KW + kw;
          acc[t][0] = fmaf(v, d.x, acc[t][0]);
          acc[t][1] = fmaf(v, d.y, acc[t][1]);
          acc[t][2] = fmaf(v, d.z, acc[t][2]);
          acc[t][3] = fmaf(v, d.w, acc[t][3]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < T; ++t)
#pragma unroll
      for (int j = 0; j < 4; ++j) sh[(((int64_t)r * Cout + 4 * g + j) * 4 + ci) * T + t] = acc[t][j];
  }
  __syncthreads();
  const int per = Cout * 4 * T;
  for (int i = threadIdx.x; i < per; i += blockDim.x) {
    float s = 0.0f;
    for (int k = 0; k < R; ++k) s += sh[(int64_t)k * per + i];
    part[(int64_t)blockIdx.x * per + i] = s;
  }
}

// dw[i] = sum over splits of part[split][i] (f64, split order); i = (co*4 + ci)*T + tap
__global__ void k_conv_c4_wgrad_finish(const float* __restrict__ part, int splits, int per, float* __restrict__ dw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= per) return;
  double s = 0.0;
  for (int k = 0; k < splits; ++k) s += part[(int64_t)k * per + i];
  dw[i] = (float)s;
}

// True when the 4-channel kernels apply: x has exactly 4 channels, 3x3
// filters, Cout % 4 == 0 and <= 256, 16-byte aligned buffers.
bool conv_c4_ok(int64_t Cin, int KH, int KW, int64_t Cout, const void* a, const void* b) {
  return Cin == 4 && KH == 3 && KW == 3 && Cout % 4 == 0 && Cout >= 4 && Cout <= 256 &&
         ((uintptr_t)a & 15) == 0 && ((uintptr_t)b & 15) == 0;
}

void conv_c4_fwd(const float* x, const float* w, const float* bias, float* y, int64_t N, int64_t H, int64_t W,
                 int64_t Cout, int PH, int PW) {
  const int OH = (int)(H + 2 * PH - 2), OW = (int)(W + 2 * PW - 2);
  const int64_t P = N * OH * OW;
  if (P == 0) return;
  TP_REQUIRE(bias == nullptr || ((uintptr_t)bias & 15) == 0, "conv2d: bias must be 16-byte aligned");
  const int G = (int)(Cout / 4), R = SC_THREADS / G;
  size_t shb = (size_t)9 * 4 * G * sizeof(float4);
  int64_t blocks = (P + R - 1) / R;
  int64_t cap = (int64_t)sm_count() * 8;
  auto kfn = k_conv_c4_fwd<3, 3>;
  TP_LAUNCH(kfn, (unsigned)(blocks < cap ? blocks : cap), SC_THREADS, shb, reinterpret_cast<const float4*>(x), w,
            bias, reinterpret_cast<float4*>(y), P, (int)H, (int)W, OH, OW, PH, PW, (int)Cout);
}

void conv_c4_wgrad(const float* dy, const float* x, float* dw, int64_t N, int64_t H, int64_t W, int64_t Cout, int PH,
                   int PW) {
  const int OH = (int)(H + 2 * PH - 2), OW = (int)(W + 2 * PW - 2);
  const int64_t P = N * OH * OW;
  const int per = (int)(Cout * 4 * 9);
  const int G = (int)(Cout / 4), R = SC_THREADS / (4 * G);
  int64_t splits = (int64_t)sm_count() * 4;
  int64_t maxs = P / ((int64_t)R * 64);
  if (maxs < 1) maxs = 1;
  if (splits > maxs) splits = maxs;
  const int64_t rows = (P + splits - 1) / splits;
  splits = P > 0 ? (P + rows - 1) / rows : 1;
  float* part = (float*)scratch((size_t)splits * per * sizeof(float));
  if (P > 0) {
    size_t shb = (size_t)R * per * sizeof(float);
    auto kfn = k_conv_c4_wgrad<3, 3>;
    TP_LAUNCH(kfn, (unsigned)splits, SC_THREADS, shb, reinterpret_cast<const float4*>(dy), x, part, P, (int)H,
              (int)W, OH, OW, PH, PW, (int)Cout, rows);
  } else {
    TP_CUDA(cudaMemsetAsync(part, 0, (size_t)per * sizeof(float), stream()));
    splits = 1;
  }
  TP_LAUNCH(k_conv_c4_wgrad_finish, (unsigned)((per + 255) / 256), 256, 0, part, (int)splits, per, dw);
}

}  // namespace tp
