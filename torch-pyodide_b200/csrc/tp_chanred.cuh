// Per-channel reductions over the N x spatial plane of an NCHW tensor (BN
// statistics, BN backward sums, conv bias gradient).
//
// grid (C, splits): CTA (c, split) covers images [n0, n1) of channel c.  The
// (image, position) pairs are flattened so every thread has loads in flight
// whatever the spatial size S is (the VGG planes go down to 2x2, where a loop
// over images with a loop over S inside would leave most threads idle).
// 128-bit loads when S % 4 == 0.  Accumulation in f64; per-CTA partials are
// combined by a finishing kernel in a fixed order (deterministic).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "tp_fastdiv.cuh"

namespace tp {

// Each functor: acc4 / acc1 for one float4 / float at a flat index; load4 +
// use4 split the float4 step so several loads can be in flight.

// a += x, b += x*x
struct ChanStatsF {
  const float* x;
  using V = float4;
  __device__ __forceinline__ V load4(int64_t i4) const { return reinterpret_cast<const float4*>(x)[i4]; }
  __device__ __forceinline__ void use4(const V& v, int64_t, double& a, double& b) const {
    a += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
    b += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  }
  __device__ __forceinline__ void acc4(int64_t i4, int64_t, double& a, double& b) const {
    float4 v = reinterpret_cast<const float4*>(x)[i4];
    a += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
    b += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  }
  __device__ __forceinline__ void acc1(int64_t i, int64_t, double& a, double& b) const {
    double v = x[i];
    a += v;
    b += v * v;
  }
};

// a += x (b unused)
struct ChanSumF {
  const float* x;
  using V = float4;
  __device__ __forceinline__ V load4(int64_t i4) const { return reinterpret_cast<const float4*>(x)[i4]; }
  __device__ __forceinline__ void use4(const V& v, int64_t, double& a, double&) const {
    a += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
  }
  __device__ __forceinline__ void acc4(int64_t i4, int64_t, double& a, double&) const {
    float4 v = reinterpret_cast<const float4*>(x)[i4];
    a += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
  }
  __device__ __forceinline__ void acc1(int64_t i, int64_t, double& a, double&) const { a += x[i]; }
};

// g = dy masked by relu_src > 0 (if given); a += g, b += g * x_hat
struct ChanBnBwdF {
  const float* dy;
  const float* x;
  const float* relu_src;
  const float* mean;
  const float* invstd;
  __device__ __forceinline__ float g1(float g, float r) const { return (relu_src && !(r > 0.0f)) ? 0.0f : g; }
  struct V {
    float4 g, x;
  };
  __device__ __forceinline__ V load4(int64_t i4) const {
    V v;
    v.g = reinterpret_cast<const float4*>(dy)[i4];
    v.x = reinterpret_cast<const float4*>(x)[i4];
    if (relu_src) {
      float4 r = reinterpret_cast<const float4*>(relu_src)[i4];
      v.g.x = g1(v.g.x, r.x);
      v.g.y = g1(v.g.y, r.y);
      v.g.z = g1(v.g.z, r.z);
      v.g.w = g1(v.g.w, r.w);
    }
    return v;
  }
  __device__ __forceinline__ void use4(const V& v, int64_t c, double& a, double& b) const {
    float mu = mean[c], is = invstd[c];
    a += (double)v.g.x + (double)v.g.y + (double)v.g.z + (double)v.g.w;
    b += (double)v.g.x * ((v.x.x - mu) * is) + (double)v.g.y * ((v.x.y - mu) * is) +
         (double)v.g.z * ((v.x.z - mu) * is) + (double)v.g.w * ((v.x.w - mu) * is);
  }
  __device__ __forceinline__ void acc4(int64_t i4, int64_t c, double& a, double& b) const {
    float4 g = reinterpret_cast<const float4*>(dy)[i4];
    float4 xv = reinterpret_cast<const float4*>(x)[i4];
    if (relu_src) {
      float4 r = reinterpret_cast<const float4*>(relu_src)[i4];
      g.x = g1(g.x, r.x);
      g.y = g1(g.y, r.y);
      g.z = g1(g.z, r.z);
      g.w = g1(g.w, r.w);
    }
    float mu = mean[c], is = invstd[c];
    a += (double)g.x + (double)g.y + (double)g.z + (double)g.w;
    b += (double)g.x * ((xv.x - mu) * is) + (double)g.y * ((xv.y - mu) * is) + (double)g.z * ((xv.z - mu) * is) +
         (double)g.w * ((xv.w - mu) * is);
  }
  __device__ __forceinline__ void acc1(int64_t i, int64_t c, double& a, double& b) const {
    float g = dy[i];
    if (relu_src) g = g1(g, relu_src[i]);
    a += g;
    b += (double)g * ((x[i] - mean[c]) * invstd[c]);
  }
};

// fs4 / fs: division by S/4 and by S (flat index -> image, position)
template <class F>
__global__ void __launch_bounds__(256) k_chan_reduce(F f, int64_t N, int64_t C, int64_t S, int splits,
                                                     double* __restrict__ part, FastDiv fs4, FastDiv fs) {
  ::tp::pdl_enter();
  __shared__ double sh_a[32], sh_b[32];
  const int64_t c = blockIdx.x;
  const int split = blockIdx.y;
  const int64_t per = (N + splits - 1) / splits;
  const int64_t n0 = split * per, n1 = n0 + per < N ? n0 + per : N;
  double a = 0.0, b = 0.0;
  if (n1 > n0) {
    if ((S & 3) == 0) {
      const uint32_t S4 = (uint32_t)(S >> 2);
      const uint32_t cnt = (uint32_t)((n1 - n0) * S4);
      const uint32_t step = blockDim.x;
      uint32_t i = threadIdx.x;
      // 4 vectors per step, all loaded before any is used
      for (; i + 3 * step < cnt; i += 4 * step) {
        typename F::V v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t ii = i + u * step, dn = fs4.div(ii), s4 = ii - dn * S4;
          v[u] = f.load4(((n0 + dn) * C + c) * (int64_t)S4 + s4);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) f.use4(v[u], c, a, b);
      }
      for (; i < cnt; i += step) {
        uint32_t dn = fs4.div(i), s4 = i - dn * S4;
        int64_t i4 = ((n0 + dn) * C + c) * (int64_t)S4 + s4;
        f.acc4(i4, c, a, b);
      }
    } else {
      const uint32_t Su = (uint32_t)S;
      const uint32_t cnt = (uint32_t)((n1 - n0) * S);
      for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
        uint32_t dn = fs.div(i), s = i - dn * Su;
        f.acc1(((n0 + dn) * C + c) * S + s, c, a, b);
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) {
    sh_a[w] = a;
    sh_b[w] = b;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double ta = 0.0, tb = 0.0;
    for (int k = 0; k < nw; ++k) {
      ta += sh_a[k];
      tb += sh_b[k];
    }
    part[(c * splits + split) * 2] = ta;
    part[(c * splits + split) * 2 + 1] = tb;
  }
}

// The fast divisors k_chan_reduce takes (the flat counts stay below 2^31).
inline FastDiv chan_div4(int64_t S) { return fast_div((uint32_t)((S >> 2) > 0 ? (S >> 2) : 1)); }
inline FastDiv chan_div1(int64_t S) { return fast_div((uint32_t)(S > 0 ? S : 1)); }

// Splits per channel: enough CTAs for a few waves, each with >= ~4K values.
inline int chan_splits(int64_t C, int64_t N, int64_t S, int sms) {
  int splits = 1;
  while (C * splits < (int64_t)sms * 4 && splits * 2 <= N && (N / (splits * 2)) * S >= 4096) splits *= 2;
  return splits;
}

}  // namespace tp
