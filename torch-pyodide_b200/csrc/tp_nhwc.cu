// Channels-last ([pixels][C]) companions of the NCHW norm / pool / bias
// kernels, for a training step that keeps its activations channels-last:
// BatchNorm train forward (+ReLU) and backward (+ReLU mask), the per-channel
// sum (conv bias gradient), 2x2 / stride-2 max pooling with indices, and the
// NCHW -> channels-last input conversion.
//
// Same arithmetic as the NCHW kernels in tp_norm.cu / tp_pool.cu (which follow
// the reference's intended BatchNorm training semantics, tensor_nn_ops.py:92-254
// and autograd_rules.py:1049-1130, and max_pool2d.wgsl:22-49): f64 partial
// sums per channel combined in a fixed order, identical per-element formulas,
// strict > with row-major window order for the pool.  Only the memory order
// differs: channels are contiguous, so every kernel moves 16-byte vectors of 4
// channels and a per-channel reduction is a column reduction over pixel rows.
// The BatchNorm backward's normalising pass also sums its output per channel,
// which is the gradient of the conv bias feeding the BatchNorm, so that bias
// gradient costs no extra pass over the activations.
#include <cuda_runtime.h>

#include "tp_core.h"
#include "tp_fastdiv.cuh"
#include "tp_launch.h"

namespace tp {

// ---- finishing: one warp per channel sums its splits' f64 partials (lane-strided,
// then a fixed xor-shuffle tree, so the order is the same on every run) ----------------------
__device__ __forceinline__ void warp_part_sum(const double* __restrict__ part, int64_t c, int splits, double& a,
                                              double& b) {
  const int lane = threadIdx.x & 31;
  a = 0.0;
  b = 0.0;
  for (int k = lane; k < splits; k += 32) {
    a += part[(c * splits + k) * 2];
    b += part[(c * splits + k) * 2 + 1];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
}

// mean, biased var -> inv_std; running stats with the unbiased variance
// (the formulas of the NCHW finishing kernel in tp_norm.cu)
__global__ void k_col_bn_finish(const double* __restrict__ part, int64_t C, int splits, double M, float eps,
                                float momentum, float* __restrict__ save_mean, float* __restrict__ save_invstd,
                                float* __restrict__ rm, float* __restrict__ rv) {
  ::tp::pdl_enter();
  const int64_t c = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (c >= C) return;
  double s, q;
  warp_part_sum(part, c, splits, s, q);
  if ((threadIdx.x & 31) != 0) return;
  double mean = s / M;
  double var = q / M - mean * mean;
  if (var < 0.0) var = 0.0;
  save_mean[c] = (float)mean;
  save_invstd[c] = (float)(1.0 / sqrt(var + (double)eps));
  if (rm) rm[c] = (float)(mean * momentum + (double)rm[c] * (1.0 - momentum));
  if (rv) rv[c] = (float)(var * M / (M - 1.0) * momentum + (double)rv[c] * (1.0 - momentum));
}

// coef[c] = {w*invstd, sum_dy/M, sum_dyxh/M}; dw, db
__global__ void k_col_bn_bwd_finish(const double* __restrict__ part, int64_t C, int splits, double M,
                                    const float* __restrict__ w, const float* __restrict__ invstd,
                                    float* __restrict__ coef, float* __restrict__ dw, float* __restrict__ db) {
  ::tp::pdl_enter();
  const int64_t c = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (c >= C) return;
  double a, b;
  warp_part_sum(part, c, splits, a, b);
  if ((threadIdx.x & 31) != 0) return;
  coef[c * 3] = (w ? w[c] : 1.0f) * invstd[c];
  coef[c * 3 + 1] = (float)(a / M);
  coef[c * 3 + 2] = (float)(b / M);
  if (dw) dw[c] = (float)b;
  if (db) db[c] = (float)a;
}

__global__ void k_col_sum_finish(const double* __restrict__ part, int64_t C, int splits, float* __restrict__ out) {
  ::tp::pdl_enter();
  const int64_t c = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (c >= C) return;
  double a, b;
  warp_part_sum(part, c, splits, a, b);
  if ((threadIdx.x & 31) == 0) out[c] = (float)a;
}

static unsigned finish_grid(int64_t C) { return (unsigned)((C + 7) / 8); }

// ---- column reductions over [P][C] ----------------------------------------------------------
// CTA (split, column block) covers rows [p0, p1) of CB channels.  Thread t:
// channel group g = t % (CB/4) (4 channels), row lane r = t / (CB/4).  Per-thread
// f64 sums are combined over row lanes in shared memory in lane order, giving
// part[(c*splits + split)*2 + {0,1}].

// The BatchNorm output value of the forward pass, also used to recompute the
// ReLU mask in the backward: fma(x - mean, invstd*gamma, beta), so both see the
// same float.
__device__ __forceinline__ float bn_val(float x, float mu, float sc, float bs) { return __fmaf_rn(x - mu, sc, bs); }

// Functors: ctx(c0) loads what the thread's 4 channels need once; load(p, cg)
// fetches the operands of pixel row p, channel group cg (4 channels; GT groups
// per row) and use() consumes them, so the row loop can have several rows'
// loads in flight.
struct NoCtx {};

struct ColStatsF {  // a += x, b += x*x
  const float* x;
  int GT;
  static constexpr int kUnroll = 8, kMinBlocks = 4, kMinRows = 16;
  using Ctx = NoCtx;
  using V = float4;
  __device__ __forceinline__ Ctx ctx(int) const { return {}; }
  __device__ __forceinline__ V load(int64_t p, int cg) const {
    return reinterpret_cast<const float4*>(x)[p * GT + cg];
  }
  __device__ __forceinline__ void use(int64_t, int, const V& v, const Ctx&, double (&a)[4], double (&b)[4]) const {
    a[0] += v.x, a[1] += v.y, a[2] += v.z, a[3] += v.w;
    b[0] += (double)v.x * v.x, b[1] += (double)v.y * v.y, b[2] += (double)v.z * v.z, b[3] += (double)v.w * v.w;
  }
};

struct ColSumF {  // a += x
  const float* x;
  int GT;
  static constexpr int kUnroll = 8, kMinBlocks = 4, kMinRows = 16;
  using Ctx = NoCtx;
  using V = float4;
  __device__ __forceinline__ Ctx ctx(int) const { return {}; }
  __device__ __forceinline__ V load(int64_t p, int cg) const {
    return reinterpret_cast<const float4*>(x)[p * GT + cg];
  }
  __device__ __forceinline__ void use(int64_t, int, const V& v, const Ctx&, double (&a)[4], double (&)[4]) const {
    a[0] += v.x, a[1] += v.y, a[2] += v.z, a[3] += v.w;
  }
};

// Per-channel values a BatchNorm backward thread keeps for its 4 channels.
struct BwdCtx {
  float mu[4], is[4], sc[4], bs[4], k0[4], k1[4], k2[4];
};

__device__ __forceinline__ BwdCtx bwd_ctx(int c0, const float* mean, const float* invstd, const float* gamma,
                                          const float* beta, const float* coef) {
  BwdCtx c;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    c.mu[j] = mean[c0 + j];
    c.is[j] = invstd[c0 + j];
    c.sc[j] = invstd[c0 + j] * (gamma ? gamma[c0 + j] : 1.0f);
    c.bs[j] = beta ? beta[c0 + j] : 0.0f;
    c.k0[j] = coef ? coef[(c0 + j) * 3] : 0.0f;
    c.k1[j] = coef ? coef[(c0 + j) * 3 + 1] : 0.0f;
    c.k2[j] = coef ? coef[(c0 + j) * 3 + 2] : 0.0f;
  }
  return c;
}

// ReLU mask recomputed from the BatchNorm input: the forward's output
// bn_val(x) was > 0 exactly where the stored activation is.
__device__ __forceinline__ void relu_mask_from_x(float4& g, const float4& x, const BwdCtx& c) {
  if (!(bn_val(x.x, c.mu[0], c.sc[0], c.bs[0]) > 0.0f)) g.x = 0.0f;
  if (!(bn_val(x.y, c.mu[1], c.sc[1], c.bs[1]) > 0.0f)) g.y = 0.0f;
  if (!(bn_val(x.z, c.mu[2], c.sc[2], c.bs[2]) > 0.0f)) g.z = 0.0f;
  if (!(bn_val(x.w, c.mu[3], c.sc[3], c.bs[3]) > 0.0f)) g.w = 0.0f;
}

// Where the BatchNorm backward takes the gradient g at its output and its
// input x.  A source's row p covers NPIX pixels; V holds their g and x and the
// first pixel's index, and off(v, k, cg) is the float4 index of pixel k.
//
// PixSrc: one pixel per row, g read from dy [P][C]; the ReLU mask from the
// stored activation (relu_src > 0) or recomputed from x (relu_from_x).
struct PixSrc {
  static constexpr int NPIX = 1, kUnroll = 4, kMinBlocks = 2, kMinRows = 16;
  struct V {
    float4 g[1], x[1];
    int64_t base;
  };
  const float* dy;
  const float* x;
  const float* relu_src;
  int GT, relu_from_x;
  __device__ __forceinline__ int64_t off(const V& v, int, int cg) const { return v.base * GT + cg; }
  __device__ __forceinline__ V load(int64_t p, int cg, const BwdCtx& c) const {
    V v;
    v.base = p;
    const int64_t i4 = p * GT + cg;
    v.x[0] = reinterpret_cast<const float4*>(x)[i4];
    v.g[0] = reinterpret_cast<const float4*>(dy)[i4];
    if (relu_src) {
      const float4 r = reinterpret_cast<const float4*>(relu_src)[i4];
      if (!(r.x > 0.0f)) v.g[0].x = 0.0f;
      if (!(r.y > 0.0f)) v.g[0].y = 0.0f;
      if (!(r.z > 0.0f)) v.g[0].z = 0.0f;
      if (!(r.w > 0.0f)) v.g[0].w = 0.0f;
    } else if (relu_from_x) {
      relu_mask_from_x(v.g[0], v.x[0], c);
    }
    return v;
  }
};

// PoolSrc: row q is a 2x2 window of a stride-2 max-pool that followed the
// BatchNorm(+ReLU); the gradient of its 4 pixels is the pooled gradient gp
// [N][H/2][W/2][C] where the window's argmax (idx, plane offset h*W + w) is
// that pixel, else 0 -- the max-pool backward, read in place -- masked by the
// ReLU recomputed from x (relu).
struct PoolSrc {
  // a row is 4 pixels (6 loads): fewer rows per lane, one row per step
  static constexpr int NPIX = 4, kUnroll = 1, kMinBlocks = 2, kMinRows = 4;
  struct V {
    float4 g[4], x[4];
    int64_t base;
  };
  const float* gp;
  const int32_t* idx;
  const float* x;
  FastDiv ow_div, oh_div;  // pooled width, pooled height
  int W, GT, relu;
  __device__ __forceinline__ int64_t off(const V& v, int k, int cg) const {
    return (v.base + (k >> 1) * (int64_t)W + (k & 1)) * GT + cg;
  }
  __device__ __forceinline__ V load(int64_t q, int cg, const BwdCtx& c) const {
    V v;
    const uint32_t t = ow_div.div((uint32_t)q);  // n * OH + oh
    const uint32_t ow = (uint32_t)q - t * ow_div.d;
    const uint32_t oh = t - oh_div.div(t) * oh_div.d;
    v.base = (int64_t)t * 2 * W + 2 * ow;  // pixel (n, 2 oh, 2 ow)
    const float4 g4 = reinterpret_cast<const float4*>(gp)[q * GT + cg];
    const int4 ix = reinterpret_cast<const int4*>(idx)[q * GT + cg];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v.x[k] = reinterpret_cast<const float4*>(x)[off(v, k, cg)];
      const int me = (int)((2 * oh + (k >> 1)) * W + 2 * ow + (k & 1));
      v.g[k] = make_float4(ix.x == me ? g4.x : 0.0f, ix.y == me ? g4.y : 0.0f, ix.z == me ? g4.z : 0.0f,
                           ix.w == me ? g4.w : 0.0f);
      if (relu) relu_mask_from_x(v.g[k], v.x[k], c);
    }
    return v;
  }
};

template <class S>
struct ColBnBwdF {  // a += g, b += g * x_hat
  S src;
  const float *mean, *invstd, *gamma, *beta;
  static constexpr int kUnroll = S::kUnroll, kMinBlocks = S::kMinBlocks, kMinRows = S::kMinRows;
  using Ctx = BwdCtx;
  using V = typename S::V;
  __device__ __forceinline__ Ctx ctx(int c0) const { return bwd_ctx(c0, mean, invstd, gamma, beta, nullptr); }
  __device__ __forceinline__ V load(int64_t p, int cg, const Ctx& c) const { return src.load(p, cg, c); }
  __device__ __forceinline__ void use(int64_t, int, const V& v, const Ctx& c, double (&a)[4], double (&b)[4]) const {
#pragma unroll
    for (int k = 0; k < S::NPIX; ++k) {
      const float4 g = v.g[k], x = v.x[k];
      a[0] += g.x, a[1] += g.y, a[2] += g.z, a[3] += g.w;
      b[0] += (double)g.x * ((x.x - c.mu[0]) * c.is[0]);
      b[1] += (double)g.y * ((x.y - c.mu[1]) * c.is[1]);
      b[2] += (double)g.z * ((x.z - c.mu[2]) * c.is[2]);
      b[3] += (double)g.w * ((x.w - c.mu[3]) * c.is[3]);
    }
  }
};

// dx = coef0 * (g - coef1 - x_hat * coef2) (the NCHW backward's formula),
// stored; a += dx (the gradient of a bias added before the BatchNorm)
template <class S>
struct ColBnBwdApplyF {
  S src;
  const float *mean, *invstd, *gamma, *beta, *coef;
  float* dx;
  static constexpr int kUnroll = S::kUnroll, kMinBlocks = S::kMinBlocks, kMinRows = S::kMinRows;
  using Ctx = BwdCtx;
  using V = typename S::V;
  __device__ __forceinline__ Ctx ctx(int c0) const { return bwd_ctx(c0, mean, invstd, gamma, beta, coef); }
  __device__ __forceinline__ V load(int64_t p, int cg, const Ctx& c) const { return src.load(p, cg, c); }
  __device__ __forceinline__ void use(int64_t, int cg, const V& v, const Ctx& c, double (&a)[4],
                                      double (&)[4]) const {
#pragma unroll
    for (int k = 0; k < S::NPIX; ++k) {
      const float g[4] = {v.g[k].x, v.g[k].y, v.g[k].z, v.g[k].w};
      const float xs[4] = {v.x[k].x, v.x[k].y, v.x[k].z, v.x[k].w};
      float o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float xh = (xs[j] - c.mu[j]) * c.is[j];
        o[j] = c.k0[j] * (g[j] - c.k1[j] - xh * c.k2[j]);
        a[j] += o[j];
      }
      reinterpret_cast<float4*>(dx)[src.off(v, k, cg)] = make_float4(o[0], o[1], o[2], o[3]);
    }
  }
};

// load(p, cg) for functors without a context, load(p, cg, ctx) for the others
template <class F>
__device__ __forceinline__ auto load_of(const F& f, int64_t p, int cg, const NoCtx&) -> decltype(f.load(p, cg)) {
  return f.load(p, cg);
}
template <class F>
__device__ __forceinline__ typename F::V load_of(const F& f, int64_t p, int cg, const BwdCtx& c) {
  return f.load(p, cg, c);
}

constexpr int COL_THREADS = 256;

template <class F>
__global__ void __launch_bounds__(COL_THREADS, F::kMinBlocks) k_col_reduce(F f, int64_t P, int C, int CB, int64_t rows_per_split,
                                                            int splits, double* __restrict__ part) {
  ::tp::pdl_enter();
  extern __shared__ double sh[];  // [R][CB][2]
  const int GB = CB >> 2, R = COL_THREADS / GB;
  const int t = threadIdx.x, g = t % GB, r = t / GB;
  const int cg = blockIdx.y * GB + g;  // this thread's channel group
  const int split = blockIdx.x;
  const int64_t p0 = (int64_t)split * rows_per_split;
  const int64_t p1 = p0 + rows_per_split < P ? p0 + rows_per_split : P;
  double a[4] = {0.0, 0.0, 0.0, 0.0}, b[4] = {0.0, 0.0, 0.0, 0.0};
  if (r < R) {
    const typename F::Ctx cx = f.ctx(4 * cg);
    int64_t p = p0 + r;
    // U rows per step: all their loads are issued before any is used
    constexpr int U = F::kUnroll;
    for (; p + (U - 1) * R < p1; p += U * R) {
      typename F::V v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = load_of(f, p + u * R, cg, cx);
#pragma unroll
      for (int u = 0; u < U; ++u) f.use(p + u * R, cg, v[u], cx, a, b);
    }
    for (; p < p1; p += R) f.use(p, cg, load_of(f, p, cg, cx), cx, a, b);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sh[((int64_t)r * CB + 4 * g + j) * 2] = a[j];
      sh[((int64_t)r * CB + 4 * g + j) * 2 + 1] = b[j];
    }
  }
  __syncthreads();
  for (int c = t; c < CB; c += COL_THREADS) {
    double sa = 0.0, sb = 0.0;
    for (int k = 0; k < R; ++k) {
      sa += sh[((int64_t)k * CB + c) * 2];
      sb += sh[((int64_t)k * CB + c) * 2 + 1];
    }
    const int64_t ch = (int64_t)blockIdx.y * CB + c;
    part[(ch * splits + split) * 2] = sa;
    part[(ch * splits + split) * 2 + 1] = sb;
  }
}

// CTAs of 64 channels (all C when C <= 64 or C is not a multiple of 64) by
// row splits: ~8 CTAs per SM, each with >= kMinRows rows per row lane, so enough
// loads are in flight to cover HBM latency.
struct ColPlan {
  int splits, cb;
  int64_t rows;
  size_t part_bytes;  // C * splits * 2 doubles, rounded up to 256 bytes
};

static ColPlan col_plan(int64_t P, int C, int min_rows = 16) {
  TP_REQUIRE(C % 4 == 0 && C >= 4 && C <= 4 * COL_THREADS, "channels-last reduction needs C %% 4 == 0, C <= %d",
             4 * COL_THREADS);
  ColPlan pl;
  pl.cb = (C > 64 && C % 64 == 0) ? 64 : C;
  const int R = COL_THREADS / (pl.cb / 4);
  int64_t want = (int64_t)sm_count() * 8 / (C / pl.cb);
  if (want < 1) want = 1;
  int64_t maxs = P / ((int64_t)R * min_rows);
  if (maxs < 1) maxs = 1;
  int64_t s = want < maxs ? want : maxs;
  pl.rows = (P + s - 1) / s;
  if (pl.rows < 1) pl.rows = 1;
  pl.splits = (int)((P + pl.rows - 1) / pl.rows);
  if (pl.splits < 1) pl.splits = 1;
  pl.part_bytes = ((size_t)C * pl.splits * 2 * sizeof(double) + 255) & ~(size_t)255;
  return pl;
}

template <class F>
static void col_launch(const F& f, int64_t P, int C, const ColPlan& pl, double* part) {
  const int R = COL_THREADS / (pl.cb / 4);
  size_t shb = (size_t)R * pl.cb * 2 * sizeof(double);
  auto kfn = k_col_reduce<F>;
  TP_LAUNCH(kfn, dim3((unsigned)pl.splits, (unsigned)(C / pl.cb)), COL_THREADS, shb, f, P, C, pl.cb, pl.rows,
            pl.splits, part);
}

// ---- element-wise passes (float4 over 4 consecutive channels) ---------------------------------

// When the grid stride is a multiple of G (256 % G == 0 and the block size
// 256) every thread keeps one channel group, so its 4 channels' parameters
// are loaded once; 4 vectors per step are loaded before any is stored.
__device__ __forceinline__ float4 bn_apply4(float4 v, const float (&mu)[4], const float (&sc)[4],
                                            const float (&bs)[4], int relu) {
  float r[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    r[j] = bn_val(r[j], mu[j], sc[j], bs[j]);
    if (relu) r[j] = fmaxf(r[j], 0.0f);
  }
  return make_float4(r[0], r[1], r[2], r[3]);
}

__global__ void k_bn_apply_nhwc(const float4* __restrict__ x, const float* __restrict__ mean,
                                const float* __restrict__ invstd, const float* __restrict__ w,
                                const float* __restrict__ b, float4* __restrict__ y, int64_t n4, int G, int relu) {
  ::tp::pdl_enter();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (stride % G == 0) {
    const int c = 4 * (int)(i % G);
    float mu[4], sc[4], bs[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      mu[j] = mean[c + j];
      sc[j] = invstd[c + j] * (w ? w[c + j] : 1.0f);
      bs[j] = b ? b[c + j] : 0.0f;
    }
    for (; i + 3 * stride < n4; i += 4 * stride) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = x[i + u * stride];
#pragma unroll
      for (int u = 0; u < 4; ++u) y[i + u * stride] = bn_apply4(v[u], mu, sc, bs, relu);
    }
    for (; i < n4; i += stride) y[i] = bn_apply4(x[i], mu, sc, bs, relu);
    return;
  }
  for (; i < n4; i += stride) {
    const int c = 4 * (int)(i % G);
    float mu[4], sc[4], bs[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      mu[j] = mean[c + j];
      sc[j] = invstd[c + j] * (w ? w[c + j] : 1.0f);
      bs[j] = b ? b[c + j] : 0.0f;
    }
    y[i] = bn_apply4(x[i], mu, sc, bs, relu);
  }
}

// BatchNorm apply (+ReLU) fused with the 2x2 / stride-2 max-pool that follows
// it: one thread per (pooled pixel, channel group) computes the 4 window
// values with bn_apply4 and keeps their maximum and its plane offset h*W + w
// (strict >, row-major window order: k_maxpool2x2_nhwc_fwd's rule), so the
// full-size activation is written only when a is given.
struct PoolFwd {
  const float4* x;
  float4* y;
  int4* idx;
  float4* a;
  FastDiv ow_div, oh_div;
  int W, G, relu;
  __device__ __forceinline__ void run(uint32_t q, int g, const float (&mu)[4], const float (&sc)[4],
                                      const float (&bs)[4]) const {
    const uint32_t t = ow_div.div(q);  // n * OH + oh
    const uint32_t ow = q - t * ow_div.d;
    const uint32_t oh = t - oh_div.div(t) * oh_div.d;
    const int64_t base = (int64_t)t * 2 * W + 2 * ow;
    float4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = x[(base + (k >> 1) * (int64_t)W + (k & 1)) * G + g];
    float m[4] = {-3.402823e+38f, -3.402823e+38f, -3.402823e+38f, -3.402823e+38f};
    int mi[4] = {-1, -1, -1, -1};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 r = bn_apply4(v[k], mu, sc, bs, relu);
      if (a) a[(base + (k >> 1) * (int64_t)W + (k & 1)) * G + g] = r;
      const float rs[4] = {r.x, r.y, r.z, r.w};
      const int me = (int)((2 * oh + (k >> 1)) * W + 2 * ow + (k & 1));
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (rs[j] > m[j]) {
          m[j] = rs[j];
          mi[j] = me;
        }
    }
    y[(int64_t)q * G + g] = make_float4(m[0], m[1], m[2], m[3]);
    idx[(int64_t)q * G + g] = make_int4(mi[0], mi[1], mi[2], mi[3]);
  }
};

__device__ __forceinline__ void bn_params4(int c, const float* mean, const float* invstd, const float* w,
                                           const float* b, float (&mu)[4], float (&sc)[4], float (&bs)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    mu[j] = mean[c + j];
    sc[j] = invstd[c + j] * (w ? w[c + j] : 1.0f);
    bs[j] = b ? b[c + j] : 0.0f;
  }
}

__global__ void __launch_bounds__(256) k_bn_pool_nhwc(PoolFwd f, const float* __restrict__ mean,
                                                      const float* __restrict__ invstd, const float* __restrict__ w,
                                                      const float* __restrict__ b, int64_t n4) {
  ::tp::pdl_enter();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  float mu[4], sc[4], bs[4];
  if (stride % f.G == 0) {  // one channel group per thread: parameters loaded once
    const int g = (int)(i % f.G);
    bn_params4(4 * g, mean, invstd, w, b, mu, sc, bs);
    for (; i < n4; i += stride) f.run((uint32_t)(i / f.G), g, mu, sc, bs);
    return;
  }
  for (; i < n4; i += stride) {
    const int g = (int)(i % f.G);
    bn_params4(4 * g, mean, invstd, w, b, mu, sc, bs);
    f.run((uint32_t)(i / f.G), g, mu, sc, bs);
  }
}

// 2x2 windows, stride 2: one thread per (n, oh, ow, 4 channels).  idx holds the
// plane offset h*W + w of the maximum (the NCHW kernels' index), visiting the
// window row-major with strict >.
__global__ void k_maxpool2x2_nhwc_fwd(const float4* __restrict__ x, float4* __restrict__ y, int4* __restrict__ idx,
                                      int64_t n4, int H, int W, int G) {
  ::tp::pdl_enter();
  const int OH = H >> 1, OW = W >> 1;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    const int g = (int)(i % G);
    int64_t t = i / G;
    const int ow = (int)(t % OW);
    t /= OW;
    const int oh = (int)(t % OH);
    const int64_t n = t / OH;
    float m[4] = {-3.402823e+38f, -3.402823e+38f, -3.402823e+38f, -3.402823e+38f};
    int mi[4] = {-1, -1, -1, -1};
#pragma unroll
    for (int kh = 0; kh < 2; ++kh)
#pragma unroll
      for (int kw = 0; kw < 2; ++kw) {
        const int h = 2 * oh + kh, w = 2 * ow + kw;
        float4 v = x[((n * H + h) * W + w) * G + g];
        float vs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (vs[j] > m[j]) {
            m[j] = vs[j];
            mi[j] = h * W + w;
          }
      }
    y[i] = make_float4(m[0], m[1], m[2], m[3]);
    if (idx) idx[i] = make_int4(mi[0], mi[1], mi[2], mi[3]);
  }
}

__global__ void k_maxpool2x2_nhwc_bwd(const float4* __restrict__ gy, const int4* __restrict__ idx,
                                      float4* __restrict__ gx, int64_t n4, int H, int W, int G) {
  ::tp::pdl_enter();
  const int OH = H >> 1, OW = W >> 1;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    const int g = (int)(i % G);
    int64_t t = i / G;
    const int ow = (int)(t % OW);
    t /= OW;
    const int oh = (int)(t % OH);
    const int64_t n = t / OH;
    float4 v = gy[i];
    int4 ix = idx[i];
#pragma unroll
    for (int kh = 0; kh < 2; ++kh)
#pragma unroll
      for (int kw = 0; kw < 2; ++kw) {
        const int h = 2 * oh + kh, w = 2 * ow + kw, me = h * W + w;
        gx[((n * H + h) * W + w) * G + g] =
            make_float4(ix.x == me ? v.x : 0.0f, ix.y == me ? v.y : 0.0f, ix.z == me ? v.z : 0.0f,
                        ix.w == me ? v.w : 0.0f);
      }
  }
}

// NCHW [N][C][H][W] -> channels-last [N][H][W][Cp], channels C..Cp-1 zero.
__global__ void k_nchw_to_nhwc(const float* __restrict__ x, float* __restrict__ y, int64_t N, int C, int64_t HW,
                               int Cp) {
  ::tp::pdl_enter();
  int64_t total = N * HW * Cp;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    const int c = (int)(i % Cp);
    const int64_t t = i / Cp, p = t % HW, n = t / HW;
    y[i] = c < C ? x[(n * C + c) * HW + p] : 0.0f;
  }
}

// [N][C][HW] <-> [N][HW][C] through 32 x 32 shared-memory tiles (both sides
// coalesced).  grid (ceil(HW/32), ceil(C/32), N), block (32, 8).
template <bool TO_NHWC>
__global__ void k_transpose_cs(const float* __restrict__ in, float* __restrict__ out, int64_t C, int64_t HW) {
  ::tp::pdl_enter();
  __shared__ float t[32][33];
  const int64_t n = blockIdx.z, p0 = (int64_t)blockIdx.x * 32, c0 = (int64_t)blockIdx.y * 32;
  const float* src = in + n * C * HW;
  float* dst = out + n * C * HW;
  for (int j = threadIdx.y; j < 32; j += 8) {
    if (TO_NHWC) {  // read rows of C: in[c][p]
      const int64_t c = c0 + j, p = p0 + threadIdx.x;
      t[j][threadIdx.x] = (c < C && p < HW) ? src[c * HW + p] : 0.0f;
    } else {  // read rows of HW: in[p][c]
      const int64_t p = p0 + j, c = c0 + threadIdx.x;
      t[j][threadIdx.x] = (c < C && p < HW) ? src[p * C + c] : 0.0f;
    }
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += 8) {
    if (TO_NHWC) {  // write out[p][c]
      const int64_t p = p0 + j, c = c0 + threadIdx.x;
      if (c < C && p < HW) dst[p * C + c] = t[threadIdx.x][j];
    } else {  // write out[c][p]
      const int64_t c = c0 + j, p = p0 + threadIdx.x;
      if (c < C && p < HW) dst[c * HW + p] = t[threadIdx.x][j];
    }
  }
}

// The same with 16-byte accesses on both sides (C % 4 == 0, HW % 4 == 0, both
// buffers 16-byte aligned): a 32-channel x 64-pixel tile per CTA, read as
// float4 along the contiguous dimension of `in`, written as float4 along the
// contiguous dimension of `out` through a padded shared-memory tile.
// grid (ceil(HW/64), ceil(C/32), N), 256 threads.
template <bool TO_NHWC>
__global__ void __launch_bounds__(256) k_transpose_cs4(const float* __restrict__ in, float* __restrict__ out,
                                                       int64_t C, int64_t HW) {
  ::tp::pdl_enter();
  __shared__ float t[32][65];  // [channel][pixel]
  const int64_t n = blockIdx.z, p0 = (int64_t)blockIdx.x * 64, c0 = (int64_t)blockIdx.y * 32;
  const float* src = in + n * C * HW;
  float* dst = out + n * C * HW;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int e = threadIdx.x + 256 * j;  // 512 float4 per tile
    if (TO_NHWC) {  // in[c][p]: 32 rows of 16 float4
      const int c = e >> 4, q = (e & 15) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c0 + c < C && p0 + q < HW) v = *reinterpret_cast<const float4*>(src + (c0 + c) * HW + p0 + q);
      t[c][q] = v.x, t[c][q + 1] = v.y, t[c][q + 2] = v.z, t[c][q + 3] = v.w;
    } else {  // in[p][c]: 64 rows of 8 float4
      const int p = e >> 3, q = (e & 7) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (p0 + p < HW && c0 + q < C) v = *reinterpret_cast<const float4*>(src + (p0 + p) * C + c0 + q);
      t[q][p] = v.x, t[q + 1][p] = v.y, t[q + 2][p] = v.z, t[q + 3][p] = v.w;
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int e = threadIdx.x + 256 * j;
    if (TO_NHWC) {  // out[p][c]: 64 rows of 8 float4
      const int p = e >> 3, q = (e & 7) * 4;
      if (p0 + p < HW && c0 + q < C)
        *reinterpret_cast<float4*>(dst + (p0 + p) * C + c0 + q) = make_float4(t[q][p], t[q + 1][p], t[q + 2][p], t[q + 3][p]);
    } else {  // out[c][p]: 32 rows of 16 float4
      const int c = e >> 4, q = (e & 15) * 4;
      if (c0 + c < C && p0 + q < HW)
        *reinterpret_cast<float4*>(dst + (c0 + c) * HW + p0 + q) = make_float4(t[c][q], t[c][q + 1], t[c][q + 2], t[c][q + 3]);
    }
  }
}

void transpose_nchw_nhwc(const float* in, float* out, int64_t N, int64_t C, int64_t HW, bool to_nhwc) {
  if (N == 0 || C == 0 || HW == 0) return;
  if (C % 4 == 0 && HW % 4 == 0 && (((uintptr_t)in | (uintptr_t)out) & 15) == 0 && N <= 65535 &&
      (C + 31) / 32 <= 65535) {
    dim3 grid((unsigned)((HW + 63) / 64), (unsigned)((C + 31) / 32), (unsigned)N);
    if (to_nhwc) TP_LAUNCH(k_transpose_cs4<true>, grid, 256, 0, in, out, C, HW);
    else TP_LAUNCH(k_transpose_cs4<false>, grid, 256, 0, in, out, C, HW);
    return;
  }
  TP_REQUIRE(N <= 65535 && (C + 31) / 32 <= 65535, "layout transpose: tensor too large for the grid");
  dim3 grid((unsigned)((HW + 31) / 32), (unsigned)((C + 31) / 32), (unsigned)N), block(32, 8);
  if (to_nhwc) TP_LAUNCH(k_transpose_cs<true>, grid, block, 0, in, out, C, HW);
  else TP_LAUNCH(k_transpose_cs<false>, grid, block, 0, in, out, C, HW);
}

static void check_vec(const void* p, const char* what) {
  TP_REQUIRE(((uintptr_t)p & 15) == 0, "%s: channels-last buffers must be 16-byte aligned", what);
}

// The two passes of the BatchNorm backward over `rows` rows of source S
// (M values per channel): sums of g and g*x_hat, the per-channel
// coefficients (and dgamma, dbeta), then dx and its per-channel sum.
template <class S>
static void bn_backward_cols(const S& src, int64_t rows, int64_t M, int64_t C, const float* w, const float* b,
                             const float* mean, const float* invstd, float* dx, float* dw, float* db,
                             float* dx_sum) {
  ColPlan pl = col_plan(rows, (int)C, S::kMinRows);
  char* ws = (char*)scratch(2 * pl.part_bytes + (((size_t)C * 3 * sizeof(float) + 255) & ~(size_t)255));
  double* part = (double*)ws;
  double* part2 = (double*)(ws + pl.part_bytes);
  float* coef = (float*)(ws + 2 * pl.part_bytes);
  col_launch(ColBnBwdF<S>{src, mean, invstd, w, b}, rows, (int)C, pl, part);
  TP_LAUNCH(k_col_bn_bwd_finish, finish_grid(C), 256, 0, part, C, pl.splits, (double)M, w, invstd, coef, dw, db);
  col_launch(ColBnBwdApplyF<S>{src, mean, invstd, w, b, coef, dx}, rows, (int)C, pl, part2);
  if (dx_sum) TP_LAUNCH(k_col_sum_finish, finish_grid(C), 256, 0, part2, C, pl.splits, dx_sum);
}

}  // namespace tp

using namespace tp;

extern "C" {

TP_API int tpk_bn_train_nhwc(const float* x, const float* w, const float* b, float* running_mean,
                             float* running_var, float* y, float* save_mean, float* save_invstd, int64_t P, int64_t C,
                             float eps, float momentum, int relu) {
  return guard([&] {
    TP_REQUIRE(P > 1, "batch_norm training needs more than one value per channel");
    check_vec(x, "batch_norm");
    check_vec(y, "batch_norm");
    ColPlan pl = col_plan(P, (int)C);
    double* part = (double*)scratch(pl.part_bytes);
    col_launch(ColStatsF{x, (int)(C / 4)}, P, (int)C, pl, part);
    TP_LAUNCH(k_col_bn_finish, finish_grid(C), 256, 0, part, C, pl.splits, (double)P, eps, momentum, save_mean,
              save_invstd, running_mean, running_var);
    int64_t n4 = P * C / 4;
    unsigned grid = (unsigned)((n4 + 255) / 256 < (int64_t)sm_count() * 8 ? (n4 + 255) / 256 : sm_count() * 8);
    TP_LAUNCH(k_bn_apply_nhwc, grid, 256, 0, reinterpret_cast<const float4*>(x), save_mean,
              save_invstd, w, b, reinterpret_cast<float4*>(y), n4, (int)(C / 4), relu ? 1 : 0);
  });
}

TP_API int tpk_bn_train_pool_nhwc(const float* x, const float* w, const float* b, float* running_mean,
                                  float* running_var, float* y, int32_t* idx, float* a, float* save_mean,
                                  float* save_invstd, int64_t N, int64_t H, int64_t W, int64_t C, float eps,
                                  float momentum, int relu) {
  return guard([&] {
    const int64_t P = N * H * W;
    TP_REQUIRE(P > 1, "batch_norm training needs more than one value per channel");
    TP_REQUIRE(H % 2 == 0 && W % 2 == 0 && C % 4 == 0 && P * C / 16 < ((int64_t)1 << 31),
               "batch_norm + 2x2 max-pool (channels-last) needs even H, W, C %% 4 == 0 and fewer than 2^31 "
               "pooled vectors");
    check_vec(x, "batch_norm");
    check_vec(y, "max_pool2d");
    check_vec(idx, "max_pool2d");
    if (a) check_vec(a, "batch_norm");
    ColPlan pl = col_plan(P, (int)C);
    double* part = (double*)scratch(pl.part_bytes);
    col_launch(ColStatsF{x, (int)(C / 4)}, P, (int)C, pl, part);
    TP_LAUNCH(k_col_bn_finish, finish_grid(C), 256, 0, part, C, pl.splits, (double)P, eps, momentum, save_mean,
              save_invstd, running_mean, running_var);
    const int64_t n4 = P * C / 16;
    unsigned grid = (unsigned)((n4 + 255) / 256 < (int64_t)sm_count() * 8 ? (n4 + 255) / 256 : sm_count() * 8);
    PoolFwd f{reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), reinterpret_cast<int4*>(idx),
              reinterpret_cast<float4*>(a), fast_div((uint32_t)(W / 2)), fast_div((uint32_t)(H / 2)), (int)W,
              (int)(C / 4), relu ? 1 : 0};
    TP_LAUNCH(k_bn_pool_nhwc, grid, 256, 0, f, save_mean, save_invstd, w, b, n4);
  });
}

TP_API int tpk_bn_backward_nhwc(const float* dy, const float* x, const float* relu_src, const float* w,
                                const float* mean, const float* invstd, float* dx, float* dw, float* db,
                                float* dx_sum, int64_t P, int64_t C) {
  return guard([&] {
    check_vec(dy, "batch_norm backward");
    check_vec(x, "batch_norm backward");
    check_vec(dx, "batch_norm backward");
    if (relu_src) check_vec(relu_src, "batch_norm backward");
    bn_backward_cols(PixSrc{dy, x, relu_src, (int)(C / 4), 0}, P, P, C, w, nullptr, mean, invstd, dx, dw, db,
                     dx_sum);
  });
}

TP_API int tpk_bn_backward_fused_nhwc(const float* g, const int32_t* idx, const float* x, const float* w,
                                      const float* b, const float* mean, const float* invstd, float* dx, float* dw,
                                      float* db, float* dx_sum, int64_t N, int64_t H, int64_t W, int64_t C,
                                      int relu) {
  return guard([&] {
    check_vec(g, "batch_norm backward");
    check_vec(x, "batch_norm backward");
    check_vec(dx, "batch_norm backward");
    const int64_t P = N * H * W;
    if (!idx) {
      bn_backward_cols(PixSrc{g, x, nullptr, (int)(C / 4), relu ? 1 : 0}, P, P, C, w, b, mean, invstd, dx, dw, db,
                       dx_sum);
      return;
    }
    check_vec(idx, "batch_norm backward");
    TP_REQUIRE(H % 2 == 0 && W % 2 == 0 && P < ((int64_t)1 << 31),
               "batch_norm backward through a 2x2 max-pool needs even H, W and N*H*W < 2^31");
    PoolSrc src{g, idx, x, fast_div((uint32_t)(W / 2)), fast_div((uint32_t)(H / 2)), (int)W, (int)(C / 4),
                relu ? 1 : 0};
    bn_backward_cols(src, P / 4, P, C, w, b, mean, invstd, dx, dw, db, dx_sum);
  });
}

TP_API int tpk_channel_sum_nhwc(const float* x, int64_t P, int64_t C, float* out) {
  return guard([&] {
    check_vec(x, "channel sum");
    ColPlan pl = col_plan(P, (int)C);
    double* part = (double*)scratch(pl.part_bytes);
    col_launch(ColSumF{x, (int)(C / 4)}, P, (int)C, pl, part);
    TP_LAUNCH(k_col_sum_finish, finish_grid(C), 256, 0, part, C, pl.splits, out);
  });
}

TP_API int tpk_maxpool2x2_nhwc_fwd(const float* x, float* y, int32_t* idx, int64_t N, int64_t H, int64_t W,
                                   int64_t C) {
  return guard([&] {
    TP_REQUIRE(H % 2 == 0 && W % 2 == 0 && C % 4 == 0 && H * W < ((int64_t)1 << 31),
               "2x2 max-pool (channels-last) needs even H, W and C %% 4 == 0");
    check_vec(x, "max_pool2d");
    check_vec(y, "max_pool2d");
    if (idx) check_vec(idx, "max_pool2d");
    int64_t n4 = N * (H / 2) * (W / 2) * C / 4;
    if (n4 == 0) return;
    TP_LAUNCH(k_maxpool2x2_nhwc_fwd, grid_for(n4, 256), 256, 0, reinterpret_cast<const float4*>(x),
              reinterpret_cast<float4*>(y), reinterpret_cast<int4*>(idx), n4, (int)H, (int)W, (int)(C / 4));
  });
}

TP_API int tpk_maxpool2x2_nhwc_bwd(const float* dy, const int32_t* idx, float* dx, int64_t N, int64_t H, int64_t W,
                                   int64_t C) {
  return guard([&] {
    TP_REQUIRE(H % 2 == 0 && W % 2 == 0 && C % 4 == 0 && H * W < ((int64_t)1 << 31),
               "2x2 max-pool (channels-last) needs even H, W and C %% 4 == 0");
    check_vec(dy, "max_pool2d backward");
    check_vec(idx, "max_pool2d backward");
    check_vec(dx, "max_pool2d backward");
    int64_t n4 = N * (H / 2) * (W / 2) * C / 4;
    if (n4 == 0) return;
    TP_LAUNCH(k_maxpool2x2_nhwc_bwd, grid_for(n4, 256), 256, 0, reinterpret_cast<const float4*>(dy),
              reinterpret_cast<const int4*>(idx), reinterpret_cast<float4*>(dx), n4, (int)H, (int)W, (int)(C / 4));
  });
}

TP_API int tpk_nchw_to_nhwc(const float* x, float* y, int64_t N, int64_t C, int64_t H, int64_t W, int64_t Cpad) {
  return guard([&] {
    TP_REQUIRE(Cpad >= C && C > 0, "nchw_to_nhwc: padded channel count below C");
    int64_t total = N * H * W * Cpad;
    if (total == 0) return;
    TP_LAUNCH(k_nchw_to_nhwc, grid_for(total, 256), 256, 0, x, y, N, (int)C, H * W, (int)Cpad);
  });
}

}  // extern "C"
