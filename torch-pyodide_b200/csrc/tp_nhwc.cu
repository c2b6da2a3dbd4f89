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

// Functors: ctx(c0) loads what the thread's 4 channels need once; load(i4)
// fetches the float4 operands at index i4 and use() consumes them, so the
// row loop can have several rows' loads in flight.
struct NoCtx {};

struct ColStatsF {  // a += x, b += x*x
  const float* x;
  static constexpr int kUnroll = 8;
  using Ctx = NoCtx;
  using V = float4;
  __device__ __forceinline__ Ctx ctx(int) const { return {}; }
  __device__ __forceinline__ V load(int64_t i4) const { return reinterpret_cast<const float4*>(x)[i4]; }
  __device__ __forceinline__ void use(int64_t, const V& v, const Ctx&, double (&a)[4], double (&b)[4]) const {
    a[0] += v.x, a[1] += v.y, a[2] += v.z, a[3] += v.w;
    b[0] += (double)v.x * v.x, b[1] += (double)v.y * v.y, b[2] += (double)v.z * v.z, b[3] += (double)v.w * v.w;
  }
};

struct ColSumF {  // a += x
  const float* x;
  static constexpr int kUnroll = 8;
  using Ctx = NoCtx;
  using V = float4;
  __device__ __forceinline__ Ctx ctx(int) const { return {}; }
  __device__ __forceinline__ V load(int64_t i4) const { return reinterpret_cast<const float4*>(x)[i4]; }
  __device__ __forceinline__ void use(int64_t, const V& v, const Ctx&, double (&a)[4], double (&)[4]) const {
    a[0] += v.x, a[1] += v.y, a[2] += v.z, a[3] += v.w;
  }
};

struct BwdV {
  float4 g, x;
};

__device__ __forceinline__ BwdV load_bwd(const float* dy, const float* x, const float* relu_src, int64_t i4) {
  BwdV v;
  v.g = reinterpret_cast<const float4*>(dy)[i4];
  v.x = reinterpret_cast<const float4*>(x)[i4];
  if (relu_src) {
    float4 r = reinterpret_cast<const float4*>(relu_src)[i4];
    if (!(r.x > 0.0f)) v.g.x = 0.0f;
    if (!(r.y > 0.0f)) v.g.y = 0.0f;
    if (!(r.z > 0.0f)) v.g.z = 0.0f;
    if (!(r.w > 0.0f)) v.g.w = 0.0f;
  }
  return v;
}

struct ColBnBwdF {  // g = dy masked by relu_src > 0; a += g, b += g * x_hat
  const float* dy;
  const float* x;
  const float* relu_src;
  const float* mean;
  const float* invstd;
  static constexpr int kUnroll = 4;
  struct Ctx {
    float mu[4], is[4];
  };
  using V = BwdV;
  __device__ __forceinline__ Ctx ctx(int c0) const {
    Ctx c;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      c.mu[j] = mean[c0 + j];
      c.is[j] = invstd[c0 + j];
    }
    return c;
  }
  __device__ __forceinline__ V load(int64_t i4) const { return load_bwd(dy, x, relu_src, i4); }
  __device__ __forceinline__ void use(int64_t, const V& v, const Ctx& c, double (&a)[4], double (&b)[4]) const {
    a[0] += v.g.x, a[1] += v.g.y, a[2] += v.g.z, a[3] += v.g.w;
    b[0] += (double)v.g.x * ((v.x.x - c.mu[0]) * c.is[0]);
    b[1] += (double)v.g.y * ((v.x.y - c.mu[1]) * c.is[1]);
    b[2] += (double)v.g.z * ((v.x.z - c.mu[2]) * c.is[2]);
    b[3] += (double)v.g.w * ((v.x.w - c.mu[3]) * c.is[3]);
  }
};

// dx = coef0 * (g - coef1 - x_hat * coef2) (the NCHW backward's formula),
// stored; a += dx (the gradient of a bias added before the BatchNorm)
struct ColBnBwdApplyF {
  const float* dy;
  const float* x;
  const float* relu_src;
  const float* mean;
  const float* invstd;
  const float* coef;
  float* dx;
  static constexpr int kUnroll = 4;
  struct Ctx {
    float mu[4], is[4], k0[4], k1[4], k2[4];
  };
  using V = BwdV;
  __device__ __forceinline__ Ctx ctx(int c0) const {
    Ctx c;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      c.mu[j] = mean[c0 + j];
      c.is[j] = invstd[c0 + j];
      c.k0[j] = coef[(c0 + j) * 3];
      c.k1[j] = coef[(c0 + j) * 3 + 1];
      c.k2[j] = coef[(c0 + j) * 3 + 2];
    }
    return c;
  }
  __device__ __forceinline__ V load(int64_t i4) const { return load_bwd(dy, x, relu_src, i4); }
  __device__ __forceinline__ void use(int64_t i4, const V& v, const Ctx& c, double (&a)[4], double (&)[4]) const {
    const float g[4] = {v.g.x, v.g.y, v.g.z, v.g.w}, xs[4] = {v.x.x, v.x.y, v.x.z, v.x.w};
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float xh = (xs[j] - c.mu[j]) * c.is[j];
      o[j] = c.k0[j] * (g[j] - c.k1[j] - xh * c.k2[j]);
      a[j] += o[j];
    }
    reinterpret_cast<float4*>(dx)[i4] = make_float4(o[0], o[1], o[2], o[3]);
  }
};

constexpr int COL_THREADS = 256;

template <class F>
__global__ void __launch_bounds__(COL_THREADS) k_col_reduce(F f, int64_t P, int C, int CB, int64_t rows_per_split,
                                                            int splits, double* __restrict__ part) {
  extern __shared__ double sh[];  // [R][CB][2]
  const int GT = C >> 2, GB = CB >> 2, R = COL_THREADS / GB;
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
      for (int u = 0; u < U; ++u) v[u] = f.load((p + u * R) * GT + cg);
#pragma unroll
      for (int u = 0; u < U; ++u) f.use((p + u * R) * GT + cg, v[u], cx, a, b);
    }
    for (; p < p1; p += R) f.use(p * GT + cg, f.load(p * GT + cg), cx, a, b);
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
// row splits: ~8 CTAs per SM, each with >= 16 rows per row lane, so enough
// loads are in flight to cover HBM latency.
struct ColPlan {
  int splits, cb;
  int64_t rows;
  size_t part_bytes;  // C * splits * 2 doubles, rounded up to 256 bytes
};

static ColPlan col_plan(int64_t P, int C) {
  TP_REQUIRE(C % 4 == 0 && C >= 4 && C <= 4 * COL_THREADS, "channels-last reduction needs C %% 4 == 0, C <= %d",
             4 * COL_THREADS);
  ColPlan pl;
  pl.cb = (C > 64 && C % 64 == 0) ? 64 : C;
  const int R = COL_THREADS / (pl.cb / 4);
  int64_t want = (int64_t)sm_count() * 8 / (C / pl.cb);
  if (want < 1) want = 1;
  int64_t maxs = P / ((int64_t)R * 16);
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
    r[j] = (r[j] - mu[j]) * sc[j] + bs[j];
    if (relu) r[j] = fmaxf(r[j], 0.0f);
  }
  return make_float4(r[0], r[1], r[2], r[3]);
}

__global__ void k_bn_apply_nhwc(const float4* __restrict__ x, const float* __restrict__ mean,
                                const float* __restrict__ invstd, const float* __restrict__ w,
                                const float* __restrict__ b, float4* __restrict__ y, int64_t n4, int G, int relu) {
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

// 2x2 windows, stride 2: one thread per (n, oh, ow, 4 channels).  idx holds the
// plane offset h*W + w of the maximum (the NCHW kernels' index), visiting the
// window row-major with strict >.
__global__ void k_maxpool2x2_nhwc_fwd(const float4* __restrict__ x, float4* __restrict__ y, int4* __restrict__ idx,
                                      int64_t n4, int H, int W, int G) {
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

void transpose_nchw_nhwc(const float* in, float* out, int64_t N, int64_t C, int64_t HW, bool to_nhwc) {
  if (N == 0 || C == 0 || HW == 0) return;
  TP_REQUIRE(N <= 65535 && (C + 31) / 32 <= 65535, "layout transpose: tensor too large for the grid");
  dim3 grid((unsigned)((HW + 31) / 32), (unsigned)((C + 31) / 32), (unsigned)N), block(32, 8);
  if (to_nhwc) TP_LAUNCH(k_transpose_cs<true>, grid, block, 0, in, out, C, HW);
  else TP_LAUNCH(k_transpose_cs<false>, grid, block, 0, in, out, C, HW);
}

static void check_vec(const void* p, const char* what) {
  TP_REQUIRE(((uintptr_t)p & 15) == 0, "%s: channels-last buffers must be 16-byte aligned", what);
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
    col_launch(ColStatsF{x}, P, (int)C, pl, part);
    TP_LAUNCH(k_col_bn_finish, finish_grid(C), 256, 0, part, C, pl.splits, (double)P, eps, momentum, save_mean,
              save_invstd, running_mean, running_var);
    int64_t n4 = P * C / 4;
    unsigned grid = (unsigned)((n4 + 255) / 256 < (int64_t)sm_count() * 8 ? (n4 + 255) / 256 : sm_count() * 8);
    TP_LAUNCH(k_bn_apply_nhwc, grid, 256, 0, reinterpret_cast<const float4*>(x), save_mean,
              save_invstd, w, b, reinterpret_cast<float4*>(y), n4, (int)(C / 4), relu ? 1 : 0);
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
    ColPlan pl = col_plan(P, (int)C);
    char* ws = (char*)scratch(2 * pl.part_bytes + (((size_t)C * 3 * sizeof(float) + 255) & ~(size_t)255));
    double* part = (double*)ws;
    double* part2 = (double*)(ws + pl.part_bytes);
    float* coef = (float*)(ws + 2 * pl.part_bytes);
    col_launch(ColBnBwdF{dy, x, relu_src, mean, invstd}, P, (int)C, pl, part);
    TP_LAUNCH(k_col_bn_bwd_finish, finish_grid(C), 256, 0, part, C, pl.splits, (double)P, w, invstd, coef, dw, db);
    col_launch(ColBnBwdApplyF{dy, x, relu_src, mean, invstd, coef, dx}, P, (int)C, pl, part2);
    if (dx_sum) TP_LAUNCH(k_col_sum_finish, finish_grid(C), 256, 0, part2, C, pl.splits, dx_sum);
  });
}

TP_API int tpk_channel_sum_nhwc(const float* x, int64_t P, int64_t C, float* out) {
  return guard([&] {
    check_vec(x, "channel sum");
    ColPlan pl = col_plan(P, (int)C);
    double* part = (double*)scratch(pl.part_bytes);
    col_launch(ColSumF{x}, P, (int)C, pl, part);
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
