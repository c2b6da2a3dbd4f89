// Max pooling: forward (optionally writing the argmax index) and backward.
//
// Reference: max_pool2d.wgsl:22-49 (one thread per output, init -3.402823e38,
// strict >, padded taps skipped).  The reference registers no autograd node for
// max-pool (python/torch/tensor_nn_ops.py:57-72), so gradients stop there; the
// index output and the backward below are new (PyTorch's rule: the gradient of
// each window goes to its first maximum).
#include <cuda_runtime.h>

#include "tp_core.h"
#include "tp_launch.h"

namespace tp {

__global__ void k_maxpool_fwd(const float* __restrict__ x, float* __restrict__ y, int32_t* __restrict__ idx,
                              PoolGeom g, int64_t total) {
  ::tp::pdl_enter();
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    int64_t ow = i % g.OW, oh = (i / g.OW) % g.OH, bc = i / (g.OW * g.OH);
    const float* xp = x + bc * g.H * g.W;
    float m = -3.402823e+38f;
    int32_t mi = -1;
    for (int kh = 0; kh < g.KH; ++kh) {
      int64_t ih = oh * g.SH + (int64_t)kh * g.DH - g.PH;
      if (ih < 0 || ih >= g.H) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        int64_t iw = ow * g.SW + (int64_t)kw * g.DW - g.PW;
        if (iw < 0 || iw >= g.W) continue;
        float v = xp[ih * g.W + iw];
        if (v > m) {
          m = v;
          mi = (int32_t)(ih * g.W + iw);
        }
      }
    }
    y[i] = m;
    if (idx) idx[i] = mi;
  }
}

// One thread per input element gathers the gradients of every window that
// chose it, visiting windows in increasing output order (the order the CPU
// oracle accumulates in), so overlapping windows sum identically.
__global__ void k_maxpool_bwd(const float* __restrict__ gy, const int32_t* __restrict__ idx, float* __restrict__ gx,
                              PoolGeom g, int64_t total) {
  ::tp::pdl_enter();
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    int64_t iw = i % g.W, ih = (i / g.W) % g.H, bc = i / (g.W * g.H);
    int32_t me = (int32_t)(ih * g.W + iw);
    const float* gyp = gy + bc * g.OH * g.OW;
    const int32_t* ip = idx + bc * g.OH * g.OW;
    float acc = 0.0f;
    for (int kh = g.KH - 1; kh >= 0; --kh) {
      int64_t t = ih + g.PH - (int64_t)kh * g.DH;
      if (t < 0 || t % g.SH) continue;
      int64_t oh = t / g.SH;
      if (oh >= g.OH) continue;
      for (int kw = g.KW - 1; kw >= 0; --kw) {
        int64_t u = iw + g.PW - (int64_t)kw * g.DW;
        if (u < 0 || u % g.SW) continue;
        int64_t ow = u / g.SW;
        if (ow >= g.OW) continue;
        int64_t o = oh * g.OW + ow;
        if (ip[o] == me) acc += gyp[o];
      }
    }
    gx[i] = acc;
  }
}

// poolingOps.ts:18-48 argument handling: kernel [kh,kw?], stride defaults to
// the kernel, padding / dilation default 0 / 1, second value defaults to first.
static PoolGeom pool_geom(const Tensor& x, const int64_t* k, int nk, const int64_t* s, int ns, const int64_t* p,
                          int np, const int64_t* d, int nd) {
  TP_REQUIRE(x.ndim == 4, "max_pool2d expects an NCHW tensor, got rank %d", x.ndim);
  TP_REQUIRE(nk >= 1, "max_pool2d: kernel_size is empty");
  PoolGeom g;
  g.N = x.shape[0];
  g.C = x.shape[1];
  g.H = x.shape[2];
  g.W = x.shape[3];
  g.KH = (int)k[0];
  g.KW = (int)(nk > 1 ? k[1] : k[0]);
  g.SH = (int)(ns > 0 ? s[0] : g.KH);
  g.SW = (int)(ns > 1 ? s[1] : (ns > 0 ? s[0] : g.KW));
  g.PH = (int)(np > 0 ? p[0] : 0);
  g.PW = (int)(np > 1 ? p[1] : g.PH);
  g.DH = (int)(nd > 0 ? d[0] : 1);
  g.DW = (int)(nd > 1 ? d[1] : g.DH);
  TP_REQUIRE(g.KH > 0 && g.KW > 0 && g.SH > 0 && g.SW > 0 && g.DH > 0 && g.DW > 0 && g.PH >= 0 && g.PW >= 0,
             "max_pool2d: invalid window");
  g.OH = (g.H + 2 * g.PH - ((int64_t)g.DH * (g.KH - 1) + 1)) / g.SH + 1;
  g.OW = (g.W + 2 * g.PW - ((int64_t)g.DW * (g.KW - 1) + 1)) / g.SW + 1;
  TP_REQUIRE(g.OH > 0 && g.OW > 0, "max_pool2d: output would be empty");
  return g;
}

// 2x2 windows, stride 2, no padding, even H and W (every VGG pool): windows
// tile the input exactly, so each input element belongs to one window.  One
// thread per output reads its window as two 8-byte rows; the backward writes
// the whole window (the gradient at the recorded maximum, zero elsewhere).
// Same visiting order and strict > as the general kernel.
__global__ void k_maxpool2x2_fwd(const float* __restrict__ x, float* __restrict__ y, int32_t* __restrict__ idx,
                                 int64_t planes, int H, int W) {
  ::tp::pdl_enter();
  const int OH = H >> 1, OW = W >> 1;
  const int64_t total = planes * OH * OW;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    int ow = (int)(i % OW);
    int64_t t = i / OW;
    int oh = (int)(t % OH);
    int64_t bc = t / OH;
    const float* xp = x + bc * H * W;
    int r0 = 2 * oh * W + 2 * ow;
    float2 a = *reinterpret_cast<const float2*>(xp + r0);
    float2 b = *reinterpret_cast<const float2*>(xp + r0 + W);
    float m = -3.402823e+38f;
    int mi = -1;
    if (a.x > m) { m = a.x; mi = r0; }
    if (a.y > m) { m = a.y; mi = r0 + 1; }
    if (b.x > m) { m = b.x; mi = r0 + W; }
    if (b.y > m) { m = b.y; mi = r0 + W + 1; }
    y[i] = m;
    if (idx) idx[i] = mi;
  }
}

__global__ void k_maxpool2x2_bwd(const float* __restrict__ gy, const int32_t* __restrict__ idx,
                                 float* __restrict__ gx, int64_t planes, int H, int W) {
  ::tp::pdl_enter();
  const int OH = H >> 1, OW = W >> 1;
  const int64_t total = planes * OH * OW;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    int ow = (int)(i % OW);
    int64_t t = i / OW;
    int oh = (int)(t % OH);
    int64_t bc = t / OH;
    float g = gy[i];
    int j = idx[i];
    int r0 = 2 * oh * W + 2 * ow;
    float* gp = gx + bc * H * W;
    *reinterpret_cast<float2*>(gp + r0) = make_float2(j == r0 ? g : 0.0f, j == r0 + 1 ? g : 0.0f);
    *reinterpret_cast<float2*>(gp + r0 + W) = make_float2(j == r0 + W ? g : 0.0f, j == r0 + W + 1 ? g : 0.0f);
  }
}

static bool is_2x2(const PoolGeom& g) {
  return g.KH == 2 && g.KW == 2 && g.SH == 2 && g.SW == 2 && g.PH == 0 && g.PW == 0 && g.DH == 1 && g.DW == 1 &&
         (g.H % 2) == 0 && (g.W % 2) == 0 && g.H * g.W <= (int64_t)1 << 30;
}

void launch_maxpool_fwd(const float* x, float* y, int32_t* idx, const PoolGeom& g) {
  int64_t total = g.N * g.C * g.OH * g.OW;
  if (total == 0) return;
  if (is_2x2(g) && ((uintptr_t)x & 7) == 0)
    TP_LAUNCH(k_maxpool2x2_fwd, grid_for(total, 256), 256, 0, x, y, idx, g.N * g.C, (int)g.H, (int)g.W);
  else
    TP_LAUNCH(k_maxpool_fwd, grid_for(total, 256), 256, 0, x, y, idx, g, total);
}

void launch_maxpool_bwd(const float* gy, const int32_t* idx, float* gx, const PoolGeom& g) {
  int64_t total = g.N * g.C * g.H * g.W;
  if (total == 0) return;
  if (is_2x2(g) && ((uintptr_t)gx & 7) == 0)
    TP_LAUNCH(k_maxpool2x2_bwd, grid_for(g.N * g.C * g.OH * g.OW, 256), 256, 0, gy, idx, gx, g.N * g.C, (int)g.H,
              (int)g.W);
  else
    TP_LAUNCH(k_maxpool_bwd, grid_for(total, 256), 256, 0, gy, idx, gx, g, total);
}

}  // namespace tp

using namespace tp;

extern "C" {

TP_API int tp_max_pool2d(int64_t id, const int64_t* k, int nk, const int64_t* s, int ns, const int64_t* p, int np,
                         const int64_t* d, int nd, tp_handle* out) {
  return guard([&] {
    Tensor& x = get(id);
    PoolGeom g = pool_geom(x, k, nk, s, ns, p, np, d, nd);
    int64_t shp[4] = {g.N, g.C, g.OH, g.OW};
    Tensor y = make(shp, 4, x.dtype);
    launch_maxpool_fwd(x.f(), y.f(), nullptr, g);
    emit(y, out);
  });
}

TP_API int tp_max_pool2d_with_indices(int64_t id, const int64_t* k, int nk, const int64_t* s, int ns,
                                      const int64_t* p, int np, const int64_t* d, int nd, tp_handle* out,
                                      tp_handle* indices) {
  return guard([&] {
    Tensor& x = get(id);
    PoolGeom g = pool_geom(x, k, nk, s, ns, p, np, d, nd);
    int64_t shp[4] = {g.N, g.C, g.OH, g.OW};
    Tensor y = make(shp, 4, x.dtype);
    Tensor ix = make(shp, 4, TP_INT32, PHYS_I32);
    launch_maxpool_fwd(x.f(), y.f(), ix.i(), g);
    emit(y, out);
    emit(ix, indices);
  });
}

TP_API int tp_max_pool2d_backward(int64_t grad_out, int64_t indices, const int64_t* input_shape, const int64_t* k,
                                  int nk, const int64_t* s, int ns, const int64_t* p, int np, const int64_t* d,
                                  int nd, tp_handle* out) {
  return guard([&] {
    Tensor& gy = get(grad_out);
    Tensor& ix = get(indices);
    TP_REQUIRE(ix.phys == PHYS_I32, "max_pool2d_backward: indices must come from max_pool2d_with_indices");
    Tensor shape_only;
    shape_only.ndim = 4;
    for (int i = 0; i < 4; ++i) shape_only.shape[i] = input_shape[i];
    PoolGeom g = pool_geom(shape_only, k, nk, s, ns, p, np, d, nd);
    TP_REQUIRE(gy.numel == g.N * g.C * g.OH * g.OW && ix.numel == gy.numel,
               "max_pool2d_backward: grad/indices do not match the pooled shape");
    Tensor gx = make(input_shape, 4, gy.dtype);
    launch_maxpool_bwd(gy.f(), ix.i(), gx.f(), g);
    emit(gx, out);
  });
}

}  // extern "C"
