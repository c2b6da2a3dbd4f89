// Reductions, softmax family and cross-entropy.
//
// Reference: reduce_sum.wgsl / reduce_max.wgsl run a 256-wide tree per pass
// with a host readback of the scalar (reductionOps.ts:161-213); reduce_dim.wgsl
// runs one thread per output with a serial loop (:215-251); softmax.wgsl and
// log_softmax.wgsl use one thread per row and three passes.  Here:
//   * full reductions are one pass over HBM (128-bit loads, warp shuffles,
//     per-block partials, last block finishes in a fixed order) and the scalar
//     stays in HBM;
//   * reductions along the last dim use a warp (short rows) or a block (long
//     rows) per row; along other dims, a column-tiled kernel with coalesced
//     row reads and an optional deterministic split over the reduced dim;
//   * softmax / log-softmax keep the row in registers between the statistics
//     and the write (one HBM read, one write).
#include <cuda_runtime.h>

#include <mutex>

#include <cfloat>
#include <climits>
#include <cmath>

#include "tp_core.h"
#include "tp_launch.h"

namespace tp {

constexpr int RED_MAX_BLOCKS = 1024;

__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// (value, index) max with first-index tie-break; index INT_MAX marks a lane
// that saw no element.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (oi != INT_MAX && (i == INT_MAX || ov > v || (ov == v && oi < i))) {
      v = ov;
      i = oi;
    }
  }
}

// Block-wide reduction for blockDim.x a multiple of 32 (<= 1024).
template <bool MAX>
__device__ float block_reduce(float v, float* sh) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = MAX ? warp_max(v) : warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = lane < nw ? sh[lane] : (MAX ? -FLT_MAX : 0.0f);
    v = MAX ? warp_max(v) : warp_sum(v);
    if (lane == 0) sh[0] = v;
  }
  __syncthreads();
  float r = sh[0];
  __syncthreads();
  return r;
}

// ---- full reduction -----------------------------------------------------------
// ws layout: [RED_MAX_BLOCKS partial floats][uint32 ticket]
__global__ void k_reduce_all(const float* __restrict__ x, int64_t n, int mode, float* __restrict__ out,
                             float* __restrict__ partials, unsigned int* __restrict__ ticket) {
  ::tp::pdl_enter();
  __shared__ float sh[32];
  __shared__ bool last;
  const bool is_max = mode == 2;
  float acc = is_max ? -FLT_MAX : 0.0f;
  int64_t n4 = n >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 v = x4[i];
    if (is_max) acc = fmaxf(fmaxf(acc, fmaxf(v.x, v.y)), fmaxf(v.z, v.w));
    else acc += (v.x + v.y) + (v.z + v.w);
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    acc = is_max ? fmaxf(acc, x[i]) : acc + x[i];
  acc = is_max ? block_reduce<true>(acc, sh) : block_reduce<false>(acc, sh);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = acc;
    __threadfence();
    unsigned int t = atomicAdd(ticket, 1u);
    last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  float v = is_max ? -FLT_MAX : 0.0f;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
    float p = *((volatile float*)&partials[i]);
    v = is_max ? fmaxf(v, p) : v + p;
  }
  v = is_max ? block_reduce<true>(v, sh) : block_reduce<false>(v, sh);
  if (threadIdx.x == 0) {
    // mean: the f32 sum divided in f64 and rounded to f32 (reductionOps.ts:203-210)
    out[0] = (mode == 1) ? (float)((double)v / (double)n) : v;
    *ticket = 0u;  // leave the workspace ready for the next launch
  }
}

static float* g_red_ws = nullptr;

float* reduce_workspace() {
  if (!g_red_ws) {
    g_red_ws = (float*)dalloc((RED_MAX_BLOCKS + 32) * sizeof(float));
    TP_CUDA(cudaMemsetAsync(g_red_ws, 0, (RED_MAX_BLOCKS + 32) * sizeof(float), stream()));
  }
  return g_red_ws;
}

void launch_reduce_all(const float* x, int64_t n, int mode, float* out) {
  if (n == 0) {
    float v = mode == 2 ? -1.0e38f : 0.0f;
    TP_CUDA(cudaMemcpyAsync(out, &v, 4, cudaMemcpyHostToDevice, stream()));  // pageable: staged before return
    return;
  }
  float* ws = reduce_workspace();
  unsigned blocks = grid_for(n, 256, 8);
  unsigned cap = (unsigned)sm_count() * 4;
  if (blocks > cap) blocks = cap;
  if (blocks > RED_MAX_BLOCKS) blocks = RED_MAX_BLOCKS;
  TP_LAUNCH(k_reduce_all, blocks, 256, 0, x, n, mode, out, ws, (unsigned int*)(ws + RED_MAX_BLOCKS));
}

// ---- reduction along the last dim (inner == 1) ------------------------------------
// mode 0 sum, 1 mean, 2 max, 3 max+index (first index), 4 argmax (index only)
__global__ void k_reduce_rows_warp(const float* __restrict__ x, int64_t rows, int64_t red, int mode,
                                   float* __restrict__ out, int32_t* __restrict__ idx) {
  ::tp::pdl_enter();
  int lane = threadIdx.x & 31;
  int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const float* xr = x + row * red;
  if (mode <= 1) {
    float s = 0.0f;
    for (int64_t i = lane; i < red; i += 32) s += xr[i];
    s = warp_sum(s);
    if (lane == 0) out[row] = mode == 1 ? s / (float)red : s;
  } else {
    float v = -FLT_MAX;
    int vi = INT_MAX;
    for (int64_t i = lane; i < red; i += 32) {
      float t = xr[i];
      if (vi == INT_MAX || t > v) {  // increasing i per lane: strict > keeps the first
        v = t;
        vi = (int)i;
      }
    }
    warp_argmax(v, vi);
    if (lane == 0) {
      if (mode != 4) out[row] = v;
      if (idx) idx[row] = vi;
    }
  }
}

__global__ void k_reduce_rows_block(const float* __restrict__ x, int64_t rows, int64_t red, int mode,
                                    float* __restrict__ out, int32_t* __restrict__ idx) {
  ::tp::pdl_enter();
  __shared__ float shv[32];
  __shared__ int shi[32];
  int64_t row = blockIdx.x;
  const float* xr = x + row * red;
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (mode <= 1) {
    float s = 0.0f;
    if ((red & 3) == 0 && (((uintptr_t)xr) & 15) == 0) {
      const float4* x4 = reinterpret_cast<const float4*>(xr);
      for (int64_t i = threadIdx.x; i < (red >> 2); i += blockDim.x) {
        float4 v = x4[i];
        s += (v.x + v.y) + (v.z + v.w);
      }
    } else {
      for (int64_t i = threadIdx.x; i < red; i += blockDim.x) s += xr[i];
    }
    s = block_reduce<false>(s, shv);
    if (threadIdx.x == 0) out[row] = mode == 1 ? s / (float)red : s;
  } else {
    float v = -FLT_MAX;
    int vi = INT_MAX;
    if ((red & 3) == 0 && (((uintptr_t)xr) & 15) == 0) {
      // 16-byte loads; within a vector the first maximum wins (strict >)
      const float4* x4 = reinterpret_cast<const float4*>(xr);
      for (int64_t i = threadIdx.x; i < (red >> 2); i += blockDim.x) {
        const float4 q = x4[i];
        const float t[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (vi == INT_MAX || t[j] > v) {
            v = t[j];
            vi = (int)(4 * i + j);
          }
      }
    } else {
      for (int64_t i = threadIdx.x; i < red; i += blockDim.x) {
        float t = xr[i];
        if (vi == INT_MAX || t > v) {
          v = t;
          vi = (int)i;
        }
      }
    }
    warp_argmax(v, vi);
    if (lane == 0) {
      shv[w] = v;
      shi[w] = vi;
    }
    __syncthreads();
    if (w == 0) {
      v = lane < nw ? shv[lane] : -FLT_MAX;
      vi = lane < nw ? shi[lane] : INT_MAX;
      warp_argmax(v, vi);
      if (lane == 0) {
        if (mode != 4) out[row] = v;
        if (idx) idx[row] = vi;
      }
    }
  }
}

// ---- reduction along a non-last dim: x viewed as [outer, red, inner] ------------------
// grid (ceil(inner/32), outer, splits), block (32, 8).  Each split covers a
// contiguous range of the reduced dim; with splits > 1 the partials land in
// ws[split][outer*inner] and k_reduce_cols_finish combines them in order.
__global__ void k_reduce_cols(const float* __restrict__ x, int64_t outer, int64_t red, int64_t inner, int mode,
                              int splits, float* __restrict__ out, int32_t* __restrict__ idx,
                              float* __restrict__ wsv, int32_t* __restrict__ wsi) {
  ::tp::pdl_enter();
  __shared__ float shv[8][33];
  __shared__ int shi[8][33];
  int64_t col = (int64_t)blockIdx.x * 32 + threadIdx.x;
  int64_t o = blockIdx.y;
  int split = blockIdx.z;
  int64_t per = (red + splits - 1) / splits;
  int64_t r0 = split * per, r1 = r0 + per < red ? r0 + per : red;
  bool is_sum = mode <= 1;
  float acc = is_sum ? 0.0f : -FLT_MAX;
  int ai = INT_MAX;
  if (col < inner) {
    const float* base = x + o * red * inner + col;
    for (int64_t r = r0 + threadIdx.y; r < r1; r += 8) {
      float v = base[r * inner];
      if (is_sum) acc += v;
      else if (ai == INT_MAX || v > acc) {
        acc = v;
        ai = (int)r;
      }
    }
  }
  shv[threadIdx.y][threadIdx.x] = acc;
  shi[threadIdx.y][threadIdx.x] = ai;
  __syncthreads();
  if (threadIdx.y == 0 && col < inner) {
    for (int k = 1; k < 8; ++k) {
      float v = shv[k][threadIdx.x];
      int vi = shi[k][threadIdx.x];
      if (is_sum) acc += v;
      else if (vi != INT_MAX && (ai == INT_MAX || v > acc || (v == acc && vi < ai))) {
        acc = v;
        ai = vi;
      }
    }
    int64_t oi = o * inner + col;
    if (splits == 1) {
      out[oi] = (mode == 1) ? acc / (float)red : acc;
      if (idx) idx[oi] = ai;
    } else {
      wsv[(int64_t)split * outer * inner + oi] = acc;
      if (wsi) wsi[(int64_t)split * outer * inner + oi] = ai;
    }
  }
}

// inner % 4 == 0: thread x takes 4 adjacent columns (16-byte loads), rows
// step by 8 with 4 rows of loads in flight; grid (ceil(inner/128), outer,
// splits).  Same per-column combination order as k_reduce_cols.
__global__ void k_reduce_cols4(const float* __restrict__ x, int64_t outer, int64_t red, int64_t inner, int mode,
                               int splits, float* __restrict__ out, int32_t* __restrict__ idx,
                               float* __restrict__ wsv, int32_t* __restrict__ wsi) {
  ::tp::pdl_enter();
  __shared__ float4 shv[8][32];
  __shared__ int4 shi[8][32];
  const int64_t c4 = (int64_t)blockIdx.x * 32 + threadIdx.x, col = 4 * c4;
  const int64_t o = blockIdx.y;
  const int split = blockIdx.z;
  const int64_t per = (red + splits - 1) / splits;
  const int64_t r0 = split * per, r1 = r0 + per < red ? r0 + per : red;
  const bool is_sum = mode <= 1;
  float acc[4];
  int ai[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc[j] = is_sum ? 0.0f : -FLT_MAX;
    ai[j] = INT_MAX;
  }
  if (col < inner) {
    const float* base = x + o * red * inner + col;
    int64_t r = r0 + threadIdx.y;
    for (; r + 24 < r1; r += 32) {
      float4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = *reinterpret_cast<const float4*>(base + (r + 8 * u) * inner);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float t[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (is_sum) acc[j] += t[j];
          else if (ai[j] == INT_MAX || t[j] > acc[j]) {
            acc[j] = t[j];
            ai[j] = (int)(r + 8 * u);
          }
        }
      }
    }
    for (; r < r1; r += 8) {
      const float4 q = *reinterpret_cast<const float4*>(base + r * inner);
      const float t[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (is_sum) acc[j] += t[j];
        else if (ai[j] == INT_MAX || t[j] > acc[j]) {
          acc[j] = t[j];
          ai[j] = (int)r;
        }
      }
    }
  }
  shv[threadIdx.y][threadIdx.x] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  shi[threadIdx.y][threadIdx.x] = make_int4(ai[0], ai[1], ai[2], ai[3]);
  __syncthreads();
  if (threadIdx.y == 0 && col < inner) {
    for (int k = 1; k < 8; ++k) {
      const float4 qv = shv[k][threadIdx.x];
      const int4 qi = shi[k][threadIdx.x];
      const float v[4] = {qv.x, qv.y, qv.z, qv.w};
      const int vi[4] = {qi.x, qi.y, qi.z, qi.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (is_sum) acc[j] += v[j];
        else if (vi[j] != INT_MAX && (ai[j] == INT_MAX || v[j] > acc[j] || (v[j] == acc[j] && vi[j] < ai[j]))) {
          acc[j] = v[j];
          ai[j] = vi[j];
        }
      }
    }
    const int64_t oi = o * inner + col;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (col + j >= inner) break;
      if (splits == 1) {
        out[oi + j] = (mode == 1) ? acc[j] / (float)red : acc[j];
        if (idx) idx[oi + j] = ai[j];
      } else {
        wsv[(int64_t)split * outer * inner + oi + j] = acc[j];
        if (wsi) wsi[(int64_t)split * outer * inner + oi + j] = ai[j];
      }
    }
  }
}

__global__ void k_reduce_cols_finish(int64_t n, int64_t red, int mode, int splits, const float* __restrict__ wsv,
                                     const int32_t* __restrict__ wsi, float* __restrict__ out,
                                     int32_t* __restrict__ idx) {
  ::tp::pdl_enter();
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  bool is_sum = mode <= 1;
  float acc = wsv[i];
  int ai = wsi ? wsi[i] : 0;
  for (int s = 1; s < splits; ++s) {
    float v = wsv[(int64_t)s * n + i];
    if (is_sum) acc += v;
    else {
      int vi = wsi[(int64_t)s * n + i];
      if (vi != INT_MAX && (ai == INT_MAX || v > acc)) {
        acc = v;
        ai = vi;
      }
    }
  }
  out[i] = (mode == 1) ? acc / (float)red : acc;
  if (idx) idx[i] = ai;
}

// out may be null for argmax-only; idx null for value-only.
void launch_reduce_dim(const float* x, int64_t outer, int64_t red, int64_t inner, int mode, float* out,
                       int32_t* idx) {
  int64_t nout = outer * inner;
  if (nout == 0) return;
  if (inner == 1) {
    if (red <= 1024) {
      int64_t threads = nout * 32;
      TP_LAUNCH(k_reduce_rows_warp, (unsigned)((threads + 255) / 256), 256, 0, x, nout, red, mode, out, idx);
    } else {
      TP_LAUNCH(k_reduce_rows_block, (unsigned)nout, 256, 0, x, nout, red, mode, out, idx);
    }
    return;
  }
  int64_t tiles = ((inner + ((inner & 3) == 0 ? 127 : 31)) / ((inner & 3) == 0 ? 128 : 32)) * outer;
  int splits = 1;
  int64_t target = (int64_t)sm_count() * 8;
  while (tiles * splits < target && red / (splits * 2) >= 64 && splits < 64) splits *= 2;
  dim3 grid((unsigned)((inner + 31) / 32), (unsigned)outer, (unsigned)splits);
  bool need_idx = mode >= 2;
  float* wsv = nullptr;
  int32_t* wsi = nullptr;
  if (splits > 1) {
    size_t nb = (size_t)splits * nout * 4 * (need_idx ? 2 : 1);
    wsv = (float*)scratch(nb);
    if (need_idx) wsi = (int32_t*)(wsv + (size_t)splits * nout);
  }
  if ((inner & 3) == 0 && (((uintptr_t)x) & 15) == 0) {
    dim3 grid4((unsigned)((inner + 127) / 128), (unsigned)outer, (unsigned)splits);
    TP_LAUNCH(k_reduce_cols4, grid4, dim3(32, 8), 0, x, outer, red, inner, mode, splits, out, idx, wsv, wsi);
  } else {
    TP_LAUNCH(k_reduce_cols, grid, dim3(32, 8), 0, x, outer, red, inner, mode, splits, out, idx, wsv, wsi);
  }
  if (splits > 1)
    TP_LAUNCH(k_reduce_cols_finish, (unsigned)((nout + 255) / 256), 256, 0, nout, red, mode, splits, wsv, wsi,
              out, idx);
}

// ---- softmax / log-softmax along the last dim -----------------------------------------
// One block of 256 threads per row; up to 32 values per thread stay in
// registers (rows <= 8192); longer rows re-read from L2.
template <int PER, bool LOG>
__global__ void __launch_bounds__(256) k_softmax_rows(const float* __restrict__ x, float* __restrict__ y,
                                                      int64_t C) {
  ::tp::pdl_enter();
  __shared__ float sh[32];
  const float* xr = x + (int64_t)blockIdx.x * C;
  float* yr = y + (int64_t)blockIdx.x * C;
  float v[PER > 0 ? PER : 1];
  float m = -FLT_MAX;
  if (PER > 0) {
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int64_t i = threadIdx.x + (int64_t)k * 256;
      v[k] = i < C ? xr[i] : -FLT_MAX;
      m = fmaxf(m, v[k]);
    }
  } else {
    for (int64_t i = threadIdx.x; i < C; i += 256) m = fmaxf(m, xr[i]);
  }
  m = block_reduce<true>(m, sh);
  float s = 0.0f;
  if (PER > 0) {
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int64_t i = threadIdx.x + (int64_t)k * 256;
      if (i < C) {
        const float e = expf(v[k] - m);
        s += e;
        if (!LOG) v[k] = e;  // kept for the output pass: one exp per element
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < C; i += 256) s += expf(xr[i] - m);
  }
  s = block_reduce<false>(s, sh);
  // one reciprocal per thread instead of a division per element (within 2 ulp of e / s)
  const float lse = LOG ? logf(s) : 0.0f, inv = LOG ? 0.0f : 1.0f / s;
  if (PER > 0) {
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int64_t i = threadIdx.x + (int64_t)k * 256;
      if (i < C) yr[i] = LOG ? (v[k] - m) - lse : v[k] * inv;
    }
  } else {
    for (int64_t i = threadIdx.x; i < C; i += 256) yr[i] = LOG ? (xr[i] - m) - lse : expf(xr[i] - m) * inv;
  }
}

// As k_softmax_rows with 16-byte accesses: thread t owns the float4 columns
// t + 256 k (C % 4 == 0, 16-byte aligned rows).
template <int V, bool LOG>
__global__ void __launch_bounds__(256) k_softmax_rows_vec(const float4* __restrict__ x, float4* __restrict__ y,
                                                          int64_t C) {
  ::tp::pdl_enter();
  __shared__ float sh[32];
  const int64_t C4 = C >> 2;
  const float4* xr = x + (int64_t)blockIdx.x * C4;
  float4* yr = y + (int64_t)blockIdx.x * C4;
  float4 v[V];
  float m = -FLT_MAX;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int64_t i = threadIdx.x + (int64_t)k * 256;
    v[k] = i < C4 ? xr[i] : make_float4(-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX);
    m = fmaxf(m, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
  }
  m = block_reduce<true>(m, sh);
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int64_t i = threadIdx.x + (int64_t)k * 256;
    if (i < C4) {
      const float4 e = make_float4(expf(v[k].x - m), expf(v[k].y - m), expf(v[k].z - m), expf(v[k].w - m));
      s += (e.x + e.y) + (e.z + e.w);
      if (!LOG) v[k] = e;  // kept for the output pass: one exp per element
    }
  }
  s = block_reduce<false>(s, sh);
  const float lse = LOG ? logf(s) : 0.0f, inv = LOG ? 0.0f : 1.0f / s;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int64_t i = threadIdx.x + (int64_t)k * 256;
    if (i < C4) {
      if (LOG)
        yr[i] = make_float4((v[k].x - m) - lse, (v[k].y - m) - lse, (v[k].z - m) - lse, (v[k].w - m) - lse);
      else
        yr[i] = make_float4(v[k].x * inv, v[k].y * inv, v[k].z * inv, v[k].w * inv);
    }
  }
}

// Short rows (C <= 32*8): one warp per row, values in registers.
template <bool LOG>
__global__ void k_softmax_rows_warp(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int64_t C) {
  ::tp::pdl_enter();
  int lane = threadIdx.x & 31;
  int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const float* xr = x + row * C;
  float v[8];
  float m = -FLT_MAX;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    int64_t i = lane + k * 32;
    v[k] = i < C ? xr[i] : -FLT_MAX;
    m = fmaxf(m, v[k]);
  }
  m = warp_max(m);
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    if (lane + k * 32 < C) {
      const float e = expf(v[k] - m);
      s += e;
      if (!LOG) v[k] = e;
    }
  s = warp_sum(s);
  const float lse = LOG ? logf(s) : 0.0f, inv = LOG ? 0.0f : 1.0f / s;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    int64_t i = lane + k * 32;
    if (i < C) y[row * C + i] = LOG ? (v[k] - m) - lse : v[k] * inv;
  }
}

// Softmax along a non-last dim (softmax.wgsl's general mapping): one thread
// per (outer, inner) row, three passes with stride `inner`.
__global__ void k_softmax_strided(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int64_t axis,
                                  int64_t inner, int log_mode) {
  ::tp::pdl_enter();
  int64_t row = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (row >= rows) return;
  int64_t base = (row / inner) * axis * inner + (row % inner);
  float m = x[base];
  for (int64_t c = 1; c < axis; ++c) m = fmaxf(m, x[base + c * inner]);
  float s = 0.0f;
  for (int64_t c = 0; c < axis; ++c) s += expf(x[base + c * inner] - m);
  float lse = logf(s);
  for (int64_t c = 0; c < axis; ++c) {
    float t = x[base + c * inner];
    y[base + c * inner] = log_mode ? (t - m) - lse : expf(t - m) / s;
  }
}

void launch_softmax(const float* x, float* y, int64_t outer, int64_t axis, int64_t inner, bool log_mode) {
  int64_t rows = outer * inner;
  if (rows == 0 || axis == 0) return;
  if (inner != 1) {
    TP_LAUNCH(k_softmax_strided, (unsigned)((rows + 255) / 256), 256, 0, x, y, rows, axis, inner, log_mode ? 1 : 0);
    return;
  }
  if (axis <= 256) {
    unsigned blocks = (unsigned)((rows * 32 + 255) / 256);
    if (log_mode) TP_LAUNCH(k_softmax_rows_warp<true>, blocks, 256, 0, x, y, rows, axis);
    else TP_LAUNCH(k_softmax_rows_warp<false>, blocks, 256, 0, x, y, rows, axis);
    return;
  }
  if (axis % 4 == 0 && axis <= 256 * 32 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 15) == 0) {
    const float4* x4 = (const float4*)x;
    float4* y4 = (float4*)y;
#define TP_SOFTMAX_VEC(V)                                                                                   \
  if (log_mode) TP_LAUNCH((k_softmax_rows_vec<V, true>), (unsigned)rows, 256, 0, x4, y4, axis);           \
  else TP_LAUNCH((k_softmax_rows_vec<V, false>), (unsigned)rows, 256, 0, x4, y4, axis);
    if (axis <= 256 * 4) {
      TP_SOFTMAX_VEC(1)
    } else if (axis <= 256 * 8) {
      TP_SOFTMAX_VEC(2)
    } else if (axis <= 256 * 16) {
      TP_SOFTMAX_VEC(4)
    } else {
      TP_SOFTMAX_VEC(8)
    }
#undef TP_SOFTMAX_VEC
    return;
  }
#define TP_SOFTMAX_CASE(P)                                                                    \
  if (log_mode) TP_LAUNCH((k_softmax_rows<P, true>), (unsigned)rows, 256, 0, x, y, axis);    \
  else TP_LAUNCH((k_softmax_rows<P, false>), (unsigned)rows, 256, 0, x, y, axis);
  if (axis <= 256 * 4) {
    TP_SOFTMAX_CASE(4)
  } else if (axis <= 256 * 8) {
    TP_SOFTMAX_CASE(8)
  } else if (axis <= 256 * 16) {
    TP_SOFTMAX_CASE(16)
  } else if (axis <= 256 * 32) {
    TP_SOFTMAX_CASE(32)
  } else {
    TP_SOFTMAX_CASE(0)
  }
#undef TP_SOFTMAX_CASE
}

// softmax_backward.wgsl: gi = s*(go - sum(go*s));  log_softmax_backward.wgsl:
// gi = go - s*sum(go).  One warp per row (rows are classes-long).
template <bool LOG>
__global__ void k_softmax_bwd(const float* __restrict__ go, const float* __restrict__ s, float* __restrict__ gi,
                              int64_t rows, int64_t C) {
  ::tp::pdl_enter();
  int lane = threadIdx.x & 31;
  int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const float* g = go + row * C;
  const float* sr = s + row * C;
  float acc = 0.0f;
  for (int64_t i = lane; i < C; i += 32) acc += LOG ? g[i] : g[i] * sr[i];
  acc = warp_sum(acc);
  for (int64_t i = lane; i < C; i += 32) gi[row * C + i] = LOG ? g[i] - sr[i] * acc : sr[i] * (g[i] - acc);
}

// Rows of 256 < C <= 8192, C % 4 == 0, 16-byte aligned: one CTA per row with
// the row's go and s in registers as float4 (thread t owns columns t + 256 k),
// so both are read from HBM once (the warp-per-row kernel's second pass re-reads
// rows that no longer fit in L1).
template <int V, bool LOG>
__global__ void __launch_bounds__(256) k_softmax_bwd_vec(const float4* __restrict__ go, const float4* __restrict__ s,
                                                         float4* __restrict__ gi, int64_t C) {
  ::tp::pdl_enter();
  __shared__ float sh[32];
  const int64_t C4 = C >> 2;
  const int64_t base = (int64_t)blockIdx.x * C4;
  float4 g[V], sv[V];
  float acc = 0.0f;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int64_t i = threadIdx.x + (int64_t)k * 256;
    if (i < C4) {
      g[k] = go[base + i];
      sv[k] = s[base + i];
      acc += LOG ? (g[k].x + g[k].y) + (g[k].z + g[k].w)
                 : (g[k].x * sv[k].x + g[k].y * sv[k].y) + (g[k].z * sv[k].z + g[k].w * sv[k].w);
    }
  }
  acc = block_reduce<false>(acc, sh);
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int64_t i = threadIdx.x + (int64_t)k * 256;
    if (i < C4) {
      const float4 a = g[k], b = sv[k];
      gi[base + i] = LOG ? make_float4(a.x - b.x * acc, a.y - b.y * acc, a.z - b.z * acc, a.w - b.w * acc)
                         : make_float4(b.x * (a.x - acc), b.y * (a.y - acc), b.z * (a.z - acc), b.w * (a.w - acc));
    }
  }
}

// cross_entropy.wgsl: loss[row] = logsumexp(x[row]) - x[row, t], t = clamp(i32(target), 0, C-1).
__device__ __forceinline__ int ce_target(float t, int64_t C) {
  int ti = (int)t;
  if (ti < 0) ti = 0;
  if (ti > (int)(C - 1)) ti = (int)(C - 1);
  return ti;
}

__global__ void k_cross_entropy(const float* __restrict__ x, const float* __restrict__ tgt, float* __restrict__ loss,
                                int64_t B, int64_t C) {
  ::tp::pdl_enter();
  int lane = threadIdx.x & 31;
  int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (row >= B) return;
  const float* xr = x + row * C;
  float m = -FLT_MAX;
  for (int64_t i = lane; i < C; i += 32) m = fmaxf(m, xr[i]);
  m = warp_max(m);
  float s = 0.0f;
  for (int64_t i = lane; i < C; i += 32) s += expf(xr[i] - m);
  s = warp_sum(s);
  if (lane == 0) loss[row] = (m + logf(s)) - xr[ce_target(tgt[row], C)];
}

// cross_entropy_backward.wgsl: gi = (softmax - onehot) * upstream * scale.
__global__ void k_cross_entropy_bwd(const float* __restrict__ go, int go_scalar, const float* __restrict__ x,
                                    const float* __restrict__ tgt, float* __restrict__ gi, int64_t B, int64_t C,
                                    float scale) {
  ::tp::pdl_enter();
  int lane = threadIdx.x & 31;
  int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (row >= B) return;
  const float* xr = x + row * C;
  float m = -FLT_MAX;
  for (int64_t i = lane; i < C; i += 32) m = fmaxf(m, xr[i]);
  m = warp_max(m);
  float s = 0.0f;
  for (int64_t i = lane; i < C; i += 32) s += expf(xr[i] - m);
  s = warp_sum(s);
  int t = ce_target(tgt[row], C);
  float up = go_scalar ? go[0] : go[row];
  float rs = up * scale;
  for (int64_t i = lane; i < C; i += 32) {
    float p = expf(xr[i] - m) / s;
    gi[row * C + i] = (p - (i == t ? 1.0f : 0.0f)) * rs;
  }
}

void launch_cross_entropy(const float* x, const float* tgt, float* loss, int64_t B, int64_t C) {
  if (B == 0) return;
  TP_LAUNCH(k_cross_entropy, (unsigned)((B * 32 + 255) / 256), 256, 0, x, tgt, loss, B, C);
}

void launch_cross_entropy_bwd(const float* go, int go_scalar, const float* x, const float* tgt, float* gi, int64_t B,
                              int64_t C, float scale) {
  if (B == 0) return;
  TP_LAUNCH(k_cross_entropy_bwd, (unsigned)((B * 32 + 255) / 256), 256, 0, go, go_scalar, x, tgt, gi, B, C, scale);
}

// ---- allocation-free cross-entropy mean ------------------------------------------------
// Working memory for tpk_cross_entropy_mean_noalloc, reserved when the library
// is loaded: the per-row losses, the per-block partial sums of the mean and the
// last-block ticket.  Every GPU that loads the library keeps this array
// (about 1 MB) until the process exits.
constexpr int64_t CE_NOALLOC_MAX_ROWS = 262144;
constexpr int64_t CE_NOALLOC_FLOATS = CE_NOALLOC_MAX_ROWS + RED_MAX_BLOCKS + 64;
static __device__ __align__(256) float g_ce_noalloc_scratch[CE_NOALLOC_FLOATS];

// Device address of the array on the library's device (the one its stream
// belongs to), looked up once with that device current: host code cannot use
// the symbol itself as a device pointer.  The lookup is guarded, so a first
// call from several threads at once is safe.
static float* g_ce_noalloc_addr[64] = {};
static std::mutex g_ce_noalloc_mu;

static float* ce_noalloc_scratch() {
  const int dev = device();  // initialises the library (device, stream) if needed
  TP_REQUIRE(dev >= 0 && dev < 64, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_ce_noalloc_mu);
  if (!g_ce_noalloc_addr[dev]) {
    int cur = -1;
    TP_CUDA(cudaGetDevice(&cur));
    if (cur != dev) TP_CUDA(cudaSetDevice(dev));
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_ce_noalloc_scratch);
    if (cur != dev) cudaSetDevice(cur);
    if (e != cudaSuccess) fail(TP_ERR_CUDA, "cudaGetSymbolAddress(g_ce_noalloc_scratch) failed: %s",
                               cudaGetErrorString(e));
    g_ce_noalloc_addr[dev] = static_cast<float*>(p);
  }
  return g_ce_noalloc_addr[dev];
}

static void split_dims(const Tensor& t, int dim, int64_t& outer, int64_t& red, int64_t& inner) {
  outer = prod(t.shape, dim);
  red = t.shape[dim];
  inner = prod(t.shape + dim + 1, t.ndim - dim - 1);
}

static int norm_dim(int dim, int rank) {
  if (rank == 0) fail(TP_ERR_ARG, "operation requires at least 1 dimension.");
  int d = dim < 0 ? dim + rank : dim;
  if (d < 0 || d >= rank) fail(TP_ERR_ARG, "dim %d out of range for rank %d", dim, rank);
  return d;
}

}  // namespace tp

using namespace tp;

extern "C" {

TP_API int tp_reduce_all(int64_t id, int mode, tp_handle* out) {
  return guard([&] {
    TP_REQUIRE(mode >= 0 && mode <= 2, "unknown reduce mode %d", mode);
    Tensor& a = get(id);
    TP_REQUIRE(a.phys == PHYS_F32, "reduce takes float storage");
    Tensor o = make(nullptr, 0, a.dtype);
    launch_reduce_all(a.f(), a.numel, mode, o.f());
    emit(o, out);
  });
}
TP_API int tp_sum(int64_t id, tp_handle* out) { return tp_reduce_all(id, 0, out); }
TP_API int tp_mean(int64_t id, tp_handle* out) { return tp_reduce_all(id, 1, out); }
TP_API int tp_max(int64_t id, tp_handle* out) { return tp_reduce_all(id, 2, out); }

TP_API int tp_reduce_dim(int64_t id, int dim, int keepdim, int mode, tp_handle* out) {
  return guard([&] {
    TP_REQUIRE(mode == 0 || mode == 1, "reduce_dim mode must be 0 (sum) or 1 (mean)");
    Tensor& a = get(id);
    int d = norm_dim(dim, a.ndim);
    int64_t outer, red, inner;
    split_dims(a, d, outer, red, inner);
    std::vector<int64_t> s;
    for (int i = 0; i < a.ndim; ++i) {
      if (i == d) {
        if (keepdim) s.push_back(1);
      } else {
        s.push_back(a.shape[i]);
      }
    }
    Tensor o = make_like_shape(s, a.dtype);
    launch_reduce_dim(a.f(), outer, red, inner, mode, o.f(), nullptr);
    emit(o, out);
  });
}
TP_API int tp_sum_dim(int64_t id, int dim, int keepdim, tp_handle* out) { return tp_reduce_dim(id, dim, keepdim, 0, out); }
TP_API int tp_mean_dim(int64_t id, int dim, int keepdim, tp_handle* out) { return tp_reduce_dim(id, dim, keepdim, 1, out); }

TP_API int tp_max_dim(int64_t id, int dim, int keepdim, tp_handle* values, tp_handle* indices) {
  return guard([&] {
    Tensor& a = get(id);
    int d = norm_dim(dim, a.ndim);
    int64_t outer, red, inner;
    split_dims(a, d, outer, red, inner);
    TP_REQUIRE(red > 0, "max along an empty dim");
    std::vector<int64_t> s;
    for (int i = 0; i < a.ndim; ++i) {
      if (i == d) {
        if (keepdim) s.push_back(1);
      } else {
        s.push_back(a.shape[i]);
      }
    }
    Tensor v = make_like_shape(s, a.dtype);
    Tensor ix = make_like_shape(s, TP_INT64, PHYS_I32);
    launch_reduce_dim(a.f(), outer, red, inner, 3, v.f(), ix.i());
    emit(v, values);
    emit(ix, indices);
  });
}

TP_API int tp_argmax(int64_t id, tp_handle* out) {
  return guard([&] {
    Tensor& a = get(id);
    TP_REQUIRE(a.ndim >= 1 && a.shape[a.ndim - 1] > 0, "argmax of an empty tensor");
    int64_t rows = prod(a.shape, a.ndim - 1), red = a.shape[a.ndim - 1];
    std::vector<int64_t> s(a.shape, a.shape + a.ndim - 1);
    if (s.empty()) s.push_back(1);  // reductionOps.ts:135
    Tensor o = make_like_shape(s, TP_INT32, PHYS_I32);
    launch_reduce_dim(a.f(), rows, red, 1, 4, nullptr, o.i());
    emit(o, out);
  });
}

TP_API int tp_softmax(int64_t id, int dim, tp_handle* out) {
  return guard([&] {
    Tensor& a = get(id);
    int d = norm_dim(dim, a.ndim);
    int64_t outer, axis, inner;
    split_dims(a, d, outer, axis, inner);
    Tensor o = make(a.shape, a.ndim, a.dtype);
    launch_softmax(a.f(), o.f(), outer, axis, inner, false);
    emit(o, out);
  });
}

TP_API int tp_log_softmax(int64_t id, int dim, tp_handle* out) {
  return guard([&] {
    Tensor& a = get(id);
    int d = norm_dim(dim, a.ndim);
    int64_t outer, axis, inner;
    split_dims(a, d, outer, axis, inner);
    Tensor o = make(a.shape, a.ndim, a.dtype);
    launch_softmax(a.f(), o.f(), outer, axis, inner, true);
    emit(o, out);
  });
}

static int softmax_bwd_impl(bool log_mode, int64_t go, int64_t s, int64_t B, int64_t C, tp_handle* out) {
  return guard([&] {
    Tensor& g = get(go);
    Tensor& sm = get(s);
    TP_REQUIRE(g.numel >= B * C && sm.numel >= B * C, "softmax backward: tensors hold fewer than %lld values",
               (long long)(B * C));
    int64_t shp[2] = {B, C};
    Tensor o = make(shp, 2, g.dtype);
    const bool vec = C > 256 && C <= 256 * 32 && C % 4 == 0 && ((uintptr_t)g.f() & 15) == 0 &&
                     ((uintptr_t)sm.f() & 15) == 0 && ((uintptr_t)o.f() & 15) == 0;
    if (B * C > 0 && vec) {
      const float4 *g4 = (const float4*)g.f(), *s4 = (const float4*)sm.f();
      float4* o4 = (float4*)o.f();
      const unsigned rows = (unsigned)B;
#define TP_SMBWD_VEC(V)                                                                           \
  if (log_mode) TP_LAUNCH((k_softmax_bwd_vec<V, true>), rows, 256, 0, g4, s4, o4, C);           \
  else TP_LAUNCH((k_softmax_bwd_vec<V, false>), rows, 256, 0, g4, s4, o4, C);
      if (C <= 256 * 4) {
        TP_SMBWD_VEC(1)
      } else if (C <= 256 * 8) {
        TP_SMBWD_VEC(2)
      } else if (C <= 256 * 16) {
        TP_SMBWD_VEC(4)
      } else {
        TP_SMBWD_VEC(8)
      }
#undef TP_SMBWD_VEC
    } else if (B * C > 0) {
      unsigned blocks = (unsigned)((B * 32 + 255) / 256);
      if (log_mode) TP_LAUNCH(k_softmax_bwd<true>, blocks, 256, 0, g.f(), sm.f(), o.f(), B, C);
      else TP_LAUNCH(k_softmax_bwd<false>, blocks, 256, 0, g.f(), sm.f(), o.f(), B, C);
    }
    emit(o, out);
  });
}

TP_API int tp_softmax_backward(int64_t go, int64_t s, int64_t B, int64_t C, tp_handle* out) {
  return softmax_bwd_impl(false, go, s, B, C, out);
}
TP_API int tp_log_softmax_backward(int64_t go, int64_t s, int64_t B, int64_t C, tp_handle* out) {
  return softmax_bwd_impl(true, go, s, B, C, out);
}

TP_API int tp_cross_entropy(int64_t input, int64_t targets, tp_handle* out) {
  return guard([&] {
    Tensor& x = get(input);
    Tensor& t = get(targets);
    TP_REQUIRE(x.ndim >= 1, "cross_entropy expects [batch, classes] logits");
    int64_t B = t.numel, C = x.shape[x.ndim - 1];
    TP_REQUIRE(B * C == x.numel, "cross_entropy: %lld targets for %lld logits of %lld classes", (long long)B,
               (long long)x.numel, (long long)C);
    int64_t s[1] = {B};
    Tensor o = make(s, 1, x.dtype);
    launch_cross_entropy(x.f(), t.f(), o.f(), B, C);
    emit(o, out);
  });
}

// Mean cross-entropy loss of B rows of C logits, for callers that must not
// allocate device memory: a process that reserves its whole HBM budget at
// start-up and forbids allocation afterwards, or a latency-critical loop where
// an allocation could block or fail.  Inputs and the one-float output are the
// caller's; the per-row losses and reduction partials live in a fixed
// file-scope device array, so B is limited to CE_NOALLOC_MAX_ROWS.  The first
// call on a device looks up that array's device address (cudaGetSymbolAddress);
// make that first call before any stream capture.  All calls share the one
// array, which keeps the last call's contents: the ticket is cleared before
// every launch, and calls whose work overlaps on the GPU (other streams,
// other threads) race on it.  Calls on the library stream are ordered.
TP_API int tpk_cross_entropy_mean_noalloc(const float* logits, const float* targets, float* loss_mean, int64_t B,
                                          int64_t C) {
  return guard([&] {
    TP_REQUIRE(B >= 0 && B <= CE_NOALLOC_MAX_ROWS,
               "cross_entropy_mean_noalloc: %lld rows is outside [0, %lld], the size of its fixed work area",
               (long long)B, (long long)CE_NOALLOC_MAX_ROWS);
    TP_REQUIRE(C >= 1, "cross_entropy_mean_noalloc: need at least one class");
    if (B == 0) {  // the mean of no rows is 0, as tpk_cross_entropy_mean writes
      TP_CUDA(cudaMemsetAsync(loss_mean, 0, sizeof(float), stream()));
      return;
    }
    float* base = ce_noalloc_scratch();
    float* rows = base;
    float* partials = base + CE_NOALLOC_MAX_ROWS;
    unsigned int* ticket = reinterpret_cast<unsigned int*>(partials + RED_MAX_BLOCKS);
    TP_CUDA(cudaMemsetAsync(ticket, 0, sizeof(unsigned int), stream()));
    TP_LAUNCH(k_cross_entropy, (unsigned)((B * 32 + 255) / 256), 256, 0, logits, targets, rows, B, C);
    unsigned blocks = grid_for(B, 256, 8);
    unsigned cap = (unsigned)sm_count() * 4;
    if (blocks > cap) blocks = cap;
    if (blocks > RED_MAX_BLOCKS) blocks = RED_MAX_BLOCKS;
    TP_LAUNCH(k_reduce_all, blocks, 256, 0, rows, B, 1, loss_mean, partials, ticket);
  });
}

TP_API int tp_cross_entropy_backward(int64_t grad_out, int64_t input, int64_t targets, int reduction,
                                     tp_handle* out) {
  return guard([&] {
    Tensor& g = get(grad_out);
    Tensor& x = get(input);
    Tensor& t = get(targets);
    int64_t B = t.numel, C = x.shape[x.ndim - 1];
    TP_REQUIRE(B * C == x.numel, "cross_entropy_backward: shape mismatch");
    int go_scalar = g.numel == 1 ? 1 : 0;
    TP_REQUIRE(go_scalar || g.numel >= B, "cross_entropy_backward: grad_output too short");
    float scale = reduction == 2 ? 1.0f / (float)(B > 1 ? B : 1) : 1.0f;
    int64_t s[2] = {B, C};
    Tensor o = make(s, 2, x.dtype);
    launch_cross_entropy_bwd(g.f(), go_scalar, x.f(), t.f(), o.f(), B, C, scale);
    emit(o, out);
  });
}

}  // extern "C"
