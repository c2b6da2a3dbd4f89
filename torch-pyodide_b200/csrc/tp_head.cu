// The classifier head of a training step in one launch: linear layer, mean
// cross-entropy and both their gradients.
//
// The reference composes it from ~10 dispatches (linear: transpose + matmul +
// add, runtime/src/ops/arithmeticOps.ts:260-308; cross_entropy.wgsl and
// cross_entropy_backward.wgsl through reductionOps.ts:471-531; the backward
// matmuls and the bias sum from python/torch/autograd_rules.py), and the
// per-op path here takes 10 launches too (two GEMMs with their split-K
// reduces, the CE rows, their mean, the CE backward, the bias sum and its
// finish).  At a classifier's size (B rows x F = 512 features x K = 10
// classes) each of those is a few microseconds of launch and ramp for
// nanoseconds of work, so the head is one kernel:
//
//   CTA j owns rows [j R, (j + 1) R), a warp per row at a time (W in shared memory):
//     logits[r][k] = x[r] . w[k] + b[k]              (warp dot products)
//     loss[r] = logsumexp(logits[r]) - logits[r][t]   (k_cross_entropy's arithmetic)
//     g[r][k] = (softmax(logits[r])[k] - [k == t]) * scale
//     dx[r][f] = sum_k g[r][k] w[k][f]
//   then, over its rows in order: partial dW = sum_r g[r]^T x[r], partial db,
//   partial loss sum; the last CTA to finish (a self-resetting ticket) adds the
//   partials of all CTAs in CTA order.  Every sum runs in a fixed order, so
//   the result does not depend on scheduling.
//
// The ticket is one word per device: calls must not overlap on the GPU (all
// library launches go to its one stream, in order).
#include <cuda_runtime.h>
#include <float.h>

#include "tp_core.h"

namespace tp {

constexpr int HEAD_THREADS = 256;
constexpr int HEAD_MAX_K = 32;
constexpr int HEAD_MAX_F = 1024;
constexpr int HEAD_MAX_CTAS = 16;  // grid size bound (rows per CTA = ceil(B / 16), at least 8)

static __device__ unsigned int g_head_ticket;

__device__ __forceinline__ float head_warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float head_warp_max(float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int head_target(float t, int K) {  // cross_entropy.wgsl's clamp
  int ti = (int)t;
  if (ti < 0) ti = 0;
  if (ti > K - 1) ti = K - 1;
  return ti;
}

struct HeadArgs {
  const float* x;     // [B][F]
  const float* w;     // [K][F]
  const float* b;     // [K] or null
  const float* tgt;   // [B] class indices as floats
  float* logits;      // [B][K] or null
  float* loss_rows;   // [B] or null
  float* loss_mean;   // [1] or null
  float* dx;          // [B][F] or null
  float* dw;          // [K][F] or null
  float* db;          // [K] or null
  float* part;        // [grid][K*F + K + 1]
  int B, F, K, R;     // R: rows per CTA
  float scale;
};

// dynamic shared memory: w [K][F], then g [R][K], then loss [R]
template <int FPL>  // features per lane (F <= 32 * FPL)
__global__ void __launch_bounds__(HEAD_THREADS) k_linear_ce_step(HeadArgs a) {
  extern __shared__ float sm[];
  float* ws = sm;
  float* gs = ws + (size_t)a.K * a.F;
  float* ls = gs + (size_t)a.R * a.K;
  __shared__ unsigned int last;
  ::tp::pdl_enter();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = HEAD_THREADS / 32;
  for (int i = tid; i < a.K * a.F; i += HEAD_THREADS) ws[i] = a.w[i];
  __syncthreads();
  const int r0 = blockIdx.x * a.R;
  const int r1 = min(r0 + a.R, a.B);
  for (int r = r0 + warp; r < r1; r += nwarp) {
    float xv[FPL];
#pragma unroll
    for (int i = 0; i < FPL; ++i) {
      const int f = lane + 32 * i;
      xv[i] = f < a.F ? a.x[(int64_t)r * a.F + f] : 0.0f;
    }
    // lane k keeps logit k
    float mine = -FLT_MAX;
    for (int k = 0; k < a.K; ++k) {
      float s = 0.0f;
#pragma unroll
      for (int i = 0; i < FPL; ++i) {
        const int f = lane + 32 * i;
        if (f < a.F) s = fmaf(xv[i], ws[k * a.F + f], s);
      }
      s = head_warp_sum(s) + (a.b ? a.b[k] : 0.0f);
      if (lane == k) mine = s;
    }
    const bool has = lane < a.K;
    const float m = head_warp_max(has ? mine : -FLT_MAX);
    const float e = has ? expf(mine - m) : 0.0f;
    const float se = head_warp_sum(e);
    const int t = head_target(a.tgt[r], a.K);
    const float lt = __shfl_sync(0xffffffffu, mine, t);
    const float g = has ? (e / se - (lane == t ? 1.0f : 0.0f)) * a.scale : 0.0f;
    if (has) {
      if (a.logits) a.logits[(int64_t)r * a.K + lane] = mine;
      gs[(r - r0) * a.K + lane] = g;
    }
    if (lane == 0) {
      const float loss = (m + logf(se)) - lt;
      ls[r - r0] = loss;
      if (a.loss_rows) a.loss_rows[r] = loss;
    }
    if (a.dx) {
      float d[FPL];
#pragma unroll
      for (int i = 0; i < FPL; ++i) d[i] = 0.0f;
      for (int k = 0; k < a.K; ++k) {
        const float gk = __shfl_sync(0xffffffffu, g, k);
#pragma unroll
        for (int i = 0; i < FPL; ++i) {
          const int f = lane + 32 * i;
          if (f < a.F) d[i] = fmaf(gk, ws[k * a.F + f], d[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < FPL; ++i) {
        const int f = lane + 32 * i;
        if (f < a.F) a.dx[(int64_t)r * a.F + f] = d[i];
      }
    }
  }
  __syncthreads();
  // this CTA's partials, rows in order
  const int stride = a.K * a.F + a.K + 1;
  float* pp = a.part + (size_t)blockIdx.x * stride;
  for (int f = tid; f < a.F; f += HEAD_THREADS) {
    float acc[HEAD_MAX_K];
#pragma unroll
    for (int k = 0; k < HEAD_MAX_K; ++k) acc[k] = 0.0f;
    for (int r = r0; r < r1; ++r) {
      const float xf = a.x[(int64_t)r * a.F + f];
#pragma unroll
      for (int k = 0; k < HEAD_MAX_K; ++k)
        if (k < a.K) acc[k] = fmaf(gs[(r - r0) * a.K + k], xf, acc[k]);
    }
#pragma unroll
    for (int k = 0; k < HEAD_MAX_K; ++k)
      if (k < a.K) pp[k * a.F + f] = acc[k];
  }
  if (tid < a.K) {
    float s = 0.0f;
    for (int r = r0; r < r1; ++r) s += gs[(r - r0) * a.K + tid];
    pp[a.K * a.F + tid] = s;
  }
  if (tid == 0) {
    float s = 0.0f;
    for (int r = r0; r < r1; ++r) s += ls[r - r0];
    pp[a.K * a.F + a.K] = s;
  }
  // the last CTA adds every CTA's partials (ticket returns to 0 after gridDim.x arrivals)
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    last = atomicInc(&g_head_ticket, gridDim.x - 1) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // four outputs per thread and step, all HEAD_MAX_CTAS partials of each loaded before
  // any is added (this CTA's time is the launch's tail), then added in CTA order
  const int nb = gridDim.x;
  for (int i0 = tid; i0 < stride; i0 += 4 * HEAD_THREADS) {
    float v[4][HEAD_MAX_CTAS];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * HEAD_THREADS;
#pragma unroll
      for (int j = 0; j < HEAD_MAX_CTAS; ++j)
        v[u][j] = (j < nb && i < stride) ? __ldcg(a.part + (size_t)j * stride + i) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * HEAD_THREADS;
      if (i >= stride) continue;
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < HEAD_MAX_CTAS; ++j)
        if (j < nb) s += v[u][j];
      if (i < a.K * a.F) {
        if (a.dw) a.dw[i] = s;
      } else if (i < a.K * a.F + a.K) {
        if (a.db) a.db[i - a.K * a.F] = s;
      } else if (a.loss_mean) {
        a.loss_mean[0] = a.B > 0 ? s / (float)a.B : 0.0f;
      }
    }
  }
}

template <int FPL>
static void head_launch(int grid, size_t smem, const HeadArgs& a) {
  static bool attr = false;  // one per instantiation
  if (!attr) {
    TP_CUDA(cudaFuncSetAttribute(k_linear_ce_step<FPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr = true;
  }
  TP_LAUNCH(k_linear_ce_step<FPL>, (unsigned)grid, HEAD_THREADS, smem, a);
}

}  // namespace tp

using namespace tp;

extern "C" {

TP_API int tpk_linear_cross_entropy_step(const float* x, const float* w, const float* b, const float* targets,
                                         float* logits, float* loss_rows, float* loss_mean, float* dx, float* dw,
                                         float* db, int64_t B, int64_t F, int64_t K, float scale) {
  return guard([&] {
    TP_REQUIRE(B >= 1 && B < ((int64_t)1 << 30), "linear_cross_entropy_step: 1 <= B < 2^30 rows");
    TP_REQUIRE(F >= 1 && F <= HEAD_MAX_F, "linear_cross_entropy_step: 1 <= F <= %d features", HEAD_MAX_F);
    TP_REQUIRE(K >= 1 && K <= HEAD_MAX_K, "linear_cross_entropy_step: 1 <= K <= %d classes", HEAD_MAX_K);
    TP_REQUIRE(x && w && targets, "linear_cross_entropy_step: x, w and targets are required");
    // about 16 CTAs: each adds its rows' dW in order, the last adds 16 partials
    int R = (int)((B + 15) / 16);
    if (R < 8) R = 8;
    const int grid = (int)((B + R - 1) / R);
    TP_REQUIRE(grid <= HEAD_MAX_CTAS, "linear_cross_entropy_step: grid of %d CTAs", grid);
    const size_t smem = ((size_t)K * F + (size_t)R * K + R) * sizeof(float);
    TP_REQUIRE(smem <= 200 * 1024, "linear_cross_entropy_step: K*F + R*(K+1) floats exceed shared memory");
    float* part = (float*)scratch((size_t)grid * (K * F + K + 1) * sizeof(float));
    HeadArgs a{x, w, b, targets, logits, loss_rows, loss_mean, dx, dw, db, part,
               (int)B, (int)F, (int)K, R, scale};
    if (F <= 256)
      head_launch<8>(grid, smem, a);
    else if (F <= 512)
      head_launch<16>(grid, smem, a);
    else
      head_launch<32>(grid, smem, a);
  });
}

}  // extern "C"
