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
//   CTA j owns rows [j R, (j + 1) R), a warp per row at a time (W in shared memory,
//   the warp's next row loaded while it works on the current one):
//     logits[r][k] = x[r] . w[k] + b[k]              (warp dot products)
//     loss[r] = logsumexp(logits[r]) - logits[r][t]   (k_cross_entropy's arithmetic)
//     g[r][k] = (softmax(logits[r])[k] - [k == t]) * scale
//     dx[r][f] = sum_k g[r][k] w[k][f]
//   then, over its rows in order: partial dW = sum_r g[r]^T x[r], partial db,
//   partial loss sum; the last CTA of each group to finish (a self-resetting
//   ticket) adds its group's partials in CTA order (one group of up to 16 CTAs,
//   else groups of 8 whose sums the last group adds in group order).  Every sum runs in a fixed order, so the result
//   does not depend on scheduling.  Up to 128 CTAs of one warp-row per warp: the
//   work is a few microseconds of latency-bound dot products, so it is spread
//   over as many SMs as there are rows for.
//
// The tickets are words per device: calls must not overlap on the GPU (all
// library launches go to its one stream, in order).
#include <cuda_runtime.h>
#include <float.h>

#include "tp_core.h"

namespace tp {

constexpr int HEAD_THREADS = 256;
constexpr int HEAD_MAX_K = 32;
constexpr int HEAD_MAX_F = 1024;
constexpr int HEAD_GROUP = 8;        // CTAs whose partials one CTA adds first
constexpr int HEAD_MAX_GROUPS = 16;
constexpr int HEAD_MAX_CTAS = HEAD_GROUP * HEAD_MAX_GROUPS;  // rows per CTA = max(8, ceil(B / 128))

static __device__ unsigned int g_head_ticket;
static __device__ unsigned int g_head_group_ticket[HEAD_MAX_GROUPS];

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
  float* part;        // [grid + groups][K*F + K + 1]: CTA partials, then group sums
  int B, F, K, R;     // R: rows per CTA
  float scale;
};

// out(i, sum over j < n of src[j * stride + i]) for every i < stride, j in order;
// four outputs per thread and step, all n partials of each loaded before any is
// added (the adding CTA's time is the launch's tail).
template <int NMAX, class Out>
__device__ __forceinline__ void head_add_partials(const float* src, int n, int stride, int tid, Out&& out) {
  for (int i0 = tid; i0 < stride; i0 += 4 * HEAD_THREADS) {
    float v[4][NMAX];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * HEAD_THREADS;
#pragma unroll
      for (int j = 0; j < NMAX; ++j) v[u][j] = (j < n && i < stride) ? __ldcg(src + (size_t)j * stride + i) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * HEAD_THREADS;
      if (i >= stride) continue;
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < NMAX; ++j)
        if (j < n) acc += v[u][j];
      out(i, acc);
    }
  }
}

// Lane l ends with the warp's sum of v[l % KP] (KP = 16 or 32 partial logits per
// lane): a reduce-scatter, each xor stage keeps the half of the values whose
// index bit matches the lane's and adds the partner's copy of them (KP = 16:
// stages 8 .. 1 inside each half-warp, then one xor-16 add).  31 shuffles in 5
// dependent steps instead of a 5-step tree per logit.
template <int KP>
__device__ __forceinline__ float head_reduce_scatter(float (&v)[KP], int lane) {
  static_assert(KP == 16 || KP == 32, "16 or 32 partial logits per lane");
#pragma unroll
  for (int o = KP / 2; o > 0; o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < o; ++j) {
      const float send = up ? v[j] : v[j + o];
      const float keep = up ? v[j + o] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  if (KP == 16) v[0] += __shfl_xor_sync(0xffffffffu, v[0], 16);
  return v[0];
}

// dynamic shared memory: w [K][F], then g [R][K], then loss [R]
template <int FPL, int KP>  // features per lane (F <= 32 * FPL), logits per lane (K <= KP)
__global__ void __launch_bounds__(HEAD_THREADS) k_linear_ce_step(HeadArgs a) {
  extern __shared__ __align__(16) float sm[];
  float* ws = sm;
  float* gs = ws + (size_t)a.K * a.F;
  float* ls = gs + (size_t)a.R * a.K;
  __shared__ unsigned int last;
  ::tp::pdl_enter();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = HEAD_THREADS / 32;
  {  // W into shared memory, 16-byte vectors 8 per thread in flight (W is 16-byte aligned
     // and K*F a multiple of 4, else one float at a time)
    const int n = a.K * a.F;
    if ((n & 3) == 0 && ((uintptr_t)a.w & 15) == 0) {
      const float4* w4 = reinterpret_cast<const float4*>(a.w);
      float4* s4 = reinterpret_cast<float4*>(ws);
#pragma unroll 8
      for (int i = tid; i < n / 4; i += HEAD_THREADS) s4[i] = __ldg(w4 + i);
    } else {
#pragma unroll 8
      for (int i = tid; i < n; i += HEAD_THREADS) ws[i] = __ldg(a.w + i);
    }
  }
  const int r0 = blockIdx.x * a.R;
  const int r1 = min(r0 + a.R, a.B);
  // the warp's first row is loaded while W is staged; each row's successor while it is used
  float xv[FPL], xn[FPL];
  float tv = 0.0f, tn = 0.0f;
  const float bias = (a.b && lane < a.K) ? a.b[lane] : 0.0f;
  if (r0 + warp < r1) {
#pragma unroll
    for (int i = 0; i < FPL; ++i) {
      const int f = lane + 32 * i;
      xv[i] = f < a.F ? a.x[(int64_t)(r0 + warp) * a.F + f] : 0.0f;
    }
    tv = a.tgt[r0 + warp];
  }
  __syncthreads();
  for (int r = r0 + warp; r < r1; r += nwarp) {
    const int rn = r + nwarp;
    if (rn < r1) {
#pragma unroll
      for (int i = 0; i < FPL; ++i) {
        const int f = lane + 32 * i;
        xn[i] = f < a.F ? a.x[(int64_t)rn * a.F + f] : 0.0f;
      }
      tn = a.tgt[rn];
    }
    // partial dot products of all logits, then lane k keeps logit k
    float s[KP];
#pragma unroll
    for (int k = 0; k < KP; ++k) {
      s[k] = 0.0f;
      if (k < a.K) {
#pragma unroll
        for (int i = 0; i < FPL; ++i) {
          const int f = lane + 32 * i;
          if (f < a.F) s[k] = fmaf(xv[i], ws[k * a.F + f], s[k]);
        }
      }
    }
    const bool has = lane < a.K;
    float mine = head_reduce_scatter<KP>(s, lane);
    mine = has ? mine + bias : -FLT_MAX;
    const float m = head_warp_max(mine);
    const float e = has ? expf(mine - m) : 0.0f;
    const float se = head_warp_sum(e);
    const int t = head_target(tv, a.K);
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
#pragma unroll
    for (int i = 0; i < FPL; ++i) xv[i] = xn[i];
    tv = tn;
  }
  __syncthreads();
  // this CTA's partials, rows in order
  const int stride = a.K * a.F + a.K + 1;
  float* pp = a.part + (size_t)blockIdx.x * stride;
  // every (k, f) over the CTA's rows in order; a thread owns FT features, and
  // fetches RB rows of them at a time (32 loads in flight)
  constexpr int FT = FPL / 8;  // F <= 256 FT
  constexpr int RB = 32 / FT;
  {
    float acc[FT][KP];
#pragma unroll
    for (int ft = 0; ft < FT; ++ft)
#pragma unroll
      for (int k = 0; k < KP; ++k) acc[ft][k] = 0.0f;
    int r = r0;
    for (; r + RB <= r1; r += RB) {
      float xf[RB][FT];
#pragma unroll
      for (int u = 0; u < RB; ++u)
#pragma unroll
        for (int ft = 0; ft < FT; ++ft) {
          const int f = tid + HEAD_THREADS * ft;
          xf[u][ft] = f < a.F ? a.x[(int64_t)(r + u) * a.F + f] : 0.0f;
        }
#pragma unroll
      for (int u = 0; u < RB; ++u)
#pragma unroll
        for (int k = 0; k < KP; ++k)
          if (k < a.K) {
            const float gk = gs[(r + u - r0) * a.K + k];
#pragma unroll
            for (int ft = 0; ft < FT; ++ft) acc[ft][k] = fmaf(gk, xf[u][ft], acc[ft][k]);
          }
    }
    for (; r < r1; ++r) {
#pragma unroll
      for (int ft = 0; ft < FT; ++ft) {
        const int f = tid + HEAD_THREADS * ft;
        const float xf = f < a.F ? a.x[(int64_t)r * a.F + f] : 0.0f;
#pragma unroll
        for (int k = 0; k < KP; ++k)
          if (k < a.K) acc[ft][k] = fmaf(gs[(r - r0) * a.K + k], xf, acc[ft][k]);
      }
    }
#pragma unroll
    for (int ft = 0; ft < FT; ++ft) {
      const int f = tid + HEAD_THREADS * ft;
      if (f < a.F) {
#pragma unroll
        for (int k = 0; k < KP; ++k)
          if (k < a.K) pp[k * a.F + f] = acc[ft][k];
      }
    }
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
  // Fixed-order sums: the last CTA of each group to finish adds its group's partials
  // in CTA order; with more than one group (more than HEAD_MAX_GROUPS CTAs, groups of
  // HEAD_GROUP) the last group to finish then adds the group sums in group order
  // (each ticket returns to 0 after its arrivals).
  auto emit = [&](int i, float v) {
    if (i < a.K * a.F) {
      if (a.dw) a.dw[i] = v;
    } else if (i < a.K * a.F + a.K) {
      if (a.db) a.db[i - a.K * a.F] = v;
    } else if (a.loss_mean) {
      a.loss_mean[0] = a.B > 0 ? v / (float)a.B : 0.0f;
    }
  };
  const int gsz = gridDim.x <= (unsigned)HEAD_MAX_GROUPS ? (int)gridDim.x : HEAD_GROUP;
  const int ngroups = ((int)gridDim.x + gsz - 1) / gsz;
  const int grp = (int)blockIdx.x / gsz;
  const int g0 = grp * gsz;
  const int gn = min(gsz, (int)gridDim.x - g0);
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    last = atomicInc(&g_head_group_ticket[grp], (unsigned)gn - 1) == (unsigned)gn - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (ngroups == 1) {
    head_add_partials<HEAD_MAX_GROUPS>(a.part, gn, stride, tid, emit);
    return;
  }
  float* gsum = a.part + ((size_t)gridDim.x + grp) * stride;
  head_add_partials<HEAD_GROUP>(a.part + (size_t)g0 * stride, gn, stride, tid,
                                [&](int i, float v) { gsum[i] = v; });
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    last = atomicInc(&g_head_ticket, (unsigned)ngroups - 1) == (unsigned)ngroups - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  head_add_partials<HEAD_MAX_GROUPS>(a.part + (size_t)gridDim.x * stride, ngroups, stride, tid, emit);
}

template <int FPL, int KP>
static void head_launch_k(int grid, size_t smem, const HeadArgs& a) {
  static bool attr = false;  // one per instantiation
  if (!attr) {
    TP_CUDA(cudaFuncSetAttribute(k_linear_ce_step<FPL, KP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 200 * 1024));
    attr = true;
  }
  TP_LAUNCH((k_linear_ce_step<FPL, KP>), (unsigned)grid, HEAD_THREADS, smem, a);
}

template <int FPL>
static void head_launch(int grid, size_t smem, const HeadArgs& a) {
  if (a.K <= 16) head_launch_k<FPL, 16>(grid, smem, a);
  else head_launch_k<FPL, 32>(grid, smem, a);
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
    // up to 128 CTAs of at least 8 rows (a warp per row): each adds its rows' dW in
    // order, then one group of up to HEAD_MAX_GROUPS partials, or groups of HEAD_GROUP
    // and their sums
    int64_t R = (B + HEAD_MAX_CTAS - 1) / HEAD_MAX_CTAS;
    if (R < 8) R = 8;
    const int grid = (int)((B + R - 1) / R);
    TP_REQUIRE(grid <= HEAD_MAX_CTAS, "linear_cross_entropy_step: grid of %d CTAs", grid);
    const size_t smem = ((size_t)K * F + (size_t)R * K + R) * sizeof(float);
    TP_REQUIRE(smem <= 200 * 1024, "linear_cross_entropy_step: K*F + R*(K+1) floats exceed shared memory");
    const int ngroups = (grid + HEAD_GROUP - 1) / HEAD_GROUP;
    float* part = (float*)scratch((size_t)(grid + ngroups) * (K * F + K + 1) * sizeof(float));
    HeadArgs a{x, w, b, targets, logits, loss_rows, loss_mean, dx, dw, db, part,
               (int)B, (int)F, (int)K, (int)R, scale};
    if (F <= 256)
      head_launch<8>(grid, smem, a);
    else if (F <= 512)
      head_launch<16>(grid, smem, a);
    else
      head_launch<32>(grid, smem, a);
  });
}

}  // extern "C"
