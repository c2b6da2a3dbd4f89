// Fused optimizer steps: one multi-tensor launch per parameter group.
//
// Reference: adam_step.wgsl / adamw_step.wgsl / sgd_step.wgsl update one
// parameter per dispatch (three uniform buffers each, reductionOps.ts:533-653)
// and the Python optimizers loop over parameters (optim/__init__.py:158-205,
// 238-312, 345-418).  Here a device table lists every tensor of the group and a
// chunk table splits them into 64K-element chunks; a grid sized to the SM
// count walks the chunks with 128-bit loads, reading param, grad and state
// once and writing param and state once (AdamW: 28 B per element, SGD with
// momentum: 20 B).
//
// The per-element arithmetic is the WGSL's, operation by operation, with
// explicit round-to-nearest intrinsics so no multiply-add is contracted: the
// result is bit-identical to the CPU oracle's restatement compiled with
// -ffp-contract=off (sqrt and division are IEEE-rounded in both).
#include <cuda_runtime.h>

#include <unordered_map>

#include "tp_core.h"
#include "tp_launch.h"

namespace tp {

constexpr int64_t OPT_CHUNK = 65536;

struct OptRow {
  float* p;
  const float* g;
  float* s0;
  float* s1;
  float* lo;  // SGD: the updated parameter's tf32 low parts (optional)
  int64_t n;
};
struct OptChunk {
  int32_t row;
  int32_t len;
  int64_t start;
};

struct AdamHP {
  float lr, b1, b2, eps, wd, step_size, inv_sqrt_bc2, omb1, omb2, lrwd;
};

// adamw_step.wgsl:26-39 (ADAMW) and adam_step.wgsl:25-38 (ADAM).
template <bool ADAMW>
__device__ __forceinline__ void adam_elem(float& p, float g, float& m, float& v, const AdamHP& h) {
  if (ADAMW) {
    if (h.wd != 0.0f) p = __fsub_rn(p, __fmul_rn(h.lrwd, p));
  } else {
    if (h.wd != 0.0f) g = __fadd_rn(g, __fmul_rn(h.wd, p));
  }
  m = __fadd_rn(__fmul_rn(m, h.b1), __fmul_rn(h.omb1, g));
  v = __fadd_rn(__fmul_rn(v, h.b2), __fmul_rn(__fmul_rn(h.omb2, g), g));
  float denom = __fadd_rn(__fmul_rn(__fsqrt_rn(v), h.inv_sqrt_bc2), h.eps);
  float upd = __fmul_rn(__fdiv_rn(m, denom), h.step_size);
  p = __fsub_rn(p, upd);
}

template <bool ADAMW>
__global__ void __launch_bounds__(256) k_adam_multi(const OptRow* __restrict__ rows, const OptChunk* __restrict__ chunks,
                                                    int nchunks, AdamHP h) {
  ::tp::pdl_enter();
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    OptChunk ch = chunks[c];
    OptRow r = rows[ch.row];
    float* __restrict__ P = r.p + ch.start;
    const float* __restrict__ G = r.g + ch.start;
    float* __restrict__ M = r.s0 + ch.start;
    float* __restrict__ V = r.s1 + ch.start;
    int len = ch.len;
    int len4 = len >> 2;
    float4* P4 = reinterpret_cast<float4*>(P);
    const float4* G4 = reinterpret_cast<const float4*>(G);
    float4* M4 = reinterpret_cast<float4*>(M);
    float4* V4 = reinterpret_cast<float4*>(V);
    int i = threadIdx.x;
    // two float4 per thread per iteration, loads issued before the math
    for (; i + (int)blockDim.x < len4; i += 2 * blockDim.x) {
      int j = i + blockDim.x;
      float4 p0 = P4[i], g0 = G4[i], m0 = M4[i], v0 = V4[i];
      float4 p1 = P4[j], g1 = G4[j], m1 = M4[j], v1 = V4[j];
      adam_elem<ADAMW>(p0.x, g0.x, m0.x, v0.x, h);
      adam_elem<ADAMW>(p0.y, g0.y, m0.y, v0.y, h);
      adam_elem<ADAMW>(p0.z, g0.z, m0.z, v0.z, h);
      adam_elem<ADAMW>(p0.w, g0.w, m0.w, v0.w, h);
      adam_elem<ADAMW>(p1.x, g1.x, m1.x, v1.x, h);
      adam_elem<ADAMW>(p1.y, g1.y, m1.y, v1.y, h);
      adam_elem<ADAMW>(p1.z, g1.z, m1.z, v1.z, h);
      adam_elem<ADAMW>(p1.w, g1.w, m1.w, v1.w, h);
      P4[i] = p0; M4[i] = m0; V4[i] = v0;
      P4[j] = p1; M4[j] = m1; V4[j] = v1;
    }
    for (; i < len4; i += blockDim.x) {
      float4 p0 = P4[i], g0 = G4[i], m0 = M4[i], v0 = V4[i];
      adam_elem<ADAMW>(p0.x, g0.x, m0.x, v0.x, h);
      adam_elem<ADAMW>(p0.y, g0.y, m0.y, v0.y, h);
      adam_elem<ADAMW>(p0.z, g0.z, m0.z, v0.z, h);
      adam_elem<ADAMW>(p0.w, g0.w, m0.w, v0.w, h);
      P4[i] = p0; M4[i] = m0; V4[i] = v0;
    }
    for (int k = (len4 << 2) + threadIdx.x; k < len; k += blockDim.x) {
      float p = P[k], m = M[k], v = V[k];
      adam_elem<ADAMW>(p, G[k], m, v, h);
      P[k] = p; M[k] = m; V[k] = v;
    }
  }
}

struct SgdHP {
  float lr, mom, wd, omd, scale;
  int has_m, nesterov;
};

// sgd_step.wgsl:21-41; `scale` (1 for the reference op) multiplies the grad on
// read so averaged data-parallel gradients need no separate pass.
__device__ __forceinline__ void sgd_elem(float& p, float g, float& buf, const SgdHP& h) {
  if (h.scale != 1.0f) g = __fmul_rn(g, h.scale);
  if (h.wd != 0.0f) g = __fadd_rn(g, __fmul_rn(h.wd, p));
  float upd = g;
  if (h.has_m) {
    buf = __fadd_rn(__fmul_rn(buf, h.mom), __fmul_rn(g, h.omd));
    upd = h.nesterov ? __fadd_rn(g, __fmul_rn(h.mom, buf)) : buf;
  }
  p = __fsub_rn(p, __fmul_rn(h.lr, upd));
}

// x - (x with its 13 low mantissa bits cleared) per lane: the 3xTF32 low part
__device__ __forceinline__ float4 tf32_lo4(float4 v) {
  return make_float4(v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u),
                     v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u),
                     v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u),
                     v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u));
}

__global__ void __launch_bounds__(256) k_sgd_multi(const OptRow* __restrict__ rows, const OptChunk* __restrict__ chunks,
                                                   int nchunks, SgdHP h) {
  ::tp::pdl_enter();
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    OptChunk ch = chunks[c];
    OptRow r = rows[ch.row];
    float* __restrict__ P = r.p + ch.start;
    const float* __restrict__ G = r.g + ch.start;
    float* __restrict__ B = r.s0 + ch.start;
    int len = ch.len, len4 = len >> 2;
    float4* P4 = reinterpret_cast<float4*>(P);
    const float4* G4 = reinterpret_cast<const float4*>(G);
    float4* B4 = reinterpret_cast<float4*>(B);
    // the updated parameter's tf32 low parts, for rows that keep them
    float* __restrict__ LO = r.lo ? r.lo + ch.start : nullptr;
    float4* LO4 = reinterpret_cast<float4*>(LO);
    int i = threadIdx.x;
    for (; i + (int)blockDim.x < len4; i += 2 * blockDim.x) {
      int j = i + blockDim.x;
      float4 p0 = P4[i], g0 = G4[i], p1 = P4[j], g1 = G4[j];
      float4 b0 = h.has_m ? B4[i] : make_float4(0, 0, 0, 0);
      float4 b1 = h.has_m ? B4[j] : make_float4(0, 0, 0, 0);
      sgd_elem(p0.x, g0.x, b0.x, h); sgd_elem(p0.y, g0.y, b0.y, h);
      sgd_elem(p0.z, g0.z, b0.z, h); sgd_elem(p0.w, g0.w, b0.w, h);
      sgd_elem(p1.x, g1.x, b1.x, h); sgd_elem(p1.y, g1.y, b1.y, h);
      sgd_elem(p1.z, g1.z, b1.z, h); sgd_elem(p1.w, g1.w, b1.w, h);
      P4[i] = p0; P4[j] = p1;
      if (h.has_m) { B4[i] = b0; B4[j] = b1; }
      if (LO4) { LO4[i] = tf32_lo4(p0); LO4[j] = tf32_lo4(p1); }
    }
    for (; i < len4; i += blockDim.x) {
      float4 p0 = P4[i], g0 = G4[i];
      float4 b0 = h.has_m ? B4[i] : make_float4(0, 0, 0, 0);
      sgd_elem(p0.x, g0.x, b0.x, h); sgd_elem(p0.y, g0.y, b0.y, h);
      sgd_elem(p0.z, g0.z, b0.z, h); sgd_elem(p0.w, g0.w, b0.w, h);
      P4[i] = p0;
      if (h.has_m) B4[i] = b0;
      if (LO4) LO4[i] = tf32_lo4(p0);
    }
    for (int k = (len4 << 2) + threadIdx.x; k < len; k += blockDim.x) {
      float p = P[k], b = h.has_m ? B[k] : 0.0f;
      sgd_elem(p, G[k], b, h);
      P[k] = p;
      if (h.has_m) B[k] = b;
      if (LO) LO[k] = p - __uint_as_float(__float_as_uint(p) & 0xFFFFE000u);
    }
  }
}

// ---- the other fused steps (rmsprop_step.wgsl, extended_step.wgsl) ---------------------
// Same multi-tensor walk; the per-element arithmetic is each entry point's,
// operation by operation, with round-to-nearest intrinsics (no contraction), so
// the results are bit-identical to the oracle's restatement.
enum ExtKind { EXT_RMSPROP = 0, EXT_ADAGRAD = 1, EXT_ADAMAX = 2, EXT_NADAM = 3, EXT_RADAM = 4 };

struct ExtHP {
  float lr, b1, b2, eps, wd;  // RMSprop: b1 = alpha; Adagrad uses lr, eps, wd
  float step_size;            // Adamax, NAdam, RAdam
  float x0, x1;               // RMSprop: momentum; Adamax: bias_correction1; NAdam: mu;
                              // RAdam: beta1^t, beta2^t
  float t;                    // RAdam: the step count as f32 (at least 1)
  int use_momentum;           // RMSprop
};

template <int KIND>
__device__ __forceinline__ void ext_elem(float& p, float g, float& s0, float& s1, const ExtHP& h) {
  if (h.wd != 0.0f) g = __fadd_rn(g, __fmul_rn(h.wd, p));
  if (KIND == EXT_RMSPROP) {  // rmsprop_step.wgsl:22-41
    const float sq = __fadd_rn(__fmul_rn(s0, h.b1), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, h.b1), g), g));
    s0 = sq;
    const float denom = __fadd_rn(__fsqrt_rn(sq), h.eps);
    float upd = __fdiv_rn(g, denom);
    if (h.use_momentum) {
      s1 = __fadd_rn(__fmul_rn(s1, h.x0), upd);
      upd = s1;
    }
    p = __fsub_rn(p, __fmul_rn(h.lr, upd));
  } else if (KIND == EXT_ADAGRAD) {  // extended_step.wgsl adagrad_step
    const float s = __fadd_rn(s0, __fmul_rn(g, g));
    s0 = s;
    const float sd = __fadd_rn(__fsqrt_rn(s), h.eps);
    p = __fsub_rn(p, __fdiv_rn(__fmul_rn(h.lr, g), sd));
  } else if (KIND == EXT_ADAMAX) {  // extended_step.wgsl adamax_step
    const float m = __fadd_rn(__fmul_rn(s0, h.b1), __fmul_rn(__fsub_rn(1.0f, h.b1), g));
    const float u = fmaxf(__fmul_rn(s1, h.b2), fabsf(g));
    s0 = m;
    s1 = u;
    const float denom = __fadd_rn(u, h.eps);
    p = __fsub_rn(p, __fmul_rn(__fmul_rn(__fdiv_rn(m, denom), h.step_size), h.x0));
  } else {
    const float m = __fadd_rn(__fmul_rn(s0, h.b1), __fmul_rn(__fsub_rn(1.0f, h.b1), g));
    const float v = __fadd_rn(__fmul_rn(s1, h.b2), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, h.b2), g), g));
    s0 = m;
    s1 = v;
    if (KIND == EXT_NADAM) {  // extended_step.wgsl nadam_step
      const float m_hat = __fadd_rn(__fmul_rn(h.x0, m), __fmul_rn(__fsub_rn(1.0f, h.x0), g));
      const float denom = __fadd_rn(__fsqrt_rn(v), h.eps);
      p = __fsub_rn(p, __fmul_rn(__fdiv_rn(m_hat, denom), h.step_size));
    } else {  // extended_step.wgsl radam_step
      const float m_hat = __fdiv_rn(m, __fsub_rn(1.0f, h.x0));
      const float rho_inf = __fsub_rn(__fdiv_rn(2.0f, __fsub_rn(1.0f, h.b2)), 1.0f);
      const float omb2t = __fsub_rn(1.0f, h.x1);
      const float rho_t =
          __fsub_rn(rho_inf, __fdiv_rn(__fmul_rn(__fmul_rn(2.0f, h.t), h.x1), fmaxf(omb2t, 1e-10f)));
      float upd;
      if (rho_t > 5.0f) {
        const float num = __fmul_rn(__fmul_rn(__fsub_rn(rho_t, 4.0f), __fsub_rn(rho_t, 2.0f)), rho_inf);
        const float den = __fmul_rn(__fmul_rn(__fsub_rn(rho_inf, 4.0f), __fsub_rn(rho_inf, 2.0f)), rho_t);
        const float rect = __fsqrt_rn(__fdiv_rn(num, den));
        upd = __fmul_rn(__fmul_rn(h.step_size, m_hat), rect);
      } else {
        upd = __fmul_rn(h.step_size, m_hat);
      }
      p = __fsub_rn(p, upd);
    }
  }
}

template <int KIND>
__global__ void __launch_bounds__(256) k_ext_multi(const OptRow* __restrict__ rows, const OptChunk* __restrict__ chunks,
                                                   int nchunks, ExtHP h) {
  ::tp::pdl_enter();
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    OptChunk ch = chunks[c];
    OptRow r = rows[ch.row];
    float* __restrict__ P = r.p + ch.start;
    const float* __restrict__ G = r.g + ch.start;
    float* __restrict__ S0 = r.s0 + ch.start;
    float* __restrict__ S1 = r.s1 + ch.start;
    // Adagrad keeps one state tensor, RMSprop without momentum never touches the second
    const bool two = KIND != EXT_ADAGRAD && (KIND != EXT_RMSPROP || h.use_momentum);
    const int len = ch.len, len4 = len >> 2;
    float4* P4 = reinterpret_cast<float4*>(P);
    const float4* G4 = reinterpret_cast<const float4*>(G);
    float4* A4 = reinterpret_cast<float4*>(S0);
    float4* B4 = reinterpret_cast<float4*>(S1);
    int i = threadIdx.x;
    // two float4 per thread per iteration, all loads issued before the math
    for (; i + (int)blockDim.x < len4; i += 2 * blockDim.x) {
      const int j = i + blockDim.x;
      float4 p0 = P4[i], g0 = G4[i], a0 = A4[i], p1 = P4[j], g1 = G4[j], a1 = A4[j];
      float4 b0 = two ? B4[i] : make_float4(0, 0, 0, 0);
      float4 b1 = two ? B4[j] : make_float4(0, 0, 0, 0);
      ext_elem<KIND>(p0.x, g0.x, a0.x, b0.x, h);
      ext_elem<KIND>(p0.y, g0.y, a0.y, b0.y, h);
      ext_elem<KIND>(p0.z, g0.z, a0.z, b0.z, h);
      ext_elem<KIND>(p0.w, g0.w, a0.w, b0.w, h);
      ext_elem<KIND>(p1.x, g1.x, a1.x, b1.x, h);
      ext_elem<KIND>(p1.y, g1.y, a1.y, b1.y, h);
      ext_elem<KIND>(p1.z, g1.z, a1.z, b1.z, h);
      ext_elem<KIND>(p1.w, g1.w, a1.w, b1.w, h);
      P4[i] = p0;
      A4[i] = a0;
      P4[j] = p1;
      A4[j] = a1;
      if (two) {
        B4[i] = b0;
        B4[j] = b1;
      }
    }
    for (; i < len4; i += blockDim.x) {
      float4 p = P4[i], g = G4[i], a = A4[i];
      float4 b = two ? B4[i] : make_float4(0, 0, 0, 0);
      ext_elem<KIND>(p.x, g.x, a.x, b.x, h);
      ext_elem<KIND>(p.y, g.y, a.y, b.y, h);
      ext_elem<KIND>(p.z, g.z, a.z, b.z, h);
      ext_elem<KIND>(p.w, g.w, a.w, b.w, h);
      P4[i] = p;
      A4[i] = a;
      if (two) B4[i] = b;
    }
    for (int k = (len4 << 2) + threadIdx.x; k < len; k += blockDim.x) {
      float p = P[k], a = S0[k], b = two ? S1[k] : 0.0f;
      ext_elem<KIND>(p, G[k], a, b, h);
      P[k] = p;
      S0[k] = a;
      if (two) S1[k] = b;
    }
  }
}

// ---- groups --------------------------------------------------------------------

struct Group {
  OptRow* rows = nullptr;
  OptChunk* chunks = nullptr;
  int nrows = 0;
  int nchunks = 0;
};

static std::unordered_map<int64_t, Group> g_groups;
static int64_t g_next_group = 1;

static Group build_group(const std::vector<OptRow>& rows) {
  std::vector<OptChunk> chunks;
  for (size_t r = 0; r < rows.size(); ++r) {
    const OptRow& x = rows[r];
    TP_REQUIRE((((uintptr_t)x.p | (uintptr_t)x.g | (uintptr_t)x.s0 | (uintptr_t)x.s1 | (uintptr_t)x.lo) & 15) == 0,
               "optimizer tensors must be 16-byte aligned");
    for (int64_t s = 0; s < x.n; s += OPT_CHUNK) {
      OptChunk c;
      c.row = (int32_t)r;
      c.start = s;
      c.len = (int32_t)(x.n - s < OPT_CHUNK ? x.n - s : OPT_CHUNK);
      chunks.push_back(c);
    }
  }
  Group g;
  g.nrows = (int)rows.size();
  g.nchunks = (int)chunks.size();
  size_t rb = rows.size() * sizeof(OptRow), cb = chunks.size() * sizeof(OptChunk);
  char* buf = (char*)dalloc(rb + cb + 16);
  g.rows = (OptRow*)buf;
  g.chunks = (OptChunk*)(buf + ((rb + 15) & ~(size_t)15));
  if (rb) TP_CUDA(cudaMemcpyAsync(g.rows, rows.data(), rb, cudaMemcpyHostToDevice, stream()));
  if (cb) TP_CUDA(cudaMemcpyAsync(g.chunks, chunks.data(), cb, cudaMemcpyHostToDevice, stream()));
  return g;
}

static void free_group(Group& g) {
  dfree(g.rows);
  g.rows = nullptr;
}

static unsigned opt_grid(int nchunks) {
  unsigned cap = (unsigned)sm_count() * 4;
  return (unsigned)(nchunks < (int)cap ? (nchunks > 0 ? nchunks : 1) : cap);
}

static AdamHP adam_hp(float lr, float b1, float b2, float eps, float wd, float ss, float isb) {
  AdamHP h;
  h.lr = lr; h.b1 = b1; h.b2 = b2; h.eps = eps; h.wd = wd; h.step_size = ss; h.inv_sqrt_bc2 = isb;
  h.omb1 = 1.0f - b1;  // f32 uniform arithmetic, as in the shader
  h.omb2 = 1.0f - b2;
  h.lrwd = lr * wd;
  return h;
}

void launch_adam_group(const Group& g, bool adamw, const AdamHP& h) {
  if (g.nchunks == 0) return;
  if (adamw) TP_LAUNCH(k_adam_multi<true>, opt_grid(g.nchunks), 256, 0, g.rows, g.chunks, g.nchunks, h);
  else TP_LAUNCH(k_adam_multi<false>, opt_grid(g.nchunks), 256, 0, g.rows, g.chunks, g.nchunks, h);
}

void launch_sgd_group(const Group& g, const SgdHP& h) {
  if (g.nchunks == 0) return;
  TP_LAUNCH(k_sgd_multi, opt_grid(g.nchunks), 256, 0, g.rows, g.chunks, g.nchunks, h);
}

static unsigned opt_grid(int nchunks);

template <int KIND>
static void launch_ext(const Group& g, const ExtHP& h) {
  if (g.nchunks == 0) return;
  TP_LAUNCH(k_ext_multi<KIND>, opt_grid(g.nchunks), 256, 0, g.rows, g.chunks, g.nchunks, h);
}

static void launch_ext_kind(int kind, const Group& g, const ExtHP& h) {
  switch (kind) {
    case EXT_RMSPROP: launch_ext<EXT_RMSPROP>(g, h); break;
    case EXT_ADAGRAD: launch_ext<EXT_ADAGRAD>(g, h); break;
    case EXT_ADAMAX: launch_ext<EXT_ADAMAX>(g, h); break;
    case EXT_NADAM: launch_ext<EXT_NADAM>(g, h); break;
    default: launch_ext<EXT_RADAM>(g, h); break;
  }
}

static std::vector<OptRow> rows_from_ids(const int64_t* p, const int64_t* gr, const int64_t* s0, const int64_t* s1,
                                         int n, const char* what) {
  std::vector<OptRow> rows((size_t)n);
  for (int i = 0; i < n; ++i) {
    Tensor& tp_ = get(p[i]);
    Tensor& tg = get(gr[i]);
    Tensor& t0 = get(s0[i]);
    Tensor* t1 = s1 ? &get(s1[i]) : nullptr;
    if (tg.numel != tp_.numel || t0.numel != tp_.numel || (t1 && t1->numel != tp_.numel))
      fail(TP_ERR_ARG, "%s: tensor lengths must match", what);
    rows[i] = OptRow{tp_.f(), tg.f(), t0.f(), t1 ? t1->f() : t0.f(), nullptr, tp_.numel};
  }
  return rows;
}

}  // namespace tp

using namespace tp;

extern "C" {

TP_API int tp_adamw_step_multi(const int64_t* p, const int64_t* g, const int64_t* m, const int64_t* v, int n,
                               float lr, float b1, float b2, float eps, float wd, float ss, float isb) {
  return guard([&] {
    Group grp = build_group(rows_from_ids(p, g, m, v, n, "adamWStep"));
    launch_adam_group(grp, true, adam_hp(lr, b1, b2, eps, wd, ss, isb));
    free_group(grp);
  });
}

TP_API int tp_adam_step_multi(const int64_t* p, const int64_t* g, const int64_t* m, const int64_t* v, int n,
                              float lr, float b1, float b2, float eps, float wd, float ss, float isb) {
  return guard([&] {
    Group grp = build_group(rows_from_ids(p, g, m, v, n, "adamStep"));
    launch_adam_group(grp, false, adam_hp(lr, b1, b2, eps, wd, ss, isb));
    free_group(grp);
  });
}

TP_API int tp_adamw_step(int64_t p, int64_t g, int64_t m, int64_t v, float lr, float b1, float b2, float eps,
                         float wd, float ss, float isb) {
  return tp_adamw_step_multi(&p, &g, &m, &v, 1, lr, b1, b2, eps, wd, ss, isb);
}

TP_API int tp_adam_step(int64_t p, int64_t g, int64_t m, int64_t v, float lr, float b1, float b2, float eps, float wd,
                        float ss, float isb) {
  return tp_adam_step_multi(&p, &g, &m, &v, 1, lr, b1, b2, eps, wd, ss, isb);
}

TP_API int tp_sgd_step_multi(const int64_t* p, const int64_t* g, const int64_t* b, int n, float lr, float mom,
                             float wd, float damp, int nesterov) {
  return guard([&] {
    Group grp = build_group(rows_from_ids(p, g, b, nullptr, n, "sgdStep"));
    SgdHP h{lr, mom, wd, 1.0f - damp, 1.0f, mom != 0.0f ? 1 : 0, nesterov ? 1 : 0};
    launch_sgd_group(grp, h);
    free_group(grp);
  });
}

TP_API int tp_sgd_step(int64_t p, int64_t g, int64_t b, float lr, float mom, float wd, float damp, int nesterov) {
  return tp_sgd_step_multi(&p, &g, &b, 1, lr, mom, wd, damp, nesterov);
}

TP_API int tpk_group_create_lo(int n, float* const* params, float* const* grads, float* const* state0,
                               float* const* state1, float* const* lo, const int64_t* numels, int64_t* out_group) {
  return guard([&] {
    TP_REQUIRE(n >= 0, "negative group size");
    std::vector<OptRow> rows((size_t)n);
    for (int i = 0; i < n; ++i)
      rows[i] = OptRow{params[i], grads[i], state0[i], state1 ? state1[i] : state0[i], lo ? lo[i] : nullptr,
                       numels[i]};
    Group g = build_group(rows);
    int64_t id = g_next_group++;
    g_groups[id] = g;
    *out_group = id;
  });
}

TP_API int tpk_group_create(int n, float* const* params, float* const* grads, float* const* state0,
                            float* const* state1, const int64_t* numels, int64_t* out_group) {
  return tpk_group_create_lo(n, params, grads, state0, state1, nullptr, numels, out_group);
}

TP_API int tpk_group_destroy(int64_t group) {
  return guard([&] {
    auto it = g_groups.find(group);
    if (it == g_groups.end()) return;
    free_group(it->second);
    g_groups.erase(it);
  });
}

TP_API int tpk_adam_group(int64_t group, int kind, float lr, float b1, float b2, float eps, float wd, float ss,
                          float isb) {
  return guard([&] {
    auto it = g_groups.find(group);
    TP_REQUIRE(it != g_groups.end(), "unknown tensor group %lld", (long long)group);
    launch_adam_group(it->second, kind == 0, adam_hp(lr, b1, b2, eps, wd, ss, isb));
  });
}

TP_API int tpk_sgd_group(int64_t group, float lr, float mom, float wd, float damp, int nesterov, float grad_scale) {
  return guard([&] {
    auto it = g_groups.find(group);
    TP_REQUIRE(it != g_groups.end(), "unknown tensor group %lld", (long long)group);
    SgdHP h{lr, mom, wd, 1.0f - damp, grad_scale, mom != 0.0f ? 1 : 0, nesterov ? 1 : 0};
    launch_sgd_group(it->second, h);
  });
}

static int ext_multi(int kind, const int64_t* p, const int64_t* g, const int64_t* s0, const int64_t* s1, int n,
                     const ExtHP& h, const char* what) {
  return guard([&] {
    TP_REQUIRE(n >= 0, "%s: negative tensor count", what);
    Group grp = build_group(rows_from_ids(p, g, s0, s1, n, what));
    launch_ext_kind(kind, grp, h);
    free_group(grp);
  });
}

static ExtHP ext_hp(float lr, float b1, float b2, float eps, float wd, float ss, float x0, float x1, float t,
                    int use_m) {
  ExtHP h;
  h.lr = lr; h.b1 = b1; h.b2 = b2; h.eps = eps; h.wd = wd; h.step_size = ss; h.x0 = x0; h.x1 = x1;
  h.t = t; h.use_momentum = use_m;
  return h;
}

TP_API int tp_rmsprop_step_multi(const int64_t* p, const int64_t* g, const int64_t* sq, const int64_t* mb, int n,
                                 float lr, float alpha, float eps, float wd, float momentum) {
  return ext_multi(EXT_RMSPROP, p, g, sq, mb, n,
                   ext_hp(lr, alpha, 0.0f, eps, wd, 0.0f, momentum, 0.0f, 0.0f, momentum != 0.0f ? 1 : 0),
                   "rmspropStep");
}

TP_API int tp_rmsprop_step(int64_t p, int64_t g, int64_t sq, int64_t mb, float lr, float alpha, float eps, float wd,
                           float momentum) {
  return tp_rmsprop_step_multi(&p, &g, &sq, &mb, 1, lr, alpha, eps, wd, momentum);
}

TP_API int tp_adagrad_step_multi(const int64_t* p, const int64_t* g, const int64_t* sum, int n, float lr, float eps,
                                 float wd) {
  return ext_multi(EXT_ADAGRAD, p, g, sum, nullptr, n, ext_hp(lr, 0.0f, 0.0f, eps, wd, 0.0f, 0.0f, 0.0f, 0.0f, 0),
                   "adagradStep");
}

TP_API int tp_adagrad_step(int64_t p, int64_t g, int64_t sum, float lr, float eps, float wd) {
  return tp_adagrad_step_multi(&p, &g, &sum, 1, lr, eps, wd);
}

TP_API int tp_adamax_step_multi(const int64_t* p, const int64_t* g, const int64_t* m, const int64_t* u, int n,
                                float lr, float b1, float b2, float eps, float wd, float step_size, float bc1) {
  return ext_multi(EXT_ADAMAX, p, g, m, u, n, ext_hp(lr, b1, b2, eps, wd, step_size, bc1, 0.0f, 0.0f, 0),
                   "adamaxStep");
}

TP_API int tp_adamax_step(int64_t p, int64_t g, int64_t m, int64_t u, float lr, float b1, float b2, float eps,
                          float wd, float step_size, float bc1) {
  return tp_adamax_step_multi(&p, &g, &m, &u, 1, lr, b1, b2, eps, wd, step_size, bc1);
}

TP_API int tp_nadam_step_multi(const int64_t* p, const int64_t* g, const int64_t* m, const int64_t* v, int n,
                               float lr, float b1, float b2, float eps, float wd, float step_size, float mu) {
  return ext_multi(EXT_NADAM, p, g, m, v, n, ext_hp(lr, b1, b2, eps, wd, step_size, mu, 0.0f, 0.0f, 0),
                   "nadamStep");
}

TP_API int tp_nadam_step(int64_t p, int64_t g, int64_t m, int64_t v, float lr, float b1, float b2, float eps,
                         float wd, float step_size, float mu) {
  return tp_nadam_step_multi(&p, &g, &m, &v, 1, lr, b1, b2, eps, wd, step_size, mu);
}

TP_API int tp_radam_step_multi(const int64_t* p, const int64_t* g, const int64_t* m, const int64_t* v, int n,
                               float lr, float b1, float b2, float eps, float wd, float step_size, float b1pow,
                               float b2pow, int64_t step) {
  const float t = (float)(step > 1 ? (uint32_t)step : 1u);  // max(f32(u32 step), 1.0)
  return ext_multi(EXT_RADAM, p, g, m, v, n, ext_hp(lr, b1, b2, eps, wd, step_size, b1pow, b2pow, t, 0),
                   "radamStep");
}

TP_API int tp_radam_step(int64_t p, int64_t g, int64_t m, int64_t v, float lr, float b1, float b2, float eps,
                         float wd, float step_size, float b1pow, float b2pow, int64_t step) {
  return tp_radam_step_multi(&p, &g, &m, &v, 1, lr, b1, b2, eps, wd, step_size, b1pow, b2pow, step);
}

}  // extern "C"
