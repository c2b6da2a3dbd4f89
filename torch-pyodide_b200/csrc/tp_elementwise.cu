// Element-wise, creation, RNG and layout kernels.
//
// The reference materialises every broadcast operand with expand_broadcast.wgsl
// before a same-shape element-wise dispatch (broadcastOps.ts:84-111) and copies
// buffers for reshape (shapeOps.ts:72-81).  Here a broadcast operand is read
// in place through zero strides, dimensions are collapsed on the host so the
// common patterns become rank <= 3, and same-shape operands use 128-bit loads.
#include <cuda_runtime.h>

#include <cmath>

#include "tp_core.h"
#include "tp_launch.h"
#include "tp_fastdiv.cuh"

namespace tp {

// ---- op tables -------------------------------------------------------------

// elementwise.wgsl:85-100 integer_pow: exponentiation by squaring in f32.
__device__ __forceinline__ float integer_pow(float base, float exponent) {
  float rounded = floorf(exponent + 0.5f);
  int n = (int)fabsf(rounded);
  float acc = 1.0f, factor = base;
  while (n > 0) {
    if ((n % 2) == 1) acc = __fmul_rn(acc, factor);
    factor = __fmul_rn(factor, factor);
    n = n / 2;
  }
  if (rounded < 0.0f) return 1.0f / acc;
  return acc;
}

__device__ __forceinline__ float binop(int op, float a, float b) {
  switch (op) {
    case TP_ADD: return __fadd_rn(a, b);
    case TP_SUB: return __fsub_rn(a, b);
    case TP_MUL: return __fmul_rn(a, b);
    case TP_DIV: return __fdiv_rn(a, b);
    case TP_POW: {  // elementwise.wgsl:103-114 pow_op
      float rounded = floorf(b + 0.5f);
      if (fabsf(b - rounded) < 0.000001f && fabsf(rounded) <= 64.0f) return integer_pow(a, b);
      return powf(a, b);
    }
    case TP_MAXIMUM: return fmaxf(a, b);
    case TP_MINIMUM: return fminf(a, b);
    case TP_EQ: return a == b ? 1.0f : 0.0f;  // compare.wgsl:8-55
    case TP_NE: return a != b ? 1.0f : 0.0f;
    case TP_LT: return a < b ? 1.0f : 0.0f;
    case TP_LE: return a <= b ? 1.0f : 0.0f;
    case TP_GT: return a > b ? 1.0f : 0.0f;
    case TP_GE: return a >= b ? 1.0f : 0.0f;
  }
  return __int_as_float(0x7fc00000);
}

__device__ __forceinline__ float unop(int op, float x) {
  switch (op) {  // unary.wgsl entry points
    case TP_NEG: return -x;
    case TP_ABS: return fabsf(x);
    case TP_SQRT: return sqrtf(x);
    case TP_EXP: return expf(x);
    case TP_LOG: return logf(x);
    case TP_RELU: return fmaxf(0.0f, x);
    case TP_RSQRT: return __fdiv_rn(1.0f, sqrtf(x));
    case TP_RECIPROCAL: return __fdiv_rn(1.0f, x);
    case TP_SQUARE: return __fmul_rn(x, x);
    case TP_SIGMOID: return __fdiv_rn(1.0f, 1.0f + expf(-x));
    case TP_TANH: return tanhf(x);
  }
  return __int_as_float(0x7fc00000);
}

// ---- kernels ----------------------------------------------------------------

__global__ void k_fill(float* __restrict__ out, int64_t n, float v) {
  ::tp::pdl_enter();
  int64_t n4 = n >> 2;
  float4 v4 = make_float4(v, v, v, v);
  float4* o4 = reinterpret_cast<float4*>(out);
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) o4[i] = v4;
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) out[i] = v;
}

// random.wgsl:11-21 xorshift and uint_to_float; :23-91 samplers.
__device__ __forceinline__ uint32_t xorshift32(uint32_t x) {
  x ^= x << 13;
  x ^= x >> 17;
  x ^= x << 5;
  return x;
}
__device__ __forceinline__ float u32_to_unit(uint32_t x) { return __fmul_rn(__uint2float_rn(x), 2.3283064365386963e-10f); }

__global__ void k_random(float* __restrict__ out, int64_t n, uint32_t seed, int kind, float p0, float p1) {
  ::tp::pdl_enter();
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    uint32_t idx = (uint32_t)i;
    uint32_t s1 = xorshift32(seed ^ (idx * 1664525u + 1013904223u));
    float r;
    if (kind == 0) {
      r = u32_to_unit(s1);
    } else if (kind == 1 || kind == 2) {
      uint32_t s2 = xorshift32(s1);
      float u1 = u32_to_unit(s1), u2 = u32_to_unit(s2);
      float rad = sqrtf(__fmul_rn(-2.0f, logf(fmaxf(u1, 0.0000001f))));
      float theta = __fmul_rn(6.283185307179586f, u2);
      float z = __fmul_rn(rad, cosf(theta));
      r = (kind == 1) ? z : __fadd_rn(p0, __fmul_rn(p1, z));
    } else if (kind == 3) {
      r = u32_to_unit(s1) < p0 ? 1.0f : 0.0f;
    } else {
      float u = fmaxf(u32_to_unit(s1), 1e-7f);
      r = __fdiv_rn(-logf(u), p0);
    }
    out[i] = r;
  }
}

__global__ void k_binary_same(int op, const float* __restrict__ a, const float* __restrict__ b,
                              float* __restrict__ out, int64_t n) {
  ::tp::pdl_enter();
  int64_t n4 = n >> 2;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float4* a4 = reinterpret_cast<const float4*>(a);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  float4* o4 = reinterpret_cast<float4*>(out);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 x = a4[i], y = b4[i];
    o4[i] = make_float4(binop(op, x.x, y.x), binop(op, x.y, y.y), binop(op, x.z, y.z), binop(op, x.w, y.w));
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = binop(op, a[i], b[i]);
}

// Up to 8 collapsed dims; operand strides are 0 on broadcast dims.
struct BcastGeom {
  int nd;
  int64_t size[TP_MAX_DIMS];
  int64_t sa[TP_MAX_DIMS];
  int64_t sb[TP_MAX_DIMS];
};

__global__ void k_binary_bcast(int op, const float* __restrict__ a, const float* __restrict__ b,
                               float* __restrict__ out, int64_t n, BcastGeom g) {
  ::tp::pdl_enter();
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t rem = i, ia = 0, ib = 0;
    for (int d = g.nd - 1; d >= 0; --d) {
      int64_t c = rem % g.size[d];
      rem /= g.size[d];
      ia += c * g.sa[d];
      ib += c * g.sb[d];
    }
    out[i] = binop(op, a[ia], b[ib]);
  }
}

// The common broadcast shapes after dim merging: [R][N] (R = 1 for a scalar
// operand) where each operand's inner stride is 1 (a full row) or 0 (one value
// per row), N % 4 == 0: 16-byte accesses along N and the row from one
// multiply-high instead of a 64-bit divide per dim and element.
__global__ void k_binary_2d(int op, const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out,
                            uint32_t n4, FastDiv fq, int64_t sa0, int sa1, int64_t sb0, int sb1) {
  ::tp::pdl_enter();
  const uint32_t stride = gridDim.x * blockDim.x;
  float4* o4 = reinterpret_cast<float4*>(out);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const uint32_t r = fq.div(i), c = (i - r * fq.d) * 4;
    const float* pa = a + (int64_t)r * sa0;
    const float* pb = b + (int64_t)r * sb0;
    const float4 x = sa1 ? *reinterpret_cast<const float4*>(pa + c) : make_float4(pa[0], pa[0], pa[0], pa[0]);
    const float4 y = sb1 ? *reinterpret_cast<const float4*>(pb + c) : make_float4(pb[0], pb[0], pb[0], pb[0]);
    o4[i] = make_float4(binop(op, x.x, y.x), binop(op, x.y, y.y), binop(op, x.z, y.z), binop(op, x.w, y.w));
  }
}

__global__ void k_unary(int op, const float* __restrict__ in, float* __restrict__ out, int64_t n) {
  ::tp::pdl_enter();
  int64_t n4 = n >> 2;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float4* i4 = reinterpret_cast<const float4*>(in);
  float4* o4 = reinterpret_cast<float4*>(out);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 x = i4[i];
    o4[i] = make_float4(unop(op, x.x), unop(op, x.y), unop(op, x.z), unop(op, x.w));
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = unop(op, in[i]);
}

__global__ void k_mul_scalar(const float* __restrict__ in, float v, float* __restrict__ out, int64_t n) {
  ::tp::pdl_enter();
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) out[i] = __fmul_rn(in[i], v);
}

// Generic strided gather: out[i] = in[sum coord_d * s_d] (expand, permute).
__global__ void k_gather(const float* __restrict__ in, float* __restrict__ out, int64_t n, BcastGeom g) {
  ::tp::pdl_enter();
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t rem = i, src = 0;
    for (int d = g.nd - 1; d >= 0; --d) {
      int64_t c = rem % g.size[d];
      rem /= g.size[d];
      src += c * g.sa[d];
    }
    out[i] = in[src];
  }
}

// 32x32 shared-memory tile transpose (transpose.wgsl semantics, coalesced).
__global__ void k_transpose2d(const float* __restrict__ in, float* __restrict__ out, int64_t rows, int64_t cols) {
  ::tp::pdl_enter();
  __shared__ float tile[32][33];
  int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    int64_t r = r0 + j, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[j][threadIdx.x] = in[r * cols + c];
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    int64_t c = c0 + j, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * rows + r] = tile[threadIdx.x][j];
  }
}

// ---- host helpers -------------------------------------------------------------

std::vector<int64_t> broadcast_shape(const Tensor& a, const Tensor& b) {
  int n = a.ndim > b.ndim ? a.ndim : b.ndim;
  std::vector<int64_t> out(n);
  for (int i = 0; i < n; ++i) {
    int ia = a.ndim - n + i, ib = b.ndim - n + i;
    int64_t ad = ia >= 0 ? a.shape[ia] : 1, bd = ib >= 0 ? b.shape[ib] : 1;
    if (ad != bd && ad != 1 && bd != 1) {
      std::string sa, sb;
      for (int k = 0; k < a.ndim; ++k) sa += (k ? "," : "") + std::to_string(a.shape[k]);
      for (int k = 0; k < b.ndim; ++k) sb += (k ? "," : "") + std::to_string(b.shape[k]);
      fail(TP_ERR_ARG, "Shapes [%s] and [%s] cannot be broadcast together.", sa.c_str(), sb.c_str());
    }
    out[i] = ad > bd ? ad : bd;
  }
  return out;
}

// Right-align a and b against out, compute zero-stride geometry and merge
// adjacent dims that share a broadcast pattern.
static BcastGeom make_geom(const std::vector<int64_t>& out, const Tensor& a, const Tensor* b) {
  int n = (int)out.size();
  int64_t sa[TP_MAX_DIMS], sb[TP_MAX_DIMS], ra = 1, rb = 1;
  for (int d = n - 1; d >= 0; --d) {
    int ia = a.ndim - n + d;
    int64_t ad = ia >= 0 ? a.shape[ia] : 1;
    sa[d] = ad == 1 ? 0 : ra;
    ra *= ad;
    if (b) {
      int ib = b->ndim - n + d;
      int64_t bd = ib >= 0 ? b->shape[ib] : 1;
      sb[d] = bd == 1 ? 0 : rb;
      rb *= bd;
    } else {
      sb[d] = 0;
    }
  }
  BcastGeom g;
  g.nd = 0;
  for (int d = 0; d < n; ++d) {
    if (out[d] == 1) continue;
    if (g.nd > 0) {
      int p = g.nd - 1;
      // merge with previous if both operands stay linear across the boundary
      if (g.sa[p] == sa[d] * out[d] && g.sb[p] == sb[d] * out[d]) {
        g.size[p] *= out[d];
        g.sa[p] = sa[d];
        g.sb[p] = sb[d];
        continue;
      }
    }
    g.size[g.nd] = out[d];
    g.sa[g.nd] = sa[d];
    g.sb[g.nd] = sb[d];
    g.nd++;
  }
  if (g.nd == 0) {
    g.nd = 1;
    g.size[0] = 1;
    g.sa[0] = 0;
    g.sb[0] = 0;
  }
  return g;
}

static inline bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

void launch_binary(int op, const float* a, const float* b, float* out, int64_t n) {
  if (n == 0) return;
  if (aligned16(a) && aligned16(b) && aligned16(out)) {
    TP_LAUNCH(k_binary_same, grid_for(n, 256, 4), 256, 0, op, a, b, out, n);
  } else {
    BcastGeom g;
    g.nd = 1;
    g.size[0] = n;
    g.sa[0] = 1;
    g.sb[0] = 1;
    TP_LAUNCH(k_binary_bcast, grid_for(n, 256), 256, 0, op, a, b, out, n, g);
  }
}

void launch_unary(int op, const float* in, float* out, int64_t n) {
  if (n == 0) return;
  TP_LAUNCH(k_unary, grid_for(n, 256, 4), 256, 0, op, in, out, n);
}

void launch_fill(float* out, int64_t n, float v) {
  if (n == 0) return;
  if (v == 0.0f && !signbit(v)) {
    TP_CUDA(cudaMemsetAsync(out, 0, (size_t)n * 4, stream()));
    return;
  }
  TP_LAUNCH(k_fill, grid_for(n, 256, 4), 256, 0, out, n, v);
}

static uint32_t g_seed = 42;  // creationOps.ts:17

static int64_t binary_impl(int op, int64_t ida, int64_t idb, tp_handle* out) {
  Tensor& a = get(ida);
  Tensor& b = get(idb);
  TP_REQUIRE(a.phys == PHYS_F32 && b.phys == PHYS_F32, "element-wise ops take float storage");
  std::vector<int64_t> oshape = broadcast_shape(a, b);
  int dtype = (op >= TP_EQ) ? TP_BOOL : a.dtype;
  Tensor o = make_like_shape(oshape, dtype);
  bool same = a.ndim == b.ndim && a.numel == b.numel;
  for (int i = 0; same && i < a.ndim; ++i) same = a.shape[i] == b.shape[i];
  if (same) {
    launch_binary(op, a.f(), b.f(), o.f(), o.numel);
  } else if (o.numel > 0) {
    BcastGeom g = make_geom(oshape, a, &b);
    // [R][N] fast path (see k_binary_2d)
    const bool two = g.nd == 2;
    const int64_t N = g.size[g.nd - 1], R = two ? g.size[0] : 1;
    const int64_t sa1 = g.sa[g.nd - 1], sb1 = g.sb[g.nd - 1], sa0 = two ? g.sa[0] : 0, sb0 = two ? g.sb[0] : 0;
    const bool fast = g.nd <= 2 && N % 4 == 0 && (sa1 == 0 || sa1 == 1) && (sb1 == 0 || sb1 == 1) &&
                      (sa1 == 0 || sa0 % 4 == 0) && (sb1 == 0 || sb0 % 4 == 0) && R * N / 4 < ((int64_t)1 << 31) &&
                      aligned16(a.f()) && aligned16(b.f()) && aligned16(o.f());
    if (fast) {
      const int64_t n4 = R * N / 4;
      TP_LAUNCH(k_binary_2d, grid_for(n4, 256), 256, 0, op, a.f(), b.f(), o.f(), (uint32_t)n4,
                fast_div((uint32_t)(N / 4)), sa0, (int)sa1, sb0, (int)sb1);
    } else {
      TP_LAUNCH(k_binary_bcast, grid_for(o.numel, 256), 256, 0, op, a.f(), b.f(), o.f(), o.numel, g);
    }
  }
  return emit(o, out);
}

}  // namespace tp

using namespace tp;

extern "C" {

TP_API int tp_full(const int64_t* shape, int ndim, int dtype, float value, tp_handle* out) {
  return guard([&] {
    Tensor t = make(shape, ndim, dtype);
    // creationOps.ts:147-169 coerceScalarByDType before the fill
    float v = value;
    if (dtype == TP_BOOL) v = value != 0.0f ? 1.0f : 0.0f;
    else if (dtype == TP_INT8 || dtype == TP_INT16 || dtype == TP_INT32 || dtype == TP_INT64) v = truncf(value);
    else if (dtype >= TP_UINT8 && dtype <= TP_UINT64) v = fmaxf(0.0f, truncf(value));
    launch_fill(t.f(), t.numel, v);
    emit(t, out);
  });
}

TP_API int tp_full_like(int64_t id, int dtype, float value, tp_handle* out) {
  Tensor* src = nullptr;
  int rc = guard([&] { src = &get(id); });
  if (rc) return rc;
  return tp_full(src->shape, src->ndim, dtype < 0 ? src->dtype : dtype, value, out);
}

TP_API int tp_fill(int64_t id, float value, tp_handle* out) {
  return guard([&] {
    Tensor& s = get(id);
    Tensor t = make(s.shape, s.ndim, s.dtype);
    launch_fill(t.f(), t.numel, value);
    emit(t, out);
  });
}

TP_API int tp_set_seed(uint32_t seed) {
  g_seed = seed;
  return TP_OK;
}

TP_API int tp_random(const int64_t* shape, int ndim, int dtype, int kind, float p0, float p1, tp_handle* out) {
  return guard([&] {
    TP_REQUIRE(kind >= 0 && kind <= 4, "unknown sampler kind %d", kind);
    Tensor t = make(shape, ndim, dtype);
    uint32_t seed = g_seed++;
    if (t.numel > 0) TP_LAUNCH(k_random, grid_for(t.numel, 256), 256, 0, t.f(), t.numel, seed, kind, p0, p1);
    emit(t, out);
  });
}

TP_API int tp_binary(int op, int64_t a, int64_t b, tp_handle* out) {
  return guard([&] {
    TP_REQUIRE((op >= TP_ADD && op <= TP_MINIMUM) || (op >= TP_EQ && op <= TP_GE), "unknown binary op %d", op);
    binary_impl(op, a, b, out);
  });
}
TP_API int tp_add(int64_t a, int64_t b, tp_handle* out) { return tp_binary(TP_ADD, a, b, out); }
TP_API int tp_sub(int64_t a, int64_t b, tp_handle* out) { return tp_binary(TP_SUB, a, b, out); }
TP_API int tp_mul(int64_t a, int64_t b, tp_handle* out) { return tp_binary(TP_MUL, a, b, out); }
TP_API int tp_div(int64_t a, int64_t b, tp_handle* out) { return tp_binary(TP_DIV, a, b, out); }
TP_API int tp_pow(int64_t a, int64_t b, tp_handle* out) { return tp_binary(TP_POW, a, b, out); }
TP_API int tp_gt(int64_t a, int64_t b, tp_handle* out) { return tp_binary(TP_GT, a, b, out); }

TP_API int tp_mul_scalar(int64_t id, float value, tp_handle* out) {
  return guard([&] {
    Tensor& a = get(id);
    Tensor o = make(a.shape, a.ndim, a.dtype);
    if (o.numel > 0) TP_LAUNCH(k_mul_scalar, grid_for(o.numel, 256), 256, 0, a.f(), value, o.f(), o.numel);
    emit(o, out);
  });
}

TP_API int tp_unary(int op, int64_t id, tp_handle* out) {
  return guard([&] {
    TP_REQUIRE(op >= TP_NEG && op <= TP_TANH, "unknown unary op %d", op);
    Tensor& a = get(id);
    TP_REQUIRE(a.phys == PHYS_F32, "unary ops take float storage");
    Tensor o = make(a.shape, a.ndim, a.dtype);
    launch_unary(op, a.f(), o.f(), o.numel);
    emit(o, out);
  });
}
TP_API int tp_relu(int64_t a, tp_handle* out) { return tp_unary(TP_RELU, a, out); }
TP_API int tp_rsqrt(int64_t a, tp_handle* out) { return tp_unary(TP_RSQRT, a, out); }
TP_API int tp_neg(int64_t a, tp_handle* out) { return tp_unary(TP_NEG, a, out); }

TP_API int tp_reshape(int64_t id, const int64_t* shape, int ndim, tp_handle* out) {
  return guard([&] {
    Tensor& a = get(id);
    int64_t n = prod(shape, ndim);
    if (n != a.numel) {
      std::string s;
      for (int k = 0; k < ndim; ++k) s += (k ? "," : "") + std::to_string(shape[k]);
      fail(TP_ERR_ARG, "reshape: product %s != %lld", s.c_str(), (long long)a.numel);
    }
    Tensor o = make(shape, ndim, a.dtype, a.phys);
    if (n > 0) TP_CUDA(cudaMemcpyAsync(o.ptr, a.ptr, (size_t)n * 4, cudaMemcpyDeviceToDevice, stream()));
    emit(o, out);
  });
}

TP_API int tp_transpose2d(int64_t id, tp_handle* out) {
  return guard([&] {
    Tensor& a = get(id);
    TP_REQUIRE(a.ndim == 2, "transpose2d expects a 2-D tensor, got rank %d", a.ndim);
    int64_t rows = a.shape[0], cols = a.shape[1];
    int64_t s[2] = {cols, rows};
    Tensor o = make(s, 2, a.dtype, a.phys);
    if (a.numel > 0) {
      dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
      TP_LAUNCH(k_transpose2d, grid, dim3(32, 8), 0, a.f(), o.f(), rows, cols);
    }
    emit(o, out);
  });
}

TP_API int tp_permute(int64_t id, const int32_t* dims, int ndim, tp_handle* out) {
  return guard([&] {
    Tensor& a = get(id);
    TP_REQUIRE(ndim == a.ndim, "permute: dims length mismatch");
    int64_t instr[TP_MAX_DIMS], r = 1;
    for (int d = a.ndim - 1; d >= 0; --d) {
      instr[d] = r;
      r *= a.shape[d];
    }
    bool seen[TP_MAX_DIMS] = {false};
    std::vector<int64_t> oshape(ndim);
    BcastGeom g;
    g.nd = ndim;
    for (int d = 0; d < ndim; ++d) {
      int s = dims[d] < 0 ? dims[d] + ndim : dims[d];
      TP_REQUIRE(s >= 0 && s < ndim && !seen[s], "permute: invalid dims");
      seen[s] = true;
      oshape[d] = a.shape[s];
      g.size[d] = a.shape[s];
      g.sa[d] = instr[s];
      g.sb[d] = 0;
    }
    if (ndim == 0) {
      g.nd = 1;
      g.size[0] = 1;
      g.sa[0] = 0;
    }
    Tensor o = make_like_shape(oshape, a.dtype, a.phys);
    if (o.numel > 0) TP_LAUNCH(k_gather, grid_for(o.numel, 256), 256, 0, a.f(), o.f(), o.numel, g);
    emit(o, out);
  });
}

TP_API int tp_expand(int64_t id, const int64_t* shape, int ndim, tp_handle* out) {
  return guard([&] {
    Tensor& a = get(id);
    TP_REQUIRE(ndim >= a.ndim, "expand: target rank %d below tensor rank %d", ndim, a.ndim);
    std::vector<int64_t> oshape(shape, shape + ndim);
    for (int d = 0; d < a.ndim; ++d) {
      int64_t od = oshape[ndim - a.ndim + d];
      TP_REQUIRE(a.shape[d] == od || a.shape[d] == 1, "expand: size %lld cannot expand to %lld",
                 (long long)a.shape[d], (long long)od);
    }
    Tensor o = make_like_shape(oshape, a.dtype, a.phys);
    if (o.numel > 0) {
      BcastGeom g = make_geom(oshape, a, nullptr);
      TP_LAUNCH(k_gather, grid_for(o.numel, 256), 256, 0, a.f(), o.f(), o.numel, g);
    }
    emit(o, out);
  });
}

}  // extern "C"
