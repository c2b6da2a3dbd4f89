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
// Per-CTA sums of the weight gradient are combined over pixel lanes in shared
// memory in a fixed order and the per-CTA partials in f64 by a second kernel
// in a fixed order, so the gradient is the same on every run.
#include <cuda_runtime.h>

#include "tp_core.h"
#include "tp_launch.h"

namespace tp {

constexpr int SC_THREADS = 256;

// A 16-byte shared-memory load the compiler keeps in place (so filter vectors
// are re-read per row instead of all 36 being held in registers).
__device__ __forceinline__ float4 lds4(const float4* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
  return v;
}

// Forward: thread = (image row lane, CH consecutive output pixels of the row,
// 4 output channels).  Per filter row kh it loads the CH + 2 input pixels
// (16-byte vectors) once and reuses each filter vector from shared memory for
// all CH pixels.
template <int CH>
__global__ void __launch_bounds__(SC_THREADS, 2)
    k_conv_c4_fwd(const float4* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias,
                  float4* __restrict__ y, int rows, int H, int W, int OH, int OW, int PH, int PW, int Cout) {
  ::tp::pdl_enter();
  extern __shared__ float4 wsm[];  // [tap][ci][G]: (w[4g..4g+3][ci][tap])
  const int G = Cout >> 2;
  for (int i = threadIdx.x; i < 9 * 4 * G; i += blockDim.x) {
    const int g = i % G, ci = (i / G) & 3, tap = i / (4 * G);
    float4 v;
    v.x = w[((4 * g + 0) * 4 + ci) * 9 + tap];
    v.y = w[((4 * g + 1) * 4 + ci) * 9 + tap];
    v.z = w[((4 * g + 2) * 4 + ci) * 9 + tap];
    v.w = w[((4 * g + 3) * 4 + ci) * 9 + tap];
    wsm[i] = v;
  }
  __syncthreads();
  const int per_row = (OW / CH) * G, lanes = SC_THREADS / per_row;
  const int rl = threadIdx.x / per_row, rem = threadIdx.x % per_row, g = rem % G, ow0 = (rem / G) * CH;
  if (rl >= lanes) return;
  const float4 b4 = bias ? reinterpret_cast<const float4*>(bias)[g] : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int row = blockIdx.x * lanes + rl; row < rows; row += gridDim.x * lanes) {
    const int n = row / OH, oh = row - n * OH;
    float4 acc[CH];
#pragma unroll
    for (int p = 0; p < CH; ++p) acc[p] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int kh = 0; kh < 3; ++kh) {
      const int ih = oh + kh - PH;
      const bool rok = ih >= 0 && ih < H;
      const float4* xr = x + ((int64_t)n * H + ih) * W;
      float4 xv[CH + 2];
#pragma unroll
      for (int j = 0; j < CH + 2; ++j) {
        const int iw = ow0 - PW + j;
        xv[j] = (rok && iw >= 0 && iw < W) ? xr[iw] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int kw = 0; kw < 3; ++kw) {
#pragma unroll
        for (int ci = 0; ci < 4; ++ci) {
          const float4 wv = lds4(&wsm[((kh * 3 + kw) * 4 + ci) * G + g]);
#pragma unroll
          for (int p = 0; p < CH; ++p) {
            const float4 q = xv[p + kw];
            const float xs = ci == 0 ? q.x : (ci == 1 ? q.y : (ci == 2 ? q.z : q.w));
            acc[p].x = fmaf(xs, wv.x, acc[p].x);
            acc[p].y = fmaf(xs, wv.y, acc[p].y);
            acc[p].z = fmaf(xs, wv.z, acc[p].z);
            acc[p].w = fmaf(xs, wv.w, acc[p].w);
          }
        }
      }
    }
    float4* yr = y + ((int64_t)row * OW + ow0) * G + g;
#pragma unroll
    for (int p = 0; p < CH; ++p)
      yr[(int64_t)p * G] = make_float4(acc[p].x + b4.x, acc[p].y + b4.y, acc[p].z + b4.z, acc[p].w + b4.w);
  }
}

// Weight gradient: thread = (row lane r, input channel ci, 4 output channels).
// Lane r takes rows row0 + r, row0 + r + R, ... of the CTA's range [row0,
// row1) and walks each whole output row with the 3x3 input window in
// registers, loading one new window column (3 values) and one 16-byte dy
// vector per pixel, 8 pixels' loads issued before their 288 multiply-adds so
// the loads' latency is covered by the other warps' arithmetic.
constexpr int C4W_PIX = 8;
__global__ void __launch_bounds__(SC_THREADS, 2)
    k_conv_c4_wgrad(const float4* __restrict__ dy, const float* __restrict__ x, float* __restrict__ part, int rows,
                    int H, int W, int OH, int OW, int PH, int PW, int Cout, int rows_per_split) {
  ::tp::pdl_enter();
  extern __shared__ float sh[];  // [R][Cout][4][9]
  const int G = Cout >> 2, R = SC_THREADS / (4 * G);
  const int g = threadIdx.x % G, ci = (threadIdx.x / G) & 3, r = threadIdx.x / (4 * G);
  const int row0 = blockIdx.x * rows_per_split, row1 = min(row0 + rows_per_split, rows);
  float acc[9][4];
#pragma unroll
  for (int t = 0; t < 9; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
  for (int row = row0 + r; row < row1 && r < R; row += R) {
    const int n = row / OH, oh = row - n * OH;
    const float* xr[3];
    bool rok[3];
#pragma unroll
    for (int kh = 0; kh < 3; ++kh) {
      const int ih = oh + kh - PH;
      rok[kh] = ih >= 0 && ih < H;
      xr[kh] = x + (((int64_t)n * H + ih) * W) * 4 + ci;
    }
    float win[3][3];
#pragma unroll
    for (int kh = 0; kh < 3; ++kh)
#pragma unroll
      for (int kw = 0; kw < 2; ++kw) {
        const int iw = kw - PW;
        win[kh][kw] = (rok[kh] && iw >= 0 && iw < W) ? xr[kh][iw * 4] : 0.0f;
      }
    const float4* dr = dy + (int64_t)row * OW * G + g;
    for (int ow8 = 0; ow8 < OW; ow8 += C4W_PIX) {
      float col[C4W_PIX][3];
      float4 d[C4W_PIX];
#pragma unroll
      for (int q = 0; q < C4W_PIX; ++q) {
        const int iw = ow8 + q - PW + 2;
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) col[q][kh] = (rok[kh] && iw >= 0 && iw < W) ? xr[kh][iw * 4] : 0.0f;
        d[q] = dr[(int64_t)(ow8 + q) * G];
      }
#pragma unroll
      for (int q = 0; q < C4W_PIX; ++q) {
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) win[kh][2] = col[q][kh];
#pragma unroll
        for (int kh = 0; kh < 3; ++kh)
#pragma unroll
          for (int kw = 0; kw < 3; ++kw) {
            const float v = win[kh][kw];
            float* a = acc[kh * 3 + kw];
            a[0] = fmaf(v, d[q].x, a[0]);
            a[1] = fmaf(v, d[q].y, a[1]);
            a[2] = fmaf(v, d[q].z, a[2]);
            a[3] = fmaf(v, d[q].w, a[3]);
          }
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
          win[kh][0] = win[kh][1];
          win[kh][1] = win[kh][2];
        }
      }
    }
  }
  if (r < R) {
#pragma unroll
    for (int t = 0; t < 9; ++t)
#pragma unroll
      for (int j = 0; j < 4; ++j) sh[(((int64_t)r * Cout + 4 * g + j) * 4 + ci) * 9 + t] = acc[t][j];
  }
  __syncthreads();
  const int per = Cout * 36;
  for (int i = threadIdx.x; i < per; i += blockDim.x) {
    float s = 0.0f;
    for (int k = 0; k < R; ++k) s += sh[(int64_t)k * per + i];
    part[(int64_t)blockIdx.x * per + i] = s;
  }
}

// dw[i] = sum over splits of part[split][i] in f64: each of a block's 8 warps
// sums a contiguous slice of splits for 32 consecutive i, then the slices are
// added in slice order (deterministic).  i = (co*4 + ci)*9 + tap.  A slice's
// values are loaded 8 at a time before they are added (in order), so the loads
// overlap instead of each waiting for the previous add.
__global__ void k_conv_c4_wgrad_finish(const float* __restrict__ part, int splits, int per, float* __restrict__ dw) {
  ::tp::pdl_enter();
  __shared__ double sl[8][32];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + lane;
  const int per_w = (splits + 7) / 8, k0 = wp * per_w, k1 = min(k0 + per_w, splits);
  double s = 0.0;
  if (i < per) {
    int k = k0;
    for (; k + 8 <= k1; k += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = part[(int64_t)(k + u) * per + i];
#pragma unroll
      for (int u = 0; u < 8; ++u) s += v[u];
    }
    for (; k < k1; ++k) s += part[(int64_t)k * per + i];
  }
  sl[wp][lane] = s;
  __syncthreads();
  if (wp == 0 && i < per) {
    double t = 0.0;
    for (int k = 0; k < 8; ++k) t += sl[k][lane];
    dw[i] = (float)t;
  }
}

// ---- data gradient for a few input channels (NCHW dx), any stride ----------------------------
// dx[n][ci][ih][iw] = sum over (co, kh, kw) with ih + P - kh = oh*S (and the same
// for w) of dy[n][co][oh][ow] * w[co][ci][kh][kw], dy read channels-last.
// Input pixels are taken phase by phase (ih mod S, iw mod S), so the threads
// of a warp share their filter taps: thread = (n, phase, y', x'), 4 input
// channels in registers, filter taps from shared memory as float4 over ci.
// The reference's stride-aware data-gradient shader does the same sum one
// thread per input element (conv_backward.wgsl:24-61).
__global__ void __launch_bounds__(256)
    k_conv_dgrad_smallc(const float4* __restrict__ dy, const float* __restrict__ w, float* __restrict__ dx, int N,
                        int Cin, int H, int W, int Cout, int OH, int OW, int KH, int KW, int S, int P) {
  ::tp::pdl_enter();
  extern __shared__ float4 wt[];  // [kh][kw][co]: (w[co][0..3][kh][kw])
  const int T = KH * KW, G = Cout >> 2;
  for (int i = threadIdx.x; i < T * Cout; i += blockDim.x) {
    const int co = i % Cout, tap = i / Cout;
    float v[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) v[c] = c < Cin ? w[((int64_t)co * Cin + c) * T + tap] : 0.0f;
    wt[i] = make_float4(v[0], v[1], v[2], v[3]);
  }
  __syncthreads();
  // phase grid: per image S*S phases of ceil(H/S) x ceil(W/S) input pixels
  const int HP = (H + S - 1) / S, WP = (W + S - 1) / S;
  const int64_t per_img = (int64_t)S * S * HP * WP;
  const int64_t total = (int64_t)N * per_img;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(t / per_img);
    int64_t r = t - (int64_t)n * per_img;
    const int xq = (int)(r % WP);
    r /= WP;
    const int yq = (int)(r % HP);
    const int ph = (int)(r / HP);
    const int rh = ph / S, rw = ph - (ph / S) * S;
    const int ih = yq * S + rh, iw = xq * S + rw;
    if (ih >= H || iw >= W) continue;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int kh = (rh + P) % S; kh < KH; kh += S) {
      const int oh = (ih + P - kh) / S;
      if (oh < 0 || oh >= OH) continue;
      for (int kw = (rw + P) % S; kw < KW; kw += S) {
        const int ow = (iw + P - kw) / S;
        if (ow < 0 || ow >= OW) continue;
        const float4* drow = dy + (((int64_t)n * OH + oh) * OW + ow) * G;
        const float4* wrow = wt + (kh * KW + kw) * Cout;
        for (int g = 0; g < G; ++g) {
          const float4 d = drow[g];
          const float ds[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 q = wrow[4 * g + j];
            acc[0] = fmaf(ds[j], q.x, acc[0]);
            acc[1] = fmaf(ds[j], q.y, acc[1]);
            acc[2] = fmaf(ds[j], q.z, acc[2]);
            acc[3] = fmaf(ds[j], q.w, acc[3]);
          }
        }
      }
    }
    for (int c = 0; c < Cin; ++c) dx[(((int64_t)n * Cin + c) * H + ih) * W + iw] = acc[c];
  }
}

// NCHW data gradient for Cin <= 4 through a channels-last copy of dy; false
// if the shape does not qualify.
bool conv_dgrad_smallc(const float* dy, const float* w, float* dx, int64_t N, int64_t Cin, int64_t H, int64_t W,
                       int64_t Cout, int64_t OH, int64_t OW, int KH, int KW, int S, int PH, int PW, bool same_stride) {
  if (Cin > 4 || Cout % 4 || Cout > 256 || KH * KW > 49 || !same_stride || PH != PW || KH != KW) return false;
  if (N * OH * OW * Cout >= ((int64_t)1 << 31) || N * Cin * H * W >= ((int64_t)1 << 31)) return false;
  float* dyn = (float*)dalloc((size_t)N * OH * OW * Cout * 4);
  transpose_nchw_nhwc(dy, dyn, N, Cout, OH * OW, true);
  const size_t shb = (size_t)KH * KW * Cout * sizeof(float4);
  static bool attr = false;
  if (!attr) {
    TP_CUDA(cudaFuncSetAttribute(k_conv_dgrad_smallc, cudaFuncAttributeMaxDynamicSharedMemorySize, 49 * 256 * 16));
    attr = true;
  }
  const int64_t HP = (H + S - 1) / S, WP = (W + S - 1) / S, total = N * S * S * HP * WP;
  int64_t blocks = (total + 255) / 256, cap = (int64_t)sm_count() * 16;
  TP_LAUNCH(k_conv_dgrad_smallc, (unsigned)(blocks < cap ? blocks : cap), 256, shb,
            reinterpret_cast<const float4*>(dyn), w, dx, (int)N, (int)Cin, (int)H, (int)W, (int)Cout, (int)OH,
            (int)OW, KH, KW, S, PH);
  dfree(dyn);
  return true;
}

// True when the 4-channel kernels apply: x has exactly 4 channels, 3x3
// filters, 64 <= Cout <= 256 with Cout % 4 == 0, output rows a multiple of 16
// wide, 16-byte aligned buffers.
bool conv_c4_ok(int64_t N, int64_t H, int64_t W, int64_t Cin, int KH, int KW, int64_t Cout, const void* a,
                const void* b) {
  (void)H;
  return Cin == 4 && KH == 3 && KW == 3 && Cout % 4 == 0 && Cout >= 64 && Cout <= 256 && W % 16 == 0 && W <= 256 &&
         ((uintptr_t)a & 15) == 0 && ((uintptr_t)b & 15) == 0 && N * (H + 2) * (W + 2) * Cout < ((int64_t)1 << 31);
}

void conv_c4_fwd(const float* x, const float* w, const float* bias, float* y, int64_t N, int64_t H, int64_t W,
                 int64_t Cout, int PH, int PW) {
  const int OH = (int)(H + 2 * PH - 2), OW = (int)(W + 2 * PW - 2);
  const int64_t rows = N * OH;
  if (rows == 0 || OW <= 0) return;
  TP_REQUIRE(OW % 8 == 0, "conv2d (4 channels): output width must be a multiple of 8");
  TP_REQUIRE(bias == nullptr || ((uintptr_t)bias & 15) == 0, "conv2d: bias must be 16-byte aligned");
  const int G = (int)(Cout / 4), per_row = (OW / 8) * G;
  TP_REQUIRE(per_row <= SC_THREADS, "conv2d (4 channels): row too wide");
  const int lanes = SC_THREADS / per_row;
  size_t shb = (size_t)9 * 4 * G * sizeof(float4);
  int64_t blocks = (rows + lanes - 1) / lanes;
  int64_t cap = (int64_t)sm_count() * 4;
  auto kfn = k_conv_c4_fwd<8>;
  TP_LAUNCH(kfn, (unsigned)(blocks < cap ? blocks : cap), SC_THREADS, shb, reinterpret_cast<const float4*>(x), w,
            bias, reinterpret_cast<float4*>(y), (int)rows, (int)H, (int)W, OH, OW, PH, PW, (int)Cout);
}

void conv_c4_wgrad(const float* dy, const float* x, float* dw, int64_t N, int64_t H, int64_t W, int64_t Cout, int PH,
                   int PW) {
  const int OH = (int)(H + 2 * PH - 2), OW = (int)(W + 2 * PW - 2);
  const int64_t rows = N * OH;
  const int per = (int)(Cout * 36);
  const int G = (int)(Cout / 4), R = SC_THREADS / (4 * G);
  TP_REQUIRE(R >= 1 && OW % C4W_PIX == 0, "conv2d weight gradient (4 channels): unsupported width");
  // two CTAs per SM, but at least 2 rows per row lane (batch 128: 296 CTAs of 14
  // rows instead of 128 of 32 -- a single half-full wave took 44 us)
  int64_t splits = (int64_t)sm_count() * 2;
  if (splits > rows / (2 * R)) splits = rows / (2 * R);
  if (splits < 1) splits = 1;
  const int64_t rps = rows > 0 ? (rows + splits - 1) / splits : 1;
  splits = rows > 0 ? (rows + rps - 1) / rps : 1;
  float* part = (float*)scratch((size_t)splits * per * sizeof(float));
  if (rows > 0 && OW > 0) {
    size_t shb = (size_t)R * per * sizeof(float);
    TP_LAUNCH(k_conv_c4_wgrad, (unsigned)splits, SC_THREADS, shb, reinterpret_cast<const float4*>(dy), x, part,
              (int)rows, (int)H, (int)W, OH, OW, PH, PW, (int)Cout, (int)rps);
  } else {
    TP_CUDA(cudaMemsetAsync(part, 0, (size_t)per * sizeof(float), stream()));
    splits = 1;
  }
  TP_LAUNCH(k_conv_c4_wgrad_finish, (unsigned)((per + 31) / 32), 256, 0, part, (int)splits, per, dw);
}

}  // namespace tp
