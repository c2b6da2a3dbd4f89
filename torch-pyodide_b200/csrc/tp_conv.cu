// Dense contractions of the hot path: matmul / linear and conv2d forward,
// data-gradient, weight-gradient and bias-gradient, all as gather-GEMMs.
//
// Reference: matmul.wgsl:52-85 (one thread per output, sequential k, the tiled
// entry :17-50 unused), conv.wgsl:25-60 and conv_backward.wgsl:24-119 (one
// thread per output / input / weight element with serial loops).  The
// implicit-GEMM mappings (tp_gemm.cuh) never materialise im2col or a
// transposed operand.
#include <cuda_runtime.h>

#include <vector>

#include "tp_core.h"
#include "tp_launch.h"
#include "tp_gemm_dispatch.cuh"
#include "tp_chanred.cuh"

namespace tp {

// Kernel selection (tp_gemm_dispatch.cuh): 0 TMA (CTA pairs for large N) /
// gather tensor cores, 1 CUDA cores only, 2 gather tensor cores without TMA, 3
// as 0 without CTA pairs, 4 as 0 with CTA pairs wherever they fit.
static int g_gemm_path = 0;
int gemm_path() { return g_gemm_path; }
static int g_gemm_twocta = 1;
int gemm_twocta() { return g_gemm_twocta; }

// Most k-blocks (32 k each) one split of a tensor-core GEMM accumulates in
// TMEM once K exceeds 4x that (0: no cap).  Over thousands of MMAs into one
// fp32 accumulator the sum drifts (measured on the 7x7 stride-2 weight
// gradient over 1.6 M pixels: 3.0e-4 of the output scale uncapped, 1.1e-4 at
// 512, 3.1e-5 at 128, 1.5e-5 at 64 k-blocks per split), so long reductions are
// cut into splits whose partials are added on CUDA cores.
static int g_gemm_kmax = 64;
int gemm_kmax() { return g_gemm_kmax; }

// Each translation unit that holds tensor-core kernels has its own copy of
// tc::g_status (this one and tp_conv_nhwc.cu), and the one-launch BatchNorm of
// tp_norm.cu has its own word; the status is the first nonzero.
int tc_status(bool reset) {
  int v = 0;
  TP_CUDA(cudaMemcpyFromSymbol(&v, tc::g_status, sizeof(int)));
  if (reset && v) {
    int z = 0;
    TP_CUDA(cudaMemcpyToSymbol(tc::g_status, &z, sizeof(int)));
  }
  const int w = tc_status_nhwc(reset);
  const int n = norm_status(reset);
  return v ? v : (w ? w : n);
}

// ---- per-channel sum of an NCHW tensor (conv_backward.wgsl:103-119) ---------------
__global__ void k_channel_sum_finish(const double* __restrict__ part, int64_t C, int splits,
                                     float* __restrict__ out) {
  ::tp::pdl_enter();
  int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (c >= C) return;
  double s = 0.0;
  for (int k = 0; k < splits; ++k) s += part[(c * splits + k) * 2];
  out[c] = (float)s;
}

void launch_channel_sum(const float* x, int64_t N, int64_t C, int64_t P, float* out) {
  if (C == 0) return;
  int splits = chan_splits(C, N, P, sm_count());
  double* part = (double*)scratch((size_t)C * splits * 2 * sizeof(double));
  auto kcs = k_chan_reduce<ChanSumF>;
  TP_LAUNCH(kcs, dim3((unsigned)C, (unsigned)splits), 256, 0, ChanSumF{x}, N, C, P, splits, part, chan_div4(P),
            chan_div1(P));
  TP_LAUNCH(k_channel_sum_finish, (unsigned)((C + 127) / 128), 128, 0, part, C, splits, out);
}

// ---- convolution launchers (pointer level) -------------------------------------------
ConvShape conv_shape(int64_t N, int64_t Cin, int64_t H, int64_t W, int64_t Cout, int KH, int KW, int SH, int SW,
                     int PH, int PW, int groups) {
  TP_REQUIRE(SH > 0 && SW > 0 && PH >= 0 && PW >= 0 && KH > 0 && KW > 0, "conv2d: invalid stride/padding/kernel");
  TP_REQUIRE(groups >= 1 && Cin % groups == 0 && Cout % groups == 0, "conv2d: channels not divisible by groups");
  ConvShape s;
  s.N = N;
  s.Cin = Cin;
  s.H = H;
  s.W = W;
  s.Cout = Cout;
  s.KH = KH;
  s.KW = KW;
  s.SH = SH;
  s.SW = SW;
  s.PH = PH;
  s.PW = PW;
  s.icpg = (int)(Cin / groups);
  s.ocpg = (int)(Cout / groups);
  s.OH = (H + 2 * PH - KH) / SH + 1;  // convOps.ts:35-36 (dilation ignored)
  s.OW = (W + 2 * PW - KW) / SW + 1;
  TP_REQUIRE(s.OH > 0 && s.OW > 0, "conv2d: output would be empty");
  return s;
}

// Repack filters for the filter-major K order k = (kh, kw, c):
//   mode 0 (forward):  wp[o][tap][c] = w[o][c][tap]             (o < Cout, c < icpg)
//   mode 1 (dgrad):    wp[i][tap][o] = w[o][i][KHW-1-tap]        (flipped, in/out swapped)
//   mode 2 (dgrad):    the same from filters stored w[o][tap][i]
__global__ void k_pack_filters(const float* __restrict__ w, float* __restrict__ wp, int64_t Cout, int64_t Cin_pg,
                               int khw, int mode) {
  ::tp::pdl_enter();
  int64_t total = Cout * Cin_pg * khw;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    int tap = (int)(i % khw);
    int64_t t = i / khw;
    int64_t c = t % Cin_pg, o = t / Cin_pg;  // w index i = (o*Cin_pg + c)*khw + tap
    if (mode == 2) {  // source stored [o][tap][c] (same flipped, transposed destination as mode 1)
      const int64_t c2 = i % Cin_pg, t2 = i / Cin_pg;
      const int tap2 = (int)(t2 % khw);
      const int64_t o2 = t2 / khw;
      wp[(c2 * khw + (khw - 1 - tap2)) * Cout + o2] = w[i];
      continue;
    }
    float v = w[i];
    if (mode == 0) wp[(o * khw + tap) * Cin_pg + c] = v;
    else wp[(c * khw + (khw - 1 - tap)) * Cout + o] = v;
  }
}

static bool tc_ok(int64_t M) { return g_gemm_path != 1 && M >= 64; }

void conv_fwd(const ConvShape& s, const float* x, const float* w, const float* bias, float* y) {
  if (conv_fwd_via_nhwc(s, x, w, bias, y)) return;
  if (conv_fwd_s2d(s, x, w, bias, y)) return;
  int groups = (int)(s.Cin / s.icpg);
  int khw = s.KH * s.KW;
  int64_t M = s.N * s.OH * s.OW, K = (int64_t)s.icpg * khw;
  EpNCHW ep{y, bias, s.Cout, s.OH * s.OW, s.ocpg};
  if (tc_ok(M) && s.icpg % 32 == 0) {
    // filter-major K: each 32-wide k-block is one tap x 32 channels
    float* wp = (float*)scratch2((size_t)s.Cout * K * sizeof(float));
    TP_LAUNCH(k_pack_filters, grid_for(s.Cout * K, 256), 256, 0, w, wp, s.Cout, (int64_t)s.icpg, khw, 0);
    LdConvFM la{x, s.Cin, s.icpg, s.H, s.W, s.OH, s.OW, s.KW, s.SH, s.SW, s.PH, s.PW};
    LdRowMajor lb{wp, K, (int64_t)s.ocpg * K};
    gemm_tc(la, lb, ep, M, s.ocpg, K, groups);
    return;
  }
  LdConvIm2col la{x, s};
  LdConvWeight lb{w, K, s.ocpg};
  gemm_auto(la, lb, ep, M, s.ocpg, K, groups);
}

void conv_dgrad(const ConvShape& s, const float* dy, const float* w, float* dx) {
  if (conv_dgrad_via_nhwc(s, dy, w, dx)) return;
  if (conv_dgrad_s2d(s, dy, w, dx)) return;
  if (g_gemm_path == 0 && s.icpg == s.Cin &&
      conv_dgrad_smallc(dy, w, dx, s.N, s.Cin, s.H, s.W, s.Cout, s.OH, s.OW, s.KH, s.KW, s.SH, s.PH, s.PW,
                        s.SH == s.SW))
    return;
  int khw = s.KH * s.KW;
  int64_t M = s.N * s.H * s.W, K = s.Cout * khw;
  EpNCHW ep{dx, nullptr, s.Cin, s.H * s.W, (int)s.Cin};
  if (tc_ok(M) && s.SH == 1 && s.SW == 1 && s.Cout % 32 == 0 && s.PH <= s.KH - 1 && s.PW <= s.KW - 1 &&
      s.OH == s.H + 2 * s.PH - s.KH + 1 && s.OW == s.W + 2 * s.PW - s.KW + 1) {
    // stride 1: dx = forward convolution of dy with the flipped, transposed
    // filters and padding K-1-P
    float* wp = (float*)scratch2((size_t)s.Cin * K * sizeof(float));
    TP_LAUNCH(k_pack_filters, grid_for(s.Cout * s.Cin * khw, 256), 256, 0, w, wp, s.Cout, s.Cin, khw, 1);
    LdConvFM la{dy, s.Cout, (int)s.Cout, s.OH, s.OW, s.H, s.W, s.KW, 1, 1, s.KH - 1 - s.PH, s.KW - 1 - s.PW};
    LdRowMajor lb{wp, K, 0};
    gemm_tc(la, lb, ep, M, s.Cin, K, 1);
    return;
  }
  LdConvDgradA la{dy, s};
  LdConvDgradB lb{w, s};
  gemm_auto(la, lb, ep, M, s.Cin, K, 1);
}

void conv_wgrad(const ConvShape& s, const float* dy, const float* x, float* dw) {
  if (conv_wgrad_via_nhwc(s, dy, x, dw)) return;
  if (conv_wgrad_s2d(s, dy, x, dw)) return;
  int khw = s.KH * s.KW;
  int64_t K = s.N * s.OH * s.OW;
  if (tc_ok(s.Cout) && s.icpg == s.Cin && s.Cin >= 32) {
    // one GEMM per filter tap (batch index): C_tap[oc][ic] = sum_(n,p) dy . x shifted
    LdWgradTapDy la{dy, s.Cout, s.OH * s.OW};
    LdWgradTapX lb{x, s.Cin, s.H, s.W, s.OH, s.OW, s.KW, s.SH, s.SW, s.PH, s.PW};
    EpWgradTap ep{dw, s.Cin, khw};
    gemm_tc(la, lb, ep, s.Cout, s.Cin, K, khw);
    return;
  }
  LdConvWgradA la{dy, s};
  LdConvWgradB lb{x, s};
  int64_t R = s.Cin * khw;
  EpRowMajor ep{dw, R, 0, nullptr, 0};
  gemm_auto(la, lb, ep, s.Cout, R, K, 1);
}

// matmul.wgsl semantics: C[b] = A[b] (M x K) . B[b or shared] (K x N), row-major.
void matmul_launch(const float* A, const float* B, float* C, int64_t batch, int64_t M, int64_t K, int64_t N,
                   bool b_batched) {
  LdRowMajor la{A, K, M * K};
  LdColMajor lb{B, N, b_batched ? K * N : 0};
  EpRowMajor ep{C, N, M * N, nullptr, 0};
  TP_REQUIRE(batch <= 65535, "matmul: batch exceeds the grid limit");
  if (gemm_tma(MatOp{A, false, K, M * K, batch > 1}, MatOp{B, true, N, K * N, b_batched && batch > 1}, ep, M, N, K,
               (int)batch))
    return;
  gemm_auto(la, lb, ep, M, N, K, (int)batch);
}

// y[M, N] = x[M, K] . W[N, K]^T (+ bias[N]) (+ ReLU): nn.Linear without the
// transpose / expand / add dispatches of functional.py:95-101.
void linear_launch(const float* x, const float* w, const float* bias, float* y, int64_t M, int64_t K, int64_t N,
                   bool relu) {
  LdRowMajor la{x, K, 0};
  LdRowMajor lb{w, K, 0};
  EpRowMajor ep{y, N, 0, bias, relu ? 1 : 0};
  if (gemm_tma(MatOp{x, false, K, 0, false}, MatOp{w, false, K, 0, false}, ep, M, N, K, 1)) return;
  gemm_auto(la, lb, ep, M, N, K, 1);
}

void gemm_launch(const float* A, bool a_t, const float* B, bool b_t, float* C, int64_t M, int64_t N, int64_t K,
                 const float* bias) {
  EpRowMajor ep{C, N, 0, bias, 0};
  if (gemm_tma(MatOp{A, a_t, a_t ? M : K, 0, false}, MatOp{B, !b_t, b_t ? K : N, 0, false}, ep, M, N, K, 1)) return;
  if (!a_t && b_t) gemm_auto(LdRowMajor{A, K, 0}, LdRowMajor{B, K, 0}, ep, M, N, K, 1);
  else if (!a_t && !b_t) gemm_auto(LdRowMajor{A, K, 0}, LdColMajor{B, N, 0}, ep, M, N, K, 1);
  else if (a_t && b_t) gemm_auto(LdColMajor{A, M, 0}, LdRowMajor{B, K, 0}, ep, M, N, K, 1);
  else gemm_auto(LdColMajor{A, M, 0}, LdColMajor{B, N, 0}, ep, M, N, K, 1);
}

static int at(const int64_t* v, int n, int i, int dflt) { return n > i ? (int)v[i] : (n > 0 ? (int)v[0] : dflt); }

}  // namespace tp

using namespace tp;

extern "C" {

TP_API int tp_set_gemm_path(int path) {
  return guard([&] {
    TP_REQUIRE(path >= 0 && path <= 4,
               "gemm path must be 0 (tensor cores, TMA-fed where possible, CTA pairs for large N), 1 (CUDA cores), "
               "2 (tensor cores without TMA), 3 (as 0 on single CTAs) or 4 (as 0 with CTA pairs wherever they fit)");
    g_gemm_path = path;
  });
}

TP_API int tp_set_gemm_twocta(int mode) {
  return guard([&] {
    TP_REQUIRE(mode >= 0 && mode <= 2, "tp_set_gemm_twocta: 0 (never), 1 (more CTAs than SMs) or 2 (always)");
    g_gemm_twocta = mode;
  });
}

TP_API int tp_set_gemm_kmax(int kblocks) {
  return guard([&] {
    TP_REQUIRE(kblocks >= 0, "tp_set_gemm_kmax: k-blocks per split must be >= 0 (0: no cap)");
    g_gemm_kmax = kblocks;
  });
}

// One CTA waits, bounded by limit_ns, on an mbarrier that nothing arrives on:
// the wait function of the tensor-core kernels runs out, records `code` in the
// status word and returns.  No copy or tensor memory is involved.
__global__ void k_wait_probe(unsigned long long limit_ns, int code) {
  ::tp::pdl_enter();
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) tc::mbar_init(&bar, 1);
  __syncthreads();
  if (threadIdx.x == 0) tc::mbar_wait_for(&bar, 0, code, limit_ns);
  __syncthreads();
}

TP_API int tp_wait_probe(int64_t limit_ns) {
  return guard([&] {
    TP_REQUIRE(limit_ns >= 1000 && limit_ns <= 2000000000, "tp_wait_probe: limit_ns must be in [1e3, 2e9]");
    TP_LAUNCH(k_wait_probe, 1, 32, 0, (unsigned long long)limit_ns, 99);
  });
}

TP_API int tp_gemm_status(int* out, int reset) {
  return guard([&] {
    TP_CUDA(cudaStreamSynchronize(stream()));
    *out = tc_status(reset != 0);
  });
}

TP_API int tp_matmul(int64_t a, int64_t b, tp_handle* out) {
  return guard([&] {
    Tensor& A = get(a);
    Tensor& B = get(b);
    // arithmeticOps.ts:260-308 shape rules
    if (A.ndim == 2 && B.ndim == 1) {
      int64_t m = A.shape[0], k = A.shape[1];
      TP_REQUIRE(k == B.shape[0], "matmul dimension mismatch: [%lld,%lld] x [%lld].", (long long)m, (long long)k,
                 (long long)B.shape[0]);
      int64_t s[2] = {m, 1};
      Tensor C = make(s, 2, A.dtype);
      matmul_launch(A.f(), B.f(), C.f(), 1, m, k, 1, false);
      emit(C, out);
    } else if (A.ndim == 1 && B.ndim == 2) {
      int64_t k = A.shape[0], n = B.shape[1];
      TP_REQUIRE(k == B.shape[0], "matmul dimension mismatch: [%lld] x [%lld,%lld].", (long long)k,
                 (long long)B.shape[0], (long long)n);
      int64_t s[2] = {1, n};
      Tensor C = make(s, 2, B.dtype);
      matmul_launch(A.f(), B.f(), C.f(), 1, 1, k, n, false);
      emit(C, out);
    } else if (A.ndim == 3 && B.ndim == 3) {
      int64_t bt = A.shape[0], m = A.shape[1], k = A.shape[2], n = B.shape[2];
      TP_REQUIRE(bt == B.shape[0], "matmul batch dim mismatch: %lld vs %lld.", (long long)bt, (long long)B.shape[0]);
      TP_REQUIRE(k == B.shape[1], "matmul dimension mismatch: [%lld,%lld,%lld] x [%lld,%lld,%lld].", (long long)bt,
                 (long long)m, (long long)k, (long long)B.shape[0], (long long)B.shape[1], (long long)n);
      int64_t s[3] = {bt, m, n};
      Tensor C = make(s, 3, A.dtype);
      matmul_launch(A.f(), B.f(), C.f(), bt, m, k, n, true);
      emit(C, out);
    } else if (A.ndim == 2 && B.ndim == 2) {
      int64_t m = A.shape[0], k = A.shape[1], n = B.shape[1];
      TP_REQUIRE(k == B.shape[0], "matmul dimension mismatch: [%lld,%lld] x [%lld,%lld].", (long long)m,
                 (long long)k, (long long)B.shape[0], (long long)n);
      int64_t s[2] = {m, n};
      Tensor C = make(s, 2, A.dtype);
      matmul_launch(A.f(), B.f(), C.f(), 1, m, k, n, false);
      emit(C, out);
    } else if (A.ndim >= 3 && B.ndim == 2) {
      int64_t bt = prod(A.shape, A.ndim - 2), m = A.shape[A.ndim - 2], k = A.shape[A.ndim - 1], n = B.shape[1];
      TP_REQUIRE(k == B.shape[0], "matmul dimension mismatch: [...,%lld,%lld] x [%lld,%lld].", (long long)m,
                 (long long)k, (long long)B.shape[0], (long long)n);
      int64_t s[3] = {bt, m, n};
      Tensor C = make(s, 3, A.dtype);
      // one GEMM over the flattened rows: B is shared by every batch
      matmul_launch(A.f(), B.f(), C.f(), 1, bt * m, k, n, false);
      emit(C, out);
    } else {
      fail(TP_ERR_ARG, "matmul unsupported shapes: rank %d and rank %d.", A.ndim, B.ndim);
    }
  });
}

TP_API int tp_linear(int64_t x, int64_t w, int64_t bias, tp_handle* out) {
  return guard([&] {
    Tensor& X = get(x);
    Tensor& Wt = get(w);
    TP_REQUIRE(Wt.ndim == 2 && X.ndim >= 1, "linear expects weight [out, in]");
    int64_t K = Wt.shape[1], N = Wt.shape[0];
    TP_REQUIRE(X.shape[X.ndim - 1] == K, "linear: input features %lld != weight in_features %lld",
               (long long)X.shape[X.ndim - 1], (long long)K);
    const float* bp = nullptr;
    if (bias) {
      Tensor& B = get(bias);
      TP_REQUIRE(B.numel == N, "linear: bias has %lld values, expected %lld", (long long)B.numel, (long long)N);
      bp = B.f();
    }
    std::vector<int64_t> s(X.shape, X.shape + X.ndim);
    s.back() = N;
    Tensor Y = make_like_shape(s, X.dtype);
    linear_launch(X.f(), Wt.f(), bp, Y.f(), X.numel / K, K, N, false);
    emit(Y, out);
  });
}

// convOps.ts:17-62: bias arrives as a host list (or null), dilation is ignored.
TP_API int tp_conv2d(int64_t input, int64_t weight, const float* bias, int nbias, const int64_t* stride, int ns,
                     const int64_t* padding, int np, const int64_t* dilation, int nd, int groups, tp_handle* out) {
  (void)dilation;
  (void)nd;
  return guard([&] {
    Tensor& X = get(input);
    Tensor& Wt = get(weight);
    TP_REQUIRE(X.ndim == 4 && Wt.ndim == 4, "conv2d expects NCHW input and OIHW weight");
    int g = groups > 0 ? groups : 1;
    TP_REQUIRE(Wt.shape[1] * g == X.shape[1], "conv2d: weight in_channels %lld x groups %d != input channels %lld",
               (long long)Wt.shape[1], g, (long long)X.shape[1]);
    ConvShape s = conv_shape(X.shape[0], X.shape[1], X.shape[2], X.shape[3], Wt.shape[0], (int)Wt.shape[2],
                             (int)Wt.shape[3], at(stride, ns, 0, 1), at(stride, ns, 1, 1), at(padding, np, 0, 0),
                             at(padding, np, 1, 0), g);
    float* db = nullptr;
    if (bias && nbias > 0) {
      TP_REQUIRE(nbias == s.Cout, "conv2d: bias has %d values, expected %lld", nbias, (long long)s.Cout);
      db = (float*)dalloc((size_t)nbias * 4);  // its own block: the GEMM may grow the shared scratch
      TP_CUDA(cudaMemcpyAsync(db, bias, (size_t)nbias * 4, cudaMemcpyHostToDevice, stream()));
    }
    int64_t shp[4] = {s.N, s.Cout, s.OH, s.OW};
    Tensor Y = make(shp, 4, X.dtype);
    conv_fwd(s, X.f(), Wt.f(), db, Y.f());
    if (db) dfree(db);  // stream-ordered: released after the convolution ran
    emit(Y, out);
  });
}

// New: conv2d with the bias as a device tensor (bias_id 0: none).  The
// reference passes the bias as a host list, read back from the device on every
// call (tensor_nn_ops.py:27), which makes each convolution a host sync; this
// entry keeps it on the device and gives the same values.
TP_API int tp_conv2d_dev_bias(int64_t input, int64_t weight, int64_t bias_id, const int64_t* stride, int ns,
                              const int64_t* padding, int np, const int64_t* dilation, int nd, int groups,
                              tp_handle* out) {
  (void)dilation;
  (void)nd;
  return guard([&] {
    Tensor& X = get(input);
    Tensor& Wt = get(weight);
    TP_REQUIRE(X.ndim == 4 && Wt.ndim == 4, "conv2d expects NCHW input and OIHW weight");
    int g = groups > 0 ? groups : 1;
    TP_REQUIRE(Wt.shape[1] * g == X.shape[1], "conv2d: weight in_channels %lld x groups %d != input channels %lld",
               (long long)Wt.shape[1], g, (long long)X.shape[1]);
    ConvShape s = conv_shape(X.shape[0], X.shape[1], X.shape[2], X.shape[3], Wt.shape[0], (int)Wt.shape[2],
                             (int)Wt.shape[3], at(stride, ns, 0, 1), at(stride, ns, 1, 1), at(padding, np, 0, 0),
                             at(padding, np, 1, 0), g);
    const float* db = nullptr;
    if (bias_id) {
      Tensor& Bt = get(bias_id);
      TP_REQUIRE(Bt.numel == s.Cout, "conv2d: bias has %lld values, expected %lld", (long long)Bt.numel,
                 (long long)s.Cout);
      db = Bt.f();
    }
    int64_t shp[4] = {s.N, s.Cout, s.OH, s.OW};
    Tensor Y = make(shp, 4, X.dtype);
    conv_fwd(s, X.f(), Wt.f(), db, Y.f());
    emit(Y, out);
  });
}

// convOps.ts:64-108 (groups forced to 1 by the reference).
TP_API int tp_conv2d_input_backward(int64_t grad_out, int64_t weight, const int64_t* input_shape,
                                    const int64_t* grad_out_shape, const int64_t* stride, int ns,
                                    const int64_t* padding, int np, tp_handle* out) {
  return guard([&] {
    Tensor& G = get(grad_out);
    Tensor& Wt = get(weight);
    TP_REQUIRE(Wt.ndim == 4, "conv2dInputBackward expects an OIHW weight");
    ConvShape s = conv_shape(input_shape[0], input_shape[1], input_shape[2], input_shape[3], grad_out_shape[1],
                             (int)Wt.shape[2], (int)Wt.shape[3], at(stride, ns, 0, 1), at(stride, ns, 1, 1),
                             at(padding, np, 0, 0), at(padding, np, 1, 0), 1);
    s.OH = grad_out_shape[2];
    s.OW = grad_out_shape[3];
    TP_REQUIRE(G.numel == s.N * s.Cout * s.OH * s.OW, "conv2dInputBackward: grad_output size mismatch");
    TP_REQUIRE(Wt.numel == s.Cout * s.Cin * s.KH * s.KW, "conv2dInputBackward: weight size mismatch");
    Tensor X = make(input_shape, 4, G.dtype);
    conv_dgrad(s, G.f(), Wt.f(), X.f());
    emit(X, out);
  });
}

// convOps.ts:110-155.
TP_API int tp_conv2d_weight_backward(int64_t grad_out, int64_t input, const int64_t* weight_shape,
                                     const int64_t* grad_out_shape, const int64_t* input_shape, const int64_t* stride,
                                     int ns, const int64_t* padding, int np, tp_handle* out) {
  return guard([&] {
    Tensor& G = get(grad_out);
    Tensor& X = get(input);
    ConvShape s = conv_shape(input_shape[0], input_shape[1], input_shape[2], input_shape[3], weight_shape[0],
                             (int)weight_shape[2], (int)weight_shape[3], at(stride, ns, 0, 1), at(stride, ns, 1, 1),
                             at(padding, np, 0, 0), at(padding, np, 1, 0), 1);
    s.OH = grad_out_shape[2];
    s.OW = grad_out_shape[3];
    TP_REQUIRE(G.numel == s.N * s.Cout * s.OH * s.OW, "conv2dWeightBackward: grad_output size mismatch");
    TP_REQUIRE(X.numel == s.N * s.Cin * s.H * s.W, "conv2dWeightBackward: input size mismatch");
    TP_REQUIRE(weight_shape[1] == s.Cin, "conv2dWeightBackward: groups are not supported (as in the reference)");
    Tensor Wg = make(weight_shape, 4, G.dtype);
    conv_wgrad(s, G.f(), X.f(), Wg.f());
    emit(Wg, out);
  });
}

// convOps.ts:157-198.
TP_API int tp_conv2d_bias_backward(int64_t grad_out, int64_t out_ch, const int64_t* grad_out_shape, tp_handle* out) {
  return guard([&] {
    Tensor& G = get(grad_out);
    int64_t N = grad_out_shape[0], P = grad_out_shape[2] * grad_out_shape[3];
    TP_REQUIRE(G.numel == N * out_ch * P, "conv2dBiasBackward: grad_output size mismatch");
    int64_t s[1] = {out_ch};
    Tensor B = make(s, 1, G.dtype);
    launch_channel_sum(G.f(), N, out_ch, P, B.f());
    emit(B, out);
  });
}

}  // extern "C"
