// Internal launchers shared between the C-ABI translation units.  All run on
// the library stream; none allocates except where noted (scratch()).
#pragma once

#include <stdint.h>

#include "tp_core.h"
#include "tp_gemm.cuh"

namespace tp {

struct PoolGeom {
  int64_t N, C, H, W, OH, OW;
  int KH, KW, SH, SW, PH, PW, DH, DW;
};

// tp_elementwise.cu
void launch_binary(int op, const float* a, const float* b, float* out, int64_t n);
void launch_unary(int op, const float* in, float* out, int64_t n);
void launch_fill(float* out, int64_t n, float v);

// tp_reduce.cu
void launch_reduce_all(const float* x, int64_t n, int mode, float* out);
void launch_reduce_dim(const float* x, int64_t outer, int64_t red, int64_t inner, int mode, float* out,
                       int32_t* idx);
void launch_softmax(const float* x, float* y, int64_t outer, int64_t axis, int64_t inner, bool log_mode);
void launch_cross_entropy(const float* x, const float* tgt, float* loss, int64_t B, int64_t C);
void launch_cross_entropy_bwd(const float* go, int go_scalar, const float* x, const float* tgt, float* gi, int64_t B,
                              int64_t C, float scale);

// tp_pool.cu
void launch_maxpool_fwd(const float* x, float* y, int32_t* idx, const PoolGeom& g);
void launch_maxpool_bwd(const float* gy, const int32_t* idx, float* gx, const PoolGeom& g);

// tp_norm.cu
void launch_bn_train(const float* x, const float* w, const float* b, float* rm, float* rv, float* y,
                     float* save_mean, float* save_invstd, int64_t N, int64_t C, int64_t S, float eps,
                     float momentum, bool relu);
void launch_bn_backward(const float* dy, const float* x, const float* relu_src, const float* w, const float* mean,
                        const float* invstd, float* dx, float* dw, float* db, int64_t N, int64_t C, int64_t S);
// status word of the one-launch BatchNorm's bounded waits (0: none expired)
int norm_status(bool reset);
void launch_ln_fwd(const float* x, const float* g, const float* b, float* y, float* sm, float* sr, int64_t rows,
                   int64_t D, float eps);
void launch_ln_bwd(const float* dy, const float* x, const float* g, const float* sm, const float* sr, float* dx,
                   float* dg, float* db, int64_t rows, int64_t D);

// tp_conv.cu
ConvShape conv_shape(int64_t N, int64_t Cin, int64_t H, int64_t W, int64_t Cout, int KH, int KW, int SH, int SW,
                     int PH, int PW, int groups);
void conv_fwd(const ConvShape& s, const float* x, const float* w, const float* bias, float* y);
void conv_dgrad(const ConvShape& s, const float* dy, const float* w, float* dx);
void conv_wgrad(const ConvShape& s, const float* dy, const float* x, float* dw);
void launch_channel_sum(const float* x, int64_t N, int64_t C, int64_t P, float* out);

// tp_nhwc.cu: [N][C][HW] <-> [N][HW][C]
void transpose_nchw_nhwc(const float* in, float* out, int64_t N, int64_t C, int64_t HW, bool to_nhwc);

// tp_conv_nhwc.cu: NCHW convolutions run through channels-last copies on the
// TMA-fed kernel when the shape allows it (stride 1, groups 1, channel counts
// multiples of 32); false (nothing launched) otherwise
bool conv_fwd_via_nhwc(const ConvShape& s, const float* x, const float* w, const float* bias, float* y);
bool conv_dgrad_via_nhwc(const ConvShape& s, const float* dy, const float* w, float* dx);
bool conv_wgrad_via_nhwc(const ConvShape& s, const float* dy, const float* x, float* dw);
// stride-2 convolutions of <= 8 channels through space-to-depth (tp_conv_nhwc.cu)
bool conv_fwd_s2d(const ConvShape& s, const float* x, const float* w, const float* bias, float* y);
bool conv_dgrad_s2d(const ConvShape& s, const float* dy, const float* w, float* dx);
bool conv_wgrad_s2d(const ConvShape& s, const float* dy, const float* x, float* dw);

// tp_conv_small.cu: NCHW data gradient for Cin <= 4 (any stride) on CUDA cores
bool conv_dgrad_smallc(const float* dy, const float* w, float* dx, int64_t N, int64_t Cin, int64_t H, int64_t W,
                       int64_t Cout, int64_t OH, int64_t OW, int KH, int KW, int S, int PH, int PW, bool same_stride);
void matmul_launch(const float* A, const float* B, float* C, int64_t batch, int64_t M, int64_t K, int64_t N,
                   bool b_batched);
void linear_launch(const float* x, const float* w, const float* bias, float* y, int64_t M, int64_t K, int64_t N,
                   bool relu);
// C[M,N] = op(A) op(B): a_t: A stored [K,M] (else [M,K]); b_t: B stored [N,K] (else [K,N]).
void gemm_launch(const float* A, bool a_t, const float* B, bool b_t, float* C, int64_t M, int64_t N, int64_t K,
                 const float* bias);

}  // namespace tp
