// Pointer-level C ABI (tpk_*) and CUDA-graph capture.
//
// The handle-level tp_* entries allocate every output, as the reference
// runtime does (one fresh GPUBuffer per op).  A training step driver instead
// owns its buffers and calls these entries on raw device pointers with plain
// sizes; nothing here allocates once the shared scratch has reached its size,
// so a whole step can be captured into one CUDA graph and replayed
// (tp_graph_*).  That replaces the reference's per-op queue.submit
// (dispatch.ts:104-133) and Python loop overhead with one graph launch.
#include <cuda_runtime.h>

#include <unordered_map>

#include "tp_core.h"
#include "tp_launch.h"

namespace tp {

struct GraphRec {
  cudaGraphExec_t exec;
  int64_t kernels;  // kernel launches recorded while capturing
};
static std::unordered_map<int64_t, GraphRec> g_graphs;
static int64_t g_next_graph = 1;
static cudaGraph_t g_capturing = nullptr;
static int64_t g_capture_launches0 = 0;

static PoolGeom square_pool(int64_t N, int64_t C, int64_t H, int64_t W, int k, int s, int p) {
  TP_REQUIRE(k > 0 && s > 0 && p >= 0, "max_pool2d: invalid window");
  PoolGeom g;
  g.N = N;
  g.C = C;
  g.H = H;
  g.W = W;
  g.KH = g.KW = k;
  g.SH = g.SW = s;
  g.PH = g.PW = p;
  g.DH = g.DW = 1;
  g.OH = (H + 2 * p - k) / s + 1;
  g.OW = (W + 2 * p - k) / s + 1;
  TP_REQUIRE(g.OH > 0 && g.OW > 0, "max_pool2d: output would be empty");
  return g;
}

}  // namespace tp

using namespace tp;

extern "C" {

TP_API int tpk_conv2d_fwd(const float* x, const float* w, const float* bias, float* y, int64_t N, int64_t Cin,
                          int64_t H, int64_t W, int64_t Cout, int KH, int KW, int SH, int SW, int PH, int PW) {
  return guard([&] { conv_fwd(conv_shape(N, Cin, H, W, Cout, KH, KW, SH, SW, PH, PW, 1), x, w, bias, y); });
}

TP_API int tpk_conv2d_dgrad(const float* dy, const float* w, float* dx, int64_t N, int64_t Cin, int64_t H, int64_t W,
                            int64_t Cout, int KH, int KW, int SH, int SW, int PH, int PW) {
  return guard([&] { conv_dgrad(conv_shape(N, Cin, H, W, Cout, KH, KW, SH, SW, PH, PW, 1), dy, w, dx); });
}

TP_API int tpk_conv2d_wgrad(const float* dy, const float* x, float* dw, int64_t N, int64_t Cin, int64_t H, int64_t W,
                            int64_t Cout, int KH, int KW, int SH, int SW, int PH, int PW) {
  return guard([&] { conv_wgrad(conv_shape(N, Cin, H, W, Cout, KH, KW, SH, SW, PH, PW, 1), dy, x, dw); });
}

TP_API int tpk_channel_sum(const float* x, int64_t N, int64_t C, int64_t P, float* out) {
  return guard([&] { launch_channel_sum(x, N, C, P, out); });
}

TP_API int tpk_bn_train(const float* x, const float* w, const float* b, float* running_mean, float* running_var,
                        float* y, float* save_mean, float* save_invstd, int64_t N, int64_t C, int64_t S, float eps,
                        float momentum, int relu) {
  return guard([&] {
    TP_REQUIRE(N * S > 1, "batch_norm training needs more than one value per channel");
    launch_bn_train(x, w, b, running_mean, running_var, y, save_mean, save_invstd, N, C, S, eps, momentum, relu != 0);
  });
}

TP_API int tpk_bn_backward(const float* dy, const float* x, const float* relu_src, const float* w, const float* mean,
                           const float* invstd, float* dx, float* dw, float* db, int64_t N, int64_t C, int64_t S) {
  return guard([&] { launch_bn_backward(dy, x, relu_src, w, mean, invstd, dx, dw, db, N, C, S); });
}

TP_API int tpk_maxpool_fwd(const float* x, float* y, int32_t* idx, int64_t N, int64_t C, int64_t H, int64_t W, int k,
                           int s, int p) {
  return guard([&] { launch_maxpool_fwd(x, y, idx, square_pool(N, C, H, W, k, s, p)); });
}

TP_API int tpk_maxpool_bwd(const float* dy, const int32_t* idx, float* dx, int64_t N, int64_t C, int64_t H, int64_t W,
                           int k, int s, int p) {
  return guard([&] { launch_maxpool_bwd(dy, idx, dx, square_pool(N, C, H, W, k, s, p)); });
}

TP_API int tpk_gemm(const float* A, int a_t, const float* B, int b_t, float* C, int64_t M, int64_t N, int64_t K,
                    const float* bias) {
  return guard([&] { gemm_launch(A, a_t != 0, B, b_t != 0, C, M, N, K, bias); });
}

TP_API int tpk_cross_entropy_mean(const float* logits, const float* targets, float* loss_rows, float* loss_mean,
                                  int64_t B, int64_t C) {
  return guard([&] {
    launch_cross_entropy(logits, targets, loss_rows, B, C);
    launch_reduce_all(loss_rows, B, 1, loss_mean);
  });
}

TP_API int tpk_cross_entropy_backward(const float* logits, const float* targets, float* grad, int64_t B, int64_t C,
                                      float scale) {
  return guard([&] {
    // upstream gradient 1 for a mean loss: grad = (softmax - onehot) * scale
    static float* one = nullptr;
    if (!one) {
      one = (float*)dalloc(4);
      launch_fill(one, 1, 1.0f);
    }
    launch_cross_entropy_bwd(one, 1, logits, targets, grad, B, C, scale);
  });
}

TP_API int tpk_fill(float* x, int64_t n, float value) { return guard([&] { launch_fill(x, n, value); }); }

TP_API int tp_graph_begin(void) {
  return guard([&] {
    TP_REQUIRE(g_capturing == nullptr, "a graph capture is already open");
    TP_CUDA(cudaStreamBeginCapture(stream(), cudaStreamCaptureModeThreadLocal));
    g_capturing = (cudaGraph_t)1;
    g_capture_launches0 = g_launches.load();
  });
}

TP_API int tp_graph_end(int64_t* out_graph) {
  return guard([&] {
    TP_REQUIRE(g_capturing != nullptr, "no graph capture is open");
    g_capturing = nullptr;
    cudaGraph_t graph = nullptr;
    TP_CUDA(cudaStreamEndCapture(stream(), &graph));
    cudaGraphExec_t exec = nullptr;
    // kernels keep the priority of the stream they were captured on (the
    // communicator's stream may run at a higher one)
    cudaError_t e = cudaGraphInstantiate(&exec, graph, cudaGraphInstantiateFlagUseNodePriority);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) fail(TP_ERR_CUDA, "cudaGraphInstantiate failed: %s", cudaGetErrorString(e));
    int64_t id = g_next_graph++;
    g_graphs[id] = GraphRec{exec, g_launches.load() - g_capture_launches0};
    *out_graph = id;
  });
}

TP_API int tp_graph_launch(int64_t graph) {
  return guard([&] {
    auto it = g_graphs.find(graph);
    TP_REQUIRE(it != g_graphs.end(), "unknown graph %lld", (long long)graph);
    TP_CUDA(cudaGraphLaunch(it->second.exec, stream()));
    g_launches += it->second.kernels;
  });
}

TP_API int tp_graph_destroy(int64_t graph) {
  return guard([&] {
    auto it = g_graphs.find(graph);
    if (it == g_graphs.end()) return;
    TP_CUDA(cudaGraphExecDestroy(it->second.exec));
    g_graphs.erase(it);
  });
}

}  // extern "C"
