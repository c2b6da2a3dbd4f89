// Data-parallel gradient all-reduce over NCCL on a dedicated communication
// stream.
//
// The reference has no parallelism of any kind (one WebGPU device, one queue).
// The data-parallel VGG-11-BN step needs exactly one exchange: the sum of the
// gradients over ranks.  Buckets of the flat gradient buffer are reduced in
// place as soon as backward has finished them: the main stream records an
// event, the comm stream waits on it and runs ncclAllReduce, and the optimizer
// launch waits for the comm stream's last event.  All of this is captured by a
// CUDA graph together with the compute kernels.
//
// NCCL is opened with dlopen at tp_comm_init, so the library loads (and the
// single-GPU paths run) without it; nccl.h supplies only the types.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "tp_core.h"

namespace tp {

struct NcclApi {
  void* h = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

static NcclApi g_nccl;
static ncclComm_t g_comm = nullptr;
static cudaStream_t g_comm_stream = nullptr;

cudaStream_t comm_stream() {
  TP_REQUIRE(g_comm_stream != nullptr, "no communicator: its stream does not exist");
  return g_comm_stream;
}
bool comm_active() { return g_comm_stream != nullptr; }
static std::vector<cudaEvent_t> g_events;
static size_t g_next_event = 0;
static bool g_pending = false;
static int g_rank = 0, g_world = 1;
// 1 (default): the comm stream at the device's highest stream priority, so each
// all-reduce's CTAs start ahead of the backward's pending ones (VGG-11-BN on 8
// GPUs, 128 images per rank: 1.23 -> 1.14 ms per step); 0: normal priority
static int g_comm_prio = 1;

static void load_nccl() {
  if (g_nccl.h) return;
  // NVLink SHARP (NVLS) off unless the caller chose: its all-reduce keeps 24 CTAs per
  // GPU busy beside the backward kernels, and the VGG-11-BN step on 8 GPUs (9.4 MB
  // buckets, 128 images per rank) ran 1.145 -> 1.116 ms per step on the ring / tree
  // algorithms.  Set before NCCL reads its environment (the first NCCL call).
  setenv("NCCL_NVLS_ENABLE", "0", 0);
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) fail(TP_ERR_NCCL, "cannot load libnccl.so.2: %s", dlerror());
#define TP_SYM(name)                                                                        \
  g_nccl.name = reinterpret_cast<decltype(g_nccl.name)>(dlsym(h, "nccl" #name));            \
  if (!g_nccl.name) fail(TP_ERR_NCCL, "libnccl.so.2 lacks nccl%s", #name);
  TP_SYM(GetUniqueId)
  TP_SYM(CommInitRank)
  TP_SYM(AllReduce)
  TP_SYM(CommDestroy)
  TP_SYM(CommAbort)
  TP_SYM(CommGetAsyncError)
  TP_SYM(GetErrorString)
#undef TP_SYM
  g_nccl.h = h;
}

#define TP_NCCL(call)                                                                      \
  do {                                                                                     \
    ncclResult_t r_ = (call);                                                              \
    if (r_ != ncclSuccess) fail(TP_ERR_NCCL, "%s failed: %s", #call, g_nccl.GetErrorString(r_)); \
  } while (0)

static cudaEvent_t next_event() {
  if (g_next_event == g_events.size()) {
    cudaEvent_t e;
    TP_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    g_events.push_back(e);
  }
  return g_events[g_next_event++];
}

}  // namespace tp

using namespace tp;

extern "C" {

TP_API int tp_comm_unique_id(char* out, int len) {
  return guard([&] {
    TP_REQUIRE(len >= (int)sizeof(ncclUniqueId), "unique id buffer needs %d bytes", (int)sizeof(ncclUniqueId));
    load_nccl();
    ncclUniqueId id;
    TP_NCCL(g_nccl.GetUniqueId(&id));
    memcpy(out, &id, sizeof(id));
  });
}

TP_API int tp_set_comm_priority(int high) {
  return guard([&] {
    TP_REQUIRE(g_comm == nullptr, "tp_set_comm_priority: call it before tp_comm_init");
    g_comm_prio = high ? 1 : 0;
  });
}

TP_API int tp_comm_init(int rank, int world, const char* unique_id, int len) {
  return guard([&] {
    TP_REQUIRE(len >= (int)sizeof(ncclUniqueId), "unique id holds %d bytes", (int)sizeof(ncclUniqueId));
    TP_REQUIRE(world >= 1 && rank >= 0 && rank < world, "bad rank %d of %d", rank, world);
    TP_REQUIRE(g_comm == nullptr, "communicator already initialised");
    load_nccl();
    ensure_init();
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof(id));
    TP_NCCL(g_nccl.CommInitRank(&g_comm, world, id, rank));
    if (g_comm_prio) {
      int lo = 0, hi = 0;
      TP_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
      TP_CUDA(cudaStreamCreateWithPriority(&g_comm_stream, cudaStreamNonBlocking, hi));
    } else {
      TP_CUDA(cudaStreamCreateWithFlags(&g_comm_stream, cudaStreamNonBlocking));
    }
    g_rank = rank;
    g_world = world;
  });
}

// Sum `count` floats at `ptr` over all ranks, in place, on the comm stream,
// after everything already queued on the library stream.
TP_API int tp_comm_allreduce_async(float* ptr, int64_t count) {
  return guard([&] {
    TP_REQUIRE(g_comm != nullptr, "communicator not initialised");
    if (g_next_event >= 4096) g_next_event = 0;
    cudaEvent_t ready = next_event();
    TP_CUDA(cudaEventRecord(ready, stream()));
    TP_CUDA(cudaStreamWaitEvent(g_comm_stream, ready, 0));
    TP_NCCL(g_nccl.AllReduce(ptr, ptr, (size_t)count, ncclFloat32, ncclSum, g_comm, g_comm_stream));
    g_pending = true;
  });
}

// Make the library stream wait for every all-reduce issued so far.
TP_API int tp_comm_wait(void) {
  return guard([&] {
    if (!g_pending) return;
    cudaEvent_t done = next_event();
    TP_CUDA(cudaEventRecord(done, g_comm_stream));
    TP_CUDA(cudaStreamWaitEvent(stream(), done, 0));
    g_pending = false;
    g_next_event = 0;  // events may be reused once joined
  });
}

// Host-side watchdog: wait up to timeout_ms for the library stream; on a
// communicator error or a timeout, abort the communicator and return an error
// (the other ranks then fail their own next collective instead of hanging).
TP_API int tp_comm_sync(int timeout_ms) {
  return guard([&] {
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
      cudaError_t q = cudaStreamQuery(stream());
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) fail(TP_ERR_CUDA, "stream error: %s", cudaGetErrorString(q));
      if (g_comm) {
        ncclResult_t ar = ncclSuccess;
        g_nccl.CommGetAsyncError(g_comm, &ar);
        if (ar != ncclSuccess && ar != ncclInProgress) {
          g_nccl.CommAbort(g_comm);
          g_comm = nullptr;
          fail(TP_ERR_NCCL, "communicator error: %s", g_nccl.GetErrorString(ar));
        }
      }
      auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
      if (timeout_ms >= 0 && ms > timeout_ms) {
        if (g_comm) {
          g_nccl.CommAbort(g_comm);
          g_comm = nullptr;
        }
        fail(TP_ERR_TIMEOUT, "step did not finish within %d ms; communicator aborted", timeout_ms);
      }
      std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
    const int st = tc_status(true);
    if (st) fail(TP_ERR_TIMEOUT, "a device-side wait gave up (code %d): this step's results are incomplete", st);
  });
}

TP_API int tp_comm_destroy(void) {
  return guard([&] {
    if (g_comm) {
      TP_CUDA(cudaStreamSynchronize(g_comm_stream));
      TP_NCCL(g_nccl.CommDestroy(g_comm));
      g_comm = nullptr;
    }
    if (g_comm_stream) {
      cudaStreamDestroy(g_comm_stream);
      g_comm_stream = nullptr;
    }
  });
}

TP_API int tp_comm_info(int* rank, int* world) {
  return guard([&] {
    *rank = g_rank;
    *world = g_comm ? g_world : 1;
  });
}

}  // extern "C"
