// Internal header of libtpcuda: handle table, HBM allocator, stream, errors.
//
// The reference runtime keeps an id -> GPUBuffer registry with a host shadow of
// every buffer (runtime/src/ops/tensorRegistry.ts:3-59, device.ts:272-288).
// Here the registry maps an int64 id to an HBM allocation from a stream-ordered
// caching pool (cudaMallocAsync on the device's default pool, release threshold
// raised so freed blocks are reused instead of returned to the driver).  There
// is no host shadow: tensors live only in HBM.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "../../include/tpcuda.h"

namespace tp {

// Storage of every logical dtype is f32 (runtime/src/ops/device.ts:362-364),
// except index tensors created by the new pooling/max entry points, which are
// physically int32.
enum Phys : int32_t { PHYS_F32 = 0, PHYS_I32 = 1 };

struct Tensor {
  void* ptr = nullptr;
  int64_t numel = 0;
  int32_t ndim = 0;
  int32_t dtype = TP_FLOAT32;
  int32_t phys = PHYS_F32;
  int64_t shape[TP_MAX_DIMS] = {0};
  size_t bytes = 0;
  float* f() const { return static_cast<float*>(ptr); }
  int32_t* i() const { return static_cast<int32_t*>(ptr); }
};

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int code, const char* fmt, ...);
void set_error(const char* msg);

#define TP_REQUIRE(cond, ...)                        \
  do {                                               \
    if (!(cond)) ::tp::fail(TP_ERR_ARG, __VA_ARGS__); \
  } while (0)

#define TP_CUDA(call)                                                                          \
  do {                                                                                         \
    cudaError_t e_ = (call);                                                                   \
    if (e_ != cudaSuccess) ::tp::fail(TP_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// Kernel-launch check: catches configuration errors immediately; execution
// errors surface at the next synchronising call.
#define TP_LAUNCH_CHECK() TP_CUDA(cudaGetLastError())

// Run a C-ABI body, translating exceptions into status codes.
template <class F>
int guard(F&& f) {
  try {
    f();
    return TP_OK;
  } catch (const Error& e) {
    set_error(e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    set_error("host allocation failed");
    return TP_ERR_OOM;
  } catch (const std::exception& e) {
    set_error(e.what());
    return TP_ERR_INTERNAL;
  }
}

// ---- device state --------------------------------------------------------
void ensure_init();
cudaStream_t stream();
int device();
int sm_count();

// First nonzero code a bounded device-side wait of a tensor-core kernel
// recorded since the last reset (0: none); reset clears it.  Reading it copies
// from device memory, so call it only once the library streams are idle.
int tc_status(bool reset);

// ---- allocator -----------------------------------------------------------
void* dalloc(size_t bytes);
void dfree(void* p);

// ---- registry ------------------------------------------------------------
Tensor& get(int64_t id);
int64_t put(const Tensor& t);
Tensor make(const int64_t* shape, int ndim, int dtype, int phys = PHYS_F32);
Tensor make_like_shape(const std::vector<int64_t>& shape, int dtype, int phys = PHYS_F32);
void fill_handle(const Tensor& t, int64_t id, tp_handle* out);
int64_t emit(const Tensor& t, tp_handle* out);  // register + fill handle
std::vector<int64_t> shape_of(const Tensor& t);
int64_t prod(const int64_t* s, int n);

inline unsigned grid_for(int64_t n, int threads, int per_thread = 1) {
  int64_t blocks = (n + (int64_t)threads * per_thread - 1) / ((int64_t)threads * per_thread);
  int64_t cap = (int64_t)sm_count() * 32;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (unsigned)blocks;
}

// Scratch space reused across launches on the library stream (stream order
// makes reuse safe).  Grows on demand; never shrinks.
void* scratch(size_t bytes);
// The communicator's stream (tp_comm.cu); fails when no communicator exists.
cudaStream_t comm_stream();
bool comm_active();
// A second, independent scratch area (repacked filters), same rules.
void* scratch2(size_t bytes);
// A third one (the tf32 low parts of a GEMM operand), same rules.
void* scratch3(size_t bytes);

}  // namespace tp

namespace tp {
extern std::atomic<int64_t> g_launches;
// 1: kernels are launched as programmatic dependents of their stream
// predecessor (set by tp_set_pdl, default from TP_PDL, on unless "0").
extern int g_pdl;

// Programmatic dependent launch.  A kernel launched with
// programmaticStreamSerializationAllowed may be scheduled once every CTA of the
// kernel before it in the stream has executed pdl_trigger() (or exited), so its
// launch and prologue overlap that kernel's last CTAs.  Every kernel of this
// library therefore starts with pdl_wait(), which returns once the predecessor
// grid has completed and its memory is visible: no global access precedes it.
// Kernels that allocate tensor memory trigger only after the allocation, so a
// CTA that waits never holds TMEM a running CTA might need, and a dependent grid
// only starts when all CTAs of its predecessor are resident: neither can block
// the kernel it waits for.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
  pdl_wait();
  pdl_trigger();
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_on(cudaStream_t st, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
}  // namespace tp

// Launch a kernel on the library stream, count it and check the launch.
#define TP_LAUNCH(kernel, grid, block, smem, ...)                                              \
  do {                                                                                         \
    TP_CUDA(::tp::launch_on(::tp::stream(), kernel, dim3(grid), dim3(block), (smem), __VA_ARGS__)); \
    ::tp::g_launches++;                                                                        \
  } while (0)
