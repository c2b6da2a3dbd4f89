// libtpcuda core: device init, stream, HBM pool, handle table, errors and the
// registry / copy entry points of the C ABI.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include <cstdlib>

#include "tp_core.h"

namespace tp {

static thread_local std::string g_err;
static int g_device = -1;
static cudaStream_t g_stream = nullptr;
// A second stream for work that may overlap the main one (a convolution's
// weight gradient beside its data gradient); launches go to g_aux between
// tp_aux_fork and tp_aux_return on the calling thread.
static cudaStream_t g_aux = nullptr;
// 0: library stream, 1: auxiliary stream, 2: the side stream (between
// tp_side_fork and tp_side_return): the communicator's stream when one exists
// (work that must follow a gradient all-reduce), else a library stream of its own
static thread_local int g_cur = 0;
static cudaStream_t g_side = nullptr;
static int g_sms = 148;
static std::unordered_map<int64_t, Tensor> g_tensors;
static int64_t g_next_id = 1;
static int64_t g_allocated = 0;
// scratch areas per stream (index g_cur), so overlapping work never shares one
static void* g_scratch[3] = {nullptr, nullptr, nullptr};
static size_t g_scratch_bytes[3] = {0, 0, 0};
std::atomic<int64_t> g_launches{0};
static int pdl_default() {
  const char* e = getenv("TP_PDL");
  return e && e[0] == '0' ? 0 : 1;
}
int g_pdl = pdl_default();

void set_error(const char* msg) { g_err = msg ? msg : ""; }

void fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  throw Error(code, buf);
}

void ensure_init() {
  if (g_device >= 0) return;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) fail(TP_ERR_CUDA, "no CUDA device available (%s)", cudaGetErrorString(e));
  int dev = 0;
  TP_CUDA(cudaGetDevice(&dev));
  TP_CUDA(cudaSetDevice(dev));
  TP_CUDA(cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking));
  cudaDeviceProp prop;
  TP_CUDA(cudaGetDeviceProperties(&prop, dev));
  g_sms = prop.multiProcessorCount;
  // Keep freed blocks cached in the pool (a caching allocator on top of the
  // driver's stream-ordered pool).
  cudaMemPool_t pool;
  TP_CUDA(cudaDeviceGetDefaultMemPool(&pool, dev));
  uint64_t thr = UINT64_MAX;
  TP_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr));
  g_device = dev;
}

static cudaStream_t aux_stream() {
  ensure_init();
  if (!g_aux) TP_CUDA(cudaStreamCreateWithFlags(&g_aux, cudaStreamNonBlocking));
  return g_aux;
}

static cudaStream_t side_stream() {
  ensure_init();
  if (comm_active()) return comm_stream();
  if (!g_side) TP_CUDA(cudaStreamCreateWithFlags(&g_side, cudaStreamNonBlocking));
  return g_side;
}

cudaStream_t stream() {
  ensure_init();
  return g_cur == 0 ? g_stream : (g_cur == 1 ? aux_stream() : side_stream());
}
int device() {
  ensure_init();
  return g_device;
}
int sm_count() {
  ensure_init();
  return g_sms;
}

void* dalloc(size_t bytes) {
  ensure_init();
  if (bytes == 0) bytes = 4;
  void* p = nullptr;
  cudaError_t e = cudaMallocAsync(&p, bytes, stream());
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(TP_ERR_OOM, "device allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
  }
  return p;
}

void dfree(void* p) {
  if (p) TP_CUDA(cudaFreeAsync(p, stream()));
}

static void* grow(void** slot, size_t* have, size_t bytes) {
  if (bytes > *have) {
    if (*slot) dfree(*slot);
    size_t nb = bytes < (1u << 20) ? (1u << 20) : bytes;
    *slot = dalloc(nb);
    *have = nb;
  }
  return *slot;
}

void* scratch(size_t bytes) { return grow(&g_scratch[g_cur], &g_scratch_bytes[g_cur], bytes); }

static void* g_scratch2[3] = {nullptr, nullptr, nullptr};
static size_t g_scratch2_bytes[3] = {0, 0, 0};

void* scratch2(size_t bytes) { return grow(&g_scratch2[g_cur], &g_scratch2_bytes[g_cur], bytes); }

static void* g_scratch3[3] = {nullptr, nullptr, nullptr};
static size_t g_scratch3_bytes[3] = {0, 0, 0};

void* scratch3(size_t bytes) { return grow(&g_scratch3[g_cur], &g_scratch3_bytes[g_cur], bytes); }

// ---- the auxiliary stream ----------------------------------------------------------------
static cudaEvent_t g_fork_ev = nullptr, g_join_ev = nullptr, g_sfork_ev = nullptr, g_sfork_aux_ev = nullptr,
                   g_sjoin_ev = nullptr;
static bool g_aux_live = false;
static cudaEvent_t g_slot_ev[64];
static bool g_slot_made[64];

static cudaEvent_t make_event(cudaEvent_t* e) {
  if (!*e) TP_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  return *e;
}

// The side stream waits for everything queued so far on the library and
// auxiliary streams, then takes the calling thread's launches.
void side_fork() {
  TP_REQUIRE(g_cur == 0, "tp_side_fork: not on the library stream");
  cudaStream_t c = side_stream();
  TP_CUDA(cudaEventRecord(make_event(&g_sfork_ev), g_stream));
  TP_CUDA(cudaStreamWaitEvent(c, g_sfork_ev, 0));
  if (g_aux_live) {  // the auxiliary stream was forked and not yet joined
    TP_CUDA(cudaEventRecord(make_event(&g_sfork_aux_ev), g_aux));
    TP_CUDA(cudaStreamWaitEvent(c, g_sfork_aux_ev, 0));
  }
  g_cur = 2;
}

void side_return() { g_cur = 0; }

void side_join() {
  ensure_init();
  if (!comm_active() && !g_side) return;
  TP_CUDA(cudaEventRecord(make_event(&g_sjoin_ev), side_stream()));
  TP_CUDA(cudaStreamWaitEvent(g_stream, g_sjoin_ev, 0));
}

void aux_fork() {
  TP_REQUIRE(g_cur == 0, "tp_aux_fork: already on the auxiliary stream");
  cudaStream_t a = aux_stream();
  TP_CUDA(cudaEventRecord(make_event(&g_fork_ev), g_stream));
  TP_CUDA(cudaStreamWaitEvent(a, g_fork_ev, 0));
  g_aux_live = true;
  g_cur = 1;
}

void aux_return() { g_cur = 0; }

void aux_record(int slot) {
  TP_REQUIRE(slot >= 0 && slot < 64, "event slot must be in [0, 64)");
  if (!g_slot_made[slot]) {
    TP_CUDA(cudaEventCreateWithFlags(&g_slot_ev[slot], cudaEventDisableTiming));
    g_slot_made[slot] = true;
  }
  TP_CUDA(cudaEventRecord(g_slot_ev[slot], aux_stream()));
}

void main_wait(int slot) {
  TP_REQUIRE(slot >= 0 && slot < 64 && g_slot_made[slot], "event slot %d was never recorded", slot);
  ensure_init();
  TP_CUDA(cudaStreamWaitEvent(g_stream, g_slot_ev[slot], 0));
}

void aux_join() {
  ensure_init();
  if (!g_aux) return;
  TP_CUDA(cudaEventRecord(make_event(&g_join_ev), g_aux));
  TP_CUDA(cudaStreamWaitEvent(g_stream, g_join_ev, 0));
  g_aux_live = false;
}

int64_t prod(const int64_t* s, int n) {
  int64_t r = 1;
  for (int i = 0; i < n; ++i) r *= s[i];
  return r;
}

Tensor& get(int64_t id) {
  auto it = g_tensors.find(id);
  if (it == g_tensors.end()) fail(TP_ERR_ARG, "Unknown tensor id: %lld.", (long long)id);
  return it->second;
}

int64_t put(const Tensor& t) {
  int64_t id = g_next_id++;
  g_tensors.emplace(id, t);
  g_allocated += (int64_t)t.bytes;
  return id;
}

Tensor make(const int64_t* shape, int ndim, int dtype, int phys) {
  TP_REQUIRE(ndim >= 0 && ndim <= TP_MAX_DIMS, "tensor rank %d exceeds %d", ndim, TP_MAX_DIMS);
  TP_REQUIRE(dtype >= TP_FLOAT32 && dtype <= TP_BOOL, "Unsupported dtype code: %d.", dtype);
  Tensor t;
  t.ndim = ndim;
  t.dtype = dtype;
  t.phys = phys;
  for (int i = 0; i < ndim; ++i) {
    TP_REQUIRE(shape[i] >= 0, "negative dimension %lld", (long long)shape[i]);
    t.shape[i] = shape[i];
  }
  t.numel = prod(shape, ndim);
  t.bytes = (size_t)(t.numel > 0 ? t.numel : 1) * 4;
  t.ptr = dalloc(t.bytes);
  return t;
}

Tensor make_like_shape(const std::vector<int64_t>& shape, int dtype, int phys) {
  return make(shape.data(), (int)shape.size(), dtype, phys);
}

std::vector<int64_t> shape_of(const Tensor& t) { return std::vector<int64_t>(t.shape, t.shape + t.ndim); }

void fill_handle(const Tensor& t, int64_t id, tp_handle* out) {
  if (!out) return;
  out->id = id;
  out->ndim = t.ndim;
  out->dtype = t.dtype;
  for (int i = 0; i < TP_MAX_DIMS; ++i) out->shape[i] = i < t.ndim ? t.shape[i] : 0;
}

int64_t emit(const Tensor& t, tp_handle* out) {
  int64_t id = put(t);
  fill_handle(t, id, out);
  return id;
}

// rows[i] of a [R][row] tensor -> out[i]: one CTA per output row, 16-byte
// accesses when the row length allows it
__global__ void k_gather_rows(const float* __restrict__ src, const int64_t* __restrict__ rows, int64_t n,
                              int64_t row, float* __restrict__ out) {
  ::tp::pdl_enter();
  for (int64_t i = blockIdx.x; i < n; i += gridDim.x) {
    const float* s = src + rows[i] * row;
    float* d = out + i * row;
    if ((row & 3) == 0) {
      const float4* s4 = reinterpret_cast<const float4*>(s);
      float4* d4 = reinterpret_cast<float4*>(d);
      for (int64_t k = threadIdx.x; k < (row >> 2); k += blockDim.x) d4[k] = s4[k];
    } else {
      for (int64_t k = threadIdx.x; k < row; k += blockDim.x) d[k] = s[k];
    }
  }
}

// int64 element <-> the f32 value the runtime stores for an integer dtype
// (truncation toward zero on the way out, as toList decodes, device.ts:38-54)
__global__ void k_f32_to_i64(const float* in, long long* out, int64_t n) {
  ::tp::pdl_enter();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (long long)truncf(in[i]);
}

__global__ void k_i64_to_f32(const long long* in, float* out, int64_t n) {
  ::tp::pdl_enter();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (float)in[i];
}

__global__ void k_i32_to_f32(const int32_t* in, float* out, int64_t n) {
  ::tp::pdl_enter();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (float)in[i];
}

}  // namespace tp

using namespace tp;

extern "C" {

TP_API const char* tp_last_error(void) { return g_err.c_str(); }

TP_API int tp_init(int dev) {
  return guard([&] {
    if (g_device < 0 && dev >= 0) TP_CUDA(cudaSetDevice(dev));
    ensure_init();
  });
}

TP_API int tp_is_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n > 0 ? 1 : 0;
}

TP_API int tp_device_count(int* out) {
  return guard([&] {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    *out = n;
  });
}

TP_API int tp_synchronize(void) {
  return guard([&] {
    ensure_init();
    TP_CUDA(cudaStreamSynchronize(g_stream));
    if (g_aux) TP_CUDA(cudaStreamSynchronize(g_aux));
    // A tensor-core kernel whose bounded wait ran out skipped its output: the
    // results queued so far are not to be trusted, so the caller hears of it.
    const int st = tc_status(true);
    if (st) fail(TP_ERR_TIMEOUT, "a device-side wait gave up (code %d): the results of the work synchronised are "
                                 "incomplete", st);
  });
}

TP_API int tp_aux_fork(void) { return guard([&] { aux_fork(); }); }
TP_API int tp_aux_return(void) { return guard([&] { aux_return(); }); }
TP_API int tp_aux_record(int slot) { return guard([&] { aux_record(slot); }); }
TP_API int tp_main_wait(int slot) { return guard([&] { main_wait(slot); }); }
TP_API int tp_aux_join(void) { return guard([&] { aux_join(); }); }
TP_API int tp_side_fork(void) { return guard([&] { side_fork(); }); }
TP_API int tp_side_return(void) { return guard([&] { side_return(); }); }
TP_API int tp_side_join(void) { return guard([&] { side_join(); }); }

TP_API int tp_get_stream(void** out) { return guard([&] { *out = (void*)stream(); }); }

TP_API int tp_memory_allocated(int64_t* out) { return guard([&] { *out = g_allocated; }); }

TP_API int tp_memory_reserved(int64_t* out) {
  return guard([&] {
    cudaMemPool_t pool;
    TP_CUDA(cudaDeviceGetDefaultMemPool(&pool, device()));
    uint64_t v = 0;
    TP_CUDA(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &v));
    *out = (int64_t)v;
  });
}

TP_API int tp_device_name(char* buf, int len) {
  return guard([&] {
    cudaDeviceProp prop;
    TP_CUDA(cudaGetDeviceProperties(&prop, device()));
    snprintf(buf, (size_t)len, "%s", prop.name);
  });
}

TP_API int tp_kernel_launches(int64_t* out) { return guard([&] { *out = g_launches.load(); }); }

TP_API int tp_set_pdl(int on) {
  return guard([&] {
    TP_REQUIRE(on == 0 || on == 1, "tp_set_pdl: 0 (plain stream order) or 1 (programmatic dependent launch)");
    g_pdl = on;
  });
}

TP_API int tp_tensor_from_data(const float* host, const int64_t* shape, int ndim, int dtype, tp_handle* out) {
  return guard([&] {
    Tensor t = make(shape, ndim, dtype);
    if (t.numel > 0) TP_CUDA(cudaMemcpyAsync(t.ptr, host, (size_t)t.numel * 4, cudaMemcpyHostToDevice, stream()));
    emit(t, out);
  });
}

TP_API int tp_to_host(int64_t id, float* dst, int64_t numel) {
  return guard([&] {
    Tensor& t = get(id);
    TP_REQUIRE(numel == t.numel, "toList: buffer holds %lld values, tensor has %lld", (long long)numel,
               (long long)t.numel);
    if (t.numel == 0) return;
    if (t.phys == PHYS_I32) {
      float* tmp = (float*)dalloc((size_t)t.numel * 4);
      k_i32_to_f32<<<grid_for(t.numel, 256), 256, 0, stream()>>>(t.i(), tmp, t.numel);
      g_launches++;
      TP_LAUNCH_CHECK();
      TP_CUDA(cudaMemcpyAsync(dst, tmp, (size_t)t.numel * 4, cudaMemcpyDeviceToHost, stream()));
      dfree(tmp);
    } else {
      TP_CUDA(cudaMemcpyAsync(dst, t.ptr, (size_t)t.numel * 4, cudaMemcpyDeviceToHost, stream()));
    }
    TP_CUDA(cudaStreamSynchronize(stream()));
  });
}

// ---- batches of a device-resident dataset ----------------------------------------------

TP_API int tp_gather_rows(int64_t src, const int64_t* rows, int64_t n, tp_handle* out) {
  return guard([&] {
    Tensor& S = get(src);
    TP_REQUIRE(S.ndim >= 1, "gatherRows: the source needs a first dimension");
    TP_REQUIRE(S.phys == PHYS_F32, "gatherRows: index tensors are not supported");
    TP_REQUIRE(n >= 0, "gatherRows: negative row count");
    for (int64_t i = 0; i < n; ++i)
      TP_REQUIRE(rows[i] >= 0 && rows[i] < S.shape[0], "index %lld is out of bounds for dimension 0 with size %lld",
                 (long long)rows[i], (long long)S.shape[0]);
    std::vector<int64_t> shp(S.shape, S.shape + S.ndim);
    shp[0] = n;
    Tensor O = make_like_shape(shp, S.dtype);
    const int64_t row = S.shape[0] > 0 ? S.numel / S.shape[0] : 0;
    if (n > 0 && row > 0) {
      int64_t* drows = (int64_t*)dalloc((size_t)n * sizeof(int64_t));
      TP_CUDA(cudaMemcpyAsync(drows, rows, (size_t)n * sizeof(int64_t), cudaMemcpyHostToDevice, stream()));
      const int64_t cap = (int64_t)sm_count() * 16;
      TP_LAUNCH(k_gather_rows, (unsigned)(n < cap ? n : cap), 256, 0, S.f(), drows, n, row, O.f());
      dfree(drows);
      TP_CUDA(cudaStreamSynchronize(stream()));  // the caller's row list may be released on return
    }
    emit(O, out);
  });
}

// ---- bulk byte I/O (checkpoints) and pinned uploads -----------------------------------

TP_API int tp_to_bytes(int64_t id, void* dst, int64_t nbytes, int format) {
  return guard([&] {
    Tensor& t = get(id);
    TP_REQUIRE(format == 0 || format == 1, "toBytes: format 0 (float32) or 1 (int64)");
    const int64_t esz = format == 0 ? 4 : 8;
    TP_REQUIRE(nbytes == t.numel * esz, "toBytes: buffer holds %lld bytes, tensor needs %lld", (long long)nbytes,
               (long long)(t.numel * esz));
    if (t.numel == 0) return;
    const float* src = t.f();
    float* tmp = nullptr;
    if (t.phys == PHYS_I32) {
      tmp = (float*)dalloc((size_t)t.numel * 4);
      TP_LAUNCH(k_i32_to_f32, grid_for(t.numel, 256), 256, 0, (const int32_t*)t.ptr, tmp, t.numel);
      src = tmp;
    }
    if (format == 0) {
      TP_CUDA(cudaMemcpyAsync(dst, src, (size_t)nbytes, cudaMemcpyDeviceToHost, stream()));
    } else {
      long long* wide = (long long*)dalloc((size_t)nbytes);
      TP_LAUNCH(k_f32_to_i64, grid_for(t.numel, 256), 256, 0, src, wide, t.numel);
      TP_CUDA(cudaMemcpyAsync(dst, wide, (size_t)nbytes, cudaMemcpyDeviceToHost, stream()));
      dfree(wide);
    }
    if (tmp) dfree(tmp);
    TP_CUDA(cudaStreamSynchronize(stream()));
  });
}

TP_API int tp_from_bytes(const void* src, int64_t nbytes, int format, const int64_t* shape, int ndim, int dtype,
                         tp_handle* out) {
  return guard([&] {
    TP_REQUIRE(format == 0 || format == 1, "fromBytes: format 0 (float32) or 1 (int64)");
    Tensor t = make(shape, ndim, dtype);
    const int64_t esz = format == 0 ? 4 : 8;
    if (nbytes != t.numel * esz) {
      dfree(t.ptr);
      fail(TP_ERR_ARG, "fromBytes: %lld bytes for %lld elements of %lld bytes", (long long)nbytes,
           (long long)t.numel, (long long)esz);
    }
    if (t.numel > 0) {
      if (format == 0) {
        TP_CUDA(cudaMemcpyAsync(t.ptr, src, (size_t)nbytes, cudaMemcpyHostToDevice, stream()));
      } else {
        long long* wide = (long long*)dalloc((size_t)nbytes);
        TP_CUDA(cudaMemcpyAsync(wide, src, (size_t)nbytes, cudaMemcpyHostToDevice, stream()));
        TP_LAUNCH(k_i64_to_f32, grid_for(t.numel, 256), 256, 0, (const long long*)wide, t.f(), t.numel);
        dfree(wide);
      }
      // the caller's buffer may be pageable and released on return
      TP_CUDA(cudaStreamSynchronize(stream()));
    }
    emit(t, out);
  });
}

TP_API int tp_host_alloc(int64_t bytes, void** out) {
  return guard([&] {
    TP_REQUIRE(bytes >= 0, "negative allocation size");
    ensure_init();
    void* p = nullptr;
    cudaError_t e = cudaHostAlloc(&p, (size_t)(bytes > 0 ? bytes : 16), cudaHostAllocPortable);
    if (e != cudaSuccess) {
      cudaGetLastError();
      fail(TP_ERR_OOM, "pinned host allocation of %lld bytes failed: %s", (long long)bytes, cudaGetErrorString(e));
    }
    *out = p;
  });
}

TP_API int tp_host_free(void* p) {
  return guard([&] {
    if (p) TP_CUDA(cudaFreeHost(p));
  });
}

// Uploads from pinned host memory run on their own copy stream, so the copy of
// the next batch overlaps the kernels of the current one; the destination is
// allocated in the copy stream's order (the pool makes cross-stream reuse safe)
// and the library streams wait for the copy's event before any later kernel.
// Each upload gets a ticket: tp_ticket_wait(ticket) returns once that copy has
// finished, after which the host buffer may be reused.
static cudaStream_t g_copy = nullptr;
constexpr int TICKETS = 256;
static cudaEvent_t g_ticket_ev[TICKETS];
static bool g_ticket_made[TICKETS];
static int64_t g_next_ticket = 1;

TP_API int tp_tensor_from_host_async(const void* host, const int64_t* shape, int ndim, int dtype, int defer,
                                     tp_handle* out, int64_t* ticket) {
  return guard([&] {
    ensure_init();
    if (!g_copy) TP_CUDA(cudaStreamCreateWithFlags(&g_copy, cudaStreamNonBlocking));
    cudaPointerAttributes attr;
    TP_CUDA(cudaPointerGetAttributes(&attr, host));
    TP_REQUIRE(attr.type == cudaMemoryTypeHost, "tensorFromHostAsync: the source must be pinned host memory "
                                                "(tp_host_alloc)");
    TP_REQUIRE(ndim >= 0 && ndim <= TP_MAX_DIMS, "tensor rank %d exceeds %d", ndim, TP_MAX_DIMS);
    TP_REQUIRE(dtype >= TP_FLOAT32 && dtype <= TP_BOOL, "Unsupported dtype code: %d.", dtype);
    Tensor t;
    t.ndim = ndim;
    t.dtype = dtype;
    t.phys = PHYS_F32;
    for (int i = 0; i < ndim; ++i) {
      TP_REQUIRE(shape[i] >= 0, "negative dimension %lld", (long long)shape[i]);
      t.shape[i] = shape[i];
    }
    t.numel = prod(shape, ndim);
    t.bytes = (size_t)(t.numel > 0 ? t.numel : 1) * 4;
    cudaError_t e = cudaMallocAsync(&t.ptr, t.bytes, g_copy);
    if (e != cudaSuccess) {
      cudaGetLastError();
      fail(TP_ERR_OOM, "device allocation of %zu bytes failed: %s", t.bytes, cudaGetErrorString(e));
    }
    if (t.numel > 0) TP_CUDA(cudaMemcpyAsync(t.ptr, host, (size_t)t.numel * 4, cudaMemcpyHostToDevice, g_copy));
    const int64_t tk = g_next_ticket++;
    const int slot = (int)(tk % TICKETS);
    if (!g_ticket_made[slot]) {
      TP_CUDA(cudaEventCreateWithFlags(&g_ticket_ev[slot], cudaEventDisableTiming));
      g_ticket_made[slot] = true;
    }
    TP_CUDA(cudaEventRecord(g_ticket_ev[slot], g_copy));
    if (!defer) {
      TP_CUDA(cudaStreamWaitEvent(g_stream, g_ticket_ev[slot], 0));
      if (g_aux) TP_CUDA(cudaStreamWaitEvent(g_aux, g_ticket_ev[slot], 0));
    }
    emit(t, out);
    *ticket = tk;
  });
}

TP_API int tp_ticket_use(int64_t ticket) {
  return guard([&] {
    TP_REQUIRE(ticket > 0 && ticket < g_next_ticket, "unknown upload ticket %lld", (long long)ticket);
    cudaEvent_t ev = g_ticket_ev[ticket % TICKETS];  // a later copy's event in a reused slot: a later wait
    TP_CUDA(cudaStreamWaitEvent(g_stream, ev, 0));
    if (g_aux) TP_CUDA(cudaStreamWaitEvent(g_aux, ev, 0));
  });
}

TP_API int tp_ticket_wait(int64_t ticket) {
  return guard([&] {
    TP_REQUIRE(ticket > 0 && ticket < g_next_ticket, "unknown upload ticket %lld", (long long)ticket);
    // A slot reused by a later upload holds that later copy's event, which
    // completes after this one (one copy stream, in order): still a safe wait.
    TP_CUDA(cudaEventSynchronize(g_ticket_ev[ticket % TICKETS]));
  });
}

TP_API int tp_destroy(int64_t id) {
  return guard([&] {
    auto it = g_tensors.find(id);
    if (it == g_tensors.end()) return;  // destroying twice is a no-op (device.ts:466-468)
    g_allocated -= (int64_t)it->second.bytes;
    dfree(it->second.ptr);
    g_tensors.erase(it);
  });
}

TP_API int tp_meta(int64_t id, tp_handle* out) {
  return guard([&] { fill_handle(get(id), id, out); });
}

TP_API int tp_device_ptr(int64_t id, void** out) { return guard([&] { *out = get(id).ptr; }); }

TP_API int tp_alloc(int64_t bytes, void** out) {
  return guard([&] {
    TP_REQUIRE(bytes >= 0, "negative allocation size");
    *out = dalloc((size_t)bytes);
  });
}

TP_API int tp_free(void* p) { return guard([&] { dfree(p); }); }

TP_API int tp_memcpy_h2d(void* dst, const void* src, int64_t bytes) {
  return guard([&] {
    if (bytes > 0) TP_CUDA(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyHostToDevice, stream()));
  });
}

TP_API int tp_memcpy_d2h(void* dst, const void* src, int64_t bytes) {
  return guard([&] {
    if (bytes > 0) TP_CUDA(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDeviceToHost, stream()));
    TP_CUDA(cudaStreamSynchronize(stream()));
  });
}

TP_API int tp_memcpy_d2d(void* dst, const void* src, int64_t bytes) {
  return guard([&] {
    if (bytes > 0) TP_CUDA(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDeviceToDevice, stream()));
  });
}

TP_API int tp_memset(void* dst, int value, int64_t bytes) {
  return guard([&] {
    if (bytes > 0) TP_CUDA(cudaMemsetAsync(dst, value, (size_t)bytes, stream()));
  });
}

}  // extern "C"
