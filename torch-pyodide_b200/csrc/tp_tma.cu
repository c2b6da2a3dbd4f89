// Tensor-map encoding for the TMA-fed GEMM.  The driver entry point is looked
// up through the runtime (cudaGetDriverEntryPoint), so the library does not
// link libcuda and still loads on machines without a driver.
#include <cuda.h>
#include <cuda_runtime.h>

#include "tp_core.h"
#include "tp_launch.h"
#include "tp_tma.h"

namespace tp {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    TP_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TP_REQUIRE(q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

bool tma_aligned(const void* p, const uint64_t* strides, int n) {
  if (((uintptr_t)p & 15) != 0) return false;
  for (int i = 0; i < n; ++i)
    if ((strides[i] & 15) != 0 || strides[i] >= ((uint64_t)1 << 40)) return false;
  return true;
}

void make_map_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                  const uint32_t* box, bool atom32) {
  TP_REQUIRE(rank >= 2 && rank <= 5, "tensor map rank %d", rank);
  TP_REQUIRE(tma_aligned(base, strides, rank - 1), "tensor map: base or stride not 16-byte aligned");
  TP_REQUIRE(box[0] == 32, "tensor map: the inner box must be 32 floats (one 128-byte swizzle row)");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    TP_REQUIRE(dims[i] >= 1 && dims[i] < ((uint64_t)1 << 32), "tensor map: dimension %d out of range", i);
    TP_REQUIRE(box[i] >= 1 && box[i] <= 256, "tensor map: box extent %d out of range", i);
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) s[i] = strides[i];
  CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<void*>(base), d, s, b,
                           e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TP_REQUIRE(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d)", (int)r);
}

__global__ void k_tf32_lo(const float4* __restrict__ x, float4* __restrict__ lo, int64_t n4) {
  ::tp::pdl_enter();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = x[i];
    lo[i] = make_float4(v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u),
                        v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u),
                        v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u),
                        v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u));
  }
}

__global__ void k_tf32_lo_tail(const float* __restrict__ x, float* __restrict__ lo, int64_t i0, int64_t n) {
  ::tp::pdl_enter();
  const int64_t i = i0 + threadIdx.x;
  if (i < n) lo[i] = x[i] - __uint_as_float(__float_as_uint(x[i]) & 0xFFFFE000u);
}

void tf32_lo_plane(const float* x, float* lo, int64_t n) {
  TP_REQUIRE((((uintptr_t)x | (uintptr_t)lo) & 15) == 0, "tf32 split: buffers must be 16-byte aligned");
  const int64_t n4 = n / 4;
  if (n4 > 0)
    TP_LAUNCH(k_tf32_lo, grid_for(n4, 256), 256, 0, reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(lo),
              n4);
  if (n > n4 * 4) TP_LAUNCH(k_tf32_lo_tail, 1, 32, 0, x, lo, n4 * 4, n);
}

}  // namespace tp
