// Host side of TMA: tiled fp32 tensor maps with 128-byte swizzle.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace tp {

// Encode a tiled fp32 tensor map over `base`: dims[0] is the contiguous
// dimension, strides[i] (bytes) is the stride of dims[i + 1], box[i] is the
// tile extent.  Out-of-range boxes read zeros.  The shared-memory image is
// 128-byte swizzled (box[0] must be 32 floats): 16-byte chunks permuted over
// 8-row periods for a K-major operand tile, 32-byte chunks over 4-row periods
// (atom32) for an MN-major one, the only MN-major form the tensor core reads
// for tf32.  Fails with TP_ERR_ARG when the address or a stride breaks the
// TMA alignment rules.
void make_map_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                  const uint32_t* box, bool atom32 = false);

// True if TMA can address `p` with these byte strides (16-byte aligned).
bool tma_aligned(const void* p, const uint64_t* strides, int n);

// lo[i] = x[i] - tf32(x[i]) with tf32 = x with its 13 low mantissa bits
// cleared (the 3xTF32 GEMM's split of a B operand), into `lo` (n floats, both
// 16-byte aligned); launched on the library stream.
void tf32_lo_plane(const float* x, float* lo, int64_t n);

}  // namespace tp
