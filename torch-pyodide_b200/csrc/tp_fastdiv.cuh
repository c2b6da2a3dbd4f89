// Unsigned division by a runtime constant d for n < 2^31: with l = ceil(log2 d)
// and m = floor(2^32 (2^l - d) / d) + 1, n / d = (umulhi(n, m) + n) >> l
// (Granlund & Montgomery, "Division by invariant integers using
// multiplication", 1994; the sum stays below 2^32 because n < 2^31).
#pragma once

#include <stdint.h>

namespace tp {

struct FastDiv {
  uint32_t d, m, l;
  __device__ __forceinline__ uint32_t div(uint32_t n) const { return (__umulhi(n, m) + n) >> l; }
  __device__ __forceinline__ uint32_t mod(uint32_t n) const { return n - div(n) * d; }
};

inline FastDiv fast_div(uint32_t d) {
  uint32_t l = 0;
  while (((uint64_t)1 << l) < d) ++l;
  const uint64_t m = ((uint64_t)1 << 32) * (((uint64_t)1 << l) - d) / d + 1;
  return {d, (uint32_t)m, l};
}

}  // namespace tp
