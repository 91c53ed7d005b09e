// requant.cuh -- the reference's fused-output requantization on the GPU: v / 2^shift rounded half to even,
// the model its own test checks the NPU output stage against, bit for bit (ork-driver
// examples/test_mm_i8_out8.c:24-33: floor shift, then +1 when the remainder is above half or exactly half
// with an odd quotient). Exact for every int64 v; shift 0 leaves v unchanged.
#pragma once
#include <stdint.h>

namespace orkb {

__device__ __forceinline__ int64_t requant_rne(int64_t v, int shift) {
  if (shift <= 0) return v;
  const int64_t q = v >> shift;  // arithmetic: floor
  const int64_t rem = v - (q << shift), half = (int64_t)1 << (shift - 1);
  return (rem > half || (rem == half && (q & 1))) ? q + 1 : q;
}

}  // namespace orkb
